"""Isolated kernel sweep through the C ABI operator entry
points, timed with CUDA events on the launch stream.

  python -m minimind_orangepi_b200.sweep [--case projection|attention|lm_head|all]
      [--batch B ...] [--ctx C ...] [--hd D ...] [--shape NxK ...] [--iters N] [--json]

(a) projections [N x K] in {512x512, 128x512, 1408x512, 512x1408, 768x768,
    192x768, 2048x768, 768x2048, 6400x768} at batch 1, 8, 64, 256 (weights
    N(0, 0.02) fp16, activations N(0, 1));
(b) fused GQA decode attention, 8 q / 2 kv heads, head_dim 64 and 96, context
    1, 128, 1024, 8192, 32768 at batch 1, 64, 256 (paged fp16 cache, 64-position
    pages scattered over the pool);
(c) lm_head 6400 x 768 + argmax.
Each line reports the kernel's algorithmic bytes (and FLOPs) per launch, the
mean launch time and the fraction of the measured HBM / tensor peaks
(MEASURED_PEAKS.json). Launches run back to back between two CUDA events
after a warm-up; projection weights rotate over enough copies (> 3x L2) that
every launch streams them from HBM; the attention cases that matter exceed L2
on their own.
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
from pathlib import Path

import numpy as np

from ._lib import check, lib

ROOT = Path(__file__).resolve().parents[1]
L2_BYTES = 126 * 2**20
PROJ_SHAPES = [(512, 512), (128, 512), (1408, 512), (512, 1408), (768, 768), (192, 768), (2048, 768), (768, 2048),
               (6400, 768)]


def _peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    d = json.loads(p.read_text()) if p.exists() else {}
    return d.get("hbm_gbs", 6650.0), d.get("bf16_tflops", 1590.0), ("measured" if d else "fallback")


class Timer:
    """Back-to-back launches between two CUDA events on one stream, after a
    warm-up that brings the clocks up. The timed launches are captured once
    into a CUDA graph and replayed, so the host-side cost of each C-ABI call
    (argument checks, tensor-map encoding) does not leave the GPU idle
    between launches; if capture fails the launches are issued eagerly.
    Callers rotate over enough copies of their inputs that each launch reads
    from HBM, not L2."""

    def __init__(self, torch, iters: int):
        self.torch = torch
        self.iters = iters
        self.stream = torch.cuda.Stream()
        self.mode = "graph"

    def run(self, fn) -> float:
        """Mean ms per launch of fn(stream_ptr, i) for i in range(iters)."""
        t = self.torch
        sp = self.stream.cuda_stream
        with t.cuda.stream(self.stream):
            for i in range(max(3, self.iters // 4)):
                fn(sp, i)
        self.stream.synchronize()
        graph = None
        try:
            graph = t.cuda.CUDAGraph()
            with t.cuda.graph(graph, stream=self.stream):
                for i in range(self.iters):
                    fn(sp, i)
        except Exception:  # noqa: BLE001 - fall back to eager launches
            graph = None
            self.mode = "eager"
            t.cuda.synchronize()
        with t.cuda.stream(self.stream):
            if graph is not None:
                graph.replay()  # warm replay
            t.cuda._sleep(2_000_000)  # let the host run ahead of the device
            e0, e1 = t.cuda.Event(enable_timing=True), t.cuda.Event(enable_timing=True)
            e0.record(self.stream)
            if graph is not None:
                graph.replay()
            else:
                for i in range(self.iters):
                    fn(sp, i)
            e1.record(self.stream)
            e1.synchronize()
        return e0.elapsed_time(e1) / self.iters


def copies_for(bytes_per_set: int) -> int:
    """Input sets needed so consecutive launches never find their data in L2."""
    return max(1, min(64, (3 * L2_BYTES) // max(bytes_per_set, 1) + 1))


def dev(t):
    return C.c_void_p(t.data_ptr())


def sweep_projection(torch, timer, batches, shapes):
    hbm, tc, src = _peaks()
    out = []
    for n, k in shapes:
        g = torch.Generator(device="cpu").manual_seed(n + k)
        ncp = copies_for(2 * n * k)
        w0 = (torch.randn(n, k, generator=g) * 0.02).half().cuda()
        ws = [w0.clone() for _ in range(ncp)]
        for b in batches:
            x = torch.randn(b, k, generator=g).cuda()
            xa = x if b <= 4 else x.half().contiguous()
            y = torch.empty(b, n, device="cuda")
            ms = timer.run(lambda s, i: check(lib().mmc_op_projection(b, n, k, dev(ws[i % ncp]), dev(xa), dev(y),
                                                                      C.c_void_p(s))))
            bytes_ = 2 * n * k + xa.element_size() * b * k + 4 * b * n
            flops = 2 * b * n * k
            gbs, tfl = bytes_ / ms / 1e6, flops / ms / 1e9
            out.append({"case": "projection", "n": n, "k": k, "batch": b, "path": "gemv" if b <= 4 else "tcgen05",
                        "ms": ms, "bytes": bytes_, "GB/s": gbs, "hbm_frac": gbs / hbm, "TFLOP/s": tfl,
                        "tensor_frac": tfl / tc, "peaks": src})
    return out


def build_paged_cache(torch, batch, ctx, hd, nkv, layers=1, seed=0):
    """Random paged cache with pages scattered (shuffled) over the pool."""
    rng = np.random.default_rng(seed)
    pages_per = (ctx + 63) // 64
    n_pages = batch * pages_per + 1
    perm = rng.permutation(n_pages - 1) + 1
    bt = perm[: batch * pages_per].reshape(batch, pages_per).astype(np.int32)
    pool = torch.empty(n_pages * layers * 2 * nkv * 64 * hd, dtype=torch.half, device="cuda")
    pool.normal_(0, 1)
    return pool, torch.from_numpy(bt).cuda(), pages_per


def sweep_attention(torch, timer, batches, ctxs, hds, nq=8, nkv=2):
    hbm, _, src = _peaks()
    out = []
    for hd in hds:
        for b in batches:
            for ctx in ctxs:
                kv_bytes = b * ctx * nkv * hd * 2 * 2
                if kv_bytes > 40 * 2**30:
                    continue
                pool, bt, max_pages = build_paged_cache(torch, b, ctx, hd, nkv)
                pos = torch.full((b,), ctx - 1, dtype=torch.int32, device="cuda")
                slots = torch.arange(b, dtype=torch.int32, device="cuda")
                qkv = torch.randn(b, (nq + 2 * nkv) * hd, device="cuda")
                qn = torch.ones(hd, device="cuda")
                kn = torch.ones(hd, device="cuda")
                half = hd // 2
                cos = torch.ones(ctx * half, device="cuda")
                sin = torch.zeros(ctx * half, device="cuda")
                o = torch.empty(b, nq * hd, device="cuda")
                ws_n = C.c_size_t()
                check(lib().mmc_op_attention_workspace_size(b, nq, nkv, hd, ctx, C.byref(ws_n)))
                ws = torch.empty(ws_n.value, dtype=torch.uint8, device="cuda")

                def fn(s, i):
                    check(lib().mmc_op_attention(b, nq, nkv, hd, 0, 1, dev(qkv), dev(qn), dev(kn), dev(cos), dev(sin),
                                                 ctx, 1e-5, dev(pool), dev(bt), max_pages, dev(pos), dev(slots), ctx,
                                                 dev(o), dev(ws), ws_n.value, C.c_void_p(s)))
                ms = timer.run(fn)
                bytes_ = kv_bytes + b * (nq + 2 * nkv) * hd * 4 + b * nq * hd * 4
                gbs = bytes_ / ms / 1e6
                out.append({"case": "attention", "hd": hd, "batch": b, "ctx": ctx, "ms": ms, "bytes": bytes_,
                            "GB/s": gbs, "hbm_frac": gbs / hbm, "peaks": src})
                del pool
    return out


def sweep_lm_head(torch, timer, batches, n=6400, k=768):
    hbm, tc, src = _peaks()
    out = []
    ncp = copies_for(2 * n * k)
    w0 = (torch.randn(n, k) * 0.02).half().cuda()
    wl = [w0.clone() for _ in range(ncp)]
    for b in batches:
        x = torch.randn(b, k, device="cuda")
        xa = x if b <= 4 else x.half().contiguous()
        nxt = torch.empty(b, dtype=torch.int32, device="cuda")
        ws_n = C.c_size_t()
        check(lib().mmc_op_lm_head_argmax_workspace_size(b, n, k, C.byref(ws_n)))
        ws = torch.empty(ws_n.value, dtype=torch.uint8, device="cuda")
        ms = timer.run(lambda s, i: check(lib().mmc_op_lm_head_argmax(b, n, k, dev(wl[i % ncp]), dev(xa), None,
                                                                      dev(nxt), dev(ws), ws_n.value, C.c_void_p(s))))
        bytes_ = 2 * n * k + xa.element_size() * b * k + 4 * b
        gbs = bytes_ / ms / 1e6
        out.append({"case": "lm_head_argmax", "n": n, "k": k, "batch": b, "ms": ms, "bytes": bytes_, "GB/s": gbs,
                    "hbm_frac": gbs / hbm, "TFLOP/s": 2 * b * n * k / ms / 1e9, "peaks": src})
    return out


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--case", default="all", choices=["projection", "attention", "lm_head", "all"])
    ap.add_argument("--batch", type=int, nargs="*")
    ap.add_argument("--ctx", type=int, nargs="*")
    ap.add_argument("--hd", type=int, nargs="*")
    ap.add_argument("--shape", type=str, nargs="*", help="projection shapes as NxK (default: the config-5 list)")
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--json", action="store_true")
    args = ap.parse_args(argv)
    import torch
    timer = Timer(torch, args.iters)
    rows = []
    if args.case in ("projection", "all"):
        shapes = [tuple(int(v) for v in sh.split("x")) for sh in args.shape] if args.shape else PROJ_SHAPES
        rows += sweep_projection(torch, timer, args.batch or [1, 8, 64, 256], shapes)
    if args.case in ("attention", "all"):
        rows += sweep_attention(torch, timer, args.batch or [1, 64, 256], args.ctx or [1, 128, 1024, 8192, 32768],
                                args.hd or [64, 96])
    if args.case in ("lm_head", "all"):
        rows += sweep_lm_head(torch, timer, args.batch or [1, 8, 64, 256])
    for r in rows:
        if args.json:
            print(json.dumps(r), flush=True)
            continue
        keys = [k for k in ("n", "k", "hd", "batch", "ctx", "path") if k in r]
        desc = " ".join(f"{k}={r[k]}" for k in keys)
        extra = f" {r['TFLOP/s']:.1f} TFLOP/s" if "TFLOP/s" in r else ""
        print(f"{r['case']:<15} {desc:<40} {r['ms'] * 1000:9.2f} us {r['GB/s']:8.1f} GB/s "
              f"({100 * r['hbm_frac']:5.1f}% hbm){extra}", flush=True)
    if not args.json:
        print(f"# timed launches: {timer.mode} (CUDA events on the launch stream)", flush=True)


if __name__ == "__main__":
    main()
