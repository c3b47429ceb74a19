#!/usr/bin/env python3
"""Decode throughput benchmark (BASELINE.json metric: decode tokens/sec and
fraction of the bytes-moved roofline).

Default workload = BASELINE config 4: batched greedy decode on MiniMind2
(hidden 768, 16 layers, 8 q / 2 kv heads, head_dim 96, intermediate 2048,
vocab 6400; random-init N(0, 0.02) weights exported to the runtime format),
256 independent sequences with prompt lengths U[16, 2048] and ids U[3, 6400),
sharded over the GPUs (strong scaling, no collective on the data path).
The prompts are fed untimed (token-by-token batched decode); then W warm-up and
K timed decode steps run as replays of the captured CUDA graph on each GPU.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--workload cfg4|cfg3|cfg2|cfg1] [--impl ours|reference]

Under torchrun each rank drives LOCAL_RANK's GPU; timings are device events,
max over ranks. Rank 0 prints one JSON line.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

from minimind_orangepi_b200.sharding import plan_shards, shard_imbalance  # noqa: E402
from minimind_orangepi_b200.synthetic import SHAPES, write_runtime_model  # noqa: E402

MODEL_CACHE = Path(os.environ.get("MMC_BENCH_MODELS", "/tmp/mmc_bench_models"))
PEAKS = ROOT / "MEASURED_PEAKS.json"

WORKLOADS = {
    "cfg4": dict(shape="minimind2", n_seqs=256, prompt=(16, 2048), steps=256,
                 desc="BASELINE config 4: batched decode, MiniMind2 (768 hidden, 16 layers, 8q/2kv, hd 96, "
                      "inter 2048, vocab 6400), 256 sequences, prompt lengths U[16,2048], 256 greedy steps, "
                      "paged fp16 KV"),
    "cfg4-shard8": dict(shape="minimind2", n_seqs=32, prompt=(16, 2048), steps=64,
                        desc="one GPU's share of BASELINE config 4 on 8 GPUs (32 sequences; profiling case)"),
    "cfg4-shard2": dict(shape="minimind2", n_seqs=128, prompt=(16, 2048), steps=64,
                        desc="one GPU's share of BASELINE config 4 on 2 GPUs (128 sequences; profiling case)"),
    "cfg4-shard4": dict(shape="minimind2", n_seqs=64, prompt=(16, 2048), steps=64,
                        desc="one GPU's share of BASELINE config 4 on 4 GPUs (64 sequences; profiling case)"),
    "probe": dict(shape="minimind2", n_seqs=96, prompt=(16, 512), steps=8,
                  desc="profiling case (not a BASELINE config): MiniMind2, 96 sequences, prompt lengths U[16,512]"),
    "cfg3": dict(shape="minimind2", n_seqs=1, prompt=(128, 128), steps=1024,
                 desc="BASELINE config 3: MiniMind2 batch 1, 128-token prompt, 1024 greedy steps"),
    "cfg2": dict(shape="minimind2-small", n_seqs=1, prompt=(512, 512), steps=512,
                 desc="BASELINE config 2: MiniMind2-small batch 1, 512-token prompt, 512 greedy steps"),
    "cfg1": dict(shape="minimind2-small", n_seqs=1, prompt=(5, 5), steps=15,
                 desc="BASELINE config 1: MiniMind2-small batch 1, 5-token prompt, 16 new tokens (15 decode steps)"),
}


# measured DRAM traffic / algorithmic bytes of attention_kernel (ncu, B=128, ctx 1024, hd 96):
# (100.95 MB read + 7.51 MB written) / (100.66 MB K/V + 0.39 MB q and output)
ATTN_TRAFFIC_RATIO = (100.95 + 7.51) / (100.66 + 0.39)


def workload_prompts(w: dict, seed: int = 0):
    rng = np.random.default_rng(seed)
    lo, hi = w["prompt"]
    lens = [int(x) for x in rng.integers(lo, hi + 1, size=w["n_seqs"])]
    vocab = SHAPES[w["shape"]].vocab_size
    prompts = [[int(t) for t in rng.integers(3, vocab, size=n)] for n in lens]
    return lens, prompts


def model_path(w: dict) -> Path:
    return MODEL_CACHE / f"{w['shape']}-seed1"


def kv_bytes_per_position(shape) -> int:
    return shape.num_hidden_layers * 2 * shape.num_key_value_heads * shape.head_dim * 2


def weight_bytes(shape) -> int:
    s = shape
    q, kv = s.num_attention_heads * s.head_dim, s.num_key_value_heads * s.head_dim
    per_layer = (q + 2 * kv) * s.hidden_size + s.hidden_size * q + 2 * s.intermediate_size * s.hidden_size + \
        s.hidden_size * s.intermediate_size
    return 2 * (s.num_hidden_layers * per_layer + s.vocab_size * s.hidden_size)


# ------------------------------------------------------------------ clocks

class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu_index = gpu_index
        self.proc = None
        self.lines: list[str] = []

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                                          "-i", str(self.gpu_index), "-lms", "200"], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
            threading.Thread(target=self._read, daemon=True).start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


def physical_gpu(local_rank: int) -> int:
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        ids = [v.strip() for v in vis.split(",") if v.strip()]
        if local_rank < len(ids) and ids[local_rank].isdigit():
            return int(ids[local_rank])
    return local_rank


# ------------------------------------------------------------ CPU baselines

def cpu_reference_sample(w: dict, model_dir: Path, threads: int, steps_per_thread: int | None, seconds: float,
                         lens: list[int]):
    """Time the reference CPU decode (oracle/_ref, else the C restatement) on
    `threads` host threads, each advancing its own sequence (context drawn
    from the workload's prompt lengths, filled with seeded synthetic K/V)."""
    from oracle.oracle import Oracle, ReferenceModel, ref_available

    kind = "reference" if ref_available() else "port"
    if kind == "reference":
        model = ReferenceModel(model_dir, eps=1e-5, theta=1e6)
    else:
        model = Oracle(model_dir, eps=1e-5, theta=1e6)
    states = []
    for t in range(threads):
        st = model.new_state()
        ctx = lens[t % len(lens)]
        if kind == "reference":
            model.fill_context(st, ctx, seed=t)
        else:  # the port has no fill hook: feed a short prompt
            for tok in range(3, 3 + min(ctx, 8)):
                model.forward_token(st, tok, want_logits=False)
        states.append(st)
    # first call builds the reference's static RoPE table: do it before threading
    warm = model.new_state()
    if kind == "reference":
        model.forward_next_token(warm, 5)
    else:
        model.forward_token(warm, 5, want_logits=False)
    counts = [0] * threads
    deadline = [0.0]

    def worker(i):
        st, tok = states[i], 5
        n = 0
        while True:
            if steps_per_thread is not None and n >= steps_per_thread:
                break
            if steps_per_thread is None and time.perf_counter() >= deadline[0]:
                break
            if kind == "reference":
                tok = model.forward_next_token(st, tok)
            else:
                tok, _ = model.forward_token(st, tok, want_logits=False)
            n += 1
        counts[i] = n

    ths = [threading.Thread(target=worker, args=(i,)) for i in range(threads)]
    t0 = time.perf_counter()
    deadline[0] = t0 + seconds
    for th in ths:
        th.start()
    for th in ths:
        th.join()
    dt = time.perf_counter() - t0
    total = sum(counts)
    return {"value": total / dt, "unit": "tokens/s", "cores": threads, "kind": kind,
            "sample": f"{total} single-token decode steps of {w['shape']} over {threads} independent sequences "
                      f"(one per host thread; contexts from the workload's prompt lengths, cached K/V seeded), "
                      f"{dt:.1f} s wall"}


def run_reference_arm(args, w, rank: int) -> None:
    if rank != 0:
        return
    model_dir = write_runtime_model(model_path(w), w["shape"], 1)
    lens, _ = workload_prompts(w)
    threads = max(1, min(os.cpu_count() or 1, w["n_seqs"]))
    # warm-up steps, then exactly K timed steps per thread
    warm = cpu_reference_sample(w, model_dir, threads, max(1, args.warmup // 4), 0, lens)
    del warm
    res = cpu_reference_sample(w, model_dir, threads, args.steps, 0, lens)
    line = {
        "impl": "reference", "metric": METRIC, "value": res["value"], "unit": "tokens/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000.0 * threads / res["value"],
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": w["desc"], "global_batch": w["n_seqs"], "parallelism": "host threads"},
        "cpu_baseline": res,
        "e2e": {"value": res["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


METRIC = "decode tokens/sec"


# ------------------------------------------------------------------ main

def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None)
    ap.add_argument("--warmup", type=int, default=4)
    ap.add_argument("--workload", default="cfg4", choices=sorted(WORKLOADS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--profile-steps", type=int, default=2)
    ap.add_argument("--fill-context", action="store_true",
                    help="fast-forward each sequence to its prompt length with synthetic K/V instead of feeding "
                         "the prompt (untimed part only; used for ncu runs)")
    args = ap.parse_args()
    w = WORKLOADS[args.workload]
    if args.steps is None:
        args.steps = w["steps"]
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        run_reference_arm(args, w, rank)
        return

    import torch
    torch.cuda.set_device(local_rank)
    dist = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=torch.device("cuda", local_rank))

    from minimind_orangepi_b200 import DecodeEngine

    shape = SHAPES[w["shape"]]
    if rank == 0:
        write_runtime_model(model_path(w), w["shape"], 1)
    if dist:
        dist.barrier()
    model_dir = write_runtime_model(model_path(w), w["shape"], 1)

    lens, prompts = workload_prompts(w)
    K, W = args.steps, args.warmup
    E = K  # end-to-end steps through the host-buffer C ABI
    need = [n + W + K + E + 2 * K + 2 for n in lens]  # + K graph steps and K streamed steps
    shards = plan_shards(need, world)
    mine = shards[rank]
    B = len(mine)
    n_pages = sum((need[i] + 63) // 64 for i in mine) + 8
    # max_batch also bounds the rows of one prompt pass (mmc_prefill)
    eng = DecodeEngine(model_dir, device=local_rank, max_seqs=max(B, 1), max_batch=max(B, 1024), n_pages=n_pages)
    seqs = [eng.open_sequence(need[i]) for i in mine]
    my_prompts = [prompts[i] for i in mine]

    # untimed prompt pass
    t0 = time.perf_counter()
    if args.fill_context:
        for j, sq in enumerate(seqs):
            eng.fill_context(sq, len(my_prompts[j]) - 1, seed=mine[j])
        first, _ = eng.step(seqs, [p[-1] for p in my_prompts])
    else:
        first = eng.prompt_pass(seqs, my_prompts)
    prefill_s = time.perf_counter() - t0

    # a dedicated stream: the legacy default stream's handle is NULL, which the
    # C ABI reads as "the context's own stream"
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    sptr = stream.cuda_stream
    eng.graph_build(seqs)
    eng.graph_set_tokens(first)
    sampler = ClockSampler(physical_gpu(local_rank))
    sampler.start()
    eng.graph_run(W, sptr)
    torch.cuda.synchronize()

    # algorithmic bytes of the timed steps (weights once per step, every cached
    # K/V row read, one row appended per sequence and layer)
    pos0 = [eng.position(sq) for sq in seqs]
    kvb = kv_bytes_per_position(shape)
    timed_bytes = K * weight_bytes(shape) + sum(sum(p + i + 1 for i in range(K)) * kvb + K * kvb for p in pos0)

    # ---------------- timed: K graph replays, device events, max over ranks
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    ev0.record(stream)
    eng.graph_run(K, sptr)
    ev1.record(stream)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    dev_ms = ev0.elapsed_time(ev1)
    hist = eng.graph_tokens(K)  # also surfaces any device-side error
    assert hist.shape == (K, B)
    last = hist[-1].copy()

    # ---------------- end to end: the public host-buffer call, H2D + D2H per step
    toks = last.astype(np.int32)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(E):
        toks, _ = eng.step(seqs, toks)
    e2e_s = time.perf_counter() - t0
    # ---------------- streamed: the device loop with each step's tokens read on the host as it lands
    # (mmc_graph_stream_*: what generate_stream and --stream use), host wall clock; beside it, K plain
    # graph replays right before it (device events), so that both see nearly the same context lengths
    eng.graph_set_tokens(toks)
    ev0.record(stream)
    eng.graph_run(K, sptr)
    ev1.record(stream)
    torch.cuda.synchronize()
    graph_near_ms = ev0.elapsed_time(ev1)
    eng.graph_set_tokens(eng.graph_tokens(K)[-1].copy())
    t0 = time.perf_counter()
    for _ in eng.graph_stream(K):
        pass
    stream_s = time.perf_counter() - t0
    clocks = sampler.stop()

    # ---------------- per-kernel attribution (profiled steps, events between kernels)
    prof = {k: [0.0, 0] for k in eng.KERNEL_KINDS}
    attn_bytes = 0.0
    for _ in range(args.profile_steps):
        pos = [eng.position(s) for s in seqs]  # cached before this step
        _, kinds = eng.profile_step(seqs, toks)
        for k, (ms, n) in kinds.items():
            prof[k][0] += ms
            prof[k][1] += n
        # algorithmic bytes of one attention launch (one layer): read every
        # cached K/V row, append one row, read q|k|v, write the output
        hd, nkv, nq = shape.head_dim, shape.num_key_value_heads, shape.num_attention_heads
        attn_bytes += sum((p + 1) * nkv * hd * 2 * 2 for p in pos) + B * nkv * hd * 2 * 2 + \
            B * (nq + 2 * nkv) * hd * 4 + B * nq * hd * 4
    attn_ms = prof["attention"][0] / max(prof["attention"][1], 1)
    attn_bytes_per_launch = attn_bytes / args.profile_steps
    kernels_per_step = eng.kernels_per_step(B)

    # ---------------- reduce over ranks
    persistent = kernels_per_step == 1  # the whole step is one launch (batches of up to 64 rows)
    vals = np.array([dev_ms, e2e_s * 1000.0, attn_ms], np.float64)
    if dist:
        t = torch.tensor(vals, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        vals = t.cpu().numpy()
        dist.barrier()
    dev_ms_max, e2e_ms_max, attn_ms_max = [float(v) for v in vals]
    total_tokens = w["n_seqs"] * K
    value = total_tokens / (dev_ms_max / 1000.0)
    e2e_value = w["n_seqs"] * E / (e2e_ms_max / 1000.0)

    if rank == 0:
        peaks = json.loads(PEAKS.read_text()) if PEAKS.exists() else {}
        hbm = peaks.get("hbm_gbs")
        peak_src = "measured" if hbm else "fallback"
        hbm = hbm or 6650.0
        achieved = attn_bytes_per_launch / (attn_ms / 1000.0) / 1e9
        mean_ctx = float(np.mean([lens[i] for i in range(len(lens))])) + W + K / 2
        step_bytes = weight_bytes(shape) + w["n_seqs"] * (mean_ctx * kv_bytes_per_position(shape))
        cpu = None
        if world == 1 and not args.no_cpu_baseline:
            try:
                # batch-1 workloads: the reference decodes one sequence on one core
                # (its CPU path is single-threaded); batched: one sequence per host thread
                threads = 1 if w["n_seqs"] == 1 else max(1, min(os.cpu_count() or 1, 64))
                cpu = cpu_reference_sample(w, model_dir, threads, None,
                                           args.cpu_seconds, lens)
            except Exception as e:  # keep the GPU line even if the CPU leg fails
                cpu = {"value": None, "unit": "tokens/s", "cores": 0, "kind": "unavailable", "sample": str(e)}
        line = {
            "metric": METRIC,
            "value": value,
            "unit": "tokens/s",
            "n_gpus": world,
            "steps": K,
            "warmup": W,
            "ms_per_step": dev_ms_max / K,
            "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": None,
            "dtype": "fp16 weights/KV, fp32 accumulate",
            "data": "synthetic (seeded N(0,0.02) weights in the runtime format, uniform prompt ids)",
            "config": {
                "workload": w["desc"],
                "model": w["shape"],
                "global_batch": w["n_seqs"],
                "seq_len": f"prompt U{list(w['prompt'])} + {K} decode steps",
                "parallelism": f"sequence-sharded x{world}, no collective",
                "shard_imbalance": round(shard_imbalance(need, shards), 4),
                "l2": "inputs larger than L2 every step (MiniMind2 fp16 weights 208 MB + KV cache)"
                      if w["n_seqs"] > 1 or w["shape"] == "minimind2" else "weights fit in L2 (batch 1 small)",
                "timed": "K replays of the captured decode-step CUDA graph, CUDA events on the launch stream",
                "prefill_s_untimed": round(prefill_s, 2),
                "prompt_pass": "synthetic K/V fast-forward" if args.fill_context else "device prompt pass (mmc_prefill)",
            },
            "stream": {"value": w["n_seqs"] * K / stream_s, "unit": "tokens/s",
                       "graph_replay_before": w["n_seqs"] * K / (graph_near_ms / 1000.0),
                       "path": "graph replays whose lm_head epilogue writes each step's tokens to mapped pinned host memory, read by the host "
                               "as they land (host wall clock, rank 0)"},
            # per step: the tokens go host -> device (the sequence list only when it changes, not in this
            # loop); the next tokens come back through the argmax epilogue's write into mapped host memory,
            # plus the device error word
            "e2e": {"value": e2e_value, "unit": "tokens/s", "h2d_bytes_per_step": 4 * w["n_seqs"],
                    "d2h_bytes_per_step": 4 * w["n_seqs"] + 4,
                    "path": "mmc_decode_step (host token buffer -> pinned staging -> H2D, graph replay, next tokens "
                            "written to mapped host memory by the argmax epilogue, D2H error word, synchronous)"},
            "gpu_launches": kernels_per_step * K,
            "roofline": {
                "bound": "hbm", "kernel": "persistent decode step (the whole step in one launch)",
                "achieved": timed_bytes / (dev_ms / 1000.0) / 1e9, "peak": hbm, "unit": "GB/s",
                "frac": timed_bytes / (dev_ms / 1000.0) / 1e9 / hbm, "peak_source": f"{peak_src} hbm_gbs",
                "traffic": None, "bytes_per_launch": timed_bytes / K, "avg_launch_ms": dev_ms / K,
                "note": "one launch per step: achieved = algorithmic bytes of the timed steps (weights, every cached "
                        "K/V row, appended rows) / their device time",
            } if persistent else {
                "bound": "hbm", "kernel": "attention (fused q/k norm + RoPE + paged KV append + flash-decode)",
                "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                "peak_source": f"{peak_src} hbm_gbs",
                # DRAM bytes per launch: the ratio of dram__bytes_read.sum + dram__bytes_write.sum to the
                # algorithmic bytes in an ncu capture of a smaller launch of the same kernel (B=128, ctx 1024,
                # hd 96; traffic grows with the pages read), scaled to this launch
                "traffic": attn_bytes_per_launch * ATTN_TRAFFIC_RATIO,
                "traffic_source": "scaled from an ncu capture of a smaller launch (ratio %.3f)" % ATTN_TRAFFIC_RATIO,
                "bytes_per_launch": attn_bytes_per_launch, "avg_launch_ms": attn_ms,
                "step_bytes": step_bytes, "step_frac": step_bytes / (dev_ms_max / K / 1000.0) / 1e9 / hbm,
                "kernel_ms_per_step": {k: v[0] / args.profile_steps for k, v in prof.items()},
            },
            "clocks": clocks,
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    eng.close()
    if dist:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
