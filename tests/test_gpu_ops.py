"""Per-kernel parity through the C ABI's operator entry points (BASELINE config
5 shapes): projections, fused lm_head + argmax, fused decode attention. The
checkers are the CPU oracle's restatements of the reference formulas
(oracle/minimind_oracle.c) and torch fp32 for the plain projections."""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

from minimind_orangepi_b200._lib import check, lib

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

SWEEP_SHAPES = [(512, 512), (128, 512), (1408, 512), (512, 1408), (768, 768), (192, 768), (2048, 768),
                (768, 2048), (6400, 768)]


def dev(t):
    return C.c_void_p(t.data_ptr())


@pytest.mark.parametrize("n,k", SWEEP_SHAPES)
@pytest.mark.parametrize("batch", [1, 3, 5, 8, 64, 100, 256])
def test_projection(n, k, batch):
    g = torch.Generator(device="cpu").manual_seed(n * 7 + k + batch)
    w = (torch.randn(n, k, generator=g) * 0.02).half().cuda()
    x = torch.randn(batch, k, generator=g).cuda()
    y = torch.full((batch, n), float("nan"), device="cuda")
    # fp32 activations for the CUDA-core path (batch <= 4), fp16 for tcgen05
    xa = x if batch <= 4 else x.half().contiguous()
    check(lib().mmc_op_projection(batch, n, k, dev(w), dev(xa), dev(y), None))
    torch.cuda.synchronize()
    # batches > 4 run on tensor cores with fp16 activations; <= 4 in fp32
    xr = x if batch <= 4 else x.half().float()
    ref = xr @ w.float().t()
    tol = 1e-4 * k ** 0.5 if batch <= 4 else 2e-4 * k ** 0.5
    assert torch.isfinite(y).all()
    assert (y - ref).abs().max().item() <= tol


@pytest.mark.parametrize("n,k,batch", [(768, 2048, 100), (768, 768, 64), (1280, 768, 128)])
def test_projection_split_k_is_deterministic(n, k, batch):
    """Few-tile projections split K across a thread-block cluster and sum the
    partial accumulators in a fixed rank order: repeated runs are bit-equal."""
    g = torch.Generator(device="cpu").manual_seed(n + k + batch)
    w = (torch.randn(n, k, generator=g) * 0.02).half().cuda()
    x = torch.randn(batch, k, generator=g).half().cuda()
    outs = []
    for _ in range(3):
        y = torch.full((batch, n), float("nan"), device="cuda")
        check(lib().mmc_op_projection(batch, n, k, dev(w), dev(x), dev(y), None))
        torch.cuda.synchronize()
        outs.append(y)
    ref = x.float() @ w.float().t()
    assert (outs[0] - ref).abs().max().item() <= 2e-4 * k ** 0.5
    assert torch.equal(outs[0], outs[1]) and torch.equal(outs[0], outs[2])


@pytest.mark.parametrize("batch", [1, 2, 4, 8, 64, 256, 513, 600, 1024])
def test_lm_head_argmax_is_first_max_of_its_own_logits(batch):
    n, k = 6400, 768
    g = torch.Generator(device="cpu").manual_seed(batch)
    w = (torch.randn(n, k, generator=g) * 0.02).half()
    # plant exact ties: duplicate rows so two vocab ids give the same logit
    w[4000] = w[17]
    w[6399] = w[5]
    w = w.cuda()
    x = torch.randn(batch, k, generator=g).cuda()
    logits = torch.empty(batch, n, device="cuda")
    nxt = torch.full((batch,), -1, dtype=torch.int32, device="cuda")
    ws_bytes = C.c_size_t()
    check(lib().mmc_op_lm_head_argmax_workspace_size(batch, n, k, C.byref(ws_bytes)))
    ws = torch.empty(ws_bytes.value, dtype=torch.uint8, device="cuda")
    xa = x if batch <= 4 else x.half().contiguous()
    for _ in range(3):  # repeated launches: the arrival counters must self-reset
        check(lib().mmc_op_lm_head_argmax(batch, n, k, dev(w), dev(xa), dev(logits), dev(nxt), dev(ws),
                                          ws_bytes.value, None))
    torch.cuda.synchronize()
    lg = logits.cpu().numpy()
    got = nxt.cpu().numpy()
    for b in range(batch):
        assert got[b] == int(np.argmax(lg[b])), f"row {b}"  # np.argmax = first maximum
    xr = x if batch <= 4 else x.half().float()
    ref = (xr @ w.float().t()).cpu().numpy()
    assert np.abs(lg - ref).max() <= 2e-4 * k ** 0.5


def test_lm_head_argmax_tie_goes_to_lowest_index():
    n, k = 6400, 768
    w = torch.zeros(n, k, dtype=torch.half)
    w[:, 0] = 1.0  # every logit equal -> index 0 wins
    w = w.cuda()
    for batch in (1, 4, 16):
        x = torch.ones(batch, k, device="cuda")
        if batch > 4:
            x = x.half()
        nxt = torch.full((batch,), -1, dtype=torch.int32, device="cuda")
        ws_bytes = C.c_size_t()
        check(lib().mmc_op_lm_head_argmax_workspace_size(batch, n, k, C.byref(ws_bytes)))
        ws = torch.empty(ws_bytes.value, dtype=torch.uint8, device="cuda")
        check(lib().mmc_op_lm_head_argmax(batch, n, k, dev(w), dev(x), None, dev(nxt), dev(ws), ws_bytes.value,
                                          None))
        torch.cuda.synchronize()
        assert (nxt.cpu() == 0).all()


def _oracle():
    from oracle.oracle import fptr, lib as olib
    return olib(), fptr


def _pool_perm(hd):
    """Physical element index of each logical (row, d) of a 64 x hd page slab."""
    perm = np.array([lib().mmc_kv_row_offset(hd, r, c) for r in range(64) for c in range(hd // 8)])
    return (perm[:, None] + np.arange(8)[None, :]).reshape(-1)


def _attention_case(hd, ctxs, seed, nq=8, nkv=2, layers=2, layer=1):
    """Host arrays of one attention-op call: ragged rows with ctxs[b] cached
    positions (incl. the current one), pages assigned in order from page 1
    (page 0 stays unused), random fp16 K/V written through the swizzle."""
    eps, theta = 1e-5, 1e6
    olib, fptr = _oracle()
    rng = np.random.default_rng(seed)
    batch, max_ctx, half = len(ctxs), max(ctxs), hd // 2
    cos_t = np.empty(max_ctx * half, np.float32)
    sin_t = np.empty(max_ctx * half, np.float32)
    olib.mmo_rope_tables(max_ctx, hd, theta, fptr(cos_t), fptr(sin_t))
    qn = (1.0 + 0.1 * rng.standard_normal(hd)).astype(np.float32)
    kn = (1.0 + 0.1 * rng.standard_normal(hd)).astype(np.float32)
    qkv = rng.standard_normal((batch, (nq + 2 * nkv) * hd)).astype(np.float32)
    max_pages = (max_ctx + 63) // 64
    n_pages = sum((c + 63) // 64 for c in ctxs) + 1
    tile = 64 * hd
    perm = _pool_perm(hd)
    pool = np.zeros((n_pages, layers, 2, nkv, tile), np.float16)
    bt = -np.ones((batch, max_pages), np.int32)
    nxt_page = 1
    caches = []
    for b, c in enumerate(ctxs):
        pos, np_b = c - 1, (c + 63) // 64
        pages = np.arange(nxt_page, nxt_page + np_b)
        bt[b, :np_b] = pages
        nxt_page += np_b
        K = rng.standard_normal((pos, nkv, hd), dtype=np.float32).astype(np.float16)
        V = rng.standard_normal((pos, nkv, hd), dtype=np.float32).astype(np.float16)
        caches.append((K, V))
        for kv, arr in ((0, K), (1, V)):
            padded = np.zeros((np_b * 64, nkv, hd), np.float16)
            padded[:pos] = arr
            logical = padded.reshape(np_b, 64, nkv, hd).transpose(0, 2, 1, 3).reshape(np_b, nkv, tile)
            phys = np.zeros_like(logical)
            phys[:, :, perm] = logical
            pool[pages, layer, kv] = phys
    return dict(hd=hd, nq=nq, nkv=nkv, layers=layers, layer=layer, eps=eps, ctxs=ctxs, cos=cos_t, sin=sin_t, qn=qn,
                kn=kn, qkv=qkv, bt=bt, pool=pool, caches=caches, max_pages=max_pages, tile=tile, perm=perm)


def _attention_run(c, bt=None):
    """Runs mmc_op_attention on the case; returns (status of
    mmc_op_attention_status, out, pool after)."""
    batch, max_ctx = len(c["ctxs"]), max(c["ctxs"])
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731
    d_pool = t(c["pool"])
    d_bt, d_pos = t(c["bt"] if bt is None else bt), t(np.array([x - 1 for x in c["ctxs"]], np.int32))
    d_slots = t(np.arange(batch, dtype=np.int32))
    d_qkv, d_qn, d_kn, d_cos, d_sin = t(c["qkv"]), t(c["qn"]), t(c["kn"]), t(c["cos"]), t(c["sin"])
    nq, nkv, hd = c["nq"], c["nkv"], c["hd"]
    out = torch.full((batch, nq * hd), float("nan"), device="cuda")
    ws_bytes = C.c_size_t()
    check(lib().mmc_op_attention_workspace_size(batch, nq, nkv, hd, max_ctx, C.byref(ws_bytes)))
    ws = torch.empty(ws_bytes.value, dtype=torch.uint8, device="cuda")
    check(lib().mmc_op_attention(batch, nq, nkv, hd, c["layer"], c["layers"], dev(d_qkv), dev(d_qn), dev(d_kn),
                                 dev(d_cos), dev(d_sin), max_ctx, c["eps"], dev(d_pool), dev(d_bt), c["max_pages"],
                                 dev(d_pos), dev(d_slots), max_ctx, dev(out), dev(ws), ws_bytes.value, None))
    status = lib().mmc_op_attention_status(dev(ws), None)
    torch.cuda.synchronize()
    return status, out.cpu().numpy(), d_pool.cpu().numpy()


def _attention_check(c, got, pool_after, rows=None):
    olib, fptr = _oracle()
    nq, nkv, hd, eps, tile, perm = c["nq"], c["nkv"], c["hd"], c["eps"], c["tile"], c["perm"]
    cos_t, sin_t = c["cos"], c["sin"]
    for b in (range(len(c["ctxs"])) if rows is None else rows):
        cx = c["ctxs"][b]
        pos = cx - 1
        row = c["qkv"][b].copy()
        q = row[:nq * hd].copy()
        k = row[nq * hd:(nq + nkv) * hd].copy()
        v = row[(nq + nkv) * hd:].copy()
        for h in range(nq):
            seg = q[h * hd:(h + 1) * hd].copy()
            olib.mmo_rms_norm_inplace(fptr(seg), fptr(c["qn"]), hd, eps)
            q[h * hd:(h + 1) * hd] = seg
        for h in range(nkv):
            seg = k[h * hd:(h + 1) * hd].copy()
            olib.mmo_rms_norm_inplace(fptr(seg), fptr(c["kn"]), hd, eps)
            k[h * hd:(h + 1) * hd] = seg
        olib.mmo_apply_rope(fptr(q), nq, hd, pos, fptr(cos_t), fptr(sin_t))
        olib.mmo_apply_rope(fptr(k), nkv, hd, pos, fptr(cos_t), fptr(sin_t))
        K, V = c["caches"][b]
        Kf = np.concatenate([K.astype(np.float32), k.reshape(1, nkv, hd)], 0)
        Vf = np.concatenate([V.astype(np.float32), v.reshape(1, nkv, hd)], 0)
        ref = np.zeros(nq * hd, np.float32)
        olib.mmo_attention(fptr(q), fptr(np.ascontiguousarray(Kf)), fptr(np.ascontiguousarray(Vf)), cx, nq, nkv, hd,
                           fptr(ref))
        err = np.abs(got[b] - ref)
        assert (err <= 5e-3 + 1e-2 * np.abs(ref)).all(), f"row {b} ctx {cx}: max err {err.max():.3e}"
        # the appended row holds fp16(normed, roped k) and fp16(v)
        page = c["bt"][b, pos // 64]
        for kv, vec in ((0, k), (1, v)):
            for h in range(nkv):
                phys = pool_after[page, c["layer"], kv, h]
                logical = phys[perm].reshape(64, hd)[pos % 64]
                exp = vec[h * hd:(h + 1) * hd].astype(np.float16)
                assert np.array_equal(logical, exp) or np.abs(logical.astype(np.float32) - exp.astype(
                    np.float32)).max() <= 1e-3 * np.abs(exp.astype(np.float32)).max()
    # untouched page 0 stays zero (no stray writes)
    assert not pool_after[0].any()


@pytest.mark.parametrize("hd", [64, 96])
@pytest.mark.parametrize("ctx,batch", [(1, 1), (63, 1), (64, 2), (65, 1), (200, 3), (1024, 2), (8192, 1),
                                       (32768, 1), (1500, 9)])
def test_attention_op(hd, ctx, batch):
    c = _attention_case(hd, [max(1, ctx - 37 * b) for b in range(batch)], hd * 1000 + ctx + batch)
    status, got, pool_after = _attention_run(c)
    assert status == 0
    _attention_check(c, got, pool_after)


@pytest.mark.parametrize("hd", [64, 96])
@pytest.mark.parametrize("batch,max_ctx", [(64, 8192), (256, 8192), (64, 32768)])
def test_attention_op_sweep_batches(hd, batch, max_ctx):
    """The config-5 sweep's batch sizes: ragged contexts up to max_ctx, so many
    (row, kv head) items run several splits merged from the tail queue.
    Every row is compared at B=64; at B=256 every 5th row and the longest."""
    rng = np.random.default_rng(batch + max_ctx + hd)
    ctxs = [int(x) for x in rng.integers(1, max_ctx + 1, size=batch)]
    ctxs[batch // 2] = max_ctx
    c = _attention_case(hd, ctxs, batch * 7 + hd, layers=1, layer=0)
    status, got, pool_after = _attention_run(c)
    assert status == 0
    rows = None if batch <= 64 else sorted(set(range(0, batch, 5)) | {batch // 2})
    _attention_check(c, got, pool_after, rows)


def test_attention_op_reports_missing_page():
    """A block-table entry of -1 for a needed page: the kernel records the
    error and skips the page (it neither traps nor reads page -1);
    mmc_op_attention_status returns MMC_ERR_DEVICE and clears the word."""
    c = _attention_case(96, [300, 200], 5)
    bt = c["bt"].copy()
    bt[0, 2] = -1
    status, _, pool_after = _attention_run(c, bt)
    assert status == 5  # MMC_ERR_DEVICE
    assert b"page" in lib().mmc_last_error()
    assert not pool_after[0].any()
    # the same inputs with a complete table are clean
    status, got, pool_after = _attention_run(c)
    assert status == 0
    _attention_check(c, got, pool_after)
