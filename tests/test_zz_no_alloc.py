"""The allocation-free attention entry point (mmc_op_attention_noalloc).

It exists for callers that may not call cudaMalloc where they run (a custom
allocator's own hooks, loops with a no-allocation rule, hosts that own all
device memory): instead of a caller-provided workspace it uses a fixed scratch
array inside the library. These tests call it through the C ABI twice in a row
and compare each result with the workspace-taking mmc_op_attention on identical
inputs, check that a size beyond the fixed scratch is refused, and that a
device-side error comes back as MMC_ERR_DEVICE. This file is collected last on
purpose; it passes alone in a fresh process and after the other tests.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import pytest

from minimind_orangepi_b200._lib import MmcError, check, lib

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

ATOL, RTOL = 5e-3, 1e-2  # the attention tolerance used by tests/test_gpu_ops.py


def dev(t):
    return C.c_void_p(t.data_ptr()) if t is not None else None


def _case(seed, batch=5, ctx=700, hd=96, nq=8, nkv=2):
    g = torch.Generator(device="cpu").manual_seed(seed)
    pages = (ctx + 63) // 64
    n_pages = batch * pages + 1
    perm = torch.randperm(n_pages - 1, generator=g) + 1
    bt = perm[: batch * pages].reshape(batch, pages).to(torch.int32).cuda()
    pool = (torch.randn(n_pages * 2 * nkv * 64 * hd, generator=g)).half().cuda()
    ctxs = [max(1, ctx - 53 * b) for b in range(batch)]
    pos = torch.tensor([c - 1 for c in ctxs], dtype=torch.int32).cuda()
    slots = torch.arange(batch, dtype=torch.int32).cuda()
    qkv = torch.randn(batch, (nq + 2 * nkv) * hd, generator=g).cuda()
    qn = (1 + 0.1 * torch.randn(hd, generator=g)).cuda()
    kn = (1 + 0.1 * torch.randn(hd, generator=g)).cuda()
    ang = torch.arange(ctx).float()[:, None] * (1e6 ** (-torch.arange(hd // 2).float() * 2 / hd))[None, :]
    cos, sin = ang.cos().reshape(-1).contiguous().cuda(), ang.sin().reshape(-1).contiguous().cuda()
    return dict(batch=batch, nq=nq, nkv=nkv, hd=hd, ctx=ctx, pages=pages, bt=bt, pool=pool, pos=pos, slots=slots,
                qkv=qkv, qn=qn, kn=kn, cos=cos, sin=sin)


def _args(c, pool, out):
    return [c["batch"], c["nq"], c["nkv"], c["hd"], 0, 1, dev(c["qkv"]), dev(c["qn"]), dev(c["kn"]), dev(c["cos"]),
            dev(c["sin"]), c["ctx"], 1e-5, dev(pool), dev(c["bt"]), c["pages"], dev(c["pos"]), dev(c["slots"]),
            c["ctx"]]


def _with_workspace(c):
    pool = c["pool"].clone()
    out = torch.full((c["batch"], c["nq"] * c["hd"]), float("nan"), device="cuda")
    ws_n = C.c_size_t()
    check(lib().mmc_op_attention_workspace_size(c["batch"], c["nq"], c["nkv"], c["hd"], c["ctx"], C.byref(ws_n)))
    ws = torch.empty(ws_n.value, dtype=torch.uint8, device="cuda")
    check(lib().mmc_op_attention(*_args(c, pool, out), dev(out), dev(ws), ws_n.value, None))
    torch.cuda.synchronize()
    return out, pool


def _no_alloc(c):
    pool = c["pool"].clone()
    out = torch.full((c["batch"], c["nq"] * c["hd"]), float("nan"), device="cuda")
    check(lib().mmc_op_attention_noalloc(*_args(c, pool, out), dev(out), None))
    torch.cuda.synchronize()
    return out, pool


def test_no_alloc_attention_matches_workspace_entry_point_twice():
    for seed in (1, 2):  # two calls in a row share (and reuse) the fixed scratch
        c = _case(seed)
        ref, ref_pool = _with_workspace(c)
        got, got_pool = _no_alloc(c)
        assert torch.isfinite(got).all()
        err = (got - ref).abs()
        assert (err <= ATOL + RTOL * ref.abs()).all(), f"call {seed}: max err {err.max().item():.3e}"
        # the appended K/V rows land in the cache exactly as with a workspace
        assert torch.equal(got_pool, ref_pool)


def test_no_alloc_attention_refuses_sizes_beyond_its_scratch():
    c = _case(3, batch=2, ctx=64)
    out = torch.empty(256, 8 * 96, device="cuda")
    big = _args(c, c["pool"], out)
    big[0] = 256          # batch
    big[-1] = 32768       # max_ctx: 256 rows x 64 splits of partials >> 16 MiB
    code = lib().mmc_op_attention_noalloc(*big, dev(out), None)
    assert code == 1
    with pytest.raises(MmcError, match="scratch"):
        check(code)


def test_no_alloc_attention_reports_device_errors():
    """The caller cannot reach the error word inside the library's array, so the
    entry point reports it: a block table with -1 for a needed page returns
    MMC_ERR_DEVICE (the kernel records the error and skips the page; nothing
    traps), and the next call with a complete table succeeds again."""
    c = _case(4, batch=2, ctx=300)
    bt = c["bt"].clone()
    bt[0, 1] = -1
    bad = dict(c, bt=bt)
    pool = c["pool"].clone()
    out = torch.empty(c["batch"], c["nq"] * c["hd"], device="cuda")
    code = lib().mmc_op_attention_noalloc(*_args(bad, pool, out), dev(out), None)
    assert code == 5
    assert b"page" in lib().mmc_last_error()
    ref, _ = _with_workspace(c)
    got, _ = _no_alloc(c)
    err = (got - ref).abs()
    assert (err <= ATOL + RTOL * ref.abs()).all()
