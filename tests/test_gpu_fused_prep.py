"""Decode attention with the q/k RMSNorm + RoPE + K/V append folded into the
attention kernel (the default for decode steps) against the separate prep
launch (a context created with MMC_ATTN_FUSED=0). Both compute the same
arithmetic with the same roundings (fp32 norm + RoPE of the raw projections,
fp16 q and cache rows), so logits, tokens and the appended cache rows must be
bit-identical. The CUDA-core (batch <= 4) and tensor-core paths, a MoE model
and splits across pages are covered; batches that run as concurrent parts keep
the separate prep launch (measured faster there)."""
from __future__ import annotations

import os
from pathlib import Path

import numpy as np
import pytest

from minimind_orangepi_b200 import DecodeEngine
from minimind_orangepi_b200.synthetic import SHAPES, synthetic_prompt, write_runtime_model

pytestmark = pytest.mark.gpu


def engine(d, fused: bool, n):
    old = os.environ.get("MMC_ATTN_FUSED")
    os.environ["MMC_ATTN_FUSED"] = "1" if fused else "0"
    try:
        return DecodeEngine(d, max_seqs=n, max_batch=n)
    finally:
        if old is None:
            os.environ.pop("MMC_ATTN_FUSED")
        else:
            os.environ["MMC_ATTN_FUSED"] = old


@pytest.mark.parametrize("shape_name,n,plen", [("minimind2", 1, 700), ("minimind2-small", 3, 300),
                                               ("minimind2", 40, 900), ("minimind2-small", 100, 600),
                                               ("tiny-hd64", 9, 200), ("tiny-moe", 20, 150)])
def test_fused_prep_is_bit_identical(shape_name, n, plen):
    shape = SHAPES[shape_name]
    d = write_runtime_model(Path("/tmp/mmc_test_models") / f"fused-{shape_name}", shape, 17, eps=1e-5, theta=1e6)
    prompts = [synthetic_prompt(900 + i, 2 + (i * 71) % plen, shape.vocab_size) for i in range(n)]
    with engine(d, True, n) as a, engine(d, False, n) as b:
        assert a.kernels_per_step(n) < b.kernels_per_step(n)
        sa = [a.open_sequence(len(p) + 8) for p in prompts]
        sb = [b.open_sequence(len(p) + 8) for p in prompts]
        toks = [int(t) for t in a.prompt_pass(sa, prompts)]
        assert toks == [int(t) for t in b.prompt_pass(sb, prompts)]
        for _ in range(5):
            na, la = a.step(sa, toks, want_logits=True)
            nb, lb = b.step(sb, toks, want_logits=True)
            assert np.array_equal(la, lb) and np.array_equal(na, nb)
            toks = [int(t) for t in na]
        for layer in (0, shape.num_hidden_layers - 1):
            for i in (0, n - 1):
                ka, va = a.read_kv(sa[i], layer)
                kb, vb = b.read_kv(sb[i], layer)
                assert np.array_equal(ka, kb) and np.array_equal(va, vb)
