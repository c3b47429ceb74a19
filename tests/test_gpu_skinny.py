"""Projections of 2..64-row decode batches on the skinny mma.sync kernel
(skinny.cu, the default) against the tcgen05 projections (a context created
with MMC_SKINNY=0) on the same prompts. The two paths sum each dot product in
a different order, so logits agree to the decode tolerance, not bitwise:
within 2e-2 absolute + 1e-2 relative, and greedy ids identical except where
the other path's top-2 gap is below 2e-2. The rows also decode against the
CPU oracle in test_gpu_decode.py (batched cases of 5..37 rows)."""
from __future__ import annotations

import os
from pathlib import Path

import numpy as np
import pytest

from minimind_orangepi_b200 import DecodeEngine
from minimind_orangepi_b200.synthetic import SHAPES, synthetic_prompt, write_runtime_model

pytestmark = pytest.mark.gpu
ATOL, RTOL = 2e-2, 1e-2


def engine(d, skinny: bool, n):
    old = os.environ.get("MMC_SKINNY")
    os.environ["MMC_SKINNY"] = "1" if skinny else "0"
    try:
        return DecodeEngine(d, max_seqs=n, max_batch=max(n, 64))
    finally:
        if old is None:
            os.environ.pop("MMC_SKINNY")
        else:
            os.environ["MMC_SKINNY"] = old


@pytest.mark.parametrize("shape_name,n,plen", [("minimind2", 64, 900), ("minimind2", 41, 300),
                                               ("minimind2", 32, 1100), ("minimind2", 17, 300),
                                               ("minimind2-small", 8, 600), ("tiny-hd64", 5, 200), ("minimind2-small", 3, 400), ("tiny-hd64", 2, 100),
                                               ("tiny-hd96", 24, 150)])
def test_skinny_matches_tensor_core_path(shape_name, n, plen):
    shape = SHAPES[shape_name]
    d = write_runtime_model(Path("/tmp/mmc_test_models") / f"skinny-{shape_name}", shape, 23, eps=1e-5, theta=1e6)
    prompts = [synthetic_prompt(700 + i, 2 + (i * 97) % plen, shape.vocab_size) for i in range(n)]
    with engine(d, True, n) as a, engine(d, False, n) as b:
        sa = [a.open_sequence(len(p) + 8) for p in prompts]
        sb = [b.open_sequence(len(p) + 8) for p in prompts]
        a.prompt_pass(sa, prompts)
        toks = [int(t) for t in b.prompt_pass(sb, prompts)]
        differs = False
        for step in range(6):
            na, la = a.step(sa, toks, want_logits=True)
            nb, lb = b.step(sb, toks, want_logits=True)
            differs |= not np.array_equal(la, lb)
            err = np.abs(la - lb)
            assert (err <= ATOL + RTOL * np.abs(lb)).all(), f"step {step}: max |diff| {err.max():.3e}"
            for r in range(n):
                srt = np.sort(lb[r])
                if srt[-1] - srt[-2] >= ATOL:
                    assert na[r] == nb[r], f"step {step} row {r}: {na[r]} != {nb[r]}"
                assert int(na[r]) == int(np.argmax(la[r])), "argmax is not the first maximum of its own logits"
            toks = [int(t) for t in nb]
        # the two contexts ran different kernels (different summation orders)
        assert differs
        for i in range(n):
            assert a.position(sa[i]) == b.position(sb[i])
