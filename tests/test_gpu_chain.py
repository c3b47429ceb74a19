"""The persistent o / gate-up / down projection chain (mlp_chain.cu, enabled
per context with MMC_MLP_CHAIN=1) against the default three launches: the
same batched decode steps give the same logits within the decode tolerance
(2e-2 absolute + 1e-2 relative; the chain changes no arithmetic, only how
the tiles are scheduled) and the same positions, for a batch that runs as one
part and one that runs as several concurrent parts."""
from __future__ import annotations

import os
from pathlib import Path

import numpy as np
import pytest

from minimind_orangepi_b200 import DecodeEngine
from minimind_orangepi_b200.synthetic import SHAPES, synthetic_prompt, write_runtime_model

pytestmark = pytest.mark.gpu
ATOL, RTOL = 2e-2, 1e-2


def engine(d, chain: bool, n):
    old = os.environ.get("MMC_MLP_CHAIN")
    os.environ["MMC_MLP_CHAIN"] = "1" if chain else "0"
    try:
        return DecodeEngine(d, max_seqs=n, max_batch=n)
    finally:
        if old is None:
            os.environ.pop("MMC_MLP_CHAIN")
        else:
            os.environ["MMC_MLP_CHAIN"] = old


@pytest.mark.parametrize("shape_name,n", [("minimind2-small", 100), ("minimind2", 256)])
def test_chain_matches_separate_projections(shape_name, n):
    shape = SHAPES[shape_name]
    d = write_runtime_model(Path("/tmp/mmc_test_models") / f"chain-{shape_name}", shape, 9, eps=1e-5, theta=1e6)
    prompts = [synthetic_prompt(100 + i, 3 + (i * 37) % 150, shape.vocab_size) for i in range(n)]
    with engine(d, True, n) as a, engine(d, False, n) as b:
        assert a.kernels_per_step(n) < b.kernels_per_step(n)
        sa = [a.open_sequence(len(p) + 8) for p in prompts]
        sb = [b.open_sequence(len(p) + 8) for p in prompts]
        fa = a.prompt_pass(sa, prompts)
        fb = b.prompt_pass(sb, prompts)
        toks = [int(t) for t in fb]
        for step in range(3):
            na, la = a.step(sa, toks, want_logits=True)
            nb, lb = b.step(sb, toks, want_logits=True)
            err = np.abs(la - lb) - (ATOL + RTOL * np.abs(lb))
            assert (err <= 0).all(), f"step {step}: max excess {err.max():.3e}"
            toks = [int(t) for t in nb]
        assert (fa == fb).mean() > 0.9
        assert all(a.position(x) == b.position(y) for x, y in zip(sa, sb))
