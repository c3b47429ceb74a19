"""Split merges of the decode attention: by the split that arrives last at its
(row, kv head) (the default below 48 rows) or from the tail queue once the work
queue drains (the default from 48 rows). Both combine the same partials in the
same order, so contexts created with MMC_ATTN_MERGE_TAIL=0 and =1 must produce
bit-identical logits and tokens; the prompts are long enough for several
splits per (row, kv head)."""
from __future__ import annotations

import os
from pathlib import Path

import numpy as np
import pytest

from minimind_orangepi_b200 import DecodeEngine
from minimind_orangepi_b200.synthetic import SHAPES, synthetic_prompt, write_runtime_model

pytestmark = pytest.mark.gpu


def engine(d, tail: int, n):
    old = os.environ.get("MMC_ATTN_MERGE_TAIL")
    os.environ["MMC_ATTN_MERGE_TAIL"] = str(tail)
    try:
        return DecodeEngine(d, max_seqs=n, max_batch=max(n, 64))
    finally:
        if old is None:
            os.environ.pop("MMC_ATTN_MERGE_TAIL")
        else:
            os.environ["MMC_ATTN_MERGE_TAIL"] = old


@pytest.mark.parametrize("shape_name,n,plen", [("minimind2", 1, 1500), ("minimind2-small", 12, 900),
                                               ("tiny-hd64", 70, 1300)])
def test_merge_modes_are_bit_identical(shape_name, n, plen):
    shape = SHAPES[shape_name]
    d = write_runtime_model(Path("/tmp/mmc_test_models") / f"merge-{shape_name}", shape, 29, eps=1e-5, theta=1e6)
    prompts = [synthetic_prompt(300 + i, plen - (i * 37) % (plen // 2), shape.vocab_size) for i in range(n)]
    with engine(d, 0, n) as a, engine(d, 1, n) as b:
        sa = [a.open_sequence(len(p) + 8) for p in prompts]
        sb = [b.open_sequence(len(p) + 8) for p in prompts]
        toks = [int(t) for t in a.prompt_pass(sa, prompts)]
        assert toks == [int(t) for t in b.prompt_pass(sb, prompts)]
        for _ in range(4):
            na, la = a.step(sa, toks, want_logits=True)
            nb, lb = b.step(sb, toks, want_logits=True)
            assert np.array_equal(la, lb) and np.array_equal(na, nb)
            toks = [int(t) for t in na]
