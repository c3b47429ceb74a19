"""The persistent decode step (step_kernel.cu: the whole step as one
cooperative launch for batches of up to 64 rows) against the chained kernels
(the same model in a context built with MMC_PERSISTENT=0).

Both paths run the same fp16 weights; they differ in how activations are
rounded (the chained CUDA-core path at <= 4 rows keeps them fp32, the
persistent step feeds fp16 rows to mma.sync) and in summation order, so they
are compared within the decode tolerance (2e-2 absolute + 1e-2 relative); each
is also held to the reference by tests/test_gpu_decode.py and
tests/test_gpu_configs.py. The batch sizes cover one and two row groups,
partial n-tiles, multi-tile projection tasks, 16-row blocks for the long
down-projection rows, and attention jobs of several chunks (contexts past a
few pages)."""
from __future__ import annotations

import os
from pathlib import Path

import numpy as np
import pytest

from minimind_orangepi_b200 import DecodeEngine
from minimind_orangepi_b200.synthetic import SHAPES, synthetic_prompt, write_runtime_model

pytestmark = pytest.mark.gpu
ATOL, RTOL = 2e-2, 1e-2


def engine(d, persistent: bool, n):
    old = os.environ.get("MMC_PERSISTENT")
    os.environ["MMC_PERSISTENT"] = "1" if persistent else "0"
    try:
        return DecodeEngine(d, max_seqs=n, max_batch=n)
    finally:
        if old is None:
            os.environ.pop("MMC_PERSISTENT")
        else:
            os.environ["MMC_PERSISTENT"] = old


@pytest.mark.parametrize("shape_name,n,plen", [("minimind2", 1, 900), ("minimind2-small", 5, 400), ("minimind2", 17, 400),
                                               ("minimind2", 33, 300), ("minimind2-small", 64, 200),
                                               ("tiny-hd64", 40, 400)])
def test_persistent_step_matches_chained_kernels(shape_name, n, plen):
    shape = SHAPES[shape_name]
    d = write_runtime_model(Path("/tmp/mmc_test_models") / f"persist-{shape_name}", shape, 13, eps=1e-5, theta=1e6)
    prompts = [synthetic_prompt(500 + i, 3 + (i * 53) % plen, shape.vocab_size) for i in range(n)]
    if n == 1:
        prompts = [synthetic_prompt(500, plen, shape.vocab_size)]
    with engine(d, True, n) as a, engine(d, False, n) as b:
        assert a.kernels_per_step(n) == 1 and b.kernels_per_step(n) > 1
        sa = [a.open_sequence(len(p) + 8) for p in prompts]
        sb = [b.open_sequence(len(p) + 8) for p in prompts]
        fa = a.prompt_pass(sa, prompts)  # the prompt pass runs the chained kernels in both
        fb = b.prompt_pass(sb, prompts)
        assert np.array_equal(fa, fb)
        toks = [int(t) for t in fb]
        for step in range(4):
            na, la = a.step(sa, toks, want_logits=True)
            nb, lb = b.step(sb, toks, want_logits=True)
            err = np.abs(la - lb) - (ATOL + RTOL * np.abs(lb))
            assert (err <= 0).all(), f"step {step}: max excess {err.max():.3e}"
            for i in range(n):  # the persistent step's token is the first maximum of its own logits
                assert int(na[i]) == int(np.argmax(la[i]))
            toks = [int(t) for t in nb]
        # the K/V rows the persistent step appended equal the chained path's
        for layer in (0, shape.num_hidden_layers - 1):
            ka, va = a.read_kv(sa[-1], layer)
            kb, vb = b.read_kv(sb[-1], layer)
            assert np.abs(ka - kb).max() <= 2e-2 and np.abs(va - vb).max() <= 2e-2
        assert all(a.position(x) == b.position(y) for x, y in zip(sa, sb))


def test_persistent_graph_loop_matches_eager_steps():
    """Replays of the captured persistent step feed their own tokens back."""
    shape = SHAPES["minimind2-small"]
    d = write_runtime_model(Path("/tmp/mmc_test_models") / "persist-minimind2-small", shape, 13, eps=1e-5,
                            theta=1e6)
    n, steps = 24, 50
    prompts = [synthetic_prompt(700 + i, 5 + 11 * i, shape.vocab_size) for i in range(n)]
    with engine(d, True, 2 * n) as eng:
        a = [eng.open_sequence(len(p) + steps + 2) for p in prompts]
        b = [eng.open_sequence(len(p) + steps + 2) for p in prompts]
        first = eng.prompt_pass(a, prompts)
        assert np.array_equal(first, eng.prompt_pass(b, prompts))
        cur, eager = first.copy(), []
        for _ in range(steps):
            cur, _ = eng.step(a, cur)
            eager.append(cur.copy())
        eng.graph_build(b)
        eng.graph_set_tokens(first)
        eng.graph_run(steps)
        assert np.array_equal(np.stack(eager), eng.graph_tokens(steps))
