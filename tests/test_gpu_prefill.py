"""Device prompt pass (mmc_prefill) on the GPU.

One batched pass per up to max_batch prompt positions replaces feeding the
prompt token by token. Checked against the reference's golden fixtures (the
first generated token and every later decode step's logits, which read the
K/V the pass appended) and against the token-by-token path of this engine
(appended K/V, positions, first tokens), including prompts split across
passes and several sequences in one pass. Tolerances as in
test_gpu_decode.py: logits within 2e-2 absolute + 1e-2 relative; greedy ids
equal unless the reference's top-2 gap is below 2e-2.
"""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import pytest

from minimind_orangepi_b200 import DecodeEngine, MmcError
from minimind_orangepi_b200.synthetic import SHAPES, ModelShape, synthetic_prompt, write_runtime_model

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]
GOLDEN = ROOT / "tests" / "golden"
ATOL, RTOL = 2e-2, 1e-2


def close(a, b):
    return np.abs(a - b) <= ATOL + RTOL * np.abs(b)


def golden_model(name):
    g = np.load(GOLDEN / f"{name}.npz")
    shape = ModelShape(**json.loads(str(g["shape"])))
    d = write_runtime_model(Path("/tmp/mmc_test_models") / f"golden-{name}", shape, int(g["model_seed"]),
                            eps=float(g["eps"]), theta=float(g["theta"]))
    return g, d


@pytest.mark.parametrize("name,max_batch", [("tiny-hd96-page-cross", 128), ("tiny-hd96-page-cross", 16),
                                            ("tiny-hd64", 64), ("cfg1-minimind2-small", 8), ("tiny-moe", 16)])
def test_prompt_pass_matches_reference_golden(name, max_batch):
    """Prompt = the fixture's first n fed tokens through mmc_prefill (in passes
    of max_batch rows), then the remaining fed tokens by decode steps: every
    output matches the reference's."""
    g, d = golden_model(name)
    fed, argmax = [int(t) for t in g["fed"]], g["argmax"]
    n = min(len(g["prompt"]), len(fed) - 2)
    with DecodeEngine(d, max_seqs=2, max_batch=max_batch) as eng:
        seq = eng.open_sequence(len(fed) + 1)
        first = int(eng.prompt_pass([seq], [fed[:n]])[0])
        assert eng.position(seq) == n
        if g["top2gap"][n - 1] >= ATOL:
            assert first == int(argmax[n - 1]), f"{name}: first token {first} != reference {argmax[n - 1]}"
        for i in range(n, len(fed)):
            nxt, logits = eng.step([seq], [fed[i]], want_logits=True)
            idx, val = g["topk_idx"][i], g["topk_val"][i]
            assert close(logits[0][idx], val).all(), \
                f"{name} step {i}: top-k logits differ by {np.abs(logits[0][idx] - val).max():.3e}"
            if g["top2gap"][i] >= ATOL:
                assert int(nxt[0]) == int(argmax[i])


def test_prompt_pass_matches_token_by_token_kv():
    """Several sequences of different lengths (one longer than a pass) in one
    call: appended K/V, positions and first tokens equal the token-by-token
    prompt loop's within tolerance."""
    shape = SHAPES["minimind2-small"]
    d = write_runtime_model(Path("/tmp/mmc_test_models") / "prefill-small", shape, 5, eps=1e-5, theta=1e6)
    lens = [70, 5, 200, 1]
    prompts = [synthetic_prompt(10 + i, n, shape.vocab_size) for i, n in enumerate(lens)]
    with DecodeEngine(d, max_seqs=8, max_batch=96) as a, DecodeEngine(d, max_seqs=8, max_batch=96) as b:
        sa = [a.open_sequence(n + 4) for n in lens]
        sb = [b.open_sequence(n + 4) for n in lens]
        fa = a.prompt_pass(sa, prompts)
        fb = b.prefill(sb, prompts)
        for i, n in enumerate(lens):
            assert a.position(sa[i]) == n and b.position(sb[i]) == n
            for layer in (0, shape.num_hidden_layers - 1):
                ka, va = a.read_kv(sa[i], layer)
                kb, vb = b.read_kv(sb[i], layer)
                assert np.abs(ka - kb).max() <= 3e-2 and np.abs(va - vb).max() <= 3e-2, f"seq {i} layer {layer}"
        # the next decode step sees the same context on both engines
        na, la = a.step(sa, [int(t) for t in fa], want_logits=True)
        nb, lb = b.step(sb, [int(t) for t in fa], want_logits=True)
        assert close(la, lb).all(), f"max |diff| {np.abs(la - lb).max():.3e}"
        # first tokens: equal unless a near-tie flips one (synthetic weights give small gaps)
        assert (fa == fb).sum() >= len(lens) - 1


def test_prompt_pass_rejects_bad_input():
    shape = SHAPES["minimind2-small"]
    d = write_runtime_model(Path("/tmp/mmc_test_models") / "prefill-small", shape, 5, eps=1e-5, theta=1e6)
    with DecodeEngine(d, max_seqs=2, max_batch=8) as eng:
        s = eng.open_sequence(8)
        with pytest.raises(MmcError):
            eng.prompt_pass([s], [[shape.vocab_size]])  # token out of range
        with pytest.raises(MmcError):
            eng.prompt_pass([s, s], [[1], [2]])  # duplicate sequence
        with pytest.raises(MmcError):
            eng.prompt_pass([s], [[]])  # empty prompt
        assert eng.position(s) == 0
