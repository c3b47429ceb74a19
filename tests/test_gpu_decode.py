"""Decode-step parity on the GPU: the CUDA path (through the C ABI) against the
reference's own outputs (golden fixtures made by the reference CPU path) and
against the live CPU oracle (oracle/liboracle.so, bit-identical to the
reference).

Tolerance: logits within 2e-2 absolute + 1e-2 relative of
the fp32 reference; greedy ids identical except at steps whose reference top-2
logit gap is below 2e-2. Both sides are fed the same tokens (the reference's),
so one near-tie does not desynchronise the rest of the run.
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
ROUTER_MARGIN = 1e-2  # relative top-1 vs top-2 router margin below which an fp16 path may pick the other expert


def close(a, b):
    return np.abs(a - b) <= ATOL + RTOL * np.abs(b)


def check_step(logits, ref_logits, ref_next, got_next, where):
    ok = close(logits, ref_logits)
    assert ok.all(), f"{where}: max |diff| {np.abs(logits - ref_logits).max():.3e}"
    srt = np.sort(ref_logits)
    if srt[-1] - srt[-2] >= ATOL:
        assert got_next == ref_next, f"{where}: token {got_next} != reference {ref_next}"
    # the kernel's argmax must be exactly the first maximum of its own logits
    assert got_next == int(np.argmax(logits)), f"{where}: argmax not the first maximum of the kernel's logits"


@pytest.mark.parametrize("name", ["tiny", "tiny-hd64", "tiny-hd96-page-cross", "cfg1-minimind2-small", "tiny-moe",
                                  "cfg2-minimind2-small-long", "cfg3-minimind2"])
def test_decode_matches_reference_golden(name, tmp_path_factory):
    g = np.load(GOLDEN / f"{name}.npz")
    shape = ModelShape(**json.loads(str(g["shape"])))
    d = write_runtime_model(Path("/tmp/mmc_test_models") / f"golden-{name}", shape, int(g["model_seed"]),
                            eps=float(g["eps"]), theta=float(g["theta"]))
    fed, argmax = g["fed"], g["argmax"]
    full = {int(s): g["full_logits"][i] for i, s in enumerate(g["full_steps"])}
    with DecodeEngine(d, max_seqs=2, max_batch=2) as eng:
        seq = eng.open_sequence(len(fed) + 1)
        for i, tok in enumerate(fed):
            nxt, logits = eng.step([seq], [int(tok)], want_logits=True)
            logits = logits[0]
            where = f"{name} step {i}"
            # top-16 of the reference at every step
            idx, val = g["topk_idx"][i], g["topk_val"][i]
            assert close(logits[idx], val).all(), f"{where}: top-k logits differ by {np.abs(logits[idx] - val).max():.3e}"
            if i in full:
                assert close(logits, full[i]).all(), f"{where}: max |diff| {np.abs(logits - full[i]).max():.3e}"
            if g["top2gap"][i] >= ATOL:
                assert int(nxt[0]) == int(argmax[i]), f"{where}: token {nxt[0]} != reference {argmax[i]}"
            assert int(nxt[0]) == int(np.argmax(logits))
        assert eng.position(seq) == len(fed)


def test_generate_matches_reference_golden():
    """Free-running greedy generation equals the reference's generate()."""
    g = np.load(GOLDEN / "cfg1-minimind2-small.npz")
    shape = ModelShape(**json.loads(str(g["shape"])))
    d = write_runtime_model(Path("/tmp/mmc_test_models") / "golden-cfg1-minimind2-small", shape,
                            int(g["model_seed"]), eps=float(g["eps"]), theta=float(g["theta"]))
    with DecodeEngine(d, max_seqs=2, max_batch=2) as eng:
        out = eng.generate([int(t) for t in g["prompt"]], len(g["generated"]))
    ref = [int(t) for t in g["generated"]]
    gaps = g["top2gap"][len(g["prompt"]) - 1:]
    for i, (a, b) in enumerate(zip(out, ref)):
        if a != b:
            assert gaps[i] < ATOL, f"step {i}: {a} != {b} with reference gap {gaps[i]}"
            break


@pytest.mark.parametrize("shape,plen,steps", [("tiny-hd64", 150, 60), ("minimind2-small", 100, 40),
                                              ("minimind2", 70, 20)])
def test_decode_matches_live_oracle(shape, plen, steps, model_dir):
    from oracle.oracle import Oracle

    d = model_dir(shape, seed=11)
    s = SHAPES[shape]
    orc = Oracle(d, eps=1e-5, theta=1e6)
    ost = orc.new_state()
    prompt = synthetic_prompt(21, plen, vocab=s.vocab_size)
    with DecodeEngine(d, max_seqs=2, max_batch=2) as eng:
        seq = eng.open_sequence(plen + steps)
        tok = prompt[0]
        for i in range(plen + steps - 1):
            ref_next, ref_logits = orc.forward_token(ost, tok)
            nxt, logits = eng.step([seq], [tok], want_logits=True)
            check_step(logits[0], ref_logits, ref_next, int(nxt[0]), f"{shape} step {i}")
            tok = prompt[i + 1] if i + 1 < plen else ref_next
        # the device KV cache holds the reference's normed+roped K and raw V (fp16)
        for layer in (0, s.num_hidden_layers - 1):
            k, v = eng.read_kv(seq, layer)
            assert k.shape[0] == plen + steps - 1


@pytest.mark.parametrize("shape,batch,steps", [("tiny-moe", 3, 20), ("tiny-moe", 37, 16), ("tiny-moe", 260, 4),
                                              ("tiny-hd64", 3, 30), ("tiny-hd64", 37, 24),
                                               ("minimind2-small", 8, 12), ("tiny-hd96", 70, 12),
                                               ("minimind2", 20, 4)])
def test_batched_decode_matches_oracle(shape, batch, steps, model_dir):
    """Independent sequences with different prompt lengths decode together;
    each row must match its own single-sequence reference run."""
    from oracle.oracle import Oracle

    d = model_dir(shape, seed=5)
    s = SHAPES[shape]
    orc = Oracle(d, eps=1e-5, theta=1e6)
    rng = np.random.default_rng(batch)
    plens = [int(x) for x in rng.integers(1, 90, size=batch)]
    prompts = [synthetic_prompt(100 + i, n, vocab=s.vocab_size) for i, n in enumerate(plens)]
    states = [orc.new_state() for _ in range(batch)]
    diverged: set[int] = set()
    checked = total = 0
    with DecodeEngine(d, max_seqs=batch + 4, max_batch=batch) as eng:
        seqs = [eng.open_sequence(plens[i] + steps + 1) for i in range(batch)]
        cur = [p[0] for p in prompts]
        fed = [0] * batch
        for step in range(max(plens) + steps):
            rows = [i for i in range(batch) if fed[i] < plens[i] + steps]
            if not rows:
                break
            nxt, logits = eng.step([seqs[i] for i in rows], [cur[i] for i in rows], want_logits=True)
            for j, i in enumerate(rows):
                ref_next, ref_logits = orc.forward_token(states[i], cur[i])
                # MoE: once the reference's router top-2 margin is this small, fp16
                # rounding may route the token to the other expert and the sequence
                # legitimately diverges; it is compared up to that point only
                if orc.router_margin() < ROUTER_MARGIN:
                    diverged.add(i)
                total += 1
                if i not in diverged:
                    checked += 1
                    check_step(logits[j], ref_logits, ref_next, int(nxt[j]), f"{shape} B={batch} row {i} step {fed[i]}")
                fed[i] += 1
                cur[i] = prompts[i][fed[i]] if fed[i] < plens[i] else ref_next
        for i in range(batch):
            assert eng.position(seqs[i]) == fed[i]
        assert checked >= 0.5 * total, f"only {checked} of {total} steps compared (router near-ties)"


@pytest.mark.parametrize("shape,batch", [("minimind2-small", 1), ("tiny-hd96", 16), ("tiny-moe", 16)])
def test_graph_loop_matches_stepwise(shape, batch, model_dir):
    """The captured device-resident loop produces the same tokens as eager steps."""
    d = model_dir(shape, seed=3)
    s = SHAPES[shape]
    n = 40
    prompts = [synthetic_prompt(300 + i, 5 + 3 * i, vocab=s.vocab_size) for i in range(batch)]
    with DecodeEngine(d, max_seqs=2 * batch, max_batch=batch) as eng:
        a = [eng.open_sequence(len(p) + n + 1) for p in prompts]
        b = [eng.open_sequence(len(p) + n + 1) for p in prompts]
        first_a = eng.prefill(a, prompts)
        first_b = eng.prefill(b, prompts)
        assert (first_a == first_b).all()
        eager = []
        cur = first_a.copy()
        for _ in range(n):
            cur, _ = eng.step(a, cur)
            eager.append(cur.copy())
        eng.graph_build(b)
        eng.graph_set_tokens(first_b)
        eng.graph_run(n)
        graph = eng.graph_tokens(n)
        assert np.array_equal(np.stack(eager), graph)
        assert all(eng.position(x) == eng.position(y) for x, y in zip(a, b))


def test_errors_are_reported(model_dir):
    d = model_dir("tiny", seed=1)
    with DecodeEngine(d, max_seqs=2, max_batch=2, n_pages=2) as eng:
        seq = eng.open_sequence(64)
        with pytest.raises(MmcError) as e:
            eng.step([seq], [10_000])
        assert e.value.code == 2  # out of range, nothing ran
        assert eng.position(seq) == 0
        with pytest.raises(MmcError) as e:
            eng.step([seq, seq], [1, 2])
        assert e.value.code == 1
        other = eng.open_sequence(64)
        with pytest.raises(MmcError) as e:  # pool has 2 pages, both reserved
            eng.reserve(seq, 65)
        assert e.value.code == 4
        eng.close_sequence(other)
        eng.reserve(seq, 65)
        nxt, _ = eng.step([seq], [1])
        assert 0 <= int(nxt[0]) < 256


def test_configure_moe_validation():
    """mmc_configure_moe: only before loading, sane sizes only."""
    import ctypes as C

    from minimind_orangepi_b200._lib import lib
    from minimind_orangepi_b200.engine import ModelDesc

    s = SHAPES["tiny-moe"]
    desc = ModelDesc(s.hidden_size, s.num_hidden_layers, s.num_attention_heads, s.num_key_value_heads, s.head_dim,
                     s.intermediate_size, s.vocab_size, s.max_position_embeddings, 1e-5, 1e6)
    h = C.c_void_p()
    assert lib().mmc_create(C.byref(desc), 0, C.byref(h)) == 0
    try:
        assert lib().mmc_configure_moe(h, 0, 256) == 1  # MMC_ERR_INVALID
        assert lib().mmc_configure_moe(h, 4, 100) == 1  # not a multiple of 64
        d = write_runtime_model(Path("/tmp/mmc_test_models") / "cfg-tiny-moe", "tiny-moe", 2, eps=1e-5, theta=1e6)
        # a dense context cannot read a MoE weights.bin (tensor names differ)
        assert lib().mmc_load_weights_file(h, str(d / "weights.bin").encode()) != 0
        assert lib().mmc_configure_moe(h, 4, 256) == 0
        assert lib().mmc_load_weights_file(h, str(d / "weights.bin").encode()) == 0
        assert lib().mmc_configure_moe(h, 4, 256) == 6  # MMC_ERR_STATE after loading
    finally:
        lib().mmc_destroy(h)
