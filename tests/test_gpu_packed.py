"""Packed-weight cache (mmc_save_packed / mmc_load_packed) on the GPU: a
context filled from the cache decodes bit-identically to one loaded from
weights.bin; caches of another model, truncated or corrupt files are refused
and leave the context usable for a normal load."""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

from minimind_orangepi_b200 import DecodeEngine, MmcError
import ctypes as C

from minimind_orangepi_b200._lib import lib
from minimind_orangepi_b200.engine import ModelDesc
from minimind_orangepi_b200.synthetic import SHAPES, synthetic_prompt, write_runtime_model

pytestmark = pytest.mark.gpu


def run(eng, prompt, steps=6):
    seq = eng.open_sequence(len(prompt) + steps + 1)
    nxt = int(eng.prompt_pass([seq], [prompt])[0])
    out = []
    for _ in range(steps):
        t, logits = eng.step([seq], [nxt], want_logits=True)
        out.append(logits[0])
        nxt = int(t[0])
    return np.stack(out)


def test_packed_cache_round_trip(tmp_path):
    shape = SHAPES["minimind2-small"]
    d = write_runtime_model(Path("/tmp/mmc_test_models") / "packed-small", shape, 3, eps=1e-5, theta=1e6)
    cache = tmp_path / "w.mmcpk"
    prompt = synthetic_prompt(4, 40, shape.vocab_size)
    with DecodeEngine(d, max_seqs=2, max_batch=8, packed_cache=cache) as a:
        assert a.loaded_from == "weights.bin" and cache.exists()
        ref = run(a, prompt)
    with DecodeEngine(d, max_seqs=2, max_batch=8, packed_cache=cache) as b:
        assert b.loaded_from == "packed"
        got = run(b, prompt)
    assert np.array_equal(ref, got)


def test_packed_cache_rejects_other_model_and_truncation(tmp_path):
    small = SHAPES["minimind2-small"]
    d1 = write_runtime_model(Path("/tmp/mmc_test_models") / "packed-small", small, 3, eps=1e-5, theta=1e6)
    cache = tmp_path / "w.mmcpk"
    with DecodeEngine(d1, max_seqs=2, max_batch=8) as a:
        a.save_packed(cache)
    # an unloaded context of another model refuses the file and stays unloaded
    t = SHAPES["tiny-hd64"]
    desc = ModelDesc(t.hidden_size, t.num_hidden_layers, t.num_attention_heads, t.num_key_value_heads, t.head_dim,
                     t.intermediate_size, t.vocab_size, t.max_position_embeddings, 1e-5, 1e6)
    h = C.c_void_p()
    assert lib().mmc_create(C.byref(desc), 0, C.byref(h)) == 0
    try:
        assert lib().mmc_load_packed(h, str(cache).encode()) == 1  # MMC_ERR_INVALID
        d2 = write_runtime_model(Path("/tmp/mmc_test_models") / "packed-tiny", t, 3, eps=1e-5, theta=1e6)
        assert lib().mmc_load_weights_file(h, str(d2 / "weights.bin").encode()) == 0
    finally:
        lib().mmc_destroy(h)
    short = tmp_path / "short.mmcpk"
    short.write_bytes(cache.read_bytes()[: cache.stat().st_size // 2])
    # a stale or broken cache falls back to weights.bin and is rewritten
    with DecodeEngine(d1, max_seqs=2, max_batch=8, packed_cache=short) as f:
        assert f.loaded_from == "weights.bin"
    with DecodeEngine(d1, max_seqs=2, max_batch=8, packed_cache=short) as g:
        assert g.loaded_from == "packed"
