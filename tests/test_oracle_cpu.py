"""CPU-only checks: the oracle is pinned to the reference, the runtime format
writer is byte-identical to the reference exporter, and the C ABI library
loads and exports everything include/minimind_cuda.h declares."""
from __future__ import annotations

import ctypes as C
import json
import os
import re
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

from minimind_orangepi_b200.synthetic import ModelShape, synthetic_tensors, write_runtime_model, write_weights, \
    write_runtime_config
from oracle.oracle import Oracle, ReferenceModel, ref_available, REF_CLI

ROOT = Path(__file__).resolve().parents[1]
GOLDEN = ROOT / "tests" / "golden"
# the reference checkout: MINIMIND_REFERENCE_ROOT, else a `reference` directory
# beside this repository's own directory (as the build looks for it)
REFERENCE = Path(os.environ["MINIMIND_REFERENCE_ROOT"]) if os.environ.get("MINIMIND_REFERENCE_ROOT") else \
    ROOT.parent / "reference"
GOLDEN_CASES = ["tiny", "tiny-hd64", "tiny-hd96-page-cross", "cfg1-minimind2-small", "tiny-moe"]


def golden_model(name, tmp_root):
    g = np.load(GOLDEN / f"{name}.npz")
    shape = ModelShape(**json.loads(str(g["shape"])))
    d = write_runtime_model(tmp_root / f"golden-{name}", shape, int(g["model_seed"]), eps=float(g["eps"]),
                            theta=float(g["theta"]))
    return g, d


@pytest.mark.parametrize("name", GOLDEN_CASES)
def test_oracle_reproduces_reference_golden_bit_exact(name, tmp_path_factory):
    """The C restatement gives exactly the reference's fp32 logits."""
    g, d = golden_model(name, Path("/tmp/mmc_test_models"))
    orc = Oracle(d, eps=float(g["eps"]), theta=float(g["theta"]))
    st = orc.new_state()
    full = {int(s): g["full_logits"][i] for i, s in enumerate(g["full_steps"])}
    for i, tok in enumerate(g["fed"]):
        nxt, logits = orc.forward_token(st, int(tok))
        assert nxt == int(g["argmax"][i])
        assert np.array_equal(logits[g["topk_idx"][i]], g["topk_val"][i])
        if i in full:
            assert np.array_equal(logits, full[i])
    assert orc.generate([int(t) for t in g["prompt"]], len(g["generated"])) == [int(t) for t in g["generated"]]


def toy_model_dir(root: Path) -> Path:
    """The reference's make_toy_language_model (language_model.cpp:415-470) in
    runtime format: hidden 4, 1 layer, 2/1 heads, head_dim 2, vocab 8, theta 1e4."""
    s = ModelShape(4, 1, 2, 1, 2, 8, vocab_size=8, max_position_embeddings=16)
    eye = lambda r, c: np.eye(r, c, dtype=np.float32)  # noqa: E731
    embed = np.array([[0, 0, 0, 0], [1, 0, 0, 0], [0, 1, 0, 0], [0, 0, 1, 0], [0, 0, 0, 1], [1, 1, 0, 0],
                      [0, 1, 1, 0], [0, 0, 1, 1]], np.float32)
    lm = np.array([[0, 0, 0, 0], [.2, 0, 0, 0], [0, .2, 0, 0], [0, 0, .2, 0], [0, 0, 0, .2], [2, .1, 0, 0],
                   [0, 2, .1, 0], [0, 0, 2, .1]], np.float32)
    p = "model.layers.0."
    t = {"model.embed_tokens.weight": embed, "model.norm.weight": np.ones(4, np.float32), "lm_head.weight": lm,
         p + "input_layernorm.weight": np.ones(4, np.float32),
         p + "post_attention_layernorm.weight": np.ones(4, np.float32),
         p + "self_attn.q_norm.weight": np.ones(2, np.float32), p + "self_attn.k_norm.weight": np.ones(2, np.float32),
         p + "self_attn.q_proj.weight": eye(4, 4), p + "self_attn.k_proj.weight": eye(2, 4),
         p + "self_attn.v_proj.weight": eye(2, 4), p + "self_attn.o_proj.weight": eye(4, 4),
         p + "mlp.gate_proj.weight": eye(8, 4), p + "mlp.up_proj.weight": eye(8, 4),
         p + "mlp.down_proj.weight": eye(4, 8)}
    root.mkdir(parents=True, exist_ok=True)
    write_runtime_config(s, root, None, None)
    write_weights(s, t, root)
    return root


def test_oracle_toy_known_answer(tmp_path):
    """Known answer of the reference CLI: --tokens 1,2 --max-new-tokens 4 -> 6 6 6 6."""
    golden = (GOLDEN / "toy_cli.txt").read_text()
    assert "generated_tokens: 6 6 6 6" in golden
    orc = Oracle(toy_model_dir(tmp_path / "toy"), eps=1e-6, theta=1e4)
    assert orc.generate([1, 2], 4) == [6, 6, 6, 6]


def test_oracle_rejects_out_of_vocab(model_dir):
    orc = Oracle(model_dir("tiny"))
    with pytest.raises(IndexError):
        orc.forward_token(orc.new_state(), 256)


@pytest.mark.skipif(not ref_available(), reason="oracle/_ref not built (reference sources absent)")
@pytest.mark.parametrize("shape,steps", [("tiny", 40), ("tiny-hd96", 70)])
def test_oracle_bit_exact_with_reference_live(shape, steps, model_dir):
    from minimind_orangepi_b200.synthetic import SHAPES, synthetic_prompt
    d = model_dir(shape, seed=9)
    v = SHAPES[shape].vocab_size
    orc, ref = Oracle(d), ReferenceModel(d)
    so, sr = orc.new_state(), ref.new_state()
    for tok in synthetic_prompt(4, steps, vocab=v):
        a, la = orc.forward_token(so, tok)
        b, lb = ref.forward_token(sr, tok, v)
        assert a == b and np.array_equal(la, lb)


@pytest.mark.skipif(not REF_CLI.exists(), reason="oracle/_ref not built")
def test_reference_cli_toy_answer():
    out = subprocess.run([str(REF_CLI), "--tokens", "1,2", "--max-new-tokens", "4"], capture_output=True, text=True,
                         check=True).stdout
    assert out == (GOLDEN / "toy_cli.txt").read_text()


@pytest.mark.skipif(not (REFERENCE / "src/python/tools/export_minimind_runtime.py").exists(),
                    reason="reference exporter not present")
def test_runtime_format_matches_reference_exporter(tmp_path):
    from safetensors.numpy import save_file
    s = ModelShape(64, 2, 4, 2, 16, 128, vocab_size=256, max_position_embeddings=4096)
    tensors = synthetic_tensors(s, seed=3)
    ckpt = tmp_path / "ckpt"
    ckpt.mkdir()
    (ckpt / "config.json").write_text(json.dumps({
        "hidden_size": s.hidden_size, "num_hidden_layers": s.num_hidden_layers, "vocab_size": s.vocab_size,
        "num_attention_heads": s.num_attention_heads, "num_key_value_heads": s.num_key_value_heads,
        "head_dim": s.head_dim, "intermediate_size": s.intermediate_size,
        "max_position_embeddings": s.max_position_embeddings, "tie_word_embeddings": True, "use_moe": False}))
    save_file({k: v for k, v in tensors.items() if k != "lm_head.weight"}, str(ckpt / "model.safetensors"))
    tools = REFERENCE / "src/python/tools"
    subprocess.run([sys.executable, str(tools / "export_minimind_runtime.py"), "--model", str(ckpt), "--output",
                    str(tmp_path / "ref_out")], check=True, capture_output=True, env={**os.environ, "PYTHONPATH": str(tools)})
    ours = tmp_path / "ours"
    ours.mkdir()
    write_runtime_config(s, ours, None, None)
    write_weights(s, tensors, ours)
    for f in ("minimind_runtime_config.txt", "weights.bin"):
        assert (ours / f).read_bytes() == (tmp_path / "ref_out" / f).read_bytes(), f


def test_cuda_library_exports_every_declared_symbol():
    from minimind_orangepi_b200._lib import EXPORTS, LIB_PATH
    header = (ROOT / "include" / "minimind_cuda.h").read_text()
    declared = set(re.findall(r"MMC_EXPORT\s+[\w\s\*]+?\b(mmc_\w+)\s*\(", header))
    assert declared, "no declarations parsed"
    assert declared == set(EXPORTS), declared ^ set(EXPORTS)
    L = C.CDLL(str(LIB_PATH))  # loads without a GPU: no device work at load time
    for name in sorted(declared):
        assert hasattr(L, name), name
    L.mmc_abi_version.restype = C.c_int
    assert L.mmc_abi_version() == 1
    L.mmc_kv_row_offset.restype = C.c_int64
    L.mmc_kv_row_offset.argtypes = [C.c_int32] * 3
    # swizzled rows: each row is a permutation of its own 16-byte chunks
    for hd in (16, 32, 64, 96, 128):
        for r in range(64):
            offs = sorted(L.mmc_kv_row_offset(hd, r, c) for c in range(hd // 8))
            assert offs == [r * hd + 8 * c for c in range(hd // 8)]


def test_cuda_library_refuses_without_gpu_or_bad_shape():
    """Creating a context validates the shape before touching a device."""
    from minimind_orangepi_b200._lib import MmcError, ModelDesc, check, lib
    L = lib()
    bad = ModelDesc(100, 2, 4, 2, 25, 128, 256, 4096, 1e-5, 1e6)
    h = C.c_void_p()
    code = L.mmc_create(C.byref(bad), 0, C.byref(h))
    assert code == 1 and b"head_dim" in L.mmc_last_error()
    with pytest.raises(MmcError):
        check(code)
