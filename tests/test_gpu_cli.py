"""The drop-in surface on the GPU: the minimind_generate / bench_decode CLIs
(C++ LanguageModel over the C ABI), DecodeEngine streaming and the in-process
TextSession, on a seeded
MiniMind2-small model, against the reference's own greedy output (golden
fixture made by the reference CPU path)."""
from __future__ import annotations

import json
import subprocess
from pathlib import Path

import numpy as np
import pytest

from minimind_orangepi_b200.session import TextSession
from minimind_orangepi_b200.synthetic import ModelShape, write_runtime_model

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]
BIN = ROOT / "minimind_orangepi_b200" / "bin"
G = np.load(ROOT / "tests" / "golden" / "cfg1-minimind2-small.npz")


@pytest.fixture(scope="module")
def model():
    shape = ModelShape(**json.loads(str(G["shape"])))
    return write_runtime_model(Path("/tmp/mmc_test_models") / "golden-cfg1-minimind2-small", shape,
                               int(G["model_seed"]), eps=float(G["eps"]), theta=float(G["theta"]))


def _expected():
    ref = [int(t) for t in G["generated"]]
    gaps = G["top2gap"][len(G["prompt"]) - 1:]
    return ref, gaps


def _same_until_near_tie(got, ref, gaps):
    for i, (a, b) in enumerate(zip(got, ref)):
        if a != b:
            assert gaps[i] < 2e-2, f"step {i}: {a} != {b} (reference top-2 gap {gaps[i]})"
            return
    assert len(got) == len(ref)


def test_cli_generate_matches_reference(model):
    prompt = ",".join(str(int(t)) for t in G["prompt"])
    out = subprocess.run([str(BIN / "minimind_generate"), "--model", str(model), "--tokens", prompt,
                          "--max-new-tokens", str(len(G["generated"]))], capture_output=True, text=True, check=True).stdout
    lines = out.splitlines()
    assert lines[0] == "prompt_tokens: " + " ".join(str(int(t)) for t in G["prompt"])
    got = [int(t) for t in lines[-1].split(":", 1)[1].split()]
    _same_until_near_tie(got, *_expected())


@pytest.mark.parametrize("new_tokens", [6, 40])
def test_cli_stream_equals_blocking(model, new_tokens):
    """--stream prints one token: line per token; 40 tokens run on the streamed
    graph loop (6 on eager steps). Both must equal the blocking output."""
    cmd = [str(BIN / "minimind_generate"), "--model", str(model), "--tokens", "5,6,7", "--max-new-tokens",
           str(new_tokens)]
    out = subprocess.run(cmd + ["--stream"], capture_output=True, text=True, check=True).stdout
    blocking = subprocess.run(cmd, capture_output=True, text=True, check=True).stdout
    toks = [int(l.split()[1]) for l in out.splitlines() if l.startswith("token:")]
    final = [l for l in out.splitlines() if l.startswith("generated_tokens:")][0]
    assert toks == [int(t) for t in final.split(":", 1)[1].split()]
    assert len(toks) <= new_tokens
    assert final == blocking.splitlines()[-1]


def test_engine_stream_matches_reference(model):
    """DecodeEngine.generate_stream (prompt pass + streamed graph loop) yields
    the reference's greedy tokens, one at a time."""
    from minimind_orangepi_b200 import DecodeEngine

    with DecodeEngine(model, max_seqs=2, max_batch=1) as eng:
        got = list(eng.generate_stream([int(t) for t in G["prompt"]], len(G["generated"]), eos=-1))
        again = eng.generate([int(t) for t in G["prompt"]], len(G["generated"]), eos=-1)
    assert got == again
    _same_until_near_tie(got, *_expected())


@pytest.mark.parametrize("batch", [1, 8])
def test_bench_decode_reports_the_reference_keys(model, batch):
    out = subprocess.run([str(BIN / "bench_decode"), "--model", str(model), "--input-tokens", "5,6,7,8,9",
                          "--tokens", "16", "--warmup", "1", "--batch", str(batch)],
                         capture_output=True, text=True, check=True).stdout
    kv = dict(l.split("=", 1) for l in out.splitlines())
    for k in ("prompt_tokens", "generated_tokens", "prefill_tokens", "prefill_seconds", "prefill_tokens_per_second",
              "decode_steps", "decode_seconds", "decode_tokens_per_second"):
        assert k in kv
    assert kv["decode_steps"] == "15" and float(kv["decode_tokens_per_second"]) > 0


def test_text_session_in_process(model):
    """The in-process session: streamed results end with the blocking result."""
    with TextSession(model) as s:
        blocking = s.generate_result("hello", 12)
        streamed = list(s.stream_generate_result("hello", 12))
    assert streamed[-1].generated_tokens == blocking.generated_tokens
    assert streamed[-1].raw_output.endswith(blocking.raw_output.splitlines()[-1] + "\n")
    assert blocking.prompt_tokens == [ord(c) for c in "hello"]
