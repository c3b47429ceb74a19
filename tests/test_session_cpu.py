"""Python wrapper (TextSession) and CLI surface checks that need no GPU: the
same behaviour the reference's session tests pin, run against a stand-in
executable that prints the CLI's line format."""
from __future__ import annotations

import subprocess
import sys
from pathlib import Path

import pytest

from minimind_orangepi_b200.session import (GenerationResult, TextSession, chat_prompt, chat_prompt_from_history,
                                            parse_stream_token_line, parse_token_line, validate_runtime_model_dir)

ROOT = Path(__file__).resolve().parents[1]
CLI = ROOT / "minimind_orangepi_b200" / "bin" / "minimind_generate"


def test_parse_token_line():
    out = "prompt_tokens: 1 2\ngenerated_tokens: 3 4\n"
    assert parse_token_line(out, "prompt_tokens") == [1, 2]
    assert parse_token_line(out, "generated_tokens") == [3, 4]
    with pytest.raises(ValueError):
        parse_token_line(out, "missing")


def test_parse_stream_token_line():
    assert parse_stream_token_line("token: 42") == 42
    with pytest.raises(ValueError):
        parse_stream_token_line("generated_tokens: 42")
    with pytest.raises(ValueError):
        parse_stream_token_line("token: 1 2")


def test_generation_result_format():
    r = GenerationResult("prompt_tokens: 1\ngenerated_tokens: 2\n", [1], [2], "hello")
    assert r.format().endswith("generated_text: hello\n")
    assert GenerationResult("x\n", [], [], None).format() == "x\n"


def test_chat_prompts():
    assert chat_prompt("hi") == "<|im_start|>user\nhi<|im_end|>\n<|im_start|>assistant\n"
    assert chat_prompt("hi", open_thinking=True).endswith("assistant\n<think>\n")
    assert chat_prompt_from_history([("hi", "")]) == chat_prompt("hi")
    two = chat_prompt_from_history([("a", "b"), ("c", "")], open_thinking=True)
    assert two == ("<|im_start|>user\na<|im_end|>\n<|im_start|>assistant\nb<|im_end|>\n"
                   "<|im_start|>user\nc<|im_end|>\n<|im_start|>assistant\n<think>\n")
    with pytest.raises(ValueError, match="history cannot be empty"):
        chat_prompt_from_history([])


def test_validate_runtime_model_dir(tmp_path):
    validate_runtime_model_dir(None)
    with pytest.raises(FileNotFoundError):
        validate_runtime_model_dir(tmp_path / "missing")
    f = tmp_path / "file"
    f.write_text("x")
    with pytest.raises(NotADirectoryError):
        validate_runtime_model_dir(f)
    d = tmp_path / "m"
    d.mkdir()
    with pytest.raises(ValueError, match="minimind_runtime_config.txt"):
        validate_runtime_model_dir(d)
    (d / "minimind_runtime_config.txt").write_text("hidden_size=4\n")
    with pytest.raises(ValueError, match="weights.bin"):
        validate_runtime_model_dir(d)
    (d / "weights.bin").write_bytes(b"MMRTW001")
    validate_runtime_model_dir(d)


class FakeEngine:
    """Stands in for DecodeEngine: a deterministic greedy stream (no GPU)."""

    class config:
        vocab_size = 8
        bos_token_id = 1
        eos_token_id = 2

    def __init__(self):
        self.calls = []

    def generate_stream(self, prompt, max_new_tokens, eos=None):
        self.calls.append((list(prompt), max_new_tokens))
        for i in range(max_new_tokens):
            t = (prompt[-1] + 3 * i + 3) % 8
            yield t
            if t == self.config.eos_token_id:
                return


@pytest.fixture
def model_dir_stub(tmp_path):
    d = tmp_path / "model"
    d.mkdir()
    (d / "minimind_runtime_config.txt").write_text("hidden_size=64\n")
    (d / "weights.bin").write_bytes(b"MMRTW001")
    return d


def test_text_session_stream_matches_blocking(model_dir_stub):
    eng = FakeEngine()
    s = TextSession(model_dir_stub, engine=eng)
    streamed = list(s.stream_generate_result("hi", 3))
    blocking = s.generate_result("hi", 3)
    # byte fallback folded into the vocabulary, as the CLI does
    assert blocking.prompt_tokens == [ord("h") % 8, ord("i") % 8]
    assert len(streamed) == len(blocking.generated_tokens) + 1  # token lines + the final summary
    assert streamed[-1].generated_tokens == blocking.generated_tokens
    assert streamed[-1].prompt_tokens == blocking.prompt_tokens
    # raw output in the CLI's line format, parseable by the same helpers
    assert parse_token_line(blocking.raw_output, "generated_tokens") == blocking.generated_tokens
    assert [parse_stream_token_line(ln) for ln in streamed[-1].raw_output.splitlines() if ln.startswith("token:")] \
        == blocking.generated_tokens
    assert streamed[-1].format() == streamed[-1].raw_output  # no tokenizer -> no text line
    chat = list(s.stream_generate_chat_result([("hi", "hello"), ("who", "")], 2))
    assert chat[-1].generated_tokens and "generated_tokens" in chat[-1].raw_output
    # the chat prompt is passed raw (markers already applied)
    assert eng.calls[-1][0] == [b % 8 for b in chat_prompt_from_history([("hi", "hello"), ("who", "")]).encode()]


def test_text_session_stops_at_eos_and_empty_prompt(model_dir_stub):
    s = TextSession(model_dir_stub, engine=FakeEngine())
    r = s.generate_result("\x05", 10)  # 5 -> 0, 3, 6, 1, 4, 7, 2 (eos)
    assert r.generated_tokens[-1] == 2 and len(r.generated_tokens) < 10
    assert s.generate_result("", 1).prompt_tokens == [1]  # empty prompt -> bos


def test_text_session_requires_a_runtime_model(tmp_path):
    with pytest.raises(FileNotFoundError):
        TextSession(tmp_path / "missing")


@pytest.mark.skipif(not CLI.exists(), reason="CLI not built")
def test_cli_refuses_the_toy_model_without_cpu_fallback():
    """Without a model directory the CLI picks the reference's toy model
    (head_dim 2), which the CUDA kernels do not support: it must fail loudly,
    not compute on the CPU."""
    r = subprocess.run([str(CLI), "--tokens", "1,2", "--max-new-tokens", "4"], capture_output=True, text=True)
    assert r.returncode != 0
    assert "head_dim" in r.stderr
