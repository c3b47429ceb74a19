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


@pytest.fixture
def fake_cli(tmp_path):
    """A stand-in for minimind_generate with the same flags and output lines."""
    script = tmp_path / "fake_generate"
    script.write_text(f"""#!{sys.executable}
import sys
a = sys.argv[1:]
n = int(a[a.index('--max-new-tokens') + 1])
toks = [int(t) for t in a[a.index('--tokens') + 1].split(',')] if '--tokens' in a else [ord(c) for c in a[a.index('--prompt') + 1]]
print('prompt_tokens: ' + ' '.join(map(str, toks)), flush=True)
gen = [(toks[-1] + i + 1) % 8 for i in range(n)]
if '--stream' in a:
    for t in gen:
        print(f'token: {{t}}', flush=True)
print('generated_tokens: ' + ' '.join(map(str, gen)), flush=True)
""")
    script.chmod(0o755)
    return script


def test_text_session_stream_matches_blocking(fake_cli):
    s = TextSession(fake_cli, None)
    streamed = list(s.stream_generate_result("hi", 3))
    blocking = s.generate_result("hi", 3)
    assert len(streamed) == 4  # three token lines + the final summary line
    assert streamed[-1].generated_tokens == blocking.generated_tokens
    assert streamed[-1].prompt_tokens == blocking.prompt_tokens == [ord("h"), ord("i")]
    chat = list(s.stream_generate_chat_result([("hi", "hello"), ("who", "")], 2))
    assert chat[-1].generated_tokens and "generated_tokens" in chat[-1].raw_output


@pytest.mark.skipif(not CLI.exists(), reason="CLI not built")
def test_cli_refuses_the_toy_model_without_cpu_fallback():
    """Without a model directory the CLI picks the reference's toy model
    (head_dim 2), which the CUDA kernels do not support: it must fail loudly,
    not compute on the CPU."""
    r = subprocess.run([str(CLI), "--tokens", "1,2", "--max-new-tokens", "4"], capture_output=True, text=True)
    assert r.returncode != 0
    assert "head_dim" in r.stderr
