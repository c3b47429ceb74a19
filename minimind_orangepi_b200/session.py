"""Python text session over the minimind_generate CLI.

Same API as the reference wrapper (src/python/minimind_orangepi/session.py:
TextSession, GenerationResult, chat prompt builders, line parsers). The
process boundary is unchanged: the session runs the CLI and parses its
``prompt_tokens:`` / ``token:`` / ``generated_tokens:`` lines. The default
executable is this package's CUDA build (``bin/minimind_generate``).
"""
from __future__ import annotations

import subprocess
from dataclasses import dataclass
from pathlib import Path
from typing import Iterator, Sequence

DEFAULT_EXECUTABLE = Path(__file__).resolve().parent / "bin" / "minimind_generate"
RUNTIME_FILES = ("minimind_runtime_config.txt", "weights.bin")


@dataclass(frozen=True)
class GenerationResult:
    raw_output: str
    prompt_tokens: list[int]
    generated_tokens: list[int]
    generated_text: str | None = None

    def format(self) -> str:
        if self.generated_text is None:
            return self.raw_output
        return f"{self.raw_output}generated_text: {self.generated_text}\n"


def _user(text: str) -> str:
    return f"<|im_start|>user\n{text}<|im_end|>\n"


def _assistant_open(open_thinking: bool) -> str:
    return "<|im_start|>assistant\n<think>\n" if open_thinking else "<|im_start|>assistant\n"


def chat_prompt(prompt: str, open_thinking: bool = False) -> str:
    """MiniMind chat markers around one user turn, ready for the reply."""
    return _user(prompt) + _assistant_open(open_thinking)


def chat_prompt_from_history(history: Sequence[tuple[str, str | None]], open_thinking: bool = False) -> str:
    """Markers for a whole conversation; thinking mode applies to the last turn only."""
    if not history:
        raise ValueError("history cannot be empty")
    out = []
    last = len(history) - 1
    for i, (user, reply) in enumerate(history):
        if not user.strip():
            raise ValueError("history contains an empty user message")
        out.append(_user(user))
        if reply:
            out.append(f"<|im_start|>assistant\n{reply}<|im_end|>\n")
        if i == last:
            out.append(_assistant_open(open_thinking))
    return "".join(out)


def validate_runtime_model_dir(model: Path | None) -> None:
    """None means the CLI's built-in toy model; otherwise the directory must hold
    the runtime config and weights."""
    if model is None:
        return
    if not model.exists():
        raise FileNotFoundError(f"model directory does not exist: {model}")
    if not model.is_dir():
        raise NotADirectoryError(f"model path is not a directory: {model}")
    missing = [f for f in RUNTIME_FILES if not (model / f).exists()]
    if missing:
        raise ValueError(f"invalid MiniMind text runtime model directory {model}; missing: {', '.join(missing)}")


def parse_token_values(value: str) -> list[int]:
    return [int(v) for v in value.split()]


def parse_token_line(output: str, label: str) -> list[int]:
    for line in output.splitlines():
        if line.startswith(label + ":"):
            return parse_token_values(line.split(":", 1)[1])
    raise ValueError(f"missing {label} in runtime output")


def parse_stream_token_line(line: str) -> int:
    if not line.startswith("token:"):
        raise ValueError("missing token line")
    values = parse_token_values(line.split(":", 1)[1])
    if len(values) != 1:
        raise ValueError("stream token line must contain exactly one token")
    return values[0]


class TextSession:
    def __init__(self, executable: Path | None = None, model: Path | None = None) -> None:
        self.executable = Path(executable) if executable is not None else DEFAULT_EXECUTABLE
        self.model = Path(model) if model is not None else None

    def _load_tokenizer(self):
        if self.model is None or not (self.model / "tokenizer.json").exists():
            return None
        try:
            from tokenizers import Tokenizer
        except ImportError as exc:
            raise RuntimeError("tokenizer.json requires the tokenizers package") from exc
        return Tokenizer.from_file(str(self.model / "tokenizer.json"))

    def _command(self, prompt: str, max_new_tokens: int, raw_prompt: bool, open_thinking: bool, stream: bool):
        cmd = [str(self.executable), "--max-new-tokens", str(max_new_tokens)]
        if stream:
            cmd.append("--stream")
        if self.model is not None:
            cmd += ["--model", str(self.model)]
        tokenizer = self._load_tokenizer()
        if tokenizer is None:
            cmd += ["--prompt", prompt]
        else:
            text = prompt if raw_prompt else chat_prompt(prompt, open_thinking)
            cmd += ["--tokens", ",".join(str(t) for t in tokenizer.encode(text).ids)]
        return cmd, tokenizer

    @staticmethod
    def _result(raw: str, prompt_tokens, generated, tokenizer) -> GenerationResult:
        text = tokenizer.decode(generated) if tokenizer is not None else None
        return GenerationResult(raw, list(prompt_tokens), list(generated), text)

    def generate_result(self, prompt: str, max_new_tokens: int = 8, raw_prompt: bool = False,
                        open_thinking: bool = False) -> GenerationResult:
        cmd, tokenizer = self._command(prompt, max_new_tokens, raw_prompt, open_thinking, False)
        out = subprocess.run(cmd, check=True, capture_output=True, text=True).stdout
        return self._result(out, parse_token_line(out, "prompt_tokens"), parse_token_line(out, "generated_tokens"),
                            tokenizer)

    def stream_generate_result(self, prompt: str, max_new_tokens: int = 8, raw_prompt: bool = False,
                               open_thinking: bool = False) -> Iterator[GenerationResult]:
        cmd, tokenizer = self._command(prompt, max_new_tokens, raw_prompt, open_thinking, True)
        proc = subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.PIPE, text=True, bufsize=1)
        assert proc.stdout is not None
        raw: list[str] = []
        prompt_tokens: list[int] = []
        generated: list[int] = []
        try:
            for line in proc.stdout:
                raw.append(line)
                s = line.strip()
                if s.startswith("prompt_tokens:"):
                    prompt_tokens = parse_token_values(s.split(":", 1)[1])
                elif s.startswith("token:"):
                    generated.append(parse_stream_token_line(s))
                    yield self._result("".join(raw), prompt_tokens, generated, tokenizer)
                elif s.startswith("generated_tokens:"):
                    generated = parse_token_values(s.split(":", 1)[1])
                    yield self._result("".join(raw), prompt_tokens, generated, tokenizer)
            err = proc.stderr.read() if proc.stderr is not None else ""
            rc = proc.wait()
        except Exception:
            proc.kill()
            proc.wait()
            raise
        if rc != 0:
            raise subprocess.CalledProcessError(rc, cmd, output="".join(raw), stderr=err)

    def stream_generate_chat_result(self, history: Sequence[tuple[str, str | None]], max_new_tokens: int = 8,
                                    open_thinking: bool = False) -> Iterator[GenerationResult]:
        yield from self.stream_generate_result(chat_prompt_from_history(history, open_thinking), max_new_tokens,
                                               True, False)

    def generate(self, prompt: str, max_new_tokens: int = 8, raw_prompt: bool = False,
                 open_thinking: bool = False) -> str:
        return self.generate_result(prompt, max_new_tokens, raw_prompt, open_thinking).format()
