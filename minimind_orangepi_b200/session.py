"""In-process text session on the CUDA decode engine.

The reference's Python wrapper (src/python/minimind_orangepi/session.py) runs
the minimind_generate CLI as a subprocess for every request and parses its
stdout. That wrapper still works unchanged against this repository's CLI
(pass ``executable=`` .../bin/minimind_generate). This module is the
in-process alternative: one ``DecodeEngine`` (weights loaded once, KV pages
reused across requests) serves every call, and streaming reads tokens from the
device loop as each step finishes instead of from a pipe.

The public methods and results match the reference wrapper's
(``generate_result``, ``stream_generate_result``,
``stream_generate_chat_result``, ``generate``; ``GenerationResult``), and
``raw_output`` is written in the CLI's line format (``prompt_tokens:``,
``token:`` while streaming, ``generated_tokens:``), so code that parses either
keeps working. The chat markers and line formats are interface and are kept
exactly; everything else is this module's own.
"""
from __future__ import annotations

from dataclasses import dataclass
from pathlib import Path
from typing import Callable, Iterator, Sequence

RUNTIME_FILES = ("minimind_runtime_config.txt", "weights.bin")

# MiniMind chat template pieces (the prompt format the models were trained on)
_USER = "<|im_start|>user\n{}<|im_end|>\n"
_ASSISTANT = "<|im_start|>assistant\n{}<|im_end|>\n"
_REPLY_OPEN = "<|im_start|>assistant\n"
_THINK_OPEN = "<think>\n"


@dataclass(frozen=True)
class GenerationResult:
    raw_output: str
    prompt_tokens: list[int]
    generated_tokens: list[int]
    generated_text: str | None = None

    def format(self) -> str:
        """The CLI's output, plus a ``generated_text:`` line when a tokenizer decoded it."""
        if self.generated_text is None:
            return self.raw_output
        return self.raw_output + f"generated_text: {self.generated_text}\n"


def chat_prompt(prompt: str, open_thinking: bool = False) -> str:
    """One user turn followed by the opening of the assistant's reply."""
    return _USER.format(prompt) + _REPLY_OPEN + (_THINK_OPEN if open_thinking else "")


def chat_prompt_from_history(history: Sequence[tuple[str, str | None]], open_thinking: bool = False) -> str:
    """A whole conversation; earlier replies are closed turns, the last turn
    opens the reply (with a thinking block when asked)."""
    if not history:
        raise ValueError("history cannot be empty")
    parts = []
    for user, reply in history:
        if not user.strip():
            raise ValueError("history contains an empty user message")
        parts.append(_USER.format(user))
        if reply:
            parts.append(_ASSISTANT.format(reply))
    parts.append(_REPLY_OPEN + (_THINK_OPEN if open_thinking else ""))
    return "".join(parts)


def validate_runtime_model_dir(model: Path | None) -> None:
    """None is accepted (the CLI's built-in model); a directory must hold the
    runtime config and weights."""
    if model is None:
        return
    model = Path(model)
    if not model.exists():
        raise FileNotFoundError(f"model directory does not exist: {model}")
    if not model.is_dir():
        raise NotADirectoryError(f"model path is not a directory: {model}")
    missing = [name for name in RUNTIME_FILES if not (model / name).is_file()]
    if missing:
        raise ValueError(f"invalid MiniMind text runtime model directory {model}; missing: {', '.join(missing)}")


def parse_token_values(value: str) -> list[int]:
    return [int(v) for v in value.split()]


def parse_token_line(output: str, label: str) -> list[int]:
    """Ids of the first ``label:`` line of CLI output."""
    prefix = label + ":"
    line = next((ln for ln in output.splitlines() if ln.startswith(prefix)), None)
    if line is None:
        raise ValueError(f"missing {label} in runtime output")
    return parse_token_values(line[len(prefix):])


def parse_stream_token_line(line: str) -> int:
    """The id of one streamed ``token: N`` line."""
    if not line.startswith("token:"):
        raise ValueError("missing token line")
    ids = parse_token_values(line[len("token:"):])
    if len(ids) != 1:
        raise ValueError("stream token line must contain exactly one token")
    return ids[0]


def _ids_line(label: str, ids: Sequence[int]) -> str:
    return label + ":" + "".join(f" {t}" for t in ids) + "\n"


class TextSession:
    """Greedy text generation on one GPU, in this process.

    ``model`` is a runtime model directory. ``engine`` (optional) is anything
    with the ``DecodeEngine`` methods used here (``generate_stream``,
    ``config``); by default a ``DecodeEngine`` is created on first use and kept
    for the session's lifetime. Prompts are tokenized with the model's
    ``tokenizer.json`` when it exists (``tokenizers`` package), otherwise as
    bytes folded into the vocabulary, as the CLI does.
    """

    def __init__(self, model: Path, device: int = 0, *, engine=None,
                 engine_factory: Callable[[Path, int], object] | None = None) -> None:
        self.model = Path(model)
        validate_runtime_model_dir(self.model)
        self.device = device
        self._engine = engine
        self._engine_factory = engine_factory
        self._tokenizer = None
        self._tokenizer_loaded = False

    # ------------------------------------------------------------ plumbing
    @property
    def engine(self):
        if self._engine is None:
            if self._engine_factory is not None:
                self._engine = self._engine_factory(self.model, self.device)
            else:
                from .engine import DecodeEngine
                self._engine = DecodeEngine(self.model, device=self.device, max_seqs=2, max_batch=1)
        return self._engine

    def close(self) -> None:
        if self._engine is not None and hasattr(self._engine, "close"):
            self._engine.close()
        self._engine = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    @property
    def tokenizer(self):
        if not self._tokenizer_loaded:
            self._tokenizer_loaded = True
            path = self.model / "tokenizer.json"
            if path.exists():
                try:
                    from tokenizers import Tokenizer
                except ImportError as exc:
                    raise RuntimeError("tokenizer.json requires the tokenizers package") from exc
                self._tokenizer = Tokenizer.from_file(str(path))
        return self._tokenizer

    def _prompt_ids(self, prompt: str, raw_prompt: bool, open_thinking: bool) -> list[int]:
        tok = self.tokenizer
        cfg = self.engine.config
        if tok is not None:
            ids = list(tok.encode(prompt if raw_prompt else chat_prompt(prompt, open_thinking)).ids)
        else:  # the CLI's byte fallback: the raw prompt text, folded into the vocabulary
            ids = [b % cfg.vocab_size for b in prompt.encode("utf-8")]
        return ids or [cfg.bos_token_id]

    def _result(self, lines: list[str], prompt_ids, generated) -> GenerationResult:
        text = self.tokenizer.decode(list(generated)) if self.tokenizer is not None else None
        return GenerationResult("".join(lines), list(prompt_ids), list(generated), text)

    # ------------------------------------------------------------ public API
    def stream_generate_result(self, prompt: str, max_new_tokens: int = 8, raw_prompt: bool = False,
                               open_thinking: bool = False) -> Iterator[GenerationResult]:
        """One result per generated token (its ``token:`` line appended), then
        the final result with the ``generated_tokens:`` line."""
        ids = self._prompt_ids(prompt, raw_prompt, open_thinking)
        lines = [_ids_line("prompt_tokens", ids)]
        generated: list[int] = []
        for t in self.engine.generate_stream(ids, max_new_tokens):
            generated.append(int(t))
            lines.append(f"token: {int(t)}\n")
            yield self._result(lines, ids, generated)
        lines.append(_ids_line("generated_tokens", generated))
        yield self._result(lines, ids, generated)

    def generate_result(self, prompt: str, max_new_tokens: int = 8, raw_prompt: bool = False,
                        open_thinking: bool = False) -> GenerationResult:
        ids = self._prompt_ids(prompt, raw_prompt, open_thinking)
        generated = [int(t) for t in self.engine.generate_stream(ids, max_new_tokens)]
        return self._result([_ids_line("prompt_tokens", ids), _ids_line("generated_tokens", generated)], ids,
                            generated)

    def stream_generate_chat_result(self, history: Sequence[tuple[str, str | None]], max_new_tokens: int = 8,
                                    open_thinking: bool = False) -> Iterator[GenerationResult]:
        yield from self.stream_generate_result(chat_prompt_from_history(history, open_thinking), max_new_tokens,
                                               raw_prompt=True)

    def generate(self, prompt: str, max_new_tokens: int = 8, raw_prompt: bool = False,
                 open_thinking: bool = False) -> str:
        return self.generate_result(prompt, max_new_tokens, raw_prompt, open_thinking).format()
