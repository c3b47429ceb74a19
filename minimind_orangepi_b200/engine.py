"""Python face of the decode engine: one CUDA context per GPU.

``DecodeEngine`` wraps the C ABI the same way the C++ runtime does
(csrc/runtime/language_model.cpp): load a runtime model directory
(``minimind_runtime_config.txt`` + ``weights.bin``), open sequences (the device
side of ``DecoderState``), and run greedy decode steps for any batch of them.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass
from pathlib import Path

import numpy as np

from ._lib import ModelDesc, check, lib

DEFAULT_EPS = 1e-6      # MiniMindConfig::rms_norm_eps (config.h:36)
DEFAULT_THETA = 1e6     # MiniMindConfig::rope_theta (config.h:37)


@dataclass
class RuntimeConfig:
    hidden_size: int = 768
    num_hidden_layers: int = 8
    use_moe: bool = False
    vocab_size: int = 6400
    num_attention_heads: int = 8
    num_key_value_heads: int = 4
    head_dim: int = 96
    intermediate_size: int = 2432
    max_position_embeddings: int = 32768
    tie_word_embeddings: bool = True
    num_experts: int = 4
    moe_intermediate_size: int = 0  # 0: intermediate_size
    rms_norm_eps: float = DEFAULT_EPS
    rope_theta: float = DEFAULT_THETA
    bos_token_id: int = 1
    eos_token_id: int = 2


def read_runtime_config(model_dir) -> RuntimeConfig:
    """Same keys and fallbacks as config_from_file (runtime_loader.cpp:71-88), plus
    the optional rms_norm_eps / rope_theta keys."""
    path = Path(model_dir) / "minimind_runtime_config.txt"
    values: dict[str, str] = {}
    for raw in path.read_text().splitlines():
        line = raw.strip()
        if not line or line.startswith("#"):
            continue
        if "=" not in line:
            raise ValueError(f"invalid runtime config line: {line}")
        k, v = line.split("=", 1)
        values[k.strip()] = v.strip()
    c = RuntimeConfig()
    gi = lambda k, d: int(values[k]) if k in values else d  # noqa: E731
    gb = lambda k, d: values[k] in ("1", "true", "True") if k in values else d  # noqa: E731
    c.hidden_size = gi("hidden_size", c.hidden_size)
    c.num_hidden_layers = gi("num_hidden_layers", c.num_hidden_layers)
    c.use_moe = gb("use_moe", False)
    c.vocab_size = gi("vocab_size", c.vocab_size)
    c.num_attention_heads = gi("num_attention_heads", c.num_attention_heads)
    c.num_key_value_heads = gi("num_key_value_heads", c.num_key_value_heads)
    c.head_dim = gi("head_dim", c.hidden_size // c.num_attention_heads)
    c.intermediate_size = gi("intermediate_size", c.intermediate_size)
    c.max_position_embeddings = gi("max_position_embeddings", c.max_position_embeddings)
    c.tie_word_embeddings = gb("tie_word_embeddings", c.tie_word_embeddings)
    c.num_experts = gi("num_experts", c.num_experts)
    c.moe_intermediate_size = gi("moe_intermediate_size", c.intermediate_size)
    if "rms_norm_eps" in values:
        c.rms_norm_eps = float(values["rms_norm_eps"])
    if "rope_theta" in values:
        c.rope_theta = float(values["rope_theta"])
    return c


def _i32(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.int32))


class DecodeEngine:
    def __init__(self, model_dir, device: int = 0, *, n_pages: int | None = None, max_seqs: int = 64,
                 max_batch: int = 64, eps: float | None = None, theta: float | None = None,
                 pages_budget_tokens: int | None = None, packed_cache=None):
        self.L = lib()
        self.config = read_runtime_config(model_dir)
        c = self.config
        d = ModelDesc(c.hidden_size, c.num_hidden_layers, c.num_attention_heads, c.num_key_value_heads, c.head_dim,
                      c.intermediate_size, c.vocab_size, c.max_position_embeddings,
                      eps if eps is not None else c.rms_norm_eps, theta if theta is not None else c.rope_theta)
        h = C.c_void_p()
        check(self.L.mmc_create(C.byref(d), device, C.byref(h)))
        self.h = h
        self.device = device
        try:
            if c.use_moe:  # top-1 MoE MLP (decoder_layer.cpp:370-389)
                check(self.L.mmc_configure_moe(self.h, c.num_experts, c.moe_intermediate_size))
            self.loaded_from = self._load(Path(model_dir), packed_cache)
            if n_pages is None:
                tokens = pages_budget_tokens or max_seqs * 2048
                n_pages = max(1, (tokens + 63) // 64 + max_seqs)
            check(self.L.mmc_kv_init(self.h, n_pages, max_seqs, max_batch))
        except Exception:
            self.close()
            raise
        self.max_batch = max_batch

    def _load(self, model_dir: Path, packed_cache) -> str:
        """weights.bin, or the packed cache (True: model_dir/weights.mmcpk) when
        it is at least as new as weights.bin; a missing or stale cache is
        rebuilt from weights.bin."""
        bin_path = model_dir / "weights.bin"
        if packed_cache:
            cache = model_dir / "weights.mmcpk" if packed_cache is True else Path(packed_cache)
            if cache.exists() and cache.stat().st_mtime >= bin_path.stat().st_mtime:
                if self.L.mmc_load_packed(self.h, str(cache).encode()) == 0:
                    return "packed"
            check(self.L.mmc_load_weights_file(self.h, str(bin_path).encode()))
            check(self.L.mmc_save_packed(self.h, str(cache).encode()))
            return "weights.bin"
        check(self.L.mmc_load_weights_file(self.h, str(bin_path).encode()))
        return "weights.bin"

    def save_packed(self, path) -> None:
        check(self.L.mmc_save_packed(self.h, str(path).encode()))

    # ------------------------------------------------------------ lifecycle
    def close(self):
        if getattr(self, "h", None):
            self.L.mmc_destroy(self.h)
            self.h = None

    def __del__(self):
        self.close()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    # ------------------------------------------------------------ sequences
    def open_sequence(self, reserve_tokens: int = 64) -> int:
        s = C.c_int32()
        check(self.L.mmc_seq_open(self.h, reserve_tokens, C.byref(s)))
        return s.value

    def reserve(self, seq: int, tokens: int) -> None:
        check(self.L.mmc_seq_reserve(self.h, seq, tokens))

    def close_sequence(self, seq: int) -> None:
        check(self.L.mmc_seq_close(self.h, seq))

    def position(self, seq: int) -> int:
        p = C.c_int64()
        check(self.L.mmc_seq_position(self.h, seq, C.byref(p)))
        return p.value

    def fill_context(self, seq: int, n_tokens: int, seed: int = 0) -> None:
        """Fast-forward an empty sequence to `n_tokens` cached positions of
        seeded synthetic K/V (benchmarks and profiling only)."""
        check(self.L.mmc_debug_fill_kv(self.h, seq, n_tokens, seed))

    def page_bytes(self) -> int:
        b = C.c_int64()
        check(self.L.mmc_kv_page_bytes(self.h, C.byref(b)))
        return b.value

    def read_kv(self, seq: int, layer: int):
        n = self.position(seq)
        shape = (n, self.config.num_key_value_heads, self.config.head_dim)
        k = np.zeros(shape, np.float32)
        v = np.zeros(shape, np.float32)
        check(self.L.mmc_debug_read_kv(self.h, seq, layer, k.ctypes.data, v.ctypes.data))
        return k, v

    # ------------------------------------------------------------ decoding
    def step(self, seq_ids, tokens, want_logits: bool = False):
        """One synchronous greedy step; returns (next_tokens, logits or None)."""
        s, t = _i32(seq_ids), _i32(tokens)
        assert s.shape == t.shape and s.ndim == 1
        nxt = np.empty_like(t)
        logits = np.empty((len(s), self.config.vocab_size), np.float32) if want_logits else None
        check(self.L.mmc_decode_step(self.h, len(s), s.ctypes.data, t.ctypes.data, nxt.ctypes.data,
                                     logits.ctypes.data if want_logits else None))
        return nxt, logits

    KERNEL_KINDS = ("qkv", "attention", "o_proj", "gate_up", "down", "lm_head", "embed")

    def profile_step(self, seq_ids, tokens):
        """One step with per-kernel CUDA events; returns (next, {kind: (ms, launches)})."""
        s, t = _i32(seq_ids), _i32(tokens)
        nxt = np.empty_like(t)
        ms = np.zeros(7, np.float32)
        n = np.zeros(7, np.int32)
        check(self.L.mmc_profile_step(self.h, len(s), s.ctypes.data, t.ctypes.data, nxt.ctypes.data, ms.ctypes.data,
                                      n.ctypes.data))
        return nxt, {k: (float(ms[i]), int(n[i])) for i, k in enumerate(self.KERNEL_KINDS)}

    def step_async(self, seq_ids, d_tokens: int, d_next: int, d_logits: int | None = None, stream: int | None = None):
        s = _i32(seq_ids)
        check(self.L.mmc_decode_step_async(self.h, len(s), s.ctypes.data, d_tokens, d_next, d_logits, stream))

    def graph_build(self, seq_ids) -> None:
        s = _i32(seq_ids)
        self._graph_seqs = s
        check(self.L.mmc_graph_build(self.h, len(s), s.ctypes.data))

    def graph_set_tokens(self, tokens) -> None:
        t = _i32(tokens)
        check(self.L.mmc_graph_set_tokens(self.h, t.ctypes.data))

    def graph_run(self, n_steps: int, stream: int | None = None) -> None:
        check(self.L.mmc_graph_run(self.h, n_steps, stream))

    def graph_tokens(self, n_steps: int) -> np.ndarray:
        out = np.empty((n_steps, len(self._graph_seqs)), np.int32)
        check(self.L.mmc_graph_tokens(self.h, n_steps, out.ctypes.data))
        return out

    def synchronize(self) -> None:
        check(self.L.mmc_synchronize(self.h))

    def kernels_per_step(self, batch: int) -> int:
        k = C.c_int32()
        check(self.L.mmc_kernels_per_step(self.h, batch, C.byref(k)))
        return k.value

    def prefill(self, seq_ids, prompts) -> np.ndarray:
        """Feed each sequence's prompt token by token (batched across
        sequences, as LanguageModel::generate_stream does on the CPU path,
        language_model.cpp:384-386); returns the first generated token of each."""
        seq_ids = list(seq_ids)
        first = np.zeros(len(seq_ids), np.int32)
        longest = max(len(p) for p in prompts)
        for t in range(longest):
            rows = [i for i, p in enumerate(prompts) if len(p) > t]
            nxt, _ = self.step([seq_ids[i] for i in rows], [prompts[i][t] for i in rows])
            for j, i in enumerate(rows):
                if t == len(prompts[i]) - 1:
                    first[i] = nxt[j]
        return first

    def prompt_pass(self, seq_ids, prompts) -> np.ndarray:
        """Feed whole prompts on the device in batched passes (mmc_prefill: one
        row per prompt position, causal attention within each sequence);
        returns the first generated token of each sequence, like prefill()."""
        seq_ids = _i32(seq_ids)
        lens = _i32([len(p) for p in prompts])
        toks = _i32([int(t) for p in prompts for t in p])
        first = np.empty(len(seq_ids), np.int32)
        check(self.L.mmc_prefill(self.h, len(seq_ids), seq_ids.ctypes.data, lens.ctypes.data, toks.ctypes.data,
                                 first.ctypes.data))
        return first

    def graph_stream(self, n_steps: int):
        """Streams n_steps replays of the built graph: yields each step's
        tokens ([batch]) as soon as that step has finished on the device, while
        later steps are already queued (mmc_graph_stream_*). Closing the
        generator early stops the run after the steps already queued."""
        check(self.L.mmc_graph_stream_start(self.h, n_steps))
        out = np.empty(len(self._graph_seqs), np.int32)
        try:
            for _ in range(n_steps):
                check(self.L.mmc_graph_stream_next(self.h, out.ctypes.data))
                yield out.copy()
        finally:
            check(self.L.mmc_graph_stream_stop(self.h))

    def generate_stream(self, prompt, max_new_tokens: int, eos: int | None = None):
        """LanguageModel::generate_stream on the device: yields each generated
        token as it is produced (greedy, stops after eos), the prompt in one
        device pass and the decode steps on the streamed graph loop."""
        if not prompt:
            raise ValueError("prompt_tokens cannot be empty")
        if max_new_tokens < 0:
            raise ValueError("max_new_tokens cannot be negative")
        if max_new_tokens == 0:
            return
        eos = self.config.eos_token_id if eos is None else eos
        seq = self.open_sequence(len(prompt) + max_new_tokens + 1)
        try:
            nxt = int(self.prompt_pass([seq], [list(prompt)])[0])
            yield nxt
            if nxt == eos or max_new_tokens == 1:
                return
            self.graph_build([seq])
            self.graph_set_tokens([nxt])
            stream = self.graph_stream(max_new_tokens - 1)
            try:
                for toks in stream:
                    nxt = int(toks[0])
                    yield nxt
                    if nxt == eos:
                        return
            finally:
                stream.close()
        finally:
            self.close_sequence(seq)

    def generate(self, prompt, max_new_tokens: int, eos: int | None = None):
        """LanguageModel::generate on the device (greedy, eos stop)."""
        if not prompt:
            raise ValueError("prompt_tokens cannot be empty")
        if max_new_tokens < 0:
            raise ValueError("max_new_tokens cannot be negative")
        eos = self.config.eos_token_id if eos is None else eos
        seq = self.open_sequence(len(prompt) + max(max_new_tokens, 1))
        try:
            nxt = int(self.prompt_pass([seq], [list(prompt)])[0])
            out = []
            for i in range(max_new_tokens):
                out.append(nxt)
                if nxt == eos or i + 1 == max_new_tokens:
                    break
                nxt = int(self.step([seq], [nxt])[0][0])
            return out
        finally:
            self.close_sequence(seq)
