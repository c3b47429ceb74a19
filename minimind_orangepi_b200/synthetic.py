"""Seeded synthetic MiniMind models in the reference runtime format.

Writes ``minimind_runtime_config.txt`` + ``weights.bin`` exactly as the
reference exporter does (src/python/tools/export_minimind_runtime.py:114-148
tensor order, :175-191 config keys, :218-228 ``MMRTW001`` + per tensor
``u64 name_len, name, u64 count, f32[count]``). The format must stay byte-for-byte
identical so the same directory loads in the reference runtime and in ours;
tests/test_runtime_format.py checks this against the reference exporter.

Two keys are appended that the reference loader ignores (unknown keys are
skipped, runtime_loader.cpp:29-49): ``rms_norm_eps`` and ``rope_theta``. The
CUDA runtime reads them; without them it uses the reference defaults 1e-6/1e6.

Weights follow the benchmark recipe: every projection and the embedding are
N(0, 0.02) fp32, every norm weight is 1, ``lm_head`` is a copy of the embedding
(tied, as the exporter does when ``lm_head.weight`` is missing, :204-205).
"""
from __future__ import annotations

import struct
from dataclasses import dataclass, asdict
from pathlib import Path

import numpy as np


@dataclass(frozen=True)
class ModelShape:
    hidden_size: int
    num_hidden_layers: int
    num_attention_heads: int
    num_key_value_heads: int
    head_dim: int
    intermediate_size: int
    vocab_size: int = 6400
    max_position_embeddings: int = 32768
    num_experts: int = 0  # > 0: top-1 MoE MLP (use_moe=1) with this many experts
    moe_intermediate_size: int = 0  # 0: intermediate_size


SHAPES = {
    # MiniMind2-small (2)
    "minimind2-small": ModelShape(512, 8, 8, 2, 64, 1408),
    # MiniMind2 (4)
    "minimind2": ModelShape(768, 16, 8, 2, 96, 2048),
    # small cases the CPU oracle finishes in milliseconds
    "tiny": ModelShape(64, 2, 4, 2, 16, 128, vocab_size=256, max_position_embeddings=4096),
    "tiny-hd64": ModelShape(256, 2, 4, 2, 64, 384, vocab_size=512, max_position_embeddings=8192),
    "tiny-hd96": ModelShape(384, 2, 4, 1, 96, 512, vocab_size=1024, max_position_embeddings=8192),
    # top-1 MoE variants (the reference's CPU path, decoder_layer.cpp:370-389)
    "tiny-moe": ModelShape(256, 2, 4, 2, 64, 384, vocab_size=512, max_position_embeddings=8192, num_experts=4,
                           moe_intermediate_size=256),
    "minimind2-small-moe": ModelShape(512, 8, 8, 2, 64, 1408, num_experts=4, moe_intermediate_size=1408),
}


def moe_inter(s: ModelShape) -> int:
    return s.moe_intermediate_size or s.intermediate_size


def tensor_order(s: ModelShape) -> list[tuple[str, tuple[int, ...]]]:
    q, kv, h, i = s.num_attention_heads * s.head_dim, s.num_key_value_heads * s.head_dim, s.hidden_size, s.intermediate_size
    out = [("model.embed_tokens.weight", (s.vocab_size, h)), ("model.norm.weight", (h,)), ("lm_head.weight", (s.vocab_size, h))]
    for layer in range(s.num_hidden_layers):
        p = f"model.layers.{layer}."
        out += [
            (p + "input_layernorm.weight", (h,)),
            (p + "post_attention_layernorm.weight", (h,)),
            (p + "self_attn.q_norm.weight", (s.head_dim,)),
            (p + "self_attn.k_norm.weight", (s.head_dim,)),
            (p + "self_attn.q_proj.weight", (q, h)),
            (p + "self_attn.k_proj.weight", (kv, h)),
            (p + "self_attn.v_proj.weight", (kv, h)),
            (p + "self_attn.o_proj.weight", (h, q)),
        ]
        if s.num_experts > 0:  # export_minimind_runtime.py:128-138
            mi = moe_inter(s)
            out.append((p + "mlp.gate.weight", (s.num_experts, h)))
            for e in range(s.num_experts):
                ep = p + f"mlp.experts.{e}."
                out += [(ep + "gate_proj.weight", (mi, h)), (ep + "up_proj.weight", (mi, h)),
                        (ep + "down_proj.weight", (h, mi))]
        else:
            out += [
                (p + "mlp.gate_proj.weight", (i, h)),
                (p + "mlp.up_proj.weight", (i, h)),
                (p + "mlp.down_proj.weight", (h, i)),
            ]
    return out


def synthetic_tensors(s: ModelShape, seed: int, std: float = 0.02) -> dict[str, np.ndarray]:
    rng = np.random.default_rng(seed)
    tensors: dict[str, np.ndarray] = {}
    for name, shape in tensor_order(s):
        if name == "lm_head.weight":
            continue
        if len(shape) == 1:
            tensors[name] = np.ones(shape, dtype=np.float32)
        else:
            tensors[name] = rng.standard_normal(shape, dtype=np.float32) * np.float32(std)
    tensors["lm_head.weight"] = tensors["model.embed_tokens.weight"]
    return tensors


def write_runtime_config(s: ModelShape, out: Path, eps: float | None, theta: float | None) -> None:
    lines = [
        f"hidden_size={s.hidden_size}",
        f"num_hidden_layers={s.num_hidden_layers}",
        f"use_moe={1 if s.num_experts > 0 else 0}",
        f"vocab_size={s.vocab_size}",
        f"num_attention_heads={s.num_attention_heads}",
        f"num_key_value_heads={s.num_key_value_heads}",
        f"head_dim={s.head_dim}",
        f"intermediate_size={s.intermediate_size}",
        f"max_position_embeddings={s.max_position_embeddings}",
        "tie_word_embeddings=1",
        f"num_experts={s.num_experts if s.num_experts > 0 else 4}",
        "num_experts_per_tok=1",
        f"moe_intermediate_size={moe_inter(s)}",
    ]
    if eps is not None:
        lines.append(f"rms_norm_eps={eps!r}")
    if theta is not None:
        lines.append(f"rope_theta={theta!r}")
    (out / "minimind_runtime_config.txt").write_text("\n".join(lines) + "\n")


def write_weights(s: ModelShape, tensors: dict[str, np.ndarray], out: Path) -> None:
    with (out / "weights.bin").open("wb") as f:
        f.write(b"MMRTW001")
        for name, shape in tensor_order(s):
            t = np.ascontiguousarray(tensors[name], dtype="<f4")
            assert t.shape == shape, (name, t.shape, shape)
            raw = name.encode()
            f.write(struct.pack("<Q", len(raw)))
            f.write(raw)
            f.write(struct.pack("<Q", t.size))
            f.write(t.tobytes())


def write_runtime_model(out_dir, shape: str | ModelShape, seed: int, eps: float | None = 1e-5,
                        theta: float | None = 1e6, std: float = 0.02) -> Path:
    """Create (or reuse, when the stamp matches) a seeded model directory."""
    s = SHAPES[shape] if isinstance(shape, str) else shape
    out = Path(out_dir)
    out.mkdir(parents=True, exist_ok=True)
    stamp = repr((asdict(s), seed, eps, theta, std))
    stamp_file = out / ".synthetic_stamp"
    if stamp_file.exists() and stamp_file.read_text() == stamp and (out / "weights.bin").exists():
        return out
    write_runtime_config(s, out, eps, theta)
    write_weights(s, synthetic_tensors(s, seed, std), out)
    stamp_file.write_text(stamp)
    return out


def synthetic_prompt(seed: int, length: int, vocab: int = 6400, low: int = 3) -> list[int]:
    """Prompt ids uniform in [low, vocab)."""
    rng = np.random.default_rng(seed)
    return [int(x) for x in rng.integers(low, vocab, size=length)]
