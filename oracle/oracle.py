"""TEST INFRASTRUCTURE ONLY — ctypes access to the CPU oracles.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline legs import
this module. Two oracles, both CPU, both fp32:

* ``Oracle`` — ``oracle/liboracle.so``, the C restatement of the reference
  decode step (``oracle/minimind_oracle.c``).
* ``ReferenceModel`` — ``oracle/_ref/libminimind_ref.so``, the reference's own
  sources (LanguageModel, language_model.cpp:297-333) compiled by
  ``oracle/build_ref.sh``. Present wherever it was built; it travels with the
  repository snapshot as a built file.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ORACLE_SO = HERE / "liboracle.so"
REF_SO = HERE / "_ref" / "libminimind_ref.so"
REF_CLI = HERE / "_ref" / "minimind_generate_ref"


class MmoConfig(C.Structure):
    _fields_ = [(n, C.c_int64) for n in ("hidden", "layers", "vocab", "nq", "nkv", "hd", "inter", "max_pos")] + [
        ("eps", C.c_float), ("theta", C.c_float)] + [(n, C.c_int64) for n in ("use_moe", "experts", "moe_inter")]


_lib = None


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not ORACLE_SO.exists():
            raise FileNotFoundError(f"{ORACLE_SO} missing: run `make -C oracle liboracle.so`")
        L = C.CDLL(str(ORACLE_SO))
        P, F, I64, I32 = C.c_void_p, C.POINTER(C.c_float), C.c_int64, C.c_int32
        L.mmo_load.restype = P
        L.mmo_load.argtypes = [C.c_char_p, C.c_float, C.c_float]
        L.mmo_free.argtypes = [P]
        L.mmo_state_new.restype = P
        L.mmo_state_new.argtypes = [P]
        L.mmo_state_free.argtypes = [P, P]
        L.mmo_position.restype = I64
        L.mmo_position.argtypes = [P]
        L.mmo_forward_token.restype = I32
        L.mmo_forward_token.argtypes = [P, P, I32, F]
        L.mmo_generate.restype = I64
        L.mmo_generate.argtypes = [P, C.POINTER(I32), I64, I64, I32, C.POINTER(I32)]
        L.mmo_config_of.argtypes = [P, C.POINTER(MmoConfig)]
        L.mmo_last_error.restype = C.c_char_p
        L.mmo_last_router_margin.restype = C.c_float
        L.mmo_matvec.argtypes = [F, I64, I64, F, F]
        L.mmo_rms_norm_inplace.argtypes = [F, F, I64, C.c_float]
        L.mmo_rms_norm_final.argtypes = [F, F, I64, C.c_float, F]
        L.mmo_rope_tables.argtypes = [I64, I64, C.c_float, F, F]
        L.mmo_apply_rope.argtypes = [F, I64, I64, I64, F, F]
        L.mmo_swiglu.argtypes = [F, I64, F]
        L.mmo_attention.argtypes = [F, F, F, I64, I64, I64, I64, F]
        L.mmo_argmax.restype = I32
        L.mmo_argmax.argtypes = [F, I64]
        _lib = L
    return _lib


def fptr(a: np.ndarray):
    assert a.dtype == np.float32 and a.flags.c_contiguous
    return a.ctypes.data_as(C.POINTER(C.c_float))


class Oracle:
    """The C restatement: one model, any number of independent sequences."""

    def __init__(self, model_dir, eps: float = 1e-5, theta: float = 1e6):
        self.L = lib()
        self.h = self.L.mmo_load(str(model_dir).encode(), eps, theta)
        if not self.h:
            raise RuntimeError(self.L.mmo_last_error().decode())
        cfg = MmoConfig()
        self.L.mmo_config_of(self.h, C.byref(cfg))
        self.config = {f: getattr(cfg, f) for f, _ in MmoConfig._fields_}

    def close(self):
        if self.h:
            self.L.mmo_free(self.h)
            self.h = None

    def __del__(self):
        self.close()

    def new_state(self):
        return _State(self, self.L.mmo_state_new(self.h))

    def forward_token(self, state, token: int, want_logits: bool = True):
        logits = np.empty(self.config["vocab"], np.float32) if want_logits else None
        nxt = self.L.mmo_forward_token(self.h, state.h, int(token), fptr(logits) if want_logits else None)
        if nxt < 0:
            raise IndexError(self.L.mmo_last_error().decode())
        return nxt, logits

    def router_margin(self) -> float:
        """Smallest top-1 vs top-2 router margin (relative to |top-1|) over the
        layers of the last forward_token; inf for dense models. A small margin
        means an implementation with fp16 weights may route that token to the
        other expert."""
        return float(self.L.mmo_last_router_margin())

    def generate(self, prompt, max_new: int, eos: int = 2):
        p = (C.c_int32 * len(prompt))(*prompt)
        out = (C.c_int32 * max(max_new, 1))()
        n = self.L.mmo_generate(self.h, p, len(prompt), max_new, eos, out)
        if n < 0:
            raise ValueError("oracle generate failed")
        return list(out[:n])


class _State:
    def __init__(self, owner, h):
        self.owner, self.h = owner, h

    @property
    def position(self):
        return self.owner.L.mmo_position(self.h)

    def __del__(self):
        if self.h and self.owner.h:
            self.owner.L.mmo_state_free(self.owner.h, self.h)
            self.h = None


# --------------------------------------------------------------- reference

_ref = None


def ref_available() -> bool:
    return REF_SO.exists()


def ref_lib() -> C.CDLL:
    global _ref
    if _ref is None:
        if not REF_SO.exists():
            raise FileNotFoundError(f"{REF_SO} missing: run oracle/build_ref.sh where the reference is present")
        L = C.CDLL(str(REF_SO))
        P, F, I64, I32 = C.c_void_p, C.POINTER(C.c_float), C.c_int64, C.c_int32
        L.mmref_load.restype = P
        L.mmref_load.argtypes = [C.c_char_p, C.c_float, C.c_float]
        L.mmref_toy_model.restype = P
        L.mmref_free.argtypes = [P]
        L.mmref_state_new.restype = P
        L.mmref_state_new.argtypes = [P]
        L.mmref_state_free.argtypes = [P]
        L.mmref_position.restype = I64
        L.mmref_position.argtypes = [P]
        L.mmref_forward_token.restype = I32
        L.mmref_forward_token.argtypes = [P, P, I32, F]
        L.mmref_forward_next_token.restype = I32
        L.mmref_forward_next_token.argtypes = [P, P, I32]
        L.mmref_generate.restype = I64
        L.mmref_generate.argtypes = [P, C.POINTER(I32), I64, I64, C.POINTER(I32)]
        L.mmref_fill_context.restype = C.c_int
        L.mmref_fill_context.argtypes = [P, P, I64, C.c_uint64]
        L.mmref_last_error.restype = C.c_char_p
        _ref = L
    return _ref


class ReferenceModel:
    """The reference's own LanguageModel (CPU fp32 path) behind a C driver."""

    def __init__(self, model_dir=None, eps: float = 1e-5, theta: float = 1e6, vocab: int | None = None):
        self.L = ref_lib()
        self.h = self.L.mmref_load(str(model_dir).encode(), eps, theta) if model_dir else self.L.mmref_toy_model()
        if not self.h:
            raise RuntimeError(self.L.mmref_last_error().decode())
        self.vocab = vocab

    def close(self):
        if self.h:
            self.L.mmref_free(self.h)
            self.h = None

    def __del__(self):
        self.close()

    def new_state(self):
        return _RefState(self, self.L.mmref_state_new(self.h))

    def forward_token(self, state, token: int, vocab: int):
        logits = np.empty(vocab, np.float32)
        nxt = self.L.mmref_forward_token(self.h, state.h, int(token), fptr(logits))
        if nxt < 0:
            raise IndexError(self.L.mmref_last_error().decode())
        return nxt, logits

    def forward_next_token(self, state, token: int) -> int:
        nxt = self.L.mmref_forward_next_token(self.h, state.h, int(token))
        if nxt < 0:
            raise IndexError(self.L.mmref_last_error().decode())
        return nxt

    def generate(self, prompt, max_new: int):
        p = (C.c_int32 * len(prompt))(*prompt)
        out = (C.c_int32 * max(max_new, 1))()
        n = self.L.mmref_generate(self.h, p, len(prompt), max_new, out)
        if n < 0:
            raise ValueError(self.L.mmref_last_error().decode())
        return list(out[:n])

    def fill_context(self, state, ctx: int, seed: int = 0):
        if self.L.mmref_fill_context(self.h, state.h, ctx, seed) != 0:
            raise RuntimeError(self.L.mmref_last_error().decode())


class _RefState:
    def __init__(self, owner, h):
        self.owner, self.h = owner, h

    @property
    def position(self):
        return self.owner.L.mmref_position(self.h)

    def __del__(self):
        if self.h and self.owner.h:
            self.owner.L.mmref_state_free(self.h)
            self.h = None
