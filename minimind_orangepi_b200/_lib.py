"""ctypes binding of libminimind_cuda.so (include/minimind_cuda.h).

The library is loaded from ``minimind_orangepi_b200/lib`` (or the path in the
MMC_LIBRARY environment variable, e.g. a build with other tuning macros). If it is missing the
import of anything that computes fails loudly: there is no CPU fallback.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

LIB_PATH = Path(os.environ.get("MMC_LIBRARY") or Path(__file__).resolve().parent / "lib" / "libminimind_cuda.so")

MMC_OK = 0
STATUS = {1: "MMC_ERR_INVALID", 2: "MMC_ERR_OUT_OF_RANGE", 3: "MMC_ERR_CUDA", 4: "MMC_ERR_NO_PAGES",
          5: "MMC_ERR_DEVICE", 6: "MMC_ERR_STATE", 7: "MMC_ERR_IO"}


class MmcError(RuntimeError):
    def __init__(self, code: int, message: str):
        super().__init__(f"{STATUS.get(code, code)}: {message}")
        self.code = code


class ModelDesc(C.Structure):
    _fields_ = [
        ("hidden_size", C.c_int64),
        ("num_hidden_layers", C.c_int64),
        ("num_attention_heads", C.c_int64),
        ("num_key_value_heads", C.c_int64),
        ("head_dim", C.c_int64),
        ("intermediate_size", C.c_int64),
        ("vocab_size", C.c_int64),
        ("max_position_embeddings", C.c_int64),
        ("rms_norm_eps", C.c_float),
        ("rope_theta", C.c_float),
    ]


EXPORTS = {
    # name: (restype, argtypes)
    "mmc_last_error": (C.c_char_p, []),
    "mmc_abi_version": (C.c_int, []),
    "mmc_create": (C.c_int, [C.POINTER(ModelDesc), C.c_int, C.POINTER(C.c_void_p)]),
    "mmc_destroy": (None, [C.c_void_p]),
    "mmc_load_weights": (C.c_int, [C.c_void_p, C.POINTER(C.POINTER(C.c_float)), C.POINTER(C.c_int64), C.c_int32]),
    "mmc_load_weights_file": (C.c_int, [C.c_void_p, C.c_char_p]),
    "mmc_kv_page_bytes": (C.c_int, [C.c_void_p, C.POINTER(C.c_int64)]),
    "mmc_kv_init": (C.c_int, [C.c_void_p, C.c_int64, C.c_int32, C.c_int32]),
    "mmc_seq_open": (C.c_int, [C.c_void_p, C.c_int64, C.POINTER(C.c_int32)]),
    "mmc_seq_reserve": (C.c_int, [C.c_void_p, C.c_int32, C.c_int64]),
    "mmc_seq_close": (C.c_int, [C.c_void_p, C.c_int32]),
    "mmc_seq_position": (C.c_int, [C.c_void_p, C.c_int32, C.POINTER(C.c_int64)]),
    "mmc_debug_read_kv": (C.c_int, [C.c_void_p, C.c_int32, C.c_int32, C.c_void_p, C.c_void_p]),
    "mmc_debug_fill_kv": (C.c_int, [C.c_void_p, C.c_int32, C.c_int64, C.c_uint32]),
    "mmc_debug_scratch": (C.c_int, [C.c_void_p, C.c_int32, C.c_void_p, C.c_int64]),
    "mmc_debug_step_trace": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int64, C.POINTER(C.c_int64)]),
    "mmc_decode_step": (C.c_int, [C.c_void_p, C.c_int32, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]),
    "mmc_configure_moe": (C.c_int, [C.c_void_p, C.c_int32, C.c_int64]),
    "mmc_save_packed": (C.c_int, [C.c_void_p, C.c_char_p]),
    "mmc_load_packed": (C.c_int, [C.c_void_p, C.c_char_p]),
    "mmc_prefill": (C.c_int, [C.c_void_p, C.c_int32, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p]),
    "mmc_profile_step": (C.c_int, [C.c_void_p, C.c_int32, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                   C.c_void_p]),
    "mmc_decode_step_async": (C.c_int, [C.c_void_p, C.c_int32, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                        C.c_void_p]),
    "mmc_graph_build": (C.c_int, [C.c_void_p, C.c_int32, C.c_void_p]),
    "mmc_graph_set_tokens": (C.c_int, [C.c_void_p, C.c_void_p]),
    "mmc_graph_run": (C.c_int, [C.c_void_p, C.c_int32, C.c_void_p]),
    "mmc_graph_tokens": (C.c_int, [C.c_void_p, C.c_int32, C.c_void_p]),
    "mmc_graph_stream_start": (C.c_int, [C.c_void_p, C.c_int32]),
    "mmc_graph_stream_next": (C.c_int, [C.c_void_p, C.c_void_p]),
    "mmc_graph_stream_stop": (C.c_int, [C.c_void_p]),
    "mmc_synchronize": (C.c_int, [C.c_void_p]),
    "mmc_kernels_per_step": (C.c_int, [C.c_void_p, C.c_int32, C.POINTER(C.c_int32)]),
    "mmc_op_projection": (C.c_int, [C.c_int32, C.c_int32, C.c_int32, C.c_void_p, C.c_void_p, C.c_void_p,
                                    C.c_void_p]),
    "mmc_op_lm_head_argmax_workspace_size": (C.c_int, [C.c_int32, C.c_int32, C.c_int32, C.POINTER(C.c_size_t)]),
    "mmc_op_lm_head_argmax": (C.c_int, [C.c_int32, C.c_int32, C.c_int32, C.c_void_p, C.c_void_p, C.c_void_p,
                                        C.c_void_p, C.c_void_p, C.c_size_t, C.c_void_p]),
    "mmc_op_attention_workspace_size": (C.c_int, [C.c_int32, C.c_int32, C.c_int32, C.c_int32, C.c_int32,
                                                  C.POINTER(C.c_size_t)]),
    "mmc_op_attention": (C.c_int, [C.c_int32, C.c_int32, C.c_int32, C.c_int32, C.c_int32, C.c_int32,
                                   C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int32,
                                   C.c_float, C.c_void_p, C.c_void_p, C.c_int32, C.c_void_p, C.c_void_p,
                                   C.c_int32, C.c_void_p, C.c_void_p, C.c_size_t, C.c_void_p]),
    "mmc_op_attention_status": (C.c_int, [C.c_void_p, C.c_void_p]),
    "mmc_op_attention_noalloc": (C.c_int, [C.c_int32, C.c_int32, C.c_int32, C.c_int32, C.c_int32, C.c_int32,
                                           C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int32,
                                           C.c_float, C.c_void_p, C.c_void_p, C.c_int32, C.c_void_p, C.c_void_p,
                                           C.c_int32, C.c_void_p, C.c_void_p]),
    "mmc_kv_row_offset": (C.c_int64, [C.c_int32, C.c_int32, C.c_int32]),
}

_lib: C.CDLL | None = None


def lib() -> C.CDLL:
    """Load libminimind_cuda.so (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise FileNotFoundError(
                f"{LIB_PATH} is missing: build it with `python -m minimind_orangepi_b200.build` "
                "(the CUDA path has no CPU fallback)")
        L = C.CDLL(str(LIB_PATH))
        for name, (res, args) in EXPORTS.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


def check(code: int) -> None:
    if code != MMC_OK:
        raise MmcError(code, lib().mmc_last_error().decode())
