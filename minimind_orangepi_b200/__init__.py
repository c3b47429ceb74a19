"""B200-native single-token decode for MiniMind models (drop-in for the
lvyufeng/minimind-orangepi decode path). The compute runs in
``lib/libminimind_cuda.so`` (sm_100a CUDA kernels behind a C ABI)."""
from .engine import DecodeEngine, RuntimeConfig, read_runtime_config  # noqa: F401
from ._lib import LIB_PATH, MmcError, lib  # noqa: F401

__all__ = ["DecodeEngine", "RuntimeConfig", "read_runtime_config", "MmcError", "lib", "LIB_PATH"]
