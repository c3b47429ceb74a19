"""Build recipe for the native parts of minimind_orangepi_b200.

Products (all in-tree, so they travel with a repository snapshot):
  lib/libminimind_cuda.so   CUDA kernels + C ABI (include/minimind_cuda.h), sm_100a only
  lib/libminimind_runtime.so  C++ drop-in runtime (LanguageModel & co.) over the C ABI
  bin/minimind_generate, bin/bench_decode   the reference CLIs, same flags and output

Run ``python -m minimind_orangepi_b200.build`` or ``__graft_entry__.build()``.
Object files go to ``_build/`` (git-ignored). Rebuilds are incremental by mtime.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
BUILD = ROOT / "_build"
LIB = PKG / "lib"
BIN = PKG / "bin"
INCLUDE = ROOT / "include"

NVCC = os.environ.get("NVCC", shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc")
CXX = os.environ.get("CXX", "g++")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
                     "--expt-relaxed-constexpr", f"-I{INCLUDE}"]
CXX_FLAGS = ["-std=c++17", "-O3", "-fPIC", "-Wall", "-Wextra", f"-I{INCLUDE}", f"-I{CSRC / 'runtime'}"]

CUDA_SOURCES = [
    CSRC / "kernels" / "gemv.cu",
    CSRC / "kernels" / "gemm_tc.cu",
    CSRC / "kernels" / "mlp_chain.cu",
    CSRC / "kernels" / "attention.cu",
    CSRC / "kernels" / "pack.cu",
    CSRC / "kernels" / "step_kernel.cu",
    CSRC / "kernels" / "skinny.cu",
    CSRC / "mmc_api.cu",
    CSRC / "attention_noalloc.cu",
]
RUNTIME_SOURCES = [
    CSRC / "runtime" / "config.cpp",
    CSRC / "runtime" / "language_model.cpp",
    CSRC / "runtime" / "runtime_loader.cpp",
    CSRC / "runtime" / "tokenizer.cpp",
]


def _run(cmd: list[str]) -> None:
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(" ".join(map(str, cmd)) + "\n" + r.stdout + r.stderr)
        raise RuntimeError(f"build step failed: {Path(cmd[-1]).name}")


def _stale(out: Path, deps: list[Path]) -> bool:
    if not out.exists():
        return True
    t = out.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def _headers() -> list[Path]:
    return list((CSRC / "kernels").glob("*.cuh")) + list((CSRC / "kernels").glob("*.h")) + \
        list((CSRC / "runtime").glob("*.h")) + list(INCLUDE.glob("*.h"))


def build_cuda() -> Path:
    BUILD.mkdir(exist_ok=True)
    LIB.mkdir(exist_ok=True)
    hdrs = _headers()
    jobs = []
    objs = []
    for src in CUDA_SOURCES:
        obj = BUILD / (src.stem + ".o")
        objs.append(obj)
        if _stale(obj, [src, *hdrs, Path(__file__)]):
            jobs.append([NVCC, *NVCC_FLAGS, "-c", str(src), "-o", str(obj)])
    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 2)) as ex:
        list(ex.map(_run, jobs))
    so = LIB / "libminimind_cuda.so"
    if jobs or _stale(so, objs):
        _run([NVCC, *ARCH, "-shared", "-o", str(so), *map(str, objs), "-lcudart_static", "-lrt", "-ldl", "-lpthread"])
    return so


def build_runtime() -> None:
    if not all(p.exists() for p in RUNTIME_SOURCES):
        return
    hdrs = _headers()
    objs = []
    jobs = []
    for src in RUNTIME_SOURCES:
        obj = BUILD / ("rt_" + src.stem + ".o")
        objs.append(obj)
        if _stale(obj, [src, *hdrs]):
            jobs.append([CXX, *CXX_FLAGS, "-c", str(src), "-o", str(obj)])
    with ThreadPoolExecutor(max_workers=4) as ex:
        list(ex.map(_run, jobs))
    rt = LIB / "libminimind_runtime.so"
    cuda = LIB / "libminimind_cuda.so"
    if jobs or _stale(rt, objs + [cuda]):
        _run([CXX, "-shared", "-o", str(rt), *map(str, objs), f"-L{LIB}", "-lminimind_cuda",
              "-Wl,-rpath,$ORIGIN"])
    BIN.mkdir(exist_ok=True)
    for name, src in (("minimind_generate", CSRC / "tools" / "minimind_generate.cpp"),
                      ("bench_decode", CSRC / "bench" / "bench_decode.cpp")):
        if not src.exists():
            continue
        exe = BIN / name
        if _stale(exe, [src, rt, *hdrs]):
            _run([CXX, *CXX_FLAGS, "-o", str(exe), str(src), f"-L{LIB}", "-lminimind_runtime", "-lminimind_cuda",
                  "-Wl,-rpath,$ORIGIN/../lib"])


def build_oracle() -> None:
    """The CPU oracle (test infrastructure): C restatement, and the reference's
    own CPU path when its sources are present on this machine."""
    oracle = ROOT / "oracle"
    so = oracle / "liboracle.so"
    src = oracle / "minimind_oracle.c"
    if _stale(so, [src]):
        _run(["gcc", "-std=c11", "-O3", "-DNDEBUG", "-fPIC", "-shared", "-o", str(so), str(src), "-lm"])
    # the reference checkout: MINIMIND_REFERENCE_ROOT, else a `reference`
    # directory beside this repository's own directory
    env = os.environ.get("MINIMIND_REFERENCE_ROOT")
    ref_root = Path(env) if env else ROOT.parent / "reference"
    if (ref_root / "src" / "csrc").exists():
        _run(["bash", str(oracle / "build_ref.sh"), str(ref_root)])


def build_all() -> None:
    build_cuda()
    build_runtime()
    build_oracle()


if __name__ == "__main__":
    build_all()
    print("built", LIB)
