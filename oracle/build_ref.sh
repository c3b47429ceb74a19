#!/usr/bin/env bash
# TEST INFRASTRUCTURE ONLY (oracle). Builds the reference's own fp32 CPU decode
# path from its unmodified sources, where they lie, into oracle/_ref/:
#   oracle/_ref/libminimind_ref.so      reference LanguageModel + our C driver
#   oracle/_ref/minimind_generate_ref   the reference CLI (tools/minimind_generate.cpp)
# The reference's CMake build is not used (it probes for CANN). Two compile
# shims, neither of which edits a reference file:
#   1. language_model.cpp calls cube_* without including ascend_matmul.h in the
#      CPU build -> passed with `-include ascend_matmul.h`.
#   2. ascend_matmul.cpp does not compile on CPU (cpu_matvec undeclared at
#      :627/:690) -> left out; oracle/ref_shim.cpp supplies the CPU-build
#      symbols (cube_*_available() == false, so the CPU path is taken).
# Flags follow the reference's Release build (-O3 -DNDEBUG, C++17), no -march,
# no fast-math, so float arithmetic is plain IEEE SSE2.
# Usage: oracle/build_ref.sh [REFERENCE_ROOT]
#   (default: $MINIMIND_REFERENCE_ROOT, else `reference` beside this repository)
set -euo pipefail
HERE="$(cd "$(dirname "${BASH_SOURCE[0]}")" && pwd)"
REF="${1:-${MINIMIND_REFERENCE_ROOT:-$(cd "$HERE/../.." && pwd)/reference}}"
SRC="$REF/src/csrc"
OUT="$HERE/_ref"
if [ ! -d "$SRC/models/minimind" ]; then
  echo "build_ref: reference sources not found under $REF; skipping" >&2
  exit 0
fi
mkdir -p "$OUT/obj"
CXX="${CXX:-g++}"
FLAGS=(-std=c++17 -O3 -DNDEBUG -fPIC -w -I"$SRC/include" -I"$SRC/models/minimind")
M="$SRC/models/minimind"
objs=()
compile() {  # src obj [extra flags]
  local src="$1" obj="$OUT/obj/$2"; shift 2
  if [ ! -f "$obj" ] || [ "$src" -nt "$obj" ] || [ "$HERE/build_ref.sh" -nt "$obj" ]; then
    "$CXX" "${FLAGS[@]}" "$@" -c "$src" -o "$obj"
  fi
  objs+=("$obj")
}
compile "$M/config.cpp" config.o
compile "$M/decoder_layer.cpp" decoder_layer.o
compile "$M/language_model.cpp" language_model.o -include "$M/ascend_matmul.h"
compile "$M/runtime_loader.cpp" runtime_loader.o
compile "$M/ascend_custom_ops.cpp" ascend_custom_ops.o
compile "$SRC/lib/tokenizer.cpp" tokenizer.o
compile "$SRC/lib/weights.cpp" weights.o
compile "$HERE/ref_shim.cpp" ref_shim.o
runtime=("${objs[@]}")
compile "$HERE/ref_driver.cpp" ref_driver.o
"$CXX" -shared -o "$OUT/libminimind_ref.so" "${objs[@]}"
"$CXX" "${FLAGS[@]}" -o "$OUT/minimind_generate_ref" "$SRC/tools/minimind_generate.cpp" "${runtime[@]}"
echo "build_ref: built $OUT/libminimind_ref.so and $OUT/minimind_generate_ref"
