#!/bin/sh
# Builds tests/native/_build/libttref_cuda.so: the reference's own front end
# and tape (src/core, src/frontend, src/tape, src/tape/passes), compiled
# unmodified from where they lie, with tt_lazy_b200/binding/OperationHandlers.cpp
# in place of src/tape/OperationHandlers.cpp and libtt_cuda.so in place of the
# CPU library tt_math_lib (the link of CMakeLists.txt:264-270 of the
# reference), plus the test entry points of reference_binding_entry.cpp.
# Test infrastructure: the GPU test tests/test_reference_binding_gpu.py loads it.
# -Bsymbolic binds the library's references to its own definitions: a
# process that also loaded this repository's front end (libtt_lazy.so, whose
# classes share the reference's names) keeps the two apart.
#
# The reference sources come from $TT_REFERENCE_ROOT (default: a checkout
# named "reference" beside this repository). Boost's small_vector comes from
# the oracle's shim, spdlog (header-only) from the copy bundled with flashinfer.
set -e
HERE=$(cd "$(dirname "$0")" && pwd)
REPO=$(cd "$HERE/../.." && pwd)
REF=${TT_REFERENCE_ROOT:-$REPO/../reference}
OUT="$HERE/_build"
if [ ! -d "$REF/src/tape" ]; then
    echo "build_reference_binding.sh: reference sources not found at $REF; skipping" >&2
    exit 0
fi
PURELIB=$(python -c "import sysconfig; print(sysconfig.get_paths()['purelib'])")
SPDLOG="$PURELIB/flashinfer/data/spdlog/include"
mkdir -p "$OUT"
SRCS="$REF/src/core/Context.cpp $REF/src/core/Node.cpp $REF/src/core/Tensor.cpp $REF/src/core/MemoryManager.cpp \
      $REF/src/frontend/operations.cpp \
      $REF/src/tape/Tape.cpp $REF/src/tape/TapeExecutor.cpp $REF/src/tape/TapeGenerator.cpp \
      $REF/src/tape/TapeEvaluationManager.cpp \
      $REF/src/tape/passes/TapeOptimizationPass.cpp $REF/src/tape/passes/DeadCodeEliminationPass.cpp \
      $REF/src/tape/passes/MLPFusionPass.cpp"
g++ -std=c++17 -O2 -DNDEBUG -fPIC -shared -w \
    -I"$REPO/oracle/shim" -I"$REF/src/core" -I"$REF/src/frontend" -I"$REF/src/tape" -I"$REF/src/tape/passes" \
    -I"$SPDLOG" -I"$REPO/include" \
    $SRCS "$REPO/tt_lazy_b200/binding/OperationHandlers.cpp" "$HERE/reference_binding_entry.cpp" \
    -L"$REPO/tt_lazy_b200/lib" -l:libtt_cuda.so -Wl,-rpath,'$ORIGIN/../../../tt_lazy_b200/lib' \
    -Wl,--no-undefined -Wl,-Bsymbolic -o "$OUT/libttref_cuda.so.tmp"
mv "$OUT/libttref_cuda.so.tmp" "$OUT/libttref_cuda.so"
echo "built $OUT/libttref_cuda.so"
