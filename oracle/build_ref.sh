#!/bin/sh
# Builds oracle/_ref/libttref.so: the reference's own C++ sources, compiled
# unmodified from where they lie, plus oracle/ref_capi.cpp (extern "C" entry
# points) and a small_vector shim (oracle/shim). Test infrastructure only.
#
# The reference's CMake/Conan build is not used (no Conan, Boost or gtest in
# this image); the same release flags (-O3 -DNDEBUG, CMakeLists.txt:116) are.
# spdlog is header-only and comes from the copy bundled with flashinfer.
set -e
HERE=$(cd "$(dirname "$0")" && pwd)
# the reference checkout: $TT_REFERENCE_ROOT, default a directory named
# "reference" beside this repository
REF=${TT_REFERENCE_ROOT:-$(cd "$HERE/../.." && pwd)/reference}
OUT="$HERE/_ref"
if [ ! -d "$REF/src/backend/cpu" ]; then
    echo "build_ref.sh: reference sources not found at $REF; skipping" >&2
    exit 0
fi
PURELIB=$(python -c "import sysconfig; print(sysconfig.get_paths()['purelib'])")
SPDLOG="$PURELIB/flashinfer/data/spdlog/include"
mkdir -p "$OUT"
SRCS="$REF/src/core/Context.cpp $REF/src/core/Node.cpp $REF/src/core/Tensor.cpp $REF/src/core/MemoryManager.cpp \
      $REF/src/frontend/operations.cpp \
      $REF/src/tape/Tape.cpp $REF/src/tape/TapeExecutor.cpp $REF/src/tape/TapeGenerator.cpp \
      $REF/src/tape/TapeEvaluationManager.cpp $REF/src/tape/OperationHandlers.cpp \
      $REF/src/tape/passes/TapeOptimizationPass.cpp $REF/src/tape/passes/DeadCodeEliminationPass.cpp \
      $REF/src/tape/passes/MLPFusionPass.cpp \
      $REF/src/backend/cpu/eltwise.cpp $REF/src/backend/cpu/matmul.cpp $REF/src/backend/cpu/reduce_sum.cpp \
      $REF/src/backend/cpu/split.cpp $REF/src/backend/cpu/transpose.cpp $REF/src/backend/cpu/fused_ops.cpp"
g++ -std=c++17 -O3 -DNDEBUG -fPIC -shared -w \
    -I"$HERE/shim" -I"$REF/src/core" -I"$REF/src/frontend" -I"$REF/src/tape" -I"$REF/src/tape/passes" \
    -I"$REF/src/backend/cpu" -I"$SPDLOG" \
    $SRCS "$HERE/ref_capi.cpp" -o "$OUT/libttref.so.tmp"
mv "$OUT/libttref.so.tmp" "$OUT/libttref.so"
echo "built $OUT/libttref.so"
