#!/usr/bin/env bash
# Builds oracle/_ref/libalpaka_ref.so: the reference's own host backend (alpaka3 headers, unmodified, read in place)
# behind the C entry points of oracle/ref_harness.cpp. Test infrastructure only.
#
# usage: oracle/build_ref.sh REFERENCE_ROOT   (the alpaka3 source tree)
# FP contraction is pinned off so element-wise results are IEEE-exact per operation (the CUDA kernels use the
# same explicitly rounded _rn operations), which makes copy/mul/add/triad bit-comparable.
set -euo pipefail
REF="${1:?usage: build_ref.sh REFERENCE_ROOT}"
HERE="$(cd "$(dirname "$0")" && pwd)"
OUT="$HERE/_ref"
mkdir -p "$OUT"
if [ ! -d "$REF/include/alpaka" ]; then
    echo "reference tree not found at $REF; oracle/_ref not rebuilt" >&2
    exit 0
fi
g++ -std=c++20 -O3 -march=x86-64-v3 -fopenmp -ffp-contract=off -fPIC -shared \
    -I"$REF/include" \
    -I"$REF/example/heatEquation2D/src" \
    -I"$REF/example/nBody/src" \
    -I"$REF/benchmark/HACCmk/src" \
    -o "$OUT/libalpaka_ref.so.tmp" "$HERE/ref_harness.cpp"
mv "$OUT/libalpaka_ref.so.tmp" "$OUT/libalpaka_ref.so"
echo "built $OUT/libalpaka_ref.so"

# The reference's CUDA backend on the same workloads (GPU comparator), for sm_100a with nvcc's defaults (FMA
# contraction on, as the reference's own CUDA builds use). Philox inputs come from ../liboracle.so.
if command -v nvcc > /dev/null && [ -f "$HERE/liboracle.so" ]; then
    nvcc -x cu -std=c++20 -O3 --expt-relaxed-constexpr --extended-lambda \
        -gencode arch=compute_100a,code=sm_100a \
        -I"$REF/include" \
        -I"$REF/example/heatEquation2D/src" \
        -I"$REF/example/nBody/src" \
        -o "$OUT/ref_cuda_bench.tmp" "$HERE/ref_cuda_bench.cpp" \
        -L"$HERE" -loracle -Xlinker -rpath -Xlinker '$ORIGIN/..'
    mv "$OUT/ref_cuda_bench.tmp" "$OUT/ref_cuda_bench"
    echo "built $OUT/ref_cuda_bench"
fi
