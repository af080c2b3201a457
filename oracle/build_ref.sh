#!/bin/sh
# Builds oracle/_ref/ref_kernels_bench: the timing harness in this directory
# compiled against the reference's own, unmodified CUDA headers (src/ of
# ssubbotin/windlass) for sm_100a. Test/baseline infrastructure only; the
# output stays out of git (oracle/_ref/ is ignored) and travels to the GPU box
# with the tree. Usage: oracle/build_ref.sh [reference checkout]
set -e
HERE=$(cd "$(dirname "$0")" && pwd)
REF=${1:-/root/reference}
if [ ! -f "$REF/src/glm_layer_runner.cuh" ]; then
    echo "reference sources not found under $REF; nothing built" >&2
    exit 0
fi
NVCC=${NVCC:-$(command -v nvcc || echo /usr/local/cuda/bin/nvcc)}
mkdir -p "$HERE/_ref"
"$NVCC" -gencode arch=compute_100a,code=sm_100a -O2 -std=c++17 -Wno-deprecated-gpu-targets \
    -I "$REF/src" "$HERE/ref_kernels_bench.cu" -o "$HERE/_ref/ref_kernels_bench.tmp" -lpthread
mv "$HERE/_ref/ref_kernels_bench.tmp" "$HERE/_ref/ref_kernels_bench"
echo "$HERE/_ref/ref_kernels_bench"
