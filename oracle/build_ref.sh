#!/usr/bin/env bash
# Builds the reference's own CUDA kernels (unmodified, compiled where they lie in the
# reference tree) plus oracle/ref_shim.cu into oracle/_ref/libragrt_ref.so.  Test
# infrastructure only: the product never links it.  Needs the reference tree: the
# directory named by RAGRT_REFERENCE_DIR, else a checkout named `reference` beside this
# repository; the built .so travels to the GPU box with the repo snapshot.
set -euo pipefail
HERE="$(cd "$(dirname "${BASH_SOURCE[0]}")" && pwd)"
REF="${RAGRT_REFERENCE_DIR:-$(cd "$HERE/../.." && pwd)/reference}"
[ -f "$REF/src/ragrt_fused_kernel.cu" ] || { echo "reference tree not found at $REF" >&2; exit 1; }
mkdir -p "$HERE/_ref"
nvcc -gencode arch=compute_100a,code=sm_100a -O3 -std=c++17 -shared -Xcompiler -fPIC \
     -o "$HERE/_ref/libragrt_ref.so" \
     "$REF/src/ragrt_fused_kernel.cu" "$REF/src/tile_maxsim_fused_decomp.cu" "$HERE/ref_shim.cu"
echo "built $HERE/_ref/libragrt_ref.so"
