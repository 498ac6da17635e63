#!/bin/bash
# Compiles the reference's own attention kernels from their sources (where they lie under the
# reference checkout, read-only) for sm_100a, with the C-linkage shim beside this script, into
# oracle/_ref/libcmpext3_ref_kernels.so.  Test infrastructure only: the GPU tests load it as a
# second checker when it exists.  Usage: oracle/build_ref.sh [reference checkout]
set -euo pipefail
HERE="$(cd "$(dirname "$0")" && pwd)"
REF="${1:-/root/reference}"
SRC="$REF/src/cuda"
[ -f "$SRC/fp16_flash_attention_hfma2.cu" ] || { echo "reference sources not found under $SRC" >&2; exit 2; }
mkdir -p "$HERE/_ref"
NVCC="${NVCC:-nvcc}"
"$NVCC" -gencode arch=compute_100a,code=sm_100a -O3 -std=c++17 -shared -Xcompiler -fPIC \
  -o "$HERE/_ref/libcmpext3_ref_kernels.so" \
  "$SRC/fp16_flash_attention_hfma2.cu" "$SRC/fp16_attention.cu" "$SRC/fp32_attention.cu" \
  "$HERE/ref_kernels_shim.cu"
echo "$HERE/_ref/libcmpext3_ref_kernels.so"
