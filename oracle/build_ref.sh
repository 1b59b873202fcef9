#!/usr/bin/env bash
# Compile the reference repository's own CUDA kernels, unmodified, from the
# read-only reference tree into oracle/_ref/ (git-ignored; the .so files travel
# with the source tree to GPU machines).  They are a checker only: the GPU test
# tests/test_reference_kernels.py runs them at their hard-coded qk4_v8 head
# layout (ref solution/cuda/kernel.cu:10-11, kernel_prefill.cu:11-12) to pin
# the CPU oracle against the reference's real arithmetic.
#
# Usage: oracle/build_ref.sh [REFERENCE_ROOT]
#   REFERENCE_ROOT defaults to $GDN_REFERENCE_ROOT, else a `reference` directory
#   beside this repository.
set -euo pipefail
HERE="$(cd "$(dirname "${BASH_SOURCE[0]}")" && pwd)"
REF="${1:-${GDN_REFERENCE_ROOT:-$(dirname "$(dirname "$HERE")")/reference}}"
OUT="$HERE/_ref"
if [ ! -f "$REF/solution/cuda/kernel.cu" ]; then
  echo "reference sources not found under $REF; nothing to build" >&2
  exit 0
fi
PY="${PYTHON:-python}"
TVM_INC="$($PY -c 'from tvm_ffi import libinfo; print(libinfo.find_include_path())')"
DL_INC="$($PY -c 'from tvm_ffi import libinfo; print(libinfo.find_dlpack_include_path())')"
TVM_LIB="$(dirname "$($PY -c 'from tvm_ffi import libinfo; print(libinfo.find_libtvm_ffi())')")"
mkdir -p "$OUT"
for pair in "kernel.cu:ref_decode.so" "kernel_prefill.cu:ref_prefill.so"; do
  src="${pair%%:*}"; dst="${pair##*:}"
  nvcc -gencode arch=compute_100a,code=sm_100a -O3 -std=c++17 -Xcompiler -fPIC -shared \
    -I"$TVM_INC" -I"$DL_INC" -L"$TVM_LIB" -ltvm_ffi -Xlinker -rpath -Xlinker "$TVM_LIB" \
    -o "$OUT/$dst" "$REF/solution/cuda/$src"
  echo "built $OUT/$dst"
done
