#!/usr/bin/env bash
# Builds the reference's own CUDA decode kernels (TVM-FFI exports kernel_cuda and
# kernel_cuda_v4 of solution/cuda/kernel.cu) from the reference checkout, in place,
# into oracle/_ref/libref_kernel.so.  Test infrastructure: used only by
# tests/test_reference_cuda_gpu.py as a second, GPU-side parity reference and a
# same-machine timing comparison.  Flags follow the reference's own build
# (solution/cuda/binding.py:19-28: --use_fast_math via tvm_ffi.cpp.build), with the
# architecture made explicit for sm_100a because this machine has no GPU to query.
#
# Usage: oracle/build_ref.sh [REFERENCE_ROOT]   (default: $GDN_REFERENCE_ROOT; there is
# no built-in location: __graft_entry__.build() passes the checkout it found)
set -euo pipefail
HERE="$(cd "$(dirname "${BASH_SOURCE[0]}")" && pwd)"
REF="${1:-${GDN_REFERENCE_ROOT:-}}"
if [ -z "$REF" ]; then echo "usage: build_ref.sh REFERENCE_ROOT (or set GDN_REFERENCE_ROOT)" >&2; exit 2; fi
SRC="$REF/solution/cuda/kernel.cu"
OUT="$HERE/_ref/libref_kernel.so"
if [ ! -f "$SRC" ]; then echo "reference source not found: $SRC" >&2; exit 2; fi
read -r TVM_INC DLPACK_INC TVM_LIBDIR < <(python - <<'PY'
import os
from tvm_ffi import libinfo
print(libinfo.find_include_path(), libinfo.find_dlpack_include_path(),
      os.path.dirname(libinfo.find_libtvm_ffi()))
PY
)
mkdir -p "$HERE/_ref"
nvcc -O3 --use_fast_math -std=c++17 -gencode arch=compute_100a,code=sm_100a \
  -shared -Xcompiler -fPIC -I"$TVM_INC" -I"$DLPACK_INC" "$SRC" -o "$OUT.tmp" \
  -L"$TVM_LIBDIR" -ltvm_ffi -Xlinker -rpath="$TVM_LIBDIR"
mv "$OUT.tmp" "$OUT"
echo "$OUT"
