#!/usr/bin/env bash
# build_ref.sh -- compile the reference operator (YuWei-CH/Fused-MoE-YWS
# solution/cuda/kernel.cu) from its own source location into oracle/_ref/ref_kernel.so.
#
# TEST INFRASTRUCTURE ONLY: the result is used to pin the CPU oracle against the
# reference itself on a B200 (tests/test_gpu_parity.py::test_oracle_pinned_to_reference_kernel,
# tests/golden/make_ref_goldens.py)
# and as the timed comparator of `bench.py --impl reference`. No reference source is
# copied into this repository; the compiler reads it in place.
#
# Flags follow solution/cuda/binding.py:23-29 (-O3 --use_fast_math, compute_100/sm_100),
# except -std=c++21, which nvcc 12.9 rejects; c++17 is used instead. CUTLASS headers come
# from the flashinfer wheel (solution/cuda/kernel.cu includes cutlass/*), TVM-FFI headers
# and libtvm_ffi.so from the tvm_ffi wheel.
set -euo pipefail
HERE="$(cd "$(dirname "$0")" && pwd)"
# the reference checkout: FMOE_REFERENCE_ROOT, else a `reference` directory beside this
# repository's own directory
REF_ROOT="${FMOE_REFERENCE_ROOT:-$(cd "$HERE/../.." && pwd)/reference}"
REF_SRC="$REF_ROOT/solution/cuda/kernel.cu"
OUT="$HERE/_ref"
if [ ! -f "$REF_SRC" ]; then
  echo "reference source not found at $REF_SRC; skipping" >&2
  exit 0
fi
SP="$(python -c 'import sysconfig; print(sysconfig.get_paths()["purelib"])')"
mkdir -p "$OUT"
if [ -f "$OUT/ref_kernel.so" ] && [ "$OUT/ref_kernel.so" -nt "$REF_SRC" ]; then
  exit 0
fi
nvcc -O3 --use_fast_math -std=c++17 -gencode=arch=compute_100,code=sm_100 -shared \
  -Xcompiler -fPIC \
  -I"$SP/flashinfer/data/cutlass/include" -I"$SP/flashinfer/data/cutlass/tools/util/include" \
  -I"$SP/tvm_ffi/include" -I"$SP/tvm_ffi/3rdparty/dlpack/include" \
  "$REF_SRC" -o "$OUT/ref_kernel.so" \
  -L"$SP/tvm_ffi/lib" -ltvm_ffi -Xlinker -rpath -Xlinker "$SP/tvm_ffi/lib"
echo "built $OUT/ref_kernel.so"
