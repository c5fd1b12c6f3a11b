#!/bin/sh
# Builds oracle/_ref/libmobius_native_ref.so: the reference's native FP64 Möbius evaluator,
# compiled from its own sources where they lie (REFERENCE/rune/mobius/src/*.cu, unmodified)
# against the GPUMD stand-ins in this directory, plus the C ABI of ref_native.cu. Test
# infrastructure only; the output stays out of git (oracle/_ref/ is ignored).
#   usage: oracle/native/build.sh REFERENCE_CHECKOUT
set -e
REF="${1:?usage: build.sh REFERENCE_CHECKOUT}"
HERE="$(cd "$(dirname "$0")" && pwd)"
OUT="$HERE/../_ref"
SRC="$REF/rune/mobius/src"
NVCC="${CUDA_HOME:-/usr/local/cuda}/bin/nvcc"
mkdir -p "$OUT/obj"
FLAGS="-O3 -std=c++17 -gencode arch=compute_100a,code=sm_100a -Xcompiler -fPIC -I $HERE -I $SRC"
pids=""
for f in "$SRC"/*.cu "$HERE/ref_native.cu"; do
  "$NVCC" $FLAGS -c "$f" -o "$OUT/obj/$(basename "$f" .cu).o" &
  pids="$pids $!"
done
for p in $pids; do wait "$p"; done
"$NVCC" -gencode arch=compute_100a,code=sm_100a -shared -o "$OUT/libmobius_native_ref.so" \
  "$OUT"/obj/*.o -lcublas
echo "$OUT/libmobius_native_ref.so"
