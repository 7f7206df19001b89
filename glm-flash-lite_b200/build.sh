#!/usr/bin/env bash
# Builds libglmx.so (sm_100a) in-tree: glm-flash-lite_b200/lib/libglmx.so. Static CUDA runtime, no torch linkage.
set -euo pipefail
HERE="$(cd "$(dirname "${BASH_SOURCE[0]}")" && pwd)"
NVCC="${NVCC:-nvcc}"
OUT="$HERE/lib"
OBJ="$HERE/_build"
mkdir -p "$OUT" "$OBJ"
FLAGS=(-std=c++17 -O3 -lineinfo -gencode arch=compute_100a,code=sm_100a -Xcompiler -fPIC -Xcompiler -fvisibility=hidden
       --expt-relaxed-constexpr -I"$HERE/../include" ${GLMX_NVCC_EXTRA:-})
SRCS=(route.cu moe_decode.cu moe_i16.cu moe_prefill.cu capi.cu noalloc.cu selftest.cu router.cu peer.cu hc.cu)
objs=()
pids=()
for s in "${SRCS[@]}"; do
  o="$OBJ/${s%.cu}.o"
  extra=()
  # the hyper-connection site kernels use the reference's own compile flags for its kernels (-O3 --use_fast_math),
  # so that their fast intrinsics and flush-to-zero arithmetic give the reference's bits
  [ "$s" = hc.cu ] && extra=(--use_fast_math)
  "$NVCC" "${FLAGS[@]}" "${extra[@]}" -c "$HERE/csrc/$s" -o "$o" &
  pids+=($!)
  objs+=("$o")
done
for p in "${pids[@]}"; do wait "$p"; done     # set -e: the first failed compile stops the build
"$NVCC" -shared -gencode arch=compute_100a,code=sm_100a -Xcompiler -fPIC "${objs[@]}" -o "$OUT/libglmx.so.tmp"
mv "$OUT/libglmx.so.tmp" "$OUT/libglmx.so"
echo "built $OUT/libglmx.so"
