#!/usr/bin/env bash
# Compiles vk-compute's own C sources, where they lie, into oracle/_ref.
# These artefacts are checkers only (golden-vector generation and the
# drop-in demonstration); nothing in the product links them.
#
#   VKC_REFERENCE=/root/reference bash oracle/build_ref.sh
#
#  _ref/libvkref_data.so  src/data.c, built with the reference Makefile's -O2,
#                         plus oracle/ref_harness.c (raw-bit fp16 table)
#  _ref/ref_dropin        src/compute.c + src/main.c + src/data.c, unmodified,
#                         linked against libvkcompute (headers from include/)
#  _ref/ref_dropin_lib    src/compute.c + src/main.c only: data.h functions
#                         also come from libvkcompute
set -euo pipefail
REF=${VKC_REFERENCE:-/root/reference}
HERE=$(cd "$(dirname "$0")" && pwd)
ROOT=$(dirname "$HERE")
OUT=$HERE/_ref
mkdir -p "$OUT"

if [ "${VKC_FORCE:-0}" = "1" ] || [ ! -f "$OUT/libvkref_data.so" ] || [ "$REF/src/data.c" -nt "$OUT/libvkref_data.so" ] || [ "$HERE/ref_harness.c" -nt "$OUT/libvkref_data.so" ]; then
  gcc -O2 -fPIC -shared -o "$OUT/libvkref_data.so" "$REF/src/data.c" "$HERE/ref_harness.c" -lm
fi

LIBDIR=$ROOT/vk_compute_b200
if [ -f "$LIBDIR/libvkcompute.so" ]; then
  INC=(-I"$ROOT/include/vkshim" -I"$ROOT/include")
  LNK=(-L"$LIBDIR" -lvkcompute -Wl,-rpath,'$ORIGIN/../../vk_compute_b200' -lm)
  gcc -O2 -w "${INC[@]}" -o "$OUT/ref_dropin" \
      "$REF/src/compute.c" "$REF/src/main.c" "$REF/src/data.c" "${LNK[@]}"
  gcc -O2 -w "${INC[@]}" -o "$OUT/ref_dropin_lib" \
      "$REF/src/compute.c" "$REF/src/main.c" "${LNK[@]}"
fi
