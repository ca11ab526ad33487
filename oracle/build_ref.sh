#!/usr/bin/env bash
# Compiles vk-compute's own C sources, where they lie, into oracle/_ref.
# These artefacts are checkers only (golden-vector generation and the
# drop-in demonstration); nothing in the product links them.  This recipe is
# the one place that reads the reference sources: it takes their location
# from VKC_REFERENCE, else the read-only mount below, and exits 3 (nothing
# built) where they are absent, as on a machine that only runs the prebuilt
# files.
#
#   [VKC_REFERENCE=<vk-compute checkout>] bash oracle/build_ref.sh
#
#  _ref/libvkref_data.so  src/data.c, built with the reference Makefile's -O2,
#                         plus oracle/ref_harness.c (raw-bit fp16 table)
#  _ref/loops/*.inc       src/compute.c's CPU check loops (216-290), each line
#                         range extracted as written, comment markers removed
#  _ref/libvkref_loops.so oracle/ref_loops.c around those loops + src/data.c
#  _ref/ref_dropin        src/compute.c + src/main.c + src/data.c, unmodified,
#                         linked against libvkcompute (headers from include/)
#  _ref/ref_dropin_lib    src/compute.c + src/main.c only: data.h functions
#                         also come from libvkcompute
set -euo pipefail
REF=${VKC_REFERENCE:-/root/reference}
if [ ! -f "$REF/src/data.c" ] || [ ! -f "$REF/src/compute.c" ]; then
  echo "vk-compute sources not found at $REF: reference artefacts not built" >&2
  exit 3
fi
HERE=$(cd "$(dirname "$0")" && pwd)
ROOT=$(dirname "$HERE")
OUT=$HERE/_ref
mkdir -p "$OUT" "$OUT/loops"

if [ "${VKC_FORCE:-0}" = "1" ] || [ ! -f "$OUT/libvkref_data.so" ] || [ "$REF/src/data.c" -nt "$OUT/libvkref_data.so" ] || [ "$HERE/ref_harness.c" -nt "$OUT/libvkref_data.so" ]; then
  gcc -O2 -fPIC -shared -o "$OUT/libvkref_data.so" "$REF/src/data.c" "$HERE/ref_harness.c" -lm
fi

# src/compute.c's check loops: name, first line, last line, a fragment the
# range must contain (so a different compute.c fails here, not silently).
extract() {
  local name=$1 first=$2 last=$3 must=$4
  sed -n "${first},${last}p" "$REF/src/compute.c" | sed 's#^\([[:space:]]*\)// \{0,1\}#\1#' > "$OUT/loops/$name.inc"
  if ! grep -qF -- "$must" "$OUT/loops/$name.inc"; then
    echo "src/compute.c:$first-$last does not hold the expected loop ($must)" >&2
    exit 1
  fi
}
extract gemv_f32          216 218 'result += input[i] * weight[i*N + idx];'
extract rms               221 223 'rms = sqrt(rms / (float)K) + 1e-5;'
extract rmsnorm_gemv_f32  224 226 'result += (input[i] * gamma[i]) / rms * weight[i*N + idx];'
extract swiglu_f32        229 241 'gate /= (1.0 + exp2(-gate * 1.44269504));'
extract swiglu_int8       244 256 'weightINT8.data[i*N+idx] * weightINT8.scale[i] - weightINT8.z[i]'
extract swiglu_int4       258 272 '(weightINT4.data[(i*(N/2)+idx/2)] >> 4) & 0x0F'
extract gemv_int4         277 283 'quantizedResult += input[i] * d_q;'
extract gemv_int8         284 290 'int q = weightINT8.data[i*N+idx];'
gcc -O2 -fPIC -shared -w -I"$REF/include" -I"$OUT/loops" -o "$OUT/libvkref_loops.so" \
    "$HERE/ref_loops.c" "$REF/src/data.c" -lm

LIBDIR=$ROOT/vk_compute_b200
if [ -f "$LIBDIR/libvkcompute.so" ]; then
  INC=(-I"$ROOT/include/vkshim" -I"$ROOT/include")
  LNK=(-L"$LIBDIR" -lvkcompute -Wl,-rpath,'$ORIGIN/../../vk_compute_b200' -lm)
  gcc -O2 -w "${INC[@]}" -o "$OUT/ref_dropin" \
      "$REF/src/compute.c" "$REF/src/main.c" "$REF/src/data.c" "${LNK[@]}"
  gcc -O2 -w "${INC[@]}" -o "$OUT/ref_dropin_lib" \
      "$REF/src/compute.c" "$REF/src/main.c" "${LNK[@]}"
fi
