"""Generates tests/golden/reference_data.npz from vk-compute's own src/data.c.

The reference library is compiled from the vk-compute sources by
oracle/build_ref.sh into oracle/_ref/libvkref_data.so; this script calls it
through ctypes and stores its outputs (small arrays in full, large ones as
SHA-256 digests).  The fixtures pin the oracle and the product's data
functions bit-for-bit to the reference.

    bash oracle/build_ref.sh && python tests/golden/make_golden.py

It also runs src/compute.c's own CPU check loops (oracle/_ref/libvkref_loops.so)
and stores their results, which pin the oracle's operator arithmetic.
"""
from __future__ import annotations

import ctypes as C
import hashlib
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
REF = ROOT / "oracle" / "_ref" / "libvkref_data.so"
REF_LOOPS = ROOT / "oracle" / "_ref" / "libvkref_loops.so"

# src/compute.c's own CPU check loops (oracle/ref_loops.c around the line
# ranges oracle/build_ref.sh extracts), on compute.c's inputs: x seed 4321,
# gamma 58923, weights 936 (src/compute.c:18-20, 28, 32).  Shapes: compute.c's
# own K=4096, N=12288, and a small one.  The quantised loops read the first
# scale block and INT4's high nibble, so indices are even and below 256.
LOOP_OPS = ("gemv_f32", "rmsnorm_gemv_f32", "swiglu_f32", "gemv_int8", "gemv_int4", "swiglu_int8", "swiglu_int4")
LOOP_SHAPES = ((4096, 12288), (1024, 512))
LOOP_IDX = np.array([0, 2, 10, 64, 128, 200, 254], np.int32)
OUT = Path(__file__).resolve().parent / "reference_data.npz"


class QuantizedData(C.Structure):  # include/data.h:14-22
    _fields_ = [("data", C.POINTER(C.c_uint8)), ("scale", C.POINTER(C.c_float)), ("z", C.POINTER(C.c_float)),
                ("group_size", C.c_int), ("M", C.c_int), ("N", C.c_int), ("type", C.c_int)]


def digest(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


# Special fp32 inputs for float_to_fp16 (src/data.c:30-51): zeros, the
# subnormal branch, rounding boundaries, overflow, infinities and NaN.
SPECIAL = np.array([0.0, -0.0, 1.0, -1.0, 0.5, 1e-8, 2.0**-24, 2.0**-25, 2.0**-15, 2.0**-14,
                    3.0 * 2.0**-16, 6.1e-5, 65504.0, 65519.0, 65520.0, 70000.0, 1e30, -1e30,
                    np.inf, -np.inf, np.nan, 0.1, 0.333333, -0.999999, 1.0 + 2.0**-11,
                    1.0 + 2.0**-10, 2049.5], np.float32)


def main() -> None:
    L = C.CDLL(str(REF))
    libc = C.CDLL(None)
    libc.free.argtypes = [C.c_void_p]
    L.get_pseudo_random.restype, L.get_pseudo_random.argtypes = C.c_float, [C.c_int] * 3
    L.getData.restype, L.getData.argtypes = C.POINTER(C.c_float), [C.c_int] * 3
    L.getDataFP16.restype, L.getDataFP16.argtypes = C.POINTER(C.c_uint16), [C.c_int] * 3
    L.getDataINT8.restype, L.getDataINT8.argtypes = QuantizedData, [C.c_int] * 3
    L.getDataINT4.restype, L.getDataINT4.argtypes = QuantizedData, [C.c_int] * 3
    L.float_to_fp16.restype, L.float_to_fp16.argtypes = C.c_uint16, [C.c_float]
    L.fp16_to_float.restype, L.fp16_to_float.argtypes = C.c_float, [C.c_uint16]
    L.transpose_block16.restype = None
    L.transpose_block16.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int]

    def arr(ptr, n, dtype):
        a = np.ctypeslib.as_array(ptr, shape=(n,)).astype(dtype, copy=True)
        libc.free(C.cast(ptr, C.c_void_p))
        return a

    def quant(fn, seed, M, N, bits):
        q = fn(seed, M, N)
        data = np.ctypeslib.as_array(q.data, shape=(M * N * bits // 8,)).copy()
        s = np.ctypeslib.as_array(q.scale, shape=(M * (N // 256),)).copy()
        z = np.ctypeslib.as_array(q.z, shape=(M * (N // 256),)).copy()
        for p in (q.data, q.scale, q.z):
            libc.free(C.cast(p, C.c_void_p))
        return data, s, z, q.group_size

    def pack(raw: np.ndarray, M, N, bits):
        raw = np.ascontiguousarray(raw).view(np.uint8)
        out = np.zeros(M * N * bits // 8, np.uint8)
        L.transpose_block16(raw.ctypes.data_as(C.c_void_p), out.ctypes.data_as(C.c_void_p), M, N, bits)
        return out

    g: dict[str, np.ndarray] = {}
    idx = np.array([0, 1, 2, 7, 100, 1023, 4095, 4096, 12287, 65535, 100000, 1 << 20], np.int32)
    seeds = np.array([4321, 58923, 936, 1348, 0, -7], np.int32)
    pr = np.empty((len(seeds), len(idx), len(idx)), np.float32)
    for a, s in enumerate(seeds):
        for b, i in enumerate(idx):
            for c, j in enumerate(idx):
                pr[a, b, c] = L.get_pseudo_random(int(i), int(j), int(s))
    g["pr_idx"], g["pr_seeds"], g["pr_values"] = idx, seeds, pr

    x = arr(L.getData(4321, 1, 4096), 4096, np.float32)
    gm = arr(L.getData(58923, 1, 4096), 4096, np.float32)
    g["x_4321_head"], g["x_4321_sha256"] = x[:512].copy(), np.array(digest(x))
    g["gamma_58923_head"], g["gamma_58923_sha256"] = gm[:512].copy(), np.array(digest(gm))
    w32 = arr(L.getData(936, 32, 128), 32 * 128, np.float32)
    g["w32_936_32x128"] = w32

    g["f2h_in"] = SPECIAL
    g["f2h_out"] = np.array([L.float_to_fp16(float(v)) for v in SPECIAL], np.uint16)
    L.vkref_fp16_to_float_all.restype, L.vkref_fp16_to_float_all.argtypes = None, [C.c_void_p]
    allh = np.zeros(65536, np.uint32)
    L.vkref_fp16_to_float_all(allh.ctypes.data_as(C.c_void_p))
    allh = allh.view(np.float32)
    g["h2f_all_sha256"] = np.array(digest(allh))
    g["h2f_sample"] = allh[::257].copy()

    h16 = arr(L.getDataFP16(936, 32, 256), 32 * 256, np.uint16)
    g["w16_936_32x256"] = h16

    for bits, fn in ((8, L.getDataINT8), (4, L.getDataINT4)):
        rows = 32 if bits == 8 else 64
        data, s, z, gs = quant(fn, 936, rows, 512, bits)
        g[f"q{bits}_936_data"], g[f"q{bits}_936_scale"], g[f"q{bits}_936_zero"] = data, s, z
        g[f"q{bits}_group_size"] = np.array(gs)
        data, s, z, _ = quant(fn, 1348, rows, 512, bits)
        g[f"q{bits}_1348_sha256"] = np.array([digest(data), digest(s), digest(z)])
        # a larger shape through digests only (K=256 rows, N=1024 outputs)
        data, s, z, _ = quant(fn, 936, 256, 1024, bits)
        g[f"q{bits}_936_256x1024_sha256"] = np.array([digest(data), digest(s), digest(z)])
        g[f"q{bits}_936_256x1024_packed_sha256"] = np.array(digest(pack(data, 256, 1024, bits)))

    g["pack32"] = pack(w32, 32, 128, 32)
    g["pack16"] = pack(h16, 32, 256, 16)
    g["pack8"] = pack(g["q8_936_data"], 32, 512, 8)
    g["pack4"] = pack(g["q4_936_data"], 64, 512, 4)

    loops = C.CDLL(str(REF_LOOPS))
    g["refloop_idx"] = LOOP_IDX
    g["refloop_seeds"] = np.array([4321, 58923, 936], np.int32)
    for K, N in LOOP_SHAPES:
        for op in LOOP_OPS:
            fn = getattr(loops, f"vkref_{op}")
            fn.restype = None
            fn.argtypes = [C.c_int] * 5 + [C.c_void_p, C.c_int, C.c_void_p]
            out = np.zeros(len(LOOP_IDX), np.float32)
            fn(K, N, 4321, 58923, 936, LOOP_IDX.ctypes.data_as(C.c_void_p), len(LOOP_IDX),
               out.ctypes.data_as(C.c_void_p))
            g[f"refloop_{op}_{K}x{N}"] = out

    np.savez_compressed(OUT, **g)
    print(f"wrote {OUT} ({OUT.stat().st_size} bytes)")


if __name__ == "__main__":
    main()
