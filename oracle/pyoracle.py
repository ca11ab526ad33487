"""numpy binding of oracle/liboracle.so (the C restatement in oracle.c).

TEST INFRASTRUCTURE ONLY: the checker for tests/, the smoke check and the
benchmark's CPU baseline.  Each wrapper names the reference code it follows
through the C function it calls (see oracle.c).
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "liboracle.so"
REF_DATA_PATH = HERE / "_ref" / "libvkref_data.so"

_lib = None
_P = C.c_void_p


def _ptr(a: np.ndarray | None):
    return None if a is None else a.ctypes.data_as(_P)


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(f"{LIB_PATH} missing: run python -m vk_compute_b200._build")
        L = C.CDLL(str(LIB_PATH))
        i, f = C.c_int, C.c_float
        sig = {
            "vko_pseudo_random": (f, [i, i, i]),
            "vko_get_data": (None, [i, i, i, _P]),
            "vko_float_to_fp16": (C.c_uint16, [f]),
            "vko_fp16_to_float": (f, [C.c_uint16]),
            "vko_get_data_fp16": (None, [i, i, i, _P]),
            "vko_get_data_int8": (None, [i, i, i, _P, _P, _P]),
            "vko_get_data_int4": (None, [i, i, i, _P, _P, _P]),
            "vko_transpose_block16": (None, [_P, _P, i, i, i]),
            "vko_quantize_asym": (None, [_P, i, i, i, _P, _P, _P]),
            "vko_quantize_sym": (None, [_P, i, i, i, i, _P, _P, _P]),
            "vko_dequant": (None, [_P, _P, _P, i, i, i, _P]),
            "vko_fp16_matrix_to_float": (None, [_P, C.c_int64, _P]),
            "vko_gemv": (None, [_P, _P, i, i, _P]),
            "vko_inv_rms": (f, [_P, i, i, f]),
            "vko_rmsnorm_rows": (None, [_P, _P, i, i, f]),
            "vko_rmsnorm_gemv": (None, [_P, _P, _P, i, i, i, f, _P]),
            "vko_rope_reference": (None, [_P, i, i, _P]),
            "vko_rope_pairs": (None, [_P, i, i, i, i, _P]),
            "vko_swiglu": (None, [_P, _P, _P, _P, i, i, i, f, _P]),
            "vko_attention": (None, [_P, _P, _P, i, i, i, i, f, _P]),
            "vko_attention_f32q": (None, [_P, _P, _P, i, i, i, i, f, _P]),
            "vko_gemm": (None, [_P, _P, i, i, i, _P]),
            "vko_set_threads": (None, [i]),
            "vko_get_threads": (i, []),
            "vko_qgemv": (None, [_P, _P, _P, _P, _P, i, i, i, i, f, _P]),
            "vko_qswiglu": (None, [_P, _P, _P, _P, _P, _P, _P, _P, i, i, i, i, f, _P]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype, fn.argtypes = res, args
        _lib = L
    return _lib


# ---- data generation (src/data.c) ----------------------------------------
def get_data(seed: int, M: int, N: int) -> np.ndarray:
    out = np.empty((M, N), np.float32)
    lib().vko_get_data(seed, M, N, _ptr(out))
    return out


def get_data_fp16(seed: int, M: int, N: int) -> np.ndarray:
    out = np.empty((M, N), np.uint16)
    lib().vko_get_data_fp16(seed, M, N, _ptr(out))
    return out


def get_data_quant(seed: int, M: int, N: int, bits: int):
    data = np.zeros(M * N * bits // 8, np.uint8)
    s = np.zeros(M * (N // 256), np.float32)
    z = np.zeros_like(s)
    fn = lib().vko_get_data_int8 if bits == 8 else lib().vko_get_data_int4
    fn(seed, M, N, _ptr(data), _ptr(s), _ptr(z))
    return data, s, z


def float_to_fp16(values) -> np.ndarray:
    v = np.asarray(values, np.float32).ravel()
    return np.array([lib().vko_float_to_fp16(float(x)) for x in v], np.uint16)


def fp16_to_float(bits: np.ndarray) -> np.ndarray:
    b = np.ascontiguousarray(bits, np.uint16)
    out = np.empty(b.shape, np.float32)
    lib().vko_fp16_matrix_to_float(_ptr(b), b.size, _ptr(out))
    return out


def transpose_block16(raw: np.ndarray, K: int, N: int, bits: int) -> np.ndarray:
    raw = np.ascontiguousarray(raw).view(np.uint8)
    out = np.zeros(K * N * bits // 8, np.uint8)
    lib().vko_transpose_block16(_ptr(raw), _ptr(out), K, N, bits)
    return out


def quantize(w: np.ndarray, bits: int, symmetric: bool, fp16_scale: bool = True):
    w = np.ascontiguousarray(w, np.float32)
    K, N = w.shape
    data = np.zeros(K * N * bits // 8, np.uint8)
    s = np.zeros(K * (N // 256), np.float32)
    z = np.zeros_like(s)
    if symmetric:
        lib().vko_quantize_sym(_ptr(w), K, N, bits, int(fp16_scale), _ptr(data), _ptr(s), _ptr(z))
    else:
        lib().vko_quantize_asym(_ptr(w), K, N, bits, _ptr(data), _ptr(s), _ptr(z))
    return data, s, z


def dequant(data, s, z, K: int, N: int, bits: int) -> np.ndarray:
    out = np.empty((K, N), np.float32)
    lib().vko_dequant(_ptr(np.ascontiguousarray(data)), _ptr(s), _ptr(z), K, N, bits, _ptr(out))
    return out


# ---- operators -------------------------------------------------------------
def set_threads(n: int) -> None:
    lib().vko_set_threads(int(n))


def qgemv(x, gamma, data, s, z, bits: int, K: int, N: int, rms_dim: int | None = None,
          eps: float = 1e-5) -> np.ndarray:
    """GEMV (gamma None) or RmsNorm-GEMV on the reference's unpacked storage:
    bits 32 (fp32 K x N), 16 (fp16 bits), 8/4 (codes + block-major s/z)."""
    y = np.empty(N, np.float32)
    x = np.ascontiguousarray(x, np.float32)
    g = None if gamma is None else np.ascontiguousarray(gamma, np.float32)
    lib().vko_qgemv(_ptr(x), _ptr(g), _ptr(np.ascontiguousarray(data)), _ptr(s), _ptr(z), bits, K, N,
                    rms_dim or K, eps, _ptr(y))
    return y


def qswiglu(x, gamma, gate, up, bits: int, K: int, N: int, rms_dim: int | None = None,
            eps: float = 1e-5) -> np.ndarray:
    """gate/up: (data, s, z) triples (s, z None for fp16/fp32)."""
    h = np.empty(N, np.float32)
    dg, sg, zg = gate
    du, su, zu = up
    lib().vko_qswiglu(_ptr(np.ascontiguousarray(x, np.float32)), _ptr(np.ascontiguousarray(gamma, np.float32)),
                      _ptr(np.ascontiguousarray(dg)), _ptr(sg), _ptr(zg), _ptr(np.ascontiguousarray(du)),
                      _ptr(su), _ptr(zu), bits, K, N, rms_dim or K, eps, _ptr(h))
    return h


def rmsnorm_rows(x: np.ndarray, gamma: np.ndarray, eps: float = 1e-5) -> np.ndarray:
    """shader/RmsNorm.comp on a copy of x ([rows][width])."""
    y = np.array(x, np.float32)
    rows, width = y.shape
    lib().vko_rmsnorm_rows(_ptr(y), _ptr(np.ascontiguousarray(gamma, np.float32)), rows, width, eps)
    return y


def gemv_dense(x, w) -> np.ndarray:
    """y = W^T x for a dense row-major K x N fp32 matrix (shader/gemv2.comp)."""
    w = np.ascontiguousarray(w, np.float32)
    K, N = w.shape
    y = np.empty(N, np.float32)
    lib().vko_gemv(_ptr(np.ascontiguousarray(x, np.float32)), _ptr(w), K, N, _ptr(y))
    return y


def inv_rms(x, rms_dim: int, eps: float) -> float:
    x = np.ascontiguousarray(x, np.float32)
    return lib().vko_inv_rms(_ptr(x), x.size, rms_dim, eps)


def rope_reference(y: np.ndarray, pos: int, theta: np.ndarray) -> np.ndarray:
    y = np.array(y, np.float32)
    lib().vko_rope_reference(_ptr(y), y.size, pos, _ptr(np.ascontiguousarray(theta, np.float32)))
    return y


def rope_pairs(y: np.ndarray, head_dim: int, rot_rows: int, pos: int, theta: np.ndarray) -> np.ndarray:
    y = np.array(y, np.float32)
    lib().vko_rope_pairs(_ptr(y), y.size, head_dim, rot_rows, pos, _ptr(np.ascontiguousarray(theta, np.float32)))
    return y


def attention(q, kcache, vcache, n_q: int, n_kv: int, head_dim: int, ctx: int, scale: float) -> np.ndarray:
    out = np.empty(n_q * head_dim, np.float32)
    lib().vko_attention(_ptr(np.ascontiguousarray(q, np.uint16)), _ptr(np.ascontiguousarray(kcache, np.uint16)),
                        _ptr(np.ascontiguousarray(vcache, np.uint16)), n_q, n_kv, head_dim, ctx, scale, _ptr(out))
    return out


def attention_f32q(q, kcache, vcache, n_q: int, n_kv: int, head_dim: int, ctx: int, scale: float) -> np.ndarray:
    out = np.empty(n_q * head_dim, np.float32)
    lib().vko_attention_f32q(_ptr(np.ascontiguousarray(q, np.float32)), _ptr(np.ascontiguousarray(kcache, np.uint16)),
                             _ptr(np.ascontiguousarray(vcache, np.uint16)), n_q, n_kv, head_dim, ctx, scale, _ptr(out))
    return out


def gemm(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    a = np.ascontiguousarray(a, np.float32)
    b = np.ascontiguousarray(b, np.float32)
    M, K = a.shape
    _, N = b.shape
    c = np.empty((M, N), np.float32)
    lib().vko_gemm(_ptr(a), _ptr(b), M, N, K, _ptr(c))
    return c
