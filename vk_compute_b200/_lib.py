"""ctypes binding of libvkcompute.so (the in-tree sm_100a library).

Loading fails loudly when the library has not been built: there is no
fallback implementation of any operator.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libvkcompute.so"

_lib: C.CDLL | None = None

_i, _f, _p, _sz = C.c_int, C.c_float, C.c_void_p, C.c_size_t

# name -> (restype, argtypes); mirrors include/vk_compute_b200.h
SIGNATURES = {
    "vkc_last_error": (C.c_char_p, []),
    "vkc_version": (_i, []),
    "vkc_set_pdl": (None, [_i]),
    "vkc_get_pdl": (_i, []),
    "vkc_set_timing": (None, [_i]),
    "vkc_get_timing": (_i, []),
    "vkc_has_operator": (_i, [C.c_char_p]),
    "vkc_device_status": (_i, [C.POINTER(C.c_uint), _i]),
    "vkc_wait_limits": (None, [C.POINTER(C.c_uint64), C.POINTER(C.c_uint64)]),
    "vkc_set_gemv_plan": (_i, [_i]),
    "vkc_set_gemv_int_dot": (None, [_i]),
    "vkc_get_gemv_int_dot": (_i, []),
    "vkc_set_attention_plan": (_i, [_i]),
    "vkc_get_attention_plan": (_i, []),
    "vkc_rmsnorm_gemv_gather": (_i, [_i, _p, _p, _p, _p, _p, _p, _i, _i, _i, _i, _i, _f, _i, _p]),
    "vkc_gather_wait": (_i, [_p, _i, _i, _p, _p, _p]),
    "vkc_attention_plan_info": (_i, [_i, _i, _i, _i, C.POINTER(_i)]),
    "vkc_get_gemv_plan": (_i, []),
    "vkc_gemv": (_i, [_i, _p, _p, _p, _p, _p, _i, _i, _p]),
    "vkc_rmsnorm_gemv": (_i, [_i, _p, _p, _p, _p, _p, _p, _i, _i, _f, _i, _p]),
    "vkc_rmsnorm_gemv_rope": (_i, [_i, _p, _p, _p, _p, _p, _p, _p, _i, _i, _f, _i, _i, _i, _i, _i, _p]),
    "vkc_rmsnorm_swiglu": (_i, [_i, _p, _p, _p, _p, _p, _p, _p, _p, _p, _i, _i, _f, _i, _p]),
    "vkc_gemv_residual": (_i, [_i, _p, _p, _p, _p, _p, _p, _i, _i, _p]),
    "vkc_rmsnorm_gemv_rope_kv": (_i, [_i, _p, _p, _p, _p, _p, _p, _p, _i, _i, _f, _i, _i, _i, _i, _i, _i, _p, _p, _i,
                                      _p]),
    "vkc_attention_workspace_bytes": (_sz, [_i, _i, _i, _i]),
    "vkc_attention_decode": (_i, [_p, _i, _p, _p, _p, _i, _i, _i, _i, _f, _p, _sz, _p]),
    "vkc_attention_decode_cache": (_i, [_p, _i, _p, _p, _p, _i, _i, _i, _i, _i, _f, _p, _sz, _p]),
    "vkc_attention_decode_append": (_i, [_p, _i, _p, _p, _p, _i, _i, _i, _i, _i, _f, _p, _sz, _p]),
    "vkc_gemm_f32": (_i, [_p, _p, _p, _i, _i, _i, _p]),
    "vkc_rmsnorm_rows": (_i, [_p, _p, _i, _i, _f, _p]),
    "vkc_gemv_rowmajor": (_i, [_p, _p, _p, _i, _i, _p]),
    "vkc_gemm_bf16": (_i, [_p, _p, _p, _i, _i, _i, _p]),
    "vkc_gemm_bf16_status": (_i, [C.POINTER(C.c_uint), _i]),
    "vkc_generate": (_i, [_i, _i, _i, _i, _p, _p]),
    "vkc_quantize": (_i, [_p, _i, _i, _i, _i, _i, _p, _p, _p, _p]),
    "vkc_pack_block16": (_i, [_p, _p, _i, _i, _i, _p]),
    "vkc_allgather_p2p": (_i, [_p, _p, _p, _i, _i, _i, _p, _p]),
    "vkc_allreduce_residual_p2p": (_i, [_p, _p, _p, _i, _i, _i, _p, _p, _p, _p]),
    "vkc_ipc_alloc": (_i, [_sz, C.POINTER(C.c_void_p), _p]),
    "vkc_ipc_open": (_i, [_p, C.POINTER(C.c_void_p)]),
    "vkc_ipc_close": (_i, [_p]),
    "vkc_ipc_free": (_i, [_p]),
    "vkc_gemv_peer": (_i, [_i, _p, _p, _p, _p, _p, _i, _i, _i, _i, _p]),
    "vkc_gemv_batched": (_i, [_i, _p, _p, _p, _p, _p, _i, _i, _i, _p]),
    "vkc_rmsnorm_gemv_batched": (_i, [_i, _p, _p, _p, _p, _p, _p, _i, _i, _i, _f, _i, _p]),
    "vkc_rmsnorm_gemv_rope_kv_peer": (_i, [_i, _p, _p, _p, _p, _p, _p, _p, _p, _i, _i, _f, _i, _i, _i, _i, _i, _i,
                                           _p, _p, _i, _p]),
    "vkc_rmsnorm_swiglu_peer": (_i, [_i, _p, _p, _p, _p, _p, _p, _p, _p, _p, _p, _i, _i, _f, _i, _p]),
}


class WeightEntry(C.Structure):
    """vkc_weight_entry (include/vk_compute_b200.h)."""
    _fields_ = [("name", C.c_char * 64), ("bits", C.c_int), ("K", C.c_int), ("N", C.c_int),
                ("data", C.c_void_p), ("scale", C.c_void_p), ("zero", C.c_void_p)]


class DecodeDims(C.Structure):
    """vkc_decode_dims (include/vk_compute_b200.h)."""
    _fields_ = [(n, C.c_int) for n in ("layers", "hidden", "inter", "n_q", "n_kv", "head_dim", "ctx_cap", "bits")] + [
        ("eps", C.c_float)]


class DecodeLayer(C.Structure):
    """vkc_decode_layer (include/vk_compute_b200.h)."""
    _fields_ = [(f"{m}{s}", C.c_void_p) for m in ("qkv", "o", "gate", "up", "down") for s in ("", "_scale", "_zero")] + [
        ("gamma_attn", C.c_void_p), ("gamma_ffn", C.c_void_p), ("kcache", C.c_void_p), ("vcache", C.c_void_p)]


class DecodeBuffers(C.Structure):
    """vkc_decode_buffers (include/vk_compute_b200.h)."""
    _fields_ = [(n, C.c_void_p) for n in ("x", "x_mid", "qkv", "attn", "h")]


SIGNATURES.update({
    "vkc_decode_program_bytes": (_sz, [C.POINTER(DecodeDims)]),
    "vkc_decode_program_build": (_i, [C.POINTER(DecodeDims), C.POINTER(DecodeLayer), C.POINTER(DecodeBuffers), _p, _p,
                                      _sz, _p]),
    "vkc_decode_program_run": (_i, [C.POINTER(DecodeDims), _p, _i, _p]),
})

SIGNATURES.update({
    "vkc_weights_write": (_i, [C.c_char_p, C.POINTER(WeightEntry), _i]),
    "vkc_weights_open": (_i, [C.c_char_p, C.POINTER(C.c_void_p)]),
    "vkc_weights_count": (_i, [_p]),
    "vkc_weights_find": (_i, [_p, C.c_char_p]),
    "vkc_weights_info": (_i, [_p, _i, C.POINTER(WeightEntry)]),
    "vkc_weights_read": (_i, [_p, _i, _p, _p, _p, _p]),
    "vkc_weights_read_host": (_i, [_p, _i, _p, _p, _p]),
    "vkc_weights_close": (None, [_p]),
})


class VkcError(RuntimeError):
    pass


def lib() -> C.CDLL:
    """The loaded library (loaded once, with its argument types declared)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise VkcError(
                f"{LIB_PATH} is missing: build it with `python -m vk_compute_b200._build` "
                "(there is no non-CUDA implementation)")
        handle = C.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


def check(rc: int) -> None:
    if rc != 0:
        msg = lib().vkc_last_error().decode(errors="replace")
        raise VkcError(f"libvkcompute error {rc}: {msg}")
