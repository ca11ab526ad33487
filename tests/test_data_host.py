"""libvkcompute's own include/data.h functions (host code, no GPU needed)
against the reference fixtures: the drop-in must generate the reference's
exact bytes."""
import ctypes as C
import hashlib

import numpy as np
import pytest

from vk_compute_b200._lib import lib


class QuantizedData(C.Structure):
    _fields_ = [("data", C.POINTER(C.c_uint8)), ("scale", C.POINTER(C.c_float)), ("z", C.POINTER(C.c_float)),
                ("group_size", C.c_int), ("M", C.c_int), ("N", C.c_int), ("type", C.c_int)]


@pytest.fixture(scope="module")
def L():
    L = lib()
    L.getData.restype, L.getData.argtypes = C.POINTER(C.c_float), [C.c_int] * 3
    L.getDataFP16.restype, L.getDataFP16.argtypes = C.POINTER(C.c_uint16), [C.c_int] * 3
    for n in ("getDataINT8", "getDataINT4"):
        getattr(L, n).restype, getattr(L, n).argtypes = QuantizedData, [C.c_int] * 3
    L.float_to_fp16.restype, L.float_to_fp16.argtypes = C.c_uint16, [C.c_float]
    L.fp16_to_float.restype, L.fp16_to_float.argtypes = C.c_float, [C.c_uint16]
    L.transpose_block16.restype = None
    L.transpose_block16.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int]
    L.free_quantized_data.restype, L.free_quantized_data.argtypes = None, [QuantizedData]
    return L


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def test_generators(L, golden):
    x = np.ctypeslib.as_array(L.getData(4321, 1, 4096), shape=(4096,)).copy()
    assert sha(x) == str(golden["x_4321_sha256"])
    w = np.ctypeslib.as_array(L.getData(936, 32, 128), shape=(32 * 128,)).copy()
    assert np.array_equal(w, golden["w32_936_32x128"])
    h = np.ctypeslib.as_array(L.getDataFP16(936, 32, 256), shape=(32 * 256,)).copy()
    assert np.array_equal(h, golden["w16_936_32x256"])


def test_fp16(L, golden):
    out = np.array([L.float_to_fp16(float(v)) for v in golden["f2h_in"]], np.uint16)
    assert np.array_equal(out, golden["f2h_out"])
    # Per-element ctypes calls return doubles, which quiets signalling NaNs
    # the same way for both libraries; the oracle's raw bits are pinned to
    # the reference in test_oracle_golden.
    from oracle import pyoracle as o
    prod = np.array([L.fp16_to_float(i) for i in range(65536)], np.float32)
    orc = np.array([o.lib().vko_fp16_to_float(i) for i in range(65536)], np.float32)
    assert np.array_equal(prod.view(np.uint32), orc.view(np.uint32))


@pytest.mark.parametrize("bits", [8, 4])
def test_quantisers_and_packer(L, golden, bits):
    rows = 32 if bits == 8 else 64
    fn = L.getDataINT8 if bits == 8 else L.getDataINT4
    q = fn(936, rows, 512)
    assert q.group_size == 256
    data = np.ctypeslib.as_array(q.data, shape=(rows * 512 * bits // 8,)).copy()
    s = np.ctypeslib.as_array(q.scale, shape=(rows * 2,)).copy()
    z = np.ctypeslib.as_array(q.z, shape=(rows * 2,)).copy()
    assert np.array_equal(data, golden[f"q{bits}_936_data"])
    assert np.array_equal(s, golden[f"q{bits}_936_scale"])
    assert np.array_equal(z, golden[f"q{bits}_936_zero"])
    packed = np.zeros_like(data)
    L.transpose_block16(data.ctypes.data_as(C.c_void_p), packed.ctypes.data_as(C.c_void_p), rows, 512, bits)
    assert np.array_equal(packed, golden[f"pack{bits}"])
    L.free_quantized_data(q)
