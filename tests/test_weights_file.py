"""The on-disk weight format (csrc/weights_file.cu) on the CPU: matrices in
the reference's packed storage (made by the oracle's restatement of
src/data.c) written and read back bit for bit, lookup by name, and files
that are truncated, foreign or inconsistent rejected with a message."""
import ctypes as C

import numpy as np
import pytest

from oracle import pyoracle as o
from vk_compute_b200._lib import WeightEntry, lib


def _packed(seed, K, N, bits):
    if bits == 32:
        return o.transpose_block16(o.get_data(seed, K, N), K, N, 32), None, None
    if bits == 16:
        return o.transpose_block16(o.get_data_fp16(seed, K, N), K, N, 16), None, None
    d, s, z = o.get_data_quant(seed, K, N, bits)
    return o.transpose_block16(d, K, N, bits), s, z


MATS = [("blk.0.qkv", 4, 1024, 768), ("blk.0.down", 8, 512, 256), ("norm", 16, 64, 40), ("f32", 32, 12, 8)]


def _write(path, mats):
    entries = (WeightEntry * len(mats))()
    keep = []
    for e, (name, bits, K, N) in zip(entries, mats):
        d, s, z = _packed(7, K, N, bits)
        keep.append((d, s, z))
        e.name, e.bits, e.K, e.N = name.encode(), bits, K, N
        e.data = d.ctypes.data
        if s is not None:
            e.scale, e.zero = s.ctypes.data, z.ctypes.data
    return lib().vkc_weights_write(str(path).encode(), entries, len(mats)), keep


def _open(path):
    f = C.c_void_p()
    rc = lib().vkc_weights_open(str(path).encode(), C.byref(f))
    return rc, f


def test_round_trip_bit_exact(tmp_path):
    path = tmp_path / "w.vkcw"
    rc, keep = _write(path, MATS)
    assert rc == 0, lib().vkc_last_error()
    rc, f = _open(path)
    assert rc == 0, lib().vkc_last_error()
    try:
        assert lib().vkc_weights_count(f) == len(MATS)
        for i, (name, bits, K, N) in enumerate(MATS):
            assert lib().vkc_weights_find(f, name.encode()) == i
            info = WeightEntry()
            assert lib().vkc_weights_info(f, i, C.byref(info)) == 0
            assert (info.name.decode(), info.bits, info.K, info.N) == (name, bits, K, N)
            d, s, z = keep[i]
            gd = np.zeros_like(d)
            gs = None if s is None else np.zeros_like(s)
            gz = None if z is None else np.zeros_like(z)
            assert lib().vkc_weights_read_host(f, i, gd.ctypes.data, None if gs is None else gs.ctypes.data,
                                               None if gz is None else gz.ctypes.data) == 0
            assert np.array_equal(gd, d)
            if s is not None:
                assert np.array_equal(gs, s) and np.array_equal(gz, z)
        assert lib().vkc_weights_find(f, b"missing") == -1
    finally:
        lib().vkc_weights_close(f)
    # every section starts on a 256-byte boundary
    raw = path.read_bytes()
    assert raw[:8] == b"VKCWGT01"


def test_rejects_bad_files(tmp_path):
    path = tmp_path / "w.vkcw"
    assert _write(path, MATS)[0] == 0
    raw = path.read_bytes()
    cases = {"truncated": raw[: len(raw) // 2], "header only": raw[:40], "magic": b"XXXXXXXX" + raw[8:]}
    bad_shape = bytearray(raw)
    bad_shape[64 + 64:64 + 68] = (5).to_bytes(4, "little")  # bits of the first matrix
    cases["shape"] = bytes(bad_shape)
    for what, data in cases.items():
        p = tmp_path / f"bad_{what.replace(' ', '_')}.vkcw"
        p.write_bytes(data)
        rc, f = _open(p)
        assert rc != 0, what
        assert lib().vkc_last_error(), what
    rc, f = _open(tmp_path / "absent.vkcw")
    assert rc != 0


def test_rejects_bad_entries(tmp_path):
    e = (WeightEntry * 1)()
    e[0].name, e[0].bits, e[0].K, e[0].N = b"x", 8, 64, 100  # N not a multiple of 256
    arr = np.zeros(64 * 100, np.uint8)
    e[0].data = arr.ctypes.data
    assert lib().vkc_weights_write(str(tmp_path / "x.vkcw").encode(), e, 1) != 0
    e[0].N = 256
    assert lib().vkc_weights_write(str(tmp_path / "x.vkcw").encode(), e, 1) != 0  # no scale / zero
