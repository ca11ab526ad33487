"""The oracle (oracle/oracle.c) against vk-compute's own src/data.c, through
fixtures made by tests/golden/make_golden.py from the compiled reference."""
import hashlib

import numpy as np

from oracle import pyoracle as o


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def test_pseudo_random_grid(golden):
    idx, seeds, vals = golden["pr_idx"], golden["pr_seeds"], golden["pr_values"]
    L = o.lib()
    for a, s in enumerate(seeds):
        for b, i in enumerate(idx):
            for c, j in enumerate(idx):
                assert np.float32(L.vko_pseudo_random(int(i), int(j), int(s))) == vals[a, b, c]


def test_get_data_vectors(golden):
    x = o.get_data(4321, 1, 4096).ravel()
    g = o.get_data(58923, 1, 4096).ravel()
    assert np.array_equal(x[:512], golden["x_4321_head"])
    assert sha(x) == str(golden["x_4321_sha256"])
    assert sha(g) == str(golden["gamma_58923_sha256"])
    assert np.array_equal(o.get_data(936, 32, 128).ravel(), golden["w32_936_32x128"])


def test_fp16_conversions(golden):
    assert np.array_equal(o.float_to_fp16(golden["f2h_in"]), golden["f2h_out"])
    allh = o.fp16_to_float(np.arange(65536, dtype=np.uint16))
    assert sha(allh) == str(golden["h2f_all_sha256"])
    assert np.array_equal(allh[::257], golden["h2f_sample"], equal_nan=True)
    assert np.array_equal(o.get_data_fp16(936, 32, 256).ravel(), golden["w16_936_32x256"])


def test_quantisers(golden):
    for bits in (8, 4):
        rows = 32 if bits == 8 else 64
        d, s, z = o.get_data_quant(936, rows, 512, bits)
        assert np.array_equal(d, golden[f"q{bits}_936_data"])
        assert np.array_equal(s, golden[f"q{bits}_936_scale"])
        assert np.array_equal(z, golden[f"q{bits}_936_zero"])
        d, s, z = o.get_data_quant(1348, rows, 512, bits)
        assert [sha(d), sha(s), sha(z)] == list(golden[f"q{bits}_1348_sha256"])
        d, s, z = o.get_data_quant(936, 256, 1024, bits)
        assert [sha(d), sha(s), sha(z)] == list(golden[f"q{bits}_936_256x1024_sha256"])
        assert sha(o.transpose_block16(d, 256, 1024, bits)) == str(golden[f"q{bits}_936_256x1024_packed_sha256"])


def test_transpose_block16(golden):
    assert np.array_equal(o.transpose_block16(golden["w32_936_32x128"], 32, 128, 32), golden["pack32"])
    assert np.array_equal(o.transpose_block16(golden["w16_936_32x256"], 32, 256, 16), golden["pack16"])
    assert np.array_equal(o.transpose_block16(golden["q8_936_data"], 32, 512, 8), golden["pack8"])
    assert np.array_equal(o.transpose_block16(golden["q4_936_data"], 64, 512, 4), golden["pack4"])
