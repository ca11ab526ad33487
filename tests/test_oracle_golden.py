"""The oracle (oracle/oracle.c) against vk-compute's own src/data.c and its
own CPU check loops (src/compute.c:216-290), through fixtures made by
tests/golden/make_golden.py from the compiled reference."""
import hashlib

import numpy as np
import pytest

from conftest import assert_close
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


# ---- operator arithmetic against src/compute.c's own CPU check loops --------
# The fixtures hold the results of the reference's loops (src/compute.c:216-290,
# compiled from the reference sources by oracle/build_ref.sh and run by
# tests/golden/make_golden.py) on compute.c's inputs.  Those loops put eps
# outside the square root, rms = sqrt(sum x^2 / K) + 1e-5
# (src/compute.c:221-223), where the shaders and the oracle put it inside,
# sqrt(sum x^2 / K + eps); the oracle is called with the eps that makes the
# two equal for this input, so the comparison pins the dequantisation
# (q*s - z), the INT4 nibble order, the RMS scaling and the SiLU form.  The
# loops accumulate in fp32, the oracle in double: bar 2e-5 norm-relative.
@pytest.mark.parametrize("K,N", [(1024, 512), (4096, 12288)])
def test_operators_match_reference_cpu_loops(golden, K, N):
    idx = golden["refloop_idx"]
    sx, sg, sw = (int(v) for v in golden["refloop_seeds"])
    x = o.get_data(sx, 1, K).ravel()
    g = o.get_data(sg, 1, K).ravel()
    a = float(np.sum(x.astype(np.float64) ** 2)) / K
    eps = (np.sqrt(a) + 1e-5) ** 2 - a  # sqrt(a + eps) == sqrt(a) + 1e-5
    w32 = o.get_data(sw, K, N)
    q8 = o.get_data_quant(sw, K, N, 8)
    q4 = o.get_data_quant(sw, K, N, 4)
    f32 = (w32, None, None)
    ours = {
        "gemv_f32": o.qgemv(x, None, w32, None, None, 32, K, N),
        "rmsnorm_gemv_f32": o.qgemv(x, g, w32, None, None, 32, K, N, K, eps),
        "swiglu_f32": o.qswiglu(x, g, f32, f32, 32, K, N, K, eps),
        "gemv_int8": o.qgemv(x, None, *q8, 8, K, N),
        "gemv_int4": o.qgemv(x, None, *q4, 4, K, N),
        "swiglu_int8": o.qswiglu(x, g, q8, q8, 8, K, N, K, eps),
        "swiglu_int4": o.qswiglu(x, g, q4, q4, 4, K, N, K, eps),
    }
    for op, y in ours.items():
        ref = golden[f"refloop_{op}_{K}x{N}"]
        assert_close(y[idx], ref, 2e-5, f"oracle {op} vs src/compute.c's loop at {K}x{N}")
