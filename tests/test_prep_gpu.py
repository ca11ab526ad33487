"""Device weight preparation (vkc_generate / vkc_quantize / vkc_pack_block16)
is bit-identical to the oracle, which is pinned to src/data.c."""
import numpy as np
import pytest
import torch

from oracle import pyoracle as o
from vk_compute_b200 import ops
from vk_compute_b200._lib import check, lib

pytestmark = pytest.mark.gpu


def _p(t):
    return ops._p(t)


@pytest.mark.parametrize("M,N", [(1, 4096), (64, 256), (33, 777)])
def test_generate(M, N):
    v = torch.empty(M * N, dtype=torch.float32, device="cuda")
    check(lib().vkc_generate(936, M, N, 32, _p(v), ops._s()))
    assert np.array_equal(v.cpu().numpy(), o.get_data(936, M, N).ravel())
    h = torch.empty(M * N, dtype=torch.int16, device="cuda")
    check(lib().vkc_generate(1348, M, N, 16, _p(h), ops._s()))
    assert np.array_equal(h.cpu().numpy().view(np.uint16), o.get_data_fp16(1348, M, N).ravel())


@pytest.mark.parametrize("bits", [8, 4])
@pytest.mark.parametrize("K,N", [(64, 512), (96, 1024)])
def test_quantize_reference(bits, K, N):
    w = ops.reference_weight(936, K, N, bits)
    data, s, z = o.get_data_quant(936, K, N, bits)
    assert np.array_equal(w.scale.cpu().numpy(), s)
    assert np.array_equal(w.zero.cpu().numpy(), z)
    assert np.array_equal(w.packed.cpu().numpy(), o.transpose_block16(data, K, N, bits))


@pytest.mark.parametrize("bits", [8, 4])
@pytest.mark.parametrize("fp16_scale", [True, False])
def test_quantize_symmetric(bits, fp16_scale):
    g = torch.Generator().manual_seed(7)
    K, N = 64, 768
    w = torch.randn(K, N, generator=g) * 0.02
    w[3, :256] = 0.0  # an all-zero block
    pw = ops.pack_dense(w.cuda(), bits, symmetric=True, fp16_scale=fp16_scale)
    data, s, z = o.quantize(w.numpy(), bits, True, fp16_scale)
    assert np.array_equal(pw.scale.cpu().numpy(), s)
    assert np.array_equal(pw.zero.cpu().numpy(), z)
    assert np.array_equal(pw.packed.cpu().numpy(), o.transpose_block16(data, K, N, bits))


@pytest.mark.parametrize("bits", [32, 16])
def test_pack_float(bits):
    K, N = 64, 96
    w = ops.reference_weight(936, K, N, bits)
    host = o.get_data(936, K, N) if bits == 32 else o.get_data_fp16(936, K, N)
    assert np.array_equal(w.packed.cpu().numpy(), o.transpose_block16(host, K, N, bits))


def test_shard_matches_packing_the_column_slice():
    K, N = 64, 1024
    w = ops.reference_weight(936, K, N, 4)
    data, s, z = o.get_data_quant(936, K, N, 4)
    dense = o.dequant(data, s, z, K, N, 4)
    sh = w.shard(256, 768)
    got = o.dequant(_unpack4(sh.packed.cpu().numpy(), K, 512), sh.scale.cpu().numpy(), sh.zero.cpu().numpy(), K, 512, 4)
    assert np.array_equal(got, dense[:, 256:768])


def _unpack4(packed: np.ndarray, K: int, N: int) -> np.ndarray:
    """Inverse of transpose_block16 for 4-bit codes (test helper)."""
    ch = packed.reshape(K // 32, N, 16)
    out = np.zeros((K, N // 2), np.uint8)
    for t in range(32):
        byte = ch[:, :, t // 2]
        q = (byte >> 4) if t & 1 else (byte & 0x0F)
        rows = np.arange(K // 32) * 32 + t
        even = q[:, 0::2]
        odd = q[:, 1::2]
        out[rows] = (even << 4) | odd
    return out.ravel()
