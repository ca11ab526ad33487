"""GEMV-family kernels (libvkcompute through its C ABI) against the oracle
on identical seeded inputs.

Inputs follow the reference driver (src/compute.c:18-46): x = getData(4321),
gamma = getData(58923), W = getData(936) (gate) / getData(1348) (up), fp16 by
the truncating conversion, int8/int4 by the min/max quantiser.  Shapes cover
the reference's own N=12288, K=4096, the configs' sizes, and ragged edges.
"""
import numpy as np
import pytest

from conftest import TOL, assert_close
from gpu_util import (SEED_GAMMA, SEED_W, SEED_W2, SEED_X, device_vector, device_weight, host_vector,
                      host_weight, rope_theta)
from oracle import pyoracle as o
from vk_compute_b200 import ops

pytestmark = pytest.mark.gpu

BITS = [32, 16, 8, 4]

# (K, N) per width: small, ragged/odd, and full-size shapes.
SHAPES = {
    32: [(1024, 512), (12, 96), (4096, 4096)],
    16: [(1024, 512), (24, 40), (4096, 4096), (4096, 12288)],
    8: [(1024, 512), (48, 256), (4096, 12288)],
    4: [(1024, 512), (96, 256), (4096, 6144), (12288, 4096)],
}
CASES = [(b, k, n) for b in BITS for (k, n) in SHAPES[b]]


@pytest.mark.parametrize("bits,K,N", CASES)
def test_gemv(bits, K, N):
    x = device_vector(SEED_X, K)
    w = device_weight(SEED_W, K, N, bits)
    y = ops.gemv(w, x).cpu().numpy()
    d, s, z = host_weight(SEED_W, K, N, bits)
    ref = o.qgemv(host_vector(SEED_X, K), None, d, s, z, bits, K, N)
    assert_close(y, ref, TOL[bits], f"GEMV bits={bits} K={K} N={N}")


@pytest.mark.parametrize("bits,K,N", CASES)
@pytest.mark.parametrize("consts", ["reference", "config"])
def test_rmsnorm_gemv(bits, K, N, consts):
    rms_dim, eps = (4096, 1e-5) if consts == "reference" else (K, 1e-6)
    x, g = device_vector(SEED_X, K), device_vector(SEED_GAMMA, K)
    w = device_weight(SEED_W, K, N, bits)
    y = ops.rmsnorm_gemv(w, x, g, eps=eps, rms_dim=rms_dim).cpu().numpy()
    d, s, z = host_weight(SEED_W, K, N, bits)
    ref = o.qgemv(host_vector(SEED_X, K), host_vector(SEED_GAMMA, K), d, s, z, bits, K, N, rms_dim, eps)
    assert_close(y, ref, TOL[bits], f"RmsNorm-GEMV bits={bits} K={K} N={N}")


ROPE_SHAPES = [(16, 1024, 768), (8, 1024, 768), (4, 1024, 768), (4, 4096, 6144), (16, 64, 512)]


@pytest.mark.parametrize("bits,K,N", ROPE_SHAPES)
@pytest.mark.parametrize("pos", [0, 1, 4097, 8191])
def test_rope_pairs(bits, K, N, pos):
    hd = 128
    rot = N - N // 6  # Q and K heads rotate, the trailing V block does not
    rot -= rot % hd
    theta = rope_theta(hd // 2, 1e6, hd)
    x, g = device_vector(SEED_X, K), device_vector(SEED_GAMMA, K)
    w = device_weight(SEED_W, K, N, bits)
    import torch
    th = torch.from_numpy(theta).cuda()
    y = ops.rmsnorm_gemv_rope(w, x, g, th, pos, mode="pairs", head_dim=hd, rot_rows=rot).cpu().numpy()
    d, s, z = host_weight(SEED_W, K, N, bits)
    ref = o.qgemv(host_vector(SEED_X, K), host_vector(SEED_GAMMA, K), d, s, z, bits, K, N, K, 1e-6)
    ref = o.rope_pairs(ref, hd, rot, pos, theta)
    assert_close(y, ref, TOL[bits], f"Rope pairs bits={bits} pos={pos}")
    # V rows are untouched by the rotation
    plain = o.qgemv(host_vector(SEED_X, K), host_vector(SEED_GAMMA, K), d, s, z, bits, K, N, K, 1e-6)
    assert_close(y[rot:], plain[rot:], TOL[bits], "unrotated V rows")


@pytest.mark.parametrize("bits", [16, 8, 4])
@pytest.mark.parametrize("pos", [0, 37, 8191])
def test_rope_reference_epilogue(bits, pos):
    K, N = 1024, 768
    theta = rope_theta(64, 10000.0, 128)
    x, g = device_vector(SEED_X, K), device_vector(SEED_GAMMA, K)
    w = device_weight(SEED_W, K, N, bits)
    import torch
    y = ops.rmsnorm_gemv_rope(w, x, g, torch.from_numpy(theta).cuda(), pos, mode="reference",
                              eps=1e-5, rms_dim=4096).cpu().numpy()
    d, s, z = host_weight(SEED_W, K, N, bits)
    ref = o.qgemv(host_vector(SEED_X, K), host_vector(SEED_GAMMA, K), d, s, z, bits, K, N, 4096, 1e-5)
    ref = o.rope_reference(ref, pos, theta)
    assert_close(y, ref, TOL[bits], f"Rope reference bits={bits} pos={pos}")


SWIGLU = [(32, 1024, 512), (16, 1024, 512), (16, 4096, 12288), (8, 1024, 512), (8, 4096, 12288),
          (4, 1024, 512), (4, 4096, 12288), (4, 96, 256)]


@pytest.mark.parametrize("bits,K,N", SWIGLU)
def test_rmsnorm_swiglu(bits, K, N):
    x, g = device_vector(SEED_X, K), device_vector(SEED_GAMMA, K)
    wg, wu = device_weight(SEED_W, K, N, bits), device_weight(SEED_W2, K, N, bits)
    h = ops.rmsnorm_swiglu(wg, wu, x, g, eps=1e-5, rms_dim=4096).cpu().numpy()
    ref = o.qswiglu(host_vector(SEED_X, K), host_vector(SEED_GAMMA, K), host_weight(SEED_W, K, N, bits),
                    host_weight(SEED_W2, K, N, bits), bits, K, N, 4096, 1e-5)
    assert_close(h, ref, TOL[bits], f"swiglu bits={bits} K={K} N={N}")


@pytest.mark.parametrize("bits", [8, 4])
def test_config_weights_symmetric_fp16_scales(bits):
    """The configs' weights: N(0, 0.02), symmetric quantisation with fp16
    scales, x ~ N(0, 1), gamma ~ 1 + N(0, 0.1), eps 1e-6."""
    import torch
    gen = torch.Generator().manual_seed(1234)
    K, N = 4096, 12288 if bits == 8 else 4096
    w = torch.randn(K, N, generator=gen) * 0.02
    x = torch.randn(K, generator=gen)
    gamma = 1 + 0.1 * torch.randn(K, generator=gen)
    pw = ops.pack_dense(w.cuda(), bits, symmetric=True, fp16_scale=True)
    y = ops.rmsnorm_gemv(pw, x.cuda(), gamma.cuda(), eps=1e-6).cpu().numpy()
    d, s, z = o.quantize(w.numpy(), bits, True, True)
    ref = o.qgemv(x.numpy(), gamma.numpy(), d, s, z, bits, K, N, K, 1e-6)
    assert_close(y, ref, TOL[bits], f"config RmsNorm-GEMV bits={bits}")


def test_pdl_launches_match():
    """Programmatic dependent launch changes scheduling, not results."""
    import torch
    K, N = 4096, 4096
    x, g = device_vector(SEED_X, K), device_vector(SEED_GAMMA, K)
    w = device_weight(SEED_W, K, N, 4)
    ops.set_pdl(False)
    a = ops.rmsnorm_gemv(w, x, g).clone()
    ops.set_pdl(True)
    try:
        outs = [ops.rmsnorm_gemv(w, x, g) for _ in range(8)]
        torch.cuda.synchronize()
    finally:
        ops.set_pdl(False)
    for b in outs:
        assert torch.equal(a, b)


def test_deterministic():
    import torch
    K, N = 4096, 12288
    x, g = device_vector(SEED_X, K), device_vector(SEED_GAMMA, K)
    w = device_weight(SEED_W, K, N, 8)
    a = ops.rmsnorm_gemv(w, x, g).clone()
    b = ops.rmsnorm_gemv(w, x, g)
    assert torch.equal(a, b)


def test_invalid_arguments_are_rejected():
    import torch
    from vk_compute_b200._lib import VkcError
    x = torch.zeros(1000, device="cuda")
    w = device_weight(SEED_W, 1024, 512, 4)
    bad = ops.PackedWeight(4, 1000, 512, w.packed, w.scale, w.zero)  # K not a multiple of 32
    with pytest.raises(VkcError):
        ops.gemv(bad, x)
    bad = ops.PackedWeight(8, 1024, 500, w.packed, w.scale, w.zero)  # N not a multiple of 256
    with pytest.raises(VkcError):
        ops.gemv(bad, torch.zeros(1024, device="cuda"))
