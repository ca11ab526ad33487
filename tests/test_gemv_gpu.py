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


@pytest.fixture(autouse=True, params=["cluster", "per-sm", "per-sm-half", "per-sm-fma"])
def gemv_plan(request):
    """Every case runs on each single-vector kernel: clusters splitting K, and
    one CTA per SM with whole-K column ranges in its full-SM (1024 threads)
    and half-SM (512 threads) shapes, wherever those can run -- 8/4-bit
    weights there with integer dot products, and ("per-sm-fma") with fp32
    FMAs; the automatic choice picks one of them per shape."""
    plan = "per-sm-half" if request.param == "per-sm-fma" else request.param
    ops.set_gemv_plan(plan)
    ops.set_gemv_int_dot(request.param != "per-sm-fma")
    yield request.param
    ops.set_gemv_plan("auto")
    ops.set_gemv_int_dot(True)

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


def kv_split_order(q_rows, n_kv, hd, layout):
    """Row indices that list a fused QKV output as [Q | K heads | V heads]."""
    if layout == "split":
        return np.arange(q_rows + 2 * n_kv * hd)
    k = [q_rows + 2 * hd * h + d for h in range(n_kv) for d in range(hd)]
    v = [q_rows + 2 * hd * h + hd + d for h in range(n_kv) for d in range(hd)]
    return np.concatenate([np.arange(q_rows), k, v])


@pytest.mark.parametrize("layout", ["split", "interleaved"])
@pytest.mark.parametrize("bits,K,n_q,n_kv", [(4, 4096, 32, 8), (8, 1024, 8, 2), (16, 1024, 8, 2)])
def test_qkv_rope_kv_append(layout, bits, K, n_q, n_kv):
    """Fused QKV + RoPE + KV append: y against the oracle (Q and K rotated, V
    not), and the caches hold exactly y's K and V rows as fp16 at `pos` (and
    nothing anywhere else)."""
    import torch
    hd, cap, pos = 128, 64, 37
    q_rows, kv_rows = n_q * hd, n_kv * hd
    N = q_rows + 2 * kv_rows
    theta = rope_theta(hd // 2, 1e6, hd)
    x, g = device_vector(SEED_X, K), device_vector(SEED_GAMMA, K)
    w = device_weight(SEED_W, K, N, bits)
    kc = torch.zeros(cap, n_kv, hd, dtype=torch.float16, device="cuda")
    vc = torch.zeros(n_kv, hd // 8, cap, 8, dtype=torch.float16, device="cuda")
    y = ops.qkv_rope_append(w, x, g, torch.from_numpy(theta).cuda(), pos, head_dim=hd, q_rows=q_rows,
                            kv_rows=kv_rows, kcache=kc, vcache=vc, ctx_cap=cap, kv_layout=layout)
    d, s, z = host_weight(SEED_W, K, N, bits)
    plain = o.qgemv(host_vector(SEED_X, K), host_vector(SEED_GAMMA, K), d, s, z, bits, K, N, K, 1e-6)
    order = kv_split_order(q_rows, n_kv, hd, layout)
    ref = o.rope_pairs(plain[order], hd, q_rows + kv_rows, pos, theta)
    ys = y.cpu().numpy()[order]
    assert_close(ys, ref, TOL[bits], f"QKV append bits={bits} layout={layout}")
    y16 = torch.from_numpy(ys).half()
    assert torch.equal(kc[pos].cpu(), y16[q_rows:q_rows + kv_rows].view(n_kv, hd))
    assert torch.equal(vc[:, :, pos].cpu(), y16[q_rows + kv_rows:].view(n_kv, hd // 8, 8))
    kc[pos] = 0
    vc[:, :, pos] = 0
    assert not kc.any() and not vc.any(), "the append wrote outside token pos"


@pytest.mark.parametrize("bits,K,N", [(4, 12288, 4096), (8, 1024, 512), (16, 4096, 4096)])
def test_gemv_residual(bits, K, N):
    import torch
    x = device_vector(SEED_X, K)
    res = device_vector(SEED_GAMMA, N)
    w = device_weight(SEED_W, K, N, bits)
    y = ops.gemv_residual(w, x, res).cpu().numpy()
    d, s, z = host_weight(SEED_W, K, N, bits)
    ref = o.qgemv(host_vector(SEED_X, K), None, d, s, z, bits, K, N) + host_vector(SEED_GAMMA, N)
    assert_close(y, ref, TOL[bits], f"GEMV + residual bits={bits} K={K} N={N}")
    assert torch.isfinite(torch.from_numpy(y)).all()
