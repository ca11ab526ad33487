"""Batched decode GEMV (M vectors against one weight stream) against the
oracle's single-vector GEMV applied to each row, on seeded inputs: every
weight width, M = 1..8, the reference's full N=12288 x K=4096 and ragged
shapes, plain and RmsNorm variants (each row normalised by its own RMS)."""
import numpy as np
import pytest
import torch

from conftest import TOL, assert_close
from gpu_util import SEED_GAMMA, SEED_W, device_vector, device_weight, host_vector, host_weight
from oracle import pyoracle as o
from vk_compute_b200 import ops
from vk_compute_b200._lib import VkcError

pytestmark = pytest.mark.gpu

CASES = [(32, 1024, 512), (16, 1024, 512), (16, 4096, 4096), (8, 48, 256), (8, 4096, 12288), (4, 96, 256),
         (4, 4096, 6144), (4, 12288, 4096)]


def _rows(M, K):
    return [host_vector(7000 + m, K) for m in range(M)]


@pytest.mark.parametrize("bits,K,N", CASES)
@pytest.mark.parametrize("M", [2, 3, 8])
def test_gemv_batched(bits, K, N, M):
    xs = _rows(M, K)
    x = torch.stack([device_vector(7000 + m, K) for m in range(M)])
    w = device_weight(SEED_W, K, N, bits)
    y = ops.gemv_batched(w, x).cpu().numpy()
    d, s, z = host_weight(SEED_W, K, N, bits)
    for m in range(M):
        ref = o.qgemv(xs[m], None, d, s, z, bits, K, N)
        assert_close(y[m], ref, TOL[bits], f"batched GEMV bits={bits} K={K} N={N} m={m}/{M}")


@pytest.mark.parametrize("bits,K,N", CASES)
@pytest.mark.parametrize("M", [1, 4, 5, 7])
def test_rmsnorm_gemv_batched(bits, K, N, M):
    xs = _rows(M, K)
    x = torch.stack([device_vector(7000 + m, K) for m in range(M)])
    g = device_vector(SEED_GAMMA, K)
    w = device_weight(SEED_W, K, N, bits)
    y = ops.rmsnorm_gemv_batched(w, x, g, eps=1e-6, rms_dim=K).cpu().numpy()
    d, s, z = host_weight(SEED_W, K, N, bits)
    for m in range(M):
        ref = o.qgemv(xs[m], host_vector(SEED_GAMMA, K), d, s, z, bits, K, N, K, 1e-6)
        assert_close(y[m], ref, TOL[bits], f"batched RmsNorm-GEMV bits={bits} K={K} N={N} m={m}/{M}")


@pytest.mark.parametrize("int_dot,bar", [(False, 1e-5), (True, 1e-4)])
def test_batched_rows_match_single_vector_kernel(int_dot, bar):
    """Row m of a batch equals the one-vector kernel on x[m]: to fp32
    rounding against its fp32 arithmetic, and to the 16-bit activation steps
    (about 1e-5 relative) against its integer dot products."""
    K, N = 4096, 12288
    w = device_weight(SEED_W, K, N, 8)
    x = torch.stack([device_vector(7000 + m, K) for m in range(6)])
    y = ops.gemv_batched(w, x)
    before = ops.get_gemv_int_dot()
    ops.set_gemv_int_dot(int_dot)
    try:
        for m in range(6):
            single = ops.gemv(w, x[m].contiguous())
            err = (y[m] - single).abs().max().item() / single.abs().max().item()
            assert err < bar, (m, err)
    finally:
        ops.set_gemv_int_dot(before)


def test_batched_rejects_bad_m():
    w = device_weight(SEED_W, 1024, 512, 8)
    with pytest.raises(VkcError):
        ops.gemv_batched(w, torch.zeros(9, 1024, device="cuda"))
    with pytest.raises(VkcError):
        ops.gemv_batched(w, torch.zeros(0, 1024, device="cuda"))
