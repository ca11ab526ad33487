"""Prefill GEMM on the tcgen05 tensor cores (C = A W^T, bf16 in, fp32 out)
against the oracle's double-precision product of the same bf16 values, and at
the prefill configuration (64 x 4096 . 4096 x 12288) against a float64
product on the device."""
import numpy as np
import pytest
import torch

from conftest import assert_close
from oracle import pyoracle as o
from vk_compute_b200 import ops

pytestmark = pytest.mark.gpu


def make(M, N, K, seed=0):
    g = torch.Generator().manual_seed(seed)
    a = torch.randn(M, K, generator=g).to(torch.bfloat16)
    w = (torch.randn(N, K, generator=g) * 0.02).to(torch.bfloat16)
    return a, w


@pytest.mark.parametrize("M,N,K", [(64, 96, 64), (64, 192, 256), (1, 96, 128), (128, 288, 512), (200, 192, 320),
                                   (64, 960, 1024), (64, 2384, 256), (65, 4096, 128), (33, 16, 64), (64, 12288, 128)])
def test_against_oracle(M, N, K):
    a, w = make(M, N, K)
    ref = o.gemm(a.float().numpy(), w.float().numpy().T.copy())
    out = ops.gemm_bf16(a.cuda(), w.cuda())
    assert ops.gemm_bf16_status() == 0
    assert_close(out.cpu().numpy(), ref, 1e-4, f"gemm_bf16 {M}x{N}x{K}")


def test_prefill_config():
    M, N, K = 64, 12288, 4096
    a, w = make(M, N, K, seed=3)
    a, w = a.cuda(), w.cuda()
    out = ops.gemm_bf16(a, w)
    ref = a.double() @ w.double().T
    assert ops.gemm_bf16_status() == 0
    err = ((out.double() - ref).abs().max() / ref.abs().max()).item()
    assert err < 1e-4, err


def test_rejects_unsupported_shapes():
    from vk_compute_b200._lib import VkcError

    a = torch.zeros(4, 100, dtype=torch.bfloat16, device="cuda")
    w = torch.zeros(96, 100, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(VkcError, match="multiple of 64"):
        ops.gemm_bf16(a, w)
    a = torch.zeros(4, 64, dtype=torch.bfloat16, device="cuda")
    w = torch.zeros(100, 64, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(VkcError, match="multiple of 16"):
        ops.gemm_bf16(a, w)
