"""fp32 gemm (shader/gemm.comp) against the oracle, including ragged shapes."""
import numpy as np
import pytest
import torch

from conftest import assert_close
from oracle import pyoracle as o
from vk_compute_b200 import ops

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("M,N,K", [(64, 256, 128), (1, 1, 1), (17, 33, 65), (64, 12288, 512)])
def test_gemm_f32(M, N, K):
    g = torch.Generator().manual_seed(M * 7 + N)
    a = torch.randn(M, K, generator=g)
    b = torch.randn(K, N, generator=g)
    c = ops.gemm_f32(a.cuda(), b.cuda()).cpu().numpy()
    assert_close(c, o.gemm(a.numpy(), b.numpy()), 1e-4, "gemm")
