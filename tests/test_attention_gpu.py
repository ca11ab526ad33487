"""Decode attention (Att-full-FP16) against the oracle: GQA groups, head
sizes, ragged and single-token contexts, both score scales, fp16/fp32 q,
caller-owned and library-owned workspaces."""
import math

import numpy as np
import pytest
import torch

from conftest import assert_close
from oracle import pyoracle as o
from vk_compute_b200 import ops

pytestmark = pytest.mark.gpu


def make_cache(n_q, n_kv, hd, ctx, seed=0, scale=1.0):
    g = torch.Generator().manual_seed(seed)
    q = (torch.randn(n_q * hd, generator=g) * scale).half()
    k = torch.randn(ctx, n_kv, hd, generator=g).half()
    v_nat = torch.randn(ctx, n_kv, hd, generator=g).half()
    # V[kv][d/8][t][d%8] (shader/Att-full-FP16.comp:69-73)
    v = v_nat.view(ctx, n_kv, hd // 8, 8).permute(1, 2, 0, 3).contiguous()
    return q, k, v


def run(n_q, n_kv, hd, ctx, scale, q_fp32=False, workspace=True, seed=0):
    q, k, v = make_cache(n_q, n_kv, hd, ctx, seed)
    ref = o.attention(q.numpy().view(np.uint16), k.numpy().view(np.uint16), v.numpy().view(np.uint16),
                      n_q, n_kv, hd, ctx, scale)
    qd = q.float().cuda() if q_fp32 else q.cuda()
    ws = ops.attention_workspace(n_q, n_kv, hd, ctx) if workspace else None
    out = ops.attention_decode(qd, k.cuda(), v.cuda(), n_q, n_kv, hd, ctx, scale, workspace=ws)
    return out.cpu().numpy(), ref


@pytest.mark.parametrize("ctx", [1, 31, 100, 1000, 8192])
def test_config_shape(ctx):
    out, ref = run(32, 8, 128, ctx, 1.0 / math.sqrt(128))
    assert_close(out, ref, 2e-3, f"attention ctx={ctx}")


@pytest.mark.parametrize("n_q,n_kv,hd", [(8, 8, 64), (16, 8, 128), (16, 4, 256), (4, 1, 128), (32, 8, 8)])
def test_shapes(n_q, n_kv, hd):
    out, ref = run(n_q, n_kv, hd, 777, 1.0 / math.sqrt(hd))
    assert_close(out, ref, 2e-3, f"attention {n_q}/{n_kv}/{hd}")


def test_reference_scale_one():
    """The shader's scores are unscaled (shader/Att-full-FP16.comp:66)."""
    out, ref = run(16, 4, 256, 512, 1.0)
    assert_close(out, ref, 2e-3, "attention scale 1")


def test_fp32_query_and_library_workspace():
    out, ref = run(32, 8, 128, 4096, 1.0 / math.sqrt(128), q_fp32=True, workspace=False)
    assert_close(out, ref, 2e-3, "attention fp32 q")


def test_repeated_calls_reuse_workspace():
    n_q, n_kv, hd, ctx = 32, 8, 128, 2048
    ws = ops.attention_workspace(n_q, n_kv, hd, ctx)
    for seed in range(3):
        q, k, v = make_cache(n_q, n_kv, hd, ctx, seed)
        ref = o.attention(q.numpy().view(np.uint16), k.numpy().view(np.uint16), v.numpy().view(np.uint16),
                          n_q, n_kv, hd, ctx, 0.1)
        out = ops.attention_decode(q.cuda(), k.cuda(), v.cuda(), n_q, n_kv, hd, ctx, 0.1, workspace=ws)
        assert_close(out.cpu().numpy(), ref, 2e-3, f"call {seed}")
    # tickets are left at zero for the next call
    assert int(ws[:4 * n_kv].view(torch.int32).abs().sum()) == 0
