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


@pytest.fixture(autouse=True, params=["auto", "clustered", "per-sm", "per-sm-half", "per-sm-x2", "per-sm-wide"])
def attention_plan(request):
    """Every case runs under both splits of the cache for the token-slice
    kernel (head_dim 64/128): clusters of 8 CTAs per KV head, and at most one
    CTA per SM with a deep ring; other head sizes ignore the plan."""
    ops.set_attention_plan(request.param)
    yield request.param
    ops.set_attention_plan("auto")


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


@pytest.mark.parametrize("n_q,n_kv,hd", [(8, 8, 64), (16, 8, 128), (16, 4, 256), (4, 1, 128), (32, 8, 8),
                                         (64, 8, 128), (8, 1, 256), (32, 4, 64), (16, 8, 32), (12, 3, 96)])
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


@pytest.mark.parametrize("n_q,n_kv,hd,ctx", [(32, 8, 128, 3001), (64, 8, 128, 515), (16, 4, 256, 1500),
                                              (8, 2, 64, 4097)])
def test_fp32_query_full_precision(n_q, n_kv, hd, ctx):
    """fp32 q values that fp16 cannot hold (the decode chain's QKV output)."""
    _, k, v = make_cache(n_q, n_kv, hd, ctx, seed=5)
    g = torch.Generator().manual_seed(6)
    q = torch.randn(n_q * hd, generator=g) * 1.7
    ref = o.attention_f32q(q.numpy(), k.numpy().view(np.uint16), v.numpy().view(np.uint16), n_q, n_kv, hd, ctx,
                           1.0 / math.sqrt(hd))
    out = ops.attention_decode(q.cuda(), k.cuda(), v.cuda(), n_q, n_kv, hd, ctx, 1.0 / math.sqrt(hd))
    assert_close(out.cpu().numpy(), ref, 2e-3, f"attention fp32 q {n_q}/{n_kv}/{hd}/{ctx}")


def test_peaked_scores():
    """Large scores (scale 1, |q| ~ 4): the softmax is dominated by a few tokens,
    so the running maximum changes between sub-tiles and splits."""
    n_q, n_kv, hd, ctx = 32, 8, 128, 2500
    _, k, v = make_cache(n_q, n_kv, hd, ctx, seed=7)
    g = torch.Generator().manual_seed(8)
    q = torch.randn(n_q * hd, generator=g) * 4.0
    ref = o.attention_f32q(q.numpy(), k.numpy().view(np.uint16), v.numpy().view(np.uint16), n_q, n_kv, hd, ctx, 0.25)
    out = ops.attention_decode(q.cuda(), k.cuda(), v.cuda(), n_q, n_kv, hd, ctx, 0.25)
    assert_close(out.cpu().numpy(), ref, 2e-3, "attention peaked")


def test_unsupported_group_rejected():
    from vk_compute_b200._lib import VkcError
    q = torch.zeros(16 * 8, dtype=torch.float16, device="cuda")
    k = torch.zeros(4, 1, 8, dtype=torch.float16, device="cuda")
    v = torch.zeros(1, 1, 4, 8, dtype=torch.float16, device="cuda")
    with pytest.raises(VkcError, match="query heads per KV head 16"):
        ops.attention_decode(q, k, v, 16, 1, 8, 4, 1.0)


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


@pytest.mark.parametrize("n_q,n_kv,hd,ctx", [(32, 8, 128, 8192), (4, 1, 128, 777), (8, 2, 64, 300), (16, 4, 128, 65)])
def test_append_variant_matches(n_q, n_kv, hd, ctx):
    """vkc_attention_decode_append (cache rows before the newest token requested
    before the wait on the previous kernel) gives the same bits as the plain
    cache entry, right after the newest token was written by a kernel."""
    cap = ctx + 5
    g = torch.Generator().manual_seed(ctx)
    q = torch.randn(n_q * hd, generator=g).cuda()
    kc = torch.randn(cap, n_kv, hd, generator=g).half().cuda()
    vc = torch.randn(n_kv, hd // 8, cap, 8, generator=g).half().cuda()
    ws = ops.attention_workspace(n_q, n_kv, hd, ctx)
    newest_k = torch.randn(n_kv, hd, generator=g).half().cuda()
    prev = ops.get_pdl()
    ops.set_pdl(True)
    try:
        kc[ctx - 1].copy_(newest_k)  # the newest token, written by a kernel just before
        a = ops.attention_decode(q, kc, vc, n_q, n_kv, hd, ctx, hd ** -0.5, workspace=ws, ctx_cap=cap,
                                 after_append=True).clone()
        b = ops.attention_decode(q, kc, vc, n_q, n_kv, hd, ctx, hd ** -0.5, workspace=ws, ctx_cap=cap)
    finally:
        ops.set_pdl(prev)
    assert torch.equal(a, b)


def test_plan_info_matches_plan(request):
    """The plan query names the split the launch uses; the per-SM shapes keep
    the grid within one wave of the SMs."""
    plan = ops.get_attention_plan()
    info = ops.attention_plan_info(32, 8, 128, 8192)
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    if plan == "clustered":
        assert info["kernel"] == "token-slice clustered" and info["cluster"] == 8
        return
    assert info["kernel"] == "token-slice per-SM"
    assert info["splits"] * info["tokens_per_cta"] >= 8192
    ctas_per_sm = 2 if plan == "per-sm-x2" else 1
    assert info["splits"] * 8 <= ctas_per_sm * sms
    if plan in ("per-sm-wide", "auto"):
        assert info["warp_groups"] == 2
