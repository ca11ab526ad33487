"""The fp32 operators that read plain row-major data, against the oracle:
in-place RMSNorm over rows (shader/RmsNorm.comp) and GEMV over a row-major
K x N matrix (shader/gemv2.comp, gemv3.comp; gemv1.comp is the square case),
through the native API and through the reference ABI by shader name."""
import numpy as np
import pytest
import torch

from conftest import assert_close
from gpu_util import SEED_GAMMA, SEED_W, SEED_X, host_vector
from oracle import pyoracle as o
from vk_compute_b200 import dropin as D
from vk_compute_b200 import ops

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("rows,width", [(1, 256), (16, 256), (300, 256), (5, 100), (3, 4096)])
def test_rmsnorm_rows(rows, width):
    x = o.get_data(SEED_X, rows, width)
    g = host_vector(SEED_GAMMA, width)
    xd = torch.from_numpy(x).cuda()
    ops.rmsnorm_rows(xd, torch.from_numpy(g).cuda(), eps=1e-5)
    assert_close(xd.cpu().numpy(), o.rmsnorm_rows(x, g, 1e-5), 2e-6, f"RmsNorm rows={rows} width={width}")


@pytest.mark.parametrize("K,N", [(4096, 12288), (4096, 4096), (1000, 333), (12, 8), (64, 4096), (8192, 36)])
def test_gemv_rowmajor(K, N):
    w = o.get_data(SEED_W, K, N)
    x = host_vector(SEED_X, K)
    y = ops.gemv_rowmajor(torch.from_numpy(w).cuda(), torch.from_numpy(x).cuda())
    assert_close(y.cpu().numpy(), o.gemv_dense(x, w), 2e-5, f"row-major GEMV K={K} N={N}")


@pytest.fixture(scope="module")
def sess():
    s = D.create_session()
    yield s
    D.destroy_session(s)


def test_rmsnorm_by_shader_name(sess):
    rows = 48
    x = o.get_data(SEED_X, rows, 256)
    g = host_vector(SEED_GAMMA, 256)
    xb, gb = D.create_buffer(sess, x), D.create_buffer(sess, g)
    D.execute(sess, [D.operation("RmsNorm.spv", [xb, gb], [], (rows, 1, 1))])
    assert_close(D.read_buffer(sess, xb).reshape(rows, 256), o.rmsnorm_rows(x, g, 1e-5), 2e-6, "RmsNorm.spv")
    for b in (xb, gb):
        D.destroy_buffer(sess, b)


@pytest.mark.parametrize("name", ["gemv1.spv", "gemv2.spv", "gemv3.spv", "gemv4.spv", "gemv5.spv", "gemv6.spv",
                                  "gemv7.spv"])
def test_gemv_experiments_by_shader_name(sess, name):
    K, N = 1024, 768
    x = host_vector(SEED_X, K)
    if name == "gemv1.spv":  # square row-major K x K, K outputs
        w = o.get_data(SEED_W, K, K)
        wdata, n = w, K
    elif name in ("gemv2.spv", "gemv3.spv"):  # row-major K x N
        w = o.get_data(SEED_W, K, N)
        wdata, n = w, N
    else:  # the 16-byte chunk layout of gemv.comp
        w = o.get_data(SEED_W, K, N)
        wdata, n = o.transpose_block16(w, K, N, 32), N
    xb, wb = D.create_buffer(sess, x), D.create_buffer(sess, wdata)
    yb = D.create_buffer(sess, None, 4 * n)
    D.execute(sess, [D.operation(name, [xb, wb, yb], [1, N, K])])
    assert_close(D.read_buffer(sess, yb)[:n], o.gemv_dense(x, w), 2e-5, name)
    for b in (xb, wb, yb):
        D.destroy_buffer(sess, b)


def test_rowmajor_gemv_then_attention_on_library_workspaces():
    """The row-major GEMV's K-slice partials and the decode attention's split
    partials and merge tickets live in separate library workspaces: a GEMV
    that uses its workspace leaves the attention's tickets at zero."""
    import math

    w = o.get_data(SEED_W, 4096, 12288)
    x = host_vector(SEED_X, 4096)
    y = ops.gemv_rowmajor(torch.from_numpy(w).cuda(), torch.from_numpy(x).cuda())
    n_q, n_kv, hd, ctx = 32, 8, 128, 1000
    gen = torch.Generator().manual_seed(3)
    q = torch.randn(n_q * hd, generator=gen).half()
    k = torch.randn(ctx, n_kv, hd, generator=gen).half()
    v = torch.randn(n_kv, hd // 8, ctx, 8, generator=gen).half()
    att = ops.attention_decode(q.cuda(), k.cuda(), v.cuda(), n_q, n_kv, hd, ctx, 1 / math.sqrt(hd))
    ref = o.attention(q.numpy().view(np.uint16), k.numpy().view(np.uint16), v.numpy().view(np.uint16), n_q, n_kv,
                      hd, ctx, 1 / math.sqrt(hd))
    assert_close(att.cpu().numpy(), ref, 2e-3, "attention after a row-major GEMV")
    assert_close(y.cpu().numpy(), o.gemv_dense(x, w), 2e-5, "row-major GEMV")
