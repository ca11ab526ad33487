"""The reference's host ABI end to end: the call sequence of src/compute.c
(createSession, createBuffer, createTransferAndCopy, execute by shader name,
getExecutionTime, readBuffer, destroyBuffer) with host buffers made by the
oracle's restatement of src/data.c, against the oracle's operators with the
shaders' constants (eps 1e-5, RMS divisor 4096)."""
import math
import struct

import numpy as np
import pytest

from conftest import TOL, assert_close
from gpu_util import SEED_GAMMA, SEED_W, SEED_W2, SEED_X, host_vector, host_weight, rope_theta
from oracle import pyoracle as o
from vk_compute_b200 import dropin as D

pytestmark = pytest.mark.gpu

K, N = 1024, 768
NAMES = {32: "", 16: "-FP16", 8: "-INT8", 4: "-INT4"}


@pytest.fixture(scope="module")
def sess():
    s = D.create_session()
    yield s
    D.destroy_session(s)


def packed(seed, bits):
    d, s, z = host_weight(seed, K, N, bits)
    return o.transpose_block16(d, K, N, bits), s, z, (d, s, z)


def bufs(s, *arrays):
    return [D.create_buffer(s, a) for a in arrays]


@pytest.mark.parametrize("bits", [32, 16, 8, 4])
def test_gemv_and_rmsnorm_gemv(sess, bits):
    x, g = host_vector(SEED_X, K), host_vector(SEED_GAMMA, K)
    w, sc, zr, host = packed(SEED_W, bits)
    y = D.create_buffer(sess, None, 4 * N)
    xb, gb, wb = bufs(sess, x, g, w)
    extra = bufs(sess, sc, zr) if bits <= 8 else []
    D.abi().createTransferAndCopy(sess.dev.device, sess.dev.queue, None, 0)
    name = "GEMV" + NAMES[bits] + ".spv" if bits != 32 else "GEMV.spv"
    ms = D.execute(sess, [D.operation(name, [xb, wb, y] + extra, [1, N, K], ((N + 255) // 256, 1, 1))])
    assert ms > 0.0
    ref = o.qgemv(x, None, *host, bits, K, N)
    assert_close(D.read_buffer(sess, y), ref, TOL[bits], name)
    name = "RmsNorm-GEMV" + NAMES[bits] + ".spv"
    D.execute(sess, [D.operation(name, [xb, gb, wb, y] + extra, [1, N, K])])
    ref = o.qgemv(x, g, *host, bits, K, N, 4096, 1e-5)
    assert_close(D.read_buffer(sess, y), ref, TOL[bits], name)
    for b in [xb, gb, wb, y] + extra:
        D.destroy_buffer(sess, b)


@pytest.mark.parametrize("bits", [16, 8, 4])
def test_rope(sess, bits):
    x, g = host_vector(SEED_X, K), host_vector(SEED_GAMMA, K)
    w, sc, zr, host = packed(SEED_W, bits)
    theta = rope_theta(64, 10000.0, 128)
    y = D.create_buffer(sess, None, 4 * N)
    xb, gb, wb, tb = bufs(sess, x, g, w, theta)
    mid = bufs(sess, sc, zr) if bits <= 8 else []
    name = "RmsNorm-GEMV-Rope" + NAMES[bits] + ".spv"
    base = o.qgemv(x, g, *host, bits, K, N, 4096, 1e-5)
    # {M, N, K, tokenIdx}: the shader's epilogue as written
    D.execute(sess, [D.operation(name, [xb, gb, wb, y] + mid + [tb], [1, N, K, 77])])
    assert_close(D.read_buffer(sess, y), o.rope_reference(base, 77, theta), TOL[bits], name)
    # {M, N, K, tokenIdx, head_dim, rotated rows}: rotary pairs per head
    D.execute(sess, [D.operation(name, [xb, gb, wb, y] + mid + [tb], [1, N, K, 77, 128, 640])])
    assert_close(D.read_buffer(sess, y), o.rope_pairs(base, 128, 640, 77, theta), TOL[bits], name)


@pytest.mark.parametrize("bits", [32, 16, 8, 4])
def test_swiglu(sess, bits):
    x, g = host_vector(SEED_X, K), host_vector(SEED_GAMMA, K)
    wg, sg, zg, hg = packed(SEED_W, bits)
    wu, su, zu, hu = packed(SEED_W2, bits)
    y = D.create_buffer(sess, None, 4 * N)
    b = bufs(sess, x, g, wg, wu)
    extra = bufs(sess, sg, zg, su, zu) if bits <= 8 else []
    name = "RmsNorm-swiglu-ffn" + NAMES[bits] + ".spv"
    D.execute(sess, [D.operation(name, b + [y] + extra, [1, N, K])])
    ref = o.qswiglu(x, g, hg, hu, bits, K, N, 4096, 1e-5)
    assert_close(D.read_buffer(sess, y), ref, TOL[bits], name)


def test_attention_and_gemm_by_name(sess):
    import torch
    n_q, n_kv, hd, ctx = 16, 4, 256, 300
    gen = torch.Generator().manual_seed(3)
    q = torch.randn(n_q * hd, generator=gen).half().numpy().view(np.uint16)
    k = torch.randn(ctx, n_kv, hd, generator=gen).half().numpy().view(np.uint16)
    v = torch.randn(n_kv, hd // 8, ctx, 8, generator=gen).half().numpy().view(np.uint16)
    kb, vb, qb = bufs(sess, k, v, q)
    y = D.create_buffer(sess, None, 4 * n_q * hd)
    # defaults: head_dim 256, n_kv = n_q / 4, scale 1 (the shader's)
    D.execute(sess, [D.operation("Att-full-FP16.spv", [kb, vb, qb, y], [1, n_q * hd, 4096, ctx])])
    assert_close(D.read_buffer(sess, y), o.attention(q, k, v, n_q, n_kv, hd, ctx, 1.0), 2e-3, "Att-full")
    sc = struct.unpack("<i", struct.pack("<f", 1 / math.sqrt(hd)))[0]
    D.execute(sess, [D.operation("Att-full-FP16.spv", [kb, vb, qb, y], [1, n_q * hd, 4096, ctx, hd, n_kv, sc])])
    assert_close(D.read_buffer(sess, y), o.attention(q, k, v, n_q, n_kv, hd, ctx, 1 / math.sqrt(hd)), 2e-3,
                 "Att-full scaled")
    a = np.random.default_rng(0).standard_normal((64, 96)).astype(np.float32)
    bm = np.random.default_rng(1).standard_normal((96, 80)).astype(np.float32)
    ab, bb = bufs(sess, a, bm)
    cb = D.create_buffer(sess, None, 4 * 64 * 80)
    D.execute(sess, [D.operation("gemm.spv", [ab, bb, cb], [64, 80, 96])])
    assert_close(D.read_buffer(sess, cb).reshape(64, 80), o.gemm(a, bm), 1e-4, "gemm")


def test_chained_ops_in_one_execute(sess):
    """Ops of one execute() run in order (src/dispatch.c:34-44): GEMV-INT4
    feeding RmsNorm-GEMV-INT8."""
    x = host_vector(SEED_X, K)
    g = host_vector(SEED_GAMMA, K)
    d4, s4, z4 = host_weight(SEED_W, K, K, 4)
    d8, s8, z8 = host_weight(SEED_W2, K, N, 8)
    xb, gb = bufs(sess, x, g)
    w4, s4b, z4b = bufs(sess, o.transpose_block16(d4, K, K, 4), s4, z4)
    w8, s8b, z8b = bufs(sess, o.transpose_block16(d8, K, N, 8), s8, z8)
    mid = D.create_buffer(sess, None, 4 * K)
    y = D.create_buffer(sess, None, 4 * N)
    D.execute(sess, [D.operation("GEMV-INT4.spv", [xb, w4, mid, s4b, z4b], [1, K, K]),
                     D.operation("RmsNorm-GEMV-INT8.spv", [mid, gb, w8, y, s8b, z8b], [1, N, K])])
    h = o.qgemv(x, None, d4, s4, z4, 4, K, K)
    ref = o.qgemv(h, g, d8, s8, z8, 8, K, N, 4096, 1e-5)
    assert_close(D.read_buffer(sess, y), ref, 5e-3, "chain")


def test_timing_switch(sess):
    """With execute() timing off, results are unchanged and getExecutionTime
    returns 0; turned back on, it reports the device time again."""
    x = host_vector(SEED_X, K)
    w, sc, zr, host = packed(SEED_W, 8)
    y = D.create_buffer(sess, None, 4 * N)
    xb, wb, sb, zb = bufs(sess, x, w, sc, zr)
    op = [D.operation("GEMV-INT8.spv", [xb, wb, y, sb, zb], [1, N, K])]
    ref = o.qgemv(x, None, *host, 8, K, N)
    from vk_compute_b200._lib import lib as vlib
    try:
        vlib().vkc_set_timing(0)
        assert vlib().vkc_get_timing() == 0
        assert D.execute(sess, op) == 0.0
        assert_close(D.read_buffer(sess, y), ref, TOL[8], "GEMV-INT8, timing off")
    finally:
        vlib().vkc_set_timing(1)
    assert D.execute(sess, op) > 0.0
    assert_close(D.read_buffer(sess, y), ref, TOL[8], "GEMV-INT8, timing on")
    for b in (xb, wb, sb, zb, y):
        D.destroy_buffer(sess, b)


@pytest.mark.parametrize("nbytes", [4, 17, 16384, 49157, 1 << 20, (1 << 20) + 12])
def test_write_buffer_round_trip(sess, nbytes):
    """writeBuffer (an extension of the ABI) into an existing buffer: staged
    sizes up to 1 MiB, ragged tails and the larger synchronous path."""
    rng = np.random.default_rng(nbytes)
    a = rng.integers(0, 256, nbytes, dtype=np.uint8)
    b = D.create_buffer(sess, None, nbytes)
    D.write_buffer(sess, b, a)
    np.testing.assert_array_equal(D.read_buffer(sess, b, np.uint8), a)
    D.destroy_buffer(sess, b)


def test_write_buffer_sequence_then_operator(sess):
    """Several uploads without a read in between (both staging slots reused,
    the caller's array overwritten at once), then an operator on the last
    value written: the operator sees it, the other buffers keep theirs."""
    x_last = host_vector(SEED_X + 5, K)
    xs = [host_vector(SEED_X + i, K) for i in range(5)] + [x_last]
    xb = D.create_buffer(sess, None, 4 * K)
    side = [D.create_buffer(sess, None, 4 * K) for _ in range(3)]
    scratch = np.empty(K, dtype=np.float32)
    for i, x in enumerate(xs):
        scratch[:] = x
        D.write_buffer(sess, xb, scratch)
        D.write_buffer(sess, side[i % 3], scratch)
        scratch[:] = -1.0  # reused by the caller as soon as the call returns
    w, sc, zr, host = packed(SEED_W, 8)
    y = D.create_buffer(sess, None, 4 * N)
    wb, sb, zb = bufs(sess, w, sc, zr)
    D.execute(sess, [D.operation("GEMV-INT8.spv", [xb, wb, y, sb, zb], [1, N, K])])
    assert_close(D.read_buffer(sess, y), o.qgemv(x_last, None, *host, 8, K, N), TOL[8], "GEMV-INT8 after writes")
    for i in range(3):
        np.testing.assert_array_equal(D.read_buffer(sess, side[i]), xs[3 + i])
    for b in [xb, y, wb, sb, zb] + side:
        D.destroy_buffer(sess, b)


def test_weights_rewritten_between_steps(sess):
    """Weights, scales and x re-uploaded through the staged writeBuffer right
    before each execute(), and a second operator whose gamma is the first
    one's output: an operator that starts before the previous kernel ends
    (programmatic dependent launch) reads weights early, so it may do so only
    when no queued work can still write them.  Each step must see its own
    weights, and the second operator the first one's result."""
    x = host_vector(SEED_X, K)
    wq = D.create_buffer(sess, None, K * K)  # int8 K x K, the first operator
    sq = D.create_buffer(sess, None, 4 * K * (K // 256))
    zq = D.create_buffer(sess, None, 4 * K * (K // 256))
    w8 = D.create_buffer(sess, None, K * N)
    s8 = D.create_buffer(sess, None, 4 * K * (N // 256))
    z8 = D.create_buffer(sess, None, 4 * K * (N // 256))
    xb, mid, y = D.create_buffer(sess, x), D.create_buffer(sess, None, 4 * K), D.create_buffer(sess, None, 4 * N)
    for step in range(4):
        dq, sqh, zqh = host_weight(SEED_W + 10 * step, K, K, 8)
        d8, s8h, z8h = host_weight(SEED_W2 + 10 * step, K, N, 8)
        xs = host_vector(SEED_X + step, K)
        for b, a in ((wq, o.transpose_block16(dq, K, K, 8)), (sq, sqh), (zq, zqh),
                     (w8, o.transpose_block16(d8, K, N, 8)), (s8, s8h), (z8, z8h), (xb, xs)):
            D.write_buffer(sess, b, a)
        D.execute(sess, [D.operation("GEMV-INT8.spv", [xb, wq, mid, sq, zq], [1, K, K]),
                         D.operation("RmsNorm-GEMV-INT8.spv", [xb, mid, w8, y, s8, z8], [1, N, K])])
        h = o.qgemv(xs, None, dq, sqh, zqh, 8, K, K)
        ref = o.qgemv(xs, h, d8, s8h, z8h, 8, K, N, 4096, 1e-5)
        assert_close(D.read_buffer(sess, mid), h, TOL[8], f"GEMV-INT8 step {step}")
        assert_close(D.read_buffer(sess, y), ref, 5e-3, f"RmsNorm-GEMV-INT8 with gamma from the GEMV, step {step}")
    for b in (wq, sq, zq, w8, s8, z8, xb, mid, y):
        D.destroy_buffer(sess, b)
