"""The allocation-free decode attention entry point.

Callers that cannot allocate device memory when attention runs (an engine whose
pool already owns all of HBM, a decode loop that must avoid the synchronisation
cudaMalloc/cudaFree can imply, a plugin whose host forbids allocation) call
vkc_attention_decode_noalloc, which keeps its scratch in a fixed array inside
the library.  Two calls in a row through the C ABI must match the ordinary
entry point (vkc_attention_decode with a caller workspace); the second call
also checks that the merge tickets the first call left behind are clean.

The file name makes pytest collect it last, so that a run stopped at its
first failure has already run every other test if this one fails.  It
depends on no state the other tests leave: it passes alone in a fresh process
and after them, because each call looks up the array in the current context
and leaves the tickets at zero.
"""
import ctypes as C
import math

import numpy as np
import pytest
import torch

from conftest import assert_close
from vk_compute_b200 import ops
from vk_compute_b200._lib import check, lib

pytestmark = pytest.mark.gpu


def _noalloc():
    L = lib()
    fn = L.vkc_attention_decode_noalloc
    fn.restype = C.c_int
    fn.argtypes = [C.c_void_p, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int,
                   C.c_float, C.c_void_p]
    L.vkc_attention_noalloc_max_scratch.restype = C.c_size_t
    return fn, L.vkc_attention_noalloc_max_scratch()


def test_noalloc_matches_workspace_entry_point_twice():
    fn, cap = _noalloc()
    n_q, n_kv, hd, ctx = 32, 8, 128, 8192
    assert lib().vkc_attention_workspace_bytes(n_q, n_kv, hd, ctx) <= cap
    scale = 1.0 / math.sqrt(hd)
    ws = ops.attention_workspace(n_q, n_kv, hd, ctx)
    stream = torch.cuda.current_stream()
    for call in range(2):
        g = torch.Generator().manual_seed(2024 + call)
        q = torch.randn(n_q * hd, generator=g).half().cuda()
        k = torch.randn(ctx, n_kv, hd, generator=g).half().cuda()
        v = torch.randn(n_kv, hd // 8, ctx, 8, generator=g).half().cuda()
        ref = ops.attention_decode(q, k, v, n_q, n_kv, hd, ctx, scale, workspace=ws)
        out = torch.full((n_q * hd,), float("nan"), device="cuda")
        check(fn(C.c_void_p(q.data_ptr()), 16, C.c_void_p(k.data_ptr()), C.c_void_p(v.data_ptr()),
                 C.c_void_p(out.data_ptr()), n_q, n_kv, hd, ctx, scale, C.c_void_p(stream.cuda_stream)))
        torch.cuda.synchronize()
        assert_close(out.cpu().numpy(), ref.cpu().numpy().astype(np.float64), 2e-3, f"no-alloc call {call}")


def test_noalloc_rejects_shapes_beyond_its_scratch():
    fn, cap = _noalloc()
    n_q, n_kv, hd, ctx = 32, 1, 256, 65536  # one KV head: ~300 splits of 32 x 260 floats
    assert lib().vkc_attention_workspace_bytes(n_q, n_kv, hd, ctx) > cap
    rc = fn(None, 16, None, None, None, n_q, n_kv, hd, ctx, 1.0, None)
    assert rc != 0
    assert b"allocation-free" in lib().vkc_last_error()
