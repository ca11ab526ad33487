"""Failure detection without a GPU fault: a fused exchange consumer whose peer
never delivers (its slot words keep an old flag: nothing writes them) gives up
once its wait reaches the bound (one 100 ms deadline per thread, started at
the thread's first wait and shared by all the elements it waits for), records
status flag 0x8 (peer timeout) in the device status word and returns; the
device stays usable and later results are correct."""
import struct

import numpy as np
import pytest
import torch

from conftest import TOL, assert_close
from gpu_util import SEED_GAMMA, SEED_W, SEED_W2, SEED_X, device_vector, device_weight, host_vector, host_weight
from oracle import pyoracle as o
from vk_compute_b200 import ops

pytestmark = pytest.mark.gpu


def test_peer_wait_runs_out_and_reports():
    K, N = 1024, 512
    x, g = device_vector(SEED_X, K), device_vector(SEED_GAMMA, K)
    wg, wu = device_weight(SEED_W, K, N, 8), device_weight(SEED_W2, K, N, 8)
    ops.device_status(clear=True)
    # two ranks' slots for this rank (rank 0 of 2): its own words carry flag 1,
    # the peer's keep flag 0 because no peer exists
    own = struct.unpack("<I", struct.pack("<f", 0.25))[0] | (1 << 32)
    words = np.zeros(2 * K, dtype=np.uint64)
    words[:K] = own
    slots = torch.from_numpy(words.view(np.int64)).cuda()
    save = torch.empty(K, device="cuda")
    peer = ops.PeerInput(slots.data_ptr(), save.data_ptr(), 0, 2)
    ops.rmsnorm_swiglu(wg, wu, x, g, eps=1e-5, rms_dim=4096, peer=peer)
    status = ops.device_status(clear=True)
    assert status & 8, f"status {status:#x}: the wait should have run out"
    # the device still computes correctly
    y = ops.rmsnorm_gemv(wg, x, g, eps=1e-5, rms_dim=4096)
    d, s, z = host_weight(SEED_W, K, N, 8)
    ref = o.qgemv(host_vector(SEED_X, K), host_vector(SEED_GAMMA, K), d, s, z, 8, K, N, 4096, 1e-5)
    assert_close(y.cpu().numpy(), ref, TOL[8], "RmsNorm-GEMV-INT8 after a timed-out wait")
    assert ops.device_status(clear=True) == 0
