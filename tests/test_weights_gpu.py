"""Weights on disk through the device: matrices written by ops.save_weights
and read back straight into HBM are the same bytes and give the same GEMV;
a small decoder saved with decode.save_model and rebuilt from the file
(load_layer, which cuts the shards of a rank out of the full matrices) steps
to the bit-identical output."""
import numpy as np
import pytest
import torch

from conftest import TOL, assert_close
from gpu_util import SEED_X, SEED_W, device_vector, device_weight, host_vector, host_weight
from oracle import pyoracle as o
from vk_compute_b200 import ops
from vk_compute_b200.decode import DecoderConfig, ShardedDecoder, load_layer, save_model, shard_plan

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("bits,K,N", [(4, 4096, 6144), (8, 1024, 512), (16, 512, 256), (32, 64, 96)])
def test_save_load_gemv(tmp_path, bits, K, N):
    w = device_weight(SEED_W, K, N, bits)
    path = tmp_path / "m.vkcw"
    ops.save_weights(str(path), {"m": w})
    got = ops.load_weights(str(path))["m"]
    assert (got.bits, got.K, got.N) == (bits, K, N)
    assert torch.equal(got.packed, w.packed)
    if bits <= 8:
        assert torch.equal(got.scale, w.scale) and torch.equal(got.zero, w.zero)
    x = device_vector(SEED_X, K)
    y = ops.gemv(got, x).cpu().numpy()
    d, s, z = host_weight(SEED_W, K, N, bits)
    assert_close(y, o.qgemv(host_vector(SEED_X, K), None, d, s, z, bits, K, N), TOL[bits], "GEMV of loaded weights")


def test_decoder_from_file_matches(tmp_path):
    cfg = DecoderConfig(hidden=1024, inter=2048, n_q=8, n_kv=2, head_dim=128, layers=2, ctx=64, bits=4)
    dec = ShardedDecoder(cfg, seed=5)
    path = tmp_path / "model.vkcw"
    save_model(dec.layers, str(path))
    full = ops.load_weights(str(path))
    plan = shard_plan(cfg, 0, 1)
    layers = [load_layer(cfg, plan, i, torch.device("cuda"), full, seed=5) for i in range(cfg.layers)]
    dec2 = ShardedDecoder(cfg, seed=5, layers=layers)
    x0 = torch.randn(cfg.hidden, generator=torch.Generator().manual_seed(1)).cuda()
    for pos in (3, 4):
        dec.buf.x.copy_(x0)
        dec2.buf.x.copy_(x0)
        a, b = dec.step(pos).clone(), dec2.step(pos).clone()
        assert torch.equal(a, b), f"decoder from file differs at pos {pos}"


@pytest.mark.parametrize("world", [2, 4])
def test_file_shards_match_drawn_shards(tmp_path, world):
    """The shards load_layer cuts from the full matrices equal the shards
    build_layer draws for each rank (the sharded model read from one file)."""
    from vk_compute_b200.decode import build_layer

    cfg = DecoderConfig(hidden=1024, inter=2048, n_q=8, n_kv=4, head_dim=128, layers=1, ctx=16, bits=4)
    full_layers = [build_layer(cfg, shard_plan(cfg, 0, 1), 0, torch.device("cuda"), seed=2)]
    path = tmp_path / "m.vkcw"
    save_model(full_layers, str(path))
    full = ops.load_weights(str(path))
    for r in range(world):
        plan = shard_plan(cfg, r, world)
        a = load_layer(cfg, plan, 0, torch.device("cuda"), full, seed=2)
        b = build_layer(cfg, plan, 0, torch.device("cuda"), seed=2)
        for m in ("qkv", "o", "gate", "up", "down"):
            wa, wb = getattr(a, m), getattr(b, m)
            assert (wa.K, wa.N) == (wb.K, wb.N), m
            assert torch.equal(wa.packed, wb.packed) and torch.equal(wa.scale, wb.scale), f"{m} rank {r}"
        assert torch.equal(a.kcache, b.kcache) and torch.equal(a.vcache, b.vcache)
