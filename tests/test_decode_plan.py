"""Host logic of the sharded decoder (no GPU): the shard plan covers every
head and row exactly once, keeps quantised shards on 256-row scale blocks,
and the K-split projections summed over ranks (the all-reduce the decoder
relies on) reproduce the unsharded product (two gloo ranks on CPU)."""
import os

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from vk_compute_b200.decode import DecoderConfig, shard_plan


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_plan_partitions_heads_and_rows(world):
    cfg = DecoderConfig()
    plans = [shard_plan(cfg, r, world) for r in range(world)]
    qkv = sorted(c for p in plans for c in p.qkv_cols)
    assert qkv == list(range(cfg.qkv_rows))
    assert [p.q_heads for p in plans] == [(r * 32 // world, (r + 1) * 32 // world) for r in range(world)]
    assert [p.o_k for p in plans] == [(r * cfg.n_q * cfg.head_dim // world, (r + 1) * cfg.n_q * cfg.head_dim // world)
                                      for r in range(world)]
    assert sum(p.ffn_rows[1] - p.ffn_rows[0] for p in plans) == cfg.inter
    for p in plans:
        hd = cfg.head_dim
        # shard order is [Q | K0 V0 | K1 V1 ...] of the rank's own heads: two
        # contiguous ranges of the full matrix, each whole 256-row blocks
        q = p.qkv_cols[:p.n_q * hd]
        kv = p.qkv_cols[p.n_q * hd:]
        assert q == tuple(range(p.q_heads[0] * hd, p.q_heads[1] * hd))
        assert kv == tuple(range(cfg.n_q * hd + 2 * p.kv_heads[0] * hd, cfg.n_q * hd + 2 * p.kv_heads[1] * hd))
        assert q[0] % 256 == 0 and len(q) % 256 == 0 and kv[0] % 256 == 0 and len(kv) % 256 == 0
        # GQA: the rank's query heads read only its own KV heads
        group = cfg.n_q // cfg.n_kv
        assert p.q_heads[0] // group == p.kv_heads[0] and (p.q_heads[1] - 1) // group == p.kv_heads[1] - 1


def test_plan_rejects_uneven_splits():
    with pytest.raises(ValueError):
        shard_plan(DecoderConfig(n_kv=8), 0, 16)
    with pytest.raises(ValueError):
        shard_plan(DecoderConfig(hidden=1024, inter=1536, n_q=8, n_kv=8), 0, 8)  # 128-row int4 shards


def _ksplit_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cfg = DecoderConfig(hidden=512, inter=1024, n_q=8, n_kv=2, head_dim=64, bits=16)
        p = shard_plan(cfg, rank, world)
        g = torch.Generator().manual_seed(3)
        w_o = torch.randn(cfg.n_q * cfg.head_dim, cfg.hidden, generator=g, dtype=torch.float64)
        w_d = torch.randn(cfg.inter, cfg.hidden, generator=g, dtype=torch.float64)
        a = torch.randn(cfg.n_q * cfg.head_dim, generator=g, dtype=torch.float64)
        h = torch.randn(cfg.inter, generator=g, dtype=torch.float64)
        res = torch.randn(cfg.hidden, generator=g, dtype=torch.float64)
        (o0, o1), (f0, f1) = p.o_k, p.ffn_rows
        o = w_o[o0:o1].T @ a[o0:o1]
        d = w_d[f0:f1].T @ h[f0:f1]
        dist.all_reduce(o)
        dist.all_reduce(d)
        ok = bool(torch.allclose(res + o, res + w_o.T @ a, atol=1e-9)) and bool(torch.allclose(d, w_d.T @ h, atol=1e-9))
        q.put((rank, ok))
    finally:
        dist.destroy_process_group()


def test_ksplit_allreduce_two_gloo_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29600 + os.getpid() % 1000
    procs = [ctx.Process(target=_ksplit_worker, args=(r, 2, port, q)) for r in range(2)]
    for pr in procs:
        pr.start()
    for pr in procs:
        pr.join(120)
        assert pr.exitcode == 0
    res = dict(q.get(timeout=10) for _ in range(2))
    assert res == {0: True, 1: True}


def _qkv_shard_dequant(cfg, w, plan):
    """The rank's QKV shard quantised on its own (symmetric, fp16-valued
    scales, as build_layer does) and dequantised, in shard column order."""
    import numpy as np

    from oracle import pyoracle as o

    cols = np.asarray(plan.qkv_cols)
    sub = np.ascontiguousarray(w[:, cols])
    d, s, z = o.quantize(sub, cfg.bits, True, True)
    return o.dequant(d, s, z, sub.shape[0], sub.shape[1], cfg.bits)


def _full_qkv(cfg):
    import numpy as np

    g = torch.Generator().manual_seed(11)
    return (torch.randn(cfg.hidden, cfg.qkv_rows, generator=g) * 0.02).numpy().astype(np.float32)


SHARD_CFG = DecoderConfig(hidden=512, inter=1024, n_q=8, n_kv=2, head_dim=128, bits=4)


def _quant_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import numpy as np

        from oracle import pyoracle as o

        cfg = SHARD_CFG
        w = _full_qkv(cfg)
        plan = shard_plan(cfg, rank, world)
        mine = torch.from_numpy(_qkv_shard_dequant(cfg, w, plan))
        parts = [torch.empty_like(mine) for _ in range(world)]
        dist.all_gather(parts, mine)
        ok = True
        if rank == 0:
            d, s, z = o.quantize(w, cfg.bits, True, True)
            full = o.dequant(d, s, z, cfg.hidden, cfg.qkv_rows, cfg.bits)
            for r in range(world):
                cols = np.asarray(shard_plan(cfg, r, world).qkv_cols)
                ok = ok and np.array_equal(parts[r].numpy(), full[:, cols])
        q.put((rank, ok))
    finally:
        dist.destroy_process_group()


def test_qkv_shards_quantise_as_the_full_matrix_two_gloo_ranks():
    """Each rank quantises its own QKV shard ([Q | K/V pairs] of its heads);
    gathered, the shards equal the unsharded matrix's quantisation bit for
    bit, so the sharded int4 model is the one-GPU model."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29700 + os.getpid() % 1000
    procs = [ctx.Process(target=_quant_worker, args=(r, 2, port, q)) for r in range(2)]
    for pr in procs:
        pr.start()
    for pr in procs:
        pr.join(120)
        assert pr.exitcode == 0
    res = dict(q.get(timeout=10) for _ in range(2))
    assert res == {0: True, 1: True}


@pytest.mark.parametrize("world", [4, 8])
def test_qkv_shards_quantise_as_the_full_matrix(world):
    import numpy as np

    from oracle import pyoracle as o

    cfg = DecoderConfig(hidden=512, inter=2048, n_q=16, n_kv=8, head_dim=128, bits=4)
    w = _full_qkv(cfg)
    d, s, z = o.quantize(w, cfg.bits, True, True)
    full = o.dequant(d, s, z, cfg.hidden, cfg.qkv_rows, cfg.bits)
    for r in range(world):
        plan = shard_plan(cfg, r, world)
        assert np.array_equal(_qkv_shard_dequant(cfg, w, plan), full[:, np.asarray(plan.qkv_cols)])
