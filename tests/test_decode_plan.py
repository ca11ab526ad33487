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
        # shard order is [Q | K | V] of the rank's own heads
        q = p.qkv_cols[:p.n_q * hd]
        k = p.qkv_cols[p.n_q * hd:(p.n_q + p.n_kv) * hd]
        v = p.qkv_cols[(p.n_q + p.n_kv) * hd:]
        assert q[0] == p.q_heads[0] * hd and len(v) == len(k) == p.n_kv * hd
        assert k[0] == cfg.n_q * hd + p.kv_heads[0] * hd
        assert v[0] == (cfg.n_q + cfg.n_kv) * hd + p.kv_heads[0] * hd
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
