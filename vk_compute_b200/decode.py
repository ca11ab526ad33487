"""Row-sharded decoder chain built from the decode-path operators.

One decode step of a stack of transformer layers, each

    qkv  = RmsNorm-GEMV-Rope(W_qkv, x, gamma_attn)   Q,K rotated; K,V appended
                                                     to the fp16 caches at `pos`
    a    = Att-full(q, K cache, V cache)             (GQA, split-KV)
    x'   = x + W_o a
    h    = RmsNorm-SwiGLU(W_gate, W_up, x', gamma_ffn)
    x''  = x' + W_down h

with int4 (or int8 / fp16) weights in vk-compute's storage.  The reference
ships these operators as separate shaders and no driver chains them
(shader/RmsNorm-GEMV-Rope-*.comp, Att-full-FP16.comp, GEMV-*.comp,
RmsNorm-swiglu-ffn-*.comp); the chain, the KV append and the residual adds are
this library's.

The model's fused QKV matrix has its output rows in the order
[Q heads | K0 V0 | K1 V1 | ...]: each KV head's K rows followed by its V rows.
With head_dim 128 a K/V pair is exactly one 256-row scale block, so every
shard below is made of whole scale blocks of the unsharded matrix and the
quantised model is the same at 1, 2, 4 and 8 GPUs.

Sharding over `world` GPUs of one node (one process each), two exchanges per
layer: rank r owns query heads [r*nq/world, (r+1)*nq/world) and the matching
KV heads, so QKV (split by output rows, head-aligned), RoPE, the cache and
attention are local; the O projection is split along its input (the rank's
heads), so each rank produces a partial x' increment; gate/up are split by
output rows (the rank's slice of h) and down along its input (that slice).
The two partial vectors per layer are summed across ranks together with the
residual, leaving x' and x'' replicated on every rank.  By default the sum is
fused into the operators: the O and down projections store their partials
straight into every rank's slot buffer over NVLink (vkc_gemv_peer), and the
next operator (SwiGLU, or the next layer's QKV) adds the slots to the
residual while loading its input and stores the result (exchange="p2p"; the
last layer of a step ends with a standalone peer all-reduce so that x is
materialised).  exchange="p2p-kernel" runs the peer all-reduce as its own
kernel after each projection, exchange="nccl" uses torch.distributed.  Splitting O
and down along K keeps their quantisation identical to the unsharded matrices
(scales are per input row and 256-output block).
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch

from . import ops


@dataclass(frozen=True)
class DecoderConfig:
    hidden: int = 4096
    inter: int = 12288
    n_q: int = 32
    n_kv: int = 8
    head_dim: int = 128
    layers: int = 36
    ctx: int = 8192          # KV-cache capacity (tokens)
    bits: int = 4
    eps: float = 1e-6
    theta_base: float = 1e6
    w_std: float = 0.02

    @property
    def qkv_rows(self) -> int:
        return (self.n_q + 2 * self.n_kv) * self.head_dim


@dataclass(frozen=True)
class ShardPlan:
    """Which rows of each weight a rank owns."""

    rank: int
    world: int
    q_heads: tuple[int, int]     # [lo, hi) query heads
    kv_heads: tuple[int, int]    # [lo, hi) KV heads
    qkv_cols: tuple[int, ...]    # output rows of the full QKV matrix, shard order [Q | K0 V0 | ...]
    o_k: tuple[int, int]         # [lo, hi) of the O projection's input (the rank's heads x head_dim)
    ffn_rows: tuple[int, int]    # [lo, hi) of inter: gate/up outputs, down inputs

    @property
    def n_q(self) -> int:
        return self.q_heads[1] - self.q_heads[0]

    @property
    def n_kv(self) -> int:
        return self.kv_heads[1] - self.kv_heads[0]


def shard_plan(cfg: DecoderConfig, rank: int, world: int) -> ShardPlan:
    """Head-aligned shard of rank `rank` out of `world`; raises ValueError when
    the model does not split evenly into whole heads and 256-row scale blocks."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} of world {world}")
    if cfg.n_q % world or cfg.n_kv % world:
        raise ValueError(f"{cfg.n_q} query / {cfg.n_kv} KV heads do not split over {world} ranks")
    if cfg.hidden % world or cfg.inter % world:
        raise ValueError(f"hidden {cfg.hidden} / inter {cfg.inter} do not split over {world} ranks")
    hd = cfg.head_dim
    nq, nkv = cfg.n_q // world, cfg.n_kv // world
    q0, k0 = rank * nq, rank * nkv
    q_cols = range(q0 * hd, (q0 + nq) * hd)
    kv_cols = range(cfg.n_q * hd + 2 * k0 * hd, cfg.n_q * hd + 2 * (k0 + nkv) * hd)  # K/V pairs of its heads
    f = cfg.inter // world
    plan = ShardPlan(rank, world, (q0, q0 + nq), (k0, k0 + nkv), tuple(q_cols) + tuple(kv_cols),
                     (q0 * hd, (q0 + nq) * hd), (rank * f, (rank + 1) * f))
    if cfg.bits <= 8:
        # both row ranges of the QKV shard, and the gate/up shard, start and
        # end on 256-row scale blocks of the unsharded matrices
        for n in (cfg.n_q * hd, nq * hd, 2 * nkv * hd, f):
            if n % 256:
                raise ValueError(f"a {cfg.bits}-bit shard of {n} rows is not a whole number of 256-row scale blocks")
    kpc = 128 // cfg.bits
    for k in (nq * hd, f):
        if k % kpc:
            raise ValueError(f"an input slice of {k} is not a whole number of {kpc}-row chunks")
    return plan


def rope_theta(cfg: DecoderConfig, device) -> torch.Tensor:
    p = torch.arange(cfg.head_dim // 2, dtype=torch.float64)
    return (cfg.theta_base ** (-2.0 * p / cfg.head_dim)).to(torch.float32).to(device)


def dense_weight(seed: int, K: int, N: int, std: float, device) -> torch.Tensor:
    """Seeded N(0, std) K x N matrix (y = W^T x), generated on the device."""
    g = torch.Generator(device=device).manual_seed(seed)
    return torch.randn(K, N, generator=g, device=device) * std


@dataclass
class LayerShard:
    qkv: ops.PackedWeight
    o: ops.PackedWeight
    gate: ops.PackedWeight
    up: ops.PackedWeight
    down: ops.PackedWeight
    g_attn: torch.Tensor
    g_ffn: torch.Tensor
    kcache: torch.Tensor      # fp16 bits [ctx][n_kv][hd]
    vcache: torch.Tensor      # fp16 bits [n_kv][hd/8][ctx][8]


def _pack(w: torch.Tensor, bits: int) -> ops.PackedWeight:
    return ops.pack_dense(w, bits, symmetric=True, fp16_scale=True)


def build_layer(cfg: DecoderConfig, plan: ShardPlan, layer: int, device, seed: int = 0) -> LayerShard:
    """Random-init weights of one layer, this rank's shard.  Every rank draws
    the same full matrices from the same seeds and keeps its own part (QKV
    and gate/up: output rows; O and down: input rows).  Every part is made of
    whole 256-row scale blocks of the full matrix (shard_plan checks it), so
    the sharded model equals the unsharded one, quantisation included."""
    base = seed * 1000 + layer * 10
    H, I = cfg.hidden, cfg.inter
    cols = torch.tensor(plan.qkv_cols, device=device)
    qkv = _pack(dense_weight(base + 1, H, cfg.qkv_rows, cfg.w_std, device)[:, cols].contiguous(), cfg.bits)
    ok_lo, ok_hi = plan.o_k
    f_lo, f_hi = plan.ffn_rows
    o = _pack(dense_weight(base + 2, cfg.n_q * cfg.head_dim, H, cfg.w_std, device)[ok_lo:ok_hi].contiguous(),
              cfg.bits)
    gate = _pack(dense_weight(base + 3, H, I, cfg.w_std, device)[:, f_lo:f_hi].contiguous(), cfg.bits)
    up = _pack(dense_weight(base + 4, H, I, cfg.w_std, device)[:, f_lo:f_hi].contiguous(), cfg.bits)
    down = _pack(dense_weight(base + 5, I, H, cfg.w_std, device)[f_lo:f_hi].contiguous(), cfg.bits)
    g = torch.Generator(device=device).manual_seed(base + 6)
    g_attn = 1 + 0.1 * torch.randn(H, generator=g, device=device)
    g_ffn = 1 + 0.1 * torch.randn(H, generator=g, device=device)
    kcache, vcache = _cache_shard(cfg, plan, layer, device, seed, g)
    return LayerShard(qkv, o, gate, up, down, g_attn, g_ffn, kcache, vcache)


def _cache_shard(cfg: DecoderConfig, plan: ShardPlan, layer: int, device, seed: int, g=None):
    """The KV-cache contents of earlier tokens, N(0, 1), this rank's heads
    (drawn after the two norm vectors of build_layer's generator)."""
    H = cfg.hidden
    if g is None:
        g = torch.Generator(device=device).manual_seed(seed * 1000 + layer * 10 + 6)
        torch.randn(H, generator=g, device=device)
        torch.randn(H, generator=g, device=device)
    # Cache contents of earlier tokens: N(0, 1), the rank's KV heads.
    kfull = torch.randn(cfg.ctx, cfg.n_kv, cfg.head_dim, generator=g, device=device).half()
    vfull = torch.randn(cfg.n_kv, cfg.head_dim // 8, cfg.ctx, 8, generator=g, device=device).half()
    k0, k1 = plan.kv_heads
    kcache = kfull[:, k0:k1].contiguous()
    vcache = vfull[k0:k1].contiguous()
    return kcache, vcache


LAYER_MATRICES = ("qkv", "o", "gate", "up", "down")


def save_model(layers: list[LayerShard], path: str) -> None:
    """Writes the layers of an unsharded (one-GPU) model to a weights file
    (ops.save_weights): per layer the five packed matrices and the two norm
    vectors, a vector of K values being a K x 1 fp32 matrix, whose chunk
    layout is the plain vector."""
    weights = {}
    for i, L in enumerate(layers):
        for m in LAYER_MATRICES:
            weights[f"layers.{i}.{m}"] = getattr(L, m)
        for g in ("g_attn", "g_ffn"):
            v = getattr(L, g)
            weights[f"layers.{i}.{g}"] = ops.PackedWeight(32, v.numel(), 1, v.view(torch.uint8), None, None)
    ops.save_weights(path, weights)


def load_layer(cfg: DecoderConfig, plan: ShardPlan, layer: int, device, full: dict, seed: int = 0) -> LayerShard:
    """This rank's shard of layer `layer` cut from the unsharded matrices in
    `full` (ops.load_weights of a save_model file): QKV by its two output
    ranges, gate/up by output rows, O and down by input rows -- the same
    shards build_layer draws.  The KV caches of earlier tokens are drawn as
    build_layer draws them."""
    pre = f"layers.{layer}."
    hd = cfg.head_dim
    q_lo, q_hi = plan.q_heads[0] * hd, plan.q_heads[1] * hd
    kv_lo = cfg.n_q * hd + 2 * plan.kv_heads[0] * hd
    kv_hi = cfg.n_q * hd + 2 * plan.kv_heads[1] * hd
    f_lo, f_hi = plan.ffn_rows
    qkv = full[pre + "qkv"].columns([(q_lo, q_hi), (kv_lo, kv_hi)])
    o = full[pre + "o"].rows(*plan.o_k)
    gate = full[pre + "gate"].shard(f_lo, f_hi)
    up = full[pre + "up"].shard(f_lo, f_hi)
    down = full[pre + "down"].rows(f_lo, f_hi)
    g_attn = full[pre + "g_attn"].packed.view(torch.float32).clone()
    g_ffn = full[pre + "g_ffn"].packed.view(torch.float32).clone()
    kcache, vcache = _cache_shard(cfg, plan, layer, device, seed)
    return LayerShard(qkv, o, gate, up, down, g_attn, g_ffn, kcache, vcache)


@dataclass
class Buffers:
    x: torch.Tensor           # hidden state (replicated on every rank)
    x_mid: torch.Tensor       # x' after the attention block (replicated)
    qkv: torch.Tensor         # this rank's QKV rows
    attn: torch.Tensor        # this rank's attention output (its heads)
    h: torch.Tensor           # this rank's slice of the SwiGLU output
    o_part: torch.Tensor      # this rank's partial O output (world > 1)
    d_part: torch.Tensor      # this rank's partial down output (world > 1)
    ws: torch.Tensor          # attention workspace


class ShardedDecoder:
    """This rank's part of a `cfg.layers`-layer decoder.

    `step(pos)` advances the hidden state `buf.x` by one token at position
    `pos` (attending to tokens [0, pos]) and returns it.  With world > 1 the
    two all-reduces per layer run on the current stream: fused into the
    projections and their consumers (exchange="p2p", the default), as the
    library's peer all-reduce kernel (exchange="p2p-kernel"; both keep the
    partial slots in peer-mapped memory, see p2p.PeerGather) or through
    torch.distributed (exchange="nccl"); either way a step can be captured in
    a CUDA graph.  exchange="none" runs only this rank's own kernels, with no
    exchange (the shard's partial sums stay local): a one-GPU stand-in for
    timing one rank's share of a sharded step.  Call close() before the
    process group is destroyed.

    `shape` sets the CTA shapes of the step's kernels: "full" runs the GEMVs
    as one 1024-thread CTA per SM and attention through a 6-stage ring (each
    kernel owns the SMs); "half" keeps every kernel within half an SM (the
    512-thread GEMV CTA, the 3-stage attention ring), so under programmatic
    dependent launch each kernel becomes resident beside its predecessor and
    streams its first weights or cache tiles while that one finishes; "mixed"
    runs the GEMVs in half an SM (four consecutive GEMVs per layer overlap
    pairwise) and attention through the 6-stage ring; "persistent" runs the
    whole step as one cooperative kernel (one GPU, 4-bit weights), its phases
    separated by grid barriers (vkc_decode_program_run).
    """

    EXCHANGES = ("p2p", "p2p-kernel", "nccl", "none")
    # (GEMV plan, attention plan) per shape.  With "full", a 512-thread GEMV
    # CTA resident beside a clustered attention kernel would leave room for
    # only one of its two CTAs per SM and split its grid into two waves.
    SHAPES = {"full": ("auto-full", None), "half": ("per-sm-half", "per-sm-half"),
              "mixed": ("per-sm-half", "per-sm"), "persistent": ("auto-full", None)}

    def __init__(self, cfg: DecoderConfig, rank: int = 0, world: int = 1, device=None, seed: int = 0,
                 group=None, layers: list[LayerShard] | None = None, exchange: str = "p2p", shape: str = "full"):
        if shape not in self.SHAPES:
            raise ValueError(f"shape {shape!r} (expected one of {tuple(self.SHAPES)})")
        self.gemv_plan, self.attention_plan = self.SHAPES[shape]
        self.shape = shape
        self.cfg = cfg
        self.plan = shard_plan(cfg, rank, world)
        self.device = torch.device(device or "cuda")
        self.group = group
        if exchange not in self.EXCHANGES:
            raise ValueError(f"exchange {exchange!r} (expected one of {self.EXCHANGES})")
        self.exchange = exchange if world > 1 else "none"
        self.layers = layers if layers is not None else [
            build_layer(cfg, self.plan, i, self.device, seed) for i in range(cfg.layers)]
        self.theta = rope_theta(cfg, self.device)
        H, hd = cfg.hidden, cfg.head_dim
        p = self.plan
        z = lambda n: torch.zeros(n, dtype=torch.float32, device=self.device)
        self.peer = None
        self.buf = Buffers(
            x=z(H), x_mid=z(H), qkv=z(len(p.qkv_cols)), attn=z(p.n_q * hd),
            h=z(p.ffn_rows[1] - p.ffn_rows[0]), o_part=z(H), d_part=z(H),
            ws=self._with_plans(lambda: ops.attention_workspace(p.n_q, p.n_kv, hd, cfg.ctx, device=self.device)))
        self.program = None
        if shape == "persistent":
            if p.world != 1 and self.exchange != "none":
                raise ValueError("the persistent decoder step runs on one GPU")
            self._build_program()
        if self.exchange in ("p2p", "p2p-kernel"):
            from .p2p import PeerGather

            # float slots for the all-reduce kernel; flagged 8-byte words for
            # the fused exchange (x' = x + o words, saved to x_mid; x = x' + d)
            sizes = {"o": world * H, "d": world * H}
            if self.exchange == "p2p":
                sizes.update(o_ll=2 * world * H, d_ll=2 * world * H)
            self.peer = PeerGather(sizes, self.device, group)
            if self.exchange == "p2p":
                self._in_o = self.peer.peer_input("o_ll", save=self.buf.x_mid)
                self._in_d = self.peer.peer_input("d_ll", save=self.buf.x)

    # -- bytes one step streams on this rank (weights, scales, KV cache, at ctx)
    def step_bytes(self, pos: int) -> int:
        cfg, p = self.cfg, self.plan
        n = 0
        for L in self.layers:
            n += sum(w.nbytes for w in (L.qkv, L.o, L.gate, L.up, L.down))
        kv = 2 * (pos + 1) * p.n_kv * cfg.head_dim * 2
        return n + cfg.layers * kv

    def _reduce(self, slots: str, part: torch.Tensor, residual: torch.Tensor, out: torch.Tensor) -> None:
        """out = residual + the sum over ranks of `part`."""
        if self.exchange in ("p2p", "p2p-kernel"):
            self.peer.allreduce(slots, part, residual, out)
        else:
            import torch.distributed as dist

            dist.all_reduce(part, group=self.group)
            torch.add(residual, part, out=out)

    def close(self) -> None:
        """Releases the peer-mapped buffers (collective over the group)."""
        if self.peer is not None:
            self.peer.close()
            self.peer = None

    def _build_program(self) -> None:
        """The step as one persistent kernel (vkc_decode_program_build)."""
        import ctypes as C

        from ._lib import DecodeBuffers, DecodeDims, DecodeLayer, check, lib

        cfg, p, b = self.cfg, self.plan, self.buf
        self._dims = DecodeDims(layers=len(self.layers), hidden=cfg.hidden, inter=p.ffn_rows[1] - p.ffn_rows[0],
                                n_q=p.n_q, n_kv=p.n_kv, head_dim=cfg.head_dim, ctx_cap=cfg.ctx, bits=cfg.bits,
                                eps=cfg.eps)
        if self.layers[0].o.K != p.n_q * cfg.head_dim:
            raise ValueError("the O projection's input is not this rank's heads")
        arr = (DecodeLayer * len(self.layers))()
        ptr = lambda t: t.data_ptr() if t is not None else None
        for i, L in enumerate(self.layers):
            e = arr[i]
            for name, w in (("qkv", L.qkv), ("o", L.o), ("gate", L.gate), ("up", L.up), ("down", L.down)):
                setattr(e, name, ptr(w.packed))
                setattr(e, name + "_scale", ptr(w.scale))
                setattr(e, name + "_zero", ptr(w.zero))
            e.gamma_attn, e.gamma_ffn = L.g_attn.data_ptr(), L.g_ffn.data_ptr()
            e.kcache, e.vcache = L.kcache.data_ptr(), L.vcache.data_ptr()
        bufs = DecodeBuffers(x=b.x.data_ptr(), x_mid=b.x_mid.data_ptr(), qkv=b.qkv.data_ptr(), attn=b.attn.data_ptr(),
                             h=b.h.data_ptr())
        nbytes = lib().vkc_decode_program_bytes(C.byref(self._dims))
        if nbytes == 0:
            raise RuntimeError("vkc_decode_program_bytes failed")
        self.program = torch.zeros(nbytes, dtype=torch.uint8, device=self.device)
        st = torch.cuda.current_stream(self.device).cuda_stream
        check(lib().vkc_decode_program_build(C.byref(self._dims), arr, C.byref(bufs), self.theta.data_ptr(),
                                             self.program.data_ptr(), nbytes, st))

    def _run_program(self, pos: int) -> torch.Tensor:
        import ctypes as C

        from ._lib import check, lib

        if not 0 <= pos < self.cfg.ctx:
            raise ValueError(f"position {pos} outside the cache of {self.cfg.ctx} tokens")
        st = torch.cuda.current_stream(self.device).cuda_stream
        check(lib().vkc_decode_program_run(C.byref(self._dims), self.program.data_ptr(), pos, st))
        return self.buf.x

    def _with_plans(self, fn):
        """fn() under this decoder's GEMV and attention plans (per host
        thread), restoring the caller's afterwards."""
        prev_g, prev_a = ops.get_gemv_plan(), ops.get_attention_plan()
        ops.set_gemv_plan(self.gemv_plan)
        if self.attention_plan is not None:
            ops.set_attention_plan(self.attention_plan)
        try:
            return fn()
        finally:
            ops.set_gemv_plan(prev_g)
            ops.set_attention_plan(prev_a)

    def step(self, pos: int) -> torch.Tensor:
        if self.program is not None:
            return self._run_program(pos)
        return self._with_plans(lambda: self._step(pos))

    def _step(self, pos: int) -> torch.Tensor:
        cfg, p, b = self.cfg, self.plan, self.buf
        if not 0 <= pos < cfg.ctx:
            raise ValueError(f"position {pos} outside the cache of {cfg.ctx} tokens")
        hd = cfg.head_dim
        q_rows, kv_rows = p.n_q * hd, p.n_kv * hd
        scale = 1.0 / math.sqrt(hd)
        single = p.world == 1 or self.exchange == "none"
        fused = self.exchange == "p2p"
        last = len(self.layers) - 1
        for li, L in enumerate(self.layers):
            # x: the step's input, or x' + the previous layer's down slots
            base, peer_in = (b.x_mid, self._in_d) if fused and li > 0 else (b.x, None)
            ops.qkv_rope_append(L.qkv, base, L.g_attn, self.theta, pos, head_dim=hd, q_rows=q_rows, kv_rows=kv_rows,
                                kcache=L.kcache, vcache=L.vcache, ctx_cap=cfg.ctx, eps=cfg.eps, out=b.qkv,
                                peer=peer_in, kv_layout="interleaved")
            ops.attention_decode(b.qkv[:q_rows], L.kcache, L.vcache, p.n_q, p.n_kv, hd, pos + 1, scale,
                                 workspace=b.ws, out=b.attn, ctx_cap=cfg.ctx, after_append=True)
            if single:
                ops.gemv_residual(L.o, b.attn, b.x, out=b.x_mid)
                ops.rmsnorm_swiglu(L.gate, L.up, b.x_mid, L.g_ffn, eps=cfg.eps, out=b.h)
            elif fused:
                ops.gemv_peer(L.o, b.attn, self.peer.dsts["o_ll"], p.rank, p.world)
                ops.rmsnorm_swiglu(L.gate, L.up, b.x, L.g_ffn, eps=cfg.eps, out=b.h, peer=self._in_o)
            else:
                ops.gemv(L.o, b.attn, out=b.o_part)
                self._reduce("o", b.o_part, b.x, b.x_mid)
                ops.rmsnorm_swiglu(L.gate, L.up, b.x_mid, L.g_ffn, eps=cfg.eps, out=b.h)
            if single:
                ops.gemv_residual(L.down, b.h, b.x_mid, out=b.x)
            elif fused and li < last:
                ops.gemv_peer(L.down, b.h, self.peer.dsts["d_ll"], p.rank, p.world)
            else:
                ops.gemv(L.down, b.h, out=b.d_part)
                self._reduce("d", b.d_part, b.x_mid, b.x)
        return b.x

    def timed_out(self) -> bool:
        """True if a wait on another rank ran out in any step so far (reads
        and clears the device status word; synchronises)."""
        if self.peer is None:
            return False
        return self.peer.timed_out() or bool(ops.device_status(clear=True) & 8)

    def kernels_per_step(self) -> int:
        """Launches of this library per step (collective-library kernels excluded)."""
        if self.program is not None:
            return 1
        if self.exchange == "p2p":
            return 5 * self.cfg.layers + 1
        return (7 if self.exchange == "p2p-kernel" else 5) * self.cfg.layers
