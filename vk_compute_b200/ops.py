"""Torch-facing operators over the C ABI of libvkcompute.

Tensors supply device memory and the current CUDA stream; every operator
is one call into the sm_100a library (include/vk_compute_b200.h).
Weights use vk-compute's storage: the 16-byte chunk layout of
src/data.c:198-222 plus block-major fp32 scale/zero per (k, 256 outputs).
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import torch

from ._lib import check, lib

GROUP = 256


def _p(t: torch.Tensor | None) -> C.c_void_p | None:
    return None if t is None else C.c_void_p(t.data_ptr())


def _s(stream: torch.cuda.Stream | None = None) -> C.c_void_p:
    s = torch.cuda.current_stream() if stream is None else stream
    return C.c_void_p(s.cuda_stream)


def chunk_elems(bits: int) -> int:
    """Weights per 16-byte chunk (k values of one output)."""
    return 128 // bits


@dataclass
class PackedWeight:
    """One K x N weight matrix (y[j] = sum_k x[k] W[k][j]) in device memory."""

    bits: int
    K: int
    N: int
    packed: torch.Tensor          # uint8, (K / chunk_elems) * N * 16 bytes
    scale: torch.Tensor | None    # fp32 [N/256 * K], block-major (quantised only)
    zero: torch.Tensor | None

    @property
    def nbytes(self) -> int:
        n = self.packed.numel()
        if self.scale is not None:
            n += 4 * (self.scale.numel() + self.zero.numel())
        return n

    def shard(self, lo: int, hi: int) -> "PackedWeight":
        """Copy of outputs [lo, hi) (a row shard of W^T).  Chunk rows are
        contiguous N*16-byte streams, so the shard is a strided gather of
        (hi-lo)*16 bytes per chunk row; scale/zero blocks are contiguous."""
        if self.bits <= 8 and (lo % GROUP or hi % GROUP):
            raise ValueError("quantised shards must be 256-output aligned")
        R = self.K // chunk_elems(self.bits)
        p = self.packed.view(R, self.N, 16)[:, lo:hi].contiguous().view(-1)
        s = z = None
        if self.scale is not None:
            s = self.scale.view(self.N // GROUP, self.K)[lo // GROUP:hi // GROUP].contiguous().view(-1)
            z = self.zero.view(self.N // GROUP, self.K)[lo // GROUP:hi // GROUP].contiguous().view(-1)
        return PackedWeight(self.bits, self.K, hi - lo, p, s, z)

    def columns(self, ranges: list[tuple[int, int]]) -> "PackedWeight":
        """Copy of the outputs in `ranges` ([lo, hi) pairs, concatenated in
        order): a row shard of W^T made of several row ranges."""
        parts = [self.shard(lo, hi) for lo, hi in ranges]
        if len(parts) == 1:
            return parts[0]
        R = self.K // chunk_elems(self.bits)
        n = sum(p.N for p in parts)
        p = torch.cat([q.packed.view(R, q.N, 16) for q in parts], dim=1).contiguous().view(-1)
        s = z = None
        if self.scale is not None:
            s = torch.cat([q.scale.view(q.N // GROUP, self.K) for q in parts]).contiguous().view(-1)
            z = torch.cat([q.zero.view(q.N // GROUP, self.K) for q in parts]).contiguous().view(-1)
        return PackedWeight(self.bits, self.K, n, p, s, z)

    def rows(self, lo: int, hi: int) -> "PackedWeight":
        """Copy of inputs [lo, hi) (a K-split shard: y_partial = W[lo:hi]^T
        x[lo:hi]).  Chunk rows are whole runs of 128/bits inputs, so the
        shard is a contiguous byte range; scale/zero keep their blocks."""
        kpc = chunk_elems(self.bits)
        if lo % kpc or hi % kpc:
            raise ValueError(f"a {self.bits}-bit K-split shard must start and end on {kpc}-input chunks")
        R = self.K // kpc
        p = self.packed.view(R, self.N, 16)[lo // kpc:hi // kpc].contiguous().view(-1)
        s = z = None
        if self.scale is not None:
            s = self.scale.view(self.N // GROUP, self.K)[:, lo:hi].contiguous().view(-1)
            z = self.zero.view(self.N // GROUP, self.K)[:, lo:hi].contiguous().view(-1)
        return PackedWeight(self.bits, hi - lo, self.N, p, s, z)


def save_weights(path: str, weights: dict[str, PackedWeight]) -> None:
    """Writes named packed matrices to `path` in the device layout
    (vkc_weights_write; the arrays are copied to host memory first)."""
    from ._lib import WeightEntry

    entries = (WeightEntry * len(weights))()
    keep = []
    for e, (name, w) in zip(entries, weights.items()):
        if len(name.encode()) >= 64:
            raise ValueError(f"matrix name {name!r} is longer than 63 bytes")
        e.name, e.bits, e.K, e.N = name.encode(), w.bits, w.K, w.N
        arrs = [w.packed.cpu().contiguous()]
        if w.scale is not None:
            arrs += [w.scale.cpu().contiguous(), w.zero.cpu().contiguous()]
        keep.append(arrs)
        e.data = arrs[0].data_ptr()
        if w.scale is not None:
            e.scale, e.zero = arrs[1].data_ptr(), arrs[2].data_ptr()
    check(lib().vkc_weights_write(str(path).encode(), entries, len(weights)))


def load_weights(path: str, device="cuda", names=None, stream=None) -> dict[str, PackedWeight]:
    """Reads named matrices (all, or `names`) from a vkc_weights_write file
    straight into device memory."""
    from ._lib import WeightEntry

    f = C.c_void_p()
    check(lib().vkc_weights_open(str(path).encode(), C.byref(f)))
    out = {}
    try:
        n = lib().vkc_weights_count(f)
        for i in range(n):
            info = WeightEntry()
            check(lib().vkc_weights_info(f, i, C.byref(info)))
            name = info.name.decode()
            if names is not None and name not in names:
                continue
            w = _alloc_weight(info.bits, info.K, info.N, device)
            check(lib().vkc_weights_read(f, i, _p(w.packed), _p(w.scale), _p(w.zero), _s(stream)))
            out[name] = w
    finally:
        lib().vkc_weights_close(f)
    return out


def _alloc_weight(bits: int, K: int, N: int, device) -> PackedWeight:
    packed = torch.empty(K * N * bits // 8, dtype=torch.uint8, device=device)
    s = z = None
    if bits <= 8:
        s = torch.empty(N // GROUP * K, dtype=torch.float32, device=device)
        z = torch.empty_like(s)
    return PackedWeight(bits, K, N, packed, s, z)


def pack_dense(w: torch.Tensor, bits: int, symmetric: bool = True, fp16_scale: bool = True,
               stream=None) -> PackedWeight:
    """Quantise (bits 8/4) or convert (16/32) a dense K x N matrix on the GPU
    and pack it.  16-bit weights are rounded to nearest by torch."""
    K, N = w.shape
    dev = w.device
    out = _alloc_weight(bits, K, N, dev)
    st = _s(stream)
    if bits in (32, 16):
        src = w.to(torch.float32 if bits == 32 else torch.float16).contiguous()
        check(lib().vkc_pack_block16(_p(src), _p(out.packed), K, N, bits, st))
        return out
    codes = torch.empty(K * N * bits // 8, dtype=torch.uint8, device=dev)
    wf = w.to(torch.float32).contiguous()
    check(lib().vkc_quantize(_p(wf), K, N, bits, int(symmetric), int(fp16_scale), _p(codes),
                             _p(out.scale), _p(out.zero), st))
    check(lib().vkc_pack_block16(_p(codes), _p(out.packed), K, N, bits, st))
    return out


def reference_weight(seed: int, K: int, N: int, bits: int, device="cuda", stream=None) -> PackedWeight:
    """The reference's seeded weights (src/compute.c:20-46): get_pseudo_random
    values, fp16 by truncation, int8/int4 by the min/max quantiser, packed by
    transpose_block16 -- all on the GPU, bit-identical to src/data.c."""
    out = _alloc_weight(bits, K, N, device)
    st = _s(stream)
    if bits in (32, 16):
        raw = torch.empty(K * N, dtype=torch.float32 if bits == 32 else torch.int16, device=device)
        check(lib().vkc_generate(seed, K, N, bits, _p(raw), st))
        check(lib().vkc_pack_block16(_p(raw), _p(out.packed), K, N, bits, st))
        return out
    vals = torch.empty(K * N, dtype=torch.float32, device=device)
    check(lib().vkc_generate(seed, K, N, 32, _p(vals), st))
    codes = torch.empty(K * N * bits // 8, dtype=torch.uint8, device=device)
    check(lib().vkc_quantize(_p(vals), K, N, bits, 0, 0, _p(codes), _p(out.scale), _p(out.zero), st))
    check(lib().vkc_pack_block16(_p(codes), _p(out.packed), K, N, bits, st))
    return out


def reference_vector(seed: int, n: int, device="cuda", stream=None) -> torch.Tensor:
    """getData(seed, 1, n) (src/data.c:18-28) on the GPU."""
    v = torch.empty(n, dtype=torch.float32, device=device)
    check(lib().vkc_generate(seed, 1, n, 32, _p(v), _s(stream)))
    return v


def _out(n: int, like: torch.Tensor, out: torch.Tensor | None) -> torch.Tensor:
    if out is None:
        return torch.empty(n, dtype=torch.float32, device=like.device)
    return out


def gemv(w: PackedWeight, x: torch.Tensor, out=None, stream=None) -> torch.Tensor:
    y = _out(w.N, x, out)
    check(lib().vkc_gemv(w.bits, _p(w.packed), _p(w.scale), _p(w.zero), _p(x), _p(y), w.N, w.K, _s(stream)))
    return y


def gemv_batched(w: PackedWeight, x: torch.Tensor, out=None, stream=None) -> torch.Tensor:
    """y[m] = W^T x[m] for the rows of x ([M][K], M <= 8), weights read once."""
    M = x.shape[0]
    y = out if out is not None else torch.empty(M, w.N, dtype=torch.float32, device=x.device)
    check(lib().vkc_gemv_batched(w.bits, _p(w.packed), _p(w.scale), _p(w.zero), _p(x), _p(y), M, w.N, w.K,
                                 _s(stream)))
    return y


def rmsnorm_gemv_batched(w: PackedWeight, x: torch.Tensor, gamma, eps: float = 1e-6, rms_dim: int | None = None,
                         out=None, stream=None) -> torch.Tensor:
    """RmsNorm-GEMV of each row of x ([M][K], M <= 8), weights read once."""
    M = x.shape[0]
    y = out if out is not None else torch.empty(M, w.N, dtype=torch.float32, device=x.device)
    check(lib().vkc_rmsnorm_gemv_batched(w.bits, _p(w.packed), _p(w.scale), _p(w.zero), _p(x), _p(gamma), _p(y),
                                         M, w.N, w.K, eps, rms_dim or w.K, _s(stream)))
    return y


def gemv_residual(w: PackedWeight, x: torch.Tensor, residual: torch.Tensor, out=None, stream=None) -> torch.Tensor:
    """y = W^T x + residual."""
    y = _out(w.N, x, out)
    check(lib().vkc_gemv_residual(w.bits, _p(w.packed), _p(w.scale), _p(w.zero), _p(x), _p(residual), _p(y),
                                  w.N, w.K, _s(stream)))
    return y


class PeerInput(C.Structure):
    """vkc_peer_input: x = base + the `world` slots of this rank's [world][K]
    word buffer (flag << 32 | fp32 bits, filled by the ranks' gemv_peer),
    each element read once its flag matches this rank's own; x is also
    stored to `save`."""

    _fields_ = [("slots", C.c_void_p), ("save", C.c_void_p), ("rank", C.c_int), ("world", C.c_int)]


def gemv_peer(w: PackedWeight, x: torch.Tensor, slots: torch.Tensor, rank: int, world: int, stream=None) -> None:
    """This rank's K-split partial W^T x stored into slot `rank` of every
    rank's word buffer (`slots`: int64 device tensor of the ranks' buffer
    addresses), each value with its flag."""
    check(lib().vkc_gemv_peer(w.bits, _p(w.packed), _p(w.scale), _p(w.zero), _p(x), _p(slots), rank, world, w.N,
                              w.K, _s(stream)))


KV_LAYOUTS = {"split": 0, "interleaved": 1}


def qkv_rope_append(w: PackedWeight, x, gamma, theta, pos: int, *, head_dim: int, q_rows: int, kv_rows: int,
                    kcache: torch.Tensor, vcache: torch.Tensor, ctx_cap: int, eps: float = 1e-6,
                    rms_dim: int | None = None, out=None, stream=None, peer: PeerInput | None = None,
                    kv_layout: str = "split") -> torch.Tensor:
    """Fused QKV projection + RoPE + KV-cache append at token `pos`; with
    `peer`, the input is x (the base) plus the peer exchange's slots.  The
    rows after Q are [K heads | V heads] ("split") or [K0 V0 | K1 V1 | ...]
    ("interleaved")."""
    y = _out(w.N, x, out)
    lay = KV_LAYOUTS[kv_layout]
    if peer is None:
        check(lib().vkc_rmsnorm_gemv_rope_kv(w.bits, _p(w.packed), _p(w.scale), _p(w.zero), _p(x), _p(gamma),
                                             _p(theta), _p(y), w.N, w.K, eps, rms_dim or w.K, pos, head_dim, q_rows,
                                             kv_rows, lay, _p(kcache), _p(vcache), ctx_cap, _s(stream)))
    else:
        check(lib().vkc_rmsnorm_gemv_rope_kv_peer(w.bits, _p(w.packed), _p(w.scale), _p(w.zero), _p(x),
                                                  C.addressof(peer), _p(gamma), _p(theta), _p(y), w.N, w.K, eps,
                                                  rms_dim or w.K, pos, head_dim, q_rows, kv_rows, lay, _p(kcache),
                                                  _p(vcache), ctx_cap, _s(stream)))
    return y


def rmsnorm_gemv(w: PackedWeight, x, gamma, eps: float = 1e-6, rms_dim: int | None = None,
                 out=None, stream=None) -> torch.Tensor:
    y = _out(w.N, x, out)
    check(lib().vkc_rmsnorm_gemv(w.bits, _p(w.packed), _p(w.scale), _p(w.zero), _p(x), _p(gamma), _p(y),
                                 w.N, w.K, eps, rms_dim or w.K, _s(stream)))
    return y


def rmsnorm_gemv_rope(w: PackedWeight, x, gamma, theta, pos: int, *, mode: str = "pairs",
                      head_dim: int = 128, rot_rows: int | None = None, eps: float = 1e-6,
                      rms_dim: int | None = None, out=None, stream=None) -> torch.Tensor:
    y = _out(w.N, x, out)
    m = {"reference": 0, "pairs": 1}[mode]
    rot = w.N if rot_rows is None else rot_rows
    check(lib().vkc_rmsnorm_gemv_rope(w.bits, _p(w.packed), _p(w.scale), _p(w.zero), _p(x), _p(gamma),
                                      _p(theta), _p(y), w.N, w.K, eps, rms_dim or w.K, pos, m, head_dim,
                                      rot, _s(stream)))
    return y


def rmsnorm_swiglu(wg: PackedWeight, wu: PackedWeight, x, gamma, eps: float = 1e-6,
                   rms_dim: int | None = None, out=None, stream=None, peer: PeerInput | None = None) -> torch.Tensor:
    """h = SiLU(Wg^T n) * (Wu^T n), n = RmsNorm(x) * gamma; with `peer`, the
    input is x (the base) plus the peer exchange's slots."""
    h = _out(wg.N, x, out)
    if peer is None:
        check(lib().vkc_rmsnorm_swiglu(wg.bits, _p(wg.packed), _p(wg.scale), _p(wg.zero), _p(wu.packed),
                                       _p(wu.scale), _p(wu.zero), _p(x), _p(gamma), _p(h), wg.N, wg.K, eps,
                                       rms_dim or wg.K, _s(stream)))
    else:
        check(lib().vkc_rmsnorm_swiglu_peer(wg.bits, _p(wg.packed), _p(wg.scale), _p(wg.zero), _p(wu.packed),
                                            _p(wu.scale), _p(wu.zero), _p(x), C.addressof(peer), _p(gamma), _p(h),
                                            wg.N, wg.K, eps, rms_dim or wg.K, _s(stream)))
    return h


def attention_workspace(n_q: int, n_kv: int, head_dim: int, ctx: int, device="cuda") -> torch.Tensor:
    n = lib().vkc_attention_workspace_bytes(n_q, n_kv, head_dim, ctx)
    return torch.zeros(n, dtype=torch.uint8, device=device)


def attention_decode(q, kcache, vcache, n_q: int, n_kv: int, head_dim: int, ctx: int,
                     scale: float, workspace: torch.Tensor | None = None, out=None,
                     stream=None, ctx_cap: int | None = None, after_append: bool = False) -> torch.Tensor:
    """q [n_q*hd] fp16 or fp32; kcache fp16 [cap][n_kv][hd];
    vcache fp16 [n_kv][hd/8][cap][8] with cap = ctx_cap (default ctx);
    attends tokens [0, ctx).  after_append: the previous kernel wrote only
    token ctx - 1 of the caches (vkc_attention_decode_append)."""
    o = _out(n_q * head_dim, q, out)
    qb = 32 if q.dtype == torch.float32 else 16
    ws_n = 0 if workspace is None else workspace.numel()
    if after_append:
        check(lib().vkc_attention_decode_append(_p(q), qb, _p(kcache), _p(vcache), _p(o), n_q, n_kv, head_dim, ctx,
                                                ctx_cap or ctx, scale, _p(workspace), ws_n, _s(stream)))
    elif ctx_cap is None:
        check(lib().vkc_attention_decode(_p(q), qb, _p(kcache), _p(vcache), _p(o), n_q, n_kv, head_dim, ctx,
                                         scale, _p(workspace), ws_n, _s(stream)))
    else:
        check(lib().vkc_attention_decode_cache(_p(q), qb, _p(kcache), _p(vcache), _p(o), n_q, n_kv, head_dim, ctx,
                                               ctx_cap, scale, _p(workspace), ws_n, _s(stream)))
    return o


def rmsnorm_rows(x: torch.Tensor, gamma: torch.Tensor, eps: float = 1e-5, stream=None) -> torch.Tensor:
    """In-place RMSNorm of each row of x ([rows][width] fp32) with gamma[width]
    (shader/RmsNorm.comp with width 256)."""
    rows, width = x.shape
    check(lib().vkc_rmsnorm_rows(_p(x), _p(gamma), rows, width, eps, _s(stream)))
    return x


def gemv_rowmajor(w: torch.Tensor, x: torch.Tensor, out=None, stream=None) -> torch.Tensor:
    """y = W^T x for a plain row-major K x N fp32 matrix (shader/gemv2.comp,
    gemv3.comp; gemv1.comp for square W)."""
    K, N = w.shape
    y = _out(N, x, out)
    check(lib().vkc_gemv_rowmajor(_p(w), _p(x), _p(y), N, K, _s(stream)))
    return y


def gemm_f32(a: torch.Tensor, b: torch.Tensor, out=None, stream=None) -> torch.Tensor:
    M, K = a.shape
    K2, N = b.shape
    assert K == K2
    c = torch.empty(M, N, dtype=torch.float32, device=a.device) if out is None else out
    check(lib().vkc_gemm_f32(_p(a), _p(b), _p(c), M, N, K, _s(stream)))
    return c


def gemm_bf16(a: torch.Tensor, w: torch.Tensor, out=None, stream=None) -> torch.Tensor:
    """C = A W^T on the tcgen05 tensor cores: A [M, K] and W [N, K] bf16
    (contiguous), C [M, N] fp32."""
    if a.dtype != torch.bfloat16 or w.dtype != torch.bfloat16:
        raise TypeError("gemm_bf16 takes bf16 A and W")
    a, w = a.contiguous(), w.contiguous()
    M, K = a.shape
    N, K2 = w.shape
    if K != K2:
        raise ValueError(f"A is {M}x{K} but W is {N}x{K2}")
    c = torch.empty(M, N, dtype=torch.float32, device=a.device) if out is None else out
    check(lib().vkc_gemm_bf16(_p(a), _p(w), _p(c), M, N, K, _s(stream)))
    return c


def gemm_bf16_status(clear: bool = True) -> int:
    v = C.c_uint(0)
    check(lib().vkc_gemm_bf16_status(C.byref(v), int(clear)))
    return v.value


def set_pdl(enable: bool) -> None:
    lib().vkc_set_pdl(int(enable))


def get_pdl() -> bool:
    return bool(lib().vkc_get_pdl())


GEMV_PLANS = {"auto": 0, "cluster": 1, "per-sm": 2, "per-sm-half": 3, "auto-full": 4}


def set_gemv_plan(plan: str) -> None:
    """Kernel of the single-vector GEMV family (vkc_set_gemv_plan): "auto"
    chooses per shape, "cluster" always splits K across a cluster, "per-sm"
    runs one CTA per SM with whole-K column ranges wherever it can (a 1024-
    thread CTA owning the SM), "per-sm-half" the same with a 512-thread CTA
    that leaves half the SM to the next launch, "auto-full" chooses per shape
    with the 1024-thread CTA.  Per host thread."""
    check(lib().vkc_set_gemv_plan(GEMV_PLANS[plan]))


def set_gemv_int_dot(enable: bool) -> None:
    """8/4-bit weights on the per-SM GEMV kernel: integer dot products over
    16-bit activations per chunk row (True, the default) or fp32 FMAs
    (vkc_set_gemv_int_dot).  Per host thread."""
    lib().vkc_set_gemv_int_dot(int(enable))


def get_gemv_int_dot() -> bool:
    return bool(lib().vkc_get_gemv_int_dot())


ATTENTION_PLANS = {"auto": 0, "clustered": 1, "per-sm": 2, "per-sm-half": 3, "per-sm-x2": 4, "per-sm-wide": 5}


def set_attention_plan(plan: str) -> None:
    """Decode attention's split of the cache (vkc_set_attention_plan):
    "auto" per shape, "clustered" (clusters of 8 CTAs per KV head, two CTAs
    per SM), "per-sm" (at most one CTA per SM, deep ring), "per-sm-half" (the
    same with a 3-stage ring in at most half an SM), "per-sm-x2" (two such
    CTAs per SM over twice the splits), "per-sm-wide" (the per-SM shape with
    two warp groups per CTA on alternate sub-tiles; the automatic choice
    wherever the per-SM shape applies).  Per host thread."""
    check(lib().vkc_set_attention_plan(ATTENTION_PLANS[plan]))


def get_attention_plan() -> str:
    v = lib().vkc_get_attention_plan()
    return next(k for k, n in ATTENTION_PLANS.items() if n == v)


def attention_plan_info(n_q: int, n_kv: int, head_dim: int, ctx: int) -> dict:
    """The split decode attention uses for a shape under the calling thread's
    plan (vkc_attention_plan_info)."""
    import ctypes as C

    info = (C.c_int * 7)()
    check(lib().vkc_attention_plan_info(n_q, n_kv, head_dim, ctx, info))
    kinds = {1: "token-slice clustered", 2: "token-slice per-SM", 3: "tensor-core hd256", 4: "SIMT"}
    return {"kernel": kinds[info[0]], "splits": info[1], "tokens_per_cta": info[2], "stages": info[3],
            "warp_groups": info[4], "cluster": info[5], "records": info[6]}


def get_gemv_plan() -> str:
    v = lib().vkc_get_gemv_plan()
    return next(k for k, n in GEMV_PLANS.items() if n == v)


def device_status(clear: bool = False) -> int:
    """Status word of the current device (waits for it); flags 0x1 producer,
    0x2 consumer, 0x4 cluster reduction, 0x8 peer-exchange, 0x10 tcgen05
    GEMM pipeline, 0x20 persistent-decoder grid barrier wait ran out."""
    v = C.c_uint(0)
    check(lib().vkc_device_status(C.byref(v), int(clear)))
    return int(v.value)
