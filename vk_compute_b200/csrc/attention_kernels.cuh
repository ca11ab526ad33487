// Device code of decode attention (the kernels and their helpers), included
// by attention.cu for the standalone launches and by gemv.cu for the
// persistent decoder kernel, which runs the token-slice kernel's body as one
// of its phases.  Everything but the parameter block is TU-local.
#pragma once
#include "vkc_common.cuh"

#include <cuda_fp16.h>

#include <type_traits>

namespace vkc {

constexpr int kAttThreads = 256;
constexpr int kAttStages = 3;

// Ring geometry of the tensor-core decode attention kernels for one head_dim.
template <int HD>
struct MmaGeo {
    static constexpr int CH = HD / 8;              // 16-byte chunks per K row
    static constexpr int TT = 8192 / HD;           // tokens per sub-tile (32 KB of K + V)
    static constexpr int KROW = CH + 1;            // K row pitch (units), padded
    static constexpr int VROW = TT + 1;            // V run pitch (units), padded
    static constexpr int KU = TT * KROW;
    static constexpr int SU = KU + CH * VROW;      // units per ring stage
    static constexpr int NT = TT / 8;              // token tiles (scores n-tiles)
    static constexpr int KG = NT >= 8 ? 1 : 8 / NT;          // warps sharing a token tile
    static constexpr int TPW = NT >= 8 ? NT / 8 : 1;         // token tiles per warp
    static constexpr int KS = HD / 16 / KG;                  // score k-steps per warp
    static constexpr int NP = HD / 16;             // pairs of 8-dimension n-tiles
    static constexpr int WN = NP < 8 ? NP : 8;     // warps along dimensions
    static constexpr int WK = 8 / WN;              // warps along tokens
    static constexpr int PPW = NP / WN;            // dimension pairs per warp
    static constexpr int PKS = TT / 16 / WK;       // P.V k-steps per warp
    static constexpr int PROW = TT + 8;            // halves per P row (conflict-free A loads)
    static constexpr size_t ring_bytes = static_cast<size_t>(kAttStages) * SU * 16;
    static constexpr size_t sc_bytes = static_cast<size_t>(KG) * 8 * TT * sizeof(float);
    static constexpr size_t p_bytes = 2ull * 8 * PROW * sizeof(__half);
    static constexpr size_t q_bytes = static_cast<size_t>(HD / 16) * 32 * 16;
    static constexpr size_t smem_bytes = ring_bytes + sc_bytes + p_bytes + q_bytes;
    static_assert(KS % 2 == 0 && NT * KG >= 8 && WN * WK == 8 && PKS >= 1, "geometry");
};

struct AttnParams {
    const void* q;
    int q_bits;  // 16 (fp16) or 32 (fp32)
    const uint4* kc;
    const uint4* vc;
    float* out;
    float* ws;          // [n_q][splits][pitch] : acc[hd], m, l (pitch = hd + 4)
    unsigned* tickets;  // [n_kv]
    int n_q, n_kv, hd, ctx, splits, tpc;
    int ctx_cap;        // V run length per (head, chunk): the cache capacity
    int tt;             // tokens per sub-tile (a multiple of 32)
    float scale_log2;   // scale * log2(e)
    int pitch;          // floats per partial record, hd + 4 (a multiple of 4)
    int smem;           // dynamic shared memory of the launch (bytes)
    int stable;         // tokens [0, stable) are written by no kernel still in flight
    int pre_max;        // sub-tiles per warp group requested before the wait (0: as many as stable allows)
};

namespace {

constexpr float kLog2e = 1.4426950408889634f;


// One ring stage in 16-byte units: K sub-tile [tt][chunks], then the V
// sub-tile [chunks][tt + 1] (one unit of padding per run makes the P.V reads,
// lanes over 8 chunks of one token, hit 32 distinct banks).
__host__ __device__ __forceinline__ int att_v_stride(int tt) { return tt + 1; }
__host__ __device__ __forceinline__ int att_stage_units(int tt, int chunks) {
    return tt * chunks + chunks * att_v_stride(tt);
}

__device__ __forceinline__ void cp_async16_zfill(uint32_t dst, const void* src, bool valid) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(valid ? 16 : 0)
                 : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ float2 half2_bits_to_float2(uint32_t w) {
    return __half22float2(*reinterpret_cast<const __half2*>(&w));
}

// Sums G per-lane values over the `lpt` lanes of a row group (lpt a power of
// two >= G) by halving exchanges: each level trades half of the remaining
// values with the partner lane, so G heads cost log2(lpt) + G - 1 shuffles
// instead of G log2(lpt).  Returns the total of head `g` (set on return).
template <int G>
__device__ __forceinline__ float reduce_heads(float (&v)[G], int lane, int lpt, int& g) {
    int m = lpt >> 1;
    g = 0;
    if constexpr (G == 4) {
        const bool up = lane & m;
        const float s0 = up ? v[0] : v[2], s1 = up ? v[1] : v[3];
        const float k0 = up ? v[2] : v[0], k1 = up ? v[3] : v[1];
        v[0] = k0 + __shfl_xor_sync(0xffffffffu, s0, m);
        v[1] = k1 + __shfl_xor_sync(0xffffffffu, s1, m);
        g = up ? 2 : 0;
        m >>= 1;
    }
    if constexpr (G >= 2) {
        const bool up = lane & m;
        const float s0 = up ? v[0] : v[1], k0 = up ? v[1] : v[0];
        v[0] = k0 + __shfl_xor_sync(0xffffffffu, s0, m);
        g += up ? 1 : 0;
        m >>= 1;
    }
    float r = v[0];
    for (; m >= 1; m >>= 1) r += __shfl_xor_sync(0xffffffffu, r, m);
    return r;
}

// The last CTA of KV head `kv` to finish (atomic ticket) merges the S partial
// records of its G query heads in order and resets the ticket for the next
// launch:
//   w[g][s] = 2^(m_s - max_s m_s) / sum_s 2^(m_s - max_s m_s) l_s
//   out[g]  = sum_s w[g][s] acc_s
// The merge is on the critical path of every launch and is a chain of L2
// round trips, so it is kept short: when the G heads' records (contiguous in
// the workspace) fit in the CTA's shared memory they are staged with one
// round of 16-byte cp.async copies and merged there; otherwise they are read
// with many loads in flight per thread.
template <int G, int NT = kAttThreads>
__device__ __forceinline__ void merge_splits(const AttnParams& p, uint8_t* smem, int kv, int S) {
    __shared__ unsigned s_ticket;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int hd = p.hd, h0 = kv * G, pitch = p.pitch;
    __threadfence();  // this thread's partial writes, before the ticket
    __syncthreads();
    if (tid == 0) s_ticket = atomicAdd(p.tickets + kv, 1u);
    __syncthreads();
    if (s_ticket != static_cast<unsigned>(S - 1)) return;
    __threadfence();
    const float* src = p.ws + static_cast<size_t>(h0) * S * pitch;  // [G][S][pitch]
    const size_t rec_bytes = static_cast<size_t>(G) * S * pitch * sizeof(float);
    float* wts = reinterpret_cast<float*>(smem + rec_bytes);        // [G][S]
    if (rec_bytes + static_cast<size_t>(G) * S * sizeof(float) <= static_cast<size_t>(p.smem)) {
        const float* st = reinterpret_cast<const float*>(smem);
        const uint32_t dst = smem_addr(smem);
        const int units = static_cast<int>(rec_bytes / 16);
        for (int u = tid; u < units; u += NT) cp_async16_zfill(dst + u * 16, src + 4 * u, true);
        cp_commit();
        cp_wait<0>();
        __syncthreads();
        for (int g = warp; g < G; g += NT / 32) {
            float m = -INFINITY;
            for (int s2 = lane; s2 < S; s2 += 32) m = fmaxf(m, st[(g * S + s2) * pitch + hd]);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
            float den = 0.f;
            for (int s2 = lane; s2 < S; s2 += 32) {
                const float* r = st + (g * S + s2) * pitch + hd;
                const float w = exp2f(r[0] - m);
                wts[g * S + s2] = w;
                den = fmaf(w, r[1], den);
            }
            den = warp_sum(den);
            const float inv = 1.f / den;
            __syncwarp();
            for (int s2 = lane; s2 < S; s2 += 32) wts[g * S + s2] *= inv;
        }
        __syncthreads();
        for (int i = tid; i < G * hd; i += NT) {
            const int g = i / hd, d = i - g * hd;
            const float* r = st + g * S * pitch + d;
            const float* w = wts + g * S;
            float a0 = 0.f, a1 = 0.f;
            int s2 = 0;
            for (; s2 + 1 < S; s2 += 2) {
                a0 = fmaf(w[s2], r[s2 * pitch], a0);
                a1 = fmaf(w[s2 + 1], r[(s2 + 1) * pitch], a1);
            }
            if (s2 < S) a0 = fmaf(w[s2], r[s2 * pitch], a0);
            p.out[static_cast<size_t>(h0) * hd + i] = a0 + a1;
        }
    } else {
        // (m, l) of every (head, split), then four dimensions per thread with
        // the splits divided among thread groups, combined in fixed order.
        float2* ml = reinterpret_cast<float2*>(smem);                // [G][S]
        float* w2 = reinterpret_cast<float*>(ml + G * S);            // [G][S]
        for (int i = tid; i < G * S; i += NT)
            ml[i] = __ldcg(reinterpret_cast<const float2*>(src + static_cast<size_t>(i) * pitch + hd));
        __syncthreads();
        for (int g = warp; g < G; g += NT / 32) {
            float m = -INFINITY;
            for (int s2 = lane; s2 < S; s2 += 32) m = fmaxf(m, ml[g * S + s2].x);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
            float den = 0.f;
            for (int s2 = lane; s2 < S; s2 += 32) {
                const float2 v = ml[g * S + s2];
                const float w = exp2f(v.x - m);
                w2[g * S + s2] = w;
                den = fmaf(w, v.y, den);
            }
            den = warp_sum(den);
            const float inv = 1.f / den;
            __syncwarp();
            for (int s2 = lane; s2 < S; s2 += 32) w2[g * S + s2] *= inv;
        }
        __syncthreads();
        const int quads = G * hd / 4;
        const int ngroups = quads >= NT ? 1 : NT / quads;
        float4* part = reinterpret_cast<float4*>(smem + ((static_cast<size_t>(G) * S * 12 + 15) & ~size_t(15)));
        for (int qd = tid % quads; qd < quads; qd += NT) {
            const int grp = tid / quads;
            if (grp >= ngroups) break;
            const int g = (qd * 4) / hd, d = qd * 4 - g * hd;
            const float* rb = src + static_cast<size_t>(g) * S * pitch + d;
            const float* w = w2 + g * S;
            float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
            int s2 = grp;
            for (; s2 + 7 * ngroups < S; s2 += 8 * ngroups) {
                float4 v[8];
#pragma unroll
                for (int u = 0; u < 8; ++u)
                    v[u] = __ldcg(reinterpret_cast<const float4*>(rb + static_cast<size_t>(s2 + u * ngroups) * pitch));
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                    const float wu = w[s2 + u * ngroups];
                    acc.x = fmaf(wu, v[u].x, acc.x);
                    acc.y = fmaf(wu, v[u].y, acc.y);
                    acc.z = fmaf(wu, v[u].z, acc.z);
                    acc.w = fmaf(wu, v[u].w, acc.w);
                }
            }
            for (; s2 < S; s2 += ngroups) {
                const float4 v = __ldcg(reinterpret_cast<const float4*>(rb + static_cast<size_t>(s2) * pitch));
                const float wu = w[s2];
                acc.x = fmaf(wu, v.x, acc.x);
                acc.y = fmaf(wu, v.y, acc.y);
                acc.z = fmaf(wu, v.z, acc.z);
                acc.w = fmaf(wu, v.w, acc.w);
            }
            part[grp * quads + qd] = acc;
        }
        __syncthreads();
        for (int qd = tid; qd < quads; qd += NT) {
            float4 acc = part[qd];
            for (int grp = 1; grp < ngroups; ++grp) {
                const float4 v = part[grp * quads + qd];
                acc.x += v.x;
                acc.y += v.y;
                acc.z += v.z;
                acc.w += v.w;
            }
            *reinterpret_cast<float4*>(p.out + static_cast<size_t>(h0) * hd + qd * 4) = acc;
        }
    }
    if (tid == 0) p.tickets[kv] = 0u;
}

// The same merge for a record layout with at most NT float4 units per head
// group (G * HD / 4 <= NT): the last CTA of the head gives each thread four
// dimensions of one query head, and the thread folds the S records in order
// with a running maximum (rescaling its sums when the maximum grows).  The
// records are loaded 24 at a time into registers before any arithmetic, so
// the merge costs one round trip to L2 per 24 splits rather than a staged
// copy plus passes over shared memory.
// A barrier over the first NT threads of the CTA: __syncthreads() when they
// are the whole CTA (SYNC 0), else named barrier SYNC (a kernel whose other
// threads do other work meanwhile).
template <int SYNC, int NT>
__device__ __forceinline__ void part_sync() {
    if constexpr (SYNC == 0)
        __syncthreads();
    else
        asm volatile("bar.sync %0, %1;" ::"n"(SYNC), "n"(NT) : "memory");
}

template <int G, int HD, int NT, int SYNC = 0>
__device__ __forceinline__ void merge_splits_direct(const AttnParams& p, int kv, int S) {
    static_assert(G * HD / 4 <= NT, "one float4 of one head per thread");
    __shared__ unsigned s_ticket;
    const int tid = threadIdx.x;
    __threadfence();  // this CTA's record, before the ticket
    part_sync<SYNC, NT>();
    if (tid == 0) s_ticket = atomicAdd(p.tickets + kv, 1u);
    part_sync<SYNC, NT>();
    if (s_ticket != static_cast<unsigned>(S - 1)) return;
    __threadfence();
    // TPU threads per float4 unit (lanes next to each other), each folding
    // the splits s = part, part + TPU, ... in order; the parts combine in
    // part order through lane shuffles.
    constexpr int kUnits = G * HD / 4;
    constexpr int TPU = NT >= 2 * kUnits ? 2 : 1;
    const int unit = tid / TPU, part = tid % TPU;
    float M = -INFINITY, L = 0.f;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    const int g = (4 * unit) / HD, d = 4 * unit - g * HD;
    const int h = kv * G + g;
    if (unit < kUnits) {
        const float* rec = p.ws + static_cast<size_t>(h) * S * p.pitch;
        // records per round trip (fewer in a body sharing its kernel's
        // registers with other phases, SYNC != 0)
        constexpr int kChunk = SYNC == 0 ? 24 / TPU : 12 / TPU;
        for (int s0 = part; s0 < S; s0 += kChunk * TPU) {
            float2 ml[kChunk];
            float4 v[kChunk];
#pragma unroll
            for (int i = 0; i < kChunk; ++i) {
                const float* r = rec + static_cast<size_t>(min(s0 + i * TPU, S - 1)) * p.pitch;
                ml[i] = __ldcg(reinterpret_cast<const float2*>(r + HD));
                v[i] = __ldcg(reinterpret_cast<const float4*>(r + d));
            }
            float Mc = M;
#pragma unroll
            for (int i = 0; i < kChunk; ++i)
                if (s0 + i * TPU < S) Mc = fmaxf(Mc, ml[i].x);
            if (Mc == -INFINITY) continue;
            const float f = M == -INFINITY ? 0.f : exp2f(M - Mc);
            acc.x *= f;
            acc.y *= f;
            acc.z *= f;
            acc.w *= f;
            L *= f;
            M = Mc;
#pragma unroll
            for (int i = 0; i < kChunk; ++i) {
                if (s0 + i * TPU >= S || ml[i].x == -INFINITY) continue;
                const float w = exp2f(ml[i].x - M);
                L = fmaf(w, ml[i].y, L);
                acc.x = fmaf(w, v[i].x, acc.x);
                acc.y = fmaf(w, v[i].y, acc.y);
                acc.z = fmaf(w, v[i].z, acc.z);
                acc.w = fmaf(w, v[i].w, acc.w);
            }
        }
    }
    if constexpr (TPU == 2) {
        // part 0 takes part 1's state (the lane above it)
        const float M1 = __shfl_down_sync(0xffffffffu, M, 1), L1 = __shfl_down_sync(0xffffffffu, L, 1);
        float4 a1;
        a1.x = __shfl_down_sync(0xffffffffu, acc.x, 1);
        a1.y = __shfl_down_sync(0xffffffffu, acc.y, 1);
        a1.z = __shfl_down_sync(0xffffffffu, acc.z, 1);
        a1.w = __shfl_down_sync(0xffffffffu, acc.w, 1);
        const float Mt = fmaxf(M, M1);
        const float f0 = M == -INFINITY ? 0.f : exp2f(M - Mt), f1 = M1 == -INFINITY ? 0.f : exp2f(M1 - Mt);
        L = L * f0 + L1 * f1;
        acc.x = acc.x * f0 + a1.x * f1;
        acc.y = acc.y * f0 + a1.y * f1;
        acc.z = acc.z * f0 + a1.z * f1;
        acc.w = acc.w * f0 + a1.w * f1;
    }
    if (unit < kUnits && part == 0) {
        const float inv = 1.f / L;
        *reinterpret_cast<float4*>(p.out + static_cast<size_t>(h) * HD + d) =
            make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv);
    }
    if (tid == 0) p.tickets[kv] = 0u;
}

template <int G>
__global__ void __launch_bounds__(kAttThreads, 2) attention_decode_kernel(const AttnParams p) {
    extern __shared__ __align__(16) uint8_t smem[];
    __shared__ float s_m[G], s_l[G], s_f[G];

    const int split = blockIdx.x, kv = blockIdx.y;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int hd = p.hd, chunks = hd / 8, TT = p.tt;
    const int t0 = split * p.tpc;
    const int T = min(p.tpc, p.ctx - t0);
    const int nsub = (T + TT - 1) / TT;
    const int h0 = kv * G;
    const int k_units = TT * chunks, vstride = att_v_stride(TT);
    const int stage_units = att_stage_units(TT, chunks);
    uint4* ring = reinterpret_cast<uint4*>(smem);
    float* qs = reinterpret_cast<float*>(smem + static_cast<size_t>(kAttStages) * stage_units * 16);  // [G][hd]
    float* sc = qs + G * hd;                                                                          // [G][TT]

    pdl_launch_dependents();
    // The cache row of the current token and q may come from the previous kernel.
    pdl_wait();

    auto issue = [&](int s) {
        uint4* base = ring + (s % kAttStages) * stage_units;
        const int ts = t0 + s * TT;
        const int nt = min(TT, T - s * TT);
        for (int u = tid; u < TT * chunks; u += kAttThreads) {
            const int t = u / chunks, c = u - t * chunks;
            const bool ok = t < nt;
            const uint4* src = p.kc + (static_cast<size_t>(ok ? ts + t : t0) * p.n_kv + kv) * chunks + c;
            cp_async16_zfill(smem_addr(base + u), src, ok);
        }
        for (int u = tid; u < TT * chunks; u += kAttThreads) {
            const int c = u / TT, t = u - c * TT;
            const bool ok = t < nt;
            const uint4* src = p.vc + (static_cast<size_t>(kv) * chunks + c) * p.ctx_cap + (ok ? ts + t : t0);
            cp_async16_zfill(smem_addr(base + k_units + c * vstride + t), src, ok);
        }
    };
#pragma unroll
    for (int s = 0; s < kAttStages - 1; ++s) {
        if (s < nsub) issue(s);
        cp_commit();
    }

    for (int i = tid; i < G * hd; i += kAttThreads) {
        const int g = i / hd, d = i - g * hd;
        const size_t qi = static_cast<size_t>(h0 + g) * hd + d;
        qs[i] = p.q_bits == 16 ? __half2float(reinterpret_cast<const __half*>(p.q)[qi])
                               : reinterpret_cast<const float*>(p.q)[qi];
    }
    if (tid < G) {
        s_m[tid] = -INFINITY;
        s_l[tid] = 0.f;
    }
    __syncthreads();

    // Score mapping: `lpt` lanes (a power of two >= chunks) share a K row;
    // lane `sub` owns dimensions [8 sub, 8 sub + 8) and keeps q for them.
    int lpt = 1;
    while (lpt < chunks) lpt <<= 1;
    const int rpw = 32 / lpt;
    const int sub = lane & (lpt - 1), rw = lane / lpt;
    const bool split_heads = lpt >= G;
    float qr[G][8];
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
        for (int i = 0; i < 8; ++i) qr[g][i] = sub < chunks ? qs[g * hd + sub * 8 + i] : 0.f;

    // P.V mapping: thread owns dimensions (2 dp, 2 dp + 1) of every head and
    // tokens [tg * per, tg * per + per) of each sub-tile.
    const int pairs = hd / 2, ntg = kAttThreads / pairs;
    const int dp = tid % pairs, tg = tid / pairs;
    const bool pv = tg < ntg;
    const int per = (((TT + ntg - 1) / ntg) + 3) & ~3;
    const int lo = min(tg * per, TT), hi = min(lo + per, TT);
    const int vc_word = (dp >> 2) * vstride * 4 + (dp & 3);  // 32-bit word of (chunk, token 0)
    float acc[G][2];
#pragma unroll
    for (int g = 0; g < G; ++g) acc[g][0] = acc[g][1] = 0.f;

    for (int s = 0; s < nsub; ++s) {
        cp_wait<kAttStages - 2>();
        __syncthreads();  // sub-tile s landed for all; sub-tile s-1 fully consumed
        if (s + kAttStages - 1 < nsub) issue(s + kAttStages - 1);
        cp_commit();
        const uint4* base = ring + (s % kAttStages) * stage_units;
        const int nt = min(TT, T - s * TT);

        // (a) scores in base 2, -inf past the end of the range
        for (int tb = 0; tb < TT; tb += (kAttThreads / 32) * rpw) {
            const int t = tb + warp * rpw + rw;
            const bool row = t < TT;
            float dots[G];
            if (row && sub < chunks) {
                const uint4 kq = base[t * chunks + sub];
                const float2 k0 = half2_bits_to_float2(kq.x), k1 = half2_bits_to_float2(kq.y);
                const float2 k2 = half2_bits_to_float2(kq.z), k3 = half2_bits_to_float2(kq.w);
#pragma unroll
                for (int g = 0; g < G; ++g) {
                    float a = qr[g][0] * k0.x;
                    a = fmaf(qr[g][1], k0.y, a);
                    a = fmaf(qr[g][2], k1.x, a);
                    a = fmaf(qr[g][3], k1.y, a);
                    a = fmaf(qr[g][4], k2.x, a);
                    a = fmaf(qr[g][5], k2.y, a);
                    a = fmaf(qr[g][6], k3.x, a);
                    a = fmaf(qr[g][7], k3.y, a);
                    dots[g] = a;
                }
            } else {
#pragma unroll
                for (int g = 0; g < G; ++g) dots[g] = 0.f;
            }
            if (split_heads) {
                int g;
                const float r = reduce_heads<G>(dots, lane, lpt, g);
                if (row && (sub & (lpt / G - 1)) == 0) sc[g * TT + t] = t < nt ? r * p.scale_log2 : -INFINITY;
            } else {
#pragma unroll
                for (int o = 1; o < 32; o <<= 1)
                    if (o < lpt)
#pragma unroll
                        for (int g = 0; g < G; ++g) dots[g] += __shfl_xor_sync(0xffffffffu, dots[g], o);
                if (row && sub == 0)
#pragma unroll
                    for (int g = 0; g < G; ++g) sc[g * TT + t] = t < nt ? dots[g] * p.scale_log2 : -INFINITY;
            }
        }
        __syncthreads();

        // (b) online softmax, one warp per head
        if (warp < G) {
            const int g = warp;
            float mx = -INFINITY;
            for (int t = lane; t < TT; t += 32) mx = fmaxf(mx, sc[g * TT + t]);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
            const float m_old = s_m[g];
            const float m_new = fmaxf(m_old, mx);
            float sum = 0.f;
            for (int t = lane; t < TT; t += 32) {
                const float e = exp2f(sc[g * TT + t] - m_new);
                sc[g * TT + t] = e;
                sum += e;
            }
            sum = warp_sum(sum);
            if (lane == 0) {
                const float f = exp2f(m_old - m_new);
                s_m[g] = m_new;
                s_l[g] = s_l[g] * f + sum;
                s_f[g] = f;
            }
        }
        __syncthreads();

        // (c) P.V over this thread's tokens (zero V and zero weight past the end)
        if (pv) {
            const uint32_t* vw = reinterpret_cast<const uint32_t*>(base + k_units) + vc_word;
#pragma unroll
            for (int g = 0; g < G; ++g) {
                const float f = s_f[g];
                acc[g][0] *= f;
                acc[g][1] *= f;
            }
            for (int t = lo; t < hi; t += 4) {
                float4 pg[G];
#pragma unroll
                for (int g = 0; g < G; ++g) pg[g] = *reinterpret_cast<const float4*>(sc + g * TT + t);
                float2 v[4];
#pragma unroll
                for (int u = 0; u < 4; ++u) v[u] = half2_bits_to_float2(vw[(t + u) * 4]);
#pragma unroll
                for (int g = 0; g < G; ++g) {
                    acc[g][0] = fmaf(pg[g].x, v[0].x, acc[g][0]);
                    acc[g][1] = fmaf(pg[g].x, v[0].y, acc[g][1]);
                    acc[g][0] = fmaf(pg[g].y, v[1].x, acc[g][0]);
                    acc[g][1] = fmaf(pg[g].y, v[1].y, acc[g][1]);
                    acc[g][0] = fmaf(pg[g].z, v[2].x, acc[g][0]);
                    acc[g][1] = fmaf(pg[g].z, v[2].y, acc[g][1]);
                    acc[g][0] = fmaf(pg[g].w, v[3].x, acc[g][0]);
                    acc[g][1] = fmaf(pg[g].w, v[3].y, acc[g][1]);
                }
            }
        }
    }
    cp_wait<0>();
    __syncthreads();

    // Combine token groups (the ring is free now) and write the partial.
    float* red = reinterpret_cast<float*>(smem);  // [ntg][G][hd]
    if (pv)
#pragma unroll
        for (int g = 0; g < G; ++g)
            *reinterpret_cast<float2*>(red + (tg * G + g) * hd + 2 * dp) = make_float2(acc[g][0], acc[g][1]);
    __syncthreads();
    for (int i = tid; i < G * hd; i += kAttThreads) {
        const int g = i / hd, d = i - g * hd;
        float v = 0.f;
        for (int q = 0; q < ntg; ++q) v += red[(q * G + g) * hd + d];
        p.ws[(static_cast<size_t>(h0 + g) * p.splits + split) * p.pitch + d] = v;
    }
    if (tid < G) {
        float* rec = p.ws + (static_cast<size_t>(h0 + tid) * p.splits + split) * p.pitch + hd;
        rec[0] = s_m[tid];
        rec[1] = s_l[tid];
    }

    merge_splits<G>(p, smem, kv, p.splits);
}

// ---- tensor-core variant (head_dim 64 / 128 / 256) ---------------------------
//
// Same decomposition and ring; the two contractions run on mma.sync
// m16n8k16 (f16 inputs, f32 accumulation) with the G query heads as the rows
// of A (rows G..15 zero).  q and p are fp32: each is split into fp16 high and
// low parts (x = hi + lo, |lo| <= 2^-11 |x|) and both parts are multiplied, so
// the products carry about 22 significant bits, as fp32 FMAs would; K and V
// are fp16 already.  For a decode step (G <= 8 rows) the tensor cores only
// remove issue pressure: the per-token work drops from ~40 instructions to a
// few, leaving the kernel bound by the cache stream.
//
//   scores   C[g][t]  = sum_d q[g][d] K[t][d]   B = K sub-tile, ldmatrix (rows = tokens)
//   P.V      O[g][d] += sum_t p[g][t] V[t][d]   B = V sub-tile, ldmatrix.trans (rows = tokens)

__device__ __forceinline__ void mma16816(float (&c)[4], uint32_t a0, uint32_t a2, uint32_t b0, uint32_t b1) {
    // Rows 8..15 of A are zero (at most eight query heads per KV head).
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(0u), "r"(a2), "r"(0u), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t (&r)[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}
__device__ __forceinline__ uint32_t h2_bits(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
// fp16 high/low split of a pair of fp32 values.
__device__ __forceinline__ void split_pair(float x0, float x1, uint32_t& hi, uint32_t& lo) {
    const __half2 h = __floats2half2_rn(x0, x1);
    const float2 hf = __half22float2(h);
    hi = h2_bits(h);
    lo = h2_bits(__floats2half2_rn(x0 - hf.x, x1 - hf.y));
}


template <int G, int HD>
__global__ void __launch_bounds__(kAttThreads, 2) attention_mma_kernel(const AttnParams p) {
    using Geo = MmaGeo<HD>;
    constexpr int CH = Geo::CH, TT = Geo::TT, KROW = Geo::KROW, VROW = Geo::VROW, KU = Geo::KU, SU = Geo::SU;
    constexpr int NT = Geo::NT, KG = Geo::KG, TPW = Geo::TPW, KS = Geo::KS;
    constexpr int WN = Geo::WN, WK = Geo::WK, PPW = Geo::PPW, PKS = Geo::PKS, PROW = Geo::PROW;
    extern __shared__ __align__(16) uint8_t smem[];
    __shared__ float s_m[G], s_l[G], s_f[G];

    const int split = blockIdx.x, kv = blockIdx.y;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int gid = lane >> 2, t4 = lane & 3;
    const int t0 = split * p.tpc;
    const int T = min(p.tpc, p.ctx - t0);
    const int nsub = (T + TT - 1) / TT;
    const int h0 = kv * G;
    uint4* ring = reinterpret_cast<uint4*>(smem);
    float* sc = reinterpret_cast<float*>(smem + Geo::ring_bytes);                      // [KG][8][TT]
    __half* ph = reinterpret_cast<__half*>(smem + Geo::ring_bytes + Geo::sc_bytes);    // [8][PROW]
    __half* pl = ph + 8 * PROW;
    uint4* qf = reinterpret_cast<uint4*>(smem + Geo::ring_bytes + Geo::sc_bytes + Geo::p_bytes);  // [HD/16][32]
    const int kgi = KG == 1 ? 0 : warp / NT;  // this warp's k-range for scores

    pdl_launch_dependents();
    pdl_wait();

    // Copy plan: 1024 K units and 1024 V units per sub-tile, four of each per
    // thread.  K: chunk tid % CH of tokens tid / CH + i (256 / CH).  V: token
    // tid % TT of chunks tid / TT + i (256 / TT).
    const int k_tok = tid / CH, k_chk = tid % CH;
    const int v_tok = tid % TT, v_chk = tid / TT;
    const uint4* k_src0 = p.kc + (static_cast<size_t>(t0 + k_tok) * p.n_kv + kv) * CH + k_chk;
    const size_t k_step = static_cast<size_t>(256 / CH) * p.n_kv * CH;
    const uint4* v_src0 = p.vc + (static_cast<size_t>(kv) * CH + v_chk) * p.ctx_cap + t0 + v_tok;
    const size_t v_step = static_cast<size_t>(256 / TT) * p.ctx_cap;
    const int k_dst0 = k_tok * KROW + k_chk, v_dst0 = KU + v_chk * VROW + v_tok;
    auto issue = [&](int s) {
        const uint32_t base = smem_addr(ring + (s % kAttStages) * SU);
        const int nt = min(TT, T - s * TT);
        const size_t tok = static_cast<size_t>(s) * TT;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int t = k_tok + i * (256 / CH);
            const bool ok = t < nt;
            const uint4* src = ok ? k_src0 + tok * p.n_kv * CH + i * k_step : p.kc;
            cp_async16_zfill(base + (k_dst0 + i * (256 / CH) * KROW) * 16, src, ok);
        }
        const bool vok = v_tok < nt;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint4* src = vok ? v_src0 + tok + i * v_step : p.vc;
            cp_async16_zfill(base + (v_dst0 + i * (256 / TT) * VROW) * 16, src, vok);
        }
    };
    // All ring slots are filled up front; a slot is refilled once its
    // sub-tile has been consumed, so three sub-tiles are in flight.
#pragma unroll
    for (int s = 0; s < kAttStages; ++s) {
        if (s < nsub) issue(s);
        cp_commit();
    }

    // q as A fragments (rows = heads) in shared memory, split into fp16 high
    // and low parts: entry (k-step, lane) = {hi R0, hi R2, lo R0, lo R2}.
    for (int e = tid; e < (HD / 16) * 32; e += kAttThreads) {
        const int kj = e >> 5, g = (e & 31) >> 2, q4 = e & 3;
        float x[4] = {0.f, 0.f, 0.f, 0.f};
        if (g < G) {
#pragma unroll
            for (int half = 0; half < 2; ++half) {
                const size_t qi = static_cast<size_t>(h0 + g) * HD + kj * 16 + half * 8 + 2 * q4;
                float2 f;
                if (p.q_bits == 16)
                    f = __half22float2(*reinterpret_cast<const __half2*>(reinterpret_cast<const __half*>(p.q) + qi));
                else
                    f = *reinterpret_cast<const float2*>(reinterpret_cast<const float*>(p.q) + qi);
                x[2 * half] = f.x;
                x[2 * half + 1] = f.y;
            }
        }
        uint4 fr;
        split_pair(x[0], x[1], fr.x, fr.z);
        split_pair(x[2], x[3], fr.y, fr.w);
        qf[e] = fr;
    }
    const bool q_lo = p.q_bits != 16;  // fp16 q has no low part
    if (tid < G) {
        s_m[tid] = -INFINITY;
        s_l[tid] = 0.f;
    }

    float acc[PPW][2][4];
#pragma unroll
    for (int j = 0; j < PPW; ++j)
#pragma unroll
        for (int n = 0; n < 2; ++n)
#pragma unroll
            for (int i = 0; i < 4; ++i) acc[j][n][i] = 0.f;
    const int pw = warp % WN, pk = warp / WN;  // P.V: dimension pairs pw + WN j, k-steps of group pk

    for (int s = 0; s < nsub; ++s) {
        cp_wait<kAttStages - 1>();
        __syncthreads();  // sub-tile s landed for all threads
        const uint32_t base = smem_addr(ring + (s % kAttStages) * SU);
        const int nt = min(TT, T - s * TT);

        // (a) raw scores of this warp's token tiles (partial over k when KG > 1)
#pragma unroll
        for (int j = 0; j < TPW; ++j) {
            const int tile = KG == 1 ? warp + 8 * j : warp % NT;
            // Two accumulators (even / odd k-steps) halve the dependent MMA chain.
            float c[4] = {0.f, 0.f, 0.f, 0.f}, c2[4] = {0.f, 0.f, 0.f, 0.f};
            const int tok = tile * 8 + (lane & 7);
#pragma unroll
            for (int ks = 0; ks < KS; ks += 2) {
                const int chunk = (kgi * KS + ks) * 2 + (lane >> 3);
                uint32_t b[4];
                ldsm_x4(base + (tok * KROW + chunk) * 16, b);
                const uint4 qa = qf[(kgi * KS + ks) * 32 + lane], qb = qf[(kgi * KS + ks + 1) * 32 + lane];
                mma16816(c, qa.x, qa.y, b[0], b[1]);
                mma16816(c2, qb.x, qb.y, b[2], b[3]);
                if (q_lo) {
                    mma16816(c, qa.z, qa.w, b[0], b[1]);
                    mma16816(c2, qb.z, qb.w, b[2], b[3]);
                }
            }
            if (gid < G)
                *reinterpret_cast<float2*>(sc + (kgi * 8 + gid) * TT + tile * 8 + 2 * t4) =
                    make_float2(c[0] + c2[0], c[1] + c2[1]);
        }
        __syncthreads();

        // (b) online softmax, one warp per head; p split into fp16 hi / lo
        if (warp < G) {
            const int g = warp;
            float v[TT / 32];
            float mx = -INFINITY;
#pragma unroll
            for (int i = 0; i < TT / 32; ++i) {
                const int t = lane + 32 * i;
                float x = 0.f;
#pragma unroll
                for (int k = 0; k < KG; ++k) x += sc[(k * 8 + g) * TT + t];
                v[i] = t < nt ? x * p.scale_log2 : -INFINITY;
                mx = fmaxf(mx, v[i]);
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
            const float m_old = s_m[g];
            const float m_new = fmaxf(m_old, mx);
            float sum = 0.f;
#pragma unroll
            for (int i = 0; i < TT / 32; ++i) {
                const int t = lane + 32 * i;
                const float e = exp2f(v[i] - m_new);
                const __half eh = __float2half_rn(e);
                ph[g * PROW + t] = eh;
                pl[g * PROW + t] = __float2half_rn(e - __half2float(eh));
                sum += e;
            }
            sum = warp_sum(sum);
            if (lane == 0) {
                const float f = exp2f(m_old - m_new);
                s_m[g] = m_new;
                s_l[g] = s_l[g] * f + sum;
                s_f[g] = f;
            }
        }
        __syncthreads();

        // (c) P.V for this warp's dimension pairs and token k-steps
        const bool row = gid < G;
        const float f = row ? s_f[gid] : 0.f;
#pragma unroll
        for (int j = 0; j < PPW; ++j)
#pragma unroll
            for (int n = 0; n < 2; ++n) {
                acc[j][n][0] *= f;
                acc[j][n][1] *= f;
            }
#pragma unroll
        for (int k = 0; k < PKS; ++k) {
            const int kt = (pk * PKS + k) * 16;  // first token of the k-step
            uint32_t ah0 = 0, ah2 = 0, al0 = 0, al2 = 0;
            if (row) {
                ah0 = *reinterpret_cast<const uint32_t*>(ph + gid * PROW + kt + 2 * t4);
                ah2 = *reinterpret_cast<const uint32_t*>(ph + gid * PROW + kt + 8 + 2 * t4);
                al0 = *reinterpret_cast<const uint32_t*>(pl + gid * PROW + kt + 2 * t4);
                al2 = *reinterpret_cast<const uint32_t*>(pl + gid * PROW + kt + 8 + 2 * t4);
            }
            const int tok = kt + (lane & 7) + ((lane >> 3) & 1) * 8;
#pragma unroll
            for (int j = 0; j < PPW; ++j) {
                const int chunk = (pw + WN * j) * 2 + (lane >> 4);
                uint32_t b[4];
                ldsm_x4_t(base + (KU + chunk * VROW + tok) * 16, b);
                mma16816(acc[j][0], ah0, ah2, b[0], b[1]);
                mma16816(acc[j][0], al0, al2, b[0], b[1]);
                mma16816(acc[j][1], ah0, ah2, b[2], b[3]);
                mma16816(acc[j][1], al0, al2, b[2], b[3]);
            }
        }
        __syncthreads();  // slot of sub-tile s consumed by all warps
        if (s + kAttStages < nsub) issue(s + kAttStages);
        cp_commit();
    }
    cp_wait<0>();
    __syncthreads();

    // Partial of this split: acc rows gid < G, dims (2 pair + n) 8 + 2 t4.
    auto rec = [&](int g) { return p.ws + (static_cast<size_t>(h0 + g) * p.splits + split) * p.pitch; };
    if constexpr (WK == 1) {
        if (gid < G)
#pragma unroll
            for (int j = 0; j < PPW; ++j)
#pragma unroll
                for (int n = 0; n < 2; ++n) {
                    const int d = ((pw + WN * j) * 2 + n) * 8 + 2 * t4;
                    *reinterpret_cast<float2*>(rec(gid) + d) = make_float2(acc[j][n][0], acc[j][n][1]);
                }
    } else {
        float* red = reinterpret_cast<float*>(smem);  // [WK][G][HD]
        if (gid < G)
#pragma unroll
            for (int j = 0; j < PPW; ++j)
#pragma unroll
                for (int n = 0; n < 2; ++n) {
                    const int d = ((pw + WN * j) * 2 + n) * 8 + 2 * t4;
                    *reinterpret_cast<float2*>(red + (pk * G + gid) * HD + d) =
                        make_float2(acc[j][n][0], acc[j][n][1]);
                }
        __syncthreads();
        for (int i = tid; i < G * HD; i += kAttThreads) {
            const int g = i / HD, d = i - g * HD;
            float x = 0.f;
#pragma unroll
            for (int k = 0; k < WK; ++k) x += red[(k * G + g) * HD + d];
            rec(g)[d] = x;
        }
    }
    if (tid < G) {
        rec(tid)[HD] = s_m[tid];
        rec(tid)[HD + 1] = s_l[tid];
    }
    merge_splits<G>(p, smem, kv, p.splits);
}

// ---- token-slice variant with swapped operands (head_dim 64 / 128) ----------
//
// Four warps per CTA; each owns 16-token slices of every sub-tile and runs the
// whole step on them with the tokens, not the (few) query heads, as the M
// dimension of mma.sync m16n8k16, so no MMA rows are padding:
//   scores  S^T[16 tok][8 heads] = K[16 tok][hd] . q^T[hd][8 heads]     A = K  (ldmatrix)
//   P.V     O^T[hd][8 heads]    += V^T[hd][16 tok] . P^T[16 tok][8 heads] A = V^T (ldmatrix.trans)
// Heads G..7 of the 8 columns carry zero q and zero p.  Each warp keeps its own
// online softmax (running max and sum per head, in registers); P^T goes from
// the score accumulators to the B operand of P.V through movmatrix (a
// register transpose), so p never touches shared memory and the warps meet
// only at the two ring barriers per sub-tile.  q and p are fp32 values split
// into fp16 high and low parts, both multiplied (about 22 significant bits).
// The four warp states are merged through shared memory at the end.
//
// Two shapes.  Clustered: ST = 3 ring stages, CL = 8 consecutive splits of a
// KV head per cluster merging over DSMEM, two CTAs per SM.  Per-SM: ST = 6
// stages (192 KB of the cache in flight per SM), CL = 1, one CTA per SM with
// a long token range, the splits of a head merged by the last to finish.
constexpr int kFaThreads = 128;
constexpr int kFaCluster = 8;  // CTAs per cluster of the clustered shape
constexpr int kFaDeepStages = 6;

__device__ __forceinline__ void mma16816_full(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t movmatrix_t(uint32_t x) {
    uint32_t y;
    asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
    return y;
}

// The body of the token-slice kernel for CTA (split, kv), run by the first
// NWG * kFaThreads threads of the CTA with `smem` as its dynamic shared
// memory; `wait()` stands for the wait on the previous kernel (called by all
// of those threads).  SYNC 0: the threads are the whole CTA; otherwise their
// CTA-wide barriers are named barrier SYNC.
template <int G, int HD, int ST, int CL, int NWG, int SYNC, typename Wait>
__device__ __forceinline__ void attention_fa_body(const AttnParams& p, uint8_t* smem, const int split, const int kv,
                                                  Wait wait) {
    using Geo = MmaGeo<HD>;
    constexpr int CH = Geo::CH, TT = Geo::TT, KROW = Geo::KROW, VROW = Geo::VROW, KU = Geo::KU, SU = Geo::SU;
    constexpr int NT = kFaThreads * NWG;   // threads: NWG warp groups of kFaThreads
    constexpr int NW = NT / 32;            // warps
    constexpr int SPW = TT / (16 * (kFaThreads / 32));  // 16-token slices per warp per sub-tile
    constexpr int KS = HD / 16;            // score k-steps
    constexpr int MT = HD / 16;            // P.V m-tiles of 16 dimensions
    constexpr int CPT = 1024 / kFaThreads; // K (and V) copies per thread per sub-tile
    static_assert(SPW >= 1 && TT % (16 * (kFaThreads / 32)) == 0 && KS % 2 == 0, "geometry");
    static_assert(ST % NWG == 0 && (NWG == 1 || CL == 1), "warp groups take every NWG-th stage; no clusters");
    static_assert(kFaThreads % CH == 0 && kFaThreads % TT == 0, "copy plan");
    static_assert(SYNC == 0 || CL == 1, "clusters synchronise whole CTAs");
    __shared__ float s_wm[NW][8], s_wl[NW][8];
    auto cta_sync = [] { part_sync<SYNC, NT>(); };
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int gid = lane >> 2, t4 = lane & 3;
    // Warp group wg streams and processes the sub-tiles s = wg, wg + NWG, ...
    // through the ring stages s % ST, with its own copy groups and barrier.
    const int wg = tid / kFaThreads, ltid = tid % kFaThreads, lwarp = warp % (kFaThreads / 32);
    auto group_sync = [&]() {
        if constexpr (NWG == 1)
            cta_sync();
        else
            asm volatile("bar.sync %0, %1;" ::"r"(1 + wg), "n"(kFaThreads) : "memory");
    };
    const int t0 = split * p.tpc;
    const int T = min(p.tpc, p.ctx - t0);
    const int nsub = (T + TT - 1) / TT;
    const int h0 = kv * G;
    uint4* ring = reinterpret_cast<uint4*>(smem);
    constexpr size_t kRingBytes = static_cast<size_t>(ST) * SU * 16;
    uint4* qf = reinterpret_cast<uint4*>(smem + kRingBytes);  // [KS][32]

    pdl_launch_dependents();

    // Copy plan (per warp group): K chunk ltid % CH of tokens ltid / CH + i
    // (128 / CH); V token ltid % TT of chunks ltid / TT + i (128 / TT); i < CPT.
    const int k_tok = ltid / CH, k_chk = ltid % CH;
    const int v_tok = ltid % TT, v_chk = ltid / TT;
    const uint4* k_src0 = p.kc + (static_cast<size_t>(t0 + k_tok) * p.n_kv + kv) * CH + k_chk;
    const size_t k_step = static_cast<size_t>(kFaThreads / CH) * p.n_kv * CH;
    const uint4* v_src0 = p.vc + (static_cast<size_t>(kv) * CH + v_chk) * p.ctx_cap + t0 + v_tok;
    const size_t v_step = static_cast<size_t>(kFaThreads / TT) * p.ctx_cap;
    const int k_dst0 = k_tok * KROW + k_chk, v_dst0 = KU + v_chk * VROW + v_tok;
    auto issue = [&](int s) {
        const uint32_t base = smem_addr(ring + (s % ST) * SU);
        const int nt = min(TT, T - s * TT);
        const size_t tok = static_cast<size_t>(s) * TT;
#pragma unroll
        for (int i = 0; i < CPT; ++i) {
            const int t = k_tok + i * (kFaThreads / CH);
            const bool ok = t < nt;
            const uint4* src = ok ? k_src0 + tok * p.n_kv * CH + i * k_step : p.kc;
            cp_async16_zfill(base + (k_dst0 + i * (kFaThreads / CH) * KROW) * 16, src, ok);
        }
        const bool vok = v_tok < nt;
#pragma unroll
        for (int i = 0; i < CPT; ++i) {
            const uint4* src = vok ? v_src0 + tok + i * v_step : p.vc;
            cp_async16_zfill(base + (v_dst0 + i * (kFaThreads / TT) * VROW) * 16, src, vok);
        }
    };
    // Sub-tiles whose tokens all lie below p.stable (cache rows no kernel still
    // in flight writes) are requested before the wait on the previous kernel;
    // the rest, and q, after it.  Commit groups stay in sub-tile order.
    int s_pre = wg;
    for (int n = 0; s_pre < ST && s_pre < nsub && t0 + min(T, (s_pre + 1) * TT) <= p.stable &&
                    (p.pre_max == 0 || n < p.pre_max);
         ++n) {
        issue(s_pre);
        cp_commit();
        s_pre += NWG;
    }
    wait();

    // q^T as B fragments in shared memory: entry (k-step, lane) =
    // {hi b0, hi b1, lo b0, lo b1}, b0 = q[gid][16 k + 2 t4 ..], b1 = +8.
    // q is loaded before the cache copies are issued, so its few loads are
    // not queued behind this SM's ring of cache requests.
    constexpr int QE = (KS * 32 + NT - 1) / NT;  // entries per thread
    float qx[QE][4];
#pragma unroll
    for (int j = 0; j < QE; ++j) {
        const int e = tid + j * NT;
        const int kj = e >> 5, g = (e & 31) >> 2, q4 = e & 3;
#pragma unroll
        for (int i = 0; i < 4; ++i) qx[j][i] = 0.f;
        if (e < KS * 32 && g < G) {
#pragma unroll
            for (int half = 0; half < 2; ++half) {
                const size_t qi = static_cast<size_t>(h0 + g) * HD + kj * 16 + half * 8 + 2 * q4;
                // L2 loads: q may come from other CTAs of a persistent kernel
                float2 f;
                if (p.q_bits == 16) {
                    const unsigned u = __ldcg(reinterpret_cast<const unsigned*>(reinterpret_cast<const __half*>(p.q) + qi));
                    f = __half22float2(*reinterpret_cast<const __half2*>(&u));
                } else {
                    f = __ldcg(reinterpret_cast<const float2*>(reinterpret_cast<const float*>(p.q) + qi));
                }
                qx[j][2 * half] = f.x;
                qx[j][2 * half + 1] = f.y;
            }
        }
    }
    for (int s = s_pre; s < ST; s += NWG) {
        if (s < nsub) issue(s);
        cp_commit();
    }
#pragma unroll
    for (int j = 0; j < QE; ++j) {
        const int e = tid + j * NT;
        if (e < KS * 32) {
            uint4 fr;
            split_pair(qx[j][0], qx[j][1], fr.x, fr.z);
            split_pair(qx[j][2], qx[j][3], fr.y, fr.w);
            qf[e] = fr;
        }
    }
    const bool q_lo = p.q_bits != 16;  // fp16 q has no low part
    // This lane's two heads (columns 2 t4, 2 t4 + 1) and whether they exist.
    const bool hv0 = 2 * t4 < G, hv1 = 2 * t4 + 1 < G;

    float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};  // l: this lane's share
    float acc[MT][4];  // O^T: (dim 16 mt + gid [+8], head 2 t4 [+1])
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[mt][i] = 0.f;

    if constexpr (NWG > 1) cta_sync();  // q fragments of all groups
    for (int s = wg; s < nsub; s += NWG) {
        cp_wait<ST / NWG - 1>();
        group_sync();  // sub-tile s landed for the group's threads (and q fragments, first time)
        const uint32_t base = smem_addr(ring + (s % ST) * SU);
        const int nt = min(TT, T - s * TT);
#pragma unroll
        for (int sl = 0; sl < SPW; ++sl) {
            const int ts0 = (lwarp * SPW + sl) * 16;  // first token of the slice

            // scores S^T; two accumulators (even / odd k-steps) halve the MMA chain
            float c[4] = {0.f, 0.f, 0.f, 0.f}, c2[4] = {0.f, 0.f, 0.f, 0.f};
            const int tok = ts0 + (lane & 7) + ((lane >> 3) & 1) * 8;
#pragma unroll
            for (int kj = 0; kj < KS; ++kj) {
                uint32_t a[4];
                ldsm_x4(base + (tok * KROW + 2 * kj + (lane >> 4)) * 16, a);
                const uint4 qb = qf[kj * 32 + lane];
                if (kj & 1) {
                    mma16816_full(c2, a, qb.x, qb.y);
                    if (q_lo) mma16816_full(c2, a, qb.z, qb.w);
                } else {
                    mma16816_full(c, a, qb.x, qb.y);
                    if (q_lo) mma16816_full(c, a, qb.z, qb.w);
                }
            }
            // sv[i]: i = 0 (token gid, head 2t4), 1 (gid, 2t4+1), 2 (gid+8, 2t4), 3 (gid+8, 2t4+1)
            float sv[4];
            const bool tv0 = ts0 + gid < nt, tv1 = ts0 + gid + 8 < nt;
            sv[0] = tv0 && hv0 ? (c[0] + c2[0]) * p.scale_log2 : -INFINITY;
            sv[1] = tv0 && hv1 ? (c[1] + c2[1]) * p.scale_log2 : -INFINITY;
            sv[2] = tv1 && hv0 ? (c[2] + c2[2]) * p.scale_log2 : -INFINITY;
            sv[3] = tv1 && hv1 ? (c[3] + c2[3]) * p.scale_log2 : -INFINITY;
            // online softmax per head: a head's 16 tokens sit in the 8 lanes of one t4
            float mx0 = fmaxf(sv[0], sv[2]), mx1 = fmaxf(sv[1], sv[3]);
#pragma unroll
            for (int o = 4; o < 32; o <<= 1) {
                mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, o));
                mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, o));
            }
            const float mn0 = fmaxf(m_run[0], mx0), mn1 = fmaxf(m_run[1], mx1);
            const float f0 = mn0 == -INFINITY ? 1.f : exp2f(m_run[0] - mn0);
            const float f1 = mn1 == -INFINITY ? 1.f : exp2f(m_run[1] - mn1);
            float pv[4];
            pv[0] = sv[0] == -INFINITY ? 0.f : exp2f(sv[0] - mn0);
            pv[1] = sv[1] == -INFINITY ? 0.f : exp2f(sv[1] - mn1);
            pv[2] = sv[2] == -INFINITY ? 0.f : exp2f(sv[2] - mn0);
            pv[3] = sv[3] == -INFINITY ? 0.f : exp2f(sv[3] - mn1);
            l_run[0] = fmaf(l_run[0], f0, pv[0] + pv[2]);
            l_run[1] = fmaf(l_run[1], f1, pv[1] + pv[3]);
            m_run[0] = mn0;
            m_run[1] = mn1;
#pragma unroll
            for (int mt = 0; mt < MT; ++mt) {
                acc[mt][0] *= f0;
                acc[mt][1] *= f1;
                acc[mt][2] *= f0;
                acc[mt][3] *= f1;
            }
            // P^T as B fragments (k = tokens, n = heads): transpose the 8x8
            // blocks [token][head] of the accumulator layout in registers.
            uint32_t x0h, x0l, x1h, x1l;
            split_pair(pv[0], pv[1], x0h, x0l);  // tokens 0..7 of the slice
            split_pair(pv[2], pv[3], x1h, x1l);  // tokens 8..15
            const uint32_t bh0 = movmatrix_t(x0h), bh1 = movmatrix_t(x1h);
            const uint32_t bl0 = movmatrix_t(x0l), bl1 = movmatrix_t(x1l);

            // P.V: A = V^T m-tile (chunks 2 mt, 2 mt + 1) x the slice's 16 tokens
            const int tokv = ts0 + (lane & 7) + ((lane >> 4) & 1) * 8;
            const int chv = (lane >> 3) & 1;
#pragma unroll
            for (int mt = 0; mt < MT; ++mt) {
                uint32_t a[4];
                ldsm_x4_t(base + (KU + (2 * mt + chv) * VROW + tokv) * 16, a);
                mma16816_full(acc[mt], a, bh0, bh1);
                mma16816_full(acc[mt], a, bl0, bl1);
            }
        }
        group_sync();  // slot of sub-tile s consumed by the group's warps
        if (s + ST < nsub) issue(s + ST);
        cp_commit();
    }
    cp_wait<0>();

    // Merge the warp states of this CTA (the ring is free now).
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) {
        l_run[0] += __shfl_xor_sync(0xffffffffu, l_run[0], o);
        l_run[1] += __shfl_xor_sync(0xffffffffu, l_run[1], o);
    }
    if (gid == 0) {
        s_wm[warp][2 * t4] = m_run[0];
        s_wm[warp][2 * t4 + 1] = m_run[1];
        s_wl[warp][2 * t4] = l_run[0];
        s_wl[warp][2 * t4 + 1] = l_run[1];
    }
    cta_sync();
    float* red = reinterpret_cast<float*>(smem);  // [NW][G][HD]
    {
        float M0 = -INFINITY, M1 = -INFINITY;
#pragma unroll
        for (int w = 0; w < NW; ++w) {
            M0 = fmaxf(M0, s_wm[w][2 * t4]);
            M1 = fmaxf(M1, s_wm[w][2 * t4 + 1]);
        }
        const float sw0 = m_run[0] == -INFINITY ? 0.f : exp2f(m_run[0] - M0);
        const float sw1 = m_run[1] == -INFINITY ? 0.f : exp2f(m_run[1] - M1);
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
            const int d = 16 * mt + gid;
            if (hv0) {
                red[(warp * G + 2 * t4) * HD + d] = acc[mt][0] * sw0;
                red[(warp * G + 2 * t4) * HD + d + 8] = acc[mt][2] * sw0;
            }
            if (hv1) {
                red[(warp * G + 2 * t4 + 1) * HD + d] = acc[mt][1] * sw1;
                red[(warp * G + 2 * t4 + 1) * HD + d + 8] = acc[mt][3] * sw1;
            }
        }
    }
    cta_sync();
    // This CTA's record in shared memory, [G][HD + 4]: acc[HD], m, l.
    constexpr int RP = HD + 4;
    float* crec = red + NW * G * HD;
    for (int i = tid; i < G * HD; i += NT) {
        const int g = i / HD, d = i - g * HD;
        float x = 0.f;
#pragma unroll
        for (int w = 0; w < NW; ++w) x += red[(w * G + g) * HD + d];
        crec[g * RP + d] = x;
    }
    if (tid < G) {
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < NW; ++w) M = fmaxf(M, s_wm[w][tid]);
        float L = 0.f;
#pragma unroll
        for (int w = 0; w < NW; ++w) {
            const float mw = s_wm[w][tid];
            L += mw == -INFINITY ? 0.f : s_wl[w][tid] * exp2f(mw - M);
        }
        crec[tid * RP + HD] = M;
        crec[tid * RP + HD + 1] = L;
    }
    if constexpr (CL == 1) {
        // No cluster: the record goes straight to the workspace (or, with a
        // single split, the normalised output to `out`).
        cta_sync();
        if (p.splits == 1) {
            for (int i = tid; i < G * HD; i += NT) {
                const int g = i / HD, d = i - g * HD;
                p.out[static_cast<size_t>(h0) * HD + i] = crec[g * RP + d] / crec[g * RP + HD + 1];
            }
            return;
        }
        for (int i = tid; i < G * RP / 4; i += NT) {
            const int g = (4 * i) / RP, d = 4 * i - g * RP;
            *reinterpret_cast<float4*>(p.ws + (static_cast<size_t>(h0 + g) * p.splits + split) * p.pitch + d) =
                *reinterpret_cast<const float4*>(crec + g * RP + d);
        }
        if constexpr (G * HD / 4 <= NT)
            merge_splits_direct<G, HD, NT, SYNC>(p, kv, p.splits);
        else
            merge_splits<G, NT>(p, smem, kv, p.splits);
        return;
    }

    // ---- cluster of CL consecutive splits: rank 0 merges the records
    // of its peers through distributed shared memory.  Barrier 1 publishes the
    // records; barrier 2 keeps the peers resident until rank 0 has read them.
    cta_sync();
    cluster_arrive_release();
    cluster_wait_acquire();
    uint32_t rank;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(rank));
    if (rank != 0) {
        cluster_arrive_release();
        cluster_wait_acquire();
        return;
    }
    __shared__ float s_cM[8], s_cL[8];
    const uint32_t crec_addr = smem_addr(crec);
    // Four dimensions per thread: the (m, l) and values of every rank are
    // loaded in one round, then summed in rank order.
    const int nc = p.splits / CL, cidx = split / CL;
    for (int qd = tid; qd < G * HD / 4; qd += kFaThreads) {
        const int g = (qd * 4) / HD, d = qd * 4 - g * HD;
        float4 v[CL];
        float2 ml[CL];
#pragma unroll
        for (int r = 0; r < CL; ++r) {
            const uint32_t ra = map_cluster_addr(crec_addr + (g * RP + d) * 4, r);
            const uint32_t rs = map_cluster_addr(crec_addr + (g * RP + HD) * 4, r);
            asm volatile("ld.shared::cluster.v4.f32 {%0,%1,%2,%3}, [%4];"
                         : "=f"(v[r].x), "=f"(v[r].y), "=f"(v[r].z), "=f"(v[r].w)
                         : "r"(ra)
                         : "memory");
            asm volatile("ld.shared::cluster.v2.f32 {%0,%1}, [%2];" : "=f"(ml[r].x), "=f"(ml[r].y) : "r"(rs) : "memory");
        }
        float M = -INFINITY;
#pragma unroll
        for (int r = 0; r < CL; ++r) M = fmaxf(M, ml[r].x);
        float L = 0.f;
        float4 acc4 = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int r = 0; r < CL; ++r) {
            const float w = ml[r].x == -INFINITY ? 0.f : exp2f(ml[r].x - M);
            L = fmaf(w, ml[r].y, L);
            acc4.x = fmaf(w, v[r].x, acc4.x);
            acc4.y = fmaf(w, v[r].y, acc4.y);
            acc4.z = fmaf(w, v[r].z, acc4.z);
            acc4.w = fmaf(w, v[r].w, acc4.w);
        }
        if (nc == 1) {
            const float inv = 1.f / L;
            *reinterpret_cast<float4*>(p.out + static_cast<size_t>(h0) * HD + qd * 4) =
                make_float4(acc4.x * inv, acc4.y * inv, acc4.z * inv, acc4.w * inv);
        } else {
            *reinterpret_cast<float4*>(p.ws + (static_cast<size_t>(h0 + g) * nc + cidx) * p.pitch + d) = acc4;
            if (d == 0) {
                s_cM[g] = M;
                s_cL[g] = L;
            }
        }
    }
    cluster_arrive_release();  // peers' records have been read
    if (nc > 1) {
        cta_sync();
        if (tid < G) {
            float* r = p.ws + (static_cast<size_t>(h0 + tid) * nc + cidx) * p.pitch + HD;
            r[0] = s_cM[tid];
            r[1] = s_cL[tid];
        }
        if constexpr (G * HD / 4 <= kFaThreads)
            merge_splits_direct<G, HD, kFaThreads>(p, kv, nc);
        else
            merge_splits<G, kFaThreads>(p, smem, kv, nc);
    }
    cluster_wait_acquire();
}

template <int G, int HD, int ST, int CL, int NWG = 1>
__global__ void __launch_bounds__(kFaThreads * NWG, ST > 3 ? 1 : 2) attention_fa_kernel(const AttnParams p) {
    extern __shared__ __align__(16) uint8_t smem[];
    attention_fa_body<G, HD, ST, CL, NWG, 0>(p, smem, blockIdx.x, blockIdx.y, [] { pdl_wait(); });
}

}  // namespace

}  // namespace vkc
