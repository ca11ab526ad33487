// GEMV family for sm_100a: GEMV, RmsNorm-GEMV, RmsNorm-GEMV-Rope and
// RmsNorm-SwiGLU over fp32 / fp16 / int8 / int4 weights stored in vk-compute's
// 16-byte chunk layout (src/data.c:198-222).
//
// Weight layout (the reference's, unchanged): chunk row r holds k in
// [r*KPC, (r+1)*KPC) (KPC = 128/bits) of every output column j as one 16-byte
// chunk at byte (r*N + j)*16, so a chunk row is a contiguous N*16-byte stream.
// Quantised weights carry fp32 scale s and zero z per (k, 256-output block b),
// block-major at b*K + k (src/data.c:122-124), dequantised as q*s - z
// (shader/GEMV-INT8.comp:56-59).
//
// Decomposition.  A CTA of 256 threads owns C consecutive outputs
// (C in {256, 128, 64, 32}, inside one scale block) and a range of chunk rows;
// its 256/C thread groups take interleaved rows.  S CTAs of a thread-block
// cluster (S <= 8) split K, and their partial sums meet in distributed shared
// memory, where each rank runs the epilogue for C/S of the outputs.  C and S
// are chosen so that every CTA has the same work and all CTAs are resident at
// once (one wave): on a saturated memory system every CTA then streams at the
// same rate and they finish together.
//
// Streaming.  Every thread keeps its own ring of D 16-byte cp.async copies in
// shared memory (one commit group per row), so D rows per thread are in
// flight without registers and without any barrier in the steady state; a
// warp reads 512 contiguous bytes per row.  The few activation loads are
// issued before the first weight copy, so they are not queued behind the
// weight stream.
//
// Arithmetic.  The per-(k, b) scale is folded into the staged activation,
// x'_k = x_k * gamma_k * s_kb, and the zero point into a per-block constant
// c_b = sum_k x_k gamma_k z_kb, so y_j = inv_rms * (sum_k x'_k q_kj - c_b):
// one conversion and one fused multiply-add per weight.  Codes become floats
// exactly by OR-ing them into the mantissa of 2^23 and subtracting 2^23 (int4
// nibbles keep their bit position; x' carries the matching power of two);
// pairs of weights use the packed f32x2 add and FMA.  inv_rms and c_b are
// scalars applied in the epilogue, after the cluster reduction.
#include "vkc_common.cuh"
#include "vk_compute_b200.h"
#include "attention_kernels.cuh"

#include <cuda_fp16.h>

#include <algorithm>
#include <mutex>
#include <vector>

namespace vkc {

// Per-device status word (one instance per device context), bits kStatus*.
__device__ uint32_t g_status = 0;

namespace {

constexpr int kThreads = 256;
constexpr int kGroup = 256;     // outputs per scale block
constexpr int kCtasPerSm = 4;   // occupancy target (64 registers per thread)
// cp.async ring per CTA (all streams): 32 KB, or 48 KB when the grid still
// fits on the GPU in one wave with the deeper ring.
template <bool DEEP>
constexpr int ring_bytes() { return DEEP ? 49152 : 32768; }

enum Mode : int {
    kGemv = 0,       // shader/GEMV-*.comp
    kRms = 1,        // shader/RmsNorm-GEMV-*.comp
    kRopeRef = 2,    // shader/RmsNorm-GEMV-Rope-*.comp epilogue as written
    kRopePairs = 3,  // rotary embedding on adjacent pairs per head
    kSwiglu = 4,     // shader/RmsNorm-swiglu-ffn-*.comp
};

struct GemvParams {
    const uint8_t* w[2];
    const float* s[2];
    const float* z[2];
    const float* x;
    const float* gamma;
    const float* theta;
    float* y;
    int N, K, R;
    int cols;      // C: outputs per CTA
    int rows_cta;  // chunk rows per CTA (the last rank of a cluster may have fewer)
    int rbuf_floats;  // rank-0 receive buffer, S * (NS*C + 4) floats
    float eps;
    float inv_dim;  // 1 / RMS divisor
    int pos;
    int head_dim;
    int rot_rows;
    const float* residual;  // optional: y[j] += residual[j] (plain GEMV)
    // Optional KV-cache append (rotary-pairs mode): the outputs after the
    // first q_rows are K and V heads, [K heads | V heads] (kv_interleave 0) or
    // [K0 V0 | K1 V1 | ...] (kv_interleave 1); both are also stored as fp16 at
    // token `pos` into K[t][h][d] and V[h][d/8][t][d%8] caches of `ctx_cap`
    // tokens.
    uint16_t* kcache;
    uint16_t* vcache;
    int q_rows, kv_rows, ctx_cap, kv_interleave;
    // Peer output (plain GEMV, K-split shard): output j goes, as the 8-byte
    // word (flag << 32 | float bits), to element prank*N + j of every rank's
    // [pworld][N] word buffer (peer_slots: device array of pworld pointers),
    // flag = the flag this rank's own copy of the element held + 1.
    unsigned long long* const* peer_slots;
    // Peer input: x = x (the base) + the pworld slots of xslots ([pworld][K]
    // words, summed in rank order); each thread waits until a peer's element
    // carries the flag its own slot's element has (written by this rank's
    // producer, the previous kernel).  The first column block stores x in xsave.
    const unsigned long long* xslots;
    float* xsave;
    int prank, pworld;
    // Gathered output (row-sharded GEMV): output j is stored at gather_off + j
    // of every rank's full output vector (gather_dst: device array of pworld
    // pointers, the peers' through NVLink); the arrival is signalled by the
    // next kernel in the stream (vkc_gather_wait).
    float* const* gather_dst;
    int gather_off;
};

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Power-of-two pre-scale of an int4 position inside a 32-bit word.  Nibbles
// 0-4 are decoded in place (bit offsets 0..16); nibbles 5-7 after a 12-bit
// shift (offsets 8, 12, 16).
__device__ __forceinline__ float int4_prescale(int t) {
    const int i = t & 7;
    const int e = i < 5 ? 4 * i : 4 * (i - 3);
    return __int_as_float((127 - e) << 23);
}

constexpr uint32_t kMagic = 0x4B000000u;  // 2^23

// Two exact codes as an f32x2 pair (2^23 + code, both halves built in one asm
// block so the pair lands in a register pair without moves).  int4: each half
// is (word & mask) | 2^23; int8: each half is byte `sel` of the word under 2^23.
__device__ __forceinline__ uint64_t nib_pair(uint32_t a, uint32_t ma, uint32_t b, uint32_t mb) {
    uint64_t r;
    asm("{\n\t.reg .b32 lo, hi;\n\t"
        "lop3.b32 lo, %1, %2, %5, 0xEA;\n\t"
        "lop3.b32 hi, %3, %4, %5, 0xEA;\n\t"
        "mov.b64 %0, {lo, hi};\n\t}"
        : "=l"(r)
        : "r"(a), "r"(ma), "r"(b), "r"(mb), "r"(kMagic));
    return r;
}
template <uint32_t SEL_LO, uint32_t SEL_HI>
__device__ __forceinline__ uint64_t byte_pair(uint32_t w) {
    uint64_t r;
    asm("{\n\t.reg .b32 lo, hi;\n\t"
        "prmt.b32 lo, %1, %2, %3;\n\t"
        "prmt.b32 hi, %1, %2, %4;\n\t"
        "mov.b64 %0, {lo, hi};\n\t}"
        : "=l"(r)
        : "r"(w), "r"(kMagic), "n"(SEL_LO), "n"(SEL_HI));
    return r;
}

// One chunk of KPC weights of one column against the staged activations xs
// (16-byte aligned shared memory); accumulates into four pair accumulators.
template <int BITS>
__device__ __forceinline__ void chunk_fma(const uint4 c, const float* __restrict__ xs, uint64_t (&a)[4]) {
    const float4* x4 = reinterpret_cast<const float4*>(xs);
    if constexpr (BITS == 32) {
        const float4 v = x4[0];
        a[0] = f2_fma(f2_pack(v.x, v.y), f2_pack(__uint_as_float(c.x), __uint_as_float(c.y)), a[0]);
        a[1] = f2_fma(f2_pack(v.z, v.w), f2_pack(__uint_as_float(c.z), __uint_as_float(c.w)), a[1]);
    } else if constexpr (BITS == 16) {
        const uint32_t wd[4] = {c.x, c.y, c.z, c.w};
#pragma unroll
        for (int q = 0; q < 2; ++q) {
            const float4 v = x4[q];
            const float2 w0 = __half22float2(*reinterpret_cast<const __half2*>(&wd[2 * q]));
            const float2 w1 = __half22float2(*reinterpret_cast<const __half2*>(&wd[2 * q + 1]));
            a[2 * q] = f2_fma(f2_pack(v.x, v.y), f2_pack(w0.x, w0.y), a[2 * q]);
            a[2 * q + 1] = f2_fma(f2_pack(v.z, v.w), f2_pack(w1.x, w1.y), a[2 * q + 1]);
        }
    } else if constexpr (BITS == 8) {
        const uint32_t wd[4] = {c.x, c.y, c.z, c.w};
        const uint64_t neg = f2_pack(-8388608.0f, -8388608.0f);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const float4 v = x4[q];
            const uint32_t w = wd[q];
            a[q] = f2_fma(f2_pack(v.x, v.y), f2_add(byte_pair<0x7540, 0x7541>(w), neg), a[q]);
            a[q] = f2_fma(f2_pack(v.z, v.w), f2_add(byte_pair<0x7542, 0x7543>(w), neg), a[q]);
        }
    } else {  // BITS == 4
        const uint32_t wd[4] = {c.x, c.y, c.z, c.w};
        const uint64_t neg = f2_pack(-8388608.0f, -8388608.0f);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const float4 v0 = x4[2 * q];
            const float4 v1 = x4[2 * q + 1];
            const uint32_t w = wd[q];
            const uint32_t h = w >> 12;
            a[0] = f2_fma(f2_pack(v0.x, v0.y), f2_add(nib_pair(w, 0xFu, w, 0xF0u), neg), a[0]);
            a[1] = f2_fma(f2_pack(v0.z, v0.w), f2_add(nib_pair(w, 0xF00u, w, 0xF000u), neg), a[1]);
            a[2] = f2_fma(f2_pack(v1.x, v1.y), f2_add(nib_pair(w, 0xF0000u, h, 0xF00u), neg), a[2]);
            a[3] = f2_fma(f2_pack(v1.z, v1.w), f2_add(nib_pair(h, 0xF000u, h, 0xF0000u), neg), a[3]);
        }
    }
}

// Epilogue for one output column: RMS scale, zero-point constant and the
// operator's activation.  Called by every lane of a warp together (the RoPE
// partner is the neighbouring lane); `active` lanes store.
template <int MODE, int NS, bool kQuant, bool kNorm>
__device__ __forceinline__ void finalize(const GemvParams& p, int j, bool active, const float (&acc)[NS],
                                         const float (&tot)[3]) {
    float v[NS];
    const float inv = kNorm ? 1.0f / sqrtf(tot[0] * p.inv_dim + p.eps) : 1.0f;
#pragma unroll
    for (int st = 0; st < NS; ++st) v[st] = ((kQuant ? acc[st] - tot[1 + st] : acc[st])) * inv;
    float out = v[0];
    if constexpr (MODE == kRopeRef) {
        // shader/RmsNorm-GEMV-Rope-FP16.comp:76-89, reproduced as written.
        const int c = j % kGroup;
        if (active && c < 64) {
            float sa, ca;
            sincosf(static_cast<float>(p.pos) * p.theta[c / 2], &sa, &ca);
            out = (c & 1) == 0 ? out * ca - p.theta[c + 1] * sa : p.theta[c - 1] * sa + out * ca;
        }
    } else if constexpr (MODE == kRopePairs) {
        const float partner = __shfl_xor_sync(0xffffffffu, out, 1);
        // Q and K rows rotate, V rows do not
        const bool rot = p.kv_interleave ? (j < p.q_rows || (j - p.q_rows) % (2 * p.head_dim) < p.head_dim)
                                         : j < p.rot_rows;
        if (active && rot) {
            float sa, ca;
            sincosf(static_cast<float>(p.pos) * p.theta[(j % p.head_dim) >> 1], &sa, &ca);
            out = (j & 1) == 0 ? out * ca - partner * sa : partner * sa + out * ca;
        }
    } else if constexpr (MODE == kSwiglu) {
        // shader/RmsNorm-swiglu-ffn-FP16.comp:86-87
        out = out / (1.0f + exp2f(-out * 1.44269504f)) * v[1];
    }
    if constexpr (MODE == kGemv) {
        if (p.residual && active && j < p.N) out += __ldcg(p.residual + j);
    }
    if (active && j < p.N) {
        if (MODE == kGemv && p.peer_slots) {
            const size_t e = static_cast<size_t>(p.prank) * p.N + j;
            const unsigned flag = static_cast<unsigned>(__ldcg(p.peer_slots[p.prank] + e) >> 32) + 1u;
            const unsigned long long word = (static_cast<unsigned long long>(flag) << 32) | __float_as_uint(out);
            for (int q = 0; q < p.pworld; ++q) st_relaxed_sys_u64(p.peer_slots[q] + e, word);
        } else if (p.gather_dst) {
            for (int q = 0; q < p.pworld; ++q) p.gather_dst[q][p.gather_off + j] = out;
        } else {
            p.y[j] = out;
        }
        if constexpr (MODE == kRopePairs) {
            if (p.kcache && j >= p.q_rows && j < p.q_rows + 2 * p.kv_rows) {
                const int jj = j - p.q_rows;
                const int hd = p.head_dim;
                const uint16_t bits = __half_as_ushort(__float2half_rn(out));
                int h, d;
                bool is_k;
                if (p.kv_interleave) {
                    const int w = jj % (2 * hd);
                    h = jj / (2 * hd);
                    is_k = w < hd;
                    d = w % hd;
                } else {
                    is_k = jj < p.kv_rows;
                    h = (is_k ? jj : jj - p.kv_rows) / hd;
                    d = jj % hd;
                }
                if (is_k) p.kcache[(static_cast<size_t>(p.pos) * (p.kv_rows / hd) + h) * hd + d] = bits;
                else p.vcache[((static_cast<size_t>(h) * (hd / 8) + d / 8) * p.ctx_cap + p.pos) * 8 + d % 8] = bits;
            }
        }
    }
}

template <int BITS, int MODE, bool DEEP>
__global__ void __launch_bounds__(kThreads, kCtasPerSm) gemv_kernel(const GemvParams p) {
    constexpr int NS = MODE == kSwiglu ? 2 : 1;
    constexpr int KPC = 128 / BITS;
    constexpr int D = ring_bytes<DEEP>() / (NS * kThreads * 16);  // rows in flight per thread
    constexpr bool kQuant = BITS <= 8;
    constexpr bool kNorm = MODE != kGemv;

    extern __shared__ __align__(16) uint8_t smem[];
    uint4* ring = reinterpret_cast<uint4*>(smem);                         // [NS][D][256]
    float* rbuf = reinterpret_cast<float*>(smem + ring_bytes<DEEP>());     // [S][NS*C + 4] (rank 0)
    float* xs = rbuf + p.rbuf_floats;                                      // [rows_cta][NS][KPC]
    __shared__ float red[NS][kThreads];                                    // row-group partials
    __shared__ float wred[kThreads / 32][3];
    __shared__ __align__(8) uint64_t red_bar;                              // S-1 deposits (rank 0)

    uint32_t nctarank, ctarank;
    asm("mov.u32 %0, %%cluster_nctarank;" : "=r"(nctarank));
    asm("mov.u32 %0, %%cluster_ctarank;" : "=r"(ctarank));
    const int S = static_cast<int>(nctarank);
    const int rank = static_cast<int>(ctarank);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int C = p.cols, G = kThreads / C;
    const int c = tid % C, grp = tid / C;
    const int col0 = blockIdx.y * C;
    const int col = col0 + c;
    const bool col_ok = col < p.N;
    const int r0 = rank * p.rows_cta;
    const int nrows = max(0, min(p.rows_cta, p.R - r0));
    const int nk = nrows * KPC;
    const size_t sblk = static_cast<size_t>(col0 / kGroup) * p.K;

    if (S > 1) {
        if (rank == 0 && threadIdx.x == 0) {
            mbar_init(smem_addr(&red_bar), static_cast<uint32_t>(S - 1));
            mbar_init_fence();
        }
        // Rank 0's barrier is initialised before any rank deposits (the
        // matching wait comes just before the deposits).
        cluster_arrive_release();
    }
    pdl_launch_dependents();

    // ---- activations first (gamma / scale / zero, then x after the wait), in
    // passes of 1024 values held in registers; the first pass is issued before
    // the weight stream so it is not queued behind it.
    constexpr int kMaxAct = 4;  // values per thread per pass
    float av_g[kMaxAct], av_s[NS][kMaxAct], av_z[NS][kMaxAct], av_x[kMaxAct];
    auto load_acts = [&](int base) {
#pragma unroll
        for (int q = 0; q < kMaxAct; ++q) {
            const int e = base + tid + q * kThreads;
            const int k = r0 * KPC + e;
            const bool ok = e < nk;
            av_g[q] = (kNorm && ok) ? __ldg(p.gamma + k) : 1.f;
#pragma unroll
            for (int st = 0; st < NS; ++st) {
                av_s[st][q] = (kQuant && ok) ? __ldg(p.s[st] + sblk + k) : 1.f;
                av_z[st][q] = (kQuant && ok) ? __ldg(p.z[st] + sblk + k) : 0.f;
            }
        }
    };
    // One deadline per thread for all its peer waits (kPeerWaitNs after its
    // first wait); once it has passed, later elements do not wait again.
    uint64_t deadline = 0;
    bool gave_up = false;
    auto load_x = [&](int base) {
#pragma unroll
        for (int q = 0; q < kMaxAct; ++q) {
            const int e = base + tid + q * kThreads;
            float v = e < nk ? p.x[r0 * KPC + e] : 0.f;
            if (p.xslots && e < nk) {
                const int k = r0 * KPC + e;
                const unsigned flag = static_cast<unsigned>(__ldcg(p.xslots + static_cast<size_t>(p.prank) * p.K + k) >> 32);
                for (int w = 0; w < p.pworld; ++w) {
                    const unsigned long long* src = p.xslots + static_cast<size_t>(w) * p.K + k;
                    unsigned long long word = ld_relaxed_sys_u64(src);
                    if (static_cast<unsigned>(word >> 32) != flag && !gave_up) {
                        if (deadline == 0) deadline = globaltimer_ns() + kPeerWaitNs;
                        while (static_cast<unsigned>((word = ld_relaxed_sys_u64(src)) >> 32) != flag) {
                            if (globaltimer_ns() > deadline) {  // bounded: give up, flag it
                                atomicOr(&g_status, kStatusPeerTimeout);
                                gave_up = true;
                                break;
                            }
                        }
                    }
                    v += __uint_as_float(static_cast<unsigned>(word));
                }
                if (p.xsave && blockIdx.y == 0) p.xsave[k] = v;
            }
            av_x[q] = v;
        }
    };
    float ss = 0.f, cz[NS];
#pragma unroll
    for (int st = 0; st < NS; ++st) cz[st] = 0.f;
    auto fold = [&](int base) {
#pragma unroll
        for (int q = 0; q < kMaxAct; ++q) {
            const int e = base + tid + q * kThreads;
            if (e < nk) {
                const float xv = av_x[q];
                float xg = xv;
                if constexpr (kNorm) {
                    ss = fmaf(xv, xv, ss);
                    xg = xv * av_g[q];
                }
                const int rl = e / KPC, i = e % KPC;
#pragma unroll
                for (int st = 0; st < NS; ++st) {
                    float v = xg;
                    if constexpr (kQuant) {
                        v = xg * av_s[st][q];
                        cz[st] = fmaf(xg, av_z[st][q], cz[st]);
                    }
                    if constexpr (BITS == 4) v *= int4_prescale(i);
                    xs[(rl * NS + st) * KPC + i] = v;
                }
            }
        }
    };
    load_acts(0);

    // ---- weights: prime the ring with D rows per thread ---------------------
    const int my_rows = nrows > grp ? (nrows - grp + G - 1) / G : 0;  // rows grp, grp+G, ...
    auto src = [&](int st, int i) {
        const int r = r0 + grp + i * G;
        return reinterpret_cast<const uint4*>(p.w[st]) + (static_cast<size_t>(r) * p.N + col);
    };
    auto slot = [&](int st, int i) { return smem_addr(ring + (st * D + (i % D)) * kThreads + tid); };
#pragma unroll
    for (int i = 0; i < D; ++i) {
        if (i < my_rows && col_ok)
#pragma unroll
            for (int st = 0; st < NS; ++st) cp_async16(slot(st, i), src(st, i));
        cp_async_commit();
    }

    // ---- x depends on the previous kernel: wait for it, then fold --------
    pdl_wait();
    load_x(0);
    fold(0);
    for (int base = kMaxAct * kThreads; base < nk; base += kMaxAct * kThreads) {
        load_acts(base);
        load_x(base);
        fold(base);
    }
    __syncthreads();

    // ---- stream this thread's rows through its ring ------------------------
    uint64_t acc[NS][4];
#pragma unroll
    for (int st = 0; st < NS; ++st) acc[st][0] = acc[st][1] = acc[st][2] = acc[st][3] = 0ull;
    for (int i = 0; i < my_rows; ++i) {
        cp_async_wait<D - 1>();
        const int rl = grp + i * G;
#pragma unroll
        for (int st = 0; st < NS; ++st) {
            const uint4 chunk = ring[(st * D + (i % D)) * kThreads + tid];
            chunk_fma<BITS>(chunk, xs + (rl * NS + st) * KPC, acc[st]);
        }
        if (i + D < my_rows && col_ok)
#pragma unroll
            for (int st = 0; st < NS; ++st) cp_async16(slot(st, i + D), src(st, i + D));
        cp_async_commit();
    }
    cp_async_wait<0>();

    // ---- reduce: row groups in shared memory, scalars across the CTA -------
#pragma unroll
    for (int st = 0; st < NS; ++st) {
        const float2 a = f2_unpack(acc[st][0]), b = f2_unpack(acc[st][1]);
        const float2 c2 = f2_unpack(acc[st][2]), d = f2_unpack(acc[st][3]);
        red[st][tid] = ((a.x + a.y) + (b.x + b.y)) + ((c2.x + c2.y) + (d.x + d.y));
    }
    {
        const float w0 = warp_sum(ss), w1 = warp_sum(cz[0]), w2 = NS == 2 ? warp_sum(cz[NS - 1]) : 0.f;
        if (lane == 0) {
            wred[warp][0] = w0;
            wred[warp][1] = w1;
            wred[warp][2] = w2;
        }
    }
    __syncthreads();

    // ---- cluster reduction: every rank deposits its partials in rank 0's
    // shared memory and leaves; rank 0 waits for S-1 deposits and finalises.
    if (S > 1) cluster_wait_acquire();
    const int pstride = NS * C + 4;  // floats per rank slot
    const uint32_t slot0 = smem_addr(rbuf) + static_cast<uint32_t>(rank * pstride * 4);
    const uint32_t dst = S > 1 ? map_cluster_addr(slot0, 0) : slot0;
    if (tid < C) {
#pragma unroll
        for (int st = 0; st < NS; ++st) {
            float v = 0.f;
            for (int g = 0; g < G; ++g) v += red[st][g * C + tid];
            if (rank == 0) rbuf[st * C + tid] = v;
            else st_cluster_f32(dst + 4u * (st * C + tid), v);
        }
    }
    if (tid < 3) {
        float v = 0.f;
#pragma unroll
        for (int w = 0; w < kThreads / 32; ++w) v += wred[w][tid];
        if (rank == 0) rbuf[NS * C + tid] = v;
        else st_cluster_f32(dst + 4u * (NS * C + tid), v);
    }
    if (rank != 0) {
        __syncthreads();
        if (tid == 0) {
            fence_acq_rel_cluster();
            mbar_arrive_remote(map_cluster_addr(smem_addr(&red_bar), 0));
        }
        return;
    }
    if (S > 1) {
        // kClusterWaitNs (1 s on the clock) is ten times the longest the other
        // ranks can be held before they deposit (each thread's peer waits
        // total at most kPeerWaitNs), so rank 0 does not give up and exit
        // while a deposit into its shared memory is still to come.
        if (tid == 0 && !mbar_wait_cluster_ns(smem_addr(&red_bar), 0, kClusterWaitNs))
            atomicOr(&g_status, kStatusReduceTimeout);
    }
    __syncthreads();
    if (tid < C || warp == 0) {
        const bool active = tid < C;
        float a[NS], tot[3] = {0.f, 0.f, 0.f};
#pragma unroll
        for (int st = 0; st < NS; ++st) a[st] = 0.f;
        if (active) {
            for (int q = 0; q < S; ++q) {
                const float* rp = rbuf + q * pstride;
#pragma unroll
                for (int st = 0; st < NS; ++st) a[st] += rp[st * C + tid];
                tot[0] += rp[NS * C];
                tot[1] += rp[NS * C + 1];
                tot[2] += rp[NS * C + 2];
            }
        }
        finalize<MODE, NS, kQuant, kNorm>(p, col0 + tid, active, a, tot);
    }
}

// ---- Integer dot products for quantised weights ---------------------------
// dp4a: four byte products summed into a 32-bit integer (unsigned codes times
// signed or unsigned activation bytes).
__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t b, int c) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ uint32_t dp4a_uu(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d;
    asm("dp4a.u32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// One chunk of one column against the chunk row's 16-bit activations X (high
// bytes xh, low bytes xl, X = 256 hi + lo): the exact integer sum of code * X
// over the chunk, as a float.  int8: 16 codes, byte l of word w is k = 4w + l;
// int4: 32 codes, nibble s of word w is k = 8w + s, split into the even and odd
// nibbles as bytes (the staging holds X in that order).  |sum| < 2^27.
template <int BITS>
__device__ __forceinline__ float chunk_idot(const uint4 c, const uint8_t* xh, const uint8_t* xl) {
    int hi = 0;
    uint32_t lo = 0;
    if constexpr (BITS == 8) {
        const uint4 h = *reinterpret_cast<const uint4*>(xh);
        const uint4 l = *reinterpret_cast<const uint4*>(xl);
        hi = dp4a_us(c.x, h.x, hi);
        hi = dp4a_us(c.y, h.y, hi);
        hi = dp4a_us(c.z, h.z, hi);
        hi = dp4a_us(c.w, h.w, hi);
        lo = dp4a_uu(c.x, l.x, lo);
        lo = dp4a_uu(c.y, l.y, lo);
        lo = dp4a_uu(c.z, l.z, lo);
        lo = dp4a_uu(c.w, l.w, lo);
    } else {
        const uint4* h4 = reinterpret_cast<const uint4*>(xh);
        const uint4* l4 = reinterpret_cast<const uint4*>(xl);
        const uint4 h0 = h4[0], h1 = h4[1], l0 = l4[0], l1 = l4[1];
        const uint32_t wd[4] = {c.x, c.y, c.z, c.w};
        const uint32_t hw[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
        const uint32_t lw[8] = {l0.x, l0.y, l0.z, l0.w, l1.x, l1.y, l1.z, l1.w};
#pragma unroll
        for (int w = 0; w < 4; ++w) {
            const uint32_t e = wd[w] & 0x0F0F0F0Fu, o = (wd[w] >> 4) & 0x0F0F0F0Fu;
            hi = dp4a_us(e, hw[2 * w], hi);
            hi = dp4a_us(o, hw[2 * w + 1], hi);
            lo = dp4a_uu(e, lw[2 * w], lo);
            lo = dp4a_uu(o, lw[2 * w + 1], lo);
        }
    }
    return __int2float_rn(hi * 256 + static_cast<int>(lo));
}

// ---- One CTA per SM: balanced column ranges, all of K per CTA ------------
// For matrices wide enough to give every SM at least 16 outputs.  The grid is
// exactly one CTA per SM, so every SM streams the same number of bytes: the
// CTAs of a scale block
// split its 256 outputs into even-aligned ranges, blocks getting
// floor(or ceil)(SMs / blocks) CTAs, which balances the SMs to within a few
// percent at the decode shapes.  Each CTA reads all of K for its columns, so
// the RMS sum, the zero-point constant and the whole dot product stay inside
// the CTA: no cluster, no split-K reduction, deterministic sums.  Streaming
// and arithmetic are those of gemv_kernel (per-thread cp.async rings, folded
// scales, exact code conversion); the C outputs times G row groups fill the
// CTA's threads.
//
// Two shapes of CTA.  T = 1024 threads hold all of an SM's registers, so a
// launch has the SMs to itself.  T = 512 threads with at most half an SM's
// shared memory leave room for the next launch in the stream: under
// programmatic dependent launch its CTA becomes resident beside this one,
// primes its ring (its weights do not depend on this kernel) and waits, so
// consecutive launches overlap their first bytes with the previous tail.
constexpr int kSmThreadsMax = 1024;
// Shared memory (dynamic + static) that lets two CTAs share an SM: the SM's
// 228 KB less the 1 KB the hardware reserves per CTA, halved.
constexpr int kSmHalfSmem = (228 - 2) * 1024 / 2;
constexpr int kSmStaticSmem = 512;  // wred and alignment

// Column range [col0, col0 + C) of CTA `cta` of `ctas` (see above); fp32 and
// fp16 weights have no scale blocks and split N evenly in pairs.
__device__ __forceinline__ void sm_columns(int N, bool blocks, int cta, int ctas, int& col0, int& C) {
    if (blocks) {
        const int nb = N / kGroup;
        const int base = ctas / nb, extra = ctas % nb;
        int b, m, per;
        if (cta < extra * (base + 1)) {
            per = base + 1;
            b = cta / per;
            m = cta % per;
        } else {
            per = base;
            const int i = cta - extra * (base + 1);
            b = extra + i / per;
            m = i % per;
        }
        const int lo = 2 * ((m * (kGroup / 2)) / per), hi = 2 * (((m + 1) * (kGroup / 2)) / per);
        col0 = b * kGroup + lo;
        C = hi - lo;
    } else {
        const int pairs = N / 2;
        const int lo = static_cast<int>((static_cast<long long>(cta) * pairs) / ctas);
        const int hi = static_cast<int>((static_cast<long long>(cta + 1) * pairs) / ctas);
        col0 = 2 * lo;
        C = 2 * (hi - lo);
    }
}

// The body of the per-SM kernel for CTA `cta` of `ctas`, run by all
// kSmThreads threads of the CTA with `smem` as its dynamic shared memory;
// `wait()` stands for the wait on the previous kernel (called by all threads
// after the weight ring is primed).
// UNROLL false: a compact stream loop; PRIME: ring rows requested before the
// wait (the rest right after it), fewer where the wait itself goes through
// this SM's memory pipeline.
template <int BITS, int MODE, int kSmThreads, int D, bool IDP, bool UNROLL = true, int PRIME = D, typename Wait>
__device__ __forceinline__ void gemv_sm_body(const GemvParams& p, uint8_t* smem, const int cta, const int ctas,
                                             Wait wait) {
    static_assert(PRIME >= 1 && PRIME <= D, "prime rows");
    constexpr int NS = MODE == kSwiglu ? 2 : 1;
    constexpr int KPC = 128 / BITS;
    constexpr bool kQuant = BITS <= 8;
    constexpr bool kNorm = MODE != kGemv;
    constexpr bool kIdp = IDP && kQuant;  // integer dot products (quantised weights)

    uint4* ring = reinterpret_cast<uint4*>(smem);                                  // [NS][D][T]
    float* xs = reinterpret_cast<float*>(smem + NS * D * kSmThreads * 16);         // [R][NS][KPC] fp32 x'
    // integer-dot staging instead of xs: per chunk row and stream, the row's
    // 16-bit activations as high (signed) and low (unsigned) bytes, in the
    // order the code bytes are multiplied, and the row's scale
    uint8_t* xh = smem + NS * D * kSmThreads * 16;                                 // [R][NS][KPC]
    uint8_t* xl = xh + static_cast<size_t>(p.R) * NS * KPC;                        // [R][NS][KPC]
    float* xsig = reinterpret_cast<float*>(xl + static_cast<size_t>(p.R) * NS * KPC);  // [R][NS]
    float* red = reinterpret_cast<float*>(smem);                                   // [NS][G][C], after the stream
    __shared__ float wred[kSmThreads / 32][3];

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    int col0, C;
    // Reversed: the blocks split among one CTA more (the lighter CTAs) take
    // the highest CTA indices, which start last and measured slowest.
    sm_columns(p.N, kQuant, ctas - 1 - cta, ctas, col0, C);
    const int G = kSmThreads / C;
    const int c = tid % C, grp = tid / C;
    const bool streams = grp < G;  // the last threads (fewer than C) only stage activations
    const int col = col0 + c;
    const int nk = p.K;
    const size_t sblk = static_cast<size_t>(col0 / kGroup) * p.K;

    pdl_launch_dependents();

    // ---- activations, in passes of 4T values: in pass j thread tid holds the
    // four consecutive k = j*4T + 4 tid .. + 3 (one 16-byte load per array), so
    // a chunk row's KPC values sit in KPC/4 consecutive lanes and K (a multiple
    // of KPC) ends on a row boundary.  gamma * scale and gamma * zero are formed
    // before the dependency wait (they are weights); x is loaded after it.  The
    // first kPre passes keep their activations in registers across the wait.
    constexpr int kPass = 4 * kSmThreads;
    constexpr int kPre = NS == 1 ? 3 : 1;
    float4 gs[kPre][NS], gz[kPre][NS], xv[kPre];
    auto mul4 = [](float4 a, float4 b) { return make_float4(a.x * b.x, a.y * b.y, a.z * b.z, a.w * b.w); };
    auto load_acts = [&](int j, float4 (&g_s)[NS], float4 (&g_z)[NS]) {
        const int k = j * kPass + 4 * tid;
        const bool ok = k < nk;
        float4 g = make_float4(1.f, 1.f, 1.f, 1.f);
        if (kNorm && ok) g = __ldg(reinterpret_cast<const float4*>(p.gamma + k));
#pragma unroll
        for (int st = 0; st < NS; ++st) {
            if constexpr (kQuant) {
                const float4 z4 = make_float4(0.f, 0.f, 0.f, 0.f);
                g_s[st] = ok ? mul4(g, __ldg(reinterpret_cast<const float4*>(p.s[st] + sblk + k))) : z4;
                g_z[st] = ok ? mul4(g, __ldg(reinterpret_cast<const float4*>(p.z[st] + sblk + k))) : z4;
            } else {
                g_s[st] = g;
            }
        }
    };
    auto load_x = [&](int j) {
        const int k = j * kPass + 4 * tid;
        // L2 loads: x may come from other CTAs of a persistent kernel
        return k < nk ? __ldcg(reinterpret_cast<const float4*>(p.x + k)) : make_float4(0.f, 0.f, 0.f, 0.f);
    };
    float ss = 0.f, cz[NS];
#pragma unroll
    for (int st = 0; st < NS; ++st) cz[st] = 0.f;
    auto fold = [&](int j, const float4 x4, const float4 (&g_s)[NS], const float4 (&g_z)[NS]) {
        const int k = j * kPass + 4 * tid;
        const bool ok = k < nk;
        if constexpr (kNorm) ss = fmaf(x4.x, x4.x, fmaf(x4.y, x4.y, fmaf(x4.z, x4.z, fmaf(x4.w, x4.w, ss))));
        const int rl = k / KPC, i = k % KPC;  // i: a multiple of 4
#pragma unroll
        for (int st = 0; st < NS; ++st) {
            const float4 v = mul4(x4, g_s[st]);
            if constexpr (kQuant)
                cz[st] = fmaf(x4.x, g_z[st].x, fmaf(x4.y, g_z[st].y, fmaf(x4.z, g_z[st].z, fmaf(x4.w, g_z[st].w, cz[st]))));
            const size_t b = static_cast<size_t>(rl * NS + st) * KPC;
            if constexpr (kIdp) {
                // x' of the row as integers of 16 bits against the row's
                // largest magnitude m: X = rn(x' * 32767 / m), x' ~ X m / 32767
                float m = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
#pragma unroll
                for (int o = KPC / 8; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
                const float inv = m > 0.f ? __fdividef(32767.0f, m) : 0.f;
                auto q16 = [&](float f) { return max(-32767, min(32767, __float2int_rn(f * inv))); };
                const int X0 = q16(v.x), X1 = q16(v.y), X2 = q16(v.z), X3 = q16(v.w);
                if (ok) {
                    if constexpr (BITS == 8) {
                        // bytes i .. i+3 of the row, in k order
                        const uint32_t lo = (X0 & 0xFF) | ((X1 & 0xFF) << 8) | ((X2 & 0xFF) << 16) |
                                            (static_cast<uint32_t>(X3 & 0xFF) << 24);
                        const uint32_t hi = ((X0 >> 8) & 0xFF) | (((X1 >> 8) & 0xFF) << 8) |
                                            (((X2 >> 8) & 0xFF) << 16) | (static_cast<uint32_t>((X3 >> 8) & 0xFF) << 24);
                        *reinterpret_cast<uint32_t*>(xh + b + i) = hi;
                        *reinterpret_cast<uint32_t*>(xl + b + i) = lo;
                    } else {
                        // int4: per code word (k = 8w + s) the even nibbles'
                        // activations, then the odd ones: s -> ((s & 1) << 2) | (s >> 1).
                        // Values s0..s0+3 (s0 = 0 or 4) go to bytes (s0/2, s0/2 + 1)
                        // for s0, s0+2 and (4 + s0/2, 5 + s0/2) for s0+1, s0+3.
                        const int w8 = (i >> 3) << 3, sh = (i & 4) >> 1;
                        const uint32_t lo_e = (X0 & 0xFF) | ((X2 & 0xFF) << 8), lo_o = (X1 & 0xFF) | ((X3 & 0xFF) << 8);
                        const uint32_t hi_e = ((X0 >> 8) & 0xFF) | (((X2 >> 8) & 0xFF) << 8);
                        const uint32_t hi_o = ((X1 >> 8) & 0xFF) | (((X3 >> 8) & 0xFF) << 8);
                        *reinterpret_cast<uint16_t*>(xh + b + w8 + sh) = static_cast<uint16_t>(hi_e);
                        *reinterpret_cast<uint16_t*>(xh + b + w8 + 4 + sh) = static_cast<uint16_t>(hi_o);
                        *reinterpret_cast<uint16_t*>(xl + b + w8 + sh) = static_cast<uint16_t>(lo_e);
                        *reinterpret_cast<uint16_t*>(xl + b + w8 + 4 + sh) = static_cast<uint16_t>(lo_o);
                    }
                    if (i == 0) xsig[rl * NS + st] = m * (1.0f / 32767.0f);
                }
            } else if (ok) {
                float4 w = v;
                if constexpr (BITS == 4) {
                    w.x *= int4_prescale(i);
                    w.y *= int4_prescale(i + 1);
                    w.z *= int4_prescale(i + 2);
                    w.w *= int4_prescale(i + 3);
                }
                *reinterpret_cast<float4*>(xs + b + i) = w;
            }
        }
    };
#pragma unroll
    for (int j = 0; j < kPre; ++j)
        if (j * kPass < nk) load_acts(j, gs[j], gz[j]);

    // ---- weights: prime the ring with D rows per thread -------------------
    const int my_rows = streams && grp < p.R ? (p.R - grp + G - 1) / G : 0;  // rows grp, grp+G, ...
    // Row grp + i*G of column col sits at w + (grp + i*G)*N + col (16-byte
    // units); ring slot (stream st, row i) at slot0 + (st*D + i%D)*T*16.
    const size_t row_step = static_cast<size_t>(G) * p.N;
    const uint4* wp[NS];
#pragma unroll
    for (int st = 0; st < NS; ++st)
        wp[st] = reinterpret_cast<const uint4*>(p.w[st]) + (static_cast<size_t>(grp) * p.N + col);
    const uint32_t slot0 = smem_addr(ring + tid);
    auto prime = [&](int u) {
        if (u < my_rows) {
#pragma unroll
            for (int st = 0; st < NS; ++st) {
                cp_async16(slot0 + static_cast<uint32_t>((st * D + u) * kSmThreads * 16), wp[st]);
                wp[st] += row_step;
            }
        }
        cp_async_commit();
    };
#pragma unroll
    for (int u = 0; u < PRIME; ++u) prime(u);

    // ---- x depends on the previous kernel: wait for it, then fold --------
    wait();
#pragma unroll
    for (int u = PRIME; u < D; ++u) prime(u);
#pragma unroll
    for (int j = 0; j < kPre; ++j) xv[j] = j * kPass < nk ? load_x(j) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int j = 0; j < kPre; ++j)
        if (j * kPass < nk) fold(j, xv[j], gs[j], gz[j]);
    if (kPre * kPass < nk) {
        // later passes: the next pass's loads are in flight while this one folds
        float4 n_s[NS], n_z[NS], nx;
        load_acts(kPre, n_s, n_z);
        nx = load_x(kPre);
        for (int j = kPre; j * kPass < nk; ++j) {
            float4 g_s[NS], g_z[NS];
#pragma unroll
            for (int st = 0; st < NS; ++st) {
                g_s[st] = n_s[st];
                g_z[st] = n_z[st];
            }
            const float4 x4 = nx;
            if ((j + 1) * kPass < nk) {
                load_acts(j + 1, n_s, n_z);
                nx = load_x(j + 1);
            }
            fold(j, x4, g_s, g_z);
        }
    }
    __syncthreads();

    // ---- stream this thread's rows through its ring ------------------------
    uint64_t acc[NS][4];
    float accf[NS];
#pragma unroll
    for (int st = 0; st < NS; ++st) {
        acc[st][0] = acc[st][1] = acc[st][2] = acc[st][3] = 0ull;
        accf[st] = 0.f;
    }
    // Unrolled by the ring depth, so every slot offset is a constant; the
    // weight and activation pointers advance by whole rows.
    const float* xrow = xs + grp * NS * KPC;
    const int xstep = G * NS * KPC;
    int xr = grp;  // chunk row (integer-dot staging)
    if constexpr (!UNROLL) {
        // one row per iteration, the ring slot a running index: compact code
        // for a kernel that holds several phases
        int u = 0;
#pragma unroll 1
        for (int i = 0; i < my_rows; ++i) {
            cp_async_wait<D - 1>();
#pragma unroll
            for (int st = 0; st < NS; ++st) {
                const uint4 chunk = ring[(st * D + u) * kSmThreads + tid];
                if constexpr (kIdp) {
                    const int off = (xr * NS + st) * KPC;
                    accf[st] = fmaf(xsig[xr * NS + st], chunk_idot<BITS>(chunk, xh + off, xl + off), accf[st]);
                } else {
                    chunk_fma<BITS>(chunk, xrow + st * KPC, acc[st]);
                }
            }
            xrow += xstep;
            xr += G;
            if (i + D < my_rows) {
#pragma unroll
                for (int st = 0; st < NS; ++st) {
                    cp_async16(slot0 + static_cast<uint32_t>((st * D + u) * kSmThreads * 16), wp[st]);
                    wp[st] += row_step;
                }
            }
            cp_async_commit();
            u = u + 1 == D ? 0 : u + 1;
        }
    }
    for (int i = 0; UNROLL && i < my_rows; i += D) {
#pragma unroll
        for (int u = 0; u < D; ++u) {
            if (i + u < my_rows) {
                cp_async_wait<D - 1>();
#pragma unroll
                for (int st = 0; st < NS; ++st) {
                    const uint4 chunk = ring[(st * D + u) * kSmThreads + tid];
                    if constexpr (kIdp) {
                        const int off = (xr * NS + st) * KPC;
                        accf[st] = fmaf(xsig[xr * NS + st], chunk_idot<BITS>(chunk, xh + off, xl + off), accf[st]);
                    } else {
                        chunk_fma<BITS>(chunk, xrow + st * KPC, acc[st]);
                    }
                }
                xrow += xstep;
                xr += G;
                if (i + u + D < my_rows) {
#pragma unroll
                    for (int st = 0; st < NS; ++st) {
                        cp_async16(slot0 + static_cast<uint32_t>((st * D + u) * kSmThreads * 16), wp[st]);
                        wp[st] += row_step;
                    }
                }
                cp_async_commit();
            }
        }
    }
    cp_async_wait<0>();

    // ---- reduce the row groups of each column and the CTA's scalars --------
    {
        const float w0 = warp_sum(ss), w1 = warp_sum(cz[0]), w2 = NS == 2 ? warp_sum(cz[NS - 1]) : 0.f;
        if (lane == 0) {
            wred[warp][0] = w0;
            wred[warp][1] = w1;
            wred[warp][2] = w2;
        }
    }
    __syncthreads();  // every thread's ring reads are done: the ring becomes `red`
    if (streams) {
#pragma unroll
        for (int st = 0; st < NS; ++st) {
            if constexpr (kIdp) {
                red[(st * G + grp) * C + c] = accf[st];
            } else {
                const float2 a = f2_unpack(acc[st][0]), b = f2_unpack(acc[st][1]);
                const float2 c2 = f2_unpack(acc[st][2]), d = f2_unpack(acc[st][3]);
                red[(st * G + grp) * C + c] = ((a.x + a.y) + (b.x + b.y)) + ((c2.x + c2.y) + (d.x + d.y));
            }
        }
    }
    __syncthreads();
    if (warp * 32 < C) {
        const bool active = tid < C;
        float a[NS], tot[3] = {0.f, 0.f, 0.f};
#pragma unroll
        for (int st = 0; st < NS; ++st) {
            a[st] = 0.f;
            if (active)
                for (int g = 0; g < G; ++g) a[st] += red[(st * G + g) * C + tid];
        }
#pragma unroll
        for (int w = 0; w < kSmThreads / 32; ++w) {
            tot[0] += wred[w][0];
            tot[1] += wred[w][1];
            tot[2] += wred[w][2];
        }
        finalize<MODE, NS, kQuant, kNorm>(p, col0 + tid, active, a, tot);
    }
}

template <int BITS, int MODE, int kSmThreads, int D, bool IDP>
__global__ void __launch_bounds__(kSmThreads, kSmThreadsMax / kSmThreads) gemv_sm_kernel(const GemvParams p) {
    extern __shared__ __align__(16) uint8_t smem[];
    gemv_sm_body<BITS, MODE, kSmThreads, D, IDP>(p, smem, blockIdx.x, gridDim.x, [] { pdl_wait(); });
}

// ---- Batched decode: M activation vectors against one weight stream -------
// The same decomposition as gemv_kernel (cluster split K, per-thread cp.async
// ring, rank-0 reduction over DSMEM), with M staged activation rows: each
// weight chunk is decoded once into f32x2 pairs and multiplied into M
// accumulators, so the weights stream from HBM once for all M vectors.
constexpr int kMaxBatch = 8;

struct BatchParams {
    const uint8_t* w;
    const float* s;
    const float* z;
    const float* x;      // [M][K]
    const float* gamma;  // RmsNorm-GEMV; unused by the plain GEMV
    float* y;            // [M][N]
    int N, K, R;
    int cols, rows_cta, rbuf_floats;
    float eps, inv_dim;
};

// The KPC/2 weight pairs of one chunk, in the order of the staged activations
// (pair p multiplies activations 2p and 2p+1): exact codes (minus the 2^23
// bias) for int8/int4 -- int4 nibbles keep their bit position, the staged
// activations carry the matching power of two -- and converted values for
// fp16/fp32.
template <int BITS>
__device__ __forceinline__ void decode_pairs(const uint4 c, uint64_t (&w)[64 / BITS]) {
    const uint32_t wd[4] = {c.x, c.y, c.z, c.w};
    if constexpr (BITS == 32) {
        w[0] = f2_pack(__uint_as_float(c.x), __uint_as_float(c.y));
        w[1] = f2_pack(__uint_as_float(c.z), __uint_as_float(c.w));
    } else if constexpr (BITS == 16) {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&wd[q]));
            w[q] = f2_pack(f.x, f.y);
        }
    } else if constexpr (BITS == 8) {
        const uint64_t neg = f2_pack(-8388608.0f, -8388608.0f);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            w[2 * q] = f2_add(byte_pair<0x7540, 0x7541>(wd[q]), neg);
            w[2 * q + 1] = f2_add(byte_pair<0x7542, 0x7543>(wd[q]), neg);
        }
    } else {
        const uint64_t neg = f2_pack(-8388608.0f, -8388608.0f);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const uint32_t a = wd[q], h = a >> 12;
            w[4 * q + 0] = f2_add(nib_pair(a, 0xFu, a, 0xF0u), neg);
            w[4 * q + 1] = f2_add(nib_pair(a, 0xF00u, a, 0xF000u), neg);
            w[4 * q + 2] = f2_add(nib_pair(a, 0xF0000u, h, 0xF00u), neg);
            w[4 * q + 3] = f2_add(nib_pair(h, 0xF000u, h, 0xF0000u), neg);
        }
    }
}

// Cluster reduce-scatter epilogue of the batched kernels.  colsum(m, c) is
// this CTA's partial sum for vector m and column c (c < C), scal(i) its i-th
// scalar (i < 2 MS: the sum of squares and the zero-point constant of each
// vector).  Rank d finalises columns [d share, (d + 1) share): every rank
// stores its partials for those columns and its scalars into slot `rank` of
// rank d's receive buffer rbuf [S][MS share + 2 MS] over DSMEM, arrives on
// d's barrier (initialised for S - 1 arrivals), and each rank adds the S
// slots in rank order (deterministic) and writes y.
template <int MS, bool NORM, bool QUANT, typename ColSum, typename Scal>
__device__ __forceinline__ void batched_reduce_scatter(const BatchParams& p, float* rbuf, uint64_t* red_bar, int S,
                                                       int rank, int C, int col0, int M, ColSum colsum, Scal scal) {
    const int tid = threadIdx.x;
    if (S > 1) cluster_wait_acquire();  // every rank's barrier is initialised
    const int share = (C + S - 1) / S;
    const int rstride = MS * share + 2 * MS;
    const uint32_t my_slot = smem_addr(rbuf) + static_cast<uint32_t>(rank * rstride * 4);
    if (tid < C) {
        const int dest = tid / share, cl = tid % share;
        const uint32_t dst = dest == rank ? my_slot : map_cluster_addr(my_slot, dest);
        for (int m = 0; m < M; ++m) {
            const float v = colsum(m, tid);
            if (dest == rank) rbuf[rank * rstride + m * share + cl] = v;
            else st_cluster_f32(dst + 4u * (m * share + cl), v);
        }
    }
    if (tid < 2 * MS) {
        const float v = scal(tid);
        for (int d = 0; d < S; ++d) {
            if (d == rank) rbuf[rank * rstride + MS * share + tid] = v;
            else st_cluster_f32(map_cluster_addr(my_slot, d) + 4u * (MS * share + tid), v);
        }
    }
    __syncthreads();
    if (S > 1 && tid == 0) {
        fence_acq_rel_cluster();
        for (int d = 0; d < S; ++d)
            if (d != rank) mbar_arrive_remote(map_cluster_addr(smem_addr(red_bar), d));
        // the other ranks arrive once their weight streams end (no peer waits
        // in the batched kernels): kClusterWaitNs on the clock is far beyond that
        if (!mbar_wait_cluster_ns(smem_addr(red_bar), 0, kClusterWaitNs)) atomicOr(&g_status, kStatusReduceTimeout);
    }
    __syncthreads();
    const int cc = rank * share + tid;
    if (tid < share && cc < C && col0 + cc < p.N) {
        for (int m = 0; m < M; ++m) {
            float a = 0.f, sq = 0.f, zc = 0.f;
            for (int q = 0; q < S; ++q) {
                const float* rp = rbuf + q * rstride;
                a += rp[m * share + tid];
                sq += rp[MS * share + 2 * m];
                zc += rp[MS * share + 2 * m + 1];
            }
            const float inv = NORM ? 1.0f / sqrtf(sq * p.inv_dim + p.eps) : 1.0f;
            p.y[static_cast<size_t>(m) * p.N + col0 + cc] = (QUANT ? a - zc : a) * inv;
        }
    }
}

template <int BITS, int M, bool NORM>
__global__ void __launch_bounds__(kThreads, 2) gemv_batched_kernel(const BatchParams p) {
    constexpr int KPC = 128 / BITS, NP = KPC / 2;
    constexpr int D = 32768 / (kThreads * 16);  // rows in flight per thread
    constexpr bool kQuant = BITS <= 8;

    extern __shared__ __align__(16) uint8_t smem[];
    uint4* ring = reinterpret_cast<uint4*>(smem);                          // [D][256]
    float* rbuf = reinterpret_cast<float*>(smem + D * kThreads * 16);      // [S][M*share + 2M]
    float* xs = rbuf + p.rbuf_floats;                                      // [rows_cta][M][KPC]
    __shared__ float red[M][kThreads];
    __shared__ float wred[kThreads / 32][2 * M];
    __shared__ __align__(8) uint64_t red_bar;

    uint32_t nctarank, ctarank;
    asm("mov.u32 %0, %%cluster_nctarank;" : "=r"(nctarank));
    asm("mov.u32 %0, %%cluster_ctarank;" : "=r"(ctarank));
    const int S = static_cast<int>(nctarank);
    const int rank = static_cast<int>(ctarank);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int C = p.cols, G = kThreads / C;
    const int c = tid % C, grp = tid / C;
    const int col0 = blockIdx.y * C;
    const int col = col0 + c;
    const bool col_ok = col < p.N;
    const int r0 = rank * p.rows_cta;
    const int nrows = max(0, min(p.rows_cta, p.R - r0));
    const int nk = nrows * KPC;
    const size_t sblk = static_cast<size_t>(col0 / kGroup) * p.K;

    if (S > 1) {
        if (tid == 0) {  // every rank receives the other S-1 ranks' deposits
            mbar_init(smem_addr(&red_bar), static_cast<uint32_t>(S - 1));
            mbar_init_fence();
        }
        cluster_arrive_release();
    }
    pdl_launch_dependents();

    // weights never depend on the previous kernel: prime the ring first
    const int my_rows = nrows > grp ? (nrows - grp + G - 1) / G : 0;
    auto src = [&](int i) {
        return reinterpret_cast<const uint4*>(p.w) + (static_cast<size_t>(r0 + grp + i * G) * p.N + col);
    };
    auto slot = [&](int i) { return smem_addr(ring + (i % D) * kThreads + tid); };
#pragma unroll
    for (int i = 0; i < D; ++i) {
        if (i < my_rows && col_ok) cp_async16(slot(i), src(i));
        cp_async_commit();
    }

    // x'[m][k] = x[m][k] * gamma[k] * s[k] (times the int4 nibble scale);
    // per vector: sum of squares, zero-point constant sum_k x gamma z.
    pdl_wait();
    float ss[M], cz[M];
#pragma unroll
    for (int m = 0; m < M; ++m) ss[m] = cz[m] = 0.f;
    for (int e = tid; e < nk; e += kThreads) {
        const int k = r0 * KPC + e;
        const float g = NORM ? __ldg(p.gamma + k) : 1.f;
        const float sc = kQuant ? __ldg(p.s + sblk + k) : 1.f;
        const float zz = kQuant ? __ldg(p.z + sblk + k) : 0.f;
        const int rl = e / KPC, i = e % KPC;
        const float pre = BITS == 4 ? int4_prescale(i) : 1.f;
#pragma unroll
        for (int m = 0; m < M; ++m) {
            const float xv = p.x[static_cast<size_t>(m) * p.K + k];
            if (NORM) ss[m] = fmaf(xv, xv, ss[m]);
            const float xg = xv * g;
            if (kQuant) cz[m] = fmaf(xg, zz, cz[m]);
            xs[(rl * M + m) * KPC + i] = xg * sc * pre;
        }
    }
    __syncthreads();

    uint64_t acc[M][4];
#pragma unroll
    for (int m = 0; m < M; ++m) acc[m][0] = acc[m][1] = acc[m][2] = acc[m][3] = 0ull;
    for (int i = 0; i < my_rows; ++i) {
        cp_async_wait<D - 1>();
        const int rl = grp + i * G;
        uint64_t w[NP];
        decode_pairs<BITS>(ring[(i % D) * kThreads + tid], w);
        const float4* xr = reinterpret_cast<const float4*>(xs + rl * M * KPC);
#pragma unroll
        for (int m = 0; m < M; ++m) {
#pragma unroll
            for (int q = 0; q < NP; q += 2) {
                const float4 xv = xr[(m * KPC + 2 * q) / 4];
                acc[m][q & 3] = f2_fma(f2_pack(xv.x, xv.y), w[q], acc[m][q & 3]);
                acc[m][(q + 1) & 3] = f2_fma(f2_pack(xv.z, xv.w), w[q + 1], acc[m][(q + 1) & 3]);
            }
        }
        if (i + D < my_rows && col_ok) cp_async16(slot(i + D), src(i + D));
        cp_async_commit();
    }
    cp_async_wait<0>();

#pragma unroll
    for (int m = 0; m < M; ++m) {
        const float2 a = f2_unpack(acc[m][0]), b = f2_unpack(acc[m][1]);
        const float2 c2 = f2_unpack(acc[m][2]), d = f2_unpack(acc[m][3]);
        red[m][tid] = ((a.x + a.y) + (b.x + b.y)) + ((c2.x + c2.y) + (d.x + d.y));
        const float w0 = warp_sum(ss[m]), w1 = warp_sum(cz[m]);
        if (lane == 0) {
            wred[warp][2 * m] = w0;
            wred[warp][2 * m + 1] = w1;
        }
    }
    __syncthreads();

    batched_reduce_scatter<M, NORM, kQuant>(
        p, rbuf, &red_bar, S, rank, C, col0, M,
        [&](int m, int c) {
            float v = 0.f;
            for (int g = 0; g < G; ++g) v += red[m][g * C + c];
            return v;
        },
        [&](int i) {
            float v = 0.f;
#pragma unroll
            for (int w = 0; w < kThreads / 32; ++w) v += wred[w][i];
            return v;
        });
}

// ---- Batched decode on the tensor cores (int8 / int4 weights) ------------
// mma.sync m16n8k16 with 16 weight columns as the M dimension (A: the codes as
// fp16, exact) and the (up to 8) vectors as N (B: x' = x gamma s scaled by a
// per-CTA power of two and split into fp16 high and low parts, two MMAs,
// about 22 significant bits; fp32 accumulation).  Inside every 16-byte chunk
// the k order is permuted so that lane (g, t4) of a warp reads one 32-bit
// word per column, bytes [4 t4, 4 t4 + 4); the staged B fragments follow the
// same permutation (a dot product does not depend on the order).  A warp owns
// 64 columns and every RG-th chunk row of the CTA's K slice, and streams them
// through its own cp.async ring (warps never wait for each other while
// streaming).  About 1.5 instructions per weight for any batch, against
// 5-10 for the SIMT kernel.  The epilogue is the SIMT batched kernel's
// cluster reduce-scatter.
constexpr int kMmaRing = 8;  // chunk rows in flight per warp (1 KB each)

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ void mma16816_f16(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t hsub_1024(uint32_t h) {
    uint32_t d;
    asm("sub.f16x2 %0, %1, %2;" : "=r"(d) : "r"(h), "r"(0x64006400u));
    return d;
}
// int8: bytes (0,1) or (2,3) of w as an exact fp16 pair
template <uint32_t SEL>
__device__ __forceinline__ uint32_t byte_h2(uint32_t w) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(w), "r"(0x64646464u), "n"(SEL));
    return hsub_1024(d);
}
// int4: nibbles (j, j + 4) of w as an exact fp16 pair
__device__ __forceinline__ uint32_t nib_h2(uint32_t w, int j) {
    uint32_t d;
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(w >> (4 * j)), "r"(0x000F000Fu), "r"(0x64006400u));
    return hsub_1024(d);
}

template <int BITS, bool NORM>
__global__ void __launch_bounds__(kThreads, 2) gemv_batched_mma_kernel(const BatchParams p, const int M) {
    constexpr int KPC = 128 / BITS;
    constexpr int STEPS = KPC / 16;   // k16 steps per chunk: int8 1, int4 2
    constexpr int FRAG = 4 * STEPS;   // staged u32 per (row, vector, t4): {hi b0, hi b1, lo b0, lo b1} per step
    static_assert(BITS == 8 || BITS == 4, "tensor-core batched decode: int8 / int4 codes");

    extern __shared__ __align__(16) uint8_t smem[];
    uint4* ring = reinterpret_cast<uint4*>(smem);                                   // [8 warps][kMmaRing][64]
    float* rbuf = reinterpret_cast<float*>(smem + 8 * kMmaRing * 64 * 16);          // reduce-scatter slots
    uint32_t* bfr = reinterpret_cast<uint32_t*>(rbuf + p.rbuf_floats);              // [rows][8][4][FRAG]
    float* red = reinterpret_cast<float*>(smem);  // after streaming: [RG][8][C] over the ring
    __shared__ float wred[kThreads / 32][2 * kMaxBatch];
    __shared__ float s_amax[kThreads / 32];
    __shared__ __align__(8) uint64_t red_bar;

    uint32_t nctarank, ctarank;
    asm("mov.u32 %0, %%cluster_nctarank;" : "=r"(nctarank));
    asm("mov.u32 %0, %%cluster_ctarank;" : "=r"(ctarank));
    const int S = static_cast<int>(nctarank);
    const int rank = static_cast<int>(ctarank);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int g = lane >> 2, t4 = lane & 3;
    const int C = p.cols, NCG = C / 64, RG = 8 / NCG;
    const int cg = warp % NCG, rg = warp / NCG;
    const int col0 = blockIdx.y * C;
    const int r0 = rank * p.rows_cta;
    const int nrows = max(0, min(p.rows_cta, p.R - r0));
    const int nk = nrows * KPC;
    const size_t sblk = static_cast<size_t>(col0 / kGroup) * p.K;

    if (S > 1) {
        if (tid == 0) {
            mbar_init(smem_addr(&red_bar), static_cast<uint32_t>(S - 1));
            mbar_init_fence();
        }
        cluster_arrive_release();
    }
    pdl_launch_dependents();

    // weights first: this warp's rows rg, rg + RG, ... of its 64 columns
    uint4* wring = ring + warp * kMmaRing * 64;
    const int my_rows = nrows > rg ? (nrows - rg + RG - 1) / RG : 0;
    const uint4* wsrc = reinterpret_cast<const uint4*>(p.w) + col0 + cg * 64 + lane;
    auto copy_row = [&](int i) {
        const size_t r = static_cast<size_t>(r0 + rg + i * RG);
        const uint32_t dst = smem_addr(wring + (i % kMmaRing) * 64 + lane);
        cp_async16(dst, wsrc + r * p.N);
        cp_async16(dst + 32 * 16, wsrc + r * p.N + 32);
    };
#pragma unroll
    for (int i = 0; i < kMmaRing; ++i) {
        if (i < my_rows) copy_row(i);
        cp_async_commit();
    }

    // x' = x gamma s for this CTA's k slice.  Pass 1 stores it as fp32 in the
    // staging area in natural order, [row][vector][KPC] (the same bytes the
    // fragments take), with the sums of squares, zero-point constants and the
    // largest magnitude; pass 2 rewrites each (row, vector) block in place --
    // one thread per block -- as the permuted fp16 high/low fragments, scaled
    // by the per-CTA power of two that brings the magnitude to [2^14, 2^15).
    pdl_wait();
    float ss[kMaxBatch], cz[kMaxBatch];
#pragma unroll
    for (int m = 0; m < kMaxBatch; ++m) ss[m] = cz[m] = 0.f;
    float amax = 0.f;
    float* xf = reinterpret_cast<float*>(bfr);
    constexpr int U = 2;
    for (int e0 = tid; e0 < nk; e0 += U * kThreads) {
        float gm[U], sc[U], zz[U], xv[U][kMaxBatch];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int e = e0 + u * kThreads;
            const bool ok = e < nk;
            const int k = r0 * KPC + (ok ? e : 0);
            gm[u] = (NORM && ok) ? __ldg(p.gamma + k) : 1.f;
            sc[u] = ok ? __ldg(p.s + sblk + k) : 0.f;
            zz[u] = ok ? __ldg(p.z + sblk + k) : 0.f;
#pragma unroll
            for (int m = 0; m < kMaxBatch; ++m)
                xv[u][m] = (ok && m < M) ? __ldg(p.x + static_cast<size_t>(m) * p.K + k) : 0.f;
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int e = e0 + u * kThreads;
            if (e >= nk) continue;
            const int rl = e / KPC, i = e % KPC;
#pragma unroll
            for (int m = 0; m < kMaxBatch; ++m) {
                const float xg = xv[u][m] * gm[u];
                if (NORM) ss[m] = fmaf(xv[u][m], xv[u][m], ss[m]);
                cz[m] = fmaf(xg, zz[u], cz[m]);
                const float v = xg * sc[u];
                amax = fmaxf(amax, fabsf(v));
                xf[(rl * 8 + m) * KPC + i] = v;
            }
        }
    }
#pragma unroll
    for (int m = 0; m < kMaxBatch; ++m) {
        const float w0 = warp_sum(ss[m]), w1 = warp_sum(cz[m]);
        if (lane == 0) {
            wred[warp][2 * m] = w0;
            wred[warp][2 * m + 1] = w1;
        }
    }
    amax = warp_max(amax);
    if (lane == 0) s_amax[warp] = amax;
    __syncthreads();
    amax = 0.f;
#pragma unroll
    for (int w = 0; w < kThreads / 32; ++w) amax = fmaxf(amax, s_amax[w]);
    int ex = 0;
    if (amax > 0.f) ex = 14 - (((__float_as_int(amax) >> 23) & 0xFF) - 127);
    ex = max(-100, min(100, ex));
    const float up = ldexpf(1.0f, ex), down = ldexpf(1.0f, -ex);

    // pass 2: blocks of vectors m >= M are zero, which is also their fragment
    for (int blk = tid; blk < nrows * 8; blk += kThreads) {
        const int m = blk & 7;
        if (m >= M) continue;
        float4* bp = reinterpret_cast<float4*>(xf + blk * KPC);
        float v[KPC];
#pragma unroll
        for (int q = 0; q < KPC / 4; ++q) {
            const float4 f = bp[q];
            v[4 * q] = f.x * up;
            v[4 * q + 1] = f.y * up;
            v[4 * q + 2] = f.z * up;
            v[4 * q + 3] = f.w * up;
        }
        uint32_t fr[4][FRAG];  // [t4][u32]
#pragma unroll
        for (int i = 0; i < KPC; ++i) {
            int tq, u, half;
            if (BITS == 8) {
                tq = i >> 2;
                u = (i >> 1) & 1;
                half = i & 1;
            } else {
                tq = i >> 3;
                const int nib = i & 7, j = nib & 3;
                u = (j >> 1) * 4 + (j & 1);
                half = nib >> 2;
            }
            const __half hi = __float2half_rn(v[i]);
            const __half lo = __float2half_rn(v[i] - __half2float(hi));
            const uint32_t hb = __half_as_ushort(hi), lb = __half_as_ushort(lo);
            if (half == 0) {
                fr[tq][u] = hb;
                fr[tq][u + 2] = lb;
            } else {
                fr[tq][u] |= hb << 16;
                fr[tq][u + 2] |= lb << 16;
            }
        }
        uint4* op = reinterpret_cast<uint4*>(bp);
#pragma unroll
        for (int tq = 0; tq < 4; ++tq)
#pragma unroll
            for (int q = 0; q < FRAG / 4; ++q)
                op[tq * (FRAG / 4) + q] =
                    make_uint4(fr[tq][4 * q], fr[tq][4 * q + 1], fr[tq][4 * q + 2], fr[tq][4 * q + 3]);
    }
    __syncthreads();

    // stream: per row, 4 tiles of 16 columns x 16 (or 2 x 16) k
    float acc[4][4];
#pragma unroll
    for (int t = 0; t < 4; ++t) acc[t][0] = acc[t][1] = acc[t][2] = acc[t][3] = 0.f;
    for (int i = 0; i < my_rows; ++i) {
        cp_async_wait<kMmaRing - 1>();
        __syncwarp();
        const uint32_t* rowp = reinterpret_cast<const uint32_t*>(wring + (i % kMmaRing) * 64);
        const int rl = rg + i * RG;
        const uint4* bq = reinterpret_cast<const uint4*>(bfr + ((static_cast<size_t>(rl) * 8 + g) * 4 + t4) * FRAG);
        const uint4 b0 = bq[0];
        uint4 b1 = b0;
        if constexpr (STEPS == 2) b1 = bq[1];
#pragma unroll
        for (int t = 0; t < 4; ++t) {
            const uint32_t wa = rowp[(t * 16 + g) * 4 + t4];
            const uint32_t wb = rowp[(t * 16 + g + 8) * 4 + t4];
            if constexpr (BITS == 8) {
                const uint32_t a[4] = {byte_h2<0x4140>(wa), byte_h2<0x4140>(wb), byte_h2<0x4342>(wa),
                                       byte_h2<0x4342>(wb)};
                mma16816_f16(acc[t], a, b0.x, b0.y);
                mma16816_f16(acc[t], a, b0.z, b0.w);
            } else {
                const uint32_t a[4] = {nib_h2(wa, 0), nib_h2(wb, 0), nib_h2(wa, 1), nib_h2(wb, 1)};
                mma16816_f16(acc[t], a, b0.x, b0.y);
                mma16816_f16(acc[t], a, b0.z, b0.w);
                const uint32_t a2[4] = {nib_h2(wa, 2), nib_h2(wb, 2), nib_h2(wa, 3), nib_h2(wb, 3)};
                mma16816_f16(acc[t], a2, b1.x, b1.y);
                mma16816_f16(acc[t], a2, b1.z, b1.w);
            }
        }
        __syncwarp();  // every lane has read the slot before it is refilled
        if (i + kMmaRing < my_rows) copy_row(i + kMmaRing);
        cp_async_commit();
    }
    cp_async_wait<0>();
    __syncthreads();  // the ring is free: row-group partials go over it

    // D fragment of tile t: (column g, vectors 2t4, 2t4+1), (column g+8, same)
#pragma unroll
    for (int t = 0; t < 4; ++t) {
        const int c = cg * 64 + t * 16 + g;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int m = 2 * t4 + h;
            red[(rg * 8 + m) * C + c] = acc[t][h] * down;
            red[(rg * 8 + m) * C + c + 8] = acc[t][2 + h] * down;
        }
    }
    __syncthreads();

    batched_reduce_scatter<kMaxBatch, NORM, true>(
        p, rbuf, &red_bar, S, rank, C, col0, M,
        [&](int m, int c) {
            float v = 0.f;
            for (int q = 0; q < RG; ++q) v += red[(q * 8 + m) * C + c];
            return v;
        },
        [&](int i) {
            float v = 0.f;
#pragma unroll
            for (int w = 0; w < kThreads / 32; ++w) v += wred[w][i];
            return v;
        });
}

struct DeviceInfo {
    int sms = 0;
};
constexpr int kMaxDevices = 64;
std::mutex g_info_mu;
DeviceInfo g_info[kMaxDevices];

int sm_count(int* out) {
    int dev = 0;
    VKC_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= kMaxDevices) return set_error(kErrUnsupported, "device ordinal %d", dev);
    std::lock_guard<std::mutex> lock(g_info_mu);
    if (g_info[dev].sms == 0)
        VKC_CUDA_TRY(cudaDeviceGetAttribute(&g_info[dev].sms, cudaDevAttrMultiProcessorCount, dev));
    *out = g_info[dev].sms;
    return kOk;
}

// Which single-vector GEMV kernel runs (vkc_set_gemv_plan), per host thread:
// 0 chooses per shape (the per-SM kernel in its half-SM shape where it
// applies, else the cluster kernel), 1 always the cluster
// split-K kernel, 2 the one-CTA-per-SM kernel in its full-SM shape wherever it
// can run, 3 the same in its half-SM shape, 4 chooses per shape with the
// full-SM shape.
thread_local int g_gemv_plan = 0;

constexpr size_t kSmMaxDynamicSmem = 220 * 1024;

// Shared memory of a per-SM CTA: the ring (NS streams x D rows x T threads
// x 16 bytes) and the staged activations (NS x K floats).
inline size_t sm_smem_bytes(int NS, int T, int D, int K) {
    return static_cast<size_t>(NS) * D * T * 16 + static_cast<size_t>(NS) * K * 4;
}

// Shape of a per-SM launch: threads and ring depth.  The half-SM shape (512
// threads) takes the deepest ring that keeps two CTAs on an SM; when even the
// shallowest does not fit beside the staged activations, the full-SM shape.
struct SmShape {
    int T = 0, D = 0;
    size_t smem = 0;
};

SmShape sm_shape(int NS, int K, bool half) {
    SmShape sh;
    if (half) {
        const int depths[] = {12, 8, 4};
        for (int d : depths) {
            if (NS == 2 && d > 4) continue;  // 64 KB ring for two streams
            const size_t b = sm_smem_bytes(NS, 512, d, K);
            if (b + kSmStaticSmem <= static_cast<size_t>(kSmHalfSmem)) {
                sh.T = 512;
                sh.D = d;
                sh.smem = b;
                return sh;
            }
        }
    }
    sh.T = 1024;
    sh.D = NS == 1 ? 8 : 4;
    sh.smem = sm_smem_bytes(NS, 1024, sh.D, K);
    return sh;
}

// The per-SM kernel serves a shape when every SM gets at least 16 outputs (at
// least one CTA per scale block), the staged activations fit in shared memory
// beside the ring, and the input is not a peer exchange (its per-element
// waits would be repeated by every CTA).
template <int BITS, int MODE>
bool sm_kernel_fits(const GemvParams& p, int sms, const SmShape& sh, bool force = false) {
    if (p.xslots || p.N % 2 != 0 || sh.smem > kSmMaxDynamicSmem) return false;
    // activations are read as 16-byte vectors
    auto aligned = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; };
    if (!aligned(p.x) || (MODE != kGemv && !aligned(p.gamma))) return false;
    if (BITS <= 8)
        for (int st = 0; st < (MODE == kSwiglu ? 2 : 1); ++st)
            if (!aligned(p.s[st]) || !aligned(p.z[st])) return false;
    // every CTA gets at least one pair of outputs, and at most T - 2 outputs
    if (BITS <= 8 && (p.N / kGroup > sms || (sms + p.N / kGroup - 1) / (p.N / kGroup) > kGroup / 2)) return false;
    if (BITS > 8 && (p.N / 2 < sms || p.N / sms > sh.T - 2)) return false;
    if (force || g_gemv_plan == 2 || g_gemv_plan == 3) return true;
    return p.N >= 16 * sms;
}

// Quantised weights on the per-SM kernel use integer dot products
// (vkc_set_gemv_int_dot), per host thread.
thread_local bool g_gemv_idp = true;

template <int BITS, int MODE, int T, int D, bool IDP>
int launch_sm_shape_k(const GemvParams& p, cudaStream_t stream, int sms, size_t smem) {
    const void* kern = reinterpret_cast<const void*>(gemv_sm_kernel<BITS, MODE, T, D, IDP>);
    if (int e = ensure_smem(kern, smem)) return e;
    if (T == 512) {
        // the largest shared-memory carveout, so that two CTAs fit on an SM
        // (a function attribute of each device's context)
        static bool carveout_set[kMaxDevices] = {};
        int dev = 0;
        VKC_CUDA_TRY(cudaGetDevice(&dev));
        if (dev < 0 || dev >= kMaxDevices || !carveout_set[dev]) {
            VKC_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout,
                                              cudaSharedmemCarveoutMaxShared));
            if (dev >= 0 && dev < kMaxDevices) carveout_set[dev] = true;
        }
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(sms, 1, 1);
    cfg.blockDim = dim3(T, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attrs[2];
    cfg.attrs = attrs;
    cfg.numAttrs = launch_attrs(attrs, 1);
    VKC_CUDA_TRY(cudaLaunchKernelEx(&cfg, gemv_sm_kernel<BITS, MODE, T, D, IDP>, p));
    return kOk;
}

template <int BITS, int MODE, int T, int D>
int launch_sm_shape(const GemvParams& p, cudaStream_t stream, int sms, size_t smem) {
    if constexpr (BITS <= 8) {
        if (g_gemv_idp) return launch_sm_shape_k<BITS, MODE, T, D, true>(p, stream, sms, smem);
    }
    return launch_sm_shape_k<BITS, MODE, T, D, false>(p, stream, sms, smem);
}

template <int BITS, int MODE>
int launch_sm(const GemvParams& p0, cudaStream_t stream, int sms, const SmShape& sh) {
    constexpr int NS = MODE == kSwiglu ? 2 : 1;
    GemvParams p = p0;
    p.R = p.K / (128 / BITS);
    if (sh.T == 1024) return launch_sm_shape<BITS, MODE, 1024, NS == 1 ? 8 : 4>(p, stream, sms, sh.smem);
    if constexpr (NS == 1) {
        if (sh.D == 12) return launch_sm_shape<BITS, MODE, 512, 12>(p, stream, sms, sh.smem);
        if (sh.D == 8) return launch_sm_shape<BITS, MODE, 512, 8>(p, stream, sms, sh.smem);
    }
    return launch_sm_shape<BITS, MODE, 512, 4>(p, stream, sms, sh.smem);
}

template <int BITS, int MODE>
int launch_one(const GemvParams& p0, cudaStream_t stream) {
    constexpr int NS = MODE == kSwiglu ? 2 : 1;
    constexpr int KPC = 128 / BITS;
    GemvParams p = p0;
    p.R = p.K / KPC;
    int sms = 0;
    if (int e = sm_count(&sms)) return e;
    if (p.gather_dst) {
        // gathered outputs: the per-SM kernel
        const SmShape sh = sm_shape(NS, p.K, g_gemv_plan != 2 && g_gemv_plan != 4);
        if (!sm_kernel_fits<BITS, MODE>(p, sms, sh, true))
            return set_error(kErrUnsupported, "gathered GEMV: N=%d K=%d does not split over %d SMs", p.N, p.K, sms);
        return launch_sm<BITS, MODE>(p, stream, sms, sh);
    }
    if (g_gemv_plan != 1) {
        // automatic shape, as measured on B200 for every width: 512 threads
        // (the next launch primes its ring beside this one)
        const bool half = g_gemv_plan == 3 || g_gemv_plan == 0;
        const SmShape sh = sm_shape(NS, p.K, half);
        if (sm_kernel_fits<BITS, MODE>(p, sms, sh)) return launch_sm<BITS, MODE>(p, stream, sms, sh);
    }
    // Widest tile and smallest cluster that put at least two CTAs on every SM.
    int C = 32, S = 8;
    bool found = false;
    for (int cw = 256; cw >= 32 && !found; cw /= 2)
        for (int s = 1; s <= 8 && !found; s *= 2) {
            const long long ctas = static_cast<long long>((p.N + cw - 1) / cw) * s;
            if (ctas >= 2LL * sms) {
                C = cw;
                S = s;
                found = true;
            }
        }
    p.rows_cta = (p.R + S - 1) / S;
    while (S > 1 && (S - 1) * p.rows_cta >= p.R) {  // no empty ranks
        S /= 2;
        p.rows_cta = (p.R + S - 1) / S;
    }
    p.cols = C;
    p.rbuf_floats = (S * (NS * C + 4) + 3) / 4 * 4;
    const size_t rest = (static_cast<size_t>(p.rbuf_floats) + static_cast<size_t>(p.rows_cta) * NS * KPC) * sizeof(float);
    const long long ctas = static_cast<long long>(S) * ((p.N + C - 1) / C);
    const long long per_sm = (ctas + sms - 1) / sms;
    // Deep ring only if every CTA is still resident at once (static shared
    // memory and the per-CTA reservation take about 3 KB more).
    const bool deep = per_sm * (ring_bytes<true>() + rest + 3072) <= 227 * 1024 && per_sm <= kCtasPerSm;
    const size_t smem = (deep ? ring_bytes<true>() : ring_bytes<false>()) + rest;
    if (smem > 200 * 1024)
        return set_error(kErrUnsupported, "K=%d is too long for one launch (%zu bytes of staged activations)", p.K,
                         smem);
    auto go = [&](auto kern) -> int {
        if (smem > 40 * 1024)  // with the static part (about 3.3 KB), above 48 KB needs the opt-in
            if (int e = ensure_smem(reinterpret_cast<const void*>(kern), smem)) return e;
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(S, (p.N + C - 1) / C, 1);
        cfg.blockDim = dim3(kThreads, 1, 1);
        cfg.dynamicSmemBytes = smem;
        cfg.stream = stream;
        cudaLaunchAttribute attrs[2];
        cfg.attrs = attrs;
        cfg.numAttrs = launch_attrs(attrs, S);
        VKC_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, p));
        return kOk;
    };
    return deep ? go(gemv_kernel<BITS, MODE, true>) : go(gemv_kernel<BITS, MODE, false>);
}

template <int MODE>
int launch_mode(int bits, const GemvParams& p, cudaStream_t s) {
    switch (bits) {
        case 32: return launch_one<32, MODE>(p, s);
        case 16: return launch_one<16, MODE>(p, s);
        case 8: return launch_one<8, MODE>(p, s);
        case 4: return launch_one<4, MODE>(p, s);
    }
    return set_error(kErrArg, "unsupported weight width %d (expected 32, 16, 8 or 4)", bits);
}

template <int BITS, int M>
int launch_batched(const BatchParams& p0, bool norm, cudaStream_t stream) {
    constexpr int KPC = 128 / BITS;
    BatchParams p = p0;
    p.R = p.K / KPC;
    int sms = 0;
    if (int e = sm_count(&sms)) return e;
    // One wave: the most CTAs (C outputs x S-way split K, any S <= 8) that are
    // all resident at once, at two CTAs per SM (the kernel's register budget)
    // when their shared memory allows; wider tiles first on ties.
    auto rbuf_floats = [&](int cw, int s) {
        return (static_cast<size_t>(s) * (M * ((cw + s - 1) / s) + 2 * M) + 3) / 4 * 4;
    };
    auto smem_for = [&](int cw, int s) {
        const int rows = (p.R + s - 1) / s;
        return 32768 + (rbuf_floats(cw, s) + static_cast<size_t>(rows) * M * KPC) * 4;
    };
    int C = 32, S = 1;
    long long best = -1;
    for (int cw = 256; cw >= 32; cw /= 2)
        for (int s = 1; s <= 8; ++s) {
            const int rows = (p.R + s - 1) / s;
            if ((s - 1) * rows >= p.R) continue;  // no empty ranks
            const size_t sm = smem_for(cw, s);
            const int occ = 2 * (sm + 9 * 1024) <= 227 * 1024 ? 2 : 1;
            const long long ctas = static_cast<long long>((p.N + cw - 1) / cw) * s;
            if (ctas <= static_cast<long long>(occ) * sms && ctas > best) {
                best = ctas;
                C = cw;
                S = s;
            }
        }
    p.rows_cta = (p.R + S - 1) / S;
    p.cols = C;
    p.rbuf_floats = static_cast<int>(rbuf_floats(C, S));
    const size_t smem = smem_for(C, S);
    if (smem > 200 * 1024)
        return set_error(kErrUnsupported, "K=%d with %d vectors stages too many activations (%zu bytes)", p.K, M, smem);
    auto go = [&](auto kern) -> int {
        // dynamic + static shared memory above 48 KB needs the opt-in (the
        // static part is up to 9 KB here)
        if (smem > 36 * 1024)
            if (int e = ensure_smem(reinterpret_cast<const void*>(kern), smem)) return e;
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(S, (p.N + C - 1) / C, 1);
        cfg.blockDim = dim3(kThreads, 1, 1);
        cfg.dynamicSmemBytes = smem;
        cfg.stream = stream;
        cudaLaunchAttribute attrs[2];
        cfg.attrs = attrs;
        cfg.numAttrs = launch_attrs(attrs, S);
        VKC_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, p));
        return kOk;
    };
    return norm ? go(gemv_batched_kernel<BITS, M, true>) : go(gemv_batched_kernel<BITS, M, false>);
}

// Clusters of S CTAs of `func` with `smem` bytes each that can be resident at
// once (cached per device): cluster placement inside the GPCs, not the SM
// count, bounds one wave of a clustered launch.
int max_clusters(const void* func, int S, size_t smem, int* out) {
    struct Entry {
        int dev;
        const void* func;
        int S;
        size_t smem;
        int n;
    };
    static std::mutex mu;
    static std::vector<Entry> cache;
    int dev = 0;
    VKC_CUDA_TRY(cudaGetDevice(&dev));
    {
        std::lock_guard<std::mutex> lock(mu);
        for (const Entry& e : cache)
            if (e.dev == dev && e.func == func && e.S == S && e.smem == smem) {
                *out = e.n;
                return kOk;
            }
    }
    if (int e = ensure_smem(func, smem)) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(S, 1, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeClusterDimension;
    attr.val.clusterDim.x = S;
    attr.val.clusterDim.y = 1;
    attr.val.clusterDim.z = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    int n = 0;
    VKC_CUDA_TRY(cudaOccupancyMaxActiveClusters(&n, func, &cfg));
    std::lock_guard<std::mutex> lock(mu);
    cache.push_back({dev, func, S, smem, n});
    *out = n;
    return kOk;
}

template <int BITS>
int launch_batched_mma(const BatchParams& p0, int M, bool norm, cudaStream_t stream) {
    constexpr int KPC = 128 / BITS;
    constexpr int FRAG = 4 * (KPC / 16);
    BatchParams p = p0;
    p.R = p.K / KPC;
    int sms = 0;
    if (int e = sm_count(&sms)) return e;
    auto rbuf_floats = [&](int cw, int s) {
        return (static_cast<size_t>(s) * (kMaxBatch * ((cw + s - 1) / s) + 2 * kMaxBatch) + 3) / 4 * 4;
    };
    auto smem_for = [&](int cw, int s) {
        const size_t rows = static_cast<size_t>((p.R + s - 1) / s);
        return static_cast<size_t>(8 * kMmaRing * 64 * 16) + rbuf_floats(cw, s) * 4 + rows * 8 * 4 * FRAG * 4;
    };
    // one wave: the most CTAs whose clusters are all resident at once (as the
    // occupancy calculator places them), wider tiles first on ties
    const void* kern = norm ? reinterpret_cast<const void*>(gemv_batched_mma_kernel<BITS, true>)
                            : reinterpret_cast<const void*>(gemv_batched_mma_kernel<BITS, false>);
    int C = 64, S = 1;
    long long best = -1;
    for (int cw = 256; cw >= 64; cw /= 2) {
        if (p.N % cw) continue;
        for (int s = 1; s <= 8; ++s) {
            const int rows = (p.R + s - 1) / s;
            if ((s - 1) * rows >= p.R) continue;
            const size_t sm = smem_for(cw, s);
            if (sm > 200 * 1024) continue;
            const long long ctas = static_cast<long long>(p.N / cw) * s;
            if (ctas <= best || ctas > 2LL * sms) continue;
            int nc = 0;
            if (int e = max_clusters(kern, s, sm, &nc)) return e;
            if (ctas <= static_cast<long long>(nc) * s) {
                best = ctas;
                C = cw;
                S = s;
            }
        }
    }
    if (best < 0) return set_error(kErrUnsupported, "K=%d stages too many activations for a batched launch", p.K);
    p.rows_cta = (p.R + S - 1) / S;
    p.cols = C;
    p.rbuf_floats = static_cast<int>(rbuf_floats(C, S));
    const size_t smem = smem_for(C, S);
    auto go = [&](auto kern) -> int {
        if (int e = ensure_smem(reinterpret_cast<const void*>(kern), smem)) return e;
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(S, p.N / C, 1);
        cfg.blockDim = dim3(kThreads, 1, 1);
        cfg.dynamicSmemBytes = smem;
        cfg.stream = stream;
        cudaLaunchAttribute attrs[2];
        cfg.attrs = attrs;
        cfg.numAttrs = launch_attrs(attrs, S);
        VKC_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, p, M));
        return kOk;
    };
    return norm ? go(gemv_batched_mma_kernel<BITS, true>) : go(gemv_batched_mma_kernel<BITS, false>);
}

template <int BITS>
int launch_batched_m(const BatchParams& p, int M, bool norm, cudaStream_t s) {
    switch (M) {
        case 2: return launch_batched<BITS, 2>(p, norm, s);
        case 3: return launch_batched<BITS, 3>(p, norm, s);
        case 4: return launch_batched<BITS, 4>(p, norm, s);
        case 5: return launch_batched<BITS, 5>(p, norm, s);
        case 6: return launch_batched<BITS, 6>(p, norm, s);
        case 7: return launch_batched<BITS, 7>(p, norm, s);
        case 8: return launch_batched<BITS, 8>(p, norm, s);
    }
    return set_error(kErrArg, "M=%d vectors (expected 1..%d)", M, kMaxBatch);
}

// Quantised weights run on the tensor cores when N is a multiple of 64 (always,
// as their scale blocks are 256 outputs); fp16 / fp32 weights on the SIMT kernel.
int launch_batched_bits(int bits, const BatchParams& p, int M, bool norm, cudaStream_t s) {
    const bool use_mma = p.N % 64 == 0;
    switch (bits) {
        case 32: return launch_batched_m<32>(p, M, norm, s);
        case 16: return launch_batched_m<16>(p, M, norm, s);
        case 8: return use_mma ? launch_batched_mma<8>(p, M, norm, s) : launch_batched_m<8>(p, M, norm, s);
        case 4: return use_mma ? launch_batched_mma<4>(p, M, norm, s) : launch_batched_m<4>(p, M, norm, s);
    }
    return set_error(kErrArg, "unsupported weight width %d (expected 32, 16, 8 or 4)", bits);
}


// ---- Persistent decoder: every phase of every layer in one launch --------
// One CTA of kPsThreads threads per SM runs, per layer, the five phases of a
// decoder step -- the fused RMSNorm-QKV-RoPE projection with its KV-cache
// append, attention, the O projection with the residual add, RMSNorm-SwiGLU,
// the down projection with the residual add -- separated by grid-wide
// barriers instead of kernel boundaries.  Each GEMV phase is the per-SM
// kernel's body (all of K per CTA, balanced column ranges) and attention the
// two-warp-group token-slice body, so the arithmetic is that of the separate
// kernels.  A phase requests its weights (and attention the cache tiles of the
// tokens before the newest) before it waits at the barrier, so the weight
// stream of the next phase overlaps the end of the previous one on every SM.
//
// The barrier: an arrival counter in the program that only grows.  A CTA
// arrives (all its threads' stores made visible first: __syncthreads, then one
// fence and one atomic add by thread 0) once per phase; thread 0 waits until
// the counter reaches base + phases-so-far * CTAs with acquire loads, bounded
// by kGridWaitNs (on expiry it records kStatusGridTimeout and every later wait
// of the launch gives up at once).  `base` is the counter at the start of the
// launch, written by the previous launch's CTA 0 after its last barrier, so
// graphs replay without resetting anything.  All CTAs must be resident: the
// launch is cooperative.
constexpr int kPsThreads = 384;  // 12 warps: registers for the attention phase without spills
constexpr int kPsRing1 = 20;     // GEMV ring depth with one weight stream (120 KB per SM)
constexpr int kPsRing2 = 10;     // with two (SwiGLU)
// Ring rows (and attention sub-tiles per warp group) requested before a
// barrier wait: the wait's polls and the __syncthreads after it queue behind
// this SM's outstanding requests, so a phase primes only what bridges the
// barrier and requests the rest once it has passed.
constexpr int kPsPrime1 = 4;
constexpr int kPsPrime2 = 2;
constexpr int kPsAttnPrime = 1;
constexpr int kPsAttnSync = 8;  // named barrier of the attention phase's warp groups (they use 1 and 2)
constexpr uint32_t kStatusGridTimeout = 0x20u;
constexpr uint64_t kGridWaitNs = kPeerWaitNs;

struct DecodeLayer {
    GemvParams qkv, o, ffn, down;
    AttnParams att;
};

struct DecodeProgram {
    unsigned count;  // barrier arrivals, growing across launches
    unsigned base;   // the count at the start of the next launch
    int layers;
    int att_items;   // CTAs with an attention work item (n_kv * splits)
    size_t smem;     // dynamic shared memory of the launch
    int pad[2];
};
static_assert(sizeof(DecodeProgram) % 16 == 0, "layers follow the header");

__device__ __forceinline__ unsigned ld_relaxed_gpu(const unsigned* p) {
    unsigned v;
    asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Thread 0's wait for the counter to reach `target` (the caller synchronises
// its threads afterwards).
__device__ __forceinline__ void grid_spin(const DecodeProgram* prog, unsigned target) {
    const uint64_t deadline = globaltimer_ns() + kGridWaitNs;
    uint32_t it = 0;
    // relaxed polls; the fence below orders the phase's reads after them
    while (static_cast<int>(ld_relaxed_gpu(&prog->count) - target) < 0) {
        if ((++it & 63u) == 0) {
            if (*reinterpret_cast<volatile uint32_t*>(&g_status) & kStatusGridTimeout) break;
            if (globaltimer_ns() > deadline) {
                atomicOr(&g_status, kStatusGridTimeout);
                break;
            }
        }
    }
    asm volatile("fence.acq_rel.gpu;" ::: "memory");
}

template <int BITS, int G, int HD>
__global__ void __launch_bounds__(kPsThreads, 1) decode_program_kernel(DecodeProgram* prog, int pos) {
    extern __shared__ __align__(16) uint8_t smem[];
    // the parameters of this layer and the next: one word per thread is loaded
    // at the start of a layer and stored after its last phase, so no phase
    // waits for its parameters
    __shared__ DecodeLayer s_layer[2];
    __shared__ unsigned s_base;
    constexpr int kAttThreadsPs = 2 * kFaThreads;  // two warp groups
    constexpr int kWords = static_cast<int>(sizeof(DecodeLayer) / 4);
    static_assert(sizeof(DecodeLayer) % 4 == 0 && kWords <= kPsThreads, "one parameter word per thread");
    const int tid = threadIdx.x, cta = blockIdx.x, ctas = gridDim.x;
    const DecodeLayer* layers = reinterpret_cast<const DecodeLayer*>(prog + 1);
    const int L = prog->layers, att_items = prog->att_items;
    if (tid == 0) s_base = *reinterpret_cast<volatile unsigned*>(&prog->base);
    if (tid < kWords)
        reinterpret_cast<unsigned*>(&s_layer[0])[tid] = __ldcg(reinterpret_cast<const unsigned*>(&layers[0]) + tid);
    __syncthreads();
    const unsigned base = s_base;
    unsigned k = 0;  // barriers of this launch passed so far
    auto arrive = [&] {
        __syncthreads();
        if (tid == 0) {
            __threadfence();
            atomicAdd(&prog->count, 1u);
        }
        ++k;
    };
    auto wait_all = [&] {
        if (tid == 0) grid_spin(prog, base + k * static_cast<unsigned>(ctas));
        __syncthreads();
    };
    auto wait_att = [&] {
        if (tid == 0) grid_spin(prog, base + k * static_cast<unsigned>(ctas));
        part_sync<kPsAttnSync, kAttThreadsPs>();
    };
    auto gemv_phase = [&](const GemvParams& p, auto mode_tag, auto ring_tag) {
        constexpr int MODE = decltype(mode_tag)::value, D = decltype(ring_tag)::value;
        constexpr int PRIME = D == kPsRing1 ? kPsPrime1 : kPsPrime2;
        gemv_sm_body<BITS, MODE, kPsThreads, D, true, false, PRIME>(p, smem, cta, ctas, wait_all);
        arrive();
    };
    using One = std::integral_constant<int, kPsRing1>;
    using Two = std::integral_constant<int, kPsRing2>;
    for (int l = 0; l < L; ++l) {
        DecodeLayer& e = s_layer[l & 1];
        const unsigned next = l + 1 < L && tid < kWords
                                  ? __ldcg(reinterpret_cast<const unsigned*>(&layers[l + 1]) + tid)
                                  : 0u;
        if (tid == 0) {
            e.qkv.pos = pos;
            e.att.ctx = pos + 1;  // attention over tokens [0, pos]
            e.att.stable = pos;   // only this layer's QKV phase writes token pos
        }
        __syncthreads();
        gemv_phase(e.qkv, std::integral_constant<int, kRopePairs>(), One());
        if (cta < att_items) {
            if (tid < kAttThreadsPs)
                attention_fa_body<G, HD, kFaDeepStages, 1, 2, kPsAttnSync>(e.att, smem, cta % e.att.splits,
                                                                            cta / e.att.splits, wait_att);
        } else if (tid == 0) {
            grid_spin(prog, base + k * static_cast<unsigned>(ctas));
        }
        arrive();
        gemv_phase(e.o, std::integral_constant<int, kGemv>(), One());
        gemv_phase(e.ffn, std::integral_constant<int, kSwiglu>(), Two());
        gemv_phase(e.down, std::integral_constant<int, kGemv>(), One());
        if (l + 1 < L && tid < kWords) reinterpret_cast<unsigned*>(&s_layer[(l + 1) & 1])[tid] = next;
        __syncthreads();  // the next layer's block is complete before thread 0 sets its position
    }
    if (cta == 0 && tid == 0) {
        // every CTA has arrived k times: the next launch starts from here
        grid_spin(prog, base + k * static_cast<unsigned>(ctas));
        *reinterpret_cast<volatile unsigned*>(&prog->base) = base + k * static_cast<unsigned>(ctas);
        __threadfence();
    }
}

// Host side of the persistent decoder.
size_t decode_program_header_bytes(int layers) {
    const size_t b = sizeof(DecodeProgram) + static_cast<size_t>(layers) * sizeof(DecodeLayer);
    return (b + 255) & ~static_cast<size_t>(255);
}

size_t decode_gemv_smem(int NS, int K) { return sm_smem_bytes(NS, kPsThreads, NS == 1 ? kPsRing1 : kPsRing2, K); }

// Whether one GEMV phase of the persistent decoder can run the per-SM body:
// the conditions of sm_kernel_fits for kPsThreads threads.
bool decode_gemv_fits(int N, int K, int sms, bool quant) {
    if (N % 2 != 0) return false;
    if (quant) {
        const int nb = N / kGroup;
        if (N % kGroup != 0 || nb > sms || (sms + nb - 1) / nb > kGroup / 2) return false;
        // columns per CTA (at most 256 / floor(sms / nb)) leave every thread a row group
        const int per = sms / nb;
        if ((kGroup + per - 1) / per > kPsThreads) return false;
    } else if (N / 2 < sms || N / sms > kPsThreads - 2) {
        return false;
    }
    return K > 0;
}

// Per-SM attention split of the persistent decoder for a cache of ctx_cap
// tokens over `ctas` CTAs (the standalone per-SM plan, sized for the whole
// cache: CTAs whose range lies past the current context have no tokens).
void decode_attention_split(int n_kv, int hd, int ctx_cap, int ctas, int* splits, int* tpc) {
    const int tt = 8192 / hd;
    const int per_head = ctas / n_kv > 0 ? ctas / n_kv : 1;
    int t = (ctx_cap + per_head - 1) / per_head;
    t = ((t + 15) / 16) * 16;
    if (t < 2 * tt) t = 2 * tt;
    *tpc = t;
    *splits = (ctx_cap + t - 1) / t;
}

size_t decode_attention_ws_bytes(const vkc_decode_dims& d, int ctas) {
    int splits = 0, tpc = 0;
    decode_attention_split(d.n_kv, d.head_dim, d.ctx_cap, ctas, &splits, &tpc);
    return 256 + static_cast<size_t>(d.n_q) * splits * (d.head_dim + 4) * sizeof(float);
}

size_t decode_attention_smem(int hd) {
    return hd == 64 ? static_cast<size_t>(kFaDeepStages) * MmaGeo<64>::SU * 16 + MmaGeo<64>::q_bytes
                    : static_cast<size_t>(kFaDeepStages) * MmaGeo<128>::SU * 16 + MmaGeo<128>::q_bytes;
}

size_t decode_program_smem(const vkc_decode_dims& d) {
    size_t s = decode_attention_smem(d.head_dim);
    const int q_rows = d.n_q * d.head_dim;
    s = std::max(s, decode_gemv_smem(1, d.hidden));  // QKV
    s = std::max(s, decode_gemv_smem(1, q_rows));    // O
    s = std::max(s, decode_gemv_smem(2, d.hidden));  // gate/up
    s = std::max(s, decode_gemv_smem(1, d.inter));   // down
    return s;
}

int decode_check_dims(const vkc_decode_dims* d, int sms) {
    if (!d) return set_error(kErrArg, "null decoder dimensions");
    if (d->layers <= 0) return set_error(kErrArg, "layers=%d must be positive", d->layers);
    if (d->bits != 4) return set_error(kErrUnsupported, "the persistent decoder runs 4-bit weights (bits=%d)", d->bits);
    if (d->head_dim != 128 && d->head_dim != 64)
        return set_error(kErrUnsupported, "persistent decoder: head_dim %d (64 or 128)", d->head_dim);
    if (d->n_kv <= 0 || d->n_q != 4 * d->n_kv)
        return set_error(kErrUnsupported, "persistent decoder: 4 query heads per KV head (n_q=%d n_kv=%d)", d->n_q,
                         d->n_kv);
    if (d->ctx_cap <= 0) return set_error(kErrArg, "ctx_cap=%d must be positive", d->ctx_cap);
    const int q_rows = d->n_q * d->head_dim, kv_rows = d->n_kv * d->head_dim;
    const int kpc = 128 / d->bits;
    if (d->hidden % kpc || q_rows % kpc || d->inter % kpc)
        return set_error(kErrArg, "hidden, heads*head_dim and inter must be multiples of %d", kpc);
    if (!decode_gemv_fits(q_rows + 2 * kv_rows, d->hidden, sms, true) || !decode_gemv_fits(d->hidden, q_rows, sms, true) ||
        !decode_gemv_fits(d->inter, d->hidden, sms, true) || !decode_gemv_fits(d->hidden, d->inter, sms, true))
        return set_error(kErrUnsupported, "persistent decoder: a projection does not split over %d SMs", sms);
    int splits = 0, tpc = 0;
    decode_attention_split(d->n_kv, d->head_dim, d->ctx_cap, sms, &splits, &tpc);
    if (d->n_kv * splits > sms) return set_error(kErrUnsupported, "persistent decoder: attention needs more CTAs than SMs");
    if (decode_program_smem(*d) + 1024 > 227u * 1024)
        return set_error(kErrUnsupported, "persistent decoder: shared memory exceeds an SM's");
    return kOk;
}

int check_common(int bits, int N, int K, const void* w, const float* s, const float* z, const float* x,
                 const float* y, const float* gamma) {
    if (bits != 32 && bits != 16 && bits != 8 && bits != 4)
        return set_error(kErrArg, "unsupported weight width %d (expected 32, 16, 8 or 4)", bits);
    const int kpc = 128 / bits;
    if (N <= 0 || K <= 0) return set_error(kErrArg, "N=%d and K=%d must be positive", N, K);
    if (K % kpc != 0) return set_error(kErrArg, "K=%d must be a multiple of %d for %d-bit weights", K, kpc, bits);
    if (!w || !x || !y) return set_error(kErrArg, "null weight, input or output pointer");
    auto misaligned = [](const void* q) { return reinterpret_cast<uintptr_t>(q) % 16 != 0; };
    if (misaligned(w) || misaligned(x) || (gamma && misaligned(gamma)))
        return set_error(kErrArg, "weights, x and gamma must be 16-byte aligned");
    if (bits <= 8) {
        if (N % kGroup != 0) return set_error(kErrArg, "N=%d must be a multiple of 256 for quantised weights", N);
        if (!s || !z) return set_error(kErrArg, "quantised weights need scale and zero arrays");
        if (misaligned(s) || misaligned(z)) return set_error(kErrArg, "scale and zero must be 16-byte aligned");
    }
    return kOk;
}

}  // namespace
}  // namespace vkc

using namespace vkc;

extern "C" {

int vkc_gemv(int bits, const void* w, const float* scale, const float* zero, const float* x, float* y, int N,
             int K, void* stream) {
    if (int e = check_common(bits, N, K, w, scale, zero, x, y, nullptr)) return e;
    GemvParams p = {};
    p.w[0] = static_cast<const uint8_t*>(w);
    p.s[0] = scale;
    p.z[0] = zero;
    p.x = x;
    p.y = y;
    p.N = N;
    p.K = K;
    return launch_mode<kGemv>(bits, p, static_cast<cudaStream_t>(stream));
}

int vkc_gemv_residual(int bits, const void* w, const float* scale, const float* zero, const float* x,
                      const float* residual, float* y, int N, int K, void* stream) {
    if (!residual) return set_error(kErrArg, "null residual");
    if (int e = check_common(bits, N, K, w, scale, zero, x, y, nullptr)) return e;
    GemvParams p = {};
    p.w[0] = static_cast<const uint8_t*>(w);
    p.s[0] = scale;
    p.z[0] = zero;
    p.x = x;
    p.y = y;
    p.residual = residual;
    p.N = N;
    p.K = K;
    return launch_mode<kGemv>(bits, p, static_cast<cudaStream_t>(stream));
}

int vkc_gemv_peer(int bits, const void* w, const float* scale, const float* zero, const float* x,
                  void* const* slots, int rank, int world, int N, int K, void* stream) {
    if (!slots) return set_error(kErrArg, "null peer slots");
    if (world < 1 || rank < 0 || rank >= world) return set_error(kErrArg, "rank %d of world %d", rank, world);
    float dummy = 0.f;  // y is unused: check_common only wants a non-null output
    if (int e = check_common(bits, N, K, w, scale, zero, x, &dummy, nullptr)) return e;
    GemvParams p = {};
    p.w[0] = static_cast<const uint8_t*>(w);
    p.s[0] = scale;
    p.z[0] = zero;
    p.x = x;
    p.N = N;
    p.K = K;
    p.peer_slots = reinterpret_cast<unsigned long long* const*>(slots);
    p.prank = rank;
    p.pworld = world;
    return launch_mode<kGemv>(bits, p, static_cast<cudaStream_t>(stream));
}

static int set_peer_input(GemvParams& p, const vkc_peer_input* in) {
    if (!in) return kOk;
    if (!in->slots) return set_error(kErrArg, "null peer-input slots");
    if (reinterpret_cast<uintptr_t>(in->slots) % 8 != 0) return set_error(kErrArg, "peer-input slots must be 8-byte aligned");
    if (in->world < 1 || in->rank < 0 || in->rank >= in->world)
        return set_error(kErrArg, "peer input: rank %d of world %d", in->rank, in->world);
    p.xslots = static_cast<const unsigned long long*>(in->slots);
    p.xsave = in->save;
    p.prank = in->rank;
    p.pworld = in->world;
    return kOk;
}

static int rope_kv_impl(int bits, const void* w, const float* scale, const float* zero, const float* x,
                        const float* gamma, const float* theta, float* y, int N, int K, float eps, int rms_dim,
                        int pos, int head_dim, int q_rows, int kv_rows, int kv_layout, void* kcache, void* vcache,
                        int ctx_cap, void* stream, const vkc_peer_input* in) {
    if (!gamma || !theta || !kcache || !vcache) return set_error(kErrArg, "null gamma, theta or cache");
    if (int e = check_common(bits, N, K, w, scale, zero, x, y, gamma)) return e;
    if (rms_dim <= 0) return set_error(kErrArg, "rms_dim=%d must be positive", rms_dim);
    if (head_dim <= 0 || head_dim % 8 != 0)
        return set_error(kErrArg, "head_dim=%d must be a positive multiple of 8", head_dim);
    if (q_rows < 0 || kv_rows <= 0 || q_rows % head_dim || kv_rows % head_dim || q_rows + 2 * kv_rows != N)
        return set_error(kErrArg, "rows must be q_rows + 2*kv_rows = N in whole heads (q=%d kv=%d N=%d)", q_rows,
                         kv_rows, N);
    if (pos < 0 || pos >= ctx_cap) return set_error(kErrArg, "pos=%d outside the cache of %d tokens", pos, ctx_cap);
    if (kv_layout != 0 && kv_layout != 1) return set_error(kErrArg, "kv_layout=%d (expected 0 or 1)", kv_layout);
    GemvParams p = {};
    p.w[0] = static_cast<const uint8_t*>(w);
    p.s[0] = scale;
    p.z[0] = zero;
    p.x = x;
    p.gamma = gamma;
    p.theta = theta;
    p.y = y;
    p.N = N;
    p.K = K;
    p.eps = eps;
    p.inv_dim = 1.0f / static_cast<float>(rms_dim);
    p.pos = pos;
    p.head_dim = head_dim;
    p.rot_rows = q_rows + kv_rows;  // Q and K rotate, V does not
    p.kcache = static_cast<uint16_t*>(kcache);
    p.vcache = static_cast<uint16_t*>(vcache);
    p.q_rows = q_rows;
    p.kv_rows = kv_rows;
    p.kv_interleave = kv_layout;
    p.ctx_cap = ctx_cap;
    if (int e = set_peer_input(p, in)) return e;
    return launch_mode<kRopePairs>(bits, p, static_cast<cudaStream_t>(stream));
}

int vkc_rmsnorm_gemv_rope_kv(int bits, const void* w, const float* scale, const float* zero, const float* x,
                             const float* gamma, const float* theta, float* y, int N, int K, float eps,
                             int rms_dim, int pos, int head_dim, int q_rows, int kv_rows, int kv_layout,
                             void* kcache, void* vcache, int ctx_cap, void* stream) {
    return rope_kv_impl(bits, w, scale, zero, x, gamma, theta, y, N, K, eps, rms_dim, pos, head_dim, q_rows, kv_rows,
                        kv_layout, kcache, vcache, ctx_cap, stream, nullptr);
}

int vkc_rmsnorm_gemv_rope_kv_peer(int bits, const void* w, const float* scale, const float* zero,
                                  const float* x_base, const vkc_peer_input* in, const float* gamma,
                                  const float* theta, float* y, int N, int K, float eps, int rms_dim, int pos,
                                  int head_dim, int q_rows, int kv_rows, int kv_layout, void* kcache,
                                  void* vcache, int ctx_cap, void* stream) {
    if (!in) return set_error(kErrArg, "null peer input");
    return rope_kv_impl(bits, w, scale, zero, x_base, gamma, theta, y, N, K, eps, rms_dim, pos, head_dim, q_rows,
                        kv_rows, kv_layout, kcache, vcache, ctx_cap, stream, in);
}

int vkc_rmsnorm_gemv_gather(int bits, const void* w, const float* scale, const float* zero, const float* x,
                            const float* gamma, void* const* dsts, int rank, int world, int offset, int N, int K,
                            float eps, int rms_dim, void* stream) {
    if (!gamma || !dsts) return set_error(kErrArg, "null gamma or destinations");
    if (world < 1 || rank < 0 || rank >= world) return set_error(kErrArg, "rank %d of world %d", rank, world);
    if (offset < 0) return set_error(kErrArg, "offset %d", offset);
    if (rms_dim <= 0) return set_error(kErrArg, "rms_dim=%d must be positive", rms_dim);
    float dummy = 0.f;  // y is unused: check_common only wants a non-null output
    if (int e = check_common(bits, N, K, w, scale, zero, x, &dummy, gamma)) return e;
    GemvParams p = {};
    p.w[0] = static_cast<const uint8_t*>(w);
    p.s[0] = scale;
    p.z[0] = zero;
    p.x = x;
    p.gamma = gamma;
    p.N = N;
    p.K = K;
    p.eps = eps;
    p.inv_dim = 1.0f / static_cast<float>(rms_dim);
    p.gather_dst = reinterpret_cast<float* const*>(dsts);
    p.gather_off = offset;
    p.prank = rank;
    p.pworld = world;
    return launch_mode<kRms>(bits, p, static_cast<cudaStream_t>(stream));
}

int vkc_rmsnorm_gemv(int bits, const void* w, const float* scale, const float* zero, const float* x,
                     const float* gamma, float* y, int N, int K, float eps, int rms_dim, void* stream) {
    if (!gamma) return set_error(kErrArg, "null gamma");
    if (int e = check_common(bits, N, K, w, scale, zero, x, y, gamma)) return e;
    if (rms_dim <= 0) return set_error(kErrArg, "rms_dim=%d must be positive", rms_dim);
    GemvParams p = {};
    p.w[0] = static_cast<const uint8_t*>(w);
    p.s[0] = scale;
    p.z[0] = zero;
    p.x = x;
    p.gamma = gamma;
    p.y = y;
    p.N = N;
    p.K = K;
    p.eps = eps;
    p.inv_dim = 1.0f / static_cast<float>(rms_dim);
    return launch_mode<kRms>(bits, p, static_cast<cudaStream_t>(stream));
}

int vkc_rmsnorm_gemv_rope(int bits, const void* w, const float* scale, const float* zero, const float* x,
                          const float* gamma, const float* theta, float* y, int N, int K, float eps,
                          int rms_dim, int pos, int rope_mode, int head_dim, int rot_rows, void* stream) {
    if (!gamma || !theta) return set_error(kErrArg, "null gamma or theta");
    if (int e = check_common(bits, N, K, w, scale, zero, x, y, gamma)) return e;
    if (rms_dim <= 0) return set_error(kErrArg, "rms_dim=%d must be positive", rms_dim);
    GemvParams p = {};
    p.w[0] = static_cast<const uint8_t*>(w);
    p.s[0] = scale;
    p.z[0] = zero;
    p.x = x;
    p.gamma = gamma;
    p.theta = theta;
    p.y = y;
    p.N = N;
    p.K = K;
    p.eps = eps;
    p.inv_dim = 1.0f / static_cast<float>(rms_dim);
    p.pos = pos;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (rope_mode == 0) return launch_mode<kRopeRef>(bits, p, s);
    if (rope_mode != 1) return set_error(kErrArg, "rope_mode=%d (expected 0 or 1)", rope_mode);
    if (head_dim <= 0 || head_dim % 2 != 0)
        return set_error(kErrArg, "head_dim=%d must be a positive even number", head_dim);
    if (rot_rows < 0 || rot_rows > N || rot_rows % 2 != 0)
        return set_error(kErrArg, "rot_rows=%d must be even and within [0, N]", rot_rows);
    p.head_dim = head_dim;
    p.rot_rows = rot_rows;
    return launch_mode<kRopePairs>(bits, p, s);
}

static int swiglu_impl(int bits, const void* wg, const float* sg, const float* zg, const void* wu, const float* su,
                       const float* zu, const float* x, const float* gamma, float* h, int N, int K, float eps,
                       int rms_dim, void* stream, const vkc_peer_input* in) {
    if (!gamma) return set_error(kErrArg, "null gamma");
    if (int e = check_common(bits, N, K, wg, sg, zg, x, h, gamma)) return e;
    if (int e = check_common(bits, N, K, wu, su, zu, x, h, gamma)) return e;
    if (rms_dim <= 0) return set_error(kErrArg, "rms_dim=%d must be positive", rms_dim);
    GemvParams p = {};
    p.w[0] = static_cast<const uint8_t*>(wg);
    p.w[1] = static_cast<const uint8_t*>(wu);
    p.s[0] = sg;
    p.z[0] = zg;
    p.s[1] = su;
    p.z[1] = zu;
    p.x = x;
    p.gamma = gamma;
    p.y = h;
    p.N = N;
    p.K = K;
    p.eps = eps;
    p.inv_dim = 1.0f / static_cast<float>(rms_dim);
    if (int e = set_peer_input(p, in)) return e;
    return launch_mode<kSwiglu>(bits, p, static_cast<cudaStream_t>(stream));
}

int vkc_rmsnorm_swiglu(int bits, const void* wg, const float* sg, const float* zg, const void* wu,
                       const float* su, const float* zu, const float* x, const float* gamma, float* h, int N,
                       int K, float eps, int rms_dim, void* stream) {
    return swiglu_impl(bits, wg, sg, zg, wu, su, zu, x, gamma, h, N, K, eps, rms_dim, stream, nullptr);
}

int vkc_rmsnorm_swiglu_peer(int bits, const void* wg, const float* sg, const float* zg, const void* wu,
                            const float* su, const float* zu, const float* x_base, const vkc_peer_input* in,
                            const float* gamma, float* h, int N, int K, float eps, int rms_dim, void* stream) {
    if (!in) return set_error(kErrArg, "null peer input");
    return swiglu_impl(bits, wg, sg, zg, wu, su, zu, x_base, gamma, h, N, K, eps, rms_dim, stream, in);
}

int vkc_gemv_batched(int bits, const void* w, const float* scale, const float* zero, const float* x, float* y,
                     int M, int N, int K, void* stream) {
    if (M < 1 || M > kMaxBatch) return set_error(kErrArg, "M=%d vectors (expected 1..%d)", M, kMaxBatch);
    if (M == 1) return vkc_gemv(bits, w, scale, zero, x, y, N, K, stream);
    if (int e = check_common(bits, N, K, w, scale, zero, x, y, nullptr)) return e;
    if (K % 4 != 0) return set_error(kErrArg, "K=%d must be a multiple of 4 for batched rows", K);
    BatchParams p = {};
    p.w = static_cast<const uint8_t*>(w);
    p.s = scale;
    p.z = zero;
    p.x = x;
    p.y = y;
    p.N = N;
    p.K = K;
    return launch_batched_bits(bits, p, M, false, static_cast<cudaStream_t>(stream));
}

int vkc_rmsnorm_gemv_batched(int bits, const void* w, const float* scale, const float* zero, const float* x,
                             const float* gamma, float* y, int M, int N, int K, float eps, int rms_dim,
                             void* stream) {
    if (M < 1 || M > kMaxBatch) return set_error(kErrArg, "M=%d vectors (expected 1..%d)", M, kMaxBatch);
    if (M == 1) return vkc_rmsnorm_gemv(bits, w, scale, zero, x, gamma, y, N, K, eps, rms_dim, stream);
    if (!gamma) return set_error(kErrArg, "null gamma");
    if (int e = check_common(bits, N, K, w, scale, zero, x, y, gamma)) return e;
    if (rms_dim <= 0) return set_error(kErrArg, "rms_dim=%d must be positive", rms_dim);
    BatchParams p = {};
    p.w = static_cast<const uint8_t*>(w);
    p.s = scale;
    p.z = zero;
    p.x = x;
    p.gamma = gamma;
    p.y = y;
    p.N = N;
    p.K = K;
    p.eps = eps;
    p.inv_dim = 1.0f / static_cast<float>(rms_dim);
    return launch_batched_bits(bits, p, M, true, static_cast<cudaStream_t>(stream));
}

// Status word of the current device (bits: kStatus*).  Reading waits for the
// device; `clear` resets it.

size_t vkc_decode_program_bytes(const vkc_decode_dims* dims) {
    int sms = 0;
    if (!dims || sm_count(&sms) != kOk) return 0;
    return decode_program_header_bytes(dims->layers) + decode_attention_ws_bytes(*dims, sms);
}

int vkc_decode_program_build(const vkc_decode_dims* dims, const vkc_decode_layer* layers,
                             const vkc_decode_buffers* bufs, const float* theta, void* program, size_t program_bytes,
                             void* stream) {
    int sms = 0;
    if (int e = sm_count(&sms)) return e;
    if (int e = decode_check_dims(dims, sms)) return e;
    const vkc_decode_dims& d = *dims;
    if (!layers || !bufs || !theta || !program) return set_error(kErrArg, "null decoder argument");
    if (!bufs->x || !bufs->x_mid || !bufs->qkv || !bufs->attn || !bufs->h) return set_error(kErrArg, "null decoder buffer");
    if (reinterpret_cast<uintptr_t>(program) % 256 != 0) return set_error(kErrArg, "program must be 256-byte aligned");
    const size_t need = vkc_decode_program_bytes(dims);
    if (program_bytes < need) return set_error(kErrArg, "decoder program holds %zu bytes, needs %zu", program_bytes, need);
    const int hd = d.head_dim, q_rows = d.n_q * hd, kv_rows = d.n_kv * hd, nqkv = q_rows + 2 * kv_rows;
    const int kpc = 128 / d.bits;
    const size_t hbytes = decode_program_header_bytes(d.layers);
    char* ws = static_cast<char*>(program) + hbytes;
    int splits = 0, tpc = 0;
    decode_attention_split(d.n_kv, hd, d.ctx_cap, sms, &splits, &tpc);
    std::vector<char> host(hbytes, 0);
    DecodeProgram* prog = reinterpret_cast<DecodeProgram*>(host.data());
    prog->layers = d.layers;
    prog->att_items = d.n_kv * splits;
    prog->smem = decode_program_smem(d);
    DecodeLayer* out = reinterpret_cast<DecodeLayer*>(prog + 1);
    auto base_params = [&](const void* w, const float* s, const float* z, int N, int K) {
        GemvParams p = {};
        p.w[0] = static_cast<const uint8_t*>(w);
        p.s[0] = s;
        p.z[0] = z;
        p.N = N;
        p.K = K;
        p.R = K / kpc;
        return p;
    };
    for (int l = 0; l < d.layers; ++l) {
        const vkc_decode_layer& w = layers[l];
        if (int e = check_common(d.bits, nqkv, d.hidden, w.qkv, w.qkv_scale, w.qkv_zero, bufs->x, bufs->qkv,
                                 w.gamma_attn))
            return e;
        if (int e = check_common(d.bits, d.hidden, q_rows, w.o, w.o_scale, w.o_zero, bufs->attn, bufs->x_mid, nullptr))
            return e;
        if (int e = check_common(d.bits, d.inter, d.hidden, w.gate, w.gate_scale, w.gate_zero, bufs->x_mid, bufs->h,
                                 w.gamma_ffn))
            return e;
        if (int e = check_common(d.bits, d.inter, d.hidden, w.up, w.up_scale, w.up_zero, bufs->x_mid, bufs->h,
                                 w.gamma_ffn))
            return e;
        if (int e = check_common(d.bits, d.hidden, d.inter, w.down, w.down_scale, w.down_zero, bufs->h, bufs->x, nullptr))
            return e;
        if (!w.gamma_attn || !w.gamma_ffn || !w.kcache || !w.vcache) return set_error(kErrArg, "null layer %d field", l);
        if ((reinterpret_cast<uintptr_t>(w.kcache) | reinterpret_cast<uintptr_t>(w.vcache)) % 16 != 0)
            return set_error(kErrArg, "layer %d: caches must be 16-byte aligned", l);
        DecodeLayer& L = out[l];
        // RMSNorm-QKV-RoPE with the KV append, rows [Q | K0 V0 | K1 V1 | ...]
        L.qkv = base_params(w.qkv, w.qkv_scale, w.qkv_zero, nqkv, d.hidden);
        L.qkv.x = bufs->x;
        L.qkv.gamma = w.gamma_attn;
        L.qkv.theta = theta;
        L.qkv.y = bufs->qkv;
        L.qkv.eps = d.eps;
        L.qkv.inv_dim = 1.0f / static_cast<float>(d.hidden);
        L.qkv.head_dim = hd;
        L.qkv.rot_rows = q_rows + kv_rows;
        L.qkv.kcache = static_cast<uint16_t*>(w.kcache);
        L.qkv.vcache = static_cast<uint16_t*>(w.vcache);
        L.qkv.q_rows = q_rows;
        L.qkv.kv_rows = kv_rows;
        L.qkv.kv_interleave = 1;
        L.qkv.ctx_cap = d.ctx_cap;
        // attention over the layer's cache
        AttnParams& a = L.att;
        a.q = bufs->qkv;
        a.q_bits = 32;
        a.kc = static_cast<const uint4*>(w.kcache);
        a.vc = static_cast<const uint4*>(w.vcache);
        a.out = bufs->attn;
        a.tickets = reinterpret_cast<unsigned*>(ws);
        a.ws = reinterpret_cast<float*>(ws + 256);
        a.n_q = d.n_q;
        a.n_kv = d.n_kv;
        a.hd = hd;
        a.ctx = d.ctx_cap;
        a.splits = splits;
        a.tpc = tpc;
        a.ctx_cap = d.ctx_cap;
        a.tt = 8192 / hd;
        a.scale_log2 = kLog2e / sqrtf(static_cast<float>(hd));
        a.pitch = hd + 4;
        a.smem = static_cast<int>(prog->smem);
        a.pre_max = kPsAttnPrime;
        // O projection + residual: x' = x + O attn
        L.o = base_params(w.o, w.o_scale, w.o_zero, d.hidden, q_rows);
        L.o.x = bufs->attn;
        L.o.residual = bufs->x;
        L.o.y = bufs->x_mid;
        // RMSNorm-SwiGLU: h = silu(gate x'') * up x''
        L.ffn = base_params(w.gate, w.gate_scale, w.gate_zero, d.inter, d.hidden);
        L.ffn.w[1] = static_cast<const uint8_t*>(w.up);
        L.ffn.s[1] = w.up_scale;
        L.ffn.z[1] = w.up_zero;
        L.ffn.x = bufs->x_mid;
        L.ffn.gamma = w.gamma_ffn;
        L.ffn.y = bufs->h;
        L.ffn.eps = d.eps;
        L.ffn.inv_dim = 1.0f / static_cast<float>(d.hidden);
        // down projection + residual: x = x' + down h
        L.down = base_params(w.down, w.down_scale, w.down_zero, d.hidden, d.inter);
        L.down.x = bufs->h;
        L.down.residual = bufs->x_mid;
        L.down.y = bufs->x;
    }
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    VKC_CUDA_TRY(cudaMemcpyAsync(program, host.data(), hbytes, cudaMemcpyHostToDevice, s));
    VKC_CUDA_TRY(cudaMemsetAsync(ws, 0, 256, s));  // attention tickets
    VKC_CUDA_TRY(cudaStreamSynchronize(s));        // the host copy goes out of scope
    return kOk;
}

int vkc_decode_program_run(const vkc_decode_dims* dims, void* program, int pos, void* stream) {
    int sms = 0;
    if (int e = sm_count(&sms)) return e;
    if (int e = decode_check_dims(dims, sms)) return e;
    if (!program) return set_error(kErrArg, "null decoder program");
    if (pos < 0 || pos >= dims->ctx_cap) return set_error(kErrArg, "pos=%d outside the cache of %d tokens", pos, dims->ctx_cap);
    const size_t smem = decode_program_smem(*dims);
    const void* kern = dims->head_dim == 128 ? reinterpret_cast<const void*>(decode_program_kernel<4, 4, 128>)
                                             : reinterpret_cast<const void*>(decode_program_kernel<4, 4, 64>);
    if (int e = ensure_smem(kern, smem)) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(sms, 1, 1);
    cfg.blockDim = dim3(kPsThreads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = static_cast<cudaStream_t>(stream);
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeCooperative;  // every CTA resident: the phases wait on one another
    attr.val.cooperative = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    DecodeProgram* prog = static_cast<DecodeProgram*>(program);
    if (dims->head_dim == 128)
        VKC_CUDA_TRY(cudaLaunchKernelEx(&cfg, decode_program_kernel<4, 4, 128>, prog, pos));
    else
        VKC_CUDA_TRY(cudaLaunchKernelEx(&cfg, decode_program_kernel<4, 4, 64>, prog, pos));
    return kOk;
}

int vkc_set_gemv_plan(int plan) {
    if (plan < 0 || plan > 4) return set_error(kErrArg, "GEMV plan %d (expected 0 to 4)", plan);
    g_gemv_plan = plan;
    return kOk;
}
int vkc_get_gemv_plan(void) { return g_gemv_plan; }

void vkc_set_gemv_int_dot(int enable) { g_gemv_idp = enable != 0; }
int vkc_get_gemv_int_dot(void) { return g_gemv_idp ? 1 : 0; }

void vkc_wait_limits(uint64_t* peer_ns, uint64_t* cluster_ns) {
    if (peer_ns) *peer_ns = kPeerWaitNs;
    if (cluster_ns) *cluster_ns = kClusterWaitNs;
}

int vkc_device_status(unsigned* status, int clear) {
    VKC_CUDA_TRY(cudaDeviceSynchronize());
    uint32_t v = 0;
    VKC_CUDA_TRY(cudaMemcpyFromSymbol(&v, g_status, sizeof v));
    if (clear) {
        const uint32_t zero = 0;
        VKC_CUDA_TRY(cudaMemcpyToSymbol(g_status, &zero, sizeof zero));
    }
    *status = v;
    return kOk;
}

}  // extern "C"
