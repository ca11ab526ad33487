// GEMV family for sm_100a: GEMV, RmsNorm-GEMV, RmsNorm-GEMV-Rope and
// RmsNorm-SwiGLU over fp32 / fp16 / int8 / int4 weights stored in vk-compute's
// 16-byte chunk layout (src/data.c:198-222).
//
// Weight layout (the reference's, unchanged): chunk row r holds k in
// [r*KPC, (r+1)*KPC) (KPC = 128/bits) of every output column j as one 16-byte
// chunk at byte (r*N + j)*16, so a chunk row is a contiguous N*16-byte stream.
// Quantised weights carry fp32 scale s and zero z per (k, 256-output block b),
// block-major at b*K + k (src/data.c:122-124), dequantised as q*s - z
// (shader/GEMV-INT8.comp:107).
//
// Work decomposition (stream-K).  Outputs form tiles of 256 columns (one
// scale block); a unit is one chunk row of one tile, a contiguous 4 KB
// segment.  The tiles x R units, tile-major, are split into equal contiguous
// ranges over persistent CTAs (two per SM), so every CTA streams the same
// number of bytes whatever N and K are.  A CTA's range covers whole tiles and
// at most two partial tiles; a partial tile's contributors write their partial
// sums to a workspace and the last to finish (atomic ticket) adds them in
// contributor order and runs the epilogue, so results are deterministic.
//
// Pipeline.  One producer warp streams each stage -- up to 16 KB of weight
// rows plus the stage's slice of x, gamma, scale and zero -- into a ring of
// shared-memory slots with cp.async.bulk completing on mbarriers; the weight
// copies of the first ring's worth of stages are issued before
// griddepcontrol.wait, so under programmatic dependent launch they overlap the
// previous kernel.  Eight consumer warps own one column each per lane.
//
// Arithmetic.  Per stage the consumers fold the per-(k, b) scale into the
// activation, x'_k = x_k * gamma_k * s_kb, and accumulate the zero-point term
// c_b = sum_k x_k gamma_k z_kb and sum x^2, so
// y_j = inv_rms * (sum_k x'_k q_kj - c_b): one conversion and one fused
// multiply-add per weight.  Codes become floats exactly by OR-ing them into the
// mantissa of 2^23 and subtracting 2^23 (int4 nibbles keep their bit position;
// x' carries the matching power of two); pairs of weights use the packed
// f32x2 add and FMA.
#include "vkc_common.cuh"

#include <cuda_fp16.h>

#include <mutex>

namespace vkc {
namespace {

constexpr int kCols = 256;             // outputs per tile (one scale group)
constexpr int kConsumerWarps = 8;
constexpr int kConsumers = 32 * kConsumerWarps;
constexpr int kThreads = kConsumers + 32;  // + one producer warp
constexpr int kCtasPerSm = 2;
constexpr int kStageWeightBytes = 16384;   // weight bytes per pipeline stage
constexpr int kStages = 5;                 // ring depth
constexpr int kBarBytes = 128;             // mbarrier block at the start of smem
constexpr uint32_t kConsumerBar = 1;       // named barrier id of the consumer warps

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
    int N, K, R, tiles;
    int max_slots;
    float eps;
    float inv_dim;  // 1 / RMS divisor
    int pos;
    int head_dim;
    int rot_rows;
    uint32_t* status;   // workspace header word
    uint32_t* tickets;  // [tiles]
    float* partial;     // [tiles][max_slots][NS*kCols + 4]
};

template <int BITS, int NS>
struct Geometry {
    static constexpr int KPC = 128 / BITS;                       // k per chunk
    static constexpr int SR = kStageWeightBytes / (NS * kCols * 16);  // chunk rows per stage
    static constexpr int SA = SR * KPC;                           // activations per stage
    static constexpr int kActArrays = 2 + 3 * NS;                 // x, gamma, s[NS], z[NS], x'[NS]
    static constexpr int kSlotBytes = ((NS * SR * kCols * 16 + SA * 4 * kActArrays) + 127) / 128 * 128;
    static constexpr int kSmemBytes = kBarBytes + kStages * kSlotBytes;
    // Offsets inside a slot.
    static constexpr int kOffX = NS * SR * kCols * 16;
    static constexpr int kOffGamma = kOffX + SA * 4;
    static constexpr int kOffS = kOffGamma + SA * 4;
    static constexpr int kOffZ = kOffS + NS * SA * 4;
    static constexpr int kOffXp = kOffZ + NS * SA * 4;
};

// CTA owning unit u when T units are split into P equal contiguous ranges
// [floor(c*T/P), floor((c+1)*T/P)).
__host__ __device__ __forceinline__ int cta_of(long long u, long long T, int P) {
    return static_cast<int>(((u + 1) * P - 1) / T);
}

// Walks a CTA's unit range in pipeline stages that never cross a tile.
struct StageWalk {
    long long u, u1;
    int R, SR;
    __device__ bool next(int& t, int& r, int& nr) {
        if (u >= u1) return false;
        t = static_cast<int>(u / R);
        r = static_cast<int>(u % R);
        long long n = SR;
        if (n > R - r) n = R - r;
        if (n > u1 - u) n = u1 - u;
        nr = static_cast<int>(n);
        u += n;
        return true;
    }
};

// Power-of-two pre-scale of an int4 position inside a 32-bit word.  Nibbles
// 0-4 are decoded in place (bit offsets 0..16); nibbles 5-7 after a 12-bit
// shift (offsets 8, 12, 16).
__device__ __forceinline__ float int4_prescale(int t) {
    const int i = t & 7;
    const int e = i < 5 ? 4 * i : 4 * (i - 3);
    return __int_as_float((127 - e) << 23);
}

constexpr uint32_t kMagic = 0x4B000000u;  // 2^23
__device__ __forceinline__ float magic_f(uint32_t bits) { return __uint_as_float(kMagic | bits); }

// One chunk of KPC weights of one column against the staged activations xs
// (16-byte aligned shared memory); accumulates into the pair accumulators.
template <int BITS>
__device__ __forceinline__ void chunk_fma(const uint4 c, const float* __restrict__ xs, uint64_t& a0,
                                          uint64_t& a1) {
    const float4* x4 = reinterpret_cast<const float4*>(xs);
    if constexpr (BITS == 32) {
        const float4 v = x4[0];
        a0 = f2_fma(f2_pack(v.x, v.y), f2_pack(__uint_as_float(c.x), __uint_as_float(c.y)), a0);
        a1 = f2_fma(f2_pack(v.z, v.w), f2_pack(__uint_as_float(c.z), __uint_as_float(c.w)), a1);
    } else if constexpr (BITS == 16) {
        const uint32_t wd[4] = {c.x, c.y, c.z, c.w};
#pragma unroll
        for (int q = 0; q < 2; ++q) {
            const float4 v = x4[q];
            const float2 w0 = __half22float2(*reinterpret_cast<const __half2*>(&wd[2 * q]));
            const float2 w1 = __half22float2(*reinterpret_cast<const __half2*>(&wd[2 * q + 1]));
            a0 = f2_fma(f2_pack(v.x, v.y), f2_pack(w0.x, w0.y), a0);
            a1 = f2_fma(f2_pack(v.z, v.w), f2_pack(w1.x, w1.y), a1);
        }
    } else if constexpr (BITS == 8) {
        const uint32_t wd[4] = {c.x, c.y, c.z, c.w};
        const uint64_t neg = f2_pack(-8388608.0f, -8388608.0f);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const float4 v = x4[q];
            const uint32_t w = wd[q];
            const uint64_t p01 = f2_add(f2_pack(__uint_as_float(__byte_perm(w, kMagic, 0x7540)),
                                                __uint_as_float(__byte_perm(w, kMagic, 0x7541))),
                                        neg);
            const uint64_t p23 = f2_add(f2_pack(__uint_as_float(__byte_perm(w, kMagic, 0x7542)),
                                                __uint_as_float(__byte_perm(w, kMagic, 0x7543))),
                                        neg);
            a0 = f2_fma(f2_pack(v.x, v.y), p01, a0);
            a1 = f2_fma(f2_pack(v.z, v.w), p23, a1);
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
            const uint64_t p01 = f2_add(f2_pack(magic_f(w & 0xFu), magic_f(w & 0xF0u)), neg);
            const uint64_t p23 = f2_add(f2_pack(magic_f(w & 0xF00u), magic_f(w & 0xF000u)), neg);
            const uint64_t p45 = f2_add(f2_pack(magic_f(w & 0xF0000u), magic_f(h & 0xF00u)), neg);
            const uint64_t p67 = f2_add(f2_pack(magic_f(h & 0xF000u), magic_f(h & 0xF0000u)), neg);
            a0 = f2_fma(f2_pack(v0.x, v0.y), p01, a0);
            a1 = f2_fma(f2_pack(v0.z, v0.w), p23, a1);
            a0 = f2_fma(f2_pack(v1.x, v1.y), p45, a0);
            a1 = f2_fma(f2_pack(v1.z, v1.w), p67, a1);
        }
    }
}

// Epilogue for one output column: RMS scale, zero-point constant and the
// operator's activation.  Called by all consumer threads of a warp together.
template <int MODE, int NS, bool kQuant, bool kNorm>
__device__ __forceinline__ void finalize(const GemvParams& p, int t, int col, const float (&acc)[NS],
                                         const float (&tot)[3]) {
    float v[NS];
    const float inv = kNorm ? 1.0f / sqrtf(tot[0] * p.inv_dim + p.eps) : 1.0f;
#pragma unroll
    for (int st = 0; st < NS; ++st) v[st] = ((kQuant ? acc[st] - tot[1 + st] : acc[st])) * inv;
    const int j = t * kCols + col;
    float out = v[0];
    if constexpr (MODE == kRopeRef) {
        // shader/RmsNorm-GEMV-Rope-FP16.comp:76-89, reproduced as written.
        const int c = j % kCols;
        if (c < 64) {
            float sa, ca;
            sincosf(static_cast<float>(p.pos) * p.theta[c / 2], &sa, &ca);
            out = (c & 1) == 0 ? out * ca - p.theta[c + 1] * sa : p.theta[c - 1] * sa + out * ca;
        }
    } else if constexpr (MODE == kRopePairs) {
        const float partner = __shfl_xor_sync(0xffffffffu, out, 1);
        if (j < p.rot_rows) {
            float sa, ca;
            sincosf(static_cast<float>(p.pos) * p.theta[(j % p.head_dim) >> 1], &sa, &ca);
            out = (j & 1) == 0 ? out * ca - partner * sa : partner * sa + out * ca;
        }
    } else if constexpr (MODE == kSwiglu) {
        // shader/RmsNorm-swiglu-ffn-FP16.comp:86-87
        out = out / (1.0f + exp2f(-out * 1.44269504f)) * v[1];
    }
    if (j < p.N) p.y[j] = out;
}

template <int BITS, int MODE>
__global__ void __launch_bounds__(kThreads, kCtasPerSm) gemv_kernel(const GemvParams p) {
    constexpr int NS = MODE == kSwiglu ? 2 : 1;
    using G = Geometry<BITS, NS>;
    constexpr int KPC = G::KPC, SR = G::SR, SA = G::SA;
    constexpr bool kQuant = BITS <= 8;
    constexpr bool kNorm = MODE != kGemv;

    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ float red[kConsumerWarps][3];
    __shared__ int s_last;

    const uint32_t bar0 = smem_addr(smem);
    auto full_bar = [&](int i) { return bar0 + 8u * i; };
    auto empty_bar = [&](int i) { return bar0 + 8u * (kStages + i); };
    uint8_t* slots = smem + kBarBytes;

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int P = gridDim.x, cta = blockIdx.x;
    const long long T = static_cast<long long>(p.tiles) * p.R;
    const long long u0 = cta * T / P, u1 = (cta + 1) * T / P;

    if (tid == 0) {
        for (int i = 0; i < kStages; ++i) {
            mbar_init(full_bar(i), 1);
            mbar_init(empty_bar(i), kConsumerWarps);
        }
        mbar_init_fence();
    }
    __syncthreads();
    pdl_launch_dependents();

    if (warp == kConsumerWarps) {
        // ------------------------------ producer ------------------------------
        if (lane != 0) return;
        const uint64_t pol = l2_evict_first();
        auto stage_bytes = [&](int t, int nr) -> uint32_t {
            const int ncols = min(kCols, p.N - t * kCols);
            return static_cast<uint32_t>(NS * nr * ncols * 16 +
                                         nr * KPC * 4 * (1 + (kNorm ? 1 : 0) + (kQuant ? 2 * NS : 0)));
        };
        auto copy_weights = [&](int slot, int t, int r, int nr) {
            const int ncols = min(kCols, p.N - t * kCols);
            const uint32_t dst = smem_addr(slots + slot * G::kSlotBytes);
#pragma unroll
            for (int st = 0; st < NS; ++st)
                for (int i = 0; i < nr; ++i)
                    bulk_g2s(dst + static_cast<uint32_t>((st * SR + i) * kCols * 16),
                             p.w[st] + (static_cast<size_t>(r + i) * p.N + static_cast<size_t>(t) * kCols) * 16,
                             static_cast<uint32_t>(ncols * 16), full_bar(slot), pol);
        };
        auto copy_acts = [&](int slot, int t, int r, int nr) {
            const uint32_t base = smem_addr(slots + slot * G::kSlotBytes);
            const size_t k0 = static_cast<size_t>(r) * KPC;
            const uint32_t n = static_cast<uint32_t>(nr * KPC * 4);
            bulk_g2s(base + G::kOffX, p.x + k0, n, full_bar(slot));
            if (kNorm) bulk_g2s(base + G::kOffGamma, p.gamma + k0, n, full_bar(slot));
            if (kQuant) {
                const size_t sb = static_cast<size_t>(t) * p.K + k0;
#pragma unroll
                for (int st = 0; st < NS; ++st) {
                    bulk_g2s(base + G::kOffS + st * SA * 4, p.s[st] + sb, n, full_bar(slot));
                    bulk_g2s(base + G::kOffZ + st * SA * 4, p.z[st] + sb, n, full_bar(slot));
                }
            }
        };
        StageWalk walk{u0, u1, p.R, SR};
        StageWalk acts = walk;
        int t, r, nr, g = 0;
        // Weights of the first ring's worth of stages do not depend on the
        // previous kernel: issue them before waiting for it.
        while (g < kStages && walk.next(t, r, nr)) {
            mbar_arrive_expect_tx(full_bar(g), stage_bytes(t, nr));
            copy_weights(g, t, r, nr);
            ++g;
        }
        pdl_wait();
        for (int i = 0; i < g; ++i) {
            acts.next(t, r, nr);
            copy_acts(i, t, r, nr);
        }
        while (walk.next(t, r, nr)) {
            const int slot = g % kStages;
            if (!mbar_wait(empty_bar(slot), static_cast<uint32_t>((g / kStages - 1) & 1))) {
                atomicOr(p.status, kStatusProducerTimeout);
                return;
            }
            mbar_arrive_expect_tx(full_bar(slot), stage_bytes(t, nr));
            copy_weights(slot, t, r, nr);
            copy_acts(slot, t, r, nr);
            ++g;
        }
        return;
    }

    // ------------------------------ consumers -------------------------------
    pdl_wait();
    const int col = tid;  // 0..255
    StageWalk walk{u0, u1, p.R, SR};
    int t, r, nr;
    bool have = walk.next(t, r, nr);
    int frag_r0 = r;
    uint64_t acc[NS][2];
    float ss = 0.f, cz[NS];
#pragma unroll
    for (int st = 0; st < NS; ++st) {
        acc[st][0] = acc[st][1] = 0ull;
        cz[st] = 0.f;
    }
    bool ok = true;
    for (int g = 0; have; ++g) {
        const int slot = g % kStages;
        uint8_t* sp = slots + slot * G::kSlotBytes;
        if (!mbar_wait(full_bar(slot), static_cast<uint32_t>((g / kStages) & 1))) {
            if (ok && lane == 0) atomicOr(p.status, kStatusConsumerTimeout);
            ok = false;
        }
        // Fold scales into the activations of this stage.
        const float* ax = reinterpret_cast<const float*>(sp + G::kOffX);
        const float* ag = reinterpret_cast<const float*>(sp + G::kOffGamma);
        float* xp = reinterpret_cast<float*>(sp + G::kOffXp);
        const int n = nr * KPC;
        for (int i = tid; i < n; i += kConsumers) {
            const float xv = ax[i];
            float xg = xv;
            if constexpr (kNorm) {
                ss = fmaf(xv, xv, ss);
                xg = xv * ag[i];
            }
#pragma unroll
            for (int st = 0; st < NS; ++st) {
                float v = xg;
                if constexpr (kQuant) {
                    const float* as = reinterpret_cast<const float*>(sp + G::kOffS) + st * SA;
                    const float* az = reinterpret_cast<const float*>(sp + G::kOffZ) + st * SA;
                    v = xg * as[i];
                    cz[st] = fmaf(xg, az[i], cz[st]);
                }
                if constexpr (BITS == 4) v *= int4_prescale(i);
                xp[st * SA + i] = v;
            }
        }
        named_sync(kConsumerBar, kConsumers);
        const uint4* wsm = reinterpret_cast<const uint4*>(sp);
        for (int i = 0; i < nr; ++i) {
#pragma unroll
            for (int st = 0; st < NS; ++st)
                chunk_fma<BITS>(wsm[(st * SR + i) * kCols + col], xp + st * SA + i * KPC, acc[st][0],
                                acc[st][1]);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(empty_bar(slot));

        int t2 = -1, r2 = 0, nr2 = 0;
        const bool have2 = walk.next(t2, r2, nr2);
        if (!have2 || t2 != t) {
            // -------- end of this CTA's fragment of tile t: rows [frag_r0, r+nr)
            float a[NS];
#pragma unroll
            for (int st = 0; st < NS; ++st) {
                const float2 x0 = f2_unpack(acc[st][0]), x1 = f2_unpack(acc[st][1]);
                a[st] = (x0.x + x0.y) + (x1.x + x1.y);
                acc[st][0] = acc[st][1] = 0ull;
            }
            float sc[3] = {warp_sum(ss), warp_sum(cz[0]), NS == 2 ? warp_sum(cz[NS - 1]) : 0.f};
            if (lane == 0) {
                red[warp][0] = sc[0];
                red[warp][1] = sc[1];
                red[warp][2] = sc[2];
            }
            named_sync(kConsumerBar, kConsumers);
            float tot[3] = {0.f, 0.f, 0.f};
#pragma unroll
            for (int w = 0; w < kConsumerWarps; ++w) {
                tot[0] += red[w][0];
                tot[1] += red[w][1];
                tot[2] += red[w][2];
            }
            ss = 0.f;
#pragma unroll
            for (int st = 0; st < NS; ++st) cz[st] = 0.f;
            if (frag_r0 == 0 && r + nr == p.R) {
                finalize<MODE, NS, kQuant, kNorm>(p, t, col, a, tot);
            } else {
                const long long tu = static_cast<long long>(t) * p.R;
                const int first = cta_of(tu, T, P);
                const int nslots = cta_of(tu + p.R - 1, T, P) - first + 1;
                const size_t stride = NS * kCols + 4;
                float* part = p.partial + (static_cast<size_t>(t) * p.max_slots + (cta - first)) * stride;
#pragma unroll
                for (int st = 0; st < NS; ++st) part[st * kCols + col] = a[st];
                if (tid < 3) part[NS * kCols + tid] = tot[tid];
                __threadfence();
                named_sync(kConsumerBar, kConsumers);
                if (tid == 0) s_last = atomicAdd(p.tickets + t, 1u) == static_cast<uint32_t>(nslots - 1);
                named_sync(kConsumerBar, kConsumers);
                if (s_last) {
                    __threadfence();
                    float sa[NS], st3[3] = {0.f, 0.f, 0.f};
#pragma unroll
                    for (int st = 0; st < NS; ++st) sa[st] = 0.f;
                    const float* base = p.partial + static_cast<size_t>(t) * p.max_slots * stride;
                    for (int q = 0; q < nslots; ++q) {
                        const float* pq = base + q * stride;
#pragma unroll
                        for (int st = 0; st < NS; ++st) sa[st] += __ldcg(pq + st * kCols + col);
                        st3[0] += __ldcg(pq + NS * kCols);
                        st3[1] += __ldcg(pq + NS * kCols + 1);
                        st3[2] += __ldcg(pq + NS * kCols + 2);
                    }
                    finalize<MODE, NS, kQuant, kNorm>(p, t, col, sa, st3);
                    if (tid == 0) atomicExch(p.tickets + t, 0u);
                }
            }
            frag_r0 = r2;
        }
        t = t2;
        r = r2;
        nr = nr2;
        have = have2;
    }
}

struct DeviceInfo {
    int sms = 0;
};
std::mutex g_info_mu;
DeviceInfo g_info[64];

int sm_count(int* out) {
    int dev = 0;
    VKC_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) return set_error(kErrUnsupported, "device ordinal %d", dev);
    std::lock_guard<std::mutex> lock(g_info_mu);
    if (g_info[dev].sms == 0)
        VKC_CUDA_TRY(cudaDeviceGetAttribute(&g_info[dev].sms, cudaDevAttrMultiProcessorCount, dev));
    *out = g_info[dev].sms;
    return kOk;
}

template <int BITS, int MODE>
int launch_one(const GemvParams& p0, cudaStream_t stream) {
    constexpr int NS = MODE == kSwiglu ? 2 : 1;
    using G = Geometry<BITS, NS>;
    GemvParams p = p0;
    p.R = p.K / G::KPC;
    p.tiles = (p.N + kCols - 1) / kCols;
    const long long T = static_cast<long long>(p.tiles) * p.R;
    int sms = 0;
    if (int e = sm_count(&sms)) return e;
    const int P = static_cast<int>(T < static_cast<long long>(kCtasPerSm) * sms ? T : kCtasPerSm * sms);
    int max_slots = 1;
    for (int t = 0; t < p.tiles; ++t) {
        const long long tu = static_cast<long long>(t) * p.R;
        const int n = cta_of(tu + p.R - 1, T, P) - cta_of(tu, T, P) + 1;
        max_slots = n > max_slots ? n : max_slots;
    }
    p.max_slots = max_slots;
    const size_t ticket_bytes = (static_cast<size_t>(p.tiles) * 4 + 255) / 256 * 256;
    const size_t part_bytes = static_cast<size_t>(p.tiles) * max_slots * (NS * kCols + 4) * sizeof(float);
    void* ws = nullptr;
    if (int e = device_workspace(kWorkspaceHeader + ticket_bytes + part_bytes, &ws, stream)) return e;
    p.status = static_cast<uint32_t*>(ws);
    p.tickets = reinterpret_cast<uint32_t*>(static_cast<char*>(ws) + kWorkspaceHeader);
    p.partial = reinterpret_cast<float*>(static_cast<char*>(ws) + kWorkspaceHeader + ticket_bytes);

    auto kern = gemv_kernel<BITS, MODE>;
    static bool attr_set = false;  // one instantiation per (BITS, MODE)
    if (!attr_set) {
        VKC_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, G::kSmemBytes));
        attr_set = true;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(P, 1, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = G::kSmemBytes;
    cfg.stream = stream;
    cudaLaunchAttribute attrs[2];
    cfg.attrs = attrs;
    cfg.numAttrs = launch_attrs(attrs, 1);
    VKC_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, p));
    return kOk;
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
        if (N % kCols != 0) return set_error(kErrArg, "N=%d must be a multiple of 256 for quantised weights", N);
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

int vkc_rmsnorm_swiglu(int bits, const void* wg, const float* sg, const float* zg, const void* wu,
                       const float* su, const float* zu, const float* x, const float* gamma, float* h, int N,
                       int K, float eps, int rms_dim, void* stream) {
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
    return launch_mode<kSwiglu>(bits, p, static_cast<cudaStream_t>(stream));
}

// Status word of the library workspace on the current device: bit 0 a
// producer wait, bit 1 a consumer wait gave up.  Reading waits for the
// device; `clear` resets it.
int vkc_device_status(unsigned* status, int clear) {
    void* ws = nullptr;
    if (int e = device_workspace(kWorkspaceHeader, &ws, nullptr)) return e;
    VKC_CUDA_TRY(cudaDeviceSynchronize());
    uint32_t v = 0;
    VKC_CUDA_TRY(cudaMemcpy(&v, ws, sizeof v, cudaMemcpyDeviceToHost));
    if (clear) VKC_CUDA_TRY(cudaMemset(ws, 0, sizeof v));
    *status = v;
    return kOk;
}

}  // extern "C"
