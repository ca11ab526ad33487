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
// Decomposition.  A CTA (256 threads = 2 column warps x 4 k warps) owns 64
// consecutive outputs and RS chunk rows; S CTAs of one thread-block cluster
// split K between them and are reduced through distributed shared memory by
// the cluster's rank-0 CTA, which also runs the epilogue.  Every lane streams
// its column's chunks with 16-byte loads, two batches in flight, so one warp
// reads 512 contiguous bytes per chunk row.
//
// Arithmetic.  The per-(k, b) scale is folded into the staged activation,
// x'_k = x_k * gamma_k * s_kb, and the zero point into one constant per block,
// c_b = sum_k x_k gamma_k z_kb, so y_j = inv_rms * (sum_k x'_k q_kj - c_b): one
// conversion and one fused multiply-add per weight.  Codes become floats
// exactly by OR-ing them into the mantissa of 2^23 and subtracting 2^23
// (int4 nibbles keep their bit position; the staged x' carries the matching
// power of two).  inv_rms is a scalar applied in the epilogue, so no CTA waits
// for the RMS reduction before streaming weights.
#include "vkc_common.cuh"

#include <cooperative_groups.h>
#include <cuda_fp16.h>

#include <algorithm>

namespace cg = cooperative_groups;

namespace vkc {
namespace {

constexpr int kThreads = 256;
constexpr int kColWarps = 2;
constexpr int kKWarps = 4;
constexpr int kTileCols = 32 * kColWarps;  // outputs per CTA
constexpr int kGroup = 256;                // outputs per scale group

enum Mode : int {
    kGemv = 0,       // shader/GEMV-*.comp
    kRms = 1,        // shader/RmsNorm-GEMV-*.comp
    kRopeRef = 2,    // shader/RmsNorm-GEMV-Rope-*.comp epilogue as written
    kRopePairs = 3,  // rotary embedding on adjacent pairs per head
    kSwiglu = 4,     // shader/RmsNorm-swiglu-ffn-*.comp
};

struct GemvParams {
    const uint4* w[2];
    const float* s[2];
    const float* z[2];
    const float* x;
    const float* gamma;
    const float* theta;
    float* y;
    int N, K;
    int R;         // chunk rows, K / KPC
    int rows_cta;  // chunk rows per CTA (RS)
    int rows_warp; // chunk rows per k warp (RW)
    float eps;
    float inv_dim;  // 1 / RMS divisor
    int pos;
    int head_dim;
    int rot_rows;
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
__device__ __forceinline__ void chunk_fma(const uint4 c, const float* __restrict__ xs,
                                          uint64_t& a0, uint64_t& a1) {
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

template <int BITS, int MODE>
__global__ void __launch_bounds__(kThreads, 2) gemv_kernel(const GemvParams p) {
    constexpr int KPC = 128 / BITS;
    constexpr int NS = MODE == kSwiglu ? 2 : 1;
    constexpr bool kQuant = BITS <= 8;
    constexpr bool kNorm = MODE != kGemv;
    constexpr int U = NS == 2 ? 4 : 8;  // chunks per batch per stream

    extern __shared__ __align__(16) float xs_smem[];  // [NS][rows_cta * KPC]
    __shared__ float red[NS][kKWarps][kTileCols];
    __shared__ float part[NS * kTileCols + 4];  // CTA partials + {ss, cz0, cz1}
    __shared__ float wsum[kThreads / 32][3];

    cg::cluster_group cluster = cg::this_cluster();
    const int rank = static_cast<int>(cluster.block_rank());
    const int S = static_cast<int>(cluster.num_blocks());
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int wc = warp % kColWarps, wk = warp / kColWarps;
    const int tile0 = blockIdx.y * kTileCols;
    const int col = tile0 + wc * 32 + lane;
    const bool col_ok = col < p.N;
    const int RS = p.rows_cta;
    const int r_cta = rank * RS;
    const int r_cta_end = min(r_cta + RS, p.R);
    const int r_begin = min(r_cta + wk * p.rows_warp, r_cta_end);
    const int r_end = min(r_begin + p.rows_warp, r_cta_end);
    const int xs_stride = RS * KPC;

    // Weights never depend on an earlier kernel: let the next kernel in the
    // stream start its own weight stream while this one finishes.
    pdl_launch_dependents();

    uint4 ba[NS][U], bb[NS][U];
    auto load = [&](uint4 (&b)[NS][U], int r0) {
#pragma unroll
        for (int st = 0; st < NS; ++st)
#pragma unroll
            for (int i = 0; i < U; ++i) {
                const int r = r0 + i;
                if (r < r_end && col_ok)
                    b[st][i] = ld_stream(p.w[st] + static_cast<size_t>(r) * p.N + col);
                else
                    b[st][i] = make_uint4(0u, 0u, 0u, 0u);
            }
    };
    uint64_t acc[NS][2];
#pragma unroll
    for (int st = 0; st < NS; ++st) acc[st][0] = acc[st][1] = 0ull;
    auto compute = [&](const uint4 (&b)[NS][U], int r0) {
#pragma unroll
        for (int i = 0; i < U; ++i) {
            const int r = r0 + i;
            if (r < r_end) {
#pragma unroll
                for (int st = 0; st < NS; ++st)
                    chunk_fma<BITS>(b[st][i], xs_smem + st * xs_stride + (r - r_cta) * KPC,
                                    acc[st][0], acc[st][1]);
            }
        }
    };

    if (r_begin < r_end) load(ba, r_begin);

    // Activations may come from the previous kernel.
    pdl_wait();

    // Stage x' for this CTA's k range; accumulate sum(x^2) and the zero-point
    // constants over the same range.
    const int k0 = r_cta * KPC;
    const int nk = max(0, min(xs_stride, p.K - k0));
    const size_t sblk = static_cast<size_t>(tile0 / kGroup) * p.K;
    float ss = 0.f, cz[2] = {0.f, 0.f};
    for (int kk = tid; kk < nk; kk += kThreads) {
        const int k = k0 + kk;
        const float xv = p.x[k];
        float xg = xv;
        if constexpr (kNorm) {
            ss = fmaf(xv, xv, ss);
            xg = xv * p.gamma[k];
        }
#pragma unroll
        for (int st = 0; st < NS; ++st) {
            float v = xg;
            if constexpr (kQuant) {
                v = xg * p.s[st][sblk + k];
                cz[st] = fmaf(xg, p.z[st][sblk + k], cz[st]);
            }
            if constexpr (BITS == 4) v *= int4_prescale(kk);
            xs_smem[st * xs_stride + kk] = v;
        }
    }
    ss = warp_sum(ss);
    cz[0] = warp_sum(cz[0]);
    cz[1] = warp_sum(cz[1]);
    if (lane == 0) {
        wsum[warp][0] = ss;
        wsum[warp][1] = cz[0];
        wsum[warp][2] = cz[1];
    }
    __syncthreads();

    // Stream the k warp's chunk rows, two batches in flight.
    for (int r = r_begin; r < r_end;) {
        if (r + U < r_end) load(bb, r + U);
        compute(ba, r);
        r += U;
        if (r >= r_end) break;
        if (r + U < r_end) load(ba, r + U);
        compute(bb, r);
        r += U;
    }

#pragma unroll
    for (int st = 0; st < NS; ++st) {
        const float2 a = f2_unpack(acc[st][0]);
        const float2 b = f2_unpack(acc[st][1]);
        red[st][wk][wc * 32 + lane] = (a.x + a.y) + (b.x + b.y);
    }
    __syncthreads();
    if (tid < NS * kTileCols) {
        const int st = tid / kTileCols, c = tid % kTileCols;
        float v = 0.f;
#pragma unroll
        for (int q = 0; q < kKWarps; ++q) v += red[st][q][c];
        part[tid] = v;
    }
    if (tid < 3) {
        float v = 0.f;
#pragma unroll
        for (int q = 0; q < kThreads / 32; ++q) v += wsum[q][tid];
        part[NS * kTileCols + tid] = v;
    }
    cluster.sync();

    if (rank == 0 && tid < kTileCols) {
        float v[NS], czs[NS], ssum = 0.f;
#pragma unroll
        for (int st = 0; st < NS; ++st) v[st] = czs[st] = 0.f;
        for (int q = 0; q < S; ++q) {
            const float* rp = cluster.map_shared_rank(part, q);
#pragma unroll
            for (int st = 0; st < NS; ++st) {
                v[st] += rp[st * kTileCols + tid];
                czs[st] += rp[NS * kTileCols + 1 + st];
            }
            ssum += rp[NS * kTileCols];
        }
        float inv = 1.f;
        if constexpr (kNorm) inv = 1.0f / sqrtf(ssum * p.inv_dim + p.eps);
#pragma unroll
        for (int st = 0; st < NS; ++st) {
            if constexpr (kQuant) v[st] -= czs[st];
            v[st] *= inv;
        }
        const int j = tile0 + tid;
        float out = v[0];
        if constexpr (MODE == kRopeRef) {
            // shader/RmsNorm-GEMV-Rope-FP16.comp:76-89, reproduced as written.
            const int c = j % kGroup;
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
    // Keep this CTA's shared memory alive until rank 0 has read it.
    cluster.sync();
}

template <int BITS, int MODE>
int launch_one(const GemvParams& p0, cudaStream_t stream) {
    constexpr int KPC = 128 / BITS;
    constexpr int NS = MODE == kSwiglu ? 2 : 1;
    GemvParams p = p0;
    p.R = p.K / KPC;
    // Rows per k warp: 16 by default; more when K is long (cluster <= 8),
    // fewer when the grid would not cover the GPU twice.
    const int tiles = (p.N + kTileCols - 1) / kTileCols;
    int rw = 16;
    while ((p.R + kKWarps * rw - 1) / (kKWarps * rw) > 8) rw *= 2;
    if (rw == 16 && tiles * ((p.R + kKWarps * 16 - 1) / (kKWarps * 16)) < 296 &&
        (p.R + kKWarps * 8 - 1) / (kKWarps * 8) <= 8)
        rw = 8;
    p.rows_warp = rw;
    p.rows_cta = kKWarps * rw;
    const int S = (p.R + p.rows_cta - 1) / p.rows_cta;
    const size_t smem = static_cast<size_t>(NS) * p.rows_cta * KPC * sizeof(float);
    auto kern = gemv_kernel<BITS, MODE>;
    if (smem > 48 * 1024)
        VKC_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          static_cast<int>(smem)));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(S, tiles, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attrs[2];
    cfg.attrs = attrs;
    cfg.numAttrs = launch_attrs(attrs, S);
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

int check_common(int bits, int N, int K, const void* w, const float* s, const float* z,
                 const float* x, const float* y) {
    if (bits != 32 && bits != 16 && bits != 8 && bits != 4)
        return set_error(kErrArg, "unsupported weight width %d (expected 32, 16, 8 or 4)", bits);
    const int kpc = 128 / bits;
    if (N <= 0 || K <= 0) return set_error(kErrArg, "N=%d and K=%d must be positive", N, K);
    if (K % kpc != 0)
        return set_error(kErrArg, "K=%d must be a multiple of %d for %d-bit weights", K, kpc, bits);
    if (!w || !x || !y) return set_error(kErrArg, "null weight, input or output pointer");
    if (reinterpret_cast<uintptr_t>(w) % 16 != 0)
        return set_error(kErrArg, "packed weights must be 16-byte aligned");
    if (bits <= 8) {
        if (N % kGroup != 0)
            return set_error(kErrArg, "N=%d must be a multiple of 256 for quantised weights", N);
        if (!s || !z) return set_error(kErrArg, "quantised weights need scale and zero arrays");
    }
    return kOk;
}

}  // namespace
}  // namespace vkc

using namespace vkc;

extern "C" {

int vkc_gemv(int bits, const void* w, const float* scale, const float* zero, const float* x,
             float* y, int N, int K, void* stream) {
    if (int e = check_common(bits, N, K, w, scale, zero, x, y)) return e;
    GemvParams p = {};
    p.w[0] = static_cast<const uint4*>(w);
    p.s[0] = scale;
    p.z[0] = zero;
    p.x = x;
    p.y = y;
    p.N = N;
    p.K = K;
    return launch_mode<kGemv>(bits, p, static_cast<cudaStream_t>(stream));
}

int vkc_rmsnorm_gemv(int bits, const void* w, const float* scale, const float* zero,
                     const float* x, const float* gamma, float* y, int N, int K, float eps,
                     int rms_dim, void* stream) {
    if (int e = check_common(bits, N, K, w, scale, zero, x, y)) return e;
    if (!gamma) return set_error(kErrArg, "null gamma");
    if (rms_dim <= 0) return set_error(kErrArg, "rms_dim=%d must be positive", rms_dim);
    GemvParams p = {};
    p.w[0] = static_cast<const uint4*>(w);
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

int vkc_rmsnorm_gemv_rope(int bits, const void* w, const float* scale, const float* zero,
                          const float* x, const float* gamma, const float* theta, float* y,
                          int N, int K, float eps, int rms_dim, int pos, int rope_mode,
                          int head_dim, int rot_rows, void* stream) {
    if (int e = check_common(bits, N, K, w, scale, zero, x, y)) return e;
    if (!gamma || !theta) return set_error(kErrArg, "null gamma or theta");
    if (rms_dim <= 0) return set_error(kErrArg, "rms_dim=%d must be positive", rms_dim);
    GemvParams p = {};
    p.w[0] = static_cast<const uint4*>(w);
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
                       const float* su, const float* zu, const float* x, const float* gamma,
                       float* h, int N, int K, float eps, int rms_dim, void* stream) {
    if (int e = check_common(bits, N, K, wg, sg, zg, x, h)) return e;
    if (int e = check_common(bits, N, K, wu, su, zu, x, h)) return e;
    if (!gamma) return set_error(kErrArg, "null gamma");
    if (rms_dim <= 0) return set_error(kErrArg, "rms_dim=%d must be positive", rms_dim);
    GemvParams p = {};
    p.w[0] = static_cast<const uint4*>(wg);
    p.w[1] = static_cast<const uint4*>(wu);
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

}  // extern "C"
