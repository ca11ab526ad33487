// Prefill GEMM on the 5th-generation tensor cores (tcgen05 + TMEM), sm_100a:
// C[M][N] (fp32) = A[M][K] (bf16) . W[N][K]^T (bf16), both row-major, i.e. the
// weight is stored K-major (N rows of K), the usual layout of a linear layer.
// This is the batched counterpart of the decode GEMVs (shader/gemm.comp's
// contraction for a batch of tokens: 64 x 4096 . 4096 x 12288 in the prefill
// configuration).
//
// At M = 64 the product is bound by streaming W (100 MB) from HBM, not by the
// tensor cores, so the kernel is a weight stream with the MMA in the loop:
// - A CTA owns a range of output columns for all rows of one 128-row M tile,
//   and the whole K range: no split-K, no reduction.  The columns are split
//   in two widths 16 apart (each width with its own tensor map) over the
//   fewest CTAs that keep the widest range as narrow as one CTA per SM
//   allows: 12288 columns go to 128 CTAs of 96 (148 CTAs would still need
//   ranges of 96, and measured slower).
// - TMA (cp.async.bulk.tensor, 128-byte swizzle) loads K tiles of 64 into a
//   ring of kStages shared-memory stages: the A tile and the W tile.  With
//   M <= 64 only A's 64 real rows are loaded; rows 64..127 of every stage are
//   zeroed once, so the M = 128 MMA multiplies them as zeros without moving
//   them again.  One thread produces.
// - One thread issues tcgen05.mma kind::f16 (M = 128, N = the CTA's width,
//   K = 16; bf16 inputs, fp32 accumulator in TMEM), four per K tile, and
//   returns each stage to the producer with tcgen05.commit on the stage's
//   "empty" mbarrier.
// - After the last tile a commit signals the epilogue: the four warps read
//   their 32 TMEM lanes (rows) with tcgen05.ld and store fp32 rows of C.
// Every mbarrier wait is bounded; a timeout sets flag 0x10 of the status word and
// the kernel stops issuing work, waits for its copies, frees TMEM and returns.
#include "vkc_common.cuh"

#include <cuda.h>

#include <mutex>

namespace vkc {
namespace {

constexpr int kBM = 128;       // rows per MMA (A rows past M are zero)
constexpr int kBK = 64;        // K per stage: one 128-byte swizzle row of bf16
constexpr int kStages = 6;
constexpr int kTcThreads = 128;
constexpr unsigned kStatusTcTimeout = 16u;

constexpr int kBNMax = 128;  // widest CTA column range (the stage holds this many W rows)

struct TcGeo {
    static constexpr int a_bytes = kBM * kBK * 2;  // 16 KB
    static constexpr int b_bytes = kBNMax * kBK * 2;
    static constexpr int stage_bytes = a_bytes + b_bytes;
    static constexpr int tmem_cols = kBNMax;
    static constexpr size_t smem_bytes = 1024 /* alignment slack */ + static_cast<size_t>(kStages) * stage_bytes + 256;
    static_assert(kBNMax % 16 == 0 && kBNMax <= 256, "M = 128 MMA needs N in [16, 256], a multiple of 16");
    static_assert(a_bytes % 1024 == 0 && b_bytes % 1024 == 0, "stages stay 1024-byte aligned");
};

__device__ __forceinline__ void mbar_init1(uint32_t bar) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}
// Bounded wait; false when it ran out.
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity) {
    for (uint32_t i = 0; i < kSpinLimit; ++i)
        if (mbar_try(bar, parity)) return true;
    return false;
}
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
        : "memory");
}
// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row groups
// 1024 bytes apart (stride byte offset), descriptor version 1.
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t addr) {
    return static_cast<uint64_t>((addr >> 4) & 0x3FFF) | (static_cast<uint64_t>(1) << 16) |
           (static_cast<uint64_t>(1024 >> 4) << 32) | (static_cast<uint64_t>(1) << 46) |
           (static_cast<uint64_t>(2) << 61);
}
// Instruction descriptor, kind::f16: fp32 accumulator, bf16 A and B, both
// K-major, N >> 3 at bit 17, M >> 4 at bit 24.
__device__ __forceinline__ uint32_t idesc_bf16(int bn) {
    return (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(bn >> 3) << 17) |
           (static_cast<uint32_t>(kBM >> 4) << 24);
}
__device__ __forceinline__ void umma_bf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
__device__ __forceinline__ void umma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                 : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// CTAs [0, n_hi) own bn_lo + 16 columns (map_w_hi), the rest bn_lo (map_w_lo);
// a_rows is the A box height (64 when M <= 64, else 128).
__global__ void __launch_bounds__(kTcThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_w_lo,
                   const __grid_constant__ CUtensorMap map_w_hi, float* c, int M, int N, int K, int n_hi, int bn_lo,
                   int a_rows, unsigned* status) {
    using Geo = TcGeo;
    extern __shared__ uint8_t smem_raw[];
    // 1024-byte aligned stages (128-byte swizzle atoms), barriers after them.
    const uint32_t raw = smem_addr(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    uint8_t* bars_ptr = smem_raw + (base - raw) + kStages * Geo::stage_bytes;
    const uint32_t bars = smem_addr(bars_ptr);
    auto full = [&](int s) { return bars + 8u * s; };
    auto empty = [&](int s) { return bars + 8u * (kStages + s); };
    const uint32_t done = bars + 8u * (2 * kStages);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars_ptr + 8 * (2 * kStages + 1));
    __shared__ volatile int s_abort;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int cta = blockIdx.x;
    const bool wide = cta < n_hi;
    const int BN = wide ? bn_lo + 16 : bn_lo;
    const int n0 = wide ? cta * BN : n_hi * (bn_lo + 16) + (cta - n_hi) * bn_lo;
    const CUtensorMap* map_w = wide ? &map_w_hi : &map_w_lo;
    const int m0 = blockIdx.y * kBM;
    const int KT = K / kBK;
    const uint32_t a_load = static_cast<uint32_t>(a_rows) * kBK * 2;  // A bytes TMA writes per stage
    const uint32_t stage_tx = a_load + static_cast<uint32_t>(BN) * kBK * 2;

    // With a 64-row A box, rows 64..127 of every stage's A tile stay zero.
    if (a_rows < kBM) {
        for (int s = 0; s < kStages; ++s) {
            uint4* z = reinterpret_cast<uint4*>(smem_raw + (base - raw) + s * Geo::stage_bytes + a_load);
            for (int i = tid; i < static_cast<int>((Geo::a_bytes - a_load) / 16); i += kTcThreads)
                z[i] = make_uint4(0u, 0u, 0u, 0u);
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // visible to the MMA's reads
    }

    if (tid == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init1(full(s));
            mbar_init1(empty(s));
        }
        mbar_init1(done);
        s_abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    if (warp == 1) {  // TMEM accumulator: 128 lanes x tmem_cols fp32 columns
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)),
                     "r"(Geo::tmem_cols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    pdl_launch_dependents();
    pdl_wait();  // A (activations) may come from the previous kernel

    if (warp == 0 && lane == 0) {
        // ---- producer: TMA into the ring ----
        for (int kt = 0; kt < KT; ++kt) {
            const int s = kt % kStages;
            const uint32_t ph = (kt / kStages) & 1u;
            if (!mbar_wait_bounded(empty(s), ph ^ 1u)) {
                s_abort = 1;
                atomicOr(status, kStatusTcTimeout);
                break;
            }
            if (s_abort) break;
            const uint32_t sa = base + s * Geo::stage_bytes;
            mbar_expect_tx(full(s), stage_tx);
            tma_load_2d(sa, &map_a, kt * kBK, m0, full(s));
            tma_load_2d(sa + Geo::a_bytes, map_w, kt * kBK, n0, full(s));
        }
    } else if (warp == 1 && lane == 0) {
        // ---- MMA issuer ----
        const uint32_t idesc = idesc_bf16(BN);
        bool ok = true;
        for (int kt = 0; kt < KT && ok; ++kt) {
            const int s = kt % kStages;
            const uint32_t ph = (kt / kStages) & 1u;
            if (!mbar_wait_bounded(full(s), ph) || s_abort) {
                s_abort = 1;
                atomicOr(status, kStatusTcTimeout);
                ok = false;
                break;
            }
            tc_fence_after();
            const uint32_t sa = base + s * Geo::stage_bytes;
            const uint64_t ad = smem_desc_sw128(sa), bd = smem_desc_sw128(sa + Geo::a_bytes);
#pragma unroll
            for (int kk = 0; kk < kBK / 16; ++kk)  // K = 16 per MMA: 32 bytes along the swizzled row
                umma_bf16(tmem, ad + 2u * kk, bd + 2u * kk, idesc, (kt | kk) != 0 ? 1u : 0u);
            umma_commit(empty(s));  // stage s is free once these MMAs have read it
        }
        umma_commit(done);  // the accumulator is complete once every MMA above has
    }
    __syncwarp();

    // ---- epilogue: warp w reads TMEM lanes [32 w, 32 w + 32) = rows ----
    const bool have = mbar_wait_bounded(done, 0);
    if (!have) atomicOr(status, kStatusTcTimeout);
    tc_fence_after();
    const int row = m0 + warp * 32 + lane;
    if (have && m0 + warp * 32 < M) {
#pragma unroll 1
        for (int col = 0; col < BN; col += 16) {
            uint32_t v[16];
            asm volatile(
                "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, "
                "[%16];"
                : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
                  "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]),
                  "=r"(v[15])
                : "r"(tmem + (static_cast<uint32_t>(warp * 32) << 16) + static_cast<uint32_t>(col)));
            asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
            if (row < M) {
                float4* dst = reinterpret_cast<float4*>(c + static_cast<size_t>(row) * N + n0 + col);
#pragma unroll
                for (int q = 0; q < 4; ++q)
                    dst[q] = make_float4(__uint_as_float(v[4 * q]), __uint_as_float(v[4 * q + 1]),
                                         __uint_as_float(v[4 * q + 2]), __uint_as_float(v[4 * q + 3]));
            }
        }
    }

    // ---- teardown: drain an aborted ring, free TMEM ----
    if (s_abort && warp == 0 && lane == 0) {
        for (int s = 0; s < kStages; ++s) (void)mbar_wait_bounded(full(s), 0);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(Geo::tmem_cols)
                     : "memory");
    }
}

// cuTensorMapEncodeTiled from the driver, looked up once (no link to libcuda).
using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                              const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                              CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
std::mutex g_enc_mu;
EncodeFn g_encode = nullptr;

int encode_fn(EncodeFn* out) {
    std::lock_guard<std::mutex> lock(g_enc_mu);
    if (!g_encode) {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        VKC_CUDA_TRY(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q));
        if (q != cudaDriverEntryPointSuccess || !fn)
            return set_error(kErrCuda, "cuTensorMapEncodeTiled is not available from the driver");
        g_encode = reinterpret_cast<EncodeFn>(fn);
    }
    *out = g_encode;
    return kOk;
}

// 2-D bf16 row-major tensor [rows][K], boxes of 64 (K) x box_rows, 128-byte
// swizzle, zero fill past the edges.
int make_map(CUtensorMap* map, const void* ptr, int rows, int K, int box_rows) {
    EncodeFn enc = nullptr;
    if (int e = encode_fn(&enc)) return e;
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(rows)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(K) * 2};
    const cuuint32_t box[2] = {static_cast<cuuint32_t>(kBK), static_cast<cuuint32_t>(box_rows)};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(kErrCuda, "cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
    return kOk;
}

__device__ unsigned g_tc_status = 0;

}  // namespace
}  // namespace vkc

using namespace vkc;

extern "C" {

int vkc_gemm_bf16(const void* a, const void* w, float* c, int M, int N, int K, void* stream) {
    if (!a || !w || !c) return set_error(kErrArg, "null GEMM pointer");
    if (M <= 0 || N <= 0 || K <= 0) return set_error(kErrArg, "M=%d N=%d K=%d must be positive", M, N, K);
    if (K % kBK != 0) return set_error(kErrArg, "K=%d must be a multiple of %d", K, kBK);
    if (N % 16 != 0) return set_error(kErrUnsupported, "N=%d must be a multiple of 16", N);
    if ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(c)) % 16 != 0)
        return set_error(kErrArg, "A, W and C must be 16-byte aligned");
    int dev = 0, sms = 0;
    VKC_CUDA_TRY(cudaGetDevice(&dev));
    VKC_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    // Column ranges: the widest range a CTA gets is set by spreading the
    // 16-column tiles over at most one CTA per SM; the fewest CTAs that keep
    // that width then share the tiles in widths q*16 and (q + 1)*16 (12288
    // columns: 128 CTAs of 96, as wide as 148 CTAs would make the widest,
    // with less contention).  Ranges wider than kBNMax go to further waves.
    const int tiles = N / 16;
    const int max_tiles = kBNMax / 16 - 1;  // the wider range holds at most kBNMax columns
    int widest = (tiles + sms - 1) / sms;
    if (widest > max_tiles) widest = max_tiles;
    const int ctas = (tiles + widest - 1) / widest;
    const int q = tiles / ctas, r = tiles % ctas;
    const int bn_lo = 16 * q;
    const int a_rows = M <= 64 ? 64 : kBM;
    CUtensorMap ma, mw_lo, mw_hi;
    if (int e = make_map(&ma, a, M, K, a_rows)) return e;
    if (int e = make_map(&mw_lo, w, N, K, bn_lo)) return e;
    if (int e = make_map(&mw_hi, w, N, K, bn_lo + 16 <= kBNMax ? bn_lo + 16 : bn_lo)) return e;
    unsigned* status = nullptr;
    VKC_CUDA_TRY(cudaGetSymbolAddress(reinterpret_cast<void**>(&status), g_tc_status));
    auto kern = gemm_tc_kernel;
    const size_t smem = TcGeo::smem_bytes;
    if (int e = ensure_smem(reinterpret_cast<const void*>(kern), smem)) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(ctas, (M + kBM - 1) / kBM, 1);
    cfg.blockDim = dim3(kTcThreads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = static_cast<cudaStream_t>(stream);
    cudaLaunchAttribute attrs[2];
    cfg.attrs = attrs;
    cfg.numAttrs = launch_attrs(attrs, 1);
    VKC_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, ma, mw_lo, mw_hi, c, M, N, K, r, bn_lo, a_rows, status));
    return kOk;
}

// Status flags of the tensor-core GEMM on the current device (0x10: a bounded
// wait ran out); reading waits for the device, `clear` resets.
int vkc_gemm_bf16_status(unsigned* out, int clear) {
    VKC_CUDA_TRY(cudaDeviceSynchronize());
    unsigned v = 0;
    VKC_CUDA_TRY(cudaMemcpyFromSymbol(&v, g_tc_status, sizeof v));
    if (clear) {
        const unsigned z = 0;
        VKC_CUDA_TRY(cudaMemcpyToSymbol(g_tc_status, &z, sizeof z));
    }
    *out = v;
    return kOk;
}

}  // extern "C"
