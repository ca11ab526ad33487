// fp32 C = A B (row-major) for the drop-in "gemm" operator
// (shader/gemm.comp:19-59): 64x64 output tiles, 16-deep k slabs staged in
// shared memory, 4x4 outputs per thread, guarded for any M, N, K.
#include "vkc_common.cuh"

namespace vkc {
namespace {

constexpr int kTM = 64, kTN = 64, kTK = 16;

__global__ void __launch_bounds__(256) gemm_f32_kernel(const float* __restrict__ a,
                                                       const float* __restrict__ b,
                                                       float* __restrict__ c, int M, int N, int K) {
    __shared__ float as[kTK][kTM + 4];
    __shared__ float bs[kTK][kTN + 4];
    const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
    const int m0 = blockIdx.y * kTM, n0 = blockIdx.x * kTN;
    float acc[4][4] = {};
    pdl_launch_dependents();
    pdl_wait();
    for (int k0 = 0; k0 < K; k0 += kTK) {
        for (int i = threadIdx.x; i < kTM * kTK; i += 256) {
            const int mm = i / kTK, kk = i % kTK;
            const int gm = m0 + mm, gk = k0 + kk;
            as[kk][mm] = (gm < M && gk < K) ? a[static_cast<int64_t>(gm) * K + gk] : 0.f;
        }
        for (int i = threadIdx.x; i < kTK * kTN; i += 256) {
            const int kk = i / kTN, nn = i % kTN;
            const int gk = k0 + kk, gn = n0 + nn;
            bs[kk][nn] = (gk < K && gn < N) ? b[static_cast<int64_t>(gk) * N + gn] : 0.f;
        }
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < kTK; ++kk) {
            float av[4], bv[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) av[i] = as[kk][ty * 4 + i];
#pragma unroll
            for (int j = 0; j < 4; ++j) bv[j] = bs[kk][tx * 4 + j];
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int gm = m0 + ty * 4 + i, gn = n0 + tx * 4 + j;
            if (gm < M && gn < N) c[static_cast<int64_t>(gm) * N + gn] = acc[i][j];
        }
}

}  // namespace
}  // namespace vkc

using namespace vkc;

extern "C" int vkc_gemm_f32(const float* a, const float* b, float* c, int M, int N, int K,
                            void* stream) {
    if (!a || !b || !c) return set_error(kErrArg, "gemm: null pointer");
    if (M <= 0 || N <= 0 || K <= 0) return set_error(kErrArg, "gemm: M=%d N=%d K=%d", M, N, K);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((N + kTN - 1) / kTN, (M + kTM - 1) / kTM, 1);
    cfg.blockDim = dim3(256, 1, 1);
    cfg.stream = static_cast<cudaStream_t>(stream);
    cudaLaunchAttribute attrs[2];
    cfg.attrs = attrs;
    cfg.numAttrs = launch_attrs(attrs, 1);
    VKC_CUDA_TRY(cudaLaunchKernelEx(&cfg, gemm_f32_kernel, a, b, c, M, N, K));
    return kOk;
}
