// The fp32 operators of vk-compute's shader directory that read plain
// row-major data rather than the 16-byte chunk layout:
//
//  * RmsNorm (shader/RmsNorm.comp:22-52): in place, every row of `width`
//    values (the shader's 256, one workgroup per row) becomes
//    x * inv_rms * gamma with inv_rms = 1/sqrt(sum(x^2)/width + eps).
//  * GEMV over a row-major K x N fp32 matrix, y[j] = sum_k x[k] W[k*N + j]
//    (shader/gemv2.comp:27-38 and gemv3.comp:29-42, which read W[row*N + col];
//    gemv1.comp:23-36 is the square case N = K).
//
// RmsNorm: one warp per row, float4 loads when the row allows, a butterfly
// warp sum (fixed order, deterministic).  Row-major GEMV: the natural access
// of that layout is one output column per lane (a warp reads 512 contiguous
// bytes of a row with float4 per lane); K is split over enough CTAs to fill
// the SMs, and the K-slices' partial vectors are summed in slice order by a
// second small kernel (deterministic, no atomics).
#include "vkc_common.cuh"
#include "vk_compute_b200.h"

namespace vkc {
namespace {

constexpr int kRowThreads = 256;

template <bool VEC>
__global__ void __launch_bounds__(kRowThreads) rmsnorm_rows_kernel(float* __restrict__ x,
                                                                    const float* __restrict__ gamma, int rows,
                                                                    int width, float eps) {
    pdl_launch_dependents();
    pdl_wait();
    const int lane = threadIdx.x & 31;
    const int row = blockIdx.x * (kRowThreads / 32) + (threadIdx.x >> 5);
    if (row >= rows) return;
    float* xr = x + static_cast<size_t>(row) * width;
    float ss = 0.f;
    if constexpr (VEC) {
        const float4* x4 = reinterpret_cast<const float4*>(xr);
        for (int i = lane; i < width / 4; i += 32) {
            const float4 v = x4[i];
            ss = fmaf(v.x, v.x, fmaf(v.y, v.y, fmaf(v.z, v.z, fmaf(v.w, v.w, ss))));
        }
    } else {
        for (int i = lane; i < width; i += 32) ss = fmaf(xr[i], xr[i], ss);
    }
    ss = warp_sum(ss);
    const float inv = 1.0f / sqrtf(ss / static_cast<float>(width) + eps);
    if constexpr (VEC) {
        float4* x4 = reinterpret_cast<float4*>(xr);
        const float4* g4 = reinterpret_cast<const float4*>(gamma);
        for (int i = lane; i < width / 4; i += 32) {
            float4 v = x4[i];
            const float4 g = __ldg(g4 + i);
            v.x = v.x * inv * g.x;
            v.y = v.y * inv * g.y;
            v.z = v.z * inv * g.z;
            v.w = v.w * inv * g.w;
            x4[i] = v;
        }
    } else {
        for (int i = lane; i < width; i += 32) xr[i] = xr[i] * inv * __ldg(gamma + i);
    }
}

// Partial y over rows [k0, k1) of this CTA's K-slice for V consecutive
// columns per thread (V = 4: float4 loads; V = 1: any N).
template <int V>
__global__ void __launch_bounds__(kRowThreads) gemv_rowmajor_kernel(const float* __restrict__ w,
                                                                     const float* __restrict__ x,
                                                                     float* __restrict__ out, int N, int K,
                                                                     int rows_per_split) {
    pdl_launch_dependents();
    const int col = (blockIdx.x * kRowThreads + threadIdx.x) * V;
    const int k0 = blockIdx.y * rows_per_split;
    const int k1 = min(K, k0 + rows_per_split);
    pdl_wait();
    if (col >= N) return;
    float acc[V];
#pragma unroll
    for (int v = 0; v < V; ++v) acc[v] = 0.f;
    int k = k0;
    constexpr int U = 8;  // rows in flight per thread
    for (; k + U <= k1; k += U) {
        float xv[U];
        float wv[U][V];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            xv[u] = __ldg(x + k + u);
            const float* wp = w + static_cast<size_t>(k + u) * N + col;
            if constexpr (V == 4) {
                const float4 t = __ldg(reinterpret_cast<const float4*>(wp));
                wv[u][0] = t.x;
                wv[u][1] = t.y;
                wv[u][2] = t.z;
                wv[u][3] = t.w;
            } else {
                wv[u][0] = __ldg(wp);
            }
        }
#pragma unroll
        for (int u = 0; u < U; ++u)
#pragma unroll
            for (int v = 0; v < V; ++v) acc[v] = fmaf(xv[u], wv[u][v], acc[v]);
    }
    for (; k < k1; ++k) {
        const float xk = __ldg(x + k);
        const float* wp = w + static_cast<size_t>(k) * N + col;
#pragma unroll
        for (int v = 0; v < V; ++v) acc[v] = fmaf(xk, __ldg(wp + v), acc[v]);
    }
    float* o = out + static_cast<size_t>(blockIdx.y) * N + col;
#pragma unroll
    for (int v = 0; v < V; ++v) o[v] = acc[v];
}

// y[j] = sum over the S slices of part[s][j], in slice order.
__global__ void __launch_bounds__(kRowThreads) sum_slices_kernel(const float* __restrict__ part,
                                                                  float* __restrict__ y, int N, int S) {
    pdl_launch_dependents();
    pdl_wait();
    const int j = blockIdx.x * kRowThreads + threadIdx.x;
    if (j >= N) return;
    float a = 0.f;
    for (int s = 0; s < S; ++s) a += part[static_cast<size_t>(s) * N + j];
    y[j] = a;
}

int sms_of_current_device(int* out) {
    int dev = 0;
    VKC_CUDA_TRY(cudaGetDevice(&dev));
    VKC_CUDA_TRY(cudaDeviceGetAttribute(out, cudaDevAttrMultiProcessorCount, dev));
    return kOk;
}

template <typename Kern, typename... Args>
int launch_plain(Kern kern, dim3 grid, cudaStream_t stream, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(kRowThreads, 1, 1);
    cfg.stream = stream;
    cudaLaunchAttribute attrs[2];
    cfg.attrs = attrs;
    cfg.numAttrs = launch_attrs(attrs, 1);
    VKC_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, args...));
    return kOk;
}

}  // namespace
}  // namespace vkc

using namespace vkc;

extern "C" {

int vkc_rmsnorm_rows(float* x, const float* gamma, int rows, int width, float eps, void* stream) {
    if (!x || !gamma) return set_error(kErrArg, "null x or gamma");
    if (rows <= 0 || width <= 0) return set_error(kErrArg, "rows=%d and width=%d must be positive", rows, width);
    const bool vec = width % 4 == 0 && reinterpret_cast<uintptr_t>(x) % 16 == 0 &&
                     reinterpret_cast<uintptr_t>(gamma) % 16 == 0;
    const dim3 grid((rows + kRowThreads / 32 - 1) / (kRowThreads / 32), 1, 1);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    return vec ? launch_plain(rmsnorm_rows_kernel<true>, grid, s, x, gamma, rows, width, eps)
               : launch_plain(rmsnorm_rows_kernel<false>, grid, s, x, gamma, rows, width, eps);
}

int vkc_gemv_rowmajor(const float* w, const float* x, float* y, int N, int K, void* stream) {
    if (!w || !x || !y) return set_error(kErrArg, "null weight, input or output pointer");
    if (N <= 0 || K <= 0) return set_error(kErrArg, "N=%d and K=%d must be positive", N, K);
    int sms = 0;
    if (int e = sms_of_current_device(&sms)) return e;
    const bool vec = N % 4 == 0 && reinterpret_cast<uintptr_t>(w) % 16 == 0;
    const int per_cta = kRowThreads * (vec ? 4 : 1);
    const int tiles = (N + per_cta - 1) / per_cta;
    // enough K-slices for about two CTAs per SM, each at least 64 rows long
    int S = (2 * sms + tiles - 1) / tiles;
    S = S < 1 ? 1 : S;
    S = S > 64 ? 64 : S;
    if (S > (K + 63) / 64) S = (K + 63) / 64;
    if (S < 1) S = 1;
    const int rows = (K + S - 1) / S;
    S = (K + rows - 1) / rows;  // no empty slices
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    float* part = y;
    if (S > 1) {
        void* ws = nullptr;
        if (int e = device_workspace(kWorkspaceHeader + static_cast<size_t>(S) * N * sizeof(float), &ws, s,
                                     kWorkspaceRowGemv))
            return e;
        part = reinterpret_cast<float*>(static_cast<char*>(ws) + kWorkspaceHeader);
    }
    const dim3 grid(tiles, S, 1);
    int rc = vec ? launch_plain(gemv_rowmajor_kernel<4>, grid, s, w, x, part, N, K, rows)
                 : launch_plain(gemv_rowmajor_kernel<1>, grid, s, w, x, part, N, K, rows);
    if (rc || S == 1) return rc;
    return launch_plain(sum_slices_kernel, dim3((N + kRowThreads - 1) / kRowThreads, 1, 1), s,
                        static_cast<const float*>(part), y, N, S);
}

}  // extern "C"
