// Weight preparation on the device: the seeded generator, the quantisers and
// the transpose_block16 packer of vk-compute's src/data.c, bit-identical to
// the host versions, so multi-gigabyte decoder weights are made in
// milliseconds instead of minutes.
#include "vkc_common.cuh"

#include <cuda_fp16.h>

namespace vkc {
namespace {

constexpr int kGroup = 256;

// src/data.c:8-16
__device__ __forceinline__ float pseudo_random(int i, int j, int seed) {
    uint32_t h = static_cast<uint32_t>(i) * 73129u + static_cast<uint32_t>(j) * 95121u +
                 static_cast<uint32_t>(seed) * 15473u;
    h = (h ^ 61u) ^ (h >> 16);
    h += h << 3;
    h ^= h >> 4;
    h *= 0x27d4eb2du;
    h ^= h >> 15;
    return (static_cast<float>(h % 2000001u) / 1000000.0f) - 1.0f;
}

// src/data.c:30-51: truncating fp32 -> fp16 with the reference's subnormal
// branch.
__device__ __forceinline__ uint16_t trunc_fp16(float f) {
    const uint32_t b = __float_as_uint(f);
    const uint32_t sign = (b >> 16) & 0x8000u;
    const int e = static_cast<int>((b >> 23) & 0xffu) - 127;
    const uint32_t m = b & 0x7fffffu;
    if (e <= -15) {
        if (e < -24) return static_cast<uint16_t>(sign);
        return static_cast<uint16_t>(sign | ((m | 0x800000u) >> (1 - e)));
    }
    if (e >= 16) return static_cast<uint16_t>(sign | 0x7c00u);
    return static_cast<uint16_t>(sign | (static_cast<uint32_t>(e + 15) << 10) | (m >> 13));
}

__global__ void generate_kernel(int seed, int M, int N, int out_bits, void* dst) {
    const int64_t total = static_cast<int64_t>(M) * N;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int r = static_cast<int>(i / N), c = static_cast<int>(i % N);
        const float v = pseudo_random(r, c, seed);
        if (out_bits == 32)
            static_cast<float*>(dst)[i] = v;
        else
            static_cast<uint16_t*>(dst)[i] = trunc_fp16(v);
    }
}

// One thread per (row k, 256-output block b): src/data.c:109-134 (int8) and
// 153-181 (int4), or the symmetric variant.
__global__ void quantize_kernel(const float* __restrict__ w, int K, int N, int bits, int symmetric,
                                int fp16_scale, uint8_t* __restrict__ codes, float* __restrict__ scale,
                                float* __restrict__ zero) {
    const int nb = N / kGroup;
    const int64_t idx = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
    if (idx >= static_cast<int64_t>(K) * nb) return;
    const int k = static_cast<int>(idx / nb), b = static_cast<int>(idx % nb);
    const float* row = w + static_cast<int64_t>(k) * N + b * kGroup;
    const int64_t si = static_cast<int64_t>(b) * K + k;
    float s, z;
    int off = 0;
    float qmax = 0.f;
    if (!symmetric) {
        float lo = 1e9f, hi = -1e9f;
        for (int t = 0; t < kGroup; ++t) {
            const float v = row[t];
            lo = v < lo ? v : lo;
            hi = v > hi ? v : hi;
        }
        s = __fdiv_rn(hi - lo, bits == 8 ? 255.0f : 15.0f);
        z = -lo;
    } else {
        qmax = bits == 8 ? 127.0f : 7.0f;
        off = bits == 8 ? 128 : 8;
        float amax = 0.f;
        for (int t = 0; t < kGroup; ++t) amax = fmaxf(amax, fabsf(row[t]));
        s = __fdiv_rn(amax, qmax);
        if (fp16_scale) s = __half2float(__float2half_rn(s));
        z = static_cast<float>(off) * s;
    }
    scale[si] = s;
    zero[si] = z;
    for (int t = 0; t < kGroup; ++t) {
        uint32_t u;
        if (!symmetric) {
            u = static_cast<uint8_t>(roundf(__fdiv_rn(__fadd_rn(row[t], z), s)));
        } else {
            float q = 0.f;
            if (s > 0.f) q = fminf(fmaxf(roundf(__fdiv_rn(row[t], s)), -qmax), qmax);
            u = static_cast<uint32_t>(static_cast<int>(q) + off);
        }
        const int c = b * kGroup + t;
        if (bits == 8) {
            codes[static_cast<int64_t>(k) * N + c] = static_cast<uint8_t>(u);
        } else {
            uint8_t* p = codes + static_cast<int64_t>(k) * (N / 2) + c / 2;
            if ((c & 1) == 0)
                *p = static_cast<uint8_t>((u & 0x0fu) << 4);
            else
                *p = static_cast<uint8_t>(*p | (u & 0x0fu));
        }
    }
}

// One thread per 16-byte output chunk (r, j): src/data.c:198-222.
__global__ void pack_kernel(const uint8_t* __restrict__ in, uint4* __restrict__ out, int K, int N,
                            int bits) {
    const int per = 128 / bits;
    const int R = K / per;
    const int64_t idx = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
    if (idx >= static_cast<int64_t>(R) * N) return;
    const int r = static_cast<int>(idx / N), j = static_cast<int>(idx % N);
    uint32_t wd[4] = {0u, 0u, 0u, 0u};
    if (bits == 4) {
        for (int t = 0; t < per; ++t) {
            const uint8_t byte = in[static_cast<int64_t>(r * per + t) * (N / 2) + j / 2];
            const uint32_t q = (j & 1) ? (byte & 0x0fu) : (byte >> 4);
            wd[t / 8] |= q << (4 * (t % 8));
        }
    } else {
        const int eb = bits / 8;
        uint8_t* o = reinterpret_cast<uint8_t*>(wd);
        for (int t = 0; t < per; ++t)
            for (int e = 0; e < eb; ++e)
                o[t * eb + e] = in[(static_cast<int64_t>(r * per + t) * N + j) * eb + e];
    }
    out[idx] = make_uint4(wd[0], wd[1], wd[2], wd[3]);
}

int grid_for(int64_t n, int threads) {
    int64_t g = (n + threads - 1) / threads;
    return static_cast<int>(g > 148 * 64 ? 148 * 64 : (g < 1 ? 1 : g));
}

}  // namespace
}  // namespace vkc

using namespace vkc;

extern "C" {

int vkc_generate(int seed, int M, int N, int out_bits, void* dst, void* stream) {
    if (M <= 0 || N <= 0 || !dst) return set_error(kErrArg, "generate: bad shape or null output");
    if (out_bits != 32 && out_bits != 16) return set_error(kErrArg, "generate: out_bits 32 or 16");
    generate_kernel<<<grid_for(static_cast<int64_t>(M) * N, 256), 256, 0,
                      static_cast<cudaStream_t>(stream)>>>(seed, M, N, out_bits, dst);
    VKC_CUDA_TRY(cudaGetLastError());
    return kOk;
}

int vkc_quantize(const float* w, int K, int N, int bits, int symmetric, int fp16_scale,
                 uint8_t* codes, float* scale, float* zero, void* stream) {
    if (!w || !codes || !scale || !zero) return set_error(kErrArg, "quantize: null pointer");
    if (bits != 8 && bits != 4) return set_error(kErrArg, "quantize: bits must be 8 or 4");
    if (K <= 0 || N <= 0 || N % kGroup != 0)
        return set_error(kErrArg, "quantize: K=%d, N=%d (N a multiple of 256)", K, N);
    const int64_t n = static_cast<int64_t>(K) * (N / kGroup);
    quantize_kernel<<<static_cast<int>((n + 127) / 128), 128, 0, static_cast<cudaStream_t>(stream)>>>(
        w, K, N, bits, symmetric, fp16_scale, codes, scale, zero);
    VKC_CUDA_TRY(cudaGetLastError());
    return kOk;
}

int vkc_pack_block16(const void* in, void* out, int K, int N, int bits, void* stream) {
    if (!in || !out) return set_error(kErrArg, "pack: null pointer");
    if (bits != 32 && bits != 16 && bits != 8 && bits != 4)
        return set_error(kErrArg, "pack: bits must be 32, 16, 8 or 4");
    const int per = 128 / bits;
    if (K <= 0 || N <= 0 || K % per != 0 || (bits == 4 && N % 2 != 0))
        return set_error(kErrArg, "pack: K=%d must be a multiple of %d (N even for 4-bit)", K, per);
    if (reinterpret_cast<uintptr_t>(out) % 16 != 0) return set_error(kErrArg, "pack: output not 16-byte aligned");
    const int64_t n = static_cast<int64_t>(K / per) * N;
    pack_kernel<<<static_cast<int>((n + 255) / 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const uint8_t*>(in), static_cast<uint4*>(out), K, N, bits);
    VKC_CUDA_TRY(cudaGetLastError());
    return kOk;
}

}  // extern "C"
