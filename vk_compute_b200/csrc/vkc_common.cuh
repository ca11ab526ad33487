// Shared device helpers and host error plumbing for libvkcompute.
#pragma once

#include <cuda_runtime.h>
#include <cstdint>
#include <cstdio>

namespace vkc {

// ---------------------------------------------------------------------------
// Host-side status
// ---------------------------------------------------------------------------
enum Status : int {
    kOk = 0,
    kErrArg = -1,       // invalid shape, pointer or option
    kErrCuda = -2,      // a CUDA runtime call failed
    kErrUnsupported = -3,
    kErrTimeout = -4,   // a bounded device-side wait gave up
};

// Records a message for vkc_last_error() and returns `code`.
int set_error(int code, const char* fmt, ...);

#define VKC_CUDA_TRY(expr)                                                        \
    do {                                                                          \
        cudaError_t e__ = (expr);                                                 \
        if (e__ != cudaSuccess)                                                   \
            return ::vkc::set_error(::vkc::kErrCuda, "%s failed: %s", #expr,      \
                                    cudaGetErrorString(e__));                     \
    } while (0)

// Programmatic dependent launch switch shared by all launchers.
bool pdl_enabled();

// Fills the launch attributes every kernel launcher uses: an optional cluster
// shape (cluster_x > 1) and the programmatic-serialization flag.  Returns the
// number of attributes written into attrs[0..2).
int launch_attrs(cudaLaunchAttribute* attrs, int cluster_x);

// ---------------------------------------------------------------------------
// Device helpers
// ---------------------------------------------------------------------------

// 16-byte weight load: read-only path, no L1 allocation (weights are streamed
// once), 256-byte L2 prefetch since neighbouring lanes read adjacent chunks.
__device__ __forceinline__ uint4 ld_stream(const uint4* p) {
    uint4 r;
    asm("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0, %1, %2, %3}, [%4];"
        : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
        : "l"(p));
    return r;
}

// Packed fp32 pair arithmetic (sm_100 f32x2 instructions).
__device__ __forceinline__ uint64_t f2_pack(float lo, float hi) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
__device__ __forceinline__ float2 f2_unpack(uint64_t v) {
    float2 r;
    asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(v));
    return r;
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}

// Programmatic dependent launch controls (no-ops without the launch attribute).
__device__ __forceinline__ void pdl_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

}  // namespace vkc
