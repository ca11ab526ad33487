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

// Library-owned scratch of the current device, one allocation per user (the
// operators that keep state between calls in it must not share one): at
// least `bytes`, zero-filled when (re)allocated.  Kernels that use it leave
// their ticket words at zero, so consecutive launches on one stream may share
// it; launches that overlap on different streams must not.  Words [0, 64) are
// reserved for the status word written by bounded device waits.
enum : int {
    kWorkspaceAttention = 0,  // split partials and merge tickets of decode attention
    kWorkspaceRowGemv = 1,    // K-slice partials of the row-major GEMV
    kWorkspaceUsers = 2,
};
int device_workspace(size_t bytes, void** out, cudaStream_t stream, int user);
constexpr size_t kWorkspaceHeader = 256;

// Fills the launch attributes every kernel launcher uses: an optional cluster
// shape (cluster_x > 1) and the programmatic-serialization flag.  Returns the
// number of attributes written into attrs[0..2).
int launch_attrs(cudaLaunchAttribute* attrs, int cluster_x);

// cudaFuncSetAttribute(MaxDynamicSharedMemorySize) for `func` on the current
// device, skipped when an equal or larger value was already set (the call
// costs microseconds of host time on every launch otherwise).
int ensure_smem(const void* func, size_t bytes);

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

// ---- mbarrier / bulk-copy primitives (Hopper+ async proxy) ----------------
__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_init_fence() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
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
// Bounded wait on a phase of an mbarrier: false after `limit` polls.
constexpr uint32_t kSpinLimit = 1u << 22;
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
    for (uint32_t i = 0; i < kSpinLimit; ++i)
        if (mbar_try_wait(bar, parity)) return true;
    return false;
}
// L2 policy for data read exactly once (weights): evict first.
__device__ __forceinline__ uint64_t l2_evict_first() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}
// Global -> shared bulk copy completing on an mbarrier (16-byte aligned
// addresses, size a multiple of 16).  Single-destination copies only.
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar,
                                         uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;"
        ::"r"(dst), "l"(src), "r"(bytes), "r"(bar), "l"(policy)
        : "memory");
}
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 ::"r"(dst), "l"(src), "r"(bytes), "r"(bar)
                 : "memory");
}
// Named barrier over `threads` threads (a multiple of 32) with id `id` (1..15).
__device__ __forceinline__ void named_sync(uint32_t id, uint32_t threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// Cluster-scope helpers (distributed shared memory).
__device__ __forceinline__ void cluster_arrive_release() {
    asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait_acquire() {
    asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ uint32_t map_cluster_addr(uint32_t local, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local), "r"(rank));
    return r;
}
__device__ __forceinline__ void st_cluster_f32(uint32_t addr, float v) {
    asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}
__device__ __forceinline__ void fence_acq_rel_cluster() { asm volatile("fence.acq_rel.cluster;" ::: "memory"); }
__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait_cluster(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}

// Status bits a kernel records when a bounded wait gives up (see
// vkc_device_status).
enum : uint32_t {
    kStatusProducerTimeout = 1u,
    kStatusConsumerTimeout = 2u,
    kStatusReduceTimeout = 4u,
    kStatusPeerTimeout = 8u,  // a wait on other GPUs' arrivals ran out
};

// System-scope (other GPUs) relaxed accesses and the fence that orders them:
// the arrival counters of the NVLink peer exchanges.
__device__ __forceinline__ unsigned ld_relaxed_sys(const unsigned* p) {
    unsigned v;
    asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ unsigned atom_add_relaxed_sys(unsigned* p, unsigned v) {
    unsigned old;
    asm volatile("atom.add.relaxed.sys.global.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}
__device__ __forceinline__ void red_add_relaxed_sys(unsigned* p, unsigned v) {
    asm volatile("red.relaxed.sys.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void fence_acq_rel_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }
__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
// Longest a thread waits, in total, for other GPUs' data in a fused exchange:
// one deadline per thread, started at its first wait and shared by every
// element it waits for afterwards.
constexpr uint64_t kPeerWaitNs = 100ull * 1000 * 1000;
// Longest a cluster's collecting CTA waits for the other CTAs' deposits into
// its shared memory.  A depositing CTA can be held before its deposit only by
// its own peer waits (kPeerWaitNs in total per thread) and by its weight
// stream, so ten times the peer limit leaves the collecting CTA waiting well
// after every deposit that can still come: it never exits while another CTA
// may write into its shared memory.
constexpr uint64_t kClusterWaitNs = 10 * kPeerWaitNs;
static_assert(kClusterWaitNs >= 10 * kPeerWaitNs, "cluster wait must outlast every peer wait");

// 8-byte words read and written whole (single-copy atomic), for exchanges
// that carry a flag beside each value instead of ordering data and flags.
__device__ __forceinline__ unsigned long long ld_relaxed_sys_u64(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_relaxed_sys_u64(unsigned long long* p, unsigned long long v) {
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}


// Bounded wait, on the clock, for a phase of a cluster-visible mbarrier.
__device__ __forceinline__ bool mbar_wait_cluster_ns(uint32_t bar, uint32_t parity, uint64_t limit_ns) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    while (!mbar_try_wait_cluster(bar, parity))
        if (globaltimer_ns() - t0 > limit_ns) return false;
    return true;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

}  // namespace vkc
