// All-gather of fp32 slices between the GPUs of one node by direct NVLink
// stores into the peers' memory: the exchange step of the row-sharded decoder
// chain (each rank owns a contiguous slice of an activation vector and every
// rank needs the whole vector).
//
// The full buffers and the arrival counters of every rank are mapped into
// every other rank's address space (CUDA IPC; plain peer memory, no NVLink
// multicast objects).  A launch copies this rank's slice into every rank's
// buffer at offset rank * slice; after a CTA barrier one thread makes the
// stores visible system-wide with a single fence, adds one to this rank's
// counter slot on every rank (relaxed, system scope), and waits (polling with
// system-scope acquire loads, bounded) until every rank's slot in this rank's
// counters has reached this launch's target.  One fence per
// launch instead of one per thread or per atomic: measured 6-7 us per gather
// on two B200s in a CUDA graph, against 16-18 us with release atomics and
// per-thread fences and 21-23 us for NCCL's all-gather.  Counters only grow: with a fixed number of
// CTAs per launch, the k-th launch of a rank targets k * kGatherCtas, which
// each CTA derives from the value its own increment of its own slot returned,
// so captured graphs can be replayed without resetting anything.  All ranks
// must make the same sequence of launches.  A wait that runs out sets bit
// kStatusPeerTimeout in the caller's status word and returns.
#include "vkc_common.cuh"

#include <cstring>

namespace vkc {
namespace {

constexpr int kGatherCtas = 1;
constexpr int kGatherThreads = 512;

__global__ void __launch_bounds__(kGatherThreads) allgather_kernel(const float4* __restrict__ src,
                                                                   float* const* dsts, unsigned* const* ctrs,
                                                                   int slice4, int rank, int world,
                                                                   unsigned* status) {
    pdl_launch_dependents();
    pdl_wait();  // the slice comes from the previous kernel
    const int stride = gridDim.x * blockDim.x;
    for (int p = 0; p < world; ++p) {
        float4* d = reinterpret_cast<float4*>(dsts[p]) + static_cast<size_t>(rank) * slice4;
        for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < slice4; i += stride) d[i] = src[i];
    }
    __syncthreads();  // the CTA's stores, ordered before thread 0's fence below
    if (threadIdx.x == 0) {
        fence_acq_rel_sys();  // release: the slice stores before the arrivals
        unsigned target = 0;
        for (int p = 0; p < world; ++p) {
            if (p == rank) {
                const unsigned old = atom_add_relaxed_sys(ctrs[p] + rank, 1u);
                target = (old / gridDim.x + 1) * gridDim.x;
            } else {
                red_add_relaxed_sys(ctrs[p] + rank, 1u);
            }
        }
        const unsigned* mine = ctrs[rank];
        bool ok = true;
        for (int q = 0; q < world && ok; ++q) {
            uint32_t it = 0;
            // acquire: the peers' slices are read after their arrivals
            while (static_cast<int>(ld_acquire_sys(mine + q) - target) < 0) {
                if (++it > kSpinLimit) {
                    ok = false;
                    break;
                }
            }
        }
        if (!ok) atomicOr(status, kStatusPeerTimeout);
    }
    __syncthreads();
}

// All-reduce with residual for K-split projections: every rank holds a
// partial output vector (its K slice of the product); the slices are stored
// into slot `rank` of every rank's partial buffer [world][n], the same
// arrival protocol as above runs, and each rank then writes
// out = residual + sum over ranks (in rank order, so every rank computes the
// same bits) of the slots.
__global__ void __launch_bounds__(kGatherThreads) allreduce_residual_kernel(
    const float4* __restrict__ part, float* const* slots, unsigned* const* ctrs, int n4, int rank, int world,
    const float4* __restrict__ residual, float4* __restrict__ out, unsigned* status) {
    pdl_launch_dependents();
    pdl_wait();  // the partial comes from the previous kernel
    const int stride = gridDim.x * blockDim.x;
    for (int p = 0; p < world; ++p) {
        float4* d = reinterpret_cast<float4*>(slots[p]) + static_cast<size_t>(rank) * n4;
        for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += stride) d[i] = part[i];
    }
    __syncthreads();
    __shared__ int s_ok;
    if (threadIdx.x == 0) {
        fence_acq_rel_sys();
        unsigned target = 0;
        for (int p = 0; p < world; ++p) {
            if (p == rank) {
                const unsigned old = atom_add_relaxed_sys(ctrs[p] + rank, 1u);
                target = (old / gridDim.x + 1) * gridDim.x;
            } else {
                red_add_relaxed_sys(ctrs[p] + rank, 1u);
            }
        }
        const unsigned* mine = ctrs[rank];
        bool ok = true;
        for (int q = 0; q < world && ok; ++q) {
            uint32_t it = 0;
            while (static_cast<int>(ld_acquire_sys(mine + q) - target) < 0) {
                if (++it > kSpinLimit) {
                    ok = false;
                    break;
                }
            }
        }
        if (!ok) atomicOr(status, kStatusPeerTimeout);
        s_ok = ok;
    }
    __syncthreads();
    const float4* mine4 = reinterpret_cast<const float4*>(slots[rank]);
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += stride) {
        float4 a = residual[i];
        for (int q = 0; q < world; ++q) {
            const float4 v = __ldcg(mine4 + static_cast<size_t>(q) * n4 + i);
            a.x += v.x;
            a.y += v.y;
            a.z += v.z;
            a.w += v.w;
        }
        out[i] = a;
    }
}

// Completion of a gathered GEMV (vkc_rmsnorm_gemv_gather), launched after it
// on the same stream: once the GEMV has finished (its stores into every
// rank's vector performed), one system fence and one arrival on counter `rank`
// of every rank; then lanes wait, one source rank each, until every rank's
// counter slot here has reached this wait's number (`step_word`, device,
// counts this rank's waits), with acquire loads, bounded
// (kStatusPeerTimeout on expiry).
__global__ void __launch_bounds__(32) gather_wait_kernel(unsigned* const* ctrs, int rank, int world,
                                                         unsigned* step_word, unsigned* status) {
    __shared__ unsigned s_step;
    pdl_wait();  // the GEMV's stores, and the previous wait's step
    if (threadIdx.x == 0) {
        s_step = *step_word + 1u;
        *step_word = s_step;
        fence_acq_rel_sys();  // the GEMV's stores (and the step) before the arrivals
        for (int q = 0; q < world; ++q) red_add_relaxed_sys(ctrs[q] + rank, 1u);
    }
    __syncwarp();
    const unsigned target = __shfl_sync(0xffffffffu, threadIdx.x == 0 ? s_step : 0u, 0);
    pdl_launch_dependents();
    const unsigned* mine = ctrs[rank];
    for (int q = threadIdx.x; q < world; q += 32) {
        const uint64_t deadline = globaltimer_ns() + kPeerWaitNs;
        uint32_t it = 0;
        while (static_cast<int>(ld_acquire_sys(mine + q) - target) < 0) {
            if ((++it & 63u) == 0 && globaltimer_ns() > deadline) {
                atomicOr(status, kStatusPeerTimeout);
                break;
            }
        }
    }
}

}  // namespace
}  // namespace vkc

using namespace vkc;

extern "C" {

int vkc_gather_wait(unsigned* const* counters, int rank, int world, unsigned* step_word, unsigned* status,
                    void* stream) {
    if (!counters || !step_word || !status) return set_error(kErrArg, "null gather-wait pointer");
    if (world < 1 || world > 1024 || rank < 0 || rank >= world) return set_error(kErrArg, "rank %d of world %d", rank, world);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1, 1, 1);
    cfg.blockDim = dim3(32, 1, 1);
    cfg.stream = static_cast<cudaStream_t>(stream);
    cudaLaunchAttribute attrs[2];
    cfg.attrs = attrs;
    cfg.numAttrs = launch_attrs(attrs, 1);
    VKC_CUDA_TRY(cudaLaunchKernelEx(&cfg, gather_wait_kernel, counters, rank, world, step_word, status));
    return kOk;
}

int vkc_allgather_p2p(const float* src, void* const* dsts, unsigned* const* counters, int slice_floats, int rank,
                      int world, unsigned* status, void* stream) {
    if (!src || !dsts || !counters || !status) return set_error(kErrArg, "null all-gather pointer");
    if (world < 1 || rank < 0 || rank >= world) return set_error(kErrArg, "rank %d of world %d", rank, world);
    if (slice_floats <= 0 || slice_floats % 4 != 0)
        return set_error(kErrArg, "slice of %d floats (must be a positive multiple of 4)", slice_floats);
    if (reinterpret_cast<uintptr_t>(src) % 16 != 0) return set_error(kErrArg, "source must be 16-byte aligned");
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(kGatherCtas, 1, 1);
    cfg.blockDim = dim3(kGatherThreads, 1, 1);
    cfg.stream = static_cast<cudaStream_t>(stream);
    cudaLaunchAttribute attrs[2];
    cfg.attrs = attrs;
    cfg.numAttrs = launch_attrs(attrs, 1);
    VKC_CUDA_TRY(cudaLaunchKernelEx(&cfg, allgather_kernel, reinterpret_cast<const float4*>(src),
                                    reinterpret_cast<float* const*>(dsts), counters, slice_floats / 4, rank, world,
                                    status));
    return kOk;
}

int vkc_allreduce_residual_p2p(const float* part, void* const* slots, unsigned* const* counters, int n, int rank,
                               int world, const float* residual, float* out, unsigned* status, void* stream) {
    if (!part || !slots || !counters || !residual || !out || !status)
        return set_error(kErrArg, "null all-reduce pointer");
    if (world < 1 || rank < 0 || rank >= world) return set_error(kErrArg, "rank %d of world %d", rank, world);
    if (n <= 0 || n % 4 != 0) return set_error(kErrArg, "vector of %d floats (must be a positive multiple of 4)", n);
    if ((reinterpret_cast<uintptr_t>(part) | reinterpret_cast<uintptr_t>(residual) |
         reinterpret_cast<uintptr_t>(out)) % 16 != 0)
        return set_error(kErrArg, "part, residual and out must be 16-byte aligned");
    if (out == part) return set_error(kErrArg, "out must not alias part");
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(kGatherCtas, 1, 1);
    cfg.blockDim = dim3(kGatherThreads, 1, 1);
    cfg.stream = static_cast<cudaStream_t>(stream);
    cudaLaunchAttribute attrs[2];
    cfg.attrs = attrs;
    cfg.numAttrs = launch_attrs(attrs, 1);
    VKC_CUDA_TRY(cudaLaunchKernelEx(&cfg, allreduce_residual_kernel, reinterpret_cast<const float4*>(part),
                                    reinterpret_cast<float* const*>(slots), counters, n / 4, rank, world,
                                    reinterpret_cast<const float4*>(residual), reinterpret_cast<float4*>(out),
                                    status));
    return kOk;
}

// ---- peer memory: one allocation per rank, shared through CUDA IPC --------

int vkc_ipc_alloc(size_t bytes, void** ptr, void* handle) {
    if (!ptr || !handle || bytes == 0) return set_error(kErrArg, "vkc_ipc_alloc: null pointer or zero size");
    void* p = nullptr;
    VKC_CUDA_TRY(cudaMalloc(&p, bytes));
    VKC_CUDA_TRY(cudaMemset(p, 0, bytes));
    cudaIpcMemHandle_t h;
    const cudaError_t e = cudaIpcGetMemHandle(&h, p);
    if (e != cudaSuccess) {
        cudaFree(p);
        return set_error(kErrCuda, "cudaIpcGetMemHandle failed: %s", cudaGetErrorString(e));
    }
    memcpy(handle, &h, sizeof h);
    *ptr = p;
    return kOk;
}

// Maps a peer's allocation into the current device's context (peer access is
// enabled on first use).
int vkc_ipc_open(const void* handle, void** ptr) {
    if (!ptr || !handle) return set_error(kErrArg, "vkc_ipc_open: null pointer");
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof h);
    VKC_CUDA_TRY(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess));
    return kOk;
}

int vkc_ipc_close(void* ptr) {
    VKC_CUDA_TRY(cudaIpcCloseMemHandle(ptr));
    return kOk;
}

int vkc_ipc_free(void* ptr) {
    VKC_CUDA_TRY(cudaFree(ptr));
    return kOk;
}

}  // extern "C"
