// Decode attention (one new token) over an fp16 KV cache, sm_100a:
// Att-full-FP16 (shader/Att-full-FP16.comp).
//
// Semantics: for query head h the key/value head is kv = h / G (G = n_q/n_kv,
// shader/Att-full-FP16.comp:34); s_t = scale * q_h . K[t, kv];
// out_h = sum_t e^{s_t} V[t, kv] / sum_t e^{s_t}.  The running maximum is
// subtracted before exponentiation (a softmax identity; the shader
// exponentiates raw scores, comp:66).
//
// Cache layouts are the shader's: K token-major, K[t][kv][d] at
// (t*n_kv + kv)*hd + d (comp:55-59); V in 8-dimension chunks, 16 bytes per
// token, V[kv][d/8][t][d%8] (comp:69-73), so for one head and one chunk the
// tokens are a contiguous 16-byte stream.
//
// Decomposition (split-KV): CTA (split, kv) owns T consecutive tokens of one
// KV head and serves all G query heads of that head, so every K and V byte is
// read once.  Phase 1: lanes split a K row into 16-byte chunks and reduce the
// partial dots over the row's lanes.  Phase 2: per-head max and exponentials
// in shared memory.  Phase 3: warps take V dimension chunks, lanes take tokens
// (512 contiguous bytes per warp load), and a butterfly transpose-reduction
// leaves lane l with output (head, dim) pair l.  Each CTA writes its (max,
// sum, unnormalised output) to a workspace; the last CTA of a KV head to
// finish (atomic ticket) merges the splits and resets the ticket.
#include "vkc_common.cuh"

#include <cuda_fp16.h>

#include <mutex>


namespace vkc {
namespace {

constexpr int kAttThreads = 256;
constexpr float kLog2e = 1.4426950408889634f;

struct AttnParams {
    const void* q;
    int q_bits;  // 16 (fp16) or 32 (fp32)
    const uint4* kc;
    const uint4* vc;
    float* out;
    float* ws;          // [n_q][splits][hd + 2] : acc[hd], m, l
    unsigned* tickets;  // [n_kv]
    int n_q, n_kv, hd, ctx, splits, tpc;
    int ctx_cap;        // V run length per (head, chunk): the cache capacity
    float scale_log2;   // scale * log2(e)
};

__device__ __forceinline__ void half8_to_float(const uint4 c, float (&v)[8]) {
    const uint32_t w[4] = {c.x, c.y, c.z, c.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
        v[2 * i] = f.x;
        v[2 * i + 1] = f.y;
    }
}

template <int G>
__global__ void __launch_bounds__(kAttThreads) attention_decode_kernel(const AttnParams p) {
    extern __shared__ float sc[];  // [G][tpc] scores, then probabilities
    __shared__ float stat[G][2];   // per head: max, sum
    __shared__ float wred[kAttThreads / 32][G];
    __shared__ unsigned s_ticket;

    const int split = blockIdx.x, kv = blockIdx.y;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int hd = p.hd, chunks = hd / 8;
    const int t0 = split * p.tpc;
    const int T = min(p.tpc, p.ctx - t0);
    const int h0 = kv * G;

    pdl_launch_dependents();
    pdl_wait();

    // ---- phase 1: scores ----------------------------------------------------
    // A K row of hd halves is `chunks` 16-byte pieces; `lpt` lanes share a row.
    int lpt = 1;
    while (lpt < chunks) lpt <<= 1;  // power of two >= chunks, <= 32
    const int rows_per_warp = 32 / lpt;
    const int sub = lane % lpt, row_in_warp = lane / lpt;
    float qv[G][8];
#pragma unroll
    for (int g = 0; g < G; ++g) {
        if (sub >= chunks) {
#pragma unroll
            for (int i = 0; i < 8; ++i) qv[g][i] = 0.f;
        } else if (p.q_bits == 16) {
            const uint4 qc = reinterpret_cast<const uint4*>(p.q)[((h0 + g) * hd) / 8 + sub];
            half8_to_float(qc, qv[g]);
        } else {
            const float4* q4 = reinterpret_cast<const float4*>(p.q) + ((h0 + g) * hd) / 4 + 2 * sub;
            const float4 a = q4[0], b = q4[1];
            qv[g][0] = a.x; qv[g][1] = a.y; qv[g][2] = a.z; qv[g][3] = a.w;
            qv[g][4] = b.x; qv[g][5] = b.y; qv[g][6] = b.z; qv[g][7] = b.w;
        }
    }
    const size_t krow = static_cast<size_t>(p.n_kv) * chunks;  // uint4 per token
    const int step = (kAttThreads / 32) * rows_per_warp;
    for (int tb = warp * rows_per_warp; tb < T; tb += step * 4) {
        uint4 kc[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int t = tb + u * step + row_in_warp;
            kc[u] = (t < T && sub < chunks)
                        ? ld_stream(p.kc + static_cast<size_t>(t0 + t) * krow + kv * chunks + sub)
                        : make_uint4(0u, 0u, 0u, 0u);
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            float kf[8];
            half8_to_float(kc[u], kf);
            float d[G];
#pragma unroll
            for (int g = 0; g < G; ++g) {
                float a = 0.f;
#pragma unroll
                for (int i = 0; i < 8; ++i) a = fmaf(qv[g][i], kf[i], a);
                d[g] = a;
            }
#pragma unroll
            for (int o = 1; o < 32; o <<= 1)
                if (o < lpt)
#pragma unroll
                    for (int g = 0; g < G; ++g) d[g] += __shfl_xor_sync(0xffffffffu, d[g], o);
            const int t = tb + u * step + row_in_warp;
            if (sub == 0 && t < T)
#pragma unroll
                for (int g = 0; g < G; ++g) sc[g * p.tpc + t] = d[g] * p.scale_log2;
        }
    }
    __syncthreads();

    // ---- phase 2: softmax statistics (base 2) -------------------------------
    float mx[G];
#pragma unroll
    for (int g = 0; g < G; ++g) mx[g] = -INFINITY;
    for (int t = tid; t < T; t += kAttThreads)
#pragma unroll
        for (int g = 0; g < G; ++g) mx[g] = fmaxf(mx[g], sc[g * p.tpc + t]);
#pragma unroll
    for (int g = 0; g < G; ++g) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx[g] = fmaxf(mx[g], __shfl_xor_sync(0xffffffffu, mx[g], o));
        if (lane == 0) wred[warp][g] = mx[g];
    }
    __syncthreads();
    if (tid < G) {
        float m = -INFINITY;
        for (int w = 0; w < kAttThreads / 32; ++w) m = fmaxf(m, wred[w][tid]);
        stat[tid][0] = m;
    }
    __syncthreads();
    float sm[G];
#pragma unroll
    for (int g = 0; g < G; ++g) sm[g] = 0.f;
    for (int t = tid; t < T; t += kAttThreads)
#pragma unroll
        for (int g = 0; g < G; ++g) {
            const float e = exp2f(sc[g * p.tpc + t] - stat[g][0]);
            sc[g * p.tpc + t] = e;
            sm[g] += e;
        }
#pragma unroll
    for (int g = 0; g < G; ++g) {
        sm[g] = warp_sum(sm[g]);
        if (lane == 0) wred[warp][g] = sm[g];
    }
    __syncthreads();
    if (tid < G) {
        float s = 0.f;
        for (int w = 0; w < kAttThreads / 32; ++w) s += wred[w][tid];
        stat[tid][1] = s;
    }
    __syncthreads();

    // ---- phase 3: probabilities x V ------------------------------------------
    const size_t vrun = static_cast<size_t>(p.ctx_cap);  // uint4 per (kv, chunk) run
    for (int c = warp; c < chunks; c += kAttThreads / 32) {
        float acc[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) acc[i] = 0.f;
        const uint4* vbase = p.vc + (static_cast<size_t>(kv) * chunks + c) * vrun + t0;
        for (int tb = 0; tb < T; tb += 32 * 4) {
            uint4 vchunk[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int t = tb + u * 32 + lane;
                vchunk[u] = t < T ? ld_stream(vbase + t) : make_uint4(0u, 0u, 0u, 0u);
            }
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int t = tb + u * 32 + lane;
                float vf[8];
                half8_to_float(vchunk[u], vf);
#pragma unroll
                for (int g = 0; g < G; ++g) {
                    const float pr = t < T ? sc[g * p.tpc + t] : 0.f;
#pragma unroll
                    for (int i = 0; i < 8; ++i) acc[g * 8 + i] = fmaf(pr, vf[i], acc[g * 8 + i]);
                }
            }
        }
        // Butterfly transpose-reduction: lane l ends with the total of acc[l].
#pragma unroll
        for (int o = 16, n = 32; o >= 1; o >>= 1, n >>= 1) {
            const bool upper = (lane & o) != 0;
#pragma unroll
            for (int i = 0; i < n / 2; ++i) {
                const float send = upper ? acc[i] : acc[i + n / 2];
                const float keep = upper ? acc[i + n / 2] : acc[i];
                acc[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
            }
        }
        const int g = lane / 8, i = lane % 8;
        if (g < G) {
            const int h = h0 + g;
            p.ws[(static_cast<size_t>(h) * p.splits + split) * (hd + 2) + c * 8 + i] = acc[0];
        }
    }
    if (tid < G) {
        float* rec = p.ws + (static_cast<size_t>(h0 + tid) * p.splits + split) * (hd + 2) + hd;
        rec[0] = stat[tid][0];
        rec[1] = stat[tid][1];
    }

    // ---- merge: the last split of this KV head combines all splits ----------
    __threadfence();
    __syncthreads();
    if (tid == 0) s_ticket = atomicAdd(p.tickets + kv, 1u);
    __syncthreads();
    if (s_ticket != static_cast<unsigned>(p.splits - 1)) return;
    __threadfence();
    for (int e = tid; e < G * hd; e += kAttThreads) {
        const int g = e / hd, d = e % hd, h = h0 + g;
        const float* base = p.ws + static_cast<size_t>(h) * p.splits * (hd + 2);
        float m = -INFINITY;
        for (int s = 0; s < p.splits; ++s) m = fmaxf(m, __ldcg(base + s * (hd + 2) + hd));
        float num = 0.f, den = 0.f;
        for (int s = 0; s < p.splits; ++s) {
            const float* r = base + s * (hd + 2);
            const float w = exp2f(__ldcg(r + hd) - m);
            num = fmaf(w, __ldcg(r + d), num);
            den = fmaf(w, __ldcg(r + hd + 1), den);
        }
        p.out[static_cast<size_t>(h) * hd + d] = num / den;
    }
    if (tid == 0) p.tickets[kv] = 0u;
}

}  // namespace

// Splits and tokens per CTA for a context length: about two CTAs per SM.
static void attention_plan(int n_kv, int ctx, int* splits, int* tpc) {
    int target = (2 * 148 + n_kv - 1) / n_kv;
    int t = (ctx + target - 1) / target;
    t = ((t + 31) / 32) * 32;
    if (t < 32) t = 32;
    *tpc = t;
    *splits = (ctx + t - 1) / t;
}

size_t attention_workspace_bytes(int n_q, int n_kv, int hd, int ctx) {
    int splits, tpc;
    attention_plan(n_kv, ctx, &splits, &tpc);
    return 256 + static_cast<size_t>(n_q) * splits * (hd + 2) * sizeof(float) +
           static_cast<size_t>(n_kv) * sizeof(unsigned);
}

int attention_launch(const void* q, int q_bits, const void* kc, const void* vc, float* out,
                     int n_q, int n_kv, int hd, int ctx, int ctx_cap, float scale, void* ws, size_t ws_bytes,
                     cudaStream_t stream) {
    if (!q || !kc || !vc || !out) return set_error(kErrArg, "null attention pointer");
    if (q_bits != 16 && q_bits != 32) return set_error(kErrArg, "q_bits=%d (expected 16 or 32)", q_bits);
    if (n_q <= 0 || n_kv <= 0 || n_q % n_kv != 0)
        return set_error(kErrArg, "n_q=%d must be a positive multiple of n_kv=%d", n_q, n_kv);
    const int G = n_q / n_kv;
    if (G != 1 && G != 2 && G != 4)
        return set_error(kErrUnsupported, "query heads per KV head %d (supported: 1, 2, 4)", G);
    if (hd <= 0 || hd % 8 != 0 || hd > 256)
        return set_error(kErrArg, "head_dim=%d must be a multiple of 8 in [8, 256]", hd);
    if (ctx <= 0) return set_error(kErrArg, "context length %d must be positive", ctx);
    if (ctx_cap < ctx) return set_error(kErrArg, "cache capacity %d below the context length %d", ctx_cap, ctx);
    if ((reinterpret_cast<uintptr_t>(kc) | reinterpret_cast<uintptr_t>(vc) |
         reinterpret_cast<uintptr_t>(q)) % 16 != 0)
        return set_error(kErrArg, "q and the K/V caches must be 16-byte aligned");
    int splits, tpc;
    attention_plan(n_kv, ctx, &splits, &tpc);
    const size_t need = attention_workspace_bytes(n_q, n_kv, hd, ctx);
    if (!ws) return set_error(kErrArg, "attention workspace missing");
    if (ws_bytes < need)
        return set_error(kErrArg, "attention workspace holds %zu bytes, needs %zu", ws_bytes, need);
    AttnParams p = {};
    p.q = q;
    p.q_bits = q_bits;
    p.kc = static_cast<const uint4*>(kc);
    p.vc = static_cast<const uint4*>(vc);
    p.out = out;
    p.tickets = reinterpret_cast<unsigned*>(ws);
    p.ws = reinterpret_cast<float*>(static_cast<char*>(ws) + 256);
    p.n_q = n_q;
    p.n_kv = n_kv;
    p.hd = hd;
    p.ctx = ctx;
    p.ctx_cap = ctx_cap;
    p.splits = splits;
    p.tpc = tpc;
    p.scale_log2 = scale * kLog2e;
    if (n_kv * sizeof(unsigned) > 256) return set_error(kErrUnsupported, "more than 64 KV heads");
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(splits, n_kv, 1);
    cfg.blockDim = dim3(kAttThreads, 1, 1);
    cfg.dynamicSmemBytes = static_cast<size_t>(G) * tpc * sizeof(float);
    cfg.stream = stream;
    cudaLaunchAttribute attrs[2];
    cfg.attrs = attrs;
    cfg.numAttrs = launch_attrs(attrs, 1);
    switch (G) {
        case 1: VKC_CUDA_TRY(cudaLaunchKernelEx(&cfg, attention_decode_kernel<1>, p)); break;
        case 2: VKC_CUDA_TRY(cudaLaunchKernelEx(&cfg, attention_decode_kernel<2>, p)); break;
        default: VKC_CUDA_TRY(cudaLaunchKernelEx(&cfg, attention_decode_kernel<4>, p)); break;
    }
    return kOk;
}

}  // namespace vkc

using namespace vkc;

extern "C" {

size_t vkc_attention_workspace_bytes(int n_q, int n_kv, int head_dim, int ctx) {
    return attention_workspace_bytes(n_q, n_kv, head_dim, ctx);
}

int vkc_attention_decode(const void* q, int q_bits, const void* kcache, const void* vcache,
                         float* out, int n_q, int n_kv, int head_dim, int ctx, float scale,
                         void* workspace, size_t workspace_bytes, void* stream) {
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (!workspace) {
        const size_t need = attention_workspace_bytes(n_q > 0 ? n_q : 1, n_kv > 0 ? n_kv : 1,
                                                      head_dim > 0 ? head_dim : 8, ctx > 0 ? ctx : 1);
        void* base = nullptr;
        if (int e = device_workspace(need + kWorkspaceHeader, &base, s)) return e;
        workspace = static_cast<char*>(base) + kWorkspaceHeader;
        workspace_bytes = need;
    }
    return attention_launch(q, q_bits, kcache, vcache, out, n_q, n_kv, head_dim, ctx, ctx, scale,
                            workspace, workspace_bytes, s);
}

int vkc_attention_decode_cache(const void* q, int q_bits, const void* kcache, const void* vcache, float* out,
                               int n_q, int n_kv, int head_dim, int ctx, int ctx_cap, float scale, void* workspace,
                               size_t workspace_bytes, void* stream) {
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (!workspace) {
        const size_t need = attention_workspace_bytes(n_q > 0 ? n_q : 1, n_kv > 0 ? n_kv : 1,
                                                      head_dim > 0 ? head_dim : 8, ctx > 0 ? ctx : 1);
        void* base = nullptr;
        if (int e = device_workspace(need + kWorkspaceHeader, &base, s)) return e;
        workspace = static_cast<char*>(base) + kWorkspaceHeader;
        workspace_bytes = need;
    }
    return attention_launch(q, q_bits, kcache, vcache, out, n_q, n_kv, head_dim, ctx, ctx_cap, scale, workspace,
                            workspace_bytes, s);
}

// ---------------------------------------------------------------------------
// Allocation-free variant.
//
// vkc_attention_decode needs scratch for its split partials and merge tickets:
// either a buffer the caller allocated or one the library cudaMallocs on first
// use.  Some callers can do neither at the moment they run attention: an
// engine that has handed all of HBM to its own pool (weights and KV cache) so
// a cudaMalloc would fail or fragment it, a decode loop that must not take the
// device-wide synchronisation cudaMalloc/cudaFree can imply, or a plugin whose
// host forbids allocations inside its callbacks.  This entry point uses a
// fixed scratch array that is part of the loaded library image instead.
// ---------------------------------------------------------------------------
namespace vkc {
namespace {
// Scratch of the allocation-free entry point: 2 MiB, in every device's image
// of this library for as long as the library stays loaded.  Bytes [0, 256)
// hold the per-KV-head merge tickets, which must be zero when a call starts;
// each call leaves them at zero.
constexpr size_t kNoAllocScratchBytes = 2u << 20;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_noalloc_mu;
void* g_noalloc_addr[64] = {};  // device address of g_noalloc_scratch per device

// Once per device, with that device current: look up the array's device
// address (in host code its name is only a stand-in) and clear the tickets.
int noalloc_scratch(void** out, cudaStream_t stream) {
    int dev = 0;
    VKC_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) return set_error(kErrUnsupported, "device ordinal %d", dev);
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (!g_noalloc_addr[dev]) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess)
            return set_error(kErrCuda, "cudaGetSymbolAddress(attention scratch) failed: %s", cudaGetErrorString(e));
        VKC_CUDA_TRY(cudaMemsetAsync(p, 0, kWorkspaceHeader, stream));
        g_noalloc_addr[dev] = p;
    }
    *out = g_noalloc_addr[dev];
    return kOk;
}
}  // namespace
}  // namespace vkc

size_t vkc_attention_noalloc_max_scratch(void) { return kNoAllocScratchBytes; }

int vkc_attention_decode_noalloc(const void* q, int q_bits, const void* kcache, const void* vcache, float* out,
                                 int n_q, int n_kv, int head_dim, int ctx, float scale, void* stream) {
    if (n_q <= 0 || n_kv <= 0 || head_dim <= 0 || ctx <= 0)
        return set_error(kErrArg, "n_q=%d, n_kv=%d, head_dim=%d and ctx=%d must be positive", n_q, n_kv, head_dim,
                         ctx);
    const size_t need = attention_workspace_bytes(n_q, n_kv, head_dim, ctx);
    if (need > kNoAllocScratchBytes)
        return set_error(kErrArg,
                         "attention with %d query heads, head_dim %d and context %d needs %zu bytes of scratch; "
                         "the allocation-free entry point holds %zu (use vkc_attention_decode)",
                         n_q, head_dim, ctx, need, kNoAllocScratchBytes);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    void* scratch = nullptr;
    if (int e = noalloc_scratch(&scratch, s)) return e;
    return attention_launch(q, q_bits, kcache, vcache, out, n_q, n_kv, head_dim, ctx, ctx, scale, scratch,
                            kNoAllocScratchBytes, s);
}

}  // extern "C"
