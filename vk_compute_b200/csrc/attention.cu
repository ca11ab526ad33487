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
// tokens are a contiguous 16-byte stream.  A cache allocated for ctx_cap
// tokens has V runs ctx_cap long.
//
// Decomposition (split-KV, flash-decoding): CTA (split, kv) owns a range of
// tokens of one KV head and serves all G query heads of that head, so every K
// and V byte is read once.  The range streams through a three-stage ring of
// (K, V) sub-tiles in shared memory filled by 16-byte cp.async copies (zero
// fill past the end).  Per sub-tile: lanes split a
// K row into 16-byte chunks and reduce the partial dots; one warp per head
// updates the running maximum and sum (base-2 online softmax) and rescales;
// threads own one output dimension for all G heads and a share of the tokens
// for P.V.  Each CTA writes (max, sum, unnormalised output) to a workspace;
// the last CTA of a KV head to finish (atomic ticket) merges the splits in
// split order and resets the ticket.
#include "vkc_common.cuh"

#include <cuda_fp16.h>

#include <mutex>
#include <type_traits>

#include "attention_kernels.cuh"

namespace vkc {


// Tokens per sub-tile for a head size: one ring stage holds about 32 KB.
static int attention_subtile(int hd) {
    int tt = (8192 / hd) & ~31;
    return tt < 32 ? 32 : (tt > 256 ? 256 : tt);
}

// Which kernel serves a shape, and how the context is split.
struct AttnPlan {
    enum Kind { kSimt, kMma, kSlice } kind;
    int splits;   // CTAs per KV head (grid x)
    int tpc;      // tokens per CTA (a multiple of 16)
    int records;  // partial records per query head in the workspace
    bool per_sm;  // token-slice kernel in its per-SM shape (no clusters)
    int stages;   // per-SM shape: ring stages (kFaDeepStages, or kAttStages to fit half an SM)
    int groups;   // per-SM shape: warp groups of kFaThreads per CTA
};

// Attention plan (vkc_set_attention_plan), per host thread: 0 chooses per
// shape, 1 the clustered token-slice shape, 2 the per-SM shape, 3 the per-SM
// shape with a 3-stage ring (at most half an SM's shared memory, so a kernel
// next to it in the stream can be resident beside it), 4 two such CTAs per
// SM over twice the splits (eight warps and the deep ring's bytes in flight
// per SM), 5 the per-SM shape with two warp groups per CTA, each streaming
// and processing alternate sub-tiles of the CTA's range through its half of
// the deep ring (eight warps per SM, one record per CTA).  The automatic
// choice is 5 wherever the per-SM shape applies.  (Per-SM CTAs in clusters
// of 8 were measured too: B200's GPCs hold too few such clusters at once,
// and the grid ran in two waves.)
thread_local int g_attn_plan = 0;

int current_sm_count() {
    static int cached[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    if (cached[dev] == 0) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) return 148;
        cached[dev] = n;
    }
    return cached[dev];
}

// Splits: about two CTAs per SM (148 SMs), but at least three sub-tiles
// (~96 KB of cache) per CTA, so a small cache (a shard with one KV head) is
// not cut into many tiny splits whose merge would dominate.  The token-slice
// kernel groups its splits in clusters of kFaCluster and keeps one record per
// cluster; at most 32 clusters (256 CTAs) are launched, which two CTAs per SM
// hold at once.  A CTA's last sub-tile may be partial, and with clusters the
// last CTAs of a head may get no tokens at all.
static AttnPlan attention_plan(int n_q, int n_kv, int hd, int ctx) {
    AttnPlan pl;
    const int G = n_q / n_kv;
    const bool mma_g = G == 1 || G == 2 || G == 4 || G == 8;
    pl.kind = (hd == 64 || hd == 128) && mma_g ? AttnPlan::kSlice
              : (hd == 256 && mma_g)           ? AttnPlan::kMma
                                               : AttnPlan::kSimt;
    // At least three sub-tiles per CTA, two when the grid has only one or two
    // KV heads (the shards of a 4- or 8-way split): there the extra CTAs' bytes
    // in flight outweigh the longer merge (one KV head, 8192 tokens: 9.96
    // against 11.35 us; two: 10.87 against 12.0; four heads lose with two).
    const int min_tpc = (n_kv <= 2 ? 2 : 3) * (8192 / hd);
    const int by_size = (ctx + min_tpc - 1) / min_tpc;
    int target;
    if (pl.kind == AttnPlan::kSlice) {
        int nc = 32 / n_kv;
        const int nc_size = (by_size + kFaCluster - 1) / kFaCluster;
        if (nc_size < nc) nc = nc_size;
        if (nc < 1) nc = 1;
        target = nc * kFaCluster;
    } else {
        target = (2 * 148 + n_kv - 1) / n_kv;
        if (by_size < target) target = by_size;
        if (target < 1) target = 1;
    }
    int t = (ctx + target - 1) / target;
    t = ((t + 15) / 16) * 16;
    pl.tpc = t;
    pl.per_sm = false;
    pl.stages = kAttStages;
    pl.groups = 1;
    if (pl.kind == AttnPlan::kSlice) {
        pl.splits = target;
        pl.records = target / kFaCluster;
    } else {
        pl.splits = (ctx + t - 1) / t;
        pl.records = pl.splits;
    }
    if (pl.kind == AttnPlan::kSlice && g_attn_plan != 1) {
        // Per-SM shape: at most one CTA per SM over all KV heads, each with at
        // least two sub-tiles, its range streamed through the deep ring; the
        // splits of a head merge through the workspace.
        const int tt = 8192 / hd;
        const int ctas = (g_attn_plan == 4 ? 2 : 1) * current_sm_count();
        const int per_head = ctas / n_kv > 0 ? ctas / n_kv : 1;
        int tpc = (ctx + per_head - 1) / per_head;
        tpc = ((tpc + 15) / 16) * 16;
        if (tpc < 2 * tt) tpc = 2 * tt;
        const int splits = (ctx + tpc - 1) / tpc;
        // automatic choice: the per-SM shape when it gives every CTA at least
        // two sub-tiles and keeps the grid in one wave
        if (g_attn_plan >= 2 || splits * n_kv <= current_sm_count()) {
            pl.per_sm = true;
            pl.stages = g_attn_plan == 3 || g_attn_plan == 4 ? kAttStages : kFaDeepStages;
            pl.groups = g_attn_plan == 5 || g_attn_plan == 0 ? 2 : 1;
            pl.tpc = tpc;
            pl.splits = splits;
            pl.records = splits;
        }
    }
    return pl;
}

size_t attention_workspace_bytes(int n_q, int n_kv, int hd, int ctx) {
    const AttnPlan pl = attention_plan(n_q, n_kv, hd, ctx);
    return 256 + static_cast<size_t>(n_q) * pl.records * (hd + 4) * sizeof(float) +
           static_cast<size_t>(n_kv) * sizeof(unsigned);
}

int attention_launch(const void* q, int q_bits, const void* kc, const void* vc, float* out,
                     int n_q, int n_kv, int hd, int ctx, int ctx_cap, float scale, void* ws, size_t ws_bytes,
                     cudaStream_t stream, int stable = 0) {
    if (!q || !kc || !vc || !out) return set_error(kErrArg, "null attention pointer");
    if (q_bits != 16 && q_bits != 32) return set_error(kErrArg, "q_bits=%d (expected 16 or 32)", q_bits);
    if (n_q <= 0 || n_kv <= 0 || n_q % n_kv != 0)
        return set_error(kErrArg, "n_q=%d must be a positive multiple of n_kv=%d", n_q, n_kv);
    const int G = n_q / n_kv;
    if (hd <= 0 || hd % 8 != 0 || hd > 256)
        return set_error(kErrArg, "head_dim=%d must be a multiple of 8 in [8, 256]", hd);
    if (ctx <= 0) return set_error(kErrArg, "context length %d must be positive", ctx);
    const AttnPlan pl = attention_plan(n_q, n_kv, hd, ctx);
    if (pl.kind == AttnPlan::kSimt && G != 1 && G != 2 && G != 4)
        return set_error(kErrUnsupported,
                         "query heads per KV head %d (supported: 1, 2, 4; 8 with head_dim 64, 128 or 256)", G);
    if (ctx_cap < ctx) return set_error(kErrArg, "cache capacity %d below the context length %d", ctx_cap, ctx);
    if ((reinterpret_cast<uintptr_t>(kc) | reinterpret_cast<uintptr_t>(vc) | reinterpret_cast<uintptr_t>(q) |
         reinterpret_cast<uintptr_t>(out)) % 16 != 0)
        return set_error(kErrArg, "q, out and the K/V caches must be 16-byte aligned");
    const size_t need = attention_workspace_bytes(n_q, n_kv, hd, ctx);
    if (!ws) return set_error(kErrArg, "attention workspace missing");
    if (ws_bytes < need)
        return set_error(kErrArg, "attention workspace holds %zu bytes, needs %zu", ws_bytes, need);
    if (n_kv * sizeof(unsigned) > 256) return set_error(kErrUnsupported, "more than 64 KV heads");
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
    p.splits = pl.splits;
    p.tpc = pl.tpc;
    p.tt = attention_subtile(hd);
    p.scale_log2 = scale * kLog2e;
    p.pitch = hd + 4;
    p.stable = stable;
    // scratch of the final merge: staged records (when they fit) or (m, l), weights and group sums
    const size_t merge_min = ((static_cast<size_t>(G) * pl.records * 12 + 15) & ~size_t(15)) + kAttThreads * 16;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(pl.splits, n_kv, 1);
    cfg.blockDim = dim3(kAttThreads, 1, 1);
    cfg.stream = stream;
    cudaLaunchAttribute attrs[2];
    cfg.attrs = attrs;
    cfg.numAttrs = launch_attrs(attrs, pl.kind == AttnPlan::kSlice && !pl.per_sm ? kFaCluster : 1);
    auto go = [&](auto kern, size_t smem) -> int {
        if (merge_min > smem) smem = merge_min;
        cfg.dynamicSmemBytes = smem;
        p.smem = static_cast<int>(smem);
        if (int e = ensure_smem(reinterpret_cast<const void*>(kern), smem)) return e;
        VKC_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, p));
        return kOk;
    };
    if (pl.kind == AttnPlan::kSlice) {
        auto pick = [&](auto hd_tag) -> int {
            constexpr int HD = decltype(hd_tag)::value;
            cfg.blockDim = dim3(kFaThreads, 1, 1);
            if (pl.per_sm && pl.groups == 2) {
                constexpr int ST = kFaDeepStages;
                cfg.blockDim = dim3(2 * kFaThreads, 1, 1);
                const size_t smem = static_cast<size_t>(ST) * MmaGeo<HD>::SU * 16 + MmaGeo<HD>::q_bytes;
                switch (G) {
                    case 1: return go(attention_fa_kernel<1, HD, ST, 1, 2>, smem);
                    case 2: return go(attention_fa_kernel<2, HD, ST, 1, 2>, smem);
                    case 4: return go(attention_fa_kernel<4, HD, ST, 1, 2>, smem);
                    default: return go(attention_fa_kernel<8, HD, ST, 1, 2>, smem);
                }
            }
            if (pl.per_sm && pl.stages == kFaDeepStages) {
                constexpr int ST = kFaDeepStages;
                const size_t smem = static_cast<size_t>(ST) * MmaGeo<HD>::SU * 16 + MmaGeo<HD>::q_bytes;
                switch (G) {
                    case 1: return go(attention_fa_kernel<1, HD, ST, 1>, smem);
                    case 2: return go(attention_fa_kernel<2, HD, ST, 1>, smem);
                    case 4: return go(attention_fa_kernel<4, HD, ST, 1>, smem);
                    default: return go(attention_fa_kernel<8, HD, ST, 1>, smem);
                }
            }
            if (pl.per_sm) {
                constexpr int ST = kAttStages;
                const size_t smem = static_cast<size_t>(ST) * MmaGeo<HD>::SU * 16 + MmaGeo<HD>::q_bytes;
                switch (G) {
                    case 1: return go(attention_fa_kernel<1, HD, ST, 1>, smem);
                    case 2: return go(attention_fa_kernel<2, HD, ST, 1>, smem);
                    case 4: return go(attention_fa_kernel<4, HD, ST, 1>, smem);
                    default: return go(attention_fa_kernel<8, HD, ST, 1>, smem);
                }
            }
            const size_t smem = MmaGeo<HD>::ring_bytes + MmaGeo<HD>::q_bytes;
            switch (G) {
                case 1: return go(attention_fa_kernel<1, HD, kAttStages, kFaCluster>, smem);
                case 2: return go(attention_fa_kernel<2, HD, kAttStages, kFaCluster>, smem);
                case 4: return go(attention_fa_kernel<4, HD, kAttStages, kFaCluster>, smem);
                default: return go(attention_fa_kernel<8, HD, kAttStages, kFaCluster>, smem);
            }
        };
        if (hd == 64) return pick(std::integral_constant<int, 64>());
        return pick(std::integral_constant<int, 128>());
    }
    if (pl.kind == AttnPlan::kMma) {
        const size_t smem = MmaGeo<256>::smem_bytes;
        switch (G) {
            case 1: return go(attention_mma_kernel<1, 256>, smem);
            case 2: return go(attention_mma_kernel<2, 256>, smem);
            case 4: return go(attention_mma_kernel<4, 256>, smem);
            default: return go(attention_mma_kernel<8, 256>, smem);
        }
    }
    const int chunks = hd / 8;
    size_t smem = static_cast<size_t>(kAttStages) * att_stage_units(p.tt, chunks) * 16 +
                  static_cast<size_t>(G) * (hd + p.tt) * sizeof(float);
    const size_t red = static_cast<size_t>(kAttThreads / (hd / 2)) * G * hd * sizeof(float);
    if (red > smem) smem = red;
    switch (G) {
        case 1: return go(attention_decode_kernel<1>, smem);
        case 2: return go(attention_decode_kernel<2>, smem);
        default: return go(attention_decode_kernel<4>, smem);
    }
}

}  // namespace vkc

using namespace vkc;

extern "C" {

size_t vkc_attention_workspace_bytes(int n_q, int n_kv, int head_dim, int ctx) {
    return attention_workspace_bytes(n_q, n_kv, head_dim, ctx);
}

int vkc_set_attention_plan(int plan) {
    if (plan < 0 || plan > 5) return set_error(kErrArg, "attention plan %d (expected 0 to 5)", plan);
    g_attn_plan = plan;
    return kOk;
}
int vkc_get_attention_plan(void) { return g_attn_plan; }

int vkc_attention_plan_info(int n_q, int n_kv, int head_dim, int ctx, int* info) {
    if (!info) return set_error(kErrArg, "null info");
    if (n_q <= 0 || n_kv <= 0 || n_q % n_kv != 0 || head_dim <= 0 || ctx <= 0)
        return set_error(kErrArg, "bad attention shape");
    const AttnPlan pl = attention_plan(n_q, n_kv, head_dim, ctx);
    info[0] = pl.kind == AttnPlan::kSlice ? (pl.per_sm ? 2 : 1) : pl.kind == AttnPlan::kMma ? 3 : 4;
    info[1] = pl.splits;
    info[2] = pl.tpc;
    info[3] = pl.per_sm ? pl.stages : kAttStages;
    info[4] = pl.per_sm ? pl.groups : 1;
    info[5] = pl.kind == AttnPlan::kSlice && !pl.per_sm ? kFaCluster : 1;
    info[6] = pl.records;
    return kOk;
}

int vkc_attention_decode(const void* q, int q_bits, const void* kcache, const void* vcache,
                         float* out, int n_q, int n_kv, int head_dim, int ctx, float scale,
                         void* workspace, size_t workspace_bytes, void* stream) {
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (!workspace) {
        const size_t need = attention_workspace_bytes(n_q > 0 ? n_q : 1, n_kv > 0 ? n_kv : 1,
                                                      head_dim > 0 ? head_dim : 8, ctx > 0 ? ctx : 1);
        void* base = nullptr;
        if (int e = device_workspace(need + kWorkspaceHeader, &base, s, kWorkspaceAttention)) return e;
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
        if (int e = device_workspace(need + kWorkspaceHeader, &base, s, kWorkspaceAttention)) return e;
        workspace = static_cast<char*>(base) + kWorkspaceHeader;
        workspace_bytes = need;
    }
    return attention_launch(q, q_bits, kcache, vcache, out, n_q, n_kv, head_dim, ctx, ctx_cap, scale, workspace,
                            workspace_bytes, s);
}

// Decode step after an append: the kernel launched just before this one (the
// fused QKV projection) wrote only token ctx - 1 of the caches, and tokens
// [0, ctx - 1) come from earlier steps, so they are requested before the wait
// on that kernel.
int vkc_attention_decode_append(const void* q, int q_bits, const void* kcache, const void* vcache, float* out,
                                int n_q, int n_kv, int head_dim, int ctx, int ctx_cap, float scale, void* workspace,
                                size_t workspace_bytes, void* stream) {
    if (!workspace) return set_error(kErrArg, "attention workspace missing");
    return attention_launch(q, q_bits, kcache, vcache, out, n_q, n_kv, head_dim, ctx, ctx_cap, scale, workspace,
                            workspace_bytes, static_cast<cudaStream_t>(stream), ctx - 1);
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
void* g_noalloc_addr[64] = {};  // last address of g_noalloc_scratch seen per device

// On every call, with the calling device current: look up the array's device
// address in the current context (in host code its name is only a stand-in,
// and a context made after cudaDeviceReset, or by a plugin host, loads its own
// copy of the array).  When the address differs from the one this device had
// last time (the first call, or another context's copy), clear the tickets.
int noalloc_scratch(void** out, cudaStream_t stream) {
    int dev = 0;
    VKC_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) return set_error(kErrUnsupported, "device ordinal %d", dev);
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess)
        return set_error(kErrCuda, "cudaGetSymbolAddress(attention scratch) failed: %s", cudaGetErrorString(e));
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (g_noalloc_addr[dev] != p) {
        VKC_CUDA_TRY(cudaMemsetAsync(p, 0, kWorkspaceHeader, stream));
        g_noalloc_addr[dev] = p;
    }
    *out = p;
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
