/*
 * vk_compute_b200.h -- native C ABI of libvkcompute (sm_100a).
 *
 * Device pointers, plain sizes and a CUDA stream passed as void* (NULL = the
 * legacy default stream).  Every function returns 0 on success or a negative
 * status (VKC_ERR_*) with a message in vkc_last_error(); no function exits
 * the process.  Kernels are enqueued asynchronously on `stream`.
 *
 * Weight arguments use vk-compute's storage exactly:
 *   bits 32 / 16 / 8 / 4 -- fp32, fp16, u8 codes or u4 codes
 *   w      -- the transpose_block16 layout (src/data.c:198-222): chunk row r
 *             holds k in [r*128/bits, (r+1)*128/bits) of column j as 16 bytes
 *             at byte (r*N + j)*16; 16-byte aligned
 *   scale, zero -- fp32, [N/256][K] block-major (src/data.c:122-124);
 *             quantised weights dequantise as q*scale - zero; NULL for
 *             fp32/fp16 weights
 *   x, gamma -- fp32 [K]; y -- fp32 [N]
 * Each function names the reference shader whose computation it replaces
 * (paths relative to the vk-compute project root).
 */
#ifndef VK_COMPUTE_B200_H
#define VK_COMPUTE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define VKC_VERSION 1

#define VKC_OK 0
#define VKC_ERR_ARG (-1)
#define VKC_ERR_CUDA (-2)
#define VKC_ERR_UNSUPPORTED (-3)
#define VKC_ERR_TIMEOUT (-4)

/* Message of the last failed call on this thread. */
const char* vkc_last_error(void);
int vkc_version(void);
/* Launch later kernels with programmatic dependent launch (1) or plainly (0):
 * a kernel may then start streaming weights while its predecessor in the
 * stream finishes; activations are read only after the predecessor's writes
 * are visible. */
void vkc_set_pdl(int enable);
int vkc_get_pdl(void);
/* Timing of execute() for getExecutionTime (1, the default, as in the
 * reference) or none (0): every timed execute records two CUDA events around
 * its operators, which costs host time and keeps the next kernel from
 * starting early; a program that never calls getExecutionTime can turn it
 * off, after which getExecutionTime returns 0. */
void vkc_set_timing(int enable);
int vkc_get_timing(void);
/* Which kernel runs the single-vector GEMV family (vkc_gemv,
 * vkc_rmsnorm_gemv, -rope, -rope_kv, -swiglu, vkc_gemv_residual / _peer):
 * 0 (default) chooses per shape -- one CTA per SM (512 threads, leaving
 * half of each SM to the next launch), each with a balanced range
 * of whole-K output columns, when every SM gets at least 16 outputs and the
 * input is not a peer exchange; otherwise clusters that split K and reduce in
 * distributed shared memory.  1 always uses the cluster
 * kernel; 2 uses the one-CTA-per-SM kernel with 1024-thread CTAs wherever it
 * can run, 3 with 512-thread CTAs that leave half of each SM to the next
 * launch, 4 chooses per shape like 0 but with 1024-thread CTAs (for chains
 * whose other kernels need more than half of each SM).  The setting belongs to the calling host thread.  Results agree to
 * rounding.  No counterpart in the reference. */
int vkc_set_gemv_plan(int plan);
int vkc_get_gemv_plan(void);
/* Arithmetic of 8/4-bit weights on the one-CTA-per-SM kernel, for the calling
 * host thread.  1 (default): integer dot products -- each chunk row's folded
 * activations x*gamma*scale become 16-bit integers against the row's largest
 * magnitude (steps of 2^-15 of it), every code-times-activation sum is exact
 * in 32-bit integers (dp4a), and each row's sum is scaled once into an fp32
 * accumulator; about a third of the instructions per weight of 0.  0: fp32
 * fused multiply-adds on the exactly converted codes.  Dequantisation is
 * q*scale - zero either way; the two agree to about 1e-5 relative.  No
 * counterpart in the reference. */
void vkc_set_gemv_int_dot(int enable);
int vkc_get_gemv_int_dot(void);
/* 1 if `shader` ("GEMV-INT4.spv", ...) names an operator execute() runs. */
int vkc_has_operator(const char* shader);
/* Waits for the current device and returns its status word, whose flags
 * record a bounded device wait that gave up (the kernel then ends early and
 * its outputs are invalid): 0x1 a producer warp, 0x2 a consumer warp, 0x4 a
 * cluster's collecting CTA (split-K deposits), 0x8 a wait for another GPU's
 * data (peer timeout), 0x20 a grid-barrier wait of the persistent decoder
 * (the tcgen05 GEMM keeps its own word, flag 0x10).  `clear` resets the word.
 * No counterpart in the reference. */
int vkc_device_status(unsigned* status, int clear);
/* Bounds of those waits, in nanoseconds of the GPU clock: `peer_ns`, the
 * longest one thread waits in total for other GPUs' data in a fused exchange
 * (one deadline, started at its first wait); `cluster_ns`, the longest a
 * cluster's collecting CTA waits for the other CTAs' deposits into its shared
 * memory (at least ten times peer_ns, so it outlasts every wait that can hold
 * a depositing CTA back).  No counterpart in the reference. */
void vkc_wait_limits(uint64_t* peer_ns, uint64_t* cluster_ns);

/* y = W^T x.  Replaces shader/GEMV-FP16.comp, GEMV-INT8.comp, GEMV-INT4.comp
 * and gemv.comp (fp32), bindings {x, W, y[, s, z]}. */
int vkc_gemv(int bits, const void* w, const float* scale, const float* zero, const float* x,
             float* y, int N, int K, void* stream);

/* y = W^T (x * gamma * inv_rms), inv_rms = 1/sqrt(sum(x^2)/rms_dim + eps).
 * Replaces shader/RmsNorm-GEMV-FP16.comp, -INT8.comp, -INT4.comp and
 * RmsNorm-GEMV.comp (which fix rms_dim = 4096, eps = 1e-5). */
int vkc_rmsnorm_gemv(int bits, const void* w, const float* scale, const float* zero,
                     const float* x, const float* gamma, float* y, int N, int K, float eps,
                     int rms_dim, void* stream);

/* y = W^T x + residual (the decoder's O and down projections with their
 * residual connection fused).  No counterpart in the reference, whose driver
 * runs one operator and has no residual add. */
int vkc_gemv_residual(int bits, const void* w, const float* scale, const float* zero, const float* x,
                      const float* residual, float* y, int N, int K, void* stream);

/* RmsNorm-GEMV-Rope for a decoder's fused QKV projection with the KV-cache
 * append the reference lacks: outputs are q_rows of Q heads followed by
 * kv_rows of K and kv_rows of V heads (whole heads of head_dim), laid out as
 * [K heads | V heads] (kv_layout 0) or [K0 V0 | K1 V1 | ...] (kv_layout 1:
 * with head_dim 128 each K/V pair is one 256-output scale block, so a shard
 * holding whole pairs quantises exactly as the unsharded matrix does).  Q and
 * K rotate on adjacent pairs by pos*theta[p], V does not; all rows are
 * written to y (fp32) and K/V rows also, as fp16, at token `pos` into kcache
 * K[t][h][d] and vcache V[h][d/8][t][d%8] (the Att-full-FP16 layouts) of
 * ctx_cap tokens. */
int vkc_rmsnorm_gemv_rope_kv(int bits, const void* w, const float* scale, const float* zero,
                             const float* x, const float* gamma, const float* theta, float* y,
                             int N, int K, float eps, int rms_dim, int pos, int head_dim,
                             int q_rows, int kv_rows, int kv_layout, void* kcache, void* vcache,
                             int ctx_cap, void* stream);

/* RmsNorm-GEMV followed by a rotary epilogue at position `pos`.
 * rope_mode 0: the epilogue of shader/RmsNorm-GEMV-Rope-FP16.comp:76-89 as
 *   written (first 64 outputs of every 256, partner term taken from theta;
 *   theta holds >= 64 floats).
 * rope_mode 1: rotation of adjacent pairs (2p, 2p+1) of each head_dim-wide
 *   head among the first rot_rows outputs by angle pos*theta[p]
 *   (theta holds >= head_dim/2 floats); rows from rot_rows on (V) unrotated.
 * Replaces shader/RmsNorm-GEMV-Rope-FP16.comp, -INT8.comp, -INT4.comp. */
int vkc_rmsnorm_gemv_rope(int bits, const void* w, const float* scale, const float* zero,
                          const float* x, const float* gamma, const float* theta, float* y,
                          int N, int K, float eps, int rms_dim, int pos, int rope_mode,
                          int head_dim, int rot_rows, void* stream);

/* h = SiLU(Wg^T n) * (Wu^T n), n = x * gamma * inv_rms, SiLU(g) =
 * g / (1 + 2^(-g log2 e)).  Replaces shader/RmsNorm-swiglu-ffn-FP16.comp,
 * -INT8.comp, -INT4.comp and RmsNorm-swiglu-ffn.comp. */
int vkc_rmsnorm_swiglu(int bits, const void* wg, const float* sg, const float* zg, const void* wu,
                       const float* su, const float* zu, const float* x, const float* gamma,
                       float* h, int N, int K, float eps, int rms_dim, void* stream);

/* ---- Fused NVLink exchange for the sharded decoder (no counterpart in the
 * reference, which runs on one GPU).  A K-split projection (O, down) stores
 * its partial output straight into every rank's slot buffer; the next
 * operator sums the slots while loading its input.  Slot buffers hold 8-byte
 * words (flag << 32 | fp32 bits), written and read whole, so no fence or
 * counter orders data and arrival: a reader waits until a peer's word carries
 * the flag that its own rank's word for the same element carries.  Buffers
 * are peer-mapped memory (vkc_ipc_*), zeroed before the first exchange; every
 * rank makes the same sequence of launches on buffers of the same shapes.  A
 * buffer is written again only after an exchange on another buffer that
 * every rank's consumer of this one precedes (the decoder alternates two
 * buffers), so no rank overwrites slots a slower rank is still reading. */

/* Input of a fused consumer: x = base + the `world` partial vectors of
 * `slots` ([world][K] words in this rank's memory, 8-byte aligned) summed in
 * rank order; the previous launch on the stream must be this rank's
 * vkc_gemv_peer into the same buffer.  x is also stored to `save` (K floats)
 * unless NULL.  A thread whose waits reach 100 ms in total sets flag 0x8 of
 * the device status word (vkc_device_status) and stops waiting. */
typedef struct vkc_peer_input {
    const void* slots;
    float* save;
    int rank;
    int world;
} vkc_peer_input;

/* y_partial = W^T x (this rank's K slice of the projection), stored at
 * elements [rank*N, (rank+1)*N) of every rank's [world][N] word buffer
 * (slots: device array of `world` pointers), each word carrying the flag of
 * this rank's own copy of the element plus one. */
int vkc_gemv_peer(int bits, const void* w, const float* scale, const float* zero, const float* x,
                  void* const* slots, int rank, int world, int N, int K, void* stream);

/* vkc_rmsnorm_gemv_rope_kv and vkc_rmsnorm_swiglu with their input taken
 * from a peer exchange (`x_base` + the slots of `in`; host pointer, read at
 * the call). */
int vkc_rmsnorm_gemv_rope_kv_peer(int bits, const void* w, const float* scale, const float* zero,
                                  const float* x_base, const vkc_peer_input* in, const float* gamma,
                                  const float* theta, float* y, int N, int K, float eps, int rms_dim,
                                  int pos, int head_dim, int q_rows, int kv_rows, int kv_layout,
                                  void* kcache, void* vcache, int ctx_cap, void* stream);
int vkc_rmsnorm_swiglu_peer(int bits, const void* wg, const float* sg, const float* zg, const void* wu,
                            const float* su, const float* zu, const float* x_base,
                            const vkc_peer_input* in, const float* gamma, float* h, int N, int K,
                            float eps, int rms_dim, void* stream);

/* Batched decode (no counterpart in the reference: its shaders take an M push
 * constant but compute one vector).  y[m] = W^T x[m] for M in 1..8 vectors
 * (x: [M][K], y: [M][N], fp32, row-major) with the weights streamed once for
 * all of them; the RmsNorm variant normalises each vector by its own RMS.
 * M == 1 runs vkc_gemv / vkc_rmsnorm_gemv.  K must be a multiple of 4. */
int vkc_gemv_batched(int bits, const void* w, const float* scale, const float* zero, const float* x,
                     float* y, int M, int N, int K, void* stream);
int vkc_rmsnorm_gemv_batched(int bits, const void* w, const float* scale, const float* zero,
                             const float* x, const float* gamma, float* y, int M, int N, int K,
                             float eps, int rms_dim, void* stream);

/* Decode attention for one token.  Replaces shader/Att-full-FP16.comp.
 * q: [n_q][head_dim], fp16 (q_bits 16) or fp32 (q_bits 32);
 * kcache: fp16 K[t][kv][d] at (t*n_kv + kv)*head_dim + d;
 * vcache: fp16 V[kv][d/8][t][d%8] (16-byte chunks of 8 dims per token);
 * out: fp32 [n_q][head_dim]; query head h reads KV head h/(n_q/n_kv);
 * scores are scale * q.k; n_q/n_kv in {1, 2, 4}; head_dim a multiple of 8
 * up to 256.  workspace: NULL to use a library-owned per-device workspace
 * (calls on different streams must then not overlap), or caller memory of
 * vkc_attention_workspace_bytes() bytes, zero-filled before its first use. */
size_t vkc_attention_workspace_bytes(int n_q, int n_kv, int head_dim, int ctx);
/* How decode attention splits the cache (head_dim 64 or 128), for the calling
 * host thread: 0 (default) chooses per shape; 1 clusters of 8 CTAs per KV
 * head merging in distributed shared memory, two CTAs per SM; 2 at most one
 * CTA per SM, each streaming a long token range through a deep ring, the
 * splits of a head merged by the last to finish; 3 the same with a 3-stage
 * ring in at most half an SM's shared memory (so the next kernel in the
 * stream can be resident beside it under programmatic dependent launch);
 * 4 two such CTAs per SM over twice the splits; 5 the per-SM shape with
 * two warp groups per CTA working on alternate sub-tiles (what 0 uses
 * wherever the per-SM shape applies).  The workspace size
 * (vkc_attention_workspace_bytes) depends on the plan in force.  No
 * counterpart in the reference. */
int vkc_set_attention_plan(int plan);
int vkc_get_attention_plan(void);
/* The split decode attention would use for a shape under the calling
 * thread's plan: info[0] kernel (1 token-slice clustered, 2 token-slice
 * per-SM, 3 head_dim-256 tensor-core, 4 SIMT), [1] CTAs per KV head, [2]
 * tokens per CTA, [3] ring stages, [4] warp groups per CTA, [5] CTAs per
 * cluster, [6] partial records per query head.  No counterpart in the
 * reference. */
int vkc_attention_plan_info(int n_q, int n_kv, int head_dim, int ctx, int* info);

/* The decoder step as one persistent kernel (one GPU, 4-bit weights, four
 * query heads per KV head, head_dim 64 or 128).  Per layer it runs, separated
 * by grid-wide barriers instead of kernel boundaries: RMSNorm-QKV-RoPE with
 * the KV append (rows [Q | K0 V0 | K1 V1 | ...], theta per rotary pair),
 * attention over tokens [0, pos], x' = x + O attn, h = RMSNorm-SwiGLU(x'),
 * x = x' + down h -- the arithmetic of vkc_rmsnorm_gemv_rope_kv,
 * vkc_attention_decode, vkc_gemv_residual and vkc_rmsnorm_swiglu.  Each phase
 * requests its weights before it waits at the barrier.  A barrier wait that
 * runs out (kGridWaitNs, the peer-exchange limit) sets status flag 0x20 and
 * the launch gives up waiting.  The launch is cooperative (all CTAs resident;
 * it fails with an error where the device cannot hold them).
 * `program` (vkc_decode_program_bytes, 256-byte aligned device memory) holds
 * the per-layer parameters, the barrier counter and the attention workspace;
 * build it once per set of weights and buffers, then run it per token (runs
 * on one stream do not overlap).  No counterpart in the reference. */
typedef struct vkc_decode_dims {
    int layers, hidden, inter, n_q, n_kv, head_dim, ctx_cap, bits;
    float eps;
} vkc_decode_dims;
typedef struct vkc_decode_layer {
    const void* qkv; const float* qkv_scale; const float* qkv_zero;
    const void* o; const float* o_scale; const float* o_zero;
    const void* gate; const float* gate_scale; const float* gate_zero;
    const void* up; const float* up_scale; const float* up_zero;
    const void* down; const float* down_scale; const float* down_zero;
    const float* gamma_attn; const float* gamma_ffn;
    void* kcache; void* vcache;  /* fp16, the layouts of vkc_attention_decode */
} vkc_decode_layer;
typedef struct vkc_decode_buffers {
    float* x;      /* hidden state in and out [hidden] */
    float* x_mid;  /* x' [hidden] */
    float* qkv;    /* [n_q*hd + 2*n_kv*hd] */
    float* attn;   /* [n_q*hd] */
    float* h;      /* [inter] */
} vkc_decode_buffers;
size_t vkc_decode_program_bytes(const vkc_decode_dims* dims);
int vkc_decode_program_build(const vkc_decode_dims* dims, const vkc_decode_layer* layers,
                             const vkc_decode_buffers* bufs, const float* theta, void* program,
                             size_t program_bytes, void* stream);
int vkc_decode_program_run(const vkc_decode_dims* dims, void* program, int pos, void* stream);
int vkc_attention_decode(const void* q, int q_bits, const void* kcache, const void* vcache,
                         float* out, int n_q, int n_kv, int head_dim, int ctx, float scale,
                         void* workspace, size_t workspace_bytes, void* stream);

/* vkc_attention_decode over a cache allocated for ctx_cap >= ctx tokens (the
 * V layout's per-(head, chunk) token run is ctx_cap long); tokens [0, ctx)
 * are attended.  The decoder chain uses it while its cache fills. */
int vkc_attention_decode_cache(const void* q, int q_bits, const void* kcache, const void* vcache,
                               float* out, int n_q, int n_kv, int head_dim, int ctx, int ctx_cap,
                               float scale, void* workspace, size_t workspace_bytes, void* stream);

/* vkc_attention_decode_cache for a decode step right after the KV append
 * (vkc_rmsnorm_gemv_rope_kv at pos = ctx - 1): with programmatic dependent
 * launch on, cache tokens [0, ctx - 1) are requested before the wait on the
 * previous kernel, so the contract is that no kernel still running writes
 * them (the previous kernel wrote only token ctx - 1).  A workspace is
 * required. */
int vkc_attention_decode_append(const void* q, int q_bits, const void* kcache, const void* vcache,
                                float* out, int n_q, int n_kv, int head_dim, int ctx, int ctx_cap,
                                float scale, void* workspace, size_t workspace_bytes, void* stream);

/* Decode attention that allocates nothing.  No counterpart in the reference.
 * For callers that cannot allocate device memory when attention runs (an
 * engine whose memory pool already owns all of HBM, a decode loop that must not
 * take the synchronisation cudaMalloc/cudaFree can imply, a plugin whose host
 * forbids allocation in its callbacks).  Same arguments and results as
 * vkc_attention_decode, but its scratch is a fixed 2 MiB array inside the
 * library (held by every GPU that loads the library until it is unloaded);
 * shapes needing more (vkc_attention_workspace_bytes) are rejected with
 * VKC_ERR_ARG.  Every call looks up the array's address in the current
 * context; the first call on a device (and the first in a new context) also
 * clears its tickets with a memset on `stream`, so make that first call before
 * any stream capture.  All
 * calls share the array: calls that overlap on the GPU (different streams)
 * race; calls ordered on one stream do not. */
size_t vkc_attention_noalloc_max_scratch(void);
int vkc_attention_decode_noalloc(const void* q, int q_bits, const void* kcache, const void* vcache,
                                 float* out, int n_q, int n_kv, int head_dim, int ctx, float scale,
                                 void* stream);

/* In-place RMSNorm of `rows` rows of `width` fp32 values each:
 * x = x * inv_rms * gamma, inv_rms = 1/sqrt(sum(x^2)/width + eps), gamma has
 * `width` values.  Replaces shader/RmsNorm.comp (width 256, eps 1e-5, one
 * workgroup per row). */
int vkc_rmsnorm_rows(float* x, const float* gamma, int rows, int width, float eps, void* stream);

/* y[j] = sum_k x[k] W[k*N + j] for a plain row-major K x N fp32 matrix.
 * Replaces shader/gemv2.comp and gemv3.comp, and gemv1.comp with N = K (the
 * fp32 experiments that read W row-major rather than in 16-byte chunks;
 * gemv4-gemv7 read the chunk layout and are served by vkc_gemv with bits 32).
 * May use the library's per-device workspace (calls on different streams
 * must then not overlap). */
int vkc_gemv_rowmajor(const float* w, const float* x, float* y, int N, int K, void* stream);

/* C = A B, row-major fp32 (A M x K, B K x N).  Replaces shader/gemm.comp. */
int vkc_gemm_f32(const float* a, const float* b, float* c, int M, int N, int K, void* stream);

/* ---- exchange between the GPUs of one node (row-sharded decoder chain) ----
 * No counterpart in the reference (which runs on one GPU).  All-gather of an
 * fp32 vector whose rank-r slice (slice_floats values) is `src`: the slice is
 * stored over NVLink into every rank's full buffer at offset r*slice_floats.
 * dsts (device array of `world` pointers) are the ranks' full buffers and
 * counters (device array of `world` pointers) the ranks' arrival counters
 * (world unsigned each, zero before the first launch), all mapped into this
 * process (CUDA IPC).  Every rank makes the same sequence of launches; a launch
 * returns on the GPU once every rank's slice has arrived here.  A wait that
 * exceeds its bound sets flag 0x8 in *status (device memory) instead of hanging. */
int vkc_allgather_p2p(const float* src, void* const* dsts, unsigned* const* counters, int slice_floats,
                      int rank, int world, unsigned* status, void* stream);
/* Row-sharded RmsNorm-GEMV whose epilogue stores the outputs straight into
 * every rank's full vector (no counterpart in the reference): this rank's N
 * outputs (its rows of the matrix) go to `offset` of each rank's vector (dsts:
 * device array of `world` pointers, as for vkc_allgather_p2p; one-CTA-per-SM
 * kernel).  vkc_gather_wait, launched next on the same stream, signals this
 * rank's arrival on counter `rank` of every rank (counters: as for
 * vkc_allgather_p2p; do not mix the two on one set of counters) and returns on
 * the GPU once every rank's step-th launch has arrived here; step_word is a
 * device word (zero at first) counting this rank's waits; a wait beyond its
 * bound sets flag 0x8 in *status. */
int vkc_rmsnorm_gemv_gather(int bits, const void* w, const float* scale, const float* zero, const float* x,
                            const float* gamma, void* const* dsts, int rank, int world, int offset, int N, int K,
                            float eps, int rms_dim, void* stream);
int vkc_gather_wait(unsigned* const* counters, int rank, int world, unsigned* step_word, unsigned* status,
                    void* stream);
/* All-reduce with residual for K-split projections (no counterpart in the
 * reference): `part` is this rank's partial output (n floats); it is stored
 * into slot `rank` of every rank's partial buffer (slots: device array of
 * `world` pointers to [world][n] floats), and once every rank's slot has
 * arrived (same counters and protocol as vkc_allgather_p2p) each rank writes
 * out = residual + sum of the slots in rank order (out must not alias part). */
int vkc_allreduce_residual_p2p(const float* part, void* const* slots, unsigned* const* counters, int n, int rank,
                               int world, const float* residual, float* out, unsigned* status, void* stream);
/* Peer memory for the above: a zeroed device allocation of `bytes` and its
 * 64-byte CUDA IPC handle; open maps a peer's handle into the current device
 * (peer access enabled on first use); close unmaps; free releases. */
int vkc_ipc_alloc(size_t bytes, void** ptr, void* handle);
int vkc_ipc_open(const void* handle, void** ptr);
int vkc_ipc_close(void* ptr);
int vkc_ipc_free(void* ptr);

/* Prefill GEMM on the tcgen05 tensor cores: C[M][N] (fp32) = A[M][K] (bf16)
 * . W[N][K]^T (bf16); A and W row-major, so W is the K-major (N rows of K)
 * layout of a linear layer's weight.  The batched form of gemm.comp's
 * contraction (shader/gemm.comp:19-59) for prefill.  K a multiple of 64, N a
 * multiple of 16, any M (tiles of 128 rows).  Pointers 16-byte aligned. */
int vkc_gemm_bf16(const void* a, const void* w, float* c, int M, int N, int K, void* stream);
/* Status flags of vkc_gemm_bf16 on the current device (0x10: a bounded wait
 * ran out); waits for the device; `clear` resets them. */
int vkc_gemm_bf16_status(unsigned* status, int clear);

/* ---- weight preparation on the GPU (bit-identical to src/data.c) ---- */

/* dst[r*N + c] = get_pseudo_random(r, c, seed) (src/data.c:8-28); fp32 when
 * out_bits = 32, the reference's truncating fp16 (src/data.c:30-51) when 16. */
int vkc_generate(int seed, int M, int N, int out_bits, void* dst, void* stream);
/* Quantise a K x N fp32 matrix into the reference's storage: codes (u8 K x N,
 * or u4 two per byte with the even output in the high nibble) plus block-major
 * fp32 scale/zero.  symmetric 0: min/max asymmetric (src/data.c:95-185);
 * symmetric 1: s = max|w|/qmax (fp16-rounded if fp16_scale), u = q + 2^(bits-1),
 * z = 2^(bits-1) s. */
int vkc_quantize(const float* w, int K, int N, int bits, int symmetric, int fp16_scale,
                 uint8_t* codes, float* scale, float* zero, void* stream);
/* transpose_block16 (src/data.c:198-222) on the device: `in` is K x N
 * row-major (fp32, fp16, u8, or u4 two per byte). */
int vkc_pack_block16(const void* in, void* out, int K, int N, int bits, void* stream);

/* ---- weights on disk (no counterpart in the reference, which builds its
 * matrices in memory with src/data.c and keeps no model files) ----
 * A file holds named matrices in exactly the device layout above: the
 * transpose_block16 chunks and, for 8/4-bit weights, block-major fp32 scale
 * and zero, each section 256-byte aligned (format: csrc/weights_file.cu).
 * Loading copies each section from disk through pinned memory to the device
 * with no repacking.  Errors (unreadable, truncated or inconsistent files,
 * unknown shapes) return VKC_ERR_ARG with a message. */
typedef struct vkc_weight_entry {
    char name[64];       /* NUL-terminated */
    int bits, K, N;      /* 32, 16, 8 or 4; y = W^T x with W K x N */
    const void* data;    /* write: host packed chunks, K*N*bits/8 bytes */
    const float* scale;  /* write: host [N/256][K] (8/4-bit only) */
    const float* zero;
} vkc_weight_entry;
typedef struct vkc_weight_file vkc_weight_file;

/* Writes `count` matrices (host memory) to `path`. */
int vkc_weights_write(const char* path, const vkc_weight_entry* entries, int count);
/* Opens and validates a file; vkc_weights_close releases it. */
int vkc_weights_open(const char* path, vkc_weight_file** file);
int vkc_weights_count(const vkc_weight_file* file);
/* Index of the matrix called `name`, or -1. */
int vkc_weights_find(const vkc_weight_file* file, const char* name);
/* Name and shape of matrix `index` (the pointers of *info are set to NULL). */
int vkc_weights_info(const vkc_weight_file* file, int index, vkc_weight_entry* info);
/* Matrix `index` into device memory (data: K*N*bits/8 bytes; scale, zero:
 * K*N/256 floats each, ignored for 16/32-bit) through pinned host memory;
 * returns once the copies on `stream` are done. */
int vkc_weights_read(vkc_weight_file* file, int index, void* data, float* scale, float* zero, void* stream);
/* The same into host memory. */
int vkc_weights_read_host(vkc_weight_file* file, int index, void* data, float* scale, float* zero);
void vkc_weights_close(vkc_weight_file* file);

#ifdef __cplusplus
}
#endif
#endif
