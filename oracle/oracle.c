/*
 * oracle.c -- CPU restatement of vk-compute's matrix-vector decode path.
 *
 * TEST INFRASTRUCTURE ONLY (see oracle.h): used by tests/, the smoke check
 * and the benchmark's CPU-baseline leg as the checker; never by the product.
 *
 * Reference paths are relative to the vk-compute project root.
 */
#include "oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

#define GROUP 256 /* outputs per scale/zero group, src/data.c:99,143 */

/* ------------------------------------------------------------------------ */
/* Data generation: src/data.c                                              */
/* ------------------------------------------------------------------------ */

/* src/data.c:8-16.  The reference forms the seed hash with signed int
 * arithmetic and casts to unsigned; unsigned arithmetic here gives the same
 * two's-complement wrap without relying on signed overflow. */
float vko_pseudo_random(int i, int j, int seed) {
    uint32_t h = (uint32_t)i * 73129u + (uint32_t)j * 95121u + (uint32_t)seed * 15473u;
    h = (h ^ 61u) ^ (h >> 16);
    h += h << 3;
    h ^= h >> 4;
    h *= 0x27d4eb2du;
    h ^= h >> 15;
    return ((float)(h % 2000001u) / 1000000.0f) - 1.0f;
}

/* src/data.c:18-28: row-major M x N. */
void vko_get_data(int seed, int M, int N, float* out) {
    for (int r = 0; r < M; ++r)
        for (int c = 0; c < N; ++c) out[(int64_t)r * N + c] = vko_pseudo_random(r, c, seed);
}

/* src/data.c:30-51: fp32 -> fp16 by truncation of the mantissa (round toward
 * zero).  Inputs below 2^-14 take the reference's subnormal branch, whose shift
 * (1 - exp) leaves the result a factor 4 smaller than an IEEE subnormal; values
 * below 2^-24 flush to signed zero; |f| >= 2^16 saturates to infinity. */
uint16_t vko_float_to_fp16(float f) {
    uint32_t bits;
    memcpy(&bits, &f, sizeof bits);
    uint32_t sign = (bits >> 16) & 0x8000u;
    int32_t e = (int32_t)((bits >> 23) & 0xffu) - 127;
    uint32_t m = bits & 0x7fffffu;
    if (e <= -15) {
        if (e < -24) return (uint16_t)sign;
        return (uint16_t)(sign | ((m | 0x800000u) >> (1 - e)));
    }
    if (e >= 16) return (uint16_t)(sign | 0x7c00u);
    return (uint16_t)(sign | ((uint32_t)(e + 15) << 10) | (m >> 13));
}

/* src/data.c:53-81: exact fp16 -> fp32 (subnormals normalised). */
float vko_fp16_to_float(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    int32_t e = (h >> 10) & 0x1f;
    uint32_t m = h & 0x3ffu;
    uint32_t out;
    if (e == 0) {
        if (m == 0) {
            out = sign;
        } else {
            int32_t ee = -14;
            while (!(m & 0x400u)) {
                m <<= 1;
                --ee;
            }
            m &= 0x3ffu;
            out = sign | ((uint32_t)(ee + 127) << 23) | (m << 13);
        }
    } else if (e == 31) {
        out = sign | 0x7f800000u | (m << 13);
    } else {
        out = sign | ((uint32_t)(e - 15 + 127) << 23) | (m << 13);
    }
    float f;
    memcpy(&f, &out, sizeof f);
    return f;
}

/* src/data.c:83-93 */
void vko_get_data_fp16(int seed, int M, int N, uint16_t* out) {
    for (int r = 0; r < M; ++r)
        for (int c = 0; c < N; ++c)
            out[(int64_t)r * N + c] = vko_float_to_fp16(vko_pseudo_random(r, c, seed));
}

/* Shared body of the asymmetric min/max quantiser, src/data.c:95-185.
 * For row k and 256-wide block b: s = (max-min)/levels, z = -min,
 * q = (u8)roundf((v + z) / s).  Scales and zeros are block-major,
 * index b*K + k (src/data.c:122,167).  INT4 packs two outputs per byte with
 * the even output in the high nibble (src/data.c:178-179).  Only whole blocks
 * are quantised, as in the reference (blocks_per_row = N / 256). */
static void quant_asym_rows(int K, int N, int bits, uint8_t* data, float* scale, float* zero,
                            float (*value)(const void*, int, int), const void* ctx) {
    const float levels = bits == 8 ? 255.0f : 15.0f;
    const int nblocks = N / GROUP;
    for (int k = 0; k < K; ++k) {
        for (int b = 0; b < nblocks; ++b) {
            float lo = 1e9f, hi = -1e9f;
            for (int t = 0; t < GROUP; ++t) {
                float v = value(ctx, k, b * GROUP + t);
                if (v < lo) lo = v;
                if (v > hi) hi = v;
            }
            const int64_t si = (int64_t)b * K + k;
            scale[si] = (hi - lo) / levels;
            zero[si] = -lo;
            for (int t = 0; t < GROUP; ++t) {
                const int c = b * GROUP + t;
                uint8_t q = (uint8_t)roundf((value(ctx, k, c) + zero[si]) / scale[si]);
                if (bits == 8) {
                    data[(int64_t)k * N + c] = q;
                } else {
                    uint8_t* p = &data[(int64_t)k * (N / 2) + c / 2];
                    if ((c & 1) == 0)
                        *p = (uint8_t)((q & 0x0f) << 4);
                    else
                        *p = (uint8_t)(*p | (q & 0x0f));
                }
            }
        }
    }
}

typedef struct {
    int seed;
} seed_ctx;
static float seeded_value(const void* ctx, int k, int c) {
    return vko_pseudo_random(k, c, ((const seed_ctx*)ctx)->seed);
}
typedef struct {
    const float* w;
    int N;
} mat_ctx;
static float matrix_value(const void* ctx, int k, int c) {
    const mat_ctx* m = (const mat_ctx*)ctx;
    return m->w[(int64_t)k * m->N + c];
}

/* src/data.c:95-137 */
void vko_get_data_int8(int seed, int M, int N, uint8_t* data, float* scale, float* zero) {
    seed_ctx s = {seed};
    quant_asym_rows(M, N, 8, data, scale, zero, seeded_value, &s);
}

/* src/data.c:139-185 */
void vko_get_data_int4(int seed, int M, int N, uint8_t* data, float* scale, float* zero) {
    seed_ctx s = {seed};
    quant_asym_rows(M, N, 4, data, scale, zero, seeded_value, &s);
}

/* src/data.c:198-222.  Re-tiles a K x N row-major matrix of `bits`-wide
 * elements into 16-byte chunks: chunk (r, j) holds 128/bits consecutive k
 * (k = r*128/bits + t) of column j and sits at byte (r*N + j)*16.  fp16/fp32/
 * int8 elements keep their bytes in k order; int4 chunk byte t/2 holds k even in
 * its low nibble and k odd in its high nibble. */
void vko_transpose_block16(const uint8_t* in, uint8_t* out, int M, int N, int bits) {
    const int per = 128 / bits;
    for (int r = 0; r < M / per; ++r) {
        uint8_t* row = out + (int64_t)r * N * 16;
        for (int c = 0; c < N; ++c) {
            uint8_t* chunk = row + (int64_t)c * 16;
            if (bits == 4) {
                memset(chunk, 0, 16);
                for (int t = 0; t < per; ++t) {
                    uint8_t byte = in[(int64_t)(r * per + t) * (N / 2) + c / 2];
                    uint8_t q = (c & 1) ? (byte & 0x0f) : (byte >> 4);
                    chunk[t / 2] |= (uint8_t)((t & 1) ? (q << 4) : q);
                }
            } else {
                const int eb = bits / 8;
                for (int t = 0; t < per; ++t)
                    memcpy(chunk + t * eb, in + ((int64_t)(r * per + t) * N + c) * eb, eb);
            }
        }
    }
}

/* ------------------------------------------------------------------------ */
/* Quantisers for given matrices                                            */
/* ------------------------------------------------------------------------ */

/* The data.c min/max quantiser (src/data.c:95-185) applied to a given K x N
 * matrix instead of the seeded generator. */
void vko_quantize_asym(const float* w, int K, int N, int bits, uint8_t* data, float* scale,
                       float* zero) {
    mat_ctx m = {w, N};
    quant_asym_rows(K, N, bits, data, scale, zero, matrix_value, &m);
}

/* Symmetric quantiser in the reference's storage layout.  Per (k, block):
 * s = max|w| / qmax (qmax 127 or 7), optionally rounded to the nearest fp16;
 * q = clamp(roundf(w / s), -qmax, qmax); stored code u = q + 2^(bits-1) and
 * zero z = 2^(bits-1) * s, so the reference dequantisation u*s - z gives q*s.
 * A block of zeros gets s = z = 0 and code 2^(bits-1). */
void vko_quantize_sym(const float* w, int K, int N, int bits, int fp16_scale, uint8_t* data,
                      float* scale, float* zero) {
    const float qmax = bits == 8 ? 127.0f : 7.0f;
    const int off = bits == 8 ? 128 : 8;
    const int nblocks = N / GROUP;
    for (int k = 0; k < K; ++k) {
        for (int b = 0; b < nblocks; ++b) {
            float amax = 0.0f;
            for (int t = 0; t < GROUP; ++t) {
                float a = fabsf(w[(int64_t)k * N + b * GROUP + t]);
                if (a > amax) amax = a;
            }
            float s = amax / qmax;
            if (fp16_scale) s = (float)(_Float16)s;
            const int64_t si = (int64_t)b * K + k;
            scale[si] = s;
            zero[si] = (float)off * s;
            for (int t = 0; t < GROUP; ++t) {
                const int c = b * GROUP + t;
                float q = 0.0f;
                if (s > 0.0f) {
                    q = roundf(w[(int64_t)k * N + c] / s);
                    if (q > qmax) q = qmax;
                    if (q < -qmax) q = -qmax;
                }
                uint8_t u = (uint8_t)((int)q + off);
                if (bits == 8) {
                    data[(int64_t)k * N + c] = u;
                } else {
                    uint8_t* p = &data[(int64_t)k * (N / 2) + c / 2];
                    if ((c & 1) == 0)
                        *p = (uint8_t)((u & 0x0f) << 4);
                    else
                        *p = (uint8_t)(*p | (u & 0x0f));
                }
            }
        }
    }
}

/* ------------------------------------------------------------------------ */
/* Dequantisation                                                           */
/* ------------------------------------------------------------------------ */

static inline uint32_t code_at(const uint8_t* data, int bits, int K, int N, int k, int c) {
    (void)K;
    if (bits == 8) return data[(int64_t)k * N + c];
    uint8_t byte = data[(int64_t)k * (N / 2) + c / 2];
    return (c & 1) ? (byte & 0x0fu) : (uint32_t)(byte >> 4); /* src/compute.c:262 */
}

/* Dense weight: w = q * s - z with s, z of block c/256, as the shaders do it
 * (shader/GEMV-INT8.comp:56-59, GEMV-INT4.comp:57-64) and as the reference CPU
 * check writes it (src/compute.c:248,263). */
void vko_dequant(const uint8_t* data, const float* scale, const float* zero, int K, int N,
                 int bits, float* w) {
    for (int k = 0; k < K; ++k)
        for (int c = 0; c < N; ++c) {
            const int64_t si = (int64_t)(c / GROUP) * K + k;
            w[(int64_t)k * N + c] = (float)code_at(data, bits, K, N, k, c) * scale[si] - zero[si];
        }
}

void vko_fp16_matrix_to_float(const uint16_t* h, int64_t count, float* out) {
    for (int64_t i = 0; i < count; ++i) out[i] = vko_fp16_to_float(h[i]);
}

/* ------------------------------------------------------------------------ */
/* Operators on dense fp32 weights                                          */
/* ------------------------------------------------------------------------ */

/* src/compute.c:216-218 extended to every output: y[j] = sum_k x[k] W[k][j].
 * Accumulates in double (the reference accumulates in float). */
void vko_gemv(const float* x, const float* w, int K, int N, float* y) {
    double* acc = (double*)calloc((size_t)N, sizeof(double));
    for (int k = 0; k < K; ++k) {
        const double xk = x[k];
        const float* row = w + (int64_t)k * N;
        for (int c = 0; c < N; ++c) acc[c] += xk * row[c];
    }
    for (int c = 0; c < N; ++c) y[c] = (float)acc[c];
    free(acc);
}

/* The RMS factor of shader/RmsNorm-GEMV-FP16.comp:58-59:
 * 1 / sqrt(sum(x^2) / d_model + eps), where the reference divides by the
 * compile-time d_model (4096) rather than by K.  (src/compute.c:223 puts eps
 * outside the square root; the shaders put it inside, which is followed here.) */
float vko_inv_rms(const float* x, int K, int rms_dim, float eps) {
    double ss = 0.0;
    for (int k = 0; k < K; ++k) ss += (double)x[k] * x[k];
    return (float)(1.0 / sqrt(ss / (double)rms_dim + (double)eps));
}

/* shader/RmsNorm.comp:22-52: in place, each row of `width` values (the
 * shader's TS = 256, one workgroup per row) becomes (x * inv_rms) * gamma with
 * inv_rms = 1/sqrt(sum(x^2)/width + eps) (EPSILON 1e-5, comp:9).  No CPU check
 * exists in the reference; the formula is the shader's. */
void vko_rmsnorm_rows(float* x, const float* gamma, int rows, int width, float eps) {
    for (int r = 0; r < rows; ++r) {
        float* xr = x + (int64_t)r * width;
        double ss = 0.0;
        for (int i = 0; i < width; ++i) ss += (double)xr[i] * xr[i];
        const double inv = 1.0 / sqrt(ss / (double)width + (double)eps);
        for (int i = 0; i < width; ++i) xr[i] = (float)((double)xr[i] * inv * gamma[i]);
    }
}

/* shader/RmsNorm-GEMV-FP16.comp:36-73; CPU form src/compute.c:221-226. */
void vko_rmsnorm_gemv(const float* x, const float* gamma, const float* w, int K, int N,
                      int rms_dim, float eps, float* y) {
    const float inv = vko_inv_rms(x, K, rms_dim, eps);
    float* n = (float*)malloc(sizeof(float) * (size_t)K);
    for (int k = 0; k < K; ++k) n[k] = x[k] * gamma[k] * inv;
    vko_gemv(n, w, K, N, y);
    free(n);
}

/* The RoPE epilogue exactly as shader/RmsNorm-GEMV-Rope-FP16.comp:76-89 writes
 * it: in every 256-output workgroup, local output c < 64 is rotated by
 * angle = pos * theta[c/2] against theta[c+1] (even c) or theta[c-1] (odd c),
 * i.e. the partner term is a theta value, not the partner output.  No CPU
 * check exists in the reference: parity unpinned. */
void vko_rope_reference(float* y, int N, int pos, const float* theta) {
    for (int j = 0; j < N; ++j) {
        const int c = j % 256;
        if (c >= 64) continue;
        const float angle = (float)pos * theta[c / 2];
        const float ca = cosf(angle), sa = sinf(angle);
        if ((c & 1) == 0)
            y[j] = y[j] * ca - theta[c + 1] * sa;
        else
            y[j] = theta[c - 1] * sa + y[j] * ca;
    }
}

/* Rotary embedding on adjacent pairs (2p, 2p+1) of every head_dim-wide head
 * among the first rot_rows outputs (Q and K heads; V rows follow and are left
 * alone), angle = pos * theta[p].  This is the rotation the reference's
 * epilogue (shader/RmsNorm-GEMV-Rope-FP16.comp:76-89) sets out to compute;
 * parity unpinned. */
void vko_rope_pairs(float* y, int N, int head_dim, int rot_rows, int pos, const float* theta) {
    if (rot_rows > N) rot_rows = N;
    for (int j = 0; j + 1 < rot_rows; j += 2) {
        const int p = (j % head_dim) / 2;
        const double angle = (double)(float)((float)pos * theta[p]);
        const double ca = cos(angle), sa = sin(angle);
        const double a = y[j], b = y[j + 1];
        y[j] = (float)(a * ca - b * sa);
        y[j + 1] = (float)(a * sa + b * ca);
    }
}

/* shader/RmsNorm-swiglu-ffn-FP16.comp:59-87; CPU form src/compute.c:229-241:
 * h = g / (1 + 2^(-g * log2 e)) * u, g and u the gate and up projections of
 * the RMS-normalised input. */
void vko_swiglu(const float* x, const float* gamma, const float* wg, const float* wu, int K,
                int N, int rms_dim, float eps, float* h) {
    float* g = (float*)malloc(sizeof(float) * (size_t)N);
    float* u = (float*)malloc(sizeof(float) * (size_t)N);
    vko_rmsnorm_gemv(x, gamma, wg, K, N, rms_dim, eps, g);
    vko_rmsnorm_gemv(x, gamma, wu, K, N, rms_dim, eps, u);
    for (int j = 0; j < N; ++j) {
        const double gd = g[j];
        h[j] = (float)(gd / (1.0 + exp2(-gd * 1.44269504)) * (double)u[j]);
    }
    free(g);
    free(u);
}

/* Decode attention after shader/Att-full-FP16.comp:33-83: for query head h the
 * key/value head is h / (n_q / n_kv); scores s_t = scale * q . K[t];
 * out = sum_t e^{s_t} V[t] / sum_t e^{s_t}.  The maximum score is subtracted
 * before exponentiation (an identity of the softmax).  Layouts follow the
 * shader: K token-major, K[t][kv][d] at (t*n_kv + kv)*hd + d (comp:55-59);
 * V in 8-dimension chunks per token, V[kv][d/8][t][d%8] (comp:69-73).  q is
 * fp16 [n_q][hd]; out is fp32 [n_q][hd].  Parity unpinned (no CPU check). */
static void attention_impl(const uint16_t* q16, const float* q32, const uint16_t* kcache,
                           const uint16_t* vcache, int n_q, int n_kv, int head_dim, int ctx, float scale,
                           float* out) {
    const int group = n_q / n_kv;
    double* sc = (double*)malloc(sizeof(double) * (size_t)ctx);
    for (int h = 0; h < n_q; ++h) {
        const int kv = h / group;
        double mx = -INFINITY;
        for (int t = 0; t < ctx; ++t) {
            double s = 0.0;
            const uint16_t* kr = kcache + ((int64_t)t * n_kv + kv) * head_dim;
            for (int d = 0; d < head_dim; ++d) {
                const int64_t qi = (int64_t)h * head_dim + d;
                const double qv = q16 ? (double)vko_fp16_to_float(q16[qi]) : (double)q32[qi];
                s += qv * vko_fp16_to_float(kr[d]);
            }
            s *= scale;
            sc[t] = s;
            if (s > mx) mx = s;
        }
        double den = 0.0;
        for (int t = 0; t < ctx; ++t) {
            sc[t] = exp(sc[t] - mx);
            den += sc[t];
        }
        for (int d = 0; d < head_dim; ++d) {
            double acc = 0.0;
            const uint16_t* vb = vcache + (((int64_t)kv * (head_dim / 8) + d / 8) * ctx) * 8 + d % 8;
            for (int t = 0; t < ctx; ++t) acc += sc[t] * vko_fp16_to_float(vb[(int64_t)t * 8]);
            out[(int64_t)h * head_dim + d] = (float)(acc / den);
        }
    }
    free(sc);
}

void vko_attention(const uint16_t* q, const uint16_t* kcache, const uint16_t* vcache, int n_q,
                   int n_kv, int head_dim, int ctx, float scale, float* out) {
    attention_impl(q, NULL, kcache, vcache, n_q, n_kv, head_dim, ctx, scale, out);
}

/* The same with an fp32 query (the decode chain's QKV output is fp32). */
void vko_attention_f32q(const float* q, const uint16_t* kcache, const uint16_t* vcache, int n_q,
                        int n_kv, int head_dim, int ctx, float scale, float* out) {
    attention_impl(NULL, q, kcache, vcache, n_q, n_kv, head_dim, ctx, scale, out);
}

/* shader/gemm.comp:19-59: C = A B, all row-major (A M x K, B K x N). */
void vko_gemm(const float* a, const float* b, int M, int N, int K, float* c) {
    double* acc = (double*)malloc(sizeof(double) * (size_t)N);
    for (int m = 0; m < M; ++m) {
        memset(acc, 0, sizeof(double) * (size_t)N);
        for (int k = 0; k < K; ++k) {
            const double av = a[(int64_t)m * K + k];
            const float* br = b + (int64_t)k * N;
            for (int n = 0; n < N; ++n) acc[n] += av * br[n];
        }
        for (int n = 0; n < N; ++n) c[(int64_t)m * N + n] = (float)acc[n];
    }
    free(acc);
}

/* ------------------------------------------------------------------------ */
/* Threaded operators on the reference's quantised storage                   */
/* ------------------------------------------------------------------------ */

static int g_threads = 1;

void vko_set_threads(int n) {
    g_threads = n < 1 ? 1 : n;
#ifdef _OPENMP
    omp_set_num_threads(g_threads);
#endif
}

int vko_get_threads(void) { return g_threads; }

/* One weight element of the reference storage: bits 32 (fp32), 16 (fp16
 * bits), 8 or 4 (codes with block-major s/z, dequantised q*s - z). */
static inline float weight_at(const void* data, const float* scale, const float* zero, int bits,
                              int K, int N, int k, int c) {
    switch (bits) {
        case 32: return ((const float*)data)[(int64_t)k * N + c];
        case 16: return vko_fp16_to_float(((const uint16_t*)data)[(int64_t)k * N + c]);
        default: {
            const int64_t si = (int64_t)(c / GROUP) * K + k;
            return (float)code_at((const uint8_t*)data, bits, K, N, k, c) * scale[si] - zero[si];
        }
    }
}

/* Accumulate acc[c - c0] += sum_k n[k] * W[k][c] for c in [c0, c1). */
static void accumulate_cols(const float* n, const void* data, const float* scale,
                            const float* zero, int bits, int K, int N, int c0, int c1,
                            double* acc) {
    for (int k = 0; k < K; ++k) {
        const double nk = n[k];
        for (int c = c0; c < c1; ++c)
            acc[c - c0] += nk * weight_at(data, scale, zero, bits, K, N, k, c);
    }
}

static float* normalised_input(const float* x, const float* gamma, int K, int rms_dim,
                               float eps) {
    float* n = (float*)malloc(sizeof(float) * (size_t)K);
    if (!gamma) {
        memcpy(n, x, sizeof(float) * (size_t)K);
        return n;
    }
    const float inv = vko_inv_rms(x, K, rms_dim, eps);
    for (int k = 0; k < K; ++k) n[k] = x[k] * gamma[k] * inv;
    return n;
}

/* GEMV (gamma == NULL; shader/GEMV-*.comp) or RmsNorm-GEMV
 * (shader/RmsNorm-GEMV-*.comp) straight from the reference's unpacked
 * storage, each thread owning a range of 256-output blocks. */
void vko_qgemv(const float* x, const float* gamma, const void* data, const float* scale,
               const float* zero, int bits, int K, int N, int rms_dim, float eps, float* y) {
    float* n = normalised_input(x, gamma, K, rms_dim, eps);
    const int nb = (N + GROUP - 1) / GROUP;
#pragma omp parallel for schedule(static) num_threads(g_threads)
    for (int b = 0; b < nb; ++b) {
        double acc[GROUP];
        const int c0 = b * GROUP, c1 = c0 + GROUP < N ? c0 + GROUP : N;
        memset(acc, 0, sizeof acc);
        accumulate_cols(n, data, scale, zero, bits, K, N, c0, c1, acc);
        for (int c = c0; c < c1; ++c) y[c] = (float)acc[c - c0];
    }
    free(n);
}

/* RmsNorm-SwiGLU (shader/RmsNorm-swiglu-ffn-*.comp) from unpacked storage. */
void vko_qswiglu(const float* x, const float* gamma, const void* dg, const float* sg,
                 const float* zg, const void* du, const float* su, const float* zu, int bits,
                 int K, int N, int rms_dim, float eps, float* h) {
    float* n = normalised_input(x, gamma, K, rms_dim, eps);
    const int nb = (N + GROUP - 1) / GROUP;
#pragma omp parallel for schedule(static) num_threads(g_threads)
    for (int b = 0; b < nb; ++b) {
        double ga[GROUP], ua[GROUP];
        const int c0 = b * GROUP, c1 = c0 + GROUP < N ? c0 + GROUP : N;
        memset(ga, 0, sizeof ga);
        memset(ua, 0, sizeof ua);
        accumulate_cols(n, dg, sg, zg, bits, K, N, c0, c1, ga);
        accumulate_cols(n, du, su, zu, bits, K, N, c0, c1, ua);
        for (int c = c0; c < c1; ++c) {
            const double g = (float)ga[c - c0];
            h[c] = (float)(g / (1.0 + exp2(-g * 1.44269504)) * (double)(float)ua[c - c0]);
        }
    }
    free(n);
}
