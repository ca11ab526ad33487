/*
 * oracle.h -- CPU restatement of vk-compute's matrix-vector decode path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the checker: the parity tests,
 * the smoke check and the CPU-baseline leg of the benchmark load it to
 * compute the expected result.  The product (libvkcompute.so) never links,
 * loads or calls it, and nothing here is a fallback for the CUDA path.
 *
 * Every function names the reference file:line whose behaviour it restates.
 * Reference paths are given relative to the vk-compute project root.
 *
 * Pinning: the data generators, fp16 conversion, quantisers and the
 * transpose_block16 packer are checked bit-for-bit against the reference's own
 * src/data.c (compiled into oracle/_ref by oracle/build_ref.sh) through the
 * committed fixtures in tests/golden.  The operator formulas follow the
 * reference's CPU validation loops (src/compute.c:216-290) and the shader
 * arithmetic; RoPE and attention have no CPU check in the reference, so their
 * parity is unpinned (documented per function).
 */
#ifndef VKC_ORACLE_H
#define VKC_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- data generation and conversion (src/data.c) ---- */
float vko_pseudo_random(int i, int j, int seed);
void vko_get_data(int seed, int M, int N, float* out);
uint16_t vko_float_to_fp16(float f);
float vko_fp16_to_float(uint16_t h);
void vko_get_data_fp16(int seed, int M, int N, uint16_t* out);
void vko_get_data_int8(int seed, int M, int N, uint8_t* data, float* scale, float* zero);
void vko_get_data_int4(int seed, int M, int N, uint8_t* data, float* scale, float* zero);
void vko_transpose_block16(const uint8_t* in, uint8_t* out, int M, int N, int bits);

/* ---- quantisers of given fp32 matrices (same layouts as data.c) ---- */
void vko_quantize_asym(const float* w, int K, int N, int bits,
                       uint8_t* data, float* scale, float* zero);
void vko_quantize_sym(const float* w, int K, int N, int bits, int fp16_scale,
                      uint8_t* data, float* scale, float* zero);

/* ---- dequantisation into a dense K x N fp32 matrix ---- */
void vko_dequant(const uint8_t* data, const float* scale, const float* zero,
                 int K, int N, int bits, float* w);
void vko_fp16_matrix_to_float(const uint16_t* h, int64_t count, float* out);

/* ---- operators (dense K x N weights, W[k*N + j]) ---- */
void vko_gemv(const float* x, const float* w, int K, int N, float* y);
float vko_inv_rms(const float* x, int K, int rms_dim, float eps);
void vko_rmsnorm_rows(float* x, const float* gamma, int rows, int width, float eps);
void vko_rmsnorm_gemv(const float* x, const float* gamma, const float* w, int K, int N,
                      int rms_dim, float eps, float* y);
void vko_rope_reference(float* y, int N, int pos, const float* theta);
void vko_rope_pairs(float* y, int N, int head_dim, int rot_rows, int pos, const float* theta);
void vko_swiglu(const float* x, const float* gamma, const float* wg, const float* wu,
                int K, int N, int rms_dim, float eps, float* h);
void vko_attention(const uint16_t* q, const uint16_t* kcache, const uint16_t* vcache,
                   int n_q, int n_kv, int head_dim, int ctx, float scale, float* out);
void vko_attention_f32q(const float* q, const uint16_t* kcache, const uint16_t* vcache, int n_q,
                        int n_kv, int head_dim, int ctx, float scale, float* out);
void vko_gemm(const float* a, const float* b, int M, int N, int K, float* c);

/* ---- the same operators on the reference's unpacked storage, threaded ----
 * bits: 32 = fp32 K x N, 16 = fp16 bits K x N, 8 = u8 codes K x N,
 * 4 = two codes per byte (even output high nibble); scale/zero block-major.
 * gamma == NULL selects plain GEMV (no normalisation). */
void vko_set_threads(int n);
int vko_get_threads(void);
void vko_qgemv(const float* x, const float* gamma, const void* data, const float* scale,
               const float* zero, int bits, int K, int N, int rms_dim, float eps, float* y);
void vko_qswiglu(const float* x, const float* gamma, const void* dg, const float* sg,
                 const float* zg, const void* du, const float* su, const float* zu, int bits,
                 int K, int N, int rms_dim, float eps, float* h);

#ifdef __cplusplus
}
#endif
#endif
