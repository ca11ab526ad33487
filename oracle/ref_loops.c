/*
 * Checker-side harness for vk-compute's own CPU validation loops.
 *
 * TEST INFRASTRUCTURE ONLY.  src/compute.c checks one output element of each
 * operator with plain C loops (src/compute.c:216-290); most of them are
 * commented out, one at a time being active.  oracle/build_ref.sh extracts
 * those line ranges from the mounted sources, uncommented, into
 * oracle/_ref/loops/*.inc, and compiles this file against them together with
 * the reference's src/data.c, so the loops below run exactly as the reference
 * wrote them on exactly the inputs compute.c builds (src/compute.c:18-46).
 * tests/golden/make_golden.py stores their results as fixtures, which pin the
 * oracle's operator arithmetic (dequantisation q*s - z, nibble order, RMS and
 * SiLU forms) to the reference's own code.
 *
 * As written, the quantised loops read scale[i] and z[i], the scales of the
 * first 256-output block, and INT4 takes the high nibble (the even output of
 * a byte), so they are meaningful for even idx < 256 only; the harness takes
 * the indices from its caller.
 *
 * Each function: inputs input = getData(seed_x, 1, K), gamma =
 * getData(seed_g, 1, K), weight = getData(seed_w, K, N) and the INT8 / INT4
 * quantisations getDataINT8/INT4(seed_w, K, N) (src/compute.c:18-20, 28, 32);
 * out[n] = the loop's result for output idx[n].
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>

#include "data.h" /* the reference's include/data.h */

typedef struct {
    float* input;
    float* gamma;
    float* weight;
    QuantizedData weightINT8;
    QuantizedData weightINT4;
} inputs;

static inputs make_inputs(int K, int N, int seed_x, int seed_g, int seed_w) {
    inputs in;
    in.input = getData(seed_x, 1, K);
    in.gamma = getData(seed_g, 1, K);
    in.weight = getData(seed_w, K, N);
    in.weightINT8 = getDataINT8(seed_w, K, N);
    in.weightINT4 = getDataINT4(seed_w, K, N);
    return in;
}

static void free_inputs(inputs in) {
    free(in.input);
    free(in.gamma);
    free(in.weight);
    free_quantized_data(in.weightINT8);
    free_quantized_data(in.weightINT4);
}

/* The names the loops use, bound to one call's inputs. */
#define BIND(in)                                  \
    float* input = (in).input;                    \
    float* gamma = (in).gamma;                    \
    float* weight = (in).weight;                  \
    QuantizedData weightINT8 = (in).weightINT8;   \
    QuantizedData weightINT4 = (in).weightINT4;   \
    (void)input;                                  \
    (void)gamma;                                  \
    (void)weight;                                 \
    (void)weightINT8;                             \
    (void)weightINT4

/* src/compute.c:216-218: GEMV, fp32 weights. */
void vkref_gemv_f32(int K, int N, int seed_x, int seed_g, int seed_w, const int* idxs, int n, float* out) {
    inputs in = make_inputs(K, N, seed_x, seed_g, seed_w);
    BIND(in);
    for (int t = 0; t < n; ++t) {
        int idx = idxs[t];
        float result = 0.0f;
#include "gemv_f32.inc"
        out[t] = result;
    }
    free_inputs(in);
}

/* src/compute.c:221-226: RmsNorm-GEMV, fp32 weights (the active check). */
void vkref_rmsnorm_gemv_f32(int K, int N, int seed_x, int seed_g, int seed_w, const int* idxs, int n,
                            float* out) {
    inputs in = make_inputs(K, N, seed_x, seed_g, seed_w);
    BIND(in);
    for (int t = 0; t < n; ++t) {
        int idx = idxs[t];
        float result = 0.0f;
#include "rms.inc"
#include "rmsnorm_gemv_f32.inc"
        out[t] = result;
    }
    free_inputs(in);
}

/* src/compute.c:229-241: RmsNorm-SwiGLU, fp32 weights (gate and up read the
 * same matrix, as written). */
void vkref_swiglu_f32(int K, int N, int seed_x, int seed_g, int seed_w, const int* idxs, int n, float* out) {
    inputs in = make_inputs(K, N, seed_x, seed_g, seed_w);
    BIND(in);
    for (int t = 0; t < n; ++t) {
        int idx = idxs[t];
        float result = 0.0f;
#include "swiglu_f32.inc"
        out[t] = result;
    }
    free_inputs(in);
}

/* src/compute.c:221-223 then 244-256: RmsNorm-SwiGLU, INT8 (gate = up). */
void vkref_swiglu_int8(int K, int N, int seed_x, int seed_g, int seed_w, const int* idxs, int n, float* out) {
    inputs in = make_inputs(K, N, seed_x, seed_g, seed_w);
    BIND(in);
    for (int t = 0; t < n; ++t) {
        int idx = idxs[t];
        float gate, up;
#include "rms.inc"
#include "swiglu_int8.inc"
        out[t] = quantizedResult;
    }
    free_inputs(in);
}

/* src/compute.c:221-223 then 258-272: RmsNorm-SwiGLU, INT4 (gate = up). */
void vkref_swiglu_int4(int K, int N, int seed_x, int seed_g, int seed_w, const int* idxs, int n, float* out) {
    inputs in = make_inputs(K, N, seed_x, seed_g, seed_w);
    BIND(in);
    for (int t = 0; t < n; ++t) {
        int idx = idxs[t];
        float gate, up;
#include "rms.inc"
#include "swiglu_int4.inc"
        out[t] = quantizedResult;
    }
    free_inputs(in);
}

/* src/compute.c:277-283: GEMV, INT4. */
void vkref_gemv_int4(int K, int N, int seed_x, int seed_g, int seed_w, const int* idxs, int n, float* out) {
    inputs in = make_inputs(K, N, seed_x, seed_g, seed_w);
    BIND(in);
    for (int t = 0; t < n; ++t) {
        int idx = idxs[t];
        float result = 0.0f;
#include "gemv_int4.inc"
        (void)result;
        out[t] = quantizedResult;
    }
    free_inputs(in);
}

/* src/compute.c:284-290: GEMV, INT8. */
void vkref_gemv_int8(int K, int N, int seed_x, int seed_g, int seed_w, const int* idxs, int n, float* out) {
    inputs in = make_inputs(K, N, seed_x, seed_g, seed_w);
    BIND(in);
    for (int t = 0; t < n; ++t) {
        int idx = idxs[t];
        float result = 0.0f;
#include "gemv_int8.inc"
        (void)result;
        out[t] = quantizedResult;
    }
    free_inputs(in);
}
