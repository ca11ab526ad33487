/* End-to-end timing of an operator through the reference-facing C ABI, as a
 * C host program would drive it: per step writeBuffer(x) from host memory,
 * execute() of the operator by its shader name, readBuffer(y) into host
 * memory, timed on the host clock.  Weights rotate through a pool larger than
 * four times the L2 cache so every step streams them from HBM.
 *
 *   vkc_e2e_bench <op> <N> <K> <steps> <warmup> [gemv_plan]
 *   op: RmsNorm-GEMV-INT8 | GEMV-FP16; gemv_plan: vkc_set_gemv_plan's value
 *   for the calling thread (default: the library's automatic choice)
 * The program never asks for getExecutionTime, so it turns execute()'s timing
 * events off (vkc_set_timing(0)), as such a program would.
 * Prints one JSON object: us_per_step, h2d_bytes_per_step, d2h_bytes_per_step,
 * and the host time of each call (write / execute / read, us per step). */
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

#include "dispatch.h"
#include "session.h"
#include "vk_compute_b200.h"

static uint64_t rng = 0x9E3779B97F4A7C15ull;
static uint32_t next_u32(void) {
    rng ^= rng << 13;
    rng ^= rng >> 7;
    rng ^= rng << 17;
    return (uint32_t)(rng >> 11);
}
static float next_f(void) { return (float)(next_u32() & 0xFFFFFF) / 16777216.0f * 2.0f - 1.0f; }

static double now_us(void) {
    struct timespec t;
    clock_gettime(CLOCK_MONOTONIC, &t);
    return t.tv_sec * 1e6 + t.tv_nsec * 1e-3;
}

int main(int argc, char** argv) {
    if (argc < 6) {
        fprintf(stderr, "usage: %s <RmsNorm-GEMV-INT8|GEMV-FP16> <N> <K> <steps> <warmup>\n", argv[0]);
        return 2;
    }
    const char* op = argv[1];
    const int N = atoi(argv[2]), K = atoi(argv[3]), steps = atoi(argv[4]), warmup = atoi(argv[5]);
    const int int8 = strcmp(op, "RmsNorm-GEMV-INT8") == 0;
    if (!int8 && strcmp(op, "GEMV-FP16") != 0) {
        fprintf(stderr, "unknown operator %s\n", op);
        return 2;
    }
    const size_t wbytes = int8 ? (size_t)N * K : (size_t)N * K * 2;
    const size_t sbytes = int8 ? (size_t)(N / 256) * K * 4 : 0;
    const size_t l2 = 126u << 20;
    int pool = (int)((4 * l2 + wbytes + 2 * sbytes - 1) / (wbytes + 2 * sbytes));
    if (pool < 2) pool = 2;
    if (pool > 64) pool = 64;

    vkc_set_timing(0);
    if (argc > 6 && vkc_set_gemv_plan(atoi(argv[6])) != 0) {
        fprintf(stderr, "%s\n", vkc_last_error());
        return 2;
    }
    session s = createSession();
    uint8_t* hw = (uint8_t*)malloc(wbytes);
    float* hs = (float*)malloc(sbytes ? sbytes : 4);
    float* hz = (float*)malloc(sbytes ? sbytes : 4);
    float* hx = (float*)malloc((size_t)K * 4);
    float* hg = (float*)malloc((size_t)K * 4);
    float* hy = (float*)malloc((size_t)N * 4);
    for (size_t i = 0; i < wbytes / 4; ++i) ((uint32_t*)hw)[i] = int8 ? next_u32() : (next_u32() & 0x1FFF1FFFu);
    for (size_t i = 0; i < sbytes / 4; ++i) {
        hs[i] = 1e-4f * (1.0f + 0.5f * next_f());
        hz[i] = 128.0f * hs[i];
    }
    for (int i = 0; i < K; ++i) {
        hx[i] = next_f();
        hg[i] = 1.0f + 0.1f * next_f();
    }
    buffer xb = createBuffer(s.dev.device, s.dev.physicalDevice, hx, (int64_t)K * 4, MEMORY_VRAM);
    buffer gb = createBuffer(s.dev.device, s.dev.physicalDevice, hg, (int64_t)K * 4, MEMORY_VRAM);
    buffer yb = createBuffer(s.dev.device, s.dev.physicalDevice, NULL, (int64_t)N * 4, MEMORY_VRAM);
    operation* ops = (operation*)calloc((size_t)pool, sizeof(operation));
    buffer* wbs = (buffer*)calloc((size_t)pool * 3, sizeof(buffer));
    for (int p = 0; p < pool; ++p) {
        wbs[3 * p] = createBuffer(s.dev.device, s.dev.physicalDevice, hw, (int64_t)wbytes, MEMORY_VRAM);
        operation* o = &ops[p];
        snprintf(o->shader, sizeof o->shader, "%s.spv", op);
        o->pushConstants[0] = 1;
        o->pushConstants[1] = N;
        o->pushConstants[2] = K;
        o->pushConstantCount = 3;
        if (int8) {
            wbs[3 * p + 1] = createBuffer(s.dev.device, s.dev.physicalDevice, hs, (int64_t)sbytes, MEMORY_VRAM);
            wbs[3 * p + 2] = createBuffer(s.dev.device, s.dev.physicalDevice, hz, (int64_t)sbytes, MEMORY_VRAM);
            o->buffers[0] = xb;
            o->buffers[1] = gb;
            o->buffers[2] = wbs[3 * p];
            o->buffers[3] = yb;
            o->buffers[4] = wbs[3 * p + 1];
            o->buffers[5] = wbs[3 * p + 2];
            o->bufferCount = 6;
        } else {
            o->buffers[0] = xb;
            o->buffers[1] = wbs[3 * p];
            o->buffers[2] = yb;
            o->bufferCount = 3;
        }
    }
    for (int i = 0; i < warmup; ++i) {
        writeBuffer(s.dev.device, s.dev.queue, xb, hx);
        execute(s, &ops[i % pool], 1);
        readBuffer(s.dev.device, s.dev.physicalDevice, s.dev.queue, yb, hy);
    }
    double t_write = 0, t_exec = 0, t_read = 0;
    const double t0 = now_us();
    for (int i = 0; i < steps; ++i) {
        const double a = now_us();
        writeBuffer(s.dev.device, s.dev.queue, xb, hx);
        const double b = now_us();
        execute(s, &ops[(warmup + i) % pool], 1);
        const double c = now_us();
        readBuffer(s.dev.device, s.dev.physicalDevice, s.dev.queue, yb, hy);
        const double d = now_us();
        t_write += b - a;
        t_exec += c - b;
        t_read += d - c;
    }
    const double us = (now_us() - t0) / steps;
    double check = 0;
    for (int i = 0; i < N; ++i) check += hy[i];
    printf("{\"us_per_step\": %.3f, \"h2d_bytes_per_step\": %d, \"d2h_bytes_per_step\": %d, \"pool\": %d, "
           "\"steps\": %d, \"warmup\": %d, \"checksum\": %.6e, \"us_write\": %.3f, \"us_execute\": %.3f, "
           "\"us_read\": %.3f}\n",
           us, K * 4, N * 4, pool, steps, warmup, check, t_write / steps, t_exec / steps, t_read / steps);
    for (int p = 0; p < pool; ++p)
        for (int j = 0; j < (int8 ? 3 : 1); ++j) destroyBuffer(s.dev.device, wbs[3 * p + j]);
    destroyBuffer(s.dev.device, xb);
    destroyBuffer(s.dev.device, gb);
    destroyBuffer(s.dev.device, yb);
    destroySession(s);
    free(hw);
    free(hs);
    free(hz);
    free(hx);
    free(hg);
    free(hy);
    free(ops);
    free(wbs);
    return 0;
}
