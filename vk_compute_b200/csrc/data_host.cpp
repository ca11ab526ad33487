// Host data generators, quantisers and packer of include/data.h, with the
// arithmetic of vk-compute's src/data.c:8-233 (bit-identical outputs), so
// that the reference's own driver (src/compute.c) links against
// libvkcompute alone.
extern "C" {
#include "data.h"
}

#include <cmath>
#include <cstring>

namespace {
constexpr int kGroup = 256;  // src/data.c:99,143

uint32_t mix(int i, int j, int seed) {
    uint32_t h = static_cast<uint32_t>(i) * 73129u + static_cast<uint32_t>(j) * 95121u +
                 static_cast<uint32_t>(seed) * 15473u;
    h = (h ^ 61u) ^ (h >> 16);
    h += h << 3;
    h ^= h >> 4;
    h *= 0x27d4eb2du;
    h ^= h >> 15;
    return h;
}

// Shared min/max quantiser of src/data.c:95-185 (levels 255 or 15).
QuantizedData quantise(int seed, int M, int N, int bits) {
    QuantizedData q;
    memset(&q, 0, sizeof q);
    q.M = M;
    q.N = N;
    q.group_size = kGroup;
    q.type = bits == 8 ? QUANT_INT8 : QUANT_INT4;
    const int nb = N / kGroup;
    const size_t bytes = bits == 8 ? static_cast<size_t>(M) * N : static_cast<size_t>(M) * N / 2;
    q.data = static_cast<uint8_t*>(malloc(bytes ? bytes : 1));
    q.scale = static_cast<float*>(malloc(sizeof(float) * (static_cast<size_t>(M) * nb + 1)));
    q.z = static_cast<float*>(malloc(sizeof(float) * (static_cast<size_t>(M) * nb + 1)));
    const float levels = bits == 8 ? 255.0f : 15.0f;
    for (int k = 0; k < M; ++k) {
        for (int b = 0; b < nb; ++b) {
            float lo = 1e9f, hi = -1e9f;
            for (int t = 0; t < kGroup; ++t) {
                const float v = get_pseudo_random(k, b * kGroup + t, seed);
                if (v < lo) lo = v;
                if (v > hi) hi = v;
            }
            const size_t si = static_cast<size_t>(b) * M + k;
            q.scale[si] = (hi - lo) / levels;
            q.z[si] = -lo;
            for (int t = 0; t < kGroup; ++t) {
                const int c = b * kGroup + t;
                const uint8_t v = static_cast<uint8_t>(
                    roundf((get_pseudo_random(k, c, seed) + q.z[si]) / q.scale[si]));
                if (bits == 8) {
                    q.data[static_cast<size_t>(k) * N + c] = v;
                } else {
                    uint8_t& p = q.data[static_cast<size_t>(k) * (N / 2) + c / 2];
                    p = (c & 1) ? static_cast<uint8_t>(p | (v & 0x0f)) : static_cast<uint8_t>((v & 0x0f) << 4);
                }
            }
        }
    }
    return q;
}
}  // namespace

extern "C" {

float get_pseudo_random(int i, int j, int seed) {
    return (static_cast<float>(mix(i, j, seed) % 2000001u) / 1000000.0f) - 1.0f;
}

float* getData(int seed, int M, int N) {
    float* a = static_cast<float*>(malloc(sizeof(float) * static_cast<size_t>(M) * N));
    for (int i = 0; i < M; ++i)
        for (int j = 0; j < N; ++j) a[static_cast<size_t>(i) * N + j] = get_pseudo_random(i, j, seed);
    return a;
}

uint16_t float_to_fp16(float f) {
    uint32_t b;
    memcpy(&b, &f, sizeof b);
    const uint32_t sign = (b >> 16) & 0x8000u;
    const int e = static_cast<int>((b >> 23) & 0xffu) - 127;
    const uint32_t m = b & 0x7fffffu;
    if (e <= -15) {
        if (e < -24) return static_cast<uint16_t>(sign);
        return static_cast<uint16_t>(sign | ((m | 0x800000u) >> (1 - e)));
    }
    if (e >= 16) return static_cast<uint16_t>(sign | 0x7c00u);
    return static_cast<uint16_t>(sign | (static_cast<uint32_t>(e + 15) << 10) | (m >> 13));
}

float fp16_to_float(uint16_t h) {
    const uint32_t sign = static_cast<uint32_t>(h & 0x8000u) << 16;
    int e = (h >> 10) & 0x1f;
    uint32_t m = h & 0x3ffu, out;
    if (e == 0) {
        if (m == 0) {
            out = sign;
        } else {
            int ee = -14;
            while (!(m & 0x400u)) {
                m <<= 1;
                --ee;
            }
            out = sign | (static_cast<uint32_t>(ee + 127) << 23) | ((m & 0x3ffu) << 13);
        }
    } else if (e == 31) {
        out = sign | 0x7f800000u | (m << 13);
    } else {
        out = sign | (static_cast<uint32_t>(e - 15 + 127) << 23) | (m << 13);
    }
    float f;
    memcpy(&f, &out, sizeof f);
    return f;
}

uint16_t* getDataFP16(int seed, int M, int N) {
    uint16_t* a = static_cast<uint16_t*>(malloc(sizeof(uint16_t) * static_cast<size_t>(M) * N));
    for (int i = 0; i < M; ++i)
        for (int j = 0; j < N; ++j)
            a[static_cast<size_t>(i) * N + j] = float_to_fp16(get_pseudo_random(i, j, seed));
    return a;
}

QuantizedData getDataINT8(int seed, int M, int N) { return quantise(seed, M, N, 8); }
QuantizedData getDataINT4(int seed, int M, int N) { return quantise(seed, M, N, 4); }

void transpose(const float* src, float* dest, int m, int n) {
    for (int i = 0; i < m; ++i)
        for (int j = 0; j < n; ++j) dest[static_cast<size_t>(j) * m + i] = src[static_cast<size_t>(i) * n + j];
}

void transpose_block16(const uint8_t* input, uint8_t* output, int M, int N, int data_type) {
    const int per = 128 / data_type;
    for (int r = 0; r < M / per; ++r)
        for (int j = 0; j < N; ++j) {
            uint8_t* chunk = output + (static_cast<size_t>(r) * N + j) * 16;
            if (data_type == 4) {
                memset(chunk, 0, 16);
                for (int t = 0; t < per; ++t) {
                    const uint8_t byte = input[static_cast<size_t>(r * per + t) * (N / 2) + j / 2];
                    const uint8_t q = (j & 1) ? (byte & 0x0f) : static_cast<uint8_t>(byte >> 4);
                    chunk[t / 2] |= static_cast<uint8_t>((t & 1) ? (q << 4) : q);
                }
            } else {
                const int eb = data_type / 8;
                for (int t = 0; t < per; ++t)
                    memcpy(chunk + t * eb, input + (static_cast<size_t>(r * per + t) * N + j) * eb, eb);
            }
        }
}

void free_quantized_data(QuantizedData q) {
    free(q.data);
    free(q.scale);
    free(q.z);
}

}  // extern "C"
