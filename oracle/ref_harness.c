/*
 * Checker-side harness linked with vk-compute's own src/data.c by
 * oracle/build_ref.sh.  It stores the reference's fp16_to_float results as
 * raw fp32 bits, so no float->double round trip (which quiets signalling
 * NaNs) sits between the reference and the golden fixture.
 */
#include <stdint.h>
#include <string.h>

float fp16_to_float(uint16_t h); /* src/data.c:53 */

void vkref_fp16_to_float_all(uint32_t* out) {
    for (uint32_t h = 0; h < 65536u; ++h) {
        float f = fp16_to_float((uint16_t)h);
        memcpy(&out[h], &f, sizeof f);
    }
}
