/* ggml.h - the one ggml function the reference's llama.cpp bridge
 * (src/llama_bridge.c) calls, so that the bridge compiles here without
 * llama.cpp. TEST INFRASTRUCTURE ONLY (oracle/Makefile, target ref).
 *
 * ggml_fp16_to_fp32 widens an IEEE 754 binary16 value to binary32, which is
 * exact for every input; this is a plain decode of the bit fields:
 * sign, 5-bit exponent (bias 15), 10-bit fraction; zero exponent =
 * subnormal (fraction * 2^-24), exponent 31 = inf / NaN (payload kept). */
#ifndef EAKV_ORACLE_GGML_STUB_H
#define EAKV_ORACLE_GGML_STUB_H
#include <stdint.h>
#include <string.h>

static inline float ggml_fp16_to_fp32(uint16_t h) {
    const uint32_t sign = (uint32_t)(h >> 15) << 31;
    const uint32_t exp = (h >> 10) & 0x1F;
    uint32_t frac = h & 0x3FF;
    uint32_t bits;
    if (exp == 0x1F) {
        bits = sign | 0x7F800000u | (frac << 13);
    } else if (exp != 0) {
        bits = sign | ((exp + 112) << 23) | (frac << 13);
    } else if (frac == 0) {
        bits = sign;
    } else {                         /* subnormal: normalise */
        int e = -1;
        do {
            frac <<= 1;
            e++;
        } while (!(frac & 0x400));
        bits = sign | ((uint32_t)(112 - e) << 23) | ((frac & 0x3FF) << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}
#endif
