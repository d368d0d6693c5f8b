/* fp16_stub_check.c - exports the ggml_stub/ggml.h half -> float decode so
 * that tests/test_llama_oracle.py can check it against numpy on all 65536
 * half values. TEST INFRASTRUCTURE ONLY. */
#include "ggml_stub/ggml.h"

void fp16_stub_convert(const uint16_t *h, float *f, int n) {
    for (int i = 0; i < n; i++) f[i] = ggml_fp16_to_fp32(h[i]);
}
