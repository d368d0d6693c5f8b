/* eakv_ggml.h - the q4_1_eakv ggml block type, served by libeakv_b200.so.
 *
 * The first three declarations are the reference's ggml type callbacks
 * with their exact signatures (reference include/eakv_ggml.h:25-52,
 * src/ggml_type.c:21-242); a llama.cpp type registration that links the
 * reference's libeakv links this library instead. They take HOST pointers,
 * like the reference's, and copy through the GPU on every call.
 *
 * The *_device functions are the GPU forms: the same arithmetic on device
 * pointers, ordered on `stream` (NULL: the legacy default stream), for a
 * CUDA backend that keeps its KV cache in q4_1_eakv blocks.
 *
 * Results equal the reference's AVX-512 build bit for bit (blocks, d, m,
 * dequantized values, dot products), except the payload bits of a NaN that
 * arithmetic produces (x86 and the GPU make different ones). Note that this block type stores
 * d = range/15 = 0 for a constant block, where the cache's own quantizer
 * (eakv.h) stores a scale of 1.
 */
#ifndef EAKV_GGML_H
#define EAKV_GGML_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define QK_EAKV 64

/* 40-byte block of 64 elements (reference include/eakv_ggml.h:27-31). */
typedef struct {
    uint8_t qs[32]; /* lo nibble of qs[k] = element k, hi nibble = element k+32 */
    float d;        /* scale */
    float m;        /* min (bias) */
} block_q4_1_eakv;

/* from_float (reference eakv_ggml.h:36, ggml_type.c:21): k / 64 blocks. */
void eakv_quantize_row(const float *src, void *dst, int64_t k);

/* to_float (reference eakv_ggml.h:37, ggml_type.c:99): value = n*d + m. */
void eakv_dequantize_row(const void *src, float *dst, int64_t k);

/* vec_dot (reference eakv_ggml.h:50-52, ggml_type.c:138): row r of x
 * (vx + r*bx, q4_1_eakv) dotted with row r of y (vy + r*by, f32) into
 * s + r*bs, for r < nrc; n elements per row. The reference handles nrc 1
 * and 2; any nrc >= 1 works here. */
void eakv_vec_dot_q4_f32(int n, float *s, size_t bs, const void *vx, size_t bx, const void *vy,
                         size_t by, int nrc);

/* ---- GPU forms (no reference counterpart: the reference has only the CPU
 * callbacks above). Device pointers; they return EAKV_OK, EAKV_ERR_INVALID
 * for bad arguments (eakv_last_error_string() in eakv_cuda.h says which),
 * or the error of a failed launch. -------------------------------------- */
int eakv_ggml_quantize_row_device(const float *d_src, void *d_dst, int64_t k, void *stream);
int eakv_ggml_dequantize_row_device(const void *d_src, float *d_dst, int64_t k, void *stream);
int eakv_ggml_vec_dot_device(int n, float *d_s, size_t bs, const void *d_vx, size_t bx,
                             const void *d_vy, size_t by, int nrc, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* EAKV_GGML_H */
