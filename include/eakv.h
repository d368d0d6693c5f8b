/* eakv.h - public C API of the B200 Q4 KV-cache library (libeakv_b200.so).
 *
 * Drop-in for the reference library's public header (petlukk/eakv,
 * include/eakv.h:1-89): every declaration below has the same name, argument
 * list, return type and error convention as the reference, so a program
 * written against the reference links against this library unchanged.
 *
 * What differs is where the cache lives. The quantized cache (packed
 * nibbles + one f32 scale and one f32 bias per 64-element group) is held in
 * the HBM of the CUDA device that was current when the cache was created.
 * The data/queries/weights/scores/output pointers taken here are HOST
 * pointers, exactly as in the reference; device-pointer and fused/batched
 * entry points are declared in eakv_cuda.h.
 *
 * Thread safety: calls on distinct caches may run concurrently from
 * different host threads (reference include/eakv.h:3). Each cache owns its
 * own CUDA stream.
 */
#ifndef EAKV_H
#define EAKV_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Opaque handle (reference include/eakv.h:15). */
typedef struct eakv_cache eakv_cache_t;

/* Return codes (reference include/eakv.h:18-22). */
#define EAKV_OK              0
#define EAKV_ERR_IO         -1
#define EAKV_ERR_FORMAT     -2
#define EAKV_ERR_ALLOC      -3
#define EAKV_ERR_INVALID    -4

/* Lifecycle (reference src/cache.c:11-51).
 * NULL when any argument is <= 0, when n_kv_heads*head_dim is not a multiple
 * of 64, or when the device allocation fails. */
eakv_cache_t *eakv_cache_create(int n_layers, int n_kv_heads,
                                int head_dim, int max_seq_len);
void          eakv_cache_free(eakv_cache_t *cache);   /* NULL is a no-op */

/* Quantize a whole f32 cache (reference src/cache.c:60-100).
 * data: host f32[n_layers][2][n_kv_heads][seq_len][head_dim].
 * Sets seq_len. EAKV_ERR_INVALID on NULL, seq_len <= 0 or > max_seq_len. */
int eakv_cache_load_raw(eakv_cache_t *cache, const float *data, int seq_len);

/* Quantize n_tokens new positions of one (layer, K/V) pair at the current
 * seq_len (reference src/cache.c:102-151). data: host f32[n_kv_heads]
 * [n_tokens][head_dim]; kv_idx 0 = K, 1 = V. Does not change seq_len. */
int eakv_cache_append(eakv_cache_t *cache, const float *data,
                      int layer, int kv_idx, int n_tokens);

/* seq_len += n_tokens (reference src/cache.c:153-160). */
int eakv_cache_advance(eakv_cache_t *cache, int n_tokens);

/* seq_len = 0, memory kept (reference src/cache.c:162-164). */
void eakv_cache_clear(eakv_cache_t *cache);

/* O(1) checkpoint / rollback of seq_len (reference src/cache.c:166-176). */
int eakv_checkpoint(eakv_cache_t *cache);
int eakv_restore(eakv_cache_t *cache, int seq_len);

/* Attention on the quantized cache (reference src/attention.c:3-63).
 * queries f32[n_q_heads*head_dim], scores_out f32[n_q_heads*seq_len],
 * weights f32[n_q_heads*seq_len] (softmax weights from the caller),
 * output_out f32[n_q_heads*head_dim]. Q head q reads KV head
 * q / (n_q_heads/n_kv_heads). No return code, as in the reference; a
 * rejected call fills the output with NaN and records the reason for
 * eakv_last_error() (eakv_cuda.h). */
void eakv_attention_scores(const eakv_cache_t *cache, const float *queries,
                           int layer, int n_q_heads, int n_kv_heads,
                           float *scores_out);

void eakv_attention_output(const eakv_cache_t *cache, const float *weights,
                           int layer, int n_q_heads, int n_kv_heads,
                           float *output_out);

/* .eakv files (reference src/io.c:39-160), same on-disk layout. */
int eakv_cache_save(const eakv_cache_t *cache, const char *path);
int eakv_cache_load(const char *path, eakv_cache_t **out);

/* Info getters; 0 for a NULL cache (reference src/cache.c:178-201). */
int   eakv_cache_seq_len(const eakv_cache_t *cache);
int   eakv_cache_n_layers(const eakv_cache_t *cache);
int   eakv_cache_n_heads(const eakv_cache_t *cache);
int   eakv_cache_head_dim(const eakv_cache_t *cache);
int   eakv_cache_max_seq_len(const eakv_cache_t *cache);
float eakv_cache_compression_ratio(const eakv_cache_t *cache);

#ifdef __cplusplus
}
#endif

#endif /* EAKV_H */
