/* eakv_cuda.h - extension entry points of libeakv_b200.so.
 *
 * Everything in eakv.h keeps the reference's host-pointer contract. The
 * calls below add what a GPU-resident cache needs and the reference has no
 * counterpart for: device-pointer variants (no host copies, asynchronous on
 * the cache's CUDA stream), the fused softmax attention the reference
 * ships only as an unexposed kernel (reference kernels/fused_attention.ea:
 * 10-373), a batched decode step over many caches and all layers, and the
 * sequence-split partial + log-sum-exp combine used across GPUs.
 *
 * All functions return EAKV_OK or a negative EAKV_ERR_* code unless noted;
 * the reason of the last failure on the calling host thread is available
 * from eakv_last_error_string(). Pointer arguments named d_* are device
 * pointers on the cache's device; "stream" arguments are cudaStream_t
 * (NULL selects the first cache's own stream).
 */
#ifndef EAKV_CUDA_H
#define EAKV_CUDA_H

#include <stddef.h>
#include "eakv.h"

#ifdef __cplusplus
extern "C" {
#endif

/* ---- errors and device state ---------------------------------------- */

/* Code of the last failed call on this host thread, EAKV_OK if none. The
 * void attention functions of eakv.h (reference src/attention.c:3-63 has no
 * error channel) report through this. */
int         eakv_last_error(void);
const char *eakv_last_error_string(void);

/* Sticky device status word of the library's kernels on `device`: 0 when
 * clean, else a bitmask (1 = a pipeline wait ran out of its bound, 2 = a
 * decode work item failed its index check and was skipped, 4 = a decode
 * CTA found a copy still in flight at its end and drained it). reset != 0
 * clears it. Synchronizes the device.
 * Returns the status, or a negative EAKV_ERR_* code. */
int eakv_device_status(int device, int reset);

/* ---- placement ------------------------------------------------------- */

/* Device on which this host thread's later eakv_cache_create / load calls
 * place caches (the library keeps its own CUDA runtime state, so a device
 * chosen through another runtime, e.g. a framework, is not seen here). */
int    eakv_set_device(int device);

int    eakv_cache_device(const eakv_cache_t *cache);         /* -1 for NULL */
/* HBM held by the cache: its page slab plus the scratch that host-buffer
 * calls and split decodes grow on demand. */
size_t eakv_cache_device_bytes(const eakv_cache_t *cache);
/* Stream used by this cache's calls; NULL restores the cache's own. */
int    eakv_cache_set_stream(eakv_cache_t *cache, void *stream);
void  *eakv_cache_stream(const eakv_cache_t *cache);
int    eakv_cache_synchronize(const eakv_cache_t *cache);

/* ---- device-pointer variants of eakv.h ------------------------------- */

/* As eakv_cache_load_raw / eakv_cache_append with device input
 * (reference src/cache.c:60-151); asynchronous. */
int eakv_cache_load_raw_device(eakv_cache_t *cache, const float *d_data,
                               int seq_len);
int eakv_cache_append_device(eakv_cache_t *cache, const float *d_data,
                             int layer, int kv_idx, int n_tokens);
/* One launch for every layer and K/V: d_data is
 * f32[n_layers][2][n_kv_heads][n_tokens][head_dim]. Writes at seq_len and,
 * like eakv_cache_append, does not advance. */
int eakv_cache_append_step_device(eakv_cache_t *cache, const float *d_data,
                                  int n_tokens);

/* As eakv_attention_scores / eakv_attention_output (reference
 * src/attention.c:3-63) on device buffers; asynchronous. */
int eakv_attention_scores_device(const eakv_cache_t *cache,
                                 const float *d_queries, int layer,
                                 int n_q_heads, int n_kv_heads,
                                 float *d_scores);
int eakv_attention_output_device(const eakv_cache_t *cache,
                                 const float *d_weights, int layer,
                                 int n_q_heads, int n_kv_heads,
                                 float *d_output);

/* ---- fused softmax attention ----------------------------------------- */

/* output = softmax(Q K^T / sqrt(head_dim)) V for one layer, host buffers
 * (queries/output f32[n_q_heads*head_dim]); the device counterpart of
 * reference kernels/fused_attention.ea:190-373 for any head mapping. */
int eakv_attention_fused(const eakv_cache_t *cache, const float *queries,
                         int layer, int n_q_heads, int n_kv_heads,
                         float *output);
int eakv_attention_fused_device(const eakv_cache_t *cache,
                                const float *d_queries, int layer,
                                int n_q_heads, int n_kv_heads,
                                float *d_output);

/* Batched decode step: n_caches caches of identical shape (layers, KV
 * heads, head_dim, max_seq_len), each attended over its own seq_len, all
 * layers in one launch. d_queries / d_output are
 * f32[n_caches][n_layers][n_q_heads][head_dim]. n_caches <= 256. */
int eakv_decode_attention(const eakv_cache_t *const *caches, int n_caches,
                          const float *d_queries, int n_q_heads,
                          float *d_output, void *stream);
/* Same as eakv_decode_attention, for callers that cannot allocate device
 * memory: no counterpart in the reference, whose CPU path has no device
 * memory at all. A framework whose caching allocator owns the GPU, or a
 * decode loop that must not block on cudaMalloc/cudaFree, gets the
 * split-merge workspace from a fixed 4 MiB array in the library's device
 * image (held by every GPU that loads the library) instead of from cache
 * scratch grown with cudaMalloc. Calls needing more than 4 MiB of workspace
 * return EAKV_ERR_INVALID. All calls on a device share the array: calls
 * whose kernels overlap on the GPU race. The first call on a device looks
 * up the array's address and should come before any stream capture. */
int eakv_decode_attention_noalloc(const eakv_cache_t *const *caches,
                                  int n_caches, const float *d_queries,
                                  int n_q_heads, float *d_output, void *stream);
/* Same with host buffers; copies in, decodes, copies out, synchronizes.
 * From 256 KiB of queries on, the batch is cut into up to four chunks of
 * caches (or of layers, for one cache) whose copies overlap the other
 * chunks' decodes; every chunk keeps the whole batch's split plan, so the
 * outputs equal eakv_decode_attention's bit for bit. */
int eakv_decode_attention_host(const eakv_cache_t *const *caches,
                               int n_caches, const float *queries,
                               int n_q_heads, float *output, void *stream);

/* Number of kernel launches one eakv_decode_attention call over these
 * caches makes: 1 (rows cut into sequence splits are merged inside the same
 * launch by the last CTA of each row group); < 0 on error. */
int eakv_decode_launches(const eakv_cache_t *const *caches, int n_caches,
                         int n_q_heads);
/* Sequence splits per row the planner chooses for one eakv_decode_attention
 * call over these caches (1: rows are not split and no split workspace is
 * used); < 0 on error. */
int eakv_decode_splits(const eakv_cache_t *const *caches, int n_caches,
                       int n_q_heads);

/* ---- sequence-split partials and exact combine ----------------------- */

/* Attention restricted to positions [pos_begin, min(pos_end, seq_len)) of
 * every cache: d_output gets that range's normalized output and d_lse
 * (f32[n_caches][n_layers][n_q_heads]) its natural-log log-sum-exp of the
 * scaled scores (-inf when the range is empty). */
int eakv_decode_attention_partial(const eakv_cache_t *const *caches,
                                  int n_caches, const float *d_queries,
                                  int n_q_heads, int pos_begin, int pos_end,
                                  float *d_output, float *d_lse, void *stream);

/* Exact merge of n_parts partial results over disjoint position ranges:
 * d_parts f32[n_parts][n_rows][head_dim], d_lse f32[n_parts][n_rows] ->
 * d_output f32[n_rows][head_dim] (and d_lse_out f32[n_rows] if not NULL):
 * out = sum_p exp(lse_p - L) out_p with L = log sum_p exp(lse_p). */
int eakv_lse_combine(int n_parts, int n_rows, int head_dim,
                     const float *d_parts, const float *d_lse,
                     float *d_output, float *d_lse_out, void *stream);

/* ---- inspecting a resident cache ------------------------------------------ */

/* Device validate: the reference's q4_validate (kernels/validate.ea:14-71) as
 * its CLI runs it on every (layer, K/V) block (src/cli.c:39-98), without
 * copying the cache to the host. codes (host, n_layers*2 entries, index
 * layer*2 + kv) receive 0 (ok), 1 (NaN scale), 2 (NaN bias) or 3 (negative
 * scale) for the first failing group in the reference's order ([head]
 * [position][group], positions < seq_len). Returns EAKV_OK or an error. */
int eakv_cache_validate(const eakv_cache_t *cache, int32_t *codes);

/* Dequantize positions [pos_begin, pos_end) of one (layer, K/V) block into
 * f32 [n_kv_heads][pos_end - pos_begin][head_dim], value = nibble * scale +
 * bias with one rounding (reference kernels/dequantize_avx512.ea:10-89, whose
 * range form :52-89 this generalises). The _device form writes device
 * memory on `stream` (NULL: the cache's stream; d_out 16-byte aligned); the
 * other writes host memory and returns when done. EAKV_ERR_INVALID for a bad
 * block, range or alignment. */
int eakv_cache_dequantize_device(const eakv_cache_t *cache, int layer, int kv_idx, int pos_begin,
                                 int pos_end, float *d_out, void *stream);
int eakv_cache_dequantize(const eakv_cache_t *cache, int layer, int kv_idx, int pos_begin,
                          int pos_end, float *out);

/* ---- testing aid ------------------------------------------------------ */

/* Forces every later fused / decode call on this host thread to cut each
 * row into n sequence splits (0 restores the automatic choice), so tests
 * can exercise the split + combine path on small caches. */
int eakv_test_force_splits(int n);

/* The decode planner's split count, for tests of the planner without a GPU
 * (pure host code, no CUDA call): `items` rows of max_pages pages, searched
 * in [lo, hi], per_sm CTAs resident on each of `sms` SMs. The planner itself
 * takes lo and hi from the precision cap and the two-page minimum, and
 * per_sm / sms from the device. */
int eakv_test_choose_splits(long long items, int max_pages, int lo, int hi, int per_sm,
                            int sms);

/* Kernel choice of later fused / decode calls on this host thread, for tests
 * and side-by-side measurements: 1 the CUDA-core kernel even for shapes the
 * tensor-core kernels serve, 2 the mma.sync tensor-core kernel (the automatic
 * choice), 3 the tcgen05 tensor-core kernel (head_dim 128; other shapes keep
 * the automatic choice); 0 restores the automatic choice. */
int eakv_test_force_path(int path);

/* on != 0 makes later decode calls on this host thread merge their sequence
 * splits in a second kernel launch after the decode, instead of in the
 * decode kernel's last CTA of each row group; 0 restores the default. The
 * arithmetic is the same; tests compare the two bit for bit. */
int eakv_test_separate_merge(int on);

/* Failure-detection test: later fused / decode calls on this host thread
 * never request page `page` of each (row, split) work item into the
 * pipeline (page < 0 restores normal operation), and every wait of those
 * kernels gives up after `wait_budget` polls (0: the default budget). The
 * wait for the missing page then runs out: the kernel sets bit 1 of the
 * device status word (eakv_device_status), waits for the copies it did
 * request, and returns without writing its outputs. Nothing faults; the
 * context stays usable. */
int eakv_test_stall(int page, unsigned wait_budget);

#ifdef __cplusplus
}
#endif

#endif /* EAKV_CUDA_H */
