/* eakv_llama.h - import of a llama.cpp sequence state into a device cache,
 * served by libeakv_b200.so with the reference's signatures and error codes
 * (reference include/eakv_llama.h:17-41, src/llama_bridge.c:19-288).
 *
 * state_buf is a HOST buffer as returned by llama_state_seq_get_data(): the
 * cell list, then per layer the F16 K rows [cell][n_kv_heads*head_dim], then
 * per layer the F16 V block, rows like K (v_trans == 0) or columns
 * [n_kv_heads*head_dim][cell] (v_trans == 1). The cells are widened to f32,
 * reordered to [head][pos][dim] and quantized on the GPU; the cache equals
 * the reference's bit for bit. */
#ifndef EAKV_LLAMA_H
#define EAKV_LLAMA_H

#include <stddef.h>
#include <stdint.h>

#include "eakv.h"

#ifdef __cplusplus
extern "C" {
#endif

/* New cache of max_seq_len positions holding every cell of the state
 * (reference eakv_llama.h:17-29). EAKV_ERR_INVALID for bad arguments,
 * EAKV_ERR_FORMAT for a malformed or truncated buffer, no cells, more cells
 * than max_seq_len or a layer count that differs, EAKV_ERR_ALLOC when the
 * cache cannot be created. */
int eakv_from_llama_state(const uint8_t *state_buf, size_t state_size, int n_layers,
                          int n_kv_heads, int head_dim, int max_seq_len, eakv_cache_t **out);

/* Appends cells [start_pos, cell_count) of the state to `cache`, whose
 * seq_len must equal start_pos, and advances it (reference
 * eakv_llama.h:31-41). Unlike the reference, n_layers / n_kv_heads /
 * head_dim must equal the cache's (EAKV_ERR_INVALID otherwise). */
int eakv_from_llama_state_append(eakv_cache_t *cache, const uint8_t *state_buf, size_t state_size,
                                 int n_layers, int n_kv_heads, int head_dim, int start_pos);

#ifdef __cplusplus
}
#endif

#endif /* EAKV_LLAMA_H */
