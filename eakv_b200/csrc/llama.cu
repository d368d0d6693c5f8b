// llama.cu - import of a llama.cpp sequence state into the device cache
// (reference src/llama_bridge.c:19-288, include/eakv_llama.h).
//
// The state buffer (llama_state_seq_get_data) is parsed on the host with
// the reference's checks, in its order and with its error codes:
//
//   u32 n_stream, u32 cell_count, per cell {i32 pos, u32 n_seq_id,
//   i32 seq_id[n_seq_id]}, u32 v_trans, u32 n_layer,
//   K per layer: {i32 type, u64 size_row, f16 [cell][n_kv_heads*head_dim]},
//   V per layer: v_trans == 0 as K; v_trans == 1
//                {i32 type, u32 size_el, u32 n_embd_v, f16 [n_embd][cell]}.
//
// Per (layer, K/V) only the cells that are imported cross PCIe (rows for
// [cell][embd] blocks; a pitched copy of the needed columns for the
// transposed V layout). On the GPU one kernel widens f16 -> f32 (exact)
// and reorders the block to the [head][pos][dim] order that
// eakv_cache_append takes, and the cache's quantize kernel writes the
// pages: the nibbles, scales and biases are those of the reference's
// f16 -> f32 -> transpose -> eakv_cache_append sequence, bit for bit.
//
// Like the reference, an append that does not fit (seq_len + new tokens >
// max_seq_len) quantizes nothing and the final advance fails, with the
// call still returning EAKV_OK. Divergences, both where the reference
// would read or write out of bounds: the reference indexes the f16 rows
// with a stride of n_kv_heads*head_dim elements but bounds-checks only
// size_row*cell_count bytes, so here the bytes actually read are checked
// too (EAKV_ERR_FORMAT); and the append form refuses a layer / head /
// head_dim count that differs from the cache's (EAKV_ERR_INVALID).
#include <string.h>

#include <cuda_fp16.h>

#include "internal.cuh"
#include "../../include/eakv_llama.h"

namespace eakv {
namespace {

constexpr int kTile = 32;

// rows [t][embd] (t < n_tok) -> [head][t][dim]
__global__ void rows_to_heads(const __half *__restrict__ src, float *__restrict__ dst, int n_tok,
                              int n_heads, int head_dim) {
  const long long embd = (long long)n_heads * head_dim;
  const long long total = embd * n_tok;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long t = i / embd, e = i - t * embd;
    const int h = (int)(e / head_dim), d = (int)(e - (long long)h * head_dim);
    dst[((long long)h * n_tok + t) * head_dim + d] = __half2float(src[i]);
  }
}

// columns [embd][t] (pitch n_tok) -> [head][t][dim], through a shared tile
// so that both sides are read and written along contiguous runs
__global__ void cols_to_heads(const __half *__restrict__ src, float *__restrict__ dst, int n_tok,
                              int n_heads, int head_dim) {
  __shared__ float tile[kTile][kTile + 1];
  const int embd = n_heads * head_dim;
  const int e0 = blockIdx.y * kTile, t0 = blockIdx.x * kTile;
  for (int r = threadIdx.y; r < kTile; r += blockDim.y) {
    const int e = e0 + r, t = t0 + threadIdx.x;
    if (e < embd && t < n_tok) tile[r][threadIdx.x] = __half2float(src[(long long)e * n_tok + t]);
  }
  __syncthreads();
  for (int r = threadIdx.y; r < kTile; r += blockDim.y) {
    const int t = t0 + r, e = e0 + threadIdx.x;
    if (e < embd && t < n_tok) {
      const int h = e / head_dim, d = e - h * head_dim;
      dst[((long long)h * n_tok + t) * head_dim + d] = tile[threadIdx.x][r];
    }
  }
}

struct Reader {
  const uint8_t *p, *end;
  size_t left() const { return (size_t)(end - p); }
  uint32_t u32() {
    uint32_t v;
    memcpy(&v, p, 4);
    p += 4;
    return v;
  }
  uint64_t u64() {
    uint64_t v;
    memcpy(&v, p, 8);
    p += 8;
    return v;
  }
};

// Imports cells [start, cell_count) of every layer into c at its seq_len
// and advances it; `rd` stands after the cell count (reference
// llama_bridge.c:36-160 and :190-283, which share this body).
int import_state(eakv_cache_t *c, int n_layers, int n_kv_heads, int head_dim, int start,
                 uint32_t cell_count, Reader rd) {
  const int embd = n_kv_heads * head_dim;
  const int n_new = (int)cell_count - start;
  // skip cell metadata (llama_bridge.c:39-46)
  for (uint32_t i = 0; i < cell_count; i++) {
    if (rd.left() < 8) return EAKV_ERR_FORMAT;
    rd.p += 4;
    const uint32_t n_seq = rd.u32();
    if (rd.left() < (size_t)n_seq * 4) return EAKV_ERR_FORMAT;
    rd.p += (size_t)n_seq * 4;
  }
  if (rd.left() < 8) return EAKV_ERR_FORMAT;
  const uint32_t v_trans = rd.u32();
  const uint32_t file_layers = rd.u32();
  if ((int)file_layers != n_layers) return EAKV_ERR_FORMAT;

  DeviceGuard g(c->device);
  const size_t half_bytes = (size_t)embd * n_new * sizeof(__half);
  const size_t half_al = (half_bytes + 255) & ~(size_t)255;
  uint8_t *scratch = (uint8_t *)cache_scratch(c, half_al + (size_t)embd * n_new * sizeof(float));
  if (!scratch) return EAKV_ERR_ALLOC;
  __half *d_half = (__half *)scratch;
  float *d_f32 = (float *)(scratch + half_al);
  const int threads = 256;
  const long long want = ((long long)embd * n_new + threads - 1) / threads;
  const int blocks = (int)(want > 4096 ? 4096 : want);
  const uint64_t need = (uint64_t)cell_count * embd * 2;   // f16 bytes the reader touches

  // one (layer, K/V) block: copy the needed f16 cells, reorder, quantize
  auto import_block = [&](int layer, int kv, bool cols, const uint8_t *data) -> int {
    int rc;
    if (!cols) {
      rc = check_cuda(cudaMemcpyAsync(d_half, data + (size_t)start * embd * 2, half_bytes,
                                      cudaMemcpyHostToDevice, c->stream), "llama import: copy");
      if (rc) return rc;
      rows_to_heads<<<blocks, threads, 0, c->stream>>>(d_half, d_f32, n_new, n_kv_heads,
                                                        head_dim);
    } else {
      rc = check_cuda(cudaMemcpy2DAsync(d_half, (size_t)n_new * 2, data + (size_t)start * 2,
                                        (size_t)cell_count * 2, (size_t)n_new * 2, embd,
                                        cudaMemcpyHostToDevice, c->stream),
                      "llama import: copy");
      if (rc) return rc;
      dim3 grid((n_new + kTile - 1) / kTile, (embd + kTile - 1) / kTile);
      cols_to_heads<<<grid, dim3(kTile, 8), 0, c->stream>>>(d_half, d_f32, n_new, n_kv_heads,
                                                            head_dim);
    }
    rc = check_cuda(cudaGetLastError(), "llama import: reorder");
    if (rc) return rc;
    // eakv_cache_append semantics: an append that does not fit is skipped
    if (c->geom.gpd > 0 && c->seq_len + n_new <= c->max_seq_len) {
      rc = check_cuda(launch_quantize(c->geom, c->d_buf, d_f32, head_dim,
                                      (layer * 2 + kv) * n_kv_heads, n_kv_heads, n_new,
                                      c->seq_len, c->stream),
                      "llama import: quantize");
      if (rc) return rc;
    }
    // the staging buffers are reused by the next block
    return check_cuda(cudaStreamSynchronize(c->stream), "llama import");
  };

  // K layers: {i32 type, u64 size_row, f16 rows} (llama_bridge.c:74-94)
  for (int l = 0; l < n_layers; l++) {
    if (rd.left() < 12) return EAKV_ERR_FORMAT;
    rd.p += 4;
    const uint64_t size_row = rd.u64();
    if (size_row && cell_count > rd.left() / size_row) return EAKV_ERR_FORMAT;
    if (need > rd.left()) return EAKV_ERR_FORMAT;
    const int rc = import_block(l, 0, false, rd.p);
    if (rc) return rc;
    rd.p += size_row * cell_count;
  }
  // V layers (llama_bridge.c:97-146)
  for (int l = 0; l < n_layers; l++) {
    if (rd.left() < 12) return EAKV_ERR_FORMAT;
    rd.p += 4;
    int rc;
    if (v_trans) {
      const uint32_t size_el = rd.u32();
      const uint32_t n_embd_v = rd.u32();
      const uint64_t v_bytes = (uint64_t)n_embd_v * cell_count * size_el;
      if (v_bytes > rd.left() || need > rd.left()) return EAKV_ERR_FORMAT;
      rc = import_block(l, 1, true, rd.p);
      rd.p += v_bytes;
    } else {
      const uint64_t size_row = rd.u64();
      if (size_row && cell_count > rd.left() / size_row) return EAKV_ERR_FORMAT;
      if (need > rd.left()) return EAKV_ERR_FORMAT;
      rc = import_block(l, 1, false, rd.p);
      rd.p += size_row * cell_count;
    }
    if (rc) return rc;
  }
  eakv_cache_advance(c, n_new);   // fails (and is ignored) when the appends did not fit
  return EAKV_OK;
}

}  // namespace
}  // namespace eakv

using namespace eakv;

extern "C" {

int eakv_from_llama_state(const uint8_t *state_buf, size_t state_size, int n_layers,
                          int n_kv_heads, int head_dim, int max_seq_len, eakv_cache_t **out) {
  clear_error();
  if (!state_buf || !out || state_size < 8) return EAKV_ERR_INVALID;
  if (n_layers <= 0 || n_kv_heads <= 0 || head_dim <= 0 || max_seq_len <= 0)
    return EAKV_ERR_INVALID;
  Reader rd{state_buf, state_buf + state_size};
  rd.u32();   // n_stream
  const uint32_t cell_count = rd.u32();
  if (cell_count == 0 || cell_count > (uint32_t)max_seq_len) return EAKV_ERR_FORMAT;
  eakv_cache_t *c = eakv_cache_create(n_layers, n_kv_heads, head_dim, max_seq_len);
  if (!c) return EAKV_ERR_ALLOC;
  const int rc = import_state(c, n_layers, n_kv_heads, head_dim, 0, cell_count, rd);
  if (rc != EAKV_OK) {
    eakv_cache_free(c);
    return rc;
  }
  *out = c;
  return EAKV_OK;
}

int eakv_from_llama_state_append(eakv_cache_t *cache, const uint8_t *state_buf,
                                 size_t state_size, int n_layers, int n_kv_heads, int head_dim,
                                 int start_pos) {
  clear_error();
  if (!cache || !state_buf || state_size < 8) return EAKV_ERR_INVALID;
  if (start_pos < 0 || start_pos != cache->seq_len) return EAKV_ERR_INVALID;
  if (n_layers != cache->n_layers || n_kv_heads != cache->n_kv_heads ||
      head_dim != cache->head_dim) {
    set_error(EAKV_ERR_INVALID, "from_llama_state_append: shape differs from the cache");
    return EAKV_ERR_INVALID;
  }
  Reader rd{state_buf, state_buf + state_size};
  rd.u32();   // n_stream
  const uint32_t cell_count = rd.u32();
  if ((int)cell_count <= start_pos) return EAKV_OK;   // nothing new (reference's signed test)
  return import_state(cache, n_layers, n_kv_heads, head_dim, start_pos, cell_count, rd);
}

}  // extern "C"
