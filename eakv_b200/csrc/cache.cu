// cache.cu - lifecycle, quantize orchestration and info getters of the
// device-resident cache (reference src/cache.c:1-201).
//
// The reference keeps seq_len and the shape on the host and the quantized
// groups in one calloc'd buffer; here the groups live in one cudaMalloc'd
// slab in the page layout of internal.cuh, zero-filled like the reference's
// calloc, and seq_len stays a host field, so checkpoint/restore remain O(1)
// with no data movement (reference src/cache.c:166-176).
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "internal.cuh"

namespace eakv {

static thread_local int t_err_code = EAKV_OK;
static thread_local char t_err_msg[256] = "";

void set_error(int code, const char *fmt, ...) {
  t_err_code = code;
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_err_msg, sizeof t_err_msg, fmt, ap);
  va_end(ap);
}

void clear_error() {
  t_err_code = EAKV_OK;
  t_err_msg[0] = 0;
}

int check_cuda(cudaError_t e, const char *what) {
  if (e == cudaSuccess) return EAKV_OK;
  int code = (e == cudaErrorMemoryAllocation) ? EAKV_ERR_ALLOC : EAKV_ERR_INVALID;
  set_error(code, "%s: %s", what, cudaGetErrorString(e));
  cudaGetLastError();  // clear the non-sticky error
  return code;
}

int cache_workspace(const eakv_cache *c, size_t n_counters, size_t bytes, unsigned **counters,
                    void **data) {
  const size_t have_data = c->d_scratch ? c->scratch_bytes - c->cnt_bytes : 0;
  size_t cb = (n_counters * sizeof(unsigned) + 255) / 256 * 256;
  if (!c->d_scratch || cb > c->cnt_bytes || bytes > have_data) {
    // grow: neither region ever shrinks
    if (cb < c->cnt_bytes) cb = c->cnt_bytes;
    if (cb < 4096) cb = 4096;
    size_t db = bytes > have_data ? bytes : have_data;
    if (db < (1u << 20)) db = 1u << 20;
    if (c->d_scratch) {
      cudaStreamSynchronize(c->stream);
      cudaFree(c->d_scratch);
      c->d_scratch = nullptr;
      c->scratch_bytes = c->cnt_bytes = 0;
    }
    void *p = nullptr;
    int rc = check_cuda(cudaMalloc(&p, cb + db), "scratch allocation");
    if (rc) return rc;
    // the counters start at zero; the decode kernels leave them at zero
    rc = check_cuda(cudaMemsetAsync(p, 0, cb, c->stream), "scratch counters");
    if (!rc) rc = check_cuda(cudaStreamSynchronize(c->stream), "scratch counters");
    if (rc) {
      cudaFree(p);
      return rc;
    }
    c->d_scratch = p;
    c->cnt_bytes = cb;
    c->scratch_bytes = cb + db;
  }
  if (counters) *counters = (unsigned *)c->d_scratch;
  *data = (uint8_t *)c->d_scratch + c->cnt_bytes;
  return EAKV_OK;
}

void *cache_scratch(const eakv_cache *c, size_t bytes) {
  void *d = nullptr;
  return cache_workspace(c, 0, bytes, nullptr, &d) == EAKV_OK ? d : nullptr;
}

}  // namespace eakv

using namespace eakv;

extern "C" {

int eakv_last_error(void) { return t_err_code; }
const char *eakv_last_error_string(void) { return t_err_msg; }

eakv_cache_t *eakv_cache_create(int n_layers, int n_kv_heads, int head_dim,
                                int max_seq_len) {
  clear_error();
  // Same acceptance rule as reference src/cache.c:13-16.
  if (n_layers <= 0 || n_kv_heads <= 0 || head_dim <= 0 || max_seq_len <= 0) {
    set_error(EAKV_ERR_INVALID, "create: non-positive argument");
    return nullptr;
  }
  if (((long long)n_kv_heads * head_dim) % 64 != 0) {
    set_error(EAKV_ERR_INVALID, "create: n_kv_heads*head_dim not a multiple of 64");
    return nullptr;
  }
  eakv_cache *c = (eakv_cache *)calloc(1, sizeof(eakv_cache));
  if (!c) {
    set_error(EAKV_ERR_ALLOC, "create: host allocation");
    return nullptr;
  }
  c->n_layers = n_layers;
  c->n_kv_heads = n_kv_heads;
  c->head_dim = head_dim;
  c->max_seq_len = max_seq_len;
  c->seq_len = 0;
  // A head_dim that is not a multiple of 64 yields gpd = 0 exactly as the
  // reference's integer division does (src/cache.c:68): such a cache holds
  // no groups and its attention calls are rejected.
  c->geom.gpd = head_dim / kGroup;
  c->geom.n_pages = (max_seq_len + kPagePositions - 1) / kPagePositions;
  c->geom.n_heads = n_kv_heads;
  c->geom.n_layers = n_layers;
  c->geom.nib_bytes = (uint32_t)(kPagePositions * c->geom.gpd * 32);
  c->geom.page_bytes = (uint32_t)(kPagePositions * c->geom.gpd * 40);
  c->geom.vexp_offset =
      ((size_t)n_layers * 2 * n_kv_heads * c->geom.n_pages * c->geom.page_bytes + 255) & ~(size_t)255;
  c->buf_bytes = c->geom.gpd ? c->geom.vexp_offset + (size_t)n_layers * n_kv_heads * sizeof(int) : 0;
  if (cudaGetDevice(&c->device) != cudaSuccess) {
    check_cuda(cudaGetLastError(), "create: no CUDA device");
    free(c);
    return nullptr;
  }
  if (check_cuda(cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking),
                 "create: stream") != EAKV_OK) {
    free(c);
    return nullptr;
  }
  c->own_stream = 1;
  if (c->buf_bytes) {
    if (check_cuda(cudaMalloc(&c->d_buf, c->buf_bytes), "create: device allocation") != EAKV_OK) {
      cudaStreamDestroy(c->stream);
      free(c);
      return nullptr;
    }
    if (check_cuda(cudaMemsetAsync(c->d_buf, 0, c->buf_bytes, c->stream), "create: memset") != EAKV_OK ||
        check_cuda(cudaStreamSynchronize(c->stream), "create: memset") != EAKV_OK) {
      cudaFree(c->d_buf);
      cudaStreamDestroy(c->stream);
      free(c);
      return nullptr;
    }
  }
  return c;
}

void eakv_cache_free(eakv_cache_t *c) {
  if (!c) return;
  DeviceGuard g(c->device);
  cudaStreamSynchronize(c->stream);
  if (c->d_buf) cudaFree(c->d_buf);
  if (c->d_scratch) cudaFree(c->d_scratch);
  if (c->own_stream) cudaStreamDestroy(c->stream);
  free(c);
}

// ---------------------------------------------------------------------------
// Quantize orchestration (reference src/cache.c:60-151).

int eakv_cache_load_raw_device(eakv_cache_t *c, const float *d_data, int seq_len) {
  clear_error();
  if (!c || !d_data || seq_len <= 0 || seq_len > c->max_seq_len) {
    set_error(EAKV_ERR_INVALID, "load_raw: invalid argument");
    return EAKV_ERR_INVALID;
  }
  DeviceGuard g(c->device);
  if (c->geom.gpd > 0) {
    int units = c->n_layers * 2 * c->n_kv_heads;
    int rc = check_cuda(launch_quantize(c->geom, c->d_buf, d_data, c->head_dim, 0, units, seq_len, 0,
                                        c->stream), "load_raw: quantize launch");
    if (rc) return rc;
  }
  c->seq_len = seq_len;
  return EAKV_OK;
}

int eakv_cache_load_raw(eakv_cache_t *c, const float *data, int seq_len) {
  clear_error();
  if (!c || !data || seq_len <= 0 || seq_len > c->max_seq_len) {
    set_error(EAKV_ERR_INVALID, "load_raw: invalid argument");
    return EAKV_ERR_INVALID;
  }
  DeviceGuard g(c->device);
  if (c->geom.gpd > 0) {
    // One (layer, kv) slice at a time through device scratch, so the
    // staging never exceeds n_kv_heads * seq_len * head_dim floats.
    size_t slice = (size_t)c->n_kv_heads * seq_len * c->head_dim;
    float *d_stage = (float *)cache_scratch(c, slice * sizeof(float));
    if (!d_stage) return EAKV_ERR_ALLOC;
    for (int lkv = 0; lkv < c->n_layers * 2; lkv++) {
      int rc = check_cuda(cudaMemcpyAsync(d_stage, data + (size_t)lkv * slice,
                                          slice * sizeof(float), cudaMemcpyHostToDevice,
                                          c->stream), "load_raw: copy");
      if (rc) return rc;
      rc = check_cuda(launch_quantize(c->geom, c->d_buf, d_stage, c->head_dim, lkv * c->n_kv_heads,
                                      c->n_kv_heads, seq_len, 0, c->stream),
                      "load_raw: quantize launch");
      if (rc) return rc;
    }
    int rc = check_cuda(cudaStreamSynchronize(c->stream), "load_raw");
    if (rc) return rc;
  }
  c->seq_len = seq_len;
  return EAKV_OK;
}

static int append_check(const eakv_cache_t *c, const void *data, int layer, int kv_idx,
                        int n_tokens) {
  // Same checks and order as reference src/cache.c:104-111.
  if (!c || !data || n_tokens <= 0) return EAKV_ERR_INVALID;
  if (layer < 0 || layer >= c->n_layers) return EAKV_ERR_INVALID;
  if (kv_idx < 0 || kv_idx > 1) return EAKV_ERR_INVALID;
  if ((long long)c->seq_len + n_tokens > c->max_seq_len) return EAKV_ERR_INVALID;
  return EAKV_OK;
}

int eakv_cache_append_device(eakv_cache_t *c, const float *d_data, int layer, int kv_idx,
                             int n_tokens) {
  clear_error();
  if (append_check(c, d_data, layer, kv_idx, n_tokens)) {
    set_error(EAKV_ERR_INVALID, "append: invalid argument");
    return EAKV_ERR_INVALID;
  }
  if (c->geom.gpd == 0) return EAKV_OK;
  DeviceGuard g(c->device);
  return check_cuda(launch_quantize(c->geom, c->d_buf, d_data, c->head_dim,
                                    (layer * 2 + kv_idx) * c->n_kv_heads, c->n_kv_heads,
                                    n_tokens, c->seq_len, c->stream),
                    "append: quantize launch");
}

int eakv_cache_append(eakv_cache_t *c, const float *data, int layer, int kv_idx,
                      int n_tokens) {
  clear_error();
  if (append_check(c, data, layer, kv_idx, n_tokens)) {
    set_error(EAKV_ERR_INVALID, "append: invalid argument");
    return EAKV_ERR_INVALID;
  }
  if (c->geom.gpd == 0) return EAKV_OK;
  DeviceGuard g(c->device);
  size_t n = (size_t)c->n_kv_heads * n_tokens * c->head_dim;
  float *d_stage = (float *)cache_scratch(c, n * sizeof(float));
  if (!d_stage) return EAKV_ERR_ALLOC;
  int rc = check_cuda(cudaMemcpyAsync(d_stage, data, n * sizeof(float),
                                      cudaMemcpyHostToDevice, c->stream), "append: copy");
  if (rc) return rc;
  rc = check_cuda(launch_quantize(c->geom, c->d_buf, d_stage, c->head_dim,
                                  (layer * 2 + kv_idx) * c->n_kv_heads, c->n_kv_heads,
                                  n_tokens, c->seq_len, c->stream),
                  "append: quantize launch");
  if (rc) return rc;
  return check_cuda(cudaStreamSynchronize(c->stream), "append");
}

int eakv_cache_append_step_device(eakv_cache_t *c, const float *d_data, int n_tokens) {
  clear_error();
  if (append_check(c, d_data, 0, 0, n_tokens)) {
    set_error(EAKV_ERR_INVALID, "append_step: invalid argument");
    return EAKV_ERR_INVALID;
  }
  if (c->geom.gpd == 0) return EAKV_OK;
  DeviceGuard g(c->device);
  return check_cuda(launch_quantize(c->geom, c->d_buf, d_data, c->head_dim, 0,
                                    c->n_layers * 2 * c->n_kv_heads, n_tokens, c->seq_len,
                                    c->stream),
                    "append_step: quantize launch");
}

int eakv_cache_advance(eakv_cache_t *c, int n_tokens) {
  clear_error();
  if (!c || n_tokens <= 0) return EAKV_ERR_INVALID;
  if ((long long)c->seq_len + n_tokens > c->max_seq_len) return EAKV_ERR_INVALID;
  c->seq_len += n_tokens;
  return EAKV_OK;
}

void eakv_cache_clear(eakv_cache_t *c) {
  if (c) c->seq_len = 0;
}

int eakv_checkpoint(eakv_cache_t *c) { return c ? c->seq_len : 0; }

int eakv_restore(eakv_cache_t *c, int seq_len) {
  if (!c) return EAKV_ERR_INVALID;
  if (seq_len < 0 || seq_len > c->seq_len) return EAKV_ERR_INVALID;
  c->seq_len = seq_len;
  return EAKV_OK;
}

int eakv_cache_seq_len(const eakv_cache_t *c) { return c ? c->seq_len : 0; }
int eakv_cache_n_layers(const eakv_cache_t *c) { return c ? c->n_layers : 0; }
int eakv_cache_n_heads(const eakv_cache_t *c) { return c ? c->n_kv_heads : 0; }
int eakv_cache_head_dim(const eakv_cache_t *c) { return c ? c->head_dim : 0; }
int eakv_cache_max_seq_len(const eakv_cache_t *c) { return c ? c->max_seq_len : 0; }

float eakv_cache_compression_ratio(const eakv_cache_t *c) {
  // Constant 40 bytes per 64 f32 elements, 0 for an empty cache
  // (reference src/cache.c:198-201).
  if (!c || c->seq_len == 0) return 0.0f;
  return 40.0f / 256.0f;
}

// ---------------------------------------------------------------------------
// Placement.

int eakv_set_device(int device) {
  clear_error();
  return check_cuda(cudaSetDevice(device), "set_device");
}

int eakv_cache_device(const eakv_cache_t *c) { return c ? c->device : -1; }
// The page slab plus the cache's scratch (host staging, split workspace).
size_t eakv_cache_device_bytes(const eakv_cache_t *c) {
  return c ? c->buf_bytes + (c->d_scratch ? c->scratch_bytes : 0) : 0;
}
void *eakv_cache_stream(const eakv_cache_t *c) { return c ? (void *)c->stream : nullptr; }

int eakv_cache_set_stream(eakv_cache_t *c, void *stream) {
  clear_error();
  if (!c) return EAKV_ERR_INVALID;
  DeviceGuard g(c->device);
  if (stream == nullptr) {
    if (!c->own_stream) {
      int rc = check_cuda(cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking),
                          "set_stream");
      if (rc) return rc;
      c->own_stream = 1;
    }
    return EAKV_OK;
  }
  if (c->own_stream) {
    cudaStreamSynchronize(c->stream);
    cudaStreamDestroy(c->stream);
  }
  c->stream = (cudaStream_t)stream;
  c->own_stream = 0;
  return EAKV_OK;
}

int eakv_cache_synchronize(const eakv_cache_t *c) {
  clear_error();
  if (!c) return EAKV_ERR_INVALID;
  DeviceGuard g(c->device);
  return check_cuda(cudaStreamSynchronize(c->stream), "synchronize");
}

}  // extern "C"
