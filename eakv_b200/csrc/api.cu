// api.cu - extension entry points of eakv_cuda.h: fused attention (single
// layer and batched decode step), sequence-split partials, the exact
// log-sum-exp combine, and the device status word.
#include <math.h>
#include <string.h>

#include <atomic>
#include <mutex>

#include "internal.cuh"

namespace eakv {

// Sticky status word of the library's kernels (one per device).
__device__ int g_status;

// Split count forced by eakv_test_force_splits() on this host thread.
thread_local int t_force_splits = 0;
// Kernel path forced by eakv_test_force_path() on this host thread.
thread_local int t_force_path = 0;
// Stalled page and wait budget set by eakv_test_stall() on this host thread.
thread_local int t_test_stall = 0;
thread_local unsigned t_wait_budget = 0;
// Separate merge kernel selected by eakv_test_separate_merge() on this thread.
thread_local int t_sep_merge = 0;

int *device_status_ptr() {
  static std::atomic<int *> ptrs[64];
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return nullptr;
  int *p = ptrs[dev].load(std::memory_order_acquire);
  if (!p) {
    void *q = nullptr;
    if (cudaGetSymbolAddress(&q, g_status) != cudaSuccess) {
      cudaGetLastError();
      return nullptr;
    }
    p = (int *)q;
    ptrs[dev].store(p, std::memory_order_release);
  }
  return p;
}

int check_batch(const eakv_cache_t *const *caches, int n, int n_q, const char *who) {
  if (!caches || n <= 0 || n > kMaxBatch) {
    set_error(EAKV_ERR_INVALID, "%s: need 1..%d caches", who, kMaxBatch);
    return EAKV_ERR_INVALID;
  }
  const eakv_cache_t *c0 = caches[0];
  if (!c0) {
    set_error(EAKV_ERR_INVALID, "%s: NULL cache", who);
    return EAKV_ERR_INVALID;
  }
  if (c0->head_dim != 64 && c0->head_dim != 128) {
    set_error(EAKV_ERR_INVALID, "%s: head_dim %d unsupported (64 or 128)", who, c0->head_dim);
    return EAKV_ERR_INVALID;
  }
  if (n_q < c0->n_kv_heads || n_q % c0->n_kv_heads != 0) {
    set_error(EAKV_ERR_INVALID, "%s: n_q_heads %d not a multiple of n_kv_heads %d", who, n_q,
              c0->n_kv_heads);
    return EAKV_ERR_INVALID;
  }
  for (int i = 1; i < n; i++) {
    const eakv_cache_t *c = caches[i];
    if (!c || c->n_layers != c0->n_layers || c->n_kv_heads != c0->n_kv_heads ||
        c->head_dim != c0->head_dim || c->max_seq_len != c0->max_seq_len ||
        c->device != c0->device) {
      set_error(EAKV_ERR_INVALID, "%s: cache %d differs in shape or device", who, i);
      return EAKV_ERR_INVALID;
    }
  }
  return EAKV_OK;
}

// Call after the device guard: the status word is the current device's.
DecodeArgs base_args(const eakv_cache_t *c0, int n_caches, int n_q) {
  DecodeArgs a;
  memset(&a, 0, sizeof a);
  a.geom = c0->geom;
  a.head_dim = c0->head_dim;
  a.n_caches = n_caches;
  a.n_q_heads = n_q;
  a.layer0 = 0;
  a.n_layers = c0->n_layers;
  a.pos_begin = 0;
  a.pos_end = -1;
  a.status = device_status_ptr();
  a.force_splits = t_force_splits;
  a.force_path = t_force_path;
  a.test_stall = t_test_stall;
  a.wait_budget = t_wait_budget;
  a.sep_merge = t_sep_merge;
  return a;
}

void fill_batch(DecodeBatch &b, const eakv_cache_t *const *caches, int n) {
  for (int i = 0; i < n; i++) {
    b.base[i] = caches[i]->d_buf;
    b.seq_len[i] = caches[i]->seq_len;
  }
}

// ---- pipelined host-buffer decode -------------------------------------------


// Helper streams of the host-buffer decode on one device: queries in,
// outputs out, and a second compute stream, so that the next chunk's CTAs
// fill the SMs while the previous chunk's last CTAs drain. Created on first
// use, kept for the life of the process.
static std::mutex g_host_streams_mu;
static HostStreams g_host_streams[64];

int host_streams(int dev, HostStreams &hs) {
  std::lock_guard<std::mutex> lock(g_host_streams_mu);
  if (dev < 0 || dev >= 64) {
    set_error(EAKV_ERR_INVALID, "decode_attention_host: device %d out of range", dev);
    return EAKV_ERR_INVALID;
  }
  HostStreams &h = g_host_streams[dev];
  if (!h.in) {
    cudaStream_t t[4] = {nullptr, nullptr, nullptr, nullptr};
    for (int i = 0; i < 4; i++) {
      int rc = check_cuda(cudaStreamCreateWithFlags(&t[i], cudaStreamNonBlocking),
                          "decode_attention_host: stream");
      if (rc) {
        for (int j = 0; j < i; j++) cudaStreamDestroy(t[j]);
        return rc;
      }
    }
    h.in = t[0];
    h.out = t[1];
    h.alt = t[2];
    h.coll = t[3];
  }
  hs = h;
  return EAKV_OK;
}

// Chunk boundaries over n units: a one-unit chunk first and last, whose
// copies are the only ones not hidden behind a decode, and the rest in two
// halves (n <= 4: one unit per chunk). Returns the number of chunks.
int host_chunks(int n, int (&start)[5]) {
  if (n < 2) {
    start[0] = 0;
    start[1] = n;
    return 1;
  }
  if (n <= 4) {
    for (int i = 0; i <= n; i++) start[i] = i;
    return n;
  }
  const int mid = (n - 1) / 2;   // first half of the n - 2 middle units
  start[0] = 0;
  start[1] = 1;
  start[2] = 1 + mid;
  start[3] = n - 1;
  start[4] = n;
  return 4;
}

}  // namespace eakv

using namespace eakv;

namespace {

// Status word of the current device into a.status; EAKV_ERR_INVALID when its
// address cannot be looked up (the kernels would have nowhere to report).
int attach_status(DecodeArgs &a, const char *who) {
  if (!a.status) {
    set_error(EAKV_ERR_INVALID, "%s: device status word unavailable", who);
    return EAKV_ERR_INVALID;
  }
  return EAKV_OK;
}

// Runs the decode with its split counters and workspace from the first
// cache's scratch, the workspace placed after `reserve` bytes the caller
// already uses there.
int run_decode(const eakv_cache_t *c0, DecodeArgs &a, const DecodeBatch &b, size_t reserve,
               cudaStream_t s, const char *who) {
  int rc = attach_status(a, who);
  if (rc) return rc;
  const size_t ws = decode_workspace_bytes(a, b);
  const size_t nc = decode_counters(a, b);
  void *w = nullptr;
  if (ws || nc) {
    void *base = nullptr;
    rc = cache_workspace(c0, nc, reserve + ws, &a.cnt, &base);
    if (rc) return rc;
    w = (uint8_t *)base + reserve;
  }
  return decode_launch(a, b, ws ? w : nullptr, ws, s);
}

// The host-buffer decode in chunks of caches (or of layers, for a single
// cache): the queries of every chunk are copied in on one stream, each
// chunk's decode waits only for its own queries and alternates between the
// caller's stream and a second one, and each chunk's outputs are copied
// out as soon as its decode ends. Every chunk keeps the split plan of the
// whole batch, so the outputs equal eakv_decode_attention's bit for bit.
int decode_host_pipelined(const eakv_cache_t *const *caches, DecodeArgs a, const DecodeBatch &b,
                          const float *queries, float *output, cudaStream_t s, int units,
                          const int (&start)[5], int nch) {
  const eakv_cache_t *c0 = caches[0];
  const bool by_cache = a.n_caches > 1;
  const size_t n = (size_t)a.n_caches * a.n_layers * a.n_q_heads * a.head_dim;
  const size_t unit_floats = n / units;
  const size_t half = (n * sizeof(float) + 255) / 256 * 256;
  HostStreams hs;
  int rc = host_streams(c0->device, hs);
  if (rc) return rc;
  rc = attach_status(a, "decode_attention_host");
  if (rc) return rc;
  decode_fix_plan(a, b);
  // split counters: one per work item of the whole batch; a chunk's items
  // are a contiguous run of them (items are ordered cache, layer, head, ...)
  const size_t n_cnt = decode_counters(a, b);
  const size_t items_per_unit = n_cnt / units;

  DecodeArgs ca[4];
  DecodeBatch cb[4];
  size_t ws = 0;
  for (int k = 0; k < nch; k++) {
    const int u0 = start[k], cnt = start[k + 1] - start[k];
    ca[k] = a;
    if (by_cache) {
      ca[k].n_caches = cnt;
      fill_batch(cb[k], caches + u0, cnt);
    } else {
      ca[k].layer0 = u0;
      ca[k].n_layers = cnt;
      cb[k] = b;
    }
    const size_t w = decode_workspace_bytes(ca[k], cb[k]);
    if (w > ws) ws = w;
  }
  ws = (ws + 255) / 256 * 256;
  // [queries | outputs | workspace of stream s | workspace of the second stream]
  void *vbase = nullptr;
  unsigned *cnt0 = nullptr;
  rc = cache_workspace(c0, n_cnt, 2 * half + 2 * ws, &cnt0, &vbase);
  if (rc) return rc;
  uint8_t *base = (uint8_t *)vbase;
  for (int k = 0; k < nch; k++) ca[k].cnt = n_cnt ? cnt0 + start[k] * items_per_unit : nullptr;
  float *dq = (float *)base, *dout = (float *)(base + half);

  cudaEvent_t ev[9] = {};
  int made = 0;
  for (; made < 2 * nch + 1; made++) {
    rc = check_cuda(cudaEventCreateWithFlags(&ev[made], cudaEventDisableTiming),
                    "decode_attention_host: event");
    if (rc) break;
  }
  cudaEvent_t ev0 = ev[0], *ev_in = ev + 1, *ev_done = ev + 1 + nch;
  auto step = [&](cudaError_t e) {
    if (!rc) rc = check_cuda(e, "decode_attention_host: pipeline");
  };
  if (!rc) {
    // the copies in wait for earlier work on the caller's stream
    step(cudaEventRecord(ev0, s));
    step(cudaStreamWaitEvent(hs.in, ev0, 0));
    step(cudaStreamWaitEvent(hs.alt, ev0, 0));
    for (int k = 0; k < nch && !rc; k++) {
      const size_t off = start[k] * unit_floats, cnt = (start[k + 1] - start[k]) * unit_floats;
      step(cudaMemcpyAsync(dq + off, queries + off, cnt * sizeof(float), cudaMemcpyHostToDevice,
                           hs.in));
      step(cudaEventRecord(ev_in[k], hs.in));
    }
    // every decode is queued before any copy out, which blocks the host
    // when the output buffer is pageable
    for (int k = 0; k < nch && !rc; k++) {
      cudaStream_t cs = (k & 1) ? hs.alt : s;
      const size_t off = start[k] * unit_floats;
      step(cudaStreamWaitEvent(cs, ev_in[k], 0));
      if (rc) break;
      ca[k].q = dq + off;
      ca[k].out = dout + off;
      rc = decode_launch(ca[k], cb[k], ws ? base + 2 * half + (k & 1) * ws : nullptr, ws, cs);
      step(cudaEventRecord(ev_done[k], cs));
    }
    for (int k = 0; k < nch && !rc; k++) {
      const size_t off = start[k] * unit_floats, cnt = (start[k + 1] - start[k]) * unit_floats;
      step(cudaStreamWaitEvent(hs.out, ev_done[k], 0));
      step(cudaMemcpyAsync(output + off, dout + off, cnt * sizeof(float), cudaMemcpyDeviceToHost,
                           hs.out));
    }
  }
  // nothing of this call is left in flight when it returns, error or not
  const cudaStream_t all[4] = {hs.in, s, hs.alt, hs.out};
  for (cudaStream_t t : all) {
    cudaError_t e = cudaStreamSynchronize(t);
    if (!rc && e != cudaSuccess) rc = check_cuda(e, "decode_attention_host");
  }
  for (int i = 0; i < made; i++) cudaEventDestroy(ev[i]);
  return rc;
}

}  // namespace

extern "C" {

int eakv_device_status(int device, int reset) {
  clear_error();
  DeviceGuard g(device);
  int *p = device_status_ptr();
  if (!p) {
    set_error(EAKV_ERR_INVALID, "device_status: symbol lookup failed");
    return EAKV_ERR_INVALID;
  }
  int v = 0;
  int rc = check_cuda(cudaDeviceSynchronize(), "device_status");
  if (rc) return rc;
  rc = check_cuda(cudaMemcpy(&v, p, sizeof v, cudaMemcpyDeviceToHost), "device_status");
  if (rc) return rc;
  if (reset) {
    int z = 0;
    rc = check_cuda(cudaMemcpy(p, &z, sizeof z, cudaMemcpyHostToDevice), "device_status");
    if (rc) return rc;
  }
  return v;
}

int eakv_attention_fused_device(const eakv_cache_t *c, const float *d_q, int layer, int n_q,
                                int n_kv, float *d_out) {
  clear_error();
  if (!c || !d_q || !d_out || layer < 0 || layer >= c->n_layers || n_kv != c->n_kv_heads) {
    set_error(EAKV_ERR_INVALID, "attention_fused: invalid argument");
    return EAKV_ERR_INVALID;
  }
  const eakv_cache_t *cs[1] = {c};
  int rc = check_batch(cs, 1, n_q, "attention_fused");
  if (rc) return rc;
  DeviceGuard g(c->device);
  DecodeArgs a = base_args(c, 1, n_q);
  a.layer0 = layer;
  a.n_layers = 1;
  a.q = d_q;
  a.out = d_out;
  DecodeBatch b;
  fill_batch(b, cs, 1);
  return run_decode(c, a, b, 0, c->stream, "attention_fused");
}

int eakv_attention_fused(const eakv_cache_t *c, const float *queries, int layer, int n_q,
                         int n_kv, float *output) {
  clear_error();
  if (!c || !queries || !output || layer < 0 || layer >= c->n_layers || n_kv != c->n_kv_heads) {
    set_error(EAKV_ERR_INVALID, "attention_fused: invalid argument");
    return EAKV_ERR_INVALID;
  }
  const eakv_cache_t *cs[1] = {c};
  int rc = check_batch(cs, 1, n_q, "attention_fused");
  if (rc) return rc;
  DeviceGuard g(c->device);
  const size_t n = (size_t)n_q * c->head_dim;
  const size_t reserve = 2 * ((n * sizeof(float) + 255) / 256 * 256);
  DecodeArgs a = base_args(c, 1, n_q);
  a.layer0 = layer;
  a.n_layers = 1;
  DecodeBatch b;
  fill_batch(b, cs, 1);
  rc = attach_status(a, "attention_fused");
  if (rc) return rc;
  size_t ws = decode_workspace_bytes(a, b);
  void *vbase = nullptr;
  rc = cache_workspace(c, decode_counters(a, b), reserve + ws, &a.cnt, &vbase);
  if (rc) return rc;
  uint8_t *base = (uint8_t *)vbase;
  float *d_q = (float *)base;
  float *d_o = (float *)(base + reserve / 2);
  a.q = d_q;
  a.out = d_o;
  rc = check_cuda(cudaMemcpyAsync(d_q, queries, n * sizeof(float), cudaMemcpyHostToDevice,
                                  c->stream), "attention_fused: copy");
  if (rc) return rc;
  rc = decode_launch(a, b, ws ? base + reserve : nullptr, ws, c->stream);
  if (rc) return rc;
  rc = check_cuda(cudaMemcpyAsync(output, d_o, n * sizeof(float), cudaMemcpyDeviceToHost,
                                  c->stream), "attention_fused: copy");
  if (rc) return rc;
  return check_cuda(cudaStreamSynchronize(c->stream), "attention_fused");
}

int eakv_decode_attention(const eakv_cache_t *const *caches, int n_caches, const float *d_q,
                          int n_q, float *d_out, void *stream) {
  clear_error();
  int rc = check_batch(caches, n_caches, n_q, "decode_attention");
  if (rc) return rc;
  if (!d_q || !d_out) {
    set_error(EAKV_ERR_INVALID, "decode_attention: NULL buffer");
    return EAKV_ERR_INVALID;
  }
  const eakv_cache_t *c0 = caches[0];
  DeviceGuard g(c0->device);
  cudaStream_t s = stream ? (cudaStream_t)stream : c0->stream;
  DecodeArgs a = base_args(c0, n_caches, n_q);
  a.q = d_q;
  a.out = d_out;
  DecodeBatch b;
  fill_batch(b, caches, n_caches);
  return run_decode(c0, a, b, 0, s, "decode_attention");
}

int eakv_decode_launches(const eakv_cache_t *const *caches, int n_caches, int n_q) {
  clear_error();
  int rc = check_batch(caches, n_caches, n_q, "decode_launches");
  if (rc) return rc;
  // the split merge runs inside the decode kernel
  return 1;
}

int eakv_decode_splits(const eakv_cache_t *const *caches, int n_caches, int n_q) {
  clear_error();
  int rc = check_batch(caches, n_caches, n_q, "decode_splits");
  if (rc) return rc;
  DeviceGuard g(caches[0]->device);
  DecodeArgs a = base_args(caches[0], n_caches, n_q);
  DecodeBatch b;
  fill_batch(b, caches, n_caches);
  decode_fix_plan(a, b);
  return a.fix_n_splits;
}

int eakv_decode_attention_host(const eakv_cache_t *const *caches, int n_caches,
                               const float *queries, int n_q, float *output, void *stream) {
  clear_error();
  int rc = check_batch(caches, n_caches, n_q, "decode_attention_host");
  if (rc) return rc;
  if (!queries || !output) {
    set_error(EAKV_ERR_INVALID, "decode_attention_host: NULL buffer");
    return EAKV_ERR_INVALID;
  }
  const eakv_cache_t *c0 = caches[0];
  DeviceGuard g(c0->device);
  cudaStream_t s = stream ? (cudaStream_t)stream : c0->stream;
  const size_t n = (size_t)n_caches * c0->n_layers * n_q * c0->head_dim;
  const size_t half = (n * sizeof(float) + 255) / 256 * 256;
  DecodeArgs a = base_args(c0, n_caches, n_q);
  DecodeBatch b;
  fill_batch(b, caches, n_caches);
  // units the batch can be cut into: caches, or the layers of a single cache
  const int units = n_caches > 1 ? n_caches : c0->n_layers;
  int start[5];
  const int nch = n * sizeof(float) >= kPipelineMinBytes ? host_chunks(units, start) : 1;
  if (nch > 1) return decode_host_pipelined(caches, a, b, queries, output, s, units, start, nch);

  rc = attach_status(a, "decode_attention_host");
  if (rc) return rc;
  size_t ws = decode_workspace_bytes(a, b);
  void *vbase = nullptr;
  rc = cache_workspace(c0, decode_counters(a, b), 2 * half + ws, &a.cnt, &vbase);
  if (rc) return rc;
  uint8_t *base = (uint8_t *)vbase;
  a.q = (float *)base;
  a.out = (float *)(base + half);
  rc = check_cuda(cudaMemcpyAsync((void *)a.q, queries, n * sizeof(float),
                                  cudaMemcpyHostToDevice, s), "decode_attention_host: copy");
  if (rc) return rc;
  rc = decode_launch(a, b, ws ? base + 2 * half : nullptr, ws, s);
  if (rc) return rc;
  rc = check_cuda(cudaMemcpyAsync(output, a.out, n * sizeof(float), cudaMemcpyDeviceToHost, s),
                  "decode_attention_host: copy");
  if (rc) return rc;
  return check_cuda(cudaStreamSynchronize(s), "decode_attention_host");
}

int eakv_decode_attention_partial(const eakv_cache_t *const *caches, int n_caches,
                                  const float *d_q, int n_q, int pos_begin, int pos_end,
                                  float *d_out, float *d_lse, void *stream) {
  clear_error();
  int rc = check_batch(caches, n_caches, n_q, "decode_attention_partial");
  if (rc) return rc;
  if (!d_q || !d_out || !d_lse || pos_begin < 0 || (pos_end >= 0 && pos_end < pos_begin)) {
    set_error(EAKV_ERR_INVALID, "decode_attention_partial: invalid argument");
    return EAKV_ERR_INVALID;
  }
  const eakv_cache_t *c0 = caches[0];
  DeviceGuard g(c0->device);
  cudaStream_t s = stream ? (cudaStream_t)stream : c0->stream;
  DecodeArgs a = base_args(c0, n_caches, n_q);
  a.q = d_q;
  a.out = d_out;
  a.lse = d_lse;
  a.pos_begin = pos_begin;
  a.pos_end = pos_end;
  DecodeBatch b;
  fill_batch(b, caches, n_caches);
  return run_decode(c0, a, b, 0, s, "decode_attention_partial");
}

int eakv_lse_combine(int n_parts, int n_rows, int head_dim, const float *d_parts,
                     const float *d_lse, float *d_out, float *d_lse_out, void *stream) {
  clear_error();
  if (n_parts <= 0 || n_rows < 0 || head_dim <= 0 || head_dim > 1024 || !d_parts || !d_lse ||
      !d_out) {
    set_error(EAKV_ERR_INVALID, "lse_combine: invalid argument");
    return EAKV_ERR_INVALID;
  }
  return lse_combine_launch(n_parts, n_rows, head_dim, d_parts, (size_t)n_rows * head_dim, d_lse,
                            (size_t)n_rows, d_out, d_lse_out, (cudaStream_t)stream);
}

}  // extern "C"

extern "C" int eakv_test_choose_splits(long long items, int max_pages, int lo, int hi,
                                       int per_sm, int sms) {
  return eakv::choose_splits(items, max_pages, lo, hi, per_sm, sms);
}

extern "C" int eakv_test_force_path(int path) {
  eakv::t_force_path = (path >= 1 && path <= 3) ? path : 0;
  return EAKV_OK;
}

extern "C" int eakv_test_force_splits(int n) {
  eakv::t_force_splits = n > 0 ? n : 0;
  return EAKV_OK;
}

extern "C" int eakv_test_stall(int page, unsigned wait_budget) {
  eakv::t_test_stall = page >= 0 ? page + 1 : 0;
  eakv::t_wait_budget = wait_budget;
  return EAKV_OK;
}

extern "C" int eakv_test_separate_merge(int on) {
  eakv::t_sep_merge = on ? 1 : 0;
  return EAKV_OK;
}
