// split.cu - the multi-GPU decode of one long context over NCCL.
//
// The reference decodes a sequence in one serial loop over positions on one
// CPU core (kernels/fused_k_score_gqa.ea:29, kernels/fused_attention.ea:
// 38-187). Across GPUs the work is partitioned two ways:
//
// * KV-head shards: each GPU holds some KV heads (with their query heads) of
//   every sequence and layer. Heads are independent; there is no exchange,
//   and a shard calls the ordinary batched decode.
// * Sequence split: each GPU of a group holds a slice of the positions of
//   every sequence. eakv_decode_attention_split runs, on one stream,
//     1. the partial decode of the local slice, writing this rank's record
//        (normalized output, natural-log LSE) of every row into its slot of
//        a packed buffer [rank][rows x head_dim outputs | rows LSEs];
//     2. one in-place ncclAllGather of that buffer over the group's
//        communicator: the records are the only bytes that cross NVLink;
//     3. the exact merge of the group's records on every rank:
//        out = sum_r exp(lse_r - L) out_r, L = log sum_r exp(lse_r).
//   Softmax attention over a set of positions does not depend on their
//   order, so a rank's slice can sit at local positions 0.. of its caches.
//
// NCCL is resolved at run time (dlopen of libnccl.so.2, preferring a copy
// the process already has loaded, e.g. by a framework), so the library
// loads and its other entry points work where NCCL is absent; a
// communicator passed in must come from that same NCCL. Errors come back as
// EAKV_ERR_INVALID with NCCL's message in eakv_last_error_string().
#include <dlfcn.h>
#include <nccl.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <mutex>

#include "internal.cuh"

namespace eakv {
namespace {

struct NcclApi {
  decltype(&ncclGetUniqueId) get_unique_id = nullptr;
  decltype(&ncclCommInitRank) comm_init_rank = nullptr;
  decltype(&ncclCommDestroy) comm_destroy = nullptr;
  decltype(&ncclCommAbort) comm_abort = nullptr;
  decltype(&ncclAllGather) all_gather = nullptr;
  decltype(&ncclGetErrorString) error_string = nullptr;
  decltype(&ncclCommCount) comm_count = nullptr;
  decltype(&ncclCommUserRank) comm_user_rank = nullptr;
  decltype(&ncclCommCuDevice) comm_cu_device = nullptr;
  decltype(&ncclGetVersion) get_version = nullptr;
  bool loaded = false;
  char why[160] = "";
};

template <typename F>
bool bind(void *h, F &fn, const char *name, NcclApi &n) {
  fn = reinterpret_cast<F>(dlsym(h, name));
  if (!fn) snprintf(n.why, sizeof n.why, "NCCL library lacks %s", name);
  return fn != nullptr;
}

// The process's NCCL, loaded once: EAKV_NCCL_LIB if set, else a
// libnccl.so.2 already loaded, else the dynamic linker's search.
const NcclApi *nccl(const char *who) {
  static NcclApi n;
  static std::once_flag once;
  std::call_once(once, [] {
    void *h = nullptr;
    const char *env = getenv("EAKV_NCCL_LIB");
    if (env && *env) h = dlopen(env, RTLD_NOW | RTLD_LOCAL);
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
    if (!h) {
      snprintf(n.why, sizeof n.why, "libnccl.so.2 not found (%s)", dlerror());
      return;
    }
    n.loaded = bind(h, n.get_unique_id, "ncclGetUniqueId", n) &&
               bind(h, n.comm_init_rank, "ncclCommInitRank", n) &&
               bind(h, n.comm_destroy, "ncclCommDestroy", n) &&
               bind(h, n.comm_abort, "ncclCommAbort", n) &&
               bind(h, n.all_gather, "ncclAllGather", n) &&
               bind(h, n.error_string, "ncclGetErrorString", n) &&
               bind(h, n.comm_count, "ncclCommCount", n) &&
               bind(h, n.comm_user_rank, "ncclCommUserRank", n) &&
               bind(h, n.comm_cu_device, "ncclCommCuDevice", n) &&
               bind(h, n.get_version, "ncclGetVersion", n);
  });
  if (!n.loaded) {
    set_error(EAKV_ERR_INVALID, "%s: NCCL unavailable: %s", who, n.why);
    return nullptr;
  }
  return &n;
}

int check_nccl(const NcclApi *n, ncclResult_t r, const char *what) {
  if (r == ncclSuccess) return EAKV_OK;
  set_error(EAKV_ERR_INVALID, "%s: %s", what, n->error_string(r));
  return EAKV_ERR_INVALID;
}

// Floats of one rank's record block: rows outputs of head_dim, then rows
// LSEs, padded to 64 floats so every rank's block starts 256-byte aligned.
size_t record_floats(size_t rows, int head_dim) {
  return (rows * (head_dim + 1) + 63) / 64 * 64;
}

// The partial decode of batch (a, b) on stream s, its records going into this
// rank's slot of `records` (world blocks of rec floats). ws / ws_bytes are the
// decode's split workspace (a.cnt its counters).
int partial_launch(int rank, DecodeArgs a, const DecodeBatch &b, float *records, size_t rec,
                   void *ws, size_t ws_bytes, cudaStream_t s) {
  const size_t rows = (size_t)a.n_caches * a.n_layers * a.n_q_heads;
  float *mine = records + (size_t)rank * rec;
  a.out = mine;
  a.lse = mine + rows * a.head_dim;
  return decode_launch(a, b, ws, ws_bytes, s);
}

// The all-gather of the records of `rows` rows and their merge into d_out, on s.
int gather_merge(const NcclApi *n, ncclComm_t nc, int world, int rank, size_t rows, int hd,
                 float *records, size_t rec, float *d_out, cudaStream_t s) {
  if (world > 1) {
    float *mine = records + (size_t)rank * rec;
    int rc = check_nccl(n, n->all_gather(mine, records, rec, ncclFloat32, nc, s), "ncclAllGather");
    if (rc) return rc;
  }
  return lse_combine_launch(world, (int)rows, hd, records, rec, records + rows * hd, rec, d_out,
                            nullptr, s);
}

// Queues one whole split step of batch (a, b) on stream s: partial decode,
// all-gather, merge into d_out.
int split_launch(const NcclApi *n, ncclComm_t nc, int world, int rank, DecodeArgs a,
                 const DecodeBatch &b, float *records, size_t rec, void *ws, size_t ws_bytes,
                 float *d_out, cudaStream_t s) {
  int rc = partial_launch(rank, a, b, records, rec, ws, ws_bytes, s);
  if (rc) return rc;
  const size_t rows = (size_t)a.n_caches * a.n_layers * a.n_q_heads;
  return gather_merge(n, nc, world, rank, rows, a.head_dim, records, rec, d_out, s);
}

// The communicator's size, this rank, and a check that it lives on `device`.
int comm_info(const NcclApi *n, ncclComm_t nc, int device, int &world, int &rank,
              const char *who) {
  int cdev = -1;
  int rc = check_nccl(n, n->comm_count(nc, &world), "ncclCommCount");
  if (!rc) rc = check_nccl(n, n->comm_user_rank(nc, &rank), "ncclCommUserRank");
  if (!rc) rc = check_nccl(n, n->comm_cu_device(nc, &cdev), "ncclCommCuDevice");
  if (rc) return rc;
  if (cdev != device) {
    set_error(EAKV_ERR_INVALID, "%s: communicator on device %d, caches on device %d", who, cdev,
              device);
    return EAKV_ERR_INVALID;
  }
  return EAKV_OK;
}

}  // namespace
}  // namespace eakv

using namespace eakv;

extern "C" {

int eakv_nccl_version(void) {
  clear_error();
  const NcclApi *n = nccl("nccl_version");
  if (!n) return EAKV_ERR_INVALID;
  int v = 0;
  int rc = check_nccl(n, n->get_version(&v), "nccl_version");
  return rc ? rc : v;
}

int eakv_nccl_unique_id(void *id) {
  clear_error();
  if (!id) {
    set_error(EAKV_ERR_INVALID, "nccl_unique_id: NULL buffer");
    return EAKV_ERR_INVALID;
  }
  const NcclApi *n = nccl("nccl_unique_id");
  if (!n) return EAKV_ERR_INVALID;
  ncclUniqueId u;
  int rc = check_nccl(n, n->get_unique_id(&u), "ncclGetUniqueId");
  if (rc) return rc;
  memcpy(id, &u, sizeof u);
  return EAKV_OK;
}

int eakv_nccl_comm_init(void **comm, int n_ranks, const void *id, int rank, int device) {
  clear_error();
  if (!comm || !id || n_ranks < 1 || rank < 0 || rank >= n_ranks || device < 0) {
    set_error(EAKV_ERR_INVALID, "nccl_comm_init: invalid argument");
    return EAKV_ERR_INVALID;
  }
  const NcclApi *n = nccl("nccl_comm_init");
  if (!n) return EAKV_ERR_INVALID;
  DeviceGuard g(device);
  ncclUniqueId u;
  memcpy(&u, id, sizeof u);
  ncclComm_t c = nullptr;
  int rc = check_nccl(n, n->comm_init_rank(&c, n_ranks, u, rank), "ncclCommInitRank");
  if (rc) return rc;
  *comm = c;
  return EAKV_OK;
}

int eakv_nccl_comm_destroy(void *comm) {
  clear_error();
  if (!comm) return EAKV_OK;
  const NcclApi *n = nccl("nccl_comm_destroy");
  if (!n) return EAKV_ERR_INVALID;
  return check_nccl(n, n->comm_destroy((ncclComm_t)comm), "ncclCommDestroy");
}

int eakv_nccl_comm_abort(void *comm) {
  clear_error();
  if (!comm) return EAKV_OK;
  const NcclApi *n = nccl("nccl_comm_abort");
  if (!n) return EAKV_ERR_INVALID;
  return check_nccl(n, n->comm_abort((ncclComm_t)comm), "ncclCommAbort");
}

int eakv_decode_attention_split(const eakv_cache_t *const *caches, int n_caches,
                                const float *d_q, int n_q, int pos_begin, int pos_end,
                                float *d_out, void *comm, void *stream) {
  clear_error();
  const char *who = "decode_attention_split";
  int rc = check_batch(caches, n_caches, n_q, who);
  if (rc) return rc;
  if (!d_q || !d_out || !comm || pos_begin < 0 || (pos_end >= 0 && pos_end < pos_begin)) {
    set_error(EAKV_ERR_INVALID, "%s: invalid argument", who);
    return EAKV_ERR_INVALID;
  }
  const NcclApi *n = nccl(who);
  if (!n) return EAKV_ERR_INVALID;
  ncclComm_t nc = (ncclComm_t)comm;
  const eakv_cache_t *c0 = caches[0];
  int world = 0, rank = 0;
  rc = comm_info(n, nc, c0->device, world, rank, who);
  if (rc) return rc;
  DeviceGuard g(c0->device);
  cudaStream_t s = stream ? (cudaStream_t)stream : c0->stream;
  DecodeArgs a = base_args(c0, n_caches, n_q);
  if (!a.status) {
    set_error(EAKV_ERR_INVALID, "%s: device status word unavailable", who);
    return EAKV_ERR_INVALID;
  }
  a.q = d_q;
  a.pos_begin = pos_begin;
  a.pos_end = pos_end;
  DecodeBatch b;
  fill_batch(b, caches, n_caches);
  const int hd = c0->head_dim;
  const size_t unit = (size_t)c0->n_layers * n_q;   // rows of one cache
  if (n_caches < 2) {
    const size_t rows = (size_t)n_caches * unit;
    const size_t rec = record_floats(rows, hd);
    // scratch: [records of every rank | decode split workspace]
    const size_t rec_bytes = (size_t)world * rec * sizeof(float);
    const size_t ws = decode_workspace_bytes(a, b);
    void *base = nullptr;
    rc = cache_workspace(c0, decode_counters(a, b), rec_bytes + ws, &a.cnt, &base);
    if (rc) return rc;
    return split_launch(n, nc, world, rank, a, b, (float *)base, rec,
                        ws ? (uint8_t *)base + rec_bytes : nullptr, ws, d_out, s);
  }
  // Two halves of the caches, each keeping the whole batch's split plan: the
  // second half's partial decode runs on a second stream, so its CTAs fill
  // the SMs as the first half's drain, and the first half's all-gather and
  // merge run on the collective stream meanwhile; only the second half's
  // exchange is left after the last decode. Every collective is on the
  // collective stream, in the same order on every rank.
  HostStreams hs;
  rc = host_streams(c0->device, hs);
  if (rc) return rc;
  decode_fix_plan(a, b);
  const int cut[3] = {0, n_caches / 2, n_caches};
  DecodeArgs ca[2];
  DecodeBatch cb[2];
  size_t rec[2], rbytes[2], ws[2], cnt[2];
  for (int k = 0; k < 2; k++) {
    const int cn = cut[k + 1] - cut[k];
    ca[k] = a;
    ca[k].n_caches = cn;
    ca[k].q = d_q + (size_t)cut[k] * unit * hd;
    fill_batch(cb[k], caches + cut[k], cn);
    rec[k] = record_floats((size_t)cn * unit, hd);
    rbytes[k] = ((size_t)world * rec[k] * sizeof(float) + 255) / 256 * 256;
    ws[k] = (decode_workspace_bytes(ca[k], cb[k]) + 255) / 256 * 256;
    cnt[k] = decode_counters(ca[k], cb[k]);
  }
  // scratch: [records 0 | records 1 | workspace 0 | workspace 1], counters 0 then 1
  void *vbase = nullptr;
  unsigned *counters = nullptr;
  rc = cache_workspace(c0, cnt[0] + cnt[1], rbytes[0] + rbytes[1] + ws[0] + ws[1], &counters,
                       &vbase);
  if (rc) return rc;
  uint8_t *base = (uint8_t *)vbase;
  float *records[2] = {(float *)base, (float *)(base + rbytes[0])};
  void *wsp[2] = {ws[0] ? base + rbytes[0] + rbytes[1] : nullptr,
                  ws[1] ? base + rbytes[0] + rbytes[1] + ws[0] : nullptr};
  ca[0].cnt = counters;
  ca[1].cnt = counters + cnt[0];
  cudaEvent_t ev[4] = {};
  int made = 0;
  for (; made < 4; made++) {
    rc = check_cuda(cudaEventCreateWithFlags(&ev[made], cudaEventDisableTiming), who);
    if (rc) break;
  }
  auto step = [&](cudaError_t e) {
    if (!rc) rc = check_cuda(e, who);
  };
  const cudaStream_t dec[2] = {s, hs.alt};
  if (!rc) {
    // both decodes and the exchange start after earlier work on s
    step(cudaEventRecord(ev[0], s));
    step(cudaStreamWaitEvent(hs.alt, ev[0], 0));
    step(cudaStreamWaitEvent(hs.coll, ev[0], 0));
    for (int k = 0; k < 2 && !rc; k++) {
      rc = partial_launch(rank, ca[k], cb[k], records[k], rec[k], wsp[k], ws[k], dec[k]);
      step(cudaEventRecord(ev[1 + k], dec[k]));
    }
    for (int k = 0; k < 2 && !rc; k++) {
      step(cudaStreamWaitEvent(hs.coll, ev[1 + k], 0));
      if (rc) break;
      rc = gather_merge(n, nc, world, rank, (size_t)ca[k].n_caches * unit, hd, records[k], rec[k],
                        d_out + (size_t)cut[k] * unit * hd, hs.coll);
    }
    step(cudaEventRecord(ev[3], hs.coll));
    step(cudaStreamWaitEvent(s, ev[3], 0));   // later work on s sees the merged output
  }
  for (int i = 0; i < made; i++) cudaEventDestroy(ev[i]);
  return rc;
}

int eakv_decode_attention_split_host(const eakv_cache_t *const *caches, int n_caches,
                                     const float *queries, int n_q, float *output, void *comm,
                                     void *stream) {
  clear_error();
  const char *who = "decode_attention_split_host";
  int rc = check_batch(caches, n_caches, n_q, who);
  if (rc) return rc;
  if (!queries || !output || !comm) {
    set_error(EAKV_ERR_INVALID, "%s: invalid argument", who);
    return EAKV_ERR_INVALID;
  }
  const NcclApi *n = nccl(who);
  if (!n) return EAKV_ERR_INVALID;
  ncclComm_t nc = (ncclComm_t)comm;
  const eakv_cache_t *c0 = caches[0];
  int world = 0, rank = 0;
  rc = comm_info(n, nc, c0->device, world, rank, who);
  if (rc) return rc;
  DeviceGuard g(c0->device);
  cudaStream_t s = stream ? (cudaStream_t)stream : c0->stream;
  HostStreams hs;
  rc = host_streams(c0->device, hs);
  if (rc) return rc;
  DecodeArgs a = base_args(c0, n_caches, n_q);
  if (!a.status) {
    set_error(EAKV_ERR_INVALID, "%s: device status word unavailable", who);
    return EAKV_ERR_INVALID;
  }
  DecodeBatch b;
  fill_batch(b, caches, n_caches);
  decode_fix_plan(a, b);   // every chunk keeps the whole batch's split plan
  const int hd = c0->head_dim;
  const size_t unit = (size_t)c0->n_layers * n_q * hd;   // floats of one cache's queries
  const size_t nfl = (size_t)n_caches * unit;
  int start[5];
  const int nch = n_caches > 1 && nfl * sizeof(float) >= kPipelineMinBytes
                      ? host_chunks(n_caches, start) : (start[0] = 0, start[1] = n_caches, 1);
  // Chunk k decodes on stream s or the second compute stream (alternately),
  // then its all-gather and merge run on the collective stream while the
  // next chunk decodes; its copy out waits for its merge. Chunks on one
  // compute stream share that stream's split workspace and counters; every
  // chunk has its own records.
  DecodeArgs ca[4];
  DecodeBatch cb[4];
  size_t rec[4] = {}, rbytes[4] = {}, ws = 0, cnt = 0;
  for (int k = 0; k < nch; k++) {
    const int cn = start[k + 1] - start[k];
    ca[k] = a;
    ca[k].n_caches = cn;
    fill_batch(cb[k], caches + start[k], cn);
    rec[k] = record_floats((size_t)cn * c0->n_layers * n_q, hd);
    rbytes[k] = ((size_t)world * rec[k] * sizeof(float) + 255) / 256 * 256;
    const size_t w = decode_workspace_bytes(ca[k], cb[k]);
    const size_t c = decode_counters(ca[k], cb[k]);
    if (w > ws) ws = w;
    if (c > cnt) cnt = c;
  }
  ws = (ws + 255) / 256 * 256;
  const size_t half = (nfl * sizeof(float) + 255) / 256 * 256;
  size_t rec_total = 0;
  for (int k = 0; k < nch; k++) rec_total += rbytes[k];
  // scratch: [queries | outputs | records of each chunk | workspace of s | of the second stream]
  void *vbase = nullptr;
  unsigned *counters = nullptr;
  rc = cache_workspace(c0, 2 * cnt, 2 * half + rec_total + 2 * ws, &counters, &vbase);
  if (rc) return rc;
  uint8_t *base = (uint8_t *)vbase;
  float *dq = (float *)base, *dout = (float *)(base + half);
  float *records[4];
  {
    uint8_t *r = base + 2 * half;
    for (int k = 0; k < nch; k++) {
      records[k] = (float *)r;
      r += rbytes[k];
    }
  }
  uint8_t *wsp = base + 2 * half + rec_total;

  cudaEvent_t ev[13] = {};
  int made = 0;
  for (; made < 3 * nch + 1; made++) {
    rc = check_cuda(cudaEventCreateWithFlags(&ev[made], cudaEventDisableTiming), who);
    if (rc) break;
  }
  cudaEvent_t ev0 = ev[0], *ev_in = ev + 1, *ev_dec = ev + 1 + nch, *ev_done = ev + 1 + 2 * nch;
  auto step = [&](cudaError_t e) {
    if (!rc) rc = check_cuda(e, who);
  };
  if (!rc) {
    step(cudaEventRecord(ev0, s));
    step(cudaStreamWaitEvent(hs.in, ev0, 0));
    step(cudaStreamWaitEvent(hs.alt, ev0, 0));
    step(cudaStreamWaitEvent(hs.coll, ev0, 0));
    for (int k = 0; k < nch && !rc; k++) {
      const size_t off = start[k] * unit, len = (start[k + 1] - start[k]) * unit;
      step(cudaMemcpyAsync(dq + off, queries + off, len * sizeof(float), cudaMemcpyHostToDevice,
                           hs.in));
      step(cudaEventRecord(ev_in[k], hs.in));
    }
    for (int k = 0; k < nch && !rc; k++) {
      const size_t off = start[k] * unit;
      const cudaStream_t ds = (k & 1) ? hs.alt : s;
      step(cudaStreamWaitEvent(ds, ev_in[k], 0));
      if (rc) break;
      ca[k].q = dq + off;
      ca[k].cnt = counters + (k & 1) * cnt;
      rc = partial_launch(rank, ca[k], cb[k], records[k], rec[k], ws ? wsp + (k & 1) * ws : nullptr,
                          ws, ds);
      step(cudaEventRecord(ev_dec[k], ds));
    }
    for (int k = 0; k < nch && !rc; k++) {
      const size_t off = start[k] * unit;
      step(cudaStreamWaitEvent(hs.coll, ev_dec[k], 0));
      if (rc) break;
      rc = gather_merge(n, nc, world, rank, (size_t)ca[k].n_caches * c0->n_layers * n_q, hd,
                        records[k], rec[k], dout + off, hs.coll);
      step(cudaEventRecord(ev_done[k], hs.coll));
    }
    for (int k = 0; k < nch && !rc; k++) {
      const size_t off = start[k] * unit, len = (start[k + 1] - start[k]) * unit;
      step(cudaStreamWaitEvent(hs.out, ev_done[k], 0));
      step(cudaMemcpyAsync(output + off, dout + off, len * sizeof(float), cudaMemcpyDeviceToHost,
                           hs.out));
    }
  }
  // nothing of this call is left in flight when it returns, error or not
  const cudaStream_t all[5] = {hs.in, s, hs.alt, hs.coll, hs.out};
  for (cudaStream_t t : all) {
    cudaError_t e = cudaStreamSynchronize(t);
    if (!rc && e != cudaSuccess) rc = check_cuda(e, who);
  }
  for (int i = 0; i < made; i++) cudaEventDestroy(ev[i]);
  return rc;
}

}  // extern "C"
