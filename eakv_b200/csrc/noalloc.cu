// noalloc.cu - batched decode attention for callers that cannot allocate
// device memory.
//
// Who needs it: a host program whose device memory is owned by a caching
// allocator (a serving framework that reserves the GPU up front and forbids
// raw cudaMalloc), or a latency-critical decode loop that must not hit
// cudaMalloc/cudaFree, which can block or synchronize the device. The
// regular eakv_decode_attention takes the workspace for its split merge from
// scratch memory that the first cache grows with cudaMalloc on demand;
// eakv_decode_attention_noalloc runs the same kernels with that workspace
// taken from a fixed array in the library's own device memory instead, and
// allocates nothing.
//
// The array is kNoAllocScratchBytes (4 MiB) per device: it is part of the
// library's device image, so every GPU that loads the library holds it until
// the process exits. A call whose split-merge workspace would exceed it is
// rejected with EAKV_ERR_INVALID before anything is launched (shapes with
// few, long rows need no workspace at all and always fit).
//
// All calls on a device share the one array. Nothing in it has to start at
// zero: every split writes its partial record before the merge kernel reads
// it. Two calls whose kernels overlap on the GPU (different streams, no
// ordering between them) race on the array and give wrong results; calls on
// one stream, or otherwise ordered, are safe.
//
// The first call on a device (made with that device current) looks up the
// array's device address with cudaGetSymbolAddress; in host code the array's
// name is only a host-side handle, never a usable device pointer. That first
// call should therefore come before any stream capture.
#include <string.h>

#include "internal.cuh"

namespace eakv {
namespace {

constexpr size_t kNoAllocScratchBytes = 4u << 20;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// Device address of g_noalloc_scratch on the current device, looked up once
// per device.
void *noalloc_scratch_ptr(int device) {
  static void *ptrs[64] = {nullptr};
  if (device < 0 || device >= 64) {
    set_error(EAKV_ERR_INVALID, "decode_attention_noalloc: device %d out of range", device);
    return nullptr;
  }
  if (!ptrs[device]) {
    void *p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) {
      check_cuda(e, "decode_attention_noalloc: cudaGetSymbolAddress");
      return nullptr;
    }
    ptrs[device] = p;
  }
  return ptrs[device];
}

}  // namespace
}  // namespace eakv

using namespace eakv;

extern "C" int eakv_decode_attention_noalloc(const eakv_cache_t *const *caches, int n_caches,
                                             const float *d_q, int n_q, float *d_out,
                                             void *stream) {
  clear_error();
  if (!caches || n_caches <= 0 || n_caches > kMaxBatch || !caches[0] || !d_q || !d_out) {
    set_error(EAKV_ERR_INVALID, "decode_attention_noalloc: invalid argument");
    return EAKV_ERR_INVALID;
  }
  const eakv_cache_t *c0 = caches[0];
  if (c0->head_dim != 64 && c0->head_dim != 128) {
    set_error(EAKV_ERR_INVALID, "decode_attention_noalloc: head_dim %d unsupported", c0->head_dim);
    return EAKV_ERR_INVALID;
  }
  if (n_q < c0->n_kv_heads || n_q % c0->n_kv_heads != 0) {
    set_error(EAKV_ERR_INVALID, "decode_attention_noalloc: n_q_heads %d not a multiple of %d",
              n_q, c0->n_kv_heads);
    return EAKV_ERR_INVALID;
  }
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
  a.q = d_q;
  a.out = d_out;
  a.force_splits = t_force_splits;
  a.force_path = t_force_path;
  DecodeBatch b;
  for (int i = 0; i < n_caches; i++) {
    const eakv_cache_t *c = caches[i];
    if (!c || c->n_layers != c0->n_layers || c->n_kv_heads != c0->n_kv_heads ||
        c->head_dim != c0->head_dim || c->max_seq_len != c0->max_seq_len ||
        c->device != c0->device) {
      set_error(EAKV_ERR_INVALID, "decode_attention_noalloc: cache %d differs in shape or device",
                i);
      return EAKV_ERR_INVALID;
    }
    b.base[i] = c->d_buf;
    b.seq_len[i] = c->seq_len;
  }
  DeviceGuard g(c0->device);
  a.status = device_status_ptr();
  const size_t ws = decode_workspace_bytes(a, b);
  if (ws > kNoAllocScratchBytes) {
    set_error(EAKV_ERR_INVALID,
              "decode_attention_noalloc: split-merge workspace of %zu bytes exceeds the fixed "
              "%zu-byte device array; use eakv_decode_attention",
              ws, kNoAllocScratchBytes);
    return EAKV_ERR_INVALID;
  }
  void *w = nullptr;
  if (ws) {
    w = noalloc_scratch_ptr(c0->device);
    if (!w) return eakv_last_error() ? eakv_last_error() : EAKV_ERR_INVALID;
  }
  cudaStream_t s = stream ? (cudaStream_t)stream : c0->stream;
  return decode_launch(a, b, w, ws, s);
}
