// noalloc.cu - batched decode attention for callers that cannot allocate
// device memory.
//
// Who needs it: a host program whose device memory is owned by a caching
// allocator (a serving framework that reserves the GPU up front and forbids
// raw cudaMalloc), or a latency-critical decode loop that must not hit
// cudaMalloc/cudaFree, which can block or synchronize the device. The
// regular eakv_decode_attention takes the workspace for its split merge from
// scratch memory that the first cache grows with cudaMalloc on demand;
// eakv_decode_attention_noalloc runs the same kernels with the same plan,
// and takes that workspace from fixed arrays in the library's own device
// memory instead, and allocates nothing.
//
// The arrays are kNoAllocScratchBytes (4 MiB) of split records plus
// kNoAllocCounters (65536) split counters (256 KiB) per device: they are
// part of the library's device image, so every GPU that loads the library
// holds them until the process exits. A call whose split records would
// exceed 4 MiB, or whose split rows would need more than 65536 counters, is
// rejected with EAKV_ERR_INVALID before anything is launched (shapes with
// few, long rows need no workspace at all and always fit).
//
// All calls on a device share the arrays. The split records need no
// clearing: every split writes its record before the merge reads it. The
// counters start at zero (static device memory is zero-initialized) and
// every launch returns each counter it uses to zero, so the next call finds
// them cleared. Two calls whose kernels overlap on the GPU (different
// streams, no ordering between them) race on the arrays and give wrong
// results; calls on one stream, or otherwise ordered, are safe.
//
// The first call on a device (made with that device current) looks up the
// arrays' device addresses with cudaGetSymbolAddress; in host code an
// array's name is only a host-side handle, never a usable device pointer.
// That first call should therefore come before any stream capture.
#include <string.h>

#include <atomic>

#include "internal.cuh"

namespace eakv {
namespace {

constexpr size_t kNoAllocScratchBytes = 4u << 20;
constexpr size_t kNoAllocCounters = 65536;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];
static __device__ __align__(256) unsigned g_noalloc_counters[kNoAllocCounters];

// Device addresses of the two arrays on `device` (the current device),
// looked up once per device; false (and the error recorded) when a lookup
// fails.
bool noalloc_arrays(int device, void **scratch, unsigned **counters) {
  static std::atomic<void *> s_ptr[64];
  static std::atomic<void *> c_ptr[64];
  if (device < 0 || device >= 64) {
    set_error(EAKV_ERR_INVALID, "decode_attention_noalloc: device %d out of range", device);
    return false;
  }
  void *s = s_ptr[device].load(std::memory_order_acquire);
  void *c = c_ptr[device].load(std::memory_order_acquire);
  if (!s || !c) {
    cudaError_t e = cudaGetSymbolAddress(&s, g_noalloc_scratch);
    if (e == cudaSuccess) e = cudaGetSymbolAddress(&c, g_noalloc_counters);
    if (e != cudaSuccess) {
      check_cuda(e, "decode_attention_noalloc: cudaGetSymbolAddress");   // clears it
      return false;
    }
    s_ptr[device].store(s, std::memory_order_release);
    c_ptr[device].store(c, std::memory_order_release);
  }
  *scratch = s;
  *counters = (unsigned *)c;
  return true;
}

}  // namespace
}  // namespace eakv

using namespace eakv;

extern "C" int eakv_decode_attention_noalloc(const eakv_cache_t *const *caches, int n_caches,
                                             const float *d_q, int n_q, float *d_out,
                                             void *stream) {
  clear_error();
  int rc = check_batch(caches, n_caches, n_q, "decode_attention_noalloc");
  if (rc) return rc;
  if (!d_q || !d_out) {
    set_error(EAKV_ERR_INVALID, "decode_attention_noalloc: NULL buffer");
    return EAKV_ERR_INVALID;
  }
  const eakv_cache_t *c0 = caches[0];
  DeviceGuard g(c0->device);
  DecodeArgs a = base_args(c0, n_caches, n_q);
  if (!a.status) {
    set_error(EAKV_ERR_INVALID, "decode_attention_noalloc: device status word unavailable");
    return EAKV_ERR_INVALID;
  }
  a.q = d_q;
  a.out = d_out;
  DecodeBatch b;
  fill_batch(b, caches, n_caches);
  const size_t ws = decode_workspace_bytes(a, b);
  const size_t nc = decode_counters(a, b);
  if (ws > kNoAllocScratchBytes || nc > kNoAllocCounters) {
    set_error(EAKV_ERR_INVALID,
              "decode_attention_noalloc: split workspace of %zu bytes and %zu counters exceeds "
              "the fixed %zu-byte, %zu-counter device arrays; use eakv_decode_attention",
              ws, nc, kNoAllocScratchBytes, kNoAllocCounters);
    return EAKV_ERR_INVALID;
  }
  void *w = nullptr;
  if (ws || nc) {
    if (!noalloc_arrays(c0->device, &w, &a.cnt)) return eakv_last_error();
  }
  cudaStream_t s = stream ? (cudaStream_t)stream : c0->stream;
  return decode_launch(a, b, ws ? w : nullptr, ws, s);
}
