// internal.cuh - device layout of the Q4 cache, the cache object, and the
// launch interfaces shared by the .cu files of libeakv_b200.so.
//
// Device layout ("pages"). The reference keeps, per (layer, K/V), one flat
// block [nibbles][scales][biases] with a head stride of max_seq_len*hd/64
// groups (reference src/cache.c:37-48, src/internal.h:8-26). Here the same
// data is cut into PAGES of 64 consecutive positions of one head of one
// (layer, K/V):
//
//   page = [ nibbles : 64 * gpd * 32 bytes, row-major [position][group][32] ]
//          [ sb      : 64 * gpd float2 (scale, bias), [position][group]    ]
//
// with gpd = head_dim/64 groups per position. A page is 64*gpd*40 bytes
// (2560 B at hd 64, 5120 B at hd 128), every page starts 16-byte aligned,
// and pages are ordered [layer][kv][head][page]. One page is therefore a
// single contiguous bulk copy for the tensor memory accelerator, a
// position's nibble row is contiguous (64 B at hd 128), and the (scale,
// bias) of a group is one 8-byte load. The split-nibble packing of a group
// is unchanged: byte k holds element k (low nibble) and element k+32 (high
// nibble) (reference kernels/quantize_simd.ea:3-7).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>
#include <stddef.h>

#include "../../include/eakv.h"
#include "../../include/eakv_cuda.h"

namespace eakv {

constexpr int kPagePositions = 64;
constexpr int kGroup = 64;

struct PageGeom {
  int gpd;              // groups per position per head (head_dim / 64)
  int n_pages;          // pages per (layer, kv, head)
  int n_heads;          // KV heads
  int n_layers;
  uint32_t nib_bytes;   // nibble bytes of one page
  uint32_t page_bytes;  // nibbles + (scale, bias) pairs of one page
  size_t vexp_offset;   // byte offset of the V-scale exponent table in the slab
};

// Behind the pages each slab keeps int32 vexp[layer][head]: the largest
// biased f32 exponent of any V scale ever written for that (layer, head).
// Every writer (quantize, file load) raises it; nothing lowers it, so after
// restore() or clear() it is still an upper bound. The tensor-core decode
// reads it once per CTA to scale probability x V-scale operands into the
// f16 range.
__host__ __device__ inline int *vexp_table(uint8_t *slab, const PageGeom &g) {
  return reinterpret_cast<int *>(slab + g.vexp_offset);
}
__host__ __device__ inline const int *vexp_table(const uint8_t *slab, const PageGeom &g) {
  return reinterpret_cast<const int *>(slab + g.vexp_offset);
}

// Raise vexp[idx] to e (reads first so that the common case is a plain load).
__device__ inline void vexp_raise(int *vexp, int idx, float scale) {
  const int e = (int)((__float_as_uint(scale) >> 23) & 0xFF);
  if (e > *reinterpret_cast<volatile int *>(vexp + idx)) atomicMax(vexp + idx, e);
}

__host__ __device__ inline size_t page_index(const PageGeom &g, int layer, int kv,
                                             int head, int page) {
  return ((((size_t)layer * 2 + kv) * g.n_heads + head) * g.n_pages + page);
}

}  // namespace eakv

struct eakv_cache {
  int n_layers;
  int n_kv_heads;
  int head_dim;
  int max_seq_len;
  int seq_len;
  eakv::PageGeom geom;
  uint8_t *d_buf;       // device slab, geom-ordered pages
  size_t buf_bytes;
  int device;
  cudaStream_t stream;
  int own_stream;
  // grow-on-demand device scratch for the host-pointer entry points and the
  // decode's split workspace: [cnt_bytes of u32 split counters, kept at
  // zero between calls | data]. scratch_bytes is the whole allocation.
  mutable void *d_scratch;
  mutable size_t scratch_bytes;
  mutable size_t cnt_bytes;
};

namespace eakv {

// Thread-local error record behind eakv_last_error().
void set_error(int code, const char *fmt, ...);
void clear_error();
int check_cuda(cudaError_t e, const char *what);   // EAKV_OK or EAKV_ERR_*

// Makes the cache's device current for the lifetime of the guard.
struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev) {
    cudaGetDevice(&prev);
    if (prev != dev) cudaSetDevice(dev);
  }
  ~DeviceGuard() {
    int cur = -1;
    cudaGetDevice(&cur);
    if (prev >= 0 && cur != prev) cudaSetDevice(prev);
  }
};

// Data space of at least `bytes` in the cache's scratch (nullptr on failure).
// Growing it synchronizes the cache's stream and reallocates.
void *cache_scratch(const eakv_cache *c, size_t bytes);
// The same data space plus at least n_counters u32 counters that are zero
// at every call boundary (the decode kernels return each counter to zero).
// Both pointers come from one allocation, so one call gives both.
int cache_workspace(const eakv_cache *c, size_t n_counters, size_t bytes, unsigned **counters,
                    void **data);

// ---- quantize.cu ----
// Quantizes n_units units of n_tok*head_dim floats each: the n_tok*gpd
// groups of unit u go to unit (unit_base + u) at positions pos0.., where a
// unit is one (layer, kv, head) triple in [layer][kv][head] order.
cudaError_t launch_quantize(const PageGeom &g, uint8_t *d_buf, const float *d_src,
                            int head_dim, int unit_base, int n_units, int n_tok, int pos0,
                            cudaStream_t s);

// ---- attention.cu (two-call API) ----
cudaError_t launch_scores(const PageGeom &g, const uint8_t *d_buf, int layer,
                          const float *d_q, int n_q, int n_kv, int seq_len,
                          float rsqrt_d, float *d_scores, cudaStream_t s);
cudaError_t launch_vsum(const PageGeom &g, const uint8_t *d_buf, int layer,
                        const float *d_w, int n_q, int n_kv, int seq_len,
                        float *d_out, float *d_part, size_t part_floats,
                        unsigned *d_cnt, cudaStream_t s);
size_t vsum_scratch_floats(const PageGeom &g, int n_q, int n_kv, int seq_len);
// zeroed counters the V-sum needs when its sequence spans several blocks
size_t vsum_counters(int n_q, int n_kv, int seq_len);

// ---- decode.cu (fused flash-decoding) ----
constexpr int kMaxBatch = 256;
struct DecodeBatch {
  const uint8_t *base[kMaxBatch];   // device slab of each cache
  int seq_len[kMaxBatch];           // positions to attend per cache
};
struct DecodeArgs {
  PageGeom geom;
  int head_dim;
  int n_caches;
  int n_q_heads;
  int layer0, n_layers;             // layers [layer0, layer0 + n_layers)
  int pos_begin, pos_end;           // attended range clamp (pos_end < 0: up to seq_len)
  const float *q;                   // [cache][layer][q_head][head_dim]
  float *out;                       // same shape as q (normalized output)
  float *lse;                       // optional [cache][layer][q_head] natural-log LSE
  int *status;                      // device status word (bounded waits)
  int force_splits;                 // > 0: use this many splits (tests)
  int force_path;                   // 1: CUDA-core kernel even where tensor cores apply;
                                    // 2: mma.sync tensor-core kernel; 3: tcgen05 kernel
  unsigned wait_budget;             // polls per bounded wait (0: the default budget)
  int test_stall;                   // > 0: page test_stall-1 of every item is never
                                    // requested, so its wait runs out (tests only)
  int fix_split_pages, fix_n_splits;  // > 0: keep this split plan (one chunk of a
                                      // batch that was planned as a whole)
  // split merge: one counter per work item (row group) when rows are
  // split; the last CTA of an item to finish merges its splits and returns
  // the counter to zero
  unsigned *cnt;
  int sep_merge;                    // 1: merge the splits in a second kernel instead (tests)
  // filled by the planner
  int n_splits, split_pages;
  int cta_heads;                    // tensor-core path: query heads per CTA
  float *part_m, *part_l, *part_o;
};
int decode_launch(const DecodeArgs &a, const DecodeBatch &batch, void *workspace,
                  size_t workspace_bytes, cudaStream_t s);
size_t decode_workspace_bytes(const DecodeArgs &a, const DecodeBatch &batch);
// Split counters a decode launch needs (one per work item when rows are
// split, else 0); a.cnt must point at that many zeroed counters.
size_t decode_counters(const DecodeArgs &a, const DecodeBatch &batch);
// Plans `a` over the whole batch and records the split plan in
// a.fix_split_pages / a.fix_n_splits, so that chunks of it launched on their
// own keep the same splits.
void decode_fix_plan(DecodeArgs &a, const DecodeBatch &batch);
// The planner's split count for `items` rows of max_pages pages, searched in
// [lo, hi], per_sm CTAs resident on each of `sms` SMs (host code only).
int choose_splits(long long items, int max_pages, int lo, int hi, int per_sm, int sms);
// Part p of the merge reads rows at parts + p * part_stride and LSEs at
// lse + p * lse_stride (floats).
int lse_combine_launch(int n_parts, int n_rows, int head_dim, const float *parts,
                       size_t part_stride, const float *lse, size_t lse_stride, float *out,
                       float *lse_out, cudaStream_t s);
int *device_status_ptr();   // status word of the current device
// Shared by the decode entry points (api.cu): argument checks of a batch of
// caches, the default launch arguments (after the device guard: they hold
// the current device's status word), and the per-cache table of a batch.
int check_batch(const eakv_cache_t *const *caches, int n, int n_q, const char *who);
DecodeArgs base_args(const eakv_cache_t *c0, int n_caches, int n_q);
void fill_batch(DecodeBatch &b, const eakv_cache_t *const *caches, int n);

// Host-buffer pipelines (api.cu): helper streams per device (queries in,
// outputs out, a second compute stream, a collective stream), created on
// first use; and the cut of
// n units (caches) into up to four chunks whose copies overlap the other
// chunks' work, a one-unit chunk first and last. Below kPipelineMinBytes of
// queries a call is not cut.
struct HostStreams {
  cudaStream_t in = nullptr, out = nullptr, alt = nullptr;
  cudaStream_t coll = nullptr;   // collectives and merges of the multi-GPU split
};
constexpr size_t kPipelineMinBytes = 1u << 18;
int host_streams(int dev, HostStreams &hs);
int host_chunks(int n, int (&start)[5]);
// decode_mma.cu: tensor-core decode, any number of query heads per KV head
int mma_heads_per_cta(int G, int head_dim);   // 0 when the head_dim is not served
int mma_resident(int gh, int head_dim);
int mma_launch(int gh, const DecodeArgs &a, const DecodeBatch &b, int n_blocks, cudaStream_t s);
// decode_umma.cu: tcgen05 decode (head_dim 128, up to 8 query heads per CTA);
// umma_resident is 0 where it is not served
int umma_resident(int gh, int head_dim);
int umma_launch(int gh, const DecodeArgs &a, const DecodeBatch &b, int n_blocks, cudaStream_t s);
extern thread_local int t_force_path;
extern thread_local int t_force_splits;
extern thread_local int t_test_stall;
extern thread_local int t_sep_merge;
extern thread_local unsigned t_wait_budget;

}  // namespace eakv
