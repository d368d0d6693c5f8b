// decode_common.cuh - pieces shared by the fused decode kernels: the work
// item decomposition (cache, layer, KV head, query-head group, split) and
// small math helpers.
#pragma once
#include "internal.cuh"
#include "pipeline.cuh"

namespace eakv {

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

struct Item {
  int b, layer, lrow, h, hg, split;
  int r0, r1;       // attended positions [r0, r1)
  int pg0, npages;  // pages of this split
};

__device__ __forceinline__ Item decode_item(const DecodeArgs &a, const DecodeBatch &batch, int nhg) {
  Item it;
  int bid = blockIdx.x;
  it.split = bid % a.n_splits; bid /= a.n_splits;
  it.hg = bid % nhg; bid /= nhg;
  it.h = bid % a.geom.n_heads; bid /= a.geom.n_heads;
  it.lrow = bid % a.n_layers;
  it.b = bid / a.n_layers;
  it.layer = a.layer0 + it.lrow;
  const int seq = batch.seq_len[it.b];
  it.r0 = a.pos_begin > 0 ? a.pos_begin : 0;
  it.r1 = a.pos_end < 0 ? seq : min(seq, a.pos_end);
  int P0 = it.r0 / kPagePositions;
  int P1 = it.r1 > it.r0 ? (it.r1 + kPagePositions - 1) / kPagePositions : P0;
  it.pg0 = P0 + it.split * a.split_pages;
  int pg1 = min(P1, it.pg0 + a.split_pages);
  it.npages = pg1 > it.pg0 ? pg1 - it.pg0 : 0;
  return it;
}

// Self-checks of a CTA's launch arguments and work item. A CTA that fails
// one records kStatusBadIndex in the device status word and returns before
// it touches any memory: no split plan (division by zero in decode_item),
// or an item that would address outside its cache's slab, the query rows
// or the output rows.
// Records `bit` in the device status word (no-op when the launch has none).
__device__ __forceinline__ void report(const DecodeArgs &a, int bit) {
  if (a.status) atomicOr(a.status, bit);
}

__device__ __forceinline__ bool launch_ok(const DecodeArgs &a) {
  const bool ok = a.n_splits >= 1 && a.split_pages >= 1 && a.n_layers >= 1 && a.n_caches >= 1 &&
                  a.geom.n_heads >= 1 && a.n_q_heads >= a.geom.n_heads;
  if (!ok && threadIdx.x == 0) report(a, kStatusBadIndex);
  return ok;
}

__device__ __forceinline__ bool item_ok(const DecodeArgs &a, const Item &it, int q_head0,
                                        int cta_heads) {
  const bool ok = it.b >= 0 && it.b < a.n_caches && it.b < kMaxBatch && it.layer >= 0 &&
                  it.layer < a.geom.n_layers && it.h >= 0 && it.h < a.geom.n_heads &&
                  it.pg0 >= 0 && it.npages >= 0 && it.pg0 + it.npages <= a.geom.n_pages &&
                  q_head0 >= 0 && q_head0 + cta_heads <= a.n_q_heads && it.split < a.n_splits;
  if (!ok && threadIdx.x == 0) report(a, kStatusBadIndex);
  return ok;
}

// ---- split merge inside the decode launch ---------------------------------
//
// When rows are cut into n_splits splits, every CTA of a work item writes its
// partial record (unnormalized output, max, sum) to the workspace and then
// arrives on the item's counter. The last of the n_splits CTAs to arrive
// merges the item's records; no CTA ever waits for another. The counter
// counts with atomicInc wrapping at n_splits - 1, so the last arrival also
// returns it to zero for the next launch: every CTA of a launch arrives
// exactly once (CTAs that fail also arrive before they return).
//
// Called by every thread of the CTA (it synchronizes the CTA). The fence
// before the arrival publishes this CTA's records device-wide; the fence
// after it, in the last CTA, orders the reads of the other CTAs' records
// after their arrivals, and those reads bypass L1 (ld.global.cg), which is
// not coherent across SMs.
__device__ __forceinline__ bool arrive_last(const DecodeArgs &a) {
  __shared__ int s_last;
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned n = (unsigned)a.n_splits;
    const unsigned old = atomicInc(a.cnt + blockIdx.x / n, n - 1);
    s_last = old == n - 1;
  }
  __syncthreads();
  const bool last = s_last != 0;
  if (last) __threadfence();
  return last;
}

// Exact log-sum-exp merge of element d of row `row` over its splits (base-2
// maxima), in split order.
template <int HD>
__device__ __forceinline__ void merge_row(const DecodeArgs &a, size_t row, int d) {
  const int ns = a.n_splits;
  float M = -INFINITY;
  for (int s = 0; s < ns; s++) M = fmaxf(M, __ldcg(a.part_m + row * ns + s));
  float O = 0.0f, L = 0.0f;
  if (M != -INFINITY) {
    for (int s = 0; s < ns; s++) {
      const float f = ex2(__ldcg(a.part_m + row * ns + s) - M);
      O = fmaf(f, __ldcg(a.part_o + (row * ns + s) * HD + d), O);
      L = fmaf(f, __ldcg(a.part_l + row * ns + s), L);
    }
  }
  a.out[row * HD + d] = O / L;
  if (a.lse && d == 0) a.lse[row] = L > 0.0f ? (M + log2f(L)) * kLn2 : -INFINITY;
}

// The merge of rows row0 .. row0 + n_rows - 1 by the threads of one CTA.
template <int HD>
__device__ __forceinline__ void merge_splits(const DecodeArgs &a, size_t row0, int n_rows) {
  for (int idx = threadIdx.x; idx < n_rows * HD; idx += blockDim.x) {
    const int h = idx / HD;
    merge_row<HD>(a, row0 + h, idx - h * HD);
  }
}

}  // namespace eakv
