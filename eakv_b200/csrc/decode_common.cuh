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
// maxima), in split order. The records are read four splits at a time with
// their loads issued together (the sums stay in split order), so a merge
// waits for about ns / 4 round trips to L2 rather than ns.
template <int HD>
__device__ __forceinline__ void merge_row(const DecodeArgs &a, size_t row, int d) {
  const int ns = a.n_splits;
  const float *pm = a.part_m + row * ns, *pl = a.part_l + row * ns;
  const float *po = a.part_o + row * ns * HD + d;
  float M = -INFINITY;
  int s = 0;
  for (; s + 4 <= ns; s += 4) {
    const float m0 = __ldcg(pm + s), m1 = __ldcg(pm + s + 1), m2 = __ldcg(pm + s + 2),
                m3 = __ldcg(pm + s + 3);
    M = fmaxf(fmaxf(fmaxf(fmaxf(M, m0), m1), m2), m3);
  }
  for (; s < ns; s++) M = fmaxf(M, __ldcg(pm + s));
  float O = 0.0f, L = 0.0f;
  if (M != -INFINITY) {
    s = 0;
    for (; s + 4 <= ns; s += 4) {
      float m[4], o[4], l[4];
#pragma unroll
      for (int k = 0; k < 4; k++) {
        m[k] = __ldcg(pm + s + k);
        o[k] = __ldcg(po + (size_t)(s + k) * HD);
        l[k] = __ldcg(pl + s + k);
      }
#pragma unroll
      for (int k = 0; k < 4; k++) {
        const float f = ex2(m[k] - M);
        O = fmaf(f, o[k], O);
        L = fmaf(f, l[k], L);
      }
    }
    for (; s < ns; s++) {
      const float f = ex2(__ldcg(pm + s) - M);
      O = fmaf(f, __ldcg(po + (size_t)s * HD), O);
      L = fmaf(f, __ldcg(pl + s), L);
    }
  }
  a.out[row * HD + d] = O / L;
  if (a.lse && d == 0) a.lse[row] = L > 0.0f ? (M + log2f(L)) * kLn2 : -INFINITY;
}

constexpr int kMergeSmemSplits = 64;   // split counts the staged merge serves

// The merge of rows row0 .. row0 + n_rows - 1 (n_rows <= NR) by the NT
// threads of one CTA, with the same arithmetic as merge_row. Up to
// kMergeSmemSplits splits the row maxima, the split weights ex2(m_s - M) and
// the sums L are computed once per row into shared memory `ws` (NR *
// (kMergeSmemSplits + 2) floats, free at this point), and each thread then
// issues the output-record loads of all its elements, four splits at a time,
// before it adds them: a few round trips to L2 instead of one per element and
// split. More splits take merge_row per element.
template <int HD, int NR, int NT>
__device__ __forceinline__ void merge_splits(const DecodeArgs &a, size_t row0, int n_rows,
                                             float *ws) {
  const int ns = a.n_splits;
  if (ns > kMergeSmemSplits) {
    for (int idx = threadIdx.x; idx < n_rows * HD; idx += NT) {
      const int h = idx / HD;
      merge_row<HD>(a, row0 + h, idx - h * HD);
    }
    return;
  }
  float *f_s = ws;                                 // [NR][kMergeSmemSplits]: m, then weights
  float *M_s = ws + NR * kMergeSmemSplits;         // [NR]
  float *L_s = M_s + NR;                           // [NR]
  float *l_s = L_s + NR;                           // [NR][kMergeSmemSplits]
  for (int idx = threadIdx.x; idx < n_rows * ns; idx += NT) {
    const int h = idx / ns, sp = idx - h * ns;
    f_s[h * kMergeSmemSplits + sp] = __ldcg(a.part_m + (row0 + h) * ns + sp);
    l_s[h * kMergeSmemSplits + sp] = __ldcg(a.part_l + (row0 + h) * ns + sp);
  }
  __syncthreads();
  if (threadIdx.x < n_rows) {
    const int h = threadIdx.x;
    float M = -INFINITY;
    for (int sp = 0; sp < ns; sp++) M = fmaxf(M, f_s[h * kMergeSmemSplits + sp]);
    float L = 0.0f;
    if (M != -INFINITY) {
      for (int sp = 0; sp < ns; sp++) {
        const float f = ex2(f_s[h * kMergeSmemSplits + sp] - M);
        f_s[h * kMergeSmemSplits + sp] = f;
        L = fmaf(f, l_s[h * kMergeSmemSplits + sp], L);
      }
    }
    M_s[h] = M;
    L_s[h] = L;
  }
  __syncthreads();
  constexpr int EPT = (NR * HD + NT - 1) / NT;   // elements per thread
  float O[EPT];
  int hh[EPT], dd[EPT];
#pragma unroll
  for (int k = 0; k < EPT; k++) {
    const int idx = threadIdx.x + k * NT;
    hh[k] = idx / HD;
    dd[k] = idx - hh[k] * HD;
    O[k] = 0.0f;
  }
  int sp = 0;
  for (; sp + 4 <= ns; sp += 4) {
    float o[EPT][4];
#pragma unroll
    for (int k = 0; k < EPT; k++)
#pragma unroll
      for (int u = 0; u < 4; u++)
        o[k][u] = hh[k] < n_rows
                      ? __ldcg(a.part_o + ((row0 + hh[k]) * ns + sp + u) * HD + dd[k])
                      : 0.0f;
#pragma unroll
    for (int k = 0; k < EPT; k++)
#pragma unroll
      for (int u = 0; u < 4; u++)
        if (hh[k] < n_rows && M_s[hh[k]] != -INFINITY)
          O[k] = fmaf(f_s[hh[k] * kMergeSmemSplits + sp + u], o[k][u], O[k]);
  }
  for (; sp < ns; sp++) {
    float o[EPT];
#pragma unroll
    for (int k = 0; k < EPT; k++)
      o[k] = hh[k] < n_rows ? __ldcg(a.part_o + ((row0 + hh[k]) * ns + sp) * HD + dd[k]) : 0.0f;
#pragma unroll
    for (int k = 0; k < EPT; k++)
      if (hh[k] < n_rows && M_s[hh[k]] != -INFINITY)
        O[k] = fmaf(f_s[hh[k] * kMergeSmemSplits + sp], o[k], O[k]);
  }
#pragma unroll
  for (int k = 0; k < EPT; k++) {
    if (hh[k] >= n_rows) continue;
    const size_t row = row0 + hh[k];
    const float L = L_s[hh[k]], M = M_s[hh[k]];
    a.out[row * HD + dd[k]] = O[k] / L;
    if (a.lse && dd[k] == 0) a.lse[row] = L > 0.0f ? (M + log2f(L)) * kLn2 : -INFINITY;
  }
}

}  // namespace eakv
