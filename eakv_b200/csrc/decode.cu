// decode.cu - fused softmax attention over the Q4 cache (flash-decoding).
//
// Replaces the reference's two-pass fused kernel (kernels/fused_attention.ea:
// 10-373, MHA head_dim 128 only, never called by the host) and the caller-side
// composition scores -> softmax -> V-sum (src/attention.c), for any GQA ratio
// and head_dim 64/128, over many caches and all layers in one launch.
//
// Work item = (cache, layer, KV head, query-head group, split). A split is a
// run of whole pages of one KV head; one CTA streams its K and V pages
// through a ring of shared-memory stages filled by 1-D bulk copies
// (cp.async.bulk, one per page) and consumes them with an online
// (running-max) softmax. Each page is read from HBM exactly once and every
// query head of the KV head is served from it (the GQA loop flip). Splits of
// the same row are merged by an exact log-sum-exp combine inside the same
// launch: the last CTA of a row group to finish merges the group's splits
// (decode_common.cuh), so a decode is always one kernel launch.
//
// Arithmetic (CUDA cores, packed f32x2 FMA):
//   score_h(t) = s(t) * sum_i q'_h[i] n_i(t) + b(t) * sum_i q'_h[i]
//   O_h       += (p_h(t) s(t)) n(t) + p_h(t) b(t)
// per 64-element group, with q' = q / sqrt(d) * log2(e) so the softmax runs
// in base 2. This factoring removes the per-element dequantize FMA the
// reference performs; the result differs from the reference only by
// rounding, well inside the 1e-4 parity tolerance.
#include <math.h>
#include <stdio.h>

#include <atomic>

#include <vector>

#include "internal.cuh"
#include "pipeline.cuh"
#include "decode_common.cuh"

namespace eakv {
namespace {


template <int HD, int GC>
struct Cfg {
  static constexpr int DPL = GC <= 2 ? 32 : (GC == 4 ? 16 : 8);   // dims per lane
  static constexpr int BPL = DPL / 2;                              // nibble bytes per lane
  static constexpr int LPP = HD / DPL;                             // lanes per position
  static constexpr int PPW = 32 / LPP;                             // positions per warp step
  static constexpr int NW = PPW <= 8 ? 8 : 4;                      // warps per CTA
  static constexpr int THREADS = NW * 32;
  static constexpr int POS_PER_WARP = kPagePositions / NW;         // per page
  static constexpr int ITERS = POS_PER_WARP / PPW;
  static constexpr int ITB = ITERS < 16 / GC ? ITERS : 16 / GC;    // softmax block
  static constexpr int NBLK = ITERS / ITB;
  static constexpr int GPD = HD / 64;
  static constexpr int NIB = kPagePositions * GPD * 32;
  static constexpr int PB = kPagePositions * GPD * 40;             // page bytes
  static constexpr int NSTAGE = HD == 128 ? 4 : 8;
  static constexpr int STAGE_BYTES = 2 * PB;
  static constexpr int MERGE_BYTES = NW * GC * (HD + 2) * 4;
  static constexpr int RING = NSTAGE * STAGE_BYTES;
  static constexpr int SMEM = (RING > MERGE_BYTES ? RING : MERGE_BYTES) + 2 * NSTAGE * 8;
  static_assert(ITERS % ITB == 0, "block must divide the page");
  static_assert(32 % BPL == 0, "a lane's bytes stay within one group");
};


// 8 nibbles of a 32-bit word -> floats: low nibbles of bytes 0..3 and high
// nibbles of bytes 0..3, exact. Each byte is placed in the mantissa of 2^23
// (0x4B0000xx) and 2^23 is subtracted.
__device__ __forceinline__ void nib8(uint32_t w, float2 &l01, float2 &l23, float2 &h01,
                                     float2 &h23) {
  const uint32_t lo = w & 0x0F0F0F0Fu;
  const uint32_t hi = (w >> 4) & 0x0F0F0F0Fu;
  const float2 off = make_float2(-8388608.0f, -8388608.0f);
  l01 = __fadd2_rn(make_float2(__uint_as_float(__byte_perm(lo, 0x4B000000u, 0x7440)),
                               __uint_as_float(__byte_perm(lo, 0x4B000000u, 0x7441))), off);
  l23 = __fadd2_rn(make_float2(__uint_as_float(__byte_perm(lo, 0x4B000000u, 0x7442)),
                               __uint_as_float(__byte_perm(lo, 0x4B000000u, 0x7443))), off);
  h01 = __fadd2_rn(make_float2(__uint_as_float(__byte_perm(hi, 0x4B000000u, 0x7440)),
                               __uint_as_float(__byte_perm(hi, 0x4B000000u, 0x7441))), off);
  h23 = __fadd2_rn(make_float2(__uint_as_float(__byte_perm(hi, 0x4B000000u, 0x7442)),
                               __uint_as_float(__byte_perm(hi, 0x4B000000u, 0x7443))), off);
}

template <int BPL>
__device__ __forceinline__ void load_words(const uint8_t *p, uint32_t (&w)[BPL / 4]) {
  if constexpr (BPL == 16) {
    uint4 v = *reinterpret_cast<const uint4 *>(p);
    w[0] = v.x; w[1] = v.y; w[2] = v.z; w[3] = v.w;
  } else if constexpr (BPL == 8) {
    uint2 v = *reinterpret_cast<const uint2 *>(p);
    w[0] = v.x; w[1] = v.y;
  } else {
    w[0] = *reinterpret_cast<const uint32_t *>(p);
  }
}

template <int BPL>
__device__ __forceinline__ void convert(const uint32_t (&w)[BPL / 4], float2 (&nl)[BPL / 2],
                                        float2 (&nh)[BPL / 2]) {
#pragma unroll
  for (int m = 0; m < BPL / 4; m++) nib8(w[m], nl[2 * m], nl[2 * m + 1], nh[2 * m], nh[2 * m + 1]);
}

template <int HD, int GC>
__global__ void __launch_bounds__(Cfg<HD, GC>::THREADS, 1)
decode_simt_kernel(const __grid_constant__ DecodeArgs a, const __grid_constant__ DecodeBatch batch) {
  using C = Cfg<HD, GC>;
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + (C::SMEM - 2 * C::NSTAGE * 8));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = a.n_q_heads / a.geom.n_heads;
  const int nhg = G / GC;
  if (!launch_ok(a) || G % GC != 0) return;
  const Item it = decode_item(a, batch, nhg);
  if (!item_ok(a, it, it.h * G + it.hg * GC, GC)) {
    if (a.n_splits > 1 && !a.sep_merge) arrive_last(a);   // keeps the item's split counter in step
    return;
  }
  const size_t kv_stride = (size_t)a.geom.n_heads * a.geom.n_pages;   // pages from K to V
  const uint8_t *kpages =
      batch.base[it.b] + page_index(a.geom, it.layer, 0, it.h, 0) * C::PB;
  const uint8_t *vpages = kpages + kv_stride * C::PB;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::NSTAGE; s++) {
      mbar_init(smem_u32(&bars[s]), 1);                               // stage filled
      reinterpret_cast<int *>(&bars[C::NSTAGE])[s] = 0;               // release count
      reinterpret_cast<int *>(&bars[C::NSTAGE])[C::NSTAGE + s] = -1;  // last page requested
    }
    fence_mbar_init();
  }
  __syncthreads();

  // Thread 0 fills the first NSTAGE stages; afterwards the last warp to
  // release a stage refills it (no thread ever waits for a stage to drain).
  int *last_req = reinterpret_cast<int *>(&bars[C::NSTAGE]) + C::NSTAGE;
  auto issue = [&](int i) {
    if (i == a.test_stall - 1) return;   // test hook: this stage's wait runs out
    const int st = i % C::NSTAGE;
    const uint32_t full = smem_u32(&bars[st]);
    mbar_arrive_expect_tx(full, 2 * C::PB);
    const uint32_t dst = smem_u32(smem + st * C::STAGE_BYTES);
    bulk_g2s(dst, kpages + (size_t)(it.pg0 + i) * C::PB, C::PB, full);
    bulk_g2s(dst + C::PB, vpages + (size_t)(it.pg0 + i) * C::PB, C::PB, full);
    publish_requested(&last_req[st], i);
  };
  if (threadIdx.x == 0)
    for (int i = 0; i < it.npages && i < C::NSTAGE; i++) issue(i);

  // ---------------- consumers --------------------------------------------
  const int pg = lane / C::LPP;          // position slot within the warp step
  const int j = lane % C::LPP;           // lane within the position
  const int byte0 = j * C::BPL;          // first nibble byte of this lane in a row
  const int grp = byte0 / 32;
  const int k0 = byte0 % 32;
  const int qh0 = it.h * G + it.hg * GC;
  const float qscale = rsqrtf((float)HD) * kLog2e;

  float2 ql[GC][C::BPL / 2], qhv[GC][C::BPL / 2];
  float qsum[GC];
  {
    const float *qb = a.q + ((size_t)(it.b * a.n_layers + it.lrow) * a.n_q_heads + qh0) * HD;
#pragma unroll
    for (int h = 0; h < GC; h++) {
      float s = 0.0f;
#pragma unroll
      for (int p = 0; p < C::BPL / 2; p++) {
        const int dl = 64 * grp + k0 + 2 * p;
        ql[h][p] = make_float2(qb[h * HD + dl] * qscale, qb[h * HD + dl + 1] * qscale);
        qhv[h][p] = make_float2(qb[h * HD + dl + 32] * qscale, qb[h * HD + dl + 33] * qscale);
        s += ql[h][p].x + ql[h][p].y + qhv[h][p].x + qhv[h][p].y;
      }
      qsum[h] = s;
    }
  }

  float m[GC], l[GC], pb[GC];
  float2 ol[GC][C::BPL / 2], oh[GC][C::BPL / 2];
#pragma unroll
  for (int h = 0; h < GC; h++) {
    m[h] = -INFINITY;
    l[h] = 0.0f;
    pb[h] = 0.0f;
#pragma unroll
    for (int p = 0; p < C::BPL / 2; p++) {
      ol[h][p] = make_float2(0.f, 0.f);
      oh[h][p] = make_float2(0.f, 0.f);
    }
  }

  bool ok = true;
  for (int i = 0; i < it.npages; i++) {
    const int st = i % C::NSTAGE;
    if (!ok || !wait_requested(&last_req[st], i, a.wait_budget) ||
        !mbar_wait(smem_u32(&bars[st]), (i / C::NSTAGE) & 1, a.wait_budget)) {
      report(a, kStatusWaitTimeout);
      ok = false;
      break;
    }
    const uint8_t *ks = smem + st * C::STAGE_BYTES;
    const uint8_t *vs = ks + C::PB;
    const int page_pos0 = (it.pg0 + i) * kPagePositions;
#pragma unroll 1
    for (int blk = 0; blk < C::NBLK; blk++) {
      float sc[C::ITB][GC];
#pragma unroll
      for (int s = 0; s < C::ITB; s++) {
        const int pip = warp * C::POS_PER_WARP + (blk * C::ITB + s) * C::PPW + pg;
        const int pos = page_pos0 + pip;
        const bool valid = pos >= it.r0 && pos < it.r1;
        uint32_t w[C::BPL / 4];
        load_words<C::BPL>(ks + pip * (HD / 2) + byte0, w);
        const float2 sb = *reinterpret_cast<const float2 *>(ks + C::NIB + (pip * C::GPD + grp) * 8);
        float2 nl[C::BPL / 2], nh[C::BPL / 2];
        convert<C::BPL>(w, nl, nh);
#pragma unroll
        for (int h = 0; h < GC; h++) {
          float2 acc = make_float2(0.f, 0.f);
#pragma unroll
          for (int p = 0; p < C::BPL / 2; p++) {
            acc = __ffma2_rn(ql[h][p], nl[p], acc);
            acc = __ffma2_rn(qhv[h][p], nh[p], acc);
          }
          float part = fmaf(acc.x + acc.y, sb.x, sb.y * qsum[h]);
#pragma unroll
          for (int o = 1; o < C::LPP; o <<= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
          sc[s][h] = valid ? part : -INFINITY;
        }
      }
      // online softmax update, base 2
      float p[C::ITB][GC];
#pragma unroll
      for (int h = 0; h < GC; h++) {
        float bm = sc[0][h];
#pragma unroll
        for (int s = 1; s < C::ITB; s++) bm = fmaxf(bm, sc[s][h]);
#pragma unroll
        for (int o = C::LPP; o < 32; o <<= 1) bm = fmaxf(bm, __shfl_xor_sync(0xffffffffu, bm, o));
        const float mn = fmaxf(m[h], bm);
        if (mn == -INFINITY) {
#pragma unroll
          for (int s = 0; s < C::ITB; s++) p[s][h] = 0.0f;
          continue;
        }
        const float alpha = ex2(m[h] - mn);
        if (alpha != 1.0f) {
          l[h] *= alpha;
          pb[h] *= alpha;
          const float2 a2 = make_float2(alpha, alpha);
#pragma unroll
          for (int q = 0; q < C::BPL / 2; q++) {
            ol[h][q] = __fmul2_rn(ol[h][q], a2);
            oh[h][q] = __fmul2_rn(oh[h][q], a2);
          }
        }
        m[h] = mn;
#pragma unroll
        for (int s = 0; s < C::ITB; s++) {
          p[s][h] = ex2(sc[s][h] - mn);
          l[h] += p[s][h];
        }
      }
      // V accumulation
#pragma unroll
      for (int s = 0; s < C::ITB; s++) {
        const int pip = warp * C::POS_PER_WARP + (blk * C::ITB + s) * C::PPW + pg;
        const int pos = page_pos0 + pip;
        const bool valid = pos >= it.r0 && pos < it.r1;
        uint32_t w[C::BPL / 4];
        load_words<C::BPL>(vs + pip * (HD / 2) + byte0, w);
        float2 sb = *reinterpret_cast<const float2 *>(vs + C::NIB + (pip * C::GPD + grp) * 8);
        if (!valid) sb = make_float2(0.f, 0.f);
        float2 nl[C::BPL / 2], nh[C::BPL / 2];
        convert<C::BPL>(w, nl, nh);
#pragma unroll
        for (int h = 0; h < GC; h++) {
          const float ps = p[s][h] * sb.x;
          pb[h] = fmaf(p[s][h], sb.y, pb[h]);
          const float2 ps2 = make_float2(ps, ps);
#pragma unroll
          for (int q = 0; q < C::BPL / 2; q++) {
            ol[h][q] = __ffma2_rn(ps2, nl[q], ol[h][q]);
            oh[h][q] = __ffma2_rn(ps2, nh[q], oh[h][q]);
          }
        }
      }
    }
    __syncwarp();
    // the last warp to finish with this stage refills it with page i+NSTAGE
    if (lane == 0 && stage_release_last(reinterpret_cast<int *>(&bars[C::NSTAGE]) + st, C::NW) &&
        i + C::NSTAGE < it.npages)
      issue(i + C::NSTAGE);
  }
  // every wait above is bounded, so all threads get here; leave together
  if (!__syncthreads_and(ok)) {
    if (threadIdx.x == 0) drain_stages(bars, last_req, C::NSTAGE, a.wait_budget);
    // arrive without a record (the status word says why); if this CTA is
    // the item's last, nothing is merged
    if (a.n_splits > 1 && !a.sep_merge) arrive_last(a);
    return;
  }
  // every page requested was waited for, so no copy is in flight; checked,
  // and drained if not, before the ring is reused and the CTA exits
  if (threadIdx.x == 0 && !stages_idle(bars, last_req, C::NSTAGE)) {
    report(a, kStatusLateCopy);
    drain_stages(bars, last_req, C::NSTAGE, a.wait_budget);
  }

  // ---- reduce the warp's position slots --------------------------------
#pragma unroll
  for (int h = 0; h < GC; h++) {
    const float2 b2 = make_float2(pb[h], pb[h]);
#pragma unroll
    for (int q = 0; q < C::BPL / 2; q++) {
      ol[h][q] = __fadd2_rn(ol[h][q], b2);
      oh[h][q] = __fadd2_rn(oh[h][q], b2);
    }
#pragma unroll
    for (int o = C::LPP; o < 32; o <<= 1) {
      l[h] += __shfl_xor_sync(0xffffffffu, l[h], o);
#pragma unroll
      for (int q = 0; q < C::BPL / 2; q++) {
        ol[h][q].x += __shfl_xor_sync(0xffffffffu, ol[h][q].x, o);
        ol[h][q].y += __shfl_xor_sync(0xffffffffu, ol[h][q].y, o);
        oh[h][q].x += __shfl_xor_sync(0xffffffffu, oh[h][q].x, o);
        oh[h][q].y += __shfl_xor_sync(0xffffffffu, oh[h][q].y, o);
      }
    }
  }

  // ---- merge the consumer warps through shared memory -------------------
  __syncthreads();   // ring no longer read; reuse it for the merge
  float *mw = reinterpret_cast<float *>(smem);            // [NW][GC]
  float *lw = mw + C::NW * GC;                   // [NW][GC]
  float *ow = lw + C::NW * GC;                   // [NW][GC][HD]
  if (pg == 0) {
#pragma unroll
    for (int h = 0; h < GC; h++) {
      float *o = ow + (warp * GC + h) * HD + 64 * grp + k0;
#pragma unroll
      for (int q = 0; q < C::BPL / 2; q++) {
        o[2 * q] = ol[h][q].x;
        o[2 * q + 1] = ol[h][q].y;
        o[32 + 2 * q] = oh[h][q].x;
        o[32 + 2 * q + 1] = oh[h][q].y;
      }
      if (j == 0) {
        mw[warp * GC + h] = m[h];
        lw[warp * GC + h] = l[h];
      }
    }
  }
  __syncthreads();
  const size_t row0 = (size_t)(it.b * a.n_layers + it.lrow) * a.n_q_heads + qh0;
  for (int idx = threadIdx.x; idx < GC * HD; idx += C::NW * 32) {
    const int h = idx / HD, d = idx - h * HD;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < C::NW; w++) M = fmaxf(M, mw[w * GC + h]);
    float O = 0.0f, L = 0.0f;
    if (M != -INFINITY) {
#pragma unroll
      for (int w = 0; w < C::NW; w++) {
        const float f = ex2(mw[w * GC + h] - M);
        O = fmaf(f, ow[(w * GC + h) * HD + d], O);
        L = fmaf(f, lw[w * GC + h], L);
      }
    }
    const size_t row = row0 + h;
    if (a.n_splits == 1) {
      a.out[row * HD + d] = O / L;
      if (a.lse && d == 0) a.lse[row] = L > 0.0f ? (M + log2f(L)) * kLn2 : -INFINITY;
    } else {
      const size_t pr = row * a.n_splits + it.split;
      a.part_o[pr * HD + d] = O;
      if (d == 0) {
        a.part_m[pr] = M;
        a.part_l[pr] = L;
      }
    }
  }
  // the item's last split to finish merges all of them
  // (the ring is free again)
  if (a.n_splits > 1 && !a.sep_merge && arrive_last(a))
    merge_splits<HD, GC, C::THREADS>(a, row0, GC, reinterpret_cast<float *>(smem));
}

// Exact merge of partial results given as (normalized output, natural LSE).
// Part p's rows start at parts + p * part_stride and its LSEs at
// lse + p * lse_stride (floats).
__global__ void lse_combine_kernel(int n_parts, int HD, const float *parts, size_t part_stride,
                                   const float *lse, size_t lse_stride, float *out,
                                   float *lse_out) {
  const size_t row = blockIdx.x;
  const int d = threadIdx.x;
  float M = -INFINITY;
  for (int p = 0; p < n_parts; p++) M = fmaxf(M, lse[p * lse_stride + row]);
  float O = 0.0f, L = 0.0f;
  if (M != -INFINITY) {
    for (int p = 0; p < n_parts; p++) {
      const float lp = lse[p * lse_stride + row];
      if (lp == -INFINITY) continue;   // empty range: its output is 0/0
      const float f = ex2((lp - M) * kLog2e);
      if (d < HD) O = fmaf(f, parts[p * part_stride + row * HD + d], O);
      L += f;
    }
  }
  if (d < HD) out[row * HD + d] = O / L;
  if (lse_out && d == 0) lse_out[row] = L > 0.0f ? M + logf(L) : -INFINITY;
}

// The split merge as a kernel of its own (grid = rows, block = HD threads):
// what the decode kernels do in their last CTA of a row group, kept as a
// second launch for the tests that compare the two bit for bit.
__global__ void split_merge_kernel(const DecodeArgs a) {
  if (a.head_dim == 128) {
    if (threadIdx.x < 128) merge_row<128>(a, blockIdx.x, threadIdx.x);
  } else {
    if (threadIdx.x < 64) merge_row<64>(a, blockIdx.x, threadIdx.x);
  }
}

typedef void (*DecodeFn)(const DecodeArgs, const DecodeBatch);

template <int HD, int GC>
int launch_simt(const DecodeArgs &a, const DecodeBatch &b, int n_blocks, cudaStream_t s) {
  using C = Cfg<HD, GC>;
  auto fn = decode_simt_kernel<HD, GC>;
  static std::atomic<unsigned long long> attr_done{0};   // one bit per device
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(attr_done.load(std::memory_order_acquire) >> (dev & 63) & 1)) {
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    if (e != cudaSuccess) return check_cuda(e, "decode: smem attribute");
    attr_done.fetch_or(1ull << (dev & 63), std::memory_order_acq_rel);
  }
  fn<<<n_blocks, C::THREADS, C::SMEM, s>>>(a, b);
  return check_cuda(cudaGetLastError(), "decode launch");
}

template <int HD, int GC>
int resident_simt() {
  using C = Cfg<HD, GC>;
  // per device (resident CTAs per SM x SMs), filled on first use
  static std::atomic<int> cached[64];
  int dev = 0;
  cudaGetDevice(&dev);
  const int hit = cached[dev & 63].load(std::memory_order_relaxed);
  if (hit) return hit;
  cudaFuncSetAttribute(decode_simt_kernel<HD, GC>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                       C::SMEM);
  int per_sm = 1, sms = 148;
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, decode_simt_kernel<HD, GC>, C::THREADS,
                                                C::SMEM);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (per_sm < 1) per_sm = 1;
  cached[dev & 63].store(per_sm * sms, std::memory_order_relaxed);
  return per_sm * sms;
}

int pick_gc(int G) {
  if (G % 8 == 0) return 8;
  if (G % 4 == 0) return 4;
  if (G % 2 == 0) return 2;
  return 1;
}

template <int HD>
int dispatch_gc(int gc, const DecodeArgs &a, const DecodeBatch &b, int n_blocks, cudaStream_t s) {
  switch (gc) {
    case 8: return launch_simt<HD, 8>(a, b, n_blocks, s);
    case 4: return launch_simt<HD, 4>(a, b, n_blocks, s);
    case 2: return launch_simt<HD, 2>(a, b, n_blocks, s);
    default: return launch_simt<HD, 1>(a, b, n_blocks, s);
  }
}

template <int HD>
int resident_gc(int gc) {
  switch (gc) {
    case 8: return resident_simt<HD, 8>();
    case 4: return resident_simt<HD, 4>();
    case 2: return resident_simt<HD, 2>();
    default: return resident_simt<HD, 1>();
  }
}

}  // namespace

// Chooses the kernel (the tensor-core kernel for head_dim 64 and 128, the
// CUDA-core kernel when forced) and the split count.
struct Plan {
  int mma_gh;   // 0: CUDA-core kernel
  bool umma;    // tcgen05 kernel (else mma.sync) for the tensor-core path
  int gc;       // query heads per CTA
  int items;
};

constexpr int kMaxSplitPages = 256;   // 16384 positions

// Modeled duration, in page times of one CTA, of a launch of `items` rows cut
// into splits of `sp` pages (n per row), `per_sm` CTAs resident per SM on
// `sms` SMs. Every CTA costs its pages plus a fixed kCtaOverheadPages (query
// set-up, pipeline fill, merge, its share of the split merge). The busiest
// SM receives m = ceil(CTAs / sms) of them and runs them in rounds of
// per_sm; a last round of r < per_sm CTAs costs (r / per_sm)^(2/3) of a full
// one (its CTAs share the SM with fewer others and run faster, but not in
// proportion). Fitted to split sweeps on the cfg1-cfg5 shapes (one row of
// 512 pages at 4 splits: 258 us, at 2: 276 us, at 3: 296 us; cfg2 at 4: 21.7
// us, at 16: 35.0 us), whose ranking it reproduces.
constexpr double kCtaOverheadPages = 8.0;

// frac[r] = (r / per_sm)^(2/3), the cost of a last round of r CTAs.
static double split_cost(long long items, int max_pages, int sp, int per_sm, int sms,
                         const double *frac) {
  const int n = (max_pages + sp - 1) / sp;
  const long long m = (items * n + sms - 1) / sms;
  const long long rounds = (m + per_sm - 1) / per_sm;
  const long long r = m - (long long)per_sm * (rounds - 1);
  return (sp + kCtaOverheadPages) * ((double)(rounds - 1) + frac[r]);
}

// The split count in [lo, hi] of least modeled duration (the first of equals).
// Split counts with the same split length cost the same, so only the first
// count of each length is evaluated; and since decode steps repeat their
// shapes, each host thread keeps its last few answers.
int choose_splits(long long items, int max_pages, int lo, int hi, int per_sm, int sms) {
  if (max_pages < 1 || lo < 1 || hi < lo || per_sm < 1 || sms < 1) return lo > 0 ? lo : 1;
  struct Memo {
    long long items;
    int max_pages, lo, hi, per_sm, sms, ns;
  };
  thread_local Memo memo[4] = {};
  thread_local int memo_next = 0;
  for (const Memo &m : memo)
    if (m.ns && m.items == items && m.max_pages == max_pages && m.lo == lo && m.hi == hi &&
        m.per_sm == per_sm && m.sms == sms)
      return m.ns;
  std::vector<double> frac(per_sm + 1);
  for (int r = 0; r <= per_sm; r++) frac[r] = pow((double)r / per_sm, 2.0 / 3.0);
  int ns = lo;
  double best = 0.0;
  for (int k = lo; k <= hi;) {
    const int sp = (max_pages + k - 1) / k;
    const double c = split_cost(items, max_pages, sp, per_sm, sms, frac.data());
    if (k == lo || c < best) {
      best = c;
      ns = k;
    }
    if (sp == 1) break;
    k = (max_pages - 1) / (sp - 1) + 1;   // the first count whose splits are shorter
  }
  memo[memo_next] = Memo{items, max_pages, lo, hi, per_sm, sms, ns};
  memo_next = (memo_next + 1) % 4;
  return ns;
}

static int sm_count() {
  static std::atomic<int> cached[64];
  int dev = 0;
  cudaGetDevice(&dev);
  const int d = dev & 63;
  int n = cached[d].load(std::memory_order_relaxed);
  if (!n) {
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
    cached[d].store(n, std::memory_order_relaxed);
  }
  return n;
}

static Plan plan(DecodeArgs &a, const DecodeBatch &batch) {
  const int G = a.n_q_heads / a.geom.n_heads;
  Plan p;
  p.mma_gh = a.force_path == 1 ? 0 : mma_heads_per_cta(G, a.head_dim);
  p.gc = p.mma_gh ? p.mma_gh : pick_gc(G);
  p.umma = p.mma_gh && a.force_path == 3 && umma_resident(p.mma_gh, a.head_dim) > 0;
  int max_pages = 0;
  for (int i = 0; i < a.n_caches; i++) {
    int r0 = a.pos_begin > 0 ? a.pos_begin : 0;
    int r1 = a.pos_end < 0 ? batch.seq_len[i] : (batch.seq_len[i] < a.pos_end ? batch.seq_len[i] : a.pos_end);
    int pages = r1 > r0 ? (r1 + kPagePositions - 1) / kPagePositions - r0 / kPagePositions : 0;
    if (pages > max_pages) max_pages = pages;
  }
  p.items = a.n_caches * a.n_layers * a.geom.n_heads * (G / p.gc);
  if (a.fix_split_pages > 0 && a.fix_n_splits > 0) {
    // a chunk of a batch planned as a whole: the same split boundaries, so
    // every row's result equals the single launch's bit for bit
    a.split_pages = a.fix_split_pages;
    a.n_splits = a.fix_n_splits;
    return p;
  }
  const int resident = p.umma     ? umma_resident(p.mma_gh, a.head_dim)
                       : p.mma_gh ? mma_resident(p.mma_gh, a.head_dim)
                                  : (a.head_dim == 128 ? resident_gc<128>(p.gc) : resident_gc<64>(p.gc));
  int ns = 1;
  if (max_pages > 1) {
    // fewest splits: the tensor core's f32 accumulators drift with the
    // number of accumulation steps (1.1e-4 absolute after 512 pages of one
    // row, on outputs of ~0.02; about half that at 256), so no split of the
    // tensor-core kernel is longer than kMaxSplitPages pages
    const int lo = p.mma_gh ? (max_pages + kMaxSplitPages - 1) / kMaxSplitPages : 1;
    // most splits: for the tensor-core kernel at least two pages per split
    // (it gives each page to one warp, so a one-page split idles the rest)
    int hi = p.mma_gh ? max_pages / 2 : max_pages;
    if (hi < lo) hi = lo;
    if (hi > 4096) hi = 4096;
    const int sms = sm_count();
    const int per_sm = resident / sms > 0 ? resident / sms : 1;
    ns = choose_splits(p.items, max_pages, lo, hi, per_sm, sms);
    if (a.force_splits > 0) ns = a.force_splits;
    if (ns > max_pages) ns = max_pages;
    if (ns < 1) ns = 1;
  }
  a.split_pages = max_pages > 0 ? (max_pages + ns - 1) / ns : 1;
  a.n_splits = max_pages > 0 ? (max_pages + a.split_pages - 1) / a.split_pages : 1;
  return p;
}

void decode_fix_plan(DecodeArgs &a, const DecodeBatch &batch) {
  DecodeArgs t = a;
  t.fix_split_pages = t.fix_n_splits = 0;
  plan(t, batch);
  a.fix_split_pages = t.split_pages;
  a.fix_n_splits = t.n_splits;
}

size_t decode_workspace_bytes(const DecodeArgs &a0, const DecodeBatch &batch) {
  DecodeArgs a = a0;
  plan(a, batch);
  if (a.n_splits <= 1) return 0;
  size_t rows = (size_t)a.n_caches * a.n_layers * a.n_q_heads;
  return rows * a.n_splits * (size_t)(a.head_dim + 2) * sizeof(float);
}

size_t decode_counters(const DecodeArgs &a0, const DecodeBatch &batch) {
  DecodeArgs a = a0;
  const Plan p = plan(a, batch);
  return a.n_splits > 1 ? (size_t)p.items : 0;
}

int decode_launch(const DecodeArgs &a0, const DecodeBatch &batch, void *workspace,
                  size_t workspace_bytes, cudaStream_t s) {
  DecodeArgs a = a0;
  if (a.wait_budget == 0) a.wait_budget = kWaitBudget;
  const Plan p = plan(a, batch);
  if (a.n_splits > 1) {
    size_t rows = (size_t)a.n_caches * a.n_layers * a.n_q_heads;
    size_t need = rows * a.n_splits * (size_t)(a.head_dim + 2) * sizeof(float);
    if (!workspace || workspace_bytes < need) {
      set_error(EAKV_ERR_ALLOC, "decode: workspace too small (%zu < %zu)", workspace_bytes, need);
      return EAKV_ERR_ALLOC;
    }
    if (!a.cnt && !a.sep_merge) {
      set_error(EAKV_ERR_ALLOC, "decode: no split counters");
      return EAKV_ERR_ALLOC;
    }
    a.part_o = (float *)workspace;
    a.part_m = a.part_o + rows * a.n_splits * a.head_dim;
    a.part_l = a.part_m + rows * a.n_splits;
  }
  const int n_blocks = p.items * a.n_splits;
  if (n_blocks <= 0) return EAKV_OK;
  int rc;
  if (p.umma)
    rc = umma_launch(p.mma_gh, a, batch, n_blocks, s);
  else if (p.mma_gh)
    rc = mma_launch(p.mma_gh, a, batch, n_blocks, s);
  else
    rc = a.head_dim == 128 ? dispatch_gc<128>(p.gc, a, batch, n_blocks, s)
                           : dispatch_gc<64>(p.gc, a, batch, n_blocks, s);
  if (!rc && a.n_splits > 1 && a.sep_merge) {
    const size_t rows = (size_t)a.n_caches * a.n_layers * a.n_q_heads;
    split_merge_kernel<<<(unsigned)rows, a.head_dim, 0, s>>>(a);
    rc = check_cuda(cudaGetLastError(), "decode: merge launch");
  }
  return rc;
}

int lse_combine_launch(int n_parts, int n_rows, int head_dim, const float *parts,
                       size_t part_stride, const float *lse, size_t lse_stride, float *out,
                       float *lse_out, cudaStream_t s) {
  if (n_rows <= 0) return EAKV_OK;
  lse_combine_kernel<<<n_rows, head_dim, 0, s>>>(n_parts, head_dim, parts, part_stride, lse,
                                                 lse_stride, out, lse_out);
  return check_cuda(cudaGetLastError(), "lse_combine launch");
}

}  // namespace eakv
