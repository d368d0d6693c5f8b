// attention.cu - the reference's two-call attention API on the device
// cache: K-scores (reference src/attention.c:3-32 dispatching to
// kernels/fused_k_score*.ea and fused_k_score_gqa*.ea) and the V weighted
// sum (src/attention.c:34-63 -> fused_v_sum*.ea, fused_k_score_gqa*.ea).
//
// Scores are computed in exactly the reference's operation order and are
// bit-identical to it whenever its 16-lane horizontal sum is the halving
// tree: 16 threads play the 16 SIMD lanes of one position, lane l runs the
// chain acc = fma(fma(n, s, b), q, acc) over elements l, 16+l, 32+l, 48+l of
// each group in turn, and the lanes are folded with xor-8/4/2/1 shuffles.
// The dequantized K row is formed once and reused by every query head of
// the KV head (the GQA loop flip, fused_k_score_gqa.ea:31-92).
//
// The V sum is one chain per output element over positions. Inside a chunk
// of positions a thread runs that chain in position order, as the reference
// does; chunks run in parallel and are added in chunk order, so the result
// is bit-identical to the reference when the sequence fits one chunk and
// differs only by that final re-association otherwise.
#include <math.h>
#include <stdio.h>

#include <atomic>
#include <type_traits>

#include "internal.cuh"
#include "pipeline.cuh"

namespace eakv {
namespace {

constexpr int kScoreThreads = 256;   // 8 warps x 8 quads, each quad 2 positions
constexpr int kHeadChunk = 32;       // query heads per pass (shared memory bound)

// The reference's f32x16 vector of one position's chain, split over a quad of
// threads: thread t of the quad plays SIMD lanes t, t+4, t+8 and t+12, so the
// first two levels of the halving-tree reduce_add (lanes l + l+8, then l +
// l+4) stay inside the thread and only the last two (l + l+2, l + l+1) cross
// threads. Lane l of group g, step jj runs
//   acc_l = fma(fma(n, s, b), q[64 g + 16 jj + l], acc_l)
// over (g, jj) in order: jj = 0, 1 take the low nibbles of bytes l and 16 + l,
// jj = 2, 3 their high nibbles (kernels/fused_k_score.ea:41-100). Lanes (t,
// t+4) and (t+8, t+12) run as f32x2 pairs: two independent chains per
// instruction, each rounded as one fma.

// Bytes t, t+4, t+8, t+12 of a 16-byte chunk (byte t of each of its words).
__device__ __forceinline__ uint32_t gather_lane_bytes(uint4 v, uint32_t sel) {
  const uint32_t x = __byte_perm(v.x, v.y, sel);
  const uint32_t y = __byte_perm(v.z, v.w, sel);
  return __byte_perm(x, y, 0x5410);
}

// The four nibbles (one per byte) of w as two exact float pairs, dequantized
// with one rounding each: (fma(n0, s, b), fma(n1, s, b)), (fma(n2, ...), ...).
__device__ __forceinline__ void dequant4(uint32_t w, float2 s2, float2 b2, float2 &lo,
                                         float2 &hi) {
  const float2 off = make_float2(-8388608.0f, -8388608.0f);
  const float2 n01 = __fadd2_rn(make_float2(__uint_as_float(__byte_perm(w, 0x4B000000u, 0x7440)),
                                            __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7441))),
                                off);
  const float2 n23 = __fadd2_rn(make_float2(__uint_as_float(__byte_perm(w, 0x4B000000u, 0x7442)),
                                            __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7443))),
                                off);
  lo = __ffma2_rn(n01, s2, b2);
  hi = __ffma2_rn(n23, s2, b2);
}

constexpr int kScorePages = 8;   // pages a block stages at once (40 KB at head_dim 128)

// grid: (page blocks of up to kScorePages pages, n_kv, head chunks). The
// block's pages arrive in shared memory by one bulk copy each (one mbarrier,
// bounded wait) while the queries of the chunk are staged; each quad then
// scores positions p and p + 64 of every 128-position step, for every query
// head of the chunk, from one dequantization of each K row.
template <int HD>
__global__ void __launch_bounds__(kScoreThreads, 2)
scores_kernel(const uint8_t *__restrict__ buf, PageGeom g, int layer,
              const float *__restrict__ q, int q_per_kv, int seq_len, float rsqrt_d,
              float *__restrict__ scores, int pages_per_block, int *status) {
  constexpr int GPD = HD / 64;
  constexpr int PB = kPagePositions * GPD * 40, NIB = kPagePositions * GPD * 32;
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t *bar = reinterpret_cast<uint64_t *>(smem);
  uint8_t *pages = smem + 128;
  float4 *q_s = reinterpret_cast<float4 *>(pages + kScorePages * PB);   // [nh][GPD][jj][t]
  const int kvh = blockIdx.y;
  const int h0 = blockIdx.z * kHeadChunk;
  const int nh = min(kHeadChunk, q_per_kv - h0);
  const int n_seq_pages = (seq_len + kPagePositions - 1) / kPagePositions;
  const int pg0 = blockIdx.x * pages_per_block;
  const int npg = min(n_seq_pages, pg0 + pages_per_block) - pg0;
  if (threadIdx.x == 0) {
    mbar_init(smem_u32(bar), 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    mbar_arrive_expect_tx(smem_u32(bar), (uint32_t)(npg * PB));
    for (int i = 0; i < npg; i++)
      bulk_g2s(smem_u32(pages + i * PB), buf + page_index(g, layer, 0, kvh, pg0 + i) * g.page_bytes,
               PB, smem_u32(bar));
  }
  for (int i = threadIdx.x; i < nh * HD; i += blockDim.x) {
    const int j = i / HD, e = i - j * HD;
    const int grp = e >> 6, jj = (e >> 4) & 3, l = e & 15;
    reinterpret_cast<float *>(q_s)[(((j * GPD + grp) * 4 + jj) * 4 + (l & 3)) * 4 + (l >> 2)] =
        q[(size_t)(kvh * q_per_kv + h0 + j) * HD + e];
  }
  const bool ok = mbar_wait(smem_u32(bar), 0, kWaitBudget);
  if (!__syncthreads_and(ok)) {
    if (threadIdx.x == 0) {
      if (status) atomicOr(status, kStatusWaitTimeout);
      mbar_wait(smem_u32(bar), 0, kWaitBudget);   // no copy may outlive the block
    }
    return;
  }
  const int t = threadIdx.x & 3, quad = threadIdx.x >> 2;
  const uint32_t sel = (uint32_t)t | ((uint32_t)(4 + t) << 4);
  const int pos_end = npg * kPagePositions;   // block-local
  for (int pos0 = 0; pos0 < pos_end; pos0 += 2 * kPagePositions) {
    float2 k[2][GPD][4][2];   // [position][group][jj][lanes (t, t+4) | (t+8, t+12)]
    int tp[2];
#pragma unroll
    for (int p = 0; p < 2; p++) {
      tp[p] = pos0 + p * kPagePositions + quad;
      // a block's last step may hold one page only: read the first one again
      const int pos = tp[p] < pos_end ? tp[p] : pos0 + quad;
      const uint8_t *pp = pages + (pos / kPagePositions) * PB;
      const int pip = pos % kPagePositions;
      const uint4 *row = reinterpret_cast<const uint4 *>(pp + pip * (HD / 2));
      const float *sb = reinterpret_cast<const float *>(pp + NIB) + pip * GPD * 2;
#pragma unroll
      for (int grp = 0; grp < GPD; grp++) {
        const uint32_t z0 = gather_lane_bytes(row[2 * grp], sel);       // bytes l
        const uint32_t z1 = gather_lane_bytes(row[2 * grp + 1], sel);   // bytes 16 + l
        const float2 s2 = make_float2(sb[2 * grp], sb[2 * grp]);
        const float2 b2 = make_float2(sb[2 * grp + 1], sb[2 * grp + 1]);
        dequant4(z0 & 0x0F0F0F0Fu, s2, b2, k[p][grp][0][0], k[p][grp][0][1]);
        dequant4(z1 & 0x0F0F0F0Fu, s2, b2, k[p][grp][1][0], k[p][grp][1][1]);
        dequant4((z0 >> 4) & 0x0F0F0F0Fu, s2, b2, k[p][grp][2][0], k[p][grp][2][1]);
        dequant4((z1 >> 4) & 0x0F0F0F0Fu, s2, b2, k[p][grp][3][0], k[p][grp][3][1]);
      }
    }
    // NP query heads at once: 4 NP independent f32x2 chains per thread
    auto score_heads = [&](int j, auto np_tag) {
      constexpr int NP = decltype(np_tag)::value;
      float2 acc[NP][2][2];
#pragma unroll
      for (int u = 0; u < NP; u++)
#pragma unroll
        for (int p = 0; p < 2; p++) acc[u][p][0] = acc[u][p][1] = make_float2(0.0f, 0.0f);
#pragma unroll
      for (int grp = 0; grp < GPD; grp++)
#pragma unroll
        for (int jj = 0; jj < 4; jj++)
#pragma unroll
          for (int u = 0; u < NP; u++) {
            const float4 qv = q_s[(((j + u) * GPD + grp) * 4 + jj) * 4 + t];
            const float2 qa = make_float2(qv.x, qv.y), qb = make_float2(qv.z, qv.w);
#pragma unroll
            for (int p = 0; p < 2; p++) {
              acc[u][p][0] = __ffma2_rn(k[p][grp][jj][0], qa, acc[u][p][0]);
              acc[u][p][1] = __ffma2_rn(k[p][grp][jj][1], qb, acc[u][p][1]);
            }
          }
#pragma unroll
      for (int u = 0; u < NP; u++)
#pragma unroll
        for (int p = 0; p < 2; p++) {
          const float2 t1 = __fadd2_rn(acc[u][p][0], acc[u][p][1]);   // lanes l + l+8
          float r = __fadd_rn(t1.x, t1.y);                             // l + l+4
          r = __fadd_rn(r, __shfl_xor_sync(0xffffffffu, r, 2));        // l + l+2
          r = __fadd_rn(r, __shfl_xor_sync(0xffffffffu, r, 1));        // l + l+1
          const int gpos = pg0 * kPagePositions + tp[p];
          if (t == 0 && tp[p] < pos_end && gpos < seq_len)
            scores[(size_t)(kvh * q_per_kv + h0 + j + u) * seq_len + gpos] = __fmul_rn(r, rsqrt_d);
        }
    };
    int j = 0;
    for (; j + 3 < nh; j += 4) score_heads(j, std::integral_constant<int, 4>{});
    for (; j + 1 < nh; j += 2) score_heads(j, std::integral_constant<int, 2>{});
    if (j < nh) score_heads(j, std::integral_constant<int, 1>{});
  }
}

template <int HD>
size_t scores_smem() {
  return 128 + (size_t)kScorePages * kPagePositions * (HD / 64) * 40 +
         (size_t)kHeadChunk * HD * sizeof(float);
}

template <int HD>
cudaError_t launch_scores_hd(dim3 grid, const PageGeom &g, const uint8_t *d_buf, int layer,
                             const float *d_q, int q_per_kv, int seq_len, float rsqrt_d,
                             float *d_scores, int ppb, int *status, cudaStream_t s) {
  static std::atomic<unsigned long long> attr_done{0};   // one bit per device
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(attr_done.load(std::memory_order_acquire) >> (dev & 63) & 1)) {
    cudaError_t e = cudaFuncSetAttribute(scores_kernel<HD>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)scores_smem<HD>());
    if (e != cudaSuccess) return e;
    attr_done.fetch_or(1ull << (dev & 63), std::memory_order_acq_rel);
  }
  scores_kernel<HD><<<grid, kScoreThreads, scores_smem<HD>(), s>>>(
      d_buf, g, layer, d_q, q_per_kv, seq_len, rsqrt_d, d_scores, ppb, status);
  return cudaGetLastError();
}

constexpr int kVHeads = 8;          // query heads per block (accumulators per thread)
constexpr int kVThreads = 128;
constexpr int kVChunkPages = 8;     // positions of one block: 512
constexpr int kVExactMax = 512;     // up to this length the whole sum is one chain
constexpr int kVMergeInLaunch = 64; // most blocks per sequence merged inside the launch
constexpr int kVRun = 8;            // blocks per run of the two-level merge
static_assert(kVMergeInLaunch <= kVRun * kVRun, "the second merge level adds at most kVRun runs");

__device__ __forceinline__ float4 add4(float4 a, float4 b) {
  return make_float4(__fadd_rn(a.x, b.x), __fadd_rn(a.y, b.y), __fadd_rn(a.z, b.z),
                     __fadd_rn(a.w, b.w));
}

// dst[e] = src[0][e] + src[stride][e] + ... (n <= kVRun terms, in that
// order) for the float4 columns e of one (KV head, head group): all n loads
// of a column in flight at once, L1 bypassed (other blocks wrote them).
// dst4 (16-byte aligned) or, when it is null, dst (any 4-byte offset).
__device__ __forceinline__ void vsum_add_run(const float4 *src, size_t stride, int n, int cols,
                                             float4 *dst4, float *dst) {
  for (int e = threadIdx.x; e < cols; e += kVThreads) {
    float4 v[kVRun];
#pragma unroll
    for (int u = 0; u < kVRun; u++)
      if (u < n) v[u] = __ldcg(src + (size_t)u * stride + e);
    float4 a = v[0];
#pragma unroll
    for (int u = 1; u < kVRun; u++)
      if (u < n) a = add4(a, v[u]);
    if (dst4) {
      dst4[e] = a;
    } else {
      dst[4 * e] = a.x;
      dst[4 * e + 1] = a.y;
      dst[4 * e + 2] = a.z;
      dst[4 * e + 3] = a.w;
    }
  }
}

// A block's arrival at its item's counter, after its partial sums are
// written: true in the item's last block to arrive. The counter wraps back
// to zero with that arrival, ready for the next launch.
__device__ __forceinline__ bool vsum_arrive_last(unsigned *cnt, int n) {
  __shared__ int s_last;
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) s_last = atomicInc(cnt, (unsigned)n - 1) == (unsigned)n - 1;
  __syncthreads();
  const bool last = s_last != 0;
  if (last) __threadfence();
  return last;
}

// V sum. Every output element (query head h, dim d) is its own chain over
// positions, o = fma(fma(n, s, b), w[h][t], o), in position order
// (kernels/fused_v_sum.ea:111-150). A block takes up to 8 pages of one KV
// head and up to 8 query heads: one bulk copy per page brings the pages into
// shared memory (one mbarrier, bounded wait), the weights are staged beside
// them, and the positions are cut among position streams of HD/8 threads.
// Thread i of a stream owns bytes 4i..4i+3 of a position's nibble row, i.e.
// dims b..b+3 and b+32..b+35 of its group, and runs its chains as f32x2
// pairs. Up to kVExactMax positions a single stream runs the whole sequence
// (one chain per element, bit-identical to the reference); longer sequences
// add the streams' sums, then the blocks' sums, in position order, which
// re-associates the sum (within the 1e-4 bar).
//
// grid: (chunks of kVChunkPages pages, n_kv, head groups of kVHeads).
// Writes d_out directly when there is one chunk, else a partial per chunk.
template <int HD, int NH>
__global__ void __launch_bounds__(kVThreads)
vsum_kernel(const uint8_t *__restrict__ buf, PageGeom g, int layer,
            const float *__restrict__ w, int q_per_kv, int seq_len, int cp, int n_chunks,
            float *__restrict__ out, float *__restrict__ part, unsigned *__restrict__ cnt,
            int n_q, int *status) {
  constexpr int GPD = HD / 64, TPS = HD / 8, NSTREAM = kVThreads / TPS;
  constexpr int PB = kPagePositions * GPD * 40, NIB = kPagePositions * GPD * 32;
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t *bar = reinterpret_cast<uint64_t *>(smem);
  uint8_t *pages = smem + 128;
  float *w_s = reinterpret_cast<float *>(pages + cp * PB);   // [nh][cp * 64]
  const int kvh = blockIdx.y;
  const int h0 = blockIdx.z * kVHeads;
  const int nh = min(kVHeads, q_per_kv - h0);
  const int cpos = cp * kPagePositions;   // positions of a block
  const int c0 = blockIdx.x * cpos;
  const int len = min(seq_len - c0, cpos);
  const int pg0 = c0 / kPagePositions, npg = (len + kPagePositions - 1) / kPagePositions;
  if (threadIdx.x == 0) {
    mbar_init(smem_u32(bar), 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    mbar_arrive_expect_tx(smem_u32(bar), (uint32_t)(npg * PB));
    for (int i = 0; i < npg; i++)
      bulk_g2s(smem_u32(pages + i * PB),
               buf + page_index(g, layer, 1, kvh, pg0 + i) * g.page_bytes, PB, smem_u32(bar));
  }
  // weights of the chunk, eight loads in flight per thread before any store
  for (int i0 = 0; i0 < nh * len; i0 += 8 * kVThreads) {
    float wv[8];
#pragma unroll
    for (int u = 0; u < 8; u++) {
      const int i = i0 + u * kVThreads + threadIdx.x;
      const int j = i / len, tt = i - j * len;
      wv[u] = i < nh * len ? __ldg(w + (size_t)(kvh * q_per_kv + h0 + j) * seq_len + c0 + tt)
                           : 0.0f;
    }
#pragma unroll
    for (int u = 0; u < 8; u++) {
      const int i = i0 + u * kVThreads + threadIdx.x;
      const int j = i / len, tt = i - j * len;
      if (i < nh * len) w_s[j * cpos + tt] = wv[u];
    }
  }
  const bool ok = mbar_wait(smem_u32(bar), 0, kWaitBudget);
  if (!__syncthreads_and(ok)) {
    if (threadIdx.x == 0) {
      if (status) atomicOr(status, kStatusWaitTimeout);
      mbar_wait(smem_u32(bar), 0, kWaitBudget);   // no copy may outlive the block
    }
    // arrive all the same, so that the counters return to zero (the status
    // word tells the caller the result is void)
    if (cnt) {
      const int n_run = (n_chunks + kVRun - 1) / kVRun, run = blockIdx.x / kVRun;
      unsigned *gc = cnt + (size_t)(blockIdx.y * gridDim.z + blockIdx.z) * (n_run + 1);
      if (vsum_arrive_last(gc + 1 + run, min(kVRun, n_chunks - run * kVRun)) && n_run > 1)
        vsum_arrive_last(gc, n_run);
    }
    return;
  }
  const int stream = threadIdx.x / TPS, i = threadIdx.x - stream * TPS;
  const int nused = seq_len <= kVExactMax ? 1 : NSTREAM;
  // streams take runs of a multiple of 4 positions (16-byte weight loads)
  const int sub = ((len + nused - 1) / nused + 3) & ~3;
  const int t0 = stream * sub, t1 = min(len, t0 + sub);
  const int grp = (4 * i) / 32;
  float2 o[NH][4];
#pragma unroll
  for (int j = 0; j < NH; j++)
#pragma unroll
    for (int k = 0; k < 4; k++) o[j][k] = make_float2(0.0f, 0.0f);
  if (stream < nused) {
    // four positions at a time (one page: 4 divides 64), their loads first;
    // every accumulator still takes its positions in order
    int tt = t0;
    for (; tt + 4 <= t1; tt += 4) {
      const uint8_t *pp = pages + (tt / kPagePositions) * PB;
      const int pip = tt % kPagePositions;
      uint32_t wd[4];
      float2 sb[4];
#pragma unroll
      for (int u = 0; u < 4; u++) {
        wd[u] = *reinterpret_cast<const uint32_t *>(pp + (pip + u) * (HD / 2) + 4 * i);
        sb[u] = *reinterpret_cast<const float2 *>(pp + NIB + ((pip + u) * GPD + grp) * 8);
      }
      float2 v[4][4];
#pragma unroll
      for (int u = 0; u < 4; u++) {
        const float2 s2 = make_float2(sb[u].x, sb[u].x), b2 = make_float2(sb[u].y, sb[u].y);
        dequant4(wd[u] & 0x0F0F0F0Fu, s2, b2, v[u][0], v[u][1]);
        dequant4((wd[u] >> 4) & 0x0F0F0F0Fu, s2, b2, v[u][2], v[u][3]);
      }
#pragma unroll
      for (int j = 0; j < NH; j++) {
        if (j < nh) {
          const float4 w4 = *reinterpret_cast<const float4 *>(w_s + j * cpos + tt);
          const float wu[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
          for (int u = 0; u < 4; u++) {
            const float2 w2 = make_float2(wu[u], wu[u]);
#pragma unroll
            for (int k = 0; k < 4; k++) o[j][k] = __ffma2_rn(v[u][k], w2, o[j][k]);
          }
        }
      }
    }
    for (; tt < t1; tt++) {
      const uint8_t *pp = pages + (tt / kPagePositions) * PB;
      const int pip = tt % kPagePositions;
      const uint32_t word = *reinterpret_cast<const uint32_t *>(pp + pip * (HD / 2) + 4 * i);
      const float2 sb = *reinterpret_cast<const float2 *>(pp + NIB + (pip * GPD + grp) * 8);
      const float2 s2 = make_float2(sb.x, sb.x), b2 = make_float2(sb.y, sb.y);
      float2 v[4];
      dequant4(word & 0x0F0F0F0Fu, s2, b2, v[0], v[1]);
      dequant4((word >> 4) & 0x0F0F0F0Fu, s2, b2, v[2], v[3]);
#pragma unroll
      for (int j = 0; j < NH; j++) {
        if (j < nh) {
          const float wj = w_s[j * cpos + tt];
          const float2 w2 = make_float2(wj, wj);
#pragma unroll
          for (int k = 0; k < 4; k++) o[j][k] = __ffma2_rn(v[k], w2, o[j][k]);
        }
      }
    }
  }
  // element (j, dim) of this thread: dims b..b+3 (v[0], v[1]) and b+32..b+35
  const int dim0 = grp * 64 + (4 * i) % 32;
  float *dst = n_chunks == 1 ? out : part + (size_t)blockIdx.x * n_q * HD;
  if (nused == 1) {
    if (stream == 0) {
      // dst is the caller's buffer when the call is one block: 16-byte
      // stores only where it is 16-byte aligned
      const bool vec = ((uintptr_t)dst & 15) == 0;
#pragma unroll
      for (int j = 0; j < NH; j++) {
        if (j < nh) {
          float *r = dst + (size_t)(kvh * q_per_kv + h0 + j) * HD + dim0;
          if (vec) {
            *reinterpret_cast<float4 *>(r) =
                make_float4(o[j][0].x, o[j][0].y, o[j][1].x, o[j][1].y);
            *reinterpret_cast<float4 *>(r + 32) =
                make_float4(o[j][2].x, o[j][2].y, o[j][3].x, o[j][3].y);
          } else {
#pragma unroll
            for (int k = 0; k < 4; k++) {
              r[(k >> 1) * 32 + 2 * (k & 1)] = o[j][k].x;
              r[(k >> 1) * 32 + 2 * (k & 1) + 1] = o[j][k].y;
            }
          }
        }
      }
    }
    return;
  }
  // add the streams' sums in position order, through shared memory
  __syncthreads();   // the pages are no longer read
  float *acc_s = reinterpret_cast<float *>(smem + 128);   // [NSTREAM][nh][HD]
#pragma unroll
  for (int j = 0; j < NH; j++) {
    if (j < nh) {
      float *r = acc_s + (stream * nh + j) * HD + dim0;
      *reinterpret_cast<float4 *>(r) = make_float4(o[j][0].x, o[j][0].y, o[j][1].x, o[j][1].y);
      *reinterpret_cast<float4 *>(r + 32) =
          make_float4(o[j][2].x, o[j][2].y, o[j][3].x, o[j][3].y);
    }
  }
  __syncthreads();
  for (int e = threadIdx.x; e < nh * HD; e += kVThreads) {
    const int j = e / HD, d = e - j * HD;
    float a = acc_s[j * HD + d];
    for (int st = 1; st < NSTREAM; st++) a = __fadd_rn(a, acc_s[(st * nh + j) * HD + d]);
    dst[(size_t)(kvh * q_per_kv + h0 + j) * HD + d] = a;
  }
  // Blocks' sums, two levels, in chunk order: the last block of each run of
  // kVRun blocks adds the run's sums into the run's first slot (or, for a
  // single run, into the output); the last run to finish adds the runs'
  // sums into the output. Each level is one round of loads from L2 per
  // column (the partial sums sit in the library's 256-byte aligned
  // workspace; the output is the caller's buffer, written one float at a
  // time).
  if (cnt) {
    const int n_run = (n_chunks + kVRun - 1) / kVRun, run = blockIdx.x / kVRun;
    unsigned *gc = cnt + (size_t)(blockIdx.y * gridDim.z + blockIdx.z) * (n_run + 1);
    const int r0 = run * kVRun, rn = min(kVRun, n_chunks - r0);
    if (vsum_arrive_last(gc + 1 + run, rn)) {
      const size_t n4 = (size_t)n_q * HD / 4;   // float4 per chunk
      const size_t row = (size_t)(kvh * q_per_kv + h0) * HD / 4;
      const float4 *p4 = reinterpret_cast<const float4 *>(part) + row;
      const int cols = nh * HD / 4;
      if (n_run == 1) {
        vsum_add_run(p4, n4, rn, cols, nullptr, out + row * 4);
      } else {
        vsum_add_run(p4 + (size_t)r0 * n4, n4, rn, cols,
                     reinterpret_cast<float4 *>(part) + row + (size_t)r0 * n4, nullptr);
        if (vsum_arrive_last(gc, n_run))
          vsum_add_run(p4, (size_t)kVRun * n4, n_run, cols, nullptr, out + row * 4);
      }
    }
  }
}

__global__ void fill_kernel(float *p, size_t n, float v) {
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x)
    p[i] = v;
}

// out[i] = part[0][i] + part[1][i] + ... in chunk order (the same order as
// the merge inside the launch), eight loads in flight at a time.
__global__ void vsum_combine_kernel(const float *__restrict__ part, int n_chunks, size_t n,
                                    float *__restrict__ out) {
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x) {
    float acc = part[i];
    int c = 1;
    for (; c + 8 <= n_chunks; c += 8) {
      float v[8];
#pragma unroll
      for (int u = 0; u < 8; u++) v[u] = part[(size_t)(c + u) * n + i];
#pragma unroll
      for (int u = 0; u < 8; u++) acc = __fadd_rn(acc, v[u]);
    }
    for (; c < n_chunks; c++) acc = __fadd_rn(acc, part[(size_t)c * n + i]);
    out[i] = acc;
  }
}

// Pages of one block. Up to kVExactMax positions the whole sequence is one
// block (its single stream keeps the reference's order, bit for bit); beyond
// that, blocks of 1..kVChunkPages pages, about one block per SM when the
// call is small (each block pays a fixed set-up and adds one partial sum),
// so that short sequences still spread over the GPU.
int vsum_chunk_pages(int n_q, int n_kv, int seq_len) {
  const int pages = (seq_len + kPagePositions - 1) / kPagePositions;
  if (seq_len <= kVExactMax) return pages > 0 ? pages : 1;
  const int q_per_kv = n_q / n_kv;
  const long long blocks = (long long)pages * n_kv * ((q_per_kv + kVHeads - 1) / kVHeads);
  const long long cp = (blocks + 147) / 148;
  return (int)(cp < 1 ? 1 : cp > kVChunkPages ? kVChunkPages : cp);
}

int vsum_chunks(int n_q, int n_kv, int seq_len) {
  if (seq_len <= 0) return 1;
  const int cp = vsum_chunk_pages(n_q, n_kv, seq_len);
  return (seq_len + cp * kPagePositions - 1) / (cp * kPagePositions);
}

// Shared memory of a block with nh query heads and cp pages: the staged
// pages and the heads' weights, later reused for the streams' sums. Sized by
// the heads and pages a block really has, so that 4 query heads per KV head
// fit 4 blocks per SM.
template <int HD>
size_t vsum_smem(int nh, int cp) {
  const size_t staged = (size_t)cp * kPagePositions * (HD / 64) * 40 +
                        (size_t)nh * cp * kPagePositions * sizeof(float);
  const size_t sums = (size_t)(kVThreads / (HD / 8)) * nh * HD * sizeof(float);
  return 128 + (staged > sums ? staged : sums);
}

template <int HD, int NH>
cudaError_t launch_vsum_nh(dim3 grid, const PageGeom &g, const uint8_t *d_buf, int layer,
                           const float *d_w, int q_per_kv, int seq_len, int cp, int n_chunks,
                           float *d_out, float *d_part, unsigned *d_cnt, int n_q, int *status,
                           cudaStream_t s) {
  static std::atomic<unsigned long long> attr_done{0};   // one bit per device
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(attr_done.load(std::memory_order_acquire) >> (dev & 63) & 1)) {
    cudaError_t e = cudaFuncSetAttribute(vsum_kernel<HD, NH>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)vsum_smem<HD>(NH, kVChunkPages));
    if (e != cudaSuccess) return e;
    attr_done.fetch_or(1ull << (dev & 63), std::memory_order_acq_rel);
  }
  const int nh = q_per_kv < NH ? q_per_kv : NH;
  vsum_kernel<HD, NH><<<grid, kVThreads, vsum_smem<HD>(nh, cp), s>>>(
      d_buf, g, layer, d_w, q_per_kv, seq_len, cp, n_chunks, d_out, d_part, d_cnt, n_q, status);
  return cudaGetLastError();
}

// The kernel's head count: the smallest of 1, 2, 4, 8 that holds a block's
// query heads (min(q_per_kv, kVHeads)), so that its accumulators fit.
template <int HD>
cudaError_t launch_vsum_hd(dim3 grid, const PageGeom &g, const uint8_t *d_buf, int layer,
                           const float *d_w, int q_per_kv, int seq_len, int cp, int n_chunks,
                           float *d_out, float *d_part, unsigned *d_cnt, int n_q, int *status,
                           cudaStream_t s) {
  const int nh = q_per_kv < kVHeads ? q_per_kv : kVHeads;
  auto go = [&](auto nh_tag) {
    return launch_vsum_nh<HD, decltype(nh_tag)::value>(grid, g, d_buf, layer, d_w, q_per_kv,
                                                        seq_len, cp, n_chunks, d_out, d_part,
                                                        d_cnt, n_q, status, s);
  };
  if (nh <= 1) return go(std::integral_constant<int, 1>{});
  if (nh <= 2) return go(std::integral_constant<int, 2>{});
  if (nh <= 4) return go(std::integral_constant<int, 4>{});
  return go(std::integral_constant<int, 8>{});
}

}  // namespace

cudaError_t launch_scores(const PageGeom &g, const uint8_t *d_buf, int layer, const float *d_q,
                          int n_q, int n_kv, int seq_len, float rsqrt_d, float *d_scores,
                          cudaStream_t s) {
  if (seq_len <= 0) return cudaSuccess;
  const int q_per_kv = n_q / n_kv;
  const int head_dim = g.gpd * 64;
  const int pages = (seq_len + 63) / 64;
  const int chunks = (q_per_kv + kHeadChunk - 1) / kHeadChunk;
  // about four blocks per SM in all, each a whole number of 128-position
  // steps and at most kScorePages pages
  int ppb = (int)(((long long)pages * n_kv * chunks + 591) / 592);
  ppb = ppb < 2 ? 2 : (ppb + 1) / 2 * 2;
  if (ppb > kScorePages) ppb = kScorePages;
  dim3 grid((pages + ppb - 1) / ppb, n_kv, chunks);
  int *status = device_status_ptr();
  return head_dim == 128
             ? launch_scores_hd<128>(grid, g, d_buf, layer, d_q, q_per_kv, seq_len, rsqrt_d,
                                     d_scores, ppb, status, s)
             : launch_scores_hd<64>(grid, g, d_buf, layer, d_q, q_per_kv, seq_len, rsqrt_d,
                                    d_scores, ppb, status, s);
}

size_t vsum_scratch_floats(const PageGeom &g, int n_q, int n_kv, int seq_len) {
  const int n_chunks = vsum_chunks(n_q, n_kv, seq_len);
  return n_chunks > 1 ? (size_t)n_chunks * n_q * g.gpd * 64 : 0;
}

size_t vsum_counters(int n_q, int n_kv, int seq_len) {
  const int n_chunks = vsum_chunks(n_q, n_kv, seq_len);
  const int n_run = (n_chunks + kVRun - 1) / kVRun;
  return n_chunks > 1 && n_chunks <= kVMergeInLaunch
             ? (size_t)n_kv * ((n_q / n_kv + kVHeads - 1) / kVHeads) * (n_run + 1) : 0;
}

cudaError_t launch_vsum(const PageGeom &g, const uint8_t *d_buf, int layer, const float *d_w,
                        int n_q, int n_kv, int seq_len, float *d_out, float *d_part,
                        size_t part_floats, unsigned *d_cnt, cudaStream_t s) {
  const int head_dim = g.gpd * 64;
  if (seq_len <= 0) {   // reference stores the zero-initialized accumulators
    fill_kernel<<<32, 256, 0, s>>>(d_out, (size_t)n_q * head_dim, 0.0f);
    return cudaGetLastError();
  }
  const int q_per_kv = n_q / n_kv;
  const int cp = vsum_chunk_pages(n_q, n_kv, seq_len);
  const int n_chunks = vsum_chunks(n_q, n_kv, seq_len);
  if (n_chunks > 1 && ((size_t)n_chunks * n_q * head_dim > part_floats ||
                        (n_chunks <= kVMergeInLaunch && !d_cnt)))
    return cudaErrorInvalidValue;   // sized by vsum_scratch_floats and vsum_counters
  dim3 grid(n_chunks, n_kv, (q_per_kv + kVHeads - 1) / kVHeads);
  int *status = device_status_ptr();
  // few blocks per sequence: the last one adds their sums in the same launch;
  // many: a second kernel spreads those sums over the whole GPU
  unsigned *merge_cnt = n_chunks > 1 && n_chunks <= kVMergeInLaunch ? d_cnt : nullptr;
  cudaError_t e = head_dim == 128
                      ? launch_vsum_hd<128>(grid, g, d_buf, layer, d_w, q_per_kv, seq_len, cp,
                                            n_chunks, d_out, d_part, merge_cnt, n_q, status, s)
                      : launch_vsum_hd<64>(grid, g, d_buf, layer, d_w, q_per_kv, seq_len, cp,
                                           n_chunks, d_out, d_part, merge_cnt, n_q, status, s);
  if (e != cudaSuccess || n_chunks <= kVMergeInLaunch) return e;
  const size_t n = (size_t)n_q * head_dim;
  vsum_combine_kernel<<<(int)((n + 255) / 256), 256, 0, s>>>(d_part, n_chunks, n, d_out);
  return cudaGetLastError();
}

}  // namespace eakv

using namespace eakv;

// Shape checks shared by the two-call entry points. The reference does no
// validation (src/attention.c); here a call it would run out of bounds or
// through the wrong kernel is refused.
static int attn_check(const eakv_cache_t *c, const void *in, const void *out, int layer,
                      int n_q, int n_kv, const char *who) {
  if (!c || !in || !out) {
    set_error(EAKV_ERR_INVALID, "%s: NULL argument", who);
    return EAKV_ERR_INVALID;
  }
  if (layer < 0 || layer >= c->n_layers) {
    set_error(EAKV_ERR_INVALID, "%s: layer %d out of range", who, layer);
    return EAKV_ERR_INVALID;
  }
  if (c->head_dim != 64 && c->head_dim != 128) {
    set_error(EAKV_ERR_INVALID, "%s: head_dim %d unsupported (64 or 128)", who, c->head_dim);
    return EAKV_ERR_INVALID;
  }
  if (n_kv <= 0 || n_kv > c->n_kv_heads || n_q < n_kv || n_q % n_kv != 0) {
    set_error(EAKV_ERR_INVALID, "%s: bad head counts n_q=%d n_kv=%d (cache has %d)", who, n_q,
              n_kv, c->n_kv_heads);
    return EAKV_ERR_INVALID;
  }
  return EAKV_OK;
}

static void fill_nan_host(float *p, size_t n) {
  if (!p) return;
  for (size_t i = 0; i < n; i++) p[i] = NAN;
}

extern "C" {

int eakv_attention_scores_device(const eakv_cache_t *c, const float *d_q, int layer, int n_q,
                                 int n_kv, float *d_scores) {
  clear_error();
  int rc = attn_check(c, d_q, d_scores, layer, n_q, n_kv, "attention_scores");
  if (rc) return rc;
  DeviceGuard g(c->device);
  const float rsqrt_d = 1.0f / sqrtf((float)c->head_dim);
  return check_cuda(launch_scores(c->geom, c->d_buf, layer, d_q, n_q, n_kv, c->seq_len,
                                  rsqrt_d, d_scores, c->stream),
                    "attention_scores");
}

void eakv_attention_scores(const eakv_cache_t *c, const float *queries, int layer, int n_q,
                           int n_kv, float *scores_out) {
  clear_error();
  if (attn_check(c, queries, scores_out, layer, n_q, n_kv, "attention_scores")) {
    if (c && scores_out && n_q > 0) fill_nan_host(scores_out, (size_t)n_q * c->seq_len);
    return;
  }
  if (c->seq_len == 0) return;
  DeviceGuard g(c->device);
  size_t nq = (size_t)n_q * c->head_dim, ns = (size_t)n_q * c->seq_len;
  float *d_q = (float *)cache_scratch(c, (nq + ns) * sizeof(float) + 256);
  if (!d_q) {
    fill_nan_host(scores_out, ns);
    return;
  }
  float *d_s = d_q + ((nq + 63) / 64) * 64;
  const float rsqrt_d = 1.0f / sqrtf((float)c->head_dim);
  if (check_cuda(cudaMemcpyAsync(d_q, queries, nq * sizeof(float), cudaMemcpyHostToDevice,
                                 c->stream), "attention_scores: copy") ||
      check_cuda(launch_scores(c->geom, c->d_buf, layer, d_q, n_q, n_kv, c->seq_len, rsqrt_d,
                               d_s, c->stream), "attention_scores") ||
      check_cuda(cudaMemcpyAsync(scores_out, d_s, ns * sizeof(float), cudaMemcpyDeviceToHost,
                                 c->stream), "attention_scores: copy") ||
      check_cuda(cudaStreamSynchronize(c->stream), "attention_scores")) {
    fill_nan_host(scores_out, ns);
  }
}

int eakv_attention_output_device(const eakv_cache_t *c, const float *d_w, int layer, int n_q,
                                 int n_kv, float *d_out) {
  clear_error();
  int rc = attn_check(c, d_w, d_out, layer, n_q, n_kv, "attention_output");
  if (rc) return rc;
  DeviceGuard g(c->device);
  size_t pf = vsum_scratch_floats(c->geom, n_q, n_kv, c->seq_len);
  float *d_part = nullptr;
  unsigned *d_cnt = nullptr;
  if (pf) {
    void *p = nullptr;
    rc = cache_workspace(c, vsum_counters(n_q, n_kv, c->seq_len), pf * sizeof(float), &d_cnt, &p);
    if (rc) return rc;
    d_part = (float *)p;
  }
  return check_cuda(launch_vsum(c->geom, c->d_buf, layer, d_w, n_q, n_kv, c->seq_len, d_out,
                                d_part, pf, d_cnt, c->stream),
                    "attention_output");
}

void eakv_attention_output(const eakv_cache_t *c, const float *weights, int layer, int n_q,
                           int n_kv, float *output_out) {
  clear_error();
  if (attn_check(c, weights, output_out, layer, n_q, n_kv, "attention_output")) {
    if (c && output_out && n_q > 0) fill_nan_host(output_out, (size_t)n_q * c->head_dim);
    return;
  }
  DeviceGuard g(c->device);
  size_t nw = (size_t)n_q * c->seq_len, no = (size_t)n_q * c->head_dim;
  size_t pf = vsum_scratch_floats(c->geom, n_q, n_kv, c->seq_len);
  size_t nw_pad = (nw + 63) / 64 * 64, no_pad = (no + 63) / 64 * 64;
  void *p = nullptr;
  unsigned *d_cnt = nullptr;
  if (cache_workspace(c, vsum_counters(n_q, n_kv, c->seq_len),
                      (nw_pad + no_pad + pf) * sizeof(float), &d_cnt, &p) != EAKV_OK) {
    fill_nan_host(output_out, no);
    return;
  }
  float *d_w = (float *)p;
  float *d_o = d_w + nw_pad;
  float *d_part = pf ? d_o + no_pad : nullptr;
  if ((nw && check_cuda(cudaMemcpyAsync(d_w, weights, nw * sizeof(float),
                                        cudaMemcpyHostToDevice, c->stream),
                        "attention_output: copy")) ||
      check_cuda(launch_vsum(c->geom, c->d_buf, layer, d_w, n_q, n_kv, c->seq_len, d_o, d_part,
                             pf, d_cnt, c->stream), "attention_output") ||
      check_cuda(cudaMemcpyAsync(output_out, d_o, no * sizeof(float), cudaMemcpyDeviceToHost,
                                 c->stream), "attention_output: copy") ||
      check_cuda(cudaStreamSynchronize(c->stream), "attention_output")) {
    fill_nan_host(output_out, no);
  }
}

}  // extern "C"
