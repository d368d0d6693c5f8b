// decode_mma.cu - fused softmax attention over the Q4 cache on the tensor
// cores (mma.sync), for any number of query heads per KV head (MHA
// included): a CTA serves up to 8 query heads of one KV head, with its
// fragments laid out for 4 or 8.
//
// Same work decomposition, page pipeline and merge as the CUDA-core kernel
// in decode.cu; what changes is how the two contractions of a position
// block are evaluated. Per warp and 16-position step:
//
//   S[(head, limb)][pos] = Qdigits[16 x 32 dims] * Knib[32 dims x 8 pos]   (int8, per group)
//   O[dims][(head, limb)] += Vnib[16 dims x 16 pos] * P'[16 pos x (head, limb)]   (f16)
//
// Scores (integer tensor cores, mma m16n8k32 s8 x u8 -> s32):
// * Each query is written as a fixed-point integer x = rn(q 2^E) with
//   |x| <= 2^30 (E per head from its largest |q|), split into four signed
//   base-256 digits x = d0 + 2^8 d1 + 2^16 d2 + 2^24 d3 (each in [-128, 127]).
//   The (head, digit) pairs are the 16 rows of an m-tile.
// * The K nibbles enter the tensor core as they are stored: a 32-bit word of
//   a position's row holds four bytes; w & 0x0F0F0F0F are four low nibbles
//   (dims b..b+3) and w & 0xF0F0F0F0 four high nibbles times 16 (dims
//   b+32..b+35), whose queries are taken as rn(q 2^(E-4)) instead. One
//   logic op per four nibbles, no conversion.
// * Every product and sum is exact in the s32 accumulator (|digit * nibble|
//   sums over a 64-dim group stay below 2^21). A thread holds two digit rows
//   of one head; it joins them exactly in integers (t = D_l + 256 D_l+1 <
//   2^29), converts once, and (for 4 heads per CTA) adds the partner
//   thread's other two digits with one shuffle.
// * Each 64-dim group has its own accumulator, so the group's scale and
//   bias apply in f32 afterwards: score = s_k * dot + b_k * sum(q).
//
// Outputs (f16 tensor cores, mma m16n8k16 f16 -> f32):
// * The V nibbles (0..15) are exact in f16. They are turned into f16 pairs
//   in registers with one mask+or and one f16 subtract each: placing a
//   nibble in the low mantissa bits of 1024.0 (0x6400) and subtracting 1024
//   gives it exactly; a high nibble is taken in place (bits 4..7), i.e.
//   times 16, and the 1/16 is applied to the output row. The nibble bytes
//   reach the registers by one transposed ldmatrix per group and step,
//   which already pairs two positions' bytes in one register as the f16x2
//   fragment wants.
// * P' = p * s_v (a probability times the V scale) is split into two f16
//   limbs, hi = f16(x) and lo = f16(x - hi), which carry ~22 bits; the
//   tensor core accumulates in f32. P' is prescaled by 2^-E with E the
//   largest exponent of any V scale of the (layer, head) (kept by the
//   cache), so it stays inside the f16 range. The bias part p * b_v is
//   accumulated in f32 outside the tensor core.
// * Online softmax in base 2 with a lazy maximum: the running max moves only
//   when a block's max exceeds it by more than 8, so probabilities stay in
//   [0, 256] and rescaling the accumulators is rare.
#include <cuda_fp16.h>
#include <math.h>

#include <atomic>

#include <type_traits>

#include "internal.cuh"
#include "pipeline.cuh"
#include "decode_common.cuh"

namespace eakv {
namespace {

// RH: query heads a CTA's fragments are laid out for (4 or 8); a CTA
// serves gh <= RH live heads (the planner's choice), the rest of its rows
// are zero and their results are discarded.
template <int HD, int RH>
struct MCfg {
  static constexpr int NG = HD / 64;                        // groups per position
  static constexpr int KSG = 2;                             // score k-steps (32 dims) per group
  static constexpr int KMT = RH / 4;                        // score m-tiles (4 heads x 4 digits)
  static constexpr int VNT = RH == 8 ? 2 : 1;               // P' n-tiles (one per limb)
  static constexpr int VMT = 4 * NG;                        // output m-tiles of 16 dims
  static constexpr int NW = 4;                              // warps
  // warps per page: each warp takes whole pages (4 steps of 16 positions),
  // the 4 warps of a CTA pages i, i+1, i+2, i+3 in turn
  static constexpr int WPP = 1;
  static constexpr int THREADS = NW * 32;
  // unroll the steps of a whole page (registers allow it except at 8 heads, d128)
  static constexpr bool UNROLL = !(HD == 128 && RH == 8);
  // CTAs per SM the register budget is cut for (128 registers at 4)
  static constexpr int MINB = (HD == 128 && RH == 8) ? 3 : 4;
  static constexpr int NIB = kPagePositions * NG * 32;
  static constexpr int PB = kPagePositions * NG * 40;
  // pages in flight: one per warp plus spares, as many as the shared memory
  // of the CTAs that fit an SM allows (4 CTAs at 4 heads, 3 at 8)
  static constexpr int NSTAGE = HD == 128 ? (RH == 8 ? 6 : 5) : 8;
  static constexpr int STAGE_BYTES = 2 * PB;
  static constexpr int RING = NSTAGE * STAGE_BYTES;
  static constexpr int MERGE_BYTES = NW * RH * (HD + 2) * 4;
  static constexpr int MAIN = (RING > MERGE_BYTES ? RING : MERGE_BYTES);
  static constexpr int QOFF = MAIN + 2 * NSTAGE * 8;          // scaled queries [RH][HD]
  static constexpr int STATOFF = QOFF + RH * HD * 4;           // [RH] max|q|, [RH][NG] sums
  static constexpr int SMEM = STATOFF + RH * (1 + NG) * 4;
  static_assert(RH == 4 || RH == 8, "fragments are laid out for 4 or 8 query heads");
  static_assert(NW % WPP == 0 && kPagePositions % (16 * WPP) == 0, "page split");
};

constexpr uint32_t kMagic = 0x64006400u;   // f16x2 (1024, 1024)

__device__ __forceinline__ uint32_t f16x2_sub1024(uint32_t x) {
  uint32_t r;
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(x), "r"(kMagic));
  return r;
}

// (w & mask) | magic as one three-input logic op; written out because the
// compiler otherwise splits it in two when both constants are immediates.
__device__ __forceinline__ uint32_t and_or(uint32_t w, uint32_t mask, uint32_t magic) {
  uint32_t r;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r) : "r"(w), "r"(mask), "r"(magic));
  return r;
}

// f16x2 of the nibbles selected by `mask` (0x000F000F: low nibbles of bytes
// 0 and 2, value n; 0x00F000F0: high nibbles, value 16 n).
__device__ __forceinline__ uint32_t nib_pair(uint32_t w, uint32_t mask) {
  return f16x2_sub1024(and_or(w, mask, kMagic));
}

// x = hi + lo in two f16 limbs: limb 0 = f16(x), limb 1 = f16(x - f16(x)).
__device__ __forceinline__ void split2(float x0, float x1, uint32_t &h, uint32_t &l) {
  __half2 hh = __floats2half2_rn(x0, x1);
  float2 back = __half22float2(hh);
  __half2 ll = __floats2half2_rn(x0 - back.x, x1 - back.y);
  h = *reinterpret_cast<uint32_t *>(&hh);
  l = *reinterpret_cast<uint32_t *>(&ll);
}

__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void imma16832(int (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                          uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.u8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// d = A * B with a zero accumulator given as an immediate (no registers
// zeroed first).
__device__ __forceinline__ void imma16832_z(int (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                            uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.u8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {0,0,0,0};"
      : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Four transposed 8x8 b16 tiles from shared memory: lane t gives the row
// address for row t % 8 of tile t / 8 (16-byte aligned) and receives, for
// each tile, column t / 4 of rows 2 (t % 4) and 2 (t % 4) + 1 (low, high
// half of the register).
__device__ __forceinline__ void ldsm_x4_trans(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

// Signed base-256 digit l (0..3) of x, |x| <= 2^30: x = sum_l digit_l 2^(8l)
// with every digit in [-128, 127].
__device__ __forceinline__ int digit(int x, int l) {
  int d = 0;
#pragma unroll
  for (int k = 0; k < 4; k++) {
    d = (int)(int8_t)(x & 0xFF);
    if (k == l) break;
    x = (x - d) >> 8;
  }
  return d;
}

template <int HD, int RH>
__global__ void __launch_bounds__(MCfg<HD, RH>::THREADS, MCfg<HD, RH>::MINB)
decode_mma_kernel(const __grid_constant__ DecodeArgs a, const __grid_constant__ DecodeBatch batch) {
  using C = MCfg<HD, RH>;
  constexpr int NG = C::NG;
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + C::MAIN);
  float *q_s = reinterpret_cast<float *>(smem + C::QOFF);
  float *stat_s = reinterpret_cast<float *>(smem + C::STATOFF);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, c = lane & 3;
  const int G = a.n_q_heads / a.geom.n_heads;
  const int gh = a.cta_heads;   // live query heads of this CTA (<= RH)
  const int nhg = G / gh;
  if (!launch_ok(a) || gh < 1 || gh > RH || G % gh != 0) return;
  const Item it = decode_item(a, batch, nhg);
  if (!item_ok(a, it, it.h * G + it.hg * gh, gh)) {
    if (a.n_splits > 1 && !a.sep_merge) arrive_last(a);   // keeps the item's split counter in step
    return;
  }
  const size_t kv_stride = (size_t)a.geom.n_heads * a.geom.n_pages;
  const uint8_t *kpages = batch.base[it.b] + page_index(a.geom, it.layer, 0, it.h, 0) * C::PB;
  const uint8_t *vpages = kpages + kv_stride * C::PB;

  // The set-up's own global loads go out first (this CTA's queries and the
  // V-exponent entry), so that their latency overlaps the barrier set-up and
  // the first page requests: with few CTAs per SM the set-up is on the
  // launch's critical path.
  const int qh0 = it.h * G + it.hg * gh;
  const float *qb = a.q + ((size_t)(it.b * a.n_layers + it.lrow) * a.n_q_heads + qh0) * HD;
  constexpr int QPT = (RH * HD + C::THREADS - 1) / C::THREADS;   // query elements per thread
  float qv[QPT];
#pragma unroll
  for (int k = 0; k < QPT; k++) {
    const int i = threadIdx.x + k * C::THREADS;
    qv[k] = i < gh * HD ? __ldg(qb + i) : 0.0f;
  }
  const int vexp_raw = __ldg(vexp_table(batch.base[it.b], a.geom) + it.layer * a.geom.n_heads + it.h);

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::NSTAGE; s++) {
      mbar_init(smem_u32(&bars[s]), 1);                               // stage filled
      reinterpret_cast<int *>(&bars[C::NSTAGE])[s] = 0;               // release count
      reinterpret_cast<int *>(&bars[C::NSTAGE])[C::NSTAGE + s] = -1;  // last page requested
    }
    fence_mbar_init();
  }
  __syncthreads();
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

  // ---- per-thread query fragments -----------------------------------------
  // Score rows: row g of m-tile mt is (head h_mine, digit l_row + 2 mt),
  // row g+8 the next digit. With 4 heads, lanes g and g^4 share a head
  // (digits 0,1 and 2,3); with 8, m-tiles 0 and 1 give lane g all four.
  const int h_mine = (RH == 4) ? (g & 3) : g;
  const int l_row = (RH == 4) ? 2 * (g >> 2) : 0;
  const float qscale = rsqrtf((float)HD) * kLog2e;
  // stage the scaled query block; one warp per head computes max|q| and
  // the per-group sums (for the bias term)
  // (heads gh..RH-1 are idle: zero queries, results never written)
#pragma unroll
  for (int k = 0; k < QPT; k++) {
    const int i = threadIdx.x + k * C::THREADS;
    if (i < RH * HD) q_s[i] = qv[k] * qscale;
  }
  __syncthreads();
  for (int h = warp; h < RH; h += C::NW) {
    float mx = 0.0f;
    for (int d = lane; d < HD; d += 32) mx = fmaxf(mx, fabsf(q_s[h * HD + d]));
#pragma unroll
    for (int gg = 0; gg < NG; gg++) {
      float sm = q_s[h * HD + 64 * gg + lane] + q_s[h * HD + 64 * gg + 32 + lane];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) sm += __shfl_xor_sync(0xffffffffu, sm, o);
      if (lane == 0) stat_s[RH + h * NG + gg] = sm;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if (lane == 0) stat_s[h] = mx;
  }
  __syncthreads();
  // fixed point: x = rn(q 2^E) with |x| <= 2^30; E is capped at 126 so that
  // 2^-E stays a normal float (queries below 2^-96 lose low bits only)
  const float hmax = stat_s[h_mine];
  int qexp = 0;
  frexpf(hmax > 0.0f && hmax <= 3.0e38f ? hmax : 1.0f, &qexp);   // hmax in [2^(qexp-1), 2^qexp)
  const int qe = min(30 - qexp, 126);
  const float up_lo = __uint_as_float((uint32_t)(127 + qe) << 23);       // 2^E
  const float up_hi = __uint_as_float((uint32_t)(127 + qe - 4) << 23);   // 2^(E-4)
  // weight of this lane's joined digits: 2^(8 l_row - E); a query with an
  // inf or NaN element turns every score of its head into NaN
  const float w_row = (hmax <= 3.0e38f) ? __uint_as_float((uint32_t)(127 + 8 * l_row - qe) << 23)
                                        : __uint_as_float(0x7fc00000u);

  // A fragments: k-step ks of group gg, lane c holds dims 64 gg + 8c + 4ks + i
  // (low nibbles, bytes i of its K word) and the same + 32 (high nibbles)
  uint32_t aq[NG][C::KSG][C::KMT][4];
#pragma unroll
  for (int gg = 0; gg < NG; gg++)
#pragma unroll
    for (int ks = 0; ks < C::KSG; ks++)
#pragma unroll
      for (int mt = 0; mt < C::KMT; mt++) {
        const int l0 = l_row + 2 * mt;
        uint32_t r[4] = {0u, 0u, 0u, 0u};
#pragma unroll
        for (int i = 0; i < 4; i++) {
          const int d = 64 * gg + 8 * c + 4 * ks + i;
          const int xl = __float2int_rn(q_s[h_mine * HD + d] * up_lo);
          const int xh = __float2int_rn(q_s[h_mine * HD + d + 32] * up_hi);
          r[0] |= (uint32_t)(digit(xl, l0) & 0xFF) << (8 * i);       // row g,   low dims
          r[1] |= (uint32_t)(digit(xl, l0 + 1) & 0xFF) << (8 * i);   // row g+8, low dims
          r[2] |= (uint32_t)(digit(xh, l0) & 0xFF) << (8 * i);       // row g,   high dims
          r[3] |= (uint32_t)(digit(xh, l0 + 1) & 0xFF) << (8 * i);   // row g+8, high dims
        }
#pragma unroll
        for (int k = 0; k < 4; k++) aq[gg][ks][mt][k] = r[k];
      }
  // per-group query sums for the bias term; with 4 heads only the lane
  // holding digits 0,1 adds it (its partner's share arrives by shuffle)
  float qsum[NG];
#pragma unroll
  for (int gg = 0; gg < NG; gg++)
    qsum[gg] = (RH == 4 && l_row) ? 0.0f : stat_s[RH + h_mine * NG + gg];

  // ---- accumulators -----------------------------------------------------------
  float dv[C::VMT][C::VNT][4];
#pragma unroll
  for (int i = 0; i < C::VMT; i++)
#pragma unroll
    for (int n = 0; n < C::VNT; n++)
#pragma unroll
      for (int r = 0; r < 4; r++) dv[i][n][r] = 0.0f;
  float m_run = -INFINITY, m_eff = 0.0f;   // m_eff: m_run, or 0 while it is -inf
  float2 l2 = make_float2(0.0f, 0.0f);       // sum of p, two running halves
  float pb[NG];
#pragma unroll
  for (int gg = 0; gg < NG; gg++) pb[gg] = 0.0f;
  // Every V scale of this (layer, head) is below 2^(vexp - 126) (the cache's
  // exponent table), so P' = p * s * 2^(127 - vexp) < 2 p <= 512 stays in f16.
  const int vexp = min(max(vexp_raw, 1), 253);
  const float fs = __uint_as_float((uint32_t)(254 - vexp) << 23);   // 2^(127 - vexp)
  // head of each P'/output column this thread holds: n = 2c + e
  int hcol[2];
#pragma unroll
  for (int e = 0; e < 2; e++) hcol[e] = (C::VNT == 1) ? ((2 * c + e) % RH) : (2 * c + e);
  const int my_limb = (C::VNT == 1) ? (g >> 2) : 0;

  // One 16-position step of a staged page (this warp's quarter of it).
  // FULL: every position of the page is attended (no per-position masks).
  auto page_body = [&](auto full_tag, const uint8_t *ks_, int page_pos0, int p0) {
    constexpr bool FULL = decltype(full_tag)::value;
    const uint8_t *vs_ = ks_ + C::PB;

    // positions of this thread's score/probability slots: 2c, 2c+1, 2c+8, 2c+9
    int tpos[4];
    bool tval[4];
#pragma unroll
    for (int j = 0; j < 4; j++) {
      tpos[j] = p0 + 2 * c + (j & 1) + (j >> 1) * 8;
      const int pos = page_pos0 + tpos[j];
      tval[j] = FULL || (pos >= it.r0 && pos < it.r1);
    }
    // (scale, bias) of K and V for the four positions, every group
    float sk[4][NG], bk[4][NG], sv[4][NG], bv[4][NG];
#pragma unroll
    for (int j = 0; j < 4; j++) {
      if (NG == 2) {
        const float4 k4 = *reinterpret_cast<const float4 *>(ks_ + C::NIB + tpos[j] * 16);
        const float4 v4 = *reinterpret_cast<const float4 *>(vs_ + C::NIB + tpos[j] * 16);
        sk[j][0] = k4.x; bk[j][0] = k4.y; sk[j][NG - 1] = k4.z; bk[j][NG - 1] = k4.w;
        sv[j][0] = v4.x; bv[j][0] = v4.y; sv[j][NG - 1] = v4.z; bv[j][NG - 1] = v4.w;
      } else {
        const float2 k2 = *reinterpret_cast<const float2 *>(ks_ + C::NIB + tpos[j] * 8);
        const float2 v2 = *reinterpret_cast<const float2 *>(vs_ + C::NIB + tpos[j] * 8);
        sk[j][0] = k2.x; bk[j][0] = k2.y;
        sv[j][0] = v2.x; bv[j][0] = v2.y;
      }
      if (!FULL && !tval[j]) {
#pragma unroll
        for (int gg = 0; gg < NG; gg++) sv[j][gg] = bv[j][gg] = 0.0f;
      }
    }

    // ---- scores of the two 8-position tiles -------------------------------
    float sc[4];
#pragma unroll
    for (int tile = 0; tile < 2; tile++) {
      int dk[NG][C::KMT][4];
      // B fragments: lane (g, c) takes bytes 8c..8c+7 of position g's group row
      const uint8_t *row = ks_ + (p0 + 8 * tile + g) * (HD / 2) + 8 * c;
#pragma unroll
      for (int gg = 0; gg < NG; gg++) {
        const uint2 wv = *reinterpret_cast<const uint2 *>(row + 32 * gg);
#pragma unroll
        for (int ks = 0; ks < C::KSG; ks++) {
          const uint32_t w = ks ? wv.y : wv.x;
          const uint32_t b0 = w & 0x0F0F0F0Fu;   // low nibbles
          const uint32_t b1 = w & 0xF0F0F0F0u;   // high nibbles x16
#pragma unroll
          for (int mt = 0; mt < C::KMT; mt++) {
            if (ks == 0) imma16832_z(dk[gg][mt], aq[gg][ks][mt], b0, b1);
            else imma16832(dk[gg][mt], aq[gg][ks][mt], b0, b1);
          }
        }
      }
#pragma unroll
      for (int e = 0; e < 2; e++) {
        const int j = 2 * tile + e;
        float part = 0.0f;
#pragma unroll
        for (int gg = 0; gg < NG; gg++) {
          // join the lane's digit rows exactly, then convert once
          float u = (float)(dk[gg][0][e] + 256 * dk[gg][0][2 + e]);
          if (C::KMT == 2) u = fmaf((float)(dk[gg][1][e] + 256 * dk[gg][1][2 + e]), 65536.0f, u);
          part = fmaf(u, sk[j][gg], part);
        }
        part *= w_row;
#pragma unroll
        for (int gg = 0; gg < NG; gg++) part = fmaf(bk[j][gg], qsum[gg], part);
        if (RH == 4) part += __shfl_xor_sync(0xffffffffu, part, 16);
        sc[j] = (FULL || tval[j]) ? part : -INFINITY;
      }
    }

    // ---- online softmax (base 2, lazy max) ----------------------------------
    // The row's running max moves only when a score passes it by more than 8;
    // each lane tests its own four scores, and only then (rarely) is the
    // row's max formed across the quad.
    const float lmax = fmaxf(fmaxf(sc[0], sc[1]), fmaxf(sc[2], sc[3]));
    if (__any_sync(0xffffffffu, lmax > m_run + 8.0f)) {
      float tmax = fmaxf(lmax, __shfl_xor_sync(0xffffffffu, lmax, 1));
      tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, 2));
      const bool need = tmax > m_run + 8.0f;
      const float m_new = need ? tmax : m_run;
      const float alpha = need ? ex2(m_run - m_new) : 1.0f;   // exp2(-inf) = 0
      m_run = m_new;
      m_eff = m_run == -INFINITY ? 0.0f : m_run;
      l2 = __fmul2_rn(l2, make_float2(alpha, alpha));
#pragma unroll
      for (int gg = 0; gg < NG; gg++) pb[gg] *= alpha;
#pragma unroll
      for (int e = 0; e < 2; e++) {
        const float ac = __shfl_sync(0xffffffffu, alpha, 4 * hcol[e]);
#pragma unroll
        for (int mv = 0; mv < C::VMT; mv++)
#pragma unroll
          for (int n = 0; n < C::VNT; n++) {
            dv[mv][n][e] *= ac;
            dv[mv][n][2 + e] *= ac;
          }
      }
    }
    float p[4], pf[4];
#pragma unroll
    for (int j = 0; j < 4; j++) {
      p[j] = ex2(sc[j] - m_eff);
      pf[j] = p[j] * fs;   // exact: fs is a power of two
    }
    l2 = __fadd2_rn(l2, make_float2(p[0], p[1]));
    l2 = __fadd2_rn(l2, make_float2(p[2], p[3]));

    // ---- P' fragments and the V contraction, group by group ------------------
#pragma unroll
    for (int gg = 0; gg < NG; gg++) {
      float ps[4];
#pragma unroll
      for (int j = 0; j < 4; j++) {
        ps[j] = pf[j] * sv[j][gg];
        pb[gg] = fmaf(p[j], bv[j][gg], pb[gg]);
      }
      uint32_t b0[C::VNT], b1[C::VNT];   // positions (2c, 2c+1) and (2c+8, 2c+9)
      if (C::VNT == 1) {
        uint32_t h0, l0, h1, l1;   // this lane's limb of each pair
        split2(ps[0], ps[1], h0, l0);
        split2(ps[2], ps[3], h1, l1);
        b0[0] = my_limb ? l0 : h0;
        b1[0] = my_limb ? l1 : h1;
      } else {
        split2(ps[0], ps[1], b0[0], b0[C::VNT - 1]);
        split2(ps[2], ps[3], b1[0], b1[C::VNT - 1]);
      }
      // V nibbles of the step's 16 positions, as four transposed 8x8 b16
      // tiles: tile 2w + blk holds positions p0 + 8 blk .. + 7 (rows) and
      // bytes 16w .. 16w + 15 of the group (8 columns of two bytes). Lane
      // (g, c) receives bytes 16w + 2g, 16w + 2g + 1 of positions 2c, 2c+1
      // (blk 0) and 2c+8, 2c+9 (blk 1).
      uint32_t x[4];
      {
        const int t = lane >> 3, r = lane & 7;
        ldsm_x4_trans(x, smem_u32(vs_ + (p0 + 8 * (t & 1) + r) * (HD / 2) + 32 * gg + 16 * (t >> 1)));
      }
#pragma unroll
      for (int j = 0; j < 4; j++) {   // byte 16 (j/2) + 2g + (j%2) -> output m-tile 4*gg + j
        const uint32_t xa = x[2 * (j >> 1)], xb = x[2 * (j >> 1) + 1];
        const uint32_t ya = (j & 1) ? (xa >> 8) : xa, yb = (j & 1) ? (xb >> 8) : xb;
        const uint32_t a0 = nib_pair(ya, 0x000F000Fu);   // row g: low nibble, positions 2c, 2c+1
        const uint32_t a1 = nib_pair(ya, 0x00F000F0u);   // row g+8: high nibble x16
        const uint32_t a2 = nib_pair(yb, 0x000F000Fu);   // positions 2c+8, 2c+9
        const uint32_t a3 = nib_pair(yb, 0x00F000F0u);
#pragma unroll
        for (int n = 0; n < C::VNT; n++) mma16816(dv[4 * gg + j][n], a0, a1, a2, a3, b0[n], b1[n]);
      }
    }
  };

  // WPP warps share a page, each taking 64 / WPP positions as 16-position
  // steps; the NW / WPP warp groups take pages in turn, so the per-page
  // costs (wait, release, loop) are paid once per 64 / WPP positions. Page
  // i lives in stage i % NSTAGE; its consumers release it and the last of
  // them requests page i + NSTAGE into it.
  bool ok = true;
  const int wgrp = warp / C::WPP, wsub = warp % C::WPP;
  for (int i = wgrp; i < it.npages; i += C::NW / C::WPP) {
    const int st = i % C::NSTAGE;
    if (!ok || !wait_requested(&last_req[st], i, a.wait_budget) ||
        !mbar_wait(smem_u32(&bars[st]), (i / C::NSTAGE) & 1, a.wait_budget)) {
      report(a, kStatusWaitTimeout);
      ok = false;
      break;
    }
    const uint8_t *ks_ = smem + st * C::STAGE_BYTES;
    const int page_pos0 = (it.pg0 + i) * kPagePositions;
    const bool full = page_pos0 >= it.r0 && page_pos0 + kPagePositions <= it.r1;
    constexpr int STEPS = kPagePositions / (16 * C::WPP);
    if (full) {
      // a whole page: its steps unrolled, so their shared-memory addresses
      // are immediate offsets from the stage (not for the 8-head d128
      // kernel, which would spill)
      if constexpr (C::UNROLL) {
#pragma unroll
        for (int s2 = 0; s2 < STEPS; s2++)
          page_body(std::true_type{}, ks_, page_pos0, (kPagePositions / C::WPP) * wsub + 16 * s2);
      } else {
#pragma unroll 1
        for (int s2 = 0; s2 < STEPS; s2++)
          page_body(std::true_type{}, ks_, page_pos0, (kPagePositions / C::WPP) * wsub + 16 * s2);
      }
    } else {
#pragma unroll 1
      for (int s2 = 0; s2 < STEPS; s2++)
        page_body(std::false_type{}, ks_, page_pos0, (kPagePositions / C::WPP) * wsub + 16 * s2);
    }
    __syncwarp();
    // the last warp of the group to finish with this stage refills it with
    // page i+NSTAGE
    if (lane == 0 && stage_release_last(reinterpret_cast<int *>(&bars[C::NSTAGE]) + st, C::WPP) &&
        i + C::NSTAGE < it.npages)
      issue(i + C::NSTAGE);
  }
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

  // ---- per-warp totals --------------------------------------------------------
  float l_run = l2.x + l2.y;
  l_run += __shfl_xor_sync(0xffffffffu, l_run, 1);
  l_run += __shfl_xor_sync(0xffffffffu, l_run, 2);
#pragma unroll
  for (int gg = 0; gg < NG; gg++) {
    pb[gg] += __shfl_xor_sync(0xffffffffu, pb[gg], 1);
    pb[gg] += __shfl_xor_sync(0xffffffffu, pb[gg], 2);
  }
  // combine the two limbs of every output column
#pragma unroll
  for (int mv = 0; mv < C::VMT; mv++)
#pragma unroll
    for (int r = 0; r < 4; r++) {
      if (C::VNT == 1) dv[mv][0][r] += __shfl_xor_sync(0xffffffffu, dv[mv][0][r], 2);
      else dv[mv][0][r] += dv[mv][C::VNT - 1][r];
    }
  float pbc[2][NG];   // bias accumulators of this thread's two column heads
#pragma unroll
  for (int e = 0; e < 2; e++)
#pragma unroll
    for (int gg = 0; gg < NG; gg++) pbc[e][gg] = __shfl_sync(0xffffffffu, pb[gg], 4 * hcol[e]);

  __syncthreads();   // ring no longer read; reuse it for the merge
  float *mw = reinterpret_cast<float *>(smem);   // [NW][RH]
  float *lw = mw + C::NW * RH;                    // [NW][RH]
  float *ow = lw + C::NW * RH;                    // [NW][RH][HD]
  if (c == 0 && g < RH) {
    // lane (g, 0) scores head g (g < RH rows carry every head once)
    mw[warp * RH + h_mine] = m_run;
    lw[warp * RH + h_mine] = l_run;
  }
  // after the limb sum, lanes c and c^2 hold the same columns (one limb pair)
  const bool writer = (C::VNT == 1) ? (c < 2) : true;
  if (writer) {
#pragma unroll
    for (int mv = 0; mv < C::VMT; mv++) {
      const int gg = mv >> 2, j = mv & 3;
      // undo the 2^(127 - vexp) applied to P': multiply by 2^(vexp - 127)
      const float vs = __uint_as_float((uint32_t)vexp << 23);
      const int dlo = 64 * gg + 16 * (j >> 1) + 2 * g + (j & 1), dhi = dlo + 32;
#pragma unroll
      for (int e = 0; e < 2; e++) {
        const int h = hcol[e];
        ow[(warp * RH + h) * HD + dlo] = fmaf(dv[mv][0][e], vs, pbc[e][gg]);
        ow[(warp * RH + h) * HD + dhi] = fmaf(dv[mv][0][2 + e], vs * (1.0f / 16.0f), pbc[e][gg]);
      }
    }
  }
  __syncthreads();
  const size_t row0 = (size_t)(it.b * a.n_layers + it.lrow) * a.n_q_heads + qh0;
  for (int idx = threadIdx.x; idx < gh * HD; idx += C::THREADS) {
    const int h = idx / HD, d = idx - h * HD;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < C::NW; w++) M = fmaxf(M, mw[w * RH + h]);
    float O = 0.0f, L = 0.0f;
    if (M != -INFINITY) {
#pragma unroll
      for (int w = 0; w < C::NW; w++) {
        const float mwv = mw[w * RH + h];
        const float f = mwv == -INFINITY ? 0.0f : ex2(mwv - M);
        O = fmaf(f, ow[(w * RH + h) * HD + d], O);
        L = fmaf(f, lw[w * RH + h], L);
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
  // the item's last split to finish merges all of them (the ring is free)
  if (a.n_splits > 1 && !a.sep_merge && arrive_last(a))
    merge_splits<HD, RH, C::THREADS>(a, row0, gh, reinterpret_cast<float *>(smem));
}

template <int HD, int RH>
int launch_one(const DecodeArgs &a, const DecodeBatch &b, int n_blocks, cudaStream_t s) {
  using C = MCfg<HD, RH>;
  auto fn = decode_mma_kernel<HD, RH>;
  static std::atomic<unsigned long long> attr_done{0};   // one bit per device
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(attr_done.load(std::memory_order_acquire) >> (dev & 63) & 1)) {
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    if (e != cudaSuccess) return check_cuda(e, "decode_mma: smem attribute");
    attr_done.fetch_or(1ull << (dev & 63), std::memory_order_acq_rel);
  }
  fn<<<n_blocks, C::THREADS, C::SMEM, s>>>(a, b);
  return check_cuda(cudaGetLastError(), "decode_mma launch");
}

template <int HD, int RH>
int resident_one() {
  using C = MCfg<HD, RH>;
  // per device (resident CTAs per SM x SMs), filled on first use
  static std::atomic<int> cached[64];
  int dev = 0;
  cudaGetDevice(&dev);
  const int hit = cached[dev & 63].load(std::memory_order_relaxed);
  if (hit) return hit;
  cudaFuncSetAttribute(decode_mma_kernel<HD, RH>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                       C::SMEM);
  int per_sm = 1, sms = 148;
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, decode_mma_kernel<HD, RH>, C::THREADS,
                                                C::SMEM);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int r = (per_sm < 1 ? 1 : per_sm) * sms;
  cached[dev & 63].store(r, std::memory_order_relaxed);
  return r;
}

}  // namespace

int mma_heads_per_cta(int G, int head_dim) {
  if ((head_dim != 64 && head_dim != 128) || G <= 0) return 0;
  // every query head of a KV head in one CTA when they fit (the pages are
  // read once); otherwise the largest divisor of G up to 8
  for (int gh = G < 8 ? G : 8; gh > 1; gh--)
    if (G % gh == 0) return gh;
  return 1;
}

int mma_resident(int gh, int head_dim) {
  const bool r8 = gh > 4;
  if (head_dim == 128) return r8 ? resident_one<128, 8>() : resident_one<128, 4>();
  return r8 ? resident_one<64, 8>() : resident_one<64, 4>();
}

int mma_launch(int gh, const DecodeArgs &a0, const DecodeBatch &b, int n_blocks, cudaStream_t s) {
  DecodeArgs a = a0;
  a.cta_heads = gh;
  const bool r8 = gh > 4;
  if (a.head_dim == 128)
    return r8 ? launch_one<128, 8>(a, b, n_blocks, s) : launch_one<128, 4>(a, b, n_blocks, s);
  return r8 ? launch_one<64, 8>(a, b, n_blocks, s) : launch_one<64, 4>(a, b, n_blocks, s);
}

}  // namespace eakv
