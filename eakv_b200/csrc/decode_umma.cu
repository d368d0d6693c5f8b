// decode_umma.cu - fused softmax attention over the Q4 cache on the fifth-
// generation tensor cores (tcgen05.mma, kind::i8, s32 accumulators in tensor
// memory), head_dim 128, up to 8 query heads of one KV head per CTA.
//
// Work decomposition, split plan and split merge are those of the other
// decode kernels (decode_common.cuh). A CTA walks its split in blocks of 128
// positions (two pages); math thread t (warps 0-3) owns position t of the
// block (tensor-memory lane t). Per block:
//
//   S[pos][(g, h, d)]   = Kbytes[pos][32 g ..] * Qdigits[(h, d)][..]      (i8, TMEM A)
//   O[row][(g, h, d)]  += Vbytes[row][pos]    * Pdigits[pos][(g, h, d)]   (i8, SMEM A, B)
//
// Scores. The nibble byte b = lo + 16 hi of a 64-dim group's byte k holds
// dims k (lo) and k + 32 (hi). With x_lo = rn(q_lo 2^E) and x_hi =
// rn(q_hi 2^(E-4)) the integer dot product of the other tensor-core decode,
// sum x_lo lo + sum x_hi (16 hi), equals sum x_lo b + sum (x_hi - x_lo) (16 hi):
// the raw bytes need no conversion, only the high nibbles are masked out
// (w & 0xF0F0F0F0, one logic op per four bytes). Both operands go to tensor
// memory with tcgen05.st (lane = position); the query terms are four signed
// base-256 digits per head (rows (h, d) of a K-major shared-memory operand).
// Every product and sum is exact in s32; each thread joins its digits in
// integers and applies the group's scale and bias in f32 in the order of the
// other kernel, so the scores are the same bits.
//
// Outputs. The same trick with V as the A operand (rows = the 64 nibble
// bytes of a position, then their masked high nibbles; MN-major, positions
// along K) and the weights as B: P' = p * s_v * 2^(127 - vexp) * 2^29 < 2^32
// becomes an unsigned 32-bit fixed-point integer whose four bytes are its
// base-256 digits, i.e. the thread stores the integers as they are. The s32
// accumulators are exact (a digit column gains at most 255 * 255 per
// position, below 2^31 for 33025 positions; splits are at most 16384), so
// the only rounding on the V side is the fixed point of P', and the tensor
// core's accumulation adds none. Row k of the raw bytes minus its masked row
// gives dim k (lo), the masked row / 16 dim k + 32.
//
// Softmax: base 2 with a lazy maximum per head that is uniform over the CTA
// (a block whose score passes it by more than kLazy = 2 moves it, decided by
// one vote of the math warps), so p <= 4 and P' keeps 2^-30 of the block
// maximum. Fixed point is absolute, not relative: every weight below half a
// unit rounds to zero, so over 16384 positions up to 2^14 x 2^-30 of the
// weight mass can be lost; with the threshold of 8 that the f16 kernel uses
// (p <= 256, 2^-24) that was 1e-3 of the output at cfg5's length, above the
// parity bar. The integer accumulators cannot be rescaled, so a move first
// adds them into f32 per-thread accumulators (the first block, then rarely).
//
// Roles. Warps 0-3 (math), at block b: put the K rows of block b+1 into
// tensor memory and load the K rows of block b+2 into registers; read the
// scores of block b; put its V rows into their shared buffer b%3 and load
// the V rows of block b+1; run the softmax and write the P digits of block
// b. At 8 heads the K operands and scores are double-buffered and block
// b+1's K goes in before block b's scores are read; at 4 heads they are
// single and it goes in right after (128 tensor-memory columns, 3 CTAs per
// SM). The rows come from L2: the control thread prefetched their pages a
// few blocks ahead with cp.async.bulk.prefetch. Warp 4 (control, one thread)
// issues the MMAs: S(b) as soon as block b's K rows are in place (so it runs
// while the math warps finish block b-1), V(b) once block b's V rows and P
// digits are written. They meet on mbarriers only (math warps arrive once per warp, the
// MMAs complete on tcgen05.commit); every wait is bounded, suspends rather
// than spins, and a wait that runs out makes the whole CTA leave through the
// status word.
#include <math.h>

#include <atomic>

#include "internal.cuh"
#include "pipeline.cuh"
#include "decode_common.cuh"
#include "umma.cuh"

namespace eakv {
namespace {

using namespace umma;

template <int RH>
struct UCfg {
  static constexpr int HD = 128;
  static constexpr int NG = 2;                     // groups per position
  static constexpr int NM = 128;                   // math threads: one per position of a block
  static constexpr int NW = NM / 32;               // math warps
  static constexpr int NT = NM + 32;               // + the control warp
  static constexpr int HQ = RH / 2;                // head pairs
  static constexpr int BLK = 128;                  // positions per block (two pages)
  static constexpr int NS = 4 * RH;                // score columns per group: (head, digit)
  static constexpr int NV = 8 * RH;                // output columns: (group, head, digit)
  static constexpr int PROW = NV;                  // bytes of a P-digit row
  static constexpr uint32_t PLAYOUT = PROW == 64 ? kLayoutSW64 : kLayoutSW32;
  static constexpr int NBUF = 3;                   // shared V / P buffers
  // shared memory (offsets from a 1024-byte aligned base)
  static constexpr int OPV_BYTES = 2 * 128 * 64;   // raw rows, then masked rows
  static constexpr int OPV = 0;
  static constexpr int OPP = OPV + NBUF * OPV_BYTES;
  static constexpr int OPP_BYTES = BLK * PROW;
  static constexpr int QB1 = OPP + NBUF * OPP_BYTES;
  static constexpr int QB_BYTES = NS * 64;
  static constexpr int QB2 = QB1 + ((QB_BYTES + 1023) / 1024) * 1024;
  static constexpr int MISC = QB2 + ((QB_BYTES + 1023) / 1024) * 1024;
  // mbarriers: sdone[2], vdone[NBUF], drain, staged[2], pready
  static constexpr int BAR_S = MISC, BAR_V = MISC + 16, BAR_DRAIN = BAR_V + 8 * NBUF,
                       BAR_STAGED = BAR_DRAIN + 8, BAR_P = BAR_STAGED + 16;
  static constexpr int FLAGS = BAR_P + 16;         // [NBUF] accumulate flags of V(b)
  static constexpr int SLOT = FLAGS + 16;          // tensor-memory base address
  static constexpr int RED = SLOT + 16;            // [NW warps][RH] floats
  static constexpr int HCON = RED + ((NW * RH * 4 + 15) / 16) * 16;   // [RH] w, q sums g0, g1
  static constexpr int END = HCON + 3 * RH * 4;
  static_assert(BAR_S % 8 == 0 && BAR_P % 8 == 0 && SLOT % 8 == 0 && HCON % 16 == 0 &&
                FLAGS + 4 * NBUF <= SLOT, "shared-memory alignment (mbarriers, float2 reads)");
  static constexpr int SMEM = END + 1024;          // + alignment slack
  // set-up scratch inside the P buffers (free until block 0's digits)
  static constexpr int QS = OPP;                   // [RH][HD] scaled queries
  static constexpr int STAT = QS + RH * HD * 4;    // [RH] max|q|, [RH][NG] sums
  static_assert(STAT + RH * (1 + NG) * 4 <= OPP + NBUF * OPP_BYTES, "set-up scratch");
  // tensor memory columns
  // K operands (16 raw, 16 masked columns) and scores (2 NS columns) are
  // double-buffered at 8 heads (the next block's score MMAs are issued before
  // this block's scores are read) and single at 4 heads, which then fits 128
  // columns and three CTAs per SM (the next block is staged once this block's
  // scores are in registers)
  static constexpr bool DB = RH == 8;
  static constexpr int KOP = 0;
  static constexpr int DS = DB ? 64 : 32;
  static constexpr int DV = DS + (DB ? 4 : 2) * NS;   // outputs: NV columns
  static constexpr int TCOLS = (DV + NV) <= 128 ? 128 : 256;
  static constexpr int MINB = TCOLS == 128 ? 3 : 2;   // CTAs per SM
  static_assert(MINB * TCOLS <= 512, "tensor memory of the resident CTAs");
};

__device__ __forceinline__ uint4 ldg_na(const void *p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

__device__ __forceinline__ void prefetch_l2(const void *p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

__device__ __forceinline__ uint32_t f2u_rn(float x) {
  uint32_t r;
  asm("cvt.rni.sat.u32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return r;
}

// OR of `pred` over the `count` threads of named barrier `id` (all of them
// call it; it synchronizes them).
__device__ __forceinline__ bool bar_or(int id, int count, bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.or.pred q, %2, %3, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)pred), "r"(id), "r"(count)
      : "memory");
  return r != 0;
}

// Signed base-256 digit l (0..3) of x, |x| < 2^31 - 2^24: x = sum_l d_l 2^(8l)
// with every digit in [-128, 127].
__device__ __forceinline__ int sdigit(int x, int l) {
  int d = 0;
#pragma unroll
  for (int k = 0; k < 4; k++) {
    d = (int)(int8_t)(x & 0xFF);
    if (k == l) break;
    x = (x - d) >> 8;
  }
  return d;
}

// 2^e for e in [-126, 127] (a normal float).
__device__ __forceinline__ float pow2i(int e) { return __uint_as_float((uint32_t)(e + 127) << 23); }

// The f32 value of four s32 digit columns d0 + 2^8 d1 + 2^16 d2 + 2^24 d3 of
// non-negative accumulators.
__device__ __forceinline__ float join4u(uint32_t d0, uint32_t d1, uint32_t d2, uint32_t d3) {
  const float hi = fmaf(__uint2float_rn(d3), 16777216.0f, __uint2float_rn(d2) * 65536.0f);
  const float lo = fmaf(__uint2float_rn(d1), 256.0f, __uint2float_rn(d0));
  return hi + lo;
}

__device__ __forceinline__ float2 f2(float x) { return make_float2(x, x); }

constexpr float kLazy = 2.0f;   // lazy-maximum threshold (log2 units): p <= 2^kLazy
constexpr int kPFix = 29;       // P' fixed point: 2^kPFix units per unit of p * s_v * 2^(127 - vexp)

// Exact f32 pair of the joined digit columns (d0 + 256 d1) + 65536 (d2 + 256 d3)
// of two heads, as the other tensor-core kernel forms them.
__device__ __forceinline__ float2 join_pair(const uint32_t *d) {
  const int ul0 = (int)d[0] + 256 * (int)d[1], uh0 = (int)d[2] + 256 * (int)d[3];
  const int ul1 = (int)d[4] + 256 * (int)d[5], uh1 = (int)d[6] + 256 * (int)d[7];
  return __ffma2_rn(make_float2((float)uh0, (float)uh1), f2(65536.0f),
                    make_float2((float)ul0, (float)ul1));
}

// N (8, 16 or 32) consecutive 32-bit tensor-memory columns of this thread's lane.
template <int N>
__device__ __forceinline__ void tmem_ldn(uint32_t taddr, uint32_t *r) {
  if constexpr (N == 32) tmem_ld32(taddr, *reinterpret_cast<uint32_t(*)[32]>(r));
  else if constexpr (N == 16) tmem_ld16(taddr, *reinterpret_cast<uint32_t(*)[16]>(r));
  else tmem_ld8(taddr, *reinterpret_cast<uint32_t(*)[8]>(r));
}

template <int RH>
__global__ void __launch_bounds__(UCfg<RH>::NT, UCfg<RH>::MINB)
decode_umma_kernel(const __grid_constant__ DecodeArgs a, const __grid_constant__ DecodeBatch batch) {
  using C = UCfg<RH>;
  constexpr int HD = C::HD, NG = C::NG, HQ = C::HQ;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_s = smem_u32(smem_raw);
  const uint32_t sb = (raw_s + 1023u) & ~1023u;   // shared-space base, 1024-aligned
  uint8_t *sm = smem_raw + (sb - raw_s);
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  const bool math = t < C::NM;                     // warp NW: the control warp
  const int pos = t & 127;                         // position of the block (math threads)
  const int G = a.n_q_heads / a.geom.n_heads;
  const int gh = a.cta_heads;
  const int nhg = G / (gh > 0 ? gh : 1);
  if (!launch_ok(a) || gh < 1 || gh > RH || G % gh != 0) return;
  const Item it = decode_item(a, batch, nhg);
  if (!item_ok(a, it, it.h * G + it.hg * gh, gh)) {
    if (a.n_splits > 1 && !a.sep_merge) arrive_last(a);
    return;
  }
  const size_t kv_stride = (size_t)a.geom.n_heads * a.geom.n_pages;
  const uint32_t PB = a.geom.page_bytes;
  const uint8_t *kpages = batch.base[it.b] + page_index(a.geom, it.layer, 0, it.h, 0) * PB;
  const uint8_t *vpages = kpages + kv_stride * PB;
  const int nblk = (it.npages + 1) / 2;
  const int pp = pos >> 6, prow = pos & 63;        // page of the block, row of the page
  const uint32_t budget = a.wait_budget;

  // ---- set-up loads first: queries, V exponent, L2 prefetch of the first blocks ----
  const int qh0 = it.h * G + it.hg * gh;
  const float *qb = a.q + ((size_t)(it.b * a.n_layers + it.lrow) * a.n_q_heads + qh0) * HD;
  constexpr int QPT = RH * HD / C::NM;
  float qv[QPT];
#pragma unroll
  for (int k = 0; k < QPT; k++) {
    const int i = t + k * C::NM;
    qv[k] = (math && i < gh * HD) ? __ldg(qb + i) : 0.0f;
  }
  const int vexp_raw = __ldg(vexp_table(batch.base[it.b], a.geom) + it.layer * a.geom.n_heads + it.h);
  constexpr int PF = 3;   // blocks prefetched into L2 ahead of the block being loaded
  auto prefetch_block = [&](int bb, int j) {   // j: 0/1 K pages, 2/3 V pages
    const int pi = 2 * bb + (j & 1);
    if (bb < nblk && pi < it.npages)
      prefetch_l2((j < 2 ? kpages : vpages) + (size_t)(it.pg0 + pi) * PB, PB);
  };
  if (warp == C::NW && lane < 4)
    for (int bb = 0; bb <= PF; bb++) prefetch_block(bb, lane);
  // the four 16-byte chunks of this position's K or V row and its (scale,
  // bias) pairs, loaded a step ahead
  uint4 rk[4], rv[4];
  float4 rsk, rsv;
  auto row_ptr = [&](const uint8_t *pages, int bb) -> const uint8_t * {
    const int pi = 2 * bb + pp;
    return pi < it.npages ? pages + (size_t)(it.pg0 + pi) * PB : nullptr;
  };
  auto load_k = [&](int bb) {
    const uint8_t *kp = row_ptr(kpages, bb);
    if (kp) {
#pragma unroll
      for (int c = 0; c < 4; c++) rk[c] = ldg_na(kp + prow * 64 + 16 * c);
      const uint4 s4 = ldg_na(kp + 4096 + prow * 16);
      rsk = make_float4(__uint_as_float(s4.x), __uint_as_float(s4.y), __uint_as_float(s4.z),
                        __uint_as_float(s4.w));
    } else {
#pragma unroll
      for (int c = 0; c < 4; c++) rk[c] = make_uint4(0u, 0u, 0u, 0u);
      rsk = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    }
  };
  auto load_v = [&](int bb) {
    const uint8_t *vp = row_ptr(vpages, bb);
    if (vp) {
#pragma unroll
      for (int c = 0; c < 4; c++) rv[c] = ldg_na(vp + prow * 64 + 16 * c);
      const uint4 s4 = ldg_na(vp + 4096 + prow * 16);
      rsv = make_float4(__uint_as_float(s4.x), __uint_as_float(s4.y), __uint_as_float(s4.z),
                        __uint_as_float(s4.w));
    } else {
#pragma unroll
      for (int c = 0; c < 4; c++) rv[c] = make_uint4(0u, 0u, 0u, 0u);
      rsv = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    }
  };
  if (math && nblk > 0) {
    load_k(0);
    load_v(0);
  }

  // ---- barriers and tensor memory --------------------------------------------------
  const uint32_t bar_s = sb + C::BAR_S, bar_v = sb + C::BAR_V, bar_drain = sb + C::BAR_DRAIN,
                 bar_staged = sb + C::BAR_STAGED, bar_p = sb + C::BAR_P;
  volatile int *vflags = reinterpret_cast<volatile int *>(sm + C::FLAGS);
  if (t == 0) {
    mbar_init(bar_s, 1);
    mbar_init(bar_s + 8, 1);
    for (int i = 0; i < C::NBUF; i++) mbar_init(bar_v + 8 * i, 1);
    mbar_init(bar_drain, 1);
    mbar_init(bar_staged, C::NW);
    mbar_init(bar_staged + 8, C::NW);
    mbar_init(bar_p, C::NW);
    fence_mbar_init();
  }
  __syncwarp();
  if (warp == 0) {
    tmem_alloc(sb + C::SLOT, C::TCOLS);
    tmem_relinquish();
  }
  float *q_s = reinterpret_cast<float *>(sm + C::QS);
  float *stat_s = reinterpret_cast<float *>(sm + C::STAT);
  const float qscale = rsqrtf((float)HD) * kLog2e;
  if (math) {
#pragma unroll
    for (int k = 0; k < QPT; k++) q_s[t + k * C::NM] = qv[k] * qscale;
  }
  fence_before_sync();
  __syncthreads();
  fence_after_sync();
  const uint32_t tb = *reinterpret_cast<volatile uint32_t *>(sm + C::SLOT);
  const uint32_t lane_off = (uint32_t)(32 * (warp & 3)) << 16;
  for (int h = warp; math && h < RH; h += C::NW) {
    float mx = 0.0f;
    for (int d = lane; d < HD; d += 32) mx = fmaxf(mx, fabsf(q_s[h * HD + d]));
#pragma unroll
    for (int g = 0; g < NG; g++) {
      float s = q_s[h * HD + 64 * g + lane] + q_s[h * HD + 64 * g + 32 + lane];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
      if (lane == 0) stat_s[RH + h * NG + g] = s;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if (lane == 0) stat_s[h] = mx;
  }
  __syncthreads();
  // per-head fixed point (as the other tensor-core kernel): x = rn(q 2^E),
  // |x| <= 2^30, E capped at 126; w = 2^-E weighs the joined digits (NaN when
  // the head's queries hold an inf or NaN). hcon: [RH] w, [RH] query sums of
  // group 0, [RH] of group 1, read as float2 per head pair.
  float *hcon = reinterpret_cast<float *>(sm + C::HCON);
  if (t < RH) {
    const float hmax = stat_s[t];
    int qexp = 0;
    frexpf(hmax > 0.0f && hmax <= 3.0e38f ? hmax : 1.0f, &qexp);
    const int qe = min(30 - qexp, 126);
    hcon[t] = hmax <= 3.0e38f ? pow2i(-qe) : __uint_as_float(0x7fc00000u);
    hcon[RH + t] = stat_s[RH + t * NG];
    hcon[2 * RH + t] = stat_s[RH + t * NG + 1];
  }
  // query digits: rows (h, d) of the two score B operands
  for (int i = t; math && i < RH * 64; i += C::NM) {
    const int h = i >> 6, k = i & 63, g = k >> 5, j = k & 31;
    const float hmax = stat_s[h];
    int qexp = 0;
    frexpf(hmax > 0.0f && hmax <= 3.0e38f ? hmax : 1.0f, &qexp);
    const int qe = min(30 - qexp, 126);
    const int xl = __float2int_rn(q_s[h * HD + 64 * g + j] * pow2i(qe));
    const int xh = __float2int_rn(q_s[h * HD + 64 * g + 32 + j] * pow2i(qe - 4));
#pragma unroll
    for (int d = 0; d < 4; d++) {
      sm[C::QB1 + swz_off(4 * h + d, k, 64)] = (uint8_t)sdigit(xl, d);
      sm[C::QB2 + swz_off(4 * h + d, k, 64)] = (uint8_t)sdigit(xh - xl, d);
    }
  }
  fence_proxy_async_smem();
  __syncthreads();   // query digits and per-head constants in place
  const float2 *W = reinterpret_cast<const float2 *>(hcon);
  const float2 *QS0 = reinterpret_cast<const float2 *>(hcon + RH);
  const float2 *QS1 = reinterpret_cast<const float2 *>(hcon + 2 * RH);

  // ---- the MMAs (issued by the control thread) ------------------------------------------
  const uint32_t id_s = idesc_i8(128, C::NS, 0, 1, 0, 0);
  const uint32_t id_v = idesc_i8(128, C::NV, 0, 0, 1, 1);
  auto issue_s = [&](int bb) {   // scores of block bb into score buffer bb % 2
    const uint64_t dq1 = sdesc(sb + C::QB1, 16, 512, kLayoutSW64);
    const uint64_t dq2 = sdesc(sb + C::QB2, 16, 512, kLayoutSW64);
    const uint32_t ds = tb + C::DS + (C::DB ? 2 * C::NS * (bb & 1) : 0);
    fence_after_sync();
#pragma unroll
    for (int g = 0; g < NG; g++) {
      const uint32_t kop = tb + C::KOP + (C::DB ? 32 * (bb & 1) : 0);
      mma_i8_ts(ds + g * C::NS, kop + 8 * g, dq1 + 2 * g, id_s, 0u);
      mma_i8_ts(ds + g * C::NS, kop + 16 + 8 * g, dq2 + 2 * g, id_s, 1u);
    }
    // test hook: the completion of this block's scores is never signalled, so
    // the wait for it runs out
    if (2 * bb != a.test_stall - 1 && 2 * bb + 1 != a.test_stall - 1)
      mma_commit(bar_s + (C::DB ? 8 * (bb & 1) : 0));
  };
  auto issue_v = [&](int vbuf, bool acc) {   // V of the block in buffer vbuf
    const uint64_t dva = sdesc(sb + C::OPV + vbuf * C::OPV_BYTES, 8192, 512, kLayoutSW64);
    const uint64_t dpb = sdesc(sb + C::OPP + vbuf * C::OPP_BYTES, 8192, 8 * C::PROW, C::PLAYOUT);
    fence_after_sync();
#pragma unroll
    for (int kc = 0; kc < 4; kc++)   // descriptor start addresses count 16-byte units
      mma_i8_ss(tb + C::DV, dva + kc * (2048 >> 4), dpb + kc * ((32 * C::PROW) >> 4), id_v,
                (kc > 0 || acc) ? 1u : 0u);
    mma_commit(bar_v + 8 * vbuf);
  };

  // ---- control thread: L2 prefetch and the MMAs ------------------------------------------
  // S(b) as soon as block b's K operands are in place (the math warps stage
  // them one block ahead, into double buffers, so S(b) runs while they finish
  // block b-1); V(b-1) once block b-1's V rows and P digits are written.
  bool ctrl_fail = false;
  if (t == C::NM) {
    for (int b = 0; b < nblk; b++) {
#pragma unroll
      for (int j = 0; j < 4; j++) prefetch_block(b + PF + 1, j);
      if (!mbar_wait_sleep(bar_staged + 8 * (b & 1), (b >> 1) & 1, budget)) {
        ctrl_fail = true;
        break;
      }
      issue_s(b);
      if (b > 0) {
        if (!mbar_wait_sleep(bar_p, (b - 1) & 1, budget)) {
          ctrl_fail = true;
          break;
        }
        const int vb = (b - 1) % C::NBUF;
        issue_v(vb, vflags[vb] != 0);
      }
    }
    if (!ctrl_fail && nblk > 0) {
      if (mbar_wait_sleep(bar_p, (nblk - 1) & 1, budget)) {
        const int vb = (nblk - 1) % C::NBUF;
        issue_v(vb, vflags[vb] != 0);
      } else {
        ctrl_fail = true;
      }
    }
    // every MMA issued has completed before the tensor memory is released
    mma_commit(bar_drain);
    if (!mbar_wait_sleep(bar_drain, 0, budget)) ctrl_fail = true;
  }

  // ---- staging (math warps) ----------------------------------------------------------------
  // K chunks of this thread -> tensor memory (the A operands of the score MMAs);
  // the arrival of the last warp lets the control thread issue the block's
  // score MMAs
  float4 sk_next = rsk;
  auto stage_k = [&](int bb) {
    const uint32_t kc = tb + lane_off + C::KOP + (C::DB ? 32 * (bb & 1) : 0);
#pragma unroll
    for (int c = 0; c < 4; c++) {
      tmem_st4(kc + 4 * c, rk[c]);
      tmem_st4(kc + 16 + 4 * c, make_uint4(rk[c].x & 0xF0F0F0F0u, rk[c].y & 0xF0F0F0F0u,
                                           rk[c].z & 0xF0F0F0F0u, rk[c].w & 0xF0F0F0F0u));
    }
    sk_next = rsk;
    tmem_wait_st();
    fence_before_sync();
    __syncwarp();
    if (lane == 0) mbar_arrive(bar_staged + 8 * (bb & 1));
  };
  uint32_t voff[4];
#pragma unroll
  for (int c = 0; c < 4; c++) voff[c] = swz_off(pos, 16 * c, 64);
  // V chunks of this thread -> the block's shared buffer (raw rows, masked rows)
  auto stage_v = [&](int vbuf) {
    uint8_t *vr = sm + C::OPV + vbuf * C::OPV_BYTES;
#pragma unroll
    for (int c = 0; c < 4; c++) {
      *reinterpret_cast<uint4 *>(vr + voff[c]) = rv[c];
      *reinterpret_cast<uint4 *>(vr + 8192 + voff[c]) =
          make_uint4(rv[c].x & 0xF0F0F0F0u, rv[c].y & 0xF0F0F0F0u, rv[c].z & 0xF0F0F0F0u,
                     rv[c].w & 0xF0F0F0F0u);
    }
  };

  // ---- softmax state, per head ------------------------------------------------------------
  float2 M[HQ], NMEFF[HQ], NTHR[HQ], L[HQ], PB0[HQ], PB1[HQ];
  float O[RH];
#pragma unroll
  for (int q = 0; q < HQ; q++) {
    M[q] = f2(-INFINITY);
    NMEFF[q] = f2(0.0f);
    NTHR[q] = f2(INFINITY);
    L[q] = PB0[q] = PB1[q] = f2(0.0f);
  }
#pragma unroll
  for (int i = 0; i < RH; i++) O[i] = 0.0f;
  const int vexp = min(max(vexp_raw, 1), 253);
  const float fsx = pow2i(127 - vexp) * pow2i(kPFix);   // P' scale: 2^(127 - vexp) 2^kPFix
  float *red = reinterpret_cast<float *>(sm + C::RED);
  const int grp = (pos & 63) >> 5;   // group of this thread's output row
  // output accumulator columns of this thread's row: its group's (head, digit)
  const uint32_t dv_cols = tb + lane_off + C::DV + grp * 4 * RH;
  auto drain_dv = [&]() {   // adds the integer output accumulators to O
    uint32_t d[4 * RH];
    tmem_ldn<4 * RH>(dv_cols, d);
    tmem_wait_ld();
#pragma unroll
    for (int i = 0; i < RH; i++) O[i] += join4u(d[4 * i], d[4 * i + 1], d[4 * i + 2], d[4 * i + 3]);
  };
  auto vbar_wait = [&](int bb) {
    return mbar_wait_sleep(bar_v + 8 * (bb % C::NBUF), (bb / C::NBUF) & 1, budget);
  };

  if (math && nblk > 0) {
    stage_k(0);
    if (nblk > 1) load_k(1);
  }
  bool fail = false, aborted = false, vacc = false;
  int vbuf = 0;   // V and P buffers of block b
  for (int b = 0; math && b < nblk; b++) {
    const float4 sk = sk_next;
    // double buffers: K of block b+1 into its operand buffer (last read by
    // S(b-1), complete), whose score MMAs then run while block b is finished;
    // then the loads of block b+2's K rows
    if (C::DB && b + 1 < nblk) {
      stage_k(b + 1);
      if (b + 2 < nblk) load_k(b + 2);
    }
    // scores of block b (every head, both groups)
    const bool s_ok = C::DB ? mbar_wait_sleep(bar_s + 8 * (b & 1), (b >> 1) & 1, budget)
                            : mbar_wait_sleep(bar_s, b & 1, budget);
    if (!s_ok) fail = true;
    fence_after_sync();
    const uint32_t ds = tb + lane_off + C::DS + (C::DB ? 2 * C::NS * (b & 1) : 0);
    uint32_t d0[4 * RH], d1[4 * RH];   // (head, digit) columns of each group
    tmem_ldn<4 * RH>(ds, d0);
    tmem_ldn<4 * RH>(ds + C::NS, d1);
    tmem_wait_ld();
    // single buffers: the K operands and the score columns are free again once
    // S(b) has completed and its scores are in registers
    if (!C::DB && b + 1 < nblk) {
      stage_k(b + 1);
      if (b + 2 < nblk) load_k(b + 2);
    }
    float2 part[HQ];
#pragma unroll
    for (int q = 0; q < HQ; q++) {
      part[q] = __fmul2_rn(join_pair(d0 + 8 * q), f2(sk.x));
      part[q] = __ffma2_rn(join_pair(d1 + 8 * q), f2(sk.z), part[q]);
      part[q] = __fmul2_rn(part[q], W[q]);
      part[q] = __ffma2_rn(f2(sk.y), QS0[q], part[q]);
      part[q] = __ffma2_rn(f2(sk.w), QS1[q], part[q]);
    }
    // positions outside the attended range (partial blocks only) score -inf
    const int pos0 = (it.pg0 + 2 * b) * kPagePositions;
    if (!(2 * b + 1 < it.npages && pos0 >= it.r0 && pos0 + C::BLK <= it.r1)) {
      const int pi = 2 * b + pp, p = pos0 + pos;
      if (!(pi < it.npages && p >= it.r0 && p < it.r1)) {
#pragma unroll
        for (int q = 0; q < HQ; q++) part[q] = f2(-INFINITY);
      }
    }
    // lazy maximum: does any score pass its head's maximum by more than kLazy?
    float ex = -INFINITY;
#pragma unroll
    for (int q = 0; q < HQ; q++) {
      const float2 dd = __fadd2_rn(part[q], NTHR[q]);
      ex = fmaxf(ex, fmaxf(dd.x, dd.y));
    }
    if (bar_or(1, C::NM, ex > 0.0f || fail)) {
      if (bar_or(1, C::NM, fail)) {
        aborted = true;
        break;
      }
      // block maxima per head over the CTA; every thread applies the same update
#pragma unroll
      for (int q = 0; q < HQ; q++) {
        float m0 = part[q].x, m1 = part[q].y;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
          m0 = fmaxf(m0, __shfl_xor_sync(0xffffffffu, m0, o));
          m1 = fmaxf(m1, __shfl_xor_sync(0xffffffffu, m1, o));
        }
        if (lane == 0) {
          red[warp * RH + 2 * q] = m0;
          red[warp * RH + 2 * q + 1] = m1;
        }
      }
      named_sync(1, C::NM);
      if (vacc) {   // every V MMA so far: its accumulators go to O first
        if (!vbar_wait(b - 1)) fail = true;
        fence_after_sync();
        drain_dv();
      }
#pragma unroll
      for (int i = 0; i < RH; i++) {
        const float bm = fmaxf(fmaxf(red[i], red[RH + i]), fmaxf(red[2 * RH + i], red[3 * RH + i]));
        float &m = (i & 1) ? M[i / 2].y : M[i / 2].x;
        const bool need = bm > m + kLazy;
        const float mn = need ? bm : m;
        const float al = need ? ex2(m - mn) : 1.0f;   // exp2(-inf) = 0
        m = mn;
        ((i & 1) ? NMEFF[i / 2].y : NMEFF[i / 2].x) = mn == -INFINITY ? 0.0f : -mn;
        ((i & 1) ? NTHR[i / 2].y : NTHR[i / 2].x) = -(mn + kLazy);
        ((i & 1) ? L[i / 2].y : L[i / 2].x) *= al;
        ((i & 1) ? PB0[i / 2].y : PB0[i / 2].x) *= al;
        ((i & 1) ? PB1[i / 2].y : PB1[i / 2].x) *= al;
        O[i] *= al;
      }
      vacc = false;   // V(b) overwrites the accumulators
    }
    // V of block b into its buffer (last read by V(b-3)); load block b+1's V rows
    if (b >= C::NBUF && !vbar_wait(b - C::NBUF)) fail = true;
    stage_v(vbuf);
    const float4 sv = rsv;
    if (b + 1 < nblk) load_v(b + 1);
    // probabilities, bias sums and this thread's P digits of its position
    const float svx0 = sv.x * fsx, svx1 = sv.z * fsx;
    uint32_t x0[RH], x1[RH];
#pragma unroll
    for (int q = 0; q < HQ; q++) {
      const float2 x = __fadd2_rn(part[q], NMEFF[q]);
      const float2 p = make_float2(ex2(x.x), ex2(x.y));
      L[q] = __fadd2_rn(L[q], p);
      PB0[q] = __ffma2_rn(p, f2(sv.y), PB0[q]);
      PB1[q] = __ffma2_rn(p, f2(sv.w), PB1[q]);
      const float2 y0 = __fmul2_rn(p, f2(svx0)), y1 = __fmul2_rn(p, f2(svx1));
      x0[2 * q] = f2u_rn(y0.x);
      x0[2 * q + 1] = f2u_rn(y0.y);
      x1[2 * q] = f2u_rn(y1.x);
      x1[2 * q + 1] = f2u_rn(y1.y);
    }
    // words (g, h) of the P row: group g at g RH + h
    uint8_t *pr = sm + C::OPP + vbuf * C::OPP_BYTES;
#pragma unroll
    for (int c = 0; c < RH / 4; c++) {
      *reinterpret_cast<uint4 *>(pr + swz_off(pos, 16 * c, C::PROW)) =
          make_uint4(x0[4 * c], x0[4 * c + 1], x0[4 * c + 2], x0[4 * c + 3]);
      *reinterpret_cast<uint4 *>(pr + swz_off(pos, 4 * RH + 16 * c, C::PROW)) =
          make_uint4(x1[4 * c], x1[4 * c + 1], x1[4 * c + 2], x1[4 * c + 3]);
    }
    if (t == 0) vflags[vbuf] = vacc ? 1 : 0;   // V(b) accumulates onto earlier blocks
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) mbar_arrive(bar_p);
    vbuf = vbuf + 1 == C::NBUF ? 0 : vbuf + 1;
    vacc = true;
  }
  if (math && !aborted) {
    bool f = fail;
    if (nblk > 0 && !vbar_wait(nblk - 1)) f = true;
    aborted = bar_or(1, C::NM, f);
    if (!aborted && nblk > 0) {
      fence_after_sync();
      if (vacc) drain_dv();
    }
  }
  __syncwarp();   // the control warp's lanes meet again before the aligned wait
  tmem_wait_st();
  fence_before_sync();
  const bool abort_all = __syncthreads_or(aborted || ctrl_fail);
  if (warp == 0) tmem_dealloc(tb, C::TCOLS);
  if (abort_all) {
    if (t == 0) report(a, kStatusWaitTimeout);
    if (a.n_splits > 1 && !a.sep_merge) arrive_last(a);
    return;
  }

  // ---- per-CTA totals and the output rows ------------------------------------------
  float *ow = reinterpret_cast<float *>(sm + C::OPV);          // [128 rows][RH]
  float *rl = ow + 128 * RH;                                    // [4 warps][RH]
  float *rpb = rl + 4 * RH;                                     // [4 warps][RH][NG]
#pragma unroll
  for (int i = 0; i < RH && math; i++) {
    const int h = i, q = i / 2;
    ow[pos * RH + h] = O[i];
    float l = (i & 1) ? L[q].y : L[q].x;
    float p0 = (i & 1) ? PB0[q].y : PB0[q].x;
    float p1 = (i & 1) ? PB1[q].y : PB1[q].x;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      l += __shfl_xor_sync(0xffffffffu, l, o);
      p0 += __shfl_xor_sync(0xffffffffu, p0, o);
      p1 += __shfl_xor_sync(0xffffffffu, p1, o);
    }
    if (lane == 0) {
      const int w4 = warp & 3;
      rl[w4 * RH + h] = l;
      rpb[(w4 * RH + h) * NG] = p0;
      rpb[(w4 * RH + h) * NG + 1] = p1;
    }
  }
  // the maxima of every head, for the rows' records (uniform per head)
  float *mh = rpb + 4 * RH * NG;                                // [RH]
  if (math && pos == 0) {
#pragma unroll
    for (int i = 0; i < RH; i++) mh[i] = (i & 1) ? M[i / 2].y : M[i / 2].x;
  }
  __syncthreads();
  const float oscale = pow2i(-kPFix) * __uint_as_float((uint32_t)vexp << 23);   // 2^-kPFix 2^(vexp-127)
  const size_t row0 = (size_t)(it.b * a.n_layers + it.lrow) * a.n_q_heads + qh0;
  for (int idx = t; idx < gh * HD; idx += C::NT) {
    const int h = idx / HD, d = idx - h * HD;
    const int g = d >> 6, k = d & 63, jb = 32 * g + (k & 31);
    const float hi = ow[(64 + jb) * RH + h];
    const float val = k < 32 ? ow[jb * RH + h] - hi : hi * (1.0f / 16.0f);
    const float Ls = (rl[h] + rl[RH + h]) + (rl[2 * RH + h] + rl[3 * RH + h]);
    const float PBv = (rpb[h * NG + g] + rpb[(RH + h) * NG + g]) +
                      (rpb[(2 * RH + h) * NG + g] + rpb[(3 * RH + h) * NG + g]);
    const float Ov = fmaf(val, oscale, PBv);
    const float Mh = mh[h];
    const size_t row = row0 + h;
    if (a.n_splits == 1) {
      a.out[row * HD + d] = Ov / Ls;
      if (a.lse && d == 0) a.lse[row] = Ls > 0.0f ? (Mh + log2f(Ls)) * kLn2 : -INFINITY;
    } else {
      const size_t pr = row * a.n_splits + it.split;
      a.part_o[pr * HD + d] = Ov;
      if (d == 0) {
        a.part_m[pr] = Mh;
        a.part_l[pr] = Ls;
      }
    }
  }
  if (a.n_splits > 1 && !a.sep_merge && arrive_last(a))
    merge_splits<HD, RH, C::NT>(a, row0, gh, reinterpret_cast<float *>(sm + C::OPV));
}

template <int RH>
int launch_u(const DecodeArgs &a, const DecodeBatch &b, int n_blocks, cudaStream_t s) {
  using C = UCfg<RH>;
  auto fn = decode_umma_kernel<RH>;
  static std::atomic<unsigned long long> attr_done{0};   // one bit per device
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(attr_done.load(std::memory_order_acquire) >> (dev & 63) & 1)) {
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    if (e != cudaSuccess) return check_cuda(e, "decode_umma: smem attribute");
    attr_done.fetch_or(1ull << (dev & 63), std::memory_order_acq_rel);
  }
  fn<<<n_blocks, C::NT, C::SMEM, s>>>(a, b);
  return check_cuda(cudaGetLastError(), "decode_umma launch");
}

// Resident CTAs on the device (per SM x SMs), or 0 when more CTAs could be
// resident on an SM than its tensor memory serves (their allocations would
// wait for one another): the caller then uses another kernel.
template <int RH>
int resident_u() {
  using C = UCfg<RH>;
  static std::atomic<int> cached[64];
  int dev = 0;
  cudaGetDevice(&dev);
  const int hit = cached[dev & 63].load(std::memory_order_relaxed);
  if (hit) return hit > 0 ? hit : 0;
  cudaFuncSetAttribute(decode_umma_kernel<RH>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
  int per_sm = 0, sms = 148;
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, decode_umma_kernel<RH>, C::NT, C::SMEM);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  cudaGetLastError();
  const int r = (per_sm >= 1 && per_sm * C::TCOLS <= 512) ? per_sm * sms : -1;
  cached[dev & 63].store(r, std::memory_order_relaxed);
  return r > 0 ? r : 0;
}

}  // namespace

int umma_resident(int gh, int head_dim) {
  if (head_dim != 128 || gh < 1 || gh > 8) return 0;
  return gh > 4 ? resident_u<8>() : resident_u<4>();
}

int umma_launch(int gh, const DecodeArgs &a0, const DecodeBatch &b, int n_blocks, cudaStream_t s) {
  DecodeArgs a = a0;
  a.cta_heads = gh;
  return gh > 4 ? launch_u<8>(a, b, n_blocks, s) : launch_u<4>(a, b, n_blocks, s);
}

}  // namespace eakv
