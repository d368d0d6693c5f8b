// quantize.cu - Q4_1 quantize / append kernel (replaces reference
// kernels/quantize_simd.ea:9-59 and the host narrowing loop of
// src/cache.c:85-92 / :139-146).
//
// Bit-exactness contract: packed nibbles, scales and biases equal the
// reference's for every input, NaN and signed zeros included. The
// arithmetic is written with explicit round-to-nearest intrinsics so no
// multiply/add pair can be contracted into an FMA (the reference computes
// t = (x - min) * inv, then t + 0.5, each rounded), and the min/max follow
// the reference's sequential strict-compare scan:
//   * a NaN in element 0 makes min = max = that NaN;
//   * other NaNs are skipped (fminf/fmaxf ignore a NaN operand);
//   * between -0.0 and +0.0 the first one in element order wins, so when
//     the min (or max) is a zero the kernel looks up the first zero.
//
// Mapping: 2 threads per 64-float group. Thread j loads elements 16j..16j+15
// (the low nibbles of bytes 16j..16j+15) and 32+16j..32+16j+15 (their high
// nibbles) as eight 16-byte loads, and stores the 16 packed bytes as one
// 16-byte word, so a warp moves 16 groups with fully coalesced traffic and
// the per-group work (min/max reduction, the two divisions) is shared by
// 16 groups per warp instruction (4 threads per group measured 37.2 us per
// cfg4 append slice, 2 threads 35.1 us).
// HBM-bound: 256 B read + 40 B written per group.
//
// The cache keeps, per (layer, KV head), the largest biased exponent of any
// V scale (the decode kernels scale probabilities by it). The same kernel
// raises it: a warp whose groups all belong to one (layer, V, head) unit
// reduces their exponents and one lane raises the table (a load, and an
// atomicMax only when the table holds less). A separate kernel over the
// scales just written cost 8 us per V slice, a launch of its own.
#include "internal.cuh"

namespace eakv {
namespace {

constexpr int kThreads = 256;
constexpr int kTPG = 2;   // threads per 64-element group

// The reference truncates with x86 cvttss2si, which returns INT_MIN for NaN
// and for anything outside the int32 range; the clamp then gives 0. That
// case is real: a group whose range is denormal has inv = 15/range = +inf,
// so every element above the minimum maps to +inf (and the minimum to NaN).
// The device conversion would saturate +inf to INT_MAX (-> 15), so those
// inputs are sent to 0 explicitly.
__device__ __forceinline__ int quant_one(float x, float mn, float inv) {
  float t = __fadd_rn(__fmul_rn(__fsub_rn(x, mn), inv), 0.5f);
  int q = (t < 2147483648.0f) ? __float2int_rz(t) : 0;   // NaN compares false
  return q < 0 ? 0 : (q > 15 ? 15 : q);
}

// 4 blocks per SM (at most 64 registers, no spill): 33.0 us per cfg4 append
// slice against 35.0 at 3 blocks (79 registers); 5 blocks spill (36 us).
template <bool kVec>
__global__ void __launch_bounds__(kThreads, 4)
quantize_kernel(const float *__restrict__ src, uint8_t *__restrict__ dst, PageGeom g,
                int unit_base, long long n_groups, int n_tok, int pos0, int head_dim) {
  constexpr int EPT = 32 / kTPG;          // elements per thread in each half of the group
  constexpr int GPW = 32 / kTPG;          // groups per warp and iteration
  const long long groups_per_unit = (long long)n_tok * g.gpd;
  const int lane = threadIdx.x & 31;
  const int j = lane % kTPG;              // thread within the group
  const long long warps = (long long)gridDim.x * (kThreads / 32);
  const long long warp_id = (long long)blockIdx.x * (kThreads / 32) + (threadIdx.x >> 5);

  for (long long gb = warp_id * GPW; gb < n_groups; gb += warps * GPW) {
    const long long gi = gb + lane / kTPG;
    const bool valid = gi < n_groups;
    // v[e]: element EPT*j + e (low nibble of byte EPT*j + e); v[EPT + e]:
    // element 32 + EPT*j + e (its high nibble)
    float v[2 * EPT];
    long long u = 0, gih = 0;
    if (valid) {
      // Group gih of unit u: the reference quantizes n_tok*gpd consecutive
      // 64-float groups starting at the unit's first element
      // (src/cache.c:78,85-88 and :136-142).
      u = gi / groups_per_unit;
      gih = gi - u * groups_per_unit;
      const float *x = src + (size_t)u * n_tok * head_dim + (size_t)gih * 64;
      if (kVec) {
#pragma unroll
        for (int h = 0; h < 2; h++)
#pragma unroll
          for (int k = 0; k < EPT / 4; k++) {
            const float4 a = *reinterpret_cast<const float4 *>(x + 32 * h + EPT * j + 4 * k);
            v[h * EPT + 4 * k + 0] = a.x;
            v[h * EPT + 4 * k + 1] = a.y;
            v[h * EPT + 4 * k + 2] = a.z;
            v[h * EPT + 4 * k + 3] = a.w;
          }
      } else {
#pragma unroll
        for (int e = 0; e < EPT; e++) {
          v[e] = x[EPT * j + e];
          v[EPT + e] = x[32 + EPT * j + e];
        }
      }
    } else {
#pragma unroll
      for (int e = 0; e < 2 * EPT; e++) v[e] = 0.0f;
    }

    float mn = v[0], mx = v[0];
#pragma unroll
    for (int e = 1; e < 2 * EPT; e++) {
      mn = fminf(mn, v[e]);
      mx = fmaxf(mx, v[e]);
    }
#pragma unroll
    for (int o = 1; o < kTPG; o <<= 1) {
      mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    }
    const float x0 = __shfl_sync(0xffffffffu, v[0], lane & ~(kTPG - 1));

    // Signed-zero fix-up (rare, warp-uniform branch): the reference keeps
    // the first zero it meets, whichever its sign.
    const bool need_zero = valid && (x0 == x0) && (mn == 0.0f || mx == 0.0f);
    if (__any_sync(0xffffffffu, need_zero)) {
      int fz = 64;
      float zv = 0.0f;
#pragma unroll
      for (int e = 2 * EPT - 1; e >= 0; e--) {
        int idx = e < EPT ? EPT * j + e : 32 + EPT * j + (e - EPT);
        if (v[e] == 0.0f && idx < fz) {
          fz = idx;
          zv = v[e];
        }
      }
#pragma unroll
      for (int o = 1; o < kTPG; o <<= 1) {
        int ofz = __shfl_xor_sync(0xffffffffu, fz, o);
        float ozv = __shfl_xor_sync(0xffffffffu, zv, o);
        if (ofz < fz) {
          fz = ofz;
          zv = ozv;
        }
      }
      if (need_zero) {
        if (mn == 0.0f) mn = zv;
        if (mx == 0.0f) mx = zv;
      }
    }
    if (x0 != x0) {   // NaN in element 0 sticks (reference quantize_simd.ea:22-30)
      mn = x0;
      mx = x0;
    }

    const float range = __fsub_rn(mx, mn);
    float scale = 1.0f, inv = 0.0f;
    if (range > 0.0f) {
      scale = __fdiv_rn(range, 15.0f);
      inv = __fdiv_rn(15.0f, range);
    }
    // V slices: raise the cache's per-(layer, head) maximum V-scale
    // exponent. A warp's groups nearly always belong to one unit: then its
    // largest exponent is raised by one lane, with an atomic only when the
    // table holds less; at a unit boundary each group raises its own.
    {
      const long long U = unit_base + u;
      const int lkv = (int)(U / g.n_heads);
      const bool isv = valid && (lkv & 1);
      const unsigned vmask = __ballot_sync(0xffffffffu, isv);
      if (vmask) {
        const int ex = isv ? (int)((__float_as_uint(scale) >> 23) & 0xFF) : 0;
        const int lead = __ffs(vmask) - 1;
        const long long Ul = __shfl_sync(0xffffffffu, U, lead);
        if (__all_sync(0xffffffffu, !isv || U == Ul)) {
          const int m = __reduce_max_sync(0xffffffffu, ex);
          if (lane == lead) {
            const int lv = (int)(Ul / g.n_heads);
            int *p = vexp_table(dst, g) + (lv >> 1) * g.n_heads + (int)(Ul - (long long)lv * g.n_heads);
            if (m > *reinterpret_cast<volatile int *>(p)) atomicMax(p, m);
          }
        } else if (isv && j == 0) {
          int *p = vexp_table(dst, g) + (lkv >> 1) * g.n_heads + (int)(U - (long long)lkv * g.n_heads);
          if (ex > *reinterpret_cast<volatile int *>(p)) atomicMax(p, ex);
        }
      }
    }
    uint32_t word[EPT / 4];
#pragma unroll
    for (int w = 0; w < EPT / 4; w++) {
      word[w] = 0;
#pragma unroll
      for (int e = 0; e < 4; e++) {
        uint32_t lo = (uint32_t)quant_one(v[4 * w + e], mn, inv);
        uint32_t hi = (uint32_t)quant_one(v[EPT + 4 * w + e], mn, inv);
        word[w] |= (hi * 16u + lo) << (8 * e);
      }
    }
    if (valid) {
      const int t = (int)(gih / g.gpd);
      const int grp = (int)(gih - (long long)t * g.gpd);
      const int pos = pos0 + t;
      const int page = pos / kPagePositions;
      const int pip = pos - page * kPagePositions;
      uint8_t *pp = dst + ((size_t)(unit_base + u) * g.n_pages + page) * g.page_bytes;
      const int slot = pip * g.gpd + grp;
      uint8_t *wp = pp + (size_t)slot * 32 + EPT * j;
      if constexpr (EPT == 16)
        *reinterpret_cast<uint4 *>(wp) = make_uint4(word[0], word[1], word[2], word[3]);
      else if constexpr (EPT == 8)
        *reinterpret_cast<uint2 *>(wp) = make_uint2(word[0], word[EPT / 4 - 1]);
      else
        *reinterpret_cast<uint32_t *>(wp) = word[0];
      if (j == 0)
        *reinterpret_cast<float2 *>(pp + g.nib_bytes + (size_t)slot * 8) = make_float2(scale, mn);
    }
  }
}

}  // namespace

cudaError_t launch_quantize(const PageGeom &g, uint8_t *d_buf, const float *d_src,
                            int head_dim, int unit_base, int n_units, int n_tok, int pos0,
                            cudaStream_t s) {
  if (g.gpd <= 0 || n_units <= 0 || n_tok <= 0) return cudaSuccess;
  const long long n_groups = (long long)n_units * n_tok * g.gpd;
  constexpr int kGroupsPerBlock = kThreads / kTPG;
  long long blocks = (n_groups + kGroupsPerBlock - 1) / kGroupsPerBlock;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  long long cap = (long long)sms * 8;
  if (blocks > cap) blocks = cap;
  if (((uintptr_t)d_src & 15) == 0 && (head_dim & 3) == 0)
    quantize_kernel<true><<<(int)blocks, kThreads, 0, s>>>(d_src, d_buf, g, unit_base, n_groups,
                                                           n_tok, pos0, head_dim);
  else
    quantize_kernel<false><<<(int)blocks, kThreads, 0, s>>>(d_src, d_buf, g, unit_base, n_groups,
                                                            n_tok, pos0, head_dim);
  return cudaGetLastError();
}

}  // namespace eakv
