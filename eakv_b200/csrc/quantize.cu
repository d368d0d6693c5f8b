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
// Mapping: 8 threads per 64-float group. Thread j loads elements 4j..4j+3
// (the low nibbles of bytes 4j..4j+3) and 32+4j..32+4j+3 (their high
// nibbles) as two 16-byte loads, and stores the 4 packed bytes as one
// 32-bit word, so a warp moves 4 groups with fully coalesced traffic.
// HBM-bound: 256 B read + 40 B written per group.
#include "internal.cuh"

namespace eakv {
namespace {

constexpr int kThreads = 256;

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

template <bool kVec>
__global__ void __launch_bounds__(kThreads)
quantize_kernel(const float *__restrict__ src, uint8_t *__restrict__ dst, PageGeom g,
                int unit_base, long long n_groups, int n_tok, int pos0, int head_dim) {
  const long long groups_per_unit = (long long)n_tok * g.gpd;
  const int lane = threadIdx.x & 31;
  const int j = lane & 7;                 // thread within the group
  const long long warps = (long long)gridDim.x * (kThreads / 32);
  const long long warp_id = (long long)blockIdx.x * (kThreads / 32) + (threadIdx.x >> 5);
  // Largest V-scale exponent this group leader has produced for the
  // (layer, head) entry v_idx, published to the cache's exponent table when
  // the entry changes and at the end (one atomic per run of groups instead
  // of one per group).
  int v_idx = -1, v_e = 0;

  // Group gih of unit u: the reference quantizes n_tok*gpd consecutive
  // 64-float groups starting at the unit's first element
  // (src/cache.c:78,85-88 and :136-142).
  auto load = [&](long long gi, float (&v)[8]) {
    if (gi < n_groups) {
      const long long u = gi / groups_per_unit;
      const long long gih = gi - u * groups_per_unit;
      const float *x = src + (size_t)u * n_tok * head_dim + (size_t)gih * 64;
      if (kVec) {
        float4 a = *reinterpret_cast<const float4 *>(x + 4 * j);
        float4 b = *reinterpret_cast<const float4 *>(x + 32 + 4 * j);
        v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
        v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
      } else {
#pragma unroll
        for (int e = 0; e < 4; e++) {
          v[e] = x[4 * j + e];
          v[4 + e] = x[32 + 4 * j + e];
        }
      }
    } else {
#pragma unroll
      for (int e = 0; e < 8; e++) v[e] = 0.0f;
    }
  };

  // each iteration loads the next group before it quantizes this one, so
  // two loads per thread are in flight
  float nxt[8];
  load(warp_id * 4 + (lane >> 3), nxt);
  for (long long gb = warp_id * 4; gb < n_groups; gb += warps * 4) {
    const long long gi = gb + (lane >> 3);
    const bool valid = gi < n_groups;
    float v[8];
#pragma unroll
    for (int e = 0; e < 8; e++) v[e] = nxt[e];
    if (gb + warps * 4 < n_groups) load(gi + warps * 4, nxt);
    const long long u = valid ? gi / groups_per_unit : 0;
    const long long gih = gi - u * groups_per_unit;

    float mn = v[0], mx = v[0];
#pragma unroll
    for (int e = 1; e < 8; e++) {
      mn = fminf(mn, v[e]);
      mx = fmaxf(mx, v[e]);
    }
#pragma unroll
    for (int o = 1; o < 8; o <<= 1) {
      mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    }
    const float x0 = __shfl_sync(0xffffffffu, v[0], lane & 24);

    // Signed-zero fix-up (rare, warp-uniform branch): the reference keeps
    // the first zero it meets, whichever its sign.
    const bool need_zero = valid && (x0 == x0) && (mn == 0.0f || mx == 0.0f);
    if (__any_sync(0xffffffffu, need_zero)) {
      int fz = 64;
      float zv = 0.0f;
#pragma unroll
      for (int e = 7; e >= 0; e--) {
        int idx = e < 4 ? 4 * j + e : 32 + 4 * j + (e - 4);
        if (v[e] == 0.0f && idx < fz) {
          fz = idx;
          zv = v[e];
        }
      }
#pragma unroll
      for (int o = 1; o < 8; o <<= 1) {
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
    uint32_t word = 0;
#pragma unroll
    for (int e = 0; e < 4; e++) {
      uint32_t lo = (uint32_t)quant_one(v[e], mn, inv);
      uint32_t hi = (uint32_t)quant_one(v[4 + e], mn, inv);
      word |= (hi * 16u + lo) << (8 * e);
    }
    if (valid) {
      const int t = (int)(gih / g.gpd);
      const int grp = (int)(gih - (long long)t * g.gpd);
      const int pos = pos0 + t;
      const int page = pos / kPagePositions;
      const int pip = pos - page * kPagePositions;
      uint8_t *pp = dst + ((size_t)(unit_base + u) * g.n_pages + page) * g.page_bytes;
      const int slot = pip * g.gpd + grp;
      *reinterpret_cast<uint32_t *>(pp + (size_t)slot * 32 + 4 * j) = word;
      if (j == 0) {
        *reinterpret_cast<float2 *>(pp + g.nib_bytes + (size_t)slot * 8) = make_float2(scale, mn);
        const int U = unit_base + (int)u;              // (layer * 2 + kv) * heads + head
        const int lkv = U / g.n_heads;
        if (lkv & 1) {
          const int idx = (lkv >> 1) * g.n_heads + (U - lkv * g.n_heads);
          const int e = (int)((__float_as_uint(scale) >> 23) & 0xFF);
          if (idx != v_idx) {
            if (v_idx >= 0) atomicMax(vexp_table(dst, g) + v_idx, v_e);
            v_idx = idx;
            v_e = e;
          } else {
            v_e = max(v_e, e);
          }
        }
      }
    }
  }
  if (v_idx >= 0) atomicMax(vexp_table(dst, g) + v_idx, v_e);
}

}  // namespace

cudaError_t launch_quantize(const PageGeom &g, uint8_t *d_buf, const float *d_src,
                            int head_dim, int unit_base, int n_units, int n_tok, int pos0,
                            cudaStream_t s) {
  if (g.gpd <= 0 || n_units <= 0 || n_tok <= 0) return cudaSuccess;
  const long long n_groups = (long long)n_units * n_tok * g.gpd;
  long long blocks = (n_groups + 31) / 32;
  const bool vec = ((uintptr_t)d_src & 15) == 0 && (head_dim & 3) == 0;
  // one wave of resident blocks: the grid-stride loop gives every block the
  // same share, so blocks beyond the resident set would run as a second,
  // mostly idle wave
  int dev = 0, sms = 148, per_sm = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  cudaError_t e = vec ? cudaOccupancyMaxActiveBlocksPerMultiprocessor(
                            &per_sm, quantize_kernel<true>, kThreads, 0)
                      : cudaOccupancyMaxActiveBlocksPerMultiprocessor(
                            &per_sm, quantize_kernel<false>, kThreads, 0);
  if (e != cudaSuccess) return e;
  const long long cap = (long long)sms * (per_sm > 0 ? per_sm : 1);
  if (blocks > cap) blocks = cap;
  if (vec)
    quantize_kernel<true><<<(int)blocks, kThreads, 0, s>>>(d_src, d_buf, g, unit_base, n_groups,
                                                           n_tok, pos0, head_dim);
  else
    quantize_kernel<false><<<(int)blocks, kThreads, 0, s>>>(d_src, d_buf, g, unit_base, n_groups,
                                                            n_tok, pos0, head_dim);
  return cudaGetLastError();
}

}  // namespace eakv
