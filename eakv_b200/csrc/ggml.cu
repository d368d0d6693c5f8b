// ggml.cu - the q4_1_eakv ggml block type on the GPU (reference
// src/ggml_type.c:21-242, include/eakv_ggml.h:25-52).
//
// Blocks are the reference's 40-byte AoS records {qs[32], d, m} for 64
// elements, lo nibble of qs[k] = element k, hi nibble = element k+32. The
// three kernels reproduce the reference's AVX-512 build bit for bit (its
// x86 hot path, ggml_type.c:7; a NaN made by arithmetic carries the GPU's
// canonical payload instead of x86's): every 64-element block is handled by 16
// lanes (a half warp) standing for the 16 lanes of its zmm registers, each
// lane runs the same operation chain as its zmm lane, and the horizontal
// reductions follow the trees of _mm512_reduce_{min,max,add}_ps:
//
//   MINPS(a, b) = a < b ? a : b, MAXPS(a, b) = a > b ? a : b (a NaN or two
//   zeros give b); min/max tree: (hi 8 vs lo 8), (hi 4 vs lo 4), (v vs
//   v[i^2]), (v vs v[i^1]); add tree: l + l^8, + l^4, + l^2, + l^1.
//
// from_float: d = range/15 (0 when range == 0, unlike the cache quantizer's
// 1), id = 15/range or 0, q = cvtt(min(15, max(0, (x - m) * id + 0.5)))
// (NaN -> 0 after the byte narrowing; +inf -> 15). to_float: fma(n, d, m).
// vec_dot: per lane acc = fma(fma(n, d, m), y, acc) over lo(0..15),
// hi(32..47), lo(16..31), hi(48..63) of each block, then the add tree.
//
// All three are HBM-bound streaming kernels (256 B f32 in / 40 B out per
// block; 40 B in / 256 B out; 40 + 256 B in per block of a dot product).
#include <mutex>
#include <string.h>

#include "internal.cuh"
#include "../../include/eakv_ggml.h"

namespace eakv {
namespace {

constexpr int kThreads = 256;
constexpr int kBlockBytes = 40;

__device__ __forceinline__ float minps(float a, float b) { return a < b ? a : b; }
__device__ __forceinline__ float maxps(float a, float b) { return a > b ? a : b; }

// Lanes of this thread's half warp: the loops below run per half warp, and
// the two halves of a warp may leave them at different trips, so every
// shuffle names only its own half.
__device__ __forceinline__ unsigned half_mask() { return 0xFFFFu << (threadIdx.x & 16); }

// min/max reduction of the 16 lanes of a half warp (lane 0 of the half
// holds the result of the reference's tree; it is broadcast to all 16)
template <bool kMax>
__device__ __forceinline__ float reduce16(float v, int l16, unsigned hm) {
  float o = __shfl_down_sync(hm, v, 8, 16);   // T1 = upper 8 lanes, T2 = this lane
  if (l16 < 8) v = kMax ? maxps(o, v) : minps(o, v);
  o = __shfl_down_sync(hm, v, 4, 16);
  if (l16 < 4) v = kMax ? maxps(o, v) : minps(o, v);
  o = __shfl_xor_sync(hm, v, 2, 16);          // T8 = op(T6, T6[i^2])
  v = kMax ? maxps(v, o) : minps(v, o);
  o = __shfl_xor_sync(hm, v, 1, 16);          // T10 = op(T8, T8[i^1])
  v = kMax ? maxps(v, o) : minps(v, o);
  return __shfl_sync(hm, v, 0, 16);
}

// d and m of a block (two 4-byte accesses: rows may sit at any 4-byte
// aligned stride)
__device__ __forceinline__ float2 load_dm(const uint8_t *blk) {
  return make_float2(*reinterpret_cast<const float *>(blk + 32),
                     *reinterpret_cast<const float *>(blk + 36));
}

// from_float and to_float: each half warp takes kQB consecutive blocks per
// trip and loads all of them before it works on any (more loads in flight
// per warp); the arithmetic of a block is unchanged.
constexpr int kQB = 4;

__global__ void __launch_bounds__(kThreads)
ggml_quantize_kernel(const float *__restrict__ src, uint8_t *__restrict__ dst, long long nb) {
  const int l = threadIdx.x & 15;
  const unsigned hm = half_mask();
  const long long halves = (long long)gridDim.x * (kThreads / 16);
  for (long long i0 = ((long long)blockIdx.x * (kThreads / 16) + (threadIdx.x >> 4)) * kQB; i0 < nb;
       i0 += halves * kQB) {
    float xs[kQB][4];
#pragma unroll
    for (int k = 0; k < kQB; k++) {
      if (i0 + k < nb) {
        const float *x = src + (i0 + k) * 64;
        xs[k][0] = x[l];
        xs[k][1] = x[16 + l];
        xs[k][2] = x[32 + l];
        xs[k][3] = x[48 + l];
      }
    }
#pragma unroll
    for (int k = 0; k < kQB; k++) {
      if (i0 + k >= nb) break;   // uniform over the half warp
      const long long i = i0 + k;
      const float x0 = xs[k][0], x1 = xs[k][1], x2 = xs[k][2], x3 = xs[k][3];
      float vmin = x0, vmax = x0;
      vmin = minps(vmin, x1);
      vmax = maxps(vmax, x1);
      vmin = minps(vmin, x2);
      vmax = maxps(vmax, x2);
      vmin = minps(vmin, x3);
      vmax = maxps(vmax, x3);
      const float mn = reduce16<false>(vmin, l, hm);
      const float mx = reduce16<true>(vmax, l, hm);
      const float range = __fsub_rn(mx, mn);
      const float d = __fdiv_rn(range, 15.0f);
      const float id = range > 0.0f ? __fdiv_rn(15.0f, range) : 0.0f;
      // after the clamp t is in [0, 15] or NaN; cvtt(t) is then floor(t), the
      // low 4 bits of t + 2^23 added toward zero, or for NaN INT32_MIN, whose
      // low byte and whose value shifted left by 4 are both 0
      auto q = [&](float v) {
        float t = __fmul_rn(__fsub_rn(v, mn), id);
        t = minps(15.0f, maxps(0.0f, __fadd_rn(t, 0.5f)));
        return t == t ? ((unsigned)__float_as_int(__fadd_rz(t, 8388608.0f)) & 15u) : 0u;
      };
      uint8_t *blk = dst + i * kBlockBytes;
      blk[l] = (uint8_t)((q(x0) | (q(x2) << 4)) & 0xFF);
      blk[16 + l] = (uint8_t)((q(x1) | (q(x3) << 4)) & 0xFF);
      if (l == 0) {
        *reinterpret_cast<float *>(blk + 32) = d;
        *reinterpret_cast<float *>(blk + 36) = mn;
      }
    }
  }
}

__global__ void __launch_bounds__(kThreads)
ggml_dequantize_kernel(const uint8_t *__restrict__ src, float *__restrict__ dst, long long nb) {
  const int l = threadIdx.x & 15;
  const long long halves = (long long)gridDim.x * (kThreads / 16);
  for (long long i0 = ((long long)blockIdx.x * (kThreads / 16) + (threadIdx.x >> 4)) * kQB; i0 < nb;
       i0 += halves * kQB) {
    float2 dm[kQB];
    uint8_t r0[kQB], r1[kQB];
#pragma unroll
    for (int k = 0; k < kQB; k++) {
      if (i0 + k < nb) {
        const uint8_t *blk = src + (i0 + k) * kBlockBytes;
        dm[k] = load_dm(blk);
        r0[k] = blk[l];
        r1[k] = blk[16 + l];
      }
    }
#pragma unroll
    for (int k = 0; k < kQB; k++) {
      if (i0 + k >= nb) break;
      float *out = dst + (i0 + k) * 64;
      out[l] = fmaf((float)(r0[k] & 15), dm[k].x, dm[k].y);
      out[16 + l] = fmaf((float)(r1[k] & 15), dm[k].x, dm[k].y);
      out[32 + l] = fmaf((float)(r0[k] >> 4), dm[k].x, dm[k].y);
      out[48 + l] = fmaf((float)(r1[k] >> 4), dm[k].x, dm[k].y);
    }
  }
}

// One half warp per row.
__global__ void __launch_bounds__(kThreads)
ggml_vec_dot_kernel(int nb, float *s, size_t bs, const uint8_t *vx, size_t bx, const uint8_t *vy,
                    size_t by, int nrc) {
  const unsigned hm = half_mask();
  const int l = threadIdx.x & 15;
  const int halves = gridDim.x * (kThreads / 16);
  for (int r = blockIdx.x * (kThreads / 16) + (threadIdx.x >> 4); r < nrc; r += halves) {
    const uint8_t *blocks = vx + (size_t)r * bx;
    const float *y = reinterpret_cast<const float *>(vy + (size_t)r * by);
    float acc = 0.0f;
    for (int i = 0; i < nb; i++) {
      const uint8_t *blk = blocks + (size_t)i * kBlockBytes;
      const float2 dm = load_dm(blk);
#pragma unroll
      for (int c = 0; c < 2; c++) {
        const uint8_t raw = blk[c * 16 + l];
        acc = fmaf(fmaf((float)(raw & 15), dm.x, dm.y), y[c * 16 + l], acc);
        acc = fmaf(fmaf((float)(raw >> 4), dm.x, dm.y), y[c * 16 + 32 + l], acc);
      }
      y += 64;
    }
    acc += __shfl_xor_sync(hm, acc, 8, 16);
    acc += __shfl_xor_sync(hm, acc, 4, 16);
    acc += __shfl_xor_sync(hm, acc, 2, 16);
    acc += __shfl_xor_sync(hm, acc, 1, 16);
    if (l == 0) *reinterpret_cast<float *>(reinterpret_cast<char *>(s) + (size_t)r * bs) = acc;
  }
}

int grid_for(long long units) {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  long long blocks = (units + kThreads / 16 - 1) / (kThreads / 16);
  const long long cap = (long long)sms * 8;
  return (int)(blocks < 1 ? 1 : (blocks > cap ? cap : blocks));
}

// Device staging for the host-pointer entry points (one buffer per
// process, grown on demand, guarded by a mutex for the whole call).
std::mutex g_stage_mu;
void *g_stage = nullptr;
size_t g_stage_bytes = 0;
int g_stage_dev = -1;

void *stage(size_t bytes) {
  int dev = 0;
  cudaGetDevice(&dev);
  if (g_stage && (g_stage_bytes < bytes || g_stage_dev != dev)) {
    cudaSetDevice(g_stage_dev);
    cudaFree(g_stage);
    cudaSetDevice(dev);
    g_stage = nullptr;
    g_stage_bytes = 0;
  }
  if (!g_stage) {
    if (cudaMalloc(&g_stage, bytes) != cudaSuccess) {
      g_stage = nullptr;
      set_error(EAKV_ERR_ALLOC, "ggml: cannot allocate %zu bytes of device staging", bytes);
      return nullptr;
    }
    g_stage_bytes = bytes;
    g_stage_dev = dev;
  }
  return g_stage;
}

}  // namespace
}  // namespace eakv

using namespace eakv;

extern "C" {

int eakv_ggml_quantize_row_device(const float *d_src, void *d_dst, int64_t k, void *stream) {
  clear_error();
  if (k < 0 || (k >= 64 && (!d_src || !d_dst))) {
    set_error(EAKV_ERR_INVALID, "ggml_quantize_row_device: invalid argument");
    return EAKV_ERR_INVALID;
  }
  const long long nb = k / 64;
  if (nb == 0) return EAKV_OK;
  ggml_quantize_kernel<<<grid_for(nb), kThreads, 0, (cudaStream_t)stream>>>(
      d_src, (uint8_t *)d_dst, nb);
  return check_cuda(cudaGetLastError(), "ggml_quantize_row_device");
}

int eakv_ggml_dequantize_row_device(const void *d_src, float *d_dst, int64_t k, void *stream) {
  clear_error();
  if (k < 0 || (k >= 64 && (!d_src || !d_dst))) {
    set_error(EAKV_ERR_INVALID, "ggml_dequantize_row_device: invalid argument");
    return EAKV_ERR_INVALID;
  }
  const long long nb = k / 64;
  if (nb == 0) return EAKV_OK;
  ggml_dequantize_kernel<<<grid_for(nb), kThreads, 0, (cudaStream_t)stream>>>(
      (const uint8_t *)d_src, d_dst, nb);
  return check_cuda(cudaGetLastError(), "ggml_dequantize_row_device");
}

int eakv_ggml_vec_dot_device(int n, float *d_s, size_t bs, const void *d_vx, size_t bx,
                             const void *d_vy, size_t by, int nrc, void *stream) {
  clear_error();
  if (n < 0 || nrc < 0 || (nrc > 0 && (!d_s || !d_vx || !d_vy))) {
    set_error(EAKV_ERR_INVALID, "ggml_vec_dot_device: invalid argument");
    return EAKV_ERR_INVALID;
  }
  if (nrc == 0) return EAKV_OK;
  ggml_vec_dot_kernel<<<grid_for(nrc), kThreads, 0, (cudaStream_t)stream>>>(
      n / 64, d_s, bs, (const uint8_t *)d_vx, bx, (const uint8_t *)d_vy, by, nrc);
  return check_cuda(cudaGetLastError(), "ggml_vec_dot_device");
}

// ---- the reference's host-pointer entry points (eakv_ggml.h) ------------
// Same signatures and results as the reference; the data crosses PCIe
// each call, so these are for drop-in use, not speed.

void eakv_quantize_row(const float *src, void *dst, int64_t k) {
  clear_error();
  const int64_t nb = k / 64;
  if (nb <= 0 || !src || !dst) return;
  std::lock_guard<std::mutex> lock(g_stage_mu);
  const size_t in = (size_t)nb * 64 * sizeof(float), out = (size_t)nb * kBlockBytes;
  uint8_t *buf = (uint8_t *)stage(in + out);
  if (!buf) return;
  if (check_cuda(cudaMemcpy(buf, src, in, cudaMemcpyHostToDevice), "eakv_quantize_row")) return;
  if (eakv_ggml_quantize_row_device((const float *)buf, buf + in, nb * 64, nullptr)) return;
  check_cuda(cudaMemcpy(dst, buf + in, out, cudaMemcpyDeviceToHost), "eakv_quantize_row");
}

void eakv_dequantize_row(const void *src, float *dst, int64_t k) {
  clear_error();
  const int64_t nb = k / 64;
  if (nb <= 0 || !src || !dst) return;
  std::lock_guard<std::mutex> lock(g_stage_mu);
  const size_t in = (size_t)nb * kBlockBytes, out = (size_t)nb * 64 * sizeof(float);
  const size_t in_al = (in + 255) & ~(size_t)255;
  uint8_t *buf = (uint8_t *)stage(in_al + out);
  if (!buf) return;
  if (check_cuda(cudaMemcpy(buf, src, in, cudaMemcpyHostToDevice), "eakv_dequantize_row")) return;
  if (eakv_ggml_dequantize_row_device(buf, (float *)(buf + in_al), nb * 64, nullptr)) return;
  check_cuda(cudaMemcpy(dst, buf + in_al, out, cudaMemcpyDeviceToHost), "eakv_dequantize_row");
}

void eakv_vec_dot_q4_f32(int n, float *s, size_t bs, const void *vx, size_t bx, const void *vy,
                         size_t by, int nrc) {
  clear_error();
  const int nb = n / 64;
  if (nrc <= 0 || !s || !vx || !vy) return;
  // the reference reads row r at vx + r*bx, vy + r*by and writes s + r*bs;
  // the rows are gathered densely on the device
  const size_t xrow = (size_t)nb * kBlockBytes, yrow = (size_t)nb * 64 * sizeof(float);
  std::lock_guard<std::mutex> lock(g_stage_mu);
  const size_t xs = ((xrow * nrc) + 255) & ~(size_t)255, ys = ((yrow * nrc) + 255) & ~(size_t)255;
  uint8_t *buf = (uint8_t *)stage(xs + ys + (size_t)nrc * sizeof(float));
  if (!buf) return;
  for (int r = 0; r < nrc && nb > 0; r++) {
    if (check_cuda(cudaMemcpy(buf + r * xrow, (const uint8_t *)vx + (size_t)r * bx, xrow,
                              cudaMemcpyHostToDevice), "eakv_vec_dot_q4_f32") ||
        check_cuda(cudaMemcpy(buf + xs + r * yrow, (const uint8_t *)vy + (size_t)r * by, yrow,
                              cudaMemcpyHostToDevice), "eakv_vec_dot_q4_f32"))
      return;
  }
  float *d_s = (float *)(buf + xs + ys);
  if (eakv_ggml_vec_dot_device(n, d_s, sizeof(float), buf, xrow, buf + xs, yrow, nrc, nullptr))
    return;
  for (int r = 0; r < nrc; r++)
    if (check_cuda(cudaMemcpy((uint8_t *)s + (size_t)r * bs, d_s + r, sizeof(float),
                              cudaMemcpyDeviceToHost), "eakv_vec_dot_q4_f32"))
      return;
}

}  // extern "C"
