// inspect.cu - checks and read-back of a resident cache: device validate
// (reference kernels/validate.ea:14-71 as the CLI runs it, src/cli.c:39-98)
// and dequantize (reference kernels/dequantize_avx512.ea:10-89).
//
// validate: per (layer, K/V), the reference's q4_validate scans the groups
// in its dense order ([head][position][group], positions < seq_len) and
// returns at the first group that has a NaN scale (1), a NaN bias (2) or a
// scale below zero (3), checked in that order. Here every group is checked
// in parallel; a failing group offers the key index*4 + code to an
// atomicMin per (layer, K/V), so the smallest key is the reference's first
// failure and its low two bits its code. Only the (scale, bias) pairs are
// read (8 of every 40 bytes of the pages), page by page, contiguously.
//
// dequantize: value = fma(nibble, scale, bias) for the lo (element k) and
// hi (element k+32) nibble of byte k of a group, the reference's f32x16
// fma, so the values equal the reference's bit for bit.
#include "internal.cuh"

namespace eakv {
namespace {

constexpr int kThreads = 256;

__device__ __forceinline__ bool is_nan_bits(float v) {
  const int b = __float_as_int(v);   // validate.ea:51-62: > 0x7F800000, or in (-0x800000, 0)
  return b > 2139095040 || (b < 0 && b > -8388608);
}

// Block (x, y, z): pages x*kPagesPerBlock.. of KV head z of block y =
// layer*2 + kv. Its threads read the (scale, bias) pairs of those pages as
// 16-byte vectors (two slots each), kUnroll loads at a time; the position
// and group of a slot are worked out only for a failing one.
constexpr int kPagesPerBlock = 8;

__global__ void __launch_bounds__(kThreads)
validate_kernel(const uint8_t *__restrict__ buf, PageGeom g, int seq_len,
                unsigned long long *__restrict__ keys) {
  constexpr int kUnroll = 2;   // loads in flight per thread
  const int lkv = blockIdx.y;  // layer * 2 + kv
  const int h = blockIdx.z;    // KV head
  const int pg0 = blockIdx.x * kPagesPerBlock;
  const int used_pages = (seq_len + kPagePositions - 1) / kPagePositions;
  const int n_pg = min(kPagesPerBlock, used_pages - pg0);
  const int vec = kPagePositions * g.gpd / 2;   // 16-byte vectors of (scale, bias) pairs per page
  const int total = n_pg * vec;
  const uint8_t *base =
      buf + (((size_t)lkv * g.n_heads + h) * g.n_pages + pg0) * g.page_bytes + g.nib_bytes;
  unsigned long long best = ~0ull;
  for (int r0 = threadIdx.x; r0 < total; r0 += kThreads * kUnroll) {
    float4 sb[kUnroll];
    int pl[kUnroll], q[kUnroll];
#pragma unroll
    for (int k = 0; k < kUnroll; k++) {
      const int r = r0 + k * kThreads;
      pl[k] = -1;
      q[k] = 0;
      if (r < total) {
        pl[k] = r / vec;
        q[k] = r - pl[k] * vec;
        sb[k] = *reinterpret_cast<const float4 *>(base + (size_t)pl[k] * g.page_bytes + q[k] * 16);
      }
    }
#pragma unroll
    for (int k = 0; k < kUnroll; k++) {
      if (pl[k] < 0) continue;
      // slots 2q and 2q+1 of the page; slot s is position s / gpd, group s % gpd,
      // and only slots of positions below seq_len count
      const int page = pg0 + pl[k];
      const int limit = min(kPagePositions, seq_len - page * kPagePositions) * g.gpd;
#pragma unroll
      for (int e = 0; e < 2; e++) {
        const int s_ = 2 * q[k] + e;
        if (s_ >= limit) continue;
        const float sc = e ? sb[k].z : sb[k].x, bi = e ? sb[k].w : sb[k].y;
        const int code = is_nan_bits(sc) ? 1 : is_nan_bits(bi) ? 2 : (sc < 0.0f ? 3 : 0);
        if (code) {
          // dense index of the group: [head][position][group]
          const int t = page * kPagePositions + s_ / g.gpd;
          const unsigned long long gi =
              ((unsigned long long)h * seq_len + t) * g.gpd + (unsigned long long)(s_ % g.gpd);
          best = min(best, gi * 4 + code);
        }
      }
    }
  }
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
    best = other < best ? other : best;
  }
  if ((threadIdx.x & 31) == 0 && best != ~0ull) atomicMin(keys + lkv, best);
}

// One warp per (head, position) row, kRows rows per trip with all their
// loads issued first; lane l writes dims 4l..4l+3 of each 128-dim slice:
// four consecutive dims are four consecutive bytes of one group, all low or
// all high nibbles.
constexpr int kRows = 4;

__global__ void __launch_bounds__(kThreads)
dequant_kernel(const uint8_t *__restrict__ buf, PageGeom g, int head_dim, int lkv, int pos_begin,
               int n_pos, float *__restrict__ out) {
  const int lane = threadIdx.x & 31;
  const long long rows = (long long)g.n_heads * n_pos;
  const long long warps = (long long)gridDim.x * (kThreads / 32);
  for (long long row0 = ((long long)blockIdx.x * (kThreads / 32) + (threadIdx.x >> 5)) * kRows;
       row0 < rows; row0 += warps * kRows) {
    for (int d = 4 * lane; d < head_dim; d += 128) {
      const int grp = d >> 6, k = d & 63;
      const int sh = k < 32 ? 0 : 4;
      uint32_t w[kRows];
      float2 sb[kRows];
#pragma unroll
      for (int r = 0; r < kRows; r++) {
        const long long row = row0 + r;
        if (row < rows) {
          const int h = (int)(row / n_pos);
          const int t = pos_begin + (int)(row - (long long)h * n_pos);
          const int page = t / kPagePositions, pip = t - page * kPagePositions;
          const uint8_t *pp = buf + (((size_t)lkv * g.n_heads + h) * g.n_pages + page) * g.page_bytes;
          const int slot = pip * g.gpd + grp;
          w[r] = *reinterpret_cast<const uint32_t *>(pp + (size_t)slot * 32 + (k & 31));
          sb[r] = reinterpret_cast<const float2 *>(pp + g.nib_bytes)[slot];
        }
      }
#pragma unroll
      for (int r = 0; r < kRows; r++) {
        const long long row = row0 + r;
        if (row >= rows) break;
        float4 v;
        v.x = fmaf((float)((w[r] >> sh) & 15), sb[r].x, sb[r].y);
        v.y = fmaf((float)((w[r] >> (8 + sh)) & 15), sb[r].x, sb[r].y);
        v.z = fmaf((float)((w[r] >> (16 + sh)) & 15), sb[r].x, sb[r].y);
        v.w = fmaf((float)((w[r] >> (24 + sh)) & 15), sb[r].x, sb[r].y);
        *reinterpret_cast<float4 *>(out + row * head_dim + d) = v;
      }
    }
  }
}

int grid_cap(long long units) {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  long long b = (units + kThreads - 1) / kThreads;
  const long long cap = (long long)sms * 8;
  return (int)(b < 1 ? 1 : (b > cap ? cap : b));
}

int dequant_check(const eakv_cache_t *c, int layer, int kv, int pos_begin, int pos_end,
                  const void *out, const char *what) {
  if (!c || !out || layer < 0 || layer >= c->n_layers || kv < 0 || kv > 1 || pos_begin < 0 ||
      pos_end < pos_begin || pos_end > c->seq_len || c->geom.gpd == 0) {
    set_error(EAKV_ERR_INVALID, "%s: invalid argument", what);
    return EAKV_ERR_INVALID;
  }
  return EAKV_OK;
}

}  // namespace
}  // namespace eakv

using namespace eakv;

extern "C" {

int eakv_cache_validate(const eakv_cache_t *cc, int32_t *codes) {
  clear_error();
  if (!cc || !codes) {
    set_error(EAKV_ERR_INVALID, "validate: invalid argument");
    return EAKV_ERR_INVALID;
  }
  eakv_cache_t *c = const_cast<eakv_cache_t *>(cc);
  const int n = c->n_layers * 2;
  for (int i = 0; i < n; i++) codes[i] = 0;
  if (c->seq_len == 0 || c->geom.gpd == 0) return EAKV_OK;
  if (n > 65535 || c->n_kv_heads > 65535) {   // grid y and z
    set_error(EAKV_ERR_INVALID, "validate: more than 65535 (layer, K/V) blocks or KV heads");
    return EAKV_ERR_INVALID;
  }
  DeviceGuard g(c->device);
  unsigned long long *d_keys = (unsigned long long *)cache_scratch(c, (size_t)n * 8);
  if (!d_keys) return EAKV_ERR_ALLOC;
  int rc = check_cuda(cudaMemsetAsync(d_keys, 0xFF, (size_t)n * 8, c->stream), "validate");
  if (rc) return rc;
  const int used_pages = (c->seq_len + kPagePositions - 1) / kPagePositions;
  const int bx = (used_pages + kPagesPerBlock - 1) / kPagesPerBlock;
  validate_kernel<<<dim3(bx, n, c->n_kv_heads), kThreads, 0, c->stream>>>(c->d_buf, c->geom,
                                                                          c->seq_len, d_keys);
  rc = check_cuda(cudaGetLastError(), "validate: launch");
  if (rc) return rc;
  unsigned long long *keys = new unsigned long long[n];
  rc = check_cuda(cudaMemcpyAsync(keys, d_keys, (size_t)n * 8, cudaMemcpyDeviceToHost, c->stream),
                  "validate: copy");
  if (!rc) rc = check_cuda(cudaStreamSynchronize(c->stream), "validate");
  if (!rc)
    for (int i = 0; i < n; i++) codes[i] = keys[i] == ~0ull ? 0 : (int32_t)(keys[i] & 3);
  delete[] keys;
  return rc;
}

int eakv_cache_dequantize_device(const eakv_cache_t *c, int layer, int kv_idx, int pos_begin,
                                 int pos_end, float *d_out, void *stream) {
  clear_error();
  int rc = dequant_check(c, layer, kv_idx, pos_begin, pos_end, d_out, "dequantize_device");
  if (rc) return rc;
  if ((uintptr_t)d_out & 15) {   // rows are written as 16-byte vectors
    set_error(EAKV_ERR_INVALID, "dequantize_device: d_out must be 16-byte aligned");
    return EAKV_ERR_INVALID;
  }
  const int n_pos = pos_end - pos_begin;
  if (n_pos == 0) return EAKV_OK;
  DeviceGuard g(c->device);
  const long long rows = (long long)c->n_kv_heads * n_pos;
  cudaStream_t s = stream ? (cudaStream_t)stream : c->stream;
  dequant_kernel<<<grid_cap(rows * 32), kThreads, 0, s>>>(c->d_buf, c->geom, c->head_dim,
                                                          layer * 2 + kv_idx, pos_begin, n_pos,
                                                          d_out);
  return check_cuda(cudaGetLastError(), "dequantize_device: launch");
}

int eakv_cache_dequantize(const eakv_cache_t *cc, int layer, int kv_idx, int pos_begin,
                          int pos_end, float *out) {
  clear_error();
  int rc = dequant_check(cc, layer, kv_idx, pos_begin, pos_end, out, "dequantize");
  if (rc) return rc;
  eakv_cache_t *c = const_cast<eakv_cache_t *>(cc);
  const size_t bytes = (size_t)c->n_kv_heads * (pos_end - pos_begin) * c->head_dim * sizeof(float);
  if (bytes == 0) return EAKV_OK;
  DeviceGuard g(c->device);
  float *d_out = (float *)cache_scratch(c, bytes);
  if (!d_out) return EAKV_ERR_ALLOC;
  rc = eakv_cache_dequantize_device(c, layer, kv_idx, pos_begin, pos_end, d_out, c->stream);
  if (rc) return rc;
  rc = check_cuda(cudaMemcpyAsync(out, d_out, bytes, cudaMemcpyDeviceToHost, c->stream),
                  "dequantize: copy");
  if (rc) return rc;
  return check_cuda(cudaStreamSynchronize(c->stream), "dequantize");
}

}  // extern "C"
