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

#include "internal.cuh"

namespace eakv {
namespace {

constexpr int kScoreThreads = 256;   // 16 positions x 16 lanes
constexpr int kHeadChunk = 32;       // query heads per pass (shared memory bound)

// grid: (pages of the sequence, n_kv, head chunks); one page per block.
__global__ void __launch_bounds__(kScoreThreads)
scores_kernel(const uint8_t *__restrict__ buf, PageGeom g, int layer,
              const float *__restrict__ q, int q_per_kv, int head_dim, int seq_len,
              float rsqrt_d, float *__restrict__ scores) {
  extern __shared__ float smem[];
  const int kvh = blockIdx.y;
  const int h0 = blockIdx.z * kHeadChunk;
  const int nh = min(kHeadChunk, q_per_kv - h0);
  float *q_s = smem;                          // [nh][head_dim]
  float *sc_s = smem + kHeadChunk * head_dim; // [nh][64]
  const int page = blockIdx.x;
  const int l = threadIdx.x & 15;
  const int slot = threadIdx.x >> 4;          // position slot 0..15

  for (int i = threadIdx.x; i < nh * head_dim; i += blockDim.x) {
    int j = i / head_dim, d = i - j * head_dim;
    q_s[i] = q[(size_t)(kvh * q_per_kv + h0 + j) * head_dim + d];
  }
  __syncthreads();

  const uint8_t *pp = buf + page_index(g, layer, 0, kvh, page) * g.page_bytes;
  const float2 *sb = reinterpret_cast<const float2 *>(pp + g.nib_bytes);
  for (int sub = 0; sub < 4; sub++) {
    const int pip = sub * 16 + slot;
    const int t = page * kPagePositions + pip;
    const bool valid = t < seq_len;
    float k[8];   // dequantized elements of this lane, gpd <= 2
    const int gpd = g.gpd;
#pragma unroll
    for (int grp = 0; grp < 2; grp++) {
      if (grp < gpd) {
        uint32_t b0 = 0, b1 = 0;
        float2 s = make_float2(0.f, 0.f);
        if (valid) {
          const uint8_t *row = pp + (size_t)(pip * gpd + grp) * 32;
          b0 = row[l];
          b1 = row[16 + l];
          s = sb[pip * gpd + grp];
        }
        k[4 * grp + 0] = __fmaf_rn((float)(b0 & 15), s.x, s.y);
        k[4 * grp + 1] = __fmaf_rn((float)(b1 & 15), s.x, s.y);
        k[4 * grp + 2] = __fmaf_rn((float)(b0 >> 4), s.x, s.y);
        k[4 * grp + 3] = __fmaf_rn((float)(b1 >> 4), s.x, s.y);
      }
    }
    for (int j = 0; j < nh; j++) {
      const float *qj = q_s + j * head_dim;
      float acc = 0.0f;
#pragma unroll
      for (int grp = 0; grp < 2; grp++) {
        if (grp < gpd) {
#pragma unroll
          for (int jj = 0; jj < 4; jj++)
            acc = __fmaf_rn(k[4 * grp + jj], qj[grp * 64 + jj * 16 + l], acc);
        }
      }
      acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, 8));
      acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, 4));
      acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, 2));
      acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, 1));
      if (l == 0) sc_s[j * 64 + pip] = __fmul_rn(acc, rsqrt_d);
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < nh * 64; i += blockDim.x) {
    int j = i >> 6, pip = i & 63;
    int t = page * kPagePositions + pip;
    if (t < seq_len) scores[(size_t)(kvh * q_per_kv + h0 + j) * seq_len + t] = sc_s[i];
  }
}

constexpr int kVHeads = 8;   // accumulators per thread

// grid: (chunks, n_kv, head chunks of kVHeads); blockDim = head_dim.
// Writes d_out directly when there is one chunk, else per-chunk partials.
__global__ void vsum_kernel(const uint8_t *__restrict__ buf, PageGeom g, int layer,
                            const float *__restrict__ w, int q_per_kv, int head_dim,
                            int seq_len, int chunk, float *__restrict__ out,
                            float *__restrict__ part, int n_q) {
  extern __shared__ float w_s[];   // [kVHeads][chunk]
  const int kvh = blockIdx.y;
  const int h0 = blockIdx.z * kVHeads;
  const int nh = min(kVHeads, q_per_kv - h0);
  const int t0 = blockIdx.x * chunk;
  const int t1 = min(seq_len, t0 + chunk);
  const int n = t1 - t0;
  for (int i = threadIdx.x; i < nh * chunk; i += blockDim.x) {
    int j = i / chunk, tt = i - j * chunk;
    w_s[i] = tt < n ? w[(size_t)(kvh * q_per_kv + h0 + j) * seq_len + t0 + tt] : 0.0f;
  }
  __syncthreads();
  const int d = threadIdx.x;
  const int grp = d >> 6, e = d & 63;
  const int byte = e & 31, shift = (e >> 5) * 4;
  float o[kVHeads];
#pragma unroll
  for (int j = 0; j < kVHeads; j++) o[j] = 0.0f;
  for (int tt = 0; tt < n; tt++) {
    const int t = t0 + tt;
    const int page = t / kPagePositions, pip = t - page * kPagePositions;
    const uint8_t *pp = buf + page_index(g, layer, 1, kvh, page) * g.page_bytes;
    const int slot = pip * g.gpd + grp;
    const float nib = (float)((pp[(size_t)slot * 32 + byte] >> shift) & 15);
    const float2 s = reinterpret_cast<const float2 *>(pp + g.nib_bytes)[slot];
    const float v = __fmaf_rn(nib, s.x, s.y);
#pragma unroll
    for (int j = 0; j < kVHeads; j++)
      if (j < nh) o[j] = __fmaf_rn(v, w_s[j * chunk + tt], o[j]);
  }
  float *dst = gridDim.x == 1 ? out : part + (size_t)blockIdx.x * n_q * head_dim;
  for (int j = 0; j < nh; j++) dst[(size_t)(kvh * q_per_kv + h0 + j) * head_dim + d] = o[j];
}

// out[i] = part[0][i] + part[1][i] + ... in chunk order.
__global__ void vsum_combine_kernel(const float *__restrict__ part, int n_chunks, size_t n,
                                    float *__restrict__ out) {
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x) {
    float acc = part[i];
    for (int c = 1; c < n_chunks; c++) acc = __fadd_rn(acc, part[(size_t)c * n + i]);
    out[i] = acc;
  }
}

__global__ void fill_kernel(float *p, size_t n, float v) {
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x)
    p[i] = v;
}

int vsum_chunk(int seq_len, int n_kv) {
  // Whole sequence in one chunk while it is short (bit-exact with the
  // reference); otherwise enough chunks for ~2 blocks per SM.
  if (seq_len <= 512) return seq_len > 0 ? seq_len : 1;
  int want_chunks = (2 * 148 + n_kv - 1) / n_kv;
  int c = (seq_len + want_chunks - 1) / want_chunks;
  c = (c + 63) / 64 * 64;
  if (c < 256) c = 256;
  if (c > 2048) c = 2048;
  return c;
}

}  // namespace

cudaError_t launch_scores(const PageGeom &g, const uint8_t *d_buf, int layer, const float *d_q,
                          int n_q, int n_kv, int seq_len, float rsqrt_d, float *d_scores,
                          cudaStream_t s) {
  if (seq_len <= 0) return cudaSuccess;
  const int q_per_kv = n_q / n_kv;
  const int head_dim = g.gpd * 64;
  dim3 grid((seq_len + 63) / 64, n_kv, (q_per_kv + kHeadChunk - 1) / kHeadChunk);
  size_t smem = (size_t)kHeadChunk * (head_dim + 64) * sizeof(float);
  scores_kernel<<<grid, kScoreThreads, smem, s>>>(d_buf, g, layer, d_q, q_per_kv, head_dim,
                                                  seq_len, rsqrt_d, d_scores);
  return cudaGetLastError();
}

size_t vsum_scratch_floats(const PageGeom &g, int n_q, int seq_len) {
  int chunk = vsum_chunk(seq_len, 1);
  int n_chunks = (seq_len + chunk - 1) / chunk;
  return n_chunks > 1 ? (size_t)n_chunks * n_q * g.gpd * 64 : 0;
}

cudaError_t launch_vsum(const PageGeom &g, const uint8_t *d_buf, int layer, const float *d_w,
                        int n_q, int n_kv, int seq_len, float *d_out, float *d_part,
                        size_t part_floats, cudaStream_t s) {
  const int head_dim = g.gpd * 64;
  if (seq_len <= 0) {   // reference stores the zero-initialized accumulators
    fill_kernel<<<32, 256, 0, s>>>(d_out, (size_t)n_q * head_dim, 0.0f);
    return cudaGetLastError();
  }
  const int q_per_kv = n_q / n_kv;
  int chunk = vsum_chunk(seq_len, n_kv);
  int n_chunks = (seq_len + chunk - 1) / chunk;
  if (n_chunks > 1 && (size_t)n_chunks * n_q * head_dim > part_floats) {
    chunk = seq_len;   // not enough scratch: single chunk
    n_chunks = 1;
  }
  dim3 grid(n_chunks, n_kv, (q_per_kv + kVHeads - 1) / kVHeads);
  size_t smem = (size_t)kVHeads * chunk * sizeof(float);
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(vsum_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem);
    if (e != cudaSuccess) return e;
  }
  vsum_kernel<<<grid, head_dim, smem, s>>>(d_buf, g, layer, d_w, q_per_kv, head_dim, seq_len,
                                           chunk, d_out, d_part, n_q);
  if (n_chunks > 1) {
    size_t n = (size_t)n_q * head_dim;
    vsum_combine_kernel<<<(int)((n + 255) / 256), 256, 0, s>>>(d_part, n_chunks, n, d_out);
  }
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
  size_t pf = vsum_scratch_floats(c->geom, n_q, c->seq_len);
  float *d_part = nullptr;
  if (pf) {
    d_part = (float *)cache_scratch(c, pf * sizeof(float));
    if (!d_part) return EAKV_ERR_ALLOC;
  }
  return check_cuda(launch_vsum(c->geom, c->d_buf, layer, d_w, n_q, n_kv, c->seq_len, d_out,
                                d_part, pf, c->stream),
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
  size_t pf = vsum_scratch_floats(c->geom, n_q, c->seq_len);
  size_t nw_pad = (nw + 63) / 64 * 64, no_pad = (no + 63) / 64 * 64;
  float *d_w = (float *)cache_scratch(c, (nw_pad + no_pad + pf) * sizeof(float));
  if (!d_w) {
    fill_nan_host(output_out, no);
    return;
  }
  float *d_o = d_w + nw_pad;
  float *d_part = pf ? d_o + no_pad : nullptr;
  if ((nw && check_cuda(cudaMemcpyAsync(d_w, weights, nw * sizeof(float),
                                        cudaMemcpyHostToDevice, c->stream),
                        "attention_output: copy")) ||
      check_cuda(launch_vsum(c->geom, c->d_buf, layer, d_w, n_q, n_kv, c->seq_len, d_o, d_part,
                             pf, c->stream), "attention_output") ||
      check_cuda(cudaMemcpyAsync(output_out, d_o, no * sizeof(float), cudaMemcpyDeviceToHost,
                                 c->stream), "attention_output: copy") ||
      check_cuda(cudaStreamSynchronize(c->stream), "attention_output")) {
    fill_nan_host(output_out, no);
  }
}

}  // extern "C"
