// io.cu - .eakv save/load (reference src/io.c:1-160), same file layout:
//
//   [512-byte header][u64 offset table: K, V per layer][pad to 64]
//   per (layer, K/V): [nibbles n_groups*32][scales n_groups f32]
//                     [biases n_groups f32][pad to 64]
//
// with n_groups = n_kv_heads * head_dim * seq_len / 64 in dense
// [head][position][group] order and the header fields at the byte offsets
// of the reference's packed struct (io.c:11-28): magic "EAKV" @0,
// version u16 @4 (= 1), quant_scheme u16 @6, group_size u32 @8 (= 64),
// orig_dtype u16 @12, n_layers u32 @14, n_heads u32 @18, head_dim u32 @22,
// seq_len u32 @26, max_seq_len u32 @30 (written = seq_len), compression
// i16 @34, model_hash[32] @36, tokenizer_hash[32] @68, checksum u64 @100.
//
// The reference copies n_groups*32 bytes flat out of its in-memory block,
// whose heads are max_seq_len positions apart, so its files are dense (and
// loadable) only when seq_len == max_seq_len. This writer always emits the
// dense layout its loader expects; for seq_len == max_seq_len the bytes are
// identical to the reference's.
//
// The device pages are gathered into / scattered from a dense staging
// block by the pack/unpack kernels below, one (layer, K/V) block at a time.
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "internal.cuh"

namespace eakv {
namespace {

constexpr size_t kHeader = 512;

size_t align64(size_t x) { return (x + 63) & ~(size_t)63; }

// dense block <-> pages of one (layer, kv). One warp per group.
template <bool kPack>
__global__ void pack_kernel(uint8_t *pages, PageGeom g, int layer, int kv, int seq_len,
                            uint8_t *dense, size_t n_groups) {
  const int lane = threadIdx.x & 31;
  const size_t warps = (size_t)gridDim.x * (blockDim.x / 32);
  uint8_t *w = dense;
  float *sc = reinterpret_cast<float *>(dense + n_groups * 32);
  float *bi = sc + n_groups;
  for (size_t gi = (size_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5); gi < n_groups;
       gi += warps) {
    const size_t per_head = (size_t)seq_len * g.gpd;
    const int h = (int)(gi / per_head);
    const size_t r = gi - (size_t)h * per_head;
    const int t = (int)(r / g.gpd);
    const int grp = (int)(r - (size_t)t * g.gpd);
    const int page = t / kPagePositions, pip = t % kPagePositions;
    uint8_t *pp = pages + page_index(g, layer, kv, h, page) * g.page_bytes;
    const int slot = pip * g.gpd + grp;
    float2 *sb = reinterpret_cast<float2 *>(pp + g.nib_bytes) + slot;
    if (kPack) {
      w[gi * 32 + lane] = pp[(size_t)slot * 32 + lane];
      if (lane == 0) {
        float2 v = *sb;
        sc[gi] = v.x;
        bi[gi] = v.y;
      }
    } else {
      pp[(size_t)slot * 32 + lane] = w[gi * 32 + lane];
      if (lane == 0) {
        *sb = make_float2(sc[gi], bi[gi]);
        if (kv == 1) vexp_raise(vexp_table(pages, g), layer * g.n_heads + h, sc[gi]);
      }
    }
  }
}

int run_pack(bool pack, eakv_cache_t *c, int layer, int kv, uint8_t *d_dense, size_t n_groups) {
  if (n_groups == 0) return EAKV_OK;
  size_t blocks = (n_groups + 7) / 8;
  if (blocks > 4096) blocks = 4096;
  if (pack)
    pack_kernel<true><<<(int)blocks, 256, 0, c->stream>>>(c->d_buf, c->geom, layer, kv,
                                                          c->seq_len, d_dense, n_groups);
  else
    pack_kernel<false><<<(int)blocks, 256, 0, c->stream>>>(c->d_buf, c->geom, layer, kv,
                                                           c->seq_len, d_dense, n_groups);
  return check_cuda(cudaGetLastError(), pack ? "save: pack" : "load: unpack");
}

void put16(uint8_t *p, uint16_t v) { memcpy(p, &v, 2); }
void put32(uint8_t *p, uint32_t v) { memcpy(p, &v, 4); }
uint16_t get16(const uint8_t *p) { uint16_t v; memcpy(&v, p, 2); return v; }
uint32_t get32(const uint8_t *p) { uint32_t v; memcpy(&v, p, 4); return v; }

void write_zeros(FILE *f, size_t n) {
  static const uint8_t z[64] = {0};
  while (n) {
    size_t k = n < 64 ? n : 64;
    fwrite(z, 1, k, f);
    n -= k;
  }
}

}  // namespace
}  // namespace eakv

using namespace eakv;

extern "C" {

int eakv_cache_save(const eakv_cache_t *cc, const char *path) {
  clear_error();
  if (!cc || !path) return EAKV_ERR_INVALID;
  eakv_cache_t *c = const_cast<eakv_cache_t *>(cc);
  if (c->head_dim % 64 != 0) {
    set_error(EAKV_ERR_INVALID, "save: head_dim %d is not a multiple of 64", c->head_dim);
    return EAKV_ERR_INVALID;
  }
  FILE *f = fopen(path, "wb");
  if (!f) return EAKV_ERR_IO;
  DeviceGuard g(c->device);

  const size_t n_groups = (size_t)c->n_kv_heads * c->head_dim * c->seq_len / 64;
  const size_t block_raw = n_groups * 40;
  const size_t block_aligned = align64(block_raw);

  uint8_t hdr[kHeader];
  memset(hdr, 0, sizeof hdr);
  memcpy(hdr, "EAKV", 4);
  put16(hdr + 4, 1);                      // version
  put16(hdr + 6, 0);                      // quant_scheme
  put32(hdr + 8, 64);                     // group_size
  put16(hdr + 12, 0);                     // orig_dtype
  put32(hdr + 14, (uint32_t)c->n_layers);
  put32(hdr + 18, (uint32_t)c->n_kv_heads);
  put32(hdr + 22, (uint32_t)c->head_dim);
  put32(hdr + 26, (uint32_t)c->seq_len);
  put32(hdr + 30, (uint32_t)c->seq_len);  // max_seq_len as written by the reference
  fwrite(hdr, 1, kHeader, f);

  const size_t idx_bytes = (size_t)c->n_layers * 2 * 8;
  const size_t data_start = align64(kHeader + idx_bytes);
  size_t cur = data_start;
  for (int l = 0; l < c->n_layers; l++) {
    uint64_t k_off = cur;
    cur += block_aligned;
    uint64_t v_off = cur;
    cur += block_aligned;
    fwrite(&k_off, 8, 1, f);
    fwrite(&v_off, 8, 1, f);
  }
  write_zeros(f, data_start - (kHeader + idx_bytes));

  int rc = EAKV_OK;
  if (block_raw) {
    uint8_t *d_dense = (uint8_t *)cache_scratch(c, block_raw);
    uint8_t *h_dense = (uint8_t *)malloc(block_raw);
    if (!d_dense || !h_dense) rc = EAKV_ERR_ALLOC;
    for (int l = 0; l < c->n_layers && rc == EAKV_OK; l++) {
      for (int kv = 0; kv < 2 && rc == EAKV_OK; kv++) {
        rc = run_pack(true, c, l, kv, d_dense, n_groups);
        if (rc) break;
        rc = check_cuda(cudaMemcpyAsync(h_dense, d_dense, block_raw, cudaMemcpyDeviceToHost,
                                        c->stream), "save: copy");
        if (rc) break;
        rc = check_cuda(cudaStreamSynchronize(c->stream), "save");
        if (rc) break;
        if (fwrite(h_dense, 1, block_raw, f) != block_raw) rc = EAKV_ERR_IO;
        write_zeros(f, block_aligned - block_raw);
      }
    }
    free(h_dense);
  }
  if (fclose(f) != 0 && rc == EAKV_OK) rc = EAKV_ERR_IO;
  return rc;
}

int eakv_cache_load(const char *path, eakv_cache_t **out) {
  clear_error();
  if (!path || !out) return EAKV_ERR_INVALID;
  FILE *f = fopen(path, "rb");
  if (!f) return EAKV_ERR_IO;
  uint8_t hdr[kHeader];
  if (fread(hdr, 1, kHeader, f) != kHeader) {
    fclose(f);
    return EAKV_ERR_FORMAT;
  }
  if (memcmp(hdr, "EAKV", 4) != 0 || get16(hdr + 4) != 1) {
    fclose(f);
    return EAKV_ERR_FORMAT;
  }
  const int nl = (int)get32(hdr + 14), nh = (int)get32(hdr + 18), hd = (int)get32(hdr + 22);
  const int sl = (int)get32(hdr + 26);
  eakv_cache_t *c = eakv_cache_create(nl, nh, hd, sl);
  if (!c) {
    fclose(f);
    return EAKV_ERR_ALLOC;
  }
  DeviceGuard g(c->device);
  const size_t n_groups = (size_t)nh * hd * sl / 64;
  const size_t block_raw = n_groups * 40;
  const size_t idx_bytes = (size_t)nl * 2 * 8;
  uint64_t *offsets = (uint64_t *)malloc(idx_bytes);
  uint8_t *h_dense = (uint8_t *)malloc(block_raw ? block_raw : 1);
  uint8_t *d_dense = block_raw ? (uint8_t *)cache_scratch(c, block_raw) : nullptr;
  int rc = EAKV_OK;
  if (!offsets || !h_dense || (block_raw && !d_dense)) rc = EAKV_ERR_ALLOC;
  if (rc == EAKV_OK && fread(offsets, 1, idx_bytes, f) != idx_bytes) rc = EAKV_ERR_FORMAT;
  c->seq_len = sl;   // pack geometry uses the file's length
  for (int l = 0; l < nl && rc == EAKV_OK; l++) {
    for (int kv = 0; kv < 2 && rc == EAKV_OK; kv++) {
      if (fseek(f, (long)offsets[l * 2 + kv], SEEK_SET) != 0 ||
          fread(h_dense, 1, block_raw, f) != block_raw) {
        rc = EAKV_ERR_FORMAT;
        break;
      }
      if (block_raw == 0 || hd % 64 != 0) continue;
      rc = check_cuda(cudaMemcpyAsync(d_dense, h_dense, block_raw, cudaMemcpyHostToDevice,
                                      c->stream), "load: copy");
      if (rc) break;
      rc = run_pack(false, c, l, kv, d_dense, n_groups);
      if (rc) break;
      rc = check_cuda(cudaStreamSynchronize(c->stream), "load");
    }
  }
  free(offsets);
  free(h_dense);
  fclose(f);
  if (rc != EAKV_OK) {
    eakv_cache_free(c);
    return rc;
  }
  *out = c;
  return EAKV_OK;
}

}  // extern "C"
