// umma.cuh - fifth-generation tensor core (tcgen05) primitives for sm_100a,
// written as inline PTX: tensor-memory allocation, shared-memory matrix
// descriptors, the integer MMA (kind::i8) with its operands in shared or
// tensor memory, the commit to an mbarrier, and tensor-memory loads/stores.
//
// Conventions used by the decode kernel that includes this file:
// * Every shared-memory operand is an array of rows of 32 or 64 bytes in the
//   hardware's 32B/64B swizzle: 16-byte chunk c of row r sits at chunk
//   c ^ ((r >> 2) & 1) (32-byte rows) or c ^ ((r >> 1) & 3) (64-byte rows),
//   and every such array starts 1024-byte aligned. The same image serves as
//   a K-major operand (rows = M or N, the row's bytes = K) or an MN-major
//   one (rows = K, the row's bytes = M or N), depending on the descriptor.
// * Tensor-memory addresses carry the lane in bits 31..16 and the column in
//   bits 15..0; warp w of a CTA reaches lanes 32 (w % 4) .. 32 (w % 4) + 31.
#pragma once
#include <stdint.h>

namespace eakv {
namespace umma {

// Byte offset of (row, byte) in a swizzled array of `row_bytes`-byte rows.
__host__ __device__ __forceinline__ uint32_t swz_off(uint32_t row, uint32_t byte,
                                                     uint32_t row_bytes) {
  const uint32_t chunk = byte >> 4;
  const uint32_t x = row_bytes == 64 ? ((row >> 1) & 3) : ((row >> 2) & 1);
  return row * row_bytes + ((chunk ^ x) << 4) + (byte & 15);
}

constexpr uint32_t kLayoutSW64 = 4;   // descriptor layout codes (bits 61..63)
constexpr uint32_t kLayoutSW32 = 6;

// Shared-memory matrix descriptor: start address, leading-dimension and
// stride byte offsets (all in bytes, multiples of 16), sm_100 version 1,
// base offset 0 (arrays are 1024-byte aligned), swizzle layout.
//   K-major  (rows = M/N): SBO = stride of 8-row groups; LBO unused (16).
//   MN-major (rows = K):   LBO = stride of 32/64-byte M/N atoms; SBO = stride
//                          of 8-row (K) groups.
__device__ __forceinline__ uint64_t sdesc(uint32_t saddr, uint32_t lbo, uint32_t sbo,
                                          uint32_t layout) {
  uint64_t d = (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)layout << 61;
  return d;
}

// Instruction descriptor of an integer MMA (s32 accumulator): M x N tile,
// A/B signed (1) or unsigned (0), A/B MN-major (1) or K-major (0).
__host__ __device__ constexpr uint32_t idesc_i8(int M, int N, int a_signed, int b_signed,
                                                int a_mn, int b_mn) {
  return (2u << 4) | ((uint32_t)a_signed << 7) | ((uint32_t)b_signed << 10) |
         ((uint32_t)a_mn << 15) | ((uint32_t)b_mn << 16) | ((uint32_t)(N >> 3) << 17) |
         ((uint32_t)(M >> 4) << 24);
}

// ---- tensor-memory allocation (one whole warp) ---------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t smem_slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
               ::"r"(smem_slot), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;"
               ::"r"(taddr), "r"(ncols) : "memory");
}

// ---- ordering of tcgen05 operations around thread synchronization ---------------
__device__ __forceinline__ void fence_before_sync() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void fence_after_sync() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// ---- MMA: D[tmem] (+)= A * B, s32 accumulate (issued by one thread) --------------
// A and B in shared memory.
__device__ __forceinline__ void mma_i8_ss(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                          uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n\t}"
      ::"r"(d_tmem), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(0u)
      : "memory");
}
// A in tensor memory (K-major: lane = row, four int8 per 32-bit column), B in
// shared memory.
__device__ __forceinline__ void mma_i8_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc,
                                          uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], [%1], %2, %3, {%5, %5, %5, %5}, p;\n\t}"
      ::"r"(d_tmem), "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(0u)
      : "memory");
}
// Arrive once on the mbarrier when every MMA this thread issued before has
// completed (and its operand reads with it).
__device__ __forceinline__ void mma_commit(uint32_t mbar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
      ::"r"(mbar) : "memory");
}

// ---- tensor-memory loads and stores (whole warp, lane = thread) --------------------
#define EAKV_R8(a, i) "=r"(a[i]), "=r"(a[i + 1]), "=r"(a[i + 2]), "=r"(a[i + 3]), \
                      "=r"(a[i + 4]), "=r"(a[i + 5]), "=r"(a[i + 6]), "=r"(a[i + 7])
#define EAKV_W8(a, i) "r"(a[i]), "r"(a[i + 1]), "r"(a[i + 2]), "r"(a[i + 3]), \
                      "r"(a[i + 4]), "r"(a[i + 5]), "r"(a[i + 6]), "r"(a[i + 7])

// 16 consecutive 32-bit columns of this thread's lane.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : EAKV_R8(r, 0), EAKV_R8(r, 8)
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t (&r)[8]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
      : EAKV_R8(r, 0)
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : EAKV_R8(r, 0), EAKV_R8(r, 8), EAKV_R8(r, 16), EAKV_R8(r, 24)
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 "
      "[%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};"
      ::"r"(taddr), EAKV_W8(r, 0), EAKV_W8(r, 8)
      : "memory");
}
__device__ __forceinline__ void tmem_st4(uint32_t taddr, uint4 v) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1,%2,%3,%4};"
               ::"r"(taddr), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}
__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}
#undef EAKV_R8
#undef EAKV_W8

}  // namespace umma
}  // namespace eakv
