// tcgen05 (5th-generation tensor core) building blocks for sm_100a: tensor
// memory allocation, shared-memory matrix descriptors, the instruction
// descriptor of a bf16 x bf16 -> fp32 MMA, MMA issue and completion, and
// tensor-memory loads / stores.
//
// Conventions (CTA-local forms only; one CTA, cta_group::1):
//  * Operand tiles live in shared memory in the 128-byte swizzled layout that
//    a TMA load with CU_TENSOR_MAP_SWIZZLE_128B writes: rows of 128 bytes
//    (64 bf16), the 16-byte chunk c of row r stored at chunk c ^ (r % 8), each
//    8-row atom 1024 bytes and 1024-byte aligned.  A tile whose contiguous
//    extent is 128 elements is two such regions, one per 64-element block.
//  * K-major operand (K contiguous within a row; rows = M or N index):
//    descriptor start = region of the 64-wide K block + 32 bytes per 16-wide
//    K step inside it, SBO = 1024 bytes (next 8 rows), LBO unused.
//  * MN-major operand (M or N contiguous; rows = K index): descriptor start =
//    16 K rows (2048 bytes) per K step, SBO = 1024 bytes (next 8 K rows),
//    LBO = bytes between the regions of consecutive 64-wide MN blocks.
//  * D (M = 128) row i is tensor-memory lane i, column n is column base + n;
//    warp w of a warpgroup reads lanes [32 (w % 4), 32 (w % 4) + 32).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "ema_common.cuh"

namespace emab {
namespace tc {

// ---- shared-memory layout helpers ----------------------------------------
// Byte offset of element (row, col) of a 64-column bf16 region in the
// 128-byte swizzled layout (region base 1024-byte aligned).
__device__ __forceinline__ uint32_t sw128_offset(int row, int col) {
  const uint32_t o = static_cast<uint32_t>(row) * 128u + static_cast<uint32_t>(col) * 2u;
  return o ^ (((o >> 7) & 7u) << 4);
}

// Store 16 floats as bf16 into a swizzled 64-column region at (row, col0..col0+15).
__device__ __forceinline__ void st_sw16(unsigned char* region, int row, int col0, const float (&v)[16]) {
  uint4 a, b;
  a.x = pack_pair<__nv_bfloat16>(make_float2(v[0], v[1]));
  a.y = pack_pair<__nv_bfloat16>(make_float2(v[2], v[3]));
  a.z = pack_pair<__nv_bfloat16>(make_float2(v[4], v[5]));
  a.w = pack_pair<__nv_bfloat16>(make_float2(v[6], v[7]));
  b.x = pack_pair<__nv_bfloat16>(make_float2(v[8], v[9]));
  b.y = pack_pair<__nv_bfloat16>(make_float2(v[10], v[11]));
  b.z = pack_pair<__nv_bfloat16>(make_float2(v[12], v[13]));
  b.w = pack_pair<__nv_bfloat16>(make_float2(v[14], v[15]));
  *reinterpret_cast<uint4*>(region + sw128_offset(row, col0)) = a;
  *reinterpret_cast<uint4*>(region + sw128_offset(row, col0 + 8)) = b;
}
// Load 16 bf16 from a swizzled region as floats.
__device__ __forceinline__ void ld_sw16(const unsigned char* region, int row, int col0, float (&v)[16]) {
  const uint4 a = *reinterpret_cast<const uint4*>(region + sw128_offset(row, col0));
  const uint4 b = *reinterpret_cast<const uint4*>(region + sw128_offset(row, col0 + 8));
  const uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float2 f = cvt_pair<__nv_bfloat16>(w[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}

// Byte offset of row `row`, 16-byte chunk c (8 bf16) of a 128-byte swizzled tile.
__device__ __forceinline__ uint32_t chunk_off(int row, int c) {
  return static_cast<uint32_t>(row) * 128u + ((static_cast<uint32_t>(c) ^ (static_cast<uint32_t>(row) & 7u)) << 4);
}

// Bounded wait of a warp group: one warp polls, the group then meets at a
// named barrier.  False (for every thread of the group) on a timeout.
__device__ __forceinline__ bool group_wait(uint64_t* bar, uint32_t parity, uint32_t* status, bool poller,
                                           int bar_id, int nthreads, volatile uint32_t* fail) {
  if (poller && !mbar_wait_bounded(bar, parity, status) && (threadIdx.x & 31) == 0) *fail = 1u;
  named_sync(bar_id, nthreads);
  return *fail == 0u;
}

// ---- descriptors -----------------------------------------------------------
// Shared-memory matrix descriptor, 128-byte swizzle, version 1 (sm_100).
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t smem_addr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= 1ull << 46;            // version
  d |= 2ull << 61;            // SWIZZLE_128B
  return d;
}

// Instruction descriptor: bf16 A and B, fp32 D, M x N, majorness of A and B
// (false = K-major, true = MN-major).
__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N, bool a_mn, bool b_mn) {
  return (1u << 4)                       // D format f32
         | (1u << 7)                     // A format bf16
         | (1u << 10)                    // B format bf16
         | (static_cast<uint32_t>(a_mn) << 15) | (static_cast<uint32_t>(b_mn) << 16)
         | (static_cast<uint32_t>(N >> 3) << 17) | (static_cast<uint32_t>(M >> 4) << 24);
}

// ---- tensor memory ------------------------------------------------------------
// One full warp; the base address is written to *dst (shared memory).
__device__ __forceinline__ void tmem_alloc(uint32_t* dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst)), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void fence_before_sync() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void fence_after_sync() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// ---- MMA ---------------------------------------------------------------------
// D[tmem] (+)= A * B^T for one K = 16 step; issued by a single thread.
__device__ __forceinline__ void mma_bf16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                         bool accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(static_cast<uint32_t>(accumulate))
      : "memory");
}
// Arrive once on `bar` when every MMA this thread issued before has completed.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// ---- tensor memory <-> registers ------------------------------------------------
// 32 lanes x 16 consecutive 32-bit columns: thread t of the warp gets lane
// (address lane + t), columns [col, col + 16).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const float (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16};" ::"r"(taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
      "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
      "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])),
      "r"(__float_as_uint(v[11])), "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])),
      "r"(__float_as_uint(v[14])), "r"(__float_as_uint(v[15]))
      : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Tensor-memory address of (lane, column) relative to an allocation base.
__device__ __forceinline__ uint32_t tmem_at(uint32_t base, int lane, int col) {
  return base + (static_cast<uint32_t>(lane) << 16) + static_cast<uint32_t>(col);
}

// 2-D TMA load (CTA-local form) completing on `bar` by bytes.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_u32(bar))
      : "memory");
}

// 2-D TMA store (CTA-local source) into the global tensor; commit with bulk_commit().
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* src, int c0, int c1) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(c0), "r"(c1), "r"(smem_u32(src))
               : "memory");
}

}  // namespace tc
}  // namespace emab
