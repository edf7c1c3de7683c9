// Tensor-core (tcgen05 / TMEM) and tiled-TMA helpers for sm_100a kernels.
//
// Conventions used by the kernels of this library:
// * operands are bf16 / fp16 (kind::f16) or fp32 (kind::tf32), staged in
//   shared memory by tiled TMA loads with the 128-byte swizzle: a box row is
//   128 bytes (64 16-bit or 32 fp32 elements) and rows come in 1024-byte
//   groups of eight; every operand tile starts on a 1024-byte boundary;
// * one MMA is M = 128 x N x K = 16, single CTA (cta_group::1), fp32
//   accumulation in tensor memory (TMEM), lane = row of D, column = column of D;
// * no multicast: every TMA load fills only this CTA's shared memory.
#pragma once

#include <cuda.h>
#include <stdint.h>

#include "qcc_common.cuh"

namespace qcc {

// ---------------------------------------------------------------------------
// Tiled TMA loads (2-D and 3-D tensor maps), completion on an mbarrier.
// ---------------------------------------------------------------------------

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int c0, int c1, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_addr(bar))
      : "memory");
}

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int c0, int c1, int c2,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::
          "r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(smem_addr(bar))
      : "memory");
}

// The same loads with an L2 cache policy (createpolicy) for the source lines.
__device__ __forceinline__ void tma_load_2d_hint(void* dst, const CUtensorMap* map, int c0, int c1, uint64_t* bar,
                                                 uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1, {%2, %3}], "
      "[%4], %5;" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_addr(bar)), "l"(policy)
      : "memory");
}

__device__ __forceinline__ void tma_load_3d_hint(void* dst, const CUtensorMap* map, int c0, int c1, int c2,
                                                 uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1, {%2, %3, "
      "%4}], [%5], %6;" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(smem_addr(bar)), "l"(policy)
      : "memory");
}

__device__ __forceinline__ void tma_prefetch_map(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ---------------------------------------------------------------------------
// Tensor memory.
// ---------------------------------------------------------------------------

// Warp-wide: allocates `ncols` TMEM columns (power of two, >= 32) and writes
// the base address to shared memory.
__device__ __forceinline__ void tmem_alloc(uint32_t* dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(dst)), "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tc_fence_before_sync() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after_sync() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Arrives once on `bar` when every tcgen05.mma issued so far by this thread
// has completed (and its shared-memory operands may be overwritten).
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
               : "memory");
}

// D[tmem] (+)= A[smem desc] x B[smem desc]^T, kind::f16 (bf16 or fp16 in, fp32 out).
__device__ __forceinline__ void tc_mma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                           uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// The same with kind::tf32: A and B hold fp32 values, of which the MMA uses
// the tf32 part (K = 8 per instruction, 32 bytes of a row as for kind::f16).
__device__ __forceinline__ void tc_mma_tf32(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// 32 consecutive fp32 columns of this thread's TMEM lane (32x32b shape: warp
// w reads lanes 32*(w%4) .. +31).  The wait is inside the same statement, so
// the registers are valid when it returns.
__device__ __forceinline__ void tmem_load32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// 16 consecutive fp32 columns of this thread's TMEM lane, waited for.
__device__ __forceinline__ void tmem_load16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15}, [%16];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// ---------------------------------------------------------------------------
// Descriptors.
// ---------------------------------------------------------------------------

// Shared-memory matrix descriptor for an operand without swizzle, built from
// 128-byte core matrices (8 rows of 16 bytes).  For both majors `sbo` is the
// byte distance between core matrices adjacent in M (or N) and `lbo` the
// distance between core matrices adjacent in K.  K-major: a core matrix is 8
// M rows x 8 K elements (rows 16 bytes apart); MN-major: 8 K rows x 8 M
// elements (K rows 16 bytes apart).
__device__ __forceinline__ uint64_t smem_desc_none(uint32_t addr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((addr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32;
  d |= 1ull << 46;  // descriptor version for sm_100; layout type 0: no swizzle
  return d;
}

// Shared-memory matrix descriptor for a 128-byte-swizzled operand tile.
// K-major: rows of 128 bytes, groups of 8 rows `sbo` bytes apart (1024 for a
// dense tile); `lbo` is unused.  MN-major: 64 contiguous MN elements per
// 128-byte row, K rows 128 bytes apart, groups of 8 K rows `sbo` bytes apart,
// the next 64 MN elements `lbo` bytes further.
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t addr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((addr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32;
  d |= 1ull << 46;  // descriptor version for sm_100
  d |= 2ull << 61;  // 128-byte swizzle
  return d;
}

// Operand formats of kind::f16 and kind::tf32 (A and B use the same one).
constexpr int kFmtF16 = 0, kFmtBF16 = 1, kFmtTF32 = 2;

// The same for an MN-major fp32 operand of kind::tf32, which takes the
// 128-byte swizzle with 32-byte atoms (TMA CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B):
// 32 MN elements per 128-byte row, K rows 128 bytes apart in groups of four,
// `sbo` bytes between the groups of four (512 for a dense tile), `lbo` bytes
// between consecutive 32-element MN groups.
__device__ __forceinline__ uint64_t smem_desc_sw128_atom32(uint32_t addr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((addr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32;
  d |= 1ull << 46;  // descriptor version for sm_100
  d |= 1ull << 61;  // 128-byte swizzle, 32-byte atoms
  return d;
}

// Instruction descriptor of tcgen05.mma kind::f16 / kind::tf32 with fp32
// accumulation; `fmt` is one of the formats above.
__host__ __device__ constexpr uint32_t idesc_f32acc(int m, int n, int fmt, bool a_mn_major, bool b_mn_major) {
  return (1u << 4) |                                                          // D format: f32
         (static_cast<uint32_t>(fmt) << 7) | (static_cast<uint32_t>(fmt) << 10) |  // A, B format
         ((a_mn_major ? 1u : 0u) << 15) | ((b_mn_major ? 1u : 0u) << 16) |
         (static_cast<uint32_t>(n >> 3) << 17) | (static_cast<uint32_t>(m >> 4) << 24);
}

__host__ __device__ constexpr uint32_t idesc_f16_f32(int m, int n, bool bf16, bool a_mn_major, bool b_mn_major) {
  return idesc_f32acc(m, n, bf16 ? kFmtBF16 : kFmtF16, a_mn_major, b_mn_major);
}

}  // namespace qcc
