// tcgen05.cuh - 5th-generation tensor core primitives for sm_100a (inline PTX):
// tensor-memory allocation, UMMA shared-memory and instruction descriptors,
// the single-thread MMA issue, its commit to an mbarrier, and TMEM loads.
//
// Operand layout used throughout: K-major, no swizzle ("interleaved"): a
// tile of R rows x K bf16 is stored as core matrices of 8 rows x 16 bytes;
// the core matrix of row group g and 16-byte K chunk c starts at
// g * sbo + c * lbo, and row r of it at + (r % 8) * 16.
#pragma once

#include <stdint.h>

namespace cnnue {
namespace tc {

// Shared-memory matrix descriptor (tcgen05 format): start address >> 4 in
// bits [0,14), leading-dimension byte offset >> 4 in [16,30), stride-dimension
// byte offset >> 4 in [32,46), version 1 in [46,48), base offset 0, relative
// LBO mode, layout type in [61,64) (0 = no swizzle).
__device__ __forceinline__ uint64_t smem_desc(uint32_t smem_addr, uint32_t lbo_bytes, uint32_t sbo_bytes,
                                              uint32_t layout = 0) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr >> 4) & 0x3fffu);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3fffu) << 16;
  d |= (uint64_t)((sbo_bytes >> 4) & 0x3fffu) << 32;
  d |= (uint64_t)1u << 46;
  d |= (uint64_t)(layout & 7u) << 61;
  return d;
}

// Layout type of a K-major tile whose rows are 128-byte lines with the
// 16-byte chunk index XORed with (line % 8) inside each 1024-byte block (the
// TMA 128B swizzle); a K step of 16 bf16 advances the start address by 32 B.
constexpr uint32_t kSwizzle128B = 2;

// 2-D tiled TMA load (no multicast) of the box at {x, y} (x innermost, in
// elements; y may be negative or past the end: those rows fill with zeros)
// into this CTA's shared memory, completing its bytes on `bar`.
__device__ __forceinline__ void tma_load_2d(uint32_t dst_smem_addr, const void* tmap, int x, int y,
                                            uint32_t bar_smem_addr) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
      ::"r"(dst_smem_addr), "l"(reinterpret_cast<uint64_t>(tmap)), "r"(x), "r"(y), "r"(bar_smem_addr)
      : "memory");
}

// Instruction descriptor of kind::f16 with bf16 A and B, fp32 accumulator,
// both operands K-major: D format F32 (bits [4,6) = 1), A format BF16 ([7,10)
// = 1), B format BF16 ([10,13) = 1), N >> 3 in [17,23), M >> 4 in [24,29).
__host__ __device__ constexpr uint32_t idesc_bf16_f32(int m, int n) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

// D[tmem] (+)= A[smem] * B[smem]^T, issued by one thread.
__device__ __forceinline__ void mma_bf16(uint32_t tmem_d, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(tmem_d), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate));
}

// Instruction descriptor of kind::i8 with unsigned 8-bit A, signed 8-bit B,
// int32 accumulator, both operands K-major: D format S32 (bits [4,6) = 2), A
// format U8 ([7,10) = 0), B format S8 ([10,13) = 1), N >> 3 in [17,23), M >> 4
// in [24,29).
__host__ __device__ constexpr uint32_t idesc_u8s8_s32(int m, int n) {
  return (2u << 4) | (0u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

// D[tmem] (+)= A[smem] * B[smem]^T for 8-bit integers, issued by one thread.
__device__ __forceinline__ void mma_i8(uint32_t tmem_d, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(tmem_d), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate));
}

// Arrives once on `bar` when every MMA this thread issued before has completed.
__device__ __forceinline__ void commit(uint32_t bar_smem_addr) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar_smem_addr)
               : "memory");
}

// Tensor-memory allocation of `cols` columns (a power of two >= 32) by one
// whole warp; the base address is written to shared memory at dst.
__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem_addr, uint32_t cols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem_addr), "r"(cols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t tmem_addr, uint32_t cols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_addr), "r"(cols) : "memory");
}

__device__ __forceinline__ void fence_before_sync() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after_sync() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// 32 consecutive fp32 columns of this thread's TMEM lane (warp w of a
// warpgroup reads lanes 32w..32w+31; the address carries lane << 16 | column).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
        "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]),
        "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]),
        "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
      : "r"(taddr));
}

// 16 consecutive 32-bit columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
        "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
      : "r"(taddr));
}

}  // namespace tc
}  // namespace cnnue
