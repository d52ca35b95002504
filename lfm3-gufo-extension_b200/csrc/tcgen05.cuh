// tcgen05 building blocks of the prompt attention kernel: shared-memory
// operand descriptors of the 64-byte-swizzled layouts TMA writes,
// instruction descriptors of kind::f16, MMA issue and commit, tensor-memory
// allocation, loads and stores.
#pragma once
#include <stdint.h>

#include "common.cuh"

namespace lfm3 {
namespace tc {

// Byte offset of 16-byte piece `piece` (elements 8 piece .. 8 piece + 7) of
// row `row` in a K-major operand tile of 64-byte rows (32 fp16) with the
// 64-byte swizzle, the layout TMA writes with CU_TENSOR_MAP_SWIZZLE_64B.
__device__ __forceinline__ uint32_t sw64_offset(int row, int piece) {
  return uint32_t(row * 64 + ((piece ^ ((row >> 1) & 3)) << 4));
}

// Shared-memory matrix descriptor of such a tile: 8-row groups 512 bytes
// apart. Adding 2 advances K by 16 elements (32 bytes).
__device__ __forceinline__ uint64_t sw64_desc(const void* p) {
  const uint32_t addr = smem_addr(p);
  return uint64_t((addr >> 4) & 0x3FFF) | (uint64_t(1) << 16) |
         (uint64_t(512 >> 4) << 32) | (uint64_t(1) << 46) |
         (uint64_t(4) << 61);
}

// Descriptor of an MN-major operand in the same 64-byte-swizzled tiles: each
// 64-byte row holds 32 consecutive M (or N) elements of one K index, 8-row
// groups 512 bytes apart along K, and the 32-element blocks of M (N)
// `block_bytes` apart. Adding 64 advances K by 16 rows (1024 bytes).
__device__ __forceinline__ uint64_t sw64_mn_desc(const void* p,
                                                 uint32_t block_bytes) {
  const uint32_t addr = smem_addr(p);
  return uint64_t((addr >> 4) & 0x3FFF) |
         (uint64_t((block_bytes >> 4) & 0x3FFF) << 16) |
         (uint64_t(512 >> 4) << 32) | (uint64_t(1) << 46) |
         (uint64_t(4) << 61);
}

// Instruction descriptor of kind::f16: A and B fp16 K-major, D fp32, M x N.
// b_mn_major reads B (N x K) from an MN-major tile instead.
constexpr uint32_t f16_idesc(int m, int n, bool b_mn_major = false) {
  return (1u << 4) | (uint32_t(b_mn_major) << 16) | (uint32_t(n >> 3) << 17) |
         (uint32_t(m >> 4) << 24);
}

__device__ __forceinline__ void fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

// D (tensor memory) = A B^T (+ D when accumulate), A and B from shared
// memory descriptors; issued by one thread.
__device__ __forceinline__ void mma(uint32_t d_tmem, uint64_t a, uint64_t b,
                                    uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(
          d_tmem),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrives on bar once every MMA this thread issued before has completed.
__device__ __forceinline__ void commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 "
      "[%0];" ::"r"(smem_addr(bar))
      : "memory");
}

// 32 consecutive 32-bit columns of this thread's lane (warp-wide; a warp
// reaches the 32 lanes of its quarter, warp % 4).
__device__ __forceinline__ void ld32(uint32_t taddr, uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, "
      "[%32];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]),
        "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]), "=r"(v[9]),
        "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]),
        "=r"(v[15]), "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]),
        "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]),
        "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]),
        "=r"(v[30]), "=r"(v[31])
      : "r"(taddr));
}
__device__ __forceinline__ void st32(uint32_t taddr, const uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::
          "r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]),
      "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]),
      "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]), "r"(v[17]),
      "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]),
      "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]), "r"(v[29]),
      "r"(v[30]), "r"(v[31])
      : "memory");
}
__device__ __forceinline__ void wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// Whole-warp tensor-memory allocation of `columns` (a power of two >= 32);
// the base address lands in *slot.
__device__ __forceinline__ void alloc(uint32_t* slot, int columns) {
  asm volatile(
      "tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::
          "r"(smem_addr(slot)),
      "r"(columns));
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
}
__device__ __forceinline__ void dealloc(uint32_t base, int columns) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(
                   base),
               "r"(columns));
}

}  // namespace tc
}  // namespace lfm3
