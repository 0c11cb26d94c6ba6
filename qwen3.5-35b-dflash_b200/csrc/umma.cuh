// Blackwell tensor-core (tcgen05) primitives: tensor-memory allocation, shared-memory
// matrix descriptors, the single-thread MMA issue, its completion through an mbarrier,
// and tensor-memory loads for the epilogue.  Only the forms the dense expert kernels use:
// one CTA (cta_group::1), kind::f16 with fp16 or bf16 operands and fp32 accumulators, K-major
// operands in the canonical no-swizzle layout.
//
// Canonical K-major layout without swizzle, as the descriptor describes it: the matrix
// (rows = M or N, K) is cut into "core matrices" of 8 rows x 16 bytes (8 fp16 of K),
// each stored as 128 contiguous bytes (row r of the core at byte 16 r).  Here core
// (row group g, K octet o) of a tile with KO octets along K sits at byte (g * KO + o) * 128,
// so the leading byte offset (between the two K octets one K = 16 step reads) is 128
// and the stride byte offset (between row groups) is KO * 128; step s of a tile starts at
// byte s * 256.
#pragma once

#include "bulk_ring.cuh"

namespace qw {
namespace umma {

// Shared-memory matrix descriptor (sm_100): start address, leading and stride byte
// offsets (all >> 4), version 1, no swizzle.
__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFF);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFF) << 16;
  d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFF) << 32;
  d |= static_cast<uint64_t>(1) << 46;   // descriptor version (sm_100)
  return d;                               // base offset 0, layout type 0 (no swizzle)
}

// Instruction descriptor of kind::f16: A and B both fp16 or both bf16 (K-major), fp32
// D, M x N.
__host__ __device__ constexpr uint32_t idesc_16(int m, int n, bool bf16) {
  return (1u << 4)                                              // D format fp32
         | (static_cast<uint32_t>(bf16) << 7) | (static_cast<uint32_t>(bf16) << 10)   // A, B format
         | (static_cast<uint32_t>(n >> 3) << 17)                // N / 8
         | (static_cast<uint32_t>(m >> 4) << 24);               // M / 16
}

// One warp: allocate `ncols` (power of two >= 32) tensor-memory columns; the base
// address is written to *dst (shared memory).
__device__ __forceinline__ void tmem_alloc(uint32_t* dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n"
               ::"r"(smem_u32(dst)), "r"(ncols) : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
}

// The allocating warp: free them again.
__device__ __forceinline__ void tmem_free(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void fence_before_sync() {
  asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
}
__device__ __forceinline__ void fence_after_sync() {
  asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
}

// One thread: D[tmem] (+)= A[smem] * B[smem]^T, K = 16.
__device__ __forceinline__ void mma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                        bool accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n"
      ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(static_cast<uint32_t>(accumulate))
      : "memory");
}

// One thread: one arrival on `bar` once every MMA it issued before has completed.
__device__ __forceinline__ void commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n"
               ::"r"(smem_u32(bar)) : "memory");
}

// Whole warp: 16 consecutive fp32 columns of this warp's 32 tensor-memory lanes (lane
// i of the warp reads lane (32 * (warp % 4) + i) of the accumulator).
__device__ __forceinline__ void ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
  asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

}  // namespace umma
}  // namespace qw
