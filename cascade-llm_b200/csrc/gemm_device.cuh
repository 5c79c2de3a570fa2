// tcgen05 (5th-generation tensor core) building blocks of the prefill GEMM:
// TMEM allocation, UMMA shared-memory / instruction descriptors, the MMA,
// its commit to an mbarrier, TMEM -> register loads, and the 2-D TMA tile
// load. Hand-written PTX for sm_100a; the descriptor bit layouts follow the
// PTX ISA "tcgen05 matrix descriptors" (shared memory descriptor: start
// address >> 4 in bits [0,14), leading byte offset >> 4 in [16,30), stride
// byte offset >> 4 in [32,46), version 1 in [46,48), layout type in [61,64);
// instruction descriptor for kind::f16: D format [4,6), A/B format [7,10) /
// [10,13), A/B major [15] / [16], N >> 3 in [17,23), M >> 4 in [24,29)).
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>

#include "common.cuh"

namespace cb {

// cuTensorMapEncodeTiled through the runtime's driver entry point (host;
// null when the driver does not provide it).
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder();

// ----------------------------------------------------------------- TMEM
// Allocate `cols` TMEM columns (power of two >= 32) for this CTA; the base
// address is written to shared memory. Executed by one whole warp.
__device__ __forceinline__ void tmem_alloc(uint32_t* smem_dst, uint32_t cols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_dst)),
               "r"(cols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t cols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(cols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// ----------------------------------------------------------- descriptors
// K-major operand tile in shared memory written by TMA with 128-byte
// swizzle: rows of 128 bytes (64 bf16 of K), 8-row swizzle atoms 1024 bytes
// apart. The tile must start on a 1024-byte boundary; the k-th 16-element
// step of the MMA starts 32*k bytes further (the swizzle acts on the
// absolute address bits).
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= uint64_t((smem_addr >> 4) & 0x3FFFu);  // start address
  d |= uint64_t(1) << 16;                      // leading byte offset (unused for swizzled K-major): 16 B
  d |= uint64_t(1024 >> 4) << 32;              // stride byte offset: 8 rows x 128 B
  d |= uint64_t(1) << 46;                      // descriptor version (sm_100)
  d |= uint64_t(2) << 61;                      // layout: 128-byte swizzle
  return d;
}
// kind::f16 instruction descriptor: BF16 A and B (K-major), FP32 D, M x N.
__host__ __device__ constexpr uint32_t umma_idesc_bf16(int M, int N) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (uint32_t(N >> 3) << 17) | (uint32_t(M >> 4) << 24);
}

// D[tmem] (+)= A[smem] * B[smem]^T for one K=16 step, issued by one thread.
__device__ __forceinline__ void umma_bf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive once on `bar` when every tcgen05.mma issued so far by this thread
// has completed (its shared-memory operands may then be overwritten).
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

// 32 consecutive fp32 columns of this thread's TMEM lane (warp w reads lanes
// 32*(w%4) .. +31; lane offset in bits [16,32) of the address).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// ------------------------------------------------------------------ TMA
// 2-D tiled bulk tensor load global -> shared (this CTA), completing its
// bytes on `bar`. x is the innermost (K) coordinate in elements; it is always
// a multiple of 64 bf16 here (128 bytes). The tile goes to this CTA only.
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
          "r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

}  // namespace cb
