// tcgen05 (5th-generation tensor core) building blocks for the sm_100a int8 GEMMs (inline PTX): shared-memory matrix
// descriptors, the kind::i8 MMA, its commit to an mbarrier, and TMEM loads. Host side: 2-D TMA descriptors of
// K-major int8 matrices and the SM count.
#pragma once
#include <cuda.h>
#include <stdint.h>

namespace bnn {

// shared-memory matrix descriptor of a K-major tile with rows of SW bytes swizzled by SW (8-row groups of 8 * SW
// bytes); version 1 (sm_100), base offset 0 (stages are aligned to the swizzle repeat)
template <int SW>
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr) {
  constexpr uint64_t layout = SW == 128 ? 2 : SW == 64 ? 4 : 6;
  return (uint64_t)((addr & 0x3ffffu) >> 4) | ((uint64_t)1 << 16) | ((uint64_t)((8 * SW) >> 4) << 32) |
         ((uint64_t)1 << 46) | (layout << 61);
}
// D[tmem] (+)= A[smem] * B[smem]^T, signed int8 operands, int32 accumulators; accumulate = 0 starts the sum
__device__ __forceinline__ void mma_i8(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(da), "l"(db), "r"(idesc), "r"(accumulate));
}
// arrive on the mbarrier once every MMA this thread issued before has completed
__device__ __forceinline__ void mma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
// 32 lanes x 8 consecutive 32-bit columns: this thread's lane, columns taddr .. taddr + 7
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t (&r)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld4(uint32_t taddr, uint32_t (&r)[4]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(taddr));
}
// instruction descriptor of kind::i8: signed A and B, int32 D, both K-major, M 128, N n (a multiple of 16, <= 256)
__host__ __device__ constexpr uint32_t idesc_i8(int n) {
  return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
}

// host: a 2-D TMA descriptor of an int8 matrix [rows][inner] with row stride ld bytes, boxes of box_inner x box_rows,
// swizzle sw (32, 64 or 128 bytes), zero fill out of bounds; 0 or a cudaError_t
int encode_2d_ld(void *map, const void *base, int inner, long long ld, int rows, int box_inner, int box_rows, int sw);
// host: streaming multiprocessors of the current device
int num_sms();

}  // namespace bnn
