// tcgen05 (5th-generation tensor core) helpers for sm_100a: shared-memory matrix descriptors, the instruction
// descriptor of kind::f16, TMEM allocation / loads, MMA issue and commit, and the 2-D TMA tile load.
// Layout convention: both operands K-major in 128-byte-swizzled shared memory (the layout a TMA tile load with
// CU_TENSOR_MAP_SWIZZLE_128B writes): row r of a tile is 128 B (64 bf16 of K) at r*128, its 16-byte chunk j
// stored at chunk (j ^ (r & 7)); 8-row groups 1024 B apart; tile bases 1024-byte aligned.
#pragma once
#include <cstdint>
#include <cuda.h>

#include "common.cuh"

namespace cbmoe {

// Shared-memory descriptor of a K-major SWIZZLE_128B tile starting at `saddr` (shared-space byte address):
// start address >> 4 in bits [0,14), leading byte offset (unused for swizzled K-major, 1) in [16,30),
// stride byte offset 1024 >> 4 in [32,46), descriptor version 1 in [46,48), layout type 2 (128B swizzle) in
// [61,64). Advancing K by 16 bf16 inside the 64-wide swizzle atom adds 32 B to the start address.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)1 << 16;
  d |= (uint64_t)(1024 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

// Instruction descriptor, kind::f16: D fp32, A and B bf16, both K-major, M = 128, N = n (multiple of 16).
__host__ __device__ constexpr uint32_t idesc_bf16_m128(int n) {
  return (1u << 4)                        // D format: f32
         | (1u << 7)                      // A format: bf16
         | (1u << 10)                     // B format: bf16
         | ((uint32_t)(n >> 3) << 17)     // N >> 3
         | ((uint32_t)(128 >> 4) << 24);  // M >> 4
}

__device__ __forceinline__ void umma_bf16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

// The same MMA with A read from TMEM (`a_tmem`: lane 0, first column of the 16-wide K slice; row m of A in lane m,
// two bf16 of consecutive K per 32-bit column, lower half first) and B from shared memory.
__device__ __forceinline__ void umma_bf16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                                             uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

// Store of 16 lanes x 32 columns from the mma.sync fragment arrangement: thread (g = lane/4, t = lane%4) gives,
// for each of 4 repetitions i (columns 8i .. 8i+7), r[4i] -> (lane g, column 8i+2t), r[4i+1] -> (lane g,
// column 8i+2t+1), r[4i+2] -> (lane g+8, column 8i+2t), r[4i+3] -> (lane g+8, column 8i+2t+1). `taddr` holds the
// first of the 16 lanes (inside this warp's quarter) in bits 16-31 and the first column in bits 0-15.
__device__ __forceinline__ void tmem_st_16x256b_x4(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.16x256b.x4.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

// Wait until this thread's TMEM stores have completed.
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Arrive once on `bar` when every tcgen05 operation issued so far by this thread has completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Generic-proxy shared-memory writes (the dequant warps' A tiles) made visible to the tensor core's reads.
__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// Whole-warp TMEM allocation of `ncols` columns (power of two >= 32); the base address lands in *slot.
__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(slot)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// 16 consecutive fp32 columns of this thread's TMEM lane (warp w reads lanes 32*(w%4) .. +31).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// 2-D TMA tile load (no multicast) of the box at element coordinates (x = inner/K, y = row) into this CTA's
// shared memory, completing on `bar`. x * element size must be a multiple of 16 bytes.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
      "[%4];" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_addr(bar))
      : "memory");
}

__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// Byte offset of (row, 16-byte chunk j) inside a 128B-swizzled K-major tile.
__device__ __forceinline__ uint32_t sw128_off(int row, int j) { return row * 128 + ((j ^ (row & 7)) << 4); }

}  // namespace cbmoe
