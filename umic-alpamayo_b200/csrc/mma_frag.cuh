// Fragment helpers of the decode-regime GEMV engines (gemv.cu, decode_chain.cu):
// bf16 mma.sync m16n8k16 on permuted-k fragments loaded as 16-byte vectors, and the
// addressing of a 128-byte-swizzled [64 x 64] TMA box in shared memory.
#pragma once

#include "common.cuh"

namespace umic {

__device__ __forceinline__ void mma16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Two k16 steps from one 32-wide slab: rows g / g+8 of w (wlo / whi) and
// row g of x, each 8 consecutive k values held as a uint4.
__device__ __forceinline__ void slab_mma(float (&c)[4], const uint4& wlo, const uint4& whi,
                                         const uint4& xv) {
  mma16816(c, wlo.x, whi.x, wlo.y, whi.y, xv.x, xv.y);
  mma16816(c, wlo.z, whi.z, wlo.w, whi.w, xv.z, xv.w);
}

// Byte address of 16-byte chunk `chunk` of row r in a 128-byte-swizzled [64 x 64] box.
__device__ __forceinline__ uint32_t st_swz(uint32_t box, int r, int chunk) {
  return box + r * 128 + ((chunk ^ (r & 7)) << 4);
}
__device__ __forceinline__ uint4 lds128(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr));
  return v;
}
}  // namespace umic
