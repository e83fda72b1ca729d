// Tensor-core core of the decode-size 4-bit GEMV kernels (MoE experts and dense linears):
// exact bf16 codes from MLX 4-bit words, and one 64-group of a 16-row weight tile against an
// 8-token activation tile on mma.sync m16n8k16 (bf16 in, fp32 accumulate). The K order inside
// each 16-wide k-block is permuted so one 32-bit weight word feeds a thread's whole A
// fragment for two k-blocks; the activations are read in the same order.
#pragma once

#include "common.cuh"

namespace lg {

__device__ __forceinline__ uint32_t nib_pair(uint32_t w, int shift) {
  // bf16x2 {128 + nibble(shift), 128 + nibble(shift + 16)}
  uint32_t r;
  uint32_t v = w >> shift;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r) : "r"(v), "r"(0x000F000Fu), "r"(0x43004300u));
  return r;
}

__device__ __forceinline__ uint32_t bf2_sub128(uint32_t v) {
  // exact: (128 + c) - 128 for c in [0, 15]
  uint32_t r;
  asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(v), "r"(0x43004300u));
  return r;
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
  return r;
}

__device__ __forceinline__ void mma_bf16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ float bf_lo(uint32_t v) { return __uint_as_float(v << 16); }
__device__ __forceinline__ float bf_hi(uint32_t v) { return __uint_as_float(v & 0xffff0000u); }

// One 64-group of one 16-row tile against one 8-token tile.
//  wr0/wr8: the thread's two weight words (2*c4, 2*c4+1 of the group) for rows r and r+8.
//  xa: the thread's 16 activation values of token lane/4 (K 16*c4 .. 16*c4+15 of the group).
__device__ __forceinline__ void group_mma(float (&acc)[4], uint2 wr0, uint2 wr8, uint4 xa0,
                                          uint4 xa1) {
  // mma.sync.aligned needs the whole warp converged; the callers' lane-dependent loads just
  // before may leave it split, and inline asm gives the compiler no reason to rejoin it
  __syncwarp();
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const uint32_t w0 = i ? wr0.y : wr0.x;
    const uint32_t w8 = i ? wr8.y : wr8.x;
    const uint4 xv = i ? xa1 : xa0;
    // x pairs matching nib_pair order: {x0,x4},{x1,x5},{x2,x6},{x3,x7}
    const uint32_t x04 = prmt(xv.x, xv.z, 0x5410), x15 = prmt(xv.x, xv.z, 0x7632);
    const uint32_t x26 = prmt(xv.y, xv.w, 0x5410), x37 = prmt(xv.y, xv.w, 0x7632);
    // k-block 2i: cols {2c4,2c4+1} <- K {8w,8w+4}; cols {2c4+8,2c4+9} <- K {8w+1,8w+5}
    mma_bf16(acc, bf2_sub128(nib_pair(w0, 0)), bf2_sub128(nib_pair(w8, 0)),
             bf2_sub128(nib_pair(w0, 4)), bf2_sub128(nib_pair(w8, 4)), x04, x15);
    // k-block 2i+1: K {8w+2,8w+6} and {8w+3,8w+7}
    mma_bf16(acc, bf2_sub128(nib_pair(w0, 8)), bf2_sub128(nib_pair(w8, 8)),
             bf2_sub128(nib_pair(w0, 12)), bf2_sub128(nib_pair(w8, 12)), x26, x37);
  }
}

__device__ __forceinline__ float xsum16(uint4 a, uint4 b) {
  float s = 0.f;
  const uint32_t v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
  for (int j = 0; j < 8; ++j) s += bf_lo(v[j]) + bf_hi(v[j]);
  return s;
}

}  // namespace lg
