// Warp-level tensor-core products (mma.sync, sm_80 and later, here on sm_100a) in the
// split-bf16 form used for fp32-accuracy products: an fp32 value x is carried as the bf16
// pair hi = bf16(x), lo = bf16(x - hi), and a product as lo*hi + hi*lo + hi*hi with fp32
// accumulation (relative error ~1e-5). Used where the products are too small for the
// tcgen05 GEMM (a few 16-row tiles per CTA): the GRU recurrence and the wide heads.
#pragma once

#include <cuda_bf16.h>
#include <stdint.h>

namespace bt {

// fp32 pair (a, b) as bf16x2 hi = bf16(a, b) and lo = bf16 of the remainders (a in the low
// half, the order mma.sync expects for consecutive K or column indices).
__device__ __forceinline__ void split_pair(float a, float b, uint32_t& hi, uint32_t& lo) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  const __nv_bfloat162 l = __floats2bfloat162_rn(a - __low2float(h), b - __high2float(h));
  hi = *reinterpret_cast<const uint32_t*>(&h);
  lo = *reinterpret_cast<const uint32_t*>(&l);
}

// D (16 x 8, fp32) += A (16 x 16, bf16, row) B (16 x 8, bf16, col): warp-level tensor-core
// product. Fragments (gid = lane / 4, tig = lane % 4): A regs {rows gid, gid + 8} x
// {cols 2 tig.., 2 tig + 8..}, B regs k = {2 tig.., 2 tig + 8..} at n = gid, D regs
// (gid, 2 tig), (gid, 2 tig + 1), (gid + 8, 2 tig), (gid + 8, 2 tig + 1).
__device__ __forceinline__ void mma_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                          uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// One k-step of a split-bf16 product: A from an fp32 shared tile (row pointers a0 for rows
// gid and a1 for gid + 8, already offset to column 2 tig of the step), B as hi/lo fragments;
// D += A_lo B_hi + A_hi B_lo + A_hi B_hi.
__device__ __forceinline__ void load_a_split(const float* a0, const float* a1, uint32_t (&ah)[4],
                                             uint32_t (&al)[4]) {
  const float2 p00 = *reinterpret_cast<const float2*>(a0);
  const float2 p10 = *reinterpret_cast<const float2*>(a1);
  const float2 p01 = *reinterpret_cast<const float2*>(a0 + 8);
  const float2 p11 = *reinterpret_cast<const float2*>(a1 + 8);
  split_pair(p00.x, p00.y, ah[0], al[0]);
  split_pair(p10.x, p10.y, ah[1], al[1]);
  split_pair(p01.x, p01.y, ah[2], al[2]);
  split_pair(p11.x, p11.y, ah[3], al[3]);
}
__device__ __forceinline__ void mma_split(float (&d)[4], const uint32_t (&ah)[4],
                                          const uint32_t (&al)[4], const uint32_t (&bh)[2],
                                          const uint32_t (&bl)[2]) {
  mma_16816(d, al, bh[0], bh[1]);
  mma_16816(d, ah, bl[0], bl[1]);
  mma_16816(d, ah, bh[0], bh[1]);
}

}  // namespace bt
