// Three-product TF32 arithmetic on the m16n8k8 tensor-core MMA: every fp32
// operand is split in two terms (hi = x rounded to 11 significant bits by
// Veltkamp splitting on the FMA pipe, lo = x - hi passed as is: the tensor
// core reads its top 19 bits) and a product tile is lo*hi + hi*lo + hi*hi,
// about 2^-21 relative error per product.
#pragma once
#include <cstdint>

namespace m4 {

// High part of the two-term split (Veltkamp splitting with the constant
// 2^13 + 1): x rounded to 11 significant bits, exactly a tf32 value, with
// x - hi exact. Three FP32 operations instead of one ALU conversion.
__device__ __forceinline__ uint32_t split_hi(float x) {
  const float t = __fmul_rn(x, 8193.f);
  return __float_as_uint(__fsub_rn(t, __fsub_rn(t, x)));
}

// d += a b on one m16n8k8 tile: a0 = A(g, t), a1 = A(g + 8, t),
// a2 = A(g, t + 4), a3 = A(g + 8, t + 4); b0 = B(t, g), b1 = B(t + 4, g);
// d0 = D(g, 2t), d1 = D(g, 2t + 1), d2 = D(g + 8, 2t), d3 = D(g + 8, 2t + 1)
// for lane = 4g + t.
__device__ __forceinline__ void mma_tf32(float (&d)[4], const uint32_t (&a)[4], const uint32_t (&b)[2]) {
  asm(
      "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

// Two-term splits of an A fragment (4 registers) and a B fragment (2).
struct SplitA {
  uint32_t h[4], l[4];
};
struct SplitB {
  uint32_t h[2], l[2];
};
__device__ __forceinline__ void split2(float x, uint32_t& h, uint32_t& l) {
  h = split_hi(x);
  l = __float_as_uint(x - __uint_as_float(h));
}
__device__ __forceinline__ SplitA split_a(float a0, float a1, float a2, float a3) {
  SplitA s;
  split2(a0, s.h[0], s.l[0]);
  split2(a1, s.h[1], s.l[1]);
  split2(a2, s.h[2], s.l[2]);
  split2(a3, s.h[3], s.l[3]);
  return s;
}
__device__ __forceinline__ SplitB split_b(float b0, float b1) {
  SplitB s;
  split2(b0, s.h[0], s.l[0]);
  split2(b1, s.h[1], s.l[1]);
  return s;
}
// d += a b in three products.
__device__ __forceinline__ void mma3(float (&d)[4], const SplitA& a, const SplitB& b) {
  mma_tf32(d, a.l, b.h);
  mma_tf32(d, a.h, b.l);
  mma_tf32(d, a.h, b.h);
}

}  // namespace m4
