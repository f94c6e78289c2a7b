// Block LDL^T of a 64x64 symmetric positive-definite matrix held by one warp
// in m16n8k8 accumulator fragments, the products on the tensor cores.
//
// Layout. The lower triangle is covered by tiles (R, c) of 16 rows x 8
// columns (rows 16R.., columns 8c.., R in 0..3, c <= 2R + 1). Lane 4g + t
// holds a tile as the MMA accumulator fragment: v0 = (16R + g, 8c + 2t),
// v1 = (16R + g, 8c + 2t + 1), v2 = (16R + 8 + g, 8c + 2t),
// v3 = (16R + 8 + g, 8c + 2t + 1). Row block J (rows 8J..8J + 7) of a tile
// is its register pair 2(J % 2), 2(J % 2) + 1. The tiles (R, 2R + 1) lie
// above the diagonal in their first 8 rows; only v2, v3 are kept.
//
// Factorisation (right-looking, 8-column blocks J = 0..7, no pivoting: the
// matrix is symmetric positive definite, so every diagonal block of every
// Schur complement is):
//   D_J^-1   by a Gauss-Jordan sweep with 2x2 pivots on the warp's fragment
//            of the diagonal block (the sweep keeps the column pairs a lane
//            owns together);
//   L_{.,J}  = A_{.,J} D_J^-1 (one MMA per panel tile; the MMA's k index
//            permuted so a tile's own accumulator registers are its A
//            operand: column 2t is k = t, column 2t + 1 is k = t + 4, and
//            the B operand is the lane's own fragment of D_J^-1);
//   A_{.,.} -= L_{.,J} A_{.,J}^T on every trailing tile (the B operand is
//            the lane's own fragment of the unscaled panel, in the same k
//            order).
// Stored factor: unit lower L off the diagonal blocks, D_J^-1 on them.
// Every product is a three-term TF32 product (tf32.cuh).
#pragma once
#include "common.cuh"
#include "tf32.cuh"

namespace m4 {
namespace ldl {

constexpr unsigned FULL = 0xffffffffu;
constexpr int NT = 20;       // tiles
constexpr int NQ = 18;       // float4 of one lane's stored factor
// Register tile index of (R, c): full tiles (c <= 2R) at R*R + c, the tiles
// (R, 2R + 1) at 16 + R.
__host__ __device__ constexpr int ti(int R, int c) { return c <= 2 * R ? R * R + c : 16 + R; }

using Tiles = float[NT][4];

// Gauss-Jordan inverse of the symmetric diagonal block held as
// x = M[g][2t], y = M[g][2t + 1] on lane 4g + t; 2x2 pivots (2m, 2m + 1),
// m = 0..3 (a column pair is one lane's x, y). On return x, y hold M^-1.
// The pivot block's off-diagonal entries are taken as equal (the block is
// symmetric); its determinant is inverted by the hardware reciprocal
// (rcp.approx: at most one unit in the last place). The step loop stays rolled: the
// eight sweeps of a factorisation are most of its code, and an unrolled body
// overflows the instruction cache of warps at different steps.
M4_DEV void sweep(float& x, float& y, int g, int t) {
#pragma unroll 1
  for (int m = 0; m < 4; ++m) {
    const int k0 = 2 * m, k1 = 2 * m + 1;
    const float c0 = __shfl_sync(FULL, x, 4 * g + m), c1 = __shfl_sync(FULL, y, 4 * g + m);  // M[g][k0], M[g][k1]
    const float r00 = __shfl_sync(FULL, x, 4 * k0 + t), r01 = __shfl_sync(FULL, y, 4 * k0 + t);  // M[k0][2t..]
    const float r10 = __shfl_sync(FULL, x, 4 * k1 + t), r11 = __shfl_sync(FULL, y, 4 * k1 + t);  // M[k1][2t..]
    const float p00 = __shfl_sync(FULL, x, 4 * k0 + m), p01 = __shfl_sync(FULL, y, 4 * k0 + m);
    const float p11 = __shfl_sync(FULL, y, 4 * k1 + m);
    float rd;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(rd) : "f"(fmaf(p00, p11, -p01 * p01)));
    const bool pc = t == m;  // this lane's columns are the pivot columns
    // Pivot rows with the identity in the pivot columns, times the adjugate
    // of the 2x2 pivot block; the reciprocal determinant rd multiplies last,
    // so its latency overlaps this arithmetic.
    const float s00 = pc ? 1.f : r00, s01 = pc ? 0.f : r01, s10 = pc ? 0.f : r10, s11 = pc ? 1.f : r11;
    const float u00 = fmaf(p11, s00, -p01 * s10), u01 = fmaf(p11, s01, -p01 * s11);
    const float u10 = fmaf(p00, s10, -p01 * s00), u11 = fmaf(p00, s11, -p01 * s01);
    const float bx = fmaf(c0, u00, c1 * u10), by = fmaf(c0, u01, c1 * u11);
    float nx = fmaf(-rd, bx, pc ? 0.f : x);
    float ny = fmaf(-rd, by, pc ? 0.f : y);
    nx = g == k0 ? rd * u00 : (g == k1 ? rd * u10 : nx);
    ny = g == k0 ? rd * u01 : (g == k1 ? rd * u11 : ny);
    x = nx;
    y = ny;
  }
}

// Column block J of the factorisation, in two parts. panel_part: the
// unscaled panel tiles (R', J), R' >= R, split once (the A operands of the
// panel products and the B operands of the trailing products; rows of the
// diagonal block itself enter neither, their products are discarded), the
// panel L = A D^-1, and the diagonal block replaced by D^-1 (ix, iy).
template <int J>
M4_DEV void panel_part(Tiles& F, SplitA (&po)[4], float ix, float iy) {
  constexpr int R = J / 2, H = 2 * (J & 1);
  const SplitB dinv = split_b(ix, iy);
#pragma unroll
  for (int Rp = R; Rp < 4; ++Rp) {
    const float* v = F[ti(Rp, J)];
    if (Rp == R)
      po[Rp] = (J & 1) ? split_a(0.f, 0.f, 0.f, 0.f) : split_a(0.f, v[2], 0.f, v[3]);
    else
      po[Rp] = split_a(v[0], v[2], v[1], v[3]);  // k order: columns 2t, 2t + 1 at k = t, t + 4
  }
#pragma unroll
  for (int Rp = R; Rp < 4; ++Rp) {
    if ((J & 1) && Rp == R) continue;
    float d[4] = {0.f, 0.f, 0.f, 0.f};
    mma3(d, po[Rp], dinv);
    float* v = F[ti(Rp, J)];
    v[0] = d[0]; v[1] = d[1]; v[2] = d[2]; v[3] = d[3];
  }
  F[ti(R, J)][H] = ix;
  F[ti(R, J)][H + 1] = iy;
}

// trailing_part: the trailing update A -= L A_panel^T of tiles (R', c'),
// J < c' <= 2R' + 1: with CRIT only the tile holding the next diagonal block
// (c' = J + 1), otherwise all the others.
template <int J, bool CRIT>
M4_DEV void trailing_part(Tiles& F, const SplitA (&po)[4]) {
  constexpr int R = J / 2;
#pragma unroll
  for (int Rp = R; Rp < 4; ++Rp) {
    if (J + 1 > 2 * Rp + 1) continue;
    if (CRIT && Rp != (J + 1) / 2) continue;
    const float* l = F[ti(Rp, J)];
    const SplitA la = split_a(-l[0], -l[2], -l[1], -l[3]);
#pragma unroll
    for (int cp = J + 1; cp <= 2 * Rp + 1; ++cp) {
      if ((cp == J + 1 && Rp == (J + 1) / 2) != CRIT) continue;
      // Panel rows 8c'.. (unscaled): tile (c'/2, J), row half c' % 2. As a
      // B operand b0 = A[8c' + g][8J + 2t], b1 = A[8c' + g][8J + 2t + 1]:
      // in the split's A-operand order, entries 0, 2 (half 0) or 1, 3.
      const SplitA& s = po[cp / 2];
      SplitB b;
      if (cp & 1) {
        b.h[0] = s.h[1]; b.h[1] = s.h[3]; b.l[0] = s.l[1]; b.l[1] = s.l[3];
      } else {
        b.h[0] = s.h[0]; b.h[1] = s.h[2]; b.l[0] = s.l[0]; b.l[1] = s.l[2];
      }
      mma3(F[ti(Rp, cp)], la, b);
    }
  }
}

// Forward-substitution state: u_K[2t], u_K[2t + 1] per finished block K,
// the lane's share of u . v, the right-hand side r and v = D^-1 u (shared).
struct Forward {
  float ub0[8], ub1[8];
  float uv;
  const float* r;
  float* vsm;
};

// Block J of u = L^-1 r, v = D^-1 u: needs the factor's row block J left of
// the diagonal and D_J^-1 (column blocks 0..J finished).
template <int J>
M4_DEV void forward_step(const Tiles& F, Forward& f, int g, int t) {
  constexpr int H = 2 * (J & 1);
  float s = 0.f;
#pragma unroll
  for (int K = 0; K < J; ++K) {
    const float* l = F[ti(J / 2, K)];
    s = fmaf(l[H], f.ub0[K], fmaf(l[H + 1], f.ub1[K], s));
  }
  s += __shfl_xor_sync(FULL, s, 1);
  s += __shfl_xor_sync(FULL, s, 2);
  const float u = f.r[8 * J + g] - s;  // u_J[g]
  f.ub0[J] = __shfl_sync(FULL, u, 8 * t);
  f.ub1[J] = __shfl_sync(FULL, u, 8 * t + 4);
  const float* d = F[ti(J / 2, J)];
  float p = fmaf(d[H], f.ub0[J], d[H + 1] * f.ub1[J]);
  p += __shfl_xor_sync(FULL, p, 1);
  p += __shfl_xor_sync(FULL, p, 2);  // v_J[g]
  if (t == 0) {
    f.vsm[8 * J + g] = p;
    f.uv = fmaf(u, p, f.uv);
  }
}

// The factorisation with the forward substitution of one right-hand side,
// software-pipelined: column block J's pivot sweep is followed by block
// J - 1's trailing updates (all but the one that produced D_J) and forward
// substitution, which do not depend on it, then by block J's panel and the
// trailing update of the tile holding D_(J+1). The independent tensor-core
// and substitution work is in flight while the next sweep starts.
template <int J = 0>
M4_DEV void factor_forward(Tiles& F, Forward& f, SplitA (&po)[4], int g, int t) {
  constexpr int R = J / 2, H = 2 * (J & 1);
  float ix = F[ti(R, J)][H], iy = F[ti(R, J)][H + 1];
  sweep(ix, iy, g, t);
  if constexpr (J > 0) {
    trailing_part<J - 1, false>(F, po);
    forward_step<J - 1>(F, f, g, t);
  }
  panel_part<J>(F, po, ix, iy);
  if constexpr (J + 1 < 8) {
    trailing_part<J, true>(F, po);
    factor_forward<J + 1>(F, f, po, g, t);
  } else {
    forward_step<7>(F, f, g, t);
  }
}

M4_DEV void factor_forward(Tiles& F, Forward& f, int g, int t) {
  SplitA po[4];
  factor_forward<0>(F, f, po, g, t);
}

template <int J = 0>
M4_DEV void forward_steps(const Tiles& F, Forward& f, int g, int t) {
  forward_step<J>(F, f, g, t);
  if constexpr (J + 1 < 8) forward_steps<J + 1>(F, f, g, t);
}

// Forward substitution u = L^-1 r (r: 64 floats in shared memory) and
// v = D^-1 u, written to vsm, on a finished factor; returns the lane's share
// of u . v (= r^T A^-1 r summed over the warp).
M4_DEV float forward_solve(const Tiles& F, const float* r, float* vsm, int g, int t) {
  Forward f;
  f.uv = 0.f;
  f.r = r;
  f.vsm = vsm;
  forward_steps(F, f, g, t);
  return f.uv;
}

// Tile of storage slot q < 16 (full tiles in row-major tile order).
__host__ __device__ constexpr int slot_R(int q) { return q < 1 ? 0 : q < 4 ? 1 : q < 9 ? 2 : 3; }
__host__ __device__ constexpr int slot_c(int q) { return q - slot_R(q) * slot_R(q); }

// Stored form of a lane's tiles: NQ float4, the 16 full tiles in slot order,
// then the kept halves (v2, v3) of tiles 16, 17 and of tiles 18, 19.
M4_DEV float4 get4(const Tiles& F, int q) {
  if (q < 16) return make_float4(F[q][0], F[q][1], F[q][2], F[q][3]);
  const int i = 16 + 2 * (q - 16);
  return make_float4(F[i][2], F[i][3], F[i + 1][2], F[i + 1][3]);
}
M4_DEV void set4(Tiles& F, int q, float4 v) {
  if (q < 16) {
    F[q][0] = v.x; F[q][1] = v.y; F[q][2] = v.z; F[q][3] = v.w;
  } else {
    const int i = 16 + 2 * (q - 16);
    F[i][2] = v.x; F[i][3] = v.y; F[i + 1][2] = v.z; F[i + 1][3] = v.w;
  }
}

// Back substitution y = L^-T v (v: 64 floats in shared memory), written to
// ysm. Lane (g, t) sums column 8J + 2t + (g & 1): the two column sums of a
// row-pair exchange are halved with one shuffle before the reduction over g.
M4_DEV void back_solve(const Tiles& F, const float* vsm, float* ysm, int g, int t) {
  float yr[8];  // y_K[g]
  const bool odd = g & 1;
#pragma unroll
  for (int J = 7; J >= 0; --J) {
    float s0 = 0.f, s1 = 0.f;
#pragma unroll
    for (int K = J + 1; K < 8; ++K) {
      const float* l = F[ti(K / 2, J)];
      const int H = 2 * (K & 1);
      s0 = fmaf(l[H], yr[K], s0);
      s1 = fmaf(l[H + 1], yr[K], s1);
    }
    float s = (odd ? s1 : s0) + __shfl_xor_sync(FULL, odd ? s0 : s1, 4);
    s += __shfl_xor_sync(FULL, s, 8);
    s += __shfl_xor_sync(FULL, s, 16);
    const float y = vsm[8 * J + 2 * t + odd] - s;  // y_J[2t + (g & 1)]
    yr[J] = __shfl_sync(FULL, y, 4 * int(odd) + (g >> 1));
    if (g < 2) ysm[8 * J + 2 * t + g] = y;
  }
}

}  // namespace ldl
}  // namespace m4
