// Selective conjugate memory read, forward and backward, for sm_100a.
//
// Reference operator: selective_memory_fused (lm/kernels/mamba4_fused.py:372-454)
// with the contract of selective_gaussian_memory (lm/kernels/mamba4.py:228-338).
// Per head, S_t = lam_t S_(t-1) + beta_t k_t k_t^T, C_t likewise with v_t k_t^T,
// A_t = S_t + diag(floor), y_t = A_t^-1 q_t, output_t = C_t y_t,
// variance_t = q_t . y_t.
//
// Kernels (all fp32, key dim D = 64, value dim P in {64, 128}):
//   memread_states   per (batch, head): sequential rank-one evidence/cross
//                    updates; writes S at every 16-token sub-chunk start and
//                    C at every 64-token chunk start, and the final state.
//   memread_solve    one warp per (batch, head, 16-token sub-chunk): per token
//                    E <- lam E + beta k k^T in shared memory, then a
//                    register-blocked 64x64 Cholesky of E + diag(floor) on a
//                    4x8 cyclic lane grid with the query as a bordered row
//                    (gives w = L^-1 q for free), a blocked back-substitution
//                    y = L^-T w with 8x8 diagonal-block inverses, and a
//                    coalesced 128-bit streaming store of L (reciprocal
//                    pivots on the diagonal, as mamba4_fused.py:78-113 keeps).
//   memread_output   per (batch, 64-token chunk, head): output =
//                    ((Y K^T) o W) V + diag(e^P) Y C0^T (mamba4_fused.py:439-447).
//   backward         rhs g (chunk products), z = A^-1 g from the stored
//                    factors (blocked substitutions), the chunk adjoint carry,
//                    and every input gradient in chunk form; the algebra is
//                    written out in oracle/memread.py:chunked_backward.
#include "common.cuh"

namespace m4 {
namespace mem {

constexpr int KD = 64;         // key dimension
constexpr int CH = 64;         // chunk (epilogue / backward products)
constexpr int SUB = 16;        // tokens per solve warp (state stride)
constexpr int SLOTS = 72;      // L slots per lane: (m, n), m in [2n, 15], n in [0, 7]
constexpr int LSTRIDE = SLOTS * 32;  // floats of one token's stored factor (2304)
constexpr int WARPS = 4;       // solve warps per CTA

// Slot of lane-local tile entry (m, n): rows a + 4m, columns b + 8n on lane
// a*8 + b (a in 0..3, b in 0..7). Column groups n are stored contiguously.
__host__ __device__ constexpr int slot_of(int m, int n) { return 16 * n - n * (n - 1) + (m - 2 * n); }

struct Sizes {
  int B, T, H, P, Tp, nsub, nch;
  size_t l_off, y_off, s_off, c_off, resid_bytes;
  size_t g_off, z_off, sb_off, cb_off, fl_off, work_bytes;
};

inline Sizes sizes(const M4MemDims& d) {
  Sizes s;
  s.B = d.batch; s.T = d.time; s.H = d.heads; s.P = d.value_dim;
  s.Tp = (d.time + CH - 1) / CH * CH;
  s.nsub = s.Tp / SUB;
  s.nch = s.Tp / CH;
  const size_t bh = size_t(s.B) * s.H;
  size_t off = 0;
  s.l_off = off; off += align256(bh * s.Tp * LSTRIDE * sizeof(float));
  s.y_off = off; off += align256(bh * s.Tp * KD * sizeof(float));
  s.s_off = off; off += align256(bh * s.nsub * KD * KD * sizeof(float));
  s.c_off = off; off += align256(bh * s.nch * size_t(s.P) * KD * sizeof(float));
  s.resid_bytes = off;
  off = 0;
  s.g_off = off; off += align256(bh * s.Tp * KD * sizeof(float));
  s.z_off = off; off += align256(bh * s.Tp * KD * sizeof(float));
  s.sb_off = off; off += align256(bh * s.nch * KD * KD * sizeof(float));
  s.cb_off = off; off += align256(bh * s.nch * size_t(s.P) * KD * sizeof(float));
  s.fl_off = off; off += align256(size_t(s.B) * s.nch * s.H * KD * sizeof(float));
  s.work_bytes = off;
  return s;
}

// ---------------------------------------------------------------------------
// memread_states: sequential evidence/cross statistics per (batch, head).
// ---------------------------------------------------------------------------
template <int P>
__global__ void __launch_bounds__(256) states_kernel(
    int B, int T, int H, const float* __restrict__ keys, const float* __restrict__ values,
    const float* __restrict__ beta, const float* __restrict__ log_decay,
    const float* __restrict__ init_s, const float* __restrict__ init_c,
    float* __restrict__ s_start, float* __restrict__ c_start,
    float* __restrict__ s_final, float* __restrict__ c_final) {
  constexpr int CR = P / 64;
  const int bh = blockIdx.x, b = bh / H, h = bh % H;
  const int tid = threadIdx.x;
  const int Tp = (T + CH - 1) / CH * CH, nsub = Tp / SUB, nch = Tp / CH;
  const int i = tid >> 2, j0 = (tid & 3) * 16;
  __shared__ __align__(16) float ks[SUB][KD];
  __shared__ __align__(16) float vs[SUB][P];
  __shared__ float bl[SUB], ll[SUB];
  float s[16], c[CR][16];
#pragma unroll
  for (int e = 0; e < 16; ++e) {
    s[e] = init_s ? init_s[(size_t(bh) * KD + i) * KD + j0 + e] : 0.f;
#pragma unroll
    for (int r = 0; r < CR; ++r)
      c[r][e] = init_c ? init_c[(size_t(bh) * P + i + 64 * r) * KD + j0 + e] : 0.f;
  }
  for (int sub = 0; sub < nsub; ++sub) {
    float* sd = s_start + ((size_t(bh) * nsub + sub) * KD + i) * KD + j0;
#pragma unroll
    for (int e = 0; e < 16; e += 4) st4(sd + e, make_float4(s[e], s[e + 1], s[e + 2], s[e + 3]));
    if ((sub & 3) == 0) {
#pragma unroll
      for (int r = 0; r < CR; ++r) {
        float* cd = c_start + ((size_t(bh) * nch + (sub >> 2)) * P + i + 64 * r) * KD + j0;
#pragma unroll
        for (int e = 0; e < 16; e += 4)
          st4(cd + e, make_float4(c[r][e], c[r][e + 1], c[r][e + 2], c[r][e + 3]));
      }
    }
    const int t0 = sub * SUB;
    for (int idx = tid; idx < SUB * KD; idx += 256) {
      const int tt = idx / KD, d = idx % KD, t = t0 + tt;
      ks[tt][d] = t < T ? keys[((size_t(b) * T + t) * H + h) * KD + d] : 0.f;
    }
    for (int idx = tid; idx < SUB * P; idx += 256) {
      const int tt = idx / P, p = idx % P, t = t0 + tt;
      vs[tt][p] = t < T ? values[((size_t(b) * T + t) * H + h) * P + p] : 0.f;
    }
    if (tid < SUB) {
      const int t = t0 + tid;
      bl[tid] = t < T ? beta[(size_t(b) * T + t) * H + h] : 0.f;
      ll[tid] = t < T ? expf(log_decay[(size_t(b) * T + t) * H + h]) : 1.f;
    }
    __syncthreads();
#pragma unroll 2
    for (int tt = 0; tt < SUB; ++tt) {
      const float lam = ll[tt], bet = bl[tt];
      float kj[16];
#pragma unroll
      for (int e = 0; e < 16; e += 4) {
        float4 v4 = ld4(&ks[tt][j0 + e]);
        kj[e] = v4.x; kj[e + 1] = v4.y; kj[e + 2] = v4.z; kj[e + 3] = v4.w;
      }
      const float bk = bet * ks[tt][i];
#pragma unroll
      for (int e = 0; e < 16; ++e) s[e] = fmaf(bk, kj[e], lam * s[e]);
#pragma unroll
      for (int r = 0; r < CR; ++r) {
        const float bv = bet * vs[tt][i + 64 * r];
#pragma unroll
        for (int e = 0; e < 16; ++e) c[r][e] = fmaf(bv, kj[e], lam * c[r][e]);
      }
    }
    __syncthreads();
  }
#pragma unroll
  for (int e = 0; e < 16; ++e) {
    s_final[(size_t(bh) * KD + i) * KD + j0 + e] = s[e];
#pragma unroll
    for (int r = 0; r < CR; ++r) c_final[(size_t(bh) * P + i + 64 * r) * KD + j0 + e] = c[r][e];
  }
}

// ---------------------------------------------------------------------------
// Shared pieces of the per-token solve warps.
// ---------------------------------------------------------------------------

// In-place inverse of an 8x8 lower-triangular block whose diagonal holds the
// reciprocal pivots 1/L_rr (upper part zero). Result X = L_block^-1, row-major.
M4_DEV void invert_lower8(float* blk) {
  float T[8][8], X[8][8];
#pragma unroll
  for (int r = 0; r < 8; ++r) {
    float4 lo = ld4(blk + 8 * r), hi = ld4(blk + 8 * r + 4);
    T[r][0] = lo.x; T[r][1] = lo.y; T[r][2] = lo.z; T[r][3] = lo.w;
    T[r][4] = hi.x; T[r][5] = hi.y; T[r][6] = hi.z; T[r][7] = hi.w;
  }
#pragma unroll
  for (int c = 0; c < 8; ++c) {
#pragma unroll
    for (int r = 0; r < 8; ++r) X[r][c] = 0.f;
    X[c][c] = T[c][c];
#pragma unroll
    for (int r = c + 1; r < 8; ++r) {
      float acc = 0.f;
#pragma unroll
      for (int k = c; k < r; ++k) acc = fmaf(T[r][k], X[k][c], acc);
      X[r][c] = -T[r][r] * acc;
    }
  }
#pragma unroll
  for (int r = 0; r < 8; ++r) {
    st4(blk + 8 * r, make_float4(X[r][0], X[r][1], X[r][2], X[r][3]));
    st4(blk + 8 * r + 4, make_float4(X[r][4], X[r][5], X[r][6], X[r][7]));
  }
}

// Stage the 8 diagonal 8x8 blocks of the lane-distributed factor into shared
// memory and invert them (lanes 0..7 one block each).
M4_DEV void stage_and_invert_blocks(const float (&L)[SLOTS], float* blk, int lane, int a, int b) {
  __syncwarp();
#pragma unroll
  for (int J = 0; J < 8; ++J) {
    blk[J * 64 + a * 8 + b] = L[slot_of(2 * J, J)];
    blk[J * 64 + (a + 4) * 8 + b] = L[slot_of(2 * J + 1, J)];
  }
  __syncwarp();
  if (lane < 8) invert_lower8(blk + lane * 64);
  __syncwarp();
}

// Blocked back-substitution y = L^-T w. `w` is a 64-vector in shared memory;
// result returned distributed: yr[m] = y[a + 4m]; y also written to ysm.
M4_DEV void back_substitute(const float (&L)[SLOTS], const float* blk, const float* w, float* ysm,
                            float (&yr)[16], int a, int b) {
#pragma unroll
  for (int J = 7; J >= 0; --J) {
    float sp = 0.f;
#pragma unroll
    for (int K = J + 1; K < 8; ++K) {
      sp = fmaf(L[slot_of(2 * K, J)], yr[2 * K], sp);
      sp = fmaf(L[slot_of(2 * K + 1, J)], yr[2 * K + 1], sp);
    }
    sp += __shfl_xor_sync(0xffffffffu, sp, 8);
    sp += __shfl_xor_sync(0xffffffffu, sp, 16);
    const float x = w[8 * J + b] - sp;                 // x[b] on lanes (., b)
    const float xa = __shfl_sync(0xffffffffu, x, a);     // x[a]
    const float xa4 = __shfl_sync(0xffffffffu, x, a + 4);  // x[a + 4]
    float p = blk[J * 64 + a * 8 + b] * xa;
    p = fmaf(blk[J * 64 + (a + 4) * 8 + b], xa4, p);
    p += __shfl_xor_sync(0xffffffffu, p, 8);
    p += __shfl_xor_sync(0xffffffffu, p, 16);          // y[8J + b]
    yr[2 * J] = __shfl_sync(0xffffffffu, p, a);
    yr[2 * J + 1] = __shfl_sync(0xffffffffu, p, a + 4);
    if (a == 0) ysm[8 * J + b] = p;
  }
}

// Blocked forward substitution u = L^-1 g. `g` is a 64-vector in shared
// memory; u written to usm (64 floats).
M4_DEV void forward_substitute(const float (&L)[SLOTS], const float* blk, const float* g, float* usm,
                               int a, int b) {
  float ub[8];
#pragma unroll
  for (int J = 0; J < 8; ++J) {
    float s0 = 0.f, s1 = 0.f;
#pragma unroll
    for (int K = 0; K < J; ++K) {
      s0 = fmaf(L[slot_of(2 * J, K)], ub[K], s0);
      s1 = fmaf(L[slot_of(2 * J + 1, K)], ub[K], s1);
    }
#pragma unroll
    for (int o = 1; o < 8; o <<= 1) {
      s0 += __shfl_xor_sync(0xffffffffu, s0, o);
      s1 += __shfl_xor_sync(0xffffffffu, s1, o);
    }
    const float x0 = g[8 * J + a] - s0;      // x[a]     on lanes (a, .)
    const float x1 = g[8 * J + a + 4] - s1;  // x[a + 4]
    const int src = (b & 3) * 8;
    const float t0 = __shfl_sync(0xffffffffu, x0, src);
    const float t1 = __shfl_sync(0xffffffffu, x1, src);
    const float xb = b < 4 ? t0 : t1;        // x[b]
    float p0 = blk[J * 64 + a * 8 + b] * xb;
    float p1 = blk[J * 64 + (a + 4) * 8 + b] * xb;
#pragma unroll
    for (int o = 1; o < 8; o <<= 1) {
      p0 += __shfl_xor_sync(0xffffffffu, p0, o);
      p1 += __shfl_xor_sync(0xffffffffu, p1, o);
    }
    // p0 = u[8J + a], p1 = u[8J + a + 4] on lanes (a, .)
    const float u0 = __shfl_sync(0xffffffffu, p0, src);
    const float u1 = __shfl_sync(0xffffffffu, p1, src);
    ub[J] = b < 4 ? u0 : u1;                 // u[8J + b]
    if (b == 0) { usm[8 * J + a] = p0; usm[8 * J + a + 4] = p1; }
  }
  __syncwarp();
}

struct SolveSmem {
  float E[SLOTS / 4][32][4];   // running evidence, lane slot layout
  float kR[64];                // k[a + 4m] at a*16 + m
  float kC[64];                // k[b + 8n] at b*8 + n
  float qC[64];                // q[b + 8n] at b*8 + n
  float flC[64];               // floor[b + 8n] at b*8 + n
  float w[64];                 // w = L^-1 q (or u = L^-1 g)
  float y[64];                 // solution
  union {
    float col[2][144];         // column broadcast: R layout a*20+m, C layout 80+b*8+n
    float blk[8 * 64];         // diagonal blocks / inverses
  } u;
};

// ---------------------------------------------------------------------------
// memread_solve: per-token Cholesky factor + solve, L stored for backward.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(32 * WARPS) solve_kernel(
    int B, int T, int H, const float* __restrict__ keys, const float* __restrict__ queries,
    const float* __restrict__ beta, const float* __restrict__ log_decay,
    const float* __restrict__ floor_, const float* __restrict__ s_start,
    float* __restrict__ Lst, float* __restrict__ Y, float* __restrict__ variance) {
  extern __shared__ __align__(16) unsigned char solve_raw[];
  SolveSmem* smem_all = reinterpret_cast<SolveSmem*>(solve_raw);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int a = lane >> 3, b = lane & 7;
  const int Tp = (T + CH - 1) / CH * CH, nsub = Tp / SUB;
  const int wid = blockIdx.x * WARPS + warp;
  if (wid >= B * H * nsub) return;
  SolveSmem& sm = smem_all[warp];
  const int sub = wid % nsub, bh = wid / nsub, bb = bh / H, h = bh % H;

  // Evidence at the sub-chunk start into the lane slot layout.
  {
    const float* src = s_start + (size_t(bh) * nsub + sub) * KD * KD;
#pragma unroll
    for (int n = 0; n < 8; ++n)
#pragma unroll
      for (int m = 2 * n; m < 16; ++m) {
        const int s = slot_of(m, n);
        sm.E[s >> 2][lane][s & 3] = src[(a + 4 * m) * KD + b + 8 * n];
      }
    if (a == 0) {
#pragma unroll
      for (int n = 0; n < 8; ++n) sm.flC[b * 8 + n] = floor_[h * KD + b + 8 * n];
    }
  }
  __syncwarp();

  for (int tt = 0; tt < SUB; ++tt) {
    const int t = sub * SUB + tt;
    const bool live = t < T;
    // Stage k (lanes 0..15) and q (lanes 16..31) in permuted layouts.
    {
      const int l = lane & 15;
      const float* src = (lane < 16 ? keys : queries) + ((size_t(bb) * T + t) * H + h) * KD + 4 * l;
      float4 v4 = live ? ld4(src) : make_float4(0.f, 0.f, 0.f, 0.f);
      const float vv[4] = {v4.x, v4.y, v4.z, v4.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int i = 4 * l + e;
        if (lane < 16) {
          sm.kR[(i & 3) * 16 + (i >> 2)] = vv[e];
          sm.kC[(i & 7) * 8 + (i >> 3)] = vv[e];
        } else {
          sm.qC[(i & 7) * 8 + (i >> 3)] = vv[e];
        }
      }
    }
    const float bet = live ? beta[(size_t(bb) * T + t) * H + h] : 0.f;
    const float lam = live ? expf(log_decay[(size_t(bb) * T + t) * H + h]) : 1.f;
    __syncwarp();

    float A[SLOTS];
    float wr[8];
    {
      float kr[16], kc[8], fl[8];
#pragma unroll
      for (int m = 0; m < 16; m += 4) {
        float4 v4 = ld4(&sm.kR[a * 16 + m]);
        kr[m] = bet * v4.x; kr[m + 1] = bet * v4.y; kr[m + 2] = bet * v4.z; kr[m + 3] = bet * v4.w;
      }
#pragma unroll
      for (int n = 0; n < 8; n += 4) {
        float4 v4 = ld4(&sm.kC[b * 8 + n]);
        kc[n] = v4.x; kc[n + 1] = v4.y; kc[n + 2] = v4.z; kc[n + 3] = v4.w;
        float4 f4 = ld4(&sm.flC[b * 8 + n]);
        fl[n] = f4.x; fl[n + 1] = f4.y; fl[n + 2] = f4.z; fl[n + 3] = f4.w;
        float4 q4 = ld4(&sm.qC[b * 8 + n]);
        wr[n] = a == 0 ? q4.x : 0.f; wr[n + 1] = a == 0 ? q4.y : 0.f;
        wr[n + 2] = a == 0 ? q4.z : 0.f; wr[n + 3] = a == 0 ? q4.w : 0.f;
      }
#pragma unroll
      for (int q4 = 0; q4 < SLOTS / 4; ++q4) {
        float4 e4 = ld4(sm.E[q4][lane]);
        float ev[4] = {e4.x, e4.y, e4.z, e4.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int s = 4 * q4 + e;
          // decode slot -> (m, n) at compile time
          int n = 0;
#pragma unroll
          for (int nn = 1; nn < 8; ++nn) if (s >= slot_of(2 * nn, nn)) n = nn;
          const int m = s - slot_of(2 * n, n) + 2 * n;
          ev[e] = fmaf(kr[m], kc[n], lam * ev[e]);
          A[s] = ev[e];
        }
        st4(sm.E[q4][lane], make_float4(ev[0], ev[1], ev[2], ev[3]));
      }
#pragma unroll
      for (int n = 0; n < 8; ++n) {
        A[slot_of(2 * n, n)] += (b == a) ? fl[n] : 0.f;
        A[slot_of(2 * n + 1, n)] += (b == a + 4) ? fl[n] : 0.f;
      }
    }

    // Right-looking Cholesky on unscaled columns U (L[:, j] = U[:, j] / sqrt(U_jj)).
    float rc[8];
#pragma unroll
    for (int n = 0; n < 8; ++n) rc[n] = 0.f;
#pragma unroll
    for (int j = 0; j < KD; ++j) {
      const int jn = j >> 3, jb = j & 7, jm = j >> 2, ja = j & 3;
      float* cb = sm.u.col[j & 1];
      if (b == jb) {
#pragma unroll
        for (int m = 2 * jn; m < 16; ++m) {
          const float v = A[slot_of(m, jn)];
          cb[a * 20 + m] = v;
          const int row = a + 4 * m;
          cb[80 + (row & 7) * 8 + (row >> 3)] = v;
        }
        cb[a * 20 + 16] = wr[jn];
      }
      __syncwarp();
      const float piv = cb[ja * 20 + jm];
      const float r = rsqrtf(piv);
      const float r2 = r * r;
      rc[jn] = (b == jb) ? r : rc[jn];
      float R[17], C[8];
#pragma unroll
      for (int m = jm; m < 17; ++m) R[m] = cb[a * 20 + m];
      R[jm] = (a > ja) ? R[jm] : 0.f;
#pragma unroll
      for (int n = jn; n < 8; ++n) C[n] = cb[80 + b * 8 + n] * r2;
      C[jn] = (b > jb) ? C[jn] : 0.f;
#pragma unroll
      for (int n = jn; n < 8; ++n) {
#pragma unroll
        for (int m = (2 * n > jm ? 2 * n : jm); m < 16; ++m)
          A[slot_of(m, n)] = fmaf(-R[m], C[n], A[slot_of(m, n)]);
        wr[n] = fmaf(-R[16], C[n], wr[n]);
      }
    }

    // w = L^-1 q (bordered row), variance = |w|^2.
    float vpart = 0.f;
    if (a == 0) {
#pragma unroll
      for (int n = 0; n < 8; ++n) {
        const float wv = wr[n] * rc[n];
        sm.w[b + 8 * n] = wv;
        vpart = fmaf(wv, wv, vpart);
      }
    }
    const float var = warp_sum(vpart);

    // Scale to L; reciprocal pivot on the diagonal; zero the upper triangle.
#pragma unroll
    for (int n = 0; n < 8; ++n) {
#pragma unroll
      for (int m = 2 * n; m < 16; ++m) A[slot_of(m, n)] *= rc[n];
      float& d0 = A[slot_of(2 * n, n)];
      float& d1 = A[slot_of(2 * n + 1, n)];
      d0 = (b == a) ? rc[n] : (a < b ? 0.f : d0);
      d1 = (b == a + 4) ? rc[n] : (a + 4 < b ? 0.f : d1);
    }
    {
      float* dst = Lst + (size_t(bh) * Tp + t) * LSTRIDE;
#pragma unroll
      for (int q4 = 0; q4 < SLOTS / 4; ++q4)
        st4_stream(dst + (q4 * 32 + lane) * 4,
                   make_float4(A[4 * q4], A[4 * q4 + 1], A[4 * q4 + 2], A[4 * q4 + 3]));
    }

    stage_and_invert_blocks(A, sm.u.blk, lane, a, b);
    float yr[16];
    back_substitute(A, sm.u.blk, sm.w, sm.y, yr, a, b);
    __syncwarp();
    if (lane < 16) st4(Y + (size_t(bh) * Tp + t) * KD + 4 * lane, ld4(&sm.y[4 * lane]));
    if (live && lane == 0) variance[(size_t(bb) * T + t) * H + h] = var;
    __syncwarp();
  }
}

// ---------------------------------------------------------------------------
// Chunk-product kernels (one CTA of 256 threads per (batch, chunk, head)).
// Thread t owns rows ty + 16 i (i < 4) and columns tx + 16 j, ty = t/16, tx = t%16.
// Tiles are stored with odd strides so row and column reads are conflict-free.
// ---------------------------------------------------------------------------
constexpr int LD = KD + 1;

template <int NJ, int K, class FA, class FB>
M4_DEV void mm(float (&acc)[4][NJ], int ty, int tx, FA fa, FB fb) {
#pragma unroll 4
  for (int k = 0; k < K; ++k) {
    float av[4], bv[NJ];
#pragma unroll
    for (int i = 0; i < 4; ++i) av[i] = fa(ty + 16 * i, k);
#pragma unroll
    for (int j = 0; j < NJ; ++j) bv[j] = fb(k, tx + 16 * j);
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < NJ; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
  }
}

template <int NJ>
M4_DEV void zero(float (&acc)[4][NJ]) {
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < NJ; ++j) acc[i][j] = 0.f;
}

// Chunk-local inclusive prefix of log_decay and the gates, by warp 0.
M4_DEV void chunk_gates(int tid, int b, int T, int H, int h, int t0, const float* beta,
                        const float* log_decay, float* pre, float* bet) {
  if (tid < 32) {
    float carry = 0.f;
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const int tt = half * 32 + tid, t = t0 + tt;
      const float g = t < T ? log_decay[(size_t(b) * T + t) * H + h] : 0.f;
      const float inc = warp_inclusive_scan(g, tid) + carry;
      pre[tt] = inc;
      bet[tt] = t < T ? beta[(size_t(b) * T + t) * H + h] : 0.f;
      carry = __shfl_sync(0xffffffffu, inc, 31);
    }
  }
}

// Load a [64 tokens][W] chunk of a [B,T,H,W] tensor into a strided tile.
template <int W>
M4_DEV void load_tokens(float* tile, int ld, const float* src, int b, int T, int H, int h, int t0, int tid) {
  for (int idx = tid; idx < CH * W; idx += 256) {
    const int tt = idx / W, c = idx % W, t = t0 + tt;
    tile[tt * ld + c] = t < T ? src[((size_t(b) * T + t) * H + h) * W + c] : 0.f;
  }
}

// Load a dense [R][64] row-major block into a strided tile.
M4_DEV void load_block(float* tile, int rows, const float* src, int tid) {
  for (int idx = tid; idx < rows * KD; idx += 256) tile[(idx / KD) * LD + idx % KD] = src[idx];
}

template <int P>
__global__ void __launch_bounds__(256) output_kernel(
    int B, int T, int H, const float* __restrict__ keys, const float* __restrict__ values,
    const float* __restrict__ beta, const float* __restrict__ log_decay,
    const float* __restrict__ Y, const float* __restrict__ c_start, float* __restrict__ out) {
  constexpr int LP = P + 1, NJ = P / 16;
  extern __shared__ __align__(16) float sh[];
  float* Ys = sh;                 // [64][LD]
  float* Ks = Ys + CH * LD;       // [64][LD]
  float* Ms = Ks + CH * LD;       // [64][LD]
  float* Vs = Ms + CH * LD;       // [64][LP]
  float* C0 = Vs + CH * LP;       // [P][LD]
  float* pre = C0 + P * LD;       // [64]
  float* bet = pre + CH;          // [64]
  const int Tp = (T + CH - 1) / CH * CH, nch = Tp / CH;
  const int ch = blockIdx.x % nch, bh = blockIdx.x / nch, b = bh / H, h = bh % H;
  const int t0 = ch * CH, tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;
  load_block(Ys, CH, Y + (size_t(bh) * Tp + t0) * KD, tid);
  load_tokens<KD>(Ks, LD, keys, b, T, H, h, t0, tid);
  load_tokens<P>(Vs, LP, values, b, T, H, h, t0, tid);
  load_block(C0, P, c_start + (size_t(bh) * nch + ch) * P * KD, tid);
  chunk_gates(tid, b, T, H, h, t0, beta, log_decay, pre, bet);
  __syncthreads();
  {
    float acc[4][4];
    zero(acc);
    mm<4, KD>(acc, ty, tx, [&](int r, int k) { return Ys[r * LD + k]; },
              [&](int k, int c) { return Ks[c * LD + k]; });
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int r = ty + 16 * i, c = tx + 16 * j;
        Ms[r * LD + c] = c <= r ? acc[i][j] * bet[c] * expf(pre[r] - pre[c]) : 0.f;
      }
  }
  __syncthreads();
  float acc[4][NJ], inh[4][NJ];
  zero(acc);
  zero(inh);
  mm<NJ, CH>(acc, ty, tx, [&](int r, int k) { return Ms[r * LD + k]; },
             [&](int k, int c) { return Vs[k * LP + c]; });
  mm<NJ, KD>(inh, ty, tx, [&](int r, int k) { return Ys[r * LD + k]; },
             [&](int k, int c) { return C0[c * LD + k]; });
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int r = ty + 16 * i, t = t0 + r;
    if (t >= T) continue;
    const float e = expf(pre[r]);
#pragma unroll
    for (int j = 0; j < NJ; ++j)
      out[((size_t(b) * T + t) * H + h) * P + tx + 16 * j] = fmaf(e, inh[i][j], acc[i][j]);
  }
}

// ---------------------------------------------------------------------------
// Backward kernels.
// ---------------------------------------------------------------------------

// rhs_kernel: g_t = e^(P_t) C0^T dO_t + sum_s W[t,s] (dO_t . v_s) k_s + dvar_t q_t.
template <int P>
__global__ void __launch_bounds__(256) rhs_kernel(
    int B, int T, int H, const float* __restrict__ keys, const float* __restrict__ values,
    const float* __restrict__ queries, const float* __restrict__ beta,
    const float* __restrict__ log_decay, const float* __restrict__ c_start,
    const float* __restrict__ d_out, const float* __restrict__ d_var, float* __restrict__ G) {
  constexpr int LP = P + 1;
  extern __shared__ __align__(16) float sh[];
  float* Ks = sh;                 // [64][LD]
  float* Ms = Ks + CH * LD;       // [64][LD]
  float* Os = Ms + CH * LD;       // [64][LP]
  float* Vs = Os + CH * LP;       // [64][LP]
  float* C0 = Vs + CH * LP;       // [P][LD]
  float* pre = C0 + P * LD;
  float* bet = pre + CH;
  const int Tp = (T + CH - 1) / CH * CH, nch = Tp / CH;
  const int ch = blockIdx.x % nch, bh = blockIdx.x / nch, b = bh / H, h = bh % H;
  const int t0 = ch * CH, tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;
  load_tokens<KD>(Ks, LD, keys, b, T, H, h, t0, tid);
  load_tokens<P>(Os, LP, d_out, b, T, H, h, t0, tid);
  load_tokens<P>(Vs, LP, values, b, T, H, h, t0, tid);
  load_block(C0, P, c_start + (size_t(bh) * nch + ch) * P * KD, tid);
  chunk_gates(tid, b, T, H, h, t0, beta, log_decay, pre, bet);
  __syncthreads();
  {
    float acc[4][4];
    zero(acc);
    mm<4, P>(acc, ty, tx, [&](int r, int k) { return Os[r * LP + k]; },
             [&](int k, int c) { return Vs[c * LP + k]; });
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int r = ty + 16 * i, c = tx + 16 * j;
        Ms[r * LD + c] = c <= r ? acc[i][j] * bet[c] * expf(pre[r] - pre[c]) : 0.f;
      }
  }
  __syncthreads();
  float acc[4][4], inh[4][4];
  zero(acc);
  zero(inh);
  mm<4, CH>(acc, ty, tx, [&](int r, int k) { return Ms[r * LD + k]; },
            [&](int k, int c) { return Ks[k * LD + c]; });
  mm<4, P>(inh, ty, tx, [&](int r, int k) { return Os[r * LP + k]; },
           [&](int k, int c) { return C0[k * LD + c]; });
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int r = ty + 16 * i, t = t0 + r;
    const bool live = t < T;
    const float e = expf(pre[r]);
    const float dv = live ? d_var[(size_t(b) * T + t) * H + h] : 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int c = tx + 16 * j;
      const float q = live ? queries[((size_t(b) * T + t) * H + h) * KD + c] : 0.f;
      G[(size_t(bh) * Tp + t) * KD + c] = fmaf(dv, q, fmaf(e, inh[i][j], acc[i][j]));
    }
  }
}

// zsolve_kernel: z_t = A_t^-1 g_t from the stored factor (one warp per token
// at a time, 16 tokens per warp).
__global__ void __launch_bounds__(32 * WARPS) zsolve_kernel(
    int B, int T, int H, const float* __restrict__ Lst, const float* __restrict__ G,
    float* __restrict__ Z) {
  struct Smem {
    float g[64];
    float u[64];
    float z[64];
    float blk[8 * 64];
  };
  __shared__ Smem smem_all[WARPS];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int a = lane >> 3, b = lane & 7;
  const int Tp = (T + CH - 1) / CH * CH, nsub = Tp / SUB;
  const int wid = blockIdx.x * WARPS + warp;
  if (wid >= B * H * nsub) return;
  Smem& sm = smem_all[warp];
  const int sub = wid % nsub, bh = wid / nsub;
  for (int tt = 0; tt < SUB; ++tt) {
    const int t = sub * SUB + tt;
    float L[SLOTS];
    const float* src = Lst + (size_t(bh) * Tp + t) * LSTRIDE;
#pragma unroll
    for (int q4 = 0; q4 < SLOTS / 4; ++q4) {
      float4 v4 = __ldcs(reinterpret_cast<const float4*>(src + (q4 * 32 + lane) * 4));
      L[4 * q4] = v4.x; L[4 * q4 + 1] = v4.y; L[4 * q4 + 2] = v4.z; L[4 * q4 + 3] = v4.w;
    }
    if (lane < 16) st4(&sm.g[4 * lane], ld4(G + (size_t(bh) * Tp + t) * KD + 4 * lane));
    stage_and_invert_blocks(L, sm.blk, lane, a, b);
    forward_substitute(L, sm.blk, sm.g, sm.u, a, b);
    float zr[16];
    back_substitute(L, sm.blk, sm.u, sm.z, zr, a, b);
    __syncwarp();
    if (lane < 16) st4(Z + (size_t(bh) * Tp + t) * KD + 4 * lane, ld4(&sm.z[4 * lane]));
    __syncwarp();
  }
}

// carry_kernel: per (batch, head), reverse over chunks:
//   X_S = -sum_t e^(P_t) z_t y_t^T, X_C = sum_t e^(P_t) dO_t y_t^T,
//   Sbar_end[n] = carry, carry = X_S[n] + e^(P_L) carry (same for C).
// The final carries are the gradients of the initial state.
template <int P>
__global__ void __launch_bounds__(256) carry_kernel(
    int B, int T, int H, const float* __restrict__ beta, const float* __restrict__ log_decay,
    const float* __restrict__ Y, const float* __restrict__ Z, const float* __restrict__ d_out,
    const float* __restrict__ d_sfin, const float* __restrict__ d_cfin,
    float* __restrict__ sbar, float* __restrict__ cbar, float* __restrict__ d_init_s,
    float* __restrict__ d_init_c) {
  constexpr int LP = P + 1, NJ = P / 16;
  extern __shared__ __align__(16) float sh[];
  float* Ys = sh;               // [64][LD] rows t
  float* Zs = Ys + CH * LD;     // [64][LD]
  float* Os = Zs + CH * LD;     // [64][LP]
  float* pre = Os + CH * LP;
  float* bet = pre + CH;
  const int Tp = (T + CH - 1) / CH * CH, nch = Tp / CH;
  const int bh = blockIdx.x, b = bh / H, h = bh % H;
  const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;
  // carries: S [64 x 64] rows ty+16i, cols tx+16j; C [P x 64]: rows p = tx + 16 j', cols d = ty + 16 i
  float cs[4][4], cc[4][NJ];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
#pragma unroll
    for (int j = 0; j < 4; ++j)
      cs[i][j] = d_sfin ? d_sfin[(size_t(bh) * KD + ty + 16 * i) * KD + tx + 16 * j] : 0.f;
#pragma unroll
    for (int j = 0; j < NJ; ++j)
      cc[i][j] = d_cfin ? d_cfin[(size_t(bh) * P + tx + 16 * j) * KD + ty + 16 * i] : 0.f;
  }
  for (int ch = nch - 1; ch >= 0; --ch) {
    const int t0 = ch * CH;
    float* sb = sbar + (size_t(bh) * nch + ch) * KD * KD;
    float* cbp = cbar + (size_t(bh) * nch + ch) * P * KD;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
#pragma unroll
      for (int j = 0; j < 4; ++j) sb[(ty + 16 * i) * KD + tx + 16 * j] = cs[i][j];
#pragma unroll
      for (int j = 0; j < NJ; ++j) cbp[(tx + 16 * j) * KD + ty + 16 * i] = cc[i][j];
    }
    __syncthreads();  // previous iteration's readers of Ys/Zs/Os are done
    load_block(Ys, CH, Y + (size_t(bh) * Tp + t0) * KD, tid);
    load_block(Zs, CH, Z + (size_t(bh) * Tp + t0) * KD, tid);
    load_tokens<P>(Os, LP, d_out, b, T, H, h, t0, tid);
    chunk_gates(tid, b, T, H, h, t0, beta, log_decay, pre, bet);
    __syncthreads();
    const float end = expf(pre[CH - 1]);
    float xs[4][4], xc[4][NJ];
    zero(xs);
    zero(xc);
    // xs[d][e] = sum_t e^(P_t) z_t[d] y_t[e]
    mm<4, CH>(xs, ty, tx, [&](int r, int k) { return Zs[k * LD + r] * expf(pre[k]); },
              [&](int k, int c) { return Ys[k * LD + c]; });
    // xc[d][p] (transposed) = sum_t e^(P_t) y_t[d] dO_t[p]
    mm<NJ, CH>(xc, ty, tx, [&](int r, int k) { return Ys[k * LD + r] * expf(pre[k]); },
               [&](int k, int c) { return Os[k * LP + c]; });
#pragma unroll
    for (int i = 0; i < 4; ++i) {
#pragma unroll
      for (int j = 0; j < 4; ++j) cs[i][j] = fmaf(end, cs[i][j], -xs[i][j]);
#pragma unroll
      for (int j = 0; j < NJ; ++j) cc[i][j] = fmaf(end, cc[i][j], xc[i][j]);
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if (d_init_s) {
#pragma unroll
      for (int j = 0; j < 4; ++j) d_init_s[(size_t(bh) * KD + ty + 16 * i) * KD + tx + 16 * j] = cs[i][j];
    }
    if (d_init_c) {
#pragma unroll
      for (int j = 0; j < NJ; ++j) d_init_c[(size_t(bh) * P + tx + 16 * j) * KD + ty + 16 * i] = cc[i][j];
    }
  }
}

// grads_kernel: every input gradient of one chunk (chunk form, see header).
template <int P>
__global__ void __launch_bounds__(256) grads_kernel(
    int B, int T, int H, const float* __restrict__ keys, const float* __restrict__ values,
    const float* __restrict__ beta, const float* __restrict__ log_decay,
    const float* __restrict__ Y, const float* __restrict__ Z, const float* __restrict__ s_start,
    const float* __restrict__ c_start, const float* __restrict__ sbar,
    const float* __restrict__ cbar, const float* __restrict__ d_out,
    const float* __restrict__ d_var, float* __restrict__ dk, float* __restrict__ dv,
    float* __restrict__ dq, float* __restrict__ dbeta, float* __restrict__ dlog,
    float* __restrict__ floor_part) {
  constexpr int LP = P + 1, NJ = P / 16;
  extern __shared__ __align__(16) float sh[];
  float* Ys = sh;                 // [64][LD]
  float* Zs = Ys + CH * LD;       // [64][LD]
  float* Ks = Zs + CH * LD;       // [64][LD]
  float* M1 = Ks + CH * LD;       // [64][LD]  W o GY
  float* M2 = M1 + CH * LD;       // [64][LD]  W o (OV - GZ)
  float* Os = M2 + CH * LD;       // [64][LP]
  float* Vs = Os + CH * LP;       // [64][LP]
  float* Sb = Vs + CH * LP;       // [64][LD] dS_end (later: S0)
  float* Cb = Sb + CH * LD;       // [P][LD]  dC_end (later: C0)
  float* pre = Cb + P * LD;
  float* bet = pre + CH;
  float* rowA = bet + CH;         // [64] sum_s dW W [t,.]
  float* colA = rowA + CH;        // [64] sum_t dW W [.,s]  and dW D col sums
  float* colB = colA + CH;        // [64]
  float* wbar = colB + CH;        // [64] dw_s
  float* extra = wbar + CH;       // [64] per-token e^P(-z S0 y + dO C0 y)
  float* red = extra + CH;        // [64] misc reduction scratch
  const int Tp = (T + CH - 1) / CH * CH, nch = Tp / CH, nsub = Tp / SUB;
  const int ch = blockIdx.x % nch, bh = blockIdx.x / nch, b = bh / H, h = bh % H;
  const int t0 = ch * CH, tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;
  load_block(Ys, CH, Y + (size_t(bh) * Tp + t0) * KD, tid);
  load_block(Zs, CH, Z + (size_t(bh) * Tp + t0) * KD, tid);
  load_tokens<KD>(Ks, LD, keys, b, T, H, h, t0, tid);
  load_tokens<P>(Os, LP, d_out, b, T, H, h, t0, tid);
  load_tokens<P>(Vs, LP, values, b, T, H, h, t0, tid);
  load_block(Sb, KD, sbar + (size_t(bh) * nch + ch) * KD * KD, tid);
  load_block(Cb, P, cbar + (size_t(bh) * nch + ch) * P * KD, tid);
  chunk_gates(tid, b, T, H, h, t0, beta, log_decay, pre, bet);
  if (tid < CH) { rowA[tid] = 0.f; colA[tid] = 0.f; colB[tid] = 0.f; }
  __syncthreads();
  const float pl = pre[CH - 1];
  // GY, GZ, OV -> M1, M2, dW products.
  {
    float gy[4][4], gz[4][4], ov[4][4];
    zero(gy); zero(gz); zero(ov);
    mm<4, KD>(gy, ty, tx, [&](int r, int k) { return Ys[r * LD + k]; },
              [&](int k, int c) { return Ks[c * LD + k]; });
    mm<4, KD>(gz, ty, tx, [&](int r, int k) { return Zs[r * LD + k]; },
              [&](int k, int c) { return Ks[c * LD + k]; });
    mm<4, P>(ov, ty, tx, [&](int r, int k) { return Os[r * LP + k]; },
             [&](int k, int c) { return Vs[c * LP + k]; });
    float rsum[4] = {0.f, 0.f, 0.f, 0.f}, csum[4] = {0.f, 0.f, 0.f, 0.f}, cdec[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int r = ty + 16 * i, c = tx + 16 * j;
        const bool on = c <= r;
        const float dec = on ? expf(pre[r] - pre[c]) : 0.f;
        const float w = dec * bet[c];
        const float diff = ov[i][j] - gz[i][j];
        M1[r * LD + c] = w * gy[i][j];
        M2[r * LD + c] = w * diff;
        const float dw = on ? gy[i][j] * diff : 0.f;
        rsum[i] = fmaf(dw, w, rsum[i]);
        csum[j] = fmaf(dw, w, csum[j]);
        cdec[j] = fmaf(dw, dec, cdec[j]);
      }
    // Reduce over the 16 tx lanes (rows) and 16 ty groups (columns) via smem.
    // Row sums: lanes with the same ty share a half-warp.
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float v = rsum[i];
#pragma unroll
      for (int o = 1; o < 16; o <<= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      if (tx == 0) rowA[ty + 16 * i] = v;
    }
    __syncthreads();
    // Column sums: accumulate deterministically by ty in order.
    for (int g = 0; g < 16; ++g) {
      if (ty == g) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          colA[tx + 16 * j] += csum[j];
          colB[tx + 16 * j] += cdec[j];
        }
      }
      __syncthreads();
    }
  }
  // dw_s = k^T Sb k + v^T Cb k ; also (Sb + Sb^T) k and Cb^T v rows for dK, Cb k for dV.
  float tk[4][4], ck[4][NJ];
  {
    zero(tk);
    // tk[s][d] = sum_e K[s][e] (Sb[d][e] + Sb[e][d]) + sum_p V[s][p] Cb[p][d]
    mm<4, KD>(tk, ty, tx, [&](int r, int k) { return Ks[r * LD + k]; },
              [&](int k, int c) { return Sb[c * LD + k] + Sb[k * LD + c]; });
    mm<4, P>(tk, ty, tx, [&](int r, int k) { return Vs[r * LP + k]; },
             [&](int k, int c) { return Cb[k * LD + c]; });
    zero(ck);
    // ck[s][p] = sum_d Cb[p][d] K[s][d]
    mm<NJ, KD>(ck, ty, tx, [&](int r, int k) { return Ks[r * LD + k]; },
               [&](int k, int c) { return Cb[c * LD + k]; });
    // dw_s = 1/2 k.(Sb+Sb^T)k ... computed as k.(tk_S) needs split: recompute directly.
    float part[4] = {0.f, 0.f, 0.f, 0.f};
    // k^T Sb k = 1/2 k^T (Sb + Sb^T) k ; v^T Cb k = sum_p v_p (Cb k)_p
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int s = ty + 16 * i;
#pragma unroll
      for (int j = 0; j < NJ; ++j) part[i] = fmaf(Vs[s * LP + tx + 16 * j], ck[i][j], part[i]);
    }
    float sk[4][4];
    zero(sk);
    mm<4, KD>(sk, ty, tx, [&](int r, int k) { return Ks[r * LD + k]; },
              [&](int k, int c) { return Sb[c * LD + k]; });  // sk[s][d] = (Sb k_s)[d]
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int s = ty + 16 * i;
#pragma unroll
      for (int j = 0; j < 4; ++j) part[i] = fmaf(Ks[s * LD + tx + 16 * j], sk[i][j], part[i]);
      float v = part[i];
#pragma unroll
      for (int o = 1; o < 16; o <<= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      if (tx == 0) wbar[s] = v;
    }
  }
  __syncthreads();
  // dK and dV.
  {
    float acc[4][4];
    zero(acc);
    // -(M1)^T Z + (M2)^T Y : acc[s][d] = sum_t (-M1[t][s] Z[t][d] + M2[t][s] Y[t][d])
    mm<4, CH>(acc, ty, tx, [&](int r, int k) { return -M1[k * LD + r]; },
              [&](int k, int c) { return Zs[k * LD + c]; });
    mm<4, CH>(acc, ty, tx, [&](int r, int k) { return M2[k * LD + r]; },
              [&](int k, int c) { return Ys[k * LD + c]; });
    float accv[4][NJ];
    zero(accv);
    mm<NJ, CH>(accv, ty, tx, [&](int r, int k) { return M1[k * LD + r]; },
               [&](int k, int c) { return Os[k * LP + c]; });
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int s = ty + 16 * i, t = t0 + s;
      if (t >= T) continue;
      const float ws = bet[s] * expf(pl - pre[s]);
#pragma unroll
      for (int j = 0; j < 4; ++j)
        dk[((size_t(b) * T + t) * H + h) * KD + tx + 16 * j] = fmaf(ws, tk[i][j], acc[i][j]);
#pragma unroll
      for (int j = 0; j < NJ; ++j)
        dv[((size_t(b) * T + t) * H + h) * P + tx + 16 * j] = fmaf(ws, ck[i][j], accv[i][j]);
    }
  }
  // <Sb, S0>, <Cb, C0> (before overwriting Sb/Cb with S0/C0).
  __syncthreads();
  float dot_end = 0.f;
  {
    const float* s0 = s_start + (size_t(bh) * nsub + ch * (CH / SUB)) * KD * KD;
    const float* c0 = c_start + (size_t(bh) * nch + ch) * P * KD;
    float part = 0.f;
    for (int idx = tid; idx < KD * KD; idx += 256) part = fmaf(Sb[(idx / KD) * LD + idx % KD], s0[idx], part);
    for (int idx = tid; idx < P * KD; idx += 256) part = fmaf(Cb[(idx / KD) * LD + idx % KD], c0[idx], part);
    part = warp_sum(part);
    if ((tid & 31) == 0) red[tid >> 5] = part;
    __syncthreads();
    if (tid == 0) {
      float s = 0.f;
      for (int w = 0; w < 8; ++w) s += red[w];
      red[32] = s;
    }
    __syncthreads();
    dot_end = red[32];
    __syncthreads();
    load_block(Sb, KD, s0, tid);
    load_block(Cb, P, c0, tid);
  }
  __syncthreads();
  // extra_t = e^(P_t) (-z_t . (S0 y_t) + dO_t . (C0 y_t))
  {
    float sy[4][4], cy[4][NJ];
    zero(sy);
    zero(cy);
    mm<4, KD>(sy, ty, tx, [&](int r, int k) { return Ys[r * LD + k]; },
              [&](int k, int c) { return Sb[c * LD + k]; });
    mm<NJ, KD>(cy, ty, tx, [&](int r, int k) { return Ys[r * LD + k]; },
               [&](int k, int c) { return Cb[c * LD + k]; });
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int r = ty + 16 * i;
      float v = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) v = fmaf(-Zs[r * LD + tx + 16 * j], sy[i][j], v);
#pragma unroll
      for (int j = 0; j < NJ; ++j) v = fmaf(Os[r * LP + tx + 16 * j], cy[i][j], v);
#pragma unroll
      for (int o = 1; o < 16; o <<= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      if (tx == 0) extra[r] = v * expf(pre[r]);
    }
  }
  __syncthreads();
  // Per-token scalars: dbeta, dP -> reverse cumsum -> dlog_decay; dq; floor part.
  if (tid < CH) {
    const int s = tid;
    const float tail = expf(pl - pre[s]);
    const float ws = bet[s] * tail;
    red[s] = rowA[s] - colA[s] - wbar[s] * ws + extra[s];
  }
  __syncthreads();
  if (tid == 0) {
    float last = 0.f;
    for (int s = 0; s < CH; ++s) last = fmaf(wbar[s], bet[s] * expf(pl - pre[s]), last);
    red[CH - 1] += last + expf(pl) * dot_end;
  }
  __syncthreads();
  if (tid < 32) {
    // reverse inclusive cumsum over 64 entries: two halves
    float hi = red[32 + (31 - tid)];
    float shi = warp_inclusive_scan(hi, tid);   // suffix sums of upper half
    const float tot_hi = __shfl_sync(0xffffffffu, shi, 31);
    float lo = red[31 - tid];
    float slo = warp_inclusive_scan(lo, tid) + tot_hi;
    // write: position 32 + (31 - tid) gets shi, position 31 - tid gets slo
    const int thi = t0 + 32 + (31 - tid), tlo = t0 + 31 - tid;
    if (thi < T) dlog[(size_t(b) * T + thi) * H + h] = shi;
    if (tlo < T) dlog[(size_t(b) * T + tlo) * H + h] = slo;
  }
  if (tid >= 64 && tid < 128) {
    const int s = tid - 64, t = t0 + s;
    if (t < T) dbeta[(size_t(b) * T + t) * H + h] = colB[s] + wbar[s] * expf(pl - pre[s]);
  }
  // dq = z + dvar y ; floor partial = -sum_t z o y
  for (int idx = tid; idx < CH * KD; idx += 256) {
    const int r = idx / KD, c = idx % KD, t = t0 + r;
    if (t < T) {
      const float dvv = d_var[(size_t(b) * T + t) * H + h];
      dq[((size_t(b) * T + t) * H + h) * KD + c] = fmaf(dvv, Ys[r * LD + c], Zs[r * LD + c]);
    }
  }
  if (tid < KD) {
    float f = 0.f;
    for (int r = 0; r < CH; ++r) f = fmaf(-Zs[r * LD + tid], Ys[r * LD + tid], f);
    floor_part[((size_t(b) * nch + ch) * H + h) * KD + tid] = f;
  }
}

__global__ void floor_reduce_kernel(int rows, int H, const float* __restrict__ part, float* __restrict__ d_floor) {
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= H * KD) return;
  float s = 0.f;
  for (int r = 0; r < rows; ++r) s += part[size_t(r) * H * KD + idx];
  d_floor[idx] = s;
}

template <int P>
size_t output_smem() { return (3 * CH * LD + CH * (P + 1) + P * LD + 2 * CH) * sizeof(float); }
template <int P>
size_t rhs_smem() { return (2 * CH * LD + 2 * CH * (P + 1) + P * LD + 2 * CH) * sizeof(float); }
template <int P>
size_t carry_smem() { return (2 * CH * LD + CH * (P + 1) + 2 * CH) * sizeof(float); }
template <int P>
size_t grads_smem() { return (6 * CH * LD + 2 * CH * (P + 1) + P * LD + 8 * CH) * sizeof(float); }

template <int P>
int forward(const M4MemDims& d, const float* keys, const float* values, const float* queries,
            const float* beta, const float* log_decay, const float* floor_, const float* init_s,
            const float* init_c, float* out, float* var, float* s_fin, float* c_fin, char* resid,
            cudaStream_t st) {
  const Sizes z = sizes(d);
  float* Lst = reinterpret_cast<float*>(resid + z.l_off);
  float* Y = reinterpret_cast<float*>(resid + z.y_off);
  float* Ss = reinterpret_cast<float*>(resid + z.s_off);
  float* Cs = reinterpret_cast<float*>(resid + z.c_off);
  const int bh = z.B * z.H;
  states_kernel<P><<<bh, 256, 0, st>>>(z.B, z.T, z.H, keys, values, beta, log_decay, init_s, init_c,
                                       Ss, Cs, s_fin, c_fin);
  const int warps = bh * z.nsub;
  const int ssm = int(sizeof(SolveSmem) * WARPS);
  cudaFuncSetAttribute(solve_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, ssm);
  solve_kernel<<<(warps + WARPS - 1) / WARPS, 32 * WARPS, ssm, st>>>(
      z.B, z.T, z.H, keys, queries, beta, log_decay, floor_, Ss, Lst, Y, var);
  const size_t osm = output_smem<P>();
  cudaFuncSetAttribute(output_kernel<P>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(osm));
  output_kernel<P><<<bh * z.nch, 256, osm, st>>>(z.B, z.T, z.H, keys, values, beta, log_decay, Y, Cs, out);
  return launch_status();
}

template <int P>
int backward(const M4MemDims& d, const float* keys, const float* values, const float* queries,
             const float* beta, const float* log_decay, const char* resid, const float* d_out,
             const float* d_var, const float* d_sfin, const float* d_cfin, float* dk, float* dv,
             float* dq, float* dbeta, float* dlog, float* dfloor, float* d_init_s, float* d_init_c,
             char* work, cudaStream_t st) {
  const Sizes z = sizes(d);
  const float* Lst = reinterpret_cast<const float*>(resid + z.l_off);
  const float* Y = reinterpret_cast<const float*>(resid + z.y_off);
  const float* Ss = reinterpret_cast<const float*>(resid + z.s_off);
  const float* Cs = reinterpret_cast<const float*>(resid + z.c_off);
  float* G = reinterpret_cast<float*>(work + z.g_off);
  float* Zb = reinterpret_cast<float*>(work + z.z_off);
  float* sb = reinterpret_cast<float*>(work + z.sb_off);
  float* cb = reinterpret_cast<float*>(work + z.cb_off);
  float* fl = reinterpret_cast<float*>(work + z.fl_off);
  const int bh = z.B * z.H;
  const size_t rsm = rhs_smem<P>();
  cudaFuncSetAttribute(rhs_kernel<P>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(rsm));
  rhs_kernel<P><<<bh * z.nch, 256, rsm, st>>>(z.B, z.T, z.H, keys, values, queries, beta, log_decay, Cs,
                                              d_out, d_var, G);
  const int warps = bh * z.nsub;
  zsolve_kernel<<<(warps + WARPS - 1) / WARPS, 32 * WARPS, 0, st>>>(z.B, z.T, z.H, Lst, G, Zb);
  const size_t csm = carry_smem<P>();
  cudaFuncSetAttribute(carry_kernel<P>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(csm));
  carry_kernel<P><<<bh, 256, csm, st>>>(z.B, z.T, z.H, beta, log_decay, Y, Zb, d_out, d_sfin, d_cfin, sb,
                                        cb, d_init_s, d_init_c);
  const size_t gsm = grads_smem<P>();
  cudaFuncSetAttribute(grads_kernel<P>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(gsm));
  grads_kernel<P><<<bh * z.nch, 256, gsm, st>>>(z.B, z.T, z.H, keys, values, beta, log_decay, Y, Zb, Ss,
                                                Cs, sb, cb, d_out, d_var, dk, dv, dq, dbeta, dlog, fl);
  floor_reduce_kernel<<<(z.H * KD + 255) / 256, 256, 0, st>>>(z.B * z.nch, z.H, fl, dfloor);
  return launch_status();
}

inline int check(const M4MemDims* d) {
  if (!d) return M4_ERR_NULL;
  if (d->batch <= 0 || d->time <= 0 || d->heads <= 0 || d->key_dim <= 0 || d->value_dim <= 0)
    return M4_ERR_DIMS;
  if (d->key_dim != KD || (d->value_dim != 64 && d->value_dim != 128)) return M4_ERR_UNSUPPORTED;
  return M4_OK;
}

}  // namespace mem
}  // namespace m4

using namespace m4;

extern "C" size_t m4_memread_residual_bytes(const M4MemDims* d) {
  return mem::check(d) == M4_OK ? mem::sizes(*d).resid_bytes : 0;
}

extern "C" size_t m4_memread_workspace_bytes(const M4MemDims* d) {
  return mem::check(d) == M4_OK ? mem::sizes(*d).work_bytes : 0;
}

extern "C" int m4_memread_fwd(const M4MemDims* d, const float* keys, const float* values,
                              const float* queries, const float* beta, const float* log_decay,
                              const float* floor_, const float* init_s, const float* init_c,
                              float* out, float* var, float* s_fin, float* c_fin, void* resid,
                              size_t resid_bytes, void* stream) {
  int st = mem::check(d);
  if (st) return st;
  if (!keys || !values || !queries || !beta || !log_decay || !floor_ || !out || !var || !s_fin ||
      !c_fin || !resid)
    return M4_ERR_NULL;
  if ((init_s == nullptr) != (init_c == nullptr)) return M4_ERR_NULL;
  if (!aligned16(keys) || !aligned16(queries) || !aligned16(resid)) return M4_ERR_ALIGN;
  if (resid_bytes < mem::sizes(*d).resid_bytes) return M4_ERR_WORKSPACE;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (d->value_dim == 64)
    return mem::forward<64>(*d, keys, values, queries, beta, log_decay, floor_, init_s, init_c, out, var,
                            s_fin, c_fin, static_cast<char*>(resid), s);
  return mem::forward<128>(*d, keys, values, queries, beta, log_decay, floor_, init_s, init_c, out, var,
                           s_fin, c_fin, static_cast<char*>(resid), s);
}

extern "C" int m4_memread_bwd(const M4MemDims* d, const float* keys, const float* values,
                              const float* queries, const float* beta, const float* log_decay,
                              const float* floor_, const float* init_s, const float* init_c,
                              const void* resid, size_t resid_bytes, const float* d_out,
                              const float* d_var, const float* d_sfin, const float* d_cfin, float* dk,
                              float* dv, float* dq, float* dbeta, float* dlog, float* dfloor,
                              float* d_init_s, float* d_init_c, void* work, size_t work_bytes,
                              void* stream) {
  (void)floor_;
  (void)init_s;
  (void)init_c;
  int st = mem::check(d);
  if (st) return st;
  if (!keys || !values || !queries || !beta || !log_decay || !resid || !d_out || !d_var || !dk ||
      !dv || !dq || !dbeta || !dlog || !dfloor || !work)
    return M4_ERR_NULL;
  if (!aligned16(resid) || !aligned16(work)) return M4_ERR_ALIGN;
  const mem::Sizes z = mem::sizes(*d);
  if (resid_bytes < z.resid_bytes || work_bytes < z.work_bytes) return M4_ERR_WORKSPACE;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const char* r = static_cast<const char*>(resid);
  char* w = static_cast<char*>(work);
  if (d->value_dim == 64)
    return mem::backward<64>(*d, keys, values, queries, beta, log_decay, r, d_out, d_var, d_sfin, d_cfin,
                             dk, dv, dq, dbeta, dlog, dfloor, d_init_s, d_init_c, w, s);
  return mem::backward<128>(*d, keys, values, queries, beta, log_decay, r, d_out, d_var, d_sfin, d_cfin,
                            dk, dv, dq, dbeta, dlog, dfloor, d_init_s, d_init_c, w, s);
}
