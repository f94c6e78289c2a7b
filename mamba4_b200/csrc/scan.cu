// Mamba-3 SISO chunked scan (rotation, phase and trapezoidal weights fused),
// forward and backward, for sm_100a.
//
// Reference operator: mamba3_fused (lm/kernels/flashmamba.py:1114-1162) ->
// fused_scan custom VJP (:859-1102) with kernels _fused_forward_kernel
// (:589-660) and _fused_backward_kernel (:663-786). Per head h and chunk of
// `chunk` tokens, with p = chunk-local prefix of adt, the phase
// theta_t = phase0 + sum_{s<=t} rate_s dt_s, Q/K = rotated, biased C/B:
//   W[t,s] = e^(p_t-p_s) scale_s (s < t), gamma_t (s = t)
//   y      = ((Q K^T) o W) V + e^(p_t) Q state
//   state  = e^(p_L) state + K^T (V o scale o tail)
// Model-dtype (bf16) rounding points follow the reference kernel: bias add,
// rotation, masked scores, carried-state read, weighted values, output, and
// in the backward the score/value cotangent products (:734-751).
//
// This version: one CTA (4 warps) per (batch, head), chunks in sequence, the
// chunk products on bf16 mma.sync tensor-core tiles with fp32 accumulation
// (fp32 inputs use an exact CUDA-core path with the same fragment ownership).
#include "common.cuh"

#include <cuda.h>
#include <cudaTypedefs.h>

namespace m4 {
namespace scan {

constexpr int C = 64;      // chunk length
constexpr int HP = 64;     // head dim P
constexpr int LDS = 68;    // smem tile stride (floats)
constexpr int THREADS = 128;

M4_DEV uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

M4_DEV void mma16816(float (&d)[4], const uint32_t (&a)[4], const uint32_t (&b)[2]) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

// Warp tile: rows row0 + g and row0 + g + 8 (g = lane/4), columns
// nt*8 + 2c, 2c+1 (c = lane%4) for nt < 8: acc[nt][0..1] row g, [2..3] row g+8.
// C[16 x 64] += A[16 x K] B[K x 64] with element accessors fa(row, k), fb(k, col).
template <bool BF, int K, class FA, class FB>
M4_DEV void warp_gemm(float (&acc)[8][4], int row0, FA fa, FB fb) {
  const int lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
  if constexpr (BF) {
#pragma unroll
    for (int k0 = 0; k0 < K; k0 += 16) {
      uint32_t a[4];
      a[0] = pack_bf16(fa(row0 + g, k0 + 2 * c), fa(row0 + g, k0 + 2 * c + 1));
      a[1] = pack_bf16(fa(row0 + g + 8, k0 + 2 * c), fa(row0 + g + 8, k0 + 2 * c + 1));
      a[2] = pack_bf16(fa(row0 + g, k0 + 2 * c + 8), fa(row0 + g, k0 + 2 * c + 9));
      a[3] = pack_bf16(fa(row0 + g + 8, k0 + 2 * c + 8), fa(row0 + g + 8, k0 + 2 * c + 9));
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        uint32_t b[2];
        b[0] = pack_bf16(fb(k0 + 2 * c, nt * 8 + g), fb(k0 + 2 * c + 1, nt * 8 + g));
        b[1] = pack_bf16(fb(k0 + 2 * c + 8, nt * 8 + g), fb(k0 + 2 * c + 9, nt * 8 + g));
        mma16816(acc[nt], a, b);
      }
    }
  } else {
#pragma unroll 4
    for (int k = 0; k < K; ++k) {
      const float a0 = fa(row0 + g, k), a1 = fa(row0 + g + 8, k);
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        const float b0 = fb(k, nt * 8 + 2 * c), b1 = fb(k, nt * 8 + 2 * c + 1);
        acc[nt][0] = fmaf(a0, b0, acc[nt][0]);
        acc[nt][1] = fmaf(a0, b1, acc[nt][1]);
        acc[nt][2] = fmaf(a1, b0, acc[nt][2]);
        acc[nt][3] = fmaf(a1, b1, acc[nt][3]);
      }
    }
  }
}

M4_DEV void zero8(float (&acc)[8][4]) {
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
}

// Visit the warp tile's elements: f(row, col, value).
template <class F>
M4_DEV void for_tile(const float (&acc)[8][4], int row0, F f) {
  const int lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
#pragma unroll
  for (int nt = 0; nt < 8; ++nt) {
    f(row0 + g, nt * 8 + 2 * c, acc[nt][0]);
    f(row0 + g, nt * 8 + 2 * c + 1, acc[nt][1]);
    f(row0 + g + 8, nt * 8 + 2 * c, acc[nt][2]);
    f(row0 + g + 8, nt * 8 + 2 * c + 1, acc[nt][3]);
  }
}

struct Dims {
  int B, T, H, A, nch;
  bool per_head;
};

// Per-token chunk scalars shared by the forward and backward kernels.
struct Rows {
  float p[C], gam[C], scl[C], tail[C], dt[C], trap[C];
};

// Fill Rows for chunk t0 of (b, h) (threads 0..63; warp 0 does the prefix).
M4_DEV void chunk_rows(const Dims& d, int b, int h, int t0, const float* adt, const float* dt,
                       const float* trap_logits, Rows& r, float* scratch) {
  const int tid = threadIdx.x;
  if (tid < C) {
    const int t = t0 + tid;
    const bool live = t < d.T;
    const size_t i = (size_t(b) * d.T + t) * d.H + h;
    const float dtv = live ? dt[i] : 0.f;
    const float tr = live ? 1.f / (1.f + expf(-trap_logits[i])) : 0.f;
    float next = 0.f;
    if (t + 1 < d.T) {
      const size_t j = (size_t(b) * d.T + t + 1) * d.H + h;
      const float trn = 1.f / (1.f + expf(-trap_logits[j]));
      next = dt[j] * (1.f - trn);
    }
    r.dt[tid] = dtv;
    r.trap[tid] = tr;
    r.gam[tid] = dtv * tr;
    r.scl[tid] = dtv * tr + next;
    scratch[tid] = live ? adt[i] : 0.f;
  }
  __syncthreads();
  if (tid < 32) {
    const float v0 = warp_inclusive_scan(scratch[tid], tid);
    const float tot = __shfl_sync(0xffffffffu, v0, 31);
    const float v1 = warp_inclusive_scan(scratch[32 + tid], tid) + tot;
    r.p[tid] = v0;
    r.p[32 + tid] = v1;
  }
  __syncthreads();
  if (tid < C) r.tail[tid] = expf(r.p[C - 1] - r.p[tid]);
}

// Strides of the state-dim-templated tiles: [C][NS] tiles (rotated Q / K and
// the N-wide gradient tile) and [C][pairs] tables (phases).
template <int NS> constexpr int ldn() { return NS + 4; }
template <int NS> constexpr int tw() { return NS / 2 + 1; }

// Phase theta[t][i] = phase0[i] + sum_{s<=t} rate_s[i] dt_s for pairs i < A.
template <int NS>
M4_DEV void chunk_theta(const Dims& d, int b, int h, int t0, const float* angles, const Rows& r,
                        const float* phase0, float* theta) {
  const int tid = threadIdx.x;
  if (tid < d.A) {
    float acc = phase0[tid];
    for (int tt = 0; tt < C; ++tt) {
      const int t = t0 + tt;
      float rate = 0.f;
      if (t < d.T)
        rate = d.per_head ? angles[((size_t(b) * d.T + t) * d.H + h) * d.A + tid]
                          : angles[(size_t(b) * d.T + t) * d.A + tid];
      acc = fmaf(rate, r.dt[tt], acc);
      theta[tt * tw<NS>() + tid] = acc;
    }
  }
}

// Biased, rounded query/key pair (2i, 2i+1) of token t0 + tt, before rotation.
template <typename T, int NS>
M4_DEV void load_pair(const Dims& d, int b, int h, int t, const T* cq, const T* bk, const float* qb,
                      const float* kb, int i, float (&q)[2], float (&k)[2]) {
  const int n0 = 2 * i, n1 = 2 * i + 1;
  float c0 = 0.f, c1 = 0.f, b0 = 0.f, b1 = 0.f;
  if (t < d.T) {
    const size_t base = d.per_head ? ((size_t(b) * d.T + t) * d.H + h) * NS : (size_t(b) * d.T + t) * NS;
    c0 = to_f(cq[base + n0]); c1 = to_f(cq[base + n1]);
    b0 = to_f(bk[base + n0]); b1 = to_f(bk[base + n1]);
  }
  q[0] = round_to<T>(c0 + (qb ? qb[h * NS + n0] : 0.f));
  q[1] = round_to<T>(c1 + (qb ? qb[h * NS + n1] : 0.f));
  k[0] = round_to<T>(b0 + (kb ? kb[h * NS + n0] : 0.f));
  k[1] = round_to<T>(b1 + (kb ? kb[h * NS + n1] : 0.f));
}

// Rotated, rounded Q and K tiles [C][ldn<NS>()].
template <typename T, int NS>
M4_DEV void build_qk(const Dims& d, int b, int h, int t0, const T* cq, const T* bk, const float* qb,
                     const float* kb, const float* theta, float* Qs, float* Ks) {
  for (int idx = threadIdx.x; idx < C * (NS / 2); idx += THREADS) {
    const int tt = idx / (NS / 2), i = idx % (NS / 2), t = t0 + tt;
    float q[2], k[2];
    load_pair<T, NS>(d, b, h, t, cq, bk, qb, kb, i, q, k);
    float cs = 1.f, sn = 0.f;
    if (i < d.A) sincosf(theta[tt * tw<NS>() + i], &sn, &cs);
    Qs[tt * ldn<NS>() + 2 * i] = round_to<T>(q[0] * cs - q[1] * sn);
    Qs[tt * ldn<NS>() + 2 * i + 1] = round_to<T>(q[1] * cs + q[0] * sn);
    Ks[tt * ldn<NS>() + 2 * i] = round_to<T>(k[0] * cs - k[1] * sn);
    Ks[tt * ldn<NS>() + 2 * i + 1] = round_to<T>(k[1] * cs + k[0] * sn);
  }
}

template <typename T>
M4_DEV void load_values(const Dims& d, int b, int h, int t0, const T* x, float* Vs) {
  for (int idx = threadIdx.x; idx < C * HP; idx += THREADS) {
    const int tt = idx / HP, p = idx % HP, t = t0 + tt;
    Vs[tt * LDS + p] = t < d.T ? to_f(x[(size_t(b) * d.T + t) * d.H * HP + h * HP + p]) : 0.f;
  }
}

// ---------------------------------------------------------------------------
// Forward (sequential chunks per (batch, head); state dim NS in {64, 96, 128}).
// ---------------------------------------------------------------------------
template <int NS>
inline size_t fwd_smem() {
  return (2 * C * ldn<NS>() + 2 * C * LDS + NS * LDS + C * tw<NS>() + NS / 2 + C + sizeof(Rows) / 4) *
         sizeof(float);
}

template <typename T, int NS>
__global__ void __launch_bounds__(THREADS) fwd_kernel(
    Dims d, const T* __restrict__ cq, const T* __restrict__ bk, const T* __restrict__ x,
    const float* __restrict__ adt, const float* __restrict__ dt, const float* __restrict__ trap_logits,
    const float* __restrict__ angles, const float* __restrict__ qb, const float* __restrict__ kb,
    T* __restrict__ y, float* __restrict__ final_state, float* __restrict__ starts,
    float* __restrict__ phases) {
  constexpr bool BF = sizeof(T) == 2;
  constexpr int LN = ldn<NS>(), TW = tw<NS>(), NP = NS / 2;
  extern __shared__ __align__(16) float sh[];
  float* Qs = sh;
  float* Ks = Qs + C * LN;
  float* Vs = Ks + C * LN;
  float* Ms = Vs + C * LDS;
  float* St = Ms + C * LDS;           // [NS][P] fp32 state
  float* theta = St + NS * LDS;       // [C][TW]
  float* phase = theta + C * TW;      // [NP]
  float* scratch = phase + NP;        // [64]
  Rows& r = *reinterpret_cast<Rows*>(scratch + C);
  const int bh = blockIdx.x, b = bh / d.H, h = bh % d.H;
  const int tid = threadIdx.x, warp = tid >> 5;
  const int row0 = warp * 16;
  for (int i = tid; i < NS * LDS; i += THREADS) St[i] = 0.f;
  if (tid < NP) phase[tid] = 0.f;
  __syncthreads();
  for (int ch = 0; ch < d.nch; ++ch) {
    const int t0 = ch * C;
    // Residuals: chunk-start state and phase.
    {
      float* sd = starts + (size_t(bh) * d.nch + ch) * NS * HP;
      for (int i = tid; i < NS * HP; i += THREADS) sd[i] = St[(i / HP) * LDS + i % HP];
      if (tid < NP) phases[(size_t(bh) * d.nch + ch) * NP + tid] = phase[tid];
    }
    chunk_rows(d, b, h, t0, adt, dt, trap_logits, r, scratch);
    __syncthreads();
    chunk_theta<NS>(d, b, h, t0, angles, r, phase, theta);
    __syncthreads();
    build_qk<T, NS>(d, b, h, t0, cq, bk, qb, kb, theta, Qs, Ks);
    load_values<T>(d, b, h, t0, x, Vs);
    if (tid < d.A) phase[tid] = theta[(C - 1) * TW + tid];
    __syncthreads();
    // Masked, weighted scores.
    {
      float acc[8][4];
      zero8(acc);
      warp_gemm<BF, NS>(acc, row0, [&](int i, int k) { return Qs[i * LN + k]; },
                        [&](int k, int j) { return Ks[j * LN + k]; });
      for_tile(acc, row0, [&](int t, int s, float v) {
        float w = 0.f;
        if (s < t) w = expf(r.p[t] - r.p[s]) * r.scl[s];
        else if (s == t) w = r.gam[t];
        Ms[t * LDS + s] = round_to<T>(v * w);
      });
    }
    __syncthreads();
    // y = mixed V + e^p Q state.
    {
      float acc[8][4], inh[8][4];
      zero8(acc);
      zero8(inh);
      warp_gemm<BF, C>(acc, row0, [&](int i, int k) { return Ms[i * LDS + k]; },
                       [&](int k, int j) { return Vs[k * LDS + j]; });
      warp_gemm<BF, NS>(inh, row0, [&](int i, int k) { return Qs[i * LN + k]; },
                        [&](int k, int j) { return round_to<T>(St[k * LDS + j]); });
      const int lane = tid & 31, g = lane >> 2, c = lane & 3;
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        const int tt = row0 + g + 8 * half, t = t0 + tt;
        if (t >= d.T) continue;
        const float e = expf(r.p[tt]);
        T* yrow = y + (size_t(b) * d.T + t) * d.H * HP + h * HP;
#pragma unroll
        for (int nt = 0; nt < 8; ++nt) {
          const int col = nt * 8 + 2 * c;
          yrow[col] = from_f<T>(fmaf(e, inh[nt][2 * half], acc[nt][2 * half]));
          yrow[col + 1] = from_f<T>(fmaf(e, inh[nt][2 * half + 1], acc[nt][2 * half + 1]));
        }
      }
    }
    __syncthreads();
    // state = e^(p_L) state + K^T (V o scale o tail), 16 state rows per warp pass.
    {
      const float end = expf(r.p[C - 1]);
      for (int n0 = row0; n0 < NS; n0 += 4 * 16) {
        float acc[8][4];
        zero8(acc);
        warp_gemm<BF, C>(acc, n0, [&](int n, int t) { return Ks[t * LN + n]; },
                         [&](int t, int p) { return round_to<T>(Vs[t * LDS + p] * (r.scl[t] * r.tail[t])); });
        for_tile(acc, n0, [&](int n, int p, float v) { St[n * LDS + p] = fmaf(end, St[n * LDS + p], v); });
      }
    }
    __syncthreads();
  }
  float* fd = final_state + size_t(bh) * NS * HP;
  for (int i = tid; i < NS * HP; i += THREADS) fd[i] = St[(i / HP) * LDS + i % HP];
}

// ---------------------------------------------------------------------------
// Backward: reverse chunks per (batch, head). The chunk-start state is read
// from the residual and the chunk-end state cotangent (the carry) lives in
// the workspace; both are [NS][P] fp32 slices that stay in L2. Per-head
// partial outputs go to workspace; head/batch reductions and the
// trapezoid/gate chain rule run in small follow-up kernels.
// ---------------------------------------------------------------------------
struct BwdOut {
  float* dq;      // [B,T,H,N] rotation-backed query gradient (per head)
  float* dk;      // [B,T,H,N]
  float* drate;   // [B,T,H,A] angle-rate gradient (per head)
  float* dgam;    // [B,T,H] d gamma
  float* dscl;    // [B,T,H] d scale
  float* dlog;    // [B,T,H] d adt
  float* ddtp;    // [B,T,H] d dt through the phase
  float* dqb;     // [B,H,N] bias partials
  float* dkb;     // [B,H,N]
  float* carry;   // [B,H,N,P] cotangent of the current chunk's end state
};

template <int NS>
inline size_t bwd_smem() {
  return (3 * C * ldn<NS>() + 4 * C * LDS + 2 * C * tw<NS>() + NS / 2 + C + 8 * C + sizeof(Rows) / 4) *
         sizeof(float);
}

// Rotation backward of one [C][NS] gradient tile G (rotated frame), in place
// to the pre-rotation frame, written to `out` [B,T,H,N]; the pair-phase
// gradient G . J rot(u) is added into dth [C][pairs] (u = the biased,
// rounded queries (QUERY) or keys).
template <typename T, int NS, bool QUERY>
M4_DEV void rotate_back(const Dims& d, int b, int h, int t0, const T* cq, const T* bk, const float* qb,
                        const float* kb, const float* theta, float* G, float* dth, float* out) {
  constexpr int LN = ldn<NS>(), TW = tw<NS>();
  for (int idx = threadIdx.x; idx < C * (NS / 2); idx += THREADS) {
    const int tt = idx / (NS / 2), i = idx % (NS / 2), t = t0 + tt;
    float q[2], k[2];
    load_pair<T, NS>(d, b, h, t, cq, bk, qb, kb, i, q, k);
    const float u0 = QUERY ? q[0] : k[0], u1 = QUERY ? q[1] : k[1];
    float cs = 1.f, sn = 0.f;
    if (i < d.A) sincosf(theta[tt * TW + i], &sn, &cs);
    const float r0 = u0 * cs - u1 * sn, r1 = u1 * cs + u0 * sn;  // fp32 rotated, before rounding
    const float g0 = G[tt * LN + 2 * i], g1 = G[tt * LN + 2 * i + 1];
    const float p0 = g0 * cs + g1 * sn, p1 = g1 * cs - g0 * sn;
    if (t < d.T) {
      const size_t base = ((size_t(b) * d.T + t) * d.H + h) * NS;
      out[base + 2 * i] = p0;
      out[base + 2 * i + 1] = p1;
    }
    G[tt * LN + 2 * i] = p0;
    G[tt * LN + 2 * i + 1] = p1;
    // partner(rot) = (-r1, r0) (flashmamba.py:776)
    const float v = i < d.A ? g0 * (-r1) + g1 * r0 : 0.f;
    dth[tt * TW + i] = QUERY ? dth[tt * TW + i] + v : v;
  }
}

template <typename T, int NS>
__global__ void __launch_bounds__(THREADS) bwd_kernel(
    Dims d, const T* __restrict__ cq, const T* __restrict__ bk, const T* __restrict__ x,
    const float* __restrict__ adt, const float* __restrict__ dt, const float* __restrict__ trap_logits,
    const float* __restrict__ angles, const float* __restrict__ qb, const float* __restrict__ kb,
    const float* __restrict__ starts, const float* __restrict__ phases, const T* __restrict__ dy,
    const float* __restrict__ d_final, T* __restrict__ dx, BwdOut o) {
  constexpr bool BF = sizeof(T) == 2;
  constexpr int LN = ldn<NS>(), TW = tw<NS>(), NP = NS / 2;
  extern __shared__ __align__(16) float sh[];
  float* Qs = sh;                     // rounded rotated queries [C][LN]
  float* Ks = Qs + C * LN;
  float* G = Ks + C * LN;             // dK, then dQ (rotated frame, then pre-rotation) [C][LN]
  float* Vs = G + C * LN;             // values [C][LDS]
  float* Dy = Vs + C * LDS;           // dY (model dtype values)
  float* Sc = Dy + C * LDS;           // scores  Q K^T
  float* Dm = Sc + C * LDS;           // d_mixed dY V^T
  float* theta = Dm + C * LDS;        // [C][TW] phase
  float* dth = theta + C * TW;        // [C][TW] pair-phase gradient, then its suffix sums
  float* later = dth + C * TW;        // [NP] phase-gradient carry per pair
  float* scratch = later + NP;        // [64]
  float* vec = scratch + C;           // [8][64] per-token accumulators
  Rows& r = *reinterpret_cast<Rows*>(vec + 8 * C);
  const int bh = blockIdx.x, b = bh / d.H, h = bh % d.H;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int row0 = warp * 16;
  float* Cy = o.carry + size_t(bh) * NS * HP;
  for (int i = tid; i < NS * HP; i += THREADS) Cy[i] = d_final ? d_final[size_t(bh) * NS * HP + i] : 0.f;
  if (tid < NP) later[tid] = 0.f;
  float qbs = 0.f, kbs = 0.f;  // bias partial sums for column tid (tid < NS)
  __syncthreads();
  for (int ch = d.nch - 1; ch >= 0; --ch) {
    const int t0 = ch * C;
    const float* St = starts + (size_t(bh) * d.nch + ch) * NS * HP;  // chunk-start state [NS][P]
    chunk_rows(d, b, h, t0, adt, dt, trap_logits, r, scratch);
    __syncthreads();
    chunk_theta<NS>(d, b, h, t0, angles, r, phases + (size_t(bh) * d.nch + ch) * NP, theta);
    __syncthreads();
    build_qk<T, NS>(d, b, h, t0, cq, bk, qb, kb, theta, Qs, Ks);
    load_values<T>(d, b, h, t0, x, Vs);
    load_values<T>(d, b, h, t0, dy, Dy);
    for (int i = tid; i < 8 * C; i += THREADS) vec[i] = 0.f;
    __syncthreads();
    // Scores and d_mixed.
    {
      float acc[8][4];
      zero8(acc);
      warp_gemm<BF, NS>(acc, row0, [&](int i, int k) { return Qs[i * LN + k]; },
                        [&](int k, int j) { return Ks[j * LN + k]; });
      for_tile(acc, row0, [&](int t, int s, float v) { Sc[t * LDS + s] = v; });
      zero8(acc);
      warp_gemm<BF, HP>(acc, row0, [&](int i, int k) { return Dy[i * LDS + k]; },
                        [&](int k, int j) { return Vs[j * LDS + k]; });
      for_tile(acc, row0, [&](int t, int s, float v) { Dm[t * LDS + s] = v; });
    }
    __syncthreads();
    auto wgt = [&](int t, int s) -> float {
      if (s < t) return expf(r.p[t] - r.p[s]) * r.scl[s];
      return s == t ? r.gam[t] : 0.f;
    };
    const float end = expf(r.p[C - 1]);
    const int g = lane >> 2, c = lane & 3;
    // dV = rd(mixed)^T dY + src o (K rd(carry)) ; write dx.
    {
      float acc[8][4], ve[8][4];
      zero8(acc);
      zero8(ve);
      warp_gemm<BF, C>(acc, row0, [&](int s, int t) { return round_to<T>(Sc[t * LDS + s] * wgt(t, s)); },
                       [&](int t, int p) { return Dy[t * LDS + p]; });
      warp_gemm<BF, NS>(ve, row0, [&](int s, int n) { return Ks[s * LN + n]; },
                        [&](int n, int p) { return round_to<T>(Cy[n * HP + p]); });
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        const int s = row0 + g + 8 * half, t = t0 + s;
        if (t >= d.T) continue;
        const float src = r.scl[s] * r.tail[s];
        T* row = dx + (size_t(b) * d.T + t) * d.H * HP + h * HP;
#pragma unroll
        for (int nt = 0; nt < 8; ++nt) {
          const int col = nt * 8 + 2 * c;
          row[col] = from_f<T>(fmaf(src, ve[nt][2 * half], acc[nt][2 * half]));
          row[col + 1] = from_f<T>(fmaf(src, ve[nt][2 * half + 1], acc[nt][2 * half + 1]));
        }
      }
    }
    // dK = rd(Dm o W)^T Q + src o (V rd(carry)^T) -> G (64 state columns per
    // pass); d_source = sum_n K (V rd(carry)^T).
    {
      float dsrc[2] = {0.f, 0.f};
      for (int nb = 0; nb < NS; nb += 64) {
        float acc[8][4], ve[8][4];
        zero8(acc);
        zero8(ve);
        warp_gemm<BF, C>(acc, row0, [&](int s, int t) { return round_to<T>(Dm[t * LDS + s] * wgt(t, s)); },
                         [&](int t, int n) { return nb + n < NS ? Qs[t * LN + nb + n] : 0.f; });
        warp_gemm<BF, HP>(ve, row0, [&](int s, int p) { return Vs[s * LDS + p]; },
                          [&](int p, int n) { return nb + n < NS ? round_to<T>(Cy[(nb + n) * HP + p]) : 0.f; });
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          const int s = row0 + g + 8 * half;
          const float src = r.scl[s] * r.tail[s];
#pragma unroll
          for (int nt = 0; nt < 8; ++nt)
#pragma unroll
            for (int e = 0; e < 2; ++e) {
              const int n = nb + nt * 8 + 2 * c + e;
              if (n < NS) {
                dsrc[half] = fmaf(Ks[s * LN + n], ve[nt][2 * half + e], dsrc[half]);
                G[s * LN + n] = fmaf(src, ve[nt][2 * half + e], acc[nt][2 * half + e]);
              }
            }
        }
      }
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        float v = dsrc[half];
        v += __shfl_xor_sync(0xffffffffu, v, 1);
        v += __shfl_xor_sync(0xffffffffu, v, 2);
        if (c == 0) vec[0 * C + row0 + g + 8 * half] = v;  // d_source
      }
    }
    // inherited . dY (dp term) : rows t, e^(p_t) sum_p dY[t,p] (Q rd(start))[t,p]
    {
      float acc[8][4];
      zero8(acc);
      warp_gemm<BF, NS>(acc, row0, [&](int t, int n) { return Qs[t * LN + n]; },
                        [&](int n, int p) { return round_to<T>(St[n * HP + p]); });
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        const int t = row0 + g + 8 * half;
        float v = 0.f;
#pragma unroll
        for (int nt = 0; nt < 8; ++nt)
#pragma unroll
          for (int e = 0; e < 2; ++e) v = fmaf(Dy[t * LDS + nt * 8 + 2 * c + e], acc[nt][2 * half + e], v);
        v += __shfl_xor_sync(0xffffffffu, v, 1);
        v += __shfl_xor_sync(0xffffffffu, v, 2);
        if (c == 0) vec[1 * C + t] = v * expf(r.p[t]);
      }
    }
    __syncthreads();
    // Per-token scalar gradients from d_weights = Dm o Sc.
    if (tid < C) {
      const int t = tid;
      float rowoff = 0.f, coloff = 0.f, cdec = 0.f;
      for (int s = 0; s < t; ++s) {
        const float dw = Dm[t * LDS + s] * Sc[t * LDS + s];
        rowoff = fmaf(dw, expf(r.p[t] - r.p[s]) * r.scl[s], rowoff);
      }
      for (int u = t + 1; u < C; ++u) {
        const float dw = Dm[u * LDS + t] * Sc[u * LDS + t];
        const float dec = expf(r.p[u] - r.p[t]);
        coloff = fmaf(dw, dec * r.scl[t], coloff);
        cdec = fmaf(dw, dec, cdec);
      }
      const float flow = vec[0 * C + t] * r.scl[t] * r.tail[t];
      vec[2 * C + t] = rowoff - coloff - flow + vec[1 * C + t];        // dp
      vec[3 * C + t] = Dm[t * LDS + t] * Sc[t * LDS + t];                // d gamma
      vec[4 * C + t] = vec[0 * C + t] * r.tail[t] + cdec;                // d scale
      vec[5 * C + t] = flow;
    }
    // <carry, start> for the chunk-end decay.
    {
      float part = 0.f;
      for (int i = tid; i < NS * HP; i += THREADS) part = fmaf(Cy[i], St[i], part);
      part = warp_sum(part);
      if (lane == 0) scratch[warp] = part;
    }
    // Rotation backward of dK (pre-rotation gradient to o.dk, its pair-phase
    // gradient into dth).
    rotate_back<T, NS, false>(d, b, h, t0, cq, bk, qb, kb, theta, G, dth, o.dk);
    __syncthreads();
    if (tid < 32) {
      // d_log_decay = suffix sum of dp (+ chunk-end terms at the last position)
      float fl = vec[5 * C + tid] + vec[5 * C + 32 + tid];
      fl = warp_sum(fl);
      const float extra = fl + end * (scratch[0] + scratch[1] + scratch[2] + scratch[3]);
      float hi = vec[2 * C + 63 - tid] + (tid == 0 ? extra : 0.f);
      const float shi = warp_inclusive_scan(hi, tid);
      const float tot = __shfl_sync(0xffffffffu, shi, 31);
      const float slo = warp_inclusive_scan(vec[2 * C + 31 - tid], tid) + tot;
      vec[6 * C + 63 - tid] = shi;
      vec[6 * C + 31 - tid] = slo;
    }
    if (tid < NS) {  // key-bias partials over this chunk's tokens (column tid)
      float sk = 0.f;
      for (int tt = 0; tt < C && t0 + tt < d.T; ++tt) sk += G[tt * LN + tid];
      kbs += sk;
    }
    // New carry: d_start = Q^T rd(dY e^p) + e^(p_L) carry (every read of the
    // old carry in this chunk is done: dV, dK and the dot product above).
    {
      float acc[2][8][4];
#pragma unroll
      for (int k = 0; k < 2; ++k) zero8(acc[k]);
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        const int n0 = row0 + 64 * k;
        if (n0 < NS)
          warp_gemm<BF, C>(acc[k], n0, [&](int n, int t) { return Qs[t * LN + n]; },
                           [&](int t, int p) { return round_to<T>(Dy[t * LDS + p] * expf(r.p[t])); });
      }
      __syncthreads();  // G's bias sums are done too: G is rewritten below
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        const int n0 = row0 + 64 * k;
        if (n0 < NS) for_tile(acc[k], n0, [&](int n, int p, float v) { Cy[n * HP + p] = fmaf(end, Cy[n * HP + p], v); });
      }
    }
    // dQ = rd(Dm o W) K + rd(dY e^p) rd(start)^T -> G (64 state columns per pass).
    for (int nb = 0; nb < NS; nb += 64) {
      float acc[8][4];
      zero8(acc);
      warp_gemm<BF, C>(acc, row0, [&](int t, int s) { return round_to<T>(Dm[t * LDS + s] * wgt(t, s)); },
                       [&](int s, int n) { return nb + n < NS ? Ks[s * LN + nb + n] : 0.f; });
      warp_gemm<BF, HP>(acc, row0, [&](int t, int p) { return round_to<T>(Dy[t * LDS + p] * expf(r.p[t])); },
                        [&](int p, int n) { return nb + n < NS ? round_to<T>(St[(nb + n) * HP + p]) : 0.f; });
      for_tile(acc, row0, [&](int t, int n, float v) { if (nb + n < NS) G[t * LN + nb + n] = v; });
    }
    __syncthreads();
    rotate_back<T, NS, true>(d, b, h, t0, cq, bk, qb, kb, theta, G, dth, o.dq);
    __syncthreads();
    if (tid < NS) {  // query-bias partials
      float sq = 0.f;
      for (int tt = 0; tt < C && t0 + tt < d.T; ++tt) sq += G[tt * LN + tid];
      qbs += sq;
    }
    // Suffix sums of the pair-phase gradient -> rate and dt gradients.
    if (tid < d.A) {
      const int i = tid;
      float acc = later[i];
      for (int tt = C - 1; tt >= 0; --tt) {
        acc += dth[tt * TW + i];
        dth[tt * TW + i] = acc;  // d_increment (pair) at tt
      }
      later[i] = acc;
    }
    __syncthreads();
    if (tid < C) {
      const int tt = tid, t = t0 + tt;
      if (t < d.T) {
        float ddt = 0.f;
        for (int i = 0; i < d.A; ++i) {
          const float rate = d.per_head ? angles[((size_t(b) * d.T + t) * d.H + h) * d.A + i]
                                        : angles[(size_t(b) * d.T + t) * d.A + i];
          const float inc = dth[tt * TW + i];
          o.drate[((size_t(b) * d.T + t) * d.H + h) * d.A + i] = inc * r.dt[tt];
          ddt = fmaf(inc, rate, ddt);
        }
        const size_t si = (size_t(b) * d.T + t) * d.H + h;
        o.ddtp[si] = ddt;
        o.dgam[si] = vec[3 * C + tt];
        o.dscl[si] = vec[4 * C + tt];
        o.dlog[si] = vec[6 * C + tt];
      }
    }
    __syncthreads();
  }
  if (tid < NS) {
    o.dqb[size_t(bh) * NS + tid] = qbs;
    o.dkb[size_t(bh) * NS + tid] = kbs;
  }
}

// dc/db: sum the per-head pre-rotation gradients over heads (fixed order),
// or copy them for per-head layouts; cast to the model dtype.
template <typename T, int NS>
__global__ void reduce_heads_kernel(Dims d, const float* __restrict__ dq, const float* __restrict__ dk,
                                    T* __restrict__ dc, T* __restrict__ db) {
  const size_t idx = size_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (d.per_head) {
    const size_t total = size_t(d.B) * d.T * d.H * NS;
    if (idx >= total) return;
    dc[idx] = from_f<T>(dq[idx]);
    db[idx] = from_f<T>(dk[idx]);
    return;
  }
  const size_t total = size_t(d.B) * d.T * NS;
  if (idx >= total) return;
  const size_t bt = idx / NS, n = idx % NS;
  float sq = 0.f, sk = 0.f;
  for (int h = 0; h < d.H; ++h) {
    sq += dq[(bt * d.H + h) * NS + n];
    sk += dk[(bt * d.H + h) * NS + n];
  }
  dc[idx] = from_f<T>(sq);
  db[idx] = from_f<T>(sk);
}

// Gate chain rule (mamba3_fused preprocessing, flashmamba.py:1142-1147):
// gamma = dt s, prev = dt (1 - s), scale_t = gamma_t + prev_(t+1), s = sigmoid(trap).
__global__ void gates_kernel(Dims d, const float* __restrict__ dt, const float* __restrict__ trap_logits,
                             const float* __restrict__ dgam, const float* __restrict__ dscl,
                             const float* __restrict__ dlog, const float* __restrict__ ddtp,
                             const float* __restrict__ drate, float* __restrict__ d_adt,
                             float* __restrict__ d_dt, float* __restrict__ d_trap,
                             float* __restrict__ d_angles) {
  const size_t idx = size_t(blockIdx.x) * blockDim.x + threadIdx.x;
  const size_t total = size_t(d.B) * d.T * d.H;
  if (idx < total) {
    const size_t bt = idx / d.H;
    const int t = int(bt % d.T);
    const float s = 1.f / (1.f + expf(-trap_logits[idx]));
    const float g = dgam[idx] + dscl[idx];
    const float pv = t > 0 ? dscl[idx - d.H] : 0.f;
    d_dt[idx] = fmaf(g, s, pv * (1.f - s)) + ddtp[idx];
    d_trap[idx] = (g - pv) * dt[idx] * s * (1.f - s);
    d_adt[idx] = dlog[idx];
  }
  // Angle-rate gradients: per head, or summed over heads for shared angles.
  if (d.per_head) {
    const size_t ta = size_t(d.B) * d.T * d.H * d.A;
    if (idx < ta) d_angles[idx] = drate[idx];
  } else {
    const size_t ta = size_t(d.B) * d.T * d.A;
    if (idx < ta) {
      const size_t bt = idx / d.A, i = idx % d.A;
      float acc = 0.f;
      for (int h = 0; h < d.H; ++h) acc += drate[(bt * d.H + h) * d.A + i];
      d_angles[idx] = acc;
    }
  }
}

template <int NS>
__global__ void bias_kernel(Dims d, const float* __restrict__ dqb, const float* __restrict__ dkb,
                            float* __restrict__ d_qb, float* __restrict__ d_kb) {
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= d.H * NS) return;
  float sq = 0.f, sk = 0.f;
  for (int b = 0; b < d.B; ++b) {
    sq += dqb[size_t(b) * d.H * NS + idx];
    sk += dkb[size_t(b) * d.H * NS + idx];
  }
  if (d_qb) d_qb[idx] = sq;
  if (d_kb) d_kb[idx] = sk;
}

// bf16 operands at state dim 64 or 128 run the chunk-parallel tensor-core
// kernels of scan_bf16.cuh; every other case the sequential kernels above.
inline bool fast_path(const M4ScanDims& s) { return s.bf16 && (s.state_dim == 64 || s.state_dim == 128); }

struct Layout {
  size_t starts, phases, deltas, resid;
  size_t dq, dk, drate, dgam, dscl, dlog, ddtp, dqb, dkb, carries, dth, carry, work;
};

inline Layout layout(const M4ScanDims& s) {
  Layout l;
  const int nch = (s.time + C - 1) / C;
  const size_t ns = size_t(s.state_dim), np = ns / 2;
  const size_t bh = size_t(s.batch) * s.heads, bth = size_t(s.batch) * s.time * s.heads;
  const bool fast = fast_path(s);
  size_t off = 0;
  l.starts = off; off += align256(bh * nch * ns * HP * sizeof(float));
  l.phases = off; off += align256(bh * nch * np * sizeof(float));
  l.deltas = off; off += align256(bh * nch * sizeof(float));
  l.resid = off;
  off = 0;
  l.dq = off; off += align256(bth * ns * sizeof(float));
  l.dk = off; off += align256(bth * ns * sizeof(float));
  l.drate = off; off += align256(bth * np * sizeof(float));
  l.dgam = off; off += align256(bth * sizeof(float));
  l.dscl = off; off += align256(bth * sizeof(float));
  l.dlog = off; off += align256(bth * sizeof(float));
  l.ddtp = off; off += align256(bth * sizeof(float));
  l.dqb = off; off += align256(bh * nch * ns * sizeof(float));
  l.dkb = off; off += align256(bh * nch * ns * sizeof(float));
  l.carries = fast ? off : 0; off += fast ? align256(bh * nch * ns * HP * sizeof(float)) : 0;
  l.dth = off; off += align256(bh * nch * np * sizeof(float));
  l.carry = fast ? 0 : off; off += fast ? 0 : align256(bh * ns * HP * sizeof(float));
  l.work = off;
  return l;
}

inline Dims make_dims(const M4ScanDims& s) {
  Dims d;
  d.B = s.batch; d.T = s.time; d.H = s.heads; d.A = s.angle_count;
  d.nch = (s.time + C - 1) / C;
  d.per_head = s.per_head != 0;
  return d;
}

inline bool state_dim_supported(int n) { return n == 64 || n == 96 || n == 128; }

inline int check(const M4ScanDims* s) {
  if (!s) return M4_ERR_NULL;
  if (s->batch <= 0 || s->time <= 0 || s->heads <= 0 || s->head_dim <= 0 || s->state_dim <= 0 ||
      s->angle_count < 0 || s->chunk <= 0)
    return M4_ERR_DIMS;
  if (s->head_dim != HP || !state_dim_supported(s->state_dim) || s->chunk != C ||
      s->angle_count > s->state_dim / 2)
    return M4_ERR_UNSUPPORTED;
  return M4_OK;
}

inline int forward_bf16(const M4ScanDims& s, const void* c, const void* b, const void* x, const float* adt,
                        const float* dt, const float* trap, const float* angles, const float* qb,
                        const float* kb, void* y, float* fin, char* resid, cudaStream_t st);
inline int backward_bf16(const M4ScanDims& s, const void* c, const void* b, const void* x, const float* adt,
                         const float* dt, const float* trap, const float* angles, const float* qb,
                         const float* kb, const char* resid, const void* dy, const float* d_final, void* dc,
                         void* db, void* dx, float* d_adt, float* d_dt, float* d_trap, float* d_angles,
                         float* d_qb, float* d_kb, char* work, cudaStream_t st);

template <typename T, int NS>
int forward_seq(const M4ScanDims& s, const void* c, const void* b, const void* x, const float* adt,
                const float* dt, const float* trap, const float* angles, const float* qb, const float* kb,
                void* y, float* fin, char* resid, cudaStream_t st) {
  const Dims d = make_dims(s);
  const Layout l = layout(s);
  const size_t sm = fwd_smem<NS>();
  cudaFuncSetAttribute(fwd_kernel<T, NS>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(sm));
  fwd_kernel<T, NS><<<s.batch * s.heads, THREADS, sm, st>>>(
      d, static_cast<const T*>(c), static_cast<const T*>(b), static_cast<const T*>(x), adt, dt, trap,
      angles, qb, kb, static_cast<T*>(y), fin, reinterpret_cast<float*>(resid + l.starts),
      reinterpret_cast<float*>(resid + l.phases));
  return launch_status();
}

template <typename T, int NS>
int backward_seq(const M4ScanDims& s, const void* c, const void* b, const void* x, const float* adt,
                 const float* dt, const float* trap, const float* angles, const float* qb, const float* kb,
                 const char* resid, const void* dy, const float* d_final, void* dc, void* db, void* dx,
                 float* d_adt, float* d_dt, float* d_trap, float* d_angles, float* d_qb, float* d_kb,
                 char* work, cudaStream_t st) {
  const Dims d = make_dims(s);
  const Layout l = layout(s);
  BwdOut o;
  o.dq = reinterpret_cast<float*>(work + l.dq);
  o.dk = reinterpret_cast<float*>(work + l.dk);
  o.drate = reinterpret_cast<float*>(work + l.drate);
  o.dgam = reinterpret_cast<float*>(work + l.dgam);
  o.dscl = reinterpret_cast<float*>(work + l.dscl);
  o.dlog = reinterpret_cast<float*>(work + l.dlog);
  o.ddtp = reinterpret_cast<float*>(work + l.ddtp);
  o.dqb = reinterpret_cast<float*>(work + l.dqb);
  o.dkb = reinterpret_cast<float*>(work + l.dkb);
  o.carry = reinterpret_cast<float*>(work + l.carry);
  const size_t sm = bwd_smem<NS>();
  cudaFuncSetAttribute(bwd_kernel<T, NS>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(sm));
  bwd_kernel<T, NS><<<s.batch * s.heads, THREADS, sm, st>>>(
      d, static_cast<const T*>(c), static_cast<const T*>(b), static_cast<const T*>(x), adt, dt, trap,
      angles, qb, kb, reinterpret_cast<const float*>(resid + l.starts),
      reinterpret_cast<const float*>(resid + l.phases), static_cast<const T*>(dy), d_final,
      static_cast<T*>(dx), o);
  const size_t n1 = s.per_head ? size_t(s.batch) * s.time * s.heads * NS : size_t(s.batch) * s.time * NS;
  reduce_heads_kernel<T, NS><<<unsigned((n1 + 255) / 256), 256, 0, st>>>(d, o.dq, o.dk, static_cast<T*>(dc),
                                                                          static_cast<T*>(db));
  size_t n2 = size_t(s.batch) * s.time * s.heads;
  const size_t na = s.per_head ? n2 * s.angle_count : size_t(s.batch) * s.time * s.angle_count;
  if (na > n2) n2 = na;
  gates_kernel<<<unsigned((n2 + 255) / 256), 256, 0, st>>>(d, dt, trap, o.dgam, o.dscl, o.dlog, o.ddtp,
                                                            o.drate, d_adt, d_dt, d_trap, d_angles);
  if (d_qb || d_kb)
    bias_kernel<NS><<<(s.heads * NS + 255) / 256, 256, 0, st>>>(d, o.dqb, o.dkb, d_qb, d_kb);
  return launch_status();
}

template <typename T>
int forward(const M4ScanDims& s, const void* c, const void* b, const void* x, const float* adt,
            const float* dt, const float* trap, const float* angles, const float* qb, const float* kb,
            void* y, float* fin, char* resid, cudaStream_t st) {
  if (fast_path(s)) return forward_bf16(s, c, b, x, adt, dt, trap, angles, qb, kb, y, fin, resid, st);
  switch (s.state_dim) {
    case 64: return forward_seq<T, 64>(s, c, b, x, adt, dt, trap, angles, qb, kb, y, fin, resid, st);
    case 96: return forward_seq<T, 96>(s, c, b, x, adt, dt, trap, angles, qb, kb, y, fin, resid, st);
    default: return forward_seq<T, 128>(s, c, b, x, adt, dt, trap, angles, qb, kb, y, fin, resid, st);
  }
}

template <typename T>
int backward(const M4ScanDims& s, const void* c, const void* b, const void* x, const float* adt,
             const float* dt, const float* trap, const float* angles, const float* qb, const float* kb,
             const char* resid, const void* dy, const float* d_final, void* dc, void* db, void* dx,
             float* d_adt, float* d_dt, float* d_trap, float* d_angles, float* d_qb, float* d_kb,
             char* work, cudaStream_t st) {
  if (fast_path(s))
    return backward_bf16(s, c, b, x, adt, dt, trap, angles, qb, kb, resid, dy, d_final, dc, db, dx, d_adt,
                         d_dt, d_trap, d_angles, d_qb, d_kb, work, st);
#define M4_SEQ_BWD(NSV)                                                                                     \
  return backward_seq<T, NSV>(s, c, b, x, adt, dt, trap, angles, qb, kb, resid, dy, d_final, dc, db, dx, \
                              d_adt, d_dt, d_trap, d_angles, d_qb, d_kb, work, st)
  switch (s.state_dim) {
    case 64: M4_SEQ_BWD(64);
    case 96: M4_SEQ_BWD(96);
    default: M4_SEQ_BWD(128);
  }
#undef M4_SEQ_BWD
}

}  // namespace scan
}  // namespace m4

#include "scan_bf16.cuh"

namespace m4 {
namespace scan {

// TMA descriptor of a [B][T][H*64] bf16 tensor: box of 64 channels x 64
// tokens x 1 batch, 128-byte swizzle (the tcgen05 tile layout); tokens past T
// read as zeros. The driver entry point is looked up once.
inline bool encode_tokens_map(CUtensorMap* map, const void* base, int B, int T, int HP) {
  static PFN_cuTensorMapEncodeTiled_v12000 encode = [] {
    PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", reinterpret_cast<void**>(&fn), cudaEnableDefault, &q) !=
            cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      fn = nullptr;
    return fn;
  }();
  if (!encode) return false;
  const cuuint64_t dim[3] = {cuuint64_t(HP), cuuint64_t(T), cuuint64_t(B)};
  const cuuint64_t stride[2] = {cuuint64_t(HP) * 2, cuuint64_t(T) * HP * 2};
  const cuuint32_t box[3] = {64, 64, 1}, elem[3] = {1, 1, 1};
  return encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dim, stride, box, elem,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// bfloat16 operands at state dim 64 or 128 run the chunk-parallel kernels of
// scan_bf16.cuh (templated on the number of 64-row state halves).
inline scan2::Dims make_dims2(const M4ScanDims& s) {
  scan2::Dims d;
  d.B = s.batch; d.T = s.time; d.H = s.heads; d.A = s.angle_count;
  d.nch = (s.time + C - 1) / C;
  d.per_head = s.per_head != 0;
  return d;
}

template <class K>
inline void allow_smem(K kernel, size_t bytes) {
  if (bytes > 48 * 1024) cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(bytes));
}

template <int NH>
inline int forward_bf16_nh(const M4ScanDims& s, const void* c, const void* b, const void* x, const float* adt,
                           const float* dt, const float* trap, const float* angles, const float* qb,
                           const float* kb, void* y, float* fin, char* resid, cudaStream_t st) {
  using namespace scan2;
  const scan2::Dims d = make_dims2(s);
  const Layout l = layout(s);
  float* starts = reinterpret_cast<float*>(resid + l.starts);
  float* phases = reinterpret_cast<float*>(resid + l.phases);
  float* deltas = reinterpret_cast<float*>(resid + l.deltas);
  const bf16* cq = static_cast<const bf16*>(c);
  const bf16* bk = static_cast<const bf16*>(b);
  alignas(64) CUtensorMap xmap;
  if (!all_aligned16(c, b, x)) return M4_ERR_ALIGN;  // 16-byte row copies and the TMA box
  if (!encode_tokens_map(&xmap, x, d.B, d.T, d.H * P)) return M4_ERR_LAUNCH;
  const size_t fsm = fused_smem_bytes<NH>(d.A) + 1024;
  allow_smem(fused_fwd_kernel<NH>, fsm);
  fused_fwd_kernel<NH><<<d.B * d.H, GW * 32, fsm, st>>>(
      d, xmap, cq, bk, adt, dt, trap, angles, qb, kb, static_cast<bf16*>(y), starts, phases, deltas, fin);
  return launch_status();
}

inline int forward_bf16(const M4ScanDims& s, const void* c, const void* b, const void* x, const float* adt,
                        const float* dt, const float* trap, const float* angles, const float* qb,
                        const float* kb, void* y, float* fin, char* resid, cudaStream_t st) {
  if (s.state_dim == 128) return forward_bf16_nh<2>(s, c, b, x, adt, dt, trap, angles, qb, kb, y, fin, resid, st);
  return forward_bf16_nh<1>(s, c, b, x, adt, dt, trap, angles, qb, kb, y, fin, resid, st);
}

template <int NH>
inline int backward_bf16_nh(const M4ScanDims& s, const void* c, const void* b, const void* x, const float* adt,
                            const float* dt, const float* trap, const float* angles, const float* qb,
                            const float* kb, const char* resid, const void* dy, const float* d_final, void* dc,
                            void* db, void* dx, float* d_adt, float* d_dt, float* d_trap, float* d_angles,
                            float* d_qb, float* d_kb, char* work, cudaStream_t st) {
  using namespace scan2;
  if (!all_aligned16(c, b, x, dy)) return M4_ERR_ALIGN;  // 16-byte tile copies
  const scan2::Dims d = make_dims2(s);
  const Layout l = layout(s);
  const float* starts = reinterpret_cast<const float*>(resid + l.starts);
  const float* phases = reinterpret_cast<const float*>(resid + l.phases);
  const float* deltas = reinterpret_cast<const float*>(resid + l.deltas);
  float* carries = reinterpret_cast<float*>(work + l.carries);
  GradOut o;
  o.dq = reinterpret_cast<float*>(work + l.dq);
  o.dk = reinterpret_cast<float*>(work + l.dk);
  o.drate = reinterpret_cast<float*>(work + l.drate);
  o.dgam = reinterpret_cast<float*>(work + l.dgam);
  o.dscl = reinterpret_cast<float*>(work + l.dscl);
  o.dlog = reinterpret_cast<float*>(work + l.dlog);
  o.ddtp = reinterpret_cast<float*>(work + l.ddtp);
  o.dth = reinterpret_cast<float*>(work + l.dth);
  o.dqb = reinterpret_cast<float*>(work + l.dqb);
  o.dkb = reinterpret_cast<float*>(work + l.dkb);
  const bf16* cq = static_cast<const bf16*>(c);
  const bf16* bk = static_cast<const bf16*>(b);
  const bf16* xx = static_cast<const bf16*>(x);
  const bf16* g = static_cast<const bf16*>(dy);
  const int bh = d.B * d.H, chunks = bh * d.nch;
  const size_t dsm = dstart_smem_bytes<NH>(d.A) + 1024;
  allow_smem(dstart_kernel<NH>, dsm);
  dstart_kernel<NH><<<chunks, GW * 32, dsm, st>>>(d, cq, g, adt, dt, trap, angles, qb, phases, carries);
  carry_kernel<NH><<<bh * sparts<NH>(), 256, 0, st>>>(d, carries, deltas, d_final);
  allow_smem(grads_kernel<NH>, sizeof(GradSmem<NH>) + 1024);
  grads_kernel<NH><<<chunks, GW * 32, sizeof(GradSmem<NH>) + 1024, st>>>(d, cq, bk, xx, adt, dt, trap, angles, qb, kb,
                                                                  phases, starts, carries, g,
                                                                  static_cast<bf16*>(dx), o);
  later_kernel<NH><<<bh, Geo<NH>::NP, 0, st>>>(d, o.dth);
  const size_t tokens = size_t(d.B) * d.T;
  finish_kernel<NH><<<unsigned((tokens + 7) / 8), 256, 0, st>>>(d, dt, trap, angles, o.dth, o,
                                                                static_cast<bf16*>(dc), static_cast<bf16*>(db),
                                                                d_adt, d_dt, d_trap, d_angles);
  if (d_qb || d_kb) scan2::bias_kernel<NH><<<s.heads, 1024, 0, st>>>(d, o.dqb, o.dkb, d_qb, d_kb);
  return launch_status();
}

inline int backward_bf16(const M4ScanDims& s, const void* c, const void* b, const void* x, const float* adt,
                         const float* dt, const float* trap, const float* angles, const float* qb,
                         const float* kb, const char* resid, const void* dy, const float* d_final, void* dc,
                         void* db, void* dx, float* d_adt, float* d_dt, float* d_trap, float* d_angles,
                         float* d_qb, float* d_kb, char* work, cudaStream_t st) {
  if (s.state_dim == 128)
    return backward_bf16_nh<2>(s, c, b, x, adt, dt, trap, angles, qb, kb, resid, dy, d_final, dc, db, dx, d_adt,
                               d_dt, d_trap, d_angles, d_qb, d_kb, work, st);
  return backward_bf16_nh<1>(s, c, b, x, adt, dt, trap, angles, qb, kb, resid, dy, d_final, dc, db, dx, d_adt,
                             d_dt, d_trap, d_angles, d_qb, d_kb, work, st);
}

}  // namespace scan
}  // namespace m4

using namespace m4;

extern "C" int m4_device_status(void) {
  int flag = 0;
  if (cudaMemcpyFromSymbol(&flag, m4::tc::g_timeout, sizeof(int)) != cudaSuccess) return M4_ERR_LAUNCH;
  if (flag) {
    const int zero = 0;
    cudaMemcpyToSymbol(m4::tc::g_timeout, &zero, sizeof(int));
    return M4_ERR_TIMEOUT;
  }
  return M4_OK;
}

extern "C" size_t m4_scan_residual_bytes(const M4ScanDims* s) {
  return scan::check(s) == M4_OK ? scan::layout(*s).resid : 0;
}

extern "C" size_t m4_scan_workspace_bytes(const M4ScanDims* s) {
  return scan::check(s) == M4_OK ? scan::layout(*s).work : 0;
}

extern "C" int m4_scan_fwd(const M4ScanDims* s, const void* c, const void* b, const void* x,
                           const float* adt, const float* dt, const float* trap, const float* angles,
                           const float* qb, const float* kb, void* y, float* fin, void* resid,
                           size_t resid_bytes, void* stream) {
  int st = scan::check(s);
  if (st) return st;
  if (!c || !b || !x || !adt || !dt || !trap || !y || !fin || !resid) return M4_ERR_NULL;
  if (s->angle_count > 0 && !angles) return M4_ERR_NULL;
  if (resid_bytes < scan::layout(*s).resid) return M4_ERR_WORKSPACE;
  cudaStream_t strm = static_cast<cudaStream_t>(stream);
  if (s->bf16)
    return scan::forward<__nv_bfloat16>(*s, c, b, x, adt, dt, trap, angles, qb, kb, y, fin,
                                        static_cast<char*>(resid), strm);
  return scan::forward<float>(*s, c, b, x, adt, dt, trap, angles, qb, kb, y, fin,
                              static_cast<char*>(resid), strm);
}

extern "C" int m4_scan_bwd(const M4ScanDims* s, const void* c, const void* b, const void* x,
                           const float* adt, const float* dt, const float* trap, const float* angles,
                           const float* qb, const float* kb, const void* resid, size_t resid_bytes,
                           const void* dy, const float* d_final, void* dc, void* db, void* dx,
                           float* d_adt, float* d_dt, float* d_trap, float* d_angles, float* d_qb,
                           float* d_kb, void* work, size_t work_bytes, void* stream) {
  int st = scan::check(s);
  if (st) return st;
  if (!c || !b || !x || !adt || !dt || !trap || !resid || !dy || !dc || !db || !dx || !d_adt ||
      !d_dt || !d_trap || !work)
    return M4_ERR_NULL;
  if (s->angle_count > 0 && (!angles || !d_angles)) return M4_ERR_NULL;
  const scan::Layout l = scan::layout(*s);
  if (resid_bytes < l.resid || work_bytes < l.work) return M4_ERR_WORKSPACE;
  cudaStream_t strm = static_cast<cudaStream_t>(stream);
  if (s->bf16)
    return scan::backward<__nv_bfloat16>(*s, c, b, x, adt, dt, trap, angles, qb, kb,
                                         static_cast<const char*>(resid), dy, d_final, dc, db, dx, d_adt,
                                         d_dt, d_trap, d_angles, d_qb, d_kb, static_cast<char*>(work), strm);
  return scan::backward<float>(*s, c, b, x, adt, dt, trap, angles, qb, kb, static_cast<const char*>(resid),
                               dy, d_final, dc, db, dx, d_adt, d_dt, d_trap, d_angles, d_qb, d_kb,
                               static_cast<char*>(work), strm);
}

// ---------------------------------------------------------------------------
// One-token scan step against a carried cache: the scan core of the
// reference's _Mamba3StepMixer (lm/models/mamba4.py:412-481).
//   phase' = phase + rate dt; Q, K = rotate(round(c + q_bias), phase'),
//   rotate(round(b + k_bias), phase') rounded to the model dtype;
//   S' = e^(adt) (S + dt (1 - trap) k_prev v_prev^T) + dt trap K x^T;
//   y = Q^T S' (model dtype); cache' = (S', K, x, phase').
// One CTA of 4 N threads per (batch, head) (state dim N in {64, 96, 128});
// thread (n, p0) = (tid / 4, 16 (tid % 4)) updates S'[n][p0 .. p0+15]. Outputs may alias the cache
// inputs: every cache value is read before any is written.
// ---------------------------------------------------------------------------
namespace m4 {
namespace scan {

template <typename T, int NS>
__global__ void __launch_bounds__(4 * NS) step_kernel(
    int H, int A, int per_head, const float* state, const float* prev_k, const float* prev_v,
    const float* phase, const T* __restrict__ c, const T* __restrict__ bk, const T* __restrict__ x,
    const float* __restrict__ adt, const float* __restrict__ dt, const float* __restrict__ trap_logits,
    const float* __restrict__ angles, const float* __restrict__ qb, const float* __restrict__ kb,
    T* __restrict__ y, float* state_out, float* prev_k_out, float* prev_v_out, float* phase_out) {
  const int bh = blockIdx.x, bb = bh / H, h = bh % H, tid = threadIdx.x;
  __shared__ float qr[NS], kr[NS], xv[HP], pk[NS], pv[HP], ph[NS / 2];
  __shared__ float red[NS / 8][HP];
  const float dtv = dt[bh];
  const float trap = 1.f / (1.f + expf(-trap_logits[bh]));
  const float alpha = expf(adt[bh]);
  const int n = tid >> 2, p0 = (tid & 3) * 16;
  float sv[16];
  {
    const float* srow = state + (size_t(bh) * NS + n) * HP + p0;
#pragma unroll
    for (int e = 0; e < 16; e += 4) {
      const float4 v = ld4(srow + e);
      sv[e] = v.x; sv[e + 1] = v.y; sv[e + 2] = v.z; sv[e + 3] = v.w;
    }
  }
  // Inputs that no output aliases, loaded at entry with the state: the
  // token's C/B pair (plus biases) and x, so one DRAM round trip precedes the
  // rotations instead of two.
  float cq[2] = {0.f, 0.f}, ck[2] = {0.f, 0.f}, xr = 0.f;
  if (tid < NS / 2) {
    const int n0 = 2 * tid, n1 = 2 * tid + 1;
    const size_t base = per_head ? size_t(bh) * NS : size_t(bb) * NS;
    cq[0] = to_f(c[base + n0]) + (qb ? qb[h * NS + n0] : 0.f);
    cq[1] = to_f(c[base + n1]) + (qb ? qb[h * NS + n1] : 0.f);
    ck[0] = to_f(bk[base + n0]) + (kb ? kb[h * NS + n0] : 0.f);
    ck[1] = to_f(bk[base + n1]) + (kb ? kb[h * NS + n1] : 0.f);
  }
  if (tid < HP) xr = to_f(x[size_t(bh) * HP + tid]);
  float phv = 0.f;
  if (tid < NS / 2) {
    if (tid < A) {
      const float rate = angles[per_head ? size_t(bh) * A + tid : size_t(bb) * A + tid];
      phv = phase[size_t(bh) * A + tid] + rate * dtv;
    }
    ph[tid] = phv;
  }
  if (tid < NS) pk[tid] = prev_k[size_t(bh) * NS + tid];
  if (tid < HP) pv[tid] = prev_v[size_t(bh) * HP + tid];
  __syncthreads();  // every cache value is read: outputs may now overwrite them
  if (tid < NS / 2 && tid < A) phase_out[size_t(bh) * A + tid] = phv;
  if (tid < NS / 2) {
    const int i = tid, n0 = 2 * i, n1 = 2 * i + 1;
    const float q0 = round_to<T>(cq[0]), q1 = round_to<T>(cq[1]);
    const float k0 = round_to<T>(ck[0]), k1 = round_to<T>(ck[1]);
    float cs = 1.f, sn = 0.f;
    if (i < A) sincosf(ph[i], &sn, &cs);
    qr[n0] = round_to<T>(q0 * cs - q1 * sn);
    qr[n1] = round_to<T>(q1 * cs + q0 * sn);
    kr[n0] = round_to<T>(k0 * cs - k1 * sn);
    kr[n1] = round_to<T>(k1 * cs + k0 * sn);
  }
  if (tid < HP) xv[tid] = xr;
  __syncthreads();
  if (tid < NS) prev_k_out[size_t(bh) * NS + tid] = kr[tid];
  if (tid < HP) prev_v_out[size_t(bh) * HP + tid] = xv[tid];
  const float wp = dtv * (1.f - trap) * pk[n], wc = dtv * trap * kr[n], q = qr[n];
  float part[16];
#pragma unroll
  for (int e = 0; e < 16; ++e) {
    sv[e] = fmaf(wc, xv[p0 + e], alpha * fmaf(wp, pv[p0 + e], sv[e]));
    part[e] = q * sv[e];
  }
  {
    float* dst = state_out + (size_t(bh) * NS + n) * HP + p0;
#pragma unroll
    for (int e = 0; e < 16; e += 4) st4(dst + e, make_float4(sv[e], sv[e + 1], sv[e + 2], sv[e + 3]));
  }
  // y[p] = sum_n Q[n] S'[n][p]: over the warp's eight n (lanes 4 apart), then
  // over the eight warps in a fixed order.
#pragma unroll
  for (int e = 0; e < 16; ++e) {
    float v = part[e];
    v += __shfl_xor_sync(0xffffffffu, v, 4);
    v += __shfl_xor_sync(0xffffffffu, v, 8);
    v += __shfl_xor_sync(0xffffffffu, v, 16);
    part[e] = v;
  }
  const int warp = tid >> 5, lane = tid & 31;
  if (lane < 4) {
#pragma unroll
    for (int e = 0; e < 16; ++e) red[warp][p0 + e] = part[e];
  }
  __syncthreads();
  if (tid < HP) {
    float acc = 0.f;
#pragma unroll
    for (int w = 0; w < NS / 8; ++w) acc += red[w][tid];
    y[size_t(bh) * HP + tid] = from_f<T>(acc);
  }
}

}  // namespace scan
}  // namespace m4

extern "C" int m4_scan_step(const M4ScanDims* s, const float* state, const float* prev_keys,
                            const float* prev_values, const float* phase, const void* c, const void* b,
                            const void* x, const float* adt, const float* dt, const float* trap,
                            const float* angles, const float* qb, const float* kb, void* y,
                            float* state_out, float* prev_keys_out, float* prev_values_out,
                            float* phase_out, void* stream) {
  if (!s) return M4_ERR_NULL;
  if (s->batch <= 0 || s->heads <= 0 || s->head_dim <= 0 || s->state_dim <= 0 || s->angle_count < 0)
    return M4_ERR_DIMS;
  if (s->head_dim != scan::HP || !scan::state_dim_supported(s->state_dim) || s->angle_count > s->state_dim / 2)
    return M4_ERR_UNSUPPORTED;
  if (!state || !prev_keys || !prev_values || !c || !b || !x || !adt || !dt || !trap || !y || !state_out ||
      !prev_keys_out || !prev_values_out)
    return M4_ERR_NULL;
  if (s->angle_count > 0 && (!angles || !phase || !phase_out)) return M4_ERR_NULL;
  if (!all_aligned16(state, state_out)) return M4_ERR_ALIGN;
  cudaStream_t strm = static_cast<cudaStream_t>(stream);
  const int grid = s->batch * s->heads;
#define M4_STEP(T, NSV)                                                                                         \
  scan::step_kernel<T, NSV><<<grid, 4 * NSV, 0, strm>>>(                                                       \
      s->heads, s->angle_count, s->per_head, state, prev_keys, prev_values, phase, static_cast<const T*>(c),  \
      static_cast<const T*>(b), static_cast<const T*>(x), adt, dt, trap, angles, qb, kb, static_cast<T*>(y),  \
      state_out, prev_keys_out, prev_values_out, phase_out)
  if (s->bf16) {
    if (s->state_dim == 64) M4_STEP(__nv_bfloat16, 64);
    else if (s->state_dim == 96) M4_STEP(__nv_bfloat16, 96);
    else M4_STEP(__nv_bfloat16, 128);
  } else {
    if (s->state_dim == 64) M4_STEP(float, 64);
    else if (s->state_dim == 96) M4_STEP(float, 96);
    else M4_STEP(float, 128);
  }
#undef M4_STEP
  return launch_status();
}

// ---------------------------------------------------------------------------
// Backward scan for callers that cannot allocate device memory.
//
// Some callers may not allocate at all while they run this operator: an XLA
// FFI custom call or other framework plugin that must not touch the device
// allocator, code recorded into a CUDA graph, or an inference server that
// reserves all device memory up front. This entry point takes its scratch
// from a fixed array compiled into the library instead of a caller buffer.
// ---------------------------------------------------------------------------
#include <atomic>

namespace {

// Fixed scratch: 32 MiB, held on every GPU that loads the library until the
// process exits. Enough for batch x time x heads up to about 36,000
// (e.g. 2 sequences x 1,024 tokens x 16 heads).
constexpr size_t kNoAllocScratchBytes = size_t(32) << 20;
__device__ __align__(256) unsigned char g_scan_bwd_scratch[kNoAllocScratchBytes];

// Device address of the array per device, looked up once per device.
constexpr int kMaxDevices = 64;
std::atomic<void*> g_scan_bwd_scratch_ptr[kMaxDevices];

}  // namespace

extern "C" int m4_scan_bwd_noalloc(const M4ScanDims* s, const void* c, const void* b, const void* x,
                                   const float* adt, const float* dt, const float* trap,
                                   const float* angles, const float* qb, const float* kb,
                                   const void* resid, size_t resid_bytes, const void* dy,
                                   const float* d_final, void* dc, void* db, void* dx, float* d_adt,
                                   float* d_dt, float* d_trap, float* d_angles, float* d_qb,
                                   float* d_kb, void* stream) {
  int st = scan::check(s);
  if (st) return st;
  if (!c || !b || !x || !adt || !dt || !trap || !resid || !dy || !dc || !db || !dx || !d_adt ||
      !d_dt || !d_trap)
    return M4_ERR_NULL;
  if (s->angle_count > 0 && (!angles || !d_angles)) return M4_ERR_NULL;
  const scan::Layout l = scan::layout(*s);
  if (resid_bytes < l.resid) return M4_ERR_WORKSPACE;
  // Reject problems whose scratch does not fit the fixed array; nothing is launched.
  if (l.work > kNoAllocScratchBytes) return M4_ERR_WORKSPACE;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return M4_ERR_LAUNCH;
  void* scratch = g_scan_bwd_scratch_ptr[dev].load(std::memory_order_acquire);
  if (scratch == nullptr) {
    // Host code only sees a stand-in for the __device__ array; its device
    // address comes from the runtime, once per device, with that device current.
    if (cudaGetSymbolAddress(&scratch, g_scan_bwd_scratch) != cudaSuccess || scratch == nullptr)
      return M4_ERR_LAUNCH;
    g_scan_bwd_scratch_ptr[dev].store(scratch, std::memory_order_release);
  }
  // Every scratch byte the backward reads is written earlier in the same
  // call, so nothing needs clearing between calls.
  cudaStream_t strm = static_cast<cudaStream_t>(stream);
  char* work = static_cast<char*>(scratch);
  if (s->bf16)
    return scan::backward<__nv_bfloat16>(*s, c, b, x, adt, dt, trap, angles, qb, kb,
                                         static_cast<const char*>(resid), dy, d_final, dc, db, dx, d_adt,
                                         d_dt, d_trap, d_angles, d_qb, d_kb, work, strm);
  return scan::backward<float>(*s, c, b, x, adt, dt, trap, angles, qb, kb, static_cast<const char*>(resid),
                               dy, d_final, dc, db, dx, d_adt, d_dt, d_trap, d_angles, d_qb, d_kb, work,
                               strm);
}
