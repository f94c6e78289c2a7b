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
//                    E <- lam E + beta k k^T in shared memory, then a block
//                    LDL^T of E + diag(floor) with 8x8 diagonal blocks, held
//                    in m16n8k8 accumulator fragments: the panel and trailing
//                    products on the tensor cores (three-term TF32), the
//                    diagonal blocks inverted by a Gauss-Jordan sweep with
//                    2x2 pivots (ldl_tiles.cuh); the forward substitution
//                    u = L^-1 q interleaved with the column blocks, the back
//                    substitution y = L^-T D^-1 u after them, and a coalesced
//                    128-bit streaming store of the factor (unit L, D^-1
//                    blocks) for the backward, whose substitutions need no
//                    inversion. The reference factorises the same matrix by
//                    Cholesky (mamba4_fused.py:78-113); both give A^-1 q to
//                    float32 rounding.
//   memread_output   per (batch, 64-token chunk, head): output =
//                    ((Y K^T) o W) V + diag(e^P) Y C0^T (mamba4_fused.py:439-447).
//   backward         rhs g (chunk products), z = A^-1 g from the stored
//                    factors (blocked substitutions), the chunk adjoint carry,
//                    and every input gradient in chunk form; the algebra is
//                    written out in oracle/memread.py:chunked_backward.
#include "common.cuh"
#include "tf32.cuh"
#include "ldl_tiles.cuh"

namespace m4 {
namespace mem {

constexpr int KD = 64;         // key dimension
constexpr int CH = 64;         // chunk (epilogue / backward products)
constexpr int SUB = 16;        // tokens per solve warp (state stride)
constexpr int LSTRIDE = 72 * 32;  // floats of one stored factor (18 float4 per lane)
constexpr int WARPS = 4;       // solve warps per CTA
#ifndef M4_STATES_MINB
#define M4_STATES_MINB 2
#endif


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


// Each 16-token sub-chunk is applied in one pass: with P_s the inclusive
// prefix of log lambda inside the sub-chunk,
//   S_end = e^(P_15) S_start + sum_s beta_s e^(P_15 - P_s) k_s k_s^T
// (the same recurrence, every weight <= beta_s), so a token costs one paired
// FMA per two state entries and the decay one paired multiply per sub-chunk.
// Thread (rq, cq) = (tid / 16, tid % 16) owns the 4x4 block rows 4rq..4rq+3,
// columns 4cq..4cq+3 of S and of each 64-row block of C, as column pairs
// (64-bit registers). A warp's shared reads per token are sixteen distinct
// column vectors and two row vectors (conflict-free; a layout with four
// threads per row made every 128-bit read a 5-way bank conflict).
template <int P>
__global__ void __launch_bounds__(256, M4_STATES_MINB) states_kernel(
    int B, int T, int H, const float* __restrict__ keys, const float* __restrict__ values,
    const float* __restrict__ beta, const float* __restrict__ log_decay,
    const float* __restrict__ init_s, const float* __restrict__ init_c,
    float* __restrict__ s_start, float* __restrict__ c_start,
    float* __restrict__ s_final, float* __restrict__ c_final) {
  using u64 = unsigned long long;
  constexpr int CR = P / 64;
  const int bh = blockIdx.x, b = bh / H, h = bh % H;
  const int tid = threadIdx.x;
  const int Tp = (T + CH - 1) / CH * CH, nsub = Tp / SUB, nch = Tp / CH;
  const int r0 = 4 * (tid >> 4), c0 = 4 * (tid & 15);
  // Two sub-chunk buffers: the next sub-chunk's keys, values, beta and
  // log_decay stream in (cp.async) while the current one is applied.
  __shared__ __align__(16) float ks[2][SUB][KD];
  __shared__ __align__(16) float vs[2][SUB][P];
  __shared__ float bl[2][SUB], ll[2][SUB];
  __shared__ float wsub[SUB], dsub;
  auto prefetch = [&](int buf, int sub) {
    const int t0 = sub * SUB;
#pragma unroll
    for (int idx = tid; idx < SUB * KD / 4; idx += 256) {
      const int tt = idx / (KD / 4), d4 = idx % (KD / 4), t = t0 + tt;
      const bool live = t < T;
      cp16(&ks[buf][tt][4 * d4], live ? keys + ((size_t(b) * T + t) * H + h) * KD + 4 * d4 : keys, live);
    }
#pragma unroll
    for (int idx = tid; idx < SUB * P / 4; idx += 256) {
      const int tt = idx / (P / 4), p4 = idx % (P / 4), t = t0 + tt;
      const bool live = t < T;
      cp16(&vs[buf][tt][4 * p4], live ? values + ((size_t(b) * T + t) * H + h) * P + 4 * p4 : values, live);
    }
    if (tid < SUB) {
      const int t = t0 + tid;
      const bool live = t < T;
      const size_t o = (size_t(b) * T + t) * H + h;
      cp4(&bl[buf][tid], live ? beta + o : beta, live);        // beta 0 past T
      cp4(&ll[buf][tid], live ? log_decay + o : log_decay, live);  // lambda 1 past T
    }
    cp_commit();
  };
  // s[a][q]: S[r0 + a][c0 + 2q .. c0 + 2q + 1]; c[r][a][q]: C[r0 + a + 64 r][...].
  u64 s[4][2], c[CR][4][2];
#pragma unroll
  for (int a = 0; a < 4; ++a) {
    ulonglong2 v = make_ulonglong2(0ull, 0ull);
    if (init_s) v = *reinterpret_cast<const ulonglong2*>(init_s + (size_t(bh) * KD + r0 + a) * KD + c0);
    s[a][0] = v.x; s[a][1] = v.y;
#pragma unroll
    for (int r = 0; r < CR; ++r) {
      ulonglong2 w = make_ulonglong2(0ull, 0ull);
      if (init_c) w = *reinterpret_cast<const ulonglong2*>(init_c + (size_t(bh) * P + r0 + a + 64 * r) * KD + c0);
      c[r][a][0] = w.x; c[r][a][1] = w.y;
    }
  }
  prefetch(0, 0);
  for (int sub = 0; sub < nsub; ++sub) {
    const int buf = sub & 1;
    if (sub + 1 < nsub) prefetch(buf ^ 1, sub + 1);
    float* sd = s_start + (size_t(bh) * nsub + sub) * KD * KD + c0;
#pragma unroll
    for (int a = 0; a < 4; ++a)
      *reinterpret_cast<ulonglong2*>(sd + (r0 + a) * KD) = make_ulonglong2(s[a][0], s[a][1]);
    if ((sub & 3) == 0) {
      float* cd = c_start + (size_t(bh) * nch + (sub >> 2)) * P * KD + c0;
#pragma unroll
      for (int r = 0; r < CR; ++r)
#pragma unroll
        for (int a = 0; a < 4; ++a)
          *reinterpret_cast<ulonglong2*>(cd + (r0 + a + 64 * r) * KD) = make_ulonglong2(c[r][a][0], c[r][a][1]);
    }
    if (sub + 1 < nsub) cp_wait_group<1>(); else cp_wait_group<0>();
    __syncthreads();
    if (tid < 32) {
      const float inc = warp_inclusive_scan(tid < SUB ? ll[buf][tid] : 0.f, tid);
      const float pend = __shfl_sync(0xffffffffu, inc, SUB - 1);
      if (tid < SUB) wsub[tid] = bl[buf][tid] * expf(pend - inc);
      if (tid == 0) dsub = expf(pend);
    }
    __syncthreads();
    {
      u64 dd;
      asm("mov.b64 %0, {%1,%1};" : "=l"(dd) : "f"(dsub));
#pragma unroll
      for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int q = 0; q < 2; ++q) {
          asm("mul.rn.f32x2 %0, %0, %1;" : "+l"(s[a][q]) : "l"(dd));
#pragma unroll
          for (int r = 0; r < CR; ++r) asm("mul.rn.f32x2 %0, %0, %1;" : "+l"(c[r][a][q]) : "l"(dd));
        }
    }
#pragma unroll 4
    for (int tt = 0; tt < SUB; ++tt) {
      u64 ww, wk[2];
      asm("mov.b64 %0, {%1,%1};" : "=l"(ww) : "f"(wsub[tt]));
      {
        const ulonglong2 kc = *reinterpret_cast<const ulonglong2*>(&ks[buf][tt][c0]);
        asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(wk[0]) : "l"(kc.x), "l"(ww));
        asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(wk[1]) : "l"(kc.y), "l"(ww));
      }
      const float4 kr = ld4(&ks[buf][tt][r0]);
      const float krv[4] = {kr.x, kr.y, kr.z, kr.w};
#pragma unroll
      for (int a = 0; a < 4; ++a) {
        u64 d;
        asm("mov.b64 %0, {%1,%1};" : "=l"(d) : "f"(krv[a]));
        asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(s[a][0]) : "l"(d), "l"(wk[0]));
        asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(s[a][1]) : "l"(d), "l"(wk[1]));
      }
#pragma unroll
      for (int r = 0; r < CR; ++r) {
        const float4 vr = ld4(&vs[buf][tt][r0 + 64 * r]);
        const float vrv[4] = {vr.x, vr.y, vr.z, vr.w};
#pragma unroll
        for (int a = 0; a < 4; ++a) {
          u64 d;
          asm("mov.b64 %0, {%1,%1};" : "=l"(d) : "f"(vrv[a]));
          asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(c[r][a][0]) : "l"(d), "l"(wk[0]));
          asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(c[r][a][1]) : "l"(d), "l"(wk[1]));
        }
      }
    }
    __syncthreads();  // this buffer is refilled two sub-chunks later
  }
#pragma unroll
  for (int a = 0; a < 4; ++a) {
    *reinterpret_cast<ulonglong2*>(s_final + (size_t(bh) * KD + r0 + a) * KD + c0) = make_ulonglong2(s[a][0], s[a][1]);
#pragma unroll
    for (int r = 0; r < CR; ++r)
      *reinterpret_cast<ulonglong2*>(c_final + (size_t(bh) * P + r0 + a + 64 * r) * KD + c0) =
          make_ulonglong2(c[r][a][0], c[r][a][1]);
  }
}

// ---------------------------------------------------------------------------
// memread_solve with the factorisation on the tensor cores: a block LDL^T of
// each token's matrix in MMA accumulator fragments (ldl_tiles.cuh). One warp
// per 16-token sub-chunk; the running evidence is kept in shared
// memory in the stored factor's fragment layout, so the per-token update
// E = lam E + beta k k^T touches each lane's own entries.
// ---------------------------------------------------------------------------
struct TileSmem {
  float4 E[ldl::NQ][32];  // running evidence (stored-factor layout)
  float k[KD], q[KD], fl[KD], v[KD], y[KD];
};

M4_DEV float2 ld2f(const float* p) { return *reinterpret_cast<const float2*>(p); }

// One warp per CTA, 168 registers (twelve warps per SM): more warps per SM
// force spills of the fragment registers and run slower.
__global__ void __launch_bounds__(32, 12) solve_kernel(
    int B, int T, int H, const float* __restrict__ keys, const float* __restrict__ queries,
    const float* __restrict__ beta, const float* __restrict__ log_decay,
    const float* __restrict__ floor_, const float* __restrict__ s_start,
    float* __restrict__ Lst, float* __restrict__ Y, float* __restrict__ variance) {
  extern __shared__ __align__(16) unsigned char tsolve_raw[];
  TileSmem* smem_all = reinterpret_cast<TileSmem*>(tsolve_raw);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int Tp = (T + CH - 1) / CH * CH, nsub = Tp / SUB;
  const int wid = blockIdx.x;
  if (wid >= B * H * nsub) return;
  TileSmem& sm = smem_all[warp];
  const int sub = wid % nsub, bh = wid / nsub, bb = bh / H, h = bh % H;
  {
    const float* src = s_start + (size_t(bh) * nsub + sub) * KD * KD;
#pragma unroll
    for (int q = 0; q < 16; ++q) {
      const int r0 = 16 * ldl::slot_R(q) + g, c0 = 8 * ldl::slot_c(q) + 2 * t;
      const float2 lo = ld2f(src + r0 * KD + c0), hi = ld2f(src + (r0 + 8) * KD + c0);
      sm.E[q][lane] = make_float4(lo.x, lo.y, hi.x, hi.y);
    }
#pragma unroll
    for (int q = 16; q < ldl::NQ; ++q) {
      const int R0 = 2 * (q - 16), R1 = R0 + 1;
      const float2 e0 = ld2f(src + (16 * R0 + 8 + g) * KD + 8 * (2 * R0 + 1) + 2 * t);
      const float2 e1 = ld2f(src + (16 * R1 + 8 + g) * KD + 8 * (2 * R1 + 1) + 2 * t);
      sm.E[q][lane] = make_float4(e0.x, e0.y, e1.x, e1.y);
    }
    sm.fl[lane] = floor_[h * KD + lane];
    sm.fl[lane + 32] = floor_[h * KD + lane + 32];
  }
  __syncwarp();

  // Key / query (lanes 0..15 / 16..31, four entries each), beta and
  // log-decay of a token, loaded one token ahead of its use.
  const float* kq = (lane < 16 ? keys : queries) + (size_t(bb) * T * H + h) * KD + 4 * (lane & 15);
  const float* bl = (lane < 16 ? beta : log_decay) + size_t(bb) * T * H + h;
  auto fetch = [&](int tok, float4& v, float& s) {
    const bool live = tok < T;
    v = live ? ld4(kq + size_t(tok) * H * KD) : make_float4(0.f, 0.f, 0.f, 0.f);
    s = live ? bl[size_t(tok) * H] : 0.f;
  };
  float4 nkq;
  float nbl;
  fetch(sub * SUB, nkq, nbl);
  for (int tt = 0; tt < SUB; ++tt) {
    const int tok = sub * SUB + tt;
    const bool live = tok < T;
    st4((lane < 16 ? sm.k : sm.q) + 4 * (lane & 15), nkq);
    const float bet = __shfl_sync(0xffffffffu, nbl, 0);
    const float lam = expf(__shfl_sync(0xffffffffu, nbl, 16));  // 1 past the end (log-decay 0)
    if (tt + 1 < SUB) fetch(tok + 1, nkq, nbl);
    __syncwarp();

    ldl::Tiles F;
    {
      float kr[4][2];
      float2 kc[8];
#pragma unroll
      for (int R = 0; R < 4; ++R) {
        kr[R][0] = bet * sm.k[16 * R + g];
        kr[R][1] = bet * sm.k[16 * R + 8 + g];
      }
#pragma unroll
      for (int c = 0; c < 8; ++c) kc[c] = ld2f(&sm.k[8 * c + 2 * t]);
      // Paired FMAs (fma.rn.f32x2): the same roundings as two scalar FMAs.
      const float2 l2 = make_float2(lam, lam);
#pragma unroll
      for (int q = 0; q < ldl::NQ; ++q) {
        const float4 e = sm.E[q][lane];
        float2 lo, hi;
        if (q < 16) {
          const int R = ldl::slot_R(q), c = ldl::slot_c(q);
          lo = ffma2(make_float2(kr[R][0], kr[R][0]), kc[c], fmul2(l2, make_float2(e.x, e.y)));
          hi = ffma2(make_float2(kr[R][1], kr[R][1]), kc[c], fmul2(l2, make_float2(e.z, e.w)));
        } else {
          const int R0 = 2 * (q - 16), R1 = R0 + 1;
          lo = ffma2(make_float2(kr[R0][1], kr[R0][1]), kc[2 * R0 + 1], fmul2(l2, make_float2(e.x, e.y)));
          hi = ffma2(make_float2(kr[R1][1], kr[R1][1]), kc[2 * R1 + 1], fmul2(l2, make_float2(e.z, e.w)));
        }
        const float4 en = make_float4(lo.x, lo.y, hi.x, hi.y);
        sm.E[q][lane] = en;
        ldl::set4(F, q, en);
      }
    }
    // Floor on the diagonal: entries (16R + g, 16R + g) of tile (R, 2R) and
    // (16R + 8 + g, ...) of tile (R, 2R + 1), on the lanes with 2t or 2t + 1 = g.
#pragma unroll
    for (int R = 0; R < 4; ++R) {
      const float f0 = sm.fl[16 * R + g], f1 = sm.fl[16 * R + 8 + g];
      F[ldl::ti(R, 2 * R)][0] += g == 2 * t ? f0 : 0.f;
      F[ldl::ti(R, 2 * R)][1] += g == 2 * t + 1 ? f0 : 0.f;
      F[ldl::ti(R, 2 * R + 1)][2] += g == 2 * t ? f1 : 0.f;
      F[ldl::ti(R, 2 * R + 1)][3] += g == 2 * t + 1 ? f1 : 0.f;
    }
    ldl::Forward fw;
    fw.uv = 0.f;
    fw.r = sm.q;
    fw.vsm = sm.v;
    ldl::factor_forward(F, fw, g, t);
    const float var = warp_sum(fw.uv);
    {
      float* dst = Lst + (size_t(bh) * Tp + tok) * LSTRIDE;
#pragma unroll
      for (int q = 0; q < ldl::NQ; ++q) st4_stream(dst + (q * 32 + lane) * 4, ldl::get4(F, q));
    }
    __syncwarp();
    ldl::back_solve(F, sm.v, sm.y, g, t);
    __syncwarp();
    if (lane < 16) st4(Y + (size_t(bh) * Tp + tok) * KD + 4 * lane, ld4(&sm.y[4 * lane]));
    if (live && lane == 0) variance[(size_t(bb) * T + tok) * H + h] = var;
    __syncwarp();
  }
}

// ---------------------------------------------------------------------------
// memread_decode: one token per (batch, head) against a carried state
// (selective_decode, lm/kernels/mamba4.py:341-355). One warp per (b, h):
//   E' = lam E + beta k k^T, C' = lam C + beta v k^T,
//   y = (E' + diag(floor))^-1 q, output = C' y, variance = q . y,
// with the memory read's block LDL^T in tensor-core fragments (ldl_tiles.cuh).
// E' and C' may overwrite E and C: the warp reads all of E before writing
// E', and each row of C before writing that row.
// ---------------------------------------------------------------------------
struct DecodeSmem {
  float k[KD], q[KD], v[KD], y[KD];
};

template <int P>
__global__ void __launch_bounds__(32 * WARPS) decode_kernel(
    int B, int H, const float* evidence, const float* cross,
    const float* __restrict__ key, const float* __restrict__ value, const float* __restrict__ query,
    const float* __restrict__ beta, const float* __restrict__ log_decay,
    const float* __restrict__ floor_, float* __restrict__ out, float* __restrict__ variance,
    float* evidence_out, float* cross_out) {  // may alias evidence / cross
  extern __shared__ __align__(16) unsigned char decode_raw[];
  DecodeSmem* smem_all = reinterpret_cast<DecodeSmem*>(decode_raw);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int bh = blockIdx.x * WARPS + warp;
  if (bh >= B * H) return;
  DecodeSmem& sm = smem_all[warp];
  const int h = bh % H;
  // E (symmetric, row-major) into the lower tiles; every load before any store.
  const float* src = evidence + size_t(bh) * KD * KD;
  ldl::Tiles F;
#pragma unroll
  for (int q = 0; q < 16; ++q) {
    const int r0 = 16 * ldl::slot_R(q) + g, c0 = 8 * ldl::slot_c(q) + 2 * t;
    const float2 lo = ld2f(src + r0 * KD + c0), hi = ld2f(src + (r0 + 8) * KD + c0);
    F[q][0] = lo.x; F[q][1] = lo.y; F[q][2] = hi.x; F[q][3] = hi.y;
  }
#pragma unroll
  for (int R = 0; R < 4; ++R) {
    const float2 e = ld2f(src + (16 * R + 8 + g) * KD + 8 * (2 * R + 1) + 2 * t);
    F[16 + R][2] = e.x; F[16 + R][3] = e.y;
  }
  {
    const int l = lane & 15;
    st4((lane < 16 ? sm.k : sm.q) + 4 * l, ld4((lane < 16 ? key : query) + size_t(bh) * KD + 4 * l));
  }
  const float bet = beta[bh];
  const float lam = expf(log_decay[bh]);
  __syncwarp();
  // E' = lam E + beta k k^T, written back whole: the kept entries in place,
  // the strictly lower ones mirrored.
  {
    float kr[4][2];
    float2 kc[8];
#pragma unroll
    for (int R = 0; R < 4; ++R) {
      kr[R][0] = bet * sm.k[16 * R + g];
      kr[R][1] = bet * sm.k[16 * R + 8 + g];
    }
#pragma unroll
    for (int c = 0; c < 8; ++c) kc[c] = ld2f(&sm.k[8 * c + 2 * t]);
    float* dst = evidence_out + size_t(bh) * KD * KD;
#pragma unroll
    for (int q = 0; q < 16; ++q) {
      const int R = ldl::slot_R(q), c = ldl::slot_c(q);
      float* e = F[q];
      e[0] = fmaf(kr[R][0], kc[c].x, lam * e[0]);
      e[1] = fmaf(kr[R][0], kc[c].y, lam * e[1]);
      e[2] = fmaf(kr[R][1], kc[c].x, lam * e[2]);
      e[3] = fmaf(kr[R][1], kc[c].y, lam * e[3]);
      const int r0 = 16 * R + g, c0 = 8 * c + 2 * t;
      *reinterpret_cast<float2*>(dst + r0 * KD + c0) = make_float2(e[0], e[1]);
      *reinterpret_cast<float2*>(dst + (r0 + 8) * KD + c0) = make_float2(e[2], e[3]);
      if (c < 2 * R) {  // rows 16R.. below the diagonal block
        dst[c0 * KD + r0] = e[0];
        dst[(c0 + 1) * KD + r0] = e[1];
      }
      dst[c0 * KD + r0 + 8] = e[2];  // rows 16R + 8.. are below every column of the tile
      dst[(c0 + 1) * KD + r0 + 8] = e[3];
    }
#pragma unroll
    for (int R = 0; R < 4; ++R) {
      float* e = F[16 + R];
      e[2] = fmaf(kr[R][1], kc[2 * R + 1].x, lam * e[2]);
      e[3] = fmaf(kr[R][1], kc[2 * R + 1].y, lam * e[3]);
      *reinterpret_cast<float2*>(dst + (16 * R + 8 + g) * KD + 8 * (2 * R + 1) + 2 * t) = make_float2(e[2], e[3]);
    }
  }
#pragma unroll
  for (int R = 0; R < 4; ++R) {
    const float f0 = floor_[h * KD + 16 * R + g], f1 = floor_[h * KD + 16 * R + 8 + g];
    F[ldl::ti(R, 2 * R)][0] += g == 2 * t ? f0 : 0.f;
    F[ldl::ti(R, 2 * R)][1] += g == 2 * t + 1 ? f0 : 0.f;
    F[ldl::ti(R, 2 * R + 1)][2] += g == 2 * t ? f1 : 0.f;
    F[ldl::ti(R, 2 * R + 1)][3] += g == 2 * t + 1 ? f1 : 0.f;
  }
  ldl::Forward fw;
  fw.uv = 0.f;
  fw.r = sm.q;
  fw.vsm = sm.v;
  ldl::factor_forward(F, fw, g, t);
  const float var = warp_sum(fw.uv);
  __syncwarp();
  ldl::back_solve(F, sm.v, sm.y, g, t);
  __syncwarp();
  if (lane == 0) variance[bh] = var;
  float kkeep[2] = {sm.k[2 * lane], sm.k[2 * lane + 1]};
  // C' = lam C + beta v k^T, lane l on key coordinates 2l, 2l+1, rows in
  // batches of R whose loads are issued before the previous batch's stores
  // (cross_out may alias cross: row p is always read before it is written,
  // and a batch never reads a row an earlier batch wrote), so the DRAM
  // round trips overlap. output_p = C'[p] . y.
  const float2 yv = *reinterpret_cast<const float2*>(&sm.y[2 * lane]);
  const float2 bk = make_float2(bet * kkeep[0], bet * kkeep[1]);
  const float* csrc = cross + size_t(bh) * P * KD + 2 * lane;
  float* cdst = cross_out + size_t(bh) * P * KD + 2 * lane;
  const float* vrow = value + size_t(bh) * P;
  float* orow = out + size_t(bh) * P;
  constexpr int R = 16;
  float2 cur[R];
#pragma unroll
  for (int r = 0; r < R; ++r) cur[r] = *reinterpret_cast<const float2*>(csrc + r * KD);
#pragma unroll 1
  for (int p0 = 0; p0 < P; p0 += R) {
    float2 nxt[R];
    if (p0 + R < P) {
#pragma unroll
      for (int r = 0; r < R; ++r) nxt[r] = *reinterpret_cast<const float2*>(csrc + (p0 + R + r) * KD);
    }
    float part[R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const float vp = vrow[p0 + r];
      const float2 c = make_float2(fmaf(bk.x, vp, lam * cur[r].x), fmaf(bk.y, vp, lam * cur[r].y));
      *reinterpret_cast<float2*>(cdst + (p0 + r) * KD) = c;
      part[r] = fmaf(c.x, yv.x, c.y * yv.y);
    }
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const float o = warp_sum(part[r]);
      if (lane == 0) orow[p0 + r] = o;
    }
    if (p0 + R < P) {
#pragma unroll
      for (int r = 0; r < R; ++r) cur[r] = nxt[r];
    }
  }
}

// ---------------------------------------------------------------------------
// spd_solve: standalone SPD solves precision @ y = rhs (spd_solve,
// lm/kernels/mamba4.py:187-218) for `count` matrices of order dim <= 64.
// One warp per matrix with the memory read's block LDL^T (ldl_tiles.cuh).
// Only the lower triangle of each row-major [dim][dim] matrix is read (the
// diagonal blocks' upper entries are mirrored from it); orders below 64 are
// padded with an identity block and a zero right-hand side, which solves to
// zero. The factor is stored in the memory read's fragment layout (LSTRIDE
// floats per matrix: unit L, D^-1 blocks) for the backward.
// ---------------------------------------------------------------------------
M4_DEV float spd_entry(const float* M, int dim, int r, int c) {
  if (r >= dim || c >= dim) return r == c ? 1.f : 0.f;
  return r >= c ? M[r * dim + c] : M[c * dim + r];
}

struct SpdSmem {
  float r[KD], v[KD], y[KD], s[KD];
};

__global__ void __launch_bounds__(32 * WARPS) spd_fwd_kernel(
    int count, int dim, const float* __restrict__ precision, const float* __restrict__ rhs,
    float* __restrict__ solution, float* __restrict__ Lst) {
  extern __shared__ __align__(16) unsigned char spd_raw[];
  SpdSmem* smem_all = reinterpret_cast<SpdSmem*>(spd_raw);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int m = blockIdx.x * WARPS + warp;
  if (m >= count) return;
  SpdSmem& sm = smem_all[warp];
  const float* src = precision + size_t(m) * dim * dim;
  ldl::Tiles F;
#pragma unroll
  for (int q = 0; q < 16; ++q) {
    const int r0 = 16 * ldl::slot_R(q) + g, c0 = 8 * ldl::slot_c(q) + 2 * t;
    F[q][0] = spd_entry(src, dim, r0, c0);
    F[q][1] = spd_entry(src, dim, r0, c0 + 1);
    F[q][2] = spd_entry(src, dim, r0 + 8, c0);
    F[q][3] = spd_entry(src, dim, r0 + 8, c0 + 1);
  }
#pragma unroll
  for (int R = 0; R < 4; ++R) {
    const int r = 16 * R + 8 + g, c = 8 * (2 * R + 1) + 2 * t;
    F[16 + R][2] = spd_entry(src, dim, r, c);
    F[16 + R][3] = spd_entry(src, dim, r, c + 1);
  }
  const float* g_ = rhs + size_t(m) * dim;
  for (int i = lane; i < KD; i += 32) sm.r[i] = i < dim ? g_[i] : 0.f;
  __syncwarp();
  ldl::Forward fw;
  fw.uv = 0.f;
  fw.r = sm.r;
  fw.vsm = sm.v;
  ldl::factor_forward(F, fw, g, t);
  {
    float* dst = Lst + size_t(m) * LSTRIDE;
#pragma unroll
    for (int q = 0; q < ldl::NQ; ++q) st4(dst + (q * 32 + lane) * 4, ldl::get4(F, q));
  }
  __syncwarp();
  ldl::back_solve(F, sm.v, sm.y, g, t);
  __syncwarp();
  float* out = solution + size_t(m) * dim;
  for (int i = lane; i < dim; i += 32) out[i] = sm.y[i];
}

// Backward of spd_solve (lm/kernels/mamba4.py:208-215): z = A^-1 g from the
// stored factor, d rhs = z, d precision = -(z y^T + y z^T) / 2 (all dim x dim
// entries, as the reference's symmetric cotangent).
__global__ void __launch_bounds__(32 * WARPS) spd_bwd_kernel(
    int count, int dim, const float* __restrict__ Lst, const float* __restrict__ solution,
    const float* __restrict__ d_solution, float* __restrict__ d_precision, float* __restrict__ d_rhs) {
  extern __shared__ __align__(16) unsigned char spdb_raw[];
  SpdSmem* smem_all = reinterpret_cast<SpdSmem*>(spdb_raw);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int m = blockIdx.x * WARPS + warp;
  if (m >= count) return;
  SpdSmem& sm = smem_all[warp];
  ldl::Tiles F;
  {
    const float* src = Lst + size_t(m) * LSTRIDE;
#pragma unroll
    for (int q = 0; q < ldl::NQ; ++q) ldl::set4(F, q, ld4(src + (q * 32 + lane) * 4));
  }
  const float* gs = d_solution + size_t(m) * dim;
  const float* y = solution + size_t(m) * dim;
  for (int i = lane; i < KD; i += 32) {
    sm.r[i] = i < dim ? gs[i] : 0.f;
    sm.s[i] = i < dim ? y[i] : 0.f;  // the solution, kept for the outer product
  }
  __syncwarp();
  ldl::forward_solve(F, sm.r, sm.v, g, t);
  __syncwarp();
  ldl::back_solve(F, sm.v, sm.y, g, t);  // z in sm.y
  __syncwarp();
  float* dr = d_rhs + size_t(m) * dim;
  for (int i = lane; i < dim; i += 32) dr[i] = sm.y[i];
  float* dp = d_precision + size_t(m) * dim * dim;
  for (int idx = lane; idx < dim * dim; idx += 32) {
    const int i = idx / dim, j = idx - i * dim;
    dp[idx] = -0.5f * fmaf(sm.y[i], sm.s[j], sm.s[i] * sm.y[j]);
  }
}

// ---------------------------------------------------------------------------
// Chunk-product kernels: one CTA of 8 warps per (batch, 64-token chunk, head)
// (carry: one per (batch, head)). The products run on tensor cores as m16n8k8
// TF32 MMAs on a two-term split of every fp32 operand (hi = x rounded to 11
// significant bits by Veltkamp splitting on the FMA pipe, lo = x - hi passed
// as is: the tensor core reads its top 19 bits) with three products per tile
// (lo*hi + hi*lo + hi*hi): about 2^-21 relative error per product, inside the
// float32 tolerance of the reference (whose einsums run at
// Precision.HIGHEST, lm/kernels/mamba4_fused.py:411-447). Neither half needs
// an ALU conversion: the ALU pipe is the one these kernels saturate.
// Warp w owns rows 16 (w % 4) .. +15 and column half w / 4 of each product.
// ---------------------------------------------------------------------------
constexpr int LD = 68;    // tile stride in floats (conflict-free A fragments)
constexpr int CT = 256;   // threads per chunk CTA
constexpr int CTG = 512;  // threads per chunk-gradient CTA (16 warps: 4 row blocks x 4 column quarters)

// acc[nt][e] += sum_k A(row0 + g + 8(e>>1), k) B(k, col0 + 8nt + 2c + (e&1)),
// g = lane/4, c = lane%4, through element accessors fa(row, k), fb(k, col).
template <int K, int NT, class FA, class FB>
M4_DEV void gemm3(float (&acc)[NT][4], int row0, int col0, FA fa, FB fb) {
  const int lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
#pragma unroll 2
  for (int k0 = 0; k0 < K; k0 += 8) {
    const float av[4] = {fa(row0 + g, k0 + c), fa(row0 + g + 8, k0 + c), fa(row0 + g, k0 + c + 4),
                         fa(row0 + g + 8, k0 + c + 4)};
    uint32_t ah[4], al[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      ah[i] = split_hi(av[i]);
      al[i] = __float_as_uint(av[i] - __uint_as_float(ah[i]));  // read as tf32 (low bits ignored)
    }
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const float b0 = fb(k0 + c, col0 + 8 * nt + g), b1 = fb(k0 + c + 4, col0 + 8 * nt + g);
      const uint32_t bh[2] = {split_hi(b0), split_hi(b1)};
      const uint32_t bl[2] = {__float_as_uint(b0 - __uint_as_float(bh[0])),
                              __float_as_uint(b1 - __uint_as_float(bh[1]))};
      mma_tf32(acc[nt], al, bh);
      mma_tf32(acc[nt], ah, bl);
      mma_tf32(acc[nt], ah, bh);
    }
  }
}

// Two products with the same B operand (acc1 += A1 B, acc2 += A2 B): each B
// fragment is loaded and split once.
template <int K, int NT, class FA1, class FA2, class FB>
M4_DEV void gemm3_shared_b(float (&acc1)[NT][4], float (&acc2)[NT][4], int row0, int col0, FA1 fa1, FA2 fa2, FB fb) {
  const int lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
#pragma unroll 2
  for (int k0 = 0; k0 < K; k0 += 8) {
    uint32_t ah[2][4], al[2][4];
    {
      const float av[2][4] = {{fa1(row0 + g, k0 + c), fa1(row0 + g + 8, k0 + c), fa1(row0 + g, k0 + c + 4),
                               fa1(row0 + g + 8, k0 + c + 4)},
                              {fa2(row0 + g, k0 + c), fa2(row0 + g + 8, k0 + c), fa2(row0 + g, k0 + c + 4),
                               fa2(row0 + g + 8, k0 + c + 4)}};
#pragma unroll
      for (int m = 0; m < 2; ++m)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          ah[m][i] = split_hi(av[m][i]);
          al[m][i] = __float_as_uint(av[m][i] - __uint_as_float(ah[m][i]));
        }
    }
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const float b0 = fb(k0 + c, col0 + 8 * nt + g), b1 = fb(k0 + c + 4, col0 + 8 * nt + g);
      const uint32_t bh[2] = {split_hi(b0), split_hi(b1)};
      const uint32_t bl[2] = {__float_as_uint(b0 - __uint_as_float(bh[0])),
                              __float_as_uint(b1 - __uint_as_float(bh[1]))};
      mma_tf32(acc1[nt], al[0], bh);
      mma_tf32(acc2[nt], al[1], bh);
      mma_tf32(acc1[nt], ah[0], bl);
      mma_tf32(acc2[nt], ah[1], bl);
      mma_tf32(acc1[nt], ah[0], bh);
      mma_tf32(acc2[nt], ah[1], bh);
    }
  }
}

// Two products with the same A operand (acc1 += A B1 at columns col1..,
// acc2 += A B2 at columns col2..): each A fragment is loaded and split once.
template <int K, int NT1, int NT2, class FA, class FB1, class FB2>
M4_DEV void gemm3_shared_a(float (&acc1)[NT1][4], float (&acc2)[NT2][4], int row0, int col1, int col2, FA fa,
                           FB1 fb1, FB2 fb2) {
  const int lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
#pragma unroll 2
  for (int k0 = 0; k0 < K; k0 += 8) {
    const float av[4] = {fa(row0 + g, k0 + c), fa(row0 + g + 8, k0 + c), fa(row0 + g, k0 + c + 4),
                         fa(row0 + g + 8, k0 + c + 4)};
    uint32_t ah[4], al[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      ah[i] = split_hi(av[i]);
      al[i] = __float_as_uint(av[i] - __uint_as_float(ah[i]));
    }
#pragma unroll
    for (int nt = 0; nt < NT1 + NT2; ++nt) {
      const bool first = nt < NT1;
      const int col = first ? col1 + 8 * nt : col2 + 8 * (nt - NT1);
      const float b0 = first ? fb1(k0 + c, col + g) : fb2(k0 + c, col + g);
      const float b1 = first ? fb1(k0 + c + 4, col + g) : fb2(k0 + c + 4, col + g);
      const uint32_t bh[2] = {split_hi(b0), split_hi(b1)};
      const uint32_t bl[2] = {__float_as_uint(b0 - __uint_as_float(bh[0])),
                              __float_as_uint(b1 - __uint_as_float(bh[1]))};
      float(&d)[4] = first ? acc1[nt < NT1 ? nt : 0] : acc2[nt < NT1 ? 0 : nt - NT1];
      mma_tf32(d, al, bh);
      mma_tf32(d, ah, bl);
      mma_tf32(d, ah, bh);
    }
  }
}

template <int NT>
M4_DEV void zero(float (&acc)[NT][4]) {
#pragma unroll
  for (int i = 0; i < NT; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
}

// Visit accumulator elements: f(row, col, nt, e).
template <int NT, class F>
M4_DEV void each(int row0, int col0, F f) {
  const int lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int e = 0; e < 4; ++e) f(row0 + g + 8 * (e >> 1), col0 + 8 * nt + 2 * c + (e & 1), nt, e);
}

// Chunk-local inclusive prefix of log_decay, the gates and e^prefix (warp 0).
M4_DEV void chunk_gates(int tid, int b, int T, int H, int h, int t0, const float* beta,
                        const float* log_decay, float* pre, float* bet, float* ept) {
  if (tid < 32) {
    float carry = 0.f;
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const int tt = half * 32 + tid, t = t0 + tt;
      const float g = t < T ? log_decay[(size_t(b) * T + t) * H + h] : 0.f;
      const float inc = warp_inclusive_scan(g, tid) + carry;
      pre[tt] = inc;
      ept[tt] = expf(inc);
      bet[tt] = t < T ? beta[(size_t(b) * T + t) * H + h] : 0.f;
      carry = __shfl_sync(0xffffffffu, inc, 31);
    }
  }
}

// Start copying a [64 tokens][W] chunk of a [B,T,H,W] tensor into a tile of
// stride ld (tokens past T read as zero).
template <int W, int NTH = CT>
M4_DEV void load_tokens(float* tile, int ld, const float* src, int b, int T, int H, int h, int t0, int tid) {
#pragma unroll
  for (int idx = tid; idx < CH * W / 4; idx += NTH) {
    const int tt = idx / (W / 4), c4 = idx % (W / 4), t = t0 + tt;
    const bool live = t < T;
    cp16(tile + tt * ld + 4 * c4, live ? src + ((size_t(b) * T + t) * H + h) * W + 4 * c4 : src, live);
  }
}

// Start copying a dense [rows][64] row-major block into a tile of stride LD.
template <int NTH = CT>
M4_DEV void load_block(float* tile, int rows, const float* src, int tid) {
  for (int idx = tid; idx < rows * KD / 4; idx += NTH) cp16(tile + (idx / 16) * LD + 4 * (idx % 16), src + 4 * idx, true);
}

template <int P>
__global__ void __launch_bounds__(CT) output_kernel(
    int B, int T, int H, const float* __restrict__ keys, const float* __restrict__ values,
    const float* __restrict__ beta, const float* __restrict__ log_decay,
    const float* __restrict__ Y, const float* __restrict__ c_start, float* __restrict__ out) {
  constexpr int LP = P + 4, NTP = P / 16;
  extern __shared__ __align__(16) float sh[];
  float* Ys = sh;                 // [64][LD]
  float* Ks = Ys + CH * LD;       // [64][LD]
  float* Ms = Ks;                 // [64][LD] over K once the scores are in registers
  float* Vs = Ks + CH * LD;       // [64][LP]
  float* C0 = Vs + CH * LP;       // [P][LD]
  float* pre = C0 + P * LD;
  float* bet = pre + CH;
  float* ept = bet + CH;
  const int Tp = (T + CH - 1) / CH * CH, nch = Tp / CH;
  const int ch = blockIdx.x % nch, bh = blockIdx.x / nch, b = bh / H, h = bh % H;
  const int t0 = ch * CH, tid = threadIdx.x, warp = tid >> 5;
  const int row0 = 16 * (warp & 3), half = warp >> 2;
  load_block(Ys, CH, Y + (size_t(bh) * Tp + t0) * KD, tid);
  load_tokens<KD>(Ks, LD, keys, b, T, H, h, t0, tid);
  load_tokens<P>(Vs, LP, values, b, T, H, h, t0, tid);
  load_block(C0, P, c_start + (size_t(bh) * nch + ch) * P * KD, tid);
  chunk_gates(tid, b, T, H, h, t0, beta, log_decay, pre, bet, ept);
  cp_wait();
  __syncthreads();
  {
    float acc[4][4];
    zero(acc);
    gemm3<KD, 4>(acc, row0, 32 * half, [&](int r, int k) { return Ys[r * LD + k]; },
                 [&](int k, int n) { return Ks[n * LD + k]; });
    __syncthreads();  // every warp is done with K
    each<4>(row0, 32 * half, [&](int r, int n, int nt, int e) {
      Ms[r * LD + n] = n <= r ? acc[nt][e] * bet[n] * expf(pre[r] - pre[n]) : 0.f;
    });
  }
  __syncthreads();
  float acc[NTP][4], inh[NTP][4];
  zero(acc);
  zero(inh);
  const int c0 = half * (P / 2);
  gemm3<CH, NTP>(acc, row0, c0, [&](int r, int k) { return Ms[r * LD + k]; },
                 [&](int k, int p) { return Vs[k * LP + p]; });
  gemm3<KD, NTP>(inh, row0, c0, [&](int r, int k) { return Ys[r * LD + k]; },
                 [&](int k, int p) { return C0[p * LD + k]; });
  each<NTP>(row0, c0, [&](int r, int p, int nt, int e) {
    const int t = t0 + r;
    if (t < T) out[((size_t(b) * T + t) * H + h) * P + p] = fmaf(ept[r], inh[nt][e], acc[nt][e]);
  });
}

// rhs_kernel: g_t = e^(P_t) C0^T dO_t + sum_s W[t,s] (dO_t . v_s) k_s + dvar_t q_t.
template <int P>
__global__ void __launch_bounds__(CT) rhs_kernel(
    int B, int T, int H, const float* __restrict__ keys, const float* __restrict__ values,
    const float* __restrict__ queries, const float* __restrict__ beta,
    const float* __restrict__ log_decay, const float* __restrict__ c_start,
    const float* __restrict__ d_out, const float* __restrict__ d_var, float* __restrict__ G) {
  constexpr int LP = P + 4;
  extern __shared__ __align__(16) float sh[];
  float* Ks = sh;                 // [64][LD]
  float* Os = Ks + CH * LD;       // [64][LP]
  float* Vs = Os + CH * LP;       // [64][LP]
  float* Ms = Vs;                 // [64][LD] over V once dO V^T is in registers
  float* C0 = Vs + CH * LP;       // [P][LD]
  float* pre = C0 + P * LD;
  float* bet = pre + CH;
  float* ept = bet + CH;
  const int Tp = (T + CH - 1) / CH * CH, nch = Tp / CH;
  const int ch = blockIdx.x % nch, bh = blockIdx.x / nch, b = bh / H, h = bh % H;
  const int t0 = ch * CH, tid = threadIdx.x, warp = tid >> 5;
  const int row0 = 16 * (warp & 3), half = warp >> 2;
  load_tokens<KD>(Ks, LD, keys, b, T, H, h, t0, tid);
  load_tokens<P>(Os, LP, d_out, b, T, H, h, t0, tid);
  load_tokens<P>(Vs, LP, values, b, T, H, h, t0, tid);
  load_block(C0, P, c_start + (size_t(bh) * nch + ch) * P * KD, tid);
  // The epilogue's dvar_t q_t term: loads start now, into registers
  // (this thread's accumulator elements: rows row0 + g (+8), columns
  // 32 half + 8 nt + 2 c (+1)).
  float2 qv[4][2];
  float dvr[2];
  {
    const int lane = tid & 31, g = lane >> 2, c = lane & 3;
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
      const int t = t0 + row0 + g + 8 * hf;
      const bool live = t < T;
      dvr[hf] = live ? d_var[(size_t(b) * T + t) * H + h] : 0.f;
#pragma unroll
      for (int nt = 0; nt < 4; ++nt)
        qv[nt][hf] = live ? *reinterpret_cast<const float2*>(queries + ((size_t(b) * T + t) * H + h) * KD +
                                                             32 * half + 8 * nt + 2 * c)
                          : make_float2(0.f, 0.f);
    }
  }
  chunk_gates(tid, b, T, H, h, t0, beta, log_decay, pre, bet, ept);
  cp_wait();
  __syncthreads();
  {
    float acc[4][4];
    zero(acc);
    gemm3<P, 4>(acc, row0, 32 * half, [&](int r, int k) { return Os[r * LP + k]; },
                [&](int k, int s) { return Vs[s * LP + k]; });
    __syncthreads();  // every warp is done with V
    each<4>(row0, 32 * half, [&](int r, int s, int nt, int e) {
      Ms[r * LD + s] = s <= r ? acc[nt][e] * bet[s] * expf(pre[r] - pre[s]) : 0.f;
    });
  }
  __syncthreads();
  float acc[4][4], inh[4][4];
  zero(acc);
  zero(inh);
  gemm3<CH, 4>(acc, row0, 32 * half, [&](int r, int k) { return Ms[r * LD + k]; },
               [&](int k, int d) { return Ks[k * LD + d]; });
  gemm3<P, 4>(inh, row0, 32 * half, [&](int r, int k) { return Os[r * LP + k]; },
              [&](int k, int d) { return C0[k * LD + d]; });
  each<4>(row0, 32 * half, [&](int r, int d, int nt, int e) {
    const int t = t0 + r;
    const float dv = dvr[e >> 1];
    const float q = (e & 1) ? qv[nt][e >> 1].y : qv[nt][e >> 1].x;
    G[(size_t(bh) * Tp + t) * KD + d] = fmaf(dv, q, fmaf(ept[r], inh[nt][e], acc[nt][e]));
  });
}

// ---------------------------------------------------------------------------
// Backward kernels.
// ---------------------------------------------------------------------------
// zsolve_kernel: z_t = A_t^-1 g_t from the tensor-core solve's stored
// factor (unit lower L, D^-1 blocks), the factor and right-hand side of the
// next token streaming into shared memory while the current one is solved.
__global__ void __launch_bounds__(32 * WARPS, 4) zsolve_kernel(
    int B, int T, int H, const float* __restrict__ Lst, const float* __restrict__ G,
    float* __restrict__ Z) {
  extern __shared__ __align__(16) unsigned char tzsolve_raw[];
  TileSmem* smem_all = reinterpret_cast<TileSmem*>(tzsolve_raw);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int Tp = (T + CH - 1) / CH * CH, nsub = Tp / SUB;
  const int wid = blockIdx.x * WARPS + warp;
  if (wid >= B * H * nsub) return;
  TileSmem& sm = smem_all[warp];
  const int sub = wid % nsub, bh = wid / nsub;
  auto prefetch = [&](int tok) {
    const float* src = Lst + (size_t(bh) * Tp + tok) * LSTRIDE;
#pragma unroll
    for (int q = 0; q < ldl::NQ; ++q)
      cp16(reinterpret_cast<float*>(&sm.E[q][lane]), src + (q * 32 + lane) * 4, true);
    if (lane < 16) cp16(&sm.k[4 * lane], G + (size_t(bh) * Tp + tok) * KD + 4 * lane, true);
    cp_commit();
  };
  prefetch(sub * SUB);
  for (int tt = 0; tt < SUB; ++tt) {
    const int tok = sub * SUB + tt;
    cp_wait_group<0>();
    __syncwarp();
    ldl::Tiles F;
#pragma unroll
    for (int q = 0; q < ldl::NQ; ++q) ldl::set4(F, q, sm.E[q][lane]);
    if (lane < 16) st4(&sm.q[4 * lane], ld4(&sm.k[4 * lane]));
    __syncwarp();  // the buffers are refilled below
    if (tt + 1 < SUB) prefetch(tok + 1);
    ldl::forward_solve(F, sm.q, sm.v, g, t);
    __syncwarp();
    ldl::back_solve(F, sm.v, sm.y, g, t);
    __syncwarp();
    if (lane < 16) st4(Z + (size_t(bh) * Tp + tok) * KD + 4 * lane, ld4(&sm.y[4 * lane]));
    __syncwarp();
  }
}

// carry_kernel: per (batch, head), reverse over chunks:
//   X_S = -sum_t e^(P_t) z_t y_t^T, X_C = sum_t e^(P_t) dO_t y_t^T,
//   Sbar_end[n] = carry, carry = X_S[n] + e^(P_L) carry (same for C).
// The final carries are the gradients of the initial state.
template <int P>
__global__ void __launch_bounds__(CT) carry_kernel(
    int B, int T, int H, const float* __restrict__ beta, const float* __restrict__ log_decay,
    const float* __restrict__ Y, const float* __restrict__ Z, const float* __restrict__ d_out,
    const float* __restrict__ d_sfin, const float* __restrict__ d_cfin,
    float* __restrict__ sbar, float* __restrict__ cbar, float* __restrict__ d_init_s,
    float* __restrict__ d_init_c) {
  constexpr int LP = P + 4, NTP = P / 16;
  extern __shared__ __align__(16) float sh[];
  float* Ys = sh;               // [64][LD] rows t
  float* Zs = Ys + CH * LD;     // [64][LD]
  float* Os = Zs + CH * LD;     // [64][LP]
  float* pre = Os + CH * LP;
  float* bet = pre + CH;
  float* ept = bet + CH;
  const int Tp = (T + CH - 1) / CH * CH, nch = Tp / CH;
  const int bh = blockIdx.x, b = bh / H, h = bh % H;
  const int tid = threadIdx.x, warp = tid >> 5;
  const int row0 = 16 * (warp & 3), half = warp >> 2;
  const int cs0 = 32 * half, cc0 = half * (P / 2);
  // cs[d][e] rows d, cols e; cc[d][p] = Cbar[p][d] (transposed).
  float cs[4][4], cc[NTP][4];
  each<4>(row0, cs0, [&](int d, int e, int nt, int i) {
    cs[nt][i] = d_sfin ? d_sfin[(size_t(bh) * KD + d) * KD + e] : 0.f;
  });
  each<NTP>(row0, cc0, [&](int d, int p, int nt, int i) {
    cc[nt][i] = d_cfin ? d_cfin[(size_t(bh) * P + p) * KD + d] : 0.f;
  });
  for (int ch = nch - 1; ch >= 0; --ch) {
    const int t0 = ch * CH;
    float* sb = sbar + (size_t(bh) * nch + ch) * KD * KD;
    float* cbp = cbar + (size_t(bh) * nch + ch) * P * KD;
    each<4>(row0, cs0, [&](int d, int e, int nt, int i) { sb[d * KD + e] = cs[nt][i]; });
    each<NTP>(row0, cc0, [&](int d, int p, int nt, int i) { cbp[p * KD + d] = cc[nt][i]; });
    __syncthreads();  // previous iteration's readers of the tiles are done
    load_block(Ys, CH, Y + (size_t(bh) * Tp + t0) * KD, tid);
    load_block(Zs, CH, Z + (size_t(bh) * Tp + t0) * KD, tid);
    load_tokens<P>(Os, LP, d_out, b, T, H, h, t0, tid);
    chunk_gates(tid, b, T, H, h, t0, beta, log_decay, pre, bet, ept);
    cp_wait();
    __syncthreads();
    const float end = ept[CH - 1];
    float xs[4][4], xc[NTP][4];
    zero(xs);
    zero(xc);
    gemm3<CH, 4>(xs, row0, cs0, [&](int d, int t) { return Zs[t * LD + d] * ept[t]; },
                 [&](int t, int e) { return Ys[t * LD + e]; });
    gemm3<CH, NTP>(xc, row0, cc0, [&](int d, int t) { return Ys[t * LD + d] * ept[t]; },
                   [&](int t, int p) { return Os[t * LP + p]; });
#pragma unroll
    for (int nt = 0; nt < 4; ++nt)
#pragma unroll
      for (int i = 0; i < 4; ++i) cs[nt][i] = fmaf(end, cs[nt][i], -xs[nt][i]);
#pragma unroll
    for (int nt = 0; nt < NTP; ++nt)
#pragma unroll
      for (int i = 0; i < 4; ++i) cc[nt][i] = fmaf(end, cc[nt][i], xc[nt][i]);
  }
  if (d_init_s) each<4>(row0, cs0, [&](int d, int e, int nt, int i) { d_init_s[(size_t(bh) * KD + d) * KD + e] = cs[nt][i]; });
  if (d_init_c) each<NTP>(row0, cc0, [&](int d, int p, int nt, int i) { d_init_c[(size_t(bh) * P + p) * KD + d] = cc[nt][i]; });
}

// Sum a per-lane, per-row partial (rows r = row0 + g + 8*(e>>1)) over the 4
// lanes of each row and store it at dst[r] (one writer per row and warp).
M4_DEV void row_reduce_store(float v0, float v1, float* dst, int row0) {
  const int lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
  v0 += __shfl_xor_sync(0xffffffffu, v0, 1);
  v0 += __shfl_xor_sync(0xffffffffu, v0, 2);
  v1 += __shfl_xor_sync(0xffffffffu, v1, 1);
  v1 += __shfl_xor_sync(0xffffffffu, v1, 2);
  if (c == 0) { dst[row0 + g] = v0; dst[row0 + g + 8] = v1; }
}

// grads_kernel: every input gradient of one chunk (chunk form; the algebra
// is written out in oracle/memread.py:chunked_backward).
template <int P>
__global__ void __launch_bounds__(CTG) grads_kernel(
    int B, int T, int H, const float* __restrict__ keys, const float* __restrict__ values,
    const float* __restrict__ beta, const float* __restrict__ log_decay,
    const float* __restrict__ Y, const float* __restrict__ Z, const float* __restrict__ s_start,
    const float* __restrict__ c_start, const float* __restrict__ sbar,
    const float* __restrict__ cbar, const float* __restrict__ d_out,
    const float* __restrict__ d_var, float* __restrict__ dk, float* __restrict__ dv,
    float* __restrict__ dq, float* __restrict__ dbeta, float* __restrict__ dlog,
    float* __restrict__ floor_part) {
  constexpr int LP = P + 4, NTQ = P / 32;
  extern __shared__ __align__(16) float sh[];
  float* Ys = sh;                 // [64][LD]
  float* Zs = Ys + CH * LD;       // [64][LD]
  float* Ks = Zs + CH * LD;       // [64][LD]
  float* M1 = Ks + CH * LD;       // [64][LD]  W o GY
  float* M2 = M1 + CH * LD;       // [64][LD]  W o (OV - GZ)
  float* Sb = M2 + CH * LD;       // [64][LD]  dS_end, later S0
  float* Os = Sb + CH * LD;       // [64][LP]
  float* Vs = Os + CH * LP;       // [64][LP]
  float* Cb = Vs + CH * LP;       // [P][LD]   dC_end, later C0
  float* pre = Cb + P * LD;
  float* bet = pre + CH;
  float* ept = bet + CH;
  float* rowP = ept + CH;         // [4][64] column-quarter partials of sum_s dW W [t, s]
  float* colP = rowP + 4 * CH;    // [4][64] row-block partials of sum_t dW W [t, s]
  float* decP = colP + 4 * CH;    // [4][64] row-block partials of sum_t dW D [t, s]
  float* wbP = decP + 4 * CH;     // [4][64] column-quarter partials of dw_s
  float* exP = wbP + 4 * CH;      // [4][64] column-quarter partials of the per-token extra term
  float* red = exP + 4 * CH;      // [64 + 16] scratch
  float* wsv = red + CH + 16;     // [64] beta_s e^(P_L - P_s)
  const int Tp = (T + CH - 1) / CH * CH, nch = Tp / CH, nsub = Tp / SUB;
  const int ch = blockIdx.x % nch, bh = blockIdx.x / nch, b = bh / H, h = bh % H;
  const int t0 = ch * CH, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int row0 = 16 * (warp & 3), qt = warp >> 2, rb = warp & 3;
  const int c64 = 16 * qt, cP = qt * (P / 4);
  // S0 and C0 are needed only after phase 2: their loads start now, into
  // registers, so the DRAM round trip overlaps phases 1-2.
  constexpr int NS0 = KD * KD / 4 / CTG, NC0 = P * KD / 4 / CTG;
  float4 sv[NS0], cv[NC0];
  {
    const float* s0 = s_start + (size_t(bh) * nsub + ch * (CH / SUB)) * KD * KD;
    const float* c0 = c_start + (size_t(bh) * nch + ch) * P * KD;
#pragma unroll
    for (int i = 0; i < NS0; ++i) sv[i] = ld4(s0 + 4 * (tid + CTG * i));
#pragma unroll
    for (int i = 0; i < NC0; ++i) cv[i] = ld4(c0 + 4 * (tid + CTG * i));
  }
  load_block<CTG>(Ys, CH, Y + (size_t(bh) * Tp + t0) * KD, tid);
  load_block<CTG>(Zs, CH, Z + (size_t(bh) * Tp + t0) * KD, tid);
  load_tokens<KD, CTG>(Ks, LD, keys, b, T, H, h, t0, tid);
  load_tokens<P, CTG>(Os, LP, d_out, b, T, H, h, t0, tid);
  load_tokens<P, CTG>(Vs, LP, values, b, T, H, h, t0, tid);
  load_block<CTG>(Sb, KD, sbar + (size_t(bh) * nch + ch) * KD * KD, tid);
  load_block<CTG>(Cb, P, cbar + (size_t(bh) * nch + ch) * P * KD, tid);
  chunk_gates(tid, b, T, H, h, t0, beta, log_decay, pre, bet, ept);
  cp_wait();
  __syncthreads();
  const float pl = pre[CH - 1];
  if (tid < CH) wsv[tid] = bet[tid] * expf(pl - pre[tid]);  // read after the phase-1 barrier
  // Phase 1: GY, GZ, OV -> M1, M2 and the dW reductions.
  {
    float gy[2][4], gz[2][4], ov[2][4];
    zero(gy); zero(gz); zero(ov);
    gemm3_shared_b<KD, 2>(gy, gz, row0, c64, [&](int r, int k) { return Ys[r * LD + k]; },
                          [&](int r, int k) { return Zs[r * LD + k]; },
                          [&](int k, int s) { return Ks[s * LD + k]; });
    gemm3<P, 2>(ov, row0, c64, [&](int r, int k) { return Os[r * LP + k]; },
                [&](int k, int s) { return Vs[s * LP + k]; });
    float r0 = 0.f, r1 = 0.f, cw[2][2], cd[2][2];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) cw[nt][0] = cw[nt][1] = cd[nt][0] = cd[nt][1] = 0.f;
    each<2>(row0, c64, [&](int t, int s, int nt, int e) {
      const bool on = s <= t;
      const float dec = on ? expf(pre[t] - pre[s]) : 0.f;
      const float w = dec * bet[s];
      const float diff = ov[nt][e] - gz[nt][e];
      M1[t * LD + s] = w * gy[nt][e];
      M2[t * LD + s] = w * diff;
      const float dw = on ? gy[nt][e] * diff : 0.f;
      if (e < 2) r0 = fmaf(dw, w, r0); else r1 = fmaf(dw, w, r1);
      cw[nt][e & 1] = fmaf(dw, w, cw[nt][e & 1]);
      cd[nt][e & 1] = fmaf(dw, dec, cd[nt][e & 1]);
    });
    row_reduce_store(r0, r1, rowP + qt * CH, row0);
    // Column partials: reduce over the 8 row groups g of this warp.
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        float a = cw[nt][e], d = cd[nt][e];
#pragma unroll
        for (int o = 4; o < 32; o <<= 1) {
          a += __shfl_xor_sync(0xffffffffu, a, o);
          d += __shfl_xor_sync(0xffffffffu, d, o);
        }
        if (lane < 4) {
          const int s = c64 + 8 * nt + 2 * lane + e;
          colP[rb * CH + s] = a;
          decP[rb * CH + s] = d;
        }
      }
  }
  __syncthreads();
  // Phase 2: dK and dV (rows s) and dw_s.
  {
    float acc[2][4], tks[2][4], tkc[2][4], accv[NTQ][4], ck[NTQ][4];
    zero(acc); zero(tks); zero(tkc); zero(accv); zero(ck);
    // M1^T with -Z (dK) and with dO (dV); K with Sbar + Sbar^T (dK) and
    // with Cbar^T (dV): each shared operand split once.
    gemm3_shared_a<CH, 2, NTQ>(acc, accv, row0, c64, cP, [&](int s, int t) { return M1[t * LD + s]; },
                               [&](int t, int d) { return -Zs[t * LD + d]; },
                               [&](int t, int p) { return Os[t * LP + p]; });
    gemm3<CH, 2>(acc, row0, c64, [&](int s, int t) { return M2[t * LD + s]; },
                 [&](int t, int d) { return Ys[t * LD + d]; });
    gemm3_shared_a<KD, 2, NTQ>(tks, ck, row0, c64, cP, [&](int s, int e) { return Ks[s * LD + e]; },
                               [&](int e, int d) { return Sb[e * LD + d] + Sb[d * LD + e]; },
                               [&](int d, int p) { return Cb[p * LD + d]; });
    gemm3<P, 2>(tkc, row0, c64, [&](int s, int p) { return Vs[s * LP + p]; },
                [&](int p, int d) { return Cb[p * LD + d]; });
    float w0 = 0.f, w1 = 0.f;
    each<2>(row0, c64, [&](int s, int d, int nt, int e) {
      const float part = 0.5f * Ks[s * LD + d] * tks[nt][e];
      if (e < 2) w0 += part; else w1 += part;
      const int t = t0 + s;
      if (t < T) {
        const float ws = wsv[s];
        dk[((size_t(b) * T + t) * H + h) * KD + d] = fmaf(ws, tks[nt][e] + tkc[nt][e], acc[nt][e]);
      }
    });
    each<NTQ>(row0, cP, [&](int s, int p, int nt, int e) {
      const float part = Vs[s * LP + p] * ck[nt][e];
      if (e < 2) w0 += part; else w1 += part;
      const int t = t0 + s;
      if (t < T) {
        const float ws = wsv[s];
        dv[((size_t(b) * T + t) * H + h) * P + p] = fmaf(ws, ck[nt][e], accv[nt][e]);
      }
    });
    row_reduce_store(w0, w1, wbP + qt * CH, row0);
  }
  __syncthreads();
  // <dS_end, S0> + <dC_end, C0>, then S0 and C0 replace them in the tiles.
  {
    // Each thread reads its own float4 slots of Sb / Cb, then overwrites the
    // same slots with S0 / C0 (no other thread touches them in between).
    // (sv, cv were loaded at kernel entry.)
    constexpr int NS = KD * KD / 4 / CTG, NC = P * KD / 4 / CTG;
    float part = 0.f;
#pragma unroll
    for (int i = 0; i < NS; ++i) {
      const int idx = tid + CTG * i;
      float* slot = Sb + (idx / 16) * LD + 4 * (idx % 16);
      const float4 e = ld4(slot);
      part = fmaf(e.x, sv[i].x, fmaf(e.y, sv[i].y, fmaf(e.z, sv[i].z, fmaf(e.w, sv[i].w, part))));
      st4(slot, sv[i]);
    }
#pragma unroll
    for (int i = 0; i < NC; ++i) {
      const int idx = tid + CTG * i;
      float* slot = Cb + (idx / 16) * LD + 4 * (idx % 16);
      const float4 e = ld4(slot);
      part = fmaf(e.x, cv[i].x, fmaf(e.y, cv[i].y, fmaf(e.z, cv[i].z, fmaf(e.w, cv[i].w, part))));
      st4(slot, cv[i]);
    }
    part = warp_sum(part);
    if (lane == 0) red[CH + warp] = part;
  }
  __syncthreads();
  // Phase 3: extra_t = e^(P_t) (-z_t . (S0 y_t) + dO_t . (C0 y_t)).
  {
    float sy[2][4], cy[NTQ][4];
    zero(sy); zero(cy);
    gemm3_shared_a<KD, 2, NTQ>(sy, cy, row0, c64, cP, [&](int t, int k) { return Ys[t * LD + k]; },
                               [&](int k, int d) { return Sb[d * LD + k]; },
                               [&](int k, int p) { return Cb[p * LD + k]; });
    float v0 = 0.f, v1 = 0.f;
    each<2>(row0, c64, [&](int t, int d, int nt, int e) {
      const float part = -Zs[t * LD + d] * sy[nt][e];
      if (e < 2) v0 += part; else v1 += part;
    });
    each<NTQ>(row0, cP, [&](int t, int p, int nt, int e) {
      const float part = Os[t * LP + p] * cy[nt][e];
      if (e < 2) v0 += part; else v1 += part;
    });
    row_reduce_store(v0, v1, exP + qt * CH, row0);
  }
  __syncthreads();
  // Per-token scalars: dbeta, dP -> reverse cumsum -> dlog_decay.
  if (tid < CH) {
    const int s = tid;
    const float tail = expf(pl - pre[s]);
    const float ws = bet[s] * tail;
    const float wbar = wbP[s] + wbP[CH + s] + wbP[2 * CH + s] + wbP[3 * CH + s];
    const float colsum = colP[s] + colP[CH + s] + colP[2 * CH + s] + colP[3 * CH + s];
    const float decsum = decP[s] + decP[CH + s] + decP[2 * CH + s] + decP[3 * CH + s];
    red[s] = (rowP[s] + rowP[CH + s] + rowP[2 * CH + s] + rowP[3 * CH + s]) - colsum - wbar * ws +
             ept[s] * (exP[s] + exP[CH + s] + exP[2 * CH + s] + exP[3 * CH + s]);
    const int t = t0 + s;
    if (t < T) dbeta[(size_t(b) * T + t) * H + h] = decsum + wbar * tail;
    colP[s] = wbar * ws;  // reuse: dw_s w_s for the chunk-end term
  }
  __syncthreads();
  if (tid < 32) {
    float last = colP[tid] + colP[32 + tid];
    last = warp_sum(last);
    float dot_end = 0.f;
#pragma unroll
    for (int w = 0; w < CTG / 32; ++w) dot_end += red[CH + w];
    const float extra_last = last + ept[CH - 1] * dot_end;
    // reverse inclusive cumsum over 64 entries in two halves
    const float hi = red[63 - tid] + (tid == 0 ? extra_last : 0.f);
    const float shi = warp_inclusive_scan(hi, tid);
    const float tot_hi = __shfl_sync(0xffffffffu, shi, 31);
    const float slo = warp_inclusive_scan(red[31 - tid], tid) + tot_hi;
    const int thi = t0 + 63 - tid, tlo = t0 + 31 - tid;
    if (thi < T) dlog[(size_t(b) * T + thi) * H + h] = shi;
    if (tlo < T) dlog[(size_t(b) * T + tlo) * H + h] = slo;
  }
  // dq = z + dvar y ; floor partial = -sum_t z o y
  for (int idx = tid; idx < CH * KD; idx += CTG) {
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


// d_floor[c] = sum over rows of part[row][c], c < H*64. A block of 32 warps
// owns 32 columns (lane = column: coalesced rows); warp w sums rows w, w + 32,
// ... with eight loads in flight, and the 32 warp sums combine in a fixed
// order (deterministic).
__global__ void __launch_bounds__(1024) floor_reduce_kernel(int rows, int H, const float* __restrict__ part,
                                                            float* __restrict__ d_floor) {
  __shared__ float ws[32][33];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, c = blockIdx.x * 32 + lane;
  const int cols = H * KD;
  float s = 0.f;
  if (c < cols) {
    int r = warp;
    for (; r + 7 * 32 < rows; r += 8 * 32) {
      float a[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) a[j] = part[size_t(r + 32 * j) * cols + c];
#pragma unroll
      for (int j = 0; j < 8; ++j) s += a[j];
    }
    for (; r < rows; r += 32) s += part[size_t(r) * cols + c];
  }
  ws[warp][lane] = s;
  __syncthreads();
  if (warp == 0 && c < cols) {
    float t = 0.f;
#pragma unroll
    for (int w = 0; w < 32; ++w) t += ws[w][lane];
    d_floor[c] = t;
  }
}

template <int P>
size_t output_smem() { return (2 * CH * LD + CH * (P + 4) + P * LD + 3 * CH) * sizeof(float); }
template <int P>
size_t rhs_smem() { return (CH * LD + 2 * CH * (P + 4) + P * LD + 3 * CH) * sizeof(float); }
template <int P>
size_t carry_smem() { return (2 * CH * LD + CH * (P + 4) + 3 * CH) * sizeof(float); }
template <int P>
size_t grads_smem() { return (6 * CH * LD + 2 * CH * (P + 4) + P * LD + 25 * CH + 16) * sizeof(float); }

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
  const int ssm = int(sizeof(TileSmem));
  cudaFuncSetAttribute(solve_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, ssm);
  solve_kernel<<<warps, 32, ssm, st>>>(z.B, z.T, z.H, keys, queries, beta, log_decay, floor_, Ss, Lst, Y,
                                            var);
  const size_t osm = output_smem<P>();
  cudaFuncSetAttribute(output_kernel<P>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(osm));
  output_kernel<P><<<bh * z.nch, CT, osm, st>>>(z.B, z.T, z.H, keys, values, beta, log_decay, Y, Cs, out);
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
  rhs_kernel<P><<<bh * z.nch, CT, rsm, st>>>(z.B, z.T, z.H, keys, values, queries, beta, log_decay, Cs,
                                              d_out, d_var, G);
  const int warps = bh * z.nsub;
  const int ssm = int(sizeof(TileSmem) * WARPS);
  cudaFuncSetAttribute(zsolve_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, ssm);
  zsolve_kernel<<<(warps + WARPS - 1) / WARPS, 32 * WARPS, ssm, st>>>(z.B, z.T, z.H, Lst, G, Zb);
  const size_t csm = carry_smem<P>();
  cudaFuncSetAttribute(carry_kernel<P>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(csm));
  carry_kernel<P><<<bh, CT, csm, st>>>(z.B, z.T, z.H, beta, log_decay, Y, Zb, d_out, d_sfin, d_cfin, sb,
                                        cb, d_init_s, d_init_c);
  const size_t gsm = grads_smem<P>();
  cudaFuncSetAttribute(grads_kernel<P>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(gsm));
  grads_kernel<P><<<bh * z.nch, CTG, gsm, st>>>(z.B, z.T, z.H, keys, values, beta, log_decay, Y, Zb, Ss,
                                                Cs, sb, cb, d_out, d_var, dk, dv, dq, dbeta, dlog, fl);
  floor_reduce_kernel<<<(z.H * KD + 31) / 32, 1024, 0, st>>>(z.B * z.nch, z.H, fl, dfloor);
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
  if (!all_aligned16(keys, values, queries, init_s, init_c, out, s_fin, c_fin, static_cast<const float*>(resid)))
    return M4_ERR_ALIGN;
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
  if (!all_aligned16(keys, values, queries, d_out, d_sfin, d_cfin, dk, dv, dq, d_init_s, d_init_c,
                     static_cast<const float*>(resid), static_cast<const float*>(work)))
    return M4_ERR_ALIGN;
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

extern "C" int m4_memread_decode(const M4MemDims* d, const float* evidence, const float* cross,
                                 const float* key, const float* value, const float* query,
                                 const float* beta, const float* log_decay, const float* floor_,
                                 float* output, float* variance, float* evidence_out,
                                 float* cross_out, void* stream) {
  int st = mem::check(d);
  if (st) return st;
  if (!evidence || !cross || !key || !value || !query || !beta || !log_decay || !floor_ || !output ||
      !variance || !evidence_out || !cross_out)
    return M4_ERR_NULL;
  if (!all_aligned16(key, query)) return M4_ERR_ALIGN;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int bh = d->batch * d->heads;
  const int smem = int(sizeof(mem::DecodeSmem) * mem::WARPS);
  const int grid = (bh + mem::WARPS - 1) / mem::WARPS;
  if (d->value_dim == 64) {
    cudaFuncSetAttribute(mem::decode_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    mem::decode_kernel<64><<<grid, 32 * mem::WARPS, smem, s>>>(d->batch, d->heads, evidence, cross, key, value,
                                                               query, beta, log_decay, floor_, output, variance,
                                                               evidence_out, cross_out);
  } else {
    cudaFuncSetAttribute(mem::decode_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    mem::decode_kernel<128><<<grid, 32 * mem::WARPS, smem, s>>>(d->batch, d->heads, evidence, cross, key, value,
                                                                query, beta, log_decay, floor_, output, variance,
                                                                evidence_out, cross_out);
  }
  return launch_status();
}

extern "C" size_t m4_spd_solve_factor_bytes(int count, int dim) {
  if (count < 0 || dim <= 0 || dim > mem::KD) return 0;
  return size_t(count) * mem::LSTRIDE * sizeof(float);
}

extern "C" int m4_spd_solve_fwd(int count, int dim, const float* precision, const float* rhs,
                                float* solution, void* factor, size_t factor_bytes, void* stream) {
  if (count < 0 || dim <= 0) return M4_ERR_DIMS;
  if (dim > mem::KD) return M4_ERR_UNSUPPORTED;
  if (count == 0) return M4_OK;
  if (!precision || !rhs || !solution || !factor) return M4_ERR_NULL;
  if (!all_aligned16(static_cast<const float*>(factor))) return M4_ERR_ALIGN;
  if (factor_bytes < m4_spd_solve_factor_bytes(count, dim)) return M4_ERR_WORKSPACE;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int smem = int(sizeof(mem::SpdSmem) * mem::WARPS);
  cudaFuncSetAttribute(mem::spd_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  mem::spd_fwd_kernel<<<(count + mem::WARPS - 1) / mem::WARPS, 32 * mem::WARPS, smem, s>>>(
      count, dim, precision, rhs, solution, static_cast<float*>(factor));
  return launch_status();
}

extern "C" int m4_spd_solve_bwd(int count, int dim, const void* factor, size_t factor_bytes,
                                const float* solution, const float* d_solution, float* d_precision,
                                float* d_rhs, void* stream) {
  if (count < 0 || dim <= 0) return M4_ERR_DIMS;
  if (dim > mem::KD) return M4_ERR_UNSUPPORTED;
  if (count == 0) return M4_OK;
  if (!factor || !solution || !d_solution || !d_precision || !d_rhs) return M4_ERR_NULL;
  if (!all_aligned16(static_cast<const float*>(factor))) return M4_ERR_ALIGN;
  if (factor_bytes < m4_spd_solve_factor_bytes(count, dim)) return M4_ERR_WORKSPACE;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int smem = int(sizeof(mem::SpdSmem) * mem::WARPS);
  cudaFuncSetAttribute(mem::spd_bwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  mem::spd_bwd_kernel<<<(count + mem::WARPS - 1) / mem::WARPS, 32 * mem::WARPS, smem, s>>>(
      count, dim, static_cast<const float*>(factor), solution, d_solution, d_precision, d_rhs);
  return launch_status();
}
