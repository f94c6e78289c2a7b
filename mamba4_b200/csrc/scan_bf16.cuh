// Chunk-parallel bf16 Mamba-3 scan (forward and backward), sm_100a.
//
// Same recurrence, rounding points and outputs as the sequential kernels in
// scan.cu, reorganised so every (batch, head, chunk) is its own CTA:
//
// forward   phase_kernel    phase at every chunk start (prefix over chunks)
//           update_kernel   per chunk: U_n = K^T rd(V o scale o tail) and the
//                           chunk decay, U_n written into the `starts` slot
//           state_kernel    per (b, h): S_0 = 0, S_(n+1) = d_n S_n + U_n, in
//                           place (starts[n] <- S_n), final state
//           output_kernel   per chunk: y = rd(rd((Q K^T) o W) V + e^p Q rd(S_n))
// backward  dstart_kernel   per chunk: D_n = Q^T rd(dY o e^p) (into `carries`)
//           carry_kernel    per (b, h), reverse: carries[n] <- cotangent of the
//                           chunk-end state E_n; E_(n-1) = D_n + d_n E_n
//           grads_kernel    per chunk: every gradient given S_n and E_n
//           later_kernel    phase-gradient carry over chunks
// Chunk products: bf16 tiles in shared memory, ldmatrix fragments, m16n8k16
// tensor-core MMAs with fp32 accumulation.
#pragma once

namespace m4 {
namespace scan2 {

using bf16 = __nv_bfloat16;
constexpr int C = 64;        // chunk
constexpr int N = 64;        // state dim
constexpr int P = 64;        // head dim
constexpr int TS = 72;       // bf16 tile stride (144 B rows: ldmatrix conflict-free)
constexpr int FS = 68;       // fp32 tile stride
constexpr int CTH = 128;     // threads per chunk CTA (4 warps x 16 rows)

M4_DEV uint32_t smem_u32(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

M4_DEV void ldsm_x4(uint32_t (&r)[4], const bf16* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}

M4_DEV void ldsm_x4_t(uint32_t (&r)[4], const bf16* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}

M4_DEV void mma_bf16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// acc[nt][e] += sum_k A[row0 + g + 8(e>>1)][k] B[k][col0 + 8nt + 2c + (e&1)]
// (g = lane/4, c = lane%4) over K (multiple of 16), NT (even) n-tiles.
// A is row-major [m][k] (AT = false) or stored transposed [k][m] (AT = true);
// B is [n][k] (BT = false) or [k][n] (BT = true). Strides in elements.
template <int K, int NT, bool AT, bool BT>
M4_DEV void mma_tile(float (&acc)[NT][4], const bf16* A, int row0, const bf16* B, int col0) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int k0 = 0; k0 < K; k0 += 16) {
    uint32_t a[4];
    if constexpr (!AT)
      ldsm_x4(a, A + (row0 + (lane & 15)) * TS + k0 + 8 * (lane >> 4));
    else
      ldsm_x4_t(a, A + (k0 + (lane & 7) + 8 * (lane >> 4)) * TS + row0 + 8 * ((lane >> 3) & 1));
#pragma unroll
    for (int nt = 0; nt < NT; nt += 2) {
      uint32_t b[4];
      if constexpr (!BT)
        ldsm_x4(b, B + (col0 + nt * 8 + (lane & 7) + 8 * (lane >> 4)) * TS + k0 + 8 * ((lane >> 3) & 1));
      else
        ldsm_x4_t(b, B + (k0 + (lane & 7) + 8 * ((lane >> 3) & 1)) * TS + col0 + nt * 8 + 8 * (lane >> 4));
      mma_bf16(acc[nt], a, b[0], b[1]);
      mma_bf16(acc[nt + 1], a, b[2], b[3]);
    }
  }
}

template <int NT>
M4_DEV void zero(float (&acc)[NT][4]) {
#pragma unroll
  for (int i = 0; i < NT; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
}

// f(row, col, nt, e) over a warp's accumulator tile.
template <int NT, class F>
M4_DEV void each(int row0, int col0, F f) {
  const int lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int e = 0; e < 4; ++e) f(row0 + g + 8 * (e >> 1), col0 + 8 * nt + 2 * c + (e & 1), nt, e);
}

// Store a warp's accumulator tile, transformed by f(row, col, value), as bf16.
template <int NT, class F>
M4_DEV void store_bf16(bf16* T, int row0, int col0, const float (&acc)[NT][4], F f) {
  const int lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int r = row0 + g + 8 * h, col = col0 + 8 * nt + 2 * c;
      const __nv_bfloat162 v = __floats2bfloat162_rn(f(r, col, acc[nt][2 * h]), f(r, col + 1, acc[nt][2 * h + 1]));
      *reinterpret_cast<__nv_bfloat162*>(T + r * TS + col) = v;
    }
}

struct Dims {
  int B, T, H, A, nch;
  bool per_head;
};

// Per-token scalars of one chunk of (b, h) (threads 0..63 + warp 0 prefix).
struct Rows {
  float p[C], gam[C], scl[C], tail[C], dt[C], ept[C];
};

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
      next = dt[j] * (1.f - 1.f / (1.f + expf(-trap_logits[j])));
    }
    r.dt[tid] = dtv;
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
  if (tid < C) {
    r.tail[tid] = expf(r.p[C - 1] - r.p[tid]);
    r.ept[tid] = expf(r.p[tid]);
  }
}

M4_DEV float rate_at(const Dims& d, const float* angles, int b, int h, int t, int i) {
  return d.per_head ? angles[((size_t(b) * d.T + t) * d.H + h) * d.A + i]
                    : angles[(size_t(b) * d.T + t) * d.A + i];
}

// theta[t][i] = phase0[i] + sum_{s<=t} rate_s[i] dt_s within the chunk.
M4_DEV void chunk_theta(const Dims& d, int b, int h, int t0, const float* angles, const Rows& r,
                        const float* phase0, float* theta) {
  const int tid = threadIdx.x;
  if (tid < d.A) {
    float acc = phase0[tid];
    for (int tt = 0; tt < C; ++tt) {
      const int t = t0 + tt;
      const float rate = t < d.T ? rate_at(d, angles, b, h, t, tid) : 0.f;
      acc = fmaf(rate, r.dt[tt], acc);
      theta[tt * 33 + tid] = acc;
    }
  }
}

// Rotated, rounded queries/keys of a chunk as bf16 tiles. With `Qf`, also
// keeps cos/sin for the backward.
M4_DEV void build_qk(const Dims& d, int b, int h, int t0, const bf16* cq, const bf16* bk, const float* qb,
                     const float* kb, const float* theta, bf16* Qs, bf16* Ks, float* cosv, float* sinv) {
  for (int idx = threadIdx.x; idx < C * (N / 2); idx += CTH) {
    const int tt = idx / (N / 2), i = idx % (N / 2), t = t0 + tt;
    const int n0 = 2 * i;
    float c0 = 0.f, c1 = 0.f, b0 = 0.f, b1 = 0.f;
    if (t < d.T) {
      const size_t base = d.per_head ? ((size_t(b) * d.T + t) * d.H + h) * N : (size_t(b) * d.T + t) * N;
      const __nv_bfloat162 cc = *reinterpret_cast<const __nv_bfloat162*>(cq + base + n0);
      const __nv_bfloat162 bb = *reinterpret_cast<const __nv_bfloat162*>(bk + base + n0);
      c0 = __low2float(cc); c1 = __high2float(cc);
      b0 = __low2float(bb); b1 = __high2float(bb);
    }
    const float q0 = round_to<bf16>(c0 + (qb ? qb[h * N + n0] : 0.f));
    const float q1 = round_to<bf16>(c1 + (qb ? qb[h * N + n0 + 1] : 0.f));
    const float k0 = round_to<bf16>(b0 + (kb ? kb[h * N + n0] : 0.f));
    const float k1 = round_to<bf16>(b1 + (kb ? kb[h * N + n0 + 1] : 0.f));
    float cs = 1.f, sn = 0.f;
    if (i < d.A) sincosf(theta[tt * 33 + i], &sn, &cs);
    if (Qs) *reinterpret_cast<__nv_bfloat162*>(Qs + tt * TS + n0) = __floats2bfloat162_rn(q0 * cs - q1 * sn, q1 * cs + q0 * sn);
    if (Ks) *reinterpret_cast<__nv_bfloat162*>(Ks + tt * TS + n0) = __floats2bfloat162_rn(k0 * cs - k1 * sn, k1 * cs + k0 * sn);
    if (cosv) { cosv[tt * 33 + i] = cs; sinv[tt * 33 + i] = sn; }
  }
}

// Copy a [64 tokens][64] slice of a [B,T,H*64] bf16 tensor into a tile.
M4_DEV void load_tile(const Dims& d, int b, int h, int t0, const bf16* src, bf16* T) {
  for (int idx = threadIdx.x; idx < C * P / 8; idx += CTH) {
    const int tt = idx / (P / 8), c8 = idx % (P / 8), t = t0 + tt;
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (t < d.T) v = *reinterpret_cast<const uint4*>(src + (size_t(b) * d.T + t) * d.H * P + h * P + 8 * c8);
    *reinterpret_cast<uint4*>(T + tt * TS + 8 * c8) = v;
  }
}

// Load a [64][64] fp32 block (row-major) into a bf16 tile with RN rounding.
M4_DEV void load_state_bf16(const float* src, bf16* T) {
  for (int idx = threadIdx.x; idx < N * P / 4; idx += CTH) {
    const float4 v = ld4(src + 4 * idx);
    const int r = idx / (P / 4), c4 = idx % (P / 4);
    *reinterpret_cast<__nv_bfloat162*>(T + r * TS + 4 * c4) = __floats2bfloat162_rn(v.x, v.y);
    *reinterpret_cast<__nv_bfloat162*>(T + r * TS + 4 * c4 + 2) = __floats2bfloat162_rn(v.z, v.w);
  }
}

// ---------------------------------------------------------------------------
// Forward
// ---------------------------------------------------------------------------

// Phase at every chunk start: phases[b,h,n,i] = sum_{t < 64n} rate_t[i] dt_t.
__global__ void __launch_bounds__(256) phase_kernel(Dims d, const float* __restrict__ dt,
                                                    const float* __restrict__ angles,
                                                    float* __restrict__ phases) {
  extern __shared__ float loc[];  // [nch][32]
  const int bh = blockIdx.x, b = bh / d.H, h = bh % d.H;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int n = warp; n < d.nch; n += 8) {
    float acc = 0.f;
    if (lane < d.A) {
      for (int tt = 0; tt < C; ++tt) {
        const int t = n * C + tt;
        if (t >= d.T) break;
        acc = fmaf(rate_at(d, angles, b, h, t, lane), dt[(size_t(b) * d.T + t) * d.H + h], acc);
      }
    }
    loc[n * 32 + lane] = acc;
  }
  __syncthreads();
  if (warp == 0) {
    float acc = 0.f;
    for (int n = 0; n < d.nch; ++n) {
      phases[(size_t(bh) * d.nch + n) * 32 + lane] = acc;
      acc += loc[n * 32 + lane];
    }
  }
}

struct UpdSmem {
  bf16 Ks[C * TS];
  bf16 Vw[C * TS];
  float theta[C * 33];
  float scratch[C];
  Rows r;
};

// U_n = K^T rd(V o scale o tail) into starts[n]; deltas[n] = e^(p_L).
__global__ void __launch_bounds__(CTH) update_kernel(
    Dims d, const bf16* __restrict__ bk, const bf16* __restrict__ x, const float* __restrict__ adt,
    const float* __restrict__ dt, const float* __restrict__ trap_logits, const float* __restrict__ angles,
    const float* __restrict__ kb, const float* __restrict__ phases, float* __restrict__ starts,
    float* __restrict__ deltas) {
  extern __shared__ __align__(16) unsigned char raw[];
  UpdSmem& s = *reinterpret_cast<UpdSmem*>(raw);
  const int n = blockIdx.x % d.nch, bh = blockIdx.x / d.nch, b = bh / d.H, h = bh % d.H;
  const int t0 = n * C, warp = threadIdx.x >> 5;
  chunk_rows(d, b, h, t0, adt, dt, trap_logits, s.r, s.scratch);
  __syncthreads();
  chunk_theta(d, b, h, t0, angles, s.r, phases + (size_t(bh) * d.nch + n) * 32, s.theta);
  __syncthreads();
  build_qk(d, b, h, t0, bk, bk, nullptr, kb, s.theta, nullptr, s.Ks, nullptr, nullptr);
  for (int idx = threadIdx.x; idx < C * P / 2; idx += CTH) {
    const int tt = idx / (P / 2), c2 = idx % (P / 2), t = t0 + tt;
    float v0 = 0.f, v1 = 0.f;
    if (t < d.T) {
      const __nv_bfloat162 v = *reinterpret_cast<const __nv_bfloat162*>(x + (size_t(b) * d.T + t) * d.H * P + h * P + 2 * c2);
      const float src = s.r.scl[tt] * s.r.tail[tt];
      v0 = __low2float(v) * src;
      v1 = __high2float(v) * src;
    }
    *reinterpret_cast<__nv_bfloat162*>(s.Vw + tt * TS + 2 * c2) = __floats2bfloat162_rn(v0, v1);
  }
  __syncthreads();
  float acc[8][4];
  zero(acc);
  mma_tile<C, 8, true, true>(acc, s.Ks, warp * 16, s.Vw, 0);  // rows n (A = K^T), cols p
  float* dst = starts + (size_t(bh) * d.nch + n) * N * P;
  each<8>(warp * 16, 0, [&](int r, int c, int nt, int e) { dst[r * P + c] = acc[nt][e]; });
  if (threadIdx.x == 0) deltas[size_t(bh) * d.nch + n] = expf(s.r.p[C - 1]);
}

// In place over chunks: starts[n] <- S_n with S_0 = 0, S_(n+1) = d_n S_n + U_n.
__global__ void __launch_bounds__(256) state_kernel(Dims d, float* __restrict__ starts,
                                                    const float* __restrict__ deltas,
                                                    float* __restrict__ final_state) {
  const int bh = blockIdx.x;
  float4 s[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) s[k] = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int n = 0; n < d.nch; ++n) {
    float* slot = starts + (size_t(bh) * d.nch + n) * N * P;
    const float dl = deltas[size_t(bh) * d.nch + n];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int i = 4 * (threadIdx.x + 256 * k);
      const float4 u = ld4(slot + i);
      st4(slot + i, s[k]);
      s[k] = make_float4(fmaf(dl, s[k].x, u.x), fmaf(dl, s[k].y, u.y), fmaf(dl, s[k].z, u.z),
                         fmaf(dl, s[k].w, u.w));
    }
  }
#pragma unroll
  for (int k = 0; k < 4; ++k) st4(final_state + size_t(bh) * N * P + 4 * (threadIdx.x + 256 * k), s[k]);
}

struct OutSmem {
  bf16 Qs[C * TS];
  bf16 Ks[C * TS];
  bf16 Vs[C * TS];
  bf16 Ms[C * TS];
  bf16 Ss[N * TS];
  float theta[C * 33];
  float scratch[C];
  Rows r;
};

// y = rd(rd((Q K^T) o W) V + e^p Q rd(S_n)).
__global__ void __launch_bounds__(CTH) output_kernel(
    Dims d, const bf16* __restrict__ cq, const bf16* __restrict__ bk, const bf16* __restrict__ x,
    const float* __restrict__ adt, const float* __restrict__ dt, const float* __restrict__ trap_logits,
    const float* __restrict__ angles, const float* __restrict__ qb, const float* __restrict__ kb,
    const float* __restrict__ phases, const float* __restrict__ starts, bf16* __restrict__ y) {
  extern __shared__ __align__(16) unsigned char raw[];
  OutSmem& s = *reinterpret_cast<OutSmem*>(raw);
  const int n = blockIdx.x % d.nch, bh = blockIdx.x / d.nch, b = bh / d.H, h = bh % d.H;
  const int t0 = n * C, warp = threadIdx.x >> 5, row0 = warp * 16;
  chunk_rows(d, b, h, t0, adt, dt, trap_logits, s.r, s.scratch);
  __syncthreads();
  chunk_theta(d, b, h, t0, angles, s.r, phases + (size_t(bh) * d.nch + n) * 32, s.theta);
  __syncthreads();
  build_qk(d, b, h, t0, cq, bk, qb, kb, s.theta, s.Qs, s.Ks, nullptr, nullptr);
  load_tile(d, b, h, t0, x, s.Vs);
  load_state_bf16(starts + (size_t(bh) * d.nch + n) * N * P, s.Ss);
  __syncthreads();
  {
    float acc[8][4];
    zero(acc);
    mma_tile<N, 8, false, false>(acc, s.Qs, row0, s.Ks, 0);  // Q K^T: B = K as [s][n]
    store_bf16<8>(s.Ms, row0, 0, acc, [&](int t, int sidx, float v) {
      float w = 0.f;
      if (sidx < t) w = expf(s.r.p[t] - s.r.p[sidx]) * s.r.scl[sidx];
      else if (sidx == t) w = s.r.gam[t];
      return v * w;
    });
  }
  __syncwarp();  // each warp reads back only its own 16 rows of Ms
  float acc[8][4], inh[8][4];
  zero(acc);
  zero(inh);
  mma_tile<C, 8, false, true>(acc, s.Ms, row0, s.Vs, 0);   // mixed V: B = V as [s][p]
  mma_tile<N, 8, false, true>(inh, s.Qs, row0, s.Ss, 0);   // Q S: B = S as [n][p]
  const int lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
#pragma unroll
  for (int hf = 0; hf < 2; ++hf) {
    const int tt = row0 + g + 8 * hf, t = t0 + tt;
    if (t >= d.T) continue;
    const float e = s.r.ept[tt];
    bf16* yrow = y + (size_t(b) * d.T + t) * d.H * P + h * P;
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      const int col = nt * 8 + 2 * c;
      *reinterpret_cast<__nv_bfloat162*>(yrow + col) = __floats2bfloat162_rn(
          fmaf(e, inh[nt][2 * hf], acc[nt][2 * hf]), fmaf(e, inh[nt][2 * hf + 1], acc[nt][2 * hf + 1]));
    }
  }
}

// ---------------------------------------------------------------------------
// Backward
// ---------------------------------------------------------------------------
struct DsSmem {
  bf16 Qs[C * TS];
  bf16 Ds[C * TS];
  float theta[C * 33];
  float scratch[C];
  Rows r;
};

// D_n = Q^T rd(dY o e^p) into carries[n].
__global__ void __launch_bounds__(CTH) dstart_kernel(
    Dims d, const bf16* __restrict__ cq, const bf16* __restrict__ dy, const float* __restrict__ adt,
    const float* __restrict__ dt, const float* __restrict__ trap_logits, const float* __restrict__ angles,
    const float* __restrict__ qb, const float* __restrict__ phases, float* __restrict__ carries) {
  extern __shared__ __align__(16) unsigned char raw[];
  DsSmem& s = *reinterpret_cast<DsSmem*>(raw);
  const int n = blockIdx.x % d.nch, bh = blockIdx.x / d.nch, b = bh / d.H, h = bh % d.H;
  const int t0 = n * C, warp = threadIdx.x >> 5;
  chunk_rows(d, b, h, t0, adt, dt, trap_logits, s.r, s.scratch);
  __syncthreads();
  chunk_theta(d, b, h, t0, angles, s.r, phases + (size_t(bh) * d.nch + n) * 32, s.theta);
  __syncthreads();
  build_qk(d, b, h, t0, cq, cq, qb, nullptr, s.theta, s.Qs, nullptr, nullptr, nullptr);
  for (int idx = threadIdx.x; idx < C * P / 2; idx += CTH) {
    const int tt = idx / (P / 2), c2 = idx % (P / 2), t = t0 + tt;
    float v0 = 0.f, v1 = 0.f;
    if (t < d.T) {
      const __nv_bfloat162 v = *reinterpret_cast<const __nv_bfloat162*>(dy + (size_t(b) * d.T + t) * d.H * P + h * P + 2 * c2);
      v0 = __low2float(v) * s.r.ept[tt];
      v1 = __high2float(v) * s.r.ept[tt];
    }
    *reinterpret_cast<__nv_bfloat162*>(s.Ds + tt * TS + 2 * c2) = __floats2bfloat162_rn(v0, v1);
  }
  __syncthreads();
  float acc[8][4];
  zero(acc);
  mma_tile<C, 8, true, true>(acc, s.Qs, warp * 16, s.Ds, 0);  // Q^T D: rows n, cols p
  float* dst = carries + (size_t(bh) * d.nch + n) * N * P;
  each<8>(warp * 16, 0, [&](int r, int c, int nt, int e) { dst[r * P + c] = acc[nt][e]; });
}

// Reverse over chunks, in place: carries[n] <- E_n (cotangent of chunk n's end
// state); E_(nch-1) = d_final, E_(n-1) = D_n + d_n E_n.
__global__ void __launch_bounds__(256) carry_kernel(Dims d, float* __restrict__ carries,
                                                    const float* __restrict__ deltas,
                                                    const float* __restrict__ d_final) {
  const int bh = blockIdx.x;
  float4 e[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int i = 4 * (threadIdx.x + 256 * k);
    e[k] = d_final ? ld4(d_final + size_t(bh) * N * P + i) : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  for (int n = d.nch - 1; n >= 0; --n) {
    float* slot = carries + (size_t(bh) * d.nch + n) * N * P;
    const float dl = deltas[size_t(bh) * d.nch + n];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int i = 4 * (threadIdx.x + 256 * k);
      const float4 dn = ld4(slot + i);
      st4(slot + i, e[k]);
      e[k] = make_float4(fmaf(dl, e[k].x, dn.x), fmaf(dl, e[k].y, dn.y), fmaf(dl, e[k].z, dn.z),
                         fmaf(dl, e[k].w, dn.w));
    }
  }
}

struct GradOut {
  float* dq;      // [B,T,H,N] pre-rotation query gradient per head
  float* dk;      // [B,T,H,N]
  float* drate;   // [B,T,H,A] angle-rate gradient, without the later-chunk carry
  float* dgam;    // [B,T,H]
  float* dscl;    // [B,T,H]
  float* dlog;    // [B,T,H]
  float* ddtp;    // [B,T,H] dt gradient through the phase, without the carry
  float* dth;     // [B,H,nch,32] per-chunk totals of the pair phase gradient
  float* dqb;     // [B,H,nch,N] per-chunk bias partials
  float* dkb;     // [B,H,nch,N]
};

struct GradSmem {
  bf16 Qs[C * TS];
  bf16 Ks[C * TS];
  bf16 Vs[C * TS];
  bf16 Dy[C * TS];
  bf16 Ms[C * TS];   // rd(scores o W), rd(d_mixed o W), then rd(dY o e^p)
  bf16 Es[N * TS];   // rd(E_n)
  bf16 Ss[N * TS];   // rd(S_n)
  float Sc[C * FS];  // scores (fp32)
  float Dm[C * FS];  // d_mixed (fp32)
  float theta[C * 33];
  float vec[8 * C];
  float bq[4 * N];   // per-warp bias partials
  float bk[4 * N];
  float scratch[C];
  Rows r;
};

__global__ void __launch_bounds__(CTH) grads_kernel(
    Dims d, const bf16* __restrict__ cq, const bf16* __restrict__ bk, const bf16* __restrict__ x,
    const float* __restrict__ adt, const float* __restrict__ dt, const float* __restrict__ trap_logits,
    const float* __restrict__ angles, const float* __restrict__ qb, const float* __restrict__ kb,
    const float* __restrict__ phases, const float* __restrict__ starts, const float* __restrict__ carries,
    const bf16* __restrict__ dy, bf16* __restrict__ dx, GradOut o) {
  extern __shared__ __align__(16) unsigned char raw[];
  GradSmem& s = *reinterpret_cast<GradSmem*>(raw);
  const int n = blockIdx.x % d.nch, bh = blockIdx.x / d.nch, b = bh / d.H, h = bh % d.H;
  const int t0 = n * C, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, row0 = warp * 16;
  const int g = lane >> 2, cc = lane & 3;
  chunk_rows(d, b, h, t0, adt, dt, trap_logits, s.r, s.scratch);
  __syncthreads();
  chunk_theta(d, b, h, t0, angles, s.r, phases + (size_t(bh) * d.nch + n) * 32, s.theta);
  __syncthreads();
  build_qk(d, b, h, t0, cq, bk, qb, kb, s.theta, s.Qs, s.Ks, nullptr, nullptr);
  load_tile(d, b, h, t0, x, s.Vs);
  load_tile(d, b, h, t0, dy, s.Dy);
  load_state_bf16(starts + (size_t(bh) * d.nch + n) * N * P, s.Ss);
  load_state_bf16(carries + (size_t(bh) * d.nch + n) * N * P, s.Es);
  __syncthreads();
  auto wgt = [&](int t, int sidx) -> float {
    if (sidx < t) return expf(s.r.p[t] - s.r.p[sidx]) * s.r.scl[sidx];
    return sidx == t ? s.r.gam[t] : 0.f;
  };
  // Scores and d_mixed (rows t, cols s), fp32.
  {
    float acc[8][4];
    zero(acc);
    mma_tile<N, 8, false, false>(acc, s.Qs, row0, s.Ks, 0);
    each<8>(row0, 0, [&](int r, int c, int nt, int e) { s.Sc[r * FS + c] = acc[nt][e]; });
    zero(acc);
    mma_tile<P, 8, false, false>(acc, s.Dy, row0, s.Vs, 0);
    each<8>(row0, 0, [&](int r, int c, int nt, int e) { s.Dm[r * FS + c] = acc[nt][e]; });
  }
  __syncthreads();
  for (int idx = tid; idx < C * C / 2; idx += CTH) {
    const int t = idx / (C / 2), s2 = 2 * (idx % (C / 2));
    *reinterpret_cast<__nv_bfloat162*>(s.Ms + t * TS + s2) =
        __floats2bfloat162_rn(s.Sc[t * FS + s2] * wgt(t, s2), s.Sc[t * FS + s2 + 1] * wgt(t, s2 + 1));
  }
  __syncthreads();
  // dV = rd(Sc o W)^T dY + src o (K rd(E)) -> dx.
  {
    float acc[8][4], ve[8][4];
    zero(acc);
    zero(ve);
    mma_tile<C, 8, true, true>(acc, s.Ms, row0, s.Dy, 0);
    mma_tile<N, 8, false, true>(ve, s.Ks, row0, s.Es, 0);
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
      const int sr = row0 + g + 8 * hf, t = t0 + sr;
      if (t >= d.T) continue;
      const float src = s.r.scl[sr] * s.r.tail[sr];
      bf16* row = dx + (size_t(b) * d.T + t) * d.H * P + h * P;
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        const int col = nt * 8 + 2 * cc;
        *reinterpret_cast<__nv_bfloat162*>(row + col) = __floats2bfloat162_rn(
            fmaf(src, ve[nt][2 * hf], acc[nt][2 * hf]), fmaf(src, ve[nt][2 * hf + 1], acc[nt][2 * hf + 1]));
      }
    }
  }
  __syncthreads();
  for (int idx = tid; idx < C * C / 2; idx += CTH) {
    const int t = idx / (C / 2), s2 = 2 * (idx % (C / 2));
    *reinterpret_cast<__nv_bfloat162*>(s.Ms + t * TS + s2) =
        __floats2bfloat162_rn(s.Dm[t * FS + s2] * wgt(t, s2), s.Dm[t * FS + s2 + 1] * wgt(t, s2 + 1));
  }
  __syncthreads();
  // dQ, dK (rows t / s, cols n) in registers.
  float gq[8][4], gk[8][4];
  zero(gq);
  zero(gk);
  mma_tile<C, 8, false, true>(gq, s.Ms, row0, s.Ks, 0);   // rd(Dm o W) K
  mma_tile<C, 8, true, true>(gk, s.Ms, row0, s.Qs, 0);    // rd(Dm o W)^T Q
  __syncthreads();  // Ms is rewritten below
  for (int idx = tid; idx < C * P / 2; idx += CTH) {
    const int tt = idx / (P / 2), c2 = idx % (P / 2);
    const __nv_bfloat162 v = *reinterpret_cast<const __nv_bfloat162*>(s.Dy + tt * TS + 2 * c2);
    *reinterpret_cast<__nv_bfloat162*>(s.Ms + tt * TS + 2 * c2) =
        __floats2bfloat162_rn(__low2float(v) * s.r.ept[tt], __high2float(v) * s.r.ept[tt]);
  }
  __syncthreads();
  mma_tile<P, 8, false, false>(gq, s.Ms, row0, s.Ss, 0);  // rd(dY e^p) rd(S)^T
  float dsrc[2] = {0.f, 0.f}, inh_dot[2] = {0.f, 0.f};
  {
    float ve[8][4];
    zero(ve);
    mma_tile<P, 8, false, false>(ve, s.Vs, row0, s.Es, 0);  // V rd(E)^T (rows s, cols n)
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
      const int sr = row0 + g + 8 * hf;
      const float src = s.r.scl[sr] * s.r.tail[sr];
#pragma unroll
      for (int nt = 0; nt < 8; ++nt)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const float kv = __bfloat162float(s.Ks[sr * TS + nt * 8 + 2 * cc + e]);
          dsrc[hf] = fmaf(kv, ve[nt][2 * hf + e], dsrc[hf]);
          gk[nt][2 * hf + e] = fmaf(src, ve[nt][2 * hf + e], gk[nt][2 * hf + e]);
        }
    }
    zero(ve);
    mma_tile<N, 8, false, true>(ve, s.Qs, row0, s.Ss, 0);  // Q rd(S) (rows t, cols p)
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
      const int t = row0 + g + 8 * hf;
#pragma unroll
      for (int nt = 0; nt < 8; ++nt)
#pragma unroll
        for (int e = 0; e < 2; ++e)
          inh_dot[hf] = fmaf(__bfloat162float(s.Dy[t * TS + nt * 8 + 2 * cc + e]), ve[nt][2 * hf + e], inh_dot[hf]);
    }
  }
#pragma unroll
  for (int hf = 0; hf < 2; ++hf) {
    float a = dsrc[hf], v = inh_dot[hf];
    a += __shfl_xor_sync(0xffffffffu, a, 1);
    a += __shfl_xor_sync(0xffffffffu, a, 2);
    v += __shfl_xor_sync(0xffffffffu, v, 1);
    v += __shfl_xor_sync(0xffffffffu, v, 2);
    if (cc == 0) {
      const int r = row0 + g + 8 * hf;
      s.vec[0 * C + r] = a;
      s.vec[1 * C + r] = v * s.r.ept[r];
    }
  }
  // <E, S> for the chunk-end decay (fp32 values).
  {
    const float* Sg = starts + (size_t(bh) * d.nch + n) * N * P;
    const float* Eg = carries + (size_t(bh) * d.nch + n) * N * P;
    float part = 0.f;
    for (int i = tid; i < N * P / 4; i += CTH) {
      const float4 a4 = ld4(Sg + 4 * i), e4 = ld4(Eg + 4 * i);
      part = fmaf(a4.x, e4.x, fmaf(a4.y, e4.y, fmaf(a4.z, e4.z, fmaf(a4.w, e4.w, part))));
    }
    part = warp_sum(part);
    if (lane == 0) s.scratch[warp] = part;
  }
  // Rotation backward in registers: the accumulators hold each pair (2i, 2i+1)
  // on one thread. Pre-rotation gradients to workspace, the pair phase
  // gradient into theta (same element, read then written by this thread),
  // bias partials per column.
  {
    float sq[8][2], sk[8][2];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) sq[nt][0] = sq[nt][1] = sk[nt][0] = sk[nt][1] = 0.f;
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
      const int tt = row0 + g + 8 * hf, t = t0 + tt;
      const bool live = t < d.T;
      const size_t base = d.per_head ? ((size_t(b) * d.T + t) * d.H + h) * N : (size_t(b) * d.T + t) * N;
      const size_t ob = ((size_t(b) * d.T + t) * d.H + h) * N;
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        const int i = 4 * nt + cc, n0 = 2 * i;
        float cs = 1.f, sn = 0.f;
        if (i < d.A) sincosf(s.theta[tt * 33 + i], &sn, &cs);
        const float gq0 = gq[nt][2 * hf], gq1 = gq[nt][2 * hf + 1];
        const float gk0 = gk[nt][2 * hf], gk1 = gk[nt][2 * hf + 1];
        const float pq0 = gq0 * cs + gq1 * sn, pq1 = gq1 * cs - gq0 * sn;
        const float pk0 = gk0 * cs + gk1 * sn, pk1 = gk1 * cs - gk0 * sn;
        float c0 = 0.f, c1 = 0.f, b0 = 0.f, b1 = 0.f;
        if (live) {
          const __nv_bfloat162 c2 = *reinterpret_cast<const __nv_bfloat162*>(cq + base + n0);
          const __nv_bfloat162 b2 = *reinterpret_cast<const __nv_bfloat162*>(bk + base + n0);
          c0 = __low2float(c2); c1 = __high2float(c2);
          b0 = __low2float(b2); b1 = __high2float(b2);
          *reinterpret_cast<float2*>(o.dq + ob + n0) = make_float2(pq0, pq1);
          *reinterpret_cast<float2*>(o.dk + ob + n0) = make_float2(pk0, pk1);
          sq[nt][0] += pq0; sq[nt][1] += pq1;
          sk[nt][0] += pk0; sk[nt][1] += pk1;
        }
        const float q0 = round_to<bf16>(c0 + (qb ? qb[h * N + n0] : 0.f));
        const float q1 = round_to<bf16>(c1 + (qb ? qb[h * N + n0 + 1] : 0.f));
        const float k0 = round_to<bf16>(b0 + (kb ? kb[h * N + n0] : 0.f));
        const float k1 = round_to<bf16>(b1 + (kb ? kb[h * N + n0 + 1] : 0.f));
        const float qr0 = q0 * cs - q1 * sn, qr1 = q1 * cs + q0 * sn;
        const float kr0 = k0 * cs - k1 * sn, kr1 = k1 * cs + k0 * sn;
        const float dth = gq0 * (-qr1) + gq1 * qr0 + gk0 * (-kr1) + gk1 * kr0;
        if (i < 32) s.theta[tt * 33 + i] = (i < d.A && live) ? dth : 0.f;
      }
    }
#pragma unroll
    for (int nt = 0; nt < 8; ++nt)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        float q = sq[nt][e], kk = sk[nt][e];
#pragma unroll
        for (int off = 4; off < 32; off <<= 1) {
          q += __shfl_xor_sync(0xffffffffu, q, off);
          kk += __shfl_xor_sync(0xffffffffu, kk, off);
        }
        if (g == 0) {
          s.bq[warp * N + nt * 8 + 2 * cc + e] = q;
          s.bk[warp * N + nt * 8 + 2 * cc + e] = kk;
        }
      }
  }
  __syncthreads();
  // Per-token scalar gradients from d_weights = Dm o Sc.
  if (tid < C) {
    const int t = tid;
    float rowoff = 0.f, coloff = 0.f, cdec = 0.f;
    for (int sidx = 0; sidx < t; ++sidx)
      rowoff = fmaf(s.Dm[t * FS + sidx] * s.Sc[t * FS + sidx], expf(s.r.p[t] - s.r.p[sidx]) * s.r.scl[sidx], rowoff);
    for (int u = t + 1; u < C; ++u) {
      const float dw = s.Dm[u * FS + t] * s.Sc[u * FS + t];
      const float dec = expf(s.r.p[u] - s.r.p[t]);
      coloff = fmaf(dw, dec * s.r.scl[t], coloff);
      cdec = fmaf(dw, dec, cdec);
    }
    const float flow = s.vec[0 * C + t] * s.r.scl[t] * s.r.tail[t];
    s.vec[2 * C + t] = rowoff - coloff - flow + s.vec[1 * C + t];
    s.vec[3 * C + t] = s.Dm[t * FS + t] * s.Sc[t * FS + t];
    s.vec[4 * C + t] = s.vec[0 * C + t] * s.r.tail[t] + cdec;
    s.vec[5 * C + t] = flow;
  } else if (tid < C + N) {
    const int nn = tid - C;
    o.dqb[(size_t(bh) * d.nch + n) * N + nn] = s.bq[nn] + s.bq[N + nn] + s.bq[2 * N + nn] + s.bq[3 * N + nn];
    o.dkb[(size_t(bh) * d.nch + n) * N + nn] = s.bk[nn] + s.bk[N + nn] + s.bk[2 * N + nn] + s.bk[3 * N + nn];
  }
  __syncthreads();
  if (tid < 32) {
    float fl = s.vec[5 * C + tid] + s.vec[5 * C + 32 + tid];
    fl = warp_sum(fl);
    const float end = expf(s.r.p[C - 1]);
    const float extra = fl + end * (s.scratch[0] + s.scratch[1] + s.scratch[2] + s.scratch[3]);
    const float hi = s.vec[2 * C + 63 - tid] + (tid == 0 ? extra : 0.f);
    const float shi = warp_inclusive_scan(hi, tid);
    const float tot = __shfl_sync(0xffffffffu, shi, 31);
    const float slo = warp_inclusive_scan(s.vec[2 * C + 31 - tid], tid) + tot;
    s.vec[6 * C + 63 - tid] = shi;
    s.vec[6 * C + 31 - tid] = slo;
  } else if (tid >= 64 && tid - 64 < d.A) {
    // Suffix sums of the pair phase gradient within the chunk (the carry from
    // later chunks is added by later_kernel).
    const int i = tid - 64;
    float acc = 0.f;
    for (int tt = C - 1; tt >= 0; --tt) {
      acc += s.theta[tt * 33 + i];
      s.theta[tt * 33 + i] = acc;
    }
    o.dth[(size_t(bh) * d.nch + n) * 32 + i] = acc;
  }
  __syncthreads();
  if (tid < C) {
    const int tt = tid, t = t0 + tt;
    if (t < d.T) {
      float ddt = 0.f;
      for (int i = 0; i < d.A; ++i) {
        const float inc = s.theta[tt * 33 + i];
        o.drate[((size_t(b) * d.T + t) * d.H + h) * d.A + i] = inc * s.r.dt[tt];
        ddt = fmaf(inc, rate_at(d, angles, b, h, t, i), ddt);
      }
      const size_t si = (size_t(b) * d.T + t) * d.H + h;
      o.ddtp[si] = ddt;
      o.dgam[si] = s.vec[3 * C + tt];
      o.dscl[si] = s.vec[4 * C + tt];
      o.dlog[si] = s.vec[6 * C + tt];
    }
  }
}

// Phase-gradient carry: later_n[i] = sum over chunks m > n of the chunk
// totals; adds later * dt to the rate gradients and later . rate to the dt
// gradient of every token of chunk n.
__global__ void __launch_bounds__(256) later_kernel(Dims d, const float* __restrict__ dt,
                                                    const float* __restrict__ angles,
                                                    const float* __restrict__ dth,
                                                    float* __restrict__ drate, float* __restrict__ ddtp) {
  extern __shared__ float later[];  // [nch][32]
  const int bh = blockIdx.x, b = bh / d.H, h = bh % d.H;
  if (threadIdx.x < 32) {
    float acc = 0.f;
    for (int n = d.nch - 1; n >= 0; --n) {
      later[n * 32 + threadIdx.x] = acc;
      acc += threadIdx.x < d.A ? dth[(size_t(bh) * d.nch + n) * 32 + threadIdx.x] : 0.f;
    }
  }
  __syncthreads();
  for (int t = threadIdx.x; t < d.T; t += blockDim.x) {
    const int n = t / C;
    const size_t si = (size_t(b) * d.T + t) * d.H + h;
    const float dtv = dt[si];
    float add = 0.f;
    for (int i = 0; i < d.A; ++i) {
      const float l = later[n * 32 + i];
      drate[si * d.A + i] += l * dtv;
      add = fmaf(l, rate_at(d, angles, b, h, t, i), add);
    }
    ddtp[si] += add;
  }
}

// Bias gradients: sum per-chunk partials over batch and chunks (fixed order).
__global__ void bias_kernel(Dims d, const float* __restrict__ dqb, const float* __restrict__ dkb,
                            float* __restrict__ d_qb, float* __restrict__ d_kb) {
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= d.H * N) return;
  const int h = idx / N, nn = idx % N;
  float sq = 0.f, sk = 0.f;
  for (int b = 0; b < d.B; ++b)
    for (int n = 0; n < d.nch; ++n) {
      const size_t o = ((size_t(b) * d.H + h) * d.nch + n) * N + nn;
      sq += dqb[o];
      sk += dkb[o];
    }
  if (d_qb) d_qb[idx] = sq;
  if (d_kb) d_kb[idx] = sk;
}

}  // namespace scan2
}  // namespace m4
