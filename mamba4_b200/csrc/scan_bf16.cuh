// bf16 Mamba-3 scan (forward and backward), sm_100a.
//
// Same recurrence, rounding points and outputs as the sequential kernels in
// scan.cu:
//
// forward   fused_fwd_kernel  one persistent CTA per (b, h) walks the chunks
//                             with the fp32 state in registers: TMA x tiles,
//                             prefetched (cp.async) gates/angles/C/B rows,
//                             tcgen05 chunk products, residuals S_n, phases
//                             and chunk decays for the backward
// backward  dstart_kernel   per chunk: D_n = Q^T rd(dY o e^p) (into `carries`)
//           carry_kernel    per (b, h), reverse: carries[n] <- cotangent of the
//                           chunk-end state E_n; E_(n-1) = D_n + d_n E_n
//           grads_kernel    per chunk: every gradient given S_n and E_n
//           later_kernel    phase-gradient carry over chunks
// Chunk products: tcgen05 (tensor memory accumulators, 128-byte-swizzled
// shared-memory operands, one issuing thread, mbarrier commits) in every
// kernel; fp32 accumulation everywhere.
// Every kernel is templated on NH, the number of 64-row halves of the state
// (N = 64 or 128): contractions over the state accumulate the halves' products
// in one accumulator, products with state-row outputs get one M = 64
// accumulator per half.
#pragma once

#include "tc05.cuh"

namespace m4 {
namespace scan2 {

using bf16 = __nv_bfloat16;
constexpr int C = 64;        // chunk
constexpr int P = 64;        // head dim
// State dim N = 64 NH (NH = 1 or 2 halves of 64 state rows): pairs NP = N / 2,
// [C][pairs] fp32 tables with row stride TW.
template <int NH> struct Geo {
  static constexpr int N = 64 * NH, NP = 32 * NH, TW = NP + 1;
};
constexpr int GW = 8;        // warps per chunk CTA (4 row blocks x 2 column halves)
static_assert(C == 64 && (C % (4 * GW)) == 0, "warp/token maps assume 64-token chunks");

// Element (r, c) of a 64-column bf16 tile in 128-byte swizzled rows (tcgen05
// descriptors and TMA, tc::sw).
template <bool BLK>
M4_DEV bf16* at(bf16* T, int r, int c) {
  static_assert(BLK, "every tile is swizzled");
  return reinterpret_cast<bf16*>(reinterpret_cast<unsigned char*>(T) + tc::sw(r, c));
}

// D (tensor memory) = A B (+ D when `accumulate`) over K = 64 on the tensor
// cores (tcgen05, 4 MMAs of K = 16), issued by one thread. A is M x K, B is
// K x N, each a swizzled tile read K-major (K along its contiguous columns)
// or MN-major (K along its rows).
M4_DEV void tc_product(uint32_t d, const bf16* A, bool a_mn, const bf16* B, bool b_mn, bool accumulate = false) {
  const uint32_t id = tc::idesc_bf16(64, 64, a_mn ? 1 : 0, b_mn ? 1 : 0);
  const unsigned char* a = reinterpret_cast<const unsigned char*>(A);
  const unsigned char* b = reinterpret_cast<const unsigned char*>(B);
#pragma unroll 1  // one issuing thread: code size matters more than the loop overhead
  for (int ks = 0; ks < 4; ++ks) {
    const uint64_t ad = a_mn ? tc::sdesc_sw128(a + 2048 * ks, 8192, 1024) : tc::sdesc_sw128(a + 32 * ks, 16, 1024);
    const uint64_t bd = b_mn ? tc::sdesc_sw128(b + 2048 * ks, 8192, 1024) : tc::sdesc_sw128(b + 32 * ks, 16, 1024);
    tc::mma_bf16(d, ad, bd, id, accumulate || ks > 0);
  }
}

// Shared-memory base of a tcgen05 kernel, rounded up to the 1024-byte swizzle
// atom (launches reserve 1024 extra bytes).
M4_DEV unsigned char* align1024(unsigned char* p) {
  return reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~uintptr_t(1023));
}

// Everyone: wait (bounded) for the tensor-core work committed to `bar` in
// phase `phase`; a timeout raises the device error flag.
M4_DEV bool tc_wait(uint64_t* bar, uint32_t phase) {
  const bool ok = tc::mbar_wait(bar, phase, tc::WAIT_LIMIT);
  if (!ok && (threadIdx.x & 31) == 0) tc::flag_timeout();
  tc::fence_after();
  return ok;
}

// Shared writes -> visible to the tensor cores, then a CTA barrier.
M4_DEV void tc_publish() {
  tc::fence_proxy_async();
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
}

// Accumulator row this thread reads (lanes 0..15 of each warp) and its
// tensor-memory lane base; warps w and w + 4 share a lane quarter.
M4_DEV uint32_t tmem_lane_base(uint32_t tm) { return tm + (uint32_t(32 * ((threadIdx.x >> 5) & 3)) << 16); }

// 16 rows x 32 columns of an M = 64 accumulator (the warp's lane quarter from
// `taddr`) over all 32 threads: v[4 k + 2 hh + j] is row t / 4 + 8 hh,
// column 8 k + 2 (t % 4) + j (tcgen05.ld 16x256b, four repetitions).
M4_DEV void ld_16x256b_x4(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile("tcgen05.ld.sync.aligned.16x256b.x4.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
                 "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
               : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// Reduce-scatter over the lanes that differ in bits LO .. LO + L - 1 of the
// lane index: V values per lane in, V >> L sums per lane out, in place at
// v[0 .. V >> L). Level l halves the array; the lane with that bit clear keeps
// the lower half. A lane ends with the sums of the values
// [(V >> L) j, (V >> L) (j + 1)) of its group, j = its bits LO .. LO + L - 1
// read as a binary number with bit LO + L - 1 most significant.
template <int V, int L, int LO>
M4_DEV void reduce_scatter(float (&v)[V], int lane) {
  static_assert((V >> L) << L == V, "V must be divisible by 2^L");
#pragma unroll
  for (int l = L - 1; l >= 0; --l) {
    const int bit = LO + l;
    const int width = V >> (L - 1 - l);  // live values before this level
    const bool up = (lane >> bit) & 1;
#pragma unroll
    for (int i = 0; i < width / 2; ++i) {
      const float keep = up ? v[width / 2 + i] : v[i];
      const float give = up ? v[i] : v[width / 2 + i];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, give, 1 << bit);
    }
  }
}

struct Dims {
  int B, T, H, A, nch;
  bool per_head;
};

// Per-token scalars of one chunk of (b, h) (threads 0..63 + warp 0 prefix).
struct Rows {
  float p[C], gam[C], scl[C], tail[C], dt[C], ept[C];
  float seg[8 * 64];  // per-segment totals of the in-chunk scans (one segment per warp, NP pairs)
};

M4_DEV float rate_at(const Dims& d, const float* angles, int b, int h, int t, int i) {
  return d.per_head ? angles[((size_t(b) * d.T + t) * d.H + h) * d.A + i]
                    : angles[(size_t(b) * d.T + t) * d.A + i];
}

M4_DEV uint32_t ld_u32(const bf16* p) { return *reinterpret_cast<const uint32_t*>(p); }
M4_DEV float lo_f(uint32_t v) { return __uint_as_float(v << 16); }
M4_DEV float hi_f(uint32_t v) { return __uint_as_float(v & 0xffff0000u); }

// ---------------------------------------------------------------------------
// Forward
// ---------------------------------------------------------------------------

// CTAs per (b, h) in the chunk-carry pass of the backward (1,024 floats each).
template <int NH> constexpr int sparts() { return 4 * NH; }

// ---------------------------------------------------------------------------
// Persistent forward: one CTA (8 warps) per (batch, head) walks the chunks in
// order with the fp32 state carried in registers (the inter-chunk carry of
// the reference's sequential chunk grid, flashmamba.py:589-660), so no state
// pass, phase pass or per-chunk CTA setup is left. Per chunk:
//   TMA of the next chunk's x tile into the other buffer (zero fill past T);
//   gates, in-chunk phases and the rotated, rounded Q / K tiles (rotated in
//   place: the raw c / b rows land in the swizzled tiles);
//   rd(S_n) as a tile, S_n and the chunk-start phase to the residuals;
//   tcgen05 commit 1: Q K^T, Q rd(S_n), K^T rd(V o scale o tail); once it
//   completes the Q / K tiles take the next chunk's raw rows (cp.async);
//   masked scores rd((Q K^T) o W) -> tile; tcgen05 commit 2: scores V;
//   S_(n+1) = e^(p_L) S_n + K^T rd(V o scale o tail) in registers;
//   y = rd(scores V + e^p Q rd(S_n)).
// Accumulators are read with the 16-lane tensor-memory loads (16x256b), which
// spread the 16 rows an M = 64 accumulator keeps in a warp's lane quarter
// over all 32 threads: thread t of warp w holds rows 16 (w % 4) + t / 4 and
// + 8, columns 32 (w / 4) + 8 k + 2 (t % 4) + {0, 1} (k < 4) of each product
// and of the state.
// Residuals written: starts[n] = S_n, phases[n], deltas[n] = e^(p_L).
// ---------------------------------------------------------------------------
template <int NH>
struct FusedSmem {
  static constexpr int NP = Geo<NH>::NP;
  bf16 Qs[NH][C * 64]; // 128-byte-swizzled 64-column tiles on 1024-byte boundaries
  bf16 Ks[NH][C * 64];
  bf16 Vs[2][C * P];   // x tiles (TMA, double buffered)
  bf16 Vw[C * P];      // rd(V o scale o tail)
  bf16 Ms[C * C];      // masked scores
  bf16 Ss[NH][64 * P]; // rd(S_n), 64 state rows per tile
  float scratch[C];
  float phase[NP];     // phase at the current chunk start
  float adt[C];        // the current chunk's gates (dt and trap with token t0 + 64)
  float dt[C + 4];
  float trap[C + 4];
  Rows r;
  uint64_t bar;        // tensor-core commits (two per chunk)
  uint64_t bar_x[2];   // TMA of the x tiles
  uint32_t tmem;
  // Followed by three [C][fwd_ta(A)] fp32 tables: angle rates, cos and sin
  // of the pair phases (only the A rotated pairs).
};
// Row stride of the forward's angle tables.
__host__ __device__ constexpr int fwd_ta(int A) { return A > 0 ? A : 1; }
template <int NH>
constexpr size_t fused_smem_bytes(int A) { return sizeof(FusedSmem<NH>) + 3 * size_t(C) * fwd_ta(A) * sizeof(float); }

// Where a kernel stages one chunk's raw inputs (cp.async, tokens past T as
// zeros): c / b rows (bf16, row-major with `stride` elements, or in 128-byte
// swizzled 64-column tiles when SW), angle rates [token][NP], adt [64],
// dt / trap [65] (token t0 + 64 too, for the trapezoid's next-token term).
// Either c or b may be null.
struct StageRef {
  bf16* c;
  bf16* b;
  int stride;
  float* ang;
  float* adt;
  float* dt;
  float* trap;
};

// Element (r, c) of a staged [C][N] row block: row-major with `stride`, or
// column c of the swizzled 64-column tile c / 64.
template <bool SW>
M4_DEV bf16* stage_row(bf16* base, int stride, int r, int c) {
  if constexpr (SW) return at<true>(base + (c >> 6) * (C * 64), r, c & 63);
  else return base + r * stride + c;
}

// Start copying chunk n's raw inputs (one commit group per thread); the
// angle rates land at in.ang[token * as + pair].
template <bool SW, int NH>
M4_DEV void stage_prefetch(const Dims& d, int b, int h, int n, const bf16* cq, const bf16* bk, const float* adt,
                           const float* dt, const float* trap_logits, const float* angles, const StageRef& in,
                           int as = Geo<NH>::NP) {
  constexpr int N = Geo<NH>::N, PIECES = N / 8;
  const int tid = threadIdx.x, t0 = n * C;
#pragma unroll
  for (int k = 0; k < 4 * NH; ++k) {  // 2 tiles x 64 rows x N/8 16-byte pieces over 256 threads
    const int idx = tid + k * GW * 32, which = idx / (C * PIECES), rr = (idx / PIECES) % C;
    const int c8 = 8 * (idx % PIECES);
    bf16* dst = which ? in.b : in.c;
    if (dst == nullptr) continue;
    const int t = t0 + rr;
    const bool live = t < d.T;
    const size_t base = d.per_head ? ((size_t(b) * d.T + t) * d.H + h) * N : (size_t(b) * d.T + t) * N;
    const bf16* src = which ? bk : cq;
    cp16(reinterpret_cast<float*>(stage_row<SW>(dst, in.stride, rr, c8)),
         reinterpret_cast<const float*>(live ? src + base + c8 : src), live);
  }
  for (int idx = tid; idx < C * d.A; idx += GW * 32) {
    const int tt = idx / d.A, i = idx % d.A, t = t0 + tt;
    const bool live = t < d.T;
    const size_t o = d.per_head ? ((size_t(b) * d.T + t) * d.H + h) * d.A + i : (size_t(b) * d.T + t) * d.A + i;
    cp4(&in.ang[tt * as + i], live ? angles + o : angles, live);
  }
  if (tid < 3 * (C + 1)) {
    const int which = tid / (C + 1), tt = tid % (C + 1), t = t0 + tt;
    const bool live = t < d.T && (which > 0 || tt < C);
    const size_t o = (size_t(b) * d.T + t) * d.H + h;
    const float* src = which == 0 ? adt : which == 1 ? dt : trap_logits;
    float* dst = which == 0 ? in.adt : which == 1 ? in.dt : in.trap;
    if (which > 0 || tt < C) cp4(dst + tt, live ? src + o : src, live);
  }
  cp_commit();
}

// chunk_rows from the stage.
M4_DEV void stage_rows(const Dims& d, int t0, const StageRef& in, Rows& r, float* scratch) {
  const int tid = threadIdx.x;
  if (tid < C) {
    const bool live = t0 + tid < d.T;
    const float dtv = in.dt[tid];
    const float tr = live ? 1.f / (1.f + expf(-in.trap[tid])) : 0.f;
    const float next = t0 + tid + 1 < d.T ? in.dt[tid + 1] * (1.f - 1.f / (1.f + expf(-in.trap[tid + 1]))) : 0.f;
    r.dt[tid] = dtv;
    r.gam[tid] = dtv * tr;
    r.scl[tid] = dtv * tr + next;
    scratch[tid] = in.adt[tid];
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

// chunk_theta from the stage (same segment scheme): lanes over the pairs
// lane + 32 q (q < NH). Angle rates at in.ang[token * as + pair]; cos / sin
// tables [token][tw] (pairs past the angle count hold 1 / 0 where tw has
// room for them).
template <int NH>
M4_DEV void stage_theta(const Dims& d, const StageRef& in, Rows& r, const float* phase0, float* cosv, float* sinv,
                        int as = Geo<NH>::NP, int tw = Geo<NH>::TW) {
  constexpr int SEG = C / GW, NP = Geo<NH>::NP;
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
#pragma unroll
  for (int q = 0; q < NH; ++q) {
    const int i = lane + 32 * q;
    float acc = 0.f;
    if (i < d.A) {
#pragma unroll
      for (int j = 0; j < SEG; ++j) {
        const int tt = SEG * w + j;
        acc = fmaf(in.ang[tt * as + i], r.dt[tt], acc);
        cosv[tt * tw + i] = acc;
      }
    }
    r.seg[w * NP + i] = acc;
  }
  __syncthreads();
#pragma unroll 1  // one inline copy of sincosf
  for (int q = 0; q < NH; ++q) {
    const int i = lane + 32 * q;
    float off = 0.f;
    if (i < d.A) {
      off = phase0[i];
      for (int v = 0; v < w; ++v) off += r.seg[v * NP + i];
    }
    if (i < tw) {
#pragma unroll 1
      for (int j = 0; j < SEG; ++j) {
        const int e = (SEG * w + j) * tw + i;
        float cs = 1.f, sn = 0.f;
        if (i < d.A) sincosf(cosv[e] + off, &sn, &cs);
        cosv[e] = cs;
        sinv[e] = sn;
      }
    }
  }
}

// Destination element (r, c) of a rotated Q / K tile: 128-byte-swizzled
// 64-column tiles (DST_SW) or row-major rows of `stride` elements.
template <bool SW>
M4_DEV bf16* qk_at(bf16* T, int stride, int r, int c) {
  if constexpr (SW) return at<true>(T + (c >> 6) * (C * 64), r, c & 63);
  else return T + r * stride + c;
}

// build_qk from the stage: rotated, rounded Q / K tiles (either may be null);
// a stage may be the destination tile itself (each thread reads and writes
// the same pair); with both swizzled it must be (in place). Lane l handles the pairs l + 32 q (columns 2 l + 64 q);
// pairs from `na` on are not rotated (cos / sin tables [token][tw]).
template <bool SRC_SW, bool DST_SW, int NH>
M4_DEV void stage_qk(int h, const StageRef& in, const float* qb, const float* kb, const float* cosv,
                     const float* sinv, bf16* Qs, bf16* Ks, int dst_stride = 0, int na = Geo<NH>::NP,
                     int tw = Geo<NH>::TW) {
  constexpr int PER = C / GW, N = Geo<NH>::N;
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  // In place in swizzled tiles: the rows this thread visits (w + 8 k) share
  // row % 8 = w, so the swizzled byte offset is one per-thread constant plus
  // 1024 k.
  const uint32_t swz = uint32_t(w * 128 + (((lane >> 2) ^ w) << 4) + 4 * (lane & 3));
#pragma unroll
  for (int q = 0; q < NH; ++q) {
    const int n0 = 2 * lane + 64 * q, i = lane + 32 * q;
    const float qb0 = qb ? qb[h * N + n0] : 0.f, qb1 = qb ? qb[h * N + n0 + 1] : 0.f;
    const float kb0 = kb ? kb[h * N + n0] : 0.f, kb1 = kb ? kb[h * N + n0 + 1] : 0.f;
#pragma unroll
    for (int k = 0; k < PER; ++k) {
      const int tt = w + GW * k;
      const float cs = i < na ? cosv[tt * tw + i] : 1.f, sn = i < na ? sinv[tt * tw + i] : 0.f;
      if constexpr (SRC_SW && DST_SW) {
        const uint32_t off = swz + 1024u * k;
        if (Qs) {
          uint32_t* pq = reinterpret_cast<uint32_t*>(reinterpret_cast<unsigned char*>(Qs + q * C * 64) + off);
          const uint32_t cr = *pq;
          const float q0 = round_to<bf16>(lo_f(cr) + qb0), q1 = round_to<bf16>(hi_f(cr) + qb1);
          *reinterpret_cast<__nv_bfloat162*>(pq) = __floats2bfloat162_rn(q0 * cs - q1 * sn, q1 * cs + q0 * sn);
        }
        if (Ks) {
          uint32_t* pk = reinterpret_cast<uint32_t*>(reinterpret_cast<unsigned char*>(Ks + q * C * 64) + off);
          const uint32_t br = *pk;
          const float k0 = round_to<bf16>(lo_f(br) + kb0), k1 = round_to<bf16>(hi_f(br) + kb1);
          *reinterpret_cast<__nv_bfloat162*>(pk) = __floats2bfloat162_rn(k0 * cs - k1 * sn, k1 * cs + k0 * sn);
        }
        continue;
      }
      if (Qs) {
        const uint32_t cr = ld_u32(stage_row<SRC_SW>(in.c, in.stride, tt, n0));
        const float q0 = round_to<bf16>(lo_f(cr) + qb0), q1 = round_to<bf16>(hi_f(cr) + qb1);
        *reinterpret_cast<__nv_bfloat162*>(qk_at<DST_SW>(Qs, dst_stride, tt, n0)) =
            __floats2bfloat162_rn(q0 * cs - q1 * sn, q1 * cs + q0 * sn);
      }
      if (Ks) {
        const uint32_t br = ld_u32(stage_row<SRC_SW>(in.b, in.stride, tt, n0));
        const float k0 = round_to<bf16>(lo_f(br) + kb0), k1 = round_to<bf16>(hi_f(br) + kb1);
        *reinterpret_cast<__nv_bfloat162*>(qk_at<DST_SW>(Ks, dst_stride, tt, n0)) =
            __floats2bfloat162_rn(k0 * cs - k1 * sn, k1 * cs + k0 * sn);
      }
    }
  }
}

template <int NH>
__global__ void __launch_bounds__(GW * 32, 2) fused_fwd_kernel(
    Dims d, const __grid_constant__ CUtensorMap tmap_x, const bf16* __restrict__ cq, const bf16* __restrict__ bk,
    const float* __restrict__ adt, const float* __restrict__ dt, const float* __restrict__ trap_logits,
    const float* __restrict__ angles, const float* __restrict__ qb, const float* __restrict__ kb,
    bf16* __restrict__ y, float* __restrict__ starts, float* __restrict__ phases, float* __restrict__ deltas,
    float* __restrict__ final_state) {
  constexpr int N = Geo<NH>::N, NP = Geo<NH>::NP;
  extern __shared__ __align__(128) unsigned char raw[];
  FusedSmem<NH>& s = *reinterpret_cast<FusedSmem<NH>*>(align1024(raw));
  const int ta = fwd_ta(d.A);
  float* angt = reinterpret_cast<float*>(&s + 1);
  float* cosv = angt + C * ta;
  float* sinv = cosv + C * ta;
  const int bh = blockIdx.x, b = bh / d.H, h = bh % d.H;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // Accumulator fragment of this thread: rows r0 + 8 hh, columns col0 + 8 k + cq + j.
  const int r0 = 16 * (warp & 3) + (lane >> 2), cq2 = 2 * (lane & 3), col0 = 32 * (warp >> 2);
  if (warp == 0) {
    tc::tmem_alloc(&s.tmem, 256);
    tc::tmem_relinquish();
  }
  if (tid == 0) {
    tc::mbar_init(&s.bar, 1);
    tc::mbar_init(&s.bar_x[0], 1);
    tc::mbar_init(&s.bar_x[1], 1);
  }
  if (tid < NP) s.phase[tid] = 0.f;
  __syncthreads();
  tc::fence_after();
  const uint32_t tm = s.tmem;
  const uint32_t tl = tmem_lane_base(tm);
  if (tid == 0) {
    tc::mbar_expect_tx(&s.bar_x[0], C * P * sizeof(bf16));
    tc::tma_load_3d(s.Vs[0], &tmap_x, h * P, 0, b, &s.bar_x[0]);
  }
  const StageRef in{s.Qs[0], s.Ks[0], 0, angt, s.adt, s.dt, s.trap};
  stage_prefetch<true, NH>(d, b, h, 0, cq, bk, adt, dt, trap_logits, angles, in, ta);
  // fp32 state S_n: rows 64 q + r0 + 8 hh, columns col0 + 8 k + cq2 + j at st[q][4 k + 2 hh + j]
  float st[NH][16];
#pragma unroll
  for (int q = 0; q < NH; ++q)
#pragma unroll
    for (int j = 0; j < 16; ++j) st[q][j] = 0.f;
  auto put_state = [&](float* dst) {
#pragma unroll
    for (int q = 0; q < NH; ++q)
#pragma unroll
      for (int k = 0; k < 4; ++k)
#pragma unroll
        for (int hh = 0; hh < 2; ++hh)
          *reinterpret_cast<float2*>(dst + (64 * q + r0 + 8 * hh) * P + col0 + 8 * k + cq2) =
              make_float2(st[q][4 * k + 2 * hh], st[q][4 * k + 2 * hh + 1]);
  };
  bool ok = true;
  for (int n = 0; n < d.nch; ++n) {
    const int t0 = n * C, buf = n & 1;
    if (tid == 0 && n + 1 < d.nch) {
      // The other buffer was last read by chunk n - 1's score product, which
      // completed before that chunk ended.
      tc::mbar_expect_tx(&s.bar_x[buf ^ 1], C * P * sizeof(bf16));
      tc::tma_load_3d(s.Vs[buf ^ 1], &tmap_x, h * P, t0 + C, b, &s.bar_x[buf ^ 1]);
    }
    cp_wait();
    __syncthreads();  // this chunk's stage has landed
    stage_rows(d, t0, in, s.r, s.scratch);
    __syncthreads();
    stage_theta<NH>(d, in, s.r, s.phase, cosv, sinv, ta, ta);
    __syncthreads();
    if (tid < NP) {
      float inc = 0.f;
#pragma unroll
      for (int w = 0; w < GW; ++w) inc += s.r.seg[w * NP + tid];
      phases[(size_t(bh) * d.nch + n) * NP + tid] = s.phase[tid];
      s.phase[tid] += tid < d.A ? inc : 0.f;
    }
    if (tid < C) s.scratch[tid] = s.r.scl[tid] * s.r.tail[tid];
    stage_qk<true, true, NH>(h, in, qb, kb, cosv, sinv, s.Qs[0], s.Ks[0], 0, d.A, ta);
    put_state(starts + (size_t(bh) * d.nch + n) * N * P);
#pragma unroll
    for (int q = 0; q < NH; ++q)
#pragma unroll
      for (int k = 0; k < 4; ++k)
#pragma unroll
        for (int hh = 0; hh < 2; ++hh)
          *reinterpret_cast<__nv_bfloat162*>(at<true>(s.Ss[q], r0 + 8 * hh, col0 + 8 * k + cq2)) =
              __floats2bfloat162_rn(st[q][4 * k + 2 * hh], st[q][4 * k + 2 * hh + 1]);
    __syncthreads();  // scratch (scale o tail) visible
    // rd(V o scale o tail) from the x tile once it has landed.
    if (!tc::mbar_wait(&s.bar_x[buf], (n >> 1) & 1, tc::WAIT_LIMIT)) {
      if (lane == 0) tc::flag_timeout();
      ok = false;
    }
    if (ok) {
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        const int idx = tid + k * GW * 32, rr = idx >> 3, c8 = 8 * (idx & 7);
        const uint4 v = *reinterpret_cast<const uint4*>(at<true>(s.Vs[buf], rr, c8));
        const float f = s.scratch[rr];
        const uint32_t* u = reinterpret_cast<const uint32_t*>(&v);
        uint4 o;
        uint32_t* w = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const __nv_bfloat162 x2 = __floats2bfloat162_rn(lo_f(u[q]) * f, hi_f(u[q]) * f);
          w[q] = *reinterpret_cast<const uint32_t*>(&x2);
        }
        *reinterpret_cast<uint4*>(at<true>(s.Vw, rr, c8)) = o;
      }
    }
    tc_publish();
    if (tid == 0 && ok) {
      // The state-dim contractions accumulate over the halves; the update
      // K^T rd(V o scale o tail) gets one accumulator per half (columns
      // 128 + 64 q).
#pragma unroll
      for (int q = 0; q < NH; ++q) tc_product(tm, s.Qs[q], false, s.Ks[q], false, q > 0);       // Q K^T
#pragma unroll
      for (int q = 0; q < NH; ++q) tc_product(tm + 64, s.Qs[q], false, s.Ss[q], true, q > 0);   // Q rd(S_n)
#pragma unroll
      for (int q = 0; q < NH; ++q) tc_product(tm + 128 + 64 * q, s.Ks[q], true, s.Vw, true);    // K^T rd(V w)
      tc::commit(&s.bar);
    }
    ok = ok && tc_wait(&s.bar, 0);
    // The Q / K tiles are free: the next chunk's raw rows land in them.
    if (n + 1 < d.nch) stage_prefetch<true, NH>(d, b, h, n + 1, cq, bk, adt, dt, trap_logits, angles, in, ta);
    if (ok) {
      float v[16];
      ld_16x256b_x4(tl + col0, v);
      tc::wait_ld();
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const int row = r0 + 8 * hh;
        const float pt = s.r.p[row];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          float m2[2];
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            const int sidx = col0 + 8 * k + cq2 + j;
            float w = 0.f;
            if (sidx < row) w = expf(pt - s.r.p[sidx]) * s.r.scl[sidx];
            else if (sidx == row) w = s.r.gam[row];
            m2[j] = v[4 * k + 2 * hh + j] * w;
          }
          *reinterpret_cast<__nv_bfloat162*>(at<true>(s.Ms, row, col0 + 8 * k + cq2)) =
              __floats2bfloat162_rn(m2[0], m2[1]);
        }
      }
    }
    tc_publish();
    if (tid == 0 && ok) {
      tc_product(tm, s.Ms, false, s.Vs[buf], true);   // scores V
      tc::commit(&s.bar);
    }
    if (ok) {
      // S_(n+1) = e^(p_L) S_n + U_n (the update finished with commit 1).
      const float dl = expf(s.r.p[C - 1]);
#pragma unroll
      for (int q = 0; q < NH; ++q) {
        float u[16];
        ld_16x256b_x4(tl + 128 + 64 * q + col0, u);
        tc::wait_ld();
#pragma unroll
        for (int e = 0; e < 16; ++e) st[q][e] = fmaf(dl, st[q][e], u[e]);
      }
      if (tid == 0) deltas[size_t(bh) * d.nch + n] = dl;
    }
    ok = ok && tc_wait(&s.bar, 1);
    if (ok) {
      float acc[16], inh[16];
      ld_16x256b_x4(tl + col0, acc);
      ld_16x256b_x4(tl + 64 + col0, inh);
      tc::wait_ld();
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const int row = r0 + 8 * hh, t = t0 + row;
        const float e = s.r.ept[row];
        if (t < d.T) {
          bf16* yrow = y + (size_t(b) * d.T + t) * d.H * P + h * P + col0 + cq2;
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const int i = 4 * k + 2 * hh;
            *reinterpret_cast<__nv_bfloat162*>(yrow + 8 * k) =
                __floats2bfloat162_rn(fmaf(e, inh[i], acc[i]), fmaf(e, inh[i + 1], acc[i + 1]));
          }
        }
      }
    }
    tc::fence_before();
    __syncthreads();  // tensor memory and every tile are free for the next chunk
    tc::fence_after();
  }
  put_state(final_state + size_t(bh) * N * P);
  // A TMA the loop no longer waits for cannot be in flight: the last chunk
  // issues none and every earlier one was awaited.
  tc::fence_before();
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tm, 256);
}

// ---------------------------------------------------------------------------
// Backward
// ---------------------------------------------------------------------------
template <int NH>
struct DsSmem {
  static constexpr int NP = Geo<NH>::NP;
  bf16 Qs[NH][C * 64];  // blocked tiles (tcgen05 operands)
  bf16 Ds[C * P];
  float scratch[C];
  float stg[3 * C + 8 + NP];  // staged gates and the chunk-start phase
  Rows r;
  uint64_t bar;
  uint32_t tmem;
  // Followed by two [C][fwd_ta(A)] fp32 tables: cos (the phases first) and
  // sin (the angle rates first) of the rotated pairs.
};
template <int NH>
constexpr size_t dstart_smem_bytes(int A) { return sizeof(DsSmem<NH>) + 2 * size_t(C) * fwd_ta(A) * sizeof(float); }

// D_n = Q^T rd(dY o e^p) into carries[n], on the tensor cores (tcgen05):
// one M = 64 product per half of the state rows.
template <int NH>
__global__ void __launch_bounds__(GW * 32) dstart_kernel(
    Dims d, const bf16* __restrict__ cq, const bf16* __restrict__ dy, const float* __restrict__ adt,
    const float* __restrict__ dt, const float* __restrict__ trap_logits, const float* __restrict__ angles,
    const float* __restrict__ qb, const float* __restrict__ phases, float* __restrict__ carries) {
  constexpr int N = Geo<NH>::N, NP = Geo<NH>::NP;
  extern __shared__ __align__(128) unsigned char raw[];
  DsSmem<NH>& s = *reinterpret_cast<DsSmem<NH>*>(align1024(raw));
  const int ta = fwd_ta(d.A);
  float* cosv = reinterpret_cast<float*>(&s + 1);
  float* sinv = cosv + C * ta;
  const int n = blockIdx.x % d.nch, bh = blockIdx.x / d.nch, b = bh / d.H, h = bh % d.H;
  const int t0 = n * C, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (warp == 0) {
    tc::tmem_alloc(&s.tmem, 64 * NH);
    tc::tmem_relinquish();  // this CTA allocates once; others on the SM may proceed
  }
  if (threadIdx.x == 0) tc::mbar_init(&s.bar, 1);
  // Every input starts at once: c rows in place in Qs, dY rows in Ds (both
  // in the swizzled tile layout), angle rates in sinv, gates and the
  // chunk-start phase in stg.
  const StageRef in{s.Qs[0], nullptr, 0, sinv, s.stg, s.stg + C, s.stg + 2 * C + 4};
  float* phase0 = s.stg + 3 * C + 8;
  stage_prefetch<true, NH>(d, b, h, n, cq, nullptr, adt, dt, trap_logits, angles, in, ta);
  {
    const int tid = threadIdx.x;
#pragma unroll
    for (int k = 0; k < 16 / GW; ++k) {
      const int idx = tid + k * GW * 32, rr = idx >> 3, c8 = 8 * (idx & 7), t = t0 + rr;
      const bool live = t < d.T;
      cp16(reinterpret_cast<float*>(at<true>(s.Ds, rr, c8)),
           reinterpret_cast<const float*>(live ? dy + (size_t(b) * d.T + t) * d.H * P + h * P + c8 : dy), live);
    }
    if (tid < NP) cp4(phase0 + tid, phases + (size_t(bh) * d.nch + n) * NP + tid, true);
    cp_commit();
    cp_wait();
  }
  __syncthreads();
  stage_rows(d, t0, in, s.r, s.scratch);
  __syncthreads();
  stage_theta<NH>(d, in, s.r, phase0, cosv, sinv, ta, ta);
  __syncthreads();
  stage_qk<true, true, NH>(h, in, qb, nullptr, cosv, sinv, s.Qs[0], nullptr, 0, d.A, ta);
  {
    // rd(dY o e^p) in place: each thread rescales the pieces it copied.
    const int tid = threadIdx.x;
#pragma unroll
    for (int k = 0; k < 16 / GW; ++k) {
      const int idx = tid + k * GW * 32, rr = idx >> 3, c8 = 8 * (idx & 7);
      uint4* q = reinterpret_cast<uint4*>(at<true>(s.Ds, rr, c8));
      const uint4 v = *q;
      const float f = s.r.ept[rr];
      const uint32_t* u = reinterpret_cast<const uint32_t*>(&v);
      uint4 o;
      uint32_t* w = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const __nv_bfloat162 x2 = __floats2bfloat162_rn(lo_f(u[j]) * f, hi_f(u[j]) * f);
        w[j] = *reinterpret_cast<const uint32_t*>(&x2);
      }
      *q = o;
    }
  }
  tc_publish();
  const uint32_t tm = s.tmem;
  if (threadIdx.x == 0) {
#pragma unroll
    for (int q = 0; q < NH; ++q) tc_product(tm + 64 * q, s.Qs[q], true, s.Ds, true);  // Q^T D: rows n, cols p
    tc::commit(&s.bar);
  }
  if (tc_wait(&s.bar, 0)) {
    // 16-lane loads: rows r0 + 8 hh, columns col0 + 8 k + cq2 + {0, 1}.
    const int r0 = 16 * (warp & 3) + (lane >> 2), cq2 = 2 * (lane & 3), col0 = 32 * (warp >> 2);
#pragma unroll
    for (int q = 0; q < NH; ++q) {
      float v[16];
      ld_16x256b_x4(tmem_lane_base(tm) + 64 * q + col0, v);
      tc::wait_ld();
      float* dst = carries + (size_t(bh) * d.nch + n) * N * P + (64 * q + r0) * P + col0 + cq2;
#pragma unroll
      for (int k = 0; k < 4; ++k)
#pragma unroll
        for (int hh = 0; hh < 2; ++hh)
          *reinterpret_cast<float2*>(dst + 8 * hh * P + 8 * k) = make_float2(v[4 * k + 2 * hh], v[4 * k + 2 * hh + 1]);
    }
  }
  tc::fence_before();
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tm, 64 * NH);
}

// Reverse over chunks, in place: carries[n] <- E_n (cotangent of chunk n's end
// state); E_(nch-1) = d_final, E_(n-1) = D_n + d_n E_n. Same split and
// look-ahead as state_kernel.
template <int NH>
__global__ void __launch_bounds__(256) carry_kernel(Dims d, float* __restrict__ carries,
                                                    const float* __restrict__ deltas,
                                                    const float* __restrict__ d_final) {
  constexpr int N = Geo<NH>::N, SP = sparts<NH>();
  const int bh = blockIdx.x / SP, i = 4 * ((blockIdx.x % SP) * 256 + threadIdx.x);
  float4 e = d_final ? ld4(d_final + size_t(bh) * N * P + i) : make_float4(0.f, 0.f, 0.f, 0.f);
  for (int m0 = 0; m0 < d.nch; m0 += 8) {
    float4 u[8];
    float dl[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int n = d.nch - 1 - m0 - j;
      if (n >= 0) {
        u[j] = ld4(carries + (size_t(bh) * d.nch + n) * N * P + i);
        dl[j] = deltas[size_t(bh) * d.nch + n];
      }
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int n = d.nch - 1 - m0 - j;
      if (n >= 0) {
        st4(carries + (size_t(bh) * d.nch + n) * N * P + i, e);
        e = make_float4(fmaf(dl[j], e.x, u[j].x), fmaf(dl[j], e.y, u[j].y), fmaf(dl[j], e.z, u[j].z),
                        fmaf(dl[j], e.w, u[j].w));
      }
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
  float* dth;     // [B,H,nch,NP] per-chunk totals of the pair phase gradient
  float* dqb;     // [B,H,nch,N] per-chunk bias partials
  float* dkb;     // [B,H,nch,N]
};

template <int NH>
struct GradSmem {
  static constexpr int N = Geo<NH>::N, TW = Geo<NH>::TW;
  // tcgen05 operands: 128-byte-swizzled 64-column bf16 tiles on 1024-byte
  // boundaries (tc::sw); Ms and Mt adjacent (16 KB, the fp32 S_n stage at N = 64).
  bf16 Qs[NH][C * 64];  // rotated queries, state columns 64 q .. 64 q + 63
  bf16 Ks[NH][C * 64];
  bf16 Vs[C * 64];
  bf16 Dy[C * 64];
  bf16 Ms[C * 64];      // rd(scores o W), then rd(dY o e^p)
  bf16 Mt[C * 64];      // rd(d_mixed o W)
  bf16 Es[NH][64 * 64]; // rd(E_n), state rows 64 q .. 64 q + 63
  bf16 Ss[NH][64 * 64]; // rd(S_n)
  float theta[C * TW];  // cos of the pair phase, then the pair phase gradient
  float sinv[C * TW];
  // Per-token rows: 0 sum K.(V rd(E)^T), 1 e^p dY.(Q rd(S)), 2 log-decay
  // increment, 3 d gamma, 4 d scale, 5 flow, 6 d log-decay, 7 unused;
  // 8-9 / 10-11 / 12-13: the two column halves' partials of the row sums
  // of d_weights o W, of row 0 and of row 1.
  float vec[14 * C];
  float col[2][4 * C];  // per row block: column sums of d_weights o W and of d_weights o decay
  float bq[4 * N];      // per row block bias partials
  float bk[4 * N];
  float scratch[C];
  Rows r;
  uint64_t bar;         // tensor-core commits (three per chunk)
  uint32_t tmem;
};

// Tensor-memory columns of the chunk-gradient products (M = 64 accumulators).
template <int NH> struct GradCols {
  static constexpr int SC = 0, DM = 64;             // commit 1: scores, d_mixed
  static constexpr int DV = 0, VE = 64;             // commit 2: dV, K rd(E)
  static constexpr int VN = 0, QS = 64 * NH;        // commit 3: V rd(E)^T (N cols), Q rd(S)
  static constexpr int GQ = NH == 1 ? 128 : 256;    //           dQ (N cols)
  static constexpr int GK = GQ + 64 * NH;           //           dK (N cols)
  static constexpr int ALLOC = NH == 1 ? 256 : 512;
};

// The m16n8 accumulator fragments of NT 8-column tiles from tensor memory:
// acc[nt][e] is row t / 4 + 8 (e / 2), column 8 nt + 2 (t % 4) + e % 2 of
// the warp's lane quarter from column `taddr` (16x256b loads, which place an
// M = 64 accumulator's values exactly as mma.sync places them).
template <int NT>
M4_DEV void tm_frag(uint32_t taddr, float (&acc)[NT][4]) {
  static_assert(NT % 4 == 0, "whole 32-column loads");
#pragma unroll
  for (int g4 = 0; g4 < NT / 4; ++g4) {
    float v[16];
    ld_16x256b_x4(taddr + 32 * g4, v);
#pragma unroll
    for (int k = 0; k < 4; ++k)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[4 * g4 + k][e] = v[4 * k + e];
  }
  tc::wait_ld();
}

// Every gradient of one chunk given S_n and E_n. The nine chunk products run
// on the tensor cores (tcgen05, one thread issuing, three commits to an
// mbarrier; operands are 128-byte-swizzled tiles, accumulators in tensor
// memory). Eight warps read the accumulators: warp w owns rows 16 (w % 4) ..
// +15 and column half w / 4 of every product (32 token columns, or N / 2
// state columns); row sums over the two halves and column sums over the four
// row blocks meet in shared memory.
template <int NH>
__global__ void __launch_bounds__(GW * 32, NH == 1 ? 2 : 1) grads_kernel(
    Dims d, const bf16* __restrict__ cq, const bf16* __restrict__ bk, const bf16* __restrict__ x,
    const float* __restrict__ adt, const float* __restrict__ dt, const float* __restrict__ trap_logits,
    const float* __restrict__ angles, const float* __restrict__ qb, const float* __restrict__ kb,
    const float* __restrict__ phases, const float* __restrict__ starts, const float* __restrict__ carries,
    const bf16* __restrict__ dy, bf16* __restrict__ dx, GradOut o) {
  constexpr int TH = GW * 32, N = Geo<NH>::N, NP = Geo<NH>::NP, TW = Geo<NH>::TW;
  constexpr int NTN = 4 * NH;  // 8-column n-tiles of a warp's state-column half
  using TC = GradCols<NH>;
  extern __shared__ __align__(128) unsigned char raw[];
  GradSmem<NH>& s = *reinterpret_cast<GradSmem<NH>*>(align1024(raw));
  const int n = blockIdx.x % d.nch, bh = blockIdx.x / d.nch, b = bh / d.H, h = bh % d.H;
  const int t0 = n * C, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int rb = warp & 3, half = warp >> 2, row0 = 16 * rb, col0 = 32 * half, colN = (N / 2) * half;
  const int g = lane >> 2, cc = lane & 3;
  // Byte offset in a swizzled tile of (row, column 8 chunk + 2 cc) for this
  // thread's fragment rows (row % 8 == g).
  auto frag_off = [&](int row, int chunk) { return row * 128 + ((chunk ^ g) << 4) + 4 * cc; };
  if (warp == 0) {
    tc::tmem_alloc(&s.tmem, TC::ALLOC);
    tc::tmem_relinquish();
  }
  if (tid == 0) tc::mbar_init(&s.bar, 1);
  // Every pure copy starts first and lands while the gates, phases and
  // rotations are built: x and dY straight into their tiles, S_n (fp32) into
  // the score tiles (free until the scores; at N = 128 into registers), E_n
  // into registers.
  constexpr int PER = N * P / 4 / TH;
  float* Sstage = reinterpret_cast<float*>(s.Ms);  // [64][64] fp32 over Ms and Mt (N = 64)
  // c / b rows in place in Qs / Ks, angle rates in Es, gates and the
  // chunk-start phase in vec (all free until later phases).
  const StageRef in{s.Qs[0], s.Ks[0], 0, reinterpret_cast<float*>(s.Es[0]), s.vec, s.vec + C, s.vec + 2 * C + 4};
  float* phase0 = s.vec + 3 * C + 8;
  stage_prefetch<true, NH>(d, b, h, n, cq, bk, adt, dt, trap_logits, angles, in);
  if (tid < NP) cp4(phase0 + tid, phases + (size_t(bh) * d.nch + n) * NP + tid, true);
  float4 ev[PER], sv[NH == 1 ? 1 : PER];
  {
#pragma unroll
    for (int k = 0; k < 2 * (16 / GW); ++k) {
      const int idx = tid + (k % (16 / GW)) * TH, rr = idx >> 3, c8 = 8 * (idx & 7), t = t0 + rr;
      const bool live = t < d.T;
      const bf16* src = k < 16 / GW ? x : dy;
      bf16* dst = at<true>(k < 16 / GW ? s.Vs : s.Dy, rr, c8);
      cp16(reinterpret_cast<float*>(dst),
           reinterpret_cast<const float*>(live ? src + (size_t(b) * d.T + t) * d.H * P + h * P + c8 : src), live);
    }
    const float* Sg = starts + (size_t(bh) * d.nch + n) * N * P;
    const float* Eg = carries + (size_t(bh) * d.nch + n) * N * P;
    if constexpr (NH == 1) {
#pragma unroll
      for (int k = 0; k < PER; ++k) cp16(Sstage + 4 * (tid + k * TH), Sg + 4 * (tid + k * TH), true);
    } else {
#pragma unroll
      for (int k = 0; k < PER; ++k) sv[k] = ld4(Sg + 4 * (tid + k * TH));
    }
    cp_commit();
#pragma unroll
    for (int k = 0; k < PER; ++k) ev[k] = ld4(Eg + 4 * (tid + k * TH));
  }
  cp_commit();
  cp_wait();
  __syncthreads();  // every staged input has landed
  stage_rows(d, t0, in, s.r, s.scratch);
  __syncthreads();
  stage_theta<NH>(d, in, s.r, phase0, s.theta, s.sinv);
  __syncthreads();
  stage_qk<true, true, NH>(h, in, qb, kb, s.theta, s.sinv, s.Qs[0], s.Ks[0]);
  __syncthreads();  // the angle stage (Es) is consumed
  // rd(S_n), rd(E_n) as tiles and <E_n, S_n> (fp32 values) for the chunk-end decay.
  {
    float part = 0.f;
#pragma unroll
    for (int k = 0; k < PER; ++k) {
      const int idx = tid + k * TH;
      float4 a4;
      if constexpr (NH == 1) a4 = ld4(Sstage + 4 * idx);
      else a4 = sv[k];
      const float4 e4 = ev[k];
      const int r = idx / (P / 4), c4 = idx % (P / 4);
      // r % 8 is the same for every k of this thread; 4 columns = half a chunk.
      const int off = (r & 63) * 128 + (((c4 >> 1) ^ (r & 7)) << 4) + 8 * (c4 & 1);
      unsigned char* ss = reinterpret_cast<unsigned char*>(s.Ss[r >> 6]) + off;
      unsigned char* es = reinterpret_cast<unsigned char*>(s.Es[r >> 6]) + off;
      *reinterpret_cast<__nv_bfloat162*>(ss) = __floats2bfloat162_rn(a4.x, a4.y);
      *reinterpret_cast<__nv_bfloat162*>(ss + 4) = __floats2bfloat162_rn(a4.z, a4.w);
      *reinterpret_cast<__nv_bfloat162*>(es) = __floats2bfloat162_rn(e4.x, e4.y);
      *reinterpret_cast<__nv_bfloat162*>(es + 4) = __floats2bfloat162_rn(e4.z, e4.w);
      part = fmaf(a4.x, e4.x, fmaf(a4.y, e4.y, fmaf(a4.z, e4.z, fmaf(a4.w, e4.w, part))));
    }
    part = warp_sum(part);
    if (lane == 0) s.scratch[warp] = part;
  }
  tc_publish();
  const uint32_t tm = s.tmem, tl = tmem_lane_base(tm);
  if (tid == 0) {
#pragma unroll
    for (int q = 0; q < NH; ++q) tc_product(tm + TC::SC, s.Qs[q], false, s.Ks[q], false, q > 0);  // Q K^T
    tc_product(tm + TC::DM, s.Dy, false, s.Vs, false);                                          // dY V^T
    tc::commit(&s.bar);
  }
  bool ok = tc_wait(&s.bar, 0);
  // Scores Q K^T and d_mixed dY V^T (rows t, this warp's 32 columns s) from
  // tensor memory. Each element gives the two masked tiles rd(scores o W) and
  // rd(d_mixed o W) and the per-token sums of d_weights = d_mixed o scores:
  //   row t:    sum_{s<t} dw W,  column s: sum_{u>s} dw W and sum_{u>s} dw decay,
  // with W = decay(t, s) scale_s below the diagonal and gamma_t on it.
  {
    float sc[4][4], dm[4][4];
    tm_frag<4>(tl + TC::SC + col0, sc);
    tm_frag<4>(tl + TC::DM + col0, dm);
    float rsum[2] = {0.f, 0.f}, c1[4][2], c2[4][2];
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
      const int t = row0 + g + 8 * hf;
      const float pt = s.r.p[t];
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) {
        float ms[2], mt[2];
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int sidx = col0 + nt * 8 + 2 * cc + e;
          const float vs = sc[nt][2 * hf + e], vd = dm[nt][2 * hf + e], dw = vd * vs;
          float w = 0.f, dec = 0.f;
          if (sidx < t) {
            dec = expf(pt - s.r.p[sidx]);
            w = dec * s.r.scl[sidx];
          } else if (sidx == t) {
            w = s.r.gam[t];
            s.vec[3 * C + t] = dw;
          }
          ms[e] = vs * w;
          mt[e] = vd * w;
          const float dww = sidx < t ? dw * w : 0.f;
          rsum[hf] += dww;
          if (hf == 0) {
            c1[nt][e] = dww;
            c2[nt][e] = dw * dec;
          } else {
            c1[nt][e] += dww;
            c2[nt][e] = fmaf(dw, dec, c2[nt][e]);
          }
        }
        const int off = frag_off(t, (col0 >> 3) + nt);
        *reinterpret_cast<__nv_bfloat162*>(reinterpret_cast<unsigned char*>(s.Ms) + off) =
            __floats2bfloat162_rn(ms[0], ms[1]);
        *reinterpret_cast<__nv_bfloat162*>(reinterpret_cast<unsigned char*>(s.Mt) + off) =
            __floats2bfloat162_rn(mt[0], mt[1]);
      }
    }
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
      float v = rsum[hf];
      v += __shfl_xor_sync(0xffffffffu, v, 1);
      v += __shfl_xor_sync(0xffffffffu, v, 2);
      if (cc == 0) s.vec[(8 + half) * C + row0 + g + 8 * hf] = v;
    }
#pragma unroll
    for (int nt = 0; nt < 4; ++nt)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        float a = c1[nt][e], v = c2[nt][e];
#pragma unroll
        for (int off = 4; off < 32; off <<= 1) {
          a += __shfl_xor_sync(0xffffffffu, a, off);
          v += __shfl_xor_sync(0xffffffffu, v, off);
        }
        if (g == 0) {
          s.col[0][rb * C + col0 + nt * 8 + 2 * cc + e] = a;
          s.col[1][rb * C + col0 + nt * 8 + 2 * cc + e] = v;
        }
      }
  }
  tc_publish();
  if (tid == 0 && ok) {
    tc_product(tm + TC::DV, s.Ms, true, s.Dy, true);                                          // rd(Sc o W)^T dY
#pragma unroll
    for (int q = 0; q < NH; ++q) tc_product(tm + TC::VE, s.Ks[q], false, s.Es[q], true, q > 0);  // K rd(E)
    tc::commit(&s.bar);
  }
  ok = ok && tc_wait(&s.bar, 1);
  // dV = rd(Sc o W)^T dY + src o (K rd(E)) -> dx (rows s, this warp's 32 columns p).
  {
    float acc[4][4], ve[4][4];
    tm_frag<4>(tl + TC::DV + col0, acc);
    tm_frag<4>(tl + TC::VE + col0, ve);
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
      const int sr = row0 + g + 8 * hf, t = t0 + sr;
      if (t >= d.T) continue;
      const float src = s.r.scl[sr] * s.r.tail[sr];
      bf16* row = dx + (size_t(b) * d.T + t) * d.H * P + h * P;
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) {
        const int col = col0 + nt * 8 + 2 * cc;
        *reinterpret_cast<__nv_bfloat162*>(row + col) = __floats2bfloat162_rn(
            fmaf(src, ve[nt][2 * hf], acc[nt][2 * hf]), fmaf(src, ve[nt][2 * hf + 1], acc[nt][2 * hf + 1]));
      }
    }
  }
  // rd(dY o e^p) over Ms (its product has completed): thread (warp w, lane)
  // visits rows w + 8 k (row % 8 == w), columns 2 lane, 2 lane + 1.
  {
    const int swz = warp * 128 + (((lane >> 2) ^ warp) << 4) + 4 * (lane & 3);
#pragma unroll
    for (int k = 0; k < C / GW; ++k) {
      const int tt = warp + GW * k, off = swz + 1024 * k;
      const __nv_bfloat162 v =
          *reinterpret_cast<const __nv_bfloat162*>(reinterpret_cast<const unsigned char*>(s.Dy) + off);
      *reinterpret_cast<__nv_bfloat162*>(reinterpret_cast<unsigned char*>(s.Ms) + off) =
          __floats2bfloat162_rn(__low2float(v) * s.r.ept[tt], __high2float(v) * s.r.ept[tt]);
    }
  }
  tc_publish();
  if (tid == 0 && ok) {
#pragma unroll
    for (int q = 0; q < NH; ++q) {
      tc_product(tm + TC::GQ + 64 * q, s.Mt, false, s.Ks[q], true);         // rd(Dm o W) K
      tc_product(tm + TC::GQ + 64 * q, s.Ms, false, s.Ss[q], false, true);  // + rd(dY e^p) rd(S)^T
      tc_product(tm + TC::GK + 64 * q, s.Mt, true, s.Qs[q], true);          // rd(Dm o W)^T Q
      tc_product(tm + TC::VN + 64 * q, s.Vs, false, s.Es[q], false);        // V rd(E)^T
      tc_product(tm + TC::QS, s.Qs[q], false, s.Ss[q], true, q > 0);        // Q rd(S)
    }
    tc::commit(&s.bar);
  }
  // The raw c / b pairs of this thread's accumulator rows for the rotation
  // backward: at N = 128 loaded before the next products so their latency
  // hides (the kernel runs one CTA per SM there; registers are free), at
  // N = 64 just before use (two CTAs per SM need <= 128 registers).
  uint32_t craw[2][NTN], braw[2][NTN];
  auto load_raw = [&]() {
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
      const int t = t0 + row0 + g + 8 * hf;
      const size_t base = d.per_head ? ((size_t(b) * d.T + t) * d.H + h) * N : (size_t(b) * d.T + t) * N;
#pragma unroll
      for (int nt = 0; nt < NTN; ++nt) {
        craw[hf][nt] = t < d.T ? ld_u32(cq + base + colN + 8 * nt + 2 * cc) : 0u;
        braw[hf][nt] = t < d.T ? ld_u32(bk + base + colN + 8 * nt + 2 * cc) : 0u;
      }
    }
  };
  if constexpr (NH == 2) load_raw();
  ok = ok && tc_wait(&s.bar, 0);
  // dK (rows s, this warp's N / 2 columns n) from tensor memory; dQ is read
  // just before the rotation backward (fewer fragments live at once).
  float gk[NTN][4];
  tm_frag<NTN>(tl + TC::GK + colN, gk);
  {
    float dsrc[2] = {0.f, 0.f}, inh_dot[2] = {0.f, 0.f};
    {
      float vn[NTN][4];
      tm_frag<NTN>(tl + TC::VN + colN, vn);  // V rd(E)^T (rows s, cols n)
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        const int sr = row0 + g + 8 * hf;
        const float src = s.r.scl[sr] * s.r.tail[sr];
#pragma unroll
        for (int nt = 0; nt < NTN; ++nt)
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int ncol = colN + nt * 8;  // + 2 cc + e
            const bf16* kt = s.Ks[ncol >> 6];
            const float kv = __bfloat162float(*reinterpret_cast<const bf16*>(
                reinterpret_cast<const unsigned char*>(kt) + frag_off(sr, (ncol & 63) >> 3) + 2 * e));
            dsrc[hf] = fmaf(kv, vn[nt][2 * hf + e], dsrc[hf]);
            gk[nt][2 * hf + e] = fmaf(src, vn[nt][2 * hf + e], gk[nt][2 * hf + e]);
          }
      }
    }
    float ve[4][4];
    tm_frag<4>(tl + TC::QS + col0, ve);  // Q rd(S) (rows t, cols p)
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
      const int t = row0 + g + 8 * hf;
#pragma unroll
      for (int nt = 0; nt < 4; ++nt)
#pragma unroll
        for (int e = 0; e < 2; ++e)
          inh_dot[hf] = fmaf(__bfloat162float(*reinterpret_cast<const bf16*>(
                                 reinterpret_cast<const unsigned char*>(s.Dy) + frag_off(t, (col0 >> 3) + nt) + 2 * e)),
                             ve[nt][2 * hf + e], inh_dot[hf]);
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
        s.vec[(10 + half) * C + r] = a;
        s.vec[(12 + half) * C + r] = v;
      }
    }
  }
  constexpr int SG = C / GW;
  // Angle rates of this warp's tokens (last phase), loaded ahead likewise.
  float rates[SG][NH];
  auto load_rates = [&]() {
#pragma unroll
    for (int j = 0; j < SG; ++j)
#pragma unroll
      for (int q = 0; q < NH; ++q) {
        const int i = lane + 32 * q, t = t0 + SG * warp + j;
        rates[j][q] = (i < d.A && t < d.T) ? rate_at(d, angles, b, h, t, i) : 0.f;
      }
  };
  if constexpr (NH == 2) load_rates();
  if constexpr (NH == 1) load_raw();
  float gq[NTN][4];
  tm_frag<NTN>(tl + TC::GQ + colN, gq);
  // Rotation backward in registers: the accumulators hold each pair (2i, 2i+1)
  // on one thread. Pre-rotation gradients to workspace, the pair phase
  // gradient into theta (same element, read then written by this thread),
  // bias partials per column.
  {
    float sq[NTN][2], sk[NTN][2];
#pragma unroll
    for (int nt = 0; nt < NTN; ++nt) sq[nt][0] = sq[nt][1] = sk[nt][0] = sk[nt][1] = 0.f;
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
      const int tt = row0 + g + 8 * hf, t = t0 + tt;
      const bool live = t < d.T;
      const size_t ob = ((size_t(b) * d.T + t) * d.H + h) * N;
#pragma unroll
      for (int nt = 0; nt < NTN; ++nt) {
        const int i = (colN >> 1) + 4 * nt + cc, n0 = 2 * i;
        const float cs = s.theta[tt * TW + i], sn = s.sinv[tt * TW + i];
        const float gq0 = gq[nt][2 * hf], gq1 = gq[nt][2 * hf + 1];
        const float gk0 = gk[nt][2 * hf], gk1 = gk[nt][2 * hf + 1];
        const float pq0 = gq0 * cs + gq1 * sn, pq1 = gq1 * cs - gq0 * sn;
        const float pk0 = gk0 * cs + gk1 * sn, pk1 = gk1 * cs - gk0 * sn;
        const float c0 = lo_f(craw[hf][nt]), c1 = hi_f(craw[hf][nt]);
        const float b0 = lo_f(braw[hf][nt]), b1 = hi_f(braw[hf][nt]);
        if (live) {
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
        s.theta[tt * TW + i] = (i < d.A && live) ? dth : 0.f;
      }
    }
    // Column sums over the warp's 16 rows (the eight lanes of one cc, two
    // rows each): reduce-scatter, lane g ends with values [R g, R g + R).
    constexpr int V = 4 * NTN, R = V / 8;
    float v[V];
#pragma unroll
    for (int nt = 0; nt < NTN; ++nt)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        v[2 * nt + e] = sq[nt][e];
        v[2 * NTN + 2 * nt + e] = sk[nt][e];
      }
    reduce_scatter<V, 3, 2>(v, lane);
#pragma unroll
    for (int m = 0; m < R; ++m) {
      const int idx = R * g + m, j = idx % (2 * NTN), nt = j >> 1, e = j & 1;
      float* dst = idx < 2 * NTN ? s.bq : s.bk;
      dst[rb * N + colN + nt * 8 + 2 * cc + e] = v[m];
    }
  }
  __syncthreads();
  // Per-token scalar gradients.
  if (tid < C) {
    const int t = tid;
    const float dsrc = s.vec[10 * C + t] + s.vec[11 * C + t];
    s.vec[0 * C + t] = dsrc;
    s.vec[1 * C + t] = (s.vec[12 * C + t] + s.vec[13 * C + t]) * s.r.ept[t];
    const float rowoff = s.vec[8 * C + t] + s.vec[9 * C + t];
    const float coloff = s.col[0][t] + s.col[0][C + t] + s.col[0][2 * C + t] + s.col[0][3 * C + t];
    const float cdec = s.col[1][t] + s.col[1][C + t] + s.col[1][2 * C + t] + s.col[1][3 * C + t];
    const float flow = dsrc * s.r.scl[t] * s.r.tail[t];
    s.vec[2 * C + t] = rowoff - coloff - flow + s.vec[1 * C + t];
    s.vec[4 * C + t] = dsrc * s.r.tail[t] + cdec;
    s.vec[5 * C + t] = flow;
  } else if (tid < C + N) {
    const int nn = tid - C;
    o.dqb[(size_t(bh) * d.nch + n) * N + nn] = s.bq[nn] + s.bq[N + nn] + s.bq[2 * N + nn] + s.bq[3 * N + nn];
    o.dkb[(size_t(bh) * d.nch + n) * N + nn] = s.bk[nn] + s.bk[N + nn] + s.bk[2 * N + nn] + s.bk[3 * N + nn];
  }
  __syncthreads();
  // Suffix sums of the pair phase gradient: warp w over tokens SG w .. SG w +
  // SG - 1, then the totals of later segments (the carry from later chunks is
  // added by finish_kernel). Warp 0 also runs the log-decay suffix scan.
  {
#pragma unroll
    for (int q = 0; q < NH; ++q) {
      const int i = lane + 32 * q;
      float acc = 0.f;
#pragma unroll
      for (int j = SG - 1; j >= 0; --j) {
        acc += s.theta[(SG * warp + j) * TW + i];
        s.theta[(SG * warp + j) * TW + i] = acc;
      }
      s.r.seg[warp * NP + i] = acc;
    }
    if (warp == 0) {
      float fl = s.vec[5 * C + lane] + s.vec[5 * C + 32 + lane];
      fl = warp_sum(fl);
      const float end = expf(s.r.p[C - 1]);
      float es = 0.f;
#pragma unroll
      for (int w = 0; w < GW; ++w) es += s.scratch[w];
      const float extra = fl + end * es;
      const float hi = s.vec[2 * C + 63 - lane] + (lane == 0 ? extra : 0.f);
      const float shi = warp_inclusive_scan(hi, lane);
      const float tot = __shfl_sync(0xffffffffu, shi, 31);
      const float slo = warp_inclusive_scan(s.vec[2 * C + 31 - lane], lane) + tot;
      s.vec[6 * C + 63 - lane] = shi;
      s.vec[6 * C + 31 - lane] = slo;
    }
  }
  __syncthreads();
  {
    float off[NH];
#pragma unroll
    for (int q = 0; q < NH; ++q) {
      const int i = lane + 32 * q;
      off[q] = 0.f;
      for (int v = warp + 1; v < GW; ++v) off[q] += s.r.seg[v * NP + i];
      if (warp == 0 && i < d.A)
        o.dth[(size_t(bh) * d.nch + n) * NP + i] = off[q] + s.r.seg[i];
    }
    // Angle-rate and dt-through-phase gradients of this warp's SG tokens:
    // lanes over angle pairs (coalesced rows); the dt terms of the SG tokens
    // reduced together (reduce-scatter: lane l ends with token l / 4).
    if constexpr (NH == 1) load_rates();
    float part[SG];
#pragma unroll
    for (int j = 0; j < SG; ++j) {
      const int tt = SG * warp + j, t = t0 + tt;
      part[j] = 0.f;
      if (t < d.T) {
        const size_t si = (size_t(b) * d.T + t) * d.H + h;
#pragma unroll
        for (int q = 0; q < NH; ++q) {
          const int i = lane + 32 * q;
          const float inc = i < d.A ? s.theta[tt * TW + i] + off[q] : 0.f;
          if (i < d.A) o.drate[si * d.A + i] = inc * s.r.dt[tt];
          part[j] = fmaf(inc, rates[j][q], part[j]);
        }
      }
    }
    static_assert(SG == 8, "one token per group of four lanes");
    reduce_scatter<SG, 3, 2>(part, lane);
    part[0] += __shfl_xor_sync(0xffffffffu, part[0], 1);
    part[0] += __shfl_xor_sync(0xffffffffu, part[0], 2);
    if ((lane & 3) == 0) {
      const int tt = SG * warp + (lane >> 2), t = t0 + tt;
      if (t < d.T) {
        const size_t si = (size_t(b) * d.T + t) * d.H + h;
        o.ddtp[si] = part[0];
        o.dgam[si] = s.vec[3 * C + tt];
        o.dscl[si] = s.vec[4 * C + tt];
        o.dlog[si] = s.vec[6 * C + tt];
      }
    }
  }
  tc::fence_before();
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tm, TC::ALLOC);
}

// In place over chunks: dth[n] <- sum over chunks m > n of the chunk totals
// (the phase-gradient carry every token of chunk n receives).
template <int NH>
__global__ void later_kernel(Dims d, float* __restrict__ dth) {
  constexpr int NP = Geo<NH>::NP;
  const int bh = blockIdx.x, i = threadIdx.x;  // NP threads
  float acc = 0.f;
  for (int n = d.nch - 1; n >= 0; --n) {
    float* slot = dth + (size_t(bh) * d.nch + n) * NP + i;
    const float v = i < d.A ? *slot : 0.f;
    *slot = acc;
    acc += v;
  }
}

// One warp per token (b, t), lanes over angle pairs and state pairs, heads in
// order: adds the later-chunk phase carry (rate gradient += later dt, dt
// gradient += later . rate), applies the gate chain rule of the mamba3_fused
// preprocessing (flashmamba.py:1142-1147) and sums the angle-rate and
// query/key gradients over heads (shared layout) or converts them (per head).
template <int NH>
__global__ void __launch_bounds__(256) finish_kernel(
    Dims d, const float* __restrict__ dt, const float* __restrict__ trap_logits,
    const float* __restrict__ angles, const float* __restrict__ later, GradOut o, bf16* __restrict__ dc,
    bf16* __restrict__ db, float* __restrict__ d_adt, float* __restrict__ d_dt, float* __restrict__ d_trap,
    float* __restrict__ d_angles) {
  constexpr int N = Geo<NH>::N, NP = Geo<NH>::NP;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const size_t bt = size_t(blockIdx.x) * 8 + warp;
  if (bt >= size_t(d.B) * d.T) return;
  const int b = int(bt / d.T), t = int(bt % d.T), n = t / C;
  // Lane l handles angle pairs and state pairs l + 32 q (q < NH).
  bool pair[NH];
  float shared_rate[NH], ang[NH], q0[NH], q1[NH], k0[NH], k1[NH];
#pragma unroll
  for (int q = 0; q < NH; ++q) {
    const int i = lane + 32 * q;
    pair[q] = i < d.A;
    shared_rate[q] = (!d.per_head && pair[q]) ? angles[bt * d.A + i] : 0.f;
    ang[q] = q0[q] = q1[q] = k0[q] = k1[q] = 0.f;
  }
  for (int h0 = 0; h0 < d.H; h0 += 32) {
    float mine = 0.f;
    const int hn = min(32, d.H - h0);
    for (int j = 0; j < hn; ++j) {
      const int h = h0 + j;
      const size_t si = bt * d.H + h;
      float part = 0.f;
#pragma unroll
      for (int q = 0; q < NH; ++q) {
        const int i = lane + 32 * q;
        const float rate = d.per_head ? (pair[q] ? angles[si * d.A + i] : 0.f) : shared_rate[q];
        const float l = pair[q] ? later[((size_t(b) * d.H + h) * d.nch + n) * NP + i] : 0.f;
        if (pair[q]) {
          const float dr = fmaf(l, dt[si], o.drate[si * d.A + i]);
          if (d.per_head) d_angles[si * d.A + i] = dr;
          else ang[q] += dr;
        }
        part = fmaf(l, rate, part);
        const float2 gq = *reinterpret_cast<const float2*>(o.dq + si * N + 2 * i);
        const float2 gk = *reinterpret_cast<const float2*>(o.dk + si * N + 2 * i);
        if (d.per_head) {
          *reinterpret_cast<__nv_bfloat162*>(dc + si * N + 2 * i) = __floats2bfloat162_rn(gq.x, gq.y);
          *reinterpret_cast<__nv_bfloat162*>(db + si * N + 2 * i) = __floats2bfloat162_rn(gk.x, gk.y);
        } else {
          q0[q] += gq.x; q1[q] += gq.y; k0[q] += gk.x; k1[q] += gk.y;
        }
      }
      const float extra = warp_sum(part);
      if (lane == j) mine = extra;
    }
    if (lane < hn) {
      const size_t si = bt * d.H + h0 + lane;
      const float s = 1.f / (1.f + expf(-trap_logits[si]));
      const float gsum = o.dgam[si] + o.dscl[si];
      const float pv = t > 0 ? o.dscl[si - d.H] : 0.f;
      d_dt[si] = fmaf(gsum, s, pv * (1.f - s)) + (o.ddtp[si] + mine);
      d_trap[si] = (gsum - pv) * dt[si] * s * (1.f - s);
      d_adt[si] = o.dlog[si];
    }
  }
  if (!d.per_head) {
#pragma unroll
    for (int q = 0; q < NH; ++q) {
      const int i = lane + 32 * q;
      if (pair[q]) d_angles[bt * d.A + i] = ang[q];
      *reinterpret_cast<__nv_bfloat162*>(dc + bt * N + 2 * i) = __floats2bfloat162_rn(q0[q], q1[q]);
      *reinterpret_cast<__nv_bfloat162*>(db + bt * N + 2 * i) = __floats2bfloat162_rn(k0[q], k1[q]);
    }
  }
}

// Bias gradients: sum per-chunk partials over batch and chunks. Block per
// head; 1024 / N groups of N threads take interleaved (batch, chunk) slots,
// then the groups are added in a fixed order (deterministic).
template <int NH>
__global__ void __launch_bounds__(1024) bias_kernel(Dims d, const float* __restrict__ dqb,
                                                    const float* __restrict__ dkb, float* __restrict__ d_qb,
                                                    float* __restrict__ d_kb) {
  constexpr int N = Geo<NH>::N, GR = 1024 / N;
  __shared__ float part[2][GR][N];
  const int h = blockIdx.x, nn = threadIdx.x & (N - 1), grp = threadIdx.x / N;
  const int slots = d.B * d.nch;
  float sq = 0.f, sk = 0.f;
#pragma unroll 4
  for (int k = grp; k < slots; k += GR) {
    const int b = k / d.nch, n = k % d.nch;
    const size_t o = ((size_t(b) * d.H + h) * d.nch + n) * N + nn;
    sq += dqb[o];
    sk += dkb[o];
  }
  part[0][grp][nn] = sq;
  part[1][grp][nn] = sk;
  __syncthreads();
  if (threadIdx.x < N) {
    float q = 0.f, k = 0.f;
    for (int gi = 0; gi < GR; ++gi) {
      q += part[0][gi][nn];
      k += part[1][gi][nn];
    }
    if (d_qb) d_qb[h * N + nn] = q;
    if (d_kb) d_kb[h * N + nn] = k;
  }
}

}  // namespace scan2
}  // namespace m4
