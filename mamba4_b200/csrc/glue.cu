// Fused model glue around the two hot operators (sm_100a): the Mamba-3 mixer
// projection split / gates / norms before the scan and the D skip + SiLU gate
// after it (lm/models/mamba3.py:74-132), and the bf16 RMSNorm of every block
// (lm/models/common.py:25-45), each with its hand-written backward.
//
// Every kernel is a single pass over rows of the in-projection output with
// one warp per row; parameter gradients are written as per-warp partial sums
// and added by colsum_kernel in a fixed order (deterministic, no atomics).
#include "common.cuh"

namespace m4 {
namespace glue {

using bf16 = __nv_bfloat16;

M4_DEV float bf(const bf16* p) { return __bfloat162float(*p); }
M4_DEV float2 bf2(const bf16* p) { return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(p)); }
M4_DEV void st_bf2(bf16* p, float a, float b) {
  *reinterpret_cast<__nv_bfloat162*>(p) = __floats2bfloat162_rn(a, b);
}
M4_DEV void unpack8(const uint4& v, float (&f)[8]) {
  const uint32_t* u = reinterpret_cast<const uint32_t*>(&v);
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    f[2 * q] = __uint_as_float(u[q] << 16);
    f[2 * q + 1] = __uint_as_float(u[q] & 0xffff0000u);
  }
}
M4_DEV uint4 pack8(const float (&f)[8]) {
  uint4 v;
  uint32_t* u = reinterpret_cast<uint32_t*>(&v);
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(f[2 * q], f[2 * q + 1]);
    u[q] = *reinterpret_cast<const uint32_t*>(&h);
  }
  return v;
}
M4_DEV uint4 ld16(const bf16* p) { return *reinterpret_cast<const uint4*>(p); }
M4_DEV void st16(bf16* p, uint4 v) { *reinterpret_cast<uint4*>(p) = v; }

M4_DEV float sigmoid(float x) { return 1.f / (1.f + expf(-x)); }
// torch.nn.functional.softplus (beta 1, threshold 20) and its derivative.
M4_DEV float softplus(float x) { return x > 20.f ? x : log1pf(expf(x)); }
M4_DEV float softplus_grad(float x) { return x > 20.f ? 1.f : sigmoid(x); }
// heavy_tail(x) = max(x, 0) + 1 / (1 - min(x, 0)) (lm/models/mamba3.py:28-29).
M4_DEV float heavy_tail(float x) { return fmaxf(x, 0.f) + 1.f / (1.f - fminf(x, 0.f)); }
M4_DEV float heavy_tail_grad(float x) {
  const float m = 1.f - fminf(x, 0.f);
  return (x >= 0.f ? 1.f : 0.f) + (x <= 0.f ? 1.f / (m * m) : 0.f);
}

struct Mix {
  int rows, inner, heads, angles, width;  // width: row stride of proj / d_proj
  float eps;
  int off_x, off_b, off_c, off_dt, off_a, off_trap, off_ang;
};

inline Mix make_mix(const M4MixerDims& m) {
  Mix d;
  d.rows = m.rows; d.inner = m.inner; d.heads = m.heads; d.angles = m.angles; d.eps = m.eps;
  d.off_x = m.inner;
  d.off_b = 2 * m.inner;
  d.off_c = d.off_b + 64;
  d.off_dt = d.off_c + 64;
  d.off_a = d.off_dt + m.heads;
  d.off_trap = d.off_a + m.heads;
  d.off_ang = d.off_trap + m.heads;
  d.width = m.stride;
  return d;
}

constexpr int WPB = 8;  // warps per block

M4_DEV int gwarp() { return blockIdx.x * WPB + (threadIdx.x >> 5); }
M4_DEV int nwarps() { return gridDim.x * WPB; }

// RMSNorm of a 64-wide bf16 slice held as one pair per lane; returns the
// normalised pair and the inverse rms.
M4_DEV float2 norm64(float2 v, float eps, float& r) {
  const float ss = warp_sum(v.x * v.x + v.y * v.y);
  r = rsqrtf(ss * (1.f / 64.f) + eps);
  return make_float2(v.x * r, v.y * r);
}

// Mamba-3 mixer, before the scan: c = C_norm(c), b = B_norm(b) (bf16),
// x copied contiguous, dt = softplus(raw_dt + dt_bias), adt = a dt with
// a = -max(heavy_tail(raw_a), 1e-4), trap and angles widened to fp32.
__global__ void __launch_bounds__(WPB * 32) mixer_prep_fwd(Mix d, const bf16* __restrict__ proj,
                                                          const float* __restrict__ bscale,
                                                          const float* __restrict__ cscale,
                                                          const float* __restrict__ dt_bias, bf16* __restrict__ c_out,
                                                          bf16* __restrict__ b_out, bf16* __restrict__ x_out,
                                                          float* __restrict__ adt, float* __restrict__ dt,
                                                          float* __restrict__ trap, float* __restrict__ ang) {
  const int lane = threadIdx.x & 31;
  for (int row = gwarp(); row < d.rows; row += nwarps()) {
    const bf16* pr = proj + size_t(row) * d.width;
    for (int k = lane; k < d.inner / 8; k += 32) st16(x_out + size_t(row) * d.inner + 8 * k, ld16(pr + d.off_x + 8 * k));
    float r;
    const float2 bn = norm64(bf2(pr + d.off_b + 2 * lane), d.eps, r);
    st_bf2(b_out + size_t(row) * 64 + 2 * lane, bn.x * bscale[2 * lane], bn.y * bscale[2 * lane + 1]);
    const float2 cn = norm64(bf2(pr + d.off_c + 2 * lane), d.eps, r);
    st_bf2(c_out + size_t(row) * 64 + 2 * lane, cn.x * cscale[2 * lane], cn.y * cscale[2 * lane + 1]);
    if (lane < d.heads) {
      const float t = softplus(bf(pr + d.off_dt + lane) + dt_bias[lane]);
      const float a = -fmaxf(heavy_tail(bf(pr + d.off_a + lane)), 1e-4f);
      dt[size_t(row) * d.heads + lane] = t;
      adt[size_t(row) * d.heads + lane] = a * t;
      trap[size_t(row) * d.heads + lane] = bf(pr + d.off_trap + lane);
    }
    if (lane < d.angles) ang[size_t(row) * d.angles + lane] = bf(pr + d.off_ang + lane);
  }
}

// After the scan: out = rd((y + x D_h) silu(z)).
__global__ void __launch_bounds__(256) mixer_post_fwd(Mix d, const bf16* __restrict__ proj,
                                                      const bf16* __restrict__ y, const float* __restrict__ D,
                                                      bf16* __restrict__ out) {
  const int groups = d.inner / 8;
  const size_t total = size_t(d.rows) * groups;
  for (size_t idx = size_t(blockIdx.x) * blockDim.x + threadIdx.x; idx < total; idx += size_t(gridDim.x) * blockDim.x) {
    const size_t row = idx / groups;
    const int c8 = int(idx % groups), h = (8 * c8) / 64;
    const bf16* pr = proj + row * d.width;
    float yv[8], xv[8], zv[8], o[8];
    unpack8(ld16(y + row * d.inner + 8 * c8), yv);
    unpack8(ld16(pr + d.off_x + 8 * c8), xv);
    unpack8(ld16(pr + 8 * c8), zv);
    const float dh = D[h];
#pragma unroll
    for (int e = 0; e < 8; ++e) o[e] = fmaf(xv[e], dh, yv[e]) * (zv[e] * sigmoid(zv[e]));
    st16(out + row * d.inner + 8 * c8, pack8(o));
  }
}

// Backward of mixer_post_fwd: scan cotangent rd(g silu(z)), z gradient into
// the projection gradient, per-warp partials of dD.
__global__ void __launch_bounds__(WPB * 32) mixer_post_bwd(Mix d, const bf16* __restrict__ proj,
                                                          const bf16* __restrict__ y, const float* __restrict__ D,
                                                          const bf16* __restrict__ g_out, bf16* __restrict__ d_y,
                                                          bf16* __restrict__ d_proj, float* __restrict__ dD_part) {
  const int lane = threadIdx.x & 31, G = d.inner / 256;  // 8-element groups per lane
  float dd[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) dd[k] = 0.f;
  for (int row = gwarp(); row < d.rows; row += nwarps()) {
    const bf16* pr = proj + size_t(row) * d.width;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      if (k >= G) break;
      const int col = 8 * (lane + 32 * k), h = col / 64;
      float yv[8], xv[8], zv[8], gv[8], dy[8], dz[8];
      unpack8(ld16(y + size_t(row) * d.inner + col), yv);
      unpack8(ld16(pr + d.off_x + col), xv);
      unpack8(ld16(pr + col), zv);
      unpack8(ld16(g_out + size_t(row) * d.inner + col), gv);
      const float dh = D[h];
      float acc = 0.f;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float s = sigmoid(zv[e]), y32 = fmaf(xv[e], dh, yv[e]);
        dy[e] = gv[e] * (zv[e] * s);
        dz[e] = gv[e] * y32 * s * (1.f + zv[e] * (1.f - s));
        acc = fmaf(dy[e], xv[e], acc);
      }
      dd[k] += acc;
      st16(d_y + size_t(row) * d.inner + col, pack8(dy));
      st16(d_proj + size_t(row) * d.width + col, pack8(dz));
    }
  }
  // Lanes 8j..8j+7 share head j + 4k.
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    if (k >= G) break;
    float v = dd[k];
    v += __shfl_xor_sync(0xffffffffu, v, 1);
    v += __shfl_xor_sync(0xffffffffu, v, 2);
    v += __shfl_xor_sync(0xffffffffu, v, 4);
    if ((lane & 7) == 0) dD_part[size_t(gwarp()) * d.heads + lane / 8 + 4 * k] = v;
  }
}

// Backward of mixer_prep_fwd plus the x path of the D skip: writes every
// projection-gradient column except z, and per-warp partials of the B/C norm
// scales and dt_bias.
__global__ void __launch_bounds__(WPB * 32) mixer_prep_bwd(
    Mix d, const bf16* __restrict__ proj, const float* __restrict__ bscale, const float* __restrict__ cscale,
    const float* __restrict__ dt_bias, const float* __restrict__ D, const bf16* __restrict__ g_out,
    const bf16* __restrict__ dc, const bf16* __restrict__ db, const bf16* __restrict__ dx,
    const float* __restrict__ d_adt, const float* __restrict__ d_dt, const float* __restrict__ d_trap,
    const float* __restrict__ d_ang, bf16* __restrict__ d_proj, float* __restrict__ bs_part,
    float* __restrict__ cs_part, float* __restrict__ dtb_part) {
  const int lane = threadIdx.x & 31, G = d.inner / 256;
  float sb0 = 0.f, sb1 = 0.f, sc0 = 0.f, sc1 = 0.f, sdt = 0.f;
  const float2 bsc = make_float2(bscale[2 * lane], bscale[2 * lane + 1]);
  const float2 csc = make_float2(cscale[2 * lane], cscale[2 * lane + 1]);
  for (int row = gwarp(); row < d.rows; row += nwarps()) {
    const bf16* pr = proj + size_t(row) * d.width;
    bf16* gp = d_proj + size_t(row) * d.width;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      if (k >= G) break;
      const int col = 8 * (lane + 32 * k), h = col / 64;
      float xs[8], zv[8], gv[8], o[8];
      unpack8(ld16(dx + size_t(row) * d.inner + col), xs);
      unpack8(ld16(pr + col), zv);
      unpack8(ld16(g_out + size_t(row) * d.inner + col), gv);
      const float dh = D[h];
#pragma unroll
      for (int e = 0; e < 8; ++e) o[e] = fmaf(gv[e] * (zv[e] * sigmoid(zv[e])), dh, xs[e]);
      st16(gp + d.off_x + col, pack8(o));
    }
    // Norm backward: dx = r (g s - xhat mean(g s xhat)).
    {
      float r;
      const float2 xh = norm64(bf2(pr + d.off_b + 2 * lane), d.eps, r);
      const float2 g = bf2(db + size_t(row) * 64 + 2 * lane);
      const float gs0 = g.x * bsc.x, gs1 = g.y * bsc.y;
      const float m = warp_sum(gs0 * xh.x + gs1 * xh.y) * (1.f / 64.f);
      st_bf2(gp + d.off_b + 2 * lane, r * (gs0 - xh.x * m), r * (gs1 - xh.y * m));
      sb0 = fmaf(g.x, xh.x, sb0);
      sb1 = fmaf(g.y, xh.y, sb1);
    }
    {
      float r;
      const float2 xh = norm64(bf2(pr + d.off_c + 2 * lane), d.eps, r);
      const float2 g = bf2(dc + size_t(row) * 64 + 2 * lane);
      const float gs0 = g.x * csc.x, gs1 = g.y * csc.y;
      const float m = warp_sum(gs0 * xh.x + gs1 * xh.y) * (1.f / 64.f);
      st_bf2(gp + d.off_c + 2 * lane, r * (gs0 - xh.x * m), r * (gs1 - xh.y * m));
      sc0 = fmaf(g.x, xh.x, sc0);
      sc1 = fmaf(g.y, xh.y, sc1);
    }
    if (lane < d.heads) {
      const size_t i = size_t(row) * d.heads + lane;
      const float pre = bf(pr + d.off_dt + lane) + dt_bias[lane];
      const float t = softplus(pre);
      const float ra = bf(pr + d.off_a + lane), ht = heavy_tail(ra);
      const float a = -fmaxf(ht, 1e-4f);
      const float g_adt = d_adt[i];
      const float g_pre = (d_dt[i] + g_adt * a) * softplus_grad(pre);
      const float g_ra = ht >= 1e-4f ? -(g_adt * t) * heavy_tail_grad(ra) : 0.f;
      gp[d.off_dt + lane] = __float2bfloat16_rn(g_pre);
      gp[d.off_a + lane] = __float2bfloat16_rn(g_ra);
      gp[d.off_trap + lane] = __float2bfloat16_rn(d_trap[i]);
      sdt += g_pre;
    }
    if (lane < d.angles) gp[d.off_ang + lane] = __float2bfloat16_rn(d_ang[size_t(row) * d.angles + lane]);
  }
  const size_t w = gwarp();
  bs_part[w * 64 + 2 * lane] = sb0;
  bs_part[w * 64 + 2 * lane + 1] = sb1;
  cs_part[w * 64 + 2 * lane] = sc0;
  cs_part[w * 64 + 2 * lane + 1] = sc1;
  if (lane < d.heads) dtb_part[w * d.heads + lane] = sdt;
}

// out[j] = sum_w part[w][j] for j < cols, fixed order: 256 strided partial sums
// per column, then a shared-memory tree.
__global__ void __launch_bounds__(256) colsum_kernel(const float* __restrict__ part, int nrows, int cols,
                                                     float* __restrict__ out) {
  __shared__ float red[256];
  const int j = blockIdx.x;
  float acc = 0.f;
  for (int w = threadIdx.x; w < nrows; w += 256) acc += part[size_t(w) * cols + j];
  red[threadIdx.x] = acc;
  __syncthreads();
#pragma unroll
  for (int s = 128; s > 0; s >>= 1) {
    if (threadIdx.x < s) red[threadIdx.x] += red[threadIdx.x + s];
    __syncthreads();
  }
  if (threadIdx.x == 0) out[j] = red[0];
}

// bf16 RMSNorm over F = 32 * VEC * NV features (one warp per row): each lane
// owns NV groups of VEC consecutive features.
template <int NV>
__global__ void __launch_bounds__(WPB * 32) rms_fwd(int rows, float eps, const bf16* __restrict__ x,
                                                   const float* __restrict__ scale, bf16* __restrict__ y,
                                                   float* __restrict__ rstd) {
  constexpr int F = 256 * NV;
  const int lane = threadIdx.x & 31;
  for (int row = gwarp(); row < rows; row += nwarps()) {
    float v[NV][8];
    float ss = 0.f;
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      unpack8(ld16(x + size_t(row) * F + 8 * (lane + 32 * k)), v[k]);
#pragma unroll
      for (int e = 0; e < 8; ++e) ss = fmaf(v[k][e], v[k][e], ss);
    }
    const float r = rsqrtf(warp_sum(ss) * (1.f / F) + eps);
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const int col = 8 * (lane + 32 * k);
      float o[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) o[e] = v[k][e] * r * scale[col + e];
      st16(y + size_t(row) * F + col, pack8(o));
    }
    if (lane == 0) rstd[row] = r;
  }
}

template <int NV>
__global__ void __launch_bounds__(WPB * 32) rms_bwd(int rows, const bf16* __restrict__ x,
                                                   const float* __restrict__ scale, const float* __restrict__ rstd,
                                                   const bf16* __restrict__ gy, bf16* __restrict__ gx,
                                                   float* __restrict__ gs_part) {
  constexpr int F = 256 * NV;
  const int lane = threadIdx.x & 31;
  float acc[NV][8];
#pragma unroll
  for (int k = 0; k < NV; ++k)
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[k][e] = 0.f;
  for (int row = gwarp(); row < rows; row += nwarps()) {
    const float r = rstd[row];
    float xh[NV][8], gsv[NV][8];
    float dot = 0.f;
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const int col = 8 * (lane + 32 * k);
      float g[8];
      unpack8(ld16(x + size_t(row) * F + col), xh[k]);
      unpack8(ld16(gy + size_t(row) * F + col), g);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        xh[k][e] *= r;
        gsv[k][e] = g[e] * scale[col + e];
        dot = fmaf(gsv[k][e], xh[k][e], dot);
        acc[k][e] = fmaf(g[e], xh[k][e], acc[k][e]);
      }
    }
    const float m = warp_sum(dot) * (1.f / F);
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      float o[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) o[e] = r * (gsv[k][e] - xh[k][e] * m);
      st16(gx + size_t(row) * F + 8 * (lane + 32 * k), pack8(o));
    }
  }
#pragma unroll
  for (int k = 0; k < NV; ++k)
#pragma unroll
    for (int e = 0; e < 8; ++e) gs_part[size_t(gwarp()) * F + 8 * (lane + 32 * k) + e] = acc[k][e];
}

inline int row_blocks(int rows) {
  int sms = 148;
  int dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int need = (rows + WPB - 1) / WPB;
  return need < 4 * sms ? need : 4 * sms;
}

inline int check_mix(const M4MixerDims* m) {
  if (!m) return M4_ERR_NULL;
  if (m->rows <= 0 || m->inner <= 0 || m->heads <= 0 || m->angles < 0) return M4_ERR_DIMS;
  if (m->inner % 256 != 0 || m->inner > 2048 || m->heads > 32 || m->angles > 32 || m->inner != 64 * m->heads)
    return M4_ERR_UNSUPPORTED;
  if (m->stride % 8 != 0 || m->stride < 2 * m->inner + 128 + 3 * m->heads + m->angles) return M4_ERR_UNSUPPORTED;
  return M4_OK;
}

}  // namespace glue
}  // namespace m4

using namespace m4;
using namespace m4::glue;

extern "C" size_t m4_mixer_partial_rows(const M4MixerDims* m) {
  return check_mix(m) == M4_OK ? size_t(row_blocks(m->rows)) * WPB : 0;
}

extern "C" int m4_mixer_prep_fwd(const M4MixerDims* m, const void* proj, const float* bscale, const float* cscale,
                                 const float* dt_bias, void* c_out, void* b_out, void* x_out, float* adt, float* dt,
                                 float* trap, float* angles, void* stream) {
  const int st = check_mix(m);
  if (st != M4_OK) return st;
  const Mix d = make_mix(*m);
  mixer_prep_fwd<<<row_blocks(d.rows), WPB * 32, 0, static_cast<cudaStream_t>(stream)>>>(
      d, static_cast<const bf16*>(proj), bscale, cscale, dt_bias, static_cast<bf16*>(c_out),
      static_cast<bf16*>(b_out), static_cast<bf16*>(x_out), adt, dt, trap, angles);
  return launch_status();
}

extern "C" int m4_mixer_post_fwd(const M4MixerDims* m, const void* proj, const void* y, const float* D, void* out,
                                 void* stream) {
  const int st = check_mix(m);
  if (st != M4_OK) return st;
  const Mix d = make_mix(*m);
  const size_t total = size_t(d.rows) * (d.inner / 8);
  const unsigned blocks = unsigned(std::min<size_t>((total + 255) / 256, size_t(148) * 16));
  mixer_post_fwd<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      d, static_cast<const bf16*>(proj), static_cast<const bf16*>(y), D, static_cast<bf16*>(out));
  return launch_status();
}

extern "C" int m4_mixer_post_bwd(const M4MixerDims* m, const void* proj, const void* y, const float* D,
                                 const void* g_out, void* d_y, void* d_proj, float* dD_part, float* dD,
                                 void* stream) {
  const int st = check_mix(m);
  if (st != M4_OK) return st;
  const Mix d = make_mix(*m);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int blocks = row_blocks(d.rows);
  mixer_post_bwd<<<blocks, WPB * 32, 0, s>>>(d, static_cast<const bf16*>(proj), static_cast<const bf16*>(y), D,
                                              static_cast<const bf16*>(g_out), static_cast<bf16*>(d_y),
                                              static_cast<bf16*>(d_proj), dD_part);
  colsum_kernel<<<d.heads, 256, 0, s>>>(dD_part, blocks * WPB, d.heads, dD);
  return launch_status();
}

extern "C" int m4_mixer_prep_bwd(const M4MixerDims* m, const void* proj, const float* bscale, const float* cscale,
                                 const float* dt_bias, const float* D, const void* g_out, const void* dc,
                                 const void* db, const void* dx, const float* d_adt, const float* d_dt,
                                 const float* d_trap, const float* d_angles, void* d_proj, float* part,
                                 float* d_bscale, float* d_cscale, float* d_dt_bias, void* stream) {
  const int st = check_mix(m);
  if (st != M4_OK) return st;
  const Mix d = make_mix(*m);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int blocks = row_blocks(d.rows), nw = blocks * WPB;
  float* bs_part = part;
  float* cs_part = part + size_t(nw) * 64;
  float* dtb_part = part + size_t(nw) * 128;
  mixer_prep_bwd<<<blocks, WPB * 32, 0, s>>>(
      d, static_cast<const bf16*>(proj), bscale, cscale, dt_bias, D, static_cast<const bf16*>(g_out),
      static_cast<const bf16*>(dc), static_cast<const bf16*>(db), static_cast<const bf16*>(dx), d_adt, d_dt,
      d_trap, d_angles, static_cast<bf16*>(d_proj), bs_part, cs_part, dtb_part);
  colsum_kernel<<<64, 256, 0, s>>>(bs_part, nw, 64, d_bscale);
  colsum_kernel<<<64, 256, 0, s>>>(cs_part, nw, 64, d_cscale);
  colsum_kernel<<<d.heads, 256, 0, s>>>(dtb_part, nw, d.heads, d_dt_bias);
  return launch_status();
}

extern "C" size_t m4_rmsnorm_partial_rows(int rows) { return rows > 0 ? size_t(row_blocks(rows)) * WPB : 0; }

extern "C" int m4_rmsnorm_fwd(int rows, int features, float eps, const void* x, const float* scale, void* y,
                              float* rstd, void* stream) {
  if (!x || !scale || !y || !rstd) return M4_ERR_NULL;
  if (rows <= 0) return M4_ERR_DIMS;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int blocks = row_blocks(rows);
  const bf16* xi = static_cast<const bf16*>(x);
  bf16* yo = static_cast<bf16*>(y);
  switch (features) {
    case 256: rms_fwd<1><<<blocks, WPB * 32, 0, s>>>(rows, eps, xi, scale, yo, rstd); break;
    case 512: rms_fwd<2><<<blocks, WPB * 32, 0, s>>>(rows, eps, xi, scale, yo, rstd); break;
    case 768: rms_fwd<3><<<blocks, WPB * 32, 0, s>>>(rows, eps, xi, scale, yo, rstd); break;
    case 1024: rms_fwd<4><<<blocks, WPB * 32, 0, s>>>(rows, eps, xi, scale, yo, rstd); break;
    default: return M4_ERR_UNSUPPORTED;
  }
  return launch_status();
}

extern "C" int m4_rmsnorm_bwd(int rows, int features, const void* x, const float* scale, const float* rstd,
                              const void* gy, void* gx, float* part, float* gscale, void* stream) {
  if (!x || !scale || !rstd || !gy || !gx || !part || !gscale) return M4_ERR_NULL;
  if (rows <= 0) return M4_ERR_DIMS;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int blocks = row_blocks(rows);
  const bf16* xi = static_cast<const bf16*>(x);
  const bf16* g = static_cast<const bf16*>(gy);
  bf16* o = static_cast<bf16*>(gx);
  switch (features) {
    case 256: rms_bwd<1><<<blocks, WPB * 32, 0, s>>>(rows, xi, scale, rstd, g, o, part); break;
    case 512: rms_bwd<2><<<blocks, WPB * 32, 0, s>>>(rows, xi, scale, rstd, g, o, part); break;
    case 768: rms_bwd<3><<<blocks, WPB * 32, 0, s>>>(rows, xi, scale, rstd, g, o, part); break;
    case 1024: rms_bwd<4><<<blocks, WPB * 32, 0, s>>>(rows, xi, scale, rstd, g, o, part); break;
    default: return M4_ERR_UNSUPPORTED;
  }
  colsum_kernel<<<features, 256, 0, s>>>(part, blocks * WPB, features, gscale);
  return launch_status();
}
