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

// 1 / (1 + e^-x) with the correctly rounded reciprocal (the same value as the
// IEEE division, without the division's slow path).
M4_DEV float sigmoid(float x) { return __frcp_rn(1.f + expf(-x)); }
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
  int nb;                                  // width of the B and C slices (state dim)
  float eps;
  int off_x, off_b, off_c, off_dt, off_a, off_trap, off_ang;
};

inline Mix make_mix(const M4MixerDims& m) {
  Mix d;
  d.rows = m.rows; d.inner = m.inner; d.heads = m.heads; d.angles = m.angles; d.eps = m.eps;
  d.nb = m.state_dim;
  d.off_x = m.inner;
  d.off_b = 2 * m.inner;
  d.off_c = d.off_b + d.nb;
  d.off_dt = d.off_c + d.nb;
  d.off_a = d.off_dt + m.heads;
  d.off_trap = d.off_a + m.heads;
  d.off_ang = d.off_trap + m.heads;
  d.width = m.stride;
  return d;
}

constexpr int WPB = 8;  // warps per block

M4_DEV int gwarp() { return blockIdx.x * WPB + (threadIdx.x >> 5); }
M4_DEV int nwarps() { return gridDim.x * WPB; }

// RMSNorm of an nb-wide bf16 slice (nb in {64, 96, 128}): lane l holds
// elements l + 32 j (j < nb / 32; the rest zero); returns the normalised
// values in v and the inverse rms.
M4_DEV float norm_slice(const bf16* p, int nb, float eps, float (&v)[4]) {
  const int lane = threadIdx.x & 31;
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    v[j] = 32 * j < nb ? bf(p + lane + 32 * j) : 0.f;
    ss = fmaf(v[j], v[j], ss);
  }
  const float r = rsqrtf(warp_sum(ss) / float(nb) + eps);
#pragma unroll
  for (int j = 0; j < 4; ++j) v[j] *= r;
  return r;
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
    float bn[4], cn[4];
    norm_slice(pr + d.off_b, d.nb, d.eps, bn);
    norm_slice(pr + d.off_c, d.nb, d.eps, cn);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int n = lane + 32 * j;
      if (n < d.nb) {
        b_out[size_t(row) * d.nb + n] = __float2bfloat16_rn(bn[j] * bscale[n]);
        c_out[size_t(row) * d.nb + n] = __float2bfloat16_rn(cn[j] * cscale[n]);
      }
    }
    if (lane < d.heads) {
      const float t = softplus(bf(pr + d.off_dt + lane) + dt_bias[lane]);
      const float a = -fmaxf(heavy_tail(bf(pr + d.off_a + lane)), 1e-4f);
      dt[size_t(row) * d.heads + lane] = t;
      adt[size_t(row) * d.heads + lane] = a * t;
      trap[size_t(row) * d.heads + lane] = bf(pr + d.off_trap + lane);
    }
    for (int i = lane; i < d.angles; i += 32) ang[size_t(row) * d.angles + i] = bf(pr + d.off_ang + i);
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
  float sb[4] = {0.f, 0.f, 0.f, 0.f}, sc[4] = {0.f, 0.f, 0.f, 0.f}, sdt = 0.f;
  float bsc[4], csc[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int n = lane + 32 * j;
    bsc[j] = n < d.nb ? bscale[n] : 0.f;
    csc[j] = n < d.nb ? cscale[n] : 0.f;
  }
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
#pragma unroll
    for (int which = 0; which < 2; ++which) {
      float xh[4], gs[4], g[4];
      const float r = norm_slice(pr + (which ? d.off_c : d.off_b), d.nb, d.eps, xh);
      const bf16* grow = (which ? dc : db) + size_t(row) * d.nb;
      float dot = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int n = lane + 32 * j;
        g[j] = n < d.nb ? bf(grow + n) : 0.f;
        gs[j] = g[j] * (which ? csc[j] : bsc[j]);
        dot = fmaf(gs[j], xh[j], dot);
      }
      const float m = warp_sum(dot) / float(d.nb);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int n = lane + 32 * j;
        if (n < d.nb) gp[(which ? d.off_c : d.off_b) + n] = __float2bfloat16_rn(r * (gs[j] - xh[j] * m));
        if (which) sc[j] = fmaf(g[j], xh[j], sc[j]);
        else sb[j] = fmaf(g[j], xh[j], sb[j]);
      }
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
    for (int i = lane; i < d.angles; i += 32)
      gp[d.off_ang + i] = __float2bfloat16_rn(d_ang[size_t(row) * d.angles + i]);
  }
  const size_t w = gwarp();
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int n = lane + 32 * j;
    if (n < d.nb) {
      bs_part[w * d.nb + n] = sb[j];
      cs_part[w * d.nb + n] = sc[j];
    }
  }
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

// Residual add fused with the next RMSNorm (decode): x_out = rd(x + d),
// y = rd(rmsnorm(x_out) scale). x_out may alias x (each lane reads its own
// columns before writing them).
template <int NV>
__global__ void __launch_bounds__(WPB * 32) add_rms_fwd(int rows, float eps, const bf16* x,
                                                       const bf16* __restrict__ d,
                                                       const float* __restrict__ scale, bf16* x_out,
                                                       bf16* __restrict__ y) {
  constexpr int F = 256 * NV;
  const int lane = threadIdx.x & 31;
  for (int row = gwarp(); row < rows; row += nwarps()) {
    float v[NV][8];
    float ss = 0.f;
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const size_t at = size_t(row) * F + 8 * (lane + 32 * k);
      float a[8], b[8];
      unpack8(ld16(x + at), a);
      unpack8(ld16(d + at), b);
#pragma unroll
      for (int e = 0; e < 8; ++e) v[k][e] = __bfloat162float(__float2bfloat16_rn(a[e] + b[e]));
      st16(x_out + at, pack8(v[k]));
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
  if (m->state_dim != 64 && m->state_dim != 96 && m->state_dim != 128) return M4_ERR_UNSUPPORTED;
  if (m->inner % 256 != 0 || m->inner > 2048 || m->heads > 32 || m->angles > m->state_dim / 2 ||
      m->inner != 64 * m->heads)
    return M4_ERR_UNSUPPORTED;
  if (m->stride % 8 != 0 || m->stride < 2 * m->inner + 2 * m->state_dim + 3 * m->heads + m->angles)
    return M4_ERR_UNSUPPORTED;
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
  if (!all_aligned16(proj, c_out, b_out, x_out, adt, dt, trap, angles)) return M4_ERR_ALIGN;
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
  if (!all_aligned16(proj, y, out)) return M4_ERR_ALIGN;
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
  if (!all_aligned16(proj, y, g_out, d_y, d_proj, dD_part)) return M4_ERR_ALIGN;
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
  if (!all_aligned16(proj, g_out, dc, db, dx, d_adt, d_dt, d_trap, d_angles, d_proj, part)) return M4_ERR_ALIGN;
  const Mix d = make_mix(*m);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int blocks = row_blocks(d.rows), nw = blocks * WPB;
  float* bs_part = part;
  float* cs_part = part + size_t(nw) * d.nb;
  float* dtb_part = part + size_t(nw) * 2 * d.nb;
  mixer_prep_bwd<<<blocks, WPB * 32, 0, s>>>(
      d, static_cast<const bf16*>(proj), bscale, cscale, dt_bias, D, static_cast<const bf16*>(g_out),
      static_cast<const bf16*>(dc), static_cast<const bf16*>(db), static_cast<const bf16*>(dx), d_adt, d_dt,
      d_trap, d_angles, static_cast<bf16*>(d_proj), bs_part, cs_part, dtb_part);
  colsum_kernel<<<d.nb, 256, 0, s>>>(bs_part, nw, d.nb, d_bscale);
  colsum_kernel<<<d.nb, 256, 0, s>>>(cs_part, nw, d.nb, d_cscale);
  colsum_kernel<<<d.heads, 256, 0, s>>>(dtb_part, nw, d.heads, d_dt_bias);
  return launch_status();
}

extern "C" size_t m4_rmsnorm_partial_rows(int rows) { return rows > 0 ? size_t(row_blocks(rows)) * WPB : 0; }

extern "C" int m4_add_rmsnorm_fwd(int rows, int features, float eps, const void* x, const void* delta,
                                  const float* scale, void* x_out, void* y, void* stream) {
  if (!x || !delta || !scale || !x_out || !y) return M4_ERR_NULL;
  if (rows <= 0) return M4_ERR_DIMS;
  if (!all_aligned16(x, delta, x_out, y)) return M4_ERR_ALIGN;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int blocks = row_blocks(rows);
  const bf16* xi = static_cast<const bf16*>(x);
  const bf16* di = static_cast<const bf16*>(delta);
  bf16* xo = static_cast<bf16*>(x_out);
  bf16* yo = static_cast<bf16*>(y);
  switch (features) {
    case 256: add_rms_fwd<1><<<blocks, WPB * 32, 0, s>>>(rows, eps, xi, di, scale, xo, yo); break;
    case 512: add_rms_fwd<2><<<blocks, WPB * 32, 0, s>>>(rows, eps, xi, di, scale, xo, yo); break;
    case 768: add_rms_fwd<3><<<blocks, WPB * 32, 0, s>>>(rows, eps, xi, di, scale, xo, yo); break;
    case 1024: add_rms_fwd<4><<<blocks, WPB * 32, 0, s>>>(rows, eps, xi, di, scale, xo, yo); break;
    default: return M4_ERR_UNSUPPORTED;
  }
  return launch_status();
}

extern "C" int m4_rmsnorm_fwd(int rows, int features, float eps, const void* x, const float* scale, void* y,
                              float* rstd, void* stream) {
  if (!x || !scale || !y || !rstd) return M4_ERR_NULL;
  if (rows <= 0) return M4_ERR_DIMS;
  if (!all_aligned16(x, y)) return M4_ERR_ALIGN;
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
  if (!all_aligned16(x, gy, gx)) return M4_ERR_ALIGN;
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

// ---------------------------------------------------------------------------
// Selective-memory mixer glue (lm/models/mamba4.py:155-260). Key dim 64,
// value dim 128, up to 16 memory heads. The projection columns after
// the gate ("rest", row stride `stride`) hold value [128h], key [64h],
// query [64h], beta_raw [h], dt_raw [h], order_raw [h]; the depthwise causal
// convolution runs over the 256h value/key/query channels.
// ---------------------------------------------------------------------------
namespace m4 {
namespace glue {

struct MemMix {
  int B, T, heads, stride, gstride;  // gstride: row stride of the gate view
  float beta_max;
  // prep, one-token step: only the last token of each row window (T rows of
  // history + current) is written, and its key is not shifted (the caller
  // carries the previous token's key).
  int step;
};

M4_DEV float silu_grad(float x) {
  const float s = sigmoid(x);
  return s * (1.f + x * (1.f - s));
}

// Depthwise causal convolution of 8 channels at (b, t): bias + sum_j w[j] x[t-3+j].
M4_DEV void conv8(const MemMix& d, const bf16* rest, int b, int t, int ch, const float* w_s, const float* bias_s,
                  int C, float (&o)[8]) {
#pragma unroll
  for (int e = 0; e < 8; ++e) o[e] = bias_s[ch + e];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int s = t - 3 + j;
    if (s < 0) continue;
    float x[8];
    unpack8(ld16(rest + (size_t(b) * d.T + s) * d.stride + ch), x);
#pragma unroll
    for (int e = 0; e < 8; ++e) o[e] = fmaf(w_s[j * C + ch + e], x[e], o[e]);
  }
}

// Stage conv weights (minus `bound`) and bias in shared memory: [4][C] + [C].
// 16-byte loads, eight in flight per thread before their stores (C is a
// multiple of 256; w and bias 16-byte aligned).
M4_DEV void stage_conv(const float* w, const float* bias, float bound, int C, float* w_s, float* bias_s) {
  const float4* w4 = reinterpret_cast<const float4*>(w);
  float4* ws4 = reinterpret_cast<float4*>(w_s);
  for (int i0 = threadIdx.x; i0 < C; i0 += 8 * blockDim.x) {
    float4 v[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int i = i0 + u * blockDim.x;
      v[u] = i < C ? w4[i] : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int i = i0 + u * blockDim.x;
      if (i < C) ws4[i] = make_float4(v[u].x - bound, v[u].y - bound, v[u].z - bound, v[u].w - bound);
    }
  }
  const float4* b4 = reinterpret_cast<const float4*>(bias);
  float4* bs4 = reinterpret_cast<float4*>(bias_s);
  for (int i = threadIdx.x; i < C / 4; i += blockDim.x) bs4[i] = b4[i];
  __syncthreads();
}

// Forward: values = silu(conv) [B,T,h,128]; keys = unit(silu(conv_key)) of the
// previous token (zero at t = 0); queries = unit(silu(conv_query)); beta,
// log_decay, order logit [B,T,h]. One warp per token; lane owns channel
// groups lane + 32k (8 channels each), so the 8 lanes 8j..8j+7 hold one
// key/query head and reduce its norm with three shuffles.
__global__ void __launch_bounds__(WPB * 32) mem_prep_fwd(
    MemMix d, const bf16* __restrict__ rest, const float* __restrict__ conv_w, const float* __restrict__ conv_b,
    float bound, const float* __restrict__ beta_bias, const float* __restrict__ dt_bias,
    const float* __restrict__ a_log, float* __restrict__ values, float* __restrict__ keys,
    float* __restrict__ queries, float* __restrict__ beta, float* __restrict__ log_decay,
    float* __restrict__ order_logit) {
  extern __shared__ float smem[];
  const int h = d.heads, C = 256 * h;
  float* w_s = smem;
  float* bias_s = smem + 4 * C;
  stage_conv(conv_w, conv_b, bound, C, w_s, bias_s);
  // Work: over token rows, one warp per row and all its channel groups; in
  // the one-token step one block per sequence, its warps over the groups.
  const int lane = threadIdx.x & 31, rows = d.step ? d.B : d.B * d.T;
  const int row0 = d.step ? blockIdx.x : gwarp(), rstep = d.step ? gridDim.x : nwarps();
  const int k0 = d.step ? threadIdx.x >> 5 : 0, kstep = d.step ? WPB : 1;
  for (int row = row0; row < rows; row += rstep) {
    // Output row `row` is token (b, t); inputs are read at rows b T + s.
    const int b = d.step ? row : row / d.T, t = d.step ? d.T - 1 : row % d.T;
    const int kt = d.step ? t : t - 1;  // token whose key this row writes
    for (int k = k0; k < h; k += kstep) {
      // Channel group lane + 32k: value below 16h, key below 24h, query above.
      const int cg = lane + 32 * k, ch = 8 * cg;
      const int cls = cg < 16 * h ? 0 : (cg < 24 * h ? 1 : 2);
      float o[8];
      if (cls == 1 && kt < 0) {
#pragma unroll
        for (int e = 0; e < 8; ++e) o[e] = 0.f;
      } else {
        conv8(d, rest, b, cls == 1 ? kt : t, ch, w_s, bias_s, C, o);
#pragma unroll
        for (int e = 0; e < 8; ++e) o[e] *= sigmoid(o[e]);
      }
      float ss = 0.f;
#pragma unroll
      for (int e = 0; e < 8; ++e) ss = fmaf(o[e], o[e], ss);
      ss += __shfl_xor_sync(0xffffffffu, ss, 1);
      ss += __shfl_xor_sync(0xffffffffu, ss, 2);
      ss += __shfl_xor_sync(0xffffffffu, ss, 4);
      const float r = cls == 0 ? 1.f : rsqrtf(ss + 1e-6f);
      float* dst = cls == 0 ? values + size_t(row) * 128 * h + ch
                            : (cls == 1 ? keys + size_t(row) * 64 * h + (ch - 128 * h)
                                        : queries + size_t(row) * 64 * h + (ch - 192 * h));
      st4(dst, make_float4(o[0] * r, o[1] * r, o[2] * r, o[3] * r));
      st4(dst + 4, make_float4(o[4] * r, o[5] * r, o[6] * r, o[7] * r));
    }
    if (k0 == 0 && lane < h) {
      const bf16* pr = rest + (size_t(b) * d.T + t) * d.stride + C;
      const size_t i = size_t(row) * h + lane;
      beta[i] = d.beta_max * sigmoid(bf(pr + lane) + beta_bias[lane]);
      log_decay[i] = -expf(a_log[lane]) * softplus(bf(pr + h + lane) + dt_bias[lane]);
      order_logit[i] = bf(pr + 2 * h + lane) + 2.f;
    }
  }
}

// Backward, part 1: cotangent of the convolution output d_conv [B,T,256h]
// (through the SiLU, the unit norms and the key shift) and the head-scalar
// columns of d_rest, with per-warp partials of beta_bias, dt_bias, a_log.
__global__ void __launch_bounds__(WPB * 32) mem_prep_bwd1(
    MemMix d, const bf16* __restrict__ rest, const float* __restrict__ conv_w, const float* __restrict__ conv_b,
    float bound, const float* __restrict__ beta_bias, const float* __restrict__ dt_bias,
    const float* __restrict__ a_log, const float* __restrict__ d_values, const float* __restrict__ d_keys,
    const float* __restrict__ d_queries, const float* __restrict__ d_beta, const float* __restrict__ d_log_decay,
    const float* __restrict__ d_order, float* __restrict__ d_conv, bf16* __restrict__ d_rest,
    float* __restrict__ part) {
  extern __shared__ float smem[];
  const int h = d.heads, C = 256 * h;
  float* w_s = smem;
  float* bias_s = smem + 4 * C;
  stage_conv(conv_w, conv_b, bound, C, w_s, bias_s);
  const int lane = threadIdx.x & 31;
  float pb = 0.f, pd = 0.f, pa = 0.f;
  for (int row = gwarp(); row < d.B * d.T; row += nwarps()) {
    const int b = row / d.T, t = row % d.T;
    for (int k = 0; k < h; ++k) {
      const int cg = lane + 32 * k, ch = 8 * cg;
      const int cls = cg < 16 * h ? 0 : (cg < 24 * h ? 1 : 2);
      float o[8], m[8], gy[8];
      conv8(d, rest, b, t, ch, w_s, bias_s, C, o);
#pragma unroll
      for (int e = 0; e < 8; ++e) m[e] = o[e] * sigmoid(o[e]);
      // The key written at token t is read by token t + 1.
      const bool live = cls != 1 || t + 1 < d.T;
      const float* gsrc = cls == 0 ? d_values + size_t(row) * 128 * h + ch
                                   : (cls == 1 ? d_keys + (size_t(row) + 1) * 64 * h + (ch - 128 * h)
                                               : d_queries + size_t(row) * 64 * h + (ch - 192 * h));
      if (live) {
        const float4 a0 = ld4(gsrc), a1 = ld4(gsrc + 4);
        gy[0] = a0.x; gy[1] = a0.y; gy[2] = a0.z; gy[3] = a0.w;
        gy[4] = a1.x; gy[5] = a1.y; gy[6] = a1.z; gy[7] = a1.w;
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) gy[e] = 0.f;
      }
      float ss = 0.f, dot = 0.f;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        ss = fmaf(m[e], m[e], ss);
        dot = fmaf(m[e], gy[e], dot);
      }
#pragma unroll
      for (int off = 1; off < 8; off <<= 1) {
        ss += __shfl_xor_sync(0xffffffffu, ss, off);
        dot += __shfl_xor_sync(0xffffffffu, dot, off);
      }
      float dc[8];
      if (cls == 0) {
#pragma unroll
        for (int e = 0; e < 8; ++e) dc[e] = gy[e] * silu_grad(o[e]);
      } else {
        // unit(m) = m r: d m = r (g - u (u . g)), u = m r.
        const float r = rsqrtf(ss + 1e-6f), ug = dot * r;
#pragma unroll
        for (int e = 0; e < 8; ++e) dc[e] = r * (gy[e] - m[e] * r * ug) * silu_grad(o[e]);
      }
      float* dst = d_conv + size_t(row) * C + ch;
      st4(dst, make_float4(dc[0], dc[1], dc[2], dc[3]));
      st4(dst + 4, make_float4(dc[4], dc[5], dc[6], dc[7]));
    }
    if (lane < h) {
      const bf16* pr = rest + size_t(row) * d.stride + C;
      bf16* gr = d_rest + size_t(row) * d.stride + C;
      const size_t i = size_t(row) * h + lane;
      const float bs = sigmoid(bf(pr + lane) + beta_bias[lane]);
      const float g_beta = d_beta[i] * d.beta_max * bs * (1.f - bs);
      const float pre = bf(pr + h + lane) + dt_bias[lane];
      const float rate = expf(a_log[lane]), dt = softplus(pre);
      const float g_ld = d_log_decay[i];
      const float g_pre = -g_ld * rate * softplus_grad(pre);
      gr[lane] = __float2bfloat16_rn(g_beta);
      gr[h + lane] = __float2bfloat16_rn(g_pre);
      gr[2 * h + lane] = __float2bfloat16_rn(d_order[i]);
      pb += g_beta;
      pd += g_pre;
      pa = fmaf(g_ld, -rate * dt, pa);
    }
  }
  if (lane < h) {
    const size_t w = gwarp();
    part[w * 3 * h + lane] = pb;
    part[w * 3 * h + h + lane] = pd;
    part[w * 3 * h + 2 * h + lane] = pa;
  }
}

// Backward, part 2: the depthwise causal convolution. Thread per channel pair,
// block per (64-token tile of one sequence, 512 channels); d_x[t] =
// sum_j w[j] d_conv[t + 3 - j] into d_rest, and per-tile partials of the
// weight ([4][C]) and bias ([C]) gradients (tile-major rows of 5C).
__global__ void __launch_bounds__(256) mem_prep_bwd2(MemMix d, const bf16* __restrict__ rest,
                                                     const float* __restrict__ conv_w, float bound,
                                                     const float* __restrict__ d_conv, bf16* __restrict__ d_rest,
                                                     float* __restrict__ wpart) {
  const int h = d.heads, C = 256 * h;
  const int tiles = (d.T + 63) / 64;
  const int tile = blockIdx.x % tiles, b = blockIdx.x / tiles;
  const int ch = 2 * (blockIdx.y * 256 + threadIdx.x);
  if (ch >= C) return;
  const int t0 = tile * 64, t1 = min(d.T, t0 + 64);
  float w[4][2];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    w[j][0] = conv_w[j * C + ch] - bound;
    w[j][1] = conv_w[j * C + ch + 1] - bound;
  }
  auto dconv = [&](int t) -> float2 {
    return t < d.T ? *reinterpret_cast<const float2*>(d_conv + (size_t(b) * d.T + t) * C + ch) : make_float2(0.f, 0.f);
  };
  auto xin = [&](int t) -> float2 {
    return t >= 0 ? bf2(rest + (size_t(b) * d.T + t) * d.stride + ch) : make_float2(0.f, 0.f);
  };
  float2 g[4], x[4];  // g[j] = d_conv[t + j], x[j] = x[t - 3 + j]
#pragma unroll
  for (int j = 0; j < 3; ++j) {
    g[j + 1] = dconv(t0 + j);
    x[j + 1] = xin(t0 - 3 + j);
  }
  float gw[4][2] = {{0.f, 0.f}, {0.f, 0.f}, {0.f, 0.f}, {0.f, 0.f}}, gb[2] = {0.f, 0.f};
  for (int t = t0; t < t1; ++t) {
#pragma unroll
    for (int j = 0; j < 3; ++j) {
      g[j] = g[j + 1];
      x[j] = x[j + 1];
    }
    g[3] = dconv(t + 3);
    x[3] = xin(t);
    // d_x[t] = sum_j w[j] d_conv[t + 3 - j]
    float dx0 = 0.f, dx1 = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      dx0 = fmaf(w[j][0], g[3 - j].x, dx0);
      dx1 = fmaf(w[j][1], g[3 - j].y, dx1);
    }
    st_bf2(d_rest + (size_t(b) * d.T + t) * d.stride + ch, dx0, dx1);
    // d_w[j] += d_conv[t] x[t - 3 + j]
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      gw[j][0] = fmaf(g[0].x, x[j].x, gw[j][0]);
      gw[j][1] = fmaf(g[0].y, x[j].y, gw[j][1]);
    }
    gb[0] += g[0].x;
    gb[1] += g[0].y;
  }
  float* wp = wpart + size_t(b * tiles + tile) * 5 * C;
#pragma unroll
  for (int j = 0; j < 4; ++j) *reinterpret_cast<float2*>(wp + j * C + ch) = make_float2(gw[j][0], gw[j][1]);
  *reinterpret_cast<float2*>(wp + 4 * C + ch) = make_float2(gb[0], gb[1]);
}

// Order head h_t = lam_t h_(t-1) + (1 - lam_t) v_t, lam = sigmoid(logit)
// (lm/models/mamba4.py:59-95, which evaluates the same recurrence in 64-token
// chunks). Segment-parallel: the sequence splits into OSEG-token segments;
// pass 1 scans each segment from zero (end state, product of lam), pass 2
// carries the segment starts across segments, pass 3 rescans each segment
// from its true start. Blocks per (b, head, segment), thread per channel.
// The backward runs the reverse recurrence G_t = g_t + lam_(t+1) G_(t+1) the
// same way.
constexpr int OSEG = 64, OLA = 16;

__host__ __device__ inline int nseg_of(const MemMix& d) { return (d.T + OSEG - 1) / OSEG; }

// Scan tokens [t0, t1) forward from `state`; optionally write h_t.
M4_DEV float order_run(const MemMix& d, const float* values, const float* logit, int b, int hh, int p, int t0, int t1,
                       float state, float* prod, float* ordered) {
  const int h = d.heads;
  for (int tb = t0; tb < t1; tb += OLA) {
    float v[OLA], l[OLA];
#pragma unroll
    for (int j = 0; j < OLA; ++j) {
      const int t = tb + j;
      const size_t r = size_t(b) * d.T + t;
      v[j] = t < t1 ? values[(r * h + hh) * 128 + p] : 0.f;
      l[j] = t < t1 ? logit[r * h + hh] : 0.f;
    }
#pragma unroll
    for (int j = 0; j < OLA; ++j) {
      const int t = tb + j;
      if (t >= t1) break;
      const float e = expf(-l[j]), lam = __frcp_rn(1.f + e);  // 1 - lam = e lam
      state = fmaf(lam, state, (e * lam) * v[j]);
      if (prod) *prod *= lam;
      if (ordered) ordered[((size_t(b) * d.T + t) * h + hh) * 128 + p] = state;
    }
  }
  return state;
}

__global__ void __launch_bounds__(128) order_seg_fwd(MemMix d, const float* __restrict__ values,
                                                     const float* __restrict__ logit, float* __restrict__ ends,
                                                     float* __restrict__ prods) {
  const int ns = nseg_of(d), seg = blockIdx.x % ns, bh = blockIdx.x / ns, b = bh / d.heads, hh = bh % d.heads;
  const int p = threadIdx.x, t0 = seg * OSEG, t1 = min(d.T, t0 + OSEG);
  float prod = 1.f;
  const float e = order_run(d, values, logit, b, hh, p, t0, t1, 0.f, &prod, nullptr);
  ends[(size_t(bh) * ns + seg) * 128 + p] = e;
  if (p == 0) prods[size_t(bh) * ns + seg] = prod;
}

// Pass 2 (forward): start[s] = start[s-1] prod[s-1] + end[s-1], in place over `ends`.
__global__ void order_carry_fwd(MemMix d, float* __restrict__ ends, const float* __restrict__ prods) {
  const int idx = blockIdx.x * blockDim.x + threadIdx.x, ns = nseg_of(d);
  if (idx >= d.B * d.heads * 128) return;
  const int bh = idx / 128, p = idx % 128;
  float c = 0.f;
  for (int sg = 0; sg < ns; ++sg) {
    float* slot = ends + (size_t(bh) * ns + sg) * 128 + p;
    const float e = *slot;
    *slot = c;
    c = fmaf(prods[size_t(bh) * ns + sg], c, e);
  }
}

__global__ void __launch_bounds__(128) order_fwd(MemMix d, const float* __restrict__ values,
                                                 const float* __restrict__ logit, const float* __restrict__ starts,
                                                 float* __restrict__ ordered) {
  const int ns = nseg_of(d), seg = blockIdx.x % ns, bh = blockIdx.x / ns, b = bh / d.heads, hh = bh % d.heads;
  const int p = threadIdx.x, t0 = seg * OSEG, t1 = min(d.T, t0 + OSEG);
  order_run(d, values, logit, b, hh, p, t0, t1, starts[(size_t(bh) * ns + seg) * 128 + p], nullptr, ordered);
}

// Reverse scan of tokens [t0, t1) from G_(t1) = G (and lam_(t1) = lam_next).
// Pass 1 (out == false): returns the local G_(t0) and the product
// lam_(t0+1) .. lam_(t1) in *prod. Pass 3 (out == true): writes d_values and
// the four per-warp partials of d logit.
template <bool OUT>
M4_DEV float order_back(const MemMix& d, const float* values, const float* logit, const float* ordered,
                        const float* g_ord, int b, int hh, int p, int t0, int t1, float G, float lam_next,
                        float* prod, float* d_values, float* d_logit4) {
  const int h = d.heads, lane = p & 31, warp = p >> 5;
  for (int tb = t1; tb > t0; tb -= OLA) {
    float v[OLA], l[OLA], g[OLA], hp[OLA];
#pragma unroll
    for (int j = 0; j < OLA; ++j) {
      const int t = tb - 1 - j;
      const size_t r = size_t(b) * d.T + t;
      const bool live = t >= t0;
      l[j] = live ? logit[r * h + hh] : 0.f;
      g[j] = live ? g_ord[(r * h + hh) * 128 + p] : 0.f;
      if (OUT) {
        v[j] = live ? values[(r * h + hh) * 128 + p] : 0.f;
        hp[j] = (live && t >= 1) ? ordered[((r - 1) * h + hh) * 128 + p] : 0.f;
      }
    }
#pragma unroll
    for (int j = 0; j < OLA; ++j) {
      const int t = tb - 1 - j;
      if (t < t0) break;
      const float e = expf(-l[j]), lam = __frcp_rn(1.f + e);
      G = fmaf(lam_next, G, g[j]);
      if (!OUT) *prod *= lam_next;
      if (OUT) {
        const float inflow = e * lam;
        const size_t r = size_t(b) * d.T + t;
        d_values[(r * h + hh) * 128 + p] = inflow * G;
        const float dl = warp_sum(G * (hp[j] - v[j])) * lam * inflow;
        if (lane == 0) d_logit4[(r * h + hh) * 4 + warp] = dl;
      }
      lam_next = lam;
    }
  }
  return G;
}

__global__ void __launch_bounds__(128) order_seg_bwd(MemMix d, const float* __restrict__ logit,
                                                     const float* __restrict__ g_ord, float* __restrict__ gstart,
                                                     float* __restrict__ prods) {
  const int ns = nseg_of(d), seg = blockIdx.x % ns, bh = blockIdx.x / ns, b = bh / d.heads, hh = bh % d.heads;
  const int p = threadIdx.x, t0 = seg * OSEG, t1 = min(d.T, t0 + OSEG);
  // lam of the first token of the next segment multiplies the carried G.
  const float lam_next = t1 < d.T ? sigmoid(logit[(size_t(b) * d.T + t1) * d.heads + hh]) : 0.f;
  float prod = 1.f;
  const float G = order_back<false>(d, nullptr, logit, nullptr, g_ord, b, hh, p, t0, t1, 0.f, lam_next, &prod,
                                    nullptr, nullptr);
  gstart[(size_t(bh) * ns + seg) * 128 + p] = G;
  if (p == 0) prods[size_t(bh) * ns + seg] = prod;
}

// Pass 2 (backward, reverse over segments): Gtrue_start[s] = local[s] +
// prod[s] Gtrue_start[s+1]; stored in place as the carry G_(t1) of segment s.
__global__ void order_carry_bwd(MemMix d, float* __restrict__ gstart, const float* __restrict__ prods) {
  const int idx = blockIdx.x * blockDim.x + threadIdx.x, ns = nseg_of(d);
  if (idx >= d.B * d.heads * 128) return;
  const int bh = idx / 128, p = idx % 128;
  float c = 0.f;  // true G at the start of segment s + 1
  for (int sg = ns - 1; sg >= 0; --sg) {
    float* slot = gstart + (size_t(bh) * ns + sg) * 128 + p;
    const float local = *slot;
    *slot = c;
    c = fmaf(prods[size_t(bh) * ns + sg], c, local);
  }
}

__global__ void __launch_bounds__(128) order_bwd(MemMix d, const float* __restrict__ values,
                                                 const float* __restrict__ logit, const float* __restrict__ ordered,
                                                 const float* __restrict__ g_ord, const float* __restrict__ gcarry,
                                                 float* __restrict__ d_values, float* __restrict__ d_logit4) {
  const int ns = nseg_of(d), seg = blockIdx.x % ns, bh = blockIdx.x / ns, b = bh / d.heads, hh = bh % d.heads;
  const int p = threadIdx.x, t0 = seg * OSEG, t1 = min(d.T, t0 + OSEG);
  const float lam_next = t1 < d.T ? sigmoid(logit[(size_t(b) * d.T + t1) * d.heads + hh]) : 0.f;
  order_back<true>(d, values, logit, ordered, g_ord, b, hh, p, t0, t1, gcarry[(size_t(bh) * ns + seg) * 128 + p],
                   lam_next, nullptr, d_values, d_logit4);
}

// After the read: r = out c + D v + sigmoid(order_mix) o with the confidence
// gate c = sigmoid(1 - conf_scale log1p(var)); y = rd(rd(rmsnorm(r) s) silu(gate)).
// One warp per (b, t, head) row of 128 values (float4 per lane).
// STEP (one cached token): the order head advances here,
// o = s o_prev + (1 - s) v with s = sigmoid(order logit) (`ordered` holds the
// logits [rows], o_prev / order_out the carried order state; o_prev null:
// no order head, o = 0), and rstd is not written.
template <bool STEP>
__global__ void __launch_bounds__(WPB * 32) mem_post_fwd(
    MemMix d, float eps, const float* __restrict__ out, const float* __restrict__ var,
    const float* __restrict__ values, const float* __restrict__ ordered, const bf16* __restrict__ gate,
    const float* __restrict__ conf_scale, const float* __restrict__ Dskip, const float* __restrict__ order_mix,
    const float* __restrict__ scale, bf16* __restrict__ y, float* __restrict__ rstd,
    const float* __restrict__ order_prev = nullptr, float* __restrict__ order_out = nullptr) {
  const int lane = threadIdx.x & 31, h = d.heads;
  for (int row = gwarp(); row < d.B * d.T * h; row += nwarps()) {
    const int hh = row % h, tok = row / h;
    const float cg = sigmoid(1.f - conf_scale[hh] * log1pf(var[row]));
    const float dh = Dskip[hh], om = sigmoid(order_mix[hh]);
    const float4 o4 = ld4(out + size_t(row) * 128 + 4 * lane), v4 = ld4(values + size_t(row) * 128 + 4 * lane);
    float4 q4;
    if constexpr (STEP) {
      if (order_prev != nullptr) {
        const float sg = sigmoid(ordered[row]), fl = 1.f - sg;
        const float4 p4 = ld4(order_prev + size_t(row) * 128 + 4 * lane);
        q4 = make_float4(sg * p4.x + fl * v4.x, sg * p4.y + fl * v4.y, sg * p4.z + fl * v4.z,
                         sg * p4.w + fl * v4.w);
        st4(order_out + size_t(row) * 128 + 4 * lane, q4);
      } else {
        q4 = make_float4(0.f, 0.f, 0.f, 0.f);
      }
    } else {
      q4 = ld4(ordered + size_t(row) * 128 + 4 * lane);
    }
    const float r[4] = {fmaf(om, q4.x, fmaf(dh, v4.x, o4.x * cg)), fmaf(om, q4.y, fmaf(dh, v4.y, o4.y * cg)),
                        fmaf(om, q4.z, fmaf(dh, v4.z, o4.z * cg)), fmaf(om, q4.w, fmaf(dh, v4.w, o4.w * cg))};
    const float ss = warp_sum(r[0] * r[0] + r[1] * r[1] + r[2] * r[2] + r[3] * r[3]);
    const float rs = rsqrtf(ss * (1.f / 128.f) + eps);
    const float2 g01 = bf2(gate + size_t(tok) * d.gstride + hh * 128 + 4 * lane);
    const float2 g23 = bf2(gate + size_t(tok) * d.gstride + hh * 128 + 4 * lane + 2);
    const float gz[4] = {g01.x, g01.y, g23.x, g23.y};
    float o[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float n = __bfloat162float(__float2bfloat16_rn(r[e] * rs * scale[4 * lane + e]));
      o[e] = n * (gz[e] * sigmoid(gz[e]));
    }
    bf16* dst = y + size_t(row) * 128 + 4 * lane;
    st_bf2(dst, o[0], o[1]);
    st_bf2(dst + 2, o[2], o[3]);
    if (!STEP && lane == 0) rstd[row] = rs;
  }
}

// Partial-sum row of mem_post_bwd: scale [128], conf_scale, D, order_mix, pad
// (132 floats keep every row 16-byte aligned for the float4 stores).
constexpr int PROW = 132;

// Backward of mem_post_fwd. Per-warp partials (a warp keeps one head because
// the warp count is a multiple of h) in rows of PROW floats.
__global__ void __launch_bounds__(WPB * 32) mem_post_bwd(
    MemMix d, const float* __restrict__ out, const float* __restrict__ var, const float* __restrict__ values,
    const float* __restrict__ ordered, const bf16* __restrict__ gate, const float* __restrict__ conf_scale,
    const float* __restrict__ Dskip, const float* __restrict__ order_mix, const float* __restrict__ scale,
    const float* __restrict__ rstd, const bf16* __restrict__ g_y, float* __restrict__ d_out,
    float* __restrict__ d_var, float* __restrict__ d_values, float* __restrict__ d_ordered,
    bf16* __restrict__ d_gate, float* __restrict__ part) {
  const int lane = threadIdx.x & 31, h = d.heads;
  const float4 sc = ld4(scale + 4 * lane);
  const float s4[4] = {sc.x, sc.y, sc.z, sc.w};
  float ps[4] = {0.f, 0.f, 0.f, 0.f}, pcs = 0.f, pD = 0.f, pom = 0.f;
  for (int row = gwarp(); row < d.B * d.T * h; row += nwarps()) {
    const int hh = row % h, tok = row / h;
    const float lv = log1pf(var[row]), cs = conf_scale[hh];
    const float u = 1.f - cs * lv, cg = sigmoid(u);
    const float dh = Dskip[hh], om = sigmoid(order_mix[hh]);
    const float4 o4 = ld4(out + size_t(row) * 128 + 4 * lane), v4 = ld4(values + size_t(row) * 128 + 4 * lane);
    const float4 q4 = ld4(ordered + size_t(row) * 128 + 4 * lane);
    const float ov[4] = {o4.x, o4.y, o4.z, o4.w}, vv[4] = {v4.x, v4.y, v4.z, v4.w}, qv[4] = {q4.x, q4.y, q4.z, q4.w};
    const float rs = rstd[row];
    const float2 g01 = bf2(gate + size_t(tok) * d.gstride + hh * 128 + 4 * lane);
    const float2 g23 = bf2(gate + size_t(tok) * d.gstride + hh * 128 + 4 * lane + 2);
    const float gz[4] = {g01.x, g01.y, g23.x, g23.y};
    const float2 y01 = bf2(g_y + size_t(row) * 128 + 4 * lane), y23 = bf2(g_y + size_t(row) * 128 + 4 * lane + 2);
    const float gy[4] = {y01.x, y01.y, y23.x, y23.y};
    float rh[4], dn[4], dgz[4], dot = 0.f;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float r = fmaf(om, qv[e], fmaf(dh, vv[e], ov[e] * cg));
      rh[e] = r * rs;
      const float n = __bfloat162float(__float2bfloat16_rn(rh[e] * s4[e]));
      const float sg = sigmoid(gz[e]);
      dn[e] = gy[e] * (gz[e] * sg);
      dgz[e] = gy[e] * n * sg * (1.f + gz[e] * (1.f - sg));
      ps[e] = fmaf(dn[e], rh[e], ps[e]);
      dot = fmaf(dn[e] * s4[e], rh[e], dot);
    }
    const float m = warp_sum(dot) * (1.f / 128.f);
    float dr[4], go = 0.f, gD = 0.f, gq = 0.f;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      dr[e] = rs * (dn[e] * s4[e] - rh[e] * m);
      go = fmaf(dr[e], ov[e], go);
      gD = fmaf(dr[e], vv[e], gD);
      gq = fmaf(dr[e], qv[e], gq);
    }
    st4(d_out + size_t(row) * 128 + 4 * lane, make_float4(dr[0] * cg, dr[1] * cg, dr[2] * cg, dr[3] * cg));
    st4(d_values + size_t(row) * 128 + 4 * lane, make_float4(dr[0] * dh, dr[1] * dh, dr[2] * dh, dr[3] * dh));
    st4(d_ordered + size_t(row) * 128 + 4 * lane, make_float4(dr[0] * om, dr[1] * om, dr[2] * om, dr[3] * om));
    bf16* gg = d_gate + size_t(tok) * d.gstride + hh * 128 + 4 * lane;
    st_bf2(gg, dgz[0], dgz[1]);
    st_bf2(gg + 2, dgz[2], dgz[3]);
    go = warp_sum(go);
    gD = warp_sum(gD);
    gq = warp_sum(gq);
    const float dsg = cg * (1.f - cg);
    if (lane == 0) d_var[row] = go * dsg * (-cs / (1.f + var[row]));
    pcs = fmaf(go * dsg, -lv, pcs);
    pD += gD;
    pom = fmaf(gq, om * (1.f - om), pom);
  }
  float* pw = part + size_t(gwarp()) * PROW;
  st4(pw + 4 * lane, make_float4(ps[0], ps[1], ps[2], ps[3]));
  if (lane == 0) {
    pw[128] = pcs;
    pw[129] = pD;
    pw[130] = pom;
    pw[131] = 0.f;
  }
}

// Per-head sums of the mem_post_bwd partials: warp w holds head w % h. One
// block per head; thread i sums the head's warps i, i + 256, ... and a fixed
// tree (warp sums, then warp 0 over the eight warp totals) finishes, so the
// order of the additions does not depend on scheduling.
__global__ void __launch_bounds__(256) head_sum_kernel(const float* __restrict__ part, int nw, int h,
                                                       float* __restrict__ d_cs, float* __restrict__ d_D,
                                                       float* __restrict__ d_om) {
  __shared__ float red[3][8];
  const int hh = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  float a = 0.f, b = 0.f, c = 0.f;
  for (int w = hh + h * tid; w < nw; w += h * 256) {
    a += part[size_t(w) * PROW + 128];
    b += part[size_t(w) * PROW + 129];
    c += part[size_t(w) * PROW + 130];
  }
  a = warp_sum(a);
  b = warp_sum(b);
  c = warp_sum(c);
  if (lane == 0) {
    red[0][warp] = a;
    red[1][warp] = b;
    red[2][warp] = c;
  }
  __syncthreads();
  if (warp == 0) {
    a = warp_sum(lane < 8 ? red[0][lane] : 0.f);
    b = warp_sum(lane < 8 ? red[1][lane] : 0.f);
    c = warp_sum(lane < 8 ? red[2][lane] : 0.f);
    if (lane == 0) {
      d_cs[hh] = a;
      d_D[hh] = b;
      d_om[hh] = c;
    }
  }
}

inline int mem_blocks(int rows, int h) {
  int blocks = row_blocks(rows);
  blocks = ((blocks + h - 1) / h) * h;  // warp count a multiple of h
  return blocks;
}

inline int check_mem(const M4MemMixDims* m) {
  if (!m) return M4_ERR_NULL;
  if (m->batch <= 0 || m->time <= 0 || m->heads <= 0) return M4_ERR_DIMS;
  if (m->heads > 16 || m->stride % 8 != 0 || m->stride < 259 * m->heads ||
      m->gate_stride % 2 != 0 || m->gate_stride < 128 * m->heads)
    return M4_ERR_UNSUPPORTED;
  return M4_OK;
}

inline MemMix make_memmix(const M4MemMixDims& m) {
  MemMix d;
  d.B = m.batch; d.T = m.time; d.heads = m.heads; d.stride = m.stride; d.gstride = m.gate_stride;
  d.beta_max = m.beta_max;
  d.step = 0;
  return d;
}

}  // namespace glue
}  // namespace m4

extern "C" size_t m4_memmix_partial_floats(const M4MemMixDims* m) {
  if (check_mem(m) != M4_OK) return 0;
  const int h = m->heads, rows = m->batch * m->time, C = 256 * h;
  const size_t nw_prep = size_t(row_blocks(rows)) * WPB;
  const size_t tiles = size_t(m->batch) * ((m->time + 63) / 64);
  const size_t nw_post = size_t(mem_blocks(rows * h, h)) * WPB;
  const size_t a = nw_prep * 3 * h, b = tiles * 5 * C, c = nw_post * PROW;
  return std::max(a, std::max(b, c));
}

extern "C" int m4_memmix_prep_fwd(const M4MemMixDims* m, const void* rest, const float* conv_w, const float* conv_b,
                                  float bound, const float* beta_bias, const float* dt_bias, const float* a_log,
                                  float* values, float* keys, float* queries, float* beta, float* log_decay,
                                  float* order_logit, void* stream) {
  const int st = check_mem(m);
  if (st != M4_OK) return st;
  if (!all_aligned16(rest, conv_w, conv_b, values, keys, queries, beta, log_decay, order_logit)) return M4_ERR_ALIGN;
  const MemMix d = make_memmix(*m);
  const size_t smem = size_t(5) * 256 * d.heads * sizeof(float);
  cudaFuncSetAttribute(mem_prep_fwd, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  mem_prep_fwd<<<row_blocks(d.B * d.T), WPB * 32, smem, static_cast<cudaStream_t>(stream)>>>(
      d, static_cast<const bf16*>(rest), conv_w, conv_b, bound, beta_bias, dt_bias, a_log, values, keys, queries,
      beta, log_decay, order_logit);
  return launch_status();
}

extern "C" int m4_memmix_prep_bwd(const M4MemMixDims* m, const void* rest, const float* conv_w, const float* conv_b,
                                  float bound, const float* beta_bias, const float* dt_bias, const float* a_log,
                                  const float* d_values, const float* d_keys, const float* d_queries,
                                  const float* d_beta, const float* d_log_decay, const float* d_order,
                                  float* d_conv, void* d_rest, float* part, float* d_conv_w, float* d_conv_b,
                                  float* d_beta_bias, float* d_dt_bias, float* d_a_log, void* stream) {
  const int st = check_mem(m);
  if (st != M4_OK) return st;
  if (!all_aligned16(rest, conv_w, conv_b, d_values, d_keys, d_queries, d_conv, d_rest, part)) return M4_ERR_ALIGN;
  const MemMix d = make_memmix(*m);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int h = d.heads, C = 256 * h, rows = d.B * d.T;
  const size_t smem = size_t(5) * C * sizeof(float);
  cudaFuncSetAttribute(mem_prep_bwd1, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  const int blocks = row_blocks(rows), nw = blocks * WPB;
  mem_prep_bwd1<<<blocks, WPB * 32, smem, s>>>(d, static_cast<const bf16*>(rest), conv_w, conv_b, bound, beta_bias,
                                               dt_bias, a_log, d_values, d_keys, d_queries, d_beta, d_log_decay,
                                               d_order, d_conv, static_cast<bf16*>(d_rest), part);
  colsum_kernel<<<h, 256, 0, s>>>(part, nw, 3 * h, d_beta_bias);
  colsum_kernel<<<h, 256, 0, s>>>(part + h, nw, 3 * h, d_dt_bias);
  colsum_kernel<<<h, 256, 0, s>>>(part + 2 * h, nw, 3 * h, d_a_log);
  const int tiles = (d.T + 63) / 64;
  mem_prep_bwd2<<<dim3(d.B * tiles, (C + 511) / 512), 256, 0, s>>>(d, static_cast<const bf16*>(rest), conv_w, bound,
                                                          d_conv, static_cast<bf16*>(d_rest), part);
  colsum_kernel<<<4 * C, 256, 0, s>>>(part, d.B * tiles, 5 * C, d_conv_w);
  colsum_kernel<<<C, 256, 0, s>>>(part + 4 * C, d.B * tiles, 5 * C, d_conv_b);
  return launch_status();
}

extern "C" size_t m4_memmix_order_scratch_floats(const M4MemMixDims* m) {
  if (check_mem(m) != M4_OK) return 0;
  const size_t segs = size_t(m->batch) * m->heads * ((m->time + OSEG - 1) / OSEG);
  return segs * 129;
}

extern "C" int m4_memmix_order_fwd(const M4MemMixDims* m, const float* values, const float* logit, float* ordered,
                                   float* scratch, void* stream) {
  const int st = check_mem(m);
  if (st != M4_OK) return st;
  if (!scratch) return M4_ERR_NULL;
  if (!all_aligned16(values, logit, ordered)) return M4_ERR_ALIGN;
  const MemMix d = make_memmix(*m);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int ns = nseg_of(d), blocks = d.B * d.heads * ns, lanes = d.B * d.heads * 128;
  float* ends = scratch;
  float* prods = scratch + size_t(blocks) * 128;
  order_seg_fwd<<<blocks, 128, 0, s>>>(d, values, logit, ends, prods);
  order_carry_fwd<<<(lanes + 255) / 256, 256, 0, s>>>(d, ends, prods);
  order_fwd<<<blocks, 128, 0, s>>>(d, values, logit, ends, ordered);
  return launch_status();
}

extern "C" int m4_memmix_order_bwd(const M4MemMixDims* m, const float* values, const float* logit,
                                   const float* ordered, const float* g_ordered, float* d_values, float* d_logit4,
                                   float* scratch, void* stream) {
  const int st = check_mem(m);
  if (st != M4_OK) return st;
  if (!scratch) return M4_ERR_NULL;
  if (!all_aligned16(values, logit, ordered, g_ordered, d_values, d_logit4)) return M4_ERR_ALIGN;
  const MemMix d = make_memmix(*m);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int ns = nseg_of(d), blocks = d.B * d.heads * ns, lanes = d.B * d.heads * 128;
  float* gstart = scratch;
  float* prods = scratch + size_t(blocks) * 128;
  order_seg_bwd<<<blocks, 128, 0, s>>>(d, logit, g_ordered, gstart, prods);
  order_carry_bwd<<<(lanes + 255) / 256, 256, 0, s>>>(d, gstart, prods);
  order_bwd<<<blocks, 128, 0, s>>>(d, values, logit, ordered, g_ordered, gstart, d_values, d_logit4);
  return launch_status();
}

extern "C" int m4_memmix_post_fwd(const M4MemMixDims* m, float eps, const float* out, const float* var,
                                  const float* values, const float* ordered, const void* gate,
                                  const float* conf_scale, const float* D, const float* order_mix,
                                  const float* scale, void* y, float* rstd, void* stream) {
  const int st = check_mem(m);
  if (st != M4_OK) return st;
  if (!all_aligned16(out, var, values, ordered, gate, scale, y, rstd)) return M4_ERR_ALIGN;
  const MemMix d = make_memmix(*m);
  const int rows = d.B * d.T * d.heads;
  mem_post_fwd<false><<<mem_blocks(rows, d.heads), WPB * 32, 0, static_cast<cudaStream_t>(stream)>>>(
      d, eps, out, var, values, ordered, static_cast<const bf16*>(gate), conf_scale, D, order_mix, scale,
      static_cast<bf16*>(y), rstd);
  return launch_status();
}

extern "C" int m4_memmix_prep_step(const M4MemMixDims* m, const void* rest, const float* conv_w,
                                   const float* conv_b, float bound, const float* beta_bias, const float* dt_bias,
                                   const float* a_log, float* values, float* keys, float* queries, float* beta,
                                   float* log_decay, float* order_logit, void* stream) {
  const int st = check_mem(m);
  if (st != M4_OK) return st;
  if (!all_aligned16(rest, conv_w, conv_b, values, keys, queries, beta, log_decay, order_logit)) return M4_ERR_ALIGN;
  MemMix d = make_memmix(*m);
  d.step = 1;
  const size_t smem = size_t(5) * 256 * d.heads * sizeof(float);
  cudaFuncSetAttribute(mem_prep_fwd, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  mem_prep_fwd<<<std::min(d.B, 4 * 148), WPB * 32, smem, static_cast<cudaStream_t>(stream)>>>(
      d, static_cast<const bf16*>(rest), conv_w, conv_b, bound, beta_bias, dt_bias, a_log, values, keys, queries,
      beta, log_decay, order_logit);
  return launch_status();
}

extern "C" int m4_memmix_post_step(const M4MemMixDims* m, float eps, const float* out, const float* var,
                                   const float* values, const float* order_logit, const float* order_prev,
                                   float* order_out, const void* gate, const float* conf_scale, const float* D,
                                   const float* order_mix, const float* scale, void* y, void* stream) {
  const int st = check_mem(m);
  if (st != M4_OK) return st;
  if (m->time != 1) return M4_ERR_DIMS;
  if ((order_prev == nullptr) != (order_out == nullptr)) return M4_ERR_DIMS;
  if (!all_aligned16(out, var, values, gate, scale, y)) return M4_ERR_ALIGN;
  if (order_prev != nullptr && !all_aligned16(order_logit, order_prev, order_out)) return M4_ERR_ALIGN;
  const MemMix d = make_memmix(*m);
  const int rows = d.B * d.heads;
  mem_post_fwd<true><<<mem_blocks(rows, d.heads), WPB * 32, 0, static_cast<cudaStream_t>(stream)>>>(
      d, eps, out, var, values, order_logit, static_cast<const bf16*>(gate), conf_scale, D, order_mix, scale,
      static_cast<bf16*>(y), nullptr, order_prev, order_out);
  return launch_status();
}

extern "C" int m4_memmix_post_bwd(const M4MemMixDims* m, const float* out, const float* var, const float* values,
                                  const float* ordered, const void* gate, const float* conf_scale, const float* D,
                                  const float* order_mix, const float* scale, const float* rstd, const void* g_y,
                                  float* d_out, float* d_var, float* d_values, float* d_ordered, void* d_gate,
                                  float* part, float* d_conf_scale, float* d_D, float* d_order_mix,
                                  float* d_scale, void* stream) {
  const int st = check_mem(m);
  if (st != M4_OK) return st;
  if (!all_aligned16(out, values, ordered, gate, scale, g_y, d_out, d_values, d_ordered, d_gate, part)) return M4_ERR_ALIGN;
  const MemMix d = make_memmix(*m);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int rows = d.B * d.T * d.heads, blocks = mem_blocks(rows, d.heads), nw = blocks * WPB;
  mem_post_bwd<<<blocks, WPB * 32, 0, s>>>(d, out, var, values, ordered, static_cast<const bf16*>(gate), conf_scale,
                                           D, order_mix, scale, rstd, static_cast<const bf16*>(g_y), d_out, d_var,
                                           d_values, d_ordered, static_cast<bf16*>(d_gate), part);
  colsum_kernel<<<128, 256, 0, s>>>(part, nw, PROW, d_scale);
  head_sum_kernel<<<d.heads, 256, 0, s>>>(part, nw, d.heads, d_conf_scale, d_D, d_order_mix);
  return launch_status();
}

// ---------------------------------------------------------------------------
// Cross-entropy over bf16 logits (lm/train.py:81-87: logits cast to float32,
// optax softmax cross-entropy with integer labels). Forward: per-row loss and
// log-sum-exp from one streaming pass; backward: the logits buffer is
// overwritten with g_r (softmax - onehot), in bf16.
// ---------------------------------------------------------------------------
namespace m4 {
namespace glue {

constexpr int CE_THREADS = 512;

M4_DEV void lse_merge(float& m, float& s, float m2, float s2) {
  const float mx = fmaxf(m, m2);
  s = (m == -INFINITY ? 0.f : s * expf(m - mx)) + (m2 == -INFINITY ? 0.f : s2 * expf(m2 - mx));
  m = mx;
}

__global__ void __launch_bounds__(CE_THREADS) ce_fwd(int vocab, int ld, const bf16* __restrict__ logits,
                                                     const int64_t* __restrict__ targets, float* __restrict__ loss,
                                                     float* __restrict__ lse) {
  __shared__ float red_m[CE_THREADS / 32], red_s[CE_THREADS / 32];
  const int row = blockIdx.x, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const bf16* lr = logits + size_t(row) * ld;
  float m = -INFINITY, s = 0.f;
  for (int k = threadIdx.x; k < (vocab + 7) / 8; k += CE_THREADS) {
    float v[8];
    unpack8(ld16(lr + 8 * k), v);
#pragma unroll
    for (int e = 0; e < 8; ++e)
      if (8 * k + e >= vocab) v[e] = -INFINITY;
    float bm = v[0];
#pragma unroll
    for (int e = 1; e < 8; ++e) bm = fmaxf(bm, v[e]);
    float bs = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) bs += expf(v[e] - bm);
    lse_merge(m, s, bm, bs);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, o), s2 = __shfl_xor_sync(0xffffffffu, s, o);
    lse_merge(m, s, m2, s2);
  }
  if (lane == 0) {
    red_m[warp] = m;
    red_s[warp] = s;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float M = red_m[0], S = red_s[0];
    for (int w = 1; w < CE_THREADS / 32; ++w) lse_merge(M, S, red_m[w], red_s[w]);
    const float l = M + logf(S);
    lse[row] = l;
    const int64_t tg = targets[row];
    loss[row] = (tg >= 0 && tg < vocab) ? l - __bfloat162float(lr[tg]) : 0.f;
  }
}

__global__ void __launch_bounds__(CE_THREADS) ce_bwd(int vocab, int ld, bf16* __restrict__ logits,
                                                     const int64_t* __restrict__ targets,
                                                     const float* __restrict__ lse, const float* __restrict__ g) {
  const int row = blockIdx.x;
  bf16* lr = logits + size_t(row) * ld;
  const float gr = g[row], l = lse[row];
  const int64_t tg = targets[row];
  for (int k = threadIdx.x; k < ld / 8; k += CE_THREADS) {
    float v[8];
    unpack8(ld16(lr + 8 * k), v);
#pragma unroll
    for (int e = 0; e < 8; ++e)
      v[e] = 8 * k + e < vocab ? gr * (expf(v[e] - l) - (8 * k + e == tg ? 1.f : 0.f)) : 0.f;
    st16(lr + 8 * k, pack8(v));
  }
}

}  // namespace glue
}  // namespace m4

extern "C" int m4_cross_entropy_fwd(int rows, int vocab, int ld, const void* logits, const int64_t* targets,
                                    float* loss, float* lse, void* stream) {
  if (!logits || !targets || !loss || !lse) return M4_ERR_NULL;
  if (rows <= 0 || vocab <= 0 || ld < vocab) return M4_ERR_DIMS;
  if (ld % 8 != 0) return M4_ERR_UNSUPPORTED;
  if (!all_aligned16(logits)) return M4_ERR_ALIGN;
  ce_fwd<<<rows, CE_THREADS, 0, static_cast<cudaStream_t>(stream)>>>(vocab, ld, static_cast<const bf16*>(logits),
                                                                      targets, loss, lse);
  return launch_status();
}

extern "C" int m4_cross_entropy_bwd(int rows, int vocab, int ld, void* logits, const int64_t* targets,
                                    const float* lse, const float* g, void* stream) {
  if (!logits || !targets || !lse || !g) return M4_ERR_NULL;
  if (rows <= 0 || vocab <= 0 || ld < vocab) return M4_ERR_DIMS;
  if (ld % 8 != 0) return M4_ERR_UNSUPPORTED;
  if (!all_aligned16(logits)) return M4_ERR_ALIGN;
  ce_bwd<<<rows, CE_THREADS, 0, static_cast<cudaStream_t>(stream)>>>(vocab, ld, static_cast<bf16*>(logits), targets,
                                                                      lse, g);
  return launch_status();
}
