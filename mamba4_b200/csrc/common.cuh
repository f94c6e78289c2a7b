// Shared device helpers for the mamba4_b200 kernels (sm_100a).
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "../../include/mamba4_b200.h"

#define M4_DEV __device__ __forceinline__

namespace m4 {

constexpr int kWarp = 32;

M4_DEV float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Inclusive prefix sum over a warp (Kogge-Stone).
M4_DEV float warp_inclusive_scan(float v, int lane) {
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    float n = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v += n;
  }
  return v;
}

M4_DEV float4 ld4(const float* p) { return *reinterpret_cast<const float4*>(p); }
M4_DEV void st4(float* p, float4 v) { *reinterpret_cast<float4*>(p) = v; }

// Asynchronous global -> shared copies (cp.async): 16 bytes (.cg) or 4 bytes
// (.ca); an invalid source copies zeros (src-size 0; the address stays a
// valid one). Groups are committed and awaited per pipeline stage.
M4_DEV void cp16(float* dst, const float* src, bool valid) {
  const unsigned d = static_cast<unsigned>(__cvta_generic_to_shared(dst));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(d), "l"(src), "r"(valid ? 16 : 0) : "memory");
}
M4_DEV void cp4(float* dst, const float* src, bool valid) {
  const unsigned d = static_cast<unsigned>(__cvta_generic_to_shared(dst));
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;\n" ::"r"(d), "l"(src), "r"(valid ? 4 : 0) : "memory");
}
M4_DEV void cp_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
M4_DEV void cp_wait_group() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory"); }
// Wait for all of this thread's copies; a __syncthreads must follow before
// other threads read them.
M4_DEV void cp_wait() { asm volatile("cp.async.wait_all;\n" ::: "memory"); }

// Paired fp32 arithmetic (fma.rn.f32x2 / mul.rn.f32x2, sm_100a): two
// lanes of work per instruction, each rounded like fmaf / __fmul_rn.
M4_DEV unsigned long long pk2(float2 v) {
  unsigned long long r;
  asm("mov.b64 %0, {%1,%2};" : "=l"(r) : "f"(v.x), "f"(v.y));
  return r;
}
M4_DEV float2 upk2(unsigned long long r) {
  float2 v;
  asm("mov.b64 {%0,%1}, %2;" : "=f"(v.x), "=f"(v.y) : "l"(r));
  return v;
}
M4_DEV float2 ffma2(float2 a, float2 b, float2 c) {
  unsigned long long d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(pk2(a)), "l"(pk2(b)), "l"(pk2(c)));
  return upk2(d);
}
M4_DEV float2 fmul2(float2 a, float2 b) {
  unsigned long long d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(pk2(a)), "l"(pk2(b)));
  return upk2(d);
}

// Streaming (evict-first) 128-bit global store for write-once residuals.
M4_DEV void st4_stream(float* p, float4 v) { __stcs(reinterpret_cast<float4*>(p), v); }

// Load a scalar that may be float or bfloat16.
template <typename T> M4_DEV float to_f(T v);
template <> M4_DEV float to_f<float>(float v) { return v; }
template <> M4_DEV float to_f<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }

template <typename T> M4_DEV T from_f(float v);
template <> M4_DEV float from_f<float>(float v) { return v; }
template <> M4_DEV __nv_bfloat16 from_f<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }

// Round to the model dtype and back (identity for float).
template <typename T> M4_DEV float round_to(float v) { return to_f<T>(from_f<T>(v)); }

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Every given pointer is 16-byte aligned (NULL counts as aligned).
template <class... Ps>
inline bool all_aligned16(const Ps*... ps) { return (aligned16(ps) && ...); }

inline size_t align256(size_t n) { return (n + 255) & ~size_t(255); }

inline int launch_status() {
  return cudaGetLastError() == cudaSuccess ? M4_OK : M4_ERR_LAUNCH;
}

}  // namespace m4
