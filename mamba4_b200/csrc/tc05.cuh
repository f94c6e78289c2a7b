// tcgen05 helpers (sm_100a): tensor-memory allocation, shared-memory matrix
// descriptors (no swizzle, 8 x 16-byte core matrices), bf16 MMA with fp32
// accumulation in tensor memory, commit to an mbarrier, tensor-memory loads.
//
// Tile layout used with these descriptors: a [64][64] bf16 tile (c
// contiguous in global memory) is stored as 64 rows of 128 bytes with the
// 128-byte swizzle (16-byte chunk index XOR row % 8, tc::sw), the layout TMA
// writes with CU_TENSOR_MAP_SWIZZLE_128B; tiles start on 1024-byte
// boundaries. As a K-major operand (K = c) the descriptor has SBO 1024 and a
// K step of 16 advances 32 bytes inside the swizzled rows; as an MN-major
// operand (MN = c, K = r) it has SBO 1024 and a K step advances 2048 bytes.
// An M = 64 accumulator puts row m in tensor-memory lane (m % 16) +
// 32 (m / 16): warp w reads rows 16 (w % 4) .. +15 on its lanes 0..15.
#pragma once
#include <cstdint>
namespace m4 {
namespace tc {
__device__ __forceinline__ uint32_t su32(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }
__device__ __forceinline__ void mbar_init(uint64_t* bar, int count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(su32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ bool mbar_try(uint64_t* bar, uint32_t phase) {
  uint32_t ok;
  asm volatile("{\n\t.reg .pred P1;\n\tmbarrier.try_wait.parity.shared::cta.b64 P1, [%1], %2;\n\tselp.b32 %0, 1, 0, P1;\n\t}"
               : "=r"(ok) : "r"(su32(bar)), "r"(phase) : "memory");
  return ok != 0;
}
// Bounded wait: false after `limit` polls.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t phase, int limit) {
  for (int i = 0; i < limit; ++i)
    if (mbar_try(bar, phase)) return true;
  return false;
}
__device__ __forceinline__ void tmem_alloc(uint32_t* dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(su32(dst)), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
// Shared-memory matrix descriptor, no swizzle: lbo = byte stride between
// 8-element groups along K, sbo = byte stride between 8-row groups along M/N.
__device__ __forceinline__ uint64_t sdesc(const void* smem, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= uint64_t((su32(smem) >> 4) & 0x3FFFu);
  d |= uint64_t((lbo >> 4) & 0x3FFFu) << 16;
  d |= uint64_t((sbo >> 4) & 0x3FFFu) << 32;
  d |= uint64_t(1) << 46;  // descriptor version of sm_100
  return d;               // base offset 0, layout type 0 (no swizzle)
}
// Instruction descriptor: bf16 x bf16 -> f32, M x N, A/B major (0 K, 1 MN).
__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N, int a_mn, int b_mn) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (uint32_t(a_mn) << 15) | (uint32_t(b_mn) << 16) |
         (uint32_t(N >> 3) << 17) | (uint32_t(M >> 4) << 24);
}
__device__ __forceinline__ void mma_bf16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t acc) {
  const uint32_t z = 0;
  asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
               "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}"
               ::"r"(d_tmem), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc), "r"(z), "r"(z), "r"(z), "r"(z)
               : "memory");
}
__device__ __forceinline__ void commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(su32(bar)) : "memory");
}
__device__ __forceinline__ void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
                 "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
               : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
// Byte offset of element (r, c) of a [R][64] bf16 tile in 8x8 core matrices:
// cores along c adjacent (128 B), 8-row groups 1024 B apart.
__host__ __device__ constexpr uint32_t blk(int r, int c) {
  return uint32_t(((r >> 3) * 8 + (c >> 3)) * 128 + (r & 7) * 16 + (c & 7) * 2);
}
// Swizzled (128B) variant of sdesc.
__device__ __forceinline__ uint64_t sdesc_sw128(const void* smem, uint32_t lbo, uint32_t sbo) {
  return sdesc(smem, lbo, sbo) | (uint64_t(2) << 61);
}
// Byte offset of element (r, c) of a 128-byte-swizzled [64][64] bf16 tile.
__host__ __device__ constexpr uint32_t sw(int r, int c) {
  return uint32_t(r * 128 + (((c >> 3) ^ (r & 7)) << 4) + (c & 7) * 2);
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(su32(bar)), "r"(bytes) : "memory");
}
// TMA tile load (no multicast) of a 3-D tensor map box into shared memory,
// completing `bar`'s transaction count.
__device__ __forceinline__ void tma_load_3d(void* dst, const void* tmap, int c0, int c1, int c2, uint64_t* bar) {
  asm volatile("cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];"
               ::"r"(su32(dst)), "l"(tmap), "r"(c0), "r"(c1), "r"(c2), "r"(su32(bar)) : "memory");
}

// Device-side error flag: a bounded wait on the tensor cores gave up.
__device__ int g_timeout;
__device__ __forceinline__ void flag_timeout() { atomicExch(&g_timeout, 1); }
constexpr int WAIT_LIMIT = 1 << 24;
}  // namespace tc
}  // namespace m4
