// chol_tc_ptx.cuh — inline-PTX wrappers for tcgen05 / TMEM / TMA / mbarrier shared by the
// tensor-core kernels (chol_tc.cu, chol_panel.cu), and the 3xTF32 operand split.
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>

#include "chol_common.cuh"

namespace chol {

namespace tcx {

constexpr int kBK = 32;  // fp32 elements of K per stage = one 128-byte swizzle row

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s

// Bounded wait for the completion of phase `parity`. Returns false (and records the
// timeout in the status word) if it does not complete within kWaitLimitNs.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* status) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  for (uint32_t it = 0;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 255u) == 255u && global_ns() - t0 > kWaitLimitNs) {
      atomicExch(status, CHOL_ERR_WAIT_TIMEOUT);
      return false;
    }
  }
}

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int x, int y,
                                            int z, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void prefetch_map(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// K-major operand, 128-byte swizzle: rows of 128 B, 8-row groups 1024 B apart.
__device__ __forceinline__ uint64_t sw128_desc(const void* smem_tile) {
  const uint32_t addr = smem_u32(smem_tile);
  uint64_t d = 0;
  d |= uint64_t((addr >> 4) & 0x3FFF);  // start address
  d |= uint64_t(1) << 16;               // leading byte offset (unused for SW128 K-major)
  d |= uint64_t(1024 >> 4) << 32;       // stride byte offset: 8 rows x 128 B
  d |= uint64_t(1) << 46;               // descriptor version (sm_100)
  d |= uint64_t(2) << 61;               // SWIZZLE_128B
  return d;
}

// Instruction descriptor: D f32, A/B tf32, K-major both, M x N.
template <int M, int BN>
__device__ __forceinline__ uint32_t tf32_idesc() {
  return (1u << 4)                       // D format f32
         | (2u << 7)                     // A format tf32
         | (2u << 10)                    // B format tf32
         | (uint32_t(BN >> 3) << 17)     // N >> 3
         | (uint32_t(M >> 4) << 24);     // M >> 4
}

__device__ __forceinline__ void mma_tf32(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// hi/lo split of one 16-byte chunk: lo to the twin buffer; hi written back in place when
// WRITE_HI (otherwise the tensor core's own TF32 conversion of x must equal hi).
template <bool WRITE_HI>
__device__ __forceinline__ void split4(float4* hi_p, float4* lo_p) {
  const float4 x = *hi_p;
  float4 h, l;
  h.x = __uint_as_float(__float_as_uint(x.x) & 0xFFFFE000u);
  h.y = __uint_as_float(__float_as_uint(x.y) & 0xFFFFE000u);
  h.z = __uint_as_float(__float_as_uint(x.z) & 0xFFFFE000u);
  h.w = __uint_as_float(__float_as_uint(x.w) & 0xFFFFE000u);
  l.x = x.x - h.x;
  l.y = x.y - h.y;
  l.z = x.z - h.z;
  l.w = x.w - h.w;
  if (WRITE_HI) *hi_p = h;
  *lo_p = l;
}

// Origin of the view inside the tensor maps (element coordinates: x = column, y = row).
struct TmaOrigin {
  int px, py, qx, qy;
  int lpx, lqx;  // K origin of P and Q inside precomputed-lo buffers (rows as for P and Q)
};

// Split of chunk i of a 128B-swizzled K-major tile (8 chunks of 4 floats per row; the
// chunk at physical slot p of row r holds logical columns 4 * (p ^ (r & 7)) .. +3) with
// columns >= kval set to zero in both the raw buffer and lo.
__device__ __forceinline__ void split4_masked(float4* hi_p, float4* lo_p, int i, int kval) {
  const int row = i >> 3, phys = i & 7;
  const int col0 = 4 * (phys ^ (row & 7));
  float4 x = *hi_p;
  if (col0 + 0 >= kval) x.x = 0.f;
  if (col0 + 1 >= kval) x.y = 0.f;
  if (col0 + 2 >= kval) x.z = 0.f;
  if (col0 + 3 >= kval) x.w = 0.f;
  *hi_p = x;
  split4<false>(hi_p, lo_p);
}


}  // namespace tcx
}  // namespace chol
