// chol_warp.cuh — warp-level right-looking Cholesky of an NP x NP block held in registers.
//
// Layout: a group of LPM = min(NP, 32) lanes owns one matrix; lane gl of the group holds
// rows i = s*LPM + gl (s = 0..R-1, R = NP/LPM). Row i of slot s is kept as column pairs
// a[s][p] = (A[i][2p], A[i][2p+1]) for p < (s+1)*LPM/2: slot s never needs columns past
// its last row, so the per-slot register bound is static and the triangular shape costs
// no predicated work beyond one slot width. Pairs sit in aligned 64-bit registers, which
// is what the packed f32x2 FMA reads and writes.
//
// Algorithm (LAPACK xPOTF2, right-looking form; the reference's small kernels use the
// same recurrence, cholesky/b4096n32/DESIGN.md:13-21, cholesky/cholesky.py:294-387):
//   for j: d = a[j][j]; L[j][j] = sqrt(d); L[i][j] = a[i][j] / L[j][j]  (i > j)
//          a[i][k] -= L[i][j] * L[k][j]                                   (j < k <= i)
// computed as r = rsqrt(d), L[i][j] = a[i][j]*r (for i == j this is d*r = sqrt(d)).
//
// Per column: the pivot comes from the lane that owns row j through one shuffle; that lane
// prepared it in the previous column from its own registers (look-ahead), so the serial
// chain is shuffle -> rsqrt -> multiply -> fma. Column j is broadcast through a
// ping-pong shared buffer (one store per lane, 128-bit broadcast loads) and the rank-1
// update runs as packed f32x2 FMAs. Entries above the diagonal are left as garbage and
// must be masked by the caller when the rows are written out; they never feed the lower
// triangle. A non-positive pivot gives NaN/Inf from rsqrt, which the caller detects on
// the diagonal of the result.
#pragma once

#include "chol_common.cuh"

namespace chol {

template <int NP>
struct WarpShape {
  static constexpr int LPM = NP < 32 ? NP : 32;  // lanes per matrix
  static constexpr int R = NP / LPM;             // rows per lane
  static constexpr int MPW = 32 / LPM;           // matrices per warp
  static_assert(NP >= 4 && NP <= 64 && (NP & (NP - 1)) == 0, "NP must be 4..64, power of 2");
};

__device__ __forceinline__ float rsqrt_approx(float x) {
  float y;
  asm("rsqrt.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

template <int NP>
__device__ __forceinline__ float pair_get(const float2 (&row)[NP / 2], int k) {
  return (k & 1) ? row[k >> 1].y : row[k >> 1].x;
}
template <int NP>
__device__ __forceinline__ void pair_set(float2 (&row)[NP / 2], int k, float v) {
  if (k & 1)
    row[k >> 1].y = v;
  else
    row[k >> 1].x = v;
}

// col: this group's 2*NP floats of shared memory (16-byte aligned).
template <int NP>
__device__ __forceinline__ void warp_potrf_rows(float2 (&a)[WarpShape<NP>::R][NP / 2], float* col,
                                                int gl) {
  constexpr int LPM = WarpShape<NP>::LPM;
  constexpr int R = WarpShape<NP>::R;
  float dnext = a[0][0].x;
#pragma unroll
  for (int j = 0; j < NP; ++j) {
    const float d = __shfl_sync(0xffffffffu, dnext, j % LPM, LPM);
    const float r = rsqrt_approx(d);
    float* cb = col + (j & 1) * NP;
    float lv[R];
#pragma unroll
    for (int s = 0; s < R; ++s) {
      lv[s] = 0.f;
      if ((s + 1) * LPM - 1 < j) continue;  // every row of this slot is above row j
      // lane j holds a[j][j] == d (bitwise: same fma as the look-ahead), so this is d*r
      const float l = pair_get<NP>(a[s], j) * r;
      pair_set<NP>(a[s], j, l);
      lv[s] = l;
      cb[s * LPM + gl] = l;
    }
    if (j + 1 < NP) {
      const int sn = (j + 1) / LPM;
      // Same operands as the update below applies to a[sn][j+1] in this lane, so the
      // look-ahead pivot is bitwise the value the update produces.
      dnext = fmaf(-lv[sn], lv[sn], pair_get<NP>(a[sn], j + 1));
    }
    __syncwarp();
    if (j + 1 < NP) {
      const int q0 = (j + 1) >> 2;
      float2 cv[NP / 2];
#pragma unroll
      for (int q = q0; q < NP / 4; ++q) {
        const float4 v = *reinterpret_cast<const float4*>(cb + 4 * q);
        cv[2 * q] = make_float2(v.x, v.y);
        cv[2 * q + 1] = make_float2(v.z, v.w);
      }
#pragma unroll
      for (int s = 0; s < R; ++s) {
        if ((s + 1) * LPM - 1 <= j) continue;
        const float nl = -lv[s];
        int p0 = (j + 1) >> 1;
        if ((j + 1) & 1) {  // odd first column: scalar fma, then whole pairs
          a[s][p0].y = fmaf(nl, cv[p0].y, a[s][p0].y);
          ++p0;
        }
        const float2 nl2 = make_float2(nl, nl);
#pragma unroll
        for (int p = p0; p < (s + 1) * LPM / 2; ++p) a[s][p] = ffma2(nl2, cv[p], a[s][p]);
      }
    }
  }
}

}  // namespace chol
