// chol_warp.cuh — warp-level right-looking Cholesky of an NP x NP block held in registers.
//
// Layout: a group of LPM = min(NP, 32) lanes owns one matrix; lane gl of the group holds
// rows i = s*LPM + gl (s = 0..R-1, R = NP/LPM) in a[s][0 .. (s+1)*LPM-1]. Slot s only ever
// needs columns k <= i < (s+1)*LPM, so the per-slot register bound is static and the
// triangular shape costs no predicated work beyond one slot width.
//
// Algorithm (LAPACK xPOTF2, right-looking form; the reference's small kernels use the
// same recurrence, cholesky/b4096n32/DESIGN.md:13-21, cholesky/cholesky.py:294-387):
//   for j: d = a[j][j]; L[j][j] = sqrt(d); L[i][j] = a[i][j] / L[j][j]  (i > j)
//          a[i][k] -= L[i][j] * L[k][j]                                   (j < k <= i)
// computed as r = rsqrt(d), L[j][j] = d*r, L[i][j] = a[i][j]*r.
//
// Per column: the pivot comes from the lane that owns row j through one shuffle; that lane
// prepared it in the previous column from its own registers (look-ahead), so the serial
// chain is shuffle -> rsqrt -> multiply -> fma. Column j is broadcast through a
// ping-pong shared buffer (one store per lane, 128-bit broadcast loads) and the rank-1
// update runs as packed f32x2 FMAs.
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

// col: this group's 2*NP floats of shared memory (16-byte aligned).
// fail: set to the 1-based column of the first non-positive (or NaN) pivot, if 0 before.
template <int NP>
__device__ __forceinline__ void warp_potrf_rows(float (&a)[WarpShape<NP>::R][NP], float* col,
                                                int gl, int& fail) {
  constexpr int LPM = WarpShape<NP>::LPM;
  constexpr int R = WarpShape<NP>::R;
  float dnext = a[0][0];
#pragma unroll
  for (int j = 0; j < NP; ++j) {
    const float d = __shfl_sync(0xffffffffu, dnext, j % LPM, LPM);
    const float r = rsqrtf(d);
    if (!(d > 0.f) && fail == 0) fail = j + 1;
    float* cb = col + (j & 1) * NP;
    float lv[R];
#pragma unroll
    for (int s = 0; s < R; ++s) {
      lv[s] = 0.f;
      if ((s + 1) * LPM - 1 < j) continue;  // every row of this slot is above row j
      const int i = s * LPM + gl;
      const float l = (i == j) ? d * r : a[s][j] * r;
      a[s][j] = l;
      lv[s] = l;
      cb[i] = (i > j) ? l : 0.f;
    }
    if (j + 1 < NP) {
      const int sn = (j + 1) / LPM;
      // Same operands as the packed update below applies to a[sn][j+1] in this lane, so
      // the look-ahead pivot is bitwise the value the update produces.
      dnext = fmaf(-lv[sn], lv[sn], a[sn][j + 1]);
    }
    __syncwarp();
    if (j + 1 < NP) {
      const int q0 = (j + 1) >> 2;
      float cv[NP];
#pragma unroll
      for (int q = q0; q < NP / 4; ++q) {
        const float4 v = *reinterpret_cast<const float4*>(cb + 4 * q);
        cv[4 * q + 0] = v.x;
        cv[4 * q + 1] = v.y;
        cv[4 * q + 2] = v.z;
        cv[4 * q + 3] = v.w;
      }
#pragma unroll
      for (int s = 0; s < R; ++s) {
        if ((s + 1) * LPM - 1 <= j) continue;
        const float2 nl = make_float2(-lv[s], -lv[s]);
#pragma unroll
        for (int k = (j + 1) & ~1; k < (s + 1) * LPM; k += 2) {
          // cb[j] was written as 0, so a pair that starts at column j leaves L[i][j] as is.
          const float2 res =
              ffma2(nl, make_float2(cv[k], cv[k + 1]), make_float2(a[s][k], a[s][k + 1]));
          a[s][k] = res.x;
          a[s][k + 1] = res.y;
        }
      }
    }
  }
}

}  // namespace chol
