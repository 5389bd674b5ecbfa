// chol_warp.cuh — warp-level right-looking Cholesky of an NP x NP block held in registers.
//
// Layout: a group of LPM = min(NP, 32) lanes owns one matrix; lane gl of the group holds
// rows i = s*LPM + gl (s = 0..R-1, R = NP/LPM). Row i of slot s is kept as column pairs
// a[s][p] = (A[i][2p], A[i][2p+1]) for p < (s+1)*LPM/2 in 64-bit registers: slot s never
// needs columns past its last row, so the per-slot register bound is static, and the packed
// f32x2 FMA reads and writes the pairs with no packing moves.
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

// LPM lanes share one matrix (default min(NP, 32)); fewer lanes per matrix means more
// matrices per warp sharing every per-column instruction (shuffle, rsqrt, broadcast).
template <int NP, int LPM_ = (NP < 32 ? NP : 32)>
struct WarpShape {
  static constexpr int LPM = LPM_;               // lanes per matrix
  static constexpr int R = NP / LPM;             // rows per lane
  static constexpr int MPW = 32 / LPM;           // matrices per warp
  static constexpr int COLS = 2 * NP + 8;        // per-group column buffer stride (floats)
  static_assert(NP >= 4 && NP <= 64 && (NP & (NP - 1)) == 0, "NP must be 4..64, power of 2");
  static_assert(LPM >= 4 && LPM <= 32 && NP % LPM == 0, "LPM");
};

__device__ __forceinline__ float rsqrt_approx(float x) {
  float y;
  asm("rsqrt.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Row storage: a[s][p] holds columns 2p (low half) and 2p+1 (high half) of one row as a
// 64-bit register pair; the packed FMA consumes and produces these pairs directly.
template <int NP>
__device__ __forceinline__ float pair_get(const uint64_t (&row)[NP / 2], int k) {
  return (k & 1) ? hi_of(row[k >> 1]) : lo_of(row[k >> 1]);
}
template <int NP>
__device__ __forceinline__ void pair_set(uint64_t (&row)[NP / 2], int k, float v) {
  const uint64_t cur = row[k >> 1];
  row[k >> 1] = (k & 1) ? pack2(lo_of(cur), v) : pack2(v, hi_of(cur));
}

// col: this group's 2*NP floats of shared memory (16-byte aligned).
template <int NP, int LPM_ = (NP < 32 ? NP : 32)>
__device__ __forceinline__ void warp_potrf_rows(uint64_t (&a)[NP / LPM_][NP / 2], float* col,
                                                int gl) {
  constexpr int LPM = LPM_;
  constexpr int R = NP / LPM;
  float dnext = lo_of(a[0][0]);
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
      uint64_t cv[NP / 2];
#pragma unroll
      for (int q = q0; q < NP / 4; ++q) {
        const ulonglong2 v = *reinterpret_cast<const ulonglong2*>(cb + 4 * q);
        cv[2 * q] = v.x;
        cv[2 * q + 1] = v.y;
      }
#pragma unroll
      for (int s = 0; s < R; ++s) {
        if ((s + 1) * LPM - 1 <= j) continue;
        const float nl = -lv[s];
        int p0 = (j + 1) >> 1;
        if ((j + 1) & 1) {  // odd first column: scalar fma on the high half, then whole pairs
          const uint64_t cur = a[s][p0];
          a[s][p0] = pack2(lo_of(cur), fmaf(nl, hi_of(cv[p0]), hi_of(cur)));
          ++p0;
        }
        const uint64_t nl2 = pack2(nl, nl);
#pragma unroll
        for (int p = p0; p < (s + 1) * LPM / 2; ++p) a[s][p] = ffma2_u64(nl2, cv[p], a[s][p]);
      }
    }
  }
}

// ---------------------------------------------------------------------------------------
// 64 x 64 diagonal-block helpers shared by the block kernels. `tile` is row-major in shared
// memory with row stride LD (a multiple of 4 floats); the lower triangle holds the block.

// One warp factors the block in place: lower triangle of L, exact zeros above the
// diagonal. rdiag receives 1 / L[i][i]. Returns in every lane the 1-based index of the
// first column whose pivot is not > 0 (NaN included), or 0.
template <int LD>
__device__ __forceinline__ int tile64_potrf(float* tile, float* col, float* rdiag, int lane) {
  uint64_t a[2][32];
#pragma unroll
  for (int s = 0; s < 2; ++s) {
    const float* rp = tile + (s * 32 + lane) * LD;
#pragma unroll
    for (int q = 0; q < (s + 1) * 8; ++q) {
      const ulonglong2 v = *reinterpret_cast<const ulonglong2*>(rp + 4 * q);
      a[s][2 * q] = v.x;
      a[s][2 * q + 1] = v.y;
    }
  }
  warp_potrf_rows<64>(a, col, lane);
  __syncwarp();
#pragma unroll
  for (int s = 0; s < 2; ++s) {
    const int i = s * 32 + lane;
    float* rp = tile + i * LD;
#pragma unroll
    for (int q = 0; q < 16; ++q) {
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (4 * q < (s + 1) * 32) {
        v.x = (4 * q + 0 <= i) ? lo_of(a[s][2 * q]) : 0.f;
        v.y = (4 * q + 1 <= i) ? hi_of(a[s][2 * q]) : 0.f;
        v.z = (4 * q + 2 <= i) ? lo_of(a[s][2 * q + 1]) : 0.f;
        v.w = (4 * q + 3 <= i) ? hi_of(a[s][2 * q + 1]) : 0.f;
      }
      *reinterpret_cast<float4*>(rp + 4 * q) = v;
    }
  }
  __syncwarp();
  const float d0 = tile[lane * LD + lane];
  const float d1 = tile[(lane + 32) * LD + lane + 32];
  rdiag[lane] = __frcp_rn(d0);
  rdiag[lane + 32] = __frcp_rn(d1);
  const unsigned b0 = __ballot_sync(0xffffffffu, !(d0 > 0.f));
  const unsigned b1 = __ballot_sync(0xffffffffu, !(d1 > 0.f));
  __syncwarp();
  return b0 ? __ffs(b0) : (b1 ? 32 + __ffs(b1) : 0);
}

// Column c of T = inv(L) for the factored block (one thread per column), by forward
// substitution on e_c:  t[i] = -rdiag[i] * sum_{m<i} L[i][m] t[m] (i > c), t[c] = rdiag[c],
// t[i] = 0 (i < c).
template <int LD>
__device__ __forceinline__ void tile64_inverse_column(const float* tile, const float* rdiag,
                                                      int c, float (&t)[64]) {
#pragma unroll
  for (int i = 0; i < 64; ++i) {
    const float* rp = tile + i * LD;
    float2 acc = make_float2(0.f, 0.f);
#pragma unroll
    for (int q = 0; q < i / 4; ++q) {
      const float4 v = *reinterpret_cast<const float4*>(rp + 4 * q);
      acc = ffma2(make_float2(v.x, v.y), make_float2(t[4 * q], t[4 * q + 1]), acc);
      acc = ffma2(make_float2(v.z, v.w), make_float2(t[4 * q + 2], t[4 * q + 3]), acc);
    }
    float sum = acc.x + acc.y;
#pragma unroll
    for (int mm = (i / 4) * 4; mm < i; ++mm) sum = fmaf(rp[mm], t[mm], sum);
    const float ri = rdiag[i];
    t[i] = (i == c) ? ri : ((i < c) ? 0.f : -ri * sum);
  }
}

}  // namespace chol
