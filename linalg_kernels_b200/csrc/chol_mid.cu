// chol_mid.cu — batched Cholesky for 64 < n <= 128: one CTA per matrix, the matrix in
// shared memory, right-looking over 32-wide panels. The reference factors its n = 128
// benchmark shape (b = 256) with a dedicated kernel too, one CTA per matrix
// (cutlass_blocked_128_kernel, cholesky/cholesky.py:419-826, launched at :803-817); the
// blocked schedule's diagonal-block kernel, built for a few large matrices, needs ~70 us
// for that shape.
//
// Per matrix (256 threads, 8 warps):
//   load      the lower triangle of A into shared memory by cp.async (all copies in
//             flight at once, one wait), row-major with an odd row stride (n | 1 floats),
//             so that a column read by 32 consecutive rows hits 32 distinct banks; warp w
//             copies rows w, w + 8, ... (coalesced).
//   per panel k0 = 0, 32, ...:
//     factor  warp 0, lane i holding row k0 + i of the 32 x 32 diagonal block in
//             registers: per column j the pivot comes from lane j by shuffle, r = rsqrt(d),
//             L[j][j] = d r and L[i][j] = a[i][j] r below it (the pivot arithmetic of the
//             small kernel), and the rank-1 update of the rest of the block takes each
//             L[c][j] from lane c by shuffle. r is kept per column for the solve.
//     solve   one thread per row below the block: x = a L_D^{-T} by forward substitution
//             (x_j = (a_j - sum_{i<j} x_i L_D[j][i]) r_j) in chunks of 8 columns, the L_D
//             entries read as shared-memory broadcasts.
//     update  the lower triangle of the trailing rows and columns minus X X^T, K = 32,
//             thread (tx, ty) of a 16 x 16 grid owning the rows ty + 16 i and columns
//             tx + 16 c (conflict-free shared-memory reads).
//   store     L row by row with zeros above the diagonal (coalesced); info = the first
//             diagonal entry that is not > 0 (a non-positive pivot makes every later pivot
//             NaN, so the first one is LAPACK's info).
// Shared memory: n (n | 1) floats (66 KB at n = 128); 2 CTAs per SM (the register budget
// of 128 per thread lets the factor keep its shuffles in flight). No workspace, no
// waits on other CTAs. A == L (in place) is allowed: a CTA reads its whole matrix before
// it writes any of it.
#include "chol_common.cuh"

namespace chol {
namespace {

constexpr int kMidMax = 128;
constexpr int kMidThreads = 256;
constexpr int kMidCtasPerSm = 2;

__device__ __forceinline__ float mid_rsqrt(float x) {
  float y;
  asm("rsqrt.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Warp 0: factor the w x w diagonal block at (k0, k0) in place; rdg[k0 + j] = r_j.
__device__ __forceinline__ void mid_factor_diag(float* As, int ld, int k0, int w, int lane,
                                                float* rdg) {
  float a[32];
  const bool own = lane < w;
  float* row = As + (k0 + lane) * ld + k0;
#pragma unroll
  for (int j = 0; j < 32; ++j) a[j] = (own && j <= lane) ? row[j] : 0.f;
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    if (j < w) {
      const float d = __shfl_sync(0xffffffffu, a[j], j);
      const float r = mid_rsqrt(d);
      a[j] = lane == j ? d * r : (lane > j ? a[j] * r : a[j]);
      if (lane == 0) rdg[k0 + j] = r;
#pragma unroll
      for (int c = j + 1; c < 32; ++c) {
        const float lc = __shfl_sync(0xffffffffu, a[j], c);
        a[c] = c <= lane ? fmaf(-a[j], lc, a[c]) : a[c];
      }
    }
  }
  if (own) {
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (j <= lane) row[j] = a[j];
  }
}

// One thread: row R of the panel, x = a L_D^{-T}, in chunks of 8 columns: a chunk first
// takes the contributions of the columns already solved (read back from the row itself),
// then solves its own 8 x 8 triangle in registers.
__device__ __forceinline__ void mid_solve_row(float* As, int ld, int k0, int w, int R,
                                              const float* rdg) {
  float* row = As + R * ld + k0;
  for (int q = 0; q < w; q += 8) {
    float x[8];
#pragma unroll
    for (int c = 0; c < 8; ++c) x[c] = (q + c < w) ? row[q + c] : 0.f;
    const float* lq = As + (k0 + q) * ld + k0;  // L_D[q + c][i] at lq[c * ld + i]
#pragma unroll 4
    for (int i = 0; i < q; ++i) {
      const float xi = row[i];
#pragma unroll
      for (int c = 0; c < 8; ++c)
        if (q + c < w) x[c] = fmaf(-xi, lq[c * ld + i], x[c]);
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if (q + j < w) {
        x[j] *= rdg[k0 + q + j];
#pragma unroll
        for (int c = j + 1; c < 8; ++c)
          if (q + c < w) x[c] = fmaf(-x[j], lq[c * ld + q + j], x[c]);
      }
    }
#pragma unroll
    for (int c = 0; c < 8; ++c)
      if (q + c < w) row[q + c] = x[c];
  }
}

// All threads: the lower triangle of rows / columns [k1, n) minus X X^T, where X is
// columns [k0, k0 + w) of those rows. Thread (tx, ty) owns rows k1 + ty + 16 i and columns
// k1 + tx + 16 c with c <= i < 6 (for c > i every entry lies above the diagonal): per k a
// warp reads 2 rows (broadcasts) and 16 consecutive rows n | 1 floats apart (distinct
// banks), so the reads are conflict-free.
__device__ __forceinline__ void mid_update(float* As, int ld, int n, int k0, int w, int k1,
                                           int tid) {
  const int tx = tid & 15, ty = tid >> 4;
  const int tiles = (n - k1 + 15) >> 4;  // <= 6
  int ro[6], co[6];
#pragma unroll
  for (int i = 0; i < 6; ++i) {
    // rows past n read row n - 1 (in bounds); their results are not written
    ro[i] = min(k1 + ty + 16 * i, n - 1) * ld + k0;
    co[i] = min(k1 + tx + 16 * i, n - 1) * ld + k0;
  }
  float acc[6][6];
#pragma unroll
  for (int i = 0; i < 6; ++i)
#pragma unroll
    for (int c = 0; c <= i; ++c) acc[i][c] = 0.f;
#pragma unroll 4
  for (int j = 0; j < w; ++j) {
    float xr[6], xc[6];
#pragma unroll
    for (int i = 0; i < 6; ++i) {
      xr[i] = i < tiles ? As[ro[i] + j] : 0.f;
      xc[i] = i < tiles ? As[co[i] + j] : 0.f;
    }
#pragma unroll
    for (int i = 0; i < 6; ++i)
#pragma unroll
      for (int c = 0; c <= i; ++c) acc[i][c] = fmaf(xr[i], xc[c], acc[i][c]);
  }
#pragma unroll
  for (int i = 0; i < 6; ++i)
#pragma unroll
    for (int c = 0; c <= i; ++c) {
      const int r = k1 + ty + 16 * i, col = k1 + tx + 16 * c;
      if (i < tiles && r < n && col <= r) As[r * ld + col] -= acc[i][c];
    }
}

__global__ void __launch_bounds__(kMidThreads, kMidCtasPerSm)
    mid_potrf_kernel(const float* A, float* L, int64_t batch, int n, int* info) {
  griddep_wait();
  griddep_launch();
  extern __shared__ float As[];
  __shared__ float rdg[kMidMax];
  const int ld = n | 1;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int64_t m = blockIdx.x; m < batch; m += gridDim.x) {
    const float* Am = A + m * int64_t(n) * n;
    float* Lm = L + m * int64_t(n) * n;
    for (int r = warp; r < n; r += kMidThreads / 32)
      for (int c = lane; c <= r; c += 32) cp_async4(&As[r * ld + c], Am + int64_t(r) * n + c);
    cp_async_wait_all();
    __syncthreads();
    for (int k0 = 0; k0 < n; k0 += 32) {
      const int w = min(32, n - k0);
      if (warp == 0) mid_factor_diag(As, ld, k0, w, lane, rdg);
      __syncthreads();
      const int k1 = k0 + w;
      if (k1 < n) {
        if (tid < n - k1) mid_solve_row(As, ld, k0, w, k1 + tid, rdg);
        __syncthreads();
        mid_update(As, ld, n, k0, w, k1, tid);
        __syncthreads();
      }
    }
    for (int r = warp; r < n; r += kMidThreads / 32)
      for (int c = lane; c < n; c += 32) Lm[int64_t(r) * n + c] = c <= r ? As[r * ld + c] : 0.f;
    if (info != nullptr && warp == 0) {
      int first = 0;
      for (int c0 = 0; c0 < n; c0 += 32) {
        const int c = c0 + lane;
        const bool bad = c < n && !(As[c * ld + c] > 0.f);
        const unsigned mask = __ballot_sync(0xffffffffu, bad);
        if (mask != 0u && first == 0) first = c0 + __ffs(int(mask));
      }
      if (lane == 0) info[m] = first;
    }
    __syncthreads();  // the next matrix's loads overwrite As
  }
}

size_t mid_smem_bytes(int n) { return size_t(n) * size_t(n | 1) * sizeof(float); }

}  // namespace

int g_mid_kernel = 1;

bool use_mid(int64_t n) { return g_mid_kernel != 0 && n > 64 && n <= kMidMax; }

cudaError_t prepare_mid() {
  return cudaFuncSetAttribute(mid_potrf_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              int(mid_smem_bytes(kMidMax)));
}

int launch_mid(const float* A, float* L, int64_t batch, int n, int* info, cudaStream_t q) {
  if (n <= 64 || n > kMidMax) return CHOL_ERR_UNSUPPORTED;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t grid = std::min<int64_t>(batch, int64_t(sms) * kMidCtasPerSm * 16);
  return status_from(launch_pdl(mid_potrf_kernel, dim3(unsigned(grid)), dim3(kMidThreads),
                                mid_smem_bytes(n), q, true, A, L, batch, n, info));
}

}  // namespace chol
