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
//     panel   the warps that hold rows k0..n-1 (one row per thread, its w <= 32 panel
//             entries in registers) factor the whole n - k0 by w panel in one right-looking
//             pass: per column j every thread scales its entry by r = rsqrt(d), where the
//             pivot d comes from shared memory (the owner of row k0 + j prepared it in the
//             previous column: look-ahead), the diagonal block's rows publish their entry
//             of column j into a ping-pong buffer, one named barrier of the panel's warps,
//             and each row takes the rank-1 update of its remaining entries from broadcast
//             reads. The diagonal block's factor and the solve of the rows below it are
//             the same pass, so no warp waits for one warp's factor (the first version
//             factored the block in warp 0 and then solved one row per thread:
//             58.3 us at b256n128).
//     update  the lower triangle of the trailing rows and columns minus X X^T, K = 32,
//             thread (tx, ty) of a 16 x 16 grid owning the rows ty + 16 i and columns
//             tx + 16 c (conflict-free shared-memory reads).
//   store     L row by row with zeros above the diagonal (coalesced); info = the first
//             diagonal entry that is not > 0 (a non-positive pivot makes every later pivot
//             NaN, so the first one is LAPACK's info).
// Shared memory: n (n | 1) floats (66 KB at n = 128) plus the panel's column buffer and
// pivots; 2 CTAs per SM (128 registers per thread hold a thread's 32 panel entries and the
// update's 21 accumulators without spilling). No workspace, no
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

// Rank-1 update of column j (compile-time) on entries j+1..31 of one row held as packed
// pairs: a[k] -= l * cj[k], cj the published column (16-byte aligned shared memory).
__device__ __forceinline__ void row_update(uint64_t (&a)[16], int j, float l, const float* cj) {
  const float nl = -l;
  int p0 = (j + 1) >> 1;
  if ((j + 1) & 1) {  // odd first entry: the high half alone, then whole pairs
    const uint64_t v = a[p0];
    a[p0] = pack2(lo_of(v), fmaf(nl, cj[j + 1], hi_of(v)));
    ++p0;
  }
  const uint64_t nl2 = pack2(nl, nl);
#pragma unroll
  for (int q = p0 >> 1; q < 8; ++q) {
    const ulonglong2 v = *reinterpret_cast<const ulonglong2*>(cj + 4 * q);
    if (2 * q >= p0) a[2 * q] = ffma2_u64(nl2, v.x, a[2 * q]);
    a[2 * q + 1] = ffma2_u64(nl2, v.y, a[2 * q + 1]);
  }
}

// One warp of a panel (rows k0..n-1 of the w <= 32 panel columns, lane = row, entries as
// packed pairs in registers), right-looking, with no synchronisation beyond the warp: every
// warp holds the panel's diagonal block too (d: lane = diagonal row; the first warp's own
// rows are that block, kDiag) and factors its copy in step with the others, so it has the
// column it needs without waiting for another warp. Per column j: the pivot comes from lane
// j by shuffle (prepared in the previous column from that lane's registers: look-ahead);
// r = rsqrt(pivot); the diagonal row gets pivot * r = sqrt(pivot) and the rows below
// a * r; the copy's column goes to this warp's ping-pong buffer (cw: 2 x 32 floats); after
// __syncwarp every row takes the rank-1 update of its remaining entries from broadcast
// reads. The diagonal block's factor and the solve of the rows below are one pass, and every
// warp computes the same copy with the same operations, so the result does not depend on
// the number of warps. Entries above the diagonal of the block are garbage, never read.
template <bool kDiag>
__device__ __forceinline__ void panel_rows_factor(uint64_t (&d)[16], uint64_t (&a)[16], int w,
                                                  int lane, float* cw) {
  float dnext = lo_of(d[0]);  // lane j's value is pivot j
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    if (j < w) {
      const float piv = __shfl_sync(0xffffffffu, dnext, j);
      const float r = mid_rsqrt(piv);
      const uint64_t cd = d[j >> 1];
      const float ld = ((j & 1) ? hi_of(cd) : lo_of(cd)) * r;
      d[j >> 1] = (j & 1) ? pack2(lo_of(cd), ld) : pack2(ld, hi_of(cd));
      float la = 0.f;
      if (!kDiag) {
        const uint64_t ca = a[j >> 1];
        la = ((j & 1) ? hi_of(ca) : lo_of(ca)) * r;
        a[j >> 1] = (j & 1) ? pack2(lo_of(ca), la) : pack2(la, hi_of(ca));
      }
      float* cj = cw + (j & 1) * 32;
      if (lane > j && lane < w) cj[lane] = ld;
      if (j + 1 < w) {
        // the same operands as the update below applies to d[j+1] in lane j+1
        const uint64_t nx = d[(j + 1) >> 1];
        dnext = fmaf(-ld, ld, ((j + 1) & 1) ? hi_of(nx) : lo_of(nx));
      }
      __syncwarp();
      if (j + 1 < 32) {
        row_update(d, j, ld, cj);  // rows <= j change only entries above their diagonal
        if (!kDiag) row_update(a, j, la, cj);
      }
    }
  }
}

// The panel in shared memory: rows 0..rows-1 at P + t * ld (P = its element (k0, k0)).
// cb: 8 x 64 floats, 16-byte aligned (each warp's column buffer).
__device__ __forceinline__ void smem_panel(float* P, int ld, int rows, int w, int tid, float* cb) {
  const int nthr = (rows + 31) & ~31;
  if (tid >= nthr) return;
  const int lane = tid & 31, wp = tid >> 5;
  const bool own = tid < rows;
  float* dp = P + lane * ld;  // this lane's row of the diagonal block
  float* rp = P + (own ? tid : 0) * ld;
  uint64_t d[16], a[16];
#pragma unroll
  for (int p = 0; p < 16; ++p)
    d[p] = pack2((lane < w && 2 * p < w) ? dp[2 * p] : 0.f,
                 (lane < w && 2 * p + 1 < w) ? dp[2 * p + 1] : 0.f);
  float* cw = cb + wp * 64;
  if (wp > 0) {
    // a warp below the diagonal block: w == 32 (only the last panel is narrower, and it
    // has no rows below its diagonal block)
#pragma unroll
    for (int p = 0; p < 16; ++p)
      a[p] = pack2(own ? rp[2 * p] : 0.f, own ? rp[2 * p + 1] : 0.f);
  }
  // every warp has read the diagonal block before the first warp writes it back
  asm volatile("bar.sync 1, %0;" ::"r"(nthr) : "memory");
  if (wp == 0) {
    panel_rows_factor<true>(d, a, w, lane, cw);
    if (lane < w) {
#pragma unroll
      for (int p = 0; p < 16; ++p) {
        if (2 * p < w) dp[2 * p] = lo_of(d[p]);
        if (2 * p + 1 < w) dp[2 * p + 1] = hi_of(d[p]);
      }
    }
    return;
  }
  panel_rows_factor<false>(d, a, w, lane, cw);
  if (own) {
#pragma unroll
    for (int p = 0; p < 16; ++p) {
      rp[2 * p] = lo_of(a[p]);
      rp[2 * p + 1] = hi_of(a[p]);
    }
  }
}

// All threads: the lower triangle of rows / columns [k1, n) minus X X^T, where X is
// columns [k0, k0 + w) of those rows. Thread (tx, ty) owns rows k1 + ty + 16 i and columns
// k1 + tx + 16 c with c <= i < T, T = the trailing rows' 16-row tiles (<= 6, a compile-time
// count so that no work or select is spent on absent tiles; for c > i every entry lies
// above the diagonal): per k a warp reads 2 rows (broadcasts) and 16 consecutive rows
// n | 1 floats apart (distinct banks), so the reads are conflict-free. Rows are paired for
// the packed FMA.
template <int T>
__device__ __forceinline__ void mid_update_t(float* As, int ld, int n, int k0, int w, int k1,
                                             int tid) {
  constexpr int P = (T + 1) / 2;  // row pairs
  const int tx = tid & 15, ty = tid >> 4;
  int ro[2 * P], co[T];
#pragma unroll
  for (int i = 0; i < 2 * P; ++i)  // rows past n read row n - 1 (in bounds); not written
    ro[i] = min(k1 + ty + 16 * i, n - 1) * ld + k0;
#pragma unroll
  for (int c = 0; c < T; ++c) co[c] = min(k1 + tx + 16 * c, n - 1) * ld + k0;
  // acc[p][c] = (rows 2p, 2p+1) x column c, packed for fma.rn.f32x2; c <= 2p + 1
  uint64_t acc[P][T];
#pragma unroll
  for (int p = 0; p < P; ++p)
#pragma unroll
    for (int c = 0; c < T; ++c) acc[p][c] = 0ull;
#pragma unroll 4
  for (int j = 0; j < w; ++j) {
    uint64_t xr[P];
    float xc[T];
#pragma unroll
    for (int p = 0; p < P; ++p) xr[p] = pack2(As[ro[2 * p] + j], As[ro[2 * p + 1] + j]);
#pragma unroll
    for (int c = 0; c < T; ++c) xc[c] = As[co[c] + j];
#pragma unroll
    for (int p = 0; p < P; ++p)
#pragma unroll
      for (int c = 0; c < T; ++c)
        if (c <= 2 * p + 1) acc[p][c] = ffma2_u64(xr[p], pack2(xc[c], xc[c]), acc[p][c]);
  }
#pragma unroll
  for (int p = 0; p < P; ++p)
#pragma unroll
    for (int c = 0; c < T; ++c)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int i = 2 * p + h;
        const int r = k1 + ty + 16 * i, col = k1 + tx + 16 * c;
        if (c <= 2 * p + 1 && i < T && r < n && col <= r)
          As[r * ld + col] -= h ? hi_of(acc[p][c]) : lo_of(acc[p][c]);
      }
}

// All threads, one instantiation per count of 16-row tiles of the trailing matrix.
__device__ __forceinline__ void mid_update(float* As, int ld, int n, int k0, int w, int k1,
                                           int tid) {
  switch ((n - k1 + 15) >> 4) {
    case 1: mid_update_t<1>(As, ld, n, k0, w, k1, tid); break;
    case 2: mid_update_t<2>(As, ld, n, k0, w, k1, tid); break;
    case 3: mid_update_t<3>(As, ld, n, k0, w, k1, tid); break;
    case 4: mid_update_t<4>(As, ld, n, k0, w, k1, tid); break;
    case 5: mid_update_t<5>(As, ld, n, k0, w, k1, tid); break;
    default: mid_update_t<6>(As, ld, n, k0, w, k1, tid); break;
  }
}

// The warps' column buffers follow the matrix (offset in floats, 16-byte aligned).
__host__ __device__ __forceinline__ int mid_aux_offset(int n) { return (n * (n | 1) + 3) & ~3; }

__global__ void __launch_bounds__(kMidThreads, kMidCtasPerSm)
    mid_potrf_kernel(const float* A, float* L, int64_t batch, int n, int* info) {
  griddep_wait();
  griddep_launch();
  extern __shared__ float As[];
  const int ld = n | 1;
  float* cb = As + mid_aux_offset(n);  // the warps' column buffers, 16-byte aligned
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
      smem_panel(As + k0 * ld + k0, ld, n - k0, w, tid, cb);
      __syncthreads();
      const int k1 = k0 + w;
      if (k1 < n) {
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

// ---------------------------------------------------------------------------------------
// 128 < n <= 256: one CTA of 512 threads per matrix. The matrix (256 KB) does not fit in
// shared memory; it is worked on in place in L (a CTA's 256 KB stay in L2), and shared
// memory holds the current panel's rows (stride 33). Per 32-wide panel: all threads stage
// the panel's rows in shared memory (coalesced 128-byte row segments), the panel's warps
// (up to 8) factor them with panel_rows_factor, all threads write the panel back to L, and
// all 16 warps update the trailing lower triangle, C -= X X^T with X = the panel's rows
// below its diagonal block, in column chunks of 64 (thread (tx, ty) of a 16 x 32
// grid: columns tx + 16 c, c < 4, rows ty + 32 i, i < RI), reading C from the source (A for
// the first panel, L after it) and writing L. Every lower entry of L is written by the first
// panel and its update, so later panels read L only; A == L is allowed.
constexpr int kWideMax = 256;
constexpr int kWideThreads = 512;
constexpr int kXld = 33;
constexpr int kProws = kWideMax;

// Columns [k1 + c0, k1 + c0 + 64) of the trailing matrix, rows from k1 + c0 down: RI row
// groups of 32 (compile-time, so absent groups cost nothing).
template <int RI>
__device__ __forceinline__ void wide_update_t(const float* src, float* dst, int n, int k1,
                                              int c0, int w, int tid, const float* X) {
  const int tx = tid & 15, ty = tid >> 4;
  const int m = n - k1;
  int xr[RI], xc[4];
#pragma unroll
  for (int i = 0; i < RI; ++i) xr[i] = min(c0 + ty + 32 * i, m - 1) * kXld;
#pragma unroll
  for (int c = 0; c < 4; ++c) xc[c] = min(c0 + tx + 16 * c, m - 1) * kXld;
  // acc[i][q] = row group i x columns (2q, 2q + 1), packed; (i = 0, q = 1) lies above the
  // diagonal for every thread and is skipped
  uint64_t acc[RI][2];
#pragma unroll
  for (int i = 0; i < RI; ++i) acc[i][0] = acc[i][1] = 0ull;
#pragma unroll 4
  for (int k = 0; k < w; ++k) {
    const uint64_t q0 = pack2(X[xc[0] + k], X[xc[1] + k]);
    const uint64_t q1 = pack2(X[xc[2] + k], X[xc[3] + k]);
#pragma unroll
    for (int i = 0; i < RI; ++i) {
      const float v = X[xr[i] + k];
      const uint64_t vv = pack2(v, v);
      acc[i][0] = ffma2_u64(vv, q0, acc[i][0]);
      if (i > 0) acc[i][1] = ffma2_u64(vv, q1, acc[i][1]);
    }
  }
#pragma unroll
  for (int i = 0; i < RI; ++i)
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      if (i == 0 && c >= 2) continue;
      const int r = k1 + c0 + ty + 32 * i, col = k1 + c0 + tx + 16 * c;
      if (r < n && col <= r) {
        const int64_t o = int64_t(r) * n + col;
        const uint64_t v = acc[i][c >> 1];
        dst[o] = src[o] - ((c & 1) ? hi_of(v) : lo_of(v));
      }
    }
}

__device__ __forceinline__ void wide_update(const float* src, float* dst, int n, int k1, int c0,
                                            int w, int tid, const float* X) {
  switch ((n - k1 - c0 + 31) >> 5) {
    case 1: wide_update_t<1>(src, dst, n, k1, c0, w, tid, X); break;
    case 2: wide_update_t<2>(src, dst, n, k1, c0, w, tid, X); break;
    case 3: wide_update_t<3>(src, dst, n, k1, c0, w, tid, X); break;
    case 4: wide_update_t<4>(src, dst, n, k1, c0, w, tid, X); break;
    case 5: wide_update_t<5>(src, dst, n, k1, c0, w, tid, X); break;
    case 6: wide_update_t<6>(src, dst, n, k1, c0, w, tid, X); break;
    default: wide_update_t<7>(src, dst, n, k1, c0, w, tid, X); break;
  }
}

__global__ void __launch_bounds__(kWideThreads, 1)
    wide_potrf_kernel(const float* A, float* L, int64_t batch, int n, int* info) {
  griddep_wait();
  griddep_launch();
  extern __shared__ float sm[];
  float* P = sm;  // the current panel's rows, stride kXld
  float* cb = sm + kProws * kXld + 4 - (kProws * kXld) % 4;  // 16-byte aligned
  int* first = reinterpret_cast<int*>(cb + 8 * 64);  // one per warp of the diagonal scan
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int64_t m = blockIdx.x; m < batch; m += gridDim.x) {
    const float* Am = A + m * int64_t(n) * n;
    float* Lm = L + m * int64_t(n) * n;
    for (int r = warp; r < n; r += kWideThreads / 32)  // exact zeros above the diagonal
      for (int c = r + 1 + lane; c < n; c += 32) Lm[int64_t(r) * n + c] = 0.f;
    for (int k0 = 0; k0 < n; k0 += 32) {
      const int w = min(32, n - k0);
      const float* src = k0 == 0 ? Am : Lm;
      const int rows = n - k0;
      // the panel's rows into shared memory, one warp per 128-byte row segment (coalesced)
      for (int e = tid; e < rows * 32; e += kWideThreads) {
        const int r = e >> 5, c = e & 31;
        if (c < w) P[r * kXld + c] = src[int64_t(k0 + r) * n + k0 + c];
      }
      __syncthreads();
      smem_panel(P, kXld, rows, w, tid, cb);
      __syncthreads();
      for (int e = tid; e < rows * 32; e += kWideThreads) {  // the factored panel to L
        const int r = e >> 5, c = e & 31;
        if (c < w && c <= r) Lm[int64_t(k0 + r) * n + k0 + c] = P[r * kXld + c];
      }
      const int k1 = k0 + w;
      if (k1 < n)  // X = the panel's rows below its diagonal block
        for (int c0 = 0; c0 < n - k1; c0 += 64)
          wide_update(src, Lm, n, k1, c0, w, tid, P + w * kXld);
      __syncthreads();
    }
    if (info != nullptr) {
      // the first diagonal entry that is not > 0 (warps 0..7 scan 32 rows each)
      if (warp < 8) {
        const int c = warp * 32 + lane;
        const bool bad = c < n && !(Lm[int64_t(c) * n + c] > 0.f);
        const unsigned mask = __ballot_sync(0xffffffffu, bad);
        if (lane == 0) first[warp] = mask ? warp * 32 + __ffs(int(mask)) : 0;
      }
      __syncthreads();
      if (tid == 0) {
        int f = 0;
        for (int q = 0; q < 8 && f == 0; ++q) f = first[q];
        info[m] = f;
      }
    }
    __syncthreads();  // the next matrix's panel overwrites X
  }
}

size_t wide_smem_bytes() {
  return (size_t(kProws * kXld + 4 - (kProws * kXld) % 4) + 8 * 64 + 8) * sizeof(float);
}

size_t mid_smem_bytes(int n) { return (size_t(mid_aux_offset(n)) + 4 * 64) * sizeof(float); }

}  // namespace

int g_mid_kernel = 1;

// 64 < n <= 128: always. 128 < n <= 256: the wide kernel where the blocked schedule's
// one-launch path is weak, i.e. a ragged last 64-wide tile (n % 64 != 0), for batches of at
// most two CTAs per SM of a B200, or for n < 144 at any batch (A/B of library builds, us per
// call, wide against blocked: b64n129 41 / 79, b64n200 77 / 116, b16n255 110 / 139,
// b256n200 157 / 179, b148n160 48 / 88, b1024n129 304 / 346; but b1024n200 617 / 564,
// b600n160 249 / 206, b300n255 359 / 346, and for n % 64 == 0 the blocked path wins:
// b64n256 106 / 75, b64n192 63 / 51).
constexpr int64_t kWideBatchMax = 2 * 148;
bool use_mid(int64_t batch, int64_t n) {
  if (g_mid_kernel == 0 || n <= 64 || n > kWideMax) return false;
  if (n <= kMidMax) return true;
  return n % 64 != 0 && (batch <= kWideBatchMax || n < 144);
}

cudaError_t prepare_mid() {
  cudaError_t e = cudaFuncSetAttribute(mid_potrf_kernel,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       int(mid_smem_bytes(kMidMax)));
  if (e != cudaSuccess) return e;
  return cudaFuncSetAttribute(wide_potrf_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              int(wide_smem_bytes()));
}

int launch_mid(const float* A, float* L, int64_t batch, int n, int* info, cudaStream_t q) {
  if (n <= 64 || n > kWideMax) return CHOL_ERR_UNSUPPORTED;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (n > kMidMax) {
    const int64_t grid = std::min<int64_t>(batch, int64_t(sms) * 16);
    return status_from(launch_pdl(wide_potrf_kernel, dim3(unsigned(grid)), dim3(kWideThreads),
                                  wide_smem_bytes(), q, true, A, L, batch, n, info));
  }
  const int64_t grid = std::min<int64_t>(batch, int64_t(sms) * kMidCtasPerSm * 16);
  return status_from(launch_pdl(mid_potrf_kernel, dim3(unsigned(grid)), dim3(kMidThreads),
                                mid_smem_bytes(n), q, true, A, L, batch, n, info));
}

}  // namespace chol
