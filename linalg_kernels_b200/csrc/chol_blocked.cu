// chol_blocked.cu — building blocks of the blocked (n > 64) path.
//
//   copy_lower_kernel   L = tril(A) with exact zeros above the diagonal (one HBM pass).
//   potrf_block_kernel  factor one kb x kb (kb <= 64) diagonal block in place and write its
//                       inverse T = inv(L_kk) (lower, row-major 64 x 64) to workspace.
//   gemm_nt_simt        C = alpha * P * Q^T + beta * C on FP32 FMA, lower-tile aware; used
//                       for the panel solve X <- X * T^T (alpha 1, beta 0, in place) and
//                       the trailing update C -= P * Q^T (alpha -1, beta 1) when the
//                       tensor-core path does not apply.
//
// The reference's blocked shapes use the same three roles (factor_kernel / solve_kernel /
// cublasGemmStridedBatchedEx at cholesky/cholesky.py:2032-2656; factor128_kernel computing
// the diagonal block and its inverse T, then gemm_apply X*T^T, cholesky/cholesky.py:5440-5489,
// 5670-5690).
#include "chol_warp.cuh"

namespace chol {

// =====================================================================================
// copy_lower: L[m][i][j] = (j <= i) ? A[m][i][j] : 0.  One thread per 4 consecutive
// elements of a row (vector path when n % 4 == 0 and both bases are 16-byte aligned).
// =====================================================================================
template <bool VEC>
__global__ void __launch_bounds__(256)
    copy_lower_kernel(const float* __restrict__ A, float* __restrict__ L, int64_t batch,
                      int64_t n) {
  griddep_wait();
  griddep_launch();
  const int64_t per_row = VEC ? n / 4 : n;
  const int64_t total = batch * n * per_row;
  for (int64_t t = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; t < total;
       t += int64_t(gridDim.x) * blockDim.x) {
    const int64_t row_g = t / per_row;  // global row index over the batch
    const int64_t c = (t - row_g * per_row) * (VEC ? 4 : 1);
    const int64_t i = row_g % n;
    const int64_t off = row_g * n + c;
    if (VEC) {
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (c <= i) v = __ldcs(reinterpret_cast<const float4*>(A + off));
      if (c + 1 > i) v.y = 0.f;
      if (c + 2 > i) v.z = 0.f;
      if (c + 3 > i) v.w = 0.f;
      *reinterpret_cast<float4*>(L + off) = v;
    } else {
      L[off] = (c <= i) ? __ldcs(A + off) : 0.f;
    }
  }
}

int launch_copy_lower(const float* A, float* L, int64_t batch, int64_t n, cudaStream_t q,
                      bool pdl) {
  const bool vec = (n % 4 == 0) && ((reinterpret_cast<uintptr_t>(A) & 15) == 0) &&
                   ((reinterpret_cast<uintptr_t>(L) & 15) == 0);
  const int64_t work = batch * n * (vec ? n / 4 : n);
  int64_t blocks = (work + 255) / 256;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (blocks > int64_t(sms) * 16) blocks = int64_t(sms) * 16;
  if (blocks < 1) blocks = 1;
  cudaError_t e = vec ? launch_pdl(copy_lower_kernel<true>, dim3(unsigned(blocks)), dim3(256), 0,
                                   q, pdl, A, L, batch, n)
                      : launch_pdl(copy_lower_kernel<false>, dim3(unsigned(blocks)), dim3(256), 0,
                                   q, pdl, A, L, batch, n);
  return status_from(e);
}

// =====================================================================================
// zero_upper: L[m][i][j] = 0 for j >= bw * (i / bw + 1), the part of the strict upper
// triangle right of each row's bw-wide diagonal block (the diagonal blocks themselves are
// written whole, zeros included, by the block factor). Replaces copy_lower when the schedule
// reads A directly. One thread per 4 consecutive elements (vector path when n % 4 == 0).
// =====================================================================================
template <bool VEC>
__global__ void __launch_bounds__(256) zero_upper_kernel(float* __restrict__ L, int64_t batch,
                                                         int64_t n, int64_t bw) {
  griddep_wait();
  griddep_launch();
  const int64_t per_row = VEC ? n / 4 : n;
  const int64_t total = batch * n * per_row;
  for (int64_t t = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; t < total;
       t += int64_t(gridDim.x) * blockDim.x) {
    const int64_t row_g = t / per_row;
    const int64_t c = (t - row_g * per_row) * (VEC ? 4 : 1);
    const int64_t i = row_g % n;
    if (c < (i / bw + 1) * bw) continue;
    if (VEC)
      *reinterpret_cast<float4*>(L + row_g * n + c) = make_float4(0.f, 0.f, 0.f, 0.f);
    else
      L[row_g * n + c] = 0.f;
  }
}

int launch_zero_upper(float* L, int64_t batch, int64_t n, cudaStream_t q, bool pdl, int64_t bw) {
  const bool vec = (n % 4 == 0) && ((reinterpret_cast<uintptr_t>(L) & 15) == 0);
  const int64_t work = batch * n * (vec ? n / 4 : n);
  int64_t blocks = (work + 255) / 256;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (blocks > int64_t(sms) * 16) blocks = int64_t(sms) * 16;
  if (blocks < 1) blocks = 1;
  cudaError_t e = vec ? launch_pdl(zero_upper_kernel<true>, dim3(unsigned(blocks)), dim3(256), 0,
                                   q, pdl, L, batch, n, bw)
                      : launch_pdl(zero_upper_kernel<false>, dim3(unsigned(blocks)), dim3(256),
                                   0, q, pdl, L, batch, n, bw);
  return status_from(e);
}

// =====================================================================================
// potrf_block: one CTA per matrix factors the kb x kb block at (k, k).
//   S (+ m*sstride) with leading dimension lds is where the block is read from (A for the
//   first block when the copy is fused, else L); the factor goes to L (+ m*stride, ld).
//   Strict upper part of the block is written as zeros.
//   Tinv (+ m*tstride, leading dimension tld), if not null, receives inv(L_kk) as a 64 x 64
//   lower triangle with explicit zeros above the diagonal (rows/cols >= kb are identity).
//   info[m]: first failing global column (1-based); written when info[m] == 0 or k == 0.
// =====================================================================================
constexpr int kPB = 64;         // block size handled by one CTA
constexpr int kPBLD = kPB + 4;  // smem row stride

// NT = 128: threads 64..127 write the factored block while 0..63 compute the inverse (the
// shortest CTA; 3 per SM). NT = 64: two warps do both in turn (6 CTAs per SM): for batches
// beyond one wave of 128-thread CTAs (b640n512: 30 -> ~15 us per launch).
template <int NT>
__global__ void __launch_bounds__(NT)
    potrf_block_kernel(const float* __restrict__ S, int64_t sstride, int64_t lds,
                       float* __restrict__ L, int64_t stride, int64_t ld, int64_t k, int kb,
                       float* __restrict__ Tinv, int64_t tstride, int64_t tld,
                       int* __restrict__ info) {
  __shared__ __align__(16) float tile[kPB * kPBLD];
  __shared__ __align__(16) float col[2 * kPB];
  __shared__ float rdiag[kPB];
  const int tid = threadIdx.x;
  const int64_t m = blockIdx.x;
  const float* src = S + m * sstride + k * lds + k;
  float* dst = L + m * stride + k * ld + k;

  griddep_wait();
  griddep_launch();

  // load the block: every 4-byte element of the lower part in flight at once (cp.async),
  // identity outside kb, zeros above the diagonal
  for (int idx = tid; idx < kPB * kPB; idx += NT) {
    const int r = idx / kPB, c = idx % kPB;
    if (r < kb && c < kb) {
      if (c <= r)
        cp_async4(&tile[r * kPBLD + c], src + r * lds + c);
      else
        tile[r * kPBLD + c] = 0.f;
    } else {
      tile[r * kPBLD + c] = (r == c) ? 1.f : 0.f;
    }
  }
  cp_async_wait_all();
  __syncthreads();

  if (tid < 32) {
    const int fail = tile64_potrf<kPBLD>(tile, col, rdiag, tid);
    if (tid == 0 && info != nullptr) {
      const int f = (fail > kb) ? 0 : fail;
      if (k == 0)
        info[m] = f ? int(k) + f : 0;
      else if (f && info[m] == 0)
        info[m] = int(k) + f;
    }
  }
  __syncthreads();

  // T = inv(L_kk): thread c (< 64) computes column c in registers and writes it out
  if (Tinv != nullptr && tid < 64) {
    const int c = tid;
    float t[kPB];
    tile64_inverse_column<kPBLD>(tile, rdiag, c, t);
    float* tp = Tinv + m * tstride;
#pragma unroll
    for (int i = 0; i < kPB; ++i) tp[i * tld + c] = t[i];
  }
  // the factored block (rows/cols < kb) to L: threads 64..127, or all threads after T
  const int w0 = NT > 64 ? 64 : 0;
  if (tid >= w0) {
    for (int idx = tid - w0; idx < kb * kb; idx += NT - w0) {
      const int r = idx / kb, c = idx - r * kb;
      dst[r * ld + c] = tile[r * kPBLD + c];
    }
  }
}

int launch_potrf_block(const float* S, int64_t sstride, int64_t lds, float* L, int64_t stride,
                       int64_t ld, int64_t batch, int64_t k, int64_t kb, float* Tinv, int* info,
                       cudaStream_t q, bool pdl, int64_t tstride, int64_t tld) {
  if (kb < 1 || kb > kPB || tld < kPB) return CHOL_ERR_UNSUPPORTED;
  if (batch > 0x7fffffffLL) return CHOL_ERR_UNSUPPORTED;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  cudaError_t e =
      batch > int64_t(sms) * 3
          ? launch_pdl(potrf_block_kernel<64>, dim3(unsigned(batch)), dim3(64), 0, q, pdl, S,
                       sstride, lds, L, stride, ld, k, int(kb), Tinv, tstride, tld, info)
          : launch_pdl(potrf_block_kernel<128>, dim3(unsigned(batch)), dim3(128), 0, q, pdl, S,
                       sstride, lds, L, stride, ld, k, int(kb), Tinv, tstride, tld, info);
  return status_from(e);
}

// =====================================================================================
// potrf_block128: one CTA (128 threads) per matrix factors the 128 x 128 block at (k, k) as
// 2 x 2 blocks of 64 and writes T = inv(L_kk) (128 x 128, lower, zeros above):
//   L00 = chol(A00), T0 = inv(L00)          (one warp factors; 64 threads invert by columns)
//   L10 = A10 T0^T
//   L11 = chol(A11 - L10 L10^T), T1 = inv(L11)
//   T10 = -T1 (L10 T0)
// The 64 x 64 products run on FP32 FMA, 4 x 8 outputs per thread. The diagonal block of the
// 128-wide chain: one launch instead of two 64-wide factors, a GEMM and a solve, and the
// chain's GEMMs then take 128 columns at a time (half the launches and half the re-reads of
// the panel left of the block column). S (+ m*sstride, leading dimension lds) is where the
// block is read (A or L); only its lower part is read. The factor goes to L (+ m*stride, ld)
// with exact zeros above the diagonal of the block, and with zero_cols > 0 the zeros of
// L's rows k..k+127 right of the block (zero_cols columns) are written too (the upper part
// of L that no other step writes; the kernel's own work is latency-bound, so these stores
// cost little). T (+ m*tstride, leading dimension tld). info[m] as for potrf_block.
// Shared memory: four 64 x 64 tiles (row stride kPBLD).
// =====================================================================================
constexpr int kP2T = 128;  // threads
constexpr size_t kP2Smem = size_t(4 * 64 * kPBLD + 2 * kPB + kPB) * sizeof(float);

// acc[i][j] += sum_k X[k][4 tr + i] * Y[k][c_j] over the 64 x 64 tiles X, Y (row stride kPBLD),
// c_j = 4 tc + j (j < 4) and 32 + 4 tc + (j - 4) (j >= 4): each quarter-warp reads 32
// consecutive floats of a Y row (no bank conflicts). tr = tid >> 3 (0..15), tc = tid & 7.
__device__ __forceinline__ void p2_fma(float2 (&acc)[4][4], const float* X, const float* Y,
                                       int tr, int tc) {
#pragma unroll 4
  for (int k = 0; k < 64; ++k) {
    const float4 a = *reinterpret_cast<const float4*>(X + k * kPBLD + 4 * tr);
    const float4 b0 = *reinterpret_cast<const float4*>(Y + k * kPBLD + 4 * tc);
    const float4 b1 = *reinterpret_cast<const float4*>(Y + k * kPBLD + 32 + 4 * tc);
    const float av[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 ai = make_float2(av[i], av[i]);
      acc[i][0] = ffma2(ai, make_float2(b0.x, b0.y), acc[i][0]);
      acc[i][1] = ffma2(ai, make_float2(b0.z, b0.w), acc[i][1]);
      acc[i][2] = ffma2(ai, make_float2(b1.x, b1.y), acc[i][2]);
      acc[i][3] = ffma2(ai, make_float2(b1.z, b1.w), acc[i][3]);
    }
  }
}
__device__ __forceinline__ int p2_col(int tc, int j) { return j < 2 ? 4 * tc + 2 * j : 32 + 4 * tc + 2 * (j - 2); }
__device__ __forceinline__ void p2_zero(float2 (&acc)[4][4]) {
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = make_float2(0.f, 0.f);
}
// this thread's outputs (rows 4 tr + i, columns p2_col(tc, j), +1) to a row-major tile
// (global with leading dimension ld, or shared with kPBLD), scaled by sign
__device__ __forceinline__ void p2_store(float* X, int64_t ld, const float2 (&acc)[4][4],
                                         float sign, int tr, int tc) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float* rp = X + (4 * tr + i) * ld;
    *reinterpret_cast<float4*>(rp + 4 * tc) =
        make_float4(sign * acc[i][0].x, sign * acc[i][0].y, sign * acc[i][1].x, sign * acc[i][1].y);
    *reinterpret_cast<float4*>(rp + 32 + 4 * tc) =
        make_float4(sign * acc[i][2].x, sign * acc[i][2].y, sign * acc[i][3].x, sign * acc[i][3].y);
  }
}
// ... and transposed into a shared tile: X[c][r] = out[r][c]
__device__ __forceinline__ void p2_store_t(float* X, const float2 (&acc)[4][4], int tr, int tc) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int c = p2_col(tc, j);
    *reinterpret_cast<float4*>(X + c * kPBLD + 4 * tr) =
        make_float4(acc[0][j].x, acc[1][j].x, acc[2][j].x, acc[3][j].x);
    *reinterpret_cast<float4*>(X + (c + 1) * kPBLD + 4 * tr) =
        make_float4(acc[0][j].y, acc[1][j].y, acc[2][j].y, acc[3][j].y);
  }
}

// The unrolled factor and column inverse as single non-inlined copies: each runs twice per
// CTA, and a second inlined copy would be fetched cold from memory like the first.
__device__ __noinline__ int p2_factor64(float* tile, float* col, float* rdiag, int lane) {
  return tile64_potrf<kPBLD>(tile, col, rdiag, lane);
}
// column c of inv(L) for the factored tile: to dst (+ i * ldd + c, global) and as row c of Tt
__device__ __noinline__ void p2_inverse_col(const float* tile, const float* rdiag, int c,
                                            float* dst, int64_t ldd, float* Tt, float* Tr) {
  float t[kPB];
  tile64_inverse_column<kPBLD>(tile, rdiag, c, t);
#pragma unroll
  for (int i = 0; i < kPB; ++i) {
    dst[i * ldd + c] = t[i];
    if (Tr != nullptr) Tr[i * kPBLD + c] = t[i];
  }
#pragma unroll
  for (int i = 0; i < kPB; i += 4)
    *reinterpret_cast<float4*>(Tt + c * kPBLD + i) = make_float4(t[i], t[i + 1], t[i + 2], t[i + 3]);
}

__global__ void __launch_bounds__(kP2T, 3)
    potrf_block128_kernel(const float* __restrict__ S, int64_t sstride, int64_t lds,
                          float* __restrict__ L, int64_t stride, int64_t ld, int64_t k,
                          float* __restrict__ T, int64_t tstride, int64_t tld,
                          int* __restrict__ info, int64_t zero_cols) {
  extern __shared__ __align__(16) float p2_smem[];
  float* P0 = p2_smem;
  float* P1 = P0 + 64 * kPBLD;
  float* P2 = P1 + 64 * kPBLD;
  float* P3 = P2 + 64 * kPBLD;
  float* col = P3 + 64 * kPBLD;
  float* rdiag = col + 2 * kPB;
  const int tid = threadIdx.x, lane = tid & 31;
  const int tr = tid >> 3, tc = tid & 7;
  const int64_t m = blockIdx.x;
  const float* src = S + m * sstride + k * lds + k;
  float* dst = L + m * stride + k * ld + k;
  float* tm = T + m * tstride;

  griddep_wait();
  griddep_launch();

  // A00 (lower) -> P0; A10 -> P3 transposed (P3[c][r] = A10[r][c]); zeros above the diagonal
  for (int idx = tid; idx < 64 * 16; idx += kP2T) {
    const int r = idx >> 4, c4 = (idx & 15) * 4;
    if (c4 <= r) cp_async16(P0 + r * kPBLD + c4, src + r * lds + c4);
    const float4 v = __ldcg(reinterpret_cast<const float4*>(src + (64 + r) * lds + c4));
    P3[(c4 + 0) * kPBLD + r] = v.x;
    P3[(c4 + 1) * kPBLD + r] = v.y;
    P3[(c4 + 2) * kPBLD + r] = v.z;
    P3[(c4 + 3) * kPBLD + r] = v.w;
  }
  cp_async_wait_all();
  __syncthreads();
  for (int idx = tid; idx < 64 * 64; idx += kP2T) {
    const int r = idx >> 6, c = idx & 63;
    if (c > r) P0[r * kPBLD + c] = 0.f;
  }
  __syncthreads();
  int f0 = 0;
  if (tid < 32) f0 = p2_factor64(P0, col, rdiag, lane);
  __syncthreads();
  if (tid < 64) {
    // column c of T0: to global T, row-major to P1 (for L10 T0) and as row c of P2 (T0^T)
    p2_inverse_col(P0, rdiag, tid, tm, tld, P2, P1);
  } else {
    // L00 (and zeros to its right) to L; zeros right of T0 in T
    for (int idx = tid - 64; idx < 64 * 32; idx += 64) {
      const int r = idx >> 5, c4 = (idx & 31) * 4;
      const float4 v = c4 < 64 ? *reinterpret_cast<const float4*>(P0 + r * kPBLD + c4)
                               : make_float4(0.f, 0.f, 0.f, 0.f);
      *reinterpret_cast<float4*>(dst + r * ld + c4) = v;
      if (c4 >= 64) *reinterpret_cast<float4*>(tm + r * tld + c4) = v;
    }
  }
  __syncthreads();
  // A11 (lower) -> P0 while L10 = A10 T0^T is formed
  for (int idx = tid; idx < 64 * 16; idx += kP2T) {
    const int r = idx >> 4, c4 = (idx & 15) * 4;
    if (c4 <= r) cp_async16(P0 + r * kPBLD + c4, src + (64 + r) * lds + 64 + c4);
  }
  float2 acc[4][4];
  p2_zero(acc);
  p2_fma(acc, P3, P2, tr, tc);
  __syncthreads();
  p2_store(dst + 64 * ld, ld, acc, 1.f, tr, tc);  // L10
  p2_store_t(P3, acc, tr, tc);                      // P3 = L10^T
  cp_async_wait_all();
  __syncthreads();
  // S11 = A11 - L10 L10^T (lower part, zeros above) in P0
  p2_zero(acc);
  p2_fma(acc, P3, P3, tr, tc);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int r = 4 * tr + i;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int c = p2_col(tc, j);
      float* sp = P0 + r * kPBLD + c;
      sp[0] = (c <= r) ? sp[0] - acc[i][j].x : 0.f;
      sp[1] = (c + 1 <= r) ? sp[1] - acc[i][j].y : 0.f;
    }
  }
  __syncthreads();
  int f1 = 0;
  if (tid < 32) f1 = p2_factor64(P0, col, rdiag, lane);
  __syncthreads();
  if (tid < 64) {
    // column c of T1: to global T and as row c of P2 (T1^T)
    p2_inverse_col(P0, rdiag, tid, tm + 64 * tld + 64, tld, P2, nullptr);
  } else {
    // L11 to L
    for (int idx = tid - 64; idx < 64 * 16; idx += 64) {
      const int r = idx >> 4, c4 = (idx & 15) * 4;
      *reinterpret_cast<float4*>(dst + (64 + r) * ld + 64 + c4) =
          *reinterpret_cast<const float4*>(P0 + r * kPBLD + c4);
    }
  }
  // zeros of rows k..k+127 right of the block (streaming stores)
  for (int64_t idx = tid; idx < 128 * (zero_cols / 4); idx += kP2T) {
    const int64_t r = idx / (zero_cols / 4), c4 = (idx - r * (zero_cols / 4)) * 4;
    __stcs(reinterpret_cast<float4*>(dst + r * ld + 128 + c4), make_float4(0.f, 0.f, 0.f, 0.f));
  }
  // Y = L10 T0 (P3 = L10^T, P1 = T0 row-major) into P0 once L11 is out
  p2_zero(acc);
  p2_fma(acc, P3, P1, tr, tc);
  __syncthreads();
  p2_store(P0, kPBLD, acc, 1.f, tr, tc);
  __syncthreads();
  // T10 = -T1 Y (P2 = T1^T)
  p2_zero(acc);
  p2_fma(acc, P2, P0, tr, tc);
  p2_store(tm + 64 * tld, tld, acc, -1.f, tr, tc);
  if (tid == 0 && info != nullptr) {
    const int f = f0 ? f0 : (f1 ? 64 + f1 : 0);
    if (k == 0)
      info[m] = f ? int(k) + f : 0;
    else if (f && info[m] == 0)
      info[m] = int(k) + f;
  }
}

int launch_potrf_block128(const float* S, int64_t sstride, int64_t lds, float* L, int64_t stride,
                          int64_t ld, int64_t batch, int64_t k, float* T, int64_t tstride,
                          int64_t tld, int* info, cudaStream_t q, int64_t zero_cols) {
  if (batch > 0x7fffffffLL || tld < 128 || lds % 4 || ld % 4 || tld % 4 || zero_cols % 4 ||
      (reinterpret_cast<uintptr_t>(S) & 15) || (reinterpret_cast<uintptr_t>(L) & 15) ||
      (reinterpret_cast<uintptr_t>(T) & 15))
    return CHOL_ERR_UNSUPPORTED;
  return status_from(launch_pdl(potrf_block128_kernel, dim3(unsigned(batch)), dim3(kP2T), kP2Smem,
                                q, true, S, sstride, lds, L, stride, ld, k, T, tstride, tld, info,
                                zero_cols));
}

// =====================================================================================
// trtri_panel: V = inv(L11) for the KB x KB diagonal block of an outer panel
// (KB = 64 * nblk), given the diagonal inverses T_j = inv(L_jj) that potrf_block already
// wrote into V's diagonal blocks. Column block jb of V solves L11 V[:, jb] = E[:, jb] by
// block forward substitution:
//   V[jb][jb] = T_jb,   V[i][jb] = -T_i * sum_{k=jb}^{i-1} L[i][k] V[k][jb]   (i > jb).
// The columns of V are independent, so each CTA owns kTW columns of one column block,
// keeps its column slice of V in shared memory, and streams the 64 x 64 tiles it needs
// (L[i][k] for k < i, then T_i) through a two-slot cp.async ring in the order it uses them.
// It also writes zeros to V's blocks above the diagonal block, so V is a full lower
// triangle for the GEMM that reads whole rows of it. FP32 FMA throughout.
// =====================================================================================
constexpr int kTW = 8;        // V columns per CTA
constexpr int kTLD = 68;      // ring tile row stride (floats)
constexpr int kTRing = 64 * kTLD;

size_t trtri_smem(int nblk) {
  return (size_t(nblk) * 64 * kTW + 2 * kTRing + 64 * kTW) * sizeof(float);
}

__global__ void __launch_bounds__(128)
    trtri_panel_kernel(const float* __restrict__ L11, int64_t lstride, int64_t ld,
                       float* __restrict__ V, int64_t vstride, int64_t ldv, int nblk,
                       int64_t batch) {
  extern __shared__ __align__(16) float tsm[];
  griddep_wait();
  griddep_launch();
  const int64_t mi = int64_t(blockIdx.y) + int64_t(blockIdx.z) * 65535;
  if (mi >= batch) return;
  float* Vs = tsm;                           // [nblk*64][kTW]: this CTA's column slice
  float* ring = Vs + nblk * 64 * kTW;        // 2 x [64][kTLD]
  float* As = ring + 2 * kTRing;             // [64][kTW]: block row sum before T_i
  constexpr int kPer = 64 / kTW;
  const int jb = blockIdx.x / kPer;
  const int c0 = jb * 64 + (blockIdx.x % kPer) * kTW;  // first V column of this CTA
  const int tid = threadIdx.x;
  const int r = tid >> 1, cg = (tid & 1) * 4;          // output row, first of 4 columns
  const float* Lm = L11 + mi * lstride;
  float* Vm = V + mi * vstride;

  // tile s of the sequence: for i = jb+1.., tiles L[i][k] (k = jb..i-1) then T_i (k == i)
  auto tile_of = [&](int s, int& ti, int& tk) {
    int i = jb + 1;
    while (s > i - jb) {
      s -= i - jb + 1;
      ++i;
    }
    ti = i;
    tk = jb + s;
  };
  const int total = (nblk - 1 - jb) * (nblk - jb + 2) / 2;
  auto issue = [&](int s) {
    int ti, tk;
    tile_of(s, ti, tk);
    const float* src = (tk < ti) ? Lm + int64_t(ti) * 64 * ld + tk * 64
                                 : Vm + int64_t(ti) * 64 * ldv + ti * 64;
    const int64_t lds = (tk < ti) ? ld : ldv;
    float* dst = ring + (s & 1) * kTRing;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int idx = tid + e * 128;
      const int rr = idx >> 4, cc = (idx & 15) * 4;
      cp_async16(dst + rr * kTLD + cc, src + rr * lds + cc);
    }
  };

  if (total > 0) issue(0);
  cp_async_commit();
  const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int i = 0; i < jb; ++i)
    *reinterpret_cast<float4*>(Vm + int64_t(i * 64 + r) * ldv + c0 + cg) = z;
  *reinterpret_cast<float4*>(Vs + (jb * 64 + r) * kTW + cg) =
      *reinterpret_cast<const float4*>(Vm + int64_t(jb * 64 + r) * ldv + c0 + cg);
  __syncthreads();

  int s = 0;
  for (int i = jb + 1; i < nblk; ++i) {
    float2 acc0 = make_float2(0.f, 0.f), acc1 = make_float2(0.f, 0.f);
    for (int k = jb; k <= i; ++k, ++s) {
      if (s + 1 < total) issue(s + 1);
      cp_async_commit();
      cp_async_wait_group<1>();
      __syncthreads();
      const float* tile = ring + (s & 1) * kTRing + r * kTLD;
      if (k < i) {
        const float* vk = Vs + k * 64 * kTW + cg;
#pragma unroll 16
        for (int kk = 0; kk < 64; ++kk) {
          const float a = tile[kk];
          const float4 b = *reinterpret_cast<const float4*>(vk + kk * kTW);
          acc0 = ffma2(make_float2(a, a), make_float2(b.x, b.y), acc0);
          acc1 = ffma2(make_float2(a, a), make_float2(b.z, b.w), acc1);
        }
      } else {
        *reinterpret_cast<float4*>(As + r * kTW + cg) = make_float4(acc0.x, acc0.y, acc1.x, acc1.y);
        __syncthreads();
        float2 o0 = make_float2(0.f, 0.f), o1 = make_float2(0.f, 0.f);
#pragma unroll 16
        for (int kk = 0; kk < 64; ++kk) {  // T_i is lower with zeros above its diagonal
          const float t = tile[kk];
          const float4 b = *reinterpret_cast<const float4*>(As + kk * kTW + cg);
          o0 = ffma2(make_float2(t, t), make_float2(b.x, b.y), o0);
          o1 = ffma2(make_float2(t, t), make_float2(b.z, b.w), o1);
        }
        const float4 o = make_float4(-o0.x, -o0.y, -o1.x, -o1.y);
        *reinterpret_cast<float4*>(Vs + (i * 64 + r) * kTW + cg) = o;
        *reinterpret_cast<float4*>(Vm + int64_t(i * 64 + r) * ldv + c0 + cg) = o;
      }
      __syncthreads();  // the slot is refilled by the next iteration's issue
    }
  }
  cp_async_wait_group<0>();
}

cudaError_t prepare_blocked() {
  cudaError_t e = cudaFuncSetAttribute(potrf_block128_kernel,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, int(kP2Smem));
  if (e != cudaSuccess) return e;
  return cudaFuncSetAttribute(trtri_panel_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              int(trtri_smem(16)));
}

int launch_trtri_panel(const float* L11, int64_t lstride, int64_t ld, float* V, int64_t vstride,
                       int64_t ldv, int nblk, int64_t batch, cudaStream_t q) {
  if (nblk < 1 || batch <= 0) return CHOL_OK;
  if (nblk > 16 || ld % 4 || ldv % 4 || ldv < 64 * nblk) return CHOL_ERR_UNSUPPORTED;
  if ((reinterpret_cast<uintptr_t>(L11) & 15) || (reinterpret_cast<uintptr_t>(V) & 15))
    return CHOL_ERR_UNSUPPORTED;
  const int64_t gy = batch < 65535 ? batch : 65535;
  const int64_t gz = (batch + 65534) / 65535;
  if (gz > 65535) return CHOL_ERR_UNSUPPORTED;
  const dim3 grid(unsigned(nblk * (64 / kTW)), unsigned(gy), unsigned(gz));
  return status_from(launch_pdl(trtri_panel_kernel, grid, dim3(128), trtri_smem(nblk), q, true,
                                L11, lstride, ld, V, vstride, ldv, nblk, batch));
}

// =====================================================================================
// gemm_nt_simt: C[r][c] = alpha * sum_q P[r][q] Q[c][q] + beta * C[r][c]
//   r in [0, m), c in [0, ncols), q in [0, K); all row-major with K contiguous.
//   lower_only: only elements with c <= r + diag_offset are written (tiles wholly above
//   that line exit at once). Batched over blockIdx.z (+ blockIdx.y * 65535).
//   Tile BM x BN = 128 x BN, 8 x 8 outputs per thread, K chunks of 16.
//   In-place use (C aliases P, beta == 0) is valid when ncols <= BN: every CTA reads all
//   of its rows' K range before its epilogue and no other CTA reads those rows.
// =====================================================================================

template <int BN, bool VEC>
__global__ void __launch_bounds__(BN * 2)
    gemm_nt_simt(GemmArgs g) {
  constexpr int BM = 128, BK = 16, TM = 8, TN = 8;
  constexpr int NT = BN * 2;          // threads
  constexpr int TX = BN / TN;         // threads along N
  __shared__ __align__(16) float Ps[2][BK][BM + 4];
  __shared__ __align__(16) float Qs[2][BK][BN + 4];

  // Wait before any early exit: a kernel whose CTAs all left early could otherwise
  // complete before its predecessor and release the next kernel's wait too soon.
  griddep_wait();
  griddep_launch();
  const int64_t mi = int64_t(blockIdx.z) + int64_t(blockIdx.y) * 65535;
  if (mi >= g.batch) return;
  const int tiles_n = int((g.ncols + BN - 1) / BN);
  const int tm = blockIdx.x / tiles_n, tn = blockIdx.x % tiles_n;
  const int64_t r0 = int64_t(tm) * BM, c0 = int64_t(tn) * BN;
  if (g.lower_only && c0 > r0 + BM - 1 + g.diag_offset) return;

  const float* P = g.P + mi * g.pstride + r0 * g.ldp;
  const float* Q = g.Q + mi * g.qstride + c0 * g.ldq;
  float* C = g.C + mi * g.cstride;
  const int tid = threadIdx.x;
  const int tx = tid % TX, ty = tid / TX;

  float acc[TM][TN];
#pragma unroll
  for (int i = 0; i < TM; ++i)
#pragma unroll
    for (int j = 0; j < TN; ++j) acc[i][j] = 0.f;

  // global -> register staging
  constexpr int PV = BM * BK / 4 / NT;  // float4 per thread for P
  constexpr int QV = BN * BK / 4 / NT;  // float4 per thread for Q
  float4 pr[PV > 0 ? PV : 1], qr[QV > 0 ? QV : 1];
  const int64_t mrows = g.m - r0, nrows = g.ncols - c0;

  auto load = [&](int64_t kq) {
#pragma unroll
    for (int v = 0; v < PV; ++v) {
      const int idx = tid + v * NT;
      const int row = idx / (BK / 4), kk = (idx % (BK / 4)) * 4;
      float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
      if (row < mrows) {
        const float* p = P + row * g.ldp + kq + kk;
        if (VEC && kq + kk + 3 < g.K) {
          x = *reinterpret_cast<const float4*>(p);
        } else {
          if (kq + kk + 0 < g.K) x.x = p[0];
          if (kq + kk + 1 < g.K) x.y = p[1];
          if (kq + kk + 2 < g.K) x.z = p[2];
          if (kq + kk + 3 < g.K) x.w = p[3];
        }
      }
      pr[v] = x;
    }
#pragma unroll
    for (int v = 0; v < QV; ++v) {
      const int idx = tid + v * NT;
      const int row = idx / (BK / 4), kk = (idx % (BK / 4)) * 4;
      float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
      if (row < nrows) {
        const float* p = Q + row * g.ldq + kq + kk;
        if (VEC && kq + kk + 3 < g.K) {
          x = *reinterpret_cast<const float4*>(p);
        } else {
          if (kq + kk + 0 < g.K) x.x = p[0];
          if (kq + kk + 1 < g.K) x.y = p[1];
          if (kq + kk + 2 < g.K) x.z = p[2];
          if (kq + kk + 3 < g.K) x.w = p[3];
        }
      }
      qr[v] = x;
    }
  };
  auto store = [&](int buf) {
#pragma unroll
    for (int v = 0; v < PV; ++v) {
      const int idx = tid + v * NT;
      const int row = idx / (BK / 4), kk = (idx % (BK / 4)) * 4;
      Ps[buf][kk + 0][row] = pr[v].x;
      Ps[buf][kk + 1][row] = pr[v].y;
      Ps[buf][kk + 2][row] = pr[v].z;
      Ps[buf][kk + 3][row] = pr[v].w;
    }
#pragma unroll
    for (int v = 0; v < QV; ++v) {
      const int idx = tid + v * NT;
      const int row = idx / (BK / 4), kk = (idx % (BK / 4)) * 4;
      Qs[buf][kk + 0][row] = qr[v].x;
      Qs[buf][kk + 1][row] = qr[v].y;
      Qs[buf][kk + 2][row] = qr[v].z;
      Qs[buf][kk + 3][row] = qr[v].w;
    }
  };

  load(0);
  store(0);
  __syncthreads();
  int buf = 0;
  for (int64_t kq = 0; kq < g.K; kq += BK) {
    const bool more = kq + BK < g.K;
    if (more) load(kq + BK);
#pragma unroll
    for (int kk = 0; kk < BK; ++kk) {
      const float4 a0 = *reinterpret_cast<const float4*>(&Ps[buf][kk][ty * TM]);
      const float4 a1 = *reinterpret_cast<const float4*>(&Ps[buf][kk][ty * TM + 4]);
      const float4 b0 = *reinterpret_cast<const float4*>(&Qs[buf][kk][tx * TN]);
      const float4 b1 = *reinterpret_cast<const float4*>(&Qs[buf][kk][tx * TN + 4]);
      const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
      const float2 bv[4] = {make_float2(b0.x, b0.y), make_float2(b0.z, b0.w),
                            make_float2(b1.x, b1.y), make_float2(b1.z, b1.w)};
#pragma unroll
      for (int i = 0; i < TM; ++i) {
        const float2 ai = make_float2(av[i], av[i]);
#pragma unroll
        for (int j = 0; j < TN / 2; ++j) {
          const float2 r = ffma2(ai, bv[j], make_float2(acc[i][2 * j], acc[i][2 * j + 1]));
          acc[i][2 * j] = r.x;
          acc[i][2 * j + 1] = r.y;
        }
      }
    }
    if (more) {
      store(buf ^ 1);
      __syncthreads();
      buf ^= 1;
    }
  }

  // epilogue
#pragma unroll
  for (int i = 0; i < TM; ++i) {
    const int64_t r = r0 + ty * TM + i;
    if (r >= g.m) continue;
    float* crow = C + r * g.ldc;
    const float* srow = (g.Csrc != nullptr ? g.Csrc + mi * g.cstride : C) + r * g.ldc;
#pragma unroll
    for (int j = 0; j < TN; ++j) {
      const int64_t c = c0 + tx * TN + j;
      if (c >= g.ncols) continue;
      if (g.lower_only && c > r + g.diag_offset) continue;
      float v = g.alpha * acc[i][j];
      if (g.beta != 0.f) v = fmaf(g.beta, srow[c], v);
      crow[c] = v;
    }
  }
}

int launch_gemm_simt(const GemmArgs& g, cudaStream_t q, bool pdl) {
  if (g.m <= 0 || g.ncols <= 0) return CHOL_OK;
  const bool vec = (g.ldp % 4 == 0) && (g.ldq % 4 == 0) && (g.pstride % 4 == 0) &&
                   (g.qstride % 4 == 0) && ((reinterpret_cast<uintptr_t>(g.P) & 15) == 0) &&
                   ((reinterpret_cast<uintptr_t>(g.Q) & 15) == 0);
  const bool narrow = g.ncols <= 64;
  const int BN = narrow ? 64 : 128;
  const int64_t tiles = ((g.m + 127) / 128) * ((g.ncols + BN - 1) / BN);
  if (tiles > 0x7fffffffLL) return CHOL_ERR_UNSUPPORTED;
  const int64_t bz = g.batch < 65535 ? g.batch : 65535;
  const int64_t by = (g.batch + 65534) / 65535;
  const dim3 grid = dim3(unsigned(tiles), unsigned(by), unsigned(bz));
  cudaError_t e;
  if (narrow)
    e = vec ? launch_pdl(gemm_nt_simt<64, true>, grid, dim3(128), 0, q, pdl, g)
            : launch_pdl(gemm_nt_simt<64, false>, grid, dim3(128), 0, q, pdl, g);
  else
    e = vec ? launch_pdl(gemm_nt_simt<128, true>, grid, dim3(256), 0, q, pdl, g)
            : launch_pdl(gemm_nt_simt<128, false>, grid, dim3(256), 0, q, pdl, g);
  return status_from(e);
}

}  // namespace chol
