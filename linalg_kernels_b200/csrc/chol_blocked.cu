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
// potrf_block: one CTA (128 threads) per matrix factors the kb x kb block at (k, k).
//   S (+ m*sstride) with leading dimension lds is where the block is read from (A for the
//   first block when the copy is fused, else L); the factor goes to L (+ m*stride, ld).
//   Strict upper part of the block is written as zeros.
//   Tinv (+ m*4096), if not null, receives inv(L_kk) as a row-major 64 x 64 lower
//   triangle (rows/cols >= kb are identity).
//   info[m]: first failing global column (1-based); written when info[m] == 0 or k == 0.
// =====================================================================================
constexpr int kPB = 64;         // block size handled by one CTA
constexpr int kPBLD = kPB + 4;  // smem row stride

__global__ void __launch_bounds__(128)
    potrf_block_kernel(const float* __restrict__ S, int64_t sstride, int64_t lds,
                       float* __restrict__ L, int64_t stride, int64_t ld, int64_t k, int kb,
                       float* __restrict__ Tinv, int* __restrict__ info) {
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
  for (int idx = tid; idx < kPB * kPB; idx += 128) {
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
    uint64_t a[2][32];
#pragma unroll
    for (int s = 0; s < 2; ++s) {
      const float* rp = tile + (s * 32 + tid) * kPBLD;
#pragma unroll
      for (int q = 0; q < (s + 1) * 8; ++q) {
        const ulonglong2 v = *reinterpret_cast<const ulonglong2*>(rp + 4 * q);
        a[s][2 * q] = v.x;
        a[s][2 * q + 1] = v.y;
      }
    }
    warp_potrf_rows<64>(a, col, tid);
    __syncwarp();
#pragma unroll
    for (int s = 0; s < 2; ++s) {
      const int i = s * 32 + tid;
      float* rp = tile + i * kPBLD;
#pragma unroll
      for (int q = 0; q < kPB / 4; ++q) {
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
    const float d0 = tile[tid * kPBLD + tid];
    const float d1 = tile[(tid + 32) * kPBLD + tid + 32];
    rdiag[tid] = __frcp_rn(d0);
    rdiag[tid + 32] = __frcp_rn(d1);
    // first row whose diagonal is not > 0 (NaN included) is the first failing column
    const unsigned b0 = __ballot_sync(0xffffffffu, !(d0 > 0.f));
    const unsigned b1 = __ballot_sync(0xffffffffu, !(d1 > 0.f));
    const int fail = b0 ? __ffs(b0) : (b1 ? 32 + __ffs(b1) : 0);
    if (tid == 0 && info != nullptr) {
      const int f = (fail > kb) ? 0 : fail;
      if (k == 0)
        info[m] = f ? int(k) + f : 0;
      else if (f && info[m] == 0)
        info[m] = int(k) + f;
    }
  }
  __syncthreads();

  if (tid >= 64) {
    // threads 64..127: write the factored block (rows/cols < kb) to L
    for (int idx = tid - 64; idx < kb * kb; idx += 64) {
      const int r = idx / kb, c = idx - r * kb;
      dst[r * ld + c] = tile[r * kPBLD + c];
    }
  } else if (Tinv != nullptr) {
    // threads 0..63: column c of T = inv(L_kk) by forward substitution on e_c,
    //   t[i] = -rdiag[i] * sum_{m<i} L[i][m] t[m]  (i > c),  t[c] = rdiag[c],  t[i<c] = 0
    const int c = tid;
    float t[kPB];
#pragma unroll
    for (int i = 0; i < kPB; ++i) {
      const float* rp = tile + i * kPBLD;
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
    float* tp = Tinv + m * (kPB * kPB);
#pragma unroll
    for (int i = 0; i < kPB; ++i) tp[i * kPB + c] = t[i];
  }
}

int launch_potrf_block(const float* S, int64_t sstride, int64_t lds, float* L, int64_t stride,
                       int64_t ld, int64_t batch, int64_t k, int64_t kb, float* Tinv, int* info,
                       cudaStream_t q, bool pdl) {
  if (kb < 1 || kb > kPB) return CHOL_ERR_UNSUPPORTED;
  if (batch > 0x7fffffffLL) return CHOL_ERR_UNSUPPORTED;
  cudaError_t e = launch_pdl(potrf_block_kernel, dim3(unsigned(batch)), dim3(128), 0, q, pdl, S,
                             sstride, lds, L, stride, ld, k, int(kb), Tinv, info);
  return status_from(e);
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
#pragma unroll
    for (int j = 0; j < TN; ++j) {
      const int64_t c = c0 + tx * TN + j;
      if (c >= g.ncols) continue;
      if (g.lower_only && c > r + g.diag_offset) continue;
      float v = g.alpha * acc[i][j];
      if (g.beta != 0.f) v = fmaf(g.beta, crow[c], v);
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
