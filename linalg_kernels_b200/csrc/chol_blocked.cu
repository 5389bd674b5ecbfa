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
// zero_upper: L[m][i][j] = 0 for j >= 64 * (i / 64 + 1), the part of the strict upper
// triangle right of each row's 64-wide diagonal block (the diagonal blocks themselves are
// written whole, zeros included, by potrf_block). Replaces copy_lower when the schedule
// reads A directly. One thread per 4 consecutive elements (vector path when n % 4 == 0).
// =====================================================================================
template <bool VEC>
__global__ void __launch_bounds__(256) zero_upper_kernel(float* __restrict__ L, int64_t batch,
                                                         int64_t n) {
  griddep_wait();
  griddep_launch();
  const int64_t per_row = VEC ? n / 4 : n;
  const int64_t total = batch * n * per_row;
  for (int64_t t = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; t < total;
       t += int64_t(gridDim.x) * blockDim.x) {
    const int64_t row_g = t / per_row;
    const int64_t c = (t - row_g * per_row) * (VEC ? 4 : 1);
    const int64_t i = row_g % n;
    if (c < (i / 64 + 1) * 64) continue;
    if (VEC)
      *reinterpret_cast<float4*>(L + row_g * n + c) = make_float4(0.f, 0.f, 0.f, 0.f);
    else
      L[row_g * n + c] = 0.f;
  }
}

int launch_zero_upper(float* L, int64_t batch, int64_t n, cudaStream_t q, bool pdl) {
  const bool vec = (n % 4 == 0) && ((reinterpret_cast<uintptr_t>(L) & 15) == 0);
  const int64_t work = batch * n * (vec ? n / 4 : n);
  int64_t blocks = (work + 255) / 256;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (blocks > int64_t(sms) * 16) blocks = int64_t(sms) * 16;
  if (blocks < 1) blocks = 1;
  cudaError_t e = vec ? launch_pdl(zero_upper_kernel<true>, dim3(unsigned(blocks)), dim3(256), 0,
                                   q, pdl, L, batch, n)
                      : launch_pdl(zero_upper_kernel<false>, dim3(unsigned(blocks)), dim3(256),
                                   0, q, pdl, L, batch, n);
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
