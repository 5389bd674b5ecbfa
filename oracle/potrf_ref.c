/*
 * potrf_ref.c — CPU ORACLE (test infrastructure only; never part of the product path).
 *
 * A plain-C restatement of the algorithm the reference path runs for its CPU/default
 * case: custom_kernel falls back to torch.linalg.cholesky_ex(data, check_errors=False).L
 * (cholesky/cholesky.py:5850, submission.py:6-7), which calls LAPACK xPOTRF with
 * uplo='L' (here: Intel MKL 2024.2, bundled with torch 2.11; not vendored in the
 * reference tree). LAPACK's published blocked algorithm for the lower case is restated:
 *
 *   SPOTRF (lower, block size nb):
 *     for j = 0, nb, 2nb, ...:            jb = min(nb, n - j)
 *       A[j:j+jb, j:j+jb] -= A[j:j+jb, 0:j] A[j:j+jb, 0:j]^T        (SSYRK, lower)
 *       SPOTF2(A[j:j+jb, j:j+jb])                                   (unblocked)
 *       A[j+jb:, j:j+jb] -= A[j+jb:, 0:j] A[j:j+jb, 0:j]^T         (SGEMM)
 *       A[j+jb:, j:j+jb] <- A[j+jb:, j:j+jb] L_jj^{-T}             (STRSM, right, lower^T)
 *   SPOTF2 (lower):
 *     for j: ajj = a[j][j] - dot(a[j][0:j], a[j][0:j]);  if !(ajj > 0): info = j+1, stop
 *            ajj = sqrt(ajj);  a[j][j] = ajj
 *            a[i][j] = (a[i][j] - dot(a[i][0:j], a[j][0:j])) * (1/ajj)     (i > j)
 *
 * All arithmetic is IEEE float32 with float32 accumulation, as in reference BLAS. MKL uses
 * its own (recursive, vectorised) blocking, so this oracle agrees with the reference to
 * rounding, not bitwise; tests/golden holds the reference's own outputs to pin that.
 * The strict upper triangle of the output is set to zero (torch's cholesky_ex does the
 * same to the returned L).
 *
 * Interface (row-major, batch of n x n, matrix m at a + m*n*n):
 *   int oracle_spotrf_batched(const float* a, float* l, long batch, long n, int nb, int* info)
 *   int oracle_dpotrf_batched(const float* a, double* l, long batch, long n, int* info)
 *       (float64 unblocked factor of the same float32 input, for diagnostics)
 *   returns the number of matrices with info > 0.
 */
#include <math.h>
#include <stdlib.h>
#include <string.h>

static int spotf2_lower(float* a, long n, long lda) {
  for (long j = 0; j < n; ++j) {
    float* aj = a + j * lda;
    float dot = 0.f;
    for (long k = 0; k < j; ++k) dot += aj[k] * aj[k];
    float ajj = aj[j] - dot;
    if (!(ajj > 0.f)) {
      aj[j] = ajj;
      return (int)(j + 1);
    }
    ajj = sqrtf(ajj);
    aj[j] = ajj;
    const float r = 1.f / ajj;
    for (long i = j + 1; i < n; ++i) {
      float* ai = a + i * lda;
      float s = 0.f;
      for (long k = 0; k < j; ++k) s += ai[k] * aj[k];
      ai[j] = (ai[j] - s) * r;
    }
  }
  return 0;
}

/* C[r][c] -= sum_k P[r][k] Q[c][k]  for r < m, c < ncols (c <= r when lower). */
static void sgemm_nt_sub(float* c, long ldc, const float* p, long ldp, const float* q, long ldq,
                         long m, long ncols, long kdim, int lower) {
  for (long r = 0; r < m; ++r) {
    const float* pr = p + r * ldp;
    const long cend = lower ? (r + 1 < ncols ? r + 1 : ncols) : ncols;
    for (long cc = 0; cc < cend; ++cc) {
      const float* qc = q + cc * ldq;
      float s = 0.f;
      for (long k = 0; k < kdim; ++k) s += pr[k] * qc[k];
      c[r * ldc + cc] -= s;
    }
  }
}

/* X <- X L^{-T}, X is m x jb, L lower jb x jb (row-major, ld). Forward substitution per row. */
static void strsm_rlt(float* x, long ldx, const float* l, long ldl, long m, long jb) {
  for (long r = 0; r < m; ++r) {
    float* xr = x + r * ldx;
    for (long j = 0; j < jb; ++j) {
      const float* lj = l + j * ldl;
      float s = xr[j];
      for (long k = 0; k < j; ++k) s -= xr[k] * lj[k];
      xr[j] = s / lj[j];
    }
  }
}

static int spotrf_lower(float* a, long n, long lda, int nb) {
  if (nb <= 1 || nb >= n) return spotf2_lower(a, n, lda);
  for (long j = 0; j < n; j += nb) {
    const long jb = (n - j) < nb ? (n - j) : nb;
    float* ajj = a + j * lda + j;
    sgemm_nt_sub(ajj, lda, a + j * lda, lda, a + j * lda, lda, jb, jb, j, 1);
    int info = spotf2_lower(ajj, jb, lda);
    if (info) return (int)j + info;
    if (j + jb < n) {
      float* below = a + (j + jb) * lda + j;
      sgemm_nt_sub(below, lda, a + (j + jb) * lda, lda, a + j * lda, lda, n - j - jb, jb, j, 0);
      strsm_rlt(below, lda, ajj, lda, n - j - jb, jb);
    }
  }
  return 0;
}

int oracle_spotrf_batched(const float* a, float* l, long batch, long n, int nb, int* info) {
  int bad = 0;
  for (long m = 0; m < batch; ++m) {
    const float* src = a + m * n * n;
    float* dst = l + m * n * n;
    for (long i = 0; i < n; ++i)
      for (long j = 0; j < n; ++j) dst[i * n + j] = (j <= i) ? src[i * n + j] : 0.f;
    int inf = spotrf_lower(dst, n, n, nb);
    if (info) info[m] = inf;
    if (inf) ++bad;
    for (long i = 0; i < n; ++i)
      for (long j = i + 1; j < n; ++j) dst[i * n + j] = 0.f;
  }
  return bad;
}

int oracle_dpotrf_batched(const float* a, double* l, long batch, long n, int* info) {
  int bad = 0;
  for (long m = 0; m < batch; ++m) {
    const float* src = a + m * n * n;
    double* d = l + m * n * n;
    int inf = 0;
    for (long i = 0; i < n; ++i)
      for (long j = 0; j < n; ++j) d[i * n + j] = (j <= i) ? (double)src[i * n + j] : 0.0;
    for (long j = 0; j < n && !inf; ++j) {
      double* dj = d + j * n;
      double s = dj[j];
      for (long k = 0; k < j; ++k) s -= dj[k] * dj[k];
      if (!(s > 0.0)) {
        inf = (int)(j + 1);
        break;
      }
      s = sqrt(s);
      dj[j] = s;
      for (long i = j + 1; i < n; ++i) {
        double* di = d + i * n;
        double t = di[j];
        for (long k = 0; k < j; ++k) t -= di[k] * dj[k];
        di[j] = t / s;
      }
    }
    if (info) info[m] = inf;
    if (inf) ++bad;
  }
  return bad;
}
