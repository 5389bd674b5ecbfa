// chol_check.cu — the property gates of a factor, checked on the device.
//
// The reference's checker validates finiteness, lower-triangular structure, a positive
// diagonal and the reconstruction residual against the original FP32 input (reference
// AGENTS.md:47-50; the harness gate of cholesky/b4096n32/cholesky_b4096n32_modal.py:307-334
// adds the scaled inf-norm residual). On the host these need L L^T in FP64: at n = 32768
// that is a 4 GiB copy and minutes of CPU time. Here two kernels compute, per matrix, with
// S the symmetric matrix the lower triangle of A defines and R = tril(L) tril(L)^T - S:
//
//   residual_tile_kernel  one CTA per 64 x 64 tile (I, J), I >= J, of the lower triangle:
//                         P = sum_k L[r][k] L[c][k] over k < 64 (J + 1) in FP64 (the product
//                         of two FP32 values is exact in FP64, so only the FP64 additions
//                         round), R = P - S on the tile; ||R||_F^2 and ||S||_F^2 (entries
//                         off the diagonal count twice, once for each triangle), and the
//                         row sums of |R| and |S| (each lower entry adds to its row and, off
//                         the diagonal, to the row of its mirror) by FP64 atomics.
//   scan_kernel           one warp per row of L: non-finite entries, non-zero entries above
//                         the diagonal, diagonal entries that are not > 0, and the maximum
//                         row sums (atomicMax on the bit patterns, which order like the
//                         values for non-negative doubles; a NaN sorts above +inf).
//
// Tiles are staged in shared memory as FP64, row-major with one double of padding: the
// loads (a warp reads 32 consecutive k of one row, 128 bytes) and the stores are
// conflict-free, and so are the inner-loop reads, where thread (tx, ty) owns rows
// ty + 16 i and columns tx + 16 j (i, j < 4): the 16 column rows a warp reads lie 33
// doubles apart, i.e. in distinct bank pairs.
#include "chol_common.cuh"

namespace chol {
namespace {

constexpr int kVT = 64;        // tile edge
constexpr int kVK = 32;        // k chunk
constexpr int kVLD = kVK + 1;  // padded row length (doubles)
constexpr int kOut = 8;        // doubles of output per matrix

__device__ __forceinline__ void tile_of(int64_t t, int64_t& I, int64_t& J) {
  // t = I (I + 1) / 2 + J, 0 <= J <= I
  int64_t i = int64_t((sqrt(8.0 * double(t) + 1.0) - 1.0) * 0.5);
  while (i * (i + 1) / 2 > t) --i;
  while ((i + 1) * (i + 2) / 2 <= t) ++i;
  I = i;
  J = t - i * (i + 1) / 2;
}

__device__ __forceinline__ double warp_sum(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__global__ void __launch_bounds__(256) residual_tile_kernel(const float* __restrict__ A,
                                                            const float* __restrict__ L,
                                                            int64_t batch, int64_t n,
                                                            int64_t tiles, double* out,
                                                            double* rowR, double* rowS) {
  __shared__ double As[kVT * kVLD];
  __shared__ double Bs[kVT * kVLD];
  __shared__ double racc[2][kVT];  // |R| row sums: rows of block I, rows of block J
  __shared__ double sacc[2][kVT];  // |S| likewise
  __shared__ double red[2][8];

  const int tid = threadIdx.x;
  const int tx = tid & 15, ty = tid >> 4;
  const int64_t total = batch * tiles;
  for (int64_t g = blockIdx.x; g < total; g += gridDim.x) {
    const int64_t m = g / tiles;
    int64_t I, J;
    tile_of(g - m * tiles, I, J);
    const float* Lm = L + m * n * n;
    const float* Am = A + m * n * n;
    const int64_t r0 = I * kVT, c0 = J * kVT;
    const int64_t kend = min(c0 + kVT, n);

    double acc[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[i][j] = 0.0;
    if (tid < kVT) {
      racc[0][tid] = racc[1][tid] = 0.0;
      sacc[0][tid] = sacc[1][tid] = 0.0;
    }

    for (int64_t k0 = 0; k0 < kend; k0 += kVK) {
      __syncthreads();  // previous chunk's reads done
#pragma unroll
      for (int e = 0; e < (kVT * kVK) / 256; ++e) {
        const int idx = tid + 256 * e;
        const int rr = idx / kVK, kk = idx % kVK;
        const int64_t k = k0 + kk;
        const int64_t ra = r0 + rr, rb = c0 + rr;
        float va = 0.f, vb = 0.f;
        if (ra < n && k < n && k <= ra) va = Lm[ra * n + k];
        if (rb < n && k < n && k <= rb) vb = Lm[rb * n + k];
        As[rr * kVLD + kk] = double(va);
        Bs[rr * kVLD + kk] = double(vb);
      }
      __syncthreads();
#pragma unroll 4
      for (int kk = 0; kk < kVK; ++kk) {
        double a[4], b[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) a[i] = As[(ty + 16 * i) * kVLD + kk];
#pragma unroll
        for (int j = 0; j < 4; ++j) b[j] = Bs[(tx + 16 * j) * kVLD + kk];
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) acc[i][j] = fma(a[i], b[j], acc[i][j]);
      }
    }

    // epilogue: R = P - S on the tile's lower entries
    double r2 = 0.0, s2 = 0.0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int lr = ty + 16 * i;
      const int64_t r = r0 + lr;
      double rrow = 0.0, srow = 0.0;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int lc = tx + 16 * j;
        const int64_t c = c0 + lc;
        if (r < n && c < n && c <= r) {
          const double s = double(Am[r * n + c]);
          const double d = acc[i][j] - s;
          const double w = (c == r) ? 1.0 : 2.0;
          r2 += w * d * d;
          s2 += w * s * s;
          rrow += fabs(d);
          srow += fabs(s);
          if (c != r) {
            atomicAdd(&racc[1][lc], fabs(d));
            atomicAdd(&sacc[1][lc], fabs(s));
          }
        }
      }
      if (rrow != 0.0) atomicAdd(&racc[0][lr], rrow);
      if (srow != 0.0) atomicAdd(&sacc[0][lr], srow);
    }
    r2 = warp_sum(r2);
    s2 = warp_sum(s2);
    if ((tid & 31) == 0) {
      red[0][tid >> 5] = r2;
      red[1][tid >> 5] = s2;
    }
    __syncthreads();
    if (tid < 32) {
      double a = tid < 8 ? red[0][tid] : 0.0;
      double b = tid < 8 ? red[1][tid] : 0.0;
      a = warp_sum(a);
      b = warp_sum(b);
      if (tid == 0) {
        atomicAdd(&out[m * kOut + 0], a);
        atomicAdd(&out[m * kOut + 1], b);
      }
    }
    if (tid < kVT) {
      if (r0 + tid < n) {
        atomicAdd(&rowR[m * n + r0 + tid], racc[0][tid]);
        atomicAdd(&rowS[m * n + r0 + tid], sacc[0][tid]);
      }
      if (c0 + tid < n && (racc[1][tid] != 0.0 || sacc[1][tid] != 0.0)) {
        atomicAdd(&rowR[m * n + c0 + tid], racc[1][tid]);
        atomicAdd(&rowS[m * n + c0 + tid], sacc[1][tid]);
      }
    }
  }
}

__device__ __forceinline__ void atomic_max_nonneg(double* p, double v) {
  atomicMax(reinterpret_cast<unsigned long long*>(p),
            static_cast<unsigned long long>(__double_as_longlong(v)));
}

__global__ void __launch_bounds__(256) scan_kernel(const float* __restrict__ L, int64_t batch,
                                                   int64_t n, double* out,
                                                   const double* __restrict__ rowR,
                                                   const double* __restrict__ rowS) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = int64_t(gridDim.x) * (blockDim.x >> 5);
  for (int64_t row = int64_t(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
       row < batch * n; row += warps) {
    const int64_t m = row / n, i = row - m * n;
    const float* Lr = L + row * n;
    unsigned nonfinite = 0, upper = 0, diag = 0;
    for (int64_t j = lane; j < n; j += 32) {
      const float v = Lr[j];
      nonfinite += !isfinite(v);
      upper += (j > i) && (v != 0.f);
      diag += (j == i) && !(v > 0.f);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      nonfinite += __shfl_xor_sync(0xffffffffu, nonfinite, o);
      upper += __shfl_xor_sync(0xffffffffu, upper, o);
      diag += __shfl_xor_sync(0xffffffffu, diag, o);
    }
    if (lane == 0) {
      if (nonfinite) atomicAdd(&out[m * kOut + 4], double(nonfinite));
      if (upper) atomicAdd(&out[m * kOut + 5], double(upper));
      if (diag) atomicAdd(&out[m * kOut + 6], double(diag));
      atomic_max_nonneg(&out[m * kOut + 2], rowR[row]);
      atomic_max_nonneg(&out[m * kOut + 3], rowS[row]);
    }
  }
}

}  // namespace
}  // namespace chol

using namespace chol;

extern "C" size_t chol_validate_work_bytes(int64_t batch, int64_t n) {
  if (batch <= 0 || n <= 0) return 0;
  return size_t(2) * size_t(batch) * size_t(n) * sizeof(double);
}

extern "C" int chol_validate_f32(const float* A, const float* L, int64_t batch, int64_t n,
                                 double* out, void* work, void* queue) {
  if (batch < 0 || n < 0) return CHOL_ERR_INVALID_ARG;
  if (batch == 0 || n == 0) return CHOL_OK;
  if (A == nullptr || L == nullptr || out == nullptr || work == nullptr)
    return CHOL_ERR_INVALID_ARG;
  if ((reinterpret_cast<uintptr_t>(out) & 7) || (reinterpret_cast<uintptr_t>(work) & 7))
    return CHOL_ERR_INVALID_ARG;
  if (n > (int64_t(1) << 20) || batch > (int64_t(1) << 40) / (n * n))
    return CHOL_ERR_UNSUPPORTED;
  cudaStream_t q = static_cast<cudaStream_t>(queue);
  double* rowR = static_cast<double*>(work);
  double* rowS = rowR + batch * n;
  if (cudaMemsetAsync(out, 0, size_t(batch) * kOut * sizeof(double), q) != cudaSuccess ||
      cudaMemsetAsync(work, 0, chol_validate_work_bytes(batch, n), q) != cudaSuccess)
    return CHOL_ERR_LAUNCH;
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) != cudaSuccess) return CHOL_ERR_DEVICE;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t nt = (n + kVT - 1) / kVT;
  const int64_t tiles = nt * (nt + 1) / 2;
  const int64_t grid1 = std::min<int64_t>(batch * tiles, int64_t(sms) * 64);
  // plain stream-ordered launches (no programmatic early start); launch_pdl also tells the
  // small-call overlap tracker that another kernel now sits on the queue
  int st = status_from(launch_pdl(residual_tile_kernel, dim3(unsigned(grid1)), dim3(256), 0, q,
                                  false, A, L, batch, n, tiles, out, rowR, rowS));
  if (st) return st;
  const int64_t grid2 = std::min<int64_t>((batch * n + 7) / 8, int64_t(sms) * 32);
  return status_from(launch_pdl(scan_kernel, dim3(unsigned(grid2)), dim3(256), 0, q, false, L,
                                batch, n, out, static_cast<const double*>(rowR),
                                static_cast<const double*>(rowS)));
}
