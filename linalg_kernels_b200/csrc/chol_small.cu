// chol_small.cu — batched Cholesky for n <= 64: one matrix per warp (n > 16) or per
// lane group (n <= 16), whole factorisation in registers, HBM-bound.
//
// Replaces the reference's per-shape small kernels for b=4096 n=32 and b=1024 n=64
// (cutlass_subwarp_left_32_kernel, cholesky/cholesky.py:149-228; right_looking_64_kernel,
// cholesky/cholesky.py:294-387) with one template over the padded size NP.
//
// Data movement per matrix: the lower triangle of A is read with coalesced 128-bit loads
// (chunks that lie wholly above the diagonal are not fetched), staged through shared
// memory (row stride NP+4: conflict-free 128-bit row reads), factored in registers by
// warp_potrf_rows<NP>, staged back and written as full rows (upper triangle as exact
// zeros) with coalesced 128-bit streaming stores.
#include "chol_warp.cuh"

namespace chol {

namespace {

constexpr int kSmallWarps = 4;

template <int NP>
constexpr size_t small_smem_bytes() {
  return size_t(kSmallWarps) * WarpShape<NP>::MPW * (size_t(NP) * (NP + 4) + 2 * NP) * 4;
}

// FULL: n == NP and 16-byte aligned rows (vector path). Otherwise scalar loads with
// identity padding of rows/columns n..NP-1.
template <int NP, bool FULL>
__global__ void __launch_bounds__(kSmallWarps * 32, NP <= 32 ? 8 : 1)
    small_potrf_kernel(const float* __restrict__ A, float* __restrict__ L, int64_t batch, int n,
                       int* __restrict__ info) {
  constexpr int LPM = WarpShape<NP>::LPM;
  constexpr int R = WarpShape<NP>::R;
  constexpr int MPW = WarpShape<NP>::MPW;
  constexpr int LDS = NP + 4;
  constexpr int TILE = NP * LDS;
  extern __shared__ float4 smem_raw[];
  float* smem = reinterpret_cast<float*>(smem_raw);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int grp = lane / LPM;
  const int gl = lane % LPM;
  float* stage = smem + size_t(warp) * MPW * TILE;
  float* col = smem + size_t(kSmallWarps) * MPW * TILE + size_t(warp * MPW + grp) * 2 * NP;
  const int64_t mbase = (int64_t(blockIdx.x) * kSmallWarps + warp) * MPW;
  if (FULL) n = NP;

  griddep_wait();
  griddep_launch();

  // ---- load: lower triangle, coalesced, into this warp's staging tiles ----
#pragma unroll 1
  for (int mm = 0; mm < MPW; ++mm) {
    const int64_t m = mbase + mm;
    float* st = stage + mm * TILE;
    int rpad = 0;
    if (m < batch) {
      const float* src = A + m * int64_t(n) * n;
      if (FULL) {
        // 16-byte chunks that hold at least one lower-triangle element, all in flight
        constexpr int C4 = NP / 4;
#pragma unroll
        for (int idx = lane; idx < NP * C4; idx += 32) {
          const int r = idx / C4, c4 = idx % C4;
          if (c4 * 4 <= r) cp_async16(st + r * LDS + c4 * 4, src + r * NP + c4 * 4);
        }
        rpad = NP;
      } else {
        const int nn = n * n;
        for (int idx = lane; idx < nn; idx += 32) {
          const int r = idx / n, c = idx - r * n;
          if (c <= r) cp_async4(st + r * LDS + c, src + idx);
        }
        rpad = n;
      }
    }
    // identity padding: rows rpad..NP-1 (all rows when the matrix is past the batch)
    for (int idx = lane; idx < (NP - rpad) * NP; idx += 32) {
      const int r = rpad + idx / NP, c = idx % NP;
      st[r * LDS + c] = (r == c) ? 1.f : 0.f;
    }
  }
  cp_async_wait_all();
  __syncwarp();

  // ---- rows to registers (column pairs) ----
  float2 a[R][NP / 2];
  const float* mst = stage + grp * TILE;
#pragma unroll
  for (int s = 0; s < R; ++s) {
    const float* rp = mst + (s * LPM + gl) * LDS;
#pragma unroll
    for (int q = 0; q < (s + 1) * LPM / 4; ++q) {
      const float4 v = *reinterpret_cast<const float4*>(rp + 4 * q);
      a[s][2 * q] = make_float2(v.x, v.y);
      a[s][2 * q + 1] = make_float2(v.z, v.w);
    }
  }

  warp_potrf_rows<NP>(a, col, gl);
  __syncwarp();

  // ---- registers to staging, strict upper part as exact zeros ----
  // A non-positive (or NaN) pivot in column j makes L[j][j] NaN or non-positive and every
  // later pivot NaN, so the first row whose diagonal is not > 0 is LAPACK's info - 1.
  bool bad[R];
#pragma unroll
  for (int s = 0; s < R; ++s) {
    const int i = s * LPM + gl;
    float* rp = stage + grp * TILE + i * LDS;
    bad[s] = false;
#pragma unroll
    for (int q = 0; q < NP / 4; ++q) {
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (4 * q < (s + 1) * LPM) {
        const float2 lo = a[s][2 * q], hi = a[s][2 * q + 1];
        v.x = (4 * q + 0 <= i) ? lo.x : 0.f;
        v.y = (4 * q + 1 <= i) ? lo.y : 0.f;
        v.z = (4 * q + 2 <= i) ? hi.x : 0.f;
        v.w = (4 * q + 3 <= i) ? hi.y : 0.f;
        if (4 * q <= i && i < 4 * q + 4) {
          const float dg = (i & 2) ? ((i & 1) ? hi.y : hi.x) : ((i & 1) ? lo.y : lo.x);
          bad[s] = !(dg > 0.f);
        }
      }
      *reinterpret_cast<float4*>(rp + 4 * q) = v;
    }
  }
  int fail = 0;
#pragma unroll
  for (int s = R - 1; s >= 0; --s) {
    const unsigned bits = (__ballot_sync(0xffffffffu, bad[s]) >> (grp * LPM)) &
                          (LPM == 32 ? 0xffffffffu : ((1u << LPM) - 1u));
    if (bits) fail = s * LPM + __ffs(bits);  // 1-based row of the first failure in slot s
  }
  __syncwarp();

  // ---- store: full rows. Vector path: one bulk async copy per row, issued by the lane
  // that holds the row; scalar path: coalesced 4-byte stores. ----
  if (FULL) {
    fence_proxy_async_smem();
    __syncwarp();
#pragma unroll 1
    for (int mm = 0; mm < MPW; ++mm) {
      const int64_t m = mbase + mm;
      if (m >= batch) break;
      const float* st = stage + mm * TILE;
      float* dst = L + m * int64_t(NP) * NP;
      for (int r = lane; r < NP; r += 32) bulk_store(dst + r * NP, st + r * LDS, NP * 4);
    }
    bulk_store_wait_read();
  } else {
#pragma unroll 1
    for (int mm = 0; mm < MPW; ++mm) {
      const int64_t m = mbase + mm;
      if (m >= batch) break;
      const float* st = stage + mm * TILE;
      float* dst = L + m * int64_t(n) * n;
      const int nn = n * n;
      for (int idx = lane; idx < nn; idx += 32) {
        const int r = idx / n, c = idx - r * n;
        __stcs(dst + idx, st[r * LDS + c]);
      }
    }
  }
  if (info != nullptr && gl == 0) {
    const int64_t m = mbase + grp;
    if (m < batch) info[m] = (fail > n) ? 0 : fail;
  }
}

template <int NP>
int launch_np(const float* A, float* L, int64_t batch, int n, int* info, cudaStream_t q) {
  constexpr int MPC = kSmallWarps * WarpShape<NP>::MPW;
  const int64_t blocks = (batch + MPC - 1) / MPC;
  if (blocks > 0x7fffffffLL) return CHOL_ERR_UNSUPPORTED;
  const size_t smem = small_smem_bytes<NP>();
  const bool full = (n == NP) && ((reinterpret_cast<uintptr_t>(A) & 15) == 0) &&
                    ((reinterpret_cast<uintptr_t>(L) & 15) == 0);
  cudaError_t e;
  if (full)
    e = launch_pdl(small_potrf_kernel<NP, true>, dim3(unsigned(blocks)), dim3(kSmallWarps * 32),
                   smem, q, true, A, L, batch, n, info);
  else
    e = launch_pdl(small_potrf_kernel<NP, false>, dim3(unsigned(blocks)),
                   dim3(kSmallWarps * 32), smem, q, true, A, L, batch, n, info);
  return status_from(e);
}

template <int NP>
cudaError_t set_smem_np() {
  cudaError_t e = cudaFuncSetAttribute(small_potrf_kernel<NP, true>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       int(small_smem_bytes<NP>()));
  if (e != cudaSuccess) return e;
  return cudaFuncSetAttribute(small_potrf_kernel<NP, false>,
                              cudaFuncAttributeMaxDynamicSharedMemorySize,
                              int(small_smem_bytes<NP>()));
}

}  // namespace

cudaError_t prepare_small() {
  cudaError_t e;
  if ((e = set_smem_np<4>()) != cudaSuccess) return e;
  if ((e = set_smem_np<8>()) != cudaSuccess) return e;
  if ((e = set_smem_np<16>()) != cudaSuccess) return e;
  if ((e = set_smem_np<32>()) != cudaSuccess) return e;
  return set_smem_np<64>();
}

int launch_small(const float* A, float* L, int64_t batch, int n, int* info, cudaStream_t q) {
  if (n <= 4) return launch_np<4>(A, L, batch, n, info, q);
  if (n <= 8) return launch_np<8>(A, L, batch, n, info, q);
  if (n <= 16) return launch_np<16>(A, L, batch, n, info, q);
  if (n <= 32) return launch_np<32>(A, L, batch, n, info, q);
  if (n <= 64) return launch_np<64>(A, L, batch, n, info, q);
  return CHOL_ERR_UNSUPPORTED;
}

}  // namespace chol
