// chol_panel.cu — one fused kernel per 64-wide step of the blocked Cholesky.
//
// For block column k of an outer panel that starts at column K0, every CTA owns 64 rows
// below the diagonal block (rows R = k+kb+64*i ...) and computes, with no waits on other
// CTAs:
//   1. the left-looking update of [diagonal rows; own rows] x 64 columns,
//        C = A[rows, k:k+kb] - A[rows, K0:k] A[k:k+kb, K0:k]^T
//      as ONE tcgen05 MMA tile M128 x N64 (rows 0..63 = the diagonal block, rows 64..127 =
//      its own rows; B = the diagonal rows, i.e. the first half of the A tile), 3xTF32;
//   2. the Cholesky factor of the 64 x 64 diagonal block (redundantly in every CTA, one
//      warp, registers) and its inverse T (column-parallel forward substitution);
//   3. the panel solve of its own rows, X = C_own T^T (FP32 FMA), written to L.
// The diagonal block itself is written by the LAST CTA of the matrix to finish (a per-matrix
// arrival counter in the workspace): every CTA has read the block's pre-update values by
// then, and the last CTA computed the same factor, so nobody waits on anybody.
//
// This replaces three launches per step (GEMM, diagonal factor, GEMM solve) of the
// reference-style schedule (factor128_kernel + gemm_inner/gemm_apply,
// cholesky/cholesky.py:5440-5690) with one, and keeps T in shared memory.
#include "chol_tc_ptx.cuh"
#include "chol_warp.cuh"

namespace chol {
namespace {

using namespace tcx;

constexpr int kPS_Threads = 192;  // producer, MMA, 4 converter/epilogue warps
constexpr int kPS_Stages = 3;
constexpr int kPS_ABytes = 128 * kBK * 4;           // 16 KB: 128 rows x 32 floats
constexpr int kPS_StageBytes = 2 * kPS_ABytes;      // A and its lo twin
constexpr int kPS_SLD = 68;                         // factor/solve tile stride (floats)
constexpr int kPS_TileBytes = 128 * kPS_SLD * 4;    // C tile after the update
constexpr int kPS_TBytes = 64 * kPS_SLD * 4;        // T
constexpr int kPS_Work = (kPS_Stages * kPS_StageBytes > kPS_TileBytes + kPS_TBytes)
                             ? kPS_Stages * kPS_StageBytes
                             : kPS_TileBytes + kPS_TBytes;
constexpr size_t kPS_Smem = size_t(kPS_Work) + 1024 + 1024;

struct PanelArgs {
  float* L;
  int64_t n, ld, mstride, batch;  // n: rows of the panel (row limit), ld: row stride
  int64_t k, kb, K0;
  int* info;
  unsigned int* counters;  // one per matrix, zero between launches
  int* status;
  float* tout;             // optional: inv(L_kk) (+ m * tstride, leading dimension tld)
  int64_t tstride, tld;
};

__device__ __forceinline__ void named_sync_128() {
  asm volatile("bar.sync 1, 128;" ::: "memory");
}

__global__ void __launch_bounds__(kPS_Threads, 2)
    panel_step_kernel(const __grid_constant__ CUtensorMap tmL, PanelArgs a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  griddep_wait();

  const int64_t mi = int64_t(blockIdx.y) + int64_t(blockIdx.z) * 65535;
  if (mi >= a.batch) return;
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  auto stA = [&](int s) { return reinterpret_cast<float*>(smem + size_t(s) * kPS_StageBytes); };
  auto stAlo = [&](int s) { return stA(s) + kPS_ABytes / 4; };
  float* S = reinterpret_cast<float*>(smem);                   // reused after the mainloop
  float* T = reinterpret_cast<float*>(smem + kPS_TileBytes);
  uint8_t* tail = smem + kPS_Work;
  uint64_t* full = reinterpret_cast<uint64_t*>(tail);
  uint64_t* conv = full + kPS_Stages;
  uint64_t* empty = conv + kPS_Stages;
  uint64_t* accum = empty + kPS_Stages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accum + 1);
  float* colbuf = reinterpret_cast<float*>(tail + 256);        // 2*64 floats, 16B aligned
  float* rdiag = colbuf + 128;                                 // 64 floats
  int* flags = reinterpret_cast<int*>(rdiag + 64);             // [0] fail, [1] last CTA

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t k = a.k, kb = a.kb;
  const int64_t own0 = k + kb + int64_t(blockIdx.x) * 64;  // first own row
  const int num_k = int((k - a.K0 + kBK - 1) / kBK);
  float* Lm = a.L + mi * a.mstride;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kPS_Stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&conv[s], 4);
      mbar_init(&empty[s], 1);
    }
    mbar_init(accum, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    if (num_k > 0) prefetch_map(&tmL);
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(64u)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  griddep_launch();
  const uint32_t tmem = *tmem_slot;
  bool ok = true;

  if (warp == 0) {
    if (lane == 0) {
      for (int kt = 0; kt < num_k; ++kt) {
        const int s = kt % kPS_Stages;
        const uint32_t ph = uint32_t(kt / kPS_Stages) & 1u;
        if (kt >= kPS_Stages && !mbar_wait(&empty[s], ph ^ 1u, a.status)) break;
        const int x = int(a.K0) + kt * kBK;
        mbar_expect_tx(&full[s], kPS_ABytes);
        tma_load_3d(stA(s), &tmL, x, int(k), int(mi), &full[s]);                   // rows 0..63
        tma_load_3d(stA(s) + 64 * kBK, &tmL, x, int(own0), int(mi), &full[s]);     // rows 64..127
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = tf32_idesc<128, 64>();
      for (int kt = 0; kt < num_k; ++kt) {
        const int s = kt % kPS_Stages;
        const uint32_t ph = uint32_t(kt / kPS_Stages) & 1u;
        if (!mbar_wait(&conv[s], ph, a.status)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint64_t da = sw128_desc(stA(s)), dal = sw128_desc(stAlo(s));
#pragma unroll
        for (int kk = 0; kk < kBK / 8; ++kk) {
          const uint64_t adv = uint64_t(kk * 32 / 16);
          // B = rows 0..63 of the same tile (the diagonal block's rows)
          mma_tf32(tmem, da + adv, da + adv, idesc, (kt | kk) ? 1u : 0u);
          mma_tf32(tmem, da + adv, dal + adv, idesc, 1u);
          mma_tf32(tmem, dal + adv, da + adv, idesc, 1u);
        }
        mma_commit(&empty[s]);
      }
      if (ok) mma_commit(accum);  // with num_k == 0 this arrives at once
    }
  } else {
    const int et = threadIdx.x - 64;  // 0..127
    for (int kt = 0; kt < num_k; ++kt) {
      const int s = kt % kPS_Stages;
      const uint32_t ph = uint32_t(kt / kPS_Stages) & 1u;
      if (!mbar_wait(&full[s], ph, a.status)) {
        ok = false;
        break;
      }
      float4* x = reinterpret_cast<float4*>(stA(s));
      float4* xl = reinterpret_cast<float4*>(stAlo(s));
#pragma unroll
      for (int i = et; i < kPS_ABytes / 16; i += 128) split4<false>(x + i, xl + i);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&conv[s]);
    }
    if (ok && !mbar_wait(accum, 0, a.status)) ok = false;
    tc_fence_after();

    // ---- C = A - update, into S (row r: r < 64 diagonal row k+r, else own row) ----
    const int q = warp & 3;
    const int r = q * 32 + lane;
    const int64_t grow = (r < 64) ? k + r : own0 + (r - 64);
    const bool valid = (r < 64) ? (r < kb) : (grow < a.n);
    const float* arow = Lm + grow * a.ld + k;
#pragma unroll
    for (int cc = 0; cc < 2; ++cc) {
      float v[32];
      if (num_k > 0) {
        tmem_ld32(tmem + (uint32_t(q * 32) << 16) + uint32_t(cc * 32), v);
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = 0.f;
      }
      float* srow = S + r * kPS_SLD + cc * 32;
#pragma unroll
      for (int j = 0; j < 32; j += 4) {
        float4 c4 = make_float4(0.f, 0.f, 0.f, 0.f);
        const int c = cc * 32 + j;
        if (valid) {
          if (c + 3 < kb && ((reinterpret_cast<uintptr_t>(arow + c) & 15) == 0)) {
            c4 = *reinterpret_cast<const float4*>(arow + c);
          } else {
            if (c + 0 < kb) c4.x = arow[c + 0];
            if (c + 1 < kb) c4.y = arow[c + 1];
            if (c + 2 < kb) c4.z = arow[c + 2];
            if (c + 3 < kb) c4.w = arow[c + 3];
          }
        }
        float4 o = make_float4(c4.x - v[j], c4.y - v[j + 1], c4.z - v[j + 2], c4.w - v[j + 3]);
        if (r < 64) {  // diagonal block: identity outside kb, lower part only
          const float e[4] = {o.x, o.y, o.z, o.w};
          float f[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const int cu = c + u;
            f[u] = (r < kb && cu < kb) ? (cu <= r ? e[u] : 0.f) : (cu == r ? 1.f : 0.f);
          }
          o = make_float4(f[0], f[1], f[2], f[3]);
        } else if (!valid) {
          o = make_float4(0.f, 0.f, 0.f, 0.f);
        }
        *reinterpret_cast<float4*>(srow + j) = o;
      }
    }
    // every read of this matrix's diagonal block in L is done: count this CTA in
    named_sync_128();
    if (et == 0) {
      __threadfence();
      const unsigned prev = atomicAdd(&a.counters[mi], 1u);
      const bool last = (prev + 1 == gridDim.x);
      if (last) a.counters[mi] = 0u;  // ready for the next launch
      __threadfence();
      flags[1] = last ? 1 : 0;
    }

    // ---- factor the diagonal block (one warp, registers) ----
    if (warp == 2) {
      uint64_t ar[2][32];
#pragma unroll
      for (int s = 0; s < 2; ++s) {
        const float* rp = S + (s * 32 + lane) * kPS_SLD;
#pragma unroll
        for (int qq = 0; qq < (s + 1) * 8; ++qq) {
          const ulonglong2 v = *reinterpret_cast<const ulonglong2*>(rp + 4 * qq);
          ar[s][2 * qq] = v.x;
          ar[s][2 * qq + 1] = v.y;
        }
      }
      warp_potrf_rows<64>(ar, colbuf, lane);
      __syncwarp();
#pragma unroll
      for (int s = 0; s < 2; ++s) {
        const int i = s * 32 + lane;
        float* rp = S + i * kPS_SLD;
#pragma unroll
        for (int qq = 0; qq < 16; ++qq) {
          float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
          if (4 * qq < (s + 1) * 32) {
            v.x = (4 * qq + 0 <= i) ? lo_of(ar[s][2 * qq]) : 0.f;
            v.y = (4 * qq + 1 <= i) ? hi_of(ar[s][2 * qq]) : 0.f;
            v.z = (4 * qq + 2 <= i) ? lo_of(ar[s][2 * qq + 1]) : 0.f;
            v.w = (4 * qq + 3 <= i) ? hi_of(ar[s][2 * qq + 1]) : 0.f;
          }
          *reinterpret_cast<float4*>(rp + 4 * qq) = v;
        }
      }
      __syncwarp();
      const float d0 = S[lane * kPS_SLD + lane];
      const float d1 = S[(lane + 32) * kPS_SLD + lane + 32];
      rdiag[lane] = __frcp_rn(d0);
      rdiag[lane + 32] = __frcp_rn(d1);
      const unsigned b0 = __ballot_sync(0xffffffffu, !(d0 > 0.f));
      const unsigned b1 = __ballot_sync(0xffffffffu, !(d1 > 0.f));
      if (lane == 0) flags[0] = b0 ? __ffs(b0) : (b1 ? 32 + __ffs(b1) : 0);
    }
    named_sync_128();

    // ---- T = inv(L_kk): thread c (< 64) computes column c ----
    if (et < 64) {
      const int c = et;
      float t[64];
#pragma unroll
      for (int i = 0; i < 64; ++i) {
        const float* rp = S + i * kPS_SLD;
        float2 acc = make_float2(0.f, 0.f);
#pragma unroll
        for (int qq = 0; qq < i / 4; ++qq) {
          const float4 v = *reinterpret_cast<const float4*>(rp + 4 * qq);
          acc = ffma2(make_float2(v.x, v.y), make_float2(t[4 * qq], t[4 * qq + 1]), acc);
          acc = ffma2(make_float2(v.z, v.w), make_float2(t[4 * qq + 2], t[4 * qq + 3]), acc);
        }
        float sum = acc.x + acc.y;
#pragma unroll
        for (int mm = (i / 4) * 4; mm < i; ++mm) sum = fmaf(rp[mm], t[mm], sum);
        const float ri = rdiag[i];
        t[i] = (i == c) ? ri : ((i < c) ? 0.f : -ri * sum);
      }
#pragma unroll
      for (int i = 0; i < 64; ++i) T[i * kPS_SLD + c] = t[i];  // T stored row-major
    }
    named_sync_128();

    // ---- own rows: X = C_own T^T, x[r][c] = sum_i C[r][i] T[c][i] (row c of T) ----
    // thread et: own row rr = et >> 1, columns c in [32h, 32h+32) with h = et & 1.
    {
      const int rr = et >> 1, h = et & 1;
      const int64_t orow = own0 + rr;
      if (orow < a.n && kb > 0) {
        const float* crow = S + (64 + rr) * kPS_SLD;
        float cr[64];
#pragma unroll
        for (int qq = 0; qq < 16; ++qq) {
          const float4 v = *reinterpret_cast<const float4*>(crow + 4 * qq);
          cr[4 * qq] = v.x;
          cr[4 * qq + 1] = v.y;
          cr[4 * qq + 2] = v.z;
          cr[4 * qq + 3] = v.w;
        }
        float* dst = Lm + orow * a.ld + k + h * 32;
#pragma unroll 1
        for (int jc = 0; jc < 32; jc += 4) {
          float xo[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float* tc = T + (h * 32 + jc + j) * kPS_SLD;
            float2 acc = make_float2(0.f, 0.f);
#pragma unroll
            for (int qq = 0; qq < 16; ++qq) {
              const float4 v = *reinterpret_cast<const float4*>(tc + 4 * qq);
              acc = ffma2(make_float2(cr[4 * qq], cr[4 * qq + 1]), make_float2(v.x, v.y), acc);
              acc = ffma2(make_float2(cr[4 * qq + 2], cr[4 * qq + 3]), make_float2(v.z, v.w), acc);
            }
            xo[j] = acc.x + acc.y;
          }
          const int c0 = h * 32 + jc;
          if (c0 + 3 < kb && ((reinterpret_cast<uintptr_t>(dst + jc) & 15) == 0)) {
            *reinterpret_cast<float4*>(dst + jc) = make_float4(xo[0], xo[1], xo[2], xo[3]);
          } else {
#pragma unroll
            for (int u = 0; u < 4; ++u)
              if (c0 + u < kb) dst[jc + u] = xo[u];
          }
        }
      }
    }

    // ---- the last CTA of the matrix writes the diagonal block, its inverse and info ----
    if (flags[1]) {
      for (int idx = et; idx < kb * kb; idx += 128) {
        const int i = idx / int(kb), c = idx - i * int(kb);
        Lm[(k + i) * a.ld + k + c] = S[i * kPS_SLD + c];
      }
      if (a.tout != nullptr) {
        float* tm = a.tout + mi * a.tstride;
        for (int idx = et; idx < 64 * 16; idx += 128) {
          const int i = idx >> 4, c = (idx & 15) * 4;
          *reinterpret_cast<float4*>(tm + i * a.tld + c) =
              *reinterpret_cast<const float4*>(T + i * kPS_SLD + c);
        }
      }
      if (et == 0 && a.info != nullptr) {
        const int f = flags[0] > kb ? 0 : flags[0];
        if (k == 0)
          a.info[mi] = f ? int(k) + f : 0;
        else if (f && a.info[mi] == 0)
          a.info[mi] = int(k) + f;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(64u)
                 : "memory");
  }
}

PFN_cuTensorMapEncodeTiled_v12000 g_enc = nullptr;

}  // namespace

cudaError_t prepare_panel() {
  return cudaFuncSetAttribute(panel_step_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              int(kPS_Smem));
}

// Tensor map over the whole of L for this kernel (64-row boxes).
bool panel_make_map(void* map128, const float* L, int64_t n, int64_t batch) {
  if (g_enc == nullptr) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) !=
            cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return false;
    g_enc = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  }
  if ((reinterpret_cast<uintptr_t>(L) & 15) || n % 4) return false;
  cuuint64_t dims[3] = {cuuint64_t(n), cuuint64_t(n), cuuint64_t(batch)};
  cuuint64_t strides[2] = {cuuint64_t(n) * 4, cuuint64_t(n) * cuuint64_t(n) * 4};
  cuuint32_t box[3] = {cuuint32_t(kBK), 64, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  return g_enc(reinterpret_cast<CUtensorMap*>(map128), CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3,
               const_cast<float*>(L), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
               CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int launch_panel_step(const void* map128, float* L, int64_t n, int64_t batch, int64_t k,
                      int64_t kb, int64_t K0, int* info, unsigned int* counters, cudaStream_t q,
                      int64_t row_end, float* tout, int64_t tstride, int64_t tld) {
  if (row_end <= 0 || row_end > n) row_end = n;
  if (tout != nullptr && (tld % 4 || (reinterpret_cast<uintptr_t>(tout) & 15)))
    return CHOL_ERR_UNSUPPORTED;
  PanelArgs a{};
  a.L = L;
  a.n = row_end;
  a.ld = n;
  a.tout = tout;
  a.tstride = tstride;
  a.tld = tld;
  a.mstride = n * n;
  a.batch = batch;
  a.k = k;
  a.kb = kb;
  a.K0 = K0;
  a.info = info;
  a.counters = counters;
  a.status = device_status_ptr();
  if (a.status == nullptr) return CHOL_ERR_DEVICE;
  const int64_t below = row_end - k - kb;
  const int64_t tiles = below > 0 ? (below + 63) / 64 : 1;
  const int64_t by = batch < 65535 ? batch : 65535;
  const int64_t bz = (batch + 65534) / 65535;
  const dim3 grid = dim3(unsigned(tiles), unsigned(by), unsigned(bz));
  return status_from(launch_pdl(panel_step_kernel, grid, dim3(kPS_Threads), kPS_Smem, q, true,
                                *reinterpret_cast<const CUtensorMap*>(map128), a));
}

}  // namespace chol
