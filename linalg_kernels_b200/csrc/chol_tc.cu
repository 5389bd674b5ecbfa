// chol_tc.cu — tensor-core (tcgen05 / TMEM / TMA) NT-GEMM with a 3xTF32 split, the
// trailing-update and panel-solve engine of the blocked path.
//
//   C[r][c] = alpha * sum_q P[r][q] Q[c][q] + beta * C[r][c]     (lower tiles optional)
//
// FP32 accuracy from TF32 tensor cores: every operand x is split into hi = x with its low
// 13 mantissa bits cleared (exactly representable in TF32) and lo = x - hi (exact in
// FP32; its TF32 truncation loses < 2^-21 |x|), and the product is accumulated as
//   P_hi Q_hi + P_hi Q_lo + P_lo Q_hi            (the lo*lo term, < 2^-22 |P||Q|, dropped)
// in one FP32 TMEM accumulator. Plain TF32 (the reference's cuBLAS FAST_TF32 GEMMs,
// cholesky/cholesky.py:2529-2553, 5625-5690) has ~1e-3 relative error per product, which
// fails a 1e-5 residual; 3xTF32 keeps the factor at FP32 accuracy.
//
// One CTA computes one BM x BN tile (BM = 128 rows of P, BN = 64/128/256 rows of Q):
//   warp 0      TMA producer: 128B-swizzled K-major boxes of P and Q (32 floats = 128 B
//               of K per row) into a STAGES-deep ring, mbarrier complete_tx.
//   warp 1      TMEM allocator; one elected thread issues tcgen05.mma kind::tf32
//               (M128 x N x K8, 3 per K8 step) and tcgen05.commit to release stages.
//   warps 2..5  split each landed stage into hi (in place) and lo (second buffer), then
//               the epilogue: tcgen05.ld 32x32b rows of the accumulator, combine with C,
//               write back (rows of a warp = its TMEM lane quarter).
// Every mbarrier wait is bounded by %globaltimer (2 s); on expiry the kernel records
// CHOL_ERR_WAIT_TIMEOUT in the device status word, skips the remaining work, frees its
// TMEM and returns.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "chol_tc_ptx.cuh"

namespace chol {

__device__ int g_device_status = 0;

namespace {

using namespace tcx;

constexpr int kBM = 128;
constexpr int kThreads = 320;  // producer, MMA, 4 converter warps, 4 epilogue warps

template <int BN>
struct TcCfg {
  static constexpr int STAGES = BN >= 256 ? 2 : (BN == 128 ? 3 : 4);
  static constexpr int A_BYTES = kBM * kBK * 4;
  static constexpr int B_BYTES = BN * kBK * 4;
  static constexpr int STAGE_BYTES = 2 * A_BYTES + 2 * B_BYTES;
  static constexpr int TMEM_COLS = BN;
  static constexpr int EPI_LD = 36;  // staging row stride (floats): conflict-free 16B access
  static constexpr int EPI_BYTES = 4 * 32 * EPI_LD * 4;  // one 32x32 tile per epilogue warp
  static constexpr size_t SMEM = size_t(STAGES) * STAGE_BYTES + EPI_BYTES + 1024 + 256;
  // TMEM: two BN-column FP32 accumulators (double buffer), 2*BN <= 512
  static_assert(BN == 64 || BN == 128 || BN == 256, "BN");
};

// Tile enumeration: per matrix, row tiles tm = 0..TM-1 and, in row tm, column tiles
// tn = 0..last(tm) where last(tm) = TN-1 for a full GEMM and the last tile touching the
// lower part (c <= r + diag_offset) otherwise. Tiles of one matrix are numbered row by row.
constexpr int kRowTable = 256;  // row tiles covered by the prefix table (kernel parameter): m <= 32768

struct TileSpace {
  int64_t tiles_m, tiles_n, per_matrix, total;
  int64_t diag_offset;
  int lower_only;
  int bn;
  int64_t col_step;  // global columns between consecutive column tiles (bn, or the cyclic stride)
  int use_table;     // row_start[] valid (tiles_m <= kRowTable)
  int32_t row_start[kRowTable + 1];  // index of tile (tm, 0) within a matrix
  __device__ __forceinline__ int64_t row_count(int64_t tm) const {
    if (!lower_only) return tiles_n;
    const int64_t last_c = tm * 128 + 127 + diag_offset;
    if (last_c < 0) return 0;
    const int64_t cnt = last_c / col_step + 1;
    return cnt < tiles_n ? cnt : tiles_n;
  }
  // Row tile holding in-matrix tile index r, searching from row tm0 (r >= row_start(tm0)).
  __device__ __forceinline__ void locate(int64_t r, int64_t& tm, int64_t& base) const {
    if (!lower_only) {
      tm = r / tiles_n;
      base = tm * tiles_n;
      return;
    }
    if (use_table) {
      int lo = int(tm), hi = int(tiles_m) - 1;  // invariant: row_start[lo] <= r
      while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (row_start[mid] <= r)
          lo = mid;
        else
          hi = mid - 1;
      }
      tm = lo;
      base = row_start[lo];
      return;
    }
    for (;;) {
      const int64_t cnt = row_count(tm);
      if (r < base + cnt) return;
      base += cnt;
      ++tm;
    }
  }
};

// PRELO: the low parts of P and Q come from precomputed buffers (tmPlo / tmQlo, same row
// coordinates, K from org.lpx / org.lqx): four TMA boxes per stage, no split pass, the
// MMA waits on TMA completion directly. Otherwise converter warps write lo in shared memory.
template <int BN, bool PRELO>
__global__ void __launch_bounds__(kThreads, 1)
    tc_gemm_kernel(const __grid_constant__ CUtensorMap tmP, const __grid_constant__ CUtensorMap tmQ,
                   const __grid_constant__ CUtensorMap tmPlo,
                   const __grid_constant__ CUtensorMap tmQlo, GemmArgs g, TileSpace ts,
                   TmaOrigin org, int* status) {
  using Cfg = TcCfg<BN>;
  constexpr int S = Cfg::STAGES;
  extern __shared__ __align__(1024) uint8_t smem_raw[];

  griddep_wait();  // before anything else: keeps the PDL chain ordered

  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  auto stA = [&](int s) { return reinterpret_cast<float*>(smem + size_t(s) * Cfg::STAGE_BYTES); };
  auto stAlo = [&](int s) { return stA(s) + Cfg::A_BYTES / 4; };
  auto stB = [&](int s) { return stAlo(s) + Cfg::A_BYTES / 4; };
  auto stBlo = [&](int s) { return stB(s) + Cfg::B_BYTES / 4; };
  float* epi = reinterpret_cast<float*>(smem + size_t(S) * Cfg::STAGE_BYTES);
  uint64_t* bars =
      reinterpret_cast<uint64_t*>(smem + size_t(S) * Cfg::STAGE_BYTES + Cfg::EPI_BYTES);
  uint64_t* full = bars;
  uint64_t* conv = bars + S;
  uint64_t* empty = bars + 2 * S;
  uint64_t* tfull = bars + 3 * S;       // [2] accumulator ready
  uint64_t* tempty = bars + 3 * S + 2;  // [2] accumulator drained
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 3 * S + 4);
  int* st_word = status ? status : &g_device_status;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&conv[s], 4);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 4);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    prefetch_map(&tmP);
    prefetch_map(&tmQ);
    if (PRELO) {
      prefetch_map(&tmPlo);
      prefetch_map(&tmQlo);
    }
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(uint32_t(2 * Cfg::TMEM_COLS))
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  griddep_launch();
  const uint32_t tmem = *tmem_slot;
  const int num_k = int((g.K + kBK - 1) / kBK);

  // This CTA's tiles: t = blockIdx.x, blockIdx.x + gridDim.x, ...  Walk (matrix, tm, tn).
  struct Cursor {
    int64_t t, mi, tm, tn, row_base;  // row_base: index of tile (mi, tm, 0) within matrix
    bool valid;
  };
  auto first_tile = [&](Cursor& c) {
    c.t = blockIdx.x;
    c.valid = c.t < ts.total;
    if (!c.valid) return;
    c.mi = c.t / ts.per_matrix;
    const int64_t r = c.t - c.mi * ts.per_matrix;
    c.tm = 0;
    c.row_base = 0;
    ts.locate(r, c.tm, c.row_base);
    c.tn = r - c.row_base;
  };
  auto next_tile = [&](Cursor& c) {
    c.t += gridDim.x;
    c.valid = c.t < ts.total;
    if (!c.valid) return;
    const int64_t mi = c.t / ts.per_matrix;
    const int64_t r = c.t - mi * ts.per_matrix;
    if (mi != c.mi) {
      c.mi = mi;
      c.tm = 0;
      c.row_base = 0;
    }
    ts.locate(r, c.tm, c.row_base);
    c.tn = r - c.row_base;
  };

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      Cursor c;
      first_tile(c);
      uint32_t kt = 0;
      bool ok = true;
      for (; c.valid && ok; next_tile(c)) {
        const int zc = int(c.mi);
        const int y0 = org.py + int(c.tm * kBM), y1 = org.qy + int(c.tn * ts.col_step);
        for (int k = 0; k < num_k; ++k, ++kt) {
          const int s = int(kt % S);
          const uint32_t ph = (kt / S) & 1u;
          if (kt >= uint32_t(S) && !mbar_wait(&empty[s], ph ^ 1u, st_word)) {
            ok = false;
            break;
          }
          mbar_expect_tx(&full[s], (PRELO ? 2 : 1) * (Cfg::A_BYTES + Cfg::B_BYTES));
          tma_load_3d(stA(s), &tmP, org.px + k * kBK, y0, zc, &full[s]);
          tma_load_3d(stB(s), &tmQ, org.qx + k * kBK, y1, zc, &full[s]);
          if (PRELO) {
            tma_load_3d(stAlo(s), &tmPlo, org.lpx + k * kBK, y0, zc, &full[s]);
            tma_load_3d(stBlo(s), &tmQlo, org.lqx + k * kBK, y1, zc, &full[s]);
          }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      const uint32_t idesc = tf32_idesc<kBM, BN>();
      Cursor c;
      first_tile(c);
      uint32_t kt = 0, it = 0;
      bool ok = true;
      for (; c.valid && ok; next_tile(c), ++it) {
        const uint32_t buf = it & 1u;
        if (it >= 2 && !mbar_wait(&tempty[buf], ((it >> 1) & 1u) ^ 1u, st_word)) break;
        tc_fence_after();
        const uint32_t acc = tmem + buf * uint32_t(Cfg::TMEM_COLS);
        for (int k = 0; k < num_k; ++k, ++kt) {
          const int s = int(kt % S);
          const uint32_t ph = (kt / S) & 1u;
          if (!mbar_wait(PRELO ? &full[s] : &conv[s], ph, st_word)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t da = sw128_desc(stA(s)), dal = sw128_desc(stAlo(s));
          const uint64_t db = sw128_desc(stB(s)), dbl = sw128_desc(stBlo(s));
#pragma unroll
          for (int kk = 0; kk < kBK / 8; ++kk) {
            const uint64_t adv = uint64_t(kk * 32 / 16);  // 8 tf32 = 32 bytes along K
            mma_tf32(acc, da + adv, db + adv, idesc, (k | kk) ? 1u : 0u);
            mma_tf32(acc, da + adv, dbl + adv, idesc, 1u);
            mma_tf32(acc, dal + adv, db + adv, idesc, 1u);
          }
          mma_commit(&empty[s]);
        }
        if (ok) mma_commit(&tfull[buf]);
      }
    }
  } else if (warp < 6) {
    // ---------------- converters: lo = x - trunc_tf32(x) ----------------
    if (!PRELO) {
    const int ct = threadIdx.x - 64;
    Cursor c;
    first_tile(c);
    uint32_t kt = 0;
    bool ok = true;
    for (; c.valid && ok; next_tile(c)) {
      for (int k = 0; k < num_k; ++k, ++kt) {
        const int s = int(kt % S);
        const uint32_t ph = (kt / S) & 1u;
        if (!mbar_wait(&full[s], ph, st_word)) {
          ok = false;
          break;
        }
        float4* a = reinterpret_cast<float4*>(stA(s));
        float4* al = reinterpret_cast<float4*>(stAlo(s));
        float4* b = reinterpret_cast<float4*>(stB(s));
        float4* bl = reinterpret_cast<float4*>(stBlo(s));
        const int64_t kval = g.K - int64_t(k) * kBK;  // valid K columns in this stage
        if (kval >= kBK) {
#pragma unroll
          for (int i = ct; i < Cfg::A_BYTES / 16; i += 128) split4<false>(a + i, al + i);
#pragma unroll
          for (int i = ct; i < Cfg::B_BYTES / 16; i += 128) split4<false>(b + i, bl + i);
        } else {
          // last partial stage: the box may reach past the view's K range (maps cover
          // the whole matrix), so columns >= kval are zeroed in both buffers
          for (int i = ct; i < Cfg::A_BYTES / 16; i += 128) split4_masked(a + i, al + i, i, int(kval));
          for (int i = ct; i < Cfg::B_BYTES / 16; i += 128) split4_masked(b + i, bl + i, i, int(kval));
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&conv[s]);
      }
    }
    }
  } else {
    // ---------------- epilogue: TMEM -> C ----------------
    // Per 32-column chunk: tcgen05.ld (thread = row), transpose through this warp's 32x32
    // staging tile, then rows of 32 floats read/written as coalesced 128-byte segments
    // (8 lanes per row, 4 rows per instruction).
    const int q = warp & 3;  // TMEM lane quarter this warp may read
    float* tile = epi + (warp - 6) * 32 * Cfg::EPI_LD;
    const int sub_r = lane >> 3, sub_c = (lane & 7) * 4;
    Cursor c;
    first_tile(c);
    uint32_t it = 0;
    for (; c.valid; next_tile(c), ++it) {
      const uint32_t buf = it & 1u;
      if (!mbar_wait(&tfull[buf], (it >> 1) & 1u, st_word)) break;
      tc_fence_after();
      const uint32_t acc = tmem + buf * uint32_t(Cfg::TMEM_COLS) + (uint32_t(q * 32) << 16);
      const int64_t row_base = c.tm * kBM + q * 32;  // first row of this warp's quarter
      const int64_t col0 = c.tn * BN;
      float* cbase = g.C + c.mi * g.cstride;
      const float* sbase = (g.Csrc != nullptr ? g.Csrc : g.C) + c.mi * g.cstride;
#pragma unroll 1
      for (int cc = 0; cc < BN / 32; ++cc) {
        const int64_t gc0 = col0 + cc * 32;
        if (gc0 >= g.ncols) break;
        float v[32];
        tmem_ld32(acc + uint32_t(cc * 32), v);
        // global column of local column gc0 (column-cyclic layouts shift whole blocks)
        const int64_t shift = g.cmap_block ? (gc0 / g.cmap_block) * (g.cmap_stride - g.cmap_block)
                                           : 0;
        // whole chunk above the lower boundary for every row of the quarter: nothing to do
        if (g.lower_only && gc0 + shift > row_base + 31 + g.diag_offset) continue;
        if (row_base >= g.m) continue;
        float* trow = tile + lane * Cfg::EPI_LD;
#pragma unroll
        for (int j = 0; j < 8; ++j)
          *reinterpret_cast<float4*>(trow + 4 * j) =
              make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
        __syncwarp();
        const int64_t col = gc0 + sub_c;
        // all eight row groups' C loads in flight before any use
        float4 cv[8];
        bool vec[8];
        int64_t lim[8];
#pragma unroll
        for (int rr = 0; rr < 8; ++rr) {
          const int64_t grow = row_base + rr * 4 + sub_r;
          float* cp = cbase + grow * g.ldc + col;
          const float* sp = sbase + grow * g.ldc + col;
          lim[rr] = grow >= g.m ? -1
                                : (g.lower_only ? (grow + g.diag_offset - shift < g.ncols - 1
                                                       ? grow + g.diag_offset - shift
                                                       : g.ncols - 1)
                                                : g.ncols - 1);
          vec[rr] = col + 3 <= lim[rr] && ((reinterpret_cast<uintptr_t>(cp) & 15) == 0);
          cv[rr] = make_float4(0.f, 0.f, 0.f, 0.f);
          if (vec[rr] && g.beta != 0.f) cv[rr] = *reinterpret_cast<const float4*>(sp);
        }
#pragma unroll
        for (int rr = 0; rr < 8; ++rr) {
          const int tr = rr * 4 + sub_r;
          if (lim[rr] < col) continue;
          const int64_t grow = row_base + tr;
          const float4 a4 = *reinterpret_cast<const float4*>(tile + tr * Cfg::EPI_LD + sub_c);
          float* cp = cbase + grow * g.ldc + col;
          const float* sp = sbase + grow * g.ldc + col;
          if (vec[rr]) {
            float4 o;
            o.x = fmaf(g.alpha, a4.x, g.beta * cv[rr].x);
            o.y = fmaf(g.alpha, a4.y, g.beta * cv[rr].y);
            o.z = fmaf(g.alpha, a4.z, g.beta * cv[rr].z);
            o.w = fmaf(g.alpha, a4.w, g.beta * cv[rr].w);
            *reinterpret_cast<float4*>(cp) = o;
          } else {
            const float av[4] = {a4.x, a4.y, a4.z, a4.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              if (col + e > lim[rr]) break;
              cp[e] = (g.beta != 0.f) ? fmaf(g.alpha, av[e], g.beta * sp[e]) : g.alpha * av[e];
            }
          }
        }
        __syncwarp();
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[buf]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(uint32_t(2 * Cfg::TMEM_COLS))
                 : "memory");
  }
}

// ------------------------------- host side ------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;

bool resolve_encode() {
  std::call_once(g_encode_once, []() {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  return g_encode != nullptr;
}

// 3-D map over (K, rows, batch) of row-major float32 rows with leading dimension ld.
bool make_map(CUtensorMap* map, const float* base, int64_t K, int64_t rows, int64_t batch,
              int64_t ld, int64_t bstride, int box_rows) {
  cuuint64_t dims[3] = {cuuint64_t(K), cuuint64_t(rows), cuuint64_t(batch)};
  cuuint64_t strides[2] = {cuuint64_t(ld) * 4, cuuint64_t(batch > 1 ? bstride : ld * rows) * 4};
  cuuint32_t box[3] = {cuuint32_t(kBK), cuuint32_t(box_rows), 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float*>(base), dims,
                        strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

TileSpace make_tiles(const GemmArgs& g, int bn) {
  TileSpace ts{};
  ts.tiles_m = (g.m + kBM - 1) / kBM;
  ts.tiles_n = (g.ncols + bn - 1) / bn;
  ts.diag_offset = g.diag_offset;
  ts.lower_only = g.lower_only;
  ts.bn = bn;
  ts.col_step = g.cmap_block ? g.cmap_stride : bn;
  ts.use_table = ts.lower_only && ts.tiles_m <= kRowTable;
  int64_t per = 0;
  for (int64_t tm = 0; tm < ts.tiles_m; ++tm) {
    if (ts.use_table) ts.row_start[tm] = int32_t(per);
    if (!ts.lower_only) {
      per += ts.tiles_n;
      continue;
    }
    const int64_t last_c = tm * kBM + kBM - 1 + ts.diag_offset;
    if (last_c < 0) continue;
    const int64_t cnt = last_c / ts.col_step + 1;
    per += cnt < ts.tiles_n ? cnt : ts.tiles_n;
  }
  if (ts.use_table) ts.row_start[ts.tiles_m] = int32_t(per);
  if (per > 0x7fffffffLL) ts.use_table = 0;
  ts.per_matrix = per;
  ts.total = per * g.batch;
  return ts;
}

int g_num_sms = 0;

template <int BN>
int launch_tc_maps(const GemmArgs& g, const CUtensorMap& mp, const CUtensorMap& mq,
                   TmaOrigin org, cudaStream_t q, bool pdl, int* status,
                   const CUtensorMap* mplo = nullptr, const CUtensorMap* mqlo = nullptr,
                   int max_ctas = 0) {
  using Cfg = TcCfg<BN>;
  const TileSpace ts = make_tiles(g, BN);
  if (ts.total == 0) return CHOL_OK;
  int sms = g_num_sms;
  if (sms <= 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  }
  int64_t ctas = ts.total < sms ? ts.total : sms;
  if (max_ctas > 0 && ctas > max_ctas) ctas = max_ctas;
  const int cap = gemm_cta_cap();
  if (cap > 0 && ctas > cap) ctas = cap;
  if (mplo != nullptr && mqlo != nullptr)
    return status_from(launch_pdl(tc_gemm_kernel<BN, true>, dim3(unsigned(ctas)), dim3(kThreads),
                                  Cfg::SMEM, q, pdl, mp, mq, *mplo, *mqlo, g, ts, org, status));
  return status_from(launch_pdl(tc_gemm_kernel<BN, false>, dim3(unsigned(ctas)), dim3(kThreads),
                                Cfg::SMEM, q, pdl, mp, mq, mp, mq, g, ts, org, status));
}

template <int BN>
int launch_tc_bn(const GemmArgs& g, cudaStream_t q, bool pdl, int* status) {
  CUtensorMap mp, mq;
  if (!make_map(&mp, g.P, g.K, g.m, g.batch, g.ldp, g.pstride, kBM)) return CHOL_ERR_UNSUPPORTED;
  // with a column-cyclic map Q's rows reach the last mapped row
  const int64_t qrows = g.cmap_block ? (g.ncols - 1) + ((g.ncols - 1) / g.cmap_block) *
                                                          (g.cmap_stride - g.cmap_block) + 1
                                     : g.ncols;
  if (!make_map(&mq, g.Q, g.K, qrows, g.batch, g.ldq, g.qstride, BN))
    return CHOL_ERR_UNSUPPORTED;
  return launch_tc_maps<BN>(g, mp, mq, TmaOrigin{0, 0, 0, 0, 0, 0}, q, pdl, status);
}

}  // namespace

// Per-launch maps with precomputed low parts: P = Q (the same rows; Q's rows follow the
// column-cyclic map), lo = the TF32 low parts of P (same rows, leading dimension ldlo).
int launch_gemm_tc_prelo(const GemmArgs& g, const float* lo, int64_t ldlo, cudaStream_t q,
                         bool pdl) {
  constexpr int BN = 256;
  if (g.P != g.Q || g.ldp != g.ldq || g.batch != 1) return CHOL_ERR_UNSUPPORTED;
  if ((reinterpret_cast<uintptr_t>(lo) & 15) || ldlo % 4) return CHOL_ERR_UNSUPPORTED;
  if (g.cmap_block && (g.cmap_block != 256 || g.cmap_stride < 256 || g.cmap_stride % 256))
    return CHOL_ERR_UNSUPPORTED;
  const int64_t qrows = g.cmap_block ? (g.ncols - 1) + ((g.ncols - 1) / g.cmap_block) *
                                                          (g.cmap_stride - g.cmap_block) + 1
                                     : g.ncols;
  if (qrows > g.m) return CHOL_ERR_UNSUPPORTED;  // Q's rows are rows of P
  CUtensorMap mp, mq, mplo, mqlo;
  if (!make_map(&mp, g.P, g.K, g.m, 1, g.ldp, 0, kBM) ||
      !make_map(&mq, g.Q, g.K, qrows, 1, g.ldq, 0, BN) ||
      !make_map(&mplo, lo, g.K, g.m, 1, ldlo, 0, kBM) ||
      !make_map(&mqlo, lo, g.K, qrows, 1, ldlo, 0, BN))
    return CHOL_ERR_UNSUPPORTED;
  return launch_tc_maps<BN>(g, mp, mq, TmaOrigin{0, 0, 0, 0, 0, 0}, q, pdl, nullptr, &mplo,
                            &mqlo);
}

bool tc_supported(const GemmArgs& g) {
  if (!resolve_encode()) return false;
  auto al16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  if (!al16(g.P) || !al16(g.Q)) return false;
  if (g.ldp % 4 || g.ldq % 4 || g.pstride % 4 || g.qstride % 4) return false;
  if (g.K < 1 || g.m < 1 || g.ncols < 1) return false;
  if (g.m > 0x7fffffffLL || g.ncols > 0x7fffffffLL || g.K > 0x7fffffffLL) return false;
  return true;
}

bool tc_make_matrix_maps(const float* base, int64_t rows, int64_t cols, int64_t ld,
                         int64_t batch, int64_t bstride, TcMatrixMaps* maps) {
  if (!resolve_encode()) return false;
  if ((reinterpret_cast<uintptr_t>(base) & 15) || ld % 4 || (batch > 1 && bstride % 4))
    return false;
  maps->base = base;
  maps->ld = ld;
  maps->bstride = bstride;
  return make_map(reinterpret_cast<CUtensorMap*>(maps->p128), base, cols, rows, batch, ld, bstride,
                  kBM) &&
         make_map(reinterpret_cast<CUtensorMap*>(maps->q64), base, cols, rows, batch, ld, bstride,
                  64) &&
         make_map(reinterpret_cast<CUtensorMap*>(maps->q128), base, cols, rows, batch, ld, bstride,
                  128) &&
         make_map(reinterpret_cast<CUtensorMap*>(maps->q256), base, cols, rows, batch, ld, bstride,
                  256);
}

// P and Q are views of the matrices behind pm / qm (element offsets from their bases).
int launch_gemm_tc_mapped(const GemmArgs& g, const TcMatrixMaps& pm, const TcMatrixMaps& qm,
                          cudaStream_t q, bool pdl, int max_ctas) {
  const int64_t po = g.P - pm.base, qo = g.Q - qm.base;
  if (po < 0 || qo < 0 || g.ldp != pm.ld || g.ldq != qm.ld) return CHOL_ERR_INVALID_ARG;
  if (g.batch > 1 && (g.pstride != pm.bstride || g.qstride != qm.bstride))
    return CHOL_ERR_INVALID_ARG;
  TmaOrigin org{int(po % pm.ld), int(po / pm.ld), int(qo % qm.ld), int(qo / qm.ld), 0, 0};
  if ((org.px & 3) || (org.qx & 3)) return CHOL_ERR_INVALID_ARG;  // TMA x must be 16-byte aligned
  const CUtensorMap& mp = *reinterpret_cast<const CUtensorMap*>(pm.p128);
  if (g.ncols <= 64)
    return launch_tc_maps<64>(g, mp, *reinterpret_cast<const CUtensorMap*>(qm.q64), org, q, pdl,
                              nullptr, nullptr, nullptr, max_ctas);
  if (g.ncols <= 128)
    return launch_tc_maps<128>(g, mp, *reinterpret_cast<const CUtensorMap*>(qm.q128), org, q,
                               pdl, nullptr, nullptr, nullptr, max_ctas);
  return launch_tc_maps<256>(g, mp, *reinterpret_cast<const CUtensorMap*>(qm.q256), org, q, pdl,
                             nullptr, nullptr, nullptr, max_ctas);
}

// As launch_gemm_tc_mapped with the low parts of P and Q read from a precomputed buffer
// (maps lm, rows indexed like P/Q's matrix, K origin lk) instead of split in the kernel.
int launch_gemm_tc_mapped_lo(const GemmArgs& g, const TcMatrixMaps& pm, const TcMatrixMaps& qm,
                             const TcMatrixMaps& lm, int64_t lk, cudaStream_t q, bool pdl,
                             int max_ctas) {
  const int64_t po = g.P - pm.base, qo = g.Q - qm.base;
  if (po < 0 || qo < 0 || g.ldp != pm.ld || g.ldq != qm.ld) return CHOL_ERR_INVALID_ARG;
  TmaOrigin org{int(po % pm.ld), int(po / pm.ld), int(qo % qm.ld), int(qo / qm.ld), int(lk),
                int(lk)};
  if ((org.px & 3) || (org.qx & 3) || (lk & 3)) return CHOL_ERR_INVALID_ARG;
  const CUtensorMap& mp = *reinterpret_cast<const CUtensorMap*>(pm.p128);
  const CUtensorMap& mpl = *reinterpret_cast<const CUtensorMap*>(lm.p128);
  if (g.ncols <= 64)
    return launch_tc_maps<64>(g, mp, *reinterpret_cast<const CUtensorMap*>(qm.q64), org, q, pdl,
                              nullptr, &mpl, reinterpret_cast<const CUtensorMap*>(lm.q64),
                              max_ctas);
  if (g.ncols <= 128)
    return launch_tc_maps<128>(g, mp, *reinterpret_cast<const CUtensorMap*>(qm.q128), org, q,
                               pdl, nullptr, &mpl, reinterpret_cast<const CUtensorMap*>(lm.q128),
                               max_ctas);
  return launch_tc_maps<256>(g, mp, *reinterpret_cast<const CUtensorMap*>(qm.q256), org, q, pdl,
                             nullptr, &mpl, reinterpret_cast<const CUtensorMap*>(lm.q256),
                             max_ctas);
}

int launch_gemm_tc(const GemmArgs& g, cudaStream_t q, bool pdl, int* status) {
  if (g.cmap_block) {
    if (g.cmap_block != 256 || g.cmap_stride < 256 || g.cmap_stride % 256) return CHOL_ERR_UNSUPPORTED;
    return launch_tc_bn<256>(g, q, pdl, status);
  }
  if (g.ncols <= 64) return launch_tc_bn<64>(g, q, pdl, status);
  if (g.ncols <= 128) return launch_tc_bn<128>(g, q, pdl, status);
  return launch_tc_bn<256>(g, q, pdl, status);
}

template <int BN>
cudaError_t set_tc_smem() {
  cudaError_t e = cudaFuncSetAttribute(tc_gemm_kernel<BN, false>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       int(TcCfg<BN>::SMEM));
  if (e != cudaSuccess) return e;
  return cudaFuncSetAttribute(tc_gemm_kernel<BN, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              int(TcCfg<BN>::SMEM));
}

// lo = x - trunc_tf32(x) for a rows x cols view (float4 columns; cols % 4 == 0).
__global__ void __launch_bounds__(256) tf32_lo_kernel(const float* src, int64_t lds, float* dst,
                                                      int64_t ldd, int64_t rows, int64_t cols4,
                                                      int64_t batch, int64_t sstride,
                                                      int64_t dstride, float* copy,
                                                      int64_t ldcopy, int64_t cstride) {
  griddep_wait();
  griddep_launch();
  const int64_t total = batch * rows * cols4;
  for (int64_t t = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; t < total;
       t += int64_t(gridDim.x) * blockDim.x) {
    const int64_t c4 = t % cols4;
    const int64_t rr = t / cols4;
    const int64_t r = rr % rows, m = rr / rows;
    const float4 x = *reinterpret_cast<const float4*>(src + m * sstride + r * lds + 4 * c4);
    float4 l;
    l.x = x.x - __uint_as_float(__float_as_uint(x.x) & 0xFFFFE000u);
    l.y = x.y - __uint_as_float(__float_as_uint(x.y) & 0xFFFFE000u);
    l.z = x.z - __uint_as_float(__float_as_uint(x.z) & 0xFFFFE000u);
    l.w = x.w - __uint_as_float(__float_as_uint(x.w) & 0xFFFFE000u);
    if (copy != nullptr) *reinterpret_cast<float4*>(copy + m * cstride + r * ldcopy + 4 * c4) = x;
    *reinterpret_cast<float4*>(dst + m * dstride + r * ldd + 4 * c4) = l;
  }
}

cudaError_t prepare_tc() {
  cudaError_t e;
  int dev = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev);
  if ((e = set_tc_smem<64>()) != cudaSuccess) return e;
  if ((e = set_tc_smem<128>()) != cudaSuccess) return e;
  if ((e = set_tc_smem<256>()) != cudaSuccess) return e;
  resolve_encode();
  return cudaSuccess;
}

int launch_tf32_lo(const float* src, int64_t lds, float* dst, int64_t ldd, int64_t rows,
                   int64_t cols, int64_t batch, int64_t sstride, int64_t dstride, cudaStream_t q,
                   float* copy, int64_t ldcopy, int64_t cstride) {
  if (rows <= 0 || cols <= 0 || batch <= 0) return CHOL_OK;
  if (cols % 4 || lds % 4 || ldd % 4 || (copy != nullptr && ldcopy % 4))
    return CHOL_ERR_UNSUPPORTED;
  const int64_t work = batch * rows * (cols / 4);
  int64_t blocks = (work + 255) / 256;
  const int64_t cap = int64_t(g_num_sms > 0 ? g_num_sms : 148) * 16;
  if (blocks > cap) blocks = cap;
  return status_from(launch_pdl(tf32_lo_kernel, dim3(unsigned(blocks)), dim3(256), 0, q, true,
                                src, lds, dst, ldd, rows, cols / 4, batch, sstride, dstride, copy,
                                ldcopy, cstride));
}

int* device_status_ptr() {
  static int* ptrs[64] = {};
  static std::mutex mu;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lock(mu);
  if (ptrs[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_device_status) == cudaSuccess) ptrs[dev] = static_cast<int*>(p);
  }
  return ptrs[dev];
}

int read_and_clear_status(int* out) {
  int zero = 0, v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_device_status, sizeof(int));
  if (e != cudaSuccess) return CHOL_ERR_DEVICE;
  if (v) cudaMemcpyToSymbol(g_device_status, &zero, sizeof(int));
  if (out) *out = v;
  return CHOL_OK;
}

}  // namespace chol
