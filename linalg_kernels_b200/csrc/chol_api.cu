// chol_api.cu — the C-ABI entry points and the host-side launch schedule.
//
// Mirrors the reference boundary custom_kernel(data) -> L (cholesky/cholesky.py:5845-5850):
// where the reference routes exact shapes to per-shape modules and sends everything else
// to torch, this library plans every (batch, n) on the GPU:
//   n <= 64   one launch of the warp-register kernel (chol_small.cu)
//   n <= 128  one launch of the shared-memory kernel, one CTA per matrix (chol_mid.cu)
//   n  > 64   right-looking blocked schedule, 64-wide diagonal blocks, outer panels of
//             width NB, left-looking inside a panel and right-looking between panels:
//               copy tril(A) -> L
//               for each outer panel [K0, K0+NB):
//                 for each 64-wide block column k in the panel:
//                   L[k:, k:k+64] -= L[k:, K0:k] L[k:k+64, K0:k]^T   (GEMM, K = k - K0)
//                   potrf_block(k)            factor + inverse T_k   (1 CTA / matrix)
//                   X = L[k+64:, k] * T_k^T   panel solve, in place  (GEMM)
//                 L[K0+NB:, K0+NB:] -= P * P^T, P = L[K0+NB:, K0:K0+NB]  (lower tiles, K = NB)
// All launches go on the caller's queue with programmatic dependent launch.
#include <mutex>
#include <vector>

#include "chol_common.cuh"

namespace chol {

namespace {

constexpr int64_t kBlock = 64;

int g_outer_width = 0;  // 0: default (below)

// n <= 1024: one outer panel. Larger: panels of width NB with a rank-NB trailing update
// between them. A wider diagonal block is one launch whose tile tasks run concurrently, so
// fewer, wider panels shorten the serial chain of blocks (B200: b1n4096 1.38 / 1.33 / 1.21 ms
// at NB = 512 / 768 / 1024, b1n16384 12.56 / 12.19 / 12.21, b1n32768 81.5 / 76.9 / 77.0).
// But the panel solve and the trailing update run K = NB through the 3xTF32 accumulator,
// whose error grows with K: on spectral inputs of condition 1e5 the relative residual is
// 5.0e-6 / 7.5e-6 / 1.0e-5 (n = 4096), against the 1e-5 gate. So NB = 768 above n = 2048
// (the gate kept with a margin) and 512 up to n = 2048 (b8n2048: 0.83 ms against 0.85).
int64_t outer_width(int64_t n) {
  if (g_outer_width > 0 && g_outer_width % 64 == 0) return n <= g_outer_width ? n : g_outer_width;
  if (n <= 1024) return n;
  return n <= 2048 ? 512 : 768;
}

struct DeviceState {
  std::once_flag once;
  int status = CHOL_OK;
  std::mutex ws_mu;
  void* ws = nullptr;
  size_t ws_bytes = 0;
};

DeviceState* device_state(int dev) {
  static DeviceState states[64];
  if (dev < 0 || dev >= 64) return nullptr;
  return &states[dev];
}

int prepare_device(int dev) {
  DeviceState* st = device_state(dev);
  if (!st) return CHOL_ERR_DEVICE;
  std::call_once(st->once, [&]() {
    int prev = 0;
    if (cudaGetDevice(&prev) != cudaSuccess) {
      st->status = CHOL_ERR_DEVICE;
      return;
    }
    if (prev != dev && cudaSetDevice(dev) != cudaSuccess) {
      st->status = CHOL_ERR_DEVICE;
      return;
    }
    int major = 0, minor = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
    if (major != 10) {
      st->status = CHOL_ERR_DEVICE;
    } else if (prepare_small() != cudaSuccess || prepare_kernels(dev) != CHOL_OK) {
      st->status = CHOL_ERR_DEVICE;
    }
    if (prev != dev) cudaSetDevice(prev);
  });
  return st->status;
}

bool overlaps_partially(const float* a, const float* b, int64_t count) {
  if (a == b) return false;
  const uintptr_t a0 = reinterpret_cast<uintptr_t>(a), b0 = reinterpret_cast<uintptr_t>(b);
  const uintptr_t bytes = uintptr_t(count) * sizeof(float);
  return a0 < b0 + bytes && b0 < a0 + bytes;
}

// Workspace of the blocked path: the inverse diagonal blocks (64 x 64 floats per matrix,
// used by the 64-wide chain and the FP32-FMA schedule) are required. When there is a
// trailing update (n > outer width
// NB, n % 4 == 0) two optional regions follow: the panel buffer (n x NB floats per matrix),
// which holds the panel solve's output and then the low TF32 parts of the solved panel that
// the trailing GEMM loads instead of splitting in shared memory, and V = inv(L11) of the
// panel's NB x NB diagonal block (NB x NB floats per matrix).
size_t blocked_workspace_min(int64_t batch, int64_t n) {
  if (n <= 64 || use_mid(batch, n)) return 0;
  return size_t(batch) * kBlock * kBlock * sizeof(float);
}
size_t blocked_lo_bytes(int64_t batch, int64_t n) {
  const int64_t NB = outer_width(n);
  if (n <= 64 || NB >= n || n % 4) return 0;
  return size_t(batch) * size_t(n) * size_t(NB) * sizeof(float);
}
// V, then the diagonal-block kernel's flags (kDiagFlags ints per matrix) and one ticket
// counter per outer panel; all zeroed once per call.
size_t blocked_inv_bytes(int64_t batch, int64_t n) {
  const int64_t NB = outer_width(n);
  if (blocked_lo_bytes(batch, n) == 0 || NB % kBlock || NB > 16 * kBlock) return 0;
  const int64_t panels = (n + NB - 1) / NB;
  return size_t(batch) * size_t(NB) * size_t(NB) * sizeof(float) +
         size_t(batch) * kDiagFlags * sizeof(int) + ((size_t(panels) * 4 + 255) & ~size_t(255));
}
// n <= outer width (one panel), n % 64 == 0, n <= 1024: the whole matrix is factored by
// one diagonal-block launch when the batch is small enough for its latency to matter more
// than throughput: its tile tasks run FP32 FMA at about 10 TFMA/s on a B200, against the
// tensor-core GEMM chain's ~30 us per 64 columns of latency. batch * n^3 <= kDiagWork is the
// measured crossover (b64n256: 77 us against 121 us; b640n512: 2.7 ms against 1.48 ms).
// It needs the 64 x 64 inverse blocks, the tile flags and a ticket counter (zeroed per call).
constexpr double kDiagWork = 1.2e10;
size_t blocked_diag_bytes(int64_t batch, int64_t n) {
  if (n <= 64 || outer_width(n) < n || n % kBlock || n > 16 * kBlock) return 0;
  if (double(batch) * double(n) * double(n) * double(n) > kDiagWork) return 0;
  const int64_t nb = n / kBlock;
  return size_t(batch) * (size_t(nb) * kBlock * kBlock * sizeof(float) + kDiagFlags * sizeof(int)) +
         256;
}
// One panel, batches beyond the one-launch crossover, n % 128 == 0: the left-looking chain
// takes 128-wide block columns (CHOL_OPT_CHAIN_WIDTH, 128 by default), each diagonal block
// factored with its inverse T (128 x 128 per matrix, this region) by one launch. Against the
// 64-wide chain: half the launches and half the re-reads of the panel left of each block
// column (b640n512: 2.75 -> 1.9 GB of traffic per call; 1.31 -> 1.03 ms). One CTA of that
// block factor takes ~50 us, mostly fetching its unrolled 64 x 64 factor code, so it pays only
// with several CTAs per SM to overlap: batches of at least kChain128Batch (b60n1024 keeps
// the 64-wide chain: 0.95 against 0.97 ms).
int g_chain_width = 128;
constexpr int64_t kChain128Batch = 256;
size_t blocked_t128_bytes(int64_t batch, int64_t n) {
  if (g_chain_width != 128 || n < 256 || n % 128 || outer_width(n) < n || n > 16 * kBlock ||
      batch < kChain128Batch)
    return 0;
  if (blocked_diag_bytes(batch, n)) return 0;  // the one-launch path takes these
  return size_t(batch) * 128 * 128 * sizeof(float);
}
size_t blocked_workspace(int64_t batch, int64_t n) {
  if (use_mid(batch, n)) return 0;
  return blocked_workspace_min(batch, n) + blocked_lo_bytes(batch, n) +
         blocked_inv_bytes(batch, n) + blocked_diag_bytes(batch, n) +
         blocked_t128_bytes(batch, n);
}

// The 128-wide left-looking chain over one panel (reads A directly, like the 64-wide one):
//   for each block column k (128 wide):
//     L[k:, k:k+128] = A[k:, k:k+128] - L[k:, 0:k] L[k:k+128, 0:k]^T     (k > 0, lower part)
//     potrf_block128: L_kk and T_k = inv(L_kk), and the zeros of L's rows right of L_kk
//     L[k+128:, k:k+128] <- L[k+128:, k:k+128] T_k^T                     (in place; A at k = 0)
// The solve runs in place: its GEMM tiles are 128 x 128 with K = 128, so each tile reads its
// whole P block before its epilogue writes the same rows and columns. Returns
// CHOL_ERR_UNSUPPORTED (nothing launched) when the tensor maps cannot be built.
int run_chain128(const float* A, float* L, int64_t batch, int64_t n, int* info, float* T128,
                 cudaStream_t q) {
  const int64_t mstride = n * n;
  TcMatrixMaps lm, am, tm;
  if (!tc_make_matrix_maps(L, n, n, n, batch, mstride, &lm) ||
      !tc_make_matrix_maps(A, n, n, n, batch, mstride, &am) ||
      !tc_make_matrix_maps(T128, 128, 128, 128, batch, 128 * 128, &tm))
    return CHOL_ERR_UNSUPPORTED;
  int st = CHOL_OK;
  for (int64_t k = 0; k < n; k += 128) {
    if (k > 0) {
      GemmArgs u{};
      u.C = L + k * n + k;
      u.Csrc = A + k * n + k;
      u.cstride = mstride;
      u.ldc = n;
      u.P = L + k * n;
      u.pstride = mstride;
      u.ldp = n;
      u.Q = u.P;
      u.qstride = mstride;
      u.ldq = n;
      u.m = n - k;
      u.ncols = 128;
      u.K = k;
      u.alpha = -1.f;
      u.beta = 1.f;
      u.lower_only = 1;
      u.batch = batch;
      if ((st = launch_gemm_tc_mapped(u, lm, lm, q, true))) return st;
    }
    const float* S = k == 0 ? A : L;
    if ((st = launch_potrf_block128(S, mstride, n, L, mstride, n, batch, k, T128, 128 * 128, 128,
                                    info, q, n - k - 128)))
      return st;
    const int64_t below = n - k - 128;
    if (below <= 0) continue;
    GemmArgs x{};
    x.C = L + (k + 128) * n + k;
    x.cstride = mstride;
    x.ldc = n;
    x.P = S + (k + 128) * n + k;
    x.pstride = mstride;
    x.ldp = n;
    x.Q = T128;
    x.qstride = 128 * 128;
    x.ldq = 128;
    x.m = below;
    x.ncols = 128;
    x.K = 128;
    x.alpha = 1.f;
    x.beta = 0.f;
    x.lower_only = 0;
    x.batch = batch;
    if ((st = launch_gemm_tc_mapped(x, k == 0 ? am : lm, tm, q, true))) return st;
  }
  return CHOL_OK;
}

// Tensor-core GEMMs of one call share tensor maps built once over L and the inverse blocks;
// views are addressed by TMA coordinates. Falls back to FP32 FMA when the maps cannot be
// built (unaligned rows) or the engine option asks for it.
struct BlockedMaps {
  bool ok = false;
  TcMatrixMaps L, T, A;  // A: only for the one-panel chain that reads the input directly
};

int gemm_on(const GemmArgs& g, const BlockedMaps& bm, const TcMatrixMaps& pm,
            const TcMatrixMaps& qm, cudaStream_t q, int max_ctas = 0) {
  if (g.m <= 0 || g.ncols <= 0) return CHOL_OK;
  if (bm.ok && g_gemm_engine != 1) return launch_gemm_tc_mapped(g, pm, qm, q, true, max_ctas);
  if (g_gemm_engine == 2) return CHOL_ERR_UNSUPPORTED;
  return launch_gemm_simt(g, q, true);
}

// Look-ahead between outer panels (large n): the trailing update of panel J is split into
// T1 (panel J+1's own columns, on the caller's queue) and T2 (everything to its right, on a
// library side queue with its grid capped so that g_chain_sms SMs stay free); panel J+1's
// diagonal block, panel solve and split then run beside T2. The cap slows T2 by about
// sms / (sms - g_chain_sms), so the split is taken only while T2 is short enough for the
// overlap to win: batch * rest^2 <= kLookaheadWork (rest = rows below the next panel; about
// 1 ms of T2 on a B200 against ~0.2 ms of per-panel chain). Automatic (-1, the default):
// on for n <= kLookaheadAutoN, where it measured faster (b1n4096 1.41 -> 1.38 ms, b2n4096
// 1.55 -> 1.49, b1n8192 3.58 -> 3.29); at n = 16384 the capped T2 costs more than the
// overlap wins (12.80 against 12.72 ms), so it stays off there.
int g_lookahead = -1;
int g_chain_sms = 24;
constexpr double kLookaheadWork = 4.0e8;
constexpr int64_t kLookaheadAutoN = 8192;

bool lookahead_on(int64_t n) {
  return g_lookahead == 1 || (g_lookahead < 0 && n <= kLookaheadAutoN);
}
bool lookahead_split(int64_t batch, int64_t n, int64_t rest_after_next) {
  return lookahead_on(n) && rest_after_next > 0 &&
         double(batch) * double(rest_after_next) * double(rest_after_next) <= kLookaheadWork;
}

struct SideQueue {
  std::once_flag once;
  std::mutex order;  // one enqueue at a time: the events are shared by all callers
  bool ok = false;
  cudaStream_t s = nullptr;
  cudaEvent_t ready[2] = {nullptr, nullptr};
  cudaEvent_t done[2] = {nullptr, nullptr};
};

SideQueue* side_queue(int dev) {
  static SideQueue qs[64];
  if (dev < 0 || dev >= 64) return nullptr;
  SideQueue* sq = &qs[dev];
  std::call_once(sq->once, [sq]() {
    bool ok = cudaStreamCreateWithFlags(&sq->s, cudaStreamNonBlocking) == cudaSuccess;
    for (int i = 0; i < 2 && ok; ++i)
      ok = cudaEventCreateWithFlags(&sq->ready[i], cudaEventDisableTiming) == cudaSuccess &&
           cudaEventCreateWithFlags(&sq->done[i], cudaEventDisableTiming) == cudaSuccess;
    sq->ok = ok;
  });
  return sq->ok ? sq : nullptr;
}

// One panel (n <= 1024, n % 64 == 0): the whole matrix goes through diag_block_kernel in one
// launch (option value 1, the default). Several panels:
// Panel solve by the inverse of the diagonal block (default; needs the optional workspace):
// one launch (diag_block_kernel) factors the panel's NB x NB diagonal block and writes
// V = inv(L11), and the rows below the block are solved by ONE tensor-core GEMM,
// X = A21 V^T, over every row at once. 2 = the same, with the block factored by the chain
// of small kernels and V from trtri_panel. 0 = the chain covers every row of the panel
// (left-looking GEMMs with m = n - k).
int g_panel_inverse = 1;

int run_blocked(const float* A, float* L, int64_t batch, int64_t n, int* info, float* Tws,
                size_t ws_bytes, cudaStream_t q) {
  const int64_t mstride = n * n;
  const size_t min_bytes = blocked_workspace_min(batch, n);
  const size_t lo_bytes = blocked_lo_bytes(batch, n);
  const size_t inv_bytes = blocked_inv_bytes(batch, n);
  char* ws = reinterpret_cast<char*>(Tws);
  float* lo = (lo_bytes && ws_bytes >= min_bytes + lo_bytes)
                  ? reinterpret_cast<float*>(ws + min_bytes)
                  : nullptr;
  float* V = (lo && inv_bytes && ws_bytes >= min_bytes + lo_bytes + inv_bytes)
                 ? reinterpret_cast<float*>(ws + min_bytes + lo_bytes)
                 : nullptr;
  const size_t dg_bytes = blocked_diag_bytes(batch, n);
  if (dg_bytes && g_panel_inverse == 1 && g_gemm_engine != 1 && ws_bytes >= min_bytes + dg_bytes) {
    // one panel: the diagonal-block kernel factors the whole matrix in one launch
    const int nb = int(n / kBlock);
    float* tblk = reinterpret_cast<float*>(ws + min_bytes);
    int* fl = reinterpret_cast<int*>(tblk + batch * nb * kBlock * kBlock);
    unsigned* tk = reinterpret_cast<unsigned*>(fl + batch * kDiagFlags);
    if (cudaMemsetAsync(fl, 0, size_t(batch) * kDiagFlags * sizeof(int) + 256, q) != cudaSuccess)
      return CHOL_ERR_LAUNCH;
    int st = launch_copy_lower(A, L, batch, n, q, true);
    if (st) return st;
    return launch_diag_block(L, mstride, n, tblk, int64_t(nb) * kBlock * kBlock, kBlock, nb,
                             false, fl, tk, 1, info, 0, batch, q);
  }
  const size_t t128 = blocked_t128_bytes(batch, n);
  if (t128 && g_gemm_engine != 1 && ws_bytes >= min_bytes + t128) {
    const int st = run_chain128(A, L, batch, n, info, reinterpret_cast<float*>(ws + min_bytes), q);
    if (st != CHOL_ERR_UNSUPPORTED) return st;
  }
  BlockedMaps bm;
  TcMatrixMaps lomap, vmap;
  const int64_t NBw = outer_width(n);
  if (g_gemm_engine != 1)
    bm.ok = tc_make_matrix_maps(L, n, n, n, batch, mstride, &bm.L) &&
            tc_make_matrix_maps(Tws, kBlock, kBlock, kBlock, batch, kBlock * kBlock, &bm.T);
  if (!bm.ok || (lo && !tc_make_matrix_maps(lo, n, NBw, NBw, batch, n * NBw, &lomap)))
    lo = nullptr;
  if (!lo || !g_panel_inverse || (V && !tc_make_matrix_maps(V, NBw, NBw, NBw, batch, NBw * NBw,
                                                             &vmap)))
    V = nullptr;
  const bool inv = V != nullptr;
  const bool diag_kernel = inv && g_panel_inverse == 1;
  int* dflags = inv ? reinterpret_cast<int*>(V + batch * NBw * NBw) : nullptr;
  unsigned* tickets = inv ? reinterpret_cast<unsigned*>(dflags + batch * kDiagFlags) : nullptr;
  if (inv && cudaMemsetAsync(V, 0, inv_bytes, q) != cudaSuccess) return CHOL_ERR_LAUNCH;
  int dev = 0;
  cudaGetDevice(&dev);
  SideQueue* sq = (lo != nullptr && lookahead_on(n)) ? side_queue(dev) : nullptr;
  std::unique_lock<std::mutex> hold;
  if (sq != nullptr) hold = std::unique_lock<std::mutex>(sq->order);
  int pending = -1, ev = 0, chain_cap = 0;
  // One panel (n <= outer width), 64-wide chain: every block column of L is produced once,
  // so the chain reads A where the copy would be read: the first diagonal block and solve
  // take A, each left-looking update takes its beta * C term from A and writes L, and only
  // the part of L right of the diagonal blocks needs zeros (a third of copy_lower's traffic).
  const bool from_a = NBw >= n &&
                      (!bm.ok || tc_make_matrix_maps(A, n, n, n, batch, mstride, &bm.A));
  int st = from_a ? launch_zero_upper(L, batch, n, q, true)
                  : launch_copy_lower(A, L, batch, n, q, true);
  if (st) return st;
  // the previous panel's side-queue update must finish before the panel buffer is rewritten
  auto join_pending = [&]() -> int {
    if (pending < 0) return CHOL_OK;
    if (cudaStreamWaitEvent(q, sq->done[pending], 0) != cudaSuccess) return CHOL_ERR_LAUNCH;
    pending = -1;
    return CHOL_OK;
  };
  const int64_t NB = NBw;
  for (int64_t K0 = 0; K0 < n; K0 += NB) {
    const int64_t KB = (n - K0) < NB ? (n - K0) : NB;
    const int64_t rest = n - K0 - KB;
    // rows the in-panel chain updates and solves: the diagonal block only, or every row
    const int64_t chain_end = inv ? K0 + KB : n;
    const bool one_launch = diag_kernel && KB % kBlock == 0;
    if (one_launch) {
      st = launch_diag_block(L + K0 * n + K0, mstride, n, V, NBw * NBw, NBw, int(KB / kBlock),
                             rest > 0, dflags, tickets + K0 / NB, int(K0 / NB) + 1, info, K0,
                             batch, q);
      if (st) return st;
    }
    for (int64_t k = K0; !one_launch && k < K0 + KB; k += kBlock) {
      const int64_t kb = (K0 + KB - k) < kBlock ? (K0 + KB - k) : kBlock;
      // inv(L_kk) goes to V's diagonal block (inverse schedule) or the 64 x 64 slot
      float* Tk = inv ? V + (k - K0) * NBw + (k - K0) : Tws;
      const int64_t tstride = inv ? NBw * NBw : kBlock * kBlock;
      const int64_t tld = inv ? NBw : kBlock;
      if (k > K0) {
        // left-looking inside the outer panel: block column k receives the updates of the
        // panel's already factored columns [K0, k) in one GEMM (K = k - K0)
        GemmArgs u{};
        u.C = L + k * n + k;
        if (from_a) u.Csrc = A + k * n + k;
        u.cstride = mstride;
        u.ldc = n;
        u.P = L + k * n + K0;
        u.pstride = mstride;
        u.ldp = n;
        u.Q = u.P;
        u.qstride = mstride;
        u.ldq = n;
        u.m = chain_end - k;
        u.ncols = kb;
        u.K = k - K0;
        u.alpha = -1.f;
        u.beta = 1.f;
        u.diag_offset = 0;
        u.lower_only = 1;
        u.batch = batch;
        st = gemm_on(u, bm, bm.L, bm.L, q, chain_cap);
        if (st) return st;
      }
      // (from_a: block column 0 is read from A, the others after their left update in L)
      const bool first_from_a = from_a && k == 0;
      st = launch_potrf_block(first_from_a ? A : L, mstride, n, L, mstride, n, batch, k, kb, Tk,
                              info, q, true,
                              tstride, tld);
      if (st) return st;
      const int64_t below = chain_end - k - kb;
      if (below <= 0) continue;
      // panel solve: L[k+kb:, k:k+kb] <- L[k+kb:, k:k+kb] * T^T (in place)
      GemmArgs s{};
      s.C = L + (k + kb) * n + k;
      s.cstride = mstride;
      s.ldc = n;
      s.P = first_from_a ? A + (k + kb) * n + k : s.C;
      s.pstride = mstride;
      s.ldp = n;
      s.Q = Tk;
      s.qstride = tstride;
      s.ldq = tld;
      s.m = below;
      s.ncols = kb;
      s.K = kb;
      s.alpha = 1.f;
      s.beta = 0.f;
      s.lower_only = 0;
      s.batch = batch;
      st = gemm_on(s, bm, first_from_a ? bm.A : bm.L, inv ? vmap : bm.T, q, chain_cap);
      if (st) return st;
    }
    if (rest <= 0) continue;
    GemmArgs t{};
    t.C = L + (K0 + KB) * n + (K0 + KB);
    t.cstride = mstride;
    t.ldc = n;
    t.P = L + (K0 + KB) * n + K0;
    t.pstride = mstride;
    t.ldp = n;
    t.Q = t.P;
    t.qstride = mstride;
    t.ldq = n;
    t.m = rest;
    t.ncols = rest;
    t.K = KB;
    t.alpha = -1.f;
    t.beta = 1.f;
    t.diag_offset = 0;
    t.lower_only = 1;
    t.batch = batch;
    if (lo == nullptr || KB != NBw || g_gemm_engine == 1) {
      st = gemm_on(t, bm, bm.L, bm.L, q);
      if (st) return st;
      continue;
    }
    if ((st = join_pending())) return st;
    float* pbuf = lo + (K0 + KB) * NBw;  // panel buffer rows of the rows below the block
    if (inv) {
      if (!one_launch) {
        st = launch_trtri_panel(L + K0 * n + K0, mstride, n, V, NBw * NBw, NBw,
                                int(KB / kBlock), batch, q);
        if (st) return st;
      }
      // X = A21 V^T for every row below the diagonal block, into the panel buffer (the GEMM
      // reads whole rows of A21, so it cannot write them in place)
      GemmArgs x{};
      x.C = pbuf;
      x.cstride = n * NBw;
      x.ldc = NBw;
      x.P = t.P;
      x.pstride = mstride;
      x.ldp = n;
      x.Q = V;
      x.qstride = NBw * NBw;
      x.ldq = NBw;
      x.m = rest;
      x.ncols = KB;
      x.K = KB;
      x.alpha = 1.f;
      x.beta = 0.f;
      x.lower_only = 0;
      x.batch = batch;
      st = launch_gemm_tc_mapped(x, bm.L, vmap, q, true);
      if (st) return st;
      // L21 <- X, and the panel buffer <- low TF32 parts of X for the trailing GEMM
      st = launch_tf32_lo(pbuf, NBw, pbuf, NBw, rest, KB, batch, n * NBw, n * NBw, q,
                          L + (K0 + KB) * n + K0, n, mstride);
    } else {
      // low parts of the panel rows below it, computed once, read by every tile
      st = launch_tf32_lo(t.P, n, pbuf, NBw, rest, KB, batch, mstride, n * NBw, q);
    }
    if (st) return st;
    const int64_t K0n = K0 + KB;
    const int64_t KBn = rest < NBw ? rest : NBw;
    if (sq != nullptr && rest > KBn && lookahead_split(batch, n, rest - KBn)) {
      // T1: next panel's columns, here; T2: the rest, on the side queue
      GemmArgs t1 = t;
      t1.ncols = KBn;
      st = launch_gemm_tc_mapped_lo(t1, bm.L, bm.L, lomap, 0, q, true);
      if (st) return st;
      if (cudaEventRecord(sq->ready[ev], q) != cudaSuccess ||
          cudaStreamWaitEvent(sq->s, sq->ready[ev], 0) != cudaSuccess)
        return CHOL_ERR_LAUNCH;
      GemmArgs t2 = t;
      t2.C = L + (K0n + KBn) * n + (K0n + KBn);
      t2.P = L + (K0n + KBn) * n + K0;
      t2.Q = t2.P;
      t2.m = rest - KBn;
      t2.ncols = rest - KBn;
      int sms = 148;
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
      st = launch_gemm_tc_mapped_lo(t2, bm.L, bm.L, lomap, 0, sq->s, false, sms - g_chain_sms);
      if (st) return st;
      if (cudaEventRecord(sq->done[ev], sq->s) != cudaSuccess) return CHOL_ERR_LAUNCH;
      pending = ev;
      ev ^= 1;
      chain_cap = inv ? 0 : g_chain_sms;
      continue;
    }
    chain_cap = 0;
    st = launch_gemm_tc_mapped_lo(t, bm.L, bm.L, lomap, 0, q, true);
    if (st) return st;
  }
  return join_pending();
}

// Launch count of run_blocked for (batch, n); keep in step with the schedule above.
int64_t blocked_launches(int64_t batch, int64_t n) {
  if (blocked_diag_bytes(batch, n) && g_panel_inverse == 1 && g_gemm_engine != 1)
    return 2;  // copy_lower + diagonal-block kernel
  if (blocked_t128_bytes(batch, n) && g_gemm_engine != 1) {
    int64_t count = 0;
    for (int64_t k = 0; k < n; k += 128)
      count += (k > 0 ? 1 : 0) + 1 + (n - k - 128 > 0 ? 1 : 0);  // update, factor, solve
    return count;
  }
  const bool pre = blocked_lo_bytes(batch, n) > 0 && g_gemm_engine != 1;
  const bool inv = pre && g_panel_inverse && blocked_inv_bytes(batch, n) > 0;
  const bool diag_kernel = inv && g_panel_inverse == 1;
  int64_t count = 1;  // copy_lower
  const int64_t NB = outer_width(n);
  for (int64_t K0 = 0; K0 < n; K0 += NB) {
    const int64_t KB = (n - K0) < NB ? (n - K0) : NB;
    const int64_t rest = n - K0 - KB;
    const int64_t chain_end = inv ? K0 + KB : n;
    const bool one_launch = diag_kernel && KB % kBlock == 0;
    if (one_launch) count += 1;  // diagonal block + its inverse
    for (int64_t k = K0; !one_launch && k < K0 + KB; k += kBlock) {
      const int64_t kb = (K0 + KB - k) < kBlock ? (K0 + KB - k) : kBlock;
      if (k > K0) count += 1;                  // left-looking panel update
      count += 1;                              // diagonal block
      if (chain_end - k - kb > 0) count += 1;  // panel solve
    }
    if (rest <= 0) continue;
    if (!pre) {
      count += 1;  // trailing update
      continue;
    }
    count += inv ? (one_launch ? 2 : 3) : 1;     // ((trtri +) solve GEMM +) split/lo pass
    count += 1;                                  // trailing update
    if (rest > NB && lookahead_split(batch, n, rest - NB)) count += 1;  // T1 + T2
  }
  return count;
}

int check_common(const float* A, float* L, int64_t batch, int64_t n) {
  if (batch < 0 || n < 0) return CHOL_ERR_INVALID_ARG;
  if (batch == 0 || n == 0) return CHOL_OK;
  if (A == nullptr || L == nullptr) return CHOL_ERR_INVALID_ARG;
  if (n > (int64_t(1) << 20)) return CHOL_ERR_UNSUPPORTED;
  if (overlaps_partially(A, L, batch * n * n)) return CHOL_ERR_INVALID_ARG;
  return CHOL_OK;
}

int potrf_impl(const float* A, float* L, int64_t batch, int64_t n, int* info, void* ws,
               size_t ws_bytes, cudaStream_t q) {
  if (n <= 64) return launch_small(A, L, batch, int(n), info, q);
  if (use_mid(batch, n)) return launch_mid(A, L, batch, int(n), info, q);
  if (ws == nullptr || ws_bytes < blocked_workspace_min(batch, n)) return CHOL_ERR_WORKSPACE;
  if (batch > 0x7fffffffLL) return CHOL_ERR_UNSUPPORTED;
  return run_blocked(A, L, batch, n, info, static_cast<float*>(ws), ws_bytes, q);
}

// Scratch of the panel factor by the block inverse (V, tile flags, ticket, the solved rows),
// cached per device and grown on demand, like the workspace of chol_potrf_batched_f32.
struct PanelScratch {
  std::mutex mu;
  void* p = nullptr;
  size_t bytes = 0;
};

void* cached_scratch(PanelScratch& s, size_t need) {
  std::lock_guard<std::mutex> lock(s.mu);
  if (s.bytes < need) {
    if (s.p != nullptr) cudaFree(s.p);
    s.p = nullptr;
    s.bytes = 0;
    if (cudaMalloc(&s.p, need) != cudaSuccess) return nullptr;
    s.bytes = need;
  }
  return s.p;
}

void* panel_scratch(int dev, size_t need) {
  static PanelScratch ps[64];
  if (dev < 0 || dev >= 64) return nullptr;
  return cached_scratch(ps[dev], need);
}

// Panel of width w (w % 64 == 0, w <= 1024): diag_block_kernel factors the w x w top block
// and writes V = inv(L11); one GEMM solves every row below, X = A21 V^T, into scratch;
// tf32_lo_kernel copies X back into L (its low-part output stays in scratch, unused).
// With out != nullptr the solve writes X straight into rows w.. of out (m x w, row-major,
// contiguous), and the top block is copied there too: the packed panel, ready to send.
int panel_potrf_inverse(float* L, int64_t ld, int64_t m, int64_t w, int* info, int dev,
                        cudaStream_t q, float* out = nullptr, bool copy_back = true) {
  const int nb = int(w / kBlock);
  const size_t vbytes = size_t(w) * size_t(w) * sizeof(float);
  const size_t fbytes = kDiagFlags * sizeof(int) + 256;
  const size_t xbytes = size_t(m - w) * size_t(w) * sizeof(float);
  char* base = static_cast<char*>(panel_scratch(dev, vbytes + fbytes + xbytes));
  if (base == nullptr) return CHOL_ERR_WORKSPACE;
  float* V = reinterpret_cast<float*>(base);
  int* flags = reinterpret_cast<int*>(base + vbytes);
  unsigned* ticket = reinterpret_cast<unsigned*>(flags + kDiagFlags);
  float* scratch_x = reinterpret_cast<float*>(base + vbytes + fbytes);
  float* X = out != nullptr ? out + w * w : scratch_x;
  if (cudaMemsetAsync(V, 0, vbytes + fbytes, q) != cudaSuccess) return CHOL_ERR_LAUNCH;
  int st = launch_diag_block(L, 0, ld, V, 0, w, nb, m > w, flags, ticket, 1, info, 0, 1, q);
  if (st) return st;
  if (out != nullptr &&
      cudaMemcpy2DAsync(out, size_t(w) * sizeof(float), L, size_t(ld) * sizeof(float),
                        size_t(w) * sizeof(float), size_t(w), cudaMemcpyDeviceToDevice,
                        q) != cudaSuccess)
    return CHOL_ERR_LAUNCH;
  if (m == w) return CHOL_OK;
  GemmArgs x{};
  x.C = X;
  x.ldc = w;
  x.P = L + w * ld;
  x.ldp = ld;
  x.Q = V;
  x.ldq = w;
  x.m = m - w;
  x.ncols = w;
  x.K = w;
  x.alpha = 1.f;
  x.beta = 0.f;
  x.batch = 1;
  if ((st = launch_gemm(x, q, true))) return st;
  if (!copy_back) return CHOL_OK;  // the caller copies out's rows w.. into L itself
  return launch_tf32_lo(X, w, scratch_x, w, m - w, w, 1, 0, 0, q, L + w * ld, ld, 0);
}

}  // namespace

int prepare_device_checked(int dev) { return prepare_device(dev); }
int check_potrf_args(const float* A, float* L, int64_t batch, int64_t n) {
  return check_common(A, L, batch, n);
}
size_t workspace_min_bytes(int64_t batch, int64_t n) {
  return (batch <= 0 || n <= 0) ? 0 : blocked_workspace_min(batch, n);
}
int potrf_with_workspace(const float* A, float* L, int64_t batch, int64_t n, int* info, void* ws,
                         size_t ws_bytes, cudaStream_t q) {
  return potrf_impl(A, L, batch, n, info, ws, ws_bytes, q);
}

int prepare_kernels(int /*device*/) {
  return (prepare_tc() == cudaSuccess && prepare_blocked() == cudaSuccess &&
          prepare_mid() == cudaSuccess)
             ? CHOL_OK
             : CHOL_ERR_DEVICE;
}

uint64_t g_wait_limit_ns = 2000000000ull;
uint64_t wait_limit_ns() { return g_wait_limit_ns; }

thread_local int t_gemm_ctas = 0;
int gemm_cta_cap() { return t_gemm_ctas; }

int g_gemm_engine = 0;

int launch_gemm(const GemmArgs& g, cudaStream_t q, bool pdl) {
  if (g.m <= 0 || g.ncols <= 0) return CHOL_OK;
  const bool tc = tc_supported(g);
  if (g_gemm_engine == 2 && !tc) return CHOL_ERR_UNSUPPORTED;
  if (g_gemm_engine != 1 && tc) return launch_gemm_tc(g, q, pdl, nullptr);
  return launch_gemm_simt(g, q, pdl);
}

}  // namespace chol

using namespace chol;

extern "C" {

int chol_version(void) { return 100; }

const char* chol_strerror(int status) {
  switch (status) {
    case CHOL_OK: return "success";
    case CHOL_ERR_INVALID_ARG: return "invalid argument (shape, null pointer or partial aliasing)";
    case CHOL_ERR_LAUNCH: return "kernel launch failed";
    case CHOL_ERR_NOT_SPD: return "matrix is not positive definite (info > 0)";
    case CHOL_ERR_WAIT_TIMEOUT: return "bounded device-side wait timed out";
    case CHOL_ERR_WORKSPACE: return "workspace missing or too small";
    case CHOL_ERR_DEVICE: return "no usable sm_100 CUDA device";
    case CHOL_ERR_UNSUPPORTED: return "size not supported by this build";
    case CHOL_ERR_SCRATCH_LIMIT:
      return "problem needs more scratch than the fixed buffer of the no-allocation entry point";
    default: return "unknown status";
  }
}

int chol_prepare(int device) { return prepare_device(device); }

size_t chol_workspace_bytes(int64_t batch, int64_t n) {
  if (batch <= 0 || n <= 0) return 0;
  return blocked_workspace(batch, n);
}

int chol_potrf_batched_ws_f32(const float* A, float* L, int64_t batch, int64_t n, int* info,
                              void* workspace, size_t workspace_bytes, void* queue) {
  int st = check_common(A, L, batch, n);
  if (st || batch == 0 || n == 0) return st;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return CHOL_ERR_DEVICE;
  if ((st = prepare_device(dev))) return st;
  return potrf_impl(A, L, batch, n, info, workspace, workspace_bytes,
                    static_cast<cudaStream_t>(queue));
}

int chol_potrf_batched_f32(const float* A, float* L, int64_t batch, int64_t n, int* info,
                           void* queue) {
  int st = check_common(A, L, batch, n);
  if (st || batch == 0 || n == 0) return st;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return CHOL_ERR_DEVICE;
  if ((st = prepare_device(dev))) return st;
  const size_t need = blocked_workspace(batch, n);
  void* ws = nullptr;
  if (need) {
    DeviceState* ds = device_state(dev);
    std::lock_guard<std::mutex> lock(ds->ws_mu);
    if (ds->ws_bytes < need) {
      // Growing: the old buffer may still be read by queued work, so wait for the device.
      if (ds->ws) {
        cudaDeviceSynchronize();
        cudaFree(ds->ws);
        ds->ws = nullptr;
        ds->ws_bytes = 0;
      }
      if (cudaMalloc(&ds->ws, need) != cudaSuccess) return CHOL_ERR_WORKSPACE;
      ds->ws_bytes = need;
    }
    ws = ds->ws;
  }
  return potrf_impl(A, L, batch, n, info, ws, need, static_cast<cudaStream_t>(queue));
}

int64_t chol_launch_count(int64_t batch, int64_t n) {
  if (batch <= 0 || n <= 0) return 0;
  if (n <= 64 || use_mid(batch, n)) return 1;
  return blocked_launches(batch, n);
}

int chol_set_option(int option, int value) {
  if (option == CHOL_OPT_GEMM_ENGINE) {
    if (value < 0 || value > 2) return CHOL_ERR_INVALID_ARG;
    g_gemm_engine = value;
    return CHOL_OK;
  }
  if (option == CHOL_OPT_OUTER_WIDTH) {
    if (value < 0 || value % 64) return CHOL_ERR_INVALID_ARG;
    g_outer_width = value;
    return CHOL_OK;
  }
  if (option == CHOL_OPT_LOOKAHEAD) {
    if (value < -1 || value > 1) return CHOL_ERR_INVALID_ARG;
    g_lookahead = value;
    return CHOL_OK;
  }
  if (option == CHOL_OPT_CHAIN_SMS) {
    if (value < 1 || value > 120) return CHOL_ERR_INVALID_ARG;
    g_chain_sms = value;
    return CHOL_OK;
  }
  if (option == CHOL_OPT_MID_KERNEL) {
    if (value < 0 || value > 1) return CHOL_ERR_INVALID_ARG;
    g_mid_kernel = value;
    return CHOL_OK;
  }
  if (option == CHOL_OPT_OVERLAP_CALLS) {
    if (value < 0 || value > 1) return CHOL_ERR_INVALID_ARG;
    set_overlap_small(value);
    return CHOL_OK;
  }
  if (option == CHOL_OPT_PANEL_INVERSE) {
    if (value < 0 || value > 2) return CHOL_ERR_INVALID_ARG;
    g_panel_inverse = value;
    return CHOL_OK;
  }
  if (option == CHOL_OPT_CHAIN_WIDTH) {
    if (value != 64 && value != 128) return CHOL_ERR_INVALID_ARG;
    g_chain_width = value;
    return CHOL_OK;
  }
  if (option == CHOL_OPT_GEMM_CTAS) {
    if (value < 0 || value > 4096) return CHOL_ERR_INVALID_ARG;
    t_gemm_ctas = value;
    return CHOL_OK;
  }
  if (option == CHOL_OPT_WAIT_LIMIT_US) {
    if (value < 0 || value > 60000000) return CHOL_ERR_INVALID_ARG;
    g_wait_limit_ns = value == 0 ? 2000000000ull : uint64_t(value) * 1000ull;
    return CHOL_OK;
  }
  return CHOL_ERR_INVALID_ARG;  // includes option 2, the fused panel step of earlier versions
}

int chol_overlap_stats(int64_t* started_early, int64_t* withdrawn) {
  int dev = 0, st;
  if (cudaGetDevice(&dev) != cudaSuccess) return CHOL_ERR_DEVICE;
  if ((st = prepare_device(dev))) return st;
  return overlap_stats(started_early, withdrawn);
}

int chol_test_flag_wait(int* words, int value, void* queue) {
  if (words == nullptr || (reinterpret_cast<uintptr_t>(words) & 3)) return CHOL_ERR_INVALID_ARG;
  int dev = 0, st;
  if (cudaGetDevice(&dev) != cudaSuccess) return CHOL_ERR_DEVICE;
  if ((st = prepare_device(dev))) return st;
  return launch_flag_wait(words, value, static_cast<cudaStream_t>(queue));
}

int chol_status_check(void* queue) {
  if (cudaStreamSynchronize(static_cast<cudaStream_t>(queue)) != cudaSuccess)
    return CHOL_ERR_DEVICE;
  int v = 0;
  int st = read_and_clear_status(&v);
  if (st) return st;
  return v ? v : CHOL_OK;
}

int chol_info_check(const int* info, int64_t batch, void* queue, int64_t* first_bad) {
  if (first_bad) *first_bad = -1;
  if (batch <= 0) return CHOL_OK;
  if (info == nullptr) return CHOL_ERR_INVALID_ARG;
  std::vector<int> h(static_cast<size_t>(batch));
  cudaStream_t q = static_cast<cudaStream_t>(queue);
  if (cudaMemcpyAsync(h.data(), info, size_t(batch) * sizeof(int), cudaMemcpyDeviceToHost, q) !=
      cudaSuccess)
    return CHOL_ERR_DEVICE;
  if (cudaStreamSynchronize(q) != cudaSuccess) return CHOL_ERR_DEVICE;
  for (int64_t m = 0; m < batch; ++m) {
    if (h[size_t(m)] > 0) {
      if (first_bad) *first_bad = m;
      return CHOL_ERR_NOT_SPD;
    }
  }
  return CHOL_OK;
}

int chol_block_potrf_f32(float* L, int64_t batch, int64_t stride, int64_t ld, int64_t k,
                         int64_t kb, float* Tinv, int* info, void* queue) {
  if (L == nullptr || batch < 0 || kb < 1 || kb > kBlock || k < 0 || ld < k + kb)
    return CHOL_ERR_INVALID_ARG;
  if (batch == 0) return CHOL_OK;
  int dev = 0, st;
  if (cudaGetDevice(&dev) != cudaSuccess) return CHOL_ERR_DEVICE;
  if ((st = prepare_device(dev))) return st;
  return launch_potrf_block(L, stride, ld, L, stride, ld, batch, k, kb, Tinv, info,
                            static_cast<cudaStream_t>(queue), true);
}

int chol_gemm_nt_f32(float* C, int64_t batch, int64_t cstride, int64_t ldc, int64_t m,
                     int64_t ncols, int64_t K, const float* P, int64_t pstride, int64_t ldp,
                     const float* Q, int64_t qstride, int64_t ldq, float alpha, float beta,
                     int64_t diag_offset, int lower_only, void* queue) {
  if (batch < 0 || m < 0 || ncols < 0 || K < 0) return CHOL_ERR_INVALID_ARG;
  if (batch == 0 || m == 0 || ncols == 0) return CHOL_OK;
  if (C == nullptr || (K > 0 && (P == nullptr || Q == nullptr))) return CHOL_ERR_INVALID_ARG;
  if (ldc < ncols || (K > 0 && (ldp < K || ldq < K))) return CHOL_ERR_INVALID_ARG;
  if (C == P && (beta != 0.f || ncols > 64)) return CHOL_ERR_INVALID_ARG;
  int dev = 0, st;
  if (cudaGetDevice(&dev) != cudaSuccess) return CHOL_ERR_DEVICE;
  if ((st = prepare_device(dev))) return st;
  GemmArgs g{};
  g.C = C;
  g.cstride = cstride;
  g.ldc = ldc;
  g.P = P;
  g.pstride = pstride;
  g.ldp = ldp;
  g.Q = Q;
  g.qstride = qstride;
  g.ldq = ldq;
  g.m = m;
  g.ncols = ncols;
  g.K = K;
  g.alpha = alpha;
  g.beta = beta;
  g.diag_offset = diag_offset;
  g.lower_only = lower_only;
  g.batch = batch;
  return launch_gemm(g, static_cast<cudaStream_t>(queue), true);
}

int chol_panel_potrf_f32(float* L, int64_t ld, int64_t m, int64_t w, float* Tinv, int* info,
                         void* queue) {
  if (L == nullptr || Tinv == nullptr || m < 0 || w < 0 || w > m || ld < w)
    return CHOL_ERR_INVALID_ARG;
  if (m == 0 || w == 0) return CHOL_OK;
  int dev = 0, st;
  if (cudaGetDevice(&dev) != cudaSuccess) return CHOL_ERR_DEVICE;
  if ((st = prepare_device(dev))) return st;
  cudaStream_t q = static_cast<cudaStream_t>(queue);
  if (g_panel_inverse == 1 && g_gemm_engine != 1 && w % kBlock == 0 && w <= 16 * kBlock &&
      ld % 4 == 0 && (reinterpret_cast<uintptr_t>(L) & 15) == 0)
    return panel_potrf_inverse(L, ld, m, w, info, dev, q);
  for (int64_t k = 0; k < w; k += kBlock) {
    const int64_t kb = (w - k) < kBlock ? (w - k) : kBlock;
    if (k > 0) {
      GemmArgs u{};
      u.C = L + k * ld + k;
      u.ldc = ld;
      u.P = L + k * ld;
      u.ldp = ld;
      u.Q = u.P;
      u.ldq = ld;
      u.m = m - k;
      u.ncols = kb;
      u.K = k;
      u.alpha = -1.f;
      u.beta = 1.f;
      u.lower_only = 1;
      u.batch = 1;
      if ((st = launch_gemm(u, q, true))) return st;
    }
    if ((st = launch_potrf_block(L, 0, ld, L, 0, ld, 1, k, kb, Tinv, info, q, true))) return st;
    if (m - k - kb <= 0) continue;
    GemmArgs x{};
    x.C = L + (k + kb) * ld + k;
    x.ldc = ld;
    x.P = x.C;
    x.ldp = ld;
    x.Q = Tinv;
    x.ldq = kBlock;
    x.m = m - k - kb;
    x.ncols = kb;
    x.K = kb;
    x.alpha = 1.f;
    x.beta = 0.f;
    x.batch = 1;
    if ((st = launch_gemm(x, q, true))) return st;
  }
  return CHOL_OK;
}

int chol_diag_potrf_inv_f32(float* L, int64_t ld, int64_t w, float* V, int* info, void* queue) {
  if (L == nullptr || V == nullptr || w < 0 || ld < w) return CHOL_ERR_INVALID_ARG;
  if (w == 0) return CHOL_OK;
  if (w % kBlock || w > 16 * kBlock || ld % 4 || (reinterpret_cast<uintptr_t>(L) & 15) ||
      (reinterpret_cast<uintptr_t>(V) & 15))
    return CHOL_ERR_UNSUPPORTED;
  const uintptr_t v0 = reinterpret_cast<uintptr_t>(V), v1 = v0 + uintptr_t(w * w) * 4;
  const uintptr_t l0 = reinterpret_cast<uintptr_t>(L);
  if (v0 < l0 + uintptr_t((w - 1) * ld + w) * 4 && l0 < v1) return CHOL_ERR_INVALID_ARG;
  int dev = 0, st;
  if (cudaGetDevice(&dev) != cudaSuccess) return CHOL_ERR_DEVICE;
  if ((st = prepare_device(dev))) return st;
  cudaStream_t q = static_cast<cudaStream_t>(queue);
  const size_t fbytes = kDiagFlags * sizeof(int) + 256;
  char* base = static_cast<char*>(panel_scratch(dev, fbytes));
  if (base == nullptr) return CHOL_ERR_WORKSPACE;
  int* flags = reinterpret_cast<int*>(base);
  unsigned* ticket = reinterpret_cast<unsigned*>(flags + kDiagFlags);
  if (cudaMemsetAsync(base, 0, fbytes, q) != cudaSuccess ||
      cudaMemsetAsync(V, 0, size_t(w) * size_t(w) * sizeof(float), q) != cudaSuccess)
    return CHOL_ERR_LAUNCH;
  return launch_diag_block(L, 0, ld, V, 0, w, int(w / kBlock), true, flags, ticket, 1, info, 0,
                           1, q);
}

int chol_panel_potrf_out_f32(float* L, int64_t ld, int64_t m, int64_t w, float* out, int flags,
                             int* info, void* queue) {
  if (flags & ~CHOL_PANEL_OUT_ONLY) return CHOL_ERR_INVALID_ARG;
  if (L == nullptr || out == nullptr || m < 0 || w < 0 || w > m || ld < w)
    return CHOL_ERR_INVALID_ARG;
  if (m == 0 || w == 0) return CHOL_OK;
  if (w % kBlock || w > 16 * kBlock || ld % 4 || (reinterpret_cast<uintptr_t>(L) & 15) ||
      (reinterpret_cast<uintptr_t>(out) & 15) || g_gemm_engine == 1)
    return CHOL_ERR_UNSUPPORTED;
  const uintptr_t lo = reinterpret_cast<uintptr_t>(out), hi = lo + uintptr_t(m * w) * 4;
  const uintptr_t l0 = reinterpret_cast<uintptr_t>(L);
  if (lo < l0 + uintptr_t((m - 1) * ld + w) * 4 && l0 < hi) return CHOL_ERR_INVALID_ARG;
  int dev = 0, st;
  if (cudaGetDevice(&dev) != cudaSuccess) return CHOL_ERR_DEVICE;
  if ((st = prepare_device(dev))) return st;
  return panel_potrf_inverse(L, ld, m, w, info, dev, static_cast<cudaStream_t>(queue), out,
                             (flags & CHOL_PANEL_OUT_ONLY) == 0);
}

int chol_gemm_nt_cyclic_f32(float* C, int64_t ldc, int64_t m, int64_t ncols, int64_t K,
                            const float* P, int64_t ldp, const float* Q, int64_t ldq, float alpha,
                            float beta, int64_t diag_offset, int lower_only, int64_t col_block,
                            int64_t col_stride, void* queue) {
  if (m < 0 || ncols < 0 || K < 0) return CHOL_ERR_INVALID_ARG;
  if (m == 0 || ncols == 0) return CHOL_OK;
  if (C == nullptr || P == nullptr || Q == nullptr || ldc < ncols || ldp < K || ldq < K)
    return CHOL_ERR_INVALID_ARG;
  if (col_block != 256 || col_stride < col_block || col_stride % col_block)
    return CHOL_ERR_UNSUPPORTED;
  int dev = 0, st;
  if (cudaGetDevice(&dev) != cudaSuccess) return CHOL_ERR_DEVICE;
  if ((st = prepare_device(dev))) return st;
  GemmArgs g{};
  g.C = C;
  g.ldc = ldc;
  g.P = P;
  g.ldp = ldp;
  g.Q = Q;
  g.ldq = ldq;
  g.m = m;
  g.ncols = ncols;
  g.K = K;
  g.alpha = alpha;
  g.beta = beta;
  g.diag_offset = diag_offset;
  g.lower_only = lower_only;
  g.batch = 1;
  g.cmap_block = col_block;
  g.cmap_stride = col_stride;
  if (!tc_supported(g)) return CHOL_ERR_UNSUPPORTED;
  cudaStream_t q = static_cast<cudaStream_t>(queue);
  // Several column blocks: each row tile of P feeds many output tiles, so its low TF32 parts
  // are computed once (cached scratch) and loaded by TMA instead of split in shared memory
  // for every tile. One block (the look-ahead update): each row tile is used once, and the
  // separate pass costs more than it saves (m = 32512, K = 256: 13 + 53 us against 44 us
  // for the in-kernel split).
  if (P == Q && ldp == ldq && K % 4 == 0 && g_gemm_engine != 1 && ncols > col_block) {
    static PanelScratch lo_cache[64];
    float* lo = dev < 64 ? static_cast<float*>(cached_scratch(lo_cache[dev],
                                                              size_t(m) * size_t(K) * 4))
                         : nullptr;
    if (lo != nullptr) {
      if ((st = launch_tf32_lo(P, ldp, lo, K, m, K, 1, 0, 0, q))) return st;
      st = launch_gemm_tc_prelo(g, lo, K, q, true);
      if (st != CHOL_ERR_UNSUPPORTED) return st;
    }
  }
  return launch_gemm_tc(g, q, true, nullptr);
}

}  // extern "C"
