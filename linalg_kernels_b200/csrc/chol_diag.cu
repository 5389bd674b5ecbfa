// chol_diag.cu — one launch factors an outer panel's diagonal block and inverts it.
//
// The KB x KB diagonal block (KB = 64 * nb, nb <= 16) of an outer panel is cut into 64 x 64
// tiles. Every CTA takes one task from a ticket counter and runs it as soon as the tiles it
// reads are published:
//   D(0)      tile (0, 0): factor A_00 = L_00 L_00^T, T_0 = inv(L_00).
//   O(i,j)    tile (i, j), i > j:  L_ij = (A_ij - sum_{p<j} L_ip L_jp^T) T_j^T. For i = j + 1
//             the same CTA then factors the next diagonal tile,
//               A_ii - sum_{p<=j} L_ip L_ip^T = L_ii L_ii^T,  T_i = inv(L_ii)
//             reusing the L_ip tiles it already staged (this is the critical path: the task
//             that produces L_{j+1,j} goes straight on to the factor that needs it).
//   W(i,j)    block (i, j) of V = inv(L11), i > j:  V_ij = -T_i sum_{p=j}^{i-1} L_ip V_pj
//             (V_jj = T_j), i.e. block forward substitution down column block j.
// L_jj goes to L and T_j to V's diagonal block.
// Tasks are numbered so that every task reads only tasks with smaller numbers (column by
// column: D(0), O(1..nb-1, 0), O(2..nb-1, 1), ...; then the W tasks row by row) and matrices
// of a batch interleave. A CTA learns its task from an atomic ticket, so every task it
// waits on is held by a CTA that is already running or done: the waits always end, whatever
// the grid size or residency. A finished tile is published by a release store of the
// launch's epoch into its flag; readers poll with acquire loads (bounded by a time limit
// that records CHOL_ERR_WAIT_TIMEOUT in the status word and lets every waiter return) and
// read tiles through L2 (ld.global.cg).
//
// Factors: the register-resident warp factor (warp_potrf_rows) and the blocked inverse
// (inverse_blocked64) are fully unrolled, several thousand instructions that a task runs
// once. The diagonal tasks after D(0) run both once on scratch data while they wait for
// their inputs, so the real run starts with this SM's instruction cache warm.
//
// This replaces the per-step chain of the blocked schedule for the block — 3 launches per
// 64 columns (left-looking GEMM, potrf_block, solve GEMM), each bound by launch and pipeline
// latency — with one launch whose critical path is the chain of 64 x 64 factors. All
// arithmetic is FP32 FMA (no TF32 anywhere in the block). The reference factors the same
// block with its factor/solve/update kernel sequence (cholesky/cholesky.py:5440-5690).
#include "chol_tc_ptx.cuh"
#include "chol_warp.cuh"

namespace chol {
namespace {

constexpr int kDT = 256;   // threads: a 16 x 16 grid of 4 x 4 output blocks
constexpr int kDLD = 68;   // shared tile row stride (floats)
constexpr int kFlagO = 256, kFlagW = 512;
// Flag slot 255 of the first matrix (no task uses slots 16..255) is the launch's abort word.
constexpr int kFlagAbort = 255;

struct DiagArgs {
  float* L;            // (0, 0) of the diagonal block of matrix 0
  int64_t mstride, ld;
  float* V;            // V = inv(L11), KB x KB per matrix (want_v), else nb 64 x 64 T blocks
  int64_t vstride, ldv;
  int* flags;          // kDiagFlags per matrix, zero before the call's first launch
  unsigned* ticket;    // this launch's ticket counter, zero before the launch
  int* info;
  int64_t col0;        // global index of the block's first column (for info)
  int64_t batch;
  int nb, want_v, epoch;
  int* status;
  uint64_t limit_ns;   // bound of every flag wait
};

__device__ __forceinline__ int ld_acquire(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release(int* p, int v) {
  asm volatile("st.release.gpu.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// All threads: true once *flag == epoch. Thread 0 polls; false (for every thread) when the
// time limit passes or another CTA of the same launch has already given up. A CTA that gives
// up records CHOL_ERR_WAIT_TIMEOUT in the library's status word (read and cleared by
// chol_status_check) and writes its launch's epoch into the launch's abort word, so the
// other waiters of this launch return too. Other launches do not look at either word: an
// earlier failure does not make later calls drop their work.
__device__ __forceinline__ bool cta_wait(const int* flag, int epoch, int* status, int* abort,
                                         uint64_t limit_ns) {
  int ok = 1;
  if (threadIdx.x == 0 && ld_acquire(flag) != epoch) {
    const uint64_t t0 = tcx::global_ns();
    for (;;) {
      __nanosleep(32);
      if (ld_acquire(flag) == epoch) break;
      if (*reinterpret_cast<volatile int*>(abort) == epoch) {
        ok = 0;
        break;
      }
      if (tcx::global_ns() - t0 > limit_ns) {
        atomicExch(status, CHOL_ERR_WAIT_TIMEOUT);
        atomicExch(abort, epoch);
        ok = 0;
        break;
      }
    }
  }
  return __syncthreads_and(ok) != 0;
}

// Xs[k][r] = X[r][k] for the 64 x 64 tile X (row stride ldx), read through L2.
__device__ __forceinline__ void stage_t(float* Xs, const float* X, int64_t ldx) {
  const int t = threadIdx.x;
  const int r = t & 63, c0 = (t >> 6) * 4;
  float4 v[4];
#pragma unroll
  for (int it = 0; it < 4; ++it)
    v[it] = __ldcg(reinterpret_cast<const float4*>(X + r * ldx + c0 + 16 * it));
#pragma unroll
  for (int it = 0; it < 4; ++it) {
    const int c = c0 + 16 * it;
    Xs[(c + 0) * kDLD + r] = v[it].x;
    Xs[(c + 1) * kDLD + r] = v[it].y;
    Xs[(c + 2) * kDLD + r] = v[it].z;
    Xs[(c + 3) * kDLD + r] = v[it].w;
  }
}
// Ys[k][c] = Y[k][c], read through L2.
__device__ __forceinline__ void stage_n(float* Ys, const float* Y, int64_t ldy) {
  const int t = threadIdx.x;
  const int k = t >> 4, c = (t & 15) * 4;
  float4 v[4];
#pragma unroll
  for (int it = 0; it < 4; ++it)
    v[it] = __ldcg(reinterpret_cast<const float4*>(Y + (k + 16 * it) * ldy + c));
#pragma unroll
  for (int it = 0; it < 4; ++it)
    *reinterpret_cast<float4*>(Ys + (k + 16 * it) * kDLD + c) = v[it];
}

// acc[i] (row 4tr+i; .x/.y of [i][0] = columns 4tc, 4tc+1, of [i][1] = 4tc+2, 4tc+3)
//   += sum_k Xs[k][4tr+i] * Ys[k][4tc+j]
__device__ __forceinline__ void tile_fma(float2 (&acc)[4][2], const float* Xs, const float* Ys,
                                         int tr, int tc) {
#pragma unroll 8
  for (int k = 0; k < 64; ++k) {
    const float4 a = *reinterpret_cast<const float4*>(Xs + k * kDLD + 4 * tr);
    const float4 b = *reinterpret_cast<const float4*>(Ys + k * kDLD + 4 * tc);
    const float2 b01 = make_float2(b.x, b.y), b23 = make_float2(b.z, b.w);
    acc[0][0] = ffma2(make_float2(a.x, a.x), b01, acc[0][0]);
    acc[0][1] = ffma2(make_float2(a.x, a.x), b23, acc[0][1]);
    acc[1][0] = ffma2(make_float2(a.y, a.y), b01, acc[1][0]);
    acc[1][1] = ffma2(make_float2(a.y, a.y), b23, acc[1][1]);
    acc[2][0] = ffma2(make_float2(a.z, a.z), b01, acc[2][0]);
    acc[2][1] = ffma2(make_float2(a.z, a.z), b23, acc[2][1]);
    acc[3][0] = ffma2(make_float2(a.w, a.w), b01, acc[3][0]);
    acc[3][1] = ffma2(make_float2(a.w, a.w), b23, acc[3][1]);
  }
}

// This thread's 4 x 4 block of a 64 x 64 global tile (row stride ld).
__device__ __forceinline__ void load_block(float4 (&v)[4], const float* X, int64_t ld, int tr,
                                           int tc) {
#pragma unroll
  for (int i = 0; i < 4; ++i)
    v[i] = __ldcg(reinterpret_cast<const float4*>(X + (4 * tr + i) * ld + 4 * tc));
}
__device__ __forceinline__ void store_block(float* X, int64_t ld, const float2 (&acc)[4][2],
                                            float sign, int tr, int tc) {
#pragma unroll
  for (int i = 0; i < 4; ++i)
    *reinterpret_cast<float4*>(X + (4 * tr + i) * ld + 4 * tc) =
        make_float4(sign * acc[i][0].x, sign * acc[i][0].y, sign * acc[i][1].x,
                    sign * acc[i][1].y);
}

__device__ __forceinline__ void zero(float2 (&acc)[4][2]) {
#pragma unroll
  for (int i = 0; i < 4; ++i) acc[i][0] = acc[i][1] = make_float2(0.f, 0.f);
}

// Task number -> (type, i, j): 0 = D(0), 1 = O(i, j) (with the factor of tile (i, i) when
// i == j + 1), 2 = W(i, j).
__device__ __forceinline__ void decode_task(int t, int nb, int& type, int& i, int& j) {
  if (t < nb) {  // column 0: D(0), O(1, 0), ..., O(nb-1, 0)
    j = 0;
    i = t;
    type = (t == 0) ? 0 : 1;
    return;
  }
  t -= nb;
  const int nO = nb * (nb - 1) / 2 - (nb - 1);  // O tasks of columns 1 .. nb-2
  if (t < nO) {
    j = 1;
    while (t >= nb - 1 - j) {
      t -= nb - 1 - j;
      ++j;
    }
    i = j + 1 + t;
    type = 1;
    return;
  }
  t -= nO;
  i = 1;
  while (t >= i) {
    t -= i;
    ++i;
  }
  j = t;
  type = 2;
}

// S = this thread's 4 x 4 block of (A - acc), lower part only (zeros above the diagonal).
__device__ __forceinline__ void put_lower(float* S, const float4 (&av)[4],
                                          const float2 (&acc)[4][2], int tr, int tc) {
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    const int r = 4 * tr + u, c = 4 * tc;
    float4 o = make_float4(av[u].x - acc[u][0].x, av[u].y - acc[u][0].y,
                           av[u].z - acc[u][1].x, av[u].w - acc[u][1].y);
    if (c + 0 > r) o.x = 0.f;
    if (c + 1 > r) o.y = 0.f;
    if (c + 2 > r) o.z = 0.f;
    if (c + 3 > r) o.w = 0.f;
    *reinterpret_cast<float4*>(S + r * kDLD + c) = o;
  }
}
// Xs[c][r] = this thread's 4 x 4 block of M (transposed store).
__device__ __forceinline__ void put_transposed(float* Xs, const float (&m)[4][4], int tr,
                                               int tc) {
#pragma unroll
  for (int v = 0; v < 4; ++v)
    *reinterpret_cast<float4*>(Xs + (4 * tc + v) * kDLD + 4 * tr) =
        make_float4(m[0][v], m[1][v], m[2][v], m[3][v]);
}
__device__ __forceinline__ void to_array(float (&m)[4][4], const float2 (&acc)[4][2]) {
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    m[u][0] = acc[u][0].x;
    m[u][1] = acc[u][0].y;
    m[u][2] = acc[u][1].x;
    m[u][3] = acc[u][1].y;
  }
}

// The unrolled warp factor and the blocked inverse, each as ONE function: every call site
// (and the warm-up run) executes the same instructions, and their register needs stay apart
// from the task code around them.
__device__ __noinline__ int warp_factor64(float* S, float* col, float* rdiag, int lane) {
  return tile64_potrf<kDLD>(S, col, rdiag, lane);
}
// T = inv(L) for the factored 64 x 64 block in S as a 2 x 2 block inverse, all kDT threads:
//   T11 = inv(L11), T22 = inv(L22)      (32-row forward substitutions, side by side:
//                                        thread c < 64 computes column c of its block)
//   T21 = -T22 (L21 T11)                (two 32 x 32 x 32 products, 4 outputs per thread)
// Half the dependent chain of the column-by-column inverse. W: 32 x kDLD floats of scratch.
__device__ __noinline__ void inverse_blocked64(const float* S, const float* rdiag, float* Ts,
                                               float* W) {
  const int t = threadIdx.x;
  if (t < 64) {
    const int c = t, base = (t < 32) ? 0 : 32;  // column c of the diagonal block at base
    float x[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const float* rp = S + (base + i) * kDLD + base;
      float2 acc = make_float2(0.f, 0.f);
#pragma unroll
      for (int q = 0; q < i / 4; ++q) {
        const float4 v = *reinterpret_cast<const float4*>(rp + 4 * q);
        acc = ffma2(make_float2(v.x, v.y), make_float2(x[4 * q], x[4 * q + 1]), acc);
        acc = ffma2(make_float2(v.z, v.w), make_float2(x[4 * q + 2], x[4 * q + 3]), acc);
      }
      float sum = acc.x + acc.y;
#pragma unroll
      for (int m = (i / 4) * 4; m < i; ++m) sum = fmaf(rp[m], x[m], sum);
      const float ri = rdiag[base + i];
      const int cc = c - base;
      x[i] = (i == cc) ? ri : ((i < cc) ? 0.f : -ri * sum);
    }
#pragma unroll
    for (int i = 0; i < 32; ++i) Ts[(base + i) * kDLD + c] = x[i];
    if (base == 32) {  // the block above T22 is zero (T21, below T11, follows)
#pragma unroll
      for (int i = 0; i < 32; ++i) Ts[i * kDLD + c] = 0.f;
    }
  }
  __syncthreads();
  const int i = t >> 3, j0 = (t & 7) * 4;  // output row i, columns j0..j0+3 of a 32 x 32 block
  {
    // W = L21 T11 (T11 lower: k >= j)
    float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
    const float* lrow = S + (32 + i) * kDLD;
#pragma unroll 8
    for (int k = 0; k < 32; ++k) {
      const float a = lrow[k];
      const float4 b = *reinterpret_cast<const float4*>(Ts + k * kDLD + j0);
      o.x = fmaf(a, b.x, o.x);
      o.y = fmaf(a, b.y, o.y);
      o.z = fmaf(a, b.z, o.z);
      o.w = fmaf(a, b.w, o.w);
    }
    *reinterpret_cast<float4*>(W + i * kDLD + j0) = o;
  }
  __syncthreads();
  {
    // T21 = -T22 W (T22 lower: k <= i)
    float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
    const float* trow = Ts + (32 + i) * kDLD + 32;
#pragma unroll 8
    for (int k = 0; k < 32; ++k) {
      const float a = trow[k];
      const float4 b = *reinterpret_cast<const float4*>(W + k * kDLD + j0);
      o.x = fmaf(a, b.x, o.x);
      o.y = fmaf(a, b.y, o.y);
      o.z = fmaf(a, b.z, o.z);
      o.w = fmaf(a, b.w, o.w);
    }
    *reinterpret_cast<float4*>(Ts + (32 + i) * kDLD + j0) = make_float4(-o.x, -o.y, -o.z, -o.w);
  }
  __syncthreads();
}

// Publish: every thread's global stores, then the flag (release at GPU scope).
__device__ __forceinline__ void publish(int* flag, int epoch) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    st_release(flag, epoch);
  }
}

__global__ void __launch_bounds__(kDT, 1) diag_block_kernel(DiagArgs a) {
  __shared__ __align__(16) float Xs[64 * kDLD];
  __shared__ __align__(16) float Ys[64 * kDLD];
  __shared__ __align__(16) float Ws[32 * kDLD];  // scratch of the blocked inverse
  __shared__ __align__(16) float col[128];
  __shared__ float rdiag[64];
  __shared__ unsigned s_ticket;
  __shared__ int s_flag[1];
  griddep_wait();
  const int tid = threadIdx.x;
  if (tid == 0) s_ticket = atomicAdd(a.ticket, 1u);
  __syncthreads();
  griddep_launch();
  const int64_t tk = s_ticket;
  const int64_t task = tk / a.batch, mi = tk - task * a.batch;
  const int nb = a.nb;
  const int ntask = 1 + nb * (nb - 1) / 2 + (a.want_v ? nb * (nb - 1) / 2 : 0);
  if (task >= ntask) return;
  int type, i, j;
  decode_task(int(task), nb, type, i, j);

  float* Lm = a.L + mi * a.mstride;
  float* Vm = a.V + mi * a.vstride;
  int* F = a.flags + mi * kDiagFlags;
  int* abort_w = a.flags + kFlagAbort;
  const int ep = a.epoch;
  const int64_t ld = a.ld, ldv = a.ldv;
  auto tileL = [&](int bi, int bj) { return Lm + int64_t(bi) * 64 * ld + bj * 64; };
  auto tileV = [&](int bi, int bj) { return Vm + int64_t(bi) * 64 * ldv + bj * 64; };
  // T_d = inv(L_dd): V's diagonal block, or (without V) the d-th 64 x 64 slot of Vm
  const int64_t ldt = a.want_v ? ldv : 64;
  auto tileT = [&](int d) { return a.want_v ? tileV(d, d) : Vm + int64_t(d) * 64 * 64; };
  const int tr = tid >> 4, tc = tid & 15;

  float2 acc[4][2];
  zero(acc);
  int dtile = -1;  // diagonal tile this task factors after its main work
  if (type == 0) {
    // ---------------- D(0) ----------------
    float4 av[4];
    load_block(av, tileL(0, 0), ld, tr, tc);
    put_lower(Ys, av, acc, tr, tc);
    __syncthreads();
    dtile = 0;
  } else if (type == 1) {
    // ---------------- O(i, j) [+ factor of tile (i, i) when i == j + 1] ----------------
    const bool diag_next = (i == j + 1);
    float4 av[4], ad[4];
    load_block(av, tileL(i, j), ld, tr, tc);
    float2 accd[4][2];
    zero(accd);
    if (diag_next) {
      load_block(ad, tileL(i, i), ld, tr, tc);
      // warm this SM's instruction cache with the factor and inverse (results discarded)
      put_lower(Ys, ad, accd, tr, tc);
      __syncthreads();
      if (tid < 32) warp_factor64(Ys, col, rdiag, tid);
      __syncthreads();
      inverse_blocked64(Ys, rdiag, Xs, Ws);
    }
    for (int p = 0; p < j; ++p) {
      if (!cta_wait(&F[kFlagO + i * 16 + p], ep, a.status, abort_w, a.limit_ns)) return;
      if (!cta_wait(&F[kFlagO + j * 16 + p], ep, a.status, abort_w, a.limit_ns)) return;
      stage_t(Xs, tileL(i, p), ld);
      stage_t(Ys, tileL(j, p), ld);
      __syncthreads();
      tile_fma(acc, Xs, Ys, tr, tc);
      if (diag_next) tile_fma(accd, Xs, Xs, tr, tc);
      __syncthreads();
    }
    // C = A - acc, transposed into Xs for the solve X = C T_j^T
    {
      float m[4][4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        m[u][0] = av[u].x - acc[u][0].x;
        m[u][1] = av[u].y - acc[u][0].y;
        m[u][2] = av[u].z - acc[u][1].x;
        m[u][3] = av[u].w - acc[u][1].y;
      }
      put_transposed(Xs, m, tr, tc);
    }
    if (!cta_wait(&F[j], ep, a.status, abort_w, a.limit_ns)) return;
    stage_t(Ys, tileT(j), ldt);  // Ys[k][c] = T_j[c][k]
    __syncthreads();
    zero(acc);
    tile_fma(acc, Xs, Ys, tr, tc);
    store_block(tileL(i, j), ld, acc, 1.f, tr, tc);
    if (!diag_next) {
      publish(&F[kFlagO + i * 16 + j], ep);
    } else {
      __syncthreads();  // Xs and Ys are free
      float m[4][4];
      to_array(m, acc);
      put_transposed(Xs, m, tr, tc);  // Xs[k][r] = L_ij[r][k]
      publish(&F[kFlagO + i * 16 + j], ep);
      tile_fma(accd, Xs, Xs, tr, tc);
      put_lower(Ys, ad, accd, tr, tc);
      __syncthreads();
      dtile = i;
    }
  } else {
    // ---------------- W(i, j) ----------------
    for (int p = j; p < i; ++p) {
      if (!cta_wait(&F[kFlagO + i * 16 + p], ep, a.status, abort_w, a.limit_ns)) return;
      if (!cta_wait(p == j ? &F[j] : &F[kFlagW + p * 16 + j], ep, a.status, abort_w, a.limit_ns)) return;
      stage_t(Xs, tileL(i, p), ld);
      stage_n(Ys, tileV(p, j), ldv);
      __syncthreads();
      tile_fma(acc, Xs, Ys, tr, tc);
      __syncthreads();
    }
    // Ys = the sum (row-major), Xs[k][r] = T_i[r][k]
#pragma unroll
    for (int u = 0; u < 4; ++u)
      *reinterpret_cast<float4*>(Ys + (4 * tr + u) * kDLD + 4 * tc) =
          make_float4(acc[u][0].x, acc[u][0].y, acc[u][1].x, acc[u][1].y);
    if (!cta_wait(&F[i], ep, a.status, abort_w, a.limit_ns)) return;
    stage_t(Xs, tileV(i, i), ldv);
    __syncthreads();
    zero(acc);
    tile_fma(acc, Xs, Ys, tr, tc);
    store_block(tileV(i, j), ldv, acc, -1.f, tr, tc);
    publish(&F[kFlagW + i * 16 + j], ep);
  }
  if (dtile < 0) return;

  // ---- diagonal tile d (S in Ys, lower part): factor, T_d = inv(L_dd) into Xs, write
  // L_dd and T_d, record info, publish D(d) ----
  const int d = dtile;
  if (tid < 32) {
    const int w = warp_factor64(Ys, col, rdiag, tid);
    if (tid == 0) s_flag[0] = w;
  }
  __syncthreads();
  const int f = s_flag[0];
  inverse_blocked64(Ys, rdiag, Xs, Ws);
  float* dl = tileL(d, d);
  float* dv = tileT(d);
  for (int e = tid; e < 64 * 16; e += kDT) {
    const int r = e >> 4, c = (e & 15) * 4;
    *reinterpret_cast<float4*>(dl + r * ld + c) = *reinterpret_cast<const float4*>(Ys + r * kDLD + c);
    *reinterpret_cast<float4*>(dv + r * ldt + c) = *reinterpret_cast<const float4*>(Xs + r * kDLD + c);
  }
  if (tid == 0 && a.info != nullptr) {
    const int64_t c0 = a.col0 + int64_t(d) * 64;
    if (c0 == 0)
      a.info[mi] = f;
    else if (f && a.info[mi] == 0)
      a.info[mi] = int(c0) + f;
  }
  publish(&F[d], ep);
}

// One CTA waits with cta_wait for words[0] == value; words[1] is its abort word. For the
// test of the wait bound (chol_test_flag_wait): a flag that nothing sets.
__global__ void __launch_bounds__(64) flag_wait_kernel(int* words, int value, int* status,
                                                       uint64_t limit_ns) {
  cta_wait(words, value, status, words + 1, limit_ns);
}

}  // namespace

int launch_flag_wait(int* words, int value, cudaStream_t q) {
  int* status = device_status_ptr();
  if (status == nullptr) return CHOL_ERR_DEVICE;
  return status_from(launch_pdl(flag_wait_kernel, dim3(1), dim3(64), 0, q, false, words, value,
                                status, wait_limit_ns()));
}

int launch_diag_block(float* L11, int64_t mstride, int64_t ld, float* V, int64_t vstride,
                      int64_t ldv, int nb, bool want_v, int* flags, unsigned* ticket, int epoch,
                      int* info, int64_t col0, int64_t batch, cudaStream_t q) {
  if (nb < 1 || batch <= 0) return CHOL_OK;
  if (nb > 16 || ld % 4 || ldv % 4 || (want_v && ldv < 64 * nb) || epoch <= 0)
    return CHOL_ERR_UNSUPPORTED;
  if ((reinterpret_cast<uintptr_t>(L11) & 15) || (reinterpret_cast<uintptr_t>(V) & 15))
    return CHOL_ERR_UNSUPPORTED;
  DiagArgs a{};
  a.L = L11;
  a.mstride = mstride;
  a.ld = ld;
  a.V = V;
  a.vstride = vstride;
  a.ldv = ldv;
  a.flags = flags;
  a.ticket = ticket;
  a.info = info;
  a.col0 = col0;
  a.batch = batch;
  a.nb = nb;
  a.want_v = want_v ? 1 : 0;
  a.epoch = epoch;
  a.status = device_status_ptr();
  if (a.status == nullptr) return CHOL_ERR_DEVICE;
  a.limit_ns = wait_limit_ns();
  const int64_t ntask = 1 + int64_t(nb) * (nb - 1) / 2 + (want_v ? int64_t(nb) * (nb - 1) / 2 : 0);
  const int64_t ctas = ntask * batch;
  if (ctas > 0x7fffffffLL) return CHOL_ERR_UNSUPPORTED;
  return status_from(launch_pdl(diag_block_kernel, dim3(unsigned(ctas)), dim3(kDT), 0, q, true, a));
}

}  // namespace chol
