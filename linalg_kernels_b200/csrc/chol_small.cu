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
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstring>
#include <mutex>

#include "chol_warp.cuh"

namespace chol {

namespace {

// Warps per CTA and the CTAs per SM the launch bounds ask for. n = 64 uses 2-warp CTAs
// (72 KB of staging each, 2-3 per SM): back-to-back calls then find room on every SM for
// the next call's CTAs (9.8 us per call at b=1024 against 10.9 us with 4-warp CTAs).
template <int NP>
constexpr int small_warps() {
  return NP >= 64 ? 2 : 4;
}
template <int NP>
constexpr int small_min_ctas() {
  return NP <= 32 ? 3 : 2;
}

// Lanes per matrix for each padded size: 8 lanes x 4 rows for n <= 32 (four matrices per
// warp share each per-column step), a full warp x 2 rows for n = 64.
template <int NP>
constexpr int small_lpm() {
  return NP >= 64 ? 16 : (NP >= 32 ? 8 : (NP >= 16 ? 8 : NP));
}
template <int NP>
using SmallShape = WarpShape<NP, small_lpm<NP>()>;

// Staging of one matrix.
// Tensor-store layout (n = 32 and n = 64 with aligned rows): the factor is written back as
// 32 x 32 tiles in the 128-byte-swizzled layout of the tensor store (16-byte chunk k of
// tile row r at slot k ^ (r & 7)) and leaves with one tensor store per tile. At n = 64 the
// loads use the same layout (conflict-free row reads without padding) and only three tiles
// are kept: the one above the diagonal is never read and is stored from a zero tile shared
// by the CTA, 12 KiB per matrix against 17 KiB of padded rows, so 4 CTAs fit per SM and
// back-to-back calls overlap further (b=1024: 9.9 -> 9.1 us per call). At n = 32 the loads
// keep padded rows (measured faster there: more CTAs per SM did not pay).
// Otherwise: NP rows of stride NP + 4 floats, rounded to 1 KiB.
template <int NP, bool FULL>
constexpr bool small_quad() {  // tensor-store layout for the write-back and the stores
  return FULL && NP >= 32;
}
template <int NP, bool FULL>
constexpr bool small_quad_load() {  // ... and for the loads
  return FULL && NP == 64;
}
template <int NP, bool FULL>
constexpr int small_tile_floats() {
  return small_quad_load<NP, FULL>() ? 3 * 1024
                                     : ((NP * (NP + 4) * 4 + 1023) / 1024) * 1024 / 4;
}
template <int NP, bool FULL>
constexpr int small_zero_floats() {
  return small_quad_load<NP, FULL>() ? 1024 : 0;
}
template <int NP, bool FULL>
constexpr size_t small_smem_bytes() {
  return (size_t(small_zero_floats<NP, FULL>()) +
          size_t(small_warps<NP>()) * SmallShape<NP>::MPW *
              (size_t(small_tile_floats<NP, FULL>()) + SmallShape<NP>::COLS)) * 4 + 1024;
}
// Float offset of element (r, c) in the quadrant layout (c % 4 == 0 for a 16-byte chunk).
template <int NP>
__device__ __forceinline__ int quad_off(int r, int c) {
  const int t = (NP == 64 && r >= 32) ? ((c >= 32) ? 2 : 1) : 0;
  const int rr = r & 31, cc = c & 31;
  return t * 1024 + rr * 32 + ((((cc >> 2) ^ (rr & 7))) << 2) + (cc & 3);
}

// Per-queue CTA counters of the overlap check: for run-table entry e, call parity p and
// stripe s, g_run_ctas[e][p][s][0] counts the CTAs (blockIdx.x % kStripes == s) of that
// queue's small calls of parity p that have started, [1] those that have finished (both wrap
// modulo 2^32; only their difference is used). The stripes spread the atomics of a grid's
// CTAs over 32 addresses: on one address they serialise in L2 and delay every CTA's exit.
// g_overlap_stats[s][0] counts CTAs that started early, [s][1] CTAs whose early start the
// check withdrew.
constexpr int kRunEntries = 64;
constexpr int kStripes = 32;
__device__ __align__(16) unsigned g_run_ctas[kRunEntries][2][kStripes][2];
__device__ unsigned long long g_overlap_stats[kStripes][2];

// One 8-byte-aligned load of a {started, finished} counter pair (started in the low word).
__device__ __forceinline__ unsigned long long ld_relaxed_u64(const unsigned* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// FULL: n == NP and 16-byte aligned rows (vector path). Otherwise scalar loads with
// identity padding of rows/columns n..NP-1.
//
// early: where the kernel takes its programmatic-dependency wait (its grid always completes
// after its predecessor's), chosen by the host from the buffers of the calls that may still
// run on the queue (may_start_early):
//   0  at the start (this call reads what one of them writes, or nothing is known);
//   1  before the stores (it only writes what one of them reads or writes: the usual case
//      of back-to-back calls whose output tensors reuse one allocation);
//   2  at the end (all buffers disjoint).
// With 1 or 2 a call's loads and pivot chain run under the previous call's factor and stores.
//
// The host only knows the library's own calls. Work that someone else enqueued on the queue
// between two calls (a kernel that writes this call's input, e.g. the clone in
// custom_kernel(clone(data))) is invisible to it, and a kernel that reads before
// griddepcontrol.wait has no guarantee of seeing that work's writes. So each CTA checks on
// the device that its predecessor is the library's previous call on this queue, still
// running: prev_ctr counts the started and finished CTAs of that call and of the earlier
// calls of the same parity on the queue. Started != finished means one of them is still
// running, so this grid began before the previous call completed. Anything enqueued
// between the two (a kernel, copy or memset without programmatic serialisation) would have
// had to wait for that completion, and this grid for it, so nothing was. Calls on one queue
// complete in order (each takes griddepcontrol.wait), and the next call of the same parity
// cannot start before every CTA of this grid has passed this check, so only calls up to the
// predecessor contribute. Started == finished proves nothing: the CTA then takes the full
// wait and loads its input again (the first loads are issued while the counters are read,
// so the check adds no latency when it passes). my_ctr is this call's pair (nullptr: no
// counting, early must be 0).
template <int NP, bool FULL>
__global__ void __launch_bounds__(small_warps<NP>() * 32, small_min_ctas<NP>())
    small_potrf_kernel(const float* __restrict__ A, float* __restrict__ L, int64_t batch, int n,
                       int* __restrict__ info, const __grid_constant__ CUtensorMap out_map,
                       int early, const unsigned* prev_ctr, unsigned* my_ctr) {
  constexpr int LPM = SmallShape<NP>::LPM;
  constexpr int R = SmallShape<NP>::R;
  constexpr int MPW = SmallShape<NP>::MPW;
  constexpr int LDS = NP + 4;
  constexpr int TILE = small_tile_floats<NP, FULL>();
  constexpr bool QUAD = small_quad<NP, FULL>();       // write-back layout, tensor stores
  constexpr bool QLOAD = small_quad_load<NP, FULL>();  // load layout
  constexpr int ZF = small_zero_floats<NP, FULL>();
  extern __shared__ __align__(1024) float4 smem_raw[];
  float* zero_tile = reinterpret_cast<float*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                              ~uintptr_t(1023));
  float* smem = zero_tile + ZF;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (ZF > 0) {
    // the tile above the diagonal of every n = 64 output, stored by TMA from here
    for (int i = threadIdx.x; i < ZF; i += blockDim.x) zero_tile[i] = 0.f;
    fence_proxy_async_smem();
    __syncthreads();
  }
  const int grp = lane / LPM;
  const int gl = lane % LPM;
  float* stage = smem + size_t(warp) * MPW * TILE;
  float* col = smem + size_t(small_warps<NP>()) * MPW * TILE +
               size_t(warp * MPW + grp) * SmallShape<NP>::COLS;
  const int64_t mbase = (int64_t(blockIdx.x) * small_warps<NP>() + warp) * MPW;
  if (FULL) n = NP;

  // ---- overlap check, part 1: the predecessor's CTA counts, one 64-bit snapshot of each
  // stripe (warp 0, lane s reads stripe s). No static shared memory here: the dynamic buffer
  // is 1024-byte aligned, so even one static word costs 1 KiB per CTA, and at n = 64 that
  // is one CTA fewer per SM ----
  const int stripe = int(blockIdx.x % kStripes);
  unsigned long long pair = 0;
  if (my_ctr != nullptr && warp == 0) {
    if (early > 0) pair = ld_relaxed_u64(prev_ctr + 2 * lane);
    if (lane == 0) atomicAdd(my_ctr + 2 * stripe, 1u);  // this CTA has started
  }
  if (early == 0) {
    griddep_wait();
    griddep_launch();
  }

  // ---- load: lower triangle, coalesced, into this warp's staging tiles. With early > 0 the
  // loads are issued while the check's snapshot is in flight, and issued again after the
  // full wait if the check withdraws the early start ----
  // pass 0: the loads (speculative when early > 0); pass 1 only when the check withdrew the
  // early start (one copy of the load code either way)
#pragma unroll 1
  for (int pass = 0; pass < 2; ++pass) {
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
          if (c4 * 4 <= r)
            cp_async16(QLOAD ? st + quad_off<NP>(r, c4 * 4) : st + r * LDS + c4 * 4,
                       src + r * NP + c4 * 4);
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
      if (QLOAD) {
        if (NP == 64 && r < 32 && c >= 32) continue;  // no storage above the diagonal tile
        st[quad_off<NP>(r, c)] = (r == c) ? 1.f : 0.f;
      } else {
        st[r * LDS + c] = (r == c) ? 1.f : 0.f;
      }
    }
  }
  if (pass > 0 || early == 0) break;
  // ---- overlap check, part 2 (see above): started != finished proves the predecessor
  // was still running after this grid began. The dependents' trigger comes after the
  // decision, so no CTA of the next call can have touched the snapshot's counters ----
  const bool running =
      __syncthreads_or(warp == 0 && unsigned(pair) != unsigned(pair >> 32)) != 0;
  if (threadIdx.x == 0) atomicAdd(&g_overlap_stats[stripe][running ? 0 : 1], 1ull);
  griddep_launch();
  if (running) break;
  // withdrawn: the speculative loads may predate writes of work queued before this call
  cp_async_wait_all();
  __syncwarp();
  griddep_wait();
  early = 0;
  }
  cp_async_wait_all();
  __syncwarp();

  // ---- rows to registers (column pairs) ----
  uint64_t a[R][NP / 2];
  const float* mst = stage + grp * TILE;
#pragma unroll
  for (int s = 0; s < R; ++s) {
    const int row = s * LPM + gl;
    const float* rp = mst + row * LDS;
#pragma unroll
    for (int q = 0; q < (s + 1) * LPM / 4; ++q) {
      const ulonglong2 v = *reinterpret_cast<const ulonglong2*>(
          QLOAD ? mst + quad_off<NP>(row, 4 * q) : rp + 4 * q);
      a[s][2 * q] = v.x;
      a[s][2 * q + 1] = v.y;
    }
  }

  warp_potrf_rows<NP, LPM>(a, col, gl);
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
        const float lx = lo_of(a[s][2 * q]), ly = hi_of(a[s][2 * q]);
        const float hx = lo_of(a[s][2 * q + 1]), hy = hi_of(a[s][2 * q + 1]);
        v.x = (4 * q + 0 <= i) ? lx : 0.f;
        v.y = (4 * q + 1 <= i) ? ly : 0.f;
        v.z = (4 * q + 2 <= i) ? hx : 0.f;
        v.w = (4 * q + 3 <= i) ? hy : 0.f;
        if (4 * q <= i && i < 4 * q + 4) {
          const float dg = (i & 2) ? ((i & 1) ? hy : hx) : ((i & 1) ? ly : lx);
          bad[s] = !(dg > 0.f);
        }
      }
      if (QUAD) {
        // quadrant layout (no storage for the tile above the diagonal at n = 64)
        if (!(NP == 64 && i < 32 && q >= 8))
          *reinterpret_cast<float4*>(stage + grp * TILE + quad_off<NP>(i, 4 * q)) = v;
      } else {
        *reinterpret_cast<float4*>(rp + 4 * q) = v;
      }
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

  if (early == 1) griddep_wait();  // every buffer write below comes after the predecessors

  // ---- store. n = 32/64: one tensor store per 32-column half of each matrix from the
  // swizzled tiles; smaller full sizes: one bulk copy per row; otherwise 4-byte stores ----
  if (QUAD) {
    fence_proxy_async_smem();
    __syncwarp();
    if (lane < MPW) {
      const int64_t m = mbase + lane;
      if (m < batch) {
        // one 32 x 32 tensor store per tile (box 32 x 32); at n = 64 the tile above the
        // diagonal comes from the zero tile
        const float* base = stage + lane * TILE;
        auto store_tile = [&](int x, int y, const float* src) {
          asm volatile(
              "cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%1, %2, %3}], [%4];" ::
                  "l"(reinterpret_cast<uint64_t>(&out_map)),
              "r"(x), "r"(y), "r"(int(m)), "r"(smem_u32(src))
              : "memory");
        };
        store_tile(0, 0, base);
        if (NP == 64) {
          store_tile(0, 32, base + 1024);
          store_tile(32, 32, base + 2048);
          store_tile(32, 0, zero_tile);
        }
      }
      bulk_store_wait_read();
    }
  } else if (FULL) {
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
  if (early == 2) griddep_wait();
  // finished: counted when warp 0 is done (without waiting for the other warps, which can
  // only make a later check see this CTA as done early, the safe direction)
  if (my_ctr != nullptr && threadIdx.x == 0) atomicAdd(my_ctr + 2 * stripe + 1, 1u);
}

PFN_cuTensorMapEncodeTiled_v12000 g_small_enc = nullptr;

// Store map over L as (n, n, batch) with 32-column x NP-row boxes, 128-byte swizzle.
bool small_out_map(CUtensorMap* map, float* L, int64_t batch, int n, int np) {
  if (g_small_enc == nullptr) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult qr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &qr) !=
            cudaSuccess ||
        qr != cudaDriverEntryPointSuccess)
      return false;
    g_small_enc = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  }
  cuuint64_t dims[3] = {cuuint64_t(n), cuuint64_t(n), cuuint64_t(batch)};
  cuuint64_t strides[2] = {cuuint64_t(n) * 4, cuuint64_t(n) * cuuint64_t(n) * 4};
  cuuint32_t box[3] = {32, cuuint32_t(np), 1};
  cuuint32_t estr[3] = {1, 1, 1};
  return g_small_enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, L, dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                     CU_TENSOR_MAP_L2_PROMOTION_NONE,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Encoded store maps keyed by (L, batch, n): torch's caching allocator hands the same
// output addresses back in steady state, so most calls skip the host-side encode.
struct OutMapCache {
  static constexpr int kSlots = 16;
  struct Slot {
    float* L = nullptr;
    int64_t batch = 0;
    int n = 0, np = 0;
    alignas(64) CUtensorMap map;
  } slots[kSlots];
  int next = 0;
  std::mutex mu;
};

bool cached_out_map(CUtensorMap* out, float* L, int64_t batch, int n, int np) {
  static OutMapCache cache;
  std::lock_guard<std::mutex> lock(cache.mu);
  for (auto& s : cache.slots) {
    if (s.L == L && s.batch == batch && s.n == n && s.np == np) {
      *out = s.map;
      return true;
    }
  }
  auto& s = cache.slots[cache.next];
  if (!small_out_map(&s.map, L, batch, n, np)) {
    s.L = nullptr;
    return false;
  }
  s.L = L;
  s.batch = batch;
  s.n = n;
  s.np = np;
  cache.next = (cache.next + 1) % OutMapCache::kSlots;
  *out = s.map;
  return true;
}

// ---- overlap of back-to-back small calls ----
// Per (device, queue), the calls that may still be running: a call that took its dependency
// wait at the start ended the run (everything before it had completed); a call that waits
// later joins it. Any other kernel the library launches on the queue clears the run; work
// enqueued by others is caught on the device (small_potrf_kernel's predecessor check).
// Entries are bound to their (device, queue) for the life of the process, so the device
// counters of an entry only ever count that queue's CTAs; queues beyond the first
// kRunEntries get no entry and their calls never start early.
struct Span {
  uintptr_t lo = 0, hi = 0;
  bool meets(const Span& o) const { return lo < o.hi && o.lo < hi; }
};
struct SmallCall {
  Span a, l, info;
};
struct QueueRun {
  cudaStream_t q = nullptr;
  int dev = -1;  // the same handle (the legacy default queue) exists on every device
  bool used = false;
  int count = 0;
  unsigned parity = 0;  // parity of the next call on this queue
  SmallCall calls[8];
};
int g_overlap_small = 1;
std::mutex g_run_mu;
QueueRun g_runs[kRunEntries];
thread_local bool t_in_small_launch = false;
unsigned* g_run_ctas_dev[64] = {};  // device address of g_run_ctas, per device

int current_device() {
  int d = -1;
  cudaGetDevice(&d);
  return d;
}

// The entry of (q, dev), bound on first use; nullptr when the table is full.
QueueRun* find_run(cudaStream_t q, int dev) {
  for (auto& r : g_runs)
    if (r.used && r.q == q && r.dev == dev) return &r;
  for (auto& r : g_runs) {
    if (!r.used) {
      r.used = true;
      r.q = q;
      r.dev = dev;
      r.count = 0;
      r.parity = 0;
      return &r;
    }
  }
  return nullptr;
}

// Where the new call waits (the kernel's `early`): 0 when it reads a buffer that a call of
// the run writes, 1 when it only writes a buffer that one of them reads or writes, else 2.
int may_start_early(const QueueRun* run, const SmallCall& c) {
  if (!g_overlap_small || run == nullptr || run->count == 0 ||
      run->count >= int(sizeof(run->calls) / sizeof(run->calls[0])))
    return 0;
  int level = 2;
  for (int i = 0; i < run->count; ++i) {
    const SmallCall& e = run->calls[i];
    if (c.a.meets(e.l) || c.a.meets(e.info)) return 0;  // read after write
    if (c.l.meets(e.a) || c.l.meets(e.l) || c.l.meets(e.info) || c.info.meets(e.a) ||
        c.info.meets(e.l) || c.info.meets(e.info))
      level = 1;  // write after read / write
  }
  return level;
}

template <int NP>
int launch_np(const float* A, float* L, int64_t batch, int n, int* info, cudaStream_t q) {
  constexpr int MPC = small_warps<NP>() * SmallShape<NP>::MPW;
  const int64_t blocks = (batch + MPC - 1) / MPC;
  if (blocks > 0x7fffffffLL) return CHOL_ERR_UNSUPPORTED;
  const bool full = (n == NP) && ((reinterpret_cast<uintptr_t>(A) & 15) == 0) &&
                    ((reinterpret_cast<uintptr_t>(L) & 15) == 0);
  const size_t smem = full ? small_smem_bytes<NP, true>() : small_smem_bytes<NP, false>();
  alignas(64) CUtensorMap map;
  memset(&map, 0, sizeof(map));
  // tensor stores of 32 x 32 tiles (the quadrant layout)
  if (full && small_quad<NP, true>() && !cached_out_map(&map, L, batch, n, 32))
    return CHOL_ERR_UNSUPPORTED;
  cudaError_t e;
  SmallCall call;
  const uintptr_t bytes = uintptr_t(batch) * uintptr_t(n) * uintptr_t(n) * sizeof(float);
  call.a = {reinterpret_cast<uintptr_t>(A), reinterpret_cast<uintptr_t>(A) + bytes};
  call.l = {reinterpret_cast<uintptr_t>(L), reinterpret_cast<uintptr_t>(L) + bytes};
  if (info != nullptr)
    call.info = {reinterpret_cast<uintptr_t>(info),
                 reinterpret_cast<uintptr_t>(info) + uintptr_t(batch) * sizeof(int)};
  const int dev = current_device();
  std::lock_guard<std::mutex> lock(g_run_mu);
  unsigned* ctrs = (dev >= 0 && dev < 64) ? g_run_ctas_dev[dev] : nullptr;
  QueueRun* run = ctrs != nullptr ? find_run(q, dev) : nullptr;
  const int early = may_start_early(run, call);
  const unsigned* prev_ctr = nullptr;
  unsigned* my_ctr = nullptr;
  if (run != nullptr) {
    const int entry = int(run - g_runs);
    my_ctr = ctrs + (entry * 2 + int(run->parity)) * kStripes * 2;
    prev_ctr = ctrs + (entry * 2 + int(run->parity ^ 1u)) * kStripes * 2;
  }
  t_in_small_launch = true;
  if (full)
    e = launch_pdl(small_potrf_kernel<NP, true>, dim3(unsigned(blocks)), dim3(small_warps<NP>() * 32),
                   smem, q, true, A, L, batch, n, info, map, early, prev_ctr, my_ctr);
  else
    e = launch_pdl(small_potrf_kernel<NP, false>, dim3(unsigned(blocks)),
                   dim3(small_warps<NP>() * 32), smem, q, true, A, L, batch, n, info, map, early,
                   prev_ctr, my_ctr);
  t_in_small_launch = false;
  if (e != cudaSuccess) {
    if (run != nullptr) run->count = 0;
    return status_from(e);
  }
  if (run == nullptr) return CHOL_OK;
  run->parity ^= 1u;
  if (early > 0) {
    run->calls[run->count++] = call;  // may_start_early needs a run with room
  } else {
    // this call waits for everything before it: the run restarts with it
    run->count = 0;
    run->calls[run->count++] = call;
  }
  return CHOL_OK;
}

template <int NP>
cudaError_t set_smem_np() {
  cudaError_t e = cudaFuncSetAttribute(small_potrf_kernel<NP, true>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       int(small_smem_bytes<NP, true>()));
  if (e != cudaSuccess) return e;
  return cudaFuncSetAttribute(small_potrf_kernel<NP, false>,
                              cudaFuncAttributeMaxDynamicSharedMemorySize,
                              int(small_smem_bytes<NP, false>()));
}

}  // namespace

// Per device (current at the call): kernel attributes and the device address of the
// overlap counters (host code cannot pass the symbol itself to a kernel).
cudaError_t prepare_small() {
  cudaError_t e;
  int dev = -1;
  if ((e = cudaGetDevice(&dev)) != cudaSuccess) return e;
  if (dev >= 0 && dev < 64) {
    void* p = nullptr;
    if ((e = cudaGetSymbolAddress(&p, g_run_ctas)) != cudaSuccess) return e;
    std::lock_guard<std::mutex> lock(g_run_mu);
    g_run_ctas_dev[dev] = static_cast<unsigned*>(p);
  }
  if ((e = set_smem_np<4>()) != cudaSuccess) return e;
  if ((e = set_smem_np<8>()) != cudaSuccess) return e;
  if ((e = set_smem_np<16>()) != cudaSuccess) return e;
  if ((e = set_smem_np<32>()) != cudaSuccess) return e;
  return set_smem_np<64>();
}

// Called by launch_pdl before every kernel launch: the queue's run of small calls ends
// (the small launcher updates the run itself around its own launch).
void note_launch(cudaStream_t q) {
  if (t_in_small_launch) return;
  const int dev = current_device();
  std::lock_guard<std::mutex> lock(g_run_mu);
  for (auto& r : g_runs)
    if (r.q == q && r.dev == dev) r.count = 0;
}

void set_overlap_small(int on) {
  std::lock_guard<std::mutex> lock(g_run_mu);
  g_overlap_small = on;
  for (auto& r : g_runs) r.count = 0;
}

// CTAs that started early / whose early start the device check withdrew, on the current
// device since the library was loaded (reads device memory: synchronous).
int overlap_stats(int64_t* started_early, int64_t* withdrawn) {
  unsigned long long v[kStripes][2] = {};
  if (cudaMemcpyFromSymbol(v, g_overlap_stats, sizeof(v)) != cudaSuccess) return CHOL_ERR_DEVICE;
  int64_t e = 0, w = 0;
  for (int i = 0; i < kStripes; ++i) {
    e += int64_t(v[i][0]);
    w += int64_t(v[i][1]);
  }
  if (started_early) *started_early = e;
  if (withdrawn) *withdrawn = w;
  return CHOL_OK;
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
