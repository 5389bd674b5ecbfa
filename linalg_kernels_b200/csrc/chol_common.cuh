// chol_common.cuh — shared device/host helpers for the sm_100a Cholesky kernels.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/chol_b200.h"

namespace chol {

// ---------------------------------------------------------------------------------
// Programmatic dependent launch (PDL). Every kernel of the blocked schedule starts
// with griddep_wait() before it touches memory written by the previous kernel on
// the queue, and calls griddep_launch() once its CTAs are resident, so the next
// kernel's launch latency overlaps this kernel's tail. Both are no-ops when the
// kernel was launched without the programmatic-serialization attribute.
// ---------------------------------------------------------------------------------
__device__ __forceinline__ void griddep_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void griddep_launch() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---------------------------------------------------------------------------------
// Packed FP32x2 fused multiply-add (sm_100: one instruction, two IEEE fma.rn lanes).
// d = a * b + c elementwise on (x, y); bitwise identical to two scalar fmaf calls.
// ---------------------------------------------------------------------------------
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
  uint64_t ra, rb, rc, rd;
  asm("mov.b64 %0, {%1, %2};" : "=l"(ra) : "f"(a.x), "f"(a.y));
  asm("mov.b64 %0, {%1, %2};" : "=l"(rb) : "f"(b.x), "f"(b.y));
  asm("mov.b64 %0, {%1, %2};" : "=l"(rc) : "f"(c.x), "f"(c.y));
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(rd) : "l"(ra), "l"(rb), "l"(rc));
  float2 d;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(d.x), "=f"(d.y) : "l"(rd));
  return d;
}

// ---------------------------------------------------------------------------------
// Asynchronous copies. cp.async moves global -> shared without registers, so every copy a
// warp issues is in flight at once; cp.async.bulk stores shared -> global through the
// async (TMA) engine. Both finish with hardware waits (no spin loops).
// ---------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gmem_src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem_dst)),
               "l"(gmem_src)
               : "memory");
}
__device__ __forceinline__ void cp_async4(void* smem_dst, const void* gmem_src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(smem_dst)),
               "l"(gmem_src)
               : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
// Wait until at most N of this thread's committed groups are still in flight.
template <int N>
__device__ __forceinline__ void cp_async_wait_group() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
// Order this thread's generic-proxy shared-memory writes before async-proxy reads.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
// Bulk copy shared -> global (both 16-byte aligned, bytes a multiple of 16).
__device__ __forceinline__ void bulk_store(void* gmem_dst, const void* smem_src, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(gmem_dst),
               "r"(smem_u32(smem_src)), "r"(bytes)
               : "memory");
}
// Wait until this thread's bulk stores have finished reading shared memory.
__device__ __forceinline__ void bulk_store_wait_read() {
  asm volatile("cp.async.bulk.commit_group;\n\tcp.async.bulk.wait_group.read 0;" ::: "memory");
}

// The same on values already held as 64-bit register pairs (no packing moves).
__device__ __forceinline__ uint64_t ffma2_u64(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t pack2(float x, float y) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(x), "f"(y));
  return r;
}
__device__ __forceinline__ float lo_of(uint64_t v) { return __uint_as_float(uint32_t(v)); }
__device__ __forceinline__ float hi_of(uint64_t v) { return __uint_as_float(uint32_t(v >> 32)); }

// Every kernel launch on a queue ends the run of back-to-back small calls that may overlap
// on it (overlap_small_calls in chol_small.cu); the small launcher records its own calls.
void note_launch(cudaStream_t q);

// Host-side launch helper: cudaLaunchKernelEx with the PDL attribute.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                              cudaStream_t q, bool pdl, Args... args) {
  note_launch(q);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = q;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

inline int status_from(cudaError_t e) {
  if (e == cudaSuccess) return CHOL_OK;
  return CHOL_ERR_LAUNCH;
}

// Arguments of the NT update/solve GEMM: C = alpha * P * Q^T + beta * C.
struct GemmArgs {
  float* C;
  int64_t cstride, ldc;
  const float* P;
  int64_t pstride, ldp;
  const float* Q;
  int64_t qstride, ldq;
  int64_t m, ncols, K;
  int64_t diag_offset;  // lower_only: write only c <= r + diag_offset
  float alpha, beta;
  int lower_only;
  int64_t batch;
  // Column-cyclic mapping (multi-GPU block-cyclic layouts): when cmap_block > 0, local
  // column c of C (and row c of Q) stands for global column
  //   c + (c / cmap_block) * (cmap_stride - cmap_block),
  // i.e. consecutive local blocks of cmap_block columns are cmap_stride global columns
  // apart; lower_only compares global columns with rows. Q's rows follow the same map.
  int64_t cmap_block, cmap_stride;
  // Optional source of the beta * C term (same layout as C): C = alpha P Q^T + beta Csrc.
  // nullptr: C itself (read-modify-write).
  const float* Csrc;
};

// Entry-point plumbing shared by the C-ABI files (chol_api.cu).
int prepare_device_checked(int dev);
int check_potrf_args(const float* A, float* L, int64_t batch, int64_t n);
// Smallest workspace a call can run with (the blocked path then splits every operand in
// shared memory instead of reading precomputed low parts).
size_t workspace_min_bytes(int64_t batch, int64_t n);
int potrf_with_workspace(const float* A, float* L, int64_t batch, int64_t n, int* info, void* ws,
                         size_t ws_bytes, cudaStream_t q);

// Host launchers implemented in the .cu files.
cudaError_t prepare_small();
int prepare_kernels(int device);
int launch_small(const float* A, float* L, int64_t batch, int n, int* info, cudaStream_t q);
// 64 < n <= 128: one CTA per matrix in shared memory (chol_mid.cu), unless
// CHOL_OPT_MID_KERNEL is 0.
extern int g_mid_kernel;
bool use_mid(int64_t batch, int64_t n);
cudaError_t prepare_mid();
int launch_mid(const float* A, float* L, int64_t batch, int n, int* info, cudaStream_t q);
// Overlap of back-to-back independent small calls on one queue (on by default).
void set_overlap_small(int on);
// CTAs of small calls that started early / whose early start the device check withdrew.
int overlap_stats(int64_t* started_early, int64_t* withdrawn);
int launch_copy_lower(const float* A, float* L, int64_t batch, int64_t n, cudaStream_t q,
                      bool pdl);
// Zeros of L right of each row's bw-wide diagonal block (columns >= bw * (r / bw + 1)).
int launch_zero_upper(float* L, int64_t batch, int64_t n, cudaStream_t q, bool pdl,
                      int64_t bw = 64);
// 128 x 128 diagonal block at (k, k): factor from S into L and T = inv(L_kk) (128 x 128,
// leading dimension tld >= 128) in one launch, one 128-thread CTA per matrix; zero_cols
// zeros of L's rows k..k+127 right of the block are written too.
int launch_potrf_block128(const float* S, int64_t sstride, int64_t lds, float* L, int64_t stride,
                          int64_t ld, int64_t batch, int64_t k, float* T, int64_t tstride,
                          int64_t tld, int* info, cudaStream_t q, int64_t zero_cols);
// Tinv (+ m * tstride, leading dimension tld) receives inv(L_kk) as a 64 x 64 lower triangle.
int launch_potrf_block(const float* S, int64_t sstride, int64_t lds, float* L, int64_t stride,
                       int64_t ld, int64_t batch, int64_t k, int64_t kb, float* Tinv, int* info,
                       cudaStream_t q, bool pdl, int64_t tstride = 4096, int64_t tld = 64);
// One launch: factor the (64 * nb)-square diagonal block at L11 in place and, with want_v,
// write V = inv(L11) (lower blocks; the caller zeroes the blocks above the diagonal once);
// without want_v, V (+ m * vstride) only receives the nb inverse diagonal blocks, 64 x 64
// each, one after another.
// flags: kDiagFlags ints per matrix and ticket: one counter, both zero before the first
// launch; epoch: > 0, distinct for every launch that shares the flags (chol_diag.cu).
constexpr int kDiagFlags = 768;
int launch_diag_block(float* L11, int64_t mstride, int64_t ld, float* V, int64_t vstride,
                      int64_t ldv, int nb, bool want_v, int* flags, unsigned* ticket, int epoch,
                      int* info, int64_t col0, int64_t batch, cudaStream_t q);
// V = inv(L11) for a (64 * nblk)-square diagonal block L11 whose 64 x 64 diagonal inverses
// are already in V's diagonal blocks (chol_blocked.cu).
cudaError_t prepare_blocked();
int launch_trtri_panel(const float* L11, int64_t lstride, int64_t ld, float* V, int64_t vstride,
                       int64_t ldv, int nblk, int64_t batch, cudaStream_t q);
int launch_gemm_simt(const GemmArgs& g, cudaStream_t q, bool pdl);
bool tc_supported(const GemmArgs& g);
// Prebuilt TMA maps over one whole (rows x cols, leading dimension ld) matrix per batch
// entry, one per box height the GEMM uses; opaque 128-byte CUtensorMap storage.
struct TcMatrixMaps {
  alignas(64) unsigned char p128[128];
  alignas(64) unsigned char q64[128];
  alignas(64) unsigned char q128[128];
  alignas(64) unsigned char q256[128];
  const float* base;
  int64_t ld, bstride;
};
bool tc_make_matrix_maps(const float* base, int64_t rows, int64_t cols, int64_t ld, int64_t batch,
                         int64_t bstride, TcMatrixMaps* maps);
// max_ctas > 0 caps the persistent grid (leaves SMs for concurrent work on another queue).
int launch_gemm_tc_mapped(const GemmArgs& g, const TcMatrixMaps& pm, const TcMatrixMaps& qm,
                          cudaStream_t q, bool pdl, int max_ctas = 0);
int launch_gemm_tc_mapped_lo(const GemmArgs& g, const TcMatrixMaps& pm, const TcMatrixMaps& qm,
                             const TcMatrixMaps& lm, int64_t lk, cudaStream_t q, bool pdl,
                             int max_ctas = 0);
// dst = low TF32 part of src (src - its 19-bit truncation); with copy != nullptr, src is also
// copied to copy (+ m * cstride, leading dimension ldcopy). src and dst may be the same.
int launch_tf32_lo(const float* src, int64_t lds, float* dst, int64_t ldd, int64_t rows,
                   int64_t cols, int64_t batch, int64_t sstride, int64_t dstride, cudaStream_t q,
                   float* copy = nullptr, int64_t ldcopy = 0, int64_t cstride = 0);
int launch_gemm_tc(const GemmArgs& g, cudaStream_t q, bool pdl, int* status);
// P == Q with their TF32 low parts precomputed in lo (same rows, leading dimension ldlo);
// BN = 256, column-cyclic map allowed.
int launch_gemm_tc_prelo(const GemmArgs& g, const float* lo, int64_t ldlo, cudaStream_t q,
                         bool pdl);
cudaError_t prepare_tc();
int read_and_clear_status(int* out);
// Bound of the inter-CTA flag waits (CHOL_OPT_WAIT_LIMIT_US; 2 s by default).
uint64_t wait_limit_ns();
// Cap on tensor-core GEMM grids set by the calling thread (CHOL_OPT_GEMM_CTAS; 0 = none).
int gemm_cta_cap();
// One CTA waiting with the bounded flag wait for words[0] == value (words[1]: abort word).
int launch_flag_wait(int* words, int value, cudaStream_t q);
// Device address of the status word (for kernels in other translation units).
int* device_status_ptr();
// Engine choice for the NT-GEMM: 0 auto (tensor cores when the operands allow TMA), 1 FP32
// FMA only, 2 tensor cores only (CHOL_ERR_UNSUPPORTED where TMA cannot be used).
extern int g_gemm_engine;
int launch_gemm(const GemmArgs& g, cudaStream_t q, bool pdl);

}  // namespace chol
