/*
 * chol_b200.h — C ABI of the B200 (sm_100a) batched FP32 Cholesky library.
 *
 * This is the drop-in boundary for the reference's single hot path,
 *   custom_kernel(data: (b, n, n) float32 SPD) -> L (lower, exact-zero upper)
 * of Mark123M/linalg-kernels:
 *   - submission.py:6-7           (torch.linalg.cholesky_ex(data, check_errors=False).L)
 *   - cholesky/cholesky.py:5845-5850  (custom_kernel: exact-shape dispatch, torch fallback)
 *   - cholesky/cholesky.py:232-250, 391-409, 2598-2656, 3373-3435, 5764-5802
 *     (the per-shape pybind entry points `run(data) -> L` that the dispatcher calls)
 *
 * The reference binds per-shape C++ through pybind (`m.def("run", ...)`) and throws
 * `TORCH_CHECK` errors. Here one set of plain-C entry points covers every (b, n):
 * pointers, sizes and an opaque queue handle in, an integer status out. No torch types,
 * no C++ exceptions cross this boundary.
 *
 * Layout: A and L are row-major contiguous (batch, n, n) float32 arrays in device
 * memory (matrix m starts at m*n*n). Only the lower triangle of A is read (LAPACK
 * uplo='L', which is what torch.linalg.cholesky uses). A is never written unless
 * A == L (exact in-place). L receives the factor with exact zeros above the diagonal.
 *
 * `queue` is a cudaStream_t passed as void* (NULL = the legacy default queue). All work
 * is enqueued asynchronously on it; the call returns before the GPU finishes.
 *
 * Status codes (int): see CHOL_* below. Non-SPD input is reported per matrix in `info`
 * (LAPACK convention: 0 = success, k > 0 = the leading minor of order k is not positive
 * definite); the factor of such a matrix is unspecified from column k on, as with
 * torch.linalg.cholesky_ex(check_errors=False).
 */
#ifndef CHOL_B200_H
#define CHOL_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define CHOL_API __attribute__((visibility("default")))
#else
#define CHOL_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define CHOL_OK 0
#define CHOL_ERR_INVALID_ARG 1   /* bad shape, null pointer, partial aliasing */
#define CHOL_ERR_LAUNCH 2        /* a kernel launch failed (cudaGetLastError) */
#define CHOL_ERR_NOT_SPD 3       /* reported by chol_info_check when some info[m] > 0 */
#define CHOL_ERR_WAIT_TIMEOUT 4  /* a bounded device-side wait ran out (status word set) */
#define CHOL_ERR_WORKSPACE 5     /* caller workspace missing or smaller than required */
#define CHOL_ERR_DEVICE 6        /* no usable sm_100 device / CUDA runtime error */
#define CHOL_ERR_UNSUPPORTED 7   /* size outside what this build supports */
#define CHOL_ERR_SCRATCH_LIMIT 8 /* needs more scratch than chol_potrf_batched_noalloc_f32 has */

/* Library version as MAJOR*10000 + MINOR*100 + PATCH. */
CHOL_API int chol_version(void);

/* Human-readable text for a status code (static storage, never NULL). */
CHOL_API const char* chol_strerror(int status);

/*
 * One-time per-device set-up: checks the device is sm_100, raises the dynamic
 * shared-memory limits of the kernels and resolves driver entry points (TMA maps).
 * Replaces the reference's per-module `prepare()` (cholesky/cholesky.py:2590-2596,
 * called from the lazily-built module, :5807-5820). Idempotent and thread-safe; the
 * factor entry points call it implicitly, but calling it before any CUDA-graph capture
 * keeps the attribute calls out of the capture.
 */
CHOL_API int chol_prepare(int device);

/*
 * Bytes of device workspace chol_potrf_batched_ws_f32 needs for (batch, n).
 * 0 when the chosen kernels need none (n <= 128, and 128 < n <= 256 where the one-CTA-per-
 * matrix kernel takes it, with the default options: see CHOL_OPT_MID_KERNEL).
 */
CHOL_API size_t chol_workspace_bytes(int64_t batch, int64_t n);

/*
 * Batched Cholesky, library-managed workspace.
 * Replaces custom_kernel(data) -> L (cholesky/cholesky.py:5845-5850; submission.py:6-7):
 * the caller allocates L (the reference allocates it with at::empty_like inside the
 * per-shape C++ entry point, e.g. cholesky/cholesky.py:2603, :5766).
 *   A, L   : device pointers to batch*n*n floats; A == L allowed (in place), partial overlap rejected
 *   info   : NULL or device pointer to batch ints (written on the queue)
 *   queue  : cudaStream_t as void*
 * The workspace (if the size needs one) is ONE cache per device, shared by every queue and
 * host thread, grown with cudaMalloc (after cudaDeviceSynchronize, since queued work may
 * still read the old buffer) when a call needs more than it holds. Consequences: calls that
 * overlap on the GPU (different queues, or host threads without ordering) race on it and
 * must be serialised by the caller, and a call that grows it cannot be captured into a CUDA
 * graph. Callers that overlap or capture calls supply a workspace per queue through
 * chol_potrf_batched_ws_f32 instead.
 */
CHOL_API int chol_potrf_batched_f32(const float* A, float* L, int64_t batch, int64_t n,
                           int* info, void* queue);

/*
 * Same as chol_potrf_batched_f32 with caller-provided device workspace of at least
 * chol_workspace_bytes(batch, n) bytes (256-byte aligned). Makes no allocation; this is
 * the form the Python wrapper uses (the workspace comes from torch's caching allocator).
 */
CHOL_API int chol_potrf_batched_ws_f32(const float* A, float* L, int64_t batch, int64_t n,
                              int* info, void* workspace, size_t workspace_bytes,
                              void* queue);

/*
 * Same factorisation, allocating no device memory. No counterpart in the reference, which
 * always allocates its output and workspaces per call. For callers that cannot call
 * cudaMalloc (a host that owns all device memory through its own pool, or a path where
 * cudaMalloc's implicit device synchronisation is not allowed): the caller passes A, L
 * and info as usual, and the scratch comes from a fixed 4 MiB device array inside the
 * library, held on every GPU that loads the library until exit. A call on the blocked path
 * (n > 128, except the sizes CHOL_OPT_MID_KERNEL gives the one-CTA-per-matrix kernel) needs
 * 16 KiB per matrix (the 64 x 64 inverse diagonal blocks), so at most 256 such matrices per
 * call; larger batches return CHOL_ERR_SCRATCH_LIMIT. n <= 128 needs none (with the default
 * options). The optional
 * regions of the blocked schedule are taken from the array when they fit after that.
 * The first call on a device looks up the array's device address with that device
 * current; make that first call before any stream capture. All calls share the array:
 * calls that overlap on the GPU race and must be serialised by the caller.
 */
CHOL_API int chol_potrf_batched_noalloc_f32(const float* A, float* L, int64_t batch, int64_t n,
                                            int* info, void* queue);

/*
 * Number of kernel launches one chol_potrf_batched_*_f32 call makes for (batch, n)
 * (host-only arithmetic on the launch plan; no device call). Used to report launch counts.
 */
CHOL_API int64_t chol_launch_count(int64_t batch, int64_t n);

/*
 * Library options (process-wide, for tests and benchmarks):
 *   CHOL_OPT_GEMM_ENGINE: 0 = auto (tcgen05 3xTF32 tensor cores where the operands allow
 *   TMA, FP32 FMA otherwise; default), 1 = FP32 FMA only, 2 = tensor cores only.
 */
#define CHOL_OPT_GEMM_ENGINE 1
/*   (Option 2, a fused one-launch 64-wide panel step, was removed: it measured slower than
 *   the three-launch step for every shape. Setting it returns CHOL_ERR_INVALID_ARG.) */
/*   CHOL_OPT_OUTER_WIDTH: width of the outer panels of the blocked path (multiple of 64;
 *   0 = default: n for n <= 1024, else 512). */
#define CHOL_OPT_OUTER_WIDTH 3
/*   CHOL_OPT_LOOKAHEAD: 1 = for large n, most of the trailing update of an outer panel runs
 *   on a library side queue beside the next panel's factorisation, for the panels whose
 *   update is short enough for the overlap to pay (the call still completes on the
 *   caller's queue); 0 = everything in order on the caller's queue; -1 (default) = 1 for
 *   1024 < n <= 8192, else 0. The side queue is shared by the calls on a device (they take
 *   turns through a lock), so a call that uses it cannot be captured into a CUDA graph;
 *   set 0 before capturing such calls.
 *   CHOL_OPT_CHAIN_SMS: SMs the side-queue update leaves free for the panel chain (24). */
#define CHOL_OPT_LOOKAHEAD 4
#define CHOL_OPT_CHAIN_SMS 5
/*   CHOL_OPT_PANEL_INVERSE: 1 (default) = each outer panel's diagonal block (the whole
 *   matrix when n <= 1024 and n % 64 == 0) is factored in one launch of 64 x 64 tile
 *   tasks, and the rows below it are solved by one GEMM with the block's inverse; 2 = the
 *   same solve, with the block factored by 64-wide kernel steps; 0 = 64-wide left-looking
 *   steps over every row of the panel. */
#define CHOL_OPT_PANEL_INVERSE 6
/*   CHOL_OPT_OVERLAP_CALLS: 1 (default) = a call with n <= 64 whose A, L and info are
 *   disjoint from those of this library's calls still possibly running on the same queue
 *   starts loading before they finish (it still completes after them). Each CTA first checks
 *   on the device that the previous call on the queue is still running; if it is not, other
 *   work may have been enqueued in between (a kernel writing this call's input, say), and
 *   the CTA waits for everything before it as usual. 0 = every call waits for the previous
 *   work on its queue before reading. */
#define CHOL_OPT_OVERLAP_CALLS 7
/*   CHOL_OPT_MID_KERNEL: 1 (default) = 64 < n <= 128 is factored by one launch with one CTA
 *   per matrix held in shared memory, and 128 < n <= 256 with n % 64 != 0 (batch <= 296, or
 *   n < 144) by one launch with one 512-thread CTA per matrix, both needing no workspace;
 *   0 = the blocked schedule (the workspace sizes then follow it: size workspaces after
 *   setting this). */
#define CHOL_OPT_MID_KERNEL 8
/*   CHOL_OPT_WAIT_LIMIT_US: bound, in microseconds, of the waits in which one CTA waits for
 *   a tile another CTA publishes (the diagonal-block kernel); 0 = the default, 2 s. A wait
 *   that runs out records CHOL_ERR_WAIT_TIMEOUT (see chol_status_check) and makes the
 *   launch's remaining tasks return; the factor of that call is then invalid. The waits on
 *   the TMA and tensor-core completions of one CTA keep a fixed 2 s bound. */
#define CHOL_OPT_WAIT_LIMIT_US 9
/*   CHOL_OPT_CHAIN_WIDTH: block-column width of the left-looking chain that factors one panel
 *   (n <= 1024) for batches too large for the one-launch path: 128 (default; taken when
 *   n % 128 == 0 and batch >= 256, else 64) or 64. With 128 each diagonal block is factored and inverted by one launch and
 *   the chain's GEMMs take 128 columns at a time; it needs 64 KiB more workspace per matrix
 *   (chol_workspace_bytes includes it; a smaller workspace falls back to 64). */
#define CHOL_OPT_CHAIN_WIDTH 10
/*   CHOL_OPT_GEMM_CTAS: cap on the grid of every tensor-core GEMM launch that the CALLING
 *   THREAD issues (0 = default: one CTA per SM; the only thread-local option). A caller that
 *   feeds two queues of one device from one thread sets it before each queue's calls, so that
 *   the two queues' persistent GEMMs hold disjoint shares of the SMs and neither waits for
 *   the other to finish (the multi-GPU driver's panel chain and trailing update). */
#define CHOL_OPT_GEMM_CTAS 11
CHOL_API int chol_set_option(int option, int value);

/*
 * Counts, on the current device since the library was loaded, of the CTAs of n <= 64 calls
 * that started before their predecessor on the queue finished (*started_early), and of those
 * whose early start the device-side predecessor check withdrew (*withdrawn). Synchronous
 * (reads device memory); for tests and diagnostics. Either pointer may be NULL.
 */
CHOL_API int chol_overlap_stats(int64_t* started_early, int64_t* withdrawn);

/*
 * Synchronises the queue, then reads and clears the device status word that the kernels'
 * bounded waits write on expiry. Returns CHOL_OK, CHOL_ERR_WAIT_TIMEOUT or
 * CHOL_ERR_DEVICE. The word is per device and sticky: CHOL_ERR_WAIT_TIMEOUT means that at
 * least one call on the device since the last check has an invalid result. It does not
 * affect later calls (each launch aborts on its own timeouts only). The factor entry points
 * do not read it, since that needs a synchronisation; callers that need the guarantee check
 * it after their calls. (The reference's flag waits have no bound and no status,
 * cholesky/cholesky.py:3588-3598, 4846-4853.)
 */
CHOL_API int chol_status_check(void* queue);

/*
 * Test hook for the bounded waits: one CTA waits, with the same bounded flag wait the
 * diagonal-block kernel uses, until words[0] == value (words: 2 device ints, the second the
 * launch's abort word, normally both 0). A flag that nothing sets makes the wait run out
 * after CHOL_OPT_WAIT_LIMIT_US, and chol_status_check then reports CHOL_ERR_WAIT_TIMEOUT.
 * No counterpart in the reference, whose flag waits are unbounded.
 */
CHOL_API int chol_test_flag_wait(int* words, int value, void* queue);

/*
 * Host-side helper: copies info (batch ints, device) to the host after synchronising
 * the queue and returns CHOL_ERR_NOT_SPD if any entry is > 0 (first failing matrix in
 * *first_bad, or -1). torch.linalg.cholesky (check_errors=True) behaviour; the
 * reference's custom_kernel never checks (check_errors=False, cholesky/cholesky.py:5850).
 */
CHOL_API int chol_info_check(const int* info, int64_t batch, void* queue, int64_t* first_bad);

/*
 * Building blocks of the blocked path, exported for the multi-GPU block-column-cyclic
 * driver (which owns the panel schedule and the NCCL broadcasts) and for tests. Each acts
 * on `batch` row-major matrices spaced `stride` floats apart with leading dimension `ld`
 * (floats). They correspond to the steps of the reference's single-GPU schedule:
 * factor128_kernel (diagonal block + its inverse), gemm_apply (X * T^T) and
 * gemm_history / gemm_inner (C -= P * Q^T) at cholesky/cholesky.py:5440-5489, 5670-5690,
 * 5625-5668. The reference has no multi-GPU path.
 */

/* Factor the kb x kb diagonal block at (k, k) in place (1 <= kb <= 64), zero its strict
   upper part, and, if Tinv is not NULL, write inv(L[k:k+kb, k:k+kb]) as a row-major
   64 x 64 lower triangle at Tinv + m*4096 (identity beyond kb). info (nullable): first
   non-positive pivot column (1-based, global), written when k == 0 or info[m] == 0. */
CHOL_API int chol_block_potrf_f32(float* L, int64_t batch, int64_t stride, int64_t ld, int64_t k,
                         int64_t kb, float* Tinv, int* info, void* queue);

/* C[r][c] = alpha * sum_{q<K} P[r][q] * Q[c][q] + beta * C[r][c] for r < m, c < ncols,
   where C, P, Q point at the (0, 0) element of their views (row-major, K contiguous in
   P and Q). lower_only != 0 writes only elements with c <= r + diag_offset. With beta
   == 0 and ncols <= 64, C may alias P (the panel solve X <- X * T^T runs in place).
   Runs on the tensor cores (tcgen05, 3xTF32 split) where the shape allows, else on
   FP32 FMA. */
CHOL_API int chol_gemm_nt_f32(float* C, int64_t batch, int64_t cstride, int64_t ldc, int64_t m,
                     int64_t ncols, int64_t K, const float* P, int64_t pstride, int64_t ldp,
                     const float* Q, int64_t qstride, int64_t ldq, float alpha, float beta,
                     int64_t diag_offset, int lower_only, void* queue);

/* Factor a tall panel in place: the first w columns of an m-row row-major view (leading
   dimension ld) whose element (0, 0) sits on the matrix diagonal. With w a multiple of 64
   (<= 1024) and 16-byte aligned rows: the w x w top block and its inverse in one launch,
   then one GEMM solves every row below (scratch cached by the library per device, grown
   with cudaMalloc on first need); otherwise left-looking 64-wide steps (diagonal block +
   inverse, solve of the rows below). Tinv: 64*64 floats of device workspace (used by the
   64-wide steps). info (nullable, one int): first failing column of the panel (1-based) or
   0. The per-panel step of the multi-GPU block-column-cyclic driver. The cached scratch is
   shared by every call on the device: calls that overlap on the GPU (different queues)
   race on it. */
CHOL_API int chol_panel_potrf_f32(float* L, int64_t ld, int64_t m, int64_t w, float* Tinv,
                                  int* info, void* queue);

/* chol_panel_potrf_f32 (the one-launch form: w a multiple of 64, <= 1024, 16-byte aligned
   rows) that also writes the factored panel to out: m x w floats, row-major, contiguous,
   disjoint from L. The panel solve writes its rows straight into out, so the multi-GPU
   driver sends out without packing the panel first. With flags = CHOL_PANEL_OUT_ONLY the
   solved rows below the w x w top block are left in out only (L receives the top block);
   the caller copies them into L, e.g. beside the send. flags = 0: L receives the whole
   factored panel too. CHOL_ERR_UNSUPPORTED for shapes the one-launch form does not take. */
#define CHOL_PANEL_OUT_ONLY 1
CHOL_API int chol_panel_potrf_out_f32(float* L, int64_t ld, int64_t m, int64_t w, float* out,
                                      int flags, int* info, void* queue);

/* The diagonal-block step of chol_panel_potrf_out_f32 alone: factors the w x w block at L
   (row stride ld) in place with one launch and writes V = inv(L11) to V (w x w floats,
   row-major, contiguous, disjoint from L; the entries above its diagonal are zero), so
   that a caller can solve the rows below as X = A21 V^T (chol_gemm_nt_f32) wherever they
   are: the multi-GPU driver sends the unfactored panel while its owner factors the block,
   then sends L11 and V, and every rank solves its copy. w: a multiple of 64, <= 1024;
   16-byte aligned rows. info (nullable, one int): first failing column (1-based) or 0.
   Uses the same cached scratch as chol_panel_potrf_f32 (calls on different queues race). */
CHOL_API int chol_diag_potrf_inv_f32(float* L, int64_t ld, int64_t w, float* V, int* info,
                                     void* queue);

/* chol_gemm_nt_f32 for one matrix whose columns are stored block-cyclically: local column c
   of C (and row c of Q) stands for global column c + (c / col_block) * (col_stride -
   col_block), and lower_only compares that global column with the row. One launch updates
   every trailing block a rank owns. col_block must be 256 and col_stride a multiple of it
   (tensor-core path; needs 16-byte aligned rows). With P == Q (the driver's case) and more
   than one column block, the TF32 low parts of P are computed once into a scratch buffer
   the library caches per device (grown with cudaMalloc on first need; calls that overlap
   on the GPU race on it) and loaded by the GEMM instead of split in shared memory. */
CHOL_API int chol_gemm_nt_cyclic_f32(float* C, int64_t ldc, int64_t m, int64_t ncols, int64_t K,
                                     const float* P, int64_t ldp, const float* Q, int64_t ldq,
                                     float alpha, float beta, int64_t diag_offset, int lower_only,
                                     int64_t col_block, int64_t col_stride, void* queue);

/*
 * Device-side check of a factor: the property gates of the reference's checker
 * (finiteness, lower-triangular structure, positive diagonal, reconstruction residual
 * against the FP32 input; reference AGENTS.md:47-50, harness gate
 * cholesky/b4096n32/cholesky_b4096n32_modal.py:307-334), computed on the GPU so that a
 * large factor needs no host copy. No kernel of the reference does this; the reference's
 * checker runs in PyTorch. For each matrix m, with S the symmetric matrix the lower
 * triangle of A defines and R = tril(L) tril(L)^T - S accumulated in FP64:
 *   out[8m+0] = ||R||_F^2              out[8m+1] = ||S||_F^2
 *   out[8m+2] = max_i sum_j |R_ij|     out[8m+3] = max_i sum_j |S_ij|
 *   out[8m+4] = number of non-finite entries of L
 *   out[8m+5] = number of entries strictly above the diagonal of L that are not +-0
 *   out[8m+6] = number of diagonal entries of L that are not > 0
 *   out[8m+7] = 0
 * out: 8*batch doubles of device memory; work: chol_validate_work_bytes(batch, n) bytes of
 * device memory (FP64 row sums). Both 8-byte aligned; both overwritten. Asynchronous on
 * `queue`: read out after synchronising it. A non-zero upper part of L does not enter R;
 * out[8m+5] reports it.
 */
CHOL_API size_t chol_validate_work_bytes(int64_t batch, int64_t n);
CHOL_API int chol_validate_f32(const float* A, const float* L, int64_t batch, int64_t n,
                               double* out, void* work, void* queue);

#ifdef __cplusplus
}
#endif

#endif /* CHOL_B200_H */
