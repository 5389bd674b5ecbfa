// chol_noalloc.cu — batched Cholesky entry point that allocates no device memory.
//
// Some callers cannot call cudaMalloc: a host application that owns all device memory
// through its own pool and forbids plugins from allocating outside it, or code on a path
// where the implicit device-wide synchronisation of cudaMalloc/cudaFree is not
// acceptable. chol_potrf_batched_f32 grows a cached workspace with cudaMalloc, and
// chol_potrf_batched_ws_f32 needs the caller to allocate one. This entry point instead
// takes its scratch from one fixed file-scope device array, g_noalloc_scratch, of
// kNoAllocScratchBytes (4 MiB). The scratch a call must have (n > 128 only) is the inverse
// of each 64 x 64 diagonal block of the blocked path, 16 KiB per matrix: at most 256
// matrices per call.
// The blocked schedule also places its optional regions (the one-launch diagonal-block
// buffers, the panel buffer of precomputed low parts, V = inv(L11)) in the array when they
// fit after that, and runs without them otherwise. Every GPU that loads the library holds
// the array until the process exits.
//
// Host code may not pass the array's name to a kernel: on the host it is only a stand-in
// symbol, not a device address. The device address is obtained once per device with
// cudaGetSymbolAddress, with that device current, by the first call on the device; that
// first call should therefore come before any stream capture.
//
// All calls share the one array and it keeps the previous call's contents. The regions
// that must start at zero (tile flags, tickets) are cleared by every call on its
// queue (cudaMemsetAsync); the inverse blocks are written before they are read,
// but calls whose work overlaps on the GPU (different queues, or different host threads
// without ordering) race on it and must be serialised by the caller.
#include <mutex>

#include "chol_common.cuh"

namespace chol {
namespace {

// 256 matrices with n > 128: 4 MiB of inverse blocks
constexpr size_t kNoAllocScratchBytes = size_t(4) << 20;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

struct NoAllocDevice {
  std::once_flag once;
  void* ptr = nullptr;
  int status = CHOL_OK;
};

NoAllocDevice* noalloc_device(int dev) {
  static NoAllocDevice devs[64];
  if (dev < 0 || dev >= 64) return nullptr;
  return &devs[dev];
}

// Device address of g_noalloc_scratch on `dev` (which must be the current device).
int noalloc_scratch(int dev, void** out) {
  NoAllocDevice* d = noalloc_device(dev);
  if (d == nullptr) return CHOL_ERR_DEVICE;
  std::call_once(d->once, [d]() {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || p == nullptr) {
      d->status = CHOL_ERR_DEVICE;
      return;
    }
    d->ptr = p;
  });
  *out = d->ptr;
  return d->status;
}

}  // namespace
}  // namespace chol

using namespace chol;

extern "C" int chol_potrf_batched_noalloc_f32(const float* A, float* L, int64_t batch, int64_t n,
                                              int* info, void* queue) {
  int st = check_potrf_args(A, L, batch, n);
  if (st || batch == 0 || n == 0) return st;
  const size_t need = workspace_min_bytes(batch, n);
  if (need > kNoAllocScratchBytes) return CHOL_ERR_SCRATCH_LIMIT;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return CHOL_ERR_DEVICE;
  if ((st = prepare_device_checked(dev))) return st;
  void* scratch = nullptr;
  if ((st = noalloc_scratch(dev, &scratch))) return st;
  return potrf_with_workspace(A, L, batch, n, info, scratch, kNoAllocScratchBytes,
                              static_cast<cudaStream_t>(queue));
}
