// bloth_rmsnorm_bwd_noalloc: the RMSNorm backward for callers that cannot
// allocate device memory.
//
// Some callers hand a kernel only its inputs and outputs: an operator or
// plugin interface that owns the device memory plan (every buffer is decided
// by the host framework before execution, so there is no workspace argument
// to pass), or a process whose device memory is all reserved by another
// allocator at start-up, where a cudaMalloc would fail or split that
// reservation. bloth_rmsnorm_bwd needs a workspace for its per-CTA
// weight-gradient partial sums; this variant keeps those partials in a
// file-scope device array of fixed size instead, so it allocates nothing.
//
// The array costs every GPU that loads the library BLOTH_NOALLOC_SCRATCH_BYTES
// of device memory until the process exits. Host code cannot use its name as
// a device address, so the first call on each device (with that device
// current) looks the address up once with cudaGetSymbolAddress; make that
// first call before any stream capture. All calls share the array and it
// keeps the last call's contents: every partial row is fully rewritten by the
// kernel before the fixed-order reduce reads it, so nothing needs clearing,
// but two calls whose kernels overlap on the GPU (different streams, or
// different host threads without ordering) race on it.
#include <map>
#include <mutex>

#include "common.cuh"

// The entry point with the caller-provided workspace (capi.cu).
extern "C" int bloth_rmsnorm_bwd(const void* dy, int64_t lddy, const void* x, int64_t ldx,
                                 const void* w, float w_offset, const float* rstd, void* dx, int64_t lddx,
                                 void* dw, int64_t M, int64_t N, int dtype, int w_dtype,
                                 void* workspace, size_t workspace_bytes, void* stream);
extern "C" size_t bloth_rmsnorm_bwd_workspace_bytes(int64_t M, int64_t N, int dtype);

namespace {

static __device__ __align__(256) unsigned char g_noalloc_scratch[BLOTH_NOALLOC_SCRATCH_BYTES];

// Device address of g_noalloc_scratch on the current device (looked up once
// per device), or nullptr with *status set when the lookup fails.
void* scratch_address(int* status) {
  static std::mutex mu;
  static std::map<int, void*> cache;
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    *status = bloth::cuda_status(e);
    return nullptr;
  }
  std::lock_guard<std::mutex> lk(mu);
  auto it = cache.find(dev);
  if (it != cache.end()) return it->second;
  void* p = nullptr;
  e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
  if (e != cudaSuccess || p == nullptr) {
    *status = bloth::cuda_status(e != cudaSuccess ? e : cudaErrorInvalidSymbol);
    return nullptr;
  }
  cache[dev] = p;
  return p;
}

}  // namespace

extern "C" int bloth_rmsnorm_bwd_noalloc(const void* dy, int64_t lddy, const void* x,
                                         int64_t ldx, const void* w, float w_offset,
                                         const float* rstd, void* dx,
                                         int64_t lddx, void* dw, int64_t M, int64_t N, int dtype,
                                         int w_dtype, void* stream) {
  // Same partial-sum layout as bloth_rmsnorm_bwd, so the results are the same.
  const size_t need = bloth_rmsnorm_bwd_workspace_bytes(M, N, dtype);
  if (need > (size_t)BLOTH_NOALLOC_SCRATCH_BYTES) return BLOTH_ERR_WORKSPACE;
  int status = BLOTH_OK;
  void* scratch = scratch_address(&status);
  if (scratch == nullptr) return status;
  return bloth_rmsnorm_bwd(dy, lddy, x, ldx, w, w_offset, rstd, dx, lddx, dw, M, N, dtype, w_dtype, scratch,
                           (size_t)BLOTH_NOALLOC_SCRATCH_BYTES, stream);
}
