// Launch bookkeeping shared by every entry point (SM count and occupancy
// caches, CUDA error capture) and the deterministic weight-gradient reduce.
#include <atomic>
#include <map>
#include <mutex>
#include <set>
#include <tuple>

#include "bulk.cuh"
#include "common.cuh"
#include "rows_impl.cuh"

namespace bloth {

// Fault bits recorded by kernels that gave up a bounded wait (kFault*).
// Kernels in other translation units receive its address as an argument.
__device__ unsigned int g_device_fault = 0;

static thread_local int g_last_cuda_error = 0;

// Kernels launched (or recorded into a capturing stream) by this library in
// this process, over all threads and devices.
static std::atomic<long long> g_launches{0};

int cuda_status(cudaError_t err) {
  if (err == cudaSuccess) return BLOTH_OK;
  g_last_cuda_error = (int)err;
  return BLOTH_ERR_CUDA;
}

int launched(cudaError_t err) {
  if (err == cudaSuccess) g_launches.fetch_add(1, std::memory_order_relaxed);
  return cuda_status(err);
}

long long launch_count() { return g_launches.load(std::memory_order_relaxed); }

int last_cuda_error() { return g_last_cuda_error; }

static int current_device() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    return -1;
  }
  return dev;
}

int device_sm_count() {
  static std::mutex mu;
  static std::map<int, int> cache;
  const int dev = current_device();
  std::lock_guard<std::mutex> lk(mu);
  auto it = cache.find(dev);
  if (it != cache.end()) return it->second;
  int n = 0;
  if (dev < 0 || cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
    cudaGetLastError();
    n = 0;
  }
  if (n <= 0) return 1;  // not cached: no usable device yet
  cache[dev] = n;
  return n;
}

int occupancy(const void* func, int block, size_t smem) {
  using Key = std::tuple<int, const void*, int, size_t>;
  static std::mutex mu;
  static std::map<Key, int> cache;
  const int dev = current_device();
  const Key key{dev, func, block, smem};
  {
    std::lock_guard<std::mutex> lk(mu);
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
  }
  int n = 0;
  if (dev < 0 ||
      cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, func, block, smem) != cudaSuccess) {
    cudaGetLastError();
    return 1;
  }
  if (n <= 0) n = 1;
  std::lock_guard<std::mutex> lk(mu);
  cache[key] = n;
  return n;
}

// The attribute is a ceiling per kernel and device: setting it lowers it as
// well as raising it, so it is only ever raised (to the largest size any call
// has asked for), never set back to a smaller request, which would make a
// later launch with a larger, already-seen size fail.
int prepare_smem(const void* func, size_t smem) {
  using Key = std::tuple<int, const void*>;
  static std::mutex mu;
  static std::map<Key, size_t> ceiling;
  const int dev = current_device();
  const Key key{dev, func};
  std::lock_guard<std::mutex> lk(mu);
  auto it = ceiling.find(key);
  if (it != ceiling.end() && it->second >= smem) return BLOTH_OK;
  const cudaError_t e =
      cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) {
    cudaGetLastError();  // do not leave the error for the next launch check
    return cuda_status(e);
  }
  ceiling[key] = smem;
  return BLOTH_OK;
}

unsigned int* fault_word() {
  static std::mutex mu;
  static std::map<int, unsigned int*> cache;
  const int dev = current_device();
  std::lock_guard<std::mutex> lk(mu);
  auto it = cache.find(dev);
  if (it != cache.end()) return it->second;
  void* p = nullptr;
  if (dev < 0 || cudaGetSymbolAddress(&p, g_device_fault) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  cache[dev] = static_cast<unsigned int*>(p);
  return static_cast<unsigned int*>(p);
}

int device_fault(int reset) {
  unsigned int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_device_fault, sizeof(v));
  if (e != cudaSuccess) return -cuda_status(e);
  if (reset) {
    const unsigned int z = 0;
    e = cudaMemcpyToSymbol(g_device_fault, &z, sizeof(z));
    if (e != cudaSuccess) return -cuda_status(e);
  }
  return (int)v;
}

// Column sums of P accumulator rows of N. A CTA of 256 threads takes 8
// columns: thread t sums column 8*blockIdx.x + t % 8 over rows g, g + 32,
// g + 64, ... (g = t / 8) in that order, and the 32 row groups' totals are then
// added in group order, so the result does not depend on scheduling (a warp's
// load covers 4 rows x 32 bytes, whole sectors). Columns [0, n0) go to dw0
// and [n0, N) to dw1 (skipped when dw1 is NULL), cast to w_dt.
//
// Launched as a programmatic dependent of the backward kernel that wrote the
// partial rows (which allows it at its start): its CTAs are small enough to
// become resident beside the backward's CTAs while those still run, so they
// start summing as soon as the backward has completed; nothing is read before
// that (wait_for_prior_grid). Measured at 4096 tokens of the Llama-3-8B step
// on B200 (two reduces per step): 1024-thread CTAs (32 columns each) in
// stream order 91.5 us per step, as dependents 89.8 us; these 256-thread
// CTAs as dependents a further 0.65 us less (interleaved A/B medians).
constexpr int kReduceCols = 8;
constexpr int kReduceGroups = 32;

template <typename AccT>
__global__ void __launch_bounds__(kReduceCols * kReduceGroups)
    dw_reduce_kernel(const AccT* __restrict__ part, int64_t P, int N, void* dw0, int n0, void* dw1,
                     int w_dt) {
  __shared__ double sm[kReduceGroups][kReduceCols + 1];
  wait_for_prior_grid();
  const int ci = threadIdx.x % kReduceCols;
  const int g = threadIdx.x / kReduceCols;
  const int col = blockIdx.x * kReduceCols + ci;
  double s = 0.0;
  if (col < N) {
    // loads issued kBatch at a time, ahead of the sums: a column costs
    // ceil(P / (32 * kBatch)) memory round trips
    constexpr int kBatch = 16;
    for (int64_t p0 = g; p0 < P; p0 += (int64_t)kBatch * kReduceGroups) {
      AccT v[kBatch];
#pragma unroll
      for (int k = 0; k < kBatch; ++k) {
        const int64_t p = p0 + (int64_t)k * kReduceGroups;
        v[k] = p < P ? part[p * N + col] : AccT(0);
      }
#pragma unroll
      for (int k = 0; k < kBatch; ++k) s += (double)v[k];
    }
  }
  sm[g][ci] = s;
  __syncthreads();
  if (g == 0 && col < N) {
    double t = 0.0;
#pragma unroll
    for (int i = 0; i < kReduceGroups; ++i) t += sm[i][ci];
    const float v = (float)t;
    if (col < n0) st_any(dw0, col, w_dt, v);
    else if (dw1 != nullptr) st_any(dw1, col - n0, w_dt, v);
  }
}

template <typename AccT>
int launch_dw_reduce(const AccT* part, int64_t P, int N, void* dw0, int n0, void* dw1, int w_dt,
                     cudaStream_t st) {
  if (N <= 0) return BLOTH_OK;
  const unsigned grid = (unsigned)((N + kReduceCols - 1) / kReduceCols);
  return launched(launch_dependent(dw_reduce_kernel<AccT>, grid, kReduceCols * kReduceGroups, 0,
                                   st, part, P, N, dw0, n0, dw1, w_dt));
}

template int launch_dw_reduce<float>(const float*, int64_t, int, void*, int, void*, int,
                                     cudaStream_t);

// Source of the self-test's bulk copies (32 bytes, 16-byte aligned).
__device__ __align__(16) unsigned char g_selftest_src[32];

// One thread runs the pipelines' expiry path on a two-slot ring without any
// fault. Slot 1 holds a copy issued as usual. Slot 0 expects 16 bytes whose
// copy is not issued, so its bounded wait must give up after limit_ns and
// record kFaultCopyTimeout. The copy of slot 0 is then issued late (as a copy
// that lands after its wait gave up would), and the ring is drained as the
// kernels drain it: both slots land within the limit, so kFaultDrainTimeout
// stays clear, and nothing is in flight when the kernel returns.
__global__ void wait_expiry_kernel(unsigned int* fault, unsigned long long limit_ns) {
  __shared__ __align__(16) unsigned char buf[32];
  __shared__ uint64_t bars[2];
  mbar_init(&bars[0], 1);
  mbar_init(&bars[1], 1);
  mbar_init_fence();
  mbar_arrive_expect_tx(&bars[1], 16);
  bulk_load(buf + 16, g_selftest_src + 16, 16, &bars[1]);
  mbar_arrive_expect_tx(&bars[0], 16);
  if (!mbar_wait(&bars[0], 0, fault, limit_ns)) {
    bulk_load(buf, g_selftest_src, 16, &bars[0]);
    drain_ring(bars, 2, 0, 0, 2, fault, limit_ns);
  }
}

int selftest_wait_expiry(int limit_ms, cudaStream_t st) {
  if (limit_ms < 1 || limit_ms > 2000) return BLOTH_ERR_ARG;
  unsigned int* fault = fault_word();
  if (fault == nullptr) return cuda_status(cudaErrorInvalidDevice);
  wait_expiry_kernel<<<1, 1, 0, st>>>(fault, (unsigned long long)limit_ms * 1000000ull);
  return launched(cudaGetLastError());
}
template int launch_dw_reduce<double>(const double*, int64_t, int, void*, int, void*, int,
                                      cudaStream_t);

}  // namespace bloth
