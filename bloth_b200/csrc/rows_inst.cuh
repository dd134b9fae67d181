// Host-side launchers of the row kernels for one element type. Included by
// rows_f32.cu / rows_bf16.cu / rows_f16.cu, each of which instantiates them
// for its type, so the kernel variants compile in parallel.
#pragma once

#include "rows_impl.cuh"

namespace bloth {

template <typename T, int VEC, typename Cfg, bool ROPE>
int launch_row_fwd(const RowArgs& a, cudaStream_t st) {
  constexpr int BLOCK = Cfg::TPR * Cfg::RPC;
  auto kern = row_fwd_kernel<T, VEC, Cfg::TPR, Cfg::VPT, Cfg::RPC, ROPE>;
  const int occ = occupancy((const void*)kern, BLOCK, 0);
  const int64_t wave = (int64_t)device_sm_count() * (occ > 0 ? occ : 1);
  const int64_t need = ceil_div(a.M, Cfg::RPC);
  const int64_t grid = need < wave ? need : wave;
  if (grid <= 0) return BLOTH_OK;
  kern<<<(unsigned)grid, BLOCK, 0, st>>>(a);
  return cuda_status(cudaGetLastError());
}

template <typename T, int VEC, typename Cfg, bool ROPE>
int launch_row_bwd(const RowArgs& a0, void* ws, size_t ws_bytes, void* dw, cudaStream_t st) {
  using AccT = typename AccOf<T>::type;
  constexpr int BLOCK = Cfg::TPR * Cfg::RPC;
  const int64_t grid = row_bwd_grid<T, VEC, Cfg, ROPE>(a0.M);
  if ((size_t)grid * a0.N * sizeof(AccT) > ws_bytes || (grid > 0 && ws == nullptr))
    return BLOTH_ERR_WORKSPACE;
  if (grid > 0) {
    RowArgs a = a0;
    a.partials = ws;
    auto kern = row_bwd_kernel<T, VEC, Cfg::TPR, Cfg::VPT, Cfg::RPC, ROPE>;
    constexpr size_t smem = row_bwd_smem<T, VEC, Cfg>();
    kern<<<(unsigned)grid, BLOCK, smem, st>>>(a);
    const int rc = cuda_status(cudaGetLastError());
    if (rc != BLOTH_OK) return rc;
  }
  return launch_dw_reduce<AccT>(reinterpret_cast<const AccT*>(ws), grid, a0.N, dw, a0.N, nullptr,
                                a0.w_dt, st);
}

template <typename T>
int rows_fwd(const RowArgs& a, bool rope, bool vec, cudaStream_t st) {
  constexpr int V = 16 / sizeof(T);
  int rc = BLOTH_ERR_SHAPE;
  auto go = [&](auto cfg, auto vecc) {
    using C = decltype(cfg);
    constexpr int VV = decltype(vecc)::value;
    rc = rope ? launch_row_fwd<T, VV, C, true>(a, st) : launch_row_fwd<T, VV, C, false>(a, st);
  };
  if (vec)
    dispatch_row_cfg<V>(a.N, [&](auto cfg) { go(cfg, std::integral_constant<int, V>{}); });
  else
    dispatch_row_cfg<1>(a.N, [&](auto cfg) { go(cfg, std::integral_constant<int, 1>{}); });
  return rc;
}

template <typename T>
int rows_bwd(const RowArgs& a, bool rope, bool vec, void* ws, size_t ws_bytes, void* dw,
             cudaStream_t st) {
  constexpr int V = 16 / sizeof(T);
  int rc = BLOTH_ERR_SHAPE;
  auto go = [&](auto cfg, auto vecc) {
    using C = decltype(cfg);
    constexpr int VV = decltype(vecc)::value;
    rc = rope ? launch_row_bwd<T, VV, C, true>(a, ws, ws_bytes, dw, st)
              : launch_row_bwd<T, VV, C, false>(a, ws, ws_bytes, dw, st);
  };
  if (vec)
    dispatch_row_cfg<V>(a.N, [&](auto cfg) { go(cfg, std::integral_constant<int, V>{}); });
  else
    dispatch_row_cfg<1>(a.N, [&](auto cfg) { go(cfg, std::integral_constant<int, 1>{}); });
  return rc;
}

// Workspace for the backward: the larger of the vector and scalar paths'
// needs, so the size does not depend on the pointers' alignment.
template <typename T>
size_t rows_bwd_workspace(int64_t M, int N, bool rope) {
  using AccT = typename AccOf<T>::type;
  constexpr int V = 16 / sizeof(T);
  int64_t grid = 0;
  auto take = [&](auto cfg, auto vecc) {
    using C = decltype(cfg);
    constexpr int VV = decltype(vecc)::value;
    const int64_t g = rope ? row_bwd_grid<T, VV, C, true>(M) : row_bwd_grid<T, VV, C, false>(M);
    if (g > grid) grid = g;
  };
  dispatch_row_cfg<V>(N, [&](auto cfg) { take(cfg, std::integral_constant<int, V>{}); });
  dispatch_row_cfg<1>(N, [&](auto cfg) { take(cfg, std::integral_constant<int, 1>{}); });
  return (size_t)grid * (size_t)N * sizeof(AccT);
}

}  // namespace bloth

#define BLOTH_INSTANTIATE_ROWS(T)                                                   \
  namespace bloth {                                                                 \
  template int rows_fwd<T>(const RowArgs&, bool, bool, cudaStream_t);               \
  template int rows_bwd<T>(const RowArgs&, bool, bool, void*, size_t, void*,        \
                           cudaStream_t);                                           \
  template size_t rows_bwd_workspace<T>(int64_t, int, bool);                        \
  }
