// Host-side launchers of the per-head kernels for one element type. Included
// by heads_f32.cu / heads_bf16.cu / heads_f16.cu.
#pragma once

#include "heads_pipe.cuh"
#include "rows_impl.cuh"

namespace bloth {

// CTAs of a launch over `ntok` tokens: one wave of resident CTAs, or fewer.
template <typename T, int D, int MODE>
int64_t head_pipe_grid(int64_t ntok) {
  using P = HP<T, D, MODE>;
  auto kern = head_pipe_kernel<T, D, MODE>;
  if (prepare_smem((const void*)kern, P::SMEM) != BLOTH_OK) return -1;
  const int occ = occupancy((const void*)kern, P::WPB * 32, P::SMEM);
  const int64_t wave = (int64_t)device_sm_count() * (occ > 0 ? occ : 1);
  const int64_t need = ceil_div(ntok, P::WPB);
  return need < wave ? (need > 0 ? need : 0) : wave;
}

template <typename T, int D, int MODE>
int launch_head_fwd(const HeadArgs& a, cudaStream_t st) {
  using P = HP<T, D, MODE>;
  const int64_t grid = head_pipe_grid<T, D, MODE>(a.B * a.S);
  if (grid < 0) return BLOTH_ERR_CUDA;
  if (grid == 0) return BLOTH_OK;
  head_pipe_kernel<T, D, MODE><<<(unsigned)grid, P::WPB * 32, P::SMEM, st>>>(a);
  return launched(cudaGetLastError());
}

template <typename T, int D>
int launch_head_bwd(const HeadArgs& a0, void* ws, size_t ws_bytes, void* dw0, void* dw1,
                    cudaStream_t st) {
  using P = HP<T, D, kHeadNormBwd>;
  using AccT = typename AccOf<T>::type;
  const int64_t grid = head_pipe_grid<T, D, kHeadNormBwd>(a0.B * a0.S);
  if (grid < 0) return BLOTH_ERR_CUDA;
  if ((size_t)grid * 2 * D * sizeof(AccT) > ws_bytes || (grid > 0 && ws == nullptr))
    return BLOTH_ERR_WORKSPACE;
  if (grid > 0) {
    HeadArgs a = a0;
    a.partials = ws;
    head_pipe_kernel<T, D, kHeadNormBwd><<<(unsigned)grid, P::WPB * 32, P::SMEM, st>>>(a);
    const int rc = launched(cudaGetLastError());
    if (rc != BLOTH_OK) return rc;
  }
  return launch_dw_reduce<AccT>(reinterpret_cast<const AccT*>(ws), grid, 2 * D, dw0, D, dw1,
                                a0.w_dt, st);
}

template <typename F>
bool dispatch_head_dim(int D, F&& f) {
  switch (D) {
    case 64: f(std::integral_constant<int, 64>{}); return true;
    case 128: f(std::integral_constant<int, 128>{}); return true;
    case 256: f(std::integral_constant<int, 256>{}); return true;
    default: return false;
  }
}

template <typename T>
int heads_fwd(const HeadArgs& a, int D, bool norm, cudaStream_t st) {
  int rc = BLOTH_ERR_SHAPE;
  dispatch_head_dim(D, [&](auto dd) {
    constexpr int DD = decltype(dd)::value;
    rc = norm ? launch_head_fwd<T, DD, kHeadNormFwd>(a, st)
              : launch_head_fwd<T, DD, kHeadRopeFwd>(a, st);
  });
  return rc;
}

template <typename T>
int heads_bwd(const HeadArgs& a, int D, void* ws, size_t ws_bytes, void* dw0, void* dw1,
              cudaStream_t st) {
  int rc = BLOTH_ERR_SHAPE;
  dispatch_head_dim(D, [&](auto dd) {
    constexpr int DD = decltype(dd)::value;
    rc = launch_head_bwd<T, DD>(a, ws, ws_bytes, dw0, dw1, st);
  });
  return rc;
}

template <typename T>
size_t heads_bwd_workspace(int64_t ntok, int D) {
  using AccT = typename AccOf<T>::type;
  size_t bytes = 0;
  dispatch_head_dim(D, [&](auto dd) {
    constexpr int DD = decltype(dd)::value;
    const int64_t g = head_pipe_grid<T, DD, kHeadNormBwd>(ntok);
    bytes = (size_t)(g > 0 ? g : 0) * 2 * DD * sizeof(AccT);
  });
  return bytes;
}

}  // namespace bloth

#define BLOTH_INSTANTIATE_HEADS(T)                                              \
  namespace bloth {                                                             \
  template int heads_fwd<T>(const HeadArgs&, int, bool, cudaStream_t);          \
  template int heads_bwd<T>(const HeadArgs&, int, void*, size_t, void*, void*,  \
                            cudaStream_t);                                      \
  template size_t heads_bwd_workspace<T>(int64_t, int);                         \
  }
