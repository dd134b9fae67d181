// Host-side launchers of the per-head kernels for one element type. Included
// by heads_f32.cu / heads_bf16.cu / heads_f16.cu.
#pragma once

#include "heads_pipe.cuh"
#include "qk_tok.cuh"
#include "rows_impl.cuh"

namespace bloth {

// Target bytes of row data per token block, forward and backward, and the
// slot limit beyond which the per-head kernel takes the call. Measured at the
// Llama-3-8B shape (32 + 8 heads of 128, bf16), in interleaved A/B replays of
// the whole step: backward blocks of 2 tokens (41 KB) beat 1 token by 10 us
// per step at 32768 tokens and 1 us at 4096.
constexpr int kTokSlotTarget[2] = {20 * 1024, 40 * 1024};
constexpr int kTokSlotMax = 96 * 1024;
// The forward takes the token-block kernel up to this many tokens and the
// per-head kernel above: measured at the Llama-3-8B shape, token blocks are
// 3.4 us per step faster at 4096 tokens and per-head warps 10 us faster at
// 32768.
constexpr int64_t kTokFwdMaxTokens = 8192;

// Whether the token-block kernel takes the call, and its plan: cos/sin come
// from inv_freq; every head tensor of the call (inputs, outputs, and for the
// backward the forward inputs) is a contiguous [B, S, H, D] tensor; for the
// backward, each rstd run of a block is a 16-byte unit (H % 4 == 0, rstd
// 16-byte aligned) so that it moves with the block's bulk copies.
template <typename T, int D, bool BWD>
bool qk_tok_plan(const HeadArgs& a, TokPlan& pl) {
  using Q = QT<T, D, BWD>;
  if (a.inv_freq == nullptr || a.cos != nullptr) return false;
  const int64_t ntok = a.B * a.S;
  const int64_t Hs[2] = {a.H[0], a.H[1]};
  if (Hs[0] + Hs[1] < 1) return false;
  for (int t = 0; t < 2; ++t) {
    const int64_t H = Hs[t];
    if (H == 0) continue;
    auto contig = [&](const HT& h) {
      return (H == 1 || h.sh == D) && (a.S <= 1 || h.ss == H * D) &&
             (a.B <= 1 || h.sb == a.S * H * D);
    };
    if (!contig(a.src[t]) || !contig(a.dst[t]) || (BWD && !contig(a.x[t]))) return false;
    if (BWD && (H % 4 != 0 || reinterpret_cast<uintptr_t>(a.rstd_in[t]) % 16 != 0)) return false;
  }
  const int hq = (int)Hs[0], hk = (int)Hs[1];
  if (!BWD && ntok > kTokFwdMaxTokens) return false;
  int tb = kTokSlotTarget[BWD ? 1 : 0] / ((hq + hk) * Q::ROWB * Q::NT);
  tb = tb < 1 ? 1 : (tb > Q::TBMAX ? Q::TBMAX : tb);
  if (ntok < tb) tb = (int)(ntok > 0 ? ntok : 1);
  pl.tb = tb;
  pl.slot = Q::slot_bytes(tb, hq, hk);
  if (pl.slot > kTokSlotMax) return false;
  pl.nst = 2;
  pl.s_div = FastDiv::make((uint32_t)(a.S > 0 ? a.S : 1));
  return true;
}

// Grid of the token-block kernel: one wave of resident CTAs or fewer (-1: the
// kernel cannot be prepared on this device).
template <typename T, int D, bool BWD>
int64_t qk_tok_grid(const HeadArgs& a, const TokPlan& pl) {
  using Q = QT<T, D, BWD>;
  auto kern = qk_token_kernel<T, D, BWD>;
  const size_t smem = Q::smem(pl.nst, pl.slot);
  if (prepare_smem((const void*)kern, smem) != BLOTH_OK) return -1;
  const int occ = occupancy((const void*)kern, Q::BLOCK, smem);
  const int64_t wave = (int64_t)device_sm_count() * (occ > 0 ? occ : 1);
  const int64_t nblk = ceil_div(a.B * a.S, pl.tb);
  return nblk < wave ? (nblk > 0 ? nblk : 0) : wave;
}

// Most CTAs a backward launch of the token-block kernel can have on this
// device: a wave at the smallest shared-memory plan (an upper bound of every
// plan's grid, for the workspace query, which does not know the head counts).
template <typename T, int D>
int64_t qk_tok_bwd_max_grid() {
  using Q = QT<T, D, true>;
  auto kern = qk_token_kernel<T, D, true>;
  const size_t smem = Q::smem(2, 16);
  if (prepare_smem((const void*)kern, smem) != BLOTH_OK) return -1;
  const int occ = occupancy((const void*)kern, Q::BLOCK, smem);
  return (int64_t)device_sm_count() * (occ > 0 ? occ : 1);
}

template <typename T, int D, bool BWD>
int launch_qk_tok(const HeadArgs& a, const TokPlan& pl, int64_t grid, cudaStream_t st) {
  using Q = QT<T, D, BWD>;
  return launched(launch_ex(qk_token_kernel<T, D, BWD>, (unsigned)grid, Q::BLOCK,
                            Q::smem(pl.nst, pl.slot), st, a, pl));
}

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
  TokPlan pl;
  if (MODE == kHeadNormFwd && qk_tok_plan<T, D, false>(a, pl)) {
    const int64_t grid = qk_tok_grid<T, D, false>(a, pl);
    if (grid < 0) return BLOTH_ERR_CUDA;
    return grid == 0 ? BLOTH_OK : launch_qk_tok<T, D, false>(a, pl, grid, st);
  }
  const int64_t grid = head_pipe_grid<T, D, MODE>(a.B * a.S);
  if (grid < 0) return BLOTH_ERR_CUDA;
  if (grid == 0) return BLOTH_OK;
  return launched(launch_ex(head_pipe_kernel<T, D, MODE>, (unsigned)grid, P::WPB * 32, P::SMEM,
                            st, a));
}

template <typename T, int D>
int launch_head_bwd(const HeadArgs& a0, void* ws, size_t ws_bytes, void* dw0, void* dw1,
                    cudaStream_t st) {
  using P = HP<T, D, kHeadNormBwd>;
  using AccT = typename AccOf<T>::type;
  TokPlan pl;
  const bool tok = qk_tok_plan<T, D, true>(a0, pl);
  const int64_t grid = tok ? qk_tok_grid<T, D, true>(a0, pl)
                           : head_pipe_grid<T, D, kHeadNormBwd>(a0.B * a0.S);
  if (grid < 0) return BLOTH_ERR_CUDA;
  const int wrc = check_workspace<AccT>(ws, (size_t)grid * 2 * D * sizeof(AccT), ws_bytes);
  if (wrc != BLOTH_OK) return wrc;
  if (grid > 0) {
    HeadArgs a = a0;
    a.partials = ws;
    int rc;
    if (tok) {
      rc = launch_qk_tok<T, D, true>(a, pl, grid, st);
    } else {
      rc = launched(launch_ex(head_pipe_kernel<T, D, kHeadNormBwd>, (unsigned)grid, P::WPB * 32,
                              P::SMEM, st, a));
    }
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
    // the head kernel's grid, or the most CTAs the token-block kernel (which
    // takes contiguous tensors; its grid depends on the head counts, which the
    // query does not know) can launch
    int64_t g = head_pipe_grid<T, DD, kHeadNormBwd>(ntok);
    if (ntok > 0) {
      const int64_t gt = qk_tok_bwd_max_grid<T, DD>();
      if (gt > g) g = gt;
    }
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
