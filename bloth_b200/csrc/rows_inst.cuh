// Host-side launchers of the row kernels for one element type. Included by
// rows_f32.cu / rows_bf16.cu / rows_f16.cu, each of which instantiates them
// for its type, so the kernel variants compile in parallel.
#pragma once

#include "rows_pipe.cuh"

namespace bloth {

template <typename T, int VEC, typename Cfg, int KIND>
int launch_row_fwd(const RowArgs& a, cudaStream_t st) {
  constexpr int BLOCK = Cfg::TPR * Cfg::RPC;
  auto kern = row_fwd_kernel<T, VEC, Cfg::TPR, Cfg::VPT, Cfg::RPC, KIND>;
  const int occ = occupancy((const void*)kern, BLOCK, 0);
  const int64_t wave = (int64_t)device_sm_count() * (occ > 0 ? occ : 1);
  const int64_t need = ceil_div(a.M, Cfg::RPC);
  const int64_t grid = need < wave ? need : wave;
  if (grid <= 0) return BLOTH_OK;
  return launched(launch_ex(kern, (unsigned)grid, BLOCK, 0, st, a));
}

template <typename T, int VEC, typename Cfg, int KIND>
int launch_row_bwd(const RowArgs& a0, void* ws, size_t ws_bytes, void* dw, cudaStream_t st) {
  using AccT = typename AccOf<T>::type;
  constexpr int BLOCK = Cfg::TPR * Cfg::RPC;
  const int64_t grid = row_bwd_grid<T, VEC, Cfg, KIND>(a0.M);
  const int wrc = check_workspace<AccT>(ws, (size_t)grid * a0.N * sizeof(AccT), ws_bytes);
  if (wrc != BLOTH_OK) return wrc;
  if (grid > 0) {
    RowArgs a = a0;
    a.partials = ws;
    auto kern = row_bwd_kernel<T, VEC, Cfg::TPR, Cfg::VPT, Cfg::RPC, KIND>;
    constexpr size_t smem = row_bwd_smem<T, VEC, Cfg>();
    const int rc = launched(launch_ex(kern, (unsigned)grid, BLOCK, smem, st, a));
    if (rc != BLOTH_OK) return rc;
  }
  return launch_dw_reduce<AccT>(reinterpret_cast<const AccT*>(ws), grid, a0.N, dw, a0.N, nullptr,
                                a0.w_dt, st);
}

// Resident CTAs per SM of the pipelined row kernels (128-thread CTAs), by
// what they compute. Measured on B200 at rows of 2048 and 4096 bf16 (same
// optimum at both): fewer CTAs than the occupancy limit stream faster for the
// kernels with two or three input tensors (e.g. the RMSNorm backward at 3 CTAs
// per SM: 133.7 us at 32768 x 4096, against 154.8 us at 4 and 157.3 us at 2).
constexpr int pipe_ctas_per_sm(int kind, bool bwd) {
  return kind == kRowAdd ? (bwd ? 3 : 2) : (bwd ? 3 : 4);
}

// Shared-memory plan of the pipelined row kernels for rows of N: a
// double-buffered ring (two slots: one block's copy in flight while the
// previous block is computed), which measured 6-10% faster than three or four
// slots at rows of 1024-8192; narrow rows (256-thread CTAs, see PipeCfg) take
// three. nst == 0 when two slots do not fit the per-CTA budget (72 KB for
// 128-thread CTAs, 112 KB for 256, 200 KB for larger), and the register
// kernels take the rows.
template <typename T, typename PC>
RowPipe pipe_plan(int N, int kind, bool bwd, bool contiguous, const RowArgs* a = nullptr) {
  RowPipe pp;
  pp.row_bytes = N * (int)sizeof(T);
  pp.slot_bytes = PC::RPC * pp.row_bytes * row_pipe_inputs(kind, bwd);
  pp.contiguous = contiguous ? 1 : 0;
  pp.fault = fault_word();
  pp.cs_row_bytes = 0;
  pp.cs_ld_bytes = 0;
  pp.cs_contiguous = 0;
  const size_t budget = PC::BLOCK <= 128 ? 72 * 1024 : (PC::BLOCK <= 256 ? 112 * 1024 : 200 * 1024);
  // narrow rows: three slots for the backward and for forward slots under
  // 8 KB, two otherwise (measured: rows of 512 bf16 forward, 87.2 vs 94.2 us)
  auto slots = [&](size_t slot_bytes) {
    const int want = PC::NARROW && (bwd || slot_bytes < 8192) ? 3 : 2;
    if ((size_t)want * (slot_bytes + 8) <= budget) return want;
    return 2 * (slot_bytes + 8) <= budget ? 2 : 0;
  };
  pp.nst = slots((size_t)pp.slot_bytes);
  // Table RoPE: stage the block's cos and sin rows in the slot too (instead
  // of a dependent global load per vector in the rotation) when they can be
  // bulk-copied: 16-byte aligned rows whose length is a multiple of 16 bytes.
  if (row_rope(kind) && a != nullptr && pp.nst > 0) {
    const int es = a->cs_dt == BLOTH_F32 ? 4 : 2;
    const int64_t row = a->half * es;
    const int64_t ld = a->ldcs * es;
    const bool aligned = reinterpret_cast<uintptr_t>(a->cos) % 16 == 0 &&
                         reinterpret_cast<uintptr_t>(a->sin) % 16 == 0;
    const size_t staged = (size_t)pp.slot_bytes + 2 * (size_t)PC::RPC * (size_t)row;
    const int nst = slots(staged);
    if (aligned && row % 16 == 0 && ld % 16 == 0 && row <= (1 << 20) && nst > 0) {
      pp.cs_row_bytes = (int)row;
      pp.cs_ld_bytes = ld;
      pp.cs_contiguous = a->ldcs == a->half ? 1 : 0;
      pp.slot_bytes = (int)staged;
      pp.nst = nst;
    }
  }
  // the staged-only kernels cannot run unstaged: leave those rows to the
  // register kernels
  if ((kind == kRowRopeVec || kind == kRowRopePair) && pp.cs_row_bytes == 0) pp.nst = 0;
  // (the per-kind caps were measured for wide rows; the paired table layout
  // runs as many CTAs as fit)
  pp.ctas_per_sm = PC::BLOCK <= 128 && kind != kRowRopePair ? pipe_ctas_per_sm(kind, bwd) : 0;
  return pp;
}

inline size_t pipe_smem(const RowPipe& pp, int N) {
  (void)N;
  return (size_t)pp.nst * (pp.slot_bytes + 8);
}

// Grid of the pipelined kernel (one wave of resident CTAs or fewer), or -1 if
// the kernel cannot be prepared on this device.
template <typename T, int VEC, typename PC, int KIND, bool BWD>
int64_t row_pipe_grid(int64_t M, int N, const RowPipe& pp) {
  auto kern = row_pipe_kernel<T, VEC, PC::TPR, PC::VPT, PC::RPC, KIND, BWD>;
  const size_t smem = pipe_smem(pp, N);
  if (prepare_smem((const void*)kern, smem) != BLOTH_OK) return -1;
  int occ = occupancy((const void*)kern, PC::BLOCK, smem);
  if (occ < 1) occ = 1;
  if (pp.ctas_per_sm > 0 && pp.ctas_per_sm < occ) occ = pp.ctas_per_sm;
  const int64_t wave = (int64_t)device_sm_count() * occ;
  const int64_t need = ceil_div(M, PC::RPC);
  return need < wave ? (need > 0 ? need : 0) : wave;
}

template <typename T, int VEC, typename PC, int KIND>
int launch_row_pipe_fwd(const RowArgs& a, const RowPipe& pp, cudaStream_t st) {
  const int64_t grid = row_pipe_grid<T, VEC, PC, KIND, false>(a.M, a.N, pp);
  if (grid < 0) return BLOTH_ERR_CUDA;
  if (grid == 0) return BLOTH_OK;
  return launched(launch_ex(row_pipe_kernel<T, VEC, PC::TPR, PC::VPT, PC::RPC, KIND, false>,
                            (unsigned)grid, PC::BLOCK, pipe_smem(pp, a.N), st, a, pp));
}

template <typename T, int VEC, typename PC, int KIND>
int launch_row_pipe_bwd(const RowArgs& a0, const RowPipe& pp, void* ws, size_t ws_bytes, void* dw,
                        cudaStream_t st) {
  using AccT = typename AccOf<T>::type;
  const int64_t grid = row_pipe_grid<T, VEC, PC, KIND, true>(a0.M, a0.N, pp);
  if (grid < 0) return BLOTH_ERR_CUDA;
  const int wrc = check_workspace<AccT>(ws, (size_t)grid * a0.N * sizeof(AccT), ws_bytes);
  if (wrc != BLOTH_OK) return wrc;
  if (grid > 0) {
    RowArgs a = a0;
    a.partials = ws;
    const int rc =
        launched(launch_ex(row_pipe_kernel<T, VEC, PC::TPR, PC::VPT, PC::RPC, KIND, true>,
                           (unsigned)grid, PC::BLOCK, pipe_smem(pp, a0.N), st, a, pp));
    if (rc != BLOTH_OK) return rc;
  }
  return launch_dw_reduce<AccT>(reinterpret_cast<const AccT*>(ws), grid, a0.N, dw, a0.N, nullptr,
                                a0.w_dt, st);
}

// Calls f(std::integral_constant<int, kind>{}) for a RowKind known at run time.
template <typename F>
int with_row_kind(int kind, F&& f) {
  switch (kind) {
    case kRowNorm: return f(std::integral_constant<int, kRowNorm>{});
    case kRowRope: return f(std::integral_constant<int, kRowRope>{});
    case kRowRopeVec: return f(std::integral_constant<int, kRowRopeVec>{});
    case kRowAdd: return f(std::integral_constant<int, kRowAdd>{});
    case kRowRopePair: return f(std::integral_constant<int, kRowRopePair>{});
    default: return BLOTH_ERR_ARG;
  }
}

// Every input row of the kind's tensors is adjacent to the next (ld == N), so
// a block of rows moves as one bulk copy.
inline bool rows_contiguous(const RowArgs& a, int kind, bool bwd) {
  if (a.ldx != a.N) return false;
  if (bwd && a.lddy != a.N) return false;
  if (kind == kRowAdd && a.ldres != a.N) return false;
  return true;
}

// Threads per row of the paired table RoPE layout for rows of 2 * half
// (one thread per VEC columns of the first half, holding their partners of
// the second half too) or, for 16-bit tensors, of 4 * half (the same, plus
// the thread's two vectors of the columns past the rotated part, as in
// rotary embeddings on half the head dimension), or 0 where the layout does
// not apply. Measured at 2^20 rows, fwd+bwd, against the one-vector staged
// kernel: bf16 rows of 128 / 256 rotated on 64 / 128 columns 257 vs 450 us /
// 495 vs 899 us; fp32 rows 540 vs 569 us / 1068 vs 975 us, so fp32 rows of
// 4 * half keep the one-vector kernel.
template <int V>
constexpr int pair_tpr(int64_t N, int64_t half) {
  if ((N != 2 * half && !(N == 4 * half && V == 8)) || half % V != 0) return 0;
  const int64_t t = half / V;
  return t == 2 || t == 4 || t == 8 || t == 16 || t == 32 ? (int)t : 0;
}

// Vectors per thread of the paired layout: 2, or 4 for rows of 4 * half.
constexpr int pair_vpt(int64_t N, int64_t half) { return N == 4 * half ? 4 : 2; }

// Calls f(RowCfg<TPR, 2, 128>{}) for the paired layout's TPR. Its pipelined
// kernels run 128-thread CTAs: the backward (112-125 registers) then fits
// 4 CTAs, 16 warps, per SM with half as many warps per block barrier as
// 2 CTAs of 256 threads (measured at 2^20 rows of 128 bf16: backward 179.1 vs
// 191.5 us, forward 129.1 us either way).
template <int VPT, typename F>
bool dispatch_pair_tpr(int tpr, F&& f) {
  switch (tpr) {
    case 2: f(RowCfg<2, VPT, 128>{}); return true;
    case 4: f(RowCfg<4, VPT, 128>{}); return true;
    case 8: f(RowCfg<8, VPT, 128>{}); return true;
    case 16: f(RowCfg<16, VPT, 128>{}); return true;
    case 32: f(RowCfg<32, VPT, 128>{}); return true;
    default: return false;
  }
}

template <typename F>
bool dispatch_pair_cfg(int tpr, int vpt, F&& f) {
  return vpt == 4 ? dispatch_pair_tpr<4>(tpr, f) : dispatch_pair_tpr<2>(tpr, f);
}

// The pipelined kernels' table RoPE without the per-element fallback, when
// the tables allow VEC-wide access everywhere and can be staged; the paired
// layout when, in addition, the whole row is rotated.
template <int V>
int pipe_kind(const RowArgs& a, int kind, bool vec) {
  if (kind != kRowRope || !vec || !a.cs_vec || a.half % V != 0) return kind;
  const int es = a.cs_dt == BLOTH_F32 ? 4 : 2;  // staging needs 16-byte table rows
  if ((a.half * es) % 16 != 0 || (a.ldcs * es) % 16 != 0) return kind;
  return pair_tpr<V>(a.N, a.half) ? kRowRopePair : kRowRopeVec;
}

template <typename T>
int rows_fwd(const RowArgs& a, int kind, bool vec, cudaStream_t st) {
  constexpr int V = 16 / sizeof(T);
  kind = pipe_kind<V>(a, kind, vec);
  return with_row_kind(kind, [&](auto kc) {
    constexpr int K = decltype(kc)::value;
    int rc = BLOTH_ERR_SHAPE;
    if (vec) {
      auto run = [&](auto cfg) {
        using C = decltype(cfg);
        using PC = PipeCfg<C::TPR, C::VPT, C::PIPE_BLOCK>;
        const RowPipe pp = pipe_plan<T, PC>(a.N, K, false, rows_contiguous(a, K, false), &a);
        rc = pp.nst > 0 ? launch_row_pipe_fwd<T, V, PC, K>(a, pp, st)
                        : launch_row_fwd<T, V, C, reg_kind(K)>(a, st);
      };
      if constexpr (K == kRowRopePair)
        dispatch_pair_cfg(pair_tpr<V>(a.N, a.half), pair_vpt(a.N, a.half), run);
      else dispatch_row_cfg<V>(a.N, run);
    } else {
      dispatch_row_cfg<1>(a.N, [&](auto cfg) {
        rc = launch_row_fwd<T, 1, decltype(cfg), reg_kind(K)>(a, st);
      });
    }
    return rc;
  });
}

template <typename T>
int rows_bwd(const RowArgs& a, int kind, bool vec, void* ws, size_t ws_bytes, void* dw,
             cudaStream_t st) {
  constexpr int V = 16 / sizeof(T);
  // the residual add without a gradient from the residual stream is the plain backward
  if (kind == kRowAdd && a.res == nullptr) kind = kRowNorm;
  kind = pipe_kind<V>(a, kind, vec);
  return with_row_kind(kind, [&](auto kc) {
    constexpr int K = decltype(kc)::value;
    int rc = BLOTH_ERR_SHAPE;
    if (vec) {
      auto run = [&](auto cfg) {
        using C = decltype(cfg);
        using PC = PipeCfg<C::TPR, C::VPT, C::PIPE_BLOCK>;
        const RowPipe pp = pipe_plan<T, PC>(a.N, K, true, rows_contiguous(a, K, true), &a);
        rc = pp.nst > 0 ? launch_row_pipe_bwd<T, V, PC, K>(a, pp, ws, ws_bytes, dw, st)
                        : launch_row_bwd<T, V, C, reg_kind(K)>(a, ws, ws_bytes, dw, st);
      };
      if constexpr (K == kRowRopePair)
        dispatch_pair_cfg(pair_tpr<V>(a.N, a.half), pair_vpt(a.N, a.half), run);
      else dispatch_row_cfg<V>(a.N, run);
    } else {
      dispatch_row_cfg<1>(a.N, [&](auto cfg) {
        rc = launch_row_bwd<T, 1, decltype(cfg), reg_kind(K)>(a, ws, ws_bytes, dw, st);
      });
    }
    return rc;
  });
}

// Workspace for the backward: the largest need of the pipelined, vector and
// scalar paths of the kind (and of the plain kind the residual add falls back
// to without dz_out), so the size depends on neither alignment nor dz_out.
template <typename T>
size_t rows_bwd_workspace(int64_t M, int N, int kind) {
  using AccT = typename AccOf<T>::type;
  constexpr int V = 16 / sizeof(T);
  int64_t grid = 0;
  auto take = [&](int64_t g) {
    if (g > grid) grid = g;
  };
  auto one_kind = [&](auto kc) {
    constexpr int K = decltype(kc)::value;
    if constexpr (K != kRowRopePair) {  // the paired layout's shapes are counted below
      dispatch_row_cfg<V>(N, [&](auto cfg) {
        using C = decltype(cfg);
        using PC = PipeCfg<C::TPR, C::VPT, C::PIPE_BLOCK>;
        take(row_bwd_grid<T, V, C, reg_kind(K)>(M));
        if (N % V == 0) {
          RowPipe pp = pipe_plan<T, PC>(N, K, true, true);
          // the staged-table kernel's plan (nst 0 here, without tables) is
          // made per call: count it too
          if (pp.nst > 0 || K == kRowRopeVec) {
            if (pp.nst > 0) take(row_pipe_grid<T, V, PC, K, true>(M, N, pp));
            // two unstaged slots: the least shared memory any plan of this
            // shape uses, so the most CTAs (staged tables may lower the count)
            pp.nst = 2;
            take(row_pipe_grid<T, V, PC, K, true>(M, N, pp));
          }
        }
      });
      dispatch_row_cfg<1>(N, [&](auto cfg) {
        take(row_bwd_grid<T, 1, decltype(cfg), reg_kind(K)>(M));
      });
    }
    return 0;
  };
  with_row_kind(kind, one_kind);
  if (kind == kRowAdd) with_row_kind(kRowNorm, one_kind);
  if (kind == kRowRope) with_row_kind(kRowRopeVec, one_kind);
  // the paired layout of rows rotated in full (half = N / 2) or in half
  // (half = N / 4), and its fallback
  for (int parts = 2; parts <= 4; parts += 2) {
    const int64_t h = N / parts;
    if (kind != kRowRope || N % parts != 0 || pair_tpr<V>(N, h) == 0) continue;
    dispatch_pair_cfg(pair_tpr<V>(N, h), pair_vpt(N, h), [&](auto cfg) {
      using C = decltype(cfg);
      using PC = PipeCfg<C::TPR, C::VPT, C::PIPE_BLOCK>;
      take(row_bwd_grid<T, V, C, kRowRope>(M));
      RowPipe pp = pipe_plan<T, PC>(N, kRowRopePair, true, true);
      pp.nst = 2;  // unstaged: the least shared memory, so the most CTAs
      take(row_pipe_grid<T, V, PC, kRowRopePair, true>(M, N, pp));
    });
  }
  return (size_t)grid * (size_t)N * sizeof(AccT);
}

}  // namespace bloth

#define BLOTH_INSTANTIATE_ROWS(T)                                                   \
  namespace bloth {                                                                 \
  template int rows_fwd<T>(const RowArgs&, int, bool, cudaStream_t);                \
  template int rows_bwd<T>(const RowArgs&, int, bool, void*, size_t, void*,         \
                           cudaStream_t);                                           \
  template size_t rows_bwd_workspace<T>(int64_t, int, int);                         \
  }
