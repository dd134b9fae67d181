// Per-head kernels over [B, S, H, D] head tensors: RMSNorm of each
// (token, head) row of D followed by rotate-half RoPE, for q and k in one
// launch (NORM = true), or RoPE alone (NORM = false); forward and backward.
//
// Lane layout. One warp owns one token at a time. It derives the token's
// cos/sin once - either evaluated in-register from the position and
// inv_freq, each lane computing D/64 of the D/2 angles and the lanes
// exchanging them by shuffle, or read from a table row - and reuses them for
// every q and k head of that token. A head row of D elements is held by
// LPR = D / (2 * VEC) lanes (8 at D = 128 bf16), each with two 16-byte
// vectors: columns li*VEC.. of the first half and D/2 + li*VEC.. of the
// second. A warp covers RPW = 32/LPR rows per step. The kernels themselves
// (bulk-copy pipeline) are in heads_pipe.cuh.
//
// Pairing. Column c pairs with c + D/2, which is always the lane's other
// vector: the rotation needs no data exchange between lanes, and a row's sum
// is a log2(LPR)-level butterfly.
//
// Math (fp32 throughout, one rounding on store), following the reference's
// fused kernel (bloth/bloth/kernels/fused_norm_qkv_rope.py:59-92) per row:
//   rstd = rsqrt(sum(x^2)/D + eps), n = (x*rstd)*w,
//   y_first = n1*cos - n2*sin, y_second = n1*sin + n2*cos,
// and its gradient for the backward: dn = R^T dy, then the RMSNorm backward.
// cos/sin follow BlothRoPE._build_cache (bloth/bloth/ops/rope.py:71-75):
// angle = float(pos) * inv_freq[i] in fp32.
#pragma once

#include "common.cuh"

namespace bloth {

struct HT {
  const void* p;
  int64_t sb, ss, sh;  // element strides of batch, sequence, head
};

struct HeadArgs {
  HT src[2];  // forward: q, k.  backward: dq_out, dk_out (gradients of the outputs)
  HT x[2];    // backward: q, k (forward inputs)
  HT dst[2];  // forward: q_out, k_out.  backward: dq, dk
  const void* w[2];
  int w_dt;
  float w_off;  // added to every weight: 1 for (1 + w) norms (Gemma), else 0
  int H[2];
  float* rstd_out[2];
  const float* rstd_in[2];
  void* partials;  // backward: [gridDim.x][2*D] accumulator rows
  const void* pos;
  int pos_dt;
  int64_t pos_sb, pos_ss;
  const float* inv_freq;
  const void* cos;
  const void* sin;
  int cs_dt;
  int cs_vec;
  int64_t cs_sb, cs_sp;
  int64_t cs_rows;  // rows of a table indexed by position; p is clamped to [0, cs_rows)
  float cs_scale;   // cos and sin are multiplied by this (HF attention_scaling)
  int64_t B, S;
  float eps;
  int transpose;  // RoPE-only: apply R^T
  int rstd_bulk;  // backward: rstd rows can be bulk-copied (H % 4 == 0, 16-byte aligned)
  unsigned int* fault;  // device fault word (bounded waits record timeouts here)
};

template <typename T, int D>
struct HG {
  static constexpr int VEC = 16 / sizeof(T);
  static constexpr int NV = D / VEC;               // vectors per row
  static constexpr int LPR = NV / 2;               // lanes per row
  static constexpr int VPL = 2;                    // vectors per lane: one in each half
  static constexpr int RPW = 32 / LPR;             // rows per warp step
  static constexpr int HALF = D / 2;
  static constexpr int APL = HALF / 32;            // angles evaluated per lane
  static_assert(D % (2 * VEC) == 0, "head_dim must be a multiple of 2 vectors");
  static_assert(LPR >= 1 && LPR <= 32 && (LPR & (LPR - 1)) == 0, "lanes per row: power of 2");
  static_assert(APL >= 1 && VEC % APL == 0, "angle split must divide the vector");
};

// Slot 0 of every lane lies in the first half of the row, slot 1 in the second.
template <typename T, int D>
__device__ __forceinline__ bool slot_first(int j, int li) {
  (void)li;
  return j == 0;
}

// Column of element 0 of slot j in lane li.
template <typename T, int D>
__device__ __forceinline__ int slot_col(int j, int li) {
  using G = HG<T, D>;
  return (j * G::LPR + li) * G::VEC;
}

// Partner values of both slots: each slot's partner is the lane's other slot.
template <typename T, int D>
__device__ __forceinline__ void partner(const Pack<T, HG<T, D>::VEC> (&v)[HG<T, D>::VPL],
                                        float (&pf)[HG<T, D>::VPL][HG<T, D>::VEC]) {
  unpack(v[1], pf[0]);
  unpack(v[0], pf[1]);
}

template <typename T, int D>
__device__ __forceinline__ int64_t token_pos(const HeadArgs& a, int64_t b, int64_t s) {
  if (a.pos == nullptr) return s;
  const int64_t o = b * a.pos_sb + s * a.pos_ss;
  if (a.pos_dt == BLOTH_I64) return __ldg(reinterpret_cast<const long long*>(a.pos) + o);
  return __ldg(reinterpret_cast<const int*>(a.pos) + o);
}

// cos/sin of the lane's VEC pair indices i = pg*VEC + e for one token.
template <typename T, int D>
__device__ __forceinline__ void token_cos_sin(const HeadArgs& a, int64_t b, int64_t p, int lane,
                                              int pg, const float (&invf)[HG<T, D>::APL],
                                              float (&cs)[HG<T, D>::VEC],
                                              float (&sn)[HG<T, D>::VEC]) {
  using G = HG<T, D>;
  if (a.cos != nullptr) {
    const int64_t pr = p < 0 ? 0 : (p >= a.cs_rows ? a.cs_rows - 1 : p);
    const int64_t off = b * a.cs_sb + pr * a.cs_sp + (int64_t)pg * G::VEC;
    ld_any_vec<G::VEC>(a.cos, off, a.cs_dt, a.cs_vec != 0, cs);
    ld_any_vec<G::VEC>(a.sin, off, a.cs_dt, a.cs_vec != 0, sn);
  } else {
    const float pf = (float)p;
    float cv[G::APL], sv[G::APL];
#pragma unroll
    for (int q = 0; q < G::APL; ++q) sincosf(__fmul_rn(pf, invf[q]), &sv[q], &cv[q]);
#pragma unroll
    for (int e = 0; e < G::VEC; ++e) {
      const int src = (pg * G::VEC + e) / G::APL;
      cs[e] = __shfl_sync(0xffffffffu, cv[e % G::APL], src);
      sn[e] = __shfl_sync(0xffffffffu, sv[e % G::APL], src);
    }
  }
#pragma unroll
  for (int e = 0; e < G::VEC; ++e) {
    cs[e] *= a.cs_scale;
    sn[e] *= a.cs_scale;
  }
  (void)lane;
}

__device__ __forceinline__ void acc_add(float& acc, float a, float b) { acc = fmaf(a, b, acc); }
__device__ __forceinline__ void acc_add(double& acc, float a, float b) {
  acc = fma((double)a, (double)b, acc);
}

// Host launchers, instantiated per element type in heads_<type>.cu.
template <typename T>
int heads_fwd(const HeadArgs& a, int D, bool norm, cudaStream_t st);
template <typename T>
int heads_bwd(const HeadArgs& a, int D, void* ws, size_t ws_bytes, void* dw0, void* dw1,
              cudaStream_t st);
template <typename T>
size_t heads_bwd_workspace(int64_t ntok, int D);

}  // namespace bloth
