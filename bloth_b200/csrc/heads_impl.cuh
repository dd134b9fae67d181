// Per-head kernels over [B, S, H, D] head tensors: RMSNorm of each
// (token, head) row of D followed by rotate-half RoPE, for q and k in one
// launch (NORM = true), or RoPE alone (NORM = false); forward and backward.
//
// Work split. One warp owns one token at a time (grid-stride over the B*S
// tokens). It derives the token's cos/sin once - either evaluated in-register
// from the position and inv_freq, each lane computing D/64 of the D/2 angles
// and the lanes exchanging them by shuffle, or read from a table row - and
// reuses them for every q and k head of that token. A head row of D elements
// is held by LPR lanes, one or two 16-byte vectors per lane, so a warp covers
// RPW = 32/LPR rows per step and U steps are loaded before any is consumed
// (U*16 bytes in flight per lane).
//
// Pairing. Column c pairs with c + D/2. With one vector per lane the partner
// vector sits in lane li ^ (LPR/2) of the same row group and is fetched with
// __shfl_xor_sync; with two vectors per lane (D*sizeof(T) = 1 KiB) the partner
// is the lane's other vector.
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
  int64_t B, S;
  float eps;
  int transpose;  // RoPE-only: apply R^T
};

template <typename T, int D>
struct HG {
  static constexpr int VEC = 16 / sizeof(T);
  static constexpr int NV = D / VEC;               // vectors per row
  static constexpr int LPR = NV < 32 ? NV : 32;     // lanes per row
  static constexpr int VPL = NV / LPR;              // vectors per lane
  static constexpr int RPW = 32 / LPR;              // rows per warp step
  static constexpr int HALF = D / 2;
  static constexpr int APL = HALF / 32;             // angles evaluated per lane
  static constexpr int U = 4;                       // warp steps loaded ahead (forward)
  static constexpr int UB = 2;                      // warp steps loaded ahead (backward)
  static constexpr int WPB = 8;                     // warps per CTA
  static_assert(D % (2 * VEC) == 0, "head_dim must be a multiple of 2 vectors");
  static_assert(VPL == 1 || VPL == 2, "one or two vectors per lane");
  static_assert(APL >= 1 && VEC % APL == 0, "angle split must divide the vector");
};

template <typename T, int D>
__device__ __forceinline__ bool slot_first(int j, int li) {
  using G = HG<T, D>;
  if constexpr (G::VPL == 1) return li < G::LPR / 2;
  else return j == 0;
}

// Column of element e of slot j in lane li.
template <typename T, int D>
__device__ __forceinline__ int slot_col(int j, int li) {
  using G = HG<T, D>;
  return (j * G::LPR + li) * G::VEC;
}

// Partner vector of slot j: the row's other half.
template <typename T, int D>
__device__ __forceinline__ void partner(const Pack<T, HG<T, D>::VEC> (&v)[HG<T, D>::VPL],
                                        float (&pf)[HG<T, D>::VPL][HG<T, D>::VEC]) {
  using G = HG<T, D>;
  if constexpr (G::VPL == 1) {
    uint32_t wds[4];
    memcpy(wds, &v[0], 16);
#pragma unroll
    for (int q = 0; q < 4; ++q) wds[q] = __shfl_xor_sync(0xffffffffu, wds[q], G::LPR / 2);
    Pack<T, G::VEC> pk;
    memcpy(&pk, wds, 16);
    unpack(pk, pf[0]);
  } else {
    unpack(v[1], pf[0]);
    unpack(v[0], pf[1]);
  }
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
  (void)lane;
}

// Forward over the H rows of one tensor of one token.
template <typename T, int D, bool NORM>
__device__ __forceinline__ void head_rows_fwd(const HT& src, const HT& dst, int H, int64_t b,
                                              int64_t s, float* rstd_tok,
                                              const float (&wo)[HG<T, D>::VPL][HG<T, D>::VEC],
                                              const float (&wp)[HG<T, D>::VPL][HG<T, D>::VEC],
                                              const float (&cs)[HG<T, D>::VEC],
                                              const float (&sn)[HG<T, D>::VEC], float eps,
                                              int rg, int li) {
  using G = HG<T, D>;
  const T* sbase = reinterpret_cast<const T*>(src.p) + b * src.sb + s * src.ss;
  T* dbase = reinterpret_cast<T*>(const_cast<void*>(dst.p)) + b * dst.sb + s * dst.ss;
  for (int r0 = 0; r0 < H; r0 += G::U * G::RPW) {
    Pack<T, G::VEC> xp[G::U][G::VPL];
#pragma unroll
    for (int u = 0; u < G::U; ++u) {
      const int r = r0 + u * G::RPW + rg;
#pragma unroll
      for (int j = 0; j < G::VPL; ++j) {
        if (r < H) {
          xp[u][j] = ldg_pack<T, G::VEC>(sbase + r * src.sh + slot_col<T, D>(j, li));
        } else {
#pragma unroll
          for (int e = 0; e < G::VEC; ++e) xp[u][j].v[e] = from_f<T>(0.f);
        }
      }
    }
#pragma unroll
    for (int u = 0; u < G::U; ++u) {
      const int r = r0 + u * G::RPW + rg;
      float xf[G::VPL][G::VEC], pf[G::VPL][G::VEC];
#pragma unroll
      for (int j = 0; j < G::VPL; ++j) unpack(xp[u][j], xf[j]);
      partner<T, D>(xp[u], pf);
      float rstd = 1.f;
      if constexpr (NORM) {
        float ss = 0.f;
#pragma unroll
        for (int j = 0; j < G::VPL; ++j)
#pragma unroll
          for (int e = 0; e < G::VEC; ++e) ss = fmaf(xf[j][e], xf[j][e], ss);
        ss = group_lane_sum<G::LPR>(ss);
        rstd = rsqrtf(ss / (float)D + eps);
      }
      if (r < H) {
#pragma unroll
        for (int j = 0; j < G::VPL; ++j) {
          const bool first = slot_first<T, D>(j, li);
          float o[G::VEC];
#pragma unroll
          for (int e = 0; e < G::VEC; ++e) {
            float n1 = xf[j][e], n2 = pf[j][e];
            if constexpr (NORM) {
              n1 = n1 * rstd * wo[j][e];
              n2 = n2 * rstd * wp[j][e];
            }
            o[e] = first ? (n1 * cs[e] - n2 * sn[e]) : (n2 * sn[e] + n1 * cs[e]);
          }
          stg_pack<T, G::VEC>(dbase + r * dst.sh + slot_col<T, D>(j, li), pack<T, G::VEC>(o));
        }
        if constexpr (NORM) {
          if (li == 0) rstd_tok[r] = rstd;
        }
      }
    }
  }
}

template <typename T, int D, bool NORM>
__global__ void __launch_bounds__(HG<T, D>::WPB * 32, 2) head_fwd_kernel(const HeadArgs a) {
  using G = HG<T, D>;
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int rg = lane / G::LPR;
  const int li = lane % G::LPR;
  const int pg = G::VPL == 1 ? li % (G::LPR / 2) : li;

  float invf[G::APL];
#pragma unroll
  for (int q = 0; q < G::APL; ++q) invf[q] = a.inv_freq ? __ldg(a.inv_freq + lane * G::APL + q) : 0.f;

  // weights of this lane's columns and of their partners, for q and k
  float wo[2][G::VPL][G::VEC], wp[2][G::VPL][G::VEC];
#pragma unroll
  for (int t = 0; t < 2; ++t)
#pragma unroll
    for (int j = 0; j < G::VPL; ++j)
#pragma unroll
      for (int e = 0; e < G::VEC; ++e) {
        wo[t][j][e] = 1.f;
        wp[t][j][e] = 1.f;
      }
  if constexpr (NORM) {
#pragma unroll
    for (int t = 0; t < 2; ++t) {
      if (a.H[t] == 0) continue;
#pragma unroll
      for (int j = 0; j < G::VPL; ++j) {
        const int c = slot_col<T, D>(j, li);
        const int pc = c < G::HALF ? c + G::HALF : c - G::HALF;
        ld_any_vec<G::VEC>(a.w[t], c, a.w_dt, true, wo[t][j]);
        ld_any_vec<G::VEC>(a.w[t], pc, a.w_dt, true, wp[t][j]);
      }
    }
  }

  const int64_t ntok = a.B * a.S;
  const float sgn = a.transpose ? -1.f : 1.f;
  for (int64_t t = (int64_t)blockIdx.x * G::WPB + warp; t < ntok;
       t += (int64_t)gridDim.x * G::WPB) {
    const int64_t b = t / a.S;
    const int64_t s = t - b * a.S;
    const int64_t p = token_pos<T, D>(a, b, s);
    float cs[G::VEC], sn[G::VEC];
    token_cos_sin<T, D>(a, b, p, lane, pg, invf, cs, sn);
#pragma unroll
    for (int e = 0; e < G::VEC; ++e) sn[e] *= sgn;
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      if (a.H[q] == 0) continue;
      head_rows_fwd<T, D, NORM>(a.src[q], a.dst[q], a.H[q], b, s,
                                NORM ? a.rstd_out[q] + t * a.H[q] : nullptr, wo[q], wp[q], cs, sn,
                                a.eps, rg, li);
    }
  }
}

__device__ __forceinline__ void acc_add(float& acc, float a, float b) { acc = fmaf(a, b, acc); }
__device__ __forceinline__ void acc_add(double& acc, float a, float b) {
  acc = fma((double)a, (double)b, acc);
}

// Backward (NORM) over the H rows of one tensor of one token.
template <typename T, int D>
__device__ __forceinline__ void head_rows_bwd(
    const HT& gsrc, const HT& xsrc, const HT& dst, int H, int64_t b, int64_t s,
    const float* rstd_tok, const float (&wo)[HG<T, D>::VPL][HG<T, D>::VEC],
    const float (&cs)[HG<T, D>::VEC], const float (&sn)[HG<T, D>::VEC],
    typename AccOf<T>::type (&acc)[HG<T, D>::VPL][HG<T, D>::VEC], int rg, int li) {
  using G = HG<T, D>;
  const T* gbase = reinterpret_cast<const T*>(gsrc.p) + b * gsrc.sb + s * gsrc.ss;
  const T* xbase = reinterpret_cast<const T*>(xsrc.p) + b * xsrc.sb + s * xsrc.ss;
  T* dbase = reinterpret_cast<T*>(const_cast<void*>(dst.p)) + b * dst.sb + s * dst.ss;
  for (int r0 = 0; r0 < H; r0 += G::UB * G::RPW) {
    Pack<T, G::VEC> gp[G::UB][G::VPL], xp[G::UB][G::VPL];
    float rs[G::UB];
#pragma unroll
    for (int u = 0; u < G::UB; ++u) {
      const int r = r0 + u * G::RPW + rg;
      rs[u] = r < H ? __ldg(rstd_tok + r) : 0.f;
#pragma unroll
      for (int j = 0; j < G::VPL; ++j) {
        if (r < H) {
          gp[u][j] = ldg_pack<T, G::VEC>(gbase + r * gsrc.sh + slot_col<T, D>(j, li));
          xp[u][j] = ldg_pack<T, G::VEC>(xbase + r * xsrc.sh + slot_col<T, D>(j, li));
        } else {
#pragma unroll
          for (int e = 0; e < G::VEC; ++e) {
            gp[u][j].v[e] = from_f<T>(0.f);
            xp[u][j].v[e] = from_f<T>(0.f);
          }
        }
      }
    }
#pragma unroll
    for (int u = 0; u < G::UB; ++u) {
      const int r = r0 + u * G::RPW + rg;
      const float rstd = rs[u];
      float gf[G::VPL][G::VEC], pf[G::VPL][G::VEC];
#pragma unroll
      for (int j = 0; j < G::VPL; ++j) unpack(gp[u][j], gf[j]);
      partner<T, D>(gp[u], pf);
      float g[G::VPL][G::VEC], xh[G::VPL][G::VEC];
      float dot = 0.f;
#pragma unroll
      for (int j = 0; j < G::VPL; ++j) {
        const bool first = slot_first<T, D>(j, li);
        float xf[G::VEC];
        unpack(xp[u][j], xf);
#pragma unroll
        for (int e = 0; e < G::VEC; ++e) {
          const float dn = first ? (gf[j][e] * cs[e] + pf[j][e] * sn[e])
                                 : (gf[j][e] * cs[e] - pf[j][e] * sn[e]);
          xh[j][e] = xf[e] * rstd;
          g[j][e] = dn * wo[j][e];
          dot = fmaf(g[j][e], xh[j][e], dot);
          acc_add(acc[j][e], dn, xh[j][e]);
        }
      }
      dot = group_lane_sum<G::LPR>(dot) / (float)D;
      if (r < H) {
#pragma unroll
        for (int j = 0; j < G::VPL; ++j) {
          float o[G::VEC];
#pragma unroll
          for (int e = 0; e < G::VEC; ++e) o[e] = rstd * (g[j][e] - xh[j][e] * dot);
          stg_pack<T, G::VEC>(dbase + r * dst.sh + slot_col<T, D>(j, li), pack<T, G::VEC>(o));
        }
      }
    }
  }
}

template <typename T, int D>
__global__ void __launch_bounds__(HG<T, D>::WPB * 32, 2) head_bwd_kernel(const HeadArgs a) {
  using G = HG<T, D>;
  using AccT = typename AccOf<T>::type;
  __shared__ AccT red[G::WPB][2 * D];
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int rg = lane / G::LPR;
  const int li = lane % G::LPR;
  const int pg = G::VPL == 1 ? li % (G::LPR / 2) : li;

  float invf[G::APL];
#pragma unroll
  for (int q = 0; q < G::APL; ++q) invf[q] = a.inv_freq ? __ldg(a.inv_freq + lane * G::APL + q) : 0.f;

  float wo[2][G::VPL][G::VEC];
  AccT acc[2][G::VPL][G::VEC];
#pragma unroll
  for (int t = 0; t < 2; ++t)
#pragma unroll
    for (int j = 0; j < G::VPL; ++j) {
      if (a.H[t] != 0) ld_any_vec<G::VEC>(a.w[t], slot_col<T, D>(j, li), a.w_dt, true, wo[t][j]);
      else
#pragma unroll
        for (int e = 0; e < G::VEC; ++e) wo[t][j][e] = 0.f;
#pragma unroll
      for (int e = 0; e < G::VEC; ++e) acc[t][j][e] = AccT(0);
    }

  const int64_t ntok = a.B * a.S;
  for (int64_t t = (int64_t)blockIdx.x * G::WPB + warp; t < ntok;
       t += (int64_t)gridDim.x * G::WPB) {
    const int64_t b = t / a.S;
    const int64_t s = t - b * a.S;
    const int64_t p = token_pos<T, D>(a, b, s);
    float cs[G::VEC], sn[G::VEC];
    token_cos_sin<T, D>(a, b, p, lane, pg, invf, cs, sn);
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      if (a.H[q] == 0) continue;
      head_rows_bwd<T, D>(a.src[q], a.x[q], a.dst[q], a.H[q], b, s, a.rstd_in[q] + t * a.H[q],
                          wo[q], cs, sn, acc[q], rg, li);
    }
  }

  // Weight-gradient partials: fold the row groups of each warp (lanes with
  // equal li), then the warps of the CTA in a fixed order.
#pragma unroll
  for (int t = 0; t < 2; ++t)
#pragma unroll
    for (int j = 0; j < G::VPL; ++j)
#pragma unroll
      for (int e = 0; e < G::VEC; ++e) {
#pragma unroll
        for (int o = G::LPR; o < 32; o <<= 1) acc[t][j][e] += __shfl_xor_sync(0xffffffffu, acc[t][j][e], o);
        if (rg == 0) red[warp][t * D + slot_col<T, D>(j, li) + e] = acc[t][j][e];
      }
  __syncthreads();
  AccT* part = reinterpret_cast<AccT*>(a.partials) + (int64_t)blockIdx.x * 2 * D;
  for (int c = threadIdx.x; c < 2 * D; c += G::WPB * 32) {
    AccT sum = AccT(0);
#pragma unroll
    for (int wi = 0; wi < G::WPB; ++wi) sum += red[wi][c];
    part[c] = sum;
  }
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
