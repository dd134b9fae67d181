// Pipelined per-head kernels: each warp streams its tokens' head rows
// global -> shared with bulk copies through a private ring of NST slots, and
// computes from shared memory.
//
// Work unit (chunk): up to R consecutive head rows of one tensor of one token,
// R = 4 KiB / row bytes forward (16 rows at D = 128 bf16), 2 KiB / row bytes
// backward (whose chunk also carries the forward input rows). A token is C0 chunks of q
// then C1 chunks of k. Warp gw owns tokens gw, gw + W, gw + 2W, ... (W = warps
// in the grid) and walks their chunks in order; before computing chunk g it
// issues the copy of chunk g + NST - 1 into the slot that chunk g - 1 has just
// released, so NST - 1 chunks (8-12 KiB per warp, 128-150 KiB per SM) are in
// flight while one is computed. The forward runs 12 warps per CTA with 4
// slots, the backward 16 warps with 3 (its chunks walk all q chunks of the
// warp's tokens, then all k chunks). Lane 0 issues one bulk copy per chunk and
// tensor when the token's heads are contiguous (head stride == D), else lanes
// issue one copy per row. The backward chunk carries the output gradient
// rows, the forward input rows and (when 16-byte aligned) the rows' rstd.
// Outputs are written with streaming stores (measured 3-5% faster here).
//
// cos/sin are derived once per token (see token_cos_sin) and the position of
// the warp's next token is loaded one token ahead. Per-row math is that of the
// reference's fused kernel (bloth/bloth/kernels/fused_norm_qkv_rope.py:59-92)
// and its exact gradient; see heads_impl.cuh.
#pragma once

#include "bulk.cuh"
#include "heads_impl.cuh"

namespace bloth {

enum HeadMode : int { kHeadNormFwd = 0, kHeadRopeFwd = 1, kHeadNormBwd = 2 };

template <typename T, int D, int MODE>
struct HP {
  using G = HG<T, D>;
  using AccT = typename AccOf<T>::type;
  static constexpr bool BWD = MODE == kHeadNormBwd;
  static constexpr int ROWB = D * (int)sizeof(T);            // bytes of one head row
  static constexpr int R = (BWD ? 2048 : 4096) / ROWB;       // rows per chunk and tensor
  static constexpr int NT = BWD ? 2 : 1;                     // tensors per chunk
  static constexpr int RSTD_OFF = NT * R * ROWB;
  static constexpr bool RSTD_BULK = BWD && (R % 4 == 0);     // rstd rows fill 16-byte units
  static constexpr int SLOT = RSTD_OFF + (BWD ? ((R * 4 + 15) / 16) * 16 : 0);
  static constexpr int NST = BWD ? 3 : 4;                    // ring slots per warp
  // shared memory of a CTA of `wpb` warps: rings, mbarriers, the fp32 weights
  // of q and k, and (backward) the q-phase weight-gradient partials per warp
  static constexpr int smem_for(int wpb) {
    return wpb * NST * SLOT + wpb * NST * 8 + 2 * D * 4 + (BWD ? wpb * D * (int)sizeof(AccT) : 0);
  }
  static constexpr int kSmemMax = 227 * 1024;
  static constexpr int WPB = !BWD ? 12 : (smem_for(16) <= kSmemMax ? 16 : (smem_for(14) <= kSmemMax ? 14 : 12));
  static constexpr int RING = WPB * NST * SLOT;
  static constexpr int BARS = RING;                          // one mbarrier per slot
  static constexpr int WSM = BARS + WPB * NST * 8;           // q and k weights, fp32 [2][D]
  static constexpr int REDQ = WSM + 2 * D * 4;               // backward: [WPB][D] q partials
  static constexpr int SMEM = smem_for(WPB);
  static_assert(R % G::RPW == 0, "chunk rows must fill whole warp steps");
  static_assert(SLOT % 16 == 0, "bulk-copy destinations must be 16-byte aligned");
  static_assert(SMEM <= kSmemMax, "ring must fit in shared memory");
};

// Per-token rotation coefficients of one lane for one tensor (forward):
// y = rstd * (x_own * alpha + x_partner * beta) with alpha = w_own * cos and
// beta = -w_partner * sin in the first half, +w_partner * sin in the second
// (y1 = n1*cos - n2*sin, y2 = n1*sin + n2*cos with n = x*rstd*w).
template <typename T, int D>
struct FwdCoef {
  float al[HG<T, D>::VPL][HG<T, D>::VEC];
  float be[HG<T, D>::VPL][HG<T, D>::VEC];
};

// Coefficients for the lane's two slots from its own-column weights w (slot
// j's partner column is slot 1-j's column, so its weight is w[1-j]).
template <typename T, int D>
__device__ __forceinline__ void make_fwd_coef(FwdCoef<T, D>& k,
                                              const float (&w)[HG<T, D>::VPL][HG<T, D>::VEC],
                                              const float (&cs)[HG<T, D>::VEC],
                                              const float (&sn)[HG<T, D>::VEC]) {
  using G = HG<T, D>;
#pragma unroll
  for (int e = 0; e < G::VEC; ++e) {
    k.al[0][e] = w[0][e] * cs[e];
    k.al[1][e] = w[1][e] * cs[e];
    k.be[0][e] = -(w[1][e] * sn[e]);  // first half:  y1 = n1*cos - n2*sin
    k.be[1][e] = w[0][e] * sn[e];     // second half: y2 = n1*sin + n2*cos
  }
}

// The lane's own-column weights of tensor `ten` from the fp32 copy in shared
// memory (all ones for RoPE alone).
template <typename T, int D, bool NORM>
__device__ __forceinline__ void lane_weights(const float* wsm, int ten, int li,
                                             float (&w)[HG<T, D>::VPL][HG<T, D>::VEC]) {
  using G = HG<T, D>;
#pragma unroll
  for (int j = 0; j < G::VPL; ++j)
#pragma unroll
    for (int e = 0; e < G::VEC; e += 4) {
      if constexpr (NORM) {
        const float4 v = *reinterpret_cast<const float4*>(wsm + ten * D + slot_col<T, D>(j, li) + e);
        w[j][e] = v.x;
        w[j][e + 1] = v.y;
        w[j][e + 2] = v.z;
        w[j][e + 3] = v.w;
      } else {
        w[j][e] = w[j][e + 1] = w[j][e + 2] = w[j][e + 3] = 1.f;
      }
    }
}

// One chunk of the forward: rows r0 .. r0+rc-1 of tensor TEN of token (b, s).
// FULL: rc == R, so every step is unrolled with compile-time offsets.
template <typename T, int D, int MODE, int TEN, bool FULL>
__device__ __forceinline__ void pipe_fwd_chunk(const HeadArgs& a, const unsigned char* slot,
                                               int64_t t, int64_t b, int64_t s, int r0, int rc,
                                               const FwdCoef<T, D>& k, int rg, int li) {
  using G = HG<T, D>;
  using P = HP<T, D, MODE>;
  constexpr bool NORM = MODE == kHeadNormFwd;
  constexpr float kInvD = 1.0f / (float)D;  // exact: D is a power of two
  const HT& dh = a.dst[TEN];
  const int64_t dsh = dh.sh;
  // lane's first element of its first row in this chunk
  T* dptr = reinterpret_cast<T*>(const_cast<void*>(dh.p)) + b * dh.sb + s * dh.ss +
            (int64_t)(r0 + rg) * dsh + slot_col<T, D>(0, li);
  const unsigned char* sptr = slot + rg * P::ROWB + slot_col<T, D>(0, li) * (int)sizeof(T);
  float* rstd_out = NORM ? a.rstd_out[TEN] + t * a.H[TEN] + r0 + rg : nullptr;
#pragma unroll
  for (int u = 0; u < P::R / G::RPW; ++u) {
    if (!FULL && u * G::RPW >= rc) break;  // partial chunk: no rows left in this step
    const int rl = u * G::RPW + rg;
    Pack<T, G::VEC> xp[G::VPL];
#pragma unroll
    for (int j = 0; j < G::VPL; ++j)
      xp[j] = lds_pack<T, G::VEC>(sptr + u * G::RPW * P::ROWB +
                                  j * G::LPR * G::VEC * (int)sizeof(T));
    float xf[G::VPL][G::VEC], pf[G::VPL][G::VEC];
#pragma unroll
    for (int j = 0; j < G::VPL; ++j) unpack(xp[j], xf[j]);
    partner<T, D>(xp, pf);
    float rstd = 1.f;
    if constexpr (NORM) {
      float2 sa = f2(0.f, 0.f), sb = f2(0.f, 0.f);
#pragma unroll
      for (int j = 0; j < G::VPL; ++j)
#pragma unroll
        for (int e = 0; e < G::VEC; e += 4) {
          const float2 x0 = f2(xf[j][e], xf[j][e + 1]), x1 = f2(xf[j][e + 2], xf[j][e + 3]);
          sa = f2_fma(x0, x0, sa);
          sb = f2_fma(x1, x1, sb);
        }
      const float ss = group_lane_sum<G::LPR>((sa.x + sa.y) + (sb.x + sb.y));
      rstd = rsqrtf(fmaf(ss, kInvD, a.eps));
    }
    if (FULL || rl < rc) {
      T* drow = dptr + (int64_t)(u * G::RPW) * dsh;
#pragma unroll
      for (int j = 0; j < G::VPL; ++j) {
        float o[G::VEC];
        const float2 r2 = f2s(rstd);
#pragma unroll
        for (int e = 0; e < G::VEC; e += 2) {
          const float2 t = f2_mul(f2(pf[j][e], pf[j][e + 1]), f2(k.be[j][e], k.be[j][e + 1]));
          const float2 y = f2_mul(
              f2_fma(f2(xf[j][e], xf[j][e + 1]), f2(k.al[j][e], k.al[j][e + 1]), t), r2);
          o[e] = y.x;
          o[e + 1] = y.y;
        }
        stg_pack_stream<T, G::VEC>(drow + j * G::LPR * G::VEC, pack<T, G::VEC>(o));
      }
      if constexpr (NORM) {
        if (li == 0) rstd_out[u * G::RPW] = rstd;
      }
    }
  }
}

// One chunk of the backward: dn = R^T dy = dy_own*cos + dy_partner*sin in
// the first half (slot 0), dy_own*cos - dy_partner*sin in the second
// (slot 1); g = dn*w, dx = rstd*(g - xhat*sum(g*xhat)/D), dweight += dn*xhat.
template <typename T, int D, bool FULL>
__device__ __forceinline__ void pipe_bwd_chunk(
    const HeadArgs& a, int TEN, const unsigned char* slot, int64_t t, int64_t b, int64_t s, int r0,
    int rc, const float (&wo)[HG<T, D>::VPL][HG<T, D>::VEC], const float (&cs)[HG<T, D>::VEC],
    const float (&sn)[HG<T, D>::VEC], const float (&snn)[HG<T, D>::VEC],
    typename AccOf<T>::type (&acc)[HG<T, D>::VPL][HG<T, D>::VEC], int rg, int li) {
  using G = HG<T, D>;
  using P = HP<T, D, kHeadNormBwd>;
  constexpr float kInvD = 1.0f / (float)D;
  const HT& dh = a.dst[TEN];
  const int64_t dsh = dh.sh;
  T* dptr = reinterpret_cast<T*>(const_cast<void*>(dh.p)) + b * dh.sb + s * dh.ss +
            (int64_t)(r0 + rg) * dsh + slot_col<T, D>(0, li);
  const unsigned char* gptr = slot + rg * P::ROWB + slot_col<T, D>(0, li) * (int)sizeof(T);
  const unsigned char* xptr = gptr + P::R * P::ROWB;
  const float* rstd_smem = reinterpret_cast<const float*>(slot + P::RSTD_OFF) + rg;
  const float* rstd_src = a.rstd_in[TEN] + t * a.H[TEN] + r0 + rg;
  const bool rstd_in_smem = P::RSTD_BULK && a.rstd_bulk;
#pragma unroll
  for (int u = 0; u < P::R / G::RPW; ++u) {
    if (!FULL && u * G::RPW >= rc) break;  // partial chunk: no rows left in this step
    const int rl = u * G::RPW + rg;
    const bool valid = FULL || rl < rc;
    const float rstd = rstd_in_smem ? rstd_smem[u * G::RPW]
                                    : (valid ? __ldg(rstd_src + u * G::RPW) : 0.f);
    Pack<T, G::VEC> gp[G::VPL], xp[G::VPL];
#pragma unroll
    for (int j = 0; j < G::VPL; ++j) {
      const int off = u * G::RPW * P::ROWB + j * G::LPR * G::VEC * (int)sizeof(T);
      gp[j] = lds_pack<T, G::VEC>(gptr + off);
      xp[j] = lds_pack<T, G::VEC>(xptr + off);
    }
    float gf[G::VPL][G::VEC], pf[G::VPL][G::VEC];
#pragma unroll
    for (int j = 0; j < G::VPL; ++j) unpack(gp[j], gf[j]);
    partner<T, D>(gp, pf);
    float g[G::VPL][G::VEC], xh[G::VPL][G::VEC];
    float2 da = f2(0.f, 0.f), db = f2(0.f, 0.f);
    const float2 r2 = f2s(rstd);
#pragma unroll
    for (int j = 0; j < G::VPL; ++j) {
      float xf[G::VEC];
      unpack(xp[j], xf);
#pragma unroll
      for (int e = 0; e < G::VEC; e += 2) {
        // slot 0: dn = dy*cos + dy_p*sin; slot 1: dn = dy*cos - dy_p*sin
        const float2 s2 = j == 0 ? f2(sn[e], sn[e + 1]) : f2(snn[e], snn[e + 1]);
        const float2 dn = f2_fma(f2(pf[j][e], pf[j][e + 1]), s2,
                                 f2_mul(f2(gf[j][e], gf[j][e + 1]), f2(cs[e], cs[e + 1])));
        const float2 x2 = f2_mul(f2(xf[e], xf[e + 1]), r2);
        const float2 g2 = f2_mul(dn, f2(wo[j][e], wo[j][e + 1]));
        if ((e / 2) & 1) db = f2_fma(g2, x2, db);
        else da = f2_fma(g2, x2, da);
        xh[j][e] = x2.x;
        xh[j][e + 1] = x2.y;
        g[j][e] = g2.x;
        g[j][e + 1] = g2.y;
        if (valid) {
          if constexpr (std::is_same<typename AccOf<T>::type, float>::value) {
            const float2 a2 = f2_fma(dn, x2, f2(acc[j][e], acc[j][e + 1]));
            acc[j][e] = a2.x;
            acc[j][e + 1] = a2.y;
          } else {
            acc_add(acc[j][e], dn.x, x2.x);
            acc_add(acc[j][e + 1], dn.y, x2.y);
          }
        }
      }
    }
    const float dot = group_lane_sum<G::LPR>((da.x + da.y) + (db.x + db.y)) * kInvD;
    if (valid) {
      T* drow = dptr + (int64_t)(u * G::RPW) * dsh;
#pragma unroll
      for (int j = 0; j < G::VPL; ++j) {
        float o[G::VEC];
        const float2 nd = f2s(-dot);
#pragma unroll
        for (int e = 0; e < G::VEC; e += 2) {
          const float2 y = f2_mul(
              f2_fma(f2(xh[j][e], xh[j][e + 1]), nd, f2(g[j][e], g[j][e + 1])), r2);
          o[e] = y.x;
          o[e + 1] = y.y;
        }
        stg_pack_stream<T, G::VEC>(drow + j * G::LPR * G::VEC, pack<T, G::VEC>(o));
      }
    }
  }
}

// Fold a warp's per-lane weight-gradient accumulators of one tensor: add the
// row groups (lanes with equal li) in a fixed butterfly order, then lanes of
// row group 0 store the warp's D totals to dst[0..D).
template <typename T, int D>
__device__ __forceinline__ void fold_warp_acc(
    typename AccOf<T>::type (&acc)[HG<T, D>::VPL][HG<T, D>::VEC], typename AccOf<T>::type* dst,
    int rg, int li) {
  using G = HG<T, D>;
#pragma unroll
  for (int j = 0; j < G::VPL; ++j)
#pragma unroll
    for (int e = 0; e < G::VEC; ++e) {
#pragma unroll
      for (int o = G::LPR; o < 32; o <<= 1)
        acc[j][e] += __shfl_xor_sync(0xffffffffu, acc[j][e], o);
      if (rg == 0) dst[slot_col<T, D>(j, li) + e] = acc[j][e];
    }
}

template <typename T, int D, int MODE>
__global__ void __launch_bounds__(HP<T, D, MODE>::WPB * 32, 1)
    head_pipe_kernel(const HeadArgs a) {
  using G = HG<T, D>;
  using P = HP<T, D, MODE>;
  using AccT = typename AccOf<T>::type;
  constexpr bool BWD = MODE == kHeadNormBwd;
  constexpr bool NORM = MODE != kHeadRopeFwd;
  extern __shared__ __align__(128) unsigned char smem[];
  if constexpr (BWD) allow_dependent_launch();  // the dweight reduce waits for this grid
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int rg = lane / G::LPR;
  const int li = lane % G::LPR;
  const int pg = li;  // the lane's pair indices are li*VEC .. li*VEC+VEC-1
  unsigned char* ring = smem + warp * P::NST * P::SLOT;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + P::BARS) + warp * P::NST;
  if (lane == 0) {
#pragma unroll
    for (int q = 0; q < P::NST; ++q) mbar_init(&bars[q], 1);
    mbar_init_fence();
  }
  __syncwarp();

  float invf[G::APL];
#pragma unroll
  for (int q = 0; q < G::APL; ++q)
    invf[q] = a.inv_freq ? __ldg(a.inv_freq + lane * G::APL + q) : 0.f;


  const int C[2] = {(a.H[0] + P::R - 1) / P::R, (a.H[1] + P::R - 1) / P::R};
  // token counts fit in 32 bits (the host rejects B*S >= 2^31)
  const int ntok = (int)(a.B * a.S);
  const int S = (int)a.S;
  const int W = (int)gridDim.x * P::WPB;
  const int gw = (int)blockIdx.x * P::WPB + warp;
  const int my_tok = gw < ntok ? (ntok - 1 - gw) / W + 1 : 0;
  const int b0 = my_tok > 0 ? gw / S : 0;
  const int s0 = gw - b0 * S;

  // Chunk walk. Forward: token-major (a token's q chunks, then its k chunks).
  // Backward: tensor-major (all of the warp's q chunks, then all its k chunks),
  // so only one tensor's weights and weight-gradient sums are live at a time.
  struct Cursor {
    int t, b, s, ti, left, j, ten;
  };
  auto advance = [&](Cursor& c) {
    --c.left;
    const int cnt = BWD ? C[c.ten] : C[0] + C[1];
    if (++c.j < cnt) return;
    c.j = 0;
    if (BWD && ++c.ti == my_tok) {  // q phase done: restart the tokens for k
      c.ti = 0;
      c.ten = 1;
      c.t = gw;
      c.b = b0;
      c.s = s0;
      return;
    }
    if (!BWD) ++c.ti;
    c.t += W;
    c.s += W;
    if (c.s >= S) {
      const int q = (int)((unsigned)c.s / (unsigned)S);
      c.b += q;
      c.s -= q * S;
    }
  };
  // tensor, first row and row count of the chunk under the cursor
  auto chunk_of = [&](const Cursor& c, int& ten, int& r0, int& rc) {
    if (BWD) {
      ten = c.ten;
      r0 = c.j * P::R;
    } else {
      ten = c.j < C[0] ? 0 : 1;
      r0 = (ten == 0 ? c.j : c.j - C[0]) * P::R;
    }
    rc = min(P::R, a.H[ten] - r0);
  };

  // Issues the chunk under `c` into ring slot `sl`.
  auto issue = [&](const Cursor& c, int sl) {
    int ten, r0, rc;
    chunk_of(c, ten, r0, rc);
    unsigned char* dst = ring + sl * P::SLOT;
    uint64_t* bar = &bars[sl];
    const bool rstd_copy = P::RSTD_BULK && a.rstd_bulk;
    const uint32_t bytes = (uint32_t)(rc * P::ROWB * P::NT) + (rstd_copy ? (uint32_t)rc * 4u : 0u);
    if (lane == 0) mbar_arrive_expect_tx(bar, bytes);
    __syncwarp();
#pragma unroll
    for (int q = 0; q < P::NT; ++q) {
      const HT& h = q == 0 ? a.src[ten] : a.x[ten];
      const T* base = reinterpret_cast<const T*>(h.p) + (int64_t)c.b * h.sb +
                      (int64_t)c.s * h.ss + (int64_t)r0 * h.sh;
      unsigned char* d = dst + q * P::R * P::ROWB;
      if (h.sh == D) {
        if (lane == 0) bulk_load(d, base, (uint32_t)(rc * P::ROWB), bar);
      } else if (lane < rc) {
        bulk_load(d + lane * P::ROWB, base + (int64_t)lane * h.sh, (uint32_t)P::ROWB, bar);
      }
    }
    if (rstd_copy && lane == 0)
      bulk_load(dst + P::RSTD_OFF, a.rstd_in[ten] + (int64_t)c.t * a.H[ten] + r0, (uint32_t)rc * 4u,
                bar);
  };

  const int nchunk = my_tok * (C[0] + C[1]);
  Cursor cc{gw, b0, s0, 0, nchunk, 0, 0};
  Cursor ic = cc;  // issue cursor, NST - 1 chunks ahead
  int isl = 0;
  int inflight = 0;  // chunks issued and not yet computed
  // the first NST - 1 chunks go out before anything waits on memory, so their
  // latency overlaps the weight loads below
  for (int q = 0; q < P::NST - 1 && ic.left > 0; ++q) {
    issue(ic, isl);
    advance(ic);
    ++inflight;
    isl = isl + 1 == P::NST ? 0 : isl + 1;
  }

  // Weights of q and k as fp32 in shared memory, shared by the CTA's warps.
  float* wsm = reinterpret_cast<float*>(smem + P::WSM);
  if constexpr (NORM) {
    for (int c = threadIdx.x; c < 2 * D; c += P::WPB * 32) {
      const int q = c / D;
      wsm[c] = a.H[q] != 0 ? ld_any(a.w[q], c - q * D, a.w_dt) + a.w_off : 0.f;
    }
  }
  __syncthreads();

  float cs[G::VEC], sn[G::VEC];
  float snn[G::VEC];         // backward: -sin
  FwdCoef<T, D> kc;          // forward: coefficients of the current tensor and token
  float wc[G::VPL][G::VEC];  // backward: weights of the current tensor
  AccT acc[G::VPL][G::VEC];  // backward: weight-gradient sums of the current tensor
#pragma unroll
  for (int j = 0; j < G::VPL; ++j)
#pragma unroll
    for (int e = 0; e < G::VEC; ++e) acc[j][e] = AccT(0);
  AccT* redq = reinterpret_cast<AccT*>(smem + P::REDQ) + warp * D;  // backward only
  int cur_ten = -1;
  int64_t pos_next = 0;
  const float sgn = a.transpose ? -1.f : 1.f;
  int csl = 0;
  uint32_t cph = 0;
  while (cc.left > 0) {
    if (ic.left > 0) {
      issue(ic, isl);
      advance(ic);
      ++inflight;
      isl = isl + 1 == P::NST ? 0 : isl + 1;
    }
    int ten, r0, rc;
    chunk_of(cc, ten, r0, rc);
    if (BWD && ten != cur_ten) {  // phase start: this tensor's weights, first token's position
      if (cur_ten == 0) {
        fold_warp_acc<T, D>(acc, redq, rg, li);
#pragma unroll
        for (int j = 0; j < G::VPL; ++j)
#pragma unroll
          for (int e = 0; e < G::VEC; ++e) acc[j][e] = AccT(0);
      }
      cur_ten = ten;
      lane_weights<T, D, NORM>(wsm, ten, li, wc);
      pos_next = token_pos<T, D>(a, cc.b, cc.s);
    }
    if (!BWD && cur_ten < 0) {
      cur_ten = 0;
      pos_next = token_pos<T, D>(a, cc.b, cc.s);
    }
    if (cc.j == 0) {  // token start: cos/sin, and the next token's position
      const int64_t p = pos_next;
      if (cc.ti + 1 < my_tok) {
        int s2 = cc.s + W, b2 = cc.b;
        if (s2 >= S) {
          const int q = (int)((unsigned)s2 / (unsigned)S);
          b2 += q;
          s2 -= q * S;
        }
        pos_next = token_pos<T, D>(a, b2, s2);
      }
      token_cos_sin<T, D>(a, cc.b, p, lane, pg, invf, cs, sn);
      if constexpr (MODE == kHeadRopeFwd) {
#pragma unroll
        for (int e = 0; e < G::VEC; ++e) sn[e] *= sgn;
      }
      if constexpr (BWD) {
#pragma unroll
        for (int e = 0; e < G::VEC; ++e) snn[e] = -sn[e];
      }
    }
    if (!BWD && (cc.j == 0 || cc.j == C[0])) {  // forward: coefficients of this tensor
      float w[G::VPL][G::VEC];
      lane_weights<T, D, NORM>(wsm, ten, li, w);
      make_fwd_coef<T, D>(kc, w, cs, sn);
    }
    const bool landed = mbar_wait(&bars[csl], cph, a.fault);
    if (!__all_sync(0xffffffffu, landed)) {
      // give up the rest of the work, but not before the copies already
      // issued into this warp's ring have landed
      drain_ring(bars, P::NST, csl, cph, inflight, a.fault);
      break;
    }
    --inflight;
    const unsigned char* slot = ring + csl * P::SLOT;
    if constexpr (BWD) {
      if (rc == P::R)
        pipe_bwd_chunk<T, D, true>(a, ten, slot, cc.t, cc.b, cc.s, r0, rc, wc, cs, sn, snn, acc, rg, li);
      else
        pipe_bwd_chunk<T, D, false>(a, ten, slot, cc.t, cc.b, cc.s, r0, rc, wc, cs, sn, snn, acc, rg, li);
    } else {
      if (rc == P::R) {
        if (ten == 0) pipe_fwd_chunk<T, D, MODE, 0, true>(a, slot, cc.t, cc.b, cc.s, r0, rc, kc, rg, li);
        else pipe_fwd_chunk<T, D, MODE, 1, true>(a, slot, cc.t, cc.b, cc.s, r0, rc, kc, rg, li);
      } else {
        if (ten == 0) pipe_fwd_chunk<T, D, MODE, 0, false>(a, slot, cc.t, cc.b, cc.s, r0, rc, kc, rg, li);
        else pipe_fwd_chunk<T, D, MODE, 1, false>(a, slot, cc.t, cc.b, cc.s, r0, rc, kc, rg, li);
      }
    }
    // release the slot: order this lane's reads before the next bulk write
    fence_proxy_async_smem();
    __syncwarp();
    advance(cc);
    if (++csl == P::NST) {
      csl = 0;
      cph ^= 1u;
    }
  }

  if constexpr (BWD) {
    // q partials are in redq; the k partials (or q's, when the warp ended in
    // the q phase) go to the idle ring memory. Then fold the warps of the CTA
    // in a fixed order into this CTA's partial row [q D | k D].
    __syncthreads();
    AccT* redk = reinterpret_cast<AccT*>(smem);  // [WPB][D]
    if (cur_ten == 1) {
      fold_warp_acc<T, D>(acc, redk + warp * D, rg, li);
    } else {
      fold_warp_acc<T, D>(acc, redq, rg, li);  // q phase only (or no tokens)
      if (rg == 0)
#pragma unroll
        for (int j = 0; j < G::VPL; ++j)
#pragma unroll
          for (int e = 0; e < G::VEC; ++e) redk[warp * D + slot_col<T, D>(j, li) + e] = AccT(0);
    }
    __syncthreads();
    const AccT* redq0 = reinterpret_cast<const AccT*>(smem + P::REDQ);
    AccT* part = reinterpret_cast<AccT*>(a.partials) + (int64_t)blockIdx.x * 2 * D;
    for (int c = threadIdx.x; c < 2 * D; c += P::WPB * 32) {
      const AccT* src = c < D ? redq0 + c : redk + (c - D);
      AccT sum = AccT(0);
#pragma unroll
      for (int wi = 0; wi < P::WPB; ++wi) sum += src[wi * D];
      part[c] = sum;
    }
  }
}

}  // namespace bloth
