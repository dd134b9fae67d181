// Per-head q/k RMSNorm + RoPE for contiguous head tensors, in token blocks.
//
// q [B, S, Hq, D] and k [B, S, Hk, D], contiguous, are [B*S*H, D] rows,
// token-major. A block is TB consecutive tokens: their Hq q rows and Hk k
// rows, which are two contiguous runs of memory, so a block moves global ->
// shared as one bulk copy per tensor (plus, backward, one per forward input
// and one per rstd run) into a ring of NST slots, NST - 1 blocks ahead of
// the one computed. CTAs take blocks c, c + G, c + 2G, ... (G = grid size).
//
// Layout (paired): a row is held by TPR = (D/2)/VEC threads, each with two
// 16-byte vectors, columns lt*VEC.. of the first half and D/2 + lt*VEC.. of
// the second, so a column's rotation partner is in the same thread. The 128
// threads of a CTA form RG = 128/TPR row groups; group g computes rows g,
// g + RG, ... of the block's q run and then of its k run (every group runs
// the same number of steps, so the row-sum shuffles always have the whole
// warp; rows past the run compute on stale bytes and store nothing). The
// token of a row follows from a cursor advanced by RG rows per step (no
// division in the loop).
//
// cos/sin. The block's TB tokens need TB * D/2 angles, shared by q and k:
// thread tid evaluates angle i = tid % (D/2) of tokens tid / (D/2) +
// m * 128/(D/2), m < APT (the host keeps TB * D/2 <= 128 * APT),
// angle = float(pos) * inv_freq[i] in fp32 (BlothRoPE._build_cache,
// bloth/bloth/ops/rope.py:71-75), sincosf, times rope_scale, into shared
// memory before the block's barrier. Positions are loaded one block ahead.
//
// Math per row, fp32 with one rounding on store, as the reference's fused row
// kernel (bloth/bloth/kernels/fused_norm_qkv_rope.py:59-92) and its exact
// gradient:
//   forward:  rstd = rsqrt(sum(x^2)/D + eps), a = x*w,
//             y_c = rstd*(a_c cos - a_p sin), y_p = rstd*(a_p cos + a_c sin)
//   backward: dn_c = dy_c cos + dy_p sin, dn_p = dy_p cos - dy_c sin,
//             g = dn*w, xhat = x*rstd, dx = rstd*(g - xhat*sum(g*xhat)/D),
//             dweight += dn*xhat (per-thread sums for q and for k, folded
//             per CTA in a fixed order into one partial row [q D | k D],
//             reduced by dw_reduce_kernel).
#pragma once

#include "bulk.cuh"
#include "heads_impl.cuh"

namespace bloth {

// n / d for 0 <= n < 2^31 without a division: m = ceil(2^(31+l) / d) with
// l = ceil(log2 d) fits in 32 bits, and floor(n * m / 2^(31+l)) == n / d
// because n * (m*d - 2^(31+l)) < 2^31 * d <= 2^(31+l) (the multiply-shift
// method of Granlund and Montgomery, 1994).
struct FastDiv {
  uint32_t m;
  int shift;
  static FastDiv make(uint32_t d) {
    int l = 0;
    while ((1ull << l) < d) ++l;
    FastDiv f;
    f.m = (uint32_t)(((1ull << (31 + l)) + d - 1) / d);
    f.shift = 31 + l;
    return f;
  }
  __device__ __forceinline__ uint32_t div(uint32_t n) const {
    return (uint32_t)(((uint64_t)n * m) >> shift);
  }
};

// Launch plan of the token-block kernels (host-chosen).
struct TokPlan {
  int tb;    // tokens per block
  int nst;   // ring slots
  int slot;  // bytes per slot (a multiple of 16)
  FastDiv s_div;  // token -> (batch row, sequence index)
};

template <typename T, int D, bool BWD>
struct QT {
  using AccT = typename AccOf<T>::type;
  static constexpr int VEC = 16 / (int)sizeof(T);
  static constexpr int HALF = D / 2;
  static constexpr int TPR = HALF / VEC;  // threads per row
  static constexpr int BLOCK = 128;
  static constexpr int RG = BLOCK / TPR;  // row groups
  static constexpr int ROWB = D * (int)sizeof(T);
  static constexpr int NT = BWD ? 2 : 1;   // row tensors per block and head set
  static constexpr int APT = 2;            // angles per thread and block, at most
  static constexpr int TBMAX = APT * BLOCK / HALF;
  static constexpr int WARPS = BLOCK / 32;
  static constexpr int CS_FLOATS = TBMAX * HALF;
  // bytes of one slot for TB tokens (rows of each tensor, then fp32 rstd runs)
  static int slot_bytes(int tb, int hq, int hk) {
    const int rows = tb * (hq + hk);
    const int b = rows * ROWB * NT + (BWD ? rows * 4 : 0);
    return (b + 15) / 16 * 16;
  }
  // shared memory after the ring (nst * slot bytes): cos and sin
  // [TBMAX][HALF] fp32 (16-byte aligned), the weight-gradient totals
  // [WARPS][2D] (backward), then the ring's mbarriers
  static constexpr int TAB_BYTES = 2 * CS_FLOATS * 4;
  static constexpr int RED_BYTES = BWD ? WARPS * 2 * D * (int)sizeof(AccT) : 0;
  __host__ __device__ static size_t tab_off(int nst, int slot) { return (size_t)nst * slot; }
  __host__ __device__ static size_t red_off(int nst, int slot) {
    return tab_off(nst, slot) + TAB_BYTES;
  }
  __host__ __device__ static size_t bar_off(int nst, int slot) {
    return red_off(nst, slot) + RED_BYTES;
  }
  __host__ __device__ static size_t smem(int nst, int slot) {
    return bar_off(nst, slot) + (size_t)nst * 8;
  }
  static_assert(TPR >= 2 && TPR <= 32 && (TPR & (TPR - 1)) == 0, "threads per row");
  static_assert(32 % TPR == 0, "row groups must not straddle warps");
  static_assert(BLOCK % HALF == 0, "every angle of a token lands on one thread per token");
  static_assert(ROWB % 16 == 0 && (CS_FLOATS * 4) % 16 == 0, "16-byte units");
  static_assert(TAB_BYTES % 8 == 0 && RED_BYTES % 8 == 0, "mbarriers need 8-byte alignment");
};

// Index of pair i's cos (or sin) of block token j in the shared table. The
// VEC pairs a thread reads are split in 16-byte planes, so that the TPR
// threads of a row read consecutive 16-byte units.
template <typename T, int D>
__device__ __forceinline__ int qt_cs_index(int j, int i) {
  using Q = QT<T, D, false>;
  const int lt = i / Q::VEC, q = (i % Q::VEC) / 4, r = i % 4;
  return j * Q::HALF + q * (Q::TPR * 4) + lt * 4 + r;
}

template <typename T, int D>
__device__ __forceinline__ void qt_load_cs(const float* tab, int j, int lt,
                                           float (&v)[QT<T, D, false>::VEC]) {
  using Q = QT<T, D, false>;
#pragma unroll
  for (int q = 0; q < Q::VEC / 4; ++q) {
    const float4 f =
        *reinterpret_cast<const float4*>(tab + j * Q::HALF + q * (Q::TPR * 4) + lt * 4);
    v[4 * q] = f.x;
    v[4 * q + 1] = f.y;
    v[4 * q + 2] = f.z;
    v[4 * q + 3] = f.w;
  }
}

// Cursor over the rows g, g + RG, ... of a run of rows of H heads: the token
// (within the block) of the current row, advanced without a division.
struct RowCursor {
  int j, rem, dj, dr, h;
  __device__ __forceinline__ void init(int g, int step, int H) {
    h = H;
    j = g / H;
    rem = g - j * H;
    dj = step / H;
    dr = step - dj * H;
  }
  __device__ __forceinline__ void next() {
    j += dj;
    rem += dr;
    if (rem >= h) {
      rem -= h;
      ++j;
    }
  }
};

template <typename T, int D, bool BWD>
__global__ void __launch_bounds__(128, BWD ? 3 : 4)
    qk_token_kernel(const HeadArgs a, const TokPlan pl) {
  using Q = QT<T, D, BWD>;
  using AccT = typename Q::AccT;
  constexpr int VEC = Q::VEC, TPR = Q::TPR, RG = Q::RG, HALF = Q::HALF, ROWB = Q::ROWB;
  constexpr float kInvD = 1.0f / (float)D;  // exact: D is a power of two
  extern __shared__ __align__(128) unsigned char smem[];
  const int tid = threadIdx.x;
  const int grp = tid / TPR;
  const int lt = tid % TPR;
  const int nst = pl.nst, TB = pl.tb;
  if constexpr (BWD) allow_dependent_launch();  // the dweight reduce waits for this grid
  float* cs_tab = reinterpret_cast<float*>(smem + Q::tab_off(nst, pl.slot));
  float* sn_tab = cs_tab + Q::CS_FLOATS;
  AccT* red = reinterpret_cast<AccT*>(smem + Q::red_off(nst, pl.slot));  // [WARPS][2D]
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Q::bar_off(nst, pl.slot));
  if (tid == 0) {
    for (int q = 0; q < nst; ++q) mbar_init(&bars[q], 1);
    mbar_init_fence();
  }

  const int Hq = a.H[0], Hk = a.H[1];
  const int ntok = (int)(a.B * a.S);  // < 2^31 / max(Hq, Hk) (host check)
  const int S = (int)a.S;
  const int nblk = (ntok + TB - 1) / TB;
  const int G = (int)gridDim.x;
  const int my_blk = (int)blockIdx.x < nblk ? (nblk - 1 - (int)blockIdx.x) / G + 1 : 0;
  // slot regions: rows of q then k (gradients of the outputs, backward), then
  // (backward) the forward inputs q, k, then the rstd runs of q and k
  const int oq = 0, ok = TB * Hq * ROWB;
  const int ox = TB * (Hq + Hk) * ROWB;
  const int orq = BWD ? 2 * ox : 0, ork = orq + TB * Hq * 4;

  // the thread's angles: pair ai of block tokens aj + m * (128 / HALF)
  const int ai = tid % HALF, aj = tid / HALF;
  const float inv_f = __ldg(a.inv_freq + ai);
  auto pos_of = [&](int t) -> int64_t {
    const int bb = (int)pl.s_div.div((uint32_t)t);
    const int ss = t - bb * S;
    if (a.pos == nullptr) return ss;
    const int64_t o = (int64_t)bb * a.pos_sb + (int64_t)ss * a.pos_ss;
    if (a.pos_dt == BLOTH_I64) return __ldg(reinterpret_cast<const long long*>(a.pos) + o);
    return __ldg(reinterpret_cast<const int*>(a.pos) + o);
  };

  const uint64_t pol = BWD ? 0ull : evict_first_policy();
  // thread 0 issues local block i into ring slot sl
  auto issue = [&](int i, int sl) {
    if (i >= my_blk || tid != 0) return;
    const int t0 = ((int)blockIdx.x + i * G) * TB;
    const int nt = min(TB, ntok - t0);
    unsigned char* dst = smem + (size_t)sl * pl.slot;
    const uint32_t bq = (uint32_t)(nt * Hq * ROWB), bk = (uint32_t)(nt * Hk * ROWB);
    const uint32_t rs = BWD ? (uint32_t)(nt * (Hq + Hk) * 4) : 0u;
    mbar_arrive_expect_tx(&bars[sl], (bq + bk) * Q::NT + rs);
#pragma unroll
    for (int q = 0; q < Q::NT; ++q) {
      const HT& hq = q == 0 ? a.src[0] : a.x[0];
      const HT& hk = q == 0 ? a.src[1] : a.x[1];
      unsigned char* d = dst + q * ox;
      if (bq) {
        const T* s = reinterpret_cast<const T*>(hq.p) + (int64_t)t0 * Hq * D;
        if constexpr (BWD) bulk_load(d + oq, s, bq, &bars[sl]);
        else bulk_load_hint(d + oq, s, bq, &bars[sl], pol);
      }
      if (bk) {
        const T* s = reinterpret_cast<const T*>(hk.p) + (int64_t)t0 * Hk * D;
        if constexpr (BWD) bulk_load(d + ok, s, bk, &bars[sl]);
        else bulk_load_hint(d + ok, s, bk, &bars[sl], pol);
      }
    }
    if constexpr (BWD) {
      if (Hq) bulk_load(dst + orq, a.rstd_in[0] + (int64_t)t0 * Hq, (uint32_t)(nt * Hq * 4), &bars[sl]);
      if (Hk) bulk_load(dst + ork, a.rstd_in[1] + (int64_t)t0 * Hk, (uint32_t)(nt * Hk * 4), &bars[sl]);
    }
  };

  // the thread's weights (own columns) of q and k
  float wq0[VEC], wq1[VEC], wk0[VEC], wk1[VEC];
  auto load_w = [&](int ten, float (&w0)[VEC], float (&w1)[VEC]) {
    if (a.H[ten] == 0) {
#pragma unroll
      for (int e = 0; e < VEC; ++e) w0[e] = w1[e] = 0.f;
      return;
    }
    ld_any_vec<VEC>(a.w[ten], lt * VEC, a.w_dt, true, w0);
    ld_any_vec<VEC>(a.w[ten], HALF + lt * VEC, a.w_dt, true, w1);
#pragma unroll
    for (int e = 0; e < VEC; ++e) {
      w0[e] += a.w_off;
      w1[e] += a.w_off;
    }
  };
  // the first NST - 1 blocks go out before anything waits on memory, so their
  // latency overlaps the weight loads
  for (int q = 0; q < nst - 1; ++q) issue(q, q);
  load_w(0, wq0, wq1);
  load_w(1, wk0, wk1);

  AccT aq0[VEC], aq1[VEC], ak0[VEC], ak1[VEC];
#pragma unroll
  for (int e = 0; e < VEC; ++e) aq0[e] = aq1[e] = ak0[e] = ak1[e] = AccT(0);
  __syncthreads();  // barrier init visible before any wait

  // steps per block of each run (the same for every row group), and the row
  // group's cursor at the first step of a run (the same for every block)
  const int steps_q = (TB * Hq + RG - 1) / RG, steps_k = (TB * Hk + RG - 1) / RG;
  RowCursor cur0[2];
  cur0[0].init(grp, RG, Hq > 0 ? Hq : 1);
  cur0[1].init(grp, RG, Hk > 0 ? Hk : 1);
  int isl = nst - 1, csl = 0;
  uint32_t cph = 0;
  int64_t pos_next[Q::APT];
#pragma unroll
  for (int m = 0; m < Q::APT; ++m) pos_next[m] = 0;
  auto load_pos = [&](int i) {
    const int t0 = ((int)blockIdx.x + i * G) * TB;
    const int nt = min(TB, ntok - t0);
#pragma unroll
    for (int m = 0; m < Q::APT; ++m) {
      const int j = aj + m * (Q::BLOCK / HALF);
      if (j < nt) pos_next[m] = pos_of(t0 + j);
    }
  };
  if (my_blk > 0) load_pos(0);

  for (int i = 0; i < my_blk; ++i) {
    issue(i + nst - 1, isl);
    isl = isl + 1 == nst ? 0 : isl + 1;
    const int t0 = ((int)blockIdx.x + i * G) * TB;
    const int nt = min(TB, ntok - t0);
    // this block's cos/sin into shared memory (the previous block's readers
    // are past the trailing barrier of the last iteration)
#pragma unroll
    for (int m = 0; m < Q::APT; ++m) {
      const int j = aj + m * (Q::BLOCK / HALF);
      if (j < nt) {
        float sv, cv;
        sincosf(__fmul_rn((float)pos_next[m], inv_f), &sv, &cv);
        const int k = qt_cs_index<T, D>(j, ai);
        cs_tab[k] = cv * a.cs_scale;
        sn_tab[k] = sv * a.cs_scale;
      }
    }
    if (i + 1 < my_blk) load_pos(i + 1);
    const bool landed = mbar_wait(&bars[csl], cph, a.fault);
    if (!__syncthreads_and(landed)) {
      drain_ring(bars, nst, csl, cph, min(nst, my_blk - i), a.fault);
      break;
    }
    const unsigned char* slot = smem + (size_t)csl * pl.slot;
    if (++csl == nst) {
      csl = 0;
      cph ^= 1u;
    }

    // the block's q run, then its k run (unrolled: each copy names its own
    // tensor's weight and sum registers)
#pragma unroll
    for (int ten = 0; ten < 2; ++ten) {
      const int H = ten == 0 ? Hq : Hk;
      const int nrows = nt * H;
      const int steps = ten == 0 ? steps_q : steps_k;
      if (steps == 0) continue;
      const unsigned char* run = slot + (ten == 0 ? oq : ok) + lt * VEC * (int)sizeof(T);
      const float* rsrun = reinterpret_cast<const float*>(slot + (ten == 0 ? orq : ork));
      T* out = reinterpret_cast<T*>(const_cast<void*>(a.dst[ten].p)) +
               ((int64_t)t0 * H) * D + lt * VEC;
      float* rstd_out = BWD ? nullptr : a.rstd_out[ten] + (int64_t)t0 * H;
      const float* w0 = ten == 0 ? wq0 : wk0;
      const float* w1 = ten == 0 ? wq1 : wk1;
      RowCursor cur = cur0[ten];
#pragma unroll 1
      for (int st = 0; st < steps; ++st, cur.next()) {
        const int r = grp + st * RG;
        const bool valid = r < nrows;
        const int j = valid ? cur.j : 0;
        float cs[VEC], sn[VEC];
        qt_load_cs<T, D>(cs_tab, j, lt, cs);
        qt_load_cs<T, D>(sn_tab, j, lt, sn);
        // rows past the run read the run's first row instead (their results
        // are discarded): the step may end past the slot and its ring
        const unsigned char* rp = run + (valid ? r : 0) * ROWB;
        if constexpr (!BWD) {
          float x0[VEC], x1[VEC];
          unpack(lds_pack<T, VEC>(rp), x0);
          unpack(lds_pack<T, VEC>(rp + HALF * (int)sizeof(T)), x1);
          float2 sa = f2(0.f, 0.f), sb = f2(0.f, 0.f);
#pragma unroll
          for (int e = 0; e < VEC; e += 2) {
            const float2 u = f2(x0[e], x0[e + 1]), v = f2(x1[e], x1[e + 1]);
            sa = f2_fma(u, u, sa);
            sb = f2_fma(v, v, sb);
          }
          const float ss = group_lane_sum<TPR>((sa.x + sa.y) + (sb.x + sb.y));
          const float rstd = rsqrtf(fmaf(ss, kInvD, a.eps));
          const float2 r2 = f2s(rstd), nr2 = f2s(-rstd);
          float y0[VEC], y1[VEC];
#pragma unroll
          for (int e = 0; e < VEC; e += 2) {
            const float2 a0 = f2_mul(f2(x0[e], x0[e + 1]), f2(w0[e], w0[e + 1]));
            const float2 a1 = f2_mul(f2(x1[e], x1[e + 1]), f2(w1[e], w1[e + 1]));
            const float2 c2 = f2_mul(f2(cs[e], cs[e + 1]), r2);
            const float2 s2 = f2(sn[e], sn[e + 1]);
            const float2 o0 = f2_fma(a1, f2_mul(s2, nr2), f2_mul(a0, c2));
            const float2 o1 = f2_fma(a0, f2_mul(s2, r2), f2_mul(a1, c2));
            y0[e] = o0.x;
            y0[e + 1] = o0.y;
            y1[e] = o1.x;
            y1[e + 1] = o1.y;
          }
          if (valid) {
            if (lt == 0) rstd_out[r] = rstd;
            T* o = out + (int64_t)r * D;
            stg_pack_stream<T, VEC>(o, pack<T, VEC>(y0));
            stg_pack_stream<T, VEC>(o + HALF, pack<T, VEC>(y1));
          }
        } else {
          const unsigned char* xp = rp + ox;
          float g0[VEC], g1[VEC], x0[VEC], x1[VEC];
          unpack(lds_pack<T, VEC>(rp), g0);
          unpack(lds_pack<T, VEC>(rp + HALF * (int)sizeof(T)), g1);
          unpack(lds_pack<T, VEC>(xp), x0);
          unpack(lds_pack<T, VEC>(xp + HALF * (int)sizeof(T)), x1);
          const float rstd = valid ? rsrun[r] : 0.f;
          const float2 r2 = f2s(rstd);
          float2 da = f2(0.f, 0.f), db = f2(0.f, 0.f);
          float gw0[VEC], gw1[VEC], xh0[VEC], xh1[VEC], dn0[VEC], dn1[VEC];
#pragma unroll
          for (int e = 0; e < VEC; e += 2) {
            const float2 c2 = f2(cs[e], cs[e + 1]), s2 = f2(sn[e], sn[e + 1]);
            const float2 d0 = f2(g0[e], g0[e + 1]), d1 = f2(g1[e], g1[e + 1]);
            // dn = R^T dy
            const float2 n0 = f2_fma(d1, s2, f2_mul(d0, c2));
            const float2 n1 = f2_fma(d0, f2_mul(s2, f2s(-1.f)), f2_mul(d1, c2));
            const float2 h0 = f2_mul(f2(x0[e], x0[e + 1]), r2);
            const float2 h1 = f2_mul(f2(x1[e], x1[e + 1]), r2);
            const float2 q0 = f2_mul(n0, f2(w0[e], w0[e + 1]));
            const float2 q1 = f2_mul(n1, f2(w1[e], w1[e + 1]));
            da = f2_fma(q0, h0, da);
            db = f2_fma(q1, h1, db);
            gw0[e] = q0.x;
            gw0[e + 1] = q0.y;
            gw1[e] = q1.x;
            gw1[e + 1] = q1.y;
            xh0[e] = h0.x;
            xh0[e + 1] = h0.y;
            xh1[e] = h1.x;
            xh1[e + 1] = h1.y;
            dn0[e] = n0.x;
            dn0[e + 1] = n0.y;
            dn1[e] = n1.x;
            dn1[e + 1] = n1.y;
          }
          if (valid) {  // weight-gradient sums of this row's tensor
            AccT(&s0)[VEC] = ten == 0 ? aq0 : ak0;
            AccT(&s1)[VEC] = ten == 0 ? aq1 : ak1;
#pragma unroll
            for (int e = 0; e < VEC; ++e) {
              acc_add(s0[e], dn0[e], xh0[e]);
              acc_add(s1[e], dn1[e], xh1[e]);
            }
          }
          const float dot = group_lane_sum<TPR>((da.x + da.y) + (db.x + db.y)) * kInvD;
          const float2 nd = f2s(-dot);
          float o0[VEC], o1[VEC];
#pragma unroll
          for (int e = 0; e < VEC; e += 2) {
            const float2 u =
                f2_mul(f2_fma(f2(xh0[e], xh0[e + 1]), nd, f2(gw0[e], gw0[e + 1])), r2);
            const float2 v =
                f2_mul(f2_fma(f2(xh1[e], xh1[e + 1]), nd, f2(gw1[e], gw1[e + 1])), r2);
            o0[e] = u.x;
            o0[e + 1] = u.y;
            o1[e] = v.x;
            o1[e + 1] = v.y;
          }
          if (valid) {
            T* o = out + (int64_t)r * D;
            stg_pack_stream<T, VEC>(o, pack<T, VEC>(o0));
            stg_pack_stream<T, VEC>(o + HALF, pack<T, VEC>(o1));
          }
        }
      }
    }
    // release the slot and the cos/sin tables: this thread's reads are
    // ordered before the next bulk write, and every thread is past them
    fence_proxy_async_smem();
    __syncthreads();
  }

  if constexpr (BWD) {
    // This CTA's partial row [q D | k D]: lanes with equal lt (the warp's row
    // groups) in a fixed butterfly, the warps' totals through shared memory,
    // summed in warp order.
    const int lane = tid & 31, warp = tid >> 5;
#pragma unroll
    for (int e = 0; e < VEC; ++e) {
#pragma unroll
      for (int o = TPR; o < 32; o <<= 1) {
        aq0[e] += __shfl_xor_sync(0xffffffffu, aq0[e], o);
        aq1[e] += __shfl_xor_sync(0xffffffffu, aq1[e], o);
        ak0[e] += __shfl_xor_sync(0xffffffffu, ak0[e], o);
        ak1[e] += __shfl_xor_sync(0xffffffffu, ak1[e], o);
      }
      if (lane < TPR) {
        AccT* rw = red + warp * 2 * D;
        rw[lt * VEC + e] = aq0[e];
        rw[HALF + lt * VEC + e] = aq1[e];
        rw[D + lt * VEC + e] = ak0[e];
        rw[D + HALF + lt * VEC + e] = ak1[e];
      }
    }
    __syncthreads();
    AccT* part = reinterpret_cast<AccT*>(a.partials) + (int64_t)blockIdx.x * 2 * D;
    for (int c = tid; c < 2 * D; c += Q::BLOCK) {
      AccT s = AccT(0);
#pragma unroll
      for (int wi = 0; wi < Q::WARPS; ++wi) s += red[wi * 2 * D + c];
      part[c] = s;
    }
  }
}

}  // namespace bloth
