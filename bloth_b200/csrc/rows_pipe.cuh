// Pipelined row kernels: RMSNorm (optionally + table RoPE) over rows of N,
// forward and backward, with the rows staged global -> shared by bulk copies.
//
// A CTA of RPC row groups x TPR threads (same thread -> column map as the
// register kernels in rows_impl.cuh) walks blocks of RPC consecutive rows
// with a grid stride. Block i lands in ring slot i % NST; thread 0 issues the
// copy of block i + NST - 1 (one bulk copy of the whole block when the rows
// are contiguous, else one per row from the lanes of warp 0) before the CTA
// waits for block i, so NST - 1 blocks are in flight while one is computed.
// A slot holds the block's rows of each input tensor, one after another:
// x (forward), dy then x (backward), and for the residual add x then r
// (forward) or dy, z then dz_out (backward), then, for the table RoPE, the
// rows' cos and sin. NST and the slot size are chosen on the host from N so
// that a CTA stays within its shared-memory budget. The trailing
// __syncthreads of an iteration releases its slot.
//
// Math: as rows_impl.cuh (reference bloth/bloth/kernels/rms_norm.py:59-111,
// fused_norm_qkv_rope.py:59-96). The table RoPE's partner half is either in
// the thread's other vector (paired layout, kRowRopePair) or read from the
// staged row in shared memory.
#pragma once

#include "bulk.cuh"
#include "rows_impl.cuh"

namespace bloth {

struct RowPipe {
  int nst;           // ring slots
  int row_bytes;     // N * sizeof(T), a multiple of 16
  int slot_bytes;    // RPC * row_bytes * (number of input tensors)
  int contiguous;    // rows of a block are adjacent in memory (ld == N) for every input
  int ctas_per_sm;   // resident CTAs per SM to launch (0: as many as fit)
  // Table RoPE: the block's cos and sin rows are staged in the slot after the
  // input rows (cs_row_bytes = half * element size, 0: read from global).
  int cs_row_bytes;
  int64_t cs_ld_bytes;  // table row stride in bytes
  int cs_contiguous;    // table rows adjacent (ld == half): one copy per block
  unsigned int* fault;
};

// Element i of a staged cos/sin row at p (element type dt).
__device__ __forceinline__ float lds_any(const unsigned char* p, int64_t i, int dt) {
  switch (dt) {
    case BLOTH_BF16: return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
    case BLOTH_F16: return __half2float(reinterpret_cast<const __half*>(p)[i]);
    default: return reinterpret_cast<const float*>(p)[i];
  }
}

// Elements i .. i+VEC-1 of a staged cos/sin row (i a multiple of VEC, so the
// access is aligned to VEC elements).
template <int VEC>
__device__ __forceinline__ void lds_any_vec(const unsigned char* p, int64_t i, int dt,
                                            float (&out)[VEC]) {
  if (dt == BLOTH_F32) {
    static_assert(VEC % 4 == 0, "fp32 table reads take whole float4s");
#pragma unroll
    for (int q = 0; q < VEC / 4; ++q) {
      const float4 v = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(p) + i)[q];
      out[4 * q] = v.x;
      out[4 * q + 1] = v.y;
      out[4 * q + 2] = v.z;
      out[4 * q + 3] = v.w;
    }
  } else if (dt == BLOTH_BF16) {
    // copied by value into registers first: unpacking straight from the
    // shared-memory reference read it byte by byte (16 loads per pack, each
    // 2-way bank-conflicted across the warp's two rows; measured by ncu)
    unpack(lds_pack<__nv_bfloat16, VEC>(p + i * 2), out);
  } else {
    unpack(lds_pack<__half, VEC>(p + i * 2), out);
  }
}

// Input tensors a pipelined row kernel stages per row.
constexpr int row_pipe_inputs(int kind, bool bwd) {
  return (bwd ? 2 : 1) + (kind == kRowAdd ? 1 : 0);
}

// CTA shape of the pipelined kernels: TPR threads per row and VPT vectors per
// thread as the register kernels, with RPC rows per block: one row for wide
// rows (TPR >= 128), 128-thread CTAs for medium rows, 256-thread CTAs for
// narrow ones, or a fixed CTA size. Several CTAs share an SM.
template <int TPR_, int VPT_, int BLOCK_ = 0>
struct PipeCfg {
  static constexpr int TPR = TPR_;
  static constexpr int VPT = VPT_;
  // Narrow rows (at most 64 vectors, e.g. bf16 head rows of 128-512) get
  // 256-thread CTAs, so that a block of rows (4-8 KB) amortises the per-block
  // wait and barrier: 1.4-1.6x faster than 128 threads at rows of 128-512.
  // BLOCK_ > 0 fixes the CTA size instead (the paired table RoPE layout).
  static constexpr bool NARROW = TPR * VPT <= 64;
  static constexpr int RPC =
      BLOCK_ > 0 ? BLOCK_ / TPR : (TPR >= 128 ? 1 : (NARROW ? 256 : 128) / TPR);
  static constexpr int BLOCK = TPR * RPC;
  static constexpr int MIN_BLOCKS = BLOCK >= 512 ? 1 : 512 / BLOCK;
};

// csp / snp: this row's staged cos / sin (nullptr: read the tables in global
// memory); wpv: the signed weights of the partner columns held in registers
// by the caller (nullptr: load them).
//
// With the rotation's sign folded into the partner weight,
//   y_c = n_c cos_i + x_p rstd w^s_p sin_i,  w^s_p = -w_{c+h} (c < h), w_{c-h} (c >= h),
// which is two packed multiplies and one packed fma per element pair.
template <typename T, int VEC, bool CSV>
__device__ __forceinline__ void rope_pipe_fwd(float (&o)[VEC], int c, const unsigned char* rowp,
                                              float rstd, const RowArgs& a, int64_t row,
                                              const unsigned char* csp, const unsigned char* snp,
                                              const float* wpv) {
  const int64_t h = a.half;
  if (c >= 2 * h) return;
  if (CSV || (h % VEC) == 0) {
    const bool first = c < h;
    const int64_t pc = first ? c + h : c - h;
    const int64_t i = first ? c : c - h;
    float xp[VEC], wp[VEC], cs[VEC], sn[VEC];
    unpack(lds_pack<T, VEC>(rowp + pc * (int64_t)sizeof(T)), xp);
    if (wpv != nullptr) {
#pragma unroll
      for (int e = 0; e < VEC; ++e) wp[e] = wpv[e];
    } else {
      ld_weight_vec<VEC>(a, pc, a.w_vec, wp);
#pragma unroll
      for (int e = 0; e < VEC; ++e) wp[e] = first ? -wp[e] : wp[e];
    }
    if (CSV || csp != nullptr) {
      lds_any_vec<VEC>(csp, i, a.cs_dt, cs);
      lds_any_vec<VEC>(snp, i, a.cs_dt, sn);
    } else if constexpr (!CSV) {
      ld_any_vec<VEC>(a.cos, row * a.ldcs + i, a.cs_dt, a.cs_vec != 0, cs);
      ld_any_vec<VEC>(a.sin, row * a.ldcs + i, a.cs_dt, a.cs_vec != 0, sn);
    }
    const float2 r2 = f2s(rstd);
#pragma unroll
    for (int e = 0; e < VEC; e += 2) {
      const float2 np = f2_mul(f2_mul(f2(xp[e], xp[e + 1]), r2), f2(wp[e], wp[e + 1]));
      const float2 y = f2_fma(np, f2(sn[e], sn[e + 1]), f2_mul(f2(o[e], o[e + 1]), f2(cs[e], cs[e + 1])));
      o[e] = y.x;
      o[e + 1] = y.y;
    }
  } else if constexpr (!CSV) {
    const T* xr = reinterpret_cast<const T*>(rowp);
#pragma unroll
    for (int e = 0; e < VEC; ++e) {
      const int64_t cc = c + e;
      if (cc < 2 * h && cc < a.N) {
        const bool first = cc < h;
        const int64_t pc = first ? cc + h : cc - h;
        const int64_t i = first ? cc : cc - h;
        const float np = to_f(xr[pc]) * rstd * ld_weight(a, pc);
        const float cs = csp ? lds_any(csp, i, a.cs_dt) : ld_any(a.cos, row * a.ldcs + i, a.cs_dt);
        const float sn = snp ? lds_any(snp, i, a.cs_dt) : ld_any(a.sin, row * a.ldcs + i, a.cs_dt);
        o[e] = first ? (o[e] * cs - np * sn) : (np * sn + o[e] * cs);
      }
    }
  }
}

template <typename T, int VEC, bool CSV>
__device__ __forceinline__ void rope_pipe_bwd(float (&d)[VEC], int c, const unsigned char* dyp,
                                              const RowArgs& a, int64_t row,
                                              const unsigned char* csp,
                                              const unsigned char* snp) {
  const int64_t h = a.half;
  if (c >= 2 * h) return;
  if (CSV || (h % VEC) == 0) {
    const bool first = c < h;
    const int64_t pc = first ? c + h : c - h;
    const int64_t i = first ? c : c - h;
    float dp[VEC], cs[VEC], sn[VEC];
    unpack(lds_pack<T, VEC>(dyp + pc * (int64_t)sizeof(T)), dp);
    if (CSV || csp != nullptr) {
      lds_any_vec<VEC>(csp, i, a.cs_dt, cs);
      lds_any_vec<VEC>(snp, i, a.cs_dt, sn);
    } else if constexpr (!CSV) {
      ld_any_vec<VEC>(a.cos, row * a.ldcs + i, a.cs_dt, a.cs_vec != 0, cs);
      ld_any_vec<VEC>(a.sin, row * a.ldcs + i, a.cs_dt, a.cs_vec != 0, sn);
    }
    // dn_c = dy_c cos_i + s dy_p sin_i, s = +1 (c < h), -1 (c >= h)
    const float2 sg = f2s(first ? 1.f : -1.f);
#pragma unroll
    for (int e = 0; e < VEC; e += 2) {
      const float2 y = f2_fma(f2_mul(f2(dp[e], dp[e + 1]), sg), f2(sn[e], sn[e + 1]),
                              f2_mul(f2(d[e], d[e + 1]), f2(cs[e], cs[e + 1])));
      d[e] = y.x;
      d[e + 1] = y.y;
    }
  } else if constexpr (!CSV) {
    const T* dr = reinterpret_cast<const T*>(dyp);
#pragma unroll
    for (int e = 0; e < VEC; ++e) {
      const int64_t cc = c + e;
      if (cc < 2 * h && cc < a.N) {
        const bool first = cc < h;
        const int64_t pc = first ? cc + h : cc - h;
        const int64_t i = first ? cc : cc - h;
        const float dp = to_f(dr[pc]);
        const float cs = csp ? lds_any(csp, i, a.cs_dt) : ld_any(a.cos, row * a.ldcs + i, a.cs_dt);
        const float sn = snp ? lds_any(snp, i, a.cs_dt) : ld_any(a.sin, row * a.ldcs + i, a.cs_dt);
        d[e] = first ? (d[e] * cs + dp * sn) : (d[e] * cs - dp * sn);
      }
    }
  }
}

// Minimum resident CTAs the register allocation must allow: three for the
// staged-table RoPE backward of narrow rows with one vector per thread
// (256-thread CTAs, at most 80 registers, no spills; measured 12% faster
// than the 2 CTAs its 86-94 registers allowed; the other narrow backward
// kinds fit in 80 registers anyway, and wider rows spill under that cap),
// else enough for 384 threads.
constexpr int row_pipe_min_ctas(int block, int vectors_per_thread, int kind, bool bwd) {
  return bwd && kind == kRowRopeVec && block == 256 && vectors_per_thread == 1
             ? 3
             : (block >= 384 ? 1 : 384 / block);
}

template <typename T, int VEC, int TPR, int VPT, int RPC, int KIND, bool BWD>
__global__ void __launch_bounds__(TPR* RPC, row_pipe_min_ctas(TPR * RPC, VPT, KIND, BWD))
    row_pipe_kernel(const RowArgs a, const RowPipe pp) {
  constexpr bool ROPE = row_rope(KIND);
  // partner of a thread's vector 0 in its vector 1 (TPR * VEC == half, VPT == 2)
  constexpr bool PAIR = KIND == kRowRopePair;
  // the paired layout holds a column and its rotation partner (vectors 0 and
  // 1); rows of 4 * half add the two vectors of the columns past the rotated
  // part, which are normalised only
  static_assert(!PAIR || VPT == 2 || VPT == 4, "paired rows are 2 or 4 halves wide");
  constexpr bool CSV = KIND == kRowRopeVec || PAIR;  // staged tables, vector access
  constexpr bool RES = KIND == kRowAdd;
  constexpr int NTEN = row_pipe_inputs(KIND, BWD);
  using RR = RowReduce<TPR, RPC>;
  using AccT = typename AccOf<T>::type;
  __shared__ float red[RR::SMEM_FLOATS];
  extern __shared__ __align__(128) unsigned char smem[];
  const int grp = threadIdx.x / TPR;
  const int lt = threadIdx.x % TPR;
  const int N = a.N;
  const float inv_n = 1.0f / (float)N;
  const bool wv = a.w_vec != 0;
  const int NST = pp.nst;
  // the dweight reduce that follows may launch now (it waits for this grid)
  if constexpr (BWD) allow_dependent_launch();
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + (size_t)NST * pp.slot_bytes);
  if (threadIdx.x == 0) {
    for (int q = 0; q < NST; ++q) mbar_init(&bars[q], 1);
    mbar_init_fence();
  }

  const int64_t nblk = (a.M + RPC - 1) / RPC;
  const int64_t my_blk = blockIdx.x < nblk ? (nblk - 1 - blockIdx.x) / gridDim.x + 1 : 0;

  const uint64_t pol = BWD ? 0ull : evict_first_policy();
  // Thread 0 (with the lanes of warp 0 for per-row copies) issues block i
  // into ring slot sl.
  auto issue = [&](int64_t i, int sl) {
    if (i >= my_blk || threadIdx.x >= 32) return;
    const int64_t row0 = ((int64_t)blockIdx.x + i * gridDim.x) * RPC;
    const int nrow = (int)min((int64_t)RPC, a.M - row0);
    unsigned char* dst = smem + (size_t)sl * pp.slot_bytes;
    uint64_t* bar = &bars[sl];
    const uint32_t cs_bytes = ROPE ? 2u * (uint32_t)nrow * (uint32_t)pp.cs_row_bytes : 0u;
    if (threadIdx.x == 0)
      mbar_arrive_expect_tx(bar, (uint32_t)(nrow * pp.row_bytes * NTEN) + cs_bytes);
    __syncwarp();
    if constexpr (ROPE) {  // the block's cos and sin rows, after the input rows
      if (pp.cs_row_bytes > 0) {
        unsigned char* cdst = dst + (size_t)RPC * pp.row_bytes * NTEN;
#pragma unroll
        for (int q = 0; q < 2; ++q) {
          const unsigned char* src = reinterpret_cast<const unsigned char*>(q == 0 ? a.cos : a.sin);
          unsigned char* d = cdst + (size_t)q * RPC * pp.cs_row_bytes;
          if (pp.cs_contiguous) {
            if (threadIdx.x == 0)
              bulk_load(d, src + row0 * pp.cs_ld_bytes, (uint32_t)(nrow * pp.cs_row_bytes), bar);
          } else {  // one copy per row; blocks can hold more rows than warp 0 has lanes
            for (int r = (int)threadIdx.x; r < nrow; r += 32)
              bulk_load(d + (size_t)r * pp.cs_row_bytes, src + (row0 + r) * pp.cs_ld_bytes,
                        (uint32_t)pp.cs_row_bytes, bar);
          }
        }
      }
    }
#pragma unroll
    for (int q = 0; q < NTEN; ++q) {
      // forward: x [, r]; backward: dy, x [, dz_out]
      const int k = BWD ? q : q + 1;  // 0 dy, 1 x, 2 r / dz_out
      const T* src = reinterpret_cast<const T*>(k == 0 ? a.dy : (k == 1 ? a.x : a.res));
      const int64_t ld = k == 0 ? a.lddy : (k == 1 ? a.ldx : a.ldres);
      unsigned char* d = dst + (size_t)q * RPC * pp.row_bytes;
      // forward inputs are read once: evict-first in L2 (measured faster for
      // the forward, slower for the backward, whose rows compete with dx)
      if (pp.contiguous) {
        if (threadIdx.x == 0) {
          if constexpr (BWD) bulk_load(d, src + row0 * ld, (uint32_t)(nrow * pp.row_bytes), bar);
          else bulk_load_hint(d, src + row0 * ld, (uint32_t)(nrow * pp.row_bytes), bar, pol);
        }
      } else {  // one copy per row, from the lanes of warp 0
        for (int r = (int)threadIdx.x; r < nrow; r += 32) {
          if constexpr (BWD)
            bulk_load(d + (size_t)r * pp.row_bytes, src + (row0 + r) * ld, (uint32_t)pp.row_bytes,
                      bar);
          else
            bulk_load_hint(d + (size_t)r * pp.row_bytes, src + (row0 + r) * ld,
                           (uint32_t)pp.row_bytes, bar, pol);
        }
      }
    }
  };

  // The first NST - 1 blocks go out before anything else waits on memory,
  // so the copies' latency overlaps the weight loads below.
  for (int q = 0; q < NST - 1; ++q) issue(q, q);

  // The thread's columns are the same for every row it processes: keep their
  // weights in registers (VPT * VEC <= 32 for every pipelined shape), and for
  // the table RoPE on narrow rows those of their rotation partners (c +- half)
  // too (wide rows load them per vector, as registers are short there).
  constexpr bool WP_REG = ROPE && !PAIR && VPT * VEC <= 16;
  // between the backward's two passes, rows of at most 8 values per thread
  // keep dn and xhat in registers; the paired layout (16 values) keeps dn
  constexpr bool KEEPX = VPT * VEC <= 8;
  constexpr bool KEEP = KEEPX || PAIR;
  float wr[VPT][VEC];
  float wpr[WP_REG ? VPT : 1][VEC];
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int c = (j * TPR + lt) * VEC;
    if (c < N) {
      ld_weight_vec<VEC>(a, c, wv, wr[j]);
    } else {
#pragma unroll
      for (int e = 0; e < VEC; ++e) wr[j][e] = 0.f;
    }
    if constexpr (WP_REG) {  // signed as rope_pipe_fwd expects
      const int64_t h = a.half;
      if (c < 2 * h && h % VEC == 0) {
        ld_weight_vec<VEC>(a, c < h ? c + h : c - h, wv, wpr[j]);
#pragma unroll
        for (int e = 0; e < VEC; ++e) wpr[j][e] = c < h ? -wpr[j][e] : wpr[j][e];
      } else {
#pragma unroll
        for (int e = 0; e < VEC; ++e) wpr[j][e] = 0.f;
      }
    }
  }
  __syncthreads();
  int isl = NST - 1;  // slot of the next block to issue
  int csl = 0;        // slot of the block being computed, and its phase
  uint32_t cph = 0;

  AccT acc[VPT][VEC];
#pragma unroll
  for (int j = 0; j < VPT; ++j)
#pragma unroll
    for (int e = 0; e < VEC; ++e) acc[j][e] = AccT(0);

  int parity = 0;
  float rstd_next = 0.f;
  if (BWD && my_blk > 0) {
    const int64_t r = (int64_t)blockIdx.x * RPC + grp;
    rstd_next = r < a.M ? __ldg(a.rstd_in + r) : 0.f;
  }
  for (int64_t i = 0; i < my_blk; ++i, parity ^= 1) {
    issue(i + NST - 1, isl);
    isl = isl + 1 == NST ? 0 : isl + 1;
    const int64_t row = ((int64_t)blockIdx.x + i * gridDim.x) * RPC + grp;
    const bool valid = row < a.M;
    float rstd_in = 0.f;
    if constexpr (BWD) {
      rstd_in = rstd_next;
      const int64_t r2 = row + (int64_t)gridDim.x * RPC;
      if (i + 1 < my_blk && r2 < a.M) rstd_next = __ldg(a.rstd_in + r2);
    }
    const bool landed = mbar_wait(&bars[csl], cph, pp.fault);
    if (!__syncthreads_and(landed)) {
      // give up the rest of the work, but not before the blocks already
      // issued (this one and up to NST - 1 after it) have landed
      drain_ring(bars, NST, csl, cph, (int)min((int64_t)NST, my_blk - i), pp.fault);
      break;
    }
    const unsigned char* slot = smem + (size_t)csl * pp.slot_bytes;
    if (++csl == NST) {
      csl = 0;
      cph ^= 1u;
    }
    const unsigned char* csp = nullptr;  // this row's staged cos and sin
    const unsigned char* snp = nullptr;
    if constexpr (ROPE) {
      if (pp.cs_row_bytes > 0) {
        csp = slot + (size_t)RPC * pp.row_bytes * NTEN + (size_t)grp * pp.cs_row_bytes;
        snp = csp + (size_t)RPC * pp.cs_row_bytes;
      }
    }
    if constexpr (!BWD) {
      const unsigned char* rowp = slot + (size_t)grp * pp.row_bytes;
      Pack<T, VEC> xp[VPT];
      float2 sa = f2(0.f, 0.f), sb = f2(0.f, 0.f);
#pragma unroll
      for (int j = 0; j < VPT; ++j) {
        const int c = (j * TPR + lt) * VEC;
        if (valid && c < N) {
          xp[j] = lds_pack<T, VEC>(rowp + (int64_t)c * sizeof(T));
          if constexpr (RES) {  // z = x + r, rounded once to T, stored, normalised below
            float f[VEC], g[VEC];
            unpack(xp[j], f);
            unpack(lds_pack<T, VEC>(rowp + (size_t)RPC * pp.row_bytes + (int64_t)c * sizeof(T)),
                   g);
#pragma unroll
            for (int e = 0; e < VEC; e += 2) {
              const float2 z2 = f2_add(f2(f[e], f[e + 1]), f2(g[e], g[e + 1]));
              f[e] = z2.x;
              f[e + 1] = z2.y;
            }
            xp[j] = pack<T, VEC>(f);
            stg_pack<T, VEC>(reinterpret_cast<T*>(a.res_out) + row * a.ldres_out + c, xp[j]);
          }
        } else {
#pragma unroll
          for (int e = 0; e < VEC; ++e) xp[j].v[e] = from_f<T>(0.f);
        }
        float f[VEC];
        unpack(xp[j], f);
#pragma unroll
        for (int e = 0; e < VEC; e += 2) {
          const float2 x2 = f2(f[e], f[e + 1]);
          if ((e / 2) & 1) sb = f2_fma(x2, x2, sb);
          else sa = f2_fma(x2, x2, sa);
        }
      }
      const float ss = RR::sum((sa.x + sa.y) + (sb.x + sb.y), red, grp, lt, parity);
      const float rstd = rsqrtf(ss * inv_n + a.eps);
      if (valid) {
        if (lt == 0) a.rstd_out[row] = rstd;
        T* yr = reinterpret_cast<T*>(a.out) + row * a.ldo;
        if constexpr (PAIR) {
          // y_c = rstd (a_c cos - a_p sin), y_p = rstd (a_p cos + a_c sin) for
          // column c < half and its partner p = c + half, a = x w; cos and sin
          // read once for both, the partner already in registers
          const int c0 = lt * VEC;
          float f0[VEC], f1[VEC], cs[VEC], sn[VEC];
          unpack(xp[0], f0);
          unpack(xp[1], f1);
          lds_any_vec<VEC>(csp, c0, a.cs_dt, cs);
          lds_any_vec<VEC>(snp, c0, a.cs_dt, sn);
          const float2 r2 = f2s(rstd), nr2 = f2s(-rstd);
#pragma unroll
          for (int e = 0; e < VEC; e += 2) {
            const float2 a0 = f2_mul(f2(f0[e], f0[e + 1]), f2(wr[0][e], wr[0][e + 1]));
            const float2 a1 = f2_mul(f2(f1[e], f1[e + 1]), f2(wr[1][e], wr[1][e + 1]));
            const float2 c2 = f2_mul(f2(cs[e], cs[e + 1]), r2);
            const float2 s2 = f2(sn[e], sn[e + 1]);
            const float2 y0 = f2_fma(a1, f2_mul(s2, nr2), f2_mul(a0, c2));
            const float2 y1 = f2_fma(a0, f2_mul(s2, r2), f2_mul(a1, c2));
            f0[e] = y0.x;
            f0[e + 1] = y0.y;
            f1[e] = y1.x;
            f1[e + 1] = y1.y;
          }
          stg_pack_stream<T, VEC>(yr + c0, pack<T, VEC>(f0));
          stg_pack_stream<T, VEC>(yr + c0 + TPR * VEC, pack<T, VEC>(f1));
#pragma unroll
          for (int j = 2; j < VPT; ++j) {  // columns past the rotated part
            float f[VEC];
            unpack(xp[j], f);
#pragma unroll
            for (int e = 0; e < VEC; e += 2) {
              const float2 y = f2_mul(f2_mul(f2(f[e], f[e + 1]), r2), f2(wr[j][e], wr[j][e + 1]));
              f[e] = y.x;
              f[e + 1] = y.y;
            }
            stg_pack_stream<T, VEC>(yr + (j * TPR + lt) * VEC, pack<T, VEC>(f));
          }
        } else {
#pragma unroll
        for (int j = 0; j < VPT; ++j) {
          const int c = (j * TPR + lt) * VEC;
          if (c < N) {
            float f[VEC];
            unpack(xp[j], f);
            const float2 r2 = f2s(rstd);
#pragma unroll
            for (int e = 0; e < VEC; e += 2) {
              const float2 y = f2_mul(f2_mul(f2(f[e], f[e + 1]), r2), f2(wr[j][e], wr[j][e + 1]));
              f[e] = y.x;
              f[e + 1] = y.y;
            }
            if constexpr (ROPE)
              rope_pipe_fwd<T, VEC, CSV>(f, c, rowp, rstd, a, row, csp, snp,
                                    WP_REG ? wpr[WP_REG ? j : 0] : nullptr);
            // streaming stores: 1.7% faster for the RMSNorm forward, none
            // for the residual-add forward (measured on B200)
            if constexpr (RES) stg_pack<T, VEC>(yr + c, pack<T, VEC>(f));
            else stg_pack_stream<T, VEC>(yr + c, pack<T, VEC>(f));
          }
        }
        }
      }
    } else {
      const unsigned char* dyp = slot + (size_t)grp * pp.row_bytes;
      const unsigned char* xrp = slot + (size_t)(RPC + grp) * pp.row_bytes;
      const float rstd = rstd_in;
      // pass 1: dot = sum(dn*w*xhat), dweight terms dn*xhat
      float2 da = f2(0.f, 0.f), db = f2(0.f, 0.f);
      const float2 r2 = f2s(rstd);
      // narrow rows keep dn and xhat in registers for pass 2 (instead of
      // re-reading the slot and, for RoPE, rotating dy again)
      float dnk[KEEP ? VPT : 1][VEC], xk[KEEPX ? VPT : 1][VEC];
      // paired layout: dn = R^T dy of both vectors at once,
      //   dn_c = dy_c cos + dy_p sin,  dn_p = dy_p cos - dy_c sin
      float dpr[PAIR ? 2 : 1][VEC];
      if constexpr (PAIR) {
        if (valid) {
          const int c0 = lt * VEC;
          float g0[VEC], g1[VEC], cs[VEC], sn[VEC];
          unpack(lds_pack<T, VEC>(dyp + (int64_t)c0 * sizeof(T)), g0);
          unpack(lds_pack<T, VEC>(dyp + (int64_t)(c0 + TPR * VEC) * sizeof(T)), g1);
          lds_any_vec<VEC>(csp, c0, a.cs_dt, cs);
          lds_any_vec<VEC>(snp, c0, a.cs_dt, sn);
#pragma unroll
          for (int e = 0; e < VEC; e += 2) {
            const float2 c2 = f2(cs[e], cs[e + 1]), s2 = f2(sn[e], sn[e + 1]);
            const float2 d0 = f2(g0[e], g0[e + 1]), d1 = f2(g1[e], g1[e + 1]);
            const float2 n0 = f2_fma(d1, s2, f2_mul(d0, c2));
            const float2 n1 = f2_fma(d0, f2_mul(s2, f2s(-1.f)), f2_mul(d1, c2));
            dpr[0][e] = n0.x;
            dpr[0][e + 1] = n0.y;
            dpr[PAIR ? 1 : 0][e] = n1.x;
            dpr[PAIR ? 1 : 0][e + 1] = n1.y;
          }
        }
      }
#pragma unroll
      for (int j = 0; j < VPT; ++j) {
        const int c = (j * TPR + lt) * VEC;
        if (valid && c < N) {
          float xf[VEC], dn[VEC];
          if (PAIR && j < 2) {  // rotated: R^T dy from above
#pragma unroll
            for (int e = 0; e < VEC; ++e) dn[e] = dpr[PAIR && j < 2 ? j : 0][e];
          } else {  // (paired rows: columns past the rotated part take dy as it is)
            unpack(lds_pack<T, VEC>(dyp + (int64_t)c * sizeof(T)), dn);
          }
          unpack(lds_pack<T, VEC>(xrp + (int64_t)c * sizeof(T)), xf);
          if constexpr (ROPE && !PAIR) rope_pipe_bwd<T, VEC, CSV>(dn, c, dyp, a, row, csp, snp);
#pragma unroll
          for (int e = 0; e < VEC; e += 2) {
            const float2 d2 = f2(dn[e], dn[e + 1]);
            const float2 x2 = f2_mul(f2(xf[e], xf[e + 1]), r2);
            if constexpr (KEEP) {
              dnk[KEEP ? j : 0][e] = d2.x;
              dnk[KEEP ? j : 0][e + 1] = d2.y;
            }
            if constexpr (KEEPX) {
              xk[KEEPX ? j : 0][e] = x2.x;
              xk[KEEPX ? j : 0][e + 1] = x2.y;
            }
            const float2 t = f2_mul(d2, f2(wr[j][e], wr[j][e + 1]));
            if ((e / 2) & 1) db = f2_fma(t, x2, db);
            else da = f2_fma(t, x2, da);
            if constexpr (std::is_same<AccT, float>::value) {
              const float2 a2 = f2_fma(d2, x2, f2(acc[j][e], acc[j][e + 1]));
              acc[j][e] = a2.x;
              acc[j][e + 1] = a2.y;
            } else {
              acc_fma(acc[j][e], d2.x, x2.x);
              acc_fma(acc[j][e + 1], d2.y, x2.y);
            }
          }
        }
      }
      const float dot = RR::sum((da.x + da.y) + (db.x + db.y), red, grp, lt, parity) * inv_n;
      // pass 2: dx = rstd*(dn*w - xhat*dot), dn and xhat re-read from the slot
      if (valid) {
        T* dxr = reinterpret_cast<T*>(a.out) + row * a.ldo;
#pragma unroll
        for (int j = 0; j < VPT; ++j) {
          const int c = (j * TPR + lt) * VEC;
          if (c < N) {
            float xf[VEC], dn[VEC], o[VEC];
            if constexpr (KEEP) {
#pragma unroll
              for (int e = 0; e < VEC; ++e) dn[e] = dnk[KEEP ? j : 0][e];
              if constexpr (KEEPX) {
#pragma unroll
                for (int e = 0; e < VEC; ++e) xf[e] = xk[KEEPX ? j : 0][e];
              } else {
                unpack(lds_pack<T, VEC>(xrp + (int64_t)c * sizeof(T)), xf);
              }
            } else {
              unpack(lds_pack<T, VEC>(dyp + (int64_t)c * sizeof(T)), dn);
              unpack(lds_pack<T, VEC>(xrp + (int64_t)c * sizeof(T)), xf);
              if constexpr (ROPE) rope_pipe_bwd<T, VEC, CSV>(dn, c, dyp, a, row, csp, snp);
            }
            const float2 nd = f2s(-dot);
#pragma unroll
            for (int e = 0; e < VEC; e += 2) {
              // xf holds xhat already when kept
              const float2 x2 = KEEPX ? f2(xf[e], xf[e + 1]) : f2_mul(f2(xf[e], xf[e + 1]), r2);
              const float2 y = f2_mul(
                  f2_fma(x2, nd, f2_mul(f2(dn[e], dn[e + 1]), f2(wr[j][e], wr[j][e + 1]))), r2);
              o[e] = y.x;
              o[e + 1] = y.y;
            }
            if constexpr (RES) {  // dz = dz_out + the RMSNorm gradient of z
              float g[VEC];
              unpack(lds_pack<T, VEC>(xrp + (size_t)RPC * pp.row_bytes + (int64_t)c * sizeof(T)),
                     g);
#pragma unroll
              for (int e = 0; e < VEC; e += 2) {
                const float2 s2 = f2_add(f2(o[e], o[e + 1]), f2(g[e], g[e + 1]));
                o[e] = s2.x;
                o[e + 1] = s2.y;
              }
            }
            stg_pack<T, VEC>(dxr + c, pack<T, VEC>(o));
          }
        }
      }
    }
    // release the slot: order this thread's reads before the next bulk write
    fence_proxy_async_smem();
    __syncthreads();
  }

  if constexpr (BWD) {
    // This CTA's partial dweight row: the RPC row groups' accumulators are
    // stored side by side in the idle ring memory ([RPC][N], which always
    // fits: the ring holds at least two slots of two input rows per group),
    // then each thread sums columns over the groups in a fixed order.
    __syncthreads();
    AccT* part = reinterpret_cast<AccT*>(a.partials) + (int64_t)blockIdx.x * N;
    if constexpr (RPC > 1) {
      AccT* buf = reinterpret_cast<AccT*>(smem);
#pragma unroll
      for (int j = 0; j < VPT; ++j) {
        const int c = (j * TPR + lt) * VEC;
#pragma unroll
        for (int e = 0; e < VEC; ++e)
          if (c + e < N) buf[grp * N + c + e] = acc[j][e];
      }
      __syncthreads();
      for (int col = (int)threadIdx.x; col < N; col += TPR * RPC) {
        AccT sum = buf[col];
        for (int g = 1; g < RPC; ++g) sum += buf[g * N + col];
        part[col] = sum;
      }
    } else {
#pragma unroll
      for (int j = 0; j < VPT; ++j) {
        const int c = (j * TPR + lt) * VEC;
        if (c < N) store_acc_vec<AccT, VEC>(part + c, acc[j], N - c);
      }
    }
  }
}

}  // namespace bloth
