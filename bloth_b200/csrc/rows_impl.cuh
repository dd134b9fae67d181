// Row kernels: RMSNorm over rows of N, optionally followed by rotate-half
// RoPE on the first 2*half columns with per-row cos/sin tables (the
// reference's fused_norm_rope contract) or preceded by a residual add
// (z = x + r, stored, then normalised), forward and backward.
//
// Layout. A row group of TPR threads owns one row at a time; thread lt holds
// vectors j = 0..VPT-1 at columns (j*TPR + lt)*VEC .. +VEC, so every
// warp-wide access is one contiguous 16-byte-per-lane transaction. A CTA
// holds RPC row groups and walks the rows with a grid stride, so a launch is
// at most (SMs x resident CTAs) CTAs and the backward's weight-gradient
// partials stay one row per CTA.
//
// Reference semantics followed (bloth/bloth/kernels/rms_norm.py:39-113 and
// bloth/bloth/kernels/fused_norm_qkv_rope.py:40-96):
//   rstd = rsqrt(sum(x^2)/N + eps), y = (x*rstd)*w, all in fp32, one rounding
//   on store; rotation y1 = n1*cos - n2*sin, y2 = n1*sin + n2*cos on pairs
//   (c, c+half) of the normalised row n; backward dx = rstd*(g - xhat*dot/N)
//   with g = dn*w, dot = sum(g*xhat) and dn the rotation-transposed dy.
#pragma once

#include <type_traits>

#include "common.cuh"

namespace bloth {

struct RowArgs {
  const void* x;
  int64_t ldx;
  const void* dy;  // backward only
  int64_t lddy;
  void* out;  // y (forward) or dx (backward)
  int64_t ldo;
  const void* w;
  int w_dt;
  int w_vec;  // w aligned for VEC-wide loads
  float w_off;  // added to every weight: 1 for (1 + w) norms (Gemma), else 0
  float* rstd_out;      // forward
  const float* rstd_in; // backward
  void* partials;       // backward: [gridDim.x][N] accumulator rows
  const void* cos;
  const void* sin;
  int64_t ldcs;
  int cs_dt;
  int cs_vec;  // cos/sin rows aligned for VEC-wide loads
  int64_t half;
  const void* res;   // kRowAdd: r (forward) or dz_out, z's gradient from the residual stream (backward; may be null)
  int64_t ldres;
  void* res_out;     // kRowAdd forward: z = x + r in x's type
  int64_t ldres_out;
  int64_t M;
  int N;
  float eps;
};

// What a row kernel computes besides the RMSNorm.
enum RowKind : int {
  kRowNorm = 0,  // RMSNorm
  kRowRope = 1,  // RMSNorm, then rotate-half RoPE with per-row cos/sin tables
  kRowAdd = 2,   // z = x + r rounded to x's type and stored, then RMSNorm of z;
                 // the backward adds dz_out to the RMSNorm gradient of z
  kRowRopeVec = 3,  // kRowRope whose tables are staged in the ring and allow
                    // vector access (pipelined kernels only: neither the global
                    // table reads nor the per-element fallback are compiled)
  kRowRopePair = 4,  // kRowRopeVec on rows rotated in full (N == 2 * half,
                     // VPT == 2) or on their first half (N == 4 * half,
                     // VPT == 4) laid out so that a thread's second vector
                     // holds the rotation partners of its first
                     // (TPR * VEC == half); vectors 2 and 3 are normalised only
};

constexpr bool row_rope(int kind) {
  return kind == kRowRope || kind == kRowRopeVec || kind == kRowRopePair;
}
// The kind the register kernels run for `kind` (they have one table RoPE).
constexpr int reg_kind(int kind) { return row_rope(kind) ? kRowRope : kind; }

// Weight of column c as the kernels apply it, w[c] + w_off, in fp32.
__device__ __forceinline__ float ld_weight(const RowArgs& a, int64_t c) {
  return ld_any(a.w, c, a.w_dt) + a.w_off;
}

template <int VEC>
__device__ __forceinline__ void ld_weight_vec(const RowArgs& a, int64_t c, bool vec_ok,
                                              float (&w)[VEC]) {
  ld_any_vec<VEC>(a.w, c, a.w_dt, vec_ok, w);
#pragma unroll
  for (int e = 0; e < VEC; ++e) w[e] += a.w_off;
}

template <int TPR, int RPC>
struct RowReduce {
  static constexpr int NW = TPR > 32 ? TPR / 32 : 1;
  static constexpr int SMEM_FLOATS = 2 * RPC * NW;
  // Sum of v over the TPR threads of row group `grp`. For TPR > 32 this
  // contains a __syncthreads(), so every thread of the CTA must call it the
  // same number of times. The two-slot parity buffer makes one barrier per
  // call enough: a slot is rewritten only after every thread has passed the
  // next call's barrier, i.e. finished reading it.
  __device__ __forceinline__ static float sum(float v, float* red, int grp, int lt, int parity) {
    if constexpr (TPR <= 32) {
      return group_lane_sum<TPR>(v);
    } else {
      v = group_lane_sum<32>(v);
      float* r = red + (parity * RPC + grp) * NW;
      if ((lt & 31) == 0) r[lt >> 5] = v;
      __syncthreads();
      float s = 0.f;
#pragma unroll
      for (int i = 0; i < NW; ++i) s += r[i];
      return s;
    }
  }
};

// Element-wise rotation for rows whose cos/sin or half width do not allow
// VEC-wide partner loads. Kept out of line so that its scalar loads do not
// inflate the register allocation of the vector path.
template <typename T>
__device__ __noinline__ float rope_scalar_fwd(float own, int64_t cc, const T* xr, float rstd,
                                              const RowArgs& a, int64_t row) {
  const int64_t h = a.half;
  const bool first = cc < h;
  const int64_t pc = first ? cc + h : cc - h;
  const int64_t i = first ? cc : cc - h;
  const float np = to_f(xr[pc]) * rstd * ld_weight(a, pc);
  const float cs = ld_any(a.cos, row * a.ldcs + i, a.cs_dt);
  const float sn = ld_any(a.sin, row * a.ldcs + i, a.cs_dt);
  return first ? (own * cs - np * sn) : (np * sn + own * cs);
}

template <typename T>
__device__ __noinline__ float rope_scalar_bwd(float own, int64_t cc, const T* dyr,
                                              const RowArgs& a, int64_t row) {
  const int64_t h = a.half;
  const bool first = cc < h;
  const int64_t pc = first ? cc + h : cc - h;
  const int64_t i = first ? cc : cc - h;
  const float dp = to_f(dyr[pc]);
  const float cs = ld_any(a.cos, row * a.ldcs + i, a.cs_dt);
  const float sn = ld_any(a.sin, row * a.ldcs + i, a.cs_dt);
  return first ? (own * cs + dp * sn) : (own * cs - dp * sn);
}

// Rotation of one VEC-wide slice of a normalised row, forward direction.
// o[] holds n = x*rstd*w for columns c..c+VEC-1 and is overwritten with y.
// The partner half is re-read from global memory (an L1/L2 hit: the row was
// just streamed in by this row group), as the reference kernel does
// (fused_norm_qkv_rope.py:76-80).
template <typename T, int VEC>
__device__ __forceinline__ void rope_rows_fwd(float (&o)[VEC], int c, const T* xr, float rstd,
                                              const RowArgs& a, int64_t row) {
  const int64_t h = a.half;
  if (c >= 2 * h) return;
  if ((h % VEC) == 0) {
    const bool first = c < h;
    const int64_t pc = first ? c + h : c - h;
    const int64_t i = first ? c : c - h;
    float xp[VEC], wp[VEC], cs[VEC], sn[VEC];
    unpack(ldg_pack<T, VEC>(xr + pc), xp);
    ld_weight_vec<VEC>(a, pc, a.w_vec, wp);
    ld_any_vec<VEC>(a.cos, row * a.ldcs + i, a.cs_dt, a.cs_vec != 0, cs);
    ld_any_vec<VEC>(a.sin, row * a.ldcs + i, a.cs_dt, a.cs_vec != 0, sn);
#pragma unroll
    for (int e = 0; e < VEC; ++e) {
      const float np = xp[e] * rstd * wp[e];
      o[e] = first ? (o[e] * cs[e] - np * sn[e]) : (np * sn[e] + o[e] * cs[e]);
    }
  } else {
#pragma unroll
    for (int e = 0; e < VEC; ++e)
      if (c + e < 2 * h && c + e < a.N) o[e] = rope_scalar_fwd<T>(o[e], c + e, xr, rstd, a, row);
  }
}

// Transposed rotation of one VEC-wide slice of dy (backward). d[] holds dy
// for columns c..c+VEC-1 and is overwritten with dn = R^T dy:
//   first half  (c <  half): dn = dy_c*cos + dy_{c+half}*sin
//   second half (c >= half): dn = dy_c*cos - dy_{c-half}*sin
template <typename T, int VEC>
__device__ __forceinline__ void rope_rows_bwd(float (&d)[VEC], int c, const T* dyr,
                                              const RowArgs& a, int64_t row) {
  const int64_t h = a.half;
  if (c >= 2 * h) return;
  if ((h % VEC) == 0) {
    const bool first = c < h;
    const int64_t pc = first ? c + h : c - h;
    const int64_t i = first ? c : c - h;
    float dp[VEC], cs[VEC], sn[VEC];
    unpack(ldg_pack<T, VEC>(dyr + pc), dp);
    ld_any_vec<VEC>(a.cos, row * a.ldcs + i, a.cs_dt, a.cs_vec != 0, cs);
    ld_any_vec<VEC>(a.sin, row * a.ldcs + i, a.cs_dt, a.cs_vec != 0, sn);
#pragma unroll
    for (int e = 0; e < VEC; ++e)
      d[e] = first ? (d[e] * cs[e] + dp[e] * sn[e]) : (d[e] * cs[e] - dp[e] * sn[e]);
  } else {
#pragma unroll
    for (int e = 0; e < VEC; ++e)
      if (c + e < 2 * h && c + e < a.N) d[e] = rope_scalar_bwd<T>(d[e], c + e, dyr, a, row);
  }
}

template <typename T, int VEC, int TPR, int VPT, int RPC, int KIND>
__global__ void __launch_bounds__(TPR* RPC, TPR * RPC <= 256 ? 2 : 1) row_fwd_kernel(const RowArgs a) {
  constexpr bool ROPE = KIND == kRowRope;
  constexpr bool RES = KIND == kRowAdd;
  using RR = RowReduce<TPR, RPC>;
  __shared__ float red[RR::SMEM_FLOATS];
  const int grp = threadIdx.x / TPR;
  const int lt = threadIdx.x % TPR;
  const T* __restrict__ x = reinterpret_cast<const T*>(a.x);
  T* __restrict__ y = reinterpret_cast<T*>(a.out);
  const int N = a.N;
  const bool wv = a.w_vec != 0;
  int parity = 0;
  for (int64_t base = (int64_t)blockIdx.x * RPC; base < a.M;
       base += (int64_t)gridDim.x * RPC, parity ^= 1) {
    const int64_t row = base + grp;
    const bool valid = row < a.M;
    const T* xr = x + row * a.ldx;
    Pack<T, VEC> xp[VPT];
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
      const int c = (j * TPR + lt) * VEC;
      if (valid && c < N) {
        xp[j] = ldg_pack<T, VEC>(xr + c);
        if constexpr (RES) {  // z = x + r, rounded once to T, stored, normalised below
          float f[VEC], g[VEC];
          unpack(xp[j], f);
          unpack(ldg_pack<T, VEC>(reinterpret_cast<const T*>(a.res) + row * a.ldres + c), g);
#pragma unroll
          for (int e = 0; e < VEC; ++e) f[e] += g[e];
          xp[j] = pack<T, VEC>(f);
          stg_pack<T, VEC>(reinterpret_cast<T*>(a.res_out) + row * a.ldres_out + c, xp[j]);
        }
      } else {
#pragma unroll
        for (int e = 0; e < VEC; ++e) xp[j].v[e] = from_f<T>(0.f);
      }
    }
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
      float f[VEC];
      unpack(xp[j], f);
#pragma unroll
      for (int e = 0; e < VEC; ++e) ss = fmaf(f[e], f[e], ss);
    }
    ss = RR::sum(ss, red, grp, lt, parity);
    const float rstd = rsqrtf(ss / (float)N + a.eps);
    if (!valid) continue;
    if (lt == 0) a.rstd_out[row] = rstd;
    T* yr = y + row * a.ldo;
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
      const int c = (j * TPR + lt) * VEC;
      if (c < N) {
        float f[VEC], w[VEC];
        unpack(xp[j], f);
        ld_weight_vec<VEC>(a, c, wv, w);
#pragma unroll
        for (int e = 0; e < VEC; ++e) f[e] = f[e] * rstd * w[e];
        if constexpr (ROPE) rope_rows_fwd<T, VEC>(f, c, xr, rstd, a, row);
        stg_pack<T, VEC>(yr + c, pack<T, VEC>(f));
      }
    }
  }
}

__device__ __forceinline__ void acc_fma(float& acc, float a, float b) { acc = fmaf(a, b, acc); }
__device__ __forceinline__ void acc_fma(double& acc, float a, float b) {
  acc = fma((double)a, (double)b, acc);
}

template <typename T, int VEC, int TPR, int VPT, int RPC, int KIND>
__global__ void __launch_bounds__(TPR* RPC, TPR * RPC <= 256 ? 2 : 1) row_bwd_kernel(const RowArgs a) {
  constexpr bool ROPE = KIND == kRowRope;
  constexpr bool RES = KIND == kRowAdd;
  using RR = RowReduce<TPR, RPC>;
  using AccT = typename AccOf<T>::type;
  __shared__ float red[RR::SMEM_FLOATS];
  extern __shared__ __align__(16) unsigned char dsmem[];
  allow_dependent_launch();  // the dweight reduce waits for this grid
  const int grp = threadIdx.x / TPR;
  const int lt = threadIdx.x % TPR;
  const T* __restrict__ x = reinterpret_cast<const T*>(a.x);
  const T* __restrict__ dy = reinterpret_cast<const T*>(a.dy);
  T* __restrict__ dx = reinterpret_cast<T*>(a.out);
  const int N = a.N;
  const bool wv = a.w_vec != 0;
  AccT acc[VPT][VEC];
#pragma unroll
  for (int j = 0; j < VPT; ++j)
#pragma unroll
    for (int e = 0; e < VEC; ++e) acc[j][e] = AccT(0);

  int parity = 0;
  for (int64_t base = (int64_t)blockIdx.x * RPC; base < a.M;
       base += (int64_t)gridDim.x * RPC, parity ^= 1) {
    const int64_t row = base + grp;
    const bool valid = row < a.M;
    const T* xr = x + row * a.ldx;
    const T* dyr = dy + row * a.lddy;
    Pack<T, VEC> xp[VPT], dp[VPT];
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
      const int c = (j * TPR + lt) * VEC;
      if (valid && c < N) {
        dp[j] = ldg_pack<T, VEC>(dyr + c);
        xp[j] = ldg_pack<T, VEC>(xr + c);
      } else {
#pragma unroll
        for (int e = 0; e < VEC; ++e) {
          dp[j].v[e] = from_f<T>(0.f);
          xp[j].v[e] = from_f<T>(0.f);
        }
      }
    }
    const float rstd = valid ? __ldg(a.rstd_in + row) : 0.f;
    // pass 1: dot = sum(g * xhat) with g = dn*w, and the dweight terms
    float dot = 0.f;
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
      const int c = (j * TPR + lt) * VEC;
      if (valid && c < N) {
        float dn[VEC], xf[VEC], w[VEC];
        unpack(dp[j], dn);
        unpack(xp[j], xf);
        if constexpr (ROPE) rope_rows_bwd<T, VEC>(dn, c, dyr, a, row);
        ld_weight_vec<VEC>(a, c, wv, w);
#pragma unroll
        for (int e = 0; e < VEC; ++e) {
          const float xh = xf[e] * rstd;
          dot = fmaf(dn[e] * w[e], xh, dot);
          acc_fma(acc[j][e], dn[e], xh);
        }
      }
    }
    dot = RR::sum(dot, red, grp, lt, parity) / (float)N;
    if (!valid) continue;
    // pass 2: dx = rstd * (g - xhat * dot), recomputing g and xhat from the
    // packed inputs still in registers
    T* dxr = dx + row * a.ldo;
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
      const int c = (j * TPR + lt) * VEC;
      if (c < N) {
        float dn[VEC], xf[VEC], w[VEC], o[VEC];
        unpack(dp[j], dn);
        unpack(xp[j], xf);
        if constexpr (ROPE) rope_rows_bwd<T, VEC>(dn, c, dyr, a, row);
        ld_weight_vec<VEC>(a, c, wv, w);
#pragma unroll
        for (int e = 0; e < VEC; ++e) o[e] = rstd * (dn[e] * w[e] - (xf[e] * rstd) * dot);
        if constexpr (RES) {
          if (a.res != nullptr) {
            float g[VEC];
            unpack(ldg_pack<T, VEC>(reinterpret_cast<const T*>(a.res) + row * a.ldres + c), g);
#pragma unroll
            for (int e = 0; e < VEC; ++e) o[e] += g[e];
          }
        }
        stg_pack<T, VEC>(dxr + c, pack<T, VEC>(o));
      }
    }
  }

  // Fold the RPC row groups' accumulators into group 0 in a fixed order,
  // then write this CTA's partial row.
  if constexpr (RPC > 1) {
    AccT* buf = reinterpret_cast<AccT*>(dsmem);
    for (int g = RPC - 1; g >= 1; --g) {
      __syncthreads();
      if (grp == g) {
#pragma unroll
        for (int j = 0; j < VPT; ++j)
#pragma unroll
          for (int e = 0; e < VEC; ++e) buf[(j * TPR + lt) * VEC + e] = acc[j][e];
      }
      __syncthreads();
      if (grp == 0) {
#pragma unroll
        for (int j = 0; j < VPT; ++j)
#pragma unroll
          for (int e = 0; e < VEC; ++e) acc[j][e] += buf[(j * TPR + lt) * VEC + e];
      }
    }
  }
  if (grp == 0) {
    AccT* part = reinterpret_cast<AccT*>(a.partials) + (int64_t)blockIdx.x * N;
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
      const int c = (j * TPR + lt) * VEC;
      if (c < N) store_acc_vec<AccT, VEC>(part + c, acc[j], N - c);
    }
  }
}

// ---------------------------------------------------------------------------
// launch configuration
// ---------------------------------------------------------------------------
template <int TPR_, int VPT_, int PIPE_BLOCK_ = 0>
struct RowCfg {
  static constexpr int TPR = TPR_;
  static constexpr int VPT = VPT_;
  static constexpr int RPC = TPR >= 256 ? 1 : 256 / TPR;
  // threads per CTA of the pipelined kernel for this shape (0: PipeCfg's rule)
  static constexpr int PIPE_BLOCK = PIPE_BLOCK_;
};

// Picks the smallest row-group shape that holds a row of N in registers and
// calls f(RowCfg<...>{}). VEC == 1 is the unaligned scalar path.
template <int VEC, typename F>
__host__ bool dispatch_row_cfg(int N, F&& f) {
  const int nv = (N + VEC - 1) / VEC;
  if constexpr (VEC == 1) {
    if (nv <= 256) { f(RowCfg<32, 8>{}); return true; }
    if (nv <= 2048) { f(RowCfg<256, 8>{}); return true; }
    if (nv <= 8192) { f(RowCfg<1024, 8>{}); return true; }
    return false;
  } else {
    if (nv <= 8) { f(RowCfg<8, 1>{}); return true; }
    if (nv <= 16) { f(RowCfg<16, 1>{}); return true; }
    if (nv <= 32) { f(RowCfg<32, 1>{}); return true; }
    if (nv <= 64) { f(RowCfg<32, 2>{}); return true; }
    if (nv <= 128) { f(RowCfg<32, 4>{}); return true; }
    if (nv <= 256) { f(RowCfg<64, 4>{}); return true; }
    if (nv <= 512) { f(RowCfg<128, 4>{}); return true; }
    if (nv <= 1024) { f(RowCfg<256, 4>{}); return true; }
    if (nv <= 2048) { f(RowCfg<512, 4>{}); return true; }
    if (nv <= 4096) { f(RowCfg<1024, 4>{}); return true; }
    if (nv <= 8192) { f(RowCfg<1024, 8>{}); return true; }
    return false;
  }
}

template <typename T, int VEC, typename Cfg>
constexpr size_t row_bwd_smem() {
  using AccT = typename AccOf<T>::type;
  return Cfg::RPC > 1 ? (size_t)Cfg::TPR * Cfg::VPT * VEC * sizeof(AccT) : 0;
}

inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

// Number of CTAs (and partial rows) the backward uses for M rows of N:
// one wave of resident CTAs, or fewer when there are fewer row blocks.
template <typename T, int VEC, typename Cfg, int KIND>
int64_t row_bwd_grid(int64_t M) {
  auto kern = row_bwd_kernel<T, VEC, Cfg::TPR, Cfg::VPT, Cfg::RPC, KIND>;
  const int occ = occupancy((const void*)kern, Cfg::TPR * Cfg::RPC, row_bwd_smem<T, VEC, Cfg>());
  const int64_t wave = (int64_t)device_sm_count() * (occ > 0 ? occ : 1);
  const int64_t need = ceil_div(M, Cfg::RPC);
  return need < wave ? (need > 0 ? need : 0) : wave;
}

// Host entry points (instantiated per element type in rows_<type>.cu).
// kind: a RowKind; vec: every row pointer and stride allows 16-byte accesses.
template <typename T>
int rows_fwd(const RowArgs& a, int kind, bool vec, cudaStream_t st);
template <typename T>
int rows_bwd(const RowArgs& a, int kind, bool vec, void* ws, size_t ws_bytes, void* dw,
             cudaStream_t st);
template <typename T>
size_t rows_bwd_workspace(int64_t M, int N, int kind);

// Checks a weight-gradient workspace for `need` bytes of AccT partial rows:
// BLOTH_ERR_WORKSPACE when it is missing or smaller, BLOTH_ERR_ALIGN when its
// base is not aligned to AccT (the kernels store AccT values, as 16-byte
// vectors where the base is 16-byte aligned).
template <typename AccT>
inline int check_workspace(const void* ws, size_t need, size_t ws_bytes) {
  if (need > ws_bytes || (need > 0 && ws == nullptr)) return BLOTH_ERR_WORKSPACE;
  if (reinterpret_cast<uintptr_t>(ws) % sizeof(AccT) != 0) return BLOTH_ERR_ALIGN;
  return BLOTH_OK;
}

// Deterministic column sum of [P][N] accumulator partials into dw (w_dt).
template <typename AccT>
int launch_dw_reduce(const AccT* part, int64_t P, int N, void* dw0, int n0, void* dw1, int w_dt,
                     cudaStream_t st);

}  // namespace bloth
