// extern "C" entry points declared in include/bloth_b200.h: argument
// validation, element-type dispatch and the choice between the 16-byte vector
// path and the scalar path of the row kernels.
#include <cstring>

#include "common.cuh"
#include "heads_impl.cuh"
#include "rows_impl.cuh"

namespace bloth {
int last_cuda_error();
int device_fault(int reset);
long long launch_count();
}

using namespace bloth;

namespace {

constexpr int kVersion = (0 << 16) | (2 << 8) | 0;

bool is_float_dt(int dt) { return dt == BLOTH_F32 || dt == BLOTH_BF16 || dt == BLOTH_F16; }
int elem_size(int dt) { return dt == BLOTH_F32 ? 4 : 2; }
bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

template <typename F>
int dispatch_dtype(int dt, F&& f) {
  switch (dt) {
    case BLOTH_F32: return f(float{});
    case BLOTH_BF16: return f(__nv_bfloat16{});
    case BLOTH_F16: return f(__half{});
    default: return BLOTH_ERR_DTYPE;
  }
}

int64_t max_row(int dtype) { return dtype == BLOTH_F32 ? 32768 : 65536; }
constexpr int64_t kMaxScalarRow = 8192;

int check_rows(int64_t M, int64_t N, int dtype, int w_dtype) {
  if (!is_float_dt(dtype) || !is_float_dt(w_dtype)) return BLOTH_ERR_DTYPE;
  if (M < 0 || N < 1 || N > max_row(dtype)) return BLOTH_ERR_SHAPE;
  return BLOTH_OK;
}

// Whether rows with these pointers/strides can use 16-byte accesses.
bool rows_vec_ok(int dtype, int64_t N, std::initializer_list<const void*> ptrs,
                 std::initializer_list<int64_t> lds) {
  const int vec = 16 / elem_size(dtype);
  if (N % vec != 0) return false;
  for (const void* p : ptrs)
    if (!aligned(p, 16)) return false;
  for (int64_t ld : lds)
    if (ld % vec != 0) return false;
  return true;
}

int check_ld(int64_t M, int64_t N, std::initializer_list<int64_t> lds) {
  if (M <= 1) return BLOTH_OK;
  for (int64_t ld : lds)
    if (ld < N) return BLOTH_ERR_SHAPE;
  return BLOTH_OK;
}

int check_rope_table(const void* cos, const void* sin, int64_t ldcs, int cs_dtype, int64_t half,
                     int64_t M, int64_t N) {
  if (!is_float_dt(cs_dtype)) return BLOTH_ERR_DTYPE;
  if (half < 1 || 2 * half > N) return BLOTH_ERR_SHAPE;
  if (M > 0 && (cos == nullptr || sin == nullptr)) return BLOTH_ERR_NULL;
  if (M > 1 && ldcs < half) return BLOTH_ERR_SHAPE;
  return BLOTH_OK;
}

RowArgs make_rows(int64_t M, int64_t N, float eps, const void* w, float w_offset, int w_dtype) {
  RowArgs a;
  std::memset(&a, 0, sizeof(a));
  a.M = M;
  a.N = (int)N;
  a.eps = eps;
  a.w = w;
  a.w_dt = w_dtype;
  a.w_vec = aligned(w, 16) ? 1 : 0;
  a.w_off = w_offset;
  return a;
}

cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// ---- per-head validation ----
bool head_dim_ok(int64_t D) { return D == 64 || D == 128 || D == 256; }
constexpr int64_t kMaxTokens = (int64_t)1 << 31;  // B*S must stay below this

int check_heads_tensor(const void* p, const int64_t* st, int dtype) {
  if (p == nullptr || st == nullptr) return BLOTH_ERR_NULL;
  const int vec = 16 / elem_size(dtype);
  if (!aligned(p, 16)) return BLOTH_ERR_ALIGN;
  for (int i = 0; i < 3; ++i)
    if (st[i] % vec != 0) return BLOTH_ERR_ALIGN;
  return BLOTH_OK;
}

HT make_ht(const void* p, const int64_t* st) {
  HT t;
  t.p = p;
  t.sb = st ? st[0] : 0;
  t.ss = st ? st[1] : 0;
  t.sh = st ? st[2] : 0;
  return t;
}

// Position and cos/sin source shared by the per-head entry points.
int fill_rope_source(HeadArgs& a, const void* pos, const int64_t* pos_strides, int pos_dtype,
                     const float* inv_freq, const void* cos, const void* sin,
                     const int64_t* cs_strides, int64_t cs_rows, int cs_dtype,
                     float rope_scale, int dtype, int64_t D) {
  a.pos = pos;
  a.cs_scale = rope_scale;
  if (pos != nullptr) {
    if (pos_dtype != BLOTH_I64 && pos_dtype != BLOTH_I32) return BLOTH_ERR_DTYPE;
    if (pos_strides == nullptr) return BLOTH_ERR_NULL;
    a.pos_dt = pos_dtype;
    a.pos_sb = pos_strides[0];
    a.pos_ss = pos_strides[1];
  }
  const bool table = cos != nullptr || sin != nullptr;
  if (table && inv_freq != nullptr) return BLOTH_ERR_ARG;
  if (!table && inv_freq == nullptr) return BLOTH_ERR_NULL;
  if (table) {
    if (cos == nullptr || sin == nullptr || cs_strides == nullptr) return BLOTH_ERR_NULL;
    if (!is_float_dt(cs_dtype)) return BLOTH_ERR_DTYPE;
    if (cs_rows < 1) return BLOTH_ERR_SHAPE;
    a.cs_rows = cs_rows;
    a.cos = cos;
    a.sin = sin;
    a.cs_dt = cs_dtype;
    a.cs_sb = cs_strides[0];
    a.cs_sp = cs_strides[1];
    const int vec = 16 / elem_size(dtype);
    a.cs_vec = aligned(cos, 16) && aligned(sin, 16) && a.cs_sb % vec == 0 && a.cs_sp % vec == 0;
  } else {
    a.inv_freq = inv_freq;
  }
  (void)D;
  return BLOTH_OK;
}

}  // namespace

extern "C" {

int bloth_version(void) { return kVersion; }

const char* bloth_strerror(int status) {
  switch (status) {
    case BLOTH_OK: return "ok";
    case BLOTH_ERR_DTYPE: return "unsupported element type";
    case BLOTH_ERR_SHAPE: return "size out of the supported range or inconsistent sizes";
    case BLOTH_ERR_ALIGN: return "pointer or stride not aligned for the kernel's 16-byte accesses";
    case BLOTH_ERR_WORKSPACE: return "workspace missing or too small";
    case BLOTH_ERR_NULL: return "a required pointer is NULL";
    case BLOTH_ERR_CUDA: return "CUDA runtime error (see bloth_last_cuda_error)";
    case BLOTH_ERR_ARG: return "contradictory arguments";
    default: return "unknown status";
  }
}

int bloth_last_cuda_error(void) { return bloth::last_cuda_error(); }

int bloth_device_fault(int reset) { return bloth::device_fault(reset); }

int64_t bloth_kernel_launch_count(void) { return (int64_t)bloth::launch_count(); }

int bloth_selftest_wait_expiry(int limit_ms, void* stream) {
  return bloth::selftest_wait_expiry(limit_ms, as_stream(stream));
}

// ---------------------------------------------------------------- RMSNorm
int bloth_rmsnorm_fwd(const void* x, int64_t ldx, const void* w, float w_offset, void* y,
                      int64_t ldy,
                      float* rstd, int64_t M, int64_t N, float eps, int dtype, int w_dtype,
                      void* stream) {
  int rc = check_rows(M, N, dtype, w_dtype);
  if (rc) return rc;
  if (M == 0) return BLOTH_OK;
  if (!x || !w || !y || !rstd) return BLOTH_ERR_NULL;
  if ((rc = check_ld(M, N, {ldx, ldy}))) return rc;
  const bool vec = rows_vec_ok(dtype, N, {x, y}, {ldx, ldy});
  if (!vec && N > kMaxScalarRow) return BLOTH_ERR_ALIGN;
  RowArgs a = make_rows(M, N, eps, w, w_offset, w_dtype);
  a.x = x;
  a.ldx = ldx;
  a.out = y;
  a.ldo = ldy;
  a.rstd_out = rstd;
  return dispatch_dtype(dtype, [&](auto t) {
    return rows_fwd<decltype(t)>(a, kRowNorm, vec, as_stream(stream));
  });
}

size_t bloth_rmsnorm_bwd_workspace_bytes(int64_t M, int64_t N, int dtype) {
  if (check_rows(M, N, dtype, dtype)) return 0;
  size_t bytes = 0;
  dispatch_dtype(dtype, [&](auto t) {
    bytes = rows_bwd_workspace<decltype(t)>(M, (int)N, kRowNorm);
    return 0;
  });
  return bytes;
}

int bloth_rmsnorm_bwd(const void* dy, int64_t lddy, const void* x, int64_t ldx, const void* w,
                      float w_offset, const float* rstd, void* dx, int64_t lddx, void* dw, int64_t M, int64_t N,
                      int dtype, int w_dtype, void* workspace, size_t workspace_bytes,
                      void* stream) {
  int rc = check_rows(M, N, dtype, w_dtype);
  if (rc) return rc;
  if (!w || !dw) return BLOTH_ERR_NULL;
  if (M > 0 && (!dy || !x || !rstd || !dx)) return BLOTH_ERR_NULL;
  if ((rc = check_ld(M, N, {lddy, ldx, lddx}))) return rc;
  const bool vec = rows_vec_ok(dtype, N, {dy, x, dx}, {lddy, ldx, lddx});
  if (!vec && N > kMaxScalarRow) return BLOTH_ERR_ALIGN;
  RowArgs a = make_rows(M, N, 0.f, w, w_offset, w_dtype);
  a.dy = dy;
  a.lddy = lddy;
  a.x = x;
  a.ldx = ldx;
  a.out = dx;
  a.ldo = lddx;
  a.rstd_in = rstd;
  return dispatch_dtype(dtype, [&](auto t) {
    return rows_bwd<decltype(t)>(a, kRowNorm, vec, workspace, workspace_bytes, dw,
                                 as_stream(stream));
  });
}

// ------------------------------------------------- fused RMSNorm + RoPE (table)
int bloth_norm_rope_fwd(const void* x, int64_t ldx, const void* w, float w_offset, const void* cos,
                        const void* sin, int64_t ldcs, int cs_dtype, int64_t half, void* y,
                        int64_t ldy, float* rstd, int64_t M, int64_t N, float eps, int dtype,
                        int w_dtype, void* stream) {
  int rc = check_rows(M, N, dtype, w_dtype);
  if (rc) return rc;
  if ((rc = check_rope_table(cos, sin, ldcs, cs_dtype, half, M, N))) return rc;
  if (M == 0) return BLOTH_OK;
  if (!x || !w || !y || !rstd) return BLOTH_ERR_NULL;
  if ((rc = check_ld(M, N, {ldx, ldy}))) return rc;
  const bool vec = rows_vec_ok(dtype, N, {x, y}, {ldx, ldy});
  if (!vec && N > kMaxScalarRow) return BLOTH_ERR_ALIGN;
  RowArgs a = make_rows(M, N, eps, w, w_offset, w_dtype);
  a.x = x;
  a.ldx = ldx;
  a.out = y;
  a.ldo = ldy;
  a.rstd_out = rstd;
  a.cos = cos;
  a.sin = sin;
  a.ldcs = ldcs;
  a.cs_dt = cs_dtype;
  a.half = half;
  const int vecw = 16 / elem_size(dtype);
  a.cs_vec = aligned(cos, 16) && aligned(sin, 16) && ldcs % vecw == 0;
  return dispatch_dtype(dtype, [&](auto t) {
    return rows_fwd<decltype(t)>(a, kRowRope, vec, as_stream(stream));
  });
}

size_t bloth_norm_rope_bwd_workspace_bytes(int64_t M, int64_t N, int dtype) {
  if (check_rows(M, N, dtype, dtype)) return 0;
  size_t bytes = 0;
  dispatch_dtype(dtype, [&](auto t) {
    bytes = rows_bwd_workspace<decltype(t)>(M, (int)N, kRowRope);
    return 0;
  });
  return bytes;
}

int bloth_norm_rope_bwd(const void* dy, int64_t lddy, const void* x, int64_t ldx, const void* w,
                        float w_offset, const void* cos, const void* sin, int64_t ldcs, int cs_dtype,
                        int64_t half, const float* rstd, void* dx, int64_t lddx, void* dw,
                        int64_t M, int64_t N, int dtype, int w_dtype, void* workspace,
                        size_t workspace_bytes, void* stream) {
  int rc = check_rows(M, N, dtype, w_dtype);
  if (rc) return rc;
  if ((rc = check_rope_table(cos, sin, ldcs, cs_dtype, half, M, N))) return rc;
  if (!w || !dw) return BLOTH_ERR_NULL;
  if (M > 0 && (!dy || !x || !rstd || !dx)) return BLOTH_ERR_NULL;
  if ((rc = check_ld(M, N, {lddy, ldx, lddx}))) return rc;
  const bool vec = rows_vec_ok(dtype, N, {dy, x, dx}, {lddy, ldx, lddx});
  if (!vec && N > kMaxScalarRow) return BLOTH_ERR_ALIGN;
  RowArgs a = make_rows(M, N, 0.f, w, w_offset, w_dtype);
  a.dy = dy;
  a.lddy = lddy;
  a.x = x;
  a.ldx = ldx;
  a.out = dx;
  a.ldo = lddx;
  a.rstd_in = rstd;
  a.cos = cos;
  a.sin = sin;
  a.ldcs = ldcs;
  a.cs_dt = cs_dtype;
  a.half = half;
  const int vecw = 16 / elem_size(dtype);
  a.cs_vec = aligned(cos, 16) && aligned(sin, 16) && ldcs % vecw == 0;
  return dispatch_dtype(dtype, [&](auto t) {
    return rows_bwd<decltype(t)>(a, kRowRope, vec, workspace, workspace_bytes, dw,
                                 as_stream(stream));
  });
}

// ------------------------------------------------ residual add + RMSNorm
int bloth_add_rmsnorm_fwd(const void* x, int64_t ldx, const void* r, int64_t ldr, void* z,
                          int64_t ldz, const void* w, float w_offset, void* y, int64_t ldy,
                          float* rstd, int64_t M, int64_t N, float eps, int dtype, int w_dtype,
                          void* stream) {
  int rc = check_rows(M, N, dtype, w_dtype);
  if (rc) return rc;
  if (M == 0) return BLOTH_OK;
  if (!x || !r || !z || !w || !y || !rstd) return BLOTH_ERR_NULL;
  if ((rc = check_ld(M, N, {ldx, ldr, ldz, ldy}))) return rc;
  const bool vec = rows_vec_ok(dtype, N, {x, r, z, y}, {ldx, ldr, ldz, ldy});
  if (!vec && N > kMaxScalarRow) return BLOTH_ERR_ALIGN;
  RowArgs a = make_rows(M, N, eps, w, w_offset, w_dtype);
  a.x = x;
  a.ldx = ldx;
  a.res = r;
  a.ldres = ldr;
  a.res_out = z;
  a.ldres_out = ldz;
  a.out = y;
  a.ldo = ldy;
  a.rstd_out = rstd;
  return dispatch_dtype(dtype, [&](auto t) {
    return rows_fwd<decltype(t)>(a, kRowAdd, vec, as_stream(stream));
  });
}

size_t bloth_add_rmsnorm_bwd_workspace_bytes(int64_t M, int64_t N, int dtype) {
  if (check_rows(M, N, dtype, dtype)) return 0;
  size_t bytes = 0;
  dispatch_dtype(dtype, [&](auto t) {
    bytes = rows_bwd_workspace<decltype(t)>(M, (int)N, kRowAdd);
    return 0;
  });
  return bytes;
}

int bloth_add_rmsnorm_bwd(const void* dy, int64_t lddy, const void* dz_out, int64_t lddz_out,
                          const void* z, int64_t ldz, const void* w, float w_offset,
                          const float* rstd, void* dz, int64_t lddz, void* dw, int64_t M,
                          int64_t N, int dtype, int w_dtype, void* workspace,
                          size_t workspace_bytes, void* stream) {
  int rc = check_rows(M, N, dtype, w_dtype);
  if (rc) return rc;
  if (!w || !dw) return BLOTH_ERR_NULL;
  if (M > 0 && (!dy || !z || !rstd || !dz)) return BLOTH_ERR_NULL;
  const int64_t ld_g = dz_out ? lddz_out : N;
  if ((rc = check_ld(M, N, {lddy, ld_g, ldz, lddz}))) return rc;
  const bool vec = dz_out ? rows_vec_ok(dtype, N, {dy, dz_out, z, dz}, {lddy, lddz_out, ldz, lddz})
                          : rows_vec_ok(dtype, N, {dy, z, dz}, {lddy, ldz, lddz});
  if (!vec && N > kMaxScalarRow) return BLOTH_ERR_ALIGN;
  RowArgs a = make_rows(M, N, 0.f, w, w_offset, w_dtype);
  a.dy = dy;
  a.lddy = lddy;
  a.x = z;
  a.ldx = ldz;
  a.res = dz_out;
  a.ldres = ld_g;
  a.out = dz;
  a.ldo = lddz;
  a.rstd_in = rstd;
  return dispatch_dtype(dtype, [&](auto t) {
    return rows_bwd<decltype(t)>(a, kRowAdd, vec, workspace, workspace_bytes, dw,
                                 as_stream(stream));
  });
}

// ------------------------------------------------------ per-head q/k kernels
int bloth_qk_norm_rope_fwd(const void* q, const int64_t* q_strides, const void* k,
                           const int64_t* k_strides, const void* wq, const void* wk,
                           float w_offset, void* q_out, const int64_t* qo_strides, void* k_out,
                           const int64_t* ko_strides, float* rstd_q, float* rstd_k,
                           const void* pos, const int64_t* pos_strides, int pos_dtype,
                           const float* inv_freq, const void* cos, const void* sin,
                           const int64_t* cs_strides, int64_t cs_rows, int cs_dtype,
                           float rope_scale, int64_t B, int64_t S, int64_t Hq,
                           int64_t Hk, int64_t D, float eps, int dtype, int w_dtype, void* stream) {
  if (!is_float_dt(dtype) || !is_float_dt(w_dtype)) return BLOTH_ERR_DTYPE;
  if (!head_dim_ok(D) || B < 0 || S < 0 || Hq < 0 || Hk < 0 || Hq + Hk < 1 || Hq > (1 << 20) ||
      Hk > (1 << 20) || (S > 0 && B >= kMaxTokens / S))
    return BLOTH_ERR_SHAPE;
  HeadArgs a;
  std::memset(&a, 0, sizeof(a));
  a.fault = fault_word();
  int rc = fill_rope_source(a, pos, pos_strides, pos_dtype, inv_freq, cos, sin, cs_strides,
                            cs_rows, cs_dtype, rope_scale, dtype, D);
  if (rc) return rc;
  if (B * S == 0) return BLOTH_OK;
  const void* src[2] = {q, k};
  const int64_t* sst[2] = {q_strides, k_strides};
  void* dst[2] = {q_out, k_out};
  const int64_t* dstst[2] = {qo_strides, ko_strides};
  const void* w[2] = {wq, wk};
  float* rs[2] = {rstd_q, rstd_k};
  const int64_t H[2] = {Hq, Hk};
  for (int t = 0; t < 2; ++t) {
    if (H[t] == 0) continue;
    if ((rc = check_heads_tensor(src[t], sst[t], dtype))) return rc;
    if ((rc = check_heads_tensor(dst[t], dstst[t], dtype))) return rc;
    if (w[t] == nullptr || rs[t] == nullptr) return BLOTH_ERR_NULL;
    if (!aligned(w[t], 16)) return BLOTH_ERR_ALIGN;
    a.src[t] = make_ht(src[t], sst[t]);
    a.dst[t] = make_ht(dst[t], dstst[t]);
    a.w[t] = w[t];
    a.rstd_out[t] = rs[t];
    a.H[t] = (int)H[t];
  }
  a.w_dt = w_dtype;
  a.w_off = w_offset;
  a.B = B;
  a.S = S;
  a.eps = eps;
  return dispatch_dtype(dtype, [&](auto t) {
    return heads_fwd<decltype(t)>(a, (int)D, true, as_stream(stream));
  });
}

size_t bloth_qk_norm_rope_bwd_workspace_bytes(int64_t B, int64_t S, int64_t D, int dtype) {
  if (!is_float_dt(dtype) || !head_dim_ok(D) || B < 0 || S < 0) return 0;
  size_t bytes = 0;
  dispatch_dtype(dtype, [&](auto t) {
    bytes = heads_bwd_workspace<decltype(t)>(B * S, (int)D);
    return 0;
  });
  return bytes;
}

int bloth_qk_norm_rope_bwd(const void* dq_out, const int64_t* dqo_strides, const void* dk_out,
                           const int64_t* dko_strides, const void* q, const int64_t* q_strides,
                           const void* k, const int64_t* k_strides, const void* wq,
                           const void* wk, float w_offset, const float* rstd_q,
                           const float* rstd_k, void* dq,
                           const int64_t* dq_strides, void* dk, const int64_t* dk_strides,
                           void* dwq, void* dwk, const void* pos, const int64_t* pos_strides,
                           int pos_dtype, const float* inv_freq, const void* cos,
                           const void* sin, const int64_t* cs_strides, int64_t cs_rows,
                           int cs_dtype, float rope_scale, int64_t B, int64_t S, int64_t Hq,
                           int64_t Hk, int64_t D,
                           int dtype, int w_dtype, void* workspace, size_t workspace_bytes,
                           void* stream) {
  if (!is_float_dt(dtype) || !is_float_dt(w_dtype)) return BLOTH_ERR_DTYPE;
  if (!head_dim_ok(D) || B < 0 || S < 0 || Hq < 0 || Hk < 0 || Hq + Hk < 1 || Hq > (1 << 20) ||
      Hk > (1 << 20) || (S > 0 && B >= kMaxTokens / S))
    return BLOTH_ERR_SHAPE;
  HeadArgs a;
  std::memset(&a, 0, sizeof(a));
  a.fault = fault_word();
  int rc = fill_rope_source(a, pos, pos_strides, pos_dtype, inv_freq, cos, sin, cs_strides,
                            cs_rows, cs_dtype, rope_scale, dtype, D);
  if (rc) return rc;
  const void* g[2] = {dq_out, dk_out};
  const int64_t* gst[2] = {dqo_strides, dko_strides};
  const void* x[2] = {q, k};
  const int64_t* xst[2] = {q_strides, k_strides};
  void* dst[2] = {dq, dk};
  const int64_t* dstst[2] = {dq_strides, dk_strides};
  const void* w[2] = {wq, wk};
  const float* rs[2] = {rstd_q, rstd_k};
  void* dw[2] = {dwq, dwk};
  const int64_t H[2] = {Hq, Hk};
  for (int t = 0; t < 2; ++t) {
    if (H[t] == 0) continue;
    if (w[t] == nullptr || dw[t] == nullptr) return BLOTH_ERR_NULL;
    if (!aligned(w[t], 16)) return BLOTH_ERR_ALIGN;
    a.w[t] = w[t];
    a.H[t] = (int)H[t];
    if (B * S == 0) continue;
    if ((rc = check_heads_tensor(g[t], gst[t], dtype))) return rc;
    if ((rc = check_heads_tensor(x[t], xst[t], dtype))) return rc;
    if ((rc = check_heads_tensor(dst[t], dstst[t], dtype))) return rc;
    if (rs[t] == nullptr) return BLOTH_ERR_NULL;
    a.src[t] = make_ht(g[t], gst[t]);
    a.x[t] = make_ht(x[t], xst[t]);
    a.dst[t] = make_ht(dst[t], dstst[t]);
    a.rstd_in[t] = rs[t];
  }
  a.w_dt = w_dtype;
  a.w_off = w_offset;
  a.B = B;
  a.S = S;
  a.rstd_bulk = (Hq % 4 == 0) && (Hk % 4 == 0) && aligned(rstd_q, 16) &&
                (Hk == 0 || aligned(rstd_k, 16));
  return dispatch_dtype(dtype, [&](auto t) {
    return heads_bwd<decltype(t)>(a, (int)D, workspace, workspace_bytes, dwq,
                                  Hk > 0 ? dwk : nullptr, as_stream(stream));
  });
}

int bloth_rope(const void* q, const int64_t* q_strides, void* q_out, const int64_t* qo_strides,
               const void* k, const int64_t* k_strides, void* k_out, const int64_t* ko_strides,
               const void* pos, const int64_t* pos_strides, int pos_dtype, const float* inv_freq,
               const void* cos, const void* sin, const int64_t* cs_strides, int64_t cs_rows,
               int cs_dtype, float rope_scale, int64_t B, int64_t S, int64_t Hq, int64_t Hk,
               int64_t D, int transpose, int dtype, void* stream) {
  if (!is_float_dt(dtype)) return BLOTH_ERR_DTYPE;
  if (!head_dim_ok(D) || B < 0 || S < 0 || Hq < 0 || Hk < 0 || Hq + Hk < 1 || Hq > (1 << 20) ||
      Hk > (1 << 20) || (S > 0 && B >= kMaxTokens / S))
    return BLOTH_ERR_SHAPE;
  HeadArgs a;
  std::memset(&a, 0, sizeof(a));
  a.fault = fault_word();
  int rc = fill_rope_source(a, pos, pos_strides, pos_dtype, inv_freq, cos, sin, cs_strides,
                            cs_rows, cs_dtype, rope_scale, dtype, D);
  if (rc) return rc;
  if (B * S == 0) return BLOTH_OK;
  const void* src[2] = {q, k};
  const int64_t* sst[2] = {q_strides, k_strides};
  void* dst[2] = {q_out, k_out};
  const int64_t* dstst[2] = {qo_strides, ko_strides};
  const int64_t H[2] = {Hq, Hk};
  for (int t = 0; t < 2; ++t) {
    if (H[t] == 0) continue;
    if ((rc = check_heads_tensor(src[t], sst[t], dtype))) return rc;
    if ((rc = check_heads_tensor(dst[t], dstst[t], dtype))) return rc;
    a.src[t] = make_ht(src[t], sst[t]);
    a.dst[t] = make_ht(dst[t], dstst[t]);
    a.H[t] = (int)H[t];
  }
  a.B = B;
  a.S = S;
  a.transpose = transpose ? 1 : 0;
  a.w_dt = BLOTH_F32;
  return dispatch_dtype(dtype, [&](auto t) {
    return heads_fwd<decltype(t)>(a, (int)D, false, as_stream(stream));
  });
}

}  // extern "C"
