/*
 * bloth_b200.h - C ABI of the B200 (sm_100a) RMSNorm and fused RMSNorm+RoPE kernels.
 *
 * Plain C: raw device pointers, element strides, an element-type code and a
 * cudaStream_t passed as void*. Nothing here allocates; the caller owns every
 * buffer, including the weight-gradient workspace whose size the
 * *_workspace_bytes() functions report (its base aligned to 8 bytes, or 4 for
 * 16-bit tensors: BLOTH_ERR_ALIGN otherwise; 16-byte aligned bases are
 * written with 16-byte stores). Every entry point is asynchronous on
 * the given stream, returns BLOTH_OK or a status code (never aborts), and
 * keeps no state between calls apart from per-device launch caches. The
 * device used is the calling thread's current CUDA device, and the stream
 * passed must belong to that device (launch sizes, shared-memory limits and
 * device addresses are looked up for the current device).
 *
 * Row convention (as in the reference's Triton kernels): a "row" is one
 * normalised vector of N elements; x[row, col] is at x + row*ldx + col.
 * Head convention (per-head q/k kernels): element [b, s, h, d] of a
 * [B, S, H, D] head tensor is at ptr + b*strides[0] + s*strides[1] +
 * h*strides[2] + d, i.e. the head dimension is contiguous.
 *
 * Weight offset: every normalising entry point takes w_offset, a constant
 * added in fp32 to each weight element before it multiplies the normalised
 * value: 0 for the usual x_hat * w (Llama, Qwen, Mistral, the reference's
 * kernels), 1 for the (1 + w) weighting of Gemma-family norms
 * (transformers GemmaRMSNorm.forward). The weight gradient is the same for
 * both (d(w + c)/dw = 1).
 */
#ifndef BLOTH_B200_H_
#define BLOTH_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* element types */
#define BLOTH_F32 0
#define BLOTH_BF16 1
#define BLOTH_F16 2
#define BLOTH_I32 3
#define BLOTH_I64 4

/* status codes */
#define BLOTH_OK 0
#define BLOTH_ERR_DTYPE 1     /* unsupported element-type combination */
#define BLOTH_ERR_SHAPE 2     /* size out of the supported range, or inconsistent sizes */
#define BLOTH_ERR_ALIGN 3     /* a pointer or stride the kernel cannot address */
#define BLOTH_ERR_WORKSPACE 4 /* workspace missing or smaller than *_workspace_bytes() */
#define BLOTH_ERR_NULL 5      /* a required pointer is NULL */
#define BLOTH_ERR_CUDA 6      /* the CUDA runtime reported an error; see bloth_last_cuda_error() */
#define BLOTH_ERR_ARG 7       /* contradictory arguments (e.g. both cos/sin tables and inv_freq) */

/* Largest row length of the row kernels (the reference's limit,
   bloth/bloth/kernels/rms_norm.py:21 MAX_FUSED_SIZE): 65536 for 16-bit
   rows, 32768 for fp32 rows. Rows whose base or stride is not 16-byte
   aligned run on a scalar path limited to 8192. */
#define BLOTH_MAX_ROW 65536

/* Library version, (major << 16) | (minor << 8) | patch. */
int bloth_version(void);

/* Human-readable text of a status code (static storage). */
const char* bloth_strerror(int status);

/* cudaError_t of the last failing CUDA call made by the calling thread inside
   this library (0 if none). */
int bloth_last_cuda_error(void);

/* Fault bits kernels recorded on the current device since the last reset.
   Bit 0: a bulk-copy completion wait gave up after its time limit (2 s) and
   the kernel returned early, after waiting (with the same limit) for the
   copies it had already issued; the outputs of that call are invalid.
   Bit 1: one of those waits for already-issued copies gave up as well.
   Synchronises with the device; reset != 0 clears the bits. Negative on a
   CUDA error. The kernels never read this word: a caller that must know
   whether a step's results are valid reads it after the step. */
int bloth_device_fault(int reset);
/* Diagnostic: one thread runs the kernels' expiry path on a two-slot ring
   without any fault. One slot's copy is issued normally; the other slot
   expects bytes whose copy is issued only after its bounded wait has given up
   after limit_ms (1..2000), which sets fault bit 0 on the current device as a
   real expired copy would. The ring is then drained as the kernels drain it;
   both copies land, so bit 1 stays clear and nothing is in flight when the
   kernel returns. Lets a deployment confirm that an expired wait ends the
   kernel and reaches bloth_device_fault(). No counterpart in the reference. */
int bloth_selftest_wait_expiry(int limit_ms, void* stream);

/* Kernels this library has launched (or recorded into a capturing stream) in
   this process, over all threads and devices. No counterpart in the
   reference. */
int64_t bloth_kernel_launch_count(void);

/* ------------------------------------------------------------------------
 * RMSNorm over rows of N: y = x * rsqrt(mean(x^2) + eps) * w, computed in
 * fp32 and rounded once to the type of x; rstd[M] (fp32) saved for backward.
 * Replaces the _rms_norm_fwd_kernel launch of _RMSNormFunction.forward
 * (bloth/bloth/kernels/rms_norm.py:119-140; kernel :39-73).
 * dtype: type of x and y (F32, BF16, F16); w_dtype: type of w (F32 or dtype).
 * ---------------------------------------------------------------------- */
int bloth_rmsnorm_fwd(const void* x, int64_t ldx, const void* w, float w_offset, void* y,
                      int64_t ldy, float* rstd, int64_t M, int64_t N, float eps, int dtype, int w_dtype,
                      void* stream);

/* Bytes of workspace bloth_rmsnorm_bwd needs for M rows of N on the current
   device (per-CTA weight-gradient partial sums). */
size_t bloth_rmsnorm_bwd_workspace_bytes(int64_t M, int64_t N, int dtype);

/* RMSNorm backward: dx = rstd * (dy*w - xhat * mean(dy*w*xhat)), xhat = x*rstd,
   and dw = sum over rows of dy*xhat written in w_dtype. dw is reduced
   deterministically (per-CTA partials in the workspace, then a fixed-order
   sum), not with atomics.
   Replaces _RMSNormFunction.backward (bloth/bloth/kernels/rms_norm.py:143-160;
   kernel :76-113). */
int bloth_rmsnorm_bwd(const void* dy, int64_t lddy, const void* x, int64_t ldx, const void* w,
                      float w_offset, const float* rstd, void* dx, int64_t lddx, void* dw, int64_t M, int64_t N,
                      int dtype, int w_dtype, void* workspace, size_t workspace_bytes,
                      void* stream);

/* Bytes of the static device scratch that bloth_rmsnorm_bwd_noalloc uses in
   place of a workspace (held by every GPU that loads the library). */
#define BLOTH_NOALLOC_SCRATCH_BYTES (16u * 1024u * 1024u)

/* bloth_rmsnorm_bwd for callers that cannot allocate device memory (an
   operator interface that passes only inputs and outputs, or a process whose
   device memory is reserved by another allocator). Same arguments minus the
   workspace, same results: the weight-gradient partial sums live in a
   library-owned static device array of BLOTH_NOALLOC_SCRATCH_BYTES. Returns
   BLOTH_ERR_WORKSPACE, doing nothing, when the call needs more partial-sum
   space than that (bloth_rmsnorm_bwd_workspace_bytes(M, N, dtype) >
   BLOTH_NOALLOC_SCRATCH_BYTES). Allocates nothing. The first call on each
   device sets up the array's device address (make it before any stream
   capture). As for every entry point, the stream must belong to the calling
   thread's current device: the array's address and the launch size are those
   of the current device. All calls share the array, so calls that overlap on
   the GPU race. No counterpart in the reference. */
int bloth_rmsnorm_bwd_noalloc(const void* dy, int64_t lddy, const void* x, int64_t ldx,
                              const void* w, float w_offset, const float* rstd, void* dx, int64_t lddx, void* dw,
                              int64_t M, int64_t N, int dtype, int w_dtype, void* stream);

/* ------------------------------------------------------------------------
 * Residual add + RMSNorm over rows of N: z = x + r rounded to the type of x
 * (stored: the decoder's residual stream), then y = z * rsqrt(mean(z^2) +
 * eps) * (w + w_offset) in fp32, rounded once; rstd[M] fp32 saved. One pass
 * over the rows instead of an add kernel and a norm kernel. z may be the same
 * buffer as x or r (in place); other overlaps are undefined.
 * No counterpart in the reference (which has no residual fusion): it fuses
 * HF's `hidden_states = residual + hidden_states` with the
 * post_attention_layernorm call that follows it in every Llama-family decoder
 * layer (transformers models/llama/modeling_llama.py, LlamaDecoderLayer).
 * ---------------------------------------------------------------------- */
int bloth_add_rmsnorm_fwd(const void* x, int64_t ldx, const void* r, int64_t ldr, void* z,
                          int64_t ldz, const void* w, float w_offset, void* y, int64_t ldy,
                          float* rstd, int64_t M, int64_t N, float eps, int dtype, int w_dtype,
                          void* stream);
size_t bloth_add_rmsnorm_bwd_workspace_bytes(int64_t M, int64_t N, int dtype);
/* Backward of bloth_add_rmsnorm_fwd: dz = dz_out + the RMSNorm gradient of z
   for dy, which is the gradient of both x and r; dw as bloth_rmsnorm_bwd.
   dz_out (the gradient reaching z from the rest of the residual stream) may
   be NULL, meaning zero. dz may be the same buffer as dy or dz_out. */
int bloth_add_rmsnorm_bwd(const void* dy, int64_t lddy, const void* dz_out, int64_t lddz_out,
                          const void* z, int64_t ldz, const void* w, float w_offset,
                          const float* rstd, void* dz, int64_t lddz, void* dw, int64_t M,
                          int64_t N, int dtype, int w_dtype, void* workspace,
                          size_t workspace_bytes, void* stream);
/* ------------------------------------------------------------------------
 * Fused RMSNorm + rotate-half RoPE with per-row cos/sin tables, the
 * reference's fused_norm_rope(x, weight, cos, sin, eps) contract: each row of
 * N is RMS-normalised over all N columns; columns [0, 2*half) are rotated in
 * pairs (c, c+half) with cos/sin[row, c]: y1 = n1*cos - n2*sin,
 * y2 = n1*sin + n2*cos; columns >= 2*half are only normalised.
 * cos/sin: [M, half] with row stride ldcs, type cs_dtype (F32, BF16, F16).
 * Replaces _FusedNormRoPEFunction.forward
 * (bloth/bloth/kernels/fused_norm_qkv_rope.py:132-159; kernel :40-96).
 * ---------------------------------------------------------------------- */
int bloth_norm_rope_fwd(const void* x, int64_t ldx, const void* w, float w_offset, const void* cos,
                        const void* sin, int64_t ldcs, int cs_dtype, int64_t half, void* y,
                        int64_t ldy, float* rstd, int64_t M, int64_t N, float eps, int dtype,
                        int w_dtype, void* stream);

size_t bloth_norm_rope_bwd_workspace_bytes(int64_t M, int64_t N, int dtype);

/* Backward of bloth_norm_rope_fwd: applies the transposed rotation to dy,
   then the RMSNorm backward; dw in w_dtype. This is the gradient of the
   forward above; the reference's _fused_norm_rope_bwd_kernel
   (bloth/bloth/kernels/fused_norm_qkv_rope.py:99-126) omits the rotation.
   Replaces _FusedNormRoPEFunction.backward (:161-176). */
int bloth_norm_rope_bwd(const void* dy, int64_t lddy, const void* x, int64_t ldx, const void* w,
                        float w_offset, const void* cos, const void* sin, int64_t ldcs, int cs_dtype,
                        int64_t half, const float* rstd, void* dx, int64_t lddx, void* dw,
                        int64_t M, int64_t N, int dtype, int w_dtype, void* workspace,
                        size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------
 * Per-head q/k RMSNorm + RoPE over [B, S, H, D] head tensors in one launch.
 * Each (token, head) row of D is normalised with its tensor's weight (wq for
 * q, wk for k), then rotated in pairs (d, d + D/2) by the angle of the
 * token's position. cos/sin come from exactly one of:
 *   - inv_freq [D/2] fp32: angle = float(pos) * inv_freq[i] rounded to fp32,
 *     cos/sin evaluated in-register once per token and shared by all heads;
 *   - cos/sin tables: row = table + b*cs_strides[0] + p*cs_strides[1], with
 *     p = pos[b, s] (or s when pos is NULL) clamped to [0, cs_rows - 1];
 *     elements [0, D/2) of the row are used, so full-width [.., D] tables
 *     with duplicated halves also work.
 * rope_scale multiplies cos and sin from either source (HF's
 *   attention_scaling of YaRN / LongRoPE rotary embeddings; 1 otherwise).
 * pos: [B, S] positions (I64 or I32) at pos + b*pos_strides[0] +
 *   s*pos_strides[1]; NULL means pos = s. Packed sequences pass positions that
 *   restart at each document.
 * rstd_q [B*S*Hq], rstd_k [B*S*Hk]: fp32, token-major, saved for backward.
 * k, wk, k_out, rstd_k may be NULL when Hk == 0. D: 64, 128 or 256.
 * New entry point with no single counterpart in the reference: it fuses the
 * reference's per-row fused_norm_rope (fused_norm_qkv_rope.py:40-96) for both
 * tensors with the cos/sin construction of BlothRoPE._build_cache
 * (bloth/bloth/ops/rope.py:71-77), replacing the HF q_norm/k_norm +
 * apply_rotary_pos_emb pair that patch_model leaves in place (patch.py:46-76).
 * ---------------------------------------------------------------------- */
int bloth_qk_norm_rope_fwd(const void* q, const int64_t* q_strides, const void* k,
                           const int64_t* k_strides, const void* wq, const void* wk,
                           float w_offset, void* q_out, const int64_t* qo_strides, void* k_out,
                           const int64_t* ko_strides, float* rstd_q, float* rstd_k,
                           const void* pos, const int64_t* pos_strides, int pos_dtype,
                           const float* inv_freq, const void* cos, const void* sin,
                           const int64_t* cs_strides, int64_t cs_rows, int cs_dtype,
                           float rope_scale, int64_t B, int64_t S, int64_t Hq,
                           int64_t Hk, int64_t D, float eps, int dtype, int w_dtype, void* stream);

size_t bloth_qk_norm_rope_bwd_workspace_bytes(int64_t B, int64_t S, int64_t D, int dtype);

/* Backward of bloth_qk_norm_rope_fwd: dq, dk (same layout rules) and the
   weight gradients dwq, dwk [D] in w_dtype (reduced deterministically through
   the workspace). dk, dwk may be NULL when Hk == 0. */
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
                           void* stream);

/* ------------------------------------------------------------------------
 * Rotate-half RoPE alone over q [B, S, Hq, D] and k [B, S, Hk, D] head
 * tensors in one launch (same cos/sin, position and rope_scale rules as
 * above; k, k_out may be NULL when Hk == 0). transpose = 0 applies the
 * rotation (y1 = x1*cos - x2*sin, y2 = x1*sin + x2*cos); transpose = 1
 * applies its transpose, which is the backward (dx from dy).
 * Replaces rope_embedding / _rope_kernel (bloth/bloth/ops/rope.py:9-58), which
 * is forward-only, rotates one tensor and always stores bf16; here the
 * outputs have the inputs' type. With q and k it also replaces HF's
 * apply_rotary_pos_emb(q, k, cos, sin) for RoPE-only attention (Llama,
 * Mistral, Qwen2).
 * ---------------------------------------------------------------------- */
int bloth_rope(const void* q, const int64_t* q_strides, void* q_out, const int64_t* qo_strides,
               const void* k, const int64_t* k_strides, void* k_out, const int64_t* ko_strides,
               const void* pos, const int64_t* pos_strides, int pos_dtype, const float* inv_freq,
               const void* cos, const void* sin, const int64_t* cs_strides, int64_t cs_rows,
               int cs_dtype, float rope_scale, int64_t B, int64_t S, int64_t Hq, int64_t Hk,
               int64_t D, int transpose, int dtype, void* stream);
#ifdef __cplusplus
}
#endif

#endif /* BLOTH_B200_H_ */
