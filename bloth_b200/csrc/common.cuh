// Shared device helpers for the RMSNorm / RoPE kernels: element conversion,
// 16-byte packed global loads and stores, warp and row-group reductions, and
// the host-side launch bookkeeping (SM count and occupancy caches).
//
// Every kernel in this library is HBM-bound: each element is read once from
// global memory as part of a 16-byte vector, converted to fp32, reduced with
// warp shuffles, and written once. Tensor cores are not used.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include <type_traits>

#include "../../include/bloth_b200.h"

namespace bloth {

// ---------------------------------------------------------------------------
// element conversion
// ---------------------------------------------------------------------------
__device__ __forceinline__ float to_f(float v) { return v; }
__device__ __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
__device__ __forceinline__ float to_f(__half v) { return __half2float(v); }

template <typename T> __device__ __forceinline__ T from_f(float v);
template <> __device__ __forceinline__ float from_f<float>(float v) { return v; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}
template <> __device__ __forceinline__ __half from_f<__half>(float v) { return __float2half_rn(v); }

template <typename T> struct DTypeOf;
template <> struct DTypeOf<float> { static constexpr int value = BLOTH_F32; };
template <> struct DTypeOf<__nv_bfloat16> { static constexpr int value = BLOTH_BF16; };
template <> struct DTypeOf<__half> { static constexpr int value = BLOTH_F16; };

// Accumulator type of the weight-gradient partial sums: fp64 for fp32 tensors
// (so that dweight stays within a few fp32 ulps of the exact sum at any row
// count), fp32 for 16-bit tensors (whose dweight is rounded to 16 bits anyway).
template <typename T> struct AccOf { using type = float; };
template <> struct AccOf<float> { using type = double; };

// Stores a thread's VEC consecutive accumulators v to dst[0 .. VEC) (n of
// them, n <= VEC, are in range): as 16-byte stores when all VEC are in range
// and dst is 16-byte aligned, else one by one. A warp's partial-row stores
// then move 16 bytes per lane per instruction instead of 4 or 8; with scalar
// stores the partial rows of the RMSNorm backward took 2 us of a 27 us
// launch at 4096 rows of 4096 (measured on B200).
template <typename AccT, int VEC>
__device__ __forceinline__ void store_acc_vec(AccT* dst, const AccT (&v)[VEC], int n) {
  constexpr int PER16 = 16 / (int)sizeof(AccT);
  if constexpr (VEC % PER16 == 0) {
    if (n >= VEC && (reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
#pragma unroll
      for (int e = 0; e < VEC; e += PER16) {
        if constexpr (PER16 == 4)
          *reinterpret_cast<float4*>(dst + e) = make_float4(v[e], v[e + 1], v[e + 2], v[e + 3]);
        else
          *reinterpret_cast<double2*>(dst + e) = make_double2(v[e], v[e + 1]);
      }
      return;
    }
  }
#pragma unroll
  for (int e = 0; e < VEC; ++e)
    if (e < n) dst[e] = v[e];
}

// Programmatic dependent launch (sm_90+). A kernel launched with
// launch_dependent() may start while the kernel before it in the stream is
// still running, once every CTA of that kernel has executed
// allow_dependent_launch() (or exited); it must call wait_for_prior_grid()
// before its first global memory access, which returns once the prior kernel
// has completed and its writes are visible. Kernels not launched that way
// pass through both instructions.
__device__ __forceinline__ void allow_dependent_launch() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void wait_for_prior_grid() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}

// ---------------------------------------------------------------------------
// packed global access: VEC elements of T as one aligned access
// ---------------------------------------------------------------------------
template <typename T, int VEC>
struct alignas(sizeof(T) * VEC) Pack {
  T v[VEC];
};

template <int NB> struct RawOf;
template <> struct RawOf<16> { using type = uint4; };
template <> struct RawOf<8> { using type = uint2; };
template <> struct RawOf<4> { using type = unsigned int; };
template <> struct RawOf<2> { using type = unsigned short; };

// Read-only (non-coherent) load of one pack. Inputs are never written by the
// kernel that reads them, so the read-only path is always legal here.
template <typename T, int VEC>
__device__ __forceinline__ Pack<T, VEC> ldg_pack(const T* p) {
  using R = typename RawOf<sizeof(T) * VEC>::type;
  R r = __ldg(reinterpret_cast<const R*>(p));
  Pack<T, VEC> out;
  memcpy(&out, &r, sizeof(out));
  return out;
}

template <typename T, int VEC>
__device__ __forceinline__ void stg_pack(T* p, const Pack<T, VEC>& v) {
  *reinterpret_cast<Pack<T, VEC>*>(p) = v;
}

// Store with the streaming (evict-first) cache hint, for outputs this kernel
// never reads back: their lines leave L2 for DRAM first, ahead of lines still
// being filled. 16-byte packs only (p 16-byte aligned).
template <typename T, int VEC>
__device__ __forceinline__ void stg_pack_stream(T* p, const Pack<T, VEC>& v) {
  static_assert(sizeof(Pack<T, VEC>) == 16, "streaming stores take 16-byte packs");
  uint32_t w[4];
  memcpy(w, &v, 16);
  asm volatile("st.global.cs.v4.b32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(w[0]), "r"(w[1]),
               "r"(w[2]), "r"(w[3])
               : "memory");
}

template <typename T, int VEC>
__device__ __forceinline__ void unpack(const Pack<T, VEC>& pk, float (&f)[VEC]) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value && VEC % 2 == 0) {
    // A bf16 value is the upper half of the fp32 with the same bits, so each
    // element of a packed pair converts with one shift or mask of the word.
    uint32_t w[VEC / 2];
    memcpy(w, &pk, sizeof(w));
#pragma unroll
    for (int q = 0; q < VEC / 2; ++q) {
      f[2 * q] = __uint_as_float(w[q] << 16);
      f[2 * q + 1] = __uint_as_float(w[q] & 0xffff0000u);
    }
  } else {
#pragma unroll
    for (int e = 0; e < VEC; ++e) f[e] = to_f(pk.v[e]);
  }
}

// Rounds VEC floats to T (nearest even); 16-bit types convert two at a time
// (one cvt.rn.{bf16x2,f16x2}.f32 per pair).
template <typename T, int VEC>
__device__ __forceinline__ Pack<T, VEC> pack(const float (&f)[VEC]) {
  Pack<T, VEC> pk;
  if constexpr (sizeof(T) == 2 && VEC % 2 == 0) {
#pragma unroll
    for (int e = 0; e < VEC; e += 2) {
      if constexpr (std::is_same<T, __nv_bfloat16>::value) {
        const __nv_bfloat162 h = __floats2bfloat162_rn(f[e], f[e + 1]);
        pk.v[e] = h.x;
        pk.v[e + 1] = h.y;
      } else {
        const __half2 h = __floats2half2_rn(f[e], f[e + 1]);
        pk.v[e] = h.x;
        pk.v[e + 1] = h.y;
      }
    }
  } else {
#pragma unroll
    for (int e = 0; e < VEC; ++e) pk.v[e] = from_f<T>(f[e]);
  }
  return pk;
}

// Scalar load of element i of a tensor whose element type is only known at
// run time (weights, cos/sin tables). The switch is uniform across the grid.
__device__ __forceinline__ float ld_any(const void* base, int64_t i, int dt) {
  switch (dt) {
    case BLOTH_BF16: return __bfloat162float(__ldg(reinterpret_cast<const __nv_bfloat16*>(base) + i));
    case BLOTH_F16: return __half2float(__ldg(reinterpret_cast<const __half*>(base) + i));
    default: return __ldg(reinterpret_cast<const float*>(base) + i);
  }
}

// VEC consecutive elements starting at element i, runtime element type.
// `vec_ok` promises that base + i is aligned to VEC * element size, so the
// load can be issued as packed accesses.
template <int VEC>
__device__ __forceinline__ void ld_any_vec(const void* base, int64_t i, int dt, bool vec_ok,
                                           float (&out)[VEC]) {
  if (vec_ok) {
    if (dt == BLOTH_F32) {
      if constexpr (VEC % 4 == 0) {
#pragma unroll
        for (int q = 0; q < VEC / 4; ++q) {
          float4 v = __ldg(reinterpret_cast<const float4*>(reinterpret_cast<const float*>(base) + i) + q);
          out[4 * q + 0] = v.x; out[4 * q + 1] = v.y; out[4 * q + 2] = v.z; out[4 * q + 3] = v.w;
        }
        return;
      }
    } else if (dt == BLOTH_BF16) {
      if constexpr (VEC == 8 || VEC == 4) {
        Pack<__nv_bfloat16, VEC> pk = ldg_pack<__nv_bfloat16, VEC>(reinterpret_cast<const __nv_bfloat16*>(base) + i);
        unpack(pk, out);
        return;
      }
    } else {
      if constexpr (VEC == 8 || VEC == 4) {
        Pack<__half, VEC> pk = ldg_pack<__half, VEC>(reinterpret_cast<const __half*>(base) + i);
        unpack(pk, out);
        return;
      }
    }
  }
#pragma unroll
  for (int e = 0; e < VEC; ++e) out[e] = ld_any(base, i + e, dt);
}

__device__ __forceinline__ void st_any(void* base, int64_t i, int dt, float v) {
  switch (dt) {
    case BLOTH_BF16: reinterpret_cast<__nv_bfloat16*>(base)[i] = __float2bfloat16_rn(v); break;
    case BLOTH_F16: reinterpret_cast<__half*>(base)[i] = __float2half_rn(v); break;
    default: reinterpret_cast<float*>(base)[i] = v; break;
  }
}

// ---------------------------------------------------------------------------
// packed fp32 pairs (sm_100: add/mul/fma.rn.f32x2 issue two IEEE fp32
// operations as one instruction; results equal the scalar ones bit for bit)
// ---------------------------------------------------------------------------
__device__ __forceinline__ float2 f2_fma(float2 a, float2 b, float2 c) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\tmov.b64 rc, {%6, %7};\n\t"
      "fma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return d;
}

__device__ __forceinline__ float2 f2_mul(float2 a, float2 b) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "mul.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}

__device__ __forceinline__ float2 f2_add(float2 a, float2 b) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "add.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}

__device__ __forceinline__ float2 f2(float a, float b) { return make_float2(a, b); }
__device__ __forceinline__ float2 f2s(float a) { return make_float2(a, a); }

// ---------------------------------------------------------------------------
// reductions
// ---------------------------------------------------------------------------
// Butterfly sum over aligned groups of WIDTH lanes (WIDTH a power of two
// <= 32). Every lane of a group ends with the bit-identical total, because
// each step adds the same two operands in both partner lanes.
template <int WIDTH>
__device__ __forceinline__ float group_lane_sum(float v) {
#pragma unroll
  for (int o = WIDTH / 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// ---------------------------------------------------------------------------
// launches
// ---------------------------------------------------------------------------
// Launches kern<<<grid, block, smem, st>>>(args...) and returns the launch's
// error (cleared, so that it does not surface at another launch).
template <typename... KArgs, typename... Args>
cudaError_t launch_ex(void (*kern)(KArgs...), unsigned grid, unsigned block, size_t smem,
                      cudaStream_t st, Args... args) {
  kern<<<grid, block, smem, st>>>(static_cast<KArgs>(args)...);
  return cudaGetLastError();
}

// launch_ex as a programmatic dependent of the kernel before it in the
// stream (see allow_dependent_launch): the launch and the CTAs' start overlap
// that kernel's tail, and kern waits in wait_for_prior_grid().
template <typename... KArgs, typename... Args>
cudaError_t launch_dependent(void (*kern)(KArgs...), unsigned grid, unsigned block, size_t smem,
                             cudaStream_t st, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(block);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
  if (e != cudaSuccess) cudaGetLastError();  // not left for the next launch check
  return e;
}

// ---------------------------------------------------------------------------
// host-side helpers (defined in launch.cu)
// ---------------------------------------------------------------------------
int device_sm_count();  // SM count of the current device (cached per device)
// Resident CTAs per SM for `func` at `block` threads and `smem` dynamic bytes
// (cached per device and function).
int occupancy(const void* func, int block, size_t smem);
// Raises `func`'s dynamic shared-memory limit to `smem` bytes on the current
// device (once per device and function).
int prepare_smem(const void* func, size_t smem);
// Device address of the library's fault word on the current device.
unsigned int* fault_word();
// Records `err` as the calling thread's last CUDA error and maps it to a status.
int cuda_status(cudaError_t err);
// cuda_status of a kernel launch's cudaGetLastError(), counting the launch
// when it succeeded (bloth_kernel_launch_count).
int launched(cudaError_t err);
// Kernels launched by this library in this process so far.
long long launch_count();
// Launches the bounded-wait expiry check (bloth_selftest_wait_expiry).
int selftest_wait_expiry(int limit_ms, cudaStream_t st);


}  // namespace bloth
