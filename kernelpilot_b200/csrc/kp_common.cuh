// Shared device helpers for the sm_100a kernels: element conversions, fixed 32-lane
// warp reductions, 128-bit global accesses with cache hints, and the host-side
// status plumbing behind the C ABI.
//
// Replaces kernelpilot's csrc/compat.h (HIP<->CUDA aliases, runtime-warpSize
// reductions, to_float/from_float for fp32/fp16 only, compat.h:6-87) with a
// CUDA-only header: the warp size is the constant 32, bf16 is a first-class type and
// launch failures become status codes instead of exceptions.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <string>
#include <type_traits>

#include "kp_b200.h"

namespace kpb {

constexpr int kWarp = 32;
constexpr unsigned kFull = 0xffffffffu;

// ------------------------------------------------------------------ host status

void set_error(const std::string& msg);
int fail(int code, const std::string& msg);
int cuda_fail(cudaError_t err, const char* what, const char* file, int line);
// SM count of the current device (cached per device).
int sm_count();
// Per-device, per-kernel launch facts, queried once (capi.cu): the dynamic
// shared-memory opt-in, and the occupancy of a block size / shared-memory size /
// cluster size (cfg's grid is not part of the answer).
int ensure_dyn_smem(const void* func, int bytes);
int occupancy_blocks(const void* func, int threads, size_t smem, int* out);
int occupancy_clusters(const void* func, const cudaLaunchConfig_t& cfg, int cluster, int* out);

#define KPB_CUDA(call)                                                   \
  do {                                                                   \
    cudaError_t e_ = (call);                                             \
    if (e_ != cudaSuccess) return ::kpb::cuda_fail(e_, #call, __FILE__, __LINE__); \
  } while (0)

#define KPB_LAUNCHED(what)                                               \
  do {                                                                   \
    cudaError_t e_ = cudaGetLastError();                                 \
    if (e_ != cudaSuccess) return ::kpb::cuda_fail(e_, what, __FILE__, __LINE__); \
  } while (0)

inline int64_t cdiv(int64_t a, int64_t b) { return (a + b - 1) / b; }

// ------------------------------------------------------------------ element types

template <typename T> struct Elem;
template <> struct Elem<float> {
  __device__ __forceinline__ static float to_f(float x) { return x; }
  __device__ __forceinline__ static float from_f(float x) { return x; }
};
template <> struct Elem<__half> {
  __device__ __forceinline__ static float to_f(__half x) { return __half2float(x); }
  __device__ __forceinline__ static __half from_f(float x) { return __float2half_rn(x); }
};
template <> struct Elem<__nv_bfloat16> {
  __device__ __forceinline__ static float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }
  __device__ __forceinline__ static __nv_bfloat16 from_f(float x) { return __float2bfloat16_rn(x); }
};

template <typename T> __device__ __forceinline__ float to_f(T x) { return Elem<T>::to_f(x); }
template <typename T> __device__ __forceinline__ T from_f(float x) { return Elem<T>::from_f(x); }

// Elements of T in one 16-byte vector.
template <typename T> struct Vec { static constexpr int kN = 16 / sizeof(T); };

// Unpack a 16-byte vector into kN floats.
template <typename T>
__device__ __forceinline__ void unpack(const uint4& v, float* f) {
  if constexpr (sizeof(T) == 4) {
    f[0] = __uint_as_float(v.x); f[1] = __uint_as_float(v.y);
    f[2] = __uint_as_float(v.z); f[3] = __uint_as_float(v.w);
  } else {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      if constexpr (std::is_same<T, __half>::value) {
        const float2 p = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
        f[2 * i] = p.x; f[2 * i + 1] = p.y;
      } else {
        const float2 p = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[i]));
        f[2 * i] = p.x; f[2 * i + 1] = p.y;
      }
    }
  }
}

// Pack kN floats (round to nearest even) into a 16-byte vector.
template <typename T>
__device__ __forceinline__ uint4 pack(const float* f) {
  uint4 v;
  if constexpr (sizeof(T) == 4) {
    v.x = __float_as_uint(f[0]); v.y = __float_as_uint(f[1]);
    v.z = __float_as_uint(f[2]); v.w = __float_as_uint(f[3]);
  } else {
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      if constexpr (std::is_same<T, __half>::value) {
        const __half2 h = __floats2half2_rn(f[2 * i], f[2 * i + 1]);
        w[i] = *reinterpret_cast<const uint32_t*>(&h);
      } else {
        const __nv_bfloat162 h = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
        w[i] = *reinterpret_cast<const uint32_t*>(&h);
      }
    }
    v = make_uint4(w[0], w[1], w[2], w[3]);
  }
  return v;
}

// ------------------------------------------------------------------ global memory

// L2 eviction-priority policy for the cache_hint loads below.
__device__ __forceinline__ uint64_t evict_first_policy() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// 128-bit read-only streaming load: not kept in L1, first to leave L2 (`pol` from
// evict_first_policy()).
__device__ __forceinline__ uint4 ld_stream(const void* p, uint64_t pol) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.v4.u32 {%0,%1,%2,%3}, [%4], %5;"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p), "l"(pol));
  return v;
}

// 128-bit read-only load that keeps normal L2 priority (data read twice).
__device__ __forceinline__ uint4 ld_keep(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}

// 128-bit streaming store (written once, not re-read by this kernel).
__device__ __forceinline__ void st_stream(void* p, const uint4& v) {
  asm volatile("st.global.cs.v4.u32 [%0], {%1,%2,%3,%4};"
               :: "l"(p), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w) : "memory");
}

// ------------------------------------------------------------------ arithmetic

// 2^x on the multi-function unit (ex2.approx.ftz: relative error about 2^-22; results
// below 2^-126 flush to zero).
__device__ __forceinline__ float ex2f(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// max(a, b, c) in one instruction (sm_100).
__device__ __forceinline__ float max3f(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// ------------------------------------------------------------------ warp / block reductions

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = kWarp / 2; o > 0; o >>= 1) v += __shfl_xor_sync(kFull, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = kWarp / 2; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(kFull, v, o));
  return v;
}

// Block-wide sum/max; every thread returns the result. `scratch` holds 32 floats
// and must not be reused by the caller until the next __syncthreads after return.
template <bool kMax>
__device__ __forceinline__ float block_reduce(float v, float* scratch) {
  const int lane = threadIdx.x & (kWarp - 1), wid = threadIdx.x / kWarp;
  const int nwarps = (blockDim.x + kWarp - 1) / kWarp;
  v = kMax ? warp_max(v) : warp_sum(v);
  if (lane == 0) scratch[wid] = v;
  __syncthreads();
  const float init = kMax ? -INFINITY : 0.f;
  float w = lane < nwarps ? scratch[lane] : init;
  return kMax ? warp_max(w) : warp_sum(w);
}

}  // namespace kpb
