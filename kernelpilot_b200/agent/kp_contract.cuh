// Contract header for candidate kernels evaluated by kernelpilot_b200.agent.worker.
//
// Replaces kernelpilot's csrc/compat.h (:1-87) for candidates: CUDA only, built for
// sm_100a (B200) alone, so there is no HIP mapping and no runtime warp-size branching:
// a warp is 32 threads. The names a candidate uses stay those of compat.h
// (KP_SHFL_DOWN / KP_SHFL_XOR, KP_CHECK_LAUNCH, kp::kMaxWarps, kp::ceil_div,
// kp::to_float / kp::from_float, kp::warp_sum / kp::warp_max, kp::block_reduce), with
// bfloat16 added next to float and half. Inline PTX for sm_100a (tcgen05, TMA bulk
// copies, mbarriers) compiles as well, since nothing else is targeted.
//
// The header stands alone (no torch headers), so it can be compiled and checked
// without PyTorch.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>
#include <stdexcept>
#include <string>

#define KP_SHFL_DOWN(v, d) __shfl_down_sync(0xffffffffu, (v), (d))
#define KP_SHFL_XOR(v, d) __shfl_xor_sync(0xffffffffu, (v), (d))

// Throws std::runtime_error (a Python RuntimeError through the extension) when the
// last launch failed.
#define KP_CHECK_LAUNCH()                                                          \
  do {                                                                             \
    cudaError_t err_ = cudaGetLastError();                                         \
    if (err_ != cudaSuccess) {                                                     \
      throw std::runtime_error(std::string("kernel launch failed: ") +             \
                               cudaGetErrorString(err_) + " at " + __FILE__ + ":" + \
                               std::to_string(__LINE__));                          \
    }                                                                              \
  } while (0)

namespace kp {

constexpr int kWarp = 32;                    // threads per warp on sm_100a
constexpr int kMaxWarps = 1024 / kWarp;      // warps in the largest CTA
constexpr int kSms = 148;                    // streaming multiprocessors of a B200

inline int ceil_div(int64_t a, int64_t b) { return static_cast<int>((a + b - 1) / b); }

__device__ __forceinline__ float to_float(float x) { return x; }
__device__ __forceinline__ float to_float(__half x) { return __half2float(x); }
__device__ __forceinline__ float to_float(__nv_bfloat16 x) { return __bfloat162float(x); }

template <typename T>
__device__ __forceinline__ T from_float(float x);
template <>
__device__ __forceinline__ float from_float<float>(float x) { return x; }
template <>
__device__ __forceinline__ __half from_float<__half>(float x) { return __float2half_rn(x); }
template <>
__device__ __forceinline__ __nv_bfloat16 from_float<__nv_bfloat16>(float x) {
  return __float2bfloat16_rn(x);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int off = kWarp / 2; off > 0; off >>= 1) v += KP_SHFL_XOR(v, off);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int off = kWarp / 2; off > 0; off >>= 1) v = fmaxf(v, KP_SHFL_XOR(v, off));
  return v;
}

// CTA-wide sum or max; every thread gets the result. `scratch` holds kMaxWarps floats.
template <bool IsMax>
__device__ __forceinline__ float block_reduce(float v, float* scratch) {
  const int lane = threadIdx.x % kWarp;
  const int wid = threadIdx.x / kWarp;
  const int nwarps = (blockDim.x + kWarp - 1) / kWarp;
  v = IsMax ? warp_max(v) : warp_sum(v);
  __syncthreads();  // scratch may still be read by a previous call
  if (lane == 0) scratch[wid] = v;
  __syncthreads();
  v = threadIdx.x < nwarps ? scratch[threadIdx.x] : (IsMax ? -INFINITY : 0.f);
  if (wid == 0) {
    v = IsMax ? warp_max(v) : warp_sum(v);
    if (lane == 0) scratch[0] = v;
  }
  __syncthreads();
  return scratch[0];
}

}  // namespace kp
