// LayerNorm over the last dimension of a contiguous (M, N) matrix (kp.layernorm):
// y = (x - mean) / sqrt(var + eps) * w + b with the biased variance, fp32
// statistics, output in the input dtype.
//
// Replaces kernelpilot's csrc/kernels/layernorm.hip (stages naive / block_two_pass /
// welford_fused, :77-130). The statistics here are exact two-pass ones (the mean,
// then the mean of squared deviations) taken from values already in registers, so
// there is no need for a one-pass Welford/Chan merge:
//
//   variant 0  thread per row, three passes over global memory (baseline)
//   variant 1  CTA per row, three coalesced passes (sum, squared deviations,
//              normalise) with block reductions; also what variant 2 falls back to
//              for rows longer than it holds in registers (65536 16-bit / 32768 fp32
//              elements) and for rows, w, b or y off 16-byte boundaries
//   variant 2  rows in registers: a row is split over 1..32 warps (several rows per
//              CTA when it needs fewer than 8), each thread holding up to 8 16-byte
//              vectors of it, read with one streaming load each (L1 bypassed, L2
//              evict-first) so that HBM sees one read and one write per element and
//              L1 keeps w and b. Sum -> mean -> squared deviations -> 1/sqrt(var + eps)
//              -> affine, in packed float2 arithmetic; warp shuffles, and one shared-
//              memory exchange per statistic when a row spans several warps. The grid
//              is not persistent: a CTA per row group, so the hardware scheduler keeps
//              every SM full and the bytes in flight per SM high. Needs rows, w, b and
//              y on 16-byte boundaries (N * sizeof(T) a multiple of 16).
//
// Measured on B200 (HBM copy 6.55-6.8 TB/s): fp32 8192 x 8192 6.4 TB/s, bf16 8192 x
// 8192 5.0 TB/s, bf16 16384 x 8192 5.6 TB/s; torch.nn.functional.layer_norm 3.6 and
// 2.6 TB/s on the first two.
#include <algorithm>
#include <type_traits>

#include "kp_common.cuh"

namespace kpb {
namespace {

// ------------------------------------------------------------------ variant 0

template <typename T>
__global__ void ln_thread_row(const T* __restrict__ x, const T* __restrict__ w,
                              const T* __restrict__ b, T* __restrict__ y, int64_t M, int64_t N,
                              float eps) {
  const int64_t row = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (row >= M) return;
  const T* xr = x + row * N;
  T* yr = y + row * N;
  float s = 0.f;
  for (int64_t j = 0; j < N; ++j) s += to_f(xr[j]);
  const float mean = s / static_cast<float>(N);
  float q = 0.f;
  for (int64_t j = 0; j < N; ++j) {
    const float d = to_f(xr[j]) - mean;
    q = fmaf(d, d, q);
  }
  const float rstd = rsqrtf(q / static_cast<float>(N) + eps);
  for (int64_t j = 0; j < N; ++j)
    yr[j] = from_f<T>(fmaf((to_f(xr[j]) - mean) * rstd, to_f(w[j]), to_f(b[j])));
}

// ------------------------------------------------------------------ variant 1

template <typename T>
__global__ void __launch_bounds__(256)
ln_block_row(const T* __restrict__ x, const T* __restrict__ w, const T* __restrict__ b,
             T* __restrict__ y, int64_t N, float eps) {
  __shared__ float s_a[kWarp], s_b[kWarp];
  const T* xr = x + static_cast<int64_t>(blockIdx.x) * N;
  T* yr = y + static_cast<int64_t>(blockIdx.x) * N;
  float s = 0.f;
  for (int64_t j = threadIdx.x; j < N; j += blockDim.x) s += to_f(xr[j]);
  const float mean = block_reduce<false>(s, s_a) / static_cast<float>(N);
  float q = 0.f;
  for (int64_t j = threadIdx.x; j < N; j += blockDim.x) {
    const float d = to_f(xr[j]) - mean;
    q = fmaf(d, d, q);
  }
  const float rstd = rsqrtf(block_reduce<false>(q, s_b) / static_cast<float>(N) + eps);
  for (int64_t j = threadIdx.x; j < N; j += blockDim.x)
    yr[j] = from_f<T>(fmaf((to_f(xr[j]) - mean) * rstd, to_f(w[j]), to_f(b[j])));
}

// ------------------------------------------------------------------ variant 2: rows in registers

// unpack<T> again, in a form the compiler cannot merge with an earlier unpack of the
// same vector: without it, the floats of all V vectors stay live across the three
// passes (64 more registers at V = 8 for 16-bit types), which costs occupancy.
template <typename T>
__device__ __forceinline__ void unpack_again(const uint4& v, float* f) {
  if constexpr (sizeof(T) == 4) {
    unpack<T>(v, f);
  } else {
    const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      uint32_t lo, hi;
      if constexpr (std::is_same_v<T, __nv_bfloat16>) {
        asm volatile("{ shl.b32 %0, %2, 16; and.b32 %1, %2, 0xffff0000; }"
                     : "=r"(lo), "=r"(hi) : "r"(u[i]));
      } else {
        asm volatile("{ .reg .b16 l, h; mov.b32 {l, h}, %2; cvt.f32.f16 %0, l; cvt.f32.f16 %1, h; }"
                     : "=r"(lo), "=r"(hi) : "r"(u[i]));
      }
      f[2 * i] = __uint_as_float(lo);
      f[2 * i + 1] = __uint_as_float(hi);
    }
  }
}

// kThreads threads per CTA, `wpr` warps per row (a power of two dividing
// kThreads / 32), each thread holding V vectors; 32 * wpr * V >= N / VN. Rows, w, b
// and y all start on 16-byte boundaries (checked on the host).
template <typename T, int V, int kThreads>
__global__ void __launch_bounds__(kThreads)
ln_rows(const T* __restrict__ x, const T* __restrict__ w, const T* __restrict__ b,
        T* __restrict__ y, int64_t M, int N, float eps, int wpr) {
  constexpr int VN = Vec<T>::kN;
  __shared__ float red[2][kThreads / kWarp];
  const int warp = threadIdx.x / kWarp, lane = threadIdx.x & (kWarp - 1);
  const int tpr = wpr * kWarp;
  const int t = threadIdx.x % tpr;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * (kThreads / tpr) + threadIdx.x / tpr;
  const bool live = row < M;
  const int64_t r = live ? row : M - 1;  // a dead row group still joins the barriers
  const int nv = N / VN;

  const uint4* xr = reinterpret_cast<const uint4*>(x + r * N);
  const uint64_t pol = evict_first_policy();
  uint4 raw[V];
#pragma unroll
  for (int k = 0; k < V; ++k) {
    const int j = t + k * tpr;
    raw[k] = j < nv ? ld_stream(xr + j, pol) : make_uint4(0u, 0u, 0u, 0u);
  }
  // the zero padding adds nothing to the sum
  float2 s2 = make_float2(0.f, 0.f);
#pragma unroll
  for (int k = 0; k < V; ++k) {
    float f[VN];
    unpack<T>(raw[k], f);
#pragma unroll
    for (int l = 0; l < VN; l += 2) s2 = __fadd2_rn(s2, make_float2(f[l], f[l + 1]));
  }
  float s = warp_sum(s2.x + s2.y);
  if (wpr > 1) {
    if (lane == 0) red[0][warp] = s;
    __syncthreads();
    s = 0.f;
    for (int i = 0; i < wpr; ++i) s += red[0][warp - warp % wpr + i];
  }
  const float mean = s / static_cast<float>(N);
  const float2 nmean = make_float2(-mean, -mean);

  float2 q2 = make_float2(0.f, 0.f);
#pragma unroll
  for (int k = 0; k < V; ++k) {
    if (t + k * tpr >= nv) continue;
    float f[VN];
    unpack_again<T>(raw[k], f);
#pragma unroll
    for (int l = 0; l < VN; l += 2) {
      const float2 d = __fadd2_rn(make_float2(f[l], f[l + 1]), nmean);
      q2 = __ffma2_rn(d, d, q2);
    }
  }
  float q = warp_sum(q2.x + q2.y);
  if (wpr > 1) {
    if (lane == 0) red[1][warp] = q;
    __syncthreads();
    q = 0.f;
    for (int i = 0; i < wpr; ++i) q += red[1][warp - warp % wpr + i];
  }
  const float rstd = rsqrtf(q / static_cast<float>(N) + eps);
  const float2 rstd2 = make_float2(rstd, rstd);
  if (!live) return;

  uint4* yr = reinterpret_cast<uint4*>(y + r * N);
#pragma unroll
  for (int k = 0; k < V; ++k) {
    const int j = t + k * tpr;
    if (j >= nv) continue;
    float f[VN], wf[VN], bf[VN];
    unpack_again<T>(raw[k], f);
    unpack<T>(__ldg(reinterpret_cast<const uint4*>(w) + j), wf);
    unpack<T>(__ldg(reinterpret_cast<const uint4*>(b) + j), bf);
#pragma unroll
    for (int l = 0; l < VN; l += 2) {
      const float2 d = __fmul2_rn(__fadd2_rn(make_float2(f[l], f[l + 1]), nmean), rstd2);
      const float2 o = __ffma2_rn(d, make_float2(wf[l], wf[l + 1]), make_float2(bf[l], bf[l + 1]));
      f[l] = o.x;
      f[l + 1] = o.y;
    }
    st_stream(yr + j, pack<T>(f));
  }
}

// ------------------------------------------------------------------ launch

constexpr int kRowsMaxVectors = 8192;  // 32 warps x 32 lanes x 8 vectors

int next_pow2(int v) {
  int p = 1;
  while (p < v) p <<= 1;
  return p;
}

template <typename T, int V, int kThreads>
int launch_rows(const T* x, const T* w, const T* b, T* y, int64_t M, int64_t N, float eps,
                int wpr, cudaStream_t s) {
  const int rows_per_cta = kThreads / (kWarp * wpr);
  ln_rows<T, V, kThreads><<<static_cast<unsigned>(cdiv(M, rows_per_cta)), kThreads, 0, s>>>(
      x, w, b, y, M, static_cast<int>(N), eps, wpr);
  KPB_LAUNCHED("layernorm rows in registers");
  return KPB_OK;
}

// Row split measured on B200 (bf16 and fp32, N = 1024 .. 32768): 4 vectors per thread
// up to 512 vectors per row, 8 beyond; CTAs of 256 threads until a row needs more.
// Every branch covers the row: 32 lanes x wpr x V >= nv.
template <typename T>
int dispatch_rows(const T* x, const T* w, const T* b, T* y, int64_t M, int64_t N, float eps,
                  int nv, cudaStream_t s) {
  if (nv <= 32) return launch_rows<T, 1, 256>(x, w, b, y, M, N, eps, 1, s);
  if (nv <= 64) return launch_rows<T, 2, 256>(x, w, b, y, M, N, eps, 1, s);
  if (nv <= 512) return launch_rows<T, 4, 256>(x, w, b, y, M, N, eps, next_pow2(cdiv(nv, 128)), s);
  if (nv <= 2048) return launch_rows<T, 8, 256>(x, w, b, y, M, N, eps, next_pow2(cdiv(nv, 256)), s);
  if (nv <= 4096) return launch_rows<T, 8, 512>(x, w, b, y, M, N, eps, 16, s);
  // (16-bit types spill ~150 bytes a thread here at the 64-register cap; still one
  // HBM pass, unlike the three of the block-per-row kernel)
  return launch_rows<T, 8, 1024>(x, w, b, y, M, N, eps, 32, s);
}

template <typename T>
int launch(int variant, const T* x, const T* w, const T* b, T* y, int64_t M, int64_t N,
           float eps, cudaStream_t s) {
  if (M == 0 || N == 0) return KPB_OK;
  const uintptr_t ptrs[4] = {reinterpret_cast<uintptr_t>(x), reinterpret_cast<uintptr_t>(w),
                             reinterpret_cast<uintptr_t>(b), reinterpret_cast<uintptr_t>(y)};
  for (uintptr_t p : ptrs)
    if (p % sizeof(T) != 0) return fail(KPB_EINVAL, "layernorm: tensors must be element-aligned");
  if (variant == 0) {
    ln_thread_row<T><<<static_cast<unsigned>(cdiv(M, 128)), 128, 0, s>>>(x, w, b, y, M, N, eps);
    KPB_LAUNCHED("layernorm variant 0");
    return KPB_OK;
  }
  constexpr int VN = Vec<T>::kN;
  // every row, w and b on 16-byte boundaries, or the masked path
  const bool aligned = (ptrs[0] | ptrs[1] | ptrs[2] | ptrs[3]) % 16 == 0 &&
                       (N * static_cast<int64_t>(sizeof(T))) % 16 == 0;
  if (variant == 2 && aligned && N / VN <= kRowsMaxVectors)
    return dispatch_rows<T>(x, w, b, y, M, N, eps, static_cast<int>(N / VN), s);
  // Misaligned rows: the block kernel's scalar loads are coalesced at any alignment
  // and measured at least as fast on B200 as register-resident variants that either
  // load scalars (too few bytes in flight) or shift vectors per row (2-3.5 TB/s).
  ln_block_row<T><<<static_cast<unsigned>(M), 256, 0, s>>>(x, w, b, y, N, eps);
  KPB_LAUNCHED("layernorm block per row");
  return KPB_OK;
}

}  // namespace

int layernorm(int variant, int dtype, const void* x, const void* w, const void* b, void* y,
              int64_t M, int64_t N, float eps, cudaStream_t s) {
  switch (dtype) {
    case KPB_F32:
      return launch(variant, static_cast<const float*>(x), static_cast<const float*>(w),
                    static_cast<const float*>(b), static_cast<float*>(y), M, N, eps, s);
    case KPB_F16:
      return launch(variant, static_cast<const __half*>(x), static_cast<const __half*>(w),
                    static_cast<const __half*>(b), static_cast<__half*>(y), M, N, eps, s);
    case KPB_BF16:
      return launch(variant, static_cast<const __nv_bfloat16*>(x),
                    static_cast<const __nv_bfloat16*>(w), static_cast<const __nv_bfloat16*>(b),
                    static_cast<__nv_bfloat16*>(y), M, N, eps, s);
    default: return fail(KPB_EINVAL, "layernorm: unknown dtype " + std::to_string(dtype));
  }
}

}  // namespace kpb
