// CUDA-core GEMM kernels for kp.matmul: variants 0-2 for every dtype, and the fp32
// path of variant 3 (the fp32 contract forbids TF32, kernelpilot/specs.py:196, and
// its tolerance, specs.py:188-189, is below what a single TF32 pass reaches, so fp32
// stays on exact FFMA). All accumulate in fp32 and handle any M, N, K.
//
// Replaces the SIMT stages of kernelpilot's csrc/kernels/matmul.hip (:16-208):
//   0 naive       one thread per C element
//   1 smem_tiled  32x32 shared-memory tiles, one element per thread
//   2 reg_tiled   64x64 CTA tile, BK=16, 4x4 outputs per thread
#include "kp_common.cuh"

namespace kpb {

template <typename T>
__global__ void mm_naive(const T* __restrict__ A, const T* __restrict__ B, T* __restrict__ C,
                         int64_t M, int64_t N, int64_t K) {
  const int64_t c = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t r = static_cast<int64_t>(blockIdx.y) * blockDim.y + threadIdx.y;
  if (r >= M || c >= N) return;
  float acc = 0.f;
  for (int64_t k = 0; k < K; ++k) acc = fmaf(to_f(A[r * K + k]), to_f(B[k * N + c]), acc);
  C[r * N + c] = from_f<T>(acc);
}

constexpr int kT1 = 32;

template <typename T>
__global__ void __launch_bounds__(kT1 * kT1) mm_smem(const T* __restrict__ A,
                                                     const T* __restrict__ B,
                                                     T* __restrict__ C, int64_t M, int64_t N,
                                                     int64_t K) {
  __shared__ float sa[kT1][kT1 + 1], sb[kT1][kT1 + 1];
  const int tx = threadIdx.x, ty = threadIdx.y;
  const int64_t r = static_cast<int64_t>(blockIdx.y) * kT1 + ty;
  const int64_t c = static_cast<int64_t>(blockIdx.x) * kT1 + tx;
  float acc = 0.f;
  for (int64_t k0 = 0; k0 < K; k0 += kT1) {
    sa[ty][tx] = (r < M && k0 + tx < K) ? to_f(A[r * K + k0 + tx]) : 0.f;
    sb[ty][tx] = (k0 + ty < K && c < N) ? to_f(B[(k0 + ty) * N + c]) : 0.f;
    __syncthreads();
#pragma unroll
    for (int k = 0; k < kT1; ++k) acc = fmaf(sa[ty][k], sb[k][tx], acc);
    __syncthreads();
  }
  if (r < M && c < N) C[r * N + c] = from_f<T>(acc);
}

constexpr int kBM2 = 64, kBN2 = 64, kBK2 = 16;

// 256 threads as a 16x16 grid; thread (ty, tx) owns rows ty + 16*i and columns
// tx + 16*j (i, j < 4), so both shared-memory reads are conflict-free broadcasts.
template <typename T>
__global__ void __launch_bounds__(256) mm_regtile(const T* __restrict__ A,
                                                  const T* __restrict__ B, T* __restrict__ C,
                                                  int64_t M, int64_t N, int64_t K) {
  __shared__ float sa[kBK2][kBM2 + 4];  // A tile stored k-major
  __shared__ float sb[kBK2][kBN2 + 4];
  const int tid = threadIdx.x, tx = tid % 16, ty = tid / 16;
  const int64_t m0 = static_cast<int64_t>(blockIdx.y) * kBM2;
  const int64_t n0 = static_cast<int64_t>(blockIdx.x) * kBN2;
  float acc[4][4] = {};
  for (int64_t k0 = 0; k0 < K; k0 += kBK2) {
    // A tile: 64 rows x 16 k = 1024 elements, 4 per thread
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int e = tid + i * 256, rr = e / kBK2, kk = e % kBK2;
      const int64_t gr = m0 + rr, gk = k0 + kk;
      sa[kk][rr] = (gr < M && gk < K) ? to_f(A[gr * K + gk]) : 0.f;
    }
    // B tile: 16 k x 64 cols
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int e = tid + i * 256, kk = e / kBN2, cc = e % kBN2;
      const int64_t gk = k0 + kk, gc = n0 + cc;
      sb[kk][cc] = (gk < K && gc < N) ? to_f(B[gk * N + gc]) : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < kBK2; ++kk) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = sa[kk][ty + 16 * i];
#pragma unroll
      for (int j = 0; j < 4; ++j) b[j] = sb[kk][tx + 16 * j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t r = m0 + ty + 16 * i;
    if (r >= M) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int64_t c = n0 + tx + 16 * j;
      if (c < N) C[r * N + c] = from_f<T>(acc[i][j]);
    }
  }
}

template <typename T>
int matmul_simt_t(int variant, const T* A, const T* B, T* C, int64_t M, int64_t N, int64_t K,
                  cudaStream_t s) {
  if (variant == 0) {
    const dim3 block(16, 16), grid(static_cast<unsigned>(cdiv(N, 16)), static_cast<unsigned>(cdiv(M, 16)));
    if (grid.y > 65535) return fail(KPB_EUNSUPPORTED, "matmul variant 0: M too large");
    mm_naive<T><<<grid, block, 0, s>>>(A, B, C, M, N, K);
  } else if (variant == 1) {
    const dim3 block(kT1, kT1), grid(static_cast<unsigned>(cdiv(N, kT1)), static_cast<unsigned>(cdiv(M, kT1)));
    if (grid.y > 65535) return fail(KPB_EUNSUPPORTED, "matmul variant 1: M too large");
    mm_smem<T><<<grid, block, 0, s>>>(A, B, C, M, N, K);
  } else {
    const dim3 grid(static_cast<unsigned>(cdiv(N, kBN2)), static_cast<unsigned>(cdiv(M, kBM2)));
    if (grid.y > 65535) return fail(KPB_EUNSUPPORTED, "matmul SIMT: M too large");
    mm_regtile<T><<<grid, 256, 0, s>>>(A, B, C, M, N, K);
  }
  KPB_LAUNCHED("matmul SIMT");
  return KPB_OK;
}

int matmul_simt(int variant, int dtype, const void* A, const void* B, void* C, int64_t M,
                int64_t N, int64_t K, cudaStream_t s) {
  switch (dtype) {
    case KPB_F32:
      return matmul_simt_t(variant, static_cast<const float*>(A), static_cast<const float*>(B),
                           static_cast<float*>(C), M, N, K, s);
    case KPB_F16:
      return matmul_simt_t(variant, static_cast<const __half*>(A), static_cast<const __half*>(B),
                           static_cast<__half*>(C), M, N, K, s);
    case KPB_BF16:
      return matmul_simt_t(variant, static_cast<const __nv_bfloat16*>(A),
                           static_cast<const __nv_bfloat16*>(B),
                           static_cast<__nv_bfloat16*>(C), M, N, K, s);
    default: return fail(KPB_EINVAL, "matmul: unknown dtype");
  }
}

}  // namespace kpb
