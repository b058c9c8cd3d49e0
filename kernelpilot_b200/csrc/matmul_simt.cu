// CUDA-core GEMM kernels for kp.matmul: variants 0-2 for every dtype, and the fp32
// path of variant 3 (the fp32 contract forbids TF32, kernelpilot/specs.py:196, and
// its tolerance, specs.py:188-189, is below what a single TF32 pass reaches, so fp32
// stays on exact FFMA). All accumulate in fp32 and handle any M, N, K.
//
// Replaces the SIMT stages of kernelpilot's csrc/kernels/matmul.hip (:16-208):
//   0 naive       one thread per C element
//   1 smem_tiled  32x32 shared-memory tiles, one element per thread
//   2 reg_tiled   128x128 CTA tile, 8 k per step, 8x8 outputs per thread read from
//                 shared memory as 16-byte vectors, the next step's tile prefetched
//                 into registers while the current one is multiplied
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

// ---- variant 2: 128 x 128 tiles, 8 x 8 outputs per thread
//
// 256 threads as a 16 x 16 grid. Thread (ty, tx) owns the rows {4ty..4ty+3} and
// {64+4ty..64+4ty+3} and the same two column groups in tx: four 4x4 blocks, 64
// accumulators. Shared memory holds the A tile transposed (k-major, [8][128]) and
// the B tile as is ([8][128]), both as fp32, so each k step reads two float4 of A
// and two float4 of B per thread: the 16 threads of a half-warp that share ty read
// the same A vectors (a broadcast) and 16 consecutive B vectors. Two shared-memory
// buffers alternate; the global loads of step s+1 are issued into registers before
// step s is multiplied, so one barrier per step suffices.
constexpr int kRT = 128, kRK = 8;

template <typename T>
struct TileLoader {
  // A tile: 128 rows x 8 k; thread t takes row t / 2 and k (t % 2) * 4 .. + 3.
  // B tile: 8 k x 128 columns; thread t takes k t / 32 and columns (t % 32) * 4 .. + 3.
  float a[4], b[4];

  __device__ __forceinline__ void load(const T* __restrict__ A, const T* __restrict__ B,
                                       int64_t M, int64_t N, int64_t K, int64_t m0, int64_t n0,
                                       int64_t k0, int tid) {
    const int64_t ar = m0 + tid / 2, ak = k0 + (tid % 2) * 4;
    const int64_t bk = k0 + tid / 32, bc = n0 + (tid % 32) * 4;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      a[i] = (ar < M && ak + i < K) ? to_f(A[ar * K + ak + i]) : 0.f;
      b[i] = (bk < K && bc + i < N) ? to_f(B[bk * N + bc + i]) : 0.f;
    }
  }

  __device__ __forceinline__ void store(float (*sa)[kRT], float (*sb)[kRT], int tid) const {
    const int ar = tid / 2, ak = (tid % 2) * 4;
#pragma unroll
    for (int i = 0; i < 4; ++i) sa[ak + i][ar] = a[i];
    *reinterpret_cast<float4*>(&sb[tid / 32][(tid % 32) * 4]) = make_float4(b[0], b[1], b[2], b[3]);
  }
};

template <typename T>
__global__ void __launch_bounds__(256) mm_regtile(const T* __restrict__ A,
                                                  const T* __restrict__ B, T* __restrict__ C,
                                                  int64_t M, int64_t N, int64_t K) {
  __shared__ __align__(16) float sa[2][kRK][kRT];
  __shared__ __align__(16) float sb[2][kRK][kRT];
  const int tid = threadIdx.x, tx = tid % 16, ty = tid / 16;
  const int64_t m0 = static_cast<int64_t>(blockIdx.y) * kRT;
  const int64_t n0 = static_cast<int64_t>(blockIdx.x) * kRT;
  float acc[8][8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;

  TileLoader<T> ld;
  ld.load(A, B, M, N, K, m0, n0, 0, tid);
  ld.store(sa[0], sb[0], tid);
  __syncthreads();
  const int64_t steps = (K + kRK - 1) / kRK;
  for (int64_t st = 0; st < steps; ++st) {
    const int cur = static_cast<int>(st & 1);
    if (st + 1 < steps) ld.load(A, B, M, N, K, m0, n0, (st + 1) * kRK, tid);
#pragma unroll
    for (int k = 0; k < kRK; ++k) {
      const float4 a0 = *reinterpret_cast<const float4*>(&sa[cur][k][4 * ty]);
      const float4 a1 = *reinterpret_cast<const float4*>(&sa[cur][k][64 + 4 * ty]);
      const float4 b0 = *reinterpret_cast<const float4*>(&sb[cur][k][4 * tx]);
      const float4 b1 = *reinterpret_cast<const float4*>(&sb[cur][k][64 + 4 * tx]);
      const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
      const float bv[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
    }
    if (st + 1 < steps) ld.store(sa[cur ^ 1], sb[cur ^ 1], tid);
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int64_t r = m0 + (i < 4 ? 4 * ty + i : 64 + 4 * ty + i - 4);
    if (r >= M) continue;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int64_t c = n0 + (j < 4 ? 4 * tx + j : 64 + 4 * tx + j - 4);
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
    const dim3 grid(static_cast<unsigned>(cdiv(N, kRT)), static_cast<unsigned>(cdiv(M, kRT)));
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
