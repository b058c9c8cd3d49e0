// Elementwise c = a + b over n elements (kp.vector_add), fp32 arithmetic, result
// rounded to the input dtype.
//
// Replaces kernelpilot's csrc/kernels/vector_add.hip (stages naive / gridstride /
// vectorized). The operation moves 3 * n * sizeof(T) bytes and does n adds, so the
// only bound is HBM:
//
//   variant 0  one element per thread (baseline)
//   variant 1  grid-stride loop, one element per thread per step
//   variant 2  a CTA of 256 threads per tile of 512 16-byte vectors of each array
//              (two per thread, both loads of a and b issued before any add):
//              128-bit read-only evict-first loads, 128-bit stores. The grid is not
//              persistent: on B200 one short-lived CTA per tile keeps more bytes in
//              flight than a grid-stride loop (7.1 vs 6.6 TB/s measured for fp32 2^26).
//              When a, b and c share the same offset from a 16-byte boundary, the
//              elements before the first boundary and after the last whole vector are
//              done one by one by CTA 0; otherwise the grid-stride kernel does every
//              element (the 2-byte-aligned case has no common vector grid).
#include <algorithm>

#include "kp_common.cuh"

namespace kpb {
namespace {

constexpr int kTileThreads = 256;
constexpr int kTileVectors = 2;  // per thread and array
constexpr int kTile = kTileThreads * kTileVectors;

template <typename T>
__device__ __forceinline__ T add1(T a, T b) {
  return from_f<T>(to_f(a) + to_f(b));
}

template <typename T>
__global__ void vadd_naive(const T* __restrict__ a, const T* __restrict__ b, T* __restrict__ c,
                           int64_t n) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i < n) c[i] = add1(a[i], b[i]);
}

template <typename T>
__global__ void vadd_gridstride(const T* __restrict__ a, const T* __restrict__ b,
                                T* __restrict__ c, int64_t n) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride)
    c[i] = add1(a[i], b[i]);
}

// a, b, c are 16-byte aligned after `head` elements; the vector body covers
// [head, head + nvec * VN), CTA b owns vectors [b * kTile, (b + 1) * kTile); the head
// and the tail (< VN elements each) go to CTA 0.
template <typename T>
__global__ void __launch_bounds__(kTileThreads)
vadd_tile(const T* __restrict__ a, const T* __restrict__ b, T* __restrict__ c, int64_t n,
          int head) {
  constexpr int VN = Vec<T>::kN;
  const int64_t nvec = (n - head) / VN;
  if (blockIdx.x == 0) {
    const int64_t tail0 = head + nvec * VN;
    const int i = threadIdx.x;
    if (i < head) c[i] = add1(a[i], b[i]);
    if (i < n - tail0) c[tail0 + i] = add1(a[tail0 + i], b[tail0 + i]);
  }
  const uint4* av = reinterpret_cast<const uint4*>(a + head);
  const uint4* bv = reinterpret_cast<const uint4*>(b + head);
  uint4* cv = reinterpret_cast<uint4*>(c + head);
  const uint64_t pol = evict_first_policy();
  const int64_t base = static_cast<int64_t>(blockIdx.x) * kTile + threadIdx.x;
  uint4 x[kTileVectors], y[kTileVectors];
#pragma unroll
  for (int u = 0; u < kTileVectors; ++u) {
    const int64_t i = base + u * kTileThreads;
    if (i < nvec) {
      x[u] = ld_stream(av + i, pol);
      y[u] = ld_stream(bv + i, pol);
    }
  }
#pragma unroll
  for (int u = 0; u < kTileVectors; ++u) {
    const int64_t i = base + u * kTileThreads;
    if (i >= nvec) continue;
    float f[VN], g[VN];
    unpack<T>(x[u], f);
    unpack<T>(y[u], g);
#pragma unroll
    for (int l = 0; l < VN; l += 2) {
      const float2 s = __fadd2_rn(make_float2(f[l], f[l + 1]), make_float2(g[l], g[l + 1]));
      f[l] = s.x;
      f[l + 1] = s.y;
    }
    cv[i] = pack<T>(f);
  }
}

template <typename T>
int launch(int variant, const T* a, const T* b, T* c, int64_t n, cudaStream_t s) {
  if (n == 0) return KPB_OK;
  const uintptr_t pa = reinterpret_cast<uintptr_t>(a), pb = reinterpret_cast<uintptr_t>(b),
                  pc = reinterpret_cast<uintptr_t>(c);
  if ((pa | pb | pc) % sizeof(T) != 0)
    return fail(KPB_EINVAL, "vector_add: a, b and c must be element-aligned");
  const int sms = sm_count();
  if (variant == 0) {
    vadd_naive<T><<<static_cast<unsigned>(cdiv(n, 256)), 256, 0, s>>>(a, b, c, n);
    KPB_LAUNCHED("vector_add variant 0");
    return KPB_OK;
  }
  const bool common_grid = (pa % 16 == pb % 16) && (pa % 16 == pc % 16);
  if (variant == 1 || !common_grid) {
    const int64_t blocks = std::min<int64_t>(cdiv(n, 256), int64_t(sms) * 8);
    vadd_gridstride<T><<<static_cast<unsigned>(blocks), 256, 0, s>>>(a, b, c, n);
    KPB_LAUNCHED("vector_add grid-stride");
    return KPB_OK;
  }
  constexpr int VN = Vec<T>::kN;
  const int head = static_cast<int>(std::min<int64_t>(n, ((16 - pa % 16) % 16) / sizeof(T)));
  const int64_t nvec = (n - head) / VN;
  const int64_t blocks = std::max<int64_t>(1, cdiv(nvec, kTile));
  vadd_tile<T><<<static_cast<unsigned>(blocks), kTileThreads, 0, s>>>(a, b, c, n, head);
  KPB_LAUNCHED("vector_add tiles");
  return KPB_OK;
}

}  // namespace

int vector_add(int variant, int dtype, const void* a, const void* b, void* c, int64_t n,
               cudaStream_t s) {
  switch (dtype) {
    case KPB_F32:
      return launch(variant, static_cast<const float*>(a), static_cast<const float*>(b),
                    static_cast<float*>(c), n, s);
    case KPB_F16:
      return launch(variant, static_cast<const __half*>(a), static_cast<const __half*>(b),
                    static_cast<__half*>(c), n, s);
    case KPB_BF16:
      return launch(variant, static_cast<const __nv_bfloat16*>(a),
                    static_cast<const __nv_bfloat16*>(b), static_cast<__nv_bfloat16*>(c), n, s);
    default: return fail(KPB_EINVAL, "vector_add: unknown dtype " + std::to_string(dtype));
  }
}

}  // namespace kpb
