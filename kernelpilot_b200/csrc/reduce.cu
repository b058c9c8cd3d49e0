// Full sum of a 1-D tensor into one fp32 value (kp.reduce_sum).
//
// Replaces kernelpilot's csrc/kernels/reduction.hip (stages :15-87, dispatch
// :96-123). That code ends every CTA with a float atomicAdd into a zeroed output,
// so its result depends on CTA timing. Here every variant is a two-level tree with
// a fixed combination order, so the result is bit-reproducible:
//   level 1  each CTA reduces its share and writes one fp32 partial;
//   level 2  one CTA adds the partials in a fixed order and writes out[0]
//            (launched with programmatic dependent launch, so its launch latency
//            overlaps level 1).
// Variants:
//   0 chunked    one CTA per 1024 elements, scalar loads (the simple baseline)
//   1 gridstride grid-stride scalar loads over at most 1024 CTAs
//   2 persistent one wave of CTAs (3 per SM), 128-bit streaming loads, 4 in flight
//                per thread; the HBM-bound B200 kernel
#include "kp_common.cuh"
#include "kp_sm100.cuh"

namespace kpb {
namespace {

constexpr int kChunkThreads = 256;   // variant 0
constexpr int kChunkPerThread = 4;
constexpr int kStrideThreads = 256;  // variant 1
constexpr int kStrideMaxCtas = 1024;
constexpr int kVecThreads = 512;     // variant 2
constexpr int kVecCtasPerSm = 3;
constexpr int kVecUnroll = 4;
constexpr int kFinishThreads = 1024;

template <typename T>
__global__ void __launch_bounds__(kChunkThreads) sum_chunked(const T* __restrict__ x,
                                                             float* __restrict__ partials,
                                                             int64_t n) {
  __shared__ float scratch[kWarp];
  const int64_t base = static_cast<int64_t>(blockIdx.x) * kChunkThreads * kChunkPerThread;
  float acc = 0.f;
#pragma unroll
  for (int k = 0; k < kChunkPerThread; ++k) {
    const int64_t i = base + k * kChunkThreads + threadIdx.x;
    if (i < n) acc += to_f(x[i]);
  }
  acc = block_reduce<false>(acc, scratch);
  if (threadIdx.x == 0) partials[blockIdx.x] = acc;
  pdl_launch_dependents();
}

template <typename T>
__global__ void __launch_bounds__(kStrideThreads) sum_gridstride(const T* __restrict__ x,
                                                                 float* __restrict__ partials,
                                                                 int64_t n) {
  __shared__ float scratch[kWarp];
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  float a0 = 0.f, a1 = 0.f;
  int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  for (; i + stride < n; i += 2 * stride) {
    a0 += to_f(x[i]);
    a1 += to_f(x[i + stride]);
  }
  if (i < n) a0 += to_f(x[i]);
  const float acc = block_reduce<false>(a0 + a1, scratch);
  if (threadIdx.x == 0) partials[blockIdx.x] = acc;
  pdl_launch_dependents();
}

template <typename T>
__device__ __forceinline__ float vsum(const uint4& v) {
  float f[Vec<T>::kN];
  unpack<T>(v, f);
  float s0 = 0.f, s1 = 0.f;
#pragma unroll
  for (int i = 0; i < Vec<T>::kN; i += 2) {
    s0 += f[i];
    s1 += f[i + 1];
  }
  return s0 + s1;
}

// The input is split into an unaligned head (< 16 bytes), nvec 16-byte vectors
// and a scalar tail. The vectors are cut into chunks of kVecThreads*kVecUnroll
// vectors; CTA b takes chunks b, b+grid, ... so each CTA streams contiguous 32 KB
// (fp32) pieces and every thread keeps kVecUnroll independent loads in flight.
template <typename T>
__global__ void __launch_bounds__(kVecThreads, kVecCtasPerSm)
sum_persistent(const T* __restrict__ x, float* __restrict__ partials, int64_t n, int head) {
  __shared__ float scratch[kWarp];
  constexpr int VN = Vec<T>::kN;
  constexpr int64_t kChunk = static_cast<int64_t>(kVecThreads) * kVecUnroll;
  pdl_launch_dependents();
  const uint64_t pol = evict_first_policy();
  const int64_t nvec = (n - head) / VN;
  const uint4* xv = reinterpret_cast<const uint4*>(x + head);
  const int64_t nchunk = nvec / kChunk;
  float acc[kVecUnroll];
#pragma unroll
  for (int k = 0; k < kVecUnroll; ++k) acc[k] = 0.f;

  for (int64_t c = blockIdx.x; c < nchunk; c += gridDim.x) {
    const uint4* p = xv + c * kChunk + threadIdx.x;
    uint4 v[kVecUnroll];
#pragma unroll
    for (int k = 0; k < kVecUnroll; ++k) v[k] = ld_stream(p + k * kVecThreads, pol);
#pragma unroll
    for (int k = 0; k < kVecUnroll; ++k) acc[k] += vsum<T>(v[k]);
  }
  // leftover vectors after the last whole chunk
  const int64_t stride = static_cast<int64_t>(gridDim.x) * kVecThreads;
  for (int64_t i = nchunk * kChunk + static_cast<int64_t>(blockIdx.x) * kVecThreads + threadIdx.x;
       i < nvec; i += stride)
    acc[0] += vsum<T>(ld_stream(xv + i, pol));
  // unaligned head and scalar tail, by the last CTA
  if (blockIdx.x == gridDim.x - 1) {
    if (threadIdx.x < head) acc[1 % kVecUnroll] += to_f(x[threadIdx.x]);
    for (int64_t j = head + nvec * VN + threadIdx.x; j < n; j += kVecThreads)
      acc[2 % kVecUnroll] += to_f(x[j]);
  }
  float s = 0.f;
#pragma unroll
  for (int k = 0; k < kVecUnroll; ++k) s += acc[k];
  s = block_reduce<false>(s, scratch);
  if (threadIdx.x == 0) partials[blockIdx.x] = s;
}

// Level 2: out[0] = partials[0] + ... + partials[count-1] in a fixed order.
__global__ void __launch_bounds__(kFinishThreads) sum_finish(const float* __restrict__ partials,
                                                             int64_t count,
                                                             float* __restrict__ out) {
  __shared__ float scratch[kWarp];
  pdl_wait_primary();
  float s = 0.f;
  for (int64_t i = threadIdx.x; i < count; i += kFinishThreads) s += partials[i];
  s = block_reduce<false>(s, scratch);
  if (threadIdx.x == 0) out[0] = s;
}

__global__ void write_zero(float* out) { out[0] = 0.f; }

// Level-1 CTA count of a variant for n elements.
int64_t level1_ctas(int variant, int64_t n, int sms) {
  if (variant == 0) return cdiv(n, kChunkThreads * kChunkPerThread);
  if (variant == 1) return std::min<int64_t>(kStrideMaxCtas, std::max<int64_t>(1, cdiv(n, kStrideThreads)));
  const int64_t want = cdiv(n, int64_t(kVecThreads) * 16);  // >= 16 vectors of work per thread
  return std::max<int64_t>(1, std::min<int64_t>(int64_t(sms) * kVecCtasPerSm, want));
}

// Level 1 of `variant`: one partial per CTA into partials[0 .. *ctas).
template <typename T>
int launch_level1(int variant, const T* x, int64_t n, float* partials, int64_t* ctas_out,
                  cudaStream_t s) {
  const int64_t ctas = level1_ctas(variant, n, sm_count());
  *ctas_out = ctas;
  if (variant == 0) {
    sum_chunked<T><<<static_cast<unsigned>(ctas), kChunkThreads, 0, s>>>(x, partials, n);
  } else if (variant == 1) {
    sum_gridstride<T><<<static_cast<unsigned>(ctas), kStrideThreads, 0, s>>>(x, partials, n);
  } else {
    const uintptr_t addr = reinterpret_cast<uintptr_t>(x);
    if (addr % sizeof(T) != 0) return fail(KPB_EINVAL, "reduce_sum: x is not element-aligned");
    int64_t head = static_cast<int64_t>(((16 - (addr & 15)) & 15) / sizeof(T));
    if (head > n) head = n;
    sum_persistent<T><<<static_cast<unsigned>(ctas), kVecThreads, 0, s>>>(
        x, partials, n, static_cast<int>(head));
  }
  KPB_LAUNCHED("reduce_sum level 1");
  return KPB_OK;
}

template <typename T>
int launch(int variant, const T* x, float* out, int64_t n, float* partials, cudaStream_t s) {
  int64_t ctas = 0;
  if (int rc = launch_level1(variant, x, n, partials, &ctas, s)) return rc;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(1);
  cfg.blockDim = dim3(kFinishThreads);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  KPB_CUDA(cudaLaunchKernelEx(&cfg, sum_finish, static_cast<const float*>(partials), ctas, out));
  return KPB_OK;
}

}  // namespace

// Partials a call of `variant` on n elements writes on the current device.
int64_t reduce_partials_needed(int variant, int64_t n) {
  return n <= 0 ? 0 : level1_ctas(variant, n, sm_count());
}

size_t reduce_workspace_bytes(int variant, int64_t n) {
  if (n <= 0) return 0;
  // variant 2's CTA count depends on the SM count; size for the largest B200-class part
  const int64_t ctas = variant == 2 ? int64_t(kVecCtasPerSm) * 256 : level1_ctas(variant, n, 256);
  return static_cast<size_t>(ctas) * sizeof(float);
}

// Level 1 of the persistent variant alone (n > 0): the partials for a caller that
// finishes the sum itself. partials must hold reduce_partials_needed(2, n) floats.
int reduce_level1_persistent(int dtype, const void* x, int64_t n, float* partials,
                             int64_t* ctas, cudaStream_t s) {
  switch (dtype) {
    case KPB_F32: return launch_level1(2, static_cast<const float*>(x), n, partials, ctas, s);
    case KPB_F16: return launch_level1(2, static_cast<const __half*>(x), n, partials, ctas, s);
    case KPB_BF16:
      return launch_level1(2, static_cast<const __nv_bfloat16*>(x), n, partials, ctas, s);
    default: return fail(KPB_EINVAL, "reduce_sum: unknown dtype " + std::to_string(dtype));
  }
}

int reduce_sum(int variant, int dtype, const void* x, float* out, int64_t n, void* ws,
               size_t ws_bytes, cudaStream_t s) {
  if (n == 0) {
    write_zero<<<1, 1, 0, s>>>(out);
    KPB_LAUNCHED("reduce_sum zero");
    return KPB_OK;
  }
  const int64_t ctas = level1_ctas(variant, n, sm_count());
  if (ws == nullptr || ws_bytes < static_cast<size_t>(ctas) * sizeof(float))
    return fail(KPB_EINVAL, "reduce_sum: workspace too small (" + std::to_string(ws_bytes) +
                                " bytes, need " + std::to_string(ctas * 4) + ")");
  if (reinterpret_cast<uintptr_t>(ws) % 4 != 0)
    return fail(KPB_EINVAL, "reduce_sum: workspace must be 4-byte aligned");
  float* partials = static_cast<float*>(ws);
  switch (dtype) {
    case KPB_F32: return launch(variant, static_cast<const float*>(x), out, n, partials, s);
    case KPB_F16: return launch(variant, static_cast<const __half*>(x), out, n, partials, s);
    case KPB_BF16:
      return launch(variant, static_cast<const __nv_bfloat16*>(x), out, n, partials, s);
    default: return fail(KPB_EINVAL, "reduce_sum: unknown dtype " + std::to_string(dtype));
  }
}

}  // namespace kpb
