// Row softmax over the last dimension of a contiguous (M, N) matrix (kp.softmax).
//
// Replaces kernelpilot's csrc/kernels/softmax.hip (stages :14-113, dispatch
// :116-152). The contract is the same (fp32 math, output in the input dtype,
// empty input is a no-op); the B200 kernel is new:
//
//   variant 0  thread per row, three passes over global memory (baseline)
//   variant 1  CTA per row, three coalesced passes with block reductions
//   variant 2  "staged": a persistent grid; each CTA owns a ring of row buffers in
//              shared memory filled by 1-D bulk (TMA) copies issued `stages` rows
//              ahead, so HBM reads of later rows overlap the reductions of the
//              current one. Every thread keeps its slice of the row in registers:
//              max -> exp2 -> sum -> scale -> 128-bit streaming stores. HBM sees one
//              read and one write per element. The arithmetic is packed (3-input max,
//              f32x2 FMA/add/mul) and exp2 runs on the MUFU directly, about 4.5
//              instructions per element, so the kernel stays memory-bound.
//              Rows longer than 1024 threads x 24 (fp32) / 32 (16-bit) values take
//              "two-pass": online (max, sum) in one read, normalise in a second.
//
// Rows need not start on a 16-byte boundary (fp32 N=4097 rows are 16388 bytes):
// each row is viewed through the aligned window that contains it. Whole 16-byte
// vectors inside the row are moved as vectors; the partial vectors at each end of a
// row use masked scalar accesses, and the bulk copy never reaches outside x. When
// every row is aligned (kAligned) the masking disappears from the kernel.
#include <algorithm>

#include "kp_common.cuh"
#include "kp_sm100.cuh"

namespace kpb {
namespace {

constexpr float kLog2e = 1.4426950408889634f;
constexpr int kMaxStages = 8;
// 16-byte vectors per thread in the staged kernel: at most 24 (fp32) or 32 (16-bit)
// row values live in registers, which keeps 1024-thread CTAs free of spills.
template <typename T> constexpr int staged_max_v() { return sizeof(T) == 4 ? 6 : 4; }

// ------------------------------------------------------------------ variant 0

template <typename T>
__global__ void softmax_thread_row(const T* __restrict__ x, T* __restrict__ y, int64_t M,
                                   int64_t N) {
  const int64_t row = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (row >= M) return;
  const T* xr = x + row * N;
  T* yr = y + row * N;
  float m = -INFINITY;
  for (int64_t j = 0; j < N; ++j) m = fmaxf(m, to_f(xr[j]));
  const float ml = m * kLog2e;
  float d = 0.f;
  for (int64_t j = 0; j < N; ++j) d += exp2f(fmaf(to_f(xr[j]), kLog2e, -ml));
  const float inv = 1.f / d;
  for (int64_t j = 0; j < N; ++j) yr[j] = from_f<T>(exp2f(fmaf(to_f(xr[j]), kLog2e, -ml)) * inv);
}

// ------------------------------------------------------------------ variant 1

template <typename T>
__global__ void __launch_bounds__(256) softmax_block_row(const T* __restrict__ x,
                                                         T* __restrict__ y, int64_t N) {
  __shared__ float s_max[kWarp], s_sum[kWarp];
  const T* xr = x + static_cast<int64_t>(blockIdx.x) * N;
  T* yr = y + static_cast<int64_t>(blockIdx.x) * N;
  float m = -INFINITY;
  for (int64_t j = threadIdx.x; j < N; j += blockDim.x) m = fmaxf(m, to_f(xr[j]));
  m = block_reduce<true>(m, s_max);
  const float ml = m * kLog2e;
  float d = 0.f;
  for (int64_t j = threadIdx.x; j < N; j += blockDim.x)
    d += exp2f(fmaf(to_f(xr[j]), kLog2e, -ml));
  d = block_reduce<false>(d, s_sum);
  const float inv = 1.f / d;
  for (int64_t j = threadIdx.x; j < N; j += blockDim.x)
    yr[j] = from_f<T>(exp2f(fmaf(to_f(xr[j]), kLog2e, -ml)) * inv);
}

// ------------------------------------------------------------------ variant 2: staged

// Geometry of one row seen through its aligned window.
struct RowView {
  uintptr_t win;    // 16-byte aligned address at or below the row start
  int a;            // elements between `win` and the row start
  int nv;           // 16-byte vectors covering the row
};

template <typename T>
__device__ __forceinline__ RowView row_view(uintptr_t row_start, int N) {
  constexpr int VN = Vec<T>::kN;
  RowView r;
  r.win = row_start & ~uintptr_t(15);
  r.a = static_cast<int>((row_start - r.win) / sizeof(T));
  r.nv = (r.a + N + VN - 1) / VN;
  return r;
}

// Per-vector element math on registers, two lanes at a time.
template <int VN>
__device__ __forceinline__ float vmax(const float (&f)[VN], float m) {
#pragma unroll
  for (int l = 0; l < VN; l += 2) m = max3f(m, f[l], f[l + 1]);
  return m;
}

// f <- exp2(f * log2e - ml); returns the running sum of the new values (two partials).
template <int VN>
__device__ __forceinline__ float2 vexp(float (&f)[VN], float2 acc, float neg_ml) {
  const float2 s2 = make_float2(kLog2e, kLog2e), c2 = make_float2(neg_ml, neg_ml);
#pragma unroll
  for (int l = 0; l < VN; l += 2) {
    float2 t = __ffma2_rn(make_float2(f[l], f[l + 1]), s2, c2);
    t.x = ex2f(t.x);
    t.y = ex2f(t.y);
    f[l] = t.x;
    f[l + 1] = t.y;
    acc = __fadd2_rn(acc, t);
  }
  return acc;
}

template <int VN>
__device__ __forceinline__ void vscale(float (&f)[VN], float inv) {
  const float2 i2 = make_float2(inv, inv);
#pragma unroll
  for (int l = 0; l < VN; l += 2) {
    const float2 t = __fmul2_rn(make_float2(f[l], f[l + 1]), i2);
    f[l] = t.x;
    f[l + 1] = t.y;
  }
}

template <typename T, int V, bool kAligned>
__global__ void __launch_bounds__(1024)
softmax_staged(const T* __restrict__ x, T* __restrict__ y, int64_t M, int N, int stages,
               uint32_t stage_bytes, unsigned* err) {
  constexpr int VN = Vec<T>::kN;
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint8_t* ring = smem + 128;
  __shared__ float s_max[kWarp], s_sum[kWarp];

  const uintptr_t xbase = reinterpret_cast<uintptr_t>(x);
  const uintptr_t xend = xbase + static_cast<uintptr_t>(M) * N * sizeof(T);
  const uintptr_t ok_lo = (xbase + 15) & ~uintptr_t(15);  // bulk copies stay in [ok_lo, ok_hi)
  const uintptr_t ok_hi = xend & ~uintptr_t(15);
  const size_t row_bytes = static_cast<size_t>(N) * sizeof(T);
  const bool y_vec = ((reinterpret_cast<uintptr_t>(y) ^ xbase) & 15) == 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) mbar_init(&full[s], 1);
    fence_mbar_init();
  }
  __syncthreads();
  const uint64_t policy = l2_evict_first_policy();

  // copied part of a row's window, in vectors: [vlo, vhi)
  auto copy_span = [&](const RowView& rv, int& vlo, int& vhi) {
    const uintptr_t cs = rv.win > ok_lo ? rv.win : ok_lo;
    const uintptr_t we = rv.win + static_cast<uintptr_t>(rv.nv) * 16;
    const uintptr_t ce = we < ok_hi ? we : ok_hi;
    vlo = static_cast<int>((cs - rv.win) / 16);
    vhi = ce > cs ? static_cast<int>((ce - rv.win) / 16) : vlo;
  };

  // Thread 0: start the copy of `row` into ring slot `slot`.
  auto issue = [&](int64_t row, int slot) {
    const RowView rv = row_view<T>(xbase + static_cast<uintptr_t>(row) * row_bytes, N);
    int vlo, vhi;
    copy_span(rv, vlo, vhi);
    if (vhi > vlo) {
      const uint32_t bytes = static_cast<uint32_t>(vhi - vlo) * 16;
      mbar_arrive_expect_tx(&full[slot], bytes);
      bulk_g2s(ring + size_t(slot) * stage_bytes + vlo * 16,
               reinterpret_cast<const void*>(rv.win + static_cast<uintptr_t>(vlo) * 16), bytes,
               &full[slot], policy);
    } else {
      mbar_arrive(&full[slot]);
    }
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      const int64_t r = blockIdx.x + static_cast<int64_t>(s) * gridDim.x;
      if (r < M) issue(r, s);
    }
  }

  int it = 0;
  for (int64_t row = blockIdx.x; row < M; row += gridDim.x, ++it) {
    const int slot = it % stages;
    const bool ok = mbar_wait(&full[slot], static_cast<uint32_t>((it / stages) & 1), err);
    if (__syncthreads_or(!ok)) return;

    const RowView rv = row_view<T>(xbase + static_cast<uintptr_t>(row) * row_bytes, N);
    int vlo = 0, vhi = rv.nv;
    if (!kAligned) copy_span(rv, vlo, vhi);
    const uint8_t* stage = ring + size_t(slot) * stage_bytes;
    const T* xr = x + row * N;

    float f[V][VN];
    float mx = -INFINITY;
#pragma unroll
    for (int k = 0; k < V; ++k) {
      const int j = threadIdx.x + k * blockDim.x;
      if (kAligned) {
        if (j < rv.nv) {
          unpack<T>(*reinterpret_cast<const uint4*>(stage + j * 16), f[k]);
        } else {
#pragma unroll
          for (int l = 0; l < VN; ++l) f[k][l] = -INFINITY;
        }
      } else {
        const int e0 = j * VN - rv.a;
        if (j >= vlo && j < vhi && e0 >= 0 && e0 + VN <= N) {
          unpack<T>(*reinterpret_cast<const uint4*>(stage + j * 16), f[k]);
        } else {
#pragma unroll
          for (int l = 0; l < VN; ++l) {
            const int e = e0 + l;
            f[k][l] = (j < rv.nv && e >= 0 && e < N) ? to_f(xr[e]) : -INFINITY;
          }
        }
      }
      mx = vmax<VN>(f[k], mx);
    }
    mx = block_reduce<true>(mx, s_max);
    // every thread has read its slice of the slot: refill it with a later row
    if (threadIdx.x == 0) {
      const int64_t nr = row + static_cast<int64_t>(stages) * gridDim.x;
      if (nr < M) issue(nr, slot);
    }

    const float neg_ml = -(mx * kLog2e);
    float2 acc = make_float2(0.f, 0.f);
#pragma unroll
    for (int k = 0; k < V; ++k) acc = vexp<VN>(f[k], acc, neg_ml);
    const float sum = block_reduce<false>(acc.x + acc.y, s_sum);
    const float inv = 1.f / sum;

    T* yr = y + row * N;
    uint8_t* ywin = reinterpret_cast<uint8_t*>(reinterpret_cast<uintptr_t>(yr) - rv.a * sizeof(T));
#pragma unroll
    for (int k = 0; k < V; ++k) {
      const int j = threadIdx.x + k * blockDim.x;
      if (j >= rv.nv) continue;
      vscale<VN>(f[k], inv);
      const int e0 = j * VN - rv.a;
      if (kAligned || (y_vec && e0 >= 0 && e0 + VN <= N)) {
        st_stream(ywin + j * 16, pack<T>(f[k]));
      } else {
#pragma unroll
        for (int l = 0; l < VN; ++l)
          if (e0 + l >= 0 && e0 + l < N) yr[e0 + l] = from_f<T>(f[k][l]);
      }
    }
  }
}

// ------------------------------------------------------------------ variant 2: two-pass

// Online-softmax state: ml = round(max * log2e), d = sum of exp2(x*log2e - ml).
// Every exponent is taken against a rounded ml with one FMA, and rescaling uses
// differences of the same rounded values, so all partial sums stay consistent with
// the final normalisation exp2(fma(x, log2e, -ml)).
__device__ __forceinline__ void online_merge(float& ml, float& d, float ml2, float d2) {
  const float mn = fmaxf(ml, ml2);
  if (mn == -INFINITY) return;
  d = d * ex2f(ml - mn) + d2 * ex2f(ml2 - mn);
  ml = mn;
}

template <typename T>
__global__ void __launch_bounds__(1024)
softmax_two_pass(const T* __restrict__ x, T* __restrict__ y, int N) {
  constexpr int VN = Vec<T>::kN;
  __shared__ float s_m[kWarp], s_d[kWarp];
  const int64_t row = blockIdx.x;
  const T* xr = x + row * N;
  T* yr = y + row * N;
  const RowView rv = row_view<T>(reinterpret_cast<uintptr_t>(xr), N);
  const bool y_vec = ((reinterpret_cast<uintptr_t>(y) ^ reinterpret_cast<uintptr_t>(x)) & 15) == 0;

  // pass 1: online (max, sum); the row stays in L2 for pass 2 (normal priority)
  float m = -INFINITY, d = 0.f;  // m holds round(max * log2e)
  for (int j = threadIdx.x; j < rv.nv; j += blockDim.x) {
    const int e0 = j * VN - rv.a;
    float f[VN];
    if (e0 >= 0 && e0 + VN <= N) {
      unpack<T>(ld_keep(reinterpret_cast<const void*>(rv.win + static_cast<uintptr_t>(j) * 16)), f);
    } else {
#pragma unroll
      for (int l = 0; l < VN; ++l)
        f[l] = (e0 + l >= 0 && e0 + l < N) ? to_f(xr[e0 + l]) : -INFINITY;
    }
    const float mn = fmaxf(m, vmax<VN>(f, -INFINITY) * kLog2e);
    const float2 s = vexp<VN>(f, make_float2(0.f, 0.f), -mn);
    d = (m == -INFINITY ? 0.f : d * ex2f(m - mn)) + (s.x + s.y);
    m = mn;
  }
#pragma unroll
  for (int o = kWarp / 2; o > 0; o >>= 1) {
    const float m2 = __shfl_xor_sync(kFull, m, o), d2 = __shfl_xor_sync(kFull, d, o);
    online_merge(m, d, m2, d2);
  }
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  if (lane == 0) { s_m[wid] = m; s_d[wid] = d; }
  __syncthreads();
  const int nw = blockDim.x / kWarp;
  m = lane < nw ? s_m[lane] : -INFINITY;
  d = lane < nw ? s_d[lane] : 0.f;
#pragma unroll
  for (int o = kWarp / 2; o > 0; o >>= 1) {
    const float m2 = __shfl_xor_sync(kFull, m, o), d2 = __shfl_xor_sync(kFull, d, o);
    online_merge(m, d, m2, d2);
  }
  const float neg_ml = -m, inv = 1.f / d;

  // pass 2: normalise
  const uint64_t pol = evict_first_policy();
  uint8_t* ywin = reinterpret_cast<uint8_t*>(reinterpret_cast<uintptr_t>(yr) - rv.a * sizeof(T));
  for (int j = threadIdx.x; j < rv.nv; j += blockDim.x) {
    const int e0 = j * VN - rv.a;
    float f[VN];
    if (e0 >= 0 && e0 + VN <= N) {
      unpack<T>(ld_stream(reinterpret_cast<const void*>(rv.win + static_cast<uintptr_t>(j) * 16), pol), f);
      vexp<VN>(f, make_float2(0.f, 0.f), neg_ml);
      vscale<VN>(f, inv);
      if (y_vec) {
        st_stream(ywin + static_cast<uintptr_t>(j) * 16, pack<T>(f));
        continue;
      }
    } else {
#pragma unroll
      for (int l = 0; l < VN; ++l)
        f[l] = (e0 + l >= 0 && e0 + l < N) ? ex2f(fmaf(to_f(xr[e0 + l]), kLog2e, neg_ml)) * inv : 0.f;
    }
#pragma unroll
    for (int l = 0; l < VN; ++l)
      if (e0 + l >= 0 && e0 + l < N) yr[e0 + l] = from_f<T>(f[l]);
  }
}

// ------------------------------------------------------------------ launch

struct StagedPlan {
  int threads, v, stages, ctas_per_sm;
  uint32_t stage_bytes;
};

// Every row starts on a 16-byte boundary and is a whole number of vectors.
template <typename T>
bool rows_aligned(const T* x, const T* y, int64_t N) {
  return reinterpret_cast<uintptr_t>(x) % 16 == 0 && reinterpret_cast<uintptr_t>(y) % 16 == 0 &&
         (N * static_cast<int64_t>(sizeof(T))) % 16 == 0;
}

// Vectors per row window: N/VN when every row starts 16-byte aligned, else the
// worst case over row start offsets.
template <typename T>
int64_t window_vectors(bool aligned, int64_t N) {
  constexpr int VN = Vec<T>::kN;
  return aligned ? cdiv(N, VN) : (N + 2 * VN - 2) / VN;
}

template <typename T>
StagedPlan plan_staged(int64_t nv_max) {
  StagedPlan p{};
  // Cost of one row per CTA ~ threads * (V + 5): V vectors of element work plus a
  // fixed per-row share (two block reductions, the slot wait, the refill) worth about
  // five vectors. Fewer, fuller threads win for short rows.
  int64_t best = INT64_MAX;
  for (int t = 64; t <= 1024; t += 64) {
    const int64_t v = cdiv(nv_max, t);
    if (v > staged_max_v<T>()) continue;
    const int64_t cost = t * (v + 5);
    if (cost < best) {
      best = cost;
      p.threads = t;
      p.v = static_cast<int>(v);
    }
  }
  p.stage_bytes = static_cast<uint32_t>(cdiv(nv_max * 16, 128) * 128);
  // Most CTAs per SM (independent rows reducing at once) that still leaves each CTA
  // two ring slots, i.e. one row loading while one is reduced; a lone CTA may take
  // up to kMaxStages slots.
  const int64_t smem_per_sm = 220 * 1024;
  p.stages = 1;
  p.ctas_per_sm = 1;
  for (int c = 2048 / p.threads; c >= 1; --c) {
    const int64_t st = std::min<int64_t>(kMaxStages, smem_per_sm / c / (p.stage_bytes + 1024));
    if (st >= 2 || (c == 1 && st >= 1)) {
      p.stages = static_cast<int>(st);
      p.ctas_per_sm = c;
      break;
    }
  }
  return p;
}

template <typename T, int V, bool kAligned>
int launch_staged(const T* x, T* y, int64_t M, int64_t N, const StagedPlan& p, unsigned* err,
                  cudaStream_t s) {
  auto kern = softmax_staged<T, V, kAligned>;
  const size_t smem = 128 + size_t(p.stages) * p.stage_bytes;
  KPB_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                static_cast<int>(smem)));
  int occ = 0;
  KPB_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, p.threads, smem));
  if (occ < 1) return fail(KPB_ECUDA, "softmax: staged kernel does not fit on an SM");
  const int64_t grid = std::min<int64_t>(M, int64_t(sm_count()) * std::min(occ, p.ctas_per_sm));
  kern<<<static_cast<unsigned>(grid), p.threads, smem, s>>>(x, y, M, static_cast<int>(N),
                                                            p.stages, p.stage_bytes, err);
  KPB_LAUNCHED("softmax staged");
  return KPB_OK;
}

template <typename T, bool kAligned>
int dispatch_v(const T* x, T* y, int64_t M, int64_t N, const StagedPlan& p, unsigned* err,
               cudaStream_t s) {
  constexpr bool f32 = sizeof(T) == 4;
  switch (p.v) {
    case 1: return launch_staged<T, 1, kAligned>(x, y, M, N, p, err, s);
    case 2: return launch_staged<T, 2, kAligned>(x, y, M, N, p, err, s);
    case 3: return launch_staged<T, 3, kAligned>(x, y, M, N, p, err, s);
    case 4: return launch_staged<T, 4, kAligned>(x, y, M, N, p, err, s);
    case 5: return launch_staged<T, f32 ? 5 : 4, kAligned>(x, y, M, N, p, err, s);
    default: return launch_staged<T, f32 ? 6 : 4, kAligned>(x, y, M, N, p, err, s);
  }
}

template <typename T>
int launch(int variant, const T* x, T* y, int64_t M, int64_t N, unsigned* err, cudaStream_t s) {
  if (M == 0 || N == 0) return KPB_OK;
  if (reinterpret_cast<uintptr_t>(x) % sizeof(T) || reinterpret_cast<uintptr_t>(y) % sizeof(T))
    return fail(KPB_EINVAL, "softmax: x and y must be element-aligned");
  if (variant == 0) {
    softmax_thread_row<T><<<static_cast<unsigned>(cdiv(M, 128)), 128, 0, s>>>(x, y, M, N);
    KPB_LAUNCHED("softmax variant 0");
    return KPB_OK;
  }
  if (variant == 1) {
    softmax_block_row<T><<<static_cast<unsigned>(M), 256, 0, s>>>(x, y, N);
    KPB_LAUNCHED("softmax variant 1");
    return KPB_OK;
  }
  const bool aligned = rows_aligned(x, y, N);
  const int64_t nv_max = window_vectors<T>(aligned, N);
  if (nv_max > 1024 * staged_max_v<T>()) {
    softmax_two_pass<T><<<static_cast<unsigned>(M), 1024, 0, s>>>(x, y, static_cast<int>(N));
    KPB_LAUNCHED("softmax two-pass");
    return KPB_OK;
  }
  const StagedPlan p = plan_staged<T>(nv_max);
  return aligned ? dispatch_v<T, true>(x, y, M, N, p, err, s)
                 : dispatch_v<T, false>(x, y, M, N, p, err, s);
}

}  // namespace

int softmax(int variant, int dtype, const void* x, void* y, int64_t M, int64_t N,
            unsigned* err, cudaStream_t s) {
  switch (dtype) {
    case KPB_F32:
      return launch(variant, static_cast<const float*>(x), static_cast<float*>(y), M, N, err, s);
    case KPB_F16:
      return launch(variant, static_cast<const __half*>(x), static_cast<__half*>(y), M, N, err, s);
    case KPB_BF16:
      return launch(variant, static_cast<const __nv_bfloat16*>(x),
                    static_cast<__nv_bfloat16*>(y), M, N, err, s);
    default: return fail(KPB_EINVAL, "softmax: unknown dtype " + std::to_string(dtype));
  }
}

}  // namespace kpb
