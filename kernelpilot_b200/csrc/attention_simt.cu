// CUDA-core attention kernels for kp.attention / kp.attention_causal: variant 0 for
// every dtype, and the fp32 (and unsupported head-dim) path of variant 1. fp32 keeps
// exact fp32 math end to end, which its (1e-5, 1e-4) tolerance
// (kernelpilot/specs.py:281-282) requires.
//
// Replaces kernelpilot's csrc/kernels/attention.hip (:13-110):
//   naive       one CTA per (head, query): the score row lives in shared memory
//   warp_flash  one warp per query, 8 queries per CTA sharing K/V tiles of 32 keys
//               in shared memory; lane l scores key l of the tile, the online
//               softmax runs across the warp, and lane l accumulates output dims
//               l, l+32, ... (no per-thread D-wide arrays, so D=128 does not spill)
#include "kp_common.cuh"

namespace kpb {

constexpr float kLog2eA = 1.4426950408889634f;

template <typename T, bool kCausal>
__global__ void __launch_bounds__(128) attn_naive(const T* __restrict__ q, const T* __restrict__ k,
                                                  const T* __restrict__ v, T* __restrict__ o,
                                                  int64_t S, int D, float scale_log2) {
  extern __shared__ float sm[];
  float* qs = sm;      // D
  float* sc = sm + D;  // S
  __shared__ float s_max[kWarp], s_sum[kWarp];
  const int64_t i = blockIdx.x;
  const int64_t base = static_cast<int64_t>(blockIdx.y) * S * D;
  for (int d = threadIdx.x; d < D; d += blockDim.x) qs[d] = to_f(q[base + i * D + d]);
  __syncthreads();
  const int64_t nk = kCausal ? i + 1 : S;
  float mx = -INFINITY;
  for (int64_t j = threadIdx.x; j < nk; j += blockDim.x) {
    const T* kr = k + base + j * D;
    float s = 0.f;
    for (int d = 0; d < D; ++d) s = fmaf(qs[d], to_f(kr[d]), s);
    s *= scale_log2;
    sc[j] = s;
    mx = fmaxf(mx, s);
  }
  mx = block_reduce<true>(mx, s_max);
  float sum = 0.f;
  for (int64_t j = threadIdx.x; j < nk; j += blockDim.x) {
    const float p = exp2f(sc[j] - mx);
    sc[j] = p;
    sum += p;
  }
  sum = block_reduce<false>(sum, s_sum);
  __syncthreads();  // all probabilities written
  const float inv = 1.f / sum;
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float acc = 0.f;
    for (int64_t j = 0; j < nk; ++j) acc = fmaf(sc[j], to_f(v[base + j * D + d]), acc);
    o[base + i * D + d] = from_f<T>(acc * inv);
  }
}

constexpr int kWfWarps = 8;
constexpr int kWfKeys = 32;

template <typename T, int DPL, bool kCausal>
__global__ void __launch_bounds__(kWfWarps * 32)
attn_warp_flash(const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
                T* __restrict__ o, int64_t S, int D, float scale_log2) {
  extern __shared__ float sm[];
  const int DP = D + 1;
  float* ks = sm;                        // [32][D+1]
  float* vs = ks + kWfKeys * DP;         // [32][D]
  float* qs = vs + kWfKeys * D;          // [8][D]
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int64_t base = static_cast<int64_t>(blockIdx.y) * S * D;
  const int64_t q0 = static_cast<int64_t>(blockIdx.x) * kWfWarps;
  const int64_t i = q0 + warp;
  const bool active = i < S;
  float* qw = qs + warp * D;
  for (int d = lane; d < D; d += 32) qw[d] = active ? to_f(q[base + i * D + d]) * scale_log2 : 0.f;

  float m = -INFINITY, l = 0.f, acc[DPL];
#pragma unroll
  for (int t = 0; t < DPL; ++t) acc[t] = 0.f;
  const int64_t q_last = (q0 + kWfWarps - 1 < S ? q0 + kWfWarps - 1 : S - 1);
  const int64_t kend = kCausal ? q_last + 1 : S;
  for (int64_t j0 = 0; j0 < kend; j0 += kWfKeys) {
    __syncthreads();  // previous tile fully consumed (and q rows written, first time)
    const int nk = static_cast<int>(kend - j0 < kWfKeys ? kend - j0 : kWfKeys);
    for (int e = threadIdx.x; e < kWfKeys * D; e += blockDim.x) {
      const int r = e / D, c = e % D;
      const bool ok = r < nk;
      ks[r * DP + c] = ok ? to_f(k[base + (j0 + r) * D + c]) : 0.f;
      vs[r * D + c] = ok ? to_f(v[base + (j0 + r) * D + c]) : 0.f;
    }
    __syncthreads();
    if (!active) continue;
    const int64_t j = j0 + lane;
    const bool valid = lane < nk && (!kCausal || j <= i);
    float s = -INFINITY;
    if (valid) {
      s = 0.f;
      const float* kr = ks + lane * DP;
      for (int d = 0; d < D; ++d) s = fmaf(qw[d], kr[d], s);
    }
    const float mt = warp_max(s);
    const float mn = fmaxf(m, mt);
    if (mn == -INFINITY) continue;  // every key of this tile is masked for this query
    const float p = exp2f(s - mn);
    const float corr = exp2f(m - mn);
    l = l * corr + warp_sum(p);
#pragma unroll
    for (int t = 0; t < DPL; ++t) acc[t] *= corr;
    for (int ll = 0; ll < nk; ++ll) {
      const float pl = __shfl_sync(kFull, p, ll);
      const float* vr = vs + ll * D;
#pragma unroll
      for (int t = 0; t < DPL; ++t) {
        const int d = lane + 32 * t;
        if (d < D) acc[t] = fmaf(pl, vr[d], acc[t]);
      }
    }
    m = mn;
  }
  if (!active) return;
  const float inv = 1.f / l;
#pragma unroll
  for (int t = 0; t < DPL; ++t) {
    const int d = lane + 32 * t;
    if (d < D) o[base + i * D + d] = from_f<T>(acc[t] * inv);
  }
}

template <typename T, bool kCausal>
int attention_simt_t(int variant, const T* q, const T* k, const T* v, T* o, int64_t BH,
                     int64_t S, int D, cudaStream_t s) {
  const float scale_log2 = kLog2eA / sqrtf(static_cast<float>(D));
  if (variant == 0) {
    const size_t smem = static_cast<size_t>(S + D) * sizeof(float);
    if (smem > 220 * 1024)
      return fail(KPB_EUNSUPPORTED, "attention variant 0: S too large for the score row");
    auto kern = attn_naive<T, kCausal>;
    if (smem > 48 * 1024)
      KPB_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    static_cast<int>(smem)));
    kern<<<dim3(static_cast<unsigned>(S), static_cast<unsigned>(BH)), 128, smem, s>>>(
        q, k, v, o, S, D, scale_log2);
    KPB_LAUNCHED("attention naive");
    return KPB_OK;
  }
  const size_t smem = static_cast<size_t>(kWfKeys * (D + 1) + kWfKeys * D + kWfWarps * D) *
                      sizeof(float);
  const dim3 grid(static_cast<unsigned>(cdiv(S, kWfWarps)), static_cast<unsigned>(BH));
  auto go = [&](auto kern) -> int {
    if (smem > 48 * 1024)
      KPB_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    static_cast<int>(smem)));
    kern<<<grid, kWfWarps * 32, smem, s>>>(q, k, v, o, S, D, scale_log2);
    KPB_LAUNCHED("attention warp_flash");
    return KPB_OK;
  };
  if (D <= 32) return go(attn_warp_flash<T, 1, kCausal>);
  if (D <= 64) return go(attn_warp_flash<T, 2, kCausal>);
  if (D <= 128) return go(attn_warp_flash<T, 4, kCausal>);
  return go(attn_warp_flash<T, 8, kCausal>);
}

template <typename T>
int attention_simt_c(int variant, bool causal, const void* q, const void* k, const void* v,
                     void* o, int64_t BH, int64_t S, int D, cudaStream_t s) {
  auto qq = static_cast<const T*>(q), kk = static_cast<const T*>(k), vv = static_cast<const T*>(v);
  auto oo = static_cast<T*>(o);
  return causal ? attention_simt_t<T, true>(variant, qq, kk, vv, oo, BH, S, D, s)
                : attention_simt_t<T, false>(variant, qq, kk, vv, oo, BH, S, D, s);
}

int attention_simt(int variant, int dtype, bool causal, const void* q, const void* k,
                   const void* v, void* o, int64_t BH, int64_t S, int64_t D, cudaStream_t s) {
  const int d = static_cast<int>(D);
  switch (dtype) {
    case KPB_F32: return attention_simt_c<float>(variant, causal, q, k, v, o, BH, S, d, s);
    case KPB_F16: return attention_simt_c<__half>(variant, causal, q, k, v, o, BH, S, d, s);
    case KPB_BF16:
      return attention_simt_c<__nv_bfloat16>(variant, causal, q, k, v, o, BH, S, d, s);
    default: return fail(KPB_EINVAL, "attention: unknown dtype");
  }
}

}  // namespace kpb
