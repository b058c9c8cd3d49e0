// A correct, plain candidate for the softmax contract: one CTA per row, three passes
// over the row (max, sum of exponentials, normalise) with CTA-wide reductions from
// kp_contract.cuh. fp32 math for every dtype.
#include <ATen/cuda/CUDAContext.h>

template <typename T>
__global__ void softmax_rows(const T* __restrict__ x, T* __restrict__ y, int64_t n) {
  __shared__ float scratch[kp::kMaxWarps];
  const T* xr = x + blockIdx.x * n;
  T* yr = y + blockIdx.x * n;
  float m = -INFINITY;
  for (int64_t j = threadIdx.x; j < n; j += blockDim.x) m = fmaxf(m, kp::to_float(xr[j]));
  m = kp::block_reduce<true>(m, scratch);
  float s = 0.f;
  for (int64_t j = threadIdx.x; j < n; j += blockDim.x) s += expf(kp::to_float(xr[j]) - m);
  s = kp::block_reduce<false>(s, scratch);
  for (int64_t j = threadIdx.x; j < n; j += blockDim.x)
    yr[j] = kp::from_float<T>(expf(kp::to_float(xr[j]) - m) / s);
}

torch::Tensor kernel_fn(torch::Tensor x0) {
  auto y = torch::empty_like(x0);
  const int64_t n = x0.size(-1);
  const int64_t rows = n ? x0.numel() / n : 0;
  if (rows == 0) return y;
  auto stream = at::cuda::getCurrentCUDAStream();
  if (x0.scalar_type() == at::kFloat) {
    softmax_rows<float><<<rows, 256, 0, stream>>>(x0.data_ptr<float>(), y.data_ptr<float>(), n);
  } else if (x0.scalar_type() == at::kHalf) {
    softmax_rows<__half><<<rows, 256, 0, stream>>>(
        reinterpret_cast<const __half*>(x0.data_ptr()), reinterpret_cast<__half*>(y.data_ptr()), n);
  } else {
    softmax_rows<__nv_bfloat16><<<rows, 256, 0, stream>>>(
        reinterpret_cast<const __nv_bfloat16*>(x0.data_ptr()),
        reinterpret_cast<__nv_bfloat16*>(y.data_ptr()), n);
  }
  KP_CHECK_LAUNCH();
  return y;
}
