// A candidate that compiles and runs but computes a - b: the worker must reject it at
// the correctness stage, whatever its speed.
#include <ATen/cuda/CUDAContext.h>

__global__ void sub(const float* a, const float* b, float* c, int64_t n) {
  const int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (i < n) c[i] = a[i] - b[i];
}

torch::Tensor kernel_fn(torch::Tensor x0, torch::Tensor x1) {
  auto c = torch::empty_like(x0);
  const int64_t n = x0.numel();
  if (n) {
    sub<<<kp::ceil_div(n, 256), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
        x0.data_ptr<float>(), x1.data_ptr<float>(), c.data_ptr<float>(), n);
    KP_CHECK_LAUNCH();
  }
  return c;
}
