// kpb_reduce_sum_noalloc: the full sum (the persistent variant-2 kernels) with its
// per-CTA partials kept in a fixed device array compiled into this library, so the
// call allocates nothing.
//
// Who needs it: callers that must not allocate device memory at the moment they call
// us. Examples are code that receives a fixed memory budget at start-up and may not
// grow it, code whose device memory belongs to another allocator (a cudaMalloc here
// would bypass that allocator's accounting and can synchronise the whole device in
// the middle of a pipeline), and runtimes that forbid allocation after
// initialisation. They still pass their own input and output; only the scratch is
// built in.
//
// Limits and behaviour:
//   * the scratch holds kNoAllocMaxPartials fp32 partials (16 KB). Every GPU that loads
//     this library keeps that array until the process exits. A call that would need
//     more partials (more than 4096 level-1 CTAs, i.e. a GPU with over 1365 SMs) is
//     rejected with KPB_EINVAL and a message;
//   * the first call on each device looks up the array's device address
//     (cudaGetSymbolAddress) with that device current and caches it; make that first
//     call before any stream capture begins;
//   * every call on a device shares the one array and it keeps the last call's
//     partials. Nothing needs clearing: each call writes every partial it later reads.
//     Calls that overlap on the GPU (different streams, or different host threads
//     without ordering) race on the array and may return wrong sums; order them on one
//     stream.
#include <mutex>

#include "kp_common.cuh"

namespace kpb {

int reduce_sum(int variant, int dtype, const void* x, float* out, int64_t n, void* ws,
               size_t ws_bytes, cudaStream_t s);
int64_t reduce_partials_needed(int variant, int64_t n);

namespace {

constexpr int kNoAllocMaxPartials = 4096;
constexpr int kNoAllocVariant = 2;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) float g_noalloc_partials[kNoAllocMaxPartials];

std::mutex g_noalloc_mu;
float* g_noalloc_ptr[kMaxDevices] = {nullptr};

// Device address of this device's copy of g_noalloc_partials (host code cannot use
// the symbol itself: on the host it names a host-side stand-in, not device memory).
int noalloc_partials(float** out) {
  int dev = -1;
  KPB_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices)
    return fail(KPB_EUNSUPPORTED, "reduce_sum_noalloc: device index out of range");
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (g_noalloc_ptr[dev] == nullptr) {
    void* p = nullptr;
    KPB_CUDA(cudaGetSymbolAddress(&p, g_noalloc_partials));
    g_noalloc_ptr[dev] = static_cast<float*>(p);
  }
  *out = g_noalloc_ptr[dev];
  return KPB_OK;
}

}  // namespace
}  // namespace kpb

extern "C" int kpb_reduce_sum_noalloc(int dtype, const void* x, float* out, int64_t n,
                                      void* stream) {
  using namespace kpb;
  set_error("");
  if (dtype != KPB_F32 && dtype != KPB_F16 && dtype != KPB_BF16)
    return fail(KPB_EINVAL, "reduce_sum_noalloc: dtype must be 0 (f32), 1 (f16) or 2 (bf16)");
  if (n < 0) return fail(KPB_EINVAL, "reduce_sum_noalloc: n must be >= 0");
  if (out == nullptr || (n > 0 && x == nullptr))
    return fail(KPB_EINVAL, "reduce_sum_noalloc: null pointer");
  const int64_t need = reduce_partials_needed(kNoAllocVariant, n);
  if (need > kNoAllocMaxPartials)
    return fail(KPB_EINVAL, "reduce_sum_noalloc: this device needs " + std::to_string(need) +
                                " partials but the built-in scratch holds " +
                                std::to_string(kNoAllocMaxPartials));
  float* partials = nullptr;
  if (int rc = noalloc_partials(&partials)) return rc;
  return reduce_sum(kNoAllocVariant, dtype, x, out, n, partials,
                    sizeof(float) * kNoAllocMaxPartials, static_cast<cudaStream_t>(stream));
}
