// kpb_peer_sum_*: the full sum of a vector sharded over the GPUs of one node (one
// process per GPU), with the exchange of the per-GPU partials inside the finishing
// kernel, over NVLink peer memory, instead of a separate collective.
//
// kernelpilot itself has no multi-GPU code; its reduction ends in a float atomicAdd
// on one GPU (csrc/kernels/reduction.hip:86). The data-parallel layer here shards
// the vector and needs one exchange step: the sum of the per-GPU partials. Done as
// an NCCL all_reduce of one float that step costs a separate kernel and ~10-15 us of
// collective latency per call. Here the one-CTA finishing kernel of the persistent
// reduction does it:
//   * every rank owns an exchange buffer (cudaMalloc'd once, exported as a CUDA IPC
//     handle; every rank opens the others' handles once) holding 2 rows x 8 slots of
//     64-bit words that peers write, and two control words only its own rank uses:
//     the call counter and a sticky "out of step" flag;
//   * the call number k lives in device memory: each finishing kernel reads the
//     counter, uses k = counter + 1 and writes k back. Calls are ordered on one
//     stream, so a CUDA graph that captured the call advances k on every replay just
//     as eager calls do;
//   * call k uses row k & 1: the kernel adds its local partials in a fixed order, then
//     stores the word (k << 32 | bits of its sum) into slot [k & 1][rank] of every
//     rank's buffer (a system-scope release store, over NVLink for the peers), then
//     one thread per rank polls its own buffer's slot [k & 1][r] until the word
//     carries k, and the sums are added in rank order. Every rank therefore computes
//     the same value, bit for bit, whatever the timing;
//   * two rows suffice: a rank can only start call k + 2 (reusing row k & 1) after it
//     has read every rank's call-(k + 1) word, which each rank writes only after it
//     has read its call-k words;
//   * each poll is bounded (kWaitLimitNs): a rank that never arrives makes the others
//     set kErrTimeout in the device error word, write NaN and set the sticky flag.
//     Once the flag is set the ranks are out of step for good, so every later call
//     writes NaN and sets kErrTimeout at once instead of waiting again;
//     kpb_peer_sum_status reads the flag.
// There are no multicast loads and no memory of another GPU is given to TMA.
#include <cstring>

#include "kp_common.cuh"
#include "kp_sm100.cuh"

namespace kpb {

int reduce_level1_persistent(int dtype, const void* x, int64_t n, float* partials,
                             int64_t* ctas, cudaStream_t s);
size_t reduce_workspace_bytes(int variant, int64_t n);
int device_error_word(unsigned** out);

namespace {

constexpr int kPeerMax = 8;                      // GPUs of one node
constexpr int kPeerFinishThreads = 1024;
// words 0 .. 2*kPeerMax-1: the two exchange rows; then the local control words
constexpr int kCtlSeq = 2 * kPeerMax;            // last call number this rank ran
constexpr int kCtlBroken = 2 * kPeerMax + 1;     // non-zero once a wait gave up
constexpr size_t kExchangeBytes = 32 * sizeof(unsigned long long);
static_assert(kCtlBroken < 32, "control words fit the exchange buffer");

struct PeerSlots {
  unsigned long long* buf[kPeerMax];             // each rank's exchange buffer, mapped here
};

__device__ __forceinline__ void st_release_sys_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" :: "l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_acquire_sys_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__global__ void __launch_bounds__(kPeerFinishThreads)
sum_finish_peers(const float* __restrict__ partials, int64_t count, float* __restrict__ out,
                 PeerSlots slots, int rank, int world, unsigned* err) {
  __shared__ float scratch[kWarp];
  __shared__ float vals[kPeerMax];
  __shared__ int all_ok;
  __shared__ unsigned call;
  __shared__ int broken;
  pdl_wait_primary();
  unsigned long long* own = slots.buf[rank];
  if (threadIdx.x == 0) {
    // only this rank's finishing kernels touch its control words, one after the
    // other in stream order, so plain accesses suffice
    unsigned k = static_cast<unsigned>(own[kCtlSeq]) + 1u;
    if (k == 0) k = 1;  // 0 marks a slot never written
    own[kCtlSeq] = k;
    call = k;
    broken = own[kCtlBroken] != 0;
    all_ok = 1;
  }
  float s = 0.f;
  for (int64_t i = threadIdx.x; i < count; i += kPeerFinishThreads) s += partials[i];
  s = block_reduce<false>(s, scratch);  // every thread holds the CTA sum (and sees call)
  const unsigned seq = call;
  if (broken) {
    if (threadIdx.x == 0) {
      atomicOr(err, kErrTimeout);
      out[0] = __int_as_float(0x7fc00000);
    }
    return;
  }
  const int row = static_cast<int>(seq & 1u) * kPeerMax;
  const unsigned long long word =
      (static_cast<unsigned long long>(seq) << 32) | __float_as_uint(s);
  // publish this rank's partial to every rank (itself included)
  if (threadIdx.x < world) st_release_sys_u64(slots.buf[threadIdx.x] + row + rank, word);
  __syncthreads();
  // collect every rank's partial of this call from the own buffer
  if (threadIdx.x < world) {
    const unsigned long long* slot = own + row + threadIdx.x;
    unsigned long long v = ld_acquire_sys_u64(slot);
    if (static_cast<unsigned>(v >> 32) != seq) {
      const uint64_t t0 = global_timer_ns();
      while (true) {
#pragma unroll 1
        for (int i = 0; i < 32 && static_cast<unsigned>(v >> 32) != seq; ++i)
          v = ld_acquire_sys_u64(slot);
        if (static_cast<unsigned>(v >> 32) == seq) break;
        if (global_timer_ns() - t0 > kWaitLimitNs) {
          atomicOr(err, kErrTimeout);
          all_ok = 0;
          break;
        }
      }
    }
    vals[threadIdx.x] = __uint_as_float(static_cast<unsigned>(v));
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float total = 0.f;
    for (int r = 0; r < world; ++r) total += vals[r];  // rank order: the same on every rank
    out[0] = all_ok ? total : __int_as_float(0x7fc00000);
    if (!all_ok) own[kCtlBroken] = 1;
  }
}

}  // namespace
}  // namespace kpb

struct kpb_peer_sum {
  int rank = 0, world = 0, device = -1;
  unsigned long long* local = nullptr;
  unsigned long long* peer[kpb::kPeerMax] = {};
  bool opened[kpb::kPeerMax] = {};
  bool connected = false;
};

extern "C" {

int kpb_peer_sum_create(int rank, int world, void* ipc_handle_out, kpb_peer_sum** out) {
  using namespace kpb;
  set_error("");
  if (out == nullptr || ipc_handle_out == nullptr)
    return fail(KPB_EINVAL, "peer_sum_create: null pointer");
  *out = nullptr;
  if (world < 1 || world > kPeerMax || rank < 0 || rank >= world)
    return fail(KPB_EINVAL, "peer_sum_create: need 1 <= world <= " + std::to_string(kPeerMax) +
                                " and 0 <= rank < world (got rank " + std::to_string(rank) +
                                ", world " + std::to_string(world) + ")");
  auto* ps = new kpb_peer_sum();
  ps->rank = rank;
  ps->world = world;
  cudaError_t e = cudaGetDevice(&ps->device);
  if (e == cudaSuccess) e = cudaMalloc(reinterpret_cast<void**>(&ps->local), kExchangeBytes);
  if (e == cudaSuccess) e = cudaMemset(ps->local, 0, kExchangeBytes);
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, ps->local);
  if (e != cudaSuccess) {
    if (ps->local) cudaFree(ps->local);
    delete ps;
    return cuda_fail(e, "peer_sum_create", __FILE__, __LINE__);
  }
  std::memcpy(ipc_handle_out, &h, sizeof(h));
  *out = ps;
  return KPB_OK;
}

size_t kpb_peer_sum_handle_bytes(void) { return sizeof(cudaIpcMemHandle_t); }

int kpb_peer_sum_connect(kpb_peer_sum* ps, const void* all_handles) {
  using namespace kpb;
  set_error("");
  if (ps == nullptr || all_handles == nullptr)
    return fail(KPB_EINVAL, "peer_sum_connect: null pointer");
  if (ps->connected) return fail(KPB_EINVAL, "peer_sum_connect: already connected");
  const auto* handles = static_cast<const cudaIpcMemHandle_t*>(all_handles);
  for (int r = 0; r < ps->world; ++r) {
    if (r == ps->rank) {
      ps->peer[r] = ps->local;
      continue;
    }
    void* p = nullptr;
    const cudaError_t e = cudaIpcOpenMemHandle(&p, handles[r], cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return cuda_fail(e, "peer_sum_connect (cudaIpcOpenMemHandle)", __FILE__, __LINE__);
    ps->peer[r] = static_cast<unsigned long long*>(p);
    ps->opened[r] = true;
  }
  ps->connected = true;
  return KPB_OK;
}

size_t kpb_peer_sum_workspace_bytes(int64_t n) {
  return n > 0 ? kpb::reduce_workspace_bytes(2, n) : 0;
}

int kpb_peer_sum_run(kpb_peer_sum* ps, int dtype, const void* x, float* out, int64_t n,
                     void* workspace, size_t workspace_bytes, void* stream) {
  using namespace kpb;
  set_error("");
  if (ps == nullptr || out == nullptr || (n > 0 && x == nullptr))
    return fail(KPB_EINVAL, "peer_sum_run: null pointer");
  if (!ps->connected) return fail(KPB_EINVAL, "peer_sum_run: call kpb_peer_sum_connect first");
  if (dtype != KPB_F32 && dtype != KPB_F16 && dtype != KPB_BF16)
    return fail(KPB_EINVAL, "peer_sum_run: dtype must be 0 (f32), 1 (f16) or 2 (bf16)");
  if (n < 0) return fail(KPB_EINVAL, "peer_sum_run: n must be >= 0");
  const size_t need = kpb_peer_sum_workspace_bytes(n);
  if (need > 0 && (workspace == nullptr || workspace_bytes < need ||
                   reinterpret_cast<uintptr_t>(workspace) % 4 != 0))
    return fail(KPB_EINVAL, "peer_sum_run: workspace missing, misaligned or smaller than " +
                                std::to_string(need) + " bytes");
  int dev = -1;
  KPB_CUDA(cudaGetDevice(&dev));
  if (dev != ps->device)
    return fail(KPB_EINVAL, "peer_sum_run: current device differs from the one it was created on");
  unsigned* err = nullptr;
  if (int rc = device_error_word(&err)) return rc;
  auto s = static_cast<cudaStream_t>(stream);
  float* partials = static_cast<float*>(workspace);
  int64_t ctas = 0;
  if (n > 0) {
    if (int rc = reduce_level1_persistent(dtype, x, n, partials, &ctas, s)) return rc;
  }
  PeerSlots slots{};
  for (int r = 0; r < ps->world; ++r) slots.buf[r] = ps->peer[r];
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(1);
  cfg.blockDim = dim3(kPeerFinishThreads);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = n > 0 ? 1 : 0;
  KPB_CUDA(cudaLaunchKernelEx(&cfg, sum_finish_peers, static_cast<const float*>(partials), ctas,
                              out, slots, ps->rank, ps->world, err));
  return KPB_OK;
}

int kpb_peer_sum_status(kpb_peer_sum* ps, int* out_of_step) {
  using namespace kpb;
  set_error("");
  if (ps == nullptr || out_of_step == nullptr)
    return fail(KPB_EINVAL, "peer_sum_status: null pointer");
  int dev = -1;
  KPB_CUDA(cudaGetDevice(&dev));
  if (dev != ps->device)
    return fail(KPB_EINVAL, "peer_sum_status: current device differs from the one it was created on");
  unsigned long long flag = 0;
  KPB_CUDA(cudaDeviceSynchronize());
  KPB_CUDA(cudaMemcpy(&flag, ps->local + kCtlBroken, sizeof(flag), cudaMemcpyDeviceToHost));
  *out_of_step = flag != 0;
  return KPB_OK;
}

int kpb_peer_sum_destroy(kpb_peer_sum* ps) {
  using namespace kpb;
  set_error("");
  if (ps == nullptr) return KPB_OK;
  int rc = KPB_OK;
  for (int r = 0; r < kPeerMax; ++r)
    if (ps->opened[r] && cudaIpcCloseMemHandle(ps->peer[r]) != cudaSuccess) rc = KPB_ECUDA;
  if (ps->local && cudaFree(ps->local) != cudaSuccess) rc = KPB_ECUDA;
  delete ps;
  if (rc) set_error("peer_sum_destroy: a CUDA release call failed");
  return rc;
}

}  // extern "C"
