// The extern "C" boundary (include/kp_b200.h): argument validation, status codes,
// per-thread error messages, stream-ordered scratch from a pool of its own, and the
// per-device error word that bounded waits inside kernels report timeouts to.
#include <map>
#include <mutex>
#include <string>
#include <tuple>

#include "kp_common.cuh"

namespace kpb {

// implemented by the kernel translation units
size_t reduce_workspace_bytes(int variant, int64_t n);
int reduce_sum(int variant, int dtype, const void* x, float* out, int64_t n, void* ws,
               size_t ws_bytes, cudaStream_t s);
int softmax(int variant, int dtype, const void* x, void* y, int64_t M, int64_t N,
            unsigned* err, cudaStream_t s);
size_t matmul_workspace_bytes(int variant, int dtype, int64_t M, int64_t N, int64_t K);
int matmul(int variant, int dtype, const void* A, const void* B, void* C, int64_t M, int64_t N,
           int64_t K, void* ws, size_t ws_bytes, unsigned* err, cudaStream_t s);
int vector_add(int variant, int dtype, const void* a, const void* b, void* c, int64_t n,
               cudaStream_t s);
int layernorm(int variant, int dtype, const void* x, const void* w, const void* b, void* y,
              int64_t M, int64_t N, float eps, cudaStream_t s);
int attention(int variant, int dtype, bool causal, const void* q, const void* k, const void* v,
              void* o, int64_t BH, int64_t S, int64_t D, unsigned* err, cudaStream_t s);

namespace {
thread_local std::string g_last_error;

constexpr int kMaxDevices = 64;
std::mutex g_mu;
int g_sms[kMaxDevices] = {0};
unsigned* g_err_ptr[kMaxDevices] = {nullptr};

// Set by kernels whose bounded waits gave up (kErrTimeout); read by kpb_device_errors.
__device__ unsigned g_device_error_word = 0;
}  // namespace

void set_error(const std::string& msg) { g_last_error = msg; }

int fail(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

int cuda_fail(cudaError_t err, const char* what, const char* file, int line) {
  g_last_error = std::string("CUDA error ") + cudaGetErrorName(err) + " (" +
                 cudaGetErrorString(err) + ") in " + what + " at " + file + ":" +
                 std::to_string(line);
  return KPB_ECUDA;
}

int sm_count() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return 148;
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_sms[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    g_sms[dev] = n;
  }
  return g_sms[dev];
}

// Scratch of the allocating entry points comes from a stream-ordered pool per device
// owned by this library, which keeps its memory between calls (release threshold
// unlimited). The device's default pool returns its memory at every synchronisation,
// so the next call would map it again on the host after the GPU had already reached
// the call, and the GPU would wait for it.
namespace {
cudaMemPool_t g_pool[kMaxDevices] = {};
}  // namespace

int scratch_alloc(void** p, size_t bytes, cudaStream_t s) {
  int dev = 0;
  KPB_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) return fail(KPB_EUNSUPPORTED, "device index out of range");
  cudaMemPool_t pool = nullptr;
  {
    std::lock_guard<std::mutex> lk(g_mu);
    if (g_pool[dev] == nullptr) {
      cudaMemPoolProps props = {};
      props.allocType = cudaMemAllocationTypePinned;
      props.location.type = cudaMemLocationTypeDevice;
      props.location.id = dev;
      cudaMemPool_t created = nullptr;
      KPB_CUDA(cudaMemPoolCreate(&created, &props));
      uint64_t keep = UINT64_MAX;
      const cudaError_t e = cudaMemPoolSetAttribute(created, cudaMemPoolAttrReleaseThreshold, &keep);
      if (e != cudaSuccess) {
        cudaMemPoolDestroy(created);
        return cuda_fail(e, "cudaMemPoolSetAttribute", __FILE__, __LINE__);
      }
      g_pool[dev] = created;
    }
    pool = g_pool[dev];
  }
  KPB_CUDA(cudaMallocFromPoolAsync(p, bytes, pool, s));
  return KPB_OK;
}

// Launch facts of a kernel that do not change within a process, per device: the
// dynamic shared-memory opt-in is only raised when a launch needs more, and each
// occupancy answer is queried once for its block size, shared memory and cluster size
// (a whole launch call then costs 6-15 us of host time, with or without the cache).
namespace {
enum class Fact { kSmemOptIn, kBlocksPerSm, kClusters };
// (device, kernel, fact, threads, dynamic shared memory, cluster size)
using LaunchKey = std::tuple<int, const void*, Fact, int, size_t, int>;
std::map<LaunchKey, int> g_launch_facts;

int current_device(int* dev) {
  KPB_CUDA(cudaGetDevice(dev));
  return KPB_OK;
}
}  // namespace

// The opt-in is one value per kernel and device, and a launch may use any amount up
// to it: it is only ever raised, to the largest amount asked for so far.
int ensure_dyn_smem(const void* func, int bytes) {
  int dev = 0;
  if (int rc = current_device(&dev)) return rc;
  const LaunchKey key{dev, func, Fact::kSmemOptIn, 0, 0, 0};
  std::lock_guard<std::mutex> lk(g_mu);
  auto it = g_launch_facts.find(key);
  if (it != g_launch_facts.end() && it->second >= bytes) return KPB_OK;
  KPB_CUDA(cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
  g_launch_facts[key] = bytes;
  return KPB_OK;
}

int occupancy_blocks(const void* func, int threads, size_t smem, int* out) {
  int dev = 0;
  if (int rc = current_device(&dev)) return rc;
  const LaunchKey key{dev, func, Fact::kBlocksPerSm, threads, smem, 0};
  std::lock_guard<std::mutex> lk(g_mu);
  auto it = g_launch_facts.find(key);
  if (it == g_launch_facts.end()) {
    int occ = 0;
    KPB_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, func, threads, smem));
    it = g_launch_facts.emplace(key, occ).first;
  }
  *out = it->second;
  return KPB_OK;
}

int occupancy_clusters(const void* func, const cudaLaunchConfig_t& cfg, int cluster, int* out) {
  int dev = 0;
  if (int rc = current_device(&dev)) return rc;
  const LaunchKey key{dev, func, Fact::kClusters, static_cast<int>(cfg.blockDim.x),
                      cfg.dynamicSmemBytes, cluster};
  std::lock_guard<std::mutex> lk(g_mu);
  auto it = g_launch_facts.find(key);
  if (it == g_launch_facts.end()) {
    int active = 0;
    KPB_CUDA(cudaOccupancyMaxActiveClusters(&active, func, &cfg));
    it = g_launch_facts.emplace(key, active).first;
  }
  *out = it->second;
  return KPB_OK;
}

// Device address of this device's error word (looked up once per device).
int device_error_word(unsigned** out) {
  int dev = 0;
  KPB_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) return fail(KPB_EUNSUPPORTED, "device index out of range");
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_err_ptr[dev] == nullptr) {
    void* p = nullptr;
    KPB_CUDA(cudaGetSymbolAddress(&p, g_device_error_word));
    g_err_ptr[dev] = static_cast<unsigned*>(p);
  }
  *out = g_err_ptr[dev];
  return KPB_OK;
}

static bool valid_dtype(int dt) { return dt == KPB_F32 || dt == KPB_F16 || dt == KPB_BF16; }

static int check_common(const char* op, int variant, int dtype) {
  const int nv = kpb_num_variants(op);
  if (variant < 0 || variant >= nv)
    return fail(KPB_EINVAL, std::string(op) + ": variant must be in [0, " + std::to_string(nv) +
                                ")");
  if (!valid_dtype(dtype))
    return fail(KPB_EINVAL, std::string(op) + ": dtype must be 0 (f32), 1 (f16) or 2 (bf16)");
  return KPB_OK;
}

static size_t elem_bytes(int dtype) { return dtype == KPB_F32 ? 4 : 2; }

}  // namespace kpb

using namespace kpb;

extern "C" {

const char* kpb_last_error(void) { return g_last_error.c_str(); }

int kpb_version(void) { return 100; }

int kpb_num_variants(const char* op) {
  if (op == nullptr) return -1;
  const std::string s(op);
  if (s == "vector_add" || s == "reduce_sum" || s == "softmax" || s == "layernorm") return 3;
  if (s == "matmul") return 4;
  if (s == "attention" || s == "attention_causal") return 2;
  return -1;
}

int kpb_device_errors(unsigned* bits) {
  g_last_error.clear();
  unsigned v = 0, zero = 0;
  KPB_CUDA(cudaMemcpyFromSymbol(&v, g_device_error_word, sizeof(v)));
  KPB_CUDA(cudaMemcpyToSymbol(g_device_error_word, &zero, sizeof(zero)));
  if (bits) *bits = v;
  return KPB_OK;
}

int kpb_vector_add(int variant, int dtype, const void* a, const void* b, void* c, int64_t n,
                   void* stream) {
  g_last_error.clear();
  if (int rc = check_common("vector_add", variant, dtype)) return rc;
  if (n < 0) return fail(KPB_EINVAL, "vector_add: n must be >= 0");
  if (n > 0 && (a == nullptr || b == nullptr || c == nullptr))
    return fail(KPB_EINVAL, "vector_add: null pointer");
  return vector_add(variant, dtype, a, b, c, n, static_cast<cudaStream_t>(stream));
}

size_t kpb_reduce_sum_workspace_bytes(int variant, int64_t n) {
  return reduce_workspace_bytes(variant, n);
}

int kpb_reduce_sum_ws(int variant, int dtype, const void* x, float* out, int64_t n,
                      void* workspace, size_t workspace_bytes, void* stream) {
  g_last_error.clear();
  if (int rc = check_common("reduce_sum", variant, dtype)) return rc;
  if (n < 0) return fail(KPB_EINVAL, "reduce_sum: n must be >= 0");
  if (out == nullptr || (n > 0 && x == nullptr))
    return fail(KPB_EINVAL, "reduce_sum: null pointer");
  return reduce_sum(variant, dtype, x, out, n, workspace, workspace_bytes,
                    static_cast<cudaStream_t>(stream));
}

int kpb_reduce_sum(int variant, int dtype, const void* x, float* out, int64_t n, void* stream) {
  g_last_error.clear();
  if (int rc = check_common("reduce_sum", variant, dtype)) return rc;
  if (n < 0) return fail(KPB_EINVAL, "reduce_sum: n must be >= 0");
  if (out == nullptr || (n > 0 && x == nullptr))
    return fail(KPB_EINVAL, "reduce_sum: null pointer");
  auto s = static_cast<cudaStream_t>(stream);
  const size_t bytes = reduce_workspace_bytes(variant, n);
  void* ws = nullptr;
  if (bytes) {
    if (int rc = scratch_alloc(&ws, bytes, s)) return rc;
  }
  const int rc = reduce_sum(variant, dtype, x, out, n, ws, bytes, s);
  if (ws) {
    const cudaError_t e = cudaFreeAsync(ws, s);
    if (rc == KPB_OK && e != cudaSuccess) return cuda_fail(e, "cudaFreeAsync", __FILE__, __LINE__);
  }
  return rc;
}

int kpb_softmax(int variant, int dtype, const void* x, void* y, int64_t M, int64_t N,
                void* stream) {
  g_last_error.clear();
  if (int rc = check_common("softmax", variant, dtype)) return rc;
  if (M < 0 || N < 0 || M >= (int64_t{1} << 31) || N >= (int64_t{1} << 31))
    return fail(KPB_EINVAL, "softmax: M and N must be in [0, 2^31)");
  if (M * N > 0 && (x == nullptr || y == nullptr)) return fail(KPB_EINVAL, "softmax: null pointer");
  unsigned* err = nullptr;
  if (int rc = device_error_word(&err)) return rc;
  return softmax(variant, dtype, x, y, M, N, err, static_cast<cudaStream_t>(stream));
}

int kpb_layernorm(int variant, int dtype, const void* x, const void* w, const void* b, void* y,
                  int64_t M, int64_t N, float eps, void* stream) {
  g_last_error.clear();
  if (int rc = check_common("layernorm", variant, dtype)) return rc;
  if (M < 0 || N < 0 || M >= (int64_t{1} << 31) || N >= (int64_t{1} << 31))
    return fail(KPB_EINVAL, "layernorm: M and N must be in [0, 2^31)");
  if (M * N > 0 && (x == nullptr || w == nullptr || b == nullptr || y == nullptr))
    return fail(KPB_EINVAL, "layernorm: null pointer");
  return layernorm(variant, dtype, x, w, b, y, M, N, eps, static_cast<cudaStream_t>(stream));
}

size_t kpb_matmul_workspace_bytes(int variant, int dtype, int64_t M, int64_t N, int64_t K) {
  if (!valid_dtype(dtype) || M < 0 || N < 0 || K < 0) return 0;
  return matmul_workspace_bytes(variant, dtype, M, N, K);
}

int kpb_matmul_ws(int variant, int dtype, const void* A, const void* B, void* C, int64_t M,
                  int64_t N, int64_t K, void* workspace, size_t workspace_bytes, void* stream) {
  g_last_error.clear();
  if (int rc = check_common("matmul", variant, dtype)) return rc;
  const int64_t lim = int64_t{1} << 31;
  if (M < 0 || N < 0 || K < 0 || M >= lim || N >= lim || K >= lim)
    return fail(KPB_EINVAL, "matmul: M, N, K must be in [0, 2^31)");
  if (M * N > 0 && (C == nullptr || (K > 0 && (A == nullptr || B == nullptr))))
    return fail(KPB_EINVAL, "matmul: null pointer");
  auto s = static_cast<cudaStream_t>(stream);
  if (M == 0 || N == 0) return KPB_OK;
  if (K == 0) {
    KPB_CUDA(cudaMemsetAsync(C, 0, static_cast<size_t>(M * N) * elem_bytes(dtype), s));
    return KPB_OK;
  }
  unsigned* err = nullptr;
  if (int rc = device_error_word(&err)) return rc;
  return matmul(variant, dtype, A, B, C, M, N, K, workspace, workspace_bytes, err, s);
}

int kpb_matmul(int variant, int dtype, const void* A, const void* B, void* C, int64_t M,
               int64_t N, int64_t K, void* stream) {
  g_last_error.clear();
  if (int rc = check_common("matmul", variant, dtype)) return rc;
  if (M < 0 || N < 0 || K < 0) return fail(KPB_EINVAL, "matmul: negative size");
  auto s = static_cast<cudaStream_t>(stream);
  const size_t bytes = matmul_workspace_bytes(variant, dtype, M, N, K);
  void* ws = nullptr;
  if (bytes) {
    if (int rc = scratch_alloc(&ws, bytes, s)) return rc;
  }
  const int rc = kpb_matmul_ws(variant, dtype, A, B, C, M, N, K, ws, bytes, stream);
  if (ws) {
    const std::string msg = g_last_error;
    const cudaError_t e = cudaFreeAsync(ws, s);
    if (rc == KPB_OK && e != cudaSuccess) return cuda_fail(e, "cudaFreeAsync", __FILE__, __LINE__);
    g_last_error = msg;
  }
  return rc;
}

static int attention_entry(const char* op, bool causal, int variant, int dtype, const void* q,
                           const void* k, const void* v, void* o, int64_t BH, int64_t S,
                           int64_t D, void* stream) {
  g_last_error.clear();
  if (int rc = check_common(op, variant, dtype)) return rc;
  if (BH < 0 || S < 0 || D < 0) return fail(KPB_EINVAL, std::string(op) + ": negative size");
  if (D > 256 || BH >= 65536)
    return fail(KPB_EINVAL, std::string(op) + ": supports D <= 256 and B*H < 65536");
  if (S >= (int64_t{1} << 31)) return fail(KPB_EINVAL, std::string(op) + ": S too large");
  if (BH * S * D > 0 && (!q || !k || !v || !o))
    return fail(KPB_EINVAL, std::string(op) + ": null pointer");
  if (BH == 0 || S == 0 || D == 0) return KPB_OK;
  unsigned* err = nullptr;
  if (int rc = device_error_word(&err)) return rc;
  return attention(variant, dtype, causal, q, k, v, o, BH, S, D, err,
                   static_cast<cudaStream_t>(stream));
}

int kpb_attention(int variant, int dtype, const void* q, const void* k, const void* v, void* o,
                  int64_t BH, int64_t S, int64_t D, void* stream) {
  return attention_entry("attention", false, variant, dtype, q, k, v, o, BH, S, D, stream);
}

int kpb_attention_causal(int variant, int dtype, const void* q, const void* k, const void* v,
                         void* o, int64_t BH, int64_t S, int64_t D, void* stream) {
  return attention_entry("attention_causal", true, variant, dtype, q, k, v, o, BH, S, D, stream);
}

}  // extern "C"
