// torch.ops.kp.* on top of the C ABI in include/kp_b200.h.
//
// Same operator schemas and checks as kernelpilot's csrc/bindings.cpp:118-134
// (inputs on the GPU and contiguous :25-28, matching shapes/dtypes :38/:71/:88-90/:106,
// size limits :60/:73/:93/:109, variant ranges :30-33/:77/:111, launch on the current
// stream :12-17,
// fresh outputs from the caching allocator). Additions: bf16 inputs (dtype_of,
// :19-23, accepted float32/float16 only) and the attention_causal operator.
// Errors surface as c10::Error (Python RuntimeError) carrying kpb_last_error().
//
// Scratch (reduction partials, the aligned copy of B for odd N) comes from the
// caching allocator on the op's stream, so concurrent calls on different streams
// never share it.
#include <ATen/ATen.h>
#include <c10/core/impl/DeviceGuardImplInterface.h>
#include <torch/library.h>

#include "kp_b200.h"

namespace {

void* current_stream(const at::Tensor& t) {
  auto impl = c10::impl::getDeviceGuardImpl(t.device().type());
  return impl->getStream(t.device()).native_handle();
}

int dtype_of(const at::Tensor& t) {
  switch (t.scalar_type()) {
    case at::kFloat: return KPB_F32;
    case at::kHalf: return KPB_F16;
    case at::kBFloat16: return KPB_BF16;
    default:
      TORCH_CHECK(false, "kernelpilot kernels support float32, float16 and bfloat16, got ",
                  t.scalar_type());
  }
}

void check_input(const at::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda(), name, " must be a GPU tensor");
  TORCH_CHECK(t.is_contiguous(), name, " must be contiguous");
}

int64_t check_variant(const char* op, int64_t v) {
  const int64_t n = kpb_num_variants(op);
  TORCH_CHECK(v >= 0 && v < n, "variant must be in [0, ", n, ")");
  return v;
}

void check_rc(int rc, const char* op) {
  TORCH_CHECK(rc == KPB_OK, "kp.", op, " failed (status ", rc, "): ", kpb_last_error());
}

// Scratch bytes from the caching allocator, stream-ordered with the op.
at::Tensor scratch(const at::Tensor& like, size_t bytes) {
  return at::empty({static_cast<int64_t>(bytes > 0 ? bytes : 1)},
                   like.options().dtype(at::kByte));
}

at::Tensor vector_add(const at::Tensor& a, const at::Tensor& b, int64_t variant) {
  check_input(a, "a");
  check_input(b, "b");
  TORCH_CHECK(a.sizes() == b.sizes() && a.scalar_type() == b.scalar_type(),
              "a and b must match in shape and dtype");
  const int v = static_cast<int>(check_variant("vector_add", variant));
  auto c = at::empty_like(a);
  check_rc(kpb_vector_add(v, dtype_of(a), a.data_ptr(), b.data_ptr(), c.data_ptr(), a.numel(),
                          current_stream(a)),
           "vector_add");
  return c;
}

at::Tensor reduce_sum(const at::Tensor& x, int64_t variant) {
  check_input(x, "x");
  const int v = static_cast<int>(check_variant("reduce_sum", variant));
  const int dt = dtype_of(x);
  // kpb writes out[0] (no zero-init needed, unlike the reference's at::zeros)
  auto out = at::empty({}, x.options().dtype(at::kFloat));
  auto ws = scratch(x, kpb_reduce_sum_workspace_bytes(v, x.numel()));
  check_rc(kpb_reduce_sum_ws(v, dt, x.data_ptr(), out.data_ptr<float>(), x.numel(),
                             ws.data_ptr(), static_cast<size_t>(ws.numel()), current_stream(x)),
           "reduce_sum");
  return out;
}

at::Tensor softmax(const at::Tensor& x, int64_t variant) {
  check_input(x, "x");
  TORCH_CHECK(x.dim() >= 1, "softmax needs at least 1 dimension");
  const int v = static_cast<int>(check_variant("softmax", variant));
  auto y = at::empty_like(x);
  const int64_t N = x.size(-1);
  const int64_t M = N == 0 ? 0 : x.numel() / N;
  TORCH_CHECK(M < (int64_t{1} << 31) && N < (int64_t{1} << 31), "softmax shape too large");
  check_rc(kpb_softmax(v, dtype_of(x), x.data_ptr(), y.data_ptr(), M, N, current_stream(x)),
           "softmax");
  return y;
}

at::Tensor matmul(const at::Tensor& a, const at::Tensor& b, int64_t variant) {
  check_input(a, "a");
  check_input(b, "b");
  TORCH_CHECK(a.dim() == 2 && b.dim() == 2 && a.size(1) == b.size(0),
              "matmul expects (M, K) @ (K, N), got ", a.sizes(), " and ", b.sizes());
  TORCH_CHECK(a.scalar_type() == b.scalar_type(), "a and b must have the same dtype");
  const int v = static_cast<int>(check_variant("matmul", variant));
  const int64_t M = a.size(0), K = a.size(1), N = b.size(1);
  TORCH_CHECK(M < (int64_t{1} << 31) && N < (int64_t{1} << 31) && K < (int64_t{1} << 31),
              "matmul shape too large");
  const int dt = dtype_of(a);
  auto c = at::empty({M, N}, a.options());
  if (M == 0 || N == 0) return c;
  if (K == 0) return c.zero_();
  auto ws = scratch(a, kpb_matmul_workspace_bytes(v, dt, M, N, K));
  check_rc(kpb_matmul_ws(v, dt, a.data_ptr(), b.data_ptr(), c.data_ptr(), M, N, K,
                         ws.data_ptr(), static_cast<size_t>(ws.numel()), current_stream(a)),
           "matmul");
  return c;
}

at::Tensor layernorm(const at::Tensor& x, const at::Tensor& w, const at::Tensor& b, double eps,
                     int64_t variant) {
  check_input(x, "x");
  check_input(w, "weight");
  check_input(b, "bias");
  TORCH_CHECK(x.dim() >= 1, "layernorm needs at least 1 dimension");
  const int64_t N = x.size(-1);
  TORCH_CHECK(w.numel() == N && b.numel() == N, "weight and bias must have size ", N);
  TORCH_CHECK(w.scalar_type() == x.scalar_type() && b.scalar_type() == x.scalar_type(),
              "x, weight and bias must share a dtype");
  const int var = static_cast<int>(check_variant("layernorm", variant));
  auto y = at::empty_like(x);
  const int64_t M = N == 0 ? 0 : x.numel() / N;
  TORCH_CHECK(M < (int64_t{1} << 31) && N < (int64_t{1} << 31), "layernorm shape too large");
  check_rc(kpb_layernorm(var, dtype_of(x), x.data_ptr(), w.data_ptr(), b.data_ptr(), y.data_ptr(),
                         M, N, static_cast<float>(eps), current_stream(x)),
           "layernorm");
  return y;
}

at::Tensor attention_impl(const char* op, const at::Tensor& q, const at::Tensor& k,
                          const at::Tensor& v, int64_t variant) {
  check_input(q, "q");
  check_input(k, "k");
  check_input(v, "v");
  TORCH_CHECK(q.dim() == 4 && q.sizes() == k.sizes() && q.sizes() == v.sizes(),
              "q, k, v must all be (B, H, S, D)");
  TORCH_CHECK(q.scalar_type() == k.scalar_type() && q.scalar_type() == v.scalar_type(),
              "q, k, v must share a dtype");
  const int var = static_cast<int>(check_variant(op, variant));
  const int64_t BH = q.size(0) * q.size(1), S = q.size(2), D = q.size(3);
  TORCH_CHECK(D <= 256 && BH < 65536, "attention supports D <= 256 and B*H < 65536");
  auto o = at::empty_like(q);
  const int dt = dtype_of(q);
  const int rc = std::string(op) == "attention"
                     ? kpb_attention(var, dt, q.data_ptr(), k.data_ptr(), v.data_ptr(),
                                     o.data_ptr(), BH, S, D, current_stream(q))
                     : kpb_attention_causal(var, dt, q.data_ptr(), k.data_ptr(), v.data_ptr(),
                                            o.data_ptr(), BH, S, D, current_stream(q));
  check_rc(rc, op);
  return o;
}

at::Tensor attention(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                     int64_t variant) {
  return attention_impl("attention", q, k, v, variant);
}

at::Tensor attention_causal(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                            int64_t variant) {
  return attention_impl("attention_causal", q, k, v, variant);
}

}  // namespace

TORCH_LIBRARY(kp, m) {
  m.def("vector_add(Tensor a, Tensor b, int variant) -> Tensor");
  m.def("reduce_sum(Tensor x, int variant) -> Tensor");
  m.def("softmax(Tensor x, int variant) -> Tensor");
  m.def("matmul(Tensor a, Tensor b, int variant) -> Tensor");
  m.def("layernorm(Tensor x, Tensor weight, Tensor bias, float eps, int variant) -> Tensor");
  m.def("attention(Tensor q, Tensor k, Tensor v, int variant) -> Tensor");
  m.def("attention_causal(Tensor q, Tensor k, Tensor v, int variant) -> Tensor");
}

TORCH_LIBRARY_IMPL(kp, CUDA, m) {
  m.impl("vector_add", &vector_add);
  m.impl("reduce_sum", &reduce_sum);
  m.impl("softmax", &softmax);
  m.impl("matmul", &matmul);
  m.impl("layernorm", &layernorm);
  m.impl("attention", &attention);
  m.impl("attention_causal", &attention_causal);
}
