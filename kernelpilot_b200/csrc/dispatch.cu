// Variant/dtype routing for kp.matmul and kp.attention(_causal): the tensor-core
// (tcgen05) kernels take fp16/bf16 at the highest variant; everything else runs on
// the CUDA-core kernels.
#include "kp_common.cuh"

namespace kpb {

int matmul_simt(int variant, int dtype, const void* A, const void* B, void* C, int64_t M,
                int64_t N, int64_t K, cudaStream_t s);
int attention_simt(int variant, int dtype, bool causal, const void* q, const void* k,
                   const void* v, void* o, int64_t BH, int64_t S, int64_t D, cudaStream_t s);
// tensor-core paths; return KPB_EUNSUPPORTED for shapes they do not take
size_t matmul_tc_workspace_bytes(int dtype, int64_t M, int64_t N, int64_t K);
int matmul_tc(int dtype, const void* A, const void* B, void* C, int64_t M, int64_t N, int64_t K,
              void* ws, size_t ws_bytes, unsigned* err, cudaStream_t s);
int attention_tc(int dtype, bool causal, const void* q, const void* k, const void* v, void* o,
                 int64_t BH, int64_t S, int64_t D, unsigned* err, cudaStream_t s);

size_t matmul_workspace_bytes(int variant, int dtype, int64_t M, int64_t N, int64_t K) {
  if (variant != 3 || dtype == KPB_F32) return 0;
  return matmul_tc_workspace_bytes(dtype, M, N, K);
}

int matmul(int variant, int dtype, const void* A, const void* B, void* C, int64_t M, int64_t N,
           int64_t K, void* ws, size_t ws_bytes, unsigned* err, cudaStream_t s) {
  if (variant == 3 && dtype != KPB_F32) {
    const int rc = matmul_tc(dtype, A, B, C, M, N, K, ws, ws_bytes, err, s);
    if (rc != KPB_EUNSUPPORTED) return rc;
  }
  return matmul_simt(variant, dtype, A, B, C, M, N, K, s);
}

int attention(int variant, int dtype, bool causal, const void* q, const void* k, const void* v,
              void* o, int64_t BH, int64_t S, int64_t D, unsigned* err, cudaStream_t s) {
  if (variant == 1 && dtype != KPB_F32) {
    const int rc = attention_tc(dtype, causal, q, k, v, o, BH, S, D, err, s);
    if (rc != KPB_EUNSUPPORTED) return rc;
  }
  return attention_simt(variant, dtype, causal, q, k, v, o, BH, S, D, s);
}

}  // namespace kpb
