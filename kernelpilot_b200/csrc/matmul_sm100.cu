// tcgen05 GEMM for kp.matmul variant 3 (fp16/bf16).
#include "kp_common.cuh"

namespace kpb {

size_t matmul_tc_workspace_bytes(int, int64_t, int64_t, int64_t) { return 0; }

int matmul_tc(int, const void*, const void*, void*, int64_t, int64_t, int64_t, void*, size_t,
              unsigned*, cudaStream_t) {
  return KPB_EUNSUPPORTED;
}

}  // namespace kpb
