// tcgen05 flash attention for kp.attention(_causal) variant 1 (fp16/bf16).
#include "kp_common.cuh"

namespace kpb {

int attention_tc(int, bool, const void*, const void*, const void*, void*, int64_t, int64_t,
                 int64_t, unsigned*, cudaStream_t) {
  return KPB_EUNSUPPORTED;
}

}  // namespace kpb
