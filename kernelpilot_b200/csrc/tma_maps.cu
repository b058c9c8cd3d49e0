// TMA tensor maps (cuTensorMapEncodeTiled, fetched from the driver at run time so the
// library loads on machines without a GPU driver).
#include <cudaTypedefs.h>

#include <mutex>

#include "kp_common.cuh"

namespace kpb {
namespace {

PFN_cuTensorMapEncodeTiled_v12000 tmap_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault,
                                         &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

int encode(CUtensorMap* map, bool bf16, int rank, const void* base, const cuuint64_t* dims,
           const cuuint64_t* strides, const cuuint32_t* box) {
  auto enc = tmap_encoder();
  if (!enc) return fail(KPB_ECUDA, "cuTensorMapEncodeTiled is not available from the driver");
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = enc(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                         rank, const_cast<void*>(base), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(KPB_ECUDA, "cuTensorMapEncodeTiled failed: " + std::to_string(r));
  return KPB_OK;
}

}  // namespace

// Row-major (outer x inner) 16-bit matrix, boxes of (box_outer rows x 64 elements),
// 128-byte swizzle; elements outside the matrix read as zero.
int make_tmap_2d_sw128(CUtensorMap* map, const void* base, bool bf16, uint64_t inner,
                       uint64_t outer, uint64_t pitch_bytes, uint32_t box_outer) {
  const cuuint64_t dims[2] = {inner, outer};
  const cuuint64_t strides[1] = {pitch_bytes};
  const cuuint32_t box[2] = {64, box_outer};
  return encode(map, bf16, 2, base, dims, strides, box);
}

// Contiguous (BH, S, D) 16-bit tensor as a 3-D map (D, S, BH) with (64 x box_rows x 1)
// boxes and 128-byte swizzle: rows past S of one head read as zero, never as the next
// head's rows.
int make_tmap_bhsd(CUtensorMap* map, const void* base, bool bf16, int64_t BH, int64_t S,
                   int64_t D, uint32_t box_rows) {
  const cuuint64_t dims[3] = {static_cast<cuuint64_t>(D), static_cast<cuuint64_t>(S),
                              static_cast<cuuint64_t>(BH)};
  const cuuint64_t strides[2] = {static_cast<cuuint64_t>(D * 2), static_cast<cuuint64_t>(S * D * 2)};
  const cuuint32_t box[3] = {64, box_rows, 1};
  return encode(map, bf16, 3, base, dims, strides, box);
}

}  // namespace kpb
