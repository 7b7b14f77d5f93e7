// Host-side tensor-map encoding through the driver entry point (no link-time
// dependency on libcuda: the library loads on machines without a GPU driver).
#include <mutex>

#include "pmoe_tma.cuh"

namespace pmoe {

namespace {
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
std::once_flag g_once;
EncodeTiledFn g_encode = nullptr;

void resolve() {
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) ==
          cudaSuccess &&
      q == cudaDriverEntryPointSuccess)
    g_encode = reinterpret_cast<EncodeTiledFn>(fn);
}
}  // namespace

bool make_tmap_bf16_2d(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer,
                       uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer,
                       bool swizzle128) {
  std::call_once(g_once, resolve);
  if (!g_encode) return false;
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0 || row_stride_bytes % 16 != 0) return false;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims,
                        strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

bool make_tmap_bf16_nd(CUtensorMap* map, const void* base, int rank, const uint64_t* dims,
                       const uint64_t* stride_bytes, const uint32_t* box) {
  std::call_once(g_once, resolve);
  if (!g_encode || rank < 1 || rank > 5) return false;
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0) return false;
  cuuint64_t d[5], st[4];
  cuuint32_t b[5], estr[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    b[i] = box[i];
    estr[i] = 1;
    if (i > 0) {
      if (stride_bytes[i - 1] % 16 != 0) return false;
      st[i - 1] = stride_bytes[i - 1];
    }
  }
  CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, rank, const_cast<void*>(base), d,
                        st, b, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

}  // namespace pmoe
