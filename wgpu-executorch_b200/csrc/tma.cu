// Tensor-map encoding through the driver entry point (no link-time
// dependency on libcuda).
#include <cudaTypedefs.h>

#include "tma.h"

namespace wgx {

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    check_cuda(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q),
               "cuTensorMapEncodeTiled entry point");
    if (q != cudaDriverEntryPointSuccess || !p) fail("cuTensorMapEncodeTiled is unavailable");
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

void encode_nchw_tmap(CUtensorMap *map, const void *base, int B, int C, int HW, int box_c) {
  if ((reinterpret_cast<uintptr_t>(base) & 15) || HW % 8 || box_c < 1 || box_c > 256)
    fail("conv2d: tensor map needs a 16-byte aligned base and HW % 8 == 0");
  const cuuint64_t dims[3] = {cuuint64_t(HW), cuuint64_t(C), cuuint64_t(B)};
  const cuuint64_t strides[2] = {cuuint64_t(HW) * 2, cuuint64_t(C) * HW * 2};
  const cuuint32_t box[3] = {64, cuuint32_t(box_c), 1};
  const cuuint32_t estride[3] = {1, 1, 1};
  const CUresult r = encode_fn()(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void *>(base),
                                 dims, strides, box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                 CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                 CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) fail("conv2d: cuTensorMapEncodeTiled failed (" + std::to_string(int(r)) + ")");
}

}  // namespace wgx
