#include "tma.h"

#include <mutex>
#include <string>

namespace sana {
namespace {

using EncodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                 const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiled encoder() {
    static EncodeTiled fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess) {
            fn = reinterpret_cast<EncodeTiled>(p);
        }
    });
    if (!fn) throw CudaError("cuTensorMapEncodeTiled is not available from the driver");
    return fn;
}

}  // namespace

void tma_encode_tiled(CUtensorMap* map, CUtensorMapDataType type, cuuint32_t rank, const void* addr,
                      const cuuint64_t* dims, const cuuint64_t* strides_bytes, const cuuint32_t* box,
                      CUtensorMapSwizzle swizzle) {
    const cuuint32_t estr[5] = {1, 1, 1, 1, 1};
    // out-of-bounds elements of a box read as zero (FLOAT_OOB_FILL_NONE)
    const CUresult r = encoder()(map, type, rank, const_cast<void*>(addr), dims, strides_bytes, box, estr,
                                 CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                 CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) throw CudaError("cuTensorMapEncodeTiled failed: " + std::to_string(static_cast<int>(r)));
}

}  // namespace sana
