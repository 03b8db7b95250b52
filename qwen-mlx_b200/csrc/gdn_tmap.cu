// gdn_tmap.cu -- host-side encoding of TMA tensor maps (cuTensorMapEncodeTiled, taken from the driver
// through the runtime's entry-point query, so nothing links against libcuda directly).
#include <cuda.h>
#include <cuda_runtime.h>

#include "gdn_internal.h"

namespace gdn {

namespace {

using EncodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                 const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiled encoder() {
    static const EncodeTiled fn = []() -> EncodeTiled {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            return nullptr;
        return reinterpret_cast<EncodeTiled>(p);
    }();
    return fn;
}

}  // namespace

bool tmap_bf16_2d_sw128(CUtensorMap* map, const void* base, uint64_t cols, uint64_t rows, uint64_t ld_bytes,
                        uint32_t box_cols, uint32_t box_rows) {
    const EncodeTiled fn = encoder();
    if (!fn || ((uintptr_t)base & 15u) != 0 || ld_bytes % 16 != 0 || box_cols * 2 > 128 || cols == 0 || rows == 0)
        return false;
    const cuuint64_t dims[2] = {cols, rows};
    const cuuint64_t strides[1] = {ld_bytes};
    const cuuint32_t box[2] = {box_cols, box_rows};
    const cuuint32_t estr[2] = {1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool tmap_records(CUtensorMap* map, const void* recs, int n_tokens, long long rec_cap, int n_heads, int rec_bytes,
                  uint32_t box_tokens, uint32_t box_chunks) {
    const EncodeTiled fn = encoder();
    if (!fn || ((uintptr_t)recs & 15u) != 0 || rec_bytes % 16 != 0 || n_tokens <= 0 || n_heads <= 0) return false;
    // element (e, t, c, h) at recs + h * rec_cap * rec_bytes + t * rec_bytes + c * 16 + e * 2
    const cuuint64_t dims[4] = {8, (cuuint64_t)n_tokens, (cuuint64_t)(rec_bytes / 16), (cuuint64_t)n_heads};
    const cuuint64_t strides[3] = {(cuuint64_t)rec_bytes, 16, (cuuint64_t)rec_cap * rec_bytes};
    const cuuint32_t box[4] = {8, box_tokens, box_chunks, 1};
    const cuuint32_t estr[4] = {1, 1, 1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT16, 4, const_cast<void*>(recs), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace gdn
