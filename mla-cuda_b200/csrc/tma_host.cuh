// Host-side TMA tensor-map construction (cuTensorMapEncodeTiled through the
// runtime's driver entry point, so the library does not link libcuda directly).
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <type_traits>

namespace mla {

inline PFN_cuTensorMapEncodeTiled_v12000 tma_encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        cudaDriverEntryPointQueryResult q;
        void* f = nullptr;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
    }
    return fn;
}

template <typename T> constexpr CUtensorMapDataType tma_dtype() {
    return std::is_same<T, float>::value ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
         : std::is_same<T, __half>::value ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                          : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
}

// 3-D map: dims innermost first (elements), strides of dims 1 and 2 in elements,
// box in elements, 128-byte swizzle when `swz` (with 32-byte swizzle atoms when
// `atom32`: the layout the tensor cores want for MN-major 32-bit operands).
template <typename T>
inline bool make_map_3d(CUtensorMap* m, const void* base, const int64_t dims[3], const int64_t strides[2],
                        const uint32_t box[3], bool swz, bool atom32 = false) {
    auto fn = tma_encode_fn();
    if (!fn) return false;
    cuuint64_t d[3] = {cuuint64_t(dims[0]), cuuint64_t(dims[1]), cuuint64_t(dims[2])};
    cuuint64_t s[2] = {cuuint64_t(strides[0]) * sizeof(T), cuuint64_t(strides[1]) * sizeof(T)};
    cuuint32_t b[3] = {box[0], box[1], box[2]};
    cuuint32_t e[3] = {1, 1, 1};
    return fn(m, tma_dtype<T>(), 3, const_cast<void*>(base), d, s, b, e, CU_TENSOR_MAP_INTERLEAVE_NONE,
              !swz ? CU_TENSOR_MAP_SWIZZLE_NONE
                   : atom32 ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_128B,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace mla
