// Host-side TMA tensor-map encoding shared by the decode and prefill launchers.
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include "../../include/dvattn_b200.h"

namespace dvb {

inline PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
    }
    return fn;
}

// [tokens = NB*BS][Hkv][E] cache as a 3-D map, box = 64 columns x 1 head x boxr tokens,
// 128-byte swizzle.
// [tokens][Hkv][E] cache as a 4-D map {64 columns, tokens, E/64 panels, Hkv heads} whose box
// {64, boxr, E/64, Hkv} is one page for all heads, landing as [head][panel][row][128 B]
// with the 128-byte swizzle.
inline bool encode_cache_map_all_heads(CUtensorMap* m, const void* base, int dtype, int E, int Hkv, long long tokens,
                                int boxr) {
    auto fn = tensor_map_encoder();
    if (!fn) return false;
    cuuint64_t dims[4] = {64, (cuuint64_t)tokens, (cuuint64_t)(E / 64), (cuuint64_t)Hkv};
    cuuint64_t strides[3] = {(cuuint64_t)Hkv * E * 2, 128, (cuuint64_t)E * 2};
    cuuint32_t box[4] = {64, (cuuint32_t)boxr, (cuuint32_t)(E / 64), (cuuint32_t)Hkv};
    cuuint32_t es[4] = {1, 1, 1, 1};
    const CUtensorMapDataType dt =
        dtype == DVATTN_FLOAT16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    return fn(m, dt, 4, const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
              CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Contiguous fragment [B][Hkv][rows][E] as a 5-D map whose box (64 columns x boxr rows x
// all panels x all heads x 1 batch entry) lands in shared memory in the same
// [head][panel][row][128 B] order as encode_cache_map_all_heads's page box.
inline bool encode_fragment_map(CUtensorMap* m, const void* base, int dtype, int E, int Hkv, long long rows, int B,
                                int boxr) {
    auto fn = tensor_map_encoder();
    if (!fn) return false;
    const cuuint64_t r = rows > 0 ? (cuuint64_t)rows : 1;
    cuuint64_t dims[5] = {64, r, (cuuint64_t)(E / 64), (cuuint64_t)Hkv, (cuuint64_t)(B > 0 ? B : 1)};
    cuuint64_t strides[4] = {(cuuint64_t)E * 2, 128, r * E * 2, (cuuint64_t)Hkv * r * E * 2};
    cuuint32_t box[5] = {64, (cuuint32_t)boxr, (cuuint32_t)(E / 64), (cuuint32_t)Hkv, 1};
    cuuint32_t es[5] = {1, 1, 1, 1, 1};
    const CUtensorMapDataType dt =
        dtype == DVATTN_FLOAT16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    return fn(m, dt, 5, const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
              CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

inline bool encode_cache_map(CUtensorMap* m, const void* base, int dtype, int E, int Hkv, long long tokens, int boxr) {
    auto fn = tensor_map_encoder();
    if (!fn) return false;
    cuuint64_t dims[3] = {(cuuint64_t)E, (cuuint64_t)Hkv, (cuuint64_t)tokens};
    cuuint64_t strides[2] = {(cuuint64_t)E * 2, (cuuint64_t)Hkv * E * 2};
    cuuint32_t box[3] = {64, 1, (cuuint32_t)boxr};
    cuuint32_t es[3] = {1, 1, 1};
    const CUtensorMapDataType dt =
        dtype == DVATTN_FLOAT16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    return fn(m, dt, 3, const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
              CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace dvb
