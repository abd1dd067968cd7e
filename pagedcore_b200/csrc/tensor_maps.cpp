// TMA tensor maps: see tensor_maps.h.

#include "tensor_maps.h"

#include <cuda_runtime.h>

#include <functional>
#include <mutex>
#include <string>
#include <unordered_map>

#include "pagedkv.h"
#include "status.h"

namespace pkv {

EncodeTiled encode_fn() {
    static EncodeTiled fn = [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess) {
            p = nullptr;
        }
        return reinterpret_cast<EncodeTiled>(p);
    }();
    return fn;
}

namespace {

struct MapKey {
    uintptr_t pool;
    int32_t blocks;
    bool operator==(const MapKey &o) const { return pool == o.pool && blocks == o.blocks; }
};
struct MapKeyHash {
    size_t operator()(const MapKey &k) const { return std::hash<uintptr_t>()(k.pool) ^ (size_t(k.blocks) << 1); }
};

}  // namespace

int pool_tensor_map(const void *pool, int32_t num_blocks, CUtensorMap *out) {
    static std::mutex mutex;
    static std::unordered_map<MapKey, CUtensorMap, MapKeyHash> cache;
    const MapKey key{reinterpret_cast<uintptr_t>(pool), num_blocks};
    std::lock_guard<std::mutex> lock(mutex);
    auto it = cache.find(key);
    if (it != cache.end()) {
        *out = it->second;
        return PKV_OK;
    }
    EncodeTiled encode = encode_fn();
    if (encode == nullptr) return fail(PKV_CUDA_ERROR, "cuTensorMapEncodeTiled is unavailable");
    constexpr cuuint64_t kRowBytes = PKV_HEAD_DIM * 2;
    const cuuint64_t rows = static_cast<cuuint64_t>(PKV_LAYERS) * 2 * num_blocks * PKV_BLOCK_TOKENS;
    const cuuint64_t dims[3] = {PKV_HEAD_DIM, PKV_KV_HEADS, rows};
    const cuuint64_t strides[2] = {kRowBytes, PKV_KV_HEADS * kRowBytes};
    const cuuint32_t box[3] = {PKV_HEAD_DIM, 1u, PKV_BLOCK_TOKENS};
    const cuuint32_t elem[3] = {1u, 1u, 1u};
    CUtensorMap map;
    const CUresult r = encode(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void *>(pool), dims, strides, box,
                              elem, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        return fail(PKV_CUDA_ERROR, "cuTensorMapEncodeTiled failed with code " + std::to_string(int(r)));
    }
    cache.emplace(key, map);
    *out = map;
    return PKV_OK;
}

int matrix_tensor_map(const void *base, uint64_t rows, uint64_t cols, uint64_t row_stride, uint32_t box_rows,
                      CUtensorMap *out) {
    EncodeTiled encode = encode_fn();
    if (encode == nullptr) return fail(PKV_CUDA_ERROR, "cuTensorMapEncodeTiled is unavailable");
    const cuuint64_t dims[2] = {cols, rows};
    const cuuint64_t strides[1] = {row_stride * 2};
    const cuuint32_t box[2] = {64u, box_rows};
    const cuuint32_t elem[2] = {1u, 1u};
    const CUresult r = encode(out, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void *>(base), dims, strides, box,
                              elem, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        return fail(PKV_CUDA_ERROR, "cuTensorMapEncodeTiled (matrix) failed with code " + std::to_string(int(r)));
    }
    return PKV_OK;
}

}  // namespace pkv
