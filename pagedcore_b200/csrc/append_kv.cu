// KV append through slot ids, with K-RoPE (and optionally Q-RoPE) fused.
//
// Replaces, on the device, the per-block strided copy_ of
// KVAllocator.append (src/pagedcore/kv_cache.py:161-172), the per-(request,
// layer) copy_ of write_decode_layer (kv_cache.py:244-245) and the FP16
// elementwise rotation of apply_rope (src/pagedcore/dense.py:48-59).
//
// Work unit: one 16-byte chunk (8 FP16 values) of one head of one token of
// one layer.  A (layer, token) row of K or V is 4 heads x 64 dims = 512 B,
// contiguous both in the source and in the pool, so 32 consecutive threads
// move one row with fully coalesced 16-byte loads and stores.  The kernel is
// HBM-bound: per (layer, token) it reads 1 KiB of K/V (+256 B of the RoPE
// table from L2) and writes 1 KiB.
//
// Bit-exactness of the rotation: the reference computes, in FP16 eager ops,
//   k' = k * cos + cat(-k[32:], k[:32]) * sin
// i.e. two separately rounded FP16 products and one rounded FP16 sum, with
// cos/sin already rounded to FP16.  Each step here is the FP32 operation on
// the FP16 operands followed by round-to-nearest-even to FP16.  FP32 carries
// 24 >= 2*11+2 significand bits, so FP32-then-round equals the correctly
// rounded FP16 operation, which is what the reference's ATen kernels produce.
// The cos/sin values come from a table that the host builds with the
// reference's own op sequence (dense.py:48-54); no device trigonometry.

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "pagedkv.h"
#include "status.h"

namespace {

constexpr int kHeadDim = PKV_HEAD_DIM;
constexpr int kKvHeads = PKV_KV_HEADS;
constexpr int kQueryHeads = PKV_QUERY_HEADS;
constexpr int kRopeHalf = kHeadDim / 2;   // 32 distinct frequencies
constexpr int kChunkElems = 8;            // FP16 values per 16-byte chunk
constexpr int kChunksPerHead = kHeadDim / kChunkElems;             // 8
constexpr int kKvChunks = kKvHeads * kChunksPerHead;               // 32 per K or V row
constexpr int kQueryChunks = kQueryHeads * kChunksPerHead;         // 256 per Q row

__device__ __forceinline__ uint4 load16(const __half *p) {
    return *reinterpret_cast<const uint4 *>(p);
}

__device__ __forceinline__ void store16(__half *p, uint4 v) {
    *reinterpret_cast<uint4 *>(p) = v;
}

__device__ __forceinline__ __half round_mul(__half a, __half b) {
    return __float2half_rn(__half2float(a) * __half2float(b));
}

__device__ __forceinline__ __half round_add(__half a, __half b) {
    return __float2half_rn(__half2float(a) + __half2float(b));
}

// x: own 8 values, y: the values 32 dims away, negate: own chunk is in the
// first half (rotate_half gives -x[d+32] there).
__device__ __forceinline__ uint4 rotate_chunk(uint4 x, uint4 y, uint4 c, uint4 s, bool negate) {
    const __half *xh = reinterpret_cast<const __half *>(&x);
    const __half *yh = reinterpret_cast<const __half *>(&y);
    const __half *ch = reinterpret_cast<const __half *>(&c);
    const __half *sh = reinterpret_cast<const __half *>(&s);
    uint4 out;
    __half *oh = reinterpret_cast<__half *>(&out);
#pragma unroll
    for (int i = 0; i < kChunkElems; ++i) {
        const __half rot = negate ? __hneg(yh[i]) : yh[i];
        oh[i] = round_add(round_mul(xh[i], ch[i]), round_mul(rot, sh[i]));
    }
    return out;
}

__global__ void __launch_bounds__(256) append_kv_kernel(
    __half *__restrict__ pool, int32_t num_blocks, int32_t layer_begin, int32_t layer_count,
    const __half *__restrict__ key, const __half *__restrict__ value, int64_t src_layer_stride,
    int64_t src_token_stride, const int32_t *__restrict__ slots,
    const int32_t *__restrict__ positions, int32_t tokens, const __half *__restrict__ rope_cos,
    const __half *__restrict__ rope_sin, const __half *__restrict__ query_in,
    __half *__restrict__ query_out, int64_t q_layer_stride, int64_t q_token_stride,
    int32_t *__restrict__ error_flag) {
    const int chunks_per_item = 2 * kKvChunks + (query_in != nullptr ? kQueryChunks : 0);
    const int64_t total = static_cast<int64_t>(layer_count) * tokens * chunks_per_item;
    const int64_t step = static_cast<int64_t>(gridDim.x) * blockDim.x;
    for (int64_t c = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; c < total;
         c += step) {
        const int64_t item = c / chunks_per_item;
        const int r = static_cast<int>(c - item * chunks_per_item);
        const int l = static_cast<int>(item / tokens);
        const int t = static_cast<int>(item - static_cast<int64_t>(l) * tokens);
        const int layer = layer_begin + l;
        if (r < 2 * kKvChunks) {
            const int kind = r / kKvChunks;  // 0: K, 1: V
            const int head = (r % kKvChunks) / kChunksPerHead;
            const int chunk = r % kChunksPerHead;
            const int32_t slot = slots[t];
            const int32_t block = slot >> 4;
            if (slot < 0 || block >= num_blocks) {
                atomicOr(error_flag, PKV_DEVICE_BAD_BLOCK);
                continue;
            }
            const int64_t src_row = l * src_layer_stride + t * src_token_stride + head * kHeadDim;
            uint4 x = load16((kind == 0 ? key : value) + src_row + chunk * kChunkElems);
            if (kind == 0 && rope_cos != nullptr) {
                const int32_t pos = positions[t];
                if (pos < 0 || pos >= PKV_CONTEXT_LIMIT) {
                    atomicOr(error_flag, PKV_DEVICE_BAD_POSITION);
                    continue;
                }
                const uint4 y = load16(key + src_row + (chunk ^ 4) * kChunkElems);
                const int64_t tab = static_cast<int64_t>(pos) * kRopeHalf + (chunk & 3) * kChunkElems;
                x = rotate_chunk(x, y, load16(rope_cos + tab), load16(rope_sin + tab), chunk < 4);
            }
            const int64_t dst = ((((static_cast<int64_t>(layer) * 2 + kind) * num_blocks + block) *
                                      PKV_BLOCK_TOKENS +
                                  (slot & 15)) *
                                     kKvHeads +
                                 head) *
                                    kHeadDim +
                                chunk * kChunkElems;
            store16(pool + dst, x);
        } else {
            const int q = r - 2 * kKvChunks;
            const int head = q / kChunksPerHead;
            const int chunk = q % kChunksPerHead;
            const int64_t row = l * q_layer_stride + t * q_token_stride + head * kHeadDim;
            uint4 x = load16(query_in + row + chunk * kChunkElems);
            if (rope_cos != nullptr) {
                const int32_t pos = positions[t];
                if (pos < 0 || pos >= PKV_CONTEXT_LIMIT) {
                    atomicOr(error_flag, PKV_DEVICE_BAD_POSITION);
                    continue;
                }
                const uint4 y = load16(query_in + row + (chunk ^ 4) * kChunkElems);
                const int64_t tab = static_cast<int64_t>(pos) * kRopeHalf + (chunk & 3) * kChunkElems;
                x = rotate_chunk(x, y, load16(rope_cos + tab), load16(rope_sin + tab), chunk < 4);
            }
            store16(query_out + row + chunk * kChunkElems, x);
        }
    }
}

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int sm_count_of_current_device() {
    int device = 0, sms = 148;
    if (cudaGetDevice(&device) == cudaSuccess) {
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
    }
    return sms;
}

}  // namespace

extern "C" int64_t pkv_rope_table_bytes(void) {
    return 2LL * PKV_CONTEXT_LIMIT * kRopeHalf * static_cast<int64_t>(sizeof(__half));
}

extern "C" int pkv_append_kv(void *pool, int32_t num_blocks, int32_t layer_begin,
                             int32_t layer_count, const void *key, const void *value,
                             int64_t src_layer_stride, int64_t src_token_stride,
                             const int32_t *slots, const int32_t *positions, int32_t tokens,
                             const void *rope_table, const void *query_in, void *query_out,
                             int64_t q_layer_stride, int64_t q_token_stride, int32_t *error_flag,
                             void *stream) {
    pkv::clear_error();
    if (pool == nullptr || key == nullptr || value == nullptr || slots == nullptr ||
        error_flag == nullptr) {
        return pkv::fail(PKV_VALUE_ERROR, "append: pool, key, value, slots and error flag are required");
    }
    if (num_blocks < 1 || tokens < 0 || layer_count < 0 || layer_begin < 0 ||
        layer_begin + layer_count > PKV_LAYERS) {
        return pkv::fail(PKV_VALUE_ERROR, "append: layer range or sizes out of bounds");
    }
    if ((query_in == nullptr) != (query_out == nullptr)) {
        return pkv::fail(PKV_VALUE_ERROR, "append: query_in and query_out go together");
    }
    if (rope_table != nullptr && positions == nullptr) {
        return pkv::fail(PKV_VALUE_ERROR, "append: RoPE needs positions");
    }
    if (!aligned16(pool) || !aligned16(key) || !aligned16(value) || src_layer_stride % 8 ||
        src_token_stride % 8 || (rope_table && !aligned16(rope_table)) ||
        (query_in && (!aligned16(query_in) || !aligned16(query_out) || q_layer_stride % 8 ||
                      q_token_stride % 8))) {
        return pkv::fail(PKV_VALUE_ERROR, "append: tensors must be 16-byte aligned with strides in multiples of 8");
    }
    if (tokens == 0 || layer_count == 0) return PKV_OK;
    const int chunks = 2 * kKvChunks + (query_in ? kQueryChunks : 0);
    const int64_t total = static_cast<int64_t>(layer_count) * tokens * chunks;
    const int threads = 256;
    const int64_t wanted = (total + threads - 1) / threads;
    const int64_t cap = static_cast<int64_t>(sm_count_of_current_device()) * 16;
    const int grid = static_cast<int>(wanted < cap ? wanted : cap);
    const __half *cos_table = static_cast<const __half *>(rope_table);
    const __half *sin_table = cos_table ? cos_table + PKV_CONTEXT_LIMIT * kRopeHalf : nullptr;
    append_kv_kernel<<<grid, threads, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<__half *>(pool), num_blocks, layer_begin, layer_count,
        static_cast<const __half *>(key), static_cast<const __half *>(value), src_layer_stride,
        src_token_stride, slots, positions, tokens, cos_table, sin_table,
        static_cast<const __half *>(query_in), static_cast<__half *>(query_out), q_layer_stride,
        q_token_stride, error_flag);
    const cudaError_t err = cudaGetLastError();
    if (err != cudaSuccess) {
        return pkv::fail(PKV_CUDA_ERROR, std::string("append launch failed: ") + cudaGetErrorString(err));
    }
    return PKV_OK;
}
