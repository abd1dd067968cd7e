// KV append through slot ids, with K-RoPE (and optionally Q-RoPE) fused.
//
// Replaces, on the device, the per-block strided copy_ of
// KVAllocator.append (src/pagedcore/kv_cache.py:161-172), the per-(request,
// layer) copy_ of write_decode_layer (kv_cache.py:244-245) and the FP16
// elementwise rotation of apply_rope (src/pagedcore/dense.py:48-59).
//
// Work unit: one warp per (token, up to 4 consecutive layers).  A (layer,
// token) row of K or V is 4 heads x 64 dims = 512 B, contiguous both in the
// source and in the pool, so lane j moves chunk j (16 B) of every row with
// fully coalesced accesses, and the rotate_half partner 32 dims away sits in
// lane j ^ 4 (a shuffle, not a second load).  The token's slot, position and
// cos/sin chunk are read once per unit and all K/V loads of the unit are in
// flight before the first store.  HBM-bound: per (layer, token) 1 KiB of K/V
// read and 1 KiB written, plus the RoPE row once per unit (L2).  An earlier
// thread-per-chunk form (two 64-bit divisions and a dependent slot load per
// 16 B, the partner chunk loaded again) reached a quarter of HBM bandwidth.
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

#include <atomic>

#include "pagedkv.h"
#include "status.h"

namespace {

constexpr int kHeadDim = PKV_HEAD_DIM;
constexpr int kKvHeads = PKV_KV_HEADS;
constexpr int kQueryHeads = PKV_QUERY_HEADS;
constexpr int kRopeHalf = kHeadDim / 2;   // 32 distinct frequencies
constexpr int kChunkElems = 8;            // FP16 values per 16-byte chunk
constexpr int kChunksPerHead = kHeadDim / kChunkElems;             // 8
static_assert(kKvHeads * kChunksPerHead == 32, "a K or V row is one chunk per lane");
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

// Two FP16 values per 32-bit word, low half first.  x: own values, y: the
// values 32 dims away, negate: own chunk is in the first half (rotate_half
// gives -x[d + 32] there).  Bit views, no address taken, so the operands
// stay in registers.
__device__ __forceinline__ uint32_t rotate_word(uint32_t x, uint32_t y, uint32_t c, uint32_t s, bool negate) {
    uint32_t out = 0;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const int shift = 16 * h;
        const __half xv = __ushort_as_half(static_cast<unsigned short>(x >> shift));
        const __half yv = __ushort_as_half(static_cast<unsigned short>(y >> shift));
        const __half cv = __ushort_as_half(static_cast<unsigned short>(c >> shift));
        const __half sv = __ushort_as_half(static_cast<unsigned short>(s >> shift));
        const __half rot = negate ? __hneg(yv) : yv;
        const __half r = round_add(round_mul(xv, cv), round_mul(rot, sv));
        out |= static_cast<uint32_t>(__half_as_ushort(r)) << shift;
    }
    return out;
}

__device__ __forceinline__ uint4 rotate_chunk(uint4 x, uint4 y, uint4 c, uint4 s, bool negate) {
    return make_uint4(rotate_word(x.x, y.x, c.x, s.x, negate), rotate_word(x.y, y.y, c.y, s.y, negate),
                      rotate_word(x.z, y.z, c.z, s.z, negate), rotate_word(x.w, y.w, c.w, s.w, negate));
}

// Shuffle a chunk from lane ^ 4: the chunk 32 dims away in the same head.
__device__ __forceinline__ uint4 partner_chunk(uint4 x) {
    uint4 y;
    y.x = __shfl_xor_sync(0xffffffffu, x.x, 4);
    y.y = __shfl_xor_sync(0xffffffffu, x.y, 4);
    y.z = __shfl_xor_sync(0xffffffffu, x.z, 4);
    y.w = __shfl_xor_sync(0xffffffffu, x.w, 4);
    return y;
}

// One warp per unit of (token, up to kLayersPerUnit consecutive layers).
// Lane j holds chunk j of a 512 B K or V row (head j / 8, dims 8 * (j % 8)
// .. + 7), so the row moves with one coalesced 16-byte access per lane and
// the rotate_half partner, 32 dims away, is in lane j ^ 4.  The token's slot,
// position and cos/sin chunk are read once per unit, and every K and V load
// of the unit is issued before the first store.
constexpr int kLayersPerUnit = 4;
constexpr int kWarpsPerCta = 8;

template <bool WITH_Q>
__global__ void __launch_bounds__(kWarpsPerCta * 32, WITH_Q ? 1 : 2) append_kv_kernel(
    __half *__restrict__ pool, int32_t num_blocks, int32_t layer_begin, int32_t layer_count,
    const __half *__restrict__ key, const __half *__restrict__ value, int64_t src_layer_stride,
    int64_t src_token_stride, const int32_t *__restrict__ slots,
    const int32_t *__restrict__ positions, int32_t tokens, const __half *__restrict__ rope_cos,
    const __half *__restrict__ rope_sin,
    // query_in and query_out may be the same buffer (Q rotated in place):
    // no __restrict__ on either, each chunk is read before it is written.
    const __half *query_in, __half *query_out, int64_t q_layer_stride, int64_t q_token_stride,
    int32_t *__restrict__ error_flag) {
    const int lane = threadIdx.x & 31;
    const int head = lane >> 3;
    const int chunk = lane & 7;
    const bool first_half = chunk < 4;  // rotate_half gives -x[d + 32] there
    // With Q (single-layer calls: per-layer decode writes, prefill chunks) a
    // unit is one layer, which keeps the Q chunks in registers.
    constexpr int kUnitLayers = WITH_Q ? 1 : kLayersPerUnit;
    const int groups = (layer_count + kUnitLayers - 1) / kUnitLayers;
    const int64_t units = static_cast<int64_t>(tokens) * groups;
    const int64_t warps = static_cast<int64_t>(gridDim.x) * kWarpsPerCta;
    for (int64_t unit = static_cast<int64_t>(blockIdx.x) * kWarpsPerCta + (threadIdx.x >> 5); unit < units;
         unit += warps) {
        const int t = static_cast<int>(unit / groups);
        const int l0 = static_cast<int>(unit - static_cast<int64_t>(t) * groups) * kUnitLayers;
        const int n = min(kUnitLayers, layer_count - l0);
        const int64_t src = static_cast<int64_t>(l0) * src_layer_stride + static_cast<int64_t>(t) * src_token_stride +
                            head * kHeadDim + chunk * kChunkElems;
        uint4 kx[kUnitLayers], vx[kUnitLayers];
#pragma unroll
        for (int i = 0; i < kUnitLayers; ++i) {
            if (i < n) {
                kx[i] = load16(key + src + i * src_layer_stride);
                vx[i] = load16(value + src + i * src_layer_stride);
            }
        }
        const int32_t slot = slots[t];
        const int32_t block = slot >> 4;
        const bool slot_ok = slot >= 0 && block < num_blocks;
        if (!slot_ok && lane == 0) atomicOr(error_flag, PKV_DEVICE_BAD_BLOCK);
        bool pos_ok = true;
        uint4 c = make_uint4(0, 0, 0, 0), sn = make_uint4(0, 0, 0, 0);
        if (rope_cos != nullptr) {
            const int32_t pos = positions[t];
            pos_ok = pos >= 0 && pos < PKV_CONTEXT_LIMIT;
            if (!pos_ok && lane == 0) atomicOr(error_flag, PKV_DEVICE_BAD_POSITION);
            const int64_t tab = static_cast<int64_t>(pos_ok ? pos : 0) * kRopeHalf + (chunk & 3) * kChunkElems;
            c = load16(rope_cos + tab);
            sn = load16(rope_sin + tab);
        }
        // Pool row of (layer, K|V, block, slot % 16, head): the slot term is
        // the same for every layer; the layer and K/V terms are multiples of
        // the block count.
        const int64_t row_stride = static_cast<int64_t>(num_blocks) * PKV_BLOCK_TOKENS * kKvHeads * kHeadDim;
        const int64_t dst0 = ((static_cast<int64_t>(block) * PKV_BLOCK_TOKENS + (slot & 15)) * kKvHeads + head) *
                                 kHeadDim + chunk * kChunkElems;
#pragma unroll
        for (int i = 0; i < kUnitLayers; ++i) {
            if (i < n) {
                uint4 k = kx[i];
                if (rope_cos != nullptr) k = rotate_chunk(kx[i], partner_chunk(kx[i]), c, sn, first_half);
                if (slot_ok) {
                    const int64_t layer = layer_begin + l0 + i;
                    if (pos_ok) store16(pool + (layer * 2 + 0) * row_stride + dst0, k);
                    store16(pool + (layer * 2 + 1) * row_stride + dst0, vx[i]);
                }
            }
        }
        if constexpr (WITH_Q) {
            // Q rows: 32 heads x 8 chunks; lane j holds chunks j + 32 m
            // (head 4 m + j / 8, same chunk j % 8), partner again in lane j ^ 4.
#pragma unroll 1
            for (int i = 0; i < n; ++i) {
                const int64_t row = static_cast<int64_t>(l0 + i) * q_layer_stride +
                                    static_cast<int64_t>(t) * q_token_stride + lane * kChunkElems;
                constexpr int kBatch = 4;  // of the kQueryChunks / 32 chunks each lane holds
#pragma unroll 1
                for (int m0 = 0; m0 < kQueryChunks / 32; m0 += kBatch) {
                    uint4 qx[kBatch];
#pragma unroll
                    for (int m = 0; m < kBatch; ++m) qx[m] = load16(query_in + row + (m0 + m) * 32 * kChunkElems);
#pragma unroll
                    for (int m = 0; m < kBatch; ++m) {
                        uint4 q = qx[m];
                        if (rope_cos != nullptr) q = rotate_chunk(qx[m], partner_chunk(qx[m]), c, sn, first_half);
                        if (pos_ok) store16(query_out + row + (m0 + m) * 32 * kChunkElems, q);
                    }
                }
            }
        }
    }
}

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int sm_count_of_current_device() {
    constexpr int kMaxDevices = 64;
    static std::atomic<int> cached[kMaxDevices] = {};
    int device = 0;
    if (cudaGetDevice(&device) != cudaSuccess) return 148;
    if (device >= 0 && device < kMaxDevices) {
        const int known = cached[device].load(std::memory_order_relaxed);
        if (known > 0) return known;
    }
    int sms = 148;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
    if (device >= 0 && device < kMaxDevices && sms > 0) cached[device].store(sms, std::memory_order_relaxed);
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
    const int unit_layers = query_in != nullptr ? 1 : kLayersPerUnit;
    const int64_t units = static_cast<int64_t>(tokens) * ((layer_count + unit_layers - 1) / unit_layers);
    const int64_t wanted = (units + kWarpsPerCta - 1) / kWarpsPerCta;
    const int64_t cap = static_cast<int64_t>(sm_count_of_current_device()) * 8;
    const int grid = static_cast<int>(wanted < cap ? wanted : cap);
    const int threads = kWarpsPerCta * 32;
    const __half *cos_table = static_cast<const __half *>(rope_table);
    const __half *sin_table = cos_table ? cos_table + PKV_CONTEXT_LIMIT * kRopeHalf : nullptr;
    auto kernel = query_in != nullptr ? append_kv_kernel<true> : append_kv_kernel<false>;
    kernel<<<grid, threads, 0, static_cast<cudaStream_t>(stream)>>>(
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
