// Causal prompt (prefill) attention through the block table, GQA, sm_100a.
//
// The attention of a prompt chunk whose K/V already sit in the pool: token t
// of the chunk (position start + t) attends to positions 0 .. start + t of
// its request, over the 16-token blocks its block table lists.  It stands in
// for the causal attention of PagedCore's dense prefill (dense_attention,
// src/pagedcore/dense.py:69-82, with the mask of decoder.py:225) with
// the numerics of its paged attention (attention.py:14-53: FP32 scores,
// softmax and sum from FP16 pages, one FP16 rounding of the output):
//   out[t,h] = sum_{p <= start+t} softmax_p(q[t,h] . K[p, h/8] * 0.125) V[p, h/8]
//
// Work split - one CTA per (query tile, KV head), 8 warps; a warp holds 2
// tokens of the tile with the 8 query heads of the KV head as the 16 rows of
// its MMA tiles (row r: token 2w + r/8, head r%8).  Whole tiles (16 tokens)
// stream the blocks 0 .. (last position)/16 once, so every K/V block is read
// once per 128 query rows (the one-token decode kernel reads it once per 8).
// When whole tiles would not fill one wave (two CTAs per SM), split tiles
// (8 tokens) halve the key range between two groups of 4 warps, each with its
// own copy ring and barrier, and merge the two (m, l, O) in shared memory:
// twice the CTAs, half the longest CTA (measured 17.0 against 24.8 us at 512
// tokens; at 2047, 102 against 97 us, so whole tiles are kept there).  Tiles
// are taken longest first across all four heads (the last tile of the chunk
// has the most blocks), so the short ones fill in behind the long ones.
//
// Data movement - a group's threads each copy one (whole) or two (split)
// 16-byte chunks of the block's 16 K rows or 16 V rows of this head
// (cp.async.cg, L2 only: the block is read again by the chunk's other tiles)
// into shared memory with the 128-byte XOR swizzle (chunk c of row r at
// c ^ (r & 7)), so the ldmatrix reads are bank-conflict free, through a
// 4-deep ring of (K, V) tiles (8 deep measured the same); the block ids are
// staged in shared memory once.  Slots at or past start + tokens (not written
// yet; they may hold anything) are zero-filled by the copy itself, so 0 * NaN
// never reaches the PV sum.  No wait in this kernel polls a flag:
// cp.async.wait_group and the barriers complete when the issued copies do.
//
// Math - mma.sync m16n8k16, FP16 in, FP32 accumulate:
//   S[16 rows x 16 keys]  = Q[16 x 64] . K^T[64 x 16]     (8 MMAs)
//   O[16 rows x 64 dims] += P[16 x 16] . V[16 x 64]       (8 MMAs)
// The S accumulator is the P operand in place (the m16n8 C layout of two
// adjacent key tiles is the m16k16 A layout).  Online softmax in base 2 with
// FP32 state; P is rounded to FP16 after scaling by 2^15, and the normaliser
// sums the same rounded weights, as in the decode kernel.  Only the blocks
// that cross a row's last position are masked, the scale is folded into the
// exponent's FMA, and O and l are rescaled only when a row's maximum moves
// (the factor would be exactly 1 otherwise).

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <string>

#include "pagedkv.h"
#include "ptx.cuh"
#include "status.h"

namespace {

constexpr int kHeadDim = PKV_HEAD_DIM;
constexpr int kKvHeads = PKV_KV_HEADS;
constexpr int kQueryHeads = PKV_QUERY_HEADS;
constexpr int kGroup = kQueryHeads / kKvHeads;  // 8 query heads per KV head
constexpr int kBlockTokens = PKV_BLOCK_TOKENS;
constexpr int kRowBytes = kHeadDim * 2;              // 128 B: one head of one token
constexpr int kTileBytes = kBlockTokens * kRowBytes; // 2 KiB: one head of one block
constexpr int kStages = 4;
constexpr int kMaxTableBlocks = PKV_CONTEXT_LIMIT / PKV_BLOCK_TOKENS;  // 128
constexpr int kThreads = 256;
constexpr float kScaleLog2 = 0.125f * 1.4426950408889634f;  // 64^-0.5 * log2(e)
constexpr float kWeightShift = 15.0f;                       // P scaled by 2^15 before FP16

// The two CTA shapes.  Whole: a 16-token tile, 8 warps over all of its blocks.
// Split: an 8-token tile whose key range is halved between two groups of 4
// warps (each with its own copy ring), merged in shared memory at the end;
// twice the CTAs for chunks whose whole tiles would not fill the GPU.
template <bool SPLIT>
struct Shape {
    static constexpr int kTileTokens = SPLIT ? 8 : 16;
    static constexpr int kGroups = SPLIT ? 2 : 1;
    static constexpr int kGroupWarps = kTileTokens / 2;  // a warp: 2 tokens x 8 heads = 16 MMA rows
    static constexpr int kGroupThreads = kGroupWarps * 32;
    static constexpr int kCopies = 2 * kBlockTokens * (kRowBytes / 16) / kGroupThreads;  // 16-byte copies a block
    static_assert(kGroups * kGroupThreads == kThreads, "every thread belongs to a group");
};
static_assert(kGroup == 8, "a KV head's query heads fill 8 MMA rows");

struct PrefillArgs {
    const __half *pool;
    const __half *query;
    __half *out;
    const int32_t *blocks;  // physical block of each 16-position block of the request
    int64_t query_stride;   // elements between tokens
    int64_t out_stride;
    int32_t num_blocks;
    int32_t layer;
    int32_t start;   // position of the chunk's first token
    int32_t tokens;  // chunk tokens
    int32_t *error_flag;
};

__device__ __forceinline__ float quad_max(float v) {
    // The 4 lanes of a quad hold the 16 keys of one MMA row.
    v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 1));
    return fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 2));
}

__device__ __forceinline__ float quad_sum(float v) {
    v += __shfl_xor_sync(0xffffffffu, v, 1);
    return v + __shfl_xor_sync(0xffffffffu, v, 2);
}

// Barrier of one split group's 128 threads (ids 1 and 2; __syncthreads is 0).
__device__ __forceinline__ void group_sync(int group) {
    if (group) {
        asm volatile("bar.sync 2, %0;" ::"n"(kThreads / 2) : "memory");
    } else {
        asm volatile("bar.sync 1, %0;" ::"n"(kThreads / 2) : "memory");
    }
}

__device__ __forceinline__ uint32_t ld32(const __half *p) { return *reinterpret_cast<const uint32_t *>(p); }

template <bool SPLIT>
__global__ void __launch_bounds__(kThreads) prefill_attention_kernel(const PrefillArgs a) {
    using S = Shape<SPLIT>;
    __shared__ __align__(128) uint8_t ring[S::kGroups * kStages * 2 * kTileBytes];
    __shared__ int32_t table[kMaxTableBlocks];

    // Longest tiles first over all heads: the hardware starts CTAs in
    // blockIdx order, so the head varies fastest.
    const int tile = gridDim.x / kKvHeads - 1 - static_cast<int>(blockIdx.x) / kKvHeads;
    const int kv = blockIdx.x % kKvHeads;
    const int t0 = tile * S::kTileTokens;
    const int last_token = min(t0 + S::kTileTokens - 1, a.tokens - 1);
    const int blocks = (a.start + last_token) / kBlockTokens + 1;  // blocks 0 .. blocks-1
    const int written = a.start + a.tokens;                         // positions below hold K/V
    // The tile's block ids, staged once (start + tokens <= 2048: at most 128).
    for (int j = threadIdx.x; j < blocks; j += kThreads) table[j] = a.blocks[j];
    __syncthreads();

    // This thread's group and its range of blocks (split: group 1 takes the
    // second half, with the diagonal).
    const int group = SPLIT ? static_cast<int>(threadIdx.x) / S::kGroupThreads : 0;
    const int gtid = threadIdx.x % S::kGroupThreads;
    const int half = (blocks + 1) / 2;
    const int g_begin = group ? half : 0;
    const int g_end = SPLIT && !group ? half : blocks;
    const int g_count = g_end - g_begin;
    // This thread's copies: kCopies consecutive 16-byte chunks of K or V row `key` of each block.
    const int first = gtid * S::kCopies;
    const int part = first >> 7;  // 0: K, 1: V
    const int key = (first >> 3) & (kBlockTokens - 1);
    const int ch0 = first & 7;
    const uint32_t ring_base = pkv::smem_addr(ring) + group * (kStages * 2 * kTileBytes);
    const uint32_t dst_row = ring_base + part * kTileBytes + key * kRowBytes;
    const int64_t part_blocks = (static_cast<int64_t>(a.layer) * 2 + part) * a.num_blocks;
    const __half *copy_src = a.pool + kv * kHeadDim + ch0 * 8;
    auto issue = [&](int jl) {
        const int j = g_begin + jl;
        const int32_t block = table[j];
        const bool ok = block >= 0 && block < a.num_blocks;
        if (!ok && gtid == 0) atomicOr(a.error_flag, PKV_DEVICE_BAD_BLOCK);
        const __half *src =
            copy_src + ((part_blocks + (ok ? block : 0)) * kBlockTokens + key) * (kKvHeads * kHeadDim);
        const uint32_t bytes = ok && j * kBlockTokens + key < written ? 16u : 0u;
        const uint32_t stage = dst_row + (jl % kStages) * (2 * kTileBytes);
#pragma unroll
        for (int c = 0; c < S::kCopies; ++c) {
            pkv::cp_async_16(stage + (((ch0 + c) ^ (key & 7)) << 4), src + 8 * c, bytes);
        }
    };
#pragma unroll
    for (int jl = 0; jl < kStages - 1; ++jl) {
        if (jl < g_count) issue(jl);
        pkv::cp_async_commit();
    }

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int g = lane >> 2;
    const int t = lane & 3;
    const int token_a = t0 + 2 * (warp % S::kGroupWarps);  // MMA rows g     (head g of the group)
    const int token_b = token_a + 1;                      // MMA rows g + 8
    const int qa = min(token_a, a.tokens - 1);
    const int qb = min(token_b, a.tokens - 1);
    const int lim_a = a.start + qa;  // last position each row attends to
    const int lim_b = a.start + qb;
    const int warp_end = token_a < a.tokens ? min(g_end, lim_b / kBlockTokens + 1) : g_begin;
    const int head = kv * kGroup + g;

    // Q as the A operand: (row g | g+8, dims 16ks + 2t, +1 | +8, +9).
    uint32_t qf[4][4];
    {
        const __half *qa_row = a.query + qa * a.query_stride + head * kHeadDim + 2 * t;
        const __half *qb_row = a.query + qb * a.query_stride + head * kHeadDim + 2 * t;
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) {
            qf[ks][0] = ld32(qa_row + 16 * ks);
            qf[ks][1] = ld32(qb_row + 16 * ks);
            qf[ks][2] = ld32(qa_row + 16 * ks + 8);
            qf[ks][3] = ld32(qb_row + 16 * ks + 8);
        }
    }

    float m_a = -INFINITY, m_b = -INFINITY, l_a = 0.f, l_b = 0.f;
    float o[8][4];
#pragma unroll
    for (int dt = 0; dt < 8; ++dt) o[dt][0] = o[dt][1] = o[dt][2] = o[dt][3] = 0.f;

    for (int jl = 0; jl < g_count; ++jl) {
        const int j = g_begin + jl;
        // Block j's copies (copy group jl) are complete; every warp of the
        // group is done with the stage the next copy overwrites.
        pkv::cp_async_wait<kStages - 2>();
        if (SPLIT) {
            group_sync(group);
        } else {
            __syncthreads();
        }
        if (jl + kStages - 1 < g_count) issue(jl + kStages - 1);
        pkv::cp_async_commit();
        if (j >= warp_end) continue;

        const uint32_t ktile = ring_base + (jl % kStages) * (2 * kTileBytes);
        const uint32_t vtile = ktile + kTileBytes;
        // kf[ks]: (keys 0-7 | 8-15) x (dims 16ks.. | 16ks+8..).
        uint32_t kf[4][4];
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) {
            const int mat = lane >> 3;
            const int tok = (lane & 7) + ((mat & 1) << 3);
            const int chunk = 2 * ks + (mat >> 1);
            pkv::ldmatrix_x4(ktile + tok * kRowBytes + ((chunk ^ (tok & 7)) << 4), kf[ks][0], kf[ks][1], kf[ks][2],
                             kf[ks][3]);
        }
        // vf[mt]: V^T fragments of dims 16mt .. 16mt+15 (loading them after the S MMAs
        // measured 17% slower: the PV MMAs then wait on them).
        uint32_t vf[4][4];
#pragma unroll
        for (int mt = 0; mt < 4; ++mt) {
            const int mat = lane >> 3;
            const int tok = (lane & 7) + ((mat >> 1) << 3);
            const int chunk = 2 * mt + (mat & 1);
            pkv::ldmatrix_x4_trans(vtile + tok * kRowBytes + ((chunk ^ (tok & 7)) << 4), vf[mt][0], vf[mt][1],
                                   vf[mt][2], vf[mt][3]);
        }
        // S = Q . K^T: s[nt] holds keys 8nt + 2t, +1 of rows g (0, 1) and g + 8 (2, 3).
        float s[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) {
            pkv::mma_f16_16816(s[0], qf[ks][0], qf[ks][1], qf[ks][2], qf[ks][3], kf[ks][0], kf[ks][2]);
            pkv::mma_f16_16816(s[1], qf[ks][0], qf[ks][1], qf[ks][2], qf[ks][3], kf[ks][1], kf[ks][3]);
        }
        if (j * kBlockTokens + kBlockTokens - 1 > lim_a) {  // a diagonal block: mask positions past each row
            const int p0 = j * kBlockTokens + 2 * t;
#pragma unroll
            for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                    const int pos = p0 + 8 * nt + e;
                    if (pos > lim_a) s[nt][e] = -INFINITY;
                    if (pos > lim_b) s[nt][2 + e] = -INFINITY;
                }
            }
        }
        // Running maxima in log2 units (the scale is positive, so it commutes
        // with the max).  Whole tiles start at block 0, which holds position 0
        // of every row, so their maxima are finite from the first block on; in
        // a split tile's second half a row may have no position yet (-inf).
        const float mn_a =
            fmaxf(m_a, quad_max(fmaxf(fmaxf(s[0][0], s[0][1]), fmaxf(s[1][0], s[1][1]))) * kScaleLog2);
        const float mn_b =
            fmaxf(m_b, quad_max(fmaxf(fmaxf(s[0][2], s[0][3]), fmaxf(s[1][2], s[1][3]))) * kScaleLog2);
        if (__any_sync(0xffffffffu, mn_a != m_a || mn_b != m_b)) {  // some row's maximum moved: rescale
            const float alpha_a = SPLIT && m_a == mn_a ? 1.f : pkv::exp2_approx(m_a - mn_a);
            const float alpha_b = SPLIT && m_b == mn_b ? 1.f : pkv::exp2_approx(m_b - mn_b);
            l_a *= alpha_a;
            l_b *= alpha_b;
#pragma unroll
            for (int dt = 0; dt < 8; ++dt) {
                o[dt][0] *= alpha_a;
                o[dt][1] *= alpha_a;
                o[dt][2] *= alpha_b;
                o[dt][3] *= alpha_b;
            }
            m_a = mn_a;
            m_b = mn_b;
        }
        // With no position yet the row's scores are all -inf: any finite shift gives p = 0.
        const float shift_a = SPLIT && m_a == -INFINITY ? 0.f : kWeightShift - m_a;
        const float shift_b = SPLIT && m_b == -INFINITY ? 0.f : kWeightShift - m_b;
        __half2 p[2][2];  // p[nt][0]: row g, p[nt][1]: row g + 8 (keys 8nt + 2t, +1)
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) {
            p[nt][0] = __floats2half2_rn(pkv::exp2_approx(fmaf(s[nt][0], kScaleLog2, shift_a)),
                                         pkv::exp2_approx(fmaf(s[nt][1], kScaleLog2, shift_a)));
            p[nt][1] = __floats2half2_rn(pkv::exp2_approx(fmaf(s[nt][2], kScaleLog2, shift_b)),
                                         pkv::exp2_approx(fmaf(s[nt][3], kScaleLog2, shift_b)));
        }
        const float2 fa0 = __half22float2(p[0][0]), fa1 = __half22float2(p[1][0]);
        const float2 fb0 = __half22float2(p[0][1]), fb1 = __half22float2(p[1][1]);
        l_a += (fa0.x + fa0.y) + (fa1.x + fa1.y);
        l_b += (fb0.x + fb0.y) + (fb1.x + fb1.y);
        // O += P . V: P's A fragments are the S accumulators of key tiles 0 and 1.
        const uint32_t a0 = pkv::pack_half2(p[0][0]), a1 = pkv::pack_half2(p[0][1]);
        const uint32_t a2 = pkv::pack_half2(p[1][0]), a3 = pkv::pack_half2(p[1][1]);
#pragma unroll
        for (int mt = 0; mt < 4; ++mt) {
            pkv::mma_f16_16816(o[2 * mt], a0, a1, a2, a3, vf[mt][0], vf[mt][2]);
            pkv::mma_f16_16816(o[2 * mt + 1], a0, a1, a2, a3, vf[mt][1], vf[mt][3]);
        }
    }
    pkv::cp_async_wait<0>();
    l_a = quad_sum(l_a);
    l_b = quad_sum(l_b);

    if (SPLIT) {
        // Merge the halves in shared memory (the rings are free once both groups
        // are past their loops): group 1 leaves (m, l, O), group 0 combines.
        __syncthreads();
        float *xo = reinterpret_cast<float *>(ring);          // [group warp][32 values][32 lanes]
        float *xm = xo + S::kGroupWarps * 32 * 32;             // [group warp][m_a, m_b, l_a, l_b][32 lanes]
        const int wg = warp % S::kGroupWarps;
        if (group == 1) {
#pragma unroll
            for (int i = 0; i < 32; ++i) xo[(wg * 32 + i) * 32 + lane] = o[i / 4][i % 4];
            xm[(wg * 4 + 0) * 32 + lane] = m_a;
            xm[(wg * 4 + 1) * 32 + lane] = m_b;
            xm[(wg * 4 + 2) * 32 + lane] = l_a;
            xm[(wg * 4 + 3) * 32 + lane] = l_b;
        }
        __syncthreads();
        if (group == 1) return;
        // Group 0 holds block 0, so its maxima are finite for every stored row.
        const float m1a = xm[(wg * 4 + 0) * 32 + lane], m1b = xm[(wg * 4 + 1) * 32 + lane];
        const float big_a = fmaxf(m_a, m1a), big_b = fmaxf(m_b, m1b);
        const float w0a = pkv::exp2_approx(m_a - big_a), w0b = pkv::exp2_approx(m_b - big_b);
        const float w1a = m1a == -INFINITY ? 0.f : pkv::exp2_approx(m1a - big_a);
        const float w1b = m1b == -INFINITY ? 0.f : pkv::exp2_approx(m1b - big_b);
        l_a = l_a * w0a + xm[(wg * 4 + 2) * 32 + lane] * w1a;
        l_b = l_b * w0b + xm[(wg * 4 + 3) * 32 + lane] * w1b;
#pragma unroll
        for (int dt = 0; dt < 8; ++dt) {
            o[dt][0] = o[dt][0] * w0a + xo[(wg * 32 + 4 * dt + 0) * 32 + lane] * w1a;
            o[dt][1] = o[dt][1] * w0a + xo[(wg * 32 + 4 * dt + 1) * 32 + lane] * w1a;
            o[dt][2] = o[dt][2] * w0b + xo[(wg * 32 + 4 * dt + 2) * 32 + lane] * w1b;
            o[dt][3] = o[dt][3] * w0b + xo[(wg * 32 + 4 * dt + 3) * 32 + lane] * w1b;
        }
    }
    if (token_a < a.tokens) {
        __half *dst = a.out + token_a * a.out_stride + head * kHeadDim + 2 * t;
#pragma unroll
        for (int dt = 0; dt < 8; ++dt) {
            *reinterpret_cast<__half2 *>(dst + 8 * dt) =
                __floats2half2_rn(__fdiv_rn(o[dt][0], l_a), __fdiv_rn(o[dt][1], l_a));
        }
    }
    if (token_b < a.tokens) {
        __half *dst = a.out + token_b * a.out_stride + head * kHeadDim + 2 * t;
#pragma unroll
        for (int dt = 0; dt < 8; ++dt) {
            *reinterpret_cast<__half2 *>(dst + 8 * dt) =
                __floats2half2_rn(__fdiv_rn(o[dt][2], l_b), __fdiv_rn(o[dt][3], l_b));
        }
    }
}

// SMs of the current device (cached per device).
int sm_count() {
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

extern "C" int pkv_prefill_attention_mma(const void *pool, int32_t num_blocks, int32_t layer, const void *query,
                                     int64_t query_stride, const int32_t *blocks, int32_t start, int32_t tokens,
                                     void *out, int64_t out_stride, int32_t *error_flag, void *stream) {
    pkv::clear_error();
    if (pool == nullptr || query == nullptr || blocks == nullptr || out == nullptr || error_flag == nullptr) {
        return pkv::fail(PKV_VALUE_ERROR, "prefill attention: null pointer argument");
    }
    if (layer < 0 || layer >= PKV_LAYERS) {
        return pkv::fail(PKV_VALUE_ERROR, "layer_index must identify one of the 22 decoder layers");
    }
    if (num_blocks < 1 || static_cast<int64_t>(PKV_LAYERS) * 2 * num_blocks * kBlockTokens > INT32_MAX) {
        return pkv::fail(PKV_VALUE_ERROR, "prefill attention: pool block count out of range");
    }
    if (tokens < 1 || start < 0 || static_cast<int64_t>(start) + tokens > PKV_CONTEXT_LIMIT) {
        return pkv::fail(PKV_VALUE_ERROR, "prefill attention: the chunk must hold 1 or more tokens at positions below 2048");
    }
    const int64_t row = static_cast<int64_t>(kQueryHeads) * kHeadDim;
    if ((reinterpret_cast<uintptr_t>(pool) & 15) || (reinterpret_cast<uintptr_t>(query) & 3) ||
        (reinterpret_cast<uintptr_t>(out) & 3) || (reinterpret_cast<uintptr_t>(blocks) & 3) || query_stride % 2 ||
        out_stride % 2 || query_stride < row || out_stride < row) {
        return pkv::fail(PKV_VALUE_ERROR, "prefill attention: misaligned tensor");
    }
    PrefillArgs args;
    args.pool = static_cast<const __half *>(pool);
    args.query = static_cast<const __half *>(query);
    args.out = static_cast<__half *>(out);
    args.blocks = blocks;
    args.query_stride = query_stride;
    args.out_stride = out_stride;
    args.num_blocks = num_blocks;
    args.layer = layer;
    args.start = start;
    args.tokens = tokens;
    args.error_flag = error_flag;
    cudaLaunchConfig_t config = {};
    // Whole 16-token tiles when they fill at least one wave of two CTAs per
    // SM, else split tiles (twice the CTAs).
    const int whole = (tokens + Shape<false>::kTileTokens - 1) / Shape<false>::kTileTokens * kKvHeads;
    const bool split = whole < 2 * sm_count();
    const int tile_tokens = split ? Shape<true>::kTileTokens : Shape<false>::kTileTokens;
    config.gridDim = dim3((tokens + tile_tokens - 1) / tile_tokens * kKvHeads);
    config.blockDim = dim3(kThreads);
    config.dynamicSmemBytes = 0;
    config.stream = static_cast<cudaStream_t>(stream);
    const cudaError_t e = split ? cudaLaunchKernelEx(&config, prefill_attention_kernel<true>, args)
                                : cudaLaunchKernelEx(&config, prefill_attention_kernel<false>, args);
    if (e != cudaSuccess) {
        return pkv::fail(PKV_CUDA_ERROR, std::string("prefill attention launch failed: ") + cudaGetErrorString(e));
    }
    return PKV_OK;
}

namespace pkv {
int launch_prefill_attention_tc(const void *pool, int32_t num_blocks, int32_t layer, const void *query,
                                int64_t query_stride, const int32_t *blocks, int32_t start, int32_t tokens,
                                void *out, int64_t out_stride, int32_t *error_flag, cudaStream_t stream);
}

extern "C" int pkv_prefill_attention(const void *pool, int32_t num_blocks, int32_t layer, const void *query,
                                        int64_t query_stride, const int32_t *blocks, int32_t start, int32_t tokens,
                                        void *out, int64_t out_stride, int32_t *error_flag, void *stream) {
    pkv::clear_error();
    if (pool == nullptr || query == nullptr || blocks == nullptr || out == nullptr || error_flag == nullptr) {
        return pkv::fail(PKV_VALUE_ERROR, "prefill attention: null pointer argument");
    }
    if (layer < 0 || layer >= PKV_LAYERS) {
        return pkv::fail(PKV_VALUE_ERROR, "layer_index must identify one of the 22 decoder layers");
    }
    if (num_blocks < 1 || static_cast<int64_t>(PKV_LAYERS) * 2 * num_blocks * kBlockTokens > INT32_MAX) {
        return pkv::fail(PKV_VALUE_ERROR, "prefill attention: pool block count out of range");
    }
    if (tokens < 1 || start < 0 || static_cast<int64_t>(start) + tokens > PKV_CONTEXT_LIMIT) {
        return pkv::fail(PKV_VALUE_ERROR, "prefill attention: the chunk must hold 1 or more tokens at positions below 2048");
    }
    const int64_t row = static_cast<int64_t>(kQueryHeads) * kHeadDim;
    if ((reinterpret_cast<uintptr_t>(pool) & 15) || (reinterpret_cast<uintptr_t>(query) & 15) ||
        (reinterpret_cast<uintptr_t>(out) & 15) || (reinterpret_cast<uintptr_t>(blocks) & 3) || query_stride % 8 ||
        out_stride % 8 || query_stride < row || out_stride < row) {
        return pkv::fail(PKV_VALUE_ERROR, "prefill attention: misaligned tensor");
    }
    return pkv::launch_prefill_attention_tc(pool, num_blocks, layer, query, query_stride, blocks, start, tokens, out,
                                            out_stride, error_flag, static_cast<cudaStream_t>(stream));
}
