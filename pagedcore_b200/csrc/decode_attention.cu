// Batched one-token block-table decode attention with GQA on sm_100a.
//
// Replaces PagedCore's paged_attention (src/pagedcore/attention.py:14-53),
// which for one request and one layer computes, in FP32 from FP16 pages,
//   o[h] = sum_t softmax_t(q[h] . k[t, h/8] * 0.125) v[t, h/8]
// and rounds once to FP16.  A whole batch of requests is served at once.
//
// Work split - balanced split-K over the batch's 16-token blocks.  The batch's
// block tables are concatenated into one flat list (flat[prefix[b] + j] =
// physical block of logical block j of row b); CTA g owns one contiguous
// piece of it (the plan's Partition: normally [g*W, (g+1)*W)), which may
// cover the tail of one row, whole short rows and the head of another, so
// every CTA streams the same number of KV bytes whatever the ragged lengths.
// With a piece table the host sizes the pieces (blocks, row switches, and the
// measured speed of each slot), and when the grid is one full wave the CTAs
// claim slots by the SM they run on (slot s * k + j is the j-th CTA on SM s):
// the hardware places CTAs on SMs in a different order at every launch, while
// an SM's speed stays the same from launch to launch, so only SM-bound slots
// can be given work by speed.
// Warp w of a CTA serves KV head w and its 8 query heads (GQA).
//
// Data movement - each warp runs its own TMA pipeline of STAGES stages: per
// block, two 2 KiB boxes (the 16 K rows and 16 V rows of its head, 128 B
// each, 512 B apart in the pool) land in shared memory with the 128-byte
// swizzle, so ldmatrix reads are bank-conflict free; the boxes carry an L2
// evict-first policy (the KV stream is read once).  The piece's block ids
// are held in registers 32 at a time and row boundaries come from a register
// window of 32 rows, so no refill waits on a global load; each row's Q, RoPE
// pairs and new token are prefetched into L2 when the CTA starts.  Waits are
// bounded.
//
// Math - tensor-core tiles (mma.sync m16n8k16, FP16 in, FP32 accumulate):
//   S^T[16 tok x 8 heads]  = K[16 x 64] . Q^T[64 x 8]         (4 MMAs)
//   O^T[64 dims x 8 heads] += V^T[64 x 16] . P^T[16 x 8]      (2 x 4 MMAs)
// so the 8-head GQA group fills the N=8 side exactly; the S^T accumulator
// becomes the P^T operand with two movmatrix transposes.  Softmax is the
// online (running max) form in base 2 with FP32 state.  The reference keeps
// P in FP32 (attention.py:46-52); here the FP32 weight p = 2^(s - m + 15)
// (<= 2^15, so weights down to ~2^-24 of the row maximum stay normal FP16
// numbers) is split into hi = fp16(p) and lo = fp16(p - hi), and O^T takes
// both P.V products, which carries P to about 2^-22: FP32 class, where one
// FP16 operand alone would carry 2^-11.  The normaliser l sums the FP32
// weights.  Unwritten slots of a row's
// last block may hold anything (the pool is uninitialised; tests fill it with
// NaN): their scores are masked to -inf and their V rows are zeroed in shared
// memory before the PV MMA.
//
// Split rows - a row inside one CTA is normalised and written as FP16
// directly.  A row split across CTAs leaves (m, l, O) partials at index
// row + cta (unique: along the CTA order the (row, cta) pairs form a
// monotone staircase, so row + cta strictly increases), and
// decode_combine_kernel merges them, launched as a programmatic dependent of
// the split kernel so its launch overlaps the split kernel's tail.  (A merge
// inside the split kernel by the last piece of each row, counted with
// atomics, measured 1.5 us per layer slower: it puts a merge on the tail of
// every CTA.)
//
// The fused decode-layer variant also does the layer's KV append: it applies
// RoPE to Q (every CTA of the row, in registers) and to the new token's K
// (bit-exact with dense.py:48-59), writes K and V of the new token to the
// pool slot (kv_cache.py:244-245) and patches that slot of the staged tile in
// shared memory, so attention sees the token in the same launch.

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>
#include <cstdlib>
#include <mutex>
#include <string>
#include <unordered_map>

#include "pagedkv.h"
#include "ptx.cuh"
#include "status.h"
#include "tensor_maps.h"

namespace {

constexpr int kHeadDim = PKV_HEAD_DIM;
constexpr int kKvHeads = PKV_KV_HEADS;
constexpr int kQueryHeads = PKV_QUERY_HEADS;
constexpr int kGroup = kQueryHeads / kKvHeads;  // 8 query heads per KV head
constexpr int kBlockTokens = PKV_BLOCK_TOKENS;
constexpr int kRopeHalf = kHeadDim / 2;
constexpr int kRowBytes = kHeadDim * 2;                  // 128 B: one head of one token
constexpr int kTileBytes = kBlockTokens * kRowBytes;     // 2 KiB: one head of one block
constexpr int kStageBytes = 2 * kTileBytes;              // K tile + V tile
constexpr int kWarps = kKvHeads;
constexpr int kThreads = kWarps * 32;
constexpr int kMaxStages = 4;  // mbarriers reserved per warp (the pipeline depth used)
constexpr uint32_t kWaitPolls = 1u << 24;
constexpr float kScaleLog2 = 0.125f * 1.4426950408889634f;  // 64^-0.5 * log2(e)
constexpr float kWeightShift = 15.0f;                       // P scaled by 2^15 before FP16
constexpr int kPartialFloats = kQueryHeads * (kHeadDim + 2);
// Slot claims: one counter per SM (up to kClaimWords SMs); two such sets,
// used by layers of alternate parity.  The combine kernel zeroes a launch's
// set once the split kernel has completed.
constexpr int kClaimWords = 256;
constexpr int kCombineThreads = 256;
static_assert(kClaimWords <= kCombineThreads, "one combine CTA zeroes a claim set");

template <int STAGES>
constexpr int smem_bytes() {
    return kWarps * STAGES * kStageBytes + 1024;  // + alignment slack
}

struct LayerArgs {
    const __half *query;       // [B][32][64], rows query_stride apart (rotated unless FUSED)
    int64_t query_stride;
    const __half *key_new;     // FUSED: new token's unrotated K [B][4][64]
    const __half *value_new;   // FUSED: new token's V [B][4][64]
    int64_t new_stride;        // elements between rows of key_new / value_new
    const __half *rope_cos;    // FUSED: FP16 [2048][32]
    const __half *rope_sin;
    __half *pool;              // FUSED: pool base, for the new token's K/V
    const int32_t *lengths;    // [B]
    const int32_t *prefix;     // [B+1]
    const int32_t *flat;       // [total_blocks]
    int32_t batch;
    int32_t total_blocks;
    int32_t blocks_per_cta;    // size of the big pieces
    int32_t big_ctas;          // number of big pieces
    int32_t tail_blocks;       // size of the tail pieces
    int32_t num_blocks;
    int32_t layer;
    __half *out;               // [B][32][64], rows out_stride apart
    int64_t out_stride;
    float *part_o;             // [(B + grid)][32][64]
    float *part_ml;            // [(B + grid)][32][2]
    unsigned *cta_ns;          // [grid][4]: each warp's wall time, accumulated over launches (or null)
    int32_t *claims;           // [2][kClaimWords]: per-SM slot counters (or null)
    int32_t sm_slots;          // > 0: CTAs take the slots of the SM they run on (sm_slots per SM)
    const int32_t *pieces;     // [grid][4]: begin, end, first row and that row's first block of each
                               // CTA's piece (or null: the Partition below, rows found by search)
    int32_t *error_flag;
    int32_t early_kv;          // FUSED: start streaming K/V before the previous kernel completes
};

// The plan's partition of the flat block list into one contiguous piece per
// CTA when no piece tables are given: `big` pieces of `per_cta` blocks, then
// pieces of `tail` blocks (big == grid: all pieces per_cta).  pkv_decode_plan
// makes r pieces of q + 1 blocks and grid - r of q, one per CTA slot.
struct Partition {
    int32_t total;
    int32_t per_cta;
    int32_t big;
    int32_t tail;
};

__host__ __device__ __forceinline__ void piece_range(const Partition &p, int piece, int &begin, int &end) {
    if (piece < p.big) {
        begin = piece * p.per_cta;
        end = begin + p.per_cta;
    } else {
        begin = p.big * p.per_cta + (piece - p.big) * p.tail;
        end = begin + p.tail;
    }
    if (end > p.total) end = p.total;
}

// The piece holding global block `block`.
__host__ __device__ __forceinline__ int piece_of(const Partition &p, int block) {
    const int split = p.big * p.per_cta;
    return block < split ? block / p.per_cta : p.big + (block - split) / p.tail;
}

__device__ __forceinline__ float warp_max8(float v) {
    // Reduce over the 8 lanes that share lane % 4 (the token rows of a fragment).
    v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 4));
    v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 8));
    v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 16));
    return v;
}

__device__ __forceinline__ float warp_sum8(float v) {
    v += __shfl_xor_sync(0xffffffffu, v, 4);
    v += __shfl_xor_sync(0xffffffffu, v, 8);
    v += __shfl_xor_sync(0xffffffffu, v, 16);
    return v;
}

// One FP16 RoPE step, as the reference's eager ops round it:
// fp16(fp16(x * c) + fp16(r * s)) with r = -rot or rot, on a half2 pair.
__device__ __forceinline__ uint32_t rope_half2(uint32_t x, uint32_t rot, bool negate, uint32_t c, uint32_t s) {
    const float2 xf = __half22float2(*reinterpret_cast<const __half2 *>(&x));
    float2 rf = __half22float2(*reinterpret_cast<const __half2 *>(&rot));
    const float2 cf = __half22float2(*reinterpret_cast<const __half2 *>(&c));
    const float2 sf = __half22float2(*reinterpret_cast<const __half2 *>(&s));
    if (negate) {
        rf.x = -rf.x;
        rf.y = -rf.y;
    }
    const float a0 = __half2float(__float2half_rn(xf.x * cf.x));
    const float a1 = __half2float(__float2half_rn(xf.y * cf.y));
    const float b0 = __half2float(__float2half_rn(rf.x * sf.x));
    const float b1 = __half2float(__float2half_rn(rf.y * sf.y));
    __half2 r = __halves2half2(__float2half_rn(a0 + b0), __float2half_rn(a1 + b1));
    return *reinterpret_cast<uint32_t *>(&r);
}

__device__ __forceinline__ uint32_t ld32(const __half *p) { return *reinterpret_cast<const uint32_t *>(p); }

// One step of the split-partial merge, in a fixed operation order: the running (M, L, A) of a head absorbs a partial (m, l, o) as
//   M' = max(M, m),  L' = L a + l b,  A' = A a + o b,  a = 2^(M - M'),  b = 2^(m - M').
struct MergeWeights {
    float a, b;
};

__device__ __forceinline__ MergeWeights merge_weights(float &M, float m) {
    const float mn = fmaxf(M, m);
    const MergeWeights w{pkv::exp2_approx(M - mn), pkv::exp2_approx(m - mn)};
    M = mn;
    return w;
}

__device__ __forceinline__ float merge_value(float A, float o, MergeWeights w) {
    return __fmaf_rn(A, w.a, __fmul_rn(o, w.b));
}

// Fetch one block's K and V boxes of KV head `head` into a pipeline stage
// (called by one lane).  An out-of-range block id sets the error flag and
// completes the stage's phase without data, so no waiter is left behind.
__device__ __forceinline__ void issue_block(const CUtensorMap *map, int32_t block, int32_t num_blocks,
                                            int32_t k_rows, int32_t v_rows, int head, uint32_t dst,
                                            uint32_t bar, int32_t *error_flag, uint64_t policy,
                                            uint32_t after = 0u) {
    // `after` ties the issue to a value computed from the stage's last reads.
    asm volatile("" ::"r"(after) : "memory");
    if (block < 0 || block >= num_blocks) {
        atomicOr(error_flag, PKV_DEVICE_BAD_BLOCK);
        pkv::mbar_arrive(bar);
        return;
    }
    pkv::mbar_arrive_expect_tx(bar, kStageBytes);
    pkv::tma_load_3d_hint(dst, map, 0, head, k_rows + block * kBlockTokens, bar, policy);
    pkv::tma_load_3d_hint(dst + kTileBytes, map, 0, head, v_rows + block * kBlockTokens, bar, policy);
}

// Per-row inputs of a segment.  The head (where the row ends in the flat
// list, and its length) comes from a row window held in registers; the body
// (Q fragments, RoPE pairs, the new token) is loaded one row ahead, from L2:
// the kernel prefetches the bodies of its range's rows into L2 at its start,
// so row switches do not wait on DRAM latency behind the KV stream.
struct RowHead {
    int32_t last;    // prefix[row + 1]
    int32_t length;  // lengths[row]
};

// Lane j holds prefix[base + j + 1] and lengths[base + j]: the heads of rows
// base .. base + 31, read by shuffle.
struct RowWindow {
    int32_t base;
    int32_t last;
    int32_t length;
};

struct RowBody {
    uint32_t q[4][2];      // raw Q fragments of this warp's 8 heads
    uint32_t cs[4], sn[4]; // FUSED: cos/sin pairs for Q dims (16*ks + 8*h + 2t) & 31, index 2*ks + h
    uint32_t kcs, ksn;     // FUSED: cos/sin pair for the new K's dims (2*lane) & 31
    uint32_t k_own, k_partner, v_own;  // FUSED: new token's K (dims 2*lane, partner) and V
    int32_t last_block;    // FUSED: flat[last - 1]
};

__device__ __forceinline__ RowWindow load_row_window(const LayerArgs &a, int base, int lane) {
    RowWindow w;
    w.base = base;
    const int r = base + lane;
    w.last = r < a.batch ? a.prefix[r + 1] : INT32_MAX;
    w.length = r < a.batch ? a.lengths[r] : 0;
    return w;
}

// Head of `row` (warp-uniform, base <= row < base + 32).
__device__ __forceinline__ RowHead window_head(const RowWindow &w, int row) {
    RowHead h;
    h.last = __shfl_sync(0xffffffffu, w.last, row - w.base);
    h.length = __shfl_sync(0xffffffffu, w.length, row - w.base);
    return h;
}

__device__ __forceinline__ int clamp_position(const LayerArgs &a, int length, int lane) {
    int pos = length - 1;
    if (pos < 0 || pos >= PKV_CONTEXT_LIMIT) {
        if (lane == 0) atomicOr(a.error_flag, PKV_DEVICE_BAD_POSITION);
        pos = 0;
    }
    return pos;
}

// Prefetch into L2 the lines row_body will read for `row` and KV head `warp`.
template <bool FUSED>
__device__ __forceinline__ void prefetch_row(const LayerArgs &a, int row, int length, int last, int warp) {
    const char *q = reinterpret_cast<const char *>(a.query + row * a.query_stride + warp * kGroup * kHeadDim);
#pragma unroll
    for (int offset = 0; offset < kGroup * kRowBytes; offset += 128) pkv::prefetch_l2(q + offset);
    pkv::prefetch_l2(q + kGroup * kRowBytes - 1);
    if constexpr (FUSED) {
        const __half *kn = a.key_new + row * a.new_stride + warp * kHeadDim;
        const __half *vn = a.value_new + row * a.new_stride + warp * kHeadDim;
        pkv::prefetch_l2(kn);
        pkv::prefetch_l2(kn + kHeadDim - 1);
        pkv::prefetch_l2(vn);
        pkv::prefetch_l2(vn + kHeadDim - 1);
        const int pos = length >= 1 && length <= PKV_CONTEXT_LIMIT ? length - 1 : 0;
        pkv::prefetch_l2(a.rope_cos + pos * kRopeHalf);
        pkv::prefetch_l2(a.rope_cos + pos * kRopeHalf + kRopeHalf - 1);
        pkv::prefetch_l2(a.rope_sin + pos * kRopeHalf);
        pkv::prefetch_l2(a.rope_sin + pos * kRopeHalf + kRopeHalf - 1);
        if (last >= 1 && last <= a.total_blocks) pkv::prefetch_l2(a.flat + last - 1);
    }
}

// Lane j >= 1 prefetches the body of window row base + j if that row starts
// inside [.., end) (row base is loaded directly).
template <bool FUSED>
__device__ __forceinline__ void prefetch_window(const LayerArgs &a, const RowWindow &w, int end, int lane, int warp) {
    const int start = __shfl_up_sync(0xffffffffu, w.last, 1);  // prefix[base + lane]
    if (lane >= 1 && w.base + lane < a.batch && start < end) prefetch_row<FUSED>(a, w.base + lane, w.length, w.last, warp);
}

template <bool FUSED>
__device__ __forceinline__ void row_body(const LayerArgs &a, int row, const RowHead &h, int warp, int lane,
                                         RowBody &m) {
    const int g = lane >> 2, t = lane & 3;
    const __half *q = a.query + row * a.query_stride + (warp * kGroup + g) * kHeadDim;
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {
        m.q[ks][0] = ld32(q + 16 * ks + 2 * t);
        m.q[ks][1] = ld32(q + 16 * ks + 8 + 2 * t);
    }
    if constexpr (FUSED) {
        const int pos = clamp_position(a, h.length, lane);
        const __half *cs = a.rope_cos + pos * kRopeHalf;
        const __half *sn = a.rope_sin + pos * kRopeHalf;
#pragma unroll
        for (int ks = 0; ks < 2; ++ks) {
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
                const int d = 16 * ks + 8 * hh + 2 * t;
                m.cs[2 * ks + hh] = ld32(cs + d);
                m.sn[2 * ks + hh] = ld32(sn + d);
            }
        }
        const int d = 2 * lane;
        const int dk = d & (kRopeHalf - 1);
        m.kcs = ld32(cs + dk);
        m.ksn = ld32(sn + dk);
        const __half *kn = a.key_new + row * a.new_stride + warp * kHeadDim;
        m.k_own = ld32(kn + d);
        m.k_partner = ld32(kn + ((d + kRopeHalf) & (kHeadDim - 1)));
        m.v_own = ld32(a.value_new + row * a.new_stride + warp * kHeadDim + d);
        m.last_block = h.last >= 1 && h.last <= a.total_blocks ? a.flat[h.last - 1] : -1;
    }
}

// Write this warp's (m, l, O) of its 8 heads to partial slot `index`.  In the
// MMA fragment layout lane (g, t) holds heads head0 = 8*warp + 2t and
// head0 + 1, dims 16*mt + g and 16*mt + g + 8 (o[mt][0|2] for head0,
// o[mt][1|3] for head0 + 1).
__device__ __forceinline__ void store_partial(const LayerArgs &a, int64_t index, int head0, int g,
                                              const float (&o)[4][4], float m0, float l0, float m1, float l1) {
    float *po = a.part_o + index * kQueryHeads * kHeadDim;
#pragma unroll
    for (int mt = 0; mt < 4; ++mt) {
        const int d = 16 * mt + g;
        po[head0 * kHeadDim + d] = o[mt][0];
        po[(head0 + 1) * kHeadDim + d] = o[mt][1];
        po[head0 * kHeadDim + d + 8] = o[mt][2];
        po[(head0 + 1) * kHeadDim + d + 8] = o[mt][3];
    }
    if (g == 0) {
        *reinterpret_cast<float4 *>(a.part_ml + index * kQueryHeads * 2 + head0 * 2) = make_float4(m0, l0, m1, l1);
    }
}

// Normalise and round to FP16 into out[row].
__device__ __forceinline__ void write_output(const LayerArgs &a, int row, int head0, int g, const float (&o)[4][4],
                                             float l0, float l1) {
    __half *dst = a.out + row * a.out_stride;
#pragma unroll
    for (int mt = 0; mt < 4; ++mt) {
        const int d = 16 * mt + g;
        dst[head0 * kHeadDim + d] = __float2half_rn(__fdiv_rn(o[mt][0], l0));
        dst[(head0 + 1) * kHeadDim + d] = __float2half_rn(__fdiv_rn(o[mt][1], l1));
        dst[head0 * kHeadDim + d + 8] = __float2half_rn(__fdiv_rn(o[mt][2], l0));
        dst[(head0 + 1) * kHeadDim + d + 8] = __float2half_rn(__fdiv_rn(o[mt][3], l1));
    }
}

// The slot of this CTA when slots are claimed per SM (warp 0, all lanes).
// The pieces of SM s are slots s * k .. s * k + k - 1 (k = sm_slots), so the
// work an SM gets, and the speed the host measures for a slot, belong to one
// SM whatever order the hardware places the CTAs in.  A CTA takes the next
// slot of its own SM; one that finds them all taken (an SM hosting more CTAs
// than k) takes a slot left by another SM in one pass over the counters.
// Counters only grow during a launch and there are as many slots as CTAs, so
// every CTA gets exactly one: -1 means the counters were not zero at launch.
__device__ __forceinline__ int claim_slot(const LayerArgs &a, int32_t *claims, int lane) {
    const int k = a.sm_slots;
    const int groups = static_cast<int>(gridDim.x) / k;
    unsigned smid;
    asm volatile("mov.u32 %0, %%smid;" : "=r"(smid));
    int slot = -1;
    if (lane == 0 && smid < static_cast<unsigned>(groups)) {
        const int c = atomicAdd(claims + smid, 1);
        if (c < k) slot = static_cast<int>(smid) * k + c;
    }
    slot = __shfl_sync(0xffffffffu, slot, 0);
    for (int base = 0; slot < 0 && base < groups; base += 32) {
        const int s = base + lane;
        const bool open = s < groups && *reinterpret_cast<volatile int32_t *>(claims + s) < k;
        unsigned candidates = __ballot_sync(0xffffffffu, open);
        while (candidates != 0 && slot < 0) {
            const int pick = base + __ffs(candidates) - 1;
            candidates &= candidates - 1;
            int got = -1;
            if (lane == 0) {
                const int c = atomicAdd(claims + pick, 1);
                if (c < k) got = pick * k + c;
            }
            slot = __shfl_sync(0xffffffffu, got, 0);
        }
    }
    return slot;
}

// One CTA's piece: piece `slot` of the table (or of the partition).
template <int STAGES, bool FUSED>
__device__ __forceinline__ void decode_cta(const CUtensorMap &pool_map, const LayerArgs &a, const int slot,
                                           const uint64_t started) {
    extern __shared__ uint8_t smem_raw[];
    __shared__ __align__(8) uint64_t barriers[kWarps * kMaxStages];

    int begin, end, row = 0, row_first = 0;
    if (a.pieces != nullptr) {
        const int4 piece = reinterpret_cast<const int4 *>(a.pieces)[slot];
        begin = piece.x;
        end = piece.y;
        row = piece.z;
        row_first = piece.w;
        if (begin < 0 || end > a.total_blocks || row < 0 || row >= a.batch || row_first > begin) {
            if (threadIdx.x == 0) atomicOr(a.error_flag, PKV_DEVICE_BAD_BLOCK);
            return;
        }
    } else {
        piece_range(Partition{a.total_blocks, a.blocks_per_cta, a.big_ctas, a.tail_blocks}, slot, begin, end);
    }
    if (begin >= end) return;

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int g = lane >> 2;  // fragment row group
    const int t = lane & 3;   // fragment column pair
    uint8_t *smem = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    uint8_t *warp_tiles = smem + warp * STAGES * kStageBytes;
    const uint32_t tiles = pkv::smem_addr(warp_tiles);
    const uint32_t bar0 = pkv::smem_addr(&barriers[warp * kMaxStages]);

    if (lane == 0) {
        for (int s = 0; s < STAGES; ++s) pkv::mbar_init(bar0 + 8 * s, 1);
        pkv::fence_barrier_init();
    }
    __syncwarp();

    // Rows of this head's K and V boxes in the 3-D view of the pool
    // (dim 64, kv head 4, pool row = ((layer*2 + kv)*num_blocks + block)*16).
    const int32_t k_rows = (a.layer * 2 + 0) * a.num_blocks * kBlockTokens;
    const int32_t v_rows = (a.layer * 2 + 1) * a.num_blocks * kBlockTokens;

    const uint64_t policy = pkv::l2_policy_evict_first();  // the KV stream is read once

    // Producer state: the next global block to fetch (tracked by every lane;
    // lane 0 issues).  The physical block ids of the range are held in
    // registers, 32 at a time (lane j holds the window's j-th id), and the
    // next window is loaded a whole window ahead, so a refill never waits on
    // a global load of the block table.
    int next_fetch = begin;
    int ids = begin + lane < end ? a.flat[begin + lane] : 0;
    int ids_next = begin + 32 + lane < end ? a.flat[begin + 32 + lane] : 0;
    {
        const int n = min(STAGES, end - begin);
        for (int s = 0; s < n; ++s) {
            const int32_t block = __shfl_sync(0xffffffffu, ids, s);
            if (lane == 0) {
                issue_block(&pool_map, block, a.num_blocks, k_rows, v_rows, warp, tiles + s * kStageBytes,
                            bar0 + 8 * s, a.error_flag, policy);
            }
            ++next_fetch;
        }
    }
    if (a.early_kv) asm volatile("griddepcontrol.wait;" ::: "memory");

    // First row of the range (the largest b with prefix[b] <= begin) and its
    // first block: from the piece table, else a 32-way search.
    if (a.pieces == nullptr) {
        int lo = 0, hi = a.batch - 1, lo_value = 0;
        while (hi > lo) {
            const int step = (hi - lo + 32) / 32;
            const int probe = lo + lane * step;
            const int value = probe <= hi ? a.prefix[probe] : INT32_MAX;
            const unsigned mask = __ballot_sync(0xffffffffu, value <= begin);
            const int best = 31 - __clz(mask);  // lane 0 probes lo, whose prefix is <= begin
            lo_value = __shfl_sync(0xffffffffu, value, best);
            lo += best * step;
            hi = min(hi, lo + step - 1);
        }
        row = lo;
        row_first = lo_value;
    }

    RowWindow rows = load_row_window(a, row, lane);
    prefetch_window<FUSED>(a, rows, end, lane, warp);
    RowHead head = window_head(rows, row);
    RowBody body, body1;
    row_body<FUSED>(a, row, head, warp, lane, body);

    int consumed = 0;
    bool failed = false;        // a bounded wait ran out
    bool failed_range = false;  // the range runs past the last row
    int i = begin;
    while (true) {
        const int row_last = head.last;
        const int seg_end = min(end, row_last);
        const int length = head.length;
        const bool has_next = row_last < end;
        // Load the next row's body now; it is used at the next row switch.
        RowHead head1{0, 0};
        if (has_next && row + 1 >= a.batch) {
            // prefix[batch] < end: the caller's prefix and total_blocks disagree.
            if (lane == 0) atomicOr(a.error_flag, PKV_DEVICE_BAD_BLOCK);
            failed_range = true;
        } else if (has_next) {
            if (row + 1 - rows.base >= 32) {  // past the window (a range of over 32 rows)
                rows = load_row_window(a, row + 1, lane);
                prefetch_window<FUSED>(a, rows, end, lane, warp);
            }
            head1 = window_head(rows, row + 1);
            row_body<FUSED>(a, row + 1, head1, warp, lane, body1);
        }

        // Q^T fragments (B operand): lane holds dims 16ks + 2t + {0,1} and
        // 16ks + 8 + 2t + {0,1} of head 8*warp + g.
        uint32_t qf[4][2];
        uint32_t new_k = 0, new_v = 0;
        int new_slot = -1;
        if constexpr (FUSED) {
            // RoPE of Q in registers: dims d < 32 pair with d + 32 (k-step ks ^ 2).
#pragma unroll
            for (int ks = 0; ks < 4; ++ks) {
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const int c = 2 * (ks & 1) + h;
                    qf[ks][h] = rope_half2(body.q[ks][h], body.q[ks ^ 2][h], ks < 2, body.cs[c], body.sn[c]);
                }
            }
            if (seg_end == row_last) {
                // This CTA holds the row's last block: rotate the new K (lane owns
                // dims 2*lane, 2*lane+1 of head `warp`) and write K/V to the pool.
                const int d = 2 * lane;
                new_k = rope_half2(body.k_own, body.k_partner, d < kRopeHalf, body.kcs, body.ksn);
                new_v = body.v_own;
                new_slot = (length - 1) & (kBlockTokens - 1);
                const int32_t block = body.last_block;
                if (block >= 0 && block < a.num_blocks && length >= 1 && length <= PKV_CONTEXT_LIMIT) {
                    const int64_t base =
                        (((static_cast<int64_t>(a.layer) * 2) * a.num_blocks + block) * kBlockTokens + new_slot) *
                            (kKvHeads * kHeadDim) +
                        warp * kHeadDim + d;
                    const int64_t v_offset = static_cast<int64_t>(a.num_blocks) * kBlockTokens * kKvHeads * kHeadDim;
                    *reinterpret_cast<uint32_t *>(a.pool + base) = new_k;
                    *reinterpret_cast<uint32_t *>(a.pool + base + v_offset) = new_v;
                } else {
                    new_slot = -1;
                    if (lane == 0) atomicOr(a.error_flag, PKV_DEVICE_BAD_BLOCK);
                }
            }
        } else {
#pragma unroll
            for (int ks = 0; ks < 4; ++ks) {
                qf[ks][0] = body.q[ks][0];
                qf[ks][1] = body.q[ks][1];
            }
        }

        float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
        float o[4][4];
#pragma unroll
        for (int mt = 0; mt < 4; ++mt) o[mt][0] = o[mt][1] = o[mt][2] = o[mt][3] = 0.f;

        for (; i < seg_end; ++i, ++consumed) {
            const int stage = consumed % STAGES;
            const uint32_t parity = (consumed / STAGES) & 1;
            if (!pkv::mbar_wait_bounded(bar0 + 8 * stage, parity, kWaitPolls)) {
                failed = true;
                break;
            }
            const uint32_t ktile = tiles + stage * kStageBytes;
            const uint32_t vtile = ktile + kTileBytes;
            const int valid = min(kBlockTokens, length - (i - row_first) * kBlockTokens);
            uint8_t *stage_tiles = warp_tiles + stage * kStageBytes;
            bool wrote = false;
            if (valid < kBlockTokens) {
                // Zero the V rows of unwritten slots: P is 0 there, but 0 * NaN is NaN.
                uint8_t *vrows = stage_tiles + kTileBytes;
                for (int idx = lane; idx < (kBlockTokens - valid) * 8; idx += 32) {
                    *reinterpret_cast<uint4 *>(vrows + (valid + idx / 8) * kRowBytes + (idx % 8) * 16) =
                        make_uint4(0, 0, 0, 0);
                }
                wrote = true;
            }
            if (FUSED && new_slot >= 0 && i == row_last - 1) {
                // Patch the new token's row of the staged tiles (swizzled 16 B chunks).
                const int chunk = (lane >> 2) ^ (new_slot & 7);
                const int offset = new_slot * kRowBytes + chunk * 16 + (lane & 3) * 4;
                *reinterpret_cast<uint32_t *>(stage_tiles + offset) = new_k;
                *reinterpret_cast<uint32_t *>(stage_tiles + kTileBytes + offset) = new_v;
                wrote = true;
            }
            if (wrote) __syncwarp();

            // K (row-major tokens x dims) and V^T fragments of the whole block.
            uint32_t kf[4][4], vf[4][4];
#pragma unroll
            for (int ks = 0; ks < 4; ++ks) {
                const int mat = lane >> 3;
                const int tok = (lane & 7) + ((mat & 1) << 3);
                const int chunk = 2 * ks + (mat >> 1);
                pkv::ldmatrix_x4(ktile + tok * kRowBytes + ((chunk ^ (tok & 7)) << 4), kf[ks][0], kf[ks][1],
                                 kf[ks][2], kf[ks][3]);
            }
#pragma unroll
            for (int mt = 0; mt < 4; ++mt) {
                const int mat = lane >> 3;
                const int tok = (lane & 7) + ((mat >> 1) << 3);
                const int chunk = 2 * mt + (mat & 1);
                pkv::ldmatrix_x4_trans(vtile + tok * kRowBytes + ((chunk ^ (tok & 7)) << 4), vf[mt][0], vf[mt][1],
                                       vf[mt][2], vf[mt][3]);
            }
            // Hand the stage back to the TMA pipeline before the math.  The
            // refill is issued after every lane holds its fragments (it takes a
            // value computed from all of them, after the warp-wide shuffle that
            // hands lane 0 the block id) and after a proxy fence ordering this
            // stage's generic accesses before it.
            {
                uint32_t ready = 0;
#pragma unroll
                for (int x = 0; x < 4; ++x) {
                    ready ^= kf[x][0] ^ kf[x][1] ^ kf[x][2] ^ kf[x][3] ^ vf[x][0] ^ vf[x][1] ^ vf[x][2] ^ vf[x][3];
                }
                asm volatile("" ::"r"(ready) : "memory");
                pkv::fence_proxy_async_smem();
                if (next_fetch < end) {
                    const int slot = (next_fetch - begin) & 31;
                    if (slot == 0) {
                        // Entering the next window of block ids; prefetch the one after it.
                        ids = ids_next;
                        const int ahead = next_fetch + 32 + lane;
                        ids_next = ahead < end ? a.flat[ahead] : 0;
                    }
                    const int32_t block = __shfl_sync(0xffffffffu, ids, slot);
                    if (lane == 0) {
                        issue_block(&pool_map, block, a.num_blocks, k_rows, v_rows, warp, ktile,
                                    bar0 + 8 * stage, a.error_flag, policy, ready);
                    }
                    ++next_fetch;
                }
            }
            // S^T = K . Q^T over 64 dims (4 k-steps).
            float s[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int ks = 0; ks < 4; ++ks) {
                pkv::mma_f16_16816(s, kf[ks][0], kf[ks][1], kf[ks][2], kf[ks][3], qf[ks][0], qf[ks][1]);
            }
            // s[0]: (token g, head 2t), s[1]: (g, 2t+1), s[2]: (g+8, 2t), s[3]: (g+8, 2t+1)
            const float s0 = g < valid ? s[0] * kScaleLog2 : -INFINITY;
            const float s1 = g < valid ? s[1] * kScaleLog2 : -INFINITY;
            const float s2 = g + 8 < valid ? s[2] * kScaleLog2 : -INFINITY;
            const float s3 = g + 8 < valid ? s[3] * kScaleLog2 : -INFINITY;
            const float mn0 = fmaxf(m0, warp_max8(fmaxf(s0, s2)));
            const float mn1 = fmaxf(m1, warp_max8(fmaxf(s1, s3)));
            const float alpha0 = pkv::exp2_approx(m0 - mn0);
            const float alpha1 = pkv::exp2_approx(m1 - mn1);
            m0 = mn0;
            m1 = mn1;
            const float e0 = pkv::exp2_approx(s0 - mn0 + kWeightShift);
            const float e1 = pkv::exp2_approx(s1 - mn1 + kWeightShift);
            const float e2 = pkv::exp2_approx(s2 - mn0 + kWeightShift);
            const float e3 = pkv::exp2_approx(s3 - mn1 + kWeightShift);
            // P = hi + lo: the FP16 weight and the FP16 rounding of what it
            // left out, so the two P.V MMAs carry P to about 2^-22, FP32 class.
            const __half2 p01 = __floats2half2_rn(e0, e1);
            const __half2 p23 = __floats2half2_rn(e2, e3);
            const float2 f01 = __half22float2(p01);
            const float2 f23 = __half22float2(p23);
            const __half2 r01 = __floats2half2_rn(e0 - f01.x, e1 - f01.y);
            const __half2 r23 = __floats2half2_rn(e2 - f23.x, e3 - f23.y);
            l0 = l0 * alpha0 + (e0 + e2);
            l1 = l1 * alpha1 + (e1 + e3);
#pragma unroll
            for (int mt = 0; mt < 4; ++mt) {
                o[mt][0] *= alpha0;
                o[mt][1] *= alpha1;
                o[mt][2] *= alpha0;
                o[mt][3] *= alpha1;
            }
            // P^T fragments: transpose the (token x head) 8x8 halves.
            const uint32_t b0 = pkv::movmatrix_trans(pkv::pack_half2(p01));
            const uint32_t b1 = pkv::movmatrix_trans(pkv::pack_half2(p23));
            const uint32_t c0 = pkv::movmatrix_trans(pkv::pack_half2(r01));
            const uint32_t c1 = pkv::movmatrix_trans(pkv::pack_half2(r23));

            // O^T += V^T . P^T over 16 tokens (4 dim tiles of 16), hi then lo.
#pragma unroll
            for (int mt = 0; mt < 4; ++mt) {
                pkv::mma_f16_16816(o[mt], vf[mt][0], vf[mt][1], vf[mt][2], vf[mt][3], b0, b1);
                pkv::mma_f16_16816(o[mt], vf[mt][0], vf[mt][1], vf[mt][2], vf[mt][3], c0, c1);
            }
        }
        if (failed) break;

        l0 = warp_sum8(l0);
        l1 = warp_sum8(l1);
        const int head0 = warp * kGroup + 2 * t;  // heads of o[.][0|2] and o[.][1|3]
        if (row_first >= begin && row_last <= end) {  // the whole row is in this CTA's piece
            write_output(a, row, head0, g, o, l0, l1);
        } else {  // merged by decode_combine_kernel
            store_partial(a, static_cast<int64_t>(row) + slot, head0, g, o, m0, l0, m1, l1);
        }
        if (!has_next || failed_range) break;
        ++row;
        row_first = row_last;
        head = head1;
        body = body1;
    }

    if (failed && lane == 0) atomicOr(a.error_flag, PKV_DEVICE_WAIT_TIMEOUT);
    // Let the copies this warp issued and did not consume finish before its
    // shared memory is released (none are left when the range completed).
    for (int c = consumed; c < next_fetch - begin; ++c) {
        pkv::mbar_wait_bounded(bar0 + 8 * (c % STAGES), (c / STAGES) & 1, kWaitPolls);
    }
    // The host may weight the pieces by each slot's measured speed.
    if (lane == 0 && a.cta_ns != nullptr) {
        atomicAdd(&a.cta_ns[4 * slot + warp], static_cast<unsigned>(pkv::global_timer_ns() - started));
    }
}

// Three 4-stage CTAs fit an SM's shared memory; the bound holds registers to
// match (65536 / (3 * 128) = 170 per thread).
template <int STAGES, bool FUSED>
__global__ void __launch_bounds__(kThreads, 3)
    decode_kernel(const __grid_constant__ CUtensorMap pool_map, const __grid_constant__ LayerArgs a) {
    __shared__ int claimed;
    // The kernel is launched as a programmatic dependent of whatever precedes
    // it on the stream, so its launch overlaps that kernel's tail.  Normally
    // nothing here touches memory before that kernel has completed and its
    // writes are visible.  With early_kv the caller guarantees that kernel
    // writes no pool data of this layer and none of the step's tables: the
    // slot claim, the piece, block ids and the first K/V boxes are then
    // fetched before the wait, and everything else (queries, new tokens,
    // outputs) after it.
    //
    // Claim counters: launch n's set is zeroed by its combine after launch
    // n has completed, and the next launch may claim before that combine
    // has run (early_kv), so consecutive launches use alternate sets (by
    // layer parity).  Launch n's set is next used by launch n + 2, whose
    // launch needs launch n + 1's signal, which launch n + 1 gives only after
    // its griddepcontrol.wait, i.e. after launch n's combine has completed.
    // (A launch without early_kv waits before claiming.)
    if (!a.early_kv) asm volatile("griddepcontrol.wait;" ::: "memory");
    const uint64_t started = pkv::global_timer_ns();
    const int lane = threadIdx.x & 31;
    int32_t *const claims = a.sm_slots > 0 ? a.claims + (a.layer & 1) * kClaimWords : nullptr;
    int slot = static_cast<int>(blockIdx.x);
    if (a.sm_slots > 0) {
        if (threadIdx.x < 32) {
            const int got = claim_slot(a, claims, lane);
            if (lane == 0) claimed = got;
        }
        __syncthreads();
        slot = claimed;
        if (slot < 0 && threadIdx.x == 0) atomicOr(a.error_flag, PKV_DEVICE_BAD_BLOCK);
    }
    if (slot >= 0) decode_cta<STAGES, FUSED>(pool_map, a, slot, started);
    // The combine kernel (launched as a programmatic dependent) may start.
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Second pass: one warp per (row, pair of query heads) of a split row merges
// its partials, 16 lanes per head and 4 dims per lane (two heads per warp
// keep the grid to one wave of CTAs, so the kernel's signal to its own
// dependents is not held back by CTAs waiting for room).  It is launched as a
// programmatic dependent of the split kernel, so its launch and prologue
// overlap the split kernel's tail.
__global__ void __launch_bounds__(kCombineThreads) decode_combine_kernel(
    const float *__restrict__ part_o, const float *__restrict__ part_ml,
    const int32_t *__restrict__ prefix, const int32_t *__restrict__ row_pieces, int32_t batch, Partition partition,
    __half *__restrict__ out, int64_t out_stride, int32_t *__restrict__ claims) {
    const int pair = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    const int row = pair / (kQueryHeads / 2);
    const int head = 2 * (pair % (kQueryHeads / 2)) + (lane >> 4);
    const int dim = 4 * (lane & 15);
    int cta_first = 0, cta_last = 0;
    if (row < batch) {
        if (row_pieces != nullptr) {
            cta_first = row_pieces[2 * row];
            cta_last = row_pieces[2 * row + 1];
        } else {
            cta_first = piece_of(partition, prefix[row]);
            cta_last = piece_of(partition, prefix[row + 1] - 1);
        }
    }
    // The next split kernel (another layer) reads nothing this kernel writes
    // before its own wait: let it launch now.
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");
    // The split kernel has completed: its slot claims are done with.
    if (claims != nullptr && blockIdx.x == 0 && threadIdx.x < kClaimWords) claims[threadIdx.x] = 0;
    if (row >= batch || cta_first == cta_last) return;  // written directly by the split kernel
    float M = -INFINITY, L = 0.f, A[4] = {0.f, 0.f, 0.f, 0.f};
    // Pieces in order, four at a time: all four partials are loaded before
    // any is merged, so a row costs about one L2 round trip per four pieces.
    constexpr int kBatch = 4;
    for (int c0 = cta_first; c0 <= cta_last; c0 += kBatch) {
        float2 ml[kBatch];
        float4 v[kBatch];
#pragma unroll
        for (int j = 0; j < kBatch; ++j) {
            if (c0 + j <= cta_last) {
                const int64_t idx = (static_cast<int64_t>(row) + c0 + j) * kQueryHeads + head;
                ml[j] = *reinterpret_cast<const float2 *>(part_ml + idx * 2);
                v[j] = *reinterpret_cast<const float4 *>(part_o + idx * kHeadDim + dim);
            }
        }
#pragma unroll
        for (int j = 0; j < kBatch; ++j) {
            if (c0 + j <= cta_last) {
                const MergeWeights w = merge_weights(M, ml[j].x);
                L = merge_value(L, ml[j].y, w);
                A[0] = merge_value(A[0], v[j].x, w);
                A[1] = merge_value(A[1], v[j].y, w);
                A[2] = merge_value(A[2], v[j].z, w);
                A[3] = merge_value(A[3], v[j].w, w);
            }
        }
    }
    __half2 *dst = reinterpret_cast<__half2 *>(out + row * out_stride + head * kHeadDim + dim);
    dst[0] = __floats2half2_rn(__fdiv_rn(A[0], L), __fdiv_rn(A[1], L));
    dst[1] = __floats2half2_rn(__fdiv_rn(A[2], L), __fdiv_rn(A[3], L));
}

// ---------------------------------------------------------------------------
// Host side: tensor-map cache, launch plan, entry points.
// ---------------------------------------------------------------------------

using pkv::EncodeTiled;
using pkv::encode_fn;
using pkv::pool_tensor_map;

// Pipeline depth per warp: 4 stages keep three CTAs per SM (registers and shared memory).
constexpr int kStages = 4;

template <int STAGES, bool FUSED>
int prepare_kernel(int *ctas_per_sm) {
    auto kernel = decode_kernel<STAGES, FUSED>;
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes<STAGES>());
    if (e == cudaSuccess) {
        e = cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared);
    }
    if (e != cudaSuccess) return pkv::fail(PKV_CUDA_ERROR, std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(e));
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(ctas_per_sm, kernel, kThreads, smem_bytes<STAGES>());
    if (e != cudaSuccess) return pkv::fail(PKV_CUDA_ERROR, std::string("occupancy query: ") + cudaGetErrorString(e));
    return PKV_OK;
}

template <int STAGES>
int prepare_both(int *ctas_per_sm) {
    int fused = 0;
    int rc = prepare_kernel<STAGES, false>(ctas_per_sm);
    if (rc) return rc;
    rc = prepare_kernel<STAGES, true>(&fused);
    if (rc) return rc;
    if (fused < *ctas_per_sm) *ctas_per_sm = fused;
    return PKV_OK;
}

struct DeviceInfo {
    int sms = 0;
    int ctas_per_sm = 0;
};

int device_info(int device, DeviceInfo *info) {
    static std::mutex mutex;
    static std::unordered_map<int, DeviceInfo> cache;
    std::lock_guard<std::mutex> lock(mutex);
    auto it = cache.find(device);
    if (it != cache.end()) {
        *info = it->second;
        return PKV_OK;
    }
    int previous = 0;
    cudaGetDevice(&previous);
    cudaError_t e = cudaSetDevice(device);
    if (e != cudaSuccess) return pkv::fail(PKV_CUDA_ERROR, std::string("cudaSetDevice: ") + cudaGetErrorString(e));
    DeviceInfo d;
    cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, device);
    int rc = PKV_OK;
    rc = prepare_both<kStages>(&d.ctas_per_sm);
    if (rc == PKV_OK) {
        // The combine needs no shared memory, but an SM that alternates between
        // it and the split kernel would otherwise re-partition L1 and shared
        // memory at every layer; keeping the split kernel's partition avoids that.
        const cudaError_t e = cudaFuncSetAttribute(decode_combine_kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                                                   cudaSharedmemCarveoutMaxShared);
        if (e != cudaSuccess) rc = pkv::fail(PKV_CUDA_ERROR, std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(e));
    }
    cudaSetDevice(previous);
    if (rc) return rc;
    if (d.ctas_per_sm < 1) d.ctas_per_sm = 1;
    cache.emplace(device, d);
    *info = d;
    return PKV_OK;
}

template <bool FUSED>
cudaError_t launch_decode(int grid, const CUtensorMap &map, const LayerArgs &args, cudaStream_t stream) {
    // Programmatic dependent launch: see the griddepcontrol.wait at the top of
    // decode_kernel.
    cudaLaunchConfig_t config = {};
    config.gridDim = dim3(grid);
    config.blockDim = dim3(kThreads);
    config.stream = stream;
    cudaLaunchAttribute attribute[1];
    attribute[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attribute[0].val.programmaticStreamSerializationAllowed = 1;
    config.attrs = attribute;
    config.numAttrs = 1;
    config.dynamicSmemBytes = smem_bytes<kStages>();
    return cudaLaunchKernelEx(&config, decode_kernel<kStages, FUSED>, map, args);
}

// The slot claim counters first, then each slot's four warp wall-time
// counters (both at the same place whatever the launch shape: launches of
// other shapes write their partials after their own counters, never over the
// claim counters, which must stay zero between launches), then the split
// partials of (batch + grid) (row, piece) slots.
int64_t workspace_bytes_for(int32_t batch, int32_t grid) {
    return 2 * kClaimWords * static_cast<int64_t>(sizeof(int32_t)) +
           static_cast<int64_t>(grid) * 4 * static_cast<int64_t>(sizeof(unsigned)) +
           (static_cast<int64_t>(batch) + grid) * kPartialFloats * static_cast<int64_t>(sizeof(float));
}

// The pieces of (grid, per_cta, big, tail) are nonempty and cover exactly
// total_blocks blocks.
bool partition_matches(int32_t total, int32_t grid, int32_t per_cta, int32_t big, int32_t tail) {
    if (grid < 1 || per_cta < 1 || big < 1 || big > grid || tail < 1) return false;
    if (big == grid) {
        return static_cast<int64_t>(grid) * per_cta >= total && static_cast<int64_t>(grid - 1) * per_cta < total;
    }
    const int64_t split = static_cast<int64_t>(big) * per_cta;
    if (split >= total) return false;
    return grid - big == (total - split + tail - 1) / tail;
}

// Checks shared by both entry points; fills the common part of LayerArgs.
int common_checks(const void *pool, int32_t num_blocks, int32_t layer, const void *query, int64_t query_stride,
                  const int32_t *lengths, const int32_t *prefix, const int32_t *flat, const int32_t *pieces,
                  const int32_t *row_pieces,
                  int32_t batch, int32_t total_blocks, int32_t grid, int32_t blocks_per_cta, int32_t big_ctas,
                  int32_t tail_blocks, void *out, int64_t out_stride, void *workspace, int64_t workspace_bytes,
                  int32_t *error_flag, LayerArgs *args) {
    if (pool == nullptr || query == nullptr || lengths == nullptr || prefix == nullptr ||
        flat == nullptr || out == nullptr || error_flag == nullptr) {
        return pkv::fail(PKV_VALUE_ERROR, "decode attention: null pointer argument");
    }
    if (layer < 0 || layer >= PKV_LAYERS) {
        return pkv::fail(PKV_VALUE_ERROR, "layer_index must identify one of the 22 decoder layers");
    }
    // With piece tables the tables define the pieces; otherwise the partition does.
    const bool plan_ok = pieces != nullptr
                             ? grid >= 1 && grid <= total_blocks
                             : partition_matches(total_blocks, grid, blocks_per_cta, big_ctas, tail_blocks);
    if (batch < 1 || total_blocks < batch || !plan_ok) {
        return pkv::fail(PKV_VALUE_ERROR, "decode attention: launch plan does not match the batch");
    }
    if (num_blocks < 1 || static_cast<int64_t>(PKV_LAYERS) * 2 * num_blocks * kBlockTokens > INT32_MAX) {
        return pkv::fail(PKV_VALUE_ERROR, "decode attention: pool block count out of range");
    }
    if ((pieces == nullptr) != (row_pieces == nullptr)) {
        return pkv::fail(PKV_VALUE_ERROR, "decode attention: pieces and row_pieces must be given together");
    }
    if ((reinterpret_cast<uintptr_t>(query) & 3) || (reinterpret_cast<uintptr_t>(out) & 3) ||
        query_stride % 2 || out_stride % 2 || (reinterpret_cast<uintptr_t>(pool) & 15) ||
        (reinterpret_cast<uintptr_t>(workspace) & 15) || (reinterpret_cast<uintptr_t>(pieces) & 15) ||
        (reinterpret_cast<uintptr_t>(row_pieces) & 3)) {
        return pkv::fail(PKV_VALUE_ERROR, "decode attention: misaligned tensor");
    }
    if (grid > 1 && (workspace == nullptr || workspace_bytes < workspace_bytes_for(batch, grid))) {
        return pkv::fail(PKV_VALUE_ERROR, "decode attention: workspace is smaller than the plan needs");
    }
    LayerArgs &x = *args;
    x = LayerArgs{};
    x.query = static_cast<const __half *>(query);
    x.query_stride = query_stride;
    x.pool = static_cast<__half *>(const_cast<void *>(pool));
    x.lengths = lengths;
    x.prefix = prefix;
    x.flat = flat;
    x.pieces = pieces;
    x.batch = batch;
    x.total_blocks = total_blocks;
    x.blocks_per_cta = blocks_per_cta;
    x.big_ctas = big_ctas;
    x.tail_blocks = tail_blocks;
    x.num_blocks = num_blocks;
    x.layer = layer;
    x.out = static_cast<__half *>(out);
    x.out_stride = out_stride;
    if (workspace != nullptr) {
        x.claims = static_cast<int32_t *>(workspace);
        x.cta_ns = reinterpret_cast<unsigned *>(x.claims + 2 * kClaimWords);
        x.part_o = reinterpret_cast<float *>(x.cta_ns + 4 * static_cast<int64_t>(grid));
        x.part_ml = x.part_o + (static_cast<int64_t>(batch) + grid) * kQueryHeads * kHeadDim;
        // Per-SM slots when the pieces come from a table and the grid is one
        // full wave of CTAs.
        DeviceInfo info;
        int device = 0;
        if (pieces != nullptr && cudaGetDevice(&device) == cudaSuccess && device_info(device, &info) == PKV_OK &&
            info.sms <= kClaimWords && grid == info.sms * info.ctas_per_sm) {
            x.sm_slots = info.ctas_per_sm;
        }
    }
    x.error_flag = error_flag;
    return PKV_OK;
}

// Launch the split kernel, then (when rows can be split) the combine kernel
// as its programmatic dependent on the same stream.
template <bool FUSED>
int launch_pass(int grid, const CUtensorMap &map, const LayerArgs &args, const int32_t *row_pieces,
                cudaStream_t stream, const char *what) {
    cudaError_t e = launch_decode<FUSED>(grid, map, args, stream);
    if (e != cudaSuccess) return pkv::fail(PKV_CUDA_ERROR, std::string(what) + " launch failed: " + cudaGetErrorString(e));
    if (grid == 1) return PKV_OK;
    const int warps_per_cta = kCombineThreads / 32;
    const int pairs = args.batch * (kQueryHeads / 2);
    cudaLaunchConfig_t config = {};
    config.gridDim = dim3((pairs + warps_per_cta - 1) / warps_per_cta);
    config.blockDim = dim3(warps_per_cta * 32);
    config.dynamicSmemBytes = 0;
    config.stream = stream;
    cudaLaunchAttribute attribute[1];
    attribute[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attribute[0].val.programmaticStreamSerializationAllowed = 1;
    config.attrs = attribute;
    config.numAttrs = 1;
    const Partition partition{args.total_blocks, args.blocks_per_cta, args.big_ctas, args.tail_blocks};
    e = cudaLaunchKernelEx(&config, decode_combine_kernel, static_cast<const float *>(args.part_o),
                           static_cast<const float *>(args.part_ml), args.prefix, row_pieces, args.batch, partition,
                           args.out, args.out_stride,
                           args.sm_slots > 0 ? args.claims + (args.layer & 1) * kClaimWords : nullptr);
    if (e != cudaSuccess) {
        return pkv::fail(PKV_CUDA_ERROR, std::string("decode combine launch failed: ") + cudaGetErrorString(e));
    }
    return PKV_OK;
}

}  // namespace

extern "C" int pkv_decode_plan(int32_t device, int32_t batch, int32_t total_blocks, int32_t *out_grid,
                               int32_t *out_blocks_per_cta, int32_t *out_big_ctas, int32_t *out_tail_blocks,
                               int64_t *out_workspace_bytes) {
    pkv::clear_error();
    if (batch < 1 || total_blocks < batch) {
        return pkv::fail(PKV_VALUE_ERROR, "decode plan needs batch >= 1 and a nonempty block per row");
    }
    DeviceInfo info;
    int rc = device_info(device, &info);
    if (rc) return rc;
    // One piece per CTA slot (one wave), the blocks spread as evenly as
    // integers allow: r pieces of q + 1 blocks, then grid - r pieces of q.
    const int64_t slots = static_cast<int64_t>(info.sms) * info.ctas_per_sm;
    const int32_t grid = static_cast<int32_t>(std::min<int64_t>(slots, total_blocks));
    const int32_t q = total_blocks / grid, r = total_blocks % grid;
    *out_grid = grid;
    *out_blocks_per_cta = r == 0 ? q : q + 1;
    *out_big_ctas = r == 0 ? grid : r;
    *out_tail_blocks = q;
    *out_workspace_bytes = workspace_bytes_for(batch, grid);
    return PKV_OK;
}

extern "C" int pkv_decode_attention(const void *pool, int32_t num_blocks, int32_t layer,
                                    const void *query, int64_t query_stride, const int32_t *lengths,
                                    const int32_t *prefix, const int32_t *flat, const int32_t *pieces,
                                    const int32_t *row_pieces, int32_t batch, int32_t total_blocks, int32_t grid,
                                    int32_t blocks_per_cta,
                                    int32_t big_ctas, int32_t tail_blocks, void *out, int64_t out_stride,
                                    void *workspace, int64_t workspace_bytes, int32_t *error_flag, void *stream) {
    pkv::clear_error();
    LayerArgs args;
    int rc = common_checks(pool, num_blocks, layer, query, query_stride, lengths, prefix, flat, pieces, row_pieces, batch,
                           total_blocks, grid, blocks_per_cta, big_ctas, tail_blocks, out, out_stride, workspace,
                           workspace_bytes, error_flag, &args);
    if (rc) return rc;
    int device = 0;
    cudaGetDevice(&device);
    DeviceInfo info;
    if ((rc = device_info(device, &info))) return rc;
    CUtensorMap map;
    if ((rc = pool_tensor_map(pool, num_blocks, &map))) return rc;
    return launch_pass<false>(grid, map, args, row_pieces, static_cast<cudaStream_t>(stream), "decode attention");
}

extern "C" int pkv_decode_layer(void *pool, int32_t num_blocks, int32_t layer, const void *query,
                                int64_t query_stride, const void *key, const void *value, int64_t kv_stride,
                                const void *rope_table, const int32_t *lengths, const int32_t *prefix,
                                const int32_t *flat, const int32_t *pieces, const int32_t *row_pieces,
                                int32_t batch, int32_t total_blocks, int32_t grid, int32_t blocks_per_cta,
                                int32_t big_ctas, int32_t tail_blocks,
                                void *out, int64_t out_stride, void *workspace, int64_t workspace_bytes,
                                int32_t *error_flag, int32_t flags, void *stream) {
    pkv::clear_error();
    LayerArgs args;
    int rc = common_checks(pool, num_blocks, layer, query, query_stride, lengths, prefix, flat, pieces, row_pieces, batch,
                           total_blocks, grid, blocks_per_cta, big_ctas, tail_blocks, out, out_stride, workspace,
                           workspace_bytes, error_flag, &args);
    if (rc) return rc;
    if (key == nullptr || value == nullptr || rope_table == nullptr) {
        return pkv::fail(PKV_VALUE_ERROR, "decode layer: key, value and RoPE table are required");
    }
    if ((reinterpret_cast<uintptr_t>(key) & 3) || (reinterpret_cast<uintptr_t>(value) & 3) || kv_stride % 2 ||
        (reinterpret_cast<uintptr_t>(rope_table) & 3)) {
        return pkv::fail(PKV_VALUE_ERROR, "decode layer: misaligned tensor");
    }
    args.key_new = static_cast<const __half *>(key);
    args.value_new = static_cast<const __half *>(value);
    args.new_stride = kv_stride;
    args.rope_cos = static_cast<const __half *>(rope_table);
    args.rope_sin = args.rope_cos + PKV_CONTEXT_LIMIT * kRopeHalf;
    if (flags & ~PKV_DECODE_EARLY_KV) return pkv::fail(PKV_VALUE_ERROR, "decode layer: unknown flags");
    args.early_kv = (flags & PKV_DECODE_EARLY_KV) != 0;
    int device = 0;
    cudaGetDevice(&device);
    DeviceInfo info;
    if ((rc = device_info(device, &info))) return rc;
    CUtensorMap map;
    if ((rc = pool_tensor_map(pool, num_blocks, &map))) return rc;
    return launch_pass<true>(grid, map, args, row_pieces, static_cast<cudaStream_t>(stream), "decode layer");
}

// ---------------------------------------------------------------------------
// Decode attention without any allocation (pkv_decode_attention_noalloc).
//
// Some hosts cannot hand this library device memory for its split partials:
// a serving process whose device memory is entirely owned by another
// allocator (the KV pool reserved up front, no further cudaMalloc allowed),
// or a plugin host that offers no workspace callback.  For them the partials
// live in one file-scope device array of fixed size, and the host code below
// reaches it through cudaGetSymbolAddress: in host code the array's name is
// only a stand-in for the symbol, not a device address.
// ---------------------------------------------------------------------------
namespace {

constexpr int64_t kNoAllocScratchBytes = 8ll << 20;  // 8 MiB, held by every device that loads the library
constexpr int kNoAllocMaxDevices = 64;

static __device__ __align__(256) float g_noalloc_partials[kNoAllocScratchBytes / sizeof(float)];

std::mutex g_noalloc_mutex;
void *g_noalloc_scratch[kNoAllocMaxDevices] = {};

// Once per device, with that device current: the array's device address and
// the kernels' shared-memory attribute.  Nothing here allocates.
int noalloc_setup(int device, void **scratch) {
    if (device < 0 || device >= kNoAllocMaxDevices) {
        return pkv::fail(PKV_VALUE_ERROR, "no-alloc decode attention: device ordinal out of range");
    }
    std::lock_guard<std::mutex> lock(g_noalloc_mutex);
    if (g_noalloc_scratch[device] == nullptr) {
        void *ptr = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_partials);
        if (e != cudaSuccess || ptr == nullptr) {
            return pkv::fail(PKV_CUDA_ERROR, std::string("no-alloc decode attention: cudaGetSymbolAddress failed: ") +
                                                 cudaGetErrorString(e));
        }
        e = cudaFuncSetAttribute(decode_kernel<kStages, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 smem_bytes<kStages>());
        if (e != cudaSuccess) {
            return pkv::fail(PKV_CUDA_ERROR, std::string("no-alloc decode attention: cudaFuncSetAttribute: ") +
                                                 cudaGetErrorString(e));
        }
        g_noalloc_scratch[device] = ptr;
    }
    *scratch = g_noalloc_scratch[device];
    return PKV_OK;
}

// The pool's tensor map, encoded into a local value (no cache, no allocation).
int noalloc_pool_map(const void *pool, int32_t num_blocks, CUtensorMap *map) {
    EncodeTiled encode = encode_fn();
    if (encode == nullptr) return pkv::fail(PKV_CUDA_ERROR, "cuTensorMapEncodeTiled is unavailable");
    const cuuint64_t rows = static_cast<cuuint64_t>(PKV_LAYERS) * 2 * num_blocks * kBlockTokens;
    const cuuint64_t dims[3] = {static_cast<cuuint64_t>(kHeadDim), static_cast<cuuint64_t>(kKvHeads), rows};
    const cuuint64_t strides[2] = {static_cast<cuuint64_t>(kRowBytes), static_cast<cuuint64_t>(kKvHeads * kRowBytes)};
    const cuuint32_t box[3] = {static_cast<cuuint32_t>(kHeadDim), 1u, static_cast<cuuint32_t>(kBlockTokens)};
    const cuuint32_t elem[3] = {1u, 1u, 1u};
    const CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void *>(pool), dims, strides, box,
                              elem, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        return pkv::fail(PKV_CUDA_ERROR, "cuTensorMapEncodeTiled failed with code " + std::to_string(int(r)));
    }
    return PKV_OK;
}

}  // namespace

extern "C" int pkv_decode_attention_noalloc(const void *pool, int32_t num_blocks, int32_t layer, const void *query,
                                            int64_t query_stride, const int32_t *lengths, const int32_t *prefix,
                                            const int32_t *flat, const int32_t *pieces,
                                            const int32_t *row_pieces, int32_t batch,
                                            int32_t total_blocks, int32_t grid, int32_t blocks_per_cta,
                                            int32_t big_ctas, int32_t tail_blocks, void *out, int64_t out_stride,
                                            int32_t *error_flag, void *stream) {
    pkv::clear_error();
    if (batch < 0 || grid < 0 || workspace_bytes_for(batch, grid) > kNoAllocScratchBytes) {
        return pkv::fail(PKV_VALUE_ERROR,
                         "no-alloc decode attention: the plan needs " +
                             std::to_string(workspace_bytes_for(batch, grid)) +
                             " bytes of split partials, over the static scratch limit of " +
                             std::to_string(kNoAllocScratchBytes) + " (8 MiB); use pkv_decode_attention with a workspace");
    }
    int device = 0;
    cudaError_t e = cudaGetDevice(&device);
    if (e != cudaSuccess) return pkv::fail(PKV_CUDA_ERROR, std::string("cudaGetDevice: ") + cudaGetErrorString(e));
    void *scratch = nullptr;
    int rc = noalloc_setup(device, &scratch);
    if (rc) return rc;
    LayerArgs args;
    rc = common_checks(pool, num_blocks, layer, query, query_stride, lengths, prefix, flat, pieces, row_pieces, batch,
                       total_blocks, grid, blocks_per_cta, big_ctas, tail_blocks, out, out_stride, scratch,
                       kNoAllocScratchBytes, error_flag, &args);
    if (rc) return rc;
    CUtensorMap map;
    if ((rc = noalloc_pool_map(pool, num_blocks, &map))) return rc;
    // The array keeps the last call's contents.  The slot-claim counters at its
    // start must be zero when the split kernel starts; every completed call
    // leaves them so, and this clear covers a call that did not complete.
    e = cudaMemsetAsync(scratch, 0, 2 * kClaimWords * sizeof(int32_t), static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) {
        return pkv::fail(PKV_CUDA_ERROR, std::string("no-alloc decode attention: clearing the claim counters: ") +
                                             cudaGetErrorString(e));
    }
    return launch_pass<false>(grid, map, args, row_pieces, static_cast<cudaStream_t>(stream),
                              "no-alloc decode attention");
}
