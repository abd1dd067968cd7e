// Causal prompt (prefill) attention through the block table on the sm_100a
// tensor cores (tcgen05, TMEM accumulators, TMA staging).
//
// Same operation and numerics as prefill_attention.cu's contract: token t of
// a chunk (position start + t) attends to positions 0 .. start + t of its
// request through its block table, FP32 scores and sums from FP16 pages, one
// FP16 rounding of the output (PagedCore's dense_attention with the mask of
// decoder.py:225, computed as attention.py:14-53 computes a row):
//   out[t,h] = sum_{p <= start+t} softmax_p(q[t,h] . K[p, h/8] * 0.125) V[p, h/8]
//
// Work split - one CTA per (16-token tile, KV head): its M = 128 MMA rows are
// the tile's 16 tokens x the 8 query heads of the KV head (row r: token r/8,
// head r%8), so every K/V block is read once per 128 query rows.  Tiles run
// longest first across the four heads.  A CTA walks its keys 64 at a time
// (four 16-token pool blocks), from block 0 to the block of its last token.
//
// Roles (192 threads):
// - warp 4 (one thread): TMA loads of each step's K and V boxes (one head of
//   one block: 16 rows x 128 B, 128-byte swizzle, no multicast) into a
//   3-stage ring of shared memory.
// - warp 5 (one thread; the warp owns the TMEM allocation): tcgen05.mma.
//   S_j = Q . K_j^T  (M 128, N 64, K 64: four K=16 MMAs) into one of two TMEM
//   S buffers, then O += P_j . V_j (M 128, N 64, one K=16 MMA per block) into
//   the TMEM O; S_{j+1} is issued before P_j . V_j, so the tensor cores work
//   on the next scores while the softmax works on these.
// - warps 0-3 (128 threads, thread r = row r, TMEM lane r): the softmax.  A
//   thread reads its row of S_j from TMEM (tcgen05.ld), masks positions past
//   its token, and keeps the online softmax state in base 2 in FP32: a
//   reference maximum m that moves only when the row's maximum passes it by
//   more than 2^8.  It writes P_j = 2^(s - m + 7) (<= 2^15) as FP16 into
//   shared memory in the MMA's K-major swizzled layout.  The normaliser l is
//   the MMA's too: P_j times a 64 x 16 matrix of ones accumulates the row sums
//   of the same FP16 weights in FP32 in TMEM.  When m moves, the thread
//   rescales its row of O and l in TMEM (ld, multiply, st) once the previous
//   P.V has completed.  At the end O / l is rounded to FP16.
//
// Slots at or past start + tokens hold no K/V yet (the pool may hold
// anything there): their scores are masked, and their V rows are zeroed in
// shared memory before the P.V that would read them, so 0 * NaN never
// reaches the sum.  Block ids outside the pool set PKV_DEVICE_BAD_BLOCK and
// read as zeros.  Every wait is bounded: on a timeout the thread sets
// PKV_DEVICE_WAIT_TIMEOUT, the CTA stops issuing work, waits (bounded) for
// its MMAs and copies in flight and frees its TMEM.

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <string>

#include "pagedkv.h"
#include "ptx.cuh"
#include "status.h"
#include "tcgen05.cuh"
#include "tensor_maps.h"

namespace {

constexpr int kHeadDim = PKV_HEAD_DIM;
constexpr int kKvHeads = PKV_KV_HEADS;
constexpr int kBlockTokens = PKV_BLOCK_TOKENS;
constexpr int kMaxTableBlocks = PKV_CONTEXT_LIMIT / PKV_BLOCK_TOKENS;  // 128
constexpr int kTileTokens = 16;
constexpr int kRows = 128;                  // MMA M: 16 tokens x 8 query heads
constexpr int kStepBlocks = 4;              // pool blocks per step
constexpr int kStepKeys = kStepBlocks * kBlockTokens;  // 64: MMA N of S, K of P.V
constexpr int kStages = 3;
constexpr int kRowBytes = kHeadDim * 2;     // 128 B
constexpr int kBoxBytes = kBlockTokens * kRowBytes;    // 2 KiB: one head of one block
constexpr int kQBytes = kRows * kRowBytes;             // 16 KiB
constexpr int kPBytes = kRows * kStepKeys * 2;         // 16 KiB
constexpr int kHalfStageBytes = kStepBlocks * kBoxBytes;  // 8 KiB of K (or V)
constexpr int kStageBytes = 2 * kHalfStageBytes;
constexpr int kOnesBytes = kBlockTokens * kRowBytes;    // 2 KiB: 16 x 64 FP16 ones (B of the row-sum MMA)
constexpr int kSmemBytes = kQBytes + 2 * kPBytes + kOnesBytes + kStages * kStageBytes + 1024;  // + alignment slack
constexpr int kSoftmaxWarps = 4;           // thread r of warps 0-3 owns row r (TMEM lane r)
constexpr int kSoftmaxThreads = kSoftmaxWarps * 32;
constexpr int kThreads = kSoftmaxThreads + 64;
constexpr int kProducerWarp = kSoftmaxWarps;
constexpr int kMmaWarp = kSoftmaxWarps + 1;
constexpr uint32_t kTmemCols = 256;  // S0 [0, 64), S1 [64, 128), O [128, 192), L [192, 208)
constexpr uint32_t kTmemO = 128;
constexpr uint32_t kTmemL = 192;     // row sums of P: 16 equal columns
constexpr uint32_t kWaitPolls = 1u << 24;
constexpr uint32_t kAbortPolls = 1u << 12;  // once the CTA aborts, later waits give up quickly
constexpr float kScaleLog2 = 0.125f * 1.4426950408889634f;  // 64^-0.5 * log2(e)
// P = 2^(s - m + 7) with m the row maximum at its last rescale; m is moved
// only when a row's maximum exceeds it by more than 2^8, so P <= 2^15 stays
// inside FP16 while O and l are rescaled at most a few times per row.
constexpr float kWeightShift = 7.0f;
constexpr float kRescaleLog2 = 8.0f;
static_assert(kRows == kTileTokens * (PKV_QUERY_HEADS / kKvHeads), "a tile's rows are its tokens x 8 heads");

// Instruction descriptors: S = Q . K^T (both K-major), O += P . V (P K-major, V MN-major).
constexpr uint32_t kIdescS = pkv::tc::idesc_f16_f32(kRows, kStepKeys, false, false);
constexpr uint32_t kIdescO = pkv::tc::idesc_f16_f32(kRows, kHeadDim, false, true);
// l += P . 1: the row sums of the FP16 weights, accumulated in FP32 by the MMA (N = 16, ones K-major).
constexpr uint32_t kIdescL = pkv::tc::idesc_f16_f32(kRows, 16, false, false);

struct TcArgs {
    const __half *query;
    __half *out;
    const int32_t *blocks;
    int64_t query_stride;
    int64_t out_stride;
    int32_t num_blocks;
    int32_t layer;
    int32_t start;
    int32_t tokens;
    int32_t *error_flag;
};

// Barriers of one CTA (8-byte mbarriers in static shared memory).
struct Barriers {
    uint64_t kv_full[kStages];   // TMA -> MMA: the stage's K/V landed (tx count)
    uint64_t kv_empty[kStages];  // MMA -> TMA: the stage's P.V completed
    uint64_t s_full[2];          // MMA -> softmax: S_j in TMEM
    uint64_t s_empty[2];         // softmax -> MMA: S_j read (4 warp arrivals)
    uint64_t p_full[2];          // softmax -> MMA: P_j written, O corrected (4 warp arrivals)
    uint64_t pv_done[2];         // MMA -> softmax: P_j . V_j completed
    uint64_t drained;            // MMA -> teardown: every MMA issued completed
};

__device__ __forceinline__ uint32_t bar_addr(const uint64_t &b) { return pkv::smem_addr(&b); }

// Bounded wait; on a timeout flags the CTA as aborting.
__device__ __forceinline__ bool wait_or_abort(uint32_t bar, uint32_t parity, volatile int *abort,
                                              int32_t *error_flag) {
    if (pkv::mbar_wait_bounded(bar, parity, *abort ? kAbortPolls : kWaitPolls)) return true;
    atomicOr(error_flag, PKV_DEVICE_WAIT_TIMEOUT);
    *abort = 1;
    return false;
}

// The same wait by every lane of a warp, with one outcome for the whole warp
// (the warp then runs .sync.aligned TMEM instructions together or not at all).
__device__ __forceinline__ bool warp_wait(uint32_t bar, uint32_t parity, volatile int *abort, int32_t *error_flag) {
    const bool ok = wait_or_abort(bar, parity, abort, error_flag);
    return __all_sync(0xffffffffu, ok);
}

__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
    return pkv::pack_half2(__floats2half2_rn(lo, hi));
}

__global__ void __launch_bounds__(kThreads, 2)
    prefill_tc_kernel(const __grid_constant__ CUtensorMap pool_map, const TcArgs a) {
    extern __shared__ uint8_t dyn_smem[];
    __shared__ Barriers bars;
    __shared__ int32_t table[kMaxTableBlocks];
    __shared__ uint32_t tmem_slot;
    __shared__ volatile int abort_flag;

    const uint32_t raw = pkv::smem_addr(dyn_smem);
    const uint32_t base = (raw + 1023u) & ~1023u;  // 1024-aligned: swizzle atoms
    uint8_t *const base_ptr = dyn_smem + (base - raw);
    const uint32_t q_smem = base;
    const uint32_t p_smem = base + kQBytes;                  // P[2]
    const uint32_t ones_smem = base + kQBytes + 2 * kPBytes;  // 16 x 64 FP16 ones
    const uint32_t kv_smem = ones_smem + kOnesBytes;          // stages: K 8 KiB then V 8 KiB

    const int tiles = gridDim.x / kKvHeads;
    const int tile = tiles - 1 - static_cast<int>(blockIdx.x) / kKvHeads;  // longest first
    const int kv = static_cast<int>(blockIdx.x) % kKvHeads;
    const int t0 = tile * kTileTokens;
    const int last_t = min(t0 + kTileTokens - 1, a.tokens - 1);
    const int nblocks = (a.start + last_t) / kBlockTokens + 1;
    const int steps = (nblocks + kStepBlocks - 1) / kStepBlocks;
    const int written = a.start + a.tokens;  // positions below hold K/V
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    int armed = 0;  // producer: steps whose copies were issued

    // ---- set-up ----------------------------------------------------------
    for (int j = threadIdx.x; j < nblocks; j += kThreads) table[j] = a.blocks[j];
    if (warp == kMmaWarp) {
        pkv::tc::tmem_alloc(pkv::smem_addr(&tmem_slot), kTmemCols);
        pkv::tc::tmem_relinquish();
    }
    if (threadIdx.x == kProducerWarp * 32) {
        for (int s = 0; s < kStages; ++s) {
            pkv::mbar_init(bar_addr(bars.kv_full[s]), 1);
            pkv::mbar_init(bar_addr(bars.kv_empty[s]), 1);
        }
        for (int b = 0; b < 2; ++b) {
            pkv::mbar_init(bar_addr(bars.s_full[b]), 1);
            pkv::mbar_init(bar_addr(bars.s_empty[b]), kSoftmaxWarps);
            pkv::mbar_init(bar_addr(bars.p_full[b]), kSoftmaxWarps);
            pkv::mbar_init(bar_addr(bars.pv_done[b]), 1);
        }
        pkv::mbar_init(bar_addr(bars.drained), 1);
        abort_flag = 0;
        pkv::fence_barrier_init();
    }
    if (warp < kSoftmaxWarps) {
        // Q as the A operand: row r = (token r/8, head kv*8 + r%8), 128 B, chunk c at c ^ (r%8).
        const int r = threadIdx.x;
        const int t = min(t0 + (r >> 3), a.tokens - 1);
        const uint4 *src = reinterpret_cast<const uint4 *>(a.query + t * a.query_stride +
                                                           (kv * 8 + (r & 7)) * kHeadDim);
        uint8_t *row = base_ptr + (r >> 3) * 1024 + (r & 7) * kRowBytes;
#pragma unroll
        for (int c = 0; c < 8; ++c) {
            *reinterpret_cast<uint4 *>(row + ((c ^ (r & 7)) << 4)) = src[c];
        }
        // The ones matrix (16 rows of 64 FP16 1.0, 2 KiB): 16 bytes a thread.
        reinterpret_cast<uint4 *>(base_ptr + (ones_smem - base))[r] = make_uint4(0x3c003c00u, 0x3c003c00u,
                                                                                 0x3c003c00u, 0x3c003c00u);
        pkv::fence_proxy_async_smem();  // generic writes -> the MMA's (async proxy) reads
    }
    pkv::tc::fence_before_sync();
    __syncthreads();
    pkv::tc::fence_after_sync();
    const uint32_t tmem = tmem_slot;

    if (warp == kProducerWarp) {
        // ---- TMA producer ----------------------------------------------------
        if (lane == 0) {
            const int32_t k_rows = (a.layer * 2) * a.num_blocks;
            const int32_t v_rows = (a.layer * 2 + 1) * a.num_blocks;
            for (int j = 0; j < steps && !abort_flag; ++j) {
                const int st = j % kStages;
                if (j >= kStages &&
                    !wait_or_abort(bar_addr(bars.kv_empty[st]), ((j / kStages) - 1) & 1, &abort_flag, a.error_flag)) {
                    break;
                }
                const uint32_t k_dst = kv_smem + st * kStageBytes;
                const uint32_t v_dst = k_dst + kHalfStageBytes;
                const int nb = min(kStepBlocks, nblocks - j * kStepBlocks);
                int loads = 0;
                for (int kb = 0; kb < nb; ++kb) {
                    const int32_t block = table[j * kStepBlocks + kb];
                    if (block >= 0 && block < a.num_blocks) {
                        ++loads;
                    } else {
                        // Outside the pool: flag it and read zeros (no copy).
                        atomicOr(a.error_flag, PKV_DEVICE_BAD_BLOCK);
                        uint4 *k_tile = reinterpret_cast<uint4 *>(base_ptr + (k_dst - base) + kb * kBoxBytes);
                        uint4 *v_tile = reinterpret_cast<uint4 *>(base_ptr + (v_dst - base) + kb * kBoxBytes);
                        for (int i = 0; i < kBoxBytes / 16; ++i) k_tile[i] = v_tile[i] = make_uint4(0, 0, 0, 0);
                    }
                }
                pkv::fence_proxy_async_smem();
                pkv::mbar_arrive_expect_tx(bar_addr(bars.kv_full[st]), loads * 2 * kBoxBytes);
                for (int kb = 0; kb < nb; ++kb) {
                    const int32_t block = table[j * kStepBlocks + kb];
                    if (block < 0 || block >= a.num_blocks) continue;
                    pkv::tma_load_3d(k_dst + kb * kBoxBytes, &pool_map, 0, kv, (k_rows + block) * kBlockTokens,
                                     bar_addr(bars.kv_full[st]));
                    pkv::tma_load_3d(v_dst + kb * kBoxBytes, &pool_map, 0, kv, (v_rows + block) * kBlockTokens,
                                     bar_addr(bars.kv_full[st]));
                }
                armed = j + 1;
            }
        }
    } else if (warp == kMmaWarp) {
        // ---- MMA issuer ------------------------------------------------------
        if (lane == 0) {
            auto issue_pv = [&](int i) -> bool {
                if (!wait_or_abort(bar_addr(bars.p_full[i & 1]), (i >> 1) & 1, &abort_flag, a.error_flag)) {
                    return false;
                }
                pkv::tc::fence_after_sync();
                const int st = i % kStages;
                const uint32_t v_base = kv_smem + st * kStageBytes + kHalfStageBytes;
                const uint32_t p_base = p_smem + (i & 1) * kPBytes;
                const int nb = min(kStepBlocks, nblocks - i * kStepBlocks);
                for (int kb = 0; kb < nb; ++kb) {
                    const uint64_t p_desc = pkv::tc::desc_k_major_sw128(p_base + 32 * kb);
                    pkv::tc::mma_f16_ss(tmem + kTmemO, p_desc, pkv::tc::desc_mn_major_sw128(v_base + kb * kBoxBytes),
                                        kIdescO, i > 0 || kb > 0);
                    pkv::tc::mma_f16_ss(tmem + kTmemL, p_desc, pkv::tc::desc_k_major_sw128(ones_smem + 32 * kb),
                                        kIdescL, i > 0 || kb > 0);
                }
                pkv::tc::commit(bar_addr(bars.pv_done[i & 1]));
                pkv::tc::commit(bar_addr(bars.kv_empty[st]));
                return true;
            };
            bool ok = true;
            for (int j = 0; j < steps && ok; ++j) {
                const int st = j % kStages;
                ok = wait_or_abort(bar_addr(bars.kv_full[st]), (j / kStages) & 1, &abort_flag, a.error_flag);
                if (ok && j >= 2) {
                    ok = wait_or_abort(bar_addr(bars.s_empty[j & 1]), ((j - 2) >> 1) & 1, &abort_flag, a.error_flag);
                }
                if (!ok) break;
                pkv::tc::fence_after_sync();
                const uint32_t k_base = kv_smem + st * kStageBytes;
#pragma unroll
                for (int k = 0; k < kHeadDim / 16; ++k) {
                    pkv::tc::mma_f16_ss(tmem + (j & 1) * kStepKeys, pkv::tc::desc_k_major_sw128(q_smem + 32 * k),
                                        pkv::tc::desc_k_major_sw128(k_base + 32 * k), kIdescS, k > 0);
                }
                pkv::tc::commit(bar_addr(bars.s_full[j & 1]));
                if (j >= 1) ok = issue_pv(j - 1);
            }
            if (ok && steps > 0) issue_pv(steps - 1);
            // Teardown: wait until every MMA issued so far has completed.
            pkv::tc::commit(bar_addr(bars.drained));
            if (!pkv::mbar_wait_bounded(bar_addr(bars.drained), 0, kWaitPolls)) {  // in flight: wait in full
                atomicOr(a.error_flag, PKV_DEVICE_WAIT_TIMEOUT);
            }
        }
    } else {
        // ---- softmax (thread r = MMA row r = TMEM lane r) --------------------
        const int r = threadIdx.x;
        const int t = t0 + (r >> 3);
        const int pos = a.start + min(t, a.tokens - 1);  // last position this row attends to
        const uint32_t lanes = tmem + (static_cast<uint32_t>(warp * 32) << 16);
        const int head = kv * 8 + (r & 7);
        // The step whose last block holds unwritten slots (the chunk's last block), if any.
        const bool ragged = nblocks * kBlockTokens > written;
        const int ragged_step = (nblocks - 1) / kStepBlocks;
        float m = -INFINITY;  // the row maximum at its last rescale (log2 units)
        bool ok = true;
        for (int j = 0; j < steps && ok; ++j) {
            const int b = j & 1;
            if (!warp_wait(bar_addr(bars.s_full[b]), (j >> 1) & 1, &abort_flag, a.error_flag)) {
                ok = false;
                break;
            }
            pkv::tc::fence_after_sync();
            uint32_t sr[2][32];
            pkv::tc::tmem_ld32(lanes + b * kStepKeys, sr[0]);
            pkv::tc::tmem_ld32(lanes + b * kStepKeys + 32, sr[1]);
            pkv::tc::tmem_wait_ld();
            pkv::tc::fence_before_sync();
            __syncwarp();
            if (lane == 0) pkv::mbar_arrive(bar_addr(bars.s_empty[b]));

            float s[64];
#pragma unroll
            for (int c = 0; c < 64; ++c) s[c] = __uint_as_float(sr[c >> 5][c & 31]);
            const int key0 = j * kStepKeys;
            if (key0 + kStepKeys - 1 > a.start + t0) {  // the diagonal: mask positions past the row
#pragma unroll
                for (int c = 0; c < 64; ++c) {
                    if (key0 + c > pos) s[c] = -INFINITY;
                }
            }
            // Row maximum over 8 independent chains: one dependent chain of 64
            // would cost its full latency every step.
            float mx8[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) mx8[e] = s[e];
#pragma unroll
            for (int c = 8; c < 64; ++c) mx8[c & 7] = fmaxf(mx8[c & 7], s[c]);
            const float mx = fmaxf(fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3])),
                                   fmaxf(fmaxf(mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7])));
            // Step 0 holds position 0, which every row attends to: m is finite from step 0 on.
            const float m_blk = mx * kScaleLog2;
            const float m_new = m_blk > m + kRescaleLog2 ? m_blk : m;  // m = -inf at step 0: always moves
            if (j >= 2) {
                // P_j reuses the buffer of P_{j-2}: that P.V must be complete.
                if (!warp_wait(bar_addr(bars.pv_done[b]), ((j - 2) >> 1) & 1, &abort_flag, a.error_flag)) {
                    ok = false;
                    break;
                }
                pkv::tc::fence_after_sync();
            }
            // P_j as FP16 (x 2^7) into buffer b, row r, K-major with the 128-byte swizzle.
            const float shift = kWeightShift - m_new;
            uint8_t *prow = base_ptr + (p_smem - base) + b * kPBytes + (r >> 3) * 1024 + (r & 7) * kRowBytes;
#pragma unroll
            for (int c8 = 0; c8 < 8; ++c8) {
                __half2 h[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    h[e] = __floats2half2_rn(pkv::exp2_approx(fmaf(s[8 * c8 + 2 * e], kScaleLog2, shift)),
                                             pkv::exp2_approx(fmaf(s[8 * c8 + 2 * e + 1], kScaleLog2, shift)));
                }
                *reinterpret_cast<uint4 *>(prow + ((c8 ^ (r & 7)) << 4)) =
                    make_uint4(pkv::pack_half2(h[0]), pkv::pack_half2(h[1]), pkv::pack_half2(h[2]),
                               pkv::pack_half2(h[3]));
            }
            if (j >= 1 && __any_sync(0xffffffffu, m_new != m)) {
                // Some row's reference maximum moved: rescale its O and l (scaled
                // by the old one so far) once P_{j-1} . V_{j-1} is in them,
                // before P_j . V_j adds to them.
                if (!warp_wait(bar_addr(bars.pv_done[(j - 1) & 1]), ((j - 1) >> 1) & 1, &abort_flag,
                               a.error_flag)) {
                    ok = false;
                    break;
                }
                pkv::tc::fence_after_sync();
                const float corr = m_new != m ? pkv::exp2_approx(m - m_new) : 1.f;
#pragma unroll
                for (int hf = 0; hf < 3; ++hf) {  // O [128, 192) and L [192, 224)
                    uint32_t o[32];
                    const uint32_t taddr = lanes + kTmemO + 32 * hf;
                    pkv::tc::tmem_ld32(taddr, o);
                    pkv::tc::tmem_wait_ld();
#pragma unroll
                    for (int c = 0; c < 32; ++c) o[c] = __float_as_uint(__uint_as_float(o[c]) * corr);
                    pkv::tc::tmem_st32(taddr, o);
                }
                pkv::tc::tmem_wait_st();
            }
            m = m_new;
            if (ragged && j == ragged_step) {
                // Zero the V rows of unwritten slots in the chunk's last block
                // (thread r: slot r/8, 16-byte chunk r%8) once its copy landed.
                const int st = j % kStages;
                if (!warp_wait(bar_addr(bars.kv_full[st]), (j / kStages) & 1, &abort_flag, a.error_flag)) {
                    ok = false;
                    break;
                }
                const int slot = r >> 3;
                if ((nblocks - 1) * kBlockTokens + slot >= written) {
                    const int kb = (nblocks - 1) - j * kStepBlocks;
                    uint8_t *vrow = base_ptr + (kv_smem - base) + st * kStageBytes + kHalfStageBytes +
                                    kb * kBoxBytes + slot * kRowBytes;
                    *reinterpret_cast<uint4 *>(vrow + ((r & 7) << 4)) = make_uint4(0, 0, 0, 0);
                }
            }
            pkv::fence_proxy_async_smem();
            pkv::tc::fence_before_sync();
            __syncwarp();
            if (lane == 0) pkv::mbar_arrive(bar_addr(bars.p_full[b]));
        }
        if (ok && steps > 0 &&
            warp_wait(bar_addr(bars.pv_done[(steps - 1) & 1]), ((steps - 1) >> 1) & 1, &abort_flag, a.error_flag)) {
            pkv::tc::fence_after_sync();
            uint32_t o[2][32];
            uint32_t sums[16];
            pkv::tc::tmem_ld32(lanes + kTmemO, o[0]);
            pkv::tc::tmem_ld32(lanes + kTmemO + 32, o[1]);
            pkv::tc::tmem_ld16(lanes + kTmemL, sums);
            pkv::tc::tmem_wait_ld();
            const float l = __uint_as_float(sums[0]);
            if (t < a.tokens) {
                uint4 *dst = reinterpret_cast<uint4 *>(a.out + t * a.out_stride + head * kHeadDim);
#pragma unroll
                for (int c8 = 0; c8 < 8; ++c8) {
                    float v[8];
#pragma unroll
                    for (int e = 0; e < 8; ++e) v[e] = __fdiv_rn(__uint_as_float(o[c8 >> 2][(c8 & 3) * 8 + e]), l);
                    dst[c8] = make_uint4(pack2(v[0], v[1]), pack2(v[2], v[3]), pack2(v[4], v[5]), pack2(v[6], v[7]));
                }
            }
        }
        pkv::tc::fence_before_sync();
    }

    // ---- teardown --------------------------------------------------------
    __syncthreads();
    if (warp == kProducerWarp && lane == 0 && abort_flag) {
        // Copies may still be in flight after an abort: wait (bounded) for the
        // last armed phase of every stage.
        for (int j = max(0, armed - kStages); j < armed; ++j) {
            pkv::mbar_wait_bounded(bar_addr(bars.kv_full[j % kStages]), (j / kStages) & 1, kWaitPolls);
        }
    }
    __syncthreads();
    if (warp == kMmaWarp) {
        pkv::tc::fence_after_sync();
        pkv::tc::tmem_dealloc(tmem, kTmemCols);
    }
}

constexpr int kMaxDevices = 64;

// Per device: the kernel's dynamic shared-memory limit raised once.
int prepare(int device) {
    static std::atomic<int> done[kMaxDevices] = {};
    if (device >= 0 && device < kMaxDevices && done[device].load(std::memory_order_acquire)) return PKV_OK;
    const cudaError_t e = cudaFuncSetAttribute(prefill_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               kSmemBytes);
    if (e != cudaSuccess) {
        return pkv::fail(PKV_CUDA_ERROR, std::string("prefill attention: cudaFuncSetAttribute: ") +
                                             cudaGetErrorString(e));
    }
    if (device >= 0 && device < kMaxDevices) done[device].store(1, std::memory_order_release);
    return PKV_OK;
}

}  // namespace

namespace pkv {

// Launch of the tcgen05 prefill attention (arguments checked by the caller).
int launch_prefill_attention_tc(const void *pool, int32_t num_blocks, int32_t layer, const void *query,
                                int64_t query_stride, const int32_t *blocks, int32_t start, int32_t tokens,
                                void *out, int64_t out_stride, int32_t *error_flag, cudaStream_t stream) {
    int device = 0;
    cudaError_t e = cudaGetDevice(&device);
    if (e != cudaSuccess) return fail(PKV_CUDA_ERROR, std::string("cudaGetDevice: ") + cudaGetErrorString(e));
    int rc = prepare(device);
    if (rc) return rc;
    CUtensorMap map;
    if ((rc = pool_tensor_map(pool, num_blocks, &map))) return rc;
    TcArgs args;
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
    const int tiles = (tokens + kTileTokens - 1) / kTileTokens;
    prefill_tc_kernel<<<tiles * kKvHeads, kThreads, kSmemBytes, stream>>>(map, args);
    e = cudaGetLastError();
    if (e != cudaSuccess) {
        return fail(PKV_CUDA_ERROR, std::string("prefill attention launch failed: ") + cudaGetErrorString(e));
    }
    return PKV_OK;
}

}  // namespace pkv
