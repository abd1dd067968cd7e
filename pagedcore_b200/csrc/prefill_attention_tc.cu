// Causal prompt (prefill) attention through the block table on the sm_100a
// tensor cores (tcgen05 MMAs, TMEM accumulators).
//
// Same operation and numerics as prefill_attention.cu's contract: token t of
// a chunk (position start + t) attends to positions 0 .. start + t of its
// request through its block table, FP32 scores and sums from FP16 pages, one
// FP16 rounding of the output (PagedCore's dense_attention with the mask of
// decoder.py:225, computed as attention.py:14-53 computes a row):
//   out[t,h] = sum_{p <= start+t} softmax_p(q[t,h] . K[p, h/8] * 0.125) V[p, h/8]
//
// Work split - a work item is a (16-token tile, KV head) pair: its M = 128
// MMA rows are the tile's 16 tokens x the 8 query heads of the KV head (row
// r: token r/8, head r%8), so every K/V block is read once per 128 query
// rows.  The grid is persistent (two CTAs per SM); items are ordered longest
// first and CTA c of G takes items c, 2G-1-c, 2G+c, ... so that long and short
// items pair up.  An item walks its keys 64 at a time (four 16-token pool
// blocks), from block 0 to the block of its last token; the CTA's steps are
// counted across its items, so rings, TMEM buffers and barrier phases run on
// from one item to the next without a drain.
//
// Roles (256 threads):
// - warps 4 and 6: the K and V producers.  Each lane copies 16-byte chunks of
//   the step's four blocks (one head: 16 rows x 128 B each) with cp.async
//   into the MMA's 128-byte-swizzled layout, in two rings of shared memory (4
//   K stages, 3 V stages).  Slots at or past start + tokens and blocks outside
//   the pool are zero-filled, so 0 * NaN never reaches a sum.  A step is
//   published after the copies of the step 2 (K) or 1 (V) ahead have been
//   issued and its own have landed (cp.async.wait_group, a proxy fence, an
//   mbarrier arrival per lane).  (TMA loads of the same 2 KiB boxes from one
//   issuing thread measured slower.)
// - warps 5 and 7 (one thread each; warp 5 owns the TMEM allocation): the
//   MMA issuers.  Warp 5 issues S_g = Q . K_g^T (M 128, N 64, K 64: four K=16
//   MMAs) into TMEM S buffer g % 3 once K_g has landed and P.V_{g-3}, which
//   read P_{g-3} from that buffer, has completed; warp 7 issues
//   O += P_g . V_g (M 128, N 64, one K=16 MMA per block) with P_g read from
//   TMEM (the A operand) and V_g from shared memory, into the TMEM O.  Two
//   issuing threads: an MMA and every mbarrier wait take hundreds of cycles,
//   and the two streams are independent.
// - warps 0-3 (128 threads, thread r = row r, TMEM lane r): the softmax.  A
//   thread reads its row of S_g from TMEM (tcgen05.ld), masks positions past
//   its token, and keeps the online softmax state in base 2 in FP32: a
//   reference maximum m that moves only when the row's maximum passes it by
//   more than 2^8.  It writes P_g = 2^(s - m + 7) (<= 2^15) as FP16 over the
//   first 32 columns of S_g's buffer (tcgen05.st, two keys to a column), and
//   sums the FP32 weights into the normaliser l.  When m moves, the thread
//   rescales its row of O in TMEM (ld, multiply, st) once the previous P.V has
//   completed, and l in registers.  At the end of an item O * (1 / l) is
//   rounded to FP16.  The softmax threads also load each item's Q tile
//   (cp.async): the first at start-up, each later one during the last step of
//   the item before it, once s_full shows that every S MMA reading the old
//   tile has completed.
//
// TMEM: S/P buffers at columns 0, 64, 128, O at 192 (256 columns, two CTAs
// per SM).  Shared memory: Q (16 KiB) and the K and V rings.
//
// Block ids outside the pool set PKV_DEVICE_BAD_BLOCK and read as zeros.
// Every wait is bounded: on a timeout the thread sets
// PKV_DEVICE_WAIT_TIMEOUT, the CTA stops issuing work, waits (bounded) for
// its MMAs and its copies in flight, and frees its TMEM.

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>
#include <atomic>
#include <string>

#include "pagedkv.h"
#include "ptx.cuh"
#include "status.h"
#include "tcgen05.cuh"

namespace {

constexpr int kHeadDim = PKV_HEAD_DIM;
constexpr int kKvHeads = PKV_KV_HEADS;
constexpr int kBlockTokens = PKV_BLOCK_TOKENS;
constexpr int kMaxTableBlocks = PKV_CONTEXT_LIMIT / PKV_BLOCK_TOKENS;  // 128
constexpr int kTileTokens = 16;
constexpr int kRows = 128;                  // MMA M: 16 tokens x 8 query heads
constexpr int kStepBlocks = 4;              // pool blocks per step
constexpr int kStepKeys = kStepBlocks * kBlockTokens;  // 64: MMA N of S, K of P.V
constexpr int kKStages = 4;  // K ring: a stage is free once its S MMAs have completed
constexpr int kVStages = 3;  // V ring: a stage is free once its P.V MMAs have completed
constexpr int kRowBytes = kHeadDim * 2;     // 128 B
constexpr int kBoxBytes = kBlockTokens * kRowBytes;    // 2 KiB: one head of one block
constexpr int kBlockElems = kBlockTokens * kKvHeads * kHeadDim;  // one block of one layer's K (or V)
// A producer publishes step j after issuing step j + lag's copies: up to
// lag + 1 steps in flight.  The lag is below the ring's stages (a stage is
// waited for only after the step that last used it was published); V's is 1
// so that V_j is published once P.V_{j-2} has freed its stage, not P.V_{j-1}.
constexpr int kKCopyLag = 2;
constexpr int kVCopyLag = 1;
constexpr int kQBytes = kRows * kRowBytes;             // 16 KiB
constexpr int kRingBytes = kStepBlocks * kBoxBytes;    // 8 KiB: one step's K (or V)
constexpr int kSmemBytes = kQBytes + (kKStages + kVStages) * kRingBytes + 1024;  // + alignment slack
constexpr int kSoftmaxWarps = 4;           // thread r of warps 0-3 owns row r (TMEM lane r)
constexpr int kSoftmaxThreads = kSoftmaxWarps * 32;
constexpr int kThreads = kSoftmaxThreads + 128;
constexpr int kKProducerWarp = kSoftmaxWarps;
constexpr int kMmaWarp = kSoftmaxWarps + 1;  // issues S; owns the TMEM allocation
constexpr int kVProducerWarp = kSoftmaxWarps + 2;
constexpr int kPvWarp = kSoftmaxWarps + 3;   // issues P.V
// TMEM columns: S buffers b = 0, 1, 2 at [64 b, 64 b + 64) (FP32 S_g in buffer
// g % 3, then FP16 P_g over its first 32 columns), O at [192, 256).
constexpr int kSBuffers = 3;
constexpr uint32_t kTmemCols = 256;
constexpr uint32_t kTmemO = kSBuffers * kStepKeys;
static_assert(kTmemO + kHeadDim <= kTmemCols, "S buffers and O exceed the TMEM allocation");
constexpr uint32_t kWaitPolls = 1u << 24;
constexpr uint32_t kSleepNs = 10000;          // a poll sleeps up to 10 us ...
constexpr uint32_t kSleepPolls = 1u << 17;    // ... so a wait gives up after about 1.3 s
constexpr uint32_t kAbortPolls = 1u << 12;  // once the CTA aborts, later waits give up quickly
constexpr float kScaleLog2 = 0.125f * 1.4426950408889634f;  // 64^-0.5 * log2(e)
// P = 2^(s - m + 7) with m the row maximum at its last rescale; m is moved
// only when a row's maximum exceeds it by more than 2^8, so P <= 2^15 stays
// inside FP16 while O and l are rescaled at most a few times per row.
constexpr float kWeightShift = 7.0f;
constexpr float kRescaleLog2 = 8.0f;
static_assert(kRows == kTileTokens * (PKV_QUERY_HEADS / kKvHeads), "a tile's rows are its tokens x 8 heads");
static_assert(kKCopyLag < kKStages && kVCopyLag < kVStages, "a producer would wait for a stage it has not published");

// Instruction descriptors: S = Q . K^T (both K-major), O += P . V (P K-major, V MN-major).
constexpr uint32_t kIdescS = pkv::tc::idesc_f16_f32(kRows, kStepKeys, false, false);
constexpr uint32_t kIdescO = pkv::tc::idesc_f16_f32(kRows, kHeadDim, false, true);

struct TcArgs {
    const __half *pool;
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
    uint64_t k_full[kKStages];   // producer -> MMA: the step's K landed (32 lane arrivals)
    uint64_t k_empty[kKStages];  // MMA -> producer: the step's S MMAs completed
    uint64_t v_full[kVStages];   // producer -> MMA: the step's V landed (32 lane arrivals)
    uint64_t v_empty[kVStages];  // MMA -> producer: the step's P.V MMAs completed
    uint64_t s_full[kSBuffers];  // MMA -> softmax: S_g in TMEM
    uint64_t p_full[kSBuffers];  // softmax -> MMA: P_g in TMEM, O corrected (4 warp arrivals)
    uint64_t pv_done[kSBuffers]; // MMA -> softmax: P_g . V_g completed (its S buffer is free)
    uint64_t q_full;             // softmax -> MMA: the item's Q tile is in place (4 warp arrivals)
    uint64_t s_drained;          // S issuer -> teardown: every S MMA issued completed
    uint64_t pv_drained;         // P.V issuer -> teardown: every P.V MMA issued completed
};

__device__ __forceinline__ uint32_t bar_addr(const uint64_t &b) { return pkv::smem_addr(&b); }

// Bounded wait; on a timeout flags the CTA as aborting.  Each poll may sleep
// up to kSleepNs (the thread wakes when the phase completes), so waiting
// threads do not take issue slots from the softmax by spinning.
__device__ __forceinline__ bool wait_or_abort(uint32_t bar, uint32_t parity, volatile int *abort,
                                              int32_t *error_flag) {
    const uint32_t polls = *abort ? kAbortPolls : kSleepPolls;
    for (uint32_t i = 0; i < polls; ++i) {
        if (pkv::mbar_try_wait_sleep(bar, parity, kSleepNs)) return true;
    }
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

// Work items are (16-token tile, KV head) pairs, longest first: item w is
// tile tiles - 1 - w / 4 of head w % 4.  CTA c of G walks the items c,
// 2G - 1 - c, 2G + c, 4G - 1 - c, ... (a snake over rounds of G items), so a
// CTA that took a long item first takes a short one next.
__device__ __forceinline__ int item_of(int round, int cta, int ctas) {
    return round * ctas + ((round & 1) ? ctas - 1 - cta : cta);
}

struct Item {
    int t0;       // first token of the tile
    int kv;       // KV head
    int nblocks;  // pool blocks up to the tile's last token
    int steps;    // 64-key steps over them
};

__device__ __forceinline__ Item item_info(int w, int tiles, const TcArgs &a) {
    Item it;
    it.kv = w % kKvHeads;
    it.t0 = (tiles - 1 - w / kKvHeads) * kTileTokens;
    const int last_t = min(it.t0 + kTileTokens - 1, a.tokens - 1);
    it.nblocks = (a.start + last_t) / kBlockTokens + 1;
    it.steps = (it.nblocks + kStepBlocks - 1) / kStepBlocks;
    return it;
}

// Row r of an item's Q tile (token r / 8, head kv * 8 + r % 8; 128 B, chunk c
// at c ^ (r % 8)) copied by thread r with cp.async, as one commit group.
__device__ __forceinline__ void load_q_row(uint32_t q_smem, const TcArgs &a, const Item &it, int r) {
    const int t = min(it.t0 + (r >> 3), a.tokens - 1);
    const __half *src = a.query + static_cast<int64_t>(t) * a.query_stride + (it.kv * 8 + (r & 7)) * kHeadDim;
    const uint32_t row = q_smem + (r >> 3) * 1024 + (r & 7) * kRowBytes;
#pragma unroll
    for (int c = 0; c < 8; ++c) pkv::cp_async_16(row + ((c ^ (r & 7)) << 4), src + c * 8, 16u);
    pkv::cp_async_commit();
}

// At most 120 registers a thread: two CTAs of 256 threads then fit an SM
// (the occupancy calculation gives one CTA at 125).
__global__ void __maxnreg__(120)
    prefill_tc_kernel(const TcArgs a) {
    extern __shared__ uint8_t dyn_smem[];
    __shared__ Barriers bars;
    __shared__ int32_t table[kMaxTableBlocks];
    __shared__ uint32_t tmem_slot;
    __shared__ volatile int abort_flag;

    const uint32_t raw = pkv::smem_addr(dyn_smem);
    const uint32_t base = (raw + 1023u) & ~1023u;  // 1024-aligned: swizzle atoms
    const uint32_t q_smem = base;
    const uint32_t k_smem = base + kQBytes;                   // K ring, 8 KiB a stage
    const uint32_t v_smem = k_smem + kKStages * kRingBytes;   // V ring, 8 KiB a stage

    const int tiles = (a.tokens + kTileTokens - 1) / kTileTokens;
    const int items = tiles * kKvHeads;
    const int cta = static_cast<int>(blockIdx.x);
    const int ctas = static_cast<int>(gridDim.x);
    const int written = a.start + a.tokens;  // positions below hold K/V
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    // ---- set-up ----------------------------------------------------------
    // Every item reads the same block table (the chunk's request).
    for (int j = threadIdx.x; j <= (written - 1) / kBlockTokens; j += kThreads) table[j] = a.blocks[j];
    if (warp == kMmaWarp) {
        pkv::tc::tmem_alloc(pkv::smem_addr(&tmem_slot), kTmemCols);
        pkv::tc::tmem_relinquish();
    }
    if (threadIdx.x == kKProducerWarp * 32) {
        for (int s = 0; s < kKStages; ++s) {
            pkv::mbar_init(bar_addr(bars.k_full[s]), 32);  // every producer lane
            pkv::mbar_init(bar_addr(bars.k_empty[s]), 1);
        }
        for (int s = 0; s < kVStages; ++s) {
            pkv::mbar_init(bar_addr(bars.v_full[s]), 32);
            pkv::mbar_init(bar_addr(bars.v_empty[s]), 1);
        }
        for (int b = 0; b < kSBuffers; ++b) {
            pkv::mbar_init(bar_addr(bars.s_full[b]), 1);
            pkv::mbar_init(bar_addr(bars.p_full[b]), kSoftmaxWarps);
            pkv::mbar_init(bar_addr(bars.pv_done[b]), 1);
        }
        pkv::mbar_init(bar_addr(bars.q_full), kSoftmaxWarps);
        pkv::mbar_init(bar_addr(bars.s_drained), 1);
        pkv::mbar_init(bar_addr(bars.pv_drained), 1);
        abort_flag = 0;
        pkv::fence_barrier_init();
    }
    pkv::tc::fence_before_sync();
    __syncthreads();
    pkv::tc::fence_after_sync();
    const uint32_t tmem = tmem_slot;

    // Every role walks the same items; g counts the CTA's 64-key steps over all
    // of them (ring stages, TMEM S buffers and barrier phases follow g).
    if (warp == kKProducerWarp || warp == kVProducerWarp) {
        // ---- producers: K (one warp) and V (another), each its own ring ----
        // A step's four blocks are 512 16-byte chunks: lane l copies chunk
        // l % 8 of slots (l / 8) + 4q, q = 0..3, of every block with cp.async
        // (four 128-byte rows per warp instruction).  Slots at or past
        // start + tokens and blocks outside the pool are zero-filled.  Step g
        // is published once the copies of step g + lag have been issued and
        // its own have landed (cp.async.wait_group, then a proxy fence: the
        // MMA reads the ring through the async proxy).
        const bool is_k = warp == kKProducerWarp;
        const int stages = is_k ? kKStages : kVStages;
        uint64_t *const full = is_k ? bars.k_full : bars.v_full;
        uint64_t *const empty = is_k ? bars.k_empty : bars.v_empty;
        const uint32_t ring = is_k ? k_smem : v_smem;
        const int chunk = lane & 7;
        const int lag = is_k ? kKCopyLag : kVCopyLag;
        const __half *const layer_plane =
            a.pool + static_cast<int64_t>(a.layer * 2 + (is_k ? 0 : 1)) * a.num_blocks * kBlockElems + chunk * 8;
        int g = 0;
        bool stop = false;
        for (int round = 0; !stop; ++round) {
            const int w = item_of(round, cta, ctas);
            if (w >= items) break;
            const Item it = item_info(w, tiles, a);
            const __half *const plane = layer_plane + it.kv * kHeadDim;
            for (int j = 0; j < it.steps; ++j, ++g) {
                if (__any_sync(0xffffffffu, abort_flag)) {  // one decision for the warp
                    stop = true;
                    break;
                }
                const int st = g % stages;
                if (g >= stages &&
                    !warp_wait(bar_addr(empty[st]), ((g / stages) - 1) & 1, &abort_flag, a.error_flag)) {
                    stop = true;
                    break;
                }
                const uint32_t dst = ring + st * kRingBytes;
                const int nb = min(kStepBlocks, it.nblocks - j * kStepBlocks);
#pragma unroll
                for (int kb = 0; kb < kStepBlocks; ++kb) {
                    if (kb >= nb) break;
                    const int index = j * kStepBlocks + kb;
                    const int32_t block = table[index];
                    const bool valid = block >= 0 && block < a.num_blocks;
                    if (!valid && lane == 0) atomicOr(a.error_flag, PKV_DEVICE_BAD_BLOCK);
                    const __half *src = plane + static_cast<int64_t>(valid ? block : 0) * kBlockElems;
#pragma unroll
                    for (int q = 0; q < kBlockTokens / 4; ++q) {
                        const int slot = q * 4 + (lane >> 3);
                        const bool live = valid && index * kBlockTokens + slot < written;
                        pkv::cp_async_16(dst + kb * kBoxBytes + slot * kRowBytes + ((chunk ^ (slot & 7)) << 4),
                                         src + slot * kKvHeads * kHeadDim, live ? 16u : 0u);
                    }
                }
                pkv::cp_async_commit();
                if (g >= lag) {
                    if (is_k) {
                        pkv::cp_async_wait<kKCopyLag>();
                    } else {
                        pkv::cp_async_wait<kVCopyLag>();
                    }
                    pkv::fence_proxy_async_smem();
                    pkv::mbar_arrive(bar_addr(full[(g - lag) % stages]));
                }
            }
        }
        // The last steps (and, after an abort, whatever was issued) land here.
        pkv::cp_async_wait<0>();
        pkv::fence_proxy_async_smem();
        for (int k = max(0, g - lag); k < g; ++k) pkv::mbar_arrive(bar_addr(full[k % stages]));
    } else if (warp == kMmaWarp) {
        // ---- S issuer: S_g = Q . K_g^T into TMEM S buffer g % 2 ---------------
        if (lane == 0) {
            // Descriptors of the tiles' bases; a 16-byte step of a start address
            // is +1 on the descriptor (K slices 32 B apart: +2).
            const uint64_t q_desc = pkv::tc::desc_k_major_sw128(q_smem);
            int g = 0;
            bool stop = false;
            for (int round = 0; !stop; ++round) {
                const int w = item_of(round, cta, ctas);
                if (w >= items) break;
                const Item it = item_info(w, tiles, a);
                // The item's Q tile is in place (the softmax loads it).
                if (!wait_or_abort(bar_addr(bars.q_full), round & 1, &abort_flag, a.error_flag)) break;
                for (int j = 0; j < it.steps; ++j, ++g) {
                    const int st = g % kKStages;
                    // S_g goes into TMEM buffer g % 3 once P.V_{g-3}, which read P_{g-3}
                    // from it, has completed.
                    if (!wait_or_abort(bar_addr(bars.k_full[st]), (g / kKStages) & 1, &abort_flag, a.error_flag) ||
                        (g >= kSBuffers &&
                         !wait_or_abort(bar_addr(bars.pv_done[g % kSBuffers]), ((g - kSBuffers) / kSBuffers) & 1,
                                        &abort_flag, a.error_flag))) {
                        stop = true;
                        break;
                    }
                    pkv::tc::fence_after_sync();
                    const uint64_t k_desc = pkv::tc::desc_k_major_sw128(k_smem + st * kRingBytes);
#pragma unroll
                    for (int k = 0; k < kHeadDim / 16; ++k) {
                        pkv::tc::mma_f16_ss(tmem + (g % kSBuffers) * kStepKeys, q_desc + 2 * k, k_desc + 2 * k, kIdescS,
                                            k > 0);
                    }
                    pkv::tc::commit(bar_addr(bars.s_full[g % kSBuffers]));
                    pkv::tc::commit(bar_addr(bars.k_empty[st]));
                }
            }
            // Teardown: wait until every MMA this thread issued has completed.
            pkv::tc::commit(bar_addr(bars.s_drained));
            if (!pkv::mbar_wait_bounded(bar_addr(bars.s_drained), 0, kWaitPolls)) {
                atomicOr(a.error_flag, PKV_DEVICE_WAIT_TIMEOUT);
            }
        }
    } else if (warp == kPvWarp) {
        // ---- P.V issuer: O += P_g . V_g, one K=16 MMA per block ---------------
        // (a second issuing thread: the S and P.V streams are independent and
        // each commit covers the MMAs of the thread that issued them)
        if (lane == 0) {
            int g = 0;
            bool stop = false;
            for (int round = 0; !stop; ++round) {
                const int w = item_of(round, cta, ctas);
                if (w >= items) break;
                const Item it = item_info(w, tiles, a);
                for (int j = 0; j < it.steps; ++j, ++g) {
                    const int st = g % kVStages;
                    if (!wait_or_abort(bar_addr(bars.p_full[g % kSBuffers]), (g / kSBuffers) & 1, &abort_flag,
                                       a.error_flag) ||
                        !wait_or_abort(bar_addr(bars.v_full[st]), (g / kVStages) & 1, &abort_flag, a.error_flag)) {
                        stop = true;
                        break;
                    }
                    pkv::tc::fence_after_sync();
                    // V boxes are 2 KiB apart (+128 on the descriptor); P's K=16
                    // slices are 8 TMEM columns apart.
                    const uint64_t v_desc = pkv::tc::desc_mn_major_sw128(v_smem + st * kRingBytes);
                    const uint32_t p_tmem = tmem + (g % kSBuffers) * kStepKeys;
                    const int nb = min(kStepBlocks, it.nblocks - j * kStepBlocks);
                    for (int kb = 0; kb < nb; ++kb) {
                        // The item's first MMA overwrites O (read out by the softmax
                        // before it published P_g).
                        pkv::tc::mma_f16_ts(tmem + kTmemO, p_tmem + 8 * kb, v_desc + 128 * kb, kIdescO,
                                            j > 0 || kb > 0);
                    }
                    pkv::tc::commit(bar_addr(bars.pv_done[g % kSBuffers]));
                    pkv::tc::commit(bar_addr(bars.v_empty[st]));
                }
            }
            pkv::tc::commit(bar_addr(bars.pv_drained));
            if (!pkv::mbar_wait_bounded(bar_addr(bars.pv_drained), 0, kWaitPolls)) {
                atomicOr(a.error_flag, PKV_DEVICE_WAIT_TIMEOUT);
            }
        }
    } else {
        // ---- softmax (thread r = MMA row r = TMEM lane r) --------------------
        const int r = threadIdx.x;
        const uint32_t lanes = tmem + (static_cast<uint32_t>(warp * 32) << 16);
        bool ok = true;
        bool s_ready = false;  // s_full(g) seen complete by a test during step g - 1
        int g = 0;
        // The first item's Q tile; each later one is loaded during the last step
        // of the item before it, once every S MMA that read the tile has completed.
        if (item_of(0, cta, ctas) < items) {
            load_q_row(q_smem, a, item_info(item_of(0, cta, ctas), tiles, a), r);
            pkv::cp_async_wait<0>();
            pkv::fence_proxy_async_smem();  // generic-proxy copies -> the MMA's (async proxy) reads
            __syncwarp();
            if (lane == 0) pkv::mbar_arrive(bar_addr(bars.q_full));
        }
        for (int round = 0; ok; ++round) {
            const int w = item_of(round, cta, ctas);
            if (w >= items) break;
            const Item it = item_info(w, tiles, a);
            const int next = item_of(round + 1, cta, ctas);
            const int t = it.t0 + (r >> 3);
            const int pos = a.start + min(t, a.tokens - 1);  // last position this row attends to
            const int head = it.kv * 8 + (r & 7);
            float m = -INFINITY;  // the row maximum at its last rescale (log2 units)
            float l = 0.f;        // sum of this row's weights, relative to m
            for (int j = 0; j < it.steps; ++j, ++g) {
                const uint32_t sbuf = lanes + (g % kSBuffers) * kStepKeys;  // S_g, then P_g
                const bool last = j == it.steps - 1;
                if (!__all_sync(0xffffffffu, s_ready) &&
                    !warp_wait(bar_addr(bars.s_full[g % kSBuffers]), (g / kSBuffers) & 1, &abort_flag,
                               a.error_flag)) {
                    ok = false;
                    break;
                }
                pkv::tc::fence_after_sync();
                uint32_t sr[2][32];
                pkv::tc::tmem_ld32(sbuf, sr[0]);
                pkv::tc::tmem_ld32(sbuf + 32, sr[1]);
                pkv::tc::tmem_wait_ld();
                // s_full of the item's last step: every S MMA of the item has
                // completed, so the next item's Q may replace this one's.
                if (last && next < items) load_q_row(q_smem, a, item_info(next, tiles, a), r);

                float s[64];
#pragma unroll
                for (int c = 0; c < 64; ++c) s[c] = __uint_as_float(sr[c >> 5][c & 31]);
                const int key0 = j * kStepKeys;
                if (key0 + kStepKeys - 1 > a.start + it.t0) {  // the diagonal: mask positions past the row
#pragma unroll
                    for (int c = 0; c < 64; ++c) {
                        if (key0 + c > pos) s[c] = -INFINITY;
                    }
                }
                // Row maximum over 8 independent chains of 3-input maxima: one
                // dependent chain of 64 would cost its full latency every step.
                float mx8[8];
#pragma unroll
                for (int e = 0; e < 8; ++e) mx8[e] = pkv::fmax3(s[e], s[e + 8], s[e + 16]);
#pragma unroll
                for (int e = 0; e < 8; ++e) mx8[e] = pkv::fmax3(mx8[e], s[e + 24], s[e + 32]);
#pragma unroll
                for (int e = 0; e < 8; ++e) mx8[e] = pkv::fmax3(mx8[e], s[e + 40], s[e + 48]);
#pragma unroll
                for (int e = 0; e < 8; ++e) mx8[e] = fmaxf(mx8[e], s[e + 56]);
                const float mx = pkv::fmax3(pkv::fmax3(mx8[0], mx8[1], mx8[2]), pkv::fmax3(mx8[3], mx8[4], mx8[5]),
                                            fmaxf(mx8[6], mx8[7]));
                // Step 0 holds position 0, which every row attends to: m is finite from step 0 on.
                const float m_blk = mx * kScaleLog2;
                const float m_new = m_blk > m + kRescaleLog2 ? m_blk : m;  // m = -inf at step 0: always moves
                // P_g as FP16 (x 2^7) over the first 32 columns of its S buffer,
                // two keys to a column (the A operand of P.V from TMEM); l sums the
                // FP32 weights over 8 independent chains.
                // Pairs of keys go through the packed FP32 instructions (the same
                // rounding as two scalar ones, half the instructions).
                const float shift = kWeightShift - m_new;
                const uint64_t scale2 = pkv::f32x2(kScaleLog2, kScaleLog2);
                const uint64_t shift2 = pkv::f32x2(shift, shift);
                uint64_t l4[4] = {0, 0, 0, 0};  // FP32 pairs: 8 independent chains
#pragma unroll
                for (int half = 0; half < 2; ++half) {
                    uint32_t pr[16];
#pragma unroll
                    for (int c = 0; c < 16; ++c) {
                        const int k = 32 * half + 2 * c;
                        const float2 x = pkv::unpack_f32x2(pkv::fma_f32x2(pkv::f32x2(s[k], s[k + 1]), scale2, shift2));
                        const float lo = pkv::exp2_approx(x.x);
                        const float hi = pkv::exp2_approx(x.y);
                        l4[c & 3] = pkv::add_f32x2(l4[c & 3], pkv::f32x2(lo, hi));
                        pr[c] = pkv::pack_half2(__floats2half2_rn(lo, hi));
                    }
                    pkv::tc::tmem_st16(sbuf + 16 * half, pr);
                }
                float l8[8];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float2 v = pkv::unpack_f32x2(l4[e]);
                    l8[2 * e] = v.x;
                    l8[2 * e + 1] = v.y;
                }
                // Test s_full(g + 1) now: its answer is needed only at the next
                // step, so the test's latency overlaps this step's work.
                s_ready = pkv::mbar_test_wait(bar_addr(bars.s_full[(g + 1) % kSBuffers]), ((g + 1) / kSBuffers) & 1);
                const float corr = m_new != m ? pkv::exp2_approx(m - m_new) : 1.f;  // 0 at step 0, where l is 0
                l = l * corr + (((l8[0] + l8[1]) + (l8[2] + l8[3])) + ((l8[4] + l8[5]) + (l8[6] + l8[7])));
                if (j >= 1 && __any_sync(0xffffffffu, m_new != m)) {
                    // Some row's reference maximum moved: rescale its O (scaled by the
                    // old one so far) once P_{g-1} . V_{g-1} is in it, before
                    // P_g . V_g adds to it.
                    if (!warp_wait(bar_addr(bars.pv_done[(g - 1) % kSBuffers]), ((g - 1) / kSBuffers) & 1, &abort_flag,
                                   a.error_flag)) {
                        ok = false;
                        break;
                    }
                    pkv::tc::fence_after_sync();
#pragma unroll
                    for (int hf = 0; hf < 2; ++hf) {  // O [128, 192)
                        uint32_t o[32];
                        const uint32_t taddr = lanes + kTmemO + 32 * hf;
                        pkv::tc::tmem_ld32(taddr, o);
                        pkv::tc::tmem_wait_ld();
#pragma unroll
                        for (int c = 0; c < 32; ++c) o[c] = __float_as_uint(__uint_as_float(o[c]) * corr);
                        pkv::tc::tmem_st32(taddr, o);
                    }
                }
                pkv::tc::tmem_wait_st();  // P_g (and a rescaled O) written
                m = m_new;
                if (last && next < items) {
                    pkv::cp_async_wait<0>();         // the next item's Q row landed
                    pkv::fence_proxy_async_smem();   // and is ordered before the MMA's (async proxy) reads
                }
                pkv::tc::fence_before_sync();
                __syncwarp();
                if (lane == 0) {
                    pkv::mbar_arrive(bar_addr(bars.p_full[g % kSBuffers]));
                    if (last && next < items) pkv::mbar_arrive(bar_addr(bars.q_full));
                }
            }
            if (!ok) break;
            // The item's output: O / l once its last P.V has completed.
            if (!warp_wait(bar_addr(bars.pv_done[(g - 1) % kSBuffers]), ((g - 1) / kSBuffers) & 1, &abort_flag,
                           a.error_flag)) {
                break;
            }
            pkv::tc::fence_after_sync();
            uint32_t o[2][32];
            pkv::tc::tmem_ld32(lanes + kTmemO, o[0]);
            pkv::tc::tmem_ld32(lanes + kTmemO + 32, o[1]);
            pkv::tc::tmem_wait_ld();
            if (t < a.tokens) {
                uint4 *dst = reinterpret_cast<uint4 *>(a.out + static_cast<int64_t>(t) * a.out_stride +
                                                       head * kHeadDim);
                const float inv = __frcp_rn(l);  // O * (1 / l): within an FP32 ulp of O / l
#pragma unroll
                for (int c8 = 0; c8 < 8; ++c8) {
                    float v[8];
#pragma unroll
                    for (int e = 0; e < 8; ++e) v[e] = __uint_as_float(o[c8 >> 2][(c8 & 3) * 8 + e]) * inv;
                    dst[c8] = make_uint4(pack2(v[0], v[1]), pack2(v[2], v[3]), pack2(v[4], v[5]), pack2(v[6], v[7]));
                }
            }
        }
        pkv::cp_async_wait<0>();  // after an abort: no copy still in flight at exit
        pkv::tc::fence_before_sync();
    }

    // ---- teardown --------------------------------------------------------
    __syncthreads();
    if (warp == kMmaWarp) {
        pkv::tc::fence_after_sync();
        pkv::tc::tmem_dealloc(tmem, kTmemCols);
    }
}

constexpr int kMaxDevices = 64;
constexpr int kCtasPerSm = 2;

// Per device, once: the kernel's dynamic shared-memory limit raised, and the
// number of its CTAs that run at once (2 per SM) recorded in *ctas.
int prepare(int device, int *ctas) {
    static std::atomic<int> resident[kMaxDevices] = {};
    if (device >= 0 && device < kMaxDevices) {
        *ctas = resident[device].load(std::memory_order_acquire);
        if (*ctas > 0) return PKV_OK;
    }
    cudaError_t e = cudaFuncSetAttribute(prefill_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
    if (e == cudaSuccess) {
        // All of the SM's unified L1/shared memory as shared memory: two CTAs' worth.
        e = cudaFuncSetAttribute(prefill_tc_kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                                 cudaSharedmemCarveoutMaxShared);
    }
    if (e != cudaSuccess) {
        return pkv::fail(PKV_CUDA_ERROR, std::string("prefill attention: cudaFuncSetAttribute: ") +
                                             cudaGetErrorString(e));
    }
    int sms = 0;
    e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
    if (e != cudaSuccess || sms < 1) {
        return pkv::fail(PKV_CUDA_ERROR, std::string("prefill attention: SM count query failed: ") +
                                             cudaGetErrorString(e));
    }
    // Two CTAs fit an SM: 2 x (105 KiB + static) of shared memory, 2 x 256
    // columns of TMEM, 2 x 256 threads at 120 registers.
    const int per_sm = kCtasPerSm;
    *ctas = sms * per_sm;
    if (device >= 0 && device < kMaxDevices) resident[device].store(*ctas, std::memory_order_release);
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
    int resident = 0;
    int rc = prepare(device, &resident);
    if (rc) return rc;
    TcArgs args;
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
    // One CTA per resident slot at most; each walks its share of the items.
    const int items = (tokens + kTileTokens - 1) / kTileTokens * kKvHeads;
    prefill_tc_kernel<<<std::min(items, resident), kThreads, kSmemBytes, stream>>>(args);
    e = cudaGetLastError();
    if (e != cudaSuccess) {
        return fail(PKV_CUDA_ERROR, std::string("prefill attention launch failed: ") + cudaGetErrorString(e));
    }
    return PKV_OK;
}

}  // namespace pkv
