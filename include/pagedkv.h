/*
 * pagedkv.h - C ABI of the B200 paged KV-cache hot path.
 *
 * This is the drop-in boundary that replaces the Python hot path of
 * PagedCore (src/pagedcore/kv_cache.py and src/pagedcore/attention.py).
 * Every entry point takes plain pointers and sizes; no framework types
 * cross this boundary.  Device pointers are CUDA device addresses on the
 * current device; `stream` is a cudaStream_t passed as void*.
 *
 * Status convention: every int-returning function returns PKV_OK (0) on
 * success, otherwise one of the PKV_* codes below, and the calling thread's
 * message is available from pkv_last_error().  A host binding maps
 * PKV_VALUE_ERROR -> ValueError, PKV_RUNTIME_ERROR / PKV_CUDA_ERROR ->
 * RuntimeError, PKV_KEY_ERROR -> KeyError, which is the exception contract of
 * the reference's KVAllocator and paged_attention.  A failing call leaves
 * the ledger unchanged (kv_cache.py:174-178, 204-219).
 *
 * Pool layout (kv_cache.py:39-43): FP16 [22][2][num_blocks][16][4][64],
 * contiguous.  A slot id is physical_block * 16 + slot_in_block.
 */
#ifndef PAGEDKV_H
#define PAGEDKV_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define PKV_ABI_VERSION 1

/* Geometry fixed by the reference (kv_cache.py:39-43, 72-82; config.py:24-89). */
#define PKV_LAYERS 22
#define PKV_KV_HEADS 4
#define PKV_QUERY_HEADS 32
#define PKV_HEAD_DIM 64
#define PKV_BLOCK_TOKENS 16
#define PKV_CONTEXT_LIMIT 2048
#define PKV_MAX_CREDITS 128

enum {
    PKV_OK = 0,
    PKV_VALUE_ERROR = 1,
    PKV_RUNTIME_ERROR = 2,
    PKV_KEY_ERROR = 3,
    PKV_CUDA_ERROR = 4
};

/* Validation levels of a ledger. FULL re-checks every invariant of
 * KVAllocator._assert_accounting (kv_cache.py:314-357) on every call;
 * INCREMENTAL checks only the requests and blocks a call touches. */
enum { PKV_VALIDATE_INCREMENTAL = 0, PKV_VALIDATE_FULL = 1 };

/* Device error-flag bits set by the kernels (host reads the int32 flag). */
enum {
    PKV_DEVICE_BAD_BLOCK = 1,     /* physical block id outside [0, num_blocks) */
    PKV_DEVICE_BAD_POSITION = 2,  /* RoPE position outside [0, 2048) */
    PKV_DEVICE_WAIT_TIMEOUT = 4   /* a bounded mbarrier wait gave up */
};

/* Thread-local message of the last failing call on this thread. */
const char *pkv_last_error(void);
int pkv_abi_version(void);

/* ------------------------------------------------------------------------ */
/* Block ledger (host).  Replaces KVAllocator's bookkeeping.                 */
/* ------------------------------------------------------------------------ */
typedef struct pkv_ledger pkv_ledger;

/* KVAllocator.__init__ (kv_cache.py:71-90): LIFO free list [N-1, ..., 0],
 * so the first pops are 0, 1, 2, ... */
int pkv_ledger_new(int32_t num_blocks, int32_t validation, pkv_ledger **out);
void pkv_ledger_free(pkv_ledger *ledger);
int pkv_ledger_set_validation(pkv_ledger *ledger, int32_t validation);

/* KVAllocator.create (kv_cache.py:92-110): grant credits, assign nothing. */
int pkv_ledger_reserve(pkv_ledger *ledger, int64_t request, int64_t credits);

/* KVAllocator.release_all (kv_cache.py:286-298): the request's first block
 * becomes the top of the free stack. */
int pkv_ledger_release(pkv_ledger *ledger, int64_t request);

/* KVAllocator.capacity (kv_cache.py:112-115, 348-357): out = {total, free,
 * owned, reserved, active_slots, live_cached_token_slots}. */
int pkv_ledger_capacity(pkv_ledger *ledger, int64_t out[6]);

/* KVAllocator.cached_length / block_table (kv_cache.py:117-125). */
int pkv_ledger_length(pkv_ledger *ledger, int64_t request, int32_t *out_length);
int pkv_ledger_table(pkv_ledger *ledger, int64_t request, int32_t *out_blocks,
                     int32_t capacity, int32_t *out_count);

/* KVAllocator.append, split in two (kv_cache.py:127-179).  plan validates and
 * writes the slot id of each of `tokens` new positions (new blocks come from
 * the top of the free stack: free[-1], free[-2], ...) without changing state;
 * commit publishes them after the device write was issued. */
int pkv_ledger_append_plan(pkv_ledger *ledger, int64_t request, int32_t tokens,
                           int32_t *out_slots, int32_t *out_start_position);
int pkv_ledger_append_commit(pkv_ledger *ledger, int64_t request, int32_t tokens);

/* Several KVAllocator.append calls at once, for a batched write of several
 * prompts in one kernel launch.  Request i (all distinct) is planned as if
 * requests 0..i-1 had been committed before it, so the slots are those that
 * the same appends made one after another would get; out_slots receives
 * tokens[0] + ... + tokens[count-1] slot ids in request order and
 * out_start_positions[i] each request's first position.  No state changes
 * until commit_many, which checks every request before changing any (a
 * failing batch changes nothing). */
int pkv_ledger_append_plan_many(pkv_ledger *ledger, const int64_t *requests, const int32_t *tokens,
                                int32_t count, int32_t *out_slots, int32_t *out_start_positions);
int pkv_ledger_append_commit_many(pkv_ledger *ledger, const int64_t *requests, const int32_t *tokens,
                                  int32_t count);

/* KVAllocator.append_decode (kv_cache.py:181-219): stage length+1 for each
 * request, borrowing free[-1], free[-2], ... in request order for requests
 * whose length is a multiple of 16.  Writes each row's slot id and RoPE
 * position (= cached length before the append). */
int pkv_ledger_decode_begin(pkv_ledger *ledger, const int64_t *requests, int32_t count,
                            int32_t *out_slots, int32_t *out_positions);
/* write_decode_layer's checks (kv_cache.py:226-243) for one staged request,
 * or for every staged request when request == -1; returns its slot/position. */
int pkv_ledger_decode_check(pkv_ledger *ledger, int64_t request, int32_t layer,
                            int32_t *out_slot, int32_t *out_position);
/* Record that `layer` was written (kv_cache.py:246); request == -1: all rows. */
int pkv_ledger_decode_mark(pkv_ledger *ledger, int64_t request, int32_t layer);
/* Record layers first .. first+count-1 as written for every staged row, each
 * row's next layer being `first` (the checks of pkv_ledger_decode_check, once;
 * for a step whose launches were enqueued together, e.g. as a CUDA graph). */
int pkv_ledger_decode_mark_layers(pkv_ledger *ledger, int32_t first, int32_t count);
/* Commit needs all 22 layers written (kv_cache.py:208-217); both commit and
 * abort leave no staged state behind. */
int pkv_ledger_decode_commit(pkv_ledger *ledger);
void pkv_ledger_decode_abort(pkv_ledger *ledger);
int pkv_ledger_decode_active(pkv_ledger *ledger);

/* The table and length that attention sees for one request at `layer`: the
 * staged view for a staged request whose layer was written, else the
 * committed one (kv_cache.py:248-270). */
int pkv_ledger_view(pkv_ledger *ledger, int64_t request, int32_t layer, int32_t *out_blocks,
                    int32_t capacity, int32_t *out_count, int32_t *out_length);

/* Device-ready metadata for a batch at `layer` (the batched form of
 * iter_layer_blocks): lengths[count], prefix[count+1] (cumulative block
 * counts) and the flat concatenation of the tables, flat[prefix[b] + j] =
 * physical block of logical block j of row b.  flat_capacity bounds flat.
 * layer == PKV_VIEW_STAGED gives every staged row's staged view (length + 1,
 * new block included) whatever layers were written: the view of a caller
 * that writes the new token in the same launch (pkv_decode_layer). */
#define PKV_VIEW_STAGED (-2)
int pkv_ledger_batch(pkv_ledger *ledger, const int64_t *requests, int32_t count, int32_t layer,
                     int32_t *out_lengths, int32_t *out_prefix, int32_t *out_flat,
                     int32_t flat_capacity, int32_t *out_total_blocks);

/* Full invariant check of kv_cache.py:314-357. */
int pkv_ledger_audit(pkv_ledger *ledger);

/* Free stack, bottom to top (the reference's _free_blocks list order). */
int pkv_ledger_free_list(pkv_ledger *ledger, int32_t *out, int32_t capacity, int32_t *out_count);
/* Replace the free stack by a permutation of itself (seeded fragmentation;
 * the reference's invariants treat the free list as a set, kv_cache.py:331-340). */
int pkv_ledger_reorder_free(pkv_ledger *ledger, const int32_t *blocks, int32_t count);

/* White-box hooks for corruption tests (the reference's tests write
 * _sequences and _free_blocks directly, tests/unit/test_kv_cache.py:572-677).
 * They bypass every check and are never used by the product path. */
int pkv_ledger_debug_set_table(pkv_ledger *ledger, int64_t request, const int32_t *blocks,
                               int32_t count, int32_t length);
int pkv_ledger_debug_set_free(pkv_ledger *ledger, const int32_t *blocks, int32_t count);

/* ------------------------------------------------------------------------ */
/* Device kernels (sm_100a).                                                */
/* ------------------------------------------------------------------------ */

/* Bytes of the RoPE table the caller provides: FP16 cos[2048][32] followed by
 * FP16 sin[2048][32], built with the reference's exact op sequence
 * (dense.py:48-54) so the rotation is bit-exact. */
int64_t pkv_rope_table_bytes(void);

/* Scatter K/V rows into the pool through slot ids, optionally rotating K
 * (and a query tensor) with the RoPE table.  Replaces the per-block copy_ of
 * KVAllocator.append (kv_cache.py:161-172), the two copy_ of
 * write_decode_layer (kv_cache.py:244-245) and, when rope_table is not NULL,
 * apply_rope (dense.py:33-61) on K and Q:
 *   k' = fp16(fp16(k*cos) + fp16(rotate_half(k)*sin)).
 * key/value: FP16, element (l, t, h, d) at base + l*src_layer_stride +
 * t*src_token_stride + h*64 + d, for l in [0, layer_count), t in [0, tokens).
 * Pool layer = layer_begin + l.  slots[t], positions[t]: int32 device arrays.
 * query_in/query_out (nullable, both or neither): FP16, element (l, t, h, d) at
 * base + l*q_layer_stride + t*q_token_stride + h*64 + d, h in [0, 32).
 * All element strides must be multiples of 8 and base pointers 16-byte aligned. */
int pkv_append_kv(void *pool, int32_t num_blocks, int32_t layer_begin, int32_t layer_count,
                  const void *key, const void *value, int64_t src_layer_stride,
                  int64_t src_token_stride, const int32_t *slots, const int32_t *positions,
                  int32_t tokens, const void *rope_table, const void *query_in, void *query_out,
                  int64_t q_layer_stride, int64_t q_token_stride, int32_t *error_flag,
                  void *stream);

/* Launch plan of the split-K decode attention for `total_blocks` 16-token
 * blocks of a batch of `batch` sequences on `device`.  The flat block list is
 * cut into one contiguous piece per CTA: big_ctas pieces of blocks_per_cta
 * blocks, then grid - big_ctas pieces of tail_blocks blocks (the last piece
 * may be shorter); big_ctas == grid is the uniform split.  Also returns the
 * bytes of workspace the caller must provide, zeroed before its first use
 * and otherwise left to the library: the first 2 KiB hold slot-claim
 * counters (when the grid is one full wave of CTAs, each CTA takes the
 * pieces assigned to the SM it runs on; every launch leaves these at zero),
 * then 16 * grid bytes of four uint32 wall-time counters per piece
 * (nanoseconds each warp ran, added to on every launch, never cleared by the
 * library), then the split partials.  Launches that share a workspace must not overlap
 * on the GPU. */
int pkv_decode_plan(int32_t device, int32_t batch, int32_t total_blocks, int32_t *out_grid,
                    int32_t *out_blocks_per_cta, int32_t *out_big_ctas, int32_t *out_tail_blocks,
                    int64_t *out_workspace_bytes);

/* Piece tables of a batch (host memory in and out; no device work).  Cuts the
 * flat list of prefix[batch] blocks into `grid` contiguous, nonempty pieces
 * (1 <= grid <= prefix[batch]) so that every piece carries the same cost,
 * where a block costs 1 and each row start inside a piece costs `row_cost`
 * more (the row switch of the decode kernel), times the piece's relative
 * speed weights[g] when `weights` (host float [grid], positive) is given.
 * Writes pieces [grid][4] = (begin, end, first row, that row's first block)
 * and row_pieces [batch][2] = (first, last piece) of each row.  The result
 * depends only on the arguments. */
int pkv_decode_tables(const int32_t *prefix, int32_t batch, int32_t grid, const float *weights, float row_cost,
                      int32_t *pieces, int32_t *row_pieces);

/* Batched one-token block-table decode attention with GQA (8 query heads per
 * KV head).  Replaces paged_attention (attention.py:14-53) for a whole batch:
 *   out[b,h] = sum_t softmax_t(q[b,h] . K[t, h/8] * 0.125) V[t, h/8]
 * over the lengths[b] cached tokens of row b at pool layer `layer`, FP32
 * accumulation, one FP16 rounding.  query: FP16 [batch][32][64] with row
 * stride query_stride (elements); out likewise with out_stride.
 * lengths[batch], prefix[batch+1] (prefix[0] == 0), flat[total_blocks]:
 * int32 device arrays as written by pkv_ledger_batch.  grid / blocks_per_cta /
 * big_ctas / tail_blocks / workspace come from pkv_decode_plan for the same
 * (batch, total_blocks), or describe another partition that covers the
 * blocks exactly.  pieces / row_pieces (nullable, both or neither; device):
 * the tables pkv_decode_tables makes for `grid` pieces, 16- and 4-byte
 * aligned; with them the pieces are the tables' (grid must match them, the
 * partition arguments are ignored), without them every CTA takes the
 * partition's piece and searches prefix for its first row.  Two launches: the split kernel and, when
 * grid > 1, the combine kernel as its programmatic dependent. */
int pkv_decode_attention(const void *pool, int32_t num_blocks, int32_t layer, const void *query,
                         int64_t query_stride, const int32_t *lengths, const int32_t *prefix,
                         const int32_t *flat, const int32_t *pieces, const int32_t *row_pieces, int32_t batch,
                         int32_t total_blocks, int32_t grid, int32_t blocks_per_cta, int32_t big_ctas,
                         int32_t tail_blocks, void *out, int64_t out_stride, void *workspace, int64_t workspace_bytes,
                         int32_t *error_flag, void *stream);

/* pkv_decode_layer flags.  PKV_DECODE_EARLY_KV: the kernel enqueued just
 * before this call on `stream` writes no pool data of `layer` and none of the
 * tables (lengths, prefix, flat, pieces, row_pieces), and if it is the second
 * kernel of a decode launch on the same workspace, that launch was for a layer
 * of the other parity (consecutive layers); the split kernel then claims its
 * piece and starts streaming K/V before that kernel completes (it is launched
 * as a programmatic dependent either way). */
#define PKV_DECODE_EARLY_KV 1

/* One decode layer for a staged batch: the fused form of write_decode_layer
 * (kv_cache.py:221-246) + apply_rope on Q and K (dense.py:33-61) +
 * paged_attention (attention.py:14-53).  For every row b the new token sits
 * at position lengths[b]-1 (lengths/prefix/flat from pkv_ledger_batch with
 * PKV_VIEW_STAGED); its K (rotated) and V are written to its pool slot at
 * `layer`, Q is rotated at the same position, and the attention over all
 * lengths[b] tokens is written to out.  query: unrotated FP16 [batch][32][64]
 * (rows query_stride apart); key/value: FP16 [batch][4][64] (rows kv_stride
 * apart); rope_table as for pkv_append_kv.  Plan, workspace and piece tables as
 * for pkv_decode_attention; one split launch plus, when grid > 1, the
 * combine launch. */
int pkv_decode_layer(void *pool, int32_t num_blocks, int32_t layer, const void *query, int64_t query_stride,
                     const void *key, const void *value, int64_t kv_stride, const void *rope_table,
                     const int32_t *lengths, const int32_t *prefix, const int32_t *flat, const int32_t *pieces,
                     const int32_t *row_pieces, int32_t batch, int32_t total_blocks, int32_t grid,
                     int32_t blocks_per_cta, int32_t big_ctas, int32_t tail_blocks, void *out, int64_t out_stride,
                     void *workspace, int64_t workspace_bytes, int32_t *error_flag, int32_t flags, void *stream);

/* Causal attention of a prompt chunk through its block table: the attention
 * step of the prefill (dense_attention, dense.py:69-82, with decoder.py:225's
 * mask) computed from the pool with paged_attention's numerics
 * (attention.py:14-53: FP32 from FP16 pages, one FP16 rounding).  The chunk's
 * `tokens` tokens sit at positions start .. start+tokens-1 of one request, and
 * their K/V at `layer` are already in the pool (pkv_append_kv); token t attends
 * to positions 0 .. start+t.  blocks: int32 device array, the physical block of
 * each of the ceil((start+tokens)/16) blocks of the request (its block table);
 * slots at or past start+tokens are never read.  query: rotated FP16
 * [tokens][32][64], rows query_stride elements apart; out likewise with
 * out_stride; pool, query and out 16-byte aligned, both strides multiples of
 * 8.  start + tokens <= 2048.  Allocates nothing, no workspace; one launch of
 * min(ceil(tokens/16) x 4, 2 x SMs) persistent CTAs on the tensor cores
 * (tcgen05).  Block ids outside [0, num_blocks) set PKV_DEVICE_BAD_BLOCK and
 * read as zeros. */
int pkv_prefill_attention(const void *pool, int32_t num_blocks, int32_t layer, const void *query,
                          int64_t query_stride, const int32_t *blocks, int32_t start, int32_t tokens, void *out,
                          int64_t out_stride, int32_t *error_flag, void *stream);

/* pkv_decode_attention without any allocation.  No counterpart in the
 * reference: it is for callers that cannot allocate device memory for this
 * library (a host whose device memory is all owned by another allocator, or a
 * plugin host with no workspace callback).  Same arguments and result as
 * pkv_decode_attention minus the workspace: the split partials live in one
 * 8 MiB file-scope device array, which every GPU that loads the library holds
 * until exit.  Limit: the plan's workspace_bytes (pkv_decode_plan),
 * 2048 + 16 * grid + 8448 * (batch + grid), must not exceed 8 MiB, i.e.
 * batch + grid <= (8388608 - 2048 - 16 * grid) / 8448 (991 at the full-wave
 * grid of 444 on a B200, so batch <= 547), else PKV_VALUE_ERROR.  The first
 * call on a device looks up the array's device address (cudaGetSymbolAddress)
 * and sets the kernel attributes with that device current; make that first
 * call before any stream capture.  All calls share the array and it keeps the
 * last call's contents (every partial is written before it is read within one
 * call; each call clears the slot-claim counters at its start on `stream`,
 * without allocating), so calls that overlap on the
 * GPU - on different streams, or on one device from different threads - race
 * and must be serialised by the caller.  The per-slot warp wall-time counters
 * in the array grow with every call and are never cleared (nothing reads them
 * on this entry point).  Calls no cudaMalloc / cudaFree. */
int pkv_decode_attention_noalloc(const void *pool, int32_t num_blocks, int32_t layer, const void *query,
                                 int64_t query_stride, const int32_t *lengths, const int32_t *prefix,
                                 const int32_t *flat, const int32_t *pieces, const int32_t *row_pieces, int32_t batch,
                                 int32_t total_blocks, int32_t grid, int32_t blocks_per_cta, int32_t big_ctas,
                                 int32_t tail_blocks, void *out, int64_t out_stride, int32_t *error_flag,
                                 void *stream);

/* ---- Batched decoder step: fused elementwise chains ------------------------
 * Replace chains of eager ops of the reference's dense decoder
 * (src/pagedcore/dense.py) for the rows of a batched decode step; each keeps
 * the chain's FP16 rounding points (only the order of the FP32 sum of squares
 * differs).  FP16 row-major tensors, 16-byte aligned; kernels on `stream`. */

/* Residual add and RMSNorm (dense.py:17-21): when delta is not null,
 * hidden[r] = fp16(hidden[r] + delta[r]) in place; then
 * out[r] = fp16(weight * fp16(hidden[r] * rsqrt(mean(hidden[r]^2) + eps))),
 * the mean and rsqrt in FP32.  hidden, delta, out [rows][dim], weight [dim];
 * dim a multiple of 8 up to 8192. */
int pkv_add_rms_norm(void *hidden, const void *delta, const void *weight, void *out, int32_t rows, int32_t dim,
                     float eps, void *stream);

/* SwiGLU's product (dense.py:84-91): out[r][c] = fp16(fp16(silu(g)) * u) with
 * g = gate_up[r][c], u = gate_up[r][inter + c], silu in FP32.  gate_up
 * [rows][2 * inter], out [rows][inter]. */
int pkv_silu_mul(const void *gate_up, void *out, int32_t rows, int32_t inter, void *stream);

/* A linear layer (F.linear, dense.py's projections) for 1 to 8 rows:
 * y[m][n] = fp16(sum_k x[m][k] * w[n][k]), the FP32 sum rounded once.  x
 * [rows][k] with rows x_stride elements apart, w [n][k] contiguous, y rows
 * y_stride elements apart; k a multiple of 8, x and w 16-byte aligned.  At
 * decode batches of a few rows the layer is bound by reading w once. */
int pkv_gemv(const void *x, int64_t x_stride, const void *w, int32_t rows, int32_t n, int32_t k, void *y,
             int64_t y_stride, void *stream);

/* Linear layer of the batched decode step on the tcgen05 tensor cores
 * (replaces the batch-shaped F.linear of the reference's projections,
 * dense.py:24-30, 84-109, called row by row in decoder.py:178-198):
 * y[t][n] = sum_k x[t][k] * w[n][k] for 1..256 rows of x, FP16 operands, FP32
 * accumulation.  x [rows][k] with rows x_stride elements apart (x_stride a
 * multiple of 8, x 16-byte aligned), w [n][k] contiguous and 16-byte aligned,
 * n a multiple of 128 and k of 64.  The K range is cut into `splits` pieces
 * (1 .. k/64; pkv_linear_splits gives the one that covers the GPU): with one
 * split y is written as FP16 to out (rows out_stride elements apart); with
 * more, FP32 partial sums go to partials [splits][rows][n] (16-byte aligned)
 * and a consumer adds them in split order: pkv_split_sum, or the fused
 * pkv_add_rms_norm_split / pkv_silu_mul_split.  A timed-out pipeline wait sets
 * PKV_DEVICE_WAIT_TIMEOUT in error_flag.  Allocates nothing. */
int pkv_linear_splits(int32_t rows, int32_t n, int32_t k, int32_t *out_splits);
int pkv_linear(const void *x, int64_t x_stride, const void *w, int32_t rows, int32_t n, int32_t k, int32_t splits,
               void *out, int64_t out_stride, void *partials, int32_t *error_flag, void *stream);

/* out[t][c] = fp16(sum_s partials[s][t][c]) in split order (the FP16 output
 * of a split pkv_linear); n a multiple of 4, out rows out_stride apart. */
int pkv_split_sum(const void *partials, int32_t splits, int32_t rows, int32_t n, void *out, int64_t out_stride,
                  void *stream);

/* pkv_add_rms_norm with delta = fp16(sum_s partials[s]) of a split pkv_linear
 * ([splits][rows][dim] FP32): the output projection's or the down
 * projection's split sums go straight into the next residual add and norm. */
int pkv_add_rms_norm_split(void *hidden, const void *partials, int32_t splits, const void *weight, void *out,
                           int32_t rows, int32_t dim, float eps, void *stream);

/* pkv_silu_mul with gate_up = fp16(sum_s partials[s]) of a split gate/up
 * pkv_linear ([splits][rows][2 * inter] FP32); inter a multiple of 8. */
int pkv_silu_mul_split(const void *partials, int32_t splits, void *out, int32_t rows, int32_t inter, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* PAGEDKV_H */
