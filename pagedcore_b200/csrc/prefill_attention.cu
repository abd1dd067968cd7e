// C-ABI entry of the causal prompt (prefill) attention: argument checks, then
// the tcgen05 kernel of prefill_attention_tc.cu.
//
// The attention of a prompt chunk whose K/V already sit in the pool: token t
// of the chunk (position start + t) attends to positions 0 .. start + t of
// its request, over the 16-token blocks its block table lists.  It stands in
// for the causal attention of PagedCore's dense prefill (dense_attention,
// src/pagedcore/dense.py:69-82, with the mask of decoder.py:225) with the
// numerics of its paged attention (attention.py:14-53: FP32 scores, softmax
// and sum from FP16 pages, one FP16 rounding of the output):
//   out[t,h] = sum_{p <= start+t} softmax_p(q[t,h] . K[p, h/8] * 0.125) V[p, h/8]

#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "pagedkv.h"
#include "status.h"

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
    if (num_blocks < 1 || static_cast<int64_t>(PKV_LAYERS) * 2 * num_blocks * PKV_BLOCK_TOKENS > INT32_MAX) {
        return pkv::fail(PKV_VALUE_ERROR, "prefill attention: pool block count out of range");
    }
    if (tokens < 1 || start < 0 || static_cast<int64_t>(start) + tokens > PKV_CONTEXT_LIMIT) {
        return pkv::fail(PKV_VALUE_ERROR, "prefill attention: the chunk must hold 1 or more tokens at positions below 2048");
    }
    // 16-byte copies of pool rows and query rows (cp.async) and of output rows.
    const int64_t row = static_cast<int64_t>(PKV_QUERY_HEADS) * PKV_HEAD_DIM;
    if ((reinterpret_cast<uintptr_t>(pool) & 15) || (reinterpret_cast<uintptr_t>(query) & 15) ||
        (reinterpret_cast<uintptr_t>(out) & 15) || (reinterpret_cast<uintptr_t>(blocks) & 3) || query_stride % 8 ||
        out_stride % 8 || query_stride < row || out_stride < row) {
        return pkv::fail(PKV_VALUE_ERROR, "prefill attention: misaligned tensor");
    }
    return pkv::launch_prefill_attention_tc(pool, num_blocks, layer, query, query_stride, blocks, start, tokens, out,
                                            out_stride, error_flag, static_cast<cudaStream_t>(stream));
}
