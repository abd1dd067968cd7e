// Linear layers of the batched decode step on the sm_100a tensor cores:
// y[t][n] = sum_k x[t][k] * w[n][k]  (F.linear without bias, the projections of
// PagedCore's dense.py:24-30, 84-109), FP16 operands, FP32 accumulation.
//
// Shape of the problem.  A decode step multiplies a few hundred rows (one per
// sequence) by weight matrices of 2048-32000 rows: the weight is the large
// operand and is read once, so the layer is bound by streaming it (at 256
// rows it also reaches the tensor peak).  The MMA therefore takes the weight
// as its M side ("swap AB"): D[128 weight rows][T tokens] = W_tile . X^T with
// M = 128, N = T rounded up to 16 (<= 256), K = 16 per instruction, D in
// TMEM (one column per token).
//
// Work split.  One CTA per (128-row weight tile, K split): the K range of a
// tile is cut into `splits` contiguous pieces so that tiles x splits CTAs
// cover the GPU even for the 2048-row projections.  With splits = 1 the CTA
// writes y as FP16; with more, each CTA writes its FP32 partial sums to
// partials[split][t][n] and the next kernel of the step adds the splits in a
// fixed order (pkv_split_sum, or the fused residual-add + RMSNorm / SwiGLU
// kernels), so results do not depend on timing.
//
// Roles (192 threads): warp 4 issues the TMA loads (a 128 x 64 weight box
// and a T x 64 box of x per stage, 128-byte swizzle, no multicast; rows of x
// past T read as zeros) into a 4-stage ring; warp 5 owns the TMEM allocation
// and one of its threads issues the MMAs (4 per stage) and commits each stage
// back to the producer; warps 0-3 (thread r = weight row r = TMEM lane r)
// read D from TMEM 32 tokens at a time, turn it around in shared memory and
// store each token's 128 outputs as one coalesced row of 16-byte stores.
// Every wait is bounded; a timeout sets PKV_DEVICE_WAIT_TIMEOUT.

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <functional>
#include <mutex>
#include <string>
#include <unordered_map>

#include "pagedkv.h"
#include "ptx.cuh"
#include "status.h"
#include "tcgen05.cuh"
#include "pdl.h"
#include "tensor_maps.h"

namespace {

constexpr int kTileRows = 128;   // MMA M: weight rows per tile
constexpr int kKBlock = 64;      // K per stage: one 128-byte swizzle row
constexpr int kMaxTokens = 256;  // MMA N limit
constexpr int kMaxStages = 4;
constexpr int kSmemPerCta = 4 * (16 + 32) * 1024 + 1024;  // 4 stages at 256 rows: one CTA per SM
constexpr int kThreads = 192;
constexpr int kProducerWarp = 4;
constexpr int kMmaWarp = 5;
constexpr int kWBytes = kTileRows * kKBlock * 2;  // 16 KiB
constexpr uint32_t kWaitPolls = 1u << 24;

struct LinearArgs {
    __half *out;          // splits == 1: y [tokens][out_stride]
    float *partials;      // splits > 1: [splits][tokens][n]
    int64_t out_stride;
    int32_t tokens;
    int32_t padded;       // tokens rounded up to 16: MMA N and the x box height
    int32_t n;
    int32_t k_blocks;
    int32_t splits;
    int32_t tiles;
    int32_t stages;       // ring depth (the smem of two CTAs per SM)
    uint32_t tmem_cols;
    int32_t *error_flag;
};

__device__ __forceinline__ bool wait_bounded(uint32_t bar, uint32_t parity, int32_t *error_flag) {
    if (pkv::mbar_wait_bounded(bar, parity, kWaitPolls)) return true;
    atomicOr(error_flag, PKV_DEVICE_WAIT_TIMEOUT);
    return false;
}

__global__ void __launch_bounds__(kThreads, 1)
    linear_tc_kernel(const __grid_constant__ CUtensorMap w_map, const __grid_constant__ CUtensorMap x_map,
                     const LinearArgs a) {
    extern __shared__ uint8_t dyn_smem[];
    __shared__ uint64_t full[kMaxStages], empty[kMaxStages], done;
    __shared__ uint32_t tmem_slot;

    const uint32_t raw = pkv::smem_addr(dyn_smem);
    const uint32_t base = (raw + 1023u) & ~1023u;
    const uint32_t x_bytes = static_cast<uint32_t>(a.padded) * kKBlock * 2;
    const uint32_t stage_bytes = kWBytes + ((x_bytes + 1023u) & ~1023u);

    const int tile = static_cast<int>(blockIdx.x) % a.tiles;
    const int split = static_cast<int>(blockIdx.x) / a.tiles;
    const int kb_begin = static_cast<int>(static_cast<int64_t>(split) * a.k_blocks / a.splits);
    const int kb_end = static_cast<int>(static_cast<int64_t>(split + 1) * a.k_blocks / a.splits);
    const int count = kb_end - kb_begin;
    const int n0 = tile * kTileRows;
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    int issued = 0;  // producer: stages whose copies were issued

    if (warp == kMmaWarp) {
        pkv::tc::tmem_alloc(pkv::smem_addr(&tmem_slot), a.tmem_cols);
        pkv::tc::tmem_relinquish();
    }
    if (threadIdx.x == kProducerWarp * 32) {
        for (int s = 0; s < a.stages; ++s) {
            pkv::mbar_init(pkv::smem_addr(&full[s]), 1);
            pkv::mbar_init(pkv::smem_addr(&empty[s]), 1);
        }
        pkv::mbar_init(pkv::smem_addr(&done), 1);
        pkv::fence_barrier_init();
    }
    pkv::tc::fence_before_sync();
    __syncthreads();
    pkv::tc::fence_after_sync();
    const uint32_t tmem = tmem_slot;
    // Launched as a programmatic dependent: the next kernel may launch now
    // (it waits for this grid before touching its output).
    pkv::pdl_launch_dependents();

    if (warp == kProducerWarp) {
        if (lane == 0) {
            // The weight is streamed once; x is re-read by every tile of its split.
            const uint64_t stream_once = pkv::l2_policy_evict_first();
            const uint64_t reused = pkv::l2_policy_evict_last();
            // The weight does not depend on the previous kernel: the first
            // stages' weight boxes are issued before waiting for it, x after.
            const int early = min(count, a.stages);
            for (int i = 0; i < early; ++i) {
                const uint32_t bar = pkv::smem_addr(&full[i]);
                pkv::mbar_arrive_expect_tx(bar, kWBytes + x_bytes);
                pkv::tma_load_2d_hint(base + i * stage_bytes, &w_map, (kb_begin + i) * kKBlock, n0, bar, stream_once);
            }
            issued = early;
            pkv::pdl_wait();
            for (int i = 0; i < early; ++i) {
                pkv::tma_load_2d_hint(base + i * stage_bytes + kWBytes, &x_map, (kb_begin + i) * kKBlock, 0,
                                      pkv::smem_addr(&full[i]), reused);
            }
            for (int i = early; i < count; ++i) {
                const int st = i % a.stages;
                if (!wait_bounded(pkv::smem_addr(&empty[st]), ((i / a.stages) - 1) & 1, a.error_flag)) break;
                issued = i + 1;
                const uint32_t w_dst = base + st * stage_bytes;
                const uint32_t bar = pkv::smem_addr(&full[st]);
                pkv::mbar_arrive_expect_tx(bar, kWBytes + x_bytes);
                const int kx = (kb_begin + i) * kKBlock;
                pkv::tma_load_2d_hint(w_dst, &w_map, kx, n0, bar, stream_once);
                pkv::tma_load_2d_hint(w_dst + kWBytes, &x_map, kx, 0, bar, reused);
            }
        } else {
            pkv::pdl_wait();
        }
    } else if (warp == kMmaWarp) {
        pkv::pdl_wait();
        if (lane == 0) {
            const uint32_t idesc = pkv::tc::idesc_f16_f32(kTileRows, a.padded, false, false);
            for (int i = 0; i < count; ++i) {
                const int st = i % a.stages;
                if (!wait_bounded(pkv::smem_addr(&full[st]), (i / a.stages) & 1, a.error_flag)) break;
                pkv::tc::fence_after_sync();
                const uint32_t w_src = base + st * stage_bytes;
#pragma unroll
                for (int k = 0; k < kKBlock / 16; ++k) {
                    pkv::tc::mma_f16_ss(tmem, pkv::tc::desc_k_major_sw128(w_src + 32 * k),
                                        pkv::tc::desc_k_major_sw128(w_src + kWBytes + 32 * k), idesc, i > 0 || k > 0);
                }
                pkv::tc::commit(pkv::smem_addr(&empty[st]));
            }
            pkv::tc::commit(pkv::smem_addr(&done));
        }
    } else {
        // Epilogue (warps 0-3): thread r holds weight row n0 + r of every token
        // column.  32 columns at a time go through shared memory (the stage
        // ring is free once every MMA has completed) as [token][128 rows] FP32,
        // so each token's 128 outputs leave as one coalesced row of 16-byte
        // stores instead of 128 scattered ones.
        pkv::pdl_wait();  // the output may still be read by the previous kernel until it completes
        const int r = threadIdx.x;
        const bool ok = wait_bounded(pkv::smem_addr(&done), 0, a.error_flag);
        // One outcome for all 4 epilogue warps (barrier 1 with an AND), so none
        // waits at the barriers below for a warp that gave up.
        uint32_t all_ok;
        asm volatile(
            "{\n\t.reg .pred p, q;\n\t"
            "setp.ne.u32 p, %1, 0;\n\t"
            "bar.red.and.pred q, 1, 128, p;\n\t"
            "selp.u32 %0, 1, 0, q;\n\t}"
            : "=r"(all_ok)
            : "r"(ok ? 1u : 0u)
            : "memory");
        if (all_ok) {
            pkv::tc::fence_after_sync();
            const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;
            float *const staging = reinterpret_cast<float *>(dyn_smem + (base - raw));  // 2 x [32][128] FP32
            for (int c0 = 0, chunk = 0; c0 < a.padded; c0 += 32, ++chunk) {
                uint32_t d[32];
                pkv::tc::tmem_ld32(tmem + lane_base + c0, d);
                pkv::tc::tmem_wait_ld();
                float *tile = staging + (chunk & 1) * (32 * kTileRows);
#pragma unroll
                for (int j = 0; j < 32; ++j) tile[j * kTileRows + r] = __uint_as_float(d[j]);
                // The 4 epilogue warps only (named barrier 1): the two buffers
                // alternate, so one barrier per chunk orders both reuse hazards.
                asm volatile("bar.sync 1, 128;" ::: "memory");
#pragma unroll
                for (int jj = 0; jj < 8; ++jj) {
                    const int j = warp * 8 + jj;
                    const int tok = c0 + j;
                    if (tok >= a.tokens) break;
                    const float4 v = reinterpret_cast<const float4 *>(tile + j * kTileRows)[lane];
                    if (a.splits == 1) {
                        __half2 *dst = reinterpret_cast<__half2 *>(a.out + static_cast<int64_t>(tok) * a.out_stride +
                                                                   n0 + 4 * lane);
                        dst[0] = __floats2half2_rn(v.x, v.y);
                        dst[1] = __floats2half2_rn(v.z, v.w);
                    } else {
                        float *dst = a.partials + (static_cast<int64_t>(split) * a.tokens + tok) * a.n + n0 + 4 * lane;
                        *reinterpret_cast<float4 *>(dst) = v;
                    }
                }
            }
        }
        pkv::tc::fence_before_sync();
    }
    if (warp == kProducerWarp && lane == 0) {
        // No copy may land after the CTA exits: the last phase of each stage
        // (all consumed already unless a wait timed out).
        for (int i = max(0, issued - a.stages); i < issued; ++i) {
            pkv::mbar_wait_bounded(pkv::smem_addr(&full[i % a.stages]), (i / a.stages) & 1, kWaitPolls);
        }
    }
    __syncthreads();
    if (warp == kMmaWarp) {
        pkv::tc::fence_after_sync();
        pkv::tc::tmem_dealloc(tmem, a.tmem_cols);
    }
}

// Sum of the split partials of a linear layer into FP16 y (pkv_split_sum):
// one thread per 4 consecutive outputs of a row.
__global__ void split_sum_kernel(const float *__restrict__ partials, int splits, int tokens, int n,
                                 __half *__restrict__ out, int64_t out_stride) {
    pkv::pdl_launch_dependents();
    pkv::pdl_wait();
    const int quads = n / 4;
    const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (idx >= static_cast<int64_t>(tokens) * quads) return;
    const int t = static_cast<int>(idx / quads);
    const int c = static_cast<int>(idx % quads) * 4;
    const int64_t plane = static_cast<int64_t>(tokens) * n;
    const float *src = partials + static_cast<int64_t>(t) * n + c;
    float4 acc = *reinterpret_cast<const float4 *>(src);
    for (int s = 1; s < splits; ++s) {
        const float4 v = *reinterpret_cast<const float4 *>(src + s * plane);
        acc.x += v.x;
        acc.y += v.y;
        acc.z += v.z;
        acc.w += v.w;
    }
    __half2 *dst = reinterpret_cast<__half2 *>(out + t * out_stride + c);
    dst[0] = __floats2half2_rn(acc.x, acc.y);
    dst[1] = __floats2half2_rn(acc.z, acc.w);
}

// ---------------------------------------------------------------------------
// Host side.
// ---------------------------------------------------------------------------
constexpr int kMaxDevices = 64;

struct MatKey {
    uintptr_t base;
    uint64_t rows, cols, stride;
    uint32_t box_rows;
    bool operator==(const MatKey &o) const {
        return base == o.base && rows == o.rows && cols == o.cols && stride == o.stride && box_rows == o.box_rows;
    }
};
struct MatKeyHash {
    size_t operator()(const MatKey &k) const {
        return std::hash<uintptr_t>()(k.base) ^ (k.rows << 7) ^ (k.cols << 19) ^ (k.stride << 31) ^ k.box_rows;
    }
};

// Tensor maps of weights and activations, cached by (address, shape): the
// decoder's weights and its step buffers keep their addresses.
int cached_matrix_map(const void *base, uint64_t rows, uint64_t cols, uint64_t stride, uint32_t box_rows,
                      CUtensorMap *out) {
    static std::mutex mutex;
    static std::unordered_map<MatKey, CUtensorMap, MatKeyHash> cache;
    const MatKey key{reinterpret_cast<uintptr_t>(base), rows, cols, stride, box_rows};
    std::lock_guard<std::mutex> lock(mutex);
    auto it = cache.find(key);
    if (it != cache.end()) {
        *out = it->second;
        return PKV_OK;
    }
    int rc = pkv::matrix_tensor_map(base, rows, cols, stride, box_rows, out);
    if (rc) return rc;
    if (cache.size() > 4096) cache.clear();
    cache.emplace(key, *out);
    return PKV_OK;
}

int sm_count(int device) {
    static std::atomic<int> cached[kMaxDevices] = {};
    if (device >= 0 && device < kMaxDevices) {
        const int known = cached[device].load(std::memory_order_relaxed);
        if (known > 0) return known;
    }
    int sms = 148;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
    if (device >= 0 && device < kMaxDevices && sms > 0) cached[device].store(sms, std::memory_order_relaxed);
    return sms;
}

int stage_bytes_of(int padded) { return kWBytes + (((padded * kKBlock * 2) + 1023) & ~1023); }

// Ring depth: 4 stages (measured: two CTAs per SM with 2-3 stages each were
// slower at every row count; a deep ring per CTA matters more).
int ring_stages(int padded) {
    const int stages = (kSmemPerCta - 1024) / stage_bytes_of(padded);
    return stages < 2 ? 2 : (stages > kMaxStages ? kMaxStages : stages);
}

int smem_bytes(int padded) { return ring_stages(padded) * stage_bytes_of(padded) + 1024; }

int prepare(int device) {
    static std::atomic<int> done[kMaxDevices] = {};
    if (device >= 0 && device < kMaxDevices && done[device].load(std::memory_order_acquire)) return PKV_OK;
    const cudaError_t e = cudaFuncSetAttribute(linear_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               kSmemPerCta);
    if (e != cudaSuccess) return pkv::fail(PKV_CUDA_ERROR, std::string("linear: cudaFuncSetAttribute: ") + cudaGetErrorString(e));
    if (device >= 0 && device < kMaxDevices) done[device].store(1, std::memory_order_release);
    return PKV_OK;
}

}  // namespace

extern "C" int pkv_linear_splits(int32_t rows, int32_t n, int32_t k, int32_t *out_splits) {
    pkv::clear_error();
    if (out_splits == nullptr || rows < 1 || rows > kMaxTokens || n < kTileRows || n % kTileRows ||
        k < kKBlock || k % kKBlock) {
        return pkv::fail(PKV_VALUE_ERROR, "linear: rows must lie in [1, 256], n and k be multiples of 128 and 64");
    }
    int device = 0;
    cudaGetDevice(&device);
    const int sms = sm_count(device);
    const int tiles = n / kTileRows;
    const int k_blocks = k / kKBlock;
    // About one CTA per SM, at least two K blocks per split.
    int splits = (sms + tiles / 2) / tiles;
    if (splits < 1) splits = 1;
    if (splits > k_blocks / 2) splits = k_blocks / 2 > 0 ? k_blocks / 2 : 1;
    *out_splits = splits;
    return PKV_OK;
}

extern "C" int pkv_linear(const void *x, int64_t x_stride, const void *w, int32_t rows, int32_t n, int32_t k,
                          int32_t splits, void *out, int64_t out_stride, void *partials, int32_t *error_flag,
                          void *stream) {
    pkv::clear_error();
    if (x == nullptr || w == nullptr || error_flag == nullptr) {
        return pkv::fail(PKV_VALUE_ERROR, "linear: null pointer argument");
    }
    if (rows < 1 || rows > kMaxTokens || n < kTileRows || n % kTileRows || k < kKBlock || k % kKBlock) {
        return pkv::fail(PKV_VALUE_ERROR, "linear: rows must lie in [1, 256], n and k be multiples of 128 and 64");
    }
    if (splits < 1 || splits > k / kKBlock) return pkv::fail(PKV_VALUE_ERROR, "linear: splits out of range");
    if (splits == 1 ? out == nullptr : partials == nullptr) {
        return pkv::fail(PKV_VALUE_ERROR, "linear: one split writes out (FP16), more write partials (FP32)");
    }
    if ((reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(w) & 15) || x_stride % 8 ||
        x_stride < k || (splits == 1 && ((reinterpret_cast<uintptr_t>(out) & 1) || out_stride < n)) ||
        (splits > 1 && (reinterpret_cast<uintptr_t>(partials) & 15))) {
        return pkv::fail(PKV_VALUE_ERROR, "linear: misaligned tensor");
    }
    int device = 0;
    cudaError_t e = cudaGetDevice(&device);
    if (e != cudaSuccess) return pkv::fail(PKV_CUDA_ERROR, std::string("cudaGetDevice: ") + cudaGetErrorString(e));
    int rc = prepare(device);
    if (rc) return rc;
    const int padded = (rows + 15) & ~15;
    CUtensorMap w_map, x_map;
    if ((rc = cached_matrix_map(w, static_cast<uint64_t>(n), static_cast<uint64_t>(k), static_cast<uint64_t>(k),
                                kTileRows, &w_map))) {
        return rc;
    }
    if ((rc = cached_matrix_map(x, static_cast<uint64_t>(rows), static_cast<uint64_t>(k),
                                static_cast<uint64_t>(x_stride), static_cast<uint32_t>(padded), &x_map))) {
        return rc;
    }
    LinearArgs args;
    args.out = static_cast<__half *>(out);
    args.partials = static_cast<float *>(partials);
    args.out_stride = out_stride;
    args.tokens = rows;
    args.padded = padded;
    args.n = n;
    args.k_blocks = k / kKBlock;
    args.splits = splits;
    args.tiles = n / kTileRows;
    args.stages = ring_stages(padded);
    uint32_t cols = 32;
    while (cols < static_cast<uint32_t>(padded)) cols <<= 1;
    args.tmem_cols = cols;
    args.error_flag = error_flag;
    cudaLaunchConfig_t config = {};
    config.gridDim = dim3(args.tiles * splits);
    config.blockDim = dim3(kThreads);
    config.dynamicSmemBytes = smem_bytes(padded);
    config.stream = static_cast<cudaStream_t>(stream);
    cudaLaunchAttribute attribute[1];
    attribute[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attribute[0].val.programmaticStreamSerializationAllowed = 1;
    config.attrs = attribute;
    config.numAttrs = 1;
    e = cudaLaunchKernelEx(&config, linear_tc_kernel, w_map, x_map, args);
    if (e != cudaSuccess) return pkv::fail(PKV_CUDA_ERROR, std::string("linear launch failed: ") + cudaGetErrorString(e));
    return PKV_OK;
}

extern "C" int pkv_split_sum(const void *partials, int32_t splits, int32_t rows, int32_t n, void *out,
                             int64_t out_stride, void *stream) {
    pkv::clear_error();
    if (partials == nullptr || out == nullptr || splits < 1 || rows < 1 || n < 4 || n % 4 || out_stride < n ||
        out_stride % 2 || (reinterpret_cast<uintptr_t>(partials) & 15) || (reinterpret_cast<uintptr_t>(out) & 3)) {
        return pkv::fail(PKV_VALUE_ERROR, "split sum: bad arguments");
    }
    const int64_t threads = static_cast<int64_t>(rows) * (n / 4);
    const int block = 256;
    const cudaError_t e = pkv::launch_pdl(split_sum_kernel, dim3(static_cast<unsigned>((threads + block - 1) / block)),
                                          dim3(block), static_cast<cudaStream_t>(stream),
                                          static_cast<const float *>(partials), splits, rows, n,
                                          static_cast<__half *>(out), out_stride);
    if (e != cudaSuccess) return pkv::fail(PKV_CUDA_ERROR, std::string("split sum launch failed: ") + cudaGetErrorString(e));
    return PKV_OK;
}
