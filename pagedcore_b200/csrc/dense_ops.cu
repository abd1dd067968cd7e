// Fused elementwise steps of the batched TinyLlama decoder step.
//
// The reference's decoder (src/pagedcore/dense.py) runs each of these as a
// chain of eager FP16/FP32 tensor ops; on a batch of decode rows every op is
// a separate launch over a few KB, so a decoder step was mostly launch
// latency.  Each kernel here does one chain in one pass and keeps the
// chain's rounding points:
//
//   add_rms_norm  (dense.py:17-21, and the residual adds of dense.py /
//                  decoder.py that precede each norm)
//       hidden = fp16(hidden + delta)                      (when delta given)
//       y      = fp16(hidden * rsqrt(mean(hidden^2) + eps))   in FP32
//       out    = fp16(weight * y)
//   silu_mul      (dense.py:84-91)
//       out = fp16(fp16(silu(gate)) * up),  silu(x) = x / (1 + exp(-x)) in FP32
//
// Every elementwise step is the FP32 operation on FP16 operands rounded to
// FP16, which is what the eager ops compute.  The one difference is the
// order of the FP32 sum of squares (a tree over the row here), so a norm can
// differ from the eager one in the last bit of rare elements.

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "pagedkv.h"
#include "pdl.h"
#include "ptx.cuh"
#include "status.h"

namespace {

constexpr int kNormThreads = 256;
constexpr int kChunk = 8;  // FP16 values per 16-byte access

__device__ __forceinline__ float h2f(__half x) { return __half2float(x); }

// One CTA per row of `dim` values (dim a multiple of 8, at most
// kNormThreads * kChunk * kMaxChunksPerThread).
constexpr int kMaxChunksPerThread = 4;

// fp16 of the sum over `splits` FP32 partial planes (`plane` floats apart) of
// 8 consecutive values: a split-K linear layer's output, rounded once, as the
// FP16 GEMM would round it.
__device__ __forceinline__ uint4 split_sum8(const float *__restrict__ src, int splits, int64_t plane) {
    float4 a = *reinterpret_cast<const float4 *>(src);
    float4 b = *reinterpret_cast<const float4 *>(src + 4);
    for (int s = 1; s < splits; ++s) {
        const float4 c = *reinterpret_cast<const float4 *>(src + s * plane);
        const float4 d = *reinterpret_cast<const float4 *>(src + s * plane + 4);
        a.x += c.x, a.y += c.y, a.z += c.z, a.w += c.w;
        b.x += d.x, b.y += d.y, b.z += d.z, b.w += d.w;
    }
    uint4 r;
    __half2 *h = reinterpret_cast<__half2 *>(&r);
    h[0] = __floats2half2_rn(a.x, a.y);
    h[1] = __floats2half2_rn(a.z, a.w);
    h[2] = __floats2half2_rn(b.x, b.y);
    h[3] = __floats2half2_rn(b.z, b.w);
    return r;
}

// delta is either FP16 [rows][dim] or, with `partials`, the FP16 sum of
// `splits` FP32 planes [splits][rows][dim] of a split-K linear layer.
__global__ void __launch_bounds__(kNormThreads) add_rms_norm_kernel(
    __half *__restrict__ hidden, const __half *__restrict__ delta, const float *__restrict__ partials, int splits,
    int64_t plane, const __half *__restrict__ weight, __half *__restrict__ out, int dim, float eps) {
    __shared__ float partial[kNormThreads / 32];
    // Launched as a programmatic dependent (pkv::launch_pdl): let the next
    // kernel launch, then wait for the previous one before any access.
    pkv::pdl_launch_dependents();
    pkv::pdl_wait();
    const int64_t base = static_cast<int64_t>(blockIdx.x) * dim;
    const int chunks = dim / kChunk;
    float v[kMaxChunksPerThread][kChunk];
    float sum = 0.f;
#pragma unroll
    for (int j = 0; j < kMaxChunksPerThread; ++j) {
        const int c = threadIdx.x + j * kNormThreads;
        if (c < chunks) {
            uint4 raw = *reinterpret_cast<const uint4 *>(hidden + base + c * kChunk);
            const __half *h = reinterpret_cast<const __half *>(&raw);
            if (delta != nullptr || partials != nullptr) {
                const uint4 draw = partials != nullptr ? split_sum8(partials + base + c * kChunk, splits, plane)
                                                       : *reinterpret_cast<const uint4 *>(delta + base + c * kChunk);
                const __half *d = reinterpret_cast<const __half *>(&draw);
                uint4 sum_raw;
                __half *s = reinterpret_cast<__half *>(&sum_raw);
#pragma unroll
                for (int i = 0; i < kChunk; ++i) s[i] = __float2half_rn(h2f(h[i]) + h2f(d[i]));
                *reinterpret_cast<uint4 *>(hidden + base + c * kChunk) = sum_raw;
                raw = sum_raw;
                h = reinterpret_cast<const __half *>(&raw);
            }
#pragma unroll
            for (int i = 0; i < kChunk; ++i) {
                v[j][i] = h2f(h[i]);
                sum += v[j][i] * v[j][i];
            }
        }
    }
#pragma unroll
    for (int offset = 16; offset > 0; offset >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, offset);
    if ((threadIdx.x & 31) == 0) partial[threadIdx.x >> 5] = sum;
    __syncthreads();
    float total = 0.f;
#pragma unroll
    for (int w = 0; w < kNormThreads / 32; ++w) total += partial[w];
    const float inv = rsqrtf(total / static_cast<float>(dim) + eps);
#pragma unroll
    for (int j = 0; j < kMaxChunksPerThread; ++j) {
        const int c = threadIdx.x + j * kNormThreads;
        if (c < chunks) {
            const uint4 wraw = *reinterpret_cast<const uint4 *>(weight + c * kChunk);
            const __half *w = reinterpret_cast<const __half *>(&wraw);
            uint4 oraw;
            __half *o = reinterpret_cast<__half *>(&oraw);
#pragma unroll
            for (int i = 0; i < kChunk; ++i) {
                const __half y = __float2half_rn(v[j][i] * inv);
                o[i] = __float2half_rn(h2f(w[i]) * h2f(y));
            }
            *reinterpret_cast<uint4 *>(out + base + c * kChunk) = oraw;
        }
    }
}

// The same operation for rows of up to 2048 values, one warp per row and
// two rows per CTA, bit for bit add_rms_norm_kernel's result: lane l holds
// the chunks of that kernel's threads l, 32 + l, ..., 224 + l (one chunk
// each at this width), sums each one's squares in the same order, reduces
// each group of 32 across the lanes with the same butterfly as that kernel's
// warps, and adds the eight group sums in order.  A lane has all of its
// loads (hidden, delta and weight) in flight at once, and a prompt's rows fit
// one wave, where one CTA of 256 threads per row (three resident per SM)
// waits on its loads, its block-wide reduction and then its weight row, in
// several waves.  Used from kRowKernelMinRows rows: measured on B200 at 2047
// rows a prefill step took 5.27 ms with it against 5.38-5.43, while at 256
// rows (one wave of the CTA kernel) a form with eight rows per CTA made the
// decoder step slower (2.264 against 2.217-2.223 ms).
constexpr int kRowWarps = 2;                      // rows per CTA
constexpr int kRowKernelMinRows = 512;
constexpr int kRowGroups = kNormThreads / 32;     // add_rms_norm_kernel's warps
constexpr int kRowMaxDim = kRowGroups * 32 * kChunk;  // 2048

__global__ void __launch_bounds__(kRowWarps * 32) add_rms_norm_rows_kernel(
    __half *__restrict__ hidden, const __half *__restrict__ delta, const __half *__restrict__ weight,
    __half *__restrict__ out, int rows, int dim, float eps) {
    pkv::pdl_launch_dependents();
    pkv::pdl_wait();
    const int lane = threadIdx.x & 31;
    const int row = blockIdx.x * kRowWarps + (threadIdx.x >> 5);
    if (row >= rows) return;
    const int64_t base = static_cast<int64_t>(row) * dim;
    const int chunks = dim / kChunk;
    uint4 raw[kRowGroups], draw[kRowGroups], wraw[kRowGroups];
#pragma unroll
    for (int g = 0; g < kRowGroups; ++g) {
        const int c = g * 32 + lane;
        if (c < chunks) {
            raw[g] = *reinterpret_cast<const uint4 *>(hidden + base + c * kChunk);
            if (delta != nullptr) draw[g] = *reinterpret_cast<const uint4 *>(delta + base + c * kChunk);
            wraw[g] = *reinterpret_cast<const uint4 *>(weight + c * kChunk);
        }
    }
    float group[kRowGroups];
#pragma unroll
    for (int g = 0; g < kRowGroups; ++g) {
        const int c = g * 32 + lane;
        float sum = 0.f;
        if (c < chunks) {
            if (delta != nullptr) {
                const __half *h = reinterpret_cast<const __half *>(&raw[g]);
                const __half *d = reinterpret_cast<const __half *>(&draw[g]);
                uint4 sum_raw;
                __half *s = reinterpret_cast<__half *>(&sum_raw);
#pragma unroll
                for (int i = 0; i < kChunk; ++i) s[i] = __float2half_rn(h2f(h[i]) + h2f(d[i]));
                *reinterpret_cast<uint4 *>(hidden + base + c * kChunk) = sum_raw;
                raw[g] = sum_raw;
            }
            const __half *h = reinterpret_cast<const __half *>(&raw[g]);
#pragma unroll
            for (int i = 0; i < kChunk; ++i) {
                const float v = h2f(h[i]);
                sum += v * v;
            }
        }
        group[g] = sum;
    }
#pragma unroll
    for (int offset = 16; offset > 0; offset >>= 1) {
#pragma unroll
        for (int g = 0; g < kRowGroups; ++g) group[g] += __shfl_xor_sync(0xffffffffu, group[g], offset);
    }
    float total = 0.f;
#pragma unroll
    for (int g = 0; g < kRowGroups; ++g) total += group[g];
    const float inv = rsqrtf(total / static_cast<float>(dim) + eps);
#pragma unroll
    for (int g = 0; g < kRowGroups; ++g) {
        const int c = g * 32 + lane;
        if (c < chunks) {
            const __half *h = reinterpret_cast<const __half *>(&raw[g]);
            const __half *w = reinterpret_cast<const __half *>(&wraw[g]);
            uint4 oraw;
            __half *o = reinterpret_cast<__half *>(&oraw);
#pragma unroll
            for (int i = 0; i < kChunk; ++i) {
                const __half y = __float2half_rn(h2f(h[i]) * inv);
                o[i] = __float2half_rn(h2f(w[i]) * h2f(y));
            }
            *reinterpret_cast<uint4 *>(out + base + c * kChunk) = oraw;
        }
    }
}

__device__ __forceinline__ __half silu_times(__half gate, __half up) {
    const float g = h2f(gate);
    const __half silu = __float2half_rn(g / (1.0f + expf(-g)));
    return __float2half_rn(h2f(silu) * h2f(up));
}

// gate_up [rows][2 * inter] (gate, then up) -> out [rows][inter].  Row
// blockIdx.y (+ gridDim.y ...), 16-byte chunks of 8 values along x.  With
// `partials` the gate/up values are the FP16 sums of `splits` FP32 planes
// [splits][rows][2 * inter] of the split-K gate/up linear layer.
__global__ void silu_mul_kernel(const __half *__restrict__ gate_up, const float *__restrict__ partials, int splits,
                                __half *__restrict__ out, int rows, int inter) {
    pkv::pdl_launch_dependents();
    pkv::pdl_wait();
    const int chunks = inter / kChunk;
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= chunks) return;
    const int64_t plane = static_cast<int64_t>(rows) * 2 * inter;
    for (int row = blockIdx.y; row < rows; row += gridDim.y) {
        const int64_t at = static_cast<int64_t>(row) * 2 * inter + c * kChunk;
        uint4 g, u;
        if (partials != nullptr) {
            g = split_sum8(partials + at, splits, plane);
            u = split_sum8(partials + at + inter, splits, plane);
        } else {
            g = *reinterpret_cast<const uint4 *>(gate_up + at);
            u = *reinterpret_cast<const uint4 *>(gate_up + at + inter);
        }
        const __half *gh = reinterpret_cast<const __half *>(&g);
        const __half *uh = reinterpret_cast<const __half *>(&u);
        uint4 r;
        __half *rh = reinterpret_cast<__half *>(&r);
#pragma unroll
        for (int i = 0; i < kChunk; ++i) rh[i] = silu_times(gh[i], uh[i]);
        *reinterpret_cast<uint4 *>(out + static_cast<int64_t>(row) * inter + c * kChunk) = r;
    }
}

// Any inter, any alignment: one value a thread.
__global__ void silu_mul_scalar_kernel(const __half *__restrict__ gate_up, __half *__restrict__ out, int rows,
                                       int inter) {
    const int col = blockIdx.x * blockDim.x + threadIdx.x;
    if (col >= inter) return;
    for (int row = blockIdx.y; row < rows; row += gridDim.y) {
        const int64_t base = static_cast<int64_t>(row) * 2 * inter;
        out[static_cast<int64_t>(row) * inter + col] = silu_times(gate_up[base + col], gate_up[base + inter + col]);
    }
}

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

extern "C" int pkv_add_rms_norm(void *hidden, const void *delta, const void *weight, void *out, int32_t rows,
                                int32_t dim, float eps, void *stream) {
    pkv::clear_error();
    if (hidden == nullptr || weight == nullptr || out == nullptr) {
        return pkv::fail(PKV_VALUE_ERROR, "rms norm: hidden, weight and out are required");
    }
    if (rows < 0 || dim < kChunk || dim % kChunk || dim > kNormThreads * kChunk * kMaxChunksPerThread) {
        return pkv::fail(PKV_VALUE_ERROR, "rms norm: dim must be a multiple of 8 up to 8192");
    }
    if (!aligned16(hidden) || !aligned16(weight) || !aligned16(out) || (delta && !aligned16(delta))) {
        return pkv::fail(PKV_VALUE_ERROR, "rms norm: tensors must be 16-byte aligned");
    }
    if (rows == 0) return PKV_OK;
    const cudaError_t err =
        dim <= kRowMaxDim && rows >= kRowKernelMinRows
            ? pkv::launch_pdl(add_rms_norm_rows_kernel, dim3((rows + kRowWarps - 1) / kRowWarps), dim3(kRowWarps * 32),
                              static_cast<cudaStream_t>(stream), static_cast<__half *>(hidden),
                              static_cast<const __half *>(delta), static_cast<const __half *>(weight),
                              static_cast<__half *>(out), static_cast<int>(rows), static_cast<int>(dim), eps)
            : pkv::launch_pdl(add_rms_norm_kernel, dim3(rows), dim3(kNormThreads), static_cast<cudaStream_t>(stream),
                              static_cast<__half *>(hidden), static_cast<const __half *>(delta),
                              static_cast<const float *>(nullptr), 0, static_cast<int64_t>(0),
                              static_cast<const __half *>(weight), static_cast<__half *>(out), dim, eps);
    if (err != cudaSuccess) return pkv::fail(PKV_CUDA_ERROR, std::string("rms norm launch failed: ") + cudaGetErrorString(err));
    return PKV_OK;
}

extern "C" int pkv_silu_mul(const void *gate_up, void *out, int32_t rows, int32_t inter, void *stream) {
    pkv::clear_error();
    if (gate_up == nullptr || out == nullptr || rows < 0 || inter < 1) {
        return pkv::fail(PKV_VALUE_ERROR, "silu_mul: bad arguments");
    }
    if (rows == 0) return PKV_OK;
    const int threads = 128;
    const auto s = static_cast<cudaStream_t>(stream);
    const dim3 grid_rows(1, static_cast<unsigned>(rows < 65535 ? rows : 65535));
    if (inter % kChunk == 0 && aligned16(gate_up) && aligned16(out)) {
        const int chunks = inter / kChunk;
        dim3 grid = grid_rows;
        grid.x = (chunks + threads - 1) / threads;
        const cudaError_t launched = pkv::launch_pdl(silu_mul_kernel, grid, dim3(threads), s,
                                                     static_cast<const __half *>(gate_up),
                                                     static_cast<const float *>(nullptr), 0,
                                                     static_cast<__half *>(out), rows, inter);
        if (launched != cudaSuccess) {
            return pkv::fail(PKV_CUDA_ERROR, std::string("silu_mul launch failed: ") + cudaGetErrorString(launched));
        }
    } else {
        dim3 grid = grid_rows;
        grid.x = (inter + threads - 1) / threads;
        silu_mul_scalar_kernel<<<grid, threads, 0, s>>>(static_cast<const __half *>(gate_up),
                                                        static_cast<__half *>(out), rows, inter);
    }
    const cudaError_t err = cudaGetLastError();
    if (err != cudaSuccess) return pkv::fail(PKV_CUDA_ERROR, std::string("silu_mul launch failed: ") + cudaGetErrorString(err));
    return PKV_OK;
}

extern "C" int pkv_add_rms_norm_split(void *hidden, const void *partials, int32_t splits, const void *weight,
                                      void *out, int32_t rows, int32_t dim, float eps, void *stream) {
    pkv::clear_error();
    if (hidden == nullptr || partials == nullptr || weight == nullptr || out == nullptr || splits < 1) {
        return pkv::fail(PKV_VALUE_ERROR, "rms norm: hidden, partials, weight and out are required");
    }
    if (rows < 0 || dim < kChunk || dim % kChunk || dim > kNormThreads * kChunk * kMaxChunksPerThread) {
        return pkv::fail(PKV_VALUE_ERROR, "rms norm: dim must be a multiple of 8 up to 8192");
    }
    if (!aligned16(hidden) || !aligned16(weight) || !aligned16(out) || !aligned16(partials)) {
        return pkv::fail(PKV_VALUE_ERROR, "rms norm: tensors must be 16-byte aligned");
    }
    if (rows == 0) return PKV_OK;
    const cudaError_t err = pkv::launch_pdl(
        add_rms_norm_kernel, dim3(rows), dim3(kNormThreads), static_cast<cudaStream_t>(stream),
        static_cast<__half *>(hidden), static_cast<const __half *>(nullptr), static_cast<const float *>(partials),
        splits, static_cast<int64_t>(rows) * dim, static_cast<const __half *>(weight), static_cast<__half *>(out), dim,
        eps);
    if (err != cudaSuccess) return pkv::fail(PKV_CUDA_ERROR, std::string("rms norm launch failed: ") + cudaGetErrorString(err));
    return PKV_OK;
}

extern "C" int pkv_silu_mul_split(const void *partials, int32_t splits, void *out, int32_t rows, int32_t inter,
                                  void *stream) {
    pkv::clear_error();
    if (partials == nullptr || out == nullptr || rows < 0 || splits < 1 || inter < kChunk || inter % kChunk ||
        !aligned16(partials) || !aligned16(out)) {
        return pkv::fail(PKV_VALUE_ERROR, "silu_mul: bad arguments");
    }
    if (rows == 0) return PKV_OK;
    const int threads = 128;
    dim3 grid((inter / kChunk + threads - 1) / threads, static_cast<unsigned>(rows < 65535 ? rows : 65535));
    const cudaError_t err = pkv::launch_pdl(silu_mul_kernel, grid, dim3(threads), static_cast<cudaStream_t>(stream),
                                            static_cast<const __half *>(nullptr),
                                            static_cast<const float *>(partials), splits,
                                            static_cast<__half *>(out), rows, inter);
    if (err != cudaSuccess) return pkv::fail(PKV_CUDA_ERROR, std::string("silu_mul launch failed: ") + cudaGetErrorString(err));
    return PKV_OK;
}

// ---------------------------------------------------------------------------
// Small-batch linear layer: y[m][n] = fp16(sum_k x[m][k] * w[n][k]) for M <= 8
// rows of x, the FP32 sum rounded once (as F.linear's FP16 GEMM, in another
// summation order).  At decode batches of a few rows a linear layer is a
// matrix-vector product bound by reading W once; this kernel streams W at
// HBM speed where the library GEMM's small-M tiles do not.  One warp per row
// of W: lane j reads 16-byte chunks j, j + 32, ... of the row, with up to 8
// chunks in flight, and x (a few KB, L1-resident) alongside.
// ---------------------------------------------------------------------------
namespace {

constexpr int kGemvWarps = 8;
constexpr int kGemvUnroll = 8;

__device__ __forceinline__ float dot8(const uint4 &a, const uint4 &b) {
    const __half2 *ah = reinterpret_cast<const __half2 *>(&a);
    const __half2 *bh = reinterpret_cast<const __half2 *>(&b);
    float sum = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float2 af = __half22float2(ah[i]);
        const float2 bf = __half22float2(bh[i]);
        sum = fmaf(af.x, bf.x, sum);
        sum = fmaf(af.y, bf.y, sum);
    }
    return sum;
}

template <int M>
__global__ void __launch_bounds__(kGemvWarps * 32) gemv_kernel(const __half *__restrict__ x, int64_t x_stride,
                                                               const __half *__restrict__ w, int n_rows, int k,
                                                               __half *__restrict__ y, int64_t y_stride) {
    const int lane = threadIdx.x & 31;
    const int chunks = k / kChunk;
    // Launched as a programmatic dependent: the weight does not depend on the
    // previous kernel, so the warp's first row is brought into L2 before the
    // wait for that kernel (which wrote x); x and y only after it.
    pkv::pdl_launch_dependents();
    const int first = blockIdx.x * kGemvWarps + (threadIdx.x >> 5);
    if (first < n_rows) {
        for (int c = lane; c < chunks; c += 32) pkv::prefetch_l2(w + static_cast<int64_t>(first) * k + c * kChunk);
    }
    pkv::pdl_wait();
    for (int n = first; n < n_rows; n += gridDim.x * kGemvWarps) {
        const __half *row = w + static_cast<int64_t>(n) * k;
        float acc[M];
#pragma unroll
        for (int m = 0; m < M; ++m) acc[m] = 0.f;
        for (int c0 = lane; c0 < chunks; c0 += 32 * kGemvUnroll) {
            uint4 wv[kGemvUnroll];
#pragma unroll
            for (int u = 0; u < kGemvUnroll; ++u) {
                const int c = c0 + 32 * u;
                if (c < chunks) wv[u] = *reinterpret_cast<const uint4 *>(row + c * kChunk);
            }
#pragma unroll
            for (int u = 0; u < kGemvUnroll; ++u) {
                const int c = c0 + 32 * u;
                if (c < chunks) {
#pragma unroll
                    for (int m = 0; m < M; ++m) {
                        const uint4 xv = *reinterpret_cast<const uint4 *>(x + m * x_stride + c * kChunk);
                        acc[m] += dot8(wv[u], xv);
                    }
                }
            }
        }
#pragma unroll
        for (int m = 0; m < M; ++m) {
#pragma unroll
            for (int offset = 16; offset > 0; offset >>= 1) acc[m] += __shfl_xor_sync(0xffffffffu, acc[m], offset);
        }
        if (lane == 0) {
#pragma unroll
            for (int m = 0; m < M; ++m) y[m * y_stride + n] = __float2half_rn(acc[m]);
        }
    }
}

template <int M>
cudaError_t launch_gemv(const __half *x, int64_t x_stride, const __half *w, int n, int k, __half *y,
                        int64_t y_stride, cudaStream_t stream) {
    const int grid = (n + kGemvWarps - 1) / kGemvWarps;
    return pkv::launch_pdl(gemv_kernel<M>, dim3(grid), dim3(kGemvWarps * 32), stream, x, x_stride, w, n, k, y,
                           y_stride);
}

}  // namespace

extern "C" int pkv_gemv(const void *x, int64_t x_stride, const void *w, int32_t rows, int32_t n, int32_t k, void *y,
                        int64_t y_stride, void *stream) {
    pkv::clear_error();
    if (x == nullptr || w == nullptr || y == nullptr) return pkv::fail(PKV_VALUE_ERROR, "gemv: x, w and y are required");
    if (rows < 1 || rows > 8 || n < 1 || k < kChunk || k % kChunk) {
        return pkv::fail(PKV_VALUE_ERROR, "gemv: 1 to 8 rows of x, k a multiple of 8");
    }
    if (!aligned16(x) || !aligned16(w) || x_stride % kChunk || y_stride < n) {
        return pkv::fail(PKV_VALUE_ERROR, "gemv: x and w must be 16-byte aligned with row strides in multiples of 8");
    }
    const auto *xh = static_cast<const __half *>(x);
    const auto *wh = static_cast<const __half *>(w);
    auto *yh = static_cast<__half *>(y);
    const auto s = static_cast<cudaStream_t>(stream);
    cudaError_t err = cudaSuccess;
    switch (rows) {
        case 1: err = launch_gemv<1>(xh, x_stride, wh, n, k, yh, y_stride, s); break;
        case 2: err = launch_gemv<2>(xh, x_stride, wh, n, k, yh, y_stride, s); break;
        case 3: err = launch_gemv<3>(xh, x_stride, wh, n, k, yh, y_stride, s); break;
        case 4: err = launch_gemv<4>(xh, x_stride, wh, n, k, yh, y_stride, s); break;
        case 5: err = launch_gemv<5>(xh, x_stride, wh, n, k, yh, y_stride, s); break;
        case 6: err = launch_gemv<6>(xh, x_stride, wh, n, k, yh, y_stride, s); break;
        case 7: err = launch_gemv<7>(xh, x_stride, wh, n, k, yh, y_stride, s); break;
        default: err = launch_gemv<8>(xh, x_stride, wh, n, k, yh, y_stride, s); break;
    }
    if (err != cudaSuccess) return pkv::fail(PKV_CUDA_ERROR, std::string("gemv launch failed: ") + cudaGetErrorString(err));
    return PKV_OK;
}
