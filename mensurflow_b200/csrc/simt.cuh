// Bandwidth-bound SIMT kernels of the path: gemv/matvec, the standalone bias_add/activation
// pass, and the "no products" (k == 0) epilogue.
#pragma once

#include <cstdint>

#include "gemm_tc.cuh"

namespace mfk {

// ---- gemv ------------------------------------------------------------------------------------
// y[i] = alpha * sum_j A[i, j] x[j] + beta * y0[i], the sum accumulated in double as the
// reference's gemv_f32 / matvec_f32 do (src/backends/cpu/ops/blas/blas.cpp:55-80). A is
// row-major with row stride lda. One warp per row; each lane streams 16-byte chunks of the row,
// so a warp reads 512 contiguous bytes per load instruction.

constexpr int kGemvThreads = 256;
constexpr int kGemvBlocksPerSm = 32;  // at most, launched per SM (four resident at 64 registers)
constexpr int kGemvLoads = 8;        // 16-byte loads of A in flight per lane

__device__ __forceinline__ double warp_sum(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float gemv_finish(double sum, float alpha, float beta,
                                             const float* y0, long long i) {
    return static_cast<float>(static_cast<double>(alpha) * sum +
                              (beta == 0.0f ? 0.0 : static_cast<double>(beta) * y0[i]));
}

// A streamed once: read-only, not kept in L1, and the L2 asked to fetch whole 256-byte sectors.
__device__ __forceinline__ float4 ld_stream_f4(const float4* p) {
    float4 v;
    asm("ld.global.nc.L1::no_allocate.L2::256B.v4.f32 {%0, %1, %2, %3}, [%4];"
        : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
        : "l"(p));
    return v;
}

// The products of four fp32 pairs are exact in double; summed left to right.
__device__ __forceinline__ double dot4_f64(float4 v, float4 w) {
    return (double)v.x * w.x + (double)v.y * w.y + (double)v.z * w.z + (double)v.w * w.w;
}

// One warp per row where the grid allows (the block scheduler then balances the rows; a grid
// stride beyond kGemvBlocksPerSm blocks per SM); a lane keeps kGemvLoads 16-byte loads of its
// row in flight and sums their products on four double chains. At 65536 x 8192 in a probe of
// back-to-back launches on one B200: 6.87 TB/s, against 6.72 with 8 blocks per SM walking ~7
// rows per warp and 5.3 for two rows per warp with four loads in flight.
__global__ void __launch_bounds__(kGemvThreads, 4) gemv_n_vec4_kernel(
    const float* __restrict__ a, long long rows, long long cols, long long lda,
    const float* __restrict__ x, float alpha, float beta, const float* __restrict__ y0,
    float* __restrict__ y) {
    constexpr int kWarps = kGemvThreads / 32;
    const int lane = threadIdx.x % 32;
    const long long nwarps = static_cast<long long>(gridDim.x) * kWarps;
    const long long cols4 = cols / 4;
    const float4* x4 = reinterpret_cast<const float4*>(x);
    for (long long row = static_cast<long long>(blockIdx.x) * kWarps + threadIdx.x / 32;
         row < rows; row += nwarps) {
        const float4* a4 = reinterpret_cast<const float4*>(a + row * lda);
        double s[4] = {0.0, 0.0, 0.0, 0.0};
        long long j = lane;
        for (; j + 32 * (kGemvLoads - 1) < cols4; j += 32 * kGemvLoads) {
            float4 v[kGemvLoads];
#pragma unroll
            for (int u = 0; u < kGemvLoads; ++u) v[u] = ld_stream_f4(a4 + j + 32 * u);
#pragma unroll
            for (int u = 0; u < kGemvLoads; ++u) s[u % 4] += dot4_f64(v[u], __ldg(x4 + j + 32 * u));
        }
        for (; j < cols4; j += 32) s[0] += dot4_f64(ld_stream_f4(a4 + j), __ldg(x4 + j));
        for (long long t = cols4 * 4 + lane; t < cols; t += 32) {
            s[1] += (double)a[row * lda + t] * (double)x[t];
        }
        const double sum = warp_sum((s[0] + s[1]) + (s[2] + s[3]));
        if (lane == 0) y[row] = gemv_finish(sum, alpha, beta, y0, row);
    }
}

__global__ void __launch_bounds__(kGemvThreads) gemv_n_scalar_kernel(
    const float* __restrict__ a, long long rows, long long cols, long long lda,
    const float* __restrict__ x, long long incx, float alpha, float beta,
    const float* __restrict__ y0, float* __restrict__ y) {
    const int lane = threadIdx.x % 32;
    const long long row = (static_cast<long long>(blockIdx.x) * kGemvThreads + threadIdx.x) / 32;
    if (row >= rows) return;
    double s = 0.0;
    for (long long j = lane; j < cols; j += 32) s += (double)a[row * lda + j] * (double)x[j * incx];
    s = warp_sum(s);
    if (lane == 0) y[row] = gemv_finish(s, alpha, beta, y0, row);
}

// Transposed: y[i] = alpha * sum_j A[j, i] x[j] + beta*y0[i] for i < cols. Threads run along
// i (coalesced rows of A); the j range is split over blockIdx.y into partial double sums,
// reduced in a fixed order by gemv_t_finish_kernel (deterministic).
constexpr int kGemvTRowsPerChunk = 512;

__global__ void __launch_bounds__(256) gemv_t_partial_kernel(const float* __restrict__ a,
                                                             long long rows, long long cols,
                                                             long long lda,
                                                             const float* __restrict__ x,
                                                             long long incx,
                                                             double* __restrict__ partial) {
    const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= cols) return;
    const long long j0 = static_cast<long long>(blockIdx.y) * kGemvTRowsPerChunk;
    const long long j1 = min(rows, j0 + kGemvTRowsPerChunk);
    double s = 0.0;
    for (long long j = j0; j < j1; ++j) s += (double)a[j * lda + i] * (double)x[j * incx];
    partial[static_cast<long long>(blockIdx.y) * cols + i] = s;
}

__global__ void __launch_bounds__(256) gemv_t_finish_kernel(const double* __restrict__ partial,
                                                            int chunks, long long cols,
                                                            float alpha, float beta,
                                                            const float* __restrict__ y0,
                                                            float* __restrict__ y) {
    const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= cols) return;
    double s = 0.0;
    for (int c = 0; c < chunks; ++c) s += partial[static_cast<long long>(c) * cols + i];
    y[i] = gemv_finish(s, alpha, beta, y0, i);
}

// ---- bias_add + activation -------------------------------------------------------------------
// out[r, j] = act(x[r, j] + bias[j]) for a contiguous [rows, cols] x (bias optional): the
// reference's bias_add_f32 (elementwise.cpp:128-137) and relu_f32 / gelu_f32 (:158, :173-192).
__global__ void __launch_bounds__(256) bias_act_vec4_kernel(const float4* __restrict__ x,
                                                            const float* __restrict__ bias,
                                                            float4* __restrict__ out,
                                                            long long total4, long long cols,
                                                            int act) {
    const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
    for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < total4;
         i += stride) {
        float4 v = x[i];
        if (bias != nullptr) {
            const long long j = (i * 4) % cols;  // cols % 4 == 0: all four share the row
            v.x = __fadd_rn(v.x, bias[j]);
            v.y = __fadd_rn(v.y, bias[j + 1]);
            v.z = __fadd_rn(v.z, bias[j + 2]);
            v.w = __fadd_rn(v.w, bias[j + 3]);
        }
        v.x = apply_act(v.x, act);
        v.y = apply_act(v.y, act);
        v.z = apply_act(v.z, act);
        v.w = apply_act(v.w, act);
        out[i] = v;
    }
}

__global__ void __launch_bounds__(256) bias_act_scalar_kernel(const float* __restrict__ x,
                                                              const float* __restrict__ bias,
                                                              float* __restrict__ out,
                                                              long long total, long long cols,
                                                              int act) {
    const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
    for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += stride) {
        float v = x[i];
        if (bias != nullptr) v = __fadd_rn(v, bias[i % cols]);
        out[i] = apply_act(v, act);
    }
}

// ---- k == 0 ------------------------------------------------------------------------------
// No products: C = act(alpha*0 + beta*C_in + bias), batched, C row-major (ldc, c_bs).
__global__ void __launch_bounds__(256) epilogue_only_kernel(GemmArgs g) {
    const long long total = static_cast<long long>(g.batch) * g.m * g.n;
    const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
    const bool has_cin = g.c_in != nullptr && g.beta != 0.0f;
    for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += stride) {
        const long long b = i / (static_cast<long long>(g.m) * g.n);
        const long long rem = i - b * g.m * g.n;
        const long long r = rem / g.n, j = rem - r * g.n;
        const float cin = has_cin ? g.c_in[b * g.c_in_bs + r * g.c_in_rs + j * g.c_in_cs] : 0.0f;
        const float bv = g.bias != nullptr ? g.bias[j] : 0.0f;
        g.c[b * g.c_bs + r * g.ldc + j] =
            epilogue_value(0.0f, g.alpha, g.beta, cin, has_cin, bv, g.bias != nullptr, g.act);
    }
}

}  // namespace mfk

namespace mfk {

// ---- softmax / log_softmax / where (the ops between attention's two GEMMs) -------------------
// Softmax along one axis of a contiguous [outer, length, inner] tensor, as the reference's
// softmax_f32 / log_softmax_f32 (src/backends/cpu/ops/softmax/softmax.cpp:11-80): the line's max
// (a NaN anywhere makes the whole line NaN), e = exp(x - max) in fp32, the sum of e in double,
// out = e * float(1 / sum) — or, for log_softmax, (x - max) - float(log(sum)). A line that is
// entirely -inf gives zeros (softmax) or -inf (log_softmax). `keep`/`causal` (attention) mask
// entries to -inf first, as the reference's where(keep, scores, -inf) does before its softmax
// (src/ops/attention.cpp:82-96): entry (b, i, j) of a [batch, rows, cols] last-axis softmax is
// kept when keep[b*keep_bs + i*keep_rs + j] != 0 and, with causal, j <= i.

__device__ __forceinline__ float nan_max(float a, float b) {
    return (isnan(a) || a > b) ? a : b;
}

__device__ __forceinline__ float warp_nan_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = nan_max(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

struct SoftmaxMask {
    const unsigned char* keep;  // optional
    long long keep_bs, keep_rs;
    int causal;
    long long rows;             // lines per matrix (for the causal index and keep addressing)
};

__device__ __forceinline__ float masked_value(float v, const SoftmaxMask& mk, long long line,
                                              long long j) {
    if (mk.causal || mk.keep) {
        const long long i = line % mk.rows;
        if (mk.causal && j > i) return -INFINITY;
        if (mk.keep) {
            const long long b = line / mk.rows;
            if (!mk.keep[b * mk.keep_bs + i * mk.keep_rs + j]) return -INFINITY;
        }
    }
    return v;
}

// Last-axis lines (inner == 1): one warp per line; values re-read from L1/L2 between passes.
__global__ void __launch_bounds__(256) softmax_lastdim_kernel(const float* __restrict__ x,
                                                              float* __restrict__ out,
                                                              long long lines, long long length,
                                                              int log_softmax, SoftmaxMask mk) {
    const int lane = threadIdx.x % 32;
    const long long line = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) / 32;
    if (line >= lines) return;
    const float* in = x + line * length;
    float* dst = out + line * length;
    float m = -INFINITY;
    for (long long j = lane; j < length; j += 32) m = nan_max(m, masked_value(in[j], mk, line, j));
    m = warp_nan_max(m);
    if (m == -INFINITY) {
        for (long long j = lane; j < length; j += 32) dst[j] = log_softmax ? -INFINITY : 0.0f;
        return;
    }
    double sum = 0.0;
    for (long long j = lane; j < length; j += 32) {
        const float e = expf(masked_value(in[j], mk, line, j) - m);
        if (!log_softmax) dst[j] = e;
        sum += static_cast<double>(e);
    }
    sum = warp_sum(sum);
    if (log_softmax) {
        const float log_sum = static_cast<float>(log(sum));
        for (long long j = lane; j < length; j += 32)
            dst[j] = (masked_value(in[j], mk, line, j) - m) - log_sum;
    } else {
        const float scale = static_cast<float>(1.0 / sum);
        __syncwarp();
        for (long long j = lane; j < length; j += 32) dst[j] *= scale;
    }
}

// Lines along a non-last axis (inner > 1): one thread per line, neighbouring threads on
// neighbouring `inner` positions so every pass reads coalesced.
__global__ void __launch_bounds__(256) softmax_strided_kernel(const float* __restrict__ x,
                                                              float* __restrict__ out,
                                                              long long outer, long long length,
                                                              long long inner, int log_softmax) {
    const long long line = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (line >= outer * inner) return;
    const long long base = (line / inner) * length * inner + line % inner;
    const float* in = x + base;
    float* dst = out + base;
    float m = -INFINITY;
    for (long long j = 0; j < length; ++j) m = nan_max(m, in[j * inner]);
    if (m == -INFINITY) {
        for (long long j = 0; j < length; ++j) dst[j * inner] = log_softmax ? -INFINITY : 0.0f;
        return;
    }
    double sum = 0.0;
    for (long long j = 0; j < length; ++j) {
        const float e = expf(in[j * inner] - m);
        if (!log_softmax) dst[j * inner] = e;
        sum += static_cast<double>(e);
    }
    if (log_softmax) {
        const float log_sum = static_cast<float>(log(sum));
        for (long long j = 0; j < length; ++j) dst[j * inner] = (in[j * inner] - m) - log_sum;
    } else {
        const float scale = static_cast<float>(1.0 / sum);
        for (long long j = 0; j < length; ++j) dst[j * inner] *= scale;
    }
}

// out[i] = cond[i] ? x[i] : y[i] over contiguous, already broadcast inputs (where_f32).
__global__ void __launch_bounds__(256) where_kernel(const unsigned char* __restrict__ cond,
                                                    const float* __restrict__ x,
                                                    const float* __restrict__ y,
                                                    float* __restrict__ out, long long n) {
    const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
    for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += stride)
        out[i] = cond[i] ? x[i] : y[i];
}

}  // namespace mfk

// ---- bias_add backward: the bias gradient ----------------------------------------------------
//
// out[j] = sum over rows r of g[r*ld + j], accumulated in fp32 in row order from 0 — the
// reference's loop (src/ops/elementwise.cpp:263-283, on the host there), so the result is
// identical bit for bit. The order leaves one sequential chain per column; the kernel gives each
// block 32 columns, stages 128-row tiles of them through a 3-deep cp.async ring (all 256 threads
// load, a warp reads one 128-byte row segment per instruction) and lets warp 0 run the 32
// chains out of shared memory, so HBM latency hides behind the ring rather than the chains.
namespace mfk {

constexpr int kBgCols = 32;
constexpr int kBgRows = 128;
constexpr int kBgStages = 3;
constexpr int kBgThreads = 256;

__device__ __forceinline__ void cp_async_4(uint32_t dst, const float* src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(dst), "l"(src) : "memory");
}

__global__ void __launch_bounds__(kBgThreads) bias_grad_kernel(const float* __restrict__ g,
                                                               long long rows, long long cols,
                                                               long long ld,
                                                               float* __restrict__ out) {
    __shared__ float tile[kBgStages][kBgRows][kBgCols];  // 48 KB
    const int lane = threadIdx.x % 32;
    const int warp = threadIdx.x / 32;
    const long long col = static_cast<long long>(blockIdx.x) * kBgCols + lane;
    const bool col_ok = col < cols;
    const long long ntiles = (rows + kBgRows - 1) / kBgRows;
    auto load = [&](long long t) {
        const int buf = static_cast<int>(t % kBgStages);
        const long long r0 = t * kBgRows;
#pragma unroll
        for (int i = 0; i < kBgRows / (kBgThreads / 32); ++i) {
            const int r = warp + (kBgThreads / 32) * i;
            if (col_ok && r0 + r < rows) {
                cp_async_4(static_cast<uint32_t>(__cvta_generic_to_shared(&tile[buf][r][lane])),
                           g + (r0 + r) * ld + col);
            }
        }
        cp_async_commit();  // one group per tile, empty or not, so the wait counts line up
    };
    for (long long t = 0; t < kBgStages - 1; ++t) load(t);
    float acc = 0.0f;
    for (long long t = 0; t < ntiles; ++t) {
        load(t + kBgStages - 1);           // past the last tile: an empty group
        cp_async_wait<kBgStages - 1>();    // tile t has landed (this thread's copies)
        __syncthreads();                   // ... and every thread's
        if (warp == 0 && col_ok) {
            const int buf = static_cast<int>(t % kBgStages);
            const long long left = rows - t * kBgRows;
            const int nr = left < kBgRows ? static_cast<int>(left) : kBgRows;
            for (int r = 0; r < nr; ++r) acc += tile[buf][r][lane];
        }
        __syncthreads();                   // the buffer is free before it is refilled
    }
    if (warp == 0 && col_ok) out[col] = acc;
}

// ---- self-test of the bounded waits ---------------------------------------------------------
// One CTA waits on an mbarrier that nothing will ever complete, through the same bounded wait
// the GEMM pipeline uses, with a short limit: the wait gives up, records `kErrSelfTest` in the
// device error word and the kernel returns normally, leaving the context usable.
constexpr unsigned int kErrSelfTest = 1u << 4;

__global__ void wait_selftest_kernel(unsigned long long limit_ns, unsigned int* gave_up) {
    __shared__ uint64_t bar;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        fence_barrier_init();
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        // nothing arrives on `bar`, so phase 0 never completes
        const bool done = mbar_wait(&bar, 0, kErrSelfTest, limit_ns);
        *gave_up = done ? 0u : 1u;
    }
}

}  // namespace mfk
