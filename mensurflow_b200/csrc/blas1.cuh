// Level-1 kernels the CUDA backend registers besides the GEMM path: the elementwise add / sub /
// mul / div and scal that `gemm`'s composed form and the reference's elementwise ops dispatch,
// and dot. All are single passes over HBM, 16-byte loads where the pointers allow.
//
// Replaces the reference's CUDA backend's cuBLAS compositions (src/backends/cuda/backend.cpp:
// 122-134 dot through cublasSdot, :160-191 add/sub as a copy plus cublasSaxpy, mul as
// cublasSdgmm) with kernels whose results equal the CPU backend's bit for bit: add/sub/mul/div and
// scal are single IEEE fp32 operations per element (src/backends/cpu/ops/elementwise/
// elementwise.cpp add_f32 ..., src/backends/cpu/ops/blas/blas.cpp:23 scal_f32), and dot sums the
// products in double and rounds once (blas.cpp:14-21 dot_f32).
#pragma once

#include <cstdint>

namespace mfk {

enum BinaryOp : int { kBinAdd = 0, kBinSub = 1, kBinMul = 2, kBinDiv = 3 };

template <int Op>
__device__ __forceinline__ float binary_apply(float x, float y) {
    if constexpr (Op == kBinAdd) return __fadd_rn(x, y);
    if constexpr (Op == kBinSub) return __fsub_rn(x, y);
    if constexpr (Op == kBinMul) return __fmul_rn(x, y);
    return __fdiv_rn(x, y);
}

// n4 float4 groups, grid-stride; out may alias x or y (each element is read before it is written
// by the same thread).
template <int Op>
__global__ void __launch_bounds__(256) binary_vec4_kernel(const float4* x, const float4* y,
                                                          float4* out, long long n4) {
    for (long long i = blockIdx.x * 256LL + threadIdx.x; i < n4; i += gridDim.x * 256LL) {
        const float4 a = x[i], b = y[i];
        out[i] = make_float4(binary_apply<Op>(a.x, b.x), binary_apply<Op>(a.y, b.y),
                             binary_apply<Op>(a.z, b.z), binary_apply<Op>(a.w, b.w));
    }
}

template <int Op>
__global__ void __launch_bounds__(256) binary_scalar_kernel(const float* x, const float* y,
                                                            float* out, long long n) {
    for (long long i = blockIdx.x * 256LL + threadIdx.x; i < n; i += gridDim.x * 256LL)
        out[i] = binary_apply<Op>(x[i], y[i]);
}

__global__ void __launch_bounds__(256) scal_vec4_kernel(float alpha, const float4* x, float4* out,
                                                        long long n4) {
    for (long long i = blockIdx.x * 256LL + threadIdx.x; i < n4; i += gridDim.x * 256LL) {
        const float4 a = x[i];
        out[i] = make_float4(__fmul_rn(alpha, a.x), __fmul_rn(alpha, a.y), __fmul_rn(alpha, a.z),
                             __fmul_rn(alpha, a.w));
    }
}

__global__ void __launch_bounds__(256) scal_scalar_kernel(float alpha, const float* x, float* out,
                                                          long long n) {
    for (long long i = blockIdx.x * 256LL + threadIdx.x; i < n; i += gridDim.x * 256LL)
        out[i] = __fmul_rn(alpha, x[i]);
}

// dot, pass 1: block b sums the products of its grid-stride share in double (each product of
// two floats is exact in double) and writes one partial. The order depends only on n and the
// grid, so the result does not change from call to call.
__global__ void __launch_bounds__(256) dot_partial_kernel(const float* __restrict__ x,
                                                          const float* __restrict__ y,
                                                          long long n, int vec4,
                                                          double* __restrict__ partial) {
    double s = 0.0;
    if (vec4) {
        const float4* x4 = reinterpret_cast<const float4*>(x);
        const float4* y4 = reinterpret_cast<const float4*>(y);
        const long long n4 = n / 4;
        for (long long i = blockIdx.x * 256LL + threadIdx.x; i < n4; i += gridDim.x * 256LL) {
            const float4 a = __ldcs(x4 + i), b = __ldcs(y4 + i);
            s += (double)a.x * b.x + (double)a.y * b.y + (double)a.z * b.z + (double)a.w * b.w;
        }
        for (long long i = n4 * 4 + blockIdx.x * 256LL + threadIdx.x; i < n;
             i += gridDim.x * 256LL)
            s += (double)x[i] * y[i];
    } else {
        for (long long i = blockIdx.x * 256LL + threadIdx.x; i < n; i += gridDim.x * 256LL)
            s += (double)x[i] * y[i];
    }
    __shared__ double warp_sums[8];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (threadIdx.x % 32 == 0) warp_sums[threadIdx.x / 32] = s;
    __syncthreads();
    if (threadIdx.x == 0) {
        double t = 0.0;
#pragma unroll
        for (int w = 0; w < 8; ++w) t += warp_sums[w];
        partial[blockIdx.x] = t;
    }
}

// dot, pass 2: one warp adds the partials in a fixed order and rounds once to fp32.
__global__ void dot_finish_kernel(const double* __restrict__ partial, int parts,
                                  float* __restrict__ out) {
    double s = 0.0;
    for (int i = threadIdx.x; i < parts; i += 32) s += partial[i];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (threadIdx.x == 0) *out = static_cast<float>(s);
}

}  // namespace mfk
