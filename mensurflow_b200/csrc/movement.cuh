// Data movement on the device: the strided copy behind Tensor::contiguous() and the Copy op.
//
// The reference gathers a non-contiguous CUDA tensor through a host std::vector (d2h + h2d,
// src/core/tensor.cpp:208-230) because it has no device-side strided copy; on the CPU it runs
// cpu::strided_copy_f32 (one memcpy per innermost contiguous row, an element loop otherwise) or
// cpu::transpose_f32 (32x32 tiles) (src/backends/cpu/ops/movement/movement.cpp:12-67). These
// kernels produce the same bytes on the device. The host has already merged the view's dimensions
// (size-1 dims dropped, dims that are contiguous with their neighbour merged), so the kernel sees
// the fewest dimensions that describe the view:
//  * copy_contig_*: the view is one contiguous run (the Copy op);
//  * copy_rows_kernel: the innermost dim is contiguous in the input (a slice): one warp per
//    4096-element piece of an output row, 16-byte accesses when every row start is 16-byte
//    aligned;
//  * copy_transpose_kernel: some other dim p has input stride 1 (a transposed or permuted
//    view): 64x64 tiles through shared memory, read along p and written along the innermost
//    dim, so both sides are coalesced;
//  * copy_rows_kernel with a strided inner dim: the remaining gathers (no dim of stride 1).
#pragma once

#include <cstdint>

namespace mfk {

constexpr int kMaxCopyDims = 12;

// A view after merging: element (i_0, ..., i_{n-1}) at x[sum_d i_d * stride[d]]; the output is
// row-major over shape.
struct CopyView {
    int ndim;
    long long shape[kMaxCopyDims];
    long long stride[kMaxCopyDims];
};

__global__ void __launch_bounds__(256) copy_contig_vec4_kernel(const float4* __restrict__ x,
                                                               float4* __restrict__ out,
                                                               long long n4) {
    const long long step = static_cast<long long>(gridDim.x) * blockDim.x;
    for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n4;
         i += step) {
        __stcs(out + i, __ldcs(x + i));
    }
}

__global__ void __launch_bounds__(256) copy_contig_kernel(const float* __restrict__ x,
                                                          float* __restrict__ out, long long n) {
    const long long step = static_cast<long long>(gridDim.x) * blockDim.x;
    for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += step) {
        out[i] = x[i];
    }
}

// Input offset of output row `row` (all dims but the innermost), walking the row index from the
// innermost outer dim outwards as the reference's strided_copy_f32 does.
__device__ __forceinline__ long long row_offset(const CopyView& v, long long row) {
    long long off = 0;
    for (int d = v.ndim - 2; d >= 0; --d) {
        const long long s = v.shape[d];
        const long long q = row / s;
        off += (row - q * s) * v.stride[d];
        row = q;
    }
    return off;
}

// One warp per piece of an output row: a row of L = shape[ndim-1] elements is cut into pieces of
// kCopyPiece elements, so a view that merged into a few long rows (a stepped slice of a whole
// matrix is one evenly strided run) still spreads over every SM. VEC4: L % 4 == 0, input stride
// 1, every row start 16-byte aligned on both sides. Launched with one piece per warp where the
// grid allows (a grid stride beyond that), so the block scheduler balances the pieces.
constexpr long long kCopyPiece = 4096;
constexpr int kCopyLoads = 8;

template <bool VEC4>
__global__ void __launch_bounds__(256) copy_rows_kernel(const float* __restrict__ x,
                                                        float* __restrict__ out, CopyView v,
                                                        long long rows) {
    const int lane = threadIdx.x % 32;
    const long long warps = static_cast<long long>(gridDim.x) * (blockDim.x / 32);
    const long long L = v.shape[v.ndim - 1];
    const long long sl = v.stride[v.ndim - 1];
    const long long pieces = (L + kCopyPiece - 1) / kCopyPiece;
    const long long items = rows * pieces;
    for (long long w = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) / 32;
         w < items; w += warps) {
        const long long row = w / pieces;
        const long long j0 = (w - row * pieces) * kCopyPiece;
        const long long len = min(kCopyPiece, L - j0);
        const float* src = x + row_offset(v, row) + j0 * sl;
        float* dst = out + row * L + j0;
        if (VEC4) {
            // kCopyLoads 16-byte loads in flight per lane before their stores
            const float4* s4 = reinterpret_cast<const float4*>(src);
            float4* d4 = reinterpret_cast<float4*>(dst);
            const long long L4 = len / 4;
            long long j = lane;
            for (; j + 32 * (kCopyLoads - 1) < L4; j += 32 * kCopyLoads) {
                float4 t[kCopyLoads];
#pragma unroll
                for (int u = 0; u < kCopyLoads; ++u) t[u] = __ldcs(s4 + j + 32 * u);
#pragma unroll
                for (int u = 0; u < kCopyLoads; ++u) __stcs(d4 + j + 32 * u, t[u]);
            }
            for (; j < L4; j += 32) __stcs(d4 + j, __ldcs(s4 + j));
        } else {
            // four loads in flight per lane before their stores
            long long j = lane;
            for (; j + 96 < len; j += 128) {
                const float a = src[j * sl], b = src[(j + 32) * sl];
                const float c = src[(j + 64) * sl], d = src[(j + 96) * sl];
                dst[j] = a;
                dst[j + 32] = b;
                dst[j + 64] = c;
                dst[j + 96] = d;
            }
            for (; j < len; j += 32) dst[j] = src[j * sl];
        }
    }
}

// Short rows (L < 32): one thread per output row.
__global__ void __launch_bounds__(256) copy_short_rows_kernel(const float* __restrict__ x,
                                                              float* __restrict__ out,
                                                              CopyView v, long long rows) {
    const long long step = static_cast<long long>(gridDim.x) * blockDim.x;
    const long long L = v.shape[v.ndim - 1];
    const long long sl = v.stride[v.ndim - 1];
    for (long long row = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
         row < rows; row += step) {
        const float* src = x + row_offset(v, row);
        float* dst = out + row * L;
        for (long long j = 0; j < L; ++j) dst[j] = src[j * sl];
    }
}

// Transposed / permuted views: dim p (< ndim-1) has input stride 1. The output is walked in
// 64 x 64 tiles of (p, innermost) per batch entry, where the batch runs over every other dim.
// A tile is read along p (coalesced input) into shared memory and written along the innermost
// dim (coalesced output). 256 threads; each issues its 16 loads of a tile before storing any,
// so an SM keeps ~64 KB of reads in flight (a 32 x 32 tile with 4 loads per thread left the
// kernel at ~40% of HBM bandwidth, latency-bound).
constexpr int kCopyTile = 64;

__global__ void __launch_bounds__(256) copy_transpose_kernel(const float* __restrict__ x,
                                                             float* __restrict__ out,
                                                             CopyView v, int p,
                                                             long long batch) {
    __shared__ float tile[kCopyTile][kCopyTile + 1];  // [j - j0][i - i0]
    const int n = v.ndim;
    const long long L = v.shape[n - 1];
    const long long P = v.shape[p];
    const long long sl = v.stride[n - 1];
    // output stride of dim p: the product of the sizes after it
    long long op = 1;
    for (int d = p + 1; d < n; ++d) op *= v.shape[d];
    const long long tiles_j = (L + kCopyTile - 1) / kCopyTile;
    const long long tiles_i = (P + kCopyTile - 1) / kCopyTile;
    const long long per_batch = tiles_i * tiles_j;
    const long long total = per_batch * batch;
    const int tx = threadIdx.x % 32, ty = threadIdx.x / 32;
    for (long long t = blockIdx.x; t < total; t += gridDim.x) {
        const long long b = t / per_batch;
        const long long r = t - b * per_batch;
        const long long ti = r / tiles_j;
        const long long i0 = ti * kCopyTile;
        const long long j0 = (r - ti * tiles_j) * kCopyTile;
        // batch coordinates: every dim except p and the innermost, innermost-first
        long long in_off = 0, out_off = 0, rem = b, ostride = L;
        for (int d = n - 2; d >= 0; --d) {
            if (d == p) {
                ostride *= v.shape[d];
                continue;
            }
            const long long s = v.shape[d];
            const long long q = rem / s;
            const long long c = rem - q * s;
            in_off += c * v.stride[d];
            out_off += c * ostride;
            ostride *= s;
            rem = q;
        }
        const bool full = i0 + kCopyTile <= P && j0 + kCopyTile <= L;
        float vals[8][2];
        const float* src = x + in_off + i0 + tx + (j0 + ty) * sl;
        if (full) {
#pragma unroll
            for (int jj = 0; jj < 8; ++jj) {
#pragma unroll
                for (int ii = 0; ii < 2; ++ii) vals[jj][ii] = __ldcs(src + 32 * ii + 8 * jj * sl);
            }
        } else {
#pragma unroll
            for (int jj = 0; jj < 8; ++jj) {
#pragma unroll
                for (int ii = 0; ii < 2; ++ii) {
                    const long long i = i0 + tx + 32 * ii, j = j0 + ty + 8 * jj;
                    vals[jj][ii] = (i < P && j < L) ? __ldcs(src + 32 * ii + 8 * jj * sl) : 0.0f;
                }
            }
        }
        __syncthreads();  // the previous tile's reads of `tile` are done
#pragma unroll
        for (int jj = 0; jj < 8; ++jj) {
#pragma unroll
            for (int ii = 0; ii < 2; ++ii) tile[ty + 8 * jj][tx + 32 * ii] = vals[jj][ii];
        }
        __syncthreads();
        float* dst = out + out_off + (i0 + ty) * op + j0 + tx;
        if (full) {
#pragma unroll
            for (int ii = 0; ii < 8; ++ii) {
#pragma unroll
                for (int jj = 0; jj < 2; ++jj) {
                    __stcs(dst + 8 * ii * op + 32 * jj, tile[tx + 32 * jj][ty + 8 * ii]);
                }
            }
        } else {
#pragma unroll
            for (int ii = 0; ii < 8; ++ii) {
#pragma unroll
                for (int jj = 0; jj < 2; ++jj) {
                    const long long i = i0 + ty + 8 * ii, j = j0 + tx + 32 * jj;
                    if (i < P && j < L) dst[8 * ii * op + 32 * jj] = tile[tx + 32 * jj][ty + 8 * ii];
                }
            }
        }
    }
}

}  // namespace mfk
