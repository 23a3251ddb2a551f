// Operand staging for the tensor-core GEMM: gathers a strided fp32 operand into the K-major,
// 16-byte-aligned, K-padded layout that TMA tiles need, and (3xTF32) splits it into a
// tf32 (hi, lo) pair on the way.
//
// The reference reads any strided view in place inside its packing step
// (src/backends/cpu/ops/gemm/gemm_pack.hpp, pack_a/pack_b); this is the GPU counterpart: one
// pass over the operand, coalesced on both sides through a 32x32 shared-memory tile, so a
// transposed view, a sliced view or a broadcast batch never goes through the host.
#pragma once

#include <cstdint>

namespace mfk {

enum PackMode : int {
    kPackCopy = 0,   // hi = x
    kPackRound = 1,  // hi = round_tf32(x)
    kPackSplit = 2,  // split_tf32: hi = x truncated to tf32, lo = tf32(x - hi)
};

// op(X) of matrix b: element (r, p) at x[off(b) + r*rs + p*cs], with off(b) = offsets[b] when
// offsets is non-null, else b*bstride. Writes hi/lo as [batch, R, Kp] row-major (row stride
// Kp), zero in the padding columns K..Kp-1. In kPackSplit mode an infinite element sets
// *inf_word = inf_tag (when inf_word is non-null), for the GEMM's fix-up of inf * 0 terms.
__global__ void __launch_bounds__(256) pack_kmajor_kernel(
    const float* __restrict__ x, const long long* __restrict__ offsets, long long bstride,
    long long rs, long long cs, int R, int K, int Kp, float* __restrict__ hi,
    float* __restrict__ lo, int mode, int p_contig, unsigned* inf_word, unsigned inf_tag) {
    __shared__ float tile[32][33];
    const int b = blockIdx.z;
    const int r0 = blockIdx.y * 32;
    const int p0 = blockIdx.x * 32;
    const long long base = offsets ? offsets[b] : static_cast<long long>(b) * bstride;
    const float* xb = x + base;
    const int tx = threadIdx.x, ty = threadIdx.y;
    if (p_contig) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int r = r0 + ty + 8 * i, p = p0 + tx;
            tile[ty + 8 * i][tx] =
                (r < R && p < K) ? xb[static_cast<long long>(r) * rs + static_cast<long long>(p) * cs]
                                 : 0.0f;
        }
    } else {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int p = p0 + ty + 8 * i, r = r0 + tx;
            tile[tx][ty + 8 * i] =
                (r < R && p < K) ? xb[static_cast<long long>(r) * rs + static_cast<long long>(p) * cs]
                                 : 0.0f;
        }
    }
    __syncthreads();
    const long long out_base = static_cast<long long>(b) * R * Kp;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int r = r0 + ty + 8 * i, p = p0 + tx;
        if (r < R && p < Kp) {
            const float v = tile[ty + 8 * i][tx];
            const long long o = out_base + static_cast<long long>(r) * Kp + p;
            if (mode == kPackCopy) {
                hi[o] = v;
            } else if (mode == kPackRound) {
                hi[o] = round_tf32(v);
            } else {
                float h, l;
                split_tf32(v, h, l);
                hi[o] = h;
                lo[o] = l;
                if (inf_word != nullptr && fabsf(v) == __int_as_float(0x7f800000)) *inf_word = inf_tag;
            }
        }
    }
}

// The same pass for an operand that is already K-major with 16-byte aligned rows and K % 4 == 0
// (the common case: A row-major, or B read transposed): no transpose needed, so each float4 goes
// straight through, coalesced on both sides. One warp per output row (grid-stride over the
// batch x R rows; the row's source found with one division), lanes along the row's Kp/4 float4s,
// two rows in flight per warp.
__device__ __forceinline__ void pack_store4(float* hi, float* lo, long long i, float4 v, int mode) {
    float4* h4 = reinterpret_cast<float4*>(hi) + i;
    if (mode == kPackCopy) {
        *h4 = v;
    } else if (mode == kPackRound) {
        *h4 = make_float4(round_tf32(v.x), round_tf32(v.y), round_tf32(v.z), round_tf32(v.w));
    } else {
        float4 h, l;
        split_tf32(v.x, h.x, l.x);
        split_tf32(v.y, h.y, l.y);
        split_tf32(v.z, h.z, l.z);
        split_tf32(v.w, h.w, l.w);
        *h4 = h;
        reinterpret_cast<float4*>(lo)[i] = l;
    }
}

__global__ void __launch_bounds__(256) pack_kmajor_vec4_kernel(
    const float* __restrict__ x, const long long* __restrict__ offsets, long long bstride,
    long long rs, int R, int K, int Kp, int batch, float* __restrict__ hi,
    float* __restrict__ lo, int mode, unsigned* inf_word, unsigned inf_tag) {
    const int lane = threadIdx.x % 32;
    const int per_row = Kp / 4;
    const long long rows = static_cast<long long>(batch) * R;
    const long long nwarps = static_cast<long long>(gridDim.x) * (blockDim.x / 32);
    auto source = [&](long long row) {
        const long long b = row / R;
        const long long r = row - b * R;
        return x + (offsets ? offsets[b] : b * bstride) + r * rs;
    };
    for (long long row0 = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) / 32;
         row0 < rows; row0 += 2 * nwarps) {
        const long long row1 = row0 + nwarps;
        const float* s0 = source(row0);
        const float* s1 = row1 < rows ? source(row1) : nullptr;
#pragma unroll 4
        for (int j = lane; j < per_row; j += 32) {
            const int p = 4 * j;
            const float4 zero = make_float4(0.f, 0.f, 0.f, 0.f);
            const float4 v0 = p < K ? __ldcs(reinterpret_cast<const float4*>(s0 + p)) : zero;
            const float4 v1 =
                (s1 != nullptr && p < K) ? __ldcs(reinterpret_cast<const float4*>(s1 + p)) : zero;
            pack_store4(hi, lo, row0 * per_row + j, v0, mode);
            if (s1 != nullptr) pack_store4(hi, lo, row1 * per_row + j, v1, mode);
            if (inf_word != nullptr && (any_inf(v0) || any_inf(v1))) *inf_word = inf_tag;
        }
    }
}

}  // namespace mfk
