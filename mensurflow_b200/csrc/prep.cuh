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

// The transposing pass for an operand whose rows run along memory (op(X)(r, p) with |rs| < |cs|,
// e.g. B [K, N] row-major read as N rows of K): 64 x 64 tiles of (r, p), one per block where the
// grid allows. Each thread issues its 16 loads of a tile (coalesced along r) before it stores
// any, the tile is turned through shared memory, and the rows of hi / lo are written along p
// (coalesced). Tiles are numbered over [batch][R / 64][Kp / 64]; the columns K..Kp-1 are written
// as zeros. On the transposed 1024 x 4096 and 4096 x 1024 weights of C3 and the 8192 x 32768 B of
// C5 this replaces 32 x 32 tiles with four loads per thread, which left a pass latency-bound.
constexpr int kPackTile = 64;

__global__ void __launch_bounds__(256) pack_transpose_kernel(
    const float* __restrict__ x, const long long* __restrict__ offsets, long long bstride,
    long long rs, long long cs, int R, int K, int Kp, int batch, float* __restrict__ hi,
    float* __restrict__ lo, int mode, unsigned* inf_word, unsigned inf_tag) {
    __shared__ float tile[kPackTile][kPackTile + 1];  // [p - p0][r - r0]
    const long long tiles_r = (R + kPackTile - 1) / kPackTile;
    const long long tiles_p = (Kp + kPackTile - 1) / kPackTile;
    const long long per_batch = tiles_r * tiles_p;
    const long long total = per_batch * batch;
    const int tx = threadIdx.x % 32, ty = threadIdx.x / 32;
    bool inf = false;  // this thread has met an infinity
    for (long long t = blockIdx.x; t < total; t += gridDim.x) {
        const long long b = t / per_batch;
        const long long rem = t - b * per_batch;
        const long long tr = rem / tiles_p;
        const int r0 = static_cast<int>(tr * kPackTile);
        const int p0 = static_cast<int>((rem - tr * tiles_p) * kPackTile);
        const float* xb = x + (offsets ? offsets[b] : b * bstride);
        float vals[8][2];
#pragma unroll
        for (int jj = 0; jj < 8; ++jj) {
#pragma unroll
            for (int ii = 0; ii < 2; ++ii) {
                const int r = r0 + tx + 32 * ii, p = p0 + ty + 8 * jj;
                vals[jj][ii] = (r < R && p < K)
                                   ? __ldcs(xb + static_cast<long long>(r) * rs +
                                            static_cast<long long>(p) * cs)
                                   : 0.0f;
            }
        }
        __syncthreads();  // the previous tile's reads of `tile` are done
#pragma unroll
        for (int jj = 0; jj < 8; ++jj) {
#pragma unroll
            for (int ii = 0; ii < 2; ++ii) tile[ty + 8 * jj][tx + 32 * ii] = vals[jj][ii];
        }
        __syncthreads();
        const long long out_base = b * R * static_cast<long long>(Kp);
#pragma unroll
        for (int ii = 0; ii < 8; ++ii) {
#pragma unroll
            for (int jj = 0; jj < 2; ++jj) {
                const int r = r0 + ty + 8 * ii, p = p0 + tx + 32 * jj;
                if (r < R && p < Kp) {
                    const float v = tile[tx + 32 * jj][ty + 8 * ii];
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
                        inf |= fabsf(v) == __int_as_float(0x7f800000);
                    }
                }
            }
        }
    }
    if (inf && inf_word != nullptr) *inf_word = inf_tag;
}

// The same pass for an operand that is already K-major with 16-byte aligned rows and K % 4 == 0
// (the common case: A row-major, or B read transposed): no transpose needed, so each float4 goes
// straight through, coalesced on both sides. One warp per output row (grid-stride over the
// batch x R rows; the row's source found with one division), lanes along the row's Kp/4 float4s
// with kPackLoads 16-byte loads in flight per lane. Launched with one row per warp where the
// grid allows, so the block scheduler balances the rows: on C2's B (8192 x 8192, split) 136 us
// against 165 us for two rows per warp on a grid of 8 blocks per SM (one B200).
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

constexpr int kPackThreads = 256;
constexpr int kPackLoads = 4;

__global__ void __launch_bounds__(kPackThreads, 4) pack_kmajor_vec4_kernel(
    const float* __restrict__ x, const long long* __restrict__ offsets, long long bstride,
    long long rs, int R, int K, int Kp, int batch, float* __restrict__ hi,
    float* __restrict__ lo, int mode, unsigned* inf_word, unsigned inf_tag) {
    const int lane = threadIdx.x % 32;
    const int per_row = Kp / 4;
    const long long rows = static_cast<long long>(batch) * R;
    const long long nwarps = static_cast<long long>(gridDim.x) * (kPackThreads / 32);
    const float4 zero = make_float4(0.f, 0.f, 0.f, 0.f);
    bool inf = false;  // this thread has met an infinity
    for (long long row = (static_cast<long long>(blockIdx.x) * kPackThreads + threadIdx.x) / 32;
         row < rows; row += nwarps) {
        const long long b = row / R;
        const float* s = x + (offsets ? offsets[b] : b * bstride) + (row - b * R) * rs;
        const long long out = row * per_row;
        int j = lane;
        for (; j + 32 * (kPackLoads - 1) < per_row; j += 32 * kPackLoads) {
            float4 v[kPackLoads];
#pragma unroll
            for (int u = 0; u < kPackLoads; ++u) {
                const int p = 4 * (j + 32 * u);
                v[u] = p < K ? __ldcs(reinterpret_cast<const float4*>(s + p)) : zero;
            }
#pragma unroll
            for (int u = 0; u < kPackLoads; ++u) {
                pack_store4(hi, lo, out + j + 32 * u, v[u], mode);
                inf |= any_inf(v[u]);
            }
        }
        for (; j < per_row; j += 32) {
            const int p = 4 * j;
            const float4 v = p < K ? __ldcs(reinterpret_cast<const float4*>(s + p)) : zero;
            pack_store4(hi, lo, out + j, v, mode);
            inf |= any_inf(v);
        }
    }
    if (inf && inf_word != nullptr) *inf_word = inf_tag;
}

}  // namespace mfk
