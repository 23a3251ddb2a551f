// Fused scaled-dot-product attention on tcgen05 for fp32 data (3xTF32 throughout):
//   O = softmax(scale * Q K^T, over keys; causal: key <= query) V
// per head, with Q, K, V, O [heads, L, 128] (head dimension 128). One kernel: the scores never
// leave the SM, and with the causal mask the key tiles above the diagonal are never visited.
//
// Replaces, for the causal / unmasked case with head dimension 128, the reference's composition
// (src/ops/attention.cpp:48-98: gemm_strided_batched for S, where(-inf) for the mask, softmax,
// gemm_strided_batched for P V), which writes and re-reads the whole [L, L] score matrix of every
// head. Softmax follows the reference's numerics where it matters (the row maximum is that of
// fl(scale * QK), the row's exponentials are normalised by their sum;
// src/backends/cpu/ops/softmax/softmax.cpp:11-80) but is evaluated online: running row maximum m
// and sum l per key tile, O rescaled when m grows (only when it grows by more than 8, so the
// rescaling is rare and every exponential stays below e^8), O / l at the end.
//
// Design (sm_100a), one CTA pair (cta_group::2) per work unit = (head, block of 256 queries):
//  * Q of the unit (each CTA its 128 rows) is loaded raw by TMA into shared memory and split in
//    place into tf32 (hi, lo) by two converter warps; it stays there for all of the unit's key
//    tiles (the A operand of S = Q K^T);
//  * K and V stream through a ring of shared-memory stages by TMA, 32-wide chunks of the
//    contraction per stage: four K chunks (32 head dimensions of 64 keys per CTA) for S_j, four
//    V chunks (32 keys of 64 head dimensions per CTA) for the product with P_j. Both arrive raw,
//    as they lie in memory, and the converter warps split each stage in place. K is read
//    K-major; V, whose rows are keys (the contraction of O = P V), is read MN-major in the
//    128-byte swizzle on 32-byte atoms, so no pass transposes or splits it beforehand;
//  * tensor memory (512 columns): O [0, 128), two S buffers [128, 256) and [256, 384), P lo
//    [384, 512). The softmax warps overwrite S_j with P_j's hi part and write its lo part beside
//    it; the MMA then reads P from tensor memory as its A operand;
//  * the MMA issuer (one thread) runs S_0, S_1, PV_0, S_2, PV_1, ...: while the softmax warps
//    work on S_j the tensor cores compute S_{j+1} and PV_{j-1};
//  * eight softmax warps per CTA, two per query row (one per half of the columns), two passes
//    over each S tile (row maximum, swapped with the other half's through shared memory, then
//    exponentials, their sum and the split, the scores held in registers between them), the
//    epilogue O / l written straight from registers.
#pragma once

#include "mfk_ptx.cuh"

namespace mfk {

constexpr int kAttnD = 128;        // head dimension
constexpr int kAttnRows = 128;     // query rows per CTA (TMEM lanes)
constexpr int kAttnUnitRows = 256; // query rows per CTA pair
constexpr int kAttnKeys = 128;     // keys per key tile
constexpr int kAttnChunk = 32;     // contraction per ring stage (one 128-byte swizzle row)
constexpr int kAttnStages = 5;
constexpr int kAttnThreads = 384;  // warp 0 TMA, 1 MMA, 2-3 split Q K V, 4-11 softmax + epilogue
constexpr int kAttnCvtWarp0 = 2;
constexpr int kAttnSoftWarp0 = 4;
constexpr float kAttnRescaleAbove = 8.0f;  // raise the running max only past m + 8

// Shared memory per CTA (offsets from the 1024-aligned base).
constexpr int kAttnQChunkBytes = kAttnRows * kAttnChunk * 4;            // 16 KB
constexpr int kAttnQBytes = kAttnQChunkBytes * (kAttnD / kAttnChunk);   // 64 KB (hi or lo)
constexpr int kAttnHalfBytes = (kAttnKeys / 2) * kAttnChunk * 4;        // 8 KB: 64 rows
constexpr int kAttnStageBytes = 2 * kAttnHalfBytes;                     // hi | lo
// A V stage's half: two MN-major blocks of 32 keys x 32 head dimensions (128-byte rows, one per
// key); the MMA reads them with the blocks kAttnVBlockBytes apart along the head dimension and
// the 4-key swizzle atoms 512 bytes apart along the keys.
constexpr int kAttnVBlockBytes = kAttnChunk * 32 * 4;                  // 4 KB
constexpr int kAttnVAtomBytes = 4 * 128;
static_assert(2 * kAttnVBlockBytes == kAttnHalfBytes, "attention: V stage layout");
constexpr int kAttnOffQLo = kAttnQBytes;
constexpr int kAttnOffRing = 2 * kAttnQBytes;
constexpr int kAttnOffSwap = kAttnOffRing + kAttnStages * kAttnStageBytes;
constexpr int kAttnOffBars = kAttnOffSwap + 2 * 8 * 32 * 4;           // swap slots [2][8][32]
constexpr int kAttnBarBytes = 320;
constexpr int kAttnSmemBytes = 1024 + kAttnOffBars + kAttnBarBytes;
static_assert(kAttnSmemBytes <= 232448, "attention: shared memory per CTA exceeded");

// tensor memory columns
constexpr uint32_t kAttnColO = 0;
constexpr uint32_t kAttnColS = 128;  // buffer b at 128 + 128 b
constexpr uint32_t kAttnColPLo = 384;

enum : unsigned int {
    kErrAttnProducer = 1u << 0,
    kErrAttnMma = 1u << 1,
    kErrAttnSoftmax = 1u << 2,
    kErrAttnConvert = 1u << 3,
};

struct AttnArgs {
    int heads;      // matrices (batch x heads)
    int len;        // L: queries = keys
    int num_qb;     // ceil(L / 256)
    int causal;
    float scale;
    long long num_units;  // heads * num_qb
    int raw_hi;           // the tensor cores truncate fp32 operands: raw Q and K serve as hi
    // MASK kernels: key k may be seen by query q of matrix b where keep[b*keep_bs + q*keep_rs +
    // k*keep_cs] != 0 (strides in bytes; 0 broadcasts), as the reference's where(mask, s, -inf)
    const uint8_t* keep;
    long long keep_bs, keep_rs, keep_cs;
};

// The keep bits of 64 keys from 16-byte loads: bit i set where byte i is nonzero.
__device__ __forceinline__ uint32_t attn_keep_bits16(uint4 x) {
    auto nib = [](uint32_t w) {
        const uint32_t m = __vcmpne4(w, 0u) & 0x01010101u;  // one bit per byte, at bit 8 i
        return (m | (m >> 7) | (m >> 14) | (m >> 21)) & 0xFu;
    };
    return nib(x.x) | (nib(x.y) << 4) | (nib(x.z) << 8) | (nib(x.w) << 12);
}

// Work unit u -> (head, query block): the longest units (last query blocks under the causal
// mask) first, so the persistent pairs finish together.
__device__ __forceinline__ void attn_unit(const AttnArgs& a, long long u, int& head, int& qb) {
    qb = a.num_qb - 1 - static_cast<int>(u / a.heads);
    head = static_cast<int>(u % a.heads);
}

// Key tiles a query block needs: up to its last query (causal) or all of them.
__device__ __forceinline__ int attn_tiles(const AttnArgs& a, int qb) {
    const int keys = a.causal ? min(a.len, (qb + 1) * kAttnUnitRows) : a.len;
    return (keys + kAttnKeys - 1) / kAttnKeys;
}

// ---- producer: Q per unit, then K_0, K_1, V_0, K_2, V_1, ..., V_J through the ring ----------
// Each CTA loads its own half of a stage, raw, into the stage's hi part (the converters write lo
// beside it) and counts the bytes on its own `landed` barrier: a K stage in one box of 64 keys x
// 32 head dimensions, a V stage in two boxes of 32 keys x 32 head dimensions.
__device__ __forceinline__ void attn_producer(const AttnArgs& a, const CUtensorMap* tmQ,
                                              const CUtensorMap* tmK, const CUtensorMap* tmV,
                                              uint8_t* smem, uint64_t* landed, uint64_t* empty,
                                              uint64_t* q_full, uint64_t* q_free, uint32_t rank) {
    const uint64_t keep = l2_policy_evict_last();
    int stage = 0;
    uint32_t phase = 0;
    long long n = 0;  // units of this pair so far
    // one box of m at (x, y, z), or two (x and x + 32) for a V stage
    auto load_stage = [&](const CUtensorMap* m, bool v, int x, int y, int z) {
        if (!mbar_wait(&empty[stage], phase ^ 1u, kErrAttnProducer)) return false;
        uint8_t* s = smem + kAttnOffRing + stage * kAttnStageBytes;
        mbar_arrive_expect_tx(&landed[stage], kAttnHalfBytes);
        tma_load_3d(s, m, &landed[stage], x, y, z, keep);
        if (v) tma_load_3d(s + kAttnVBlockBytes, m, &landed[stage], x + 32, y, z, keep);
        if (++stage == kAttnStages) {
            stage = 0;
            phase ^= 1u;
        }
        return true;
    };
    for (long long u = blockIdx.x / 2; u < a.num_units; u += gridDim.x / 2, ++n) {
        int head, qb;
        attn_unit(a, u, head, qb);
        const int tiles = attn_tiles(a, qb);
        // Q: after the previous unit's S products have read it
        if (n > 0 && !mbar_wait(q_free, static_cast<uint32_t>((n - 1) & 1), kErrAttnProducer))
            return;
        const int qrow = qb * kAttnUnitRows + static_cast<int>(rank) * kAttnRows;
        for (int kc = 0; kc < kAttnD / kAttnChunk; ++kc) {  // one barrier per 32-column chunk
            mbar_arrive_expect_tx(&q_full[kc], kAttnQChunkBytes);
            tma_load_3d(smem + kc * kAttnQChunkBytes, tmQ, &q_full[kc], kc * kAttnChunk, qrow,
                        head, keep);
        }
        const int krow = static_cast<int>(rank) * (kAttnKeys / 2);  // this CTA's keys of K_j
        const int vcol = static_cast<int>(rank) * (kAttnD / 2);     // its head dims of V_j
        for (int j = 0; j <= tiles; ++j) {
            if (j < tiles) {  // K_j (raw): 64 keys of the tile per CTA, four chunks of the head dim
                for (int kc = 0; kc < kAttnD / kAttnChunk; ++kc)
                    if (!load_stage(tmK, false, kc * kAttnChunk, j * kAttnKeys + krow, head))
                        return;
            }
            if (j >= 1) {  // V_{j-1}: 64 head dims per CTA, four chunks of keys
                for (int kc = 0; kc < kAttnKeys / kAttnChunk; ++kc)
                    if (!load_stage(tmV, true, vcol, (j - 1) * kAttnKeys + kc * kAttnChunk, head))
                        return;
            }
        }
    }
}

// ---- converters: Q, K and V raw -> (hi, lo) in shared memory, stage by stage --------------
// The two converter warps walk the ring in the producer's order. Every stage is split in place,
// element by element in whatever layout it landed in (lo written beside the raw values, at the
// same offset in the stage's lo half, so it shares their swizzle; the raw values are the hi
// part where the tensor cores truncate fp32, else hi is rewritten too); then both warps of both
// CTAs arrive on the stage's `ready` barrier in the first CTA, which the MMA issuer waits on. Q is split chunk by chunk, each chunk just before the stage of K_0 with the same head
// dimensions, so a unit's first S product can start after one chunk of each.
__device__ __forceinline__ void attn_split_vecs(float4* hi, float4* lo, int begin, int end,
                                                int ct, bool raw_hi) {
    if (raw_hi) {
#pragma unroll 4
        for (int i = begin + ct; i < end; i += 64) {
            const float4 x = hi[i];
            float4 h, l;  // h unused: the raw value is hi
            split_tf32(x.x, h.x, l.x);
            split_tf32(x.y, h.y, l.y);
            split_tf32(x.z, h.z, l.z);
            split_tf32(x.w, h.w, l.w);
            lo[i] = l;
        }
    } else {
#pragma unroll 4
        for (int i = begin + ct; i < end; i += 64) {
            const float4 x = hi[i];
            float4 h, l;
            split_tf32(x.x, h.x, l.x);
            split_tf32(x.y, h.y, l.y);
            split_tf32(x.z, h.z, l.z);
            split_tf32(x.w, h.w, l.w);
            hi[i] = h;
            lo[i] = l;
        }
    }
}

__device__ __forceinline__ void attn_convert(const AttnArgs& a, uint8_t* smem, uint64_t* q_full,
                                            uint64_t* q_ready, uint64_t* landed,
                                            uint64_t* ready) {
    const int ct = threadIdx.x - kAttnCvtWarp0 * 32;
    const int lane = threadIdx.x % 32;
    const bool raw_hi = a.raw_hi != 0;
    constexpr int kChunkVecs = kAttnQChunkBytes / 16;
    constexpr int kHalfVecs = kAttnHalfBytes / 16;
    int stage = 0;
    uint32_t phase = 0;
    // the next ring stage: split it, then release it to the MMA issuer
    auto pass_stage = [&]() {
        if (!mbar_wait(&landed[stage], phase, kErrAttnConvert)) return false;
        uint8_t* st = smem + kAttnOffRing + stage * kAttnStageBytes;
        attn_split_vecs(reinterpret_cast<float4*>(st),
                        reinterpret_cast<float4*>(st + kAttnHalfBytes), 0, kHalfVecs, ct, raw_hi);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(mapa_shared(&ready[stage], 0));
        if (++stage == kAttnStages) {
            stage = 0;
            phase ^= 1u;
        }
        return true;
    };
    long long n = 0;
    for (long long u = blockIdx.x / 2; u < a.num_units; u += gridDim.x / 2, ++n) {
        int head, qb;
        attn_unit(a, u, head, qb);
        const int tiles = attn_tiles(a, qb);
        for (int kc = 0; kc < kAttnD / kAttnChunk; ++kc) {
            if (!mbar_wait(&q_full[kc], static_cast<uint32_t>(n & 1), kErrAttnConvert)) return;
            attn_split_vecs(reinterpret_cast<float4*>(smem),
                            reinterpret_cast<float4*>(smem + kAttnOffQLo), kc * kChunkVecs,
                            (kc + 1) * kChunkVecs, ct, raw_hi);
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(mapa_shared(&q_ready[kc], 0));
            if (!pass_stage()) return;  // K_0, the same head dimensions
        }
        for (int j = 1; j <= tiles; ++j) {
            if (j < tiles) {
                for (int kc = 0; kc < kAttnD / kAttnChunk; ++kc)
                    if (!pass_stage()) return;  // K_j
            }
            for (int kc = 0; kc < kAttnKeys / kAttnChunk; ++kc)
                if (!pass_stage()) return;  // V_{j-1}
        }
    }
}

// ---- MMA issuer (one thread of the pair's first CTA) -----------------------------------------
__device__ __forceinline__ void attn_mma(const AttnArgs& a, uint32_t tmem, uint8_t* smem,
                                         uint64_t* ready, uint64_t* empty, uint64_t* q_ready,
                                         uint64_t* q_free, uint64_t* s_full, uint64_t* p_full,
                                         uint64_t* pv_done) {
    constexpr uint32_t idesc = idesc_tf32(kAttnUnitRows, 128, false, false);
    constexpr uint32_t idesc_pv = idesc_tf32(kAttnUnitRows, 128, false, true);  // V MN-major
    constexpr uint16_t kPair = 3;
    const uint32_t q_hi = smem_u32(smem);
    const uint32_t q_lo = q_hi + kAttnOffQLo;
    const uint32_t ring = q_hi + kAttnOffRing;
    int stage = 0;
    uint32_t phase = 0;
    long long t = 0;  // key tiles of this pair so far (S buffer t & 1)
    long long n = 0;
    auto next_stage = [&]() {
        if (++stage == kAttnStages) {
            stage = 0;
            phase ^= 1u;
        }
    };
    // S_t = Q K_j^T into S buffer t & 1. On the unit's first tile each chunk of Q is waited for
    // (q_ready[kc], phase `qphase`) just before its MMAs.
    auto s_product = [&](long long tt, bool first, uint32_t qphase) {
        const uint32_t d = tmem + kAttnColS + static_cast<uint32_t>((tt & 1) * 128);
        for (int kc = 0; kc < kAttnD / kAttnChunk; ++kc) {
            if (first && !mbar_wait(&q_ready[kc], qphase, kErrAttnMma)) return false;
            if (!mbar_wait(&ready[stage], phase, kErrAttnMma)) return false;
            tc_fence_after();
            const uint32_t bh = ring + stage * kAttnStageBytes;
            const uint32_t bl = bh + kAttnHalfBytes;
            const uint32_t ah = q_hi + kc * kAttnQChunkBytes;
            const uint32_t al = q_lo + kc * kAttnQChunkBytes;
#pragma unroll
            for (int ks = 0; ks < kAttnChunk / 8; ++ks) {
                const uint32_t koff = ks * 32;
                const uint64_t dah = smem_desc(ah + koff, 16, 1024, kSwizzle128B);
                const uint64_t dal = smem_desc(al + koff, 16, 1024, kSwizzle128B);
                const uint64_t dbh = smem_desc(bh + koff, 16, 1024, kSwizzle128B);
                const uint64_t dbl = smem_desc(bl + koff, 16, 1024, kSwizzle128B);
                // Q hi read once for its two products (A collector)
                mma_tf32_cg2_a_fill(d, dah, dbh, idesc, (kc > 0 || ks > 0) ? 1u : 0u);
                mma_tf32_cg2_a_lastuse(d, dah, dbl, idesc, 1u);
                mma_tf32_cg2(d, dal, dbh, idesc, 1u);
            }
            mma_commit_cg2_mc(&empty[stage], kPair);
            next_stage();
        }
        mma_commit_cg2_mc(&s_full[tt & 1], kPair);
        return true;
    };
    // O (+)= P_t V_j: P (hi in S buffer t & 1, lo in the P lo columns) from tensor memory, V
    // from the stage's MN-major blocks (8 keys per MMA = two 4-key swizzle atoms)
    auto pv_product = [&](long long tt, bool first) {
        if (!mbar_wait(&p_full[tt & 1], static_cast<uint32_t>((tt >> 1) & 1), kErrAttnMma))
            return false;
        tc_fence_after();
        const uint32_t ph = tmem + kAttnColS + static_cast<uint32_t>((tt & 1) * 128);
        const uint32_t pl = tmem + kAttnColPLo;
        for (int kc = 0; kc < kAttnKeys / kAttnChunk; ++kc) {
            if (!mbar_wait(&ready[stage], phase, kErrAttnMma)) return false;
            tc_fence_after();
            const uint32_t bh = ring + stage * kAttnStageBytes;
            const uint32_t bl = bh + kAttnHalfBytes;
#pragma unroll
            for (int ks = 0; ks < kAttnChunk / 8; ++ks) {
                const uint32_t koff = ks * 2 * kAttnVAtomBytes;
                const uint32_t col = static_cast<uint32_t>(kc * kAttnChunk + ks * 8);
                const uint64_t dbh = smem_desc(bh + koff, kAttnVBlockBytes, kAttnVAtomBytes,
                                               kSwizzle128BBase32B);
                const uint64_t dbl = smem_desc(bl + koff, kAttnVBlockBytes, kAttnVAtomBytes,
                                               kSwizzle128BBase32B);
                const uint32_t acc = (!first || kc > 0 || ks > 0) ? 1u : 0u;
                mma_tf32_ts_cg2(tmem + kAttnColO, pl + col, dbh, idesc_pv, acc);
                mma_tf32_ts_cg2(tmem + kAttnColO, ph + col, dbl, idesc_pv, 1u);
                mma_tf32_ts_cg2(tmem + kAttnColO, ph + col, dbh, idesc_pv, 1u);
            }
            mma_commit_cg2_mc(&empty[stage], kPair);
            next_stage();
        }
        mma_commit_cg2_mc(pv_done, kPair);
        return true;
    };
    for (long long u = blockIdx.x / 2; u < a.num_units; u += gridDim.x / 2, ++n) {
        int head, qb;
        attn_unit(a, u, head, qb);
        const int tiles = attn_tiles(a, qb);
        const long long t0 = t;
        for (int j = 0; j < tiles; ++j) {
            if (!s_product(t0 + j, j == 0, static_cast<uint32_t>(n & 1))) return;
            if (j == tiles - 1) mma_commit_cg2_mc(q_free, kPair);  // every S of the unit
            if (j >= 1 && !pv_product(t0 + j - 1, j == 1)) return;
        }
        if (!pv_product(t0 + tiles - 1, tiles == 1)) return;
        t = t0 + tiles;
    }
}

// ---- softmax and epilogue (eight warps per CTA: two per TMEM lane quarter) -----------------
// Warp w (4..11) owns query row 32 (w % 4) + lane of its CTA's block and half h = (w - 4) / 4 of
// the tile's 128 columns (keys, and later output columns); the other warp of its lane quarter
// owns the other half. A warp reads and writes only its own columns of S_j / P_j: the two halves'
// row maxima (per tile) and row sums (per unit) are swapped through shared memory.

// The two warps of a lane quarter swap one float per lane: event e writes slot e & 1 and waits
// for phase e of the quarter's barrier (both warps arrive). A slot is rewritten two events later,
// only after the partner has arrived for the event in between, i.e. after it read the value.
struct AttnSwap {
    float* xch;     // [2 slots][8 warps][32 lanes]
    uint64_t* bar;  // the lane quarter's barrier, two arrivals per event
    int me, partner, lane;
    long long e;
    __device__ __forceinline__ bool swap(float v, float& other) {
        float* slot = xch + (e & 1) * (8 * 32);
        slot[me * 32 + lane] = v;
        __threadfence_block();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar);
        if (!mbar_wait(bar, static_cast<uint32_t>(e & 1), kErrAttnSoftmax)) return false;
        other = slot[partner * 32 + lane];
        ++e;
        return true;
    }
};

// `kbits` has bit i set where key own0 + i of the tile is valid: in range, under the causal
// limit and, in MASK kernels, kept by the mask. (As a bitmask rather than a compare against the
// count of valid keys the pass compiles to 138 registers instead of 168 with spills: 1 % faster.)
template <bool MASK>
__device__ __forceinline__ bool attn_softmax_row_half(const AttnArgs& a, uint32_t sb,
                                                      uint32_t pl, int h, uint64_t kbits,
                                                      float& m, double& l,
                                                      bool rescale_allowed, uint32_t olanes,
                                                      uint64_t* pv_done, long long t, int j,
                                                      AttnSwap& sw) {
    const float ninf = __int_as_float(0xff800000);
    const int own0 = h * 64;
    // pass 1: the maximum of fl(scale * s) over this half's valid keys, the raw scores kept in
    // registers; then the row's maximum with the other half's. Rounding is monotonic, so for
    // scale >= 0 that maximum is fl(scale * max s), and for scale < 0 fl(scale * min s): one
    // multiply per row instead of one per score. Four independent chains.
    uint32_t sr[2][32];
    tmem_ld_issue_32x32b_x32(sb + own0, sr[0]);
    tmem_ld_issue_32x32b_x32(sb + own0 + 32, sr[1]);
    tmem_ld_wait();
    const float* s = reinterpret_cast<const float*>(&sr[0][0]);
    // no masked key in this half
    const bool full = __all_sync(0xffffffffu, kbits == ~0ull);
    auto valid = [&](int i) { return ((kbits >> i) & 1ull) != 0ull; };
    const bool neg = a.scale < 0.0f;
    const float pinf = __int_as_float(0x7f800000);
    float ext[4];
#pragma unroll
    for (int c = 0; c < 4; ++c) ext[c] = neg ? pinf : ninf;
    if (full && !neg) {
#pragma unroll
        for (int i = 0; i < 64; ++i) ext[i & 3] = fmaxf(ext[i & 3], s[i]);
    } else if (!neg) {
#pragma unroll
        for (int i = 0; i < 64; ++i)
            if (valid(i)) ext[i & 3] = fmaxf(ext[i & 3], s[i]);
    } else {
#pragma unroll
        for (int i = 0; i < 64; ++i)
            if (valid(i)) ext[i & 3] = fminf(ext[i & 3], s[i]);
    }
    const float e01 = neg ? fminf(ext[0], ext[1]) : fmaxf(ext[0], ext[1]);
    const float e23 = neg ? fminf(ext[2], ext[3]) : fmaxf(ext[2], ext[3]);
    const float ex = neg ? fminf(e01, e23) : fmaxf(e01, e23);
    float mt = kbits != 0ull ? __fmul_rn(a.scale, ex) : ninf;
    float mo;
    if (!sw.swap(mt, mo)) return false;
    mt = fmaxf(mt, mo);
    float mn = m;
    if (mt != ninf && (m == ninf || mt > m + kAttnRescaleAbove)) mn = fmaxf(m, mt);
    // the previous tile's product has finished: P lo is free and O holds it
    if (j >= 1) {
        if (!mbar_wait(pv_done, static_cast<uint32_t>((t - 1) & 1), kErrAttnSoftmax)) return false;
        tc_fence_after();
    }
    if (rescale_allowed && __any_sync(0xffffffffu, mn != m)) {
        const float f = mn != m ? expf(m - mn) : 1.0f;
#pragma unroll
        for (int c = 0; c < 64; c += 16) {
            uint32_t r[16];
            tmem_ld_issue_32x32b_x16(olanes + own0 + c, r);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 16; ++i) r[i] = __float_as_uint(__fmul_rn(__uint_as_float(r[i]), f));
            tmem_st_32x32b_x16(olanes + own0 + c, r);
        }
        l *= static_cast<double>(f);
    }
    m = mn;
    // pass 2: P = exp(scale s - m) on valid keys (0 elsewhere), split into tf32 (hi, lo); P >= 0
    // is finite, so the split needs no special cases: hi = P with its 13 low bits cleared, lo =
    // P - hi (exact) rounded to tf32. exp(scale s - m) = 2^(s fl(scale log2 e) - fl(m log2 e)),
    // the exponent from one FMA of the raw score (an absolute error of about
    // (|scale s| + |m|) 2^-23 in it, a relative one of 0.7 times that in P: below 1e-6 for
    // scores up to ~10)
    float lt[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    uint32_t* hb = &sr[0][0];  // P's hi part replaces the scores it came from
    const float ml = m * 1.44269504088896340736f;
    const float sl = a.scale * 1.44269504088896340736f;  // exponent of fl(scale s) - m: s sl - ml
#pragma unroll
    for (int c = 0; c < 64; c += 16) {
        uint32_t lo[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            const float e = exp2f(fmaf(s[c + i], sl, -ml));
            const float p = (full || valid(c + i)) ? e : 0.0f;
            lt[i & 3] += p;
            const uint32_t hi = __float_as_uint(p) & 0xFFFFE000u;
            lo[i] = tf32_round_bits(__float_as_uint(p - __uint_as_float(hi)));
            hb[c + i] = hi;
        }
        tmem_st_32x32b_x16(sb + own0 + c, *reinterpret_cast<const uint32_t(*)[16]>(hb + c));
        tmem_st_32x32b_x16(pl + own0 + c, lo);
    }
    l += static_cast<double>((lt[0] + lt[1]) + (lt[2] + lt[3]));
    return true;
}

template <bool MASK>
__device__ __forceinline__ void attn_softmax(const AttnArgs& a, float* out, uint32_t tmem,
                                             uint64_t* s_full, uint64_t* p_full,
                                             uint64_t* pv_done, uint64_t* x_bar, float* xch,
                                             uint32_t rank) {
    const int warp = threadIdx.x / 32;
    const int lane = threadIdx.x % 32;
    const int q = warp % 4;                       // TMEM lane quarter
    const int h = (warp - kAttnSoftWarp0) / 4;    // column half
    const uint32_t lanes = tmem + (static_cast<uint32_t>(q * 32) << 16);
    AttnSwap sw{xch, &x_bar[q], warp - kAttnSoftWarp0, warp - kAttnSoftWarp0 + (h ? -4 : 4),
                lane, 0};
    long long t = 0;
    long long n = 0;
    bool ok = true;  // a bounded wait gave up: leave every loop
    for (long long u = blockIdx.x / 2; ok && u < a.num_units; u += gridDim.x / 2, ++n) {
        int head, qb;
        attn_unit(a, u, head, qb);
        const int tiles = attn_tiles(a, qb);
        const int row0 = qb * kAttnUnitRows + static_cast<int>(rank) * kAttnRows + q * 32;
        const int row = row0 + lane;
        // keys valid for this row: key < L, and key <= row under the causal mask
        const int kend = a.causal ? min(a.len, row + 1) : a.len;
        float m = __int_as_float(0xff800000);
        double l = 0.0;
        for (int j = 0; j < tiles; ++j, ++t) {
            const uint32_t sb = lanes + kAttnColS + static_cast<uint32_t>((t & 1) * 128);
            // MASK: this row's keep bits for the half's 64 keys in range, loaded before the
            // scores are waited for
            uint64_t kbits = 0ull;
            if constexpr (!MASK) {
                const int nk = max(0, min(64, kend - (j * kAttnKeys + h * 64)));
                kbits = nk >= 64 ? ~0ull : ((1ull << nk) - 1ull);
            } else {
                const int key0 = j * kAttnKeys + h * 64;
                const int nk = max(0, min(64, kend - key0));
                if (row < a.len && nk > 0) {
                    const uint8_t* mrow = a.keep + static_cast<long long>(head) * a.keep_bs +
                                          static_cast<long long>(row) * a.keep_rs +
                                          static_cast<long long>(key0) * a.keep_cs;
                    if (nk == 64 && a.keep_cs == 1 &&
                        (reinterpret_cast<uintptr_t>(mrow) & 15u) == 0u) {
                        const uint4* p4 = reinterpret_cast<const uint4*>(mrow);
#pragma unroll
                        for (int w = 0; w < 4; ++w)
                            kbits |= static_cast<uint64_t>(attn_keep_bits16(__ldg(p4 + w)))
                                     << (16 * w);
                    } else {
                        for (int i = 0; i < nk; ++i)
                            kbits |= static_cast<uint64_t>(
                                         __ldg(mrow + static_cast<long long>(i) * a.keep_cs) != 0)
                                     << i;
                    }
                }
            }
            if (!mbar_wait(&s_full[t & 1], static_cast<uint32_t>((t >> 1) & 1), kErrAttnSoftmax)) {
                ok = false;
                break;
            }
            tc_fence_after();
            if (!attn_softmax_row_half<MASK>(a, sb, lanes + kAttnColPLo, h, kbits, m, l, j >= 1,
                                             lanes + kAttnColO, pv_done, t, j, sw)) {
                ok = false;
                break;
            }
            tmem_st_wait();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(mapa_shared(&p_full[t & 1], 0));
        }
        if (!ok) break;
        // the row sum: this half's plus the other warp's
        float lo_half;
        if (!sw.swap(static_cast<float>(l), lo_half)) break;
        l += static_cast<double>(lo_half);
        // epilogue: O / l once the last product has finished
        if (!mbar_wait(pv_done, static_cast<uint32_t>((t - 1) & 1), kErrAttnSoftmax)) break;
        tc_fence_after();
        // a row whose every key is masked out: zeros, as the reference's softmax gives
        const float inv = (MASK && l == 0.0) ? 0.0f : static_cast<float>(1.0 / l);
        float* orow = out + (static_cast<long long>(head) * a.len + row) * kAttnD + h * 64;
#pragma unroll
        for (int c = 0; c < 64; c += 32) {
            uint32_t r[32];
            tmem_ld_issue_32x32b_x32(lanes + kAttnColO + h * 64 + c, r);
            tmem_ld_wait();
            if (row < a.len) {
#pragma unroll
                for (int v = 0; v < 8; ++v) {
                    reinterpret_cast<float4*>(orow + c)[v] =
                        make_float4(__fmul_rn(__uint_as_float(r[4 * v]), inv),
                                    __fmul_rn(__uint_as_float(r[4 * v + 1]), inv),
                                    __fmul_rn(__uint_as_float(r[4 * v + 2]), inv),
                                    __fmul_rn(__uint_as_float(r[4 * v + 3]), inv));
                }
            }
        }
        // the epilogue's reads of O are done before the next unit's first product overwrites it:
        // the next p_full arrival comes after them (tcgen05.wait::ld above)
    }
}

template <bool MASK>
__global__ void __launch_bounds__(kAttnThreads, 1)
    attn_tc_kernel(const __grid_constant__ CUtensorMap tmQ,
                   const __grid_constant__ CUtensorMap tmK,
                   const __grid_constant__ CUtensorMap tmV, float* out, const AttnArgs a) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kAttnOffBars);
    uint64_t* landed = bars;                  // [stages]: this CTA's half of the stage arrived
    uint64_t* ready = landed + kAttnStages;   // [stages]: both halves split, for the MMA issuer
    uint64_t* empty = ready + kAttnStages;
    uint64_t* q_full = empty + kAttnStages;  // [4]: per 32-column chunk of Q
    uint64_t* q_ready = q_full + 4;          // [4]
    uint64_t* q_free = q_ready + 4;
    uint64_t* s_full = q_free + 1;   // [2]
    uint64_t* p_full = s_full + 2;   // [2]
    uint64_t* pv_done = p_full + 2;
    uint64_t* drain = pv_done + 1;
    uint64_t* x_bar = drain + 1;     // [4]: the two warps of a lane quarter
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(x_bar + 4);
    float* xch = reinterpret_cast<float*>(smem + kAttnOffSwap);
    static_assert((3 * kAttnStages + 20) * 8 + 4 <= kAttnBarBytes,
                  "attention: barrier area too small");

    const int warp = threadIdx.x / 32;
    const int lane = threadIdx.x % 32;
    const uint32_t rank = cluster_ctarank();
    if (threadIdx.x == 0) {
        for (int s = 0; s < kAttnStages; ++s) {
            mbar_init(&landed[s], 1);
            mbar_init(&ready[s], 2 * 2);  // both converter warps of both CTAs
            mbar_init(&empty[s], 1);
        }
        for (int c = 0; c < 4; ++c) {
            mbar_init(&q_full[c], 1);
            mbar_init(&q_ready[c], 2 * 2);  // both converter warps of both CTAs
        }
        mbar_init(q_free, 1);
        for (int b = 0; b < 2; ++b) {
            mbar_init(&s_full[b], 1);
            mbar_init(&p_full[b], 8 * 2);  // the eight softmax warps of both CTAs
        }
        mbar_init(pv_done, 1);
        mbar_init(drain, 1);
        for (int i = 0; i < 4; ++i) mbar_init(&x_bar[i], 2);
        fence_barrier_init();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&tmQ);
        tma_prefetch_desc(&tmK);
        tma_prefetch_desc(&tmV);
    }
    if (warp == 1) tmem_alloc_cg2(tmem_holder, 512);
    tc_fence_before();
    __syncthreads();
    cluster_sync();
    tc_fence_after();
    const uint32_t tmem = *tmem_holder;

    if (warp == 0) {
        if (lane == 0)
            attn_producer(a, &tmQ, &tmK, &tmV, smem, landed, empty, q_full, q_free, rank);
    } else if (warp == 1) {
        if (lane == 0 && rank == 0) {
            attn_mma(a, tmem, smem, ready, empty, q_ready, q_free, s_full, p_full, pv_done);
            // every MMA issued must finish before tensor memory is released
            mma_commit_cg2(drain);
            mbar_wait(drain, 0, kErrAttnMma);
        }
        __syncwarp();
    } else if (warp < kAttnSoftWarp0) {
        attn_convert(a, smem, q_full, q_ready, landed, ready);
    } else {
        attn_softmax<MASK>(a, out, tmem, s_full, p_full, pv_done, x_bar, xch, rank);
    }

    tc_fence_before();
    __syncthreads();
    cluster_sync();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc_cg2(tmem, 512);
    }
}

}  // namespace mfk
