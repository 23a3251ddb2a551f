// The tcgen05 tensor-core GEMM for fp32 data: C = act(alpha * op(A) op(B) + beta * C_in + bias).
//
// Replaces the reference's CPU packed GEMM (src/backends/cpu/ops/gemm/gemm_packed.cpp:1505
// gemm_parallel, :313 kernel_6x16) plus the alpha/beta/bias/activation passes that follow it
// (src/ops/blas.cpp:246-260, gemm_batched.cpp:12-28 finish_matrix, elementwise.cpp:128 bias_add).
//
// Design (sm_100a):
//  * persistent: one CTA (CG = 1) or one CTA pair (CG = 2, a 2-CTA cluster on neighbouring SMs)
//    per output tile of (128*CG) x BN, walking tiles in a grouped raster order so the A and B
//    panels in flight stay in L2;
//  * warp-specialised, 384 threads per CTA: warp 0 issues TMA loads into an mbarrier ring of
//    STAGES shared-memory stages; warp 1 owns TMEM and one lane of the pair's first CTA issues
//    tcgen05.mma; warps 2-3 split A in shared memory (ASPLIT kernels); warps 4-11 are the
//    epilogue (TMEM -> registers -> alpha/beta/bias/activation -> shared box -> TMA store);
//  * ATMEM kernels (3xTF32, N <= 128, A read in place), 512 threads: A arrives raw and two
//    groups of four converter warps (warps 4-7 and 12-15, alternate k-blocks) write its
//    (hi, lo) split into a ring of TMEM slots that the MMA reads as its A operand (tcgen05.mma
//    with A in tensor memory), so shared memory holds only raw A and B; warps 8-11 are the
//    epilogue;
//  * operands are K-major fp32 tiles of 32 elements (128 B) per row, SWIZZLE_128B, read by the
//    MMA through shared-memory descriptors; kind::tf32 with an fp32 accumulator in TMEM;
//  * CG = 2 (cta_group::2): each CTA of the pair loads its 128 rows of A and its BN/2 rows of B
//    into its own shared memory (plain TMA loads, completion counted on the first CTA's
//    barrier); one MMA of M = 256 reads both halves, so a CTA reads half the operand bytes per
//    flop from shared memory and from L2 that a 1-CTA MMA would;
//  * 3xTF32 (SPLIT3): each operand arrives as a (hi, lo) pair with hi = tf32(x), lo = tf32(x-hi)
//    and three MMAs per k-step accumulate lo*hi + hi*lo + hi*hi (Ootomo & Yokota 2022; the
//    split-precision "3xTF32" scheme); 1xTF32 issues one MMA per k-step;
//  * two TMEM accumulators, so the epilogue of tile i overlaps the main loop of tile i+1.
#pragma once

#include "mfk_ptx.cuh"

namespace mfk {

constexpr int kBM = 128;          // rows of A per CTA = TMEM lanes
constexpr int kBK = 32;           // fp32 depth per stage: one 128-byte swizzle row
constexpr int kGemmThreads = 384;
constexpr int kEpiWarp0 = 4;      // warps 4..11 are the epilogue (two warpgroups)
constexpr int kEpiWarps = 8;
constexpr int kEpiCols = 16;      // columns per epilogue chunk (one TMEM load, one store box)
constexpr int kCvtWarp0 = 2;      // warps 2..3 split A in shared memory (ASPLIT kernels)
constexpr int kCvtThreads = 64;
// ATMEM kernels (A split into tensor memory), 512 threads: warps 4..7 and 12..15 convert (two
// groups of one warp per TMEM lane quarter, taking alternate k-blocks), warps 8..11 are the
// epilogue.
constexpr int kTmCvtWarp0 = 4;
constexpr int kTmCvtWarp1 = 12;
constexpr int kTmEpiWarp0 = 8;
constexpr int kTmThreads = 512;

enum : unsigned int {
    kErrProducerWait = 1u << 0,
    kErrMmaWait = 1u << 1,
    kErrEpilogueWait = 1u << 2,
    kErrConvertWait = 1u << 3,
};

enum Activation : int { kActNone = 0, kActRelu = 1, kActGelu = 2, kActGeluTanh = 3 };

struct GemmArgs {
    int m, n, k;
    int num_kb;        // ceil(k / kBK)
    int batch;
    int tiles_m, tiles_n;
    int group_m;       // M-tiles per raster group
    long long num_tiles;
    int a_batch_bcast; // 1: every matrix uses A's matrix 0
    int b_batch_bcast;
    float alpha, beta;
    const float* c_in;
    long long c_in_rs, c_in_cs, c_in_bs;
    float* c;
    long long ldc, c_bs;
    const float* bias;
    int act;
    int tma_store;     // 1: C is written by TMA stores through shared memory (tmC is valid)
    int raw_hi;        // ASPLIT: the MMA reads raw A as hi (truncating), write only lo
    int c_peer;        // C lies in another GPU's memory: the epilogue's stores cross NVLink
    // Stream-K tail (sk_units > 0): tiles [0, dp_tiles) go whole to the units in turn; the
    // k-iterations of tiles [dp_tiles, num_tiles) are split evenly over all sk_units units
    // (unit u: sk_q + 1 iterations if u < sk_r, else sk_q). Every part of a split tile but the
    // first writes its raw accumulator to its unit's slot 0 of sk_part and counts itself in
    // sk_count. The unit holding the first k-blocks reaches the tile last; if the count is then
    // complete it sums the parts in k order and runs the epilogue, else it writes its own part
    // to slot 1 and counts itself too, and whichever part is counted last does the sum. No part
    // ever waits for another.
    int sk_units;
    long long dp_tiles;
    long long sk_q;
    int sk_r;
    float* sk_part;    // [unit][2 slots][CG][kBM * BN] floats
    int* sk_count;     // [(num_tiles - dp_tiles) * CG * epilogue warps], zero at launch; the
                       // parts counted in bits 0-15, those that met an infinity from bit 16
    // 3xTF32 with infinite operands (nonfinite_fixup_tmem). op(A)(i, p) of matrix z at
    // ra[z*ra_bs + i*ra_rs + p] — A as the kernel reads it: raw where it is split in the kernel,
    // else its packed hi — and op(B)(p, j) at rb[z*rb_bs + j*rb_rs + p], B's packed hi; both
    // K-major with 16-byte aligned rows. ra is null outside 3xTF32. nf_word[i] == nf_tag[i] says
    // a packing pass met an infinity (i = 0: this call's own passes, 1: a pre-split B).
    const float* ra;
    long long ra_rs, ra_bs;
    const float* rb;
    long long rb_rs, rb_bs;
    const unsigned* nf_word[2];
    unsigned nf_tag[2];
};

// CG: CTAs per MMA (1 or 2). BN: N of one MMA (columns of the tile). Per CTA: kBM rows of A,
// BN/CG rows of B, a kBM x BN accumulator in TMEM. ATMEM: A arrives raw and is split into a
// ring of (hi, lo) slots in tensor memory, so a stage holds raw A and B's (hi, lo) only.
template <int CG, int BN, bool SPLIT3, bool ATMEM = false>
struct TcConfig {
    static constexpr int kBRows = BN / CG;
    static constexpr int kTileM = kBM * CG;
    static constexpr int kABytes = kBM * kBK * 4;
    static constexpr int kBBytes = kBRows * kBK * 4;
    static constexpr int kOps = SPLIT3 ? 2 : 1;
    // per CTA; stage layout: A (hi or raw) | B hi | A lo | B lo  (ATMEM: A raw | B hi | B lo)
    static constexpr int kStageBytes = ATMEM ? kABytes + 2 * kBBytes : kOps * (kABytes + kBBytes);
    static constexpr int kOffBHi = kABytes;
    static constexpr int kOffALo = kABytes + kBBytes;
    static constexpr int kOffBLo = ATMEM ? kABytes + kBBytes : 2 * kABytes + kBBytes;
    static constexpr int kStages = (192 * 1024) / kStageBytes;
    static constexpr int kAccStages = 2;
    static constexpr int kTmemCols = ATMEM                      ? 512
                                     : (kAccStages * BN <= 32)  ? 32
                                     : (kAccStages * BN <= 64)  ? 64
                                     : (kAccStages * BN <= 128) ? 128
                                     : (kAccStages * BN <= 256) ? 256
                                                                : 512;
    // ATMEM: slots of 64 columns (hi: 32, lo: 32 — one k-block) after the accumulators
    static constexpr int kACol0 = kAccStages * BN;
    static constexpr int kASlots = ATMEM ? (512 - kACol0) / 64 : 0;
    static constexpr int kThreads = ATMEM ? kTmThreads : kGemmThreads;
    static constexpr int kEpiWarp0C = ATMEM ? kTmEpiWarp0 : kEpiWarp0;
    static constexpr int kEpiWarpsC = ATMEM ? 4 : kEpiWarps;
    // Epilogue staging: each epilogue warp owns two 32 x 16 fp32 boxes (2 KB each).
    static constexpr int kEpiBoxBytes = 32 * kEpiCols * 4;
    static constexpr int kEpiBytes = kEpiWarpsC * 2 * kEpiBoxBytes;
    static constexpr int kBarrierBytes = 512;
    static constexpr int kSmemBytes = 1024 + kStages * kStageBytes + kEpiBytes + kBarrierBytes;
    static_assert(kSmemBytes <= 232448, "shared memory per CTA exceeded");
    static_assert(CG == 1 || CG == 2, "one or two CTAs per MMA");
    static_assert(kAccStages * BN <= 512, "accumulators exceed TMEM");
    static_assert(BN % 32 == 0 && BN >= 32 && BN <= 256, "BN must be 32..256, multiple of 32");
    static_assert(kBRows % 8 == 0, "B rows per CTA must be a multiple of 8");
    static_assert(kStages >= 2, "need at least two stages");
    static_assert(!ATMEM || (SPLIT3 && kASlots >= 2), "ATMEM: 3xTF32 with two or more A slots");
};

struct TileCoord {
    int b, tm, tn;
};

__device__ __forceinline__ TileCoord tile_coord(const GemmArgs& g, long long t) {
    const long long per_batch = static_cast<long long>(g.tiles_m) * g.tiles_n;
    TileCoord c;
    c.b = static_cast<int>(t / per_batch);
    const int r = static_cast<int>(t - static_cast<long long>(c.b) * per_batch);
    const int group_size = g.group_m * g.tiles_n;
    const int grp = r / group_size;
    const int first_m = grp * g.group_m;
    const int gm = min(g.tiles_m - first_m, g.group_m);
    const int in_group = r - grp * group_size;
    c.tm = first_m + in_group % gm;
    c.tn = in_group / gm;
    return c;
}

// Exact GELU, 0.5*v*erfc(-v/sqrt 2), evaluated in double as the reference does
// (src/backends/cpu/ops/elementwise/elementwise.cpp:173-192). Used by the standalone
// bias_add/activation kernel, where it matches the reference to 1 ulp.
__device__ __forceinline__ float gelu_exact(float value) {
    if (isinf(value)) return value < 0.0f ? -0.0f : value;
    const double v = value;
    return static_cast<float>(0.5 * v * erfc(-v * 0.70710678118654752440));
}

__device__ __forceinline__ float gelu_tanh(float value) {
    if (isinf(value)) return value < 0.0f ? -0.0f : value;
    const double v = value;
    const double u = 0.79788456080286535588 * v * (1.0 + 0.044715 * v * v);
    const double z = 2.0 * u;
    const double s = z >= 0.0 ? 1.0 / (1.0 + exp(-z)) : exp(z) / (1.0 + exp(z));
    return static_cast<float>(v * s);
}

// The same functions in fp32 for the GEMM epilogue, where double throughput would cost more
// than the tile's MMAs. The erfc argument -v/sqrt(2) is carried as a float pair (the product's
// rounding error recovered with an FMA) and erfcf is corrected to first order in the low part
// (d/dx erfc(x) = -2/sqrt(pi) e^{-x^2}), so the deep negative tail keeps its relative accuracy.
__device__ __forceinline__ float gelu_exact_f32(float v) {
    if (isinf(v)) return v < 0.0f ? -0.0f : v;
    const float c_hi = 0.70710677f;       // float(1/sqrt 2)
    const float c_lo = 1.21016175e-08f;   // 1/sqrt 2 - c_hi
    const float x = -v * c_hi;
    const float xe = fmaf(-v, c_hi, -x) - v * c_lo;
    float e = erfcf(x);
    e = fmaf(-1.12837917f * expf(-x * x), xe, e);
    return 0.5f * v * e;
}

// v * sigmoid(z), z = 2*sqrt(2/pi)*(v + 0.044715 v^3): z is accumulated as a float pair
// (products' rounding errors recovered with FMAs, the sum with TwoSum) and exp(-|z|) corrected
// to first order in the low part, since exp amplifies an argument error by |z|.
__device__ __forceinline__ float gelu_tanh_f32(float v) {
    // beyond |v| = 30 the sigmoid is 1 or underflows (z ~ 1270): v or -0, as in double
    if (fabsf(v) > 30.0f) return v < 0.0f ? -0.0f : v;
    const float a_hi = 1.59576917f, a_lo = -4.53406805e-08f;    // 2*sqrt(2/pi)
    const float b_hi = 0.0713548139f, b_lo = 2.39883247e-09f;   // 2*sqrt(2/pi)*0.044715
    const float v2 = v * v;
    const float v2e = fmaf(v, v, -v2);
    const float v3 = v2 * v;
    const float v3e = fmaf(v2, v, -v3) + v2e * v;
    const float z1 = a_hi * v;
    const float z1e = fmaf(a_hi, v, -z1) + a_lo * v;
    const float z2 = b_hi * v3;
    const float z2e = fmaf(b_hi, v3, -z2) + b_lo * v3 + b_hi * v3e;
    const float z = z1 + z2;
    const float bb = z - z1;
    const float ze = ((z1 - (z - bb)) + (z2 - bb)) + z1e + z2e;
    const float sg = z >= 0.0f ? 1.0f : -1.0f;
    const float w = expf(-fabsf(z)) * (1.0f - sg * ze);  // exp(-|z + ze|)
    const float s = z >= 0.0f ? 1.0f / (1.0f + w) : w / (1.0f + w);
    return v * s;
}

// Out-of-line copies for the epilogue's unrolled loops: one body in the instruction stream
// instead of 32. Four values per call: each evaluation is a long dependent chain, and four
// independent ones interleave (the same arithmetic per value as the scalar form).
__device__ __noinline__ float4 gelu_exact_f32_x4(float4 v) {
    return make_float4(gelu_exact_f32(v.x), gelu_exact_f32(v.y), gelu_exact_f32(v.z),
                       gelu_exact_f32(v.w));
}
__device__ __noinline__ float4 gelu_tanh_f32_x4(float4 v) {
    return make_float4(gelu_tanh_f32(v.x), gelu_tanh_f32(v.y), gelu_tanh_f32(v.z),
                       gelu_tanh_f32(v.w));
}

__device__ __forceinline__ float apply_act(float v, int act) {
    switch (act) {
    case kActRelu:
        return v < 0.0f ? 0.0f : v;
    case kActGelu:
        return gelu_exact(v);
    case kActGeluTanh:
        return gelu_tanh(v);
    default:
        return v;
    }
}

__device__ __forceinline__ float apply_act_f32(float v, int act) {
    switch (act) {
    case kActRelu:
        return v < 0.0f ? 0.0f : v;
    case kActGelu:
        return gelu_exact_f32(v);
    case kActGeluTanh:
        return gelu_tanh_f32(v);
    default:
        return v;
    }
}

// The reference composes alpha*AB (mul), + beta*C (scal then add) and + bias (bias_add) as
// separate fp32 operations; each rounding step is kept (no contraction into an FMA).
__device__ __forceinline__ float epilogue_value(float acc, float alpha, float beta, float cin,
                                                bool has_cin, float bias, bool has_bias,
                                                int act) {
    float v = alpha == 1.0f ? acc : __fmul_rn(alpha, acc);
    if (has_cin) v = __fadd_rn(v, __fmul_rn(beta, cin));
    if (has_bias) v = __fadd_rn(v, bias);
    return apply_act_f32(v, act);
}

template <int CG>
__device__ __forceinline__ long long first_tile() {
    return blockIdx.x / CG;
}

template <int CG>
__device__ __forceinline__ long long tile_step() {
    return gridDim.x / CG;
}

// One piece of a unit's work: k-blocks [kb0, kb1) of tile `tile`.
struct Work {
    long long tile;
    int kb0, kb1;
};

// First stream-K iteration of unit u, and the unit that owns iteration `it`.
__device__ __forceinline__ long long sk_start(const GemmArgs& g, long long u) {
    return u * g.sk_q + min(u, static_cast<long long>(g.sk_r));
}

__device__ __forceinline__ long long sk_unit_of(const GemmArgs& g, long long it) {
    const long long big = static_cast<long long>(g.sk_r) * (g.sk_q + 1);
    if (it < big || g.sk_q == 0) return it / (g.sk_q + 1);
    return g.sk_r + (it - big) / g.sk_q;
}

// The same sequence of work for every role of a CTA: this unit's share of the stream-K
// iterations (cut at tile boundaries) first, then its whole tiles — so the summing of a split
// tile's parts in the epilogue overlaps the MMAs of the whole tiles that follow.
template <int CG>
struct WorkIter {
    long long t, it, it_end;
    __device__ __forceinline__ explicit WorkIter(const GemmArgs& g) {
        t = first_tile<CG>();
        it = it_end = 0;
        if (g.sk_units > 0) {
            const long long u = blockIdx.x / CG;
            it = sk_start(g, u);
            it_end = sk_start(g, u + 1);
        }
    }
    __device__ __forceinline__ bool next(const GemmArgs& g, Work& w) {
        if (it < it_end) {
            const long long tr = it / g.num_kb;
            w.tile = g.dp_tiles + tr;
            w.kb0 = static_cast<int>(it - tr * g.num_kb);
            w.kb1 = static_cast<int>(min(static_cast<long long>(g.num_kb), w.kb0 + (it_end - it)));
            it += w.kb1 - w.kb0;
            return true;
        }
        const long long dp_end = g.sk_units > 0 ? g.dp_tiles : g.num_tiles;
        if (t < dp_end) {
            w.tile = t;
            w.kb0 = 0;
            w.kb1 = g.num_kb;
            t += tile_step<CG>();
            return true;
        }
        return false;
    }
};

// ASPLIT (3xTF32 only): A arrives as raw fp32 in the A_hi slot, completing on this CTA's own
// a_full barrier, and the converter warps write hi and lo (in shared memory, or for ATMEM into
// tensor memory); B arrives pre-split.
template <int CG, int BN, bool SPLIT3, bool ASPLIT, bool ATMEM>
__device__ __forceinline__ void tc_producer(const GemmArgs& g, const CUtensorMap* tmA0,
                                            const CUtensorMap* tmA1, const CUtensorMap* tmB0,
                                            const CUtensorMap* tmB1, uint8_t* stages,
                                            uint64_t* full, uint64_t* empty, uint64_t* a_full,
                                            uint32_t rank) {
    using C = TcConfig<CG, BN, SPLIT3, ATMEM>;
    static_assert(!ASPLIT || SPLIT3, "the in-kernel split is a 3xTF32 feature");
    const uint64_t pol = l2_policy_evict_last();
    // bytes that complete on `full`: everything, or only B's pair when A has its own barrier
    constexpr uint32_t kFullBytes = ASPLIT ? 2 * C::kBBytes : C::kStageBytes;
    int stage = 0;
    uint32_t phase = 0;
    WorkIter<CG> wi(g);
    for (Work w; wi.next(g, w);) {
        const TileCoord tc = tile_coord(g, w.tile);
        const int za = g.a_batch_bcast ? 0 : tc.b;
        const int zb = g.b_batch_bcast ? 0 : tc.b;
        const int ya = tc.tm * C::kTileM + static_cast<int>(rank) * kBM;
        const int yb = tc.tn * BN + static_cast<int>(rank) * C::kBRows;
        for (int kb = w.kb0; kb < w.kb1; ++kb) {
            if (!mbar_wait(&empty[stage], phase ^ 1u, kErrProducerWait)) return;
            uint8_t* s = stages + stage * C::kStageBytes;
            uint8_t* s_ahi = s;
            uint8_t* s_bhi = s + C::kOffBHi;
            uint8_t* s_alo = s + C::kOffALo;
            uint8_t* s_blo = s + C::kOffBLo;
            const int kx = kb * kBK;
            if constexpr (ASPLIT) {
                mbar_arrive_expect_tx(&a_full[stage], C::kABytes);
                tma_load_3d(s_ahi, tmA0, &a_full[stage], kx, ya, za, pol);
            }
            if constexpr (CG == 1) {
                mbar_arrive_expect_tx(&full[stage], kFullBytes);
                if constexpr (!ASPLIT) tma_load_3d(s_ahi, tmA0, &full[stage], kx, ya, za, pol);
                tma_load_3d(s_bhi, tmB0, &full[stage], kx, yb, zb, pol);
                if constexpr (SPLIT3) {
                    if constexpr (!ASPLIT) tma_load_3d(s_alo, tmA1, &full[stage], kx, ya, za, pol);
                    tma_load_3d(s_blo, tmB1, &full[stage], kx, yb, zb, pol);
                }
            } else {
                // Both CTAs' bytes complete on the first CTA's barrier, which expects them all.
                if (rank == 0) mbar_arrive_expect_tx(&full[stage], CG * kFullBytes);
                const uint32_t bar = mapa_shared(&full[stage], 0);
                if constexpr (!ASPLIT) tma_load_3d_cg2(s_ahi, tmA0, bar, kx, ya, za, pol);
                tma_load_3d_cg2(s_bhi, tmB0, bar, kx, yb, zb, pol);
                if constexpr (SPLIT3) {
                    if constexpr (!ASPLIT) tma_load_3d_cg2(s_alo, tmA1, bar, kx, ya, za, pol);
                    tma_load_3d_cg2(s_blo, tmB1, bar, kx, yb, zb, pol);
                }
            }
            if (++stage == C::kStages) {
                stage = 0;
                phase ^= 1u;
            }
        }
    }
}

// The converter warps of an ASPLIT kernel: for every stage, once this CTA's raw A tile has
// landed, split_tf32(x) writes hi in place and lo into the A_lo slot (an elementwise pass, so
// the 128-byte swizzle of the tile carries over) — or, where the tensor cores are known to
// truncate fp32 operands (g.raw_hi), only lo, since truncated x is hi — then a proxy fence
// so the MMA's async reads see the generic writes, and one arrival per warp on the MMA issuer's
// `converted` barrier.
template <int CG, int BN, bool SPLIT3>
__device__ __forceinline__ void tc_convert(const GemmArgs& g, uint8_t* stages, uint64_t* a_full,
                                           uint64_t* converted, uint32_t* inf_seen) {
    using C = TcConfig<CG, BN, SPLIT3>;
    const int ct = threadIdx.x - kCvtWarp0 * 32;
    const int lane = threadIdx.x % 32;
    int stage = 0;
    uint32_t phase = 0;
    bool inf = false;  // this thread has met an infinity in A (for the epilogue's fix-up)
    WorkIter<CG> wi(g);
    for (Work w; wi.next(g, w);) {
        for (int kb = w.kb0; kb < w.kb1; ++kb) {
            if (!mbar_wait(&a_full[stage], phase, kErrConvertWait)) return;
            float4* hi = reinterpret_cast<float4*>(stages + stage * C::kStageBytes);
            float4* lo = reinterpret_cast<float4*>(stages + stage * C::kStageBytes + C::kABytes +
                                                   C::kBBytes);
            if (g.raw_hi) {
                // the tensor cores truncate fp32 to tf32, so x already is hi: only lo is written
#pragma unroll 4
                for (int i = ct; i < C::kABytes / 16; i += kCvtThreads) {
                    const float4 x = hi[i];
                    float4 h, l;
                    split_tf32(x.x, h.x, l.x);
                    split_tf32(x.y, h.y, l.y);
                    split_tf32(x.z, h.z, l.z);
                    split_tf32(x.w, h.w, l.w);
                    inf |= any_inf(x);
                    lo[i] = l;
                }
            } else {
#pragma unroll 4
                for (int i = ct; i < C::kABytes / 16; i += kCvtThreads) {
                    const float4 x = hi[i];
                    float4 h, l;
                    split_tf32(x.x, h.x, l.x);
                    split_tf32(x.y, h.y, l.y);
                    split_tf32(x.z, h.z, l.z);
                    split_tf32(x.w, h.w, l.w);
                    inf |= any_inf(x);
                    hi[i] = h;
                    lo[i] = l;
                }
            }
            if (inf) *reinterpret_cast<volatile uint32_t*>(inf_seen) = 1u;
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
                if constexpr (CG == 1) {
                    mbar_arrive(&converted[stage]);
                } else {
                    mbar_arrive_cluster(mapa_shared(&converted[stage], 0));
                }
            }
            if (++stage == C::kStages) {
                stage = 0;
                phase ^= 1u;
            }
        }
    }
}

// The converter warps of an ATMEM kernel, one per TMEM lane quarter (warp % 4): thread `lane`
// of warp q owns row 32q + lane of the CTA's A tile. For every k-block it reads the row's 32
// raw fp32 values out of the swizzled stage (16-byte chunk c of row r sits at c ^ (r % 8)),
// releases the stage's A half, and writes split_tf32(x) into the next slot of the TMEM ring:
// columns [slot*64, +32) hold hi, [+32, +64) lo, one k per column. hi and lo are both exact
// tf32 values, so the MMA's own fp32 -> tf32 conversion never applies.
template <int CG, int BN>
__device__ __forceinline__ void tc_convert_tmem(const GemmArgs& g, uint8_t* stages,
                                                uint64_t* a_full, uint64_t* empty,
                                                uint64_t* tfull, uint64_t* tempty,
                                                uint32_t tmem_base, int group,
                                                uint32_t* inf_seen) {
    using C = TcConfig<CG, BN, true, true>;
    const int warp = threadIdx.x / 32;
    const int lane = threadIdx.x % 32;
    const int q = warp % 4;
    const int row = q * 32 + lane;
    const uint32_t lane_base = tmem_base + (static_cast<uint32_t>(q * 32) << 16);
    long long total = 0;  // k-blocks in this CTA's whole sequence of work
    {
        WorkIter<CG> wi(g);
        for (Work w; wi.next(g, w);) total += w.kb1 - w.kb0;
    }
    // k-block i of this CTA's sequence uses stage i % kStages and slot i % kASlots
    for (long long i = group; i < total; i += 2) {
        {
            const int stage = static_cast<int>(i % C::kStages);
            const uint32_t phase = static_cast<uint32_t>((i / C::kStages) & 1);
            const int slot = static_cast<int>(i % C::kASlots);
            const uint32_t tphase = static_cast<uint32_t>((i / C::kASlots) & 1);
            if (!mbar_wait(&a_full[stage], phase, kErrConvertWait)) return;
            const uint32_t rowp = smem_u32(stages + stage * C::kStageBytes) + row * 128;
            float x[32];
            bool inf = false;
#pragma unroll
            for (int c = 0; c < 8; ++c) {
                const float4 v = ld_shared_v4(rowp + ((c ^ (row & 7)) << 4));
                x[4 * c] = v.x;
                x[4 * c + 1] = v.y;
                x[4 * c + 2] = v.z;
                x[4 * c + 3] = v.w;
                inf |= any_inf(v);
            }
            // raised before this k-block's arrival on tfull, so before the MMAs that read it
            if (inf) *reinterpret_cast<volatile uint32_t*>(inf_seen) = 1u;
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[stage]);  // this warp's rows of A are read
            if (!mbar_wait(&tempty[slot], tphase ^ 1u, kErrConvertWait)) return;
            tc_fence_after();
            const uint32_t col = static_cast<uint32_t>(C::kACol0 + slot * 64);
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                uint32_t hi[16], lo[16];
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    float fh, fl;
                    split_tf32(x[16 * h + j], fh, fl);
                    hi[j] = __float_as_uint(fh);
                    lo[j] = __float_as_uint(fl);
                }
                tmem_st_32x32b_x16(lane_base + col + 16 * h, hi);
                tmem_st_32x32b_x16(lane_base + col + 32 + 16 * h, lo);
            }
            tmem_st_wait();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                if constexpr (CG == 1) {
                    mbar_arrive(&tfull[slot]);
                } else {
                    mbar_arrive_cluster(mapa_shared(&tfull[slot], 0));
                }
            }
        }
    }
}

// Runs on one lane of the pair's first CTA (or of the single CTA).
template <int CG, int BN, bool SPLIT3, bool ASPLIT, bool ATMEM>
__device__ __forceinline__ void tc_mma(const GemmArgs& g, uint32_t tmem_base, uint8_t* stages,
                                       uint64_t* full, uint64_t* empty, uint64_t* acc_full,
                                       uint64_t* acc_empty, uint64_t* converted,
                                       uint64_t* tempty) {
    using C = TcConfig<CG, BN, SPLIT3, ATMEM>;
    constexpr uint32_t idesc = idesc_tf32(C::kTileM, BN, false, false);
    constexpr uint16_t kPair = (1u << CG) - 1u;
    int stage = 0;
    uint32_t phase = 0;
    int acc = 0;
    uint32_t acc_phase = 0;
    int slot = 0;             // ATMEM: the TMEM ring slot holding this k-block's A (hi, lo)
    uint32_t tphase = 0;
    const uint32_t stage0 = smem_u32(stages);
    WorkIter<CG> wi(g);
    for (Work w; wi.next(g, w);) {
        if (!mbar_wait(&acc_empty[acc], acc_phase ^ 1u, kErrMmaWait)) return;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
        for (int kb = w.kb0; kb < w.kb1; ++kb) {
            if (!mbar_wait(&full[stage], phase, kErrMmaWait)) return;
            if constexpr (ATMEM) {
                if (!mbar_wait(&converted[slot], tphase, kErrMmaWait)) return;
            } else if constexpr (ASPLIT) {
                if (!mbar_wait(&converted[stage], phase, kErrMmaWait)) return;
            }
            tc_fence_after();
            const uint32_t a_hi = stage0 + stage * C::kStageBytes;
            const uint32_t b_hi = a_hi + C::kOffBHi;
            const uint32_t a_lo = a_hi + C::kOffALo;
            const uint32_t b_lo = a_hi + C::kOffBLo;
            if constexpr (ATMEM) {
                // A from the TMEM slot: hi at column kACol0 + slot*64 + k, lo 32 columns on
                const uint32_t ta = tmem_base + static_cast<uint32_t>(C::kACol0 + slot * 64);
#pragma unroll
                for (int ks = 0; ks < kBK / 8; ++ks) {
                    const uint32_t koff = ks * 32;
                    const uint64_t dbh = smem_desc(b_hi + koff, 16, 1024, kSwizzle128B);
                    const uint64_t dbl = smem_desc(b_lo + koff, 16, 1024, kSwizzle128B);
                    const uint32_t tah = ta + ks * 8;
                    const uint32_t tal = tah + 32;
                    const uint32_t accumulate = (kb > w.kb0 || ks > 0) ? 1u : 0u;
                    if constexpr (CG == 1) {
                        mma_tf32_ts(d_tmem, tal, dbh, idesc, accumulate);
                        mma_tf32_ts(d_tmem, tah, dbl, idesc, 1u);
                        mma_tf32_ts(d_tmem, tah, dbh, idesc, 1u);
                    } else {
                        mma_tf32_ts_cg2(d_tmem, tal, dbh, idesc, accumulate);
                        mma_tf32_ts_cg2(d_tmem, tah, dbl, idesc, 1u);
                        mma_tf32_ts_cg2(d_tmem, tah, dbh, idesc, 1u);
                    }
                }
                if constexpr (CG == 1) {
                    mma_commit(&empty[stage]);
                    mma_commit(&tempty[slot]);
                } else {
                    mma_commit_cg2_mc(&empty[stage], kPair);
                    mma_commit_cg2_mc(&tempty[slot], kPair);
                }
                if (++slot == C::kASlots) {
                    slot = 0;
                    tphase ^= 1u;
                }
            } else {
#pragma unroll
                for (int ks = 0; ks < kBK / 8; ++ks) {
                    const uint32_t koff = ks * 32;  // 8 tf32 = 32 bytes along the swizzled row
                    const uint64_t dah = smem_desc(a_hi + koff, 16, 1024, kSwizzle128B);
                    const uint64_t dbh = smem_desc(b_hi + koff, 16, 1024, kSwizzle128B);
                    const uint32_t accumulate = (kb > w.kb0 || ks > 0) ? 1u : 0u;
                    if constexpr (SPLIT3) {
                        const uint64_t dal = smem_desc(a_lo + koff, 16, 1024, kSwizzle128B);
                        const uint64_t dbl = smem_desc(b_lo + koff, 16, 1024, kSwizzle128B);
                        if constexpr (CG == 1) {
                            mma_tf32(d_tmem, dal, dbh, idesc, accumulate);
                            mma_tf32(d_tmem, dah, dbl, idesc, 1u);
                            mma_tf32(d_tmem, dah, dbh, idesc, 1u);
                        } else {
                            mma_tf32_cg2(d_tmem, dal, dbh, idesc, accumulate);
                            mma_tf32_cg2(d_tmem, dah, dbl, idesc, 1u);
                            mma_tf32_cg2(d_tmem, dah, dbh, idesc, 1u);
                        }
                    } else {
                        if constexpr (CG == 1) {
                            mma_tf32(d_tmem, dah, dbh, idesc, accumulate);
                        } else {
                            mma_tf32_cg2(d_tmem, dah, dbh, idesc, accumulate);
                        }
                    }
                }
                if constexpr (CG == 1) {
                    mma_commit(&empty[stage]);
                } else {
                    mma_commit_cg2_mc(&empty[stage], kPair);  // frees the stage in both CTAs
                }
            }
            if (++stage == C::kStages) {
                stage = 0;
                phase ^= 1u;
            }
        }
        if constexpr (CG == 1) {
            mma_commit(&acc_full[acc]);
        } else {
            mma_commit_cg2_mc(&acc_full[acc], kPair);
        }
        if (++acc == C::kAccStages) {
            acc = 0;
            acc_phase ^= 1u;
        }
    }
}

// This warp's block of unit u's stream-K slot `slot` (kBM x BN floats per CTA rank): warp
// (half, ew)'s chunk ci is a 2 KB block at ((half*kChunks + ci)*4 + ew) * 512 floats, stored as
// four 512-byte rows of float4 (float4 q of lane l at q*32 + l), so each warp instruction moves
// 512 contiguous bytes.
template <int CG, int BN>
__device__ __forceinline__ float4* sk_part_block(const GemmArgs& g, long long u, int slot,
                                                 uint32_t rank, int half, int ew, int ci,
                                                 int kChunks) {
    float* base = g.sk_part + ((u * 2 + slot) * CG + rank) * static_cast<long long>(kBM * BN);
    return reinterpret_cast<float4*>(
        base + ((static_cast<long long>(half) * kChunks + ci) * 4 + ew) * 512);
}

// This warp's raw accumulator (TMEM, all chunks) into unit u's slot `slot`, then counted.
// Returns the count before this part (so count + 1 parts are written).
template <int CG, int BN, int kChunks>
__device__ __forceinline__ int sk_write_part(const GemmArgs& g, uint32_t tbase, long long u,
                                             int slot, uint32_t rank, int half, int ew, int lane,
                                             int* count, int add) {
#pragma unroll 1
    for (int ci = 0; ci < kChunks; ci += 2) {
        uint32_t r0[kEpiCols], r1[kEpiCols];
        tmem_ld_issue_32x32b_x16(tbase + ci * kEpiCols, r0);
        tmem_ld_issue_32x32b_x16(tbase + (ci + 1) * kEpiCols, r1);
        tmem_ld_wait();
        float4* d0 = sk_part_block<CG, BN>(g, u, slot, rank, half, ew, ci, kChunks);
        float4* d1 = sk_part_block<CG, BN>(g, u, slot, rank, half, ew, ci + 1, kChunks);
#pragma unroll
        for (int q = 0; q < kEpiCols / 4; ++q) {
            __stcg(d0 + q * 32 + lane,
                   make_float4(__uint_as_float(r0[4 * q]), __uint_as_float(r0[4 * q + 1]),
                               __uint_as_float(r0[4 * q + 2]), __uint_as_float(r0[4 * q + 3])));
            __stcg(d1 + q * 32 + lane,
                   make_float4(__uint_as_float(r1[4 * q]), __uint_as_float(r1[4 * q + 1]),
                               __uint_as_float(r1[4 * q + 2]), __uint_as_float(r1[4 * q + 3])));
        }
    }
    __threadfence();
    __syncwarp();
    int prev = 0;
    if (lane == 0) prev = atomicAdd(count, add);
    return __shfl_sync(0xffffffffu, prev, 0);
}

// Replaces this warp's own part in TMEM with the sum over every part of the split tile, added
// in k order (unit u_first's part first) so the bits do not depend on which part was counted
// last; the regular epilogue then reads the tile from TMEM as usual. The parts of units after
// u_first are in their slot 0, u_first's (when another unit sums) in its slot 1, this unit's
// own in TMEM. Chunk by chunk, the other parts' loads of a pair in flight together.
template <int CG, int BN, int kChunks>
__device__ __forceinline__ void sk_fixup_tmem(const GemmArgs& g, uint32_t tbase,
                                              long long u_first, long long u_last, long long me,
                                              uint32_t rank, int half, int ew, int lane) {
    constexpr int kGroup = 2;
    __threadfence();  // the parts counted before this point are visible
#pragma unroll 1
    for (int ci = 0; ci < kChunks; ++ci) {
        uint32_t own[kEpiCols];
        tmem_ld_issue_32x32b_x16(tbase + ci * kEpiCols, own);
        tmem_ld_wait();
        float sum[kEpiCols];
#pragma unroll
        for (int j = 0; j < kEpiCols; ++j) sum[j] = 0.0f;
#pragma unroll 1
        for (long long v0 = u_first; v0 <= u_last; v0 += kGroup) {
            float4 part[kGroup][kEpiCols / 4];
#pragma unroll
            for (int p = 0; p < kGroup; ++p) {
                const long long v = v0 + p;
                if (v <= u_last && v != me) {
                    const float4* src = sk_part_block<CG, BN>(g, v, v == u_first ? 1 : 0, rank,
                                                              half, ew, ci, kChunks);
#pragma unroll
                    for (int q = 0; q < kEpiCols / 4; ++q) part[p][q] = __ldcg(src + q * 32 + lane);
                }
            }
#pragma unroll
            for (int p = 0; p < kGroup; ++p) {
                const long long v = v0 + p;
                if (v <= u_last) {
                    float val[kEpiCols];
                    if (v == me) {
#pragma unroll
                        for (int j = 0; j < kEpiCols; ++j) val[j] = __uint_as_float(own[j]);
                    } else {
#pragma unroll
                        for (int q = 0; q < kEpiCols / 4; ++q) {
                            val[4 * q] = part[p][q].x;
                            val[4 * q + 1] = part[p][q].y;
                            val[4 * q + 2] = part[p][q].z;
                            val[4 * q + 3] = part[p][q].w;
                        }
                    }
#pragma unroll
                    for (int j = 0; j < kEpiCols; ++j)
                        sum[j] = v == u_first ? val[j] : __fadd_rn(sum[j], val[j]);
                }
            }
        }
#pragma unroll
        for (int j = 0; j < kEpiCols; ++j) own[j] = __float_as_uint(sum[j]);
        tmem_st_32x32b_x16(tbase + ci * kEpiCols, own);
    }
    tmem_st_wait();
}

// Infinite operands in 3xTF32. An infinite x splits into hi = x and lo = 0, so a product
// hi(a)*hi(b) + hi(a)*lo(b) + lo(a)*hi(b) with a = inf and b exact in tf32 (lo(b) = 0) holds
// inf * 0 = NaN where the reference's fp32 product is an infinity. A dot product that meets an
// infinity has a non-finite result that the order of its sum does not change (NaN if any term is
// NaN or two infinite terms differ in sign, else the infinity), so each NaN accumulator of such a
// tile is replaced by the plain fp32 dot product from the operands in memory, in tensor memory
// before the epilogue reads it. Entries the tensor cores got right are not touched, and tiles
// that cannot hold such an entry never come here (the flags the packing passes and the
// converter warps raise on meeting an infinity). B is read as its packed hi, which keeps every
// sign, zero and infinity of B (only a denormal below 2^-136 truncates to zero).
__device__ __forceinline__ float nonfinite_dot(const GemmArgs& g, int b, int row, int col) {
    const float* a = g.ra + static_cast<long long>(b) * g.ra_bs + static_cast<long long>(row) * g.ra_rs;
    const float* x = g.rb + static_cast<long long>(b) * g.rb_bs + static_cast<long long>(col) * g.rb_rs;
    float acc = 0.0f;
#pragma unroll 1
    for (int p = 0; p < g.k; ++p) acc = fmaf(__ldg(a + p), __ldg(x + p), acc);
    return acc;
}

// This warp's columns [colbase, colbase + kChunks*kEpiCols) of row `row` of the tile in tensor
// memory at tbase: every NaN entry recomputed by nonfinite_dot and written back, one column at a
// time (few registers live besides the epilogue's). Warp-uniform.
template <int kChunks>
__device__ __forceinline__ void nonfinite_fixup_tmem(const GemmArgs& g, uint32_t tbase, int b,
                                                     int row, bool row_ok, int colbase) {
#pragma unroll 1
    for (int ci = 0; ci < kChunks; ++ci) {
        const int col0 = colbase + ci * kEpiCols;
        uint32_t nan_mask = 0;
        {
            uint32_t r[kEpiCols];
            tmem_ld_issue_32x32b_x16(tbase + ci * kEpiCols, r);
            tmem_ld_wait();
#pragma unroll
            for (int j = 0; j < kEpiCols; ++j)
                if (isnan(__uint_as_float(r[j]))) nan_mask |= 1u << j;
        }
        const int cols = g.n - col0;
        if (!row_ok || cols <= 0) nan_mask = 0;
        if (cols < kEpiCols) nan_mask &= (1u << max(cols, 0)) - 1u;
        // the columns where some lane of the warp holds a NaN
        for (uint32_t m = __reduce_or_sync(0xffffffffu, nan_mask); m != 0; m &= m - 1) {
            const int j = __ffs(m) - 1;
            const uint32_t taddr = tbase + ci * kEpiCols + j;
            uint32_t v;
            tmem_ld_issue_32x32b_x1(taddr, v);
            tmem_ld_wait();
            if (nan_mask & (1u << j)) v = __float_as_uint(nonfinite_dot(g, b, row, col0 + j));
            __syncwarp();  // the store below is warp-collective
            tmem_st_32x32b_x1(taddr, v);
        }
    }
    tmem_st_wait();
}

// The epilogue of one kEpiCols-column chunk of a thread's row: alpha, beta*C_in, bias,
// activation, with the reference's rounding steps. The activation is applied in a separate pass
// over the values so each unrolled loop stays short.
struct EpiRow {
    const float* cin_row;
    bool has_cin, has_bias, vec_cin;
    // The bias of the warp's columns of the tile, spread over the lanes: lane l holds columns
    // 4l .. 4l+3 of the warp's part (loaded once per tile, before the accumulator is ready), and
    // a chunk's values are broadcast from there with shuffles instead of 16 dependent loads.
    float4 bias4;
    int chunk;  // the chunk being computed: its 16 columns sit in lanes 4 chunk .. 4 chunk + 3
    // cin_pre: this chunk's C_in was copied ahead into the thread's row of a staging box, at
    // shared address cin_smem (16-byte piece q at q ^ cin_swz), and is read from there.
    bool cin_pre;
    uint32_t cin_smem;
    uint32_t cin_swz;
};

// Copies this lane's 64 bytes of C_in for the chunk at col0 into row `lane` of the staging box
// at `buf`, in the box's swizzled layout, with cp.async: the loads are in flight without
// holding registers. Commits one group per call (empty when the lane has no whole chunk there).
__device__ __forceinline__ void cin_fetch(const EpiRow& e, uint32_t buf, int col0, int n,
                                          int lane) {
    if (e.has_cin && col0 + kEpiCols <= n) {
        const float* src = e.cin_row + col0;
#pragma unroll
        for (int q = 0; q < kEpiCols / 4; ++q)
            cp_async_16(buf + lane * (kEpiCols * 4) + ((q ^ ((lane >> 1) & 3)) << 4), src + 4 * q);
    }
    cp_async_commit();
}

// Bias of column j (0..15) of the current chunk, from the lane that holds it. Warp-uniform.
__device__ __forceinline__ float chunk_bias(const EpiRow& e, int j) {
    const float b = (j & 3) == 0 ? e.bias4.x : (j & 3) == 1 ? e.bias4.y
                  : (j & 3) == 2 ? e.bias4.z : e.bias4.w;
    return __shfl_sync(0xffffffffu, b, e.chunk * 4 + (j >> 2));
}

// The warp's bias values for columns [col_base, col_base + cols) of the tile (cols <= 128), lane
// l taking columns 4l .. 4l+3; columns at or past n read as 0 (never used).
__device__ __forceinline__ float4 load_tile_bias(const GemmArgs& g, int col_base, int cols,
                                                 int lane) {
    float4 b = make_float4(0.f, 0.f, 0.f, 0.f);
    const int c = col_base + 4 * lane;
    if (g.bias == nullptr || 4 * lane >= cols || c >= g.n) return b;
    if (c + 4 <= g.n && (reinterpret_cast<uintptr_t>(g.bias + c) & 15) == 0) {
        b = __ldg(reinterpret_cast<const float4*>(g.bias + c));
    } else {
        b.x = __ldg(g.bias + c);
        if (c + 1 < g.n) b.y = __ldg(g.bias + c + 1);
        if (c + 2 < g.n) b.z = __ldg(g.bias + c + 2);
        if (c + 3 < g.n) b.w = __ldg(g.bias + c + 3);
    }
    return b;
}

__device__ __forceinline__ void epilogue_general(const GemmArgs& g, const EpiRow& e, int col0,
                                                 const uint32_t (&r)[kEpiCols],
                                                 float (&v)[kEpiCols]) {
    if (col0 + kEpiCols <= g.n && (!e.has_cin || e.vec_cin)) {
#pragma unroll
        for (int j = 0; j < kEpiCols; j += 4) {
            float4 cin4 = make_float4(0.f, 0.f, 0.f, 0.f);
            if (e.has_cin) {
                cin4 = e.cin_pre
                           ? ld_shared_v4(e.cin_smem + (((j >> 2) ^ e.cin_swz) << 4))
                           : *reinterpret_cast<const float4*>(e.cin_row + col0 + j);
            }
            const float c4[4] = {cin4.x, cin4.y, cin4.z, cin4.w};
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                float x = __uint_as_float(r[j + q]);
                if (g.alpha != 1.0f) x = __fmul_rn(g.alpha, x);
                if (e.has_cin) x = __fadd_rn(x, __fmul_rn(g.beta, c4[q]));
                if (e.has_bias) x = __fadd_rn(x, chunk_bias(e, j + q));
                v[j + q] = x;
            }
        }
    } else {
#pragma unroll
        for (int j = 0; j < kEpiCols; ++j) {
            const int col = col0 + j;
            float x = __uint_as_float(r[j]);
            if (g.alpha != 1.0f) x = __fmul_rn(g.alpha, x);
            if (col < g.n) {
                if (e.has_cin) x = __fadd_rn(x, __fmul_rn(g.beta, e.cin_row[static_cast<long long>(col) * g.c_in_cs]));
                if (e.has_bias) x = __fadd_rn(x, chunk_bias(e, j));
            }
            v[j] = x;
        }
    }
    if (g.act == kActRelu) {
#pragma unroll
        for (int j = 0; j < kEpiCols; ++j) v[j] = v[j] < 0.0f ? 0.0f : v[j];
    } else if (g.act == kActGelu) {
#pragma unroll
        for (int j = 0; j < kEpiCols; j += 4) {
            const float4 r = gelu_exact_f32_x4(make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]));
            v[j] = r.x;
            v[j + 1] = r.y;
            v[j + 2] = r.z;
            v[j + 3] = r.w;
        }
    } else if (g.act == kActGeluTanh) {
#pragma unroll
        for (int j = 0; j < kEpiCols; j += 4) {
            const float4 r = gelu_tanh_f32_x4(make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]));
            v[j] = r.x;
            v[j + 1] = r.y;
            v[j + 2] = r.z;
            v[j + 3] = r.w;
        }
    }
}

// The epilogue warps (eight, or four in ATMEM kernels): warp w reads TMEM lane quarter (w % 4)
// — the 32 rows it may access — and, with eight warps, the columns of its half of the tile, in
// chunks of kEpiCols.
template <int CG, int BN, bool SPLIT3, bool ATMEM, bool CINA>
__device__ __forceinline__ void tc_epilogue(const GemmArgs& g, const CUtensorMap* tmC,
                                            uint8_t* epi_smem, uint32_t tmem_base,
                                            uint64_t* acc_full, uint64_t* acc_empty,
                                            uint32_t rank, const uint32_t* inf_seen) {
    using C = TcConfig<CG, BN, SPLIT3, ATMEM>;
    constexpr int kHalf = BN / (C::kEpiWarpsC / 4);  // columns per warp
    constexpr int kChunks = kHalf / kEpiCols;
    static_assert(kChunks % 2 == 0, "the peer-store path writes chunks in pairs");
    const int warp = threadIdx.x / 32;
    const int lane = threadIdx.x % 32;
    const int ew = warp % 4;                            // TMEM lane quarter this warp may access
    const int half = (warp - C::kEpiWarp0C) / 4;        // which part of the tile's columns
    EpiRow e;
    const bool has_cin = g.c_in != nullptr && g.beta != 0.0f;
    e.has_bias = g.bias != nullptr;
    e.vec_cin = has_cin && g.c_in_cs == 1 && (g.c_in_rs % 4 == 0) && (g.c_in_bs % 4 == 0) &&
                ((reinterpret_cast<uintptr_t>(g.c_in) & 15) == 0);
    // Only alpha to apply: the warp-uniform short path.
    const bool plain = !has_cin && !e.has_bias && g.act == kActNone;
    const bool vec_out = (g.ldc % 4 == 0) && ((reinterpret_cast<uintptr_t>(g.c) & 15) == 0) &&
                         (g.c_bs % 4 == 0);
    // This warp's two staging boxes: 32 rows of 64 B, SWIZZLE_64B as the TMA store reads them.
    const uint32_t box0 = smem_u32(epi_smem + (warp - C::kEpiWarp0C) * 2 * C::kEpiBoxBytes);
    // CINA (short K, where the epilogue bounds the kernel) and TMA stores: the boxes also carry
    // C_in. Each chunk's C_in is copied into the box its result will be staged in, one chunk
    // ahead (the tile's first chunk while the accumulator is still being computed), and the
    // result overwrites it in place.
    const bool pre_cin = CINA && e.vec_cin && g.tma_store;
    e.cin_pre = false;
    e.cin_smem = 0u;
    e.cin_swz = static_cast<uint32_t>((lane >> 1) & 3);
    int box = 0;
    int acc = 0;
    uint32_t acc_phase = 0;
    const int wid = warp - C::kEpiWarp0C;
    const long long me = blockIdx.x / CG;
    // a packing pass of this call met an infinity (written before the launch)
    bool inf_packed = false;
    if constexpr (SPLIT3) {
        for (int i = 0; i < 2; ++i)
            inf_packed |= g.ra != nullptr && g.nf_word[i] != nullptr && *g.nf_word[i] == g.nf_tag[i];
    }
    static_assert(kHalf <= 128, "a warp's bias columns must fit four per lane");
    WorkIter<CG> wi(g);
    for (Work w; wi.next(g, w);) {
        const TileCoord tc = tile_coord(g, w.tile);
        const int row0 = tc.tm * C::kTileM + static_cast<int>(rank) * kBM + ew * 32;
        const int row = row0 + lane;
        const bool row_ok = row < g.m;
        float* crow = g.c + static_cast<long long>(tc.b) * g.c_bs + static_cast<long long>(row) * g.ldc;
        e.has_cin = has_cin && row_ok;
        e.cin_row = e.has_cin ? g.c_in + static_cast<long long>(tc.b) * g.c_in_bs +
                                    static_cast<long long>(row) * g.c_in_rs
                              : nullptr;
        const int col_w = tc.tn * BN + half * kHalf;  // this warp's first column of the tile
        // the bias of this warp's columns, in flight while the accumulator is finished
        if (e.has_bias) e.bias4 = load_tile_bias(g, col_w, kHalf, lane);
        // and the first chunk's C_in, for a whole tile (a stream-K part fetches it only once it
        // knows it sums the tile), into the box no store is reading any more
        bool cin_ahead = false;
        if (pre_cin && w.kb0 == 0 && w.kb1 == g.num_kb && row0 < g.m && col_w < g.n) {
            if (lane == 0) bulk_wait_read<0>();
            __syncwarp();
            cin_fetch(e, box0 + box * C::kEpiBoxBytes, col_w, g.n, lane);
            cin_ahead = true;
        }
        if (!mbar_wait(&acc_full[acc], acc_phase, kErrEpilogueWait)) break;
        tc_fence_after();
        const uint32_t tbase = tmem_base + (static_cast<uint32_t>(ew * 32) << 16) +
                               static_cast<uint32_t>(acc * BN + half * kHalf);
        // 3xTF32: the k-blocks behind this accumulator may have met an infinity. The converters
        // raise their flag before arriving for the k-block that held it, so before the MMAs this
        // accumulator waited on.
        bool inf_tile = false;
        if constexpr (SPLIT3)
            inf_tile = inf_packed || *reinterpret_cast<const volatile uint32_t*>(inf_seen) != 0u;
        // A stream-K part of a tile (see GemmArgs::sk_units): either this warp sums the tile's
        // parts and falls through to the regular epilogue, or it leaves its part for another
        // unit and moves on. Nothing here waits for another unit. Each part adds 1 to the
        // tile's count, plus 1 << 16 if its k-blocks may have met an infinity.
        if (w.kb0 != 0 || w.kb1 != g.num_kb) {
            const long long tr = w.tile - g.dp_tiles;
            const long long u_first = sk_unit_of(g, tr * g.num_kb);
            const long long u_last = sk_unit_of(g, (tr + 1) * g.num_kb - 1);
            const int others = static_cast<int>(u_last - u_first);  // parts besides one
            int* count = &g.sk_count[(tr * CG + rank) * C::kEpiWarpsC + wid];
            const int add = inf_tile ? 1 + (1 << 16) : 1;
            int seen = 0;  // the count before this part's: the other parts written so far
            if (w.kb0 != 0) {
                // a later part: counted last means every other part is written
                seen = sk_write_part<CG, BN, kChunks>(g, tbase, me, 0, rank, half, ew, lane,
                                                      count, add);
            } else {
                if (lane == 0) seen = atomicAdd(count, 0);
                seen = __shfl_sync(0xffffffffu, seen, 0);
                if ((seen & 0xffff) != others)
                    seen = sk_write_part<CG, BN, kChunks>(g, tbase, me, 1, rank, half, ew, lane,
                                                          count, add);
            }
            const bool sums = (seen & 0xffff) == others;
            inf_tile |= (seen >> 16) != 0;
            if (!sums) {
                tc_fence_before();
                __syncwarp();
                if (lane == 0) {
                    if constexpr (CG == 1) {
                        mbar_arrive(&acc_empty[acc]);
                    } else {
                        mbar_arrive_cluster(mapa_shared(&acc_empty[acc], 0));
                    }
                }
                if (++acc == C::kAccStages) {
                    acc = 0;
                    acc_phase ^= 1u;
                }
                continue;
            }
            sk_fixup_tmem<CG, BN, kChunks>(g, tbase, u_first, u_last, me, rank, half, ew, lane);
        }
        if constexpr (SPLIT3) {
            if (g.ra != nullptr && __any_sync(0xffffffffu, inf_tile))
                nonfinite_fixup_tmem<kChunks>(g, tbase, tc.b, row, row_ok,
                                              tc.tn * BN + half * kHalf);
        }
        // Two register sets: the next chunk's TMEM load is in flight while this one is used.
        uint32_t ra[kEpiCols], rb[kEpiCols];
        tmem_ld_issue_32x32b_x16(tbase, ra);
        tmem_ld_wait();
        // Chunk pairs, the pair's two chunks unrolled (each with its own register set). With
        // eight epilogue warps two copies of the chunk code instead of kChunks keep the epilogue
        // within the instruction cache; the four-warp ATMEM epilogue, at its register limit,
        // keeps every chunk unrolled.
        constexpr int kPairUnroll = ATMEM ? kChunks / 2 : 1;
#pragma unroll kPairUnroll
        for (int cp = 0; cp < kChunks; cp += 2) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int ci = cp + h;
            uint32_t (&r)[kEpiCols] = h ? rb : ra;
            uint32_t (&rn)[kEpiCols] = h ? ra : rb;
            if (ci + 1 < kChunks) tmem_ld_issue_32x32b_x16(tbase + (ci + 1) * kEpiCols, rn);
            const int col0 = col_w + ci * kEpiCols;
            if (col0 < g.n && row0 < g.m) {
                if (pre_cin) {
                    // this chunk's C_in goes to `box` (unless fetched already), the next chunk's
                    // to the other box once the store issued from it has read it
                    if (!cin_ahead) {
                        if (lane == 0) bulk_wait_read<0>();
                        __syncwarp();
                        cin_fetch(e, box0 + box * C::kEpiBoxBytes, col0, g.n, lane);
                        cin_ahead = true;
                    }
                    if (ci + 1 < kChunks) {
                        if (lane == 0) bulk_wait_read<0>();
                        __syncwarp();
                        cin_fetch(e, box0 + (box ^ 1) * C::kEpiBoxBytes, col0 + kEpiCols, g.n,
                                  lane);
                        cp_async_wait<1>();
                    } else {
                        cp_async_wait<0>();
                    }
                    e.cin_pre = true;
                    e.cin_smem = box0 + box * C::kEpiBoxBytes + lane * (kEpiCols * 4);
                }
                float v[kEpiCols];
                if (plain) {
#pragma unroll
                    for (int j = 0; j < kEpiCols; ++j) {
                        const float x = __uint_as_float(r[j]);
                        v[j] = g.alpha == 1.0f ? x : __fmul_rn(g.alpha, x);
                    }
                } else {
                    e.chunk = ci;
                    epilogue_general(g, e, col0, r, v);
                }
                if (g.tma_store) {
                    const uint32_t buf = box0 + box * C::kEpiBoxBytes;
                    if (lane == 0) bulk_wait_read<1>();  // the store issued from this box has read it
                    __syncwarp();
                    // row `lane` of the box: four 16-byte chunks, chunk q at q ^ ((lane >> 1) & 3)
#pragma unroll
                    for (int q = 0; q < kEpiCols / 4; ++q) {
                        st_shared_v4(buf + lane * (kEpiCols * 4) + ((q ^ ((lane >> 1) & 3)) << 4),
                                     v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
                    }
                    fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0) {
                        tma_store_3d(tmC, epi_smem + (buf - smem_u32(epi_smem)), col0, row0, tc.b);
                        bulk_commit();
                    }
                    box ^= 1;
                } else if (g.c_peer) {
                    // stage the chunk (box ci & 1); the pair is written below as 128-byte rows
                    const uint32_t buf = box0 + h * C::kEpiBoxBytes;
#pragma unroll
                    for (int q = 0; q < kEpiCols / 4; ++q) {
                        st_shared_v4(buf + lane * (kEpiCols * 4) + ((q ^ ((lane >> 1) & 3)) << 4),
                                     v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
                    }
                } else if (row_ok) {
                    if (col0 + kEpiCols <= g.n && vec_out) {
#pragma unroll
                        for (int j = 0; j < kEpiCols; j += 4) {
                            *reinterpret_cast<float4*>(crow + col0 + j) =
                                make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
                        }
                    } else {
#pragma unroll
                        for (int j = 0; j < kEpiCols; ++j) {
                            if (col0 + j < g.n) crow[col0 + j] = v[j];
                        }
                    }
                }
            }
            if (g.c_peer && h == 1) {
                // C in another GPU's memory: every request crosses NVLink, so the two staged
                // chunks (32 columns) go out as full 128-byte row segments — eight lanes per row,
                // four rows per store instruction — instead of one 16-byte piece per lane.
                const int pair0 = col0 - kEpiCols;
                __syncwarp();
                if (pair0 < g.n && row0 < g.m) {
                    const int c4 = lane & 7;
#pragma unroll
                    for (int it = 0; it < 8; ++it) {
                        const int r = it * 4 + (lane >> 3);
                        const int q = c4 & 3;
                        const float4 val = ld_shared_v4(box0 + (c4 >> 2) * C::kEpiBoxBytes +
                                                        r * (kEpiCols * 4) +
                                                        ((q ^ ((r >> 1) & 3)) << 4));
                        const int grow = row0 + r;
                        const int gcol = pair0 + c4 * 4;
                        if (grow < g.m) {
                            float* dst = g.c + static_cast<long long>(tc.b) * g.c_bs +
                                         static_cast<long long>(grow) * g.ldc + gcol;
                            if (gcol + 4 <= g.n && vec_out) {
                                *reinterpret_cast<float4*>(dst) = val;
                            } else {
                                const float e4[4] = {val.x, val.y, val.z, val.w};
#pragma unroll
                                for (int j = 0; j < 4; ++j) {
                                    if (gcol + j < g.n) dst[j] = e4[j];
                                }
                            }
                        }
                    }
                }
                __syncwarp();
            }
            if (ci + 1 < kChunks) tmem_ld_wait();
        }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
            if constexpr (CG == 1) {
                mbar_arrive(&acc_empty[acc]);
            } else {
                mbar_arrive_cluster(mapa_shared(&acc_empty[acc], 0));  // the MMA issuer's CTA
            }
        }
        if (++acc == C::kAccStages) {
            acc = 0;
            acc_phase ^= 1u;
        }
    }
    // Stores must have finished reading shared memory (and landed) before the CTA exits, and so
    // must C_in copies still in flight (a loop left early, after a wait gave up).
    if (g.tma_store && lane == 0) bulk_wait<0>();
    if constexpr (CINA) cp_async_wait<0>();
    // Stores into a peer GPU's memory are performed at system scope before the kernel ends, so
    // whatever the other GPU orders after this kernel (an event wait, a collective) sees them.
    if (g.c_peer) __threadfence_system();
    __syncwarp();
}

template <int CG, int BN, bool SPLIT3, bool ASPLIT, bool ATMEM = false, bool CINA = false>
__global__ void __launch_bounds__(TcConfig<CG, BN, SPLIT3, ATMEM>::kThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA0,
                   const __grid_constant__ CUtensorMap tmA1,
                   const __grid_constant__ CUtensorMap tmB0,
                   const __grid_constant__ CUtensorMap tmB1,
                   const __grid_constant__ CUtensorMap tmC, const GemmArgs g) {
    using C = TcConfig<CG, BN, SPLIT3, ATMEM>;
    static_assert(!ATMEM || ASPLIT, "the TMEM split is a form of the in-kernel split");
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* stages = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    uint8_t* epi_smem = stages + C::kStages * C::kStageBytes;  // 1024-aligned
    uint64_t* bars = reinterpret_cast<uint64_t*>(epi_smem + C::kEpiBytes);
    uint64_t* full = bars;
    uint64_t* empty = full + C::kStages;
    uint64_t* acc_full = empty + C::kStages;
    uint64_t* acc_empty = acc_full + C::kAccStages;
    uint64_t* drain = acc_empty + C::kAccStages;
    uint64_t* a_full = drain + 1;                // ASPLIT: raw A landed in this CTA
    // ASPLIT: both CTAs' A split (first CTA's barrier; per stage, or per TMEM slot for ATMEM)
    uint64_t* converted = a_full + C::kStages;
    uint64_t* tempty = converted + C::kStages;   // ATMEM: the MMAs reading a TMEM slot are done
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(tempty + (ATMEM ? C::kASlots : 0));
    uint32_t* inf_seen = tmem_holder + 1;        // ASPLIT: the converters met an infinity in A
    static_assert((3 * C::kStages + 2 * C::kAccStages + 1 + C::kASlots) * 8 + 8 <=
                      C::kBarrierBytes,
                  "barrier area too small");

    const int warp = threadIdx.x / 32;
    const int lane = threadIdx.x % 32;
    const uint32_t rank = CG == 1 ? 0u : cluster_ctarank();

    if (threadIdx.x == 0) {
        for (int s = 0; s < C::kStages; ++s) {
            mbar_init(&full[s], 1);
            // ATMEM: the MMAs' commit (B read) and this CTA's four converter warps (A read)
            mbar_init(&empty[s], ATMEM ? 5 : 1);
        }
        for (int s = 0; s < C::kAccStages; ++s) {
            mbar_init(&acc_full[s], 1);
            mbar_init(&acc_empty[s], C::kEpiWarpsC * CG);  // every epilogue warp of the pair
        }
        mbar_init(drain, 1);
        *inf_seen = 0u;
        if constexpr (ATMEM) {
            for (int s = 0; s < C::kStages; ++s) mbar_init(&a_full[s], 1);
            for (int s = 0; s < C::kASlots; ++s) {
                mbar_init(&converted[s], 4 * CG);  // the four converter warps of every CTA
                mbar_init(&tempty[s], 1);
            }
        } else if constexpr (ASPLIT) {
            for (int s = 0; s < C::kStages; ++s) {
                mbar_init(&a_full[s], 1);
                mbar_init(&converted[s], 2 * CG);  // both converter warps of every CTA
            }
        }
        fence_barrier_init();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&tmA0);
        tma_prefetch_desc(&tmB0);
        if constexpr (SPLIT3) {
            tma_prefetch_desc(&tmA1);
            tma_prefetch_desc(&tmB1);
        }
        if (g.tma_store) tma_prefetch_desc(&tmC);
    }
    if (warp == 1) {
        if constexpr (CG == 1) {
            tmem_alloc(tmem_holder, C::kTmemCols);
        } else {
            tmem_alloc_cg2(tmem_holder, C::kTmemCols);
        }
    }
    tc_fence_before();
    __syncthreads();
    if constexpr (CG == 2) cluster_sync();  // peer barriers initialised before any remote use
    tc_fence_after();
    const uint32_t tmem_base = *tmem_holder;

    if (warp == 0) {
        if (lane == 0)
            tc_producer<CG, BN, SPLIT3, ASPLIT, ATMEM>(g, &tmA0, &tmA1, &tmB0, &tmB1, stages, full,
                                                       empty, a_full, rank);
    } else if (warp == 1) {
        if (lane == 0 && rank == 0) {
            tc_mma<CG, BN, SPLIT3, ASPLIT, ATMEM>(g, tmem_base, stages, full, empty, acc_full,
                                                  acc_empty, converted, tempty);
            // Every MMA issued above must finish before TMEM is released, also on an error exit.
            if constexpr (CG == 1) {
                mma_commit(drain);
            } else {
                mma_commit_cg2(drain);
            }
            mbar_wait(drain, 0, kErrMmaWait);
        }
        __syncwarp();
    } else if (ATMEM && ((warp >= kTmCvtWarp0 && warp < kTmCvtWarp0 + 4) || warp >= kTmCvtWarp1)) {
        if constexpr (ATMEM) {
            tc_convert_tmem<CG, BN>(g, stages, a_full, empty, converted, tempty, tmem_base,
                                    warp >= kTmCvtWarp1 ? 1 : 0, inf_seen);
        }
    } else if (!ATMEM && ASPLIT && warp >= kCvtWarp0 && warp < kCvtWarp0 + kCvtThreads / 32) {
        tc_convert<CG, BN, SPLIT3>(g, stages, a_full, converted, inf_seen);
    } else if (warp >= C::kEpiWarp0C && warp < C::kEpiWarp0C + C::kEpiWarpsC) {
        tc_epilogue<CG, BN, SPLIT3, ATMEM, CINA>(g, &tmC, epi_smem, tmem_base, acc_full, acc_empty,
                                           rank, inf_seen);
    }

    tc_fence_before();
    __syncthreads();
    if constexpr (CG == 2) cluster_sync();  // no CTA leaves while its peer may still signal it
    if (warp == 1) {
        tc_fence_after();
        if constexpr (CG == 1) {
            tmem_dealloc(tmem_base, C::kTmemCols);
        } else {
            tmem_dealloc_cg2(tmem_base, C::kTmemCols);
        }
    }
}

}  // namespace mfk
