// The C ABI declared in include/mfk.h: argument checks, operand staging decisions, TMA tensor
// maps, the stream-ordered workspace and the kernel launches. One translation unit holds every
// kernel of the library (the device error word is shared without relocatable device code).
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <atomic>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <new>
#include <string>
#include <type_traits>
#include <vector>

#include "mfk.h"

#include "attn_tc.cuh"
#include "blas1.cuh"
#include "gemm_tc.cuh"
#include "movement.cuh"
#include "prep.cuh"
#include "simt.cuh"

// A B operand split once (mfk_pack_b_f32): op(B) as K-major panels [n][kp] of tf32 values, hi
// and (3xTF32) lo, in device memory the handle owns.
struct mfk_packed_b {
    float* hi = nullptr;
    float* lo = nullptr;
    int64_t k = 0, n = 0, kp = 0;
    int32_t precision = MFK_PRECISION_3XTF32;
    int device = 0;
    unsigned* inf_word = nullptr;  // 3xTF32: 1 when the packing pass met an infinity in B
    bool pooled = false;           // hi came from the stream-ordered pool (cudaMallocAsync)
};

namespace {

using mfk::GemmArgs;

// Scratch of mfk_gemm_f32_noalloc: one fixed array per device, held for the life of the process.
// Host code must not take its address directly (that is a host-side stand-in); the device
// address comes from cudaGetSymbolAddress, once per device (DeviceInfo::noalloc_scratch).
static __device__ __align__(256) unsigned char g_noalloc_scratch[MFK_NOALLOC_SCRATCH_BYTES];

// Where the wait self-test kernel reports whether its wait gave up.
static __device__ unsigned int g_selftest_flag;

// A caller-fixed workspace used instead of the stream-ordered allocator.
struct FixedScratch {
    uint8_t* ptr;
    size_t bytes;
};

thread_local std::string t_cuda_error;
std::atomic<int> g_default_precision{MFK_PRECISION_3XTF32};

constexpr int kMaxDevices = 64;

std::atomic<int64_t> g_launches{0};

// Tags for the packing passes' infinity flag, one per GEMM call, never 0 (fresh memory reads 0).
std::atomic<unsigned> g_inf_tag{0};
unsigned next_inf_tag() {
    unsigned t = g_inf_tag.fetch_add(1) + 1;
    return t != 0 ? t : g_inf_tag.fetch_add(1) + 1;
}

// Optional CUDA-event pairs around the main kernel launch of each call (mfk_kernel_timer).
struct KernelTimer {
    std::mutex mu;
    bool enabled = false;
    std::vector<std::pair<cudaEvent_t, cudaEvent_t>> pending;
    std::vector<std::pair<cudaEvent_t, cudaEvent_t>> spare;
} g_timer;

struct TimedLaunch {
    cudaEvent_t stop = nullptr;
    cudaStream_t stream;
    explicit TimedLaunch(cudaStream_t s) : stream(s) {
        std::lock_guard<std::mutex> lock(g_timer.mu);
        if (!g_timer.enabled) return;
        std::pair<cudaEvent_t, cudaEvent_t> ev{nullptr, nullptr};
        if (!g_timer.spare.empty()) {
            ev = g_timer.spare.back();
            g_timer.spare.pop_back();
        } else if (cudaEventCreate(&ev.first) != cudaSuccess ||
                   cudaEventCreate(&ev.second) != cudaSuccess) {
            return;
        }
        cudaEventRecord(ev.first, stream);
        g_timer.pending.push_back(ev);
        stop = ev.second;
    }
    ~TimedLaunch() {
        if (stop != nullptr) cudaEventRecord(stop, stream);
    }
};

int cuda_fail(cudaError_t e, const char* what) {
    t_cuda_error = std::string(what) + ": " + cudaGetErrorString(e);
    if (e == cudaErrorMemoryAllocation) return MFK_ERR_OUT_OF_MEMORY;
    return MFK_ERR_CUDA;
}

#define MFK_CUDA(call)                                      \
    do {                                                    \
        const cudaError_t e_ = (call);                      \
        if (e_ != cudaSuccess) return cuda_fail(e_, #call); \
    } while (0)

struct DeviceInfo {
    bool ready = false;
    int sm_count = 0;
    int major = 0, minor = 0;
    bool smem_set[16] = {};
    int resident_units[16] = {};  // CTAs (CG = 1) or clusters (CG = 2) resident at once
    void* noalloc_scratch = nullptr;  // device address of g_noalloc_scratch on this device
    // Whether tcgen05 kind::tf32 reads an fp32 operand by truncating it to tf32 (measured once
    // per device by a known-answer GEMM; until known, 3xTF32 splits hi explicitly).
    std::atomic<int> tf32_truncates{-1};  // -1 unknown, 0 no, 1 yes
};

std::mutex g_mutex;
DeviceInfo g_devices[kMaxDevices];

int current_device(int* dev, DeviceInfo** info) {
    MFK_CUDA(cudaGetDevice(dev));
    if (*dev < 0 || *dev >= kMaxDevices) return MFK_ERR_UNSUPPORTED;
    std::lock_guard<std::mutex> lock(g_mutex);
    DeviceInfo& d = g_devices[*dev];
    if (!d.ready) {
        MFK_CUDA(cudaDeviceGetAttribute(&d.sm_count, cudaDevAttrMultiProcessorCount, *dev));
        MFK_CUDA(cudaDeviceGetAttribute(&d.major, cudaDevAttrComputeCapabilityMajor, *dev));
        MFK_CUDA(cudaDeviceGetAttribute(&d.minor, cudaDevAttrComputeCapabilityMinor, *dev));
        // Stream-ordered workspace: keep freed blocks in the pool instead of returning them to
        // the driver after every call.
        cudaMemPool_t pool;
        if (cudaDeviceGetDefaultMemPool(&pool, *dev) == cudaSuccess) {
            uint64_t threshold = UINT64_MAX;
            cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &threshold);
        }
        d.ready = true;
    }
    *info = &d;
    if (d.major != 10) return MFK_ERR_NO_DEVICE;  // sm_100a code only
    return MFK_OK;
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) !=
                cudaSuccess ||
            q != cudaDriverEntryPointSuccess) {
            return static_cast<PFN_cuTensorMapEncodeTiled_v12000>(nullptr);
        }
        return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }();
    return fn;
}

// A K-major operand view for TMA: `rows` rows of `depth` fp32 values, row r of matrix z at
// base + z*bstride + r*rstride (elements). Box: 32 values (128 B, SWIZZLE_128B) x box_rows.
bool make_kmajor_map(CUtensorMap* map, const float* base, int64_t depth, int64_t rows,
                     int64_t nmat, int64_t rstride, int64_t bstride, int box_rows,
                     CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B) {
    auto fn = encode_fn();
    if (fn == nullptr) return false;
    if (nmat == 1) bstride = rstride * std::max<int64_t>(rows, 1);
    cuuint64_t dims[3] = {static_cast<cuuint64_t>(depth), static_cast<cuuint64_t>(rows),
                          static_cast<cuuint64_t>(nmat)};
    cuuint64_t strides[2] = {static_cast<cuuint64_t>(rstride) * 4,
                             static_cast<cuuint64_t>(bstride) * 4};
    cuuint32_t box[3] = {32, static_cast<cuuint32_t>(box_rows), 1};
    cuuint32_t estr[3] = {1, 1, 1};
    const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3,
                          const_cast<float*>(base), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

// The output C as a TMA store target: n columns x m rows x nmat matrices, row stride ldc, matrix
// stride c_bs (elements), boxes of 16 columns x 32 rows with the 64-byte swizzle the epilogue
// stages in.
bool make_store_map(CUtensorMap* map, float* c, int64_t n, int64_t m, int64_t nmat, int64_t ldc,
                    int64_t c_bs) {
    auto fn = encode_fn();
    if (fn == nullptr) return false;
    if (nmat == 1) c_bs = ldc * std::max<int64_t>(m, 1);
    cuuint64_t dims[3] = {static_cast<cuuint64_t>(n), static_cast<cuuint64_t>(m),
                          static_cast<cuuint64_t>(nmat)};
    cuuint64_t strides[2] = {static_cast<cuuint64_t>(ldc) * 4, static_cast<cuuint64_t>(c_bs) * 4};
    cuuint32_t box[3] = {static_cast<cuuint32_t>(mfk::kEpiCols), 32, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, c, dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B,
              CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Batch placement of one operand: matrix z starts at shift + z*stride elements, or at
// offsets[z] when the caller's offsets are not evenly spaced.
struct BatchLayout {
    const int64_t* offsets = nullptr;  // host, uneven spacing only
    int64_t shift = 0;
    int64_t stride = 0;
};

BatchLayout batch_layout(const int64_t* offsets, int64_t stride, int64_t batch) {
    BatchLayout l;
    if (offsets == nullptr) {
        l.stride = stride;
        return l;
    }
    l.shift = offsets[0];
    l.stride = batch > 1 ? offsets[1] - offsets[0] : 0;
    for (int64_t i = 1; i < batch; ++i) {
        if (offsets[i] - offsets[i - 1] != l.stride) {
            l.offsets = offsets;
            l.shift = 0;
            l.stride = 0;
            break;
        }
    }
    return l;
}

// One GEMM operand as K-major rows: row r (of R), depth p (of K) at
// ptr + off(z) + r*rs + p*cs.
struct Operand {
    const float* ptr;
    int64_t rs, cs;
    int64_t rows;
    BatchLayout bl;
    bool direct = false;      // TMA reads the caller's memory
    float* hi = nullptr;      // packed copies (workspace)
    float* lo = nullptr;
    int64_t* dev_offsets = nullptr;
};

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Whether TMA can read the operand where it lies: K-major, 16-byte aligned rows and matrices.
bool tma_readable(const Operand& o, int64_t k) {
    if (o.cs != 1 || o.bl.offsets != nullptr) return false;
    if (!aligned16(o.ptr) || o.rs <= 0 || (o.rs % 4) != 0 || o.rs < k) return false;
    if (o.bl.stride < 0 || (o.bl.stride % 4) != 0) return false;
    if (o.rs >= (int64_t(1) << 37) || o.bl.stride >= (int64_t(1) << 37)) return false;
    return true;
}

// 1xTF32 reads a readable operand in place. 3xTF32 needs it split: the pre-pass costs 12 bytes of
// HBM traffic per element and a launch, the in-kernel split of A (converter warps, only lo written
// where the tensor cores truncate) costs issue slots and shared-memory bandwidth on every N-tile
// of the product, off the MMA's critical path. With the bit-arithmetic rounding and CTA-scope
// arrives the in-kernel split of A wins at every width measured on B200 (pre-pass -> in-kernel):
// C2 8192^3 3.89 -> 3.74 ms, 8192 x 4096 x 8192 2.25 -> 2.03 ms, 8192 x 1024 x 8192 0.64 -> 0.50
// ms, C3's 4096 x 1024 x 4096 0.21 -> 0.17 ms, C4's S = QK^T 0.77 -> 0.73 ms per 128 heads (the
// first build, with cvt.rna rounding and cluster-scope arrives, lost above N ~ 360). So A is split
// in the kernel whenever TMA can read it where it lies; B, and an A it cannot read, are packed.
constexpr int64_t kInKernelSplitMaxN = INT64_MAX;

// The C_in-ahead epilogue (see run_gemm) for K up to this many k-blocks, counted three times in
// 3xTF32: K <= 256 in 3xTF32, K <= 768 in 1xTF32.
constexpr int kCinAheadMaxKBlocks = 24;



// One kernel instantiation per (CG, BN, SPLIT3, ASPLIT, ATMEM, CINA); `slot` indexes its
// per-device set-up flags.
template <int CG, int BN, bool SPLIT3, bool ASPLIT, bool ATMEM = false, bool CINA = false>
int launch_tc(const CUtensorMap& a0, const CUtensorMap& a1, const CUtensorMap& b0,
              const CUtensorMap& b1, const CUtensorMap& cmap, const GemmArgs& g_in,
              DeviceInfo* info, int slot, cudaStream_t stream, bool allow_sk) {
    GemmArgs g = g_in;
    using C = mfk::TcConfig<CG, BN, SPLIT3, ATMEM>;
    auto kernel = mfk::gemm_tc_kernel<CG, BN, SPLIT3, ASPLIT, ATMEM, CINA>;
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    cfg.blockDim = dim3(C::kThreads, 1, 1);
    cfg.dynamicSmemBytes = C::kSmemBytes;
    cfg.stream = stream;
    if (CG > 1) {
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = CG;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
    }
    {
        std::lock_guard<std::mutex> lock(g_mutex);
        if (!info->smem_set[slot]) {
            MFK_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          C::kSmemBytes));
            int units = info->sm_count / CG;
            if (CG > 1) {
                cfg.gridDim = dim3(static_cast<unsigned>(info->sm_count / CG * CG), 1, 1);
                int clusters = 0;
                if (cudaOccupancyMaxActiveClusters(&clusters, kernel, &cfg) == cudaSuccess &&
                    clusters > 0) {
                    units = clusters;
                }
                cudaGetLastError();
            }
            info->resident_units[slot] = units;
            info->smem_set[slot] = true;
        }
    }
    const long long resident = info->resident_units[slot];
    long long units = std::min<long long>(g.num_tiles, resident);
    // Stream-K tail: when the last wave of tiles would leave many units idle (under 92% of the
    // units busy on average), the tiles of that wave are shared by k-iterations across every
    // unit instead. Each extra part of a tile costs one round trip of a kBM x BN accumulator
    // through L2, so the share per unit must be at least four k-blocks. No part waits for
    // another (the last part counted sums them), so GEMMs running at once on several streams
    // cannot hold each other up. Measured on B200 (kernel time, off -> on), it pays in 3xTF32
    // when whole waves come first, so the summing of split tiles overlaps their MMAs (4096 x 4096
    // x 1024: 129 -> 124 us), or when the tiles fill at most half the units (100 x 1000 x 4096:
    // 98 -> 53 us; 1024 x 300 x 2048: 66 -> 46 us), and not otherwise: with every SM streaming
    // tf32 operands 1xTF32 is short of L2 bandwidth (4096 x 1024 x 4096: 53 -> 63 us), and a tail
    // that is the whole problem leaves the summing exposed (138 -> 145 us).
    struct SkWorkspace {
        void* p = nullptr;
        cudaStream_t s;
        ~SkWorkspace() {
            if (p) cudaFreeAsync(p, s);
        }
    } sk{nullptr, stream};
    if (allow_sk && resident > 0 && g.num_tiles % resident != 0 && g.num_tiles < 16 * resident) {
        const long long waves = g.num_tiles / resident;
        const long long rem = g.num_tiles % resident;
        const double busy = static_cast<double>(g.num_tiles) /
                            static_cast<double>((waves + 1) * resident);
        const long long iters = rem * g.num_kb;
        if (SPLIT3 && busy < 0.92 && iters >= 4 * resident &&
            (waves >= 1 || 2 * g.num_tiles <= resident)) {
            const size_t part_bytes =
                static_cast<size_t>(resident) * 2 * CG * mfk::kBM * BN * sizeof(float);
            const size_t count_bytes = static_cast<size_t>(rem) * CG * C::kEpiWarpsC * sizeof(int);
            MFK_CUDA(cudaMallocAsync(&sk.p, part_bytes + count_bytes, stream));
            MFK_CUDA(cudaMemsetAsync(static_cast<uint8_t*>(sk.p) + part_bytes, 0, count_bytes,
                                     stream));
            g.sk_units = static_cast<int>(resident);
            g.dp_tiles = waves * resident;
            g.sk_q = iters / resident;
            g.sk_r = static_cast<int>(iters % resident);
            g.sk_part = static_cast<float*>(sk.p);
            g.sk_count = reinterpret_cast<int*>(static_cast<uint8_t*>(sk.p) + part_bytes);
            units = resident;
        }
    }
    cfg.gridDim = dim3(static_cast<unsigned>(units * CG), 1, 1);
    {
        TimedLaunch timed(stream);
        MFK_CUDA(cudaLaunchKernelEx(&cfg, kernel, a0, a1, b0, b1, cmap, g));
    }
    g_launches.fetch_add(1);
    return MFK_OK;
}

// Writes op(X) of operand `o` as K-major panels [batch][rows][Kp] into o.hi (and o.lo for the
// 3xTF32 split), zero in the columns k..Kp-1. o.dev_offsets must hold the per-matrix offsets on
// the device when o.bl.offsets is set.
int launch_pack(const Operand& o, int64_t k, int64_t Kp, int64_t batch, int mode,
                const DeviceInfo* info, cudaStream_t stream, unsigned* inf_word = nullptr,
                unsigned inf_tag = 0) {
    if (mode != mfk::kPackSplit) inf_word = nullptr;
    if (o.cs == 1 && o.rs % 4 == 0 && k % 4 == 0 && aligned16(o.ptr) &&
        (o.dev_offsets != nullptr || o.bl.stride % 4 == 0)) {
        // already K-major and aligned: a straight vectorised pass
        bool offs_aligned = true;
        if (o.bl.offsets) {
            for (int64_t i = 0; i < batch && offs_aligned; ++i) offs_aligned = o.bl.offsets[i] % 4 == 0;
        }
        if (offs_aligned) {
            // one warp per row (the block scheduler balances them), a grid stride beyond 32
            // blocks per SM
            const int64_t rows = o.rows * batch;
            const int64_t warps_per_block = mfk::kPackThreads / 32;
            const int64_t blocks = std::min<int64_t>((rows + warps_per_block - 1) / warps_per_block,
                                                     static_cast<int64_t>(info->sm_count) * 32);
            mfk::pack_kmajor_vec4_kernel<<<static_cast<unsigned>(blocks), mfk::kPackThreads, 0,
                                           stream>>>(
                o.ptr, reinterpret_cast<const long long*>(o.dev_offsets), o.bl.stride, o.rs,
                static_cast<int>(o.rows), static_cast<int>(k), static_cast<int>(Kp),
                static_cast<int>(batch), o.hi, o.lo, mode, inf_word, inf_tag);
            g_launches.fetch_add(1);
            MFK_CUDA(cudaGetLastError());
            return MFK_OK;
        }
    }
    const int p_contig = (o.cs == 1) || (o.rs != 1 && std::llabs(o.cs) <= std::llabs(o.rs));
    if (!p_contig) {
        // rows run along memory: 64 x 64 tiles turned through shared memory, one per block
        // where the grid allows
        const int64_t tiles = (o.rows + mfk::kPackTile - 1) / mfk::kPackTile *
                              ((Kp + mfk::kPackTile - 1) / mfk::kPackTile) * batch;
        const int64_t blocks = std::min<int64_t>(tiles, static_cast<int64_t>(info->sm_count) * 32);
        mfk::pack_transpose_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(
            o.ptr, reinterpret_cast<const long long*>(o.dev_offsets), o.bl.stride, o.rs, o.cs,
            static_cast<int>(o.rows), static_cast<int>(k), static_cast<int>(Kp),
            static_cast<int>(batch), o.hi, o.lo, mode, inf_word, inf_tag);
        g_launches.fetch_add(1);
        MFK_CUDA(cudaGetLastError());
        return MFK_OK;
    }
    if (o.rows > 65535LL * 32) return MFK_ERR_UNSUPPORTED;
    for (int64_t z0 = 0; z0 < batch; z0 += 65535) {
        const int64_t nz = std::min<int64_t>(65535, batch - z0);
        dim3 grid(static_cast<unsigned>(Kp / 32), static_cast<unsigned>((o.rows + 31) / 32),
                  static_cast<unsigned>(nz));
        const long long* offs =
            o.dev_offsets ? reinterpret_cast<const long long*>(o.dev_offsets) + z0 : nullptr;
        const float* src = o.dev_offsets ? o.ptr : o.ptr + z0 * o.bl.stride;
        const int64_t out_shift = z0 * o.rows * Kp;
        mfk::pack_kmajor_kernel<<<grid, dim3(32, 8), 0, stream>>>(
            src, offs, o.bl.stride, o.rs, o.cs, static_cast<int>(o.rows),
            static_cast<int>(k), static_cast<int>(Kp), o.hi + out_shift,
            o.lo ? o.lo + out_shift : nullptr, mode, p_contig, inf_word, inf_tag);
        g_launches.fetch_add(1);
        MFK_CUDA(cudaGetLastError());
    }
    return MFK_OK;
}

// Where C lies, as the caller states it: kCOutputInfer looks at the pointer's attributes (a
// device pointer of another GPU is peer memory), kCOutputPeer is certain that C is another
// GPU's memory (a peer buffer or a CUDA IPC mapping of one, whose reported device need not be the
// owner): then no tensor map ever covers C, whatever its attributes say.
enum COutput { kCOutputInfer = 0, kCOutputPeer = 1 };

int run_gemm(const mfk_gemm_desc* d, const mfk_batch_desc* bd, cudaStream_t stream,
             const FixedScratch* fixed, const mfk_packed_b* pb = nullptr,
             COutput c_where = kCOutputInfer);

// Known answer: 1xTF32 reads A in place; a = 1 + 3*2^-12 holds 0.75 ulp of tf32 beyond 1, so
// a * 1 is 1 when the tensor cores truncate fp32 operands and 1 + 2^-10 when they round. Runs
// once per device, on a private stream, only where allocating is allowed and the caller's
// stream is not being captured; any failure leaves the explicit (always valid) split in use.
bool tf32_truncates(DeviceInfo* info, cudaStream_t caller, bool may_allocate) {
    // MFK_EXPLICIT_SPLIT set (and not "0"): always write the split's hi part explicitly, as on
    // tensor cores that round, so that path can be checked on hardware that truncates.
    static const bool explicit_split = [] {
        const char* e = std::getenv("MFK_EXPLICIT_SPLIT");
        return e != nullptr && e[0] != '\0' && !(e[0] == '0' && e[1] == '\0');
    }();
    if (explicit_split) return false;
    const int known = info->tf32_truncates.load();
    if (known >= 0) return known == 1;
    if (!may_allocate) return false;
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(caller, &cap) != cudaSuccess || cap != cudaStreamCaptureStatusNone) {
        cudaGetLastError();
        return false;
    }
    float host_a[32] = {}, host_b[32] = {}, host_c = 0.0f;
    host_a[0] = 1.0f + 3.0f * 0x1p-12f;
    host_b[0] = 1.0f;
    float* buf = nullptr;
    cudaStream_t s = nullptr;
    int verdict = 0;
    if (cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking) == cudaSuccess &&
        cudaMalloc(&buf, 4 * 96) == cudaSuccess &&
        cudaMemcpyAsync(buf, host_a, sizeof(host_a), cudaMemcpyHostToDevice, s) == cudaSuccess &&
        cudaMemcpyAsync(buf + 32, host_b, sizeof(host_b), cudaMemcpyHostToDevice, s) ==
            cudaSuccess) {
        mfk_gemm_desc d{};
        d.a = buf;                // A [1, 32], row-major, read in place
        d.a_rs = 32;
        d.a_cs = 1;
        d.b = buf + 32;           // B [32, 1]
        d.b_rs = 1;
        d.b_cs = 1;
        d.c = buf + 64;
        d.ldc = 1;
        d.m = 1;
        d.n = 1;
        d.k = 32;
        d.alpha = 1.0f;
        d.precision = MFK_PRECISION_1XTF32;
        if (run_gemm(&d, nullptr, s, nullptr) == MFK_OK &&
            cudaMemcpyAsync(&host_c, buf + 64, 4, cudaMemcpyDeviceToHost, s) == cudaSuccess &&
            cudaStreamSynchronize(s) == cudaSuccess) {
            verdict = host_c == 1.0f ? 1 : 0;
        }
    }
    if (buf != nullptr) cudaFree(buf);
    if (s != nullptr) cudaStreamDestroy(s);
    cudaGetLastError();
    info->tf32_truncates.store(verdict);
    return verdict == 1;
}

int check_desc(const mfk_gemm_desc* d) {
    if (d == nullptr) return MFK_ERR_INVALID_ARGUMENT;
    if (d->m < 0 || d->n < 0 || d->k < 0) return MFK_ERR_INVALID_ARGUMENT;
    if (d->activation < MFK_ACT_NONE || d->activation > MFK_ACT_GELU_TANH)
        return MFK_ERR_INVALID_ARGUMENT;
    if (d->precision < MFK_PRECISION_DEFAULT || d->precision > MFK_PRECISION_1XTF32)
        return MFK_ERR_INVALID_ARGUMENT;
    if (d->m > 0 && d->n > 0) {
        if (d->c == nullptr || d->ldc < d->n) return MFK_ERR_INVALID_ARGUMENT;
        if (d->k > 0 && (d->a == nullptr || d->b == nullptr)) return MFK_ERR_INVALID_ARGUMENT;
        if (d->beta != 0.0f && d->c_in == nullptr) return MFK_ERR_INVALID_ARGUMENT;
    }
    return MFK_OK;
}

int run_gemm(const mfk_gemm_desc* d, const mfk_batch_desc* bd, cudaStream_t stream,
             const FixedScratch* fixed, const mfk_packed_b* pb, COutput c_where) {
    int rc = check_desc(d);
    if (rc != MFK_OK) return rc;
    const int64_t batch = bd ? bd->batch : 1;
    if (batch < 0) return MFK_ERR_INVALID_ARGUMENT;
    if (d->m == 0 || d->n == 0 || batch == 0) return MFK_OK;
    if (d->m > (int64_t(1) << 31) - 256 || d->n > (int64_t(1) << 31) - 256 ||
        d->k > (int64_t(1) << 31) - 256 || batch > (int64_t(1) << 31) - 1)
        return MFK_ERR_UNSUPPORTED;

    int dev = 0;
    DeviceInfo* info = nullptr;
    rc = current_device(&dev, &info);
    if (rc != MFK_OK) return rc;

    const int precision = d->precision == MFK_PRECISION_DEFAULT ? g_default_precision.load()
                                                                 : d->precision;
    const bool split3 = precision == MFK_PRECISION_3XTF32;
    if (pb != nullptr) {
        if (pb->k != d->k || pb->n != d->n) return MFK_ERR_INVALID_ARGUMENT;
        if (pb->device != dev) return MFK_ERR_INVALID_ARGUMENT;
        if (split3 && pb->precision != MFK_PRECISION_3XTF32) return MFK_ERR_INVALID_ARGUMENT;
    }
    // The in-kernel split of A may leave hi as the raw fp32 values where the tensor cores are
    // known to truncate them (writing only lo: a third less shared-memory traffic).
    const bool raw_hi = split3 && d->k > 0 && d->n > 128 && d->n <= kInKernelSplitMaxN &&
                        d->m > mfk::kBM && tf32_truncates(info, stream, fixed == nullptr);

    GemmArgs g{};
    g.m = static_cast<int>(d->m);
    g.n = static_cast<int>(d->n);
    g.k = static_cast<int>(d->k);
    g.batch = static_cast<int>(batch);
    g.alpha = d->alpha;
    g.beta = d->beta;
    g.c_in = d->beta != 0.0f ? d->c_in : nullptr;
    g.c_in_rs = d->c_in_rs;
    g.c_in_cs = d->c_in_cs;
    g.c_in_bs = bd ? bd->c_in_stride : 0;
    g.c = d->c;
    g.ldc = d->ldc;
    g.c_bs = bd ? bd->c_stride : 0;
    g.bias = d->bias;
    g.act = d->activation;

    if (d->k == 0) {
        const long long total = static_cast<long long>(batch) * d->m * d->n;
        const long long blocks = std::min<long long>((total + 255) / 256, 65535LL * 8);
        mfk::epilogue_only_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(g);
        g_launches.fetch_add(1);
        MFK_CUDA(cudaGetLastError());
        return MFK_OK;
    }

    // Tile shape: a CTA pair (M = 256 per MMA) unless the problem has a single 128-row tile;
    // N = 256 per MMA unless the output is at most 128 wide.
    const int cg = d->m > mfk::kBM ? 2 : 1;
    const int BN = (cg == 2 && d->n > 128) ? 256 : 128;
    const int b_box_rows = BN / cg;
    const int64_t Kp = (d->k + mfk::kBK - 1) / mfk::kBK * mfk::kBK;

    Operand A{d->a, d->a_rs, d->a_cs, d->m,
              batch_layout(bd ? bd->a_offsets : nullptr, bd ? bd->a_stride : 0, batch)};
    // op(B) element (p, j) at p*b_rs + j*b_cs: as K-major rows over j, rs = b_cs, cs = b_rs.
    Operand B{d->b, d->b_cs, d->b_rs, d->n,
              batch_layout(bd ? bd->b_offsets : nullptr, bd ? bd->b_stride : 0, batch)};
    A.ptr += A.bl.shift;
    B.ptr += B.bl.shift;

    // Direct TMA reads when the layout allows; the maps are encoded now so that a layout the
    // driver rejects falls back to packing instead of failing. In 3xTF32 A is read in place and
    // split inside the kernel; B is packed as an explicitly rounded (hi, lo) pair (a pre-pass
    // writing B's lo only, with raw B as hi, measured ~9% slower on the 8192^3 kernel under the
    // power cap: the 13 low bits left in hi keep toggling through shared memory and the MMA
    // datapath, where rounded hi has them zeroed).
    CUtensorMap ma0, ma1, mb0, mb1;
    auto direct_map = [&](Operand& o, int box_rows, CUtensorMap* m0, CUtensorMap* m1,
                          int* bcast) {
        const bool is_a = &o == &A;
        const bool in_kernel = split3 && is_a && d->n <= kInKernelSplitMaxN;
        if (split3 && !in_kernel) return;
        if (!tma_readable(o, d->k)) return;
        *bcast = (o.bl.stride == 0 && batch > 1) ? 1 : 0;
        const int64_t nmat = *bcast ? 1 : batch;
        if (make_kmajor_map(m0, o.ptr, d->k, o.rows, nmat, o.rs, o.bl.stride, box_rows)) {
            *m1 = *m0;
            o.direct = true;
        } else {
            *bcast = 0;
        }
    };
    direct_map(A, mfk::kBM, &ma0, &ma1, &g.a_batch_bcast);
    if (pb == nullptr) direct_map(B, b_box_rows, &mb0, &mb1, &g.b_batch_bcast);

    // Workspace: packed operands plus device copies of non-arithmetic offset tables.
    const int nops = split3 ? 2 : 1;
    auto packed_elems = [&](const Operand& o) { return o.rows * Kp * batch; };
    auto copies = [&](const Operand& o) {
        return (o.direct || (pb != nullptr && &o == &B)) ? 0 : nops;
    };
    size_t bytes = 0;
    auto reserve = [&](size_t n) {
        const size_t off = bytes;
        bytes += (n + 255) / 256 * 256;
        return off;
    };
    size_t a_off = 0, b_off = 0, ao_off = 0, bo_off = 0;
    if (copies(A)) a_off = reserve(sizeof(float) * packed_elems(A) * copies(A));
    if (copies(B)) b_off = reserve(sizeof(float) * packed_elems(B) * copies(B));
    if (copies(A) && A.bl.offsets) ao_off = reserve(sizeof(int64_t) * batch);
    if (copies(B) && B.bl.offsets) bo_off = reserve(sizeof(int64_t) * batch);
    // The packing passes' infinity flag (3xTF32): set to this call's tag when they meet one. A
    // word left over from an earlier call holds another tag; a chance match only costs the
    // kernel a scan for NaN accumulators.
    const bool inf_flag = split3 && (copies(A) || copies(B));
    const size_t inf_off = inf_flag ? reserve(sizeof(unsigned)) : 0;
    const unsigned inf_tag = inf_flag ? next_inf_tag() : 0;

    uint8_t* ws = nullptr;
    if (bytes > 0 && fixed != nullptr) {
        if (bytes > fixed->bytes) return MFK_ERR_SCRATCH_LIMIT;
        ws = fixed->ptr;
    } else if (bytes > 0) {
        MFK_CUDA(cudaMallocAsync(reinterpret_cast<void**>(&ws), bytes, stream));
    }
    struct Free {
        uint8_t* p;
        cudaStream_t s;
        ~Free() {
            if (p) cudaFreeAsync(p, s);
        }
    } release{fixed != nullptr ? nullptr : ws, stream};

    auto pack = [&](Operand& o, size_t off, size_t offs_off) -> int {
        o.hi = reinterpret_cast<float*>(ws + off);
        o.lo = split3 ? o.hi + packed_elems(o) : nullptr;
        if (o.bl.offsets) {
            o.dev_offsets = reinterpret_cast<int64_t*>(ws + offs_off);
            MFK_CUDA(cudaMemcpyAsync(o.dev_offsets, o.bl.offsets, sizeof(int64_t) * batch,
                                     cudaMemcpyHostToDevice, stream));
        }
        return launch_pack(o, d->k, Kp, batch, split3 ? mfk::kPackSplit : mfk::kPackRound,
                           info, stream, reinterpret_cast<unsigned*>(ws + inf_off), inf_tag);
    };
    if (copies(A) && (rc = pack(A, a_off, ao_off)) != MFK_OK) return rc;
    if (copies(B) && (rc = pack(B, b_off, bo_off)) != MFK_OK) return rc;

    auto packed_maps = [&](const Operand& o, int box_rows, CUtensorMap* m0, CUtensorMap* m1) {
        bool ok = make_kmajor_map(m0, o.hi, Kp, o.rows, batch, Kp, o.rows * Kp, box_rows);
        if (split3) {
            ok = ok && make_kmajor_map(m1, o.lo, Kp, o.rows, batch, Kp, o.rows * Kp, box_rows);
        } else {
            *m1 = *m0;
        }
        return ok;
    };
    if ((copies(A) && !packed_maps(A, mfk::kBM, &ma0, &ma1)) ||
        (copies(B) && !packed_maps(B, b_box_rows, &mb0, &mb1))) {
        t_cuda_error = "cuTensorMapEncodeTiled rejected a packed operand";
        return MFK_ERR_UNSUPPORTED;
    }
    if (pb != nullptr) {
        // the pre-split B, one matrix shared by every batch entry
        bool ok = make_kmajor_map(&mb0, pb->hi, pb->kp, pb->n, 1, pb->kp, pb->n * pb->kp,
                                  b_box_rows);
        if (split3) {
            ok = ok && make_kmajor_map(&mb1, pb->lo, pb->kp, pb->n, 1, pb->kp, pb->n * pb->kp,
                                       b_box_rows);
        } else {
            mb1 = mb0;
        }
        if (!ok) {
            t_cuda_error = "cuTensorMapEncodeTiled rejected a pre-split B";
            return MFK_ERR_UNSUPPORTED;
        }
        g.b_batch_bcast = batch > 1 ? 1 : 0;
    }
    if (split3) {
        // The operands as the kernel reads them, for the exact recomputation of entries an
        // infinity turned into NaN (inf * 0 among the split products).
        if (A.direct) {
            g.ra = A.ptr;
            g.ra_rs = A.rs;
            g.ra_bs = A.bl.stride;
        } else {
            g.ra = A.hi;
            g.ra_rs = Kp;
            g.ra_bs = A.rows * Kp;
        }
        if (pb != nullptr) {
            g.rb = pb->hi;
            g.rb_rs = pb->kp;
            g.rb_bs = 0;
            g.nf_word[1] = pb->inf_word;
            g.nf_tag[1] = 1u;
        } else {
            g.rb = B.hi;
            g.rb_rs = Kp;
            g.rb_bs = B.rows * Kp;
        }
        if (inf_flag) {
            g.nf_word[0] = reinterpret_cast<const unsigned*>(ws + inf_off);
            g.nf_tag[0] = inf_tag;
        }
    }

    g.num_kb = static_cast<int>(Kp / mfk::kBK);
    g.tiles_m = static_cast<int>((d->m + mfk::kBM * cg - 1) / (mfk::kBM * cg));
    g.tiles_n = static_cast<int>((d->n + BN - 1) / BN);
    // Tiles in flight form a group_m x (units / group_m) block; a square block keeps the fewest
    // distinct A and B panels live in L2.
    g.group_m = cg == 2 ? 8 : 12;
    g.num_tiles = static_cast<long long>(batch) * g.tiles_m * g.tiles_n;

    // C through TMA stores when its layout allows (16-byte aligned rows and matrices) and it lies
    // in this GPU's memory. C on another GPU (the gather target of a sharded product, reached over
    // NVLink) is written with plain stores from the epilogue: no tensor map covers peer memory.
    bool c_local = c_where != kCOutputPeer;
    if (c_local) {
        cudaPointerAttributes pa{};
        if (cudaPointerGetAttributes(&pa, d->c) == cudaSuccess) {
            c_local = pa.type != cudaMemoryTypeDevice || pa.device == dev;
        } else {
            cudaGetLastError();
        }
    }
    CUtensorMap mc;
    std::memset(&mc, 0, sizeof(mc));
    const bool c_ok = c_local && aligned16(d->c) && d->ldc % 4 == 0 && (batch == 1 || g.c_bs % 4 == 0) &&
                      d->ldc < (int64_t(1) << 37) && g.c_bs >= 0 && g.c_bs < (int64_t(1) << 37);
    g.tma_store = (c_ok && make_store_map(&mc, d->c, d->n, d->m, batch, d->ldc, g.c_bs)) ? 1 : 0;
    g.c_peer = c_local ? 0 : 1;

    // 3xTF32 with A read in place: the kernel splits A in shared memory.
    const bool asplit = split3 && A.direct;
    g.raw_hi = raw_hi ? 1 : 0;
    // Short K with C_in: the epilogue, not the MMAs, bounds the kernel, and the variant that
    // copies C_in into the staging boxes a chunk ahead pays (8192 x 8192 x 128, beta 1, bias:
    // 215 -> 189 us). Where the MMAs of a tile outlast its epilogue it does not (K = 1024:
    // 521 -> 538 us), so only short K takes it.
    const bool cin_ahead = g.c_in != nullptr && g.tma_store &&
                           g.num_kb * (split3 ? 3 : 1) <= kCinAheadMaxKBlocks;
    if (cg == 2 && BN == 256) {
        if (asplit) {
            return cin_ahead
                ? launch_tc<2, 256, true, true, false, true>(ma0, ma1, mb0, mb1, mc, g, info, 11, stream, fixed == nullptr)
                : launch_tc<2, 256, true, true>(ma0, ma1, mb0, mb1, mc, g, info, 6, stream, fixed == nullptr);
        }
        if (!split3 && cin_ahead)
            return launch_tc<2, 256, false, false, false, true>(ma0, ma1, mb0, mb1, mc, g, info, 12, stream, fixed == nullptr);
        return split3 ? launch_tc<2, 256, true, false>(ma0, ma1, mb0, mb1, mc, g, info, 0, stream, fixed == nullptr)
                      : launch_tc<2, 256, false, false>(ma0, ma1, mb0, mb1, mc, g, info, 1, stream, fixed == nullptr);
    }
    // N <= 128 with A split in place: the split goes to tensor memory (ATMEM), which leaves
    // shared memory to the B tiles and the raw A stages.
    if (cg == 2) {
        if (asplit) {
            return launch_tc<2, 128, true, true, true>(ma0, ma1, mb0, mb1, mc, g, info, 9, stream, fixed == nullptr);
        }
        return split3 ? launch_tc<2, 128, true, false>(ma0, ma1, mb0, mb1, mc, g, info, 2, stream, fixed == nullptr)
                      : launch_tc<2, 128, false, false>(ma0, ma1, mb0, mb1, mc, g, info, 3, stream, fixed == nullptr);
    }
    if (asplit) return launch_tc<1, 128, true, true, true>(ma0, ma1, mb0, mb1, mc, g, info, 10, stream, fixed == nullptr);
    return split3 ? launch_tc<1, 128, true, false>(ma0, ma1, mb0, mb1, mc, g, info, 4, stream, fixed == nullptr)
                  : launch_tc<1, 128, false, false>(ma0, ma1, mb0, mb1, mc, g, info, 5, stream, fixed == nullptr);
}

}  // namespace

extern "C" {

int mfk_gemm_f32(const mfk_gemm_desc* desc, void* stream) {
    return run_gemm(desc, nullptr, static_cast<cudaStream_t>(stream), nullptr);
}

int mfk_gemm_peer_f32(const mfk_gemm_desc* desc, void* stream) {
    return run_gemm(desc, nullptr, static_cast<cudaStream_t>(stream), nullptr, nullptr,
                    kCOutputPeer);
}

int mfk_gemm_f32_noalloc(const mfk_gemm_desc* desc, void* stream) {
    int dev = 0;
    DeviceInfo* info = nullptr;
    const int rc = current_device(&dev, &info);
    if (rc != MFK_OK) return rc;
    FixedScratch scratch{nullptr, MFK_NOALLOC_SCRATCH_BYTES};
    {
        // Set-up, once per device with that device current: the array's device address.
        std::lock_guard<std::mutex> lock(g_mutex);
        if (info->noalloc_scratch == nullptr) {
            void* p = nullptr;
            MFK_CUDA(cudaGetSymbolAddress(&p, g_noalloc_scratch));
            info->noalloc_scratch = p;
        }
        scratch.ptr = static_cast<uint8_t*>(info->noalloc_scratch);
    }
    return run_gemm(desc, nullptr, static_cast<cudaStream_t>(stream), &scratch);
}

int mfk_sharded_gemm_f32(const mfk_gemm_desc* per_rank, int32_t nranks, const int32_t* devices,
                         void* const* streams, int32_t gather, int32_t root, float* gathered,
                         int64_t ld_gathered) {
    if (per_rank == nullptr || devices == nullptr || streams == nullptr || nranks < 1)
        return MFK_ERR_INVALID_ARGUMENT;
    int count = 0;
    MFK_CUDA(cudaGetDeviceCount(&count));
    for (int r = 0; r < nranks; ++r) {
        if (devices[r] < 0 || devices[r] >= count) return MFK_ERR_INVALID_ARGUMENT;
        const int rc = check_desc(&per_rank[r]);
        if (rc != MFK_OK) return rc;
        if (per_rank[r].n != per_rank[0].n) return MFK_ERR_INVALID_ARGUMENT;
    }
    if (gather) {
        if (root < 0 || root >= nranks || gathered == nullptr || ld_gathered < per_rank[0].n)
            return MFK_ERR_INVALID_ARGUMENT;
    }
    int caller_device = 0;
    MFK_CUDA(cudaGetDevice(&caller_device));
    struct Restore {
        int dev;
        ~Restore() { cudaSetDevice(dev); }
    } restore{caller_device};
    const int root_dev = gather ? devices[root] : 0;
    // one queue: the same stream on the same device (NULL is each device's own default stream)
    auto same_queue = [&](int r, int q) {
        return devices[r] == devices[q] && streams[r] == streams[q];
    };
    if (gather) {
        // No rank writes into `gathered` before the work already queued on the root's stream
        // (a reader of its previous contents, for one) has finished.
        MFK_CUDA(cudaSetDevice(root_dev));
        cudaEvent_t ready;
        MFK_CUDA(cudaEventCreateWithFlags(&ready, cudaEventDisableTiming));
        struct DestroyEvent {
            cudaEvent_t e;
            ~DestroyEvent() { cudaEventDestroy(e); }
        } ready_owner{ready};
        MFK_CUDA(cudaEventRecord(ready, static_cast<cudaStream_t>(streams[root])));
        for (int r = 0; r < nranks; ++r) {
            if (same_queue(r, root)) continue;
            MFK_CUDA(cudaSetDevice(devices[r]));
            MFK_CUDA(cudaStreamWaitEvent(static_cast<cudaStream_t>(streams[r]), ready, 0));
        }
    }
    int64_t row0 = 0;
    for (int r = 0; r < nranks; ++r) {
        mfk_gemm_desc d = per_rank[r];
        MFK_CUDA(cudaSetDevice(devices[r]));
        if (gather) {
            d.c = gathered + row0 * ld_gathered;
            d.ldc = ld_gathered;
            if (devices[r] != root_dev) {
                int can = 0;
                MFK_CUDA(cudaDeviceCanAccessPeer(&can, devices[r], root_dev));
                if (!can) {
                    t_cuda_error = "the gather target's GPU is not reachable as a peer";
                    return MFK_ERR_UNSUPPORTED;
                }
                const cudaError_t e = cudaDeviceEnablePeerAccess(root_dev, 0);
                if (e == cudaErrorPeerAccessAlreadyEnabled) {
                    cudaGetLastError();
                } else if (e != cudaSuccess) {
                    return cuda_fail(e, "cudaDeviceEnablePeerAccess");
                }
            }
        }
        const bool peer = gather && devices[r] != root_dev;
        const int rc = run_gemm(&d, nullptr, static_cast<cudaStream_t>(streams[r]), nullptr,
                                nullptr, peer ? kCOutputPeer : kCOutputInfer);
        if (rc != MFK_OK) return rc;
        row0 += d.m;
    }
    if (gather) {
        // The gathered C is complete on the root's stream once every rank's GEMM has finished.
        for (int r = 0; r < nranks; ++r) {
            if (same_queue(r, root)) continue;
            MFK_CUDA(cudaSetDevice(devices[r]));
            cudaEvent_t ev;
            MFK_CUDA(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming));
            cudaError_t e = cudaEventRecord(ev, static_cast<cudaStream_t>(streams[r]));
            if (e == cudaSuccess) {
                cudaSetDevice(root_dev);
                e = cudaStreamWaitEvent(static_cast<cudaStream_t>(streams[root]), ev, 0);
            }
            cudaEventDestroy(ev);
            if (e != cudaSuccess) return cuda_fail(e, "cross-device stream wait");
        }
    }
    return MFK_OK;
}

int mfk_ipc_get_handle(const void* ptr, void* handle, int64_t* offset) {
    if (ptr == nullptr || handle == nullptr || offset == nullptr) return MFK_ERR_INVALID_ARGUMENT;
    static PFN_cuMemGetAddressRange_v3020 range_fn = [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) !=
                cudaSuccess || q != cudaDriverEntryPointSuccess) {
            return static_cast<PFN_cuMemGetAddressRange_v3020>(nullptr);
        }
        return reinterpret_cast<PFN_cuMemGetAddressRange_v3020>(p);
    }();
    if (range_fn == nullptr) return MFK_ERR_UNSUPPORTED;
    CUdeviceptr base = 0;
    size_t size = 0;
    if (range_fn(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS) {
        t_cuda_error = "cuMemGetAddressRange: not a device allocation";
        return MFK_ERR_INVALID_ARGUMENT;
    }
    cudaIpcMemHandle_t h;
    MFK_CUDA(cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base)));
    static_assert(sizeof(h) == MFK_IPC_HANDLE_BYTES, "IPC handle size");
    std::memcpy(handle, &h, sizeof(h));
    *offset = static_cast<int64_t>(reinterpret_cast<uintptr_t>(ptr) - static_cast<uintptr_t>(base));
    return MFK_OK;
}

int mfk_ipc_open_handle(const void* handle, void** base) {
    if (handle == nullptr || base == nullptr) return MFK_ERR_INVALID_ARGUMENT;
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle, sizeof(h));
    MFK_CUDA(cudaIpcOpenMemHandle(base, h, cudaIpcMemLazyEnablePeerAccess));
    return MFK_OK;
}

int mfk_ipc_close_handle(void* base) {
    if (base == nullptr) return MFK_ERR_INVALID_ARGUMENT;
    MFK_CUDA(cudaIpcCloseMemHandle(base));
    return MFK_OK;
}

int mfk_gemm_strided_batched_f32(const mfk_gemm_desc* desc, const mfk_batch_desc* batch,
                                 void* stream) {
    if (batch == nullptr) return MFK_ERR_INVALID_ARGUMENT;
    return run_gemm(desc, batch, static_cast<cudaStream_t>(stream), nullptr);
}

int mfk_pack_b_f32(const float* b, int64_t rsb, int64_t csb, int64_t k, int64_t n,
                   int32_t precision, void* stream_, mfk_packed_b** out) {
    if (out == nullptr) return MFK_ERR_INVALID_ARGUMENT;
    *out = nullptr;
    if (k < 0 || n < 0 || precision < MFK_PRECISION_DEFAULT || precision > MFK_PRECISION_1XTF32)
        return MFK_ERR_INVALID_ARGUMENT;
    if (k > 0 && n > 0 && b == nullptr) return MFK_ERR_INVALID_ARGUMENT;
    if (k > (int64_t(1) << 31) - 256 || n > (int64_t(1) << 31) - 256) return MFK_ERR_UNSUPPORTED;
    int dev = 0;
    DeviceInfo* info = nullptr;
    int rc = current_device(&dev, &info);
    if (rc != MFK_OK) return rc;
    cudaStream_t stream = static_cast<cudaStream_t>(stream_);
    auto* p = new (std::nothrow) mfk_packed_b;
    if (p == nullptr) return MFK_ERR_OUT_OF_MEMORY;
    p->k = k;
    p->n = n;
    p->kp = (k + mfk::kBK - 1) / mfk::kBK * mfk::kBK;
    p->precision = precision == MFK_PRECISION_DEFAULT ? g_default_precision.load() : precision;
    p->device = dev;
    if (k > 0 && n > 0) {
        const bool split3 = p->precision == MFK_PRECISION_3XTF32;
        const size_t elems = static_cast<size_t>(n) * static_cast<size_t>(p->kp);
        const size_t panel_bytes = sizeof(float) * elems * (split3 ? 2 : 1);
        // From the stream-ordered pool, which keeps freed blocks (a plain cudaMalloc of a large
        // B costs milliseconds of host time); a plain allocation while the stream is captured.
        cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
        if (cudaStreamIsCapturing(stream, &cap) != cudaSuccess) {
            cudaGetLastError();
            cap = cudaStreamCaptureStatusActive;
        }
        p->pooled = cap == cudaStreamCaptureStatusNone;
        const cudaError_t alloc =
            p->pooled ? cudaMallocAsync(reinterpret_cast<void**>(&p->hi), panel_bytes + 16, stream)
                      : cudaMalloc(reinterpret_cast<void**>(&p->hi), panel_bytes + 16);
        if (alloc != cudaSuccess) {
            cudaGetLastError();
            delete p;
            return MFK_ERR_OUT_OF_MEMORY;
        }
        p->lo = split3 ? p->hi + elems : nullptr;
        if (split3) {
            p->inf_word = reinterpret_cast<unsigned*>(reinterpret_cast<uint8_t*>(p->hi) + panel_bytes);
            if (cudaMemsetAsync(p->inf_word, 0, sizeof(unsigned), stream) != cudaSuccess) {
                cudaGetLastError();
                mfk_packed_b_free(p);
                return MFK_ERR_CUDA;
            }
        }
        // op(B) element (p, j) at p*rsb + j*csb: K-major rows over j, row stride csb, depth rsb
        Operand o{b, csb, rsb, n, BatchLayout{}};
        o.hi = p->hi;
        o.lo = p->lo;
        rc = launch_pack(o, k, p->kp, 1, split3 ? mfk::kPackSplit : mfk::kPackRound, info, stream,
                         p->inf_word, 1u);
        if (rc != MFK_OK) {
            mfk_packed_b_free(p);
            return rc;
        }
    }
    *out = p;
    return MFK_OK;
}

int mfk_packed_b_shape(const mfk_packed_b* packed, int64_t* k, int64_t* n, int32_t* precision) {
    if (packed == nullptr) return MFK_ERR_INVALID_ARGUMENT;
    if (k) *k = packed->k;
    if (n) *n = packed->n;
    if (precision) *precision = packed->precision;
    return MFK_OK;
}

int mfk_packed_b_free(mfk_packed_b* packed) {
    if (packed == nullptr) return MFK_OK;
    int rc = MFK_OK;
    if (packed->hi != nullptr) {
        int cur = 0;
        const bool switch_dev = cudaGetDevice(&cur) == cudaSuccess && cur != packed->device;
        if (switch_dev) cudaSetDevice(packed->device);
        if (packed->pooled) {
            // nothing in flight reads it after the synchronisation: back to the pool at once
            if (cudaDeviceSynchronize() != cudaSuccess ||
                cudaFreeAsync(packed->hi, cudaStreamLegacy) != cudaSuccess)
                rc = MFK_ERR_CUDA;
        } else if (cudaFree(packed->hi) != cudaSuccess) {
            rc = MFK_ERR_CUDA;
        }
        if (switch_dev) cudaSetDevice(cur);
        cudaGetLastError();
    }
    delete packed;
    return rc;
}

int mfk_gemm_prepacked_f32(const mfk_gemm_desc* desc, const mfk_packed_b* packed, void* stream) {
    if (desc == nullptr || packed == nullptr) return MFK_ERR_INVALID_ARGUMENT;
    mfk_gemm_desc d = *desc;
    d.b = packed->hi != nullptr ? packed->hi : desc->a;  // B is read from the handle
    d.b_rs = 1;
    d.b_cs = 1;
    if (packed->hi == nullptr) d.k = 0;                      // an empty B: the product is zero
    if (d.n != packed->n || desc->k != packed->k) return MFK_ERR_INVALID_ARGUMENT;
    return run_gemm(&d, nullptr, static_cast<cudaStream_t>(stream), nullptr,
                    packed->hi != nullptr ? packed : nullptr);
}

int mfk_gemv_f32(const float* a, int64_t rows, int64_t cols, int64_t lda, int32_t transpose,
                 const float* x, int64_t incx, float alpha, float beta, const float* y0, float* y,
                 void* stream_) {
    cudaStream_t stream = static_cast<cudaStream_t>(stream_);
    if (rows < 0 || cols < 0 || lda < cols || incx < 1) return MFK_ERR_INVALID_ARGUMENT;
    const int64_t n_out = transpose ? cols : rows;
    const int64_t n_in = transpose ? rows : cols;
    if (n_out == 0) return MFK_OK;
    if (y == nullptr || (beta != 0.0f && y0 == nullptr)) return MFK_ERR_INVALID_ARGUMENT;
    if (n_in > 0 && (a == nullptr || x == nullptr)) return MFK_ERR_INVALID_ARGUMENT;
    int dev = 0;
    DeviceInfo* info = nullptr;
    int rc = current_device(&dev, &info);
    if (rc != MFK_OK) return rc;
    if (!transpose) {
        const bool vec = incx == 1 && lda % 4 == 0 && aligned16(a) && aligned16(x);
        TimedLaunch timed(stream);
        g_launches.fetch_add(1);
        if (vec) {
            // one warp per row (the block scheduler balances them), a grid stride beyond
            // kGemvBlocksPerSm blocks per SM
            const int64_t warps_per_block = mfk::kGemvThreads / 32;
            const int64_t blocks = std::min<int64_t>(
                (rows + warps_per_block - 1) / warps_per_block,
                static_cast<int64_t>(info->sm_count) * mfk::kGemvBlocksPerSm);
            mfk::gemv_n_vec4_kernel<<<static_cast<unsigned>(blocks), mfk::kGemvThreads, 0,
                                      stream>>>(a, rows, cols, lda, x, alpha, beta, y0, y);
        } else {
            const int64_t blocks = (rows * 32 + mfk::kGemvThreads - 1) / mfk::kGemvThreads;
            if (blocks > INT32_MAX) return MFK_ERR_UNSUPPORTED;
            mfk::gemv_n_scalar_kernel<<<static_cast<unsigned>(blocks), mfk::kGemvThreads, 0,
                                        stream>>>(a, rows, cols, lda, x, incx, alpha, beta, y0, y);
        }
        MFK_CUDA(cudaGetLastError());
        return MFK_OK;
    }
    const int64_t chunks = std::max<int64_t>(1, (rows + mfk::kGemvTRowsPerChunk - 1) /
                                                    mfk::kGemvTRowsPerChunk);
    if (chunks > 65535) return MFK_ERR_UNSUPPORTED;
    double* partial = nullptr;
    MFK_CUDA(cudaMallocAsync(reinterpret_cast<void**>(&partial),
                             sizeof(double) * chunks * std::max<int64_t>(cols, 1), stream));
    const unsigned bx = static_cast<unsigned>((cols + 255) / 256);
    g_launches.fetch_add(2);
    if (rows > 0) {
        TimedLaunch timed(stream);
        mfk::gemv_t_partial_kernel<<<dim3(bx, static_cast<unsigned>(chunks)), 256, 0, stream>>>(
            a, rows, cols, lda, x, incx, partial);
    } else {
        cudaMemsetAsync(partial, 0, sizeof(double) * cols, stream);
    }
    mfk::gemv_t_finish_kernel<<<bx, 256, 0, stream>>>(partial, static_cast<int>(chunks), cols,
                                                      alpha, beta, y0, y);
    const cudaError_t e = cudaGetLastError();
    cudaFreeAsync(partial, stream);
    if (e != cudaSuccess) return cuda_fail(e, "gemv_t launch");
    return MFK_OK;
}

int mfk_matvec_f32(const float* a, int64_t m, int64_t k, const float* x, float* y, void* stream) {
    return mfk_gemv_f32(a, m, k, k, 0, x, 1, 1.0f, 0.0f, nullptr, y, stream);
}

int mfk_bias_act_f32(const float* x, const float* bias, float* out, int64_t rows, int64_t cols,
                     int32_t activation, void* stream_) {
    cudaStream_t stream = static_cast<cudaStream_t>(stream_);
    if (rows < 0 || cols < 0) return MFK_ERR_INVALID_ARGUMENT;
    if (activation < MFK_ACT_NONE || activation > MFK_ACT_GELU_TANH) return MFK_ERR_INVALID_ARGUMENT;
    const int64_t total = rows * cols;
    if (total == 0) return MFK_OK;
    if (x == nullptr || out == nullptr) return MFK_ERR_INVALID_ARGUMENT;
    int dev = 0;
    DeviceInfo* info = nullptr;
    int rc = current_device(&dev, &info);
    if (rc != MFK_OK) return rc;
    const int64_t max_blocks = static_cast<int64_t>(info->sm_count) * 8;
    g_launches.fetch_add(1);
    if (cols % 4 == 0 && aligned16(x) && aligned16(out)) {
        const int64_t total4 = total / 4;
        const int64_t blocks = std::min<int64_t>((total4 + 255) / 256, max_blocks);
        mfk::bias_act_vec4_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(
            reinterpret_cast<const float4*>(x), bias, reinterpret_cast<float4*>(out), total4,
            cols, activation);
    } else {
        const int64_t blocks = std::min<int64_t>((total + 255) / 256, max_blocks);
        mfk::bias_act_scalar_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(
            x, bias, out, total, cols, activation);
    }
    MFK_CUDA(cudaGetLastError());
    return MFK_OK;
}

int mfk_bias_grad_f32(const float* grad, int64_t rows, int64_t cols, int64_t ld, float* dbias,
                      void* stream_) {
    cudaStream_t stream = static_cast<cudaStream_t>(stream_);
    if (rows < 0 || cols < 0 || (rows > 0 && ld < cols)) return MFK_ERR_INVALID_ARGUMENT;
    if (cols == 0) return MFK_OK;
    if (dbias == nullptr || (rows > 0 && grad == nullptr)) return MFK_ERR_INVALID_ARGUMENT;
    int dev = 0;
    DeviceInfo* info = nullptr;
    int rc = current_device(&dev, &info);
    if (rc != MFK_OK) return rc;
    const int64_t blocks = (cols + mfk::kBgCols - 1) / mfk::kBgCols;
    if (blocks > INT32_MAX) return MFK_ERR_UNSUPPORTED;
    g_launches.fetch_add(1);
    mfk::bias_grad_kernel<<<static_cast<unsigned>(blocks), mfk::kBgThreads, 0, stream>>>(
        grad, rows, cols, ld, dbias);
    MFK_CUDA(cudaGetLastError());
    return MFK_OK;
}

}  // extern "C"

namespace {

int launch_softmax(const float* x, float* out, int64_t outer, int64_t length, int64_t inner,
                   int log, const mfk::SoftmaxMask& mk, cudaStream_t stream) {
    if (outer < 0 || length < 0 || inner < 1) return MFK_ERR_INVALID_ARGUMENT;
    if (outer == 0 || length == 0) return MFK_OK;
    if (x == nullptr || out == nullptr) return MFK_ERR_INVALID_ARGUMENT;
    int dev = 0;
    DeviceInfo* info = nullptr;
    const int rc = current_device(&dev, &info);
    if (rc != MFK_OK) return rc;
    g_launches.fetch_add(1);
    if (inner == 1) {
        const int64_t blocks = (outer * 32 + 255) / 256;
        if (blocks > INT32_MAX) return MFK_ERR_UNSUPPORTED;
        mfk::softmax_lastdim_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(
            x, out, outer, length, log, mk);
    } else {
        const int64_t blocks = (outer * inner + 255) / 256;
        if (blocks > INT32_MAX) return MFK_ERR_UNSUPPORTED;
        mfk::softmax_strided_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(
            x, out, outer, length, inner, log);
    }
    MFK_CUDA(cudaGetLastError());
    return MFK_OK;
}

}  // namespace

extern "C" {

int mfk_softmax_f32(const float* x, float* out, int64_t outer, int64_t length, int64_t inner,
                    int32_t log, void* stream) {
    mfk::SoftmaxMask mk{nullptr, 0, 0, 0, 1};
    return launch_softmax(x, out, outer, length, inner, log != 0, mk,
                          static_cast<cudaStream_t>(stream));
}

}  // extern "C"

namespace {

// The fused attention for both entry points: keep == nullptr runs the kernel without a mask.
template <bool MASK>
int run_attention(const float* q, const float* k, const float* v, const uint8_t* keep,
                  int64_t keep_bs, int64_t keep_rs, int64_t keep_cs, float* out, int64_t heads,
                  int64_t len, int64_t head_dim, int32_t causal, float scale, void* stream_) {
    if (heads < 0 || len < 0 || head_dim < 0) return MFK_ERR_INVALID_ARGUMENT;
    if (MASK && (keep == nullptr || keep_bs < 0 || keep_rs < 0 || keep_cs < 0))
        return MFK_ERR_INVALID_ARGUMENT;
    if (heads == 0 || len == 0) return MFK_OK;
    if (q == nullptr || k == nullptr || v == nullptr || out == nullptr)
        return MFK_ERR_INVALID_ARGUMENT;
    if (head_dim != mfk::kAttnD || !aligned16(q) || !aligned16(k) || !aligned16(v) ||
        !aligned16(out))
        return MFK_ERR_UNSUPPORTED;
    if (len > (int64_t(1) << 30) || heads > (int64_t(1) << 30)) return MFK_ERR_UNSUPPORTED;
    int dev = 0;
    DeviceInfo* info = nullptr;
    int rc = current_device(&dev, &info);
    if (rc != MFK_OK) return rc;
    const cudaStream_t stream = static_cast<cudaStream_t>(stream_);
    const int64_t d = head_dim;
    // Q, K and V are read as they lie and split inside the kernel (where the tensor cores are
    // known to truncate fp32 operands to tf32 the raw values serve as the hi parts, bit for bit,
    // and only lo is computed): no pass before the kernel and no workspace. V's boxes use the
    // 128-byte swizzle on 32-byte atoms, the layout the kernel reads it MN-major in.
    const bool raw_hi = tf32_truncates(info, stream, true);
    CUtensorMap mq, mk, mv;
    const bool maps =
        make_kmajor_map(&mq, q, d, len, heads, d, len * d, mfk::kAttnRows) &&
        make_kmajor_map(&mk, k, d, len, heads, d, len * d, mfk::kAttnKeys / 2) &&
        make_kmajor_map(&mv, v, d, len, heads, d, len * d, mfk::kAttnChunk,
                        CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B);
    if (!maps) {
        t_cuda_error = "cuTensorMapEncodeTiled rejected an attention operand";
        return MFK_ERR_UNSUPPORTED;
    }
    mfk::AttnArgs a{};
    a.heads = static_cast<int>(heads);
    a.len = static_cast<int>(len);
    a.num_qb = static_cast<int>((len + mfk::kAttnUnitRows - 1) / mfk::kAttnUnitRows);
    a.causal = causal != 0 ? 1 : 0;
    a.scale = scale;
    a.num_units = static_cast<long long>(a.heads) * a.num_qb;
    a.raw_hi = raw_hi ? 1 : 0;
    a.keep = keep;
    a.keep_bs = keep_bs;
    a.keep_rs = keep_rs;
    a.keep_cs = keep_cs;
    auto kernel = mfk::attn_tc_kernel<MASK>;
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    cfg.blockDim = dim3(mfk::kAttnThreads, 1, 1);
    cfg.dynamicSmemBytes = mfk::kAttnSmemBytes;
    cfg.stream = stream;
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    constexpr int kSlot = MASK ? 14 : 15;  // this kernel's per-device set-up flags
    {
        std::lock_guard<std::mutex> lock(g_mutex);
        if (!info->smem_set[kSlot]) {
            MFK_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          mfk::kAttnSmemBytes));
            int units = info->sm_count / 2;
            cfg.gridDim = dim3(static_cast<unsigned>(info->sm_count / 2 * 2), 1, 1);
            int clusters = 0;
            if (cudaOccupancyMaxActiveClusters(&clusters, kernel, &cfg) == cudaSuccess &&
                clusters > 0)
                units = clusters;
            cudaGetLastError();
            info->resident_units[kSlot] = units;
            info->smem_set[kSlot] = true;
        }
    }
    const long long pairs = std::min<long long>(a.num_units, info->resident_units[kSlot]);
    cfg.gridDim = dim3(static_cast<unsigned>(pairs * 2), 1, 1);
    {
        TimedLaunch timed(stream);
        MFK_CUDA(cudaLaunchKernelEx(&cfg, kernel, mq, mk, mv, out, a));
    }
    g_launches.fetch_add(1);
    return MFK_OK;
}

}  // namespace

extern "C" {

int mfk_attention_f32(const float* q, const float* k, const float* v, float* out, int64_t heads,
                      int64_t len, int64_t head_dim, int32_t causal, float scale, void* stream) {
    return run_attention<false>(q, k, v, nullptr, 0, 0, 0, out, heads, len, head_dim, causal,
                                scale, stream);
}

int mfk_attention_masked_f32(const float* q, const float* k, const float* v, const uint8_t* keep,
                             int64_t keep_bs, int64_t keep_rs, int64_t keep_cs, float* out,
                             int64_t heads, int64_t len, int64_t head_dim, int32_t causal,
                             float scale, void* stream) {
    return run_attention<true>(q, k, v, keep, keep_bs, keep_rs, keep_cs, out, heads, len,
                               head_dim, causal, scale, stream);
}

int mfk_masked_softmax_f32(const float* scores, const uint8_t* keep, int64_t keep_bs,
                           int64_t keep_rs, int32_t causal, float* out, int64_t batch,
                           int64_t rows, int64_t cols, void* stream) {
    if (batch < 0 || rows < 0 || cols < 0 || keep_bs < 0 || keep_rs < 0)
        return MFK_ERR_INVALID_ARGUMENT;
    mfk::SoftmaxMask mk{keep, keep_bs, keep_rs, causal != 0 ? 1 : 0, rows > 0 ? rows : 1};
    return launch_softmax(scores, out, batch * rows, cols, 1, 0, mk,
                          static_cast<cudaStream_t>(stream));
}

int mfk_where_f32(const uint8_t* cond, const float* x, const float* y, float* out, int64_t n,
                  void* stream) {
    if (n < 0) return MFK_ERR_INVALID_ARGUMENT;
    if (n == 0) return MFK_OK;
    if (cond == nullptr || x == nullptr || y == nullptr || out == nullptr)
        return MFK_ERR_INVALID_ARGUMENT;
    int dev = 0;
    DeviceInfo* info = nullptr;
    const int rc = current_device(&dev, &info);
    if (rc != MFK_OK) return rc;
    const int64_t blocks = std::min<int64_t>((n + 255) / 256, int64_t(info->sm_count) * 8);
    g_launches.fetch_add(1);
    mfk::where_kernel<<<static_cast<unsigned>(blocks), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        cond, x, y, out, n);
    MFK_CUDA(cudaGetLastError());
    return MFK_OK;
}

}  // extern "C"

namespace {

int launch_contig_copy(const float* x, float* out, int64_t n, const DeviceInfo* info,
                       cudaStream_t stream) {
    const int64_t max_blocks = int64_t(info->sm_count) * 8;
    g_launches.fetch_add(1);
    if (aligned16(x) && aligned16(out) && n % 4 == 0) {
        const int64_t n4 = n / 4;
        const int64_t blocks = std::min<int64_t>((n4 + 255) / 256, max_blocks);
        mfk::copy_contig_vec4_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(
            reinterpret_cast<const float4*>(x), reinterpret_cast<float4*>(out), n4);
    } else {
        const int64_t blocks = std::min<int64_t>((n + 255) / 256, max_blocks);
        mfk::copy_contig_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(x, out, n);
    }
    MFK_CUDA(cudaGetLastError());
    return MFK_OK;
}

}  // namespace

extern "C" {

int mfk_strided_copy_f32(const float* x, const int64_t* shape, const int64_t* strides,
                         int32_t ndim, float* out, void* stream_) {
    cudaStream_t stream = static_cast<cudaStream_t>(stream_);
    if (ndim < 0 || (ndim > 0 && (shape == nullptr || strides == nullptr)))
        return MFK_ERR_INVALID_ARGUMENT;
    // Merge the view: drop size-1 dims, fold a dim into its outer neighbour when the pair is one
    // evenly strided run. The output is row-major over the same shape either way.
    mfk::CopyView v{};
    int64_t numel = 1;
    for (int d = 0; d < ndim; ++d) {
        if (shape[d] < 0) return MFK_ERR_INVALID_ARGUMENT;
        if (__builtin_mul_overflow(numel, shape[d], &numel)) return MFK_ERR_INVALID_ARGUMENT;
    }
    if (numel == 0) return MFK_OK;
    if (x == nullptr || out == nullptr) return MFK_ERR_INVALID_ARGUMENT;
    for (int d = 0; d < ndim; ++d) {
        if (shape[d] == 1) continue;
        if (v.ndim > 0 && v.stride[v.ndim - 1] == strides[d] * shape[d]) {
            v.shape[v.ndim - 1] *= shape[d];
            v.stride[v.ndim - 1] = strides[d];
            continue;
        }
        if (v.ndim == mfk::kMaxCopyDims) return MFK_ERR_UNSUPPORTED;
        v.shape[v.ndim] = shape[d];
        v.stride[v.ndim] = strides[d];
        ++v.ndim;
    }
    int dev = 0;
    DeviceInfo* info = nullptr;
    const int rc = current_device(&dev, &info);
    if (rc != MFK_OK) return rc;
    if (v.ndim == 0) return launch_contig_copy(x, out, 1, info, stream);
    if (v.ndim == 1 && v.stride[0] == 1) return launch_contig_copy(x, out, numel, info, stream);

    const int n = v.ndim;
    const int64_t L = v.shape[n - 1];
    const int64_t rows = numel / L;
    const int64_t max_blocks = int64_t(info->sm_count) * 8;
    int p = -1;
    if (v.stride[n - 1] != 1) {
        for (int d = n - 2; d >= 0; --d) {
            if (v.stride[d] == 1) {
                p = d;
                break;
            }
        }
    }
    g_launches.fetch_add(1);
    TimedLaunch timed(stream);
    if (p >= 0) {
        const int64_t batch = rows / v.shape[p];
        const int64_t tiles = ((L + mfk::kCopyTile - 1) / mfk::kCopyTile) *
                              ((v.shape[p] + mfk::kCopyTile - 1) / mfk::kCopyTile) * batch;
        const int64_t blocks = std::min<int64_t>(tiles, max_blocks);
        mfk::copy_transpose_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(
            x, out, v, p, batch);
    } else if (L < 32) {
        const int64_t blocks = std::min<int64_t>((rows + 255) / 256, max_blocks);
        mfk::copy_short_rows_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(
            x, out, v, rows);
    } else {
        bool vec4 = v.stride[n - 1] == 1 && L % 4 == 0 && aligned16(x) && aligned16(out);
        for (int d = 0; d + 1 < n; ++d) vec4 = vec4 && v.stride[d] % 4 == 0;
        // one warp per piece where the grid allows: the block scheduler balances them
        const int64_t pieces = (L + mfk::kCopyPiece - 1) / mfk::kCopyPiece;
        const int64_t blocks = std::min<int64_t>((rows * pieces * 32 + 255) / 256,
                                                 int64_t(info->sm_count) * 32);
        if (vec4) {
            mfk::copy_rows_kernel<true><<<static_cast<unsigned>(blocks), 256, 0, stream>>>(
                x, out, v, rows);
        } else {
            mfk::copy_rows_kernel<false><<<static_cast<unsigned>(blocks), 256, 0, stream>>>(
                x, out, v, rows);
        }
    }
    MFK_CUDA(cudaGetLastError());
    return MFK_OK;
}

int mfk_copy_f32(const float* x, float* out, int64_t n, void* stream) {
    if (n < 0) return MFK_ERR_INVALID_ARGUMENT;
    if (n == 0) return MFK_OK;
    if (x == nullptr || out == nullptr) return MFK_ERR_INVALID_ARGUMENT;
    int dev = 0;
    DeviceInfo* info = nullptr;
    const int rc = current_device(&dev, &info);
    if (rc != MFK_OK) return rc;
    return launch_contig_copy(x, out, n, info, static_cast<cudaStream_t>(stream));
}

int mfk_binary_f32(int32_t op, const float* x, const float* y, float* out, int64_t n,
                   void* stream_) {
    if (op < MFK_BINARY_ADD || op > MFK_BINARY_DIV || n < 0) return MFK_ERR_INVALID_ARGUMENT;
    if (n == 0) return MFK_OK;
    if (x == nullptr || y == nullptr || out == nullptr) return MFK_ERR_INVALID_ARGUMENT;
    int dev = 0;
    DeviceInfo* info = nullptr;
    const int rc = current_device(&dev, &info);
    if (rc != MFK_OK) return rc;
    const cudaStream_t stream = static_cast<cudaStream_t>(stream_);
    const int64_t max_blocks = static_cast<int64_t>(info->sm_count) * 8;
    const bool vec = aligned16(x) && aligned16(y) && aligned16(out) && n % 4 == 0;
    const int64_t work = vec ? n / 4 : n;
    const unsigned blocks = static_cast<unsigned>(std::min<int64_t>((work + 255) / 256, max_blocks));
    auto launch = [&](auto op_tag) {
        constexpr int kOp = decltype(op_tag)::value;
        if (vec) {
            mfk::binary_vec4_kernel<kOp><<<blocks, 256, 0, stream>>>(
                reinterpret_cast<const float4*>(x), reinterpret_cast<const float4*>(y),
                reinterpret_cast<float4*>(out), work);
        } else {
            mfk::binary_scalar_kernel<kOp><<<blocks, 256, 0, stream>>>(x, y, out, n);
        }
    };
    switch (op) {
    case MFK_BINARY_ADD: launch(std::integral_constant<int, mfk::kBinAdd>{}); break;
    case MFK_BINARY_SUB: launch(std::integral_constant<int, mfk::kBinSub>{}); break;
    case MFK_BINARY_MUL: launch(std::integral_constant<int, mfk::kBinMul>{}); break;
    default: launch(std::integral_constant<int, mfk::kBinDiv>{}); break;
    }
    g_launches.fetch_add(1);
    MFK_CUDA(cudaGetLastError());
    return MFK_OK;
}

int mfk_scal_f32(float alpha, const float* x, float* out, int64_t n, void* stream_) {
    if (n < 0) return MFK_ERR_INVALID_ARGUMENT;
    if (n == 0) return MFK_OK;
    if (x == nullptr || out == nullptr) return MFK_ERR_INVALID_ARGUMENT;
    int dev = 0;
    DeviceInfo* info = nullptr;
    const int rc = current_device(&dev, &info);
    if (rc != MFK_OK) return rc;
    const cudaStream_t stream = static_cast<cudaStream_t>(stream_);
    const int64_t max_blocks = static_cast<int64_t>(info->sm_count) * 8;
    if (aligned16(x) && aligned16(out) && n % 4 == 0) {
        const unsigned blocks =
            static_cast<unsigned>(std::min<int64_t>((n / 4 + 255) / 256, max_blocks));
        mfk::scal_vec4_kernel<<<blocks, 256, 0, stream>>>(
            alpha, reinterpret_cast<const float4*>(x), reinterpret_cast<float4*>(out), n / 4);
    } else {
        const unsigned blocks = static_cast<unsigned>(std::min<int64_t>((n + 255) / 256, max_blocks));
        mfk::scal_scalar_kernel<<<blocks, 256, 0, stream>>>(alpha, x, out, n);
    }
    g_launches.fetch_add(1);
    MFK_CUDA(cudaGetLastError());
    return MFK_OK;
}

int mfk_dot_f32(const float* x, const float* y, int64_t n, float* out, void* stream_) {
    if (n < 0 || out == nullptr) return MFK_ERR_INVALID_ARGUMENT;
    if (n > 0 && (x == nullptr || y == nullptr)) return MFK_ERR_INVALID_ARGUMENT;
    int dev = 0;
    DeviceInfo* info = nullptr;
    const int rc = current_device(&dev, &info);
    if (rc != MFK_OK) return rc;
    const cudaStream_t stream = static_cast<cudaStream_t>(stream_);
    if (n == 0) {
        MFK_CUDA(cudaMemsetAsync(out, 0, sizeof(float), stream));
        return MFK_OK;
    }
    // two blocks of 256 threads per SM, each thread with eight float4 of each input at least
    const int parts = static_cast<int>(std::max<int64_t>(
        1, std::min<int64_t>((n + 8191) / 8192, static_cast<int64_t>(info->sm_count) * 2)));
    double* partial = nullptr;
    MFK_CUDA(cudaMallocAsync(reinterpret_cast<void**>(&partial), sizeof(double) * parts, stream));
    const int vec = aligned16(x) && aligned16(y) ? 1 : 0;
    mfk::dot_partial_kernel<<<parts, 256, 0, stream>>>(x, y, n, vec, partial);
    mfk::dot_finish_kernel<<<1, 32, 0, stream>>>(partial, parts, out);
    g_launches.fetch_add(2);
    const cudaError_t launched = cudaGetLastError();
    cudaFreeAsync(partial, stream);
    if (launched != cudaSuccess) return cuda_fail(launched, "dot kernels");
    return MFK_OK;
}

int mfk_copy_peer(void* dst, int32_t dst_device, const void* src, int32_t src_device,
                  int64_t bytes, void* stream) {
    if (bytes < 0 || dst_device < 0 || src_device < 0) return MFK_ERR_INVALID_ARGUMENT;
    if (bytes == 0) return MFK_OK;
    if (dst == nullptr || src == nullptr) return MFK_ERR_INVALID_ARGUMENT;
    int count = 0;
    MFK_CUDA(cudaGetDeviceCount(&count));
    if (dst_device >= count || src_device >= count) return MFK_ERR_INVALID_ARGUMENT;
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (dst_device == src_device) {
        MFK_CUDA(cudaMemcpyAsync(dst, src, static_cast<size_t>(bytes), cudaMemcpyDeviceToDevice, s));
    } else {
        MFK_CUDA(cudaMemcpyPeerAsync(dst, dst_device, src, src_device, static_cast<size_t>(bytes), s));
    }
    return MFK_OK;
}

}  // extern "C"

extern "C" {

int mfk_set_default_precision(int32_t precision) {
    if (precision != MFK_PRECISION_3XTF32 && precision != MFK_PRECISION_1XTF32)
        return MFK_ERR_INVALID_ARGUMENT;
    g_default_precision.store(precision);
    return MFK_OK;
}

int32_t mfk_get_default_precision(void) { return g_default_precision.load(); }

int mfk_device_status(uint32_t* bits, int32_t clear) {
    if (bits == nullptr) return MFK_ERR_INVALID_ARGUMENT;
    MFK_CUDA(cudaDeviceSynchronize());
    unsigned int v = 0;
    MFK_CUDA(cudaMemcpyFromSymbol(&v, mfk::g_device_error, sizeof(v)));
    if (clear && v != 0) {
        const unsigned int zero = 0;
        MFK_CUDA(cudaMemcpyToSymbol(mfk::g_device_error, &zero, sizeof(zero)));
    }
    *bits = v;
    return v != 0 ? MFK_ERR_DEVICE_FAULT : MFK_OK;
}

int mfk_selftest_wait_timeout(uint64_t limit_ns, uint32_t* gave_up, void* stream) {
    if (gave_up == nullptr || limit_ns == 0 || limit_ns > MFK_WAIT_LIMIT_NS)
        return MFK_ERR_INVALID_ARGUMENT;
    int dev = 0;
    DeviceInfo* info = nullptr;
    const int rc = current_device(&dev, &info);
    if (rc != MFK_OK) return rc;
    void* flag_addr = nullptr;
    MFK_CUDA(cudaGetSymbolAddress(&flag_addr, g_selftest_flag));
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    unsigned int* flag = static_cast<unsigned int*>(flag_addr);
    g_launches.fetch_add(1);
    mfk::wait_selftest_kernel<<<1, 32, 0, s>>>(static_cast<unsigned long long>(limit_ns), flag);
    MFK_CUDA(cudaGetLastError());
    MFK_CUDA(cudaMemcpyAsync(gave_up, flag, sizeof(uint32_t), cudaMemcpyDeviceToHost, s));
    MFK_CUDA(cudaStreamSynchronize(s));
    return MFK_OK;
}

int mfk_kernel_timer(int32_t enable) {
    std::lock_guard<std::mutex> lock(g_timer.mu);
    g_timer.enabled = enable != 0;
    return MFK_OK;
}

int mfk_kernel_timer_read(double* total_ms, int64_t* launches) {
    if (total_ms == nullptr || launches == nullptr) return MFK_ERR_INVALID_ARGUMENT;
    std::lock_guard<std::mutex> lock(g_timer.mu);
    double sum = 0.0;
    for (auto& ev : g_timer.pending) {
        MFK_CUDA(cudaEventSynchronize(ev.second));
        float ms = 0.0f;
        MFK_CUDA(cudaEventElapsedTime(&ms, ev.first, ev.second));
        sum += ms;
        g_timer.spare.push_back(ev);
    }
    *total_ms = sum;
    *launches = static_cast<int64_t>(g_timer.pending.size());
    g_timer.pending.clear();
    return MFK_OK;
}

int64_t mfk_launch_count(void) { return g_launches.load(); }

const char* mfk_status_string(int32_t status) {
    switch (status) {
    case MFK_OK:
        return "ok";
    case MFK_ERR_INVALID_ARGUMENT:
        return "invalid argument";
    case MFK_ERR_UNSUPPORTED:
        return "unsupported shape or layout";
    case MFK_ERR_CUDA:
        return "CUDA runtime error";
    case MFK_ERR_OUT_OF_MEMORY:
        return "out of device memory";
    case MFK_ERR_NO_DEVICE:
        return "no sm_100 device is current";
    case MFK_ERR_DEVICE_FAULT:
        return "a kernel recorded a fault";
    case MFK_ERR_SCRATCH_LIMIT:
        return "the operand copies need more than the no-allocation entry point's fixed scratch";
    default:
        return "unknown status";
    }
}

const char* mfk_last_cuda_error(void) { return t_cuda_error.c_str(); }

int32_t mfk_version(void) { return (1 << 16) | 0; }

}  // extern "C"
