/* mfk.h — the C ABI of the B200 (sm_100a) kernels for Mensurflow's dense fp32 contraction path.
 *
 * This is the drop-in boundary. The reference's CUDA backend registers a C++ KernelFn per
 * (op, device, dtype) with its dispatcher (src/core/dispatcher.hpp:199 `KernelFn`, :249
 * `register_kernel`; src/backends/cuda/backend.cpp:231-238 `register_kernels`). A backend
 * adapter unpacks `OpArgs` (dispatcher.hpp:164-197) into the plain descriptors below and calls
 * these functions; nothing here uses C++ or torch types.
 *
 * Conventions
 *   - All pointers are device pointers on the current CUDA device, except where a comment says
 *     "host". `stream` is a cudaStream_t (NULL = the legacy default stream).
 *   - Calls are asynchronous on `stream`, like every kernel launch of the reference's CUDA
 *     backend (include/mensurflow/ops/blas.hpp:1-3).
 *   - Return value: MFK_OK, or an mfk_status error code (text: mfk_status_string). Argument
 *     errors are reported before anything is launched. The reference's adapters turn a non-zero
 *     status into std::runtime_error / std::invalid_argument (src/backends/cuda/backend.cpp:22-34).
 *   - Faults inside a kernel (a bounded pipeline wait that gave up) are recorded in a per-device
 *     error word, read with mfk_device_status().
 */
#ifndef MFK_H
#define MFK_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum mfk_status {
    MFK_OK = 0,
    MFK_ERR_INVALID_ARGUMENT = 1, /* a shape, stride, pointer or enum value is not valid */
    MFK_ERR_UNSUPPORTED = 2,      /* valid, but beyond what this build handles */
    MFK_ERR_CUDA = 3,             /* a CUDA runtime call failed (launch, attribute, copy) */
    MFK_ERR_OUT_OF_MEMORY = 4,    /* the stream-ordered workspace could not be allocated */
    MFK_ERR_NO_DEVICE = 5,        /* no sm_100 device is current */
    MFK_ERR_DEVICE_FAULT = 6,     /* a kernel recorded a fault (see mfk_device_status) */
    MFK_ERR_SCRATCH_LIMIT = 7     /* needs more than MFK_NOALLOC_SCRATCH_BYTES (no-alloc entry) */
} mfk_status;

/* Epilogue activation, applied after alpha/beta/bias: relu (elementwise.hpp:56), exact GELU
 * 0.5*v*erfc(-v/sqrt 2) or its tanh form (elementwise.hpp:62, approximate=true). */
typedef enum mfk_activation {
    MFK_ACT_NONE = 0,
    MFK_ACT_RELU = 1,
    MFK_ACT_GELU = 2,
    MFK_ACT_GELU_TANH = 3
} mfk_activation;

/* Tensor-core arithmetic for the fp32 GEMMs. 3xTF32 splits each operand into tf32 hi + lo and
 * accumulates three products in fp32 (fp32-faithful: |C - C_ref| <= 1e-5 * (|A||B|)_ij + 1e-6);
 * 1xTF32 is one tf32 product per term (<= 2e-3 * (|A||B|)_ij). The split's hi part is x with its
 * 13 low mantissa bits cleared; where a one-time check finds that the tensor cores truncate fp32
 * operands to tf32, operands split inside a kernel keep their raw values as hi (only lo is
 * written). The environment variable MFK_EXPLICIT_SPLIT (set, and not "0") makes every split
 * write hi explicitly, as on tensor cores that round; the results are the same bits. */
typedef enum mfk_precision {
    MFK_PRECISION_DEFAULT = -1, /* the process-wide setting (mfk_set_default_precision) */
    MFK_PRECISION_3XTF32 = 0,
    MFK_PRECISION_1XTF32 = 1
} mfk_precision;

/* Bits of the device error word. */
#define MFK_DEVERR_PRODUCER_TIMEOUT 0x1u
#define MFK_DEVERR_MMA_TIMEOUT 0x2u
#define MFK_DEVERR_EPILOGUE_TIMEOUT 0x4u
#define MFK_DEVERR_CONVERT_TIMEOUT 0x8u
#define MFK_DEVERR_SELFTEST_TIMEOUT 0x10u

/* One GEMM: c = act(alpha * op(A) op(B) + beta * c_in + bias).
 * op(A) is m x k with element (i, p) at a[i*a_rs + p*a_cs]; op(B) is k x n with element (p, j)
 * at b[p*b_rs + j*b_cs]. A transpose is a swap of the two strides, exactly as the reference's
 * strided kernels take it (cpu::BatchedGemm rsa/csa/rsb/csb, gemm_batched.hpp:21-37;
 * matmul_f32_packed_strided, gemm_packed.hpp:138). c_in is read only when beta != 0 (it may be
 * c itself), with element (i, j) at c_in[i*c_in_rs + j*c_in_cs] (a row broadcast has
 * c_in_rs = 0). c is row-major with row stride ldc >= n. bias (optional) has n entries. */
typedef struct mfk_gemm_desc {
    const float* a;
    int64_t a_rs, a_cs;
    const float* b;
    int64_t b_rs, b_cs;
    const float* c_in;
    int64_t c_in_rs, c_in_cs;
    float* c;
    int64_t ldc;
    int64_t m, n, k;
    float alpha, beta;
    const float* bias;
    int32_t activation; /* mfk_activation */
    int32_t precision;  /* mfk_precision */
} mfk_gemm_desc;

/* The batch of a strided-batched GEMM. Matrix i of op(A) starts at a + a_offsets[i] and of op(B)
 * at b + b_offsets[i] (host arrays of `batch` element offsets, the reference's odometer walk in
 * gemm_batched_kernel, src/backends/cpu/backend.cpp:251-270). When an offsets pointer is NULL the
 * matrices are evenly spaced by a_stride / b_stride elements (0 = one matrix shared by all).
 * c_in of matrix i starts at c_in + i*c_in_stride (0 = shared), c of matrix i at c + i*c_stride. */
typedef struct mfk_batch_desc {
    int64_t batch;
    const int64_t* a_offsets; /* host, may be NULL */
    const int64_t* b_offsets; /* host, may be NULL */
    int64_t a_stride, b_stride;
    int64_t c_in_stride;
    int64_t c_stride;
} mfk_batch_desc;

/* gemm / matmul on CUDA in one call. Replaces the OpId::Matmul kernel (CPU adapter:
 * src/backends/cpu/backend.cpp:131-164) and the mul / scal / add / bias_add dispatches that
 * mensurflow::gemm and bias_add chain after it (src/ops/blas.cpp:234-262,
 * src/ops/elementwise.cpp:251-284). matmul is alpha = 1, beta = 0, no bias, no activation. */
int mfk_gemm_f32(const mfk_gemm_desc* desc, void* stream);

/* mfk_gemm_f32 for callers that cannot allocate device memory. No counterpart in the reference.
 *
 * Some hosts must not allocate on the device while they run: a serving process that reserves
 * its whole memory plan at start-up, a framework whose own caching allocator owns every byte of
 * the device, or a latency-critical loop where an allocation may synchronise with the device.
 * mfk_gemm_f32 asks the stream-ordered allocator for the tf32 (hi, lo) operand copies; this entry
 * point instead uses one fixed scratch array of MFK_NOALLOC_SCRATCH_BYTES that the library keeps
 * in device memory (a static __device__ array: every GPU that loads the library holds it until
 * the process exits). It calls no cudaMalloc/cudaFree or other allocating routine.
 *
 * Same descriptor and the same error bound as mfk_gemm_f32 (3xTF32: |C - C_ref| <= 1e-5 *
 * (|A||B|)_ij + 1e-6; 1xTF32: 2e-3 relative), but not always the same bits: this entry point
 * never uses the stream-K schedule (whose partial tiles would need memory of their own), so on
 * shapes where mfk_gemm_f32 shares the last wave's tiles by k-iterations the two sum in a
 * different order. The caller still provides every input and the output. The operand copies
 * must fit: 4 bytes x (number of copies) x (rows of each packed operand) x k rounded up to 32,
 * plus 256 bytes per packed operand and one more word. 3xTF32 packs B (n rows) twice, and A
 * (m rows) twice only when TMA cannot read it where it lies (not K-major, or rows not 16-byte
 * aligned); 1xTF32 packs once only an operand TMA cannot read. Larger problems return
 * MFK_ERR_SCRATCH_LIMIT before anything is launched.
 *
 * The first call on a device looks up the scratch array's device address (cudaGetSymbolAddress)
 * with that device current; make that first call before any stream capture. All calls share the
 * one array and it keeps the previous call's contents (every byte a call reads is written by the
 * same call first), so calls whose kernels overlap on the GPU — on different streams, or from
 * different host threads — race on it; order them on one stream. */
#define MFK_NOALLOC_SCRATCH_BYTES (64u * 1024u * 1024u)
int mfk_gemm_f32_noalloc(const mfk_gemm_desc* desc, void* stream);

/* mfk_gemm_f32 with C in another GPU's memory: a peer allocation or a CUDA IPC mapping of one
 * (mfk_ipc_open_handle), written over NVLink. The caller states it, rather than the library
 * inferring it from the pointer's attributes (which for an IPC mapping need not name the owning
 * GPU): the epilogue then writes C with plain stores of full 128-byte row segments, never
 * through a tensor map, and ends with a system-scope fence, so work the other GPU orders after
 * this kernel (an event wait, a collective) sees the rows. Also valid, only slower, on local
 * memory. No counterpart in the reference (single device); the gather of the row-block split. */
int mfk_gemm_peer_f32(const mfk_gemm_desc* desc, void* stream);

/* A GEMM split by row blocks over several GPUs of this process, optionally gathered into one
 * device's buffer in the same kernels. Rank r (of nranks) computes its rows with per_rank[r] (every
 * pointer on devices[r]) on streams[r] (NULL: that device's default stream). With gather == 0
 * each rank writes its own per_rank[r].c. With gather != 0, per_rank[r].c and .ldc are ignored:
 * rank r's epilogue stores its rows straight into `gathered` (an [sum of m, n] buffer with row
 * stride ld_gathered on devices[root]) at row offset sum_{q<r} per_rank[q].m — the ranks on other
 * GPUs write over NVLink (peer access is enabled here), so the gather needs no extra kernel or
 * collective — and streams[root] waits for every rank, so work queued on it after this call sees
 * the whole C; the ranks' writes in turn start only after the work queued on streams[root] before
 * this call (a reader of the previous contents of `gathered`, for one). The reference has no multi-device path (its GEMM runs on one device); this is the
 * row-block partition plus the gather that a single-device result needs, in place of an NCCL
 * all-gather of C. Returns once every launch is queued; the caller's current device is kept. */
int mfk_sharded_gemm_f32(const mfk_gemm_desc* per_rank, int32_t nranks, const int32_t* devices,
                         void* const* streams, int32_t gather, int32_t root, float* gathered,
                         int64_t ld_gathered);

/* Device memory shared between processes (one process per GPU), so a rank's GEMM can write its
 * rows into another rank's buffer over NVLink: mfk_ipc_get_handle returns the IPC handle of the
 * allocation holding `ptr` (MFK_IPC_HANDLE_BYTES bytes into `handle`) and ptr's byte offset in it;
 * mfk_ipc_open_handle maps a handle from another process on the current device (peer access
 * enabled) and returns the allocation's base; mfk_ipc_close_handle unmaps it. No counterpart in
 * the reference (single process). */
#define MFK_IPC_HANDLE_BYTES 64
int mfk_ipc_get_handle(const void* ptr, void* handle, int64_t* offset);
int mfk_ipc_open_handle(const void* handle, void** base);
int mfk_ipc_close_handle(void* base);

/* gemm_strided_batched on CUDA. Replaces the OpId::GemmBatched kernel (CPU adapter:
 * src/backends/cpu/backend.cpp:239-293 -> cpu::gemm_batched_f32_parallel, gemm_batched.cpp:58)
 * and so both batched GEMMs of attention (src/ops/attention.cpp:69, :97). desc->m/n/k describe
 * one matrix; desc->a and desc->b are the base pointers the batch offsets apply to. */
int mfk_gemm_strided_batched_f32(const mfk_gemm_desc* desc, const mfk_batch_desc* batch,
                                 void* stream);

/* B split once, for many products with the same B: the device analogue of the reference's
 * PackedB (src/backends/cpu/ops/gemm/gemm_packed.hpp:147-191: pack_b_f32, matmul_f32_prepacked),
 * for weights that are only evaluated. The handle owns device memory on the device current at
 * packing time holding op(B) as K-major tf32 panels — (hi, lo) for 3xTF32, rounded values for
 * 1xTF32 — so products with it skip B's split pass.
 *
 * mfk_pack_b_f32: B is k x n on the current device, element (p, j) at b[p*rsb + j*csb] (row-major
 * weights: rsb = n, csb = 1; weights stored [outputs, inputs]: rsb = 1, csb = k). b may be freed
 * or changed once the stream has run the pack. precision: MFK_PRECISION_3XTF32 / _1XTF32, or
 * DEFAULT for the library default at packing time. k == 0 or n == 0 gives an empty handle whose
 * products are zeros (plus beta*C_in and bias). The panels come from the device's stream-ordered
 * memory pool, allocated on `stream` (a plain allocation while the stream is being captured), so
 * the handle may be used on another stream only after that stream has waited for `stream`. The
 * handle is released by mfk_packed_b_free (device-synchronising; not while a product using it is
 * in flight).
 *
 * mfk_gemm_prepacked_f32: the mfk_gemm_f32 product with B taken from the handle: desc->b, b_rs and
 * b_cs are ignored; desc->k and desc->n must equal the handle's k and n, and the call must run
 * on the handle's device. A 1xTF32 handle cannot serve a 3xTF32 product (MFK_ERR_INVALID_ARGUMENT);
 * a 3xTF32 handle serves both. For 3xTF32 the result is bit-identical to mfk_gemm_f32 with the
 * same B. */
typedef struct mfk_packed_b mfk_packed_b;
int mfk_pack_b_f32(const float* b, int64_t rsb, int64_t csb, int64_t k, int64_t n,
                   int32_t precision, void* stream, mfk_packed_b** out);
int mfk_packed_b_shape(const mfk_packed_b* packed, int64_t* k, int64_t* n, int32_t* precision);
int mfk_packed_b_free(mfk_packed_b* packed);
int mfk_gemm_prepacked_f32(const mfk_gemm_desc* desc, const mfk_packed_b* packed, void* stream);

/* gemv: y = alpha * op(A) x + beta * y0 with A row-major [rows, cols] (row stride lda), op(A) = A
 * or its transpose, sums accumulated in double. Replaces the OpId::Gemv kernel (CPU adapter:
 * src/backends/cpu/backend.cpp:120-125 -> cpu::gemv_f32, src/backends/cpu/ops/blas/blas.cpp:66).
 * y0 is read only when beta != 0. incx is x's element stride. */
int mfk_gemv_f32(const float* a, int64_t rows, int64_t cols, int64_t lda, int32_t transpose,
                 const float* x, int64_t incx, float alpha, float beta, const float* y0, float* y,
                 void* stream);

/* matvec: y = A x, A [m, k] contiguous. Replaces the OpId::Matvec kernel (cpu::matvec_f32,
 * src/backends/cpu/ops/blas/blas.cpp:55). */
int mfk_matvec_f32(const float* a, int64_t m, int64_t k, const float* x, float* y, void* stream);

/* out = act(x + bias) over a contiguous [rows, cols] x; bias (cols entries) may be NULL, so this
 * is also the standalone relu / gelu. Replaces the OpId::BiasAdd, Relu and Gelu kernels (CPU
 * adapters: src/backends/cpu/backend.cpp:762-767 bias_add_kernel, :658 gelu_kernel). out may be
 * x. */
int mfk_bias_act_f32(const float* x, const float* bias, float* out, int64_t rows, int64_t cols,
                     int32_t activation, void* stream);

/* The bias gradient of bias_add: dbias[j] = sum over rows of grad[r*ld + j], accumulated in
 * fp32 in row order from 0 — bit-identical to the reference's backward closure, which runs this
 * loop on the host after copying the gradient back (src/ops/elementwise.cpp:263-283). grad is
 * rows x cols (row stride ld >= cols); rows == 0 gives zeros. */
int mfk_bias_grad_f32(const float* grad, int64_t rows, int64_t cols, int64_t ld, float* dbias,
                      void* stream);

/* softmax (log_softmax when `log` != 0) along the middle axis of a contiguous [outer, length,
 * inner] tensor: max (NaN poisons the line), exp in fp32, sum in double, multiply by 1/sum; an
 * all -inf line gives zeros (-inf for log_softmax). Replaces the OpId::Softmax / LogSoftmax kernels
 * (CPU adapter: src/backends/cpu/backend.cpp:549-552 -> softmax_f32 / log_softmax_f32,
 * src/backends/cpu/ops/softmax/softmax.cpp:11-80). out may be x. */
int mfk_softmax_f32(const float* x, float* out, int64_t outer, int64_t length, int64_t inner,
                    int32_t log, void* stream);

/* Scaled-dot-product attention in one kernel: out = softmax(scale * q k^T) v per head, over the
 * keys, with causal != 0 masking every key after the query (key > query). q, k, v and out are
 * contiguous [heads, len, head_dim] fp32 (queries = keys = len), 16-byte aligned; head_dim must be
 * 128 (MFK_ERR_UNSUPPORTED otherwise). For these shapes it computes what the reference's
 * attention(q, k, v, nullptr, causal, scale) composes from gemm_strided_batched, where and softmax
 * (src/ops/attention.cpp:48-98), in 3xTF32 throughout, without writing the [len, len] scores,
 * and with the causal mask it skips the key tiles above the diagonal. The softmax is evaluated
 * online (running row maximum and sum, the output rescaled as the maximum grows), so the result
 * agrees with the composed path within the reference's attention tolerance (1e-4 relative), not
 * bit for bit. Non-finite inputs are not supported (results are unspecified); callers that may
 * hold them use the composed path. Q, K and V are read as they lie and split into tf32 (hi, lo)
 * inside the kernel: one launch, no workspace, nothing allocated. */
int mfk_attention_f32(const float* q, const float* k, const float* v, float* out, int64_t heads,
                      int64_t len, int64_t head_dim, int32_t causal, float scale, void* stream);

/* The same with a Bool keep mask, as the reference's attention(q, k, v, &mask, causal, scale):
 * key j may be seen by query i of matrix b when keep[b*keep_bs + i*keep_rs + j*keep_cs] != 0
 * (device bytes, strides in bytes, 0 broadcasts; a [len, len] mask shared by every matrix has
 * keep_bs = 0), together with the causal limit when causal != 0. A query whose keys are all
 * masked out gets zeros, as the reference's softmax gives them. */
int mfk_attention_masked_f32(const float* q, const float* k, const float* v, const uint8_t* keep,
                             int64_t keep_bs, int64_t keep_rs, int64_t keep_cs, float* out,
                             int64_t heads, int64_t len, int64_t head_dim, int32_t causal,
                             float scale, void* stream);

/* The softmax between attention's GEMMs with its masking fused in: for a contiguous
 * [batch, rows, cols] score tensor, entry (b, i, j) counts as -inf unless (keep == NULL or
 * keep[b*keep_bs + i*keep_rs + j] != 0) and (causal == 0 or j <= i); then softmax along cols.
 * Equal to the reference's where(keep, scores, -inf) [+ causal where] followed by softmax(-1)
 * (src/ops/attention.cpp:82-96) in one pass. keep is a Bool (one byte per entry) mask with unit
 * column stride; keep_bs / keep_rs may be 0 (broadcast). out may be scores. No counterpart kernel
 * in the reference (it composes where and softmax). */
int mfk_masked_softmax_f32(const float* scores, const uint8_t* keep, int64_t keep_bs,
                           int64_t keep_rs, int32_t causal, float* out, int64_t batch,
                           int64_t rows, int64_t cols, void* stream);

/* out[i] = cond[i] ? x[i] : y[i] over n contiguous elements (cond: one byte per element, Bool).
 * Replaces the OpId::Where kernel (CPU adapter src/backends/cpu/backend.cpp:625-630 -> where_f32);
 * the op expands and packs its inputs first (src/ops/elementwise.cpp:455-481). */
int mfk_where_f32(const uint8_t* cond, const float* x, const float* y, float* out, int64_t n,
                  void* stream);

/* Tensor::contiguous() on the device: gathers the strided view x (element (i_0..i_{n-1}) at
 * x[sum_d i_d * strides[d]], strides in elements, any sign, 0 for broadcast dims) into the
 * row-major buffer out of the same shape. shape/strides are host arrays of ndim entries. Replaces
 * the host round trip of non-CPU tensors in src/core/tensor.cpp:208-230 (copy_to_host into a
 * std::vector, then copy_from_host) and matches the CPU path's cpu::strided_copy_f32 /
 * cpu::transpose_f32 (src/backends/cpu/ops/movement/movement.cpp:12-67) byte for byte. After
 * merging size-1 and contiguous neighbouring dims at most 12 dims may remain
 * (MFK_ERR_UNSUPPORTED beyond). out must not overlap x. */
int mfk_strided_copy_f32(const float* x, const int64_t* shape, const int64_t* strides,
                         int32_t ndim, float* out, void* stream);

/* out[i] = x[i] for n contiguous elements. Replaces the OpId::Copy kernel (CPU adapter:
 * src/backends/cpu/backend.cpp:110-113 -> cpu::copy_f32; op: src/ops/blas.cpp:106-117). */
int mfk_copy_f32(const float* x, float* out, int64_t n, void* stream);

/* Elementwise out[i] = x[i] op y[i] over n contiguous elements, one IEEE fp32 operation per
 * element (round to nearest, no contraction), bit-identical to the CPU backend's add_f32 / sub_f32
 * / mul_f32 / div_f32 (src/backends/cpu/backend.cpp:865-868, via binary_kernel :595-598). Replaces
 * the reference's CUDA Add/Sub/Mul kernels, which composed a copy with cublasSaxpy and used
 * cublasSdgmm (src/backends/cuda/backend.cpp:160-191), and adds Div, which it lacked. The op layer
 * expands and packs broadcast inputs first (src/ops/elementwise.cpp:158-225). out may be x or
 * y. */
typedef enum mfk_binary_op {
    MFK_BINARY_ADD = 0,
    MFK_BINARY_SUB = 1,
    MFK_BINARY_MUL = 2,
    MFK_BINARY_DIV = 3
} mfk_binary_op;
int mfk_binary_f32(int32_t op, const float* x, const float* y, float* out, int64_t n,
                   void* stream);

/* out[i] = alpha * x[i] over n contiguous elements: the OpId::Scal kernel (CPU adapter
 * src/backends/cpu/backend.cpp:95-98 -> cpu::scal_f32, src/backends/cpu/ops/blas/blas.cpp:23),
 * which the reference's gemm uses for beta * c (src/ops/blas.cpp:257) and which its CUDA backend
 * lacked. Bit-identical to the CPU. out may be x. */
int mfk_scal_f32(float alpha, const float* x, float* out, int64_t n, void* stream);

/* *out = sum of x[i] * y[i] over n contiguous elements, the products summed in double and the sum
 * rounded once to fp32, as cpu::dot_f32 does (src/backends/cpu/ops/blas/blas.cpp:14-21); replaces
 * the reference's CUDA Dot kernel (cublasSdot, src/backends/cuda/backend.cpp:122-134). out is a
 * device pointer to one float; n == 0 writes 0. The order of the double sum is fixed for a given
 * n on a given GPU model, so repeated calls give the same bits. */
int mfk_dot_f32(const float* x, const float* y, int64_t n, float* out, void* stream);

/* Tensor::to(device) between two CUDA devices: `bytes` from src on src_device to dst on
 * dst_device, device to device over NVLink (a stream-ordered peer copy on `stream`), instead of
 * the reference's staging through a host std::vector (src/core/tensor.cpp:193-206). The same
 * device gives a device-to-device copy. */
int mfk_copy_peer(void* dst, int32_t dst_device, const void* src, int32_t src_device,
                  int64_t bytes, void* stream);

/* Process-wide precision used when a descriptor says MFK_PRECISION_DEFAULT. The reference's
 * public signatures have no precision argument, so its adapters leave the default in place. */
int mfk_set_default_precision(int32_t precision);
int32_t mfk_get_default_precision(void);

/* Reads (and clears when `clear` != 0) the error word of the current device after waiting for the
 * device to finish its work. *bits receives MFK_DEVERR_* bits; returns MFK_OK, or
 * MFK_ERR_DEVICE_FAULT when bits were set, or MFK_ERR_CUDA. */
int mfk_device_status(uint32_t* bits, int32_t clear);

/* Self-test of the failure path (no counterpart in the reference): one kernel waits, through the
 * same bounded wait the GEMM pipeline uses, on a barrier that nothing completes, with a limit of
 * limit_ns (at most the pipeline's own 2 s). The wait gives up, sets MFK_DEVERR_SELFTEST_TIMEOUT
 * in the device error word and the kernel ends normally; *gave_up is 1 when it did. Synchronises
 * the stream. Read (and clear) the error word with mfk_device_status afterwards; the context
 * stays usable. */
int mfk_selftest_wait_timeout(uint64_t limit_ns, uint32_t* gave_up, void* stream);

/* Instrumentation (no counterpart in the reference's kernels; the reference times ops with
 * host-side trace spans in run_on, src/core/dispatcher.cpp:298-317, which cannot see device time).
 * mfk_kernel_timer(1) makes every later call record a CUDA event pair around its main kernel
 * launch (the tensor-core GEMM, or the gemv kernel) on the caller's stream; mfk_kernel_timer_read
 * waits for those events, returns the summed device time in ms and the number of timed launches,
 * and forgets them. mfk_kernel_timer(0) stops recording. */
int mfk_kernel_timer(int32_t enable);
int mfk_kernel_timer_read(double* total_ms, int64_t* launches);

/* Number of kernels this library has launched in this process (all entry points). */
int64_t mfk_launch_count(void);

/* Human-readable text of a status code (static storage). */
const char* mfk_status_string(int32_t status);

/* Text of the last CUDA error seen by this thread inside the library ("" when none). */
const char* mfk_last_cuda_error(void);

/* ABI version: (major << 16) | minor. */
int32_t mfk_version(void);

#ifdef __cplusplus
}
#endif

#endif /* MFK_H */
