// The reference-side binding: a CUDA backend for Mensurflow's dispatcher whose kernels are the
// sm_100a library behind include/mfk.h. It replaces src/backends/cuda/backend.cpp of
// bakir004/mensurflow (same Backend / Buffer / Stream classes, same registration entry point
// `register_cuda_backend`, src/core/registry.hpp:45), with no cuBLAS.
//
// Each KernelFn unpacks OpArgs (src/core/dispatcher.hpp:164-197) into the C ABI's plain
// descriptors. Ops have validated shapes before dispatch, so the adapters only translate layouts
// and turn a non-zero status into the exceptions the reference uses (std::invalid_argument for
// argument errors, std::runtime_error otherwise; src/backends/cuda/backend.cpp:22-34).
//
// Built only against the reference's headers (include/, src/). With the op-layer patches of
// host/patches applied to those sources (MENSURFLOW_HAS_OPID_GEMM), it also registers the
// one-kernel gemm (OpId::Gemm, with bias and activation fused) and bias_add's bias gradient
// (OpId::BiasGrad) and attention in one kernel (OpId::Attention), and provides the
// device-to-device copy that Tensor::to() uses between GPUs.
#include "backends/backend.hpp"
#include "core/dispatcher.hpp"
#include "core/registry.hpp"
#include "core/tensor_access.hpp"
#include "cuda_stream.hpp"
#include "mfk.h"

#include <cuda_runtime.h>

#include <cstddef>
#include <memory>
#include <mutex>
#include <stdexcept>
#include <string>
#include <vector>

namespace mensurflow::detail {

namespace {

void check(cudaError_t status, const char* what) {
    if (status != cudaSuccess) {
        throw std::runtime_error(std::string("CUDA ") + what + " failed: " +
                                 cudaGetErrorString(status));
    }
}

void check_mfk(int status, const char* op) {
    if (status == MFK_OK) {
        return;
    }
    const std::string what = std::string(op) + ": " + mfk_status_string(status);
    if (status == MFK_ERR_INVALID_ARGUMENT) {
        throw std::invalid_argument(what);
    }
    throw std::runtime_error(what + " " + mfk_last_cuda_error());
}

class CudaBuffer final : public Buffer {
  public:
    CudaBuffer(int device, std::size_t bytes) : device_(device), size_(bytes) {
        if (bytes > 0) {
            check(cudaSetDevice(device), "cudaSetDevice");
            check(cudaMalloc(&data_, bytes), "cudaMalloc");
        }
    }
    ~CudaBuffer() override {
        if (data_ != nullptr) {
            cudaSetDevice(device_);
            cudaFree(data_);
        }
    }
    CudaBuffer(const CudaBuffer&) = delete;
    CudaBuffer& operator=(const CudaBuffer&) = delete;
    std::size_t size() const override { return size_; }
    void* native() const override { return data_; }

  private:
    int device_;
    std::size_t size_;
    void* data_ = nullptr;
};

// One non-blocking stream per device; copies complete before they return (Stream contract,
// src/backends/backend.hpp:32-44).
class CudaStream final : public Stream {
  public:
    explicit CudaStream(int device) : device_(device) {
        activate();
        check(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking), "cudaStreamCreate");
    }
    ~CudaStream() override {
        cudaSetDevice(device_);
        cudaStreamDestroy(stream_);
    }
    CudaStream(const CudaStream&) = delete;
    CudaStream& operator=(const CudaStream&) = delete;

    void activate() const { check(cudaSetDevice(device_), "cudaSetDevice"); }
    cudaStream_t raw() const { return stream_; }

    void copy_h2d(Buffer& dst, std::size_t offset, const void* src, std::size_t bytes) override {
        activate();
        check(cudaMemcpyAsync(static_cast<std::byte*>(dst.native()) + offset, src, bytes,
                              cudaMemcpyHostToDevice, stream_),
              "cudaMemcpyAsync (host to device)");
        synchronize();
    }
    void copy_d2h(void* dst, const Buffer& src, std::size_t offset, std::size_t bytes) override {
        activate();
        check(cudaMemcpyAsync(dst, static_cast<const std::byte*>(src.native()) + offset, bytes,
                              cudaMemcpyDeviceToHost, stream_),
              "cudaMemcpyAsync (device to host)");
        synchronize();
    }
    void synchronize() override {
        activate();
        check(cudaStreamSynchronize(stream_), "cudaStreamSynchronize");
    }

  private:
    int device_;
    cudaStream_t stream_ = nullptr;
};

CudaStream& cuda(Stream& stream) {
    auto& s = static_cast<CudaStream&>(stream);
    s.activate();
    return s;
}

// OpId::Matmul: a [m, k] and b [k, n] with any strides (the op makes them contiguous on
// non-CPU devices today, src/ops/blas.cpp:216-218; strided views work as they are), out
// contiguous [m, n]. Same contract as the CPU adapter (src/backends/cpu/backend.cpp:131-164).
void matmul_kernel(const OpArgs& args, Stream& stream) {
    auto& s = cuda(stream);
    const Tensor& a = args.inputs[0];
    const Tensor& b = args.inputs[1];
    const Tensor& out = args.outputs[0];
    mfk_gemm_desc d{};
    d.a = TensorAccess::data<float>(a);
    d.a_rs = a.strides()[0];
    d.a_cs = a.strides()[1];
    d.b = TensorAccess::data<float>(b);
    d.b_rs = b.strides()[0];
    d.b_cs = b.strides()[1];
    d.c = TensorAccess::data<float>(out);
    d.ldc = out.size(1);
    d.m = a.size(0);
    d.n = b.size(1);
    d.k = a.size(1);
    d.alpha = 1.0f;
    d.beta = 0.0f;
    d.activation = MFK_ACT_NONE;
    d.precision = MFK_PRECISION_DEFAULT;
    check_mfk(mfk_gemm_f32(&d, s.raw()), "matmul");
}

// OpId::GemmBatched: views with the full batch shape (broadcast batch dims have stride 0), a
// contiguous output and, when beta != 0, a contiguous c of the output's shape (the op's
// contract, src/ops/blas.cpp:378-392). Matrix offsets come from the same odometer walk as the
// CPU adapter (src/backends/cpu/backend.cpp:251-270).
void gemm_batched_kernel(const OpArgs& args, Stream& stream) {
    auto& s = cuda(stream);
    const Tensor& a = args.inputs[0];
    const Tensor& b = args.inputs[1];
    const Tensor& out = args.outputs[0];
    const int batch_dims = out.dim() - 2;
    std::int64_t batch = 1;
    for (int d = 0; d < batch_dims; ++d) {
        batch *= out.size(d);
    }
    std::vector<std::int64_t> a_offsets(static_cast<std::size_t>(batch));
    std::vector<std::int64_t> b_offsets(static_cast<std::size_t>(batch));
    std::vector<std::int64_t> index(static_cast<std::size_t>(batch_dims), 0);
    std::int64_t a_offset = 0, b_offset = 0;
    for (std::int64_t i = 0; i < batch; ++i) {
        a_offsets[static_cast<std::size_t>(i)] = a_offset;
        b_offsets[static_cast<std::size_t>(i)] = b_offset;
        for (int d = batch_dims - 1; d >= 0; --d) {
            const auto du = static_cast<std::size_t>(d);
            if (++index[du] < out.size(d)) {
                a_offset += a.strides()[du];
                b_offset += b.strides()[du];
                break;
            }
            a_offset -= (index[du] - 1) * a.strides()[du];
            b_offset -= (index[du] - 1) * b.strides()[du];
            index[du] = 0;
        }
    }
    const auto bd_ = static_cast<std::size_t>(batch_dims);
    const std::int64_t m = out.size(-2), n = out.size(-1);
    mfk_gemm_desc d{};
    d.a = TensorAccess::data<float>(a);
    d.a_rs = a.strides()[bd_];
    d.a_cs = a.strides()[bd_ + 1];
    d.b = TensorAccess::data<float>(b);
    d.b_rs = b.strides()[bd_];
    d.b_cs = b.strides()[bd_ + 1];
    d.c = TensorAccess::data<float>(out);
    d.ldc = n;
    d.m = m;
    d.n = n;
    d.k = a.size(-1);
    d.alpha = args.alpha;
    d.beta = args.inputs.size() > 2 ? args.beta : 0.0f;
    if (args.inputs.size() > 2) {
        d.c_in = TensorAccess::data<float>(args.inputs[2]);
        d.c_in_rs = n;
        d.c_in_cs = 1;
    }
    d.activation = MFK_ACT_NONE;
    d.precision = MFK_PRECISION_DEFAULT;
    mfk_batch_desc bd{};
    bd.batch = batch;
    bd.a_offsets = a_offsets.data();
    bd.b_offsets = b_offsets.data();
    bd.c_in_stride = m * n;
    bd.c_stride = m * n;
    check_mfk(mfk_gemm_strided_batched_f32(&d, &bd, s.raw()), "gemm_strided_batched");
}

#ifdef MENSURFLOW_HAS_OPID_GEMM
// OpId::Gemm, the whole of gemm in one kernel (patched src/ops/blas.cpp): inputs {op(a), op(b)}
// as views with any strides, then c when beta != 0, then the bias when with_bias; out contiguous
// [m, n]; alpha, beta and the activation in OpArgs. alpha * op(a) op(b), + beta * c, + bias and
// the activation are rounded in the order gemm's composed ops and bias_add round them
// (src/ops/blas.cpp:246-260, src/ops/elementwise.cpp:251-258).
void gemm_kernel(const OpArgs& args, Stream& stream) {
    auto& s = cuda(stream);
    const Tensor& a = args.inputs[0];
    const Tensor& b = args.inputs[1];
    const Tensor& out = args.outputs[0];
    mfk_gemm_desc d{};
    d.a = TensorAccess::data<float>(a);
    d.a_rs = a.strides()[0];
    d.a_cs = a.strides()[1];
    d.b = TensorAccess::data<float>(b);
    d.b_rs = b.strides()[0];
    d.b_cs = b.strides()[1];
    d.c = TensorAccess::data<float>(out);
    d.ldc = out.size(1);
    d.m = out.size(0);
    d.n = out.size(1);
    d.k = a.size(1);
    d.alpha = args.alpha;
    const std::size_t with_c = args.inputs.size() - (args.with_bias ? 1 : 0) > 2 ? 1 : 0;
    d.beta = with_c ? args.beta : 0.0f;
    if (with_c) {
        const Tensor& c = args.inputs[2];
        d.c_in = TensorAccess::data<float>(c);
        d.c_in_rs = c.strides()[0];
        d.c_in_cs = c.strides()[1];
    }
    if (args.with_bias) {
        d.bias = TensorAccess::data<float>(args.inputs.back());
    }
    switch (args.activation) {
    case 0:
        d.activation = MFK_ACT_NONE;
        break;
    case 1:
        d.activation = MFK_ACT_RELU;
        break;
    case 2:
        d.activation = MFK_ACT_GELU;
        break;
    case 3:
        d.activation = MFK_ACT_GELU_TANH;
        break;
    default:
        throw std::invalid_argument("gemm: unknown activation");
    }
    d.precision = MFK_PRECISION_DEFAULT;
    check_mfk(mfk_gemm_f32(&d, s.raw()), "gemm");
}

// OpId::Attention (patched src/ops/attention.cpp): q, k, v of one contiguous shape
// [..., L, 128], out of that shape, alpha the scale, `causal` the mask. One kernel in 3xTF32
// (whatever the process-wide precision: the op promises the reference's fp32 results).
void attention_kernel(const OpArgs& args, Stream& stream) {
    auto& s = cuda(stream);
    const Tensor& q = args.inputs[0];
    const Tensor& out = args.outputs[0];
    const std::int64_t len = q.size(-2), depth = q.size(-1);
    const std::int64_t heads = len * depth > 0 ? q.numel() / (len * depth) : 0;
    if (args.inputs.size() > 3) {
        // the Bool keep mask, expanded to the scores [..., len, len] by the op with one stride
        // over the batch dimensions (the innermost one's; 0 when all are broadcast)
        const Tensor& keep = args.inputs[3];
        const Strides& st = keep.strides();
        const std::size_t nb = st.size() - 2;
        check_mfk(mfk_attention_masked_f32(
                      TensorAccess::data<float>(q), TensorAccess::data<float>(args.inputs[1]),
                      TensorAccess::data<float>(args.inputs[2]),
                      TensorAccess::data<std::uint8_t>(keep), nb > 0 ? st[nb - 1] : 0, st[nb],
                      st[nb + 1], TensorAccess::data<float>(out), heads, len, depth,
                      args.causal ? 1 : 0, args.alpha, s.raw()),
                  "attention");
        return;
    }
    check_mfk(mfk_attention_f32(TensorAccess::data<float>(q),
                                TensorAccess::data<float>(args.inputs[1]),
                                TensorAccess::data<float>(args.inputs[2]),
                                TensorAccess::data<float>(out), heads, len, depth,
                                args.causal ? 1 : 0, args.alpha, s.raw()),
              "attention");
}

// OpId::BiasGrad (patched bias_add backward, src/ops/elementwise.cpp:263-283): the column sums
// of a contiguous [rows, features] gradient in row order, the host loop's bits.
void bias_grad_kernel(const OpArgs& args, Stream& stream) {
    auto& s = cuda(stream);
    const Tensor& g = args.inputs[0];
    const std::int64_t cols = g.dim() > 0 ? g.size(-1) : 1;
    const std::int64_t rows = cols > 0 ? g.numel() / cols : 0;
    check_mfk(mfk_bias_grad_f32(TensorAccess::data<float>(g), rows, cols, cols,
                                TensorAccess::data<float>(args.outputs[0]), s.raw()),
              "bias_grad");
}
#endif

// OpId::Dot: contiguous 1-D x and y, a 0-d output on the device (src/ops/blas.cpp:41-68; the CPU
// adapter, src/backends/cpu/backend.cpp:89-93, writes the same double-accumulated sum).
void dot_kernel(const OpArgs& args, Stream& stream) {
    auto& s = cuda(stream);
    const Tensor& x = args.inputs[0];
    check_mfk(mfk_dot_f32(TensorAccess::data<float>(x), TensorAccess::data<float>(args.inputs[1]),
                          x.numel(), TensorAccess::data<float>(args.outputs[0]), s.raw()),
              "dot");
}

// OpId::Scal: out = alpha * x over a contiguous 1-D x (src/ops/blas.cpp:70-79; CPU adapter
// src/backends/cpu/backend.cpp:95-98).
void scal_kernel(const OpArgs& args, Stream& stream) {
    auto& s = cuda(stream);
    const Tensor& out = args.outputs[0];
    check_mfk(mfk_scal_f32(args.alpha, TensorAccess::data<float>(args.inputs[0]),
                           TensorAccess::data<float>(out), out.numel(), s.raw()),
              "scal");
}

// OpId::Add / Sub / Mul / Div: the op packs both inputs to the output's shape
// (src/ops/elementwise.cpp:158-225), as the CPU adapter reads them (backend.cpp:595-598).
template <int Op>
void binary_kernel(const OpArgs& args, Stream& stream) {
    auto& s = cuda(stream);
    const Tensor& out = args.outputs[0];
    static const char* const names[] = {"add", "sub", "mul", "div"};
    check_mfk(mfk_binary_f32(Op, TensorAccess::data<float>(args.inputs[0]),
                             TensorAccess::data<float>(args.inputs[1]),
                             TensorAccess::data<float>(out), out.numel(), s.raw()),
              names[Op]);
}

// OpId::BiasAdd: contiguous x [batch, features], bias [features] (backend.cpp:762-767).
void bias_add_kernel(const OpArgs& args, Stream& stream) {
    auto& s = cuda(stream);
    const Tensor& out = args.outputs[0];
    check_mfk(mfk_bias_act_f32(TensorAccess::data<float>(args.inputs[0]),
                               TensorAccess::data<float>(args.inputs[1]),
                               TensorAccess::data<float>(out), out.size(0), out.size(1),
                               MFK_ACT_NONE, s.raw()),
              "bias_add");
}

template <int Activation>
void activation_kernel(const OpArgs& args, Stream& stream) {
    auto& s = cuda(stream);
    const Tensor& out = args.outputs[0];
    const int act = (Activation == MFK_ACT_GELU && args.approximate) ? MFK_ACT_GELU_TANH
                                                                     : Activation;
    check_mfk(mfk_bias_act_f32(TensorAccess::data<float>(args.inputs[0]), nullptr,
                               TensorAccess::data<float>(out), 1, out.numel(), act, s.raw()),
              Activation == MFK_ACT_RELU ? "relu" : "gelu");
}

// OpId::Gemv: contiguous a [rows, cols], x, optional y (backend.cpp:120-125).
void gemv_kernel(const OpArgs& args, Stream& stream) {
    auto& s = cuda(stream);
    const Tensor& a = args.inputs[0];
    const float* y0 = args.inputs.size() > 2 ? TensorAccess::data<float>(args.inputs[2]) : nullptr;
    check_mfk(mfk_gemv_f32(TensorAccess::data<float>(a), a.size(0), a.size(1), a.size(1),
                           args.transpose ? 1 : 0, TensorAccess::data<float>(args.inputs[1]), 1,
                           args.alpha, y0 != nullptr ? args.beta : 0.0f, y0,
                           TensorAccess::data<float>(args.outputs[0]), s.raw()),
              "gemv");
}

// OpId::Copy: out = a packed copy of the input. The op hands over a contiguous input
// (src/ops/blas.cpp:106-117); a strided input is gathered in the same launch, which is what the
// patched Tensor::contiguous() dispatches for a CUDA view instead of the unpatched host round
// trip (src/core/tensor.cpp:224-229). Same contract as the CPU adapter
// (src/backends/cpu/backend.cpp:110-113).
void copy_kernel(const OpArgs& args, Stream& stream) {
    auto& s = cuda(stream);
    const Tensor& x = args.inputs[0];
    const Tensor& out = args.outputs[0];
    if (x.is_contiguous()) {
        check_mfk(mfk_copy_f32(TensorAccess::data<float>(x), TensorAccess::data<float>(out),
                               out.numel(), s.raw()),
                  "copy");
        return;
    }
    const std::vector<std::int64_t> shape(x.shape().begin(), x.shape().end());
    const std::vector<std::int64_t> strides(x.strides().begin(), x.strides().end());
    check_mfk(mfk_strided_copy_f32(TensorAccess::data<float>(x), shape.data(), strides.data(),
                                   x.dim(), TensorAccess::data<float>(out), s.raw()),
              "contiguous");
}

// OpId::Matvec: contiguous a [m, k], x [k].
void matvec_kernel(const OpArgs& args, Stream& stream) {
    auto& s = cuda(stream);
    const Tensor& a = args.inputs[0];
    check_mfk(mfk_matvec_f32(TensorAccess::data<float>(a), a.size(0), a.size(1),
                             TensorAccess::data<float>(args.inputs[1]),
                             TensorAccess::data<float>(args.outputs[0]), s.raw()),
              "matvec");
}

// OpId::Softmax / LogSoftmax: a contiguous input, the axis in OpArgs (src/ops/softmax.cpp:33-43),
// lines around that axis as the CPU adapter's lines_around (src/backends/cpu/backend.cpp:549).
template <int Log>
void softmax_kernel(const OpArgs& args, Stream& stream) {
    auto& s = cuda(stream);
    const Tensor& x = args.inputs[0];
    std::int64_t outer = 1, length = 1, inner = 1;
    if (x.dim() > 0) {
        for (int d = 0; d < x.dim(); ++d) {
            if (d < args.axis) {
                outer *= x.size(d);
            } else if (d == args.axis) {
                length = x.size(d);
            } else {
                inner *= x.size(d);
            }
        }
    }
    check_mfk(mfk_softmax_f32(TensorAccess::data<float>(x),
                              TensorAccess::data<float>(args.outputs[0]), outer, length, inner,
                              Log, s.raw()),
              Log ? "log_softmax" : "softmax");
}

// OpId::Where: values {x, y} then the Bool condition, all expanded and packed by the op
// (src/ops/elementwise.cpp:455-481), as the CPU adapter reads them (backend.cpp:625-630).
void where_kernel(const OpArgs& args, Stream& stream) {
    auto& s = cuda(stream);
    const Tensor& out = args.outputs[0];
    check_mfk(mfk_where_f32(TensorAccess::data<std::uint8_t>(args.inputs[2]),
                            TensorAccess::data<float>(args.inputs[0]),
                            TensorAccess::data<float>(args.inputs[1]),
                            TensorAccess::data<float>(out), out.numel(), s.raw()),
              "where");
}

class CudaBackend final : public Backend {
  public:
    CudaBackend() {
        int count = 0;
        count_ = cudaGetDeviceCount(&count) == cudaSuccess ? count : 0;
        streams_.resize(static_cast<std::size_t>(count_));
    }
    DeviceType type() const override { return DeviceType::CUDA; }
    int device_count() const override { return count_; }
    DeviceInfo info(int index) const override {
        cudaDeviceProp props;
        check(cudaGetDeviceProperties(&props, index), "cudaGetDeviceProperties");
        return {props.name, props.totalGlobalMem};
    }
    std::shared_ptr<Buffer> allocate(int index, std::size_t bytes) override {
        return std::make_shared<CudaBuffer>(index, bytes);
    }
    Stream& stream(int index) override {
        std::lock_guard<std::mutex> lock(mutex_);
        auto& slot = streams_[static_cast<std::size_t>(index)];
        if (!slot) {
            slot = std::make_unique<CudaStream>(index);
        }
        return *slot;
    }
    void register_kernels(Dispatcher& dispatcher) override {
        const auto key = [](OpId op) { return KernelKey{op, DeviceType::CUDA, DType::F32}; };
        dispatcher.register_kernel(key(OpId::Matmul), matmul_kernel);
        dispatcher.register_kernel(key(OpId::GemmBatched), gemm_batched_kernel);
        dispatcher.register_kernel(key(OpId::BiasAdd), bias_add_kernel);
        dispatcher.register_kernel(key(OpId::Relu), activation_kernel<MFK_ACT_RELU>);
        dispatcher.register_kernel(key(OpId::Gelu), activation_kernel<MFK_ACT_GELU>);
        dispatcher.register_kernel(key(OpId::Gemv), gemv_kernel);
        dispatcher.register_kernel(key(OpId::Matvec), matvec_kernel);
        dispatcher.register_kernel(key(OpId::Softmax), softmax_kernel<0>);
        dispatcher.register_kernel(key(OpId::LogSoftmax), softmax_kernel<1>);
        dispatcher.register_kernel(key(OpId::Where), where_kernel);
        dispatcher.register_kernel(key(OpId::Copy), copy_kernel);
        dispatcher.register_kernel(key(OpId::Dot), dot_kernel);
        dispatcher.register_kernel(key(OpId::Scal), scal_kernel);
        dispatcher.register_kernel(key(OpId::Add), binary_kernel<MFK_BINARY_ADD>);
        dispatcher.register_kernel(key(OpId::Sub), binary_kernel<MFK_BINARY_SUB>);
        dispatcher.register_kernel(key(OpId::Mul), binary_kernel<MFK_BINARY_MUL>);
        dispatcher.register_kernel(key(OpId::Div), binary_kernel<MFK_BINARY_DIV>);
#ifdef MENSURFLOW_HAS_OPID_GEMM
        dispatcher.register_kernel(key(OpId::Gemm), gemm_kernel);
        dispatcher.register_kernel(key(OpId::BiasGrad), bias_grad_kernel);
        dispatcher.register_kernel(key(OpId::Attention), attention_kernel);
#endif
    }

  private:
    int count_ = 0;
    std::mutex mutex_;
    std::vector<std::unique_ptr<CudaStream>> streams_;
};

} // namespace

void register_cuda_backend(Registry& registry) { registry.add(std::make_unique<CudaBackend>()); }

void* cuda_stream_handle(Stream& stream) { return cuda(stream).raw(); }

// Tensor::to() between CUDA devices (patched src/core/tensor.cpp): one stream-ordered copy on the
// source device's stream, after the work that produced src, then a wait, as the host path's
// copy_d2h + copy_h2d pair would have waited.
bool cuda_device_copy(void* dst, int dst_index, const void* src, int src_index,
                      std::size_t bytes) {
    Backend* backend = Registry::instance().find(DeviceType::CUDA);
    if (backend == nullptr) {
        return false;
    }
    auto& s = cuda(backend->stream(src_index));
    check_mfk(mfk_copy_peer(dst, dst_index, src, src_index, static_cast<std::int64_t>(bytes),
                            s.raw()),
              "Tensor::to");
    s.synchronize();
    return true;
}

} // namespace mensurflow::detail
