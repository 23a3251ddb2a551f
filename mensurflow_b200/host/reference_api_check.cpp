// Checks the drop-in at the reference's PUBLIC API: the same calls with Execution::GPU on cuda:0
// tensors (this repository's kernels, through cuda_backend.cpp) and with Execution::CPU (the
// reference's own kernels), compared elementwise. Covers what the reference's test programs do
// not run on a GPU: gemm_strided_batched (the 19 API cases of tests/ops/gemm_batched_test.cpp),
// attention (the cases of tests/ops/softmax_loss_test.cpp test_attention), softmax, bias_add,
// relu and gelu. Prints one line per check and exits non-zero on the first mismatch.
#include "core/dispatcher.hpp"
#include "mensurflow/mensurflow.hpp"

#include <cmath>
#include <cstdint>
#include <iostream>
#include <stdexcept>
#include <string>
#include <vector>

using namespace mensurflow;

namespace {

int checks = 0;

// |gpu - cpu| <= rel * max(|cpu|, magnitude) + abs, elementwise, where magnitude (optional) is
// the scale rounding error is relative to (for a product, sum |a*b|, as the reference's tests
// use); NaN and inf must match exactly.
void require_close(const Tensor& gpu, const Tensor& cpu, double rel, double abs,
                   const std::string& what, const Tensor* magnitude = nullptr) {
    if (gpu.shape() != cpu.shape()) {
        throw std::runtime_error(what + ": shape " + to_string(gpu.shape()) + " vs " +
                                 to_string(cpu.shape()));
    }
    if (gpu.device().type != DeviceType::CUDA) {
        throw std::runtime_error(what + ": the GPU result is not on the CUDA device");
    }
    const auto g = gpu.to_vector<float>();
    const auto c = cpu.to_vector<float>();
    const auto mag = magnitude ? magnitude->to_vector<float>() : std::vector<float>(c.size(), 0.0f);
    for (std::size_t i = 0; i < g.size(); ++i) {
        if (std::isnan(c[i]) || std::isinf(c[i])) {
            if (!(std::isnan(g[i]) == std::isnan(c[i]) && (std::isnan(c[i]) || g[i] == c[i]))) {
                throw std::runtime_error(what + ": entry " + std::to_string(i) + " " +
                                         std::to_string(g[i]) + " vs " + std::to_string(c[i]));
            }
            continue;
        }
        const double bound = rel * std::max<double>(std::fabs(c[i]), mag[i]) + abs;
        if (!(std::fabs(static_cast<double>(g[i]) - c[i]) <= bound)) {
            throw std::runtime_error(what + ": entry " + std::to_string(i) + " " +
                                     std::to_string(g[i]) + " vs " + std::to_string(c[i]));
        }
    }
    ++checks;
    std::cout << "  ok " << what << '\n';
}

Tensor input(Shape shape, std::uint64_t seed, float stddev = 1.0f) {
    return normal(std::move(shape), 0.0f, stddev, seed);
}

void check_batched(Device gpu) {
    struct Case {
        const char* name;
        Shape a, b;
        bool ta, tb;
        float alpha;
        Shape c;
        float beta;
    };
    const Case cases[] = {
        {"plain batch", {3, 4, 5}, {3, 5, 2}, false, false, 1.0f, {}, 0.0f},
        {"shared right-hand side", {4, 3, 5}, {5, 2}, false, false, 1.0f, {}, 0.0f},
        {"shared left-hand side", {3, 5}, {4, 5, 2}, false, false, 1.0f, {}, 0.0f},
        {"broadcast batch dims", {2, 1, 3, 4}, {5, 4, 6}, false, false, 1.0f, {}, 0.0f},
        {"plain matrices", {7, 9}, {9, 4}, false, false, 1.0f, {}, 0.0f},
        {"transpose a", {2, 5, 3}, {2, 5, 4}, true, false, 1.0f, {}, 0.0f},
        {"transpose b", {2, 3, 5}, {2, 4, 5}, false, true, 1.0f, {}, 0.0f},
        {"transpose both", {2, 5, 3}, {1, 4, 5}, true, true, 1.0f, {}, 0.0f},
        {"alpha only", {2, 3, 4}, {2, 4, 5}, false, false, -1.5f, {}, 0.0f},
        {"alpha and full c", {2, 3, 4}, {2, 4, 5}, false, false, 2.0f, {2, 3, 5}, 0.5f},
        {"c broadcast over batch", {4, 3, 4}, {4, 5}, false, false, 1.0f, {3, 5}, -1.0f},
        {"c as a row", {2, 3, 4}, {2, 4, 5}, false, false, 1.0f, {5}, 1.0f},
        {"c given, beta 0", {2, 3, 4}, {2, 4, 5}, false, false, 1.0f, {2, 3, 5}, 0.0f},
        {"many small", {100, 2, 3}, {100, 3, 2}, false, false, 1.0f, {}, 0.0f},
        {"larger", {3, 70, 90}, {3, 90, 60}, false, false, 1.0f, {}, 0.0f},
        {"attention-like", {8, 128, 64}, {8, 256, 64}, false, true, 0.125f, {}, 0.0f},
    };
    std::uint64_t seed = 100;
    for (const Case& t : cases) {
        const Tensor a = input(t.a, seed++), b = input(t.b, seed++);
        const Tensor c = t.c.empty() ? Tensor() : input(t.c, seed++);
        const Tensor* cp = t.c.empty() ? nullptr : &c;
        const Tensor want = gemm_strided_batched(a, b, t.alpha, cp, t.beta, t.ta, t.tb,
                                                 Execution::CPU);
        const Tensor cg = t.c.empty() ? Tensor() : c.to(gpu);
        const Tensor got = gemm_strided_batched(a.to(gpu), b.to(gpu), t.alpha,
                                                t.c.empty() ? nullptr : &cg, t.beta, t.ta, t.tb,
                                                Execution::GPU);
        // the path's 3xTF32 bound: 1e-5 of |alpha| (|A||B|)_ij + |beta c_ij|, plus 1e-6
        const Tensor ca = t.c.empty() ? Tensor() : mensurflow::abs(c, Execution::CPU);
        const Tensor mag = gemm_strided_batched(mensurflow::abs(a, Execution::CPU),
                                                mensurflow::abs(b, Execution::CPU),
                                                std::fabs(t.alpha), t.c.empty() ? nullptr : &ca,
                                                std::fabs(t.beta), t.ta, t.tb, Execution::CPU);
        require_close(got, want, 1e-5, 1e-6, std::string("gemm_strided_batched ") + t.name, &mag);
    }
}

void check_attention(Device gpu) {
    const std::int64_t b = 2, h = 3, lq = 5, lk = 7, d = 8, dv = 4;
    const Tensor q = input({b, h, lq, d}, 21), k = input({b, h, lk, d}, 22),
                 v = input({b, h, lk, dv}, 23);
    std::vector<std::uint8_t> keep(static_cast<std::size_t>(lq * lk));
    for (std::int64_t i = 0; i < lq; ++i) {
        for (std::int64_t j = 0; j < lk; ++j) {
            keep[static_cast<std::size_t>(i * lk + j)] = i != 2 && (i + j) % 3 != 0;
        }
    }
    const Tensor mask = Tensor::from_host(keep.data(), {lq, lk}, DType::Bool);
    const Tensor mask_g = mask.to(gpu);
    struct Case {
        bool use_mask, causal;
        float scale;
        const char* name;
    };
    for (const Case& c : {Case{false, false, 0.0f, "plain"}, Case{true, false, 0.0f, "mask"},
                          Case{false, true, 0.0f, "causal"}, Case{true, true, 0.5f, "both"}}) {
        const Tensor want = attention(q, k, v, c.use_mask ? &mask : nullptr, c.causal, c.scale,
                                      Execution::CPU);
        const Tensor got = attention(q.to(gpu), k.to(gpu), v.to(gpu),
                                     c.use_mask ? &mask_g : nullptr, c.causal, c.scale,
                                     Execution::GPU);
        require_close(got, want, 1e-4, 1e-6, std::string("attention ") + c.name);
    }
    const Tensor q2 = input({4, 256, 64}, 31, 0.125f), k2 = input({4, 256, 64}, 32, 0.125f),
                 v2 = input({4, 256, 64}, 33, 0.125f);
    require_close(attention(q2.to(gpu), k2.to(gpu), v2.to(gpu), nullptr, true, 0.0f,
                            Execution::GPU),
                  attention(q2, k2, v2, nullptr, true, 0.0f, Execution::CPU), 1e-4, 1e-6,
                  "attention causal 4x256x64");
}

void check_elementwise(Device gpu) {
    const Tensor x = input({64, 96}, 41, 3.0f);
    const Tensor bias = input({96}, 42, 0.1f);
    require_close(bias_add(x.to(gpu), bias.to(gpu), Execution::GPU),
                  bias_add(x, bias, Execution::CPU), 0.0, 0.0, "bias_add (bit-exact)");
    require_close(relu(x.to(gpu), Execution::GPU), relu(x, Execution::CPU), 0.0, 0.0,
                  "relu (bit-exact)");
    require_close(gelu(x.to(gpu), false, Execution::GPU), gelu(x, false, Execution::CPU), 2.4e-7,
                  1e-30, "gelu exact (1 ulp)");
    require_close(gelu(x.to(gpu), true, Execution::GPU), gelu(x, true, Execution::CPU), 2.4e-7,
                  1e-30, "gelu tanh (1 ulp)");
    for (int axis : {-1, 0}) {
        require_close(softmax(x.to(gpu), axis, Execution::GPU), softmax(x, axis, Execution::CPU),
                      5e-7, 1e-30, "softmax axis " + std::to_string(axis) + " (4 ulp)");
    }
    const Tensor ax = mensurflow::abs(x, Execution::CPU);
    const Tensor mag = matmul(ax, ax.transpose(0, 1), Execution::CPU);
    require_close(matmul(x.to(gpu), x.transpose(0, 1).contiguous().to(gpu), Execution::GPU),
                  matmul(x, x.transpose(0, 1), Execution::CPU), 1e-5, 1e-6, "matmul 64x96x64",
                  &mag);
}

// Device-side packing of views: the reference's public copy() on a CUDA tensor, and OpId::Copy
// dispatched with a strided CUDA view as its input — the call Tensor::contiguous() makes once it
// routes CUDA views through OpId::Copy instead of a host round trip — against
// the CPU's Tensor::contiguous() of the same view. Copies are exact.
void check_copy(Device gpu) {
    const Tensor x = input({6, 7, 8}, 51);
    const Tensor xg = x.to(gpu);
    require_close(copy(xg, Execution::GPU), copy(x, Execution::CPU), 0.0, 0.0, "copy");
    struct View {
        const char* name;
        Tensor (*make)(const Tensor&);
    };
    const View views[] = {
        {"transpose", [](const Tensor& t) { return t.view({42, 8}).transpose(0, 1); }},
        {"permute 2,0,1", [](const Tensor& t) { return t.permute({2, 0, 1}); }},
        {"permute 1,2,0", [](const Tensor& t) { return t.permute({1, 2, 0}); }},
        {"column slice", [](const Tensor& t) { return t.slice(2, 1, 7); }},
        {"stepped slices", [](const Tensor& t) { return t.slice(0, 1, 6, 2).slice(2, 0, 8, 3); }},
        {"expand", [](const Tensor& t) { return t.slice(0, 0, 1).expand({4, 6, 7, 8}); }},
        {"transpose + slice", [](const Tensor& t) { return t.transpose(0, 1).slice(2, 3, 4); }},
    };
    for (const View& v : views) {
        const Tensor view_g = v.make(xg);
        Tensor out = Tensor::empty(view_g.shape(), DType::F32, gpu);
        detail::OpArgs args{{view_g}, {out}};
        detail::dispatch(detail::OpId::Copy, args, Execution::GPU);
        require_close(out, v.make(x).contiguous(), 0.0, 0.0,
                      std::string("contiguous on the device: ") + v.name);
    }
}

} // namespace

int main() {
    try {
        const Device gpu = parse_device("cuda:0");
        if (!device_available(gpu)) {
            std::cout << "reference_api_check: no CUDA device, nothing checked\n";
            return 0;
        }
        check_batched(gpu);
        check_attention(gpu);
        check_elementwise(gpu);
        check_copy(gpu);
        std::cout << "reference_api_check passed (" << checks << " checks on " << to_string(gpu)
                  << ")\n";
        return 0;
    } catch (const std::exception& e) {
        std::cerr << "reference_api_check FAILED: " << e.what() << '\n';
        return 1;
    }
}
