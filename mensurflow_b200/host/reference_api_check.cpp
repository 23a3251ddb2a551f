// Checks the drop-in at the reference's PUBLIC API: the same calls with Execution::GPU on cuda:0
// tensors (this repository's kernels, through cuda_backend.cpp) and with Execution::CPU (the
// reference's own kernels), compared elementwise. Covers what the reference's test programs do
// not run on a GPU: gemm_strided_batched (the 19 API cases of tests/ops/gemm_batched_test.cpp),
// attention (the cases of tests/ops/softmax_loss_test.cpp test_attention), softmax, bias_add,
// relu and gelu; and, with the op-layer patches applied, gemm in one dispatch (C1 and the C2 call
// of the benchmark configs, the fused bias/activation overload), dot / scal / add / sub / mul /
// div, the bias and matmul gradients on the device, Tensor::contiguous() of CUDA views and
// Tensor::to() between GPUs. Prints one line per check and exits non-zero on the first mismatch.
#include "core/autograd.hpp"
#include "core/dispatcher.hpp"
#include "core/registry.hpp"
#include "core/tensor_access.hpp"
#include "cuda_stream.hpp"
#include "mensurflow/mensurflow.hpp"
#include "mfk.h"

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
    // head dim 128 without a mask: the patched attention dispatches the one-kernel path
    {
        const Tensor q3 = input({2, 4, 384, 128}, 34, 0.088f), k3 = input({2, 4, 384, 128}, 35, 0.088f),
                     v3 = input({2, 4, 384, 128}, 36, 0.088f);
        // a first call on the device may run the one-time tf32 truncation check as well
        attention(q3.to(gpu), k3.to(gpu), v3.to(gpu), nullptr, true, 0.0f, Execution::GPU);
        for (bool causal : {true, false}) {
            const std::int64_t launches = mfk_launch_count();
            const Tensor got = attention(q3.to(gpu), k3.to(gpu), v3.to(gpu), nullptr, causal, 0.0f,
                                         Execution::GPU);
            const std::int64_t ran = mfk_launch_count() - launches;
            // the attention kernel alone (Q, K and V are split inside it); the composed path
            // would run two batched GEMMs with their packing passes, where and softmax
            if (ran != 1) {
                throw std::runtime_error("attention with head dim 128 ran " + std::to_string(ran) +
                                         " kernels, not the fused path's 1");
            }
            require_close(got, attention(q3, k3, v3, nullptr, causal, 0.0f, Execution::CPU), 1e-4,
                          1e-6, causal ? "attention in one kernel, causal 2x4x384x128"
                                       : "attention in one kernel 2x4x384x128");
        }
        // with a Bool mask shared by every head (one query masked out entirely, so its row is
        // zeros): the one kernel's masked form, in one launch as well
        std::vector<std::uint8_t> keep3(static_cast<std::size_t>(384 * 384));
        for (std::int64_t i = 0; i < 384; ++i) {
            for (std::int64_t j = 0; j < 384; ++j) {
                keep3[static_cast<std::size_t>(i * 384 + j)] = i != 5 && (i * 7 + j) % 5 != 0;
            }
        }
        const Tensor mask3 = Tensor::from_host(keep3.data(), {384, 384}, DType::Bool);
        const Tensor mask3_g = mask3.to(gpu);
        for (bool causal : {true, false}) {
            const std::int64_t launches = mfk_launch_count();
            const Tensor got = attention(q3.to(gpu), k3.to(gpu), v3.to(gpu), &mask3_g, causal,
                                         0.0f, Execution::GPU);
            const std::int64_t ran = mfk_launch_count() - launches;
            if (ran != 1) {
                throw std::runtime_error("attention with a mask and head dim 128 ran " +
                                         std::to_string(ran) + " kernels, not the fused path's 1");
            }
            require_close(got, attention(q3, k3, v3, &mask3, causal, 0.0f, Execution::CPU), 1e-4,
                          1e-6, causal ? "attention in one kernel with a mask, causal 2x4x384x128"
                                       : "attention in one kernel with a mask 2x4x384x128");
        }
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

// Device-side packing of views: the reference's public copy() on a CUDA tensor, OpId::Copy
// dispatched with a strided CUDA view as its input, and the patched Tensor::contiguous() of the
// view (which dispatches that same Copy on the device, so kernels of this library run and no host
// round trip happens), each against the CPU's Tensor::contiguous() of the same view. Exact.
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
        const std::int64_t launches = mfk_launch_count();
        const Tensor packed = v.make(xg).contiguous();
        if (mfk_launch_count() == launches) {
            throw std::runtime_error(std::string("Tensor::contiguous() of the ") + v.name +
                                     " view ran no device kernel");
        }
        require_close(packed, v.make(x).contiguous(), 0.0, 0.0,
                      std::string("Tensor::contiguous() of a CUDA view: ") + v.name);
    }
}

// The magnitude the 3xTF32 bound is relative to: |alpha| (|op(a)| |op(b)|) + |beta c| (+ |bias|).
Tensor gemm_magnitude(const Tensor& a, const Tensor& b, float alpha, const Tensor* c, float beta,
                      bool ta, bool tb, const Tensor* bias = nullptr) {
    const Tensor ca = c ? mensurflow::abs(*c, Execution::CPU) : Tensor();
    Tensor mag = gemm(mensurflow::abs(a, Execution::CPU), mensurflow::abs(b, Execution::CPU),
                      std::fabs(alpha), c ? &ca : nullptr, std::fabs(beta), ta, tb,
                      Execution::CPU);
    if (bias != nullptr) {
        mag = bias_add(mag, mensurflow::abs(*bias, Execution::CPU), Execution::CPU);
    }
    return mag;
}

// gemm through the reference's public API in one dispatch (OpId::Gemm): C1 whole, the headline
// C2 call on sampled row blocks, the fused bias/activation overload, and the cases of the
// reference's gemm test shapes (transposes, alpha/beta, c given with beta 0, k = 0).
void check_gemm(Device gpu) {
    {
        // C1: 1024^3, A and B uniform[-1, 1) from seed 0, C zero, alpha 1, beta 0
        const std::int64_t n = 1024;
        const Tensor a = uniform({n, n}, -1.0f, 1.0f, 0, 0);
        const Tensor b = uniform({n, n}, -1.0f, 1.0f, 0, static_cast<std::uint64_t>(n * n));
        const Tensor c = Tensor::zeros({n, n}, DType::F32);
        const Tensor cg = c.to(gpu);
        const std::int64_t launches = mfk_launch_count();
        const Tensor got = gemm(a.to(gpu), b.to(gpu), 1.0f, &cg, 0.0f, false, false,
                                Execution::GPU);
        if (mfk_launch_count() - launches < 1) {
            throw std::runtime_error("gemm on CUDA launched none of this library's kernels");
        }
        const Tensor mag = gemm_magnitude(a, b, 1.0f, &c, 0.0f, false, false);
        require_close(got, gemm(a, b, 1.0f, &c, 0.0f, false, false, Execution::CPU), 1e-5, 1e-6,
                      "gemm C1 1024^3 (one dispatch)", &mag);
    }
    {
        // C2: gemm(a, b, 0.5, &c, 1.0, false, true) + bias_add at 8192^3, A, B, C normal(0, 1)
        // and bias uniform[-0.1, 0.1) from seed 1; row blocks compared with the CPU's gemm +
        // bias_add on the same rows
        const std::int64_t n = 8192;
        const auto nn = static_cast<std::uint64_t>(n * n);
        const Tensor a = normal({n, n}, 0.0f, 1.0f, 1, 0);
        const Tensor b = normal({n, n}, 0.0f, 1.0f, 1, nn);
        const Tensor c = normal({n, n}, 0.0f, 1.0f, 1, 2 * nn);
        const Tensor bias = uniform({n}, -0.1f, 0.1f, 1, 3 * nn);
        const Tensor ag = a.to(gpu), bg = b.to(gpu), cg = c.to(gpu), biasg = bias.to(gpu);
        const Tensor two_calls =
            bias_add(gemm(ag, bg, 0.5f, &cg, 1.0f, false, true, Execution::GPU), biasg,
                     Execution::GPU);
        const Tensor fused = gemm(ag, bg, 0.5f, &cg, 1.0f, false, true, &biasg,
                                  GemmActivation::None, Execution::GPU);
        require_close(fused, two_calls, 0.0, 0.0,
                      "gemm + bias_add C2 8192^3: fused overload equals the two calls");
        for (std::int64_t r0 : {std::int64_t{0}, std::int64_t{4064}, n - 32}) {
            const Tensor a_rows = a.slice(0, r0, r0 + 32), c_rows = c.slice(0, r0, r0 + 32);
            const Tensor want =
                bias_add(gemm(a_rows, b, 0.5f, &c_rows, 1.0f, false, true, Execution::CPU), bias,
                         Execution::CPU);
            const Tensor mag = gemm_magnitude(a_rows, b, 0.5f, &c_rows, 1.0f, false, true, &bias);
            require_close(two_calls.slice(0, r0, r0 + 32), want, 1e-5, 1e-6,
                          "gemm + bias_add C2 8192^3 rows " + std::to_string(r0) + "..+32", &mag);
        }
    }
    {
        // the fused overload with an activation (C3's first layer shape, scaled down)
        const Tensor x = input({300, 256}, 61), w = input({256, 520}, 62, 0.0625f),
                     bias = input({520}, 63, 0.1f);
        const Tensor xg = x.to(gpu), wg = w.to(gpu), bg = bias.to(gpu);
        const Tensor mag = gemm_magnitude(x, w, 1.0f, nullptr, 0.0f, false, false, &bias);
        for (auto [act, name] : {std::pair{GemmActivation::Relu, "relu"},
                                 std::pair{GemmActivation::Gelu, "gelu"},
                                 std::pair{GemmActivation::GeluTanh, "gelu tanh"}}) {
            const Tensor got = gemm(xg, wg, 1.0f, nullptr, 0.0f, false, false, &bg, act,
                                    Execution::GPU);
            const Tensor want = gemm(x, w, 1.0f, nullptr, 0.0f, false, false, &bias, act,
                                     Execution::CPU);
            // GELU's slope is below 1.13; the fp32 epilogue activation adds a few ulp
            require_close(got, want, 1.2e-5, 1e-6,
                          std::string("gemm + bias + ") + name + " 300x520x256 (one kernel)",
                          &mag);
        }
    }
    struct Case {
        const char* name;
        Shape a, b;
        bool ta, tb;
        float alpha, beta;
        bool with_c;
    };
    const Case cases[] = {
        {"plain", {37, 53}, {53, 29}, false, false, 1.0f, 0.0f, false},
        {"transpose a", {53, 37}, {53, 29}, true, false, 1.0f, 0.0f, false},
        {"transpose b", {37, 53}, {29, 53}, false, true, 1.0f, 0.0f, false},
        {"transpose both", {53, 37}, {29, 53}, true, true, -2.0f, 0.0f, false},
        {"alpha and beta", {130, 70}, {70, 260}, false, false, 0.5f, -1.5f, true},
        {"c given, beta 0", {40, 30}, {30, 20}, false, false, 1.0f, 0.0f, true},
        {"k = 0", {5, 0}, {0, 7}, false, false, 1.0f, 2.0f, true},
    };
    std::uint64_t seed = 300;
    for (const Case& t : cases) {
        const Tensor a = input(t.a, seed++), b = input(t.b, seed++);
        const std::int64_t m = t.ta ? t.a[1] : t.a[0], n = t.tb ? t.b[0] : t.b[1];
        const Tensor c = t.with_c ? input({m, n}, seed++) : Tensor();
        const Tensor cg = t.with_c ? c.to(gpu) : Tensor();
        const Tensor got = gemm(a.to(gpu), b.to(gpu), t.alpha, t.with_c ? &cg : nullptr, t.beta,
                                t.ta, t.tb, Execution::GPU);
        const Tensor want = gemm(a, b, t.alpha, t.with_c ? &c : nullptr, t.beta, t.ta, t.tb,
                                 Execution::CPU);
        const Tensor mag = gemm_magnitude(a, b, t.alpha, t.with_c ? &c : nullptr, t.beta, t.ta,
                                          t.tb);
        require_close(got, want, 1e-5, 1e-6, std::string("gemm ") + t.name, &mag);
    }
    // argument errors are the composed path's
    const Tensor a = input({4, 5}, 1).to(gpu), b = input({6, 3}, 2).to(gpu);
    bool threw = false;
    try {
        gemm(a, b, 1.0f, nullptr, 0.0f, false, false, Execution::GPU);
    } catch (const std::invalid_argument&) {
        threw = true;
    }
    if (!threw) {
        throw std::runtime_error("gemm with mismatched inner dimensions did not throw");
    }
    ++checks;
    std::cout << "  ok gemm argument errors\n";
}

// The level-1 kernels the CUDA backend registers: dot (double accumulation on both sides: within
// one rounding), scal and the four elementwise ops (bit-exact), with broadcasting done by the op.
void check_level_one(Device gpu) {
    for (std::int64_t n : {1, 17, 1000, 100003, (1 << 20) + 7}) {
        const Tensor x = input({n}, 71), y = input({n}, 72);
        require_close(dot(x.to(gpu), y.to(gpu), Execution::GPU), dot(x, y, Execution::CPU),
                      1.2e-7, 1e-30, "dot n=" + std::to_string(n));
    }
    const Tensor x = input({1000}, 73, 2.0f);
    require_close(scal(-0.75f, x.to(gpu), Execution::GPU), scal(-0.75f, x, Execution::CPU), 0.0,
                  0.0, "scal (bit-exact)");
    const Tensor a = input({33, 70}, 74, 2.0f), b = input({70}, 75, 2.0f);
    const Tensor ag = a.to(gpu), bg = b.to(gpu);
    require_close(add(ag, bg, Execution::GPU), add(a, b, Execution::CPU), 0.0, 0.0,
                  "add, row broadcast (bit-exact)");
    require_close(sub(ag, bg, Execution::GPU), sub(a, b, Execution::CPU), 0.0, 0.0,
                  "sub, row broadcast (bit-exact)");
    require_close(mul(ag, ag, Execution::GPU), mul(a, a, Execution::CPU), 0.0, 0.0,
                  "mul (bit-exact)");
    require_close(div(ag, bg, Execution::GPU), div(a, b, Execution::CPU), 0.0, 0.0,
                  "div, row broadcast (bit-exact)");
}

// Gradients on the device: bias_add's bias gradient (OpId::BiasGrad, the host loop's bits) and
// matmul's (strided transposes read in place), pushed through the recorded closures with a given
// output gradient, against the same on the CPU.
void check_gradients(Device gpu) {
    const Tensor x = input({70, 130}, 81), bias = input({130}, 82), grad = input({70, 130}, 83);
    Tensor bias_cpu = bias;  // leaf copies that record
    bias_cpu.set_requires_grad(true);
    Tensor bias_gpu = bias.to(gpu);
    bias_gpu.set_requires_grad(true);
    detail::autograd::propagate(bias_add(x, bias_cpu, Execution::CPU), grad);
    detail::autograd::propagate(bias_add(x.to(gpu), bias_gpu, Execution::GPU), grad.to(gpu));
    require_close(bias_gpu.grad(), bias_cpu.grad(), 0.0, 0.0,
                  "bias_add bias gradient on the device (bit-exact)");

    Tensor a_cpu = input({40, 90}, 84), b_cpu = input({90, 50}, 85);
    const Tensor g = input({40, 50}, 86);
    Tensor a_gpu = a_cpu.to(gpu), b_gpu = b_cpu.to(gpu);
    for (Tensor* t : {&a_cpu, &b_cpu, &a_gpu, &b_gpu}) {
        t->set_requires_grad(true);
    }
    detail::autograd::propagate(matmul(a_cpu, b_cpu, Execution::CPU), g);
    detail::autograd::propagate(matmul(a_gpu, b_gpu, Execution::GPU), g.to(gpu));
    const Tensor ga = mensurflow::abs(g, Execution::CPU);
    const Tensor mag_a = matmul(ga, mensurflow::abs(b_cpu, Execution::CPU).transpose(0, 1),
                                Execution::CPU);
    const Tensor mag_b = matmul(mensurflow::abs(a_cpu, Execution::CPU).transpose(0, 1), ga,
                                Execution::CPU);
    require_close(a_gpu.grad(), a_cpu.grad(), 1e-5, 1e-6, "matmul dA on the device", &mag_a);
    require_close(b_gpu.grad(), b_cpu.grad(), 1e-5, 1e-6, "matmul dB on the device", &mag_b);
}

void check(int status) {
    if (status != MFK_OK) {
        throw std::runtime_error(std::string("mfk: ") + mfk_status_string(status) + " " +
                                 mfk_last_cuda_error());
    }
}

// The pre-split weight owner a maintainer would put next to the CUDA backend (the class of the
// integration notes, compiled and run as written there), on the backend's own stream.
class CudaPackedB {
  public:
    CudaPackedB(const Tensor& b, detail::Stream& s) { // b: k x n on the CUDA device, any strides
        check(mfk_pack_b_f32(detail::TensorAccess::data<float>(b), b.strides()[0],
                             b.strides()[1], b.shape()[0], b.shape()[1], MFK_PRECISION_DEFAULT,
                             detail::cuda_stream_handle(s), &h_));
    }
    ~CudaPackedB() { mfk_packed_b_free(h_); }
    CudaPackedB(const CudaPackedB&) = delete;
    CudaPackedB& operator=(const CudaPackedB&) = delete;
    const mfk_packed_b* get() const { return h_; }

  private:
    mfk_packed_b* h_ = nullptr;
};

void check_packed_b(Device gpu) {
    const Tensor x = input({200, 96}, 95), w = input({96, 130}, 96);
    const Tensor xg = x.to(gpu), wg = w.to(gpu);
    detail::Stream& s = detail::Registry::instance().get(gpu).stream(gpu.index);
    const CudaPackedB packed(wg.transpose(0, 1).transpose(0, 1), s);
    Tensor out = Tensor::empty({200, 130}, DType::F32, gpu);
    mfk_gemm_desc d{};
    d.a = detail::TensorAccess::data<float>(xg);
    d.a_rs = 96;
    d.a_cs = 1;
    d.c = detail::TensorAccess::data<float>(out);
    d.ldc = 130;
    d.m = 200;
    d.n = 130;
    d.k = 96;
    d.alpha = 1.0f;
    d.precision = MFK_PRECISION_DEFAULT;
    check(mfk_gemm_prepacked_f32(&d, packed.get(), detail::cuda_stream_handle(s)));
    const Tensor mag = gemm_magnitude(x, w, 1.0f, nullptr, 0.0f, false, false);
    require_close(out, matmul(x, w, Execution::CPU), 1e-5, 1e-6,
                  "pre-split weight on the backend's stream (CudaPackedB)", &mag);
}

// Tensor::to() from one GPU to another: one device-to-device copy (exact), when there are two.
void check_transfers(Device gpu) {
    const Device other = parse_device("cuda:1");
    if (!device_available(other)) {
        std::cout << "  (one CUDA device: Tensor::to() between GPUs not checked)\n";
        return;
    }
    const Tensor x = input({300, 257}, 91);
    const Tensor there = x.to(gpu).to(other);
    if (there.device() != other) {
        throw std::runtime_error("Tensor::to(cuda:1) left the tensor elsewhere");
    }
    const Tensor back = there.to(gpu);
    require_close(back, x, 0.0, 0.0, "Tensor::to() cuda:0 -> cuda:1 -> cuda:0 (exact)");
    const Tensor view = x.to(gpu).transpose(0, 1).to(other).to(gpu);
    require_close(view, x.transpose(0, 1).contiguous(), 0.0, 0.0,
                  "Tensor::to() of a transposed view between GPUs (exact)");
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
        check_gemm(gpu);
        check_level_one(gpu);
        check_gradients(gpu);
        check_transfers(gpu);
        check_packed_b(gpu);
        std::cout << "reference_api_check passed (" << checks << " checks on " << to_string(gpu)
                  << ")\n";
        return 0;
    } catch (const std::exception& e) {
        std::cerr << "reference_api_check FAILED: " << e.what() << '\n';
        return 1;
    }
}
