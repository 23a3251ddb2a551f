// TEST INFRASTRUCTURE ONLY — never part of the product path.
//
// A C-ABI over the unmodified reference library (bakir004/mensurflow, built from its own
// sources by oracle/Makefile into oracle/_ref/). Everything here calls the reference's PUBLIC
// API with Execution::CPU, so the numbers it returns are the reference's own CPU results:
//   gemm                  include/mensurflow/ops/blas.hpp:59   (src/ops/blas.cpp:234-262)
//   matmul                include/mensurflow/ops/blas.hpp:55   (src/ops/blas.cpp:186-232)
//   gemm_strided_batched  include/mensurflow/ops/blas.hpp:75   (src/ops/blas.cpp:297-394)
//   gemv / matvec         include/mensurflow/ops/blas.hpp:35,40 (src/ops/blas.cpp:119-183)
//   bias_add / relu/gelu  include/mensurflow/ops/elementwise.hpp:43,56,62
//   backward of bias_add and matmul, through the reference's autograd (Tensor::backward)
//   uniform / normal      include/mensurflow/ops/random.hpp:20,25
//   Tensor::contiguous of views (permute / slice / expand), include/mensurflow/tensor.hpp
// Used by tests/golden/make_golden.py (fixtures), by tests that pin the C restatement in
// oracle/mf_oracle.c against the reference, and by bench.py's CPU-baseline and reference arms.
// Every entry returns 0 on success and -1 on a C++ exception (text in mfref_last_error()).
#include "backends/cpu/threads.hpp"
#include "mensurflow/mensurflow.hpp"

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <exception>
#include <string>
#include <vector>

using namespace mensurflow;

namespace {

thread_local std::string g_error;

template <typename F> int guarded(F&& f) {
    try {
        f();
        return 0;
    } catch (const std::exception& e) {
        g_error = e.what();
        return -1;
    }
}

Shape make_shape(const std::int64_t* dims, int nd) { return Shape(dims, dims + nd); }

Tensor host_tensor(const float* data, const Shape& shape) {
    return Tensor::from_host(data, shape, DType::F32, Device{});
}

void copy_out(const Tensor& t, float* out) {
    if (t.numel() > 0) {
        t.copy_to_host(out);
    }
}

double now() {
    return std::chrono::duration<double>(std::chrono::steady_clock::now().time_since_epoch())
        .count();
}

} // namespace

extern "C" {

const char* mfref_last_error() { return g_error.c_str(); }

int mfref_openmp() { return cpu::has_openmp() ? 1 : 0; }

int mfref_max_threads() { return cpu::max_threads(); }

void mfref_set_threads(int threads) { cpu::set_max_threads(threads); }

int mfref_uniform(float* out, std::int64_t n, float low, float high, std::uint64_t seed,
                  std::uint64_t offset) {
    return guarded([&] { copy_out(uniform({n}, low, high, seed, offset, Execution::CPU), out); });
}

int mfref_normal(float* out, std::int64_t n, float mean, float stddev, std::uint64_t seed,
                 std::uint64_t offset) {
    return guarded(
        [&] { copy_out(normal({n}, mean, stddev, seed, offset, Execution::CPU), out); });
}

// a is stored [ar, ac], b is stored [br, bc], c (optional) is the [m, n] result shape.
int mfref_gemm(const float* a, std::int64_t ar, std::int64_t ac, const float* b, std::int64_t br,
               std::int64_t bc, const float* c, float alpha, float beta, int transpose_a,
               int transpose_b, float* out) {
    return guarded([&] {
        const Tensor ta = host_tensor(a, {ar, ac});
        const Tensor tb = host_tensor(b, {br, bc});
        const std::int64_t m = transpose_a ? ac : ar;
        const std::int64_t n = transpose_b ? br : bc;
        Tensor tc;
        if (c != nullptr) {
            tc = host_tensor(c, {m, n});
        }
        copy_out(gemm(ta, tb, alpha, c ? &tc : nullptr, beta, transpose_a != 0, transpose_b != 0,
                      Execution::CPU),
                 out);
    });
}

int mfref_matmul(const float* a, std::int64_t m, std::int64_t k, const float* b, std::int64_t n,
                 float* out) {
    return guarded([&] {
        copy_out(matmul(host_tensor(a, {m, k}), host_tensor(b, {k, n}), Execution::CPU), out);
    });
}

// Shapes as stored (before the transpose flags). out_shape receives the result's shape
// (up to 8 dims) and out_nd its rank; out must hold numel(result) floats.
int mfref_gemm_strided_batched(const float* a, const std::int64_t* a_shape, int a_nd,
                               const float* b, const std::int64_t* b_shape, int b_nd,
                               const float* c, const std::int64_t* c_shape, int c_nd, float alpha,
                               float beta, int transpose_a, int transpose_b, float* out,
                               std::int64_t* out_shape, int* out_nd) {
    return guarded([&] {
        const Tensor ta = host_tensor(a, make_shape(a_shape, a_nd));
        const Tensor tb = host_tensor(b, make_shape(b_shape, b_nd));
        Tensor tc;
        if (c != nullptr) {
            tc = host_tensor(c, make_shape(c_shape, c_nd));
        }
        const Tensor r = gemm_strided_batched(ta, tb, alpha, c ? &tc : nullptr, beta,
                                              transpose_a != 0, transpose_b != 0, Execution::CPU);
        *out_nd = r.dim();
        for (int d = 0; d < r.dim(); ++d) {
            out_shape[d] = r.size(d);
        }
        if (out != nullptr) {
            copy_out(r, out);
        }
    });
}

int mfref_bias_add(const float* x, std::int64_t rows, std::int64_t cols, const float* bias,
                   float* out) {
    return guarded([&] {
        copy_out(bias_add(host_tensor(x, {rows, cols}), host_tensor(bias, {cols}), Execution::CPU),
                 out);
    });
}

// The reference's own backward passes, driven through its autograd: loss = sum(out * g) has
// d loss / d out = g exactly (mul's backward multiplies the ones from sum by g), so the leaves'
// gradients are what bias_add's and matmul's recorded backward closures compute from g
// (src/ops/elementwise.cpp:263-283; src/ops/blas.cpp:220-230).
int mfref_bias_add_backward(const float* g, std::int64_t rows, std::int64_t cols, float* dbias) {
    return guarded([&] {
        Tensor x = Tensor::zeros({rows, cols}, DType::F32, Device{});
        Tensor bias = Tensor::zeros({cols}, DType::F32, Device{});
        bias.set_requires_grad(true);
        Tensor loss = sum(mul(bias_add(x, bias, Execution::CPU), host_tensor(g, {rows, cols}),
                              Execution::CPU),
                          Execution::CPU);
        loss.backward();
        copy_out(bias.grad(), dbias);
    });
}

int mfref_matmul_backward(const float* a, const float* b, const float* g, std::int64_t m,
                          std::int64_t k, std::int64_t n, float* da, float* db) {
    return guarded([&] {
        Tensor ta = host_tensor(a, {m, k});
        Tensor tb = host_tensor(b, {k, n});
        ta.set_requires_grad(true);
        tb.set_requires_grad(true);
        Tensor loss = sum(mul(matmul(ta, tb, Execution::CPU), host_tensor(g, {m, n}),
                              Execution::CPU),
                          Execution::CPU);
        loss.backward();
        copy_out(ta.grad(), da);
        copy_out(tb.grad(), db);
    });
}

int mfref_gelu(const float* x, std::int64_t n, int approximate, float* out) {
    return guarded(
        [&] { copy_out(gelu(host_tensor(x, {n}), approximate != 0, Execution::CPU), out); });
}

int mfref_relu(const float* x, std::int64_t n, float* out) {
    return guarded([&] { copy_out(relu(host_tensor(x, {n}), Execution::CPU), out); });
}

// a stored [rows, cols]; y (optional) has op(a)'s row count.
int mfref_gemv(const float* a, std::int64_t rows, std::int64_t cols, const float* x, float alpha,
               const float* y, float beta, int transpose_a, float* out) {
    return guarded([&] {
        const Tensor ta = host_tensor(a, {rows, cols});
        const std::int64_t in = transpose_a ? rows : cols;
        const std::int64_t outn = transpose_a ? cols : rows;
        Tensor ty;
        if (y != nullptr) {
            ty = host_tensor(y, {outn});
        }
        copy_out(gemv(ta, host_tensor(x, {in}), alpha, y ? &ty : nullptr, beta, transpose_a != 0,
                      Execution::CPU),
                 out);
    });
}

int mfref_matvec(const float* a, std::int64_t m, std::int64_t k, const float* x, float* out) {
    return guarded(
        [&] { copy_out(matvec(host_tensor(a, {m, k}), host_tensor(x, {k}), Execution::CPU), out); });
}

// softmax / log_softmax along `axis` of a host tensor of the given shape.
int mfref_softmax(const float* x, const std::int64_t* shape, int nd, int axis, int log_softmax_,
                  float* out) {
    return guarded([&] {
        const Tensor t = host_tensor(x, make_shape(shape, nd));
        copy_out(log_softmax_ ? log_softmax(t, axis, Execution::CPU) : softmax(t, axis, Execution::CPU),
                 out);
    });
}

// The reference's attention (src/ops/attention.cpp:48-98) on host tensors; mask (optional) is a
// Bool tensor given as bytes. out_shape/out_nd receive the result's shape.
int mfref_attention(const float* q, const std::int64_t* qs, int qnd, const float* k,
                    const std::int64_t* ks, int knd, const float* v, const std::int64_t* vs,
                    int vnd, const std::uint8_t* mask, const std::int64_t* ms, int mnd, int causal,
                    float scale, float* out, std::int64_t* out_shape, int* out_nd) {
    return guarded([&] {
        const Tensor tq = host_tensor(q, make_shape(qs, qnd));
        const Tensor tk = host_tensor(k, make_shape(ks, knd));
        const Tensor tv = host_tensor(v, make_shape(vs, vnd));
        Tensor tm;
        if (mask != nullptr) {
            tm = Tensor::from_host(mask, make_shape(ms, mnd), DType::Bool, Device{});
        }
        const Tensor r = attention(tq, tk, tv, mask ? &tm : nullptr, causal != 0, scale,
                                   Execution::CPU);
        *out_nd = r.dim();
        for (int d = 0; d < r.dim(); ++d) {
            out_shape[d] = r.size(d);
        }
        if (out != nullptr) {
            copy_out(r, out);
        }
    });
}

// Timing harness for the CPU baselines: inputs are made once by the reference's own normal() /
// uniform() factories (outside any timed region), then each run times `reps` calls of the
// reference's public gemm (+ bias_add) exactly as a user would make them.
struct GemmBench {
    Tensor a, b, c, bias;
    bool transpose_b = false;
};

void* mfref_gemm_bench_new(std::int64_t m, std::int64_t n, std::int64_t k, int transpose_b,
                           std::uint64_t seed) {
    GemmBench* h = nullptr;
    const int rc = guarded([&] {
        auto* g = new GemmBench;
        g->transpose_b = transpose_b != 0;
        g->a = normal({m, k}, 0.0f, 1.0f, seed, 0, Execution::CPU);
        g->b = g->transpose_b
                   ? normal({n, k}, 0.0f, 1.0f, seed, std::uint64_t(m * k), Execution::CPU)
                   : normal({k, n}, 0.0f, 1.0f, seed, std::uint64_t(m * k), Execution::CPU);
        g->c = normal({m, n}, 0.0f, 1.0f, seed, std::uint64_t(m * k + n * k), Execution::CPU);
        g->bias = uniform({n}, -0.1f, 0.1f, seed, std::uint64_t(m * k + n * k + m * n),
                          Execution::CPU);
        h = g;
    });
    return rc == 0 ? h : nullptr;
}

int mfref_gemm_bench_run(void* handle, float alpha, float beta, int with_bias, int reps,
                         double* seconds) {
    return guarded([&] {
        auto* g = static_cast<GemmBench*>(handle);
        for (int i = 0; i < reps; ++i) {
            const double t0 = now();
            Tensor r = gemm(g->a, g->b, alpha, beta != 0.0f ? &g->c : nullptr, beta, false,
                            g->transpose_b, Execution::CPU);
            if (with_bias) {
                r = bias_add(r, g->bias, Execution::CPU);
            }
            seconds[i] = now() - t0;
        }
    });
}

void mfref_gemm_bench_free(void* handle) { delete static_cast<GemmBench*>(handle); }

// Times the reference's public gemv on A [rows, cols] and x [cols] from uniform(-1, 1).
int mfref_time_gemv(std::int64_t rows, std::int64_t cols, std::uint64_t seed, int warmup, int reps,
                    double* seconds) {
    return guarded([&] {
        const Tensor a = uniform({rows, cols}, -1.0f, 1.0f, seed, 0, Execution::CPU);
        const Tensor x = uniform({cols}, -1.0f, 1.0f, seed, std::uint64_t(rows * cols),
                                 Execution::CPU);
        for (int i = 0; i < warmup; ++i) {
            gemv(a, x, 1.0f, nullptr, 0.0f, false, Execution::CPU);
        }
        for (int i = 0; i < reps; ++i) {
            const double t0 = now();
            const Tensor r = gemv(a, x, 1.0f, nullptr, 0.0f, false, Execution::CPU);
            seconds[i] = now() - t0;
            (void)r;
        }
    });
}

// Times the reference's two-layer MLP forward on CPU inputs made once:
// y = bias_add(matmul(gelu(bias_add(matmul(x, w1), b1)), w2), b2), x ~ N(0, 1), w1 / w2
// Xavier-uniform, zero biases, with the public ops a user would call.
int mfref_time_mlp(std::int64_t rows, std::int64_t d_in, std::int64_t d_hid, std::uint64_t seed,
                   int warmup, int reps, double* seconds) {
    return guarded([&] {
        const float lim = std::sqrt(6.0f / static_cast<float>(d_in + d_hid));
        const Tensor x = normal({rows, d_in}, 0.0f, 1.0f, seed, 0, Execution::CPU);
        const Tensor w1 = uniform({d_in, d_hid}, -lim, lim, seed, std::uint64_t(rows * d_in),
                                  Execution::CPU);
        const Tensor w2 = uniform({d_hid, d_in}, -lim, lim, seed,
                                  std::uint64_t(rows * d_in + d_in * d_hid), Execution::CPU);
        const Tensor b1 = Tensor::zeros({d_hid});
        const Tensor b2 = Tensor::zeros({d_in});
        auto step = [&] {
            const Tensor h = gelu(bias_add(matmul(x, w1, Execution::CPU), b1, Execution::CPU),
                                  false, Execution::CPU);
            return bias_add(matmul(h, w2, Execution::CPU), b2, Execution::CPU);
        };
        for (int i = 0; i < warmup; ++i) {
            step();
        }
        for (int i = 0; i < reps; ++i) {
            const double t0 = now();
            const Tensor y = step();
            seconds[i] = now() - t0;
            (void)y;
        }
    });
}

// Times the reference's two batched GEMMs of attention on `heads` matrices:
// S = gemm_strided_batched(q, k, 1/sqrt(dh), transpose_b) and O = gemm_strided_batched(S, v),
// q, k, v ~ N(0, 1/sqrt(dh)) (S stands in for the softmax weights: same shape, same work).
int mfref_time_attention_gemms(std::int64_t heads, std::int64_t seq, std::int64_t dh,
                               std::uint64_t seed, int warmup, int reps, double* seconds) {
    return guarded([&] {
        const float sd = 1.0f / std::sqrt(static_cast<float>(dh));
        const std::uint64_t n = std::uint64_t(heads * seq * dh);
        const Tensor q = normal({heads, seq, dh}, 0.0f, sd, seed, 0, Execution::CPU);
        const Tensor k = normal({heads, seq, dh}, 0.0f, sd, seed, n, Execution::CPU);
        const Tensor v = normal({heads, seq, dh}, 0.0f, sd, seed, 2 * n, Execution::CPU);
        auto step = [&] {
            const Tensor sc = gemm_strided_batched(q, k, sd, nullptr, 0.0f, false, true,
                                                   Execution::CPU);
            return gemm_strided_batched(sc, v, 1.0f, nullptr, 0.0f, false, false,
                                        Execution::CPU);
        };
        for (int i = 0; i < warmup; ++i) {
            step();
        }
        for (int i = 0; i < reps; ++i) {
            const double t0 = now();
            const Tensor o = step();
            seconds[i] = now() - t0;
            (void)o;
        }
    });
}

// A strided view built with the reference's public view ops, then made contiguous by
// Tensor::contiguous() (src/core/tensor.cpp:208-230 -> cpu::transpose_f32 for a transposed
// matrix, cpu::strided_copy_f32 otherwise): x is a contiguous host tensor of base_shape (nd
// dims); the view is x.permute(order), then slice(d, start[d], end[d], step[d]) for every d,
// then expand(expand_shape) when expand_shape is non-null (out_nd dims). `out` receives the
// contiguous result, `out_shape` its shape (nd, or out_nd after expand).
int mfref_contiguous_view(const float* x, const std::int64_t* base_shape, int nd,
                          const int* order, const std::int64_t* start, const std::int64_t* end,
                          const std::int64_t* step, const std::int64_t* expand_shape, int out_nd,
                          float* out, std::int64_t* out_shape) {
    return guarded([&] {
        Tensor t = host_tensor(x, make_shape(base_shape, nd));
        t = t.permute(std::vector<int>(order, order + nd));
        for (int d = 0; d < nd; ++d) {
            t = t.slice(d, start[d], end[d], step[d]);
        }
        if (expand_shape != nullptr) {
            t = t.expand(make_shape(expand_shape, out_nd));
        }
        const Tensor c = t.contiguous();
        for (int d = 0; d < c.dim(); ++d) {
            out_shape[d] = c.shape()[d];
        }
        copy_out(c, out);
    });
}

// Times the reference's Tensor::contiguous() of a transposed [rows, cols] matrix (the view of a
// contiguous [cols, rows] tensor), the CPU path cpu::transpose_f32.
int mfref_time_transpose_contiguous(std::int64_t rows, std::int64_t cols, int warmup, int reps,
                                    double* seconds) {
    return guarded([&] {
        const Tensor base = uniform({cols, rows}, -1.0f, 1.0f, 5, 0, Execution::CPU);
        const Tensor view = base.transpose(0, 1);
        for (int i = 0; i < warmup; ++i) {
            view.contiguous();
        }
        for (int i = 0; i < reps; ++i) {
            const double t0 = now();
            const Tensor r = view.contiguous();
            seconds[i] = now() - t0;
            (void)r;
        }
    });
}

} // extern "C"
