/* TEST INFRASTRUCTURE ONLY — the parity oracle. Nothing in the product path may call this.
 *
 * A plain-C restatement of the reference's CPU algorithms for the dense fp32 contraction path
 * (bakir004/mensurflow). Each function names the reference file:line it restates. It is pinned
 * two ways by tests/test_oracle.py: against golden vectors produced by the unmodified reference
 * (tests/golden/, made by tests/golden/make_golden.py through oracle/_ref), and against the
 * known answers written in the reference's own tests (tests/ops/matmul_test.cpp:102-125).
 *
 * Built by oracle/Makefile into oracle/_build/libmforacle.so (gcc -O2 -fopenmp). OpenMP only
 * splits independent output elements, so results do not depend on the thread count.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

/* ---- Philox4x32-10 ------------------------------------------------------------------------
 * src/backends/cpu/ops/random/philox.hpp:14-36: ten rounds with multipliers 0xD2511F53 and
 * 0xCD9E8D57 and Weyl key increments 0x9E3779B9 / 0xBB67AE85; block b of a stream uses counter
 * {lo32(b), hi32(b), 0, 0} and key {lo32(seed), hi32(seed)}. Published by Salmon et al. (SC11). */
static void philox_block(uint64_t seed, uint64_t block, uint32_t out[4]) {
    uint32_t c0 = (uint32_t)block, c1 = (uint32_t)(block >> 32), c2 = 0, c3 = 0;
    uint32_t k0 = (uint32_t)seed, k1 = (uint32_t)(seed >> 32);
    for (int round = 0; round < 10; ++round) {
        const uint64_t p0 = (uint64_t)0xD2511F53u * c0;
        const uint64_t p1 = (uint64_t)0xCD9E8D57u * c2;
        const uint32_t n0 = (uint32_t)(p1 >> 32) ^ c1 ^ k0;
        const uint32_t n1 = (uint32_t)p1;
        const uint32_t n2 = (uint32_t)(p0 >> 32) ^ c3 ^ k1;
        const uint32_t n3 = (uint32_t)p0;
        c0 = n0; c1 = n1; c2 = n2; c3 = n3;
        k0 += 0x9E3779B9u;
        k1 += 0xBB67AE85u;
    }
    out[0] = c0; out[1] = c1; out[2] = c2; out[3] = c3;
}

uint32_t mfo_philox_word(uint64_t seed, uint64_t block, int lane) {
    uint32_t w[4];
    philox_block(seed, block, w);
    return w[lane & 3];
}

/* uniform_f32, src/backends/cpu/ops/random/random.cpp:47-63 (stream walk :16-33): element i of
 * a call with `offset` is word (offset+i)%4 of block (offset+i)/4; value = low + (high-low)*u
 * with u = (word>>8)*2^-24 in double, rounded to float and clamped to [low, nextafter(high,low)]. */
void mfo_uniform(float* out, int64_t n, float low, float high, uint64_t seed, uint64_t offset) {
    if (low == high) {
        for (int64_t i = 0; i < n; ++i) out[i] = low;
        return;
    }
    const double width = (double)high - low;
    const float last = nextafterf(high, low);
#pragma omp parallel for schedule(static) if (n > (1 << 16))
    for (int64_t i = 0; i < n; ++i) {
        const uint64_t pos = offset + (uint64_t)i;
        uint32_t w[4];
        philox_block(seed, pos / 4, w);
        const double u = (double)(w[pos % 4] >> 8) * 0x1p-24;
        float v = (float)((double)low + width * u);
        if (v < low) v = low;
        if (v > last) v = last;
        out[i] = v;
    }
}

/* normal_f32, random.cpp:65-96: block words (2q, 2q+1) give one Box-Muller pair in double,
 * u = (word + 0.5)*2^-32, r = sqrt(-2 ln u1), a = 2*pi*u2; lane 2q+0 is r*cos(a), 2q+1 r*sin(a). */
void mfo_normal(float* out, int64_t n, float mean, float stddev, uint64_t seed, uint64_t offset) {
    if (stddev == 0.0f) {
        for (int64_t i = 0; i < n; ++i) out[i] = mean;
        return;
    }
#pragma omp parallel for schedule(static) if (n > (1 << 16))
    for (int64_t i = 0; i < n; ++i) {
        const uint64_t pos = offset + (uint64_t)i;
        uint32_t w[4];
        philox_block(seed, pos / 4, w);
        const int lane = (int)(pos % 4);
        const int pair = lane / 2;
        const double u1 = ((double)w[2 * pair] + 0.5) * 0x1p-32;
        const double u2 = ((double)w[2 * pair + 1] + 0.5) * 0x1p-32;
        const double radius = sqrt(-2.0 * log(u1));
        const double angle = 6.283185307179586476925286766559 * u2;
        const double z = (lane % 2 == 0) ? radius * cos(angle) : radius * sin(angle);
        out[i] = (float)((double)mean + stddev * z);
    }
}

/* ---- The contraction -----------------------------------------------------------------------
 * The reference's CPU GEMM (src/backends/cpu/ops/gemm/gemm_packed.cpp) computes each C entry as
 * fp32 FMA chains in increasing depth p, restarted from zero for every depth block of KC terms
 * (kernel_6x16, :313-378) and added into C block by block (store_row, :362-370). `kc` restates
 * that blocking (the reference derives KC from the CPU's cache sizes, initial_blocking :227).
 *
 * Batched form as in cpu::BatchedGemm (gemm_batched.hpp:21-37): matrix i of op(A) starts at
 * a + a_off[i] with element (r,p) at r*rsa + p*csa; op(B) likewise (p,j) at p*rsb + j*csb;
 * C is row-major with row stride ldc and matrix stride c_stride. The alpha/beta post-pass is
 * finish_matrix (gemm_batched.cpp:12-28): c = alpha*c + beta*c0 (alpha 1, beta 0 skip it);
 * c0 (optional) has its own row/col/matrix strides so a broadcast c needs no copy. */
void mfo_gemm_batched(const float* a, const int64_t* a_off, int64_t rsa, int64_t csa,
                      const float* b, const int64_t* b_off, int64_t rsb, int64_t csb,
                      float* c, int64_t ldc, int64_t c_stride,
                      const float* c0, int64_t rsc0, int64_t csc0, int64_t c0_stride,
                      int64_t batch, int64_t m, int64_t n, int64_t k,
                      float alpha, float beta, int64_t kc) {
    if (kc <= 0) kc = 256;
#pragma omp parallel for collapse(2) schedule(static)
    for (int64_t bi = 0; bi < batch; ++bi) {
        for (int64_t i = 0; i < m; ++i) {
            const float* ab = a + (a_off ? a_off[bi] : 0);
            const float* bb = b + (b_off ? b_off[bi] : 0);
            float* crow = c + bi * c_stride + i * ldc;
            for (int64_t j = 0; j < n; ++j) {
                float acc = 0.0f;
                for (int64_t p0 = 0; p0 < k; p0 += kc) {
                    const int64_t p1 = p0 + kc < k ? p0 + kc : k;
                    float part = 0.0f;
                    for (int64_t p = p0; p < p1; ++p) {
                        part = fmaf(ab[i * rsa + p * csa], bb[p * rsb + j * csb], part);
                    }
                    acc = p0 == 0 ? part : acc + part;
                }
                if (!(alpha == 1.0f && beta == 0.0f)) {
                    if (beta == 0.0f) {
                        acc = alpha * acc;
                    } else {
                        const float init = c0[bi * c0_stride + i * rsc0 + j * csc0];
                        acc = alpha * acc + beta * init;
                    }
                }
                crow[j] = acc;
            }
        }
    }
}

/* (|op(A)|·|op(B)|)_ij in double — the scale that rounding error is measured against, as in the
 * reference's tests (tests/reference/blas.hpp:38-59, `magnitude`). Same layout as above. */
void mfo_abs_product(const float* a, const int64_t* a_off, int64_t rsa, int64_t csa,
                     const float* b, const int64_t* b_off, int64_t rsb, int64_t csb,
                     double* out, int64_t batch, int64_t m, int64_t n, int64_t k) {
#pragma omp parallel for collapse(2) schedule(static)
    for (int64_t bi = 0; bi < batch; ++bi) {
        for (int64_t i = 0; i < m; ++i) {
            const float* ab = a + (a_off ? a_off[bi] : 0);
            const float* bb = b + (b_off ? b_off[bi] : 0);
            for (int64_t j = 0; j < n; ++j) {
                double s = 0.0;
                for (int64_t p = 0; p < k; ++p) {
                    s += fabs((double)ab[i * rsa + p * csa] * (double)bb[p * rsb + j * csb]);
                }
                out[(bi * m + i) * n + j] = s;
            }
        }
    }
}

/* bias_add_f32, src/backends/cpu/ops/elementwise/elementwise.cpp:128-137: out[r,j] = x[r,j] +
 * bias[j], one fp32 add. */
void mfo_bias_add(const float* x, const float* bias, float* out, int64_t rows, int64_t cols) {
    for (int64_t r = 0; r < rows; ++r)
        for (int64_t j = 0; j < cols; ++j) out[r * cols + j] = x[r * cols + j] + bias[j];
}

/* bias_add's backward for the bias (src/ops/elementwise.cpp:263-283): reduced[j] is the sum
 * of the upstream gradient's column j over the rows, accumulated in float in row order from 0.
 * g is rows x cols with row stride ld. */
void mfo_bias_grad(const float* g, int64_t rows, int64_t cols, int64_t ld, float* out) {
    for (int64_t j = 0; j < cols; ++j) out[j] = 0.0f;
    for (int64_t r = 0; r < rows; ++r)
        for (int64_t j = 0; j < cols; ++j) out[j] += g[r * ld + j];
}

/* relu_f32, elementwise.cpp relu: x < 0 ? 0 : x (NaN passes through). */
void mfo_relu(const float* x, float* out, int64_t n) {
    for (int64_t i = 0; i < n; ++i) out[i] = x[i] < 0.0f ? 0.0f : x[i];
}

/* gelu_f32, elementwise.cpp:173-192. Exact: 0.5*v*erfc(-v/sqrt(2)) in double; tanh form:
 * v*sigmoid(2u), u = sqrt(2/pi)*v*(1+0.044715 v^2), sigmoid evaluated without cancellation.
 * Infinities map to -0 / +inf. */
static double stable_sigmoid(double z) {
    if (z >= 0.0) return 1.0 / (1.0 + exp(-z));
    const double e = exp(z);
    return e / (1.0 + e);
}

void mfo_gelu(const float* x, float* out, int64_t n, int approximate) {
    for (int64_t i = 0; i < n; ++i) {
        const float value = x[i];
        if (isinf(value)) {
            out[i] = value < 0.0f ? -0.0f : value;
            continue;
        }
        const double v = value;
        if (approximate) {
            const double u = 0.79788456080286535588 * v * (1.0 + 0.044715 * v * v);
            out[i] = (float)(v * stable_sigmoid(2.0 * u));
        } else {
            out[i] = (float)(0.5 * v * erfc(-v * 0.70710678118654752440));
        }
    }
}

/* gemv_f32, src/backends/cpu/ops/blas/blas.cpp:66-80: y[i] = float(alpha*sum + beta*y0[i]) with
 * the sum over products accumulated in double; a is row-major [rows, cols] with row stride lda
 * (the reference passes contiguous a, lda = cols); transpose reads a[j,i]. beta == 0 ignores y0.
 * matvec_f32 (:55-64) is the alpha 1, beta 0, no-transpose case. */
void mfo_gemv(const float* a, int64_t rows, int64_t cols, int64_t lda, const float* x,
              float alpha, float beta, const float* y0, float* y, int transpose) {
    const int64_t outputs = transpose ? cols : rows;
    const int64_t inputs = transpose ? rows : cols;
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < outputs; ++i) {
        double sum = 0.0;
        for (int64_t j = 0; j < inputs; ++j) {
            const float v = transpose ? a[j * lda + i] : a[i * lda + j];
            sum += (double)v * (double)x[j];
        }
        y[i] = (float)(alpha * sum + (beta == 0.0f ? 0.0 : beta * y0[i]));
    }
}

/* softmax_f32 / log_softmax_f32, src/backends/cpu/ops/softmax/softmax.cpp:11-80: along the middle
 * axis of a contiguous [outer, length, inner] tensor. max with NaN poisoning; an all -inf line ->
 * zeros (log: -inf); e = expf(x - max) in float, sum in double, out = e * float(1/sum); log:
 * (x - max) - float(log(sum)). */
void mfo_softmax(const float* x, float* out, int64_t outer, int64_t length, int64_t inner,
                 int log_softmax) {
#pragma omp parallel for schedule(static)
    for (int64_t line = 0; line < outer * inner; ++line) {
        const int64_t base = (line / inner) * length * inner + line % inner;
        const float* in = x + base;
        float* dst = out + base;
        float maximum = -INFINITY;
        for (int64_t j = 0; j < length; ++j) {
            const float value = in[j * inner];
            if (isnan(value) || value > maximum) {
                maximum = value;
                if (isnan(value)) break;
            }
        }
        if (maximum == -INFINITY) {
            for (int64_t j = 0; j < length; ++j) dst[j * inner] = log_softmax ? -INFINITY : 0.0f;
            continue;
        }
        double sum = 0.0;
        for (int64_t j = 0; j < length; ++j) {
            const float e = expf(in[j * inner] - maximum);
            if (!log_softmax) dst[j * inner] = e;
            sum += (double)e;
        }
        if (log_softmax) {
            const float log_sum = (float)log(sum);
            for (int64_t j = 0; j < length; ++j) dst[j * inner] = (in[j * inner] - maximum) - log_sum;
        } else {
            const float scale = (float)(1.0 / sum);
            for (int64_t j = 0; j < length; ++j) dst[j * inner] *= scale;
        }
    }
}

/* where_f32 (src/backends/cpu/backend.cpp:625-630): out = cond ? x : y over broadcast, packed
 * inputs. */
void mfo_where(const uint8_t* cond, const float* x, const float* y, float* out, int64_t n) {
    for (int64_t i = 0; i < n; ++i) out[i] = cond[i] ? x[i] : y[i];
}
