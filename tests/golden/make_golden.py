"""Generates tests/golden/*.npz from the unmodified reference library (oracle/_ref/libmfref.so,
built by `make -C oracle ref` from the reference's own sources). Run in the build container:

    python tests/golden/make_golden.py

Every case calls the reference's PUBLIC API with Execution::CPU (see oracle/ref_shim.cpp).
Inputs follow the reference's tests: `make_input` is the LCG of tests/ops/matmul_test.cpp:25-35
and tests/ops/gemm_batched_test.cpp:24-33 (multiples of 0.25 in [-4, 4]); the batched case table
is the 19 cases of gemm_batched_test.cpp:202-220; the seeded configs use the reference's own
Philox uniform/normal factories (include/mensurflow/ops/random.hpp:20-26).
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle import oracle as O  # noqa: E402


def make_input(n, seed):
    """Multiples of 0.25 in [-4, 4]: state = state*1664525 + 1013904223 (mod 2^32),
    value = ((state >> 12) % 33 - 16) / 4 (tests/ops/matmul_test.cpp:25-35)."""
    out = np.empty(n, np.float32)
    state = np.uint32(seed)
    with np.errstate(over="ignore"):
        for i in range(n):
            state = np.uint32(state * np.uint32(1664525) + np.uint32(1013904223))
            out[i] = np.float32(int(int(state >> np.uint32(12)) % 33 - 16) / 4)
    return out


# name, a_shape, b_shape, transpose_a, transpose_b, alpha, c_shape, beta, out_shape
BATCHED_CASES = [
    ("plain batch", (3, 4, 5), (3, 5, 2), False, False, 1.0, (), 0.0, (3, 4, 2)),
    ("shared right-hand side", (4, 3, 5), (5, 2), False, False, 1.0, (), 0.0, (4, 3, 2)),
    ("shared left-hand side", (3, 5), (4, 5, 2), False, False, 1.0, (), 0.0, (4, 3, 2)),
    ("broadcast batch dims", (2, 1, 3, 4), (5, 4, 6), False, False, 1.0, (), 0.0, (2, 5, 3, 6)),
    ("plain matrices", (7, 9), (9, 4), False, False, 1.0, (), 0.0, (7, 4)),
    ("transpose a", (2, 5, 3), (2, 5, 4), True, False, 1.0, (), 0.0, (2, 3, 4)),
    ("transpose b", (2, 3, 5), (2, 4, 5), False, True, 1.0, (), 0.0, (2, 3, 4)),
    ("transpose both", (2, 5, 3), (1, 4, 5), True, True, 1.0, (), 0.0, (2, 3, 4)),
    ("alpha only", (2, 3, 4), (2, 4, 5), False, False, -1.5, (), 0.0, (2, 3, 5)),
    ("alpha and full c", (2, 3, 4), (2, 4, 5), False, False, 2.0, (2, 3, 5), 0.5, (2, 3, 5)),
    ("c broadcast over batch", (4, 3, 4), (4, 5), False, False, 1.0, (3, 5), -1.0, (4, 3, 5)),
    ("c as a row", (2, 3, 4), (2, 4, 5), False, False, 1.0, (5,), 1.0, (2, 3, 5)),
    ("c given, beta 0", (2, 3, 4), (2, 4, 5), False, False, 1.0, (2, 3, 5), 0.0, (2, 3, 5)),
    ("empty batch", (0, 3, 4), (0, 4, 5), False, False, 1.0, (), 0.0, (0, 3, 5)),
    ("empty rows", (2, 0, 4), (2, 4, 5), False, False, 1.0, (), 0.0, (2, 0, 5)),
    ("k is 0", (2, 3, 0), (2, 0, 5), False, False, 1.0, (), 0.0, (2, 3, 5)),
    ("k is 0 with c", (2, 3, 0), (2, 0, 5), False, False, 1.0, (2, 3, 5), 3.0, (2, 3, 5)),
    ("many small", (100, 2, 3), (100, 3, 2), False, False, 1.0, (), 0.0, (100, 2, 2)),
    ("larger", (3, 70, 90), (3, 90, 60), False, False, 1.0, (), 0.0, (3, 70, 60)),
]

# Sizes of tests/ops/matmul_test.cpp:55-58.
MATMUL_SHAPES = [(1, 1, 1), (1, 5, 1), (5, 1, 3), (3, 5, 7), (16, 16, 16), (17, 31, 13),
                 (64, 64, 64), (65, 129, 130), (100, 300, 50), (200, 100, 300), (2, 1000, 3),
                 (1000, 2, 3), (257, 129, 257)]


# (rows, features) of the bias gradients and (m, k, n) of the matmul backward cases
BIAS_GRAD_SHAPES = [(333, 77), (1, 7), (1000, 1), (4096, 1024), (2, 3000)]
MATMUL_BWD_SHAPES = [(50, 40, 30), (129, 257, 65)]


def prod(shape):
    return int(np.prod(shape)) if len(shape) else 1


def main():
    if O.reference() is None:
        sys.exit("oracle/_ref/libmfref.so is missing: run `make -C oracle ref` first")
    out = {}

    # Known answers (tests/ops/matmul_test.cpp:102-125).
    a = np.array([[1, 2, 3], [4, 5, 6]], np.float32)
    b = np.array([[7, 8], [9, 10], [11, 12]], np.float32)
    out["known_a"], out["known_b"] = a, b
    out["known_c"] = O.ref_gemm(a, b)

    # matmul sizes with make_input seeds 4 and 5 (matmul_test.cpp:127-136).
    for (m, n, k) in MATMUL_SHAPES:
        am = make_input(m * k, 4).reshape(m, k)
        bm = make_input(k * n, 5).reshape(k, n)
        out[f"mm_{m}x{n}x{k}"] = O.ref_gemm(am, bm)
    np.savez_compressed(os.path.join(HERE, "matmul_cases.npz"), **out)

    # The 19 batched API cases (make_input seeds 4, 5, 6 as in gemm_batched_test.cpp:222-229).
    bat = {}
    for i, (name, ash, bsh, ta, tb, alpha, csh, beta, osh) in enumerate(BATCHED_CASES):
        av = make_input(prod(ash), 4).reshape(ash)
        bv = make_input(prod(bsh), 5).reshape(bsh)
        cv = make_input(prod(csh), 6).reshape(csh) if csh else None
        r = O.ref_gemm_strided_batched(av, bv, alpha, cv, beta, ta, tb)
        assert r.shape == osh, (name, r.shape, osh)
        bat[f"case{i}_out"] = r
    np.savez_compressed(os.path.join(HERE, "batched_cases.npz"), **bat)

    # Seeded configs at reduced size, with the reference's Philox inputs: a C2-shaped gemm
    # (alpha 0.5, beta 1, transB, bias), a C3-shaped MLP layer, a C4-shaped attention pair and
    # the gemv, plus the raw generator streams that pin the oracle's Philox restatement. Only
    # outputs are stored: the tests regenerate the inputs with the same calls (seeded_inputs in
    # tests/helpers.py), through the oracle's Philox, which the philox_* streams pin bit for bit.
    cfg = {}
    m = n = k = 192
    A = O.ref_normal(m * k, 0, 1, 1, 0).reshape(m, k)
    B = O.ref_normal(n * k, 0, 1, 1, m * k).reshape(n, k)
    C = O.ref_normal(m * n, 0, 1, 1, m * k + n * k).reshape(m, n)
    bias = O.ref_uniform(n, -0.1, 0.1, 1, m * k + n * k + m * n)
    cfg.update(c2_out=O.ref_bias_add(O.ref_gemm(A, B, 0.5, C, 1.0, False, True), bias))
    X = O.ref_normal(64 * 96, 0, 1, 2, 0).reshape(64, 96)
    W1 = O.ref_uniform(96 * 160, -0.034233, 0.034233, 2, 64 * 96).reshape(96, 160)
    b1 = np.zeros(160, np.float32)
    H = O.ref_gelu(O.ref_bias_add(O.ref_gemm(X, W1), b1).reshape(-1)).reshape(64, 160)
    cfg.update(c3_h=H)
    Q = O.ref_normal(4 * 64 * 32, 0, 1 / np.sqrt(32), 3, 0).reshape(4, 64, 32)
    K = O.ref_normal(4 * 64 * 32, 0, 1 / np.sqrt(32), 3, Q.size).reshape(4, 64, 32)
    V = O.ref_normal(4 * 64 * 32, 0, 1 / np.sqrt(32), 3, 2 * Q.size).reshape(4, 64, 32)
    S = O.ref_gemm_strided_batched(Q, K, float(np.float32(1 / np.sqrt(32))), None, 0.0, False, True)
    P = np.exp(S - S.max(-1, keepdims=True)).astype(np.float32)
    P = (P / P.sum(-1, keepdims=True)).astype(np.float32)
    O_ = O.ref_gemm_strided_batched(P, V)
    cfg.update(c4_s=S, c4_o=O_)
    Ag = O.ref_uniform(300 * 257, -1, 1, 4, 0).reshape(300, 257)
    xg = O.ref_uniform(257, -1, 1, 4, Ag.size)
    yg = O.ref_uniform(300, -1, 1, 4, Ag.size + 257)
    cfg.update(gemv_out=O.ref_gemv(Ag, xg, 0.75, yg, -0.5),
               gemv_t_out=O.ref_gemv(Ag, yg, 1.25, None, 0.0, True))
    G = (O.ref_normal(4096, 0, 3, 7, 0)).astype(np.float32)
    cfg.update(act_gelu=O.ref_gelu(G), act_gelu_tanh=O.ref_gelu(G, True),
               act_relu=O.ref_relu(G))
    cfg.update(philox_uniform_s0=O.ref_uniform(1031, -1, 1, 0, 0),
               philox_uniform_s4_off=O.ref_uniform(517, -1, 1, 4, 1234567),
               philox_normal_s1=O.ref_normal(1029, 0, 1, 1, 3),
               philox_normal_s3=O.ref_normal(515, 0, float(np.float32(1 / np.sqrt(128))), 3, 77))
    np.savez_compressed(os.path.join(HERE, "seeded_cases.npz"), **cfg)

    # softmax / log_softmax (src/ops/softmax.cpp) and attention (src/ops/attention.cpp) through the
    # reference, on Philox inputs regenerated by the tests (attention_inputs in tests/helpers.py):
    # the four cases of tests/ops/softmax_loss_test.cpp test_attention (plain, mask, causal, both
    # with scale 0.5; query 2 sees no key) and k/v broadcast over heads.
    att = {}
    x = O.ref_normal(3 * 5 * 17, 0, 30, 9, 0).reshape(3, 5, 17)
    x[0, 1, :] = -np.inf
    x[1, 2, 3] = np.nan
    x[2, 0, :] += 1000
    for axis in (-1, 1, 0):
        for log in (False, True):
            att[f"softmax_a{axis}_l{int(log)}"] = O.ref_softmax(x, axis, log)
    b, h, lq, lk, d, dv = 2, 3, 5, 7, 8, 4
    q = O.ref_normal(b * h * lq * d, 0, 1, 21, 0).reshape(b, h, lq, d)
    k = O.ref_normal(b * h * lk * d, 0, 1, 22, 0).reshape(b, h, lk, d)
    v = O.ref_normal(b * h * lk * dv, 0, 1, 23, 0).reshape(b, h, lk, dv)
    keep = np.array([[i != 2 and (i + j) % 3 != 0 for j in range(lk)] for i in range(lq)])
    for name, mask, causal, scale in (("plain", None, False, 0.0), ("mask", keep, False, 0.0),
                                      ("causal", None, True, 0.0), ("both", keep, True, 0.5)):
        att[f"attention_{name}"] = O.ref_attention(q, k, v, mask, causal, scale)
    k1 = O.ref_normal(b * lk * d, 0, 1, 24, 0).reshape(b, 1, lk, d)
    v1 = O.ref_normal(b * lk * dv, 0, 1, 25, 0).reshape(b, 1, lk, dv)
    att["attention_broadcast_kv"] = O.ref_attention(q, k1, v1)
    lq2 = 64
    q2 = O.ref_normal(4 * lq2 * 32, 0, 1 / np.sqrt(32), 26, 0).reshape(4, lq2, 32)
    k2 = O.ref_normal(4 * lq2 * 32, 0, 1 / np.sqrt(32), 27, 0).reshape(4, lq2, 32)
    v2 = O.ref_normal(4 * lq2 * 32, 0, 1 / np.sqrt(32), 28, 0).reshape(4, lq2, 32)
    att["attention_causal_64"] = O.ref_attention(q2, k2, v2, None, True)
    np.savez_compressed(os.path.join(HERE, "attention_cases.npz"), **att)

    # the backward closures of bias_add (src/ops/elementwise.cpp:263-283) and matmul
    # (src/ops/blas.cpp:220-230), run through the reference's autograd on Philox inputs
    # regenerated by the tests (backward_inputs in tests/helpers.py)
    bwd = {}
    for i, (rows, cols) in enumerate(BIAS_GRAD_SHAPES):
        g = O.ref_normal(rows * cols, 0, 1, 40 + i, 0).reshape(rows, cols)
        bwd[f"bias_grad_{rows}x{cols}"] = O.ref_bias_add_backward(g)
    for i, (m, k, n) in enumerate(MATMUL_BWD_SHAPES):
        a = O.ref_normal(m * k, 0, 1, 60 + i, 0).reshape(m, k)
        b = O.ref_normal(k * n, 0, 1, 60 + i, m * k).reshape(k, n)
        g = O.ref_normal(m * n, 0, 1, 60 + i, m * k + k * n).reshape(m, n)
        da, db = O.ref_matmul_backward(a, b, g)
        bwd[f"matmul_{m}x{k}x{n}_da"] = da
        bwd[f"matmul_{m}x{k}x{n}_db"] = db
    np.savez_compressed(os.path.join(HERE, "backward_cases.npz"), **bwd)

    # Tensor::contiguous() of the views in tests/helpers.py COPY_CASES (src/core/tensor.cpp:208-230
    # -> cpu::transpose_f32 / cpu::strided_copy_f32)
    sys.path.insert(0, os.path.dirname(HERE))
    from helpers import COPY_CASES, copy_case  # noqa: E402

    cpy = {}
    for i, case in enumerate(COPY_CASES):
        x, full = copy_case(i)
        cpy[case[0]] = O.ref_contiguous_view(x, case[2], full, case[4])
    np.savez_compressed(os.path.join(HERE, "copy_cases.npz"), **cpy)
    print("wrote", sorted(os.listdir(HERE)))


if __name__ == "__main__":
    main()
