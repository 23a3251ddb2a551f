"""CPU tests: the oracle (C restatement) pinned against the reference's golden vectors and its
tests' known answers, and against the reference library itself where it was built here."""
import numpy as np
import pytest

from helpers import assert_close, golden, make_input, seeded_inputs, softmax_rows, ulp_diff
from oracle import oracle as O

MATMUL_SHAPES = [(1, 1, 1), (1, 5, 1), (5, 1, 3), (3, 5, 7), (16, 16, 16), (17, 31, 13),
                 (64, 64, 64), (65, 129, 130), (100, 300, 50), (200, 100, 300), (2, 1000, 3),
                 (1000, 2, 3), (257, 129, 257)]


def test_philox_streams_bit_exact():
    g = golden("seeded_cases.npz")
    np.testing.assert_array_equal(O.uniform(1031, -1, 1, 0, 0), g["philox_uniform_s0"])
    np.testing.assert_array_equal(O.uniform(517, -1, 1, 4, 1234567), g["philox_uniform_s4_off"])
    np.testing.assert_array_equal(O.normal(1029, 0, 1, 1, 3), g["philox_normal_s1"])
    np.testing.assert_array_equal(O.normal(515, 0, float(np.float32(1 / np.sqrt(128))), 3, 77),
                                  g["philox_normal_s3"])


def test_philox_known_answer():
    """Philox4x32-10 known-answer vector (Random123 kat_vectors: counter 0, key 0)."""
    words = [O.lib().mfo_philox_word(0, 0, i) for i in range(4)]
    assert words == [0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8]


def test_known_values():
    g = golden("matmul_cases.npz")
    np.testing.assert_array_equal(O.gemm(g["known_a"], g["known_b"]), [[58, 64], [139, 154]])
    np.testing.assert_array_equal(g["known_c"], [[58, 64], [139, 154]])
    a = make_input(35, 3).reshape(5, 7)
    np.testing.assert_array_equal(O.gemm(a, np.eye(7, dtype=np.float32)), a)


def test_matmul_shapes_match_reference_exactly():
    g = golden("matmul_cases.npz")
    for (m, n, k) in MATMUL_SHAPES:
        a = make_input(m * k, 4).reshape(m, k)
        b = make_input(k * n, 5).reshape(k, n)
        np.testing.assert_array_equal(O.gemm(a, b), g[f"mm_{m}x{n}x{k}"], err_msg=f"{m}x{n}x{k}")


def test_seeded_configs():
    s = seeded_inputs()
    g = golden("seeded_cases.npz")
    got = O.gemm(s["c2_a"], s["c2_b"], 0.5, s["c2_c"], 1.0, False, True, bias=s["c2_bias"])
    mag = 0.5 * O.abs_product(s["c2_a"], s["c2_b"], False, True) + np.abs(s["c2_c"]) + \
        np.abs(s["c2_bias"])[None, :]
    assert_close(got, g["c2_out"], mag, (1e-6, 1e-7), "c2")
    h = O.activation(O.gemm(s["c3_x"], s["c3_w1"], bias=np.zeros(160, np.float32)), "gelu")
    assert_close(h, g["c3_h"], 1.2 * O.abs_product(s["c3_x"], s["c3_w1"]), (1e-6, 1e-7), "c3")
    scale = float(np.float32(1 / np.sqrt(32)))
    for i in range(4):
        S = O.gemm(s["c4_q"][i], s["c4_k"][i], scale, None, 0.0, False, True)
        assert_close(S, g["c4_s"][i], O.abs_product(s["c4_q"][i], s["c4_k"][i], False, True),
                     (1e-6, 1e-7), "c4 scores")
    P = softmax_rows(g["c4_s"])
    for i in range(4):
        assert_close(O.gemm(P[i], s["c4_v"][i]), g["c4_o"][i], O.abs_product(P[i], s["c4_v"][i]),
                     (1e-6, 1e-7), "c4 output")
    np.testing.assert_array_equal(O.gemv(s["gemv_a"], s["gemv_x"], 0.75, s["gemv_y"], -0.5),
                                  g["gemv_out"])
    np.testing.assert_array_equal(O.gemv(s["gemv_a"], s["gemv_y"], 1.25, None, 0.0, True),
                                  g["gemv_t_out"])
    np.testing.assert_array_equal(O.activation(s["act_x"], "relu"), g["act_relu"])
    assert ulp_diff(O.activation(s["act_x"], "gelu"), g["act_gelu"]).max() == 0
    assert ulp_diff(O.activation(s["act_x"], "gelu_tanh"), g["act_gelu_tanh"]).max() == 0


def test_batched_cases_match_reference():
    """The restated BatchedGemm (with the odometer offsets) reproduces the reference's 19 API
    cases bit for bit (quarter-integer inputs)."""
    from test_gemm_gpu import BATCHED_CASES

    g = golden("batched_cases.npz")
    for i, (name, ash, bsh, ta, tb, alpha, csh, beta) in enumerate(BATCHED_CASES):
        want = g[f"case{i}_out"]
        if want.size == 0:
            continue
        a = make_input(int(np.prod(ash)), 4).reshape(ash)
        b = make_input(int(np.prod(bsh)), 5).reshape(bsh)
        left = np.swapaxes(a, -1, -2) if ta else a
        right = np.swapaxes(b, -1, -2) if tb else b
        m, k, n = left.shape[-2], left.shape[-1], right.shape[-1]
        bshape = np.broadcast_shapes(left.shape[:-2], right.shape[:-2])
        batch = int(np.prod(bshape)) if bshape else 1
        L = np.ascontiguousarray(np.broadcast_to(left, bshape + (m, k))).reshape(batch, m, k)
        R = np.ascontiguousarray(np.broadcast_to(right, bshape + (k, n))).reshape(batch, k, n)
        c0 = None
        if csh and beta != 0.0:
            c = make_input(int(np.prod(csh)), 6).reshape(csh)
            c0 = np.ascontiguousarray(np.broadcast_to(c, want.shape), np.float32).reshape(-1)
        got = O.gemm_batched_raw(L.reshape(-1), np.arange(batch) * m * k, k, 1, R.reshape(-1),
                                 np.arange(batch) * k * n, n, 1, batch, m, n, k, alpha, c0,
                                 (n, 1, m * n), beta)
        np.testing.assert_array_equal(got.reshape(want.shape), want, err_msg=name)


@pytest.mark.skipif(O.reference() is None, reason="reference library not built here")
def test_restatement_tracks_reference_on_random_inputs():
    rng = np.random.default_rng(5)
    for (m, n, k) in [(33, 47, 1000), (128, 64, 300)]:
        a = rng.standard_normal((m, k)).astype(np.float32)
        b = rng.standard_normal((k, n)).astype(np.float32)
        c = rng.standard_normal((m, n)).astype(np.float32)
        got = O.gemm(a, b, 1.5, c, -0.5)
        want = O.ref_gemm(a, b, 1.5, c, -0.5)
        mag = 1.5 * O.abs_product(a, b) + 0.5 * np.abs(c)
        assert_close(got, want, mag, (1e-6, 1e-7), f"{m}x{n}x{k}")


def test_softmax_and_attention_restatements_match_reference():
    """Softmax restated bit for bit (expf per element, double sum); the composed attention oracle
    within float rounding of the reference's attention (its own tests allow 1e-4)."""
    from helpers import attention_inputs

    g = golden("attention_cases.npz")
    a = attention_inputs()
    for axis in (-1, 1, 0):
        for log in (False, True):
            np.testing.assert_array_equal(O.softmax(a["softmax_x"], axis, log),
                                          g[f"softmax_a{axis}_l{int(log)}"])
    cases = {"plain": (None, False, 0.0), "mask": (a["keep"], False, 0.0),
             "causal": (None, True, 0.0), "both": (a["keep"], True, 0.5)}
    for name, (mask, causal, scale) in cases.items():
        got = O.attention(a["q"], a["k"], a["v"], mask, causal, scale)
        np.testing.assert_allclose(got, g[f"attention_{name}"], rtol=1e-5, atol=1e-6,
                                   err_msg=name)
    np.testing.assert_allclose(O.attention(a["q"], a["k1"], a["v1"]), g["attention_broadcast_kv"],
                               rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(O.attention(a["q2"], a["k2"], a["v2"], None, True),
                               g["attention_causal_64"], rtol=1e-5, atol=1e-6)


def test_backward_restatements_match_golden():
    """bias_add's bias gradient (row-order float sums) and matmul's backward products, restated,
    equal the reference's autograd results bit for bit (tests/golden/backward_cases.npz)."""
    from helpers import backward_inputs

    g = golden("backward_cases.npz")
    inp = backward_inputs()
    for name, arr in inp.items():
        if name.startswith("bias_grad"):
            np.testing.assert_array_equal(O.bias_grad(arr), g[name], err_msg=name)
        else:
            a, b, grad = arr
            da, db = O.matmul_backward(a, b, grad)
            np.testing.assert_array_equal(da, g[name + "_da"], err_msg=name)
            np.testing.assert_array_equal(db, g[name + "_db"], err_msg=name)


@pytest.mark.skipif(O.reference() is None, reason="reference library not built here")
def test_bias_grad_restatement_on_ragged_and_empty_shapes():
    rng = np.random.default_rng(11)
    for rows, cols in [(7, 1), (129, 33), (5000, 3)]:
        x = rng.standard_normal((rows, cols)).astype(np.float32) * 100
        np.testing.assert_array_equal(O.bias_grad(x), O.ref_bias_add_backward(x),
                                      err_msg=f"{rows}x{cols}")
    # no rows: the loop adds nothing (the reference records no graph for an empty input)
    np.testing.assert_array_equal(O.bias_grad(np.zeros((0, 5), np.float32)), np.zeros(5))


def test_strided_copy_restatement_matches_reference_views():
    """oracle.strided_copy (cpu::strided_copy_f32 restated) over the reference's view arithmetic
    reproduces the reference's Tensor::contiguous() on every COPY_CASES view, bit for bit."""
    from helpers import COPY_CASES, copy_case

    gold = golden("copy_cases.npz")
    for i, case in enumerate(COPY_CASES):
        x, full = copy_case(i)
        off, shape, strides = O.view_recipe_strided(x.shape, case[2], full, case[4])
        got = O.strided_copy(x, off, shape, strides)
        want = gold[case[0]]
        assert got.shape == want.shape, case[0]
        assert np.array_equal(got, want), case[0]


@pytest.mark.skipif(O.reference() is None, reason="reference library not built here")
@pytest.mark.parametrize("shape", [(300, 64, 200), (100, 1000, 70)])
def test_restatement_matches_reference_on_infinite_operands(shape):
    """The ±inf / NaN pattern the GPU tests hold the kernels to (tests/test_gemm_gpu.py,
    test_infinite_operands*) is the restatement's: pinned here to the reference built from its
    sources, entry for entry, with infinities that meet zeros, each other and finite values."""
    m, n, k = shape
    rng = np.random.default_rng(m + n + k)
    a = (rng.integers(-16, 17, (m, k)) / 4).astype(np.float32)
    b = (rng.integers(-16, 17, (k, n)) / 4).astype(np.float32)
    a[3, 5] = np.inf
    a[m // 2, 2] = -np.inf
    a[m // 2, 9] = np.inf
    b[7, n - 1] = np.inf
    b[11, 0] = np.nan
    want = O.ref_gemm(a, b)
    got = O.gemm(a, b)
    assert (~np.isfinite(want)).any()
    np.testing.assert_array_equal(np.isnan(got), np.isnan(want))
    np.testing.assert_array_equal(got[~np.isnan(want)], want[~np.isnan(want)])


@pytest.mark.skipif(O.reference() is None, reason="reference library not built here")
@pytest.mark.parametrize("rows,cols", [(1, 1024), (3, 1001), (77, 1280), (513, 515), (64, 8195)])
def test_gemv_restatement_matches_reference_on_ragged_widths(rows, cols):
    """The gemv restatement against the reference's own gemv (double accumulation in row order,
    src/backends/cpu/ops/blas/blas.cpp:55-80) on the widths the GPU gemv tests use: equal after
    rounding to float, 1 ulp allowed for the summation order."""
    rng = np.random.default_rng(rows * 31 + cols)
    a = rng.standard_normal((rows, cols)).astype(np.float32)
    x = rng.standard_normal(cols).astype(np.float32)
    y = rng.standard_normal(rows).astype(np.float32)
    got = O.gemv(a, x, -0.5, y, 2.0)
    want = O.ref_gemv(a, x, -0.5, y, 2.0)
    assert np.max(ulp_diff(got, want)) <= 1
