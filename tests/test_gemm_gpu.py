"""GPU parity of the tensor-core GEMM path against the oracle and the reference's golden vectors.

Modelled on the reference's tests/ops/matmul_test.cpp and tests/ops/gemm_batched_test.cpp: the
same shapes, the same quarter-integer inputs (exact in tf32, so every product and short sum is
exact and the results must match bit for bit in both precisions), strided views, empty shapes,
known values; then seeded Philox inputs against the restated CPU algorithm within the bounds of
the path (3xTF32: 1e-5*(|A||B|) + 1e-6; 1xTF32: 2e-3*(|A||B|) + 1e-6).
"""
import numpy as np
import pytest
import torch

import mensurflow_b200 as mf
from helpers import (TOL_1X, TOL_3X, assert_close, golden, make_input, seeded_inputs,
                     softmax_rows)
from oracle import oracle as O

pytestmark = pytest.mark.gpu

PRECISIONS = ["3xtf32", "1xtf32"]
MATMUL_SHAPES = [(1, 1, 1), (1, 5, 1), (5, 1, 3), (3, 5, 7), (16, 16, 16), (17, 31, 13),
                 (64, 64, 64), (65, 129, 130), (100, 300, 50), (200, 100, 300), (2, 1000, 3),
                 (1000, 2, 3), (257, 129, 257)]


def dev(x, cuda):
    return torch.from_numpy(np.ascontiguousarray(x)).to(cuda)


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


def no_fault():
    assert mf.device_status() == 0, "a kernel recorded a pipeline timeout"


def tol(precision):
    return TOL_3X if precision == "3xtf32" else TOL_1X


def test_known_values(cuda):
    g = golden("matmul_cases.npz")
    for p in PRECISIONS:
        c = mf.matmul(dev(g["known_a"], cuda), dev(g["known_b"], cuda), precision=p)
        assert c.shape == (2, 2) and c.is_contiguous()
        np.testing.assert_array_equal(host(c), [[58, 64], [139, 154]])
        np.testing.assert_array_equal(host(c), g["known_c"])
    # A x I == A exactly
    m, k = 5, 7
    a = make_input(m * k, 3).reshape(m, k)
    for p in PRECISIONS:
        c = mf.matmul(dev(a, cuda), torch.eye(k, device=cuda), precision=p)
        np.testing.assert_array_equal(host(c), a)
    no_fault()


@pytest.mark.parametrize("precision", PRECISIONS)
def test_sizes_exact(cuda, precision):
    """The reference's matmul shape table; exact inputs give exact (bit-identical) results."""
    g = golden("matmul_cases.npz")
    for (m, n, k) in MATMUL_SHAPES:
        a = make_input(m * k, 4).reshape(m, k)
        b = make_input(k * n, 5).reshape(k, n)
        c = host(mf.matmul(dev(a, cuda), dev(b, cuda), precision=precision))
        np.testing.assert_array_equal(c, g[f"mm_{m}x{n}x{k}"], err_msg=f"{m}x{n}x{k}")
    no_fault()


def make_view(values, rows, cols, kind, cuda):
    """The four layouts of matmul_test.cpp make_view: contiguous, column slice of a wider
    matrix, transposed, transposed and sliced; the view always has shape (rows, cols)."""
    v = torch.from_numpy(values.reshape(rows, cols)).to(cuda)
    if kind == 0:
        return v
    if kind == 1:
        big = torch.full((rows + 2, cols + 9), -77.0, device=cuda)
        big[1:1 + rows, 3:3 + cols] = v
        return big[1:1 + rows, 3:3 + cols]
    if kind == 2:
        return v.t().contiguous().t()
    big = torch.full((cols + 3, rows + 5), -77.0, device=cuda)
    big[2:2 + cols, 4:4 + rows] = v.t()
    return big[2:2 + cols, 4:4 + rows].t()


@pytest.mark.parametrize("precision", PRECISIONS)
def test_strided_views(cuda, precision):
    """Every combination of layouts for A and B (matmul_test.cpp test_strided_large)."""
    for (m, n, k) in [(70, 60, 90), (130, 200, 150), (300, 300, 300)]:
        a = make_input(m * k, 21)
        b = make_input(k * n, 22)
        want = O.gemm(a.reshape(m, k), b.reshape(k, n))
        for ka in range(4):
            for kb in range(4):
                va = make_view(a, m, k, ka, cuda)
                vb = make_view(b, k, n, kb, cuda)
                got = host(mf.matmul(va, vb, precision=precision))
                np.testing.assert_array_equal(got, want, err_msg=f"{m}x{n}x{k} A{ka} B{kb}")
    no_fault()


def test_empty_and_k0(cuda):
    z = mf.matmul(torch.empty(3, 0, device=cuda), torch.empty(0, 4, device=cuda))
    assert z.shape == (3, 4)
    np.testing.assert_array_equal(host(z), np.zeros((3, 4), np.float32))
    assert mf.matmul(torch.empty(0, 5, device=cuda), torch.empty(5, 2, device=cuda)).shape == (0, 2)
    assert mf.matmul(torch.empty(2, 5, device=cuda), torch.empty(5, 0, device=cuda)).shape == (2, 0)
    c = torch.arange(12, dtype=torch.float32, device=cuda).reshape(3, 4)
    r = mf.gemm(torch.empty(3, 0, device=cuda), torch.empty(0, 4, device=cuda), 2.0, c, 0.5)
    np.testing.assert_array_equal(host(r), 0.5 * np.arange(12, dtype=np.float32).reshape(3, 4))
    no_fault()


def test_errors(cuda):
    m23 = torch.ones(2, 3, device=cuda)
    m32 = torch.ones(3, 2, device=cuda)
    vec = torch.ones(3, device=cuda)
    with pytest.raises(ValueError):
        mf.matmul(m23, m23)
    with pytest.raises(ValueError):
        mf.matmul(vec, m32)
    with pytest.raises(ValueError):
        mf.matmul(m23, vec)
    with pytest.raises(ValueError):
        mf.matmul(None, m32)
    with pytest.raises(ValueError):
        mf.gemm(m23, m32, 1.0, None, 1.0)
    with pytest.raises(ValueError):
        mf.matmul(m23, m32.double())
    with pytest.raises(NotImplementedError):
        mf.matmul(m23.double(), m32.double())


@pytest.mark.parametrize("precision", PRECISIONS)
def test_seeded_c2_shape(cuda, precision):
    """C2-shaped gemm (alpha 0.5, beta 1, transB, fused bias) on the reference's Philox inputs,
    against the reference's own output."""
    s = seeded_inputs()
    want = golden("seeded_cases.npz")["c2_out"]
    got = host(mf.gemm(dev(s["c2_a"], cuda), dev(s["c2_b"], cuda), 0.5, dev(s["c2_c"], cuda), 1.0,
                       False, True, bias=dev(s["c2_bias"], cuda), precision=precision))
    mag = 0.5 * O.abs_product(s["c2_a"], s["c2_b"], False, True) + np.abs(s["c2_c"]) + \
        np.abs(s["c2_bias"])[None, :]
    assert_close(got, want, mag, tol(precision), f"c2 {precision}")
    no_fault()


@pytest.mark.parametrize("precision", PRECISIONS)
@pytest.mark.parametrize("shape", [(256, 384, 1000), (384, 130, 4099), (129, 257, 33)])
@pytest.mark.parametrize("trans", [(False, False), (False, True), (True, False), (True, True)])
def test_random_gemm(cuda, precision, shape, trans):
    m, n, k = shape
    ta, tb = trans
    rng = np.random.default_rng(m * 7 + n * 3 + k)
    a = rng.standard_normal((k, m) if ta else (m, k)).astype(np.float32)
    b = rng.standard_normal((n, k) if tb else (k, n)).astype(np.float32)
    c = rng.standard_normal((m, n)).astype(np.float32)
    bias = rng.uniform(-0.1, 0.1, n).astype(np.float32)
    want = O.gemm(a, b, -0.75, c, 2.0, ta, tb, bias=bias)
    got = host(mf.gemm(dev(a, cuda), dev(b, cuda), -0.75, dev(c, cuda), 2.0, ta, tb,
                       bias=dev(bias, cuda), precision=precision))
    mag = 0.75 * O.abs_product(a, b, ta, tb) + 2 * np.abs(c) + np.abs(bias)[None, :]
    assert_close(got, want, mag, tol(precision), f"{shape} {trans} {precision}")
    no_fault()


@pytest.mark.parametrize("precision", PRECISIONS)
@pytest.mark.parametrize("shape", [(300, 64, 200), (300, 256, 200), (300, 640, 200), (100, 64, 70)])
def test_nan_operands(cuda, precision, shape):
    """A NaN in a row of A makes that row of C NaN on every kernel variant (A split in tensor
    memory for N <= 128, in shared memory for N <= 384, pre-split operands above, 1xTF32);
    the other rows are unaffected. The 3xTF32 split gives a NaN hi with a zero lo."""
    m, n, k = shape
    rng = np.random.default_rng(m + n + k)
    a = rng.standard_normal((m, k)).astype(np.float32)
    b = rng.standard_normal((k, n)).astype(np.float32)
    bad = [3, m // 2, m - 1]
    for r in bad:
        a[r, (r * 7) % k] = np.nan
    got = host(mf.matmul(dev(a, cuda), dev(b, cuda), precision=precision))
    assert np.isnan(got[bad]).all()
    good = np.setdiff1d(np.arange(m), bad)
    a_ok = a[good]
    assert_close(got[good], O.gemm(a_ok, b), O.abs_product(a_ok, b), tol(precision),
                 f"finite rows {shape} {precision}")
    no_fault()


@pytest.mark.parametrize("act", ["relu", "gelu", "gelu_tanh"])
def test_fused_activation(cuda, act):
    s = seeded_inputs()
    x, w = s["c3_x"], s["c3_w1"]
    b1 = np.linspace(-0.05, 0.05, w.shape[1]).astype(np.float32)
    pre = O.gemm(x, w, bias=b1)
    want = O.activation(pre, act)
    got = host(mf.linear(dev(x, cuda), dev(w, cuda), dev(b1, cuda), act))
    mag = O.abs_product(x, w) + np.abs(b1)[None, :]
    # the activation's slope is at most ~1.13, plus 2 ulp of rounding in the result
    bound_rel, bound_abs = TOL_3X
    assert_close(got, want, 1.2 * mag + np.abs(want) * 2.5e-7 / bound_rel, TOL_3X, act)
    if act == "gelu":
        np.testing.assert_array_equal(  # golden: the reference's gelu(x W1 + 0)
            host(mf.linear(dev(x, cuda), dev(w, cuda), torch.zeros(w.shape[1], device=cuda),
                           "gelu")).shape, golden("seeded_cases.npz")["c3_h"].shape)
    no_fault()


def test_guard_regions(cuda):
    """Output written into the middle of a NaN-poisoned buffer: exactly the [m, n] window
    changes (the reference poisons C the same way in gemm_packed_test.cpp:38)."""
    m, n, k = 131, 77, 45
    a = make_input(m * k, 9).reshape(m, k)
    b = make_input(k * n, 10).reshape(k, n)
    buf = torch.full((m + 4, n + 40), float("nan"), device=cuda)
    window = buf[2:2 + m, 5:5 + n]
    mf.gemm(dev(a, cuda), dev(b, cuda), out=window)
    got = host(buf)
    np.testing.assert_array_equal(got[2:2 + m, 5:5 + n], O.gemm(a, b))
    mask = np.ones_like(got, bool)
    mask[2:2 + m, 5:5 + n] = False
    assert np.isnan(got[mask]).all(), "a write landed outside the output window"
    no_fault()


# ---- batched -------------------------------------------------------------------------------

BATCHED_CASES = [
    ("plain batch", (3, 4, 5), (3, 5, 2), False, False, 1.0, (), 0.0),
    ("shared right-hand side", (4, 3, 5), (5, 2), False, False, 1.0, (), 0.0),
    ("shared left-hand side", (3, 5), (4, 5, 2), False, False, 1.0, (), 0.0),
    ("broadcast batch dims", (2, 1, 3, 4), (5, 4, 6), False, False, 1.0, (), 0.0),
    ("plain matrices", (7, 9), (9, 4), False, False, 1.0, (), 0.0),
    ("transpose a", (2, 5, 3), (2, 5, 4), True, False, 1.0, (), 0.0),
    ("transpose b", (2, 3, 5), (2, 4, 5), False, True, 1.0, (), 0.0),
    ("transpose both", (2, 5, 3), (1, 4, 5), True, True, 1.0, (), 0.0),
    ("alpha only", (2, 3, 4), (2, 4, 5), False, False, -1.5, (), 0.0),
    ("alpha and full c", (2, 3, 4), (2, 4, 5), False, False, 2.0, (2, 3, 5), 0.5),
    ("c broadcast over batch", (4, 3, 4), (4, 5), False, False, 1.0, (3, 5), -1.0),
    ("c as a row", (2, 3, 4), (2, 4, 5), False, False, 1.0, (5,), 1.0),
    ("c given, beta 0", (2, 3, 4), (2, 4, 5), False, False, 1.0, (2, 3, 5), 0.0),
    ("empty batch", (0, 3, 4), (0, 4, 5), False, False, 1.0, (), 0.0),
    ("empty rows", (2, 0, 4), (2, 4, 5), False, False, 1.0, (), 0.0),
    ("k is 0", (2, 3, 0), (2, 0, 5), False, False, 1.0, (), 0.0),
    ("k is 0 with c", (2, 3, 0), (2, 0, 5), False, False, 1.0, (2, 3, 5), 3.0),
    ("many small", (100, 2, 3), (100, 3, 2), False, False, 1.0, (), 0.0),
    ("larger", (3, 70, 90), (3, 90, 60), False, False, 1.0, (), 0.0),
]


def _prod(s):
    return int(np.prod(s)) if len(s) else 1


@pytest.mark.parametrize("precision", PRECISIONS)
def test_batched_api_cases(cuda, precision):
    """The reference's 19 gemm_strided_batched API cases (gemm_batched_test.cpp:202-220),
    against the reference's own outputs; exact inputs, so bit-identical."""
    g = golden("batched_cases.npz")
    for i, (name, ash, bsh, ta, tb, alpha, csh, beta) in enumerate(BATCHED_CASES):
        a = make_input(_prod(ash), 4).reshape(ash)
        b = make_input(_prod(bsh), 5).reshape(bsh)
        c = dev(make_input(_prod(csh), 6).reshape(csh), cuda) if csh else None
        got = mf.gemm_strided_batched(dev(a, cuda), dev(b, cuda), alpha, c, beta, ta, tb,
                                      precision=precision)
        want = g[f"case{i}_out"]
        assert tuple(got.shape) == want.shape, name
        assert got.is_contiguous()
        np.testing.assert_array_equal(host(got), want, err_msg=name)
    no_fault()


def test_batched_views(cuda):
    """Sliced batch, transposed view without the flag, expanded batch (gemm_batched_test.cpp
    test_views): each equals its packed copy."""
    full = dev(make_input(6 * 4 * 5, 7).reshape(6, 4, 5), cuda)
    every_other = full[0:6:2]
    b = dev(make_input(3 * 5 * 2, 8).reshape(3, 5, 2), cuda)
    np.testing.assert_array_equal(host(mf.gemm_strided_batched(every_other, b)),
                                  host(mf.gemm_strided_batched(every_other.contiguous(), b)))
    bt = dev(make_input(3 * 2 * 5, 9).reshape(3, 2, 5), cuda)
    packed = every_other.contiguous()
    np.testing.assert_array_equal(
        host(mf.gemm_strided_batched(packed, bt.transpose(1, 2))),
        host(mf.gemm_strided_batched(packed, bt, 1.0, None, 0.0, False, True)))
    one = dev(make_input(4 * 5, 10).reshape(1, 4, 5), cuda)
    expanded = one.expand(3, 4, 5)
    np.testing.assert_array_equal(host(mf.gemm_strided_batched(expanded, b)),
                                  host(mf.gemm_strided_batched(expanded.contiguous(), b)))
    x = dev(make_input(8 * 6, 11).reshape(8, 6), cuda)
    y = dev(make_input(6 * 3, 12).reshape(6, 3), cuda)
    np.testing.assert_array_equal(host(mf.gemm_strided_batched(x, y)), host(mf.matmul(x, y)))
    no_fault()


@pytest.mark.parametrize("precision", PRECISIONS)
def test_attention_gemms(cuda, precision):
    """C4-shaped attention GEMMs (S = Q K^T / sqrt(d), O = P V) against the reference."""
    s = seeded_inputs()
    g = golden("seeded_cases.npz")
    q, k, v = (dev(s[x], cuda) for x in ("c4_q", "c4_k", "c4_v"))
    scale = float(np.float32(1 / np.sqrt(32)))
    S = host(mf.gemm_strided_batched(q, k, scale, None, 0.0, False, True, precision=precision))
    mag_s = np.stack([scale * O.abs_product(s["c4_q"][i], s["c4_k"][i], False, True)
                      for i in range(4)])
    assert_close(S, g["c4_s"], mag_s, tol(precision), "scores")
    P = softmax_rows(g["c4_s"])
    out = host(mf.gemm_strided_batched(dev(P, cuda), v, precision=precision))
    mag_o = np.stack([O.abs_product(P[i], s["c4_v"][i]) for i in range(4)])
    assert_close(out, g["c4_o"], mag_o, tol(precision), "attention output")
    no_fault()


# ---- gemv / bias_add / activations -------------------------------------------------------------

def test_gemv(cuda):
    s = seeded_inputs()
    g = golden("seeded_cases.npz")
    got = host(mf.gemv(dev(s["gemv_a"], cuda), dev(s["gemv_x"], cuda), 0.75, dev(s["gemv_y"], cuda),
                       -0.5))
    # double accumulation on both sides: equal after rounding to float (allow 1 ulp)
    assert np.max(np.abs(got.view(np.int32) - g["gemv_out"].view(np.int32))) <= 1
    got_t = host(mf.gemv(dev(s["gemv_a"], cuda), dev(s["gemv_y"], cuda), 1.25, None, 0.0, True))
    assert np.max(np.abs(got_t.view(np.int32) - g["gemv_t_out"].view(np.int32))) <= 1
    a = np.random.default_rng(1).standard_normal((1031, 4096)).astype(np.float32)
    x = np.random.default_rng(2).standard_normal(4096).astype(np.float32)
    got = host(mf.matvec(dev(a, cuda), dev(x, cuda)))
    assert np.max(np.abs(got.view(np.int32) - O.gemv(a, x).view(np.int32))) <= 1
    no_fault()


@pytest.mark.parametrize("rows,cols,width", [
    (1, 1024, 1024),       # one row: a single warp
    (3, 1001, 1004),       # a column slice: lda 1004, one element past the last 16-byte chunk
    (77, 1280, 1280),      # one full round of eight loads per lane, then single chunks
    (9473, 515, 520),      # more rows than warps in flight; 3 elements past the chunks
    (20000, 8195, 8200),   # long rows with a ragged end, rows revisited by the grid stride
])
def test_gemv_ragged_rows_and_widths(cuda, rows, cols, width):
    """The streaming gemv on row counts around its grid of warps and on widths that end inside
    a round of loads or past the last 16-byte chunk (row-strided views: lda > cols), against the
    oracle's double accumulation (equal after rounding to float, 1 ulp allowed)."""
    rng = np.random.default_rng(rows + cols)
    full = rng.standard_normal((rows, width)).astype(np.float32)
    a = full[:, :cols]
    x = rng.standard_normal(cols).astype(np.float32)
    y = rng.standard_normal(rows).astype(np.float32)
    da = dev(full, cuda)[:, :cols]
    got = host(mf.gemv(da, dev(x, cuda), -0.5, dev(y, cuda), 2.0))
    want = O.gemv(a, x, -0.5, y, 2.0)
    assert np.max(np.abs(got.view(np.int32).astype(np.int64) -
                         want.view(np.int32).astype(np.int64))) <= 1
    no_fault()


def test_bias_add_and_activations(cuda):
    s = seeded_inputs()
    g = golden("seeded_cases.npz")
    x = s["act_x"]
    np.testing.assert_array_equal(host(mf.relu(dev(x, cuda))), g["act_relu"])
    for approx, key in ((False, "act_gelu"), (True, "act_gelu_tanh")):
        got = host(mf.gelu(dev(x, cuda), approximate=approx))
        d = np.abs(got.view(np.int32).astype(np.int64) - g[key].view(np.int32).astype(np.int64))
        assert d.max() <= 1, f"gelu approximate={approx}: {d.max()} ulp"
    xb = x.reshape(64, 64)
    bias = np.linspace(-1, 1, 64).astype(np.float32)
    np.testing.assert_array_equal(host(mf.bias_add(dev(xb, cuda), dev(bias, cuda))),
                                  O.bias_add(xb, bias))
    xo = np.random.default_rng(3).standard_normal((7, 13)).astype(np.float32)  # odd width
    bo = np.random.default_rng(4).standard_normal(13).astype(np.float32)
    np.testing.assert_array_equal(host(mf.bias_add(dev(xo, cuda), dev(bo, cuda))),
                                  O.bias_add(xo, bo))
    with pytest.raises(ValueError):
        mf.bias_add(dev(xb, cuda), dev(bias[:10], cuda))
    no_fault()


def test_precision_knob(cuda):
    assert mf.get_default_precision() == "3xtf32"
    mf.set_default_precision("1xtf32")
    try:
        assert mf.get_default_precision() == "1xtf32"
    finally:
        mf.set_default_precision("3xtf32")


@pytest.mark.parametrize("act,approx", [("gelu", False), ("gelu_tanh", True)])
def test_epilogue_activation_accuracy(cuda, act, approx):
    """The fused epilogue evaluates GELU in fp32 (erfcf with the argument carried as a float
    pair). A k = 0 GEMM with beta = 1 returns act(0 + C_in) exactly, isolating the activation:
    against the reference's double evaluation it stays within a few ulp (and relative 1e-6)."""
    x = np.concatenate([seeded_inputs()["act_x"], np.linspace(-12, 12, 4001, dtype=np.float32),
                        np.array([0.0, -0.0, 1e-30, -1e-30, 3.4e38, -3.4e38], np.float32)])
    x = x.astype(np.float32).reshape(-1, 1)
    c = dev(x, cuda)
    got = host(mf.gemm(torch.empty(x.shape[0], 0, device=cuda), torch.empty(0, 1, device=cuda),
                       1.0, c, 1.0, activation=act))
    want = O.activation(x, act)
    from helpers import ulp_diff
    d = ulp_diff(got, want)
    big = np.abs(want) > 1e-30
    rel = np.abs(got[big].astype(np.float64) - want[big]) / np.abs(want[big].astype(np.float64))
    print(f"{act}: max ulp {d.max()}, max rel {rel.max():.3e}")
    assert d[np.abs(x) < 10].max() <= 8, f"{act}: {d.max()} ulp"
    assert rel.max() <= 2e-6
    ref_gelu = golden("seeded_cases.npz")["act_gelu_tanh" if approx else "act_gelu"]
    assert ulp_diff(got[:4096, 0], ref_gelu).max() <= 8
    no_fault()


def test_tf32_conversion_of_raw_fp32_operands(cuda):
    """Known answer for how the tensor cores read an fp32 operand as tf32 (1xTF32 reads A in
    place): a = 1 + 3*2^-12 has 0.75 ulp of tf32 beyond 1, so truncation gives 1 and rounding
    gives 1 + 2^-10. Either is within the 1xTF32 bound; the test records which one the hardware
    does (the 3xTF32 paths never depend on it: they round hi and lo explicitly)."""
    a = torch.zeros(1, 32, device=cuda)
    a[0, 0] = 1.0 + 3.0 * 2.0 ** -12
    b = torch.zeros(32, 1, device=cuda)
    b[0, 0] = 1.0
    got = float(host(mf.matmul(a, b, precision="1xtf32"))[0, 0])
    print(f"tf32 conversion of raw fp32: {'truncation' if got == 1.0 else 'rounding'} ({got!r})")
    assert got in (1.0, 1.0 + 2.0 ** -10)
    got3 = float(host(mf.matmul(a, b, precision="3xtf32"))[0, 0])
    assert got3 == 1.0 + 3.0 * 2.0 ** -12  # the split keeps every bit
    no_fault()


@pytest.mark.parametrize("chunks", [4, None])
@pytest.mark.parametrize("trans", [(False, True), (True, False)])
def test_host_tensors_with_gpu_execution(cuda, trans, chunks):
    """Host inputs with execution="gpu": copied to the device, computed, copied back (the
    reference's run_on for data that lives elsewhere), pipelined by row blocks (four equal ones,
    or the default schedule: 640, 256, 128, 128, 128 and 20 rows here) — the same values as the
    device-resident call."""
    ta, tb = trans
    m, n, k = 1300, 700, 900
    rng = np.random.default_rng(11)
    a = rng.standard_normal((k, m) if ta else (m, k)).astype(np.float32)
    b = rng.standard_normal((n, k) if tb else (k, n)).astype(np.float32)
    c = rng.standard_normal((m, n)).astype(np.float32)
    bias = rng.uniform(-0.1, 0.1, n).astype(np.float32)
    ha, hb, hc, hbias = (torch.from_numpy(x).pin_memory() for x in (a, b, c, bias))
    got = mf.gemm(ha, hb, 0.5, hc, 1.0, ta, tb, bias=hbias, execution="gpu", chunks=chunks)
    assert got.device.type == "cpu" and tuple(got.shape) == (m, n)
    want = host(mf.gemm(dev(a, cuda), dev(b, cuda), 0.5, dev(c, cuda), 1.0, ta, tb,
                        bias=dev(bias, cuda)))
    mag = 0.5 * O.abs_product(a, b, ta, tb) + np.abs(c) + np.abs(bias)[None, :]
    assert_close(got.numpy(), want, mag, TOL_3X, "host path vs device path")
    assert_close(got.numpy(), O.gemm(a, b, 0.5, c, 1.0, ta, tb, bias=bias), mag, TOL_3X,
                 "host path vs oracle")
    with pytest.raises(NotImplementedError):
        mf.gemm(ha, hb, transpose_a=ta, transpose_b=tb)  # "auto" on host data: no CPU kernel here
    no_fault()


# Shapes whose last wave of tiles would leave most SM pairs idle, so the kernel shares that
# wave's k-iterations across every unit (stream-K tail) and sums the parts of a tile in k order:
# (m, n, k, batch). Covers the pre-split kernel (n > 384), the in-kernel split of A in shared
# memory (128 < n <= 384) and in tensor memory (n <= 128), the one-CTA kernel (m <= 128), a
# batch, and the C3 MLP shapes.
STREAM_K_SHAPES = [(1024, 1024, 1024, 1), (1024, 300, 2048, 1), (2048, 128, 2048, 1),
                   (100, 1000, 4096, 1), (300, 260, 800, 3), (4096, 4096, 1024, 1),
                   (4096, 1024, 4096, 1)]


@pytest.mark.parametrize("precision", PRECISIONS)
@pytest.mark.parametrize("shape", STREAM_K_SHAPES, ids=lambda s: "x".join(map(str, s)))
def test_stream_k_tail(cuda, shape, precision):
    """Seeded inputs against the oracle within the path's bound, with the full epilogue (alpha,
    beta*C, bias, GELU) applied to the summed parts; the same call twice gives the same bits
    (the parts are summed in a fixed order, whichever unit finishes last); and quarter-integer
    inputs stay exact."""
    m, n, k, batch = shape
    rng = np.random.default_rng(m + 7 * n + 13 * k + batch)
    a = rng.standard_normal((batch, m, k)).astype(np.float32)
    b = rng.standard_normal((batch, k, n)).astype(np.float32)
    c = rng.standard_normal((batch, m, n)).astype(np.float32)
    bias = rng.uniform(-0.1, 0.1, n).astype(np.float32)
    ta, tb, tc, tbias = dev(a, cuda), dev(b, cuda), dev(c, cuda), dev(bias, cuda)
    for i in range(batch):
        got = mf.gemm(ta[i], tb[i], 0.5, tc[i], 1.0, bias=tbias, activation="gelu",
                      precision=precision)
        again = mf.gemm(ta[i], tb[i], 0.5, tc[i], 1.0, bias=tbias, activation="gelu",
                        precision=precision)
        assert torch.equal(got, again), "stream-K parts summed in a run-dependent order"
        want = O.activation(O.gemm(a[i], b[i], 0.5, c[i], 1.0, bias=bias), "gelu")
        mag = 0.5 * O.abs_product(a[i], b[i]) + np.abs(c[i]) + np.abs(bias)[None, :]
        rel, ab = tol(precision)
        assert_close(host(got), want, 1.2 * mag, (rel, ab + 4e-7), f"{shape} [{i}]")
    if batch > 1:
        got = mf.gemm_strided_batched(ta, tb, 0.5, tc, 1.0, precision=precision)
        for i in range(batch):
            want = O.gemm(a[i], b[i], 0.5, c[i], 1.0)
            mag = 0.5 * O.abs_product(a[i], b[i]) + np.abs(c[i])
            assert_close(host(got[i]), want, mag, tol(precision), f"{shape} batched [{i}]")
    # exact inputs: every partial sum is exact, so the parts add up to the reference's bits
    qa = (rng.integers(-16, 17, (m, k)) / 4).astype(np.float32)
    qb = (rng.integers(-16, 17, (k, n)) / 4).astype(np.float32)
    np.testing.assert_array_equal(host(mf.matmul(dev(qa, cuda), dev(qb, cuda),
                                                 precision=precision)), O.gemm(qa, qb))
    no_fault()


# Short K with C_in (K <= 256 in 3xTF32, K <= 768 in 1xTF32; N > 128, C TMA-writable) takes the
# epilogue variant that copies C_in into the staging boxes a chunk ahead: ragged rows and
# columns (a partial 16-column chunk), a single k-block, a stream-K tail (124 tiles on 74
# units, 3xTF32), a batch; (m, n, k, batch).
CIN_AHEAD_SHAPES = [(1000, 1000, 100, 1), (520, 260, 16, 1), (1024, 7936, 256, 1),
                    (300, 516, 64, 3)]


@pytest.mark.parametrize("precision", PRECISIONS)
@pytest.mark.parametrize("shape", CIN_AHEAD_SHAPES, ids=lambda s: "x".join(map(str, s)))
def test_short_k_with_c_in(cuda, shape, precision):
    """The oracle's result within the path's bound; the same bits with C_in updated in place
    (C_in is C) and with C_in as a transposed view (read element by element); batched."""
    m, n, k, batch = shape
    rng = np.random.default_rng(m + 3 * n + 5 * k + batch)
    a = rng.standard_normal((batch, m, k)).astype(np.float32)
    b = rng.standard_normal((batch, k, n)).astype(np.float32)
    c = rng.standard_normal((batch, m, n)).astype(np.float32)
    bias = rng.uniform(-0.1, 0.1, n).astype(np.float32)
    ta, tb, tc, tbias = dev(a, cuda), dev(b, cuda), dev(c, cuda), dev(bias, cuda)
    got = mf.gemm(ta[0], tb[0], 0.5, tc[0], 1.0, bias=tbias, precision=precision)
    want = O.gemm(a[0], b[0], 0.5, c[0], 1.0, bias=bias)
    mag = 0.5 * O.abs_product(a[0], b[0]) + np.abs(c[0]) + np.abs(bias)[None, :]
    assert_close(host(got), want, mag, tol(precision), f"{shape} {precision}")
    in_place = tc[0].clone()
    mf.gemm(ta[0], tb[0], 0.5, in_place, 1.0, bias=tbias, precision=precision, out=in_place)
    assert torch.equal(in_place, got), "C_in updated in place differs"
    c_view = dev(np.ascontiguousarray(c[0].T), cuda).t()
    got_view = mf.gemm(ta[0], tb[0], 0.5, c_view, 1.0, bias=tbias, precision=precision)
    assert torch.equal(got_view, got), "C_in as a strided view differs"
    # C_in one row broadcast down the rows (row stride 0): every lane copies the same row
    c_row = tc[0][m // 2]
    got_bc = mf.gemm(ta[0], tb[0], 0.5, c_row.expand(m, n), 1.0, bias=tbias, precision=precision)
    got_full = mf.gemm(ta[0], tb[0], 0.5, c_row.expand(m, n).contiguous(), 1.0, bias=tbias,
                       precision=precision)
    assert torch.equal(got_bc, got_full), "C_in as a broadcast row differs"
    if batch > 1:
        out = mf.gemm_strided_batched(ta, tb, 0.5, tc, 1.0, precision=precision)
        for i in range(batch):
            want = O.gemm(a[i], b[i], 0.5, c[i], 1.0)
            mag = 0.5 * O.abs_product(a[i], b[i]) + np.abs(c[i])
            assert_close(host(out[i]), want, mag, tol(precision), f"{shape} batched [{i}]")
    no_fault()


# The shape tables of the reference's packed-GEMM test (tests/ops/gemm_packed_test.cpp): around
# every micro-tile edge (:175-179), odd extras (:181-182), the threaded and large cases (:186,
# :275), single rows (:380-381), narrow outputs (:400-403), and the strided-view shapes (:436-438).
PACKED_TEST_SHAPES = [
    (1, 1, 1), (1, 17, 3), (5, 15, 7), (6, 16, 1), (6, 16, 256), (7, 17, 257), (12, 32, 512),
    (13, 33, 255), (167, 31, 20), (168, 16, 20), (169, 17, 300), (337, 49, 513), (40, 4080, 9),
    (20, 4081, 17), (9, 8200, 5), (64, 64, 64), (100, 1, 100), (1, 100, 100),
    (11, 7, 5), (13, 9, 17), (3, 23, 7), (5, 25, 9), (24, 48, 300), (25, 49, 301), (50, 50, 1100),
    (200, 300, 100), (500, 70, 400), (37, 1000, 300), (1000, 37, 300),
    (300, 300, 300), (97, 257, 901), (600, 100, 80),
    (1, 1000, 37), (1, 37, 1000), (1, 2049, 515), (1, 5003, 301), (1, 7, 3), (1, 4096, 4),
    (64, 10, 512), (65, 10, 515), (33, 1, 100), (7, 2, 9), (40, 15, 70), (3, 12, 2000),
    (20, 5, 40000), (2000, 10, 300), (1001, 13, 77), (2, 3, 8), (2000, 64, 147), (3000, 40, 100),
    (1500, 64, 30), (900, 100, 200), (5000, 16, 33), (600, 2000, 100), (700, 900, 250),
    (32, 3000, 800), (64, 1500, 100),
]
STRIDED_TEST_SHAPES = [(1, 1, 1), (5, 15, 7), (13, 33, 255), (37, 50, 300), (169, 17, 300),
                       (64, 64, 64), (200, 100, 70), (9, 200, 5)]


@pytest.mark.parametrize("precision", PRECISIONS)
def test_reference_packed_kernel_shapes(cuda, precision):
    """Every shape of the reference's packed-GEMM test, on exact (quarter-integer) inputs: the
    device result equals the oracle's bit for bit in both precisions."""
    for i, (m, n, k) in enumerate(PACKED_TEST_SHAPES):
        rng = np.random.default_rng(1000 + i)
        a = (rng.integers(-16, 17, (m, k)) / 4).astype(np.float32)
        b = (rng.integers(-16, 17, (k, n)) / 4).astype(np.float32)
        got = host(mf.matmul(dev(a, cuda), dev(b, cuda), precision=precision))
        np.testing.assert_array_equal(got, O.gemm(a, b), err_msg=f"{m}x{n}x{k}")
    no_fault()


@pytest.mark.parametrize("precision", PRECISIONS)
def test_reference_strided_view_shapes(cuda, precision):
    """The strided shapes (gemm_packed_test.cpp:436-438) with A and B each stored plain or
    transposed and read as views (the kernels take the strides as they are)."""
    for i, (m, n, k) in enumerate(STRIDED_TEST_SHAPES):
        rng = np.random.default_rng(2000 + i)
        a = (rng.integers(-16, 17, (m, k)) / 4).astype(np.float32)
        b = (rng.integers(-16, 17, (k, n)) / 4).astype(np.float32)
        want = O.gemm(a, b)
        for ta in (False, True):
            for tb in (False, True):
                av = dev(np.ascontiguousarray(a.T), cuda).t() if ta else dev(a, cuda)
                bv = dev(np.ascontiguousarray(b.T), cuda).t() if tb else dev(b, cuda)
                got = host(mf.matmul(av, bv, precision=precision))
                np.testing.assert_array_equal(got, want, err_msg=f"{m}x{n}x{k} tA{ta} tB{tb}")
    no_fault()


def test_stream_k_gemms_on_concurrent_streams(cuda):
    """Stream-K GEMMs launched on two streams at once share the SMs, so not every CTA of one
    launch need be resident while the other runs; no part of a split tile waits for another, so
    every launch completes with the same bits and no bounded wait runs out."""
    rng = np.random.default_rng(77)
    a = dev(rng.standard_normal((1024, 1024)).astype(np.float32), cuda)
    b = dev(rng.standard_normal((1024, 1024)).astype(np.float32), cuda)
    want = mf.gemm(a, b)
    torch.cuda.synchronize()
    streams = [torch.cuda.Stream(), torch.cuda.Stream()]
    outs = []
    for i in range(24):
        with torch.cuda.stream(streams[i % 2]):
            outs.append(mf.gemm(a, b))
    torch.cuda.synchronize()
    assert all(torch.equal(o, want) for o in outs)
    no_fault()


def _inf_operands(m, n, k, seed):
    """Values exact in tf32 (lo = 0, so an infinity's partner lo gives inf * 0 in the split
    products) with infinities placed to give +-inf, and NaN where inf meets 0 or two infinite
    terms differ in sign."""
    rng = np.random.default_rng(seed)
    a = (rng.integers(-16, 17, (m, k)) / 4).astype(np.float32)
    b = (rng.integers(-16, 17, (k, n)) / 4).astype(np.float32)
    a[3, 5] = np.inf                      # row 3: +-inf, or NaN where b[5, j] == 0
    a[m // 2, 2] = -np.inf
    a[m // 2, 9] = np.inf                 # row m/2: -inf*b[2,j] + inf*b[9,j]
    b[7, n - 1] = np.inf                  # column n-1: inf * a[i, 7]
    return a, b


def _assert_nonfinite_match(got, want):
    special = ~np.isfinite(want)
    assert special.any()
    np.testing.assert_array_equal(np.isnan(got[special]), np.isnan(want[special]))
    inf_want = np.isinf(want)
    np.testing.assert_array_equal(got[inf_want], want[inf_want])
    np.testing.assert_array_equal(got[~special], want[~special])  # exact inputs elsewhere


# (m, n, k): A split in tensor memory (n <= 128), in shared memory, single-CTA tiles, stream-K
# tails (1024 x 300 x 2048, 100 x 1000 x 4096), several waves
INF_SHAPES = [(300, 64, 200), (300, 256, 200), (300, 640, 200), (100, 64, 70), (1024, 1024, 1024),
              (1024, 300, 2048), (100, 1000, 4096)]


@pytest.mark.parametrize("precision", PRECISIONS)
@pytest.mark.parametrize("shape", INF_SHAPES, ids=lambda s: "x".join(map(str, s)))
def test_infinite_operands(cuda, precision, shape):
    """Infinities in A and B give the reference's results on every kernel variant: +-inf where
    the infinite products agree in sign, NaN where inf meets 0 or opposite infinities meet. In
    3xTF32 an infinity's zero lo meets the other operand's hi and the tensor cores give NaN for
    inf * 0; the kernel recomputes such entries exactly, flagged by the converter warps (A) and
    the packing pass (B)."""
    m, n, k = shape
    a, b = _inf_operands(m, n, k, m * 5 + n + k)
    want = O.gemm(a, b)
    got = host(mf.matmul(dev(a, cuda), dev(b, cuda), precision=precision))
    _assert_nonfinite_match(got, want)
    no_fault()


@pytest.mark.parametrize("route", ["packed_a", "prepacked_b", "batched", "epilogue"])
def test_infinite_operands_routes(cuda, route):
    """The same in 3xTF32 where A is packed by the pre-pass (transposed A), where B comes
    pre-split (its flag is kept with the handle), in a batch (A broadcast, one infinity per
    matrix), and with alpha, beta * C and bias applied to the recomputed entries."""
    m, n, k = 300, 256, 200
    a, b = _inf_operands(m, n, k, 11)
    if route == "packed_a":
        at = dev(np.ascontiguousarray(a.T), cuda)
        got = host(mf.gemm(at, dev(b, cuda), transpose_a=True, precision="3xtf32"))
        want = O.gemm(a, b)
    elif route == "prepacked_b":
        clean = np.where(np.isfinite(a), a, 1.0).astype(np.float32)  # infinities only in B
        packed = mf.pack_b(dev(b, cuda), precision="3xtf32")
        got = host(mf.gemm_prepacked(dev(clean, cuda), packed, precision="3xtf32"))
        want = O.gemm(clean, b)
    elif route == "batched":
        bs = np.stack([b, np.where(np.isfinite(b), b, 0.0).astype(np.float32), b])
        bs[1, 11, 3] = -np.inf
        got = host(mf.gemm_strided_batched(dev(a, cuda), dev(bs, cuda), precision="3xtf32"))
        want = np.stack([O.gemm(a, bs[i]) for i in range(3)])
    else:
        rng = np.random.default_rng(3)
        c = (rng.integers(-8, 9, (m, n)) / 8).astype(np.float32)
        bias = (rng.integers(-8, 9, n) / 8).astype(np.float32)
        got = host(mf.gemm(dev(a, cuda), dev(b, cuda), 0.5, dev(c, cuda), 2.0,
                           bias=dev(bias, cuda), precision="3xtf32"))
        want = O.gemm(a, b, 0.5, c, 2.0, bias=bias)
    _assert_nonfinite_match(got, want)
    no_fault()
