"""The training-path adjoints on the device: bias_add's bias gradient (bit-identical to the
reference's host loop, src/ops/elementwise.cpp:263-283) and matmul's backward products through the
transposed-operand GEMM (src/ops/blas.cpp:220-230)."""
import numpy as np
import pytest
import torch

import mensurflow_b200 as mf
from helpers import TOL_1X, TOL_3X, assert_close, backward_inputs, golden
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def dev(x, cuda):
    return torch.from_numpy(np.ascontiguousarray(x)).to(cuda)


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


def test_golden_cases(cuda):
    """The reference's own backward results (tests/golden/backward_cases.npz): the bias gradient
    bit for bit, the matmul gradients within the 3xTF32 bound."""
    g = golden("backward_cases.npz")
    for name, arr in backward_inputs().items():
        if name.startswith("bias_grad"):
            np.testing.assert_array_equal(host(mf.bias_grad(dev(arr, cuda))), g[name],
                                          err_msg=name)
        else:
            a, b, grad = arr
            da, db = mf.matmul_backward(dev(grad, cuda), dev(a, cuda), dev(b, cuda))
            assert_close(host(da), g[name + "_da"], O.abs_product(grad, b, False, True), TOL_3X,
                         name + " dA")
            assert_close(host(db), g[name + "_db"], O.abs_product(a, grad, True, False), TOL_3X,
                         name + " dB")
    assert mf.device_status() == 0


@pytest.mark.parametrize("shape", [(1, 1), (3, 4099), (129, 33), (200000, 3), (4096, 1024),
                                   (128, 32), (257, 64)])
def test_bias_grad_bit_exact(cuda, shape):
    rows, cols = shape
    rng = np.random.default_rng(rows + 7 * cols)
    x = (rng.standard_normal((rows, cols)) * 10).astype(np.float32)
    np.testing.assert_array_equal(host(mf.bias_grad(dev(x, cuda))), O.bias_grad(x))


def test_bias_grad_views_and_edges(cuda):
    rng = np.random.default_rng(3)
    wide = dev(rng.standard_normal((300, 100)).astype(np.float32), cuda)
    view = wide[:, 10:77]                       # row stride 100, 67 features
    np.testing.assert_array_equal(host(mf.bias_grad(view)), O.bias_grad(host(view)))
    col_major = wide.t()                        # not row-major: packed first
    np.testing.assert_array_equal(host(mf.bias_grad(col_major)), O.bias_grad(host(col_major)))
    np.testing.assert_array_equal(host(mf.bias_grad(torch.empty(0, 5, device=cuda))),
                                  np.zeros(5, np.float32))
    assert mf.bias_grad(torch.empty(4, 0, device=cuda)).shape == (0,)
    specials = np.array([[1.0, np.inf, np.nan], [-1.0, 1.0, 0.0], [1e30, -np.inf, 1.0]],
                        np.float32)
    np.testing.assert_array_equal(host(mf.bias_grad(dev(specials, cuda))), O.bias_grad(specials))


@pytest.mark.parametrize("precision", ["3xtf32", "1xtf32"])
@pytest.mark.parametrize("shape", [(300, 200, 130), (64, 1000, 48), (1, 7, 5), (513, 129, 257)])
def test_matmul_backward(cuda, precision, shape):
    m, k, n = shape
    rng = np.random.default_rng(m * 3 + k + n)
    a = rng.standard_normal((m, k)).astype(np.float32)
    b = rng.standard_normal((k, n)).astype(np.float32)
    grad = rng.standard_normal((m, n)).astype(np.float32)
    want_da, want_db = O.matmul_backward(a, b, grad)
    da, db = mf.matmul_backward(dev(grad, cuda), dev(a, cuda), dev(b, cuda), precision=precision)
    tol = TOL_3X if precision == "3xtf32" else TOL_1X
    assert_close(host(da), want_da, O.abs_product(grad, b, False, True), tol, f"{shape} dA")
    assert_close(host(db), want_db, O.abs_product(a, grad, True, False), tol, f"{shape} dB")
    only_a, none_b = mf.matmul_backward(dev(grad, cuda), dev(a, cuda), dev(b, cuda),
                                        need_b=False, precision=precision)
    assert none_b is None
    np.testing.assert_array_equal(host(only_a), host(da))


@pytest.mark.parametrize("transpose_w", [False, True])
def test_linear_backward(cuda, transpose_w):
    """y = x @ op(w) + bias: the three adjoints, dw in w's own layout."""
    m, k, n = 257, 96, 160
    rng = np.random.default_rng(21)
    x = rng.standard_normal((m, k)).astype(np.float32)
    w = rng.standard_normal((n, k) if transpose_w else (k, n)).astype(np.float32)
    grad = rng.standard_normal((m, n)).astype(np.float32)
    dx, dw, db = mf.linear_backward(dev(grad, cuda), dev(x, cuda), dev(w, cuda),
                                    transpose_w=transpose_w)
    w_op = w.T if transpose_w else w
    want_dx, want_dw = O.matmul_backward(x, np.ascontiguousarray(w_op), grad)
    if transpose_w:
        want_dw = np.ascontiguousarray(want_dw.T)
    assert_close(host(dx), want_dx, O.abs_product(grad, np.ascontiguousarray(w_op), False, True),
                 TOL_3X, "dx")
    mag_w = O.abs_product(x, grad, True, False)
    assert_close(host(dw), want_dw, mag_w.T if transpose_w else mag_w, TOL_3X, "dw")
    np.testing.assert_array_equal(host(db), O.bias_grad(grad))
    assert mf.device_status() == 0
