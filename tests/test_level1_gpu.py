"""The level-1 kernels the CUDA backend registers beside the GEMM path (add / sub / mul / div,
scal, dot), through the Python mirror of the reference's ops. The elementwise ops and scal are one
IEEE fp32 operation per element, so they must equal the CPU's result bit for bit; dot sums the
products in double and rounds once, as cpu::dot_f32 (src/backends/cpu/ops/blas/blas.cpp:14-21),
so it is within one rounding of the exact double sum."""
import numpy as np
import pytest
import torch

import mensurflow_b200 as mf
from helpers import make_input, ulp_diff

pytestmark = pytest.mark.gpu


def _dev(x, cuda):
    return torch.from_numpy(np.ascontiguousarray(x)).to(cuda)


@pytest.mark.parametrize("shape_a,shape_b", [((1000,), (1000,)), ((33, 70), (70,)),
                                             ((4, 1, 6), (5, 1)), ((0, 3), (3,)),
                                             ((1027,), (1,))])
def test_elementwise_bit_exact(cuda, shape_a, shape_b):
    a = make_input(int(np.prod(shape_a)), 3).reshape(shape_a)
    b = make_input(int(np.prod(shape_b)), 4).reshape(shape_b)
    with np.errstate(divide="ignore", invalid="ignore"):
        want = {"add": a + b, "sub": a - b, "mul": a * b, "div": a / b}
    for name, fn in (("add", mf.add), ("sub", mf.sub), ("mul", mf.mul), ("div", mf.div)):
        got = fn(_dev(a, cuda), _dev(b, cuda)).cpu().numpy()
        assert got.shape == want[name].shape
        np.testing.assert_array_equal(got, want[name].astype(np.float32), err_msg=name)
    assert mf.device_status() == 0


def test_elementwise_unaligned_views_and_errors(cuda):
    base = torch.randn(4097, device=cuda)
    x, y = base[1:], base[:-1]  # not 16-byte aligned: the scalar kernel
    np.testing.assert_array_equal(mf.mul(x, y).cpu().numpy(),
                                  (x.cpu().numpy() * y.cpu().numpy()))
    with pytest.raises(ValueError):
        mf.add(torch.zeros(3, device=cuda), torch.zeros(4, device=cuda))
    with pytest.raises(NotImplementedError):
        mf.add(torch.zeros(3), torch.zeros(3))


def test_scal_bit_exact(cuda):
    x = np.random.default_rng(5).standard_normal(10001).astype(np.float32)
    got = mf.scal(-0.3, _dev(x, cuda)).cpu().numpy()
    np.testing.assert_array_equal(got, np.float32(-0.3) * x)
    np.testing.assert_array_equal(mf.scal(2.0, _dev(x, cuda)[::3]).cpu().numpy(), 2 * x[::3])


@pytest.mark.parametrize("n", [0, 1, 15, 17, 1000, 32769, 100003, (1 << 20) + 7, 1 << 24])
def test_dot_double_accumulation(cuda, n):
    rng = np.random.default_rng(n)
    x = rng.uniform(-2, 2, n).astype(np.float32)
    y = rng.uniform(-2, 2, n).astype(np.float32)
    got = mf.dot(_dev(x, cuda), _dev(y, cuda))
    assert got.dim() == 0 and got.device == cuda
    want = np.float32(np.dot(x.astype(np.float64), y.astype(np.float64)))
    assert ulp_diff(np.array([got.item()], np.float32), np.array([want]))[0] <= 1
    # repeated calls give the same bits
    assert mf.dot(_dev(x, cuda), _dev(y, cuda)).item() == got.item()
    assert mf.device_status() == 0
