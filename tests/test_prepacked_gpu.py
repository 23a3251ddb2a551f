"""B split once and reused (pack_b / gemm_prepacked), the device analogue of the reference's
PackedB: the shapes and cases of tests/ops/gemm_packed_test.cpp:60-84 and :335-377."""
import numpy as np
import pytest
import torch

import mensurflow_b200 as mf
from helpers import TOL_1X, TOL_3X, assert_close, make_input
from oracle import oracle as O

pytestmark = pytest.mark.gpu

PRECISIONS = ["3xtf32", "1xtf32"]

# (m, n, k): one row, few rows, many rows, widths that are not whole tiles
# (gemm_packed_test.cpp:340-342)
PACKED_SHAPES = [(1, 1, 1), (1, 37, 50), (1, 1000, 37), (1, 2049, 515), (3, 17, 9),
                 (16, 512, 100), (64, 100, 300), (97, 257, 901), (300, 300, 300), (600, 100, 80),
                 (7, 5000, 33)]


def dev(x, cuda):
    return torch.from_numpy(np.ascontiguousarray(x)).to(cuda)


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


@pytest.mark.parametrize("precision", PRECISIONS)
@pytest.mark.parametrize("shape", PACKED_SHAPES)
def test_reference_packed_shapes(cuda, precision, shape):
    """The reference's prepacked_kernel and prepacked_transposed_kernel: B packed as given and as
    its transpose (weights stored [outputs, inputs]) with the source freed before the product.
    The LCG inputs are multiples of 0.25 in [-4, 4], exact in tf32, so every product and sum is
    exact in fp32 and the result must equal the oracle bit for bit."""
    m, n, k = shape
    a = make_input(m * k, 1).reshape(m, k)
    b = make_input(k * n, 2).reshape(k, n)
    want = O.gemm(a, b)
    packed = mf.pack_b(dev(b, cuda), precision=precision)
    assert packed.depth() == k and packed.cols() == n and not packed.empty()
    np.testing.assert_array_equal(host(mf.gemm_prepacked(dev(a, cuda), packed)), want)

    bt = dev(np.ascontiguousarray(b.T), cuda)
    packed_t = mf.pack_b(bt, transpose=True, precision=precision)
    del bt
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    np.testing.assert_array_equal(host(mf.gemm_prepacked(dev(a, cuda), packed_t)), want)
    assert mf.device_status() == 0


def test_empty_depth_gives_zeros(cuda):
    """gemm_packed_test.cpp:368-377: an empty B (k == 0) gives zeros."""
    none = mf.pack_b(torch.empty(0, 4, device=cuda))
    assert none.empty() and none.depth() == 0 and none.cols() == 4
    c = mf.gemm_prepacked(torch.ones(2, 0, device=cuda), none)
    np.testing.assert_array_equal(host(c), np.zeros((2, 4), np.float32))
    # beta * c and the bias still apply
    c_in = torch.full((2, 4), 5.0, device=cuda)
    bias = torch.arange(4, dtype=torch.float32, device=cuda)
    got = mf.gemm_prepacked(torch.ones(2, 0, device=cuda), none, 1.0, c_in, 0.5, bias=bias)
    np.testing.assert_array_equal(host(got), np.full((2, 4), 2.5, np.float32) + np.arange(4))


# m <= 128 (one CTA) and m > 128 (a CTA pair); n <= 128 (A split in tensor memory), n <= 384
# (A split in shared memory), n > 384 (both operands pre-split)
@pytest.mark.parametrize("shape", [(100, 64, 300), (300, 96, 1000), (300, 256, 257),
                                   (520, 640, 130), (64, 512, 33)])
def test_bit_identical_to_gemm_3xtf32(cuda, shape):
    """In 3xTF32 the pack holds exactly the split the product would make of B itself, so the
    result equals gemm() with the same B bit for bit, epilogue included."""
    m, n, k = shape
    rng = np.random.default_rng(m * 31 + n + k)
    a = dev(rng.standard_normal((m, k)).astype(np.float32), cuda)
    w = dev(rng.standard_normal((n, k)).astype(np.float32), cuda)   # stored [outputs, inputs]
    c = dev(rng.standard_normal((m, n)).astype(np.float32), cuda)
    bias = dev(rng.uniform(-0.1, 0.1, n).astype(np.float32), cuda)
    packed = mf.pack_b(w, transpose=True, precision="3xtf32")
    want = mf.gemm(a, w, 0.5, c, 1.5, False, True, bias=bias, activation="gelu",
                   precision="3xtf32")
    got = mf.gemm_prepacked(a, packed, 0.5, c, 1.5, bias=bias, activation="gelu")
    np.testing.assert_array_equal(host(got), host(want))
    np.testing.assert_array_equal(
        host(mf.linear(a, packed, bias, "relu")),
        host(mf.linear(a, w, bias, "relu", transpose_w=True, precision="3xtf32")))


@pytest.mark.parametrize("precision", PRECISIONS)
def test_random_values_against_oracle(cuda, precision):
    m, n, k = 384, 200, 777
    rng = np.random.default_rng(7)
    a = rng.standard_normal((k, m)).astype(np.float32)     # used transposed
    b = rng.standard_normal((k, n)).astype(np.float32)
    packed = mf.pack_b(dev(b, cuda), precision=precision)
    got = host(mf.gemm_prepacked(dev(a, cuda), packed, -2.0, transpose_a=True))
    want = O.gemm(a, b, -2.0, None, 0.0, True, False)
    tol = TOL_3X if precision == "3xtf32" else TOL_1X
    assert_close(got, want, 2.0 * O.abs_product(a, b, True, False), tol, precision)


def test_precision_rules_and_errors(cuda):
    a = torch.randn(10, 20, device=cuda)
    p1 = mf.pack_b(torch.randn(20, 30, device=cuda), precision="1xtf32")
    assert p1.precision == "1xtf32"
    mf.gemm_prepacked(a, p1)                                 # its own precision
    with pytest.raises(ValueError):                          # MFK_ERR_INVALID_ARGUMENT
        mf.gemm_prepacked(a, p1, precision="3xtf32")         # no lo parts to use
    p3 = mf.pack_b(torch.randn(20, 30, device=cuda), precision="3xtf32")
    one = host(mf.gemm_prepacked(a, p3, precision="1xtf32"))  # a 3xTF32 pack serves both
    assert np.isfinite(one).all()
    with pytest.raises(ValueError):
        mf.gemm_prepacked(torch.randn(10, 21, device=cuda), p3)
    with pytest.raises(ValueError):
        mf.linear(a, p3, transpose_w=True)
    p3.free()
    assert p3.empty()
    with pytest.raises(ValueError):
        mf.gemm_prepacked(a, p3)
    assert mf.device_status() == 0
