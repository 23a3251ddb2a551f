"""Parity at BASELINE.json's full sizes. The GPU computes the whole product; the oracle recomputes
a seeded sample of rows (every row for the gemv) and each sampled element must meet the path's
bound against (|A||B|)_ij. Inputs follow the configs' distributions (seeded torch generators)."""
import numpy as np
import pytest
import torch

import mensurflow_b200 as mf
from helpers import TOL_1X, TOL_3X, assert_close, ulp_diff
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _rows(m, count, seed):
    return np.sort(np.random.default_rng(seed).choice(m, size=count, replace=False))


@pytest.mark.parametrize("precision,tol", [("3xtf32", TOL_3X), ("1xtf32", TOL_1X)])
def test_c2_full_size(cuda, precision, tol):
    """C2: 0.5 * A @ B^T + 1.0 * C_in + bias at 8192^3, N(0,1) inputs, uniform(-0.1, 0.1) bias."""
    n = 8192
    g = torch.Generator(device=cuda).manual_seed(1)
    a = torch.randn(n, n, device=cuda, generator=g)
    b = torch.randn(n, n, device=cuda, generator=g)
    c = torch.randn(n, n, device=cuda, generator=g)
    bias = torch.rand(n, device=cuda, generator=g) * 0.2 - 0.1
    out = mf.gemm(a, b, 0.5, c, 1.0, False, True, bias=bias, precision=precision)
    rows = _rows(n, 48, 2)
    idx = torch.from_numpy(rows).to(cuda)
    a_s = a[idx].cpu().numpy()
    b_h = b.cpu().numpy()
    c_s = c[idx].cpu().numpy()
    bias_h = bias.cpu().numpy()
    want = O.gemm(a_s, b_h, 0.5, c_s, 1.0, False, True, bias=bias_h)
    mag = 0.5 * O.abs_product(a_s, b_h, False, True) + np.abs(c_s) + np.abs(bias_h)[None, :]
    assert_close(out[idx].cpu().numpy(), want, mag, tol, f"C2 full size {precision}")
    assert mf.device_status() == 0


def test_c5_full_size(cuda):
    """C5: A [32768, 8192] @ B [8192, 32768], uniform[-1, 1), 3xTF32 (C alone is 4 GiB)."""
    m, k, n = 32768, 8192, 32768
    g = torch.Generator(device=cuda).manual_seed(4)
    a = torch.rand(m, k, device=cuda, generator=g) * 2 - 1
    b = torch.rand(k, n, device=cuda, generator=g) * 2 - 1
    out = mf.matmul(a, b)
    rows = _rows(m, 16, 5)
    idx = torch.from_numpy(rows).to(cuda)
    a_s = a[idx].cpu().numpy()
    b_h = b.cpu().numpy()
    del a
    want = O.gemm(a_s, b_h)
    assert_close(out[idx].cpu().numpy(), want, O.abs_product(a_s, b_h), TOL_3X, "C5 full size")
    assert mf.device_status() == 0


def test_c3_full_size_mlp(cuda):
    """C3: y = gelu(X W1 + b1) W2 + b2 at batch 4096, X ~ N(0, 1), Xavier-uniform W1 [1024, 4096]
    and W2 [4096, 1024], zero biases (the bench path: X and H split inside the GEMMs, the first
    GEMM's tail wave shared by stream-K). Sampled rows of the whole chain against the oracle; the
    bound for y adds the first GEMM's bound, carried through |W2| (GELU's slope is below 1.13)."""
    rows_n, d_in, d_hid = 4096, 1024, 4096
    g = torch.Generator(device=cuda).manual_seed(2)
    lim = (6.0 / (d_in + d_hid)) ** 0.5
    x = torch.randn(rows_n, d_in, device=cuda, generator=g)
    w1 = (torch.rand(d_in, d_hid, device=cuda, generator=g) * 2 - 1) * lim
    w2 = (torch.rand(d_hid, d_in, device=cuda, generator=g) * 2 - 1) * lim
    b1 = torch.zeros(d_hid, device=cuda)
    b2 = torch.zeros(d_in, device=cuda)
    y = mf.linear(mf.linear(x, w1, b1, "gelu"), w2, b2)
    rows = _rows(rows_n, 64, 6)
    idx = torch.from_numpy(rows).to(cuda)
    x_s = x[idx].cpu().numpy()
    w1_h, w2_h = w1.cpu().numpy(), w2.cpu().numpy()
    zeros_hid, zeros_in = np.zeros(d_hid, np.float32), np.zeros(d_in, np.float32)
    h_s = O.activation(O.gemm(x_s, w1_h, bias=zeros_hid), "gelu").astype(np.float32)
    want = O.gemm(h_s, w2_h, bias=zeros_in)
    h_bound = 1.13 * (TOL_3X[0] * O.abs_product(x_s, w1_h) + TOL_3X[1])
    mag = O.abs_product(np.abs(h_s), w2_h) + O.abs_product(h_bound, w2_h) / TOL_3X[0]
    assert_close(y[idx].cpu().numpy(), want, mag, TOL_3X, "C3 full size")
    assert mf.device_status() == 0


def test_c4_full_size_attention_gemms(cuda):
    """C4: S = Q K^T / sqrt(128) and O = P V with batch*heads 512, seq 2048, head_dim 128."""
    bh, s, d = 512, 2048, 128
    g = torch.Generator(device=cuda).manual_seed(3)
    std = 1.0 / np.sqrt(d)
    q = torch.randn(bh, s, d, device=cuda, generator=g) * std
    k = torch.randn(bh, s, d, device=cuda, generator=g) * std
    v = torch.randn(bh, s, d, device=cuda, generator=g) * std
    scale = float(np.float32(1.0 / np.sqrt(d)))
    scores = mf.gemm_strided_batched(q, k, scale, None, 0.0, False, True)
    p = torch.softmax(scores, -1)  # the stand-in for the path's softmax (not under test here)
    o = mf.gemm_strided_batched(p, v)
    for bi in (0, 137, 511):
        rows = _rows(s, 12, bi)
        idx = torch.from_numpy(rows).to(cuda)
        q_s = q[bi][idx].cpu().numpy()
        k_h = k[bi].cpu().numpy()
        want_s = O.gemm(q_s, k_h, scale, None, 0.0, False, True)
        assert_close(scores[bi][idx].cpu().numpy(), want_s,
                     scale * O.abs_product(q_s, k_h, False, True), TOL_3X, f"scores batch {bi}")
        p_s = p[bi][idx].cpu().numpy()
        v_h = v[bi].cpu().numpy()
        assert_close(o[bi][idx].cpu().numpy(), O.gemm(p_s, v_h), O.abs_product(p_s, v_h), TOL_3X,
                     f"output batch {bi}")
    assert mf.device_status() == 0


def test_gemv_full_size(cuda):
    """The companion gemv at 65536 x 8192: every entry, double accumulation on both sides."""
    m, k = 65536, 8192
    g = torch.Generator(device=cuda).manual_seed(4)
    a = torch.rand(m, k, device=cuda, generator=g) * 2 - 1
    x = torch.rand(k, device=cuda, generator=g) * 2 - 1
    y = mf.matvec(a, x).cpu().numpy()
    want = O.gemv(a.cpu().numpy(), x.cpu().numpy())
    d = ulp_diff(y, want)
    assert d.max() <= 1, f"gemv: {int(d.max())} ulp"
    assert (d == 0).mean() > 0.99
    assert mf.device_status() == 0
