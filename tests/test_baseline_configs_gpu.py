"""Parity at every BASELINE.json config, on the configs' own inputs, against the live reference.

Inputs come from the reference's own counter-based Philox generators (the unmodified library built
from its sources, `oracle/_ref`; include/mensurflow/ops/random.hpp:20-26 `uniform` / `normal`),
one seed per config and one stream per config through `offset`, in the listed order (A at offset
0, B at numel(A), C_in after B, ...). The expected values come from the same library's public API
on the CPU (`gemm`, `matmul`, `bias_add`, `gelu`, `gemm_strided_batched`, `attention`, `gemv`;
src/ops/blas.cpp:186-394, src/ops/attention.cpp:48-98), not from the restatement, and the
magnitudes of the bound from the reference's own `matmul(abs(A), abs(B))`, as its test helper
`reference::matmul_tolerance` builds them (tests/reference/blas.hpp:38-59).

Bounds (north_star): 3xTF32 |C - C_ref| <= 1e-5 (|A||B|)_ij + 1e-6; 1xTF32 2e-3 relative to the
same magnitude. Large configs compare a seeded sample of rows (the GPU computes the whole
product); C1 compares every entry.
"""
import numpy as np
import pytest
import torch

import mensurflow_b200 as mf
from helpers import TOL_1X, TOL_3X, assert_close, ulp_diff
from mensurflow_b200 import _lib
from oracle import oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ref():
    lib = O.reference()
    if lib is None:
        pytest.skip("the reference build (oracle/_ref/libmfref.so) is not present")
    return lib


def _rows(m, count, seed):
    return np.sort(np.random.default_rng(seed).choice(m, size=count, replace=False))


def _dev(x, cuda):
    return torch.from_numpy(np.ascontiguousarray(x)).to(cuda)


def test_c1_whole_output(cuda, ref):
    """C1: gemm, 1024^3, alpha 1, beta 0, A and B uniform[-1, 1) from seed 0; every entry."""
    n = 1024
    a = O.ref_uniform(n * n, -1.0, 1.0, 0, 0).reshape(n, n)
    b = O.ref_uniform(n * n, -1.0, 1.0, 0, n * n).reshape(n, n)
    c = np.zeros((n, n), np.float32)
    want = O.ref_gemm(a, b, 1.0, c, 0.0)
    mag = O.ref_gemm(np.abs(a), np.abs(b))
    for precision, tol in (("3xtf32", TOL_3X), ("1xtf32", TOL_1X)):
        got = mf.gemm(_dev(a, cuda), _dev(b, cuda), 1.0, _dev(c, cuda), 0.0,
                      precision=precision).cpu().numpy()
        assert_close(got, want, mag, tol, f"C1 {precision}")
    assert mf.device_status() == 0


@pytest.fixture(scope="module")
def c2_inputs(ref):
    n = 8192
    nn = n * n
    a = O.ref_normal(nn, 0.0, 1.0, 1, 0).reshape(n, n)
    b = O.ref_normal(nn, 0.0, 1.0, 1, nn).reshape(n, n)
    c = O.ref_normal(nn, 0.0, 1.0, 1, 2 * nn).reshape(n, n)
    bias = O.ref_uniform(n, -0.1, 0.1, 1, 3 * nn)
    return a, b, c, bias


@pytest.mark.parametrize("precision,tol", [("3xtf32", TOL_3X), ("1xtf32", TOL_1X)])
def test_c2_sampled_rows(cuda, c2_inputs, precision, tol):
    """C2: 0.5 * A @ B^T + 1.0 * C_in + bias at 8192^3 on the reference's Philox normals (seed 1),
    the bias fused in the epilogue; 48 sampled rows against the reference's gemm + bias_add."""
    a, b, c, bias = c2_inputs
    ta, tb, tc, tbias = (_dev(x, cuda) for x in (a, b, c, bias))
    out = mf.gemm(ta, tb, 0.5, tc, 1.0, False, True, bias=tbias, precision=precision)
    rows = _rows(a.shape[0], 48, 21)
    got = out[torch.from_numpy(rows).to(cuda)].cpu().numpy()
    del out, ta, tb, tc
    want = O.ref_bias_add(O.ref_gemm(a[rows], b, 0.5, c[rows], 1.0, False, True), bias)
    mag = (0.5 * O.ref_gemm(np.abs(a[rows]), np.abs(b), 1.0, None, 0.0, False, True) +
           np.abs(c[rows]) + np.abs(bias)[None, :])
    assert_close(got, want, mag, tol, f"C2 {precision}")
    assert mf.device_status() == 0


def test_c3_whole_chain_sampled_rows(cuda, ref):
    """C3: Y = gelu(X W1 + b1) W2 + b2, X [4096, 1024] normal(0, 1), W1 [1024, 4096] and
    W2 [4096, 1024] Xavier-uniform (+-0.034233), zero biases, all from seed 2. The chain runs as two
    fused GEMM calls; the reference runs matmul, bias_add, gelu, matmul, bias_add. The bound of Y
    carries the first layer's bound through |W2| (GELU's slope is below 1.13)."""
    rows_n, d_in, d_hid = 4096, 1024, 4096
    lim = 0.034233
    x = O.ref_normal(rows_n * d_in, 0.0, 1.0, 2, 0).reshape(rows_n, d_in)
    off = rows_n * d_in
    w1 = O.ref_uniform(d_in * d_hid, -lim, lim, 2, off).reshape(d_in, d_hid)
    off += d_in * d_hid
    w2 = O.ref_uniform(d_hid * d_in, -lim, lim, 2, off).reshape(d_hid, d_in)
    b1 = np.zeros(d_hid, np.float32)
    b2 = np.zeros(d_in, np.float32)
    y = mf.linear(mf.linear(_dev(x, cuda), _dev(w1, cuda), _dev(b1, cuda), "gelu"),
                  _dev(w2, cuda), _dev(b2, cuda))
    rows = _rows(rows_n, 64, 22)
    got = y[torch.from_numpy(rows).to(cuda)].cpu().numpy()
    h = O.ref_gelu(O.ref_bias_add(O.ref_matmul(x[rows], w1), b1))
    want = O.ref_bias_add(O.ref_matmul(h, w2), b2)
    h_bound = 1.13 * (TOL_3X[0] * O.ref_matmul(np.abs(x[rows]), np.abs(w1)) + TOL_3X[1])
    mag = (O.ref_matmul(np.abs(h), np.abs(w2)) +
           O.ref_matmul(h_bound.astype(np.float32), np.abs(w2)) / TOL_3X[0])
    assert_close(got, want, mag, TOL_3X, "C3 chain")
    assert mf.device_status() == 0


def test_c4_attention_gemms_and_chain(cuda, ref):
    """C4: Q, K, V [512, 2048, 128] normal(0, 1/sqrt 128) from seed 3. GEMM 1 (S = Q K^T / sqrt
    128) and GEMM 2 (O = P V) run over all 512 heads; three heads are checked against the
    reference: sampled rows of S and of O = P V (P as the device computed it, so the GEMM is
    checked alone) within the 3xTF32 bound, and the whole causal attention of each head against the
    reference's attention within its own test tolerance (softmax_loss_test.cpp: 1e-4, 1e-6)."""
    bh, s, d = 512, 2048, 128
    per = bh * s * d
    std = float(np.float32(1.0 / np.sqrt(d)))
    q = O.ref_normal(per, 0.0, std, 3, 0).reshape(bh, s, d)
    k = O.ref_normal(per, 0.0, std, 3, per).reshape(bh, s, d)
    v = O.ref_normal(per, 0.0, std, 3, 2 * per).reshape(bh, s, d)
    scale = float(np.float32(1.0 / np.sqrt(d)))
    tq, tk, tv = (_dev(x, cuda) for x in (q, k, v))
    scores = mf.gemm_strided_batched(tq, tk, scale, None, 0.0, False, True)
    heads = (0, 301, 511)
    rows = _rows(s, 16, 23)
    idx = torch.from_numpy(rows).to(cuda)
    for h in heads:
        got = scores[h][idx].cpu().numpy()
        want = O.ref_gemm(q[h][rows], k[h], scale, None, 0.0, False, True)
        mag = scale * O.ref_gemm(np.abs(q[h][rows]), np.abs(k[h]), 1.0, None, 0.0, False, True)
        assert_close(got, want, mag, TOL_3X, f"C4 S head {h}")
    # the causal softmax in place (the path's masked softmax kernel), then GEMM 2
    so = _lib.lib()
    stream = torch.cuda.current_stream().cuda_stream
    assert so.mfk_masked_softmax_f32(scores.data_ptr(), None, 0, 0, 1, scores.data_ptr(), bh, s,
                                     s, stream) == _lib.MFK_OK
    o = mf.gemm_strided_batched(scores, tv)
    for h in heads:
        p = scores[h][idx].cpu().numpy()
        got = o[h][idx].cpu().numpy()
        want = O.ref_gemm(p, v[h])
        mag = O.ref_gemm(np.abs(p), np.abs(v[h]))
        assert_close(got, want, mag, TOL_3X, f"C4 O = P V head {h}")
    del scores, o
    # the attention op end to end, causal, against the reference's attention per head
    out = mf.attention(tq, tk, tv, causal=True, scale=scale)
    for h in heads:
        want = O.ref_attention(q[h:h + 1], k[h:h + 1], v[h:h + 1], causal=True, scale=scale)
        np.testing.assert_allclose(out[h:h + 1].cpu().numpy(), want, rtol=1e-4, atol=1e-6,
                                   err_msg=f"C4 attention head {h}")
    assert mf.device_status() == 0


def test_c5_sampled_rows_and_gemv(cuda, ref):
    """C5: A [32768, 8192] @ B [8192, 32768], uniform[-1, 1) from seed 4 (C alone is 4 GiB), 16
    sampled rows against the reference's matmul; and the companion gemv, A [65536, 8192] and x
    [8192] uniform[-1, 1) from seed 4 (A at offset 0, x after it), every entry against the
    reference's gemv (double accumulation on both sides: within 1 ulp)."""
    m, k, n = 32768, 8192, 32768
    a = O.ref_uniform(m * k, -1.0, 1.0, 4, 0).reshape(m, k)
    b = O.ref_uniform(k * n, -1.0, 1.0, 4, m * k).reshape(k, n)
    ta, tb = _dev(a, cuda), _dev(b, cuda)
    out = mf.matmul(ta, tb)
    rows = _rows(m, 16, 24)
    got = out[torch.from_numpy(rows).to(cuda)].cpu().numpy()
    del out, ta, tb
    want = O.ref_matmul(a[rows], b)
    mag = O.ref_matmul(np.abs(a[rows]), np.abs(b))
    assert_close(got, want, mag, TOL_3X, "C5")
    del a, b

    gm, gk = 65536, 8192
    ga = O.ref_uniform(gm * gk, -1.0, 1.0, 4, 0).reshape(gm, gk)
    gx = O.ref_uniform(gk, -1.0, 1.0, 4, gm * gk)
    y = mf.matvec(_dev(ga, cuda), _dev(gx, cuda)).cpu().numpy()
    want = O.ref_gemv(ga, gx)
    diff = ulp_diff(y, want)
    assert diff.max() <= 1, f"C5 gemv: {int(diff.max())} ulp"
    assert mf.device_status() == 0
