"""The no-allocation GEMM entry point (mfk_gemm_f32_noalloc), called through the C ABI.

It exists for callers that cannot allocate device memory while they run (a host that reserves
its whole memory plan up front, or a framework whose caching allocator owns the device); it
keeps the tf32 operand copies in a fixed scratch array inside the library instead. Its results
must meet the path's bound against both the allocating entry point (mfk_gemm_f32) and the oracle
on the same inputs, call after call — the scratch array keeps the previous call's contents, so two
calls in a row with different inputs check that nothing stale leaks into a result.

The file is named to be collected last: a failure here leaves every other test already run.
"""
import ctypes

import numpy as np
import pytest
import torch

from helpers import TOL_1X, TOL_3X, assert_close
from mensurflow_b200 import _lib
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _desc(a, b, c_in, out, alpha, beta, bias, precision, transpose_b):
    d = _lib.GemmDesc()
    right = b.t() if transpose_b else b
    d.a, d.a_rs, d.a_cs = a.data_ptr(), a.stride(0), a.stride(1)
    d.b, d.b_rs, d.b_cs = right.data_ptr(), right.stride(0), right.stride(1)
    if c_in is not None:
        d.c_in, d.c_in_rs, d.c_in_cs = c_in.data_ptr(), c_in.stride(0), c_in.stride(1)
    d.c, d.ldc = out.data_ptr(), out.stride(0)
    d.m, d.n, d.k = out.shape[0], out.shape[1], a.shape[1]
    d.alpha, d.beta = alpha, beta
    d.bias = None if bias is None else bias.data_ptr()
    d.activation = _lib.ACT_NONE
    d.precision = precision
    return d


def _call(fn, desc):
    stream = torch.cuda.current_stream().cuda_stream
    rc = fn(ctypes.byref(desc), stream)
    assert rc == _lib.MFK_OK, _lib.lib().mfk_status_string(rc).decode()


# (m, n, k, transpose_a, transpose_b): A read in place with B packed (both layouts of B); A
# transposed, so it is not K-major and is packed into the scratch array as well (two packed
# operands plus the infinity flag word after them); and a shape whose last wave
# mfk_gemm_f32 shares out by k-iterations (stream-K) while this entry point keeps whole tiles,
# so the two entry points may differ in the last bits but both must meet the bound.
CASES = [(700, 520, 1000, False, True), (700, 520, 1000, False, False),
         (640, 384, 900, True, False), (1024, 300, 2048, False, False)]


@pytest.mark.parametrize("precision,tol", [(_lib.PRECISION_3XTF32, TOL_3X),
                                           (_lib.PRECISION_1XTF32, TOL_1X)])
@pytest.mark.parametrize("m,n,k,transpose_a,transpose_b", CASES)
def test_noalloc_matches_allocating_entry_point(cuda, precision, tol, m, n, k, transpose_a,
                                                transpose_b):
    so = _lib.lib()
    for call in range(2):  # two calls in a row, different inputs each time
        rng = np.random.default_rng(100 + call)
        a = rng.standard_normal((k, m) if transpose_a else (m, k)).astype(np.float32)
        b = rng.standard_normal((n, k) if transpose_b else (k, n)).astype(np.float32)
        c = rng.standard_normal((m, n)).astype(np.float32)
        bias = rng.uniform(-0.1, 0.1, n).astype(np.float32)
        ta, tb, tc, tbias = (torch.from_numpy(x).to(cuda) for x in (a, b, c, bias))
        left = ta.t() if transpose_a else ta
        want = torch.full((m, n), float("nan"), device=cuda)
        got = torch.full((m, n), float("nan"), device=cuda)
        _call(so.mfk_gemm_f32,
              _desc(left, tb, tc, want, 0.5, 1.0, tbias, precision, transpose_b))
        _call(so.mfk_gemm_f32_noalloc,
              _desc(left, tb, tc, got, 0.5, 1.0, tbias, precision, transpose_b))
        torch.cuda.synchronize()
        got_h = got.cpu().numpy()
        mag = (0.5 * O.abs_product(a, b, transpose_a, transpose_b) + np.abs(c) +
               np.abs(bias)[None, :])
        # against the allocating entry point ...
        assert_close(got_h, want.cpu().numpy(), mag, tol, f"no-alloc call {call + 1}")
        # ... and against the oracle (the reference's algorithm on the CPU)
        oracle = O.gemm(a, b, 0.5, c, 1.0, transpose_a, transpose_b, bias=bias)
        assert_close(got_h, oracle, mag, tol, f"no-alloc call {call + 1} vs the oracle")
    assert _lib.device_status() == 0


def test_noalloc_rejects_problems_beyond_its_scratch(cuda):
    so = _lib.lib()
    # 3xTF32 packs B (hi and lo): 8 bytes x n x k rounded up to 32 > 64 MiB here (A is
    # K-major and aligned, so the kernel splits it in place and it needs no copy).
    m = n = 4096
    k = 2080
    assert 8 * n * k > _lib.NOALLOC_SCRATCH_BYTES
    a = torch.zeros(m, k, device=cuda)
    b = torch.zeros(k, n, device=cuda)
    out = torch.zeros(m, n, device=cuda)
    rc = so.mfk_gemm_f32_noalloc(
        ctypes.byref(_desc(a, b, None, out, 1.0, 0.0, None, _lib.PRECISION_3XTF32, False)),
        torch.cuda.current_stream().cuda_stream)
    assert rc == _lib.MFK_ERR_SCRATCH_LIMIT
    assert b"scratch" in so.mfk_status_string(rc)
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
