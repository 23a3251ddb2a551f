"""Failure detection on the device without faulting the GPU.

Every wait in the kernels (pipeline mbarriers, the stream-K finisher's count) is bounded by
%globaltimer: a wait that runs out records a bit in the device error word and the kernel returns,
so a bug shows up as an error status on the host instead of a hung GPU. This test makes such a
wait run out on purpose — a barrier that nothing completes, with a 50 ms limit — and checks the
status the host reads, that reading it clears it, and that the context still runs GEMMs
correctly afterwards.
"""
import ctypes

import numpy as np
import pytest
import torch

import mensurflow_b200 as mf
from mensurflow_b200 import _lib
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def test_bounded_wait_gives_up_and_the_context_stays_usable(cuda):
    so = _lib.lib()
    assert mf.device_status() == 0
    gave_up = ctypes.c_uint32(7)
    try:
        rc = so.mfk_selftest_wait_timeout(50_000_000, ctypes.byref(gave_up),
                                          torch.cuda.current_stream().cuda_stream)
        assert rc == _lib.MFK_OK
        assert gave_up.value == 1
        bits = ctypes.c_uint32(0)
        assert so.mfk_device_status(ctypes.byref(bits), 0) == _lib.MFK_ERR_DEVICE_FAULT
        assert bits.value == 0x10  # MFK_DEVERR_SELFTEST_TIMEOUT, nothing else
        assert mf.device_status() == 0x10  # read and cleared
    finally:
        mf.device_status()  # later kernels must not see the bit, whatever happened above
    assert mf.device_status() == 0  # cleared
    # the context is intact: a GEMM right after gives the oracle's result
    rng = np.random.default_rng(1)
    a = rng.standard_normal((300, 200)).astype(np.float32)
    b = rng.standard_normal((200, 260)).astype(np.float32)
    got = mf.matmul(torch.from_numpy(a).to(cuda), torch.from_numpy(b).to(cuda)).cpu().numpy()
    err = np.abs(got.astype(np.float64) - O.gemm(a, b))
    assert (err <= 1e-5 * O.abs_product(a, b) + 1e-6).all()
    assert mf.device_status() == 0


def test_selftest_rejects_limits_beyond_the_pipeline_bound(cuda):
    so = _lib.lib()
    gave_up = ctypes.c_uint32(0)
    assert so.mfk_selftest_wait_timeout(0, ctypes.byref(gave_up), None) == \
        _lib.MFK_ERR_INVALID_ARGUMENT
    assert so.mfk_selftest_wait_timeout(3_000_000_000, ctypes.byref(gave_up), None) == \
        _lib.MFK_ERR_INVALID_ARGUMENT
