"""CPU tests of the boundary and the host logic: the C-ABI library loads and exports every symbol
include/mfk.h declares, the ctypes descriptors match the C layout, and the reference-API mirror
validates arguments and walks batch offsets like the reference (no GPU compute here)."""
import ctypes
import os
import re

import numpy as np
import pytest
import torch

import mensurflow_b200 as mf
from mensurflow_b200 import _lib, ops

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_functions():
    text = open(os.path.join(ROOT, "include", "mfk.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(mfk_\w+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    so = _lib.lib()
    declared = header_functions()
    assert declared, "no functions found in include/mfk.h"
    for name in declared:
        assert hasattr(so, name), f"{name} declared in include/mfk.h but not exported"
    assert sorted(_lib.EXPORTED) == declared


def test_version_and_status_strings():
    so = _lib.lib()
    assert so.mfk_version() >> 16 == 1
    assert so.mfk_status_string(0) == b"ok"
    assert so.mfk_status_string(1) == b"invalid argument"
    assert so.mfk_status_string(99) == b"unknown status"


def test_descriptor_layout_matches_c():
    # mfk_gemm_desc: 3 ptr+2 i64 groups (a, b, c_in), c + ldc, m n k, alpha beta, bias, 2 x i32
    assert ctypes.sizeof(_lib.GemmDesc) == 8 * 3 * 3 + 16 + 24 + 8 + 8 + 8
    assert _lib.GemmDesc.alpha.offset == 8 * 9 + 16 + 24
    assert ctypes.sizeof(_lib.BatchDesc) == 7 * 8


def test_invalid_descriptors_rejected_before_launch():
    """Argument errors come back as status codes without touching a device."""
    so = _lib.lib()
    d = _lib.GemmDesc()
    d.m, d.n, d.k = -1, 4, 4
    assert so.mfk_gemm_f32(ctypes.byref(d), None) == _lib.MFK_ERR_INVALID_ARGUMENT
    d.m = 4
    d.activation = 9
    assert so.mfk_gemm_f32(ctypes.byref(d), None) == _lib.MFK_ERR_INVALID_ARGUMENT
    d.activation = 0
    d.precision = 7
    assert so.mfk_gemm_f32(ctypes.byref(d), None) == _lib.MFK_ERR_INVALID_ARGUMENT
    d.precision = 0
    d.c = None  # m, n > 0 needs an output
    assert so.mfk_gemm_f32(ctypes.byref(d), None) == _lib.MFK_ERR_INVALID_ARGUMENT
    d.c, d.ldc = 16, 4
    d.beta = 1.0  # beta without c_in
    d.a, d.b = 16, 16
    assert so.mfk_gemm_f32(ctypes.byref(d), None) == _lib.MFK_ERR_INVALID_ARGUMENT
    assert so.mfk_gemm_strided_batched_f32(ctypes.byref(d), None, None) == \
        _lib.MFK_ERR_INVALID_ARGUMENT
    assert so.mfk_set_default_precision(5) == _lib.MFK_ERR_INVALID_ARGUMENT
    assert so.mfk_bias_act_f32(None, None, None, -1, 3, 0, None) == _lib.MFK_ERR_INVALID_ARGUMENT
    assert so.mfk_gemv_f32(None, 3, 4, 2, 0, None, 1, 1.0, 0.0, None, None, None) == \
        _lib.MFK_ERR_INVALID_ARGUMENT  # lda < cols
    # empty problems are a no-op success with no device work
    d2 = _lib.GemmDesc()
    d2.m, d2.n, d2.k = 0, 5, 3
    assert so.mfk_gemm_f32(ctypes.byref(d2), None) == _lib.MFK_OK


def test_api_validation_matches_reference_errors():
    m23, m32, vec = torch.ones(2, 3), torch.ones(3, 2), torch.ones(3)
    with pytest.raises(ValueError, match="inner dimensions differ"):
        mf.matmul(m23, m23)
    with pytest.raises(ValueError, match="must be 2-D"):
        mf.matmul(vec, m32)
    with pytest.raises(ValueError, match="undefined"):
        mf.matmul(None, m32)
    with pytest.raises(ValueError, match="dtypes differ"):
        mf.matmul(m23, m32.double())
    with pytest.raises(ValueError, match="beta requires c"):
        mf.gemm(m23, m32, 1.0, None, 1.0)
    with pytest.raises(ValueError, match="c shape"):
        mf.gemm(m23, m32, 1.0, torch.ones(3, 3), 1.0)
    a, b = torch.ones(2, 3, 4), torch.ones(2, 4, 5)
    with pytest.raises(ValueError, match="do not broadcast"):
        mf.gemm_strided_batched(a, torch.ones(3, 4, 5))
    with pytest.raises(ValueError, match="does not broadcast"):
        mf.gemm_strided_batched(a, b, 1.0, torch.ones(4, 5), 1.0)
    with pytest.raises(ValueError, match="does not broadcast"):
        mf.gemm_strided_batched(a, b, 1.0, torch.ones(1, 2, 3, 5), 1.0)
    with pytest.raises(ValueError, match="at least 2-D"):
        mf.gemm_strided_batched(torch.ones(4), b)
    with pytest.raises(ValueError, match="beta requires"):
        mf.gemm_strided_batched(a, b, 1.0, None, 1.0)
    with pytest.raises(ValueError):
        mf.bias_add(torch.ones(4, 5), torch.ones(4))
    # valid arguments on a device without these kernels: NotImplemented, never a CPU fallback
    with pytest.raises(NotImplementedError):
        mf.matmul(m23, m32)
    with pytest.raises(NotImplementedError):
        mf.gemm_strided_batched(a, b)


def reference_odometer(shape_batch, strides):
    """The reference adapter's walk (src/backends/cpu/backend.cpp:251-270), restated."""
    batch = int(np.prod(shape_batch)) if shape_batch else 1
    nd = len(shape_batch)
    index = [0] * nd
    off, out = 0, []
    for _ in range(batch):
        out.append(off)
        for d in range(nd - 1, -1, -1):
            index[d] += 1
            if index[d] < shape_batch[d]:
                off += strides[d]
                break
            off -= (index[d] - 1) * strides[d]
            index[d] = 0
    return out


@pytest.mark.parametrize("shape,expand", [((2, 1, 3, 4), (2, 5, 3, 4)), ((5, 4, 6), (2, 5, 4, 6)),
                                          ((3, 4, 5), (3, 4, 5)), ((1, 7, 2), (6, 7, 2))])
def test_batch_offsets_follow_the_reference_odometer(shape, expand):
    t = torch.zeros(shape).expand(expand)
    bshape = expand[:-2]
    got = ops._odometer_offsets(t, bshape)
    want = reference_odometer(list(bshape), list(t.stride()[:len(bshape)]))
    assert got.tolist() == want


def test_no_cpu_fallback_when_library_missing(monkeypatch, tmp_path):
    monkeypatch.setattr(_lib, "LIB_PATH", str(tmp_path / "missing.so"))
    monkeypatch.setattr(_lib, "_lib", None)
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        _lib.lib()


def test_strided_copy_argument_errors_before_launch():
    so = _lib.lib()
    i64x = ctypes.c_int64 * 13
    shape = i64x(3, -1)
    strides = i64x(1, 1)
    assert so.mfk_strided_copy_f32(None, shape, strides, 2, None, None) == \
        _lib.MFK_ERR_INVALID_ARGUMENT
    assert so.mfk_strided_copy_f32(None, shape, strides, -1, None, None) == \
        _lib.MFK_ERR_INVALID_ARGUMENT
    # an empty view copies nothing and needs no device
    shape = i64x(3, 0)
    assert so.mfk_strided_copy_f32(None, shape, strides, 2, None, None) == _lib.MFK_OK
    # 13 dims that no merge can reduce (a reversed permutation of a 2 x ... x 2 tensor)
    shape = i64x(*([2] * 13))
    strides = i64x(*[1 << d for d in range(13)])
    assert so.mfk_strided_copy_f32(ctypes.c_void_p(16), shape, strides, 13,
                                   ctypes.c_void_p(16), None) == _lib.MFK_ERR_UNSUPPORTED
    assert so.mfk_copy_f32(None, None, -1, None) == _lib.MFK_ERR_INVALID_ARGUMENT
    assert so.mfk_copy_f32(None, None, 0, None) == _lib.MFK_OK
    assert so.mfk_copy_peer(None, 0, None, 0, -1, None) == _lib.MFK_ERR_INVALID_ARGUMENT
    assert so.mfk_copy_peer(None, 0, None, 1, 0, None) == _lib.MFK_OK


def test_contiguous_and_to_refuse_cpu_tensors_like_the_dispatcher():
    x = torch.zeros(3, 4).t()
    with pytest.raises(NotImplementedError):
        mf.contiguous(x)
    with pytest.raises(NotImplementedError):
        mf.copy(torch.zeros(3))
    y = torch.zeros(3, 4)
    assert mf.contiguous(y) is y  # already contiguous: returned as is, as the reference does
    assert mf.to(y, "cpu") is y


def test_sharded_argument_checks_without_a_device():
    from mensurflow_b200 import sharded

    so = _lib.lib()
    descs = (_lib.GemmDesc * 2)()
    devs = (ctypes.c_int32 * 2)(0, 0)
    streams = (ctypes.c_void_p * 2)()
    assert so.mfk_sharded_gemm_f32(descs, 0, devs, streams, 0, 0, None, 0) == \
        _lib.MFK_ERR_INVALID_ARGUMENT
    assert so.mfk_sharded_gemm_f32(None, 2, devs, streams, 0, 0, None, 0) == \
        _lib.MFK_ERR_INVALID_ARGUMENT
    assert so.mfk_ipc_get_handle(None, None, None) == _lib.MFK_ERR_INVALID_ARGUMENT
    assert so.mfk_ipc_open_handle(None, None) == _lib.MFK_ERR_INVALID_ARGUMENT
    assert so.mfk_ipc_close_handle(None) == _lib.MFK_ERR_INVALID_ARGUMENT
    # gather="peer" needs the mapped buffer of C
    with pytest.raises(ValueError):
        sharded.sharded_gemm(torch.zeros(4, 3), torch.zeros(3, 2), 4, gather="peer")


@pytest.mark.parametrize("total,unit_bytes,align", [(8192, 4 * 16384, 128), (4096, 4 * 1024, 128),
                                                    (1000, 400, 128), (512, 3 << 20, 1), (5, 3 << 20, 1),
                                                    (130, 1, 128), (1, 8, 1), (0, 8, 1)])
def test_host_pipeline_block_schedule(total, unit_bytes, align):
    """The default row-block schedule of the host-tensor pipelines: blocks of about 64 MB of
    input, the last two blocks' worth halved down to `align` units; every unit in exactly one
    block, every boundary but the last a multiple of `align`, block sizes never growing at the
    end. An explicit block count gives that many equal blocks."""
    b = ops._block_bounds(total, unit_bytes, align, None)
    assert b[0] == 0 and b[-1] == total
    sizes = np.diff(b)
    assert (sizes > 0).all()
    assert all(x % align == 0 for x in b[:-1])
    assert all(s <= max(align, ops._GEMM_BLOCK_BYTES // unit_bytes) for s in sizes)
    assert list(sizes[-3:]) == sorted(sizes[-3:], reverse=True)
    if total >= 4 * align:
        assert sizes[-1] <= align  # the tail is one aligned unit block
    fixed = ops._block_bounds(total, unit_bytes, align, 4)
    assert fixed[0] == 0 and fixed[-1] == total and (np.diff(fixed) > 0).all()
    assert len(fixed) - 1 <= 4
