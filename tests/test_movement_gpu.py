"""Device-side packing of views (Tensor::contiguous), the Copy op and device-to-device moves
(Tensor::to) on the B200, against the reference.

The reference packs a non-CPU view by copying it to the host and back (src/core/tensor.cpp:208-230);
mfk_strided_copy_f32 does it on the device. Copies are exact, so every case must be bit-identical
to the reference's own Tensor::contiguous() of the same view (tests/golden/copy_cases.npz, made by
the reference) — the views of its tests/core/transfer_test.cpp and view_test.cpp plus shapes that
reach each kernel of the copy (row copies aligned and not, tiled transposes with ragged edges and
batch dims, gathers without a unit stride, broadcast dims, short rows, one element, empty).
"""
import ctypes

import numpy as np
import pytest
import torch

import mensurflow_b200 as mf
from helpers import COPY_CASES, copy_case, golden
from mensurflow_b200 import _lib

pytestmark = pytest.mark.gpu


def torch_view(x, case, full):
    """The same view in torch: permute, then slice with steps, then expand."""
    v = x.permute(*case[2])
    for d, (start, end, step) in enumerate(full):
        idx = [slice(None)] * v.dim()
        idx[d] = slice(start, max(start, end), step)
        v = v[tuple(idx)]
    if case[4] is not None:
        v = v.expand(*case[4])
    return v


@pytest.mark.parametrize("i", range(len(COPY_CASES)), ids=[c[0] for c in COPY_CASES])
def test_contiguous_matches_reference_views(cuda, i):
    gold = golden("copy_cases.npz")
    case = COPY_CASES[i]
    x, full = copy_case(i)
    view = torch_view(torch.from_numpy(x).to(cuda), case, full)
    before = _lib.launch_count()
    got = mf.contiguous(view)
    assert got.is_contiguous() and got.device == cuda
    want = gold[case[0]]
    assert tuple(got.shape) == want.shape
    assert np.array_equal(got.cpu().numpy(), want), case[0]
    if not view.is_contiguous():
        assert _lib.launch_count() == before + 1  # one kernel, no host staging
        assert got.data_ptr() != view.data_ptr()


def test_contiguous_leaves_guards_untouched(cuda):
    """The kernel writes exactly the output window: NaN-poisoned guard regions on both sides of
    it stay as they were (copy kernels of each kind)."""
    rng = np.random.default_rng(5)
    base = torch.from_numpy(rng.standard_normal((67, 133)).astype(np.float32)).to(cuda)
    for view in (base.t(), base[:, 5:70], base[::2, 1::3], base[3:4, :].expand(9, 133),
                 base[:, :7]):
        n = view.numel()
        buf = torch.full((n + 2048,), float("nan"), device=cuda)
        out = buf[1024:1024 + n]
        shape = (ctypes.c_int64 * view.dim())(*view.shape)
        strides = (ctypes.c_int64 * view.dim())(*view.stride())
        rc = _lib.lib().mfk_strided_copy_f32(view.data_ptr(), shape, strides, view.dim(),
                                             out.data_ptr(), torch.cuda.current_stream().cuda_stream)
        assert rc == _lib.MFK_OK
        host = buf.cpu().numpy()
        assert np.isnan(host[:1024]).all() and np.isnan(host[1024 + n:]).all()
        assert np.array_equal(host[1024:1024 + n], view.cpu().contiguous().numpy().reshape(-1))


def test_transpose_round_trip_full_size(cuda):
    """8192 x 8192 (256 MiB, the C2 operand size): packing the transpose of the packed transpose
    gives back the original bits."""
    g = torch.Generator(device=cuda)
    g.manual_seed(11)
    x = torch.randn(8192, 8192, device=cuda, generator=g)
    xt = mf.contiguous(x.t())
    back = mf.contiguous(xt.t())
    assert torch.equal(back, x)
    # and one spot check of the layout itself
    assert torch.equal(xt[17], x[:, 17])
    del x, xt, back
    torch.cuda.empty_cache()


def test_copy_is_a_new_tensor(cuda):
    x = torch.randn(1000, 333, device=cuda)
    y = mf.copy(x)
    assert y.data_ptr() != x.data_ptr() and torch.equal(x, y)
    odd = torch.randn(1001, device=cuda)[1:]  # not 16-byte aligned: the scalar copy
    assert torch.equal(mf.copy(odd), odd)
    z = mf.copy(x.t())
    assert z.is_contiguous() and torch.equal(z, x.t())
    assert mf.copy(torch.empty(0, 5, device=cuda)).shape == (0, 5)


def test_to_same_device_is_not_a_copy(cuda):
    x = torch.randn(4, 4, device=cuda)
    assert mf.to(x, cuda) is x
    assert mf.to(x, "cuda") is x
    host = mf.to(x.t(), "cpu")
    assert host.is_contiguous() and torch.equal(host, x.t().cpu())


def test_copy_peer_on_one_device(cuda):
    """mfk_copy_peer with the same source and target device is a device-to-device copy."""
    x = torch.randn(12345, device=cuda)
    y = torch.empty_like(x)
    rc = _lib.lib().mfk_copy_peer(y.data_ptr(), 0, x.data_ptr(), 0, x.numel() * 4,
                                  torch.cuda.current_stream().cuda_stream)
    assert rc == _lib.MFK_OK
    assert torch.equal(x, y)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_to_between_devices(cuda):
    """Tensor::to between two GPUs: a peer copy of the packed view, values preserved, result
    contiguous on the target (transfer_test.cpp:36-46 asks the same of a cross-device move)."""
    x = torch.randn(300, 500, device=cuda)
    other = torch.device("cuda", 1)
    moved = mf.to(x.t(), other)
    assert moved.device == other and moved.is_contiguous()
    assert torch.equal(moved.cpu(), x.t().cpu())
    back = mf.to(moved, cuda)
    assert torch.equal(back, x.t())
