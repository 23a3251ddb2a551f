"""Attention end to end on the B200 (§8(f) "next", rank 1): the batched GEMMs plus the softmax
and masking between them, against the reference's own outputs (tests/golden/attention_cases.npz,
made by running the reference's attention and softmax). Cases follow the reference's
tests/ops/softmax_loss_test.cpp test_attention: plain, Bool mask broadcast over batch and heads
(query 2 sees no key), causal, both with an explicit scale, and k/v shared by every head."""
import numpy as np
import pytest
import torch

import mensurflow_b200 as mf
from helpers import attention_inputs, golden, ulp_diff
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def dev(x, cuda):
    return torch.from_numpy(np.ascontiguousarray(x)).to(cuda)


def test_softmax_matches_reference(cuda):
    g = golden("attention_cases.npz")
    x = attention_inputs()["softmax_x"]
    for axis in (-1, 1, 0):
        for log in (False, True):
            fn = mf.log_softmax if log else mf.softmax
            got = fn(dev(x, cuda), axis).cpu().numpy()
            want = g[f"softmax_a{axis}_l{int(log)}"]
            assert np.array_equal(np.isnan(got), np.isnan(want)), "NaN lines differ"
            assert np.array_equal(np.isinf(got), np.isinf(want)), "-inf entries differ"
            ok = ~np.isnan(want) & ~np.isinf(want)
            if log:
                # (x - max) - log(sum): near zero this cancels, so bound the error by the size of
                # log(sum) (<= log(17) here): a few ulp of it, absolute
                err = np.abs(got[ok].astype(np.float64) - want[ok])
                assert err.max() <= 1e-6, f"log_softmax axis {axis}: {err.max():.3g}"
            else:
                d = ulp_diff(got[ok], want[ok])
                # exp is CUDA's expf on the device and the C library's on the host: a few ulp
                assert d.max() <= 4, f"softmax axis {axis}: {int(d.max())} ulp"
    with pytest.raises(ValueError):
        mf.softmax(dev(x, cuda), 3)
    assert mf.device_status() == 0


def test_where_matches_reference_semantics(cuda):
    rng = np.random.default_rng(2)
    cond = rng.random((4, 1, 6)) > 0.5
    x = rng.standard_normal((4, 5, 6)).astype(np.float32)
    y = np.float32(-np.inf)
    got = mf.where(dev(cond, cuda), dev(x, cuda), torch.tensor(y, device=cuda)).cpu().numpy()
    np.testing.assert_array_equal(got, O.where(cond, x, y))
    with pytest.raises(ValueError):
        mf.where(dev(x, cuda), dev(x, cuda), dev(x, cuda))  # condition must be Bool
    assert mf.device_status() == 0


@pytest.mark.parametrize("name", ["plain", "mask", "causal", "both"])
def test_attention_cases(cuda, name):
    a = attention_inputs()
    g = golden("attention_cases.npz")
    mask, causal, scale = {"plain": (None, False, 0.0), "mask": (a["keep"], False, 0.0),
                           "causal": (None, True, 0.0), "both": (a["keep"], True, 0.5)}[name]
    got = mf.attention(dev(a["q"], cuda), dev(a["k"], cuda), dev(a["v"], cuda),
                       None if mask is None else dev(mask, cuda), causal, scale).cpu().numpy()
    want = g[f"attention_{name}"]
    # the reference's own attention test tolerance (softmax_loss_test.cpp: 1e-4, 1e-6)
    np.testing.assert_allclose(got, want, rtol=1e-4, atol=1e-6, err_msg=name)
    if mask is not None:
        assert (got[:, :, 2, :] == 0.0).all(), "a query that sees no key gets zeros"
    assert mf.device_status() == 0


def test_attention_broadcast_and_causal_sizes(cuda):
    a = attention_inputs()
    g = golden("attention_cases.npz")
    got = mf.attention(dev(a["q"], cuda), dev(a["k1"], cuda), dev(a["v1"], cuda)).cpu().numpy()
    np.testing.assert_allclose(got, g["attention_broadcast_kv"], rtol=1e-4, atol=1e-6)
    got = mf.attention(dev(a["q2"], cuda), dev(a["k2"], cuda), dev(a["v2"], cuda), None,
                       True).cpu().numpy()
    np.testing.assert_allclose(got, g["attention_causal_64"], rtol=1e-4, atol=1e-6)
    with pytest.raises(ValueError):
        mf.attention(dev(a["q"], cuda), torch.zeros(2, 3, 7, 9, device=cuda), dev(a["v"], cuda))
    with pytest.raises(ValueError):
        mf.attention(dev(a["q"], cuda), dev(a["k"], cuda), dev(a["v"], cuda),
                     torch.ones(5, 7, device=cuda))  # non-Bool mask
    with pytest.raises(ValueError):
        mf.attention(dev(a["q"], cuda), dev(a["k"], cuda), dev(a["v"], cuda),
                     torch.ones(4, 1, 5, 7, dtype=torch.bool, device=cuda))
    assert mf.device_status() == 0


def test_fused_mask_equals_where_then_softmax(cuda):
    """The fused masked softmax gives the same bits as the reference's composition run with this
    library's own where and softmax kernels."""
    rng = np.random.default_rng(3)
    s = dev(rng.standard_normal((6, 33, 47)).astype(np.float32) * 4, cuda)
    keep = dev(rng.random((33, 47)) > 0.3, cuda)
    lower = torch.ones(33, 47, dtype=torch.bool, device=cuda).tril()
    composed = mf.softmax(mf.where(lower, mf.where(keep, s, torch.tensor(-np.inf, device=cuda)),
                                   torch.tensor(-np.inf, device=cuda)), -1)
    fused = s.clone()
    kk = keep.expand(6, 33, 47)
    from mensurflow_b200 import _lib
    import ctypes  # noqa: F401
    rc = _lib.lib().mfk_masked_softmax_f32(fused.data_ptr(), kk.data_ptr(), 0, 47, 1,
                                           fused.data_ptr(), 6, 33, 47,
                                           torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    assert torch.equal(fused, composed)
    assert mf.device_status() == 0


@pytest.mark.parametrize("chunks", [1, 4, 16, None])
def test_attention_on_host_tensors(cuda, chunks):
    """Execution::GPU on host-resident q, k, v: batch chunks stream through the device and the
    result comes back as a host tensor; it equals the attention of the same tensors on the device
    (each chunk is the same op on fewer batch entries) within the reference's 1e-4, with a 2-D
    mask and the causal mask."""
    rng = np.random.default_rng(12)
    q = torch.from_numpy(rng.standard_normal((2, 5, 40, 16)).astype(np.float32) * 0.5)
    k = torch.from_numpy(rng.standard_normal((2, 5, 56, 16)).astype(np.float32) * 0.5)
    v = torch.from_numpy(rng.standard_normal((2, 5, 56, 24)).astype(np.float32))
    mask = torch.from_numpy(rng.random((40, 56)) > 0.2)
    hq, hk, hv = (t.pin_memory() for t in (q, k, v))
    out = torch.empty(2, 5, 40, 24, pin_memory=True)
    got = mf.attention(hq, hk, hv, mask, causal=True, execution="gpu", out=out, chunks=chunks)
    assert got is out and got.device.type == "cpu"
    want = mf.attention(q.to(cuda), k.to(cuda), v.to(cuda), mask.to(cuda), causal=True).cpu()
    np.testing.assert_allclose(got.numpy(), want.numpy(), rtol=1e-4, atol=1e-6)
    ref = O.attention(q.numpy(), k.numpy(), v.numpy(), mask.numpy(), causal=True)
    np.testing.assert_allclose(got.numpy(), ref, rtol=1e-4, atol=1e-5)
    assert mf.device_status() == 0


def test_attention_on_host_tensors_argument_errors(cuda):
    q = torch.zeros(2, 4, 8)
    with pytest.raises(ValueError):
        mf.attention(q, torch.zeros(3, 4, 8), torch.zeros(3, 4, 8), execution="gpu")
    with pytest.raises(ValueError):  # a mask per batch entry
        mf.attention(q, q, q, torch.ones(2, 4, 4, dtype=torch.bool), execution="gpu")
    with pytest.raises(ValueError):
        mf.attention(q, q, q, execution="tpu")


# ---- the fused kernel (mfk_attention_f32) --------------------------------------------------

def _qkv(heads, length, seed, std=1.0 / np.sqrt(128)):
    rng = np.random.default_rng(seed)
    return tuple((rng.standard_normal((heads, length, 128)) * std).astype(np.float32)
                 for _ in range(3))


@pytest.mark.parametrize("heads,length,causal", [
    (3, 256, True), (2, 384, True), (2, 200, True), (1, 77, False), (2, 128, False),
    (4, 512, True), (1, 640, False), (2, 1, True)])
def test_fused_attention_matches_reference(cuda, heads, length, causal):
    """The one-kernel path against the reference's own attention (composed gemm / where / softmax
    / gemm on the CPU) within its test tolerance (softmax_loss_test.cpp: 1e-4, 1e-6), at lengths
    that are and are not multiples of the kernel's 128-key tiles and 256-query blocks."""
    q, k, v = _qkv(heads, length, 10 * heads + length)
    got = mf.attention(dev(q, cuda), dev(k, cuda), dev(v, cuda), causal=causal,
                       fused=True).cpu().numpy()
    want = O.ref_attention(q, k, v, causal=causal)
    np.testing.assert_allclose(got, want, rtol=1e-4, atol=1e-6)
    composed = mf.attention(dev(q, cuda), dev(k, cuda), dev(v, cuda), causal=causal,
                            fused=False).cpu().numpy()
    np.testing.assert_allclose(got, composed, rtol=1e-4, atol=1e-6)
    assert mf.device_status() == 0


def test_fused_attention_running_max_rescales(cuda):
    """Scores that grow along the keys by ~30 over the sequence: the running row maximum is raised
    several times (each time by more than the kernel's slack of 8), so the output accumulator is
    rescaled in tensor memory between key tiles; an explicit scale as well."""
    heads, length = 2, 768
    rng = np.random.default_rng(7)
    u = rng.standard_normal(128).astype(np.float32)
    u /= np.linalg.norm(u)
    q = (rng.standard_normal((heads, length, 128)) * 0.05 + u).astype(np.float32)
    ramp = (np.arange(length, dtype=np.float32) / length * 30.0)[None, :, None]
    k = (rng.standard_normal((heads, length, 128)) * 0.05 + ramp * u).astype(np.float32)
    v = (rng.standard_normal((heads, length, 128)) / np.sqrt(128)).astype(np.float32)
    for causal in (True, False):
        got = mf.attention(dev(q, cuda), dev(k, cuda), dev(v, cuda), causal=causal, scale=1.0,
                           fused=True).cpu().numpy()
        want = O.ref_attention(q, k, v, causal=causal, scale=1.0)
        np.testing.assert_allclose(got, want, rtol=1e-4, atol=1e-6, err_msg=f"causal={causal}")
    assert mf.device_status() == 0


@pytest.mark.parametrize("heads,length,causal,kind", [
    (2, 300, False, "shared"), (2, 300, True, "shared"), (3, 256, False, "per_head"),
    (2, 77, True, "empty_rows"), (1, 640, False, "empty_rows"), (2, 128, True, "per_head"),
    (2, 512, False, "columns")])
def test_fused_attention_with_mask(cuda, heads, length, causal, kind):
    """The one kernel with a Bool keep mask (mfk_attention_masked_f32) against the reference's
    attention(q, k, v, &mask, causal) and the composed path: a mask shared by every head, one per
    head, rows whose every key is masked out (zeros, as the reference's softmax gives them), and
    whole key columns masked; causal and not, at lengths off the tile grid."""
    q, k, v = _qkv(heads, length, 7 * heads + length)
    rng = np.random.default_rng(length + heads)
    if kind == "per_head":
        mask = rng.random((heads, length, length)) > 0.5
    else:
        mask = rng.random((length, length)) > 0.3
    if kind == "empty_rows":
        mask[[0, length // 2, length - 1], :] = False
    if kind == "columns":
        mask[:, 100:300] = False
    tq, tk, tv, tm = dev(q, cuda), dev(k, cuda), dev(v, cuda), dev(mask, cuda)
    got = mf.attention(tq, tk, tv, tm, causal=causal, fused=True).cpu().numpy()
    want = O.ref_attention(q, k, v, mask, causal=causal)
    np.testing.assert_allclose(got, want, rtol=1e-4, atol=1e-6)
    composed = mf.attention(tq, tk, tv, tm, causal=causal, fused=False).cpu().numpy()
    np.testing.assert_allclose(got, composed, rtol=1e-4, atol=1e-6)
    assert mf.device_status() == 0


@pytest.mark.parametrize("scale", [-0.3, -1e-3, 2.0])
def test_fused_attention_any_scale(cuda, scale):
    """The reference takes any nonzero scale (src/ops/attention.cpp:64-69: scale is the scores
    GEMM's alpha). The kernel finds each row's maximum of fl(scale * s) as fl(scale * max s),
    or fl(scale * min s) for a negative scale, and folds the scale into the exponent: a negative,
    a tiny and a large scale against the reference, at a length off the tile grid."""
    q, k, v = _qkv(2, 300, 31)
    for causal in (True, False):
        got = mf.attention(dev(q, cuda), dev(k, cuda), dev(v, cuda), causal=causal, scale=scale,
                           fused=True).cpu().numpy()
        want = O.ref_attention(q, k, v, causal=causal, scale=scale)
        np.testing.assert_allclose(got, want, rtol=1e-4, atol=1e-6,
                                   err_msg=f"scale={scale} causal={causal}")
    assert mf.device_status() == 0


def test_fused_attention_routing(cuda):
    """Eligible calls take the one kernel by default, a Bool mask that broadcasts to the scores
    included (mfk_attention_masked_f32); a mask on the host, a head dimension other than 128,
    shared k/v or 1xTF32 take the composed path, and fused=True refuses them."""
    q, k, v = _qkv(2, 128, 3)
    tq, tk, tv = dev(q, cuda), dev(k, cuda), dev(v, cuda)
    np.testing.assert_array_equal(mf.attention(tq, tk, tv, causal=True).cpu().numpy(),
                                  mf.attention(tq, tk, tv, causal=True, fused=True).cpu().numpy())
    mask = torch.ones(128, 128, dtype=torch.bool, device=cuda)
    np.testing.assert_array_equal(
        mf.attention(tq, tk, tv, mask=mask, causal=True).cpu().numpy(),
        mf.attention(tq, tk, tv, mask=mask, causal=True, fused=True).cpu().numpy())
    with pytest.raises(ValueError):
        mf.attention(tq, tk, tv, mask=mask.cpu(), fused=True)
    with pytest.raises(ValueError):
        mf.attention(tq[..., :64], tk[..., :64], tv[..., :64], fused=True)
    with pytest.raises(ValueError):
        mf.attention(tq, tk[:1], tv[:1], fused=True)
    with pytest.raises(ValueError):
        mf.attention(tq, tk, tv, precision="1xtf32", fused=True)
    # the composed path still serves them, and an all-true mask changes nothing
    got = mf.attention(tq, tk, tv, mask=mask, causal=True, fused=False).cpu().numpy()
    np.testing.assert_allclose(got, O.ref_attention(q, k, v, causal=True), rtol=1e-4, atol=1e-6)
    fused = mf.attention(tq, tk, tv, mask=mask, causal=True).cpu().numpy()
    np.testing.assert_allclose(fused, O.ref_attention(q, k, v, causal=True), rtol=1e-4, atol=1e-6)
    assert mf.device_status() == 0
