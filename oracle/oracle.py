"""TEST INFRASTRUCTURE ONLY — Python access to the parity oracle.

Two libraries, both built by ``oracle/Makefile``:

* ``oracle/_build/libmforacle.so`` — the C restatement (``oracle/mf_oracle.c``) of the
  reference's CPU algorithms. Always available: built here or, on a machine without the
  prebuilt file, compiled on first use with the system gcc.
* ``oracle/_ref/libmfref.so`` — the unmodified reference library compiled from its own
  sources plus ``oracle/ref_shim.cpp``. Present only where it was built (it travels with the
  repository snapshot); ``reference()`` returns None without it.

Only tests, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline/reference legs may use this
module. The product path never imports it.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
import threading

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
_ORACLE_SO = os.path.join(HERE, "_build", "libmforacle.so")
_REF_SO = os.path.join(HERE, "_ref", "libmfref.so")

_lock = threading.Lock()
_oracle = None
_ref = None
_ref_loaded = False

_i64 = ctypes.c_int64
_u64 = ctypes.c_uint64
_f32 = ctypes.c_float
_ptr = ctypes.c_void_p


def _p(arr):
    return None if arr is None else ctypes.c_void_p(arr.ctypes.data)


def build_oracle() -> str:
    if not os.path.exists(_ORACLE_SO) or os.path.getmtime(_ORACLE_SO) < os.path.getmtime(
        os.path.join(HERE, "mf_oracle.c")
    ):
        subprocess.run(["make", "-s", "-C", HERE, "oracle"], check=True)
    return _ORACLE_SO


def lib():
    """The C restatement, built on first use."""
    global _oracle
    with _lock:
        if _oracle is None:
            so = ctypes.CDLL(build_oracle())
            so.mfo_uniform.argtypes = [_ptr, _i64, _f32, _f32, _u64, _u64]
            so.mfo_normal.argtypes = [_ptr, _i64, _f32, _f32, _u64, _u64]
            so.mfo_philox_word.argtypes = [_u64, _u64, ctypes.c_int]
            so.mfo_philox_word.restype = ctypes.c_uint32
            so.mfo_gemm_batched.argtypes = [
                _ptr, _ptr, _i64, _i64, _ptr, _ptr, _i64, _i64, _ptr, _i64, _i64,
                _ptr, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _f32, _f32, _i64,
            ]
            so.mfo_abs_product.argtypes = [
                _ptr, _ptr, _i64, _i64, _ptr, _ptr, _i64, _i64, _ptr, _i64, _i64, _i64, _i64,
            ]
            so.mfo_bias_add.argtypes = [_ptr, _ptr, _ptr, _i64, _i64]
            so.mfo_bias_grad.argtypes = [_ptr, _i64, _i64, _i64, _ptr]
            so.mfo_relu.argtypes = [_ptr, _ptr, _i64]
            so.mfo_gelu.argtypes = [_ptr, _ptr, _i64, ctypes.c_int]
            so.mfo_gemv.argtypes = [_ptr, _i64, _i64, _i64, _ptr, _f32, _f32, _ptr, _ptr, ctypes.c_int]
            so.mfo_softmax.argtypes = [_ptr, _ptr, _i64, _i64, _i64, ctypes.c_int]
            so.mfo_where.argtypes = [_ptr, _ptr, _ptr, _ptr, _i64]
            _oracle = so
    return _oracle


def reference():
    """The unmodified reference library (CPU), or None where it was not built."""
    global _ref, _ref_loaded
    with _lock:
        if not _ref_loaded:
            _ref_loaded = True
            if os.path.exists(_REF_SO):
                so = ctypes.CDLL(_REF_SO)
                so.mfref_last_error.restype = ctypes.c_char_p
                so.mfref_uniform.argtypes = [_ptr, _i64, _f32, _f32, _u64, _u64]
                so.mfref_normal.argtypes = [_ptr, _i64, _f32, _f32, _u64, _u64]
                so.mfref_gemm.argtypes = [_ptr, _i64, _i64, _ptr, _i64, _i64, _ptr, _f32, _f32,
                                          ctypes.c_int, ctypes.c_int, _ptr]
                so.mfref_matmul.argtypes = [_ptr, _i64, _i64, _ptr, _i64, _ptr]
                so.mfref_gemm_strided_batched.argtypes = [
                    _ptr, _ptr, ctypes.c_int, _ptr, _ptr, ctypes.c_int, _ptr, _ptr, ctypes.c_int,
                    _f32, _f32, ctypes.c_int, ctypes.c_int, _ptr, _ptr, _ptr,
                ]
                so.mfref_bias_add.argtypes = [_ptr, _i64, _i64, _ptr, _ptr]
                so.mfref_bias_add_backward.argtypes = [_ptr, _i64, _i64, _ptr]
                so.mfref_matmul_backward.argtypes = [_ptr, _ptr, _ptr, _i64, _i64, _i64, _ptr,
                                                     _ptr]
                so.mfref_gelu.argtypes = [_ptr, _i64, ctypes.c_int, _ptr]
                so.mfref_relu.argtypes = [_ptr, _i64, _ptr]
                so.mfref_gemv.argtypes = [_ptr, _i64, _i64, _ptr, _f32, _ptr, _f32, ctypes.c_int, _ptr]
                so.mfref_matvec.argtypes = [_ptr, _i64, _i64, _ptr, _ptr]
                so.mfref_gemm_bench_new.argtypes = [_i64, _i64, _i64, ctypes.c_int, _u64]
                so.mfref_gemm_bench_new.restype = ctypes.c_void_p
                so.mfref_gemm_bench_run.argtypes = [_ptr, _f32, _f32, ctypes.c_int, ctypes.c_int,
                                                    _ptr]
                so.mfref_gemm_bench_free.argtypes = [_ptr]
                so.mfref_max_threads.restype = ctypes.c_int
                so.mfref_openmp.restype = ctypes.c_int
                so.mfref_time_gemv.argtypes = [_i64, _i64, _u64, ctypes.c_int, ctypes.c_int, _ptr]
                so.mfref_set_threads.argtypes = [ctypes.c_int]
                so.mfref_softmax.argtypes = [_ptr, _ptr, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                             _ptr]
                so.mfref_attention.argtypes = [_ptr, _ptr, ctypes.c_int, _ptr, _ptr, ctypes.c_int,
                                               _ptr, _ptr, ctypes.c_int, _ptr, _ptr, ctypes.c_int,
                                               ctypes.c_int, _f32, _ptr, _ptr, _ptr]
                so.mfref_time_mlp.argtypes = [_i64, _i64, _i64, _u64, ctypes.c_int,
                                              ctypes.c_int, _ptr]
                so.mfref_time_attention_gemms.argtypes = [_i64, _i64, _i64, _u64, ctypes.c_int,
                                                          ctypes.c_int, _ptr]
                so.mfref_contiguous_view.argtypes = [_ptr, _ptr, ctypes.c_int, _ptr, _ptr, _ptr,
                                                     _ptr, _ptr, ctypes.c_int, _ptr, _ptr]
                so.mfref_time_transpose_contiguous.argtypes = [_i64, _i64, ctypes.c_int,
                                                               ctypes.c_int, _ptr]
                _ref = so
    return _ref


def _check_ref(rc):
    if rc != 0:
        raise RuntimeError(reference().mfref_last_error().decode())


# ---- the C restatement -------------------------------------------------------------------

def uniform(n, low, high, seed, offset=0):
    out = np.empty(n, np.float32)
    lib().mfo_uniform(_p(out), n, low, high, seed, offset)
    return out


def normal(n, mean, std, seed, offset=0):
    out = np.empty(n, np.float32)
    lib().mfo_normal(_p(out), n, mean, std, seed, offset)
    return out


def _as_strided_args(x, transpose):
    """Row/col element strides of op(x) for a 2-D C-contiguous float32 array."""
    rs, cs = x.strides[0] // 4, x.strides[1] // 4
    return (cs, rs) if transpose else (rs, cs)


def gemm(a, b, alpha=1.0, c=None, beta=0.0, transpose_a=False, transpose_b=False,
         bias=None, act=None, kc=256):
    """alpha*op(a)@op(b) + beta*c (+ bias, then act) with the restated CPU algorithm."""
    a = np.ascontiguousarray(a, np.float32)
    b = np.ascontiguousarray(b, np.float32)
    m, k = (a.shape[1], a.shape[0]) if transpose_a else a.shape
    n = b.shape[0] if transpose_b else b.shape[1]
    rsa, csa = _as_strided_args(a, transpose_a)
    rsb, csb = _as_strided_args(b, transpose_b)
    out = np.empty((m, n), np.float32)
    c0 = None
    if c is not None and beta != 0.0:
        c0 = np.ascontiguousarray(np.broadcast_to(c, (m, n)), np.float32)
    lib().mfo_gemm_batched(_p(a), None, rsa, csa, _p(b), None, rsb, csb, _p(out), n, m * n,
                           _p(c0), n, 1, m * n, 1, m, n, k, alpha, beta if c0 is not None else 0.0,
                           kc)
    if bias is not None:
        out = bias_add(out, bias)
    if act is not None:
        out = activation(out, act)
    return out


def abs_product(a, b, transpose_a=False, transpose_b=False):
    """(|op(a)|·|op(b)|) in float64."""
    a = np.ascontiguousarray(a, np.float32)
    b = np.ascontiguousarray(b, np.float32)
    m, k = (a.shape[1], a.shape[0]) if transpose_a else a.shape
    n = b.shape[0] if transpose_b else b.shape[1]
    rsa, csa = _as_strided_args(a, transpose_a)
    rsb, csb = _as_strided_args(b, transpose_b)
    out = np.empty((m, n), np.float64)
    lib().mfo_abs_product(_p(a), None, rsa, csa, _p(b), None, rsb, csb, _p(out), 1, m, n, k)
    return out


def gemm_batched_raw(a, a_off, rsa, csa, b, b_off, rsb, csb, batch, m, n, k, alpha=1.0,
                     c0=None, c0_strides=(0, 0, 0), beta=0.0, kc=256):
    """The restated cpu::BatchedGemm on flat float32 buffers with explicit offsets/strides."""
    out = np.empty((batch, m, n), np.float32)
    ao = np.ascontiguousarray(a_off, np.int64)
    bo = np.ascontiguousarray(b_off, np.int64)
    lib().mfo_gemm_batched(_p(a), _p(ao), rsa, csa, _p(b), _p(bo), rsb, csb, _p(out), n, m * n,
                           _p(c0), c0_strides[0], c0_strides[1], c0_strides[2], batch, m, n, k,
                           alpha, beta if c0 is not None else 0.0, kc)
    return out


def abs_product_batched_raw(a, a_off, rsa, csa, b, b_off, rsb, csb, batch, m, n, k):
    out = np.empty((batch, m, n), np.float64)
    ao = np.ascontiguousarray(a_off, np.int64)
    bo = np.ascontiguousarray(b_off, np.int64)
    lib().mfo_abs_product(_p(a), _p(ao), rsa, csa, _p(b), _p(bo), rsb, csb, _p(out), batch, m, n, k)
    return out


def bias_add(x, bias):
    x = np.ascontiguousarray(x, np.float32)
    bias = np.ascontiguousarray(bias, np.float32)
    out = np.empty_like(x)
    lib().mfo_bias_add(_p(x), _p(bias), _p(out), x.shape[0], x.shape[1])
    return out


def bias_grad(g):
    """The bias gradient of bias_add: column sums of g in row order, in float
    (mf_oracle.c mfo_bias_grad; src/ops/elementwise.cpp:263-283)."""
    g = np.ascontiguousarray(g, np.float32)
    out = np.empty(g.shape[1], np.float32)
    lib().mfo_bias_grad(_p(g), g.shape[0], g.shape[1], g.shape[1], _p(out))
    return out


def matmul_backward(a, b, g):
    """(dA, dB) = (g @ b^T, a^T @ g), the products matmul's recorded backward makes
    (src/ops/blas.cpp:220-230), with the restated GEMM."""
    return gemm(g, b, transpose_b=True), gemm(a, g, transpose_a=True)


def activation(x, act):
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty_like(x)
    if act == "relu":
        lib().mfo_relu(_p(x), _p(out), x.size)
    elif act in ("gelu", "gelu_tanh"):
        lib().mfo_gelu(_p(x), _p(out), x.size, 1 if act == "gelu_tanh" else 0)
    else:
        raise ValueError(f"unknown activation {act!r}")
    return out


def softmax(x, axis=-1, log=False):
    """The restated softmax / log_softmax along `axis`."""
    x = np.ascontiguousarray(x, np.float32)
    axis = axis % x.ndim if x.ndim else 0
    shape = x.shape if x.ndim else (1,)
    outer = int(np.prod(shape[:axis]))
    length = shape[axis]
    inner = int(np.prod(shape[axis + 1:]))
    out = np.empty_like(x)
    lib().mfo_softmax(_p(x), _p(out), outer, length, inner, 1 if log else 0)
    return out


def where(cond, x, y):
    shape = np.broadcast_shapes(np.shape(cond), np.shape(x), np.shape(y))
    c = np.ascontiguousarray(np.broadcast_to(cond, shape), np.uint8)
    xx = np.ascontiguousarray(np.broadcast_to(x, shape), np.float32)
    yy = np.ascontiguousarray(np.broadcast_to(y, shape), np.float32)
    out = np.empty(shape, np.float32)
    lib().mfo_where(_p(c), _p(xx), _p(yy), _p(out), out.size)
    return out


def attention(q, k, v, mask=None, causal=False, scale=0.0):
    """The reference's attention composition (src/ops/attention.cpp:48-98) with the restated
    pieces: batched q k^T * scale, where(mask, s, -inf), causal where, softmax, batched w v."""
    q = np.asarray(q, np.float32)
    k = np.asarray(k, np.float32)
    v = np.asarray(v, np.float32)
    d = q.shape[-1]
    if scale == 0.0:
        scale = float(np.float32(1.0 / np.sqrt(d))) if d > 0 else 1.0
    bshape = np.broadcast_shapes(q.shape[:-2], k.shape[:-2], v.shape[:-2])
    lq, lk = q.shape[-2], k.shape[-2]
    qq = np.broadcast_to(q, bshape + q.shape[-2:]).reshape(-1, lq, d)
    kk = np.broadcast_to(k, bshape + k.shape[-2:]).reshape(-1, lk, d)
    vv = np.broadcast_to(v, bshape + v.shape[-2:]).reshape(-1, lk, v.shape[-1])
    s = np.stack([gemm(qq[i], kk[i], scale, None, 0.0, False, True) for i in range(qq.shape[0])])
    s = s.reshape(bshape + (lq, lk))
    if mask is not None:
        s = where(mask, s, np.float32(-np.inf))
    if causal:
        s = where(np.tril(np.ones((lq, lk), bool)), s, np.float32(-np.inf))
    w = softmax(s, -1).reshape(-1, lq, lk)
    out = np.stack([gemm(w[i], vv[i]) for i in range(w.shape[0])])
    return out.reshape(bshape + (lq, v.shape[-1]))


def gemv(a, x, alpha=1.0, y=None, beta=0.0, transpose_a=False):
    a = np.ascontiguousarray(a, np.float32)
    x = np.ascontiguousarray(x, np.float32)
    rows, cols = a.shape
    n_out = cols if transpose_a else rows
    out = np.empty(n_out, np.float32)
    y0 = None if y is None else np.ascontiguousarray(y, np.float32)
    lib().mfo_gemv(_p(a), rows, cols, cols, _p(x), alpha, beta, _p(y0), _p(out),
                   1 if transpose_a else 0)
    return out


# ---- the reference itself (where built) --------------------------------------------------

def ref_uniform(n, low, high, seed, offset=0):
    out = np.empty(n, np.float32)
    _check_ref(reference().mfref_uniform(_p(out), n, low, high, seed, offset))
    return out


def ref_normal(n, mean, std, seed, offset=0):
    out = np.empty(n, np.float32)
    _check_ref(reference().mfref_normal(_p(out), n, mean, std, seed, offset))
    return out


def ref_gemm(a, b, alpha=1.0, c=None, beta=0.0, transpose_a=False, transpose_b=False):
    a = np.ascontiguousarray(a, np.float32)
    b = np.ascontiguousarray(b, np.float32)
    m = a.shape[1] if transpose_a else a.shape[0]
    n = b.shape[0] if transpose_b else b.shape[1]
    out = np.empty((m, n), np.float32)
    cc = None if c is None else np.ascontiguousarray(c, np.float32)
    _check_ref(reference().mfref_gemm(_p(a), a.shape[0], a.shape[1], _p(b), b.shape[0],
                                      b.shape[1], _p(cc), alpha, beta, int(transpose_a),
                                      int(transpose_b), _p(out)))
    return out


def ref_matmul(a, b):
    """The reference's public matmul (src/ops/blas.cpp:186-232) on the CPU."""
    a = np.ascontiguousarray(a, np.float32)
    b = np.ascontiguousarray(b, np.float32)
    m, k = a.shape
    n = b.shape[1]
    out = np.empty((m, n), np.float32)
    _check_ref(reference().mfref_matmul(_p(a), m, k, _p(b), n, _p(out)))
    return out


def ref_gemm_strided_batched(a, b, alpha=1.0, c=None, beta=0.0, transpose_a=False,
                             transpose_b=False):
    a = np.ascontiguousarray(a, np.float32)
    b = np.ascontiguousarray(b, np.float32)
    cc = None if c is None else np.ascontiguousarray(c, np.float32)
    ash = np.array(a.shape, np.int64)
    bsh = np.array(b.shape, np.int64)
    csh = None if cc is None else np.array(cc.shape if cc.ndim else [1], np.int64)
    oshape = np.zeros(8, np.int64)
    ond = ctypes.c_int(0)
    lib_ = reference()
    _check_ref(lib_.mfref_gemm_strided_batched(
        _p(a), _p(ash), a.ndim, _p(b), _p(bsh), b.ndim, _p(cc), _p(csh),
        0 if cc is None else cc.ndim, alpha, beta, int(transpose_a), int(transpose_b), None,
        _p(oshape), ctypes.byref(ond)))
    shape = tuple(int(v) for v in oshape[: ond.value])
    out = np.empty(shape, np.float32)
    _check_ref(lib_.mfref_gemm_strided_batched(
        _p(a), _p(ash), a.ndim, _p(b), _p(bsh), b.ndim, _p(cc), _p(csh),
        0 if cc is None else cc.ndim, alpha, beta, int(transpose_a), int(transpose_b), _p(out),
        _p(oshape), ctypes.byref(ond)))
    return out


def ref_bias_add(x, bias):
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty_like(x)
    _check_ref(reference().mfref_bias_add(_p(x), x.shape[0], x.shape[1],
                                          _p(np.ascontiguousarray(bias, np.float32)), _p(out)))
    return out


def ref_bias_add_backward(g):
    g = np.ascontiguousarray(g, np.float32)
    out = np.empty(g.shape[1], np.float32)
    _check_ref(reference().mfref_bias_add_backward(_p(g), g.shape[0], g.shape[1], _p(out)))
    return out


def ref_matmul_backward(a, b, g):
    a = np.ascontiguousarray(a, np.float32)
    b = np.ascontiguousarray(b, np.float32)
    g = np.ascontiguousarray(g, np.float32)
    m, k = a.shape
    n = b.shape[1]
    da = np.empty((m, k), np.float32)
    db = np.empty((k, n), np.float32)
    _check_ref(reference().mfref_matmul_backward(_p(a), _p(b), _p(g), m, k, n, _p(da), _p(db)))
    return da, db


def ref_gelu(x, approximate=False):
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty_like(x)
    _check_ref(reference().mfref_gelu(_p(x), x.size, int(approximate), _p(out)))
    return out


def ref_relu(x):
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty_like(x)
    _check_ref(reference().mfref_relu(_p(x), x.size, _p(out)))
    return out


def ref_gemv(a, x, alpha=1.0, y=None, beta=0.0, transpose_a=False):
    a = np.ascontiguousarray(a, np.float32)
    rows, cols = a.shape
    out = np.empty(cols if transpose_a else rows, np.float32)
    yy = None if y is None else np.ascontiguousarray(y, np.float32)
    _check_ref(reference().mfref_gemv(_p(a), rows, cols, _p(np.ascontiguousarray(x, np.float32)),
                                      alpha, _p(yy), beta, int(transpose_a), _p(out)))
    return out


class RefGemmBench:
    """The reference's public gemm (+ bias_add) on CPU inputs made once by its own factories."""

    def __init__(self, m, n, k, transpose_b, seed):
        self.h = reference().mfref_gemm_bench_new(m, n, k, int(transpose_b), seed)
        if not self.h:
            raise RuntimeError(reference().mfref_last_error().decode())

    def run(self, alpha, beta, with_bias, reps):
        secs = np.zeros(reps, np.float64)
        _check_ref(reference().mfref_gemm_bench_run(self.h, alpha, beta, int(with_bias), reps,
                                                     _p(secs)))
        return secs

    def close(self):
        if self.h:
            reference().mfref_gemm_bench_free(self.h)
            self.h = None


def ref_time_gemv(rows, cols, seed, warmup, reps):
    secs = np.zeros(reps, np.float64)
    _check_ref(reference().mfref_time_gemv(rows, cols, seed, warmup, reps, _p(secs)))
    return secs


def ref_time_mlp(rows, d_in, d_hid, seed, warmup, reps):
    secs = np.zeros(reps, np.float64)
    _check_ref(reference().mfref_time_mlp(rows, d_in, d_hid, seed, warmup, reps, _p(secs)))
    return secs


def ref_time_attention_gemms(heads, seq, dh, seed, warmup, reps):
    secs = np.zeros(reps, np.float64)
    _check_ref(reference().mfref_time_attention_gemms(heads, seq, dh, seed, warmup, reps,
                                                      _p(secs)))
    return secs


def view_recipe_shape(base_shape, order, slices, expand=None):
    """Shape of base.permute(order) sliced by `slices` ((start, end, step) per dim) and expanded."""
    if expand is not None:
        return tuple(expand)
    shape = []
    for d, (start, end, step) in enumerate(slices):
        size = end - start
        shape.append(0 if size <= 0 else (size + step - 1) // step)
    return tuple(shape)


def view_recipe_strided(base_shape, order, slices, expand=None):
    """(offset, shape, strides) in elements of the recipe's view over a contiguous base, with the
    reference's view arithmetic: permute reorders (shape, strides) (src/core/tensor.cpp permute),
    slice moves the offset by start*stride and multiplies the stride by step, expand gives
    broadcast dims stride 0 (leading new dims included)."""
    nd = len(base_shape)
    base_strides = [1] * nd
    for d in range(nd - 2, -1, -1):
        base_strides[d] = base_strides[d + 1] * base_shape[d + 1]
    shape = [base_shape[o] for o in order]
    strides = [base_strides[o] for o in order]
    offset = 0
    for d, (start, end, step) in enumerate(slices):
        size = max(0, end - start)
        offset += start * strides[d] if size > 0 else 0
        shape[d] = 0 if size == 0 else (size + step - 1) // step
        strides[d] *= step
    if expand is not None:
        lead = len(expand) - nd
        strides = [0] * lead + [0 if (shape[d] == 1 and expand[lead + d] != 1) else strides[d]
                                for d in range(nd)]
        shape = list(expand)
    return offset, tuple(shape), tuple(strides)


def strided_copy(buf, offset, shape, strides):
    """Restatement of cpu::strided_copy_f32 (src/backends/cpu/ops/movement/movement.cpp:12-42):
    output row r (all dims but the innermost, innermost outer dim fastest) starts at the input
    offset sum_d coord_d*strides[d]; its elements are read at unit stride when the innermost
    stride is 1 (one memcpy per row in the reference), else one by one. transpose_f32 (:44-67)
    gives the same values for a transposed matrix."""
    buf = np.asarray(buf, np.float32).reshape(-1)
    n = int(np.prod(shape)) if len(shape) else 1
    out = np.empty(n, np.float32)
    if n == 0:
        return out.reshape(shape)
    nd = len(shape)
    row = shape[-1] if nd else 1
    rows = n // row
    cols = np.arange(row, dtype=np.int64) * (strides[-1] if nd else 0)
    for r in range(rows):
        src, index = offset, r
        for d in range(nd - 2, -1, -1):
            src += (index % shape[d]) * strides[d]
            index //= shape[d]
        out[r * row:(r + 1) * row] = buf[src + cols]
    return out.reshape(shape)


def ref_contiguous_view(x, order, slices, expand=None):
    """The reference's Tensor::contiguous() of x.permute(order).slice(...)[.expand(...)]."""
    x = np.ascontiguousarray(x, np.float32)
    nd = x.ndim
    base = np.array(x.shape, np.int64)
    o = np.array(order, np.int32)
    st = np.array([s[0] for s in slices], np.int64)
    en = np.array([s[1] for s in slices], np.int64)
    sp = np.array([s[2] for s in slices], np.int64)
    ex = None if expand is None else np.array(expand, np.int64)
    shape = view_recipe_shape(x.shape, order, slices, expand)
    out = np.empty(shape, np.float32)
    oshape = np.zeros(16, np.int64)
    _check_ref(reference().mfref_contiguous_view(
        _p(x), _p(base), nd, _p(o), _p(st), _p(en), _p(sp), _p(ex),
        0 if ex is None else len(expand), _p(out), _p(oshape)))
    assert tuple(int(v) for v in oshape[:len(shape)]) == tuple(shape)
    return out


def ref_time_transpose_contiguous(rows, cols, warmup, reps):
    secs = np.zeros(reps, np.float64)
    _check_ref(reference().mfref_time_transpose_contiguous(rows, cols, warmup, reps, _p(secs)))
    return secs


def ref_softmax(x, axis=-1, log=False):
    x = np.ascontiguousarray(x, np.float32)
    shape = np.array(x.shape, np.int64)
    out = np.empty_like(x)
    _check_ref(reference().mfref_softmax(_p(x), _p(shape), x.ndim, axis, int(log), _p(out)))
    return out


def ref_attention(q, k, v, mask=None, causal=False, scale=0.0):
    arrs = [np.ascontiguousarray(t, np.float32) for t in (q, k, v)]
    shapes = [np.array(t.shape, np.int64) for t in arrs]
    m = None if mask is None else np.ascontiguousarray(mask, np.uint8)
    ms = None if m is None else np.array(m.shape, np.int64)
    oshape = np.zeros(8, np.int64)
    ond = ctypes.c_int(0)
    args = []
    for t, sh in zip(arrs, shapes):
        args += [_p(t), _p(sh), t.ndim]
    lib_ = reference()
    _check_ref(lib_.mfref_attention(*args, _p(m), _p(ms), 0 if m is None else m.ndim, int(causal),
                                    scale, None, _p(oshape), ctypes.byref(ond)))
    out = np.empty(tuple(int(x) for x in oshape[: ond.value]), np.float32)
    _check_ref(lib_.mfref_attention(*args, _p(m), _p(ms), 0 if m is None else m.ndim, int(causal),
                                    scale, _p(out), _p(oshape), ctypes.byref(ond)))
    return out
