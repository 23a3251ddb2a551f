"""The reference's op API for the dense fp32 contraction path, on B200 tensors.

Same names, argument meaning and error behaviour as bakir004/mensurflow's public API
(include/mensurflow/ops/blas.hpp, elementwise.hpp): ``gemm``, ``matmul``,
``gemm_strided_batched``, ``gemv``, ``matvec``, ``bias_add``, ``relu``, ``gelu``, plus the fused
``linear`` (gemm + bias + activation in one kernel). The reference throws
``std::invalid_argument`` for bad arguments; here that is ``ValueError``.

Tensors are torch CUDA float32 tensors (torch provides device memory and streams only); every
op runs on the current stream through the C ABI in ``include/mfk.h``. Strided views (transposed,
sliced, expanded) go to the kernels as they are, with their strides — nothing is staged through
the host, unlike the reference's non-CPU path (src/core/tensor.cpp:224-229).
"""
from __future__ import annotations

import ctypes
from typing import Optional, Sequence

import numpy as np
import torch

from . import _lib
from ._lib import BatchDesc, GemmDesc, check

_ACTS = {None: _lib.ACT_NONE, "none": _lib.ACT_NONE, "relu": _lib.ACT_RELU,
         "gelu": _lib.ACT_GELU, "gelu_tanh": _lib.ACT_GELU_TANH}
_PRECISIONS = {None: _lib.PRECISION_DEFAULT, "default": _lib.PRECISION_DEFAULT,
               "3xtf32": _lib.PRECISION_3XTF32, "1xtf32": _lib.PRECISION_1XTF32}


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _require(t, op: str, name: str, dims: Optional[int] = None, at_least: bool = False):
    if t is None or not isinstance(t, torch.Tensor):
        raise ValueError(f"{op}: {name} is an undefined tensor")
    if dims is not None:
        bad = t.dim() < dims if at_least else t.dim() != dims
        if bad:
            what = f"at least {dims}-D" if at_least else f"{dims}-D"
            raise ValueError(f"{op}: {name} must be {what}, got shape {tuple(t.shape)}")


def _same(op: str, *ts):
    ts = [t for t in ts if t is not None]
    if any(t.dtype != ts[0].dtype for t in ts):
        raise ValueError(f"{op}: dtypes differ")
    if any(t.device != ts[0].device for t in ts):
        raise ValueError(f"{op}: tensors are on different devices; move one with Tensor::to()")


def _kernel_for(op: str, t: torch.Tensor):
    """The reference's NotImplemented (dispatcher.cpp:263-268): no kernel for this dtype/device."""
    if t.dtype != torch.float32:
        raise NotImplementedError(f"{op}: no kernel for dtype {t.dtype} on {t.device}")
    if t.device.type != "cuda":
        raise NotImplementedError(f"{op}: these kernels run on CUDA devices only")


def contiguous(x: torch.Tensor) -> torch.Tensor:
    """Tensor::contiguous() on the device (src/core/tensor.cpp:208-230): a contiguous tensor is
    returned as it is; a strided view (transposed, permuted, sliced with steps, expanded) is
    gathered into a new row-major tensor on the same device by one kernel
    (mfk_strided_copy_f32), where the reference stages non-CPU views through a host vector."""
    _require(x, "contiguous", "x")
    if x.is_contiguous():
        return x
    _kernel_for("contiguous", x)
    out = torch.empty(tuple(x.shape), dtype=x.dtype, device=x.device)
    nd = x.dim()
    shape = (ctypes.c_int64 * max(nd, 1))(*x.shape)
    strides = (ctypes.c_int64 * max(nd, 1))(*x.stride())
    with torch.cuda.device(x.device):
        check(_lib.lib().mfk_strided_copy_f32(x.data_ptr(), shape, strides, nd, out.data_ptr(),
                                              _stream()), "contiguous")
    return out


def copy(x: torch.Tensor) -> torch.Tensor:
    """A packed copy, as mensurflow::copy (src/ops/blas.cpp:106-117): a new tensor of x's shape
    on x's device that never shares x's storage. A strided x is gathered in the same launch (the
    reference packs it with contiguous() first and then copies again)."""
    _require(x, "copy", "x")
    _kernel_for("copy", x)
    if not x.is_contiguous():
        return contiguous(x)
    out = torch.empty(tuple(x.shape), dtype=x.dtype, device=x.device)
    if x.numel() == 0:
        return out
    with torch.cuda.device(x.device):
        check(_lib.lib().mfk_copy_f32(x.data_ptr(), out.data_ptr(), x.numel(), _stream()), "copy")
    return out


def to(x: torch.Tensor, device) -> torch.Tensor:
    """Tensor::to(device) (src/core/tensor.cpp:193-206). The same device returns x itself; a
    move between two CUDA devices is a device-to-device copy over NVLink (mfk_copy_peer) of the
    packed tensor, ordered after x's producers on x's device and before later work on the
    target's current stream, where the reference stages it through a host vector. A move to or
    from the host is a plain host copy (the reference's copy_to_host / copy_from_host)."""
    _require(x, "to", "x")
    target = torch.device(device)
    if target.type == "cuda" and target.index is None:
        target = torch.device("cuda", torch.cuda.current_device())
    if target == x.device:
        return x
    if target.type != "cuda" or x.device.type != "cuda":
        return x.to(target).contiguous() if target.type == "cpu" else x.contiguous().to(target)
    _kernel_for("to", x)
    src = contiguous(x)
    out = torch.empty(tuple(x.shape), dtype=x.dtype, device=target)
    if x.numel() == 0:
        return out
    src_stream = torch.cuda.current_stream(x.device)
    with torch.cuda.device(x.device):
        check(_lib.lib().mfk_copy_peer(out.data_ptr(), target.index, src.data_ptr(),
                                       x.device.index, src.numel() * src.element_size(),
                                       src_stream.cuda_stream), "to")
    done = torch.cuda.Event()
    done.record(src_stream)
    torch.cuda.current_stream(target).wait_event(done)
    return out


def set_default_precision(precision: str) -> None:
    """Process-wide GEMM precision ("3xtf32", the default, or "1xtf32")."""
    check(_lib.lib().mfk_set_default_precision(_PRECISIONS[precision]), "set_default_precision")


def get_default_precision() -> str:
    return {0: "3xtf32", 1: "1xtf32"}[_lib.lib().mfk_get_default_precision()]


def _gemm_desc(a_op, b_op, out, alpha, c_in, beta, bias, act, precision) -> GemmDesc:
    """a_op: op(A) [m,k] view, b_op: op(B) [k,n] view, out: [m,n] with unit column stride."""
    d = GemmDesc()
    d.a, d.a_rs, d.a_cs = _ptr(a_op), a_op.stride(0), a_op.stride(1)
    d.b, d.b_rs, d.b_cs = _ptr(b_op), b_op.stride(0), b_op.stride(1)
    if c_in is not None:
        d.c_in, d.c_in_rs, d.c_in_cs = _ptr(c_in), c_in.stride(0), c_in.stride(1)
    d.c, d.ldc = _ptr(out), out.stride(0)
    d.m, d.n, d.k = out.shape[0], out.shape[1], a_op.shape[1]
    d.alpha, d.beta = float(alpha), float(beta)
    d.bias = _ptr(bias)
    d.activation = _ACTS[act]
    d.precision = _PRECISIONS[precision]
    return d


# Input bytes per block of the host-tensor pipelines' default schedules (gemm's row blocks,
# attention's batch blocks).
_GEMM_BLOCK_BYTES = 64 << 20
_ATTENTION_BLOCK_BYTES = 192 << 20


def _block_bounds(total: int, unit_bytes: int, align: int, chunks: Optional[int],
                  block_bytes: int = _GEMM_BLOCK_BYTES) -> list:
    """Boundaries of the blocks a host-tensor pipeline streams `total` units (rows, or batch
    entries) in. `chunks` given: that many equal blocks (multiples of `align` but the last).
    Default: blocks of about `block_bytes` of input each, and the last two blocks' worth cut into
    halves down to `align` units, because the last block's product and its copy back are the part
    of the step no transfer overlaps. Measured on B200 through the host link: C2 (8192^3, 0.8 GB
    in, 0.27 GB out) 32 equal blocks 16.4-16.5 ms per step, 16 equal blocks 16.3, eight 64 MB
    blocks without the tapered end 16.6-16.9, seven and then 512 + 256 + 128 + 128 rows
    15.9-16.3; C4 attention (1.5 GB in, 0.5 GB out) 16 equal blocks 32.0 ms, tapered blocks of
    64 / 128 / 192 / 256 MB 32.2 / 31.4 / 31.2 / 31.2. Copies of 8 MB move at ~43 GB/s beside
    the other direction, 32-64 MB ones at ~50."""
    if chunks is not None:
        n = max(1, min(chunks, total))
        return sorted(set([round(i * total / n) // align * align for i in range(n)] + [total]))
    block = max(align, (block_bytes // max(1, unit_bytes)) // align * align)
    bounds, pos = [0], 0
    while total - pos > 2 * block:
        pos += block
        bounds.append(pos)
    while pos < total:
        rest = total - pos
        pos += rest if rest <= align else max(align, (rest // 2) // align * align)
        bounds.append(pos)
    return bounds


def _gemm_from_host(a, b, alpha, c, beta, transpose_a, transpose_b, bias, activation, precision,
                    out, chunks):
    """Execution::GPU on host-resident tensors, as the reference's run_on does for data that lives
    elsewhere (src/core/dispatcher.cpp:308-323: copy the inputs to the device, run, copy the
    result back) — pipelined: op(B) and the bias go first, then row blocks of op(A) and C stream
    in on one stream, are multiplied on the caller's stream and stream back on a third, so the
    transfers overlap each other and the math. Returns a host tensor; the copies are complete when
    this returns (the reference's copy_d2h waits the same way)."""
    dev = torch.device("cuda", torch.cuda.current_device())
    left = a.t() if transpose_a else a
    right = b.t() if transpose_b else b
    m, k = left.shape
    n = right.shape[1]
    if out is None:
        out = torch.empty((m, n), dtype=torch.float32, pin_memory=True)
    compute = torch.cuda.current_stream(dev)
    copy_in, copy_out = _copy_streams(dev)
    copy_in.wait_stream(compute)
    with torch.cuda.stream(copy_in):
        d_b = b.to(dev, non_blocking=True)
        d_bias = bias.to(dev, non_blocking=True) if bias is not None else None
    right_d = d_b.t() if transpose_b else d_b
    d_out = torch.empty((m, n), dtype=torch.float32, device=dev)
    # row blocks of op(A) are contiguous host slices only when A is not transposed
    if transpose_a or m < 512:
        bounds = [0, m]
    else:
        bounds = _block_bounds(m, 4 * (k + (n if c is not None else 0)), 128,
                               None if chunks is None else min(chunks, m // 256))
    nchunks = len(bounds) - 1
    # In 3xTF32 every product splits op(B) first; with several row blocks it is split once, as
    # soon as it has arrived, and shared (bit-identical to splitting it for each block).
    split_b = None
    if nchunks > 1 and k > 0 and n > 0 and \
            (get_default_precision() if precision in (None, "default") else precision) == "3xtf32":
        b_ready = torch.cuda.Event()
        b_ready.record(copy_in)
        compute.wait_event(b_ready)
        split_b = pack_b(right_d, precision="3xtf32")
    d_a = torch.empty_like(left, device=dev) if not transpose_a else None
    d_c = torch.empty((m, n), dtype=torch.float32, device=dev) if c is not None else None
    for i in range(nchunks):
        r0, r1 = bounds[i], bounds[i + 1]
        if r1 <= r0:
            continue
        with torch.cuda.stream(copy_in):
            if transpose_a:
                a_blk = a.to(dev, non_blocking=True).t()
            else:
                d_a[r0:r1].copy_(a[r0:r1], non_blocking=True)
                a_blk = d_a[r0:r1]
            c_blk = None
            if d_c is not None:
                d_c[r0:r1].copy_(c[r0:r1], non_blocking=True)
                c_blk = d_c[r0:r1]
        ready = torch.cuda.Event()
        ready.record(copy_in)
        compute.wait_event(ready)
        if split_b is not None:
            gemm_prepacked(a_blk, split_b, alpha, c_blk, beta, bias=d_bias,
                           activation=activation, precision="3xtf32", out=d_out[r0:r1])
        else:
            gemm(a_blk, right_d, alpha, c_blk, beta, False, False, bias=d_bias,
                 activation=activation, precision=precision, out=d_out[r0:r1])
        done = torch.cuda.Event()
        done.record(compute)
        copy_out.wait_event(done)
        with torch.cuda.stream(copy_out):
            out[r0:r1].copy_(d_out[r0:r1], non_blocking=True)
    # the device buffers stay alive until the copies that read them have finished
    for t in (d_a, d_c, d_b, d_bias, d_out):
        if t is not None:
            t.record_stream(copy_out)
            t.record_stream(copy_in)
    copy_out.synchronize()
    if split_b is not None:
        split_b.free()  # every product that read it has finished
    return out


_COPY_STREAMS = {}


def _copy_streams(dev: torch.device):
    """The two copy streams of the host-tensor path on `dev` (made once per device)."""
    if dev not in _COPY_STREAMS:
        _COPY_STREAMS[dev] = (torch.cuda.Stream(dev), torch.cuda.Stream(dev))
    return _COPY_STREAMS[dev]


def gemm(a: torch.Tensor, b: torch.Tensor, alpha: float = 1.0, c: Optional[torch.Tensor] = None,
         beta: float = 0.0, transpose_a: bool = False, transpose_b: bool = False, *,
         bias: Optional[torch.Tensor] = None, activation: Optional[str] = None,
         precision: Optional[str] = None, out: Optional[torch.Tensor] = None,
         execution: str = "auto", chunks: Optional[int] = None) -> torch.Tensor:
    """alpha * op(a) @ op(b) + beta * c, as mensurflow::gemm (blas.hpp:59, blas.cpp:234-262),
    in ONE kernel; `bias` and `activation` fuse the following bias_add/relu/gelu.

    `execution` follows the reference's Execution (include/mensurflow/execution.hpp): with CUDA
    tensors the op runs on their device; with host tensors "gpu" streams them through the current
    CUDA device and returns a host tensor, while "auto"/"cpu" have no kernel here
    (NotImplementedError — the reference's CPU path is not part of this library)."""
    _require(a, "gemm", "a", 2)
    _require(b, "gemm", "b", 2)
    if c is not None:
        _require(c, "gemm", "c")
    _same("gemm", a, b, c, bias)
    left = a.t() if transpose_a else a
    right = b.t() if transpose_b else b
    m, k = left.shape
    if right.shape[0] != k:
        raise ValueError(f"gemm: inner dimensions differ ({tuple(left.shape)} times "
                         f"{tuple(right.shape)})")
    n = right.shape[1]
    if c is not None and tuple(c.shape) != (m, n):
        raise ValueError("gemm: c shape does not match result")
    if c is None and beta != 0.0:
        raise ValueError("gemm: beta requires c")
    if bias is not None and (bias.dim() != 1 or bias.shape[0] != n):
        raise ValueError(f"gemm: bias must be [{n}], got {tuple(bias.shape)}")
    if activation not in _ACTS:
        raise ValueError(f"gemm: unknown activation {activation!r}")
    if execution not in ("auto", "cpu", "gpu"):
        raise ValueError(f"gemm: unknown execution {execution!r}")
    if a.device.type == "cpu" and execution == "gpu" and a.dtype == torch.float32:
        if out is not None and (tuple(out.shape) != (m, n) or out.device.type != "cpu"):
            raise ValueError("gemm: out must be a host [m, n] tensor for host inputs")
        return _gemm_from_host(a, b, alpha, c if beta != 0.0 else None, beta, transpose_a,
                               transpose_b, bias, activation, precision, out, chunks)
    _kernel_for("gemm", a)
    if bias is not None:
        bias = contiguous(bias)
    if out is None:
        out = torch.empty((m, n), dtype=torch.float32, device=a.device)
    elif tuple(out.shape) != (m, n) or out.stride(1) != 1:
        raise ValueError("gemm: out must be [m, n] with unit column stride")
    desc = _gemm_desc(left, right, out, alpha, c if beta != 0.0 else None, beta, bias,
                      activation, precision)
    check(_lib.lib().mfk_gemm_f32(ctypes.byref(desc), _stream()), "gemm")
    return out


class PackedB:
    """B split once for many products: the device analogue of the reference's cpu::PackedB
    (src/backends/cpu/ops/gemm/gemm_packed.hpp:147-191). Holds op(B) as K-major tf32 panels —
    (hi, lo) for 3xTF32, rounded values for 1xTF32 — in device memory it owns; `gemm_prepacked`
    and `linear` use it in place of B and skip B's split pass. Build it with `pack_b`."""

    def __init__(self, handle: int, k: int, n: int, precision: int, device: torch.device):
        self._handle = handle
        self._k, self._n = k, n
        self._precision = precision
        self.device = device

    def depth(self) -> int:
        """k: rows of B."""
        return self._k

    def cols(self) -> int:
        """n: columns of B."""
        return self._n

    @property
    def precision(self) -> str:
        return "3xtf32" if self._precision == _lib.PRECISION_3XTF32 else "1xtf32"

    def empty(self) -> bool:
        """True when it holds no values: B had no rows or columns, or the object was freed."""
        return self._handle is None or self._k == 0 or self._n == 0

    def free(self) -> None:
        """Releases the device copy now (device-synchronising), leaving an empty object."""
        if self._handle is not None:
            h, self._handle = self._handle, None
            self._k = self._n = 0
            check(_lib.lib().mfk_packed_b_free(h), "PackedB.free")

    def __del__(self):
        try:
            self.free()
        except Exception:  # interpreter shutdown: the driver reclaims the memory
            pass


def pack_b(b: torch.Tensor, *, transpose: bool = False,
           precision: Optional[str] = None) -> PackedB:
    """Split B [k, n] (or, with `transpose`, the weights stored [n, k]) once, as pack_b_f32
    (gemm_packed.hpp:188): any strides; `b` may be freed or changed afterwards. The precision is
    fixed at packing time (None: the library default then); a 3xTF32 pack serves both
    precisions, a 1xTF32 pack only 1xTF32."""
    _require(b, "pack_b", "b", 2)
    _kernel_for("pack_b", b)
    op_b = b.t() if transpose else b
    k, n = op_b.shape
    handle = ctypes.c_void_p()
    check(_lib.lib().mfk_pack_b_f32(_ptr(op_b) if op_b.numel() else None, op_b.stride(0),
                                    op_b.stride(1), k, n, _PRECISIONS[precision], _stream(),
                                    ctypes.byref(handle)), "pack_b")
    prec = ctypes.c_int32()
    check(_lib.lib().mfk_packed_b_shape(handle, None, None, ctypes.byref(prec)), "pack_b")
    return PackedB(handle.value, k, n, prec.value, b.device)


def gemm_prepacked(a: torch.Tensor, packed: PackedB, alpha: float = 1.0,
                   c: Optional[torch.Tensor] = None, beta: float = 0.0,
                   transpose_a: bool = False, *, bias: Optional[torch.Tensor] = None,
                   activation: Optional[str] = None, precision: Optional[str] = None,
                   out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """gemm with a pre-split B: act(alpha * op(a) @ B + beta * c + bias), as
    matmul_f32_prepacked (gemm_packed.hpp:191) plus gemm's epilogue. `precision` None means the
    pack's own precision."""
    if not isinstance(packed, PackedB):
        raise TypeError("gemm_prepacked: packed must come from pack_b")
    _require(a, "gemm_prepacked", "a", 2)
    if c is not None:
        _require(c, "gemm_prepacked", "c")
    _same("gemm_prepacked", a, c, bias)
    _kernel_for("gemm_prepacked", a)
    if packed.device != a.device:
        raise ValueError("gemm_prepacked: the pack lives on another device")
    if packed._handle is None:
        raise ValueError("gemm_prepacked: the pack was freed")
    left = a.t() if transpose_a else a
    m, k = left.shape
    n = packed.cols()
    if k != packed.depth():
        raise ValueError(f"gemm_prepacked: inner dimensions differ ({tuple(left.shape)} times "
                         f"[{packed.depth()}, {n}])")
    if c is not None and tuple(c.shape) != (m, n):
        raise ValueError("gemm_prepacked: c shape does not match result")
    if c is None and beta != 0.0:
        raise ValueError("gemm_prepacked: beta requires c")
    if bias is not None and (bias.dim() != 1 or bias.shape[0] != n):
        raise ValueError(f"gemm_prepacked: bias must be [{n}], got {tuple(bias.shape)}")
    if activation not in _ACTS:
        raise ValueError(f"gemm_prepacked: unknown activation {activation!r}")
    if bias is not None:
        bias = contiguous(bias)
    if out is None:
        out = torch.empty((m, n), dtype=torch.float32, device=a.device)
    elif tuple(out.shape) != (m, n) or out.stride(1) != 1:
        raise ValueError("gemm_prepacked: out must be [m, n] with unit column stride")
    if m == 0 or n == 0:
        return out
    d = GemmDesc()
    d.a, d.a_rs, d.a_cs = _ptr(left), left.stride(0), left.stride(1)
    if c is not None and beta != 0.0:
        d.c_in, d.c_in_rs, d.c_in_cs = _ptr(c), c.stride(0), c.stride(1)
    d.c, d.ldc = _ptr(out), out.stride(0)
    d.m, d.n, d.k = m, n, k
    d.alpha, d.beta = float(alpha), float(beta)
    d.bias = _ptr(bias)
    d.activation = _ACTS[activation]
    d.precision = (packed._precision if precision is None else _PRECISIONS[precision])
    check(_lib.lib().mfk_gemm_prepacked_f32(ctypes.byref(d), packed._handle, _stream()),
          "gemm_prepacked")
    return out


def matmul(a: torch.Tensor, b: torch.Tensor, *, precision: Optional[str] = None) -> torch.Tensor:
    """[M,K] @ [K,N] as mensurflow::matmul (blas.hpp:55, blas.cpp:186-232)."""
    _require(a, "matmul", "a", 2)
    _require(b, "matmul", "b", 2)
    _same("matmul", a, b)
    if b.shape[0] != a.shape[1]:
        raise ValueError(f"matmul: inner dimensions differ ({tuple(a.shape)} times "
                         f"{tuple(b.shape)})")
    return gemm(a, b, precision=precision)


def linear(x: torch.Tensor, w, bias: Optional[torch.Tensor] = None,
           activation: Optional[str] = None, *, transpose_w: bool = False,
           precision: Optional[str] = None) -> torch.Tensor:
    """act(x @ op(w) + bias) in one kernel: the fused form of matmul + bias_add (+ relu/gelu).
    `w` may be a PackedB (weights split once by `pack_b`)."""
    if isinstance(w, PackedB):
        if transpose_w:
            raise ValueError("linear: a PackedB already holds op(w); pack with transpose=True")
        return gemm_prepacked(x, w, bias=bias, activation=activation, precision=precision)
    return gemm(x, w, transpose_b=transpose_w, bias=bias, activation=activation,
                precision=precision)


def bias_grad(grad: torch.Tensor) -> torch.Tensor:
    """The bias gradient of bias_add: column sums of `grad` [batch, features] over the rows,
    accumulated in fp32 in row order — bit-identical to the reference's backward closure
    (src/ops/elementwise.cpp:263-283), which runs this loop on the host; here one device kernel."""
    _require(grad, "bias_grad", "grad", 2)
    _kernel_for("bias_grad", grad)
    rows, cols = grad.shape
    g = grad if grad.stride(1) == 1 and (rows <= 1 or grad.stride(0) >= cols) else contiguous(grad)
    out = torch.empty(cols, dtype=torch.float32, device=grad.device)
    ld = g.stride(0) if rows > 1 else cols
    check(_lib.lib().mfk_bias_grad_f32(_ptr(g) if g.numel() else None, rows, cols, ld,
                                       _ptr(out) if cols else None, _stream()), "bias_grad")
    return out


def matmul_backward(grad: torch.Tensor, a: torch.Tensor, b: torch.Tensor, *,
                    need_a: bool = True, need_b: bool = True,
                    precision: Optional[str] = None):
    """(dA, dB) for C = A @ B: dA = grad @ B^T and dB = A^T @ grad, the products matmul's recorded
    backward makes (src/ops/blas.cpp:220-230). The transposes are stride swaps read in place by
    the same tensor-core GEMM (the reference's op layer copies non-contiguous CUDA views through
    the host first, tensor.cpp:224-229). A gradient that is not needed is None."""
    _require(grad, "matmul_backward", "grad", 2)
    _require(a, "matmul_backward", "a", 2)
    _require(b, "matmul_backward", "b", 2)
    _same("matmul_backward", grad, a, b)
    m, k = a.shape
    if b.shape[0] != k or tuple(grad.shape) != (m, b.shape[1]):
        raise ValueError(f"matmul_backward: shapes {tuple(grad.shape)}, {tuple(a.shape)}, "
                         f"{tuple(b.shape)} do not form C = A @ B")
    da = gemm(grad, b, transpose_b=True, precision=precision) if need_a else None
    db = gemm(a, grad, transpose_a=True, precision=precision) if need_b else None
    return da, db


def linear_backward(grad: torch.Tensor, x: torch.Tensor, w: torch.Tensor, *,
                    has_bias: bool = True, transpose_w: bool = False,
                    precision: Optional[str] = None):
    """(dx, dw, dbias) for y = x @ op(w) + bias (no activation): the matmul backward products and
    the bias reduction; dw has w's own layout ([n, k] when transpose_w). dbias is None without a
    bias."""
    w_op = w.t() if transpose_w else w
    dx, dw = matmul_backward(grad, x, w_op, need_b=not transpose_w, precision=precision)
    if transpose_w:
        dw = gemm(grad, x, transpose_a=True, precision=precision)   # (x^T grad)^T = grad^T x
    return dx, dw, (bias_grad(grad) if has_bias else None)


def _broadcast_shapes(op: str, x: Sequence[int], y: Sequence[int]):
    try:
        return tuple(torch.broadcast_shapes(tuple(x), tuple(y)))
    except RuntimeError:
        raise ValueError(f"{op}: batch shapes {tuple(x)} and {tuple(y)} do not broadcast")


def _odometer_offsets(t: torch.Tensor, batch_shape) -> np.ndarray:
    """Element offset of each matrix of an expanded view, last batch dim fastest — the walk of
    the reference's gemm_batched_kernel (src/backends/cpu/backend.cpp:251-270)."""
    nd = len(batch_shape)
    if nd == 0:
        return np.zeros(1, np.int64)
    idx = np.indices(batch_shape).reshape(nd, -1).T  # row-major order = last dim fastest
    strides = np.array(t.stride()[:nd], np.int64)
    return (idx.astype(np.int64) * strides).sum(axis=1).astype(np.int64)


def gemm_strided_batched(a: torch.Tensor, b: torch.Tensor, alpha: float = 1.0,
                         c: Optional[torch.Tensor] = None, beta: float = 0.0,
                         transpose_a: bool = False, transpose_b: bool = False, *,
                         precision: Optional[str] = None) -> torch.Tensor:
    """Batched gemm with NumPy batch broadcasting, as mensurflow::gemm_strided_batched
    (blas.hpp:75, blas.cpp:297-394)."""
    op = "gemm_strided_batched"
    for t, name in ((a, "a"), (b, "b")):
        _require(t, op, name, 2, at_least=True)
    _same(op, a, b, c)
    if c is None and beta != 0.0:
        raise ValueError(f"{op}: beta requires c")
    left = a.transpose(-2, -1) if transpose_a else a
    right = b.transpose(-2, -1) if transpose_b else b
    m, k, n = left.shape[-2], left.shape[-1], right.shape[-1]
    if right.shape[-2] != k:
        raise ValueError(f"{op}: inner dimensions differ ({tuple(left.shape)} times "
                         f"{tuple(right.shape)})")
    batch_shape = _broadcast_shapes(op, left.shape[:-2], right.shape[:-2])
    out_shape = batch_shape + (m, n)
    initial = None
    if c is not None:
        ok = c.dim() <= len(out_shape)
        if ok:
            try:
                ok = tuple(torch.broadcast_shapes(tuple(c.shape), out_shape)) == out_shape
            except RuntimeError:
                ok = False
        if not ok:
            raise ValueError(f"{op}: c has shape {tuple(c.shape)}, which does not broadcast to "
                             f"{out_shape}")
        if beta != 0.0:
            initial = c.expand(out_shape)
    _kernel_for(op, a)
    out = torch.empty(out_shape, dtype=torch.float32, device=a.device)
    batch = int(np.prod(batch_shape)) if batch_shape else 1
    if out.numel() == 0:
        return out
    lv = left.expand(batch_shape + (m, k))
    rv = right.expand(batch_shape + (k, n))
    a_off = _odometer_offsets(lv, batch_shape)
    b_off = _odometer_offsets(rv, batch_shape)
    bd = BatchDesc()
    bd.batch = batch
    bd.a_offsets = a_off.ctypes.data
    bd.b_offsets = b_off.ctypes.data
    bd.c_stride = m * n
    zero = (0,) * len(batch_shape)
    desc = _gemm_desc(lv[zero], rv[zero], out.view(-1, m, n)[0], alpha, None, 0.0, None, None,
                      precision)
    # Base pointers are the expanded views' first elements; the offsets are relative to them.
    desc.a = lv.data_ptr()
    desc.b = rv.data_ptr()
    if initial is not None:
        c_off = _odometer_offsets(initial, batch_shape)
        even = batch <= 1 or bool(np.all(np.diff(c_off) == c_off[1] - c_off[0]))
        if not even:
            initial = contiguous(initial)  # the reference packs c the same way (blas.cpp:361)
            c_off = _odometer_offsets(initial, batch_shape)
        desc.c_in = initial.data_ptr()
        desc.c_in_rs, desc.c_in_cs = initial.stride(-2), initial.stride(-1)
        desc.beta = float(beta)
        bd.c_in_stride = int(c_off[1] - c_off[0]) if batch > 1 else 0
    check(_lib.lib().mfk_gemm_strided_batched_f32(ctypes.byref(desc), ctypes.byref(bd), _stream()),
          op)
    return out


def gemv(a: torch.Tensor, x: torch.Tensor, alpha: float = 1.0, y: Optional[torch.Tensor] = None,
         beta: float = 0.0, transpose_a: bool = False) -> torch.Tensor:
    """alpha * op(a) x + beta * y, sums in double, as mensurflow::gemv (blas.hpp:40)."""
    _require(a, "gemv", "a", 2)
    _require(x, "gemv", "x", 1)
    if y is None and beta != 0.0:
        raise ValueError("gemv: beta requires an output vector")
    _same("gemv", a, x, y)
    rows, cols = a.shape
    n_in, n_out = (rows, cols) if transpose_a else (cols, rows)
    if x.shape[0] != n_in:
        raise ValueError("gemv: input length does not match matrix dimensions")
    if y is not None and y.shape[0] != n_out:
        raise ValueError("gemv: output length does not match matrix dimensions")
    _kernel_for("gemv", a)
    if a.stride(1) != 1 or (rows > 1 and a.stride(0) < cols):
        a = contiguous(a)
    out = torch.empty(n_out, dtype=torch.float32, device=a.device)
    y0 = contiguous(y) if y is not None else None
    check(_lib.lib().mfk_gemv_f32(a.data_ptr(), rows, cols, max(a.stride(0), cols),
                                  1 if transpose_a else 0, x.data_ptr(), x.stride(0) or 1,
                                  float(alpha), float(beta), _ptr(y0), out.data_ptr(), _stream()),
          "gemv")
    return out


def matvec(a: torch.Tensor, x: torch.Tensor) -> torch.Tensor:
    """[M,K] @ [K] as mensurflow::matvec (blas.hpp:35)."""
    _require(a, "matvec", "a", 2)
    _require(x, "matvec", "x", 1)
    _same("matvec", a, x)
    if x.shape[0] != a.shape[1]:
        raise ValueError(f"matvec: inner dimensions differ ({tuple(a.shape)} times "
                         f"{tuple(x.shape)})")
    return gemv(a, x)


def _bias_act(x: torch.Tensor, bias: Optional[torch.Tensor], act: int, op: str) -> torch.Tensor:
    _kernel_for(op, x)
    x = contiguous(x)
    out = torch.empty_like(x)
    cols = x.shape[-1] if x.dim() > 0 else 1
    rows = x.numel() // cols if cols else 0
    check(_lib.lib().mfk_bias_act_f32(x.data_ptr(), _ptr(bias), out.data_ptr(), rows, cols, act,
                                      _stream()), op)
    return out


def bias_add(x: torch.Tensor, bias: torch.Tensor) -> torch.Tensor:
    """x [batch, features] + bias [features], as mensurflow::bias_add (elementwise.hpp:43,
    elementwise.cpp:251-284)."""
    _require(x, "bias_add", "x")
    _require(bias, "bias_add", "bias")
    if x.dim() != 2 or bias.dim() != 1 or bias.shape[0] != x.shape[1]:
        raise ValueError(f"bias_add: expected x [batch, features] and bias [features], got "
                         f"{tuple(x.shape)} and {tuple(bias.shape)}")
    _same("bias_add", x, bias)
    return _bias_act(x, contiguous(bias), _lib.ACT_NONE, "bias_add")


def relu(x: torch.Tensor) -> torch.Tensor:
    _require(x, "relu", "x")
    _same("relu", x)
    return _bias_act(x, None, _lib.ACT_RELU, "relu")


def gelu(x: torch.Tensor, approximate: bool = False) -> torch.Tensor:
    """Exact 0.5*v*erfc(-v/sqrt 2) (or the tanh form), as mensurflow::gelu (elementwise.hpp:62)."""
    _require(x, "gelu", "x")
    _same("gelu", x)
    return _bias_act(x, None, _lib.ACT_GELU_TANH if approximate else _lib.ACT_GELU, "gelu")


def _binary(a: torch.Tensor, b: torch.Tensor, code: int, op: str) -> torch.Tensor:
    """Elementwise a op b with NumPy broadcasting, as the reference's binary_op
    (src/ops/elementwise.cpp:158-225): broadcast inputs are expanded and packed to the result's
    shape, then one kernel pass computes it."""
    _require(a, op, "a")
    _require(b, op, "b")
    if a.dtype != b.dtype:
        raise ValueError(f"{op}: dtypes differ ({a.dtype} and {b.dtype})")
    _same(op, a, b)
    try:
        shape = tuple(torch.broadcast_shapes(tuple(a.shape), tuple(b.shape)))
    except RuntimeError:
        raise ValueError(f"{op}: shapes {tuple(a.shape)} and {tuple(b.shape)} do not broadcast")
    _kernel_for(op, a)
    x = contiguous(a.expand(shape))
    y = contiguous(b.expand(shape))
    out = torch.empty(shape, dtype=torch.float32, device=a.device)
    check(_lib.lib().mfk_binary_f32(code, x.data_ptr(), y.data_ptr(), out.data_ptr(), out.numel(),
                                    _stream()), op)
    return out


def add(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """a + b, as mensurflow::add (elementwise.hpp; src/ops/elementwise.cpp:227)."""
    return _binary(a, b, _lib.BINARY_ADD, "add")


def sub(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """a - b, as mensurflow::sub (src/ops/elementwise.cpp:231)."""
    return _binary(a, b, _lib.BINARY_SUB, "sub")


def mul(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """a * b, as mensurflow::mul (src/ops/elementwise.cpp:235)."""
    return _binary(a, b, _lib.BINARY_MUL, "mul")


def div(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """a / b, as mensurflow::div (src/ops/elementwise.cpp:239)."""
    return _binary(a, b, _lib.BINARY_DIV, "div")


def scal(alpha: float, x: torch.Tensor) -> torch.Tensor:
    """alpha * x for a 1-D x, as mensurflow::scal (src/ops/blas.cpp:70-79)."""
    _require(x, "scal", "x", dims=1)
    _same("scal", x)
    _kernel_for("scal", x)
    xx = contiguous(x)
    out = torch.empty_like(xx)
    check(_lib.lib().mfk_scal_f32(float(alpha), xx.data_ptr(), out.data_ptr(), xx.numel(),
                                  _stream()), "scal")
    return out


def dot(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """sum(a * b) of two 1-D tensors as a 0-d tensor on their device, as mensurflow::dot
    (src/ops/blas.cpp:41-68): products summed in double, rounded once."""
    _require(a, "dot", "a", dims=1)
    _require(b, "dot", "b", dims=1)
    if a.dtype != b.dtype:
        raise ValueError(f"dot: dtypes differ ({a.dtype} and {b.dtype})")
    _same("dot", a, b)
    if a.shape[0] != b.shape[0]:
        raise ValueError(f"dot: lengths differ ({a.shape[0]} and {b.shape[0]})")
    _kernel_for("dot", a)
    x, y = contiguous(a), contiguous(b)
    out = torch.empty((), dtype=torch.float32, device=a.device)
    check(_lib.lib().mfk_dot_f32(x.data_ptr(), y.data_ptr(), x.numel(), out.data_ptr(),
                                 _stream()), "dot")
    return out


def _softmax(x: torch.Tensor, axis: int, log: bool, op: str) -> torch.Tensor:
    _require(x, op, "input")
    if x.dtype != torch.float32:
        raise ValueError(f"{op}: input must be F32, got {x.dtype}")
    rank = x.dim()
    extent = rank if rank else 1
    ax = axis + extent if axis < 0 else axis
    if not 0 <= ax < extent:
        raise ValueError(f"{op}: axis {axis} is out of range for a {rank}-d tensor")
    _kernel_for(op, x)
    x = contiguous(x)
    shape = tuple(x.shape) if rank else (1,)
    outer = int(np.prod(shape[:ax])) if ax else 1
    inner = int(np.prod(shape[ax + 1:])) if ax + 1 < len(shape) else 1
    out = torch.empty_like(x)
    check(_lib.lib().mfk_softmax_f32(x.data_ptr(), out.data_ptr(), outer, shape[ax], inner,
                                     1 if log else 0, _stream()), op)
    return out


def softmax(x: torch.Tensor, axis: int = -1) -> torch.Tensor:
    """exp(x - max) / sum(exp(x - max)) along `axis`, as mensurflow::softmax (softmax.hpp:20):
    sums in double, an all -inf line gives zeros, a NaN poisons its line."""
    return _softmax(x, axis, False, "softmax")


def log_softmax(x: torch.Tensor, axis: int = -1) -> torch.Tensor:
    """x - logsumexp(x) along `axis`, as mensurflow::log_softmax (softmax.hpp:24)."""
    return _softmax(x, axis, True, "log_softmax")


def where(condition: torch.Tensor, x: torch.Tensor, y: torch.Tensor) -> torch.Tensor:
    """condition ? x : y with NumPy broadcasting, as mensurflow::where (elementwise.hpp:141)."""
    if x is None or y is None or not isinstance(x, torch.Tensor) or not isinstance(y, torch.Tensor):
        raise ValueError("where: undefined value tensor")
    if condition is None or not isinstance(condition, torch.Tensor):
        raise ValueError("where: undefined condition tensor")
    if condition.dtype != torch.bool:
        raise ValueError("where: condition must have Bool dtype")
    if x.dtype != y.dtype:
        raise ValueError("where: dtypes differ")
    if condition.device != x.device or x.device != y.device:
        raise ValueError("where: condition and values must be on the same device")
    try:
        shape = tuple(torch.broadcast_shapes(tuple(x.shape), tuple(y.shape), tuple(condition.shape)))
    except RuntimeError as e:
        raise ValueError(f"where: {e}")
    _kernel_for("where", x)
    xx = contiguous(x.expand(shape))
    yy = contiguous(y.expand(shape))
    cc = condition.expand(shape).contiguous()
    out = torch.empty(shape, dtype=torch.float32, device=x.device)
    check(_lib.lib().mfk_where_f32(cc.data_ptr(), xx.data_ptr(), yy.data_ptr(), out.data_ptr(),
                                   out.numel(), _stream()), "where")
    return out


def _attention_from_host(q, k, v, mask, causal, scale, precision, out, chunks, fused=None):
    """Execution::GPU on host-resident q, k, v (as gemm's host path): the batch is cut into
    chunks whose q, k, v stream in on one stream, are attended on the caller's stream and stream
    back on a third, so the copies overlap each other and the math. q, k and v must share their
    leading (batch) shape; a mask must broadcast over the batch (at most 2-D, or leading dims of
    1). Returns a host tensor; the copies are complete when this returns."""
    dev = torch.device("cuda", torch.cuda.current_device())
    lead = tuple(q.shape[:-2])
    if tuple(k.shape[:-2]) != lead or tuple(v.shape[:-2]) != lead:
        raise ValueError("attention: host tensors with execution='gpu' need q, k and v with the "
                         "same batch shape")
    if mask is not None and mask.dim() > 2 and any(s != 1 for s in mask.shape[:-2]):
        raise ValueError("attention: host tensors with execution='gpu' take a mask that is the "
                         "same for every batch entry")
    queries, depth_v = q.shape[-2], v.shape[-1]
    batch = int(np.prod(lead)) if lead else 1
    q3 = q.reshape(batch, queries, q.shape[-1])
    k3 = k.reshape(batch, k.shape[-2], k.shape[-1])
    v3 = v.reshape(batch, v.shape[-2], depth_v)
    if out is None:
        out = torch.empty(lead + (queries, depth_v), dtype=torch.float32, pin_memory=True)
    elif tuple(out.shape) != lead + (queries, depth_v) or out.device.type != "cpu":
        raise ValueError("attention: out must be a host tensor of the result's shape")
    o3 = out.view(batch, queries, depth_v)
    compute = torch.cuda.current_stream(dev)
    copy_in, copy_out = _copy_streams(dev)
    copy_in.wait_stream(compute)
    with torch.cuda.stream(copy_in):
        d_mask = mask.to(dev, non_blocking=True) if mask is not None else None
    entry_bytes = 4 * (q3.shape[1] * q3.shape[2] + k3.shape[1] * k3.shape[2] +
                       v3.shape[1] * v3.shape[2])
    bounds = _block_bounds(batch, entry_bytes, 1, chunks, _ATTENTION_BLOCK_BYTES)
    nchunks = len(bounds) - 1
    alive = []
    for i in range(nchunks):
        b0, b1 = bounds[i], bounds[i + 1]
        if b1 <= b0:
            continue
        with torch.cuda.stream(copy_in):
            dq = q3[b0:b1].to(dev, non_blocking=True)
            dk = k3[b0:b1].to(dev, non_blocking=True)
            dv = v3[b0:b1].to(dev, non_blocking=True)
        ready = torch.cuda.Event()
        ready.record(copy_in)
        compute.wait_event(ready)
        o = attention(dq, dk, dv, d_mask, causal, scale, precision=precision, fused=fused)
        done = torch.cuda.Event()
        done.record(compute)
        copy_out.wait_event(done)
        with torch.cuda.stream(copy_out):
            o3[b0:b1].copy_(o, non_blocking=True)
        alive.extend((dq, dk, dv, o))
    for t in alive + ([d_mask] if d_mask is not None else []):
        t.record_stream(copy_out)
        t.record_stream(copy_in)
    copy_out.synchronize()
    return out


FUSED_ATTENTION_HEAD_DIM = 128


def _mask_broadcasts(mask, scores_shape) -> bool:
    try:
        return tuple(torch.broadcast_shapes(tuple(mask.shape), tuple(scores_shape))) == \
            tuple(scores_shape)
    except RuntimeError:
        return False


def _keep_matrices(mask, scores_shape):
    """The Bool mask broadcast to the scores [..., Lq, Lk] as matrices [batch, Lq, Lk] with unit
    column stride: (tensor, batch stride in bytes (0 when one matrix serves all), row stride)."""
    queries, keys = scores_shape[-2], scores_shape[-1]
    batch = int(np.prod(scores_shape[:-2])) if len(scores_shape) > 2 else 1
    keep = mask.expand(scores_shape)
    flat = keep.reshape(batch, queries, keys) if keep.dim() > 2 else keep.reshape(1, queries, keys)
    if flat.stride(-1) != 1:
        flat = flat.contiguous()
    return flat, (flat.stride(0) if flat.shape[0] > 1 else 0), flat.stride(1)


def _fused_attention_eligible(q, k, v, mask, precision) -> bool:
    """The one-kernel path (mfk_attention_f32, or mfk_attention_masked_f32 with a Bool mask that
    broadcasts to the scores): q, k and v of one shape [..., L, 128] on a CUDA device, 3xTF32."""
    if q.device.type != "cuda" or q.dim() < 2:
        return False
    if mask is not None and (not isinstance(mask, torch.Tensor) or mask.dtype != torch.bool or
                             mask.device != q.device or
                             not _mask_broadcasts(mask, tuple(q.shape[:-1]) + (q.shape[-2],))):
        return False
    if tuple(q.shape) != tuple(k.shape) or tuple(q.shape) != tuple(v.shape):
        return False
    if q.shape[-1] != FUSED_ATTENTION_HEAD_DIM or q.shape[-2] == 0:
        return False
    code = _PRECISIONS[precision]
    if code == _lib.PRECISION_DEFAULT:
        code = _lib.lib().mfk_get_default_precision()
    return code == _lib.PRECISION_3XTF32


def _fused_attention(q, k, v, causal, scale, mask=None):
    _kernel_for("attention", q)
    qq, kk, vv = (contiguous(t) for t in (q, k, v))
    if any(t.data_ptr() % 16 for t in (qq, kk, vv)):
        qq, kk, vv = (t.clone() for t in (qq, kk, vv))
    out = torch.empty(tuple(q.shape), dtype=torch.float32, device=q.device)
    length, depth = q.shape[-2], q.shape[-1]
    heads = q.numel() // (length * depth)
    if mask is None:
        check(_lib.lib().mfk_attention_f32(qq.data_ptr(), kk.data_ptr(), vv.data_ptr(),
                                           out.data_ptr(), heads, length, depth,
                                           1 if causal else 0, float(scale), _stream()),
              "attention")
    else:
        keep, keep_bs, keep_rs = _keep_matrices(mask, tuple(q.shape[:-1]) + (length,))
        check(_lib.lib().mfk_attention_masked_f32(qq.data_ptr(), kk.data_ptr(), vv.data_ptr(),
                                                  keep.data_ptr(), keep_bs, keep_rs, 1,
                                                  out.data_ptr(), heads, length, depth,
                                                  1 if causal else 0, float(scale), _stream()),
              "attention")
        keep.record_stream(torch.cuda.current_stream(q.device))
    return out


def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
              mask: Optional[torch.Tensor] = None, causal: bool = False, scale: float = 0.0, *,
              precision: Optional[str] = None, execution: str = "auto",
              out: Optional[torch.Tensor] = None, chunks: Optional[int] = None,
              fused: Optional[bool] = None) -> torch.Tensor:
    """Scaled dot-product attention as mensurflow::attention (attention.hpp:21,
    src/ops/attention.cpp:48-98): scores = scale * q @ k^T (batched GEMM, scale in alpha), entries
    outside `mask` (Bool, broadcast to the scores) and, with `causal`, above the diagonal set to
    -inf, softmax over the keys, then weights @ v.

    Two device paths. Without a mask tensor, with q, k and v of one shape [..., L, 128] and
    3xTF32, one kernel computes the whole op (mfk_attention_f32: the scores stay on chip, the
    causal mask skips the key tiles above the diagonal; the softmax is evaluated online, so the
    result agrees with the composed path within the reference's 1e-4, not bit for bit; it is not
    for non-finite inputs). Otherwise, or with fused=False, the composed path: the batched GEMM,
    the masking fused into the softmax pass (one read and one write of the scores instead of the
    reference's where + softmax passes), the second batched GEMM. fused=True insists on the one
    kernel (ValueError when the inputs do not qualify).

    `execution` follows the reference's Execution: with host tensors "gpu" streams batch chunks
    through the current CUDA device and returns a host tensor (`out`, if given, receives it)."""
    if execution not in ("auto", "cpu", "gpu"):
        raise ValueError(f"attention: unknown execution {execution!r}")
    if (isinstance(q, torch.Tensor) and q.device.type == "cpu" and execution == "gpu" and
            all(isinstance(t, torch.Tensor) and t.device.type == "cpu" and
                t.dtype == torch.float32 and t.dim() >= 2 for t in (q, k, v))):
        if mask is not None and (not isinstance(mask, torch.Tensor) or mask.dtype != torch.bool):
            raise ValueError("attention: mask must be a defined Bool tensor")
        return _attention_from_host(q, k, v, mask, causal, scale, precision, out, chunks,
                                    fused)
    for t, name in ((q, "q"), (k, "k"), (v, "v")):
        if t is None or not isinstance(t, torch.Tensor):
            raise ValueError(f"attention: undefined {name}")
        if t.dtype != torch.float32:
            raise ValueError(f"attention: {name} must be F32, got {t.dtype}")
        if t.dim() < 2:
            raise ValueError(f"attention: {name} needs at least 2 dimensions, got "
                             f"{tuple(t.shape)}")
        if t.device != q.device:
            raise ValueError("attention: q, k and v must be on the same device")
    depth, queries, keys = q.shape[-1], q.shape[-2], k.shape[-2]
    if k.shape[-1] != depth:
        raise ValueError(f"attention: q {tuple(q.shape)} and k {tuple(k.shape)} differ in the last "
                         "dimension")
    if v.shape[-2] != keys:
        raise ValueError(f"attention: k {tuple(k.shape)} and v {tuple(v.shape)} differ in the "
                         "number of keys")
    if scale == 0.0:
        scale = float(np.float32(1.0 / np.sqrt(depth))) if depth > 0 else 1.0
    eligible = _fused_attention_eligible(q, k, v, mask, precision)
    if fused and not eligible:
        raise ValueError("attention: the fused kernel needs q, k and v of one shape [..., L, 128] "
                         "on a CUDA device, 3xTF32, and a mask (if any) that is a Bool tensor on "
                         "their device broadcasting to the scores")
    if eligible and fused is not False:
        return _fused_attention(q, k, v, causal, scale, mask)
    scores = gemm_strided_batched(q, k, scale, None, 0.0, False, True, precision=precision)
    keep = None
    if mask is not None:
        if not isinstance(mask, torch.Tensor) or mask.dtype != torch.bool:
            raise ValueError("attention: mask must be a defined Bool tensor")
        if mask.device != q.device:
            raise ValueError("attention: mask must be on the inputs' device")
        if not _mask_broadcasts(mask, scores.shape):
            raise ValueError(f"attention: mask {tuple(mask.shape)} does not broadcast to the "
                             f"scores {tuple(scores.shape)}")
    if scores.numel() == 0:
        return gemm_strided_batched(scores, v, precision=precision)
    batch = scores.numel() // (queries * keys)
    keep_ptr, keep_bs, keep_rs = None, 0, 0
    if mask is not None:
        keep, keep_bs, keep_rs = _keep_matrices(mask, tuple(scores.shape))  # kept alive here
        keep_ptr = keep.data_ptr()
    check(_lib.lib().mfk_masked_softmax_f32(scores.data_ptr(), keep_ptr, keep_bs, keep_rs,
                                            1 if causal else 0, scores.data_ptr(), batch, queries,
                                            keys, _stream()), "attention")
    return gemm_strided_batched(scores, v, precision=precision)


def device_status() -> int:
    """Kernel error bits of the current device (0 = none); clears them."""
    return _lib.device_status(True)
