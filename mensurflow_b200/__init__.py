"""mensurflow_b200 — B200 (sm_100a) kernels for Mensurflow's dense fp32 contraction path.

The kernels live in ``lib/libmfkernels.so`` behind the C ABI of ``include/mfk.h``; ``ops``
mirrors the reference's op API over torch CUDA tensors, ``sharded`` splits a GEMM over ranks.
"""
from ._lib import MfkError, build  # noqa: F401
from .ops import (  # noqa: F401
    PackedB,
    add,
    attention,
    bias_add,
    bias_grad,
    contiguous,
    copy,
    device_status,
    div,
    dot,
    gelu,
    gemm,
    gemm_prepacked,
    gemm_strided_batched,
    gemv,
    get_default_precision,
    linear,
    linear_backward,
    log_softmax,
    matmul,
    matmul_backward,
    matvec,
    mul,
    pack_b,
    relu,
    scal,
    set_default_precision,
    softmax,
    sub,
    to,
    where,
)

__all__ = [
    "MfkError", "PackedB", "build", "add", "attention", "bias_add", "bias_grad", "contiguous",
    "copy", "device_status", "div", "dot", "mul", "scal", "sub",
    "gelu", "gemm", "gemm_prepacked", "gemm_strided_batched", "gemv", "get_default_precision",
    "linear", "linear_backward", "log_softmax", "matmul", "matmul_backward", "matvec", "pack_b",
    "relu", "set_default_precision", "softmax", "to", "where",
]
