"""Loader for the sm_100a kernel library (``lib/libmfkernels.so``, C ABI in ``include/mfk.h``).

There is no fallback: if the library is missing or fails to load, every op raises. The
structures below mirror ``mfk_gemm_desc`` / ``mfk_batch_desc`` field for field.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
import threading

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG_DIR, "lib", "libmfkernels.so")

MFK_OK = 0
MFK_ERR_INVALID_ARGUMENT = 1
MFK_ERR_UNSUPPORTED = 2
MFK_ERR_CUDA = 3
MFK_ERR_OUT_OF_MEMORY = 4
MFK_ERR_NO_DEVICE = 5
MFK_ERR_DEVICE_FAULT = 6
MFK_ERR_SCRATCH_LIMIT = 7
NOALLOC_SCRATCH_BYTES = 64 * 1024 * 1024
IPC_HANDLE_BYTES = 64

ACT_NONE, ACT_RELU, ACT_GELU, ACT_GELU_TANH = 0, 1, 2, 3
PRECISION_DEFAULT, PRECISION_3XTF32, PRECISION_1XTF32 = -1, 0, 1
BINARY_ADD, BINARY_SUB, BINARY_MUL, BINARY_DIV = 0, 1, 2, 3

# Every symbol include/mfk.h declares.
EXPORTED = (
    "mfk_gemm_f32",
    "mfk_gemm_f32_noalloc",
    "mfk_gemm_strided_batched_f32",
    "mfk_gemm_peer_f32",
    "mfk_sharded_gemm_f32",
    "mfk_ipc_get_handle",
    "mfk_ipc_open_handle",
    "mfk_ipc_close_handle",
    "mfk_pack_b_f32",
    "mfk_packed_b_shape",
    "mfk_packed_b_free",
    "mfk_gemm_prepacked_f32",
    "mfk_gemv_f32",
    "mfk_matvec_f32",
    "mfk_bias_act_f32",
    "mfk_bias_grad_f32",
    "mfk_softmax_f32",
    "mfk_attention_f32",
    "mfk_attention_masked_f32",
    "mfk_masked_softmax_f32",
    "mfk_where_f32",
    "mfk_strided_copy_f32",
    "mfk_copy_f32",
    "mfk_copy_peer",
    "mfk_binary_f32",
    "mfk_scal_f32",
    "mfk_dot_f32",
    "mfk_set_default_precision",
    "mfk_get_default_precision",
    "mfk_device_status",
    "mfk_status_string",
    "mfk_last_cuda_error",
    "mfk_version",
    "mfk_selftest_wait_timeout",
    "mfk_kernel_timer",
    "mfk_kernel_timer_read",
    "mfk_launch_count",
)


class GemmDesc(ctypes.Structure):
    _fields_ = [
        ("a", ctypes.c_void_p), ("a_rs", ctypes.c_int64), ("a_cs", ctypes.c_int64),
        ("b", ctypes.c_void_p), ("b_rs", ctypes.c_int64), ("b_cs", ctypes.c_int64),
        ("c_in", ctypes.c_void_p), ("c_in_rs", ctypes.c_int64), ("c_in_cs", ctypes.c_int64),
        ("c", ctypes.c_void_p), ("ldc", ctypes.c_int64),
        ("m", ctypes.c_int64), ("n", ctypes.c_int64), ("k", ctypes.c_int64),
        ("alpha", ctypes.c_float), ("beta", ctypes.c_float),
        ("bias", ctypes.c_void_p),
        ("activation", ctypes.c_int32), ("precision", ctypes.c_int32),
    ]


class BatchDesc(ctypes.Structure):
    _fields_ = [
        ("batch", ctypes.c_int64),
        ("a_offsets", ctypes.c_void_p), ("b_offsets", ctypes.c_void_p),
        ("a_stride", ctypes.c_int64), ("b_stride", ctypes.c_int64),
        ("c_in_stride", ctypes.c_int64), ("c_stride", ctypes.c_int64),
    ]


class MfkError(RuntimeError):
    """A non-zero mfk_status from the kernel library."""

    def __init__(self, status: int, what: str):
        self.status = status
        super().__init__(what)


_lock = threading.Lock()
_lib = None


def build(verbose: bool = False) -> str:
    """Compiles the library in-tree with nvcc (sm_100a); no GPU is needed."""
    cmd = ["make", "-C", PKG_DIR]
    if not verbose:
        cmd.insert(1, "-s")
    subprocess.run(cmd, check=True)
    return LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(
                    f"mensurflow_b200: kernel library {LIB_PATH} is not built "
                    "(run `make -C mensurflow_b200`); there is no CPU fallback")
            so = ctypes.CDLL(LIB_PATH)
            vp, i64, i32, f32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int32, ctypes.c_float
            so.mfk_gemm_f32.argtypes = [ctypes.POINTER(GemmDesc), vp]
            so.mfk_gemm_f32_noalloc.argtypes = [ctypes.POINTER(GemmDesc), vp]
            so.mfk_gemm_peer_f32.argtypes = [ctypes.POINTER(GemmDesc), vp]
            so.mfk_gemm_strided_batched_f32.argtypes = [ctypes.POINTER(GemmDesc),
                                                        ctypes.POINTER(BatchDesc), vp]
            so.mfk_sharded_gemm_f32.argtypes = [ctypes.POINTER(GemmDesc), i32,
                                                ctypes.POINTER(i32), ctypes.POINTER(vp), i32,
                                                i32, vp, i64]
            so.mfk_ipc_get_handle.argtypes = [vp, vp, ctypes.POINTER(i64)]
            so.mfk_ipc_open_handle.argtypes = [vp, ctypes.POINTER(vp)]
            so.mfk_ipc_close_handle.argtypes = [vp]
            so.mfk_pack_b_f32.argtypes = [vp, i64, i64, i64, i64, i32, vp,
                                          ctypes.POINTER(ctypes.c_void_p)]
            so.mfk_packed_b_shape.argtypes = [vp, ctypes.POINTER(i64), ctypes.POINTER(i64),
                                              ctypes.POINTER(i32)]
            so.mfk_packed_b_free.argtypes = [vp]
            so.mfk_gemm_prepacked_f32.argtypes = [ctypes.POINTER(GemmDesc), vp, vp]
            so.mfk_gemv_f32.argtypes = [vp, i64, i64, i64, i32, vp, i64, f32, f32, vp, vp, vp]
            so.mfk_matvec_f32.argtypes = [vp, i64, i64, vp, vp, vp]
            so.mfk_bias_act_f32.argtypes = [vp, vp, vp, i64, i64, i32, vp]
            so.mfk_bias_grad_f32.argtypes = [vp, i64, i64, i64, vp, vp]
            so.mfk_softmax_f32.argtypes = [vp, vp, i64, i64, i64, i32, vp]
            so.mfk_masked_softmax_f32.argtypes = [vp, vp, i64, i64, i32, vp, i64, i64, i64, vp]
            so.mfk_attention_f32.argtypes = [vp, vp, vp, vp, i64, i64, i64, i32, f32, vp]
            so.mfk_attention_masked_f32.argtypes = [vp, vp, vp, vp, i64, i64, i64, vp, i64, i64,
                                                    i64, i32, f32, vp]
            so.mfk_where_f32.argtypes = [vp, vp, vp, vp, i64, vp]
            so.mfk_strided_copy_f32.argtypes = [vp, ctypes.POINTER(i64), ctypes.POINTER(i64),
                                                i32, vp, vp]
            so.mfk_copy_f32.argtypes = [vp, vp, i64, vp]
            so.mfk_copy_peer.argtypes = [vp, i32, vp, i32, i64, vp]
            so.mfk_binary_f32.argtypes = [i32, vp, vp, vp, i64, vp]
            so.mfk_scal_f32.argtypes = [f32, vp, vp, i64, vp]
            so.mfk_dot_f32.argtypes = [vp, vp, i64, vp, vp]
            so.mfk_set_default_precision.argtypes = [i32]
            so.mfk_get_default_precision.restype = i32
            so.mfk_device_status.argtypes = [ctypes.POINTER(ctypes.c_uint32), i32]
            so.mfk_status_string.argtypes = [i32]
            so.mfk_status_string.restype = ctypes.c_char_p
            so.mfk_last_cuda_error.restype = ctypes.c_char_p
            so.mfk_version.restype = i32
            so.mfk_selftest_wait_timeout.argtypes = [ctypes.c_uint64,
                                                     ctypes.POINTER(ctypes.c_uint32), vp]
            so.mfk_kernel_timer.argtypes = [i32]
            so.mfk_kernel_timer_read.argtypes = [ctypes.POINTER(ctypes.c_double),
                                                 ctypes.POINTER(ctypes.c_int64)]
            so.mfk_launch_count.restype = ctypes.c_int64
            _lib = so
    return _lib


def check(status: int, op: str) -> None:
    if status == MFK_OK:
        return
    so = lib()
    text = so.mfk_status_string(status).decode()
    detail = so.mfk_last_cuda_error().decode()
    msg = f"{op}: {text}" + (f" ({detail})" if detail and status in (MFK_ERR_CUDA, MFK_ERR_OUT_OF_MEMORY, MFK_ERR_UNSUPPORTED) else "")
    if status == MFK_ERR_INVALID_ARGUMENT:
        raise ValueError(msg)
    raise MfkError(status, msg)


def device_status(clear: bool = True) -> int:
    """Waits for the current device and returns (and clears) its kernel error bits."""
    bits = ctypes.c_uint32(0)
    rc = lib().mfk_device_status(ctypes.byref(bits), 1 if clear else 0)
    if rc not in (MFK_OK, MFK_ERR_DEVICE_FAULT):
        check(rc, "mfk_device_status")
    return int(bits.value)


def kernel_timer(enable: bool) -> None:
    check(lib().mfk_kernel_timer(1 if enable else 0), "mfk_kernel_timer")


def kernel_timer_read():
    """(summed device ms, number of timed launches) since the last read."""
    ms = ctypes.c_double(0.0)
    n = ctypes.c_int64(0)
    check(lib().mfk_kernel_timer_read(ctypes.byref(ms), ctypes.byref(n)), "mfk_kernel_timer_read")
    return ms.value, n.value


def launch_count() -> int:
    return int(lib().mfk_launch_count())
