"""The reference's own test programs for the path, run on the B200 through the drop-in.

mensurflow_b200/host/Makefile compiles the unmodified reference library with this repository's
CUDA backend (mensurflow_b200/host/cuda_backend.cpp, which calls the sm_100a kernels through
include/mfk.h) in place of its cuBLAS backend, with the op-layer patches of
mensurflow_b200/host/patches applied to copies of the files they touch (gemm in one dispatch,
bias gradient, contiguous() and to() on the device), and links the reference's matmul_test,
matvec_test, elementwise_ops_test, dot_test (tests/ops/) and transfer_test, view_test
(tests/core/: Tensor::to, contiguous and views) against it. Those programs check values on every device
whose dispatcher has the kernel (tests/ops/matmul_test.cpp:97-100, matvec_test.cpp:69-72,
elementwise_ops_test.cpp has_bias), so on a GPU box they run their CPU checks and then the same
checks on cuda:0. reference_api_check is this repository's own program over the same library: it
calls the reference's public API with Execution::GPU and Execution::CPU and compares them. The
build needs the reference sources, so it happens where they are; the programs run anywhere."""
import os
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BUILD = os.path.join(ROOT, "mensurflow_b200", "host", "_build")

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name", ["matmul_test", "matvec_test", "elementwise_ops_test",
                                  "dot_test", "transfer_test", "view_test",
                                  "reference_api_check"])
def test_reference_program_passes_on_b200(cuda, name):
    path = os.path.join(BUILD, name)
    if not os.path.exists(path):
        pytest.skip("integration build absent (it is made where the reference sources are)")
    r = subprocess.run([path], capture_output=True, text=True, timeout=900)
    out = r.stdout + r.stderr
    assert r.returncode == 0, out[-4000:]
    assert "passed" in out
    if name == "matmul_test":
        # the program lists each device it checks; the CUDA one must be among them
        assert "matmul on cuda:0" in out, out[-2000:]
    if name == "elementwise_ops_test":
        # add / sub / mul / div have CUDA kernels now: checked for values on cuda:0, none
        # reported missing
        assert "elementwise ops on cuda:0" in out, out[-2000:]
        for op in ("add", "sub", "mul", "div"):
            assert f"no {op} kernel on cuda:0" not in out, out[-2000:]
    if name == "dot_test":
        assert "dot on cuda:0" in out, out[-2000:]
    if name == "reference_api_check":
        # this repository's check program (mensurflow_b200/host/reference_api_check.cpp): the
        # reference's public API with Execution::GPU against Execution::CPU, including
        # gemm_strided_batched, attention and softmax, which the reference's programs do not run
        # on a GPU
        assert "on cuda:0" in out and "attention both" in out, out[-2000:]
        assert "contiguous on the device: permute 2,0,1" in out, out[-2000:]
        # the op-layer patches: gemm in one dispatch (C1, the C2 call), the fused overload, the
        # level-1 kernels, gradients and Tensor::contiguous() on the device
        for line in ("gemm C1 1024^3 (one dispatch)",
                     "gemm + bias_add C2 8192^3 rows 4064..+32",
                     "gemm + bias + gelu 300x520x256 (one kernel)",
                     "dot n=1048583", "div, row broadcast (bit-exact)",
                     "bias_add bias gradient on the device (bit-exact)",
                     "matmul dB on the device",
                     "Tensor::contiguous() of a CUDA view: stepped slices",
                     "attention in one kernel, causal 2x4x384x128",
                     "attention in one kernel with a mask, causal 2x4x384x128"):
            assert line in out, (line, out[-3000:])
