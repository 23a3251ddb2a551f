"""The explicit-split path: where the tensor cores truncate fp32 operands to tf32 (B200), the
kernels that split an operand themselves keep its raw values as the hi part; MFK_EXPLICIT_SPLIT
makes them write hi explicitly, as they must on tensor cores that round. Both must give the same
bits: the GEMM's A split in shared and in tensor memory, the short-K GEMM, and the fused
attention's Q, K and V splits, computed in a child process with the variable set and here without."""
import os
import subprocess
import sys

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


def test_explicit_split_gives_the_same_bits(cuda, tmp_path):
    import _explicit_split_child as child

    out = tmp_path / "explicit.npz"
    env = dict(os.environ, MFK_EXPLICIT_SPLIT="1")
    r = subprocess.run([sys.executable, os.path.join(HERE, "_explicit_split_child.py"), str(out)],
                       env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    explicit = np.load(out)
    default = child.run()
    assert sorted(explicit.files) == sorted(default)
    for name in explicit.files:
        np.testing.assert_array_equal(explicit[name], default[name], err_msg=name)
