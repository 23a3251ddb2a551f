"""Shared test helpers: the reference tests' input generator, seeded config inputs and the parity
bounds of the path."""
import os

import numpy as np

from oracle import oracle as O

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")

# Parity bounds (per element, relative to the magnitude (|A||B|)_ij, plus an absolute floor).
TOL_3X = (1e-5, 1e-6)
TOL_1X = (2e-3, 1e-6)


def golden(name):
    return np.load(os.path.join(GOLDEN, name))


def make_input(n, seed):
    """The reference tests' generator: multiples of 0.25 in [-4, 4] from an LCG
    (tests/ops/matmul_test.cpp:25-35). Vectorised; same sequence as make_golden.make_input."""
    n = int(n)
    out = np.empty(n, np.float32)
    state = np.uint64(seed)
    # the LCG is sequential; step it in plain Python ints (fast enough for test sizes)
    s = int(state)
    vals = np.empty(n, np.int64)
    for i in range(n):
        s = (s * 1664525 + 1013904223) & 0xFFFFFFFF
        vals[i] = (s >> 12) % 33 - 16
    out[:] = vals.astype(np.float32) / 4
    return out


def seeded_inputs():
    """Inputs of tests/golden/seeded_cases.npz, regenerated with the oracle's Philox."""
    d = {}
    m = n = k = 192
    d["c2_a"] = O.normal(m * k, 0, 1, 1, 0).reshape(m, k)
    d["c2_b"] = O.normal(n * k, 0, 1, 1, m * k).reshape(n, k)
    d["c2_c"] = O.normal(m * n, 0, 1, 1, m * k + n * k).reshape(m, n)
    d["c2_bias"] = O.uniform(n, -0.1, 0.1, 1, m * k + n * k + m * n)
    d["c3_x"] = O.normal(64 * 96, 0, 1, 2, 0).reshape(64, 96)
    d["c3_w1"] = O.uniform(96 * 160, -0.034233, 0.034233, 2, 64 * 96).reshape(96, 160)
    q = 4 * 64 * 32
    std = 1 / np.sqrt(32)
    d["c4_q"] = O.normal(q, 0, std, 3, 0).reshape(4, 64, 32)
    d["c4_k"] = O.normal(q, 0, std, 3, q).reshape(4, 64, 32)
    d["c4_v"] = O.normal(q, 0, std, 3, 2 * q).reshape(4, 64, 32)
    d["gemv_a"] = O.uniform(300 * 257, -1, 1, 4, 0).reshape(300, 257)
    d["gemv_x"] = O.uniform(257, -1, 1, 4, 300 * 257)
    d["gemv_y"] = O.uniform(300, -1, 1, 4, 300 * 257 + 257)
    d["act_x"] = O.normal(4096, 0, 3, 7, 0)
    return d


def softmax_rows(s):
    p = np.exp(s - s.max(-1, keepdims=True)).astype(np.float32)
    return (p / p.sum(-1, keepdims=True)).astype(np.float32)


def assert_close(got, want, magnitude, tol, what):
    """|got - want| <= rel * magnitude + abs, elementwise."""
    rel, ab = tol
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    assert got.shape == want.shape, f"{what}: shape {got.shape} != {want.shape}"
    err = np.abs(got - want)
    bound = rel * np.asarray(magnitude, np.float64) + ab
    bad = ~(err <= bound)
    if bad.any():
        i = np.unravel_index(np.argmax(np.where(bad, err - bound, -np.inf)), got.shape)
        raise AssertionError(
            f"{what}: {int(bad.sum())} of {got.size} entries out of tolerance; worst at {i}: "
            f"got {got[i]!r} want {want[i]!r} bound {bound[i]!r}")


def ulp_diff(a, b):
    """Distance in float32 ulps (sign-aware) between two float32 arrays."""
    ai = np.asarray(a, np.float32).view(np.int32).astype(np.int64)
    bi = np.asarray(b, np.float32).view(np.int32).astype(np.int64)
    ai = np.where(ai < 0, np.int64(-(2 ** 31)) - ai, ai)
    bi = np.where(bi < 0, np.int64(-(2 ** 31)) - bi, bi)
    return np.abs(ai - bi)


def attention_inputs():
    """Inputs of tests/golden/attention_cases.npz, regenerated with the oracle's Philox."""
    d = {}
    x = O.normal(3 * 5 * 17, 0, 30, 9, 0).reshape(3, 5, 17)
    x[0, 1, :] = -np.inf
    x[1, 2, 3] = np.nan
    x[2, 0, :] += 1000
    d["softmax_x"] = x
    b, h, lq, lk, dd, dv = 2, 3, 5, 7, 8, 4
    d["q"] = O.normal(b * h * lq * dd, 0, 1, 21, 0).reshape(b, h, lq, dd)
    d["k"] = O.normal(b * h * lk * dd, 0, 1, 22, 0).reshape(b, h, lk, dd)
    d["v"] = O.normal(b * h * lk * dv, 0, 1, 23, 0).reshape(b, h, lk, dv)
    d["keep"] = np.array([[i != 2 and (i + j) % 3 != 0 for j in range(lk)] for i in range(lq)])
    d["k1"] = O.normal(b * lk * dd, 0, 1, 24, 0).reshape(b, 1, lk, dd)
    d["v1"] = O.normal(b * lk * dv, 0, 1, 25, 0).reshape(b, 1, lk, dv)
    lq2 = 64
    d["q2"] = O.normal(4 * lq2 * 32, 0, 1 / np.sqrt(32), 26, 0).reshape(4, lq2, 32)
    d["k2"] = O.normal(4 * lq2 * 32, 0, 1 / np.sqrt(32), 27, 0).reshape(4, lq2, 32)
    d["v2"] = O.normal(4 * lq2 * 32, 0, 1 / np.sqrt(32), 28, 0).reshape(4, lq2, 32)
    return d


def backward_inputs():
    """Inputs of tests/golden/backward_cases.npz, regenerated with the oracle's Philox."""
    import sys
    sys.path.insert(0, GOLDEN)
    from make_golden import BIAS_GRAD_SHAPES, MATMUL_BWD_SHAPES
    d = {}
    for i, (rows, cols) in enumerate(BIAS_GRAD_SHAPES):
        d[f"bias_grad_{rows}x{cols}"] = O.normal(rows * cols, 0, 1, 40 + i, 0).reshape(rows, cols)
    for i, (m, k, n) in enumerate(MATMUL_BWD_SHAPES):
        d[f"matmul_{m}x{k}x{n}"] = (
            O.normal(m * k, 0, 1, 60 + i, 0).reshape(m, k),
            O.normal(k * n, 0, 1, 60 + i, m * k).reshape(k, n),
            O.normal(m * n, 0, 1, 60 + i, m * k + k * n).reshape(m, n))
    return d


# Strided views packed by Tensor::contiguous(): name, base shape (a contiguous tensor), permute
# order, slices {dim: (start, end, step)} applied after the permute, expand shape (or None), and
# the input ("iota" as the reference's tests/core tests use, else seeded normal). The first four
# are the views of the reference's tests/core/transfer_test.cpp:50-62 and view_test.cpp:80-100.
COPY_CASES = [
    ("transfer_test transpose", (3, 4), (1, 0), {}, None, "iota"),
    ("transfer_test every other column", (3, 4), (0, 1), {1: (0, 4, 2)}, None, "iota"),
    ("view_test permute", (2, 3, 4), (2, 0, 1), {}, None, "iota"),
    ("view_test transpose then slice", (2, 3, 4), (1, 0, 2), {2: (3, 4, 1)}, None, "iota"),
    ("transpose 257x129", (129, 257), (1, 0), {}, None, "normal"),
    ("transpose 1024x1024", (1024, 1024), (1, 0), {}, None, "normal"),
    ("permute rows 0,2,1,3", (3, 20, 30, 64), (0, 2, 1, 3), {}, None, "normal"),
    ("permute 3,1,2,0", (5, 6, 7, 40), (3, 1, 2, 0), {}, None, "normal"),
    ("aligned column slice", (64, 100), (0, 1), {1: (8, 72, 1)}, None, "normal"),
    ("unaligned column slice", (64, 100), (0, 1), {1: (3, 70, 1)}, None, "normal"),
    ("stepped in both dims", (50, 80), (0, 1), {0: (1, 50, 3), 1: (2, 80, 2)}, None, "normal"),
    ("expand leading and size-1", (1, 7, 48), (0, 1, 2), {}, (5, 3, 7, 48), "normal"),
    ("expand innermost", (6, 1), (0, 1), {}, (6, 40), "normal"),
    ("short rows", (200, 9, 5), (0, 1, 2), {2: (0, 3, 1)}, None, "normal"),
    ("single element", (4, 5), (0, 1), {0: (2, 3, 1), 1: (3, 4, 1)}, None, "normal"),
    ("empty", (4, 5), (0, 1), {0: (2, 2, 1)}, None, "normal"),
    ("batched transpose with slice", (8, 33, 65), (0, 2, 1), {1: (1, 65, 1)}, None, "normal"),
    ("5-D permute", (3, 4, 5, 6, 7), (4, 2, 0, 3, 1), {}, None, "normal"),
    ("stepped columns of a whole matrix", (64, 200), (0, 1), {1: (0, 200, 2)}, None, "normal"),
    ("long aligned rows", (3, 9000), (0, 1), {1: (4, 8996, 1)}, None, "normal"),
]


def copy_case(i):
    """(input array, full slice list) of COPY_CASES[i]; the slice list has (start, end, step)
    for every dim of the permuted view."""
    name, base, order, slices, expand, kind = COPY_CASES[i]
    n = int(np.prod(base))
    if kind == "iota":
        x = np.arange(n, dtype=np.float32).reshape(base)
    else:
        x = O.normal(n, 0, 1, 70 + i, 0).reshape(base)
    permuted = [base[o] for o in order]
    full = [slices.get(d, (0, permuted[d], 1)) for d in range(len(base))]
    return x, full
