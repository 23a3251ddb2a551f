"""bench.py's host-side pieces that need no GPU: the per-launch DRAM traffic it reports comes
from the committed ncu summaries, one figure per workload that has a roofline."""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import bench  # noqa: E402


@pytest.mark.parametrize("workload,precision", [("c2", "3xtf32"), ("c3", "3xtf32"),
                                                 ("c4", "3xtf32"), ("gemv", "f64acc"),
                                                 ("copy", "f32")])
def test_every_roofline_workload_has_a_profiled_traffic_figure(workload, precision):
    traffic = bench.profiled_traffic(workload, precision)
    assert traffic is not None and traffic > 0


def test_traffic_lookup_misses_unknown_keys():
    assert bench.profiled_traffic("c2", "1xtf32") is None
    assert bench.profiled_traffic("nope", "3xtf32") is None
