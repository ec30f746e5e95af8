"""The C++ restatement of the CP loop (the CPU baseline) against the NumPy loop.

Both evaluate every product and sum one term at a time in the reference's
order, so iterates, iteration counts, residuals and convergence flags are
equal; the normalised gap sums its objectives sequentially in C++ and
pairwise in NumPy, so it agrees to rounding.
"""

from dataclasses import replace

import numpy as np
import pytest

from helpers import OracleLayer
from oracle.cpu import sparse_cp_native
from purin_b200.config import ChambollePockConfig
from purin_b200.workloads import make_workload, network_flow_config


def _compare(problem, cfg, candidates, theta):
    oracle = OracleLayer(problem, cfg, np.float64)
    _, numpy_saved = oracle.solve(candidates, theta)
    oracle.proj.cp_solver = sparse_cp_native
    _, native_saved = oracle.solve(candidates, theta)
    want, got = numpy_saved["out"], native_saved["out"]
    np.testing.assert_array_equal(got.y, want.y)
    np.testing.assert_array_equal(got.dual, want.dual)
    np.testing.assert_array_equal(got.iterations, want.iterations)
    np.testing.assert_array_equal(got.residual, want.residual)
    np.testing.assert_array_equal(got.converged, want.converged)
    np.testing.assert_allclose(got.gap, want.gap, rtol=1e-10, atol=1e-12)
    return want


@pytest.mark.parametrize("overrides", [
    {},
    {"accelerated": True},
    {"tolerance": 1e-4, "max_iterations": 4000},
], ids=["fixed", "accelerated", "converging"])
def test_config0_matches_numpy_loop(overrides):
    w = make_workload(0, 12)
    out = _compare(w.problem, replace(w.config, **overrides), w.candidates, w.theta)
    if "tolerance" in overrides:
        assert out.converged.any() and not out.converged.all()


def test_ragged_rows_match_numpy_loop():
    """Network-flow rows of different lengths: padded slots in the row layout."""
    problem, theta, candidates, _ = network_flow_config(batch=4, nodes=60, edges=200,
                                                        couplings=40, seed=3)
    _compare(problem, ChambollePockConfig(max_iterations=300), candidates, theta)


def test_threads_do_not_change_results():
    w = make_workload(0, 9)
    oracle = OracleLayer(w.problem, w.config, np.float64)
    outs = []
    for threads in (1, 3):
        oracle.proj.cp_solver = lambda *a, t=threads, **k: sparse_cp_native(*a, threads=t, **k)
        outs.append(oracle.solve(w.candidates, w.theta)[1]["out"])
    np.testing.assert_array_equal(outs[0].y, outs[1].y)
    np.testing.assert_array_equal(outs[0].gap, outs[1].gap)
