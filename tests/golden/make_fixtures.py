"""Regenerate the golden fixtures of this directory.

* ``oracle_config0.npz`` / ``oracle_config1_f32.npz``: the NumPy oracle's
  forward results (fixed iteration budget) on the first samples of benchmark
  configurations 0 and 1, generated from their seeded workloads.  GPU tests
  compare the CUDA layer with them bit for bit; CPU tests check the oracle
  still reproduces them.
* ``reference_cases.json``: the analytic values and Jacobians the reference's
  own test-suite asserts for the CP path, transcribed with their source
  file:line (JAX is not installed here, so the reference cannot be run to
  produce them).

Usage: ``python tests/golden/make_fixtures.py`` from the repository root.
"""

from __future__ import annotations

import json
import sys
from dataclasses import replace
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "tests"))

REFERENCE_CASES = {
    "affine_projection": {
        "source": "tests/test_projections.py:64-74",
        "target": [[0.8, 0.7]], "parameters": [[1.0]],
        "y": [[0.55, 0.45]], "jacobian": [[0.5, -0.5], [-0.5, 0.5]],
        "atol_y": 2e-6, "atol_jacobian": 2e-5},
    "active_inequality": {
        "source": "tests/test_projections.py:77-96",
        "target": [[2.0, -1.0]], "parameters": [[1.0]], "y": [[1.0, 0.0]], "atol_y": 2e-6},
    "weighted_distance": {
        "source": "tests/test_projections.py:121-124; tests/test_training_metric_contracts.py:63-95",
        "weights": [1.0, 4.0], "target": [[2.0, 0.0]], "parameters": [[1.0]],
        "y": [[1.2, -0.2]], "jacobian": [[0.2, -0.8], [-0.2, 0.8]], "atol_y": 2e-6,
        "atol_jacobian": 2e-5},
    "regression_batch2": {
        "source": "tests/test_regression_chambolle_pock.py:25-56",
        "target": [[2.0, 0.0], [-2.0, 0.0]], "parameters": [[1.0], [1.0]],
        "y": [[1.5, -0.5], [0.0, 1.0]], "jacobian_sample0": [[0.5, -0.5], [-0.5, 0.5]],
        "theta_derivative": [[0.5, 0.5], [0.0, 1.0]], "atol_y": 1e-8},
    "tied_scaled_bounds": {
        "source": "tests/test_regression_cp_bound_presolve.py:13-27",
        "target": [[-3.0, 4.0]], "y": [[0.0, 1.0]],
        "multipliers_ineq": [[1.5, 0.75, 0.0, 3.0]], "slacks": [[0.0, 0.0, 2.0, 0.0]]},
    "admm_affine_projection": {
        "source": "tests/test_regression_admm.py:16-57",
        "target": [[2.0, 0.0], [-2.0, 0.0]], "parameters": [[1.0], [1.0]],
        "y": [[1.5, -0.5], [0.0, 1.0]], "jacobian_sample0": [[0.5, -0.5], [-0.5, 0.5]],
        "jacobian_sample1": [[0.0, 0.0], [0.0, 0.0]], "theta_derivative": [[0.5, 0.5], [0.0, 1.0]],
        "atol": 1e-8},
    "admm_two_sided_box": {
        "source": "tests/test_regression_admm_rows.py:12-40",
        "target": [[3.0, 4.0], [-2.0, -3.0], [0.5, 0.5]], "kept_rows": 2,
        "y": [[1.0, 2.0], [0.0, -1.0], [0.5, 0.5]],
        "multipliers_ineq": [[2.0, 0.0, 2.0, 0.0], [0.0, 2.0, 0.0, 2.0], [0.0, 0.0, 0.0, 0.0]],
        "slacks": [[0.0, 1.0, 0.0, 3.0], [1.0, 0.0, 3.0, 0.0], [0.5, 0.5, 1.5, 1.5]],
        "gradient_of_sum": [[0.0, 0.0], [0.0, 0.0], [1.0, 1.0]], "atol": 2e-9},
    "admm_periodic_acceptance": {
        "source": "tests/test_regression_admm_diagnostics.py:15-44",
        "target": [[3.0, -1.0], [-2.0, 2.0], [0.2, 0.4]],
        "y": [[1.0, 0.0], [0.0, 1.0], [0.4, 0.6]], "atol": 3e-9},
    "admm_parameter_dependent_active_inequality": {
        "source": "tests/test_regression_admm.py:162-180",
        "target": [[-2.0, 0.3]], "parameters": [[1.0]], "y": [[1.0, 0.3]],
        "theta_jacobian": [1.0, 0.0], "atol": 1e-8},
    "parameter_dependent_bound": {
        "source": "tests/test_regression_cp_bound_presolve.py:30-53",
        "target": [[3.0]], "parameters": [[2.0, 1.0]], "y": [[0.5]],
        "theta_jacobian": [-0.25, 0.5]},
}


def oracle_fixture(index, batch, dtype, max_iterations):
    from helpers import OracleLayer
    from purin_b200.workloads import make_workload

    w = make_workload(index, batch)
    cfg = replace(w.config, max_iterations=max_iterations)
    result, _ = OracleLayer(w.problem, cfg, dtype).solve(w.candidates, w.theta)
    keep = ("y", "multipliers_eq", "multipliers_ineq", "slacks", "status", "iterations",
            "residual_inf_norm", "gradient_eligible")
    return {k: result[k] for k in keep}


def main():
    np.savez_compressed(HERE / "oracle_config0.npz", **oracle_fixture(0, 4, np.float64, 500))
    np.savez_compressed(HERE / "oracle_config1_f32.npz", **oracle_fixture(1, 2, np.float32, 100))
    (HERE / "reference_cases.json").write_text(json.dumps(REFERENCE_CASES, indent=1) + "\n")


if __name__ == "__main__":
    main()
