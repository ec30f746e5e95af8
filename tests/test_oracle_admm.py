"""The ADMM oracle (oracle/admm.py) against the reference's own ADMM test cases (CPU).

Values and Jacobians are the analytic ones the reference's tests assert,
transcribed in tests/golden/reference_cases.json with their file:line; the
banded factor is checked against a dense solve as in
tests/test_regression_admm_factor.py:14-41.  Gradients come from the oracle's
active-set KKT VJP; derivatives w.r.t. parameters are central differences of
the oracle's forward.
"""

import json
from pathlib import Path

import numpy as np
import pytest

from helpers import OracleADMMLayer
from oracle.admm import prepare_banded
from oracle.sparse import layout
from purin_b200.config import ADMMConfig, ImplicitGradientConfig
from purin_b200.problems import Projection

CASES = json.loads((Path(__file__).parent / "golden" / "reference_cases.json").read_text())
CONVERGED, MAX_ITERATIONS, NONFINITE = 0, 1, 3


def _target_jacobian(layer, target, theta=None):
    """d y_b / d target_b per sample by the oracle's VJP with unit cotangents."""
    result, saved = layer.solve(target, theta)
    batch, n = target.shape
    jac = np.zeros((batch, n, n))
    for i in range(n):
        cot = np.zeros_like(target)
        cot[:, i] = 1
        jac[:, i, :] = layer.proj.vjp(saved, cot)["target"]
    return result, jac


def _affine_problem():
    """``tests/test_regression_admm.py:16-22``."""
    p = Projection(method="admm")
    t = p.add_parameter(["b"])
    y = p.add_variable(["u", "v"])
    p.objective = 0.0
    p.constraints.add(y.u + y.v == t.b, y.u >= 0)
    return p


@pytest.mark.parametrize("adaptive_rho", [False, True])
def test_affine_projection_and_gradients(adaptive_rho):
    case = CASES["admm_affine_projection"]
    cfg = ADMMConfig(adaptive_rho=adaptive_rho, implicit_gradient=ImplicitGradientConfig(
        differentiate_problem_parameters=True))
    layer = OracleADMMLayer(_affine_problem(), cfg)
    target, theta = np.array(case["target"]), np.array(case["parameters"])
    result, jac = _target_jacobian(layer, target, theta)
    np.testing.assert_allclose(result["y"], case["y"], atol=case["atol"])
    assert (result["status"] == CONVERGED).all()
    assert result["residual_inf_norm"].max() <= cfg.tolerance
    np.testing.assert_allclose(jac[0], case["jacobian_sample0"], atol=case["atol"])
    np.testing.assert_allclose(jac[1], case["jacobian_sample1"], atol=case["atol"])
    eps = 1e-4
    fd = (layer(target, theta + eps) - layer(target, theta - eps)) / (2 * eps)
    np.testing.assert_allclose(fd, case["theta_derivative"], atol=1e-5)


def _box_problem():
    """``tests/test_regression_admm_rows.py:12-16``: two-sided bounds as opposite rows."""
    p = Projection()
    y = p.add_variable(["x", "y"])
    p.objective = 0.0
    p.constraints.add(y.x <= 1, -y.x <= 0, y.y <= 2, -y.y <= 1)
    return p


def test_two_sided_box_original_multipliers_slacks_and_gradient():
    case = CASES["admm_two_sided_box"]
    layer = OracleADMMLayer(_box_problem(), ADMMConfig())
    assert len(layer.proj.pairs.keep) == case["kept_rows"]
    target = np.array(case["target"])
    result, jac = _target_jacobian(layer, target)
    for key in ("y", "multipliers_ineq", "slacks"):
        np.testing.assert_allclose(result[key], case[key], atol=case["atol"], err_msg=key)
    np.testing.assert_allclose(jac.sum(axis=1), case["gradient_of_sum"], atol=1e-8)
    assert (result["status"] == CONVERGED).all()


@pytest.mark.parametrize("adaptive", [False, True])
def test_periodic_acceptance_matches_every_iteration_checks(adaptive):
    """``tests/test_regression_admm_diagnostics.py:15-44``."""
    case = CASES["admm_periodic_acceptance"]
    p = Projection()
    y = p.add_variable(["u", "v"])
    p.objective = 0.0
    p.constraints.add(y.u + y.v == 1, y.u >= 0, y.u <= 1)
    target = np.array(case["target"])
    outs = []
    for interval in (1, 25):
        cfg = ADMMConfig(adaptive_rho=adaptive, rho_update_interval=7, check_interval=interval)
        result, _ = OracleADMMLayer(p, cfg).solve(target)
        assert result["gradient_eligible"].all()
        assert result["residual_inf_norm"].max() <= cfg.tolerance
        outs.append(result["y"])
    np.testing.assert_allclose(outs[0], outs[1], atol=case["atol"])
    np.testing.assert_allclose(outs[1], case["y"], atol=case["atol"])


def test_final_step_is_checked_between_intervals():
    """``tests/test_regression_admm_diagnostics.py:47-56``."""
    p = Projection()
    y = p.add_variable(["u", "v"])
    p.objective = 0.0
    p.constraints.add(y.u + y.v == 1, y.u >= 0, y.u <= 1)
    cfg = ADMMConfig(tolerance=1e-14, max_iterations=17, check_interval=25)
    result, _ = OracleADMMLayer(p, cfg).solve(np.array([[3.0, -1.0]]))
    assert result["iterations"][0] == 17
    assert np.isfinite(result["residual_inf_norm"][0])
    assert result["status"][0] == MAX_ITERATIONS and not result["gradient_eligible"][0]


def test_iteration_limit_and_nonfinite():
    """``tests/test_regression_admm.py:69-90``."""
    layer = OracleADMMLayer(_affine_problem(), ADMMConfig(max_iterations=1))
    result, saved = layer.solve(np.array([[-2.0, 0.0]]), np.ones((1, 1)))
    assert result["status"][0] == MAX_ITERATIONS and not result["gradient_eligible"][0]
    assert not layer.proj.vjp(saved, np.ones((1, 2)))["target"].any()
    result, _ = layer.solve(np.array([[np.nan, 0.0]]), np.ones((1, 1)))
    assert result["status"][0] == NONFINITE


def test_no_constraints_identity():
    """``tests/test_regression_admm.py:93-100``."""
    p = Projection()
    p.add_variable(["u", "v"])
    p.objective = 0.0
    layer = OracleADMMLayer(p, ADMMConfig())
    x = np.array([[0.2, 0.7]])
    result, jac = _target_jacobian(layer, x)
    np.testing.assert_allclose(result["y"], x, atol=1e-12)
    np.testing.assert_allclose(jac.sum(axis=1), 1, atol=1e-9)


def test_parameter_dependent_active_inequality_gradient():
    case = CASES["admm_parameter_dependent_active_inequality"]
    p = Projection()
    t = p.add_parameter(["b"])
    y = p.add_variable(["u", "v"])
    p.objective = 0.0
    p.constraints.add(y.u >= t.b)
    layer = OracleADMMLayer(p, ADMMConfig())
    x, theta = np.array(case["target"]), np.array(case["parameters"])
    np.testing.assert_allclose(layer(x, theta), case["y"], atol=case["atol"])
    eps = 1e-5
    fd = (layer(x, theta + eps) - layer(x, theta - eps))[0] / (2 * eps)
    np.testing.assert_allclose(fd, case["theta_jacobian"], atol=1e-6)


def test_infeasible_and_contradictory_rows_never_converge():
    """``tests/test_regression_admm.py:137-151``; ``test_regression_admm_rows.py:64-73``."""
    for build in ("u<=0,u>=1", "u<=0,-u<=-1"):
        p = Projection()
        y = p.add_variable(["u"])
        p.objective = 0.0
        if build == "u<=0,u>=1":
            p.constraints.add(y.u <= 0, y.u >= 1)
        else:
            p.constraints.add(y.u <= 0, -y.u <= -1)
        result, _ = OracleADMMLayer(p, ADMMConfig(max_iterations=100)).solve(np.zeros((1, 1)) + 2)
        assert result["status"][0] == MAX_ITERATIONS and not result["gradient_eligible"][0]


@pytest.mark.parametrize("n,width", [(1, 0), (8, 1), (12, 3), (18, 6)])
def test_banded_factor_matches_dense(n, width):
    """``tests/test_regression_admm_factor.py:14-41``."""
    rng = np.random.default_rng(n)
    rows = [tuple(range(i, min(i + width + 1, n))) for i in range(n)]
    support, mask, _ = layout(rows, n)
    plan = prepare_banded(support, mask, n)
    assert plan is not None
    values = rng.normal(size=(3, *support.shape)) * np.asarray(mask)
    diagonal = rng.uniform(0.2, 2.0, size=(3, n))
    rhs = rng.normal(size=(3, n))
    for scale in (1.0, 2.3):
        penalty = rng.uniform(0.1, 4.0, size=(3, n)) * scale
        actual = plan.solve(plan.factor(diagonal, values, penalty, 1e-6), rhs)
        for b in range(3):
            a = np.zeros((n, n))
            for i, row in enumerate(rows):
                a[i, list(row)] = values[b, i, :len(row)]
            matrix = np.diag(diagonal[b] + 1e-6) + a.T @ (penalty[b, :, None] * a)
            np.testing.assert_allclose(actual[b], np.linalg.solve(matrix, rhs[b]), atol=2e-12)


def test_wide_structure_has_no_band():
    support, mask, _ = layout([tuple(range(20))], 20)
    assert prepare_banded(support, mask, 20) is None


def test_pcg_path_matches_a_dense_kkt_solve():
    """The PCG path (no band) on a random dense QP against its active-set KKT solution,
    standing in for the reference's OSQP comparison
    (``tests/test_regression_admm_diagnostics.py:59-97``, osqp is not installed)."""
    from oracle.admm import sparse_admm

    rng = np.random.default_rng(53)
    n, m = 12, 16
    a = rng.normal(size=(m, n))
    q = rng.uniform(0.5, 2.0, size=n)
    c = rng.normal(size=n)
    lo = -rng.uniform(0.2, 1.0, size=m)
    hi = rng.uniform(0.2, 1.0, size=m)
    support, mask, _ = layout([tuple(range(n))] * m, n)
    for interval in (1, 25):
        out = sparse_admm(q[None], c[None], a[None], lo[None], hi[None], support, mask,
                          check_interval=interval)
        assert out.converged[0]
        assert max(out.linear_residual[0], out.primal_residual[0], out.dual_residual[0]) <= 1e-9
        # KKT at the solution: q x + c + A^T y = 0 with y >= 0 on rows at their upper
        # bound and <= 0 at the lower, zero elsewhere.
        x, y = out.x[0], out.dual[0]
        ax = a @ x
        assert np.all(ax <= hi + 1e-8) and np.all(ax >= lo - 1e-8)
        np.testing.assert_allclose(q * x + c + a.T @ y, 0, atol=1e-8)
        inactive = (ax < hi - 1e-6) & (ax > lo + 1e-6)
        np.testing.assert_allclose(y[inactive], 0, atol=1e-8)


def test_invalid_configuration():
    """``tests/test_regression_admm.py:183-199``."""
    for kwargs in ({"rho": 0.0}, {"sigma": -1.0}, {"alpha": 2.0}, {"cg_max_iterations": 0},
                   {"cg_refinement_steps": 0}, {"rho_update_interval": 0},
                   {"tolerance": float("nan")}, {"check_interval": 0}):
        with pytest.raises(ValueError):
            ADMMConfig(**kwargs)
