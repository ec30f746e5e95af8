"""The reference's analytic CP cases, evaluated by the CPU oracle.

Every case restates one test of the reference suite (cited per test) with the
same problem, configuration and tolerance.  Target Jacobians come from the
oracle's implicit VJP; parameter derivatives from central differences of the
oracle's forward solve, as the reference itself checks them.
"""

import itertools
from dataclasses import replace

import numpy as np
import pytest

from helpers import OracleLayer, make_problem, regression_problem
from oracle.cp import diagonal_step_sizes, proximal_coefficients, cp_step
from oracle.sparse import layout
from purin_b200 import ChambollePockConfig, ImplicitGradientConfig, LinearSolverConfig, Projection


def cp_config(**kw):
    return ChambollePockConfig(tolerance=1e-9, max_iterations=3000, **kw)


def theta_fd(layer, target, theta, eps=1e-4):
    """Central-difference d y / d theta: (B, n, p)."""
    theta = np.asarray(theta, float)
    out = np.zeros((target.shape[0], target.shape[1], theta.shape[1]))
    for k in range(theta.shape[1]):
        d = np.zeros_like(theta)
        d[:, k] = eps
        out[:, :, k] = (layer(target, theta + d) - layer(target, theta - d)) / (2 * eps)
    return out


def test_affine_projection_and_analytic_jacobian():
    """tests/test_projections.py:64-74"""
    layer = OracleLayer(make_problem(), cp_config())
    target, context = np.array([[0.8, 0.7]]), np.ones((1, 1))
    np.testing.assert_allclose(layer(target, context), [[0.55, 0.45]], atol=2e-6, rtol=0)
    np.testing.assert_allclose(layer.target_jacobian(target, context)[0],
                               [[0.5, -0.5], [-0.5, 0.5]], atol=2e-5, rtol=0)


@pytest.mark.parametrize("accelerated", [False, True])
def test_projection_with_active_inequality(accelerated):
    """tests/test_projections.py:77-96"""
    layer = OracleLayer(make_problem(inequalities=True), cp_config(accelerated=accelerated))
    np.testing.assert_allclose(layer(np.array([[2.0, -1.0]]), np.ones((1, 1))), [[1.0, 0.0]],
                               atol=2e-6, rtol=0)


def weighted(problem, weights, cfg):
    """metric.py:158-182: base layer on the column-scaled problem, tolerance / factor."""
    from purin_b200.problems import canonical_of

    w = np.asarray(weights, float)
    factor = max(1.0, float(np.sqrt(w.max())))
    base = OracleLayer(canonical_of(problem).scale_columns(1 / np.sqrt(w)),
                       replace(cfg, tolerance=cfg.tolerance / factor))
    sq = np.sqrt(w)
    project = lambda x, th: base(np.asarray(x) * sq, th) / sq
    jac = lambda x, th: base.target_jacobian(np.asarray(x) * sq, th) * sq[None, None, :] / sq[None, :, None]
    return project, jac


def test_weighted_projection_matches_diagonal_metric_solution():
    """tests/test_projections.py:121-124 and tests/test_training_metric_contracts.py:63-95"""
    project, jac = weighted(make_problem(), [1.0, 4.0], ChambollePockConfig())
    target, context = np.array([[2.0, 0.0]]), np.ones((1, 1))
    np.testing.assert_allclose(project(target, context), [[1.2, -0.2]], atol=2e-6, rtol=0)
    np.testing.assert_allclose(jac(target, context)[0], [[0.2, -0.8], [-0.2, 0.8]], atol=2e-5)


@pytest.mark.parametrize("accelerated", [False, True])
def test_affine_projection_and_gradients(accelerated):
    """tests/test_regression_chambolle_pock.py:25-56"""
    cfg = ChambollePockConfig(accelerated=accelerated)
    layer = OracleLayer(regression_problem(), cfg)
    values, theta = np.array([[2.0, 0.0], [-2.0, 0.0]]), np.ones((2, 1))
    result, _ = layer.solve(values, theta)
    np.testing.assert_allclose(result["y"], [[1.5, -0.5], [0.0, 1.0]], atol=1e-8)
    assert np.all(result["status"] == 0)
    assert np.max(result["residual_inf_norm"]) <= cfg.tolerance
    jac = layer.target_jacobian(values, theta)
    np.testing.assert_allclose(jac[0], [[0.5, -0.5], [-0.5, 0.5]], atol=1e-8)
    np.testing.assert_allclose(jac[1], 0, atol=1e-8)
    fd = theta_fd(layer, values, theta)
    np.testing.assert_allclose(fd[:, :, 0], [[0.5, 0.5], [0.0, 1.0]], atol=1e-5)


def test_iteration_limit_and_nonfinite_diagnostics():
    """tests/test_regression_chambolle_pock.py:68-85"""
    layer = OracleLayer(regression_problem(), ChambollePockConfig(max_iterations=1))
    result, saved = layer.solve(np.array([[-2.0, 0.0]]), np.ones((1, 1)))
    assert result["status"][0] == 1 and not result["gradient_eligible"][0]
    np.testing.assert_array_equal(layer.proj.vjp(saved, np.ones((1, 2)))["target"], 0)
    result, _ = layer.solve(np.array([[np.nan, 0.0]]), np.ones((1, 1)))
    assert result["status"][0] == 3


def test_no_constraints_identity():
    """tests/test_regression_chambolle_pock.py:88-95"""
    p = Projection()
    p.add_variable(["u", "v"])
    layer = OracleLayer(p, ChambollePockConfig())
    x = np.array([[0.2, 0.7]])
    np.testing.assert_allclose(layer(x), x, atol=1e-12)
    np.testing.assert_allclose(layer.target_jacobian(x)[0], np.eye(2), atol=1e-9)


def test_inequality_only_and_warm_start():
    """tests/test_regression_chambolle_pock.py:98-113"""
    p = Projection()
    y = p.add_variable(["u", "v"])
    p.constraints.add(y.u >= 0, y.v <= 1)
    layer = OracleLayer(p, ChambollePockConfig())
    result, _ = layer.solve(np.array([[-2.0, 3.0]]), multipliers_ineq=np.array([[0.2, 0.3]]))
    np.testing.assert_allclose(result["y"], [[0.0, 1.0]], atol=1e-8)
    assert result["gradient_eligible"][0]


def test_parameter_dependent_sparse_coefficients():
    """tests/test_regression_chambolle_pock.py:116-137"""
    p = Projection()
    t = p.add_parameter(["a"])
    y = p.add_variable(["u", "v"])
    p.constraints.add(t.a * y.u + y.v == 1)
    layer = OracleLayer(p, ChambollePockConfig())
    x, theta = np.array([[0.2, 0.3]]), np.array([[2.0]])

    def expected(a):
        row = np.array([[a, 1.0]])
        return x - row * ((row * x).sum() - 1) / (a**2 + 1)

    np.testing.assert_allclose(layer(x, theta), expected(2.0), atol=1e-8)
    fd_exp = (expected(2.0 + 1e-6) - expected(2.0 - 1e-6)) / 2e-6
    np.testing.assert_allclose(theta_fd(layer, x, theta, 1e-5)[:, :, 0], fd_exp, atol=1e-6)


def test_infeasible_problem_never_claims_convergence():
    """tests/test_regression_chambolle_pock.py:140-153"""
    p = Projection()
    y = p.add_variable(["u"])
    p.constraints.add(y.u <= 0, y.u >= 1)
    result, _ = OracleLayer(p, ChambollePockConfig(max_iterations=100)).solve(np.zeros((1, 1)))
    assert result["status"][0] == 1 and not result["gradient_eligible"][0]


def test_scaled_constraints_report_original_units():
    """tests/test_regression_chambolle_pock.py:156-164"""
    p = Projection()
    y = p.add_variable(["u", "v"])
    p.constraints.add(1000 * y.u + 1000 * y.v == 1000, y.u >= 0)
    layer = OracleLayer(p, ChambollePockConfig())
    result, _ = layer.solve(np.array([[2.0, 0.0]]))
    assert result["gradient_eligible"][0]
    assert abs(result["y"].sum() * 1000 - 1000) <= 1e-9


def test_tied_scaled_bounds_restore_duals_and_slacks():
    """tests/test_regression_cp_bound_presolve.py:13-27"""
    p = Projection()
    y = p.add_variable(["u", "v"])
    p.constraints.add(y.u >= 0, 2 * y.u >= 0, y.u <= 2, y.v <= 1)
    layer = OracleLayer(p, ChambollePockConfig())
    result, saved = layer.solve(np.array([[-3.0, 4.0]]))
    np.testing.assert_allclose(result["y"], [[0.0, 1.0]], atol=1e-10)
    np.testing.assert_allclose(result["multipliers_ineq"], [[1.5, 0.75, 0.0, 3.0]], atol=1e-9)
    np.testing.assert_allclose(result["slacks"], [[0.0, 0.0, 2.0, 0.0]], atol=1e-10)
    assert result["status"][0] == 0
    assert len(layer.proj.rows) == 0
    np.testing.assert_allclose(layer.proj.vjp(saved, np.ones((1, 2)))["target"], 0.0, atol=1e-9)


def test_parameter_dependent_bound_sign_zero_and_derivative():
    """tests/test_regression_cp_bound_presolve.py:30-53"""
    p = Projection()
    t = p.add_parameter(["a", "b"])
    y = p.add_variable(["u"])
    p.constraints.add(t.a * y.u <= t.b)
    layer = OracleLayer(p, ChambollePockConfig())
    x, theta = np.array([[3.0]]), np.array([[2.0, 1.0]])
    np.testing.assert_allclose(layer(x, theta), [[0.5]], atol=1e-10)
    np.testing.assert_allclose(theta_fd(layer, x, theta, 1e-6)[0, 0], [-0.25, 0.5], atol=1e-6)
    np.testing.assert_allclose(layer(np.array([[-3.0]]), np.array([[-2.0, 1.0]])), [[-0.5]],
                               atol=1e-10)
    result, _ = layer.solve(x, np.array([[0.0, -1.0]]))
    assert not result["gradient_eligible"][0]
    np.testing.assert_allclose(layer(x, np.array([[0.0, 1.0]])), x)


def kkt_projection(matrix, upper, me, x):
    """Exact projection onto {A[:me] y = u[:me], A[me:] y <= u[me:]} by active sets."""
    m, n = matrix.shape
    best = None
    for k in range(m - me + 1):
        for active in itertools.combinations(range(me, m), k):
            rows = list(range(me)) + list(active)
            A = matrix[rows]
            kkt = np.block([[np.eye(n), A.T], [A, np.zeros((len(rows), len(rows)))]])
            try:
                sol = np.linalg.solve(kkt, np.r_[x, upper[rows]])
            except np.linalg.LinAlgError:
                continue
            y, lam = sol[:n], sol[n:]
            if np.all(matrix[me:] @ y <= upper[me:] + 1e-12) and np.all(lam[me:] >= -1e-12):
                best = y
    return best


@pytest.mark.parametrize("seed", [12, 42])
def test_coupled_qp_matches_exact_kkt(seed):
    """tests/test_regression_cp_bound_presolve.py:56-109 (OSQP replaced by an exact KKT solve)"""
    rng = np.random.default_rng(seed)
    p = Projection()
    y = p.add_variable(["u", "v", "w"])
    p.constraints.add(y.u + y.v + y.w == 1, y.u >= 0, y.v >= -0.5, y.w <= 0.7,
                      2 * y.u - y.v <= 0.9)
    layer = OracleLayer(p, ChambollePockConfig())
    x = rng.normal(size=(1, 3))
    matrix = np.array([[1.0, 1.0, 1.0], [-1.0, 0.0, 0.0], [0.0, -1.0, 0.0], [0.0, 0.0, 1.0],
                       [2.0, -1.0, 0.0]])
    upper = np.array([1.0, 0.0, 0.5, 0.7, 0.9])
    result, saved = layer.solve(x)
    np.testing.assert_allclose(result["y"][0], kkt_projection(matrix, upper, 1, x[0]), atol=2e-8)
    mult = np.r_[result["multipliers_eq"][0], result["multipliers_ineq"][0]]
    np.testing.assert_allclose((result["y"][0] - x[0]) + matrix.T @ mult, 0.0, atol=1e-9)
    assert result["gradient_eligible"][0]
    g = rng.normal(size=(1, 3))
    analytic = layer.proj.vjp(saved, g)["target"]
    for i in range(3):
        d = np.zeros_like(x)
        d[0, i] = 1e-4
        fd = float(((layer(x + d) - layer(x - d)) * g).sum()) / 2e-4
        np.testing.assert_allclose(analytic[0, i], fd, atol=2e-5)


def test_metric_bound_with_heterogeneous_rows_and_zero_columns():
    """tests/test_regression_cp_diagonal_steps.py:13-25"""
    matrix = np.array([[100.0, 0.0, 0.2, 0.0], [0.0, 0.01, 0.0, 0.0], [0.0, 0.0, 0.0, 0.0]])
    support, mask, _ = layout([tuple(np.flatnonzero(r)) for r in matrix], 4)
    values = np.where(mask, matrix[np.arange(3)[:, None], support], 0.0)
    tau, sigma = diagonal_step_sizes(np.ones((2, 4)), values, support, mask, 0.95)
    assert np.all(np.isfinite(tau)) and np.all(tau > 0)
    assert np.all(np.isfinite(sigma)) and np.all(sigma > 0)
    for t, s in zip(tau, sigma):
        norm = np.linalg.norm(np.sqrt(s)[:, None] * matrix * np.sqrt(t)[None, :], 2)
        assert norm <= 0.95 + 1e-14


def test_diagonal_proximal_values():
    """tests/test_regression_cp_proximal_coefficients.py:11-46"""
    rng = np.random.default_rng(42)
    q = rng.uniform(0.1, 5.0, (3, 7))
    c = rng.normal(size=(3, 7))
    tau = np.array([0.1, 0.4, 0.7])
    y = rng.normal(size=(3, 7))
    a, d, offset = proximal_coefficients(q, c, tau)
    np.testing.assert_allclose(a * y - d * (2 * y) + offset,
                               (y - tau[:, None] * (2 * y + c)) / (1 + tau[:, None] * q), atol=1e-14)
    q = np.array([[0.0, 0.3, 2.0]])
    c = np.array([[1.0, -1.0, 0.5]])
    y = np.array([[0.3, 0.2, -0.1]])
    dual = np.array([[0.2, 0.3, 0.4]])
    args = ((y, dual, y), q, c, np.zeros_like(y), np.full_like(y, -2.0), np.full_like(y, 2.0),
            lambda x: x, lambda x: x, 1, np.array([0.3]), np.array([0.2]), np.ones(1))
    for a_, b_ in zip(cp_step(*args), cp_step(*args, proximal=proximal_coefficients(q, c, np.array([0.3])))):
        np.testing.assert_array_equal(a_, b_)


def test_numerical_regression_fp32():
    """.github/scripts/numerical_regression.py:23-80 (chambolle-pock, float32)"""
    cfg = replace(ChambollePockConfig(max_iterations=3000, tolerance=1e-6),
                  implicit_gradient=ImplicitGradientConfig(adjoint_tolerance=1e-5,
                                                           inexact_tolerance=1e-5),
                  linear_solver=LinearSolverConfig(tolerance=1e-6))
    layer = OracleLayer(make_problem(), cfg, np.float32)
    target, context = np.array([[0.8, 0.7]], np.float32), np.ones((1, 1), np.float32)
    np.testing.assert_allclose(layer(target, context), [[0.55, 0.45]], atol=5e-5, rtol=0)
    np.testing.assert_allclose(layer.target_jacobian(target, context)[0],
                               [[0.5, -0.5], [-0.5, 0.5]], atol=5e-5, rtol=0)
