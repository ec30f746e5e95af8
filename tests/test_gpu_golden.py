"""The reference's CP golden values and Jacobians, through the CUDA layer.

Each test restates one analytic case of the reference test-suite (file:line in
the test name's docstring) with the same problem, configuration and tolerance.
"""

import numpy as np
import pytest
import torch
from dataclasses import replace

from helpers import make_problem, regression_problem
from purin_b200 import (
    ChambollePockConfig,
    Distance,
    ImplicitGradientConfig,
    LinearSolverConfig,
    Projection,
    SolveStatus,
    WeightedDistance,
    prepare_projection,
)

pytestmark = pytest.mark.gpu
DEV = "cuda"
F64 = torch.float64


def T(a, dtype=F64):
    return torch.as_tensor(np.asarray(a), dtype=dtype, device=DEV)


def np_(t):
    return t.detach().cpu().numpy()


def cp_config(**kw):
    return ChambollePockConfig(tolerance=1e-9, max_iterations=3000, **kw)


def jacobian(fn, x):
    return np_(torch.autograd.functional.jacobian(fn, x))


def test_affine_projection_and_analytic_jacobian():
    """tests/test_projections.py:64-74"""
    project = Distance(make_problem(), "chambolle-pock", cp_config()).prepare(batch_size=1)
    target = T([[0.8, 0.7]])
    context = T(np.ones((1, 1)))
    np.testing.assert_allclose(np_(project(target, context)), [[0.55, 0.45]], atol=2e-6, rtol=0)
    jac = jacobian(lambda x: project(x[None, :], context)[0], target[0])
    np.testing.assert_allclose(jac, [[0.5, -0.5], [-0.5, 0.5]], atol=2e-5, rtol=0)


@pytest.mark.parametrize("accelerated", [False, True])
def test_projection_with_active_inequality(accelerated):
    """tests/test_projections.py:77-96"""
    project = Distance(make_problem(inequalities=True), "chambolle-pock",
                       cp_config(accelerated=accelerated)).prepare(batch_size=1)
    values = project(T([[2.0, -1.0]]), T(np.ones((1, 1))))
    np.testing.assert_allclose(np_(values), [[1.0, 0.0]], atol=2e-6, rtol=0)


def test_weighted_projection_matches_diagonal_metric_solution():
    """tests/test_projections.py:121-124"""
    project = WeightedDistance(make_problem(), [1.0, 4.0]).prepare(batch_size=1)
    values = project(T([[2.0, 0.0]]), T(np.ones((1, 1))))
    np.testing.assert_allclose(np_(values), [[1.2, -0.2]], atol=2e-6, rtol=0)


def test_weighted_metric_protocol_and_analytic_gradient():
    """tests/test_training_metric_contracts.py:63-95"""
    prepared = WeightedDistance(make_problem(), [1.0, 4.0], method="chambolle-pock").prepare(
        batch_size=1)
    target, context = T([[2.0, 0.0]]), T(np.ones((1, 1)))
    expected = [[1.2, -0.2]]
    with pytest.raises(ValueError, match="warm starts"):
        prepared.solve(target, context, initial_state=T([[1.2, -0.2]]))
    np.testing.assert_allclose(np_(prepared.solve(target, context).y), expected, atol=2e-5)
    np.testing.assert_allclose(np_(prepared.project_training(target, context).y_tilde), expected,
                               atol=2e-5)
    np.testing.assert_allclose(np_(prepared.with_info(target, context)[0]), expected, atol=2e-5)
    jac = jacobian(lambda x: prepared(x[None], context)[0], target[0])
    np.testing.assert_allclose(jac, [[0.2, -0.8], [-0.2, 0.8]], atol=2e-5)


@pytest.mark.parametrize("accelerated", [False, True])
def test_affine_projection_and_gradients(accelerated):
    """tests/test_regression_chambolle_pock.py:25-56"""
    cfg = ChambollePockConfig(accelerated=accelerated, implicit_gradient=ImplicitGradientConfig(
        differentiate_problem_parameters=True))
    layer = prepare_projection(regression_problem(), method="chambolle-pock", config=cfg,
                               batch_size=2)
    values = T([[2.0, 0.0], [-2.0, 0.0]])
    theta = T(np.ones((2, 1)))
    out = layer.solve(values, theta)
    np.testing.assert_allclose(np_(out.y), [[1.5, -0.5], [0.0, 1.0]], atol=1e-8)
    assert np.all(np_(out.status) == int(SolveStatus.CONVERGED))
    assert np.max(np_(out.residual_inf_norm)) <= cfg.tolerance
    jac = jacobian(lambda x: layer(x, theta), values)
    np.testing.assert_allclose(jac[0, :, 0, :], [[0.5, -0.5], [-0.5, 0.5]], atol=1e-8)
    np.testing.assert_allclose(jac[1, :, 1, :], 0, atol=1e-8)
    np.testing.assert_allclose(jac[0, :, 1, :], 0, atol=1e-8)
    derivative = jacobian(lambda t: layer(values, t), theta)
    np.testing.assert_allclose(derivative[0, :, 0, 0], [0.5, 0.5], atol=1e-8)
    np.testing.assert_allclose(derivative[1, :, 1, 0], [0.0, 1.0], atol=1e-8)
    eps = 1e-4
    fd = (np_(layer(values, theta + eps)) - np_(layer(values, theta - eps))) / (2 * eps)
    np.testing.assert_allclose(fd, [[0.5, 0.5], [0.0, 1.0]], atol=1e-5)


def test_rejects_nonlinear_constraints():
    """tests/test_regression_chambolle_pock.py:59-65"""
    p = Projection()
    y = p.add_variable(["u"])
    p.objective = 0.0
    p.constraints.add(y.u**2 <= 1)
    with pytest.raises(ValueError, match="affine"):
        prepare_projection(p, method="chambolle-pock", batch_size=1)


def test_iteration_limit_and_nonfinite_diagnostics():
    """tests/test_regression_chambolle_pock.py:68-85"""
    layer = prepare_projection(regression_problem(), method="chambolle-pock",
                               config=ChambollePockConfig(max_iterations=1), batch_size=1)
    out = layer.solve(T([[-2.0, 0.0]]), T(np.ones((1, 1))))
    assert int(out.status[0]) == int(SolveStatus.MAX_ITERATIONS)
    assert not bool(out.gradient_eligible[0])
    x = T([[-2.0, 0.0]]).requires_grad_(True)
    layer(x, T(np.ones((1, 1)))).sum().backward()
    np.testing.assert_allclose(np_(x.grad), 0)
    out = layer.solve(T([[np.nan, 0.0]]), T(np.ones((1, 1))))
    assert int(out.status[0]) == int(SolveStatus.NONFINITE)


def test_no_constraints_and_zero_initial_gradient():
    """tests/test_regression_chambolle_pock.py:88-95"""
    p = Projection()
    p.add_variable(["u", "v"])
    p.objective = 0.0
    layer = prepare_projection(p, method="chambolle-pock", batch_size=1)
    x = T([[0.2, 0.7]]).requires_grad_(True)
    np.testing.assert_allclose(np_(layer(x)), np_(x), atol=1e-12)
    layer(x).sum().backward()
    np.testing.assert_allclose(np_(x.grad), 1, atol=1e-9)


def test_inequality_only_and_warm_start_gradients():
    """tests/test_regression_chambolle_pock.py:98-113"""
    p = Projection()
    y = p.add_variable(["u", "v"])
    p.objective = 0.0
    p.constraints.add(y.u >= 0, y.v <= 1)
    layer = prepare_projection(p, method="chambolle-pock", batch_size=1)
    x = T([[-2.0, 3.0]]).requires_grad_(True)
    d = T([[0.2, 0.3]]).requires_grad_(True)
    out = layer.project_training(x, multipliers_ineq=d)
    np.testing.assert_allclose(np_(out.y_tilde), [[0.0, 1.0]], atol=1e-8)
    assert bool(out.forward_gradient_eligible[0])
    # Warm-start multipliers are stop-gradient inputs: their gradient is zero.
    grad = torch.autograd.grad(out.y_tilde.sum(), d, allow_unused=True)[0]
    assert grad is None or np.allclose(np_(grad), 0)


def test_parameter_dependent_sparse_coefficients():
    """tests/test_regression_chambolle_pock.py:116-137"""
    p = Projection()
    t = p.add_parameter(["a"])
    y = p.add_variable(["u", "v"])
    p.objective = 0.0
    p.constraints.add(t.a * y.u + y.v == 1)
    cfg = ChambollePockConfig(implicit_gradient=ImplicitGradientConfig(
        differentiate_problem_parameters=True))
    layer = prepare_projection(p, method="chambolle-pock", config=cfg, batch_size=1)
    x = T([[0.2, 0.3]])
    theta = T([[2.0]])

    def expected(a):
        row = torch.stack([a[:, 0], torch.ones_like(a[:, 0])], dim=1)
        return x - row * ((row * x).sum() - 1) / (a[0, 0] ** 2 + 1)

    np.testing.assert_allclose(np_(layer(x, theta)), np_(expected(theta)), atol=1e-8)
    np.testing.assert_allclose(jacobian(lambda a: layer(x, a), theta),
                               jacobian(expected, theta), atol=1e-7)


def test_infeasible_problem_never_claims_convergence():
    """tests/test_regression_chambolle_pock.py:140-153"""
    p = Projection()
    y = p.add_variable(["u"])
    p.objective = 0.0
    p.constraints.add(y.u <= 0, y.u >= 1)
    layer = prepare_projection(p, method="chambolle-pock",
                               config=ChambollePockConfig(max_iterations=100), batch_size=1)
    out = layer.solve(T(np.zeros((1, 1))))
    assert int(out.status[0]) == int(SolveStatus.MAX_ITERATIONS)
    assert not bool(out.gradient_eligible[0])


def test_scaled_constraints_report_original_units():
    """tests/test_regression_chambolle_pock.py:156-164"""
    p = Projection()
    y = p.add_variable(["u", "v"])
    p.objective = 0.0
    p.constraints.add(1000 * y.u + 1000 * y.v == 1000, y.u >= 0)
    layer = prepare_projection(p, method="chambolle-pock", batch_size=1)
    out = layer.solve(T([[2.0, 0.0]]))
    assert bool(out.gradient_eligible[0])
    assert abs(float(out.y.sum()) * 1000 - 1000) <= layer.config.tolerance


def test_tied_scaled_bounds_restore_duals_and_slacks():
    """tests/test_regression_cp_bound_presolve.py:13-27"""
    p = Projection()
    y = p.add_variable(["u", "v"])
    p.objective = 0.0
    p.constraints.add(y.u >= 0, 2 * y.u >= 0, y.u <= 2, y.v <= 1)
    layer = prepare_projection(p, method="chambolle-pock", batch_size=1)
    out = layer.solve(T([[-3.0, 4.0]]))
    np.testing.assert_allclose(np_(out.y), [[0.0, 1.0]], atol=1e-10)
    np.testing.assert_allclose(np_(out.multipliers_ineq), [[1.5, 0.75, 0.0, 3.0]], atol=1e-9)
    np.testing.assert_allclose(np_(out.slacks), [[0.0, 0.0, 2.0, 0.0]], atol=1e-10)
    assert int(out.status[0]) == int(SolveStatus.CONVERGED)
    assert len(layer._bound_projection.rows) == 0
    x = T([[-3.0, 4.0]]).requires_grad_(True)
    layer(x).sum().backward()
    np.testing.assert_allclose(np_(x.grad), 0.0, atol=1e-9)


def test_parameter_dependent_bound_sign_zero_and_derivative():
    """tests/test_regression_cp_bound_presolve.py:30-53"""
    p = Projection()
    t = p.add_parameter(["a", "b"])
    y = p.add_variable(["u"])
    p.objective = 0.0
    p.constraints.add(t.a * y.u <= t.b)
    cfg = ChambollePockConfig(implicit_gradient=ImplicitGradientConfig(
        differentiate_problem_parameters=True))
    layer = prepare_projection(p, method="chambolle-pock", config=cfg, batch_size=1)
    x = T([[3.0]])
    theta = T([[2.0, 1.0]])
    np.testing.assert_allclose(np_(layer(x, theta)), [[0.5]], atol=1e-10)
    jac = jacobian(lambda z: layer(x, z), theta)
    np.testing.assert_allclose(jac[0, 0, 0], [-0.25, 0.5], atol=1e-8)
    np.testing.assert_allclose(np_(layer(T([[-3.0]]), T([[-2.0, 1.0]]))), [[-0.5]], atol=1e-10)
    out = layer.solve(x, T([[0.0, -1.0]]))
    assert not bool(out.gradient_eligible[0])
    xg = x.clone().requires_grad_(True)
    layer(xg, T([[0.0, -1.0]])).sum().backward()
    np.testing.assert_allclose(np_(xg.grad), 0.0)
    np.testing.assert_allclose(np_(layer(x, T([[0.0, 1.0]]))), np_(x))


def _kkt_solution(matrix, upper, me, x):
    """Exact projection onto {A[:me] y = u[:me], A[me:] y <= u[me:]} by active-set enumeration."""
    import itertools

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
def test_coupled_qp_matches_exact_kkt_and_target_finite_difference(seed):
    """tests/test_regression_cp_bound_presolve.py:56-109 (OSQP replaced by an exact KKT solve)"""
    rng = np.random.default_rng(seed)
    p = Projection()
    y = p.add_variable(["u", "v", "w"])
    p.objective = 0.0
    p.constraints.add(y.u + y.v + y.w == 1, y.u >= 0, y.v >= -0.5, y.w <= 0.7,
                      2 * y.u - y.v <= 0.9)
    layer = prepare_projection(p, method="chambolle-pock", batch_size=1)
    x = rng.normal(size=(1, 3))
    matrix = np.array([[1.0, 1.0, 1.0], [-1.0, 0.0, 0.0], [0.0, -1.0, 0.0], [0.0, 0.0, 1.0],
                       [2.0, -1.0, 0.0]])
    upper = np.array([1.0, 0.0, 0.5, 0.7, 0.9])
    ref = _kkt_solution(matrix, upper, 1, x[0])
    out = layer.solve(T(x))
    np.testing.assert_allclose(np_(out.y)[0], ref, atol=2e-8)
    mult = np.r_[np_(out.multipliers_eq)[0], np_(out.multipliers_ineq)[0]]
    np.testing.assert_allclose((np_(out.y)[0] - x[0]) + matrix.T @ mult, 0.0, atol=1e-9)
    assert bool(out.gradient_eligible[0])
    g = rng.normal(size=(1, 3))
    xt = T(x).requires_grad_(True)
    (layer(xt) * T(g)).sum().backward()
    analytic = np_(xt.grad)
    for i in range(3):
        d = np.zeros_like(x)
        d[0, i] = 1e-4
        fd = float(((layer(T(x + d)) - layer(T(x - d))) * T(g)).sum()) / 2e-4
        np.testing.assert_allclose(analytic[0, i], fd, atol=2e-5)


def test_scalar_opt_out_and_no_bound_parameter_gradient():
    """tests/test_regression_cp_diagonal_steps.py:83-112"""
    p = Projection()
    t = p.add_parameter(["a"])
    y = p.add_variable(["u", "v"])
    p.objective = 0.0
    p.constraints.add(t.a * y.u + y.v == 1)
    for diagonal in (False, True):
        cfg = ChambollePockConfig(diagonal_preconditioning=diagonal,
                                  implicit_gradient=ImplicitGradientConfig(
                                      differentiate_problem_parameters=True))
        layer = prepare_projection(p, method="chambolle-pock", config=cfg, batch_size=1)
        x = T([[0.2, 0.3]])
        theta = T([[2.0]])

        def expected(a):
            row = torch.stack([a[:, 0], torch.ones_like(a[:, 0])], dim=1)
            return x - row * (a[0, 0] * 0.2 + 0.3 - 1) / (1 + a[0, 0] ** 2)

        np.testing.assert_allclose(np_(layer(x, theta)), np_(expected(theta)), atol=1e-8)
        np.testing.assert_allclose(jacobian(lambda a: layer(x, a), theta),
                                   jacobian(expected, theta), atol=2e-7)


@pytest.mark.parametrize("dtype,tolerance", [(torch.float32, 5e-5), (torch.float64, 2e-6)])
def test_numerical_regression_fp32_fp64(dtype, tolerance):
    """.github/scripts/numerical_regression.py:23-80 (chambolle-pock case)"""
    cfg = ChambollePockConfig(max_iterations=3000,
                              tolerance=1e-6 if dtype == torch.float32 else 1e-10)
    if dtype == torch.float32:
        cfg = replace(cfg, implicit_gradient=ImplicitGradientConfig(adjoint_tolerance=1e-5,
                                                                    inexact_tolerance=1e-5),
                      linear_solver=LinearSolverConfig(tolerance=1e-6))
    layer = Distance(make_problem(), "chambolle-pock", cfg).prepare(batch_size=1, dtype=dtype)
    target = T([[0.8, 0.7]], dtype)
    context = T(np.ones((1, 1)), dtype)
    np.testing.assert_allclose(np_(layer(target, context)), [[0.55, 0.45]], atol=tolerance, rtol=0)
    jac = jacobian(lambda x: layer(x[None], context)[0], target[0])
    np.testing.assert_allclose(jac, [[0.5, -0.5], [-0.5, 0.5]], atol=tolerance, rtol=0)


def test_training_contract_errors():
    """tests/test_training_metric_contracts.py:44-58 (argument validation)"""
    prepared = Distance(make_problem(inequalities=True), "chambolle-pock", cp_config()).prepare(
        batch_size=1)
    target = T([[0.8, 0.7]])
    context = T(np.ones((1, 1)))
    for params, y in [(None, target), (T(np.ones((2, 1))), target), (context, T(np.ones((2, 2))))]:
        with pytest.raises(ValueError):
            prepared.solve(y, params)
    with pytest.raises(ValueError, match="project_training"):
        prepared.solve(target, context, initial_state=T(np.zeros((1, 1))))
    eq, iq = T(np.zeros((1, 1))), T(np.ones((1, 2)))
    projected = np_(prepared.project_training(target, context, multipliers_eq=eq,
                                              multipliers_ineq=iq).y_tilde)
    for equality, inequality in [(None, iq), (eq, None)]:
        np.testing.assert_allclose(
            np_(prepared.project_training(target, context, multipliers_eq=equality,
                                          multipliers_ineq=inequality).y_tilde),
            projected, atol=2e-6)
