"""ADMM projection (method="admm") on the GPU against the ADMM oracle and the reference cases.

The forward kernel (admm_forward.cu) and the KKT mode of the adjoint kernel run
sparse_admm and its VJP (src/purin/solvers/admm/kernels.py:43-283,
solver.py:175-255).  Their inner products are parallel sums, so the PCG and
GMRES iterates round differently from the oracle's: converged solutions are
compared within the solver's tolerance (the reference's own test tolerances for
the analytic cases), iteration counts exactly where the acceptance is not at
the edge of the tolerance.
"""

import json
from dataclasses import replace
from pathlib import Path

import numpy as np
import pytest
import torch

from helpers import OracleADMMLayer, ell_to_csr, random_sparse_problem, random_theta
from purin_b200 import ADMMConfig, ImplicitGradientConfig, LinearSolverConfig, prepare_projection
from purin_b200.problems import Projection

pytestmark = pytest.mark.gpu
DEV = "cuda"
CASES = json.loads((Path(__file__).parent / "golden" / "reference_cases.json").read_text())


def _t(a, dtype=torch.float64):
    return torch.as_tensor(np.ascontiguousarray(a), dtype=dtype, device=DEV)


def _layer(problem, cfg, batch, dtype=torch.float64):
    return prepare_projection(problem, method="admm", config=cfg, batch_size=batch, dtype=dtype,
                              backend=DEV)


def _affine_problem():
    p = Projection(method="admm")
    t = p.add_parameter(["b"])
    y = p.add_variable(["u", "v"])
    p.objective = 0.0
    p.constraints.add(y.u + y.v == t.b, y.u >= 0)
    return p


@pytest.mark.parametrize("adaptive_rho", [False, True])
def test_reference_affine_projection_and_gradients(adaptive_rho):
    """``tests/test_regression_admm.py:25-57`` through the public API."""
    case = CASES["admm_affine_projection"]
    cfg = ADMMConfig(adaptive_rho=adaptive_rho, implicit_gradient=ImplicitGradientConfig(
        differentiate_problem_parameters=True))
    layer = _layer(_affine_problem(), cfg, 2)
    x = _t(case["target"]).requires_grad_(True)
    theta = _t(case["parameters"]).requires_grad_(True)
    out = layer.solve(x, theta)
    np.testing.assert_allclose(out.y.detach().cpu().numpy(), case["y"], atol=case["atol"])
    assert (out.status.cpu().numpy() == 0).all()
    assert float(out.residual_inf_norm.max()) <= cfg.tolerance
    jac = torch.autograd.functional.jacobian(lambda v: layer(v, theta.detach()), x.detach())
    np.testing.assert_allclose(jac[0, :, 0, :].cpu().numpy(), case["jacobian_sample0"],
                               atol=case["atol"])
    np.testing.assert_allclose(jac[1, :, 1, :].cpu().numpy(), case["jacobian_sample1"],
                               atol=case["atol"])
    dth = torch.autograd.functional.jacobian(lambda t: layer(x.detach(), t), theta.detach())
    np.testing.assert_allclose(dth[0, :, 0, 0].cpu().numpy(), case["theta_derivative"][0],
                               atol=case["atol"])
    np.testing.assert_allclose(dth[1, :, 1, 0].cpu().numpy(), case["theta_derivative"][1],
                               atol=case["atol"])


def test_reference_two_sided_box_uses_paired_rows():
    """``tests/test_regression_admm_rows.py:12-40``: verified pairs, original multipliers."""
    case = CASES["admm_two_sided_box"]
    p = Projection()
    y = p.add_variable(["x", "y"])
    p.objective = 0.0
    p.constraints.add(y.x <= 1, -y.x <= 0, y.y <= 2, -y.y <= 1)
    layer = _layer(p, ADMMConfig(), 3)
    assert len(layer._paired_rows.keep) == case["kept_rows"]
    x = _t(case["target"]).requires_grad_(True)
    out = layer.solve(x)
    for key in ("y", "multipliers_ineq", "slacks"):
        np.testing.assert_allclose(getattr(out, key).detach().cpu().numpy(), case[key],
                                   atol=case["atol"], err_msg=key)
    out.y.sum().backward()
    np.testing.assert_allclose(x.grad.cpu().numpy(), case["gradient_of_sum"], atol=1e-8)


@pytest.mark.parametrize("adaptive", [False, True])
def test_reference_periodic_acceptance(adaptive):
    """``tests/test_regression_admm_diagnostics.py:15-44``."""
    case = CASES["admm_periodic_acceptance"]
    p = Projection()
    y = p.add_variable(["u", "v"])
    p.objective = 0.0
    p.constraints.add(y.u + y.v == 1, y.u >= 0, y.u <= 1)
    outs = []
    for interval in (1, 25):
        cfg = ADMMConfig(adaptive_rho=adaptive, rho_update_interval=7, check_interval=interval)
        out = _layer(p, cfg, 3).solve(_t(case["target"]))
        assert bool(out.gradient_eligible.all())
        outs.append(out.y.cpu().numpy())
    np.testing.assert_allclose(outs[0], outs[1], atol=case["atol"])
    np.testing.assert_allclose(outs[1], case["y"], atol=case["atol"])


def test_limits_nonfinite_and_no_constraints():
    """``tests/test_regression_admm.py:69-100``."""
    layer = _layer(_affine_problem(), ADMMConfig(max_iterations=1), 1)
    out = layer.solve(_t([[-2.0, 0.0]]), _t([[1.0]]))
    assert int(out.status[0]) == 1 and not bool(out.gradient_eligible[0])
    out = layer.solve(_t([[float("nan"), 0.0]]), _t([[1.0]]))
    assert int(out.status[0]) == 3
    p = Projection()
    p.add_variable(["u", "v"])
    p.objective = 0.0
    free = _layer(p, ADMMConfig(), 1)
    x = _t([[0.2, 0.7]]).requires_grad_(True)
    yv = free(x)
    np.testing.assert_allclose(yv.detach().cpu().numpy(), [[0.2, 0.7]], atol=1e-12)
    yv.sum().backward()
    np.testing.assert_allclose(x.grad.cpu().numpy(), 1.0, atol=1e-9)


def _random_case(seed, n=40, me=6, mi=12, nnz=5, batch=5):
    rng = np.random.default_rng(seed)
    problem, mats = random_sparse_problem(rng, n, me, mi, nnz)
    theta = random_theta(rng, mats, batch)
    target = 1.5 * rng.normal(size=(batch, n))
    return problem, theta, target


@pytest.mark.parametrize("seed,adaptive,interval,n", [(1, False, 25, 40), (2, True, 25, 40),
                                                      (3, False, 1, 40), (4, False, 25, 300)])
def test_random_problems_match_the_oracle(seed, adaptive, interval, n):
    """Random sparse problems with box rows (a row graph too wide for the band, so the
    PCG path; the boxes pair into two-sided rows): the projection, multipliers, iteration
    counts and implicit gradients agree with the oracle.  n = 40 runs one-warp CTAs with
    the operands staged in shared memory; n = 300 (more than 256 entries per vector) the
    256-thread CTAs reading them from global memory."""
    problem, theta, target = _random_case(seed, n=n)
    cfg = ADMMConfig(adaptive_rho=adaptive, check_interval=interval, implicit_gradient=
                     ImplicitGradientConfig(differentiate_problem_parameters=True),
                     linear_solver=LinearSolverConfig(tolerance=1e-11, max_iterations=300))
    oracle = OracleADMMLayer(problem, cfg)
    want, saved = oracle.solve(target, theta)
    assert want["gradient_eligible"].all()
    layer = _layer(problem, cfg, target.shape[0])
    x = _t(target).requires_grad_(True)
    th = _t(theta).requires_grad_(True)
    out = layer.solve(x, th)
    np.testing.assert_allclose(out.y.detach().cpu().numpy(), want["y"], atol=1e-8)
    np.testing.assert_allclose(out.multipliers_eq.cpu().numpy(), want["multipliers_eq"],
                               atol=1e-7)
    np.testing.assert_allclose(out.multipliers_ineq.cpu().numpy(), want["multipliers_ineq"],
                               atol=1e-7)
    np.testing.assert_array_equal(out.status.cpu().numpy(), want["status"])
    assert layer._full.width < 0  # PCG, not the band
    # Converged-mode iteration counts within 2 % (acceptance is tested on rounding-
    # dependent residuals; with a check interval of 25 the counts coincide).
    counts, expected = out.iterations.cpu().numpy(), want["iterations"]
    assert np.all(np.abs(counts - expected) <= np.maximum(0.02 * expected, 1)), (counts, expected)
    cot = np.random.default_rng(100 + seed).normal(size=target.shape)
    (out.y * _t(cot)).sum().backward()
    grads = oracle.proj.vjp(saved, cot)
    np.testing.assert_allclose(x.grad.cpu().numpy(), grads["target"], atol=1e-7)


def test_banded_path_matches_the_oracle():
    """A chain of 3-wide rows: the row graph has a band of width 2, so the x-update is the
    banded Cholesky solve (factor.py) instead of PCG."""
    n, batch = 16, 4
    p = Projection()
    names = [f"x{i}" for i in range(n)]
    y = p.add_variable(names)
    p.objective = 0.0
    for i in range(n - 2):
        a, b, c = (getattr(y, names[i + k]) for k in range(3))
        p.constraints.add(a - 2 * b + c <= 0.1 * (i % 3))
    rng = np.random.default_rng(5)
    target = 2.0 * rng.normal(size=(batch, n))
    cfg = ADMMConfig(implicit_gradient=ImplicitGradientConfig())
    layer = _layer(p, cfg, batch)
    assert layer._full.width == 2
    oracle = OracleADMMLayer(p, cfg)
    assert oracle.proj.factor_plan is not None and oracle.proj.factor_plan.width == 2
    want, saved = oracle.solve(target)
    out = layer.solve(_t(target))
    np.testing.assert_allclose(out.y.cpu().numpy(), want["y"], atol=1e-8)
    np.testing.assert_array_equal(out.iterations.cpu().numpy(), want["iterations"])
    np.testing.assert_array_equal(out.status.cpu().numpy(), want["status"])


def test_float32_projection():
    problem, theta, target = _random_case(7)
    cfg = ADMMConfig(tolerance=1e-5)
    oracle = OracleADMMLayer(problem, cfg, np.float32)
    want, _ = oracle.solve(target.astype(np.float32), theta.astype(np.float32))
    out = _layer(problem, cfg, target.shape[0], torch.float32).solve(
        _t(target, torch.float32), _t(theta, torch.float32))
    np.testing.assert_allclose(out.y.cpu().numpy(), want["y"], atol=1e-4)
