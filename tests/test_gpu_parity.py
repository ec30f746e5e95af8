"""CUDA kernels vs the CPU oracle at the C-ABI boundary and through the public API.

Forward results at a fixed iteration count are compared bit for bit (the
kernels and the oracle perform the same IEEE operations in the same order);
quantities that involve a parallel sum in the kernel (the normalised gap, the
power-iteration norm, GMRES dot products) are compared with tolerances.
"""

import numpy as np
import pytest
import torch
from dataclasses import replace

from helpers import OracleLayer, ell_to_csr, random_sparse_problem, random_theta
from purin_b200 import ChambollePockConfig, LinearSolverConfig, prepare_projection
from purin_b200.workloads import make_workload

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _t(a, dtype):
    return torch.as_tensor(np.ascontiguousarray(a), dtype=dtype, device=DEV)


def _layer(problem, cfg, batch, dtype):
    return prepare_projection(problem, method="chambolle-pock", config=cfg, batch_size=batch,
                              dtype=dtype, backend=DEV)


def boundary_forward(layer, oracle, saved):
    """Run purin_cp_forward on the oracle's scaled arrays; returns numpy CPOutput fields."""
    dt = layer._tdtype
    data = _t(ell_to_csr(saved["values"], list(oracle.proj.mask.sum(axis=1))), dt)
    batch, n = saved["target"].shape
    m = layer._m
    out = dict(y=torch.empty((batch, n), dtype=dt, device=DEV),
               dual=torch.empty((batch, m), dtype=dt, device=DEV),
               iterations=torch.empty((batch,), dtype=torch.int32, device=DEV),
               residual=torch.empty((batch,), dtype=dt, device=DEV),
               gap=torch.empty((batch,), dtype=dt, device=DEV),
               converged=torch.empty((batch,), dtype=torch.uint8, device=DEV))
    layer._forward_native(data, _t(saved["rhs"], dt), _t(saved["target"], dt),
                          _t(saved["lower"], dt), _t(saved["upper"], dt),
                          _t(saved["initial"], dt), _t(saved["tolerance"], dt),
                          _t(saved["feasible"].astype(np.uint8), torch.uint8),
                          out["y"], out["dual"], out["iterations"], out["residual"], out["gap"],
                          out["converged"])
    torch.cuda.synchronize()
    return {k: v.cpu().numpy() for k, v in out.items()}, data


def boundary_adjoint(layer, oracle, saved, cot):
    dt = layer._tdtype
    lengths = list(oracle.proj.mask.sum(axis=1))
    data = _t(ell_to_csr(saved["values"], lengths), dt)
    out = saved["out"]
    grads = layer._adjoint_native(
        data, _t(saved["rhs"], dt), _t(saved["target"], dt), _t(saved["lower"], dt),
        _t(saved["upper"], dt), _t(out.y, dt), _t(out.dual, dt),
        _t(out.converged.astype(np.uint8), torch.uint8), _t(cot, dt), need_values=True,
        need_rhs=True, need_target=True, need_lower=True, need_upper=True)
    torch.cuda.synchronize()
    status, lres = layer._last_linear
    names = ("values", "rhs", "target", "lower", "upper")
    return ({k: g.cpu().numpy() for k, g in zip(names, grads)}, status.cpu().numpy(),
            lres.cpu().numpy())


FORWARD_CASES = [
    # (name, workload index, batch, dtype, config overrides)
    ("config0-fixed-f64", 0, 16, np.float64, {}),
    ("config0-accel-f64", 0, 16, np.float64, {"accelerated": True}),
    ("config0-fixed-f32", 0, 16, np.float32, {}),
    ("config0-diag-f64", 0, 16, np.float64, {"diagonal_preconditioning": True}),
    ("config0-power-f64", 0, 16, np.float64, {"norm_bound": False}),
    ("config0-power-f32", 0, 16, np.float32, {"norm_bound": False}),
    ("config1-accel-f64", 1, 8, np.float64, {"max_iterations": 200}),
    ("config1-accel-f32", 1, 8, np.float32, {"max_iterations": 200}),
    ("config0-converge-f64", 0, 16, np.float64, {"tolerance": 1e-4, "max_iterations": 4000}),
]


@pytest.mark.parametrize("name,index,batch,dtype,overrides", FORWARD_CASES,
                         ids=[c[0] for c in FORWARD_CASES])
def test_forward_boundary_matches_oracle(name, index, batch, dtype, overrides):
    w = make_workload(index, batch)
    cfg = replace(w.config, **overrides)
    oracle = OracleLayer(w.problem, cfg, dtype)
    expected, saved = oracle.solve(w.candidates, w.theta)
    tdt = torch.float64 if dtype == np.float64 else torch.float32
    layer = _layer(w.problem, cfg, batch, tdt)
    got, _ = boundary_forward(layer, oracle, saved)
    out = saved["out"]
    np.testing.assert_array_equal(got["iterations"], out.iterations)
    np.testing.assert_array_equal(got["converged"].astype(bool), out.converged)
    if not overrides.get("norm_bound", True):
        # tau/sigma come from a parallel-sum power iteration: agree to rounding.
        tol = 1e-9 if dtype == np.float64 else 2e-3
        np.testing.assert_allclose(got["y"], out.y, rtol=0, atol=tol)
        return
    np.testing.assert_array_equal(got["y"], out.y)
    np.testing.assert_array_equal(got["dual"], out.dual)
    np.testing.assert_array_equal(got["residual"], out.residual)
    rtol = 1e-12 if dtype == np.float64 else 1e-5
    np.testing.assert_allclose(got["gap"], out.gap, rtol=rtol, atol=rtol)


TILE_CASES = [
    ("fixed-f64", np.float64, {}),
    ("converge-f64", np.float64, {"tolerance": 1e-4, "max_iterations": 4000}),
    ("converge-accel-f32", np.float32, {"tolerance": 1e-3, "max_iterations": 3000,
                                        "accelerated": True}),
    ("diag-f64", np.float64, {"diagonal_preconditioning": True}),
]


_TILE_ORACLE = {}


@pytest.mark.parametrize("samples_per_tile,threads", [(1, 256), (2, 256), (4, 256), (8, 256),
                                                     (1, 512), (1, 1024), (2, 512), (4, 512),
                                                     (2, 768), (4, 768), (2, 1024), (4, 1024)])
@pytest.mark.parametrize("name,dtype,overrides", TILE_CASES, ids=[c[0] for c in TILE_CASES])
def test_forward_tile_widths_match_oracle(monkeypatch, samples_per_tile, threads, name, dtype,
                                          overrides):
    """Every tile shape (samples per CTA, threads per CTA), with a ragged last tile, gives the
    oracle's bits."""
    monkeypatch.setenv("PURIN_CP_SAMPLES_PER_TILE", str(samples_per_tile))
    monkeypatch.setenv("PURIN_CP_TILE_THREADS", str(threads))
    batch = 13
    w = make_workload(0, batch)
    cfg = replace(w.config, **overrides)
    if name not in _TILE_ORACLE:
        oracle = OracleLayer(w.problem, cfg, dtype)
        _TILE_ORACLE[name] = (oracle, oracle.solve(w.candidates, w.theta)[1])
    oracle, saved = _TILE_ORACLE[name]
    tdt = torch.float64 if dtype == np.float64 else torch.float32
    layer = _layer(w.problem, cfg, batch, tdt)
    got, _ = boundary_forward(layer, oracle, saved)
    out = saved["out"]
    np.testing.assert_array_equal(got["iterations"], out.iterations)
    np.testing.assert_array_equal(got["converged"].astype(bool), out.converged)
    np.testing.assert_array_equal(got["y"], out.y)
    np.testing.assert_array_equal(got["dual"], out.dual)
    np.testing.assert_array_equal(got["residual"], out.residual)
    rtol = 1e-12 if dtype == np.float64 else 1e-5
    np.testing.assert_allclose(got["gap"], out.gap, rtol=rtol, atol=rtol)


@pytest.mark.parametrize("index,batch,dtype,overrides", [
    (0, 16, np.float64, {}), (1, 4, np.float64, {}), (0, 16, np.float32, {}),
    # Values shared by the batch with diagonal preconditioning: the diagonal
    # steps are computed once per call into the workspace.
    (0, 16, np.float64, {"diagonal_preconditioning": True}),
    (1, 8, np.float32, {"diagonal_preconditioning": True, "accelerated": False}),
    (0, 16, np.float64, {"diagonal_preconditioning": True, "tolerance": 1e-4,
                         "max_iterations": 4000})])
def test_public_solve_matches_oracle(index, batch, dtype, overrides):
    """End to end: torch preprocessing + forward + post-processing kernels."""
    w = make_workload(index, batch)
    cfg = replace(w.config, max_iterations=min(w.config.max_iterations, 300))
    cfg = replace(cfg, **overrides)
    oracle = OracleLayer(w.problem, cfg, dtype)
    expected, _ = oracle.solve(w.candidates, w.theta)
    tdt = torch.float64 if dtype == np.float64 else torch.float32
    layer = _layer(w.problem, cfg, batch, tdt)
    got = layer.solve(_t(w.candidates, tdt), _t(w.theta, tdt))
    np.testing.assert_array_equal(got.y.cpu().numpy(), expected["y"])
    for field in ("multipliers_eq", "multipliers_ineq", "slacks", "residual_inf_norm"):
        np.testing.assert_array_equal(getattr(got, field).cpu().numpy(), expected[field],
                                      err_msg=field)
    np.testing.assert_array_equal(got.status.cpu().numpy(), expected["status"])
    np.testing.assert_array_equal(got.iterations.cpu().numpy(), expected["iterations"])
    np.testing.assert_array_equal(got.finite.cpu().numpy(), expected["finite"])
    np.testing.assert_array_equal(got.gradient_eligible.cpu().numpy(),
                                  expected["gradient_eligible"])


def _converging_problem(seed, n=8, me=2, mi=4, dtype=np.float64):
    rng = np.random.default_rng(seed)
    problem, mats = random_sparse_problem(rng, n, me, mi, 3)
    batch = 6
    theta = random_theta(rng, mats, batch)
    target = 1.5 * rng.normal(size=(batch, n))
    return problem, theta.astype(dtype), target.astype(dtype)


@pytest.mark.parametrize("seed,accelerated", [(1, False), (2, False), (3, False), (1, True),
                                              (5, True)])
def test_adjoint_boundary_matches_oracle(seed, accelerated):
    problem, theta, target = _converging_problem(seed)
    cfg = ChambollePockConfig(max_iterations=20000, tolerance=1e-11, accelerated=accelerated)
    oracle = OracleLayer(problem, cfg)
    expected, saved = oracle.solve(target, theta)
    assert expected["gradient_eligible"].any()
    rng = np.random.default_rng(100 + seed)
    cot = rng.normal(size=target.shape)
    stats = {}
    want = oracle.proj.vjp(saved, cot, stats=stats)
    layer = _layer(problem, cfg, target.shape[0], torch.float64)
    got, status, lres = boundary_adjoint(layer, oracle, saved, cot)
    np.testing.assert_array_equal(status, stats["code"])
    for key in ("values", "rhs", "target", "lower", "upper"):
        exp = want[key]
        if key == "values":
            exp = ell_to_csr(exp, list(oracle.proj.mask.sum(axis=1)))
        np.testing.assert_allclose(got[key], exp, rtol=0, atol=1e-9, err_msg=key)


def test_adjoint_gmres_budget_matches_oracle():
    """Hard case: GMRES stops at its 100-iteration budget without converging.

    A non-converged restarted GMRES is sensitive to rounding: perturbing the
    oracle's own tau by 2e-16 (relative) moves its final residual by up to 9%.
    What must agree is the outcome: the same status codes, residuals of the
    same size, and the same gradients -- here zero, because every residual
    stays above the adjoint tolerance (bounds.py:148-154).
    """
    w = make_workload(0, 6)
    cfg = replace(w.config, max_iterations=6000, tolerance=1e-5)
    oracle = OracleLayer(w.problem, cfg)
    expected, saved = oracle.solve(w.candidates, w.theta)
    assert expected["gradient_eligible"].any()
    cot = np.random.default_rng(7).normal(size=w.candidates.shape)
    stats = {}
    want = oracle.proj.vjp(saved, cot, stats=stats)
    assert stats["completed"] == 100 and np.any(stats["code"] == 1)
    layer = _layer(w.problem, cfg, 6, torch.float64)
    got, status, lres = boundary_adjoint(layer, oracle, saved, cot)
    np.testing.assert_array_equal(status, stats["code"])
    np.testing.assert_allclose(lres, stats["residual"], rtol=0.25, atol=1e-14)
    for key in ("values", "rhs", "target", "lower", "upper"):
        exp = want[key]
        if key == "values":
            exp = ell_to_csr(exp, list(oracle.proj.mask.sum(axis=1)))
        np.testing.assert_array_equal(got[key], exp, err_msg=key)


def test_autograd_chain_matches_fd():
    """Public API gradient w.r.t. candidate and parameters vs central differences."""
    problem, theta, target = _converging_problem(5)
    cfg = replace(ChambollePockConfig(max_iterations=20000, tolerance=1e-12),
                  implicit_gradient=replace(ChambollePockConfig().implicit_gradient,
                                            differentiate_problem_parameters=True),
                  linear_solver=LinearSolverConfig(tolerance=1e-12))
    layer = _layer(problem, cfg, target.shape[0], torch.float64)
    x = _t(target, torch.float64).requires_grad_(True)
    th = _t(theta, torch.float64).requires_grad_(True)
    g = torch.as_tensor(np.random.default_rng(9).normal(size=target.shape), device=DEV)
    result = layer.solve(x, th)
    assert bool(result.gradient_eligible.all())
    (result.y * g).sum().backward()
    eps = 1e-6
    for which, base, grad in (("x", target, x.grad), ("theta", theta, th.grad)):
        fd = np.zeros_like(base)
        for b in range(base.shape[0]):
            for i in range(base.shape[1]):
                plus, minus = base.copy(), base.copy()
                plus[b, i] += eps
                minus[b, i] -= eps
                args_p = (plus, theta) if which == "x" else (target, plus)
                args_m = (minus, theta) if which == "x" else (target, minus)
                yp = layer(_t(args_p[0], torch.float64), _t(args_p[1], torch.float64))
                ym = layer(_t(args_m[0], torch.float64), _t(args_m[1], torch.float64))
                fd[b, i] = float(((yp - ym) * g).sum()) / (2 * eps)
        np.testing.assert_allclose(grad.cpu().numpy(), fd, atol=2e-6, err_msg=which)


def test_parameter_dependent_coefficients_per_sample():
    """Coefficients that depend on the parameters differ per sample: the per-sample
    values path of the forward kernel through the public API (presolve, row scaling,
    bound rows whose coefficient is a parameter)."""
    from purin_b200.problems import Projection

    p = Projection()
    t = p.add_parameter(["a", "b", "c", "d"])
    y = p.add_variable(["u", "v", "w", "z"])
    p.objective = 0.0
    p.constraints.add(t.a * y.u + y.v - y.w == t.b)
    p.constraints.add(y.u + t.c * y.w + y.z <= 1.5)
    p.constraints.add(y.v - y.z >= -t.d)
    p.constraints.add(t.c * y.z <= 2.0)  # singleton row with a parameter coefficient
    p.constraints.add(y.u >= -1.0, y.u <= 1.0, y.w >= -2.0)
    batch = 8
    rng = np.random.default_rng(7)
    theta = np.column_stack([rng.uniform(0.5, 2.0, batch), rng.normal(size=batch),
                             rng.uniform(0.5, 2.0, batch), rng.uniform(0.0, 1.0, batch)])
    candidates = 2.0 * rng.normal(size=(batch, 4))
    cfg = ChambollePockConfig(max_iterations=400)
    oracle = OracleLayer(p, cfg, np.float64)
    expected, _ = oracle.solve(candidates, theta)
    layer = _layer(p, cfg, batch, torch.float64)
    got = layer.solve(_t(candidates, torch.float64), _t(theta, torch.float64))
    for field in ("y", "multipliers_eq", "multipliers_ineq", "slacks", "residual_inf_norm",
                  "status", "iterations"):
        np.testing.assert_array_equal(getattr(got, field).cpu().numpy(), expected[field],
                                      err_msg=field)


def test_bounded_device_wait_reports_and_context_stays_usable(monkeypatch):
    """A grid barrier that can never complete (one arrival more than the grid has,
    PURIN_CP_TEST_UNREACHABLE_BARRIER) gives up after its time limit: the call
    raises on the host through device_error, and the next call on the same
    context gives the oracle's gradients."""
    problem, theta, target = _converging_problem(1)
    cfg = ChambollePockConfig(max_iterations=20000, tolerance=1e-11)
    oracle = OracleLayer(problem, cfg)
    expected, saved = oracle.solve(target, theta)
    cot = np.random.default_rng(101).normal(size=target.shape)
    stats = {}
    want = oracle.proj.vjp(saved, cot, stats=stats)
    layer = _layer(problem, cfg, target.shape[0], torch.float64)
    monkeypatch.setenv("PURIN_CP_TEST_UNREACHABLE_BARRIER", "50")
    with pytest.raises(RuntimeError, match="bounded device wait"):
        boundary_adjoint(layer, oracle, saved, cot)
    monkeypatch.delenv("PURIN_CP_TEST_UNREACHABLE_BARRIER")
    got, status, _ = boundary_adjoint(layer, oracle, saved, cot)
    np.testing.assert_array_equal(status, stats["code"])
    for key in ("rhs", "target", "lower", "upper"):
        np.testing.assert_allclose(got[key], want[key], rtol=0, atol=1e-9, err_msg=key)


def test_gmres_budget_of_one_matches_oracle():
    """LinearSolverConfig(max_iterations=1): one Arnoldi step per solve; status codes,
    residual-gated gradients (bounds.py:148-154) and budget as in the oracle."""
    problem, theta, target = _converging_problem(3)
    cfg = ChambollePockConfig(max_iterations=20000, tolerance=1e-11,
                              linear_solver=LinearSolverConfig(max_iterations=1))
    oracle = OracleLayer(problem, cfg)
    expected, saved = oracle.solve(target, theta)
    assert expected["gradient_eligible"].any()
    cot = np.random.default_rng(103).normal(size=target.shape)
    stats = {}
    want = oracle.proj.vjp(saved, cot, stats=stats)
    assert stats["completed"] == 1
    layer = _layer(problem, cfg, target.shape[0], torch.float64)
    got, status, lres = boundary_adjoint(layer, oracle, saved, cot)
    np.testing.assert_array_equal(status, stats["code"])
    np.testing.assert_allclose(lres, stats["residual"], rtol=1e-9, atol=1e-14)
    for key in ("rhs", "target", "lower", "upper"):
        np.testing.assert_allclose(got[key], want[key], rtol=0, atol=1e-9, err_msg=key)


@pytest.mark.parametrize("seed,accelerated,tol", [(1, False, 1e-5), (2, True, 3e-5),
                                                 (5, False, 1e-5)])
def test_adjoint_fp32_matches_oracle(seed, accelerated, tol):
    """fp32 implicit VJP against the fp32 oracle: every cotangent within 1e-4 of
    the field's largest gradient (the fp32 bar), identical GMRES status codes."""
    from purin_b200 import ImplicitGradientConfig

    problem, theta, target = _converging_problem(seed, dtype=np.float32)
    cfg = ChambollePockConfig(max_iterations=20000, tolerance=tol, accelerated=accelerated,
                              linear_solver=LinearSolverConfig(tolerance=1e-5),
                              implicit_gradient=ImplicitGradientConfig(adjoint_tolerance=1e-4))
    oracle = OracleLayer(problem, cfg, np.float32)
    expected, saved = oracle.solve(target, theta)
    assert expected["gradient_eligible"].any()
    cot = np.random.default_rng(100 + seed).normal(size=target.shape).astype(np.float32)
    stats = {}
    want = oracle.proj.vjp(saved, cot, stats=stats)
    layer = _layer(problem, cfg, target.shape[0], torch.float32)
    got, status, _ = boundary_adjoint(layer, oracle, saved, cot)
    np.testing.assert_array_equal(status, stats["code"])
    for key in ("values", "rhs", "target", "lower", "upper"):
        exp = want[key]
        if key == "values":
            exp = ell_to_csr(exp, list(oracle.proj.mask.sum(axis=1)))
        scale = max(float(np.abs(exp).max()), 1e-6)
        np.testing.assert_allclose(got[key], exp, rtol=0, atol=1e-4 * scale, err_msg=key)
