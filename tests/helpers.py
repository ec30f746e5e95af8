"""Shared test helpers: reference-test problems and the canonical -> oracle bridge."""

from __future__ import annotations

import numpy as np

from oracle.projection import OracleConfig, OracleProjection
from oracle.sparse import layout
from purin_b200.problems import Projection, canonical_of


def make_problem(*, inequalities=False, nonlinear=False):
    """``tests/test_projections.py:33-45`` of the reference."""
    problem = Projection()
    p = problem.add_parameter(["b"])
    y = problem.add_variable(["u", "v"])
    problem.objective = 0.0
    if nonlinear:
        problem.constraints.add(y.u**2 + y.v**2 <= p.b)
    else:
        problem.constraints.add(y.u + y.v == p.b)
        if inequalities:
            problem.constraints.add(y.u >= 0)
            problem.constraints.add(y.v >= 0)
    return problem


def regression_problem():
    """``tests/test_regression_chambolle_pock.py:16-22`` of the reference."""
    p = Projection(method="chambolle-pock")
    t = p.add_parameter(["b"])
    y = p.add_variable(["u", "v"])
    p.objective = 0.0
    p.constraints.add(y.u + y.v == t.b, y.u >= 0)
    return p


def oracle_config(cfg) -> OracleConfig:
    """OracleConfig from a purin_b200 ChambollePockConfig."""
    return OracleConfig(
        tolerance=cfg.tolerance, max_iterations=cfg.max_iterations, accelerated=cfg.accelerated,
        safety=cfg.safety, norm_iterations=cfg.norm_iterations, norm_seed=cfg.norm_seed,
        row_scaling=cfg.row_scaling, norm_bound=cfg.norm_bound,
        diagonal_preconditioning=cfg.diagonal_preconditioning,
        linear_tolerance=cfg.linear_solver.tolerance, linear_atol=cfg.linear_solver.atol,
        linear_restart=cfg.linear_solver.restart,
        linear_max_iterations=cfg.linear_solver.max_iterations,
        adjoint_tolerance=cfg.implicit_gradient.adjoint_tolerance)


def to_ell(canonical, values_csr):
    """CSR-slot values (1|B, nnz) -> padded ELL (B, m_all, width) of the reference layout."""
    rows = list(canonical.equality_sparsity) + list(canonical.inequality_sparsity)
    support, mask, positions = layout(rows, canonical.variable_size)
    batch = values_csr.shape[0]
    out = np.zeros((batch, support.shape[0] * support.shape[1]), dtype=values_csr.dtype)
    out[:, positions] = values_csr
    return out.reshape(batch, support.shape[0], support.shape[1])


class OracleLayer:
    """A problem + config evaluated by the oracle (values from the product frontend)."""

    def __init__(self, problem, cfg, dtype=np.float64, partitionable=True):
        self.canonical = canonical_of(problem)
        self.cfg = cfg
        self.dtype = np.dtype(dtype)
        c = self.canonical
        self.proj = OracleProjection(c.equality_sparsity, c.inequality_sparsity, c.variable_size,
                                     oracle_config(cfg), partitionable)

    def arrays(self, theta, batch):
        theta = np.zeros((batch, 0), self.dtype) if theta is None else np.asarray(theta, self.dtype)
        values, rhs = self.canonical.evaluate(theta)
        values = np.broadcast_to(values, (batch, values.shape[1])).astype(self.dtype)
        rhs = np.broadcast_to(rhs, (batch, rhs.shape[1])).astype(self.dtype)
        return to_ell(self.canonical, values), rhs

    def solve(self, target, theta=None, multipliers_eq=None, multipliers_ineq=None, **kw):
        target = np.asarray(target, self.dtype)
        values, rhs = self.arrays(theta, target.shape[0])
        return self.proj.solve(values, rhs, target, multipliers_eq, multipliers_ineq, **kw)

    def __call__(self, target, theta=None):
        return self.solve(target, theta)[0]["y"]

    def target_jacobian(self, target, theta=None):
        """d y_b / d target_b per sample via the oracle's implicit VJP: (B, n, n)."""
        result, saved = self.solve(target, theta)
        target = np.asarray(target, self.dtype)
        batch, n = target.shape
        jac = np.zeros((batch, n, n), self.dtype)
        for i in range(n):
            cot = np.zeros_like(target)
            cot[:, i] = 1
            jac[:, i, :] = self.proj.vjp(saved, cot)["target"]
        return jac


def ell_to_csr(ell, row_lengths):
    """Padded ELL values (B, m, width) -> CSR-slot values (B, nnz)."""
    parts = [ell[:, i, :k] for i, k in enumerate(row_lengths)]
    if not parts:
        return np.zeros((ell.shape[0], 0), ell.dtype)
    return np.concatenate(parts, axis=1)


def random_sparse_problem(rng, n, me, mi, nnz_per_row, bounds=True, lower=-1.0, upper=1.0):
    """Random ParametricQP-like problem as a canonical Projection with box rows.

    Returns (problem, theta) with theta = [b; h] from a feasible x0.
    """
    import scipy.sparse as sp
    from purin_b200.workloads import _box_qp, _random_rows

    A_eq = _random_rows(rng, me, n, nnz_per_row)
    A_in = _random_rows(rng, mi, n, nnz_per_row)
    lo = np.full(n, lower)
    up = np.full(n, upper)
    if bounds:
        problem = _box_qp(A_eq, A_in, lo, up, "random")
    else:
        from purin_b200.problems import ParametricQP
        p = me + mi
        problem = ParametricQP(
            P=sp.identity(n), q0=np.zeros(n), A_eq=A_eq, b_eq0=np.zeros(me),
            b_eq_parameter_map=sp.hstack([sp.identity(me), sp.csr_matrix((me, mi))]).tocsr(),
            A_ineq=A_in, b_ineq0=np.zeros(mi),
            b_ineq_parameter_map=sp.hstack([sp.csr_matrix((mi, me)), sp.identity(mi)]).tocsr())
    return problem, (A_eq, A_in)


def random_theta(rng, mats, batch, slack=0.1):
    A_eq, A_in = mats
    n = A_eq.shape[1]
    x0 = rng.uniform(-0.5, 0.5, (batch, n))
    b = (A_eq @ x0.T).T
    h = (A_in @ x0.T).T + rng.uniform(0.0, slack, (batch, A_in.shape[0]))
    return np.concatenate([b, h], axis=1)


class OracleADMMLayer:
    """A problem + ADMMConfig evaluated by the ADMM oracle (values from the product frontend)."""

    def __init__(self, problem, cfg, dtype=np.float64):
        from oracle.admm import OracleADMMConfig, OracleADMMProjection

        self.canonical = canonical_of(problem)
        self.cfg = cfg
        self.dtype = np.dtype(dtype)
        c = self.canonical
        lin = cfg.linear_solver
        ocfg = OracleADMMConfig(
            tolerance=cfg.tolerance, max_iterations=cfg.max_iterations, rho=cfg.rho,
            sigma=cfg.sigma, alpha=cfg.alpha, equality_rho_multiplier=cfg.equality_rho_multiplier,
            cg_max_iterations=cfg.cg_max_iterations, cg_tolerance=cfg.cg_tolerance,
            cg_refinement_steps=cfg.cg_refinement_steps, adaptive_rho=cfg.adaptive_rho,
            rho_update_interval=cfg.rho_update_interval,
            rho_update_threshold=cfg.rho_update_threshold, row_scaling=cfg.row_scaling,
            active_tolerance=cfg.active_tolerance, check_interval=cfg.check_interval,
            linear_tolerance=lin.tolerance, linear_atol=lin.atol, linear_restart=lin.restart,
            linear_max_iterations=lin.max_iterations,
            adjoint_tolerance=cfg.implicit_gradient.adjoint_tolerance)
        zero = np.zeros((1, c.parameter_size))
        values0, _ = c.evaluate(zero)
        ell0 = to_ell(c, np.asarray(values0, np.float64))[0]
        self.proj = OracleADMMProjection(c.equality_sparsity, c.inequality_sparsity,
                                         c.variable_size, ocfg, values_at_zero=ell0)

    def arrays(self, theta, batch):
        theta = np.zeros((batch, 0), self.dtype) if theta is None else np.asarray(theta, self.dtype)
        values, rhs = self.canonical.evaluate(theta)
        values = np.broadcast_to(values, (batch, values.shape[1])).astype(self.dtype)
        rhs = np.broadcast_to(rhs, (batch, rhs.shape[1])).astype(self.dtype)
        return to_ell(self.canonical, values), rhs

    def solve(self, target, theta=None, multipliers_eq=None, multipliers_ineq=None):
        target = np.asarray(target, self.dtype)
        values, rhs = self.arrays(theta, target.shape[0])
        return self.proj.solve(values, rhs, target, multipliers_eq, multipliers_ineq)

    def __call__(self, target, theta=None):
        return self.solve(target, theta)[0]["y"]


def coupled_diagonal_qp_case():
    """tests/test_regression_cp_diagonal_steps.py:28-80 (seed 123): a diagonal QP with 2
    equality and 8 coupled inequality rows on 6 variables in [-1, 1], 3 samples.
    Returns (eq_rows, in_rows, (q, c, values, rhs, lower, upper), dense matrix)."""
    rng = np.random.default_rng(123)
    n, me, mi, batch = 6, 2, 8, 3
    matrix = rng.normal(size=(me + mi, n))
    matrix[abs(matrix) < 0.6] = 0
    q = rng.uniform(0.5, 3.0, (batch, n))
    c = rng.normal(size=(batch, n))
    feasible = rng.uniform(-0.3, 0.3, (batch, n))
    rhs = feasible @ matrix.T
    rhs[:, me:] += rng.uniform(0.3, 1.0, (batch, mi))
    rows = [tuple(int(j) for j in np.flatnonzero(r)) for r in matrix]
    width = max(max(len(r) for r in rows), 1)
    values = np.zeros((batch, me + mi, width))
    for i, r in enumerate(rows):
        values[:, i, :len(r)] = matrix[i, list(r)]
    lower, upper = -np.ones((batch, n)), np.ones((batch, n))
    return tuple(rows[:me]), tuple(rows[me:]), (q, c, values, rhs, lower, upper), matrix


def kkt_certified_qp(q, c, matrix, rhs, me, lower, upper, y, tol=1e-6):
    """The exact solution of min 0.5 y'diag(q)y + c'y s.t. A[:me] y = b[:me],
    A[me:] y <= b[me:], lower <= y <= upper, on the active set that `y` (an approximate
    solution) identifies: the KKT system of that set is solved exactly, and the result is
    returned only if it is primal feasible and its multipliers have the right signs (a
    certificate of optimality, standing in for the reference's OSQP comparison)."""
    n = len(q)
    ineq = [i for i in range(me, len(matrix)) if matrix[i] @ y >= rhs[i] - tol]
    at_up = [j for j in range(n) if y[j] >= upper[j] - tol]
    at_lo = [j for j in range(n) if y[j] <= lower[j] + tol]
    A = np.vstack([matrix[:me], matrix[ineq], np.eye(n)[at_up], np.eye(n)[at_lo]])
    b = np.r_[rhs[:me], rhs[ineq], upper[at_up], lower[at_lo]]
    k = len(A)
    kkt = np.block([[np.diag(q), A.T], [A, np.zeros((k, k))]])
    sol = np.linalg.solve(kkt, np.r_[-c, b])
    x, lam = sol[:n], sol[n:]
    assert np.all(matrix[me:] @ x <= rhs[me:] + 1e-12), "active set not primal feasible"
    assert np.all(x <= upper + 1e-12) and np.all(x >= lower - 1e-12)
    signs = np.r_[np.zeros(me), np.ones(len(ineq) + len(at_up)), -np.ones(len(at_lo))]
    assert np.all(lam[me:] * signs[me:] >= -1e-12), "multiplier signs"
    return x
