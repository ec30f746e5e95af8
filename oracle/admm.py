"""Sparse OSQP-style ADMM projection: forward, post-processing and active-set KKT VJP.

Oracle (test infrastructure).  Restates in NumPy, on canonical arrays (padded
row values ``(B, m, width)`` of ALL public rows, right-hand sides ``(B, m)``):

* ``batched_pcg`` -- ``src/purin/solvers/fischer_burmeister/solver.py:213-310``
  (Jacobi-preconditioned CG with a batch-wide loop and per-row freeze);
* ``prepare_banded`` / ``BandedPlan`` -- ``src/purin/solvers/admm/factor.py:14-144``
  (reverse Cuthill--McKee order, band of width <= 8, banded Cholesky solves);
* ``sparse_admm`` -- ``src/purin/solvers/admm/kernels.py:43-283``;
* ``prepare_pairs`` / ``PairedRows`` -- ``src/purin/solvers/admm/rows.py:10-84``
  (verified two-sided coalescing of opposite inequality rows);
* ``PreparedADMMProjection`` -- ``src/purin/solvers/admm/solver.py:29-255``
  (forward with gap and residuals, the active-set KKT VJP solved by the batched
  restarted GMRES) on the unbounded prepared-projection plumbing of
  ``src/purin/solvers/chambolle_pock/solver.py:277-366`` (row scaling, warm
  start, tolerance, multipliers, status).

ADMM keeps every public row (no singleton-row presolve, ``solver.py:59-64``).
Inner products and infinity norms are NumPy reductions here and parallel sums on
the GPU, so the two agree to rounding, not bit for bit.
"""

from __future__ import annotations

from collections import deque
from dataclasses import dataclass

import numpy as np

from oracle.cp import clip, operators
from oracle.gmres import batched_restarted_gmres
from oracle.sparse import layout, matvec

CONVERGED, MAX_ITERATIONS, LINEAR_SOLVE_FAILURE, NONFINITE = 0, 1, 2, 3


@dataclass
class OracleADMMConfig:
    """Field-for-field ``ADMMConfig`` (``src/purin/solvers/admm/config.py:10-40``)."""

    tolerance: float = 1e-9
    max_iterations: int = 10000
    rho: float = 1.0
    sigma: float = 1e-6
    alpha: float = 1.6
    equality_rho_multiplier: float = 1.0
    cg_max_iterations: int = 32
    cg_tolerance: float = 1e-10
    cg_refinement_steps: int = 1
    adaptive_rho: bool = False
    rho_update_interval: int = 50
    rho_update_threshold: float = 5.0
    row_scaling: bool = True
    active_tolerance: float = 1e-8
    check_interval: int = 25
    linear_tolerance: float = 1e-9
    linear_atol: float = 0.0
    linear_restart: int = 30
    linear_max_iterations: int = 100
    adjoint_tolerance: float = 1e-8


def inf_norm(x):
    """``kernels.py:37-39``: max |x| along each row, 0 for an empty row."""
    if x.shape[1] == 0:
        return np.zeros(x.shape[0], x.dtype)
    return np.max(np.abs(x), axis=1)


def _row_inner(a, b):
    return np.sum(a * b, axis=1)


def batched_pcg(operator, rhs, *, preconditioner, tolerance, absolute_tolerance,
                max_iterations):
    """``fischer_burmeister/solver.py:213-310``: returns (solution, iterations per row).

    Starts from zero; rows freeze when their residual's inf-norm falls to the
    threshold or an update is non-finite (or of nonpositive curvature).
    """
    dtype = rhs.dtype
    batch = rhs.shape[0]
    eps = dtype.type(np.finfo(dtype).eps)
    one = dtype.type(1)
    tol = np.full(batch, tolerance, dtype)
    threshold = np.maximum(dtype.type(absolute_tolerance), tol * inf_norm(rhs))
    x = np.zeros_like(rhs)
    residual = rhs - operator(x)
    with np.errstate(all="ignore"):
        z = preconditioner(residual)
        rz = _row_inner(residual, z)
    finite0 = (np.all(np.isfinite(residual), axis=1) & np.all(np.isfinite(z), axis=1)
               & np.isfinite(rz))
    active = finite0 & (inf_norm(residual) > threshold)
    direction = z.copy()
    iterations = np.zeros(batch, np.int32)
    it = 0
    with np.errstate(all="ignore"):
        while it < int(max_iterations) and np.any(active):
            image = operator(direction)
            curvature = _row_inner(direction, image)
            positive = curvature > eps
            alpha = rz / np.where(positive, curvature, one)
            cand_x = x + alpha[:, None] * direction
            cand_r = residual - alpha[:, None] * image
            r_inf = inf_norm(cand_r)
            cand_z = preconditioner(cand_r)
            next_rz = _row_inner(cand_r, cand_z)
            beta = next_rz / np.where(np.abs(rz) > eps, rz, one)
            cand_d = cand_z + beta[:, None] * direction
            finite = (np.all(np.isfinite(cand_x), axis=1) & np.all(np.isfinite(cand_r), axis=1)
                      & np.all(np.isfinite(cand_z), axis=1) & np.isfinite(next_rz) & positive)
            next_active = active & finite & (r_inf > threshold)
            a = active[:, None]
            x = np.where(a, cand_x, x)
            residual = np.where(a, cand_r, residual)
            z = np.where(a, cand_z, z)
            direction = np.where(a, cand_d, direction)
            rz = np.where(active, next_rz, rz)
            iterations = iterations + active.astype(np.int32)
            active = next_active
            it += 1
    return x, iterations


class BandedPlan:
    """``factor.py:14-105``: band of the ADMM matrix in RCM order and its Cholesky solves."""

    def __init__(self, permutation, inverse, rows, left, right, destination, n, width):
        self.permutation = permutation
        self.inverse = inverse
        self.rows, self.left, self.right, self.destination = rows, left, right, destination
        self.n, self.width = n, width

    def factor(self, diagonal, values, penalty, sigma):
        """``factor.py:28-64``: lower band of diag(q) + sigma I + K^T diag(rho) K, factored."""
        n, w = self.n, self.width
        batch = values.shape[0]
        dtype = values.dtype
        band = np.zeros((batch, n * (w + 1)), dtype)
        vals = np.broadcast_to(values, (batch,) + values.shape[1:])
        products = (penalty[:, self.rows] * vals[:, self.rows, self.left]
                    * vals[:, self.rows, self.right])
        for k in range(len(self.destination)):  # scatter-add in index order
            band[:, self.destination[k]] += products[:, k]
        band = band.reshape(batch, n, w + 1)
        band[:, :, 0] += diagonal[:, self.permutation] + dtype.type(sigma)
        offsets = np.arange(1, w + 1)
        with np.errstate(all="ignore"):
            for j in range(n):
                previous = j - offsets
                lj = np.where(previous[None, :] >= 0, band[:, j, 1:], dtype.type(0))
                pivot = np.sqrt(band[:, j, 0] - np.sum(lj * lj, axis=1))
                band[:, j, 0] = pivot
                for d in range(1, w + 1):
                    i = min(j + d, n - 1)
                    ds = offsets + d
                    overlap = (previous >= 0) & (ds <= w)
                    li = band[:, i, np.minimum(ds, w)]
                    entry = (band[:, i, d] - np.sum(np.where(overlap[None, :], li * lj,
                                                             dtype.type(0)), axis=1)) / pivot
                    if j + d < n:
                        band[:, i, d] = entry
        return band

    def solve(self, factor, rhs):
        """``factor.py:66-105``: forward and backward band substitutions."""
        n, w = self.n, self.width
        dtype = rhs.dtype
        offsets = np.arange(1, w + 1)
        b = rhs[:, self.permutation]
        y = np.zeros_like(b)
        with np.errstate(all="ignore"):
            for i in range(n):
                indices = np.maximum(i - offsets, 0)
                dot = np.sum(np.where((i >= offsets)[None, :], factor[:, i, 1:] * y[:, indices],
                                      dtype.type(0)), axis=1)
                y[:, i] = (b[:, i] - dot) / factor[:, i, 0]
            x = np.zeros_like(b)
            for k in range(n):
                i = n - 1 - k
                indices = np.minimum(i + offsets, n - 1)
                dot = np.sum(np.where((i + offsets < n)[None, :],
                                      factor[:, indices, offsets] * x[:, indices],
                                      dtype.type(0)), axis=1)
                x[:, i] = (y[:, i] - dot) / factor[:, i, 0]
        return x[:, self.inverse]


def prepare_banded(support, mask, n):
    """``factor.py:108-144``: RCM order of the row graph; None when the band exceeds 8."""
    support, mask = np.asarray(support), np.asarray(mask)
    graph = [set() for _ in range(n)]
    for indices, valid in zip(support, mask):
        row = indices[valid].tolist()
        for i in row:
            graph[i].update(j for j in row if j != i)
    visited, order = set(), []
    while len(order) < n:
        root = min((i for i in range(n) if i not in visited), key=lambda i: (len(graph[i]), i))
        queue = deque([root])
        visited.add(root)
        while queue:
            i = queue.popleft()
            order.append(i)
            for j in sorted(graph[i] - visited, key=lambda j: (len(graph[j]), j)):
                if j not in visited:
                    visited.add(j)
                    queue.append(j)
    permutation = np.array(order[::-1], np.int64)
    inverse = np.argsort(permutation).astype(np.int64)
    width = max((abs(int(inverse[i]) - int(inverse[j])) for i in range(n) for j in graph[i]),
                default=0)
    if width > 8:
        return None
    rows, left, right, dest = [], [], [], []
    for r, (indices, valid) in enumerate(zip(support, mask)):
        for a in np.flatnonzero(valid):
            for b in np.flatnonzero(valid):
                i, j = int(inverse[indices[a]]), int(inverse[indices[b]])
                if i >= j:
                    rows.append(r)
                    left.append(a)
                    right.append(b)
                    dest.append(i * (width + 1) + i - j)
    as_int = lambda v: np.asarray(v, np.int64)
    return BandedPlan(permutation, inverse, as_int(rows), as_int(left), as_int(right),
                      as_int(dest), n, width)


@dataclass
class ADMMOutput:
    """``kernels.py:13-26``."""

    x: np.ndarray
    z: np.ndarray
    dual: np.ndarray
    rho: np.ndarray
    iterations: np.ndarray
    inner_iterations: np.ndarray
    primal_residual: np.ndarray
    dual_residual: np.ndarray
    linear_residual: np.ndarray
    converged: np.ndarray
    finite: np.ndarray


def sparse_admm(diagonal, c, values, lower, upper, support, mask, *, rho=1.0, sigma=1e-6,
                alpha=1.6, tolerance=1e-9, max_iterations=10000, cg_iterations=32,
                cg_tolerance=1e-10, refinement_steps=1, adaptive_rho=False,
                rho_update_interval=50, rho_update_threshold=5.0, x0=None, dual0=None,
                factor_plan=None, check_interval=1):
    """``kernels.py:43-283``: batched diagonal QPs by ADMM with per-sample freeze."""
    batch, n = diagonal.shape
    dtype = diagonal.dtype
    T = dtype.type
    mv, tmv = operators(values, support, mask, n)
    _, squared_transpose = operators(values ** 2, support, mask, n)
    penalty = np.array(np.broadcast_to(np.asarray(rho, dtype), lower.shape))
    tolerance = np.broadcast_to(np.asarray(tolerance, dtype), (batch,))
    x = np.zeros_like(diagonal) if x0 is None else np.array(x0, dtype)
    dual = np.zeros_like(lower) if dual0 is None else np.array(dual0, dtype)
    z = np.zeros_like(lower) if x0 is None else clip(mv(x), lower, upper)

    def preconditioner(p):
        return diagonal + T(sigma) + squared_transpose(p)

    diag = preconditioner(penalty)
    factor = factor_plan.factor(diagonal, values, penalty, sigma) if factor_plan else None
    done = np.zeros(batch, bool)
    failed = np.zeros(batch, bool)
    counts = np.zeros(batch, np.int32)
    inner_counts = np.zeros(batch, np.int32)
    last_linear = np.full(batch, np.inf, dtype)
    tiny = T(np.finfo(dtype).tiny)
    iteration = 0
    with np.errstate(all="ignore"):
        while iteration < max_iterations and np.any(~(done | failed)):
            active = ~(done | failed)
            op = lambda v: (diagonal + T(sigma)) * v + tmv(penalty * mv(v))
            rhs = T(sigma) * x - c + tmv(penalty * z - dual)
            lin_count = np.zeros(batch, np.int32)
            if factor_plan is not None:
                xt = factor_plan.solve(factor, rhs)
            else:
                xt = x
                for _ in range(refinement_steps):
                    correction = rhs - op(xt)
                    magnitude = np.maximum(inf_norm(correction), tiny)
                    normalized = np.where(active[:, None], correction / magnitude[:, None], T(0))
                    solution, its = batched_pcg(op, normalized, preconditioner=lambda v: v / diag,
                                                tolerance=cg_tolerance,
                                                absolute_tolerance=cg_tolerance,
                                                max_iterations=cg_iterations)
                    xt = xt + magnitude[:, None] * solution
                    lin_count = lin_count + its
            ax = mv(xt)
            nx = T(alpha) * xt + (T(1) - T(alpha)) * x
            relaxed = T(alpha) * ax + (T(1) - T(alpha)) * z
            nz = clip(relaxed + dual / penalty, lower, upper)
            nd = dual + penalty * (relaxed - nz)
            checking = ((iteration + 1) % check_interval == 0) or (iteration + 1 == max_iterations)
            if adaptive_rho:
                checking = checking or ((iteration + 1) % rho_update_interval == 0)
            if checking:
                linear = inf_norm(rhs - ((diagonal + T(sigma)) * xt + tmv(penalty * ax)))
                primal = inf_norm(mv(nx) - nz)
                dual_res = inf_norm(diagonal * nx + c + tmv(nd))
                finite = (np.all(np.isfinite(nx), axis=1) & np.all(np.isfinite(nd), axis=1)
                          & np.isfinite(linear) & np.isfinite(primal) & np.isfinite(dual_res))
            else:
                linear = last_linear
                primal = np.full(batch, np.inf, dtype)
                dual_res = np.full(batch, np.inf, dtype)
                finite = np.ones(batch, bool)
            accepted = (checking & finite & (primal <= tolerance) & (dual_res <= tolerance)
                        & (linear <= tolerance))
            a = active[:, None]
            x = np.where(a, nx, x)
            z = np.where(a, nz, z)
            dual = np.where(a, nd, dual)
            counts = counts + active.astype(np.int32)
            inner_counts = inner_counts + np.where(active, lin_count, 0).astype(np.int32)
            if checking:
                last_linear = np.where(active, linear, last_linear)
            done = done | (active & accepted)
            failed = failed | (active & checking & ~finite)
            if adaptive_rho:
                pscale = np.maximum(np.maximum(inf_norm(mv(x)), inf_norm(z)), T(1e-12))
                dscale = np.maximum(np.maximum(inf_norm(diagonal * x), inf_norm(tmv(dual))),
                                    np.maximum(inf_norm(c), T(1e-12)))
                rho_factor = np.sqrt((primal / pscale + T(1e-16)) / (dual_res / dscale + T(1e-16)))
                change = (((iteration + 1) % rho_update_interval == 0) & active & ~done & finite
                          & ((rho_factor >= T(rho_update_threshold))
                             | (rho_factor <= T(1) / T(rho_update_threshold))))
                candidate = clip(penalty * rho_factor[:, None], T(1e-6), T(1e6))
                penalty = np.where(change[:, None], candidate, penalty)
                if np.any(change):
                    diag = preconditioner(penalty)
                    if factor_plan is not None:
                        factor = factor_plan.factor(diagonal, values, penalty, sigma)
            iteration += 1
        primal = inf_norm(mv(x) - z)
        dual_res = inf_norm(diagonal * x + c + tmv(dual))
        finite = (np.all(np.isfinite(x), axis=1) & np.all(np.isfinite(dual), axis=1)
                  & np.isfinite(primal) & np.isfinite(dual_res) & np.isfinite(last_linear))
    converged = (finite & (primal <= tolerance) & (dual_res <= tolerance)
                 & (last_linear <= tolerance))
    return ADMMOutput(x, z, dual, penalty, counts, inner_counts, primal, dual_res, last_linear,
                      converged, finite)


class PairedRows:
    """``rows.py:10-48``: verified two-sided coalescing of opposite inequality rows."""

    def __init__(self, keep, first, second, positions, support, mask, factor_plan):
        self.keep, self.first, self.second, self.positions = keep, first, second, positions
        self.support, self.mask, self.factor_plan = support, mask, factor_plan

    def verified(self, values, rhs):
        """``rows.py:22-31``: exact opposite coefficients and a nonempty interval, per call."""
        return bool(np.all(values[:, self.first] == -values[:, self.second])
                    and np.all(-rhs[:, self.second] < rhs[:, self.first]))

    def compact(self, rhs, initial, equality_size):
        """``rows.py:33-43``."""
        upper = rhs[:, self.keep]
        lower = np.full_like(upper, -np.inf)
        lower[:, :equality_size] = upper[:, :equality_size]
        lower[:, self.positions] = -rhs[:, self.second]
        dual = initial[:, self.keep].copy()
        dual[:, self.positions] += -initial[:, self.second]
        return lower, upper, dual

    def restore(self, compact_dual, original_rhs):
        """``rows.py:45-51``."""
        dual = np.zeros_like(original_rhs)
        dual[:, self.keep] = compact_dual
        signed = compact_dual[:, self.positions]
        dual[:, self.first] = np.maximum(signed, 0)
        dual[:, self.second] = np.maximum(-signed, 0)
        return dual


def prepare_pairs(values0, support, mask, equality_size, n, row_scaling):
    """``rows.py:54-84``: nominate pairs from the values at theta = 0 (row-scaled)."""
    values = np.array(values0, np.float64)
    if row_scaling:
        norm = np.sqrt(np.sum(values ** 2, axis=1))
        values = values * np.where(norm > 0, 1 / np.maximum(norm, 1e-30), 1.0)[:, None]
    waiting, pairs = {}, []
    for row in range(equality_size, len(values)):
        v = values[row]
        if not np.all(np.isfinite(v)) or not np.any(v):
            continue
        columns = tuple(support[row].tolist())
        key = (columns, tuple(v.tolist()))
        opposite = (columns, tuple((-v).tolist()))
        if waiting.get(opposite):
            pairs.append((waiting[opposite].pop(), row))
        else:
            waiting.setdefault(key, []).append(row)
    if not pairs:
        return None
    removed = {j for _, j in pairs}
    keep = [i for i in range(len(values)) if i not in removed]
    index = {r: i for i, r in enumerate(keep)}
    first, second = zip(*pairs)
    positions = [index[i] for i in first]
    as_int = lambda v: np.asarray(v, np.int64)
    return PairedRows(as_int(keep), as_int(first), as_int(second), as_int(positions),
                      support[keep], mask[keep], prepare_banded(support[keep], mask[keep], n))


class OracleADMMProjection:
    """``PreparedADMMProjection`` (``admm/solver.py:29-255``) on canonical arrays."""

    def __init__(self, equality_sparsity, inequality_sparsity, n, config: OracleADMMConfig,
                 values_at_zero=None):
        self.n = n
        self.me = len(equality_sparsity)
        self.mi = len(inequality_sparsity)
        self.cfg = config
        rows = tuple(equality_sparsity) + tuple(inequality_sparsity)
        self.support, self.mask, self.positions = layout(rows, n)
        self.factor_plan = prepare_banded(self.support, self.mask, n)
        self.pairs = (None if values_at_zero is None else
                      prepare_pairs(values_at_zero, self.support, self.mask, self.me, n,
                                    config.row_scaling))

    def _run(self, values, lower, upper, target, initial, tolerance, support, mask, plan):
        """``solver.py:60-97``."""
        cfg = self.cfg
        dtype = target.dtype
        penalty = np.full_like(upper, cfg.rho)
        penalty[:, :self.me] *= dtype.type(cfg.equality_rho_multiplier)
        return sparse_admm(
            np.ones_like(target), -target, values, lower, upper, support, mask, rho=penalty,
            sigma=cfg.sigma, alpha=cfg.alpha, tolerance=tolerance,
            max_iterations=cfg.max_iterations, cg_iterations=cfg.cg_max_iterations,
            cg_tolerance=cfg.cg_tolerance, refinement_steps=cfg.cg_refinement_steps,
            adaptive_rho=cfg.adaptive_rho, rho_update_interval=cfg.rho_update_interval,
            rho_update_threshold=cfg.rho_update_threshold, x0=target, dual0=initial,
            factor_plan=plan, check_interval=cfg.check_interval)

    def forward(self, values, rhs, target, initial, tolerance):
        """``solver.py:99-160``: the custom-VJP forward on scaled arrays."""
        me, n = self.me, self.n
        dtype = target.dtype
        lower = np.concatenate((rhs[:, :me], np.full_like(rhs[:, me:], -np.inf)), axis=1)
        paired = self.pairs
        if paired is not None and paired.verified(values, rhs):
            lo, hi, init = paired.compact(rhs, initial, me)
            out = self._run(values[:, paired.keep], lo, hi, target, init, tolerance,
                            paired.support, paired.mask, paired.factor_plan)
            dual = paired.restore(out.dual, rhs)
        else:
            out = self._run(values, lower, rhs, target, initial, tolerance, self.support,
                            self.mask, self.factor_plan)
            dual = out.dual
        x = out.x
        mv, tmv = operators(values, self.support, self.mask, n)
        with np.errstate(all="ignore"):
            primal = np.sum(dtype.type(0.5) * x ** 2 - target * x, axis=1)
            t = -target + tmv(dual)
            dual_objective = (-dtype.type(0.5) * np.sum(t * t, axis=1)
                              - np.sum(rhs * dual, axis=1))
            gap = (np.maximum(primal - dual_objective, 0)
                   / np.maximum(1.0, np.maximum(abs(primal), abs(dual_objective))))
        residual = np.maximum(out.primal_residual,
                              np.maximum(out.dual_residual, out.linear_residual))
        return dict(y=x, dual=dual, iterations=out.iterations, residual=residual,
                    gap=gap.astype(dtype), converged=out.converged, admm=out)

    def solve(self, values, rhs, target, multipliers_eq=None, multipliers_ineq=None):
        """``chambolle_pock/solver.py:277-366`` with the ADMM forward."""
        cfg = self.cfg
        dtype = target.dtype
        batch = target.shape[0]
        me, mi, n = self.me, self.mi, self.n
        values = np.asarray(values, dtype)
        rhs = np.asarray(rhs, dtype)
        scale = np.ones_like(rhs)
        if cfg.row_scaling and rhs.shape[1]:
            norms = np.sqrt(np.sum(values ** 2, axis=2))
            scale = np.where(norms > 0, 1 / np.maximum(norms, 1e-30), 1.0).astype(dtype)
        data = values * scale[:, :, None]
        scaled_rhs = rhs * scale
        eq = np.zeros((batch, me), dtype) if multipliers_eq is None else np.asarray(multipliers_eq, dtype)
        iq = np.zeros((batch, mi), dtype) if multipliers_ineq is None else np.asarray(multipliers_ineq, dtype)
        initial = np.concatenate((eq, iq), axis=1) / scale
        min_scale = np.minimum(np.min(scale, axis=1, initial=1.0), 1.0)
        tolerance = (dtype.type(cfg.tolerance) * min_scale).astype(dtype)
        out = self.forward(data, scaled_rhs, target, initial, tolerance)
        dual = out["dual"] * scale
        mv, tmv = operators(values, self.support, self.mask, n)
        with np.errstate(all="ignore"):
            r = mv(out["y"]) - rhs
            eq_res = np.max(np.abs(r[:, :me]), axis=1, initial=0.0)
            ineq_res = np.max(np.maximum(r[:, me:], 0), axis=1, initial=0.0)
            stationarity = np.max(np.abs(out["y"] - target + tmv(dual)), axis=1)
        residual = np.maximum(np.maximum(eq_res, ineq_res), stationarity).astype(dtype)
        finite = (np.all(np.isfinite(out["y"]), axis=1) & np.all(np.isfinite(dual), axis=1)
                  & np.isfinite(residual) & np.isfinite(out["gap"]))
        converged = finite & out["converged"] & (residual <= cfg.tolerance)
        status = np.where(converged, CONVERGED,
                          np.where(finite, MAX_ITERATIONS, NONFINITE)).astype(np.int32)
        result = dict(y=out["y"], multipliers_eq=dual[:, :me], multipliers_ineq=dual[:, me:],
                      slacks=np.maximum(-r[:, me:], 0), status=status,
                      iterations=out["iterations"], residual_inf_norm=residual, finite=finite,
                      gradient_eligible=converged)
        saved = dict(out=out, values=data, rhs=scaled_rhs, target=target, scale=scale)
        return result, saved

    def vjp(self, saved, cot_y, stats=None):
        """``solver.py:175-255``: GMRES on the active-set KKT operator, then the pullback.

        Returns the cotangents of the scaled values (padded ``(B, m, width)``),
        the scaled right-hand sides and the target.
        """
        cfg = self.cfg
        out = saved["out"]
        values, rhs = saved["values"], saved["rhs"]
        n, me = self.n, self.me
        dtype = values.dtype
        mv, tmv = operators(values, self.support, self.mask, n)
        y, dual = out["y"], out["dual"]
        with np.errstate(all="ignore"):
            slack = rhs - mv(y)
        active = np.concatenate(
            (np.ones_like(rhs[:, :me], dtype=bool),
             (dual[:, me:] > cfg.active_tolerance)
             & (slack[:, me:] <= max(cfg.active_tolerance, cfg.tolerance))), axis=1)
        active = active.astype(dtype)

        def operator(v):
            primal = v[:, :n]
            w = v[:, n:]
            return np.concatenate((primal + tmv(active * w),
                                   active * mv(primal) + (1 - active) * w), axis=1)

        g = np.concatenate((np.where(out["converged"][:, None], cot_y, 0).astype(dtype),
                            np.zeros_like(rhs)), axis=1)
        with np.errstate(all="ignore"):
            adjoint, code, residual = batched_restarted_gmres(
                operator, g, tolerance=cfg.linear_tolerance,
                absolute_tolerance=cfg.linear_atol, restart=cfg.linear_restart,
                max_iterations=cfg.linear_max_iterations, stats=stats)
        valid = (out["converged"] & np.all(np.isfinite(adjoint), axis=1) & np.isfinite(residual)
                 & ((code == 0) | (residual <= cfg.adjoint_tolerance)))
        adjoint = np.where(valid[:, None], adjoint, 0)
        primal = adjoint[:, :n]
        dual_c = active * adjoint[:, n:]
        gradient_values = -(dual[:, :, None] * primal[:, self.support]
                            + dual_c[:, :, None] * y[:, self.support])
        gradient_values = np.where(self.mask[None], gradient_values, 0)
        clean = lambda v: np.nan_to_num(v, nan=0.0, posinf=0.0, neginf=0.0)
        if stats is not None:
            stats.update(code=code, residual=residual, valid=valid, active=active)
        return dict(values=clean(gradient_values), rhs=clean(dual_c), target=clean(primal))
