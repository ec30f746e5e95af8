"""Prepared CP projection: bound presolve, scaled solve, post-processing, implicit VJP.

Oracle (test infrastructure).  Restates, on canonical arrays (padded row
values ``(B, m_all, width)`` and right-hand sides ``(B, m_all)``):

* ``prepare_bounds`` -- ``src/purin/solvers/chambolle_pock/bounds.py:320-326``
  (singleton inequality rows become per-sample box bounds);
* ``BoundProjection.solve`` -- ``bounds.py:170-317`` (presolve 193-209, row
  scaling 210-214, warm start and tolerance 215-236, CP solve 237-246,
  multiplier recovery and original-unit diagnostics 247-317);
* the custom-VJP forward/backward -- ``bounds.py:42-66`` and ``80-165``;
* the unbounded variant ``PreparedChambollePockProjection._solve`` /
  ``_make_differentiable_solve`` -- ``solver.py:140-366`` -- which is the same
  computation with no bound rows (bounds of +-inf, all samples feasible).

``vjp`` returns the cotangents at the custom-VJP boundary: scaled kept-row
values, scaled kept-row right-hand sides, target, lower and upper.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from oracle.cp import (
    clip,
    cp_step_pullback,
    diagonal_step_sizes,
    norm_estimate,
    operators,
    sparse_cp,
)
from oracle.gmres import LockstepGmres, batched_restarted_gmres
from oracle.sparse import layout

CONVERGED, MAX_ITERATIONS, LINEAR_SOLVE_FAILURE, NONFINITE = 0, 1, 2, 3


@dataclass
class OracleConfig:
    """Field-for-field ``ChambollePockConfig`` (``chambolle_pock/config.py:34-48``)
    plus the ``LinearSolverConfig``/``ImplicitGradientConfig`` fields the CP
    VJP reads (``solvers/config.py:10-44``)."""

    tolerance: float = 1e-9
    max_iterations: int = 10000
    accelerated: bool = False
    safety: float = 0.95
    norm_iterations: int = 20
    norm_seed: int = 42
    row_scaling: bool = True
    norm_bound: bool = True
    diagonal_preconditioning: bool = False
    linear_tolerance: float = 1e-9
    linear_atol: float = 0.0
    linear_restart: int = 30
    linear_max_iterations: int = 100
    adjoint_tolerance: float = 1e-8


def _seq_sum_last(x):
    out = np.zeros(x.shape[:-1], dtype=x.dtype)
    for k in range(x.shape[-1]):
        out = out + x[..., k]
    return out


class OracleProjection:
    """CPU restatement of ``PreparedChambollePockProjection`` + ``BoundProjection``."""

    def __init__(self, eq_rows, iq_rows, n, config=None, partitionable=True):
        self.config = config or OracleConfig()
        self.n = int(n)
        self.me = len(eq_rows)
        self.mi = len(iq_rows)
        self.rows_all = [tuple(r) for r in eq_rows] + [tuple(r) for r in iq_rows]
        self.support_all, self.mask_all, _ = layout(self.rows_all, self.n)
        self.bound_rows = [self.me + i for i, r in enumerate(iq_rows) if len(r) == 1]
        bound_set = set(self.bound_rows)
        self.rows = [r for r in range(self.me + self.mi) if r not in bound_set]
        self.variables = self.support_all[self.bound_rows, 0] if self.bound_rows else (
            np.zeros(0, np.int32))
        self.support = self.support_all[self.rows]
        self.mask = self.mask_all[self.rows]
        self.partitionable = partitionable
        # The CP loop (oracle.cp.sparse_cp; oracle.cpu.sparse_cp_native runs the
        # same loop in C++ on the host cores).
        self.cp_solver = sparse_cp

    # -- forward -------------------------------------------------------------
    def presolve(self, values, rhs, target):
        """``bounds.py:193-214``: box bounds, feasibility, kept rows and their scale."""
        dtype = target.dtype
        batch = target.shape[0]
        inf = dtype.type(np.inf)
        one = dtype.type(1.0)
        lower = np.full_like(target, -inf)
        upper = np.full_like(target, inf)
        feasible = np.ones(batch, bool)
        coefficient = np.zeros((batch, 0), dtype)
        threshold = np.zeros((batch, 0), dtype)
        if self.bound_rows:
            b = np.asarray(self.bound_rows)
            coefficient = values[:, b, 0]
            threshold = rhs[:, b] / np.where(coefficient != 0, coefficient, one)
            lo_upd = np.where(coefficient < 0, threshold, -inf)
            up_upd = np.where(coefficient > 0, threshold, inf)
            for k, v in enumerate(self.variables):
                lower[:, v] = np.maximum(lower[:, v], lo_upd[:, k])
                upper[:, v] = np.minimum(upper[:, v], up_upd[:, k])
            feasible = np.all(lower <= upper, axis=1) & np.all(
                (coefficient != 0) | (rhs[:, b] >= 0), axis=1)
        kept = values[:, self.rows]
        scale = np.ones_like(rhs[:, self.rows])
        if self.config.row_scaling:
            norms = np.sqrt(_seq_sum_last(kept * kept))
            scale = np.where(norms > 0, one / np.maximum(norms, dtype.type(1e-30)), one)
        return lower, upper, feasible, coefficient, threshold, kept, scale

    def solve(self, values, rhs, target, multipliers_eq=None, multipliers_ineq=None, *,
              offset=0, total=None):
        cfg = self.config
        target = np.asarray(target)
        dtype = target.dtype
        batch = target.shape[0]
        lower, upper, feasible, coefficient, threshold, kept, scale = self.presolve(
            values, rhs, target)
        eq = (np.zeros((batch, self.me), dtype) if multipliers_eq is None
              else np.asarray(multipliers_eq, dtype))
        iq = (np.zeros((batch, self.mi), dtype) if multipliers_ineq is None
              else np.asarray(multipliers_ineq, dtype))
        initial = np.concatenate((eq, iq), axis=1)[:, self.rows] / scale
        min_scale = np.min(scale, axis=1, initial=1.0).astype(dtype)
        tolerance = dtype.type(cfg.tolerance) * np.minimum(dtype.type(1.0), min_scale)
        data = kept * scale[:, :, None]
        scaled_rhs = rhs[:, self.rows] * scale
        out = self.cp_solver(
            np.ones_like(target), -target, data, scaled_rhs, self.support, self.mask,
            self.me, lower, upper, accelerated=cfg.accelerated, safety=cfg.safety,
            max_iterations=cfg.max_iterations, tolerance=tolerance,
            norm_iterations=cfg.norm_iterations, norm_seed=cfg.norm_seed, y0=target,
            dual0=initial, freeze_converged=True, check_stationarity=True,
            norm_bound=cfg.norm_bound, diagonal_preconditioning=cfg.diagonal_preconditioning,
            offset=offset, total=total, partitionable=self.partitionable,
        )
        out = out._replace(converged=out.converged & feasible)
        result = self.postprocess(values, rhs, target, out, scale, lower, upper,
                                  coefficient, threshold)
        saved = dict(out=out, values=data, rhs=scaled_rhs, target=target, lower=lower,
                     upper=upper, scale=scale, tolerance=tolerance, initial=initial,
                     feasible=feasible, offset=offset, total=total)
        return result, saved

    def postprocess(self, values, rhs, target, out, scale, lower, upper, coefficient,
                    threshold):
        """``bounds.py:247-317`` (``solver.py:333-366`` without bound rows)."""
        cfg = self.config
        dtype = target.dtype
        zero = dtype.type(0.0)
        one = dtype.type(1.0)
        batch = target.shape[0]
        dual = np.zeros_like(rhs)
        dual[:, self.rows] = out.dual * scale
        mv, tmv = operators(values, self.support_all, self.mask_all, self.n)
        if self.bound_rows:
            b = np.asarray(self.bound_rows)
            base_stationarity = out.y - target + tmv(dual)
            v = self.variables
            is_lower = (coefficient < 0) & (threshold == lower[:, v]) & (out.y[:, v] == lower[:, v])
            is_upper = (coefficient > 0) & (threshold == upper[:, v]) & (out.y[:, v] == upper[:, v])
            lower_count = np.zeros_like(target)
            upper_count = np.zeros_like(target)
            for k, var in enumerate(v):
                lower_count[:, var] += is_lower[:, k].astype(dtype)
                upper_count[:, var] += is_upper[:, k].astype(dtype)
            normal = base_stationarity[:, v]
            bound_dual = np.where(is_lower, np.maximum(normal, zero)
                                  / np.maximum(lower_count[:, v], one), zero)
            bound_dual = bound_dual + np.where(is_upper, np.maximum(-normal, zero)
                                               / np.maximum(upper_count[:, v], one), zero)
            bound_dual = bound_dual / np.where(coefficient != 0, np.abs(coefficient), one)
            dual[:, b] = bound_dual
        r = mv(out.y) - rhs
        me = self.me
        eq_res = np.max(np.abs(r[:, :me]), axis=1, initial=0.0).astype(dtype)
        iq_res = np.max(np.maximum(r[:, me:], zero), axis=1, initial=0.0).astype(dtype)
        stationarity = np.max(np.abs(out.y - target + tmv(dual)), axis=1)
        residual = np.maximum(np.maximum(eq_res, iq_res), stationarity)
        finite = (np.all(np.isfinite(out.y), axis=1) & np.all(np.isfinite(dual), axis=1)
                  & np.isfinite(residual) & np.isfinite(out.gap))
        converged = finite & out.converged & (residual <= dtype.type(cfg.tolerance))
        status = np.where(converged, CONVERGED,
                          np.where(finite, MAX_ITERATIONS, NONFINITE)).astype(np.int32)
        return dict(
            y=out.y,
            multipliers_eq=dual[:, :me],
            multipliers_ineq=dual[:, me:],
            slacks=np.maximum(-r[:, me:], zero),
            status=status,
            iterations=out.iterations,
            residual_inf_norm=residual,
            finite=finite,
            gradient_eligible=converged,
            gap=out.gap,
            cp_residual=out.residual,
            cp_converged=out.converged,
        )

    # -- backward ------------------------------------------------------------
    def vjp_step_sizes(self, data, target, offset=0, total=None):
        """``bounds.py:83-101``: tau = s/(1+L), sigma = s/L from the power iteration."""
        cfg = self.config
        dtype = target.dtype
        batch = target.shape[0]
        if cfg.diagonal_preconditioning and not cfg.accelerated:
            return diagonal_step_sizes(np.ones_like(target), data, self.support, self.mask,
                                       cfg.safety)
        mv, tmv = operators(data, self.support, self.mask, self.n)
        norm = norm_estimate(mv, tmv, batch, self.n, dtype, cfg.norm_iterations,
                             cfg.norm_seed, offset=offset, total=total,
                             partitionable=self.partitionable)
        L = np.maximum(norm, dtype.type(1e-12))
        s = dtype.type(cfg.safety)
        return s / (dtype.type(1) + L), s / L

    def pullback(self, saved, tau, sigma, v):
        """Cotangents of one CP step at the saved fixed point (``bounds.py:109-129``)."""
        out = saved["out"]
        n, m = self.n, len(self.rows)
        v_y, v_d, v_b = v[:, :n], v[:, n:n + m], v[:, n + m:]
        return cp_step_pullback((out.y, out.dual, out.y), saved["values"], saved["rhs"],
                                saved["target"], saved["lower"], saved["upper"],
                                self.support, self.mask, self.me, tau, sigma, (v_y, v_d, v_b))

    def _vjp_system(self, saved, cot_y):
        """Step sizes, the operator I - J^T and the right-hand side g (``bounds.py:83-138``)."""
        out = saved["out"]
        target = saved["target"]
        dtype = target.dtype
        tau, sigma = self.vjp_step_sizes(saved["values"], target, saved["offset"],
                                         saved["total"])
        zero = dtype.type(0)

        def operator(z):
            (sy, sd, sb), *_ = self.pullback(saved, tau, sigma, z)
            return z - np.concatenate((sy, sd, sb), axis=1)

        g = np.concatenate((np.where(out.converged[:, None], cot_y, zero),
                            np.zeros_like(out.dual), np.zeros_like(out.y)), axis=1)
        return tau, sigma, operator, g

    def _vjp_gradients(self, saved, tau, sigma, adjoint, code, residual):
        """Validity masking and the parameter pullback (``bounds.py:148-165``)."""
        cfg = self.config
        out = saved["out"]
        dtype = saved["target"].dtype
        zero = dtype.type(0)
        valid = (out.converged & np.all(np.isfinite(adjoint), axis=1) & np.isfinite(residual)
                 & ((code == 0) | (residual <= dtype.type(cfg.adjoint_tolerance))))
        adjoint = np.where(valid[:, None], adjoint, zero)
        _, gv, gb, gt, gl, gu = self.pullback(saved, tau, sigma, adjoint)
        clean = lambda a: np.nan_to_num(a, nan=0.0, posinf=0.0, neginf=0.0)
        grads = dict(values=clean(gv), rhs=clean(gb), target=clean(gt), lower=clean(gl),
                     upper=clean(gu))
        return grads, valid

    def vjp(self, saved, cot_y, stats=None):
        """``bounds.py:80-165``: GMRES on (I - J^T) v = g, then the parameter pullback."""
        cfg = self.config
        tau, sigma, operator, g = self._vjp_system(saved, cot_y)
        adjoint, code, residual = batched_restarted_gmres(
            operator, g, tolerance=cfg.linear_tolerance,
            absolute_tolerance=cfg.linear_atol, restart=cfg.linear_restart,
            max_iterations=cfg.linear_max_iterations, stats=stats)
        grads, valid = self._vjp_gradients(saved, tau, sigma, adjoint, code, residual)
        if stats is not None:
            stats.update(code=code, residual=residual, valid=valid, tau=tau, sigma=sigma)
        return grads

    def vjp_shard(self, saved, cot_y):
        """The VJP of one shard of a batch, in the phases a lockstep driver combines.

        ``prepare()`` and ``cycle(completed)`` return this shard's GMRES counters;
        ``finish()`` returns ``(gradients, code, residual)``.  Driven with the
        counters of all shards combined by max, the shards reproduce ``vjp`` of
        the whole batch (one batch-wide budget, ``operators.py:919-1103``).
        """
        cfg = self.config
        tau, sigma, operator, g = self._vjp_system(saved, cot_y)
        solver = LockstepGmres(operator, g, tolerance=cfg.linear_tolerance,
                               absolute_tolerance=cfg.linear_atol, restart=cfg.linear_restart,
                               max_iterations=cfg.linear_max_iterations)
        projection = self

        class _Shard:
            def prepare(self):
                return solver.prepare()

            def cycle(self, completed):
                return solver.cycle(completed)

            def finish(self):
                adjoint, code, residual = solver.result()
                grads, _ = projection._vjp_gradients(saved, tau, sigma, adjoint, code, residual)
                return grads, code, residual

        return _Shard()
