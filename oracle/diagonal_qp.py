"""General diagonal QP on the Chambolle--Pock kernels (``PreparedDiagonalQP``).

Oracle (test infrastructure).  Restates ``src/purin/solvers/diagonal_qp.py``:

* the layout of ALL rows, equalities then inequalities, without a bound
  presolve (``PreparedDiagonalQP.__post_init__``, diagonal_qp.py:81-89);
* the custom-VJP forward (diagonal_qp.py:99-123): ``sparse_cp`` with per-sample
  q, c, warm starts, ``freeze_converged`` and ``check_stationarity``, then
  ``converged &= all(q > 0) & all(lower <= upper)``;
* its backward (diagonal_qp.py:133-220): step sizes (diagonal, norm bound or
  power iteration, tau = s/(max q + L)), GMRES on (I - J^T) v = (cot_y,
  cot_dual, 0) and the pullback of one CP step to every ``QPData`` field;
* ``solve`` (diagonal_qp.py:225-314): shape checks, row scaling, tolerance,
  dual rescaling and the diagnostics in original units.

``qp_step_pullback`` is what ``jax.vjp`` computes for ``cp_step`` with the
proximal coefficients evaluated inside the step (``proximal=None``,
kernels.py:68-73,91-150), so q and c receive cotangents.
"""

from __future__ import annotations

import numpy as np

from oracle.cp import (
    _balanced,
    _row_max,
    clip,
    diagonal_step_sizes,
    mv_cot,
    norm_estimate,
    operators,
    sparse_cp,
)
from oracle.gmres import batched_restarted_gmres
from oracle.projection import CONVERGED, MAX_ITERATIONS, NONFINITE, OracleConfig, _seq_sum_last
from oracle.sparse import layout

QP_FIELDS = ("q", "c", "values", "rhs", "lower", "upper")


def qp_step_pullback(state, q, c, values, rhs, lower, upper, support, mask, me, tau, sigma,
                     cotangent):
    """VJP of ``cp_step(state, q, c, rhs, lower, upper, K, K.T, me, tau, sigma, 1)``.

    Returns ``((state_y, state_dual, state_ybar), {q, c, values, rhs, lower,
    upper})`` for the output cotangent ``(v_y, v_dual, v_ybar)``
    (diagonal_qp.py:164-190: ``jax.vjp(step, state, data)``).  The transposes
    follow JAX's rules: ``1/den`` passes ``-((ct * (den*den)^-1) * 1)`` to den
    (``div``'s JVP with ``integer_pow(den, -2)``), products pass ``ct`` times the
    other factor.
    """
    y, dual, ybar = state
    v_y, v_dual, v_ybar = cotangent
    dtype = y.dtype
    n = y.shape[1]
    zero = dtype.type(0.0)
    one = dtype.type(1.0)
    mv, tmv = operators(values, support, mask, n)
    sig = sigma[:, None] if sigma.ndim == 1 else sigma
    step = tau[:, None] if tau.ndim == 1 else tau
    raw_dual = dual + sig * (mv(ybar) - rhs)
    raw_in = raw_dual[:, me:]
    pos_in = np.maximum(raw_in, zero)
    next_dual = np.concatenate((raw_dual[:, :me], pos_in), axis=1)
    den = one + step * q
    inverse = one / den
    dual_weight = step * inverse
    t = tmv(next_dual)
    y_raw = inverse * y - dual_weight * t + (-dual_weight) * c
    u1 = np.maximum(lower, y_raw)
    y_next = np.minimum(upper, u1)
    g = (v_y + v_ybar) + v_ybar
    d_u1 = _balanced(u1, y_next, upper)
    d_up = _balanced(upper, y_next, u1)
    d_raw = _balanced(y_raw, u1, lower)
    d_lo = _balanced(lower, u1, y_raw)
    g_u1 = g * d_u1
    g_raw = g_u1 * d_raw
    g_lower = g_u1 * d_lo
    g_upper = g * d_up
    g_t = dual_weight * -g_raw
    g_c = (-dual_weight) * g_raw
    g_dw = ((-g_raw) * t) + (-(g_raw * c))
    g_inv = (g_raw * y) + (step * g_dw)
    g_q = step * (-((g_inv * (one / (den * den))) * one))
    mu = v_dual + mv_cot(values, support, mask, g_t)
    f_in = _balanced(raw_in, pos_in, np.zeros_like(raw_in))
    mu_raw = np.concatenate((mu[:, :me], mu[:, me:] * f_in), axis=1)
    w = sig * mu_raw
    state_y = inverse * g_raw - v_ybar
    state_ybar = tmv(w)
    g_values = np.where(
        mask[None], w[:, :, None] * ybar[:, support] + g_t[:, support] * next_dual[:, :, None],
        zero)
    grads = dict(q=g_q, c=g_c, values=g_values, rhs=-w, lower=g_lower, upper=g_upper)
    return (state_y, mu_raw, state_ybar), grads


class OracleDiagonalQP:
    """CPU restatement of ``QPStructure(...).prepare(batch_size, config)``."""

    def __init__(self, n, equality_rows, inequality_rows, config=None, partitionable=True):
        self.config = config or OracleConfig()
        self.n = int(n)
        self.me = len(equality_rows)
        self.rows = [tuple(r) for r in equality_rows] + [tuple(r) for r in inequality_rows]
        self.support, self.mask, _ = layout(self.rows, self.n)
        self.partitionable = partitionable

    # -- custom-VJP boundary ---------------------------------------------------
    def run(self, data, y0, dual0, tolerance, *, offset=0, total=None):
        """``diagonal_qp.py:99-123`` on (scaled) ``data``; returns the CPOutput."""
        cfg = self.config
        q, c, values, rhs, lower, upper = data
        out = sparse_cp(
            q, c, values, rhs, self.support, self.mask, self.me, lower, upper,
            accelerated=cfg.accelerated, safety=cfg.safety, max_iterations=cfg.max_iterations,
            tolerance=tolerance, norm_iterations=cfg.norm_iterations, norm_seed=cfg.norm_seed,
            y0=y0, dual0=dual0, freeze_converged=True, check_stationarity=True,
            norm_bound=cfg.norm_bound, diagonal_preconditioning=cfg.diagonal_preconditioning,
            offset=offset, total=total, partitionable=self.partitionable)
        valid = np.all(q > 0, axis=1) & np.all(lower <= upper, axis=1)
        return out._replace(converged=out.converged & valid)

    def step_sizes(self, data, *, offset=0, total=None):
        """``diagonal_qp.py:135-150``: the backward's (tau, sigma)."""
        cfg = self.config
        q, _, values, rhs, _, _ = data
        dtype = q.dtype
        if cfg.diagonal_preconditioning and not cfg.accelerated:
            return diagonal_step_sizes(q, values, self.support, self.mask, cfg.safety)
        if cfg.norm_bound:
            amv, atmv = operators(np.abs(values), self.support, self.mask, self.n)
            L = np.sqrt(_row_max(amv(np.ones_like(q)), 0.0) * _row_max(atmv(np.ones_like(rhs)), 0.0))
        else:
            mv, tmv = operators(values, self.support, self.mask, self.n)
            L = norm_estimate(mv, tmv, q.shape[0], self.n, dtype, cfg.norm_iterations,
                              cfg.norm_seed, offset=offset, total=total,
                              partitionable=self.partitionable)
        L = np.maximum(L, dtype.type(1e-12))
        s = dtype.type(cfg.safety)
        return (s / (np.max(q, axis=1) + L)).astype(dtype), (s / L).astype(dtype)

    def vjp(self, out, data, cot_y, cot_dual=None, *, offset=0, total=None, stats=None):
        """``diagonal_qp.py:133-220``: cotangents of every field of the (scaled) data."""
        cfg = self.config
        q = data[0]
        dtype = q.dtype
        zero = dtype.type(0)
        n, m = self.n, data[3].shape[1]
        tau, sigma = self.step_sizes(data, offset=offset, total=total)

        def pullback(v):
            return qp_step_pullback((out.y, out.dual, out.y), *data, self.support, self.mask,
                                    self.me, tau, sigma, (v[:, :n], v[:, n:n + m], v[:, n + m:]))

        def operator(v):
            (sy, sd, sb), _ = pullback(v)
            return v - np.concatenate((sy, sd, sb), axis=1)

        dual_cot = np.zeros_like(out.dual) if cot_dual is None else cot_dual
        g = np.concatenate((cot_y, dual_cot, np.zeros_like(out.y)), axis=1)
        g = np.where(out.converged[:, None], g, zero)
        adjoint, code, residual = batched_restarted_gmres(
            operator, g, tolerance=cfg.linear_tolerance, absolute_tolerance=cfg.linear_atol,
            restart=cfg.linear_restart, max_iterations=cfg.linear_max_iterations, stats=stats)
        valid = (out.converged & np.all(np.isfinite(adjoint), axis=1) & np.isfinite(residual)
                 & ((code == 0) | (residual <= dtype.type(cfg.adjoint_tolerance))))
        _, grads = pullback(np.where(valid[:, None], adjoint, zero))
        if stats is not None:
            stats.update(code=code, residual=residual, valid=valid, tau=tau, sigma=sigma)
        return {k: np.nan_to_num(v, nan=0.0, posinf=0.0, neginf=0.0) for k, v in grads.items()}

    # -- public solve ------------------------------------------------------------
    def row_scale(self, values):
        """``diagonal_qp.py:256-262``: 1/||row||_2 of the padded rows (1 for empty rows)."""
        dtype = values.dtype
        one = dtype.type(1.0)
        if not self.config.row_scaling:
            return np.ones(values.shape[:2], dtype)
        norms = np.sqrt(_seq_sum_last(np.where(self.mask[None], values * values, 0)))
        return np.where(norms > 0, one / np.maximum(norms, dtype.type(1e-30)), one)

    def solve(self, data, initial_y=None, initial_dual=None, *, offset=0, total=None):
        """``diagonal_qp.py:225-314``; returns (result dict, saved boundary state)."""
        cfg = self.config
        q, c, values, rhs, lower, upper = (np.asarray(x) for x in data)
        dtype = q.dtype
        batch, n = q.shape
        m = rhs.shape[1]
        y0 = np.zeros((batch, n), dtype) if initial_y is None else np.asarray(initial_y, dtype)
        dual0 = (np.zeros((batch, m), dtype) if initial_dual is None
                 else np.asarray(initial_dual, dtype))
        scale = self.row_scale(values)
        scaled = (q, c, values * scale[:, :, None], rhs * scale, lower, upper)
        tolerance = dtype.type(cfg.tolerance) * np.minimum(
            dtype.type(1.0), np.min(scale, axis=1, initial=1.0).astype(dtype))
        out = self.run(scaled, y0, dual0 / scale, tolerance, offset=offset, total=total)
        saved = dict(out=out, data=scaled, scale=scale, tolerance=tolerance, y0=y0,
                     dual0=dual0 / scale, offset=offset, total=total)
        dual = out.dual * scale
        mv, tmv = operators(values, self.support, self.mask, n)
        residuals = mv(out.y) - rhs
        me = self.me
        eq = _row_max(np.abs(residuals[:, :me]), 0.0)
        iq = _row_max(np.maximum(residuals[:, me:], dtype.type(0)), 0.0)
        stationarity = np.max(np.abs(out.y - clip(out.y - (q * out.y + c + tmv(dual)), lower,
                                                  upper)), axis=1)
        residual = np.maximum(np.maximum(eq, iq), stationarity)
        converged = out.converged & (residual <= dtype.type(cfg.tolerance))
        finite = (np.all(np.isfinite(out.y), axis=1) & np.all(np.isfinite(dual), axis=1)
                  & np.isfinite(residual))
        status = np.where(converged, CONVERGED, np.where(finite, MAX_ITERATIONS, NONFINITE))
        slacks = np.maximum(rhs[:, me:] - mv(out.y)[:, me:], dtype.type(0))
        result = dict(y=out.y, multipliers_eq=dual[:, :me], multipliers_ineq=dual[:, me:],
                      slacks=slacks, status=status.astype(np.int32), iterations=out.iterations,
                      residual_inf_norm=residual, finite=finite, gradient_eligible=converged)
        return result, saved
