"""Batched Chambolle--Pock iteration for diagonal QPs, and its one-step pullback.

Oracle (test infrastructure).  Restates ``src/purin/solvers/chambolle_pock/
kernels.py`` (the whole numerical section, lines 52-305) in NumPy:

    minimise 0.5 y' diag(q) y + c' y
    s.t.     K[:me] y = rhs[:me],  K[me:] y <= rhs[me:],  lower <= y <= upper.

``cp_step_pullback`` restates what ``jax.vjp`` computes for one fixed-step CP
update at ``src/purin/solvers/chambolle_pock/bounds.py:109-129`` (and
``solver.py:217-236``): the transpose of the linearised step, with JAX's
tie rule for ``max``/``min`` (a tie passes half of the cotangent to each
argument: ``jax.lax.max``'s JVP uses ``_balanced_eq``).

Maxima and minima propagate NaN like ``jax.lax.max``/``min``.  ``clip`` is
``minimum(upper, maximum(lower, x))``, the operation order of ``jnp.clip``.
"""

from __future__ import annotations

from typing import NamedTuple

import numpy as np

from oracle.prng import batch_normals
from oracle.sparse import matvec, tmatvec


class CPOutput(NamedTuple):
    """``kernels.py:15-23``: iterates, per-sample counts, residual, gap, convergence."""

    y: np.ndarray
    dual: np.ndarray
    iterations: np.ndarray
    residual: np.ndarray
    gap: np.ndarray
    converged: np.ndarray


def clip(x, lower, upper):
    """``jnp.clip``: ``minimum(upper, maximum(lower, x))`` with NaN propagation."""
    return np.minimum(upper, np.maximum(lower, x))


def _row_max(x, initial=None):
    if x.shape[1] == 0:
        return np.full(x.shape[0], 0.0 if initial is None else initial, dtype=x.dtype)
    out = np.max(x, axis=1)
    if initial is not None:
        out = np.maximum(out, x.dtype.type(initial))
    return out


def operators(values, support, mask, n):
    """``kernels.py:43-49``: batched K@x and K.T@y callables."""
    return (
        lambda x: matvec(values, support, mask, x),
        lambda y: tmatvec(values, support, mask, y, n),
    )


def norm_estimate(
    mv, tmv, batch, n, dtype, iterations=20, seed=42, *, offset=0, total=None,
    partitionable=True,
):
    """``kernels.py:52-65``: power iteration on K.T K from seeded normal starts.

    ``offset``/``total`` select rows ``offset..offset+batch-1`` of the global
    ``split(PRNGKey(seed), total)`` so a shard of the batch reproduces the
    keys the whole batch would use.
    """
    dtype = np.dtype(dtype)
    x = batch_normals(seed, batch, n, dtype, offset, total, partitionable)
    eps = dtype.type(1e-12)
    x = x / (np.sqrt(np.sum(x * x, axis=1, keepdims=True)) + eps)
    eigenvalue = np.zeros(batch, dtype)
    for _ in range(iterations):
        z = tmv(mv(x))
        eigenvalue = np.sum(x * z, axis=1)
        x = z / (np.sqrt(np.sum(z * z, axis=1, keepdims=True)) + eps)
    return np.sqrt(np.maximum(eigenvalue, dtype.type(0))) + eps


def proximal_coefficients(q, c, tau):
    """``kernels.py:68-73``: a = 1/(1+tau q), d = tau a, offset = -d c."""
    step = tau[:, None] if tau.ndim == 1 else tau
    one = q.dtype.type(1)
    inverse = one / (one + step * q)
    dual_weight = step * inverse
    return inverse, dual_weight, -dual_weight * c


def diagonal_step_sizes(q, values, support, mask, safety):
    """``kernels.py:76-88``: tau_j = safety/colsum_j, sigma_i = safety/rowsum_i of |K|."""
    dtype = q.dtype
    mv, tmv = operators(np.abs(values), support, mask, q.shape[1])
    row = mv(np.ones_like(q))
    column = tmv(np.ones_like(row))
    tiny = dtype.type(1e-12)
    one = dtype.type(1.0)
    row = np.where(row > 0, np.maximum(row, tiny), one)
    column = np.where(column > 0, np.maximum(column, tiny), one)
    s = dtype.type(safety)
    return s / column, s / row


def cp_step(state, q, c, rhs, lower, upper, mv, tmv, me, tau, sigma, theta, proximal=None,
            factored_proximal=False):
    """``kernels.py:91-150``: one CP update plus extrapolation.

    ``factored_proximal`` is the dense adapter's form (kernels.py:142-149):
    ``inverse * ((y - tau K^T l) - tau c)`` clipped as ``minimum(maximum(., l), u)``.
    """
    y, dual, ybar = state
    dtype = y.dtype
    dual_step = sigma[:, None] if sigma.ndim == 1 else sigma
    next_dual = dual + dual_step * (mv(ybar) - rhs)
    next_dual = np.concatenate(
        (next_dual[:, :me], np.maximum(next_dual[:, me:], dtype.type(0))), axis=1
    )
    inverse, dual_weight, offset = (
        proximal_coefficients(q, c, tau) if proximal is None else proximal
    )
    if factored_proximal:
        step = tau[:, None] if tau.ndim == 1 else tau
        next_y = inverse * ((y - step * tmv(next_dual)) - step * c)
        next_y = np.minimum(np.maximum(next_y, lower), upper)
    else:
        next_y = inverse * y - dual_weight * tmv(next_dual) + offset
        next_y = clip(next_y, lower, upper)
    return next_y, next_dual, next_y + theta[:, None] * (next_y - y)


def diagnostics(y, dual, q, c, rhs, lower, upper, mv, tmv, me):
    """``kernels.py:153-175``: max feasibility violation and normalised gap."""
    dtype = y.dtype
    zero = dtype.type(0.0)
    half = dtype.type(0.5)
    one = dtype.type(1.0)
    residuals = mv(y) - rhs
    eq = _row_max(np.abs(residuals[:, :me]), 0.0)
    ineq = _row_max(np.maximum(residuals[:, me:], zero), 0.0)
    bound = np.maximum(
        _row_max(np.maximum(lower - y, zero), 0.0),
        _row_max(np.maximum(y - upper, zero), 0.0),
    )
    primal = np.sum(half * q * y * y + c * y, axis=1)
    t = c + tmv(dual)
    positive = q > dtype.type(1e-12)
    free = -t / np.where(positive, q, one)
    minimizer = np.where(
        positive, clip(free, lower, upper), np.where(t >= zero, lower, upper)
    )
    dual_objective = np.sum(half * q * minimizer**2 + t * minimizer, axis=1) - np.sum(
        rhs * dual, axis=1
    )
    gap = np.maximum(primal - dual_objective, zero) / np.maximum(
        one, np.maximum(np.abs(primal), np.abs(dual_objective))
    )
    return np.maximum(np.maximum(eq, ineq), bound), gap


def step_sizes(q, values, support, mask, rhs, *, accelerated, safety, norm_iterations,
               norm_seed, norm_bound, diagonal_preconditioning, offset=0, total=None,
               partitionable=True):
    """``kernels.py:209-227``: per-sample (tau, sigma) for the forward solve."""
    batch, n = q.shape
    dtype = q.dtype
    mv, tmv = operators(values, support, mask, n)
    if diagonal_preconditioning and not accelerated:
        return diagonal_step_sizes(q, values, support, mask, safety)
    if norm_bound:
        amv, atmv = operators(np.abs(values), support, mask, n)
        row_sum = amv(np.ones_like(q))
        column_sum = atmv(np.ones_like(rhs))
        norm = np.sqrt(_row_max(row_sum, 0.0) * _row_max(column_sum, 0.0))
    else:
        norm = norm_estimate(mv, tmv, batch, n, dtype, norm_iterations, norm_seed,
                             offset=offset, total=total, partitionable=partitionable)
    L = np.maximum(norm, dtype.type(1e-12))
    s = dtype.type(safety)
    sigma = s / L
    use_accel = accelerated and np.min(q, axis=1) > 0
    tau = np.where(use_accel, s / L, s / (np.max(q, axis=1) + L))
    return tau.astype(dtype), sigma.astype(dtype)


def sparse_cp(q, c, values, rhs, support, mask, me, lower, upper, *, accelerated=False,
              safety=0.95, max_iterations=5000, tolerance=1e-9, norm_iterations=20,
              norm_seed=42, y0=None, dual0=None, freeze_converged=False,
              check_stationarity=False, norm_bound=False, diagonal_preconditioning=False,
              offset=0, total=None, partitionable=True, trace=None, factored_proximal=False):
    """``kernels.py:178-305``: batched fixed-step or accelerated CP with per-sample freeze."""
    batch, n = q.shape
    dtype = q.dtype
    zero = dtype.type(0.0)
    one = dtype.type(1.0)
    mv, tmv = operators(values, support, mask, n)
    tau, sigma = step_sizes(
        q, values, support, mask, rhs, accelerated=accelerated, safety=safety,
        norm_iterations=norm_iterations, norm_seed=norm_seed, norm_bound=norm_bound,
        diagonal_preconditioning=diagonal_preconditioning, offset=offset, total=total,
        partitionable=partitionable,
    )
    tolerance = np.broadcast_to(np.asarray(tolerance, dtype=dtype), (batch,))
    gamma = np.min(q, axis=1)
    y = np.zeros_like(q) if y0 is None else np.array(y0, dtype=dtype)
    dual = np.zeros_like(rhs) if dual0 is None else np.array(dual0, dtype=dtype)
    ybar = y.copy()
    theta = np.ones(batch, dtype)
    done = np.zeros(batch, bool)
    counts = np.zeros(batch, np.int32)
    proximal = None if accelerated else proximal_coefficients(q, c, tau)
    iteration = 0
    while iteration < max_iterations and not np.all(done):
        ny, nd, nb = cp_step((y, dual, ybar), q, c, rhs, lower, upper, mv, tmv, me, tau,
                             sigma, theta, proximal=proximal, factored_proximal=factored_proximal)
        residual, gap = diagnostics(ny, nd, q, c, rhs, lower, upper, mv, tmv, me)
        finite = (np.all(np.isfinite(ny), axis=1) & np.all(np.isfinite(nd), axis=1)
                  & np.isfinite(gap))
        active = ~done if freeze_converged else np.ones_like(done)
        y = np.where(active[:, None], ny, y)
        dual = np.where(active[:, None], nd, dual)
        ybar = np.where(active[:, None], nb, ybar)
        counts = counts + active.astype(np.int32)
        stationarity = np.max(np.abs(ny - clip(ny - (q * ny + c + tmv(nd)), lower, upper)),
                              axis=1)
        accepted = finite & (residual <= tolerance) & (gap <= tolerance)
        if check_stationarity:
            accepted = accepted & (stationarity <= tolerance)
        done = done | accepted
        if trace is not None:
            trace.append(dict(residual=residual, gap=gap, stationarity=stationarity))
        if accelerated:
            nt = one / np.sqrt(one + gamma * tau)
            tau = nt * tau
            sigma = sigma / nt
            theta = nt
        iteration += 1
    residual, gap = diagnostics(y, dual, q, c, rhs, lower, upper, mv, tmv, me)
    finite = (np.all(np.isfinite(y), axis=1) & np.all(np.isfinite(dual), axis=1)
              & np.isfinite(gap) & np.isfinite(residual))
    converged = finite & (residual <= tolerance) & (gap <= tolerance)
    if check_stationarity:
        stationarity = np.max(np.abs(y - clip(y - (q * y + c + tmv(dual)), lower, upper)),
                              axis=1)
        converged = converged & (stationarity <= tolerance)
        residual = np.maximum(residual, stationarity)
    return CPOutput(y, dual, counts, residual, gap, converged)


def _balanced(x, ans, other):
    """``jax.lax`` max/min JVP weight of argument ``x``: (x==ans) / (other==ans ? 2 : 1)."""
    dtype = ans.dtype
    hit = (x == ans).astype(dtype)
    return hit / np.where(other == ans, dtype.type(2), dtype.type(1))


def cp_step_pullback(state, values, rhs, target, lower, upper, support, mask, me, tau,
                     sigma, cotangent):
    """VJP of the fixed-step CP map ``step`` of ``bounds.py:109-129`` at ``state``.

    The map is ``cp_step((y, dual, ybar), 1, -target, rhs, lower, upper, K, K.T,
    me, tau, sigma, theta=1)``.  Returns the cotangents of (state, values,
    rhs, target, lower, upper) for the output cotangent ``(v_y, v_dual, v_ybar)``.
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
    # Primal recomputation (residuals of the linearisation).
    raw_dual = dual + sig * (mv(ybar) - rhs)
    raw_in = raw_dual[:, me:]
    pos_in = np.maximum(raw_in, zero)
    next_dual = np.concatenate((raw_dual[:, :me], pos_in), axis=1)
    inverse = one / (one + step * one)
    dual_weight = step * inverse
    t = tmv(next_dual)
    y_raw = inverse * y - dual_weight * t + (-dual_weight * -target)
    u1 = np.maximum(lower, y_raw)
    y_next = np.minimum(upper, u1)
    # Cotangents.
    g = (v_y + v_ybar) + v_ybar  # next_y feeds next_y and next_y + (next_y - y)
    d_u1 = _balanced(u1, y_next, upper)
    d_up = _balanced(upper, y_next, u1)
    d_raw = _balanced(y_raw, u1, lower)
    d_lo = _balanced(lower, u1, y_raw)
    g_u1 = g * d_u1
    g_raw = g_u1 * d_raw
    g_lower = g_u1 * d_lo
    g_upper = g * d_up
    g_t = dual_weight * -g_raw
    g_target = dual_weight * g_raw
    mu = v_dual + mv_cot(values, support, mask, g_t)
    f_in = _balanced(raw_in, pos_in, np.zeros_like(raw_in))
    mu_raw = np.concatenate((mu[:, :me], mu[:, me:] * f_in), axis=1)
    w = sig * mu_raw
    g_rhs = -w
    state_y = inverse * g_raw - v_ybar
    state_ybar = tmv(w)
    gathered_ybar = ybar[:, support]
    gathered_t = g_t[:, support]
    g_values = np.where(
        mask[None], w[:, :, None] * gathered_ybar + gathered_t * next_dual[:, :, None], zero
    )
    return ((state_y, mu_raw, state_ybar), g_values, g_rhs, g_target, g_lower, g_upper)


def mv_cot(values, support, mask, g_t):
    """Transpose of ``t = K.T @ dual`` applied to ``g_t``: gather then row sums (K @ g_t)."""
    return matvec(values, support, mask, g_t)
