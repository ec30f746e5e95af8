"""Batched restarted GMRES with CGS2 Arnoldi and incremental Givens rotations.

Oracle (test infrastructure).  Restates ``_batched_restarted_gmres`` of
``src/purin/solvers/primal_dual_interior_point/operators.py:792-1125`` for the
arguments the CP implicit VJP passes (``bounds.py:139-147``): identity right
preconditioner, no ``accepted_residual_threshold``, no prefix buckets, zero
initial guess.  The batch runs in lockstep exactly as in the reference: the
Arnoldi loop of a cycle continues while any sample is active, and the
iteration budget (``completed_iterations``) is shared by the whole batch.
"""

from __future__ import annotations

import numpy as np


def _hypot(x, y):
    """``jnp.hypot``: max * sqrt(1 + (min/max)^2), zero when both are zero."""
    dtype = x.dtype
    a = np.abs(x)
    b = np.abs(y)
    inf = np.isposinf(a) | np.isposinf(b)
    hi = np.maximum(a, b)
    lo = np.minimum(a, b)
    safe = np.where(hi == 0, dtype.type(1), hi)
    with np.errstate(invalid="ignore", over="ignore"):
        r = np.where(hi == 0, hi, hi * np.sqrt(dtype.type(1) + np.square(lo / safe)))
    return np.where(inf, dtype.type(np.inf), r)


class LockstepGmres:
    """The batched restarted GMRES of ``operators.py:792-1125``, one cycle per call.

    ``prepare`` computes the thresholds and initial residuals; ``cycle(completed)``
    runs one restart cycle (``cycle_body``, operators.py:919-1097) with the
    budget ``min(restart, max_iterations - completed)`` and returns this batch's
    counters (the cycle's Arnoldi steps, samples still above threshold);
    ``result`` gives ``(x, info, residual_inf)`` (operators.py:1109-1125).  Run
    back to back over the whole batch (``batched_restarted_gmres``) this is the
    reference's loop; run per shard with the shards' counters combined by max
    it is the same loop split across shards.
    """

    def __init__(self, matvec, rhs, *, tolerance, absolute_tolerance, restart, max_iterations):
        self.matvec = matvec
        self.rhs = rhs
        batch, width = rhs.shape
        dtype = rhs.dtype
        self.dtype = dtype
        self.max_iterations = int(max_iterations)
        self.restart = int(min(restart, max_iterations, width))
        rhs_scale = np.max(np.abs(rhs), axis=1, initial=0.0).astype(dtype)
        self.threshold = np.maximum(dtype.type(absolute_tolerance),
                                    dtype.type(tolerance) * rhs_scale)
        self.x = None
        self.residual_inf = None

    def prepare(self):
        rhs = self.rhs
        self.x = np.zeros_like(rhs)
        self.residual_inf = np.max(np.abs(rhs - self.matvec(self.x)), axis=1,
                                   initial=0.0).astype(self.dtype)
        return 0, int(np.sum(self.residual_inf > self.threshold))

    def cycle(self, completed):
        matvec, rhs, x = self.matvec, self.rhs, self.x
        batch, width = rhs.shape
        dtype = self.dtype
        restart = self.restart
        threshold = self.threshold
        residual_inf = self.residual_inf
        eps = dtype.type(1e-30)
        breakdown = dtype.type(1e-14)
        zero = dtype.type(0)
        cycle_limit = min(restart, self.max_iterations - completed)
        residual = rhs - matvec(x)
        beta = np.sqrt(np.sum(residual * residual, axis=1))
        safe_beta = np.maximum(beta, eps)
        cycle_active = residual_inf > threshold
        basis = np.zeros((batch, restart + 1, width), dtype)
        basis[:, 0, :] = residual / safe_beta[:, None]
        hess = np.zeros((batch, restart + 1, restart), dtype)
        cos = np.zeros((batch, restart), dtype)
        sin = np.zeros((batch, restart), dtype)
        g = np.zeros((batch, restart + 1), dtype)
        g[:, 0] = beta
        row_steps = np.zeros(batch, np.int32)
        active = cycle_active.copy()
        it = 0
        while it < cycle_limit and np.any(active):
            vector = basis[:, it, :]
            image = matvec(vector)
            V = basis[:, :restart, :]
            c1 = np.einsum("bid,bd->bi", V, image)
            image = image - np.einsum("bi,bid->bd", c1, V)
            c2 = np.einsum("bid,bd->bi", V, image)
            coefficients = c1 + c2
            image = image - np.einsum("bi,bid->bd", c2, V)
            next_norm = np.sqrt(np.sum(image * image, axis=1))
            next_vector = image / np.maximum(next_norm, eps)[:, None]
            basis[:, it + 1, :] = np.where(active[:, None], next_vector, basis[:, it + 1, :])
            column = np.zeros((batch, restart + 1), dtype)
            column[:, :restart] = coefficients
            column[:, it + 1] = next_norm
            for r in range(it):
                first = column[:, r].copy()
                second = column[:, r + 1].copy()
                column[:, r] = cos[:, r] * first + sin[:, r] * second
                column[:, r + 1] = -sin[:, r] * first + cos[:, r] * second
            diagonal = column[:, it]
            sub = column[:, it + 1]
            rot = _hypot(diagonal, sub)
            safe_rot = np.maximum(rot, eps)
            big = rot > eps
            new_cos = np.where(big, diagonal / safe_rot, dtype.type(1))
            new_sin = np.where(big, sub / safe_rot, zero)
            cos[:, it] = np.where(active, new_cos, cos[:, it])
            sin[:, it] = np.where(active, new_sin, sin[:, it])
            column[:, it] = rot
            column[:, it + 1] = zero
            hess[:, :, it] = np.where(active[:, None], column, hess[:, :, it])
            cur = g[:, it].copy()
            nxt = g[:, it + 1].copy()
            rc = new_cos * cur + new_sin * nxt
            rn = -new_sin * cur + new_cos * nxt
            g[:, it] = np.where(active, rc, cur)
            g[:, it + 1] = np.where(active, rn, nxt)
            row_steps = np.where(active, it + 1, row_steps)
            estimate = np.abs(rn)
            finite = np.isfinite(estimate) & np.isfinite(rot) & np.all(
                np.isfinite(next_vector), axis=1)
            happy = next_norm <= breakdown
            active = active & finite & ~happy & (estimate > threshold)
            it += 1
        # Back substitution over the full restart width (rows >= row_steps give 0).
        coeffs = np.zeros((batch, restart), dtype)
        for row in range(restart - 1, -1, -1):
            trailing = np.sum(hess[:, row, :restart] * coeffs, axis=1)
            numerator = g[:, row] - trailing
            diag = hess[:, row, row]
            safe = np.where(np.abs(diag) > eps, diag, dtype.type(1))
            value = numerator / safe
            coeffs[:, row] = np.where(row < row_steps, value, zero)
        correction = np.einsum("bi,bid->bd", coeffs, basis[:, :restart, :])
        candidate = x + correction
        cand_res = np.max(np.abs(rhs - matvec(candidate)), axis=1, initial=0.0).astype(dtype)
        x = np.where(cycle_active[:, None], candidate, x)
        residual_inf = np.where(cycle_active, cand_res, residual_inf)
        self.x = x
        self.residual_inf = residual_inf
        return it, int(np.sum(residual_inf > threshold))

    def result(self):
        x, residual_inf = self.x, self.residual_inf
        finite = np.all(np.isfinite(x), axis=1) & np.isfinite(residual_inf)
        info = np.where(~finite, 2, np.where(residual_inf <= self.threshold, 0, 1)).astype(np.int32)
        return x, info, residual_inf


def batched_restarted_gmres(matvec, rhs, *, tolerance, absolute_tolerance, restart,
                            max_iterations, stats=None):
    """Solve matvec(x) = rhs per row; returns (x, info, residual_inf)."""
    solver = LockstepGmres(matvec, rhs, tolerance=tolerance,
                           absolute_tolerance=absolute_tolerance, restart=restart,
                           max_iterations=max_iterations)
    _, active = solver.prepare()
    completed = 0
    cycles = 0
    while completed < max_iterations and active > 0:
        steps, active = solver.cycle(completed)
        completed += steps
        cycles += 1
    if stats is not None:
        stats.update(completed=completed, cycles=cycles)
    return solver.result()
