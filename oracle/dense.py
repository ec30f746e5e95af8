"""Dense / packed diagonal-QP CP adapter (``solve_dense_implicit``).

Oracle (test infrastructure).  Restates
``src/purin/solvers/chambolle_pock/dense_layer.py:13-152``:

* ``ruiz_equilibrate`` (``linalg/equilibration.py:21-57``) and the warm-start
  and multiplier rescaling around it (dense_layer.py:105-113, 146-151);
* the forward ``solve_dense`` (``dense.py:26-105``): ``sparse_cp`` with the
  factored proximal step, the batch-wide loop (no freeze, no stationarity
  test, no validity mask) and power-iteration step sizes, on rows laid out as
  dense equality rows followed by the inequality rows (full, or packed on
  ``inequality_support`` as ``sparse_layer.py`` does);
* the backward (``dense_implicit.py:59-99, 188-217``): the fixed point of one
  CP step with ``tau = s/(max q + ||K||)``, ``sigma = s/||K||``, ``theta = 1``
  and the proximal inverse frozen, so ``q`` gets no cotangent; every sample
  is differentiated.  The linear solve is restarted GMRES (the product's
  solver) in place of the reference's BiCGSTAB: both solve the same system.

The dense products here follow the padded-row order of ``oracle.sparse``; the
reference's dense ``einsum`` sums in its own order, so agreement with the
reference is to rounding, and with the CUDA path bitwise in the forward.
"""

from __future__ import annotations

import numpy as np

from oracle.cp import sparse_cp
from oracle.diagonal_qp import OracleDiagonalQP
from oracle.projection import OracleConfig


def _max_abs_columns(matrix):
    if matrix.shape[1] == 0:
        return np.zeros((matrix.shape[0], matrix.shape[2]), dtype=matrix.dtype)
    return np.max(np.abs(matrix), axis=1)


def _max_abs_rows(matrix):
    if matrix.shape[1] == 0:
        return np.zeros((matrix.shape[0], 0), dtype=matrix.dtype)
    return np.max(np.abs(matrix), axis=2)


def ruiz_equilibrate(q, c, A, b, C, d, lower, upper, *, iterations=4, eps=1e-6):
    """``equilibration.py:21-57``: per pass, columns by max(|A|, |C|, |q|), then rows."""
    dtype = q.dtype
    columns = np.ones_like(q)
    equalities, inequalities = np.ones_like(b), np.ones_like(d)
    epsilon = dtype.type(eps)
    one = dtype.type(1.0)
    for _ in range(int(iterations)):
        metric = np.maximum(_max_abs_columns(A), _max_abs_columns(C))
        metric = np.maximum(metric, np.abs(q))
        update = one / np.sqrt(np.maximum(metric, epsilon))
        A, C = A * update[:, None, :], C * update[:, None, :]
        q, c = q * (update ** 2), c * update
        lower, upper, columns = lower / update, upper / update, columns * update
        if A.shape[1]:
            update = one / np.sqrt(np.maximum(_max_abs_rows(A), epsilon))
            A, b, equalities = A * update[:, :, None], b * update, equalities * update
        if C.shape[1]:
            update = one / np.sqrt(np.maximum(_max_abs_rows(C), epsilon))
            C, d, inequalities = C * update[:, :, None], d * update, inequalities * update
    return q, c, A, b, C, d, lower, upper, columns, equalities, inequalities


class OracleDense:
    """CPU restatement of ``solve_dense_implicit`` for one row layout and option set."""

    def __init__(self, n, me, mi, *, inequality_support=None, accelerated=False, safety=0.95,
                 norm_iterations=20, norm_seed=42, max_iterations=5000, tolerance=1e-9,
                 linear_tolerance=1e-9, linear_max_iterations=100, linear_restart=30):
        if inequality_support is None:
            iq_rows = [tuple(range(n))] * mi
        else:
            iq_rows = [tuple(int(i) for i in row) for row in inequality_support]
        self.qp = OracleDiagonalQP(
            n, [tuple(range(n))] * me, iq_rows,
            OracleConfig(tolerance=tolerance, max_iterations=max_iterations,
                         accelerated=accelerated, safety=safety, norm_iterations=norm_iterations,
                         norm_seed=norm_seed, row_scaling=False, norm_bound=False,
                         linear_tolerance=linear_tolerance,
                         linear_max_iterations=linear_max_iterations,
                         linear_restart=linear_restart))
        self.n, self.me, self.mi = n, me, mi

    def values(self, A, C):
        """Padded row values (batch, m, width) gathered from the dense blocks."""
        dense = np.concatenate((A, C), axis=1)
        support, mask = self.qp.support, self.qp.mask
        rows = np.arange(support.shape[0])[:, None]
        return np.where(mask[None], dense[:, rows, support], dense.dtype.type(0))

    def scaled(self, q, c, A, b, C, d, lower, upper, *, equilibrate=False,
               equilibration_iterations=10):
        """The problem the CP loop sees, with the scales that map back (dense_layer.py:105-113)."""
        if equilibrate:
            return ruiz_equilibrate(q, c, A, b, C, d, lower, upper,
                                    iterations=equilibration_iterations)
        return (q, c, A, b, C, d, lower, upper, np.ones_like(q), np.ones_like(b),
                np.ones_like(d))

    def run(self, q, c, A, b, C, d, lower, upper, *, y0=None, lambda0=None, mu0=None):
        """``dense.py:62-99`` on an already scaled problem: the CPOutput of ``sparse_cp``."""
        cfg = self.qp.config
        batch, n = q.shape
        dtype = q.dtype
        y0 = np.zeros((batch, n), dtype) if y0 is None else y0
        lambda0 = np.zeros((batch, self.me), dtype) if lambda0 is None else lambda0
        mu0 = np.zeros((batch, self.mi), dtype) if mu0 is None else mu0
        return sparse_cp(
            q, c, self.values(A, C), np.concatenate((b, d), axis=1), self.qp.support,
            self.qp.mask, self.me, lower, upper, accelerated=cfg.accelerated, safety=cfg.safety,
            max_iterations=cfg.max_iterations, tolerance=cfg.tolerance,
            norm_iterations=cfg.norm_iterations, norm_seed=cfg.norm_seed, y0=y0,
            dual0=np.concatenate((lambda0, mu0), axis=1), freeze_converged=False,
            check_stationarity=False, norm_bound=False, factored_proximal=True)

    def solve(self, q, c, A, b, C, d, lower, upper, *, equilibrate=False,
              equilibration_iterations=10, y0=None, lambda0=None, mu0=None):
        """``dense_layer.py:82-152``: (y, equality, inequality, iterations) in original units."""
        dtype = q.dtype
        batch, n = q.shape
        (q, c, A, b, C, d, lower, upper, columns, eq_scale, iq_scale) = self.scaled(
            q, c, A, b, C, d, lower, upper, equilibrate=equilibrate,
            equilibration_iterations=equilibration_iterations)
        one = dtype.type(1.0)
        y0 = np.zeros((batch, n), dtype) if y0 is None else y0 / columns
        lambda0 = (np.zeros((batch, self.me), dtype) if lambda0 is None
                   else lambda0 / np.where(eq_scale == 0.0, one, eq_scale))
        mu0 = (np.zeros((batch, self.mi), dtype) if mu0 is None
               else mu0 / np.where(iq_scale == 0.0, one, iq_scale))
        out = self.run(q, c, A, b, C, d, lower, upper, y0=y0, lambda0=lambda0, mu0=mu0)
        me = self.me
        return (columns * out.y, eq_scale * out.dual[:, :me], iq_scale * out.dual[:, me:],
                out.iterations)

    def vjp(self, out, q, c, A, b, C, d, lower, upper, cot_y, cot_dual=None):
        """``dense_implicit.py:207-217`` on the scaled problem: cotangents of q, c, rows, rhs, bounds.

        Returns a dict with ``q`` (zero: frozen proximal), ``c``, ``values``
        (padded rows), ``rhs``, ``lower`` and ``upper``.
        """
        data = (q, c, self.values(A, C), np.concatenate((b, d), axis=1), lower, upper)
        every = out._replace(converged=np.ones(q.shape[0], dtype=bool))
        grads = self.qp.vjp(every, data, cot_y, cot_dual)
        grads["q"] = np.zeros_like(q)
        return grads
