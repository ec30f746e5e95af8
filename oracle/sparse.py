"""Padded row-sparse (ELL) layout and batched products K@x, K.T@y.

Oracle (test infrastructure).  Restates

* ``layout`` -- ``src/purin/solvers/chambolle_pock/kernels.py:26-40``;
* ``matvec`` -- ``_batched_local_jacobian_matvec``,
  ``src/purin/linalg/sparse/operators.py:507-518``: gather ``x[:, support]``,
  multiply by the coefficients, zero the padding, sum over the row width;
* ``tmatvec`` -- ``_batched_local_jacobian_transpose_matvec``,
  ``src/purin/linalg/sparse/operators.py:521-533``: scatter-add of
  ``coefficients * y[:, :, None]`` into ``zeros(n)`` at ``support``.

Both sums are accumulated one term at a time from 0.0 in the reference's
update order: along the row width for ``matvec`` and, for ``tmatvec``, in the
flattened (row, slot) order of the scatter, which is the order an unbuffered
scatter-add applies its updates to each column.  ``tmatvec`` evaluates that
sequence as a column gather over positions sorted by (row, slot), which gives
the same rounding as the scatter itself (checked against ``np.add.at`` in
tests/test_oracle_sparse.py).
"""

from __future__ import annotations

import numpy as np


def layout(rows, n):
    """Padded support (m, width) int32, mask (m, width) bool and flat value positions."""
    width = max(1, max(map(len, rows), default=0))
    support = np.zeros((len(rows), width), dtype=np.int32)
    mask = np.zeros_like(support, dtype=bool)
    positions = []
    for i, row in enumerate(rows):
        support[i, : len(row)] = row
        mask[i, : len(row)] = True
        positions.extend(i * width + j for j in range(len(row)))
    return support, mask, np.asarray(positions, dtype=np.int32)


def _coefficients(values):
    return values if values.ndim == 3 else values[None, :, :]


def matvec(values, support, mask, x):
    """Batched K @ x for padded rows: (B, n) -> (B, m)."""
    m = support.shape[0]
    if m == 0:
        return np.zeros((x.shape[0], 0), dtype=x.dtype)
    coefficients = _coefficients(values)
    zero = x.dtype.type(0.0)
    out = np.zeros((x.shape[0], m), dtype=x.dtype)
    for k in range(support.shape[1]):
        term = coefficients[:, :, k] * x[:, support[:, k]]
        out = out + np.where(mask[None, :, k], term, zero)
    return out


class _ColumnOrder:
    """Per-column list of flat (row, slot) positions in increasing order.

    Padding slots carry column index 0 in the reference layout, so their (zero)
    contributions are scattered into column 0, exactly as in the reference.
    """

    def __init__(self, support, mask, n):
        flat_cols = support.reshape(-1).astype(np.int64)
        order = np.argsort(flat_cols, kind="stable")
        # A padding contribution is +0.0, and adding +0.0 again right after one
        # changes nothing (not even the sign of a zero sum), so each run of
        # consecutive padding terms of a column is kept as its first term.  This
        # keeps column 0 (where every padding slot points) short.
        sorted_cols = flat_cols[order]
        pad = ~mask.reshape(-1)[order]
        repeat = np.zeros_like(pad)
        repeat[1:] = pad[1:] & pad[:-1] & (sorted_cols[1:] == sorted_cols[:-1])
        order = order[~repeat]  # still grouped by column, in flat order within each
        counts = np.bincount(sorted_cols[~repeat], minlength=n)
        starts = np.concatenate([[0], np.cumsum(counts)[:-1]])
        depth = max(1, int(counts.max(initial=0)))
        k = np.arange(depth)
        self.valid = k[None, :] < counts[:, None]
        index = np.where(self.valid, starts[:, None] + k[None, :], 0)
        self.positions = np.where(self.valid, order[np.minimum(index, len(order) - 1)], 0)


_ORDER_CACHE: dict = {}


def _column_order(support, mask, n):
    key = (support.tobytes(), mask.tobytes(), support.shape, n)
    order = _ORDER_CACHE.get(key)
    if order is None:
        order = _ColumnOrder(support, mask, n)
        if len(_ORDER_CACHE) > 64:
            _ORDER_CACHE.clear()
        _ORDER_CACHE[key] = order
    return order


def tmatvec(values, support, mask, y, n):
    """Batched K.T @ y by scatter-add into zeros: (B, m) -> (B, n)."""
    batch = y.shape[0]
    if support.shape[0] == 0:
        return np.zeros((batch, n), dtype=y.dtype)
    coefficients = _coefficients(values)
    zero = y.dtype.type(0.0)
    contributions = np.where(mask[None], coefficients * y[:, :, None], zero)
    flat = contributions.reshape(contributions.shape[0], -1)
    order = _column_order(support, mask, n)
    out = np.zeros((batch, n), dtype=y.dtype)
    for k in range(order.positions.shape[1]):
        term = flat[:, order.positions[:, k]]
        out = np.where(order.valid[None, :, k], out + term, out)
    return out
