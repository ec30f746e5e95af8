"""Host-side ADMM layouts of the CUDA path (purin_b200/admm.py) against the oracle's (CPU).

The band layout (reverse Cuthill--McKee order, width, banded-factor entries;
admm/factor.py:108-144) and the nominated two-sided row pairs (admm/rows.py:54-84)
are computed once at preparation by the product and, independently, by the
oracle; both must agree for the kernels and the oracle to factor and compact the
same systems.
"""

import numpy as np
import pytest

from oracle.admm import prepare_banded, prepare_pairs
from oracle.sparse import layout
from purin_b200.admm import band_layout, nominate_pairs


def _random_rows(rng, n, m, most):
    rows = []
    for _ in range(m):
        k = int(rng.integers(1, most + 1))
        rows.append(tuple(int(j) for j in rng.choice(n, k, replace=False)))
    return rows


def _chain_rows(n, span):
    return [tuple(range(i, min(i + span, n))) for i in range(n)]


@pytest.mark.parametrize("case", ["chain2", "chain4", "random-narrow", "random-wide", "single"])
def test_band_layout_matches_the_oracle(case):
    rng = np.random.default_rng(len(case))
    n = 24
    rows = {"chain2": _chain_rows(n, 2), "chain4": _chain_rows(n, 4),
            "random-narrow": _random_rows(rng, n, 30, 2),
            "random-wide": _random_rows(rng, n, 30, 6), "single": [(3,)]}[case]
    got = band_layout(rows, n)
    support, mask, _ = layout(rows, n)
    want = prepare_banded(support, mask, n)
    assert (got is None) == (want is None)
    if got is None:
        return
    assert got.width == want.width
    np.testing.assert_array_equal(got.permutation, want.permutation)
    np.testing.assert_array_equal(got.inverse, want.inverse)
    np.testing.assert_array_equal(got.entries[:, 0], want.rows)
    np.testing.assert_array_equal(got.entries[:, 1], want.left)
    np.testing.assert_array_equal(got.entries[:, 2], want.right)
    np.testing.assert_array_equal(got.entries[:, 3], want.destination)


@pytest.mark.parametrize("row_scaling", [False, True])
def test_nominated_pairs_match_the_oracle(row_scaling):
    """Box rows written as opposite inequalities (x <= u, -x <= -l), a doubled copy of a
    coupling row's negation, and rows without a partner."""
    rng = np.random.default_rng(5)
    n, me = 6, 2
    rows, values = [], []
    for _ in range(me):
        cols = tuple(int(j) for j in rng.choice(n, 3, replace=False))
        rows.append(cols)
        values.append(rng.normal(size=3))
    for j in range(n):
        rows += [(j,), (j,)]
        values += [np.array([1.0]), np.array([-1.0])]
    coupling = rng.normal(size=2)
    rows += [(0, 4), (0, 4), (1, 5)]
    values += [coupling, -2.0 * coupling, rng.normal(size=2)]
    got = nominate_pairs(rows, values, me, row_scaling)
    support, mask, _ = layout(rows, n)
    dense = np.zeros(support.shape)
    for r, v in enumerate(values):
        dense[r, :len(v)] = v
    want = prepare_pairs(dense, support, mask, me, n, row_scaling)
    assert (got is None) == (want is None)
    keep, first, second, positions = got
    np.testing.assert_array_equal(keep, want.keep)
    np.testing.assert_array_equal(first, want.first)
    np.testing.assert_array_equal(second, want.second)
    np.testing.assert_array_equal(positions, want.positions)
    # The doubled negation pairs only once rows are scaled to unit norm (a factor
    # of two scales exactly, so the scaled rows are exact opposites).
    assert (len(rows) - 2 in list(second)) == row_scaling
