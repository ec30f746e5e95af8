"""Padded-ELL products of the oracle against dense algebra and the literal scatter order.

Restates the property checked by the reference's ``tests/test_sparse_layouts.py:17-81``
(row-sparse products equal dense einsum) for the oracle's operators.
"""

import numpy as np

from oracle.sparse import layout, matvec, tmatvec


def _random(rng, m, n, batch, density=0.3):
    rows = [tuple(sorted(rng.choice(n, max(1, rng.binomial(n, density)), replace=False)))
            for _ in range(m)]
    support, mask, positions = layout(rows, n)
    values = np.where(mask[None], rng.normal(size=(batch,) + support.shape), 0.0)
    dense = np.zeros((batch, m, n))
    for i, r in enumerate(rows):
        for k, j in enumerate(r):
            dense[:, i, j] = values[:, i, k]
    return rows, support, mask, positions, values, dense


def test_layout_positions_and_padding():
    support, mask, positions = layout([(0, 2), (1,), ()], 4)
    assert support.shape == (3, 2)
    np.testing.assert_array_equal(mask, [[True, True], [True, False], [False, False]])
    np.testing.assert_array_equal(positions, [0, 1, 2])
    np.testing.assert_array_equal(support[1], [1, 0])


def test_products_match_dense():
    rng = np.random.default_rng(0)
    _, support, mask, _, values, dense = _random(rng, 7, 9, 3)
    x = rng.normal(size=(3, 9))
    y = rng.normal(size=(3, 7))
    np.testing.assert_allclose(matvec(values, support, mask, x),
                               np.einsum("bij,bj->bi", dense, x), atol=1e-13)
    np.testing.assert_allclose(tmatvec(values, support, mask, y, 9),
                               np.einsum("bij,bi->bj", dense, y), atol=1e-13)


def test_transpose_is_the_sequential_scatter_bit_for_bit():
    """The column gather adds each column's terms in (row, slot) order, like np.add.at."""
    rng = np.random.default_rng(1)
    _, support, mask, _, values, _ = _random(rng, 40, 13, 2, density=0.5)
    y = rng.normal(size=(2, 40)) * 1e3
    got = tmatvec(values, support, mask, y, 13)
    contributions = np.where(mask[None], values * y[:, :, None], 0.0)
    for b in range(2):
        ref = np.zeros(13)
        np.add.at(ref, support.reshape(-1), contributions[b].reshape(-1))
        np.testing.assert_array_equal(got[b], ref)


def test_shared_values_broadcast():
    rng = np.random.default_rng(2)
    _, support, mask, _, values, _ = _random(rng, 5, 6, 1)
    x = rng.normal(size=(4, 6))
    np.testing.assert_array_equal(matvec(values[0], support, mask, x),
                                  matvec(np.repeat(values, 4, axis=0), support, mask, x))


def test_empty_operator():
    support, mask, _ = layout([], 3)
    assert matvec(np.zeros((1, 0, 1)), support, mask, np.ones((2, 3))).shape == (2, 0)
    np.testing.assert_array_equal(tmatvec(np.zeros((1, 0, 1)), support, mask, np.ones((2, 0)), 3),
                                  np.zeros((2, 3)))
