"""Dense CP adapter oracle against the reference's analytic cases (tests/test_dense_cp.py)."""

import numpy as np
import pytest
import torch

from oracle.cp import sparse_cp
from oracle.dense import OracleDense, ruiz_equilibrate
from purin_b200.dense_layer import ruiz_equilibrate as torch_ruiz


def _equality_qp():
    """``test_dense_cp.py:22-31``: y* = (1/3, 2/3)."""
    q = np.array([[2.0, 4.0]])
    c = np.array([[-2.0, -4.0]])
    A = np.ones((1, 1, 2))
    b = np.ones((1, 1))
    C = np.array([[[-1.0, 0.0]]])
    d = np.zeros((1, 1))
    lo = np.zeros((1, 2))
    hi = np.ones((1, 2)) * 2
    return q, c, A, b, C, d, lo, hi


ANALYTIC_JACOBIAN = -np.diag([0.5, 0.25]) + np.outer([0.5, 0.25], [0.5, 0.25]) / 0.75


@pytest.mark.parametrize("accelerated", [False, True])
@pytest.mark.parametrize("equilibrate", [False, True])
def test_oracle_dense_analytic_equality_qp(accelerated, equilibrate):
    args = _equality_qp()
    oracle = OracleDense(2, 1, 1, accelerated=accelerated, tolerance=1e-13, max_iterations=20000)
    y, eq, iq, iterations = oracle.solve(*args, equilibrate=equilibrate)
    np.testing.assert_allclose(y, [[1 / 3, 2 / 3]], atol=1e-6)
    # Warm start from the solution stays there (test_dense_cp.py:40-46).
    warm = oracle.solve(*args, equilibrate=equilibrate, y0=y, lambda0=eq, mu0=iq)
    np.testing.assert_allclose(warm[0], y, atol=1e-6)
    # Implicit Jacobian dy/dc (test_dense_cp.py:47-51), through the Ruiz column
    # scaling: y = columns * y_s with c_s = columns * c.
    scaled = oracle.scaled(*args, equilibrate=equilibrate)
    columns = scaled[8]
    out = oracle.run(*scaled[:8], y0=None)
    rows = []
    for i in range(2):
        cot = np.zeros((1, 2))
        cot[0, i] = 1.0
        grads = oracle.vjp(out, *scaled[:8], cot * columns)
        rows.append((grads["c"] * columns)[0])
        assert np.all(grads["q"] == 0.0)
    np.testing.assert_allclose(np.array(rows), ANALYTIC_JACOBIAN, atol=1e-6)


def test_oracle_dense_empty_constraints():
    """``test_dense_cp.py:61-78``: no rows, box [0, 3], y* = -c / q."""
    q = np.ones((1, 2))
    c = np.array([[-1.0, -2.0]])
    empty = np.zeros((1, 0, 2))
    oracle = OracleDense(2, 0, 0, tolerance=1e-14)
    y, eq, iq, _ = oracle.solve(q, c, empty, np.zeros((1, 0)), empty, np.zeros((1, 0)),
                                np.zeros((1, 2)), np.ones((1, 2)) * 3, equilibrate=True)
    np.testing.assert_allclose(y, [[1.0, 2.0]], atol=1e-6)
    assert eq.shape == (1, 0) and iq.shape == (1, 0)


def _random_dense(batch, n, me, mi, seed):
    rng = np.random.default_rng(seed)
    q = rng.uniform(0.5, 2.0, (batch, n))
    c = rng.normal(size=(batch, n))
    A = rng.normal(size=(batch, me, n))
    C = rng.normal(size=(batch, mi, n))
    y_feasible = rng.uniform(-0.5, 0.5, (batch, n))
    b = np.einsum("bmn,bn->bm", A, y_feasible)
    d = np.einsum("bmn,bn->bm", C, y_feasible) + rng.uniform(0.0, 0.5, (batch, mi))
    return q, c, A, b, C, d, -np.ones((batch, n)), np.ones((batch, n))


def test_trip_count_two_pass_equals_shared_loop():
    """The CUDA path's two passes reproduce the reference's batch-wide loop.

    A first pass with per-sample freezing gives each sample's first
    acceptance; rerunning without freezing for max(first acceptance)
    iterations is the shared loop of ``kernels.py`` (dense.py:79-99) exactly.
    """
    q, c, A, b, C, d, lo, hi = _random_dense(4, 6, 2, 3, seed=3)
    q[0] *= 4.0  # spread the samples' iteration counts
    oracle = OracleDense(6, 2, 3, tolerance=1e-8, max_iterations=4000)
    values = oracle.values(A, C)
    rhs = np.concatenate((b, d), axis=1)
    common = dict(tolerance=1e-8, check_stationarity=False, norm_bound=False,
                  factored_proximal=True)
    support, mask = oracle.qp.support, oracle.qp.mask
    first = sparse_cp(q, c, values, rhs, support, mask, 2, lo, hi, max_iterations=4000,
                      freeze_converged=True, **common)
    trips = int(first.iterations.max())
    assert len(set(first.iterations.tolist())) > 1
    second = sparse_cp(q, c, values, rhs, support, mask, 2, lo, hi, max_iterations=trips,
                       freeze_converged=False, **common)
    shared = oracle.run(q, c, A, b, C, d, lo, hi)
    np.testing.assert_array_equal(second.y, shared.y)
    np.testing.assert_array_equal(second.dual, shared.dual)
    np.testing.assert_array_equal(shared.iterations, np.full(4, trips))


def test_ruiz_torch_matches_oracle():
    q, c, A, b, C, d, lo, hi = _random_dense(3, 5, 2, 4, seed=7)
    ref = ruiz_equilibrate(q, c, A, b, C, d, lo, hi, iterations=10)
    got = torch_ruiz(*(torch.as_tensor(x) for x in (q, c, A, b, C, d, lo, hi)), iterations=10)
    for r, g in zip(ref, got):
        np.testing.assert_allclose(g.numpy(), r, rtol=1e-15, atol=0)


def test_ruiz_empty_blocks():
    q = np.ones((2, 3))
    empty = np.zeros((2, 0, 3))
    out = ruiz_equilibrate(q, q, empty, np.zeros((2, 0)), empty, np.zeros((2, 0)), q, q)
    assert out[2].shape == (2, 0, 3) and out[9].shape == (2, 0)
    got = torch_ruiz(*(torch.as_tensor(x) for x in (q, q, empty, np.zeros((2, 0)), empty,
                                                     np.zeros((2, 0)), q, q)))
    np.testing.assert_allclose(got[8].numpy(), out[8])
