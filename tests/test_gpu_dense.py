"""Dense / packed CP adapter (``solve_dense_implicit``) on the GPU.

* The reference's analytic cases (PURIN tests/test_dense_cp.py:20-78): value,
  warm start and the implicit Jacobian dy/dc at 1e-6, with and without Ruiz
  equilibration and acceleration; no constraint rows.
* Random dense and packed problems against the oracle (oracle/dense.py):
  forward at a fixed iteration count and converged with the batch-wide trip
  count, and the implicit gradients of every input.
"""

import numpy as np
import pytest
import torch

from oracle.dense import OracleDense
from purin_b200.dense_layer import solve_dense_implicit

pytestmark = pytest.mark.gpu

DEV = "cuda"
JACOBIAN = -np.diag([0.5, 0.25]) + np.outer([0.5, 0.25], [0.5, 0.25]) / 0.75


def _equality_qp(dtype=torch.float64):
    t = lambda x: torch.tensor(x, dtype=dtype, device=DEV)
    return (t([[2.0, 4.0]]), t([[-2.0, -4.0]]), torch.ones((1, 1, 2), dtype=dtype, device=DEV),
            torch.ones((1, 1), dtype=dtype, device=DEV), t([[[-1.0, 0.0]]]),
            torch.zeros((1, 1), dtype=dtype, device=DEV),
            torch.zeros((1, 2), dtype=dtype, device=DEV),
            torch.ones((1, 2), dtype=dtype, device=DEV) * 2)


@pytest.mark.parametrize("accelerated", [False, True])
@pytest.mark.parametrize("equilibrate", [False, True])
def test_dense_analytic_equality_qp(accelerated, equilibrate):
    q, c, A, b, C, d, lo, hi = args = _equality_qp()
    kwargs = dict(accelerated=accelerated, equilibrate=equilibrate, tolerance=1e-13,
                  max_iterations=20000)
    y, eq, iq = solve_dense_implicit(*args, **kwargs)
    np.testing.assert_allclose(y.cpu().numpy(), [[1 / 3, 2 / 3]], atol=1e-6)
    warm = solve_dense_implicit(*args, y0=y, lambda0=eq, mu0=iq, **kwargs)[0]
    np.testing.assert_allclose(warm.cpu().numpy(), y.cpu().numpy(), atol=1e-6)
    jac = torch.autograd.functional.jacobian(
        lambda linear: solve_dense_implicit(q, linear[None], A, b, C, d, lo, hi, **kwargs)[0][0],
        c[0])
    np.testing.assert_allclose(jac.cpu().numpy(), JACOBIAN, atol=1e-6)
    # Equality residual and primal feasibility of the reported solution.
    assert abs(float(y.sum()) - 1.0) < 1e-7
    assert float(eq.abs().max()) > 0.0


def test_dense_analytic_float32():
    y, _, _ = solve_dense_implicit(*_equality_qp(torch.float32), tolerance=1e-6,
                                   max_iterations=20000)
    assert y.dtype == torch.float32
    np.testing.assert_allclose(y.cpu().numpy(), [[1 / 3, 2 / 3]], atol=1e-4)


def test_dense_empty_constraints():
    q = torch.ones((1, 2), dtype=torch.float64, device=DEV)
    c = torch.tensor([[-1.0, -2.0]], dtype=torch.float64, device=DEV)
    empty = torch.zeros((1, 0, 2), dtype=torch.float64, device=DEV)
    none = torch.zeros((1, 0), dtype=torch.float64, device=DEV)
    y, eq, iq = solve_dense_implicit(q, c, empty, none, empty, none, torch.zeros_like(q),
                                     torch.ones_like(q) * 3, equilibrate=True, tolerance=1e-14)
    np.testing.assert_allclose(y.cpu().numpy(), [[1.0, 2.0]], atol=1e-6)
    assert eq.shape == (1, 0) and iq.shape == (1, 0)


def test_dense_invalid_support_raises():
    args = _equality_qp()
    with pytest.raises(ValueError):
        solve_dense_implicit(*args, inequality_support=((0,), (1,)))  # two rows for one
    with pytest.raises(ValueError):
        solve_dense_implicit(*args, inequality_support=((2,),))  # column out of range
    with pytest.raises(ValueError):
        solve_dense_implicit(*args, inequality_support=((0, 0),))  # duplicate column
    with pytest.raises(ValueError):
        solve_dense_implicit(args[0][0], *args[1:])  # q without a batch axis


def _random_dense(batch, n, me, mi, seed, *, support=None):
    rng = np.random.default_rng(seed)
    q = rng.uniform(0.5, 2.0, (batch, n))
    q[0] *= 4.0  # spread the samples' iteration counts
    c = rng.normal(size=(batch, n))
    A = rng.normal(size=(batch, me, n))
    C = rng.normal(size=(batch, mi, n))
    if support is not None:
        keep = np.zeros((mi, n), dtype=bool)
        for i, row in enumerate(support):
            keep[i, list(row)] = True
        C = np.where(keep[None], C, 0.0)
    y_feasible = rng.uniform(-0.5, 0.5, (batch, n))
    b = np.einsum("bmn,bn->bm", A, y_feasible)
    d = np.einsum("bmn,bn->bm", C, y_feasible) + rng.uniform(0.0, 0.5, (batch, mi))
    return q, c, A, b, C, d, -np.ones((batch, n)), np.ones((batch, n))


SUPPORT = ((0, 2, 5), (1, 3), (4, 6, 7, 0), (2,))


@pytest.mark.parametrize("accelerated", [False, True])
@pytest.mark.parametrize("packed", [False, True])
def test_dense_parity_fixed_iterations(accelerated, packed):
    """200 iterations (no sample accepted): every output against the oracle."""
    support = SUPPORT if packed else None
    problem = _random_dense(5, 8, 2, 4, seed=11, support=support)
    oracle = OracleDense(8, 2, 4, inequality_support=support, accelerated=accelerated,
                         tolerance=1e-300, max_iterations=200)
    ref = oracle.solve(*problem)
    got = solve_dense_implicit(*(torch.as_tensor(x, device=DEV) for x in problem),
                               accelerated=accelerated, tolerance=1e-300, max_iterations=200,
                               inequality_support=support, return_iterations=True)
    for g, r in zip(got[:3], ref[:3]):
        np.testing.assert_allclose(g.cpu().numpy(), r, rtol=1e-9, atol=1e-12)
    assert got[3].cpu().tolist() == [200] * 5


@pytest.mark.parametrize("accelerated", [False, True])
@pytest.mark.parametrize("equilibrate", [False, True])
def test_dense_parity_trip_count(accelerated, equilibrate):
    """Converged solve: every sample runs the batch's trip count, as in the shared loop."""
    problem = _random_dense(4, 6, 2, 3, seed=3)
    oracle = OracleDense(6, 2, 3, accelerated=accelerated, tolerance=1e-8, max_iterations=4000)
    ref = oracle.solve(*problem, equilibrate=equilibrate)
    got = solve_dense_implicit(*(torch.as_tensor(x, device=DEV) for x in problem),
                               accelerated=accelerated, tolerance=1e-8, max_iterations=4000,
                               equilibrate=equilibrate, return_iterations=True)
    trips = int(ref[3][0])
    assert trips < 4000 and set(ref[3].tolist()) == {trips}
    assert got[3].cpu().tolist() == ref[3].tolist()
    for g, r in zip(got[:3], ref[:3]):
        np.testing.assert_allclose(g.cpu().numpy(), r, rtol=1e-9, atol=1e-11)


def test_dense_shared_matrices_match_per_sample():
    """A 2-D constraint matrix (one copy for the batch) gives the 3-D result."""
    q, c, A, b, C, d, lo, hi = _random_dense(3, 6, 2, 3, seed=5)
    A = np.broadcast_to(A[:1], A.shape)
    C = np.broadcast_to(C[:1], C.shape)
    t = lambda x: torch.as_tensor(np.array(x), device=DEV)
    per = solve_dense_implicit(t(q), t(c), t(A), t(b), t(C), t(d), t(lo), t(hi), tolerance=1e-9,
                               max_iterations=4000)
    one = solve_dense_implicit(t(q), t(c), t(A[0]), t(b), t(C[0]), t(d), t(lo), t(hi),
                               tolerance=1e-9, max_iterations=4000)
    for g, r in zip(one, per):
        torch.testing.assert_close(g, r, rtol=1e-12, atol=1e-14)
    # Gradients of the shared matrix sum the per-sample ones.
    A1 = t(A[0]).requires_grad_()
    A3 = t(A).requires_grad_()
    solve_dense_implicit(t(q), t(c), A1, t(b), t(C[0]), t(d), t(lo), t(hi), tolerance=1e-9,
                         max_iterations=4000)[0].sum().backward()
    solve_dense_implicit(t(q), t(c), A3, t(b), t(C), t(d), t(lo), t(hi), tolerance=1e-9,
                         max_iterations=4000)[0].sum().backward()
    torch.testing.assert_close(A1.grad, A3.grad.sum(dim=0), rtol=1e-9, atol=1e-11)


@pytest.mark.parametrize("accelerated", [False, True])
def test_dense_gradients_match_oracle(accelerated):
    """Implicit cotangents of c, A, b, C, d and the bounds; q gets none (frozen proximal)."""
    problem = _random_dense(4, 6, 2, 3, seed=8)
    oracle = OracleDense(6, 2, 3, accelerated=accelerated, tolerance=1e-10, max_iterations=8000)
    inputs = [torch.as_tensor(x, device=DEV).requires_grad_() for x in problem]
    y, eq, iq = solve_dense_implicit(*inputs, accelerated=accelerated, tolerance=1e-10,
                                     max_iterations=8000)
    rng = np.random.default_rng(1)
    wy, weq, wiq = rng.normal(size=(4, 6)), rng.normal(size=(4, 2)), rng.normal(size=(4, 3))
    loss = ((y * torch.as_tensor(wy, device=DEV)).sum()
            + (eq * torch.as_tensor(weq, device=DEV)).sum()
            + (iq * torch.as_tensor(wiq, device=DEV)).sum())
    loss.backward()
    out = oracle.run(*problem)
    grads = oracle.vjp(out, *problem, wy, np.concatenate((weq, wiq), axis=1))
    gq, gc, gA, gb, gC, gd, glo, ghi = (x.grad.cpu().numpy() for x in inputs)
    expect = dict(q=(gq, grads["q"]), c=(gc, grads["c"]),
                  A=(gA, grads["values"][:, :2]), C=(gC, grads["values"][:, 2:]),
                  b=(gb, grads["rhs"][:, :2]), d=(gd, grads["rhs"][:, 2:]),
                  lower=(glo, grads["lower"]), upper=(ghi, grads["upper"]))
    for name, (g, r) in expect.items():
        np.testing.assert_allclose(g, r, rtol=1e-7, atol=1e-9, err_msg=name)
    assert np.all(gq == 0.0)


@pytest.mark.parametrize("case", ["equality_only_unbounded", "inequality_only_packed",
                                  "max_iterations_reached"])
def test_dense_edge_cases_match_oracle(case):
    """Zero-width blocks, infinite bounds, and a trip count capped by max_iterations."""
    support = None
    max_iterations, tolerance = 4000, 1e-9
    if case == "equality_only_unbounded":
        q, c, A, b, C, d, lo, hi = _random_dense(3, 6, 3, 0, seed=21)
        lo, hi = np.full_like(lo, -np.inf), np.full_like(hi, np.inf)
    elif case == "inequality_only_packed":
        support = SUPPORT
        q, c, A, b, C, d, lo, hi = _random_dense(3, 8, 0, 4, seed=22, support=support)
    else:
        q, c, A, b, C, d, lo, hi = _random_dense(4, 6, 2, 3, seed=23)
        max_iterations = 180  # first acceptances 141, 149, 220, 199: two samples accept
    problem = (q, c, A, b, C, d, lo, hi)
    oracle = OracleDense(q.shape[1], A.shape[1], C.shape[1], inequality_support=support,
                         tolerance=tolerance, max_iterations=max_iterations)
    ref = oracle.solve(*problem)
    got = solve_dense_implicit(*(torch.as_tensor(x, device=DEV) for x in problem),
                               tolerance=tolerance, max_iterations=max_iterations,
                               inequality_support=support, return_iterations=True)
    assert got[3].cpu().tolist() == ref[3].tolist()
    for g, r in zip(got[:3], ref[:3]):
        np.testing.assert_allclose(g.cpu().numpy(), r, rtol=1e-9, atol=1e-11)
    if case == "max_iterations_reached":
        assert ref[3].tolist() == [180] * 4


@pytest.mark.parametrize("accelerated", [False, True])
def test_qp_forward_resume_is_bitwise_uninterrupted(accelerated):
    """purin_qp_forward resumed from (y, dual, ybar, iterations) = one uninterrupted run.

    Pass 1 freezes each sample at its first acceptance; pass 2 resumes every
    sample from there without freezing.  The result must equal, bit for bit,
    a single run without freezing for the same trip count.
    """
    from purin_b200 import _native
    from purin_b200.config import ChambollePockConfig, LinearSolverConfig
    from purin_b200.dense_layer import _FIRST_PASS, _DenseSolver
    from purin_b200.layer import resolve_device

    q, c, A, b, C, d, lo, hi = (torch.as_tensor(x, device=DEV)
                                for x in _random_dense(4, 6, 2, 3, seed=3))
    n, me, mi = 6, 2, 3
    cfg = ChambollePockConfig(accelerated=accelerated, tolerance=1e-8, max_iterations=4000,
                              norm_bound=False, row_scaling=False,
                              linear_solver=LinearSolverConfig())
    solver = _DenseSolver(n, me, tuple(tuple(range(n)) for _ in range(mi)), torch.float64,
                          resolve_device(DEV), cfg)
    values = torch.cat((A.reshape(4, -1), C.reshape(4, -1)), dim=1).contiguous()
    rhs = torch.cat((b, d), dim=1).contiguous()
    zeros = lambda k: torch.zeros((4, k), dtype=torch.float64, device=DEV)
    tol = torch.full((4,), 1e-8, dtype=torch.float64, device=DEV)
    inputs = (q, c, values, rhs, lo, hi, zeros(n), zeros(me + mi), tol)
    first = solver.forward(inputs, 4000, _FIRST_PASS)
    trips = int(first["iterations"].max())
    assert len(set(first["iterations"].tolist())) > 1 and trips < 4000
    resumed_inputs = (q, c, values, rhs, lo, hi, first["y"], first["dual"], tol)
    resumed = solver.forward(resumed_inputs, trips, _FIRST_PASS | _native.QP_NO_FREEZE,
                             ybar0=first["ybar"], start=first["iterations"])
    whole = solver.forward(inputs, trips, _FIRST_PASS | _native.QP_NO_FREEZE)
    for key in ("y", "ybar", "dual"):
        assert torch.equal(resumed[key], whole[key]), key
    assert resumed["iterations"].tolist() == [trips] * 4 == whole["iterations"].tolist()


@pytest.mark.parametrize("accelerated", [False, True])
@pytest.mark.parametrize("support", [None, ((0,),)])
@pytest.mark.parametrize("equilibrate", [False, True])
def test_iteration_counts_preserve_solution(accelerated, support, equilibrate):
    """PURIN tests/test_cp_iteration_counts.py:10-43: asking for the counts changes no
    output; the batch advances every row until the shared loop exits (8, 8), and the
    first sample alone is accepted after one iteration."""
    t = lambda x: torch.as_tensor(np.asarray(x, dtype=np.float64), device=DEV)
    arguments = (t(np.ones((2, 1))), t([[0.0], [-2.0]]), t(np.empty((0, 1))), t(np.empty((0,))),
                 t(np.ones((1, 1))), t(np.ones((1,))), t([-np.inf]), t([np.inf]))
    options = dict(accelerated=accelerated, inequality_support=support,
                   equilibrate=equilibrate, max_iterations=8, tolerance=1e-12)
    expected = solve_dense_implicit(*arguments, **options)
    *actual, iterations = solve_dense_implicit(*arguments, **options, return_iterations=True)
    for result, reference in zip(actual, expected):
        np.testing.assert_allclose(result.cpu().numpy(), reference.cpu().numpy(), atol=1e-12,
                                   rtol=1e-12)
    assert iterations.cpu().tolist() == [8, 8]
    singleton = tuple(value[:1] if i < 2 else value for i, value in enumerate(arguments))
    *_, early = solve_dense_implicit(*singleton, **options, return_iterations=True)
    assert early.cpu().tolist() == [1]


@pytest.mark.parametrize("accelerated", [False, True])
@pytest.mark.parametrize("equilibrate", [False, True])
@pytest.mark.parametrize("concentrated", [False, True])
def test_sparse_forward_and_structural_gradients(accelerated, equilibrate, concentrated):
    """PURIN tests/test_sparse_cp_layer.py:11-71: the packed support (an empty row
    included; or every row on the same two columns) gives the dense layout's outputs
    and gradients of every input to the adjoint's accuracy."""
    rng = np.random.default_rng(7)
    n, me, mi, batch = 8, 2, 3, 2
    rows = ((0, 2), (), (1, 4, 7))
    if concentrated:
        n = 32
        rows = ((0, 1),) * mi
    mask = np.zeros((mi, n))
    for i, row in enumerate(rows):
        mask[i, list(row)] = 1
    t = lambda x: torch.as_tensor(np.asarray(x, dtype=np.float64), device=DEV)
    q = t(rng.uniform(1, 2, (batch, n)))
    c = t(rng.normal(size=(batch, n)))
    a = t(rng.normal(size=(batch, me, n)))
    b = t(np.zeros((batch, me)))
    matrix = t(rng.normal(size=(batch, mi, n)))
    d = t(np.tile([0.05, 1, 0.05], (batch, 1)))
    lower, upper = -torch.ones_like(q), torch.ones_like(q)
    masked = matrix * t(mask)
    outputs, grads = [], []
    for sparse in (False, True):
        params = [x.clone().requires_grad_(True) for x in (q, c, a, b, masked, d, lower, upper)]
        out = solve_dense_implicit(*params, accelerated=accelerated, equilibrate=equilibrate,
                                   max_iterations=500, norm_iterations=25,
                                   inequality_support=rows if sparse else None)
        outputs.append([o.detach().cpu().numpy() for o in out])
        weights = [torch.as_tensor(np.random.default_rng(11 + k).normal(size=tuple(o.shape)),
                                   device=DEV) for k, o in enumerate(out)]
        sum((w * o).sum() for w, o in zip(weights, out)).backward()
        grads.append([np.zeros(tuple(p.shape)) if p.grad is None else p.grad.cpu().numpy()
                      for p in params])
    for x, y in zip(*outputs):
        np.testing.assert_allclose(x, y, atol=2e-7, rtol=2e-6)
    for k, (x, y) in enumerate(zip(*grads)):
        if k == 4:  # the matrix: only its structural entries are shared by both layouts
            x, y = x * mask, y * mask
        np.testing.assert_allclose(x, y, atol=5e-6, rtol=2e-5)
        assert np.linalg.norm(x - y) <= 1e-5 * max(1.0, np.linalg.norm(x))


@pytest.mark.parametrize("rows", [((0,),), ((0,), (8,)), ((0,), (1, 1)), ((0,), (0.5,)),
                                  ((0,), (True,))])
def test_invalid_support_rejected(rows):
    """PURIN tests/test_sparse_cp_layer.py:74-81 (and booleans, which the reference's
    validation also excludes)."""
    q = torch.ones((1, 8), dtype=torch.float64, device=DEV)
    empty = torch.zeros((1, 0, 8), dtype=torch.float64, device=DEV)
    C = torch.ones((1, 2, 8), dtype=torch.float64, device=DEV)
    with pytest.raises(ValueError):
        solve_dense_implicit(q, q, empty, torch.zeros((1, 0), device=DEV, dtype=torch.float64),
                             C, torch.ones((1, 2), dtype=torch.float64, device=DEV), -q, q,
                             inequality_support=rows)


def test_zero_constraint_blocks_with_packed_support():
    """PURIN tests/test_sparse_cp_layer.py:84-122: no rows, packed support () against the
    dense call."""
    t = lambda x: torch.as_tensor(np.asarray(x, dtype=np.float64), device=DEV)
    q, c = t([[1.0, 2.0, 3.0]]), t([[0.2, -0.6, 0.9]])
    empty, rhs = t(np.zeros((1, 0, 3))), t(np.zeros((1, 0)))
    y, eq, iq = solve_dense_implicit(q, c, empty, rhs, empty, rhs, -torch.ones_like(q),
                                     torch.ones_like(q), inequality_support=(),
                                     max_iterations=500)
    dense = solve_dense_implicit(q, c, empty, rhs, empty, rhs, -torch.ones_like(q),
                                 torch.ones_like(q), max_iterations=500)
    np.testing.assert_allclose(y.cpu().numpy(), dense[0].cpu().numpy(), atol=1e-12)
    assert tuple(eq.shape) == tuple(iq.shape) == (1, 0)
