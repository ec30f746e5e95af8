"""The diagonal-QP oracle against the reference's analytic cases, and its pullback
against torch autograd (CPU).

The analytic case is the reference's own (tests/test_diagonal_qp.py:13-47 in
PURIN): minimise y0^2 + 2 y1^2 - 2 y0 - 4 y1 subject to y0 + y1 = 1, whose
solution is (1/3, 2/3) with dy/dc = -Q^-1 + Q^-1 a (a' Q^-1 a)^-1 a' Q^-1.
"""

import numpy as np
import pytest
import torch

from helpers import coupled_diagonal_qp_case, kkt_certified_qp, oracle_config
from oracle.cp import _balanced  # noqa: F401  (tie rule exercised by the pullback)
from oracle.diagonal_qp import OracleDiagonalQP, qp_step_pullback
from oracle.sparse import layout
from purin_b200 import ChambollePockConfig
from purin_b200.diagonal_qp import QPStructure

JACOBIAN = -np.diag([0.5, 0.25]) + np.outer([0.5, 0.25], [0.5, 0.25]) / 0.75


def analytic_case():
    q = np.array([[2.0, 4.0]])
    c = np.array([[-2.0, -4.0]])
    values = np.ones((1, 1, 2))
    rhs = np.array([[1.0]])
    lower = np.full((1, 2), -np.inf)
    upper = np.full((1, 2), np.inf)
    return (q, c, values, rhs, lower, upper)


def analytic_oracle(accelerated, scaling):
    cfg = ChambollePockConfig(accelerated=accelerated, row_scaling=scaling, tolerance=1e-9,
                              max_iterations=3000)
    return OracleDiagonalQP(2, ((0, 1),), (), oracle_config(cfg))


@pytest.mark.parametrize("accelerated", [False, True])
@pytest.mark.parametrize("scaling", [False, True])
def test_oracle_value_jacobian_and_warm_start(accelerated, scaling):
    qp = analytic_oracle(accelerated, scaling)
    data = analytic_case()
    result, saved = qp.solve(data)
    np.testing.assert_allclose(result["y"], [[1 / 3, 2 / 3]], atol=1e-8)
    assert result["residual_inf_norm"][0] < 1e-8
    assert result["status"][0] == 0
    rows = []
    for i in range(2):
        cot = np.zeros((1, 2))
        cot[0, i] = 1.0
        grads = qp.vjp(saved["out"], saved["data"], cot)
        rows.append(grads["c"][0])
    np.testing.assert_allclose(np.array(rows), JACOBIAN, atol=1e-7)
    warm, _ = qp.solve(data, initial_y=result["y"], initial_dual=result["multipliers_eq"])
    np.testing.assert_allclose(warm["y"], result["y"], atol=1e-8)


def test_oracle_q_gradient_matches_finite_differences():
    """d y / d q of the analytic case against central differences of the oracle solve."""
    qp = analytic_oracle(False, True)
    data = analytic_case()
    result, saved = qp.solve(data)
    g = np.array([[0.3, -1.1]])
    grads = qp.vjp(saved["out"], saved["data"], g)
    eps = 1e-6
    fd = np.zeros(2)
    for j in range(2):
        plus = [a.copy() for a in data]
        minus = [a.copy() for a in data]
        plus[0][0, j] += eps
        minus[0][0, j] -= eps
        yp, _ = qp.solve(tuple(plus))
        ym, _ = qp.solve(tuple(minus))
        fd[j] = float(((yp["y"] - ym["y"]) * g).sum()) / (2 * eps)
    np.testing.assert_allclose(grads["q"][0], fd, atol=1e-6)


def _torch_qp_step(support, mask, me, tau, sigma, B, n):
    sup = torch.as_tensor(support, dtype=torch.long)
    msk = torch.as_tensor(mask)

    def step(y, dual, ybar, q, c, vals, rhs, lo, up):
        mv = lambda x: torch.where(msk[None], vals * x[:, sup], 0.0).sum(-1)

        def tmv(d):
            contrib = torch.where(msk[None], vals * d[:, :, None], 0.0).reshape(B, -1)
            return torch.zeros(B, n, dtype=torch.float64).index_add(1, sup.reshape(-1), contrib)

        t = torch.as_tensor(tau)[:, None]
        s = torch.as_tensor(sigma)[:, None]
        nd = dual + s * (mv(ybar) - rhs)
        nd = torch.cat([nd[:, :me], torch.clamp_min(nd[:, me:], 0)], 1)
        inverse = 1 / (1 + t * q)
        dw = t * inverse
        ny = inverse * y - dw * tmv(nd) + (-dw) * c
        ny = torch.minimum(up, torch.maximum(lo, ny))
        return ny, nd, ny + (ny - y)

    return step


@pytest.mark.parametrize("seed", [3, 4])
def test_qp_pullback_matches_autograd(seed):
    """At a point without ties the QP step's VJP equals torch autograd (q up to rounding)."""
    rng = np.random.default_rng(seed)
    B, n, me, mi = 3, 10, 2, 4
    rows = [tuple(sorted(rng.choice(n, 3, replace=False))) for _ in range(me + mi)]
    support, mask, _ = layout(rows, n)
    vals = np.where(mask[None], rng.normal(size=(B,) + support.shape), 0.0)
    q = rng.uniform(0.5, 2.0, size=(B, n))
    c = rng.normal(size=(B, n))
    rhs = rng.normal(size=(B, me + mi))
    lo = np.full((B, n), -0.8)
    up = np.full((B, n), 0.9)
    y = rng.uniform(-0.5, 0.5, size=(B, n))
    dual = rng.normal(size=(B, me + mi))
    tau = rng.uniform(0.1, 0.4, size=B)
    sigma = rng.uniform(0.1, 0.4, size=B)
    cot = tuple(rng.normal(size=s) for s in ((B, n), (B, me + mi), (B, n)))
    step = _torch_qp_step(support, mask, me, tau, sigma, B, n)
    inputs = [torch.tensor(a, requires_grad=True)
              for a in (y, dual, y.copy(), q, c, vals, rhs, lo, up)]
    outs = step(*inputs)
    torch.autograd.backward(outs, [torch.tensor(v) for v in cot])
    (sy, sd, sb), grads = qp_step_pullback((y, dual, y.copy()), q, c, vals, rhs, lo, up, support,
                                           mask, me, tau, sigma, cot)
    ref = [t.grad.numpy() for t in inputs]
    np.testing.assert_allclose(sy, ref[0], rtol=1e-13, atol=1e-15)
    np.testing.assert_allclose(sd, ref[1], rtol=1e-13, atol=1e-15)
    np.testing.assert_allclose(sb, ref[2], rtol=1e-13, atol=1e-15)
    for k, r in zip(("q", "c", "values", "rhs", "lower", "upper"), ref[3:]):
        np.testing.assert_allclose(grads[k], r, rtol=1e-12, atol=1e-14, err_msg=k)


def test_invalid_qp_structures():
    """tests/test_diagonal_qp.py:108-127 of the reference (the checks that need no device)."""
    for args in [(0,), (2, ((0, 0),)), (2, ((2,),)), (2, ((-1,),))]:
        with pytest.raises(ValueError):
            QPStructure(*args)
    structure = QPStructure(2)
    with pytest.raises(ValueError):
        structure.prepare(batch_size=0)
    with pytest.raises(ValueError):
        structure.prepare(batch_size=1, config=ChambollePockConfig(metric_diagonal=(1.0, 1.0)))
    from purin_b200.diagonal_qp import dense_qp_data

    with pytest.raises(ValueError):
        dense_qp_data(np.ones(2), np.ones(2), np.empty((0, 2)), [], np.empty((0, 2)), [], -1, 1)


@pytest.mark.parametrize("diagonal", [False, True])
def test_coupled_inequalities_match_a_certified_kkt_solution(diagonal):
    """tests/test_regression_cp_diagonal_steps.py:28-80: the general diagonal QP with
    coupled inequalities converges (tolerance 1e-9) to the exact solution, within the
    reference's 3e-8, with or without diagonal preconditioning (OSQP, which the reference
    compares against, is not installed: an exact KKT solve on the identified active set,
    checked for feasibility and multiplier signs, stands in for it)."""
    eq_rows, in_rows, data, matrix = coupled_diagonal_qp_case()
    cfg = ChambollePockConfig(tolerance=1e-9, max_iterations=20000, row_scaling=False,
                              diagonal_preconditioning=diagonal)
    result, _ = OracleDiagonalQP(6, eq_rows, in_rows, oracle_config(cfg)).solve(data)
    assert (result["status"] == 0).all()
    q, c, _, rhs, lower, upper = data
    for i in range(len(q)):
        exact = kkt_certified_qp(q[i], c[i], matrix, rhs[i], 2, lower[i], upper[i], result["y"][i])
        np.testing.assert_allclose(result["y"][i], exact, atol=3e-8)
