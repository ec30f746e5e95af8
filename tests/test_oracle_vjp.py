"""The oracle's hand-derived CP-step pullback against torch autograd, and JAX's tie rule."""

import numpy as np
import pytest
import torch

from oracle.cp import _balanced, cp_step_pullback
from oracle.sparse import layout


def _torch_step(support, mask, me, tau, sigma, B, n):
    sup = torch.as_tensor(support, dtype=torch.long)
    msk = torch.as_tensor(mask)

    def step(y, dual, ybar, vals, rhs, target, lo, up):
        mv = lambda x: torch.where(msk[None], vals * x[:, sup], 0.0).sum(-1)

        def tmv(d):
            c = torch.where(msk[None], vals * d[:, :, None], 0.0).reshape(B, -1)
            return torch.zeros(B, n, dtype=torch.float64).index_add(1, sup.reshape(-1), c)

        t = torch.as_tensor(tau)[:, None]
        s = torch.as_tensor(sigma)[:, None]
        nd = dual + s * (mv(ybar) - rhs)
        nd = torch.cat([nd[:, :me], torch.clamp_min(nd[:, me:], 0)], 1)
        a = 1 / (1 + t)
        d = t * a
        ny = a * y - d * tmv(nd) + (-d) * (-target)
        ny = torch.minimum(up, torch.maximum(lo, ny))
        return ny, nd, ny + (ny - y)

    return step


@pytest.mark.parametrize("seed", [3, 4, 5])
def test_pullback_matches_autograd(seed):
    """At a point without ties the VJP of bounds.py:109-129 equals torch autograd bit for bit."""
    rng = np.random.default_rng(seed)
    B, n, me, mi = 3, 12, 3, 5
    rows = [tuple(sorted(rng.choice(n, 4, replace=False))) for _ in range(me + mi)]
    support, mask, _ = layout(rows, n)
    vals = np.where(mask, rng.normal(size=(B,) + support.shape), 0.0)
    rhs = rng.normal(size=(B, me + mi))
    target = rng.normal(size=(B, n))
    lo = -np.abs(rng.normal(size=(B, n)))
    up = np.abs(rng.normal(size=(B, n)))
    y, dual, ybar = rng.normal(size=(B, n)), rng.normal(size=(B, me + mi)), rng.normal(size=(B, n))
    tau, sigma = np.array([0.3, 0.2, 0.4]), np.array([0.5, 0.6, 0.7])
    step = _torch_step(support, mask, me, tau, sigma, B, n)
    ts = [torch.tensor(v, dtype=torch.float64, requires_grad=True)
          for v in (y, dual, ybar, vals, rhs, target, lo, up)]
    out = step(*ts)
    cot = [rng.normal(size=o.shape) for o in out]
    grads = torch.autograd.grad(out, ts, [torch.as_tensor(c) for c in cot])
    (sy, sd, sb), gv, gb, gt, gl, gu = cp_step_pullback(
        (y, dual, ybar), vals, rhs, target, lo, up, support, mask, me, tau, sigma, tuple(cot))
    for mine, ref in zip((sy, sd, sb, gv, gb, gt, gl, gu), grads):
        np.testing.assert_array_equal(mine, ref.numpy())


def test_balanced_tie_rule():
    """jax.lax.max/min JVP: a tied argument receives half the cotangent."""
    x = np.array([1.0, 2.0, 0.5, np.nan])
    other = np.array([1.0, 1.0, 1.0, 0.0])
    ans = np.maximum(x, other)
    np.testing.assert_array_equal(_balanced(x, ans, other), [0.5, 1.0, 0.0, 0.0])
    np.testing.assert_array_equal(_balanced(other, ans, x), [0.5, 0.0, 1.0, 0.0])


def test_pullback_at_an_active_bound_tie():
    """y_raw exactly on the lower bound: half the cotangent goes to the bound."""
    support, mask, _ = layout([], 1)
    y = np.array([[0.0]])
    target = np.array([[-1.0]])  # tau chosen so that the raw step lands exactly on 0
    tau = np.array([1.0])
    # y_raw = y/(1+tau) + tau/(1+tau) * target = -0.5 -> set lower = -0.5
    lo, up = np.array([[-0.5]]), np.array([[1.0]])
    out = cp_step_pullback((y, np.zeros((1, 0)), y), np.zeros((1, 0, 1)), np.zeros((1, 0)), target,
                           lo, up, support, mask, 0, tau, np.array([1.0]),
                           (np.ones((1, 1)), np.zeros((1, 0)), np.zeros((1, 1))))
    (_, _, _), _, _, g_target, g_lower, g_upper = out
    np.testing.assert_array_equal(g_lower, [[0.5]])
    np.testing.assert_array_equal(g_target, [[0.25]])  # d * g_raw = 0.5 * 0.5
    np.testing.assert_array_equal(g_upper, [[0.0]])
