"""Seeded synthetic problems of the five benchmark configurations.

No public dataset is involved: every configuration is generated from NumPy's
``default_rng`` (seed 0 by default).  The structure shared by the batch
(constraint rows, bounds, metric weights) comes from ``default_rng(seed)`` in a
fixed order.  Per-sample data (x0, slack, candidates, loss targets) comes in
blocks of ``SAMPLE_BLOCK`` samples: block k is drawn from
``default_rng([seed, 1, k])``, so sample i's data depends on its global index
only -- not on the batch size or on how a batch is split across ranks -- and a
rank generates exactly its slice ``[offset, offset + batch)`` of a global batch.
Problems are ParametricQPs whose variable bounds are singleton inequality rows
(x_i <= u_i, -x_i <= -l_i) that the CP layer's bound presolve turns into box
bounds.  Per-sample right-hand sides enter through identity parameter maps, so
parameters are ``theta = [b; h]``.

    0  fp64, B=256,   n=64,    me=32,   mi=32,   4 nnz/row,  l=-1, u=1, fixed-step 500 it
    1  fp64/fp32, B=4096, n=1024, me=256, mi=512, 8 nnz/row, l~U(-2,-.5), u~U(.5,2), accel 1000 it
    2  fp64, B=2048,  n=2048,  me=512,  mi=1024, 8 nnz/row, loss 0.5||y-t||^2, 2000 it (+VJP)
    3  fp32, B=16384, network flow: 5000 nodes, 20000 edges, 4000 coupling rows, 1500 it
    4  fp32/fp64, B in {1,64,1024,16384,65536}, n=4096, me=1024, mi=2048, 16 nnz/row,
       WeightedDistance w~U(.5,2), accel 1000 it
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np
import scipy.sparse as sp

from purin_b200.config import ChambollePockConfig, ImplicitGradientConfig
from purin_b200.problems import ParametricQP


@dataclass
class Workload:
    name: str
    problem: ParametricQP
    theta: np.ndarray
    candidates: np.ndarray
    config: ChambollePockConfig
    dtype: str
    targets: np.ndarray | None = None
    weights: np.ndarray | None = None
    info: dict = field(default_factory=dict)


def _random_rows(rng, rows, n, k):
    indptr = np.arange(rows + 1, dtype=np.int64) * k
    indices = np.concatenate([rng.choice(n, k, replace=False) for _ in range(rows)]) if rows else (
        np.zeros(0, np.int64))
    data = rng.normal(size=rows * k)
    return sp.csr_matrix((data, indices, indptr), shape=(rows, n))


def _box_qp(A_eq, A_in, lower, upper, name):
    """ParametricQP with equality rows A_eq y = b, A_in y <= h and box bounds as singleton rows."""
    me, n = A_eq.shape
    mi = A_in.shape[0]
    eye = sp.identity(n, format="csr")
    A_ineq = sp.vstack([A_in, eye, -eye], format="csr")
    p = me + mi
    b_eq_map = sp.hstack([sp.identity(me), sp.csr_matrix((me, mi))], format="csr")
    b_in_map = sp.vstack([sp.hstack([sp.csr_matrix((mi, me)), sp.identity(mi)]),
                          sp.csr_matrix((2 * n, p))], format="csr")
    b_ineq0 = np.concatenate([np.zeros(mi), upper, -lower])
    return ParametricQP(P=sp.identity(n, format="csr"), q0=np.zeros(n), A_eq=A_eq,
                        b_eq0=np.zeros(me), b_eq_parameter_map=b_eq_map, A_ineq=A_ineq,
                        b_ineq0=b_ineq0, b_ineq_parameter_map=b_in_map, name=name)


SAMPLE_BLOCK = 64


def sample_blocks(seed, offset, batch, draw, dtype=np.float64):
    """Per-sample arrays of samples ``[offset, offset + batch)``.

    ``draw(rng, rows)`` returns a tuple of arrays with ``rows`` leading rows
    drawn from ``rng``; block k (samples ``k * SAMPLE_BLOCK`` onwards) calls it
    with ``default_rng([seed, 1, k])`` and ``rows = SAMPLE_BLOCK``.  The result
    is each array's rows of the requested samples, cast to ``dtype``.
    """
    if batch <= 0:
        parts = draw(np.random.default_rng([seed, 1, 0]), 0)
        return tuple(np.asarray(a, dtype) for a in parts)
    first, last = offset // SAMPLE_BLOCK, (offset + batch - 1) // SAMPLE_BLOCK
    out = None
    at = 0
    for k in range(first, last + 1):
        parts = draw(np.random.default_rng([seed, 1, k]), SAMPLE_BLOCK)
        lo = max(offset - k * SAMPLE_BLOCK, 0)
        hi = min(offset + batch - k * SAMPLE_BLOCK, SAMPLE_BLOCK)
        if out is None:
            out = tuple(np.empty((batch,) + np.shape(a)[1:], dtype) for a in parts)
        for dst, src in zip(out, parts):
            dst[at:at + hi - lo] = src[lo:hi]
        at += hi - lo
    return out


def random_box_config(*, batch, n, me, mi, nnz, bounds, seed=0, name="cp", offset=0,
                      array_dtype=np.float64):
    """Configs 0-2 and 4: random rows, seeded feasible x0, candidates 2 N(0,1).

    Returns (problem, theta, candidates, targets, rng): the per-sample arrays of
    samples ``[offset, offset + batch)`` (targets t ~ N(0,1)^n for the loss) and
    the structure generator, positioned after the bounds.
    """
    rng = np.random.default_rng(seed)
    A_eq = _random_rows(rng, me, n, nnz)
    A_in = _random_rows(rng, mi, n, nnz)
    if bounds == "unit":
        lower, upper = -np.ones(n), np.ones(n)
    else:
        lower = rng.uniform(-2.0, -0.5, n)
        upper = rng.uniform(0.5, 2.0, n)

    def draw(r, rows):
        x0 = r.uniform(-0.5, 0.5, (rows, n))
        slack = r.uniform(0.0, 0.1, (rows, mi))
        candidates = 2.0 * r.normal(size=(rows, n))
        targets = r.normal(size=(rows, n))
        b = (A_eq @ x0.T).T
        h = (A_in @ x0.T).T + slack
        return np.concatenate([b, h], axis=1), candidates, targets

    theta, candidates, targets = sample_blocks(seed, offset, batch, draw, array_dtype)
    problem = _box_qp(A_eq, A_in, lower, upper, name)
    return problem, theta, candidates, targets, rng


def network_flow_config(*, batch, nodes=5000, edges=20000, couplings=4000, seed=0, offset=0,
                        array_dtype=np.float64):
    """Config 3: node-incidence conservation, 2-edge coupling rows, |x| <= cap.

    Returns (problem, theta, candidates, targets) for samples ``[offset, offset + batch)``.
    """
    rng = np.random.default_rng(seed)
    order = rng.permutation(nodes)
    pairs = set()
    heads, tails = [], []
    for k in range(1, nodes):
        a, b = int(order[k]), int(order[rng.integers(0, k)])
        pairs.add((min(a, b), max(a, b)))
        heads.append(a)
        tails.append(b)
    while len(heads) < edges:
        a, b = (int(v) for v in rng.integers(0, nodes, 2))
        if a == b or (min(a, b), max(a, b)) in pairs:
            continue
        pairs.add((min(a, b), max(a, b)))
        heads.append(a)
        tails.append(b)
    heads = np.asarray(heads)
    tails = np.asarray(tails)
    flip = rng.random(edges) < 0.5
    heads, tails = np.where(flip, tails, heads), np.where(flip, heads, tails)
    cols = np.arange(edges)
    incidence = sp.csr_matrix(
        (np.concatenate([np.ones(edges), -np.ones(edges)]),
         (np.concatenate([heads, tails]), np.concatenate([cols, cols]))), shape=(nodes, edges))
    incidence.sort_indices()
    ccol = np.concatenate([rng.choice(edges, 2, replace=False) for _ in range(couplings)])
    cval = rng.choice([-1.0, 1.0], size=2 * couplings)
    coupling = sp.csr_matrix((cval, ccol, np.arange(couplings + 1) * 2), shape=(couplings, edges))
    cap = rng.uniform(1.0, 3.0, edges)

    def draw(r, rows):
        demand = r.normal(size=(rows, nodes))
        demand -= demand.mean(axis=1, keepdims=True)
        h = r.uniform(0.5, 1.5, (rows, couplings))
        candidates = 3.0 * r.normal(size=(rows, edges))
        targets = r.normal(size=(rows, edges))
        return np.concatenate([demand, h], axis=1), candidates, targets

    theta, candidates, targets = sample_blocks(seed, offset, batch, draw, array_dtype)
    problem = _box_qp(incidence, coupling, -cap, cap, "network_flow")
    return problem, theta, candidates, targets


def make_workload(index: int, batch: int | None = None, *, dtype: str | None = None,
                  seed: int = 0, mode: str = "fixed", offset: int = 0,
                  array_dtype=np.float64) -> Workload:
    """Workload of benchmark configuration ``index`` (0-4), samples ``[offset, offset + batch)``.

    ``mode="fixed"`` keeps the reference's stopping test and per-sample freeze
    with the configuration's iteration budget; ``mode="converged"`` (config 1)
    uses tolerance 1e-6.  ``array_dtype`` is the NumPy dtype of the per-sample
    arrays (float32 halves host memory for the large fp32 batches).
    """
    box = dict(seed=seed, offset=offset, array_dtype=array_dtype)
    if index == 0:
        batch = 256 if batch is None else batch
        problem, theta, cand, targets, _ = random_box_config(
            batch=batch, n=64, me=32, mi=32, nnz=4, bounds="unit", name="config0", **box)
        cfg = ChambollePockConfig(accelerated=False, max_iterations=500)
        return Workload("config0", problem, theta, cand, cfg, dtype or "float64", targets=targets)
    if index == 1:
        batch = 4096 if batch is None else batch
        problem, theta, cand, targets, _ = random_box_config(
            batch=batch, n=1024, me=256, mi=512, nnz=8, bounds="random", name="config1", **box)
        cfg = ChambollePockConfig(accelerated=True, max_iterations=1000,
                                  tolerance=1e-6 if mode == "converged" else 1e-9)
        return Workload("config1", problem, theta, cand, cfg, dtype or "float64", targets=targets)
    if index == 2:
        batch = 2048 if batch is None else batch
        problem, theta, cand, targets, _ = random_box_config(
            batch=batch, n=2048, me=512, mi=1024, nnz=8, bounds="random", name="config2", **box)
        cfg = ChambollePockConfig(
            max_iterations=2000,
            implicit_gradient=ImplicitGradientConfig(differentiate_problem_parameters=True))
        return Workload("config2", problem, theta, cand, cfg, dtype or "float64", targets=targets)
    if index == 3:
        batch = 16384 if batch is None else batch
        problem, theta, cand, targets = network_flow_config(batch=batch, **box)
        cfg = ChambollePockConfig(max_iterations=1500)
        return Workload("config3", problem, theta, cand, cfg, dtype or "float32", targets=targets)
    if index == 4:
        batch = 1024 if batch is None else batch
        problem, theta, cand, targets, rng = random_box_config(
            batch=batch, n=4096, me=1024, mi=2048, nnz=16, bounds="random", name="config4", **box)
        weights = rng.uniform(0.5, 2.0, 4096)
        cfg = ChambollePockConfig(accelerated=True, max_iterations=1000)
        return Workload("config4", problem, theta, cand, cfg, dtype or "float32", targets=targets,
                        weights=weights)
    raise ValueError("configuration index must be 0..4")


def qp_workload(batch: int, *, seed: int = 0, offset: int = 0):
    """Configuration 2's structure as a general diagonal QP (PreparedDiagonalQP).

    The same seeded rows (512 equality, 1024 inequality, 8 nnz per row over
    n = 2048 variables, values N(0,1), shared by the batch), per-variable
    bounds l ~ U(-2,-0.5), u ~ U(0.5,2) and per-sample right-hand sides from a
    seeded x0 as in configuration 2; per sample q ~ U(0.5, 2)^n and
    c = -q * candidate (a q-weighted projection of the candidate 2 N(0,1)), and
    a loss target t ~ N(0,1)^n, for samples ``[offset, offset + batch)`` (drawn
    in blocks, as ``make_workload``).  Returns (structure, q, c, values
    (1, m, 8), rhs, lower (n,), upper (n,), targets) as NumPy arrays.
    """
    from purin_b200.diagonal_qp import QPStructure

    n, me, mi, k = 2048, 512, 1024, 8
    rng = np.random.default_rng(seed)
    A_eq = _random_rows(rng, me, n, k)
    A_in = _random_rows(rng, mi, n, k)
    lower = rng.uniform(-2.0, -0.5, n)
    upper = rng.uniform(0.5, 2.0, n)

    def draw(r, rows):
        x0 = r.uniform(-0.5, 0.5, (rows, n))
        slack = r.uniform(0.0, 0.1, (rows, mi))
        candidates = 2.0 * r.normal(size=(rows, n))
        rhs = np.concatenate([(A_eq @ x0.T).T, (A_in @ x0.T).T + slack], axis=1)
        q = r.uniform(0.5, 2.0, (rows, n))
        targets = r.normal(size=(rows, n))
        return q, -q * candidates, rhs, targets

    q, c, rhs, targets = sample_blocks(seed, offset, batch, draw)
    rows = [tuple(int(j) for j in A.indices[A.indptr[i]:A.indptr[i + 1]])
            for A in (A_eq, A_in) for i in range(A.shape[0])]
    structure = QPStructure(n, tuple(rows[:me]), tuple(rows[me:]))
    values = np.concatenate([A_eq.data, A_in.data]).reshape(1, me + mi, k)
    return structure, q, c, values, rhs, lower, upper, targets


def dense_workload(batch: int, *, seed: int = 0, n: int = 64, me: int = 8, mi: int = 32,
                   offset: int = 0):
    """Batched dense diagonal QPs for ``solve_dense_implicit`` (per-sample matrices).

    Per sample: A ~ N(0,1)^(me x n), C ~ N(0,1)^(mi x n), q ~ U(0.5, 2)^n,
    c = -q * candidate (candidate 2 N(0,1)), b = A x0 and d = C x0 + slack for a
    seeded x0 ~ U(-0.5, 0.5)^n and slack ~ U(0, 0.1), bounds l ~ U(-2, -0.5),
    u ~ U(0.5, 2), and a loss target t ~ N(0,1)^n, for samples
    ``[offset, offset + batch)`` (drawn in blocks, as ``make_workload``).
    Returns (q, c, A, b, C, d, lower, upper, targets) as NumPy float64 arrays.
    """
    def draw(r, rows):
        A = r.normal(size=(rows, me, n))
        C = r.normal(size=(rows, mi, n))
        x0 = r.uniform(-0.5, 0.5, (rows, n))
        b = np.einsum("bmn,bn->bm", A, x0)
        d = np.einsum("bmn,bn->bm", C, x0) + r.uniform(0.0, 0.1, (rows, mi))
        q = r.uniform(0.5, 2.0, (rows, n))
        c = -q * (2.0 * r.normal(size=(rows, n)))
        lower = r.uniform(-2.0, -0.5, (rows, n))
        upper = r.uniform(0.5, 2.0, (rows, n))
        targets = r.normal(size=(rows, n))
        return q, c, A, b, C, d, lower, upper, targets

    return sample_blocks(seed, offset, batch, draw)
