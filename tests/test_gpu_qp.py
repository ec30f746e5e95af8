"""General diagonal QP (purin_qp_forward / purin_qp_adjoint) on the GPU.

* The reference's analytic case through the public API (PURIN's
  tests/test_diagonal_qp.py:13-47): value, dy/dc, warm start, shape checks.
* Random sparse QPs with per-sample q, c, values, rhs and bounds against the
  oracle (oracle/diagonal_qp.py): public results bit for bit at a fixed
  iteration count (fp64 and fp32; fixed-step, accelerated, diagonal
  preconditioning, power-iteration steps, converging), and gradients w.r.t.
  every QPData field within 1e-9 where the solve converges.
"""

import numpy as np
import pytest
import torch

from helpers import coupled_diagonal_qp_case, kkt_certified_qp, oracle_config
from oracle.diagonal_qp import OracleDiagonalQP
from purin_b200 import ChambollePockConfig, LinearSolverConfig
from purin_b200.diagonal_qp import QPData, QPStructure, dense_qp_data

pytestmark = pytest.mark.gpu

DEV = "cuda"
JACOBIAN = -np.diag([0.5, 0.25]) + np.outer([0.5, 0.25], [0.5, 0.25]) / 0.75
FIELDS = ("q", "c", "values", "rhs", "lower", "upper")


@pytest.mark.parametrize("accelerated", [False, True])
@pytest.mark.parametrize("scaling", [False, True])
def test_diagonal_qp_value_and_coefficient_gradient(accelerated, scaling):
    structure, data = dense_qp_data(
        torch.tensor([[2.0, 4.0]]), torch.tensor([[-2.0, -4.0]]), torch.ones((1, 2)),
        torch.tensor([1.0]), torch.empty((0, 2)), torch.empty(0), -np.inf, np.inf)
    config = ChambollePockConfig(accelerated=accelerated, row_scaling=scaling, tolerance=1e-9,
                                 max_iterations=3000)
    solver = structure.prepare(batch_size=1, config=config, dtype=torch.float64)
    result = solver.solve(data)
    np.testing.assert_allclose(result.y.cpu().numpy(), [[1 / 3, 2 / 3]], atol=1e-8)
    assert float(result.residual_inf_norm[0]) < 1e-8
    c0 = data.c[0].to(torch.float64)
    jac = torch.autograd.functional.jacobian(
        lambda c: solver.solve(data._replace(c=c[None, :])).y[0], c0.to(DEV))
    np.testing.assert_allclose(jac.cpu().numpy(), JACOBIAN, atol=1e-7)
    warm = solver.solve(data, initial_y=result.y, initial_dual=result.multipliers_eq)
    np.testing.assert_allclose(warm.y.cpu().numpy(), result.y.cpu().numpy(), atol=1e-8)
    with pytest.raises(ValueError):
        solver.solve(data._replace(q=torch.ones((2, 2))))
    with pytest.raises(ValueError):
        solver.solve(data, initial_y=torch.zeros((2, 2)))
    with pytest.raises(ValueError):
        solver.solve(data, initial_dual=torch.zeros((2, 1)))


def random_qp(seed, batch, n, me, mi, per_row, dtype=np.float64, converge=False):
    """Sparse QP with per-sample q, c, values, rhs and bounds, feasible at a seeded x0."""
    rng = np.random.default_rng(seed)
    rows = [tuple(int(j) for j in rng.choice(n, per_row, replace=False)) for _ in range(me + mi)]
    structure = QPStructure(n, tuple(rows[:me]), tuple(rows[me:]))
    width = per_row
    values = rng.normal(size=(batch, me + mi, width))
    x0 = rng.uniform(-0.5, 0.5, size=(batch, n))
    ax = np.einsum("bmw,bmw->bm", values, x0[:, np.asarray(rows)])
    rhs = ax + np.concatenate([np.zeros((batch, me)), rng.uniform(0, 0.1, size=(batch, mi))], 1)
    q = rng.uniform(0.5, 2.0, size=(batch, n))
    c = (0.5 if converge else 2.0) * rng.normal(size=(batch, n))
    lower = rng.uniform(-2.0, -0.6, size=(batch, n))
    upper = rng.uniform(0.6, 2.0, size=(batch, n))
    data = tuple(a.astype(dtype) for a in (q, c, values, rhs, lower, upper))
    return structure, data


FORWARD_CASES = [
    # (name, dtype, config overrides, max_iterations)
    ("fixed-f64", np.float64, {}, 300),
    ("accel-f64", np.float64, {"accelerated": True}, 300),
    ("fixed-f32", np.float32, {}, 300),
    ("accel-f32", np.float32, {"accelerated": True}, 300),
    ("diag-f64", np.float64, {"diagonal_preconditioning": True}, 300),
    ("power-f64", np.float64, {"norm_bound": False}, 300),
    ("noscale-f64", np.float64, {"row_scaling": False}, 300),
    ("converge-f64", np.float64, {"tolerance": 1e-5}, 20000),
]


@pytest.mark.parametrize("name,dtype,overrides,iters", FORWARD_CASES,
                         ids=[c[0] for c in FORWARD_CASES])
def test_public_solve_matches_oracle(name, dtype, overrides, iters):
    structure, data = random_qp(11, 12, 24, 4, 8, 4, dtype, converge=name.startswith("converge"))
    cfg = ChambollePockConfig(max_iterations=iters, **overrides)
    oracle = OracleDiagonalQP(structure.variable_size, structure.equality_rows,
                              structure.inequality_rows, oracle_config(cfg))
    want, _ = oracle.solve(data)
    tdt = torch.float64 if dtype == np.float64 else torch.float32
    solver = structure.prepare(batch_size=12, config=cfg, dtype=tdt)
    got = solver.solve(QPData(*(torch.as_tensor(a, device=DEV) for a in data)))
    if name.startswith("converge"):
        assert want["gradient_eligible"].any()
    # With norm_bound=False tau and sigma come from the power iteration, whose norms
    # are parallel sums in the kernel: floating results agree to rounding there.
    exact = overrides.get("norm_bound", True)
    for field in ("status", "iterations", "finite", "gradient_eligible"):
        np.testing.assert_array_equal(getattr(got, field).cpu().numpy(), want[field],
                                      err_msg=field)
    for field in ("y", "multipliers_eq", "multipliers_ineq", "slacks", "residual_inf_norm"):
        value = getattr(got, field).cpu().numpy()
        if exact:
            np.testing.assert_array_equal(value, want[field], err_msg=field)
        else:
            np.testing.assert_allclose(value, want[field], rtol=0, atol=1e-9, err_msg=field)


@pytest.mark.parametrize("seed,tol,overrides", [(1, 1e-11, {}), (2, 1e-8, {"accelerated": True}),
                                                (3, 1e-11, {"norm_bound": False}),
                                                (4, 1e-11, {"diagonal_preconditioning": True})])
def test_gradients_match_oracle(seed, tol, overrides):
    """Gradients w.r.t. every QPData field through the public API (y and multipliers)."""
    structure, data = random_qp(seed, 6, 8, 2, 4, 3, converge=True)
    cfg = ChambollePockConfig(max_iterations=20000, tolerance=tol,
                              linear_solver=LinearSolverConfig(tolerance=1e-12), **overrides)
    oracle = OracleDiagonalQP(8, structure.equality_rows, structure.inequality_rows,
                              oracle_config(cfg))
    want, saved = oracle.solve(data)
    assert want["gradient_eligible"].any()
    rng = np.random.default_rng(50 + seed)
    cot_y = rng.normal(size=data[0].shape)
    cot_eq = rng.normal(size=want["multipliers_eq"].shape)
    cot_iq = rng.normal(size=want["multipliers_ineq"].shape)
    scale = saved["scale"]
    cot_dual = np.concatenate([cot_eq, cot_iq], axis=1) * scale
    g = oracle.vjp(saved["out"], saved["data"], cot_y, cot_dual)
    g["values"] = g["values"] * scale[:, :, None]
    g["rhs"] = g["rhs"] * scale
    solver = structure.prepare(batch_size=6, config=cfg)
    tensors = [torch.as_tensor(a, device=DEV).requires_grad_(True) for a in data]
    res = solver.solve(QPData(*tensors))
    loss = ((res.y * torch.as_tensor(cot_y, device=DEV)).sum()
            + (res.multipliers_eq * torch.as_tensor(cot_eq, device=DEV)).sum()
            + (res.multipliers_ineq * torch.as_tensor(cot_iq, device=DEV)).sum())
    loss.backward()
    for name, t in zip(FIELDS, tensors):
        np.testing.assert_allclose(t.grad.cpu().numpy(), g[name], rtol=0, atol=1e-9, err_msg=name)


def test_broadcast_constraint_matrix_matches_per_sample_values():
    """values broadcast over the batch (stride 0) run as shared values: same results,
    and the broadcast tensor's gradient is the sum of the per-sample gradients."""
    structure, data = random_qp(7, 6, 8, 2, 4, 3, converge=True)
    cfg = ChambollePockConfig(max_iterations=20000, tolerance=1e-11,
                              linear_solver=LinearSolverConfig(tolerance=1e-12))
    solver = structure.prepare(batch_size=6, config=cfg)
    base = torch.as_tensor(data[2][:1], device=DEV)
    cot = torch.as_tensor(np.random.default_rng(3).normal(size=data[0].shape), device=DEV)
    outs = []
    for shared in (True, False):
        tensors = [torch.as_tensor(a, device=DEV).requires_grad_(True) for a in data]
        vals = base.clone().requires_grad_(True)
        values = vals.expand(6, -1, -1) if shared else vals.expand(6, -1, -1).contiguous()
        assert (values.stride(0) == 0) == shared
        res = solver.solve(QPData(tensors[0], tensors[1], values, *tensors[3:]))
        (res.y * cot).sum().backward()
        outs.append((res, vals.grad, [t.grad for t in tensors]))
    (a, ga, ta), (b, gb, tb) = outs
    for field in ("y", "multipliers_eq", "multipliers_ineq", "status", "iterations"):
        np.testing.assert_array_equal(getattr(a, field).detach().cpu().numpy(),
                                      getattr(b, field).detach().cpu().numpy(), err_msg=field)
    assert bool(a.gradient_eligible.any())
    np.testing.assert_allclose(ga.cpu().numpy(), gb.cpu().numpy(), rtol=1e-12, atol=1e-14)
    for k in (0, 1, 3, 4, 5):
        np.testing.assert_array_equal(ta[k].cpu().numpy(), tb[k].cpu().numpy())


def _box_case(B=4, n=6, bad_sample=None):
    rng = np.random.default_rng(5)
    q = rng.uniform(0.5, 2, (B, n))
    c = rng.normal(size=(B, n))
    lower = np.full((B, n), -0.7)
    upper = np.full((B, n), 0.9)
    if bad_sample is not None:
        lower[bad_sample, 2] = 1.5  # lower > upper: the sample is not a valid QP
    return (q, c, np.zeros((B, 0, 1)), np.zeros((B, 0)), lower, upper)


@pytest.mark.parametrize("bad_sample", [None, 1])
def test_box_only_qp(bad_sample):
    """No constraint rows: y = clip(-c/q, l, u) with dy/dc = -1/q off the bounds, 0 on
    them; a sample with lower > upper is reported unconverged with zero gradients
    (diagonal_qp.py:120-123), as the oracle does."""
    data = _box_case(bad_sample=bad_sample)
    cfg = ChambollePockConfig(max_iterations=5000, tolerance=1e-12)
    oracle = OracleDiagonalQP(6, (), (), oracle_config(cfg))
    want, _ = oracle.solve(data)
    solver = QPStructure(6).prepare(batch_size=4, config=cfg)
    tensors = [torch.as_tensor(a, device=DEV).requires_grad_(True) for a in data]
    res = solver.solve(QPData(*tensors))
    for field in ("y", "status", "iterations", "gradient_eligible"):
        np.testing.assert_array_equal(getattr(res, field).detach().cpu().numpy(), want[field],
                                      err_msg=field)
    q, c, _, _, lower, upper = data
    free = -c / q
    ok = np.ones(4, bool)
    if bad_sample is not None:
        ok[bad_sample] = False
    np.testing.assert_allclose(res.y.detach().cpu().numpy()[ok], np.clip(free, lower, upper)[ok],
                               atol=1e-10)
    res.y.sum().backward()
    inside = (free > lower) & (free < upper)
    expected = np.where(inside, -1.0 / q, 0.0)
    expected[~ok] = 0.0
    np.testing.assert_allclose(tensors[1].grad.cpu().numpy(), expected, atol=1e-9)


def test_single_sample_batch_matches_oracle():
    structure, data = random_qp(21, 1, 16, 3, 5, 4, converge=True)
    cfg = ChambollePockConfig(max_iterations=20000, tolerance=1e-7)
    oracle = OracleDiagonalQP(16, structure.equality_rows, structure.inequality_rows,
                              oracle_config(cfg))
    want, _ = oracle.solve(data)
    got = structure.prepare(batch_size=1, config=cfg).solve(
        QPData(*(torch.as_tensor(a, device=DEV) for a in data)))
    for field in ("y", "multipliers_eq", "multipliers_ineq", "status", "iterations"):
        np.testing.assert_array_equal(getattr(got, field).cpu().numpy(), want[field],
                                      err_msg=field)


def _lockstep_qp_case():
    structure, data = random_qp(1, 8, 8, 2, 4, 3, converge=True)
    cfg = ChambollePockConfig(max_iterations=20000, tolerance=1e-11,
                              linear_solver=LinearSolverConfig(tolerance=1e-16, atol=0.0))
    cot = np.random.default_rng(9).normal(size=data[0].shape)
    return structure, data, cfg, cot


def _qp_grads(solver, data, cot, device):
    tensors = [torch.as_tensor(a, device=device).requires_grad_(True) for a in data]
    res = solver.solve(QPData(*tensors))
    (res.y * torch.as_tensor(cot, device=device)).sum().backward()
    return torch.cat([res.y.detach().reshape(res.y.shape[0], -1)]
                     + [t.grad.reshape(t.shape[0], -1) for t in tensors], dim=1)


def _free_port():
    import socket

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_qp_staged_backward_equals_fused_on_one_rank():
    """set_shard(..., group) runs purin_qp_adjoint_stage through purin_b200.lockstep
    (one NCCL rank here); the gradients equal the fused purin_qp_adjoint's bit for bit."""
    import os
    from datetime import timedelta

    import torch.distributed as dist

    structure, data, cfg, cot = _lockstep_qp_case()
    want = _qp_grads(structure.prepare(batch_size=8, config=cfg), data, cot, DEV)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(_free_port())
    dist.init_process_group("nccl", rank=0, world_size=1, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", torch.cuda.current_device()))
    try:
        solver = structure.prepare(batch_size=8, config=cfg)
        solver.set_shard(0, 8, group=dist.group.WORLD)
        got = _qp_grads(solver, data, cot, DEV)
    finally:
        dist.destroy_process_group()
    np.testing.assert_array_equal(got.cpu().numpy(), want.cpu().numpy())


def _qp_rank(rank, world, port, out_path):
    import os
    from datetime import timedelta

    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    device = torch.device("cuda", rank)
    torch.cuda.set_device(device)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=device,
                            timeout=timedelta(seconds=60))
    try:
        structure, data, cfg, cot = _lockstep_qp_case()
        per = 8 // world
        lo, hi = rank * per, (rank + 1) * per
        solver = structure.prepare(batch_size=per, config=cfg, backend=str(device))
        solver.set_shard(lo, 8, group=dist.group.WORLD)
        local = _qp_grads(solver, tuple(a[lo:hi] for a in data), cot[lo:hi], device)
        gathered = [torch.zeros_like(local) for _ in range(world)]
        dist.all_gather(gathered, local)
        torch.cuda.synchronize(device)
        if rank == 0:
            np.save(out_path, torch.cat(gathered).cpu().numpy())
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_qp_two_nccl_ranks_reproduce_the_full_batch(tmp_path):
    import torch.multiprocessing as mp

    out = tmp_path / "qp_gathered.npy"
    mp.spawn(_qp_rank, args=(2, _free_port(), str(out)), nprocs=2, join=True)
    structure, data, cfg, cot = _lockstep_qp_case()
    want = _qp_grads(structure.prepare(batch_size=8, config=cfg), data, cot, DEV)
    np.testing.assert_array_equal(np.load(out), want.cpu().numpy())


def test_gradients_fp32_match_oracle():
    """fp32 QP gradients w.r.t. every field within 1e-4 of each field's largest."""
    structure, data = random_qp(1, 6, 8, 2, 4, 3, np.float32, converge=True)
    from purin_b200 import ImplicitGradientConfig

    cfg = ChambollePockConfig(max_iterations=20000, tolerance=1e-5,
                              linear_solver=LinearSolverConfig(tolerance=1e-5),
                              implicit_gradient=ImplicitGradientConfig(adjoint_tolerance=1e-4))
    oracle = OracleDiagonalQP(8, structure.equality_rows, structure.inequality_rows,
                              oracle_config(cfg))
    want, saved = oracle.solve(data)
    assert want["gradient_eligible"].any()
    cot_y = np.random.default_rng(61).normal(size=data[0].shape).astype(np.float32)
    g = oracle.vjp(saved["out"], saved["data"], cot_y, None)
    g["values"] = g["values"] * saved["scale"][:, :, None]
    g["rhs"] = g["rhs"] * saved["scale"]
    solver = structure.prepare(batch_size=6, config=cfg, dtype=torch.float32)
    tensors = [torch.as_tensor(a, device=DEV).requires_grad_(True) for a in data]
    res = solver.solve(QPData(*tensors))
    (res.y * torch.as_tensor(cot_y, device=DEV)).sum().backward()
    for name, t in zip(FIELDS, tensors):
        scale = max(float(np.abs(g[name]).max()), 1e-6)
        np.testing.assert_allclose(t.grad.cpu().numpy(), g[name], rtol=0, atol=1e-4 * scale,
                                   err_msg=name)


@pytest.mark.parametrize("diagonal", [False, True])
def test_coupled_inequalities_match_a_certified_kkt_solution(diagonal):
    """tests/test_regression_cp_diagonal_steps.py:28-80 on the QP kernels: converged
    (tolerance 1e-9) to the exact solution within 3e-8 (an exact KKT solve on the
    identified active set stands in for the reference's OSQP)."""
    eq_rows, in_rows, data, matrix = coupled_diagonal_qp_case()
    cfg = ChambollePockConfig(tolerance=1e-9, max_iterations=20000, row_scaling=False,
                              diagonal_preconditioning=diagonal)
    solver = QPStructure(6, eq_rows, in_rows).prepare(batch_size=3, config=cfg,
                                                      dtype=torch.float64)
    result = solver.solve(QPData(*(torch.as_tensor(a, device=DEV) for a in data)))
    assert (result.status.cpu().numpy() == 0).all()
    q, c, _, rhs, lower, upper = data
    y = result.y.cpu().numpy()
    for i in range(len(q)):
        exact = kkt_certified_qp(q[i], c[i], matrix, rhs[i], 2, lower[i], upper[i], y[i])
        np.testing.assert_allclose(y[i], exact, atol=3e-8)
