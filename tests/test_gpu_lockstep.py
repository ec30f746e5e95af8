"""Staged adjoint (purin_cp_adjoint_stage) and GMRES lockstep across shards, on the GPU.

* One shard driven through the three phases equals the fused single-launch
  adjoint bit for bit.
* Two shards of a batch in one process (two layers, as chunks of the batch),
  driven by ``purin_b200.lockstep.run``, equal the full batch's fused adjoint
  bit for bit, where the same halves run on their own charge a different GMRES
  budget.
* With two or more GPUs: two NCCL ranks through the public API
  (``set_shard(..., group)``) equal one process running the whole batch.
"""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp
from dataclasses import replace

from helpers import OracleLayer, ell_to_csr
from purin_b200 import ImplicitGradientConfig, lockstep, prepare_projection
from test_lockstep import BATCH, HALF, lockstep_case

pytestmark = pytest.mark.gpu

DEV = "cuda"
NAMES = ("values", "rhs", "target", "lower", "upper")


def _t(a, dtype, device=DEV):
    return torch.as_tensor(np.ascontiguousarray(a), dtype=dtype, device=device)


def _layer(problem, cfg, batch, device=DEV):
    return prepare_projection(problem, method="chambolle-pock", config=cfg, batch_size=batch,
                              dtype=torch.float64, backend=device)


def _shard(layer, oracle, saved, cot):
    """A staged adjoint shard over the oracle's saved forward state (boundary inputs)."""
    dt = torch.float64
    out = saved["out"]
    data = _t(ell_to_csr(saved["values"], list(oracle.proj.mask.sum(axis=1))), dt)
    return layer._adjoint_shard(
        data, _t(saved["rhs"], dt), _t(saved["target"], dt), _t(saved["lower"], dt),
        _t(saved["upper"], dt), _t(out.y, dt), _t(out.dual, dt),
        _t(out.converged.astype(np.uint8), torch.uint8), _t(cot, dt), need_values=True,
        need_rhs=True, need_target=True, need_lower=True, need_upper=True)


def _numpy(grads, shard):
    torch.cuda.synchronize()
    return ({k: g.cpu().numpy() for k, g in zip(NAMES, grads)}, shard.status.cpu().numpy(),
            shard.lres.cpu().numpy())


@pytest.fixture(scope="module")
def case():
    problem, cfg, theta, target, cot = lockstep_case()
    oracle = OracleLayer(problem, cfg)
    _, saved = oracle.solve(target, theta)
    halves = []
    for lo, hi in ((0, HALF), (HALF, BATCH)):
        _, s = oracle.solve(target[lo:hi], theta[lo:hi], offset=lo, total=BATCH)
        halves.append((lo, hi, s))
    return problem, cfg, theta, target, cot, oracle, saved, halves


def _full_fused(case):
    problem, cfg, theta, target, cot, oracle, saved, _ = case
    layer = _layer(problem, cfg, BATCH)
    shard = _shard(layer, oracle, saved, cot)
    return _numpy(shard.fused(), shard)


def test_staged_single_shard_equals_fused(case):
    problem, cfg, theta, target, cot, oracle, saved, _ = case
    want, want_status, want_res = _full_fused(case)
    layer = _layer(problem, cfg, BATCH)
    shard = _shard(layer, oracle, saved, cot)
    (grads,), completed, cycles = lockstep.run([shard], cfg.linear_solver.max_iterations)
    got, status, res = _numpy(grads, shard)
    assert completed > 0 and cycles > 1
    np.testing.assert_array_equal(status, want_status)
    np.testing.assert_array_equal(res, want_res)
    for k in NAMES:
        np.testing.assert_array_equal(got[k], want[k], err_msg=k)


def test_full_batch_matches_oracle(case):
    """The case itself: the GPU's full-batch gradients agree with the oracle's."""
    problem, cfg, theta, target, cot, oracle, saved, _ = case
    want = oracle.proj.vjp(saved, cot)
    got, _, _ = _full_fused(case)
    for k in NAMES:
        exp = want[k]
        if k == "values":
            exp = ell_to_csr(exp, list(oracle.proj.mask.sum(axis=1)))
        np.testing.assert_allclose(got[k], exp, rtol=0, atol=1e-9, err_msg=k)


def test_gpu_shards_in_lockstep_reproduce_the_full_batch(case):
    problem, cfg, theta, target, cot, oracle, saved, halves = case
    want, want_status, want_res = _full_fused(case)
    shards, alone = [], []
    for lo, hi, s in halves:
        layer = _layer(problem, cfg, hi - lo)
        layer.set_shard(lo, BATCH)
        shards.append(_shard(layer, oracle, s, cot[lo:hi]))
        # The same half on its own (its own budget), for the contrast below.
        solo = _shard(layer, oracle, s, cot[lo:hi])
        _, completed, cycles = lockstep.run([solo], cfg.linear_solver.max_iterations)
        alone.append((completed, cycles))
    outputs, completed, cycles = lockstep.run(shards, cfg.linear_solver.max_iterations)
    assert any(budget != (completed, cycles) for budget in alone)
    parts = [_numpy(g, s) for g, s in zip(outputs, shards)]
    np.testing.assert_array_equal(np.concatenate([p[1] for p in parts]), want_status)
    np.testing.assert_array_equal(np.concatenate([p[2] for p in parts]), want_res)
    for k in NAMES:
        np.testing.assert_array_equal(np.concatenate([p[0][k] for p in parts]), want[k],
                                      err_msg=k)


# ---- two GPUs, one NCCL rank each, through the public API ----------------------

def _public_case():
    problem, cfg, theta, target, cot = lockstep_case()
    cfg = replace(cfg, implicit_gradient=ImplicitGradientConfig(
        differentiate_problem_parameters=True))
    return problem, cfg, theta, target, cot


def _public_step(layer, theta, target, cot, device):
    x = _t(target, torch.float64, device).requires_grad_(True)
    th = _t(theta, torch.float64, device).requires_grad_(True)
    y = layer(x, th)
    (y * _t(cot, torch.float64, device)).sum().backward()
    return torch.cat([y.detach(), x.grad, th.grad], dim=1)


def _rank(rank, world, port, out_path):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    device = torch.device("cuda", rank)
    torch.cuda.set_device(device)
    from datetime import timedelta

    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=device,
                            timeout=timedelta(seconds=60))
    try:
        problem, cfg, theta, target, cot = _public_case()
        per = BATCH // world
        lo, hi = rank * per, (rank + 1) * per
        layer = _layer(problem, cfg, per, device)
        layer.set_shard(lo, BATCH, group=dist.group.WORLD)
        local = _public_step(layer, theta[lo:hi], target[lo:hi], cot[lo:hi], device)
        gathered = [torch.zeros_like(local) for _ in range(world)]
        dist.all_gather(gathered, local)
        torch.cuda.synchronize(device)
        if rank == 0:
            np.save(out_path, torch.cat(gathered).cpu().numpy())
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_nccl_ranks_reproduce_the_full_batch(tmp_path):
    out = tmp_path / "gathered.npy"
    mp.spawn(_rank, args=(2, _free_port(), str(out)), nprocs=2, join=True)
    problem, cfg, theta, target, cot = _public_case()
    layer = _layer(problem, cfg, BATCH)
    want = _public_step(layer, theta, target, cot, torch.device(DEV)).cpu().numpy()
    np.testing.assert_array_equal(np.load(out), want)


# ---- the cluster-resident GMRES kernel (problems whose basis needs a cluster) -----

def _cluster_case():
    """Configuration 2's structure (n = 2048, 512 + 1024 rows): its Krylov basis lives in
    the shared memory of 8-CTA clusters.  CP tolerance 1e-3 so the samples are accepted;
    GMRES to 1e-5 within 200 steps, which the samples reach in different cycles (the
    oracle takes 145 steps over 5 cycles)."""
    from purin_b200 import LinearSolverConfig
    from purin_b200.workloads import make_workload

    w = make_workload(2, 4)
    cfg = replace(w.config, tolerance=1e-3,
                  linear_solver=LinearSolverConfig(tolerance=1e-5, max_iterations=200))
    cot = np.random.default_rng(11).normal(size=w.candidates.shape)
    return w.problem, cfg, w.theta, w.candidates, cot


@pytest.fixture(scope="module")
def cluster_case():
    problem, cfg, theta, target, cot = _cluster_case()
    oracle = OracleLayer(problem, cfg)
    _, saved = oracle.solve(target, theta)
    halves = []
    for lo, hi in ((0, 2), (2, 4)):
        _, s = oracle.solve(target[lo:hi], theta[lo:hi], offset=lo, total=4)
        halves.append((lo, hi, s))
    return problem, cfg, cot, oracle, saved, halves


def test_cluster_gmres_staged_and_sharded_equal_fused(cluster_case):
    """The cluster kernel's one-cycle launches, driven by the lockstep, equal its fused
    launch bit for bit, for one shard and for two halves of the batch."""
    problem, cfg, cot, oracle, saved, halves = cluster_case
    assert saved["out"].converged.all()
    layer = _layer(problem, cfg, 4)
    fused = _shard(layer, oracle, saved, cot)
    want, want_status, want_res = _numpy(fused.fused(), fused)
    staged = _shard(layer, oracle, saved, cot)
    (grads,), completed, cycles = lockstep.run([staged], cfg.linear_solver.max_iterations)
    got, status, res = _numpy(grads, staged)
    assert cycles >= 1
    np.testing.assert_array_equal(status, want_status)
    np.testing.assert_array_equal(res, want_res)
    for k in NAMES:
        np.testing.assert_array_equal(got[k], want[k], err_msg=k)
    shards = []
    for lo, hi, s in halves:
        half = _layer(problem, cfg, hi - lo)
        half.set_shard(lo, 4)
        shards.append(_shard(half, oracle, s, cot[lo:hi]))
    outputs, _, _ = lockstep.run(shards, cfg.linear_solver.max_iterations)
    parts = [_numpy(g, s) for g, s in zip(outputs, shards)]
    np.testing.assert_array_equal(np.concatenate([p[1] for p in parts]), want_status)
    np.testing.assert_array_equal(np.concatenate([p[2] for p in parts]), want_res)
    for k in NAMES:
        np.testing.assert_array_equal(np.concatenate([p[0][k] for p in parts]), want[k],
                                      err_msg=k)


def test_cluster_gmres_matches_the_cta_kernel_and_the_oracle(cluster_case, monkeypatch):
    """The same solves on the CTA-per-sample kernel (PURIN_CP_GMRES_CLUSTER=0) and in the
    oracle: equal status codes, and gradients within 1e-6 of the largest gradient (GMRES
    stops at a relative residual of 1e-5, so solves that round differently agree to a
    fraction of that, not to the last bits)."""
    problem, cfg, cot, oracle, saved, _ = cluster_case
    layer = _layer(problem, cfg, 4)
    shard = _shard(layer, oracle, saved, cot)
    got, status, _ = _numpy(shard.fused(), shard)
    monkeypatch.setenv("PURIN_CP_GMRES_CLUSTER", "0")
    cta = _shard(layer, oracle, saved, cot)
    ref, ref_status, _ = _numpy(cta.fused(), cta)
    monkeypatch.delenv("PURIN_CP_GMRES_CLUSTER")
    stats = {}
    want = oracle.proj.vjp(saved, cot, stats=stats)
    np.testing.assert_array_equal(status, ref_status)
    np.testing.assert_array_equal(status, stats["code"])
    for k in NAMES:
        exp = want[k]
        if k == "values":
            exp = ell_to_csr(exp, list(oracle.proj.mask.sum(axis=1)))
        scale = max(float(np.abs(exp).max()), 1e-300)
        np.testing.assert_allclose(got[k], ref[k], rtol=0, atol=1e-6 * scale, err_msg=k)
        np.testing.assert_allclose(got[k], exp, rtol=0, atol=1e-6 * scale, err_msg=k)


def test_workspace_query_covers_either_gmres_kernel(monkeypatch):
    """The adjoint workspace a layer sizes before the call (purin_cp_workspace_size, which
    does not know the global batch) must cover the GMRES kernel the call then picks: the
    streaming kernel for a batch beyond one wave of clusters (fp32 configuration 4, 32
    samples, 8-CTA clusters), the clusters when forced.  Both give the same status codes
    and gradients to GMRES's accuracy."""
    from purin_b200 import LinearSolverConfig
    from purin_b200.workloads import make_workload

    w = make_workload(4, 32)
    cfg = replace(w.config, tolerance=0.5, linear_solver=LinearSolverConfig(tolerance=1e-4))
    layer = prepare_projection(w.problem, method="chambolle-pock", config=cfg, batch_size=32,
                               dtype=torch.float32, backend=DEV)
    grads, codes = [], []
    for mode in ("", "1"):
        if mode:
            monkeypatch.setenv("PURIN_CP_GMRES_CLUSTER", mode)
        x = _t(w.candidates, torch.float32).requires_grad_(True)
        y = layer(x, _t(w.theta, torch.float32))
        ((y - _t(w.targets, torch.float32)) ** 2).sum().backward()
        grads.append(x.grad.cpu().numpy())
        codes.append(layer._last_linear[0].cpu().numpy())
    np.testing.assert_array_equal(codes[0], codes[1])
    assert (codes[0] == 0).any()
    scale = float(np.abs(grads[0]).max())
    np.testing.assert_allclose(grads[1], grads[0], rtol=0, atol=1e-3 * scale)
