"""Lockstep GMRES across shards of a batch (CPU: oracle shards, gloo ranks).

The reference's adjoint runs one restarted GMRES over the whole batch with a
single iteration budget (operators.py:919-1103).  A shard that ran its own
loop would charge only its own cycles; ``purin_b200.lockstep.run`` combines
the shards' counters (in process, and across ranks with an all-reduce) so
that sharded gradients equal the unsharded ones bit for bit.  Here the shards
are the oracle's staged VJP (``OracleProjection.vjp_shard``), which is what
the CUDA stages (``purin_cp_adjoint_stage``) are checked against on the GPU.
"""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from helpers import OracleLayer, random_sparse_problem, random_theta
from purin_b200 import ChambollePockConfig, LinearSolverConfig, lockstep

BATCH = 8
HALF = BATCH // 2


def lockstep_case():
    """A batch whose halves, each run on its own, charge different GMRES budgets.

    GMRES runs close to its attainable accuracy (tolerance 1e-16, atol 0), where
    samples leave their cycles early and re-enter the next one, so the cycle
    lengths of a half differ from those of the whole batch.
    """
    rng = np.random.default_rng(36)
    problem, mats = random_sparse_problem(rng, 12, 3, 6, 3)
    theta = random_theta(rng, mats, BATCH)
    target = 1.5 * rng.normal(size=(BATCH, 12))
    cfg = ChambollePockConfig(max_iterations=20000, tolerance=1e-11,
                              linear_solver=LinearSolverConfig(restart=30, max_iterations=100,
                                                               tolerance=1e-16, atol=0.0))
    cot = np.random.default_rng(136).normal(size=target.shape)
    return problem, cfg, theta, target, cot


def _full(layer, theta, target, cot):
    _, saved = layer.solve(target, theta)
    stats = {}
    grads = layer.proj.vjp(saved, cot, stats=stats)
    return grads, stats


def _shard(layer, theta, target, cot, lo, hi):
    _, saved = layer.solve(target[lo:hi], theta[lo:hi], offset=lo, total=BATCH)
    return saved, layer.proj.vjp_shard(saved, cot[lo:hi])


def _flat(grads):
    return np.concatenate([grads[k].reshape(grads[k].shape[0], -1)
                           for k in ("values", "rhs", "target", "lower", "upper")], axis=1)


@pytest.fixture(scope="module")
def case():
    problem, cfg, theta, target, cot = lockstep_case()
    layer = OracleLayer(problem, cfg)
    full, stats = _full(layer, theta, target, cot)
    return layer, theta, target, cot, full, stats


def test_halves_on_their_own_charge_different_budgets(case):
    """The case has teeth: independent halves do not reproduce the full batch."""
    layer, theta, target, cot, full, stats = case
    local = []
    for lo, hi in ((0, HALF), (HALF, BATCH)):
        _, saved = layer.solve(target[lo:hi], theta[lo:hi], offset=lo, total=BATCH)
        s = {}
        local.append((layer.proj.vjp(saved, cot[lo:hi], stats=s), s))
    budgets = [(s["completed"], s["cycles"]) for _, s in local]
    assert any(b != (stats["completed"], stats["cycles"]) for b in budgets)
    joined = np.concatenate([_flat(g) for g, _ in local])
    assert not np.array_equal(joined, _flat(full))


def test_in_process_shards_reproduce_the_full_batch(case):
    """Two shards in one process (e.g. chunks of a batch) driven in lockstep."""
    layer, theta, target, cot, full, stats = case
    shards = [_shard(layer, theta, target, cot, lo, hi)[1] for lo, hi in ((0, HALF), (HALF, BATCH))]
    outputs, completed, cycles = lockstep.run(shards, 100)
    assert (completed, cycles) == (stats["completed"], stats["cycles"])
    joined = np.concatenate([_flat(g) for g, _, _ in outputs])
    np.testing.assert_array_equal(joined, _flat(full))
    code = np.concatenate([c for _, c, _ in outputs])
    np.testing.assert_array_equal(code, stats["code"])


def test_uneven_and_empty_shards(case):
    """Shards of 1, 7 and 0 samples: an empty shard reports zeros and changes nothing."""
    layer, theta, target, cot, full, stats = case

    class Empty:
        def prepare(self):
            return (0, 0)

        def cycle(self, completed):
            return (0, 0)

        def finish(self):
            return None

    shards = [_shard(layer, theta, target, cot, 0, 1)[1], Empty(),
              _shard(layer, theta, target, cot, 1, BATCH)[1]]
    outputs, completed, cycles = lockstep.run(shards, 100)
    assert (completed, cycles) == (stats["completed"], stats["cycles"])
    joined = np.concatenate([_flat(outputs[0][0]), _flat(outputs[2][0])])
    np.testing.assert_array_equal(joined, _flat(full))


def test_combine_max_and_the_stalled_cycle_guard():
    assert lockstep.combine_max([(3, 0), torch.tensor([5, 2]), np.array([1, 7])]) == (5, 7)
    with pytest.raises(ValueError):
        lockstep.combine_max([])

    class Stalled:
        def prepare(self):
            return (0, 1)

        def cycle(self, completed):
            return (0, 1)

        def finish(self):
            return None

    with pytest.raises(RuntimeError, match="no Arnoldi steps"):
        lockstep.run([Stalled()], 10)


def _worker(rank, world, port, out_path):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        problem, cfg, theta, target, cot = lockstep_case()
        layer = OracleLayer(problem, cfg)
        lo, hi = rank * HALF, (rank + 1) * HALF
        _, shard = _shard(layer, theta, target, cot, lo, hi)
        outputs, completed, cycles = lockstep.run([shard], 100, group=dist.group.WORLD)
        grads, code, _ = outputs[0]
        local = torch.as_tensor(np.concatenate([_flat(grads), code[:, None].astype(np.float64),
                                                np.full((HALF, 2), [completed, cycles],
                                                        np.float64)], axis=1))
        gathered = [torch.zeros_like(local) for _ in range(world)]
        dist.all_gather(gathered, local)
        if rank == 0:
            np.save(out_path, torch.cat(gathered).numpy())
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_two_gloo_ranks_reproduce_the_full_batch(case, tmp_path):
    layer, theta, target, cot, full, stats = case
    out = tmp_path / "gathered.npy"
    mp.spawn(_worker, args=(2, _free_port(), str(out)), nprocs=2, join=True)
    gathered = np.load(out)
    width = _flat(full).shape[1]
    np.testing.assert_array_equal(gathered[:, :width], _flat(full))
    np.testing.assert_array_equal(gathered[:, width], stats["code"])
    np.testing.assert_array_equal(gathered[:, width + 1:],
                                  np.tile([stats["completed"], stats["cycles"]], (BATCH, 1)))


def _dropping_worker(rank, world, port, out_path):
    """Rank 1 leaves between steps without joining the exchange; rank 0's lockstep
    all-reduce must end with an error (connection closed or the group's short
    timeout), not wait forever."""
    import json
    import time
    from datetime import timedelta

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=10))
    if rank == 1:
        os._exit(0)
    problem, cfg, theta, target, cot = lockstep_case()
    layer = OracleLayer(problem, cfg)
    _, shard = _shard(layer, theta, target, cot, 0, HALF)
    t0 = time.time()
    try:
        lockstep.run([shard], 100, group=dist.group.WORLD)
        outcome = "completed"
    except Exception as exc:  # the failure the peer's departure must surface
        outcome = f"error {type(exc).__name__}"
    with open(out_path, "w") as f:
        json.dump({"outcome": outcome, "seconds": time.time() - t0}, f)
    os._exit(0)


def test_dropped_rank_ends_the_exchange_with_an_error(tmp_path):
    import json

    out = tmp_path / "dropped.json"
    mp.spawn(_dropping_worker, args=(2, _free_port(), str(out)), nprocs=2, join=True)
    result = json.loads(out.read_text())
    assert result["outcome"].startswith("error"), result
    assert result["seconds"] < 60
