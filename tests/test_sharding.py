"""Sample sharding across ranks (world size 2, gloo on CPU).

Each rank solves its contiguous shard of the batch with the shard's global
sample offset (which selects the PRNG keys of the seeded power iteration);
gathering the shards must reproduce the unsharded batch exactly.  This is the
host-side logic of the multi-GPU path: ranks exchange nothing on the data path.
"""

import os
import socket
from dataclasses import replace

import numpy as np
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from helpers import OracleLayer
from purin_b200.workloads import make_workload

BATCH = 8


def _case():
    w = make_workload(0, BATCH)
    # norm_bound=False: the forward step sizes come from the seeded power iteration.
    cfg = replace(w.config, max_iterations=40, norm_bound=False)
    return w, cfg


def _worker(rank, world, port, out_path):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        w, cfg = _case()
        shard = BATCH // world
        sl = slice(rank * shard, (rank + 1) * shard)
        layer = OracleLayer(w.problem, cfg)
        result, saved = layer.solve(w.candidates[sl], w.theta[sl], offset=rank * shard, total=BATCH)
        cot = np.ones((shard, w.candidates.shape[1]))
        grads = layer.proj.vjp(saved, cot)
        local = torch.as_tensor(np.concatenate([result["y"], grads["target"]], axis=1))
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


def test_two_rank_shards_reproduce_the_full_batch(tmp_path):
    out = tmp_path / "gathered.npy"
    mp.spawn(_worker, args=(2, _free_port(), str(out)), nprocs=2, join=True)
    gathered = np.load(out)
    w, cfg = _case()
    layer = OracleLayer(w.problem, cfg)
    result, saved = layer.solve(w.candidates, w.theta)
    grads = layer.proj.vjp(saved, np.ones_like(w.candidates))
    np.testing.assert_array_equal(gathered, np.concatenate([result["y"], grads["target"]], axis=1))


def test_shard_offsets_change_the_power_iteration_keys():
    """Without the global offset a shard would draw the wrong normals (and steps)."""
    w, cfg = _case()
    layer = OracleLayer(w.problem, cfg)
    right, _ = layer.solve(w.candidates[4:], w.theta[4:], offset=4, total=BATCH)
    wrong, _ = layer.solve(w.candidates[4:], w.theta[4:])
    full, _ = layer.solve(w.candidates, w.theta)
    np.testing.assert_array_equal(right["y"], full["y"][4:])
    assert not np.array_equal(wrong["y"], full["y"][4:])
