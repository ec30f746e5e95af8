"""The forward's global stopping rule on the GPU: bit-identical outputs with it on and off.

``set_global_stop(interval, group)`` runs the forward in segments of
``interval`` iterations on the diagonal-QP kernels (q = 1, c = -target) and
stops the batch at the first segment end where no sample is still running on
any rank (``kernels.py:238-240``).  Samples freeze when accepted
(``kernels.py:266-271``), so every output -- and the implicit gradient, which
starts from them -- must equal the default per-sample stopping bit for bit.
With two GPUs, two NCCL ranks (NVLS off) sum their running samples after every
segment and must agree on the batch's trip count.
"""

import os
import socket
from dataclasses import replace

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from purin_b200 import ImplicitGradientConfig, prepare_projection
from purin_b200.workloads import make_workload

pytestmark = pytest.mark.gpu
DEV = "cuda"
FIELDS = ("y", "multipliers_eq", "multipliers_ineq", "slacks", "status", "iterations",
          "residual_inf_norm", "finite", "gradient_eligible")

CASES = [
    # (name, config index, batch, dtype, overrides, interval)
    ("fixed-f64", 0, 16, torch.float64, {"tolerance": 1e-4, "max_iterations": 4000}, 100),
    ("accel-f64", 0, 16, torch.float64, {"tolerance": 1e-4, "max_iterations": 4000,
                                         "accelerated": True}, 37),
    ("fixed-f32", 0, 16, torch.float32, {"tolerance": 1e-3, "max_iterations": 3000}, 250),
    ("diag-f64", 0, 16, torch.float64, {"tolerance": 1e-4, "max_iterations": 4000,
                                        "diagonal_preconditioning": True}, 100),
    ("power-f64", 0, 16, torch.float64, {"tolerance": 1e-4, "max_iterations": 4000,
                                         "norm_bound": False}, 100),
    ("budget-f64", 0, 16, torch.float64, {}, 64),
    ("config2-f64", 2, 4, torch.float64, {"tolerance": 1e-3}, 200),
]


def _step(layer, w, dtype):
    x = torch.as_tensor(w.candidates, dtype=dtype, device=DEV).requires_grad_(True)
    th = torch.as_tensor(w.theta, dtype=dtype, device=DEV).requires_grad_(True)
    result = layer.solve(x, th)
    (result.y * torch.as_tensor(w.targets, dtype=dtype, device=DEV)).sum().backward()
    return result, x.grad, th.grad


@pytest.mark.parametrize("name,index,batch,dtype,overrides,interval", CASES,
                         ids=[c[0] for c in CASES])
def test_global_stop_outputs_equal_per_sample_stopping(name, index, batch, dtype, overrides,
                                                       interval):
    w = make_workload(index, batch)
    cfg = replace(w.config, implicit_gradient=ImplicitGradientConfig(
        differentiate_problem_parameters=True), **overrides)
    layer = prepare_projection(w.problem, method="chambolle-pock", config=cfg, batch_size=batch,
                               dtype=dtype, backend=DEV)
    want, want_gx, want_gt = _step(layer, w, dtype)
    layer.set_global_stop(interval)
    got, got_gx, got_gt = _step(layer, w, dtype)
    layer.set_global_stop(None)
    for field in FIELDS:
        np.testing.assert_array_equal(getattr(got, field).detach().cpu().numpy(),
                                      getattr(want, field).detach().cpu().numpy(), err_msg=field)
    np.testing.assert_array_equal(got_gx.cpu().numpy(), want_gx.cpu().numpy())
    np.testing.assert_array_equal(got_gt.cpu().numpy(), want_gt.cpu().numpy())
    assert layer.last_global_trip == int(want.iterations.max())
    if name != "budget-f64":
        assert int(want.iterations.min()) < cfg.max_iterations  # some samples froze early


def _rank(rank, world, port, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    device = torch.device("cuda", rank)
    torch.cuda.set_device(device)
    from datetime import timedelta

    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=device,
                            timeout=timedelta(seconds=60))
    try:
        per = 8
        w = make_workload(0, per, offset=rank * per)
        cfg = replace(w.config, tolerance=1e-4, max_iterations=4000)
        layer = prepare_projection(w.problem, method="chambolle-pock", config=cfg,
                                   batch_size=per, backend=str(device))
        layer.set_shard(rank * per, per * world)
        layer.set_global_stop(100, dist.group.WORLD)
        result = layer.solve(torch.as_tensor(w.candidates, device=device),
                             torch.as_tensor(w.theta, device=device))
        local = torch.cat([result.y, result.iterations[:, None].double()], dim=1)
        gathered = [torch.zeros_like(local) for _ in range(world)]
        dist.all_gather(gathered, local)
        trips = [torch.zeros(1, dtype=torch.int64, device=device) for _ in range(world)]
        dist.all_gather(trips, torch.tensor([layer.last_global_trip], device=device))
        torch.cuda.synchronize(device)
        if rank == 0:
            np.save(out, torch.cat(gathered).cpu().numpy())
            np.save(out + ".trips.npy", torch.cat(trips).cpu().numpy())
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_nccl_ranks_share_the_stop(tmp_path):
    out = str(tmp_path / "gathered.npy")
    mp.spawn(_rank, args=(2, _free_port(), out), nprocs=2, join=True)
    w = make_workload(0, 16)
    cfg = replace(w.config, tolerance=1e-4, max_iterations=4000)
    layer = prepare_projection(w.problem, method="chambolle-pock", config=cfg, batch_size=16,
                               backend=DEV)
    result = layer.solve(torch.as_tensor(w.candidates, device=DEV),
                         torch.as_tensor(w.theta, device=DEV))
    want = torch.cat([result.y, result.iterations[:, None].double()], dim=1).cpu().numpy()
    np.testing.assert_array_equal(np.load(out), want)
    trips = np.load(out + ".trips.npy")
    assert (trips == int(result.iterations.max())).all()
