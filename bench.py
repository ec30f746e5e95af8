"""Benchmark of the B200 CP projection layer (forward + implicit VJP).

Contract: ``python bench.py --gpus N --steps K --warmup W [--impl reference]`` prints
ONE JSON line.  For N > 1 it runs under ``torch.distributed.run`` with one rank
per GPU; the ranks share one seeded global batch of N x B samples and rank r
solves samples [r B, (r + 1) B) (weak scaling; the forward needs no exchange,
the adjoint's GMRES counters are all-reduced once per cycle so the shards share
the batch's budget) and the step time is the maximum over ranks.  The line
carries a checksum of every rank's projections (``shard_checksums``), which a
1-GPU run over the same global batch reproduces slice by slice.

Workload: benchmark configuration 2 (fp64, B = 2048 per GPU, n = 2048,
me = 512, mi = 1024, 8 nnz per row, box bounds as 2n singleton rows, fixed
2000 fixed-step CP iterations with the reference's stopping test, loss
0.5 ||y - t||^2, gradients w.r.t. the candidates and the parameters
theta = [b; h]).  One step = forward + VJP over the whole batch.

* ``value``: samples/s with every input already resident in HBM (device time,
  CUDA events, per-step L2 flush outside the timed events).
* ``e2e``: the same step through the public API from pinned host buffers,
  host->device copies of candidates/parameters/targets and device->host copies
  of the loss and both gradients inside the timed region.
* ``roofline``: the dominant kernel's algorithmic bytes per launch divided by
  its event-timed launch duration, against MEASURED_PEAKS.json.
* ``cpu_baseline``: the oracle (a restatement of the reference's JAX path; JAX
  itself is not installed on the host) on a bounded sample, its CP loop in C++
  over every host core.
"""

from __future__ import annotations

import argparse
import dataclasses
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

CONFIG_INDEX = 2
METRIC = "CP samples/sec at fixed iters (fwd+VJP)"
DEFAULT_BATCH = {0: 256, 1: 4096, 2: 2048, 3: 2048, 4: 16384}
WORKLOADS = {
    0: "config0: fp64, n=64, me=32, mi=32, 4 nnz/row, |y|<=1, 500 fixed-step CP iterations",
    1: "config1: n=1024, me=256, mi=512, 8 nnz/row, box bounds, 1000 accelerated CP iterations",
    2: "config2: fp64, n=2048, me=512, mi=1024, 8 nnz/row, box bounds, 2000 fixed-step CP "
       "iterations",
    3: "config3: fp32 network flow, 5000 nodes, 20000 edges, 4000 coupling rows, capacity "
       "bounds, 1500 fixed-step CP iterations",
    4: "config4: WeightedDistance w~U(0.5,2), n=4096, me=1024, mi=2048, 16 nnz/row, box bounds, "
       "1000 accelerated CP iterations",
}
FALLBACK_HBM_GBS = 6650.0
# DRAM bytes (read + write) of one cp_forward_kernel launch per sample, from the
# ncu capture of 592 samples in profiles/cp_forward_config2_b592.md
# ((24.674048 MB + 512 B) / 592); the iterates stay on chip, so the traffic is
# the per-sample inputs and grows with the batch.
FORWARD_DRAM_BYTES_PER_SAMPLE = (24.674048e6 + 512.0) / 592
# The same capture: the L1 data pipe's wavefront rate (the forward's limiter) and
# the share of shared-memory load wavefronts that are bank conflicts (2.18 G of 5.07 G).
FORWARD_L1_PIPE_FRAC = 0.778
FORWARD_BANK_CONFLICT_SHARE = 2.18 / 5.07


def parse_args():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=5)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", default="native", choices=["native", "reference"])
    p.add_argument("--batch", type=int, default=None,
                   help="samples per GPU (default: 2048 for configs 2 and 3, 4096 for config 1, "
                        "16384 for config 4, 256 for config 0)")
    p.add_argument("--config", type=int, default=CONFIG_INDEX, choices=[0, 1, 2, 3, 4],
                   help="benchmark configuration (the headline is configuration 2)")
    p.add_argument("--mode", default=None, choices=["fwd", "fwd+vjp"],
                   help="forward only or forward + VJP (default: fwd+vjp for config 2, else fwd)")
    p.add_argument("--dtype", default=None, choices=["float64", "float32"],
                   help="override the configuration's dtype")
    p.add_argument("--cpu-samples", type=int, default=None,
                   help="samples in the CPU baseline (default 48 per host core, ~15 s)")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--vjp-active-tolerance", type=float, default=1e-3,
                   help="CP tolerance of the extra GMRES-active VJP measurement that the "
                        "configuration-2 fwd+VJP line carries as 'vjp_active' (0 to skip)")
    p.add_argument("--cp-tolerance", type=float, default=None,
                   help="override the CP stopping tolerance (default: the workload's 1e-9); "
                        "a loose value such as 1e-3 lets samples converge so that the VJP "
                        "runs full GMRES solves instead of being gated to zero")
    p.add_argument("--diagonal-preconditioning", action="store_true",
                   help="ChambollePockConfig(diagonal_preconditioning=True) for fixed-step runs")
    p.add_argument("--qp-values", default="shared", choices=["shared", "per-sample"],
                   help="qp: one constraint matrix for the batch (a broadcast view) or a "
                        "separate copy per sample (the same values, materialised)")
    p.add_argument("--problem", default="projection", choices=["projection", "qp", "dense", "admm"],
                   help="qp: configuration 2's structure as a general diagonal QP "
                        "(PreparedDiagonalQP), fwd + VJP w.r.t. q, c, values, rhs and bounds; "
                        "dense: solve_dense_implicit on per-sample dense matrices; "
                        "admm: configuration 0's structure through method='admm' (fwd + VJP)")
    return p.parse_args()


def peaks():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        data = json.loads(path.read_text())
        return float(data["hbm_gbs"]), "measured"
    return FALLBACK_HBM_GBS, "fallback"


def algorithmic_bytes_forward(n, m, w, iterations_total):
    """(5n + 3m) * w per sample-iteration: read y, ybar, target, lambda, rhs; write y, ybar, lambda."""
    return float(iterations_total) * (5 * n + 3 * m) * w


class ClockSampler:
    """nvidia-smi clocks/throttle reasons sampled every 200 ms during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index):
        self.device_index = device_index
        self.proc = None
        self.path = None

    def __enter__(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.device_index}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        if not self.path or not os.path.exists(self.path):
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"]}
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in Path(self.path).read_text().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
            except ValueError:
                continue
            for name, flag in zip(names, parts[5:9]):
                if flag.lower() == "active":
                    reasons.add(name)
        os.unlink(self.path)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(smax) if smax else None, "reasons": sorted(reasons),
                "samples": len(sm)}


def shard_checksums(y, world, device):
    """Sum of each rank's projections (fp64), gathered on every rank in rank order."""
    import torch
    import torch.distributed as dist

    local = y.detach().double().sum().reshape(1)
    if world == 1:
        return [float(local.item())]
    parts = [torch.zeros_like(local) for _ in range(world)]
    dist.all_gather(parts, local)
    return [float(p.item()) for p in parts]


def measure_vjp_active(args, workload, cfg, batch, world, device, barrier, tdt):
    """The headline step with the CP tolerance loosened so samples are accepted and the
    implicit VJP runs its restarted GMRES (the reference's LinearSolverConfig defaults).

    At the headline's tolerance 1e-9 no sample is accepted within 2000 iterations, so
    the reference gates every gradient to zero without solving (bounds.py:133) and the
    adjoint kernel does almost no work.  This measurement times the same step where it
    does: samples/s, the forward and adjoint kernel times, the Arnoldi steps GMRES took
    (the kernel's own counters) and the adjoint's algorithmic HBM bytes
    sum_steps (4k + 6) W w + 20 (2n + m) w per linearised sample (k basis vectors at a
    step; W = 2n + m) against the measured copy peak.
    """
    import torch
    import torch.distributed as dist

    from purin_b200 import prepare_projection

    cfg = dataclasses.replace(cfg, tolerance=args.vjp_active_tolerance)
    layer = prepare_projection(workload.problem, method="chambolle-pock", config=cfg,
                               batch_size=batch, dtype=tdt, backend=str(device))
    layer.set_shard(int(os.environ.get("RANK", "0")) * batch, batch * world,
                    group=dist.group.WORLD if world > 1 else None)
    cand = torch.as_tensor(workload.candidates, dtype=tdt, device=device)
    theta = torch.as_tensor(workload.theta, dtype=tdt, device=device)
    targ = torch.as_tensor(workload.targets, dtype=tdt, device=device)
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=device)

    def step():
        x = cand.detach().requires_grad_(True)
        th = theta.detach().requires_grad_(True)
        y = layer(x, th)
        (0.5 * ((y - targ) ** 2).sum()).backward()

    for _ in range(args.warmup):
        step()
    barrier()
    timers, step_ms = [], []
    for _ in range(args.steps):
        flush.fill_(1.0)
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        layer.record_launches(timers)
        start.record()
        step()
        end.record()
        layer.record_launches(None)
        torch.cuda.synchronize(device)
        step_ms.append(start.elapsed_time(end))
    barrier()
    per_kernel = {}
    for name, s0, e0 in timers:
        per_kernel.setdefault(name, []).append(s0.elapsed_time(e0))
    fwd_ms = sum(per_kernel.get("forward", [0.0])) / args.steps
    adj_ms = sum(per_kernel.get("adjoint", [0.0])) / args.steps
    steps, vectors = layer._last_work
    status, _ = layer._last_linear
    with torch.no_grad():
        result = layer.solve(cand, theta)
    n = workload.problem.variable_size
    m = layer._m
    w = 8 if tdt == torch.float64 else 4
    W = 2 * n + m
    linearised = int(result.gradient_eligible.sum().item())
    local = torch.tensor([float(sum(step_ms) / len(step_ms)), fwd_ms, adj_ms], device=device,
                         dtype=torch.float64)
    totals = torch.tensor([float(steps.sum().item()), float(vectors.sum().item()),
                           float(linearised), float(result.iterations.sum().item())],
                          device=device, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(local, op=dist.ReduceOp.MAX)
        dist.all_reduce(totals, op=dist.ReduceOp.SUM)
    ms, fwd_ms, adj_ms = (float(v) for v in local.tolist())
    arnoldi, krylov, linearised_all, iters_all = (float(v) for v in totals.tolist())
    # Per rank, the adjoint launch processes its own shard: bytes per launch are the
    # job's bytes divided by the ranks (one launch per rank and step).
    vjp_bytes = ((4.0 * krylov + 6.0 * arnoldi) * W * w
                 + 20.0 * (2 * n + m) * w * linearised_all) / world
    fwd_bytes = algorithmic_bytes_forward(n, m, w, iters_all) / world
    hbm, peak_kind = peaks()
    adj_gbs = vjp_bytes / (adj_ms / 1000.0) / 1e9 if adj_ms > 0 else None
    return {
        "cp_tolerance": args.vjp_active_tolerance,
        "value": batch * world / (ms / 1000.0), "unit": "samples/s", "ms_per_step": ms,
        "kernel_ms": {"forward": fwd_ms, "adjoint": adj_ms},
        "gradient_eligible": f"{int(linearised_all)}/{batch * world}",
        "gmres_codes_rank0": {str(c): int((status == c).sum().item()) for c in (0, 1, 2)},
        "arnoldi_steps": int(arnoldi), "krylov_vectors": int(krylov),
        "adjoint_roofline": {
            "bound": "hbm", "kernel": "cp_adjoint_kernel", "achieved": adj_gbs, "peak": hbm,
            "unit": "GB/s", "frac": adj_gbs / hbm if adj_gbs else None,
            "peak_source": peak_kind, "algorithmic_bytes_per_launch": vjp_bytes,
            "launch_ms": adj_ms,
            "note": "sum over Arnoldi steps of (4k+6)*W*w (CGS2 with k basis vectors) + "
                    "20*(2n+m)*w power iteration per linearised sample",
        },
        "forward_algorithmic_gbs": fwd_bytes / (fwd_ms / 1000.0) / 1e9 if fwd_ms > 0 else None,
    }


def count_native_launches(step, device):
    """Kernels of this library (namespace purin) launched by one untimed step, from the profiler."""
    import torch
    from torch.profiler import ProfilerActivity, profile

    torch.cuda.synchronize(device)
    count = 0
    # The profiler's first capture in a process can come back without device
    # events; a step always launches this library's kernels, so retry.
    for _ in range(3):
        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            step()
            torch.cuda.synchronize(device)
        count = sum(1 for e in prof.events()
                    if e.device_type == torch.autograd.DeviceType.CUDA and "purin::" in e.name)
        if count:
            break
    return count


def _native_oracle(workload, threads):
    """The oracle with its CP loop in C++ on ``threads`` host threads (checker-only code)."""
    sys.path.insert(0, str(ROOT / "tests"))
    from helpers import OracleLayer  # noqa: E402  (test infrastructure, checker only)

    from oracle.cpu import sparse_cp_native

    layer = OracleLayer(workload.problem, workload.config, np.float64)
    layer.proj.cp_solver = lambda *a, **k: sparse_cp_native(*a, threads=threads, **k)
    return layer


def _oracle_step(layer, workload, sl, total):
    result, saved = layer.solve(workload.candidates[sl], workload.theta[sl],
                                offset=sl.start or 0, total=total)
    layer.proj.vjp(saved, result["y"] - workload.targets[sl])


def cpu_baseline_oracle(workload, samples):
    """Time the oracle (fwd with the C++ CP loop on every host core + NumPy VJP)."""
    cores = len(os.sched_getaffinity(0))
    layer = _native_oracle(workload, cores)
    samples = min(samples, workload.candidates.shape[0])
    t0 = time.perf_counter()
    _oracle_step(layer, workload, slice(0, samples), workload.candidates.shape[0])
    elapsed = time.perf_counter() - t0
    return {"value": samples / elapsed, "unit": "samples/s", "cores": cores, "kind": "port",
            "sample": f"{samples} samples of config 2 (fwd 2000 it + VJP) in {elapsed:.1f} s: "
                      f"the CP loop restated in C++ (OpenMP, {cores} threads), presolve, "
                      "post-processing and VJP in the NumPy restatement"}


def run_reference(args):
    """``--impl reference``: the CPU restatement of the reference path on the host cores."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from purin_b200.workloads import make_workload

    cores = len(os.sched_getaffinity(0))
    per_step = 8 * cores
    workload = make_workload(CONFIG_INDEX, per_step)
    layer = _native_oracle(workload, cores)
    times = []
    for step in range(args.warmup + args.steps):
        t0 = time.perf_counter()
        _oracle_step(layer, workload, slice(0, per_step), per_step)
        if step >= args.warmup:
            times.append(time.perf_counter() - t0)
    ms = 1000.0 * statistics.mean(times)
    value = per_step / (ms / 1000.0)
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "samples/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f64",
        "data": "synthetic (seeded generator of benchmark configuration 2)",
        "config": {"workload": "config2: fp64 n=2048 me=512 mi=1024 8nnz/row, 2000 it, fwd+VJP",
                   "samples_per_step": per_step},
        "cpu_baseline": {"value": value, "unit": "samples/s", "cores": cores, "kind": "port",
                         "sample": f"{per_step} samples per step: CP loop in C++ (OpenMP, "
                                   f"{cores} threads), NumPy presolve, post-processing and VJP"},
        "e2e": {"value": value, "unit": "samples/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "note": "JAX is not installed on this host; the reference's own CPU path cannot run. "
                "This arm times the CPU restatement of that path (oracle/).",
    }
    print(json.dumps(line), flush=True)


QP_METRIC = "QP samples/sec at fixed iters (fwd+VJP)"


def cpu_baseline_qp(samples):
    """The NumPy diagonal-QP oracle (fwd 2000 iterations + VJP) on a bounded sample."""
    sys.path.insert(0, str(ROOT / "tests"))
    from helpers import oracle_config  # noqa: E402  (test infrastructure, checker only)
    from oracle.diagonal_qp import OracleDiagonalQP  # noqa: E402
    from purin_b200 import ChambollePockConfig
    from purin_b200.workloads import qp_workload

    structure, q, c, values, rhs, lower, upper, targets = qp_workload(samples)
    qp = OracleDiagonalQP(structure.variable_size, structure.equality_rows,
                          structure.inequality_rows,
                          oracle_config(ChambollePockConfig(max_iterations=2000)))
    b = q.shape[0]
    data = (q, c, np.broadcast_to(values, (b,) + values.shape[1:]), rhs,
            np.broadcast_to(lower, q.shape), np.broadcast_to(upper, q.shape))
    t0 = time.perf_counter()
    result, saved = qp.solve(data)
    qp.vjp(saved["out"], saved["data"], result["y"] - targets)
    elapsed = time.perf_counter() - t0
    return {"value": samples / elapsed, "unit": "samples/s", "cores": 1, "kind": "port",
            "sample": f"{samples} samples of the QP workload (fwd 2000 it + VJP) in "
                      f"{elapsed:.1f} s: the NumPy diagonal-QP restatement (oracle/)"}


def main_qp(args, world, rank, local_rank, device, barrier):
    """``--problem qp``: configuration 2's structure as a PreparedDiagonalQP."""
    import torch
    import torch.distributed as dist

    from purin_b200 import ChambollePockConfig
    from purin_b200.diagonal_qp import QPData
    from purin_b200.workloads import qp_workload

    batch = args.batch or DEFAULT_BATCH[CONFIG_INDEX]
    total = batch * world
    # Every rank holds the same structure and its own slice of one global batch.
    structure, q, c, values, rhs, lower, upper, targets = qp_workload(batch, offset=rank * batch)
    cfg = ChambollePockConfig(max_iterations=2000)
    if args.cp_tolerance is not None:
        cfg = dataclasses.replace(cfg, tolerance=args.cp_tolerance)
    solver = structure.prepare(batch_size=batch, config=cfg, dtype=torch.float64,
                               backend=str(device))
    solver.set_shard(rank * batch, total)
    n, m = q.shape[1], rhs.shape[1]
    dev = lambda a: torch.as_tensor(np.ascontiguousarray(a), dtype=torch.float64, device=device)
    q_d, c_d, rhs_d, t_d = dev(q), dev(c), dev(rhs), dev(targets)
    vals_d, lo_d, up_d = dev(values), dev(lower)[None], dev(upper)[None]
    if args.qp_values == "per-sample":
        vals_d = vals_d.expand(batch, -1, -1).contiguous()
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=device)

    def step(q_, c_, rhs_, t_):
        # The constraint matrix and the bounds are shared by the batch (stride-0 views).
        leaves = [x.detach().requires_grad_(True) for x in (q_, c_, vals_d, rhs_, lo_d, up_d)]
        values = (leaves[2].expand(batch, -1, -1) if vals_d.shape[0] == 1
                  else leaves[2])
        data = QPData(leaves[0], leaves[1], values, leaves[3],
                      leaves[4].expand(batch, -1), leaves[5].expand(batch, -1))
        res = solver.solve(data)
        loss = 0.5 * ((res.y - t_) ** 2).sum()
        loss.backward()
        return loss, leaves

    for _ in range(args.warmup):
        step(q_d, c_d, rhs_d, t_d)
    barrier()
    timers, step_ms = [], []
    with ClockSampler(local_rank) as clocks:
        barrier()
        for _ in range(args.steps):
            flush.fill_(1.0)
            start = torch.cuda.Event(enable_timing=True)
            end = torch.cuda.Event(enable_timing=True)
            solver.record_launches(timers)
            start.record()
            step(q_d, c_d, rhs_d, t_d)
            end.record()
            solver.record_launches(None)
            torch.cuda.synchronize(device)
            step_ms.append(start.elapsed_time(end))
        barrier()
    clock_info = clocks.summary()

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    ms = max_over_ranks(float(sum(step_ms) / len(step_ms)))
    per_kernel = {}
    for name, s0, e0 in timers:
        per_kernel.setdefault(name, []).append(s0.elapsed_time(e0))
    per_step = lambda name: (sum(per_kernel[name]) / args.steps if name in per_kernel
                             else float("nan"))
    fwd_ms, adj_ms = per_step("forward"), per_step("adjoint")
    launches = count_native_launches(lambda: step(q_d, c_d, rhs_d, t_d), device) * args.steps
    with torch.no_grad():
        res = solver.solve(QPData(q_d, c_d, vals_d.expand(batch, -1, -1) if vals_d.shape[0] == 1
                                  else vals_d, rhs_d,
                                  lo_d.expand(batch, -1), up_d.expand(batch, -1)))
    iters_total = int(res.iterations.sum().item())
    eligible = int(res.gradient_eligible.sum().item())
    # (6n + 3m) * 8 B per sample-iteration: read y, ybar, q, c, lambda, rhs; write
    # y, ybar, lambda (the shared constraint values are amortised, counted 0).
    fwd_bytes = float(iters_total) * (6 * n + 3 * m) * 8
    hbm, peak_kind = peaks()
    achieved = fwd_bytes / (fwd_ms / 1000.0) / 1e9

    # End to end: q, c, rhs and targets from pinned host memory; loss and the
    # gradients w.r.t. q, c and rhs back to pinned host memory.
    pin = lambda a: torch.as_tensor(np.ascontiguousarray(a), dtype=torch.float64).pin_memory()
    q_h, c_h, rhs_h, t_h = pin(q), pin(c), pin(rhs), pin(targets)
    gq_h, gc_h, grhs_h = (torch.empty_like(x).pin_memory() for x in (q_h, c_h, rhs_h))
    loss_h = torch.empty((), dtype=torch.float64).pin_memory()

    def step_e2e():
        to = lambda x: x.to(device, non_blocking=True)
        loss, leaves = step(to(q_h), to(c_h), to(rhs_h), to(t_h))
        gq_h.copy_(leaves[0].grad, non_blocking=True)
        gc_h.copy_(leaves[1].grad, non_blocking=True)
        grhs_h.copy_(leaves[3].grad, non_blocking=True)
        loss_h.copy_(loss.detach(), non_blocking=True)

    for _ in range(max(1, args.warmup)):
        step_e2e()
    barrier()
    e2e_ms = []
    for _ in range(args.steps):
        flush.fill_(1.0)
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        start.record()
        step_e2e()
        end.record()
        torch.cuda.synchronize(device)
        e2e_ms.append(start.elapsed_time(end))
    barrier()
    e2e = max_over_ranks(float(sum(e2e_ms) / len(e2e_ms)))
    h2d = (q_h.numel() + c_h.numel() + rhs_h.numel() + t_h.numel()) * 8
    d2h = (gq_h.numel() + gc_h.numel() + grhs_h.numel() + 1) * 8
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline_qp(args.cpu_samples or 8)
    if rank == 0:
        line = {
            "metric": QP_METRIC, "value": total / (ms / 1000.0), "unit": "samples/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f64",
            "data": "synthetic (configuration 2's seeded structure as a diagonal QP; no dataset)",
            "config": {
                "workload": "qp: PreparedDiagonalQP, fp64, n=2048, me=512, mi=1024, 8 nnz/row "
                            f"(values {'shared by the batch' if args.qp_values == 'shared' else 'per sample'}"
                            "), per-sample q~U(0.5,2), c=-q*candidate, "
                            "rhs; bounds shared; 2000 fixed-step CP iterations (tolerance "
                            f"{cfg.tolerance:g} stopping test kept); loss 0.5||y-t||^2, "
                            "gradients w.r.t. q, c, values, rhs, lower, upper",
                "samples_per_gpu": batch, "global_batch": total,
                "l2": "flushed between timed steps (256 MB write outside the step events)",
                "gradient_eligible": f"{eligible}/{batch} on rank 0",
            },
            "roofline": {
                "bound": "hbm", "kernel": "cp_forward_kernel<kQP>", "achieved": achieved,
                "peak": hbm, "unit": "GB/s", "frac": achieved / hbm, "traffic": None,
                "peak_source": peak_kind, "algorithmic_bytes_per_launch": fwd_bytes,
                "launch_ms": fwd_ms,
                "note": "(6n+3m)*8 B per sample-iteration x executed iterations",
            },
            "kernel_ms": {"forward": fwd_ms, "adjoint": adj_ms},
            "gpu_launches": launches,
            "e2e": {"value": total / (e2e / 1000.0), "unit": "samples/s",
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": e2e},
            "clocks": clock_info,
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


DENSE_METRIC = "dense QP samples/sec at fixed iters (fwd+VJP)"
DENSE_ITERATIONS = 2000


def cpu_baseline_dense(samples):
    """The NumPy dense-adapter oracle (fwd 2000 iterations + VJP) on a bounded sample."""
    from oracle.dense import OracleDense  # noqa: E402  (test infrastructure, checker only)
    from purin_b200.workloads import dense_workload

    q, c, A, b, C, d, lower, upper, targets = dense_workload(samples)
    oracle = OracleDense(q.shape[1], A.shape[1], C.shape[1], max_iterations=DENSE_ITERATIONS,
                         tolerance=1e-9)
    t0 = time.perf_counter()
    out = oracle.run(q, c, A, b, C, d, lower, upper)
    oracle.vjp(out, q, c, A, b, C, d, lower, upper, out.y - targets)
    elapsed = time.perf_counter() - t0
    return {"value": samples / elapsed, "unit": "samples/s", "cores": 1, "kind": "port",
            "sample": f"{samples} samples of the dense workload (fwd {DENSE_ITERATIONS} it + "
                      f"VJP) in {elapsed:.1f} s: the NumPy dense-adapter restatement (oracle/)"}


def main_dense(args, world, rank, local_rank, device, barrier):
    """``--problem dense``: ``solve_dense_implicit`` on per-sample dense matrices."""
    import torch
    import torch.distributed as dist

    from purin_b200 import dense_layer
    from purin_b200.workloads import dense_workload

    batch = args.batch or 16384
    total = batch * world
    problem = dense_workload(batch, offset=rank * batch)  # this rank's slice of the batch
    q, c, A, b, C, d, lower, upper, targets = problem
    n, me, mi = q.shape[1], A.shape[1], C.shape[1]
    m = me + mi
    tol = args.cp_tolerance if args.cp_tolerance is not None else 1e-9
    dev = lambda a: torch.as_tensor(np.ascontiguousarray(a), dtype=torch.float64, device=device)
    inputs_d = [dev(x) for x in problem]
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=device)
    solver_box = {}

    def step(inputs):
        leaves = [x.detach().requires_grad_(True) for x in inputs[:8]]
        y, _, _ = dense_layer.solve_dense_implicit(
            *leaves, tolerance=tol, max_iterations=DENSE_ITERATIONS, backend=str(device))
        loss = 0.5 * ((y - inputs[8]) ** 2).sum()
        loss.backward()
        return loss, leaves

    for _ in range(args.warmup):
        step(inputs_d)
    barrier()
    solver_box["solver"] = next(iter(dense_layer._SOLVERS.values()))  # the one solve shape
    timers, step_ms, work = [], [], []
    with ClockSampler(local_rank) as clocks:
        barrier()
        for _ in range(args.steps):
            flush.fill_(1.0)
            start = torch.cuda.Event(enable_timing=True)
            end = torch.cuda.Event(enable_timing=True)
            dense_layer.record_launches(timers)
            start.record()
            step(inputs_d)
            end.record()
            dense_layer.record_launches(None)
            torch.cuda.synchronize(device)
            step_ms.append(start.elapsed_time(end))
            work.append(sum(solver_box["solver"].last_work))
        barrier()
    clock_info = clocks.summary()

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    ms = max_over_ranks(float(sum(step_ms) / len(step_ms)))
    per_kernel = {}
    for name, s0, e0 in timers:
        per_kernel.setdefault(name, []).append(s0.elapsed_time(e0))
    per_step = lambda name: (sum(per_kernel[name]) / args.steps if name in per_kernel
                             else float("nan"))
    fwd_ms, adj_ms = per_step("forward"), per_step("adjoint")
    launches = count_native_launches(lambda: step(inputs_d), device) * args.steps
    # Per sample-iteration: read y, ybar, q, c, lambda, rhs and write y, ybar,
    # lambda ((6n + 3m) * 8 B), and read the sample's own row values twice (row
    # and column order: 2 * m * n * 8 B).
    bytes_per_iteration = ((6 * n + 3 * m) + 2 * m * n) * 8
    fwd_bytes = float(sum(work) / len(work)) * bytes_per_iteration
    hbm, peak_kind = peaks()
    achieved = fwd_bytes / (fwd_ms / 1000.0) / 1e9

    # End to end: every input from pinned host memory (the per-sample matrices
    # included); the loss and the gradients w.r.t. c and A back to pinned host memory.
    pin = lambda a: torch.as_tensor(np.ascontiguousarray(a), dtype=torch.float64).pin_memory()
    inputs_h = [pin(x) for x in problem]
    gc_h, gA_h = torch.empty_like(inputs_h[1]).pin_memory(), torch.empty_like(inputs_h[2]).pin_memory()
    loss_h = torch.empty((), dtype=torch.float64).pin_memory()

    def step_e2e():
        loss, leaves = step([x.to(device, non_blocking=True) for x in inputs_h])
        gc_h.copy_(leaves[1].grad, non_blocking=True)
        gA_h.copy_(leaves[2].grad, non_blocking=True)
        loss_h.copy_(loss.detach(), non_blocking=True)

    for _ in range(max(1, args.warmup)):
        step_e2e()
    barrier()
    e2e_ms = []
    for _ in range(args.steps):
        flush.fill_(1.0)
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        start.record()
        step_e2e()
        end.record()
        torch.cuda.synchronize(device)
        e2e_ms.append(start.elapsed_time(end))
    barrier()
    e2e = max_over_ranks(float(sum(e2e_ms) / len(e2e_ms)))
    h2d = sum(x.numel() for x in inputs_h) * 8
    d2h = (gc_h.numel() + gA_h.numel() + 1) * 8
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline_dense(args.cpu_samples or 64)
    if rank == 0:
        line = {
            "metric": DENSE_METRIC, "value": total / (ms / 1000.0), "unit": "samples/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f64",
            "data": "synthetic (seeded dense QPs; no dataset)",
            "config": {
                "workload": f"dense: solve_dense_implicit, fp64, n={n}, me={me}, mi={mi}, "
                            "dense per-sample A and C ~ N(0,1), q~U(0.5,2), c=-q*candidate, "
                            f"per-sample bounds; at most {DENSE_ITERATIONS} fixed-step CP "
                            f"iterations (tolerance {tol:g}, batch-wide trip count); loss "
                            "0.5||y-t||^2, gradients w.r.t. c, A, b, C, d, lower, upper",
                "samples_per_gpu": batch, "global_batch": total,
                "l2": "inputs larger than L2 (per-sample matrices) and flushed between "
                      "timed steps (256 MB write outside the step events)",
                "sample_iterations_per_step": float(sum(work) / len(work)),
            },
            "roofline": {
                "bound": "hbm", "kernel": "cp_forward_kernel<kQP> (per-sample values)",
                "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                "traffic": None, "peak_source": peak_kind,
                "algorithmic_bytes_per_launch": fwd_bytes, "launch_ms": fwd_ms,
                "note": "((6n+3m) + 2mn)*8 B per executed sample-iteration",
            },
            "kernel_ms": {"forward": fwd_ms, "adjoint": adj_ms},
            "gpu_launches": launches,
            "e2e": {"value": total / (e2e / 1000.0), "unit": "samples/s",
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": e2e},
            "clocks": clock_info,
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


ADMM_METRIC = "ADMM samples/sec to tolerance (fwd+VJP)"


def cpu_baseline_admm(samples, batch_cfg):
    """The NumPy ADMM oracle (forward + VJP) on a bounded sample of the ADMM workload."""
    sys.path.insert(0, str(ROOT / "tests"))
    from helpers import OracleADMMLayer  # noqa: E402  (test infrastructure, checker only)
    from purin_b200.workloads import make_workload

    w = make_workload(0, samples)
    layer = OracleADMMLayer(w.problem, batch_cfg)
    t0 = time.perf_counter()
    result, saved = layer.solve(w.candidates, w.theta)
    layer.proj.vjp(saved, result["y"] - w.targets)
    elapsed = time.perf_counter() - t0
    return {"value": samples / elapsed, "unit": "samples/s", "cores": 1, "kind": "port",
            "sample": f"{samples} samples of the ADMM workload (fwd to tolerance + VJP) in "
                      f"{elapsed:.1f} s: the NumPy ADMM restatement (oracle/admm.py)"}


def main_admm(args, world, rank, local_rank, device, barrier):
    """``--problem admm``: configuration 0's structure through ``method="admm"``."""
    import torch
    import torch.distributed as dist

    from purin_b200 import ADMMConfig, ImplicitGradientConfig, prepare_projection
    from purin_b200.workloads import make_workload

    batch = args.batch or 2048
    total = batch * world
    w = make_workload(0, batch, offset=rank * batch)
    tol = args.cp_tolerance if args.cp_tolerance is not None else 1e-9
    cfg = ADMMConfig(tolerance=tol, implicit_gradient=ImplicitGradientConfig(
        differentiate_problem_parameters=True))
    layer = prepare_projection(w.problem, method="admm", config=cfg, batch_size=batch,
                               backend=str(device))
    layer.set_shard(rank * batch, total, group=dist.group.WORLD if world > 1 else None)
    cand = torch.as_tensor(w.candidates, device=device)
    theta = torch.as_tensor(w.theta, device=device)
    targ = torch.as_tensor(w.targets, device=device)
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=device)

    def step(c_, t_, g_):
        x = c_.detach().requires_grad_(True)
        th = t_.detach().requires_grad_(True)
        y = layer(x, th)
        loss = 0.5 * ((y - g_) ** 2).sum()
        loss.backward()
        return loss, x, th

    for _ in range(args.warmup):
        step(cand, theta, targ)
    barrier()
    timers, step_ms = [], []
    with ClockSampler(local_rank) as clocks:
        barrier()
        for _ in range(args.steps):
            flush.fill_(1.0)
            start = torch.cuda.Event(enable_timing=True)
            end = torch.cuda.Event(enable_timing=True)
            layer.record_launches(timers)
            start.record()
            step(cand, theta, targ)
            end.record()
            layer.record_launches(None)
            torch.cuda.synchronize(device)
            step_ms.append(start.elapsed_time(end))
        barrier()
    clock_info = clocks.summary()

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    ms = max_over_ranks(float(sum(step_ms) / len(step_ms)))
    per_kernel = {}
    for name, s0, e0 in timers:
        per_kernel.setdefault(name, []).append(s0.elapsed_time(e0))
    per_step = lambda name: (sum(per_kernel[name]) / args.steps if name in per_kernel
                             else float("nan"))
    fwd_ms, adj_ms = per_step("forward"), per_step("adjoint")
    launches = count_native_launches(lambda: step(cand, theta, targ), device) * args.steps
    with torch.no_grad():
        result = layer.solve(cand, theta)
    iterations = result.iterations.double()
    eligible = int(result.gradient_eligible.sum().item())
    pin = lambda a: torch.as_tensor(np.ascontiguousarray(a)).pin_memory()
    cand_h, theta_h, targ_h = pin(w.candidates), pin(w.theta), pin(w.targets)
    gx_h = torch.empty_like(cand_h).pin_memory()
    gth_h = torch.empty_like(theta_h).pin_memory()
    loss_h = torch.empty((), dtype=torch.float64).pin_memory()

    def step_e2e():
        to = lambda x: x.to(device, non_blocking=True)
        loss, x, th = step(to(cand_h), to(theta_h), to(targ_h))
        gx_h.copy_(x.grad, non_blocking=True)
        gth_h.copy_(th.grad, non_blocking=True)
        loss_h.copy_(loss.detach(), non_blocking=True)

    for _ in range(max(1, args.warmup)):
        step_e2e()
    barrier()
    e2e_ms = []
    for _ in range(args.steps):
        flush.fill_(1.0)
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        start.record()
        step_e2e()
        end.record()
        torch.cuda.synchronize(device)
        e2e_ms.append(start.elapsed_time(end))
    barrier()
    e2e = max_over_ranks(float(sum(e2e_ms) / len(e2e_ms)))
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline_admm(args.cpu_samples or 4, cfg)
    if rank == 0:
        line = {
            "metric": ADMM_METRIC, "value": total / (ms / 1000.0), "unit": "samples/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f64",
            "data": "synthetic (seeded generator of benchmark configuration 0; no dataset)",
            "config": {
                "workload": "admm: configuration 0's structure (fp64, n=64, 32 equality and 32 "
                            "inequality rows of 4 nnz, |y| <= 1 as 128 singleton rows, paired "
                            f"into two-sided rows), ADMMConfig(tolerance={tol:g}) defaults "
                            "(rho 1, alpha 1.6, Jacobi PCG 32 iterations, checks every 25), "
                            "loss 0.5||y-t||^2, gradients w.r.t. candidates and parameters",
                "samples_per_gpu": batch, "global_batch": total,
                "l2": "flushed between timed steps (256 MB write outside the step events)",
                "gradient_eligible": f"{eligible}/{batch} on rank 0",
                "admm_iterations_mean": float(iterations.mean().item()),
                "admm_iterations_max": int(iterations.max().item()),
            },
            "roofline": {
                "bound": "latency", "kernel": "admm_forward_kernel", "achieved": None,
                "peak": None, "unit": None, "frac": None, "traffic": None,
                "note": "one CTA per sample with its vectors in shared memory; each ADMM "
                        "iteration runs up to 32 dependent PCG iterations of two sparse "
                        "products and three block reductions, so the kernel is bound by "
                        "barrier and shared-memory latency, not by a memory or math roof",
            },
            "kernel_ms": {"forward": fwd_ms, "adjoint": adj_ms},
            "gpu_launches": launches,
            "e2e": {"value": total / (e2e / 1000.0), "unit": "samples/s",
                    "h2d_bytes_per_step": (cand_h.numel() + theta_h.numel() + targ_h.numel()) * 8,
                    "d2h_bytes_per_step": (gx_h.numel() + gth_h.numel() + 1) * 8,
                    "ms_per_step": e2e},
            "clocks": clock_info,
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def main():
    args = parse_args()
    if args.impl == "reference":
        run_reference(args)
        return
    import torch
    import torch.distributed as dist

    from purin_b200 import prepare_projection
    from purin_b200.workloads import make_workload

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=device)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(device)

    if args.problem == "qp":
        main_qp(args, world, rank, local_rank, device, barrier)
        return
    if args.problem == "dense":
        main_dense(args, world, rank, local_rank, device, barrier)
        return
    if args.problem == "admm":
        main_admm(args, world, rank, local_rank, device, barrier)
        return

    index = args.config
    vjp = (args.mode or ("fwd+vjp" if index == CONFIG_INDEX else "fwd")) == "fwd+vjp"
    batch = args.batch or DEFAULT_BATCH[index]
    total = batch * world
    # Every rank builds the same seed-0 structure and takes its slice
    # [rank * batch, (rank + 1) * batch) of one global batch of world * batch samples.
    fp32 = (args.dtype or ("float32" if index in (3, 4) else "float64")) == "float32"
    workload = make_workload(index, batch, dtype=args.dtype, offset=rank * batch,
                             array_dtype=np.float32 if fp32 else np.float64)
    tdt = torch.float64 if workload.dtype == "float64" else torch.float32
    cfg = workload.config
    if workload.weights is not None:  # configuration 4: WeightedDistance
        cfg = dataclasses.replace(cfg, metric_diagonal=tuple(float(v) for v in workload.weights))
    if args.cp_tolerance is not None:
        cfg = dataclasses.replace(cfg, tolerance=args.cp_tolerance)
    if args.diagonal_preconditioning:
        cfg = dataclasses.replace(cfg, diagonal_preconditioning=True)
    layer = prepare_projection(workload.problem, method="chambolle-pock", config=cfg,
                               batch_size=batch, dtype=tdt, backend=str(device))
    # Ranks > 1 share the adjoint GMRES budget of the whole batch, as the
    # reference's single batched solve does (one small NCCL all-reduce per phase).
    layer.set_shard(rank * batch, total, group=dist.group.WORLD if world > 1 else None)
    n = workload.problem.variable_size
    m = layer._m
    w = 8 if tdt == torch.float64 else 4

    cand_d = torch.as_tensor(workload.candidates, dtype=tdt, device=device)
    theta_d = torch.as_tensor(workload.theta, dtype=tdt, device=device)
    targets = workload.targets
    targ_d = torch.as_tensor(targets, dtype=tdt, device=device)
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=device)

    def step_device(timers=None):
        if not vjp:
            with torch.no_grad():
                return layer(cand_d, theta_d)
        x = cand_d.detach().requires_grad_(True)
        th = theta_d.detach().requires_grad_(True)
        y = layer(x, th)
        loss = 0.5 * ((y - targ_d) ** 2).sum()
        loss.backward()
        return loss, x.grad, th.grad

    # ---- device-resident timing ------------------------------------------------
    for _ in range(args.warmup):
        step_device()
    barrier()
    timers = []
    step_ms = []
    with ClockSampler(local_rank) as clocks:
        barrier()
        for _ in range(args.steps):
            flush.fill_(1.0)
            start = torch.cuda.Event(enable_timing=True)
            end = torch.cuda.Event(enable_timing=True)
            layer.record_launches(timers)
            start.record()
            step_device()
            end.record()
            layer.record_launches(None)
            torch.cuda.synchronize(device)
            step_ms.append(start.elapsed_time(end))
        barrier()
    clock_info = clocks.summary()
    ms_local = float(sum(step_ms) / len(step_ms))
    ms = ms_local
    if world > 1:
        t = torch.tensor([ms_local], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    value = total / (ms / 1000.0)

    # Per-kernel event times inside the timed steps.
    per_kernel = {}
    for name, s, e in timers:
        per_kernel.setdefault(name, []).append(s.elapsed_time(e))
    launches = count_native_launches(step_device, device) * args.steps
    # Dominant kernel and its algorithmic bytes.
    with torch.no_grad():
        result = layer.solve(cand_d, theta_d)
    iters_total = int(result.iterations.sum().item())
    checksums = shard_checksums(result.y, world, device)
    # Per step: the staged adjoint of a multi-rank run records one entry per phase.
    per_step = lambda name: (sum(per_kernel[name]) / args.steps if name in per_kernel
                             else float("nan"))
    fwd_ms = per_step("forward")
    adj_ms = per_step("adjoint")
    post_ms = per_step("postprocess")
    fwd_bytes = algorithmic_bytes_forward(n, m, w, iters_total)
    hbm, peak_kind = peaks()
    achieved = fwd_bytes / (fwd_ms / 1000.0) / 1e9
    eligible = int(result.gradient_eligible.sum().item())

    # ---- end-to-end through the public API from pinned host buffers ---------------
    cand_h = torch.as_tensor(workload.candidates, dtype=tdt).pin_memory()
    theta_h = torch.as_tensor(workload.theta, dtype=tdt).pin_memory()
    targ_h = torch.as_tensor(targets, dtype=tdt).pin_memory()
    gx_h = torch.empty_like(cand_h).pin_memory()
    gth_h = torch.empty_like(theta_h).pin_memory()
    loss_h = torch.empty((), dtype=tdt).pin_memory()

    def step_e2e():
        if not vjp:  # forward only: candidates and parameters in, projections out
            with torch.no_grad():
                y = layer(cand_h.to(device, non_blocking=True),
                          theta_h.to(device, non_blocking=True))
                gx_h.copy_(y, non_blocking=True)
            return
        x = cand_h.to(device, non_blocking=True).requires_grad_(True)
        th = theta_h.to(device, non_blocking=True).requires_grad_(True)
        t = targ_h.to(device, non_blocking=True)
        y = layer(x, th)
        loss = 0.5 * ((y - t) ** 2).sum()
        loss.backward()
        gx_h.copy_(x.grad, non_blocking=True)
        if th.grad is not None:  # configurations that differentiate the parameters
            gth_h.copy_(th.grad, non_blocking=True)
        loss_h.copy_(loss.detach(), non_blocking=True)

    for _ in range(max(1, args.warmup)):
        step_e2e()
    barrier()
    e2e_ms = []
    for _ in range(args.steps):
        flush.fill_(1.0)
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        start.record()
        step_e2e()
        end.record()
        torch.cuda.synchronize(device)
        e2e_ms.append(start.elapsed_time(end))
    barrier()
    e2e_local = float(sum(e2e_ms) / len(e2e_ms))
    e2e = e2e_local
    if world > 1:
        t = torch.tensor([e2e_local], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e = float(t.item())
    if vjp:
        h2d = (cand_h.numel() + theta_h.numel() + targ_h.numel()) * w
        theta_grad = cfg.implicit_gradient.differentiate_problem_parameters
        d2h = (gx_h.numel() + (gth_h.numel() if theta_grad else 0) + 1) * w
    else:
        h2d = (cand_h.numel() + theta_h.numel()) * w
        d2h = gx_h.numel() * w

    headline = index == CONFIG_INDEX and vjp and tdt == torch.float64
    vjp_active = None
    if headline and args.vjp_active_tolerance > 0 and args.cp_tolerance is None:
        vjp_active = measure_vjp_active(args, workload, cfg, batch, world, device, barrier, tdt)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline and headline:
        samples = args.cpu_samples or 48 * len(os.sched_getaffinity(0))
        cpu = cpu_baseline_oracle(make_workload(CONFIG_INDEX, samples), samples)

    if rank == 0:
        line = {
            "metric": METRIC if vjp else METRIC.replace("(fwd+VJP)", "(fwd)"), "value": value,
            "unit": "samples/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f64" if w == 8 else "f32",
            "data": f"synthetic (seeded generator of benchmark configuration {index}; no dataset)",
            "config": {
                "workload": WORKLOADS[index].replace(
                    "config1: ", f"config1: {'fp64' if w == 8 else 'fp32'}, ").replace(
                    "config4: ", f"config4: {'fp64' if w == 8 else 'fp32'}, ")
                + f" (tolerance {cfg.tolerance:g} stopping test kept), "
                + ("fwd + implicit VJP w.r.t. candidates and parameters" if vjp else "forward"),
                "samples_per_gpu": batch, "global_batch": total,
                "l2": "flushed between timed steps (256 MB write outside the step events)",
                "gradient_eligible": f"{eligible}/{batch} on rank 0",
            },
            "roofline": {
                "bound": "hbm", "kernel": "cp_forward_kernel", "achieved": achieved,
                "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                "traffic": FORWARD_DRAM_BYTES_PER_SAMPLE * batch if index == CONFIG_INDEX
                else None,
                "traffic_source": ("ncu dram__bytes_read.sum + dram__bytes_write.sum of one launch "
                                   "at 592 samples, scaled by samples per launch")
                if index == CONFIG_INDEX else None,
                "peak_source": peak_kind,
                "algorithmic_bytes_per_launch": fwd_bytes,
                "launch_ms": fwd_ms,
                "note": "(5n+3m)*8 B per sample-iteration x executed iterations; the iterates "
                        "stay in shared memory, so the HBM stream is the reference layout's "
                        "traffic, not this kernel's: HBM is not what bounds it (see "
                        "roofline_onchip)",
            },
            # What does bound the forward kernel: its iterates live in shared memory and
            # the structure in L2/L1, so its limiter is the L1 data pipe (shared-memory
            # gathers plus structure loads), from the ncu capture of configuration 2.
            "roofline_onchip": {
                "bound": "l1", "kernel": "cp_forward_kernel",
                "metric": "l1tex__data_pipe_lsu_wavefronts (of peak)",
                "frac": FORWARD_L1_PIPE_FRAC if index == CONFIG_INDEX else None,
                "source": "profiles/cp_forward_config2_b592.md (ncu --set full, 592 samples)"
                if index == CONFIG_INDEX else None,
                "bank_conflict_share": FORWARD_BANK_CONFLICT_SHARE if index == CONFIG_INDEX
                else None,
            },
            "kernel_ms": {"forward": fwd_ms, "adjoint": adj_ms, "postprocess": post_ms},
            "shard_checksums": checksums,
            "vjp_active": vjp_active,
            "gpu_launches": launches,
            "e2e": {"value": total / (e2e / 1000.0), "unit": "samples/s",
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": e2e},
            "clocks": clock_info,
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
