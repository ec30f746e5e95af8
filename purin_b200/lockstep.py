"""Batch-wide lockstep of the adjoint's restarted GMRES across shards of a batch.

The reference solves the implicit-differentiation systems of a whole batch
with ONE lockstep restarted GMRES (``_batched_restarted_gmres``,
``src/purin/solvers/primal_dual_interior_point/operators.py:919-1103``):

* a restart cycle runs Arnoldi steps while ANY sample of the batch is still
  active (``arnoldi_condition``, operators.py:943-955), so the cycle lasts as
  many steps as its slowest sample needs;
* those steps are charged to one budget, ``completed_iterations``
  (operators.py:1093), and the next cycle may take at most
  ``min(restart, max_iterations - completed_iterations)`` steps
  (operators.py:921-924);
* cycles continue while any sample's true residual is above its threshold
  (``cycle_condition``, operators.py:1099-1103).

When the batch is split into shards (one per GPU, or chunks on one GPU) each
shard must therefore learn, after every cycle, the longest cycle and whether
any sample anywhere is still active; otherwise a shard whose own samples
finish their cycles early is left a larger budget and can run a longer final
cycle than the unsharded batch would.  ``run`` drives shards through the
staged adjoint (``purin_cp_adjoint_stage``): it combines their two counters
with an elementwise max, locally over the shards of this process and, given a
process group, across ranks with one all-reduce (NCCL for CUDA tensors, gloo
for CPU tensors) per phase.  Every rank takes the same collective steps in the
same order, because each decision is made from the combined counters.
"""

from __future__ import annotations

from typing import Protocol, Sequence

import torch
import torch.distributed as dist


class Shard(Protocol):
    """One shard's staged adjoint; counters are two integers (a tensor or sequence)."""

    def prepare(self): ...  # -> (0, samples above their threshold)

    def cycle(self, completed: int): ...  # -> (Arnoldi steps, samples still above)

    def finish(self): ...  # -> the shard's outputs


def combine_max(counters: Sequence, group=None) -> tuple[int, int]:
    """Elementwise max of the shards' counters here and, with ``group``, on every rank."""
    acc = None
    for c in counters:
        t = torch.as_tensor(c)
        acc = t.clone() if acc is None else torch.maximum(acc, t.to(acc.device))
    if acc is None:
        raise ValueError("combine_max needs at least one shard")
    if group is not None:
        dist.all_reduce(acc, op=dist.ReduceOp.MAX, group=group)
    length, active = (int(v) for v in acc.tolist())
    return length, active


def run(shards: Sequence[Shard], max_iterations: int, group=None):
    """Run the shards' staged adjoints with the batch-wide GMRES budget.

    Returns ``(outputs, completed, cycles)``: each shard's ``finish()`` result,
    the Arnoldi steps charged to the shared budget, and the cycles run -- the
    same on every rank and the same as an unsharded run of the whole batch.
    """
    _, active = combine_max([s.prepare() for s in shards], group)
    completed = 0
    cycles = 0
    while completed < max_iterations and active > 0:
        length, active = combine_max([s.cycle(completed) for s in shards], group)
        if length <= 0:
            # An active sample always takes at least one step; a zero here means
            # no shard ran its cycle.  Every rank sees the same value and stops.
            raise RuntimeError("lockstep GMRES: an active cycle reported no Arnoldi steps")
        completed += length
        cycles += 1
    return [s.finish() for s in shards], completed, cycles


# ---- the forward's optional global stopping rule -----------------------------------

class SegmentOutput(Protocol):
    """What one forward segment returns (tensors with the batch as leading dimension)."""

    y: torch.Tensor
    dual: torch.Tensor
    ybar: torch.Tensor
    iterations: torch.Tensor  # int32, absolute counts
    residual: torch.Tensor
    gap: torch.Tensor
    converged: torch.Tensor   # uint8, accepted within this segment


def global_stop_forward(segment, y0, dual0, batch: int, max_iterations: int, interval: int,
                        group=None):
    """The forward solve in segments of ``interval`` iterations with a batch-wide stop.

    The reference's loop runs while ``it < max_iterations and not all(done)``
    over the whole batch (``kernels.py:238-240``).  With the batch split across
    ranks, this driver makes that condition global: after every segment each
    rank counts its samples still running (not yet accepted, below the budget),
    the counts are summed over ``group`` (an all-reduce on the device, NCCL for
    CUDA tensors), and every rank stops at the first segment end where the sum
    is zero.  A sample freezes when it is accepted (``kernels.py:266-271``), so
    the outputs equal one uninterrupted solve bit for bit; the rule adds the
    batch's trip count, the same on every rank.

    ``segment(end, y, dual, ybar, start)`` continues every sample from its state
    (``ybar`` None and ``start`` None on the first segment) up to iteration
    ``end``; a sample whose ``start`` equals ``end`` takes no step.  Returns
    ``(y, dual, iterations, residual, gap, converged, trip, segments)``, where
    ``trip`` is the batch-wide trip count: the largest iteration count over the
    global batch.
    """
    if interval < 1:
        raise ValueError("the global stopping interval must be a positive number of iterations")
    y, dual, ybar, start = y0, dual0, None, None
    final = None
    done = None
    segments = 0
    end = 0
    while end < max_iterations:
        end = min(end + interval, max_iterations)
        out = segment(end, y, dual, ybar, start)
        segments += 1
        accepted = out.converged != 0
        if final is None:
            final = [out.y.clone(), out.dual.clone(), out.iterations.clone(),
                     out.residual.clone(), out.gap.clone(), out.converged.clone()]
            done = accepted.clone()
            fresh = torch.ones_like(accepted)
        else:
            fresh = ~done  # samples that ran in this segment
        # A sample's outputs are those of the segment it was accepted in, or of the
        # last segment; values of samples that did not run are kept.
        for k, v in enumerate((out.y, out.dual, out.iterations, out.residual, out.gap,
                               out.converged)):
            final[k] = torch.where(fresh.view(-1, *([1] * (v.dim() - 1))), v, final[k])
        done = done | accepted
        # The next segment continues the samples that ran in this one from their state.
        y = torch.where(fresh[:, None], out.y, y)
        dual = torch.where(fresh[:, None], out.dual, dual)
        ybar = out.ybar if ybar is None else torch.where(fresh[:, None], out.ybar, ybar)
        running = (~done) & (out.iterations < max_iterations)
        # Samples already accepted start (and stop) at the next segment's end.
        start = torch.where(done, torch.full_like(out.iterations, max_iterations),
                            out.iterations).to(torch.int32)
        active = running.sum().reshape(1).to(torch.int64)
        if group is not None:
            dist.all_reduce(active, op=dist.ReduceOp.SUM, group=group)
        if int(active.item()) == 0:
            break
    trip = final[2].max().reshape(1).to(torch.int64) if batch > 0 else torch.zeros(
        1, dtype=torch.int64)
    if group is not None:
        dist.all_reduce(trip, op=dist.ReduceOp.MAX, group=group)
    return (*final, int(trip.item()), segments)
