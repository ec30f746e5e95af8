"""The forward's optional global stopping rule (``purin_b200.lockstep.global_stop_forward``).

Host logic on the CPU: a stand-in segment solver whose samples are accepted at
known iterations (and freeze there, as the reference's loop does,
``kernels.py:266-271``) checks that the segmented loop reproduces one
uninterrupted run exactly, and that two gloo ranks stop at the same segment,
the first one after which no sample of either rank is still running
(``kernels.py:238-240``).  The kernels themselves are checked on the GPU
(``tests/test_gpu_global_stop.py``).
"""

import os
import socket
from types import SimpleNamespace

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from purin_b200.lockstep import global_stop_forward

MAX_IT = 1000


def _fake_segment(accept_at):
    """A solver whose sample b is accepted at iteration accept_at[b] (or never, -1)."""
    accept = torch.as_tensor(accept_at, dtype=torch.int64)

    def segment(end, y, dual, ybar, start):
        batch = y.shape[0]
        it0 = torch.zeros(batch, dtype=torch.int64) if start is None else torch.clamp(
            start.to(torch.int64), max=end)
        hit = (accept > it0) & (accept <= end)
        count = torch.where(hit, accept, torch.full_like(accept, end))
        ran = (count - it0).to(y.dtype)
        new_y = y + ran[:, None]
        base_bar = y if ybar is None else ybar
        return SimpleNamespace(
            y=new_y, dual=dual - 0.5 * ran[:, None], ybar=base_bar + 2.0 * ran[:, None],
            iterations=count.to(torch.int32), residual=count.to(y.dtype) * 0.25,
            gap=count.to(y.dtype) * 0.125, converged=hit.to(torch.uint8))

    return segment


def _run(accept_at, interval, group=None):
    batch = len(accept_at)
    y0 = torch.arange(batch * 3, dtype=torch.float64).reshape(batch, 3)
    d0 = torch.ones((batch, 2), dtype=torch.float64)
    return global_stop_forward(_fake_segment(accept_at), y0, d0, batch, MAX_IT, interval, group)


@pytest.mark.parametrize("interval", [1, 7, 100, 1000, 5000])
def test_segments_equal_one_uninterrupted_run(interval):
    accept_at = [3, 250, -1, 999, 1000, 100, 1]
    want = _run(accept_at, MAX_IT)
    got = _run(accept_at, interval)
    for w, g in zip(want[:6], got[:6]):
        assert torch.equal(w, g)
    assert got[6] == want[6] == MAX_IT  # a sample that never converges runs the budget


def test_stops_at_the_first_segment_end_with_nothing_running():
    accept_at = [3, 250, 120]
    y, dual, its, res, gap, conv, trip, segments = _run(accept_at, 100)
    assert trip == 250 and segments == 3  # stopped after the segment ending at 300
    assert its.tolist() == accept_at and conv.tolist() == [1, 1, 1]


def test_interval_must_be_positive():
    with pytest.raises(ValueError, match="positive"):
        _run([1], 0)


def _rank(rank, world, port, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    from datetime import timedelta

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=30))
    try:
        # Rank 0's samples are all accepted early; rank 1 holds a slow one.
        accept_at = [[5, 40], [30, 610]][rank]
        result = _run(accept_at, 100, dist.group.WORLD)
        alone = _run(accept_at, 100)
        np.save(out + f".{rank}.npy", np.array(
            [result[6], result[7], alone[6], alone[7]] + result[2].tolist()))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_two_ranks_share_the_trip_count_and_stop_together(tmp_path):
    out = str(tmp_path / "r")
    mp.spawn(_rank, args=(2, _free_port(), out), nprocs=2, join=True)
    r0, r1 = np.load(out + ".0.npy"), np.load(out + ".1.npy")
    # Both ranks: trip 610, 7 segments (stopping after the one ending at 700).
    assert r0[0] == r1[0] == 610 and r0[1] == r1[1] == 7
    # Alone, rank 0 would have stopped after its first segment with trip 40.
    assert r0[2] == 40 and r0[3] == 1
    assert r0[4:].tolist() == [5, 40] and r1[4:].tolist() == [30, 610]
