"""General positive diagonal QP layer on the sm_100a Chambolle--Pock kernels.

Mirrors ``src/purin/solvers/diagonal_qp.py`` (SOULS-TAMU/Purin 1.0.2):
``QPData``, ``QPStructure``, ``PreparedDiagonalQP.solve`` and ``dense_qp_data``,
with the same argument checks and messages.  Every ``QPData`` field -- q, c, the
row values, right-hand sides and bounds -- is differentiable: the solve is a
torch autograd op whose forward is ``purin_qp_forward`` (``sparse_cp`` with
per-sample q, c and warm starts, diagonal_qp.py:99-123) and whose backward is
``purin_qp_adjoint`` (implicit differentiation through GMRES with the dual
cotangent in the right-hand side, diagonal_qp.py:133-220).  Row scaling, the
tolerance and the diagnostics in original units (diagonal_qp.py:225-314) are
torch operations, so autograd chains through them as JAX does.

Differences: arrays are torch tensors on a CUDA device (``backend``), and
``prepare`` takes a torch dtype.
"""

from __future__ import annotations

import contextlib
from dataclasses import dataclass
from typing import NamedTuple

import numpy as np
import torch

from purin_b200 import _native, lockstep
from purin_b200.config import ChambollePockConfig
from purin_b200.layer import _ptr, ctypes_stream, resolve_device, resolve_dtype
from purin_b200.types import ProjectionResult, SolveStatus


class QPData(NamedTuple):
    """Batched diagonal objective, constraint coefficients and variable bounds."""

    q: object
    c: object
    values: object
    rhs: object
    lower: object
    upper: object


def _layout(rows, n):
    """Padded support (m, width), mask and the flat positions of the real entries.

    ``kernels.py:26-40``: row i keeps its columns in the given order; padding
    slots point at column 0 with a zero coefficient.
    """
    width = max(1, max(map(len, rows), default=0))
    support = np.zeros((len(rows), width), dtype=np.int64)
    mask = np.zeros_like(support, dtype=bool)
    for i, row in enumerate(rows):
        support[i, : len(row)] = row
        mask[i, : len(row)] = True
    positions = np.flatnonzero(mask.reshape(-1))
    return support, mask, positions


@dataclass(frozen=True)
class QPStructure:
    """Variable dimension and fixed row supports for a family of diagonal QPs."""

    variable_size: int
    equality_rows: tuple = ()
    inequality_rows: tuple = ()

    def __post_init__(self):
        if self.variable_size < 1:
            raise ValueError("variable_size must be positive")
        for key in ("equality_rows", "inequality_rows"):
            rows = tuple(tuple(int(i) for i in row) for row in getattr(self, key))
            if any(len(set(row)) != len(row) or any(i < 0 or i >= self.variable_size for i in row)
                   for row in rows):
                raise ValueError("constraint supports must contain unique valid indices")
            object.__setattr__(self, key, rows)

    @property
    def rows(self):
        """Return equality rows followed by inequality rows in solver order."""
        return self.equality_rows + self.inequality_rows

    def prepare(self, *, batch_size, config=None, dtype=torch.float64, backend="cuda"):
        """Prepare a solver for this fixed sparse structure and batch shape."""
        return PreparedDiagonalQP(self, int(batch_size), config or ChambollePockConfig(), dtype,
                                  backend)


class _QPSolve(torch.autograd.Function):
    """The custom-VJP solve of diagonal_qp.py:125-222 as a torch autograd op."""

    @staticmethod
    def forward(ctx, q, c, values, rhs, lower, upper, y0, dual0, tolerance, layer):
        batch, n = q.shape
        m = rhs.shape[1]
        dev, dt = q.device, q.dtype
        y = torch.empty((batch, n), dtype=dt, device=dev)
        dual = torch.empty((batch, m), dtype=dt, device=dev)
        iterations = torch.empty((batch,), dtype=torch.int32, device=dev)
        residual = torch.empty((batch,), dtype=dt, device=dev)
        gap = torch.empty((batch,), dtype=dt, device=dev)
        converged = torch.empty((batch,), dtype=torch.uint8, device=dev)
        # One row of values for the whole batch (a broadcast constraint matrix) is
        # passed with stride 0; otherwise one row per sample.
        stride = 0 if values.shape[0] == 1 and batch != 1 else values.shape[1]
        op = _native.QP_OP_FORWARD if stride == 0 else _native.QP_OP_FORWARD_SAMPLE_VALUES
        ws_bytes = layer._plan.workspace_size(op, batch, layer._cfg)
        ws = torch.empty((max(ws_bytes, 1),), dtype=torch.uint8, device=dev)
        args = _native.QpForwardArgs(
            batch, _ptr(q), _ptr(c), _ptr(values), stride, _ptr(rhs), _ptr(lower),
            _ptr(upper), n, _ptr(y0), _ptr(dual0), _ptr(tolerance), layer._sample_offset,
            layer._total_batch, _ptr(y), _ptr(dual), _ptr(iterations), _ptr(residual), _ptr(gap),
            _ptr(converged))
        with layer._timed("forward"):
            layer._plan.qp_forward(layer._cfg, args, ws.data_ptr(), ws_bytes, layer._stream())
        ctx.layer = layer
        ctx.save_for_backward(q, c, values, rhs, lower, upper, y, dual, converged)
        ctx.mark_non_differentiable(iterations, residual, gap, converged)
        return y, dual, iterations, residual, gap, converged

    @staticmethod
    def backward(ctx, gy, gdual, *unused):
        q, c, values, rhs, lower, upper, y, dual, converged = ctx.saved_tensors
        layer = ctx.layer
        m = rhs.shape[1]
        gy = torch.zeros_like(y) if gy is None else gy.contiguous()
        cot_dual = None
        if layer.differentiate_duals and gdual is not None and m > 0:
            cot_dual = gdual.contiguous()
        shard = _QPAdjointShard(layer, (q, c, values, rhs, lower, upper, y, dual, converged),
                                gy, cot_dual, ctx.needs_input_grad)
        if layer._lockstep_group is None:
            grads = shard.fused()
        else:
            (grads,), _, _ = lockstep.run([shard], int(layer._lin.max_iterations),
                                          group=layer._lockstep_group)
        return (*grads, None, None, None, None)


class _QPAdjointShard:
    """Outputs, workspace and C-ABI arguments of one QP adjoint call.

    ``fused()`` is ``purin_qp_adjoint``; ``prepare``/``cycle``/``finish`` are the
    phases of ``purin_qp_adjoint_stage`` for ``purin_b200.lockstep.run``.
    """

    def __init__(self, layer, saved, gy, cot_dual, need):
        q, c, values, rhs, lower, upper, y, dual, converged = saved
        batch, n = q.shape
        m = rhs.shape[1]
        dev, dt = q.device, q.dtype
        out = lambda k, shape: torch.empty(shape, dtype=dt, device=dev) if need[k] else None
        self.shared = values.shape[0] == 1 and batch != 1
        self.grads = (out(0, (batch, n)), out(1, (batch, n)), out(2, (batch, values.shape[1])),
                      out(3, (batch, m)), out(4, (batch, n)), out(5, (batch, n)))
        self.layer = layer
        self.status = torch.empty((batch,), dtype=torch.int32, device=dev)
        self.lres = torch.empty((batch,), dtype=dt, device=dev)
        self.err = torch.zeros((1,), dtype=torch.int32, device=dev)
        self.counters = torch.zeros((2,), dtype=torch.int32, device=dev)
        self.ws_bytes = layer._plan.workspace_size(_native.QP_OP_ADJOINT, batch, layer._cfg,
                                                   layer._lin)
        self.ws = torch.empty((max(self.ws_bytes, 1),), dtype=torch.uint8, device=dev)
        g_q, g_c, g_values, g_rhs, g_lower, g_upper = self.grads
        self.args = _native.QpAdjointArgs(
            batch, _ptr(q), _ptr(c), _ptr(values), 0 if self.shared else values.shape[1],
            _ptr(rhs), _ptr(lower), _ptr(upper), n, _ptr(y), _ptr(dual), _ptr(converged),
            _ptr(gy), _ptr(cot_dual), layer._sample_offset, layer._total_batch, _ptr(g_q),
            _ptr(g_c), _ptr(g_values), _ptr(g_rhs), _ptr(g_lower), _ptr(g_upper),
            _ptr(self.status), _ptr(self.lres), _ptr(self.err))
        # Keep every buffer the arguments point at alive for the shard's lifetime.
        self._inputs = (saved, gy, cot_dual)

    def _done(self):
        object.__setattr__(self.layer, "_last_linear", (self.status, self.lres))
        if int(self.err.item()) != 0:
            raise RuntimeError("purin_qp_adjoint: a bounded device wait timed out; "
                               "gradients are invalid")
        g_q, g_c, g_values, g_rhs, g_lower, g_upper = self.grads
        if self.shared and g_values is not None:
            g_values = g_values.sum(dim=0, keepdim=True)
        return g_q, g_c, g_values, g_rhs, g_lower, g_upper

    def fused(self):
        layer = self.layer
        with layer._timed("adjoint"):
            layer._plan.qp_adjoint(layer._cfg, layer._lin, self.args, self.ws.data_ptr(),
                                   self.ws_bytes, layer._stream())
        return self._done()

    def _stage(self, stage, completed=0):
        layer = self.layer
        with layer._timed("adjoint"):
            layer._plan.qp_adjoint_stage(layer._cfg, layer._lin, self.args, stage, completed,
                                         self.counters.data_ptr(), self.ws.data_ptr(),
                                         self.ws_bytes, layer._stream())
        return self.counters

    def prepare(self):
        return self._stage(_native.STAGE_PREPARE)

    def cycle(self, completed):
        return self._stage(_native.STAGE_CYCLE, completed)

    def finish(self):
        self._stage(_native.STAGE_FINISH)
        return self._done()


@dataclass(frozen=True, eq=False)
class PreparedDiagonalQP:
    """Prepared diagonal-QP solve on the shared sparse Chambolle--Pock kernels."""

    structure: QPStructure
    batch_size: int
    config: ChambollePockConfig
    dtype: object = torch.float64
    backend: str = "cuda"
    differentiate_duals: bool = True

    def __post_init__(self):
        if self.batch_size < 1:
            raise ValueError("batch_size must be positive")
        if self.config.metric_diagonal is not None:
            raise ValueError("QPData.q already defines the quadratic metric")
        set_ = lambda k, v: object.__setattr__(self, k, v)
        device = resolve_device(self.backend)
        tdtype = resolve_dtype(self.dtype)
        structure = self.structure
        n = structure.variable_size
        rows = structure.rows
        support, mask, positions = _layout(rows, n)
        row_ptr = np.zeros(len(rows) + 1, dtype=np.int32)
        row_ptr[1:] = np.cumsum([len(r) for r in rows])
        col = np.asarray([j for r in rows for j in r], dtype=np.int32)
        plan = _native.Plan(n, len(structure.equality_rows), len(structure.inequality_rows),
                            row_ptr, col, _native.PURIN_FLOAT64 if tdtype == torch.float64
                            else _native.PURIN_FLOAT32, device.index, qp=True)
        as_long = lambda a: torch.as_tensor(np.asarray(a, dtype=np.int64), device=device)
        set_("_device", device)
        set_("_tdtype", tdtype)
        set_("_plan", plan)
        set_("_me", len(structure.equality_rows))
        set_("_support_np", support)
        set_("_mask_np", mask)
        set_("_support", as_long(support))
        set_("_mask", torch.as_tensor(mask, device=device))
        set_("_positions", as_long(positions))
        # K.T @ y in the reference's scatter order: per column, the (row, slot)
        # entries in increasing flat order, accumulated one at a time.
        width = support.shape[1]
        flat_cols = np.where(mask, support, -1).reshape(-1)
        per_col = [np.flatnonzero(flat_cols == j) for j in range(n)]
        depth = max(1, max((len(p) for p in per_col), default=0))
        col_pos = np.zeros((n, depth), dtype=np.int64)
        col_ok = np.zeros((n, depth), dtype=bool)
        for j, p in enumerate(per_col):
            col_pos[j, : len(p)] = p
            col_ok[j, : len(p)] = True
        set_("_col_pos", as_long(col_pos))
        set_("_col_row", as_long(col_pos // width))
        set_("_col_ok", torch.as_tensor(col_ok, device=device))
        cfg = self.config
        set_("_cfg", _native.CpConfig(
            int(cfg.max_iterations), int(bool(cfg.accelerated)), float(cfg.safety),
            int(cfg.norm_iterations), int(cfg.norm_seed), int(bool(cfg.norm_bound)),
            int(bool(cfg.diagonal_preconditioning)), int(bool(cfg.prng_partitionable))))
        lin = cfg.linear_solver
        set_("_lin", _native.LinearConfig(float(lin.tolerance), float(lin.atol), int(lin.restart),
                                          int(lin.max_iterations),
                                          float(cfg.implicit_gradient.adjoint_tolerance)))
        set_("_sample_offset", 0)
        set_("_total_batch", int(self.batch_size))
        set_("_lockstep_group", None)
        set_("_timers", None)

    @property
    def support(self):
        return self._support_np

    @property
    def mask(self):
        return self._mask_np

    def set_shard(self, offset: int, total: int, group=None):
        """Rows ``offset..`` of a global batch of ``total``.

        The offset selects the power iteration's PRNG keys; ``group`` (a
        ``torch.distributed`` group of the ranks holding the other shards) makes
        the backward share the batch-wide GMRES budget, as for the projection
        layer (``purin_b200.lockstep``).
        """
        object.__setattr__(self, "_sample_offset", int(offset))
        object.__setattr__(self, "_total_batch", int(total))
        object.__setattr__(self, "_lockstep_group", group)

    def _stream(self):
        return ctypes_stream(torch.cuda.current_stream(self._device))

    def record_launches(self, timers: list | None):
        """Collect (kernel, start_event, end_event) for every native launch, or stop (None)."""
        object.__setattr__(self, "_timers", timers)

    @contextlib.contextmanager
    def _timed(self, name):
        """NVTX range around one native call; with ``record_launches`` also CUDA events."""
        timers = self._timers
        with torch.cuda.nvtx.range("purin_qp_" + name):
            if timers is None:
                yield
                return
            stream = torch.cuda.current_stream(self._device)
            start = torch.cuda.Event(enable_timing=True)
            end = torch.cuda.Event(enable_timing=True)
            start.record(stream)
            yield
            end.record(stream)
            timers.append((name, start, end))

    # -- ordered sparse products (the reference's accumulation order) -------------
    def _matvec(self, values, x):
        """K @ x: one term at a time along each padded row (operators.py:507-518)."""
        out = torch.zeros((x.shape[0], values.shape[1]), dtype=x.dtype, device=x.device)
        zero = torch.zeros((), dtype=x.dtype, device=x.device)
        for k in range(values.shape[2]):
            term = values[:, :, k] * x[:, self._support[:, k]]
            out = out + torch.where(self._mask[None, :, k], term, zero)
        return out

    def _tmatvec(self, values, y):
        """K.T @ y: per column, the scatter's updates in flat (row, slot) order."""
        flat = values.reshape(values.shape[0], -1)
        out = torch.zeros((y.shape[0], self.structure.variable_size), dtype=y.dtype,
                          device=y.device)
        if values.shape[1] == 0:  # no constraint rows: K.T y = 0
            return out
        zero = torch.zeros((), dtype=y.dtype, device=y.device)
        for d in range(self._col_pos.shape[1]):
            term = flat[:, self._col_pos[:, d]] * y[:, self._col_row[:, d]]
            out = out + torch.where(self._col_ok[None, :, d], term, zero)
        return out

    def _row_scale(self, values):
        """scale = 1/||row||_2 of the masked padded rows (diagonal_qp.py:256-262)."""
        batch, m, width = values.shape
        one = torch.ones((), dtype=values.dtype, device=values.device)
        if not self.config.row_scaling or m == 0:
            return torch.ones((batch, m), dtype=values.dtype, device=values.device)
        sq = torch.where(self._mask[None], values * values, torch.zeros_like(values))
        acc = torch.zeros((batch, m), dtype=values.dtype, device=values.device)
        for k in range(width):
            acc = acc + sq[:, :, k]
        norms = torch.sqrt(acc)
        scale = torch.where(norms > 0, one / torch.clamp_min(norms, 1e-30), one)
        return scale.detach()

    # -- public API -------------------------------------------------------------------
    def solve(self, data, *, initial_y=None, initial_dual=None):
        """Solve the batched diagonal QP with the supplied coefficients and warm start."""
        dev, dt = self._device, self._tdtype
        data = QPData(*(torch.as_tensor(x, dtype=dt, device=dev) for x in data))
        b, n = self.batch_size, self.structure.variable_size
        m, width = self._support_np.shape
        expected = ((b, n), (b, n), (b, m, width), (b, m), (b, n), (b, n))
        for key, value, shape in zip(QPData._fields, data, expected):
            if tuple(value.shape) != shape:
                raise ValueError(f"{key} must have shape {shape}; got {tuple(value.shape)}")
        y0 = (torch.zeros((b, n), dtype=dt, device=dev) if initial_y is None
              else torch.as_tensor(initial_y, dtype=dt, device=dev))
        dual0 = (torch.zeros((b, m), dtype=dt, device=dev) if initial_dual is None
                 else torch.as_tensor(initial_dual, dtype=dt, device=dev))
        if tuple(y0.shape) != (b, n) or tuple(dual0.shape) != (b, m):
            raise ValueError("initial primal/dual shapes do not match the prepared QP")
        # A constraint matrix broadcast over the batch (stride 0, as dense_qp_data
        # builds it) is scaled and handed to the kernels once for all samples.
        shared = b > 1 and data.values.stride(0) == 0
        values = data.values[:1] if shared else data.values
        scale = self._row_scale(values)
        scaled_values = values * scale[:, :, None]
        if shared:
            scale = scale.expand(b, m)
        scaled_rhs = data.rhs * scale
        one = torch.ones((), dtype=dt, device=dev)
        min_scale = (torch.minimum(one, scale.min(dim=1).values) if m > 0
                     else torch.ones((b,), dtype=dt, device=dev))
        tolerance = (self.config.tolerance * torch.minimum(one, min_scale)).detach()
        values_csr = scaled_values.reshape(scaled_values.shape[0], m * width)[:, self._positions]
        y, dual, iterations, _, _, cp_converged = _QPSolve.apply(
            data.q.contiguous(), data.c.contiguous(), values_csr.contiguous(),
            scaled_rhs.contiguous(), data.lower.contiguous(), data.upper.contiguous(),
            y0.detach().contiguous(), (dual0 / scale).detach().contiguous(), tolerance.contiguous(),
            self)
        dual = dual * scale
        me = self._me
        residuals = self._matvec(data.values, y) - data.rhs
        zero = torch.zeros((), dtype=dt, device=dev)
        eq = (residuals[:, :me].abs().amax(dim=1) if me > 0
              else torch.zeros((b,), dtype=dt, device=dev))
        iq = (torch.maximum(residuals[:, me:], zero).amax(dim=1) if m > me
              else torch.zeros((b,), dtype=dt, device=dev))
        eq = torch.maximum(eq, zero)
        iq = torch.maximum(iq, zero)
        inner = y - ((data.q * y + data.c) + self._tmatvec(data.values, dual))
        clipped = torch.minimum(data.upper, torch.maximum(data.lower, inner))
        stationarity = (y - clipped).abs().amax(dim=1)
        residual = torch.maximum(torch.maximum(eq, iq), stationarity).detach()
        converged = (cp_converged.bool() & (residual <= self.config.tolerance)).detach()
        finite = (torch.isfinite(y).all(dim=1) & torch.isfinite(dual).all(dim=1)
                  & torch.isfinite(residual)).detach()
        status = torch.where(
            converged, int(SolveStatus.CONVERGED),
            torch.where(finite, int(SolveStatus.MAX_ITERATIONS), int(SolveStatus.NONFINITE)))
        slacks = torch.maximum(data.rhs[:, me:] - self._matvec(data.values, y)[:, me:], zero)
        return ProjectionResult(y, dual[:, :me], dual[:, me:], slacks,
                                status.to(torch.int32), iterations, residual, finite, converged)


def dense_qp_data(q, c, A, b, C, d, lower, upper):
    """Convenience adapter (diagonal_qp.py:317-349): dense blocks to a full-support QP."""
    q = torch.as_tensor(q)
    c = torch.as_tensor(c)
    if q.ndim != 2 or q.shape != c.shape:
        raise ValueError("q and c must be matching batched matrices")
    batch, n = q.shape
    dtype = q.dtype if q.is_floating_point() else torch.float64
    as_t = lambda x: torch.as_tensor(x, dtype=dtype, device=q.device)
    q, c, A, C = as_t(q), as_t(c), as_t(A), as_t(C)
    A = torch.broadcast_to(A, (batch,) + tuple(A.shape[-2:]))
    C = torch.broadcast_to(C, (batch,) + tuple(C.shape[-2:]))
    rows = tuple(tuple(range(n)) for _ in range(A.shape[1]))
    iq = tuple(tuple(range(n)) for _ in range(C.shape[1]))
    structure = QPStructure(n, rows, iq)
    values = torch.cat((A, C), dim=1)  # every row's support is 0..n-1, so no padding
    if values.shape[1] == 0:
        values = values.new_zeros((batch, 0, 1))  # the padded layout of no rows has width 1
    rhs = torch.cat((torch.broadcast_to(as_t(b), (batch, A.shape[1])),
                     torch.broadcast_to(as_t(d), (batch, C.shape[1]))), dim=1)
    return structure, QPData(q, c, values, rhs, torch.broadcast_to(as_t(lower), q.shape),
                             torch.broadcast_to(as_t(upper), q.shape))
