"""Prepared Chambolle--Pock projection layer on B200 (torch host glue + C ABI).

Mirrors ``PreparedChambollePockProjection`` (``src/purin/solvers/chambolle_pock/
solver.py:22-402``) together with ``BoundProjection`` (``bounds.py:15-326``):
the same public methods (``__call__``, ``solve``, ``with_info``,
``project_training``), the same argument checks and messages, the same result
tuples.  The per-call preprocessing that the reference differentiates through
(coefficient evaluation from the parameters, bound presolve ``bounds.py:193-209``,
row scaling ``bounds.py:210-214``, warm start and tolerance ``bounds.py:215-236``)
runs as torch operations on the device so autograd chains through it exactly
as JAX does; the solve itself (``bounds.py:237-246`` / ``solver.py:332``), its
custom VJP (``bounds.py:68-167``) and the post-processing (``bounds.py:247-305``)
are the CUDA kernels behind ``libpurin_cp.so``.
"""

from __future__ import annotations

import contextlib
from dataclasses import dataclass
from types import SimpleNamespace
from typing import NamedTuple

import numpy as np
import torch

from purin_b200 import _native, lockstep
from purin_b200.config import ChambollePockConfig
from purin_b200.problems import CanonicalAffine, canonical_of, ell_index, rows_of
from purin_b200.types import (
    ProjectionInfo,
    ProjectionResult,
    ProjectionTrainingOutput,
)


def resolve_device(backend) -> torch.device:
    """CUDA device for ``backend`` ("cuda", "gpu", "cuda:i", "gpu:i" or a torch device).

    ``execution/runtime.py:33-78`` resolves "cpu"/"gpu"/"cuda:i" for JAX; this
    build runs only on CUDA devices and raises for any other backend.
    """
    if isinstance(backend, torch.device):
        device = backend
    else:
        text = str(backend).strip().lower()
        if text.startswith("gpu"):
            text = "cuda" + text[3:]
        if not text.startswith("cuda"):
            raise RuntimeError(
                f"purin_b200 runs the chambolle-pock projection on CUDA devices only; got backend={backend!r}")
        device = torch.device(text)
    if device.type != "cuda":
        raise RuntimeError(f"purin_b200 requires a CUDA device; got {device}")
    if not torch.cuda.is_available():
        raise RuntimeError("purin_b200 requires a CUDA device, but torch.cuda.is_available() is False")
    if device.index is None:
        device = torch.device("cuda", torch.cuda.current_device())
    return device


def resolve_dtype(dtype) -> torch.dtype:
    if dtype is None:
        return torch.float64
    if isinstance(dtype, torch.dtype):
        if dtype not in (torch.float64, torch.float32):
            raise ValueError("dtype must be float64 or float32")
        return dtype
    name = np.dtype(dtype).name
    if name == "float64":
        return torch.float64
    if name == "float32":
        return torch.float32
    raise ValueError("dtype must be float64 or float32")


def _ptr(t):
    return None if t is None else t.data_ptr()


class _CPOut(NamedTuple):
    y: torch.Tensor
    dual: torch.Tensor
    iterations: torch.Tensor
    residual: torch.Tensor
    gap: torch.Tensor
    converged: torch.Tensor


class _SolveFunction(torch.autograd.Function):
    """``jax.custom_vjp`` solve of ``bounds.py:68-167`` as a torch autograd op."""

    @staticmethod
    def forward(ctx, data, rhs, target, lower, upper, initial, tolerance, feasible, layer):
        batch, n = target.shape
        m = layer._m
        dev = target.device
        dtype = target.dtype
        y = torch.empty((batch, n), dtype=dtype, device=dev)
        dual = torch.empty((batch, m), dtype=dtype, device=dev)
        iterations = torch.empty((batch,), dtype=torch.int32, device=dev)
        residual = torch.empty((batch,), dtype=dtype, device=dev)
        gap = torch.empty((batch,), dtype=dtype, device=dev)
        converged = torch.empty((batch,), dtype=torch.uint8, device=dev)
        layer._forward_native(data, rhs, target, lower, upper, initial, tolerance, feasible,
                              y, dual, iterations, residual, gap, converged)
        ctx.layer = layer
        ctx.shared_values = data.shape[0] == 1 and batch != 1
        ctx.shared_bounds = lower.shape[0] == 1 and batch != 1
        ctx.save_for_backward(data, rhs, target, lower, upper, y, dual, converged)
        ctx.mark_non_differentiable(dual, iterations, residual, gap, converged)
        return y, dual, iterations, residual, gap, converged

    @staticmethod
    def backward(ctx, gy, *unused):
        data, rhs, target, lower, upper, y, dual, converged = ctx.saved_tensors
        layer = ctx.layer
        need = ctx.needs_input_grad
        if gy is None:
            gy = torch.zeros_like(y)
        grads = layer._adjoint_native(data, rhs, target, lower, upper, y, dual, converged,
                                      gy.contiguous(), need_values=need[0], need_rhs=need[1],
                                      need_target=need[2], need_lower=need[3], need_upper=need[4])
        g_values, g_rhs, g_target, g_lower, g_upper = grads
        if g_values is not None and ctx.shared_values:
            g_values = g_values.sum(dim=0, keepdim=True)
        if ctx.shared_bounds:
            g_lower = None if g_lower is None else g_lower.sum(dim=0, keepdim=True)
            g_upper = None if g_upper is None else g_upper.sum(dim=0, keepdim=True)
        return g_values, g_rhs, g_target, g_lower, g_upper, None, None, None, None


@dataclass(frozen=True, eq=False)
class PreparedChambollePockProjection:
    """Prepared affine distance projection on sm_100a CUDA kernels."""

    canonical: CanonicalAffine
    config: ChambollePockConfig
    batch_size: int
    dtype: object
    backend: str

    def __post_init__(self):
        metadata = self.canonical.metadata or {}
        if not (metadata.get("equalities_affine_in_variables") is True
                and metadata.get("inequalities_affine_in_variables") is True):
            raise ValueError(
                "chambolle-pock requires verified affine equalities and inequalities; "
                "nonlinear or unverified constraints are unsupported")
        if self.batch_size < 1 or self.output_size < 1:
            raise ValueError("batch_size and variable_size must be positive")
        device = resolve_device(self.backend)
        tdtype = resolve_dtype(self.dtype)
        eq = tuple(self.canonical.equality_sparsity)
        iq = tuple(self.canonical.inequality_sparsity)
        if len(eq) != self.equality_size or len(iq) != self.inequality_size:
            raise ValueError("constraint sparsity row counts do not match the problem")
        row_ptr, col = self.canonical.csr()
        plan = _native.Plan(self.output_size, self.equality_size, self.inequality_size, row_ptr,
                            col, _native.PURIN_FLOAT64 if tdtype == torch.float64
                            else _native.PURIN_FLOAT32, device.index)
        set_ = lambda k, v: object.__setattr__(self, k, v)
        set_("_device", device)
        set_("_tdtype", tdtype)
        set_("_plan", plan)
        set_("_m", plan.info.kept_rows)
        set_("_nnz", plan.info.nnz)
        as_long = lambda a: torch.as_tensor(np.asarray(a, dtype=np.int64), device=device)
        kept_rows = plan.indices(_native.KEPT_ROWS)
        kept_slots = plan.indices(_native.KEPT_SLOTS)
        kept_row_ptr = plan.indices(_native.KEPT_ROW_PTR)
        set_("_kept_rows", as_long(kept_rows))
        set_("_kept_slots", as_long(kept_slots))
        set_("_bound_rows", as_long(plan.indices(_native.BOUND_ROWS)))
        set_("_bound_slots", as_long(plan.indices(_native.BOUND_SLOTS)))
        set_("_bound_vars", as_long(plan.indices(_native.BOUND_VARIABLES)))
        set_("_n_bound", int(plan.info.bound_rows))
        param_rows = getattr(self.canonical, "rhs_parameter_rows", None)
        bound_rows = plan.indices(_native.BOUND_ROWS)
        set_("_bounds_shared", bool(
            getattr(self.canonical, "values_constant", False) and param_rows is not None
            and not np.asarray(param_rows, bool)[bound_rows].any()))
        set_("_kept_ell", as_long(ell_index(kept_row_ptr)))
        set_("_slot_row", as_long(rows_of(kept_row_ptr)))
        cfg = self.config
        set_("_cfg", _native.CpConfig(
            int(cfg.max_iterations), int(bool(cfg.accelerated)), float(cfg.safety),
            int(cfg.norm_iterations), int(cfg.norm_seed), int(bool(cfg.norm_bound)),
            int(bool(cfg.diagonal_preconditioning)), int(bool(cfg.prng_partitionable))))
        lin = cfg.linear_solver
        set_("_lin", _native.LinearConfig(float(lin.tolerance), float(lin.atol), int(lin.restart),
                                          int(lin.max_iterations),
                                          float(cfg.implicit_gradient.adjoint_tolerance)))
        set_("_constant", None)
        set_("_sample_offset", 0)
        set_("_total_batch", int(self.batch_size))
        set_("_lockstep_group", None)
        set_("_timers", None)
        set_("_global_stop", None)
        set_("_qp_plan", None)
        set_("last_global_trip", None)

    # -- sizes -----------------------------------------------------------------
    @property
    def parameter_size(self):
        return int(self.canonical.parameter_size)

    @property
    def output_size(self):
        return int(self.canonical.variable_size)

    @property
    def equality_size(self):
        return int(self.canonical.equality_size)

    @property
    def inequality_size(self):
        return int(self.canonical.inequality_size)

    def set_shard(self, offset: int, total: int, group=None):
        """Declare this layer's batch as rows ``offset..`` of a global batch of ``total``.

        Two things couple a sample to the rest of the batch in the reference.
        The seeded power iteration draws sample ``b``'s start vector from
        ``split(PRNGKey(seed), total)[offset + b]``, which the offset fixes.  And
        the adjoint's restarted GMRES charges one iteration budget for the whole
        batch (operators.py:919-1103): given ``group`` (a ``torch.distributed``
        process group whose ranks hold the other shards, each calling
        ``set_shard`` with the same group), the backward runs in phases and
        all-reduces the two GMRES counters across the group after each one, so
        the gradients equal the unsharded batch's in every case.  Without a group
        each shard keeps its own budget, which gives the same gradients unless a
        sample needs more restart cycles than the budget allows the batch.
        """
        object.__setattr__(self, "_sample_offset", int(offset))
        object.__setattr__(self, "_total_batch", int(total))
        object.__setattr__(self, "_lockstep_group", group)

    def set_global_stop(self, interval: int | None = 100, group=None):
        """Run the forward under a batch-wide stopping rule, or not (``interval=None``).

        The reference's loop stops when every sample of the batch has been
        accepted or the budget is spent (``kernels.py:238-240``).  Each sample
        freezes once accepted, so stopping per sample (the default) gives the same
        outputs.  With the rule, the forward runs in segments of ``interval``
        iterations; after each, the samples still running are counted on the
        device and summed over ``group`` (a ``torch.distributed`` process group
        whose ranks hold the other shards of the batch: one NCCL all-reduce per
        segment for CUDA tensors), and every rank stops at the first segment end
        where none remains anywhere.  The outputs are bit-identical to the
        default's; ``last_global_trip`` then holds the batch's trip count (the
        largest iteration count over the global batch), equal on every rank.
        The segments run the diagonal-QP kernels with q = 1 and c = -target,
        whose iteration is the distance projection's bit for bit, resuming each
        sample from the previous segment's state.
        """
        if interval is not None and int(interval) < 1:
            raise ValueError("the global stopping interval must be a positive number of iterations")
        object.__setattr__(self, "_global_stop", None if interval is None else (int(interval), group))

    # -- native calls --------------------------------------------------------------
    def _stream(self):
        return ctypes_stream(torch.cuda.current_stream(self._device))

    def record_launches(self, timers: list | None):
        """Collect (kernel, start_event, end_event) for every native launch, or stop (None).

        The events are recorded on the stream each kernel is launched on, so
        ``start.elapsed_time(end)`` is that launch's device duration.
        """
        object.__setattr__(self, "_timers", timers)

    @contextlib.contextmanager
    def _timed(self, name):
        """NVTX range around one native call; with ``record_launches`` also CUDA events."""
        timers = self._timers
        with torch.cuda.nvtx.range("purin_cp_" + name):
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

    def _forward_native(self, data, rhs, target, lower, upper, initial, tolerance, feasible,
                        y, dual, iterations, residual, gap, converged):
        if self._global_stop is not None:
            return self._forward_global_stop(data, rhs, target, lower, upper, initial, tolerance,
                                             feasible, y, dual, iterations, residual, gap,
                                             converged)
        batch = target.shape[0]
        per_sample = data.shape[0] != 1 and batch != 1
        ws_bytes = self._plan.workspace_size(
            _native.OP_FORWARD_SAMPLE_VALUES if per_sample else _native.OP_FORWARD, batch, self._cfg)
        ws = torch.empty((max(ws_bytes, 1),), dtype=torch.uint8, device=self._device)
        args = _native.ForwardArgs(
            batch, _ptr(data), 0 if data.shape[0] == 1 and batch != 1 else data.shape[1],
            _ptr(rhs), _ptr(target), _ptr(initial), _ptr(tolerance), _ptr(lower), _ptr(upper),
            0 if lower.shape[0] == 1 and batch != 1 else self.output_size, _ptr(feasible),
            self._sample_offset, self._total_batch, _ptr(y), _ptr(dual), _ptr(iterations),
            _ptr(residual), _ptr(gap), _ptr(converged))
        with self._timed("forward"):
            self._plan.forward(self._cfg, args, ws.data_ptr(), ws_bytes, self._stream())

    def _forward_global_stop(self, data, rhs, target, lower, upper, initial, tolerance,
                             feasible, y, dual, iterations, residual, gap, converged):
        """The forward under ``set_global_stop``: segments on the QP kernels, outputs in place."""
        from types import SimpleNamespace

        interval, group = self._global_stop
        batch, n = target.shape
        m = self._m
        dev, dt = target.device, target.dtype
        if self._qp_plan is None:
            # The kept rows as a plan whose every row is a CP row (no bound presolve).
            row_ptr = self._plan.indices(_native.KEPT_ROW_PTR)
            cols = self._plan.indices(_native.KEPT_COLS)
            me = self.equality_size
            object.__setattr__(self, "_qp_plan", _native.Plan(
                n, me, m - me, row_ptr, cols,
                _native.PURIN_FLOAT64 if dt == torch.float64 else _native.PURIN_FLOAT32,
                self._device.index, qp=True))
        plan = self._qp_plan
        q = torch.ones((batch, n), dtype=dt, device=dev)
        c = (-target).contiguous()
        stride = 0 if data.shape[0] == 1 and batch != 1 else data.shape[1]
        bounds_stride = 0 if lower.shape[0] == 1 and batch != 1 else n
        op = _native.QP_OP_FORWARD if stride == 0 else _native.QP_OP_FORWARD_SAMPLE_VALUES
        cfg = self._cfg

        def segment(end, y0, dual0, ybar0, start):
            seg_cfg = _native.CpConfig(end, cfg.accelerated, cfg.safety, cfg.norm_iterations,
                                       cfg.norm_seed, cfg.norm_bound,
                                       cfg.diagonal_preconditioning, cfg.prng_partitionable)
            out = SimpleNamespace(
                y=torch.empty((batch, n), dtype=dt, device=dev),
                dual=torch.empty((batch, m), dtype=dt, device=dev),
                ybar=torch.empty((batch, n), dtype=dt, device=dev),
                iterations=torch.empty((batch,), dtype=torch.int32, device=dev),
                residual=torch.empty((batch,), dtype=dt, device=dev),
                gap=torch.empty((batch,), dtype=dt, device=dev),
                converged=torch.empty((batch,), dtype=torch.uint8, device=dev))
            y0 = y0.contiguous()
            dual0 = dual0.contiguous()
            ybar0 = None if ybar0 is None else ybar0.contiguous()
            start = None if start is None else start.contiguous()
            ws_bytes = plan.workspace_size(op, batch, seg_cfg)
            ws = torch.empty((max(ws_bytes, 1),), dtype=torch.uint8, device=dev)
            args = _native.QpForwardArgs(
                batch, _ptr(q), _ptr(c), _ptr(data), stride, _ptr(rhs), _ptr(lower), _ptr(upper),
                bounds_stride, _ptr(y0), _ptr(dual0) if m else None, _ptr(tolerance),
                self._sample_offset, self._total_batch, _ptr(out.y), _ptr(out.dual),
                _ptr(out.iterations), _ptr(out.residual), _ptr(out.gap), _ptr(out.converged),
                _native.QP_NO_VALIDITY, _ptr(ybar0) if ybar0 is not None else None,
                _ptr(start) if start is not None else None, _ptr(out.ybar))
            with self._timed("forward"):
                plan.qp_forward(seg_cfg, args, ws.data_ptr(), ws_bytes, self._stream())
            return out

        fy, fd, fit, fres, fgap, fconv, trip, _ = lockstep.global_stop_forward(
            segment, target, initial if m else torch.zeros((batch, 0), dtype=dt, device=dev),
            batch, int(cfg.max_iterations), interval, group)
        y.copy_(fy)
        dual.copy_(fd)
        iterations.copy_(fit)
        residual.copy_(fres)
        gap.copy_(fgap)
        # converged &= feasible (bounds.py:66), as the projection kernel applies it.
        converged.copy_(fconv & feasible)
        object.__setattr__(self, "last_global_trip", trip)

    def _adjoint_native(self, data, rhs, target, lower, upper, y, dual, converged, gy, *,
                        need_values, need_rhs, need_target, need_lower, need_upper):
        shard = self._adjoint_shard(data, rhs, target, lower, upper, y, dual, converged, gy,
                                    need_values=need_values, need_rhs=need_rhs,
                                    need_target=need_target, need_lower=need_lower,
                                    need_upper=need_upper)
        if self._lockstep_group is None:
            return shard.fused()
        (grads,), _, _ = lockstep.run([shard], int(self._lin.max_iterations),
                                      group=self._lockstep_group)
        return grads

    def _adjoint_shard(self, data, rhs, target, lower, upper, y, dual, converged, gy, *,
                       need_values, need_rhs, need_target, need_lower, need_upper):
        """The backward of this layer's batch as a shard of ``purin_b200.lockstep``."""
        return _AdjointShard(self, data, rhs, target, lower, upper, y, dual, converged, gy,
                             (need_values, need_rhs, need_target, need_lower, need_upper))

    # -- preprocessing -----------------------------------------------------------------
    def _row_scale(self, kept):
        """scale = 1/||row||_2 (bounds.py:210-214), summed sequentially along each row."""
        if not self.config.row_scaling or self._m == 0:
            return torch.ones((kept.shape[0], self._m), dtype=kept.dtype, device=kept.device)
        padded = torch.cat([kept, torch.zeros_like(kept[:, :1])], dim=1)
        acc = None
        for k in range(self._kept_ell.shape[1]):
            v = padded[:, self._kept_ell[:, k]]
            acc = v * v if acc is None else acc + v * v
        norms = torch.sqrt(acc)
        one = torch.ones_like(norms)
        return torch.where(norms > 0, one / torch.clamp_min(norms, 1e-30), one)

    def _presolve(self, values, rhs, batch):
        """Box bounds from singleton inequality rows (bounds.py:193-209)."""
        n, dev, dt = self.output_size, self._device, self._tdtype
        inf = torch.tensor(float("inf"), dtype=dt, device=dev)
        # Bounds are computed once for the whole batch when neither the bound rows'
        # coefficients nor their right-hand sides depend on the parameters.
        shared = values.shape[0] == 1 and (rhs.shape[0] == 1 or self._bounds_shared)
        rows_b = 1 if shared else batch
        lower = torch.full((rows_b, n), -float("inf"), dtype=dt, device=dev)
        upper = torch.full((rows_b, n), float("inf"), dtype=dt, device=dev)
        if self._n_bound == 0:
            feasible = torch.ones((batch,), dtype=torch.uint8, device=dev)
            return lower, upper, feasible, None, None
        # index_select for gathers by unique indices: its gradient writes each
        # element once (no sort-based accumulation).
        coefficient = torch.index_select(values, 1, self._bound_slots).expand(rows_b, -1)
        b_rhs = torch.index_select(rhs[:rows_b], 1, self._bound_rows).expand(rows_b, -1)
        threshold = b_rhs / torch.where(coefficient != 0, coefficient, torch.ones_like(coefficient))
        index = self._bound_vars.unsqueeze(0).expand(rows_b, -1)
        lower = lower.scatter_reduce(1, index, torch.where(coefficient < 0, threshold, -inf), "amax",
                                     include_self=True)
        upper = upper.scatter_reduce(1, index, torch.where(coefficient > 0, threshold, inf), "amin",
                                     include_self=True)
        feasible = torch.all(lower <= upper, dim=1) & torch.all((coefficient != 0) | (b_rhs >= 0), dim=1)
        feasible = feasible.expand(batch).to(torch.uint8).contiguous()
        return lower, upper, feasible, coefficient, threshold

    def _solve(self, y_hat, parameters=None, multipliers_eq=None, multipliers_ineq=None):
        dev, dt = self._device, self._tdtype
        batch, n = self.batch_size, self.output_size
        me, mi = self.equality_size, self.inequality_size
        target = torch.as_tensor(y_hat, dtype=dt, device=dev)
        if target.ndim == 1:
            target = target[None, :]
        if tuple(target.shape) != (batch, n):
            raise ValueError(f"y_hat must have shape {(batch, n)}; got {tuple(target.shape)}")
        if parameters is None and self.parameter_size:
            raise ValueError("parameters are required for this problem")
        theta = (torch.zeros((batch, 0), dtype=dt, device=dev) if parameters is None
                 else torch.as_tensor(parameters, dtype=dt, device=dev))
        if tuple(theta.shape) != (batch, self.parameter_size):
            if self._n_bound:
                raise ValueError("parameters shape does not match the problem")
            raise ValueError(f"parameters must have shape {(batch, self.parameter_size)}; "
                             f"got {tuple(theta.shape)}")
        if not self.config.implicit_gradient.differentiate_problem_parameters:
            theta = theta.detach()
        values, rhs = self.canonical.evaluate(theta)
        if rhs.shape[0] != batch:
            rhs = rhs.expand(batch, -1)
        lower, upper, feasible, coefficient, threshold = self._presolve(values, rhs, batch)
        kept = torch.index_select(values, 1, self._kept_slots)
        scale = self._row_scale(kept)
        eq = (torch.zeros((batch, me), dtype=dt, device=dev) if multipliers_eq is None
              else torch.as_tensor(multipliers_eq, dtype=dt, device=dev))
        iq = (torch.zeros((batch, mi), dtype=dt, device=dev) if multipliers_ineq is None
              else torch.as_tensor(multipliers_ineq, dtype=dt, device=dev))
        if tuple(eq.shape) != (batch, me) or tuple(iq.shape) != (batch, mi):
            raise ValueError("warm-start multiplier shapes do not match constraints")
        scale_b = scale.expand(batch, -1) if scale.shape[0] != batch else scale
        initial = (torch.cat((eq, iq), dim=1)[:, self._kept_rows] / scale_b).detach().contiguous()
        # tol * minimum(1, min(scale, initial=1))                      bounds.py:233-236
        min_scale = (torch.clamp_max(scale_b.min(dim=1).values, 1.0) if self._m
                     else torch.ones((batch,), dtype=dt, device=dev))
        tolerance = (self.config.tolerance * torch.clamp_max(min_scale, 1.0)).detach().contiguous()
        data = (kept * scale[:, self._slot_row]).contiguous()
        scaled_rhs = (torch.index_select(rhs, 1, self._kept_rows) * scale_b).contiguous()
        out = _CPOut(*_SolveFunction.apply(data, scaled_rhs, target.contiguous(),
                                           lower.contiguous(), upper.contiguous(), initial,
                                           tolerance, feasible, self))
        return self._postprocess(values, rhs, target, out, scale_b, lower, upper)

    def _postprocess(self, values, rhs, target, out, scale, lower, upper):
        batch = target.shape[0]
        me, mi = self.equality_size, self.inequality_size
        dev, dt = self._device, self._tdtype
        meq = torch.empty((batch, me), dtype=dt, device=dev)
        miq = torch.empty((batch, mi), dtype=dt, device=dev)
        slacks = torch.empty((batch, mi), dtype=dt, device=dev)
        status = torch.empty((batch,), dtype=torch.int32, device=dev)
        resid = torch.empty((batch,), dtype=dt, device=dev)
        finite = torch.empty((batch,), dtype=torch.uint8, device=dev)
        elig = torch.empty((batch,), dtype=torch.uint8, device=dev)
        values_d = values.detach().contiguous()
        rhs_d = rhs.detach().contiguous()
        lower_d = lower.detach().contiguous()
        upper_d = upper.detach().contiguous()
        scale_d = scale.detach().contiguous()
        args = _native.PostArgs(
            batch, _ptr(values_d), 0 if values_d.shape[0] == 1 and batch != 1 else values_d.shape[1],
            _ptr(rhs_d), _ptr(target.detach().contiguous()), _ptr(lower_d), _ptr(upper_d),
            0 if lower_d.shape[0] == 1 and batch != 1 else self.output_size, _ptr(scale_d),
            _ptr(out.y.detach()), _ptr(out.dual), _ptr(out.gap), _ptr(out.converged),
            float(self.config.tolerance), _ptr(meq), _ptr(miq), _ptr(slacks), _ptr(status),
            _ptr(resid), _ptr(finite), _ptr(elig))
        with self._timed("postprocess"):
            self._plan.postprocess(args, self._stream())
        return ProjectionResult(out.y, meq, miq, slacks, status, out.iterations, resid,
                                finite.bool(), elig.bool())

    # -- public API (solver.py:368-402) ---------------------------------------------
    def solve(self, y_hat, parameters=None, initial_state=None):
        """Solve the prepared projection with the supplied targets and problem context."""
        if initial_state is not None:
            raise ValueError("Use project_training multiplier arguments for CP warm starts")
        return self._solve(y_hat, parameters)

    def __call__(self, y_hat, parameters=None):
        result = self.solve(y_hat, parameters)
        return result.y[0] if _ndim(y_hat) == 1 else result.y

    def with_info(self, y_hat, parameters=None):
        """Evaluate the projection and return its primal values with solver diagnostics."""
        r = self.solve(y_hat, parameters)
        return (r.y[0] if _ndim(y_hat) == 1 else r.y), ProjectionInfo(
            r.status, r.iterations, r.residual_inf_norm, r.finite, r.gradient_eligible)

    def project_training(self, y_hat, parameters=None, *, multipliers_eq=None,
                         multipliers_ineq=None):
        """Adapt the projection output and gradient eligibility to the shared training contract."""
        r = self._solve(y_hat, parameters, multipliers_eq, multipliers_ineq)
        return ProjectionTrainingOutput(r.y, r.multipliers_eq, r.multipliers_ineq, r.slacks,
                                        r.status, r.iterations, r.residual_inf_norm, r.finite,
                                        r.gradient_eligible)

    @property
    def _bound_projection(self):
        """Rows kept for the CP iteration and rows turned into bounds (``bounds.py:18-32``),
        or None when no inequality row is a singleton (``bounds.py:320-326``)."""
        if self._n_bound == 0:
            return None
        return SimpleNamespace(rows=self._kept_rows.tolist(), bound_rows=self._bound_rows.tolist())


class _AdjointShard:
    """Outputs, workspace and C-ABI arguments of one adjoint call.

    ``fused()`` runs the whole VJP in one launch (``purin_cp_adjoint``);
    ``prepare``/``cycle``/``finish`` run it in phases (``purin_cp_adjoint_stage``)
    for ``purin_b200.lockstep.run``, returning the shard's GMRES counters as a
    two-element device tensor.
    """

    def __init__(self, layer, data, rhs, target, lower, upper, y, dual, converged, gy, need):
        batch, n = target.shape
        m = layer._m
        dev, dt = layer._device, target.dtype
        need_values, need_rhs, need_target, need_lower, need_upper = need
        empty = lambda shape, dtype=dt: torch.empty(shape, dtype=dtype, device=dev)
        self.layer = layer
        self.grads = (empty((batch, data.shape[1])) if need_values else None,
                      empty((batch, m)) if need_rhs else None,
                      empty((batch, n)) if need_target else None,
                      empty((batch, n)) if need_lower else None,
                      empty((batch, n)) if need_upper else None)
        self.status = empty((batch,), torch.int32)
        self.lres = empty((batch,))
        self.err = torch.zeros((1,), dtype=torch.int32, device=dev)
        self.counters = torch.zeros((2,), dtype=torch.int32, device=dev)
        # GMRES work actually done (Arnoldi steps and basis vectors per sample).
        self.work = (empty((batch,), torch.int32), empty((batch,), torch.int64))
        self.ws_bytes = layer._plan.workspace_size(_native.OP_ADJOINT, batch, layer._cfg,
                                                   layer._lin)
        self.ws = torch.empty((max(self.ws_bytes, 1),), dtype=torch.uint8, device=dev)
        g_values, g_rhs, g_target, g_lower, g_upper = self.grads
        self.args = _native.AdjointArgs(
            batch, _ptr(data), 0 if data.shape[0] == 1 and batch != 1 else data.shape[1],
            _ptr(rhs), _ptr(target), _ptr(lower), _ptr(upper),
            0 if lower.shape[0] == 1 and batch != 1 else n, _ptr(y), _ptr(dual), _ptr(converged),
            _ptr(gy), layer._sample_offset, layer._total_batch, _ptr(g_values), _ptr(g_rhs),
            _ptr(g_target), _ptr(g_lower), _ptr(g_upper), _ptr(self.status), _ptr(self.lres),
            _ptr(self.err), _ptr(self.work[0]), _ptr(self.work[1]))
        # Keep every buffer the arguments point at alive for the shard's lifetime.
        self._inputs = (data, rhs, target, lower, upper, y, dual, converged, gy)

    def _done(self):
        layer = self.layer
        object.__setattr__(layer, "_last_linear", (self.status, self.lres))
        object.__setattr__(layer, "_last_work", self.work)
        if int(self.err.item()) != 0:
            raise RuntimeError("purin_cp_adjoint: a bounded device wait timed out; "
                               "gradients are invalid")
        return self.grads

    def fused(self):
        layer = self.layer
        with layer._timed("adjoint"):
            layer._plan.adjoint(layer._cfg, layer._lin, self.args, self.ws.data_ptr(),
                                self.ws_bytes, layer._stream())
        return self._done()

    def _stage(self, stage, completed=0):
        layer = self.layer
        with layer._timed("adjoint"):
            layer._plan.adjoint_stage(layer._cfg, layer._lin, self.args, stage, completed,
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


def _ndim(x):
    return x.ndim if hasattr(x, "ndim") else np.asarray(x).ndim


def ctypes_stream(stream: torch.cuda.Stream):
    return stream.cuda_stream


@dataclass(frozen=True)
class ChambollePockProjection:
    """Chambolle--Pock distance-projection definition for verified affine constraints."""

    problem: object
    config: ChambollePockConfig = ChambollePockConfig()

    def prepare(self, *, batch_size, dtype=torch.float64, backend="cuda"):
        """Prepare reusable projection resources for a fixed batch size, dtype and backend."""
        if self.config.metric_diagonal is not None:
            from purin_b200.metric import prepare_diagonal_metric

            return prepare_diagonal_metric(self.problem, self.config, type(self),
                                           batch_size=batch_size, dtype=dtype, backend=backend)
        canonical = canonical_of(self.problem)
        return PreparedChambollePockProjection(canonical, self.config, int(batch_size), dtype,
                                               str(backend))
