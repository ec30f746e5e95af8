"""ADMM distance projection on sm_100a kernels (``method="admm"``).

A drop-in for ``ADMMProjection(problem, ADMMConfig()).prepare(batch_size)``
(``src/purin/solvers/admm/solver.py:258-296``): the prepared layer keeps the
reference's ``__call__``, ``solve``, ``with_info`` and ``project_training``,
its result tuples and status codes.  Per call, on the device:

* coefficient evaluation, row scaling, warm start and tolerance in torch, as the
  unbounded prepared projection does (``chambolle_pock/solver.py:277-330``; ADMM
  keeps every public row, there is no bound presolve);
* the forward, ``sparse_admm`` (``admm/kernels.py:43-283``), in the CUDA kernel
  ``admm_forward_kernel`` (``purin_admm_forward``): Jacobi-PCG x-updates, or
  banded Cholesky solves when the row graph has a reverse Cuthill--McKee band of
  width at most 8 (``admm/factor.py:108-144``, laid out here at preparation);
* verified two-sided row pairs (``admm/rows.py``): opposite inequality rows
  nominated at preparation are checked per call and, when they hold, solved as
  one two-sided row on a compacted plan; multipliers are restored afterwards;
* the gap and residuals of the forward (``admm/solver.py:141-160``) and the
  post-processing (``chambolle_pock/solver.py:331-366``) in torch with ordered
  sparse sums;
* the implicit VJP (``admm/solver.py:175-255``), GMRES on the active-set KKT
  operator, in the adjoint kernel's ADMM mode (``purin_admm_adjoint``).
"""

from __future__ import annotations

import contextlib
from collections import deque
from dataclasses import dataclass, field
from types import SimpleNamespace

import numpy as np
import torch

from purin_b200 import _native, lockstep
from purin_b200.config import ADMMConfig
from purin_b200.layer import ctypes_stream, resolve_device, resolve_dtype
from purin_b200.problems import canonical_of, ell_index, rows_of
from purin_b200.types import ProjectionInfo, ProjectionResult, ProjectionTrainingOutput, SolveStatus


def _ptr(t):
    return 0 if t is None else t.data_ptr()


def band_layout(rows, n):
    """``admm/factor.py:108-144``: RCM order of the row graph and the band's entries.

    ``rows`` are the rows' column tuples (CSR order).  Returns None when the
    band is wider than 8, else the permutation, its inverse, the width and,
    per entry, (row, left CSR slot offset, right slot offset, destination).
    """
    graph = [set() for _ in range(n)]
    for row in rows:
        for i in row:
            graph[i].update(j for j in row if j != i)
    visited, order = set(), []
    while len(order) < n:
        root = min((i for i in range(n) if i not in visited), key=lambda i: (len(graph[i]), i))
        queue = deque([root])
        visited.add(root)
        while queue:
            i = queue.popleft()
            order.append(i)
            for j in sorted(graph[i] - visited, key=lambda j: (len(graph[j]), j)):
                if j not in visited:
                    visited.add(j)
                    queue.append(j)
    permutation = np.array(order[::-1], np.int64)
    inverse = np.argsort(permutation).astype(np.int64)
    width = max((abs(int(inverse[i]) - int(inverse[j])) for i in range(n) for j in graph[i]),
                default=0)
    if width > 8:
        return None
    entries = []
    for r, row in enumerate(rows):
        for a, ca in enumerate(row):
            for b, cb in enumerate(row):
                i, j = int(inverse[ca]), int(inverse[cb])
                if i >= j:
                    entries.append((r, a, b, i * (width + 1) + i - j))
    return SimpleNamespace(width=width, permutation=permutation, inverse=inverse,
                           entries=np.asarray(entries, np.int64).reshape(-1, 4))


def nominate_pairs(rows, values, me, row_scaling):
    """``admm/rows.py:54-84``: opposite inequality rows at the preparation values.

    ``values`` are the rows' coefficients (one array per row, CSR order) at
    theta = 0.  Returns (keep, first, second, positions) or None.
    """
    waiting, pairs = {}, []
    for r in range(me, len(rows)):
        v = np.asarray(values[r], np.float64)
        if row_scaling:
            norm = np.sqrt(np.sum(v ** 2))
            v = v * (1 / max(norm, 1e-30) if norm > 0 else 1.0)
        if not np.all(np.isfinite(v)) or not np.any(v):
            continue
        key = (tuple(rows[r]), tuple(v.tolist()))
        opposite = (tuple(rows[r]), tuple((-v).tolist()))
        if waiting.get(opposite):
            pairs.append((waiting[opposite].pop(), r))
        else:
            waiting.setdefault(key, []).append(r)
    if not pairs:
        return None
    removed = {j for _, j in pairs}
    keep = [i for i in range(len(rows)) if i not in removed]
    index = {r: i for i, r in enumerate(keep)}
    first, second = zip(*pairs)
    return keep, list(first), list(second), [index[i] for i in first]


class _System:
    """One ADMM constraint system on the device: plan, band and ordered-sum indices."""

    def __init__(self, rows, n, me, dtype_code, device, layer_device):
        m = len(rows)
        row_ptr = np.zeros(m + 1, np.int32)
        row_ptr[1:] = np.cumsum([len(r) for r in rows])
        col = np.asarray([j for r in rows for j in r], np.int32)
        self.plan = _native.Plan(n, me, m - me, row_ptr, col, dtype_code, device, qp=True)
        self.m = m
        as_i32 = lambda a: torch.as_tensor(np.asarray(a, np.int32), device=layer_device)
        band = band_layout(rows, n)
        if band is None:
            self.band = _native.AdmmBand(-1, 0, None, None, None, None, None, None)
            self.band_arrays = ()
            self.width = -1
        else:
            e = band.entries
            starts = row_ptr[e[:, 0]] if len(e) else np.zeros(0, np.int64)
            arrays = (as_i32(band.permutation), as_i32(band.inverse), as_i32(e[:, 0]),
                      as_i32(starts + e[:, 1]), as_i32(starts + e[:, 2]), as_i32(e[:, 3]))
            self.band_arrays = arrays  # kept alive with the layer
            self.band = _native.AdmmBand(band.width, len(e), *[a.data_ptr() for a in arrays])
            self.width = band.width


@dataclass(frozen=True, eq=False)
class PreparedADMMProjection:
    """Prepared ADMM distance projection on sm_100a CUDA kernels."""

    canonical: object
    config: ADMMConfig
    batch_size: int
    dtype: object
    backend: str

    def __post_init__(self):
        metadata = self.canonical.metadata or {}
        if not (metadata.get("equalities_affine_in_variables") is True
                and metadata.get("inequalities_affine_in_variables") is True):
            raise ValueError(
                "admm requires verified affine equalities and inequalities; nonlinear or "
                "unverified constraints are unsupported")
        if self.batch_size < 1 or self.output_size < 1:
            raise ValueError("batch_size and variable_size must be positive")
        device = resolve_device(self.backend)
        tdtype = resolve_dtype(self.dtype)
        set_ = lambda k, v: object.__setattr__(self, k, v)
        eq = tuple(self.canonical.equality_sparsity)
        iq = tuple(self.canonical.inequality_sparsity)
        if len(eq) != self.equality_size or len(iq) != self.inequality_size:
            raise ValueError("constraint sparsity row counts do not match the problem")
        rows = [tuple(int(j) for j in r) for r in eq + iq]
        n, me = self.output_size, self.equality_size
        code = _native.PURIN_FLOAT64 if tdtype == torch.float64 else _native.PURIN_FLOAT32
        full = _System(rows, n, me, code, device.index, device)
        row_ptr = np.zeros(len(rows) + 1, np.int64)
        row_ptr[1:] = np.cumsum([len(r) for r in rows])
        as_long = lambda a: torch.as_tensor(np.asarray(a, np.int64), device=device)
        set_("_device", device)
        set_("_tdtype", tdtype)
        set_("_full", full)
        set_("_m", len(rows))
        set_("_nnz", int(row_ptr[-1]))
        set_("_row_ell", as_long(ell_index(row_ptr)))
        set_("_slot_row", as_long(rows_of(row_ptr)))
        cols = np.asarray([j for r in rows for j in r], np.int64)
        set_("_cols", as_long(cols))
        # Padded columns: CSR slots per column in ascending row order (the reference's
        # scatter order), padding at slot nnz.
        per_col = [[] for _ in range(n)]
        for slot, j in enumerate(cols):
            per_col[j].append(slot)
        depth = max(1, max((len(c) for c in per_col), default=0))
        col_slots = np.full((n, depth), row_ptr[-1], np.int64)
        for j, c in enumerate(per_col):
            col_slots[j, :len(c)] = c
        set_("_col_slots", as_long(col_slots))
        set_("_col_rows", as_long(np.append(rows_of(row_ptr), len(rows))[col_slots]))
        # Row pairs nominated at theta = 0 and their compacted system.
        values0, _ = self.canonical.evaluate(torch.zeros((1, self.parameter_size),
                                                         dtype=torch.float64))
        v0 = values0.detach().cpu().numpy().reshape(-1)
        pairs = nominate_pairs(rows, [v0[row_ptr[r]:row_ptr[r + 1]] for r in range(len(rows))],
                               me, self.config.row_scaling)
        if pairs is None:
            set_("_pairs", None)
        else:
            keep, first, second, positions = pairs
            compact = _System([rows[r] for r in keep], n, me, code, device.index, device)
            slots = lambda rs: np.concatenate(
                [np.arange(row_ptr[r], row_ptr[r + 1]) for r in rs]) if rs else np.zeros(0)
            set_("_pairs", SimpleNamespace(
                keep=as_long(keep), first=as_long(first), second=as_long(second),
                positions=as_long(positions), keep_slots=as_long(slots(keep)),
                first_slots=as_long(slots(first)), second_slots=as_long(slots(second)),
                system=compact))
        cfg = self.config
        set_("_cfg", _native.AdmmConfig(
            float(cfg.sigma), float(cfg.alpha), int(cfg.max_iterations),
            int(cfg.cg_max_iterations), int(cfg.cg_refinement_steps), int(cfg.check_interval),
            float(cfg.cg_tolerance), int(bool(cfg.adaptive_rho)), int(cfg.rho_update_interval),
            float(cfg.rho_update_threshold)))
        lin = cfg.linear_solver
        set_("_lin", _native.LinearConfig(float(lin.tolerance), float(lin.atol), int(lin.restart),
                                          int(lin.max_iterations),
                                          float(cfg.implicit_gradient.adjoint_tolerance)))
        set_("_sample_offset", 0)
        set_("_total_batch", int(self.batch_size))
        set_("_lockstep_group", None)
        set_("_timers", None)
        set_("_last_linear", None)

    # -- sizes --------------------------------------------------------------------
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

    @property
    def _paired_rows(self):
        """The verified-pair plan (``admm/solver.py:58``), or None."""
        return self._pairs

    def set_shard(self, offset: int, total: int, group=None):
        """This layer's batch is rows ``offset..`` of a global batch of ``total``; with a
        ``torch.distributed`` group the VJP's GMRES shares the batch's budget (one
        all-reduce of two counters per cycle), as ``PreparedChambollePockProjection.set_shard``."""
        object.__setattr__(self, "_sample_offset", int(offset))
        object.__setattr__(self, "_total_batch", int(total))
        object.__setattr__(self, "_lockstep_group", group)

    def record_launches(self, timers):
        object.__setattr__(self, "_timers", timers)

    @contextlib.contextmanager
    def _timed(self, name):
        timers = self._timers
        with torch.cuda.nvtx.range("purin_admm_" + name):
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

    def _stream(self):
        return ctypes_stream(torch.cuda.current_stream(self._device))

    # -- ordered sparse products (chambolle_pock/kernels.py:43-49) -------------------
    def _mv(self, values, x):
        """K x with each row summed in slot order: values (1|B, nnz), x (B, n)."""
        if self._m == 0:
            return torch.zeros((x.shape[0], 0), dtype=x.dtype, device=x.device)
        pad = lambda t: torch.cat([t, t.new_zeros((t.shape[0], 1))], dim=1)
        vals, xp = pad(values), pad(x)
        cols = torch.cat([self._cols, torch.full_like(self._cols[:1], self.output_size)])
        acc = None
        for k in range(self._row_ell.shape[1]):
            slot = self._row_ell[:, k]
            term = vals[:, slot] * xp[:, cols[slot]]
            acc = term if acc is None else acc + term
        return acc

    def _tmv(self, values, w):
        """K^T w with each column summed in ascending row order."""
        pad = lambda t: torch.cat([t, t.new_zeros((t.shape[0], 1))], dim=1)
        vals, wp = pad(values), pad(w)
        acc = torch.zeros((w.shape[0], self.output_size), dtype=w.dtype, device=w.device)
        for k in range(self._col_slots.shape[1]):
            acc = acc + vals[:, self._col_slots[:, k]] * wp[:, self._col_rows[:, k]]
        return acc

    # -- native calls -------------------------------------------------------------------
    def _run_native(self, system, data, lower, upper, target, initial, tolerance):
        batch, n = target.shape
        m = system.m
        dev, dt = target.device, target.dtype
        penalty = torch.full((batch, m), float(self.config.rho), dtype=dt, device=dev)
        penalty[:, :self.equality_size] *= float(self.config.equality_rho_multiplier)
        q = torch.ones((batch, n), dtype=dt, device=dev)
        c = (-target).contiguous()
        empty = lambda *shape, dtype=dt: torch.empty(shape, dtype=dtype, device=dev)
        out = SimpleNamespace(x=empty(batch, n), z=empty(batch, m), dual=empty(batch, m),
                              rho=empty(batch, m), iterations=empty(batch, dtype=torch.int32),
                              inner=empty(batch, dtype=torch.int32), primal=empty(batch),
                              dual_res=empty(batch), linear=empty(batch),
                              converged=empty(batch, dtype=torch.uint8),
                              finite=empty(batch, dtype=torch.uint8))
        stride = 0 if data.shape[0] == 1 and batch != 1 else data.shape[1]
        data = data.contiguous()
        lower, upper, initial = lower.contiguous(), upper.contiguous(), initial.contiguous()
        args = _native.AdmmForwardArgs(
            batch, _ptr(q), _ptr(c), _ptr(data), stride, _ptr(lower), _ptr(upper), _ptr(penalty),
            _ptr(tolerance), _ptr(target), _ptr(initial), system.band, _ptr(out.x),
            _ptr(out.z), _ptr(out.dual), _ptr(out.rho), _ptr(out.iterations), _ptr(out.inner),
            _ptr(out.primal), _ptr(out.dual_res), _ptr(out.linear), _ptr(out.converged),
            _ptr(out.finite))
        ws_bytes = system.plan.admm_workspace_size(batch, system.width)
        ws = torch.empty((max(ws_bytes, 1),), dtype=torch.uint8, device=dev)
        with self._timed("forward"):
            system.plan.admm_forward(self._cfg, args, ws.data_ptr(), ws_bytes, self._stream())
        return out

    def _forward(self, data, rhs, target, initial, tolerance):
        """``admm/solver.py:99-160``: the custom-VJP forward on scaled arrays."""
        me = self.equality_size
        batch = target.shape[0]
        pairs = self._pairs
        use_pairs = False
        if pairs is not None:
            vals = data.expand(batch, -1)
            use_pairs = bool(torch.all(vals[:, pairs.first_slots] == -vals[:, pairs.second_slots])
                             & torch.all(-rhs[:, pairs.second] < rhs[:, pairs.first]))
        if use_pairs:
            # rows.py:33-51: two-sided rows on the compacted plan, duals restored.
            upper = rhs[:, pairs.keep]
            lower = torch.full_like(upper, -float("inf"))
            lower[:, :me] = upper[:, :me]
            lower[:, pairs.positions] = -rhs[:, pairs.second]
            init = initial[:, pairs.keep].clone()
            init[:, pairs.positions] = init[:, pairs.positions] + (-initial[:, pairs.second])
            out = self._run_native(pairs.system, data[:, pairs.keep_slots], lower, upper, target,
                                   init, tolerance)
            dual = torch.zeros_like(rhs)
            dual[:, pairs.keep] = out.dual
            signed = out.dual[:, pairs.positions]
            dual[:, pairs.first] = torch.clamp_min(signed, 0)
            dual[:, pairs.second] = torch.clamp_min(-signed, 0)
        else:
            lower = torch.cat([rhs[:, :me], torch.full_like(rhs[:, me:], -float("inf"))], dim=1)
            out = self._run_native(self._full, data, lower, rhs, target, initial, tolerance)
            dual = out.dual
        x = out.x
        half = torch.tensor(0.5, dtype=x.dtype, device=x.device)
        primal = torch.sum(half * x * x - target * x, dim=1)
        t = -target + self._tmv(data, dual)
        dual_objective = -half * torch.sum(t * t, dim=1) - torch.sum(rhs * dual, dim=1)
        one = torch.ones_like(primal)
        gap = torch.clamp_min(primal - dual_objective, 0) / torch.maximum(
            one, torch.maximum(primal.abs(), dual_objective.abs()))
        residual = torch.maximum(out.primal, torch.maximum(out.dual_res, out.linear))
        return x, dual, out.iterations, residual, gap, out.converged

    def _adjoint(self, data, rhs, y, dual, converged, gy, need):
        batch, n = y.shape
        m = self._m
        dev, dt = y.device, y.dtype
        g_values = torch.empty((batch, self._nnz), dtype=dt, device=dev) if need[0] else None
        g_rhs = torch.empty((batch, m), dtype=dt, device=dev) if need[1] else None
        g_target = torch.empty((batch, n), dtype=dt, device=dev) if need[2] else None
        status = torch.empty((batch,), dtype=torch.int32, device=dev)
        lres = torch.empty((batch,), dtype=dt, device=dev)
        err = torch.zeros((1,), dtype=torch.int32, device=dev)
        stride = 0 if data.shape[0] == 1 and batch != 1 else data.shape[1]
        data, rhs = data.contiguous(), rhs.contiguous()
        args = _native.AdmmAdjointArgs(
            batch, _ptr(data), stride, _ptr(rhs), _ptr(y), _ptr(dual), _ptr(converged), _ptr(gy),
            float(self.config.active_tolerance), float(self.config.tolerance),
            self._sample_offset, self._total_batch, _ptr(g_values), _ptr(g_rhs), _ptr(g_target),
            _ptr(status), _ptr(lres), _ptr(err))
        plan = self._full.plan
        ws_bytes = plan.admm_adjoint_workspace_size(batch, self._lin)
        ws = torch.empty((max(ws_bytes, 1),), dtype=torch.uint8, device=dev)
        keep = (data, rhs, y, dual, converged, gy)
        if self._lockstep_group is None:
            with self._timed("adjoint"):
                plan.admm_adjoint(self._lin, args, ws.data_ptr(), ws_bytes, self._stream())
        else:
            counters = torch.zeros((2,), dtype=torch.int32, device=dev)

            class _Shard:
                def _stage(shard, stage, completed=0):
                    with self._timed("adjoint"):
                        plan.admm_adjoint_stage(self._lin, args, stage, completed,
                                                counters.data_ptr(), ws.data_ptr(), ws_bytes,
                                                self._stream())
                    return counters

                def prepare(shard):
                    return shard._stage(_native.STAGE_PREPARE)

                def cycle(shard, completed):
                    return shard._stage(_native.STAGE_CYCLE, completed)

                def finish(shard):
                    shard._stage(_native.STAGE_FINISH)

            lockstep.run([_Shard()], int(self._lin.max_iterations), group=self._lockstep_group)
        del keep
        object.__setattr__(self, "_last_linear", (status, lres))
        if int(err.item()) != 0:
            raise RuntimeError("purin_admm_adjoint: a bounded device wait timed out; "
                               "gradients are invalid")
        return g_values, g_rhs, g_target

    # -- the prepared projection (chambolle_pock/solver.py:277-366) -------------------
    def _row_scale(self, values, batch):
        if not self.config.row_scaling or self._m == 0:
            return torch.ones((values.shape[0], self._m), dtype=values.dtype,
                              device=values.device)
        padded = torch.cat([values, torch.zeros_like(values[:, :1])], dim=1)
        acc = None
        for k in range(self._row_ell.shape[1]):
            v = padded[:, self._row_ell[:, k]]
            acc = v * v if acc is None else acc + v * v
        norms = torch.sqrt(acc)
        one = torch.ones_like(norms)
        return torch.where(norms > 0, one / torch.clamp_min(norms, 1e-30), one)

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
        theta = (torch.zeros((batch, 0), dtype=dt, device=dev) if self.parameter_size == 0
                 else torch.as_tensor(parameters, dtype=dt, device=dev))
        if tuple(theta.shape) != (batch, self.parameter_size):
            raise ValueError(f"parameters must have shape {(batch, self.parameter_size)}; "
                             f"got {tuple(theta.shape)}")
        if not self.config.implicit_gradient.differentiate_problem_parameters:
            theta = theta.detach()
        values, rhs = self.canonical.evaluate(theta)
        if rhs.shape[0] != batch:
            rhs = rhs.expand(batch, -1)
        scale = self._row_scale(values, batch)
        scale_b = scale.expand(batch, -1) if scale.shape[0] != batch else scale
        data = (values * scale[:, self._slot_row]).contiguous()
        scaled_rhs = (rhs * scale_b).contiguous()
        eq = (torch.zeros((batch, me), dtype=dt, device=dev) if multipliers_eq is None
              else torch.as_tensor(multipliers_eq, dtype=dt, device=dev))
        iq = (torch.zeros((batch, mi), dtype=dt, device=dev) if multipliers_ineq is None
              else torch.as_tensor(multipliers_ineq, dtype=dt, device=dev))
        if tuple(eq.shape) != (batch, me) or tuple(iq.shape) != (batch, mi):
            raise ValueError("warm-start multiplier shapes do not match constraints")
        initial = (torch.cat((eq, iq), dim=1) / scale_b).detach().contiguous()
        min_scale = (torch.clamp_max(scale_b.min(dim=1).values, 1.0) if self._m
                     else torch.ones((batch,), dtype=dt, device=dev))
        tolerance = (self.config.tolerance * torch.clamp_max(min_scale, 1.0)).detach().contiguous()
        y, dual_s, iterations, _, gap, conv = _ADMMSolve.apply(
            data, scaled_rhs, target.contiguous(), initial, tolerance, self)
        dual = dual_s * scale_b
        r = self._mv(values, y) - rhs
        eq_res = (torch.amax(r[:, :me].abs(), dim=1) if me
                  else torch.zeros((batch,), dtype=dt, device=dev))
        ineq_res = (torch.amax(torch.clamp_min(r[:, me:], 0), dim=1) if mi
                    else torch.zeros((batch,), dtype=dt, device=dev))
        stationarity = torch.amax((y - target + self._tmv(values, dual)).abs(), dim=1)
        residual = torch.maximum(torch.maximum(eq_res, ineq_res), stationarity)
        finite = (torch.isfinite(y).all(dim=1) & torch.isfinite(dual).all(dim=1)
                  & torch.isfinite(residual) & torch.isfinite(gap))
        converged = finite & (conv != 0) & (residual <= self.config.tolerance)
        status = torch.where(converged, int(SolveStatus.CONVERGED),
                             torch.where(finite, int(SolveStatus.MAX_ITERATIONS),
                                         int(SolveStatus.NONFINITE))).to(torch.int32)
        return ProjectionResult(y, dual[:, :me].detach(), dual[:, me:].detach(),
                                torch.clamp_min(-r[:, me:], 0).detach(), status, iterations,
                                residual.detach(), finite, converged)

    def solve(self, y_hat, parameters=None, initial_state=None):
        """Solve the prepared batched ADMM projection problem."""
        if initial_state is not None:
            raise ValueError("Use project_training multiplier arguments for ADMM warm starts")
        return self._solve(y_hat, parameters)

    def __call__(self, y_hat, parameters=None):
        result = self.solve(y_hat, parameters)
        return result.y[0] if torch.as_tensor(y_hat).ndim == 1 else result.y

    def with_info(self, y_hat, parameters=None):
        r = self.solve(y_hat, parameters)
        y = r.y[0] if torch.as_tensor(y_hat).ndim == 1 else r.y
        return y, ProjectionInfo(r.status, r.iterations, r.residual_inf_norm, r.finite,
                                 r.gradient_eligible)

    def project_training(self, y_hat, parameters=None, *, multipliers_eq=None,
                         multipliers_ineq=None):
        r = self._solve(y_hat, parameters, multipliers_eq, multipliers_ineq)
        return ProjectionTrainingOutput(r.y, r.multipliers_eq, r.multipliers_ineq, r.slacks,
                                        r.status, r.iterations, r.residual_inf_norm, r.finite,
                                        r.gradient_eligible)


class _ADMMSolve(torch.autograd.Function):
    """The custom-VJP solve of ``admm/solver.py:162-255`` as a torch autograd op."""

    @staticmethod
    def forward(ctx, data, rhs, target, initial, tolerance, layer):
        y, dual, iterations, residual, gap, converged = layer._forward(data, rhs, target,
                                                                       initial, tolerance)
        ctx.layer = layer
        ctx.shared_values = data.shape[0] == 1 and target.shape[0] != 1
        ctx.save_for_backward(data, rhs, y, dual, converged)
        ctx.mark_non_differentiable(dual, iterations, residual, gap, converged)
        return y, dual, iterations, residual, gap, converged

    @staticmethod
    def backward(ctx, gy, *unused):
        data, rhs, y, dual, converged = ctx.saved_tensors
        if gy is None:
            gy = torch.zeros_like(y)
        need = ctx.needs_input_grad
        g_values, g_rhs, g_target = ctx.layer._adjoint(data, rhs, y, dual, converged,
                                                       gy.contiguous(), need[:3])
        if g_values is not None and ctx.shared_values:
            g_values = g_values.sum(dim=0, keepdim=True)
        return g_values, g_rhs, g_target, None, None, None


@dataclass(frozen=True)
class ADMMProjection:
    """Definition of an ADMM distance projection for affine constraints."""

    problem: object
    config: ADMMConfig = field(default_factory=ADMMConfig)

    def prepare(self, *, batch_size, dtype=torch.float64, backend="cuda"):
        """Prepare reusable projection resources for a fixed batch size, dtype and backend."""
        if self.config.metric_diagonal is not None:
            from purin_b200.metric import prepare_diagonal_metric

            return prepare_diagonal_metric(self.problem, self.config, type(self),
                                           batch_size=batch_size, dtype=dtype, backend=backend)
        return PreparedADMMProjection(canonical_of(self.problem), self.config, int(batch_size),
                                      dtype, str(backend))
