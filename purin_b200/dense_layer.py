"""Batched dense / packed diagonal-QP CP adapter (``solve_dense_implicit``).

Mirrors ``src/purin/solvers/chambolle_pock/dense_layer.py:13-152`` (with
``dense.py:26-105``, ``dense_implicit.py:14-220``, ``sparse_layer.py`` for the
packed inequality rows and ``linalg/equilibration.py:21-57``): minimise
``0.5 sum(q y^2) + c.y`` subject to ``a y = b``, ``matrix y <= d`` and
``lower <= y <= upper`` for a batch, and differentiate the solution
implicitly.  It runs on the diagonal-QP kernels (``purin_qp_forward`` /
``purin_qp_adjoint``) in the variant of ``sparse_cp`` the dense adapter uses
(``dense.py:79-99``):

* factored proximal step ``inverse * ((y - tau K^T l) - tau c)`` clipped to
  the bounds, no stationarity test, no validity mask, power-iteration step
  sizes;
* no per-sample freeze: every sample runs the batch's trip count, the
  iteration at which the last sample is first accepted.  A first pass with
  freezing finds that count (a sample's iterates up to its first acceptance do
  not depend on freezing); when samples differ, a second pass without freezing
  resumes each sample from its first-pass state and runs it on to that count,
  so the kernels execute the batch's trip count per sample and no more;
* equality rows dense; inequality rows dense, or packed on
  ``inequality_support``.

The backward differentiates the same fixed point as ``dense_implicit.py:59-80,
207-217``: one CP step at the solution with the fixed steps
``tau = s/(max q + ||K||)``, ``sigma = s/||K||``, ``theta = 1`` and the
proximal inverse frozen, so ``q`` receives no gradient.  The reference solves
``(I - J^T) v = g`` with BiCGSTAB (relative tolerance 1e-6,
``adjoint_iterations`` steps); here restarted GMRES solves it
(``linear_solver``, default ``LinearSolverConfig()``, a tighter tolerance), so
the gradients agree with the reference's to its solver's accuracy.  A sample
whose GMRES ends above ``implicit_gradient.adjoint_tolerance`` gets a zero
gradient, where BiCGSTAB's last iterate would be returned.
"""

from __future__ import annotations

import contextlib
from numbers import Integral

import numpy as np
import torch

from purin_b200 import _native
from purin_b200.config import ChambollePockConfig, LinearSolverConfig
from purin_b200.diagonal_qp import QPStructure
from purin_b200.layer import _ptr, ctypes_stream, resolve_device

_SOLVERS: dict = {}
_TIMERS: list | None = None

_FIRST_PASS = (_native.QP_FACTORED_PROXIMAL | _native.QP_NO_STATIONARITY
               | _native.QP_NO_VALIDITY)


def record_launches(timers: list | None):
    """Collect (call, start_event, end_event) for every native call, or stop (None)."""
    global _TIMERS
    _TIMERS = timers


@contextlib.contextmanager
def _timed(name, device):
    """NVTX range around one native call; with ``record_launches`` also CUDA events."""
    timers = _TIMERS
    with torch.cuda.nvtx.range("purin_dense_" + name):
        if timers is None:
            yield
            return
        stream = torch.cuda.current_stream(device)
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        start.record(stream)
        yield
        end.record(stream)
        timers.append((name, start, end))


def max_abs_columns(matrix):
    """``equilibration.py:14-18``: max |entry| over rows per column (0 without rows)."""
    if matrix.shape[1] == 0:
        return torch.zeros((matrix.shape[0], matrix.shape[2]), dtype=matrix.dtype,
                           device=matrix.device)
    return matrix.abs().amax(dim=1)


def max_abs_rows(matrix):
    """``equilibration.py:7-11``: max |entry| along each row."""
    if matrix.shape[1] == 0:
        return torch.zeros((matrix.shape[0], 0), dtype=matrix.dtype, device=matrix.device)
    return matrix.abs().amax(dim=2)


def ruiz_equilibrate(q, c, A, b, C, d, lower, upper, *, iterations=4, eps=1e-6):
    """``equilibration.py:21-57``: column then row max-norm scaling, ``iterations`` passes.

    Returns ``(q, c, A, b, C, d, lower, upper, columns, equalities, inequalities)``
    as torch tensors; autograd differentiates through the scaling as JAX does.
    """
    columns = torch.ones_like(q)
    equalities, inequalities = torch.ones_like(b), torch.ones_like(d)
    epsilon = torch.tensor(eps, dtype=q.dtype, device=q.device)
    for _ in range(int(iterations)):
        metric = torch.maximum(max_abs_columns(A), max_abs_columns(C))
        metric = torch.maximum(metric, q.abs())
        update = 1.0 / torch.sqrt(torch.maximum(metric, epsilon))
        A, C = A * update[:, None, :], C * update[:, None, :]
        q, c = q * (update ** 2), c * update
        lower, upper, columns = lower / update, upper / update, columns * update
        if A.shape[1]:
            update = 1.0 / torch.sqrt(torch.maximum(max_abs_rows(A), epsilon))
            A, b, equalities = A * update[:, :, None], b * update, equalities * update
        if C.shape[1]:
            update = 1.0 / torch.sqrt(torch.maximum(max_abs_rows(C), epsilon))
            C, d, inequalities = C * update[:, :, None], d * update, inequalities * update
    return q, c, A, b, C, d, lower, upper, columns, equalities, inequalities


def inequality_rows(inequality_support, mi, n):
    """Column supports of the inequality rows: full rows, or the packed support,
    validated as ``sparse_layer.py:24-44`` does (one row per inequality; integer
    indices in [0, n), booleans excluded; no duplicates within a row)."""
    if inequality_support is None:
        return tuple(tuple(range(n)) for _ in range(mi))
    rows = tuple(tuple(row) for row in inequality_support)
    if len(rows) != mi:
        raise ValueError("inequality_support must have one row per inequality.")
    for row in rows:
        if any(not isinstance(i, Integral) or isinstance(i, bool) or i < 0 or i >= n for i in row):
            raise ValueError("Sparse support indices must be integers in [0, n).")
        if len(set(row)) != len(row):
            raise ValueError("Sparse support rows cannot contain duplicate indices.")
    return tuple(tuple(int(i) for i in row) for row in rows)


class _DenseSolver:
    """Plan and C-ABI configuration for one row layout, dtype, device and option set."""

    def __init__(self, n, me, mi_rows, dtype, device, cfg: ChambollePockConfig):
        structure = QPStructure(n, tuple(tuple(range(n)) for _ in range(me)), mi_rows)
        rows = structure.rows
        row_ptr = np.zeros(len(rows) + 1, dtype=np.int32)
        row_ptr[1:] = np.cumsum([len(r) for r in rows])
        col = np.asarray([j for r in rows for j in r], dtype=np.int32)
        self.plan = _native.Plan(n, me, len(mi_rows), row_ptr, col,
                                 _native.PURIN_FLOAT64 if dtype == torch.float64
                                 else _native.PURIN_FLOAT32, device.index, qp=True)
        self.n, self.me, self.m = n, me, me + len(mi_rows)
        self.device = device
        self.max_iterations = int(cfg.max_iterations)
        self.cfg = cfg
        self.last_work = []
        lin = cfg.linear_solver
        self.lin = _native.LinearConfig(float(lin.tolerance), float(lin.atol), int(lin.restart),
                                        int(lin.max_iterations),
                                        float(cfg.implicit_gradient.adjoint_tolerance))

    def cp_config(self, max_iterations):
        """Power-iteration steps, no norm bound, no diagonal preconditioning (dense.py:79-99)."""
        cfg = self.cfg
        return _native.CpConfig(int(max_iterations), int(bool(cfg.accelerated)),
                                float(cfg.safety), int(cfg.norm_iterations),
                                int(cfg.norm_seed), 0, 0, int(bool(cfg.prng_partitionable)))

    def stream(self):
        return ctypes_stream(torch.cuda.current_stream(self.device))

    def forward(self, inputs, max_iterations, flags, *, ybar0=None, start=None):
        """One ``purin_qp_forward`` call; ``ybar0`` and ``start`` resume an earlier one."""
        q, c, values, rhs, lower, upper, y0, dual0, tolerance = inputs
        batch, n = q.shape
        dev, dt = q.device, q.dtype
        out = dict(y=torch.empty((batch, n), dtype=dt, device=dev),
                   ybar=torch.empty((batch, n), dtype=dt, device=dev),
                   dual=torch.empty((batch, self.m), dtype=dt, device=dev),
                   iterations=torch.empty((batch,), dtype=torch.int32, device=dev),
                   residual=torch.empty((batch,), dtype=dt, device=dev),
                   gap=torch.empty((batch,), dtype=dt, device=dev),
                   converged=torch.empty((batch,), dtype=torch.uint8, device=dev))
        shared = values.shape[0] == 1 and batch != 1
        op = _native.QP_OP_FORWARD if shared else _native.QP_OP_FORWARD_SAMPLE_VALUES
        cfg = self.cp_config(max_iterations)
        ws_bytes = self.plan.workspace_size(op, batch, cfg)
        ws = torch.empty((max(ws_bytes, 1),), dtype=torch.uint8, device=dev)
        args = _native.QpForwardArgs(
            batch, _ptr(q), _ptr(c), _ptr(values), 0 if shared else values.shape[1], _ptr(rhs),
            _ptr(lower), _ptr(upper), n, _ptr(y0), _ptr(dual0), _ptr(tolerance), 0, batch,
            _ptr(out["y"]), _ptr(out["dual"]), _ptr(out["iterations"]), _ptr(out["residual"]),
            _ptr(out["gap"]), _ptr(out["converged"]), int(flags), _ptr(ybar0), _ptr(start),
            _ptr(out["ybar"]))
        with _timed("forward", self.device):
            self.plan.qp_forward(cfg, args, ws.data_ptr(), ws_bytes, self.stream())
        return out


class _DenseSolve(torch.autograd.Function):
    """``CP_fixed_implicit`` / ``CP_accelerated_implicit`` (dense_implicit.py:105-220)."""

    @staticmethod
    def forward(ctx, q, c, values, rhs, lower, upper, y0, dual0, tolerance, solver):
        inputs = (q, c, values, rhs, lower, upper, y0, dual0, tolerance)
        out = solver.forward(inputs, solver.max_iterations, _FIRST_PASS)
        iterations = out["iterations"]
        trips = int(iterations.max().item()) if iterations.numel() else 0
        # Iterations the kernels executed, per pass (sample-iterations).
        solver.last_work = [int(iterations.sum().item())]
        if bool((iterations != trips).any()):
            # Samples accepted before the last one keep iterating in the
            # reference's shared loop: each resumes from its state at its own
            # first acceptance (y, dual, ybar, iteration count) and runs on to
            # the batch's trip count.
            resumed = (q, c, values, rhs, lower, upper, out["y"], out["dual"], tolerance)
            out = solver.forward(resumed, trips, _FIRST_PASS | _native.QP_NO_FREEZE,
                                 ybar0=out["ybar"], start=iterations)
            solver.last_work.append(trips * iterations.numel() - solver.last_work[0])
        ctx.solver = solver
        ctx.save_for_backward(q, c, values, rhs, lower, upper, out["y"], out["dual"])
        ctx.mark_non_differentiable(out["iterations"])
        return out["y"], out["dual"], out["iterations"]

    @staticmethod
    def backward(ctx, gy, gdual, _unused):
        q, c, values, rhs, lower, upper, y, dual = ctx.saved_tensors
        solver = ctx.solver
        batch, n = q.shape
        m = rhs.shape[1]
        dev, dt = q.device, q.dtype
        shared = values.shape[0] == 1 and batch != 1
        gy = torch.zeros_like(y) if gy is None else gy.contiguous()
        cot_dual = gdual.contiguous() if (gdual is not None and m > 0) else None
        need = ctx.needs_input_grad
        out = lambda k, shape: torch.empty(shape, dtype=dt, device=dev) if need[k] else None
        g_c, g_values = out(1, (batch, n)), out(2, (batch, values.shape[1]))
        g_rhs, g_lower, g_upper = out(3, (batch, m)), out(4, (batch, n)), out(5, (batch, n))
        status = torch.empty((batch,), dtype=torch.int32, device=dev)
        lres = torch.empty((batch,), dtype=dt, device=dev)
        err = torch.zeros((1,), dtype=torch.int32, device=dev)
        # Every sample is differentiated: the reference applies no convergence mask.
        every = torch.ones((batch,), dtype=torch.uint8, device=dev)
        cfg = solver.cp_config(solver.max_iterations)
        ws_bytes = solver.plan.workspace_size(_native.QP_OP_ADJOINT, batch, cfg, solver.lin)
        ws = torch.empty((max(ws_bytes, 1),), dtype=torch.uint8, device=dev)
        args = _native.QpAdjointArgs(
            batch, _ptr(q), _ptr(c), _ptr(values), 0 if shared else values.shape[1], _ptr(rhs),
            _ptr(lower), _ptr(upper), n, _ptr(y), _ptr(dual), _ptr(every), _ptr(gy),
            _ptr(cot_dual), 0, batch, None, _ptr(g_c), _ptr(g_values), _ptr(g_rhs),
            _ptr(g_lower), _ptr(g_upper), _ptr(status), _ptr(lres), _ptr(err))
        with _timed("adjoint", solver.device):
            solver.plan.qp_adjoint(cfg, solver.lin, args, ws.data_ptr(), ws_bytes,
                                   solver.stream())
        if int(err.item()) != 0:
            raise RuntimeError("purin_qp_adjoint: a bounded device wait timed out; "
                               "gradients are invalid")
        if shared and g_values is not None:
            g_values = g_values.sum(dim=0, keepdim=True)
        # The proximal inverse is frozen (dense_implicit.py:1-5, 83-99): q gets no gradient.
        g_q = torch.zeros_like(q) if need[0] else None
        return g_q, g_c, g_values, g_rhs, g_lower, g_upper, None, None, None, None


def solve_dense_implicit(q, c, a, b, matrix, d, lower, upper, *, accelerated=False, safety=0.95,
                         norm_iterations=20, norm_seed=42, max_iterations=5000, tolerance=1e-9,
                         adjoint_iterations=50, equilibrate=False, equilibration_iterations=10,
                         y0=None, lambda0=None, mu0=None, inequality_support=None,
                         return_iterations=False, backend="cuda", linear_solver=None):
    """Solve batched diagonal QPs with the implicit-differentiable CP layer.

    Arguments and returns as ``dense_layer.py:13-152``: ``(y, equality
    multipliers, inequality multipliers)`` in the original coordinates, with
    the per-sample iteration count (the batch's shared trip count) appended
    when ``return_iterations``.  Inputs are torch tensors or array-likes; the
    computation runs on the CUDA device ``backend``.  ``adjoint_iterations``
    bounds the reference's BiCGSTAB and is accepted for the same call
    signature; the adjoint systems are solved by GMRES with ``linear_solver``.
    """
    del adjoint_iterations
    device = resolve_device(backend)
    raw = [torch.as_tensor(x, device=device) for x in (q, c, a, b, matrix, d, lower, upper)]
    dtype = torch.float64 if any(x.dtype == torch.float64 for x in raw) else torch.float32
    q, c, a, b, matrix, d, lower, upper = (x.to(dtype) for x in raw)
    if q.ndim != 2:
        raise ValueError("q must have shape (batch, n)")
    batch, n = q.shape
    shared = batch > 1 and a.ndim == 2 and matrix.ndim == 2 and not equilibrate
    if a.ndim == 2:
        a = a[None].expand(batch, -1, -1)
    if matrix.ndim == 2:
        matrix = matrix[None].expand(batch, -1, -1)
    me, mi = a.shape[1], matrix.shape[1]
    b, d, lower, upper = (torch.broadcast_to(v, (batch, v.shape[-1])) for v in (b, d, lower, upper))
    as_start = lambda v, k: (torch.zeros((batch, k), dtype=dtype, device=device) if v is None
                             else torch.as_tensor(v, dtype=dtype, device=device))
    y0, lambda0, mu0 = as_start(y0, n), as_start(lambda0, me), as_start(mu0, mi)
    if equilibrate:
        q, c, a, b, matrix, d, lower, upper, columns, eq_scale, iq_scale = ruiz_equilibrate(
            q, c, a, b, matrix, d, lower, upper, iterations=equilibration_iterations)
        y0 = y0 / columns
        lambda0 = lambda0 / torch.where(eq_scale == 0.0, torch.ones_like(eq_scale), eq_scale)
        mu0 = mu0 / torch.where(iq_scale == 0.0, torch.ones_like(iq_scale), iq_scale)
    mi_rows = inequality_rows(inequality_support, mi, n)
    cfg = ChambollePockConfig(accelerated=bool(accelerated), safety=float(safety),
                              norm_iterations=int(norm_iterations), norm_seed=int(norm_seed),
                              max_iterations=int(max_iterations), tolerance=float(tolerance),
                              norm_bound=False, row_scaling=False,
                              linear_solver=linear_solver or LinearSolverConfig())
    key = (n, me, mi_rows, dtype, device, cfg)
    solver = _SOLVERS.get(key)
    if solver is None:
        solver = _SOLVERS[key] = _DenseSolver(n, me, mi_rows, dtype, device, cfg)
    # Row values in the plan's order: dense equality rows, then the inequality
    # rows on their supports (sparse_layer.py packs the same entries).
    copies = 1 if shared else batch
    blocks = [a[:copies].reshape(copies, me * n)]
    if inequality_support is None:
        blocks.append(matrix[:copies].reshape(copies, mi * n))
    else:
        for i, row in enumerate(mi_rows):
            index = torch.as_tensor(row, dtype=torch.long, device=device)
            blocks.append(matrix[:copies, i].index_select(1, index))
    values = torch.cat(blocks, dim=1)
    rhs = torch.cat((b, d), dim=1)
    tol = torch.full((batch,), float(tolerance), dtype=dtype, device=device)
    y, dual, iterations = _DenseSolve.apply(
        q.contiguous(), c.contiguous(), values.contiguous(), rhs.contiguous(),
        lower.contiguous(), upper.contiguous(), y0.detach().contiguous(),
        torch.cat((lambda0, mu0), dim=1).detach().contiguous(), tol, solver)
    equality, inequality = dual[:, :me], dual[:, me:]
    if equilibrate:
        y, equality, inequality = columns * y, eq_scale * equality, iq_scale * inequality
    if return_iterations:
        return y, equality, inequality, iterations
    return y, equality, inequality
