"""ctypes binding of ``libpurin_cp.so`` (the C ABI declared in include/purin_cp.h).

The library is built in tree (``python -m purin_b200.csrc.build``) into
``purin_b200/_lib/``.  There is no fallback: if the library or a CUDA device
is missing, every entry point raises.
"""

from __future__ import annotations

import ctypes
from pathlib import Path

import numpy as np

_LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libpurin_cp.so"
ABI_VERSION = 3

PURIN_FLOAT64, PURIN_FLOAT32 = 0, 1
OP_FORWARD, OP_ADJOINT, QP_OP_FORWARD, QP_OP_ADJOINT = 0, 1, 2, 3
OP_FORWARD_SAMPLE_VALUES, QP_OP_FORWARD_SAMPLE_VALUES = 4, 5
STAGE_PREPARE, STAGE_CYCLE, STAGE_FINISH = 0, 1, 2
KEPT_ROWS, KEPT_SLOTS, BOUND_ROWS, BOUND_SLOTS, BOUND_VARIABLES, KEPT_ROW_PTR, KEPT_COLS = range(7)

c_i32, c_i64, c_dbl, c_vp = ctypes.c_int32, ctypes.c_int64, ctypes.c_double, ctypes.c_void_p
c_i32p = ctypes.POINTER(ctypes.c_int32)
c_u8p = ctypes.POINTER(ctypes.c_uint8)


class Structure(ctypes.Structure):
    _fields_ = [("n", c_i32), ("equality_size", c_i32), ("inequality_size", c_i32),
                ("row_ptr", c_i32p), ("col", c_i32p), ("dtype", c_i32), ("device", c_i32)]


class PlanInfo(ctypes.Structure):
    _fields_ = [("n", c_i32), ("equality_size", c_i32), ("inequality_size", c_i32),
                ("kept_rows", c_i32), ("kept_nnz", c_i32), ("bound_rows", c_i32), ("nnz", c_i32),
                ("width", c_i32), ("dtype", c_i32), ("device", c_i32)]


class CpConfig(ctypes.Structure):
    _fields_ = [("max_iterations", c_i32), ("accelerated", c_i32), ("safety", c_dbl),
                ("norm_iterations", c_i32), ("norm_seed", c_i64), ("norm_bound", c_i32),
                ("diagonal_preconditioning", c_i32), ("prng_partitionable", c_i32)]


class LinearConfig(ctypes.Structure):
    _fields_ = [("tolerance", c_dbl), ("atol", c_dbl), ("restart", c_i32),
                ("max_iterations", c_i32), ("adjoint_tolerance", c_dbl)]


class ForwardArgs(ctypes.Structure):
    _fields_ = [("batch", c_i64), ("values", c_vp), ("values_stride", c_i64), ("rhs", c_vp),
                ("target", c_vp), ("dual0", c_vp), ("tolerance", c_vp), ("lower", c_vp),
                ("upper", c_vp), ("bounds_stride", c_i64), ("feasible", c_vp),
                ("sample_offset", c_i64), ("total_batch", c_i64), ("y", c_vp), ("dual", c_vp),
                ("iterations", c_vp), ("residual", c_vp), ("gap", c_vp), ("converged", c_vp)]


class AdjointArgs(ctypes.Structure):
    _fields_ = [("batch", c_i64), ("values", c_vp), ("values_stride", c_i64), ("rhs", c_vp),
                ("target", c_vp), ("lower", c_vp), ("upper", c_vp), ("bounds_stride", c_i64),
                ("y", c_vp), ("dual", c_vp), ("converged", c_vp), ("cot_y", c_vp),
                ("sample_offset", c_i64), ("total_batch", c_i64), ("grad_values", c_vp),
                ("grad_rhs", c_vp), ("grad_target", c_vp), ("grad_lower", c_vp),
                ("grad_upper", c_vp), ("linear_status", c_vp), ("linear_residual", c_vp),
                ("device_error", c_vp), ("arnoldi_steps", c_vp), ("krylov_vectors", c_vp)]


class QpForwardArgs(ctypes.Structure):
    _fields_ = [("batch", c_i64), ("q", c_vp), ("c", c_vp), ("values", c_vp),
                ("values_stride", c_i64), ("rhs", c_vp), ("lower", c_vp), ("upper", c_vp),
                ("bounds_stride", c_i64), ("y0", c_vp), ("dual0", c_vp), ("tolerance", c_vp),
                ("sample_offset", c_i64), ("total_batch", c_i64), ("y", c_vp), ("dual", c_vp),
                ("iterations", c_vp), ("residual", c_vp), ("gap", c_vp), ("converged", c_vp),
                ("flags", c_i32), ("ybar0", c_vp), ("start_iterations", c_vp), ("ybar", c_vp)]


QP_FACTORED_PROXIMAL, QP_NO_STATIONARITY, QP_NO_FREEZE, QP_NO_VALIDITY = 1, 2, 4, 8


class QpAdjointArgs(ctypes.Structure):
    _fields_ = [("batch", c_i64), ("q", c_vp), ("c", c_vp), ("values", c_vp),
                ("values_stride", c_i64), ("rhs", c_vp), ("lower", c_vp), ("upper", c_vp),
                ("bounds_stride", c_i64), ("y", c_vp), ("dual", c_vp), ("converged", c_vp),
                ("cot_y", c_vp), ("cot_dual", c_vp), ("sample_offset", c_i64),
                ("total_batch", c_i64), ("grad_q", c_vp), ("grad_c", c_vp),
                ("grad_values", c_vp), ("grad_rhs", c_vp), ("grad_lower", c_vp),
                ("grad_upper", c_vp), ("linear_status", c_vp), ("linear_residual", c_vp),
                ("device_error", c_vp), ("arnoldi_steps", c_vp), ("krylov_vectors", c_vp)]


class PostArgs(ctypes.Structure):
    _fields_ = [("batch", c_i64), ("values_all", c_vp), ("values_all_stride", c_i64),
                ("rhs_all", c_vp), ("target", c_vp), ("lower", c_vp), ("upper", c_vp),
                ("bounds_stride", c_i64), ("scale", c_vp), ("y", c_vp), ("dual", c_vp),
                ("gap", c_vp), ("cp_converged", c_vp), ("tolerance", c_dbl),
                ("multipliers_eq", c_vp), ("multipliers_ineq", c_vp), ("slacks", c_vp),
                ("status", c_vp), ("residual_inf_norm", c_vp), ("finite", c_vp),
                ("gradient_eligible", c_vp)]


class AdmmConfig(ctypes.Structure):
    _fields_ = [("sigma", c_dbl), ("alpha", c_dbl), ("max_iterations", c_i32),
                ("cg_max_iterations", c_i32), ("cg_refinement_steps", c_i32),
                ("check_interval", c_i32), ("cg_tolerance", c_dbl), ("adaptive_rho", c_i32),
                ("rho_update_interval", c_i32), ("rho_update_threshold", c_dbl)]


class AdmmBand(ctypes.Structure):
    _fields_ = [("width", c_i32), ("entries", c_i32), ("permutation", c_vp), ("inverse", c_vp),
                ("rows", c_vp), ("slot_left", c_vp), ("slot_right", c_vp),
                ("destination", c_vp)]


class AdmmForwardArgs(ctypes.Structure):
    _fields_ = [("batch", c_i64), ("q", c_vp), ("c", c_vp), ("values", c_vp),
                ("values_stride", c_i64), ("lower", c_vp), ("upper", c_vp), ("penalty", c_vp),
                ("tolerance", c_vp), ("x0", c_vp), ("dual0", c_vp), ("band", AdmmBand),
                ("x", c_vp), ("z", c_vp), ("dual", c_vp), ("penalty_out", c_vp),
                ("iterations", c_vp), ("inner_iterations", c_vp), ("primal_residual", c_vp),
                ("dual_residual", c_vp), ("linear_residual", c_vp), ("converged", c_vp),
                ("finite", c_vp)]


class AdmmAdjointArgs(ctypes.Structure):
    _fields_ = [("batch", c_i64), ("values", c_vp), ("values_stride", c_i64), ("rhs", c_vp),
                ("y", c_vp), ("dual", c_vp), ("converged", c_vp), ("cot_y", c_vp),
                ("active_tolerance", c_dbl), ("tolerance", c_dbl), ("sample_offset", c_i64),
                ("total_batch", c_i64), ("grad_values", c_vp), ("grad_rhs", c_vp),
                ("grad_target", c_vp), ("linear_status", c_vp), ("linear_residual", c_vp),
                ("device_error", c_vp)]


EXPORTED = (
    "purin_cp_abi_version", "purin_cp_last_error", "purin_cp_plan_create",
    "purin_cp_plan_destroy", "purin_cp_plan_info", "purin_cp_plan_indices",
    "purin_cp_workspace_size", "purin_cp_forward_shape", "purin_cp_forward", "purin_cp_adjoint",
    "purin_cp_adjoint_stage",
    "purin_cp_postprocess", "purin_qp_plan_create", "purin_qp_forward", "purin_qp_adjoint",
    "purin_qp_adjoint_stage", "purin_admm_workspace_size", "purin_admm_forward",
    "purin_admm_adjoint_workspace_size", "purin_admm_adjoint", "purin_admm_adjoint_stage",
)

_lib = None


class NativeError(RuntimeError):
    """A C ABI call returned a nonzero PurinStatus."""


def library_path() -> Path:
    return _LIB_PATH


def load():
    """Load and type the shared library (raises if it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    if not _LIB_PATH.exists():
        raise RuntimeError(f"{_LIB_PATH} is not built; run `python -m purin_b200.csrc.build` "
                           "(the CP projection has no CPU fallback)")
    lib = ctypes.CDLL(str(_LIB_PATH))
    lib.purin_cp_abi_version.restype = c_i32
    lib.purin_cp_last_error.restype = ctypes.c_char_p
    lib.purin_cp_plan_create.argtypes = [ctypes.POINTER(Structure), ctypes.POINTER(c_vp)]
    lib.purin_cp_plan_destroy.argtypes = [c_vp]
    lib.purin_cp_plan_info.argtypes = [c_vp, ctypes.POINTER(PlanInfo)]
    lib.purin_cp_plan_indices.argtypes = [c_vp, c_i32, c_i32p]
    lib.purin_cp_workspace_size.argtypes = [c_vp, c_i32, c_i64, ctypes.POINTER(CpConfig),
                                            ctypes.POINTER(LinearConfig),
                                            ctypes.POINTER(ctypes.c_size_t)]
    lib.purin_cp_forward_shape.argtypes = [c_vp, ctypes.POINTER(CpConfig), c_i64, c_i32, c_i32p,
                                           c_i32p, c_i32p]
    lib.purin_cp_forward.argtypes = [c_vp, ctypes.POINTER(CpConfig), ctypes.POINTER(ForwardArgs),
                                     c_vp, ctypes.c_size_t, c_vp]
    lib.purin_cp_adjoint.argtypes = [c_vp, ctypes.POINTER(CpConfig), ctypes.POINTER(LinearConfig),
                                     ctypes.POINTER(AdjointArgs), c_vp, ctypes.c_size_t, c_vp]
    lib.purin_cp_adjoint_stage.argtypes = [c_vp, ctypes.POINTER(CpConfig),
                                           ctypes.POINTER(LinearConfig),
                                           ctypes.POINTER(AdjointArgs), c_i32, c_i32, c_vp, c_vp,
                                           ctypes.c_size_t, c_vp]
    lib.purin_cp_postprocess.argtypes = [c_vp, ctypes.POINTER(PostArgs), c_vp]
    lib.purin_qp_plan_create.argtypes = [ctypes.POINTER(Structure), ctypes.POINTER(c_vp)]
    lib.purin_qp_forward.argtypes = [c_vp, ctypes.POINTER(CpConfig), ctypes.POINTER(QpForwardArgs),
                                     c_vp, ctypes.c_size_t, c_vp]
    lib.purin_qp_adjoint.argtypes = [c_vp, ctypes.POINTER(CpConfig), ctypes.POINTER(LinearConfig),
                                     ctypes.POINTER(QpAdjointArgs), c_vp, ctypes.c_size_t, c_vp]
    lib.purin_qp_adjoint_stage.argtypes = [c_vp, ctypes.POINTER(CpConfig),
                                           ctypes.POINTER(LinearConfig),
                                           ctypes.POINTER(QpAdjointArgs), c_i32, c_i32, c_vp, c_vp,
                                           ctypes.c_size_t, c_vp]
    lib.purin_admm_workspace_size.argtypes = [c_vp, c_i64, c_i32, ctypes.POINTER(ctypes.c_size_t)]
    lib.purin_admm_forward.argtypes = [c_vp, ctypes.POINTER(AdmmConfig),
                                       ctypes.POINTER(AdmmForwardArgs), c_vp, ctypes.c_size_t, c_vp]
    lib.purin_admm_adjoint_workspace_size.argtypes = [c_vp, c_i64, ctypes.POINTER(LinearConfig),
                                                      ctypes.POINTER(ctypes.c_size_t)]
    lib.purin_admm_adjoint.argtypes = [c_vp, ctypes.POINTER(LinearConfig),
                                       ctypes.POINTER(AdmmAdjointArgs), c_vp, ctypes.c_size_t, c_vp]
    lib.purin_admm_adjoint_stage.argtypes = [c_vp, ctypes.POINTER(LinearConfig),
                                             ctypes.POINTER(AdmmAdjointArgs), c_i32, c_i32, c_vp,
                                             c_vp, ctypes.c_size_t, c_vp]
    for name in ("purin_admm_workspace_size", "purin_admm_forward",
                 "purin_admm_adjoint_workspace_size", "purin_admm_adjoint",
                 "purin_admm_adjoint_stage"):
        getattr(lib, name).restype = c_i32
    for name in ("purin_cp_plan_create", "purin_cp_plan_destroy", "purin_cp_plan_info",
                 "purin_cp_plan_indices", "purin_cp_workspace_size", "purin_cp_forward_shape",
                 "purin_cp_forward",
                 "purin_cp_adjoint", "purin_cp_adjoint_stage", "purin_cp_postprocess",
                 "purin_qp_plan_create", "purin_qp_forward", "purin_qp_adjoint",
                 "purin_qp_adjoint_stage"):
        getattr(lib, name).restype = c_i32
    version = lib.purin_cp_abi_version()
    if version != ABI_VERSION:
        raise RuntimeError(f"libpurin_cp ABI version {version} != {ABI_VERSION}")
    _lib = lib
    return lib


def check(status: int, what: str):
    if status != 0:
        message = load().purin_cp_last_error().decode(errors="replace")
        raise NativeError(f"{what} failed (status {status}): {message}")


class Plan:
    """Owning handle of a ``PurinCpPlan`` (immutable device-resident structure)."""

    def __init__(self, n, me, mi, row_ptr, col, dtype_code, device, qp=False):
        lib = load()
        self._lib = lib
        self._row_ptr = np.ascontiguousarray(row_ptr, dtype=np.int32)
        self._col = np.ascontiguousarray(col, dtype=np.int32)
        if self._col.size == 0:
            self._col = np.zeros(1, dtype=np.int32)
        s = Structure(int(n), int(me), int(mi),
                      self._row_ptr.ctypes.data_as(c_i32p), self._col.ctypes.data_as(c_i32p),
                      int(dtype_code), int(device))
        handle = c_vp()
        create = "purin_qp_plan_create" if qp else "purin_cp_plan_create"
        check(getattr(lib, create)(ctypes.byref(s), ctypes.byref(handle)), create)
        self.handle = handle
        info = PlanInfo()
        check(lib.purin_cp_plan_info(handle, ctypes.byref(info)), "purin_cp_plan_info")
        self.info = info

    def indices(self, which: int) -> np.ndarray:
        sizes = {
            KEPT_ROWS: self.info.kept_rows, KEPT_SLOTS: self.info.kept_nnz,
            BOUND_ROWS: self.info.bound_rows, BOUND_SLOTS: self.info.bound_rows,
            BOUND_VARIABLES: self.info.bound_rows, KEPT_ROW_PTR: self.info.kept_rows + 1,
            KEPT_COLS: self.info.kept_nnz,
        }
        out = np.zeros(max(sizes[which], 1), dtype=np.int32)
        check(self._lib.purin_cp_plan_indices(self.handle, int(which), out.ctypes.data_as(c_i32p)),
              "purin_cp_plan_indices")
        return out[: sizes[which]]

    def workspace_size(self, op, batch, cfg: CpConfig, lin: LinearConfig | None = None) -> int:
        size = ctypes.c_size_t()
        check(self._lib.purin_cp_workspace_size(
            self.handle, int(op), int(batch), ctypes.byref(cfg),
            ctypes.byref(lin) if lin is not None else None, ctypes.byref(size)),
            "purin_cp_workspace_size")
        return int(size.value)

    def forward_shape(self, cfg: CpConfig, batch: int, shared_values: bool = True):
        """(samples per tile, threads per CTA, tile state in shared memory) of a forward call."""
        out = [ctypes.c_int32() for _ in range(3)]
        check(self._lib.purin_cp_forward_shape(self.handle, ctypes.byref(cfg), int(batch),
                                               int(bool(shared_values)),
                                               *[ctypes.byref(o) for o in out]),
              "purin_cp_forward_shape")
        return out[0].value, out[1].value, bool(out[2].value)

    def forward(self, cfg, args, workspace_ptr, workspace_bytes, stream):
        check(self._lib.purin_cp_forward(self.handle, ctypes.byref(cfg), ctypes.byref(args),
                                         workspace_ptr, workspace_bytes, stream), "purin_cp_forward")

    def adjoint(self, cfg, lin, args, workspace_ptr, workspace_bytes, stream):
        check(self._lib.purin_cp_adjoint(self.handle, ctypes.byref(cfg), ctypes.byref(lin),
                                         ctypes.byref(args), workspace_ptr, workspace_bytes,
                                         stream), "purin_cp_adjoint")

    def adjoint_stage(self, cfg, lin, args, stage, completed, counters_ptr, workspace_ptr,
                      workspace_bytes, stream):
        check(self._lib.purin_cp_adjoint_stage(self.handle, ctypes.byref(cfg), ctypes.byref(lin),
                                               ctypes.byref(args), stage, completed, counters_ptr,
                                               workspace_ptr, workspace_bytes, stream),
              "purin_cp_adjoint_stage")

    def qp_forward(self, cfg, args, workspace_ptr, workspace_bytes, stream):
        check(self._lib.purin_qp_forward(self.handle, ctypes.byref(cfg), ctypes.byref(args),
                                         workspace_ptr, workspace_bytes, stream), "purin_qp_forward")

    def qp_adjoint(self, cfg, lin, args, workspace_ptr, workspace_bytes, stream):
        check(self._lib.purin_qp_adjoint(self.handle, ctypes.byref(cfg), ctypes.byref(lin),
                                         ctypes.byref(args), workspace_ptr, workspace_bytes,
                                         stream), "purin_qp_adjoint")

    def qp_adjoint_stage(self, cfg, lin, args, stage, completed, counters_ptr, workspace_ptr,
                         workspace_bytes, stream):
        check(self._lib.purin_qp_adjoint_stage(self.handle, ctypes.byref(cfg), ctypes.byref(lin),
                                               ctypes.byref(args), stage, completed, counters_ptr,
                                               workspace_ptr, workspace_bytes, stream),
              "purin_qp_adjoint_stage")

    def admm_workspace_size(self, batch, band_width) -> int:
        size = ctypes.c_size_t()
        check(self._lib.purin_admm_workspace_size(self.handle, int(batch), int(band_width),
                                                  ctypes.byref(size)), "purin_admm_workspace_size")
        return int(size.value)

    def admm_forward(self, cfg, args, workspace_ptr, workspace_bytes, stream):
        check(self._lib.purin_admm_forward(self.handle, ctypes.byref(cfg), ctypes.byref(args),
                                           workspace_ptr, workspace_bytes, stream),
              "purin_admm_forward")

    def admm_adjoint_workspace_size(self, batch, lin) -> int:
        size = ctypes.c_size_t()
        check(self._lib.purin_admm_adjoint_workspace_size(self.handle, int(batch), ctypes.byref(lin),
                                                          ctypes.byref(size)),
              "purin_admm_adjoint_workspace_size")
        return int(size.value)

    def admm_adjoint(self, lin, args, workspace_ptr, workspace_bytes, stream):
        check(self._lib.purin_admm_adjoint(self.handle, ctypes.byref(lin), ctypes.byref(args),
                                           workspace_ptr, workspace_bytes, stream),
              "purin_admm_adjoint")

    def admm_adjoint_stage(self, lin, args, stage, completed, counters_ptr, workspace_ptr,
                           workspace_bytes, stream):
        check(self._lib.purin_admm_adjoint_stage(self.handle, ctypes.byref(lin), ctypes.byref(args),
                                                 stage, completed, counters_ptr, workspace_ptr,
                                                 workspace_bytes, stream),
              "purin_admm_adjoint_stage")

    def postprocess(self, args, stream):
        check(self._lib.purin_cp_postprocess(self.handle, ctypes.byref(args), stream),
              "purin_cp_postprocess")

    def __del__(self):
        handle = getattr(self, "handle", None)
        if handle is not None and handle.value:
            try:
                self._lib.purin_cp_plan_destroy(handle)
            except Exception:  # pragma: no cover - interpreter shutdown
                pass
            self.handle = None


def exported_symbols():
    """Names of every entry point declared in include/purin_cp.h that the library exports."""
    lib = ctypes.CDLL(str(_LIB_PATH))
    return {name: hasattr(lib, name) for name in EXPORTED}

