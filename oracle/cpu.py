"""C++ restatement of the CP loop on the host cores (``oracle/cp_cpu.cpp``).

Oracle (test and baseline infrastructure): ``sparse_cp_native`` has the
signature of :func:`oracle.cp.sparse_cp` for the projection layer's call
(q = 1, c = -target, y0 = target, freeze and stationarity on, fp64) and is used
by the CPU baseline in bench.py; tests check it against the NumPy loop.  Step
sizes come from the NumPy restatement (:func:`oracle.cp.step_sizes`).
"""

from __future__ import annotations

import ctypes

import numpy as np

from oracle.build import LIB, build
from oracle.cp import CPOutput, step_sizes

_lib = None


def _load():
    global _lib
    if _lib is None:
        if not LIB.exists():
            build()
        lib = ctypes.CDLL(str(LIB))
        lib.oracle_cp_solve.restype = ctypes.c_int
        _lib = lib
    return _lib


def _ptr(a):
    return a.ctypes.data_as(ctypes.c_void_p)


def sparse_cp_native(q, c, values, rhs, support, mask, me, lower, upper, *, accelerated=False,
                     safety=0.95, max_iterations=5000, tolerance=1e-9, norm_iterations=20,
                     norm_seed=42, y0=None, dual0=None, freeze_converged=False,
                     check_stationarity=False, norm_bound=False,
                     diagonal_preconditioning=False, offset=0, total=None, partitionable=True,
                     threads=None):
    """``kernels.py:178-305`` for the projection layer's arguments, on the host cores."""
    batch, n = q.shape
    dtype = np.dtype(q.dtype)
    if dtype != np.float64 or not np.all(q == 1) or not freeze_converged or not check_stationarity:
        raise ValueError("the C++ loop covers the fp64 projection call (q = 1, freeze, "
                         "stationarity)")
    if diagonal_preconditioning and not accelerated:
        raise ValueError("the C++ loop takes scalar step sizes")
    target = -np.asarray(c, dtype)
    if y0 is not None and not np.array_equal(np.asarray(y0, dtype), target):
        raise ValueError("the C++ loop starts from y0 = target")
    tau, sigma = step_sizes(q, values, support, mask, rhs, accelerated=accelerated,
                            safety=safety, norm_iterations=norm_iterations, norm_seed=norm_seed,
                            norm_bound=norm_bound,
                            diagonal_preconditioning=diagonal_preconditioning, offset=offset,
                            total=total, partitionable=partitionable)
    m, width = support.shape
    vals = np.ascontiguousarray(values, dtype)
    stride = 0 if vals.ndim == 2 or vals.shape[0] == 1 else m * width
    args = [np.ascontiguousarray(a, dtype) for a in (rhs, target, lower, upper)]
    dual = (np.zeros((batch, m), dtype) if dual0 is None
            else np.ascontiguousarray(dual0, dtype))
    tol = np.ascontiguousarray(np.broadcast_to(np.asarray(tolerance, dtype), (batch,)))
    tau = np.ascontiguousarray(tau, dtype)
    sigma = np.ascontiguousarray(sigma, dtype)
    sup = np.ascontiguousarray(support, np.int32)
    msk = np.ascontiguousarray(mask, np.uint8)
    y_out = np.empty((batch, n), dtype)
    d_out = np.empty((batch, m), dtype)
    it_out = np.empty(batch, np.int32)
    res_out = np.empty(batch, dtype)
    gap_out = np.empty(batch, dtype)
    conv_out = np.empty(batch, np.uint8)
    lib = _load()
    status = lib.oracle_cp_solve(
        ctypes.c_int(0 if threads is None else int(threads)), ctypes.c_int(batch),
        ctypes.c_int(n), ctypes.c_int(m), ctypes.c_int(me), ctypes.c_int(width), _ptr(sup), _ptr(msk), _ptr(vals), ctypes.c_int64(stride),
        *[_ptr(a) for a in args], _ptr(dual), _ptr(tol), _ptr(tau), _ptr(sigma),
        ctypes.c_int(1 if accelerated else 0), ctypes.c_int(int(max_iterations)),
        _ptr(y_out), _ptr(d_out), _ptr(it_out), _ptr(res_out), _ptr(gap_out), _ptr(conv_out))
    if status != 0:
        raise RuntimeError(f"oracle_cp_solve failed with status {status}")
    return CPOutput(y_out, d_out, it_out, res_out, gap_out, conv_out.astype(bool))
