"""purin_cp_forward_noalloc: the forward solve for callers that cannot allocate.

Some callers cannot allocate device memory -- a plugin or custom-call hook
that only receives its input and output buffers, a framework that already
reserved almost all of the GPU for its own allocator.  For them the library
keeps the forward solve's scratch in one fixed device array instead of taking
a caller-provided workspace.  This test calls that entry point through the C
ABI twice in a row, on different problems, and checks that every output equals
the one purin_cp_forward produces with a caller-provided workspace (bit for
bit, the forward parity tests' tolerance).  It lives in its own file, collected
last, so a run that stops at the first failure has run every other test first.
"""

import ctypes

import numpy as np
import pytest
import torch
from dataclasses import replace

from helpers import OracleLayer, ell_to_csr
from purin_b200 import _native, prepare_projection
from purin_b200.workloads import make_workload

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _t(a, dtype):
    return torch.as_tensor(np.ascontiguousarray(a), dtype=dtype, device=DEV)


def _outputs(batch, n, m, dtype):
    return dict(y=torch.empty((batch, n), dtype=dtype, device=DEV),
                dual=torch.empty((batch, m), dtype=dtype, device=DEV),
                iterations=torch.empty((batch,), dtype=torch.int32, device=DEV),
                residual=torch.empty((batch,), dtype=dtype, device=DEV),
                gap=torch.empty((batch,), dtype=dtype, device=DEV),
                converged=torch.empty((batch,), dtype=torch.uint8, device=DEV))


def _case(index, batch, dtype, seed):
    w = make_workload(index, batch, seed=seed)
    cfg = replace(w.config, max_iterations=min(w.config.max_iterations, 300))
    oracle = OracleLayer(w.problem, cfg, dtype)
    _, saved = oracle.solve(w.candidates, w.theta)
    tdt = torch.float64 if dtype == np.float64 else torch.float32
    layer = prepare_projection(w.problem, method="chambolle-pock", config=cfg, batch_size=batch,
                               dtype=tdt, backend=DEV)
    inputs = dict(
        data=_t(ell_to_csr(saved["values"], list(oracle.proj.mask.sum(axis=1))), tdt)[:1].contiguous(),
        rhs=_t(saved["rhs"], tdt), target=_t(saved["target"], tdt),
        lower=_t(saved["lower"], tdt), upper=_t(saved["upper"], tdt),
        initial=_t(saved["initial"], tdt), tolerance=_t(saved["tolerance"], tdt),
        feasible=_t(saved["feasible"].astype(np.uint8), torch.uint8))
    return layer, inputs, tdt


def _noalloc(layer, inputs, out):
    lib = _native.load()
    fn = lib.purin_cp_forward_noalloc
    fn.argtypes = [ctypes.c_void_p, ctypes.POINTER(_native.CpConfig),
                   ctypes.POINTER(_native.ForwardArgs), ctypes.c_void_p]
    fn.restype = ctypes.c_int32
    batch, n = inputs["target"].shape
    p = lambda t: t.data_ptr()
    args = _native.ForwardArgs(
        batch, p(inputs["data"]), 0, p(inputs["rhs"]), p(inputs["target"]), p(inputs["initial"]),
        p(inputs["tolerance"]), p(inputs["lower"]), p(inputs["upper"]), n, p(inputs["feasible"]),
        0, batch, p(out["y"]), p(out["dual"]), p(out["iterations"]), p(out["residual"]),
        p(out["gap"]), p(out["converged"]))
    status = fn(layer._plan.handle, ctypes.byref(layer._cfg), ctypes.byref(args),
                torch.cuda.current_stream().cuda_stream)
    _native.check(status, "purin_cp_forward_noalloc")


def test_noalloc_forward_matches_workspace_forward_twice():
    cases = [(0, 16, np.float64, 0), (1, 8, np.float64, 1)]
    for index, batch, dtype, seed in cases:
        layer, inputs, tdt = _case(index, batch, dtype, seed)
        n, m = layer.output_size, layer._m
        want = _outputs(batch, n, m, tdt)
        layer._forward_native(inputs["data"], inputs["rhs"], inputs["target"], inputs["lower"],
                              inputs["upper"], inputs["initial"], inputs["tolerance"],
                              inputs["feasible"], want["y"], want["dual"], want["iterations"],
                              want["residual"], want["gap"], want["converged"])
        got = _outputs(batch, n, m, tdt)
        _noalloc(layer, inputs, got)
        torch.cuda.synchronize()
        for key in want:
            np.testing.assert_array_equal(got[key].cpu().numpy(), want[key].cpu().numpy(),
                                          err_msg=f"config {index}: {key}")


def test_noalloc_rejects_scratch_beyond_its_fixed_size():
    """A call whose scratch would exceed the fixed array is refused with a clear error.

    With 16000 variables one sample's iterates no longer fit in shared memory,
    so the tile state moves to scratch and a batch of 1024 needs far more than
    the fixed array.  The size check comes before any array is touched, so the
    call passes no buffers.
    """
    import scipy.sparse as sp

    from purin_b200 import ParametricQP

    n, batch = 16000, 1024
    problem = ParametricQP(P=sp.identity(n, format="csr"), q0=np.zeros(n))
    layer = prepare_projection(problem, method="chambolle-pock", batch_size=batch, backend=DEV)
    assert layer._plan.workspace_size(_native.OP_FORWARD, batch, layer._cfg) > (16 << 20)
    lib = _native.load()
    fn = lib.purin_cp_forward_noalloc
    fn.argtypes = [ctypes.c_void_p, ctypes.POINTER(_native.CpConfig),
                   ctypes.POINTER(_native.ForwardArgs), ctypes.c_void_p]
    fn.restype = ctypes.c_int32
    args = _native.ForwardArgs()
    args.batch = batch
    args.total_batch = batch
    args.bounds_stride = n
    status = fn(layer._plan.handle, ctypes.byref(layer._cfg), ctypes.byref(args),
                torch.cuda.current_stream().cuda_stream)
    assert status == 4  # PURIN_ERR_WORKSPACE
    assert b"fixed device array" in lib.purin_cp_last_error()
