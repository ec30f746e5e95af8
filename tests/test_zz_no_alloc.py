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

The cases cover every part of the scratch the fixed array holds: values
shared by the batch (the two sparse orders of one copy), values given per
sample (every sample's copy), and a problem too large for shared memory, whose
tile iterates then live in the array too.  Calls alternate between them, so
each call starts from the array as a different problem left it.
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


def _noalloc(layer, inputs, out, values_stride=0):
    lib = _native.load()
    fn = lib.purin_cp_forward_noalloc
    fn.argtypes = [ctypes.c_void_p, ctypes.POINTER(_native.CpConfig),
                   ctypes.POINTER(_native.ForwardArgs), ctypes.c_void_p]
    fn.restype = ctypes.c_int32
    batch, n = inputs["target"].shape
    p = lambda t: t.data_ptr()
    args = _native.ForwardArgs(
        batch, p(inputs["data"]), values_stride, p(inputs["rhs"]), p(inputs["target"]),
        p(inputs["initial"]),
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


def _large_case():
    """16000 variables (fp64): one sample's iterates exceed shared memory, so the tile state
    lives in the scratch array; two samples keep the whole scratch near 3 MB."""
    from helpers import random_sparse_problem, random_theta
    from purin_b200 import ChambollePockConfig

    rng = np.random.default_rng(7)
    n, me, mi, batch = 16000, 64, 64, 2
    problem, mats = random_sparse_problem(rng, n, me, mi, 4)
    theta = random_theta(rng, mats, batch)
    candidates = 2.0 * rng.normal(size=(batch, n))
    # The oracle only prepares the scaled inputs here (one iteration is enough).
    oracle = OracleLayer(problem, ChambollePockConfig(max_iterations=1))
    _, saved = oracle.solve(candidates, theta)
    cfg = ChambollePockConfig(max_iterations=150)
    layer = prepare_projection(problem, method="chambolle-pock", config=cfg, batch_size=batch,
                               dtype=torch.float64, backend=DEV)
    inputs = dict(
        data=_t(ell_to_csr(saved["values"], list(oracle.proj.mask.sum(axis=1))),
                torch.float64)[:1].contiguous(),
        rhs=_t(saved["rhs"], torch.float64), target=_t(saved["target"], torch.float64),
        lower=_t(saved["lower"], torch.float64), upper=_t(saved["upper"], torch.float64),
        initial=_t(saved["initial"], torch.float64),
        tolerance=_t(saved["tolerance"], torch.float64),
        feasible=_t(saved["feasible"].astype(np.uint8), torch.uint8))
    # y and ybar alone take 2 (n + 1) doubles a sample, beyond the 227 KB of shared memory
    # a CTA can have, so the tiles (8 samples each) keep their state in the scratch.
    need = layer._plan.workspace_size(_native.OP_FORWARD, batch, layer._cfg)
    assert 2 * (n + 1) * 8 > 227 * 1024 and need >= 8 * 2 * (n + 1) * 8
    assert need <= (16 << 20)
    return layer, inputs


def _per_sample_values(layer, inputs):
    """The same problem with a different scaling of the row values for every sample."""
    batch = inputs["target"].shape[0]
    scale = 1.0 + 0.01 * torch.arange(batch, dtype=inputs["data"].dtype, device=DEV)
    data = (inputs["data"].expand(batch, -1) * scale[:, None]).contiguous()
    need = layer._plan.workspace_size(_native.OP_FORWARD_SAMPLE_VALUES, batch, layer._cfg)
    assert need <= (16 << 20)
    return dict(inputs, data=data)


def _workspace_forward(layer, inputs):
    batch, n = inputs["target"].shape
    out = _outputs(batch, n, layer._m, inputs["target"].dtype)
    layer._forward_native(inputs["data"], inputs["rhs"], inputs["target"], inputs["lower"],
                          inputs["upper"], inputs["initial"], inputs["tolerance"],
                          inputs["feasible"], out["y"], out["dual"], out["iterations"],
                          out["residual"], out["gap"], out["converged"])
    return out


def test_noalloc_global_tile_state_and_per_sample_values_twice():
    """The array's other uses: tile iterates of a problem too large for shared memory, and
    every sample's own values.  The calls alternate, twice each, so every call finds the
    array as the other problem left it; each must equal purin_cp_forward bit for bit."""
    large, large_in = _large_case()
    small, small_in, _ = _case(0, 8, np.float64, 3)
    small_in = _per_sample_values(small, small_in)
    want_large = _workspace_forward(large, large_in)
    want_small = _workspace_forward(small, small_in)
    torch.cuda.synchronize()
    for round_ in range(2):
        for name, layer, inputs, want, stride in (
                ("global tile state", large, large_in, want_large, 0),
                ("per-sample values", small, small_in, want_small, small_in["data"].shape[1])):
            batch, n = inputs["target"].shape
            got = _outputs(batch, n, layer._m, inputs["target"].dtype)
            device_before = torch.cuda.current_device()
            _noalloc(layer, inputs, got, values_stride=stride)
            assert torch.cuda.current_device() == device_before
            torch.cuda.synchronize()
            for key in want:
                np.testing.assert_array_equal(got[key].cpu().numpy(), want[key].cpu().numpy(),
                                              err_msg=f"{name}, call {round_ + 1}: {key}")


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs two GPUs")
def test_noalloc_runs_on_the_plans_device_and_restores_the_current_one():
    """With another GPU current, the call still plans and runs on the plan's GPU (0) and
    leaves the caller's current device as it was."""
    layer, inputs, tdt = _case(0, 4, np.float64, 5)
    want = _workspace_forward(layer, inputs)
    torch.cuda.synchronize(0)
    batch, n = inputs["target"].shape
    got = _outputs(batch, n, layer._m, tdt)
    with torch.cuda.device(1):
        stream0 = torch.cuda.current_stream(0)
        lib_status_device = torch.cuda.current_device()
        fn_stream = stream0.cuda_stream
        lib = _native.load()
        fn = lib.purin_cp_forward_noalloc
        fn.argtypes = [ctypes.c_void_p, ctypes.POINTER(_native.CpConfig),
                       ctypes.POINTER(_native.ForwardArgs), ctypes.c_void_p]
        fn.restype = ctypes.c_int32
        p = lambda t: t.data_ptr()
        args = _native.ForwardArgs(
            batch, p(inputs["data"]), 0, p(inputs["rhs"]), p(inputs["target"]),
            p(inputs["initial"]), p(inputs["tolerance"]), p(inputs["lower"]),
            p(inputs["upper"]), n, p(inputs["feasible"]), 0, batch, p(got["y"]), p(got["dual"]),
            p(got["iterations"]), p(got["residual"]), p(got["gap"]), p(got["converged"]))
        status = fn(layer._plan.handle, ctypes.byref(layer._cfg), ctypes.byref(args), fn_stream)
        _native.check(status, "purin_cp_forward_noalloc")
        assert torch.cuda.current_device() == lib_status_device == 1
    torch.cuda.synchronize(0)
    for key in want:
        np.testing.assert_array_equal(got[key].cpu().numpy(), want[key].cpu().numpy(),
                                      err_msg=key)


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
