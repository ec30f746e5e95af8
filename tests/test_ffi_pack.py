"""XLA FFI buffers -> C ABI argument structs (include/purin_cp_ffi.h), on the CPU.

The jax.ffi handlers (purin_b200/csrc/jax_ffi_adapter.cc) hand every operand
and result of the reference's solve (bounds.py:237-246) and its VJP
(bounds.py:80-165) to this packing, which checks shapes and dtypes against the
plan and fills PurinCpForwardArgs / PurinCpAdjointArgs.  JAX is not installed
here, so the packing is compiled alone (g++, no XLA headers) behind a C shim and
driven with fake device pointers.
"""

import ctypes
import subprocess
from pathlib import Path

import pytest

from purin_b200 import _native

ROOT = Path(__file__).resolve().parents[1]
F64, F32, U8, S32 = 0, 1, 2, 3
B, N, M, NNZ = 3, 5, 4, 7


class Array(ctypes.Structure):
    _fields_ = [("data", ctypes.c_void_p), ("elem", ctypes.c_int32), ("rank", ctypes.c_int32),
                ("dims", ctypes.c_int64 * 4)]


FWD = ("values", "rhs", "target", "initial", "tolerance", "lower", "upper", "feasible", "y", "dual",
       "iterations", "residual", "gap", "converged")
ADJ = ("values", "rhs", "target", "lower", "upper", "y", "dual", "converged", "cot_y",
       "grad_values", "grad_rhs", "grad_target", "grad_lower", "grad_upper", "linear_status",
       "linear_residual", "device_error")


class ForwardBuffers(ctypes.Structure):
    _fields_ = [(name, Array) for name in FWD]


class AdjointBuffers(ctypes.Structure):
    _fields_ = [(name, Array) for name in ADJ]


@pytest.fixture(scope="module")
def shim(tmp_path_factory):
    out = tmp_path_factory.mktemp("ffi") / "libpack_shim.so"
    subprocess.run(["g++", "-std=c++17", "-O1", "-shared", "-fPIC", f"-I{ROOT / 'include'}",
                    str(ROOT / "tests" / "ffi" / "pack_shim.cc"), "-o", str(out)], check=True)
    lib = ctypes.CDLL(str(out))
    lib.shim_pack_forward.restype = ctypes.c_int32
    lib.shim_pack_adjoint.restype = ctypes.c_int32
    return lib


def _info(dtype=0):
    info = _native.PlanInfo()
    info.n, info.equality_size, info.inequality_size = N, 2, 4
    info.kept_rows, info.kept_nnz, info.bound_rows = M, NNZ, 2
    info.dtype = dtype
    return info


def _arr(ptr, elem, *dims):
    a = Array()
    a.data, a.elem, a.rank = ptr, elem, len(dims)
    for k, d in enumerate(dims):
        a.dims[k] = d
    return a


def _forward(elem=F64, **over):
    shapes = dict(values=(1, NNZ), rhs=(B, M), target=(B, N), initial=(B, M), tolerance=(B,),
                  lower=(1, N), upper=(1, N), feasible=(B,), y=(B, N), dual=(B, M),
                  iterations=(B,), residual=(B,), gap=(B,), converged=(B,))
    elems = dict.fromkeys(FWD, elem)
    elems.update(feasible=U8, converged=U8, iterations=S32)
    bufs = ForwardBuffers()
    for k, name in enumerate(FWD):
        shape, e = over.get(name, (shapes[name], elems[name]))
        setattr(bufs, name, _arr(0x1000 * (k + 1), e, *shape))
    return bufs


def _pack_forward(shim, bufs, info=None):
    args = _native.ForwardArgs()
    msg = ctypes.create_string_buffer(256)
    status = shim.shim_pack_forward(ctypes.byref(info or _info()), ctypes.byref(bufs),
                                    ctypes.c_int64(16), ctypes.c_int64(64), ctypes.byref(args), msg,
                                    256)
    return status, args, msg.value.decode()


def test_forward_fields_and_strides(shim):
    status, a, msg = _pack_forward(shim, _forward())
    assert status == 0, msg
    assert a.batch == B and a.values_stride == 0 and a.bounds_stride == 0
    assert (a.sample_offset, a.total_batch) == (16, 64)
    for k, name in enumerate(("values", "rhs", "target")):
        assert getattr(a, name) == 0x1000 * (k + 1)
    assert a.dual0 == 0x4000 and a.tolerance == 0x5000 and a.feasible == 0x8000
    assert (a.y, a.dual, a.iterations, a.residual, a.gap, a.converged) == tuple(
        0x1000 * k for k in range(9, 15))


def test_forward_per_sample_values_and_bounds(shim):
    bufs = _forward(values=((B, NNZ), F64), lower=((B, N), F64), upper=((B, N), F64))
    status, a, msg = _pack_forward(shim, bufs)
    assert status == 0, msg
    assert a.values_stride == NNZ and a.bounds_stride == N
    bufs = _forward(values=((NNZ,), F64), lower=((N,), F64), upper=((N,), F64))
    status, a, _ = _pack_forward(shim, bufs)
    assert status == 0 and a.values_stride == 0 and a.bounds_stride == 0


@pytest.mark.parametrize("over,expected", [
    (dict(target=((B, N + 1), F64)), "target must have shape (batch, 5)"),
    (dict(rhs=((B, M + 1), F64)), "rhs must have shape (3, 4), got (3, 5)"),
    (dict(values=((B, NNZ - 1), F64)), "values must have shape (3, 7)"),
    (dict(tolerance=((B,), F32)), "tolerance must be float64, got float32"),
    (dict(feasible=((B,), F64)), "feasible must be uint8"),
    (dict(iterations=((B,), F64)), "iterations must be int32"),
    (dict(lower=((1, N), F64), upper=((B, N), F64)), "both be shared by the batch or both"),
    (dict(converged=((B + 1,), U8)), "converged must have shape (3,)"),
])
def test_forward_rejects_mismatches(shim, over, expected):
    status, _, msg = _pack_forward(shim, _forward(**over))
    assert status == 1 and expected in msg, msg


def test_forward_missing_buffer_and_float32_plan(shim):
    bufs = _forward()
    bufs.y.data = None
    status, _, msg = _pack_forward(shim, bufs)
    assert status == 1 and msg == "y is missing"
    status, _, msg = _pack_forward(shim, _forward(elem=F32), info=_info(dtype=1))
    assert status == 0, msg
    status, _, msg = _pack_forward(shim, _forward(elem=F64), info=_info(dtype=1))
    assert status == 1 and "must be float32" in msg


def _adjoint(**over):
    shapes = dict(values=(1, NNZ), rhs=(B, M), target=(B, N), lower=(1, N), upper=(1, N),
                  y=(B, N), dual=(B, M), converged=(B,), cot_y=(B, N), grad_values=(B, NNZ),
                  grad_rhs=(B, M), grad_target=(B, N), grad_lower=(B, N), grad_upper=(B, N),
                  linear_status=(B,), linear_residual=(B,), device_error=(1,))
    elems = dict.fromkeys(ADJ, F64)
    elems.update(converged=U8, linear_status=S32, device_error=S32)
    bufs = AdjointBuffers()
    for k, name in enumerate(ADJ):
        shape, e = over.get(name, (shapes[name], elems[name]))
        setattr(bufs, name, _arr(0x100 * (k + 1), e, *shape))
    return bufs


def test_adjoint_fields_and_errors(shim):
    args = _native.AdjointArgs()
    msg = ctypes.create_string_buffer(256)
    status = shim.shim_pack_adjoint(ctypes.byref(_info()), ctypes.byref(_adjoint()),
                                    ctypes.c_int64(0), ctypes.c_int64(0), ctypes.byref(args), msg,
                                    256)
    assert status == 0, msg.value
    assert args.batch == B and args.total_batch == B and args.values_stride == 0
    assert args.cot_y == 0x900 and args.grad_values == 0xA00 and args.device_error == 0x1100
    assert not args.arnoldi_steps and not args.krylov_vectors
    status = shim.shim_pack_adjoint(ctypes.byref(_info()), ctypes.byref(
        _adjoint(device_error=((2,), S32))), ctypes.c_int64(0), ctypes.c_int64(0),
        ctypes.byref(args), msg, 256)
    assert status == 1 and b"device_error must have shape (1,)" in msg.value


def test_config_attributes(shim):
    cfg = _native.CpConfig()
    shim.shim_make_config(ctypes.c_int64(2000), 1, ctypes.c_double(0.95), ctypes.c_int64(20),
                          ctypes.c_int64(42), 0, 1, 1, ctypes.byref(cfg))
    assert (cfg.max_iterations, cfg.accelerated, cfg.norm_iterations, cfg.norm_seed,
            cfg.norm_bound, cfg.diagonal_preconditioning, cfg.prng_partitionable) == (
        2000, 1, 20, 42, 0, 1, 1)
    assert cfg.safety == 0.95


def test_jax_module_is_guarded():
    from purin_b200 import jax_ffi

    if jax_ffi.HAVE_JAX:
        pytest.skip("JAX is installed: the guard is not exercised")
    with pytest.raises(ImportError, match="needs JAX"):
        jax_ffi.register()
