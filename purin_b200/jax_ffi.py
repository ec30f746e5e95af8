"""jax.ffi registration of the CP projection's C ABI (used only where JAX is installed).

PURIN runs its CP solve as a ``jax.custom_vjp`` pair: ``solve_jit``'s forward
and ``bwd`` (``src/purin/solvers/chambolle_pock/bounds.py:68-167``, the forward
called at ``bounds.py:237-246``).  This module replaces both with XLA custom
calls into ``libpurin_cp.so``:

* ``build_adapter()`` compiles ``csrc/jax_ffi_adapter.cc`` (XLA FFI handlers
  ``PurinCpForwardFfi`` / ``PurinCpAdjointFfi``) against the headers of the
  installed jaxlib (``jax.ffi.include_dir()``) into ``_lib/libpurin_cp_xla.so``;
* ``register()`` registers them as the ``purin_cp_forward`` / ``purin_cp_adjoint``
  FFI targets for the CUDA platform;
* ``make_solve(plan, config, ...)`` returns the custom-VJP function with the
  reference's signature, ``solve(values, rhs, target, initial, tolerance, lower,
  upper, feasible) -> (y, dual, iterations, residual, gap, converged)``, whose
  backward returns the reference's seven cotangents and ``None`` for the
  feasibility mask (``bounds.py:156-165``).

There is no Pallas, Triton or XLA-lowered fallback: without JAX, or without a
GPU, these functions raise.  Shapes and dtypes are checked by the handlers
(``include/purin_cp_ffi.h``, tested on the CPU by ``tests/test_ffi_pack.py``).
"""

from __future__ import annotations

import ctypes
import shutil
import subprocess
from pathlib import Path

import numpy as np

from purin_b200 import _native

HERE = Path(__file__).resolve().parent
SOURCE = HERE / "csrc" / "jax_ffi_adapter.cc"
ADAPTER = HERE / "_lib" / "libpurin_cp_xla.so"
INCLUDE = HERE.parent / "include"

try:  # JAX is optional: the torch layer is the product path where it is absent.
    import jax
    import jax.numpy as jnp

    HAVE_JAX = True
except ImportError:  # pragma: no cover - exercised where JAX is installed
    jax = None
    jnp = None
    HAVE_JAX = False


def _require_jax():
    if not HAVE_JAX:
        raise ImportError("purin_b200.jax_ffi needs JAX (jax and a CUDA jaxlib); "
                          "use the torch layer (purin_b200.Distance) without it")


def build_adapter(force: bool = False) -> Path:
    """Compile the XLA FFI handlers against the installed jaxlib's headers."""
    _require_jax()
    lib = _native.library_path()
    if not lib.exists():
        raise RuntimeError(f"{lib} is not built; run `python -m purin_b200.csrc.build`")
    if ADAPTER.exists() and not force and ADAPTER.stat().st_mtime >= max(
            SOURCE.stat().st_mtime, lib.stat().st_mtime):
        return ADAPTER
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    cmd = [nvcc, "-std=c++17", "-O2", "-shared", "-Xcompiler", "-fPIC", "-x", "cu",
           f"-I{jax.ffi.include_dir()}", f"-I{INCLUDE}", str(SOURCE), "-o", str(ADAPTER),
           f"-L{lib.parent}", "-lpurin_cp", "-Xlinker", f"-rpath={lib.parent}"]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError("building the jax.ffi adapter failed:\n" + proc.stdout + proc.stderr)
    return ADAPTER


_registered = False


def register() -> None:
    """Register ``purin_cp_forward`` and ``purin_cp_adjoint`` as CUDA FFI targets."""
    global _registered
    _require_jax()
    if _registered:
        return
    _native.load()  # the ABI version check, before XLA can call into the library
    lib = ctypes.cdll.LoadLibrary(str(build_adapter()))
    jax.ffi.register_ffi_target("purin_cp_forward", jax.ffi.pycapsule(lib.PurinCpForwardFfi),
                                platform="CUDA")
    jax.ffi.register_ffi_target("purin_cp_adjoint", jax.ffi.pycapsule(lib.PurinCpAdjointFfi),
                                platform="CUDA")
    _registered = True


def _config_attrs(config) -> dict:
    """ChambollePockConfig fields as FFI attributes (chambolle_pock/config.py:34-48)."""
    return dict(max_iterations=np.int64(config.max_iterations),
                accelerated=bool(config.accelerated), safety=np.float64(config.safety),
                norm_iterations=np.int64(config.norm_iterations),
                norm_seed=np.int64(config.norm_seed), norm_bound=bool(config.norm_bound),
                diagonal_preconditioning=bool(config.diagonal_preconditioning),
                prng_partitionable=bool(getattr(config, "prng_partitionable", True)))


def make_solve(plan: "_native.Plan", config, *, batch: int, n: int, m: int, dtype=np.float64,
               sample_offset: int = 0, total_batch: int | None = None):
    """The custom-VJP solve of ``bounds.py:68-167`` on the registered FFI targets.

    ``plan`` comes from ``purin_cp_plan_create`` (``purin_b200._native.Plan``) and
    must outlive every call; ``config`` is a ``ChambollePockConfig``.
    """
    _require_jax()
    register()
    dt = jnp.dtype(dtype)
    attrs = dict(plan=np.int64(plan.handle), **_config_attrs(config),
                 sample_offset=np.int64(sample_offset),
                 total_batch=np.int64(total_batch or batch))
    lin = config.linear_solver
    adj_attrs = dict(attrs, linear_tolerance=np.float64(lin.tolerance),
                     linear_atol=np.float64(lin.atol), linear_restart=np.int64(lin.restart),
                     linear_max_iterations=np.int64(lin.max_iterations),
                     adjoint_tolerance=np.float64(config.implicit_gradient.adjoint_tolerance))
    kept_nnz = int(plan.info.kept_nnz)
    sds = jax.ShapeDtypeStruct
    forward_out = (sds((batch, n), dt), sds((batch, m), dt), sds((batch,), jnp.int32),
                   sds((batch,), dt), sds((batch,), dt), sds((batch,), jnp.uint8))
    adjoint_out = (sds((batch, kept_nnz), dt), sds((batch, m), dt), sds((batch, n), dt),
                   sds((batch, n), dt), sds((batch, n), dt), sds((batch,), jnp.int32),
                   sds((batch,), dt), sds((1,), jnp.int32))
    forward_call = jax.ffi.ffi_call("purin_cp_forward", forward_out)
    adjoint_call = jax.ffi.ffi_call("purin_cp_adjoint", adjoint_out)

    @jax.custom_vjp
    def solve(values, rhs, target, initial, tolerance, lower, upper, feasible):
        y, dual, iterations, residual, gap, converged = forward_call(
            values, rhs, target, initial, tolerance, lower, upper,
            feasible.astype(jnp.uint8), **attrs)
        return y, dual, iterations, residual, gap, converged.astype(bool)

    def fwd(values, rhs, target, initial, tolerance, lower, upper, feasible):
        out = solve(values, rhs, target, initial, tolerance, lower, upper, feasible)
        return out, (out, values, rhs, target, lower, upper)

    def bwd(saved, cot):
        out, values, rhs, target, lower, upper = saved
        gv, gb, gt, gl, gu, _, _, _ = adjoint_call(
            values, rhs, target, lower, upper, out[0], out[1], out[5].astype(jnp.uint8),
            cot[0], **adj_attrs)
        # Values or bounds shared by the batch get the batch's summed cotangent.
        if values.ndim == 1 or values.shape[0] != batch:
            gv = gv.sum(axis=0).reshape(values.shape)
        if lower.shape != gl.shape:
            gl = gl.sum(axis=0).reshape(lower.shape)
            gu = gu.sum(axis=0).reshape(upper.shape)
        return (gv, gb, gt, jnp.zeros_like(out[1]), jnp.zeros((batch,), dt), gl, gu, None)

    solve.defvjp(fwd, bwd)
    return solve
