"""CPU restatement of PURIN's Chambolle--Pock projection path (test infrastructure).

This package is the *checker*, never the product.  Only ``tests/``,
``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl reference`` legs of
``bench.py`` may import it.  The CUDA product path in ``purin_b200`` never calls it.

Every function restates one piece of the reference (SOULS-TAMU/Purin 1.0.2, a
JAX library) in NumPy, citing the reference file:line it follows.  JAX is not
installed in this image, so the reference itself cannot run here; parity is
pinned by

* the analytic golden values and Jacobians held by the reference's own tests
  (``tests/test_regression_chambolle_pock.py``, ``tests/test_projections.py``,
  ``tests/test_regression_cp_bound_presolve.py``, ...), ported as data into
  ``tests/golden/``;
* the published Threefry-2x32 known-answer vectors (Random123) for the PRNG
  that seeds the reference's power iteration;
* finite differences and a PyTorch-autograd restatement of one CP step that
  cross-check the hand-derived pullback.

Arithmetic is performed in the dtype of the inputs (float64 or float32), one
IEEE operation at a time, with sparse sums accumulated sequentially in the
reference's row/slot order so that fixed-iteration results can be compared
bit for bit with the CUDA kernels.
"""

from oracle.prng import prng_key, split, normal, threefry2x32
from oracle.sparse import layout, matvec, tmatvec
from oracle.cp import (
    CPOutput,
    cp_step,
    cp_step_pullback,
    diagnostics,
    diagonal_step_sizes,
    norm_estimate,
    proximal_coefficients,
    sparse_cp,
)
from oracle.gmres import batched_restarted_gmres
from oracle.projection import OracleProjection

__all__ = [
    "prng_key",
    "split",
    "normal",
    "threefry2x32",
    "layout",
    "matvec",
    "tmatvec",
    "CPOutput",
    "cp_step",
    "cp_step_pullback",
    "diagnostics",
    "diagonal_step_sizes",
    "norm_estimate",
    "proximal_coefficients",
    "sparse_cp",
    "batched_restarted_gmres",
    "OracleProjection",
]
