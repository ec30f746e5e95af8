"""Projection statuses, result tuples and method identifiers.

Mirrors ``src/purin/solvers/types.py:12-97``: the same enum values, the same
NamedTuple field names and order.  Arrays are ``torch.Tensor`` on the layer's
CUDA device instead of ``jax.Array``.
"""

from __future__ import annotations

from enum import Enum, IntEnum
from typing import Any, NamedTuple

Array = Any


class ProjectionMethod(str, Enum):
    """Projection backends known to PURIN (only ``chambolle-pock`` is built here)."""

    LINEAR_EQUALITY = "linear-equality"
    CHAMBOLLE_POCK = "chambolle-pock"
    ADMM = "admm"
    FISCHER_BURMEISTER_NEWTON = "fischer-burmeister-newton"
    FISCHER_BURMEISTER_REDUCED = "fischer-burmeister-reduced"
    PRIMAL_DUAL_INTERIOR_POINT = "primal-dual-interior-point"

    @classmethod
    def normalize(cls, value: "ProjectionMethod | str") -> "ProjectionMethod":
        """Resolve a method name or enum to its canonical projection method."""
        if isinstance(value, cls):
            return value
        try:
            return cls(str(value).strip().lower())
        except ValueError as error:
            supported = ", ".join(item.value for item in cls)
            raise ValueError(
                f"Unknown projection method {value!r}. Supported methods: {supported}."
            ) from error


class SolveStatus(IntEnum):
    """Backend-neutral solver termination status."""

    CONVERGED = 0
    MAX_ITERATIONS = 1
    LINEAR_SOLVE_FAILURE = 2
    NONFINITE = 3
    LINE_SEARCH_FAILURE = 4


class ProjectionResult(NamedTuple):
    """Complete fixed-shape projection result."""

    y: Array
    multipliers_eq: Array
    multipliers_ineq: Array
    slacks: Array
    status: Array
    iterations: Array
    residual_inf_norm: Array
    finite: Array
    gradient_eligible: Array


class ProjectionInfo(NamedTuple):
    """Lightweight diagnostics returned by ``with_info``."""

    forward_status_codes: Array
    forward_iterations: Array
    forward_residual_inf_norm: Array
    forward_state_finite: Array
    gradient_eligible: Array

    @property
    def forward_converged(self):
        """Return the per-instance convergence flags from the forward solve."""
        return self.forward_status_codes == int(SolveStatus.CONVERGED)


class ProjectionTrainingOutput(NamedTuple):
    """Projected primal/latent-dual state used by the training frontend."""

    y_tilde: Array
    multipliers_eq: Array
    multipliers_ineq: Array
    slacks: Array
    forward_status_codes: Array
    forward_iterations: Array
    forward_residual_inf_norm: Array
    forward_state_finite: Array
    forward_gradient_eligible: Array
