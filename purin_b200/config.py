"""Frozen configuration dataclasses of the CP projection path.

Field names, defaults and validation messages follow
``src/purin/solvers/chambolle_pock/config.py:10-61`` (``ChambollePockConfig``)
and ``src/purin/solvers/config.py:10-44`` (``LinearSolverConfig``,
``ImplicitGradientConfig``) so that existing configurations construct unchanged.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np


def validate_metric_diagonal(value):
    """Positive finite 1-D weights as a tuple, or None (``_utils/validation.py:56-70``)."""
    if value is None:
        return None
    weights = np.asarray(value, dtype=np.float64)
    if (
        weights.ndim != 1
        or weights.size == 0
        or not np.all(np.isfinite(weights))
        or np.any(weights <= 0)
    ):
        raise ValueError("metric_diagonal must be a nonempty vector of positive finite weights")
    return tuple(float(v) for v in weights)


@dataclass(frozen=True)
class LinearSolverConfig:
    """Linear-system solver choices and tolerances for the implicit VJP."""

    tolerance: float = 1e-9
    atol: float = 0.0
    restart: int = 30
    max_iterations: int = 100
    use_preconditioner: bool = True
    mode: str = "auto"

    def __post_init__(self):
        if self.tolerance <= 0.0 or self.atol < 0.0:
            raise ValueError("linear tolerances are invalid")
        if self.restart < 1 or self.max_iterations < 1:
            raise ValueError("linear iteration limits must be positive")


@dataclass(frozen=True)
class ImplicitGradientConfig:
    """Adjoint solve settings for implicit differentiation through a projection."""

    policy: str = "residual_checked"
    inexact_tolerance: float = 1e-6
    adjoint_tolerance: float = 1e-8
    invalid_batch_policy: str = "skip"
    differentiate_problem_parameters: bool = False

    def __post_init__(self):
        if self.policy not in {"strict", "residual_checked", "always"}:
            raise ValueError("invalid gradient policy")
        if self.invalid_batch_policy not in {"skip", "use_valid"}:
            raise ValueError("invalid batch policy")
        if self.inexact_tolerance < 0.0 or self.adjoint_tolerance < 0.0:
            raise ValueError("gradient tolerances must be nonnegative")


@dataclass(frozen=True)
class ChambollePockConfig:
    """Configure affine distance projection with Chambolle--Pock iterations.

    Attributes:
        tolerance: Positive forward convergence tolerance.
        max_iterations: Positive forward iteration limit.
        accelerated: Use the accelerated forward update when True.
        safety: Step-size safety factor strictly between zero and one.
        norm_iterations: Positive power-iteration count for norm estimation.
        norm_seed: Deterministic seed used by the norm estimator.
        row_scaling: Enable constraint-row normalization.
        norm_bound: Use the sparse operator norm-bound policy.
        linear_solver: Linear-system options for derivative solves.
        implicit_gradient: Implicit derivative policy and adjoint configuration.
        diagonal_preconditioning: Use diagonal step metrics for fixed-step CP.
        metric_diagonal: Optional positive variable-distance metric.
        prng_partitionable: Key scheme of the seeded power iteration: True is
            JAX's ``jax_threefry_partitionable`` scheme (its default since JAX
            0.5), False the legacy scheme.  Only the backward pass, and the
            forward pass with ``norm_bound=False``, draw random numbers.
    """

    tolerance: float = 1e-9
    max_iterations: int = 10000
    accelerated: bool = False
    safety: float = 0.95
    norm_iterations: int = 20
    norm_seed: int = 42
    row_scaling: bool = True
    norm_bound: bool = True
    linear_solver: LinearSolverConfig = field(default_factory=LinearSolverConfig)
    implicit_gradient: ImplicitGradientConfig = field(default_factory=ImplicitGradientConfig)
    diagonal_preconditioning: bool = False
    metric_diagonal: tuple[float, ...] | None = None
    prng_partitionable: bool = True

    def __post_init__(self):
        object.__setattr__(self, "metric_diagonal", validate_metric_diagonal(self.metric_diagonal))
        if not math.isfinite(self.tolerance) or self.tolerance <= 0:
            raise ValueError("tolerance must be positive and finite")
        if not isinstance(self.max_iterations, int) or self.max_iterations < 1:
            raise ValueError("max_iterations must be a positive integer")
        if not 0 < self.safety < 1:
            raise ValueError("safety must be between zero and one")
        if not isinstance(self.norm_iterations, int) or self.norm_iterations < 1:
            raise ValueError("norm_iterations must be a positive integer")


@dataclass(frozen=True)
class ADMMConfig:
    """Penalty, relaxation, stopping and factorization options for ADMM projection.

    Field names, defaults and validation messages follow
    ``src/purin/solvers/admm/config.py:10-69``.
    """

    tolerance: float = 1e-9
    max_iterations: int = 10000
    rho: float = 1.0
    sigma: float = 1e-6
    alpha: float = 1.6
    equality_rho_multiplier: float = 1.0
    cg_max_iterations: int = 32
    cg_tolerance: float = 1e-10
    cg_refinement_steps: int = 1
    adaptive_rho: bool = False
    rho_update_interval: int = 50
    rho_update_threshold: float = 5.0
    row_scaling: bool = True
    active_tolerance: float = 1e-8
    linear_solver: LinearSolverConfig = field(default_factory=LinearSolverConfig)
    implicit_gradient: ImplicitGradientConfig = field(default_factory=ImplicitGradientConfig)
    check_interval: int = 25
    metric_diagonal: tuple[float, ...] | None = None

    def __post_init__(self):
        object.__setattr__(self, "metric_diagonal", validate_metric_diagonal(self.metric_diagonal))
        for name in ("tolerance", "rho", "sigma", "equality_rho_multiplier", "cg_tolerance"):
            value = getattr(self, name)
            if not math.isfinite(value) or value <= 0:
                raise ValueError(f"{name} must be positive and finite")
        for name in ("max_iterations", "cg_max_iterations", "cg_refinement_steps",
                     "rho_update_interval", "check_interval"):
            value = getattr(self, name)
            if not isinstance(value, int) or value < 1:
                raise ValueError(f"{name} must be a positive integer")
        if not math.isfinite(self.alpha) or not 0 < self.alpha < 2:
            raise ValueError("alpha must be between zero and two")
        if not math.isfinite(self.rho_update_threshold) or self.rho_update_threshold < 1:
            raise ValueError("rho_update_threshold must be finite and at least one")
        if not math.isfinite(self.active_tolerance) or self.active_tolerance < 0:
            raise ValueError("active_tolerance must be finite and nonnegative")
