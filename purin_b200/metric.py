"""Constant positive diagonal projection metric (``WeightedDistance``).

Restates ``src/purin/solvers/metric.py:1-182``: with z = sqrt(D) y the weighted
projection 0.5 (y - t)' D (y - t) becomes the Euclidean projection of
sqrt(D) t onto the problem whose column j is scaled by 1/sqrt(D_j).  The base
layer runs with ``tolerance / max(1, sqrt(max D))``; results are mapped back by
1/sqrt(D) and residuals scaled by the same factor.  Autograd differentiates
through both elementwise maps (``metric.py:102-108``).
"""

from __future__ import annotations

from dataclasses import replace

import numpy as np
import torch

from purin_b200.config import validate_metric_diagonal
from purin_b200.problems import CanonicalAffine, canonical_of


def _scaled_problem(problem, inverse) -> CanonicalAffine:
    """Canonical form in z coordinates: coefficient of variable j times inverse[j]."""
    try:
        canonical = canonical_of(problem)
    except TypeError as error:
        raise TypeError(
            "weighted projection requires a symbolic problem or a frontend providing "
            "to_symbolic_problem()") from error
    n = canonical.variable_size
    if len(inverse) != n:
        raise ValueError(f"metric_diagonal must have {n} entries; got {len(inverse)}")
    return canonical.scale_columns(np.asarray(inverse, dtype=np.float64))


class PreparedDiagonalMetricProjection:
    """Same projection methods/results, expressed in original coordinates."""

    def __init__(self, base, diagonal, config):
        self.base = base
        self.config = config
        self.metric_diagonal = tuple(diagonal)
        self._sqrt = torch.sqrt(torch.as_tensor(np.asarray(diagonal), dtype=base._tdtype,
                                                device=base._device))
        self._residual_factor = max(1.0, float(np.sqrt(np.max(diagonal))))

    def __getattr__(self, name):
        return getattr(self.base, name)

    def _target(self, y_hat):
        return torch.as_tensor(y_hat, dtype=self.base._tdtype, device=self.base._device) * self._sqrt

    def __call__(self, y_hat, parameters=None):
        return self.base(self._target(y_hat), parameters) / self._sqrt

    def solve(self, y_hat, parameters=None, initial_state=None):
        initial = None if initial_state is None else torch.as_tensor(initial_state) * self._sqrt
        out = self.base.solve(self._target(y_hat), parameters, initial_state=initial)
        return out._replace(y=out.y / self._sqrt,
                            residual_inf_norm=out.residual_inf_norm * self._residual_factor)

    def project_training(self, y_hat, parameters=None, *, multipliers_eq=None,
                         multipliers_ineq=None):
        out = self.base.project_training(self._target(y_hat), parameters,
                                         multipliers_eq=multipliers_eq,
                                         multipliers_ineq=multipliers_ineq)
        return out._replace(
            y_tilde=out.y_tilde / self._sqrt,
            forward_residual_inf_norm=out.forward_residual_inf_norm * self._residual_factor)

    def with_info(self, y_hat, parameters=None):
        y, info = self.base.with_info(self._target(y_hat), parameters)
        return y / self._sqrt, info._replace(
            forward_residual_inf_norm=info.forward_residual_inf_norm * self._residual_factor)


def prepare_diagonal_metric(problem, config, definition, *, batch_size, dtype, backend):
    """Prepare the base layer on the scaled problem (``metric.py:158-182``)."""
    diagonal = validate_metric_diagonal(config.metric_diagonal)
    factor = max(1.0, float(np.sqrt(max(diagonal))))
    if all(v == 1.0 for v in diagonal):
        return definition(problem, replace(config, metric_diagonal=None)).prepare(
            batch_size=batch_size, dtype=dtype, backend=backend)
    scaled = _scaled_problem(problem, 1 / np.sqrt(np.asarray(diagonal)))
    base_config = replace(config, metric_diagonal=None, tolerance=config.tolerance / factor)
    base_config = replace(base_config, implicit_gradient=replace(
        config.implicit_gradient,
        inexact_tolerance=config.implicit_gradient.inexact_tolerance / factor))
    base = definition(scaled, base_config).prepare(batch_size=batch_size, dtype=dtype,
                                                   backend=backend)
    return PreparedDiagonalMetricProjection(base, diagonal, config)
