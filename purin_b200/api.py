"""Public preparation entry points: ``prepare_projection``, ``Distance``, ``WeightedDistance``.

Mirrors ``src/purin/solvers/api.py:106-141`` (method dispatch and default
configuration), ``src/purin/solvers/registry.py:10-31`` (third-party
registration) and ``src/purin/projections/distance.py:9-61``.  This build
provides the ``chambolle-pock`` and ``admm`` methods; other PURIN methods can be
registered with ``register_projection`` and otherwise raise a clear error.
"""

from __future__ import annotations

from collections.abc import Callable
from dataclasses import dataclass, replace

import torch

from purin_b200.admm import ADMMProjection
from purin_b200.config import ADMMConfig, ChambollePockConfig
from purin_b200.layer import ChambollePockProjection
from purin_b200.types import ProjectionMethod

_REGISTRY: dict[ProjectionMethod, Callable] = {}

_DEFAULT_FACTORIES = {ProjectionMethod.CHAMBOLLE_POCK: ChambollePockProjection,
                      ProjectionMethod.ADMM: ADMMProjection}


def register_projection(method, factory: Callable) -> None:
    """Register a projection implementation under its canonical method name."""
    selected = ProjectionMethod.normalize(method)
    if selected in _REGISTRY:
        raise ValueError(f"Projection method {selected.value!r} is already registered.")
    _REGISTRY[selected] = factory


def projection_factory(method) -> Callable:
    """Resolve the registered constructor for a requested projection method."""
    selected = ProjectionMethod.normalize(method)
    try:
        return _REGISTRY[selected]
    except KeyError as error:
        raise RuntimeError(
            f"Projection method {selected.value!r} has not been registered; this build "
            "provides 'chambolle-pock' and 'admm'.") from error


def registered_methods() -> tuple[str, ...]:
    """Built-in and explicitly registered projection methods."""
    return tuple(m.value for m in ProjectionMethod if m in _DEFAULT_FACTORIES or m in _REGISTRY)


def prepare_projection(problem, *, method, config=None, batch_size: int, dtype=torch.float64,
                       backend: str = "cuda"):
    """Prepare one fixed-shape projection backend (validation and structure once)."""
    selected = ProjectionMethod.normalize(method)
    if config is None and selected is ProjectionMethod.CHAMBOLLE_POCK:
        config = ChambollePockConfig()
    if config is None and selected is ProjectionMethod.ADMM:
        config = ADMMConfig()
    factory = _DEFAULT_FACTORIES.get(selected)
    if factory is None:
        factory = projection_factory(selected)
    definition = factory(problem, config)
    return definition.prepare(batch_size=int(batch_size), dtype=dtype, backend=str(backend))


@dataclass(frozen=True)
class Distance:
    """Euclidean nearest-feasible-point projection definition."""

    problem: object
    method: str = "fischer-burmeister-newton"
    config: object = None

    def prepare(self, *, batch_size, dtype=torch.float64, backend="cuda"):
        return prepare_projection(self.problem, method=self.method, config=self.config,
                                  batch_size=batch_size, dtype=dtype, backend=backend)


@dataclass(frozen=True)
class WeightedDistance:
    """Nearest-feasible-point projection with a positive diagonal metric."""

    problem: object
    diagonal: object
    method: str = "chambolle-pock"
    config: object = None

    def prepare(self, *, batch_size, dtype=torch.float64, backend="cuda"):
        method = ProjectionMethod.normalize(self.method)
        if method not in (ProjectionMethod.CHAMBOLLE_POCK, ProjectionMethod.ADMM):
            if self.method not in ("admm", "primal-dual-interior-point"):
                raise ValueError("weighted projection supports CP, ADMM, or interior-point")
            raise RuntimeError(f"method {self.method!r} is not part of this build")
        cfg = self.config or (ADMMConfig() if method is ProjectionMethod.ADMM
                              else ChambollePockConfig())
        cfg = replace(cfg, metric_diagonal=tuple(float(v) for v in self.diagonal))
        return Distance(self.problem, self.method, cfg).prepare(batch_size=batch_size,
                                                                dtype=dtype, backend=backend)
