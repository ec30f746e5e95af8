"""B200-native Chambolle--Pock projection layer with PURIN's API.

A drop-in for the CP path of SOULS-TAMU/Purin 1.0.2
(``Distance``/``WeightedDistance(problem, "chambolle-pock").prepare(batch_size)``),
and its ADMM projection (``method="admm"``):
the same configuration dataclasses, result tuples and prepared-layer methods,
backed by hand-written sm_100a CUDA kernels behind the C ABI in
``include/purin_cp.h``.  Arrays are torch tensors on a CUDA device.
"""

from purin_b200.api import (
    Distance,
    WeightedDistance,
    prepare_projection,
    register_projection,
    registered_methods,
)
from purin_b200.admm import ADMMProjection, PreparedADMMProjection
from purin_b200.config import (
    ADMMConfig,
    ChambollePockConfig,
    ImplicitGradientConfig,
    LinearSolverConfig,
)
from purin_b200.layer import ChambollePockProjection, PreparedChambollePockProjection
from purin_b200.problems import (
    MatrixProblem,
    ParametricLP,
    ParametricQP,
    Problem,
    Projection,
    SymbolicProblem,
)
from purin_b200.types import (
    ProjectionInfo,
    ProjectionMethod,
    ProjectionResult,
    ProjectionTrainingOutput,
    SolveStatus,
)

__version__ = "0.1.0"

__all__ = [
    "ADMMConfig",
    "ADMMProjection",
    "PreparedADMMProjection",
    "ChambollePockConfig",
    "ChambollePockProjection",
    "Distance",
    "ImplicitGradientConfig",
    "LinearSolverConfig",
    "MatrixProblem",
    "ParametricLP",
    "ParametricQP",
    "PreparedChambollePockProjection",
    "Problem",
    "Projection",
    "ProjectionInfo",
    "ProjectionMethod",
    "ProjectionResult",
    "ProjectionTrainingOutput",
    "SolveStatus",
    "SymbolicProblem",
    "WeightedDistance",
    "prepare_projection",
    "register_projection",
    "registered_methods",
]
