"""Host-side logic: problem frontends, canonical form, configs, device and dtype resolution."""

import numpy as np
import pytest
import scipy.sparse as sp
import torch

from purin_b200 import (
    ChambollePockConfig,
    ImplicitGradientConfig,
    LinearSolverConfig,
    ParametricQP,
    Projection,
    ProjectionMethod,
    SolveStatus,
    registered_methods,
)
from purin_b200.layer import resolve_device, resolve_dtype
from purin_b200.metric import _scaled_problem
from purin_b200.problems import canonical_of, ell_index, rows_of


def test_symbolic_canonical_form_follows_reference_sign_convention():
    p = Projection()
    t = p.add_parameter(["a", "b"])
    y = p.add_variable(["u", "v", "w"])
    p.constraints.add(y.w + y.u == t.b, y.u >= 0, t.a * y.v <= t.b, 2 * y.u - y.v <= 0.9)
    c = p.canonicalize()
    assert c.equality_sparsity == ((0, 2),)
    assert c.inequality_sparsity == ((0,), (1,), (0, 1))
    theta = np.array([[2.0, 3.0]])
    values, rhs = c.evaluate(theta)
    np.testing.assert_array_equal(values, [[1.0, 1.0, -1.0, 2.0, 2.0, -1.0]])
    np.testing.assert_array_equal(rhs, [[3.0, 0.0, 3.0, 0.9]])
    assert np.signbit(rhs[0, 1])  # -g(theta, 0) of "0 - u <= 0" is -0.0, as in JAX
    assert not c.values_constant
    row_ptr, col = c.csr()
    np.testing.assert_array_equal(row_ptr, [0, 2, 3, 4, 6])
    np.testing.assert_array_equal(col, [0, 2, 0, 1, 0, 1])


def test_symbolic_evaluation_is_differentiable_in_torch():
    p = Projection()
    t = p.add_parameter(["a"])
    y = p.add_variable(["u", "v"])
    p.constraints.add(t.a * y.u + y.v == 1)
    theta = torch.tensor([[2.0]], dtype=torch.float64, requires_grad=True)
    values, rhs = p.canonicalize().evaluate(theta)
    values.sum().backward()
    assert float(theta.grad) == 1.0


def test_nonlinear_rows_are_flagged():
    p = Projection()
    y = p.add_variable(["u", "v"])
    p.constraints.add(y.u ** 2 + y.v ** 2 <= 1, y.u + y.v == 1)
    meta = p.canonicalize().metadata
    assert meta["equalities_affine_in_variables"] is True
    assert meta["inequalities_affine_in_variables"] is False
    with pytest.raises(TypeError):
        bool(y.u + 1)


def test_parametric_qp_matrix_form():
    A_eq = sp.csr_matrix(np.array([[1.0, 0.0, 2.0]]))
    A_in = np.array([[0.0, -1.0, 0.0], [1.0, 1.0, 0.0]])
    qp = ParametricQP(P=np.eye(3), q0=np.zeros(3), A_eq=A_eq, b_eq0=[1.0],
                      b_eq_parameter_map=np.array([[1.0, 0.0]]), A_ineq=A_in,
                      b_ineq0=[0.0, 2.0], b_ineq_parameter_map=np.array([[0.0, 0.0], [0.0, 1.0]]))
    c = qp.compile()
    assert c.equality_sparsity == ((0, 2),) and c.inequality_sparsity == ((1,), (0, 1))
    values, rhs = c.evaluate(np.array([[0.5, 0.25], [1.0, 2.0]]))
    np.testing.assert_array_equal(values, [[1.0, 2.0, -1.0, 1.0, 1.0]])
    np.testing.assert_array_equal(rhs, [[1.5, 0.0, 2.25], [2.0, 0.0, 4.0]])
    scaled = c.scale_columns(np.array([1.0, 0.5, 0.25]))
    np.testing.assert_array_equal(scaled.evaluate(np.zeros((1, 2)))[0], [[1.0, 0.5, -0.5, 1.0, 0.5]])


def test_parametric_qp_from_bounds():
    A = np.array([[1.0, 0.0], [0.0, 1.0], [1.0, 1.0]])
    qp = ParametricQP.from_bounds(P=np.eye(2), q0=np.zeros(2), A=A, lower0=[0.0, -np.inf, 1.0],
                                  upper0=[2.0, 3.0, 1.0])
    assert qp.equality_size == 1 and qp.inequality_size == 3
    np.testing.assert_array_equal(qp.b_eq0, [1.0])
    np.testing.assert_array_equal(qp.b_ineq0, [2.0, 3.0, -0.0])


def test_weighted_problem_validation():
    p = Projection()
    y = p.add_variable(["u", "v"])
    p.constraints.add(y.u + y.v == 1)
    with pytest.raises(TypeError, match="symbolic"):
        _scaled_problem(object(), np.ones(2))
    with pytest.raises(ValueError, match="entries"):
        _scaled_problem(p, np.ones(1))


@pytest.mark.parametrize("kwargs,match", [
    ({"tolerance": 0.0}, "tolerance"), ({"max_iterations": 0}, "max_iterations"),
    ({"safety": 1.0}, "safety"), ({"norm_iterations": 0}, "norm_iterations"),
    ({"metric_diagonal": (1.0, -1.0)}, "metric_diagonal"),
])
def test_config_validation(kwargs, match):
    with pytest.raises(ValueError, match=match):
        ChambollePockConfig(**kwargs)


@pytest.mark.parametrize("bad", [[], [0.0], [np.inf], [[1.0]]])
def test_metric_diagonal_validation(bad):
    """PURIN tests/test_linear_algebra.py:153-156 (validate_metric_diagonal)."""
    with pytest.raises(ValueError):
        ChambollePockConfig(metric_diagonal=bad)
    assert ChambollePockConfig(metric_diagonal=[1.0, 2.0]).metric_diagonal == (1.0, 2.0)


@pytest.mark.parametrize("factory,kwargs", [
    (LinearSolverConfig, dict(tolerance=0)), (LinearSolverConfig, dict(atol=-1)),
    (LinearSolverConfig, dict(restart=0)), (LinearSolverConfig, dict(max_iterations=0)),
    (ImplicitGradientConfig, dict(policy="bad")),
    (ImplicitGradientConfig, dict(invalid_batch_policy="bad")),
    (ImplicitGradientConfig, dict(inexact_tolerance=-1)),
    (ImplicitGradientConfig, dict(adjoint_tolerance=-1))])
def test_linear_and_gradient_config_validation(factory, kwargs):
    """PURIN tests/test_validation.py:29-37 (the CP path's configuration classes)."""
    with pytest.raises(ValueError):
        factory(**kwargs)
    assert ChambollePockConfig().linear_solver.restart == 30


def test_enums_and_registry():
    assert int(SolveStatus.NONFINITE) == 3
    assert ProjectionMethod.normalize(" Chambolle-Pock ") is ProjectionMethod.CHAMBOLLE_POCK
    with pytest.raises(ValueError, match="Unknown projection method"):
        ProjectionMethod.normalize("simplex")
    assert "chambolle-pock" in registered_methods()


def test_device_and_dtype_resolution_have_no_cpu_fallback():
    with pytest.raises(RuntimeError, match="CUDA"):
        resolve_device("cpu")
    assert resolve_dtype(np.float32) == torch.float32
    assert resolve_dtype(None) == torch.float64
    with pytest.raises(ValueError):
        resolve_dtype(np.int32)


def test_layout_helpers():
    row_ptr = np.array([0, 2, 2, 5])
    np.testing.assert_array_equal(ell_index(row_ptr), [[0, 1, 5], [5, 5, 5], [2, 3, 4]])
    np.testing.assert_array_equal(rows_of(row_ptr), [0, 0, 2, 2, 2])


@pytest.mark.parametrize("rows", [((0,),), ((0,), (8,)), ((0,), (-1,)), ((0,), (1, 1)),
                                  ((0,), (0.5,)), ((0,), (True,))])
def test_packed_support_validation(rows):
    """The dense adapter's packed supports are validated as sparse_layer.py:24-44 does."""
    from purin_b200.dense_layer import inequality_rows
    with pytest.raises(ValueError):
        inequality_rows(rows, 2, 8)


def test_packed_support_accepts_numpy_integers_and_empty_rows():
    from purin_b200.dense_layer import inequality_rows
    assert inequality_rows(((np.int64(0), 3), ()), 2, 8) == ((0, 3), ())
    assert inequality_rows(None, 2, 3) == ((0, 1, 2), (0, 1, 2))
