"""Minimal problem frontends that compile to the CP layer's canonical affine form.

PURIN's modelling frontend (``src/purin/problems/``) is outside this build's
scope; the CP path only consumes what it compiles to (``CanonicalProblem``,
``problems/canonical.py:9-52``):

* per-row sparsity tuples, equality rows then inequality rows, each tuple the
  sorted indices of the variables the row depends on
  (``problems/problem.py:358-366``);
* the row coefficients on that support as functions of the parameters
  (``equality_jacobian_values`` / ``inequality_jacobian_values``);
* ``rhs = -g(theta, 0)`` per row (``chambolle_pock/solver.py:132-137``).

Two frontends produce that form here:

* ``Projection`` / ``Problem``: a symbolic builder for constraints affine in the
  variables, with coefficients and offsets that are expressions in the
  parameters.  ``a >= b`` is normalised to ``b - a <= 0`` and ``a == b`` /
  ``a <= b`` to ``a - b`` (``problems/expressions.py:298-310``).  Products of
  variables, powers and ``abs`` of variables make a row non-affine, which the
  CP layer rejects at preparation.
* ``ParametricQP`` (alias ``MatrixProblem``): the matrix adapter of
  ``problems/qp.py:83-235`` with ``rhs = b0 + M theta``; sparsity rows follow the
  CSR order of sparse inputs and ``flatnonzero`` order of dense ones
  (``qp.py:58-66``).

Evaluation is array-library generic: the same canonical object evaluates with
NumPy arrays (test oracles) or torch tensors (the CUDA layer, differentiable
with respect to the parameters).
"""

from __future__ import annotations

from dataclasses import asdict, is_dataclass
from typing import Any, Mapping, Sequence

import numpy as np

try:
    import scipy.sparse as _sp
except Exception:  # pragma: no cover
    _sp = None


# ---------------------------------------------------------------------------
# Parameter-only scalar expressions (coefficients and offsets).
class _P:
    """Scalar expression in the parameters; constants fold to Python floats."""

    __slots__ = ("fn", "deps", "const")

    def __init__(self, fn=None, deps=frozenset(), const=None):
        self.fn = fn
        self.deps = frozenset(deps)
        self.const = None if const is None else float(const)

    @staticmethod
    def constant(value):
        return _P(const=value)

    @staticmethod
    def parameter(index):
        return _P(fn=lambda th, k=index: th[:, k], deps={index})

    def ev(self, theta):
        return self.const if self.const is not None else self.fn(theta)

    def _bin(self, other, op):
        other = other if isinstance(other, _P) else _P.constant(other)
        if self.const is not None and other.const is not None:
            return _P.constant(op(self.const, other.const))
        a, b = self, other
        return _P(fn=lambda th: op(a.ev(th), b.ev(th)), deps=a.deps | b.deps)

    def __add__(self, o):
        return self._bin(o, lambda x, y: x + y)

    def __sub__(self, o):
        return self._bin(o, lambda x, y: x - y)

    def __mul__(self, o):
        return self._bin(o, lambda x, y: x * y)

    def __truediv__(self, o):
        return self._bin(o, lambda x, y: x / y)

    def __pow__(self, o):
        return self._bin(o, lambda x, y: x**y)

    def __neg__(self):
        if self.const is not None:
            return _P.constant(-self.const)
        a = self
        return _P(fn=lambda th: -a.ev(th), deps=a.deps)


_ZERO = _P.constant(0.0)


class Expression:
    """Scalar expression: sum_j coef_j(theta) * y_j + offset(theta), or non-affine."""

    __array_priority__ = 1000

    def __init__(self, terms=None, offset=_ZERO, *, affine=True, var_deps=None, text=""):
        self.terms: dict[int, _P] = dict(terms or {})
        self.offset: _P = offset
        self.affine = affine
        self.var_deps = frozenset(self.terms) if var_deps is None else frozenset(var_deps)
        self.text = text

    @property
    def param_deps(self):
        deps = set(self.offset.deps)
        for c in self.terms.values():
            deps |= c.deps
        return frozenset(deps)

    def _nonlinear(self, other, text):
        return Expression(affine=False, var_deps=self.var_deps | other.var_deps, text=text)

    def __add__(self, other):
        other = _as_expression(other)
        if not (self.affine and other.affine):
            return self._nonlinear(other, f"({self.text} + {other.text})")
        terms = dict(self.terms)
        for k, c in other.terms.items():
            terms[k] = terms[k] + c if k in terms else c
        return Expression(terms, self.offset + other.offset, text=f"({self.text} + {other.text})")

    __radd__ = lambda self, other: _as_expression(other) + self

    def __neg__(self):
        if not self.affine:
            return Expression(affine=False, var_deps=self.var_deps, text=f"-{self.text}")
        return Expression({k: -c for k, c in self.terms.items()}, -self.offset, text=f"-{self.text}")

    def __sub__(self, other):
        other = _as_expression(other)
        if not (self.affine and other.affine):
            return self._nonlinear(other, f"({self.text} - {other.text})")
        terms = dict(self.terms)
        for k, c in other.terms.items():
            terms[k] = terms[k] - c if k in terms else _ZERO - c
        return Expression(terms, self.offset - other.offset, text=f"({self.text} - {other.text})")

    def __rsub__(self, other):
        return _as_expression(other) - self

    def _scale(self, factor: _P, text):
        return Expression({k: c * factor for k, c in self.terms.items()}, self.offset * factor,
                          text=text)

    def __mul__(self, other):
        other = _as_expression(other)
        text = f"{self.text} * {other.text}"
        if not (self.affine and other.affine) or (self.terms and other.terms):
            return self._nonlinear(other, text)
        if not self.terms:  # parameter-only left factor
            return Expression({k: self.offset * c for k, c in other.terms.items()},
                              self.offset * other.offset, text=text)
        return self._scale(other.offset, text)

    def __rmul__(self, other):
        return _as_expression(other) * self

    def __truediv__(self, other):
        other = _as_expression(other)
        text = f"{self.text} / {other.text}"
        if other.terms or not other.affine or not self.affine:
            return self._nonlinear(other, text)
        return Expression({k: c / other.offset for k, c in self.terms.items()},
                          self.offset / other.offset, text=text)

    def __pow__(self, exponent):
        text = f"{self.text}**{exponent}"
        if self.terms or not self.affine:
            if self.affine and isinstance(exponent, (int, float)) and exponent == 1:
                return self
            return Expression(affine=False, var_deps=self.var_deps, text=text)
        e = _as_expression(exponent)
        return Expression({}, self.offset ** e.offset, text=text)

    def __abs__(self):
        if self.terms or not self.affine:
            return Expression(affine=False, var_deps=self.var_deps, text=f"abs({self.text})")
        off = self.offset
        fn = (lambda th: abs(off.ev(th))) if off.const is None else None
        return Expression({}, _P(fn=fn, deps=off.deps) if fn else _P.constant(abs(off.const)),
                          text=f"abs({self.text})")

    def __le__(self, other):
        right = _as_expression(other)
        return Constraint(self - right, "ineq", f"{self.text} <= {right.text}")

    def __ge__(self, other):
        right = _as_expression(other)
        return Constraint(right - self, "ineq", f"{self.text} >= {right.text}")

    def __eq__(self, other):  # type: ignore[override]
        right = _as_expression(other)
        return Constraint(self - right, "eq", f"{self.text} == {right.text}")

    __hash__ = object.__hash__

    def __bool__(self):
        raise TypeError("Symbolic expressions do not have a truth value. Use ==, <=, or >= "
                        "inside problem.constraints.add(...).")

    def __repr__(self):
        return f"Expression({self.text})"


def _as_expression(value) -> Expression:
    if isinstance(value, Expression):
        return value
    if isinstance(value, (int, float, np.floating, np.integer)):
        return Expression({}, _P.constant(float(value)), text=repr(float(value)))
    raise TypeError(f"unsupported operand {value!r}")


class Constraint:
    """A residual expression with kind ``"eq"`` (== 0) or ``"ineq"`` (<= 0)."""

    def __init__(self, residual: Expression, kind: str, text: str = ""):
        if kind not in {"eq", "ineq"}:
            raise ValueError(f"Constraint kind must be 'eq' or 'ineq'; got {kind!r}.")
        self.residual = residual
        self.kind = kind
        self.text = text

    def __repr__(self):
        return f"Constraint({self.text})"


class ConstraintList:
    def __init__(self):
        self._items: list[Constraint] = []

    def add(self, *items):
        for item in items:
            if isinstance(item, (list, tuple)):
                self.add(*item)
            elif isinstance(item, Constraint):
                self._items.append(item)
            else:
                raise TypeError("constraints.add expects constraints built with ==, <= or >=")
        return self

    def __iter__(self):
        return iter(self._items)

    def __len__(self):
        return len(self._items)


class _Namespace:
    def __init__(self, problem, kind, names):
        self._problem = problem
        self._kind = kind
        self._names = list(names)

    def __getattr__(self, name):
        if name.startswith("_"):
            raise AttributeError(name)
        return self._problem._symbol(self._kind, name)

    def __getitem__(self, name):
        return self._problem._symbol(self._kind, name)


class Problem:
    """Symbolic constraint system (variables, parameters, affine constraints)."""

    def __init__(self, name: str = "problem"):
        self.name = name
        self.variable_names: list[str] = []
        self.parameter_names: list[str] = []
        self.constraints = ConstraintList()
        self.objective: Any = 0.0

    def _add(self, kind, names):
        names = [names] if isinstance(names, str) else list(names)
        target = self.variable_names if kind == "variable" else self.parameter_names
        for name in names:
            if name in self.variable_names or name in self.parameter_names:
                raise ValueError(f"symbol {name!r} is already defined")
            target.append(name)
        return _Namespace(self, kind, names)

    def add_variable(self, names):
        return self._add("variable", names)

    def add_parameter(self, names):
        return self._add("parameter", names)

    def _symbol(self, kind, name):
        if kind == "variable":
            if name not in self.variable_names:
                raise AttributeError(f"unknown variable {name!r}")
            return Expression({self.variable_names.index(name): _P.constant(1.0)}, text=name)
        if name not in self.parameter_names:
            raise AttributeError(f"unknown parameter {name!r}")
        return Expression({}, _P.parameter(self.parameter_names.index(name)), text=name)

    def canonicalize(self) -> "CanonicalAffine":
        eqs = [c for c in self.constraints if c.kind == "eq"]
        iqs = [c for c in self.constraints if c.kind == "ineq"]
        rows, coefs, offsets, affine = [], [], [], []
        for c in eqs + iqs:
            res = c.residual
            support = tuple(sorted(res.var_deps))
            rows.append(support)
            affine.append(res.affine)
            if res.affine:
                coefs.append([res.terms[j] for j in support])
                offsets.append(res.offset)
            else:
                coefs.append([_ZERO for _ in support])
                offsets.append(_ZERO)
        me = len(eqs)
        metadata = {
            "kind": "symbolic",
            "variable_names": tuple(self.variable_names),
            "parameter_names": tuple(self.parameter_names),
            "equalities_affine_in_variables": all(affine[:me]),
            "inequalities_affine_in_variables": all(affine[me:]),
        }
        return _SymbolicCanonical(self.name, len(self.parameter_names), len(self.variable_names),
                                  me, len(iqs), rows, coefs, offsets, metadata)

    compile = canonicalize


class Projection(Problem):
    """Symbolic constraint system plus one selected projection backend."""

    def __init__(self, name: str = "projection", *, method: str = "fischer-burmeister-newton",
                 config: Mapping[str, Any] | Any | None = None):
        super().__init__(name=name)
        self.method = str(method)
        if config is None:
            self.config: dict[str, Any] = {}
        elif is_dataclass(config):
            self.config = asdict(config)
        elif isinstance(config, Mapping):
            self.config = dict(config)
        else:
            raise TypeError("projection config must be a mapping or dataclass.")

    def solver(self, method: str, **config) -> "Projection":
        self.method = str(method)
        self.config = dict(config)
        return self


SymbolicProblem = Problem


# ---------------------------------------------------------------------------
# Canonical affine form.
def _xp(theta):
    try:
        import torch

        if isinstance(theta, torch.Tensor):
            return torch
    except Exception:  # pragma: no cover
        pass
    return np


class CanonicalAffine:
    """Backend-neutral affine constraint data consumed by the CP layer."""

    name: str
    parameter_size: int
    variable_size: int
    equality_size: int
    inequality_size: int
    equality_sparsity: tuple
    inequality_sparsity: tuple
    metadata: dict
    values_constant: bool

    def csr(self):
        rows = tuple(self.equality_sparsity) + tuple(self.inequality_sparsity)
        row_ptr = np.zeros(len(rows) + 1, dtype=np.int32)
        row_ptr[1:] = np.cumsum([len(r) for r in rows])
        col = np.asarray([j for r in rows for j in r], dtype=np.int32)
        return row_ptr, col

    def evaluate(self, theta):
        """(values (1|B, nnz), rhs (B, me+mi)) in the dtype/device of ``theta``."""
        raise NotImplementedError

    def scale_columns(self, inverse):
        """Canonical form of the problem in z = sqrt(w) y coordinates (metric.py:15-84)."""
        raise NotImplementedError


class _SymbolicCanonical(CanonicalAffine):
    def __init__(self, name, p, n, me, mi, rows, coefs, offsets, metadata):
        self.name = name
        self.parameter_size = p
        self.variable_size = n
        self.equality_size = me
        self.inequality_size = mi
        self.equality_sparsity = tuple(rows[:me])
        self.inequality_sparsity = tuple(rows[me:])
        self._coefs = [c for row in coefs for c in row]
        self._offsets = list(offsets)
        self.metadata = metadata
        self.values_constant = all(c.const is not None for c in self._coefs)
        self.rhs_parameter_rows = np.asarray([o.const is None for o in self._offsets], bool)
        self.coef_parameter_slots = np.asarray([c.const is None for c in self._coefs], bool)

    def evaluate(self, theta):
        xp = _xp(theta)
        batch = theta.shape[0]
        if xp is np:
            dtype = theta.dtype
            full = lambda v: np.full(batch, v, dtype=dtype)
            stack = lambda vs, rows: (np.stack(vs, axis=1) if vs else np.zeros((rows, 0), dtype))
        else:
            full = lambda v: xp.full((batch,), v, dtype=theta.dtype, device=theta.device)
            stack = lambda vs, rows: (xp.stack(vs, dim=1) if vs else
                                      xp.zeros((rows, 0), dtype=theta.dtype, device=theta.device))
        if self.values_constant:
            consts = [c.const for c in self._coefs]
            if xp is np:
                values = np.asarray(consts, dtype=theta.dtype).reshape(1, -1)
            else:
                values = xp.tensor(consts, dtype=theta.dtype, device=theta.device).reshape(1, -1)
        else:
            cols = []
            for c in self._coefs:
                v = c.ev(theta)
                cols.append(full(v) if c.const is not None else v)
            values = stack(cols, batch)
        rhs_cols = []
        for o in self._offsets:
            v = o.ev(theta)
            rhs_cols.append(-(full(v) if o.const is not None else v))
        rhs = stack(rhs_cols, batch)
        return values, rhs

    def scale_columns(self, inverse):
        inverse = [float(v) for v in inverse]
        rows = list(self.equality_sparsity) + list(self.inequality_sparsity)
        coefs, k = [], 0
        for row in rows:
            scaled = []
            for j in row:
                c = self._coefs[k]
                scaled.append(_P.constant(c.const * inverse[j]) if c.const is not None
                              else c * inverse[j])
                k += 1
            coefs.append(scaled)
        out = _SymbolicCanonical(self.name + "_diagonal_metric", self.parameter_size,
                                 self.variable_size, self.equality_size, self.inequality_size,
                                 rows, coefs, self._offsets, dict(self.metadata))
        return out


def _is_sparse(value) -> bool:
    return _sp is not None and _sp.issparse(value)


def _shape(value):
    return tuple(value.shape)


def _row_entries(matrix, row):
    if _is_sparse(matrix):
        start, end = matrix.indptr[row], matrix.indptr[row + 1]
        return matrix.indices[start:end].tolist(), matrix.data[start:end].tolist()
    values = np.asarray(matrix[row])
    idx = np.flatnonzero(values)
    return idx.tolist(), values[idx].tolist()


class _MatrixCanonical(CanonicalAffine):
    """Canonical form of a ParametricQP: constant values, rhs = b0 + M theta."""

    def __init__(self, name, p, n, blocks, metadata):
        self.name = name
        self.parameter_size = p
        self.variable_size = n
        (A_eq, b_eq0, M_eq), (A_in, b_in0, M_in) = blocks
        self.equality_size = _shape(A_eq)[0]
        self.inequality_size = _shape(A_in)[0]
        rows, data = [], []
        for A in (A_eq, A_in):
            for r in range(_shape(A)[0]):
                idx, val = _row_entries(A, r)
                rows.append(tuple(int(i) for i in idx))
                data.extend(float(v) for v in val)
        me = self.equality_size
        self.equality_sparsity = tuple(rows[:me])
        self.inequality_sparsity = tuple(rows[me:])
        self._data = np.asarray(data, dtype=np.float64)
        self._b0 = np.concatenate([np.asarray(b_eq0, np.float64), np.asarray(b_in0, np.float64)])
        # Parameter map rows as a padded gather (sequential per-row sums).
        map_rows = []
        for M in (M_eq, M_in):
            for r in range(_shape(M)[0]):
                map_rows.append(_row_entries(M, r))
        width = max([len(i) for i, _ in map_rows], default=0)
        m_all = len(map_rows)
        self._map_idx = np.zeros((m_all, max(width, 1)), dtype=np.int64)
        self._map_val = np.zeros((m_all, max(width, 1)), dtype=np.float64)
        self._map_mask = np.zeros((m_all, max(width, 1)), dtype=bool)
        for r, (idx, val) in enumerate(map_rows):
            self._map_idx[r, : len(idx)] = idx
            self._map_val[r, : len(idx)] = val
            self._map_mask[r, : len(idx)] = True
        self._map_width = width
        self.rhs_parameter_rows = self._map_mask.any(axis=1)
        self.coef_parameter_slots = np.zeros(len(self._data), bool)
        self.metadata = metadata
        self.values_constant = True
        self._cache = {}

    def _const(self, name, array, like):
        xp = _xp(like)
        if xp is np:
            return array.astype(like.dtype) if array.dtype.kind == "f" else array
        key = (name, like.dtype, like.device)
        t = self._cache.get(key)
        if t is None:
            t = xp.as_tensor(array, device=like.device)
            if t.is_floating_point():
                t = t.to(like.dtype)
            self._cache[key] = t
        return t

    def evaluate(self, theta):
        xp = _xp(theta)
        values = self._const("data", self._data, theta).reshape(1, -1)
        rhs = self._const("b0", self._b0, theta).reshape(1, -1)
        batch = theta.shape[0]
        if self._map_width and self.parameter_size:
            idx = self._const("idx", self._map_idx, theta)
            val = self._const("val", self._map_val, theta)
            mask = self._const("mask", self._map_mask, theta)
            acc = None
            for k in range(self._map_width):
                # Masked slots repeat index 0 with a zero term, so a gather whose
                # gradient adds into each parameter in any order is exact.
                gathered = (theta[:, idx[:, k]] if xp is np
                            else xp.index_select(theta, 1, idx[:, k].contiguous()))
                term = gathered * val[None, :, k]
                term = xp.where(mask[None, :, k], term, xp.zeros_like(term))
                acc = term if acc is None else acc + term
            rhs = rhs + acc
        else:
            rhs = rhs + (theta[:, :0].sum(axis=1, keepdims=True) if xp is np
                         else theta[:, :0].sum(dim=1, keepdim=True))
        if rhs.shape[0] != batch:
            rhs = rhs.expand(batch, -1) if xp is not np else np.broadcast_to(rhs, (batch, rhs.shape[1]))
        return values, rhs

    def scale_columns(self, inverse):
        inverse = np.asarray(inverse, dtype=np.float64)
        out = object.__new__(_MatrixCanonical)
        out.__dict__.update(self.__dict__)
        out._cache = {}
        _, col = self.csr()
        out._data = self._data * inverse[col]
        out.name = self.name + "_diagonal_metric"
        return out


class ParametricQP:
    """Matrix-form QP adapter with affine parameters (``problems/qp.py:83-235``).

    The CP projection path uses only the constraint blocks; ``P``/``q0`` describe
    the QP objective that projection replaces with the distance to the target.
    """

    def __init__(self, P, q0, q_parameter_map=None, A_eq=None, b_eq0=None,
                 b_eq_parameter_map=None, A_ineq=None, b_ineq0=None, b_ineq_parameter_map=None,
                 name: str = "parametric_qp"):
        if len(_shape(P)) != 2 or _shape(P)[0] != _shape(P)[1]:
            raise ValueError("P must be square")
        n = _shape(P)[0]
        sizes = [_shape(v)[1] for v in (q_parameter_map, b_eq_parameter_map, b_ineq_parameter_map)
                 if v is not None]
        p = sizes[0] if sizes else 0
        if any(s != p for s in sizes):
            raise ValueError("parameter maps must share one parameter dimension")
        me = 0 if A_eq is None else _shape(A_eq)[0]
        mi = 0 if A_ineq is None else _shape(A_ineq)[0]

        def matrix(value, shape, label):
            if value is None:
                return _sp.csr_matrix(shape, dtype=np.float64) if _sp is not None else np.zeros(shape)
            if _shape(value) != shape:
                raise ValueError(f"{label} must have shape {shape}, got {_shape(value)}")
            return value.astype(np.float64).tocsr() if _is_sparse(value) else np.asarray(value, np.float64)

        def vector(value, size, label):
            if value is None:
                return np.zeros(size)
            arr = np.asarray(value, dtype=np.float64)
            if arr.shape != (size,):
                raise ValueError(f"{label} must have shape {(size,)}, got {arr.shape}")
            return arr

        self.P = matrix(P, (n, n), "P")
        self.q0 = vector(q0, n, "q0")
        self.q_parameter_map = matrix(q_parameter_map, (n, p), "q_parameter_map")
        self.A_eq = matrix(A_eq, (me, n), "A_eq")
        self.b_eq0 = vector(b_eq0, me, "b_eq0")
        self.b_eq_parameter_map = matrix(b_eq_parameter_map, (me, p), "b_eq_parameter_map")
        self.A_ineq = matrix(A_ineq, (mi, n), "A_ineq")
        self.b_ineq0 = vector(b_ineq0, mi, "b_ineq0")
        self.b_ineq_parameter_map = matrix(b_ineq_parameter_map, (mi, p), "b_ineq_parameter_map")
        self.name = name
        self._parameter_size = p

    @property
    def variable_size(self):
        return int(_shape(self.P)[0])

    @property
    def parameter_size(self):
        return int(self._parameter_size)

    @property
    def equality_size(self):
        return int(_shape(self.A_eq)[0])

    @property
    def inequality_size(self):
        return int(_shape(self.A_ineq)[0])

    def compile(self) -> CanonicalAffine:
        metadata = {"name": self.name, "kind": "parametric_qp",
                    "equalities_affine_in_variables": True,
                    "inequalities_affine_in_variables": True}
        return _MatrixCanonical(
            self.name, self.parameter_size, self.variable_size,
            ((self.A_eq, self.b_eq0, self.b_eq_parameter_map),
             (self.A_ineq, self.b_ineq0, self.b_ineq_parameter_map)),
            metadata)

    canonicalize = compile

    @classmethod
    def from_bounds(cls, *, P, q0, q_parameter_map=None, A, lower0, upper0,
                    lower_parameter_map=None, upper_parameter_map=None, name="parametric_qp"):
        """Rows with equal finite bounds become equalities, the rest one-sided inequalities."""
        lower0 = np.asarray(lower0, dtype=np.float64)
        upper0 = np.asarray(upper0, dtype=np.float64)
        if lower0.shape != upper0.shape:
            raise ValueError("lower0 and upper0 shapes must match")
        eq = np.isfinite(lower0) & np.isfinite(upper0) & (lower0 == upper0)
        up = np.isfinite(upper0) & ~eq
        lo = np.isfinite(lower0) & ~eq
        A = A.tocsr() if _is_sparse(A) else np.asarray(A)
        p = next((_shape(c)[1] for c in (q_parameter_map, lower_parameter_map, upper_parameter_map)
                  if c is not None), 0)

        def pick(mat, mask):
            return mat[mask] if _is_sparse(mat) else np.asarray(mat)[mask]

        def pmap(mat, mask, sign=1.0):
            return np.zeros((int(mask.sum()), p)) if mat is None else sign * np.asarray(mat)[mask]

        blocks, rhs, maps = [], [], []
        if up.any():
            blocks.append(pick(A, up)); rhs.append(upper0[up]); maps.append(pmap(upper_parameter_map, up))
        if lo.any():
            blocks.append(-pick(A, lo)); rhs.append(-lower0[lo]); maps.append(pmap(lower_parameter_map, lo, -1.0))
        if _is_sparse(A):
            A_in = _sp.vstack(blocks, format="csr") if blocks else _sp.csr_matrix((0, _shape(A)[1]))
        else:
            A_in = np.vstack(blocks) if blocks else np.zeros((0, _shape(A)[1]))
        return cls(P=P, q0=q0, q_parameter_map=q_parameter_map, A_eq=pick(A, eq),
                   b_eq0=upper0[eq], b_eq_parameter_map=pmap(upper_parameter_map, eq),
                   A_ineq=A_in, b_ineq0=np.concatenate(rhs) if rhs else np.zeros(0),
                   b_ineq_parameter_map=np.vstack(maps) if maps else np.zeros((0, p)), name=name)


ParametricLP = ParametricQP
MatrixProblem = ParametricQP


def canonical_of(problem) -> CanonicalAffine:
    """Canonical affine form of a frontend object (or the object itself)."""
    if isinstance(problem, CanonicalAffine):
        return problem
    if hasattr(problem, "canonicalize"):
        return problem.canonicalize()
    raise TypeError("problem must be a Problem, ParametricQP or CanonicalAffine")


def ell_index(row_ptr: np.ndarray) -> np.ndarray:
    """Padded (rows, width) index of CSR slots; padding points at slot ``nnz``."""
    rows = len(row_ptr) - 1
    lengths = np.diff(row_ptr)
    width = max(1, int(lengths.max(initial=0)))
    index = np.full((rows, width), int(row_ptr[-1]), dtype=np.int64)
    for r in range(rows):
        index[r, : lengths[r]] = np.arange(row_ptr[r], row_ptr[r + 1])
    return index


def rows_of(row_ptr: np.ndarray) -> np.ndarray:
    """Row index of each CSR slot."""
    return np.repeat(np.arange(len(row_ptr) - 1), np.diff(row_ptr)).astype(np.int64)


__all__: Sequence[str] = [
    "Problem", "Projection", "SymbolicProblem", "ParametricQP", "ParametricLP", "MatrixProblem",
    "CanonicalAffine", "Constraint", "Expression", "canonical_of",
]
