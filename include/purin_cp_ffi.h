/*
 * purin_cp_ffi.h -- XLA FFI buffers -> the C ABI's argument structs (header-only C++17).
 *
 * The reference's CP solve is a jax.custom_vjp pair, solve_jit's forward and
 * its bwd (src/purin/solvers/chambolle_pock/bounds.py:68-167, called at
 * bounds.py:237-246).  Under JAX the two run as XLA custom calls registered with
 * jax.ffi (purin_b200/csrc/jax_ffi_adapter.cc); XLA hands each handler its
 * operands and results as typed buffers plus attributes.  This header maps those
 * buffers, given as plain {pointer, element type, dimensions} views, onto
 * PurinCpForwardArgs / PurinCpAdjointArgs with every shape and dtype checked
 * against the plan, so the packing builds and is tested without XLA's headers.
 *
 * Operand order is the reference's:
 *   forward  (values, rhs, target, initial, tolerance, lower, upper, feasible)
 *            -> (y, dual, iterations, residual, gap, converged)      kernels.py:15-23
 *   adjoint  (values, rhs, target, lower, upper, y, dual, converged, cot_y)
 *            -> (grad_values, grad_rhs, grad_target, grad_lower, grad_upper,
 *                linear_status, linear_residual, device_error)       bounds.py:156-165
 * Shapes: values (1 | B, kept_nnz) or (kept_nnz,); rhs, initial, dual (B, m);
 * target, y, cot_y (B, n); lower, upper (B, n), (1, n) or (n,); tolerance,
 * residual, gap, linear_residual (B,) floating; feasible, converged (B,) uint8;
 * iterations, linear_status (B,) int32; device_error (1,) int32.  Floating
 * buffers have the plan's dtype.
 */
#ifndef PURIN_CP_FFI_H
#define PURIN_CP_FFI_H

#include <cstdint>
#include <string>

#include "purin_cp.h"

namespace purin_ffi {

/* Element types of the buffers (a subset of XLA's). */
enum Elem : int32_t { F64 = 0, F32 = 1, U8 = 2, S32 = 3, S64 = 4, OTHER = 5 };

/* One buffer as XLA hands it over. */
struct Array {
  void* data;
  int32_t elem;  /* Elem */
  int32_t rank;
  int64_t dims[4];
};

struct ForwardBuffers {
  Array values, rhs, target, initial, tolerance, lower, upper, feasible;  /* operands */
  Array y, dual, iterations, residual, gap, converged;                    /* results  */
};

struct AdjointBuffers {
  Array values, rhs, target, lower, upper, y, dual, converged, cot_y;     /* operands */
  Array grad_values, grad_rhs, grad_target, grad_lower, grad_upper;       /* results  */
  Array linear_status, linear_residual, device_error;
};

/* ChambollePockConfig (chambolle_pock/config.py:34-48) from FFI attributes. */
inline PurinCpConfig make_config(int64_t max_iterations, bool accelerated, double safety,
                                 int64_t norm_iterations, int64_t norm_seed, bool norm_bound,
                                 bool diagonal_preconditioning, bool prng_partitionable) {
  PurinCpConfig c{};
  c.max_iterations = static_cast<int32_t>(max_iterations);
  c.accelerated = accelerated ? 1 : 0;
  c.safety = safety;
  c.norm_iterations = static_cast<int32_t>(norm_iterations);
  c.norm_seed = norm_seed;
  c.norm_bound = norm_bound ? 1 : 0;
  c.diagonal_preconditioning = diagonal_preconditioning ? 1 : 0;
  c.prng_partitionable = prng_partitionable ? 1 : 0;
  return c;
}

/* LinearSolverConfig + ImplicitGradientConfig.adjoint_tolerance (solvers/config.py:10-44). */
inline PurinLinearSolverConfig make_linear(double tolerance, double atol, int64_t restart,
                                           int64_t max_iterations, double adjoint_tolerance) {
  PurinLinearSolverConfig l{};
  l.tolerance = tolerance;
  l.atol = atol;
  l.restart = static_cast<int32_t>(restart);
  l.max_iterations = static_cast<int32_t>(max_iterations);
  l.adjoint_tolerance = adjoint_tolerance;
  return l;
}

namespace detail {

inline int32_t float_elem(const PurinCpPlanInfo& info) {
  return info.dtype == PURIN_FLOAT64 ? F64 : F32;
}

inline const char* elem_name(int32_t e) {
  switch (e) {
    case F64: return "float64";
    case F32: return "float32";
    case U8: return "uint8";
    case S32: return "int32";
    case S64: return "int64";
    default: return "another type";
  }
}

inline std::string shape_of(const Array& a) {
  std::string s = "(";
  for (int32_t k = 0; k < a.rank && k < 4; ++k) {
    if (k) s += ", ";
    s += std::to_string(a.dims[k]);
  }
  return s + (a.rank == 1 ? ",)" : ")");
}

/* Checks that `a` has element type `elem` and shape `want` (rank entries). */
inline bool expect(const char* name, const Array& a, int32_t elem, int32_t rank, const int64_t* want,
                   std::string* message) {
  int64_t count = 1;
  for (int32_t k = 0; k < rank; ++k) count *= want[k];
  if (a.data == nullptr && count > 0) {  /* an empty buffer may come without storage */
    *message = std::string(name) + " is missing";
    return false;
  }
  if (a.elem != elem) {
    *message = std::string(name) + " must be " + elem_name(elem) + ", got " + elem_name(a.elem);
    return false;
  }
  bool ok = a.rank == rank;
  for (int32_t k = 0; ok && k < rank; ++k) ok = a.dims[k] == want[k];
  if (!ok) {
    Array w{};
    w.rank = rank;
    for (int32_t k = 0; k < rank && k < 4; ++k) w.dims[k] = want[k];
    *message = std::string(name) + " must have shape " + shape_of(w) + ", got " + shape_of(a);
    return false;
  }
  return true;
}

inline bool vec(const char* name, const Array& a, int32_t elem, int64_t b, std::string* m) {
  const int64_t d[1] = {b};
  return expect(name, a, elem, 1, d, m);
}

inline bool mat(const char* name, const Array& a, int32_t elem, int64_t r, int64_t c,
                std::string* m) {
  const int64_t d[2] = {r, c};
  return expect(name, a, elem, 2, d, m);
}

/* Values shared by the batch ((kept_nnz,) or (1, kept_nnz)) or per sample. */
inline bool values_stride(const char* name, const Array& a, int32_t elem, int64_t batch,
                          int64_t nnz, int64_t* stride, std::string* m) {
  if (a.rank == 1) {
    *stride = 0;
    return vec(name, a, elem, nnz, m);
  }
  const int64_t rows = a.rank == 2 && a.dims[0] == 1 ? 1 : batch;
  *stride = rows == 1 && batch != 1 ? 0 : nnz;
  return mat(name, a, elem, rows, nnz, m);
}

/* Bounds shared by the batch ((n,) or (1, n)) or per sample. */
inline bool bounds_stride(const char* name, const Array& a, int32_t elem, int64_t batch, int64_t n,
                          int64_t* stride, std::string* m) {
  if (a.rank == 1) {
    *stride = 0;
    return vec(name, a, elem, n, m);
  }
  const int64_t rows = a.rank == 2 && a.dims[0] == 1 ? 1 : batch;
  *stride = rows == 1 && batch != 1 ? 0 : n;
  return mat(name, a, elem, rows, n, m);
}

}  // namespace detail

/* Fills *args for purin_cp_forward.  Returns PURIN_OK, or
 * PURIN_ERR_INVALID_ARGUMENT with *message naming the offending buffer. */
inline int32_t pack_forward(const PurinCpPlanInfo& info, const ForwardBuffers& b,
                            int64_t sample_offset, int64_t total_batch, PurinCpForwardArgs* args,
                            std::string* message) {
  using namespace detail;
  const int32_t f = float_elem(info);
  if (b.target.rank != 2 || b.target.dims[1] != info.n) {
    *message = "target must have shape (batch, " + std::to_string(info.n) + "), got " +
               shape_of(b.target);
    return PURIN_ERR_INVALID_ARGUMENT;
  }
  const int64_t B = b.target.dims[0], n = info.n, m = info.kept_rows;
  int64_t vstride = 0, bstride = 0;
  const bool ok =
      mat("target", b.target, f, B, n, message) &&
      values_stride("values", b.values, f, B, info.kept_nnz, &vstride, message) &&
      mat("rhs", b.rhs, f, B, m, message) && mat("initial", b.initial, f, B, m, message) &&
      vec("tolerance", b.tolerance, f, B, message) &&
      bounds_stride("lower", b.lower, f, B, n, &bstride, message) &&
      [&] {
        int64_t ustride = 0;
        if (!bounds_stride("upper", b.upper, f, B, n, &ustride, message)) return false;
        if (ustride != bstride) {
          *message = "lower and upper must both be shared by the batch or both per sample";
          return false;
        }
        return true;
      }() &&
      vec("feasible", b.feasible, U8, B, message) && mat("y", b.y, f, B, n, message) &&
      mat("dual", b.dual, f, B, m, message) &&
      vec("iterations", b.iterations, S32, B, message) &&
      vec("residual", b.residual, f, B, message) && vec("gap", b.gap, f, B, message) &&
      vec("converged", b.converged, U8, B, message);
  if (!ok) return PURIN_ERR_INVALID_ARGUMENT;
  PurinCpForwardArgs a{};
  a.batch = B;
  a.values = b.values.data;
  a.values_stride = vstride;
  a.rhs = b.rhs.data;
  a.target = b.target.data;
  a.dual0 = b.initial.data;
  a.tolerance = b.tolerance.data;
  a.lower = b.lower.data;
  a.upper = b.upper.data;
  a.bounds_stride = bstride;
  a.feasible = static_cast<const uint8_t*>(b.feasible.data);
  a.sample_offset = sample_offset;
  a.total_batch = total_batch > 0 ? total_batch : B;
  a.y = b.y.data;
  a.dual = b.dual.data;
  a.iterations = static_cast<int32_t*>(b.iterations.data);
  a.residual = b.residual.data;
  a.gap = b.gap.data;
  a.converged = static_cast<uint8_t*>(b.converged.data);
  *args = a;
  return PURIN_OK;
}

/* Fills *args for purin_cp_adjoint (the GMRES work counters are left NULL). */
inline int32_t pack_adjoint(const PurinCpPlanInfo& info, const AdjointBuffers& b,
                            int64_t sample_offset, int64_t total_batch, PurinCpAdjointArgs* args,
                            std::string* message) {
  using namespace detail;
  const int32_t f = float_elem(info);
  if (b.target.rank != 2 || b.target.dims[1] != info.n) {
    *message = "target must have shape (batch, " + std::to_string(info.n) + "), got " +
               shape_of(b.target);
    return PURIN_ERR_INVALID_ARGUMENT;
  }
  const int64_t B = b.target.dims[0], n = info.n, m = info.kept_rows;
  int64_t vstride = 0, bstride = 0, ustride = 0;
  const bool ok =
      mat("target", b.target, f, B, n, message) &&
      values_stride("values", b.values, f, B, info.kept_nnz, &vstride, message) &&
      mat("rhs", b.rhs, f, B, m, message) &&
      bounds_stride("lower", b.lower, f, B, n, &bstride, message) &&
      bounds_stride("upper", b.upper, f, B, n, &ustride, message) &&
      mat("y", b.y, f, B, n, message) && mat("dual", b.dual, f, B, m, message) &&
      vec("converged", b.converged, U8, B, message) && mat("cot_y", b.cot_y, f, B, n, message) &&
      mat("grad_values", b.grad_values, f, B, info.kept_nnz, message) &&
      mat("grad_rhs", b.grad_rhs, f, B, m, message) &&
      mat("grad_target", b.grad_target, f, B, n, message) &&
      mat("grad_lower", b.grad_lower, f, B, n, message) &&
      mat("grad_upper", b.grad_upper, f, B, n, message) &&
      vec("linear_status", b.linear_status, S32, B, message) &&
      vec("linear_residual", b.linear_residual, f, B, message) &&
      vec("device_error", b.device_error, S32, 1, message);
  if (!ok) return PURIN_ERR_INVALID_ARGUMENT;
  if (ustride != bstride) {
    *message = "lower and upper must both be shared by the batch or both per sample";
    return PURIN_ERR_INVALID_ARGUMENT;
  }
  PurinCpAdjointArgs a{};
  a.batch = B;
  a.values = b.values.data;
  a.values_stride = vstride;
  a.rhs = b.rhs.data;
  a.target = b.target.data;
  a.lower = b.lower.data;
  a.upper = b.upper.data;
  a.bounds_stride = bstride;
  a.y = b.y.data;
  a.dual = b.dual.data;
  a.converged = static_cast<const uint8_t*>(b.converged.data);
  a.cot_y = b.cot_y.data;
  a.sample_offset = sample_offset;
  a.total_batch = total_batch > 0 ? total_batch : B;
  a.grad_values = b.grad_values.data;
  a.grad_rhs = b.grad_rhs.data;
  a.grad_target = b.grad_target.data;
  a.grad_lower = b.grad_lower.data;
  a.grad_upper = b.grad_upper.data;
  a.linear_status = static_cast<int32_t*>(b.linear_status.data);
  a.linear_residual = b.linear_residual.data;
  a.device_error = static_cast<int32_t*>(b.device_error.data);
  *args = a;
  return PURIN_OK;
}

}  // namespace purin_ffi

#endif /* PURIN_CP_FFI_H */
