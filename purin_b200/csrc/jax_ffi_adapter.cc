// XLA FFI handlers for the CP projection: the jax.ffi registration of the C ABI.
//
// Under JAX, PURIN's CP solve is the jax.custom_vjp pair built in
// BoundProjection._make_solve (src/purin/solvers/chambolle_pock/bounds.py:68-167):
// the forward of solve_jit (called at bounds.py:237-246) and its bwd.  These two
// handlers are those functions as XLA custom calls, dispatching into
// libpurin_cp.so:
//
//   PurinCpForwardFfi  (values, rhs, target, initial, tolerance, lower, upper,
//                       feasible) -> CPOutput fields            purin_cp_forward
//   PurinCpAdjointFfi  (values, rhs, target, lower, upper, y, dual, converged,
//                       cot_y) -> cotangents + GMRES codes      purin_cp_adjoint
//
// The plan (purin_cp_plan_create, made once per prepared layer) arrives as the
// int64 attribute `plan`; the ChambollePockConfig / LinearSolverConfig fields as
// scalar attributes of the same names.  The workspace comes from XLA's scratch
// allocator, so the handlers allocate nothing themselves, and all work goes on
// XLA's stream.  Buffer packing and validation is purin_cp_ffi.h (tested on the
// CPU without XLA).  This file needs XLA's FFI headers
// (-I $(python -c "import jax.ffi; print(jax.ffi.include_dir())")); it is built
// by purin_b200.jax_ffi.build_adapter only where JAX is installed.
#include <cuda_runtime.h>

#include <cstdint>
#include <optional>
#include <string>

#include "purin_cp.h"
#include "purin_cp_ffi.h"
#include "xla/ffi/api/ffi.h"

namespace ffi = xla::ffi;

namespace {

int32_t elem_of(ffi::DataType t) {
  switch (t) {
    case ffi::DataType::F64: return purin_ffi::F64;
    case ffi::DataType::F32: return purin_ffi::F32;
    case ffi::DataType::U8: return purin_ffi::U8;
    case ffi::DataType::S32: return purin_ffi::S32;
    case ffi::DataType::S64: return purin_ffi::S64;
    default: return purin_ffi::OTHER;
  }
}

purin_ffi::Array view(void* data, ffi::DataType type, ffi::Span<const int64_t> dims) {
  purin_ffi::Array a{};
  a.data = data;
  a.elem = elem_of(type);
  a.rank = static_cast<int32_t>(dims.size());
  for (size_t k = 0; k < dims.size() && k < 4; ++k) a.dims[k] = dims[k];
  if (dims.size() > 4) a.rank = 5;  // rejected by the shape checks
  return a;
}

purin_ffi::Array in(const ffi::AnyBuffer& b) {
  return view(const_cast<void*>(b.untyped_data()), b.element_type(), b.dimensions());
}

purin_ffi::Array out(ffi::Result<ffi::AnyBuffer>& r) {
  return view(r->untyped_data(), r->element_type(), r->dimensions());
}

ffi::Error failure(int32_t status, const std::string& what) {
  const ffi::ErrorCode code = status == PURIN_ERR_INVALID_ARGUMENT ? ffi::ErrorCode::kInvalidArgument
                              : status == PURIN_ERR_WORKSPACE      ? ffi::ErrorCode::kResourceExhausted
                                                                   : ffi::ErrorCode::kInternal;
  return ffi::Error(code, what);
}

ffi::Error CpForward(cudaStream_t stream, ffi::ScratchAllocator scratch, int64_t plan_handle,
                     int64_t max_iterations, bool accelerated, double safety,
                     int64_t norm_iterations, int64_t norm_seed, bool norm_bound,
                     bool diagonal_preconditioning, bool prng_partitionable,
                     int64_t sample_offset, int64_t total_batch, ffi::AnyBuffer values,
                     ffi::AnyBuffer rhs, ffi::AnyBuffer target, ffi::AnyBuffer initial,
                     ffi::AnyBuffer tolerance, ffi::AnyBuffer lower, ffi::AnyBuffer upper,
                     ffi::AnyBuffer feasible, ffi::Result<ffi::AnyBuffer> y,
                     ffi::Result<ffi::AnyBuffer> dual, ffi::Result<ffi::AnyBuffer> iterations,
                     ffi::Result<ffi::AnyBuffer> residual, ffi::Result<ffi::AnyBuffer> gap,
                     ffi::Result<ffi::AnyBuffer> converged) {
  auto* plan = reinterpret_cast<PurinCpPlan*>(plan_handle);
  PurinCpPlanInfo info{};
  if (int32_t s = purin_cp_plan_info(plan, &info)) return failure(s, purin_cp_last_error());
  const PurinCpConfig cfg =
      purin_ffi::make_config(max_iterations, accelerated, safety, norm_iterations, norm_seed,
                             norm_bound, diagonal_preconditioning, prng_partitionable);
  purin_ffi::ForwardBuffers b{in(values),    in(rhs),         in(target),   in(initial),
                              in(tolerance), in(lower),       in(upper),    in(feasible),
                              out(y),        out(dual),       out(iterations), out(residual),
                              out(gap),      out(converged)};
  PurinCpForwardArgs args{};
  std::string message;
  if (int32_t s = purin_ffi::pack_forward(info, b, sample_offset, total_batch, &args, &message))
    return failure(s, "purin_cp_forward: " + message);
  const int32_t op = args.values_stride == 0 ? PURIN_CP_OP_FORWARD : PURIN_CP_OP_FORWARD_SAMPLE_VALUES;
  size_t bytes = 0;
  if (int32_t s = purin_cp_workspace_size(plan, op, args.batch, &cfg, nullptr, &bytes))
    return failure(s, purin_cp_last_error());
  void* workspace = nullptr;
  if (bytes > 0) {
    std::optional<void*> mem = scratch.Allocate(bytes, 256);
    if (!mem.has_value()) return failure(PURIN_ERR_WORKSPACE, "purin_cp_forward: no XLA scratch");
    workspace = *mem;
  }
  if (int32_t s = purin_cp_forward(plan, &cfg, &args, workspace, bytes, stream))
    return failure(s, purin_cp_last_error());
  return ffi::Error::Success();
}

ffi::Error CpAdjoint(cudaStream_t stream, ffi::ScratchAllocator scratch, int64_t plan_handle,
                     int64_t max_iterations, bool accelerated, double safety,
                     int64_t norm_iterations, int64_t norm_seed, bool norm_bound,
                     bool diagonal_preconditioning, bool prng_partitionable,
                     double linear_tolerance, double linear_atol, int64_t linear_restart,
                     int64_t linear_max_iterations, double adjoint_tolerance,
                     int64_t sample_offset, int64_t total_batch, ffi::AnyBuffer values,
                     ffi::AnyBuffer rhs, ffi::AnyBuffer target, ffi::AnyBuffer lower,
                     ffi::AnyBuffer upper, ffi::AnyBuffer y, ffi::AnyBuffer dual,
                     ffi::AnyBuffer converged, ffi::AnyBuffer cot_y,
                     ffi::Result<ffi::AnyBuffer> grad_values, ffi::Result<ffi::AnyBuffer> grad_rhs,
                     ffi::Result<ffi::AnyBuffer> grad_target,
                     ffi::Result<ffi::AnyBuffer> grad_lower,
                     ffi::Result<ffi::AnyBuffer> grad_upper,
                     ffi::Result<ffi::AnyBuffer> linear_status,
                     ffi::Result<ffi::AnyBuffer> linear_residual,
                     ffi::Result<ffi::AnyBuffer> device_error) {
  auto* plan = reinterpret_cast<PurinCpPlan*>(plan_handle);
  PurinCpPlanInfo info{};
  if (int32_t s = purin_cp_plan_info(plan, &info)) return failure(s, purin_cp_last_error());
  const PurinCpConfig cfg =
      purin_ffi::make_config(max_iterations, accelerated, safety, norm_iterations, norm_seed,
                             norm_bound, diagonal_preconditioning, prng_partitionable);
  const PurinLinearSolverConfig lin = purin_ffi::make_linear(
      linear_tolerance, linear_atol, linear_restart, linear_max_iterations, adjoint_tolerance);
  purin_ffi::AdjointBuffers b{in(values),           in(rhs),             in(target),
                              in(lower),            in(upper),           in(y),
                              in(dual),             in(converged),       in(cot_y),
                              out(grad_values),     out(grad_rhs),       out(grad_target),
                              out(grad_lower),      out(grad_upper),     out(linear_status),
                              out(linear_residual), out(device_error)};
  PurinCpAdjointArgs args{};
  std::string message;
  if (int32_t s = purin_ffi::pack_adjoint(info, b, sample_offset, total_batch, &args, &message))
    return failure(s, "purin_cp_adjoint: " + message);
  size_t bytes = 0;
  if (int32_t s = purin_cp_workspace_size(plan, PURIN_CP_OP_ADJOINT, args.batch, &cfg, &lin, &bytes))
    return failure(s, purin_cp_last_error());
  std::optional<void*> mem = scratch.Allocate(bytes, 256);
  if (!mem.has_value()) return failure(PURIN_ERR_WORKSPACE, "purin_cp_adjoint: no XLA scratch");
  if (int32_t s = purin_cp_adjoint(plan, &cfg, &lin, &args, *mem, bytes, stream))
    return failure(s, purin_cp_last_error());
  return ffi::Error::Success();
}

}  // namespace

XLA_FFI_DEFINE_HANDLER_SYMBOL(PurinCpForwardFfi, CpForward,
                              ffi::Ffi::Bind()
                                  .Ctx<ffi::PlatformStream<cudaStream_t>>()
                                  .Ctx<ffi::ScratchAllocator>()
                                  .Attr<int64_t>("plan")
                                  .Attr<int64_t>("max_iterations")
                                  .Attr<bool>("accelerated")
                                  .Attr<double>("safety")
                                  .Attr<int64_t>("norm_iterations")
                                  .Attr<int64_t>("norm_seed")
                                  .Attr<bool>("norm_bound")
                                  .Attr<bool>("diagonal_preconditioning")
                                  .Attr<bool>("prng_partitionable")
                                  .Attr<int64_t>("sample_offset")
                                  .Attr<int64_t>("total_batch")
                                  .Arg<ffi::AnyBuffer>()  // values
                                  .Arg<ffi::AnyBuffer>()  // rhs
                                  .Arg<ffi::AnyBuffer>()  // target
                                  .Arg<ffi::AnyBuffer>()  // initial
                                  .Arg<ffi::AnyBuffer>()  // tolerance
                                  .Arg<ffi::AnyBuffer>()  // lower
                                  .Arg<ffi::AnyBuffer>()  // upper
                                  .Arg<ffi::AnyBuffer>()  // feasible
                                  .Ret<ffi::AnyBuffer>()  // y
                                  .Ret<ffi::AnyBuffer>()  // dual
                                  .Ret<ffi::AnyBuffer>()  // iterations
                                  .Ret<ffi::AnyBuffer>()  // residual
                                  .Ret<ffi::AnyBuffer>()  // gap
                                  .Ret<ffi::AnyBuffer>()  // converged
);

XLA_FFI_DEFINE_HANDLER_SYMBOL(PurinCpAdjointFfi, CpAdjoint,
                              ffi::Ffi::Bind()
                                  .Ctx<ffi::PlatformStream<cudaStream_t>>()
                                  .Ctx<ffi::ScratchAllocator>()
                                  .Attr<int64_t>("plan")
                                  .Attr<int64_t>("max_iterations")
                                  .Attr<bool>("accelerated")
                                  .Attr<double>("safety")
                                  .Attr<int64_t>("norm_iterations")
                                  .Attr<int64_t>("norm_seed")
                                  .Attr<bool>("norm_bound")
                                  .Attr<bool>("diagonal_preconditioning")
                                  .Attr<bool>("prng_partitionable")
                                  .Attr<double>("linear_tolerance")
                                  .Attr<double>("linear_atol")
                                  .Attr<int64_t>("linear_restart")
                                  .Attr<int64_t>("linear_max_iterations")
                                  .Attr<double>("adjoint_tolerance")
                                  .Attr<int64_t>("sample_offset")
                                  .Attr<int64_t>("total_batch")
                                  .Arg<ffi::AnyBuffer>()  // values
                                  .Arg<ffi::AnyBuffer>()  // rhs
                                  .Arg<ffi::AnyBuffer>()  // target
                                  .Arg<ffi::AnyBuffer>()  // lower
                                  .Arg<ffi::AnyBuffer>()  // upper
                                  .Arg<ffi::AnyBuffer>()  // y
                                  .Arg<ffi::AnyBuffer>()  // dual
                                  .Arg<ffi::AnyBuffer>()  // converged
                                  .Arg<ffi::AnyBuffer>()  // cot_y
                                  .Ret<ffi::AnyBuffer>()  // grad_values
                                  .Ret<ffi::AnyBuffer>()  // grad_rhs
                                  .Ret<ffi::AnyBuffer>()  // grad_target
                                  .Ret<ffi::AnyBuffer>()  // grad_lower
                                  .Ret<ffi::AnyBuffer>()  // grad_upper
                                  .Ret<ffi::AnyBuffer>()  // linear_status
                                  .Ret<ffi::AnyBuffer>()  // linear_residual
                                  .Ret<ffi::AnyBuffer>()  // device_error
);
