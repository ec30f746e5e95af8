/*
 * purin_cp.h -- C ABI of the B200 Chambolle--Pock projection layer.
 *
 * This library replaces the numerical core of PURIN's CP projection path
 * (SOULS-TAMU/Purin 1.0.2).  The reference runs that core as two jitted JAX
 * custom-VJP functions; a host binding (torch, ctypes, or a jax.ffi adapter)
 * calls the entry points below in their place:
 *
 *   purin_cp_plan_create  <- PreparedChambollePockProjection.__post_init__
 *                            (src/purin/solvers/chambolle_pock/solver.py:32-65):
 *                            padded-ELL layout (kernels.py:26-40) and the bound
 *                            presolve row selection (bounds.py:320-326).
 *   purin_cp_forward      <- BoundProjection.solve_jit forward
 *                            (bounds.py:42-66, called at bounds.py:237-246) and
 *                            _solve_jit forward (solver.py:149-176, called at
 *                            solver.py:332): sparse_cp (kernels.py:178-305).
 *   purin_cp_adjoint      <- the custom-VJP backward (bounds.py:80-165;
 *                            solver.py:186-272): power-iteration step sizes,
 *                            restarted GMRES (primal_dual_interior_point/
 *                            operators.py:792-1125) on the CP fixed-point
 *                            adjoint, and the parameter pullback.
 *   purin_cp_adjoint_stage <- the same backward one phase per call, so that
 *                            shards of a batch can share the reference's
 *                            batch-wide GMRES budget (operators.py:919-1103).
 *   purin_cp_postprocess  <- BoundProjection.solve post-processing
 *                            (bounds.py:247-317; solver.py:333-366): multiplier
 *                            recovery in original units, residuals, status.
 *
 * Conventions.  All array arguments are DEVICE pointers on the plan's device,
 * row-major, batch-major ((B, n) means B rows of n).  Floating arrays use the
 * plan's dtype (double or float).  Boolean arrays are uint8 (0/1).  Nothing
 * here allocates, synchronises the host, or calls cudaDeviceSynchronize; all
 * work is enqueued on the caller's stream (a cudaStream_t passed as void*).
 * The caller owns every buffer, including the workspace whose size
 * purin_cp_workspace_size reports.  A plan is immutable after creation and can
 * be used from several host threads on different streams, each call with its
 * own workspace.
 *
 * Errors.  Every function returns a PurinStatus; on failure
 * purin_cp_last_error() returns a thread-local message.  Numerical failures
 * (non-convergence, non-finite iterates) are not errors: they are reported per
 * sample through converged / status arrays, as in the reference.
 */
#ifndef PURIN_CP_H
#define PURIN_CP_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define PURIN_CP_ABI_VERSION 3  /* 2: PurinQpForwardArgs gained flags and the resume fields;
                                   3: the adjoint args gained the GMRES work counters */

typedef enum PurinStatus {
  PURIN_OK = 0,
  PURIN_ERR_INVALID_ARGUMENT = 1,
  PURIN_ERR_UNSUPPORTED = 2,
  PURIN_ERR_CUDA = 3,
  PURIN_ERR_WORKSPACE = 4
} PurinStatus;

typedef enum PurinDtype { PURIN_FLOAT64 = 0, PURIN_FLOAT32 = 1 } PurinDtype;

/* Which computation a workspace is sized for. */
typedef enum PurinCpOp {
  PURIN_CP_OP_FORWARD = 0,
  PURIN_CP_OP_ADJOINT = 1,
  PURIN_QP_OP_FORWARD = 2, /* purin_qp_forward */
  PURIN_QP_OP_ADJOINT = 3, /* purin_qp_adjoint */
  /* The forward solves with values given per sample (values_stride != 0): the
   * workspace also holds each sample's values in the kernels' two sparse orders.
   * The FORWARD ops size the workspace for values shared by the batch. */
  PURIN_CP_OP_FORWARD_SAMPLE_VALUES = 4,
  PURIN_QP_OP_FORWARD_SAMPLE_VALUES = 5
} PurinCpOp;

/* Index arrays derived by the plan (purin_cp_plan_indices). */
typedef enum PurinCpIndex {
  PURIN_CP_KEPT_ROWS = 0,       /* m_kept: original row of each kept row            */
  PURIN_CP_KEPT_SLOTS = 1,      /* nnz_kept: original CSR slot of each kept slot    */
  PURIN_CP_BOUND_ROWS = 2,      /* n_bound: original row of each bound row          */
  PURIN_CP_BOUND_SLOTS = 3,     /* n_bound: CSR slot of each bound row's coefficient */
  PURIN_CP_BOUND_VARIABLES = 4, /* n_bound: variable each bound row constrains      */
  PURIN_CP_KEPT_ROW_PTR = 5,    /* m_kept+1: CSR row pointer of the kept rows        */
  PURIN_CP_KEPT_COLS = 6        /* nnz_kept: column of each kept slot                */
} PurinCpIndex;

/* Phases of purin_cp_adjoint_stage. */
typedef enum PurinCpStage {
  PURIN_CP_STAGE_PREPARE = 0, /* step sizes, linearisation, initial residuals */
  PURIN_CP_STAGE_CYCLE = 1,   /* one restarted-GMRES cycle                    */
  PURIN_CP_STAGE_FINISH = 2   /* validity masking and parameter pullback      */
} PurinCpStage;

typedef struct PurinCpPlan PurinCpPlan;

/* Static sparsity of the public constraint rows: equality rows first, then
 * inequality rows, each row's columns in the order of the problem's sparsity
 * tuples (PreparedChambollePockProjection.__post_init__, solver.py:44-52). */
typedef struct PurinCpStructure {
  int32_t n;               /* variables                                 */
  int32_t equality_size;   /* me                                        */
  int32_t inequality_size; /* mi (all public inequality rows)           */
  const int32_t* row_ptr;  /* HOST pointer, me+mi+1 entries             */
  const int32_t* col;      /* HOST pointer, row_ptr[me+mi] entries      */
  int32_t dtype;           /* PurinDtype                                */
  int32_t device;          /* CUDA device ordinal                       */
} PurinCpStructure;

typedef struct PurinCpPlanInfo {
  int32_t n;
  int32_t equality_size;
  int32_t inequality_size;
  int32_t kept_rows;   /* m = me + kept inequality rows (CP rows)       */
  int32_t kept_nnz;    /* nonzeros of the kept rows                     */
  int32_t bound_rows;  /* singleton inequality rows turned into bounds  */
  int32_t nnz;         /* nonzeros of all public rows                   */
  int32_t width;       /* padded row width of the reference layout      */
  int32_t dtype;
  int32_t device;
} PurinCpPlanInfo;

/* Field-for-field ChambollePockConfig (chambolle_pock/config.py:34-48) for the
 * fields the CP kernels read; tolerance arrives per sample in the call. */
typedef struct PurinCpConfig {
  int32_t max_iterations;
  int32_t accelerated;
  double safety;
  int32_t norm_iterations;
  int64_t norm_seed;
  int32_t norm_bound;
  int32_t diagonal_preconditioning;
  int32_t prng_partitionable; /* 1: jax_threefry_partitionable key scheme (JAX >= 0.5) */
} PurinCpConfig;

/* LinearSolverConfig (solvers/config.py:10-25) + ImplicitGradientConfig
 * .adjoint_tolerance (solvers/config.py:28-44). */
typedef struct PurinLinearSolverConfig {
  double tolerance;
  double atol;
  int32_t restart;
  int32_t max_iterations;
  double adjoint_tolerance;
} PurinLinearSolverConfig;

/* purin_cp_forward: the arguments of BoundProjection.solve_jit
 * (bounds.py:237-246) and the CPOutput fields it returns (kernels.py:15-23),
 * plus `converged &= feasible` (bounds.py:66).  m = kept rows. */
typedef struct PurinCpForwardArgs {
  int64_t batch;
  const void* values;       /* scaled kept-row values, kept CSR slot order   */
  int64_t values_stride;    /* 0 (shared by the batch) or kept_nnz           */
  const void* rhs;          /* (B, m) scaled kept right-hand sides           */
  const void* target;       /* (B, n) projection targets (also y0)           */
  const void* dual0;        /* (B, m) warm-start duals, or NULL for zeros    */
  const void* tolerance;    /* (B,) per-sample solve tolerance               */
  const void* lower;        /* (B, n) or (n,) lower bounds (-inf allowed)    */
  const void* upper;        /* (B, n) or (n,) upper bounds (+inf allowed)    */
  int64_t bounds_stride;    /* 0 (shared) or n                               */
  const uint8_t* feasible;  /* (B,) presolve feasibility, or NULL (all ok)   */
  int64_t sample_offset;    /* index of sample 0 in the global batch (PRNG)  */
  int64_t total_batch;      /* global batch size (PRNG key split count)      */
  void* y;                  /* out (B, n)                                    */
  void* dual;               /* out (B, m)                                    */
  int32_t* iterations;      /* out (B,)                                      */
  void* residual;           /* out (B,)                                      */
  void* gap;                /* out (B,)                                      */
  uint8_t* converged;       /* out (B,)                                      */
} PurinCpForwardArgs;

/* purin_cp_adjoint: the saved residuals of bounds.py:78 and the cotangent of
 * y; returns the cotangents of (values, rhs, target, lower, upper) as
 * bounds.py:156-165 does.  Output pointers may be NULL to skip an output. */
typedef struct PurinCpAdjointArgs {
  int64_t batch;
  const void* values;       /* scaled kept-row values (as in the forward)    */
  int64_t values_stride;
  const void* rhs;          /* (B, m)                                        */
  const void* target;       /* (B, n)                                        */
  const void* lower;        /* (B, n) or (n,)                                */
  const void* upper;
  int64_t bounds_stride;
  const void* y;            /* (B, n) forward solution                       */
  const void* dual;         /* (B, m) forward duals                          */
  const uint8_t* converged; /* (B,) forward convergence (after feasibility)  */
  const void* cot_y;        /* (B, n) cotangent of y                         */
  int64_t sample_offset;
  int64_t total_batch;
  void* grad_values;        /* out (B, kept_nnz) per-sample, or NULL         */
  void* grad_rhs;           /* out (B, m) or NULL                            */
  void* grad_target;        /* out (B, n) or NULL                            */
  void* grad_lower;         /* out (B, n) or NULL                            */
  void* grad_upper;         /* out (B, n) or NULL                            */
  int32_t* linear_status;   /* out (B,) GMRES info 0/1/2, or NULL            */
  void* linear_residual;    /* out (B,) GMRES residual inf-norm, or NULL     */
  int32_t* device_error;    /* out (1,) 0, or nonzero when a bounded device
                               wait gave up (outputs are then unspecified)   */
  /* GMRES work actually done, for measurement (NULL to skip; both or neither):
   * the Arnoldi steps each sample took, and the sum over those steps of the
   * basis vectors each step orthogonalised against (k at a step that finds
   * basis vector k + 1).  CGS2 reads 4 k basis vectors at such a step. */
  int32_t* arnoldi_steps;   /* out (B,) or NULL                              */
  int64_t* krylov_vectors;  /* out (B,) or NULL                              */
} PurinCpAdjointArgs;

/* purin_cp_postprocess: bounds.py:247-305 on the unscaled public rows. */
typedef struct PurinCpPostArgs {
  int64_t batch;
  const void* values_all;   /* unscaled public-row values, CSR slot order    */
  int64_t values_all_stride;/* 0 or nnz                                      */
  const void* rhs_all;      /* (B, me+mi)                                    */
  const void* target;       /* (B, n)                                        */
  const void* lower;        /* (B, n) or (n,) presolve bounds                */
  const void* upper;
  int64_t bounds_stride;
  const void* scale;        /* (B, m) kept-row scaling                       */
  const void* y;            /* (B, n) forward solution                       */
  const void* dual;         /* (B, m) forward (scaled) duals                 */
  const void* gap;          /* (B,) forward gap                              */
  const uint8_t* cp_converged; /* (B,) forward convergence                   */
  double tolerance;         /* ChambollePockConfig.tolerance                 */
  void* multipliers_eq;     /* out (B, me)                                   */
  void* multipliers_ineq;   /* out (B, mi)                                   */
  void* slacks;             /* out (B, mi)                                   */
  int32_t* status;          /* out (B,) SolveStatus                          */
  void* residual_inf_norm;  /* out (B,)                                      */
  uint8_t* finite;          /* out (B,)                                      */
  uint8_t* gradient_eligible; /* out (B,)                                    */
} PurinCpPostArgs;

int32_t purin_cp_abi_version(void);
const char* purin_cp_last_error(void);

int32_t purin_cp_plan_create(const PurinCpStructure* structure, PurinCpPlan** plan);
int32_t purin_cp_plan_destroy(PurinCpPlan* plan);
int32_t purin_cp_plan_info(const PurinCpPlan* plan, PurinCpPlanInfo* info);
/* Copies the requested index array into HOST memory `out` (size per enum). */
int32_t purin_cp_plan_indices(const PurinCpPlan* plan, int32_t which, int32_t* out);

int32_t purin_cp_workspace_size(const PurinCpPlan* plan, int32_t op, int64_t batch,
                                const PurinCpConfig* config,
                                const PurinLinearSolverConfig* linear, size_t* bytes);

/* Diagnostic, no counterpart in the reference: the forward tile a
 * purin_cp_forward call of `batch` samples runs on this plan -- samples per
 * CTA, threads per CTA, and 1 when the tile state lives in shared memory (0:
 * in the workspace).  shared_values: 1 when the call's values are shared by
 * the batch.  Tile shapes differ only in speed, never in results.
 * purin_qp_forward always runs one-sample tiles; this reports the shape of a
 * purin_cp_forward call. */
int32_t purin_cp_forward_shape(const PurinCpPlan* plan, const PurinCpConfig* config, int64_t batch,
                               int32_t shared_values, int32_t* samples_per_tile, int32_t* threads,
                               int32_t* shared_state);

int32_t purin_cp_forward(const PurinCpPlan* plan, const PurinCpConfig* config,
                         const PurinCpForwardArgs* args, void* workspace,
                         size_t workspace_bytes, void* stream);

int32_t purin_cp_adjoint(const PurinCpPlan* plan, const PurinCpConfig* config,
                         const PurinLinearSolverConfig* linear,
                         const PurinCpAdjointArgs* args, void* workspace,
                         size_t workspace_bytes, void* stream);

/* purin_cp_adjoint_stage: purin_cp_adjoint one phase per call, for a batch
 * split into shards (one per GPU, or chunks on one GPU) that must reproduce
 * the unsharded batch exactly.  The reference solves the adjoint systems of
 * the whole batch with one lockstep restarted GMRES
 * (primal_dual_interior_point/operators.py:919-1103): every restart cycle
 * lasts as many Arnoldi steps as the slowest active sample needs, and those
 * steps are charged to ONE iteration budget (LinearSolverConfig.max_iterations)
 * shared by the batch.  A shard that ran its own loop would charge only its
 * own cycles and could give a sample a longer final cycle than the full batch
 * would.  The staged form exposes the two numbers the shards must agree on:
 *
 *   PREPARE  (completed ignored)  counters <- {0, samples above threshold}
 *   CYCLE    (completed = Arnoldi steps taken so far by the whole batch, in
 *             [0, max_iterations))  counters <- {steps of this cycle (max
 *             over the shard's samples), samples still above threshold}
 *   FINISH   (counters may be NULL)  writes the outputs of purin_cp_adjoint.
 *
 * The driver (every shard identically): PREPARE; combine the counters of all
 * shards by elementwise MAX (e.g. an NCCL all-reduce on the counters' device
 * words); completed = 0; while completed < max_iterations and combined[1] > 0:
 * CYCLE(completed), combine, completed += combined[0]; then FINISH.  With the
 * combined counters every shard's results equal the unsharded purin_cp_adjoint's
 * bit for bit; with one shard they equal purin_cp_adjoint's output.
 * `counters` is a device array of two int32; args, workspace and stream must
 * be the same for all phases of one solve (the workspace carries the state).
 * An empty shard (batch 0) still reports zero counters.  The phases are
 * ordinary (non-cooperative) launches on `stream` and do not synchronise; the
 * driver does, when it reads the combined counters on the host. */
int32_t purin_cp_adjoint_stage(const PurinCpPlan* plan, const PurinCpConfig* config,
                               const PurinLinearSolverConfig* linear,
                               const PurinCpAdjointArgs* args, int32_t stage,
                               int32_t completed, int32_t* counters, void* workspace,
                               size_t workspace_bytes, void* stream);

int32_t purin_cp_postprocess(const PurinCpPlan* plan, const PurinCpPostArgs* args,
                             void* stream);

/* ---- General diagonal QP ---------------------------------------------------
 * PreparedDiagonalQP (src/purin/solvers/diagonal_qp.py:72-314) on the same
 * kernels: minimise 0.5 sum(q y^2) + c.y subject to the equality rows, the
 * inequality rows (<= rhs) and lower <= y <= upper, with q, c, the row values,
 * rhs and bounds all per sample and all differentiable.
 *
 *   purin_qp_plan_create <- QPStructure.prepare / PreparedDiagonalQP.__post_init__
 *                           (diagonal_qp.py:64-89): the padded layout of ALL
 *                           rows (no singleton-row presolve); plan_info reports
 *                           kept_rows = me + mi and bound_rows = 0.
 *   purin_qp_forward     <- the custom-VJP solve's forward (diagonal_qp.py:99-131):
 *                           sparse_cp(q, c, values, rhs, ..., y0, dual0,
 *                           freeze_converged, check_stationarity), converged &=
 *                           all(q > 0) & all(lower <= upper).
 *   purin_qp_adjoint     <- its bwd (diagonal_qp.py:133-222): step sizes
 *                           (diagonal, norm bound or power iteration; tau =
 *                           s/(max q + L)), GMRES on (I - J^T) v = (cot_y,
 *                           cot_dual, 0), pullback to (q, c, values, rhs,
 *                           lower, upper).
 * Row scaling and the post-processing of PreparedDiagonalQP.solve
 * (diagonal_qp.py:225-314) are elementwise and stay with the host layer. */
int32_t purin_qp_plan_create(const PurinCpStructure* structure, PurinCpPlan** plan);

typedef struct PurinQpForwardArgs {
  int64_t batch;
  const void* q;            /* (B, n) diagonal objective                     */
  const void* c;            /* (B, n) linear objective                       */
  const void* values;       /* row values, CSR slot order of all rows        */
  int64_t values_stride;    /* 0 (shared by the batch) or nnz                */
  const void* rhs;          /* (B, m) equality then inequality rhs           */
  const void* lower;        /* (B, n) or (n,)                                */
  const void* upper;
  int64_t bounds_stride;    /* 0 or n                                        */
  const void* y0;           /* (B, n) primal warm start, or NULL for zeros   */
  const void* dual0;        /* (B, m) dual warm start, or NULL for zeros     */
  const void* tolerance;    /* (B,) per-sample solve tolerance               */
  int64_t sample_offset;    /* index of sample 0 in the global batch (PRNG)  */
  int64_t total_batch;      /* global batch size (PRNG key split count)      */
  void* y;                  /* out (B, n)                                    */
  void* dual;               /* out (B, m)                                    */
  int32_t* iterations;      /* out (B,)                                      */
  void* residual;           /* out (B,)                                      */
  void* gap;                /* out (B,)                                      */
  uint8_t* converged;       /* out (B,)                                      */
  int32_t flags;            /* 0 for PreparedDiagonalQP; PURIN_QP_* bits for
                               the dense adapter's variant of sparse_cp     */
  /* Resuming a solve (NULL = start afresh).  With y0, dual0, ybar0 and
   * start_iterations taken from an earlier call's y, dual, ybar and
   * iterations, each sample continues exactly as if that call had kept
   * iterating: the accelerated step sizes are advanced start_iterations[b]
   * times, the loop runs from start_iterations[b] to max_iterations, and
   * iterations[b] counts from there.  residual, gap and converged then cover
   * only the iterations run in this call (0, 0 and 0 for a sample with none).
   * The dense adapter's batch-wide trip count uses this (dense.py:79-99). */
  const void* ybar0;                /* in (B, n) or NULL (ybar = y0)         */
  const int32_t* start_iterations;  /* in (B,) or NULL (0); needs y0         */
  void* ybar;                       /* out (B, n) or NULL: final ybar        */
} PurinQpForwardArgs;

/* purin_qp_forward flags: the sparse_cp options the dense adapter
 * (chambolle_pock/dense.py:37-105, dense_implicit.py:14-54) runs with. */
#define PURIN_QP_FACTORED_PROXIMAL 1 /* y+ = a ((y - tau K^T l) - tau c) (kernels.py:142-145) */
#define PURIN_QP_NO_STATIONARITY 2   /* check_stationarity=False                       */
#define PURIN_QP_NO_FREEZE 4         /* freeze_converged=False: accepted samples keep
                                        iterating; the caller runs the batch's trip
                                        count as max_iterations                        */
#define PURIN_QP_NO_VALIDITY 8       /* no all(q > 0) & all(lower <= upper) mask      */

typedef struct PurinQpAdjointArgs {
  int64_t batch;
  const void* q;
  const void* c;
  const void* values;
  int64_t values_stride;
  const void* rhs;
  const void* lower;
  const void* upper;
  int64_t bounds_stride;
  const void* y;            /* (B, n) forward solution                       */
  const void* dual;         /* (B, m) forward duals                          */
  const uint8_t* converged; /* (B,) forward convergence (after validity)     */
  const void* cot_y;        /* (B, n) cotangent of y                         */
  const void* cot_dual;     /* (B, m) cotangent of the duals, or NULL (zero) */
  int64_t sample_offset;
  int64_t total_batch;
  void* grad_q;             /* out (B, n) or NULL                            */
  void* grad_c;             /* out (B, n) or NULL                            */
  void* grad_values;        /* out (B, nnz) or NULL                          */
  void* grad_rhs;           /* out (B, m) or NULL                            */
  void* grad_lower;         /* out (B, n) or NULL                            */
  void* grad_upper;         /* out (B, n) or NULL                            */
  int32_t* linear_status;   /* out (B,) GMRES info 0/1/2, or NULL            */
  void* linear_residual;    /* out (B,) or NULL                              */
  int32_t* device_error;    /* out (1,)                                      */
  int32_t* arnoldi_steps;   /* out (B,) or NULL, as in PurinCpAdjointArgs    */
  int64_t* krylov_vectors;  /* out (B,) or NULL                              */
} PurinQpAdjointArgs;

int32_t purin_qp_forward(const PurinCpPlan* plan, const PurinCpConfig* config,
                         const PurinQpForwardArgs* args, void* workspace,
                         size_t workspace_bytes, void* stream);

int32_t purin_qp_adjoint(const PurinCpPlan* plan, const PurinCpConfig* config,
                         const PurinLinearSolverConfig* linear,
                         const PurinQpAdjointArgs* args, void* workspace,
                         size_t workspace_bytes, void* stream);

/* purin_qp_adjoint_stage: purin_qp_adjoint one phase per call, with the
 * phases, counters and driver of purin_cp_adjoint_stage, so that shards of a
 * QP batch share the reference's batch-wide GMRES budget
 * (diagonal_qp.py:196-204 -> operators.py:919-1103). */
int32_t purin_qp_adjoint_stage(const PurinCpPlan* plan, const PurinCpConfig* config,
                               const PurinLinearSolverConfig* linear,
                               const PurinQpAdjointArgs* args, int32_t stage,
                               int32_t completed, int32_t* counters, void* workspace,
                               size_t workspace_bytes, void* stream);

/* ---- ADMM projection ----------------------------------------------------------
 * PreparedADMMProjection (src/purin/solvers/admm/solver.py:29-255): OSQP-style
 * ADMM for min 0.5 x'diag(q)x + c'x s.t. lower <= K x <= upper on a plan from
 * purin_qp_plan_create (every public row a constraint row, no presolve).
 *
 *   purin_admm_forward  <- sparse_admm (admm/kernels.py:43-283) as called by the
 *                          prepared projection's forward (admm/solver.py:60-97):
 *                          Jacobi PCG x-updates, or banded Cholesky solves when
 *                          the band below is given (admm/factor.py:14-105).
 *   purin_admm_adjoint  <- its bwd (admm/solver.py:175-255): restarted GMRES on
 *                          the active-set KKT operator, then the pullback to the
 *                          values, right-hand sides and target.
 *   purin_admm_adjoint_stage <- the same one phase per call, as
 *                          purin_cp_adjoint_stage, for shards sharing the batch's
 *                          GMRES budget.
 * Row scaling, paired-row compaction (admm/rows.py) and the post-processing of
 * the unbounded projection (chambolle_pock/solver.py:277-366) stay with the host. */

/* ADMMConfig (admm/config.py:10-40): the fields sparse_admm reads. */
typedef struct PurinAdmmConfig {
  double sigma;
  double alpha;
  int32_t max_iterations;
  int32_t cg_max_iterations;
  int32_t cg_refinement_steps;
  int32_t check_interval;
  double cg_tolerance;
  int32_t adaptive_rho;
  int32_t rho_update_interval;
  double rho_update_threshold;
} PurinAdmmConfig;

/* The banded factor's layout (admm/factor.py:108-144), built by the host in the
 * reverse Cuthill--McKee order of the row graph: width < 0 selects the PCG path.
 * Entry k adds penalty[rows[k]] * values[slot_left[k]] * values[slot_right[k]]
 * (CSR slots) to element destination[k] of the (n, width + 1) lower band. */
typedef struct PurinAdmmBand {
  int32_t width;
  int32_t entries;
  const int32_t* permutation;  /* device, n */
  const int32_t* inverse;      /* device, n */
  const int32_t* rows;         /* device, entries */
  const int32_t* slot_left;
  const int32_t* slot_right;
  const int32_t* destination;
} PurinAdmmBand;

typedef struct PurinAdmmForwardArgs {
  int64_t batch;
  const void* q;            /* (B, n) positive diagonal (ones for the projection) */
  const void* c;            /* (B, n) linear term (-target for the projection)   */
  const void* values;       /* CSR slot order of the plan's rows                  */
  int64_t values_stride;    /* 0 (shared by the batch) or nnz                     */
  const void* lower;        /* (B, m) row lower bounds (-inf allowed)             */
  const void* upper;        /* (B, m) row upper bounds                            */
  const void* penalty;      /* (B, m) initial rho per row                         */
  const void* tolerance;    /* (B,)                                               */
  const void* x0;           /* (B, n) warm start                                  */
  const void* dual0;        /* (B, m) or NULL                                     */
  PurinAdmmBand band;
  void* x;                  /* out (B, n)                                         */
  void* z;                  /* out (B, m)                                         */
  void* dual;               /* out (B, m)                                         */
  void* penalty_out;        /* out (B, m) final rho                               */
  int32_t* iterations;      /* out (B,)                                           */
  int32_t* inner_iterations;/* out (B,) PCG iterations                            */
  void* primal_residual;    /* out (B,)                                           */
  void* dual_residual;      /* out (B,)                                           */
  void* linear_residual;    /* out (B,)                                           */
  uint8_t* converged;       /* out (B,)                                           */
  uint8_t* finite;          /* out (B,)                                           */
} PurinAdmmForwardArgs;

int32_t purin_admm_workspace_size(const PurinCpPlan* plan, int64_t batch, int32_t band_width,
                                  size_t* bytes);
int32_t purin_admm_forward(const PurinCpPlan* plan, const PurinAdmmConfig* config,
                           const PurinAdmmForwardArgs* args, void* workspace,
                           size_t workspace_bytes, void* stream);

/* The VJP's inputs: the forward's scaled values and right-hand sides (upper
 * bounds), its solution and duals, convergence and the cotangent of x. */
typedef struct PurinAdmmAdjointArgs {
  int64_t batch;
  const void* values;
  int64_t values_stride;
  const void* rhs;          /* (B, m) scaled right-hand sides                     */
  const void* y;            /* (B, n) forward solution                            */
  const void* dual;         /* (B, m) forward duals                               */
  const uint8_t* converged; /* (B,)                                               */
  const void* cot_y;        /* (B, n)                                             */
  double active_tolerance;  /* ADMMConfig.active_tolerance                        */
  double tolerance;         /* ADMMConfig.tolerance                               */
  int64_t sample_offset;
  int64_t total_batch;
  void* grad_values;        /* out (B, nnz) or NULL                               */
  void* grad_rhs;           /* out (B, m) or NULL                                 */
  void* grad_target;        /* out (B, n) or NULL                                 */
  int32_t* linear_status;   /* out (B,) or NULL                                   */
  void* linear_residual;    /* out (B,) or NULL                                   */
  int32_t* device_error;    /* out (1,)                                           */
} PurinAdmmAdjointArgs;

int32_t purin_admm_adjoint_workspace_size(const PurinCpPlan* plan, int64_t batch,
                                          const PurinLinearSolverConfig* linear, size_t* bytes);
int32_t purin_admm_adjoint(const PurinCpPlan* plan, const PurinLinearSolverConfig* linear,
                           const PurinAdmmAdjointArgs* args, void* workspace,
                           size_t workspace_bytes, void* stream);
int32_t purin_admm_adjoint_stage(const PurinCpPlan* plan, const PurinLinearSolverConfig* linear,
                                 const PurinAdmmAdjointArgs* args, int32_t stage,
                                 int32_t completed, int32_t* counters, void* workspace,
                                 size_t workspace_bytes, void* stream);

/* purin_cp_forward_noalloc: the forward solve of purin_cp_forward for callers
 * that cannot allocate device memory -- a plugin or custom-call hook that is
 * given only its input and output buffers, a framework that has reserved
 * almost all device memory for its own allocator, or a loop where allocation
 * is not allowed.  It has no counterpart in the reference.
 *
 * The scratch that purin_cp_forward takes as `workspace` lives instead in one
 * fixed device array of PURIN_CP_NOALLOC_SCRATCH_BYTES inside the library
 * (one copy on every GPU that loads the library, kept until the process
 * exits).  The call allocates nothing; inputs and outputs are the caller's, as
 * for purin_cp_forward, and results are identical.  Problems whose scratch
 * exceeds the array are rejected with PURIN_ERR_WORKSPACE: the scratch is
 * purin_cp_workspace_size with PURIN_CP_OP_FORWARD for values shared by the
 * batch (values_stride 0, or batch 1), and with
 * PURIN_CP_OP_FORWARD_SAMPLE_VALUES for values given per sample, which also
 * hold every sample's values in the kernels' two sparse orders.  The call sets
 * the plan's device current for its duration and restores the caller's.  The
 * first call on a device looks up the array's device address with that device
 * current; make that first call before any stream capture.  All calls on a
 * device share the one array, so
 * calls whose executions overlap on the GPU (other streams, other host
 * threads) race: serialise them. */
#define PURIN_CP_NOALLOC_SCRATCH_BYTES ((size_t)16 << 20)
int32_t purin_cp_forward_noalloc(const PurinCpPlan* plan, const PurinCpConfig* config,
                                 const PurinCpForwardArgs* args, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* PURIN_CP_H */
