// Kernel parameter blocks and launchers shared by the C ABI (capi.cu).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"
#include "plan.cuh"
#include "sell.cuh"

namespace purin {

template <typename T>
struct FwdParams {
  DevStructure st;
  int64_t batch;
  const T* values;
  int64_t values_stride;
  const T* rhs;
  const T* target;
  const T* dual0;
  const T* tol;
  const T* lower;
  const T* upper;
  int64_t bounds_stride;
  const uint8_t* feasible;
  int64_t sample_offset;
  int64_t total_batch;
  T* y_out;
  T* dual_out;
  int32_t* it_out;
  T* res_out;
  T* gap_out;
  uint8_t* conv_out;
  int max_iterations;
  int accelerated;
  T safety;
  int norm_iterations;
  int64_t norm_seed;
  int norm_bound;
  int diag;
  int partitionable;
  T* gstate;  // per-tile state in global memory when it does not fit in shared memory
  SellView sell;  // sliced-ELL rows/columns in the internal orders
  const T* vr;    // shared values in SELL row order (null: per-sample values)
  const T* vc;    // shared values in SELL column order
  // Per-sample values arranged into the SELL row / column orders once per call,
  // (B, nnz_r_ps) and (B, nnz_c_ps); used when the values are not shared.
  const T* vr_ps;
  const T* vc_ps;
  int64_t nnz_r_ps;
  int64_t nnz_c_ps;
  // Diagonal steps shared by the batch (diagonal preconditioning with shared
  // values), computed once per call in the internal orders: sigma per row,
  // tau, a = 1/(1 + tau), d = tau a per column; null when each tile computes
  // its own steps into shared memory.
  const T* dg_sigma;
  const T* dg_tau;
  const T* dg_a;
  const T* dg_d;
  // Per-sample inputs permuted into the internal orders (zero at padding positions).
  const T* tgt_i;    // (B, n_pos)
  const T* rhs_i;    // (B, m_pos)
  const T* dual0_i;  // (B, m_pos) or null
  const T* lo_i;     // (B or 1, n_pos)
  const T* up_i;
  int64_t bstride_i;  // 0 (shared bounds) or n_pos
  // General diagonal QP (null for the distance projection, where q = 1,
  // c = -target and y0 = target): per-sample q, c and y0 in the internal
  // column order, (B, n_pos) each; y0_i null means zeros.
  const T* q_i;
  const T* c_i;
  const T* y0_i;
  // Variants of sparse_cp the dense adapter uses (kQP kernels only; zero for
  // the projection and the diagonal QP): PURIN_QP_FACTORED_PROXIMAL,
  // PURIN_QP_NO_STATIONARITY, PURIN_QP_NO_FREEZE, PURIN_QP_NO_VALIDITY bits.
  int qp_flags;
  // Resuming a solve (kQP kernels, one-sample tiles): the extrapolated iterate
  // in the internal column order (null: ybar = y0), the iterations each sample
  // has already run (null: 0; the accelerated step sizes are advanced that many
  // times and the count starts there), and the final extrapolated iterate in
  // the external order (null: not written).
  const T* ybar0_i;
  const int32_t* start_it;
  T* ybar_out;
};

template <typename T>
struct AdjParams {
  DevStructure st;
  int64_t batch;
  const T* values;
  int64_t values_stride;
  const T* rhs;
  const T* target;
  const T* lower;
  const T* upper;
  int64_t bounds_stride;
  const T* y;
  const T* dual;
  const uint8_t* converged;
  const T* cot_y;
  int64_t sample_offset;
  int64_t total_batch;
  T* g_values;
  T* g_rhs;
  T* g_target;
  T* g_lower;
  T* g_upper;
  int32_t* lin_status;
  T* lin_residual;
  int32_t* device_error;
  int32_t* work_steps;       // (B,) Arnoldi steps taken, or null
  long long* work_vectors;   // (B,) sum over those steps of the basis vectors, or null
  // General diagonal QP (qp = 1; diagonal_qp.py:133-222): per-sample q and c
  // replace q = 1, c = -target; the dual cotangent enters the right-hand
  // side; q and c get cotangents.
  int qp;
  const T* q;         // (B, n)
  const T* c;         // (B, n)
  const T* cot_dual;  // (B, m) or null
  T* g_q;             // (B, n) or null
  T* g_c;             // (B, n) or null
  int norm_bound;     // QP backward only: L from |K| row/column sums
  // ADMM projection (mode 1; admm/solver.py:175-255): GMRES on the active-set KKT
  // operator [v + K^T (a w); a K v + (1 - a) w] of n + m unknowns, with the
  // activity a of each row from the forward's duals and slacks.
  int mode;
  T act_tol;          // ADMMConfig.active_tolerance
  T fwd_tol;          // ADMMConfig.tolerance
  // configuration
  int accelerated;
  int diag;
  int norm_iterations;
  int partitionable;
  int64_t norm_seed;
  T safety;
  T lin_tol;
  T lin_atol;
  T adj_tol;
  int R;       // effective restart = min(restart, max_iterations, W)
  int max_it;  // GMRES iteration budget
  uint64_t timeout_ns;
  // Arrivals the grid barrier waits for beyond gridDim.x: 0, or 1 in the test
  // that makes a bounded wait run out (PURIN_CP_TEST_UNREACHABLE_BARRIER).
  unsigned barrier_extra;
  // 0: the whole VJP in one cooperative launch (grid barriers between phases).
  // 1, 2, 3: one phase per launch (prepare; one GMRES cycle; pullback) for a
  // host that exchanges the cycle counters with other shards between launches.
  int stage;
  int completed0;  // stage 2: Arnoldi steps the lockstep batch has taken so far
  // workspace
  T* x;            // B * W
  T* lamp;         // B * m
  uint8_t* ycode;  // B * n
  uint8_t* dcode;  // B * m
  T* steps;        // B * 2 : tau, sigma
  T* dsteps;       // B * (2n + m) : a, d (per column), sigma (per row); diagonal steps or QP
                   // (QP: B * (3n + m), tau per column after sigma)
  T* thresh;       // B
  T* resinf;       // B
  T* basis;        // grid * (R + 1) * W
  T* gbuf;         // grid * (W + n + m) when the vectors do not fit in shared memory
  unsigned* cycle_len;  // max_it + 2
  unsigned* cycle_act;  // max_it + 2
  GridBarrier* barrier;
};

template <typename T>
struct PostParams {
  DevStructure st;
  int64_t batch;
  const T* values_all;
  int64_t values_stride;
  const T* rhs_all;
  const T* target;
  const T* lower;
  const T* upper;
  int64_t bounds_stride;
  const T* scale;
  const T* y;
  const T* dual;
  const T* gap;
  const uint8_t* cp_conv;
  T tol;
  T* meq;
  T* miq;
  T* slacks;
  int32_t* status;
  T* resid;
  uint8_t* finite;
  uint8_t* elig;
};

// ADMM forward (admm_forward.cu): sparse_admm (src/purin/solvers/admm/kernels.py:43-283)
// of one sample per CTA over a plan whose rows are all constraint rows.
template <typename T>
struct AdmmParams {
  DevStructure st;
  int64_t batch;
  const T* q;            // (B, n) positive diagonal objective
  const T* c;            // (B, n) linear objective
  const T* values;       // CSR slot order, stride values_stride (0: shared)
  int64_t values_stride;
  const T* lower;        // (B, m)
  const T* upper;        // (B, m)
  const T* penalty0;     // (B, m) initial rho per row
  const T* tolerance;    // (B,)
  const T* x0;           // (B, n) warm start (z0 = clip(K x0))
  const T* dual0;        // (B, m) or null
  // outputs
  T* x;
  T* z;
  T* dual;
  T* penalty;            // final rho
  int32_t* iterations;
  int32_t* inner_iterations;
  T* primal_residual;
  T* dual_residual;
  T* linear_residual;
  uint8_t* converged;
  uint8_t* finite;
  // configuration (ADMMConfig, admm/config.py:10-40)
  T sigma, alpha;
  int max_iterations, cg_iterations, refinement_steps, check_interval;
  T cg_tolerance;
  int adaptive_rho, rho_update_interval;
  T rho_update_threshold;
  // Banded factor (admm/factor.py): width < 0 means the PCG path.  Entries k
  // add penalty[rows[k]] * values[slot_l[k]] * values[slot_r[k]] to
  // band[dest[k]] of the (n, width + 1) lower band in the permuted order.
  int width;
  int nband;
  const int* band_perm;
  const int* band_inv;
  const int* band_rows;
  const int* band_slot_l;
  const int* band_slot_r;
  const int* band_dest;
  T* band;               // workspace: B * n * (width + 1)
  T* gstate;             // per-CTA vectors when they do not fit in shared memory
};

template <typename T>
size_t admm_state_elems(int n, int m);
template <typename T>
cudaError_t launch_admm(const AdmmParams<T>& p, bool smem, cudaStream_t stream);

// Threads per forward CTA; one-sample tiles whose state leaves room for only one
// or two CTAs of kForwardThreads per SM run 2 x or 4 x (kWideThreads) as many.
constexpr int kForwardThreads = 256;
constexpr int kWideThreads = 1024;
// One-sample QP tiles of small problems (a few hundred variables and rows): half
// the threads, twice the resident samples per SM at the same register budget.
constexpr int kNarrowThreads = 128;

// S samples per tile, NT threads per CTA; smem: the tile state lives in shared
// memory (smem_bytes of it).
template <typename T>
cudaError_t launch_forward(const FwdParams<T>& p, int S, int NT, bool smem, size_t smem_bytes,
                           cudaStream_t stream);
// Static shared memory of one forward CTA.
template <typename T>
size_t forward_static_smem(int S, int NT);
// Resident CTAs per SM of the shared-memory forward kernel (0 when the
// occupancy query fails).
template <typename T>
int forward_blocks_per_sm(int S, int NT, bool shared_values, size_t smem_bytes, bool qp = false);
template <typename T>
cudaError_t arrange_values(const T* values, const int* slot, int count, T* out, cudaStream_t stream);
// Diagonal steps of values shared by the batch (kernels.py:76-88) in the
// internal orders: sigma[pos] = s / rowsum|K|, tau[pos] = s / colsum|K|,
// a = 1/(1 + tau), d = tau a, with the forward kernel's summation order.
template <typename T>
cudaError_t diagonal_steps(const SellView& sv, const T* vr, const T* vc, T safety, T* sigma, T* tau,
                           T* a, T* d, cudaStream_t stream);
// Per-sample values into SELL order: out[b * count + e] = values[b * stride + slot[e]]
// (0 for padding) for b < batch.
template <typename T>
cudaError_t arrange_sample_values(const T* values, int64_t stride, const int* slot, int count,
                                  int64_t batch, T* out, cudaStream_t stream);
// dst[b * npos + p] = perm[p] >= 0 ? src[b * src_stride + perm[p]] : 0 for b < rows.
template <typename T>
cudaError_t permute_rows(const T* src, int64_t src_stride, const int* perm, int npos, int64_t rows,
                         T* dst, cudaStream_t stream);

// Adjoint: shared-memory bytes for one CTA, occupancy-limited cooperative grid.
template <typename T>
size_t adjoint_smem_bytes(int n, int m, int R, bool smem_vectors);
template <typename T>
int adjoint_grid(int device_sm_count, int n, int m, int R, bool smem_vectors, int64_t batch,
                 bool admm = false);
// Threads per adjoint CTA for a Krylov vector of 2n + m entries (64, 128 or 256).
int adjoint_threads(int n, int m);
// GMRES cycles with the Krylov basis in a thread-block cluster's shared memory
// (cp_gmres_cluster.cu): the smallest cluster size (1, 2, 4 or 8) whose
// per-CTA slices fit in max_smem_optin bytes, or 0; how many such clusters can
// be resident at once; and the launch (stage 0: every cycle, cooperative, with
// grid barriers; stage 2: one cycle).
template <typename T>
int gmres_cluster_size(int n, int m, int R, int max_smem_optin);
template <typename T>
int gmres_cluster_count(int C, int n, int m, int R);
template <typename T>
cudaError_t launch_gmres_cluster(const AdjParams<T>& p, int C, int clusters, cudaStream_t stream);

template <typename T>
cudaError_t launch_adjoint(const AdjParams<T>& p, int grid, bool smem_vectors,
                           cudaStream_t stream);

template <typename T>
cudaError_t launch_post(const PostParams<T>& p, cudaStream_t stream);

}  // namespace purin
