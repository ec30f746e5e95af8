// C ABI of the CP projection library (declared in include/purin_cp.h).
//
// Host-side runtime: plan construction (the prepare step of
// PreparedChambollePockProjection, solver.py:32-65, and prepare_bounds,
// bounds.py:320-326), argument validation, workspace layout, tile planning
// and kernel dispatch.  Nothing here allocates during a solve: the plan owns
// only the immutable index arrays, the caller owns every per-call buffer.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/purin_cp.h"
#include "cp_kernels.cuh"
#include "plan.cuh"
#include "sell_order.h"

namespace {

thread_local std::string g_last_error;

int32_t fail(int32_t code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

int32_t cuda_fail(cudaError_t e, const char* where) {
  return fail(PURIN_ERR_CUDA, std::string(where) + ": " + cudaGetErrorString(e));
}

// Restores the caller's current device on scope exit.
struct DeviceGuard {
  int previous = -1;
  bool ok = false;
  explicit DeviceGuard(int device) {
    if (cudaGetDevice(&previous) != cudaSuccess) previous = -1;
    ok = cudaSetDevice(device) == cudaSuccess;
  }
  ~DeviceGuard() {
    if (previous >= 0) cudaSetDevice(previous);
  }
};

size_t align_up(size_t x) { return (x + 255) & ~(size_t)255; }
int round_up_int(int x, int to) { return (x + to - 1) / to * to; }

size_t dtype_size(int32_t dtype) { return dtype == PURIN_FLOAT64 ? 8 : 4; }

constexpr uint64_t kBarrierTimeoutNs = 60ull * 1000ull * 1000ull * 1000ull;

// Forward tile plan: samples per CTA and whether the tile state fits in shared memory.
struct FwdPlan {
  int S = 1;
  int NT = purin::kForwardThreads;  // threads per CTA
  bool smem = true;
  size_t smem_bytes = 0;
  size_t workspace = 0;  // total bytes
  size_t off_vr = 0, off_vc = 0, off_state = 0;
  size_t off_tgt = 0, off_rhs = 0, off_dual0 = 0, off_lo = 0, off_up = 0;
  size_t off_q = 0, off_c = 0, off_y0 = 0;  // diagonal QP inputs (internal order)
  size_t off_ybar0 = 0;                     // resumed QP solve: ybar (internal order)
  size_t off_vr_ps = 0, off_vc_ps = 0;      // per-sample values in the SELL orders
  size_t off_dg = 0;                        // shared diagonal steps (sigma, tau, a, d)
  int sell_index = 0;  // log2(32 / C), C = 32 / S
};

FwdPlan plan_forward_tiles(PurinCpPlan* plan, const PurinCpConfig* cfg, int64_t batch,
                           bool shared_values, bool qp);

// Values shared by the batch are arranged into the two SELL orders once; values
// given per sample are arranged per sample, which the workspace must then hold
// (PURIN_CP_OP_FORWARD_SAMPLE_VALUES / PURIN_QP_OP_FORWARD_SAMPLE_VALUES).
FwdPlan plan_forward(const PurinCpPlan* plan, const PurinCpConfig* cfg, int64_t batch,
                     bool shared_values = true, bool qp = false) {
  FwdPlan fp = plan_forward_tiles(const_cast<PurinCpPlan*>(plan), cfg, batch, shared_values, qp);
  const size_t w = dtype_size(plan->info.dtype);
  fp.sell_index = 0;  // one lane per line: slices of C = 32 for every tile width
  const purin::SellView& sv = plan->sell[fp.sell_index];
  // Workspace: shared values in both sliced-ELL orders, then the per-sample inputs
  // permuted into the internal orders, then (if needed) the global tile state.
  const size_t nb = (size_t)std::max<int64_t>(batch, 0);
  fp.off_vr = 0;
  fp.off_vc = align_up((size_t)sv.nnz_r * w);
  fp.off_tgt = fp.off_vc + align_up((size_t)sv.nnz_c * w);
  fp.off_rhs = fp.off_tgt + align_up(nb * sv.n_pos * w);
  fp.off_dual0 = fp.off_rhs + align_up(nb * sv.m_pos * w);
  fp.off_lo = fp.off_dual0 + align_up(nb * sv.m_pos * w);
  fp.off_up = fp.off_lo + align_up(nb * sv.n_pos * w);
  // The diagonal QP's q, c and y0 follow; the distance projection needs none.
  const size_t qp_vec = qp ? align_up(nb * sv.n_pos * w) : 0;
  fp.off_q = fp.off_up + align_up(nb * sv.n_pos * w);
  fp.off_c = fp.off_q + qp_vec;
  fp.off_y0 = fp.off_c + qp_vec;
  fp.off_ybar0 = fp.off_y0 + qp_vec;
  const size_t ps = shared_values ? 0 : nb;
  fp.off_vr_ps = fp.off_ybar0 + qp_vec;
  fp.off_vc_ps = fp.off_vr_ps + align_up(ps * sv.nnz_r * w);
  // Diagonal steps of shared values: once per call, m_pos + 3 n_pos scalars.
  const bool dg = cfg->diagonal_preconditioning && !cfg->accelerated && shared_values;
  fp.off_dg = fp.off_vc_ps + align_up(ps * sv.nnz_c * w);
  fp.off_state = fp.off_dg + (dg ? align_up((size_t)(sv.m_pos + 3 * (size_t)sv.n_pos) * w) : 0);
  fp.workspace = fp.off_state + fp.workspace;
  return fp;
}

FwdPlan plan_forward_tiles(PurinCpPlan* plan, const PurinCpConfig* cfg, int64_t batch,
                           bool shared_values, bool qp) {
  FwdPlan fp;
  const size_t w = dtype_size(plan->info.dtype);
  const bool f64 = plan->info.dtype == PURIN_FLOAT64;
  const bool diag = cfg->diagonal_preconditioning && !cfg->accelerated;
  // Per-tile diagonal steps in shared memory: only for values given per sample
  // (with shared values the steps are computed once per call in the workspace).
  const bool pv = diag && !shared_values;
  const int n_pos = plan->sell[0].n_pos, m_pos = plan->sell[0].m_pos;
  const size_t per_sample =
      (size_t)(2 * (n_pos + 1) + (m_pos + 1) + (pv ? 2 * (n_pos + 1) + (m_pos + 1) : 0)) * w;
  const size_t cap = (size_t)plan->max_smem_optin;
  const int64_t sms = std::max(1, plan->sm_count);
  // PURIN_CP_SAMPLES_PER_TILE (1, 2, 4 or 8) overrides the tile width when it
  // fits, PURIN_CP_TILE_THREADS (256, 512, 768 or 1024; 128 for QP plans) the
  // threads per CTA.
  int forced = 0, forced_threads = 0;
  if (const char* env = std::getenv("PURIN_CP_SAMPLES_PER_TILE")) forced = std::atoi(env);
  if (const char* env = std::getenv("PURIN_CP_TILE_THREADS")) forced_threads = std::atoi(env);
  // Default: the shape whose resident CTAs hold the most warps over the batch
  // (the iteration is latency-bound), then the most samples, then the first of
  // this list.  Every shape whose state fits in shared memory is a candidate.
  // Shapes from index kFirstWideShape on are the wide multi-sample tiles.
  static const int kShapes[kForwardShapeCount][2] = {
      {1, purin::kForwardThreads},     {2, purin::kForwardThreads}, {4, purin::kForwardThreads},
      {8, purin::kForwardThreads},     {1, 2 * purin::kForwardThreads}, {1, purin::kWideThreads},
      {1, purin::kNarrowThreads},      {2, 512}, {4, 512}, {2, 768}, {4, 768}, {2, 1024}, {4, 1024}};
  constexpr int kFirstWideShape = 7;
  // The narrow QP tile only where a sample's vectors give its 128 threads at
  // most 4 entries each: larger samples keep the 256-thread tile's parallelism.
  const bool narrow_ok = qp && (int64_t)n_pos + m_pos <= 4 * purin::kNarrowThreads;
  int best = -1;
  int64_t best_warps = -1, best_samples = -1;
  int single_blocks = 0;  // resident CTAs per SM of the one-sample 256-thread tile (shape 0)
  int pair_blocks = 0;  // ... of the two-sample one (shape 1)
  int quad_blocks = 0;  // ... and of the four-sample one (shape 2)
  for (int k = 0; k < kForwardShapeCount; ++k) {
    const int S = kShapes[k][0], NT = kShapes[k][1];
    if (qp && S != 1) continue;  // the QP kernels are built for one-sample tiles
    if (k >= kFirstWideShape && forced == 0 && forced_threads == 0) continue;  // forced only
    if (NT == purin::kNarrowThreads && !(narrow_ok || (qp && forced_threads == NT))) continue;
    const size_t stat = f64 ? purin::forward_static_smem<double>(S, NT)
                            : purin::forward_static_smem<float>(S, NT);
    // Shared-memory tiles read the 16-bit index pairs (always present when a
    // sample's state fits in shared memory).
    if (!plan->sell[0].idx16 || (size_t)S * per_sample + stat + 1024 > cap) continue;
    if (forced > 0 || forced_threads > 0) {
      const int want_s = forced > 0 ? forced : 8;
      const int want_nt = forced_threads > 0 ? forced_threads : purin::kForwardThreads;
      if (NT == want_nt && S <= want_s && (best < 0 || S > kShapes[best][0])) best = k;
      continue;
    }
    int& cached = plan->fwd_blocks[qp ? (pv ? 3 : 2) : (pv ? 1 : 0)][shared_values ? 1 : 0][k];
    if (cached < 0) {
      const size_t dyn = (size_t)S * per_sample;
      cached = f64 ? purin::forward_blocks_per_sm<double>(S, NT, shared_values, dyn, qp)
                   : purin::forward_blocks_per_sm<float>(S, NT, shared_values, dyn, qp);
    }
    if (k == 0) single_blocks = std::max(cached, 0);
    if (k == 1) pair_blocks = std::max(cached, 0);
    if (k == 2) quad_blocks = std::max(cached, 0);
    const int64_t tiles = (batch + S - 1) / S;
    const int64_t ctas = std::min<int64_t>(tiles, sms * std::max(cached, 0));
    const int64_t warps = ctas * (NT / 32);
    const int64_t samples = std::min<int64_t>(batch, ctas * S);
    if (best < 0 || warps > best_warps || (warps == best_warps && samples > best_samples)) {
      best = k;
      best_warps = warps;
      best_samples = samples;
    }
  }
  // fp32: a two-sample tile serves both samples' gathers with one 8-byte access
  // per lane and shares every structure load between them.  Measured on
  // configurations 1 and 4 it beats the one-sample tile even with a half or a
  // quarter fewer resident warps (39.9 against 49.3 ms, 929 against 1038 ms),
  // whereas for fp64 the one-sample tile stays ahead.  It is taken whenever the
  // batch fills at least two such tiles per SM.
  if (!f64 && best >= 0 && forced == 0 && forced_threads == 0 && pair_blocks >= 2 &&
      (batch + 1) / 2 >= sms * pair_blocks && kShapes[best][0] == 1)
    best = 1;
  // fp64 two-sample tiles with three CTAs per SM (80 registers) share each
  // structure load between two samples; a tile takes about 1.25x a one-sample
  // tile's time (configuration 1 fp64: 11.5 against 9.2 ms per wave), so they are
  // taken when their waves, weighted by that ratio, beat the one-sample tiles'
  // waves: configuration 1 fp64 at 4096 samples 59.3k -> 67.9k samples/s, at
  // 16 384 62.4k -> 73.3k.  Configuration 2's samples (45 KB) leave room for two
  // such tiles per SM only, and keep the one-sample tiles.
  if (f64 && best == 0 && forced == 0 && forced_threads == 0 && pair_blocks >= 3 &&
      single_blocks >= 1) {
    const int64_t single_waves = (batch + sms * single_blocks - 1) / (sms * single_blocks);
    const int64_t pair_waves = ((batch + 1) / 2 + sms * pair_blocks - 1) / (sms * pair_blocks);
    if (125 * pair_waves < 100 * single_waves) best = 1;
  }
  // fp32 four-sample tiles with three CTAs per SM share each structure load and
  // each gather instruction among four samples; a tile takes about 1.27x a
  // two-sample tile's time (configuration 1 fp32: 11.4 against 9.0 ms per wave),
  // so per sample they are faster when whole waves are compared.  Chosen when
  // their waves, weighted by that ratio, beat the two-sample tiles' waves:
  // 4096 samples 108.3k -> 113.2k samples/s (3 waves against 4); at 2048 the
  // two-sample tiles stay (2 waves each).
  if (!f64 && best == 1 && forced == 0 && forced_threads == 0 && quad_blocks >= 3 &&
      pair_blocks >= 1) {
    const int64_t pair_waves = ((batch + 1) / 2 + sms * pair_blocks - 1) / (sms * pair_blocks);
    const int64_t quad_waves = ((batch + 3) / 4 + sms * quad_blocks - 1) / (sms * quad_blocks);
    if (127 * quad_waves < 100 * pair_waves) best = 2;
  }
  // A structure far larger than the L1 beside the tile state streams from L2
  // once per tile-iteration (value plus 16-bit index per stored entry, both
  // products).  A wide tile of 4 (else 2) samples on 768 threads shares that
  // stream among its samples and keeps 24 warps.  Configuration 4 (n = 4096,
  // m = 3072, 16 nnz per row, 16 384 samples; 0.98 MB of fp64 structure):
  // fp64 1 585 -> 1 384 ms per launch (S = 2), fp32 952 -> 750 ms (S = 4),
  // and 1 360 / 696 ms with the line order chosen for these tiles' gathers;
  // configurations 1 and 2 (0.12 and 0.25 MB) are faster on the narrow tiles
  // (configuration 2: 125.2 ms against 129.7 with S = 2 and 171.6 with S = 4).
  // Taken above 384 KB of structure when the batch fills one tile per SM.
  // Every tile shape gives the same bits, so shards may differ in shape.
  if (!qp && best >= 0 && forced == 0 && forced_threads == 0 &&
      wide_structure(plan->info.kept_nnz, w)) {
    for (const int S : {4, 2}) {
      int k = kFirstWideShape;
      while (k < kForwardShapeCount && !(kShapes[k][0] == S && kShapes[k][1] == 768)) ++k;
      const size_t stat = f64 ? purin::forward_static_smem<double>(S, 768)
                              : purin::forward_static_smem<float>(S, 768);
      if (k == kForwardShapeCount || (size_t)S * per_sample + stat + 1024 > cap ||
          batch < (int64_t)S * sms)
        continue;
      int& cached = plan->fwd_blocks[pv ? 1 : 0][shared_values ? 1 : 0][k];
      if (cached < 0) {
        const size_t dyn = (size_t)S * per_sample;
        cached = f64 ? purin::forward_blocks_per_sm<double>(S, 768, shared_values, dyn, false)
                     : purin::forward_blocks_per_sm<float>(S, 768, shared_values, dyn, false);
      }
      if (cached >= 1) {
        best = k;
        break;
      }
    }
  }
  if (best >= 0) {
    fp.S = kShapes[best][0];
    fp.NT = kShapes[best][1];
    fp.smem = true;
    fp.smem_bytes = (size_t)fp.S * per_sample;
    fp.workspace = 0;
  } else {
    fp.S = qp ? 1 : 8;
    fp.NT = purin::kForwardThreads;
    fp.smem = false;
    fp.smem_bytes = 0;
    const int64_t tiles = (batch + fp.S - 1) / fp.S;
    fp.workspace = align_up((size_t)tiles * fp.S * per_sample);
  }
  return fp;
}

struct AdjLayout {
  int R = 1;
  int grid = 0;
  bool smem = true;
  // GMRES cycles on thread-block clusters holding the Krylov basis on chip: the
  // cluster size (0: the CTA-per-sample kernel runs the cycles, its basis in the
  // workspace) and the number of co-resident clusters.
  int C = 0;
  int clusters = 0;
  size_t off_x, off_lamp, off_steps, off_dsteps, off_thresh, off_resinf, off_basis, off_gbuf;
  size_t off_ycode, off_dcode, off_counters, counters_bytes, total;
};

AdjLayout plan_adjoint(const PurinCpPlan* plan, const PurinCpConfig* cfg,
                       const PurinLinearSolverConfig* lin, int64_t batch, bool qp = false,
                       int64_t total_batch = 0, bool admm = false) {
  AdjLayout L;
  const int n = plan->info.n, m = plan->info.kept_rows;
  // The CP pullback's state is (y, dual, ybar); ADMM's KKT system is (x, dual).
  const int64_t W = admm ? (int64_t)n + m : 2 * (int64_t)n + m;
  const size_t w = dtype_size(plan->info.dtype);
  L.R = (int)std::min<int64_t>(std::min<int64_t>(lin->restart, lin->max_iterations), W);
  if (L.R < 1) L.R = 1;
  const bool f64 = plan->info.dtype == PURIN_FLOAT64;
  const size_t smem_full = f64 ? purin::adjoint_smem_bytes<double>(n, m, L.R, true)
                               : purin::adjoint_smem_bytes<float>(n, m, L.R, true);
  L.smem = smem_full + 1024 <= (size_t)plan->max_smem_optin;
  L.grid = f64 ? purin::adjoint_grid<double>(plan->sm_count, n, m, L.R, L.smem, batch, admm)
               : purin::adjoint_grid<float>(plan->sm_count, n, m, L.R, L.smem, batch, admm);
  // GMRES cycles on clusters that hold the basis on chip, or on the
  // CTA-per-sample kernel that streams it from HBM.  A cluster step is bound by
  // latency (barriers across the cluster: config 2 runs about 13 us per Arnoldi
  // step on 8 SMs), a streaming step by bandwidth shared among all resident
  // samples; measured on configuration 2 (fp64, 2048 samples) the streaming
  // kernel takes 150 ms and the clusters 190 ms.  The clusters therefore take
  // the cycles of a problem whose vectors need the full 256-thread CTA and whose
  // basis slices fit a cluster of at most 8 CTAs only when the whole batch fits
  // in one wave of clusters, where the streaming kernel would leave most SMs
  // idle.  The choice depends on the problem and the GLOBAL batch (the same for
  // every shard of it), so shards of a batch round alike.
  // PURIN_CP_GMRES_CLUSTER=0 never uses the clusters, =1 whenever they fit.
  const char* cl_env = std::getenv("PURIN_CP_GMRES_CLUSTER");
  const bool cl_off = cl_env && std::string(cl_env) == "0";
  const bool cl_force = cl_env && std::string(cl_env) == "1";
  if (!cl_off && !admm && purin::adjoint_threads(n, m) == 256) {
    L.C = f64 ? purin::gmres_cluster_size<double>(n, m, L.R, plan->max_smem_optin)
              : purin::gmres_cluster_size<float>(n, m, L.R, plan->max_smem_optin);
    const int64_t global = std::max<int64_t>(total_batch > 0 ? total_batch : batch, 1);
    if (L.C > 0 && !cl_force && global > plan->sm_count / L.C) L.C = 0;  // no overflow
    if (L.C > 0) {
      const int resident = f64 ? purin::gmres_cluster_count<double>(L.C, n, m, L.R)
                               : purin::gmres_cluster_count<float>(L.C, n, m, L.R);
      L.clusters = (int)std::min<int64_t>(resident, std::max<int64_t>(batch, 1));
      if (L.clusters < 1) L.C = 0;
    }
  }
  const bool diag = cfg->diagonal_preconditioning && !cfg->accelerated;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off = align_up(off + bytes);
    return o;
  };
  L.off_x = take((size_t)batch * W * w);
  L.off_lamp = take((size_t)batch * m * w);
  L.off_steps = take((size_t)batch * 2 * w);
  // Per-variable steps: diagonal preconditioning, or every diagonal QP
  // (a_j, d_j depend on q_j; tau per column follows for the q cotangent).
  L.off_dsteps = take(qp ? (size_t)batch * (3 * n + m) * w : diag ? (size_t)batch * (2 * n + m) * w : 0);
  L.off_thresh = take((size_t)batch * w);
  L.off_resinf = take((size_t)batch * w);
  L.off_basis = take(L.C > 0 ? 0 : (size_t)std::max(L.grid, 1) * (L.R + 1) * W * w);
  L.off_gbuf = take(L.smem ? 0 : (size_t)std::max(L.grid, 1) * (W + n + m) * w);
  L.off_ycode = take((size_t)batch * n);
  L.off_dcode = take((size_t)batch * m);
  L.counters_bytes = align_up(2 * (size_t)(lin->max_iterations + 2) * sizeof(unsigned) +
                              sizeof(purin::GridBarrier));
  L.off_counters = take(L.counters_bytes);
  L.total = off;
  return L;
}

int32_t check_plan(const PurinCpPlan* plan) {
  if (!plan) return fail(PURIN_ERR_INVALID_ARGUMENT, "plan is NULL");
  return PURIN_OK;
}

int32_t check_config(const PurinCpConfig* cfg) {
  if (!cfg) return fail(PURIN_ERR_INVALID_ARGUMENT, "config is NULL");
  if (cfg->max_iterations < 1) return fail(PURIN_ERR_INVALID_ARGUMENT, "max_iterations must be a positive integer");
  if (!(cfg->safety > 0.0 && cfg->safety < 1.0))
    return fail(PURIN_ERR_INVALID_ARGUMENT, "safety must be between zero and one");
  if (cfg->norm_iterations < 1) return fail(PURIN_ERR_INVALID_ARGUMENT, "norm_iterations must be a positive integer");
  return PURIN_OK;
}

int32_t check_linear(const PurinLinearSolverConfig* lin) {
  if (!lin) return fail(PURIN_ERR_INVALID_ARGUMENT, "linear solver config is NULL");
  if (!(lin->tolerance > 0.0) || lin->atol < 0.0) return fail(PURIN_ERR_INVALID_ARGUMENT, "linear tolerances are invalid");
  if (lin->restart < 1 || lin->max_iterations < 1)
    return fail(PURIN_ERR_INVALID_ARGUMENT, "linear iteration limits must be positive");
  return PURIN_OK;
}

// The diagonal QP's extra forward inputs (purin_qp_forward); null for the
// distance projection.
struct QpInputs {
  const void* q;
  const void* c;
  const void* y0;
  int32_t flags;
  const void* ybar0;               // resume: extrapolated iterate (null: y0)
  const int32_t* start_iterations;  // resume: iterations already run (null: 0)
  void* ybar;                       // out: final extrapolated iterate (null: not written)
};

template <typename T>
int32_t run_forward(const PurinCpPlan* plan, const PurinCpConfig* cfg, const PurinCpForwardArgs* a,
                    void* workspace, size_t workspace_bytes, cudaStream_t stream,
                    const QpInputs* qp = nullptr) {
  const bool shared = a->values_stride == 0 || a->batch == 1 || plan->info.kept_nnz == 0;
  const FwdPlan fp = plan_forward(plan, cfg, a->batch, shared, qp != nullptr);
  if (workspace == nullptr || workspace_bytes < fp.workspace)
    return fail(PURIN_ERR_WORKSPACE,
                "forward workspace too small: need " + std::to_string(fp.workspace) + " bytes" +
                    (shared ? "" : " for values given per sample (size it with the *_SAMPLE_VALUES op)"));
  char* ws = static_cast<char*>(workspace);
  const purin::SellView& sv = plan->sell[fp.sell_index];
  // Values shared by the batch are arranged once per call in both sliced-ELL orders.
  T* vr = nullptr;
  T* vc = nullptr;
  if (shared && plan->info.kept_nnz > 0) {
    vr = reinterpret_cast<T*>(ws + fp.off_vr);
    vc = reinterpret_cast<T*>(ws + fp.off_vc);
    cudaError_t e = purin::arrange_values<T>(static_cast<const T*>(a->values), sv.r_slot, sv.nnz_r, vr, stream);
    if (e == cudaSuccess)
      e = purin::arrange_values<T>(static_cast<const T*>(a->values), sv.c_slot, sv.nnz_c, vc, stream);
    if (e != cudaSuccess) return cuda_fail(e, "purin_cp_forward value layout");
  }
  // Values given per sample: each sample's copy in both SELL orders, so the solve
  // reads them coalesced and without the slot indirection.
  T* vr_ps = nullptr;
  T* vc_ps = nullptr;
  if (!shared) {
    vr_ps = reinterpret_cast<T*>(ws + fp.off_vr_ps);
    vc_ps = reinterpret_cast<T*>(ws + fp.off_vc_ps);
    const T* vals = static_cast<const T*>(a->values);
    cudaError_t e = purin::arrange_sample_values<T>(vals, a->values_stride, sv.r_slot, sv.nnz_r, a->batch,
                                                    vr_ps, stream);
    if (e == cudaSuccess)
      e = purin::arrange_sample_values<T>(vals, a->values_stride, sv.c_slot, sv.nnz_c, a->batch, vc_ps,
                                          stream);
    if (e != cudaSuccess) return cuda_fail(e, "purin_cp_forward per-sample value layout");
  }
  // Per-sample inputs in the internal row/column orders (coalesced per-iteration reads).
  T* tgt_i = reinterpret_cast<T*>(ws + fp.off_tgt);
  T* rhs_i = reinterpret_cast<T*>(ws + fp.off_rhs);
  T* dual0_i = a->dual0 ? reinterpret_cast<T*>(ws + fp.off_dual0) : nullptr;
  T* lo_i = reinterpret_cast<T*>(ws + fp.off_lo);
  T* up_i = reinterpret_cast<T*>(ws + fp.off_up);
  const int64_t bound_rows = a->bounds_stride == 0 ? 1 : a->batch;
  T* q_i = qp ? reinterpret_cast<T*>(ws + fp.off_q) : nullptr;
  T* c_i = qp ? reinterpret_cast<T*>(ws + fp.off_c) : nullptr;
  T* y0_i = (qp && qp->y0) ? reinterpret_cast<T*>(ws + fp.off_y0) : nullptr;
  T* ybar0_i = (qp && qp->ybar0) ? reinterpret_cast<T*>(ws + fp.off_ybar0) : nullptr;
  {
    const int n = plan->info.n, m = plan->info.kept_rows;
    cudaError_t e = cudaSuccess;
    if (qp) {
      e = purin::permute_rows<T>(static_cast<const T*>(qp->q), n, sv.c_perm, sv.n_pos, a->batch, q_i, stream);
      if (e == cudaSuccess)
        e = purin::permute_rows<T>(static_cast<const T*>(qp->c), n, sv.c_perm, sv.n_pos, a->batch, c_i,
                                   stream);
      if (e == cudaSuccess && y0_i)
        e = purin::permute_rows<T>(static_cast<const T*>(qp->y0), n, sv.c_perm, sv.n_pos, a->batch, y0_i,
                                   stream);
      if (e == cudaSuccess && ybar0_i)
        e = purin::permute_rows<T>(static_cast<const T*>(qp->ybar0), n, sv.c_perm, sv.n_pos, a->batch,
                                   ybar0_i, stream);
    } else {
      e = purin::permute_rows<T>(static_cast<const T*>(a->target), n, sv.c_perm, sv.n_pos, a->batch, tgt_i,
                                 stream);
    }
    if (e == cudaSuccess && m > 0)
      e = purin::permute_rows<T>(static_cast<const T*>(a->rhs), m, sv.r_perm, sv.m_pos, a->batch,
                                 rhs_i, stream);
    if (e == cudaSuccess && m == 0)
      e = cudaMemsetAsync(rhs_i, 0, (size_t)a->batch * sv.m_pos * sizeof(T), stream);
    if (e == cudaSuccess && dual0_i && m > 0)
      e = purin::permute_rows<T>(static_cast<const T*>(a->dual0), m, sv.r_perm, sv.m_pos, a->batch,
                                 dual0_i, stream);
    if (e == cudaSuccess)
      e = purin::permute_rows<T>(static_cast<const T*>(a->lower), a->bounds_stride, sv.c_perm,
                                 sv.n_pos, bound_rows, lo_i, stream);
    if (e == cudaSuccess)
      e = purin::permute_rows<T>(static_cast<const T*>(a->upper), a->bounds_stride, sv.c_perm,
                                 sv.n_pos, bound_rows, up_i, stream);
    if (e != cudaSuccess) return cuda_fail(e, "purin_cp_forward input layout");
  }
  purin::FwdParams<T> p{};
  p.tgt_i = qp ? nullptr : tgt_i;
  p.q_i = q_i;
  p.c_i = c_i;
  p.y0_i = y0_i;
  p.qp_flags = qp ? qp->flags : 0;
  p.ybar0_i = ybar0_i;
  p.start_it = qp ? qp->start_iterations : nullptr;
  p.ybar_out = qp ? static_cast<T*>(qp->ybar) : nullptr;
  p.rhs_i = rhs_i;
  p.dual0_i = (dual0_i && plan->info.kept_rows > 0) ? dual0_i : nullptr;
  p.lo_i = lo_i;
  p.up_i = up_i;
  p.bstride_i = a->bounds_stride == 0 ? 0 : plan->sell[0].n_pos;
  p.st = plan->dev;
  p.batch = a->batch;
  p.values = static_cast<const T*>(a->values);
  p.values_stride = a->values_stride;
  p.rhs = static_cast<const T*>(a->rhs);
  p.target = static_cast<const T*>(a->target);
  p.dual0 = static_cast<const T*>(a->dual0);
  p.tol = static_cast<const T*>(a->tolerance);
  p.lower = static_cast<const T*>(a->lower);
  p.upper = static_cast<const T*>(a->upper);
  p.bounds_stride = a->bounds_stride;
  p.feasible = a->feasible;
  p.sample_offset = a->sample_offset;
  p.total_batch = a->total_batch > 0 ? a->total_batch : a->batch;
  p.y_out = static_cast<T*>(a->y);
  p.dual_out = static_cast<T*>(a->dual);
  p.it_out = a->iterations;
  p.res_out = static_cast<T*>(a->residual);
  p.gap_out = static_cast<T*>(a->gap);
  p.conv_out = a->converged;
  p.max_iterations = cfg->max_iterations;
  p.accelerated = cfg->accelerated ? 1 : 0;
  p.safety = (T)cfg->safety;
  p.norm_iterations = cfg->norm_iterations;
  p.norm_seed = cfg->norm_seed;
  p.norm_bound = cfg->norm_bound ? 1 : 0;
  p.diag = (cfg->diagonal_preconditioning && !cfg->accelerated) ? 1 : 0;
  p.partitionable = cfg->prng_partitionable ? 1 : 0;
  p.gstate = fp.smem ? nullptr : reinterpret_cast<T*>(ws + fp.off_state);
  p.sell = sv;
  p.vr = vr;
  p.vc = vc;
  p.vr_ps = vr_ps;
  p.vc_ps = vc_ps;
  if (p.diag && shared) {
    T* dgp = reinterpret_cast<T*>(ws + fp.off_dg);
    const int n_pos = sv.n_pos, m_pos = sv.m_pos;
    p.dg_sigma = dgp;
    p.dg_tau = dgp + m_pos;
    p.dg_a = dgp + m_pos + n_pos;
    p.dg_d = dgp + m_pos + 2 * (size_t)n_pos;
    cudaError_t e = purin::diagonal_steps<T>(sv, vr, vc, p.safety, dgp, dgp + m_pos, dgp + m_pos + n_pos,
                                             dgp + m_pos + 2 * (size_t)n_pos, stream);
    if (e != cudaSuccess) return cuda_fail(e, "purin_cp_forward diagonal steps");
  }
  p.nnz_r_ps = sv.nnz_r;
  p.nnz_c_ps = sv.nnz_c;
  cudaError_t e = purin::launch_forward<T>(p, fp.S, fp.NT, fp.smem, fp.smem_bytes, stream);
  if (e != cudaSuccess) return cuda_fail(e, "purin_cp_forward launch");
  return PURIN_OK;
}

template <typename T>
purin::AdjParams<T> adjoint_params(const PurinCpPlan* plan, const PurinCpConfig* cfg,
                                   const PurinLinearSolverConfig* lin, const PurinCpAdjointArgs* a,
                                   const AdjLayout& L, char* ws) {
  purin::AdjParams<T> p{};
  p.st = plan->dev;
  p.batch = a->batch;
  p.values = static_cast<const T*>(a->values);
  p.values_stride = a->values_stride;
  p.rhs = static_cast<const T*>(a->rhs);
  p.target = static_cast<const T*>(a->target);
  p.lower = static_cast<const T*>(a->lower);
  p.upper = static_cast<const T*>(a->upper);
  p.bounds_stride = a->bounds_stride;
  p.y = static_cast<const T*>(a->y);
  p.dual = static_cast<const T*>(a->dual);
  p.converged = a->converged;
  p.cot_y = static_cast<const T*>(a->cot_y);
  p.sample_offset = a->sample_offset;
  p.total_batch = a->total_batch > 0 ? a->total_batch : a->batch;
  p.g_values = static_cast<T*>(a->grad_values);
  p.g_rhs = static_cast<T*>(a->grad_rhs);
  p.g_target = static_cast<T*>(a->grad_target);
  p.g_lower = static_cast<T*>(a->grad_lower);
  p.g_upper = static_cast<T*>(a->grad_upper);
  p.lin_status = a->linear_status;
  p.lin_residual = static_cast<T*>(a->linear_residual);
  p.device_error = a->device_error;
  const bool work = a->arnoldi_steps != nullptr && a->krylov_vectors != nullptr;
  p.work_steps = work ? a->arnoldi_steps : nullptr;
  p.work_vectors = work ? reinterpret_cast<long long*>(a->krylov_vectors) : nullptr;
  p.accelerated = cfg->accelerated ? 1 : 0;
  p.diag = (cfg->diagonal_preconditioning && !cfg->accelerated) ? 1 : 0;
  p.norm_iterations = cfg->norm_iterations;
  p.partitionable = cfg->prng_partitionable ? 1 : 0;
  p.norm_seed = cfg->norm_seed;
  p.safety = (T)cfg->safety;
  p.lin_tol = (T)lin->tolerance;
  p.lin_atol = (T)lin->atol;
  p.adj_tol = (T)lin->adjoint_tolerance;
  p.R = L.R;
  p.max_it = lin->max_iterations;
  p.timeout_ns = kBarrierTimeoutNs;
  p.barrier_extra = 0;
  // Failure-detection test: PURIN_CP_TEST_UNREACHABLE_BARRIER=<ms> makes the
  // fused kernel's grid barrier wait for one arrival more than the grid has, so
  // the bounded wait gives up after <ms> milliseconds and the call reports it
  // through device_error (the context stays usable).
  if (const char* env = std::getenv("PURIN_CP_TEST_UNREACHABLE_BARRIER")) {
    const long ms = std::atol(env);
    if (ms > 0) {
      p.barrier_extra = 1;
      p.timeout_ns = (uint64_t)ms * 1000000ull;
    }
  }
  p.x = reinterpret_cast<T*>(ws + L.off_x);
  p.lamp = reinterpret_cast<T*>(ws + L.off_lamp);
  p.steps = reinterpret_cast<T*>(ws + L.off_steps);
  p.dsteps = reinterpret_cast<T*>(ws + L.off_dsteps);
  p.thresh = reinterpret_cast<T*>(ws + L.off_thresh);
  p.resinf = reinterpret_cast<T*>(ws + L.off_resinf);
  p.basis = reinterpret_cast<T*>(ws + L.off_basis);
  p.gbuf = L.smem ? nullptr : reinterpret_cast<T*>(ws + L.off_gbuf);
  p.ycode = reinterpret_cast<uint8_t*>(ws + L.off_ycode);
  p.dcode = reinterpret_cast<uint8_t*>(ws + L.off_dcode);
  unsigned* counters = reinterpret_cast<unsigned*>(ws + L.off_counters);
  p.cycle_len = counters;
  p.cycle_act = counters + (lin->max_iterations + 2);
  p.barrier = reinterpret_cast<purin::GridBarrier*>(counters + 2 * (lin->max_iterations + 2));
  p.stage = 0;
  p.completed0 = 0;
  return p;
}

// The diagonal QP's extra adjoint inputs and outputs (purin_qp_adjoint).
struct QpAdjoint {
  const void* q;
  const void* c;
  const void* cot_dual;
  void* grad_q;
  void* grad_c;
};

template <typename T>
void set_qp(purin::AdjParams<T>& p, const QpAdjoint* qp, const PurinCpConfig* cfg) {
  if (!qp) return;
  p.qp = 1;
  p.q = static_cast<const T*>(qp->q);
  p.c = static_cast<const T*>(qp->c);
  p.cot_dual = static_cast<const T*>(qp->cot_dual);
  p.g_q = static_cast<T*>(qp->grad_q);
  p.g_c = static_cast<T*>(qp->grad_c);
  p.norm_bound = cfg->norm_bound ? 1 : 0;
}

// ADMM's extra adjoint inputs (purin_admm_adjoint): the activity thresholds.
struct AdmmAdjoint {
  double active_tolerance;
  double tolerance;
};

template <typename T>
void set_admm(purin::AdjParams<T>& p, const AdmmAdjoint* admm) {
  if (!admm) return;
  p.mode = 1;
  p.act_tol = (T)admm->active_tolerance;
  p.fwd_tol = (T)admm->tolerance;
}

template <typename T>
int32_t run_adjoint(const PurinCpPlan* plan, const PurinCpConfig* cfg, const PurinLinearSolverConfig* lin,
                    const PurinCpAdjointArgs* a, void* workspace, size_t workspace_bytes,
                    cudaStream_t stream, const QpAdjoint* qp = nullptr,
                    const AdmmAdjoint* admm = nullptr) {
  const AdjLayout L = plan_adjoint(plan, cfg, lin, a->batch, qp != nullptr, a->total_batch, admm != nullptr);
  if (L.grid < 1) return fail(PURIN_ERR_UNSUPPORTED, "adjoint kernel cannot be made resident on this device");
  if (workspace == nullptr || workspace_bytes < L.total)
    return fail(PURIN_ERR_WORKSPACE, "adjoint workspace too small: need " + std::to_string(L.total) + " bytes");
  if (!a->device_error) return fail(PURIN_ERR_INVALID_ARGUMENT, "device_error pointer is required");
  char* ws = static_cast<char*>(workspace);
  cudaError_t e = cudaMemsetAsync(ws + L.off_counters, 0, L.counters_bytes, stream);
  if (e != cudaSuccess) return cuda_fail(e, "purin_cp_adjoint memset");
  e = cudaMemsetAsync(a->device_error, 0, sizeof(int32_t), stream);
  if (e != cudaSuccess) return cuda_fail(e, "purin_cp_adjoint memset");
  purin::AdjParams<T> p = adjoint_params<T>(plan, cfg, lin, a, L, ws);
  set_qp(p, qp, cfg);
  set_admm(p, admm);
  if (L.C > 0) {
    // Prepare on the CTA-per-sample kernel, every GMRES cycle on the clusters
    // (one cooperative launch with grid barriers between cycles), then the
    // pullback; the state passes through the workspace.
    p.stage = 1;
    e = purin::launch_adjoint<T>(p, L.grid, L.smem, stream);
    if (e != cudaSuccess) return cuda_fail(e, "purin_cp_adjoint launch (prepare)");
    p.stage = 0;
    e = purin::launch_gmres_cluster<T>(p, L.C, L.clusters, stream);
    if (e != cudaSuccess) return cuda_fail(e, "purin_cp_adjoint launch (GMRES clusters)");
    p.stage = 3;
    e = purin::launch_adjoint<T>(p, L.grid, L.smem, stream);
    if (e != cudaSuccess) return cuda_fail(e, "purin_cp_adjoint launch (pullback)");
    return PURIN_OK;
  }
  e = purin::launch_adjoint<T>(p, L.grid, L.smem, stream);
  if (e != cudaSuccess) return cuda_fail(e, "purin_cp_adjoint launch");
  return PURIN_OK;
}

// One phase of the adjoint (see purin_cp_adjoint_stage in the header).  The
// counters of the phase go to the caller's two words: stage PREPARE writes
// {0, samples above their GMRES threshold}; stage CYCLE writes {Arnoldi steps
// of the cycle (the largest over this shard's samples), samples still above
// their threshold after it}.
template <typename T>
int32_t run_adjoint_stage(const PurinCpPlan* plan, const PurinCpConfig* cfg, const PurinLinearSolverConfig* lin,
                          const PurinCpAdjointArgs* a, int32_t stage, int32_t completed, int32_t* counters,
                          void* workspace, size_t workspace_bytes, cudaStream_t stream,
                          const QpAdjoint* qp = nullptr, const AdmmAdjoint* admm = nullptr) {
  const AdjLayout L = plan_adjoint(plan, cfg, lin, a->batch, qp != nullptr, a->total_batch,
                                   admm != nullptr);
  if (L.grid < 1) return fail(PURIN_ERR_UNSUPPORTED, "adjoint kernel cannot be made resident on this device");
  if (workspace == nullptr || workspace_bytes < L.total)
    return fail(PURIN_ERR_WORKSPACE, "adjoint workspace too small: need " + std::to_string(L.total) + " bytes");
  if (!a->device_error) return fail(PURIN_ERR_INVALID_ARGUMENT, "device_error pointer is required");
  char* ws = static_cast<char*>(workspace);
  cudaError_t e = cudaSuccess;
  if (stage == PURIN_CP_STAGE_PREPARE) {
    e = cudaMemsetAsync(a->device_error, 0, sizeof(int32_t), stream);
    if (e != cudaSuccess) return cuda_fail(e, "purin_cp_adjoint_stage memset");
  }
  if (stage != PURIN_CP_STAGE_FINISH) {
    e = cudaMemsetAsync(counters, 0, 2 * sizeof(int32_t), stream);
    if (e != cudaSuccess) return cuda_fail(e, "purin_cp_adjoint_stage memset");
  }
  purin::AdjParams<T> p = adjoint_params<T>(plan, cfg, lin, a, L, ws);
  set_qp(p, qp, cfg);
  set_admm(p, admm);
  unsigned* words = reinterpret_cast<unsigned*>(counters);
  p.barrier = nullptr;
  p.completed0 = completed;
  if (stage == PURIN_CP_STAGE_PREPARE) {
    p.stage = 1;
    p.cycle_len = words;      // unused by the prepare phase
    p.cycle_act = words + 1;  // cycle_act[0] -> word 1
  } else if (stage == PURIN_CP_STAGE_CYCLE) {
    p.stage = 2;
    p.cycle_len = words;  // cycle_len[0] -> word 0
    p.cycle_act = words;  // cycle_act[1] -> word 1
  } else {
    p.stage = 3;
    p.cycle_len = nullptr;
    p.cycle_act = nullptr;
  }
  if (p.stage == 2 && L.C > 0) {
    e = purin::launch_gmres_cluster<T>(p, L.C, L.clusters, stream);
    if (e != cudaSuccess) return cuda_fail(e, "purin_cp_adjoint_stage launch (GMRES clusters)");
    return PURIN_OK;
  }
  e = purin::launch_adjoint<T>(p, L.grid, L.smem, stream);
  if (e != cudaSuccess) return cuda_fail(e, "purin_cp_adjoint_stage launch");
  return PURIN_OK;
}

template <typename T>
int32_t run_post(const PurinCpPlan* plan, const PurinCpPostArgs* a, cudaStream_t stream) {
  purin::PostParams<T> p{};
  p.st = plan->dev;
  p.batch = a->batch;
  p.values_all = static_cast<const T*>(a->values_all);
  p.values_stride = a->values_all_stride;
  p.rhs_all = static_cast<const T*>(a->rhs_all);
  p.target = static_cast<const T*>(a->target);
  p.lower = static_cast<const T*>(a->lower);
  p.upper = static_cast<const T*>(a->upper);
  p.bounds_stride = a->bounds_stride;
  p.scale = static_cast<const T*>(a->scale);
  p.y = static_cast<const T*>(a->y);
  p.dual = static_cast<const T*>(a->dual);
  p.gap = static_cast<const T*>(a->gap);
  p.cp_conv = a->cp_converged;
  p.tol = (T)a->tolerance;
  p.meq = static_cast<T*>(a->multipliers_eq);
  p.miq = static_cast<T*>(a->multipliers_ineq);
  p.slacks = static_cast<T*>(a->slacks);
  p.status = a->status;
  p.resid = static_cast<T*>(a->residual_inf_norm);
  p.finite = a->finite;
  p.elig = a->gradient_eligible;
  cudaError_t e = purin::launch_post<T>(p, stream);
  if (e != cudaSuccess) return cuda_fail(e, "purin_cp_postprocess launch");
  return PURIN_OK;
}

// Lines sorted by length, descending (stable): the sliced-ELL line order before
// the bank-aware search.
std::vector<int> length_order(int count, const std::vector<int32_t>& ptr) {
  std::vector<int> order(count);
  for (int i = 0; i < count; ++i) order[i] = i;
  std::stable_sort(order.begin(), order.end(),
                   [&](int a, int b) { return ptr[a + 1] - ptr[a] > ptr[b + 1] - ptr[b]; });
  return order;
}

// Sliced-ELL layout (sell.cuh) of `count` lines with entries ptr_in/idx_in and slots
// slot_in (identity when null), slices of C lines in the given order (position ->
// line); a slice is as wide as its longest line.
struct SellHost {
  int nsl = 0;
  std::vector<int32_t> ptr, perm, idx, slot;
  std::vector<uint32_t> idx2;  // index pairs (sell.cuh), empty when positions need 32 bits
};

SellHost build_sell(int count, const std::vector<int32_t>& ptr_in, const std::vector<int32_t>& idx_in,
                    const std::vector<int32_t>* slot_in, int C, int pad_index,
                    const std::vector<int>& order) {
  SellHost h;
  auto len = [&](int i) { return ptr_in[i + 1] - ptr_in[i]; };
  h.nsl = (count + C - 1) / C;
  h.perm.assign((size_t)h.nsl * C, -1);
  for (int q = 0; q < count; ++q) h.perm[q] = order[q];
  h.ptr.assign(h.nsl + 1, 0);
  for (int s = 0; s < h.nsl; ++s) {
    int width = 0;
    for (int q = s * C; q < std::min(count, (s + 1) * C); ++q) width = std::max(width, len(order[q]));
    h.ptr[s + 1] = h.ptr[s] + width * C;
  }
  h.idx.assign(h.ptr[h.nsl], pad_index);
  h.slot.assign(h.ptr[h.nsl], -1);
  for (int s = 0; s < h.nsl; ++s) {
    for (int c = 0; c < C; ++c) {
      const int q = s * C + c;
      if (q >= count) continue;
      const int line = order[q];
      for (int k = 0; k < len(line); ++k) {
        const int e = h.ptr[s] + k * C + c;
        const int src = ptr_in[line] + k;
        h.idx[e] = idx_in[src];
        h.slot[e] = slot_in ? (*slot_in)[src] : src;
      }
    }
  }
  return h;
}

// Counting sort of (row, slot) entries by column, stable in row-major order.
void build_csc(int n, const std::vector<int32_t>& row_ptr, const std::vector<int32_t>& col,
               std::vector<int32_t>& col_ptr, std::vector<int32_t>& csc_row,
               std::vector<int32_t>& csc_slot) {
  const int m = (int)row_ptr.size() - 1;
  const int nnz = row_ptr.back();
  col_ptr.assign(n + 1, 0);
  for (int k = 0; k < nnz; ++k) col_ptr[col[k] + 1]++;
  for (int j = 0; j < n; ++j) col_ptr[j + 1] += col_ptr[j];
  std::vector<int32_t> fill(col_ptr.begin(), col_ptr.end() - 1);
  csc_row.assign(nnz, 0);
  csc_slot.assign(nnz, 0);
  for (int i = 0; i < m; ++i) {
    for (int k = row_ptr[i]; k < row_ptr[i + 1]; ++k) {
      const int q = fill[col[k]]++;
      csc_row[q] = i;
      csc_slot[q] = k;
    }
  }
}

int32_t check_adjoint_args(const PurinCpPlan* plan, const PurinCpAdjointArgs* args) {
  const int m = plan->info.kept_rows;
  if (!args->target || !args->lower || !args->upper || !args->y || !args->converged || !args->cot_y ||
      (m > 0 && (!args->rhs || !args->dual)) || (plan->info.kept_nnz > 0 && !args->values))
    return fail(PURIN_ERR_INVALID_ARGUMENT, "a required adjoint array is NULL");
  if (args->values_stride != 0 && args->values_stride != plan->info.kept_nnz)
    return fail(PURIN_ERR_INVALID_ARGUMENT, "values_stride must be 0 or kept_nnz");
  if (args->bounds_stride != 0 && args->bounds_stride != plan->info.n)
    return fail(PURIN_ERR_INVALID_ARGUMENT, "bounds_stride must be 0 or n");
  return PURIN_OK;
}

int32_t create_plan(const PurinCpStructure* s, PurinCpPlan** out, bool presolve_bounds);

// purin_qp_adjoint (stage < 0) and purin_qp_adjoint_stage: the QP arguments on
// the shared adjoint runners.
int32_t qp_adjoint_call(const PurinCpPlan* plan, const PurinCpConfig* config, const PurinLinearSolverConfig* linear,
                        const PurinQpAdjointArgs* args, int32_t stage, int32_t completed, int32_t* counters,
                        void* workspace, size_t workspace_bytes, void* stream) {
  if (int32_t r = check_plan(plan)) return r;
  if (int32_t r = check_config(config)) return r;
  if (int32_t r = check_linear(linear)) return r;
  if (!args) return fail(PURIN_ERR_INVALID_ARGUMENT, "args is NULL");
  if (plan->info.bound_rows != 0)
    return fail(PURIN_ERR_INVALID_ARGUMENT, "purin_qp_adjoint needs a plan from purin_qp_plan_create");
  if (args->batch < 0) return fail(PURIN_ERR_INVALID_ARGUMENT, "batch must be nonnegative");
  if (stage >= 0 && stage != PURIN_CP_STAGE_FINISH && !counters)
    return fail(PURIN_ERR_INVALID_ARGUMENT, "counters is NULL");
  if (stage == PURIN_CP_STAGE_CYCLE && (completed < 0 || completed >= linear->max_iterations))
    return fail(PURIN_ERR_INVALID_ARGUMENT, "completed must lie in [0, max_iterations) for a cycle");
  DeviceGuard guard(plan->info.device);
  if (!guard.ok) return fail(PURIN_ERR_CUDA, "cudaSetDevice failed");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (args->batch == 0) {
    if (stage < 0 || stage == PURIN_CP_STAGE_FINISH) return PURIN_OK;
    cudaError_t e = cudaMemsetAsync(counters, 0, 2 * sizeof(int32_t), s);
    return e == cudaSuccess ? PURIN_OK : cuda_fail(e, "purin_qp_adjoint_stage memset");
  }
  if (!args->q || !args->c) return fail(PURIN_ERR_INVALID_ARGUMENT, "a required QP adjoint array is NULL");
  PurinCpAdjointArgs a{};
  a.batch = args->batch;
  a.values = args->values;
  a.values_stride = args->values_stride;
  a.rhs = args->rhs;
  a.target = args->c;  // satisfies the shared check; the QP kernels read c through QpAdjoint
  a.lower = args->lower;
  a.upper = args->upper;
  a.bounds_stride = args->bounds_stride;
  a.y = args->y;
  a.dual = args->dual;
  a.converged = args->converged;
  a.cot_y = args->cot_y;
  a.sample_offset = args->sample_offset;
  a.total_batch = args->total_batch;
  a.grad_values = args->grad_values;
  a.grad_rhs = args->grad_rhs;
  a.grad_target = nullptr;
  a.grad_lower = args->grad_lower;
  a.grad_upper = args->grad_upper;
  a.linear_status = args->linear_status;
  a.linear_residual = args->linear_residual;
  a.device_error = args->device_error;
  a.arnoldi_steps = args->arnoldi_steps;
  a.krylov_vectors = args->krylov_vectors;
  if (int32_t r = check_adjoint_args(plan, &a)) return r;
  const QpAdjoint qp{args->q, args->c, args->cot_dual, args->grad_q, args->grad_c};
  const bool f64 = plan->info.dtype == PURIN_FLOAT64;
  if (stage < 0)
    return f64 ? run_adjoint<double>(plan, config, linear, &a, workspace, workspace_bytes, s, &qp)
               : run_adjoint<float>(plan, config, linear, &a, workspace, workspace_bytes, s, &qp);
  return f64 ? run_adjoint_stage<double>(plan, config, linear, &a, stage, completed, counters, workspace,
                                         workspace_bytes, s, &qp)
             : run_adjoint_stage<float>(plan, config, linear, &a, stage, completed, counters, workspace,
                                        workspace_bytes, s, &qp);
}

}  // namespace

extern "C" {

int32_t purin_cp_abi_version(void) { return PURIN_CP_ABI_VERSION; }

const char* purin_cp_last_error(void) { return g_last_error.c_str(); }

int32_t purin_cp_plan_create(const PurinCpStructure* s, PurinCpPlan** out) {
  return create_plan(s, out, true);
}

int32_t purin_qp_plan_create(const PurinCpStructure* s, PurinCpPlan** out) {
  return create_plan(s, out, false);
}

}  // extern "C"

namespace {
int32_t create_plan(const PurinCpStructure* s, PurinCpPlan** out, bool presolve_bounds) {
  if (!s || !out) return fail(PURIN_ERR_INVALID_ARGUMENT, "structure and output pointers are required");
  *out = nullptr;
  const int n = s->n, me = s->equality_size, mi = s->inequality_size;
  if (n < 1) return fail(PURIN_ERR_INVALID_ARGUMENT, "batch_size and variable_size must be positive");
  if (me < 0 || mi < 0) return fail(PURIN_ERR_INVALID_ARGUMENT, "constraint row counts must be nonnegative");
  if (s->dtype != PURIN_FLOAT64 && s->dtype != PURIN_FLOAT32)
    return fail(PURIN_ERR_UNSUPPORTED, "dtype must be float64 or float32");
  const int m_all = me + mi;
  if (m_all > 0 && (!s->row_ptr || (s->row_ptr[m_all] > 0 && !s->col)))
    return fail(PURIN_ERR_INVALID_ARGUMENT, "row_ptr/col are required");
  std::vector<int32_t> row_ptr(m_all + 1, 0), col;
  if (m_all > 0) {
    if (s->row_ptr[0] != 0) return fail(PURIN_ERR_INVALID_ARGUMENT, "row_ptr[0] must be 0");
    for (int i = 0; i < m_all; ++i) {
      if (s->row_ptr[i + 1] < s->row_ptr[i]) return fail(PURIN_ERR_INVALID_ARGUMENT, "row_ptr must be nondecreasing");
      row_ptr[i + 1] = s->row_ptr[i + 1];
    }
    col.assign(s->col, s->col + row_ptr[m_all]);
    for (int32_t c : col)
      if (c < 0 || c >= n) return fail(PURIN_ERR_INVALID_ARGUMENT, "column index out of range");
  }
  int device_count = 0;
  if (cudaGetDeviceCount(&device_count) != cudaSuccess || s->device < 0 || s->device >= device_count)
    return fail(PURIN_ERR_CUDA, "CUDA device " + std::to_string(s->device) + " is not available");

  auto* plan = new PurinCpPlan();
  PurinCpPlanInfo& info = plan->info;
  info.n = n;
  info.equality_size = me;
  info.inequality_size = mi;
  info.nnz = row_ptr[m_all];
  info.dtype = s->dtype;
  info.device = s->device;
  int width = 1;
  for (int i = 0; i < m_all; ++i) width = std::max(width, row_ptr[i + 1] - row_ptr[i]);
  info.width = width;

  // prepare_bounds (bounds.py:320-326): singleton inequality rows.  The
  // diagonal QP keeps every row (diagonal_qp.py:88 lays out all rows).
  std::vector<char> is_bound(m_all, 0);
  for (int i = 0; presolve_bounds && i < mi; ++i) {
    const int r = me + i;
    if (row_ptr[r + 1] - row_ptr[r] == 1) {
      is_bound[r] = 1;
      plan->bound_rows.push_back(r);
      plan->bound_slots.push_back(row_ptr[r]);
      plan->bound_vars.push_back(col[row_ptr[r]]);
    }
  }
  // Kept rows (bounds.py:22-32), their CSR and the public-slot map.
  std::vector<int32_t> krow_ptr(1, 0), kcol;
  for (int r = 0; r < m_all; ++r) {
    if (is_bound[r]) continue;
    plan->kept_rows.push_back(r);
    for (int k = row_ptr[r]; k < row_ptr[r + 1]; ++k) {
      kcol.push_back(col[k]);
      plan->kept_slots.push_back(k);
    }
    krow_ptr.push_back((int32_t)kcol.size());
  }
  plan->kept_row_ptr = krow_ptr;
  plan->kept_cols = kcol;
  info.kept_rows = (int)plan->kept_rows.size();
  info.kept_nnz = (int)kcol.size();
  info.bound_rows = (int)plan->bound_rows.size();

  std::vector<int32_t> kcol_ptr, kcsc_row, kcsc_slot, acol_ptr, acsc_row, acsc_slot;
  build_csc(n, krow_ptr, kcol, kcol_ptr, kcsc_row, kcsc_slot);
  build_csc(n, row_ptr, col, acol_ptr, acsc_row, acsc_slot);
  std::vector<int32_t> vb_ptr(n + 1, 0), vb_list(plan->bound_rows.size());
  for (int32_t v : plan->bound_vars) vb_ptr[v + 1]++;
  for (int j = 0; j < n; ++j) vb_ptr[j + 1] += vb_ptr[j];
  {
    std::vector<int32_t> fill(vb_ptr.begin(), vb_ptr.end() - 1);
    for (size_t k = 0; k < plan->bound_vars.size(); ++k) vb_list[fill[plan->bound_vars[k]]++] = (int32_t)k;
  }

  // Pack every index array into one device block.
  std::vector<const std::vector<int32_t>*> arrays = {
      &krow_ptr, &kcol, &kcol_ptr, &kcsc_row, &kcsc_slot, &row_ptr, &col, &acol_ptr, &acsc_row,
      &acsc_slot, &plan->kept_rows, &plan->kept_slots, &plan->bound_rows, &plan->bound_slots,
      &plan->bound_vars, &vb_ptr, &vb_list};
  std::vector<size_t> offsets;
  size_t total = 0;
  for (auto* a : arrays) {
    offsets.push_back(total);
    total += std::max<size_t>(a->size(), 1);
    total = (total + 63) & ~(size_t)63;
  }
  std::vector<int32_t> host(total, 0);
  for (size_t q = 0; q < arrays.size(); ++q)
    if (!arrays[q]->empty()) std::memcpy(host.data() + offsets[q], arrays[q]->data(), arrays[q]->size() * 4);
  {
    DeviceGuard guard(s->device);
    if (!guard.ok) {
      delete plan;
      return fail(PURIN_ERR_CUDA, "cudaSetDevice failed");
    }
    cudaError_t e = cudaMalloc(&plan->device_block, total * sizeof(int32_t));
    if (e == cudaSuccess) e = cudaMemcpy(plan->device_block, host.data(), total * 4, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&plan->sm_count, cudaDevAttrMultiProcessorCount, s->device);
    if (e == cudaSuccess)
      e = cudaDeviceGetAttribute(&plan->max_smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, s->device);
    if (e != cudaSuccess) {
      if (plan->device_block) cudaFree(plan->device_block);
      delete plan;
      return cuda_fail(e, "purin_cp_plan_create");
    }
  }
  const int32_t* d = static_cast<const int32_t*>(plan->device_block);
  purin::DevStructure& st = plan->dev;
  st.n = n;
  st.me = me;
  st.m = info.kept_rows;
  st.nnz = info.kept_nnz;
  st.row_ptr = d + offsets[0];
  st.col = d + offsets[1];
  st.col_ptr = d + offsets[2];
  st.csc_row = d + offsets[3];
  st.csc_slot = d + offsets[4];
  st.m_all = m_all;
  st.nnz_all = info.nnz;
  st.row_ptr_all = d + offsets[5];
  st.col_all = d + offsets[6];
  st.col_ptr_all = d + offsets[7];
  st.csc_row_all = d + offsets[8];
  st.csc_slot_all = d + offsets[9];
  st.kept_rows = d + offsets[10];
  st.kept_slots = d + offsets[11];
  st.n_bound = info.bound_rows;
  st.bound_rows = d + offsets[12];
  st.bound_slot = d + offsets[13];
  st.bound_var = d + offsets[14];
  st.var_bound_ptr = d + offsets[15];
  st.var_bound_list = d + offsets[16];

  // Sliced-ELL layout (C = 32) in the internal row/column orders.
  {
    std::vector<SellHost> layouts;
    size_t total_sell = 0;
    const int C = 32;
    std::vector<int> rorder = length_order(info.kept_rows, krow_ptr);
    std::vector<int> corder = length_order(n, kcol_ptr);
    // PURIN_CP_BANK_ORDER=0 keeps the plain length order (for comparisons).
    const char* bank_env = std::getenv("PURIN_CP_BANK_ORDER");
    if (!(bank_env && std::string(bank_env) == "0")) {
      const int64_t lines = (int64_t)info.kept_rows + n;
      int64_t moves = std::min<int64_t>(200 * lines, 1000000);
      // PURIN_CP_BANK_MOVES overrides the search budget (for comparisons).
      if (const char* env = std::getenv("PURIN_CP_BANK_MOVES")) moves = std::atoll(env);
      // Order for the wide tiles' gathers when the forward will take them: a
      // large structure and room for two samples' state (y, ybar, duals,
      // padded to whole slices) in one CTA's shared memory.
      const size_t w = dtype_size(info.dtype);
      const size_t pair_state =
          2 * (size_t)(2 * (round_up_int(n, 32) + 1) + round_up_int(info.kept_rows, 32) + 1) * w;
      const bool wide = wide_structure(info.kept_nnz, w) &&
                        pair_state + (16u << 10) <= (size_t)plan->max_smem_optin;
      purin::bank_aware_orders(info.kept_rows, n, krow_ptr, kcol, kcol_ptr, kcsc_row, (int)w, wide,
                               moves, rorder, corder);
    }
    SellHost rows_h = build_sell(info.kept_rows, krow_ptr, kcol, nullptr, C, n, rorder);
    SellHost cols_h = build_sell(n, kcol_ptr, kcsc_row, &kcsc_slot, C, info.kept_rows, corder);
    const int m_pos = rows_h.nsl * C, n_pos = cols_h.nsl * C;
    std::vector<int32_t> pos_of_col(n + 1, n_pos), pos_of_row(info.kept_rows + 1, m_pos);
    for (int p = 0; p < n_pos; ++p)
      if (cols_h.perm[p] >= 0) pos_of_col[cols_h.perm[p]] = p;
    for (int q = 0; q < m_pos; ++q)
      if (rows_h.perm[q] >= 0) pos_of_row[rows_h.perm[q]] = q;
    for (auto& v : rows_h.idx) v = pos_of_col[v];  // padding index n -> n_pos
    for (auto& v : cols_h.idx) v = pos_of_row[v];  // padding index m -> m_pos
    // Index pairs (sell.cuh) when every internal position fits in 16 bits.
    const bool idx16 = n_pos + 1 < 65536 && m_pos + 1 < 65536;
    auto pack_pairs = [&](SellHost& h, int pad) {
      h.idx2.assign(idx16 ? h.idx.size() : 0, 0);
      if (!idx16) return;
      for (int sl = 0; sl < h.nsl; ++sl) {
        const int e0 = h.ptr[sl];
        const int width = (h.ptr[sl + 1] - e0) / C;
        for (int k = 0; k < width; k += 2)
          for (int c = 0; c < C; ++c) {
            const uint32_t lo = (uint32_t)h.idx[e0 + k * C + c];
            const uint32_t hi = (uint32_t)(k + 1 < width ? h.idx[e0 + (k + 1) * C + c] : pad);
            h.idx2[e0 + (k / 2) * C + c] = lo | (hi << 16);
          }
      }
    };
    pack_pairs(rows_h, n_pos);
    pack_pairs(cols_h, m_pos);
    layouts.push_back(std::move(rows_h));
    layouts.push_back(std::move(cols_h));
    for (auto& h : layouts) total_sell += h.ptr.size() + h.perm.size() + 3 * h.idx.size() + 80;
    std::vector<int32_t> host_sell(total_sell, 0);
    std::vector<size_t> base;
    size_t at = 0;
    for (auto& h : layouts) {
      base.push_back(at);
      for (auto* v : {&h.ptr, &h.perm, &h.idx, &h.slot}) {
        if (!v->empty()) std::memcpy(host_sell.data() + at, v->data(), v->size() * 4);
        at += v->size() + 16;
      }
      if (!h.idx2.empty()) std::memcpy(host_sell.data() + at, h.idx2.data(), h.idx2.size() * 4);
      at += h.idx2.size() + 16;
    }
    DeviceGuard guard(s->device);
    cudaError_t e = cudaMalloc(&plan->sell_block, std::max<size_t>(at, 1) * sizeof(int32_t));
    if (e == cudaSuccess) e = cudaMemcpy(plan->sell_block, host_sell.data(), at * 4, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
      cudaFree(plan->device_block);
      if (plan->sell_block) cudaFree(plan->sell_block);
      delete plan;
      return cuda_fail(e, "purin_cp_plan_create (sliced ELL)");
    }
    const int32_t* sd = static_cast<const int32_t*>(plan->sell_block);
    {
      const SellHost& r = layouts[0];
      const SellHost& c = layouts[1];
      const int32_t* rb = sd + base[0];
      const int32_t* cb = sd + base[1];
      purin::SellView& v = plan->sell[0];
      v.C = C;
      v.m_pos = m_pos;
      v.n_pos = n_pos;
      v.nsl_r = r.nsl;
      v.nsl_c = c.nsl;
      v.nnz_r = (int)r.idx.size();
      v.nnz_c = (int)c.idx.size();
      v.r_ptr = rb;
      v.r_perm = rb + r.ptr.size() + 16;
      v.r_idx = v.r_perm + r.perm.size() + 16;
      v.r_slot = v.r_idx + r.idx.size() + 16;
      v.c_ptr = cb;
      v.c_perm = cb + c.ptr.size() + 16;
      v.c_idx = v.c_perm + c.perm.size() + 16;
      v.c_slot = v.c_idx + c.idx.size() + 16;
      v.idx16 = idx16 ? 1 : 0;
      v.r_idx2 = reinterpret_cast<const uint32_t*>(v.r_slot + r.slot.size() + 16);
      v.c_idx2 = reinterpret_cast<const uint32_t*>(v.c_slot + c.slot.size() + 16);
    }
  }
  *out = plan;
  return PURIN_OK;
}
}  // namespace

extern "C" {

int32_t purin_cp_plan_destroy(PurinCpPlan* plan) {
  if (!plan) return PURIN_OK;
  if (plan->device_block || plan->sell_block) {
    DeviceGuard guard(plan->info.device);
    if (plan->device_block) cudaFree(plan->device_block);
    if (plan->sell_block) cudaFree(plan->sell_block);
  }
  delete plan;
  return PURIN_OK;
}

int32_t purin_cp_plan_info(const PurinCpPlan* plan, PurinCpPlanInfo* info) {
  if (int32_t r = check_plan(plan)) return r;
  if (!info) return fail(PURIN_ERR_INVALID_ARGUMENT, "info is NULL");
  *info = plan->info;
  return PURIN_OK;
}

int32_t purin_cp_plan_indices(const PurinCpPlan* plan, int32_t which, int32_t* out) {
  if (int32_t r = check_plan(plan)) return r;
  if (!out) return fail(PURIN_ERR_INVALID_ARGUMENT, "out is NULL");
  const std::vector<int32_t>* v = nullptr;
  switch (which) {
    case PURIN_CP_KEPT_ROWS: v = &plan->kept_rows; break;
    case PURIN_CP_KEPT_SLOTS: v = &plan->kept_slots; break;
    case PURIN_CP_BOUND_ROWS: v = &plan->bound_rows; break;
    case PURIN_CP_BOUND_SLOTS: v = &plan->bound_slots; break;
    case PURIN_CP_BOUND_VARIABLES: v = &plan->bound_vars; break;
    case PURIN_CP_KEPT_ROW_PTR: v = &plan->kept_row_ptr; break;
    case PURIN_CP_KEPT_COLS: v = &plan->kept_cols; break;
    default: return fail(PURIN_ERR_INVALID_ARGUMENT, "unknown index array");
  }
  if (!v->empty()) std::memcpy(out, v->data(), v->size() * sizeof(int32_t));
  return PURIN_OK;
}

int32_t purin_cp_workspace_size(const PurinCpPlan* plan, int32_t op, int64_t batch,
                                const PurinCpConfig* config, const PurinLinearSolverConfig* linear,
                                size_t* bytes) {
  if (int32_t r = check_plan(plan)) return r;
  if (!bytes) return fail(PURIN_ERR_INVALID_ARGUMENT, "bytes is NULL");
  if (int32_t r = check_config(config)) return r;
  if (batch < 0) return fail(PURIN_ERR_INVALID_ARGUMENT, "batch must be nonnegative");
  *bytes = 0;
  if (batch == 0) return PURIN_OK;
  DeviceGuard guard(plan->info.device);
  if (op == PURIN_CP_OP_FORWARD) {
    *bytes = plan_forward(plan, config, batch).workspace;
    return PURIN_OK;
  }
  if (op == PURIN_QP_OP_FORWARD) {
    *bytes = plan_forward(plan, config, batch, true, true).workspace;
    return PURIN_OK;
  }
  if (op == PURIN_CP_OP_FORWARD_SAMPLE_VALUES || op == PURIN_QP_OP_FORWARD_SAMPLE_VALUES) {
    *bytes = plan_forward(plan, config, batch, batch == 1, op == PURIN_QP_OP_FORWARD_SAMPLE_VALUES).workspace;
    return PURIN_OK;
  }
  if (op == PURIN_CP_OP_ADJOINT || op == PURIN_QP_OP_ADJOINT) {
    if (int32_t r = check_linear(linear)) return r;
    // The call's choice between the cluster and streaming GMRES kernels depends
    // on the global batch, which this query does not know: size for the
    // streaming kernel, whose layout holds every region the other uses.
    const AdjLayout L = plan_adjoint(plan, config, linear, batch, op == PURIN_QP_OP_ADJOINT,
                                     INT64_MAX / 2);
    if (L.grid < 1) return fail(PURIN_ERR_UNSUPPORTED, "adjoint kernel cannot be made resident on this device");
    *bytes = L.total;
    return PURIN_OK;
  }
  return fail(PURIN_ERR_INVALID_ARGUMENT, "unknown op");
}

int32_t purin_cp_forward_shape(const PurinCpPlan* plan, const PurinCpConfig* config, int64_t batch,
                               int32_t shared_values, int32_t* samples_per_tile, int32_t* threads,
                               int32_t* shared_state) {
  if (int32_t r = check_plan(plan)) return r;
  if (int32_t r = check_config(config)) return r;
  if (!samples_per_tile || !threads || !shared_state)
    return fail(PURIN_ERR_INVALID_ARGUMENT, "an output pointer is NULL");
  if (batch < 1) return fail(PURIN_ERR_INVALID_ARGUMENT, "batch must be positive");
  DeviceGuard guard(plan->info.device);
  // As purin_cp_forward plans it: a single sample counts as shared values.
  const FwdPlan fp = plan_forward(plan, config, batch, shared_values != 0 || batch == 1);
  *samples_per_tile = fp.S;
  *threads = fp.NT;
  *shared_state = fp.smem ? 1 : 0;
  return PURIN_OK;
}

int32_t purin_cp_forward(const PurinCpPlan* plan, const PurinCpConfig* config, const PurinCpForwardArgs* args,
                         void* workspace, size_t workspace_bytes, void* stream) {
  if (int32_t r = check_plan(plan)) return r;
  if (int32_t r = check_config(config)) return r;
  if (!args) return fail(PURIN_ERR_INVALID_ARGUMENT, "args is NULL");
  if (args->batch < 0) return fail(PURIN_ERR_INVALID_ARGUMENT, "batch must be nonnegative");
  if (args->batch == 0) return PURIN_OK;
  const int m = plan->info.kept_rows;
  if (!args->target || !args->tolerance || !args->lower || !args->upper || !args->y || !args->iterations ||
      !args->residual || !args->gap || !args->converged || (m > 0 && (!args->rhs || !args->dual)) ||
      (plan->info.kept_nnz > 0 && !args->values))
    return fail(PURIN_ERR_INVALID_ARGUMENT, "a required forward array is NULL");
  if (args->values_stride != 0 && args->values_stride != plan->info.kept_nnz)
    return fail(PURIN_ERR_INVALID_ARGUMENT, "values_stride must be 0 or kept_nnz");
  if (args->bounds_stride != 0 && args->bounds_stride != plan->info.n)
    return fail(PURIN_ERR_INVALID_ARGUMENT, "bounds_stride must be 0 or n");
  DeviceGuard guard(plan->info.device);
  if (!guard.ok) return fail(PURIN_ERR_CUDA, "cudaSetDevice failed");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return plan->info.dtype == PURIN_FLOAT64 ? run_forward<double>(plan, config, args, workspace, workspace_bytes, s)
                                           : run_forward<float>(plan, config, args, workspace, workspace_bytes, s);
}


int32_t purin_cp_adjoint_stage(const PurinCpPlan* plan, const PurinCpConfig* config,
                               const PurinLinearSolverConfig* linear, const PurinCpAdjointArgs* args,
                               int32_t stage, int32_t completed, int32_t* counters, void* workspace,
                               size_t workspace_bytes, void* stream) {
  if (int32_t r = check_plan(plan)) return r;
  if (int32_t r = check_config(config)) return r;
  if (int32_t r = check_linear(linear)) return r;
  if (!args) return fail(PURIN_ERR_INVALID_ARGUMENT, "args is NULL");
  if (args->batch < 0) return fail(PURIN_ERR_INVALID_ARGUMENT, "batch must be nonnegative");
  if (stage != PURIN_CP_STAGE_PREPARE && stage != PURIN_CP_STAGE_CYCLE && stage != PURIN_CP_STAGE_FINISH)
    return fail(PURIN_ERR_INVALID_ARGUMENT, "unknown adjoint stage");
  if (stage != PURIN_CP_STAGE_FINISH && !counters)
    return fail(PURIN_ERR_INVALID_ARGUMENT, "counters is NULL");
  if (stage == PURIN_CP_STAGE_CYCLE && (completed < 0 || completed >= linear->max_iterations))
    return fail(PURIN_ERR_INVALID_ARGUMENT, "completed must lie in [0, max_iterations) for a cycle");
  DeviceGuard guard(plan->info.device);
  if (!guard.ok) return fail(PURIN_ERR_CUDA, "cudaSetDevice failed");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (args->batch == 0) {
    // An empty shard still takes part in the exchange: it reports zeros.
    if (stage == PURIN_CP_STAGE_FINISH) return PURIN_OK;
    cudaError_t e = cudaMemsetAsync(counters, 0, 2 * sizeof(int32_t), s);
    return e == cudaSuccess ? PURIN_OK : cuda_fail(e, "purin_cp_adjoint_stage memset");
  }
  if (int32_t r = check_adjoint_args(plan, args)) return r;
  return plan->info.dtype == PURIN_FLOAT64
             ? run_adjoint_stage<double>(plan, config, linear, args, stage, completed, counters, workspace,
                                         workspace_bytes, s)
             : run_adjoint_stage<float>(plan, config, linear, args, stage, completed, counters, workspace,
                                        workspace_bytes, s);
}

int32_t purin_cp_adjoint(const PurinCpPlan* plan, const PurinCpConfig* config, const PurinLinearSolverConfig* linear,
                         const PurinCpAdjointArgs* args, void* workspace, size_t workspace_bytes, void* stream) {
  if (int32_t r = check_plan(plan)) return r;
  if (int32_t r = check_config(config)) return r;
  if (int32_t r = check_linear(linear)) return r;
  if (!args) return fail(PURIN_ERR_INVALID_ARGUMENT, "args is NULL");
  if (args->batch < 0) return fail(PURIN_ERR_INVALID_ARGUMENT, "batch must be nonnegative");
  if (args->batch == 0) return PURIN_OK;
  if (int32_t r = check_adjoint_args(plan, args)) return r;
  DeviceGuard guard(plan->info.device);
  if (!guard.ok) return fail(PURIN_ERR_CUDA, "cudaSetDevice failed");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return plan->info.dtype == PURIN_FLOAT64
             ? run_adjoint<double>(plan, config, linear, args, workspace, workspace_bytes, s)
             : run_adjoint<float>(plan, config, linear, args, workspace, workspace_bytes, s);
}

int32_t purin_qp_forward(const PurinCpPlan* plan, const PurinCpConfig* config, const PurinQpForwardArgs* args,
                         void* workspace, size_t workspace_bytes, void* stream) {
  if (int32_t r = check_plan(plan)) return r;
  if (int32_t r = check_config(config)) return r;
  if (!args) return fail(PURIN_ERR_INVALID_ARGUMENT, "args is NULL");
  if (plan->info.bound_rows != 0)
    return fail(PURIN_ERR_INVALID_ARGUMENT, "purin_qp_forward needs a plan from purin_qp_plan_create");
  if (args->batch < 0) return fail(PURIN_ERR_INVALID_ARGUMENT, "batch must be nonnegative");
  if (args->batch == 0) return PURIN_OK;
  const int m = plan->info.kept_rows;
  if (!args->q || !args->c || !args->tolerance || !args->lower || !args->upper || !args->y ||
      !args->iterations || !args->residual || !args->gap || !args->converged ||
      (m > 0 && (!args->rhs || !args->dual)) || (plan->info.kept_nnz > 0 && !args->values))
    return fail(PURIN_ERR_INVALID_ARGUMENT, "a required QP forward array is NULL");
  if (args->values_stride != 0 && args->values_stride != plan->info.kept_nnz)
    return fail(PURIN_ERR_INVALID_ARGUMENT, "values_stride must be 0 or nnz");
  if (args->bounds_stride != 0 && args->bounds_stride != plan->info.n)
    return fail(PURIN_ERR_INVALID_ARGUMENT, "bounds_stride must be 0 or n");
  PurinCpForwardArgs a{};
  a.batch = args->batch;
  a.values = args->values;
  a.values_stride = args->values_stride;
  a.rhs = args->rhs;
  a.target = nullptr;
  a.dual0 = args->dual0;
  a.tolerance = args->tolerance;
  a.lower = args->lower;
  a.upper = args->upper;
  a.bounds_stride = args->bounds_stride;
  a.feasible = nullptr;
  a.sample_offset = args->sample_offset;
  a.total_batch = args->total_batch;
  a.y = args->y;
  a.dual = args->dual;
  a.iterations = args->iterations;
  a.residual = args->residual;
  a.gap = args->gap;
  a.converged = args->converged;
  if (args->flags & ~(PURIN_QP_FACTORED_PROXIMAL | PURIN_QP_NO_STATIONARITY | PURIN_QP_NO_FREEZE |
                      PURIN_QP_NO_VALIDITY))
    return fail(PURIN_ERR_INVALID_ARGUMENT, "unknown purin_qp_forward flags");
  if ((args->ybar0 || args->start_iterations) && !args->y0)
    return fail(PURIN_ERR_INVALID_ARGUMENT, "resuming a QP solve (ybar0, start_iterations) needs y0");
  const QpInputs qp{args->q,     args->c,
                    args->y0,    args->flags,
                    args->ybar0, args->start_iterations,
                    args->ybar};
  DeviceGuard guard(plan->info.device);
  if (!guard.ok) return fail(PURIN_ERR_CUDA, "cudaSetDevice failed");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return plan->info.dtype == PURIN_FLOAT64
             ? run_forward<double>(plan, config, &a, workspace, workspace_bytes, s, &qp)
             : run_forward<float>(plan, config, &a, workspace, workspace_bytes, s, &qp);
}

int32_t purin_qp_adjoint(const PurinCpPlan* plan, const PurinCpConfig* config, const PurinLinearSolverConfig* linear,
                         const PurinQpAdjointArgs* args, void* workspace, size_t workspace_bytes, void* stream) {
  return qp_adjoint_call(plan, config, linear, args, -1, 0, nullptr, workspace, workspace_bytes, stream);
}

int32_t purin_qp_adjoint_stage(const PurinCpPlan* plan, const PurinCpConfig* config,
                               const PurinLinearSolverConfig* linear, const PurinQpAdjointArgs* args,
                               int32_t stage, int32_t completed, int32_t* counters, void* workspace,
                               size_t workspace_bytes, void* stream) {
  if (stage != PURIN_CP_STAGE_PREPARE && stage != PURIN_CP_STAGE_CYCLE && stage != PURIN_CP_STAGE_FINISH)
    return fail(PURIN_ERR_INVALID_ARGUMENT, "unknown adjoint stage");
  return qp_adjoint_call(plan, config, linear, args, stage, completed, counters, workspace, workspace_bytes,
                         stream);
}

}  // extern "C"

namespace {

// ADMM forward workspace: the band factor (when a band is given), then the
// per-sample vectors of problems too large for shared memory.
struct AdmmLayout {
  bool smem = true;
  size_t off_band = 0, off_state = 0, total = 0;
};

AdmmLayout plan_admm(const PurinCpPlan* plan, int64_t batch, int32_t width) {
  AdmmLayout L;
  const int n = plan->info.n, m = plan->info.kept_rows;
  const size_t w = dtype_size(plan->info.dtype);
  const size_t state = (plan->info.dtype == PURIN_FLOAT64 ? purin::admm_state_elems<double>(n, m)
                                                          : purin::admm_state_elems<float>(n, m)) * w;
  L.smem = state + 1024 <= (size_t)plan->max_smem_optin;
  const size_t nb = (size_t)std::max<int64_t>(batch, 0);
  L.off_band = 0;
  L.off_state = align_up(width >= 0 ? nb * n * (size_t)(width + 1) * w : 0);
  L.total = L.off_state + (L.smem ? 0 : align_up(nb * state));
  return L;
}

// A CP-config stand-in for the adjoint runners (ADMM's VJP has no CP steps).
PurinCpConfig admm_cp_config() {
  PurinCpConfig c{};
  c.max_iterations = 1;
  c.safety = 0.5;
  c.norm_iterations = 1;
  c.norm_bound = 1;
  return c;
}

template <typename T>
int32_t run_admm(const PurinCpPlan* plan, const PurinAdmmConfig* cfg, const PurinAdmmForwardArgs* a,
                 void* workspace, size_t workspace_bytes, cudaStream_t stream) {
  const AdmmLayout L = plan_admm(plan, a->batch, a->band.width);
  if (L.total > 0 && (workspace == nullptr || workspace_bytes < L.total))
    return fail(PURIN_ERR_WORKSPACE, "ADMM workspace too small: need " + std::to_string(L.total) + " bytes");
  char* ws = static_cast<char*>(workspace);
  purin::AdmmParams<T> p{};
  p.st = plan->dev;
  p.batch = a->batch;
  p.q = static_cast<const T*>(a->q);
  p.c = static_cast<const T*>(a->c);
  p.values = static_cast<const T*>(a->values);
  p.values_stride = a->values_stride;
  p.lower = static_cast<const T*>(a->lower);
  p.upper = static_cast<const T*>(a->upper);
  p.penalty0 = static_cast<const T*>(a->penalty);
  p.tolerance = static_cast<const T*>(a->tolerance);
  p.x0 = static_cast<const T*>(a->x0);
  p.dual0 = static_cast<const T*>(a->dual0);
  p.x = static_cast<T*>(a->x);
  p.z = static_cast<T*>(a->z);
  p.dual = static_cast<T*>(a->dual);
  p.penalty = static_cast<T*>(a->penalty_out);
  p.iterations = a->iterations;
  p.inner_iterations = a->inner_iterations;
  p.primal_residual = static_cast<T*>(a->primal_residual);
  p.dual_residual = static_cast<T*>(a->dual_residual);
  p.linear_residual = static_cast<T*>(a->linear_residual);
  p.converged = a->converged;
  p.finite = a->finite;
  p.sigma = (T)cfg->sigma;
  p.alpha = (T)cfg->alpha;
  p.max_iterations = cfg->max_iterations;
  p.cg_iterations = cfg->cg_max_iterations;
  p.refinement_steps = cfg->cg_refinement_steps;
  p.check_interval = cfg->check_interval;
  p.cg_tolerance = (T)cfg->cg_tolerance;
  p.adaptive_rho = cfg->adaptive_rho ? 1 : 0;
  p.rho_update_interval = cfg->rho_update_interval;
  p.rho_update_threshold = (T)cfg->rho_update_threshold;
  p.width = a->band.width;
  p.nband = a->band.entries;
  p.band_perm = a->band.permutation;
  p.band_inv = a->band.inverse;
  p.band_rows = a->band.rows;
  p.band_slot_l = a->band.slot_left;
  p.band_slot_r = a->band.slot_right;
  p.band_dest = a->band.destination;
  p.band = a->band.width >= 0 ? reinterpret_cast<T*>(ws + L.off_band) : nullptr;
  p.gstate = L.smem ? nullptr : reinterpret_cast<T*>(ws + L.off_state);
  cudaError_t e = purin::launch_admm<T>(p, L.smem, stream);
  if (e != cudaSuccess) return cuda_fail(e, "purin_admm_forward launch");
  return PURIN_OK;
}

int32_t check_admm_plan(const PurinCpPlan* plan) {
  if (int32_t r = check_plan(plan)) return r;
  if (plan->info.bound_rows != 0)
    return fail(PURIN_ERR_INVALID_ARGUMENT, "ADMM needs a plan from purin_qp_plan_create");
  return PURIN_OK;
}

// ADMM adjoint arguments on the shared runners (stage < 0: fused).
int32_t admm_adjoint_call(const PurinCpPlan* plan, const PurinLinearSolverConfig* linear,
                          const PurinAdmmAdjointArgs* args, int32_t stage, int32_t completed,
                          int32_t* counters, void* workspace, size_t workspace_bytes, void* stream) {
  if (int32_t r = check_admm_plan(plan)) return r;
  if (int32_t r = check_linear(linear)) return r;
  if (!args) return fail(PURIN_ERR_INVALID_ARGUMENT, "args is NULL");
  if (args->batch < 0) return fail(PURIN_ERR_INVALID_ARGUMENT, "batch must be nonnegative");
  if (stage >= 0 && stage != PURIN_CP_STAGE_FINISH && !counters)
    return fail(PURIN_ERR_INVALID_ARGUMENT, "counters is NULL");
  if (stage == PURIN_CP_STAGE_CYCLE && (completed < 0 || completed >= linear->max_iterations))
    return fail(PURIN_ERR_INVALID_ARGUMENT, "completed must lie in [0, max_iterations) for a cycle");
  DeviceGuard guard(plan->info.device);
  if (!guard.ok) return fail(PURIN_ERR_CUDA, "cudaSetDevice failed");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (args->batch == 0) {
    if (stage < 0 || stage == PURIN_CP_STAGE_FINISH) return PURIN_OK;
    cudaError_t e = cudaMemsetAsync(counters, 0, 2 * sizeof(int32_t), s);
    return e == cudaSuccess ? PURIN_OK : cuda_fail(e, "purin_admm_adjoint_stage memset");
  }
  const int m = plan->info.kept_rows;
  if (!args->y || !args->converged || !args->cot_y || (m > 0 && (!args->rhs || !args->dual)) ||
      (plan->info.kept_nnz > 0 && !args->values))
    return fail(PURIN_ERR_INVALID_ARGUMENT, "a required ADMM adjoint array is NULL");
  PurinCpAdjointArgs a{};
  a.batch = args->batch;
  a.values = args->values;
  a.values_stride = args->values_stride;
  a.rhs = args->rhs;
  // The CP fields ADMM does not read point at valid arrays of the right size.
  a.target = args->cot_y;
  a.lower = args->y;
  a.upper = args->y;
  a.bounds_stride = plan->info.n;
  a.y = args->y;
  a.dual = args->dual;
  a.converged = args->converged;
  a.cot_y = args->cot_y;
  a.sample_offset = args->sample_offset;
  a.total_batch = args->total_batch;
  a.grad_values = args->grad_values;
  a.grad_rhs = args->grad_rhs;
  a.grad_target = args->grad_target;
  a.linear_status = args->linear_status;
  a.linear_residual = args->linear_residual;
  a.device_error = args->device_error;
  if (int32_t r = check_adjoint_args(plan, &a)) return r;
  const AdmmAdjoint admm{args->active_tolerance, args->tolerance};
  const PurinCpConfig cfg = admm_cp_config();
  const bool f64 = plan->info.dtype == PURIN_FLOAT64;
  if (stage < 0)
    return f64 ? run_adjoint<double>(plan, &cfg, linear, &a, workspace, workspace_bytes, s, nullptr, &admm)
               : run_adjoint<float>(plan, &cfg, linear, &a, workspace, workspace_bytes, s, nullptr, &admm);
  return f64 ? run_adjoint_stage<double>(plan, &cfg, linear, &a, stage, completed, counters, workspace,
                                         workspace_bytes, s, nullptr, &admm)
             : run_adjoint_stage<float>(plan, &cfg, linear, &a, stage, completed, counters, workspace,
                                        workspace_bytes, s, nullptr, &admm);
}

}  // namespace

extern "C" {

int32_t purin_admm_workspace_size(const PurinCpPlan* plan, int64_t batch, int32_t band_width,
                                  size_t* bytes) {
  if (int32_t r = check_admm_plan(plan)) return r;
  if (!bytes) return fail(PURIN_ERR_INVALID_ARGUMENT, "bytes is NULL");
  if (batch < 0) return fail(PURIN_ERR_INVALID_ARGUMENT, "batch must be nonnegative");
  *bytes = batch == 0 ? 0 : plan_admm(plan, batch, band_width).total;
  return PURIN_OK;
}

int32_t purin_admm_forward(const PurinCpPlan* plan, const PurinAdmmConfig* config,
                           const PurinAdmmForwardArgs* args, void* workspace, size_t workspace_bytes,
                           void* stream) {
  if (int32_t r = check_admm_plan(plan)) return r;
  if (!config || !args) return fail(PURIN_ERR_INVALID_ARGUMENT, "config and args are required");
  if (config->max_iterations < 1 || config->cg_max_iterations < 1 || config->cg_refinement_steps < 1 ||
      config->check_interval < 1 || config->rho_update_interval < 1)
    return fail(PURIN_ERR_INVALID_ARGUMENT, "ADMM iteration counts must be positive integers");
  if (!(config->alpha > 0.0 && config->alpha < 2.0))
    return fail(PURIN_ERR_INVALID_ARGUMENT, "alpha must be between zero and two");
  if (args->batch < 0) return fail(PURIN_ERR_INVALID_ARGUMENT, "batch must be nonnegative");
  if (args->batch == 0) return PURIN_OK;
  const int m = plan->info.kept_rows;
  if (!args->q || !args->c || !args->tolerance || !args->x0 || !args->x || !args->iterations ||
      !args->inner_iterations || !args->primal_residual || !args->dual_residual ||
      !args->linear_residual || !args->converged || !args->finite ||
      (m > 0 && (!args->lower || !args->upper || !args->penalty || !args->z || !args->dual ||
                 !args->penalty_out)) ||
      (plan->info.kept_nnz > 0 && !args->values))
    return fail(PURIN_ERR_INVALID_ARGUMENT, "a required ADMM forward array is NULL");
  if (args->values_stride != 0 && args->values_stride != plan->info.kept_nnz)
    return fail(PURIN_ERR_INVALID_ARGUMENT, "values_stride must be 0 or nnz");
  if (args->band.width > 8)
    return fail(PURIN_ERR_INVALID_ARGUMENT, "the banded factor is used for widths up to 8");
  if (args->band.width >= 0 && (!args->band.permutation || !args->band.inverse ||
                                (args->band.entries > 0 && (!args->band.rows || !args->band.slot_left ||
                                                            !args->band.slot_right ||
                                                            !args->band.destination))))
    return fail(PURIN_ERR_INVALID_ARGUMENT, "a banded-factor array is NULL");
  DeviceGuard guard(plan->info.device);
  if (!guard.ok) return fail(PURIN_ERR_CUDA, "cudaSetDevice failed");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return plan->info.dtype == PURIN_FLOAT64 ? run_admm<double>(plan, config, args, workspace, workspace_bytes, s)
                                           : run_admm<float>(plan, config, args, workspace, workspace_bytes, s);
}

int32_t purin_admm_adjoint_workspace_size(const PurinCpPlan* plan, int64_t batch,
                                          const PurinLinearSolverConfig* linear, size_t* bytes) {
  if (int32_t r = check_admm_plan(plan)) return r;
  if (int32_t r = check_linear(linear)) return r;
  if (!bytes) return fail(PURIN_ERR_INVALID_ARGUMENT, "bytes is NULL");
  if (batch < 0) return fail(PURIN_ERR_INVALID_ARGUMENT, "batch must be nonnegative");
  *bytes = 0;
  if (batch == 0) return PURIN_OK;
  DeviceGuard guard(plan->info.device);
  const PurinCpConfig cfg = admm_cp_config();
  const AdjLayout L = plan_adjoint(plan, &cfg, linear, batch, false, 0, true);
  if (L.grid < 1) return fail(PURIN_ERR_UNSUPPORTED, "adjoint kernel cannot be made resident on this device");
  *bytes = L.total;
  return PURIN_OK;
}

int32_t purin_admm_adjoint(const PurinCpPlan* plan, const PurinLinearSolverConfig* linear,
                           const PurinAdmmAdjointArgs* args, void* workspace, size_t workspace_bytes,
                           void* stream) {
  return admm_adjoint_call(plan, linear, args, -1, 0, nullptr, workspace, workspace_bytes, stream);
}

int32_t purin_admm_adjoint_stage(const PurinCpPlan* plan, const PurinLinearSolverConfig* linear,
                                 const PurinAdmmAdjointArgs* args, int32_t stage, int32_t completed,
                                 int32_t* counters, void* workspace, size_t workspace_bytes, void* stream) {
  if (stage != PURIN_CP_STAGE_PREPARE && stage != PURIN_CP_STAGE_CYCLE && stage != PURIN_CP_STAGE_FINISH)
    return fail(PURIN_ERR_INVALID_ARGUMENT, "unknown adjoint stage");
  return admm_adjoint_call(plan, linear, args, stage, completed, counters, workspace, workspace_bytes,
                           stream);
}

int32_t purin_cp_postprocess(const PurinCpPlan* plan, const PurinCpPostArgs* args, void* stream) {
  if (int32_t r = check_plan(plan)) return r;
  if (!args) return fail(PURIN_ERR_INVALID_ARGUMENT, "args is NULL");
  if (args->batch < 0) return fail(PURIN_ERR_INVALID_ARGUMENT, "batch must be nonnegative");
  if (args->batch == 0) return PURIN_OK;
  const int me = plan->info.equality_size, mi = plan->info.inequality_size, m = plan->info.kept_rows;
  if (!args->target || !args->lower || !args->upper || !args->y || !args->gap || !args->cp_converged ||
      !args->status || !args->residual_inf_norm || !args->finite || !args->gradient_eligible ||
      (me > 0 && !args->multipliers_eq) || (mi > 0 && (!args->multipliers_ineq || !args->slacks)) ||
      (m > 0 && (!args->dual || !args->scale)) || (me + mi > 0 && !args->rhs_all) ||
      (plan->info.nnz > 0 && !args->values_all))
    return fail(PURIN_ERR_INVALID_ARGUMENT, "a required postprocess array is NULL");
  if (args->values_all_stride != 0 && args->values_all_stride != plan->info.nnz)
    return fail(PURIN_ERR_INVALID_ARGUMENT, "values_all_stride must be 0 or nnz");
  if (args->bounds_stride != 0 && args->bounds_stride != plan->info.n)
    return fail(PURIN_ERR_INVALID_ARGUMENT, "bounds_stride must be 0 or n");
  DeviceGuard guard(plan->info.device);
  if (!guard.ok) return fail(PURIN_ERR_CUDA, "cudaSetDevice failed");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return plan->info.dtype == PURIN_FLOAT64 ? run_post<double>(plan, args, s) : run_post<float>(plan, args, s);
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Forward solve without caller-provided scratch.
//
// Some callers cannot allocate device memory on their own: a plugin or custom-
// call hook that is handed only its input and output buffers, a host framework
// that has already reserved nearly all device memory for its own allocator, or
// a latency-critical loop that forbids allocation.  For them the scratch that
// purin_cp_forward takes from the caller (the batch-shared constraint values
// in sliced-ELL order and, for problems too large for shared memory, the tile
// state) lives in one fixed file-scope device array instead.
namespace {

constexpr size_t kNoAllocScratchBytes = PURIN_CP_NOALLOC_SCRATCH_BYTES;
constexpr int kNoAllocMaxDevices = 128;

// One copy per device that loads this library, held until the process exits.
// Host code must not use this name as an address: it only stands in for the
// device array, so the device address is looked up once per device below.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_noalloc_mutex;
void* g_noalloc_address[kNoAllocMaxDevices] = {};

}  // namespace

extern "C" int32_t purin_cp_forward_noalloc(const PurinCpPlan* plan, const PurinCpConfig* config,
                                            const PurinCpForwardArgs* args, void* stream) {
  if (int32_t r = check_plan(plan)) return r;
  if (int32_t r = check_config(config)) return r;
  if (!args) return fail(PURIN_ERR_INVALID_ARGUMENT, "args is NULL");
  if (args->batch <= 0) return purin_cp_forward(plan, config, args, nullptr, 0, stream);
  const int device = plan->info.device;
  if (device < 0 || device >= kNoAllocMaxDevices)
    return fail(PURIN_ERR_UNSUPPORTED, "purin_cp_forward_noalloc supports device ordinals below 128");
  // The tile planner queries kernel attributes and occupancy, and the symbol
  // lookup below resolves the array, on the CURRENT device: make it the plan's
  // before either, so no other GPU gets a context (and a copy of the array).
  DeviceGuard guard(device);
  if (!guard.ok) return fail(PURIN_ERR_CUDA, "cudaSetDevice failed");
  const bool shared = args->values_stride == 0 || args->batch == 1 || plan->info.kept_nnz == 0;
  const size_t need = plan_forward(plan, config, args->batch, shared).workspace;
  if (need > kNoAllocScratchBytes)
    return fail(PURIN_ERR_WORKSPACE,
                "purin_cp_forward_noalloc needs " + std::to_string(need) +
                    " bytes of scratch but its fixed device array holds " +
                    std::to_string(kNoAllocScratchBytes) +
                    " bytes; use purin_cp_forward with a caller-provided workspace");
  void* scratch = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_noalloc_mutex);
    scratch = g_noalloc_address[device];
    if (scratch == nullptr) {
      cudaError_t e = cudaGetSymbolAddress(&scratch, g_noalloc_scratch);
      if (e != cudaSuccess) return cuda_fail(e, "purin_cp_forward_noalloc cudaGetSymbolAddress");
      g_noalloc_address[device] = scratch;
    }
  }
  // Every part of the scratch this solve reads is written earlier in the same
  // solve, so nothing has to be cleared between calls.
  return purin_cp_forward(plan, config, args, scratch, kNoAllocScratchBytes, stream);
}
