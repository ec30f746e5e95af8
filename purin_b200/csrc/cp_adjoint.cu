// Implicit-differentiation VJP of the CP projection: the custom-VJP backward of
// src/purin/solvers/chambolle_pock/bounds.py:80-165 (solver.py:186-272 without
// bounds).
//
//   1. step sizes tau = s/(1+L), sigma = s/L with L from the seeded power
//      iteration (bounds.py:87-101, kernels.py:52-65), or the diagonal steps
//      (kernels.py:76-88) for fixed-step diagonal preconditioning;
//   2. the linearisation of one fixed-step CP update at the forward solution
//      (bounds.py:109-129), stored as lambda+ and per-element derivative codes
//      of the clip / max operations (JAX's tie rule: half to each argument);
//   3. restarted GMRES (primal_dual_interior_point/operators.py:792-1125) on
//      (I - J^T) v = g with g = (cot_y masked by convergence, 0, 0);
//   4. validity masking and the parameter pullback (bounds.py:148-165).
//
// The whole computation is ONE cooperative persistent kernel.  Samples are
// assigned to CTAs statically (X = blockIdx.x + k * gridDim.x); a CTA keeps the
// current Krylov vector and the pullback temporaries of its sample in shared
// memory and its Krylov basis in a per-CTA global slot, so the basis workspace
// scales with the number of resident CTAs, not with the batch.  GMRES cycles
// run in lockstep across the batch, exactly like the reference's batched
// while-loops: a bounded grid barrier after every cycle publishes the cycle
// length (the largest number of Arnoldi steps any sample took) and the count
// of samples still above their threshold, which set the shared iteration
// budget and the loop condition (operators.py:919-1103).
//
// Staged mode runs the same code one phase per launch (p.stage 1: step sizes,
// linearisation and initial residuals; 2: one GMRES cycle; 3: validity and
// pullback) and reports the cycle's counters in two words, so that a host
// holding one shard of a batch can combine them with the other shards' (an
// elementwise max) before the next cycle: the shards then share the
// reference's batch-wide budget exactly.  State between launches lives in the
// workspace (x, thresholds, residuals, linearisation codes).
#include <cuda_runtime.h>

#include <cstdlib>

#include "adjoint_common.cuh"

namespace purin {

namespace {

// Dot products of buf with basis rows [0, r) into out[0, r) (CGS pass, first half).
template <typename T>
__device__ void basis_dots(const T* V, int W, const T* buf, int r, T* out, T* red) {
  for (int c0 = 0; c0 < r; c0 += kChunk) {
    T part[kChunk];
#pragma unroll
    for (int q = 0; q < kChunk; ++q) part[q] = T(0);
#pragma unroll 2
    for (int e = threadIdx.x; e < W; e += (int)blockDim.x) {
      const T be = buf[e];
      T v[kChunk];
#pragma unroll
      for (int q = 0; q < kChunk; ++q) v[q] = (c0 + q < r) ? V[(size_t)(c0 + q) * W + e] : T(0);
#pragma unroll
      for (int q = 0; q < kChunk; ++q)
        if (c0 + q < r) part[q] = part[q] + v[q] * be;
    }
#pragma unroll
    for (int q = 0; q < kChunk; ++q) part[q] = warp_sum(part[q]);
    __syncthreads();
    if ((threadIdx.x & 31) == 0) {
#pragma unroll
      for (int q = 0; q < kChunk; ++q) red[(threadIdx.x >> 5) * kChunk + q] = part[q];
    }
    __syncthreads();
    if (threadIdx.x < kChunk && c0 + (int)threadIdx.x < r) {
      T total = T(0);
      for (int w = 0; w < (int)(blockDim.x >> 5); ++w) total = total + red[w * kChunk + threadIdx.x];
      out[c0 + threadIdx.x] = total;
    }
    __syncthreads();
  }
}

// sum_i c[i] V[i][e] over rows [0, r), accumulated in row order; the basis
// values are loaded kChunk at a time so the loads are independent.
template <typename T>
__device__ __forceinline__ T basis_combination(const T* V, int W, int e, int r, const T* c) {
  T acc = T(0);
  for (int c0 = 0; c0 < r; c0 += kChunk) {
    T v[kChunk];
#pragma unroll
    for (int q = 0; q < kChunk; ++q) v[q] = (c0 + q < r) ? V[(size_t)(c0 + q) * W + e] : T(0);
#pragma unroll
    for (int q = 0; q < kChunk; ++q)
      if (c0 + q < r) acc = acc + c[c0 + q] * v[q];
  }
  return acc;
}

// buf <- buf - sum_i c[i] V[i] over rows [0, r) (CGS pass, second half).
template <typename T>
__device__ void basis_update(const T* V, int W, T* buf, int r, const T* c) {
#pragma unroll 2
  for (int e = threadIdx.x; e < W; e += (int)blockDim.x) buf[e] = buf[e] - basis_combination(V, W, e, r, c);
  __syncthreads();
}

// Diagonal-QP backward steps (diagonal_qp.py:149-150): tau = s/(max q + L),
// sigma = s/L, and the proximal coefficients a_j = 1/(1 + tau q_j), d_j = tau a_j
// of the step whose pullback is taken (kernels.py:68-73).
template <typename T>
__device__ void qp_steps(const AdjParams<T>& p, int64_t X, const T* qx, T* base, T L, T* red) {
  const int n = p.st.n, m = p.st.m;
  T qmax = T(-INFINITY);
  for (int j = threadIdx.x; j < n; j += (int)blockDim.x) qmax = pmax(qmax, qx[j]);
  qmax = block_max_from(qmax, red);
  const T tau = p.safety / (qmax + L);
  for (int j = threadIdx.x; j < n; j += (int)blockDim.x) {
    const T a = T(1) / (T(1) + tau * qx[j]);
    base[j] = a;
    base[n + j] = tau * a;
    base[2 * n + m + j] = tau;
  }
  if (threadIdx.x == 0) {
    p.steps[2 * X] = tau;
    p.steps[2 * X + 1] = p.safety / L;
  }
  __syncthreads();
}

template <typename T, bool kAdmm>
__device__ __forceinline__ Sample<T> sample_of(const AdjParams<T>& p, int64_t X) {
  if constexpr (kAdmm) return make_admm_sample(p, X);
  else return make_sample(p, X);
}

// The adjoint system's operator: the CP pullback (mode 0) or ADMM's KKT operator.
template <typename T, bool kAdmm>
__device__ __forceinline__ void apply_any(const DevStructure& st, const Sample<T>& s, T* buf, T* tn,
                                          T* tm) {
  if constexpr (kAdmm) apply_kkt(st, s, buf, tn, tm);
  else apply_operator(st, s, buf, tn, tm);
}

// Threshold and initial residual of an ADMM sample's system (x = 0).
template <typename T>
__device__ void admm_initial_residual(const AdjParams<T>& p, const DevStructure& st, const Sample<T>& s,
                                      int64_t X, int W, T* buf, T* tn, T* tm, T* red) {
  const int n = st.n, m = st.m;
  const T zero = T(0);
  T gmax = zero;
  for (int e = threadIdx.x; e < W; e += (int)blockDim.x) {
    gmax = pmax(gmax, fabs(rhs_entry(s, n, m, e)));
    buf[e] = zero;
    p.x[X * W + e] = zero;
  }
  gmax = block_max(gmax, red);
  apply_kkt(st, s, buf, tn, tm);
  T r0 = zero;
  for (int e = threadIdx.x; e < W; e += (int)blockDim.x) r0 = pmax(r0, fabs(rhs_entry(s, n, m, e) - buf[e]));
  r0 = block_max(r0, red);
  if (threadIdx.x == 0) {
    const T thr = pmax(p.lin_atol, p.lin_tol * gmax);
    p.thresh[X] = thr;
    p.resinf[X] = r0;
    if (r0 > thr) atomicAdd(&p.cycle_act[0], 1u);
  }
  __syncthreads();
}

// ADMM's pullback (admm/solver.py:236-255) of the validated adjoint x = (v, w):
// target -> v, rhs -> a w, values -> -(dual_i v_j + a_i w_i y_j) on the support.
template <typename T>
__device__ void admm_pullback(const AdjParams<T>& p, const DevStructure& st, const Sample<T>& s,
                              int64_t X, const T* x, bool valid, int code, T ri) {
  const int n = st.n, m = st.m;
  const T zero = T(0);
  for (int j = threadIdx.x; j < n; j += (int)blockDim.x)
    if (p.g_target) p.g_target[X * n + j] = valid ? clean(x[j]) : zero;
  for (int i = threadIdx.x; i < m; i += (int)blockDim.x) {
    const T wi = valid ? T(s.dc[i]) * x[n + i] : zero;
    if (p.g_rhs) p.g_rhs[X * m + i] = clean(wi);
    if (p.g_values) {
      const T di = s.ds[i];
      T* gv = p.g_values + X * st.nnz;
      for (int k = st.row_ptr[i]; k < st.row_ptr[i + 1]; ++k) {
        const int j = st.col[k];
        const T vj = valid ? x[j] : zero;
        gv[k] = clean(-(di * vj + wi * s.ys[j]));
      }
    }
  }
  if (threadIdx.x == 0) {
    if (p.lin_status) p.lin_status[X] = code;
    if (p.lin_residual) p.lin_residual[X] = ri;
  }
  __syncthreads();
}

template <typename T, bool kSmem, bool kAdmm>
__global__ void __launch_bounds__(kThreads) cp_adjoint_kernel(const AdjParams<T> p) {
  extern __shared__ __align__(16) unsigned char dyn[];
  __shared__ int s_flag;
  const DevStructure& st = p.st;
  const int n = st.n, m = st.m, me = st.me;
  const int W = kAdmm ? n + m : 2 * n + m;
  const int R = p.R;
  T* sm = reinterpret_cast<T*>(dyn);
  T *buf, *tn, *tm, *small;
  if (kSmem) {
    buf = sm;
    tn = buf + W;
    tm = tn + n;
    small = tm + m;
  } else {
    buf = p.gbuf + (size_t)blockIdx.x * (W + n + m);
    tn = buf + W;
    tm = tn + n;
    small = sm;
  }
  T* hess = small;              // (R + 1) x R, row-major
  T* proj = hess + (R + 1) * R; // R + 1
  T* cs = proj + (R + 1);       // R
  T* sn = cs + R;               // R
  T* coef = sn + R;             // R + 1
  T* c2 = coef + (R + 1);       // R + 1
  T* bsv = c2 + (R + 1);        // R
  T* red = bsv + R;             // kWarps * kChunk
  T* V = p.basis + (size_t)blockIdx.x * (R + 1) * W;
  const T zero = T(0), one = T(1);
  const T eps = T(1e-30);
  const unsigned nblocks = gridDim.x + p.barrier_extra;
  const int stage = p.stage;

  // ---- phase 0: step sizes, linearisation, right-hand side ----------------
  // A sample whose forward solve did not converge has right-hand side
  // g = (where(converged, cot, 0), 0, 0) = 0 (bounds.py:133), so x = 0 solves its
  // system exactly and its gradients are zeros (bounds.py:148-165): it is not
  // linearised, never enters GMRES and gets zeros in the final phase.
  for (int64_t X = blockIdx.x; stage <= 1 && X < p.batch; X += gridDim.x) {
    if (threadIdx.x == 0 && p.work_steps) {
      p.work_steps[X] = 0;
      p.work_vectors[X] = 0;
    }
    if (p.converged[X] == 0) {
      if (threadIdx.x == 0) {
        p.thresh[X] = pmax(p.lin_atol, zero);
        p.resinf[X] = zero;
      }
      continue;
    }
    if constexpr (kAdmm) {
      // ADMM (admm/solver.py:184-194): rows active where equality, or where the
      // dual is positive and the slack rhs - K y is tight.
      const Sample<T> s = sample_of<T, kAdmm>(p, X);
      for (int i = threadIdx.x; i < m; i += (int)blockDim.x) {
        T acc = zero;
        for (int k = st.row_ptr[i]; k < st.row_ptr[i + 1]; ++k) acc = acc + s.vals[k] * s.ys[st.col[k]];
        const T slack = s.rhs[i] - acc;
        const bool act = i < me || (s.ds[i] > p.act_tol && slack <= pmax(p.act_tol, p.fwd_tol));
        s.dc[i] = act ? 1 : 0;
      }
      __syncthreads();
      admm_initial_residual(p, st, s, X, W, buf, tn, tm, red);
      continue;
    }
    const T* vals = p.values + X * p.values_stride;
    const T* qx = p.qp ? p.q + X * n : nullptr;
    T* base = (p.diag || p.qp) ? p.dsteps + X * ((p.qp ? 3 : 2) * (int64_t)n + m) : nullptr;
    if (p.diag) {
      for (int i = threadIdx.x; i < m; i += (int)blockDim.x) {
        T acc = zero;
        for (int k = st.row_ptr[i]; k < st.row_ptr[i + 1]; ++k) acc = acc + fabs(vals[k]) * one;
        base[2 * n + i] = p.safety / (acc > zero ? pmax(acc, T(1e-12)) : one);
      }
      for (int j = threadIdx.x; j < n; j += (int)blockDim.x) {
        T acc = zero;
        for (int e = st.col_ptr[j]; e < st.col_ptr[j + 1]; ++e)
          acc = acc + fabs(vals[st.csc_slot[e]]) * one;
        const T tau = p.safety / (acc > zero ? pmax(acc, T(1e-12)) : one);
        const T a = one / (one + tau * (qx ? qx[j] : one));
        base[j] = a;
        base[n + j] = tau * a;
        if (p.qp) base[2 * n + m + j] = tau;
      }
    } else if (p.qp && p.norm_bound) {
      // L = sqrt(max row sum |K| * max column sum |K|) (diagonal_qp.py:143-148).
      T rmax = zero, cmax = zero;
      for (int i = threadIdx.x; i < m; i += (int)blockDim.x) {
        T acc = zero;
        for (int k = st.row_ptr[i]; k < st.row_ptr[i + 1]; ++k) acc = acc + fabs(vals[k]) * one;
        rmax = pmax(rmax, acc);
      }
      for (int j = threadIdx.x; j < n; j += (int)blockDim.x) {
        T acc = zero;
        for (int e = st.col_ptr[j]; e < st.col_ptr[j + 1]; ++e)
          acc = acc + fabs(vals[st.csc_slot[e]]) * one;
        cmax = pmax(cmax, acc);
      }
      rmax = block_max(rmax, red);
      cmax = block_max(cmax, red);
      const T L = pmax(sqrt(rmax * cmax), T(1e-12));
      qp_steps(p, X, qx, base, L, red);
    } else {
      uint32_t k0, k1;
      split_key(p.norm_seed, p.sample_offset + X, p.total_batch, p.partitionable != 0, k0, k1);
      T* x = buf;
      T ss = zero;
      for (int j = threadIdx.x; j < n; j += (int)blockDim.x) {
        const T v = NormalBits<T>::draw(k0, k1, j, n, p.partitionable != 0);
        x[j] = v;
        ss = ss + v * v;
      }
      const T nrm = sqrt(block_sum(ss, red)) + T(1e-12);
      for (int j = threadIdx.x; j < n; j += (int)blockDim.x) x[j] = x[j] / nrm;
      T eig = zero;
      for (int it = 0; it < p.norm_iterations; ++it) {
        __syncthreads();
        for (int i = threadIdx.x; i < m; i += (int)blockDim.x) {
          T acc = zero;
          for (int k = st.row_ptr[i]; k < st.row_ptr[i + 1]; ++k) acc = acc + vals[k] * x[st.col[k]];
          tm[i] = acc;
        }
        __syncthreads();
        T xz = zero, zz = zero;
        for (int j = threadIdx.x; j < n; j += (int)blockDim.x) {
          T acc = zero;
          for (int e = st.col_ptr[j]; e < st.col_ptr[j + 1]; ++e)
            acc = acc + vals[st.csc_slot[e]] * tm[st.csc_row[e]];
          tn[j] = acc;
          xz = xz + x[j] * acc;
          zz = zz + acc * acc;
        }
        eig = block_sum(xz, red);
        const T zn = sqrt(block_sum(zz, red)) + T(1e-12);
        for (int j = threadIdx.x; j < n; j += (int)blockDim.x) x[j] = tn[j] / zn;
      }
      const T L = pmax(sqrt(pmax(eig, zero)) + T(1e-12), T(1e-12));
      if (p.qp) {
        qp_steps(p, X, qx, base, L, red);
      } else if (threadIdx.x == 0) {
        p.steps[2 * X] = p.safety / (one + L);
        p.steps[2 * X + 1] = p.safety / L;
      }
    }
    __syncthreads();
    const Sample<T> s = sample_of<T, kAdmm>(p, X);
    // Linearisation point (y*, lambda*, ybar = y*): lambda+ and derivative codes.
    for (int i = threadIdx.x; i < m; i += (int)blockDim.x) {
      T acc = zero;
      for (int k = st.row_ptr[i]; k < st.row_ptr[i + 1]; ++k) acc = acc + s.vals[k] * s.ys[st.col[k]];
      const T sg = s.sv ? s.sv[i] : s.sigma;
      const T raw = s.ds[i] + sg * (acc - s.rhs[i]);
      const T lp = i < me ? raw : pmax(raw, zero);
      s.dc[i] = (uint8_t)(i < me ? 2 : balanced_code(raw, lp, zero));
      tm[i] = lp;
      s.lamp[i] = lp;
    }
    __syncthreads();
    for (int j = threadIdx.x; j < n; j += (int)blockDim.x) {
      T t = zero;
      for (int e = st.col_ptr[j]; e < st.col_ptr[j + 1]; ++e)
        t = t + s.vals[st.csc_slot[e]] * tm[st.csc_row[e]];
      const T yo = s.ys[j];
      const T c = s.qp ? s.tgt[j] : -s.tgt[j];
      const T aa = s.av ? s.av[j] : s.a;
      const T dd = s.dv ? s.dv[j] : s.d;
      const T yr = (aa * yo - dd * t) + (-dd) * c;
      const T l = s.lo[j], u = s.up[j];
      const T u1 = pmax(l, yr);
      const T yn = pmin(u, u1);
      const int d_u1 = balanced_code(u1, yn, u);
      const int d_up = balanced_code(u, yn, u1);
      const int d_raw = balanced_code(yr, u1, l);
      const int d_lo = balanced_code(l, u1, yr);
      s.yc[j] = (uint8_t)(product_code(d_u1, d_raw) | (product_code(d_u1, d_lo) << 2) | (d_up << 4));
    }
    __syncthreads();
    // Right-hand side scale, threshold, x = 0 and the initial residual.
    T gmax = zero;
    for (int e = threadIdx.x; e < W; e += (int)blockDim.x) {
      gmax = pmax(gmax, fabs(rhs_entry(s, n, m, e)));
      buf[e] = zero;
      p.x[X * W + e] = zero;
    }
    gmax = block_max(gmax, red);
    apply_operator(st, s, buf, tn, tm);
    T r0 = zero;
    for (int e = threadIdx.x; e < W; e += (int)blockDim.x) r0 = pmax(r0, fabs(rhs_entry(s, n, m, e) - buf[e]));
    r0 = block_max(r0, red);
    if (threadIdx.x == 0) {
      const T thr = pmax(p.lin_atol, p.lin_tol * gmax);
      p.thresh[X] = thr;
      p.resinf[X] = r0;
      if (r0 > thr) atomicAdd(&p.cycle_act[0], 1u);
    }
    __syncthreads();
  }

  if (stage == 1) return;
  if (stage == 0 && !grid_barrier(p.barrier, nblocks, p.timeout_ns)) {
    if (threadIdx.x == 0) atomicExch(p.device_error, 1);
    return;
  }

  // ---- GMRES cycles in lockstep over the batch ------------------------------
  // Staged: exactly one cycle, whose budget and loop condition the host has
  // already established from the combined counters of every shard.
  int completed = stage == 2 ? p.completed0 : 0;
  int cycle = 0;
  bool any = stage == 2 ? true : (stage == 0 && atomicOr(&p.cycle_act[0], 0u) > 0);
  while (completed < p.max_it && any) {
    const int limit = min(R, p.max_it - completed);
    for (int64_t X = blockIdx.x; X < p.batch; X += gridDim.x) {
      const T thr = p.thresh[X];
      if (!(p.resinf[X] > thr)) continue;  // not cycle-active: frozen
      const Sample<T> s = sample_of<T, kAdmm>(p, X);
      T* x = p.x + X * W;
      // residual = g - A x, normalised into V[0]
      for (int e = threadIdx.x; e < W; e += (int)blockDim.x) buf[e] = x[e];
      __syncthreads();
      apply_any<T, kAdmm>(st, s, buf, tn, tm);
      T ss = zero;
      for (int e = threadIdx.x; e < W; e += (int)blockDim.x) {
        const T r = rhs_entry(s, n, m, e) - buf[e];
        buf[e] = r;
        ss = ss + r * r;
      }
      const T beta = sqrt(block_sum(ss, red));
      const T safe_beta = pmax(beta, eps);
      for (int e = threadIdx.x; e < W; e += (int)blockDim.x) {
        const T v = buf[e] / safe_beta;
        buf[e] = v;
        V[e] = v;
      }
      for (int q = threadIdx.x; q < (R + 1) * R; q += (int)blockDim.x) hess[q] = zero;
      for (int q = threadIdx.x; q < R + 1; q += (int)blockDim.x) proj[q] = q == 0 ? beta : zero;
      for (int q = threadIdx.x; q < R; q += (int)blockDim.x) { cs[q] = zero; sn[q] = zero; }
      if (threadIdx.x == 0) s_flag = 1;
      __syncthreads();
      int it = 0;
      while (it < limit && s_flag) {
        apply_any<T, kAdmm>(st, s, buf, tn, tm);
        basis_dots(V, W, buf, it + 1, coef, red);
        basis_update(V, W, buf, it + 1, coef);
        basis_dots(V, W, buf, it + 1, c2, red);
        basis_update(V, W, buf, it + 1, c2);
        for (int q = threadIdx.x; q <= it; q += (int)blockDim.x) coef[q] = coef[q] + c2[q];
        T nsq = zero;
        for (int e = threadIdx.x; e < W; e += (int)blockDim.x) nsq = nsq + buf[e] * buf[e];
        const T nn = sqrt(block_sum(nsq, red));
        const T sn_ = pmax(nn, eps);
        int fin = 1;
        T* Vn = V + (size_t)(it + 1) * W;
        for (int e = threadIdx.x; e < W; e += (int)blockDim.x) {
          const T v = buf[e] / sn_;
          buf[e] = v;
          Vn[e] = v;
          fin &= finite(v) ? 1 : 0;
        }
        fin = block_and(fin);
        if (threadIdx.x == 0)
          s_flag = givens_step(it, R, coef, nn, fin != 0, thr, hess, cs, sn, proj) ? 1 : 0;
        __syncthreads();
        ++it;
      }
      const int row_steps = it;
      if (threadIdx.x == 0) back_substitute(R, row_steps, hess, proj, bsv);
      __syncthreads();
#pragma unroll 2
      for (int e = threadIdx.x; e < W; e += (int)blockDim.x) {
        const T cand = x[e] + basis_combination(V, W, e, row_steps, bsv);
        buf[e] = cand;
        x[e] = cand;
      }
      __syncthreads();
      apply_any<T, kAdmm>(st, s, buf, tn, tm);
      T cn = zero;
      for (int e = threadIdx.x; e < W; e += (int)blockDim.x) cn = pmax(cn, fabs(rhs_entry(s, n, m, e) - buf[e]));
      cn = block_max(cn, red);
      if (threadIdx.x == 0) {
        p.resinf[X] = cn;
        if (p.work_steps) {
          // Step j of the cycle orthogonalises against j + 1 basis vectors.
          p.work_steps[X] += row_steps;
          p.work_vectors[X] += (long long)row_steps * (row_steps + 1) / 2;
        }
        atomicMax(&p.cycle_len[cycle], (unsigned)row_steps);
        if (cn > thr) atomicAdd(&p.cycle_act[cycle + 1], 1u);
      }
      __syncthreads();
    }
    if (stage == 2) return;
    if (!grid_barrier(p.barrier, nblocks, p.timeout_ns)) {
      if (threadIdx.x == 0) atomicExch(p.device_error, 1);
      return;
    }
    completed += (int)atomicOr(&p.cycle_len[cycle], 0u);
    any = atomicOr(&p.cycle_act[cycle + 1], 0u) > 0;
    ++cycle;
  }

  // ---- validity and parameter pullback (bounds.py:148-165) ------------------
  for (int64_t X = blockIdx.x; (stage == 0 || stage == 3) && X < p.batch; X += gridDim.x) {
    if (p.converged[X] == 0) {
      // Zero right-hand side: zero solution (status 0, residual 0), zero gradients.
      for (int j = threadIdx.x; j < n; j += (int)blockDim.x) {
        if (p.g_target) p.g_target[X * n + j] = zero;
        if (p.g_lower) p.g_lower[X * n + j] = zero;
        if (p.g_upper) p.g_upper[X * n + j] = zero;
        if (p.g_q) p.g_q[X * n + j] = zero;
        if (p.g_c) p.g_c[X * n + j] = zero;
      }
      for (int i = threadIdx.x; i < m; i += (int)blockDim.x)
        if (p.g_rhs) p.g_rhs[X * m + i] = zero;
      if (p.g_values)
        for (int k = threadIdx.x; k < st.nnz; k += (int)blockDim.x) p.g_values[X * st.nnz + k] = zero;
      if (threadIdx.x == 0) {
        if (p.lin_status) p.lin_status[X] = 0;
        if (p.lin_residual) p.lin_residual[X] = zero;
      }
      continue;
    }
    const Sample<T> s = sample_of<T, kAdmm>(p, X);
    const T* x = p.x + X * W;
    int fin = 1;
    for (int e = threadIdx.x; e < W; e += (int)blockDim.x) {
      const T v = x[e];
      buf[e] = v;
      fin &= finite(v) ? 1 : 0;
    }
    fin = block_and(fin);
    const T ri = p.resinf[X];
    const T thr = p.thresh[X];
    const bool fin_all = fin && finite(ri);
    const int code = !fin_all ? 2 : (ri <= thr ? 0 : 1);
    const bool valid = s.conv && fin && finite(ri) && (code == 0 || ri <= p.adj_tol);
    if (!valid) {
      for (int e = threadIdx.x; e < W; e += (int)blockDim.x) buf[e] = zero;
    }
    __syncthreads();
    if constexpr (kAdmm) {
      admm_pullback(p, st, s, X, buf, valid, code, ri);
      continue;
    }
    const T* zy = buf;
    const T* zd = buf + n;
    const T* zb = buf + n + m;
    for (int j = threadIdx.x; j < n; j += (int)blockDim.x) {
      const T vy = zy[j], vb = zb[j];
      const T gg = (vy + vb) + vb;
      const int code_j = s.yc[j];
      const T graw = gg * code_factor<T>(code_j & 3);
      const T glo = gg * code_factor<T>((code_j >> 2) & 3);
      const T gup = gg * balanced_factor<T>((code_j >> 4) & 3);
      const T dd = s.dv ? s.dv[j] : s.d;
      if (s.qp) {
        // Cotangents of c and q through proximal_coefficients (kernels.py:68-73):
        // offset = (-d) c, d = tau a, a = 1 / (1 + tau q), and y_raw = a y - d t + offset
        // with t = K^T lambda+ at the linearisation point, transposed as JAX does
        // (the reciprocal's cotangent is -(ct * (den * den)^-1)).
        T tj = zero;
        for (int e = st.col_ptr[j]; e < st.col_ptr[j + 1]; ++e)
          tj = tj + s.vals[st.csc_slot[e]] * s.lamp[st.csc_row[e]];
        const T tauj = p.dsteps[X * (3 * (int64_t)n + m) + 2 * n + m + j];
        const T dwbar = ((-graw) * tj) + (-(graw * s.tgt[j]));
        const T invbar = (graw * s.ys[j]) + (tauj * dwbar);
        const T den = one + tauj * p.q[X * n + j];
        if (p.g_q) p.g_q[X * n + j] = clean(tauj * (-((invbar * (one / (den * den))) * one)));
        if (p.g_c) p.g_c[X * n + j] = clean((-dd) * graw);
      }
      tn[j] = dd * (-graw);
      if (p.g_target) p.g_target[X * n + j] = clean(dd * graw);
      if (p.g_lower) p.g_lower[X * n + j] = clean(glo);
      if (p.g_upper) p.g_upper[X * n + j] = clean(gup);
    }
    __syncthreads();
    for (int i = threadIdx.x; i < m; i += (int)blockDim.x) {
      T acc = zero;
      for (int k = st.row_ptr[i]; k < st.row_ptr[i + 1]; ++k) acc = acc + s.vals[k] * tn[st.col[k]];
      const T mu = zd[i] + acc;
      const T mur = i < me ? mu : mu * balanced_factor<T>(s.dc[i]);
      const T sg = s.sv ? s.sv[i] : s.sigma;
      const T w = sg * mur;
      if (p.g_rhs) p.g_rhs[X * m + i] = clean(-w);
      if (p.g_values) {
        const T lp = s.lamp[i];
        T* gv = p.g_values + X * st.nnz;
        for (int k = st.row_ptr[i]; k < st.row_ptr[i + 1]; ++k) {
          const int j = st.col[k];
          gv[k] = clean(w * s.ys[j] + tn[j] * lp);
        }
      }
    }
    if (threadIdx.x == 0) {
      if (p.lin_status) p.lin_status[X] = code;
      if (p.lin_residual) p.lin_residual[X] = ri;
    }
    __syncthreads();
  }
}

template <typename T>
size_t small_elems(int R) {
  return (size_t)(R + 1) * R + (R + 1) + 2 * (size_t)R + 2 * (size_t)(R + 1) + R + kWarps * kChunk;
}

}  // namespace

int adjoint_threads(int n, int m) {
  if (const char* env = std::getenv("PURIN_CP_ADJOINT_THREADS")) {
    const int t = std::atoi(env);
    if (t == kSmallThreads / 2 || t == kSmallThreads || t == kThreads) return t;
  }
  const int64_t W = 2 * (int64_t)n + m;
  if (W <= (int64_t)kSmallEntriesPerThread * (kSmallThreads / 2)) return kSmallThreads / 2;
  return W <= (int64_t)kSmallEntriesPerThread * kSmallThreads ? kSmallThreads : kThreads;
}

template <typename T>
size_t adjoint_smem_bytes(int n, int m, int R, bool smem_vectors) {
  const size_t W = 2 * (size_t)n + m;
  size_t elems = small_elems<T>(R);
  if (smem_vectors) elems += W + n + m;
  return elems * sizeof(T);
}

template <typename T, bool kSmem, bool kAdmm>
int adjoint_grid_k(int sm_count, int threads, size_t smem, int64_t batch) {
  auto kern = cp_adjoint_kernel<T, kSmem, kAdmm>;
  int per_sm = 0;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, threads, smem) != cudaSuccess)
    return 0;
  int64_t grid = (int64_t)per_sm * sm_count;
  if (grid > batch) grid = batch;
  return (int)grid;
}

template <typename T>
int adjoint_grid(int sm_count, int n, int m, int R, bool smem_vectors, int64_t batch, bool admm) {
  const size_t smem = adjoint_smem_bytes<T>(n, m, R, smem_vectors);
  const int threads = adjoint_threads(n, m);
  if (admm)
    return smem_vectors ? adjoint_grid_k<T, true, true>(sm_count, threads, smem, batch)
                        : adjoint_grid_k<T, false, true>(sm_count, threads, smem, batch);
  return smem_vectors ? adjoint_grid_k<T, true, false>(sm_count, threads, smem, batch)
                      : adjoint_grid_k<T, false, false>(sm_count, threads, smem, batch);
}

template <typename T>
cudaError_t launch_adjoint(const AdjParams<T>& p, int grid, bool smem_vectors, cudaStream_t stream) {
  const int n = p.st.n, m = p.st.m;
  const size_t smem = adjoint_smem_bytes<T>(n, m, p.R, smem_vectors);
  void* args[] = {(void*)&p};
  const bool admm = p.mode == 1;
  auto kern = admm ? (smem_vectors ? cp_adjoint_kernel<T, true, true> : cp_adjoint_kernel<T, false, true>)
                   : (smem_vectors ? cp_adjoint_kernel<T, true, false> : cp_adjoint_kernel<T, false, false>);
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  const int threads = adjoint_threads(n, m);
  // Only the fused launch has grid barriers, so only it needs co-residency.
  if (p.stage == 0)
    return cudaLaunchCooperativeKernel((void*)kern, dim3(grid), dim3(threads), args, smem, stream);
  return cudaLaunchKernel((void*)kern, dim3(grid), dim3(threads), args, smem, stream);
}

template size_t adjoint_smem_bytes<double>(int, int, int, bool);
template size_t adjoint_smem_bytes<float>(int, int, int, bool);
template int adjoint_grid<double>(int, int, int, int, bool, int64_t, bool);
template int adjoint_grid<float>(int, int, int, int, bool, int64_t, bool);
template cudaError_t launch_adjoint<double>(const AdjParams<double>&, int, bool, cudaStream_t);
template cudaError_t launch_adjoint<float>(const AdjParams<float>&, int, bool, cudaStream_t);

}  // namespace purin
