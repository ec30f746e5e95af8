// Device helpers shared by the adjoint kernels (cp_adjoint.cu: the CTA-per-sample
// kernel; cp_gmres_cluster.cu: the cluster-resident GMRES cycles): block
// reductions, the per-sample view of the linearisation, the pullback operator
// z <- z - J^T z of one CP step (bounds.py:109-130), the right-hand side
// (bounds.py:131-138), jnp.hypot, and the Givens / back-substitution steps of
// restarted GMRES (primal_dual_interior_point/operators.py:873-917).
#pragma once

#include <cuda_runtime.h>

#include "common.cuh"
#include "cp_kernels.cuh"

namespace purin {
namespace {

// Threads per CTA: at most kThreads (the shared reduction arrays are sized for
// it); every loop and reduction uses blockDim.x, so a launch may use fewer.
constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
// Krylov vectors of at most this many entries per thread run on kSmallThreads
// (or half of it): a small sample gets a half or a quarter of the threads and
// an SM two or four times the samples in flight at the same register budget
// (the per-sample phases are barrier-bound).
constexpr int kSmallThreads = 128;
constexpr int kSmallEntriesPerThread = 4;
constexpr int kChunk = 8;  // basis vectors per register-resident dot-product chunk

template <typename T>
__device__ __forceinline__ T warp_sum(T v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += shfl_xor(v, o);
  return v;
}
template <typename T>
__device__ __forceinline__ T warp_max(T v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = pmax(v, shfl_xor(v, o));
  return v;
}

// Block-wide reductions; every thread receives the result.
template <typename T>
__device__ T block_sum(T v, T* red) {
  v = warp_sum(v);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  T total = T(0);
#pragma unroll
  for (int w = 0; w < (int)(blockDim.x >> 5); ++w) total = total + red[w];
  __syncthreads();
  return total;
}
template <typename T>
__device__ T block_max(T v, T* red) {
  v = warp_max(v);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  T total = T(0);
#pragma unroll
  for (int w = 0; w < (int)(blockDim.x >> 5); ++w) total = pmax(total, red[w]);
  __syncthreads();
  return total;
}
// Block-wide max whose identity is -inf (block_max starts from 0, which suits
// nonnegative quantities only).
template <typename T>
__device__ T block_max_from(T v, T* red) {
  v = warp_max(v);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  T total = red[0];
#pragma unroll
  for (int w = 1; w < (int)(blockDim.x >> 5); ++w) total = pmax(total, red[w]);
  __syncthreads();
  return total;
}
__device__ __forceinline__ int block_and(int v) {
  return __syncthreads_and(v);
}

template <typename T>
struct Sample {
  const T* vals;
  const T* tgt;
  const T* rhs;
  const T* lo;
  const T* up;
  const T* ys;     // forward solution y* (also ybar at the linearisation point)
  const T* ds;     // forward duals
  const T* cot;    // cotangent of y
  const T* cotd;   // cotangent of the duals (QP), or null
  bool conv;
  bool qp;         // tgt holds c (diagonal QP) instead of the target (c = -target)
  T* lamp;         // lambda+ at the linearisation point
  uint8_t* yc;     // per-column derivative codes
  uint8_t* dc;     // per-row derivative codes
  T a, d, sigma;   // scalar steps
  const T* av;     // diagonal steps (or null)
  const T* dv;
  const T* sv;
};

// ADMM (mode 1): the KKT operator and the pullback read the values, the
// activity codes, y, the duals and the cotangent only.
template <typename T>
__device__ Sample<T> make_admm_sample(const AdjParams<T>& p, int64_t X) {
  {
    const int n = p.st.n, m = p.st.m;
    Sample<T> s{};
    s.vals = p.values + X * p.values_stride;
    s.rhs = p.rhs + X * m;
    s.ys = p.y + X * n;
    s.ds = p.dual + X * m;
    s.cot = p.cot_y + X * n;
    s.cotd = nullptr;
    s.conv = p.converged[X] != 0;
    s.qp = false;
    s.dc = p.dcode + X * m;
    s.yc = p.ycode + X * n;
    return s;
  }
}

template <typename T>
__device__ Sample<T> make_sample(const AdjParams<T>& p, int64_t X) {
  const int n = p.st.n, m = p.st.m;
  Sample<T> s;
  s.vals = p.values + X * p.values_stride;
  s.qp = p.qp != 0;
  s.tgt = s.qp ? p.c + X * n : p.target + X * n;
  s.rhs = p.rhs + X * m;
  s.lo = p.lower + X * p.bounds_stride;
  s.up = p.upper + X * p.bounds_stride;
  s.ys = p.y + X * n;
  s.ds = p.dual + X * m;
  s.cot = p.cot_y + X * n;
  s.cotd = p.cot_dual ? p.cot_dual + X * m : nullptr;
  s.conv = p.converged[X] != 0;
  s.lamp = p.lamp + X * m;
  s.yc = p.ycode + X * n;
  s.dc = p.dcode + X * m;
  if (p.diag || p.qp) {
    T* base = p.dsteps + X * ((p.qp ? 3 : 2) * (int64_t)n + m);
    s.av = base;
    s.dv = base + n;
    s.sv = p.diag ? base + 2 * n : nullptr;
    s.a = s.d = T(0);
    s.sigma = p.diag ? T(0) : p.steps[2 * X + 1];
  } else {
    const T tau = p.steps[2 * X], sigma = p.steps[2 * X + 1];
    s.a = T(1) / (T(1) + tau * T(1));
    s.d = tau * s.a;
    s.sigma = sigma;
    s.av = s.dv = s.sv = nullptr;
  }
  return s;
}

// ADMM's active-set KKT operator (admm/solver.py:196-206) on z = (v, w):
// (v + K^T (a w), a K v + (1 - a) w) with a_i = dc[i] in {0, 1}.
template <typename T>
__device__ void apply_kkt(const DevStructure& st, const Sample<T>& s, T* buf, T* tn, T* tm) {
  const int n = st.n, m = st.m;
  T* zv = buf;
  T* zw = buf + n;
  for (int i = threadIdx.x; i < m; i += (int)blockDim.x) tm[i] = T(s.dc[i]) * zw[i];
  __syncthreads();
  for (int j = threadIdx.x; j < n; j += (int)blockDim.x) {
    T acc = T(0);
    for (int e = st.col_ptr[j]; e < st.col_ptr[j + 1]; ++e)
      acc = acc + s.vals[st.csc_slot[e]] * tm[st.csc_row[e]];
    tn[j] = acc;
  }
  for (int i = threadIdx.x; i < m; i += (int)blockDim.x) {
    T acc = T(0);
    for (int k = st.row_ptr[i]; k < st.row_ptr[i + 1]; ++k) acc = acc + s.vals[k] * zv[st.col[k]];
    const T a = T(s.dc[i]);
    zw[i] = a * acc + (T(1) - a) * zw[i];
  }
  __syncthreads();
  for (int j = threadIdx.x; j < n; j += (int)blockDim.x) zv[j] = zv[j] + tn[j];
  __syncthreads();
}

// z <- z - J^T z for the packed state z = (y, dual, ybar) (bounds.py:130).
template <typename T>
__device__ void apply_operator(const DevStructure& st, const Sample<T>& s, T* buf, T* tn, T* tm) {
  const int n = st.n, m = st.m, me = st.me;
  T* zy = buf;
  T* zd = buf + n;
  T* zb = buf + n + m;
  for (int j = threadIdx.x; j < n; j += (int)blockDim.x) {
    const T vy = zy[j], vb = zb[j];
    const T gg = (vy + vb) + vb;
    const T graw = gg * code_factor<T>(s.yc[j] & 3);
    const T aa = s.av ? s.av[j] : s.a;
    const T dd = s.dv ? s.dv[j] : s.d;
    tn[j] = dd * (-graw);
    zy[j] = vy - (aa * graw - vb);
  }
  __syncthreads();
  for (int i = threadIdx.x; i < m; i += (int)blockDim.x) {
    T acc = T(0);
    for (int k = st.row_ptr[i]; k < st.row_ptr[i + 1]; ++k) acc = acc + s.vals[k] * tn[st.col[k]];
    const T mu = zd[i] + acc;
    const T mur = i < me ? mu : mu * balanced_factor<T>(s.dc[i]);
    const T sg = s.sv ? s.sv[i] : s.sigma;
    tm[i] = sg * mur;
    zd[i] = zd[i] - mur;
  }
  __syncthreads();
  for (int j = threadIdx.x; j < n; j += (int)blockDim.x) {
    T acc = T(0);
    for (int e = st.col_ptr[j]; e < st.col_ptr[j + 1]; ++e)
      acc = acc + s.vals[st.csc_slot[e]] * tm[st.csc_row[e]];
    zb[j] = zb[j] - acc;
  }
  __syncthreads();
}

// g = (where(converged, cot_y, 0), where(converged, cot_dual, 0), 0) entry e
// (bounds.py:131-138; diagonal_qp.py:191-196 adds the dual cotangent).
template <typename T>
__device__ __forceinline__ T rhs_entry(const Sample<T>& s, int n, int m, int e) {
  if (!s.conv) return T(0);
  if (e < n) return s.cot[e];
  return (s.cotd && e < n + m) ? s.cotd[e - n] : T(0);
}

// jnp.hypot: max * sqrt(1 + (min/max)^2).
template <typename T>
__device__ __forceinline__ T jax_hypot(T x, T y) {
  const T a = fabs(x), b = fabs(y);
  const bool inf = isinf(a) || isinf(b);
  const T hi = pmax(a, b), lo = pmin(a, b);
  const T safe = hi == T(0) ? T(1) : hi;
  const T q = lo / safe;
  const T r = hi == T(0) ? hi : hi * sqrt(T(1) + q * q);
  return inf ? T(INFINITY) : r;
}

// Givens step of Arnoldi step `it` (thread-local; run by one thread): the new
// Hessenberg column (coef[0..it], nn) gets the previous rotations, a new
// rotation zeroes its subdiagonal (operators.py:873-900), and the projected
// residual is rotated.  The column is written to hess (entries below it + 1
// stay zero from the cycle's start).  The rotated entry carried from one
// rotation to the next stays in a register.  Returns whether GMRES continues:
// every quantity finite, no happy breakdown, estimate above thr.
template <typename T>
__device__ bool givens_step(int it, int R, const T* coef, T nn, bool fin, T thr, T* hess, T* cs,
                            T* sn, T* proj) {
  const T zero = T(0), one = T(1);
  const T eps = T(1e-30), breakdown = T(1e-14);
  // Rotation r acts on (column entry r, already rotated; entry r + 1, not yet).
  T carry = coef[0];
  for (int r = 0; r < it; ++r) {
    const T g2 = coef[r + 1];
    const T c = cs[r], s = sn[r];
    hess[r * R + it] = c * carry + s * g2;
    carry = -s * carry + c * g2;
  }
  const T diag = carry, sub = nn;
  const T rot = jax_hypot(diag, sub);
  const T safe_rot = pmax(rot, eps);
  const bool big = rot > eps;
  const T nc = big ? diag / safe_rot : one;
  const T ns = big ? sub / safe_rot : zero;
  cs[it] = nc;
  sn[it] = ns;
  hess[it * R + it] = rot;
  hess[(it + 1) * R + it] = zero;
  const T cur = proj[it], nxt = proj[it + 1];
  const T rc = nc * cur + ns * nxt;
  const T rn = -ns * cur + nc * nxt;
  proj[it] = rc;
  proj[it + 1] = rn;
  const T estimate = fabs(rn);
  const bool ok = finite(estimate) && finite(rot) && fin;
  const bool happy = nn <= breakdown;
  return ok && !happy && estimate > thr;
}

// Back-substitution of the rotated Hessenberg system (operators.py:902-917;
// thread-local): bsv[0..R) solves the upper triangle over the first `steps`
// rows, zero beyond.  Rows and columns from `steps` on hold exact zeros in the
// reference's full-width sums (unwritten columns, and bsv zero there), so the
// sums run over the first `steps` terms only, which gives the same values.
template <typename T>
__device__ void back_substitute(int R, int steps, const T* hess, const T* proj, T* bsv) {
  const T zero = T(0), one = T(1), eps = T(1e-30);
  for (int q = 0; q < R; ++q) bsv[q] = zero;
  for (int row = steps - 1; row >= 0; --row) {
    T trailing = zero;
    for (int q = 0; q < steps; ++q) trailing = trailing + hess[row * R + q] * bsv[q];
    const T numerator = proj[row] - trailing;
    const T diag = hess[row * R + row];
    const T safe = fabs(diag) > eps ? diag : one;
    bsv[row] = numerator / safe;
  }
}

}  // namespace
}  // namespace purin
