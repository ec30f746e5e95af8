// Oracle (test and baseline infrastructure): the batched Chambolle-Pock loop of
// oracle/cp.py::sparse_cp, which restates src/purin/solvers/chambolle_pock/
// kernels.py:178-305, written in C++ for the host cores (OpenMP over samples)
// so the CPU baseline is not limited by NumPy's per-operation overhead.
//
// fp64, q = 1 and c = -target as in the projection layer (bounds.py:42-66).
// Every product and sum is evaluated one term at a time in the reference's
// order: K @ x along each padded row (kernels.py:43-49 with
// linalg/sparse/operators.py:507-518), K.T @ y per column in the flattened
// (row, slot) order of the scatter-add (operators.py:521-533).  Padding terms
// (exact +0.0) are skipped, which can only change the sign of a zero sum.  The
// objective sums of the gap (kernels.py:164-175) are sequential here, while
// NumPy sums pairwise, so the gap agrees with the NumPy oracle to rounding.
// Maxima propagate NaN like jax.lax.max; clip is minimum(upper, maximum(lower, x)).
// Compiled with -ffp-contract=off: products and sums round separately.
#include <omp.h>

#include <cmath>
#include <cstdint>
#include <vector>

namespace {

inline double pmax(double a, double b) { return (a > b || a != a) ? a : b; }
inline double pmin(double a, double b) { return (a < b || a != a) ? a : b; }
inline double clip(double x, double lo, double hi) { return pmin(hi, pmax(lo, x)); }

struct Columns {
  std::vector<int32_t> ptr;    // n + 1
  std::vector<int32_t> entry;  // flat row * width + slot, in scatter order per column
  std::vector<int32_t> row;    // the entry's row
};

Columns build_columns(int n, int m, int width, const int32_t* support, const uint8_t* mask) {
  Columns c;
  c.ptr.assign(n + 1, 0);
  for (int64_t e = 0; e < (int64_t)m * width; ++e)
    if (mask[e]) ++c.ptr[support[e] + 1];
  for (int j = 0; j < n; ++j) c.ptr[j + 1] += c.ptr[j];
  c.entry.resize(c.ptr[n]);
  c.row.resize(c.ptr[n]);
  std::vector<int32_t> fill(c.ptr.begin(), c.ptr.end() - 1);
  for (int64_t e = 0; e < (int64_t)m * width; ++e)
    if (mask[e]) {
      c.row[fill[support[e]]] = (int32_t)(e / width);
      c.entry[fill[support[e]]++] = (int32_t)e;
    }
  return c;
}

struct Problem {
  int n, m, me, width;
  const int32_t* support;
  const uint8_t* mask;
  const Columns* cols;
};

// out[i] = sum_k v[i,k] * x[support[i,k]] (row order, padding skipped).
void matvec(const Problem& P, const double* v, const double* x, double* out) {
  for (int i = 0; i < P.m; ++i) {
    double acc = 0.0;
    const int64_t base = (int64_t)i * P.width;
    for (int k = 0; k < P.width; ++k)
      if (P.mask[base + k]) acc = acc + v[base + k] * x[P.support[base + k]];
    out[i] = acc;
  }
}

// out[j] = sum over column j's entries (i, k), in scatter order, of v[i,k] * y[i].
void tmatvec(const Problem& P, const double* v, const double* y, double* out) {
  const Columns& c = *P.cols;
  for (int j = 0; j < P.n; ++j) {
    double acc = 0.0;
    for (int e = c.ptr[j]; e < c.ptr[j + 1]; ++e) acc = acc + v[c.entry[e]] * y[c.row[e]];
    out[j] = acc;
  }
}

struct Diag {
  double residual, gap, stationarity;
  bool finite;
};

// kernels.py:153-175 and the stationarity of 272-274 at (y, dual), with t = K.T dual.
Diag diagnostics(const Problem& P, const double* v, const double* y, const double* dual,
                 const double* t, const double* target, const double* rhs, const double* lo,
                 const double* up, double* scratch_m) {
  matvec(P, v, y, scratch_m);
  double eq = 0.0, in = 0.0, bound_lo = 0.0, bound_up = 0.0;
  for (int i = 0; i < P.m; ++i) {
    const double r = scratch_m[i] - rhs[i];
    if (i < P.me) eq = pmax(eq, std::fabs(r));
    else in = pmax(in, pmax(r, 0.0));
  }
  double primal = 0.0, dual_obj = 0.0, rhs_dual = 0.0, stat = 0.0;
  bool finite = true;
  for (int j = 0; j < P.n; ++j) {
    const double c = -target[j];
    bound_lo = pmax(bound_lo, pmax(lo[j] - y[j], 0.0));
    bound_up = pmax(bound_up, pmax(y[j] - up[j], 0.0));
    primal = primal + (0.5 * 1.0 * y[j] * y[j] + c * y[j]);
    const double tt = c + t[j];
    const double mn = clip(-tt / 1.0, lo[j], up[j]);
    dual_obj = dual_obj + (0.5 * 1.0 * (mn * mn) + tt * mn);
    stat = pmax(stat, std::fabs(y[j] - clip(y[j] - ((1.0 * y[j] + c) + t[j]), lo[j], up[j])));
    finite = finite && std::isfinite(y[j]);
  }
  for (int i = 0; i < P.m; ++i) {
    rhs_dual = rhs_dual + rhs[i] * dual[i];
    finite = finite && std::isfinite(dual[i]);
  }
  const double D = dual_obj - rhs_dual;
  const double gap = pmax(primal - D, 0.0) / pmax(1.0, pmax(std::fabs(primal), std::fabs(D)));
  Diag d;
  d.residual = pmax(pmax(eq, in), pmax(bound_lo, bound_up));
  d.gap = gap;
  d.stationarity = stat;
  d.finite = finite && std::isfinite(gap);
  return d;
}

}  // namespace

extern "C" {

// One projection batch.  Arrays are row-major fp64 (int32/uint8 for the layout):
// support/mask (m, width); values (B, m*width) with stride values_stride (0 when
// shared); rhs, dual0 (B, m); target, lower, upper (B, n); tolerance, tau,
// sigma (B).  y0 = target.  Outputs y (B, n), dual (B, m), iterations (B),
// residual (B, max with stationarity), gap (B), converged (B).  threads <= 0
// uses OpenMP's default team size.
int oracle_cp_solve(int threads, int batch, int n, int m, int me, int width,
                    const int32_t* support, const uint8_t* mask, const double* values, int64_t values_stride,
                    const double* rhs, const double* target, const double* lower,
                    const double* upper, const double* dual0, const double* tolerance,
                    const double* tau0, const double* sigma0, int accelerated, int max_iterations,
                    double* y_out, double* dual_out, int32_t* it_out, double* res_out,
                    double* gap_out, uint8_t* conv_out) {
  if (batch < 0 || n < 0 || m < 0 || width < 1) return 1;
  const Columns cols = build_columns(n, m, width, support, mask);
  const Problem P{n, m, me, width, support, mask, &cols};
  const int team = threads > 0 ? threads : omp_get_max_threads();
#pragma omp parallel for schedule(dynamic, 1) num_threads(team)
  for (int b = 0; b < batch; ++b) {
    const double* v = values + (int64_t)b * values_stride;
    const double* tg = target + (int64_t)b * n;
    const double* rh = rhs + (int64_t)b * m;
    const double* lo = lower + (int64_t)b * n;
    const double* up = upper + (int64_t)b * n;
    std::vector<double> y(tg, tg + n), ybar(tg, tg + n), ny(n), nb(n), t(n);
    std::vector<double> dual(dual0 + (int64_t)b * m, dual0 + (int64_t)b * m + m), nd(m), km(m);
    double tau = tau0[b], sigma = sigma0[b], theta = 1.0;
    const double tol = tolerance[b];
    int count = 0;
    bool done = false;
    for (int it = 0; it < max_iterations && !done; ++it) {
      // cp_step (kernels.py:91-150).
      matvec(P, v, ybar.data(), km.data());
      for (int i = 0; i < m; ++i) {
        const double raw = dual[i] + sigma * (km[i] - rh[i]);
        nd[i] = i < me ? raw : pmax(raw, 0.0);
      }
      tmatvec(P, v, nd.data(), t.data());
      const double inverse = 1.0 / (1.0 + tau * 1.0);
      const double weight = tau * inverse;
      for (int j = 0; j < n; ++j) {
        const double offset = -weight * -tg[j];
        const double yr = inverse * y[j] - weight * t[j] + offset;
        ny[j] = clip(yr, lo[j], up[j]);
        nb[j] = ny[j] + theta * (ny[j] - y[j]);
      }
      const Diag d = diagnostics(P, v, ny.data(), nd.data(), t.data(), tg, rh, lo, up, km.data());
      y.swap(ny);
      dual.swap(nd);
      ybar.swap(nb);
      ++count;
      done = d.finite && d.residual <= tol && d.gap <= tol && d.stationarity <= tol;
      if (accelerated) {
        const double nt = 1.0 / std::sqrt(1.0 + 1.0 * tau);
        tau = nt * tau;
        sigma = sigma / nt;
        theta = nt;
      }
    }
    // Final report (kernels.py:291-305).
    tmatvec(P, v, dual.data(), t.data());
    const Diag d = diagnostics(P, v, y.data(), dual.data(), t.data(), tg, rh, lo, up, km.data());
    const bool finite = d.finite && std::isfinite(d.residual);
    for (int j = 0; j < n; ++j) y_out[(int64_t)b * n + j] = y[j];
    for (int i = 0; i < m; ++i) dual_out[(int64_t)b * m + i] = dual[i];
    it_out[b] = count;
    res_out[b] = pmax(d.residual, d.stationarity);
    gap_out[b] = d.gap;
    conv_out[b] = (finite && d.residual <= tol && d.gap <= tol && d.stationarity <= tol) ? 1 : 0;
  }
  return 0;
}

}  // extern "C"
