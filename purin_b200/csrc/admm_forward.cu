// ADMM forward solve: sparse_admm (src/purin/solvers/admm/kernels.py:43-283), the
// OSQP-style iteration of PreparedADMMProjection (src/purin/solvers/admm/solver.py:60-97),
// for batched diagonal QPs  min 0.5 x'diag(q)x + c'x  s.t.  lower <= K x <= upper.
//
// One CTA owns one sample for the whole solve; its vectors (x, the x-update's
// right-hand side and solution, the Jacobi preconditioner, the PCG vectors,
// z, the duals and the penalties) live in shared memory (or, for problems too
// large for it, in a per-CTA slot of the workspace).  Per ADMM iteration:
//
//   rhs = sigma x - c + K^T (rho z - y)                       kernels.py:148
//   x~  = (diag(q) + sigma I + K^T diag(rho) K)^-1 rhs:
//         banded Cholesky solves (factor.py:66-105) when the plan has a band, else
//         cg_refinement_steps rounds of Jacobi PCG on the normalised correction
//         (kernels.py:152-171; fischer_burmeister/solver.py:213-310)
//   x+  = alpha x~ + (1 - alpha) x,  r = alpha K x~ + (1 - alpha) z,
//   z+  = clip(r + y / rho, lower, upper),  y+ = y + rho (r - z+)   kernels.py:172-176
//   every check_interval iterations and on the last: the linear, primal and dual
//   residuals and finiteness; acceptance freezes the sample (kernels.py:181-227);
//   adaptive rho at its interval (kernels.py:228-256).
//
// K x sums each row in CSR order and K^T y each column in ascending row order
// (the reference's scatter order); inner products and max-norms are block
// reductions, so results agree with the reference to rounding.
#include <cuda_runtime.h>

#include "common.cuh"
#include "cp_kernels.cuh"

namespace purin {

namespace {

// Threads per sample: one warp for small problems (every vector at most
// kAdmmWarpEntries long), whose reductions are shuffles behind a one-warp
// barrier and whose samples all fit on the GPU at once; 256 otherwise.
constexpr int kAdmmThreads = 256;
constexpr int kAdmmWarpEntries = 256;
constexpr size_t kAdmmStageBytes = 24u << 10;

// Block reduction of up to three values: sums of a and b, max of c.  Every
// thread receives the results.
template <typename T>
struct Red3 {
  T a, b, c;
};

template <int kWarps, typename T>
__device__ Red3<T> block_reduce3(T a, T b, T c, T (*scratch)[3]) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    a = a + shfl_xor(a, o);
    b = b + shfl_xor(b, o);
    c = pmax(c, shfl_xor(c, o));
  }
  __syncthreads();
  if ((threadIdx.x & 31) == 0) {
    scratch[threadIdx.x >> 5][0] = a;
    scratch[threadIdx.x >> 5][1] = b;
    scratch[threadIdx.x >> 5][2] = c;
  }
  __syncthreads();
  Red3<T> r{T(0), T(0), T(0)};
#pragma unroll
  for (int w = 0; w < kWarps; ++w) {
    r.a = r.a + scratch[w][0];
    r.b = r.b + scratch[w][1];
    r.c = pmax(r.c, scratch[w][2]);
  }
  __syncthreads();
  return r;
}

// One sample's operands.  The structure, values and per-sample vectors are read
// through these pointers: global memory, or copies in shared memory (staged).
template <typename T>
struct AdmmSample {
  const int* row_ptr;   // m + 1
  const int* col;       // nnz
  const int* col_ptr;   // n + 1
  const int* csc_row;   // nnz
  const int* csc_slot;  // nnz
  const T* vals;
  const T* q;
  const T* c;
  const T* lo;
  const T* up;
  int n, m, nnz;

  // out[i] = (K v)_i for rows i (CSR order).
  __device__ void mv(const T* v, T* out) const {
    for (int i = threadIdx.x; i < m; i += blockDim.x) {
      T acc = T(0);
      for (int k = row_ptr[i]; k < row_ptr[i + 1]; ++k) acc = acc + vals[k] * v[col[k]];
      out[i] = acc;
    }
    __syncthreads();
  }
  // out[j] = (K^T w)_j (ascending rows per column); with `square`, K's entries squared.
  __device__ void tmv(const T* w, T* out, bool square = false) const {
    for (int j = threadIdx.x; j < n; j += blockDim.x) {
      T acc = T(0);
      for (int e = col_ptr[j]; e < col_ptr[j + 1]; ++e) {
        const T v = vals[csc_slot[e]];
        acc = acc + (square ? v * v : v) * w[csc_row[e]];
      }
      out[j] = acc;
    }
    __syncthreads();
  }
};

// Elements of the staged copies: T values (vals, q, c, lo, up), then ints.
__host__ __device__ inline size_t admm_stage_values(int n, int m, int nnz) {
  return (size_t)nnz + 2 * (size_t)n + 2 * (size_t)m;
}
__host__ __device__ inline size_t admm_stage_ints(int n, int m, int nnz) {
  return (size_t)(m + 1) + (size_t)(n + 1) + 3 * (size_t)nnz;
}

// Copy the sample's operands into shared memory at `at` (after the state
// vectors) and point S at the copies: every product then gathers from shared
// memory instead of making dependent L2 round trips.
template <typename T>
__device__ void stage_sample(AdmmSample<T>& S, T* at) {
  const int n = S.n, m = S.m, nnz = S.nnz;
  T* vals = at;
  T* q = vals + nnz;
  T* c = q + n;
  T* lo = c + n;
  T* up = lo + m;
  int* ints = reinterpret_cast<int*>(up + m);
  int* row_ptr = ints;
  int* col = row_ptr + m + 1;
  int* col_ptr = col + nnz;
  int* csc_row = col_ptr + n + 1;
  int* csc_slot = csc_row + nnz;
  for (int k = threadIdx.x; k < nnz; k += blockDim.x) {
    vals[k] = S.vals[k];
    col[k] = S.col[k];
    csc_row[k] = S.csc_row[k];
    csc_slot[k] = S.csc_slot[k];
  }
  for (int j = threadIdx.x; j < n; j += blockDim.x) {
    q[j] = S.q[j];
    c[j] = S.c[j];
  }
  for (int i = threadIdx.x; i < m; i += blockDim.x) {
    lo[i] = S.lo[i];
    up[i] = S.up[i];
  }
  for (int i = threadIdx.x; i <= m; i += blockDim.x) row_ptr[i] = S.row_ptr[i];
  for (int j = threadIdx.x; j <= n; j += blockDim.x) col_ptr[j] = S.col_ptr[j];
  __syncthreads();
  S.vals = vals;
  S.q = q;
  S.c = c;
  S.lo = lo;
  S.up = up;
  S.row_ptr = row_ptr;
  S.col = col;
  S.col_ptr = col_ptr;
  S.csc_row = csc_row;
  S.csc_slot = csc_slot;
}

// Vectors of one CTA: 9 of length n, 5 of length m.
template <typename T>
struct AdmmState {
  T *x, *xt, *rhs, *diag, *sol, *r, *zc, *d, *img;  // n (r and zc adjacent: 2n of scratch)
  T *z, *dual, *pen, *tm, *ax;                       // m
};

template <typename T>
__device__ AdmmState<T> carve(T* base, int n, int m) {
  AdmmState<T> s;
  T* at = base;
  T** nv[9] = {&s.x, &s.xt, &s.rhs, &s.diag, &s.sol, &s.r, &s.zc, &s.d, &s.img};
  for (int k = 0; k < 9; ++k) {
    *nv[k] = at;
    at += n;
  }
  T** mv[5] = {&s.z, &s.dual, &s.pen, &s.tm, &s.ax};
  for (int k = 0; k < 5; ++k) {
    *mv[k] = at;
    at += m;
  }
  return s;
}

// out = (q + sigma) v + K^T (rho .* (K v)) (kernels.py:147); uses tm.
template <typename T>
__device__ void admm_op(const AdmmSample<T>& S, const AdmmState<T>& V, T sigma, const T* v, T* out) {
  S.mv(v, V.tm);
  for (int i = threadIdx.x; i < S.m; i += blockDim.x) V.tm[i] = V.pen[i] * V.tm[i];
  __syncthreads();
  S.tmv(V.tm, out);
  for (int j = threadIdx.x; j < S.n; j += blockDim.x) out[j] = (S.q[j] + sigma) * v[j] + out[j];
  __syncthreads();
}

// The banded matrix's Cholesky factor (factor.py:28-64), by one thread.
template <typename T>
__device__ void band_factor(const AdmmParams<T>& p, const AdmmSample<T>& S, const T* pen, T* band,
                            T sigma) {
  if (threadIdx.x == 0) {
    const int n = S.n, w = p.width, ld = w + 1;
    for (int e = 0; e < n * ld; ++e) band[e] = T(0);
    for (int k = 0; k < p.nband; ++k)
      band[p.band_dest[k]] =
          band[p.band_dest[k]] + pen[p.band_rows[k]] * S.vals[p.band_slot_l[k]] * S.vals[p.band_slot_r[k]];
    for (int i = 0; i < n; ++i) band[i * ld] = band[i * ld] + (S.q[p.band_perm[i]] + sigma);
    for (int j = 0; j < n; ++j) {
      T ss = T(0);
      for (int o = 1; o <= w; ++o)
        if (j - o >= 0) ss = ss + band[j * ld + o] * band[j * ld + o];
      const T pivot = sqrt(band[j * ld] - ss);
      band[j * ld] = pivot;
      for (int d = 1; d <= w && j + d < n; ++d) {
        const int i = j + d;
        T acc = T(0);
        for (int o = 1; o <= w; ++o) {
          const int ds = o + d;
          if (j - o >= 0 && ds <= w) acc = acc + band[i * ld + ds] * band[j * ld + o];
        }
        band[i * ld + d] = (band[i * ld + d] - acc) / pivot;
      }
    }
  }
  __syncthreads();
}

// x = A^-1 b with the banded factor (factor.py:66-105), by one thread; y: 2n scratch.
template <typename T>
__device__ void band_solve(const AdmmParams<T>& p, int n, const T* band, const T* b, T* y, T* x) {
  if (threadIdx.x == 0) {
    const int w = p.width, ld = w + 1;
    for (int i = 0; i < n; ++i) {
      T dot = T(0);
      for (int o = 1; o <= w; ++o)
        if (i >= o) dot = dot + band[i * ld + o] * y[i - o];
      y[i] = (b[p.band_perm[i]] - dot) / band[i * ld];
    }
    for (int k = 0; k < n; ++k) {
      const int i = n - 1 - k;
      T dot = T(0);
      for (int o = 1; o <= w; ++o)
        if (i + o < n) dot = dot + band[(i + o) * ld + o] * y[n + i + o];
      y[n + i] = (y[i] - dot) / band[i * ld];
    }
    for (int i = 0; i < n; ++i) x[i] = y[n + p.band_inv[i]];
  }
  __syncthreads();
}

template <typename T, bool kSmem, int NT, bool kStage>
__global__ void __launch_bounds__(NT) admm_forward_kernel(const AdmmParams<T> p) {
  constexpr int kWarps = NT / 32;
  extern __shared__ __align__(16) unsigned char dyn[];
  __shared__ T red[kWarps][3];
  const int64_t X = blockIdx.x;
  if (X >= p.batch) return;
  const DevStructure& st = p.st;
  const int n = st.n, m = st.m;
  AdmmSample<T> S;
  S.row_ptr = st.row_ptr;
  S.col = st.col;
  S.col_ptr = st.col_ptr;
  S.csc_row = st.csc_row;
  S.csc_slot = st.csc_slot;
  S.nnz = st.nnz;
  S.vals = p.values + X * p.values_stride;
  S.q = p.q + X * n;
  S.c = p.c + X * n;
  S.lo = p.lower + X * m;
  S.up = p.upper + X * m;
  S.n = n;
  S.m = m;
  const size_t elems = 9 * (size_t)n + 5 * (size_t)m;
  T* base = kSmem ? reinterpret_cast<T*>(dyn) : p.gstate + X * elems;
  const AdmmState<T> V = carve(base, n, m);
  if constexpr (kStage) stage_sample(S, reinterpret_cast<T*>(dyn) + elems);
  const T zero = T(0), one = T(1);
  const T sigma = p.sigma, alpha = p.alpha;
  const T tol = p.tolerance[X];
  const T inf = T(INFINITY);
  const T tiny = sizeof(T) == 8 ? T(2.2250738585072014e-308) : T(1.17549435e-38);
  const T eps = sizeof(T) == 8 ? T(2.220446049250313e-16) : T(1.1920929e-07);
  T* band = p.width >= 0 ? p.band + X * (size_t)n * (p.width + 1) : nullptr;

  // ---- initial state (kernels.py:103-123): z = clip(K x0), diag, factor ------
  for (int j = threadIdx.x; j < n; j += blockDim.x) V.x[j] = p.x0[X * n + j];
  for (int i = threadIdx.x; i < m; i += blockDim.x) {
    V.pen[i] = p.penalty0[X * m + i];
    V.dual[i] = p.dual0 ? p.dual0[X * m + i] : zero;
  }
  __syncthreads();
  S.mv(V.x, V.z);
  for (int i = threadIdx.x; i < m; i += blockDim.x) V.z[i] = clip(V.z[i], S.lo[i], S.up[i]);
  S.tmv(V.pen, V.diag, true);
  for (int j = threadIdx.x; j < n; j += blockDim.x) V.diag[j] = S.q[j] + sigma + V.diag[j];
  __syncthreads();
  if (band) band_factor(p, S, V.pen, band, sigma);

  int count = 0, inner = 0;
  bool done = false, failed = false;
  T last_linear = inf;
  for (int it = 0; it < p.max_iterations && !(done || failed); ++it) {
    // rhs = sigma x - c + K^T (rho z - y)                              kernels.py:148
    for (int i = threadIdx.x; i < m; i += blockDim.x) V.tm[i] = V.pen[i] * V.z[i] - V.dual[i];
    __syncthreads();
    S.tmv(V.tm, V.rhs);
    for (int j = threadIdx.x; j < n; j += blockDim.x) V.rhs[j] = sigma * V.x[j] - S.c[j] + V.rhs[j];
    __syncthreads();
    int lin_count = 0;
    if (band) {
      band_solve(p, n, band, V.rhs, V.r, V.xt);
    } else {
      for (int j = threadIdx.x; j < n; j += blockDim.x) V.xt[j] = V.x[j];
      __syncthreads();
      for (int step = 0; step < p.refinement_steps; ++step) {
        // Normalised correction b = (rhs - op(xt)) / max|.| (kernels.py:159-165).
        admm_op(S, V, sigma, V.xt, V.img);
        T cmax = zero;
        for (int j = threadIdx.x; j < n; j += blockDim.x) {
          const T corr = V.rhs[j] - V.img[j];
          V.r[j] = corr;
          cmax = pmax(cmax, fabs(corr));
        }
        const T magnitude = pmax(block_reduce3<kWarps>(zero, zero, cmax, red).c, tiny);
        // PCG from zero (fischer_burmeister/solver.py:213-310): the residual of the
        // zero start is b itself (op(0) is an exact zero).
        T rz_part = zero, rmax0 = zero;
        int bad = 0;
        for (int j = threadIdx.x; j < n; j += blockDim.x) {
          const T rj = V.r[j] / magnitude;
          const T zj = rj / V.diag[j];
          V.r[j] = rj;
          V.zc[j] = zj;
          V.d[j] = zj;
          V.sol[j] = zero;
          rz_part = rz_part + rj * zj;
          rmax0 = pmax(rmax0, fabs(rj));
          bad |= (finite(rj) && finite(zj)) ? 0 : 1;
        }
        const Red3<T> r0 = block_reduce3<kWarps>(rz_part, T(bad), rmax0, red);
        T rz = r0.a;
        const T threshold = pmax(p.cg_tolerance, p.cg_tolerance * r0.c);
        bool active = r0.b == zero && finite(rz) && r0.c > threshold;
        int its = 0;
        for (int k = 0; k < p.cg_iterations && active; ++k) {
          admm_op(S, V, sigma, V.d, V.img);
          T cpart = zero;
          for (int j = threadIdx.x; j < n; j += blockDim.x) cpart = cpart + V.d[j] * V.img[j];
          const T curvature = block_reduce3<kWarps>(cpart, zero, zero, red).a;
          const bool positive = curvature > eps;
          const T step_len = rz / (positive ? curvature : one);
          T nrz = zero, rmax = zero;
          int nbad = 0;
          for (int j = threadIdx.x; j < n; j += blockDim.x) {
            const T xs = V.sol[j] + step_len * V.d[j];
            const T rj = V.r[j] - step_len * V.img[j];
            const T zj = rj / V.diag[j];
            V.sol[j] = xs;
            V.r[j] = rj;
            V.zc[j] = zj;
            nrz = nrz + rj * zj;
            rmax = pmax(rmax, fabs(rj));
            nbad |= (finite(xs) && finite(rj) && finite(zj)) ? 0 : 1;
          }
          const Red3<T> rr = block_reduce3<kWarps>(nrz, T(nbad), rmax, red);
          const T beta = rr.a / (fabs(rz) > eps ? rz : one);
          for (int j = threadIdx.x; j < n; j += blockDim.x) V.d[j] = V.zc[j] + beta * V.d[j];
          __syncthreads();
          const bool fin = rr.b == zero && finite(rr.a) && positive;
          rz = rr.a;
          ++its;
          active = fin && rr.c > threshold;
        }
        for (int j = threadIdx.x; j < n; j += blockDim.x) V.xt[j] = V.xt[j] + magnitude * V.sol[j];
        __syncthreads();
        lin_count += its;
      }
    }
    // Relaxed updates (kernels.py:172-176).
    S.mv(V.xt, V.ax);
    const bool checking = ((it + 1) % p.check_interval == 0) || (it + 1 == p.max_iterations) ||
                          (p.adaptive_rho && (it + 1) % p.rho_update_interval == 0);
    T linear = last_linear;
    if (checking) {
      // linear = max|rhs - ((q + sigma) xt + K^T (rho ax))|           kernels.py:183
      for (int i = threadIdx.x; i < m; i += blockDim.x) V.tm[i] = V.pen[i] * V.ax[i];
      __syncthreads();
      S.tmv(V.tm, V.img);
      T lmax = zero;
      for (int j = threadIdx.x; j < n; j += blockDim.x)
        lmax = pmax(lmax, fabs(V.rhs[j] - ((S.q[j] + sigma) * V.xt[j] + V.img[j])));
      linear = block_reduce3<kWarps>(zero, zero, lmax, red).c;
    }
    for (int j = threadIdx.x; j < n; j += blockDim.x) V.x[j] = alpha * V.xt[j] + (one - alpha) * V.x[j];
    for (int i = threadIdx.x; i < m; i += blockDim.x) {
      const T relaxed = alpha * V.ax[i] + (one - alpha) * V.z[i];
      const T nz = clip(relaxed + V.dual[i] / V.pen[i], S.lo[i], S.up[i]);
      V.dual[i] = V.dual[i] + V.pen[i] * (relaxed - nz);
      V.z[i] = nz;
    }
    __syncthreads();
    T primal = inf, dual_res = inf;
    bool fin = true;
    if (checking) {
      // primal = max|K x - z|, dual = max|q x + c + K^T y|; finiteness   kernels.py:184-193
      S.mv(V.x, V.tm);
      S.tmv(V.dual, V.img);
      T pmax_ = zero, dmax = zero;
      int bad = 0;
      for (int i = threadIdx.x; i < m; i += blockDim.x) {
        pmax_ = pmax(pmax_, fabs(V.tm[i] - V.z[i]));
        bad |= finite(V.dual[i]) ? 0 : 1;
      }
      for (int j = threadIdx.x; j < n; j += blockDim.x) {
        dmax = pmax(dmax, fabs(S.q[j] * V.x[j] + S.c[j] + V.img[j]));
        bad |= finite(V.x[j]) ? 0 : 1;
      }
      const Red3<T> a = block_reduce3<kWarps>(T(bad), zero, pmax_, red);
      const Red3<T> b = block_reduce3<kWarps>(zero, zero, dmax, red);
      primal = a.c;
      dual_res = b.c;
      fin = a.a == zero && finite(linear) && finite(primal) && finite(dual_res);
    }
    const bool accepted = checking && fin && primal <= tol && dual_res <= tol && linear <= tol;
    ++count;
    inner += lin_count;
    if (checking) last_linear = linear;
    done = done || accepted;
    failed = failed || (checking && !fin);
    if (p.adaptive_rho && (it + 1) % p.rho_update_interval == 0) {
      // OSQP residual balancing (kernels.py:228-256); K x and K^T y are in tm and img.
      T kx = zero, zm = zero, qx = zero, ky = zero, cm = zero;
      for (int i = threadIdx.x; i < m; i += blockDim.x) {
        kx = pmax(kx, fabs(V.tm[i]));
        zm = pmax(zm, fabs(V.z[i]));
      }
      for (int j = threadIdx.x; j < n; j += blockDim.x) {
        qx = pmax(qx, fabs(S.q[j] * V.x[j]));
        ky = pmax(ky, fabs(V.img[j]));
        cm = pmax(cm, fabs(S.c[j]));
      }
      const T kxm = block_reduce3<kWarps>(zero, zero, kx, red).c;
      const T zmm = block_reduce3<kWarps>(zero, zero, zm, red).c;
      const T qxm = block_reduce3<kWarps>(zero, zero, qx, red).c;
      const T kym = block_reduce3<kWarps>(zero, zero, ky, red).c;
      const T cmm = block_reduce3<kWarps>(zero, zero, cm, red).c;
      const T pscale = pmax(pmax(kxm, zmm), T(1e-12));
      const T dscale = pmax(pmax(qxm, kym), pmax(cmm, T(1e-12)));
      const T rf = sqrt((primal / pscale + T(1e-16)) / (dual_res / dscale + T(1e-16)));
      const T thr = p.rho_update_threshold;
      const bool change = !done && fin && (rf >= thr || rf <= one / thr);
      if (change) {
        for (int i = threadIdx.x; i < m; i += blockDim.x)
          V.pen[i] = clip(V.pen[i] * rf, T(1e-6), T(1e6));
        __syncthreads();
        S.tmv(V.pen, V.diag, true);
        for (int j = threadIdx.x; j < n; j += blockDim.x) V.diag[j] = S.q[j] + sigma + V.diag[j];
        __syncthreads();
        if (band) band_factor(p, S, V.pen, band, sigma);
      }
    }
  }

  // ---- final diagnostics and outputs (kernels.py:268-283) -------------------
  S.mv(V.x, V.tm);
  S.tmv(V.dual, V.img);
  T pmax_ = zero, dmax = zero;
  int bad = 0;
  for (int i = threadIdx.x; i < m; i += blockDim.x) {
    pmax_ = pmax(pmax_, fabs(V.tm[i] - V.z[i]));
    bad |= finite(V.dual[i]) ? 0 : 1;
  }
  for (int j = threadIdx.x; j < n; j += blockDim.x) {
    dmax = pmax(dmax, fabs(S.q[j] * V.x[j] + S.c[j] + V.img[j]));
    bad |= finite(V.x[j]) ? 0 : 1;
  }
  const Red3<T> a = block_reduce3<kWarps>(T(bad), zero, pmax_, red);
  const Red3<T> b = block_reduce3<kWarps>(zero, zero, dmax, red);
  for (int j = threadIdx.x; j < n; j += blockDim.x) p.x[X * n + j] = V.x[j];
  for (int i = threadIdx.x; i < m; i += blockDim.x) {
    p.z[X * m + i] = V.z[i];
    p.dual[X * m + i] = V.dual[i];
    p.penalty[X * m + i] = V.pen[i];
  }
  if (threadIdx.x == 0) {
    const T primal = a.c, dual_res = b.c;
    const bool fin = a.a == zero && finite(primal) && finite(dual_res) && finite(last_linear);
    p.iterations[X] = count;
    p.inner_iterations[X] = inner;
    p.primal_residual[X] = primal;
    p.dual_residual[X] = dual_res;
    p.linear_residual[X] = last_linear;
    p.finite[X] = fin ? 1 : 0;
    p.converged[X] = (fin && primal <= tol && dual_res <= tol && last_linear <= tol) ? 1 : 0;
  }
}

}  // namespace

template <typename T>
size_t admm_state_elems(int n, int m) {
  return 9 * (size_t)n + 5 * (size_t)m;
}

template <typename T>
cudaError_t launch_admm(const AdmmParams<T>& p, bool smem, cudaStream_t stream) {
  if (p.batch <= 0) return cudaSuccess;
  const size_t bytes = admm_state_elems<T>(p.st.n, p.st.m) * sizeof(T);
  const int n = p.st.n, m = p.st.m, nnz = p.st.nnz;
  const bool warp = n <= kAdmmWarpEntries && m <= kAdmmWarpEntries;
  // Small problems also stage their operands in shared memory when state and
  // copies together stay within kAdmmStageBytes (about ten samples per SM).
  const size_t staged = bytes + admm_stage_values(n, m, nnz) * sizeof(T) +
                        admm_stage_ints(n, m, nnz) * sizeof(int);
  if (smem && warp && staged <= kAdmmStageBytes) {
    auto kern = admm_forward_kernel<T, true, 32, true>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)staged);
    if (e != cudaSuccess) return e;
    kern<<<(unsigned)p.batch, 32, staged, stream>>>(p);
  } else if (smem) {
    auto kern = warp ? admm_forward_kernel<T, true, 32, false> : admm_forward_kernel<T, true, kAdmmThreads, false>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
    if (e != cudaSuccess) return e;
    kern<<<(unsigned)p.batch, warp ? 32 : kAdmmThreads, bytes, stream>>>(p);
  } else if (warp) {
    admm_forward_kernel<T, false, 32, false><<<(unsigned)p.batch, 32, 0, stream>>>(p);
  } else {
    admm_forward_kernel<T, false, kAdmmThreads, false><<<(unsigned)p.batch, kAdmmThreads, 0, stream>>>(p);
  }
  return cudaGetLastError();
}

template size_t admm_state_elems<double>(int, int);
template size_t admm_state_elems<float>(int, int);
template cudaError_t launch_admm<double>(const AdmmParams<double>&, bool, cudaStream_t);
template cudaError_t launch_admm<float>(const AdmmParams<float>&, bool, cudaStream_t);

}  // namespace purin
