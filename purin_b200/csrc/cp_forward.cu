// Forward CP solve: sparse_cp (src/purin/solvers/chambolle_pock/kernels.py:178-305)
// with q = 1, c = -target, y0 = target, freeze_converged and check_stationarity on,
// as called by BoundProjection (bounds.py:42-66) and the unbounded layer
// (solver.py:149-176).
//
// One CTA owns a tile of S samples for the whole solve.  The tile's iterates
// y, ybar (n each) and the duals (m) live in shared memory, interleaved by
// sample ([element * S + s]) so that a group of S lanes reading one sparse
// entry (index + value) serves all S samples with a single structure load.
// The structure is read in the sliced-ELL layout of sell.cuh: a warp owns a
// slice of C = 32 / S rows (or columns) and reads C consecutive entries per
// step.  Each iteration makes three passes:
//   A (rows)    lambda+ = proj(lambda + sigma (K ybar - rhs))         kernels.py:133-137
//   B (columns) t = K.T lambda+, y+ = clip(a y - d t + o), ybar+,
//               bound violation, primal/dual objective terms, stationarity
//                                                                     kernels.py:138-150,153-175,272-274
//   C (rows)    K y+ - rhs for the equality/inequality residuals      kernels.py:155-157
// followed by a per-sample reduction and the accept/freeze decision
// (kernels.py:262-283).  A frozen sample never changes again, so the tile
// exits as soon as all its samples are accepted; iterations and results are
// those of the reference's batch-wide loop.
#include <cuda_runtime.h>

#include "common.cuh"
#include "cp_kernels.cuh"

namespace purin {

namespace {

constexpr int kThreads = 512;
constexpr int kWarps = kThreads / 32;

template <typename T, int S>
struct TileScratch {
  T tau[S], sigma[S], theta[S], a[S], d[S], tol[S];
  T res_out[S], gap_out[S];
  int active[S], count[S], conv[S];
  T red[kWarps][S][5];
  int redf[kWarps][S];
};

// Per-sample sum / max over the tile (every thread of sample s receives the total).
template <typename T, int S>
__device__ __forceinline__ T tile_sum(T v, T* scratch) {
  v = group_sum<S>(v);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  __syncthreads();
  if (lane < S) scratch[warp * S + lane] = v;
  __syncthreads();
  const int s = threadIdx.x % S;
  T total = T(0);
#pragma unroll
  for (int w = 0; w < kWarps; ++w) total = total + scratch[w * S + s];
  return total;
}
template <typename T, int S>
__device__ __forceinline__ T tile_max(T v, T* scratch) {
  v = group_max<S>(v);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  __syncthreads();
  if (lane < S) scratch[warp * S + lane] = v;
  __syncthreads();
  const int s = threadIdx.x % S;
  T total = T(0);
#pragma unroll
  for (int w = 0; w < kWarps; ++w) total = pmax(total, scratch[w * S + s]);
  return total;
}

// Sliced-ELL dot products of one lane group: sum_k value(e) * x[index(e) * S + s].
template <typename T, int S, bool kShared>
struct SellDot {
  const int* idx;
  const int* slot;
  const T* sell_vals;  // kShared: values in SELL order
  const T* vals;       // !kShared: this sample's values in CSR slot order

  __device__ __forceinline__ T value(int e) const {
    if constexpr (kShared) {
      return __ldg(sell_vals + e);
    } else {
      const int sl = __ldg(slot + e);
      return sl >= 0 ? vals[sl] : T(0);
    }
  }
  __device__ __forceinline__ T dot(int e0, int width, const T* x, int s) const {
    constexpr int C = 32 / S;
    T acc = T(0);
    int e = e0;
#pragma unroll 4
    for (int k = 0; k < width; ++k, e += C) acc = acc + value(e) * x[(size_t)__ldg(idx + e) * S + s];
    return acc;
  }
  __device__ __forceinline__ T abs_sum(int e0, int width) const {
    constexpr int C = 32 / S;
    T acc = T(0);
    int e = e0;
#pragma unroll 4
    for (int k = 0; k < width; ++k, e += C) acc = acc + fabs(value(e)) * T(1);
    return acc;
  }
};

template <typename T, int S, bool kSmem, bool kShared>
__global__ void __launch_bounds__(kThreads, 1)
cp_forward_kernel(const FwdParams<T> p) {
  extern __shared__ __align__(16) unsigned char dyn_smem[];
  __shared__ TileScratch<T, S> sc;
  __shared__ T s_scratch[kWarps * S];
  constexpr int C = 32 / S;

  const DevStructure& st = p.st;
  const SellView& sv = p.sell;
  const int n = st.n, m = st.m, me = st.me;
  const int tid = threadIdx.x;
  const int lane = tid & 31, warp = tid >> 5;
  const int s = tid % S;
  const int g = tid / S;
  const int gw = lane / S;  // lane group within the warp: position in a slice
  constexpr int G = kThreads / S;
  const int64_t b_raw = (int64_t)blockIdx.x * S + s;
  const bool valid = b_raw < p.batch;
  const int64_t b = valid ? b_raw : (p.batch - 1);

  const size_t tile_elems = (size_t)(2 * (n + 1) + (m + 1) + (p.diag ? 2 * (n + 1) + (m + 1) : 0)) * S;
  T* base = kSmem ? reinterpret_cast<T*>(dyn_smem) : p.gstate + (size_t)blockIdx.x * tile_elems;
  T* y = base;
  T* ybar = y + (size_t)(n + 1) * S;
  T* lam = ybar + (size_t)(n + 1) * S;
  T* av = lam + (size_t)(m + 1) * S;  // diagonal steps (only when p.diag)
  T* dv = av + (size_t)(n + 1) * S;
  T* sv_ = dv + (size_t)(n + 1) * S;

  const T* vals = p.values + b * p.values_stride;
  const SellDot<T, S, kShared> rows{sv.r_idx, sv.r_slot, p.vr, vals};
  const SellDot<T, S, kShared> cols{sv.c_idx, sv.c_slot, p.vc, vals};
  const T* tgt = p.target + b * n;
  const T* rhs = p.rhs + b * m;
  const T* lo = p.lower + b * p.bounds_stride;
  const T* up = p.upper + b * p.bounds_stride;
  const T zero = T(0), one = T(1);
  const T safety = p.safety;

  // Padding elements of the gathered vectors are zero for the whole solve.
  if (tid < S) {
    y[(size_t)n * S + s] = zero;
    ybar[(size_t)n * S + s] = zero;
    lam[(size_t)m * S + s] = zero;
  }

  // ---- step sizes (kernels.py:209-227) ------------------------------------
  T L = one;
  if (p.diag) {
    // diagonal_step_sizes (kernels.py:76-88): |K| row and column sums.
    for (int sl = warp; sl < sv.nsl_r; sl += kWarps) {
      const int i = __ldg(sv.r_perm + sl * C + gw);
      const int e0 = __ldg(sv.r_ptr + sl);
      const T acc = rows.abs_sum(e0 + gw, (__ldg(sv.r_ptr + sl + 1) - e0) / C);
      if (i >= 0) {
        const T r = acc > zero ? pmax(acc, T(1e-12)) : one;
        sv_[(size_t)i * S + s] = safety / r;
      }
    }
    for (int sl = warp; sl < sv.nsl_c; sl += kWarps) {
      const int j = __ldg(sv.c_perm + sl * C + gw);
      const int e0 = __ldg(sv.c_ptr + sl);
      const T acc = cols.abs_sum(e0 + gw, (__ldg(sv.c_ptr + sl + 1) - e0) / C);
      if (j >= 0) {
        const T c = acc > zero ? pmax(acc, T(1e-12)) : one;
        const T tau = safety / c;
        const T a = one / (one + tau * one);
        av[(size_t)j * S + s] = a;
        dv[(size_t)j * S + s] = tau * a;
      }
    }
  } else if (p.norm_bound) {
    T rmax = zero, cmax = zero;
    for (int sl = warp; sl < sv.nsl_r; sl += kWarps) {
      const int e0 = __ldg(sv.r_ptr + sl);
      rmax = pmax(rmax, rows.abs_sum(e0 + gw, (__ldg(sv.r_ptr + sl + 1) - e0) / C));
    }
    for (int sl = warp; sl < sv.nsl_c; sl += kWarps) {
      const int e0 = __ldg(sv.c_ptr + sl);
      cmax = pmax(cmax, cols.abs_sum(e0 + gw, (__ldg(sv.c_ptr + sl + 1) - e0) / C));
    }
    rmax = tile_max<T, S>(rmax, s_scratch);
    cmax = tile_max<T, S>(cmax, s_scratch);
    L = pmax(sqrt(rmax * cmax), T(1e-12));
  } else {
    // norm_estimate (kernels.py:52-65): power iteration on K.T K.
    uint32_t k0, k1;
    split_key(p.norm_seed, p.sample_offset + b, p.total_batch, p.partitionable != 0, k0, k1);
    T* x = y;      // n (+ zero pad)
    T* u = lam;    // m (+ zero pad)
    T* z = ybar;   // n
    T ss = zero;
    for (int j = g; j < n; j += G) {
      const T v = NormalBits<T>::draw(k0, k1, j, n, p.partitionable != 0);
      x[(size_t)j * S + s] = v;
      ss = ss + v * v;
    }
    const T nrm = sqrt(tile_sum<T, S>(ss, s_scratch)) + T(1e-12);
    for (int j = g; j < n; j += G) x[(size_t)j * S + s] = x[(size_t)j * S + s] / nrm;
    T eig = zero;
    for (int it = 0; it < p.norm_iterations; ++it) {
      __syncthreads();
      for (int sl = warp; sl < sv.nsl_r; sl += kWarps) {
        const int i = __ldg(sv.r_perm + sl * C + gw);
        const int e0 = __ldg(sv.r_ptr + sl);
        const T acc = rows.dot(e0 + gw, (__ldg(sv.r_ptr + sl + 1) - e0) / C, x, s);
        if (i >= 0) u[(size_t)i * S + s] = acc;
      }
      __syncthreads();
      T xz = zero, zz = zero;
      for (int sl = warp; sl < sv.nsl_c; sl += kWarps) {
        const int j = __ldg(sv.c_perm + sl * C + gw);
        const int e0 = __ldg(sv.c_ptr + sl);
        const T acc = cols.dot(e0 + gw, (__ldg(sv.c_ptr + sl + 1) - e0) / C, u, s);
        if (j >= 0) {
          z[(size_t)j * S + s] = acc;
          xz = xz + x[(size_t)j * S + s] * acc;
          zz = zz + acc * acc;
        }
      }
      eig = tile_sum<T, S>(xz, s_scratch);
      const T zn = sqrt(tile_sum<T, S>(zz, s_scratch)) + T(1e-12);
      for (int j = g; j < n; j += G) x[(size_t)j * S + s] = z[(size_t)j * S + s] / zn;
    }
    L = pmax(sqrt(pmax(eig, zero)) + T(1e-12), T(1e-12));
    __syncthreads();
  }

  // ---- initial state: y = ybar = target, lambda = dual0 --------------------
  for (int j = g; j < n; j += G) {
    const T t = tgt[j];
    y[(size_t)j * S + s] = t;
    ybar[(size_t)j * S + s] = t;
  }
  for (int i = g; i < m; i += G) lam[(size_t)i * S + s] = p.dual0 ? p.dual0[b * m + i] : zero;
  if (tid < S) {
    y[(size_t)n * S + s] = zero;
    ybar[(size_t)n * S + s] = zero;
    lam[(size_t)m * S + s] = zero;
    const T tau = p.accelerated ? safety / L : safety / (one + L);
    sc.tau[s] = tau;
    sc.sigma[s] = safety / L;
    sc.theta[s] = one;
    sc.a[s] = one / (one + tau * one);
    sc.d[s] = tau * sc.a[s];
    sc.tol[s] = p.tol[b];
    sc.active[s] = valid ? 1 : 0;
    sc.count[s] = 0;
    sc.conv[s] = 0;
    sc.res_out[s] = zero;
    sc.gap_out[s] = zero;
  }
  __syncthreads();

  for (int it = 0; it < p.max_iterations; ++it) {
    int any = 0;
#pragma unroll
    for (int q = 0; q < S; ++q) any |= sc.active[q];
    if (!any) break;
    const bool act = sc.active[s] != 0;
    const T sigma = sc.sigma[s];
    const T a = sc.a[s], d = sc.d[s], theta = sc.theta[s];
    int fin = 1;
    T rd = zero;
    // Phase A: dual update.
    for (int sl = warp; sl < sv.nsl_r; sl += kWarps) {
      const int i = __ldg(sv.r_perm + sl * C + gw);
      const int e0 = __ldg(sv.r_ptr + sl);
      const T acc = rows.dot(e0 + gw, (__ldg(sv.r_ptr + sl + 1) - e0) / C, ybar, s);
      if (i >= 0 && act) {
        const T sg = p.diag ? sv_[(size_t)i * S + s] : sigma;
        const T rb = rhs[i];
        const T raw = lam[(size_t)i * S + s] + sg * (acc - rb);
        const T nl = i < me ? raw : pmax(raw, zero);
        lam[(size_t)i * S + s] = nl;
        fin &= finite(nl) ? 1 : 0;
        rd = rd + rb * nl;
      }
    }
    __syncthreads();
    // Phase B: primal update and column diagnostics.
    T resm = zero, stm = zero, ps = zero, ds = zero;
    for (int sl = warp; sl < sv.nsl_c; sl += kWarps) {
      const int j = __ldg(sv.c_perm + sl * C + gw);
      const int e0 = __ldg(sv.c_ptr + sl);
      const T t = cols.dot(e0 + gw, (__ldg(sv.c_ptr + sl + 1) - e0) / C, lam, s);
      if (j >= 0 && act) {
        const size_t js = (size_t)j * S + s;
        const T yo = y[js];
        const T c = -tgt[j];
        const T aa = p.diag ? av[js] : a;
        const T dd = p.diag ? dv[js] : d;
        const T off = (-dd) * c;
        const T yr = (aa * yo - dd * t) + off;
        const T l = lo[j], u = up[j];
        const T yn = clip(yr, l, u);
        y[js] = yn;
        ybar[js] = yn + theta * (yn - yo);
        fin &= finite(yn) ? 1 : 0;
        resm = pmax(resm, pmax(pmax(l - yn, zero), pmax(yn - u, zero)));
        ps = ps + ((T(0.5) * one * yn) * yn + c * yn);
        const T tt = c + t;
        const T mn = clip(-tt / one, l, u);
        ds = ds + (T(0.5) * one * (mn * mn) + tt * mn);
        const T inner = (one * yn + c) + t;
        stm = pmax(stm, fabs(yn - clip(yn - inner, l, u)));
      }
    }
    __syncthreads();
    // Phase C: constraint residuals of y+.
    for (int sl = warp; sl < sv.nsl_r; sl += kWarps) {
      const int i = __ldg(sv.r_perm + sl * C + gw);
      const int e0 = __ldg(sv.r_ptr + sl);
      const T acc = rows.dot(e0 + gw, (__ldg(sv.r_ptr + sl + 1) - e0) / C, y, s);
      if (i >= 0 && act) {
        const T r = acc - rhs[i];
        resm = pmax(resm, i < me ? fabs(r) : pmax(r, zero));
      }
    }
    // Per-sample reduction.
    resm = group_max<S>(resm);
    stm = group_max<S>(stm);
    ps = group_sum<S>(ps);
    ds = group_sum<S>(ds);
    rd = group_sum<S>(rd);
    fin = group_and<S>(fin);
    if (lane < S) {
      sc.red[warp][lane][0] = resm;
      sc.red[warp][lane][1] = stm;
      sc.red[warp][lane][2] = ps;
      sc.red[warp][lane][3] = ds;
      sc.red[warp][lane][4] = rd;
      sc.redf[warp][lane] = fin;
    }
    __syncthreads();
    if (tid < S) {
      T res = zero, stat = zero, P = zero, Dp = zero, Rd = zero;
      int f = 1;
#pragma unroll
      for (int w = 0; w < kWarps; ++w) {
        res = pmax(res, sc.red[w][tid][0]);
        stat = pmax(stat, sc.red[w][tid][1]);
        P = P + sc.red[w][tid][2];
        Dp = Dp + sc.red[w][tid][3];
        Rd = Rd + sc.red[w][tid][4];
        f &= sc.redf[w][tid];
      }
      const T D = Dp - Rd;
      const T gap = pmax(P - D, zero) / pmax(one, pmax(fabs(P), fabs(D)));
      const bool finite_all = f && finite(gap);
      const T tol = sc.tol[tid];
      const bool accepted = finite_all && res <= tol && gap <= tol && stat <= tol;
      if (sc.active[tid]) {
        sc.count[tid] += 1;
        sc.res_out[tid] = pmax(res, stat);
        sc.gap_out[tid] = gap;
        sc.conv[tid] = accepted ? 1 : 0;
        if (accepted) sc.active[tid] = 0;
      }
      if (p.accelerated) {
        const T tau = sc.tau[tid];
        const T nt = one / sqrt(one + one * tau);
        const T ntau = nt * tau;
        sc.tau[tid] = ntau;
        sc.sigma[tid] = sc.sigma[tid] / nt;
        sc.theta[tid] = nt;
        sc.a[tid] = one / (one + ntau * one);
        sc.d[tid] = ntau * sc.a[tid];
      }
    }
    __syncthreads();
  }

  // ---- outputs --------------------------------------------------------------
  if (valid) {
    for (int j = g; j < n; j += G) p.y_out[b * n + j] = y[(size_t)j * S + s];
    for (int i = g; i < m; i += G) p.dual_out[b * m + i] = lam[(size_t)i * S + s];
    if (g == 0) {
      p.it_out[b] = sc.count[s];
      p.res_out[b] = sc.res_out[s];
      p.gap_out[b] = sc.gap_out[s];
      const bool feas = p.feasible ? (p.feasible[b] != 0) : true;
      p.conv_out[b] = (sc.conv[s] && feas) ? 1 : 0;
    }
  }
}

// Shared values in SELL order: out[e] = values[slot[e]] (0 for padding).
template <typename T>
__global__ void arrange_values_kernel(const T* values, const int* slot, int count, T* out) {
  for (int e = blockIdx.x * blockDim.x + threadIdx.x; e < count; e += gridDim.x * blockDim.x) {
    const int sl = slot[e];
    out[e] = sl >= 0 ? values[sl] : T(0);
  }
}

template <typename T, int S, bool kShared>
cudaError_t launch_s(const FwdParams<T>& p, bool smem, size_t smem_bytes, cudaStream_t stream) {
  const unsigned grid = (unsigned)((p.batch + S - 1) / S);
  if (smem) {
    auto kern = cp_forward_kernel<T, S, true, kShared>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem_bytes);
    if (e != cudaSuccess) return e;
    kern<<<grid, kThreads, smem_bytes, stream>>>(p);
  } else {
    cp_forward_kernel<T, S, false, kShared><<<grid, kThreads, 0, stream>>>(p);
  }
  return cudaGetLastError();
}

template <typename T, bool kShared>
cudaError_t launch_shared(const FwdParams<T>& p, int S, bool smem, size_t smem_bytes,
                          cudaStream_t stream) {
  switch (S) {
    case 1: return launch_s<T, 1, kShared>(p, smem, smem_bytes, stream);
    case 2: return launch_s<T, 2, kShared>(p, smem, smem_bytes, stream);
    case 4: return launch_s<T, 4, kShared>(p, smem, smem_bytes, stream);
    case 8: return launch_s<T, 8, kShared>(p, smem, smem_bytes, stream);
    case 16: return launch_s<T, 16, kShared>(p, smem, smem_bytes, stream);
    case 32: return launch_s<T, 32, kShared>(p, smem, smem_bytes, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace

template <typename T>
size_t forward_static_smem(int S) {
  switch (S) {
    case 1: return sizeof(TileScratch<T, 1>) + kWarps * 1 * sizeof(T);
    case 2: return sizeof(TileScratch<T, 2>) + kWarps * 2 * sizeof(T);
    case 4: return sizeof(TileScratch<T, 4>) + kWarps * 4 * sizeof(T);
    case 8: return sizeof(TileScratch<T, 8>) + kWarps * 8 * sizeof(T);
    case 16: return sizeof(TileScratch<T, 16>) + kWarps * 16 * sizeof(T);
    default: return sizeof(TileScratch<T, 32>) + kWarps * 32 * sizeof(T);
  }
}

template <typename T>
cudaError_t arrange_values(const T* values, const int* slot, int count, T* out, cudaStream_t stream) {
  if (count <= 0) return cudaSuccess;
  const int threads = 256;
  const int blocks = (count + threads - 1) / threads < 1184 ? (count + threads - 1) / threads : 1184;
  arrange_values_kernel<T><<<blocks, threads, 0, stream>>>(values, slot, count, out);
  return cudaGetLastError();
}

template <typename T>
cudaError_t launch_forward(const FwdParams<T>& p, int S, bool smem, size_t smem_bytes,
                           cudaStream_t stream) {
  return p.vr ? launch_shared<T, true>(p, S, smem, smem_bytes, stream)
              : launch_shared<T, false>(p, S, smem, smem_bytes, stream);
}

template cudaError_t launch_forward<double>(const FwdParams<double>&, int, bool, size_t, cudaStream_t);
template cudaError_t launch_forward<float>(const FwdParams<float>&, int, bool, size_t, cudaStream_t);
template size_t forward_static_smem<double>(int);
template size_t forward_static_smem<float>(int);
template cudaError_t arrange_values<double>(const double*, const int*, int, double*, cudaStream_t);
template cudaError_t arrange_values<float>(const float*, const int*, int, float*, cudaStream_t);

}  // namespace purin
