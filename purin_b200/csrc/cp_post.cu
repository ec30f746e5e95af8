// Post-processing of a CP solve in the units of the public constraint rows:
// BoundProjection.solve, src/purin/solvers/chambolle_pock/bounds.py:247-305
// (and PreparedChambollePockProjection._solve, solver.py:333-355, which is the
// same computation without bound rows).
//
// One CTA per sample.  The recovered multipliers are written straight into the
// caller's multiplier arrays, which then serve as the dual vector of the final
// stationarity product.
#include <cuda_runtime.h>

#include "common.cuh"
#include "cp_kernels.cuh"

namespace purin {

namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;

template <typename T>
__device__ T block_max_post(T v, T* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = pmax(v, shfl_xor(v, o));
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  T total = T(0);
#pragma unroll
  for (int w = 0; w < kWarps; ++w) total = pmax(total, red[w]);
  __syncthreads();
  return total;
}

template <typename T>
__global__ void __launch_bounds__(kThreads) cp_post_kernel(const PostParams<T> p) {
  __shared__ T red[kWarps];
  const DevStructure& st = p.st;
  const int n = st.n, m = st.m, me = st.me, m_all = st.m_all;
  const int mi_all = m_all - me;
  const int64_t b = blockIdx.x;
  const T zero = T(0), one = T(1);
  const T* vals = p.values_all + b * p.values_stride;
  const T* rhs = p.rhs_all + b * m_all;
  const T* tgt = p.target + b * n;
  const T* lo = p.lower + b * p.bounds_stride;
  const T* up = p.upper + b * p.bounds_stride;
  const T* sc = p.scale + b * m;
  const T* y = p.y + b * n;
  const T* dual = p.dual + b * m;
  T* meq = p.meq + b * me;
  T* miq = p.miq + b * mi_all;
  auto dual_at = [&](int r) -> T& { return r < me ? meq[r] : miq[r - me]; };

  int fin = 1;
  // dual = zeros.at[:, rows].set(out.dual * scale)               bounds.py:247
  for (int i = threadIdx.x; i < m; i += kThreads) {
    const T v = dual[i] * sc[i];
    dual_at(st.kept_rows[i]) = v;
    fin &= finite(v) ? 1 : 0;
  }
  for (int k = threadIdx.x; k < st.n_bound; k += kThreads) dual_at(st.bound_rows[k]) = zero;
  __syncthreads();

  // Bound-row multipliers: split each bound's normal among tied rows (bounds.py:249-284).
  for (int k = threadIdx.x; k < st.n_bound; k += kThreads) {
    const int v = st.bound_var[k];
    const T coef = vals[st.bound_slot[k]];
    const int r = st.bound_rows[k];
    const T thr = rhs[r] / (coef != zero ? coef : one);
    const T lv = lo[v], uv = up[v], yv = y[v];
    const bool is_lower = coef < zero && thr == lv && yv == lv;
    const bool is_upper = coef > zero && thr == uv && yv == uv;
    T lower_count = zero, upper_count = zero;
    for (int q = st.var_bound_ptr[v]; q < st.var_bound_ptr[v + 1]; ++q) {
      const int k2 = st.var_bound_list[q];
      const T c2 = vals[st.bound_slot[k2]];
      const T t2 = rhs[st.bound_rows[k2]] / (c2 != zero ? c2 : one);
      lower_count = lower_count + ((c2 < zero && t2 == lv && yv == lv) ? one : zero);
      upper_count = upper_count + ((c2 > zero && t2 == uv && yv == uv) ? one : zero);
    }
    // base_stationarity[v] = y - target + K.T dual (bound rows still zero)
    T t = zero;
    for (int e = st.col_ptr[v]; e < st.col_ptr[v + 1]; ++e) {
      const int i = st.csc_row[e];
      t = t + vals[st.kept_slots[st.csc_slot[e]]] * (dual[i] * sc[i]);
    }
    const T normal = (yv - tgt[v]) + t;
    T bd = is_lower ? pmax(normal, zero) / pmax(lower_count, one) : zero;
    bd = bd + (is_upper ? pmax(-normal, zero) / pmax(upper_count, one) : zero);
    bd = bd / (coef != zero ? fabs(coef) : one);
    dual_at(r) = bd;
    fin &= finite(bd) ? 1 : 0;
  }
  __syncthreads();

  // r = K y - rhs on all public rows; residuals and slacks (bounds.py:285-289, 311).
  T res = zero;
  for (int i = threadIdx.x; i < m_all; i += kThreads) {
    T acc = zero;
    for (int k = st.row_ptr_all[i]; k < st.row_ptr_all[i + 1]; ++k) acc = acc + vals[k] * y[st.col_all[k]];
    const T r = acc - rhs[i];
    if (i < me) {
      res = pmax(res, fabs(r));
    } else {
      res = pmax(res, pmax(r, zero));
      p.slacks[b * mi_all + (i - me)] = pmax(-r, zero);
    }
  }
  // stationarity = max |y - target + K.T dual| (bounds.py:290)
  for (int j = threadIdx.x; j < n; j += kThreads) {
    T t = zero;
    for (int e = st.col_ptr_all[j]; e < st.col_ptr_all[j + 1]; ++e)
      t = t + vals[st.csc_slot_all[e]] * dual_at(st.csc_row_all[e]);
    res = pmax(res, fabs((y[j] - tgt[j]) + t));
    fin &= finite(y[j]) ? 1 : 0;
  }
  res = block_max_post(res, red);
  fin = __syncthreads_and(fin);
  if (threadIdx.x == 0) {
    const T gap = p.gap[b];
    const bool finite_all = fin && finite(res) && finite(gap);
    const bool converged = finite_all && p.cp_conv[b] && res <= p.tol;
    p.resid[b] = res;
    p.finite[b] = finite_all ? 1 : 0;
    p.elig[b] = converged ? 1 : 0;
    p.status[b] = converged ? 0 : (finite_all ? 1 : 3);
  }
}

}  // namespace

template <typename T>
cudaError_t launch_post(const PostParams<T>& p, cudaStream_t stream) {
  if (p.batch <= 0) return cudaSuccess;
  cp_post_kernel<T><<<(unsigned)p.batch, kThreads, 0, stream>>>(p);
  return cudaGetLastError();
}

template cudaError_t launch_post<double>(const PostParams<double>&, cudaStream_t);
template cudaError_t launch_post<float>(const PostParams<float>&, cudaStream_t);

}  // namespace purin
