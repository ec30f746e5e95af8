// Restarted GMRES cycles of the implicit VJP with each sample's Krylov basis held
// on chip, in the distributed shared memory of a thread-block cluster.
//
// The adjoint system (I - J^T) v = g of one sample (bounds.py:130-146) has W =
// 2n + m unknowns and its restarted GMRES (primal_dual_interior_point/
// operators.py:792-1125, CGS2 Arnoldi) keeps R + 1 basis vectors; the CGS2
// sweeps read them four times per Arnoldi step.  At benchmark sizes the basis
// (config 2: 31 x 5632 doubles = 1.4 MB) is far larger than one SM's shared
// memory, and the bases of every resident sample together exceed L2, so a
// CTA-per-sample kernel streams them from HBM.  Here a cluster of C CTAs (C = 1,
// 2, 4 or 8: the smallest whose slices fit) works on one sample: CTA r owns
// columns [r nc, (r + 1) nc) of the y and ybar blocks and rows [r mc, (r + 1) mc)
// of the dual block, i.e. a slice of every basis vector, which stays in its
// shared memory for the whole cycle.  What crosses CTAs goes through DSMEM:
//
//   * the pullback operator z <- z - J^T z: each CTA computes t = -d g_raw for
//     its columns and writes it into every CTA's replica of t (n values), then
//     its rows' sigma mu_raw into every replica of that (m values), so the
//     sparse gathers of both products read local shared memory;
//   * every dot product and norm: per-CTA partial sums are written into every
//     CTA's exchange slots and summed there in rank order, so all CTAs hold the
//     same bits and take the same decisions (the Givens rotations and the
//     stopping test run redundantly on each).
//
// Per Arnoldi step that is five cluster barriers and no HBM traffic beyond the
// structure and the per-sample step data (L2-resident).  Cycles run in lockstep
// over the batch exactly as in the CTA-per-sample kernel (cp_adjoint.cu): a
// bounded grid barrier after every cycle publishes its length and the count of
// samples still above threshold.  Staged mode (stage 2) runs one cycle for a
// host that combines the counters of several shards between cycles.  The
// prepare and finish phases (step sizes, linearisation, pullback) stay in
// cp_adjoint_kernel; they exchange the state through the workspace.
#include <cooperative_groups.h>
#include <cuda_runtime.h>

#include "adjoint_common.cuh"

namespace cg = cooperative_groups;

namespace purin {

namespace {

constexpr int kClusterThreads = 256;
// Register capacity of a thread's own operator row and column (entries beyond
// are read from the plan's arrays).
constexpr int kOwnRow = 8;
constexpr int kOwnCol = 12;

// Shared-memory layout of one CTA (elements of T, each region 16-byte aligned).
struct ClusterLayout {
  int nc, mc, lcap;  // column / row block per CTA, basis slice capacity 2 nc + mc
  size_t v, buf, tn, tm, hess, proj, cs, sn, coef, c2, bsv, dloc, part, red, total;
};

template <typename T>
__host__ __device__ inline ClusterLayout cluster_layout(int n, int m, int R, int C) {
  ClusterLayout L;
  L.nc = (n + C - 1) / C;
  L.mc = (m + C - 1) / C;
  L.lcap = 2 * L.nc + L.mc;
  const size_t a = 16 / sizeof(T);
  size_t at = 0;
  auto take = [&](size_t count) {
    const size_t o = at;
    at = (at + count + a - 1) / a * a;
    return o;
  };
  L.v = take((size_t)(R + 1) * L.lcap);
  L.buf = take(L.lcap);
  L.tn = take((size_t)n + 1);
  L.tm = take((size_t)m + 1);
  L.hess = take((size_t)(R + 1) * R);
  L.proj = take(R + 1);
  L.cs = take(R);
  L.sn = take(R);
  L.coef = take(R + 1);
  L.c2 = take(R + 1);
  L.bsv = take(R);
  L.dloc = take(R + 2);
  L.part = take(2 * (size_t)C * (R + 2));  // two exchange buffers of C x (R + 2)
  L.red = take(kClusterThreads / 32);
  L.total = at;
  return L;
}

// One thread's own column (local index threadIdx.x) and row of the pullback
// operator, held in registers for a whole sample: the CSC entries (value, row)
// and the CSR entries (value, column) up to KC / KR of them, the column's
// derivative factor and proximal coefficients.
template <typename T, int KR, int KC>
struct OwnLines {
  T cv[KC];
  int cr[KC];
  int ccount;
  T rv[KR];
  int rc[KR];
  int rcount;
  T yfac, aa, dd;

  __device__ void load(const DevStructure& st, const Sample<T>& s, int c0, int ncl, int r0, int mcl) {
    const int t = threadIdx.x;
    ccount = 0;
    rcount = 0;
    yfac = aa = dd = T(0);
    if (t < ncl) {
      const int j = c0 + t;
      const int e0 = st.col_ptr[j], len = st.col_ptr[j + 1] - e0;
      ccount = len < KC ? len : KC;
#pragma unroll
      for (int q = 0; q < KC; ++q) {
        if (q < ccount) {
          cv[q] = s.vals[st.csc_slot[e0 + q]];
          cr[q] = st.csc_row[e0 + q];
        }
      }
      yfac = code_factor<T>(s.yc[j] & 3);
      aa = s.av ? s.av[j] : s.a;
      dd = s.dv ? s.dv[j] : s.d;
    }
    if (t < mcl) {
      const int i = r0 + t;
      const int k0 = st.row_ptr[i], len = st.row_ptr[i + 1] - k0;
      rcount = len < KR ? len : KR;
#pragma unroll
      for (int q = 0; q < KR; ++q) {
        if (q < rcount) {
          rv[q] = s.vals[k0 + q];
          rc[q] = st.col[k0 + q];
        }
      }
    }
  }
};

template <typename T, int C>
struct ClusterCtx {
  int rank;
  int n, m, me, W, R;
  int c0, ncl, r0, mcl, lv;  // own columns [c0, c0 + ncl), rows [r0, r0 + mcl), slice length
  int lcap;
  T* V;
  T* buf;
  T* tn;
  T* tm;
  T* part;
  T* red;
  int parity;

  // Global index (in the packed (y, dual, ybar) vector) of local slice entry l.
  __device__ __forceinline__ int global(int l) const {
    return l < ncl ? c0 + l : (l < ncl + mcl ? n + r0 + (l - ncl) : n + m + c0 + (l - ncl - mcl));
  }

  // out[0..k) = sum over the cluster's CTAs, in rank order, of each CTA's
  // part_local[0..k) (shared memory, complete before the call).  Every CTA gets
  // the same bits.  Ends with the CTA synchronised.
  __device__ void sum(const T* part_local, int k, T* out) {
    const int stride = R + 2;
    T* slots = part + (size_t)parity * C * stride;
    for (int t = threadIdx.x; t < C * k; t += blockDim.x) {
      const int dst = t / k, i = t - dst * k;
      T* remote = cg::this_cluster().map_shared_rank(slots, dst);
      remote[rank * stride + i] = part_local[i];
    }
    cg::this_cluster().sync();
    for (int i = threadIdx.x; i < k; i += blockDim.x) {
      T acc = T(0);
#pragma unroll
      for (int r = 0; r < C; ++r) acc = acc + slots[r * stride + i];
      out[i] = acc;
    }
    parity ^= 1;
    __syncthreads();
  }
  // The same with a max over the cluster (nonnegative values).
  __device__ void max(const T* part_local, int k, T* out) {
    const int stride = R + 2;
    T* slots = part + (size_t)parity * C * stride;
    for (int t = threadIdx.x; t < C * k; t += blockDim.x) {
      const int dst = t / k, i = t - dst * k;
      T* remote = cg::this_cluster().map_shared_rank(slots, dst);
      remote[rank * stride + i] = part_local[i];
    }
    cg::this_cluster().sync();
    for (int i = threadIdx.x; i < k; i += blockDim.x) {
      T acc = T(0);
#pragma unroll
      for (int r = 0; r < C; ++r) acc = pmax(acc, slots[r * stride + i]);
      out[i] = acc;
    }
    parity ^= 1;
    __syncthreads();
  }

  // buf (this CTA's slice of z) <- slice of z - J^T z (bounds.py:130), as
  // apply_operator does for a whole vector.  The thread's first own column and
  // row come from `own` (registers, loaded once per sample); further ones, and
  // entries beyond the register capacity, are read from the plan's arrays.
  template <int KR, int KC>
  __device__ void apply(const DevStructure& st, const Sample<T>& s, const OwnLines<T, KR, KC>& own) {
    T* zy = buf;
    T* zd = buf + ncl;
    T* zb = buf + ncl + mcl;
    for (int jj = threadIdx.x; jj < ncl; jj += blockDim.x) {
      const int j = c0 + jj;
      const bool mine = jj == (int)threadIdx.x;
      const T vy = zy[jj], vb = zb[jj];
      const T gg = (vy + vb) + vb;
      const T graw = gg * (mine ? own.yfac : code_factor<T>(s.yc[j] & 3));
      const T aa = mine ? own.aa : (s.av ? s.av[j] : s.a);
      const T dd = mine ? own.dd : (s.dv ? s.dv[j] : s.d);
      const T t = dd * (-graw);
      zy[jj] = vy - (aa * graw - vb);
#pragma unroll
      for (int r = 0; r < C; ++r) cg::this_cluster().map_shared_rank(tn, r)[j] = t;
    }
    cg::this_cluster().sync();
    for (int ii = threadIdx.x; ii < mcl; ii += blockDim.x) {
      const int i = r0 + ii;
      T acc = T(0);
      int k = st.row_ptr[i];
      if (ii == (int)threadIdx.x) {
#pragma unroll
        for (int q = 0; q < KR; ++q)
          if (q < own.rcount) acc = acc + own.rv[q] * tn[own.rc[q]];
        k += own.rcount;
      }
      for (; k < st.row_ptr[i + 1]; ++k) acc = acc + s.vals[k] * tn[st.col[k]];
      const T mu = zd[ii] + acc;
      const T mur = i < me ? mu : mu * balanced_factor<T>(s.dc[i]);
      const T sg = s.sv ? s.sv[i] : s.sigma;
      const T t = sg * mur;
      zd[ii] = zd[ii] - mur;
#pragma unroll
      for (int r = 0; r < C; ++r) cg::this_cluster().map_shared_rank(tm, r)[i] = t;
    }
    cg::this_cluster().sync();
    for (int jj = threadIdx.x; jj < ncl; jj += blockDim.x) {
      const int j = c0 + jj;
      T acc = T(0);
      int e = st.col_ptr[j];
      if (jj == (int)threadIdx.x) {
#pragma unroll
        for (int q = 0; q < KC; ++q)
          if (q < own.ccount) acc = acc + own.cv[q] * tm[own.cr[q]];
        e += own.ccount;
      }
      for (; e < st.col_ptr[j + 1]; ++e) acc = acc + s.vals[st.csc_slot[e]] * tm[st.csc_row[e]];
      zb[jj] = zb[jj] - acc;
    }
    __syncthreads();
  }

  // dloc[i] = this slice's part of <V[i], buf> for i < k: one warp per basis
  // vector, lanes over the slice, four independent partial sums per lane.
  __device__ void local_dots(int k, T* dloc) const {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    for (int i = warp; i < k; i += nw) {
      const T* v = V + (size_t)i * lcap;
      T a0 = T(0), a1 = T(0), a2 = T(0), a3 = T(0);
      int l = lane;
      for (; l + 96 < lv; l += 128) {
        a0 = a0 + v[l] * buf[l];
        a1 = a1 + v[l + 32] * buf[l + 32];
        a2 = a2 + v[l + 64] * buf[l + 64];
        a3 = a3 + v[l + 96] * buf[l + 96];
      }
      for (; l < lv; l += 32) a0 = a0 + v[l] * buf[l];
      T acc = (a0 + a1) + (a2 + a3);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) acc += shfl_xor(acc, o);
      if (lane == 0) dloc[i] = acc;
    }
    __syncthreads();
  }

  // buf <- buf - sum_i c[i] V[i] over i < k on this slice (accumulated in basis
  // order); a thread updates up to four of its entries at once.
  __device__ void update(int k, const T* c) {
    const int nt = blockDim.x;
    for (int base = threadIdx.x; base < lv; base += 4 * nt) {
      const int l1 = base + nt, l2 = base + 2 * nt, l3 = base + 3 * nt;
      const bool h1 = l1 < lv, h2 = l2 < lv, h3 = l3 < lv;
      T a0 = T(0), a1 = T(0), a2 = T(0), a3 = T(0);
      for (int i = 0; i < k; ++i) {
        const T ci = c[i];
        const T* v = V + (size_t)i * lcap;
        a0 = a0 + ci * v[base];
        if (h1) a1 = a1 + ci * v[l1];
        if (h2) a2 = a2 + ci * v[l2];
        if (h3) a3 = a3 + ci * v[l3];
      }
      buf[base] = buf[base] - a0;
      if (h1) buf[l1] = buf[l1] - a1;
      if (h2) buf[l2] = buf[l2] - a2;
      if (h3) buf[l3] = buf[l3] - a3;
    }
    __syncthreads();
  }
};

template <typename T, int C>
__global__ void __launch_bounds__(kClusterThreads, 1) cp_gmres_cluster_kernel(const AdjParams<T> p) {
  extern __shared__ __align__(16) unsigned char dyn[];
  __shared__ int s_flag;
  __shared__ int s_ok;
  T* sm = reinterpret_cast<T*>(dyn);
  const DevStructure& st = p.st;
  const int n = st.n, m = st.m;
  const int R = p.R;
  const ClusterLayout L = cluster_layout<T>(n, m, R, C);
  ClusterCtx<T, C> x_;
  x_.rank = (int)cg::this_cluster().block_rank();
  x_.n = n;
  x_.m = m;
  x_.me = st.me;
  x_.W = 2 * n + m;
  x_.R = R;
  x_.c0 = min(n, x_.rank * L.nc);
  x_.ncl = min(n, x_.c0 + L.nc) - x_.c0;
  x_.r0 = min(m, x_.rank * L.mc);
  x_.mcl = min(m, x_.r0 + L.mc) - x_.r0;
  x_.lv = 2 * x_.ncl + x_.mcl;
  x_.lcap = L.lcap;
  x_.V = sm + L.v;
  x_.buf = sm + L.buf;
  x_.tn = sm + L.tn;
  x_.tm = sm + L.tm;
  x_.part = sm + L.part;
  x_.red = sm + L.red;
  x_.parity = 0;
  ClusterCtx<T, C>& cx = x_;
  T* hess = sm + L.hess;
  T* proj = sm + L.proj;
  T* cs = sm + L.cs;
  T* sn = sm + L.sn;
  T* coef = sm + L.coef;
  T* c2 = sm + L.c2;
  T* bsv = sm + L.bsv;
  T* dloc = sm + L.dloc;
  T* buf = cx.buf;
  const int W = cx.W;
  const int lv = cx.lv;
  const T zero = T(0), eps = T(1e-30);
  const int64_t cluster_id = blockIdx.x / C;
  const int64_t nclusters = gridDim.x / C;
  const unsigned nblocks = gridDim.x + p.barrier_extra;
  const int stage = p.stage;

  int completed = stage == 2 ? p.completed0 : 0;
  int cycle = 0;
  bool any = stage == 2 ? true : atomicOr(&p.cycle_act[0], 0u) > 0;
  while (completed < p.max_it && any) {
    const int limit = min(R, p.max_it - completed);
    for (int64_t X = cluster_id; X < p.batch; X += nclusters) {
      const T thr = p.thresh[X];
      if (!(p.resinf[X] > thr)) continue;  // not cycle-active: frozen (same on every CTA)
      const Sample<T> s = make_sample(p, X);
      OwnLines<T, kOwnRow, kOwnCol> own;
      own.load(st, s, cx.c0, cx.ncl, cx.r0, cx.mcl);
      T* xg = p.x + X * W;
      // residual = g - A x on this slice, normalised into V[0]
      for (int l = threadIdx.x; l < lv; l += blockDim.x) buf[l] = xg[cx.global(l)];
      __syncthreads();
      cx.apply(st, s, own);
      T ss = zero;
      for (int l = threadIdx.x; l < lv; l += blockDim.x) {
        const T r = rhs_entry(s, n, m, cx.global(l)) - buf[l];
        buf[l] = r;
        ss = ss + r * r;
      }
      ss = block_sum(ss, cx.red);
      if (threadIdx.x == 0) dloc[0] = ss;
      __syncthreads();
      cx.sum(dloc, 1, coef);
      const T beta = sqrt(coef[0]);
      const T safe_beta = pmax(beta, eps);
      for (int l = threadIdx.x; l < lv; l += blockDim.x) {
        const T v = buf[l] / safe_beta;
        buf[l] = v;
        cx.V[l] = v;
      }
      for (int q = threadIdx.x; q < (R + 1) * R; q += blockDim.x) hess[q] = zero;
      for (int q = threadIdx.x; q < R + 1; q += blockDim.x) proj[q] = q == 0 ? beta : zero;
      for (int q = threadIdx.x; q < R; q += blockDim.x) {
        cs[q] = zero;
        sn[q] = zero;
      }
      if (threadIdx.x == 0) s_flag = 1;
      __syncthreads();
      int it = 0;
      while (it < limit && s_flag) {
        cx.apply(st, s, own);
        cx.local_dots(it + 1, dloc);
        cx.sum(dloc, it + 1, coef);
        cx.update(it + 1, coef);
        cx.local_dots(it + 1, dloc);
        cx.sum(dloc, it + 1, c2);
        cx.update(it + 1, c2);
        for (int q = threadIdx.x; q <= it; q += blockDim.x) coef[q] = coef[q] + c2[q];
        // Norm and finiteness of the new vector: the normalised entries are finite
        // exactly when these are and the norm is (|v| <= 1 otherwise).
        T nsq = zero;
        int fin = 1;
        for (int l = threadIdx.x; l < lv; l += blockDim.x) {
          nsq = nsq + buf[l] * buf[l];
          fin &= finite(buf[l]) ? 1 : 0;
        }
        nsq = block_sum(nsq, cx.red);
        fin = block_and(fin);
        if (threadIdx.x == 0) {
          dloc[0] = nsq;
          dloc[1] = fin ? zero : T(1);  // count of CTAs with a non-finite entry
        }
        __syncthreads();
        cx.sum(dloc, 2, c2);
        const T nn = sqrt(c2[0]);
        const bool fin_all = c2[1] == zero;
        const T sn_ = pmax(nn, eps);
        T* Vn = cx.V + (size_t)(it + 1) * cx.lcap;
        for (int l = threadIdx.x; l < lv; l += blockDim.x) {
          const T v = buf[l] / sn_;
          buf[l] = v;
          Vn[l] = v;
        }
        if (threadIdx.x == 0)
          s_flag = givens_step(it, R, coef, nn, fin_all, thr, hess, cs, sn, proj) ? 1 : 0;
        __syncthreads();
        ++it;
      }
      const int row_steps = it;
      if (threadIdx.x == 0) back_substitute(R, row_steps, hess, proj, bsv);
      __syncthreads();
      for (int l = threadIdx.x; l < lv; l += blockDim.x) {
        T acc = zero;
        for (int i = 0; i < row_steps; ++i) acc = acc + bsv[i] * cx.V[(size_t)i * cx.lcap + l];
        const int g = cx.global(l);
        const T cand = xg[g] + acc;
        buf[l] = cand;
        xg[g] = cand;
      }
      __syncthreads();
      cx.apply(st, s, own);
      T cn = zero;
      for (int l = threadIdx.x; l < lv; l += blockDim.x)
        cn = pmax(cn, fabs(rhs_entry(s, n, m, cx.global(l)) - buf[l]));
      cn = block_max(cn, cx.red);
      if (threadIdx.x == 0) dloc[0] = cn;
      __syncthreads();
      cx.max(dloc, 1, coef);
      if (cx.rank == 0 && threadIdx.x == 0) {
        const T cnv = coef[0];
        p.resinf[X] = cnv;
        if (p.work_steps) {
          p.work_steps[X] += row_steps;
          p.work_vectors[X] += (long long)row_steps * (row_steps + 1) / 2;
        }
        atomicMax(&p.cycle_len[cycle], (unsigned)row_steps);
        if (cnv > thr) atomicAdd(&p.cycle_act[cycle + 1], 1u);
      }
      // No CTA may start the next sample (and overwrite exchange slots or
      // replicas) before every CTA of the cluster has read this one's.
      cg::this_cluster().sync();
    }
    if (stage == 2) break;
    // Every CTA of a cluster must take the same path out of the grid barrier,
    // or the others would wait at a cluster barrier that never completes:
    // agree on the outcome first (one cluster barrier, taken by all).
    const bool ok = grid_barrier(p.barrier, nblocks, p.timeout_ns);
    if (threadIdx.x == 0) {
      dloc[0] = ok ? zero : T(1);
      s_ok = 0;
    }
    __syncthreads();
    cx.sum(dloc, 1, c2);
    if (c2[0] != zero) {
      if (threadIdx.x == 0) atomicExch(p.device_error, 1);
      break;
    }
    completed += (int)atomicOr(&p.cycle_len[cycle], 0u);
    any = atomicOr(&p.cycle_act[cycle + 1], 0u) > 0;
    ++cycle;
  }
  (void)s_ok;
  // Keep this CTA's shared memory alive until the cluster's last remote access.
  cg::this_cluster().sync();
}

template <typename T, int C>
cudaError_t launch_c(const AdjParams<T>& p, int clusters, bool cooperative, cudaStream_t stream) {
  const ClusterLayout L = cluster_layout<T>(p.st.n, p.st.m, p.R, C);
  const size_t smem = L.total * sizeof(T);
  auto kern = cp_gmres_cluster_kernel<T, C>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(clusters * C));
  cfg.blockDim = dim3(kClusterThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attrs[2];
  attrs[0].id = cudaLaunchAttributeClusterDimension;
  attrs[0].val.clusterDim.x = C;
  attrs[0].val.clusterDim.y = 1;
  attrs[0].val.clusterDim.z = 1;
  attrs[1].id = cudaLaunchAttributeCooperative;
  attrs[1].val.cooperative = 1;
  cfg.attrs = attrs;
  cfg.numAttrs = cooperative ? 2 : 1;
  return cudaLaunchKernelEx(&cfg, kern, p);
}

template <typename T, int C>
int clusters_c(int n, int m, int R) {
  const ClusterLayout L = cluster_layout<T>(n, m, R, C);
  const size_t smem = L.total * sizeof(T);
  auto kern = cp_gmres_cluster_kernel<T, C>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return 0;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(C);
  cfg.blockDim = dim3(kClusterThreads);
  cfg.dynamicSmemBytes = smem;
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeClusterDimension;
  attr.val.clusterDim.x = C;
  attr.val.clusterDim.y = 1;
  attr.val.clusterDim.z = 1;
  cfg.attrs = &attr;
  cfg.numAttrs = 1;
  int clusters = 0;
  if (cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg) != cudaSuccess) return 0;
  return clusters;
}

}  // namespace

template <typename T>
int gmres_cluster_size(int n, int m, int R, int max_smem_optin) {
  for (int C : {1, 2, 4, 8}) {
    const ClusterLayout L = cluster_layout<T>(n, m, R, C);
    if (L.total * sizeof(T) + 1024 <= (size_t)max_smem_optin) return C;
  }
  return 0;
}

template <typename T>
int gmres_cluster_count(int C, int n, int m, int R) {
  switch (C) {
    case 1: return clusters_c<T, 1>(n, m, R);
    case 2: return clusters_c<T, 2>(n, m, R);
    case 4: return clusters_c<T, 4>(n, m, R);
    case 8: return clusters_c<T, 8>(n, m, R);
    default: return 0;
  }
}

template <typename T>
cudaError_t launch_gmres_cluster(const AdjParams<T>& p, int C, int clusters, cudaStream_t stream) {
  const bool cooperative = p.stage == 0;  // only the fused cycles use the grid barrier
  switch (C) {
    case 1: return launch_c<T, 1>(p, clusters, cooperative, stream);
    case 2: return launch_c<T, 2>(p, clusters, cooperative, stream);
    case 4: return launch_c<T, 4>(p, clusters, cooperative, stream);
    case 8: return launch_c<T, 8>(p, clusters, cooperative, stream);
    default: return cudaErrorInvalidValue;
  }
}

template int gmres_cluster_size<double>(int, int, int, int);
template int gmres_cluster_size<float>(int, int, int, int);
template int gmres_cluster_count<double>(int, int, int, int);
template int gmres_cluster_count<float>(int, int, int, int);
template cudaError_t launch_gmres_cluster<double>(const AdjParams<double>&, int, int, cudaStream_t);
template cudaError_t launch_gmres_cluster<float>(const AdjParams<float>&, int, int, cudaStream_t);

}  // namespace purin
