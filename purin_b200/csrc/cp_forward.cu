// Forward CP solve: sparse_cp (src/purin/solvers/chambolle_pock/kernels.py:178-305)
// with freeze_converged and check_stationarity on.  The distance projection
// (kQP false) has q = 1, c = -target, y0 = target, as called by BoundProjection
// (bounds.py:42-66) and the unbounded layer (solver.py:149-176); the general
// diagonal QP (kQP true) reads per-sample q, c and y0 (diagonal_qp.py:99-123),
// with the step sizes, proximal coefficients, stationarity, dual minimiser and
// acceleration that depend on q (kernels.py:68-73,153-175,209-227,279-283)
// and converged &= all(q > 0) & all(lower <= upper).
//
// One CTA owns a tile of S samples for the whole solve.  The tile's iterates
// y, ybar (n each) and the duals (m) live in shared memory, interleaved by
// sample ([position * S + s]) in the internal row/column orders of sell.cuh,
// into which the per-sample inputs are permuted before the launch (outputs
// are scattered back at the end).  The structure is read in the sliced-ELL
// layout with C = 32: a warp owns a slice of 32 rows (or columns), each lane
// one line, and each lane carries that line for all S samples of the tile, so
// one index load and one value load feed S multiply-adds whose operands arrive
// as one vector shared-memory load.  An iteration makes these passes:
//   A  (rows)    lambda+ = proj(lambda + sigma (K ybar - rhs))         kernels.py:133-137
//   B  (columns) t = K.T lambda+, y+ = clip(a y - d t + o), ybar+,
//                stationarity                                         kernels.py:138-150,272-274
//   B2 (rows, columns) rhs . lambda+, bound violation and the primal/dual
//                objectives of y+ (t = K.T lambda+ again)             kernels.py:153-175
//   C  (rows)    K y+ - rhs for the equality/inequality residuals      kernels.py:155-157
// followed by a per-sample reduction and the accept/freeze decision
// (kernels.py:262-283).  B2 and C only feed the acceptance test and the values
// reported for the final iterate.  B2 runs when some active sample of the tile
// has finite iterates and stationarity within tolerance, C when one also passes
// the gap and bound tests, and both on the last iteration; otherwise no sample
// can be accepted whatever their values, and every output is the same.  After
// the first iteration that needs B2, passes A and B accumulate its sums
// themselves (same lanes, same order), since a converging tile needs them on
// most later iterations.  A frozen sample never changes again, so the tile
// exits as soon as all its samples are accepted; iterations and results are
// those of the reference's batch-wide loop.
#include <cuda_runtime.h>

#include <type_traits>

#include "common.cuh"
#include "cp_kernels.cuh"

namespace purin {

namespace {

constexpr int kC = 32;  // sliced-ELL slice height: one row per lane

template <typename T, int S, int kWarps>
struct TileScratch {
  T tau[S], sigma[S], theta[S], a[S], d[S], tol[S];
  T res_out[S], gap_out[S];
  int active[S], count[S], conv[S];
  T gap_it[S], stat_it[S], resb_it[S];
  int fin_it[S], need_c[S];
  T gam[S];     // min q (the accelerated update's strong-convexity modulus)
  int valid[S]; // diagonal QP: all(q > 0) & all(lower <= upper)
  T red[kWarps][S][6];
  int redf[kWarps][S];
  T s_red[kWarps][S];
};

// S consecutive values p[0 .. S-1] with vector loads (16-byte aligned when S * sizeof(T) >= 16).
template <typename T, int S>
__device__ __forceinline__ void load_pack(const T* p, T (&out)[S]) {
  if constexpr (sizeof(T) * S % 16 == 0) {
#pragma unroll
    for (int q = 0; q < S; q += 16 / sizeof(T)) {
      if constexpr (sizeof(T) == 8) {
        const double2 t = *reinterpret_cast<const double2*>(p + q);
        out[q] = t.x;
        out[q + 1] = t.y;
      } else {
        const float4 t = *reinterpret_cast<const float4*>(p + q);
        out[q] = t.x;
        out[q + 1] = t.y;
        out[q + 2] = t.z;
        out[q + 3] = t.w;
      }
    }
  } else if constexpr (sizeof(T) * S == 8 && sizeof(T) == 4) {
    const float2 t = *reinterpret_cast<const float2*>(p);
    out[0] = t.x;
    out[1] = t.y;
  } else {
#pragma unroll
    for (int q = 0; q < S; ++q) out[q] = p[q];
  }
}

// Sliced-ELL accumulation of one lane's line for all S samples:
// acc[q] += value_q(e) * x[index(e) * S + q] over the line's entries, in order.
// kPairs: indices are read two steps per 32-bit word (sell.cuh).
template <typename T, int S, bool kShared, bool kPairs>
struct SellLines {
  const int* ptr;
  const int* perm;
  const int* idx;
  const uint32_t* idx2;
  const int* slot;
  const T* sell_vals;    // kShared: values in SELL order
  const T* const* vals;  // !kShared: each sample's values in this SELL order

  __device__ __forceinline__ void step(int e, int col, const T* x, T (&acc)[S]) const {
    T xs[S];
    load_pack<T, S>(x + (size_t)col * S, xs);
    if constexpr (kShared) {
      const T v = __ldg(sell_vals + e);
#pragma unroll
      for (int q = 0; q < S; ++q) acc[q] = acc[q] + v * xs[q];
    } else {
#pragma unroll
      for (int q = 0; q < S; ++q) acc[q] = acc[q] + vals[q][e] * xs[q];
    }
  }

  __device__ __forceinline__ void dot(int sl, int lane, const T* x, T (&acc)[S]) const {
    const int e0 = __ldg(ptr + sl);
    const int width = (__ldg(ptr + sl + 1) - e0) / kC;
#pragma unroll
    for (int q = 0; q < S; ++q) acc[q] = T(0);
    int e = e0 + lane;
    if constexpr (kPairs) {
      const uint32_t* w = idx2 + e0 + lane;
      int k = 0;
#pragma unroll 4
      for (; k + 1 < width; k += 2, e += 2 * kC, w += kC) {
        const uint32_t pair = __ldg(w);
        step(e, (int)(pair & 0xffffu), x, acc);
        step(e + kC, (int)(pair >> 16), x, acc);
      }
      if (k < width) step(e, (int)(__ldg(w) & 0xffffu), x, acc);
    } else {
#pragma unroll 8
      for (int k = 0; k < width; ++k, e += kC) step(e, __ldg(idx + e), x, acc);
    }
  }
  __device__ __forceinline__ void abs_sum(int sl, int lane, T (&acc)[S]) const {
    const int e0 = __ldg(ptr + sl);
    const int width = (__ldg(ptr + sl + 1) - e0) / kC;
#pragma unroll
    for (int q = 0; q < S; ++q) acc[q] = T(0);
    int e = e0 + lane;
    for (int k = 0; k < width; ++k, e += kC) {
      if constexpr (kShared) {
        const T v = fabs(__ldg(sell_vals + e)) * T(1);
#pragma unroll
        for (int q = 0; q < S; ++q) acc[q] = acc[q] + v;
      } else {
#pragma unroll
        for (int q = 0; q < S; ++q) acc[q] = acc[q] + fabs(vals[q][e]) * T(1);
      }
    }
  }
  __device__ __forceinline__ int line(int sl, int lane) const { return __ldg(perm + sl * kC + lane); }
};

template <typename T>
__device__ __forceinline__ T warp_sum32(T v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += shfl_xor(v, o);
  return v;
}
template <typename T>
__device__ __forceinline__ T warp_max32(T v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = pmax(v, shfl_xor(v, o));
  return v;
}

// Per-sample tile reductions; every thread receives all S totals.
template <typename T, int S, bool kMax, int kWarps>
__device__ __forceinline__ void tile_reduce(T (&v)[S], T (&scratch)[kWarps][S]) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int q = 0; q < S; ++q) v[q] = kMax ? warp_max32(v[q]) : warp_sum32(v[q]);
  __syncthreads();
  if (lane == 0) {
#pragma unroll
    for (int q = 0; q < S; ++q) scratch[warp][q] = v[q];
  }
  __syncthreads();
#pragma unroll
  for (int q = 0; q < S; ++q) {
    T total = T(0);
#pragma unroll 8
    for (int w = 0; w < kWarps; ++w) total = kMax ? pmax(total, scratch[w][q]) : total + scratch[w][q];
    v[q] = total;
  }
}

// Per-sample tile maximum of values of any sign (tile_reduce's max starts from
// zero, which suits its nonnegative quantities only).
template <typename T, int S, int kWarps>
__device__ __forceinline__ void tile_max_signed(T (&v)[S], T (&scratch)[kWarps][S]) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int q = 0; q < S; ++q) v[q] = warp_max32(v[q]);
  __syncthreads();
  if (lane == 0) {
#pragma unroll
    for (int q = 0; q < S; ++q) scratch[warp][q] = v[q];
  }
  __syncthreads();
#pragma unroll
  for (int q = 0; q < S; ++q) {
    T total = scratch[0][q];
#pragma unroll 8
    for (int w = 1; w < kWarps; ++w) total = pmax(total, scratch[w][q]);
    v[q] = total;
  }
}

template <typename T, int S>
__device__ __forceinline__ void store_pack(T* p, const T (&v)[S]) {
  if constexpr (sizeof(T) * S % 16 == 0) {
#pragma unroll
    for (int q = 0; q < S; q += 16 / sizeof(T)) {
      if constexpr (sizeof(T) == 8) {
        *reinterpret_cast<double2*>(p + q) = make_double2(v[q], v[q + 1]);
      } else {
        *reinterpret_cast<float4*>(p + q) = make_float4(v[q], v[q + 1], v[q + 2], v[q + 3]);
      }
    }
  } else if constexpr (sizeof(T) * S == 8 && sizeof(T) == 4) {
    *reinterpret_cast<float2*>(p) = make_float2(v[0], v[1]);
  } else {
#pragma unroll
    for (int q = 0; q < S; ++q) p[q] = v[q];
  }
}

// Minimiser of 0.5 q m^2 + t m over [l, u] (kernels.py:164-169): clip(-t/q)
// where q > 1e-12, else the bound that t points away from.  With q = 1
// (distance projection) it is clip(-t/1).
template <bool kQP, typename T>
__device__ __forceinline__ T dual_minimiser(T tt, T qj, T l, T u) {
  if constexpr (kQP) {
    return qj > T(1e-12) ? clip(-tt / qj, l, u) : (tt >= T(0) ? l : u);
  } else {
    return clip(-tt / qj, l, u);
  }
}

// Wide multi-sample shared-memory tiles (S, NT): one CTA per SM, registers
// 65536 / NT (128 for 512 threads, 80 for 768, 64 for 1024).
#define PURIN_WIDE_TILES                                                                   \
  PURIN_WIDE_TILE(2, 512) PURIN_WIDE_TILE(4, 512) PURIN_WIDE_TILE(2, 768) PURIN_WIDE_TILE(4, 768) \
  PURIN_WIDE_TILE(2, 1024) PURIN_WIDE_TILE(4, 1024)

// Resident CTAs per SM the register budget is sized for (64 registers per
// thread for one-sample tiles): 1 x 1024 or 768, 2 x 512 (one CTA of 512 for
// wider tiles, 128 registers), 8 x 128, or 4 / 2 / 1 CTAs of 256 threads for
// S = 1 / 2 / wider.  fp32 two-sample tiles also fit 64 registers (no spills;
// 87 unconstrained), so they keep 4 CTAs per SM like the one-sample tiles;
// fp64 two-sample and fp32 four-sample tiles fit 80 registers (3 CTAs per SM;
// 122 and 141 unconstrained, a 4-byte spill).
constexpr int forward_min_blocks(int S, int NT, int elem_bytes) {
  return NT >= 1024                    ? 1
         : NT >= 512                   ? (S == 1 ? 2 : 1)
         : NT <= 128                   ? 8
         : S == 1                      ? 4
         : (S == 2 && elem_bytes == 4) ? 4
         : S == 2                      ? 3
         : (S == 4 && elem_bytes == 4) ? 3
                                       : 1;
}

template <typename T, int S, int NT, bool kSmem, bool kShared, bool kQP>
__global__ void __launch_bounds__(NT, forward_min_blocks(S, NT, (int)sizeof(T)))
cp_forward_kernel(const FwdParams<T> p) {
  constexpr int kThreads = NT;
  constexpr int kWarps = NT / 32;
  extern __shared__ __align__(16) unsigned char dyn_smem[];
  __shared__ TileScratch<T, S, kWarps> sc;

  const DevStructure& st = p.st;
  const SellView& sv = p.sell;
  const int n = st.n, m = st.m, me = st.me;
  const int n_pos = sv.n_pos, m_pos = sv.m_pos;
  const int tid = threadIdx.x;
  const int lane = tid & 31, warp = tid >> 5;

  // Sample q of this tile (reads of the padding samples of the last tile are clamped).
  const int64_t tile0 = (int64_t)blockIdx.x * S;
  auto sample = [&](int q) -> int64_t { return tile0 + q < p.batch ? tile0 + q : p.batch - 1; };
  auto is_valid = [&](int q) -> bool { return tile0 + q < p.batch; };
  // Per-sample values (not shared): each sample's copy in the two SELL orders
  // (arranged once per call; padding entries hold zeros).
  const T* vr_q[S];
  const T* vc_q[S];
#pragma unroll
  for (int q = 0; q < S; ++q) {
    vr_q[q] = kShared ? nullptr : p.vr_ps + sample(q) * p.nnz_r_ps;
    vc_q[q] = kShared ? nullptr : p.vc_ps + sample(q) * p.nnz_c_ps;
  }

  // Per-variable proximal coefficients live in shared memory for diagonal
  // steps; a diagonal QP without them recomputes 1 / (1 + tau q_j) from the q_j
  // it reads anyway (the same operations, so the same values).
  // Diagonal steps: shared by the batch in global memory (dg), else per tile in
  // shared memory (pv).
  const bool dg = p.dg_sigma != nullptr;
  const bool pv = p.diag && !dg;
  // Iterates in internal positions: y, ybar (n_pos + 1), duals (m_pos + 1); the
  // last element of each is the zero that padding entries gather.
  const size_t tile_elems =
      (size_t)(2 * (n_pos + 1) + (m_pos + 1) + (pv ? 2 * (n_pos + 1) + (m_pos + 1) : 0)) * S;
  T* base = kSmem ? reinterpret_cast<T*>(dyn_smem) : p.gstate + (size_t)blockIdx.x * tile_elems;
  T* y = base;
  T* ybar = y + (size_t)(n_pos + 1) * S;
  T* lam = ybar + (size_t)(n_pos + 1) * S;
  T* av = lam + (size_t)(m_pos + 1) * S;  // per-variable a, d and per-row sigma (only when pv)
  T* dv = av + (size_t)(n_pos + 1) * S;
  T* sv_ = dv + (size_t)(n_pos + 1) * S;

  // Shared-memory tiles read index pairs (positions fit in 16 bits there).
  const SellLines<T, S, kShared, kSmem> rows{sv.r_ptr, sv.r_perm, sv.r_idx, sv.r_idx2, sv.r_slot,
                                              p.vr, vr_q};
  const SellLines<T, S, kShared, kSmem> cols{sv.c_ptr, sv.c_perm, sv.c_idx, sv.c_idx2, sv.c_slot,
                                              p.vc, vc_q};
  const T zero = T(0), one = T(1);
  const T safety = p.safety;

  // ---- step sizes (kernels.py:209-227) ------------------------------------
  T L[S];
#pragma unroll
  for (int q = 0; q < S; ++q) L[q] = one;
  if (pv) {
    // diagonal_step_sizes (kernels.py:76-88): |K| row and column sums.
    for (int sl = warp; sl < sv.nsl_r; sl += kWarps) {
      T acc[S];
      rows.abs_sum(sl, lane, acc);
      const int qp = sl * kC + lane;
#pragma unroll
      for (int q = 0; q < S; ++q)
        sv_[(size_t)qp * S + q] = safety / (acc[q] > zero ? pmax(acc[q], T(1e-12)) : one);
    }
    for (int sl = warp; sl < sv.nsl_c; sl += kWarps) {
      T acc[S];
      cols.abs_sum(sl, lane, acc);
      const int pp = sl * kC + lane;
#pragma unroll
      for (int q = 0; q < S; ++q) {
        const T tau = safety / (acc[q] > zero ? pmax(acc[q], T(1e-12)) : one);
        const T qj = kQP ? p.q_i[sample(q) * n_pos + pp] : one;
        const T a = one / (one + tau * qj);
        av[(size_t)pp * S + q] = a;
        dv[(size_t)pp * S + q] = tau * a;
      }
    }
  } else if (p.diag) {
    // Diagonal steps shared by the batch: computed once per call (p.dg_*).
  } else if (p.norm_bound) {
    T rmax[S], cmax[S];
#pragma unroll
    for (int q = 0; q < S; ++q) rmax[q] = cmax[q] = zero;
    for (int sl = warp; sl < sv.nsl_r; sl += kWarps) {
      T acc[S];
      rows.abs_sum(sl, lane, acc);
#pragma unroll
      for (int q = 0; q < S; ++q) rmax[q] = pmax(rmax[q], acc[q]);
    }
    for (int sl = warp; sl < sv.nsl_c; sl += kWarps) {
      T acc[S];
      cols.abs_sum(sl, lane, acc);
#pragma unroll
      for (int q = 0; q < S; ++q) cmax[q] = pmax(cmax[q], acc[q]);
    }
    tile_reduce<T, S, true>(rmax, sc.s_red);
    tile_reduce<T, S, true>(cmax, sc.s_red);
#pragma unroll
    for (int q = 0; q < S; ++q) L[q] = pmax(sqrt(rmax[q] * cmax[q]), T(1e-12));
  } else {
    // norm_estimate (kernels.py:52-65): power iteration on K.T K.
    T* x = y;      // n_pos (+ zero pad)
    T* u = lam;    // m_pos (+ zero pad)
    T* z = ybar;   // n_pos (+ zero pad)
    T ss[S];
#pragma unroll
    for (int q = 0; q < S; ++q) {
      uint32_t k0, k1;
      split_key(p.norm_seed, p.sample_offset + sample(q), p.total_batch, p.partitionable != 0, k0, k1);
      ss[q] = zero;
      for (int pp = tid; pp < n_pos; pp += kThreads) {
        const int j = __ldg(sv.c_perm + pp);
        const T v = j >= 0 ? NormalBits<T>::draw(k0, k1, j, n, p.partitionable != 0) : zero;
        x[(size_t)pp * S + q] = v;
        ss[q] = ss[q] + v * v;
      }
    }
    if (tid < S) {
      x[(size_t)n_pos * S + tid] = zero;
      u[(size_t)m_pos * S + tid] = zero;
    }
    tile_reduce<T, S, false>(ss, sc.s_red);
    for (int pp = tid; pp < n_pos; pp += kThreads) {
#pragma unroll
      for (int q = 0; q < S; ++q) x[(size_t)pp * S + q] = x[(size_t)pp * S + q] / (sqrt(ss[q]) + T(1e-12));
    }
    T eig[S];
#pragma unroll
    for (int q = 0; q < S; ++q) eig[q] = zero;
    for (int it = 0; it < p.norm_iterations; ++it) {
      __syncthreads();
      for (int sl = warp; sl < sv.nsl_r; sl += kWarps) {
        T acc[S];
        rows.dot(sl, lane, x, acc);
        store_pack<T, S>(u + (size_t)(sl * kC + lane) * S, acc);
      }
      __syncthreads();
      T xz[S], zz[S];
#pragma unroll
      for (int q = 0; q < S; ++q) xz[q] = zz[q] = zero;
      for (int sl = warp; sl < sv.nsl_c; sl += kWarps) {
        T acc[S];
        cols.dot(sl, lane, u, acc);
        const size_t pp = (size_t)(sl * kC + lane) * S;
        store_pack<T, S>(z + pp, acc);
#pragma unroll
        for (int q = 0; q < S; ++q) {
          xz[q] = xz[q] + x[pp + q] * acc[q];
          zz[q] = zz[q] + acc[q] * acc[q];
        }
      }
      tile_reduce<T, S, false>(xz, sc.s_red);
      tile_reduce<T, S, false>(zz, sc.s_red);
#pragma unroll
      for (int q = 0; q < S; ++q) eig[q] = xz[q];
      for (int pp = tid; pp < n_pos; pp += kThreads) {
#pragma unroll
        for (int q = 0; q < S; ++q) x[(size_t)pp * S + q] = z[(size_t)pp * S + q] / (sqrt(zz[q]) + T(1e-12));
      }
    }
#pragma unroll
    for (int q = 0; q < S; ++q) L[q] = pmax(sqrt(pmax(eig[q], zero)) + T(1e-12), T(1e-12));
    __syncthreads();
  }

  // ---- q-dependent scalars (kernels.py:221-227): min q, max q, and the QP's
  // validity; tau = s/L when accelerated with min q > 0, else s/(max q + L).
  T qmin[S], qmax[S];
#pragma unroll
  for (int q = 0; q < S; ++q) qmin[q] = qmax[q] = one;
  if constexpr (kQP) {
    T nmin[S], bad[S];
#pragma unroll
    for (int q = 0; q < S; ++q) {
      nmin[q] = T(-INFINITY);  // max of -q: min q without a separate min reduction
      qmax[q] = T(-INFINITY);
      bad[q] = zero;
    }
    for (int pp = tid; pp < n_pos; pp += kThreads) {
      if (__ldg(sv.c_perm + pp) < 0) continue;
#pragma unroll
      for (int q = 0; q < S; ++q) {
        const int64_t b = sample(q);
        const T qj = p.q_i[b * n_pos + pp];
        nmin[q] = pmax(nmin[q], -qj);
        qmax[q] = pmax(qmax[q], qj);
        if (!(p.lo_i[b * p.bstride_i + pp] <= p.up_i[b * p.bstride_i + pp])) bad[q] = one;
      }
    }
    tile_max_signed<T, S>(nmin, sc.s_red);
    tile_max_signed<T, S>(qmax, sc.s_red);
    tile_reduce<T, S, true>(bad, sc.s_red);
#pragma unroll
    for (int q = 0; q < S; ++q) {
      qmin[q] = -nmin[q];
      if (tid == 0) sc.valid[q] = (qmin[q] > zero && bad[q] == zero) ? 1 : 0;
    }
  }

  // Accelerated step-size update after an iteration (kernels.py:289-297).
  auto advance_steps = [&](int q) {
    const T tau = sc.tau[q];
    const T nt = one / sqrt(one + sc.gam[q] * tau);
    const T ntau = nt * tau;
    sc.tau[q] = ntau;
    sc.sigma[q] = sc.sigma[q] / nt;
    sc.theta[q] = nt;
    sc.a[q] = one / (one + ntau * one);
    sc.d[q] = ntau * sc.a[q];
  };
  // Iterations a resumed sample has already run, within [0, max_iterations].
  auto resume_iteration = [&](int q) {
    const int v = p.start_it[sample(q)];
    return v < 0 ? 0 : (v > p.max_iterations ? p.max_iterations : v);
  };

  // ---- initial state: y = ybar = y0 (the target), lambda = dual0 -----------
  for (int pp = tid; pp < n_pos; pp += kThreads) {
    T t[S];
#pragma unroll
    for (int q = 0; q < S; ++q) {
      if constexpr (kQP) t[q] = p.y0_i ? p.y0_i[sample(q) * n_pos + pp] : zero;
      else t[q] = p.tgt_i[sample(q) * n_pos + pp];
    }
    store_pack<T, S>(y + (size_t)pp * S, t);
    if constexpr (kQP) {
      if (p.ybar0_i) {
#pragma unroll
        for (int q = 0; q < S; ++q) t[q] = p.ybar0_i[sample(q) * n_pos + pp];
      }
    }
    store_pack<T, S>(ybar + (size_t)pp * S, t);
  }
  for (int qp = tid; qp < m_pos; qp += kThreads) {
    T d0[S];
#pragma unroll
    for (int q = 0; q < S; ++q) d0[q] = p.dual0_i ? p.dual0_i[sample(q) * m_pos + qp] : zero;
    store_pack<T, S>(lam + (size_t)qp * S, d0);
  }
  if (tid < S) {
    const int q = tid;
    // Padding elements of the gathered vectors stay zero for the whole solve.
    y[(size_t)n_pos * S + q] = zero;
    ybar[(size_t)n_pos * S + q] = zero;
    lam[(size_t)m_pos * S + q] = zero;
    const T tau = (p.accelerated && qmin[q] > zero) ? safety / L[q] : safety / (qmax[q] + L[q]);
    sc.tau[q] = tau;
    sc.gam[q] = qmin[q];
    sc.sigma[q] = safety / L[q];
    sc.theta[q] = one;
    sc.a[q] = one / (one + tau * one);
    sc.d[q] = tau * sc.a[q];
    sc.tol[q] = p.tol[sample(q)];
    sc.active[q] = is_valid(q) ? 1 : 0;
    sc.count[q] = 0;
    if constexpr (kQP) {
      // Resuming after start_it iterations: the count and the accelerated
      // steps continue from there (the same updates the loop applies).
      if (p.start_it && is_valid(q)) {
        const int it0 = resume_iteration(q);
        sc.count[q] = it0;
        if (p.accelerated)
          for (int k = 0; k < it0; ++k) advance_steps(q);
      }
    }
    sc.conv[q] = 0;
    sc.res_out[q] = zero;
    sc.gap_out[q] = zero;
  }
  __syncthreads();

  // Warp partials of the per-sample diagnostics: [warp][sample][0..5] = bound
  // violation max, stationarity max, primal sum, dual sum, rhs.dual sum,
  // constraint residual max.
  auto publish = [&](int slot, T (&v)[S], bool is_max) {
#pragma unroll
    for (int q = 0; q < S; ++q) {
      const T r = is_max ? warp_max32(v[q]) : warp_sum32(v[q]);
      if (lane == 0) sc.red[warp][q][slot] = r;
    }
  };
  // Phase A: dual update; with kFull also the dual objective term rhs . lambda+.
  auto phase_a = [&](auto full_c, int act, int& fin) {
    constexpr bool kFull = decltype(full_c)::value;
    T rd[S], sigma[S];
#pragma unroll
    for (int q = 0; q < S; ++q) {
      rd[q] = zero;
      sigma[q] = sc.sigma[q];  // per-sample scalars of this iteration, read once
    }
    for (int sl = warp; sl < sv.nsl_r; sl += kWarps) {
      const int i = rows.line(sl, lane);
      const int qp = sl * kC + lane;
      // Per-sample operands are loaded before the product so their latency overlaps it.
      T rbs[S];
#pragma unroll
      for (int q = 0; q < S; ++q) rbs[q] = p.rhs_i[sample(q) * m_pos + qp];
      T acc[S];
      rows.dot(sl, lane, ybar, acc);
      if (i >= 0) {
        T lv[S];
        load_pack<T, S>(lam + (size_t)qp * S, lv);
#pragma unroll
        for (int q = 0; q < S; ++q) {
          if (!((act >> q) & 1)) continue;
          const T sg = p.diag ? (dg ? __ldg(p.dg_sigma + qp) : sv_[(size_t)qp * S + q]) : sigma[q];
          const T raw = lv[q] + sg * (acc[q] - rbs[q]);
          const T nl = i < me ? raw : pmax(raw, zero);
          lv[q] = nl;
          if (!finite(nl)) fin &= ~(1 << q);
          if constexpr (kFull) rd[q] = rd[q] + rbs[q] * nl;
        }
        store_pack<T, S>(lam + (size_t)qp * S, lv);
      }
    }
    if constexpr (kFull) publish(4, rd, false);
  };
  // Phase B: primal update and stationarity; with kFull also the bound
  // violation and the primal and dual objectives of y+.
  auto phase_b = [&](auto full_c, int act, int& fin) {
    constexpr bool kFull = decltype(full_c)::value;
    T stm[S], resm[S], ps[S], ds[S], a_s[S], d_s[S], theta_s[S], tau_s[S];
#pragma unroll
    for (int q = 0; q < S; ++q) {
      stm[q] = resm[q] = ps[q] = ds[q] = zero;
      a_s[q] = sc.a[q];  // per-sample scalars of this iteration, read once
      d_s[q] = sc.d[q];
      theta_s[q] = sc.theta[q];
      tau_s[q] = sc.tau[q];
    }
    for (int sl = warp; sl < sv.nsl_c; sl += kWarps) {
      const int j = cols.line(sl, lane);
      const int pp = sl * kC + lane;
      T tg[S], lb[S], ub[S], qv[S];
#pragma unroll
      for (int q = 0; q < S; ++q) {
        const int64_t b = sample(q);
        if constexpr (kQP) {
          tg[q] = p.c_i[b * n_pos + pp];
          qv[q] = p.q_i[b * n_pos + pp];
        } else {
          tg[q] = p.tgt_i[b * n_pos + pp];
          qv[q] = one;
        }
        lb[q] = p.lo_i[b * p.bstride_i + pp];
        ub[q] = p.up_i[b * p.bstride_i + pp];
      }
      T t[S];
      cols.dot(sl, lane, lam, t);
      if (j >= 0) {
        T yv[S], bv[S];
        load_pack<T, S>(y + (size_t)pp * S, yv);
        load_pack<T, S>(ybar + (size_t)pp * S, bv);
#pragma unroll
        for (int q = 0; q < S; ++q) {
          if (!((act >> q) & 1)) continue;
          const size_t js = (size_t)pp * S + q;
          const T yo = yv[q];
          const T c = kQP ? tg[q] : -tg[q];
          const T qj = qv[q];
          T aa, dd;
          if (kQP && !pv) {
            // proximal_coefficients (kernels.py:68-73) of this iteration's tau
            // (per column with shared diagonal steps): fixed steps precompute
            // them (kernels.py:236), accelerated steps recompute them; either
            // way these are the same operations.
            const T tj = dg ? __ldg(p.dg_tau + pp) : tau_s[q];
            aa = one / (one + tj * qj);
            dd = tj * aa;
          } else {
            aa = pv ? av[js] : (dg ? __ldg(p.dg_a + pp) : a_s[q]);
            dd = pv ? dv[js] : (dg ? __ldg(p.dg_d + pp) : d_s[q]);
          }
          const T off = (-dd) * c;
          // factored_proximal (kernels.py:142-145): inverse * ((y - tau t) - tau c).
          const T yr = (kQP && (p.qp_flags & 1))
                           ? aa * ((yo - tau_s[q] * t[q]) - tau_s[q] * c)
                           : (aa * yo - dd * t[q]) + off;
          const T l = lb[q];
          const T u = ub[q];
          const T yn = clip(yr, l, u);
          yv[q] = yn;
          bv[q] = yn + theta_s[q] * (yn - yo);
          if (!finite(yn)) fin &= ~(1 << q);
          if constexpr (kFull) {
            resm[q] = pmax(resm[q], pmax(pmax(l - yn, zero), pmax(yn - u, zero)));
            ps[q] = ps[q] + ((T(0.5) * qj * yn) * yn + c * yn);
            const T tt = c + t[q];
            const T mn = dual_minimiser<kQP>(tt, qj, l, u);
            ds[q] = ds[q] + (T(0.5) * qj * (mn * mn) + tt * mn);
          }
          const T inner = (qj * yn + c) + t[q];
          stm[q] = pmax(stm[q], fabs(yn - clip(yn - inner, l, u)));
        }
        store_pack<T, S>(y + (size_t)pp * S, yv);
        store_pack<T, S>(ybar + (size_t)pp * S, bv);
      }
    }
    publish(1, stm, true);
    if constexpr (kFull) {
      publish(0, resm, true);  // bound violation part of the residual
      publish(2, ps, false);
      publish(3, ds, false);
    }
  };
  // Once a tile has needed the full stopping test it keeps evaluating it inside
  // phases A and B (a converging tile needs it on most later iterations); before
  // that, phase B2 recomputes the same sums in the same order when required.
  bool full = false;
  int it_begin = 0;
  if constexpr (kQP && S == 1) {
    if (p.start_it && is_valid(0)) it_begin = resume_iteration(0);
  }
  for (int it = it_begin; it < p.max_iterations; ++it) {
    int act = 0;
#pragma unroll
    for (int q = 0; q < S; ++q) act |= (sc.active[q] != 0) << q;
    if (!act) break;
    const bool last = it + 1 == p.max_iterations;
    int fin = (1 << S) - 1;
    if (full) phase_a(std::true_type{}, act, fin);
    else phase_a(std::false_type{}, act, fin);
    __syncthreads();
    if (full) phase_b(std::true_type{}, act, fin);
    else phase_b(std::false_type{}, act, fin);
    fin = __reduce_and_sync(kFullMask, (unsigned)fin);
    if (lane == 0) {
#pragma unroll
      for (int q = 0; q < S; ++q) sc.redf[warp][q] = (fin >> q) & 1;
    }
    __syncthreads();
    // Acceptance needs finite iterates and stationarity within tolerance.  The
    // gap and bound violation (phases A/B with `full`, else phase B2) are used
    // only when some active sample passes those tests, the feasibility residual
    // of y+ (phase C) only when some sample also passes the gap and bound tests,
    // and both on the last iteration, whose values are reported.  An iteration
    // that skips them rejects every sample, as the full test would.
    if (tid < S) {
      const int q = tid;
      T stat = zero;
      int f = 1;
#pragma unroll 8
      for (int w = 0; w < kWarps; ++w) {
        stat = pmax(stat, sc.red[w][q][1]);
        f &= sc.redf[w][q];
      }
      sc.stat_it[q] = stat;
      sc.fin_it[q] = f;
      const bool stat_ok = (kQP && (p.qp_flags & 2)) || stat <= sc.tol[q];
      sc.need_c[q] = (sc.active[q] && f && stat_ok) ? 1 : 0;
    }
    __syncthreads();
    bool need_gap = last;
#pragma unroll
    for (int q = 0; q < S; ++q) need_gap |= sc.need_c[q] != 0;
    bool need_c = last;
    if (need_gap && !full) {
      // Phase B2: dual objective term rhs . lambda+ (rows), primal and dual
      // objectives of y+ and the bound violation (columns, t = K^T lambda+ again).
      T rd[S];
#pragma unroll
      for (int q = 0; q < S; ++q) rd[q] = zero;
      for (int sl = warp; sl < sv.nsl_r; sl += kWarps) {
        const int i = rows.line(sl, lane);
        const int qp = sl * kC + lane;
        if (i >= 0) {
          T lv[S];
          load_pack<T, S>(lam + (size_t)qp * S, lv);
#pragma unroll
          for (int q = 0; q < S; ++q) {
            if (!((act >> q) & 1)) continue;
            rd[q] = rd[q] + p.rhs_i[sample(q) * m_pos + qp] * lv[q];
          }
        }
      }
      publish(4, rd, false);
      T resm[S], ps[S], ds[S];
#pragma unroll
      for (int q = 0; q < S; ++q) resm[q] = ps[q] = ds[q] = zero;
      for (int sl = warp; sl < sv.nsl_c; sl += kWarps) {
        const int j = cols.line(sl, lane);
        const int pp = sl * kC + lane;
        T tg[S], lb[S], ub[S], qv[S];
#pragma unroll
        for (int q = 0; q < S; ++q) {
          const int64_t b = sample(q);
          if constexpr (kQP) {
            tg[q] = p.c_i[b * n_pos + pp];
            qv[q] = p.q_i[b * n_pos + pp];
          } else {
            tg[q] = p.tgt_i[b * n_pos + pp];
            qv[q] = one;
          }
          lb[q] = p.lo_i[b * p.bstride_i + pp];
          ub[q] = p.up_i[b * p.bstride_i + pp];
        }
        T t[S];
        cols.dot(sl, lane, lam, t);
        if (j >= 0) {
          T yv[S];
          load_pack<T, S>(y + (size_t)pp * S, yv);
#pragma unroll
          for (int q = 0; q < S; ++q) {
            if (!((act >> q) & 1)) continue;
            const T yn = yv[q];
            const T c = kQP ? tg[q] : -tg[q];
            const T qj = qv[q];
            const T l = lb[q];
            const T u = ub[q];
            resm[q] = pmax(resm[q], pmax(pmax(l - yn, zero), pmax(yn - u, zero)));
            ps[q] = ps[q] + ((T(0.5) * qj * yn) * yn + c * yn);
            const T tt = c + t[q];
            const T mn = dual_minimiser<kQP>(tt, qj, l, u);
            ds[q] = ds[q] + (T(0.5) * qj * (mn * mn) + tt * mn);
          }
        }
      }
      publish(0, resm, true);  // bound violation part of the residual
      publish(2, ps, false);
      publish(3, ds, false);
    }
    if (need_gap) {
      __syncthreads();
      if (tid < S) {
        const int q = tid;
        T resb = zero, P = zero, Dp = zero, Rd = zero;
#pragma unroll 8
        for (int w = 0; w < kWarps; ++w) {
          resb = pmax(resb, sc.red[w][q][0]);
          P = P + sc.red[w][q][2];
          Dp = Dp + sc.red[w][q][3];
          Rd = Rd + sc.red[w][q][4];
        }
        const T D = Dp - Rd;
        const T gap = pmax(P - D, zero) / pmax(one, pmax(fabs(P), fabs(D)));
        const T tol = sc.tol[q];
        const bool finite_all = sc.fin_it[q] && finite(gap);
        sc.gap_it[q] = gap;
        sc.resb_it[q] = resb;
        sc.fin_it[q] = finite_all ? 1 : 0;
        const bool stat_ok = (kQP && (p.qp_flags & 2)) || sc.stat_it[q] <= tol;
        sc.need_c[q] = (sc.active[q] && finite_all && resb <= tol && gap <= tol && stat_ok) ? 1 : 0;
      }
      __syncthreads();
#pragma unroll
      for (int q = 0; q < S; ++q) need_c |= sc.need_c[q] != 0;
      full = true;
    }
    if (need_c) {
      // Phase C: constraint residuals of y+.
      T resc[S];
#pragma unroll
      for (int q = 0; q < S; ++q) resc[q] = zero;
      for (int sl = warp; sl < sv.nsl_r; sl += kWarps) {
        const int i = rows.line(sl, lane);
        const int qp = sl * kC + lane;
        T rbs[S];
#pragma unroll
        for (int q = 0; q < S; ++q) rbs[q] = p.rhs_i[sample(q) * m_pos + qp];
        T acc[S];
        rows.dot(sl, lane, y, acc);
        if (i >= 0) {
#pragma unroll
          for (int q = 0; q < S; ++q) {
            if (!((act >> q) & 1)) continue;
            const T r = acc[q] - rbs[q];
            resc[q] = pmax(resc[q], i < me ? fabs(r) : pmax(r, zero));
          }
        }
      }
      publish(5, resc, true);
      __syncthreads();
    }
    if (tid < S) {
      const int q = tid;
      bool accepted = false;
      if (need_c) {  // need_c implies that phase B2 ran
        T res = sc.resb_it[q];
#pragma unroll 8
        for (int w = 0; w < kWarps; ++w) res = pmax(res, sc.red[w][q][5]);
        const T gap = sc.gap_it[q], stat = sc.stat_it[q];
        const T tol = sc.tol[q];
        // check_stationarity off (kernels.py:276-277,300-304): acceptance and the
        // reported residual leave stationarity out.
        const bool no_stat = kQP && (p.qp_flags & 2);
        accepted = sc.fin_it[q] && res <= tol && gap <= tol && (no_stat || stat <= tol);
        if (sc.active[q]) {
          sc.res_out[q] = no_stat ? res : pmax(res, stat);
          sc.gap_out[q] = gap;
        }
      }
      if (sc.active[q]) {
        sc.count[q] += 1;
        sc.conv[q] = accepted ? 1 : 0;
        // freeze_converged off: an accepted sample keeps iterating (the caller
        // runs the batch's trip count; kernels.py:266-271).
        if (accepted && !(kQP && (p.qp_flags & 4))) sc.active[q] = 0;
      }
      if (p.accelerated) advance_steps(q);
    }
    __syncthreads();
  }

  // ---- outputs (back to the external orders) -------------------------------
#pragma unroll
  for (int q = 0; q < S; ++q) {
    if (!is_valid(q)) continue;
    const int64_t b = sample(q);
    for (int pp = tid; pp < n_pos; pp += kThreads) {
      const int j = __ldg(sv.c_perm + pp);
      if (j >= 0) p.y_out[b * n + j] = y[(size_t)pp * S + q];
    }
    if constexpr (kQP) {
      if (p.ybar_out)
        for (int pp = tid; pp < n_pos; pp += kThreads) {
          const int j = __ldg(sv.c_perm + pp);
          if (j >= 0) p.ybar_out[b * n + j] = ybar[(size_t)pp * S + q];
        }
    }
    for (int qp = tid; qp < m_pos; qp += kThreads) {
      const int i = __ldg(sv.r_perm + qp);
      if (i >= 0) p.dual_out[b * m + i] = lam[(size_t)qp * S + q];
    }
    if (tid == 0) {
      p.it_out[b] = sc.count[q];
      p.res_out[b] = sc.res_out[q];
      p.gap_out[b] = sc.gap_out[q];
      const bool feas = (p.feasible ? (p.feasible[b] != 0) : true) &&
                        (!kQP || (p.qp_flags & 8) || sc.valid[q]);
      p.conv_out[b] = (sc.conv[q] && feas) ? 1 : 0;
    }
  }
}

// dst[b * npos + p] = perm[p] >= 0 ? src[b * src_stride + perm[p]] : 0.
template <typename T>
__global__ void permute_rows_kernel(const T* src, int64_t src_stride, const int* perm, int npos,
                                    int64_t rows, T* dst) {
  const int64_t total = rows * npos;
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total;
       e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t b = e / npos;
    const int pp = (int)(e - b * npos);
    const int k = perm[pp];
    dst[e] = k >= 0 ? src[b * src_stride + k] : T(0);
  }
}

// Diagonal steps of shared values, one lane per sliced-ELL line: the per-line
// |K| sums in the line's entry order, as SellLines::abs_sum does in the solve.
template <typename T>
__global__ void diagonal_steps_kernel(const int* ptr, int nsl, const T* vals, T safety, bool rows,
                                      T* sigma, T* tau, T* a, T* d) {
  const int lane = threadIdx.x & 31;
  const int warps = (int)(blockDim.x >> 5) * gridDim.x;
  for (int sl = (int)(blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5)); sl < nsl; sl += warps) {
    const int e0 = ptr[sl];
    const int width = (ptr[sl + 1] - e0) / kC;
    T acc = T(0);
    for (int k = 0, e = e0 + lane; k < width; ++k, e += kC) acc = acc + fabs(vals[e]) * T(1);
    const int pos = sl * kC + lane;
    const T step = safety / (acc > T(0) ? pmax(acc, T(1e-12)) : T(1));
    if (rows) {
      sigma[pos] = step;
    } else {
      const T aa = T(1) / (T(1) + step * T(1));
      tau[pos] = step;
      a[pos] = aa;
      d[pos] = step * aa;
    }
  }
}

// Per-sample values in SELL order: out[b * count + e] = values[b * stride + slot[e]].
template <typename T>
__global__ void arrange_sample_values_kernel(const T* values, int64_t stride, const int* slot,
                                             int count, int64_t batch, T* out) {
  const int64_t total = batch * (int64_t)count;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t b = i / count;
    const int e = (int)(i - b * count);
    const int sl = slot[e];
    out[i] = sl >= 0 ? values[b * stride + sl] : T(0);
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

template <typename T, int S, int NT, bool kShared, bool kQP>
cudaError_t launch_s(const FwdParams<T>& p, bool smem, size_t smem_bytes, cudaStream_t stream) {
  const unsigned grid = (unsigned)((p.batch + S - 1) / S);
  if (smem) {
    auto kern = cp_forward_kernel<T, S, NT, true, kShared, kQP>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem_bytes);
    if (e != cudaSuccess) return e;
    kern<<<grid, NT, smem_bytes, stream>>>(p);
  } else {
    if constexpr (NT == kForwardThreads) {
      cp_forward_kernel<T, S, NT, false, kShared, kQP><<<grid, NT, 0, stream>>>(p);
    } else {
      return cudaErrorInvalidValue;
    }
  }
  return cudaGetLastError();
}

// Instantiated shapes: S = 1, 2, 4, 8 with kForwardThreads threads; S = 1 with
// 2 or 4 times as many; and the wide multi-sample tiles of PURIN_WIDE_TILES
// (not built for the QP), for samples so large that one tile fills an SM: its
// samples share every structure load, and its threads keep the SM's warps.
// The diagonal QP is built for the one-sample shapes only, plus one-sample
// tiles of kNarrowThreads threads.
template <typename T, bool kShared, bool kQP>
cudaError_t launch_shared(const FwdParams<T>& p, int S, int NT, bool smem, size_t smem_bytes,
                          cudaStream_t stream) {
  if constexpr (kQP) {
    if (NT == kNarrowThreads)
      return S == 1 && smem ? launch_s<T, 1, kNarrowThreads, kShared, true>(p, smem, smem_bytes,
                                                                            stream)
                            : cudaErrorInvalidValue;
  }
  if (S == 1 && NT == 2 * kForwardThreads)
    return launch_s<T, 1, 2 * kForwardThreads, kShared, kQP>(p, smem, smem_bytes, stream);
  if (S == 1 && NT == kWideThreads) return launch_s<T, 1, kWideThreads, kShared, kQP>(p, smem, smem_bytes, stream);
  if constexpr (!kQP) {
#define PURIN_WIDE_TILE(SS, NN) \
  if (S == SS && NT == NN) return launch_s<T, SS, NN, kShared, false>(p, smem, smem_bytes, stream);
    PURIN_WIDE_TILES
#undef PURIN_WIDE_TILE
  }
  if (NT != kForwardThreads) return cudaErrorInvalidValue;
  if constexpr (kQP) {
    return S == 1 ? launch_s<T, 1, kForwardThreads, kShared, true>(p, smem, smem_bytes, stream)
                  : cudaErrorInvalidValue;
  } else {
    switch (S) {
      case 1: return launch_s<T, 1, kForwardThreads, kShared, false>(p, smem, smem_bytes, stream);
      case 2: return launch_s<T, 2, kForwardThreads, kShared, false>(p, smem, smem_bytes, stream);
      case 4: return launch_s<T, 4, kForwardThreads, kShared, false>(p, smem, smem_bytes, stream);
      case 8: return launch_s<T, 8, kForwardThreads, kShared, false>(p, smem, smem_bytes, stream);
      default: return cudaErrorInvalidValue;
    }
  }
}

template <typename T, int S, int NT, bool kShared, bool kQP>
int blocks_per_sm_s(size_t smem_bytes) {
  auto kern = cp_forward_kernel<T, S, NT, true, kShared, kQP>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_bytes) !=
      cudaSuccess)
    return 0;
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, NT, smem_bytes) != cudaSuccess)
    return 0;
  return per_sm;
}

template <typename T, bool kShared, bool kQP>
int blocks_per_sm_shared(int S, int NT, size_t smem_bytes) {
  if constexpr (kQP) {
    if (NT == kNarrowThreads)
      return S == 1 ? blocks_per_sm_s<T, 1, kNarrowThreads, kShared, true>(smem_bytes) : 0;
  }
  if (S == 1 && NT == 2 * kForwardThreads)
    return blocks_per_sm_s<T, 1, 2 * kForwardThreads, kShared, kQP>(smem_bytes);
  if (S == 1 && NT == kWideThreads) return blocks_per_sm_s<T, 1, kWideThreads, kShared, kQP>(smem_bytes);
  if constexpr (!kQP) {
#define PURIN_WIDE_TILE(SS, NN) \
  if (S == SS && NT == NN) return blocks_per_sm_s<T, SS, NN, kShared, false>(smem_bytes);
    PURIN_WIDE_TILES
#undef PURIN_WIDE_TILE
  }
  if (NT != kForwardThreads) return 0;
  if constexpr (kQP) {
    return S == 1 ? blocks_per_sm_s<T, 1, kForwardThreads, kShared, true>(smem_bytes) : 0;
  } else {
    switch (S) {
      case 1: return blocks_per_sm_s<T, 1, kForwardThreads, kShared, false>(smem_bytes);
      case 2: return blocks_per_sm_s<T, 2, kForwardThreads, kShared, false>(smem_bytes);
      case 4: return blocks_per_sm_s<T, 4, kForwardThreads, kShared, false>(smem_bytes);
      case 8: return blocks_per_sm_s<T, 8, kForwardThreads, kShared, false>(smem_bytes);
      default: return 0;
    }
  }
}

}  // namespace

// The kernels of one (T, kShared, kQP) combination.  The library compiles this
// file once per combination with PURIN_FWD_PART_T / _SHARED / _QP defined (those
// objects instantiate only that combination's kernels, in parallel) and once
// without, for everything else, which links against the parts.
template <typename T, bool kShared, bool kQP>
cudaError_t forward_part_launch(const FwdParams<T>& p, int S, int NT, bool smem, size_t smem_bytes,
                                cudaStream_t stream);
template <typename T, bool kShared, bool kQP>
int forward_part_blocks(int S, int NT, size_t smem_bytes);

#if defined(PURIN_FWD_PART_T)

template <typename T, bool kShared, bool kQP>
cudaError_t forward_part_launch(const FwdParams<T>& p, int S, int NT, bool smem, size_t smem_bytes,
                                cudaStream_t stream) {
  return launch_shared<T, kShared, kQP>(p, S, NT, smem, smem_bytes, stream);
}
template <typename T, bool kShared, bool kQP>
int forward_part_blocks(int S, int NT, size_t smem_bytes) {
  return blocks_per_sm_shared<T, kShared, kQP>(S, NT, smem_bytes);
}
template cudaError_t forward_part_launch<PURIN_FWD_PART_T, PURIN_FWD_PART_SHARED, PURIN_FWD_PART_QP>(
    const FwdParams<PURIN_FWD_PART_T>&, int, int, bool, size_t, cudaStream_t);
template int forward_part_blocks<PURIN_FWD_PART_T, PURIN_FWD_PART_SHARED, PURIN_FWD_PART_QP>(int, int,
                                                                                          size_t);

#else  // the library's other forward functions

#define PURIN_FWD_EXTERN(T, SH, QP)                                                              \
  extern template cudaError_t forward_part_launch<T, SH, QP>(const FwdParams<T>&, int, int, bool, \
                                                             size_t, cudaStream_t);              \
  extern template int forward_part_blocks<T, SH, QP>(int, int, size_t);
PURIN_FWD_EXTERN(double, true, true)
PURIN_FWD_EXTERN(double, true, false)
PURIN_FWD_EXTERN(double, false, true)
PURIN_FWD_EXTERN(double, false, false)
PURIN_FWD_EXTERN(float, true, true)
PURIN_FWD_EXTERN(float, true, false)
PURIN_FWD_EXTERN(float, false, true)
PURIN_FWD_EXTERN(float, false, false)
#undef PURIN_FWD_EXTERN

template <typename T>
int forward_blocks_per_sm(int S, int NT, bool shared_values, size_t smem_bytes, bool qp) {
  if (qp)
    return shared_values ? forward_part_blocks<T, true, true>(S, NT, smem_bytes)
                         : forward_part_blocks<T, false, true>(S, NT, smem_bytes);
  return shared_values ? forward_part_blocks<T, true, false>(S, NT, smem_bytes)
                       : forward_part_blocks<T, false, false>(S, NT, smem_bytes);
}

template <typename T>
size_t forward_static_smem(int S, int NT) {
  if (NT == kNarrowThreads) return sizeof(TileScratch<T, 1, kNarrowThreads / 32>);
  if (S == 1 && NT == 2 * kForwardThreads) return sizeof(TileScratch<T, 1, 2 * kForwardThreads / 32>);
  if (S == 1 && NT == kWideThreads) return sizeof(TileScratch<T, 1, kWideThreads / 32>);
#define PURIN_WIDE_TILE(SS, NN) \
  if (S == SS && NT == NN) return sizeof(TileScratch<T, SS, NN / 32>);
  PURIN_WIDE_TILES
#undef PURIN_WIDE_TILE
  switch (S) {
    case 1: return sizeof(TileScratch<T, 1, kForwardThreads / 32>);
    case 2: return sizeof(TileScratch<T, 2, kForwardThreads / 32>);
    case 4: return sizeof(TileScratch<T, 4, kForwardThreads / 32>);
    default: return sizeof(TileScratch<T, 8, kForwardThreads / 32>);
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
cudaError_t diagonal_steps(const SellView& sv, const T* vr, const T* vc, T safety, T* sigma, T* tau,
                           T* a, T* d, cudaStream_t stream) {
  const int threads = 256, per_block = threads / 32;
  if (sv.nsl_r > 0)
    diagonal_steps_kernel<T><<<(sv.nsl_r + per_block - 1) / per_block, threads, 0, stream>>>(
        sv.r_ptr, sv.nsl_r, vr, safety, true, sigma, tau, a, d);
  if (sv.nsl_c > 0)
    diagonal_steps_kernel<T><<<(sv.nsl_c + per_block - 1) / per_block, threads, 0, stream>>>(
        sv.c_ptr, sv.nsl_c, vc, safety, false, sigma, tau, a, d);
  return cudaGetLastError();
}

template <typename T>
cudaError_t arrange_sample_values(const T* values, int64_t stride, const int* slot, int count,
                                  int64_t batch, T* out, cudaStream_t stream) {
  const int64_t total = batch * (int64_t)count;
  if (total <= 0) return cudaSuccess;
  const int threads = 256;
  const int64_t want = (total + threads - 1) / threads;
  const int blocks = want < 4736 ? (int)want : 4736;
  arrange_sample_values_kernel<T><<<blocks, threads, 0, stream>>>(values, stride, slot, count, batch, out);
  return cudaGetLastError();
}

template <typename T>
cudaError_t permute_rows(const T* src, int64_t src_stride, const int* perm, int npos, int64_t rows,
                         T* dst, cudaStream_t stream) {
  const int64_t total = rows * (int64_t)npos;
  if (total <= 0) return cudaSuccess;
  const int threads = 256;
  const int64_t want = (total + threads - 1) / threads;
  const int blocks = want < 2368 ? (int)want : 2368;
  permute_rows_kernel<T><<<blocks, threads, 0, stream>>>(src, src_stride, perm, npos, rows, dst);
  return cudaGetLastError();
}

template <typename T>
cudaError_t launch_forward(const FwdParams<T>& p, int S, int NT, bool smem, size_t smem_bytes,
                           cudaStream_t stream) {
  if (p.q_i)
    return p.vr ? forward_part_launch<T, true, true>(p, S, NT, smem, smem_bytes, stream)
                : forward_part_launch<T, false, true>(p, S, NT, smem, smem_bytes, stream);
  return p.vr ? forward_part_launch<T, true, false>(p, S, NT, smem, smem_bytes, stream)
              : forward_part_launch<T, false, false>(p, S, NT, smem, smem_bytes, stream);
}

template cudaError_t launch_forward<double>(const FwdParams<double>&, int, int, bool, size_t,
                                            cudaStream_t);
template cudaError_t launch_forward<float>(const FwdParams<float>&, int, int, bool, size_t,
                                           cudaStream_t);
template int forward_blocks_per_sm<double>(int, int, bool, size_t, bool);
template int forward_blocks_per_sm<float>(int, int, bool, size_t, bool);
template size_t forward_static_smem<double>(int, int);
template size_t forward_static_smem<float>(int, int);
template cudaError_t arrange_values<double>(const double*, const int*, int, double*, cudaStream_t);
template cudaError_t arrange_values<float>(const float*, const int*, int, float*, cudaStream_t);
template cudaError_t diagonal_steps<double>(const SellView&, const double*, const double*, double,
                                            double*, double*, double*, double*, cudaStream_t);
template cudaError_t diagonal_steps<float>(const SellView&, const float*, const float*, float, float*,
                                           float*, float*, float*, cudaStream_t);
template cudaError_t arrange_sample_values<double>(const double*, int64_t, const int*, int, int64_t,
                                                   double*, cudaStream_t);
template cudaError_t arrange_sample_values<float>(const float*, int64_t, const int*, int, int64_t,
                                                  float*, cudaStream_t);
template cudaError_t permute_rows<double>(const double*, int64_t, const int*, int, int64_t, double*,
                                          cudaStream_t);
template cudaError_t permute_rows<float>(const float*, int64_t, const int*, int, int64_t, float*,
                                         cudaStream_t);

#endif  // PURIN_FWD_PART_T

}  // namespace purin
