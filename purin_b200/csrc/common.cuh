// Shared device helpers for the CP kernels (sm_100a).
//
// Arithmetic conventions (all kernels are compiled with -fmad=false so every
// product and sum is rounded separately, as in the reference's elementwise
// JAX code):
//   * pmax/pmin propagate NaN like jax.lax.max/min (kernels.py uses jnp.maximum,
//     jnp.minimum and jnp.clip = minimum(upper, maximum(lower, x))).
//   * Sparse sums accumulate sequentially from zero in the reference's
//     row/slot order (linalg/sparse/operators.py:507-533).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace purin {

constexpr unsigned kFullMask = 0xffffffffu;

template <typename T>
__device__ __forceinline__ T pmax(T a, T b) {
  return (a > b || a != a) ? a : b;
}
template <typename T>
__device__ __forceinline__ T pmin(T a, T b) {
  return (a < b || a != a) ? a : b;
}
// jnp.clip(x, lo, hi) == minimum(hi, maximum(lo, x))
template <typename T>
__device__ __forceinline__ T clip(T x, T lo, T hi) {
  return pmin(hi, pmax(lo, x));
}
template <typename T>
__device__ __forceinline__ bool finite(T x) {
  return isfinite(x);
}
// nan_to_num(x, nan=0, posinf=0, neginf=0)
template <typename T>
__device__ __forceinline__ T clean(T x) {
  return isfinite(x) ? x : T(0);
}

// JAX's max/min JVP weight for argument x of op(x, other) = ans:
// (x == ans) / (other == ans ? 2 : 1)  -> one of {0, 0.5, 1}; returned as a code
// 0 -> 0, 1 -> 0.5, 2 -> 1.
template <typename T>
__device__ __forceinline__ int balanced_code(T x, T ans, T other) {
  if (!(x == ans)) return 0;
  return (other == ans) ? 1 : 2;
}
// Product of two balanced codes as a 2-bit code: 0 -> 0, 1 -> 0.25, 2 -> 0.5, 3 -> 1.
__device__ __forceinline__ int product_code(int a, int b) {
  if (a == 0 || b == 0) return 0;
  const int e = (2 - a) + (2 - b);  // halvings: 0, 1 or 2
  return 3 - e;
}
template <typename T>
__device__ __forceinline__ T code_factor(int code) {
  return code == 3 ? T(1) : (code == 2 ? T(0.5) : (code == 1 ? T(0.25) : T(0)));
}
template <typename T>
__device__ __forceinline__ T balanced_factor(int code) {
  return code == 2 ? T(1) : (code == 1 ? T(0.5) : T(0));
}

// ---------------------------------------------------------------------------
// Threefry-2x32 with 20 rounds (Salmon et al., SC'11) and JAX's key/bits scheme.
__device__ __forceinline__ uint32_t rotl32(uint32_t x, int r) {
  return (x << r) | (x >> (32 - r));
}

__device__ __forceinline__ void threefry2x32(uint32_t k0, uint32_t k1, uint32_t& x0,
                                             uint32_t& x1) {
  const uint32_t k2 = k0 ^ k1 ^ 0x1BD11BDAu;
  const int r0[4] = {13, 15, 26, 6};
  const int r1[4] = {17, 29, 16, 24};
  x0 += k0;
  x1 += k1;
#pragma unroll
  for (int i = 0; i < 4; ++i) { x0 += x1; x1 = rotl32(x1, r0[i]); x1 ^= x0; }
  x0 += k1; x1 += k2 + 1u;
#pragma unroll
  for (int i = 0; i < 4; ++i) { x0 += x1; x1 = rotl32(x1, r1[i]); x1 ^= x0; }
  x0 += k2; x1 += k0 + 2u;
#pragma unroll
  for (int i = 0; i < 4; ++i) { x0 += x1; x1 = rotl32(x1, r0[i]); x1 ^= x0; }
  x0 += k0; x1 += k1 + 3u;
#pragma unroll
  for (int i = 0; i < 4; ++i) { x0 += x1; x1 = rotl32(x1, r1[i]); x1 ^= x0; }
  x0 += k1; x1 += k2 + 4u;
#pragma unroll
  for (int i = 0; i < 4; ++i) { x0 += x1; x1 = rotl32(x1, r0[i]); x1 ^= x0; }
  x0 += k2; x1 += k0 + 5u;
}

// Legacy threefry_2x32(key, iota(count)) word `w` (count words in total).
__device__ __forceinline__ uint32_t threefry_legacy_word(uint32_t k0, uint32_t k1,
                                                         uint64_t count, uint64_t w) {
  const uint64_t padded = count + (count & 1);
  const uint64_t half = padded / 2;
  const uint64_t pair = (w < half) ? w : w - half;
  uint32_t x0 = (uint32_t)pair;
  const uint64_t second = pair + half;
  uint32_t x1 = (second < count) ? (uint32_t)second : 0u;
  threefry2x32(k0, k1, x0, x1);
  return (w < half) ? x0 : x1;
}

// Child key `index` of split(PRNGKey(seed), total).
__device__ __forceinline__ void split_key(int64_t seed, int64_t index, int64_t total,
                                          bool partitionable, uint32_t& k0, uint32_t& k1) {
  const uint32_t s0 = (uint32_t)(((uint64_t)seed >> 32) & 0xffffffffu);
  const uint32_t s1 = (uint32_t)((uint64_t)seed & 0xffffffffu);
  if (partitionable) {
    uint32_t x0 = (uint32_t)((uint64_t)index >> 32);
    uint32_t x1 = (uint32_t)((uint64_t)index & 0xffffffffu);
    threefry2x32(s0, s1, x0, x1);
    k0 = x0;
    k1 = x1;
  } else {
    const uint64_t count = 2 * (uint64_t)total;
    k0 = threefry_legacy_word(s0, s1, count, 2 * (uint64_t)index);
    k1 = threefry_legacy_word(s0, s1, count, 2 * (uint64_t)index + 1);
  }
}

template <typename T> struct NormalBits;
template <> struct NormalBits<double> {
  __device__ static double draw(uint32_t k0, uint32_t k1, int64_t j, int64_t n,
                                bool partitionable) {
    uint64_t bits;
    if (partitionable) {
      uint32_t x0 = (uint32_t)((uint64_t)j >> 32), x1 = (uint32_t)((uint64_t)j & 0xffffffffu);
      threefry2x32(k0, k1, x0, x1);
      bits = ((uint64_t)x0 << 32) | (uint64_t)x1;
    } else {
      const uint64_t words = 2 * (uint64_t)n;
      const uint32_t hi = threefry_legacy_word(k0, k1, words, (uint64_t)j);
      const uint32_t lo = threefry_legacy_word(k0, k1, words, (uint64_t)n + (uint64_t)j);
      bits = ((uint64_t)hi << 32) | (uint64_t)lo;
    }
    const uint64_t fb = (bits >> 12) | 0x3FF0000000000000ull;
    const double f = __longlong_as_double((long long)fb) - 1.0;
    const double lo = __longlong_as_double((long long)0xBFEFFFFFFFFFFFFFull);  // nextafter(-1, 0)
    const double hi = 1.0;
    const double u = pmax(lo, f * (hi - lo) + lo);
    return 1.4142135623730951 * erfinv(u);
  }
};
template <> struct NormalBits<float> {
  __device__ static float draw(uint32_t k0, uint32_t k1, int64_t j, int64_t n,
                               bool partitionable) {
    uint32_t bits;
    if (partitionable) {
      uint32_t x0 = (uint32_t)((uint64_t)j >> 32), x1 = (uint32_t)((uint64_t)j & 0xffffffffu);
      threefry2x32(k0, k1, x0, x1);
      bits = x0 ^ x1;
    } else {
      bits = threefry_legacy_word(k0, k1, (uint64_t)n, (uint64_t)j);
    }
    const uint32_t fb = (bits >> 9) | 0x3F800000u;
    const float f = __uint_as_float(fb) - 1.0f;
    const float lo = __uint_as_float(0xBF7FFFFFu);  // nextafter(-1f, 0f)
    const float hi = 1.0f;
    const float u = pmax(lo, f * (hi - lo) + lo);
    return 1.41421356f * erfinvf(u);
  }
};

// ---------------------------------------------------------------------------
// Reductions.
template <typename T>
__device__ __forceinline__ T shfl_xor(T v, int o) {
  return __shfl_xor_sync(kFullMask, v, o);
}

// Sum / NaN-propagating max across the lanes of a warp that share lane % S.
template <int S, typename T>
__device__ __forceinline__ T group_sum(T v) {
#pragma unroll
  for (int o = S; o < 32; o <<= 1) v += shfl_xor(v, o);
  return v;
}
template <int S, typename T>
__device__ __forceinline__ T group_max(T v) {
#pragma unroll
  for (int o = S; o < 32; o <<= 1) v = pmax(v, shfl_xor(v, o));
  return v;
}
template <int S>
__device__ __forceinline__ int group_and(int v) {
#pragma unroll
  for (int o = S; o < 32; o <<= 1) v &= __shfl_xor_sync(kFullMask, v, o);
  return v;
}

// ---------------------------------------------------------------------------
// Bounded grid barrier for cooperative launches.  Waits give up after
// `timeout_ns`, set `error` and return false; every later barrier returns false
// immediately so all blocks drain out of the kernel.
struct GridBarrier {
  unsigned int count;
  unsigned int generation;
  int error;
  int pad;
};

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ inline bool grid_barrier(GridBarrier* gb, unsigned int nblocks, uint64_t timeout_ns) {
  __shared__ int s_ok;
  __syncthreads();
  if (threadIdx.x == 0) {
    volatile unsigned int* vgen = &gb->generation;
    volatile int* verr = &gb->error;
    int ok = (*verr == 0);
    if (ok) {
      const unsigned int gen = *vgen;
      __threadfence();
      const unsigned int arrived = atomicAdd(&gb->count, 1u);
      if (arrived == nblocks - 1) {
        atomicExch(&gb->count, 0u);
        __threadfence();
        atomicAdd(&gb->generation, 1u);
      } else {
        const uint64_t start = global_timer_ns();
        unsigned int spins = 0;
        while (*vgen == gen) {
          if (*verr != 0) { ok = 0; break; }
          __nanosleep(128);
          if ((++spins & 1023u) == 0 && global_timer_ns() - start > timeout_ns) {
            atomicExch(&gb->error, 1);
            ok = 0;
            break;
          }
          if (spins > 0x7fffffffu) { atomicExch(&gb->error, 1); ok = 0; break; }
        }
      }
      __threadfence();
    }
    s_ok = ok;
  }
  __syncthreads();
  return s_ok != 0;
}

}  // namespace purin
