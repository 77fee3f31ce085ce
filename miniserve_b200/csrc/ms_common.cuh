// Shared device helpers for the sampling kernels: order-preserving keys,
// logit loading with the allowed-token mask, and warp/block reductions/scans.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/mssample.h"

namespace ms {

constexpr uint32_t kNegInfBits = 0xFF800000u;
constexpr uint32_t kPosInfBits = 0x7F800000u;
constexpr uint32_t kNegInfKey = 0x007FFFFFu;  // key of -inf: every valid key is larger
constexpr int kNoCut = 0x7FFFFFFF;            // "all ties kept"
constexpr int32_t kRowPending = 1 << 30;      // internal status: row left for the generic kernel

// fp32 bit pattern -> uint32 whose unsigned order is the float order.
__device__ __forceinline__ uint32_t bits_to_key(uint32_t u) {
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float key_to_float(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k);
}

// Order key of a finite-or-(-inf) float; -0 and +0 share a key, since the
// reference compares values, not bit patterns.
__device__ __forceinline__ uint32_t fkey(float v) {
  uint32_t u = __float_as_uint(v);
  if (u == 0x80000000u) u = 0u;
  return bits_to_key(u);
}

// Raw fp32 bits of logit i (bf16 widened exactly).
template <int DT>
__device__ __forceinline__ uint32_t raw_bits(const void *row, int i) {
  if (DT == MS_DTYPE_F32) return __ldg(reinterpret_cast<const unsigned int *>(row) + i);
  return static_cast<uint32_t>(__ldg(reinterpret_cast<const unsigned short *>(row) + i)) << 16;
}

// Clean a logit: masked -> -inf, NaN -> -inf (flagged), +inf flagged,
// -0 -> +0 (equal values must get equal keys: the reference compares values).
__device__ __forceinline__ uint32_t clean_bits(uint32_t u, bool allowed, uint32_t &flags) {
  if (!allowed) return kNegInfBits;
  if ((u & 0x7FFFFFFFu) > kPosInfBits) {
    flags |= MS_ROW_NONFINITE;
    return kNegInfBits;
  }
  if (u == kPosInfBits) flags |= MS_ROW_NONFINITE;
  if (u == 0x80000000u) u = 0u;
  return u;
}

__device__ __forceinline__ bool mask_allows(const uint32_t *mask_row, int i) {
  return mask_row == nullptr || ((__ldg(mask_row + (i >> 5)) >> (i & 31)) & 1u);
}

// Threshold predicate produced by a top-k or top-p cut: an element is kept
// when its key is above `key`, or equal to it with index <= `cut` (ties are
// taken in index order, like the reference's stable sorts).
struct Cut {
  uint32_t key;
  int cut;
};
__device__ __forceinline__ bool kept(const Cut &c, uint32_t key, int idx) {
  return key > c.key || (key == c.key && idx <= c.cut);
}
__device__ __forceinline__ Cut cut_all() { return Cut{kNegInfKey + 1u, kNoCut}; }

// exp(logit/T - max/T) in float64.  `dmax` is (double)max; `inv_t` is 1/T.
__device__ __forceinline__ double weight_of(float v, double dmax, double inv_t) {
  return exp(((double)v - dmax) * inv_t);
}

// ---------------------------------------------------------------- warp level
__device__ __forceinline__ double warp_sum(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
  return v;
}
__device__ __forceinline__ uint32_t warp_sum_u32(uint32_t v) {
  return __reduce_add_sync(0xFFFFFFFFu, v);
}
__device__ __forceinline__ int warp_min_i(int v) { return __reduce_min_sync(0xFFFFFFFFu, v); }

// (key, idx) max with lowest index on ties.
__device__ __forceinline__ void warp_argmax(uint32_t &key, int &idx) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    uint32_t k2 = __shfl_xor_sync(0xFFFFFFFFu, key, o);
    int i2 = __shfl_xor_sync(0xFFFFFFFFu, idx, o);
    if (k2 > key || (k2 == key && i2 < idx)) {
      key = k2;
      idx = i2;
    }
  }
}

// --------------------------------------------------------------- block level
// All helpers below must be called by every thread of the block; `red` is a
// shared scratch of at least 32 slots of the given type.  They end with a
// __syncthreads so the scratch can be reused immediately.
template <int NT>
__device__ __forceinline__ double block_sum(double v, double *red) {
  constexpr int NW = NT / 32;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = warp_sum(v);
  if (lane == 0) red[warp] = v;
  __syncthreads();
  double t = 0.0;
  if (threadIdx.x < 32) {
    t = lane < NW ? red[lane] : 0.0;
    t = warp_sum(t);
    if (lane == 0) red[32] = t;
  }
  __syncthreads();
  t = red[32];
  __syncthreads();
  return t;
}

template <int NT>
__device__ __forceinline__ uint32_t block_sum_u32(uint32_t v, uint32_t *red) {
  constexpr int NW = NT / 32;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = warp_sum_u32(v);
  if (lane == 0) red[warp] = v;
  __syncthreads();
  if (threadIdx.x < 32) {
    uint32_t t = lane < NW ? red[lane] : 0u;
    t = warp_sum_u32(t);
    if (lane == 0) red[32] = t;
  }
  __syncthreads();
  uint32_t t = red[32];
  __syncthreads();
  return t;
}

template <int NT>
__device__ __forceinline__ int block_min_i(int v, int *red) {
  constexpr int NW = NT / 32;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = warp_min_i(v);
  if (lane == 0) red[warp] = v;
  __syncthreads();
  if (threadIdx.x < 32) {
    int t = lane < NW ? red[lane] : 0x7FFFFFFF;
    t = warp_min_i(t);
    if (lane == 0) red[32] = t;
  }
  __syncthreads();
  int t = red[32];
  __syncthreads();
  return t;
}

template <int NT>
__device__ __forceinline__ float block_max_f(float v, float *red) {
  constexpr int NW = NT / 32;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xFFFFFFFFu, v, o));
  if (lane == 0) red[warp] = v;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = lane < NW ? red[lane] : -INFINITY;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t = fmaxf(t, __shfl_xor_sync(0xFFFFFFFFu, t, o));
    if (lane == 0) red[32] = t;
  }
  __syncthreads();
  const float t = red[32];
  __syncthreads();
  return t;
}

// Exclusive and inclusive prefix sums over threads in thread order.
template <int NT, typename T>
__device__ __forceinline__ void block_scan(T v, T &excl, T &incl, T &total, T *red) {
  constexpr int NW = NT / 32;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  T x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    T y = __shfl_up_sync(0xFFFFFFFFu, x, o);
    if (lane >= o) x += y;
  }
  T xprev = __shfl_up_sync(0xFFFFFFFFu, x, 1);
  if (lane == 0) xprev = T(0);
  if (lane == 31) red[warp] = x;
  __syncthreads();
  if (threadIdx.x < 32) {
    T w = lane < NW ? red[lane] : T(0);
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      T y = __shfl_up_sync(0xFFFFFFFFu, w, o);
      if (lane >= o) w += y;
    }
    red[lane] = w;  // inclusive scan of warp totals
  }
  __syncthreads();
  T base = warp ? red[warp - 1] : T(0);
  excl = base + xprev;
  incl = base + x;
  total = red[NW - 1];
  __syncthreads();
}

}  // namespace ms
