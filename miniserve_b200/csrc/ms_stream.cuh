// Streaming sampling kernel: one 512-thread CTA per logits row, two CTAs per
// SM.  The row streams from HBM through a ring of shared-memory stages filled
// by cp.async.bulk (TMA) copies, so a CTA never holds more than three 4096-
// element chunks and every synchronisation is CTA-local.
//
//   argmax rows (temperature 0, or top_k == 1)  one pass: per-thread first
//                                                maximum, block argmax
//   top-k rows (2 <= top_k <= kStTopK)          one pass: adaptive threshold
//                                                + candidate buffer, exact
//                                                finish on <= top_k entries
//   top-p-only / full-softmax rows              pass 1 (HBM) for the maximum;
//                                                later passes re-read the row
//                                                from L2 (it is loaded with
//                                                an L2 evict-last hint)
//
// Semantics follow miniserve/sampler.py:23-68 (see ms_sample.cu).  Rows
// outside what this kernel finishes exactly (NaN or +inf logits, top_k above
// kStTopK that may still cut, candidate buffers overflowing on heavy ties)
// get status kRowPending and are finished by ms_generic_pending_kernel.
#pragma once

#include "ms_common.cuh"
#include "ms_generic.cuh"

namespace ms {

constexpr int kStThreads = 512;
constexpr int kStWarps = kStThreads / 32;
constexpr int kSub = kStThreads * 4;  // elements per sub-chunk: 4 consecutive per thread
constexpr int kChunk = 2 * kSub;      // elements per chunk (one TMA copy)
constexpr int kStages = 3;
constexpr int kCandCap = 4096;        // candidate buffer entries
constexpr int kStTopK = 256;          // largest top_k resolved by the streaming pass
constexpr int kSBins = 2048;          // x-grid bins (top-p)
constexpr float kSXRange = 40.0f;     // grid depth, units of x = logit / T
constexpr int kMaxSubs = 1024;        // sub-chunk totals kept per row (V <= 2^21)

struct StShared {
  alignas(128) unsigned char stage[kStages][kChunk * 4];
  union {
    struct {
      uint32_t key[kCandCap];
      int idx[kCandCap];
    } c;
    struct {
      uint32_t cnt[kSBins];
      float mass[kSBins];
    } h;
  } w;
  uint32_t tmaxk[kStThreads];  // per-thread maxima as keys (top-k bound)
  double subsum[kMaxSubs];
  uint32_t hist256[256];
  unsigned long long full[kStages];
  double redd[33];
  uint32_t redu[33];
  int redi[33];
  float redf[33];
  int bcast_i[8];
  float bcast_f[4];
  double bcast_d[4];
  int ncand;
};

// ------------------------------------------------------------- the stream
struct StRow {
  const char *g;        // row start in global memory
  const uint32_t *mask; // row of the allowed-token bitmask, or null
  int V;
  int esz;
  bool tma;             // 16-byte aligned row: chunks arrive by TMA
  int nchunks;
};

__device__ __forceinline__ uint32_t st_smem(const void *p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ uint64_t st_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// L2 cache policies for the bulk copies.
__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// Bytes of chunk c delivered by TMA (a multiple of 16); elements past them
// (at most 3 fp32 / 7 bf16 at the row's end) are read from global memory.
__device__ __forceinline__ int tma_elems(const StRow &r, int c) {
  if (!r.tma) return 0;
  const int ne = min(kChunk, r.V - c * kChunk);
  return ((ne * r.esz) & ~15) / r.esz;
}

// thread 0: start the copy of chunk c into stage s
__device__ __forceinline__ void st_issue(StShared &sh, const StRow &r, int c, int s, uint64_t pol) {
  const uint32_t bytes = (uint32_t)(tma_elems(r, c) * r.esz);
  const uint32_t mb = st_smem(&sh.full[s]);
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(mb), "r"(bytes) : "memory");
  if (bytes) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
            st_smem(sh.stage[s])),
        "l"(r.g + (int64_t)c * kChunk * r.esz), "r"(bytes), "r"(mb), "l"(pol)
        : "memory");
  }
}

// all threads: wait for the current phase of stage s; false after ~1 s
__device__ __forceinline__ bool st_wait(StShared &sh, int s, uint32_t parity) {
  const uint32_t mb = st_smem(&sh.full[s]);
  uint32_t done = 0;
  const uint64_t t0 = st_ns();
  for (uint32_t it = 0; !done; ++it) {
    asm volatile(
        "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
        : "=r"(done)
        : "r"(mb), "r"(parity)
        : "memory");
    if (!done && (it & 1023u) == 1023u && st_ns() - t0 > 1000000000ull) return false;
  }
  return true;
}

// Four consecutive elements (chunk-local j, a multiple of 4) of chunk c in
// stage s, masked tokens and positions past the row read as -inf.
template <int DT>
__device__ __forceinline__ void st_get4(const StShared &sh, const StRow &r, int c, int s, int j,
                                        float x[4]) {
  const int ne = min(kChunk, r.V - c * kChunk);
  const int nt = tma_elems(r, c);
  if (j + 4 <= nt) {
    if (DT == MS_DTYPE_F32) {
      const float4 f = reinterpret_cast<const float4 *>(sh.stage[s])[j >> 2];
      x[0] = f.x;
      x[1] = f.y;
      x[2] = f.z;
      x[3] = f.w;
    } else {
      const uint2 h = reinterpret_cast<const uint2 *>(sh.stage[s])[j >> 2];
      x[0] = __uint_as_float(h.x << 16);
      x[1] = __uint_as_float(h.x & 0xFFFF0000u);
      x[2] = __uint_as_float(h.y << 16);
      x[3] = __uint_as_float(h.y & 0xFFFF0000u);
    }
  } else {
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int jj = j + e;
      if (jj >= ne) {
        x[e] = -INFINITY;
      } else if (jj < nt) {
        x[e] = DT == MS_DTYPE_F32
                   ? reinterpret_cast<const float *>(sh.stage[s])[jj]
                   : __uint_as_float((uint32_t)reinterpret_cast<const uint16_t *>(sh.stage[s])[jj] << 16);
      } else {
        const int64_t gi = (int64_t)c * kChunk + jj;
        x[e] = DT == MS_DTYPE_F32
                   ? __ldg(reinterpret_cast<const float *>(r.g) + gi)
                   : __uint_as_float((uint32_t)__ldg(reinterpret_cast<const unsigned short *>(r.g) + gi) << 16);
      }
    }
  }
  if (r.mask) {
    const int gi0 = c * kChunk + j;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int gi = gi0 + e;
      if (gi < r.V && !((__ldg(r.mask + (gi >> 5)) >> (gi & 31)) & 1u)) x[e] = -INFINITY;
    }
  }
}

// One pass over the row.  `body(x[4], gidx0, sub)` sees this thread's 4
// consecutive values of each sub-chunk (gidx0 = global index of x[0]; sub =
// sub-chunk number, index order).  Returns false when a copy timed out
// (after draining).  `ph` carries the stages' phase parities across passes.
template <int DT, class Body>
__device__ bool st_pass(StShared &sh, const StRow &r, uint64_t pol, uint32_t &ph, Body body) {
  const int tid = threadIdx.x;
  bool ok = true;
  if (tid == 0) {
    for (int c = 0; c < kStages && c < r.nchunks; ++c) st_issue(sh, r, c, c, pol);
  }
  for (int c = 0; c < r.nchunks; ++c) {
    const int s = c % kStages;
    if (!st_wait(sh, s, (ph >> s) & 1u)) ok = false;
    ph ^= 1u << s;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      float x[4];
      const int j = h * kSub + tid * 4;
      st_get4<DT>(sh, r, c, s, j, x);
      body(x, c * kChunk + j, c * 2 + h);
    }
    __syncthreads();  // every thread is done with stage s
    if (tid == 0 && c + kStages < r.nchunks) {
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      st_issue(sh, r, c + kStages, s, pol);
    }
  }
  return __syncthreads_and(ok) != 0;
}

// --------------------------------------------------------- block selection
// k-th largest (1-based) among n keys in shared memory, keys with a 0
// "invalid" marker excluded by the caller.  Returns the key; *n_above gets
// the number of keys strictly above it.  4 passes of 8-bit digits.
__device__ uint32_t st_select_kth(StShared &sh, const uint32_t *keys, int n, int k, int *n_above) {
  const int tid = threadIdx.x;
  uint32_t prefix = 0;
  int rem = k, above = 0;
  for (int d = 0; d < 4; ++d) {
    const int shift = 24 - 8 * d;
    for (int b = tid; b < 256; b += kStThreads) sh.hist256[b] = 0u;
    __syncthreads();
    for (int i = tid; i < n; i += kStThreads) {
      const uint32_t key = keys[i];
      if (d > 0 && (key >> (shift + 8)) != prefix) continue;
      atomicAdd(&sh.hist256[(key >> shift) & 255u], 1u);
    }
    __syncthreads();
    // digit whose running count from the top reaches rem
    if (tid < 32) {
      // each lane owns 8 digits, highest digits on lane 0
      uint32_t c8[8], s = 0;
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        c8[q] = sh.hist256[255 - (tid * 8 + q)];
        s += c8[q];
      }
      uint32_t incl = s;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const uint32_t y = __shfl_up_sync(0xFFFFFFFFu, incl, o);
        if (tid >= o) incl += y;
      }
      const uint32_t excl = incl - s;
      const unsigned hit = __ballot_sync(0xFFFFFFFFu, incl >= (uint32_t)rem && excl < (uint32_t)rem);
      if (hit) {
        const int lane = __ffs(hit) - 1;
        if (tid == lane) {
          uint32_t acc = excl;
          for (int q = 0; q < 8; ++q) {
            if (acc + c8[q] >= (uint32_t)rem) {
              sh.bcast_i[0] = 255 - (tid * 8 + q);
              sh.bcast_i[1] = (int)acc;
              break;
            }
            acc += c8[q];
          }
        }
      } else if (tid == 0) {  // fewer than rem keys: cannot happen for valid k
        sh.bcast_i[0] = 0;
        sh.bcast_i[1] = 0;
      }
    }
    __syncthreads();
    const uint32_t digit = (uint32_t)sh.bcast_i[0];
    rem -= sh.bcast_i[1];
    above += sh.bcast_i[1];
    prefix = (prefix << 8) | digit;
    __syncthreads();
  }
  *n_above = above;
  return prefix;
}

// ------------------------------------------------------------ bitonic sort
// Sort n <= cap entries (key, idx) in shared memory into (key desc, index asc)
// order, or by index ascending when by_index.  Pads to a power of two with
// entries that sort last.  All threads.
__device__ void st_sort(uint32_t *key, int *idx, int n, bool by_index) {
  const int tid = threadIdx.x;
  int N = 1;
  while (N < n) N <<= 1;
  for (int i = n + tid; i < N; i += kStThreads) {
    key[i] = 0u;
    idx[i] = 0x7FFFFFFF;
  }
  __syncthreads();
  auto before = [&](int a, int b) -> bool {  // entry a sorts before entry b
    if (by_index) return idx[a] < idx[b];
    return key[a] > key[b] || (key[a] == key[b] && idx[a] < idx[b]);
  };
  for (int size = 2; size <= N; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int t = tid; t < (N >> 1); t += kStThreads) {
        const int i = 2 * t - (t & (stride - 1));
        const int j = i + stride;
        const bool up = ((i & size) == 0);  // this block sorts in the final order
        const bool swap = up ? before(j, i) : before(i, j);
        if (swap) {
          const uint32_t tk = key[i];
          key[i] = key[j];
          key[j] = tk;
          const int ti = idx[i];
          idx[i] = idx[j];
          idx[j] = ti;
        }
      }
      __syncthreads();
    }
  }
}

// Index-order inverse CDF over m entries already sorted by index, weight w(i)
// (zero = not kept).  total is the kept set's weight.  Writes the row.
template <class W>
__device__ void st_draw_sorted(StShared &sh, const SampleArgs &a, int row, const int *idx, int m,
                               double total, double U, W w) {
  const int tid = threadIdx.x;
  if (!(U > 0.0)) {  // r == 0 stops at index 0 (miniserve/sampler.py:66)
    if (tid == 0) write_row(a, row, 0, (float)((m > 0 && idx[0] == 0 ? w(0) : 0.0) / total), 0);
    return;
  }
  const double target = U * total;
  const int per = (m + kStThreads - 1) / kStThreads;
  const int p0 = tid * per, p1 = min(m, p0 + per);
  double s = 0.0;
  for (int i = p0; i < p1; ++i) s += w(i);
  double ex, inc, tot;
  block_scan<kStThreads, double>(s, ex, inc, tot, sh.redd);
  const int who = block_min_i<kStThreads>((s > 0.0 && inc >= target) ? tid : 0x7FFFFFFF, sh.redi);
  if (who == 0x7FFFFFFF) {  // ran past the end (miniserve/sampler.py:68)
    if (tid == 0)
      write_row(a, row, a.V - 1, (float)((m > 0 && idx[m - 1] == a.V - 1 ? w(m - 1) : 0.0) / total), 0);
    return;
  }
  if (tid == who) {
    double acc = ex;
    int tok = -1, last = -1;
    double wt = 0.0, wl = 0.0;
    for (int i = p0; i < p1; ++i) {
      const double wi = w(i);
      if (wi <= 0.0) continue;
      acc += wi;
      last = idx[i];
      wl = wi;
      if (acc >= target) {
        tok = idx[i];
        wt = wi;
        break;
      }
    }
    if (tok < 0) {
      tok = last;
      wt = wl;
    }
    write_row(a, row, tok, (float)(wt / total), 0);
  }
}

// Exact finish over a candidate set that contains the top-k (or nucleus) set:
// entries (key, idx) in sh.w.c, n of them.  m_keep0 = entries kept before
// top-p (top_k, or all); total0 = the softmax normaliser over that set when
// known (<= 0: compute it over the m_keep0 best entries).  float64 weights
// exp(l/T - max/T) as in miniserve/sampler.py:35,45; top-p in sorted order
// (sampler.py:50-57); index-order draw (sampler.py:62-68).
__device__ void st_finish_set(StShared &sh, const SampleArgs &a, int row, int n, int m_keep0,
                              double total0, double T, double P, double U, float vmax) {
  const int tid = threadIdx.x;
  uint32_t *key = sh.w.c.key;
  int *idx = sh.w.c.idx;
  st_sort(key, idx, n, false);
  const int m = min(m_keep0, n);
  const double xmax = (double)vmax / T;
  auto wk = [&](uint32_t k) -> double { return exp((double)key_to_float(k) / T - xmax); };
  double total = total0;
  if (!(total > 0.0)) {
    double s = 0.0;
    for (int i = tid; i < m; i += kStThreads) s += wk(key[i]);
    total = block_sum<kStThreads>(s, sh.redd);
  }
  int nkeep = m;
  if (P < 1.0) {
    const int per = (m + kStThreads - 1) / kStThreads;
    const int p0 = tid * per, p1 = min(m, p0 + per);
    double s = 0.0;
    for (int i = p0; i < p1; ++i) s += wk(key[i]);
    double ex, inc, tot;
    block_scan<kStThreads, double>(s, ex, inc, tot, sh.redd);
    const double target = P * total;
    int cand = 0x7FFFFFFF;
    if (p0 < p1 && inc >= target) {
      double acc = ex;
      for (int i = p0; i < p1; ++i) {
        acc += wk(key[i]);
        if (acc >= target) {
          cand = i;
          break;
        }
      }
      if (cand == 0x7FFFFFFF) cand = p1 - 1;
    }
    const int first = block_min_i<kStThreads>(cand, sh.redi);
    if (first != 0x7FFFFFFF) nkeep = first + 1;
  }
  // the kept entries, by index
  st_sort(key, idx, nkeep, true);
  double s = 0.0;
  for (int i = tid; i < nkeep; i += kStThreads) s += wk(key[i]);
  const double tot_keep = block_sum<kStThreads>(s, sh.redd);
  st_draw_sorted(sh, a, row, idx, nkeep, tot_keep, U, [&](int i) { return wk(key[i]); });
}

// fp32 weight 2^((v - M) * log2(e) / T) from two FMAs and one ex2.approx:
// c = c_hi + c_lo and M*c = mc_hi + mc_lo carry the constants to ~2^-48, so
// the only roundings are the final sum (|z| * 2^-24) and ex2 (~2^-22).
struct StW {
  float c_hi, c_lo, mc_hi, mc_lo;
  __device__ __forceinline__ void init(float M, double T) {
    const double c = 1.4426950408889634 / T;  // log2(e) / T
    c_hi = (float)c;
    c_lo = (float)(c - (double)c_hi);
    const double mc = (double)M * (double)c_hi;
    mc_hi = (float)mc;
    mc_lo = (float)(mc - (double)mc_hi) + (float)((double)M * (double)c_lo);
  }
  __device__ __forceinline__ float operator()(float v) const {
    const float z = fmaf(v, c_hi, -mc_hi) + fmaf(v, c_lo, -mc_lo);
    float r;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(z));
    return r;
  }
};

struct FCutS {
  float v;
  int idx;
};

// Four consecutive elements of the row from global memory (L2), masked
// tokens and positions past the row as -inf.
template <int DT>
__device__ __forceinline__ void st_load4_global(const StRow &r, int g0, float x[4]) {
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const int gi = g0 + e;
    if (gi >= r.V) {
      x[e] = -INFINITY;
      continue;
    }
    x[e] = DT == MS_DTYPE_F32
               ? __ldg(reinterpret_cast<const float *>(r.g) + gi)
               : __uint_as_float((uint32_t)__ldg(reinterpret_cast<const unsigned short *>(r.g) + gi) << 16);
    if (r.mask && !((__ldg(r.mask + (gi >> 5)) >> (gi & 31)) & 1u)) x[e] = -INFINITY;
  }
}

enum StMode : int { kStArgmax = 0, kStTopKMode = 1, kStFull = 2, kStNucleus = 3 };

template <int DT>
__global__ void __launch_bounds__(kStThreads, 2) ms_stream_kernel(SampleArgs a) {
  extern __shared__ __align__(128) unsigned char st_raw[];
  StShared &sh = *reinterpret_cast<StShared *>(st_raw);
  const int row = blockIdx.x;
  const int tid = threadIdx.x;
  const double T = a.temperature[row];
  const int k = a.top_k[row];
  const double P = a.top_p[row];
  const double U = a.uniforms[row];
  const int V = a.V;
  if (!(T >= 0.0) || isinf(T)) {  // negative, NaN or infinite temperature
    if (tid == 0) write_row(a, row, -1, 0.0f, MS_ROW_BAD_TEMPERATURE);
    return;
  }
  int mode;
  if (T == 0.0 || k == 1) {
    mode = kStArgmax;
  } else if (k >= 2 && k < V) {
    if (k > kStTopK) {  // may still cut: the generic kernel finishes it
      if (tid == 0) a.status[row] = kRowPending;
      return;
    }
    mode = kStTopKMode;
  } else {
    mode = P < 1.0 ? kStNucleus : kStFull;
  }
  StRow r;
  r.esz = DT == MS_DTYPE_F32 ? 4 : 2;
  r.g = reinterpret_cast<const char *>(a.logits) + (int64_t)row * a.ld * r.esz;
  r.mask = a.mask ? a.mask + (int64_t)row * a.mask_ld : nullptr;
  r.V = V;
  r.tma = (reinterpret_cast<uintptr_t>(r.g) & 15u) == 0;
  r.nchunks = (V + kChunk - 1) / kChunk;
  if (tid < kStages) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(st_smem(&sh.full[tid])) : "memory");
  }
  if (tid == 0) {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    sh.ncand = 0;
  }
  __syncthreads();
  uint32_t ph = 0;
  const uint64_t pol_stream = policy_evict_first();
  const uint64_t pol_keep = policy_evict_last();
  bool ok = true;

  // ================================================================ argmax
  if (mode == kStArgmax) {
    float mv[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
    int mi[4] = {0x7FFFFFFF, 0x7FFFFFFF, 0x7FFFFFFF, 0x7FFFFFFF};
    float vsum = 0.0f;
    ok = st_pass<DT>(sh, r, pol_stream, ph, [&](const float *x, int g0, int) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        vsum += x[e];
        if (x[e] > mv[e]) {
          mv[e] = x[e];
          mi[e] = g0 + e;
        }
      }
    });
    float tm = mv[0];
    int ti = mi[0];
#pragma unroll
    for (int e = 1; e < 4; ++e)
      if (mv[e] > tm || (mv[e] == tm && mi[e] < ti)) {
        tm = mv[e];
        ti = mi[e];
      }
    const bool bad = isnan(vsum) || vsum == INFINITY;
    uint32_t bk = tm > -INFINITY ? fkey(tm) : 0u;
    int bi = tm > -INFINITY ? ti : 0x7FFFFFFF;
    warp_argmax(bk, bi);
    if ((tid & 31) == 0) {
      sh.redu[tid >> 5] = bk;
      sh.redi[tid >> 5] = bi;
    }
    const int any_bad = __syncthreads_or(bad || !ok);
    if (tid < 32) {
      uint32_t k2 = tid < kStWarps ? sh.redu[tid] : 0u;
      int i2 = tid < kStWarps ? sh.redi[tid] : 0x7FFFFFFF;
      warp_argmax(k2, i2);
      if (tid == 0) {
        if (any_bad) {
          a.status[row] = kRowPending;
        } else if (T == 0.0) {  // greedy; all -inf ties at index 0 (sampler.py:33-34)
          write_row(a, row, k2 == 0u ? 0 : i2, 1.0f, 0);
        } else if (k2 == 0u) {  // every logit -inf: zero total (sampler.py:46-47)
          write_row(a, row, -1, 0.0f, MS_ROW_ALL_MASKED);
        } else if (U > 0.0) {
          write_row(a, row, i2, 1.0f, 0);
        } else {  // r == 0 stops at index 0
          write_row(a, row, 0, i2 == 0 ? 1.0f : 0.0f, 0);
        }
      }
    }
    return;
  }

  // ================================================================= top-k
  if (mode == kStTopKMode) {
    __shared__ float s_tau;  // candidates are values >= s_tau (> when s_strict)
    __shared__ int s_strict, s_cc;
    if (tid == 0) {
      s_tau = -INFINITY;
      s_strict = 0;
      s_cc = 0;
    }
    float vmax_t = -INFINITY, vsum = 0.0f;
    const int lane = tid & 31;
    bool over = false;
    if (tid == 0) {
      for (int c = 0; c < kStages && c < r.nchunks; ++c) st_issue(sh, r, c, c, pol_stream);
    }
    __syncthreads();
    int c = 0;
    for (; c < r.nchunks && !over; ++c) {
      const int s = c % kStages;
      if (!st_wait(sh, s, (ph >> s) & 1u)) ok = false;
      ph ^= 1u << s;
      float x[8];
      st_get4<DT>(sh, r, c, s, tid * 4, x);
      st_get4<DT>(sh, r, c, s, kSub + tid * 4, x + 4);
      const int g0 = c * kChunk + tid * 4, g1 = g0 + kSub;
      float cm = -INFINITY;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        vsum += x[e];
        cm = fmaxf(cm, x[e]);
      }
      vmax_t = fmaxf(vmax_t, cm);
      // Insert this chunk's values >= tau.  When they would not fit: shrink
      // the buffer to its top-k, or raise tau to the k-th largest of this
      // chunk's thread maxima (k distinct threads hold k values >= it, so
      // the row's k-th largest is not below it).
      for (int attempt = 0; attempt < 4; ++attempt) {
        const float tau = s_tau;
        const bool strict = s_strict != 0;
        int cnt = 0;
#pragma unroll
        for (int e = 0; e < 8; ++e) cnt += (x[e] > -INFINITY && (strict ? x[e] > tau : x[e] >= tau)) ? 1 : 0;
        if (!__syncthreads_or(cnt > 0)) break;  // common case: nothing to insert
        int incl = cnt;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const int y = __shfl_up_sync(0xFFFFFFFFu, incl, o);
          if (lane >= o) incl += y;
        }
        int wbase = 0;
        if (lane == 31) wbase = atomicAdd(&s_cc, incl);
        wbase = __shfl_sync(0xFFFFFFFFu, wbase, 31);
        __syncthreads();
        const int total = s_cc;
        const int n0 = sh.ncand;
        // the first chunk always starts from the thread-maxima bound
        const bool fits = n0 + total <= kCandCap && !(c == 0 && attempt == 0 && total > k);
        if (fits) {
          int pos = n0 + wbase + incl - cnt;
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            if (x[e] > -INFINITY && (strict ? x[e] > tau : x[e] >= tau)) {
              sh.w.c.key[pos] = fkey(x[e]);
              sh.w.c.idx[pos] = e < 4 ? g0 + e : g1 + e - 4;
              ++pos;
            }
          }
        }
        __syncthreads();
        if (tid == 0) {
          if (fits) sh.ncand = n0 + total;
          s_cc = 0;
        }
        __syncthreads();
        if (fits) break;
        if (attempt == 3) {
          over = true;  // heavy ties: the generic kernel finishes the row
          break;
        }
        if (n0 > k && attempt == 0) {
          // keep the buffer's entries >= its k-th largest key (ties kept)
          int above;
          const uint32_t kk = st_select_kth(sh, sh.w.c.key, n0, k, &above);
          uint32_t kv[kCandCap / kStThreads];
          int iv[kCandCap / kStThreads];
          int nk = 0;
          for (int i = tid; i < n0; i += kStThreads) {
            if (sh.w.c.key[i] >= kk) {
              kv[nk] = sh.w.c.key[i];
              iv[nk] = sh.w.c.idx[i];
              ++nk;
            }
          }
          int kex, kin, ktot;
          block_scan<kStThreads, int>(nk, kex, kin, ktot, sh.redi);
          for (int q = 0; q < nk; ++q) {
            sh.w.c.key[kex + q] = kv[q];
            sh.w.c.idx[kex + q] = iv[q];
          }
          __syncthreads();
          if (tid == 0) {
            sh.ncand = ktot;
            s_tau = key_to_float(kk);
            s_strict = 1;  // >= k entries >= kk held: a later equal value ranks below them
          }
          __syncthreads();
          continue;
        }
        sh.tmaxk[tid] = cm > -INFINITY ? fkey(cm) : 0u;
        __syncthreads();
        int above2;
        const uint32_t bk = st_select_kth(sh, sh.tmaxk, kStThreads, k, &above2);
        if (tid == 0 && bk != 0u && key_to_float(bk) > s_tau) {
          s_tau = key_to_float(bk);
          s_strict = 0;
        }
        __syncthreads();
      }
      __syncthreads();  // stage s is free
      if (tid == 0 && !over && c + kStages < r.nchunks) {
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        st_issue(sh, r, c + kStages, s, pol_stream);
      }
    }
    // copies issued past the last consumed chunk (early stop) must land
    // before this CTA's shared memory is released
    for (int c2 = c; c2 < r.nchunks && c2 < c - 1 + kStages; ++c2) {
      const int s = c2 % kStages;
      if (!st_wait(sh, s, (ph >> s) & 1u)) ok = false;
      ph ^= 1u << s;
    }
    const bool bad = isnan(vsum) || vsum == INFINITY;
    if (__syncthreads_or(bad || !ok || over)) {
      if (tid == 0) a.status[row] = kRowPending;
      return;
    }
    const float vmax = block_max_f<kStThreads>(vmax_t, sh.redf);
    if (!(vmax > -INFINITY)) {  // every logit -inf (sampler.py:46-47)
      if (tid == 0) write_row(a, row, -1, 0.0f, MS_ROW_ALL_MASKED);
      return;
    }
    // fewer valid tokens than top_k: the buffer holds all of them (top-k off)
    const int n = sh.ncand;
    int m = n;
    if (n > k) {
      st_sort(sh.w.c.key, sh.w.c.idx, n, false);  // (key desc, index asc)
      m = k;
    }
    st_finish_set(sh, a, row, m, m, 0.0, T, P, U, vmax);
    return;
  }

  // ===================================================== top-p / full softmax
  float vmax_t = -INFINITY, vsum = 0.0f;
  ok = st_pass<DT>(sh, r, pol_keep, ph, [&](const float *x, int, int) {
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      vsum += x[e];
      vmax_t = fmaxf(vmax_t, x[e]);
    }
  });
  const bool bad = isnan(vsum) || vsum == INFINITY;
  if (__syncthreads_or(bad || !ok)) {
    if (tid == 0) a.status[row] = kRowPending;
    return;
  }
  const float vmax = block_max_f<kStThreads>(vmax_t, sh.redf);
  if (!(vmax > -INFINITY)) {  // every logit -inf (sampler.py:46-47)
    if (tid == 0) write_row(a, row, -1, 0.0f, MS_ROW_ALL_MASKED);
    return;
  }
  StW W;
  W.init(vmax, T);
  const float xscale = (float)((double)kSBins / ((double)kSXRange * T));
  const bool nucleus = mode == kStNucleus;
  const int nsubs = 2 * r.nchunks;
  for (int q = tid; q < nsubs; q += kStThreads) sh.subsum[q] = 0.0;
  if (nucleus)
    for (int b = tid; b < kSBins; b += kStThreads) {
      sh.w.h.cnt[b] = 0u;
      sh.w.h.mass[b] = 0.0f;
    }
  __syncthreads();
  auto bin_of = [&](float v) -> int {
    const float t = (vmax - v) * xscale;
    return t < (float)kSBins ? (int)t : kSBins;
  };
  // pass 2 (L2): weights, per-sub-chunk totals, histogram
  ok = st_pass<DT>(sh, r, pol_keep, ph, [&](const float *x, int, int sub) {
    float ws = 0.0f;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      if (x[e] > -INFINITY) {
        const float w = W(x[e]);
        ws += w;
        if (nucleus) {
          const int b = bin_of(x[e]);
          if (b < kSBins) {
            atomicAdd(&sh.w.h.cnt[b], 1u);
            atomicAdd(&sh.w.h.mass[b], w);
          }
        }
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ws += __shfl_xor_sync(0xFFFFFFFFu, ws, o);
    if ((tid & 31) == 0 && ws != 0.0f) atomicAdd(&sh.subsum[sub], (double)ws);
  });
  if (!__syncthreads_and(ok)) {
    if (tid == 0) a.status[row] = kRowPending;
    return;
  }
  double total;
  {
    double s = 0.0;
    for (int q = tid; q < nsubs; q += kStThreads) s += sh.subsum[q];
    total = block_sum<kStThreads>(s, sh.redd);
  }
  FCutS cut{-INFINITY, -1};  // the kept set: everything valid
  if (nucleus) {
    // crossing bin: first bin (from the top) whose running weight reaches
    // P * total; thread t owns bins 4t..4t+3
    const double thr = P * total;
    double s = 0.0;
    uint32_t cn = 0;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      s += (double)sh.w.h.mass[tid * 4 + q];
      cn += sh.w.h.cnt[tid * 4 + q];
    }
    double ex, inc, tt;
    block_scan<kStThreads, double>(s, ex, inc, tt, sh.redd);
    int cex, cin, ctt;
    block_scan<kStThreads, int>((int)cn, cex, cin, ctt, sh.redi);
    int cand = 0x7FFFFFFF;
    if (inc >= thr) {
      double acc = ex;
      for (int q = 0; q < 4; ++q) {
        const int b = tid * 4 + q;
        const double bm = (double)sh.w.h.mass[b];
        if (sh.w.h.cnt[b] > 0u && acc + bm >= thr) {
          cand = b;
          break;
        }
        acc += bm;
      }
    }
    const int bstar = block_min_i<kStThreads>(cand, sh.redi);
    if (bstar != 0x7FFFFFFF) {
      if (tid == bstar / 4) {
        double acc = ex;
        int ca = cex;
        for (int q = 0; q < 4; ++q) {
          const int b = tid * 4 + q;
          if (b == bstar) {
            sh.bcast_d[0] = acc;
            sh.bcast_i[1] = ca;
            sh.bcast_i[2] = (int)sh.w.h.cnt[b];
            break;
          }
          acc += (double)sh.w.h.mass[b];
          ca += (int)sh.w.h.cnt[b];
        }
      }
      __syncthreads();
      const double above_w = sh.bcast_d[0];
      const int above_c = sh.bcast_i[1];
      const int in_c = sh.bcast_i[2];
      __syncthreads();
      const bool all_up_to = above_c + in_c <= kCandCap;
      if (!all_up_to && in_c > kCandCap) {  // a crowded bin: generic kernel
        if (tid == 0) a.status[row] = kRowPending;
        return;
      }
      // pass 3 (L2): gather bins <= bstar, or bin bstar alone
      if (tid == 0) sh.ncand = 0;
      __syncthreads();
      ok = st_pass<DT>(sh, r, pol_keep, ph, [&](const float *x, int g0, int) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          if (x[e] > -INFINITY) {
            const int b = bin_of(x[e]);
            if (all_up_to ? b <= bstar : b == bstar) {
              const int pos = atomicAdd(&sh.ncand, 1);
              sh.w.c.key[pos] = fkey(x[e]);
              sh.w.c.idx[pos] = g0 + e;
            }
          }
        }
      });
      if (!__syncthreads_and(ok)) {
        if (tid == 0) a.status[row] = kRowPending;
        return;
      }
      const int n = sh.ncand;
      if (all_up_to) {
        // the nucleus lies among these: exact finish (total: all valid)
        st_finish_set(sh, a, row, n, n, total, T, P, U, vmax);
        return;
      }
      // the cut inside bin bstar, with the histogram's own weights
      st_sort(sh.w.c.key, sh.w.c.idx, n, false);
      {
        const int per = (n + kStThreads - 1) / kStThreads;
        const int p0 = tid * per, p1 = min(n, p0 + per);
        double s2 = 0.0;
        for (int i = p0; i < p1; ++i) s2 += (double)W(key_to_float(sh.w.c.key[i]));
        double e2, i2, t2;
        block_scan<kStThreads, double>(s2, e2, i2, t2, sh.redd);
        int cc = 0x7FFFFFFF;
        if (p0 < p1 && above_w + i2 >= thr) {
          double acc = above_w + e2;
          for (int i = p0; i < p1; ++i) {
            acc += (double)W(key_to_float(sh.w.c.key[i]));
            if (acc >= thr) {
              cc = i;
              break;
            }
          }
          if (cc == 0x7FFFFFFF) cc = p1 - 1;
        }
        int rc = block_min_i<kStThreads>(cc, sh.redi);
        if (rc == 0x7FFFFFFF) rc = n - 1;
        cut.v = key_to_float(sh.w.c.key[rc]);
        cut.idx = sh.w.c.idx[rc];
      }
      // pass 4 (L2): per-sub-chunk weight of the kept set
      __syncthreads();
      for (int q = tid; q < nsubs; q += kStThreads) sh.subsum[q] = 0.0;
      __syncthreads();
      ok = st_pass<DT>(sh, r, pol_keep, ph, [&](const float *x, int g0, int sub) {
        float ws = 0.0f;
#pragma unroll
        for (int e = 0; e < 4; ++e)
          if (x[e] > -INFINITY && (x[e] > cut.v || (x[e] == cut.v && g0 + e <= cut.idx))) ws += W(x[e]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ws += __shfl_xor_sync(0xFFFFFFFFu, ws, o);
        if ((tid & 31) == 0 && ws != 0.0f) atomicAdd(&sh.subsum[sub], (double)ws);
      });
      if (!__syncthreads_and(ok)) {
        if (tid == 0) a.status[row] = kRowPending;
        return;
      }
      double s3 = 0.0;
      for (int q = tid; q < nsubs; q += kStThreads) s3 += sh.subsum[q];
      total = block_sum<kStThreads>(s3, sh.redd);
    }
    // bstar not found: the running sum never reached top_p; all kept
  }
  // ------------------------------- index-order draw over the kept set (FULL)
  auto keptw = [&](float v, int gi) -> float {
    return (v > -INFINITY && (v > cut.v || (v == cut.v && gi <= cut.idx))) ? W(v) : 0.0f;
  };
  if (!(U > 0.0)) {  // r == 0 stops at index 0 (sampler.py:66)
    if (tid == 0) {
      float x4[4];
      st_load4_global<DT>(r, 0, x4);
      write_row(a, row, 0, (float)((double)keptw(x4[0], 0) / total), 0);
    }
    return;
  }
  const double target = U * total;
  // crossing sub-chunk: thread t owns subs 2t, 2t+1 (nsubs <= 1024)
  int qstar;
  double before;
  {
    double s = 0.0;
    for (int q = 2 * tid; q < 2 * tid + 2 && q < nsubs; ++q) s += sh.subsum[q];
    double ex, inc, tt;
    block_scan<kStThreads, double>(s, ex, inc, tt, sh.redd);
    int cand = 0x7FFFFFFF;
    if (s > 0.0 && inc >= target) {
      double acc = ex;
      for (int q = 2 * tid; q < 2 * tid + 2 && q < nsubs; ++q) {
        if (sh.subsum[q] > 0.0 && acc + sh.subsum[q] >= target) {
          cand = q;
          break;
        }
        acc += sh.subsum[q];
      }
      if (cand == 0x7FFFFFFF) cand = min(nsubs - 1, 2 * tid + 1);
    }
    qstar = block_min_i<kStThreads>(cand, sh.redi);
    if (qstar != 0x7FFFFFFF && tid == qstar / 2) {
      double acc = ex;
      for (int q = 2 * tid; q < qstar; ++q) acc += sh.subsum[q];
      sh.bcast_d[1] = acc;
    }
    __syncthreads();
    before = sh.bcast_d[1];
  }
  if (qstar == 0x7FFFFFFF) {  // ran past the end (sampler.py:68)
    if (tid == 0) {
      float x4[4];
      st_load4_global<DT>(r, V - 1, x4);
      write_row(a, row, V - 1, (float)((double)keptw(x4[0], V - 1) / total), 0);
    }
    return;
  }
  // the crossing sub-chunk, read back from L2
  const int gq = (qstar >> 1) * kChunk + (qstar & 1) * kSub + tid * 4;
  float x[4];
  st_load4_global<DT>(r, gq, x);
  float wv[4];
  double s = 0.0;
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    wv[e] = keptw(x[e], gq + e);
    s += (double)wv[e];
  }
  double ex, inc, tt;
  block_scan<kStThreads, double>(s, ex, inc, tt, sh.redd);
  int who = block_min_i<kStThreads>((s > 0.0 && before + inc >= target) ? tid : 0x7FFFFFFF, sh.redi);
  if (who == 0x7FFFFFFF) who = -block_min_i<kStThreads>(s > 0.0 ? -tid : 1, sh.redi);
  if (tid == who) {
    double acc = before + ex;
    int tok = -1, last = -1;
    double wt = 0.0, wl = 0.0;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      if (wv[e] <= 0.0f || tok >= 0) continue;
      acc += (double)wv[e];
      last = gq + e;
      wl = wv[e];
      if (acc >= target) {
        tok = gq + e;
        wt = wv[e];
      }
    }
    if (tok < 0) {
      tok = last;
      wt = wl;
    }
    write_row(a, row, tok, (float)(wt / total), 0);
  }
}
}  // namespace ms
