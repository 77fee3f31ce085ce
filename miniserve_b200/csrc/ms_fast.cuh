// Cluster-resident sampling kernel: one thread-block cluster of C CTAs per
// logits row.  Each CTA pulls its contiguous vocab slice from HBM exactly
// once (one cp.async.bulk TMA copy into shared memory) and every later pass
// -- max/argmax, temperature-scaled float64 exponentials, the top-k count
// select, the top-p mass select and the index-order draw -- reads that
// on-chip copy.  Cross-CTA steps (max, sums, histograms, candidate gathers)
// go through distributed shared memory between cluster barriers.
//
// Rows the on-chip path cannot finish exactly (a candidate set above kCap,
// a top-k/top-p cut beyond the 40-units-of-x grid) are marked
// kRowPending in row_status and finished by ms_generic_kernel.
//
// Control flow: every decision taken after a cluster barrier is computed by
// all CTAs from the same published values, so all CTAs of a cluster execute
// the same sequence of barriers.
#pragma once

#include <cooperative_groups.h>

#include "ms_common.cuh"
#include "ms_generic.cuh"

namespace ms {

namespace cg = cooperative_groups;

constexpr int kFastThreads = 512;
constexpr int kFastWarps = kFastThreads / 32;
constexpr int kMaxCluster = 16;
constexpr int kCap = 1024;                 // on-chip candidate capacity of the leader CTA
constexpr int kXBins = 2048;               // x-grid bins over [0, 40) units of (max - x)
constexpr float kXRange = 40.0f;           // exp(-40) ~ 4e-18: past it a token's weight is noise
constexpr double kQScale = 17592186044416.0;  // 2^44 fixed-point weight scale

enum FastMode : int { kModeDone = 0, kModeFull = 1, kModeTopK = 2, kModeNucleus = 3 };

struct FastCtl {
  uint32_t max_key;
  int max_idx;
  uint32_t nvalid;
  uint32_t flags;
  double sum;                 // float64 sum of this CTA's kept weights
  uint32_t rcnt;              // totals of this CTA's reduced bin range
  unsigned long long rq;
  int ncand;
  uint32_t cut_key;           // written by the leader into every CTA
  int cut_idx;
  int go;
};

struct FastScratch {
  double redd[33];
  uint32_t redu[33];
  int redi[33];
  int bi[16];
  double bd[8];
  int tma_timeout;
};

// Dynamic shared memory layout (byte offsets); all sections 16-byte aligned.
struct FastLayout {
  int keys;      // S stored keys
  int work;      // histogram / candidate union
  int red;       // reduced bin range of this CTA
  int ctl;
  int lctl;   // local copies of every CTA's control block
  int scratch;
  int mbar;
  int total;
};

constexpr int kWorkBytes = kXBins * 4 + kXBins * 8;  // 24 KB: u32 counts + u64 fixed-point weights
static_assert(kCap * 20 <= kWorkBytes, "candidate arrays must fit the histogram region");

__host__ __device__ inline int align16(int x) { return (x + 15) & ~15; }

__host__ __device__ inline FastLayout fast_layout(int S, int key_bytes, int C) {
  FastLayout L;
  L.keys = 0;
  L.work = align16(S * key_bytes);
  L.red = L.work + kWorkBytes;
  L.ctl = L.red + align16((kXBins / C) * 12);
  L.lctl = L.ctl + align16((int)sizeof(FastCtl));
  L.scratch = L.lctl + align16(kMaxCluster * (int)sizeof(FastCtl));
  L.mbar = L.scratch + align16((int)sizeof(FastScratch));
  L.total = L.mbar + 16;
  return L;
}

template <int DT>
struct KeyStore;
template <>
struct KeyStore<MS_DTYPE_F32> {
  using T = uint32_t;
  static __device__ __forceinline__ uint32_t full(T k) { return k; }
  static __device__ __forceinline__ T pack(uint32_t key) { return key; }
};
template <>
struct KeyStore<MS_DTYPE_BF16> {
  using T = uint16_t;
  static __device__ __forceinline__ uint32_t full(T k) {
    uint32_t k32 = (uint32_t)k << 16;
    return (k & 0x8000u) ? k32 : (k32 | 0xFFFFu);
  }
  static __device__ __forceinline__ T pack(uint32_t key) { return (T)(key >> 16); }
};

// Canonical order key of a finite-or-(-inf) value: -0 and +0 share a key,
// as the reference compares values, not bit patterns.
__device__ __forceinline__ uint32_t fkey(float v) {
  uint32_t u = __float_as_uint(v);
  if (u == 0x80000000u) u = 0u;
  return bits_to_key(u);
}

// Kept-set predicate on values: above the cut value, or equal to it with an
// index at or below the cut index (ties taken in index order).
struct FCut {
  float v;
  int idx;
};
__device__ __forceinline__ bool fkept(const FCut &c, float v, int idx) {
  return v > c.v || (v == c.v && idx <= c.idx);
}

// Raw slice values in shared memory: fp32 as is, bf16 widened exactly.
template <int DT>
__device__ __forceinline__ float fv(const void *vals, int i) {
  if (DT == MS_DTYPE_F32) return reinterpret_cast<const float *>(vals)[i];
  return __uint_as_float((uint32_t)reinterpret_cast<const uint16_t *>(vals)[i] << 16);
}
// Four consecutive values starting at a multiple of 4 (one 16- or 8-byte load).
template <int DT>
__device__ __forceinline__ void load4(const void *vals, int i, float x[4]) {
  if (DT == MS_DTYPE_F32) {
    const float4 f = reinterpret_cast<const float4 *>(vals)[i >> 2];
    x[0] = f.x;
    x[1] = f.y;
    x[2] = f.z;
    x[3] = f.w;
  } else {
    const uint2 h = reinterpret_cast<const uint2 *>(vals)[i >> 2];
    x[0] = __uint_as_float(h.x << 16);
    x[1] = __uint_as_float(h.x & 0xFFFF0000u);
    x[2] = __uint_as_float(h.y << 16);
    x[3] = __uint_as_float(h.y & 0xFFFF0000u);
  }
}

constexpr uint32_t kHasNegInf = 1u << 29;  // flag: a -inf logit in an unmasked row

// After a cluster barrier: C threads copy the C control blocks into local
// shared memory, so the rest of the CTA reads them locally.
template <int C>
__device__ __forceinline__ void pull_ctl(cg::cluster_group &cluster, FastCtl &ctl, FastCtl *lctl) {
  if (threadIdx.x < C) {
    const FastCtl *r = cluster.map_shared_rank(&ctl, (int)threadIdx.x);
    FastCtl &d = lctl[threadIdx.x];
    d.max_key = r->max_key;
    d.max_idx = r->max_idx;
    d.nvalid = r->nvalid;
    d.flags = r->flags;
    d.sum = r->sum;
    d.rcnt = r->rcnt;
    d.rq = r->rq;
    d.ncand = r->ncand;
  }
  __syncthreads();
}

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

// Bin of a kept element on the x grid: 0 holds the row maximum; kXBins
// means "past the grid".  Monotone non-increasing in the logit, so every
// bin is a contiguous range of the descending key order.
__device__ __forceinline__ int xbin(float v, float vmax, float scale) {
  float t = (vmax - v) * scale;
  return t < (float)kXBins ? (int)t : kXBins;
}

__device__ __forceinline__ unsigned long long qweight(double w) {
  return (unsigned long long)(w * kQScale);
}

template <int C, int DT>
__global__ void __launch_bounds__(kFastThreads, 2)
    ms_fast_kernel(SampleArgs a, int S, int R) {
  using KS = KeyStore<DT>;
  using KT = typename KS::T;
  extern __shared__ __align__(128) unsigned char smem[];
  cg::cluster_group cluster = cg::this_cluster();
  const int rank = (int)cluster.block_rank();
  const int row = blockIdx.x / C;
  const int tid = threadIdx.x;
  const FastLayout L = fast_layout(S, (int)sizeof(KT), C);
  KT *keys = reinterpret_cast<KT *>(smem + L.keys);
  uint32_t *hcnt = reinterpret_cast<uint32_t *>(smem + L.work);
  unsigned long long *hq = reinterpret_cast<unsigned long long *>(smem + L.work + kXBins * 4);
  uint32_t *ckey = reinterpret_cast<uint32_t *>(smem + L.work);
  int *cidx = reinterpret_cast<int *>(smem + L.work + kCap * 4);
  int *crank = reinterpret_cast<int *>(smem + L.work + kCap * 8);
  uint32_t *skey = reinterpret_cast<uint32_t *>(smem + L.work + kCap * 12);
  int *sidx = reinterpret_cast<int *>(smem + L.work + kCap * 16);
  constexpr int NBR = kXBins / C;  // bins this CTA reduces across the cluster
  uint32_t *rcnt = reinterpret_cast<uint32_t *>(smem + L.red);
  unsigned long long *rq = reinterpret_cast<unsigned long long *>(smem + L.red + NBR * 4);
  FastCtl &ctl = *reinterpret_cast<FastCtl *>(smem + L.ctl);
  FastCtl *lctl = reinterpret_cast<FastCtl *>(smem + L.lctl);
  FastScratch &sc = *reinterpret_cast<FastScratch *>(smem + L.scratch);
  uint64_t *mbar = reinterpret_cast<uint64_t *>(smem + L.mbar);

  const int V = a.V;
  const int lo = rank * S;
  const int n = max(0, min(V, lo + S) - lo);  // elements in this CTA's slice
  const char *grow = reinterpret_cast<const char *>(a.logits) +
                     ((int64_t)row * a.ld + lo) * (DT == MS_DTYPE_F32 ? 4 : 2);
  const uint32_t *mrow = a.mask ? a.mask + (int64_t)row * a.mask_ld : nullptr;
  const int esz = DT == MS_DTYPE_F32 ? 4 : 2;

  // ------------------------------------------------------------ load slice
  const bool tma_ok = ((reinterpret_cast<uintptr_t>(grow) & 15u) == 0);
  const int tma_elems = tma_ok ? ((n * esz) & ~15) / esz : 0;
  if (tid == 0) {
    sc.tma_timeout = 0;
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(mbar)) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  __syncthreads();
  if (tid == 0) {
    uint32_t bytes = (uint32_t)(tma_elems * esz);
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(mbar)),
                 "r"(bytes)
                 : "memory");
    if (bytes)
      asm volatile(
          "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
              smem_u32(keys)),
          "l"(grow), "r"(bytes), "r"(smem_u32(mbar))
          : "memory");
  }
  for (int i = tma_elems + tid; i < n; i += kFastThreads) {
    if (DT == MS_DTYPE_F32)
      reinterpret_cast<uint32_t *>(keys)[i] = __ldg(reinterpret_cast<const unsigned int *>(grow) + i);
    else
      reinterpret_cast<uint16_t *>(keys)[i] = __ldg(reinterpret_cast<const unsigned short *>(grow) + i);
  }
  // zero the histogram while the copy is in flight
  for (int b = tid; b < kXBins; b += kFastThreads) {
    hcnt[b] = 0u;
    hq[b] = 0ull;
  }
  {
    // bounded wait for the bulk copy (phase 0)
    uint32_t done = 0;
    for (long it = 0; it < (1l << 26) && !done; ++it) {
      asm volatile(
          "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], 0; selp.u32 %0, 1, 0, p; }"
          : "=r"(done)
          : "r"(smem_u32(mbar))
          : "memory");
    }
    if (!done) sc.tma_timeout = 1;  // the row is handed to the generic kernel below
  }
  __syncthreads();

  // ---------------------------------------------- mask pass (masked rows)
  // The slice keeps raw values; a disallowed token becomes -inf in place
  // (the logits-processor hook's convention, miniserve/model_runner.py:214).
  const int t0 = tid * R;
  const int t1 = min(n, t0 + R);
  uint32_t nvalid = 0;
  if (mrow) {
    for (int i = t0; i < t1; ++i) {
      const int gi = lo + i;
      if (!((__ldg(mrow + (gi >> 5)) >> (gi & 31)) & 1u)) {
        if (DT == MS_DTYPE_F32)
          reinterpret_cast<uint32_t *>(keys)[i] = kNegInfBits;
        else
          reinterpret_cast<uint16_t *>(keys)[i] = (uint16_t)(kNegInfBits >> 16);
      }
    }
    // counted after the writes so that every element is read once more here
    for (int i = t0; i < t1; ++i) nvalid += fv<DT>(keys, i) > -INFINITY ? 1u : 0u;
  }
  // ----------------------------------------- local max (first index if needed)
  // Rows that need the argmax (greedy, top_k == 1) track the first index of
  // the maximum; the others only need its value.  The float sum detects NaN
  // and +inf, whose rows go to the generic kernel.
  const double T0 = a.temperature[row];
  const int k0 = a.top_k[row];
  const bool need_idx = T0 == 0.0 || k0 == 1;
  float m4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
  int i4[4] = {0x7FFFFFFF, 0x7FFFFFFF, 0x7FFFFFFF, 0x7FFFFFFF};
  float vsum = 0.0f;
  {
    const int tv = t0 + ((t1 - t0) & ~3);  // end of whole groups of 4
    if (need_idx) {
      for (int i = t0; i < tv; i += 4) {
        float x[4];
        load4<DT>(keys, i, x);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          vsum += x[e];
          if (x[e] > m4[e]) {
            m4[e] = x[e];
            i4[e] = lo + i + e;
          }
        }
      }
    } else {
      for (int i = t0; i < tv; i += 4) {
        float x[4];
        load4<DT>(keys, i, x);
#pragma unroll
        for (int e = 0; e < 4; ++e) m4[e] = fmaxf(m4[e], x[e]);
        vsum += (x[0] + x[1]) + (x[2] + x[3]);
      }
    }
    for (int i = tv; i < t1; ++i) {
      const float x = fv<DT>(keys, i);
      vsum += x;
      if (x > m4[0]) {
        m4[0] = x;
        i4[0] = lo + i;
      }
    }
  }
  float tmax = m4[0];
  int tidx = i4[0];
#pragma unroll
  for (int e = 1; e < 4; ++e) {
    if (m4[e] > tmax || (m4[e] == tmax && i4[e] < tidx)) {
      tmax = m4[e];
      tidx = i4[e];
    }
  }
  uint32_t flags = 0;
  if (isnan(vsum) || vsum == INFINITY) flags |= MS_ROW_NONFINITE;
  if (vsum == -INFINITY && !mrow) flags |= kHasNegInf;
  uint32_t bk = tmax > -INFINITY ? fkey(tmax) : kNegInfKey;
  int bi = tmax > -INFINITY ? tidx : 0x7FFFFFFF;
  if (!need_idx) bi = 0;
  warp_argmax(bk, bi);
  flags = __reduce_or_sync(0xFFFFFFFFu, flags);
  nvalid = warp_sum_u32(nvalid);
  if ((tid & 31) == 0) {
    sc.redu[tid >> 5] = bk;
    sc.redi[tid >> 5] = bi;
    sc.bi[tid >> 5] = (int)nvalid;
    reinterpret_cast<uint32_t *>(sc.redd)[tid >> 5] = flags;
  }
  __syncthreads();
  if (tid < 32) {
    uint32_t k2 = tid < kFastWarps ? sc.redu[tid] : 0u;
    int i2 = tid < kFastWarps ? sc.redi[tid] : 0x7FFFFFFF;
    uint32_t f2 = tid < kFastWarps ? reinterpret_cast<uint32_t *>(sc.redd)[tid] : 0u;
    uint32_t nv = tid < kFastWarps ? (uint32_t)sc.bi[tid] : 0u;
    warp_argmax(k2, i2);
    f2 = __reduce_or_sync(0xFFFFFFFFu, f2);
    nv = warp_sum_u32(nv);
    if (tid == 0) {
      ctl.max_key = k2;
      ctl.max_idx = i2;
      ctl.nvalid = nv;
      ctl.flags = f2 | (sc.tma_timeout ? (uint32_t)kRowPending : 0u);
    }
  }
  cluster.sync();  // ---------------------------------------------------- S1
  pull_ctl<C>(cluster, ctl, lctl);
  uint32_t M_key = 0u, nval = 0u, rflags = 0u;
  int M_idx = 0x7FFFFFFF;
  for (int q = 0; q < C; ++q) {
    const FastCtl *rc = &lctl[q];
    uint32_t k2 = rc->max_key;
    int i2 = rc->max_idx;
    if (k2 > M_key || (k2 == M_key && i2 < M_idx)) {
      M_key = k2;
      M_idx = i2;
    }
    nval += rc->nvalid;
    rflags |= rc->flags;
  }
  const double T = a.temperature[row];
  const int kk = a.top_k[row];
  const double P = a.top_p[row];
  const double U = a.uniforms[row];
  const bool leader = rank == 0;

  // --------------------------------------------------------- row decisions
  int mode = kModeDone;
  if (!mrow) nval = (uint32_t)V;  // unmasked: every token counts unless -inf is present
  const uint32_t fl = 0u;
  const bool defer = (rflags & ((uint32_t)kRowPending | MS_ROW_NONFINITE)) != 0u ||
                     ((rflags & kHasNegInf) && T > 0.0 && kk > 1);
  if (defer) {
    if (leader && tid == 0) a.status[row] = kRowPending;
  } else if (T == 0.0) {  // all -inf: the first index is the (tied) maximum
    if (leader && tid == 0) write_row(a, row, M_key == kNegInfKey ? 0 : M_idx, 1.0f, (int32_t)fl);
  } else if (!(T > 0.0) || isinf(T)) {
    if (leader && tid == 0) write_row(a, row, -1, 0.0f, (int32_t)(fl | MS_ROW_BAD_TEMPERATURE));
  } else if (M_key == kNegInfKey) {  // every token is -inf: zero total (sampler.py:46-47)
    if (leader && tid == 0) write_row(a, row, -1, 0.0f, (int32_t)(fl | MS_ROW_ALL_MASKED));
  } else {
    const int keff = (kk > 0 && (uint32_t)kk < nval) ? kk : 0;
    if (keff == 1) {
      if (leader && tid == 0) {
        if (U > 0.0)
          write_row(a, row, M_idx, 1.0f, (int32_t)fl);
        else
          write_row(a, row, 0, M_idx == 0 ? 1.0f : 0.0f, (int32_t)fl);
      }
    } else if (keff > 1) {
      mode = keff <= kCap ? kModeTopK : kModeDone;
      if (mode == kModeDone && leader && tid == 0) a.status[row] = kRowPending;
    } else if (P < 1.0) {
      mode = kModeNucleus;
    } else {
      mode = kModeFull;
    }
  }
  if (mode == kModeDone) {
    cluster.sync();  // nobody may leave while others read its control block
    return;
  }
  const int keff = (kk > 0 && (uint32_t)kk < nval) ? kk : 0;
  const float vmax = key_to_float(M_key);
  const double dmax = (double)vmax;
  const double inv_t = 1.0 / T;
  const float xscale = (float)((double)kXBins / ((double)kXRange * T));

  // The draw over a kept set (FULL, or after a top-p cut): cut describes it.
  FCut cut{-INFINITY, -1};
  double my_sum = 0.0;  // this thread's run weight over the kept set

  if (mode == kModeTopK || mode == kModeNucleus) {
    // ------------------------------------------------ histogram on the x grid
    for (int i = t0; i < t1; ++i) {
      const float v = fv<DT>(keys, i);
      if (!(v > -INFINITY)) continue;
      int b = xbin(v, vmax, xscale);
      if (mode == kModeNucleus) {
        double w = exp(((double)v - dmax) * inv_t);
        my_sum += w;
        if (b < kXBins) {
          atomicAdd(&hcnt[b], 1u);
          atomicAdd(&hq[b], qweight(w));
        }
      } else if (b < kXBins) {
        atomicAdd(&hcnt[b], 1u);
      }
    }
    if (mode == kModeNucleus) {
      double s = block_sum<kFastThreads>(my_sum, sc.redd);
      if (tid == 0) ctl.sum = s;
    }
    cluster.sync();  // -------------------------------------------------- S2
    // reduce bins [rank*NBR, (rank+1)*NBR) over the cluster
    uint32_t rc_local = 0;
    unsigned long long rq_local = 0;
    for (int j = tid; j < NBR; j += kFastThreads) {
      const int b = rank * NBR + j;
      uint32_t c = 0;
      unsigned long long q = 0;
      for (int r2 = 0; r2 < C; ++r2) {
        c += cluster.map_shared_rank(hcnt, r2)[b];
        if (mode == kModeNucleus) q += cluster.map_shared_rank(hq, r2)[b];
      }
      rcnt[j] = c;
      rq[j] = q;
      rc_local += c;
      rq_local += q;
    }
    {
      uint32_t tc = block_sum_u32<kFastThreads>(rc_local, sc.redu);
      // 64-bit integer block sum via two 32-bit halves would overflow partial
      // sums; reduce with a warp tree on unsigned long long instead
      unsigned long long v = rq_local;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
      unsigned long long *wq = reinterpret_cast<unsigned long long *>(sc.redd);
      if ((tid & 31) == 0) wq[tid >> 5] = v;
      __syncthreads();
      if (tid == 0) {
        unsigned long long t = 0;
        for (int w = 0; w < kFastWarps; ++w) t += wq[w];
        ctl.rcnt = tc;
        ctl.rq = t;
      }
    }
    cluster.sync();  // -------------------------------------------------- S3
    pull_ctl<C>(cluster, ctl, lctl);
    // every CTA: total weight, threshold, crossing range and bin
    double total = 0.0;
    unsigned long long qtot = 0;
    uint32_t ctot = 0;
    uint32_t rc_all[C];
    unsigned long long rq_all[C];
    for (int q = 0; q < C; ++q) {
      const FastCtl *rc = &lctl[q];
      rc_all[q] = rc->rcnt;
      rq_all[q] = rc->rq;
      qtot += rq_all[q];
      ctot += rc_all[q];
      if (mode == kModeNucleus) total += rc->sum;
    }
    const double thr = mode == kModeTopK ? (double)keff : P * (double)qtot;
    // running totals are exact integers (counts, or 2^-44 fixed-point weights)
    auto reached = [&](unsigned long long cum_c, unsigned long long cum_q) -> bool {
      return mode == kModeTopK ? (double)cum_c >= thr : (double)cum_q >= thr;
    };
    int crange = -1;
    {
      unsigned long long ac = 0, aq = 0;
      for (int q = 0; q < C; ++q) {
        if (rc_all[q] > 0u && reached(ac + rc_all[q], aq + rq_all[q])) {
          crange = q;
          break;
        }
        ac += rc_all[q];
        aq += rq_all[q];
      }
    }
    int gather = 0;  // 0: none, 1: bins <= b*, 2: bin b* only
    int bstar = kXBins;
    uint32_t above_cnt = 0, in_cnt = 0;
    unsigned long long above_q = 0;
    if (crange >= 0) {
      // one thread per bin of the owner's reduced range; a block scan finds
      // the first non-empty bin whose running total reaches thr
      unsigned long long cb = 0, qb = 0;
      for (int q = 0; q < crange; ++q) {
        cb += rc_all[q];
        qb += rq_all[q];
      }
      const uint32_t *orc = cluster.map_shared_rank(rcnt, crange);
      const unsigned long long *orq = cluster.map_shared_rank(rq, crange);
      const unsigned long long c = tid < NBR ? (unsigned long long)orc[tid] : 0ull;
      const unsigned long long qq = (tid < NBR && mode == kModeNucleus) ? orq[tid] : 0ull;
      unsigned long long cex, cin, ctt, qex, qin, qtt;
      block_scan<kFastThreads, unsigned long long>(c, cex, cin, ctt,
                                                   reinterpret_cast<unsigned long long *>(sc.redd));
      block_scan<kFastThreads, unsigned long long>(qq, qex, qin, qtt,
                                                   reinterpret_cast<unsigned long long *>(sc.redd));
      const bool hit = tid < NBR && c > 0ull && reached(cb + cin, qb + qin);
      const int j = block_min_i<kFastThreads>(hit ? tid : 0x7FFFFFFF, sc.redi);
      if (j != 0x7FFFFFFF) {
        if (tid == j) {
          sc.bi[0] = crange * NBR + j;
          sc.bi[1] = (int)(cb + cex);
          sc.bi[2] = (int)c;
          sc.bd[0] = __longlong_as_double((long long)(qb + qex));
        }
        __syncthreads();
        bstar = sc.bi[0];
        above_cnt = (uint32_t)sc.bi[1];
        in_cnt = (uint32_t)sc.bi[2];
        above_q = (unsigned long long)__double_as_longlong(sc.bd[0]);
        __syncthreads();
      }
    }
    if (bstar < kXBins) {
      if (above_cnt + in_cnt <= (uint32_t)kCap)
        gather = 1;
      else if (mode == kModeNucleus && in_cnt <= (uint32_t)kCap)
        gather = 2;
    }
    if (gather == 0) {
      // NUCLEUS whose threshold was never reached keeps every valid token
      // (the reference's loop ran out); anything else goes to the generic path
      if (mode == kModeNucleus && crange < 0) {
        mode = kModeFull;  // reuse my_sum and total below
      } else {
        if (leader && tid == 0) a.status[row] = kRowPending;
        cluster.sync();
        return;
      }
    }
    if (gather) {
      // ---------------------------------------- compact candidates locally
      int mine = 0;
      for (int i = t0; i < t1; ++i) {
        const float v = fv<DT>(keys, i);
        if (!(v > -INFINITY)) continue;
        int b = xbin(v, vmax, xscale);
        mine += (gather == 1 ? b <= bstar : b == bstar) ? 1 : 0;
      }
      int ex, inc, tot;
      block_scan<kFastThreads, int>(mine, ex, inc, tot, sc.redi);
      if (tot <= kCap) {
        int pos = ex;
        for (int i = t0; i < t1 && pos < inc; ++i) {
          const float v = fv<DT>(keys, i);
          if (!(v > -INFINITY)) continue;
          int b = xbin(v, vmax, xscale);
          if (gather == 1 ? b <= bstar : b == bstar) {
            ckey[pos] = fkey(v);
            cidx[pos] = lo + i;
            ++pos;
          }
        }
      }
      if (tid == 0) ctl.ncand = tot;
      cluster.sync();  // ------------------------------------------------ S4
      int offs[C + 1];
      offs[0] = 0;
      pull_ctl<C>(cluster, ctl, lctl);
      for (int q = 0; q < C; ++q) offs[q + 1] = offs[q] + lctl[q].ncand;
      const int ntot = offs[C];
      if (ntot > kCap) {  // cannot happen (counts are exact); stay safe
        if (leader && tid == 0) a.status[row] = kRowPending;
        cluster.sync();
        return;
      }
      if (leader) {
        for (int q = 1; q < C; ++q) {
          const uint32_t *rk = cluster.map_shared_rank(ckey, q);
          const int *ri = cluster.map_shared_rank(cidx, q);
          for (int j = tid; j < offs[q + 1] - offs[q]; j += kFastThreads) {
            ckey[offs[q] + j] = rk[j];
            cidx[offs[q] + j] = ri[j];
          }
        }
      }
      cluster.sync();  // ------------------------------------------------ S5
      if (gather == 1) {
        if (!leader) return;
        // ---------------------------------------- leader: exact finish
        __syncthreads();
        // rank of each candidate in (key desc, index asc) order
        for (int i = tid; i < ntot; i += kFastThreads) {
          const uint32_t ki = ckey[i];
          int r2 = 0;
          for (int j = 0; j < ntot; ++j) {
            const uint32_t kj = ckey[j];
            r2 += (kj > ki || (kj == ki && j < i)) ? 1 : 0;
          }
          crank[i] = r2;
        }
        __syncthreads();
        const int m = mode == kModeTopK ? keff : ntot;  // kept before top-p
        for (int i = tid; i < ntot; i += kFastThreads) {
          if (crank[i] < m) {
            skey[crank[i]] = ckey[i];
            sidx[crank[i]] = cidx[i];
          }
        }
        __syncthreads();
        // softmax normaliser over the kept set
        double tot_m;
        if (mode == kModeTopK) {
          double s = 0.0;
          for (int r2 = tid; r2 < m; r2 += kFastThreads)
            s += exp(((double)key_to_float(skey[r2]) - dmax) * inv_t);
          tot_m = block_sum<kFastThreads>(s, sc.redd);
        } else {
          tot_m = total;
        }
        int nkeep = m;
        if (P < 1.0) {
          // running sum in sorted order; first position reaching P * tot_m
          const int per = (m + kFastThreads - 1) / kFastThreads;
          const int p0 = tid * per, p1 = min(m, p0 + per);
          double s = 0.0;
          for (int r2 = p0; r2 < p1; ++r2) s += exp(((double)key_to_float(skey[r2]) - dmax) * inv_t);
          double ex2, inc2, tot2;
          block_scan<kFastThreads, double>(s, ex2, inc2, tot2, sc.redd);
          const double target = P * tot_m;
          int cand = 0x7FFFFFFF;
          if (p0 < p1 && inc2 >= target) {
            double acc3 = ex2;
            for (int r2 = p0; r2 < p1; ++r2) {
              acc3 += exp(((double)key_to_float(skey[r2]) - dmax) * inv_t);
              if (acc3 >= target) {
                cand = r2;
                break;
              }
            }
            if (cand == 0x7FFFFFFF) cand = p1 - 1;
          }
          int first = block_min_i<kFastThreads>(cand, sc.redi);
          if (first != 0x7FFFFFFF) nkeep = first + 1;
        }
        // index-order draw over candidates with rank < nkeep
        const int per = (ntot + kFastThreads - 1) / kFastThreads;
        const int p0 = tid * per, p1 = min(ntot, p0 + per);
        double s = 0.0;
        for (int i = p0; i < p1; ++i)
          if (crank[i] < nkeep) s += exp(((double)key_to_float(ckey[i]) - dmax) * inv_t);
        double ex3, inc3, tot3;
        block_scan<kFastThreads, double>(s, ex3, inc3, tot3, sc.redd);
        const double tot_p = tot3;
        if (!(U > 0.0)) {
          if (tid == 0) {
            double w0 = (ntot > 0 && cidx[0] == 0 && crank[0] < nkeep)
                            ? exp(((double)key_to_float(ckey[0]) - dmax) * inv_t)
                            : 0.0;
            write_row(a, row, 0, (float)(w0 / tot_p), (int32_t)fl);
          }
          return;
        }
        const double target = U * tot_p;
        int cand = (s > 0.0 && inc3 >= target) ? tid : 0x7FFFFFFF;
        int who = block_min_i<kFastThreads>(cand, sc.redi);
        if (who == 0x7FFFFFFF) {
          if (tid == 0) {
            // the reference's loop ran past the end: V-1
            double wl = (ntot > 0 && cidx[ntot - 1] == V - 1 && crank[ntot - 1] < nkeep)
                            ? exp(((double)key_to_float(ckey[ntot - 1]) - dmax) * inv_t)
                            : 0.0;
            write_row(a, row, V - 1, (float)(wl / tot_p), (int32_t)fl);
          }
          return;
        }
        if (tid == who) {
          double acc3 = ex3;
          int tok = -1, last = -1;
          double wt = 0.0, wl = 0.0;
          for (int i = p0; i < p1; ++i) {
            if (crank[i] >= nkeep) continue;
            double w = exp(((double)key_to_float(ckey[i]) - dmax) * inv_t);
            acc3 += w;
            last = cidx[i];
            wl = w;
            if (acc3 >= target) {
              tok = cidx[i];
              wt = w;
              break;
            }
          }
          if (tok < 0) {
            tok = last;
            wt = wl;
          }
          write_row(a, row, tok, (float)(wt / tot_p), (int32_t)fl);
        }
        return;
      }
      // gather == 2: the leader places the top-p cut inside bin b*
      if (leader) {
        for (int i = tid; i < ntot; i += kFastThreads) {
          const uint32_t ki = ckey[i];
          int r2 = 0;
          for (int j = 0; j < ntot; ++j) {
            const uint32_t kj = ckey[j];
            r2 += (kj > ki || (kj == ki && j < i)) ? 1 : 0;
          }
          skey[r2] = ki;
          sidx[r2] = cidx[i];
        }
        __syncthreads();
        // same fixed-point weights as the histogram, so the cut agrees with it
        const int per = (ntot + kFastThreads - 1) / kFastThreads;
        const int p0 = tid * per, p1 = min(ntot, p0 + per);
        unsigned long long qs = 0;
        for (int r2 = p0; r2 < p1; ++r2)
          qs += qweight(exp(((double)key_to_float(skey[r2]) - dmax) * inv_t));
        unsigned long long qex, qin, qtt;
        block_scan<kFastThreads, unsigned long long>(qs, qex, qin, qtt,
                                                     reinterpret_cast<unsigned long long *>(sc.redd));
        int cand = 0x7FFFFFFF;
        if (p0 < p1 && (double)(above_q + qin) >= thr) {
          unsigned long long accq = above_q + qex;
          for (int r2 = p0; r2 < p1; ++r2) {
            accq += qweight(exp(((double)key_to_float(skey[r2]) - dmax) * inv_t));
            if ((double)accq >= thr) {
              cand = r2;
              break;
            }
          }
          if (cand == 0x7FFFFFFF) cand = p1 - 1;
        }
        int r_cut = block_min_i<kFastThreads>(cand, sc.redi);
        if (r_cut == 0x7FFFFFFF) r_cut = ntot - 1;
        if (tid < C) {
          FastCtl *rc = cluster.map_shared_rank(&ctl, tid);
          rc->cut_key = skey[r_cut];
          rc->cut_idx = sidx[r_cut];
        }
      }
      cluster.sync();  // ------------------------------------------------ S6
      cut.v = key_to_float(ctl.cut_key);
      cut.idx = ctl.cut_idx;
      // weights of the kept set in my run
      my_sum = 0.0;
      for (int i = t0; i < t1; ++i) {
        const float v = fv<DT>(keys, i);
        if (v > -INFINITY && fkept(cut, v, lo + i)) my_sum += exp(((double)v - dmax) * inv_t);
      }
      double s = block_sum<kFastThreads>(my_sum, sc.redd);
      if (tid == 0) ctl.sum = s;
      cluster.sync();  // ------------------------------------------------ S7
      mode = kModeFull;
    }
  } else {
    // FULL: every valid token is kept
    for (int i = t0; i < t1; ++i) {
      const float v = fv<DT>(keys, i);
      if (v > -INFINITY) my_sum += exp(((double)v - dmax) * inv_t);
    }
    double s = block_sum<kFastThreads>(my_sum, sc.redd);
    if (tid == 0) ctl.sum = s;
    cluster.sync();  // ---------------------------------------------------- S2
  }

  // ------------------------------------------------- index-order draw (FULL)
  {
    pull_ctl<C>(cluster, ctl, lctl);
    double sums[C];
    double total = 0.0;
    for (int q = 0; q < C; ++q) {
      sums[q] = lctl[q].sum;
      total += sums[q];
    }
    auto wt = [&](int i) -> double {  // i: slice-local index
      const float v = fv<DT>(keys, i);
      return (v > -INFINITY && fkept(cut, v, lo + i)) ? exp(((double)v - dmax) * inv_t) : 0.0;
    };
    if (!(U > 0.0)) {
      if (rank == 0 && tid == 0) write_row(a, row, 0, (float)(wt(0) / total), (int32_t)fl);
    } else {
      const double target = U * total;
      int cstar = -1;
      double before = 0.0, acc = 0.0;
      for (int q = 0; q < C; ++q) {
        if (sums[q] > 0.0 && acc + sums[q] >= target) {
          cstar = q;
          before = acc;
          break;
        }
        acc += sums[q];
      }
      if (cstar < 0) {
        const int owner = (V - 1) / S;
        if (rank == owner && tid == 0)
          write_row(a, row, V - 1, (float)(wt(V - 1 - lo) / total), (int32_t)fl);
      } else if (rank == cstar) {
        double ex, inc, tot;
        block_scan<kFastThreads, double>(my_sum, ex, inc, tot, sc.redd);
        int cand = (my_sum > 0.0 && before + inc >= target) ? tid : 0x7FFFFFFF;
        int who = block_min_i<kFastThreads>(cand, sc.redi);
        if (who == 0x7FFFFFFF) {
          // rounding left the crossing past this CTA's partial sums: take
          // the last kept element of the CTA
          int lastt = my_sum > 0.0 ? tid : -1;
          lastt = -block_min_i<kFastThreads>(-lastt, sc.redi);
          who = lastt;
        }
        if (tid == who) {
          double cum = before + ex;
          int tok = -1, last = -1;
          double wtk = 0.0, wl = 0.0;
          for (int i = t0; i < t1; ++i) {
            double w = wt(i);
            if (w <= 0.0) continue;
            cum += w;
            last = lo + i;
            wl = w;
            if (cum >= target) {
              tok = lo + i;
              wtk = w;
              break;
            }
          }
          if (tok < 0) {
            tok = last;
            wtk = wl;
          }
          write_row(a, row, tok, (float)(wtk / total), (int32_t)fl);
        }
      }
    }
  }
  cluster.sync();  // keep every slice alive until all remote reads are done
}

}  // namespace ms
