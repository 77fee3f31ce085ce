// Streaming sampling kernel: one 512-thread CTA per logits row, two CTAs per
// SM.  The row streams from HBM through a 48 KB ring of shared-memory stages
// filled by cp.async.bulk (TMA) copies -- three 16 KB stages of fp32 or six
// 8 KB stages of bf16, so both dtypes keep the same bytes in flight -- and
// every synchronisation is CTA-local.  A chunk is 4096 elements; each warp
// owns one "unit" of every chunk: 256 consecutive elements.
//
//   argmax rows (temperature 0, or top_k == 1)  one pass: per-thread first
//                                                maximum, block argmax
//   top-k rows (2 <= top_k <= kStTopK)          one pass: the candidate
//                                                threshold is a value of chunk
//                                                0 that the row's top-k set
//                                                lies above unless chunk 0
//                                                holds an unlikely share of
//                                                it; the buffer's size proves
//                                                it (else a second pass with
//                                                thresholds from running
//                                                maxima); exact finish on the
//                                                buffer
//   full-softmax rows (no top-k, top_p >= 1)    one pass: per-unit weight
//                                                sums; the draw re-reads one
//                                                unit
//   top-p-only rows                             pass 1: every weight (the
//                                                exact total) and the unit
//                                                maxima.  When the largest
//                                                unit maxima alone reach
//                                                top_p of the total (a narrow
//                                                nucleus) the units holding
//                                                them are re-read and every
//                                                value above the bound they
//                                                give is captured: the whole
//                                                nucleus.  Otherwise (L2) an
//                                                x-grid histogram brackets the
//                                                crossing, and a classifying
//                                                pass over the units that
//                                                reach the bracket takes the
//                                                per-unit mass above it and
//                                                the bracket's elements.
//                                                Exact cut, one-unit draw.
//
// Every weight of a softmax row is one function of the logit,
// W(v) = 2^(v * log2(e)/T - a) in fp32 with a row anchor a (the maximum of the
// first chunk holding a finite value, times log2(e)/T), so totals, cuts and
// draws agree with each other to the last bit of each term.
//
// Semantics follow miniserve/sampler.py:23-68 (see ms_sample.cu).  Rows
// outside what this kernel finishes exactly (NaN or +inf logits, top_k above
// kStTopK that may still cut, candidate buffers overflowing on heavy ties,
// temperatures below 1e-30) get status kRowPending and are finished by
// ms_generic_pending_kernel.
#pragma once

#include <cfloat>

#include "ms_common.cuh"
#include "ms_exchange.cuh"
#include "ms_generic.cuh"
#include "ms_shard.cuh"

namespace ms {

constexpr int kStThreads = 512;
constexpr int kStWarps = kStThreads / 32;
constexpr int kUnit = 256;                      // elements per unit: one warp's share of a chunk
constexpr int kChunk = kStWarps * kUnit;        // elements per chunk (one TMA copy)
constexpr int kRingBytes = 3 * kChunk * 4;      // the stage ring: 3 fp32 or 6 bf16 chunks
constexpr int kMaxStages = 6;
constexpr int kScratchBytes = 16384;            // the ring doubles as three 16 KB scratch areas after the passes
template <int DT>
__host__ __device__ constexpr int st_esz() {
  return DT == MS_DTYPE_F32 ? 4 : 2;
}
template <int DT>
__host__ __device__ constexpr int st_nstages() {  // single-chunk stages in the ring
  return kRingBytes / (kChunk * st_esz<DT>());
}
constexpr int kCandCap = 6144;                  // top-k candidate buffer entries
constexpr int kSortCap = 4096;                  // largest set st_sort handles
constexpr int kRankCap = 1024;                  // largest set sorted by rank counting
constexpr int kStTopK = 512;                    // largest top_k resolved by the streaming pass (a rank per thread)
constexpr int kMaxUnits = 2048;                 // per-unit summaries kept per row
constexpr int kStreamMaxV = kMaxUnits * kUnit;  // longest row this kernel takes
constexpr int kNarrowUnits = 128;               // top-p: the unit maxima tried as a narrow nucleus's bound
constexpr int kXBins = 4096;                    // x-grid bins per kSXRange (top-p histogram)
constexpr float kSXRange = 40.0f;               // units of x = logit / T
constexpr int kUpBins = 1024;                   // grid bins above the anchor
constexpr int kSBins = kXBins + kUpBins;        // x-grid bins in all
constexpr int kHighCap = 256;                   // values above the grid kept exactly
constexpr int kQSlots = (kSBins + 2 + kStThreads - 1) / kStThreads * kStThreads;  // histogram indices 0..kSBins+1
constexpr float kQScale = 65536.0f;             // fixed-point scale of in-bin weights
constexpr double kHistTol = 4e-5;               // bound on the histogram's running-mass error / total
constexpr double kMinTemperature = 1e-30;       // fp32 weights need a finite log2(e)/T

struct StShared {
  alignas(128) unsigned char ring[kRingBytes];
  alignas(16) uint32_t mstage[kMaxStages][kChunk / 32];  // each chunk's allowed-token bits (StRow::mtma)
  union {
    struct {
      uint32_t key[kCandCap];
      int idx[kCandCap];
    } c;  // top-k candidates
    struct {
      float m[kMaxUnits];  // unit maxima
      float s[kMaxUnits];  // full softmax: unit weight sums; top-p: the unit's mass above the bracket
      uint32_t hkey[kHighCap];  // values above the x-grid
      int hidx[kHighCap];
      union {
        uint32_t hq[kQSlots];  // x-grid histogram (fixed-point mass)
        struct {
          uint32_t key[kSortCap];
          int idx[kSortCap];
        } g;  // captured elements: the nucleus, or the bracket's elements
      } x;
    } n;
  } w;
  uint32_t wbound[kStWarps];
  int pick[kStWarps][4];  // row ordering: per-warp class counts, then their prefix over the warps
  alignas(16) uint32_t sel[4][256];  // st_select_kth: one digit histogram per round
  unsigned long long full[kMaxStages];
  double r1d[2][64];  // one-barrier reductions (st_bsum and friends): two halves
  int r1i[2][32];
  uint32_t redu[33];
  int redi[33];
  float redf[33];
  int bcast_i[8];
  float bcast_f[4];
  double bcast_d[4];
  int ncand;
  int nhigh;
  // a top-p row shared by the two CTAs of a cluster: each slot is written by
  // the partner CTA (st_peer_*) before a st_cluster_sync, then read locally
  struct {
    float g;          // the partner's first-chunk maximum
    double z0, t0;    // the partner's prediction sums on its first chunk, relative to g
    uint32_t flags;   // bit 0 NaN/+inf, bit 1 a copy timed out, bit 2 a weight beyond range, bit 3 overflow
    float vmax;       // the partner's maximum
    double zsum;      // the partner's weight total
    int nhigh;        // the partner's high-list entries
    int ncand;        // the partner's captured entries
    int kind;         // rank 0's decision (rank 1 reads it)
    float v_lo, v_hi;
    int tail;
  } xch;
};

// scratch area i (0..2) of the ring, free once no copy is in flight
__device__ __forceinline__ unsigned char *st_scratch(StShared &sh, int i) { return sh.ring + kScratchBytes * i; }

template <int DT>
__device__ __forceinline__ const unsigned char *st_stage(const StShared &sh, int s) {
  return sh.ring + s * (kChunk * st_esz<DT>());
}

// ------------------------------------------------------------- the stream
struct StRow {
  const char *g;        // row start in global memory
  const uint32_t *mask; // row of the allowed-token bitmask, or null
  int V;
  bool tma;             // 16-byte aligned row: chunks arrive by TMA
  bool mtma;            // 16-byte aligned mask row too: whole chunks' mask words arrive with them
  int nchunks;
  int nfull;            // leading chunks delivered whole by TMA
};

__device__ __forceinline__ uint32_t st_smem(const void *p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

// ---- clusters of two CTAs sharing a top-p row.  Data crosses between the
// two CTAs only as stores into the partner's shared memory followed by
// st_cluster_sync, which every thread of both CTAs reaches at the same points
// of the shared row's code; the first one comes before any such store, so
// both CTAs have started.
__device__ __forceinline__ uint32_t st_crank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// the partner CTA's shared-memory address of p
__device__ __forceinline__ uint32_t st_peer(const void *p) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(st_smem(p)), "r"(st_crank() ^ 1u));
  return r;
}
__device__ __forceinline__ void st_peer_u32(uint32_t ra, uint32_t v) {
  asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(ra), "r"(v) : "memory");
}
__device__ __forceinline__ void st_peer_f32(uint32_t ra, float v) {
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(ra), "f"(v) : "memory");
}
__device__ __forceinline__ void st_peer_f64(uint32_t ra, double v) {
  asm volatile("st.shared::cluster.f64 [%0], %1;" ::"r"(ra), "d"(v) : "memory");
}
__device__ __forceinline__ void st_peer_v4(uint32_t ra, uint4 v) {
  asm volatile("st.shared::cluster.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(ra), "r"(v.x), "r"(v.y), "r"(v.z),
               "r"(v.w)
               : "memory");
}
// every thread of both CTAs; stores before it are visible to both after it
__device__ __forceinline__ void st_cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
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

// Elements of chunk c delivered by TMA (a multiple of 16 bytes); elements past
// them (at most 3 fp32 / 7 bf16 at the row's end) are read from global memory.
template <int DT>
__device__ __forceinline__ int tma_elems(const StRow &r, int c) {
  if (!r.tma) return 0;
  const int ne = min(kChunk, r.V - c * kChunk);
  return ne & -(16 / st_esz<DT>());
}

// Chunks per stage: bf16 passes without per-chunk counts carry two chunks
// (16 KB) per stage, so a stage moves as many bytes as an fp32 one and the
// chunk barrier and copy issue are paid once per 8192 values.  Sub-chunk k of
// stage s occupies the memory (and mask words) of single-chunk stage
// s * SUB + k.
template <int DT, bool COUNT>
__host__ __device__ constexpr int st_sub() {
  return DT != MS_DTYPE_F32 && !COUNT ? 2 : 1;
}

// thread 0: start the copies of chunks [c, min(c + SUB, c1)) into stage s
// (and, for whole chunks of a row with an aligned mask row, of their kChunk /
// 32 mask words each), all completing on stage s's barrier
template <int DT, int SUB = 1>
__device__ __forceinline__ void st_issue(StShared &sh, const StRow &r, int c, int s, uint64_t pol,
                                         int c1 = 0x7FFFFFFF) {
  const int n = min(SUB, c1 - c);
  const int sb = s * SUB;  // single-chunk stage of the first chunk
  uint32_t b[SUB], m[SUB], bytes = 0, mbytes = 0;
#pragma unroll
  for (int k = 0; k < SUB; ++k) {
    b[k] = k < n ? (uint32_t)(tma_elems<DT>(r, c + k) * st_esz<DT>()) : 0u;
    m[k] = k < n && r.mtma && c + k < r.nfull ? (uint32_t)(kChunk / 8) : 0u;
    bytes += b[k];
    mbytes += m[k];
  }
  const uint32_t mb = st_smem(&sh.full[s]);
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(mb), "r"(bytes + mbytes) : "memory");
  // a whole first chunk is followed by the next one in both memories: one copy
  const bool one = SUB == 1 || b[0] == (uint32_t)(kChunk * st_esz<DT>());
#pragma unroll
  for (int k = 0; k < SUB; ++k) {
    const uint32_t bk = one ? (k == 0 ? bytes : 0u) : b[k];
    if (bk) {
      asm volatile(
          "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
              st_smem(st_stage<DT>(sh, sb + k))),
          "l"(r.g + (int64_t)(c + k) * kChunk * st_esz<DT>()), "r"(bk), "r"(mb), "l"(pol)
          : "memory");
    }
  }
  const bool mone = SUB == 1 || m[0] != 0u;  // whole chunks have their words contiguous too
#pragma unroll
  for (int k = 0; k < SUB; ++k) {
    const uint32_t mk = mone ? (k == 0 ? mbytes : 0u) : m[k];
    if (mk) {
      asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                       st_smem(sh.mstage[sb + k])),
                   "l"(r.mask + (int64_t)(c + k) * (kChunk / 32)), "r"(mk), "r"(mb)
                   : "memory");
    }
  }
}

__device__ __forceinline__ bool st_try_wait(uint32_t mb, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
      : "=r"(done)
      : "r"(mb), "r"(parity)
      : "memory");
  return done != 0;
}

// the rare case of st_wait: keep probing, false after ~1 s
__device__ __noinline__ bool st_wait_slow(uint32_t mb, uint32_t parity) {
  const uint64_t t0 = st_ns();
  for (uint32_t it = 1;; ++it) {
    if (st_try_wait(mb, parity)) return true;
    if ((it & 1023u) == 0u && st_ns() - t0 > 1000000000ull) return false;
  }
}

// all threads: wait for the current phase of stage s; false after ~1 s
__device__ __forceinline__ bool st_wait(StShared &sh, int s, uint32_t parity) {
  const uint32_t mb = st_smem(&sh.full[s]);
  return st_try_wait(mb, parity) || st_wait_slow(mb, parity);
}

// Four consecutive elements (chunk-local j, a multiple of 4) of chunk c in
// stage s, masked tokens and positions past the row read as -inf.
template <int DT>
__device__ __forceinline__ void st_get4(const StShared &sh, const StRow &r, int c, int s, int j,
                                        float x[4]) {
  const int ne = min(kChunk, r.V - c * kChunk);
  const int nt = tma_elems<DT>(r, c);
  const unsigned char *st = st_stage<DT>(sh, s);
  if (j + 4 <= nt) {
    if (DT == MS_DTYPE_F32) {
      const float4 f = reinterpret_cast<const float4 *>(st)[j >> 2];
      x[0] = f.x;
      x[1] = f.y;
      x[2] = f.z;
      x[3] = f.w;
    } else {
      const uint2 h = reinterpret_cast<const uint2 *>(st)[j >> 2];
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
        x[e] = DT == MS_DTYPE_F32 ? reinterpret_cast<const float *>(st)[jj]
                                  : __uint_as_float((uint32_t)reinterpret_cast<const uint16_t *>(st)[jj] << 16);
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

// This thread's 8 elements of chunk c (in stage s): x[0..3] at chunk offset
// warp*kUnit + lane*4, x[4..7] 128 further on, so a warp's 256 values are one
// unit.  Returns the global index of x[0].
template <int DT>
__device__ __forceinline__ int st_get8(const StShared &sh, const StRow &r, int c, int s, float x[8]) {
  const int j = (threadIdx.x >> 5) * kUnit + (threadIdx.x & 31) * 4;
  if (c < r.nfull) {  // the whole chunk is in the stage (block-uniform)
    const unsigned char *st = st_stage<DT>(sh, s);
    if (DT == MS_DTYPE_F32) {
      const float4 *p = reinterpret_cast<const float4 *>(st);
      const float4 f0 = p[j >> 2], f1 = p[(j + 128) >> 2];
      x[0] = f0.x;
      x[1] = f0.y;
      x[2] = f0.z;
      x[3] = f0.w;
      x[4] = f1.x;
      x[5] = f1.y;
      x[6] = f1.z;
      x[7] = f1.w;
    } else {
      const uint2 *p = reinterpret_cast<const uint2 *>(st);
      const uint2 h0 = p[j >> 2], h1 = p[(j + 128) >> 2];
      x[0] = __uint_as_float(h0.x << 16);
      x[1] = __uint_as_float(h0.x & 0xFFFF0000u);
      x[2] = __uint_as_float(h0.y << 16);
      x[3] = __uint_as_float(h0.y & 0xFFFF0000u);
      x[4] = __uint_as_float(h1.x << 16);
      x[5] = __uint_as_float(h1.x & 0xFFFF0000u);
      x[6] = __uint_as_float(h1.y << 16);
      x[7] = __uint_as_float(h1.y & 0xFFFF0000u);
    }
    if (r.mask) {  // each group of 4 lies in one 32-bit mask word
      uint32_t m0, m1;
      if (r.mtma) {  // the chunk's words arrived with it (kChunk is a multiple of 32)
        const uint32_t *mw = sh.mstage[s] + (j >> 5);
        m0 = mw[0] >> (j & 31);
        m1 = mw[4] >> (j & 31);
      } else {
        const int g0 = c * kChunk + j, g1 = g0 + 128;
        m0 = __ldg(r.mask + (g0 >> 5)) >> (g0 & 31);
        m1 = __ldg(r.mask + (g1 >> 5)) >> (g1 & 31);
      }
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        if (!((m0 >> e) & 1u)) x[e] = -INFINITY;
        if (!((m1 >> e) & 1u)) x[4 + e] = -INFINITY;
      }
    }
  } else {
    st_get4<DT>(sh, r, c, s, j, x);
    st_get4<DT>(sh, r, c, s, j + 128, x + 4);
  }
  return c * kChunk + j;
}

// The same 8 elements of unit u (x[0..3] at u*kUnit + lane*4, x[4..7] 128
// further on) read from global memory, masked tokens and positions past the
// row as -inf.  Returns the global index of x[0].
template <int DT>
__device__ __forceinline__ int st_load_unit(const StRow &r, int u, float x[8]) {
  const int j0 = u * kUnit + (threadIdx.x & 31) * 4;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int j = j0 + 128 * h;
    float *y = x + 4 * h;
    if (r.tma && j + 4 <= r.V) {
      if (DT == MS_DTYPE_F32) {
        const float4 f = __ldg(reinterpret_cast<const float4 *>(r.g) + (j >> 2));
        y[0] = f.x;
        y[1] = f.y;
        y[2] = f.z;
        y[3] = f.w;
      } else {
        const uint2 v = __ldg(reinterpret_cast<const uint2 *>(r.g) + (j >> 2));
        y[0] = __uint_as_float(v.x << 16);
        y[1] = __uint_as_float(v.x & 0xFFFF0000u);
        y[2] = __uint_as_float(v.y << 16);
        y[3] = __uint_as_float(v.y & 0xFFFF0000u);
      }
    } else {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int jj = j + e;
        y[e] = jj >= r.V ? -INFINITY
               : DT == MS_DTYPE_F32
                   ? __ldg(reinterpret_cast<const float *>(r.g) + jj)
                   : __uint_as_float((uint32_t)__ldg(reinterpret_cast<const unsigned short *>(r.g) + jj) << 16);
      }
    }
    if (r.mask && j < r.V) {  // j..j+3 lie in one mask word
      const uint32_t mw = __ldg(r.mask + (j >> 5)) >> (j & 31);
#pragma unroll
      for (int e = 0; e < 4; ++e)
        if (!((mw >> e) & 1u)) y[e] = -INFINITY;
    }
  }
  return j0;
}

// Maxima that let a NaN through (max.NaN), so one running maximum both finds
// the row's largest value and flags a NaN; a row holding NaN or +inf
// (st_bad) leaves the fast paths.
__device__ __forceinline__ float st_maxn(float a, float b) {
  float d;
  asm("max.NaN.f32 %0, %1, %2;" : "=f"(d) : "f"(a), "f"(b));
  return d;
}
__device__ __forceinline__ float st_max3n(float a, float b, float c) {
  float d;
  asm("max.NaN.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}
__device__ __forceinline__ float st_max8n(const float *x) {
  return st_max3n(st_max3n(x[0], x[1], x[2]), st_max3n(x[3], x[4], x[5]), st_maxn(x[6], x[7]));
}
__device__ __forceinline__ bool st_bad(float running_max) { return !(running_max < INFINITY); }
// the warp's maximum (a NaN drops out)
__device__ __forceinline__ float st_warp_max(float v) {
  float r;
  asm("redux.sync.max.f32 %0, %1, 0xffffffff;" : "=f"(r) : "f"(v));
  return r;
}

// x[e] for a run-time e without indexing the array (which would put it in
// local memory)
__device__ __forceinline__ float st_pick8(const float *x, int e) {
  const float a = (e & 1) ? x[1] : x[0], b = (e & 1) ? x[3] : x[2];
  const float c = (e & 1) ? x[5] : x[4], d = (e & 1) ? x[7] : x[6];
  const float ab = (e & 2) ? b : a, cd = (e & 2) ? d : c;
  return (e & 4) ? cd : ab;
}

// global index of x[e] given that of x[0]
__device__ __forceinline__ int st_gidx(int g0, int e) { return e < 4 ? g0 + e : g0 + 124 + e; }

// Wait for the copies of chunks [c, ce) still in flight after an early exit
// from a pass over chunks from c0 with SUB chunks per stage (c - c0 a
// multiple of SUB; chunk c sits in stage ((c - c0) / SUB) % stages).
template <int DT, int SUB = 1>
__device__ bool st_drain(StShared &sh, int c0, int c, int ce, uint32_t &ph) {
  constexpr int S = st_nstages<DT>() / SUB;
  bool ok = true;
  for (int c2 = c; c2 < ce; c2 += SUB) {
    const int s2 = ((c2 - c0) / SUB) % S;
    if (!st_wait(sh, s2, (ph >> s2) & 1u)) ok = false;
    ph ^= 1u << s2;
  }
  return ok;
}

struct StNoAfter {
  __device__ __forceinline__ bool operator()(int, int) const { return false; }
};

// One pass over chunks [c0, c1) of the row: `body(x[8], g0, u, c)` sees this
// thread's 8 values of chunk c (st_get8 layout; u = the warp's unit number,
// index order).  With COUNT, body returns this thread's flag, and after the
// chunk's barrier and the refill of its stage, `after(c, n)` (n = threads
// whose flag was set) runs in every thread and may end the pass early by
// returning true.  Returns false when a copy timed out.  `ph` carries the
// stages' phase parities across passes.  With `issued`, the copies of the
// first stages are already under way (st_peek, or the kernel's prologue).
// bf16 passes without COUNT take two chunks per stage (st_sub).
template <int DT, bool COUNT, class Body, class After>
__device__ __forceinline__ bool st_stream(StShared &sh, const StRow &r, int c0, int c1, uint64_t pol, uint32_t &ph,
                                          Body body, After after, bool issued = false) {
  constexpr int SUB = st_sub<DT, COUNT>();
  constexpr int S = st_nstages<DT>() / SUB;
  const int tid = threadIdx.x;
  if (tid == 0 && !issued) {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    for (int k = 0; k < S && c0 + k * SUB < c1; ++k) st_issue<DT, SUB>(sh, r, c0 + k * SUB, k, pol, c1);
  }
  bool ok = true;
  {
#pragma unroll 1
    for (int c = c0, s = 0; c < c1; c += SUB, s = s == S - 1 ? 0 : s + 1) {
      if (!st_wait(sh, s, (ph >> s) & 1u)) ok = false;
      ph ^= 1u << s;
      int n = 0;
#pragma unroll 1
      for (int k = 0; k < SUB; ++k) {
        const int ck = c + k;
        if (SUB > 1 && ck >= c1) break;  // block-uniform
        float x[8];
        const int g0 = st_get8<DT>(sh, r, ck, s * SUB + k, x);
        const int u = ck * kStWarps + (tid >> 5);
        if constexpr (COUNT) {
          n = __syncthreads_count(body(x, g0, u, ck));
        } else {
          body(x, g0, u, ck);
        }
      }
      if constexpr (!COUNT) __syncthreads();  // every thread is done with stage s
      if (tid == 0 && c + S * SUB < c1) {
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        st_issue<DT, SUB>(sh, r, c + S * SUB, s, pol, c1);
      }
      if constexpr (COUNT) {
        if (after(c, n)) {  // block-uniform
          if (!st_drain<DT>(sh, c0, c + 1, min(c1, c + S + 1), ph)) ok = false;
          return __syncthreads_and(ok) != 0;
        }
      }
    }
  }
  return __syncthreads_and(ok) != 0;
}

// Start a pass over chunks [c0, c1) (their first copies, unless `issued`) and
// read chunk c0 into x[8] without consuming it: st_stream(..., issued = true)
// then takes the same copies.  Returns false when the copy timed out.  All
// threads.
template <int DT>
__device__ __forceinline__ bool st_peek(StShared &sh, const StRow &r, int c0, int c1, uint64_t pol, uint32_t ph,
                                        float x[8], bool issued = false) {
  constexpr int SUB = st_sub<DT, false>();
  constexpr int S = st_nstages<DT>() / SUB;
  if (threadIdx.x == 0 && !issued) {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    for (int k = 0; k < S && c0 + k * SUB < c1; ++k) st_issue<DT, SUB>(sh, r, c0 + k * SUB, k, pol, c1);
  }
  const bool ok = st_wait(sh, 0, ph & 1u);
  st_get8<DT>(sh, r, c0, 0, x);
  return ok;
}

// The m-th largest (1 <= m <= kChunk) of the values held in x[8] by every
// thread, to its leading 16 bits (a lower bound on it, as a key): two rounds
// of 8-bit digits over the keys in registers.  All threads.
__device__ uint32_t st_sample_kth(StShared &sh, const float *x, int m) {
  const int tid = threadIdx.x, lane = tid & 31;
  uint32_t key[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) key[e] = fkey(x[e]);
  __syncthreads();  // no warp still scans the histograms of an earlier selection
  (&sh.sel[0][0])[tid] = 0u;
  __syncthreads();
  uint32_t prefix = 0;
  int rem = m;
#pragma unroll
  for (int d = 0; d < 2; ++d) {
    const int shift = 24 - 8 * d;
    uint32_t *h = sh.sel[d];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const bool in = d == 0 || (key[e] >> 24) == prefix;
      const uint32_t digit = (key[e] >> shift) & 255u;
      // keys share leading digits heavily: the first active lane's digit
      // takes one atomic for every lane that holds it
      const unsigned act = __ballot_sync(0xFFFFFFFFu, in);
      if (act) {
        const int first = __ffs(act) - 1;
        const uint32_t lead = __shfl_sync(0xFFFFFFFFu, digit, first);
        const unsigned same = __ballot_sync(0xFFFFFFFFu, in && digit == lead);
        if (lane == first) {
          atomicAdd(&h[lead], (uint32_t)__popc(same));
        } else if (in && digit != lead) {
          atomicAdd(&h[digit], 1u);
        }
      }
    }
    __syncthreads();
    // every warp: the digit whose running count from the top reaches rem;
    // lane l holds digits 255 - 8l - q, q = 0..7
    const uint4 *h4 = reinterpret_cast<const uint4 *>(h);
    const uint4 lo = h4[(248 - 8 * lane) >> 2], hi = h4[((248 - 8 * lane) >> 2) + 1];
    const uint32_t c8[8] = {hi.w, hi.z, hi.y, hi.x, lo.w, lo.z, lo.y, lo.x};
    uint32_t s8 = 0;
#pragma unroll
    for (int q = 0; q < 8; ++q) s8 += c8[q];
    uint32_t incl = s8;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t y = __shfl_up_sync(0xFFFFFFFFu, incl, o);
      if (lane >= o) incl += y;
    }
    const uint32_t excl = incl - s8;
    const unsigned hit = __ballot_sync(0xFFFFFFFFu, incl >= (uint32_t)rem && excl < (uint32_t)rem);
    uint32_t dig = 0, before = 0;
    if (hit && lane == __ffs(hit) - 1) {
      uint32_t acc = excl;
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        if (acc + c8[q] >= (uint32_t)rem) {
          dig = 255u - (uint32_t)(8 * lane + q);
          before = acc;
          break;
        }
        acc += c8[q];
      }
    }
    // no hit only for m above the values held, which callers exclude
    const int src = hit ? __ffs(hit) - 1 : 0;
    dig = __shfl_sync(0xFFFFFFFFu, dig, src);
    before = __shfl_sync(0xFFFFFFFFu, before, src);
    rem -= (int)before;
    prefix = (prefix << 8) | dig;
  }
  return prefix << 16;
}

// The m-th largest (1 <= m <= kStThreads) of one key per thread, to its
// leading 16 bits (a lower bound on it): two rounds of 8-bit digits.  Used
// with each thread's maximum of its 8 values: the m largest of those are m
// distinct values, so the result is also a lower bound on the m-th largest
// of all the values.  All threads.
__device__ uint32_t st_sample_kth1(StShared &sh, uint32_t key, int m) {
  const int tid = threadIdx.x, lane = tid & 31;
  __syncthreads();  // no warp still scans the histograms of an earlier selection
  (&sh.sel[0][0])[tid] = 0u;
  __syncthreads();
  uint32_t prefix = 0;
  int rem = m;
#pragma unroll
  for (int d = 0; d < 2; ++d) {
    const int shift = 24 - 8 * d;
    uint32_t *h = sh.sel[d];
    const bool in = d == 0 || (key >> 24) == prefix;
    const uint32_t digit = (key >> shift) & 255u;
    const unsigned act = __ballot_sync(0xFFFFFFFFu, in);
    if (act) {  // the first active lane's digit takes one atomic for every lane that holds it
      const int first = __ffs(act) - 1;
      const uint32_t lead = __shfl_sync(0xFFFFFFFFu, digit, first);
      const unsigned same = __ballot_sync(0xFFFFFFFFu, in && digit == lead);
      if (lane == first) {
        atomicAdd(&h[lead], (uint32_t)__popc(same));
      } else if (in && digit != lead) {
        atomicAdd(&h[digit], 1u);
      }
    }
    __syncthreads();
    const uint4 *h4 = reinterpret_cast<const uint4 *>(h);
    const uint4 lo = h4[(248 - 8 * lane) >> 2], hi = h4[((248 - 8 * lane) >> 2) + 1];
    const uint32_t c8[8] = {hi.w, hi.z, hi.y, hi.x, lo.w, lo.z, lo.y, lo.x};
    uint32_t s8 = 0;
#pragma unroll
    for (int q = 0; q < 8; ++q) s8 += c8[q];
    uint32_t incl = s8;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t y = __shfl_up_sync(0xFFFFFFFFu, incl, o);
      if (lane >= o) incl += y;
    }
    const uint32_t excl = incl - s8;
    const unsigned hit = __ballot_sync(0xFFFFFFFFu, incl >= (uint32_t)rem && excl < (uint32_t)rem);
    uint32_t dig = 0, before = 0;
    if (hit && lane == __ffs(hit) - 1) {
      uint32_t acc = excl;
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        if (acc + c8[q] >= (uint32_t)rem) {
          dig = 255u - (uint32_t)(8 * lane + q);
          before = acc;
          break;
        }
        acc += c8[q];
      }
    }
    const int src = hit ? __ffs(hit) - 1 : 0;
    dig = __shfl_sync(0xFFFFFFFFu, dig, src);
    before = __shfl_sync(0xFFFFFFFFu, before, src);
    rem -= (int)before;
    prefix = (prefix << 8) | dig;
  }
  return prefix << 16;
}

__device__ __forceinline__ float warp_sum_f(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
  return v;
}

// ------------------------------------------- one-barrier block reductions
// A call writes the warps' partials into one of two scratch halves,
// alternating per call (`rf` flips; every thread makes the same calls in the
// same order), and every warp combines the partials itself.  A half is
// written again only after another call's barrier, which every thread passes
// after reading it.  All threads.
__device__ __forceinline__ double st_bsum(StShared &sh, int &rf, double v) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = warp_sum(v);
  double *p = sh.r1d[rf];
  rf ^= 1;
  if (lane == 0) p[warp] = v;
  __syncthreads();
  return warp_sum(lane < kStWarps ? p[lane] : 0.0);
}
// two sums at once
__device__ __forceinline__ void st_bsum2(StShared &sh, int &rf, double a, double b, double &sa, double &sb) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  a = warp_sum(a);
  b = warp_sum(b);
  double *p = sh.r1d[rf];
  rf ^= 1;
  if (lane == 0) {
    p[warp] = a;
    p[32 + warp] = b;
  }
  __syncthreads();
  sa = warp_sum(lane < kStWarps ? p[lane] : 0.0);
  sb = warp_sum(lane < kStWarps ? p[32 + lane] : 0.0);
}
__device__ __forceinline__ int st_bmin(StShared &sh, int &rf, int v) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = __reduce_min_sync(0xFFFFFFFFu, v);
  int *p = sh.r1i[rf];
  rf ^= 1;
  if (lane == 0) p[warp] = v;
  __syncthreads();
  return __reduce_min_sync(0xFFFFFFFFu, lane < kStWarps ? p[lane] : 0x7FFFFFFF);
}
// the minima of a and of b
__device__ __forceinline__ void st_bmin2(StShared &sh, int &rf, int a, int b, int &ma, int &mb) {
  static_assert(kStWarps <= 16, "two partials per warp in one half");
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  a = __reduce_min_sync(0xFFFFFFFFu, a);
  b = __reduce_min_sync(0xFFFFFFFFu, b);
  int *p = sh.r1i[rf];
  rf ^= 1;
  if (lane == 0) {
    p[warp] = a;
    p[16 + warp] = b;
  }
  __syncthreads();
  ma = __reduce_min_sync(0xFFFFFFFFu, lane < kStWarps ? p[lane] : 0x7FFFFFFF);
  mb = __reduce_min_sync(0xFFFFFFFFu, lane < kStWarps ? p[16 + lane] : 0x7FFFFFFF);
}
// the maximum (fmaxf: a NaN drops out) and, in *any, whether some thread's
// flag is set
__device__ __forceinline__ float st_bmaxf(StShared &sh, int &rf, float v, bool flag, bool *any) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xFFFFFFFFu, v, o));
  const bool wf = __any_sync(0xFFFFFFFFu, flag);
  double *p = sh.r1d[rf];
  rf ^= 1;
  if (lane == 0) {
    p[warp] = (double)v;
    p[32 + warp] = wf ? 1.0 : 0.0;
  }
  __syncthreads();
  float t = lane < kStWarps ? (float)p[lane] : -INFINITY;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) t = fmaxf(t, __shfl_xor_sync(0xFFFFFFFFu, t, o));
  if (any) *any = __any_sync(0xFFFFFFFFu, lane < kStWarps && p[32 + lane] != 0.0);
  return t;
}
// exclusive and inclusive prefix sums over threads in thread order, and the total
__device__ __forceinline__ void st_bscan(StShared &sh, int &rf, double v, double &ex, double &inc, double &tot) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  double x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const double y = __shfl_up_sync(0xFFFFFFFFu, x, o);
    if (lane >= o) x += y;
  }
  double xprev = __shfl_up_sync(0xFFFFFFFFu, x, 1);
  if (lane == 0) xprev = 0.0;
  double *p = sh.r1d[rf];
  rf ^= 1;
  if (lane == 31) p[warp] = x;
  __syncthreads();
  double w = lane < kStWarps ? p[lane] : 0.0;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const double y = __shfl_up_sync(0xFFFFFFFFu, w, o);
    if (lane >= o) w += y;
  }
  const double prev = __shfl_sync(0xFFFFFFFFu, w, (warp + 31) & 31);
  tot = __shfl_sync(0xFFFFFFFFu, w, kStWarps - 1);
  ex = (warp > 0 ? prev : 0.0) + xprev;
  inc = (warp > 0 ? prev : 0.0) + x;
}
__device__ __forceinline__ void st_bscan_i(StShared &sh, int &rf, int v, int &ex, int &tot) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xFFFFFFFFu, x, o);
    if (lane >= o) x += y;
  }
  int *p = sh.r1i[rf];
  rf ^= 1;
  if (lane == 31) p[warp] = x;
  __syncthreads();
  int w = lane < kStWarps ? p[lane] : 0;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xFFFFFFFFu, w, o);
    if (lane >= o) w += y;
  }
  const int prev = __shfl_sync(0xFFFFFFFFu, w, (warp + 31) & 31);
  tot = __shfl_sync(0xFFFFFFFFu, w, kStWarps - 1);
  ex = (warp > 0 ? prev : 0) + x - v;
}

// --------------------------------------------------------- block selection
// The k-th largest of n keys (1 <= k <= n), by rounds of 8-bit digits from
// the top; *n_above = the keys whose leading digits are above its.  With
// rounds == 4 the key itself; with fewer, its leading 8*rounds bits followed
// by zeros (a lower bound on it).  Each round has its own histogram (cleared
// up front), and every warp scans it for itself, so a round costs one
// barrier.  All threads.
__device__ uint32_t st_select_kth(StShared &sh, const uint32_t *keys, int n, int k, int *n_above,
                                  int rounds = 4) {
  const int tid = threadIdx.x, lane = tid & 31;
  __syncthreads();  // no warp still scans the histograms of an earlier call
  for (int b = tid; b < rounds * 256; b += kStThreads) (&sh.sel[0][0])[b] = 0u;
  __syncthreads();
  uint32_t prefix = 0;
  int rem = k, above = 0;
  for (int d = 0; d < rounds; ++d) {
    const int shift = 24 - 8 * d;
    uint32_t *h = sh.sel[d];
    for (int i0 = 0; i0 < n; i0 += kStThreads) {
      const int i = i0 + tid;
      const uint32_t key = i < n ? keys[i] : 0u;
      const bool in = i < n && (d == 0 || (key >> (shift + 8)) == prefix);
      const uint32_t digit = (key >> shift) & 255u;
      // keys share leading digits heavily: the first active lane's digit
      // takes one atomic for every lane that holds it
      const unsigned act = __ballot_sync(0xFFFFFFFFu, in);
      if (act) {
        const int first = __ffs(act) - 1;
        const uint32_t lead = __shfl_sync(0xFFFFFFFFu, digit, first);
        const unsigned same = __ballot_sync(0xFFFFFFFFu, in && digit == lead);
        if (lane == first) {
          atomicAdd(&h[lead], (uint32_t)__popc(same));
        } else if (in && digit != lead) {
          atomicAdd(&h[digit], 1u);
        }
      }
    }
    __syncthreads();
    // every warp: the digit whose running count from the top reaches rem;
    // lane l holds digits 255 - 8l - q, q = 0..7
    const uint4 *h4 = reinterpret_cast<const uint4 *>(h);
    const uint4 lo = h4[(248 - 8 * lane) >> 2], hi = h4[((248 - 8 * lane) >> 2) + 1];
    const uint32_t c8[8] = {hi.w, hi.z, hi.y, hi.x, lo.w, lo.z, lo.y, lo.x};
    uint32_t s8 = 0;
#pragma unroll
    for (int q = 0; q < 8; ++q) s8 += c8[q];
    uint32_t incl = s8;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t y = __shfl_up_sync(0xFFFFFFFFu, incl, o);
      if (lane >= o) incl += y;
    }
    const uint32_t excl = incl - s8;
    const unsigned hit = __ballot_sync(0xFFFFFFFFu, incl >= (uint32_t)rem && excl < (uint32_t)rem);
    uint32_t dig = 0, before = 0;
    if (hit && lane == __ffs(hit) - 1) {
      uint32_t acc = excl;
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        if (acc + c8[q] >= (uint32_t)rem) {
          dig = 255u - (uint32_t)(8 * lane + q);
          before = acc;
          break;
        }
        acc += c8[q];
      }
    }
    // no hit only for k > n, which callers exclude
    const int src = hit ? __ffs(hit) - 1 : 0;
    dig = __shfl_sync(0xFFFFFFFFu, dig, src);
    before = __shfl_sync(0xFFFFFFFFu, before, src);
    rem -= (int)before;
    above += (int)before;
    prefix = (prefix << 8) | dig;
  }
  *n_above = above;
  return rounds == 4 ? prefix : prefix << (32 - 8 * rounds);
}

// ------------------------------------------------------------ bitonic sort
// Sort n <= kSortCap entries (key, idx) in shared memory into (key desc, index asc)
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

// Sort n <= kRankCap entries (key, idx) into (key desc, idx asc) order, or
// into index order when by_index (keys carried along), by counting for each
// entry the entries that precede it.  Stage 0 (idle) holds the composites.
// All threads.
__device__ void st_rank_sort(StShared &sh, uint32_t *key, int *idx, int n, bool by_index) {
  const int tid = threadIdx.x;
  unsigned long long *comp = reinterpret_cast<unsigned long long *>(st_scratch(sh, 0));
  // larger composite = earlier in the target order; all distinct (indices are)
  for (int i = tid; i < n; i += kStThreads) {
    const unsigned long long ni = (unsigned long long)(~(uint32_t)idx[i]);
    comp[i] = by_index ? ((ni << 32) | key[i]) : (((unsigned long long)key[i] << 32) | ni);
  }
  if (tid == 0) comp[n] = 0ull;  // pad for the paired reads
  __syncthreads();
  const ulonglong2 *c2 = reinterpret_cast<const ulonglong2 *>(comp);
  const int npair = (n + 1) >> 1;
  for (int i = tid; i < n; i += kStThreads) {
    const unsigned long long ci = comp[i];
    int rank = 0;
    for (int j = 0; j < npair; ++j) {
      const ulonglong2 q = c2[j];
      rank += (q.x > ci ? 1 : 0) + (q.y > ci ? 1 : 0);
    }
    if (by_index) {
      key[rank] = (uint32_t)ci;
      idx[rank] = (int)~(uint32_t)(ci >> 32);
    } else {
      key[rank] = (uint32_t)(ci >> 32);
      idx[rank] = (int)~(uint32_t)ci;
    }
  }
  __syncthreads();
}

// jw-th largest of the warp's running maxima, as a key (0 for -inf).
__device__ __forceinline__ uint32_t warp_kth_key(float rmax, int jw) {
  const int lane = threadIdx.x & 31;
  uint32_t key = rmax > -INFINITY ? fkey(rmax) : 0u;
#pragma unroll
  for (int size = 2; size <= 32; size <<= 1) {  // bitonic sort, ascending
#pragma unroll
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      const uint32_t o = __shfl_xor_sync(0xFFFFFFFFu, key, stride);
      const bool asc = (lane & size) == 0 || size == 32;
      const bool low = (lane & stride) == 0;
      key = (low == asc) ? min(key, o) : max(key, o);
    }
  }
  return __shfl_sync(0xFFFFFFFFu, key, 32 - jw);
}

// Lower bound on the k-th largest value of the row, as a key: each warp takes
// the jw-th largest (jw = ceil(k/16)) of its lanes' running maxima; the
// minimum over the 16 warps has at least 16*jw >= k maxima, each a distinct
// element, at or above it.  0 when some warp holds fewer than jw finite
// maxima.  All threads; one barrier.
__device__ __forceinline__ uint32_t st_topk_bound(StShared &sh, float rmax, int jw) {
  const uint32_t bw = warp_kth_key(rmax, jw);
  if ((threadIdx.x & 31) == 0) sh.wbound[threadIdx.x >> 5] = bw;
  __syncthreads();
  uint32_t bmin = 0xFFFFFFFFu;
#pragma unroll
  for (int q = 0; q < kStWarps; ++q) bmin = min(bmin, sh.wbound[q]);
  return bmin;
}

// The same bound without a barrier: each warp publishes its own (it only
// grows, running maxima only grow) and takes the minimum of what the others
// last published, which is still a valid bound.  Per warp.
__device__ __forceinline__ uint32_t st_topk_bound_nb(StShared &sh, float rmax, int jw) {
  const int lane = threadIdx.x & 31;
  const uint32_t bw = warp_kth_key(rmax, jw);
  volatile uint32_t *wb = sh.wbound;
  if (lane == 0) wb[threadIdx.x >> 5] = bw;
  __syncwarp();
  return __reduce_min_sync(0xFFFFFFFFu, lane < kStWarps ? wb[lane] : 0xFFFFFFFFu);
}

// The top-k set of a candidate buffer of n <= kRankCap unordered entries
// (sh.w.c) that holds every member of the row's top-k set, ranked by value
// descending then index ascending (the stable sort of
// miniserve/sampler.py:37-44).  Keys below thr cannot rank in that set.  The
// best m = min(k, entries) land in sh.w.c.key/idx[0..m) in rank order;
// returns m.  The entries at or above thr gather at positions taken from
// sh.nhigh (zero on entry), then each counts the entries before it.  The
// idle transfer stages hold scratch.  All threads.
__device__ int st_topk_rank(StShared &sh, int n, int k, uint32_t thr) {
  const int tid = threadIdx.x;
  unsigned long long *comp = reinterpret_cast<unsigned long long *>(st_scratch(sh, 0));
  // (key, ~index) composites: larger = earlier in rank order, all distinct
  auto compose = [&](int i) -> unsigned long long {
    return ((unsigned long long)sh.w.c.key[i] << 32) | (unsigned long long)(~(uint32_t)sh.w.c.idx[i]);
  };
  const int i1 = tid + kStThreads;
  const int f0 = (tid < n && sh.w.c.key[tid] >= thr) ? 1 : 0;
  const int f1 = (i1 < n && sh.w.c.key[i1] >= thr) ? 1 : 0;
  if (f0 + f1) {
    const int pos = atomicAdd(&sh.nhigh, f0 + f1);
    if (f0) comp[pos] = compose(tid);
    if (f1) comp[pos + f0] = compose(i1);
  }
  __syncthreads();
  const int n2 = sh.nhigh;
  const int m = min(n2, k);
  const ulonglong2 *c2 = reinterpret_cast<const ulonglong2 *>(comp);
  const int npair = n2 >> 1;
  for (int i = tid; i < n2; i += kStThreads) {
    const unsigned long long ci = comp[i];
    int rank = 0;
    for (int j = 0; j < npair; ++j) {
      const ulonglong2 q = c2[j];
      rank += (q.x > ci ? 1 : 0) + (q.y > ci ? 1 : 0);
    }
    if (n2 & 1) rank += comp[n2 - 1] > ci ? 1 : 0;
    if (rank < m) {
      sh.w.c.key[rank] = (uint32_t)(ci >> 32);
      sh.w.c.idx[rank] = (int)~(uint32_t)ci;
    }
  }
  __syncthreads();
  return m;
}

// Exact top-k finish: st_topk_rank, float64 weights exp(l/T - max/T)
// (miniserve/sampler.py:35,45; the maximum is the first ranked entry), top-p
// in rank order (sampler.py:49-58), and the index-order draw
// (sampler.py:60-68): each kept entry sums the kept weights at or before its
// index, and the smallest index whose sum reaches U * (kept total) is the
// token; U == 0 stops at index 0, a target past every sum gives V-1.  All
// threads; n >= 1.
__device__ void st_finish_small(StShared &sh, int &rf, const SampleArgs &a, int row, int n, int k, uint32_t thr,
                                double T, double P, double U) {
  const int tid = threadIdx.x;
  const int m = st_topk_rank(sh, n, k, thr);
  // thread r holds rank r (m <= kStTopK <= kStThreads)
  const double xmax = (double)key_to_float(sh.w.c.key[0]) / T;
  const int my = tid < m ? sh.w.c.idx[tid] : 0x7FFFFFFF;
  const double w = tid < m ? exp((double)key_to_float(sh.w.c.key[tid]) / T - xmax) : 0.0;
  double *dw = reinterpret_cast<double *>(st_scratch(sh, 1));  // weight by rank
  double *dinc = dw + kStTopK;                                 // running weight by rank
  if (tid < m) dw[tid] = w;
  double wex, winc, total;
  st_bscan(sh, rf, w, wex, winc, total);  // its barrier publishes dw
  if (tid < m) dinc[tid] = winc;
  int nkeep = m;
  if (P < 1.0) {  // smallest rank prefix reaching top_p, crossing entry kept
    const int first = st_bmin(sh, rf, (tid < m && winc >= P * total) ? tid : 0x7FFFFFFF);  // publishes dinc
    if (first != 0x7FFFFFFF) nkeep = first + 1;
  } else {
    __syncthreads();  // publishes dinc
  }
  const double tot_keep = dinc[nkeep - 1];
  const bool kept = tid < nkeep;
  double cum = 0.0;
  if (kept) {
    for (int j = 0; j < nkeep; ++j) cum += sh.w.c.idx[j] <= my ? dw[j] : 0.0;
  }
  const int special = U > 0.0 ? a.V - 1 : 0;  // the token when no kept entry reaches the target
  int tok, holder;
  st_bmin2(sh, rf, (kept && U > 0.0 && cum >= U * tot_keep) ? my : 0x7FFFFFFF,
           (kept && my == special) ? tid : 0x7FFFFFFF, tok, holder);
  if (tok != 0x7FFFFFFF) {
    if (kept && my == tok) write_row(a, row, tok, (float)(w / tot_keep), 0);
  } else if (holder != 0x7FFFFFFF) {
    if (tid == holder) write_row(a, row, special, (float)(w / tot_keep), 0);
  } else if (tid == 0) {
    write_row(a, row, special, 0.0f, 0);
  }
}

// Two fp32 values in one 64-bit register.  sm_100 executes add/sub/fma
// .f32x2 as one instruction for both; each half is rounded exactly as the
// scalar instruction would round it, so packed and scalar code give the same
// bits.
typedef unsigned long long f2_t;
__device__ __forceinline__ f2_t f2_pack(float lo, float hi) {
  f2_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void f2_unpack(f2_t v, float &lo, float &hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ f2_t f2_add(f2_t a, f2_t b) {
  f2_t r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ f2_t f2_sub(f2_t a, f2_t b) {
  f2_t r;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ f2_t f2_fma(f2_t a, f2_t b, f2_t c) {
  f2_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
__device__ __forceinline__ f2_t f2_add_rm(f2_t a, f2_t b) {  // rounded toward -inf
  f2_t r;
  asm("add.rm.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ float st_ex2(float z) {
  float r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(z));
  return r;
}

// fp32 weight 2^((v - M) * log2(e) / T) from two FMAs and one ex2.approx:
// c = c_hi + c_lo and M*c = mc_hi + mc_lo carry the constants to ~2^-48, so
// the only roundings are the final sum (|z| * 2^-24) and ex2 (~2^-22).
// c_hi is c rounded toward zero and c_lo > 0, so v = -inf gives z = -inf and
// weight 0 with no test.  set_t once per row, set_m per finite reference
// maximum M.
struct StW {
  float c_hi, c_lo, mc_hi, mc_lo;
  __device__ __forceinline__ void set_t(double T) {
    const double c = 1.4426950408889634 / T;  // log2(e) / T
    c_hi = __double2float_rz(c);
    c_lo = (float)(c - (double)c_hi);
    if (!(c_lo > 0.0f)) c_lo = 1.17549435e-38f;  // c exact in fp32: a negligible positive tail
  }
  __device__ __forceinline__ void set_m(float M) {
    mc_hi = M * c_hi;
    const float e = fmaf(M, c_hi, -mc_hi);  // the product's rounding error, exactly
    mc_lo = fmaf(M, c_lo, e);
  }
  __device__ __forceinline__ float operator()(float v) const {
    return st_ex2(fmaf(v, c_hi, -mc_hi) + fmaf(v, c_lo, -mc_lo));
  }
};

// The same weight for two values at once (packed arithmetic, same bits).
struct StW2 {
  f2_t ch, cl, nmh, nml;
  __device__ __forceinline__ explicit StW2(const StW &w)
      : ch(f2_pack(w.c_hi, w.c_hi)), cl(f2_pack(w.c_lo, w.c_lo)), nmh(f2_pack(-w.mc_hi, -w.mc_hi)),
        nml(f2_pack(-w.mc_lo, -w.mc_lo)) {}
  __device__ __forceinline__ f2_t operator()(f2_t v) const {
    float z0, z1;
    f2_unpack(f2_add(f2_fma(v, ch, nmh), f2_fma(v, cl, nml)), z0, z1);
    return f2_pack(st_ex2(z0), st_ex2(z1));
  }
};

// Element gi of the row from global memory (L2), masked tokens as -inf.
template <int DT>
__device__ __forceinline__ float st_load1(const StRow &r, int gi) {
  float v = DT == MS_DTYPE_F32
                ? __ldg(reinterpret_cast<const float *>(r.g) + gi)
                : __uint_as_float((uint32_t)__ldg(reinterpret_cast<const unsigned short *>(r.g) + gi) << 16);
  if (r.mask && !((__ldg(r.mask + (gi >> 5)) >> (gi & 31)) & 1u)) v = -INFINITY;
  return v;
}

// Index-order inverse CDF (miniserve/sampler.py:60-68) over a row whose kept
// mass per unit is kept[0..nu) (sum `total`): the crossing unit from a block
// scan, then that unit's 256 elements re-read with keptw(v, gi), the same
// float64 weights the unit sums were made of.  Writes the row.  All threads.
template <int DT, class KW>
__device__ void st_draw_units(StShared &sh, int &rf, const SampleArgs &a, const StRow &r, int row, int nu,
                              const double *kept, double total, double U, KW keptw) {
  const int tid = threadIdx.x;
  if (!(U > 0.0)) {  // r == 0 stops at index 0 (sampler.py:66)
    if (tid == 0) write_row(a, row, 0, (float)(keptw(st_load1<DT>(r, 0), 0) / total), 0);
    return;
  }
  const double target = U * total;
  const int u0 = 2 * tid;
  const double k0 = u0 < nu ? kept[u0] : 0.0, k1 = u0 + 1 < nu ? kept[u0 + 1] : 0.0;
  double ex, inc, tt;
  st_bscan(sh, rf, k0 + k1, ex, inc, tt);
  int cand = 0x7FFFFFFF;
  if (k0 + k1 > 0.0 && inc >= target) cand = (k0 > 0.0 && ex + k0 >= target) ? u0 : u0 + 1;
  const int us = st_bmin(sh, rf, cand);
  if (us == 0x7FFFFFFF) {  // ran past the end (sampler.py:68)
    if (tid == 0) write_row(a, row, a.V - 1, (float)(keptw(st_load1<DT>(r, a.V - 1), a.V - 1) / total), 0);
    return;
  }
  if (tid == (us >> 1)) sh.bcast_d[1] = (us == u0) ? ex : ex + k0;
  __syncthreads();
  const double before = sh.bcast_d[1];
  const int gi = us * kUnit + tid;
  const double w = (tid < kUnit && gi < a.V) ? keptw(st_load1<DT>(r, gi), gi) : 0.0;
  double wex, winc, wtot;
  st_bscan(sh, rf, w, wex, winc, wtot);
  int who = st_bmin(sh, rf, (w > 0.0 && before + winc >= target) ? tid : 0x7FFFFFFF);
  if (who == 0x7FFFFFFF) {  // rounding left the target past the unit: its last kept element
    who = -st_bmin(sh, rf, w > 0.0 ? -tid : 1);
  }
  if (who < 0) {  // no kept element in the unit (cannot happen for consistent sums)
    if (tid == 0) a.status[row] = kRowPending;
    return;
  }
  if (tid == who) write_row(a, row, gi, (float)(w / total), 0);
}

enum StMode : int { kStArgmax = 0, kStTopKMode = 1, kStFull = 2, kStNucleus = 3 };

// Candidate record of `row` in vocab-sharded mode: [count, status, kmax keys,
// kmax global ids, total (float64, two words)].  The total, for rows without
// top-k, is the slice's sum of exp((v - m) / T) over its finite logits, m the
// slice maximum (the first key).
__device__ __forceinline__ uint32_t *st_record(const SampleArgs &a, int row) {
  return a.records + (size_t)row * (size_t)(4 + 2 * a.kmax);
}
__device__ __forceinline__ void st_record_total(const SampleArgs &a, uint32_t *rec, double total) {
  const unsigned long long b = (unsigned long long)__double_as_longlong(total);
  rec[2 + 2 * a.kmax] = (uint32_t)b;
  rec[3 + 2 * a.kmax] = (uint32_t)(b >> 32);
}
__device__ __forceinline__ void st_record_empty(const SampleArgs &a, int row, uint32_t status) {
  uint32_t *rec = st_record(a, row);
  rec[0] = 0u;
  rec[1] = status;
  st_record_total(a, rec, 0.0);
}

// Estimated cost class of a row, most expensive first: 0 top-p rows (two
// passes when the nucleus is wide), 1 top-k rows with k >= 128 (many
// candidate inserts), 2 the other top-k rows and full-softmax rows, 3 argmax
// rows.  The first CTAs of a launch land one per SM, so the top-p rows (fewer
// than the SMs in a typical batch) also avoid sharing an SM with each other.
__device__ __forceinline__ int st_row_class(const SampleArgs &a, int r) {
  const double T = a.temperature[r];
  const int k = a.top_k[r];
  if (!(T > 0.0) || isinf(T) || k == 1) return 3;
  if (k >= 2 && k < a.V) return k >= 128 ? 1 : 2;
  return a.top_p[r] < 1.0 ? 0 : 2;
}

// The row this CTA takes, from the rows ordered by (cost class, index), so
// the CTAs launched first take the longest rows and the batch ends with short
// ones; -1 for none.  Every CTA computes the same order from the per-row
// parameters.  One CTA per row: CTA i takes position i.  Pair mode (clusters
// of two CTAs, 2B CTAs launched): cluster i takes work item i -- the i-th
// top-p row, shared by both CTAs (*joint set), or after those, the next two
// positions, one per CTA; the clusters past the work take none.  A batch with
// more than a.pairs top-p rows shares none (sharing shortens a top-p row but
// costs CTA time, which pays only while the top-p rows fit one wave).
__device__ int st_pick_row(StShared &sh, const SampleArgs &a, int B, bool *joint) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  *joint = false;
  if (!a.pairs && (int)blockIdx.x >= B) return -1;
  const unsigned lt = (1u << lane) - 1u;
  // One round of up to kStThreads rows: the rows of each class in this warp
  // and in earlier lanes (ballots), the per-class prefix over the warps and
  // the round's class totals (four threads).  `pre` and `cls` describe this
  // thread's row r0 + tid.
  auto round = [&](int r0, int &cls, int &pre) {
    const int r = r0 + tid;
    cls = r < B ? st_row_class(a, r) : -1;
    pre = 0;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const unsigned m = __ballot_sync(0xFFFFFFFFu, cls == c);
      if (lane == 0) sh.pick[warp][c] = __popc(m);
      if (cls == c) pre = __popc(m & lt);
    }
    __syncthreads();
    if (tid < 4) {  // exclusive prefix over the warps of class tid, and the round's total
      int run = 0;
#pragma unroll
      for (int w = 0; w < kStWarps; ++w) {
        const int v = sh.pick[w][tid];
        sh.pick[w][tid] = run;
        run += v;
      }
      sh.bcast_i[4 + tid] = run;
    }
    __syncthreads();
  };
  // class totals (the first round already holds them when B <= kStThreads)
  int cls = -1, pre = 0;
  int t0 = 0, t1 = 0, t2 = 0, t3 = 0;
  for (int r0 = 0; r0 < B; r0 += kStThreads) {
    if (r0 > 0) __syncthreads();  // the previous round's totals are read
    round(r0, cls, pre);
    t0 += sh.bcast_i[4];
    t1 += sh.bcast_i[5];
    t2 += sh.bcast_i[6];
    t3 += sh.bcast_i[7];
  }
  int want = blockIdx.x;
  if (a.pairs) {
    const int item = blockIdx.x >> 1, np = t0 <= a.pairs ? t0 : 0;
    if (item < np) {
      want = item;
      *joint = true;
    } else {
      want = np + 2 * (item - np) + (int)st_crank();
      if (want >= B) return -1;
    }
  }
  if (t0 == B || t1 == B || t2 == B || t3 == B) return want;
  // positions in (class, index) order: the class's first position, the rows
  // of that class in earlier rounds, in earlier warps of this round and in
  // earlier lanes
  int b0 = 0, b1 = t0, b2 = t0 + t1, b3 = t0 + t1 + t2;
  int found = -1;
  for (int r0 = 0; r0 < B; r0 += kStThreads) {
    if (B > kStThreads) {  // one round holds every row otherwise: its ballots are still in place
      __syncthreads();
      round(r0, cls, pre);
    }
    if (cls >= 0) {
      const int bc = cls == 0 ? b0 : cls == 1 ? b1 : cls == 2 ? b2 : b3;
      if (bc + sh.pick[warp][cls] + pre == want) found = r0 + tid;
    }
    b0 += sh.bcast_i[4];
    b1 += sh.bcast_i[5];
    b2 += sh.bcast_i[6];
    b3 += sh.bcast_i[7];
  }
  __syncthreads();
  if (found >= 0) sh.bcast_i[0] = found;
  __syncthreads();
  return sh.bcast_i[0];
}

// top-k adaptive pass: chunks whose warp bounds refresh tau (0-2, then every
// 4th) and chunks that select the buffer's k-th largest (3, 11)
__device__ __forceinline__ bool st_refresh_chunk(int c) { return c < 3 || (c & 3) == 0; }
__device__ __forceinline__ bool st_select_chunk(int c) { return c == 3 || c == 11; }

// W(v) for two values at once: 2^(v * c - a) (packed fma, two ex2)
__device__ __forceinline__ f2_t st_w2(f2_t v, f2_t C, f2_t NA) {
  float z0, z1;
  f2_unpack(f2_fma(v, C, NA), z0, z1);
  return f2_pack(st_ex2(z0), st_ex2(z1));
}

// One row of the streaming kernel (the CTA's row from st_pick_row).  XCH
// (the fused peer exchange): prow is set to the row, whose record is
// published after the body returns (every return past that point is
// block-uniform).
template <int DT, bool XCH>
__device__ __forceinline__ void st_row_body(const SampleArgs &a, StShared &sh, int &prow) {
  // every CTA of this grid has started: a programmatic dependent launch (the
  // pending-row pass) may begin launching
  asm volatile("griddepcontrol.launch_dependents;");
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  // the stage barriers first: the row ordering's barriers publish them
  if (tid < st_nstages<DT>()) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(st_smem(&sh.full[tid])) : "memory");
  }
  if (tid == 0) {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  bool joint;
  const int row = st_pick_row(sh, a, a.pairs ? a.rows : (int)gridDim.x, &joint);
  if (row < 0) return;
  if constexpr (XCH) prow = row;  // shard mode: no pairs, every path writes the record
  const int crank = joint ? (int)st_crank() : 0;
  const int V = a.V;
  StRow r;
  r.g = reinterpret_cast<const char *>(a.logits) + (int64_t)row * a.ld * st_esz<DT>();
  r.mask = a.mask ? a.mask + (int64_t)row * a.mask_ld : nullptr;
  r.V = V;
  r.tma = (reinterpret_cast<uintptr_t>(r.g) & 15u) == 0;
  r.mtma = r.mask && r.tma && (reinterpret_cast<uintptr_t>(r.mask) & 15u) == 0;
  r.nchunks = (V + kChunk - 1) / kChunk;
  r.nfull = r.tma ? V / kChunk : 0;
  const uint64_t pol_stream = policy_evict_first();
  const uint64_t pol_keep = policy_evict_last();
  // The first copies of the row's first pass go out before its parameters
  // are read: a shared row (a top-p row) its half, kept in L2 for the second
  // pass; any other row from chunk 0.  pre_c0 / pre_n: the chunks under way,
  // which every exit before the pass waits for (pre_drain).
  int pre_c0 = 0, pre_n = 0;
  uint64_t pre_pol = pol_stream;
  {
    int c1 = r.nchunks;
    if (joint) {
      pre_pol = pol_keep;
      if (r.nchunks >= 2) {
        pre_c0 = crank == 0 ? 0 : r.nchunks / 2;
        c1 = crank == 0 ? r.nchunks / 2 : r.nchunks;
      } else if (crank == 1) {
        c1 = 0;  // too short to share: the first CTA takes it alone
      }
    }
    // (fp32 rows: a bf16 row's stage layout depends on its mode)
    pre_n = DT == MS_DTYPE_F32 ? max(0, min(c1 - pre_c0, st_nstages<DT>())) : 0;
    if (tid == 0)
      for (int c = pre_c0; c < pre_c0 + pre_n; ++c) st_issue<DT>(sh, r, c, c - pre_c0, pre_pol);
  }
  uint32_t ph = 0;
  auto pre_drain = [&]() {  // all threads, before leaving with the first copies under way
    if (pre_n) st_drain<DT>(sh, pre_c0, pre_c0, pre_c0 + pre_n, ph);
    pre_n = 0;
  };
  const double T = a.temperature[row];
  int k = a.top_k[row];
  const double P = a.top_p[row];
  const double U = a.uniforms[row];
  const bool shard = a.records != nullptr;
  if (!(T >= 0.0) || isinf(T)) {  // negative, NaN or infinite temperature
    pre_drain();
    if (tid == 0 && crank == 0) {
      if (shard) st_record_empty(a, row, MS_ROW_BAD_TEMPERATURE);
      else write_row(a, row, -1, 0.0f, MS_ROW_BAD_TEMPERATURE);
    }
    return;
  }
  // a row this kernel does not finish: the generic kernel takes it, or in
  // sharded mode its record says why (nonfinite: a NaN / +inf logit)
  auto leave = [&](bool nonfinite) {
    pre_drain();
    if (tid == 0 && crank == 0) {
      if (shard) st_record_empty(a, row, nonfinite ? MS_ROW_NONFINITE : MS_ROW_UNSUPPORTED);
      else a.status[row] = kRowPending;
    }
  };
  int mode;
  bool shard_sum = false;  // shard mode, no top-k: the record carries the slice's total
  if (T == 0.0 || k == 1) {
    mode = kStArgmax;
  } else if (shard) {
    if (k >= 2 && (int64_t)k < a.Vg) {
      // the slice's top-k stands for the row's when it fits the record
      if (!(k <= a.kmax && k < V && k <= kStTopK)) {
        leave(false);
        return;
      }
    } else if (a.kmax >= 2 && a.kmax < V && a.kmax <= kStTopK && T >= kMinTemperature) {
      // no top-k: the slice's top kmax and its softmax total, which settle a
      // top-p row in the merge when the nucleus lies among the candidates
      k = a.kmax;
      shard_sum = true;
    } else {
      leave(false);
      return;
    }
    mode = kStTopKMode;
  } else if (k >= 2 && k < V) {
    mode = kStTopKMode;
  } else {
    mode = P < 1.0 ? kStNucleus : kStFull;
  }
  // top_k above what the streaming buffer resolves, or a temperature too small
  // for fp32 weights: the generic kernel finishes the row
  if (!shard && ((mode == kStTopKMode && k > kStTopK) || (mode != kStArgmax && !(T >= kMinTemperature)))) {
    leave(false);
    return;
  }
  if (tid < kStWarps) sh.wbound[tid] = 0u;
  if (tid == 0) {
    sh.ncand = 0;
    sh.nhigh = 0;  // top-k rows: st_topk_rank's counter
  }
  __syncthreads();
  bool ok = true;
  int rf = 0;  // scratch half of the next one-barrier reduction

  // ================================================================ argmax
  if (mode == kStArgmax) {
    // a thread sees its elements in increasing index order: a strictly
    // larger chunk maximum moves the thread's best to its first occurrence
    float tm = -INFINITY, tnan = -INFINITY;
    int ti = 0x7FFFFFFF;
    const bool pre = pre_n > 0;
    pre_n = 0;
    ok = st_stream<DT, false>(
        sh, r, 0, r.nchunks, pol_stream, ph,
        [&](const float *x, int g0, int, int) {
          const float cm = st_max8n(x);
          tnan = st_maxn(tnan, cm);
          if (cm > tm) {  // rare after the first chunks
            int e = 7;
#pragma unroll
            for (int q = 6; q >= 0; --q) e = x[q] == cm ? q : e;
            tm = cm;
            ti = st_gidx(g0, e);
          }
        },
        StNoAfter(), pre);
    const bool bad = st_bad(tnan);
    uint32_t bk = tm > -INFINITY ? fkey(tm) : 0u;
    int bi = tm > -INFINITY ? ti : 0x7FFFFFFF;
    warp_argmax(bk, bi);
    if (lane == 0) {
      sh.redu[tid >> 5] = bk;
      sh.redi[tid >> 5] = bi;
    }
    const int any_bad = __syncthreads_or(bad || !ok);
    if (tid < 32) {
      uint32_t k2 = tid < kStWarps ? sh.redu[tid] : 0u;
      int i2 = tid < kStWarps ? sh.redi[tid] : 0x7FFFFFFF;
      warp_argmax(k2, i2);
      if (tid == 0) {
        if (shard) {  // the slice's first maximum (none when all -inf)
          uint32_t *rec = st_record(a, row);
          rec[0] = (!any_bad && k2 != 0u) ? 1u : 0u;
          rec[1] = any_bad ? (uint32_t)MS_ROW_NONFINITE : 0u;
          rec[2] = k2;
          rec[2 + a.kmax] = (uint32_t)(a.v0 + i2);
        } else if (any_bad) {
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
    // Candidates are values >= tau (> when strict); ties at tau stay
    // candidates.  A lane with no value at or above tau skips the insert.
    //
    // First pass: tau is the m-th largest value of chunk 0 (to 16 bits).
    // Chunk 0 holds lam = k * n0 / V of the row's top-k set on average; with
    // m = lam + 3 sqrt(lam) + 2 the row's k-th largest value lies below tau
    // only when chunk 0 holds m members of that set (a Poisson tail near 1e-3
    // for a row in random order; such a row takes a second pass).  Every
    // value >= tau is a candidate, so at least k candidates prove that tau is
    // low enough; with fewer, a
    // second pass starts over with tau rising to lower bounds of the k-th
    // largest from the lanes' running maxima (st_topk_bound) and the buffer's
    // k-th largest (chunks 3 and 11).  A buffer that could overflow is cut to
    // its entries at or above its k-th largest either way.
    float tau = -INFINITY;
    float tf = -FLT_MAX;  // candidates: x >= tf (the next float above tau when strict; -inf never)
    auto set_tau = [&](float t, bool strict) {
      tau = t;
      tf = strict ? key_to_float(fkey(t) + 1u) : fmaxf(t, -FLT_MAX);
    };
    float rmax = -INFINITY;  // NaN once a NaN has been seen
    const int jw = (k + kStWarps - 1) / kStWarps;  // <= 16
    bool over = false;
    bool exact_tau = false;  // tau is the k-th largest value seen (after a compaction)
    bool compacted = false;
    int ub = 0;  // bound on the buffer's size (its size after a sync point), the same in every thread
    // shard_sum: this lane's running maximum and sum of weights relative to it
    float sm = -INFINITY, ss = 0.0f;
    StW Ws;
    const double cls = 1.4426950408889634 / T;  // log2(e) / T
    if (shard_sum) Ws.set_t(T);
    const int n0 = min(kChunk, V);
    int msamp = k;
    if (r.nchunks > 1) {
      const float lam = (float)k * (float)n0 / (float)V;
      msamp = (int)ceilf(lam + 3.0f * sqrtf(lam) + 2.0f);
    }
    msamp = min(msamp, n0);
    for (int attempt = 0;; ++attempt) {
      const bool sampled = attempt == 0;
      if (!sampled) {  // start over
        tau = -INFINITY;
        tf = -FLT_MAX;
        rmax = -INFINITY;
        over = exact_tau = compacted = false;
        ub = 0;
        sm = -INFINITY;
        ss = 0.0f;
        __syncthreads();
        if (tid < kStWarps) sh.wbound[tid] = 0u;
        if (tid == 0) sh.ncand = 0;
        __syncthreads();
      }
      const bool pre = pre_n > 0;
      pre_n = 0;
      ok = st_stream<DT, true>(
          sh, r, 0, r.nchunks, pol_stream, ph,
          [&](const float *x, int g0, int, int c) -> int {
            const float cm = st_max8n(x);
            rmax = st_maxn(rmax, cm);
            if (shard_sum) {  // online softmax total (block-uniform branch)
              const float nm = fmaxf(sm, cm);
              if (nm > sm) {
                ss = sm > -INFINITY ? ss * (float)exp2(((double)sm - (double)nm) * cls) : 0.0f;
                sm = nm;
                Ws.set_m(sm);
              }
              if (sm > -INFINITY) {
                const StW2 W2(Ws);
                f2_t a2 = W2(f2_pack(x[0], x[1]));
#pragma unroll
                for (int j = 1; j < 4; ++j) a2 = f2_add(a2, W2(f2_pack(x[2 * j], x[2 * j + 1])));
                float a0, a1;
                f2_unpack(a2, a0, a1);
                ss += a0 + a1;
              }
            }
            if (sampled) {
              if (c == 0) {  // block-uniform: the threshold from chunk 0's values
                // (from the threads' maxima when the sample rank allows)
                const uint32_t tk = msamp <= kStThreads / 8 && r.nchunks > 1
                                        ? st_sample_kth1(sh, cm > -INFINITY ? fkey(cm) : kNegInfKey, msamp)
                                        : st_sample_kth(sh, x, msamp);
                if (tk > kNegInfKey) set_tau(key_to_float(tk), false);
              }
            } else if (!exact_tau && st_refresh_chunk(c)) {
              const uint32_t bmin = c == 0 ? st_topk_bound(sh, rmax, jw) : st_topk_bound_nb(sh, rmax, jw);
              if (bmin != 0u && key_to_float(bmin) > tau) set_tau(key_to_float(bmin), false);
            }
            // insert: only lanes holding a candidate, one shared atomic per
            // lane for all its entries.  The buffer holds at most
            // kCandCap - kChunk entries before each chunk, so it cannot overflow.
            int cnt = 0;
            if (cm >= tf) {  // NaN never
              unsigned m = 0;
#pragma unroll
              for (int e = 0; e < 8; ++e) m |= (x[e] >= tf ? 1u : 0u) << e;
              cnt = __popc(m);
              int pos = atomicAdd(&sh.ncand, cnt);  // positions only
              do {
                const int e = __ffs(m) - 1;
                m &= m - 1;
                sh.w.c.key[pos] = fkey(st_pick8(x, e));
                sh.w.c.idx[pos] = st_gidx(g0, e);
                ++pos;
              } while (m);
            }
            return cnt > 0;
          },
          [&](int c, int nins) -> bool {
            // every inserting lane added at most 8 entries
            ub += 8 * nins;
            const bool sel_pt = !sampled && !exact_tau && st_select_chunk(c);
            if (sel_pt || ub > kCandCap - kChunk) {
              // a sync point: every thread reads the exact size before any inserts again
              const int nb = sh.ncand;
              __syncthreads();
              ub = nb;
              // early on (chunks 3 and 11) the buffer's k-th largest, to 16
              // leading bits (two digit rounds; a lower bound within 2^-7 of
              // it), is a far tighter tau than the warp bound and cuts the
              // inserts of the rest of the row; entries below it stay in the
              // buffer, dead
              if (sel_pt && nb >= 2 * k && nb <= kCandCap - kChunk) {
                int above;
                set_tau(key_to_float(st_select_kth(sh, sh.w.c.key, nb, k, &above, 2)), false);
                exact_tau = true;
              }
              // shrink to the entries >= the buffer's k-th largest (ties kept)
              // when the next chunk could overflow the buffer
              if (nb > kCandCap - kChunk) {
                int above;
                const uint32_t kk = st_select_kth(sh, sh.w.c.key, nb, k, &above);
                uint32_t kv[kCandCap / kStThreads];
                int iv[kCandCap / kStThreads];
                int nk = 0;
                for (int i = tid; i < nb; i += kStThreads) {
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
                if (tid == 0) sh.ncand = ktot;
                __syncthreads();
                ub = ktot;
                set_tau(key_to_float(kk), true);  // >= k entries >= kk are held: a later equal value ranks below
                exact_tau = compacted = true;
                if (ktot > kCandCap - kChunk) over = true;  // heavy ties
              }
            }
            return over;
          },
          pre);
      const bool bad = st_bad(rmax);
      if (__syncthreads_or(bad || !ok || over)) {
        leave(__syncthreads_or(bad) != 0);
        return;
      }
      // fewer than k values at or above the sampled threshold: the row's
      // top-k set may reach below it
      if (sampled && !compacted && tau > -INFINITY && sh.ncand < k) continue;
      break;
    }
    // every finite logit is a candidate while tau is -inf, so an empty buffer
    // means every logit is -inf (sampler.py:46-47)
    if (sh.ncand == 0) {
      if (tid == 0) {
        if (shard) st_record_empty(a, row, 0u);  // no candidate in this slice
        else write_row(a, row, -1, 0.0f, MS_ROW_ALL_MASKED);
      }
      return;
    }
    // exact top-k of the buffer; fewer valid tokens than top_k keep all.  thr:
    // keys below it cannot rank in the top-k set (the buffer's k-th largest
    // when the buffer is large, else the warp bound)
    int n = sh.ncand;  // no insert since the barriers above
    uint32_t thr;
    if (n > kRankCap) {
      int above;
      const uint32_t kk = st_select_kth(sh, sh.w.c.key, n, k, &above);
      uint32_t kv[kCandCap / kStThreads];
      int iv[kCandCap / kStThreads];
      int nk = 0;
      for (int i = tid; i < n; i += kStThreads) {
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
      n = ktot;
      thr = kk;
    } else if (n >= 2 * k) {
      // the k-th largest to 16 leading bits: a lower bound that leaves only
      // its ties in those bits to the exact ranking
      int above;
      thr = st_select_kth(sh, sh.w.c.key, n, k, &above, 2);
    } else {
      thr = st_topk_bound(sh, rmax, jw);
    }
    if (n > kRankCap) {  // a tie block larger than the rank sort: generic kernel
      leave(false);
      return;
    }
    if (shard) {  // the slice's top-k, in rank order, with global ids
      // the slice's total relative to its maximum (rows without top-k)
      const float vmax = shard_sum ? st_bmaxf(sh, rf, rmax, false, nullptr) : 0.0f;
      const double tot = shard_sum ? st_bsum(sh, rf, sm > -INFINITY ? (double)ss * exp2(((double)sm - (double)vmax) * cls)
                                                                     : 0.0)
                                   : 0.0;
      const int m = st_topk_rank(sh, n, k, thr);
      uint32_t *rec = st_record(a, row);
      for (int i = tid; i < m; i += kStThreads) {
        rec[2 + i] = sh.w.c.key[i];
        rec[2 + a.kmax + i] = (uint32_t)(a.v0 + sh.w.c.idx[i]);
      }
      if (tid == 0) {
        rec[0] = (uint32_t)m;
        rec[1] = 0u;
        st_record_total(a, rec, tot);
      }
      return;
    }
    st_finish_small(sh, rf, a, row, n, k, thr, T, P, U);
    return;
  }

  // ========================================================== softmax rows
  // W(v) = 2^(v * cw - aw): cw = log2(e) / T rounded once, aw = G * cw with G
  // the maximum of the first chunk holding a finite value (the row maximum on
  // the rare second try, when a later value would give a weight beyond
  // 2^60).  A rounding of cw scales every exponent alike; one of aw scales
  // every weight alike and cancels in every ratio.
  const double cl = 1.4426950408889634 / T;  // log2(e) / T
  const float cw = (float)cl;
  float G = -INFINITY, aw = 0.0f, v_ovf = INFINITY;
  auto set_anchor = [&](float g) {
    G = g;
    aw = g * cw;
    v_ovf = (float)((double)g + 60.0 / cl);
  };
  auto W = [&](float v) -> float { return st_ex2(fmaf(v, cw, -aw)); };  // -inf weighs 0
  const bool topp = mode == kStNucleus;
  const int nu = r.nchunks * kStWarps;

  // Top-p histogram.  x-grid coordinate t = (Gh - v) * xs + kUpBins + 1:
  // kXBins bins per kSXRange units of x = logit / T, anchored at Gh (the
  // weights' anchor G when built in pass 1, else the row maximum).  t < 1:
  // more than kUpBins bins above Gh, kept exactly in the high list (index 0).
  // Index floor(t) in 1..kSBins: a grid bin; kSBins + 1: the tail (and masked
  // tokens).  hq[i] holds the fixed-point sum of kQScale * e^-((t - i) * dx)
  // over the elements of index i, so index i carries mass
  // e^-((i - 1 - kUpBins) * dx) * hq[i] / kQScale relative to Gh.  The
  // histogram only places the bracket: the classifying pass checks the
  // crossing exactly, and a bracket that misses it leaves the row pending.
  const float xs = (float)((double)kXBins / ((double)kSXRange * T));
  const float dx = kSXRange / (float)kXBins;
  const float t_off = (float)(kUpBins + 1);
  // round(kQScale * e^-(fr*dx)) + 2^23 as a float (quadratic, error (fr*dx)^3/6 < 1.6e-7)
  const float q0 = 8388608.0f + kQScale, q1 = -kQScale * dx, q2 = 0.5f * kQScale * dx * dx;
  uint32_t *hq = sh.w.n.x.hq;
  float Gh = -INFINITY;
  float v_high = INFINITY;  // no value at or below it lies above the grid (t < 1)
  float v_tail = INFINITY;  // every value at or below it lies in the tail (t >= kSBins + 1)
  auto set_hist_anchor = [&](float g) {
    Gh = g;
    v_high = __double2float_rd((double)g + (double)(kUpBins - 1) / (double)xs);
    v_tail = __double2float_rd((double)g - (double)kXBins / (double)xs);
  };
  auto hist_clear = [&]() {  // the caller's next barrier orders it
    for (int i = tid; i < kQSlots; i += kStThreads) hq[i] = 0u;
    if (tid == 0) sh.nhigh = 0;
  };
  // Histogram of this lane's 8 values (x[4..7] sit 128 after x[0..3]), cm
  // their maximum, in packed pairs.  Only grid bins 1..kSBins take mass:
  // values above the grid (t < 1) are kept exactly in the high list, and the
  // tail (t >= kSBins + 1, -inf and NaN included) is left out.
  auto hist8 = [&](const float *x, int g0, float cm) {
    if (__any_sync(0xFFFFFFFFu, cm > v_high)) {  // rare: some value may lie above the grid
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        if (fmaf(Gh - x[e], xs, t_off) < 1.0f) {
          const int pos = atomicAdd(&sh.nhigh, 1);
          if (pos < kHighCap) {
            sh.w.n.hkey[pos] = fkey(x[e]);
            sh.w.n.hidx[pos] = st_gidx(g0, e);
          }
        }
      }
    }
    if (!__any_sync(0xFFFFFFFFu, cm > v_tail)) return;  // the warp's values all lie in the tail
    const f2_t G2 = f2_pack(Gh, Gh), XS2 = f2_pack(xs, xs), OFF2 = f2_pack(t_off, t_off);
    const f2_t M2 = f2_pack(8388608.0f, 8388608.0f);
    const f2_t Q0 = f2_pack(q0, q0), Q1 = f2_pack(q1, q1), Q2 = f2_pack(q2, q2);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const f2_t TC = f2_fma(f2_sub(G2, f2_pack(x[2 * j], x[2 * j + 1])), XS2, OFF2);
      // 2^23 + floor(t): the add rounds toward -inf, so for 0 <= t < 2^23 the
      // float's low mantissa bits are floor(t).  Any t outside the grid bins
      // (t < 1, t >= kSBins + 1, huge, infinite or NaN) gives an index outside
      // 1..kSBins and adds nothing.
      const f2_t TB = f2_add_rm(TC, M2);
      const f2_t FR = f2_sub(TC, f2_sub(TB, M2));
      float tb0, tb1, qa, qb;
      f2_unpack(TB, tb0, tb1);
      f2_unpack(f2_fma(f2_fma(FR, Q2, Q1), FR, Q0), qa, qb);
      const uint32_t i0 = __float_as_uint(tb0) - 0x4B000000u, i1 = __float_as_uint(tb1) - 0x4B000000u;
      if (i0 - 1u < (uint32_t)kSBins) atomicAdd(&hq[i0], __float_as_uint(qa) - 0x4B000000u);
      if (i1 - 1u < (uint32_t)kSBins) atomicAdd(&hq[i1], __float_as_uint(qb) - 0x4B000000u);
    }
  };

  // A top-p row shared by a cluster: this CTA streams chunks [c0, c1) (the
  // first CTA the first half).  The two halves meet at cluster barriers: the
  // anchor and the wide prediction, the pass-1 totals, the second half's unit
  // maxima and histogram, the first CTA's decision, and the classifying
  // pass's entries; every decision between barriers is computed in both CTAs
  // from the same exchanged values, so both reach the same barriers or leave
  // at the same point, and only the first CTA writes the row's result.
  int c0 = 0, c1 = r.nchunks;
  if (joint) {
    if (r.nchunks < 2) {  // too short to share: the first CTA takes it alone
      if (crank == 1) return;
      joint = false;
    } else {
      c0 = crank == 0 ? 0 : r.nchunks / 2;
      c1 = crank == 0 ? r.nchunks / 2 : r.nchunks;
      st_cluster_sync();  // both CTAs have started before either stores into the other
    }
  }
  float vmax = -INFINITY;
  double zsum = 0.0;  // the row's total of W
  // top-p: a wide nucleus predicted at the first chunk(s), whose histogram
  // pass 1 builds too (when the chunk's unit maxima carry under top_p of its
  // mass, the row's largest values rarely reach top_p of the total).  A wide
  // row predicted narrow costs a histogram pass, a narrow row predicted wide
  // the classifying pass instead of the narrow capture; the threshold keeps
  // the first, dearer mistake rare.
  bool wide = false;
  for (int attempt = 0;; ++attempt) {
    if (attempt > 0) set_anchor(vmax);  // no weight above 1
    wide = false;
    if (topp) hist_clear();
    double zl = 0.0;           // this lane's total
    float vmax_t = -INFINITY;  // NaN once a NaN has been seen
    bool ovf = false;
    const uint64_t pol1 = topp ? pol_keep : pol_stream;
    // the first chunk first: the anchor, and for top-p rows the prediction
    {
      float x[8];
      const bool pre = pre_n > 0;  // the first copies went out at the start
      pre_n = 0;
      if (!st_peek<DT>(sh, r, c0, c1, pol1, ph, x, pre)) ok = false;
      const float cm = st_max8n(x);
      float g = G;
      if (!(G > -INFINITY)) {
        g = st_bmaxf(sh, rf, cm, false, nullptr);  // its barrier also orders hist_clear
      } else {
        __syncthreads();
      }
      // the prediction sums relative to g: the chunk's weight and its units' maxima's
      double z0 = 0.0, t0 = 0.0;
      if (topp && g > -INFINITY) {  // block-uniform
        const float gw = g * cw;
        float part = 0.0f;
#pragma unroll
        for (int e = 0; e < 8; ++e) part += st_ex2(fmaf(x[e], cw, -gw));
        const float mu = st_warp_max(cm);
        st_bsum2(sh, rf, (double)part, lane == 0 ? (double)st_ex2(fmaf(mu, cw, -gw)) : 0.0, z0, t0);
      }
      if (joint) {
        // one anchor for both halves (the larger first-chunk maximum) and the
        // prediction sums of both halves rescaled to it
        if (tid == 0) {
          st_peer_f32(st_peer(&sh.xch.g), g);
          st_peer_f64(st_peer(&sh.xch.z0), z0);
          st_peer_f64(st_peer(&sh.xch.t0), t0);
        }
        st_cluster_sync();
        const float gp = sh.xch.g;
        const float gm = fmaxf(g, gp);
        if (gm > -INFINITY) {
          const double fa = g > -INFINITY ? exp2(((double)g - (double)gm) * cl) : 0.0;
          const double fb = gp > -INFINITY ? exp2(((double)gp - (double)gm) * cl) : 0.0;
          const double za = z0 * fa, zb = sh.xch.z0 * fb, ta = t0 * fa, tb = sh.xch.t0 * fb;
          z0 = crank == 0 ? za + zb : zb + za;  // rank order: the same bits in both CTAs
          t0 = crank == 0 ? ta + tb : tb + ta;
        }
        g = gm;
        if (!(g > -INFINITY)) {
          // neither half starts with a finite value: the first CTA takes the
          // row alone, from a fresh start (the copies under way land first)
          if (!st_drain<DT, st_sub<DT, false>()>(sh, c0, c0, min(c1, c0 + st_nstages<DT>()), ph)) ok = false;
          if (crank == 1) return;
          joint = false;
          c0 = 0;
          c1 = r.nchunks;
          --attempt;
          continue;
        }
      }
      if (!(G > -INFINITY) && g > -INFINITY) set_anchor(g);
      if (topp && G > -INFINITY) {
        wide = t0 < P * z0;
        if (wide) set_hist_anchor(G);
      }
    }
    // per chunk: the weights' total (anchored once a finite value is seen)
    // and the unit's maximum (top-p) or weight sum (full softmax)
    auto weigh = [&](const float *x, float cm, int u) {
      vmax_t = st_maxn(vmax_t, cm);
      if (!(G > -INFINITY)) {  // block-uniform: no finite value seen yet (never in a shared row)
        const float g = st_bmaxf(sh, rf, cm, false, nullptr);
        if (g > -INFINITY) set_anchor(g);
      }
      float part = 0.0f;
      if (G > -INFINITY) {
        ovf = ovf || cm > v_ovf;  // NaN never
        const f2_t C = f2_pack(cw, cw), NA = f2_pack(-aw, -aw);
        f2_t s2 = st_w2(f2_pack(x[0], x[1]), C, NA);
#pragma unroll
        for (int j = 1; j < 4; ++j) s2 = f2_add(s2, st_w2(f2_pack(x[2 * j], x[2 * j + 1]), C, NA));
        float a0, a1;
        f2_unpack(s2, a0, a1);
        part = a0 + a1;
        zl += (double)part;
      }
      if (topp) {
        const float mu = st_warp_max(cm);
        if (lane == 0) sh.w.n.m[u] = mu;
      } else {
        const float su = warp_sum_f(part);
        if (lane == 0) sh.w.n.s[u] = su;
      }
    };
    if (wide) {
      ok = st_stream<DT, false>(
               sh, r, c0, c1, pol1, ph,
               [&](const float *x, int g0, int u, int) {
                 const float cm = st_max8n(x);
                 weigh(x, cm, u);
                 hist8(x, g0, cm);
               },
               StNoAfter(), true) &&
           ok;
    } else {
      ok = st_stream<DT, false>(
               sh, r, c0, c1, pol1, ph, [&](const float *x, int, int u, int) { weigh(x, st_max8n(x), u); },
               StNoAfter(), true) &&
           ok;
    }
    bool anyovf = __syncthreads_or(ovf) != 0;
    bool anybad;
    float vm = st_bmaxf(sh, rf, vmax_t, st_bad(vmax_t) || !ok, &anybad);
    double zs = st_bsum(sh, rf, zl);
    if (joint) {  // both halves' flags, maxima, totals and high-list sizes
      if (tid == 0) {
        st_peer_u32(st_peer(&sh.xch.flags), (anybad ? 1u : 0u) | (anyovf ? 4u : 0u));
        st_peer_f32(st_peer(&sh.xch.vmax), vm);
        st_peer_f64(st_peer(&sh.xch.zsum), zs);
        st_peer_u32(st_peer(&sh.xch.nhigh), (uint32_t)sh.nhigh);
      }
      st_cluster_sync();
      const uint32_t pf = sh.xch.flags;
      anybad = anybad || (pf & 1u) != 0u;
      anyovf = anyovf || (pf & 4u) != 0u;
      vm = fmaxf(vm, sh.xch.vmax);
      zs = crank == 0 ? zs + sh.xch.zsum : sh.xch.zsum + zs;
    }
    vmax = vm;
    if (anybad) {
      if (tid == 0 && crank == 0) a.status[row] = kRowPending;
      return;
    }
    if (!(vmax > -INFINITY)) {  // every logit -inf (sampler.py:46-47)
      if (tid == 0 && crank == 0) write_row(a, row, -1, 0.0f, MS_ROW_ALL_MASKED);
      return;
    }
    if (!(fabs((double)vmax) * cl < 1e37) || (anyovf && attempt > 0)) {  // beyond fp32 range
      if (tid == 0 && crank == 0) a.status[row] = kRowPending;
      return;
    }
    if (anyovf) continue;
    zsum = zs;
    break;
  }

  if (!topp) {  // the draw over the unit sums (sampler.py:60-68)
    double *kd = reinterpret_cast<double *>(st_scratch(sh, 1));
    double zs = 0.0;
    for (int u = tid; u < nu; u += kStThreads) {
      kd[u] = (double)sh.w.n.s[u];
      zs += kd[u];
    }
    const double total = st_bsum(sh, rf, zs);  // its barrier follows every kd write
    st_draw_units<DT>(sh, rf, a, r, row, nu, kd, total, U, [&](float v, int) -> double { return (double)W(v); });
    return;
  }

  // ============================================================ top-p only
  // weights relative to the row maximum: rw(v) = W(v) * fG <= 1
  const double fG = 1.0 / (double)W(vmax);
  auto rw = [&](float v) -> double { return (double)W(v) * fG; };
  const double total = zsum * fG;
  const double pz = P * total;
  uint32_t *gk = sh.w.n.x.g.key;
  int *gi = sh.w.n.x.g.idx;
  int n = 0;               // captured entries
  bool narrow = false;     // the captured entries are every value at or above a bound below the nucleus
  double above_tot = 0.0;  // wide: the mass above the bracket
  bool tail_bracketed = false;  // wide: the bracket reaches the tail, so no cut keeps every token
  int nhigh_all = sh.nhigh;  // high-list entries of both halves (rank 0: its list holds both)

  // a shared row: the second half's unit maxima, histogram and high list go
  // to the first CTA (its ring is idle: the histogram lands there)
  if (joint) {
    nhigh_all = crank == 0 ? sh.nhigh + sh.xch.nhigh : sh.xch.nhigh + sh.nhigh;
    if (crank == 1) {
      const uint32_t m_p = st_peer(sh.w.n.m);
      for (int u = c0 * kStWarps + tid; u < c1 * kStWarps; u += kStThreads)
        st_peer_f32(m_p + 4u * (uint32_t)u, sh.w.n.m[u]);
      if (wide) {
        const uint4 *h4 = reinterpret_cast<const uint4 *>(hq);
        const uint32_t dst = st_peer(st_scratch(sh, 0));
        for (int i = tid; i < kQSlots / 4; i += kStThreads) st_peer_v4(dst + 16u * (uint32_t)i, h4[i]);
        const int n0h = sh.xch.nhigh, n1h = min(sh.nhigh, kHighCap);
        const uint32_t hk_p = st_peer(sh.w.n.hkey), hi_p = st_peer(sh.w.n.hidx);
        for (int i = tid; i < n1h && n0h + i < kHighCap; i += kStThreads) {
          st_peer_u32(hk_p + 4u * (uint32_t)(n0h + i), sh.w.n.hkey[i]);
          st_peer_u32(hi_p + 4u * (uint32_t)(n0h + i), (uint32_t)sh.w.n.hidx[i]);
        }
      }
    }
    st_cluster_sync();
    if (crank == 0 && wide) {
      const uint32_t *rcv = reinterpret_cast<const uint32_t *>(st_scratch(sh, 0));
      for (int i = tid; i < kQSlots; i += kStThreads) hq[i] += rcv[i];
      if (tid == 0) sh.nhigh = nhigh_all;
      __syncthreads();
    }
  }

  // the bracket [i_lo, i_hi] of histogram indices (-1 = the high list,
  // kSBins + 1 = the tail) where the estimated running mass crosses
  // P*total -/+ kHistTol*total, as values: above <=> v > v_lo; in the bracket
  // <=> v_hi < v <= v_lo (t < bound <=> v > Gh - (bound - t_off) / xs).  The
  // classifying pass is the arbiter: a value near a bin edge may land on
  // either side of the histogram's split, which moves only the estimate; the
  // exact checks below catch a bracket that misses the crossing.  First CTA
  // (or a CTA alone).
  float v_lo = INFINITY, v_hi = -INFINITY;
  auto bracket = [&]() {
    __syncthreads();
    // the high list: exact weights
    const int nh = min(sh.nhigh, kHighCap);
    double hs = 0.0;
    for (int i = tid; i < nh; i += kStThreads) hs += rw(key_to_float(sh.w.n.hkey[i]));
    const double H = st_bsum(sh, rf, hs);
    int i_lo, i_hi;
    constexpr int kPer = kQSlots / kStThreads;
    const double rG = exp2(((double)Gh - (double)vmax) * cl);  // anchor weight / max weight
    double mb[kPer];
    double s = 0.0;
    // bin i's weight e^-((i - 1 - kUpBins) dx) * rG / kQScale: one exp for the
    // thread's first bin, then a factor e^-dx per bin
    const double step = exp(-(double)dx);
    double wb = exp(-(double)(tid * kPer - 1 - kUpBins) * (double)dx) * (rG / (double)kQScale);
#pragma unroll
    for (int q = 0; q < kPer; ++q) {
      const int i = tid * kPer + q;
      // index 0: values above the grid, counted exactly in H; the tail's
      // mass (each < e^-30 of the anchor's weight) is left out
      mb[q] = (i >= 1 && i <= kSBins) ? (double)hq[i] * wb : 0.0;
      wb *= step;
      s += mb[q];
    }
    double ex, inc, tot;
    st_bscan(sh, rf, s, ex, inc, tot);
    const double zh = H + tot;
    const double lo_t = P * zh - kHistTol * zh, hi_t = P * zh + kHistTol * zh;
    int clo = 0x7FFFFFFF, chi = 0x7FFFFFFF;
    double acc = H + ex;
#pragma unroll
    for (int q = 0; q < kPer; ++q) {
      acc += mb[q];
      if (clo == 0x7FFFFFFF && acc >= lo_t) clo = tid * kPer + q;
      if (chi == 0x7FFFFFFF && acc >= hi_t) chi = tid * kPer + q;
    }
    int mlo, mhi;
    st_bmin2(sh, rf, clo, chi, mlo, mhi);
    i_lo = H >= lo_t ? -1 : mlo;
    i_hi = H >= hi_t ? -1 : mhi;
    if (i_lo == 0x7FFFFFFF || i_lo > kSBins) i_lo = kSBins + 1;
    if (i_hi == 0x7FFFFFFF || i_hi > kSBins) i_hi = kSBins + 1;
    auto t_to_v = [&](double tb) -> float { return (float)((double)Gh - (tb - (double)t_off) / (double)xs); };
    v_lo = i_lo < 0 ? INFINITY : t_to_v((double)i_lo);
    v_hi = i_hi < 0 ? t_to_v(1.0) : (i_hi > kSBins ? -INFINITY : t_to_v((double)(i_hi + 1)));
    tail_bracketed = i_hi > kSBins;
  };

  // kind: 0 a narrow nucleus (the first CTA finishes it alone), 1 wide with
  // the histogram of pass 1, 2 wide without a usable histogram
  int kind = 2;
  if (crank == 0) {
    // the bracket from pass 1's histogram first: the narrow attempt's
    // captures share its memory
    if (wide && nhigh_all <= kHighCap) {
      kind = 1;
      bracket();
    }
    // (skipped when pass 1 built the histogram: a wide nucleus was predicted)
    if (kind != 1) {
      // ---- a narrow nucleus: if the kNarrowUnits largest unit maxima, in
      // (value desc) order, reach top_p of the total by the j-th one, every
      // value at or above the j-th maximum holds at least that mass, so the
      // nucleus (sampler.py:50-57) lies at or above it -- and only the units
      // whose maximum reaches it hold such values
      uint32_t *uk = reinterpret_cast<uint32_t *>(st_scratch(sh, 2));
      for (int u = tid; u < nu; u += kStThreads) {
        const float mu = sh.w.n.m[u];
        uk[u] = mu > -INFINITY ? fkey(mu) : 0u;
      }
      __syncthreads();
      int above;
      const uint32_t kth = st_select_kth(sh, uk, nu, min(kNarrowUnits, nu), &above, 2);
      uint32_t *sk = reinterpret_cast<uint32_t *>(st_scratch(sh, 1) + 8192);
      int *su = reinterpret_cast<int *>(st_scratch(sh, 1) + 8192 + 4 * 4 * kNarrowUnits);
      int cnt = 0;
      for (int u = tid; u < nu; u += kStThreads) cnt += (uk[u] >= kth && uk[u] != 0u) ? 1 : 0;
      int ex, ng;
      st_bscan_i(sh, rf, cnt, ex, ng);
      if (ng <= 4 * kNarrowUnits) {  // block-uniform; more: ties in the leading bits, take the wide path
        for (int u = tid; u < nu; u += kStThreads) {
          if (uk[u] >= kth && uk[u] != 0u) {
            sk[ex] = uk[u];
            su[ex] = u;
            ++ex;
          }
        }
        __syncthreads();
        st_rank_sort(sh, sk, su, ng, false);  // (maximum desc, unit asc); thread i holds entry i below
        const double wm = tid < ng ? rw(key_to_float(sk[tid])) : 0.0;
        double wex, winc, wtot;
        st_bscan(sh, rf, wm, wex, winc, wtot);
        const int first = st_bmin(sh, rf, (tid < ng && winc >= pz) ? tid : 0x7FFFFFFF);
        if (first != 0x7FFFFFFF) {
          const uint32_t kb = sk[first];
          const float vb = key_to_float(kb);
          const int nvis = st_bmin(sh, rf, (tid < ng && sk[tid] < kb) ? tid : ng);  // the units reaching vb
          if (tid == 0) sh.ncand = 0;
          __syncthreads();
          bool gover = false;
          for (int i = tid >> 5; i < nvis; i += kStWarps) {
            float x[8];
            const int g0 = st_load_unit<DT>(r, su[i], x);
            unsigned m = 0;
  #pragma unroll
            for (int e = 0; e < 8; ++e) m |= (x[e] >= vb ? 1u : 0u) << e;
            if (m) {  // the lane's entries: one atomic for all of them
              int pos = atomicAdd(&sh.ncand, __popc(m));
              do {
                const int e = __ffs(m) - 1;
                m &= m - 1;
                if (pos < kSortCap) {
                  gk[pos] = fkey(st_pick8(x, e));
                  gi[pos] = st_gidx(g0, e);
                } else {
                  gover = true;
                }
                ++pos;
              } while (m);
            }
          }
          if (!__syncthreads_or(gover)) {
            narrow = true;
            n = sh.ncand;
          }
        }
      }
    }
    if (narrow) kind = 0;
  }
  if (joint) {  // the first CTA's decision
    if (crank == 0 && tid == 0) {
      st_peer_u32(st_peer(&sh.xch.kind), (uint32_t)kind);
      st_peer_f32(st_peer(&sh.xch.v_lo), v_lo);
      st_peer_f32(st_peer(&sh.xch.v_hi), v_hi);
    }
    st_cluster_sync();
    if (crank == 1) {
      kind = (int)sh.xch.kind;
      v_lo = sh.xch.v_lo;
      v_hi = sh.xch.v_hi;
    }
    if (kind == 0 && crank == 1) return;
  }

  if (!narrow) {
    // ---- a wide nucleus
    if (kind == 2) {
      // no histogram from pass 1 (a narrow nucleus was predicted), or many
      // values lie far above its anchor: a histogram pass (L2) anchored at
      // the row maximum, nothing above it
      __syncthreads();
      set_hist_anchor(vmax);
      hist_clear();
      __syncthreads();
      ok = st_stream<DT, false>(
          sh, r, c0, c1, pol_keep, ph, [&](const float *x, int g0, int, int) { hist8(x, g0, st_max8n(x)); },
          StNoAfter());
      if (joint) {  // the second half's histogram and copy status to the first CTA
        // first both passes end: the histogram lands in the first CTA's
        // stage ring, idle only then
        if (tid == 0) st_peer_u32(st_peer(&sh.xch.flags), ok ? 0u : 2u);
        st_cluster_sync();
        if (crank == 1) {
          const uint4 *h4 = reinterpret_cast<const uint4 *>(hq);
          const uint32_t dst = st_peer(st_scratch(sh, 0));
          for (int i = tid; i < kQSlots / 4; i += kStThreads) st_peer_v4(dst + 16u * (uint32_t)i, h4[i]);
        }
        st_cluster_sync();
        ok = ok && sh.xch.flags == 0u;
        if (crank == 0 && ok) {
          const uint32_t *rcv = reinterpret_cast<const uint32_t *>(st_scratch(sh, 0));
          for (int i = tid; i < kQSlots; i += kStThreads) hq[i] += rcv[i];
        }
      }
      if (!ok) {
        if (tid == 0 && crank == 0) a.status[row] = kRowPending;
        return;
      }
      if (crank == 0) bracket();
      if (joint) {
        if (crank == 0 && tid == 0) {
          st_peer_f32(st_peer(&sh.xch.v_lo), v_lo);
          st_peer_f32(st_peer(&sh.xch.v_hi), v_hi);
        }
        st_cluster_sync();
        if (crank == 1) {
          v_lo = sh.xch.v_lo;
          v_hi = sh.xch.v_hi;
        }
      }
    }
    // classifying pass (L2): this CTA's units reaching the bracket: per-unit
    // mass above it (into s_u) and the bracket's elements
    if (tid == 0) sh.ncand = 0;
    __syncthreads();
    bool gover = false;
    ok = st_stream<DT, false>(
        sh, r, c0, c1, pol_stream, ph,
        [&](const float *x, int g0, int u, int) {
          if (!(sh.w.n.m[u] > v_hi)) {  // nothing above or in the bracket (warp-uniform)
            if (lane == 0) sh.w.n.s[u] = 0.0f;
            return;
          }
          float above = 0.0f;
          uint32_t inb = 0u;  // bit e: x[e] lies in the bracket
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float xa = x[2 * j], xb = x[2 * j + 1];
            const bool aa = xa > v_lo, ab = xb > v_lo;
            above += (aa ? W(xa) : 0.0f) + (ab ? W(xb) : 0.0f);
            inb |= ((uint32_t)(xa > v_hi) & (uint32_t)!aa) << (2 * j);
            inb |= ((uint32_t)(xb > v_hi) & (uint32_t)!ab) << (2 * j + 1);
          }
          above = warp_sum_f(above);
          if (lane == 0) sh.w.n.s[u] = above;
          if (inb) {  // the lane's bracket entries: one atomic for all of them
            int pos = atomicAdd(&sh.ncand, __popc(inb));
            do {
              const int e = __ffs(inb) - 1;
              inb &= inb - 1;
              if (pos < kSortCap) {
                gk[pos] = fkey(st_pick8(x, e));
                gi[pos] = st_gidx(g0, e);
              } else {
                gover = true;
              }
              ++pos;
            } while (inb);
          }
        },
        StNoAfter());
    n = sh.ncand;  // st_stream ended with a barrier
    bool fail = __syncthreads_or(!ok || gover) != 0;  // a crowded bracket: generic kernel
    if (joint) {
      // entry counts and failures of both halves; then the second half's
      // entries (after the first's), and its units' masses, to the first CTA
      if (tid == 0) {
        st_peer_u32(st_peer(&sh.xch.ncand), (uint32_t)n);
        st_peer_u32(st_peer(&sh.xch.flags), fail ? 8u : 0u);
      }
      st_cluster_sync();
      const int np_ = (int)sh.xch.ncand;
      fail = fail || sh.xch.flags != 0u || n + np_ > kSortCap;
      if (fail) {  // both CTAs stop here
        if (tid == 0 && crank == 0) a.status[row] = kRowPending;
        return;
      }
      if (crank == 1) {
        const uint32_t gk_p = st_peer(gk), gi_p = st_peer(gi);
        for (int i = tid; i < n; i += kStThreads) {
          st_peer_u32(gk_p + 4u * (uint32_t)(np_ + i), gk[i]);
          st_peer_u32(gi_p + 4u * (uint32_t)(np_ + i), (uint32_t)gi[i]);
        }
        const uint32_t s_p = st_peer(sh.w.n.s);
        for (int u = c0 * kStWarps + tid; u < c1 * kStWarps; u += kStThreads)
          st_peer_f32(s_p + 4u * (uint32_t)u, sh.w.n.s[u]);
      }
      st_cluster_sync();
      if (crank == 1) return;
      n += np_;
    } else if (fail) {
      if (tid == 0) a.status[row] = kRowPending;
      return;
    }
    double as = 0.0;
    for (int u = tid; u < nu; u += kStThreads) as += (double)sh.w.n.s[u];
    above_tot = st_bsum(sh, rf, as) * fG;
    if (above_tot > 0.0 && above_tot >= pz) {  // the crossing lies above the bracket
      if (tid == 0) a.status[row] = kRowPending;
      return;
    }
  }

  // The cut: the first captured entry in (value desc, index asc) order whose
  // running mass, after above_tot, reaches P*total (miniserve/sampler.py:50-57)
  // -- (ck, ci); or none, when the captured mass falls short.
  const double need = pz - above_tot;
  // the first of m sorted entries whose running mass from `base` reaches
  // need, or 0x7FFFFFFF
  auto scan_sorted = [&](const uint32_t *sk, const int *si, int m, double base) -> int {
    const int per = (m + kStThreads - 1) / kStThreads;
    const int p0 = tid * per, p1 = min(m, p0 + per);
    double sw = 0.0;
    for (int i = p0; i < p1; ++i) sw += rw(key_to_float(sk[i]));
    double ex, inc, tt;
    st_bscan(sh, rf, sw, ex, inc, tt);
    int cand = 0x7FFFFFFF;
    if (p0 < p1 && base + inc >= need) {
      double acc = base + ex;
      for (int i = p0; i < p1; ++i) {
        acc += rw(key_to_float(sk[i]));
        if (acc >= need) {
          cand = i;
          break;
        }
      }
      if (cand == 0x7FFFFFFF) cand = p1 - 1;
    }
    return st_bmin(sh, rf, cand);
  };
  uint32_t ck = 0u;
  int ci = 0x7FFFFFFF;
  int state = 2;  // 0: the cut found, 1: none, 2: not resolved yet
  if (n > kRankCap / 4) {
    // A large set: 256 key buckets with fixed-point masses place the
    // crossing within a window of buckets, and only the window is sorted.
    // Bucket b holds keys kmin + [b << bsh, (b + 1) << bsh).
    int lo_i = 0x7FFFFFFF, hi_i = 0x7FFFFFFF;
    for (int i = tid; i < n; i += kStThreads) {
      lo_i = min(lo_i, (int)(gk[i] ^ 0x80000000u));
      hi_i = min(hi_i, (int)(~gk[i] ^ 0x80000000u));
    }
    const uint32_t kmin = (uint32_t)st_bmin(sh, rf, lo_i) ^ 0x80000000u;
    const uint32_t kmax = ~((uint32_t)st_bmin(sh, rf, hi_i) ^ 0x80000000u);
    const int bsh = max(0, 24 - __clz((int)(kmax - kmin)));
    // w * qs < 2^18 for every entry: qs from the top key's weight, with a
    // margin far above the weights' rounding
    const double qs = 262144.0 / (exp2(((double)key_to_float(kmax) - (double)vmax) * cl) * 1.001);
    uint32_t *bcnt = reinterpret_cast<uint32_t *>(st_scratch(sh, 0));  // [256] entries, [256] mass
    for (int q = tid; q < 512; q += kStThreads) bcnt[q] = 0u;
    __syncthreads();
    for (int i = tid; i < n; i += kStThreads) {
      const int bk = (int)((gk[i] - kmin) >> bsh);
      const double w = rw(key_to_float(gk[i]));
      atomicAdd(&bcnt[bk], 1u);
      atomicAdd(&bcnt[256 + bk], (uint32_t)fmin(w * qs, 524288.0));  // floor: w*qs - 1 < q <= w*qs
    }
    __syncthreads();
    // every warp: C(b), N(b) = bucket mass and entries at or above b.  The
    // exact scaled mass at or above b lies in [C(b), C(b) + N(b)), so the
    // crossing bucket b* (highest b whose exact mass reaches need) satisfies
    // b_lo <= b* <= b_hi with b_lo = highest b with C(b) >= T and b_hi =
    // highest b with C(b) + N(b) >= T.
    const double Tq = need * qs;
    uint32_t cq[8], cn[8], sq = 0, sn = 0;
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const int bk = 255 - 8 * lane - q;
      cn[q] = bcnt[bk];
      cq[q] = bcnt[256 + bk];
      sq += cq[q];
      sn += cn[q];
    }
    uint32_t iq = sq, in_ = sn;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t yq = __shfl_up_sync(0xFFFFFFFFu, iq, o), yn = __shfl_up_sync(0xFFFFFFFFu, in_, o);
      if (lane >= o) {
        iq += yq;
        in_ += yn;
      }
    }
    double cacc = (double)(iq - sq), nacc = (double)(in_ - sn);
    int blo = -1, bhi = -1;
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      cacc += (double)cq[q];
      nacc += (double)cn[q];
      if (blo < 0 && cacc >= Tq) blo = 255 - 8 * lane - q;
      if (bhi < 0 && cacc + nacc >= Tq) bhi = 255 - 8 * lane - q;
    }
    blo = __reduce_max_sync(0xFFFFFFFFu, blo);  // highest bucket: lowest lane's first hit
    bhi = __reduce_max_sync(0xFFFFFFFFu, bhi);
    if (bhi < 0) {
      state = 1;  // even the largest possible captured mass falls short of need
    } else {
      const int wlo = max(blo, 0);
      // exact mass above the window, and the window's entries gathered
      double am = 0.0;
      int wc = 0;
      for (int i = tid; i < n; i += kStThreads) {
        const int bk = (int)((gk[i] - kmin) >> bsh);
        if (bk > bhi) am += rw(key_to_float(gk[i]));
        else if (bk >= wlo) ++wc;
      }
      const double A = st_bsum(sh, rf, am);
      int wex, m;
      st_bscan_i(sh, rf, wc, wex, m);
      if (A < need && m <= kRankCap) {  // otherwise the buckets misled: sort everything
        uint32_t *wk = reinterpret_cast<uint32_t *>(st_scratch(sh, 1) + 8192);
        int *wi = reinterpret_cast<int *>(st_scratch(sh, 1) + 12288);
        for (int i = tid; i < n; i += kStThreads) {
          const int bk = (int)((gk[i] - kmin) >> bsh);
          if (bk <= bhi && bk >= wlo) {
            wk[wex] = gk[i];
            wi[wex] = gi[i];
            ++wex;
          }
        }
        __syncthreads();
        st_rank_sort(sh, wk, wi, m, false);
        const int pc = scan_sorted(wk, wi, m, A);
        if (pc != 0x7FFFFFFF) {
          ck = wk[pc];
          ci = wi[pc];
          state = 0;
        } else if (blo < 0) {
          state = 1;  // the window reaches the captured set's bottom: its mass falls short
        }
      }
    }
  }
  if (state == 2) {  // a small set, or the buckets misled: sort it all
    if (n <= kRankCap) {
      st_rank_sort(sh, gk, gi, n, false);
    } else {
      st_sort(gk, gi, n, false);
    }
    const int pc = scan_sorted(gk, gi, n, 0.0);
    if (pc != 0x7FFFFFFF) {
      ck = gk[pc];
      ci = gi[pc];
      state = 0;
    } else {
      state = 1;
    }
  }
  // no cut: with the tail bracketed the running sum never reaches top_p and
  // every token is kept; otherwise the crossing lies below the captured set
  // (for a narrow nucleus only through rounding at the bound)
  if (state == 1 && !tail_bracketed) {
    if (tid == 0) a.status[row] = kRowPending;
    return;
  }
  const float vc = state == 1 ? -INFINITY : key_to_float(ck);
  const int ic = state == 1 ? 0x7FFFFFFF : ci;
  // kept mass per unit: above the bracket (wide: s_u) plus the unit's kept
  // captured entries, those summed as 2^-50 fixed point (exact and order-free)
  unsigned long long *ex64 = reinterpret_cast<unsigned long long *>(st_scratch(sh, 2));
  for (int u = tid; u < nu; u += kStThreads) ex64[u] = 0ull;
  __syncthreads();
  for (int i = tid; i < n; i += kStThreads) {
    if (state == 1 || gk[i] > ck || (gk[i] == ck && gi[i] <= ci)) {  // at or before the cut
      const double w = rw(key_to_float(gk[i]));  // <= 1
      atomicAdd(&ex64[gi[i] / kUnit], (unsigned long long)(w * 0x1p50));
    }
  }
  __syncthreads();
  double *kd = reinterpret_cast<double *>(st_scratch(sh, 1));
  double tk = 0.0;
  for (int u = tid; u < nu; u += kStThreads) {
    kd[u] = (narrow ? 0.0 : (double)sh.w.n.s[u] * fG) + (double)ex64[u] * 0x1p-50;
    tk += kd[u];
  }
  const double tot_keep = st_bsum(sh, rf, tk);
  st_draw_units<DT>(sh, rf, a, r, row, nu, kd, tot_keep, U, [&](float v, int g) -> double {
    if (!(v > -INFINITY) || !(v > vc || (v == vc && g <= ic))) return 0.0;
    return rw(v);
  });
}

// Fused peer exchange of vocab-sharded sampling (ms_shard_exchange): after
// the CTA wrote its record of `row` into its own buffer's plain area, every
// word goes to every other rank's tagged area over NVLink, as one 8-byte
// store of (epoch, word).  No fence and no wait: the merge kernel on each
// rank checks the epochs.
__device__ __forceinline__ void st_publish(const SampleArgs &a, const XArgs &x, int row) {
  const int tid = threadIdx.x;
  const int N = x.n, me = x.rank;
  const int W = 4 + 2 * a.kmax;
  __syncthreads();  // the record is written
  const uint32_t *src = st_record(a, row);
  const int64_t slot = ((int64_t)row * N + me) * W;
  const unsigned long long tag = (unsigned long long)x.epoch << 32;
  for (int i = tid; i < W; i += kStThreads) {
    const unsigned long long v = tag | src[i];
    for (int q = 1; q < N; ++q)
      x_st_relaxed_sys(reinterpret_cast<unsigned long long *>(x.peers[(me + q) % N] + x.ll) + slot + i, v);
  }
}

template <int DT>
__global__ void __launch_bounds__(kStThreads, 2) ms_stream_kernel(SampleArgs a) {
  extern __shared__ __align__(128) unsigned char st_raw[];
  StShared &sh = *reinterpret_cast<StShared *>(st_raw);
  int prow = -1;
  st_row_body<DT, false>(a, sh, prow);
}

// The streaming kernel in vocab-sharded mode with the fused peer exchange
// (one CTA per row): the row's record, then st_publish.
template <int DT>
__global__ void __launch_bounds__(kStThreads, 2) ms_stream_xkernel(SampleArgs a, XArgs x) {
  extern __shared__ __align__(128) unsigned char st_raw[];
  StShared &sh = *reinterpret_cast<StShared *>(st_raw);
  int prow = -1;
  st_row_body<DT, true>(a, sh, prow);
  if (prow >= 0 && x.n > 1) st_publish(a, x, prow);
}
}  // namespace ms
