// Generic sampling kernel: one 1024-thread CTA per row, multi-pass over the
// row in global memory.  Exact for every input the C ABI accepts (any V, any
// top_k / top_p, ties, masks) and simple enough to trust: it only uses
// CTA-level barriers.  The streaming kernel hands it the rows it does not
// finish (status kRowPending).
//
// Semantics follow miniserve/sampler.py:23-68 (see ms_sample.cu for the map).
#pragma once

#include "ms_common.cuh"

namespace ms {

constexpr int kGenThreads = 1024;
constexpr int kBins = 2048;
constexpr int kItems = 4;  // consecutive elements per thread in ordered (tile) loops
constexpr int kTile = kGenThreads * kItems;

struct GenShared {
  uint32_t cnt[kBins];
  double mass[kBins];
  double redd[33];
  uint32_t redu[33];
  int redi[33];
  uint32_t bkey[32];
  int bidx[32];
  int bcast_i[4];
  double bcast_d[4];
};

struct SampleArgs {
  const void *logits;
  int64_t ld;
  int V;
  const double *temperature;
  const int32_t *top_k;
  const double *top_p;
  const double *uniforms;
  const uint32_t *mask;
  int64_t mask_ld;
  int64_t *tokens;
  float *probs;
  int32_t *status;
  // vocab-sharded candidate mode (ms_shard_candidates): when records is set
  // the streaming kernel writes one candidate record per row instead of a
  // token; the row is the slice [v0, v0 + V) of a Vg-token vocabulary
  uint32_t *records = nullptr;
  int kmax = 0;
  int64_t v0 = 0;
  int64_t Vg = 0;
  // pair mode (pairs > 0): the streaming kernel runs as 2 * rows CTAs in
  // clusters of two; when the batch holds at most `pairs` top-p rows each
  // takes both CTAs of a cluster, the other rows one CTA each
  int pairs = 0;
  int rows = 0;
};

template <int DT>
struct RowRef {
  const void *row;
  const uint32_t *mask_row;
  int V;
  __device__ __forceinline__ uint32_t key(int i) const {
    uint32_t f = 0;
    return bits_to_key(clean_bits(raw_bits<DT>(row, i), mask_allows(mask_row, i), f));
  }
};

__device__ __forceinline__ void write_row(const SampleArgs &a, int r, int64_t tok, float prob,
                                          int32_t st) {
  a.tokens[r] = tok;
  a.probs[r] = prob;
  a.status[r] = st;
}

// Key-radix selection inside the kept set `base`: the smallest top-ordered
// prefix (key descending, index ascending) whose weight reaches `thr`.
// COUNT: weight 1 per element (top-k, miniserve/sampler.py:38).
// MASS:  weight exp(x - max) (top-p in exp units, miniserve/sampler.py:50-57).
// Returns the cut describing that prefix; `base` itself when thr is never
// reached (the reference then keeps everything it iterated over).
template <int DT, bool MASS, int NT = kGenThreads>
__device__ Cut gen_select(const RowRef<DT> &row, Cut base, double thr, double dmax, double inv_t,
                          GenShared &sh) {
  const int tid = threadIdx.x;
  const int V = row.V;
  uint32_t prefix = 0;
  double above_w = 0.0;
  uint32_t last_cnt = 0;
  for (int level = 0; level < 3; ++level) {
    // digits of the 32-bit key: bits 31..21, 20..10, 9..0
    const int sh_ = level == 0 ? 21 : (level == 1 ? 10 : 0);
    const int bits = level == 2 ? 10 : 11;
    const int nb = 1 << bits;
    const uint32_t dmask = (uint32_t)nb - 1u;
    for (int b = tid; b < kBins; b += NT) {
      sh.cnt[b] = 0u;
      sh.mass[b] = 0.0;
    }
    __syncthreads();
    for (int i = tid; i < V; i += NT) {
      uint32_t key = row.key(i);
      if (key <= kNegInfKey || !kept(base, key, i)) continue;
      if (level > 0 && (key >> (sh_ + bits)) != prefix) continue;
      uint32_t d = (key >> sh_) & dmask;
      atomicAdd(&sh.cnt[d], 1u);
      if (MASS) atomicAdd(&sh.mass[d], weight_of(key_to_float(key), dmax, inv_t));
    }
    __syncthreads();
    // positions run from the highest digit down; each thread owns nb/NT
    const int per = nb / NT;  // 1, 2 or 4
    double s = 0.0;
    for (int j = 0; j < per; ++j) {
      int d = nb - 1 - (tid * per + j);
      s += MASS ? sh.mass[d] : (double)sh.cnt[d];
    }
    double excl, incl, tot;
    block_scan<NT, double>(s, excl, incl, tot, sh.redd);
    const double rel = thr - above_w;
    int cand = 0x7FFFFFFF;
    double acc = excl, before = 0.0;
    for (int j = 0; j < per; ++j) {
      int d = nb - 1 - (tid * per + j);
      double w = MASS ? sh.mass[d] : (double)sh.cnt[d];
      double b4 = acc;
      acc += w;
      if (sh.cnt[d] > 0u && acc >= rel) {
        cand = tid * per + j;
        before = b4;
        break;
      }
    }
    int pos = block_min_i<NT>(cand, sh.redi);
    if (pos == 0x7FFFFFFF) return base;  // never reached: keep the whole base set
    if (cand == pos) {
      sh.bcast_d[0] = before;
      sh.bcast_i[0] = (int)sh.cnt[nb - 1 - pos];
    }
    __syncthreads();
    above_w += sh.bcast_d[0];
    last_cnt = (uint32_t)sh.bcast_i[0];
    prefix = (prefix << bits) | (uint32_t)(nb - 1 - pos);
    __syncthreads();
  }
  const uint32_t tau = prefix;
  // number of ties (key == tau, index order) the prefix needs
  double need_d;
  if (MASS) {
    double e_tau = weight_of(key_to_float(tau), dmax, inv_t);
    need_d = e_tau > 0.0 ? ceil((thr - above_w) / e_tau) : (double)last_cnt;
  } else {
    need_d = thr - above_w;
  }
  int need = need_d < 1.0 ? 1 : (need_d >= (double)last_cnt ? (int)last_cnt : (int)need_d);
  const int base_cut = (tau == base.key) ? base.cut : kNoCut;
  if ((uint32_t)need >= last_cnt) return Cut{tau, base_cut};
  // find the index of the need-th tie in index order
  int running = 0;
  for (int t0 = 0; t0 < V; t0 += (NT * kItems)) {
    int c = 0;
    const int i0 = t0 + tid * kItems;
#pragma unroll
    for (int j = 0; j < kItems; ++j) {
      int i = i0 + j;
      if (i < V) {
        uint32_t key = row.key(i);
        c += (key == tau && kept(base, key, i)) ? 1 : 0;
      }
    }
    int excl_i, incl_i, tot_i;
    block_scan<NT, int>(c, excl_i, incl_i, tot_i, sh.redi);
    if (running + tot_i >= need) {
      if (running + excl_i < need && need <= running + incl_i) {
        int acc2 = running + excl_i;
        for (int j = 0; j < kItems; ++j) {
          int i = i0 + j;
          if (i >= V) break;
          uint32_t key = row.key(i);
          if (key == tau && kept(base, key, i) && ++acc2 == need) {
            sh.bcast_i[1] = i;
            break;
          }
        }
      }
      __syncthreads();
      int cut = sh.bcast_i[1];
      __syncthreads();
      return Cut{tau, cut};
    }
    running += tot_i;
  }
  return Cut{tau, base_cut};  // unreachable when counts are consistent
}

template <int DT, int NT = kGenThreads>
__device__ double gen_total(const RowRef<DT> &row, Cut c, double dmax, double inv_t, GenShared &sh) {
  double s = 0.0;
  for (int i = threadIdx.x; i < row.V; i += NT) {
    uint32_t key = row.key(i);
    if (key > kNegInfKey && kept(c, key, i)) s += weight_of(key_to_float(key), dmax, inv_t);
  }
  return block_sum<NT>(s, sh.redd);
}

// Index-order inverse CDF over the kept set (miniserve/sampler.py:62-68):
// the first index whose running weight reaches u * total; V-1 when none does.
template <int DT, int NT = kGenThreads>
__device__ void gen_draw(const RowRef<DT> &row, Cut c, double total, double u, double dmax,
                         double inv_t, const SampleArgs &a, int r, uint32_t flags, GenShared &sh) {
  const int tid = threadIdx.x;
  const int V = row.V;
  auto wt = [&](int i) -> double {
    uint32_t key = row.key(i);
    return (key > kNegInfKey && kept(c, key, i)) ? weight_of(key_to_float(key), dmax, inv_t) : 0.0;
  };
  if (!(u > 0.0)) {  // r == 0 stops at index 0 whatever its probability
    if (tid == 0) write_row(a, r, 0, (float)(wt(0) / total), (int32_t)flags);
    return;
  }
  const double target = u * total;
  double running = 0.0;
  for (int t0 = 0; t0 < V; t0 += (NT * kItems)) {
    double w[kItems];
    double s = 0.0;
    const int i0 = t0 + tid * kItems;
#pragma unroll
    for (int j = 0; j < kItems; ++j) {
      int i = i0 + j;
      w[j] = (i < V) ? wt(i) : 0.0;
      s += w[j];
    }
    double excl, incl, tot;
    block_scan<NT, double>(s, excl, incl, tot, sh.redd);
    int cand = (s > 0.0 && running + incl >= target) ? tid : 0x7FFFFFFF;
    int who = block_min_i<NT>(cand, sh.redi);
    if (who != 0x7FFFFFFF) {
      if (tid == who) {
        double cum = running + excl;
        int tok = -1, last = -1;
        double wtok = 0.0, wlast = 0.0;
#pragma unroll
        for (int j = 0; j < kItems; ++j) {
          if (w[j] > 0.0 && tok < 0) {
            cum += w[j];
            last = i0 + j;
            wlast = w[j];
            if (cum >= target) {
              tok = i0 + j;
              wtok = w[j];
            }
          }
        }
        if (tok < 0) {  // rounding put the crossing past this run's sum
          tok = last;
          wtok = wlast;
        }
        write_row(a, r, tok, (float)(wtok / total), (int32_t)flags);
      }
      return;
    }
    running += tot;
  }
  if (tid == 0) write_row(a, r, V - 1, (float)(wt(V - 1) / total), (int32_t)flags);
}

template <int DT, int NT = kGenThreads>
__device__ void gen_row(const SampleArgs &a, int r, GenShared &sh) {
  const int tid = threadIdx.x;
  RowRef<DT> row;
  row.row = DT == MS_DTYPE_F32
                ? (const void *)((const float *)a.logits + (int64_t)r * a.ld)
                : (const void *)((const unsigned short *)a.logits + (int64_t)r * a.ld);
  row.mask_row = a.mask ? a.mask + (int64_t)r * a.mask_ld : nullptr;
  row.V = a.V;
  // ---- pass 1: max (first index on ties), valid count, non-finite flags
  uint32_t flags = 0, bk = 0u, nvalid = 0;
  int bi = 0x7FFFFFFF;
  for (int i = tid; i < a.V; i += NT) {
    uint32_t u = clean_bits(raw_bits<DT>(row.row, i), mask_allows(row.mask_row, i), flags);
    uint32_t key = bits_to_key(u);
    if (key > bk) {
      bk = key;
      bi = i;
    }
    nvalid += key > kNegInfKey ? 1u : 0u;
  }
  if (bi == 0x7FFFFFFF) bk = 0u;
  warp_argmax(bk, bi);
  flags = __reduce_or_sync(0xFFFFFFFFu, flags);
  if ((tid & 31) == 0) {
    sh.bkey[tid >> 5] = bk;
    sh.bidx[tid >> 5] = bi;
    sh.redu[tid >> 5] = flags;
  }
  __syncthreads();
  if (tid < 32) {  // one slot per warp: NT / 32 of them hold values
    constexpr int NW = NT / 32;
    uint32_t k2 = tid < NW ? sh.bkey[tid] : 0u;
    int i2 = tid < NW ? sh.bidx[tid] : 0x7FFFFFFF;
    uint32_t f2 = tid < NW ? sh.redu[tid] : 0u;
    warp_argmax(k2, i2);
    f2 = __reduce_or_sync(0xFFFFFFFFu, f2);
    if (tid == 0) {
      sh.bkey[0] = k2;
      sh.bidx[0] = i2;
      sh.bcast_i[2] = (int)f2;
    }
  }
  __syncthreads();
  const uint32_t max_key = sh.bkey[0];
  const int max_idx = sh.bidx[0];
  flags = (uint32_t)sh.bcast_i[2];
  __syncthreads();
  nvalid = block_sum_u32<NT>(nvalid, sh.redu);

  const double T = a.temperature[r];
  const int k = a.top_k[r];
  const double p = a.top_p[r];
  const double u = a.uniforms[r];
  // greedy (miniserve/sampler.py:33-34)
  if (T == 0.0) {
    if (tid == 0) write_row(a, r, max_idx, 1.0f, (int32_t)flags);
    return;
  }
  if (!(T > 0.0) || isinf(T)) {
    if (tid == 0) write_row(a, r, -1, 0.0f, (int32_t)(flags | MS_ROW_BAD_TEMPERATURE));
    return;
  }
  if (nvalid == 0u) {  // ZeroDivisionError in the reference (sampler.py:46-47)
    if (tid == 0) write_row(a, r, -1, 0.0f, (int32_t)(flags | MS_ROW_ALL_MASKED));
    return;
  }
  if (max_key == bits_to_key(kPosInfBits)) {  // +inf logit: first +inf index
    if (tid == 0) write_row(a, r, max_idx, 1.0f, (int32_t)flags);
    return;
  }
  // top_k >= number of finite logits keeps everything (sampler.py:37-42)
  const int keff = (k > 0 && (uint32_t)k < nvalid) ? k : 0;
  if (keff == 1) {
    if (tid == 0) {
      if (u > 0.0)
        write_row(a, r, max_idx, 1.0f, (int32_t)flags);
      else
        write_row(a, r, 0, max_idx == 0 ? 1.0f : 0.0f, (int32_t)flags);
    }
    return;
  }
  const double dmax = (double)key_to_float(max_key);
  const double inv_t = 1.0 / T;
  Cut c = cut_all();
  if (keff > 1) c = gen_select<DT, false, NT>(row, c, (double)keff, dmax, inv_t, sh);
  double total = gen_total<DT, NT>(row, c, dmax, inv_t, sh);
  if (p < 1.0) {
    c = gen_select<DT, true, NT>(row, c, p * total, dmax, inv_t, sh);
    total = gen_total<DT, NT>(row, c, dmax, inv_t, sh);
  }
  gen_draw<DT, NT>(row, c, total, u, dmax, inv_t, a, r, flags, sh);
}

// rows: optional device list of row indices with its device count; when null
// every row 0..gridDim.x-1 is processed.
template <int DT>
__global__ void __launch_bounds__(kGenThreads, 1)
    ms_generic_kernel(SampleArgs a, const int *rows, const int *nrows) {
  __shared__ GenShared sh;
  int r = blockIdx.x;
  if (rows) {
    if (r >= *nrows) return;
    r = rows[r];
  }
  gen_row<DT>(a, r, sh);
}

// Finishes the rows the streaming kernel left with status kRowPending; a
// grid-stride loop, so the grid can stay one CTA per SM whatever B is.
template <int DT>
__global__ void __launch_bounds__(kGenThreads, 1) ms_generic_pending_kernel(SampleArgs a, int B) {
  __shared__ GenShared sh;
  // launched as a programmatic dependent of ms_stream_kernel: wait for that
  // grid (and its status writes) to complete; a no-op for a plain launch
  asm volatile("griddepcontrol.wait;" ::: "memory");
  for (int r = blockIdx.x; r < B; r += gridDim.x) {
    if (a.status[r] != kRowPending) continue;
    gen_row<DT>(a, r, sh);
    __syncthreads();
  }
}

}  // namespace ms
