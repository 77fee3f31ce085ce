// Merge step of vocab-sharded sampling: one 256-thread CTA per row reads the
// all-gathered candidate records of every rank ([nranks][B][4 + 2*kmax]
// words), ranks the union by (value descending, global id ascending) and
// finishes the row exactly as miniserve/sampler.py:23-68 does on the full
// vocabulary: the global top-k set is contained in the union of the slices'
// top-k sets, and every weight exp(l/T - max/T) is computed in float64 from
// the exact logit (its order key).  A top-p row without top-k is finished when
// its nucleus lies among the candidates: the slices' totals give the row's
// softmax total, and a crossing value above every full slice's kmax-th
// largest value has every larger value of the row among the candidates;
// otherwise the row is flagged MS_ROW_UNSUPPORTED.
//
// The row merge (mg_row) runs after an all-gather (ms_merge_kernel) or on
// the records of the fused peer exchange (ms_xmerge_kernel, ms_exchange.cuh).
#pragma once

#include "ms_common.cuh"
#include "ms_generic.cuh"

namespace ms {

constexpr int kMgThreads = 256;
constexpr int kMgCap = 2048;     // candidates per row over all ranks
constexpr int kMgTopK = 256;     // largest kmax
constexpr int kMgRanks = 256;    // largest nranks

struct MergeArgs {
  const uint32_t *records;
  int nranks;
  int B;
  int kmax;
  int64_t V;  // the full vocabulary
  const double *temperature;
  const int32_t *top_k;
  const double *top_p;
  const double *uniforms;
  int64_t *tokens;
  float *probs;
  int32_t *status;
  // fused peer exchange with more than one rank: the result of row r goes to
  // every rank's buffer instead, as three 8-byte stores tagged with the
  // call's epoch (token, prob bits, status) at 8-byte slot 4 r of word
  // offset xres
  uint32_t *const *xpeers = nullptr;
  int64_t xres = 0;
  uint32_t xepoch = 0;
};

__device__ __forceinline__ void mg_st_sys(unsigned long long *p, unsigned long long v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

struct MgShared {
  union {
    unsigned long long comp[kMgCap + 2];  // (key, ~id) composites, padded for paired reads
    double kw[kMgCap];                    // after the ranking: kept weights in index order
  } u;
  uint32_t key[kMgCap];  // candidates in rank order
  int id[kMgCap];
  int kid[kMgCap];       // kept ids in index order
  int off[kMgRanks + 1];
  int cnt[kMgRanks];     // per-rank candidate counts
  uint32_t st;
  float cut;             // the largest kmax-th value of a full slice
  double redd[33];
  int redi[33];
  unsigned long long redq[33];
};

__device__ __forceinline__ void mg_write(const MergeArgs &a, int r, int64_t tok, float prob, int32_t st) {
  if (a.xpeers) {
    const unsigned long long tag = (unsigned long long)a.xepoch << 32;
    for (int q = 0; q < a.nranks; ++q) {
      unsigned long long *e = reinterpret_cast<unsigned long long *>(a.xpeers[q] + a.xres) + 4 * (size_t)r;
      mg_st_sys(e, tag | (uint32_t)(int32_t)tok);
      mg_st_sys(e + 1, tag | __float_as_uint(prob));
      mg_st_sys(e + 2, tag | (uint32_t)st);
    }
    return;
  }
  a.tokens[r] = tok;
  a.probs[r] = prob;
  a.status[r] = st;
}

// Rank r's record of `row`; read through L2 (records that other GPUs wrote
// into a fused exchange buffer are never served from a stale L1 line).
__device__ __forceinline__ const uint32_t *mg_rec(const MergeArgs &a, int r, int row, size_t rw) {
  return a.records + ((size_t)r * a.B + row) * rw;
}
__device__ __forceinline__ uint32_t mg_ld(const uint32_t *p) { return __ldcg(p); }

// A row without top-k (miniserve/sampler.py:35-68 with top_k off): every
// candidate ranked; float64 weights exp(l/T - max/T); the row's total from the
// slices' totals; the smallest rank prefix reaching top_p (crossing entry
// kept), settled only when the crossing value lies above every full slice's
// kmax-th largest value; the index-order draw over the kept prefix.  The
// composites of the n candidates are in sh.u.comp.  All threads.
template <int NT>
__device__ void mg_nucleus(const MergeArgs &a, MgShared &sh, int row, int n, size_t rw, double T, double P,
                           double U) {
  const int tid = threadIdx.x;
  if (!(P < 1.0)) {  // the full softmax draw needs every logit
    if (tid == 0) mg_write(a, row, -1, 0.0f, MS_ROW_UNSUPPORTED);
    return;
  }
  // rank every candidate (all distinct composites)
  const ulonglong2 *c2 = reinterpret_cast<const ulonglong2 *>(sh.u.comp);
  const int npair = (n + 1) >> 1;
  for (int i = tid; i < n; i += NT) {
    const unsigned long long ci = sh.u.comp[i];
    int rank = 0;
    for (int j = 0; j < npair; ++j) {
      const ulonglong2 q = c2[j];
      rank += (q.x > ci ? 1 : 0) + (q.y > ci ? 1 : 0);
    }
    sh.key[rank] = (uint32_t)(ci >> 32);
    sh.id[rank] = (int)~(uint32_t)ci;
  }
  __syncthreads();
  // the row's total: sum over slices of total_r * exp((m_r - max) / T), m_r a
  // slice's maximum (its first key); the cut: a full slice's last value
  const float vmax = key_to_float(sh.key[0]);
  double zr = 0.0;
  if (tid < a.nranks) {
    const uint32_t *rec = mg_rec(a, tid, row, rw);
    const int mr = (int)min(mg_ld(rec), (uint32_t)a.kmax);
    if (mr > 0) {
      const unsigned long long b = (unsigned long long)mg_ld(rec + 2 + 2 * a.kmax) |
                                   ((unsigned long long)mg_ld(rec + 3 + 2 * a.kmax) << 32);
      zr = __longlong_as_double((long long)b) * exp(((double)key_to_float(mg_ld(rec + 2)) - (double)vmax) / T);
    }
  }
  __syncthreads();
  if (tid == 0) {  // the largest last value among full slices (at most kMgRanks reads)
    float cut = -INFINITY;
    for (int r = 0; r < a.nranks; ++r) {
      const uint32_t *rec = mg_rec(a, r, row, rw);
      if ((int)min(mg_ld(rec), (uint32_t)a.kmax) == a.kmax) cut = fmaxf(cut, key_to_float(mg_ld(rec + 2 + a.kmax - 1)));
    }
    sh.cut = cut;
  }
  const double Z = block_sum<NT>(zr, sh.redd);  // ends with a barrier
  const float cut = sh.cut;
  // weights in rank order, a contiguous block of ranks per thread
  const int per = (n + NT - 1) / NT;
  const int p0 = tid * per, p1 = min(n, p0 + per);
  const double xmax = (double)vmax / T;
  double sw = 0.0;
  for (int i = p0; i < p1; ++i) sw += exp((double)key_to_float(sh.key[i]) / T - xmax);
  double ex, inc, tt;
  block_scan<NT, double>(sw, ex, inc, tt, sh.redd);
  const double need = P * Z;
  int cand = 0x7FFFFFFF;
  if (p0 < p1 && inc >= need) {  // sampler.py:54-57: cumsum >= top_p, crossing entry kept
    double acc = ex;
    for (int i = p0; i < p1; ++i) {
      acc += exp((double)key_to_float(sh.key[i]) / T - xmax);
      if (acc >= need) {
        cand = i;
        break;
      }
    }
    if (cand == 0x7FFFFFFF) cand = p1 - 1;
  }
  const int j = block_min_i<NT>(cand, sh.redi);
  if (j == 0x7FFFFFFF || !(key_to_float(sh.key[j]) > cut)) {  // the nucleus may reach past the candidates
    if (tid == 0) mg_write(a, row, -1, 0.0f, MS_ROW_UNSUPPORTED);
    return;
  }
  const int nkeep = j + 1;
  // kept entries in index order (position = kept entries of smaller id)
  for (int i = tid; i < nkeep; i += NT) {
    const int my = sh.id[i];
    int pos = 0;
    for (int q = 0; q < nkeep; ++q) pos += sh.id[q] < my ? 1 : 0;
    sh.kid[pos] = my;
    sh.u.kw[pos] = exp((double)key_to_float(sh.key[i]) / T - xmax);
  }
  __syncthreads();
  // index-order inverse CDF over the kept entries (sampler.py:58-68)
  double s2 = 0.0;
  const int q0 = tid * ((nkeep + NT - 1) / NT);
  const int q1 = min(nkeep, q0 + (nkeep + NT - 1) / NT);
  for (int i = q0; i < q1; ++i) s2 += sh.u.kw[i];
  double cx, ci2, tot;
  block_scan<NT, double>(s2, cx, ci2, tot, sh.redd);
  if (!(U > 0.0)) {  // r == 0 stops at index 0
    if (tid == 0) mg_write(a, row, 0, (float)((sh.kid[0] == 0 ? sh.u.kw[0] : 0.0) / tot), 0);
    return;
  }
  const double target = U * tot;
  int who = 0x7FFFFFFF;
  if (q0 < q1 && ci2 >= target) {
    double acc = cx;
    for (int i = q0; i < q1; ++i) {
      acc += sh.u.kw[i];
      if (sh.u.kw[i] > 0.0 && acc >= target) {
        who = i;
        break;
      }
    }
    if (who == 0x7FFFFFFF) who = q1 - 1;
  }
  const int w = block_min_i<NT>(who, sh.redi);
  if (tid == 0) {
    if (w == 0x7FFFFFFF) {  // ran past the end (sampler.py:68)
      mg_write(a, row, a.V - 1, (float)((sh.kid[nkeep - 1] == a.V - 1 ? sh.u.kw[nkeep - 1] : 0.0) / tot), 0);
    } else {
      mg_write(a, row, sh.kid[w], (float)(sh.u.kw[w] / tot), 0);
    }
  }
}

// One row's merge: all NT threads of the CTA.
template <int NT>
__device__ __forceinline__ void mg_row(const MergeArgs &a, MgShared &sh, int row) {
  const int tid = threadIdx.x;
  const size_t rw = (size_t)(4 + 2 * a.kmax);
  const double T = a.temperature[row];
  const int k = a.top_k[row];
  const double P = a.top_p[row];
  const double U = a.uniforms[row];
  // per-rank counts -> offsets; statuses OR-ed
  int m_r = 0;
  uint32_t st_r = 0u;
  if (tid < a.nranks) {
    const uint32_t *rec = mg_rec(a, tid, row, rw);
    m_r = (int)min(mg_ld(rec), (uint32_t)a.kmax);
    st_r = mg_ld(rec + 1);
  }
  if (tid == 0) sh.st = 0u;
  __syncthreads();
  if (st_r) atomicOr(&sh.st, st_r);
  int ex, inc, n;
  block_scan<NT, int>(m_r, ex, inc, n, sh.redi);  // ends with a barrier
  if (tid < a.nranks) {
    sh.off[tid] = ex;
    sh.cnt[tid] = m_r;
  }
  const uint32_t st = sh.st;
  if (st != 0u) {  // bad temperature, or a slice that needs the full row
    if (tid == 0) mg_write(a, row, -1, 0.0f, (int32_t)st);
    return;
  }
  __syncthreads();
  // every (rank, slot) pair at once: the loads of all ranks' records in flight together
  const int KM = a.kmax;
#pragma unroll 4
  for (int j = tid; j < a.nranks * KM; j += NT) {
    const int r = j / KM, i = j - r * KM;
    if (i < sh.cnt[r]) {
      const uint32_t *rec = mg_rec(a, r, row, rw);
      sh.u.comp[sh.off[r] + i] =
          ((unsigned long long)mg_ld(rec + 2 + i) << 32) | (unsigned long long)(~mg_ld(rec + 2 + KM + i));
    }
  }
  if (tid == 0) {
    sh.u.comp[n] = 0ull;
    sh.u.comp[n + 1] = 0ull;
  }
  __syncthreads();
  if (n == 0) {  // every logit -inf
    if (tid == 0) {
      if (T == 0.0) mg_write(a, row, 0, 1.0f, 0);            // greedy ties at index 0 (sampler.py:33-34)
      else mg_write(a, row, -1, 0.0f, MS_ROW_ALL_MASKED);    // zero total (sampler.py:46-47)
    }
    return;
  }
  if (T == 0.0 || k == 1) {  // the first maximum (sampler.py:33-34, or top-k 1)
    unsigned long long best = 0ull;
    for (int i = tid; i < n; i += NT) best = max(best, sh.u.comp[i]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) best = max(best, __shfl_xor_sync(0xFFFFFFFFu, best, o));
    if ((tid & 31) == 0) sh.redq[tid >> 5] = best;
    __syncthreads();
    if (tid == 0) {
      for (int w = 1; w < NT / 32; ++w) best = max(best, sh.redq[w]);
      const int64_t id = (int64_t)(~(uint32_t)best);
      if (T == 0.0 || U > 0.0) mg_write(a, row, id, 1.0f, 0);
      else mg_write(a, row, 0, id == 0 ? 1.0f : 0.0f, 0);  // r == 0 stops at index 0
    }
    return;
  }
  if (!(k >= 2 && (int64_t)k < a.V)) {  // no top-k: the nucleus from the candidates
    mg_nucleus<NT>(a, sh, row, n, rw, T, P, U);
    return;
  }
  // top-k: rank every candidate; the best min(n, k) are the row's top-k set
  const int m = min(n, k);
  if (a.nranks >= 4) {
    // many ranks: each rank's run comp[off[r], off[r+1]) is sorted (value
    // descending, id ascending), so a candidate's rank is its place in its
    // own run plus a binary search in every other run
    const int N = a.nranks;
    for (int i = tid; i < n; i += NT) {
      int r = 0;
      while (r + 1 < N && sh.off[r + 1] <= i) ++r;
      const unsigned long long ci = sh.u.comp[i];
      int rank = i - sh.off[r];
      for (int r2 = 0; r2 < N && rank < m; ++r2) {
        if (r2 == r) continue;
        const int base = sh.off[r2];
        int lo = base, hi = r2 + 1 < N ? sh.off[r2 + 1] : n;
        while (lo < hi) {
          const int mid = (lo + hi) >> 1;
          if (sh.u.comp[mid] > ci) lo = mid + 1;
          else hi = mid;
        }
        rank += lo - base;
      }
      if (rank < m) {
        sh.key[rank] = (uint32_t)(ci >> 32);
        sh.id[rank] = (int)~(uint32_t)ci;
      }
    }
  } else {
    const ulonglong2 *c2 = reinterpret_cast<const ulonglong2 *>(sh.u.comp);
    const int npair = (n + 1) >> 1;
    for (int i = tid; i < n; i += NT) {
      const unsigned long long ci = sh.u.comp[i];
      int rank = 0;
      for (int j = 0; j < npair; ++j) {
        const ulonglong2 q = c2[j];
        rank += (q.x > ci ? 1 : 0) + (q.y > ci ? 1 : 0);
      }
      if (rank < m) {
        sh.key[rank] = (uint32_t)(ci >> 32);
        sh.id[rank] = (int)~(uint32_t)ci;
      }
    }
  }
  __syncthreads();
  // float64 weights over the top-k set (sampler.py:35,45): thread r, rank r
  const double xmax = (double)key_to_float(sh.key[0]) / T;
  const double w = tid < m ? exp((double)key_to_float(sh.key[tid]) / T - xmax) : 0.0;
  double wex, winc, total;
  block_scan<NT, double>(w, wex, winc, total, sh.redd);
  int nkeep = m;
  if (P < 1.0) {  // smallest rank prefix reaching top_p, crossing entry kept (sampler.py:49-58)
    const int first = block_min_i<NT>((tid < m && winc >= P * total) ? tid : 0x7FFFFFFF, sh.redi);
    if (first != 0x7FFFFFFF) nkeep = first + 1;
  }
  // kept entries in index order
  if (tid < nkeep) {
    const int my = sh.id[tid];
    int pos = 0;
    for (int j = 0; j < nkeep; ++j) pos += sh.id[j] < my ? 1 : 0;
    sh.kid[pos] = my;
    sh.u.kw[pos] = w;
  }
  const double tot = block_sum<NT>(tid < nkeep ? w : 0.0, sh.redd);  // ends with a barrier
  // index-order inverse CDF (sampler.py:60-68)
  if (!(U > 0.0)) {  // r == 0 stops at index 0
    if (tid == 0) mg_write(a, row, 0, (float)((sh.kid[0] == 0 ? sh.u.kw[0] : 0.0) / tot), 0);
    return;
  }
  const double target = U * tot;
  const double kwv = tid < nkeep ? sh.u.kw[tid] : 0.0;
  double cex, cinc, ctot;
  block_scan<NT, double>(kwv, cex, cinc, ctot, sh.redd);
  const int who = block_min_i<NT>((tid < nkeep && kwv > 0.0 && cinc >= target) ? tid : 0x7FFFFFFF, sh.redi);
  if (tid == 0 && who == 0x7FFFFFFF) {  // ran past the end
    const int last = nkeep - 1;
    mg_write(a, row, a.V - 1, (float)((sh.kid[last] == a.V - 1 ? sh.u.kw[last] : 0.0) / tot), 0);
  }
  if (tid == who) mg_write(a, row, sh.kid[tid], (float)(kwv / tot), 0);
}

__global__ void __launch_bounds__(kMgThreads) ms_merge_kernel(MergeArgs a) {
  __shared__ MgShared sh;
  mg_row<kMgThreads>(a, sh, blockIdx.x);
}

}  // namespace ms
