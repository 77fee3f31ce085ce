// Vocab-sharded rows without top-k that the candidate records cannot settle
// (miniserve/sampler.py:35-68 with top_k off): a nucleus wider than the
// candidates, or top_p >= 1 (the draw over the whole vocabulary).  No logits
// cross ranks; five kernels and three small collectives, all ranks taking the
// same steps:
//
//   1. ms_nu_hist_kernel (every rank, its slice): an x-grid histogram of the
//      row's weights, anchored at the row maximum M from the records,
//      fixed-point; the caller all-reduces (sum) the histograms.
//   2. ms_nu_bracket_kernel (every rank, identical inputs): the bins
//      [b_lo, b_hi] that must hold the top-p crossing, whatever the
//      histogram's rounding.
//   3. ms_nu_classify_kernel (every rank, its slice): the slice's weight
//      above the bracket and in all (float64), and the bracket's entries
//      (order key, global id); the caller all-gathers them.
//   4. ms_nu_cut_kernel (every rank, identical inputs): the entries ranked by
//      (value desc, id asc), the crossing entry (the first whose running mass
//      from the mass above reaches top_p of the total, kept), each rank's kept
//      mass, and the rank whose slice holds the index-order draw's target.
//   5. ms_nu_draw_kernel (the owning rank): the index-order draw over the
//      kept tokens of its slice; the caller all-reduces (max) the results.
//
// Every weight is one fp32 function of the logit, W(v) = 2^(v*cw - M*cw),
// cw = log2(e)/T, the same in every kernel and on every rank, so the totals,
// the cut and the draw agree with each other; the rounding against the
// reference's float64 exp is the 1e-6 band of the parity rule.
#pragma once

#include <cfloat>

#include "ms_common.cuh"

namespace ms {

constexpr int kNuThreads = 1024;
constexpr int kNuBins = 16384;                     // bins per kNuRange units of (M - v) / T
constexpr double kNuRange = 20.0;                  // beyond: the tail (weights below e^-20 of the maximum)
constexpr int kNuCap = 2048;                       // bracket entries one rank reports for a row
constexpr int kNuSortCap = 16384;                  // bracket entries of all ranks the cut ranks
constexpr int kNuRecWords = 5 + 2 * kNuCap;        // classify record: above f64, total f64, count, keys, ids
constexpr int kNuCutWords = 8;                     // cut record
constexpr int kNuSegs = 1024;                      // index-order segments of a slice (the draw)
constexpr int64_t kNuMaxSlice = (int64_t)1 << 20;  // longest slice
constexpr int kMaxNuRanks = 256;
constexpr int kNuStatusOk = 0;
constexpr int kNuStatusFallback = 1;               // the row needs the full-row path

// The per-slice inputs of kernels 1, 3 and 5.
struct NuSlice {
  const void *logits;
  int64_t Vloc;
  int64_t ld;
  int64_t v0;
  const uint32_t *mask;
  int64_t mask_ld;
};

// The flagged rows and what every kernel reads about them.
struct NuRows {
  const int32_t *rows;  // [F] batch rows
  int F;
  int B;
  const uint32_t *records;  // all-gathered [nranks][B][4 + 2*kmax]
  int nranks;
  int kmax;
  const double *temperature;
  const double *top_p;
  const double *uniforms;
};

// The row's maximum over all slices: the first key of every non-empty record.
__device__ __forceinline__ float nu_row_max(const NuRows &q, int row) {
  const size_t rw = (size_t)(4 + 2 * q.kmax);
  float m = -INFINITY;
  for (int r = 0; r < q.nranks; ++r) {
    const uint32_t *rec = q.records + ((size_t)r * q.B + row) * rw;
    if (rec[0] > 0u) m = fmaxf(m, key_to_float(rec[2]));
  }
  return m;
}

__device__ __forceinline__ float nu_ex2(float z) {
  float r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(z));
  return r;
}

struct NuW {
  float M, cw, aw, xs;
  __device__ __forceinline__ void set(float m, double T) {
    M = m;
    const double cl = 1.4426950408889634 / T;
    cw = (float)cl;
    aw = m * cw;
    xs = (float)((double)kNuBins / (kNuRange * T));
  }
  __device__ __forceinline__ float w(float v) const { return nu_ex2(fmaf(v, cw, -aw)); }  // -inf weighs 0
  // histogram bin of v <= M: floor((M - v) * xs), kNuBins for the tail (and -inf)
  __device__ __forceinline__ int bin(float v) const {
    const float t = (M - v) * xs;
    return t < (float)kNuBins ? (int)t : kNuBins;
  }
};

// Every value of the slice's row, in index order within each thread's share:
// fn(v, i) for v the logit (bf16 widened, -inf when masked).  16-byte loads
// over the aligned body, single loads for the unaligned head and the tail.
template <int DT, class Fn>
__device__ __forceinline__ void nu_for_each(const NuSlice &s, int row, Fn fn) {
  constexpr int esz = DT == MS_DTYPE_F32 ? 4 : 2;
  constexpr int vec = 16 / esz;  // values per 16-byte load
  const char *base = reinterpret_cast<const char *>(s.logits) + (size_t)row * s.ld * esz;
  const uint32_t *mrow = s.mask ? s.mask + (size_t)row * s.mask_ld : nullptr;
  auto allowed = [&](int64_t i) { return !mrow || ((__ldg(mrow + (i >> 5)) >> (i & 31)) & 1u); };
  const int64_t head = (int64_t)(((16 - (reinterpret_cast<uintptr_t>(base) & 15)) & 15) / esz);
  const int64_t h = head < s.Vloc ? head : s.Vloc;
  const int64_t nvec = (s.Vloc - h) / vec;
  const int tid = threadIdx.x;
  if (tid < h) fn(allowed(tid) ? __uint_as_float(raw_bits<DT>(base, tid)) : -INFINITY, (int64_t)tid);
  const uint4 *body = reinterpret_cast<const uint4 *>(base + h * esz);
  for (int64_t k = tid; k < nvec; k += kNuThreads) {
    const uint4 u = __ldg(body + k);
    const int64_t i0 = h + k * vec;
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int j = 0; j < vec; ++j) {
      const uint32_t bits = DT == MS_DTYPE_F32 ? w[j] : (j & 1 ? w[j >> 1] & 0xFFFF0000u : w[j >> 1] << 16);
      fn(allowed(i0 + j) ? __uint_as_float(bits) : -INFINITY, i0 + j);
    }
  }
  for (int64_t i = h + nvec * vec + tid; i < s.Vloc; i += kNuThreads)
    fn(allowed(i) ? __uint_as_float(raw_bits<DT>(base, (int)i)) : -INFINITY, i);
}

__device__ __forceinline__ bool nu_row_ok(double T) { return T >= 1e-30 && !isinf(T); }

// Histogram scale: every value of a bin adds round(scale * its weight
// relative to the bin's upper edge) <= scale, so the sum over all Vg values
// of the row, on one rank or all, stays below 2^31 (int32 all-reduce).
__device__ __forceinline__ float nu_hist_scale(int64_t Vg) {
  const int64_t sc = (int64_t)0x7FFFFFFF / (Vg > 0 ? Vg : 1);
  return (float)(sc < 65535 ? sc : 65535);
}

// 1. Histogram of the slice's weights (rows with top_p < 1).  Bin b covers
// (M - v) / T in [b, b + 1) * kNuRange / kNuBins; a value adds
// round(scale * e^-((t - b) * dz)) (t its bin coordinate, dz the bin width),
// its weight relative to e^-(b * dz), so bin b carries mass
// e^-(b * dz) * hist[b] / scale relative to the row maximum.
template <int DT>
__global__ void __launch_bounds__(kNuThreads) ms_nu_hist_kernel(NuSlice s, NuRows q, int64_t Vg, uint32_t *hist) {
  extern __shared__ uint32_t nu_h[];  // kNuBins
  const int f = blockIdx.x, tid = threadIdx.x;
  const int row = q.rows[f];
  for (int i = tid; i < kNuBins; i += kNuThreads) nu_h[i] = 0u;
  const double T = q.temperature[row], P = q.top_p[row];
  const float M = nu_row_max(q, row);
  __syncthreads();
  if (P < 1.0 && M > -INFINITY && nu_row_ok(T)) {  // block-uniform
    NuW W;
    W.set(M, T);
    const float scale = nu_hist_scale(Vg);
    const float c2 = (float)(-kNuRange / kNuBins * 1.4426950408889634);  // -dz * log2(e)
    nu_for_each<DT>(s, row, [&](float v, int64_t) {
      const float t = (M - v) * W.xs;  // -inf and the tail: t >= kNuBins
      if (t < (float)kNuBins) {
        const int b = (int)t;
        atomicAdd(&nu_h[b], (uint32_t)__float2uint_rn(scale * nu_ex2((t - (float)b) * c2)));
      }
    });
  }
  __syncthreads();
  for (int i = tid; i < kNuBins; i += kNuThreads) hist[(size_t)f * kNuBins + i] = nu_h[i];
}

// 2. The bracket [b_lo, b_hi] of the summed histogram.  With C(b) the
// histogram's mass in bins <= b and Z its total, every value's share is
// within 0.51 / scale + 1e-5 of its exact weight (relative: the rounding of
// the share, and of the fp32 bin coordinate and exponents), so the exact
// crossing bin -- the first whose exact running mass reaches top_p of the
// exact total -- lies at or after the first bin with C(b) > P*Z - tol and at
// or before the first with C(b) >= P*Z + tol (the tail bin kNuBins when none),
// tol = 2 * (0.51 / scale + 1e-5) * Z.  Rows with top_p >= 1 keep every
// value: the bracket lies past the tail.
__global__ void __launch_bounds__(kNuThreads) ms_nu_bracket_kernel(const uint32_t *hist, NuRows q, int64_t Vg,
                                                                  int32_t *bracket) {
  __shared__ double red[33];
  __shared__ int redi[33];
  const int f = blockIdx.x, tid = threadIdx.x;
  const int row = q.rows[f];
  const double P = q.top_p[row];
  if (!(P < 1.0)) {
    if (tid == 0) {
      bracket[2 * f] = kNuBins + 1;
      bracket[2 * f + 1] = kNuBins + 1;
    }
    return;
  }
  constexpr int per = kNuBins / kNuThreads;  // consecutive bins per thread
  const double dz = kNuRange / kNuBins;
  const uint32_t *h = hist + (size_t)f * kNuBins + tid * per;
  double loc[per];
  double sm = 0.0;
  const double e0 = exp(-(double)(tid * per) * dz), step = exp(-dz);
  double e = e0;
#pragma unroll
  for (int j = 0; j < per; ++j) {
    loc[j] = e * (double)h[j];
    sm += loc[j];
    e *= step;
  }
  double ex, inc, tot;
  block_scan<kNuThreads, double>(sm, ex, inc, tot, red);
  const double scale = (double)nu_hist_scale(Vg);
  const double tol = 2.0 * (0.51 / scale + 1e-5) * tot;
  const double lo_need = P * tot - tol, hi_need = P * tot + tol;
  int lo = 0x7FFFFFFF, hi = 0x7FFFFFFF;
  double c = ex;
#pragma unroll
  for (int j = 0; j < per; ++j) {
    c += loc[j];
    if (lo == 0x7FFFFFFF && c > lo_need) lo = tid * per + j;
    if (hi == 0x7FFFFFFF && c >= hi_need) hi = tid * per + j;
  }
  lo = block_min_i<kNuThreads>(lo, redi);
  hi = block_min_i<kNuThreads>(hi, redi);
  if (tid == 0) {
    bracket[2 * f] = lo == 0x7FFFFFFF ? kNuBins : lo;
    bracket[2 * f + 1] = hi == 0x7FFFFFFF ? kNuBins : hi;
  }
}

// Values per index-order segment of a slice (a multiple of 8, so that every
// segment starts on a 16-byte boundary of an aligned row).
__device__ __forceinline__ int64_t nu_seg_len(int64_t Vloc) {
  const int64_t S = (Vloc + kNuSegs - 1) / kNuSegs;
  return (S + 7) & ~(int64_t)7;
}

// Slice value i of the row (bf16 widened), -inf when masked.
template <int DT>
__device__ __forceinline__ float nu_val(const char *base, const uint32_t *mrow, int64_t i) {
  if (mrow && !((__ldg(mrow + (i >> 5)) >> (i & 31)) & 1u)) return -INFINITY;
  return __uint_as_float(raw_bits<DT>(base, (int)i));
}

// 3. The slice's weight above the bracket (bins < b_lo) and in all, and the
// bracket's entries: record [above f64][total f64][count][keys][ids], count
// kNuCap + 1 when the bracket holds more than kNuCap of the slice's values.
// Also, for the draw, the weight above the bracket of each of kNuSegs
// index-order segments of the slice (segments[f][s], rank-local).  Warp w
// takes segments w, w + 32, ...; its lanes read a segment 32 values apart,
// eight loads in flight.
template <int DT>
__global__ void __launch_bounds__(kNuThreads) ms_nu_classify_kernel(NuSlice s, NuRows q, const int32_t *bracket,
                                                                   uint32_t *out, double *segments) {
  __shared__ double redd[33];
  __shared__ int cnt;
  const int f = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int row = q.rows[f];
  const double T = q.temperature[row];
  const float M = nu_row_max(q, row);
  const int b_lo = bracket[2 * f], b_hi = bracket[2 * f + 1];
  uint32_t *rec = out + (size_t)f * kNuRecWords;
  double *seg = segments + (size_t)f * kNuSegs;
  if (tid == 0) cnt = 0;
  __syncthreads();
  double above = 0.0, total = 0.0;
  const bool live = M > -INFINITY && nu_row_ok(T);  // block-uniform
  constexpr int esz = DT == MS_DTYPE_F32 ? 4 : 2;
  const char *base = reinterpret_cast<const char *>(s.logits) + (size_t)row * s.ld * esz;
  const uint32_t *mrow = s.mask ? s.mask + (size_t)row * s.mask_ld : nullptr;
  const int64_t S = nu_seg_len(s.Vloc);  // values per segment
  NuW W;
  W.set(live ? M : 0.0f, live ? T : 1.0);
  double ga = 0.0;
  auto one = [&](float v, int64_t i) {
    if (!(v > -INFINITY)) return;
    const double w = (double)W.w(v);
    total += w;
    const int b = W.bin(v);
    if (b < b_lo) {
      ga += w;
    } else if (b <= b_hi) {
      const int pos = atomicAdd(&cnt, 1);
      if (pos < kNuCap) {
        rec[5 + pos] = fkey(v);
        rec[5 + kNuCap + pos] = (uint32_t)(s.v0 + i);
      }
    }
  };
  // 16-byte loads when the row starts on a 16-byte boundary (segments start
  // on whole vectors: S is a multiple of 8 values)
  constexpr int vec = 16 / esz;
  const bool vload = (reinterpret_cast<uintptr_t>(base) & 15u) == 0;
  for (int g = warp; g < kNuSegs; g += kNuThreads / 32) {
    const int64_t g0 = (int64_t)g * S, g1 = min(s.Vloc, g0 + S);
    ga = 0.0;
    if (live && vload) {
      for (int64_t i = g0 + (int64_t)lane * vec; i < g1; i += 32 * vec * 2) {
        uint4 u[2];
#pragma unroll
        for (int k = 0; k < 2; ++k) {
          const int64_t j = i + (int64_t)k * 32 * vec;
          u[k] = j + vec <= g1 ? __ldg(reinterpret_cast<const uint4 *>(base + j * esz)) : make_uint4(0, 0, 0, 0);
        }
#pragma unroll
        for (int k = 0; k < 2; ++k) {
          const int64_t j = i + (int64_t)k * 32 * vec;
          if (j + vec <= g1) {
            const uint32_t w4[4] = {u[k].x, u[k].y, u[k].z, u[k].w};
#pragma unroll
            for (int e = 0; e < vec; ++e) {
              const uint32_t bits = DT == MS_DTYPE_F32 ? w4[e] : (e & 1 ? w4[e >> 1] & 0xFFFF0000u : w4[e >> 1] << 16);
              const int64_t ie = j + e;
              one(mrow && !((__ldg(mrow + (ie >> 5)) >> (ie & 31)) & 1u) ? -INFINITY : __uint_as_float(bits), ie);
            }
          } else {
            for (int64_t ie = j; ie < g1; ++ie) one(nu_val<DT>(base, mrow, ie), ie);  // the row's ragged end
          }
        }
      }
    } else if (live) {
      for (int64_t i = g0 + lane; i < g1; i += 32 * 8) {
        float v8[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) v8[k] = i + 32 * k < g1 ? nu_val<DT>(base, mrow, i + 32 * k) : -INFINITY;
#pragma unroll
        for (int k = 0; k < 8; ++k) one(v8[k], i + 32 * k);
      }
    }
    above += ga;
    const double gs = warp_sum(ga);
    if (lane == 0) seg[g] = gs;
  }
  above = block_sum<kNuThreads>(above, redd);
  total = block_sum<kNuThreads>(total, redd);  // its barriers order cnt
  if (tid == 0) {
    const unsigned long long ab = (unsigned long long)__double_as_longlong(above);
    const unsigned long long tb = (unsigned long long)__double_as_longlong(total);
    rec[0] = (uint32_t)ab;
    rec[1] = (uint32_t)(ab >> 32);
    rec[2] = (uint32_t)tb;
    rec[3] = (uint32_t)(tb >> 32);
    rec[4] = (uint32_t)min(cnt, kNuCap + 1);
  }
}

__device__ __forceinline__ double nu_f64(const uint32_t *w) {
  return __longlong_as_double((long long)((unsigned long long)w[0] | ((unsigned long long)w[1] << 32)));
}

struct NuCut {  // the cut record, identical on every rank
  uint32_t key;   // kept: key > key, or key == key and global id <= id
  int32_t id;
  int32_t owner;  // rank whose slice holds the draw's target
  int32_t status;
  double residual;  // the target's offset into the owner's kept mass
  double total;     // the kept mass of the row
};

__device__ __forceinline__ void nu_put_cut(uint32_t *c, const NuCut &x) {
  c[0] = x.key;
  c[1] = (uint32_t)x.id;
  c[2] = (uint32_t)x.owner;
  c[3] = (uint32_t)x.status;
  const unsigned long long r = (unsigned long long)__double_as_longlong(x.residual);
  const unsigned long long t = (unsigned long long)__double_as_longlong(x.total);
  reinterpret_cast<unsigned long long *>(c)[2] = r;
  reinterpret_cast<unsigned long long *>(c)[3] = t;
}

__device__ __forceinline__ NuCut nu_get_cut(const uint32_t *c) {
  NuCut x;
  x.key = c[0];
  x.id = (int32_t)c[1];
  x.owner = (int32_t)c[2];
  x.status = (int32_t)c[3];
  x.residual = __longlong_as_double((long long)reinterpret_cast<const unsigned long long *>(c)[2]);
  x.total = __longlong_as_double((long long)reinterpret_cast<const unsigned long long *>(c)[3]);
  return x;
}

struct NuCutShared {
  unsigned long long comp[kNuSortCap];  // (key, ~id), sorted descending
  double kr[kMaxNuRanks];               // kept mass per rank
  int off[kMaxNuRanks + 1];
  double redd[33];
  int redi[33];
  int bad;
};

// 4. The cut, each rank's kept mass and the owner of the draw's target.
// entries: all-gathered classify records [nranks][F][kNuRecWords]; bounds:
// the slices' first global ids [nranks + 1].
__global__ void __launch_bounds__(kNuThreads) ms_nu_cut_kernel(const uint32_t *entries, const int64_t *bounds,
                                                              const int32_t *bracket, NuRows q, uint32_t *cut) {
  extern __shared__ __align__(16) unsigned char nu_raw[];
  NuCutShared &sh = *reinterpret_cast<NuCutShared *>(nu_raw);
  const int f = blockIdx.x, tid = threadIdx.x;
  const int row = q.rows[f];
  const double T = q.temperature[row], P = q.top_p[row], U = q.uniforms[row];
  const float M = nu_row_max(q, row);
  const int R = q.nranks;
  NuCut res;
  res.key = kNegInfKey + 1u;  // every finite value kept
  res.id = 0x7FFFFFFF;
  res.owner = 0;
  res.status = kNuStatusOk;
  res.residual = 0.0;
  res.total = 0.0;
  // per-rank counts -> offsets (thread 0: at most kMaxNuRanks ranks)
  if (tid == 0) {
    int n = 0, bad = (M > -INFINITY && nu_row_ok(T)) ? 0 : 1;
    for (int r = 0; r < R; ++r) {
      const uint32_t *rec = entries + ((size_t)r * q.F + f) * kNuRecWords;
      const int c = (int)rec[4];
      if (c > kNuCap) bad = 1;
      sh.off[r] = n;
      n += min(c, kNuCap);
    }
    sh.off[R] = n;
    if (n > kNuSortCap) bad = 1;
    sh.bad = bad;
  }
  __syncthreads();
  if (sh.bad) {
    if (tid == 0) {
      res.status = kNuStatusFallback;
      nu_put_cut(cut + (size_t)f * kNuCutWords, res);
    }
    return;
  }
  const int n = sh.off[R];
  int np2 = 1;
  while (np2 < n) np2 <<= 1;
  for (int r = 0; r < R; ++r) {
    const uint32_t *rec = entries + ((size_t)r * q.F + f) * kNuRecWords;
    const int c = sh.off[r + 1] - sh.off[r];
    for (int i = tid; i < c; i += kNuThreads)
      sh.comp[sh.off[r] + i] = ((unsigned long long)rec[5 + i] << 32) | (unsigned long long)(~rec[5 + kNuCap + i]);
  }
  for (int i = n + tid; i < np2; i += kNuThreads) sh.comp[i] = 0ull;
  __syncthreads();
  // bitonic sort, descending: (value desc, id asc) since ids are stored inverted
  for (int k = 2; k <= np2; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = tid; i < np2; i += kNuThreads) {
        const int l = i ^ j;
        if (l > i) {
          const unsigned long long a = sh.comp[i], b = sh.comp[l];
          const bool desc = (i & k) == 0;
          if (desc ? (a < b) : (a > b)) {
            sh.comp[i] = b;
            sh.comp[l] = a;
          }
        }
      }
      __syncthreads();
    }
  }
  NuW W;
  W.set(M, T);
  // above and total over ranks, in rank order (every thread, same order)
  double A = 0.0, Z = 0.0;
  for (int r = 0; r < R; ++r) {
    const uint32_t *rec = entries + ((size_t)r * q.F + f) * kNuRecWords;
    A += nu_f64(rec);
    Z += nu_f64(rec + 2);
  }
  // the crossing entry: a contiguous block of ranks per thread
  const int per = (n + kNuThreads - 1) / kNuThreads;
  const int p0 = min(n, tid * per), p1 = min(n, p0 + per);
  int ncut = n;  // entries kept (a prefix of the ranking)
  if (P < 1.0) {
    double sw = 0.0;
    for (int i = p0; i < p1; ++i) sw += (double)W.w(key_to_float((uint32_t)(sh.comp[i] >> 32)));
    double ex, inc, tot;
    block_scan<kNuThreads, double>(sw, ex, inc, tot, sh.redd);
    const double need = P * Z;
    int cand = 0x7FFFFFFF;
    if (p0 < p1 && A + inc >= need) {  // sampler.py:54-57: cumsum >= top_p, crossing entry kept
      double acc = A + ex;
      for (int i = p0; i < p1; ++i) {
        acc += (double)W.w(key_to_float((uint32_t)(sh.comp[i] >> 32)));
        if (acc >= need) {
          cand = i;
          break;
        }
      }
      if (cand == 0x7FFFFFFF) cand = p1 - 1;
    }
    const int j = block_min_i<kNuThreads>(cand, sh.redi);
    // the crossing above the bracket, or below it while values lie below it:
    // the histogram missed it (the full-row path takes the row)
    if (A >= need || (j == 0x7FFFFFFF && bracket[2 * f + 1] < kNuBins)) {
      if (tid == 0) {
        res.status = kNuStatusFallback;
        nu_put_cut(cut + (size_t)f * kNuCutWords, res);
      }
      return;
    }
    if (j == 0x7FFFFFFF) {
      ncut = n;  // the running sum never reaches top_p: every value kept
    } else {
      ncut = j + 1;
      res.key = (uint32_t)(sh.comp[j] >> 32);
      res.id = (int32_t)~(uint32_t)sh.comp[j];
    }
  }
  // kept mass per rank: above (the slice's total when every value is kept)
  // plus its kept entries, each rank's partials reduced in a fixed order
  for (int r = 0; r < R; ++r) {
    double part = 0.0;
    if (P < 1.0) {
      const int64_t lo = bounds[r], hi = bounds[r + 1];
      for (int i = p0; i < min(p1, ncut); ++i) {
        const int64_t id = (int64_t)~(uint32_t)sh.comp[i];
        if (id >= lo && id < hi) part += (double)W.w(key_to_float((uint32_t)(sh.comp[i] >> 32)));
      }
    }
    const double s = block_sum<kNuThreads>(part, sh.redd);
    if (tid == 0) {
      const uint32_t *rec = entries + ((size_t)r * q.F + f) * kNuRecWords;
      sh.kr[r] = (P < 1.0 ? nu_f64(rec) : nu_f64(rec + 2)) + s;
    }
  }
  __syncthreads();
  if (tid == 0) {
    double K = 0.0;
    for (int r = 0; r < R; ++r) K += sh.kr[r];
    res.total = K;
    // index-order inverse CDF over the slices in rank order (sampler.py:60-68)
    const double target = U * K;
    double pre = 0.0;
    int owner = -1;
    for (int r = 0; r < R; ++r) {
      if (pre + sh.kr[r] >= target && (sh.kr[r] > 0.0 || !(U > 0.0))) {
        owner = r;
        break;
      }
      pre += sh.kr[r];
    }
    if (owner < 0) {  // ran past the end (sampler.py:68): the last token
      res.owner = R - 1;
      res.residual = INFINITY;
    } else {
      res.owner = owner;
      res.residual = target - pre;
    }
    if (!(K > 0.0)) res.status = kNuStatusFallback;
    nu_put_cut(cut + (size_t)f * kNuCutWords, res);
  }
}

// 5. The draw on the owning rank (sampler.py:62-66: the first value whose
// running kept mass reaches the target, r <= cumulative).  A segment's kept
// mass is its weight above the bracket (the classifying pass) plus its kept
// bracket entries (this rank's record; summed as 2^-50 fixed point, exact
// and order-free); a scan of the kNuSegs segment masses picks the segment
// holding the residual target, and one warp walks that segment 32 values at
// a time.  out[f] = (token, float bits of its probability), (-1, 0) on the
// other ranks, so a max all-reduce gives every rank the owner's answer.
template <int DT>
__global__ void __launch_bounds__(kNuThreads) ms_nu_draw_kernel(NuSlice s, NuRows q, const uint32_t *cut,
                                                               const uint32_t *entries, const double *segments,
                                                               int rank, int64_t *out) {
  __shared__ unsigned long long fix[kNuSegs];
  __shared__ double redd[33];
  __shared__ int redi[33];
  __shared__ double seg_base;
  const int f = blockIdx.x, tid = threadIdx.x, lane = tid & 31;
  const int row = q.rows[f];
  const NuCut c = nu_get_cut(cut + (size_t)f * kNuCutWords);
  if (c.owner != rank || c.status != kNuStatusOk) {
    if (tid == 0) {
      out[2 * f] = -1;
      out[2 * f + 1] = 0;
    }
    return;
  }
  constexpr int esz = DT == MS_DTYPE_F32 ? 4 : 2;
  const char *base = reinterpret_cast<const char *>(s.logits) + (size_t)row * s.ld * esz;
  const uint32_t *mrow = s.mask ? s.mask + (size_t)row * s.mask_ld : nullptr;
  NuW W;
  W.set(nu_row_max(q, row), q.temperature[row]);
  auto kept = [&](uint32_t key, int64_t gid) { return key > c.key || (key == c.key && gid <= (int64_t)c.id); };
  auto kwv = [&](float v, int64_t i) -> double {  // the kept weight of value v at slice index i
    if (!(v > -INFINITY)) return 0.0;
    return kept(fkey(v), s.v0 + i) ? (double)W.w(v) : 0.0;
  };
  const int64_t S = nu_seg_len(s.Vloc);
  for (int g = tid; g < kNuSegs; g += kNuThreads) fix[g] = 0ull;
  __syncthreads();
  // this rank's kept bracket entries, per segment
  const uint32_t *rec = entries + ((size_t)rank * q.F + f) * kNuRecWords;
  const int n = (int)min(rec[4], (uint32_t)kNuCap);
  for (int e = tid; e < n; e += kNuThreads) {
    const uint32_t key = rec[5 + e];
    const int64_t gid = (int64_t)rec[5 + kNuCap + e];
    if (kept(key, gid)) {
      const double w = (double)W.w(key_to_float(key));
      atomicAdd(&fix[(gid - s.v0) / S], (unsigned long long)(w * 1125899906842624.0));  // 2^50
    }
  }
  __syncthreads();
  const int g = tid;  // kNuSegs == kNuThreads: one segment per thread
  const double mine = segments[(size_t)f * kNuSegs + g] + (double)fix[g] * (1.0 / 1125899906842624.0);
  double ex, inc, tot;
  block_scan<kNuThreads, double>(mine, ex, inc, tot, redd);
  const int gs = block_min_i<kNuThreads>((inc >= c.residual) ? g : 0x7FFFFFFF, redi);
  if (gs == 0x7FFFFFFF) {  // ran past the end (sampler.py:68): the slice's last value
    if (tid == 0) {
      const float v = nu_val<DT>(base, mrow, s.Vloc - 1);
      out[2 * f] = s.v0 + s.Vloc - 1;
      out[2 * f + 1] = (int64_t)__float_as_uint((float)(kwv(v, s.Vloc - 1) / c.total));
    }
    return;
  }
  if (g == gs) seg_base = ex;
  __syncthreads();
  if (tid >= 32) return;
  double acc = seg_base;
  const int64_t lo = (int64_t)gs * S, hi = min(s.Vloc, lo + S);
  for (int64_t i0 = lo; i0 < hi; i0 += 32) {
    const int64_t i = i0 + lane;
    const double x = i < hi ? kwv(nu_val<DT>(base, mrow, i), i) : 0.0;
    double incl = x;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const double y = __shfl_up_sync(0xFFFFFFFFu, incl, o);
      if (lane >= o) incl += y;
    }
    const unsigned hit = __ballot_sync(0xFFFFFFFFu, i < hi && acc + incl >= c.residual);
    if (hit) {
      const int l = __ffs(hit) - 1;
      const double wl = __shfl_sync(0xFFFFFFFFu, x, l);
      if (lane == 0) {
        out[2 * f] = s.v0 + i0 + l;
        out[2 * f + 1] = (int64_t)__float_as_uint((float)(wl / c.total));
      }
      return;
    }
    acc += __shfl_sync(0xFFFFFFFFu, incl, 31);
  }
  if (lane == 0) {  // rounding carried the target past the segment: its last value
    const float v = nu_val<DT>(base, mrow, hi - 1);
    out[2 * f] = s.v0 + hi - 1;
    out[2 * f + 1] = (int64_t)__float_as_uint((float)(kwv(v, hi - 1) / c.total));
  }
}

}  // namespace ms
