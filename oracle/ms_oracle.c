/*
 * CPU oracle for the token-sampling path -- TEST INFRASTRUCTURE ONLY.
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg load
 * this library, and only as the checker.  The product path is the CUDA
 * library libmssample.so.
 *
 * A plain-C restatement of miniserve's Sampler.sample
 * (miniserve/sampler.py:23-68) with the same float64 steps, so that on the
 * same machine (same libm exp) it returns bit-identical tokens and
 * probabilities to the Python reference:
 *   - greedy: first maximal index                       sampler.py:33-34
 *   - scaled = logit / T (IEEE division)                sampler.py:35
 *   - top-k: stable descending sort, first k kept       sampler.py:37-42
 *   - softmax with CPython 3.12 compensated sum()       sampler.py:44-47
 *   - top-p: stable sort of probs, sequential cumsum,
 *     first element reaching top_p included, renorm     sampler.py:49-60
 *   - index-order inverse CDF, fallback V-1             sampler.py:62-68
 * The allowed-token bitmask (bit set = allowed) turns a disallowed logit into
 * -inf first, the -inf convention of the logits-processor hook
 * (miniserve/model_runner.py:214, tests/test_parity.py:324-327).
 *
 * Rows run in parallel on `nthreads` POSIX threads; each row is sequential.
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define MSO_ROW_OK 0
#define MSO_ROW_ALL_MASKED 1
#define MSO_ROW_BAD_TEMPERATURE 2
#define MSO_ROW_NONFINITE 4

typedef struct {
  const void *logits;
  int dtype; /* 0 = fp32, 1 = bf16 (raw uint16 bits) */
  int64_t B, V, ld;
  const double *T;
  const int32_t *k;
  const double *p;
  const double *u;
  const uint32_t *mask;
  int64_t mask_ld;
  int64_t *tok;
  double *prob;
  int32_t *status;
  double *margin_p;
  double *margin_u;
  int64_t next_row;
  pthread_mutex_t lock;
} job_t;

typedef struct {
  double v;
  int64_t i;
} vi_t;

/* descending by value, ascending index on ties == Python's stable reverse sort */
static int cmp_desc(const void *a, const void *b) {
  const vi_t *x = (const vi_t *)a, *y = (const vi_t *)b;
  if (x->v > y->v) return -1;
  if (x->v < y->v) return 1;
  return (x->i < y->i) ? -1 : (x->i > y->i);
}

/* CPython 3.12 builtins.sum over floats (Neumaier compensation). */
static double py_sum(const double *x, int64_t n) {
  double s = 0.0, c = 0.0;
  for (int64_t j = 0; j < n; ++j) {
    double t = s + x[j];
    if (fabs(s) >= fabs(x[j]))
      c += (s - t) + x[j];
    else
      c += (x[j] - t) + s;
    s = t;
  }
  if (c != 0.0 && isfinite(c)) s += c;
  return s;
}

static double load_logit(const job_t *J, int64_t b, int64_t i) {
  if (J->dtype == 0) return (double)((const float *)J->logits)[b * J->ld + i];
  uint16_t h = ((const uint16_t *)J->logits)[b * J->ld + i];
  uint32_t w = (uint32_t)h << 16;
  float f;
  memcpy(&f, &w, 4);
  return (double)f;
}

static void sample_one(job_t *J, int64_t b, double *vals, double *work, vi_t *order) {
  const int64_t n = J->V;
  double T = J->T[b], top_p = J->p[b], u = J->u[b];
  int32_t top_k = J->k[b];
  double mp = INFINITY, mu = INFINITY;
  int32_t st = MSO_ROW_OK;
  for (int64_t i = 0; i < n; ++i) {
    double v = load_logit(J, b, i);
    if (J->mask && !((J->mask[b * J->mask_ld + (i >> 5)] >> (i & 31)) & 1u)) v = -INFINITY;
    if (isnan(v) || v == INFINITY) st |= MSO_ROW_NONFINITE;
    vals[i] = v;
  }
  if (T == 0.0) {
    int64_t best = 0;
    for (int64_t i = 1; i < n; ++i)
      if (vals[i] > vals[best]) best = i;
    J->tok[b] = best;
    J->prob[b] = 1.0;
    J->status[b] = st;
    J->margin_p[b] = mp;
    J->margin_u[b] = mu;
    return;
  }
  if (!(T > 0.0) || isinf(T)) {
    J->tok[b] = -1;
    J->prob[b] = 0.0;
    J->status[b] = st | MSO_ROW_BAD_TEMPERATURE;
    J->margin_p[b] = mp;
    J->margin_u[b] = mu;
    return;
  }
  double *scaled = vals; /* in place: l / T */
  for (int64_t i = 0; i < n; ++i) scaled[i] = scaled[i] / T;
  if (top_k > 0) {
    for (int64_t i = 0; i < n; ++i) {
      order[i].v = scaled[i];
      order[i].i = i;
    }
    qsort(order, (size_t)n, sizeof(vi_t), cmp_desc);
    int64_t kk = top_k < n ? top_k : n;
    for (int64_t i = 0; i < n; ++i) work[i] = -INFINITY;
    for (int64_t j = 0; j < kk; ++j) work[order[j].i] = scaled[order[j].i];
    memcpy(scaled, work, (size_t)n * sizeof(double));
  }
  double max_v = scaled[0];
  for (int64_t i = 1; i < n; ++i)
    if (scaled[i] > max_v) max_v = scaled[i];
  double *e = work;
  for (int64_t i = 0; i < n; ++i) e[i] = (scaled[i] != -INFINITY) ? exp(scaled[i] - max_v) : 0.0;
  double total = py_sum(e, n);
  if (total == 0.0) {
    J->tok[b] = -1;
    J->prob[b] = 0.0;
    J->status[b] = st | MSO_ROW_ALL_MASKED;
    J->margin_p[b] = mp;
    J->margin_u[b] = mu;
    return;
  }
  double *probs = vals;
  for (int64_t i = 0; i < n; ++i) probs[i] = e[i] / total;
  if (top_p < 1.0) {
    /* Zero probabilities sort last (index order) and cannot move the running
       sum, so only the positive ones need ordering. */
    int64_t m = 0;
    for (int64_t i = 0; i < n; ++i)
      if (probs[i] > 0.0) {
        order[m].v = probs[i];
        order[m].i = i;
        ++m;
      }
    qsort(order, (size_t)m, sizeof(vi_t), cmp_desc);
    double cumsum = 0.0, prev = 0.0;
    int64_t kept = m;
    int crossed = 0;
    for (int64_t j = 0; j < m; ++j) {
      prev = cumsum;
      cumsum += order[j].v;
      if (cumsum >= top_p) {
        kept = j + 1;
        crossed = 1;
        mp = fmin(cumsum - top_p, top_p - prev);
        break;
      }
    }
    if (!crossed) mp = top_p - cumsum;
    if (crossed) {
      /* keep = first `kept` of the order; everything else becomes 0 */
      for (int64_t i = 0; i < n; ++i) e[i] = 0.0;
      for (int64_t j = 0; j < kept; ++j) e[order[j].i] = probs[order[j].i];
      memcpy(probs, e, (size_t)n * sizeof(double));
    }
    double total2 = py_sum(probs, n);
    for (int64_t i = 0; i < n; ++i) probs[i] = probs[i] / total2;
  }
  double cumulative = 0.0, prev = 0.0;
  for (int64_t i = 0; i < n; ++i) {
    prev = cumulative;
    cumulative += probs[i];
    if (u <= cumulative) {
      J->tok[b] = i;
      J->prob[b] = probs[i];
      J->status[b] = st;
      J->margin_p[b] = mp;
      J->margin_u[b] = fmin(cumulative - u, probs[i] > 0.0 ? u - prev : INFINITY);
      return;
    }
  }
  J->tok[b] = n - 1;
  J->prob[b] = probs[n - 1];
  J->status[b] = st;
  J->margin_p[b] = mp;
  J->margin_u[b] = u - cumulative;
}

static void *worker(void *arg) {
  job_t *J = (job_t *)arg;
  int64_t n = J->V;
  double *vals = (double *)malloc((size_t)n * sizeof(double));
  double *work = (double *)malloc((size_t)n * sizeof(double));
  vi_t *order = (vi_t *)malloc((size_t)n * sizeof(vi_t));
  if (!vals || !work || !order) {
    free(vals);
    free(work);
    free(order);
    return (void *)1;
  }
  for (;;) {
    pthread_mutex_lock(&J->lock);
    int64_t b = J->next_row++;
    pthread_mutex_unlock(&J->lock);
    if (b >= J->B) break;
    sample_one(J, b, vals, work, order);
  }
  free(vals);
  free(work);
  free(order);
  return NULL;
}

/* Returns 0 on success, -1 on bad arguments, -2 on allocation failure. */
int mso_sample(const void *logits, int dtype, int64_t B, int64_t V, int64_t ld, const double *T,
               const int32_t *k, const double *p, const double *u, const uint32_t *mask,
               int64_t mask_ld, int64_t *tok, double *prob, int32_t *status, double *margin_p,
               double *margin_u, int nthreads) {
  if (!logits || B < 0 || V < 1 || ld < V || (dtype != 0 && dtype != 1) || !T || !k || !p || !u ||
      !tok || !prob || !status || !margin_p || !margin_u)
    return -1;
  if (mask && mask_ld < (V + 31) / 32) return -1;
  job_t J = {logits, dtype, B, V, ld, T, k, p, u, mask, mask_ld, tok, prob, status, margin_p, margin_u,
             0, PTHREAD_MUTEX_INITIALIZER};
  if (nthreads < 1) nthreads = 1;
  if (nthreads > 256) nthreads = 256;
  pthread_t th[256];
  int started = 0, rc = 0;
  for (int t = 0; t < nthreads; ++t) {
    if (pthread_create(&th[t], NULL, worker, &J) != 0) break;
    ++started;
  }
  if (started == 0) rc = (int)(intptr_t)worker(&J) ? -2 : 0;
  for (int t = 0; t < started; ++t) {
    void *r = NULL;
    pthread_join(th[t], &r);
    if (r) rc = -2;
  }
  return rc;
}

/* exported for the summation check against the interpreter's sum() */
double mso_py_sum(const double *x, int64_t n) { return py_sum(x, n); }
