// Fused peer exchange of vocab-sharded sampling: the candidate records of
// every rank cross NVLink as plain peer stores from the streaming kernel
// itself into per-rank exchange buffers (one cudaMalloc per rank, mapped
// into the other ranks by CUDA IPC), in place of an all-gather between the
// streaming kernel and the merge.
//
// Every 8-byte store carries one record word and the call's epoch (high
// half): an aligned 8-byte store is seen whole or not at all, so a reader
// that finds the epoch finds the word, and the writer needs no fence and
// never waits.  The merge on each rank waits (bounded) for the epochs of
// the row's words from every other rank.
//
// Exchange buffer layout (32-bit words; Bcap rows, nranks ranks, records of
// at most Wcap = 4 + 2 kmax_cap words; the same in every rank's buffer):
//   [rec0, +2 half)   two plain record areas, [nranks][B][W] each (the
//                     layout of an all-gather of ms_shard_candidates'
//                     records): this rank's own records from the streaming
//                     kernel, the other ranks' unpacked by the merge
//   [ll0, +2 llhalf)  two areas of tagged words (8 bytes each), [B][nranks][W]
//                     the other ranks store into
//   [res0, +2 reshalf) two areas of tagged results, [B][4] 8-byte words
//                     (token, prob bits, status, unused): row r is merged
//                     on rank r mod nranks, which stores its result into
//                     every rank's area
// Call `epoch` uses the areas (epoch & 1).
#pragma once

#include <cstdint>

#include "ms_common.cuh"
#include "ms_shard.cuh"

namespace ms {

constexpr int kXThreads = 256;

// One call of the fused exchange on one rank: peers[q] is rank q's exchange
// buffer (peers[rank] this rank's own); ll: word offset of the call's tagged
// area, the same in every buffer.
struct XArgs {
  uint32_t *const *peers;
  int rank;
  int n;
  uint32_t epoch;
  int64_t ll;
};

struct XLayout {
  int64_t rec0, half, ll0, llhalf, res0, reshalf, total;
};

__host__ __device__ inline int64_t x_round32(int64_t w) { return (w + 31) / 32 * 32; }

__host__ __device__ inline XLayout x_layout(int64_t Bcap, int nranks, int kmax_cap) {
  XLayout L;
  const int64_t words = (int64_t)nranks * Bcap * (4 + 2 * (int64_t)kmax_cap);
  L.rec0 = 0;
  L.half = x_round32(words);
  L.ll0 = 2 * L.half;
  L.llhalf = x_round32(2 * words);
  L.res0 = L.ll0 + 2 * L.llhalf;
  L.reshalf = x_round32(8 * Bcap);
  L.total = L.res0 + 2 * L.reshalf;
  return L;
}

__device__ __forceinline__ void x_st_relaxed_sys(unsigned long long *p, unsigned long long v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ unsigned long long x_ld_relaxed_sys(const unsigned long long *p) {
  unsigned long long v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ uint64_t x_now_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// The merge on every rank, one CTA per row: the other ranks' tagged words
// of the row are waited for (each at most timeout_ns after the CTA starts)
// and unpacked into the plain record area (`plain`, the call's
// [nranks][B][W]; every row, so the distributed nucleus finds every record);
// then the row's owner (row mod nranks) merges it as ms_merge_kernel does,
// with the result going to every rank (a.xpeers) or, on one rank, straight
// to the outputs.  A row with a word missing at the timeout: its owner
// reports token -1, MS_ROW_PEER_TIMEOUT.  Only other GPUs' kernels can still
// be storing while it waits: this rank's own streaming kernel ran to
// completion before it on the stream.
__global__ void __launch_bounds__(kMgThreads) ms_xmerge_kernel(MergeArgs a, uint32_t *plain,
                                                              const unsigned long long *ll, int me, uint32_t epoch,
                                                              int64_t timeout_ns) {
  __shared__ MgShared sh;
  const int row = blockIdx.x, N = a.nranks, W = 4 + 2 * a.kmax;
  const unsigned long long *src = ll + (size_t)row * N * W;
  int ok = 1;
  const uint64_t t0 = x_now_ns();
  for (int j = threadIdx.x; j < N * W && ok; j += kMgThreads) {
    const int r = j / W;
    if (r == me) continue;
    unsigned long long v = x_ld_relaxed_sys(src + j);
    while ((uint32_t)(v >> 32) != epoch) {
      if ((int64_t)(x_now_ns() - t0) > timeout_ns) {
        ok = 0;
        break;
      }
      __nanosleep(32);
      v = x_ld_relaxed_sys(src + j);
    }
    plain[((size_t)r * a.B + row) * W + (j - r * W)] = (uint32_t)v;
  }
  const bool all = __syncthreads_and(ok);
  if (row % N != me) return;
  if (!all) {
    if (threadIdx.x == 0) mg_write(a, row, -1, 0.0f, MS_ROW_PEER_TIMEOUT);
    return;
  }
  mg_row<kMgThreads>(a, sh, row);
}

// After the merge, on every rank of more than one: each row's tagged result
// from its owner (waited for at most timeout_ns) into the outputs; a row
// without one: token -1, MS_ROW_PEER_TIMEOUT.
__global__ void __launch_bounds__(kXThreads) ms_xresult_kernel(const unsigned long long *res, int B, uint32_t epoch,
                                                              int64_t timeout_ns, int64_t *tokens, float *probs,
                                                              int32_t *status) {
  const int r = blockIdx.x * kXThreads + threadIdx.x;
  if (r >= B) return;
  const unsigned long long *e = res + 4 * (size_t)r;
  unsigned long long v[3];
  bool ok = true;
  const uint64_t t0 = x_now_ns();
  for (int j = 0; j < 3 && ok; ++j) {
    v[j] = x_ld_relaxed_sys(e + j);
    while ((uint32_t)(v[j] >> 32) != epoch) {
      if ((int64_t)(x_now_ns() - t0) > timeout_ns) {
        ok = false;
        break;
      }
      __nanosleep(32);
      v[j] = x_ld_relaxed_sys(e + j);
    }
  }
  if (ok) {
    tokens[r] = (int64_t)(int32_t)(uint32_t)v[0];
    probs[r] = __uint_as_float((uint32_t)v[1]);
    status[r] = (int32_t)(uint32_t)v[2];
  } else {
    tokens[r] = -1;
    probs[r] = 0.0f;
    status[r] = MS_ROW_PEER_TIMEOUT;
  }
}

}  // namespace ms
