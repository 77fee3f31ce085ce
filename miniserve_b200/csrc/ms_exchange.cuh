// Fused peer exchange of vocab-sharded sampling: the candidate records of
// every rank and the merged results move over NVLink as plain peer stores
// into per-rank exchange buffers (one cudaMalloc per rank, mapped into the
// other ranks by CUDA IPC), with system-scope counters in place of the
// all-gather of ms_shard_candidates / ms_shard_merge.
//
// Exchange buffer layout (32-bit words; Bcap rows, nranks ranks, records of
// at most Wcap = 4 + 2 kmax_cap words; the same in every rank's buffer):
//   [0, 32)           done counter (u64 at word 0): one count per merged row,
//                     added by the merging CTA on every rank
//   [cnt, +2 Bcap)    per-row arrival counters (u64), used on the row's home
//                     rank (row mod nranks); one count per rank's record
//   [out, +4 Bcap)    result entries {token, prob bits, status, epoch}
//   [rec0, +2 half)   two record areas, [nranks][B][W] each (the layout of
//                     an all-gather of ms_shard_candidates' records); call
//                     `epoch` uses area (epoch & 1)
// Counters only grow: a row's arrival count is a multiple of nranks between
// calls, so the arrival that makes it one again is the last of its call.
#pragma once

#include <cstdint>

#include "ms_common.cuh"

namespace ms {

constexpr int kXThreads = 256;

// One call of the fused exchange on one rank: peers[q] is rank q's exchange
// buffer (peers[rank] this rank's own); cnt, out and rec are word offsets,
// the same in every buffer (rec: the call's record area).
struct XArgs {
  uint32_t *const *peers;
  int rank;
  int n;
  uint32_t epoch;
  int64_t cnt;
  int64_t out;
  int64_t rec;
};

struct XLayout {
  int64_t cnt, out, rec0, half, total;
};

__host__ __device__ inline int64_t x_round32(int64_t w) { return (w + 31) / 32 * 32; }

__host__ __device__ inline XLayout x_layout(int64_t Bcap, int nranks, int kmax_cap) {
  XLayout L;
  L.cnt = 32;
  L.out = L.cnt + x_round32(2 * Bcap);
  L.rec0 = L.out + x_round32(4 * Bcap);
  L.half = x_round32((int64_t)nranks * Bcap * (4 + 2 * (int64_t)kmax_cap));
  L.total = L.rec0 + 2 * L.half;
  return L;
}

__device__ __forceinline__ unsigned long long x_atom_add_acq_rel_sys(unsigned long long *p, unsigned long long v) {
  unsigned long long old;
  asm volatile("atom.acq_rel.sys.global.add.u64 %0, [%1], %2;" : "=l"(old) : "l"(p), "l"(v) : "memory");
  return old;
}

__device__ __forceinline__ void x_red_add_release_sys(unsigned long long *p, unsigned long long v) {
  asm volatile("red.release.sys.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ unsigned long long x_ld_acquire_sys(const unsigned long long *p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ uint64_t x_now_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// The last step on every rank: wait until this buffer's done counter reaches
// `target` (the rows of every call so far), at most timeout_ns, then copy the
// call's result entries out.  An entry without this call's epoch (a rank or
// its merge missing at the timeout) gives token -1, MS_ROW_PEER_TIMEOUT.
__global__ void __launch_bounds__(kXThreads) ms_xfinish_kernel(const uint32_t *xbuf, int64_t out, int B,
                                                              unsigned long long target, uint32_t epoch,
                                                              int64_t timeout_ns, int64_t *tokens, float *probs,
                                                              int32_t *status) {
  if (threadIdx.x == 0) {
    const unsigned long long *done = reinterpret_cast<const unsigned long long *>(xbuf);
    const uint64_t t0 = x_now_ns();
    while ((long long)(x_ld_acquire_sys(done) - target) < 0) {
      if ((int64_t)(x_now_ns() - t0) > timeout_ns) break;
      __nanosleep(64);
    }
  }
  __syncthreads();
  for (int r = blockIdx.x * kXThreads + threadIdx.x; r < B; r += gridDim.x * kXThreads) {
    const uint4 e = __ldcg(reinterpret_cast<const uint4 *>(xbuf + out) + r);
    if (e.w == epoch) {
      tokens[r] = (int64_t)(int32_t)e.x;
      probs[r] = __uint_as_float(e.y);
      status[r] = (int32_t)e.z;
    } else {
      tokens[r] = -1;
      probs[r] = 0.0f;
      status[r] = MS_ROW_PEER_TIMEOUT;
    }
  }
}

}  // namespace ms
