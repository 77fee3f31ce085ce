// Fused peer exchange of vocab-sharded sampling: the candidate records of
// every rank cross NVLink as plain peer stores from the streaming kernel
// itself into per-rank exchange buffers (one cudaMalloc per rank, mapped
// into the other ranks by CUDA IPC), in place of an all-gather between the
// streaming kernel and the merge.
//
// Exchange buffer layout (32-bit words; Bcap rows, nranks ranks, records of
// at most Wcap = 4 + 2 kmax_cap words; the same in every rank's buffer):
//   [flags, +Bcap*nranks)  arrival flags [row][rank]: the epoch of the last
//                          call whose record of that row from that rank is
//                          in this buffer
//   [rec0, +2 half)        two record areas, [nranks][B][W] each (the layout
//                          of an all-gather of ms_shard_candidates' records);
//                          call `epoch` uses area (epoch & 1)
// A rank stores its record of a row into every buffer, then (one release
// fence later) its flag of that row in every buffer.  The merge on each rank
// waits, row by row and for a bounded time, until the row's flags from
// every rank carry the call's epoch.
#pragma once

#include <cstdint>

#include "ms_common.cuh"
#include "ms_shard.cuh"

namespace ms {

// One call of the fused exchange on one rank: peers[q] is rank q's exchange
// buffer (peers[rank] this rank's own); flags and rec are word offsets, the
// same in every buffer (rec: the call's record area).
struct XArgs {
  uint32_t *const *peers;
  int rank;
  int n;
  uint32_t epoch;
  int64_t flags;
  int64_t rec;
};

struct XLayout {
  int64_t flags, rec0, half, total;
};

__host__ __device__ inline int64_t x_round32(int64_t w) { return (w + 31) / 32 * 32; }

__host__ __device__ inline XLayout x_layout(int64_t Bcap, int nranks, int kmax_cap) {
  XLayout L;
  L.flags = 0;
  L.rec0 = x_round32(Bcap * nranks);
  L.half = x_round32((int64_t)nranks * Bcap * (4 + 2 * (int64_t)kmax_cap));
  L.total = L.rec0 + 2 * L.half;
  return L;
}

__device__ __forceinline__ void x_fence_acq_rel_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }

__device__ __forceinline__ void x_st_relaxed_sys(uint32_t *p, uint32_t v) {
  asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t x_ld_acquire_sys(const uint32_t *p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ uint64_t x_now_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// The merge on every rank, one CTA per row: thread q waits (at most
// timeout_ns) for rank q's flag of the row, then the row is merged from this
// buffer's records as ms_merge_kernel does.  A row whose flags are not all
// there at the timeout: token -1, MS_ROW_PEER_TIMEOUT.  Only other GPUs'
// kernels can still be writing while it waits: this rank's own streaming
// kernel ran to completion before it on the stream.
__global__ void __launch_bounds__(kMgThreads) ms_xmerge_kernel(MergeArgs a, const uint32_t *flags, uint32_t epoch,
                                                              int64_t timeout_ns) {
  __shared__ MgShared sh;
  const int row = blockIdx.x;
  int ok = 1;
  if ((int)threadIdx.x < a.nranks) {
    const uint32_t *f = flags + (size_t)row * a.nranks + threadIdx.x;
    const uint64_t t0 = x_now_ns();
    while (x_ld_acquire_sys(f) != epoch) {
      if ((int64_t)(x_now_ns() - t0) > timeout_ns) {
        ok = 0;
        break;
      }
      __nanosleep(64);
    }
  }
  if (!__syncthreads_and(ok)) {
    if (threadIdx.x == 0) mg_write(a, row, -1, 0.0f, MS_ROW_PEER_TIMEOUT);
    return;
  }
  mg_row<kMgThreads>(a, sh, row);
}

}  // namespace ms
