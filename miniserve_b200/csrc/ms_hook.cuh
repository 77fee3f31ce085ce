// The logits-processor hook's mask: miniserve installs
// fn(logits[V], generated) -> logits[V] (miniserve/model_runner.py:166-168)
// whose convention is "disallowed token = -inf" before the argmax or the
// sampler (model_runner.py:214-216).  The sampler takes the allowed set as a
// bitmask instead; this kernel packs it from a hook's output: bit t of row b
// is set when processed[b, t] is not -inf.  Bandwidth-bound: one warp per
// 32-token word, a coalesced 128-byte (fp32) read and one ballot.
#pragma once

#include "ms_common.cuh"

namespace ms {

constexpr int kHookThreads = 256;
constexpr int kHookWordsPerCta = kHookThreads / 32;

template <int DT>
__global__ void __launch_bounds__(kHookThreads) ms_mask_from_logits_kernel(const void *logits, int64_t ld, int V,
                                                                         uint32_t *mask, int64_t mask_ld) {
  const int lane = threadIdx.x & 31;
  const int64_t b = blockIdx.y;
  const int64_t w = (int64_t)blockIdx.x * kHookWordsPerCta + (threadIdx.x >> 5);
  const int64_t words = ((int64_t)V + 31) / 32;
  if (w >= words) return;  // warp-uniform
  const int64_t t = w * 32 + lane;
  bool allowed = false;
  if (t < V) {
    const uint32_t u = raw_bits<DT>(reinterpret_cast<const char *>(logits) + b * ld * (DT == MS_DTYPE_F32 ? 4 : 2),
                                    (int)t);
    allowed = u != kNegInfBits;  // only -inf is disallowed (a NaN passes to the sampler, which flags it)
  }
  const uint32_t bits = __ballot_sync(0xFFFFFFFFu, allowed);
  if (lane == 0) mask[b * mask_ld + w] = bits;
}

}  // namespace ms
