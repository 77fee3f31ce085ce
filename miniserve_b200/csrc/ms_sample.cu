// libmssample.so -- C ABI of the B200 token sampler (declared in include/mssample.h).
//
// Reference semantics (miniserve/sampler.py, Sampler.sample):
//   :33-34  temperature == 0 -> first maximal index
//   :35     scaled = logit / T                     (here: exp((l - max) / T) in f64)
//   :37-42  top_k > 0: stable descending sort, first k kept, the rest -inf
//   :44-47  softmax over what is left (zero total -> ZeroDivisionError)
//   :49-60  top_p < 1: stable sort of probabilities, running sum, the element
//           that reaches top_p is kept, renormalise
//   :62-68  r = Random(seed).random(); first index (index order) whose running
//           probability reaches r; V-1 when none does
// The mask path applies the logits-processor hook's -inf convention
// (miniserve/model_runner.py:214) before all of the above.

#include <cuda_runtime.h>

#include <atomic>
#include <cstring>

#include "ms_common.cuh"
#include "ms_generic.cuh"
#include "ms_hook.cuh"
#include "ms_json.cuh"
#include "ms_exchange.cuh"
#include "ms_shard.cuh"
#include "ms_nucleus.cuh"
#include "ms_stream.cuh"

namespace {
thread_local int g_last_cuda_error = 0;

int cuda_fail(cudaError_t e) {
  g_last_cuda_error = (int)e;
  return MS_E_CUDA;
}

constexpr int kMaxDevices = 64;

// The streaming kernel alone: one CTA per row, or in pair mode B clusters of
// two CTAs.
template <int DT>
cudaError_t launch_stream(const ms::SampleArgs &a, int B, cudaStream_t s, int dev,
                          const ms::XArgs *x = nullptr) {
  static std::atomic<int> ready[kMaxDevices];
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  if (!ready[dev].load(std::memory_order_acquire)) {
    cudaError_t e = cudaFuncSetAttribute(ms::ms_stream_kernel<DT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)sizeof(ms::StShared));
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(ms::ms_stream_xkernel<DT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               (int)sizeof(ms::StShared));
    if (e != cudaSuccess) return e;
    ready[dev].store(1, std::memory_order_release);
  }
  if (x) {  // the fused peer exchange: one CTA per row
    ms::ms_stream_xkernel<DT><<<dim3((unsigned)B), dim3(ms::kStThreads), sizeof(ms::StShared), s>>>(a, *x);
    return cudaGetLastError();
  }
  if (!a.pairs) {
    ms::ms_stream_kernel<DT><<<dim3((unsigned)B), dim3(ms::kStThreads), sizeof(ms::StShared), s>>>(a);
    return cudaGetLastError();
  }
  // pair mode: B clusters of two CTAs, enough for every row to be a top-p row
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(2 * B));
  cfg.blockDim = dim3(ms::kStThreads);
  cfg.dynamicSmemBytes = sizeof(ms::StShared);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, ms::ms_stream_kernel<DT>, a);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

// The streaming kernel for every row it can finish, then the generic kernel
// for the rows it marked pending.
template <int DT>
cudaError_t launch_all(const ms::SampleArgs &a, int B, cudaStream_t s, int dev, bool generic_only) {
  if (generic_only || a.V > ms::kStreamMaxV) {
    ms::ms_generic_kernel<DT><<<dim3((unsigned)B), dim3(ms::kGenThreads), 0, s>>>(a, nullptr, nullptr);
    return cudaGetLastError();
  }
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  ms::SampleArgs ap = a;
  // top-p rows are shared by CTA pairs while they fit one wave (one cluster
  // per SM)
  ap.pairs = B <= (1 << 29) ? sms : 0;
  ap.rows = B;
  cudaError_t e = launch_stream<DT>(ap, B, s, dev);
  if (e != cudaSuccess) return e;
  const int grid = B < sms ? B : sms;
  // a programmatic dependent launch: the pending pass is launched while the
  // streaming kernel's last CTAs run and waits (griddepcontrol.wait) for that
  // grid's completion before it reads a status
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(ms::kGenThreads);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, ms::ms_generic_pending_kernel<DT>, a, B);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}
}  // namespace

extern "C" {

int ms_version(void) { return 100; }

int ms_last_cuda_error(void) { return g_last_cuda_error; }

const char *ms_error_string(int code) {
  switch (code) {
    case MS_OK: return "ok";
    case MS_E_INVALID: return "invalid argument (null pointer, B < 0, V < 1, V >= 2^31, ld < V or mask_ld too small)";
    case MS_E_DTYPE: return "unsupported dtype (expected MS_DTYPE_F32 or MS_DTYPE_BF16)";
    case MS_E_CUDA: return "CUDA error (see ms_last_cuda_error)";
    case MS_E_UNSUPPORTED: return "request outside what this build supports";
    case MS_E_TOO_LARGE: return "size beyond the fixed device array of the no-alloc entry point (V > 262144)";
    default: return "unknown error";
  }
}

static int sample_impl(const void *logits, int dtype, int64_t B, int64_t V, int64_t ld,
                       const double *temperature, const int32_t *top_k, const double *top_p,
                       const double *uniforms, const uint32_t *mask, int64_t mask_ld,
                       int64_t *tokens, float *probs, int32_t *row_status, ms_stream_t stream,
                       bool generic_only) {
  if (dtype != MS_DTYPE_F32 && dtype != MS_DTYPE_BF16) return MS_E_DTYPE;
  if (B < 0 || V < 1 || V > 0x7FFFFFFFll - 4096 || ld < V) return MS_E_INVALID;
  if (B > 0x7FFFFFFFll) return MS_E_INVALID;
  if (B == 0) return MS_OK;
  if (!logits || !temperature || !top_k || !top_p || !uniforms || !tokens || !probs || !row_status)
    return MS_E_INVALID;
  if (mask && mask_ld < (V + 31) / 32) return MS_E_INVALID;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  ms::SampleArgs a{logits, ld, (int)V, temperature, top_k, top_p, uniforms,
                   mask, mask_ld, tokens, probs, row_status};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e);
  e = dtype == MS_DTYPE_F32 ? launch_all<MS_DTYPE_F32>(a, (int)B, s, dev, generic_only)
                            : launch_all<MS_DTYPE_BF16>(a, (int)B, s, dev, generic_only);
  if (e != cudaSuccess) return cuda_fail(e);
  return MS_OK;
}

int ms_sample(const void *logits, int dtype, int64_t B, int64_t V, int64_t ld,
              const double *temperature, const int32_t *top_k, const double *top_p,
              const double *uniforms, const uint32_t *mask, int64_t mask_ld, int64_t *tokens,
              float *probs, int32_t *row_status, ms_stream_t stream) {
  return sample_impl(logits, dtype, B, V, ld, temperature, top_k, top_p, uniforms, mask, mask_ld,
                     tokens, probs, row_status, stream, false);
}

int ms_sample_generic(const void *logits, int dtype, int64_t B, int64_t V, int64_t ld,
                      const double *temperature, const int32_t *top_k, const double *top_p,
                      const double *uniforms, const uint32_t *mask, int64_t mask_ld,
                      int64_t *tokens, float *probs, int32_t *row_status, ms_stream_t stream) {
  return sample_impl(logits, dtype, B, V, ld, temperature, top_k, top_p, uniforms, mask, mask_ld,
                     tokens, probs, row_status, stream, true);
}

int ms_mask_from_logits(const void *logits, int dtype, int64_t B, int64_t V, int64_t ld, uint32_t *mask,
                        int64_t mask_ld, ms_stream_t stream) {
  if (dtype != MS_DTYPE_F32 && dtype != MS_DTYPE_BF16) return MS_E_DTYPE;
  if (B < 0 || B > 65535 || V < 1 || V > 0x7FFFFFFFll - 32 || ld < V || mask_ld < (V + 31) / 32) return MS_E_INVALID;
  if (B == 0) return MS_OK;
  if (!logits || !mask) return MS_E_INVALID;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int64_t words = (V + 31) / 32;
  const dim3 grid((unsigned)((words + ms::kHookWordsPerCta - 1) / ms::kHookWordsPerCta), (unsigned)B);
  if (dtype == MS_DTYPE_F32) {
    ms::ms_mask_from_logits_kernel<MS_DTYPE_F32><<<grid, ms::kHookThreads, 0, s>>>(logits, ld, (int)V, mask, mask_ld);
  } else {
    ms::ms_mask_from_logits_kernel<MS_DTYPE_BF16><<<grid, ms::kHookThreads, 0, s>>>(logits, ld, (int)V, mask, mask_ld);
  }
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? MS_OK : cuda_fail(e);
}

int64_t ms_shard_record_words(int32_t kmax) { return 4 + 2 * (int64_t)kmax; }

int ms_shard_candidates(const void *logits, int dtype, int64_t B, int64_t Vloc, int64_t ld, int64_t v0,
                        int64_t V, const double *temperature, const int32_t *top_k, const uint32_t *mask,
                        int64_t mask_ld, int32_t kmax, uint32_t *records, ms_stream_t stream) {
  if (dtype != MS_DTYPE_F32 && dtype != MS_DTYPE_BF16) return MS_E_DTYPE;
  if (B < 0 || B > 0x7FFFFFFFll || Vloc < 1 || ld < Vloc || v0 < 0 || V < v0 + Vloc ||
      V > 0x7FFFFFFFll - 4096 || kmax < 1 || kmax > ms::kMgTopK)
    return MS_E_INVALID;
  if (B == 0) return MS_OK;
  if (!logits || !temperature || !top_k || !records) return MS_E_INVALID;
  if (mask && mask_ld < (Vloc + 31) / 32) return MS_E_INVALID;
  if (Vloc > ms::kStreamMaxV) return MS_E_UNSUPPORTED;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  // top_p and the uniforms are not read in this mode; the temperature array
  // stands in for both pointers
  ms::SampleArgs a{logits, ld, (int)Vloc, temperature, top_k, temperature, temperature,
                   mask, mask_ld, nullptr, nullptr, nullptr};
  a.records = records;
  a.kmax = kmax;
  a.v0 = v0;
  a.Vg = V;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e);
  e = dtype == MS_DTYPE_F32 ? launch_stream<MS_DTYPE_F32>(a, (int)B, s, dev)
                            : launch_stream<MS_DTYPE_BF16>(a, (int)B, s, dev);
  if (e != cudaSuccess) return cuda_fail(e);
  return MS_OK;
}

int ms_shard_merge(const uint32_t *records, int32_t nranks, int64_t B, int32_t kmax, int64_t V,
                   const double *temperature, const int32_t *top_k, const double *top_p,
                   const double *uniforms, int64_t *tokens, float *probs, int32_t *row_status,
                   ms_stream_t stream) {
  if (B < 0 || B > 0x7FFFFFFFll || V < 1 || V > 0x7FFFFFFFll - 4096 || kmax < 1 || kmax > ms::kMgTopK ||
      nranks < 1)
    return MS_E_INVALID;
  if (nranks > ms::kMgRanks || (int64_t)nranks * kmax > ms::kMgCap) return MS_E_UNSUPPORTED;
  if (B == 0) return MS_OK;
  if (!records || !temperature || !top_k || !top_p || !uniforms || !tokens || !probs || !row_status)
    return MS_E_INVALID;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  ms::MergeArgs a{records, nranks, (int)B, kmax, V, temperature, top_k, top_p, uniforms,
                  tokens, probs, row_status};
  ms::ms_merge_kernel<<<dim3((unsigned)B), dim3(ms::kMgThreads), 0, s>>>(a);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e);
  return MS_OK;
}

int64_t ms_exchange_words(int64_t Bcap, int32_t nranks, int32_t kmax_cap) {
  if (Bcap < 1 || Bcap > (1 << 20) || nranks < 1 || nranks > ms::kMgRanks || kmax_cap < 1 ||
      kmax_cap > ms::kMgTopK)
    return -1;
  return ms::x_layout(Bcap, nranks, kmax_cap).total;
}

int64_t ms_exchange_records_offset(int64_t Bcap, int32_t nranks, int32_t kmax_cap, uint32_t epoch) {
  if (ms_exchange_words(Bcap, nranks, kmax_cap) < 0) return -1;
  const ms::XLayout L = ms::x_layout(Bcap, nranks, kmax_cap);
  return L.rec0 + (int64_t)(epoch & 1u) * L.half;
}

int ms_shard_exchange(const void *logits, int dtype, int64_t B, int64_t Vloc, int64_t ld, int64_t v0, int64_t V,
                      const double *temperature, const int32_t *top_k, const double *top_p, const double *uniforms,
                      const uint32_t *mask, int64_t mask_ld, int32_t kmax, uint32_t *xbuf, uint32_t *const *peers,
                      int32_t rank, int32_t nranks, int64_t Bcap, int32_t kmax_cap, uint32_t epoch,
                      ms_stream_t stream) {
  if (dtype != MS_DTYPE_F32 && dtype != MS_DTYPE_BF16) return MS_E_DTYPE;
  if (ms_exchange_words(Bcap, nranks, kmax_cap) < 0 || B < 0 || B > Bcap || Vloc < 1 || ld < Vloc || v0 < 0 ||
      V < v0 + Vloc || V > 0x7FFFFFFFll - 4096 || kmax < 1 || kmax > kmax_cap || rank < 0 || rank >= nranks ||
      epoch == 0u)
    return MS_E_INVALID;
  if ((int64_t)nranks * kmax > ms::kMgCap) return MS_E_UNSUPPORTED;
  if (B == 0) return MS_OK;
  if (!logits || !temperature || !top_k || !top_p || !uniforms || !xbuf || !peers) return MS_E_INVALID;
  if ((reinterpret_cast<uintptr_t>(xbuf) & 15u) != 0) return MS_E_INVALID;
  if (mask && mask_ld < (Vloc + 31) / 32) return MS_E_INVALID;
  if (Vloc > ms::kStreamMaxV) return MS_E_UNSUPPORTED;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const ms::XLayout L = ms::x_layout(Bcap, nranks, kmax_cap);
  const int64_t rec = L.rec0 + (int64_t)(epoch & 1u) * L.half;
  ms::SampleArgs a{logits, ld, (int)Vloc, temperature, top_k, top_p, uniforms,
                   mask, mask_ld, nullptr, nullptr, nullptr};
  a.records = xbuf + rec + (int64_t)rank * B * (4 + 2 * (int64_t)kmax);
  a.kmax = kmax;
  a.v0 = v0;
  a.Vg = V;
  a.rows = (int)B;
  const ms::XArgs x{peers, rank, nranks, epoch, L.ll0 + (int64_t)(epoch & 1u) * L.llhalf};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e);
  e = dtype == MS_DTYPE_F32 ? launch_stream<MS_DTYPE_F32>(a, (int)B, s, dev, &x)
                            : launch_stream<MS_DTYPE_BF16>(a, (int)B, s, dev, &x);
  if (e != cudaSuccess) return cuda_fail(e);
  return MS_OK;
}

int ms_exchange_merge(uint32_t *xbuf, uint32_t *const *peers, int32_t rank, int32_t nranks, int64_t B,
                      int64_t Bcap, int32_t kmax,
                      int32_t kmax_cap, int64_t V, const double *temperature, const int32_t *top_k,
                      const double *top_p, const double *uniforms, uint32_t epoch, int64_t timeout_ns,
                      int64_t *tokens, float *probs, int32_t *row_status, ms_stream_t stream) {
  if (ms_exchange_words(Bcap, nranks, kmax_cap) < 0 || B < 0 || B > Bcap || kmax < 1 || kmax > kmax_cap ||
      V < 1 || V > 0x7FFFFFFFll - 4096 || timeout_ns < 0 || epoch == 0u || rank < 0 || rank >= nranks)
    return MS_E_INVALID;
  if ((int64_t)nranks * kmax > ms::kMgCap) return MS_E_UNSUPPORTED;
  if (B == 0) return MS_OK;
  if (!xbuf || !peers || !temperature || !top_k || !top_p || !uniforms || !tokens || !probs || !row_status)
    return MS_E_INVALID;
  if ((reinterpret_cast<uintptr_t>(xbuf) & 15u) != 0) return MS_E_INVALID;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const ms::XLayout L = ms::x_layout(Bcap, nranks, kmax_cap);
  const int64_t res = L.res0 + (int64_t)(epoch & 1u) * L.reshalf;
  const int64_t rec = L.rec0 + (int64_t)(epoch & 1u) * L.half;
  ms::MergeArgs a{xbuf + rec, nranks, (int)B, kmax, V, temperature, top_k, top_p, uniforms,
                  tokens, probs, row_status};
  if (nranks > 1) {  // each row merged on its owner, the result stored into every rank's buffer
    a.xpeers = peers;
    a.xres = res;
    a.xepoch = epoch;
  }
  const unsigned long long *ll =
      reinterpret_cast<const unsigned long long *>(xbuf + L.ll0 + (int64_t)(epoch & 1u) * L.llhalf);
  ms::ms_xmerge_kernel<<<dim3((unsigned)B), dim3(ms::kMgThreads), 0, s>>>(a, xbuf + rec, ll, rank, epoch,
                                                                         timeout_ns);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e);
  return MS_OK;
}

int ms_exchange_results(const uint32_t *xbuf, int32_t nranks, int64_t B, int64_t Bcap, int32_t kmax_cap,
                        uint32_t epoch, int64_t timeout_ns, int64_t *tokens, float *probs, int32_t *row_status,
                        ms_stream_t stream) {
  if (ms_exchange_words(Bcap, nranks, kmax_cap) < 0 || B < 0 || B > Bcap || timeout_ns < 0 || epoch == 0u)
    return MS_E_INVALID;
  if (B == 0 || nranks == 1) return MS_OK;  // one rank: the merge wrote the outputs
  if (!xbuf || !tokens || !probs || !row_status) return MS_E_INVALID;
  if ((reinterpret_cast<uintptr_t>(xbuf) & 15u) != 0) return MS_E_INVALID;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const ms::XLayout L = ms::x_layout(Bcap, nranks, kmax_cap);
  const int64_t res = L.res0 + (int64_t)(epoch & 1u) * L.reshalf;
  const unsigned grid = (unsigned)((B + ms::kXThreads - 1) / ms::kXThreads);
  ms::ms_xresult_kernel<<<dim3(grid), dim3(ms::kXThreads), 0, s>>>(
      reinterpret_cast<const unsigned long long *>(xbuf + res), (int)B, epoch, timeout_ns, tokens, probs,
      row_status);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e);
  return MS_OK;
}

int ms_device_alloc(int64_t bytes, void **ptr) {
  if (!ptr || bytes < 1) return MS_E_INVALID;
  *ptr = nullptr;
  void *p = nullptr;
  cudaError_t e = cudaMalloc(&p, (size_t)bytes);
  if (e != cudaSuccess) return cuda_fail(e);
  e = cudaMemset(p, 0, (size_t)bytes);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    cudaFree(p);
    return cuda_fail(e);
  }
  *ptr = p;
  return MS_OK;
}

int ms_device_free(void *ptr) {
  if (!ptr) return MS_OK;
  cudaError_t e = cudaFree(ptr);
  return e == cudaSuccess ? MS_OK : cuda_fail(e);
}

int ms_ipc_handle(void *ptr, unsigned char *handle) {
  if (!ptr || !handle) return MS_E_INVALID;
  static_assert(sizeof(cudaIpcMemHandle_t) == 64, "64-byte IPC handle");
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, ptr);
  if (e != cudaSuccess) return cuda_fail(e);
  memcpy(handle, &h, sizeof(h));
  return MS_OK;
}

int ms_ipc_open(const unsigned char *handle, void **ptr) {
  if (!handle || !ptr) return MS_E_INVALID;
  *ptr = nullptr;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void *p = nullptr;
  cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return cuda_fail(e);
  *ptr = p;
  return MS_OK;
}

int ms_ipc_close(void *ptr) {
  if (!ptr) return MS_E_INVALID;
  cudaError_t e = cudaIpcCloseMemHandle(ptr);
  return e == cudaSuccess ? MS_OK : cuda_fail(e);
}

int64_t ms_nucleus_hist_words(void) { return ms::kNuBins; }
int64_t ms_nucleus_record_words(void) { return ms::kNuRecWords; }
int64_t ms_nucleus_cut_words(void) { return ms::kNuCutWords; }
int64_t ms_nucleus_segments(void) { return ms::kNuSegs; }

namespace {
// the dynamic shared memory of the histogram and cut kernels (once per device)
cudaError_t nucleus_attrs() {
  static std::atomic<int> ready[kMaxDevices];
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  if (ready[dev].load(std::memory_order_acquire)) return cudaSuccess;
  const int hbytes = ms::kNuBins * (int)sizeof(uint32_t);
  e = cudaFuncSetAttribute(ms::ms_nu_cut_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)sizeof(ms::NuCutShared));
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(ms::ms_nu_hist_kernel<MS_DTYPE_F32>, cudaFuncAttributeMaxDynamicSharedMemorySize, hbytes);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(ms::ms_nu_hist_kernel<MS_DTYPE_BF16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             hbytes);
  if (e == cudaSuccess) ready[dev].store(1, std::memory_order_release);
  return e;
}

int nucleus_check(int dtype, int64_t Vloc, int64_t ld, const uint32_t *mask, int64_t mask_ld, int64_t F, int64_t B,
                  int32_t nranks, int32_t kmax) {
  if (dtype != MS_DTYPE_F32 && dtype != MS_DTYPE_BF16) return MS_E_DTYPE;
  if (Vloc < 1 || ld < Vloc || F < 0 || F > 0x7FFFFFFFll || B < 1 || B > 0x7FFFFFFFll || nranks < 1 || kmax < 1 ||
      kmax > ms::kMgTopK)
    return MS_E_INVALID;
  if (mask && mask_ld < (Vloc + 31) / 32) return MS_E_INVALID;
  if (Vloc > ms::kNuMaxSlice || nranks > ms::kMaxNuRanks) return MS_E_UNSUPPORTED;
  return MS_OK;
}
}  // namespace

int ms_nucleus_hist(const void *logits, int dtype, int64_t Vloc, int64_t ld, const uint32_t *mask, int64_t mask_ld,
                    const int32_t *rows, int64_t F, int64_t B, int64_t V, const uint32_t *records, int32_t nranks,
                    int32_t kmax, const double *temperature, const double *top_p, uint32_t *hist,
                    ms_stream_t stream) {
  int rc = nucleus_check(dtype, Vloc, ld, mask, mask_ld, F, B, nranks, kmax);
  if (rc != MS_OK) return rc;
  if (V < Vloc) return MS_E_INVALID;
  if (V > 0x7FFFFFFFll / 16) return MS_E_UNSUPPORTED;  // the histogram scale stays >= 16
  if (F == 0) return MS_OK;
  if (!logits || !rows || !records || !temperature || !top_p || !hist) return MS_E_INVALID;
  cudaError_t e = nucleus_attrs();
  if (e != cudaSuccess) return cuda_fail(e);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const ms::NuSlice sl{logits, Vloc, ld, 0, mask, mask_ld};
  const ms::NuRows q{rows, (int)F, (int)B, records, nranks, kmax, temperature, top_p, nullptr};
  const size_t hb = (size_t)ms::kNuBins * sizeof(uint32_t);
  if (dtype == MS_DTYPE_F32) ms::ms_nu_hist_kernel<MS_DTYPE_F32><<<(unsigned)F, ms::kNuThreads, hb, s>>>(sl, q, V, hist);
  else ms::ms_nu_hist_kernel<MS_DTYPE_BF16><<<(unsigned)F, ms::kNuThreads, hb, s>>>(sl, q, V, hist);
  e = cudaGetLastError();
  return e == cudaSuccess ? MS_OK : cuda_fail(e);
}

int ms_nucleus_bracket(const uint32_t *hist, const int32_t *rows, int64_t F, int64_t V, const double *top_p,
                       int32_t *bracket, ms_stream_t stream) {
  if (F < 0 || F > 0x7FFFFFFFll || V < 1) return MS_E_INVALID;
  if (V > 0x7FFFFFFFll / 16) return MS_E_UNSUPPORTED;
  if (F == 0) return MS_OK;
  if (!hist || !rows || !top_p || !bracket) return MS_E_INVALID;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const ms::NuRows q{rows, (int)F, 0, nullptr, 0, 0, nullptr, top_p, nullptr};
  ms::ms_nu_bracket_kernel<<<(unsigned)F, ms::kNuThreads, 0, s>>>(hist, q, V, bracket);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? MS_OK : cuda_fail(e);
}

int ms_nucleus_classify(const void *logits, int dtype, int64_t Vloc, int64_t ld, int64_t v0, const uint32_t *mask,
                        int64_t mask_ld, const int32_t *rows, int64_t F, int64_t B, const uint32_t *records,
                        int32_t nranks, int32_t kmax, const double *temperature, const int32_t *bracket,
                        uint32_t *entries, double *segments, ms_stream_t stream) {
  int rc = nucleus_check(dtype, Vloc, ld, mask, mask_ld, F, B, nranks, kmax);
  if (rc != MS_OK) return rc;
  if (v0 < 0 || v0 + Vloc > 0x7FFFFFFFll) return MS_E_INVALID;
  if (F == 0) return MS_OK;
  if (!logits || !rows || !records || !temperature || !bracket || !entries || !segments) return MS_E_INVALID;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const ms::NuSlice sl{logits, Vloc, ld, v0, mask, mask_ld};
  const ms::NuRows q{rows, (int)F, (int)B, records, nranks, kmax, temperature, nullptr, nullptr};
  if (dtype == MS_DTYPE_F32)
    ms::ms_nu_classify_kernel<MS_DTYPE_F32><<<(unsigned)F, ms::kNuThreads, 0, s>>>(sl, q, bracket, entries,
                                                                                  segments);
  else
    ms::ms_nu_classify_kernel<MS_DTYPE_BF16><<<(unsigned)F, ms::kNuThreads, 0, s>>>(sl, q, bracket, entries,
                                                                                   segments);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? MS_OK : cuda_fail(e);
}

int ms_nucleus_cut(const uint32_t *entries, int32_t nranks, const int64_t *bounds, const int32_t *bracket,
                   const int32_t *rows, int64_t F, int64_t B, const uint32_t *records, int32_t kmax,
                   const double *temperature, const double *top_p, const double *uniforms, uint32_t *cut,
                   ms_stream_t stream) {
  if (F < 0 || F > 0x7FFFFFFFll || B < 1 || B > 0x7FFFFFFFll || nranks < 1 || kmax < 1 || kmax > ms::kMgTopK)
    return MS_E_INVALID;
  if (nranks > ms::kMaxNuRanks) return MS_E_UNSUPPORTED;
  if (F == 0) return MS_OK;
  if (!entries || !bounds || !bracket || !rows || !records || !temperature || !top_p || !uniforms || !cut)
    return MS_E_INVALID;
  cudaError_t e = nucleus_attrs();
  if (e != cudaSuccess) return cuda_fail(e);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const ms::NuRows q{rows, (int)F, (int)B, records, nranks, kmax, temperature, top_p, uniforms};
  ms::ms_nu_cut_kernel<<<(unsigned)F, ms::kNuThreads, sizeof(ms::NuCutShared), s>>>(entries, bounds, bracket, q,
                                                                                    cut);
  e = cudaGetLastError();
  return e == cudaSuccess ? MS_OK : cuda_fail(e);
}

int ms_nucleus_draw(const void *logits, int dtype, int64_t Vloc, int64_t ld, int64_t v0, const uint32_t *mask,
                    int64_t mask_ld, const int32_t *rows, int64_t F, int64_t B, const uint32_t *records,
                    int32_t nranks, int32_t kmax, const double *temperature, const uint32_t *cut,
                    const uint32_t *entries, const double *segments, int32_t rank, int64_t *out,
                    ms_stream_t stream) {
  int rc = nucleus_check(dtype, Vloc, ld, mask, mask_ld, F, B, nranks, kmax);
  if (rc != MS_OK) return rc;
  if (v0 < 0 || v0 + Vloc > 0x7FFFFFFFll || rank < 0 || rank >= nranks) return MS_E_INVALID;
  if (F == 0) return MS_OK;
  if (!logits || !rows || !records || !temperature || !cut || !entries || !segments || !out) return MS_E_INVALID;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const ms::NuSlice sl{logits, Vloc, ld, v0, mask, mask_ld};
  const ms::NuRows q{rows, (int)F, (int)B, records, nranks, kmax, temperature, nullptr, nullptr};
  if (dtype == MS_DTYPE_F32)
    ms::ms_nu_draw_kernel<MS_DTYPE_F32><<<(unsigned)F, ms::kNuThreads, 0, s>>>(sl, q, cut, entries, segments, rank,
                                                                              out);
  else
    ms::ms_nu_draw_kernel<MS_DTYPE_BF16><<<(unsigned)F, ms::kNuThreads, 0, s>>>(sl, q, cut, entries, segments, rank,
                                                                               out);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? MS_OK : cuda_fail(e);
}

int64_t ms_json_state_words(void) { return ms::kJsonStateWords; }

int ms_json_init(const uint8_t *prefix_bytes, const int64_t *prefix_off, int64_t B, uint32_t *states,
                 ms_stream_t stream) {
  if (B < 0) return MS_E_INVALID;
  if (B == 0) return MS_OK;
  if (!prefix_bytes || !prefix_off || !states) return MS_E_INVALID;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const unsigned grid = (unsigned)((B + 127) / 128);
  ms::ms_json_feed_kernel<<<grid, 128, 0, s>>>(states, B, prefix_bytes, prefix_off, B, nullptr, 1);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? MS_OK : cuda_fail(e);
}

int ms_json_advance(uint32_t *states, int64_t B, const uint8_t *vocab_bytes, const int64_t *vocab_off,
                    int64_t V, const int64_t *tokens, ms_stream_t stream) {
  if (B < 0 || V < 1) return MS_E_INVALID;
  if (B == 0) return MS_OK;
  if (!states || !vocab_bytes || !vocab_off || !tokens) return MS_E_INVALID;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const unsigned grid = (unsigned)((B + 127) / 128);
  ms::ms_json_feed_kernel<<<grid, 128, 0, s>>>(states, B, vocab_bytes, vocab_off, V, tokens, 0);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? MS_OK : cuda_fail(e);
}

namespace {
int build_json_mask(const uint32_t *states, int64_t B, const uint8_t *vocab_bytes, const int64_t *vocab_off,
                    const uint32_t *packed, const uint8_t *lens, const int32_t *order, int64_t V,
                    uint32_t *mask, int64_t mask_ld, int32_t *row_status, ms_stream_t stream) {
  if (B < 0 || B > 65535 || V < 1 || V > 0x7FFFFFFFll || mask_ld < (V + 31) / 32) return MS_E_INVALID;
  if (B == 0) return MS_OK;
  if (!states || !vocab_bytes || !vocab_off || !mask || !row_status) return MS_E_INVALID;
  if ((packed == nullptr) != (lens == nullptr) || (reinterpret_cast<uintptr_t>(packed) & 15u)) return MS_E_INVALID;
  if (order && !packed) return MS_E_INVALID;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  // rows in the same parse state share one mask: representatives first (and,
  // for the ordered vocabulary's atomic ORs, their mask words cleared)
  const int64_t nwords = (V + 31) / 32;
  ms::ms_json_dedup_kernel<<<(unsigned)((B + 3) / 4), 128, 0, s>>>(states, B, row_status,
                                                                   order ? mask : nullptr, mask_ld, nwords);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e);
  // about 64 CTAs per SM over all rows (about 16 per SM when a quarter of the
  // rows are representatives); every warp of a CTA at least one word
  int64_t x = (9472 + B - 1) / B;
  x = x < 1 ? 1 : x;
  const int64_t xmax = (nwords + ms::kJsonThreads / 32 - 1) / (ms::kJsonThreads / 32);
  x = x > xmax ? xmax : x;
  ms::JsonVocab voc{vocab_bytes, vocab_off, V, reinterpret_cast<const uint4 *>(packed), lens, order};
  ms::ms_json_mask_kernel<<<dim3((unsigned)x, (unsigned)B), ms::kJsonThreads, 0, s>>>(states, voc, mask, mask_ld,
                                                                                       row_status);
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e);
  ms::ms_json_mask_copy_kernel<<<(unsigned)B, 256, 0, s>>>(mask, mask_ld, nwords, row_status);
  e = cudaGetLastError();
  return e == cudaSuccess ? MS_OK : cuda_fail(e);
}

int pack_vocab(const uint8_t *vocab_bytes, const int64_t *vocab_off, int64_t V, const int32_t *order,
               uint32_t *packed, uint8_t *lens, ms_stream_t stream) {
  if (V < 1 || V > 0x7FFFFFFFll) return MS_E_INVALID;
  if (!vocab_bytes || !vocab_off || !packed || !lens || (reinterpret_cast<uintptr_t>(packed) & 15u)) {
    return MS_E_INVALID;
  }
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  ms::ms_json_pack_kernel<<<(unsigned)((V + 255) / 256), 256, 0, s>>>(vocab_bytes, vocab_off, V, order,
                                                                     reinterpret_cast<uint4 *>(packed), lens);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? MS_OK : cuda_fail(e);
}
}  // namespace

int ms_build_json_mask(const uint32_t *states, int64_t B, const uint8_t *vocab_bytes, const int64_t *vocab_off,
                       int64_t V, uint32_t *mask, int64_t mask_ld, int32_t *row_status, ms_stream_t stream) {
  return build_json_mask(states, B, vocab_bytes, vocab_off, nullptr, nullptr, nullptr, V, mask, mask_ld,
                         row_status, stream);
}

int ms_json_pack_vocab(const uint8_t *vocab_bytes, const int64_t *vocab_off, int64_t V, uint32_t *packed,
                       uint8_t *lens, ms_stream_t stream) {
  return pack_vocab(vocab_bytes, vocab_off, V, nullptr, packed, lens, stream);
}

int ms_build_json_mask_packed(const uint32_t *states, int64_t B, const uint8_t *vocab_bytes,
                              const int64_t *vocab_off, const uint32_t *packed, const uint8_t *lens, int64_t V,
                              uint32_t *mask, int64_t mask_ld, int32_t *row_status, ms_stream_t stream) {
  if (!packed || !lens) return MS_E_INVALID;
  return build_json_mask(states, B, vocab_bytes, vocab_off, packed, lens, nullptr, V, mask, mask_ld, row_status,
                         stream);
}

int ms_json_pack_vocab_ordered(const uint8_t *vocab_bytes, const int64_t *vocab_off, int64_t V,
                               const int32_t *order, uint32_t *packed, uint8_t *lens, ms_stream_t stream) {
  if (!order) return MS_E_INVALID;
  return pack_vocab(vocab_bytes, vocab_off, V, order, packed, lens, stream);
}

int ms_build_json_mask_ordered(const uint32_t *states, int64_t B, const uint8_t *vocab_bytes,
                               const int64_t *vocab_off, const uint32_t *packed, const uint8_t *lens,
                               const int32_t *order, int64_t V, uint32_t *mask, int64_t mask_ld,
                               int32_t *row_status, ms_stream_t stream) {
  if (!packed || !lens || !order) return MS_E_INVALID;
  return build_json_mask(states, B, vocab_bytes, vocab_off, packed, lens, order, V, mask, mask_ld, row_status,
                         stream);
}

// ------------------------------------------------ no-alloc JSON mask build
namespace {
// The fixed-width vocabulary tables of ms_build_json_mask_noalloc: up to
// kNoAllocMaxV tokens of 16 bytes, then their lengths.  File-scope device
// memory: created with the module on every GPU that loads the library and
// held until the process exits.  Nothing in it needs to start at zero: each
// call rewrites the entries of its V tokens before the mask kernel reads them.
constexpr int64_t kNoAllocMaxV = 262144;
constexpr size_t kNoAllocPackedBytes = (size_t)kNoAllocMaxV * 16;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocPackedBytes + kNoAllocMaxV];

std::atomic<unsigned char *> g_noalloc_ptr[kMaxDevices];

// The array's device address on the current device.  In host code its name
// only stands in for it, so the address is looked up (once per device, with
// that device current) and passed to the kernels.
int noalloc_scratch(unsigned char **out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e);
  if (dev < 0 || dev >= kMaxDevices) return MS_E_UNSUPPORTED;
  unsigned char *p = g_noalloc_ptr[dev].load(std::memory_order_acquire);
  if (!p) {
    e = cudaGetSymbolAddress(reinterpret_cast<void **>(&p), g_noalloc_scratch);
    if (e != cudaSuccess) return cuda_fail(e);
    g_noalloc_ptr[dev].store(p, std::memory_order_release);
  }
  *out = p;
  return MS_OK;
}
}  // namespace

int ms_build_json_mask_noalloc(const uint32_t *states, int64_t B, const uint8_t *vocab_bytes,
                               const int64_t *vocab_off, int64_t V, uint32_t *mask, int64_t mask_ld,
                               int32_t *row_status, ms_stream_t stream) {
  if (V > kNoAllocMaxV) return MS_E_TOO_LARGE;
  if (B < 0 || B > 65535 || V < 1 || mask_ld < (V + 31) / 32) return MS_E_INVALID;
  if (B == 0) return MS_OK;
  if (!states || !vocab_bytes || !vocab_off || !mask || !row_status) return MS_E_INVALID;
  unsigned char *scratch = nullptr;
  int rc = noalloc_scratch(&scratch);
  if (rc != MS_OK) return rc;
  uint32_t *packed = reinterpret_cast<uint32_t *>(scratch);
  uint8_t *lens = scratch + kNoAllocPackedBytes;
  rc = pack_vocab(vocab_bytes, vocab_off, V, nullptr, packed, lens, stream);
  if (rc != MS_OK) return rc;
  return build_json_mask(states, B, vocab_bytes, vocab_off, packed, lens, nullptr, V, mask, mask_ld, row_status,
                         stream);
}

}  // extern "C"
