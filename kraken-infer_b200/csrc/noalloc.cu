// noalloc.cu -- the fused K-quant LM-head argmax without any allocation.
//
// kib_matvec_kquant_f32_argmax needs a kib_ctx, and creating one calls
// cudaMalloc for the per-CTA argmax candidates, the completion counter and the
// error flag.  Some callers cannot allocate device memory at the point where
// they want the next token: an embedding host that hands this library a
// pre-budgeted memory pool and forbids allocations after start-up, a caller
// running under a custom allocator that owns all device memory, or code that
// runs on a path where an allocation would synchronise the device.  For them,
// kib_matvec_kquant_f32_argmax_noalloc keeps that scratch in a fixed-size
// array in the library's own device image (one copy per GPU that loads the
// library, held until the process exits) and takes the stream from the caller.
//
// Limits: the scratch holds the candidates of at most kNoAllocMaxCtas CTAs
// (the launch uses at most one CTA per SM), one token, so devices with more
// SMs than that are refused.  Every call shares the one array: two calls whose
// kernels overlap on the GPU (different streams without ordering between
// them) race on it and give wrong tokens.
#include <mutex>

#include "kib.h"
#include "kib_ctx.cuh"

namespace kib {
namespace {

constexpr int kNoAllocMaxCtas = 1024;
constexpr int kNoAllocMaxDevices = 64;

struct NoAllocScratch {
  // the kernel strides the candidates by kGemvMaxTok per CTA
  float cand_max[kNoAllocMaxCtas * kGemvMaxTok];
  float cand_sum[kNoAllocMaxCtas * kGemvMaxTok];
  int cand_idx[kNoAllocMaxCtas * kGemvMaxTok];
  unsigned counter;  // last-CTA ticket; must be 0 when a launch starts
  int err;           // bounded-wait failure flag; must be 0 when a launch starts
};

// 96 KB + 8 bytes per device.
static __device__ __align__(256) NoAllocScratch g_noalloc_scratch;

// Device address of g_noalloc_scratch per device.  On the host the symbol
// itself is only a stand-in, so the address has to come from the runtime.
NoAllocScratch* g_scratch_addr[kNoAllocMaxDevices] = {};
std::mutex g_scratch_mu;

int scratch_for_current_device(NoAllocScratch** out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0) return KIB_ERR_UNAVAILABLE;
  if (dev >= kNoAllocMaxDevices) return KIB_ERR_UNAVAILABLE;
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (g_scratch_addr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || p == nullptr) {
      cudaGetLastError();
      return KIB_ERR_INTERNAL;
    }
    g_scratch_addr[dev] = static_cast<NoAllocScratch*>(p);
  }
  *out = g_scratch_addr[dev];
  return KIB_OK;
}

}  // namespace
}  // namespace kib

using namespace kib;

extern "C" int kib_matvec_kquant_f32_argmax_noalloc(int type, const void* weight, uint64_t rows, uint64_t cols,
                                                    const float* input, int32_t* token_out, float* prob_out,
                                                    void* stream) {
  const bool type_ok = type == kTypeQ4K || type == kTypeQ5K || type == kTypeQ6K;
  if (!type_ok || weight == nullptr || input == nullptr || token_out == nullptr)
    return KIB_ERR_INVALID_ARGUMENT;
  if (rows == 0 || rows > 0x7FFFFFFFull || cols == 0 || cols % 256 != 0 || cols > 16384)
    return KIB_ERR_INVALID_ARGUMENT;
  int dev = 0, sms = 0, major = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess || major < 10)
    return KIB_ERR_UNAVAILABLE;
  if (sms > kNoAllocMaxCtas) return KIB_ERR_INVALID_ARGUMENT;  // more CTAs than the fixed scratch holds
  NoAllocScratch* s = nullptr;
  int st = scratch_for_current_device(&s);
  if (st != KIB_OK) return st;
  cudaStream_t strm = static_cast<cudaStream_t>(stream);
  // the previous call may have left a failure flag (a counter left non-zero
  // is only possible after a failed launch); both must start at zero
  if (cudaMemsetAsync(&s->counter, 0, sizeof(unsigned) + sizeof(int), strm) != cudaSuccess) return KIB_ERR_INTERNAL;
  GemvDesc d;
  d.type = type;
  d.cols = static_cast<int>(cols);
  d.ntok = 1;
  d.nseg = 1;
  d.seg[0].w = weight;
  d.seg[0].out = nullptr;
  d.seg[0].rows = static_cast<int>(rows);
  d.seg[0].ld = static_cast<int>(rows);
  d.seg[0].epilogue = kEpiArgmax;
  d.in = input;
  d.in_ld = static_cast<int>(cols);
  d.argmax = true;
  d.cand_max = s->cand_max;
  d.cand_sum = s->cand_sum;
  d.cand_idx = s->cand_idx;
  d.counter = &s->counter;
  d.token_out = token_out;
  d.prob_out = prob_out;
  d.err = &s->err;
  if (gemv_launch(d, sms, strm, nullptr) != cudaSuccess) return KIB_ERR_INTERNAL;
  return cudaGetLastError() == cudaSuccess ? KIB_OK : KIB_ERR_INTERNAL;
}
