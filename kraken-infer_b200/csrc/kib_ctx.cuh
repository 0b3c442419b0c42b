// kib_ctx.cuh -- host-side context, status plumbing and kernel launch helpers.
#pragma once

#include <cuda_runtime.h>

#include <cstdlib>
#include <string>

#include "../../include/kib.h"
#include "kquant_gemv.cuh"

struct kib_ctx {
  int device = 0;
  int num_sms = 148;
  cudaStream_t stream = nullptr;
  bool in_graph = false;
  std::string last_error;
  int* d_err = nullptr;            // device-side error flag (bounded waits)
  // LM-head argmax scratch for the op-level entry points
  float* d_cand_max = nullptr;
  float* d_cand_sum = nullptr;
  int* d_cand_idx = nullptr;
  unsigned* d_counter = nullptr;
};

namespace kib {

inline int set_error(kib_ctx* ctx, int code, const std::string& msg) {
  if (ctx) ctx->last_error = msg;
  return code;
}

inline int cuda_status(cudaError_t e, const char* expr, const char* file, int line) {
  (void)expr;
  (void)file;
  (void)line;
  return e == cudaSuccess ? KIB_OK : KIB_ERR_INTERNAL;
}

inline int check_cuda(kib_ctx* ctx, cudaError_t e, const char* what) {
  if (e == cudaSuccess) return KIB_OK;
  return set_error(ctx, KIB_ERR_INTERNAL, std::string(what) + ": " + cudaGetErrorString(e));
}

// Finishes an op: outside a graph scope the reference waits for completion
// (mps_backend.mm:4409-4428), so do the same and surface device errors.
int finish_op(kib_ctx* ctx, const char* what);

// Launch with programmatic stream serialization (PDL) so that the next
// kernel's pre-wait prologue overlaps this one's tail.
// KIB_PDL=0 turns programmatic dependent launch off (diagnostics).
inline bool pdl_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("KIB_PDL");
    return !(v && v[0] == '0');
  }();
  return on;
}

// Every kernel of the decode chain asks for the same shared-memory carveout
// (the maximum), so consecutive kernels never make an SM drain to
// re-partition L1 / shared memory.
template <typename... KArgs>
void pin_carveout(void (*kernel)(KArgs...)) {
  static bool done = false;  // one flag per kernel instantiation
  if (!done) {
    cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared);
    done = true;
  }
}

template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                       Args&&... args) {
  pin_carveout(kernel);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// The same with the CTAs grouped into thread-block clusters of `cluster`
// (grid dimensions divisible by it); sizes above 8 need the kernel's
// non-portable-cluster attribute.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl_cluster(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                               dim3 cluster, Args&&... args) {
  pin_carveout(kernel);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = cluster.x;
  attr[0].val.clusterDim.y = cluster.y;
  attr[0].val.clusterDim.z = cluster.z;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 2 : 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// ------------------------------------------------------------------ GEMV
struct GemvSegDesc {
  const void* w = nullptr;
  const void* w2 = nullptr;  // pair partner (up) for kEpiSiluMul
  float* out = nullptr;
  int rows = 0;
  int ld = 0;
  int epilogue = kEpiStore;
};

struct GemvDesc {
  int type = kTypeQ4K;
  int cols = 0;
  int ntok = 1;
  int nseg = 0;
  GemvSegDesc seg[kGemvMaxSegs];
  int prologue = kProPlain;
  const float* in = nullptr;
  int in_ld = 0;
  const float* norm_w = nullptr;
  float eps = 1e-6f;
  const float* gate = nullptr;
  int head_dim = 128;
  const float* resid = nullptr;
  float* conv_state = nullptr;
  const float* conv_w = nullptr;
  int conv_k = 4;
  // argmax
  bool argmax = false;
  float* cand_max = nullptr;
  float* cand_sum = nullptr;
  int* cand_idx = nullptr;
  unsigned* counter = nullptr;
  int* token_out = nullptr;
  float* prob_out = nullptr;
  int* token_log = nullptr;
  int* step_counter = nullptr;
  int* pos_advance = nullptr;
  float* x_out = nullptr;
  int* err = nullptr;
  unsigned long long* trace = nullptr;
};

// Validates, plans the tile geometry and launches the GEMV.  Returns a cuda error.
cudaError_t gemv_launch(const GemvDesc& d, int num_sms, cudaStream_t st, std::string* why);

}  // namespace kib

// C-ABI argument checks (the reference's Status::unavailable / invalid_argument)
#define KIB_REQUIRE_CTX(ctx)                       \
  do {                                             \
    if (!(ctx) || !(ctx)->stream) return KIB_ERR_UNAVAILABLE; \
  } while (0)
#define KIB_ARG(cond, msg)                                              \
  do {                                                                  \
    if (!(cond)) return set_error(ctx, KIB_ERR_INVALID_ARGUMENT, msg);  \
  } while (0)
