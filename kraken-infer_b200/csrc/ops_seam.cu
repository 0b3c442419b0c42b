// ops_seam.cu -- the rest of the MpsContext operator surface: the reference's
// named variants of ops that ops.cu implements generically (type-named top1 /
// argmax LM heads, the `_at` state-offset forms, single-token GDN and stateful
// conv, single-row dequantisation, non-batched norms and attention) and the
// copy / conv-state ops the runtime uses around the hot path (copy_f32_region,
// copy_f16_rows, ssm_conv_f32, build_ssm_conv_state_f32).  Every entry keeps
// the reference's argument order and meaning (include/toyllm/backends/mps/
// mps_backend.hpp), with device pointers in place of MpsBuffer handles and
// element offsets where the reference takes element offsets.
#include <cuda_fp16.h>

#include "kib_ctx.cuh"
#include "kquant.cuh"

namespace kib {
namespace {

inline unsigned seam_blocks(size_t n) { return static_cast<unsigned>((n + 255) / 256); }

// copy_f32_region (mps_backend.mm:2631-2640): dst[doff + i] = src[soff + i].
__global__ void copy_region_kernel(const float* src, float* dst, size_t n) {
  const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i < n) dst[i] = src[i];
}

// copy_f16_rows (mps_backend.mm:2668-2679): strided row copy of halves.
__global__ void copy_f16_rows_kernel(const uint16_t* src, uint16_t* dst, size_t rows, size_t rv, size_t ss, size_t so,
                                     size_t ds, size_t dof) {
  const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= rows * rv) return;
  const size_t r = i / rv, c = i % rv;
  dst[dof + r * ds + c] = src[so + r * ss + c];
}

// ssm_conv_f32 (mps_backend.mm:2376-2400): input [seq][channel][K-1+T] (the
// conv window already prepended), weights [channel][K], output
// [seq][token][channel]; a plain depthwise causal conv, no activation.
__global__ void ssm_conv_window_kernel(const float* in, const float* w, float* out, unsigned K, unsigned C, unsigned T,
                                       unsigned S) {
  const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const size_t total = static_cast<size_t>(S) * T * C;
  if (i >= total) return;
  const unsigned c = static_cast<unsigned>(i % C);
  const unsigned t = static_cast<unsigned>((i / C) % T);
  const unsigned s = static_cast<unsigned>(i / (static_cast<size_t>(C) * T));
  const unsigned span = K - 1u + T;
  const float* x = in + (static_cast<size_t>(s) * C + c) * span + t;
  const float* wc = w + static_cast<size_t>(c) * K;
  float sum = 0.0f;
  for (unsigned k = 0; k < K; ++k) sum += x[k] * wc[k];
  out[i] = sum;
}

// build_ssm_conv_state_f32 (mps_backend.mm:2428-2456): conv_input[channel] =
// [state row | the T new inputs of that channel]; the state row then becomes
// the last K-1 entries of that window.  One thread per channel.
__global__ void build_conv_state_kernel(float* state, const float* in, float* conv_in, unsigned K, unsigned C,
                                        unsigned T) {
  const unsigned c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= C) return;
  const unsigned sw = K - 1u, span = sw + T;
  float* st = state + static_cast<size_t>(c) * sw;
  float* ci = conv_in + static_cast<size_t>(c) * span;
  for (unsigned p = 0; p < sw; ++p) ci[p] = st[p];
  for (unsigned t = 0; t < T; ++t) ci[sw + t] = in[static_cast<size_t>(t) * C + c];
  // the new state reads the window just written (state entries first, so an
  // in-order rewrite never reads an entry it has already replaced)
  for (unsigned p = 0; p < sw; ++p) st[p] = ci[T + p];
}

// ssm_conv1_f32_stateful (mps_backend.mm:2402-2426): one token; the state row
// shifts left by one and takes the new input.
__global__ void conv1_stateful_kernel(float* state, const float* in, const float* w, float* out, unsigned K,
                                      unsigned C) {
  const unsigned c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= C) return;
  const unsigned sw = K - 1u;
  float* st = state + static_cast<size_t>(c) * sw;
  const float* wc = w + static_cast<size_t>(c) * K;
  const float cur = in[c];
  float sum = 0.0f;
  for (unsigned i = 0; i < sw; ++i) sum += st[i] * wc[i];
  sum += cur * wc[sw];
  for (unsigned i = 0; i + 1u < sw; ++i) st[i] = st[i + 1u];
  st[sw - 1u] = cur;
  out[c] = sum;
}

// dequantize_row_q*_k_f32 (mps_backend.mm:1693-1760): one row, by pointer.
template <int QT>
__global__ void dequant_row_kernel(const uint8_t* row, int cols, float* out) {
  const int units = cols / 64;
  for (int u = blockIdx.x * blockDim.x + threadIdx.x; u < units; u += gridDim.x * blockDim.x) {
    const int blk = u >> 2, unit = u & 3;
    float v[64];
    unit_dequant<QT>(row + static_cast<size_t>(blk) * kquant_block_bytes(QT), unit, v);
#pragma unroll
    for (int e = 0; e < 64; ++e) out[256 * blk + unit_col<QT>(unit, e)] = v[e];
  }
}

int seam_top1(kib_ctx* ctx, int type, const void* w, uint64_t rows, uint64_t cols, const float* in, int32_t* tok,
              float* prob) {
  return kib_matvec_kquant_f32_argmax(ctx, type, w, rows, cols, in, tok, prob);
}

int dequant_row(kib_ctx* ctx, int type, const void* w, uint64_t row, uint64_t cols, float* out) {
  KIB_REQUIRE_CTX(ctx);
  KIB_ARG(w && out && cols && cols % 256 == 0, "dequantize_row: invalid arguments");
  const size_t row_bytes = cols / 256 * static_cast<size_t>(kquant_block_bytes(type));
  const uint8_t* r = static_cast<const uint8_t*>(w) + row * row_bytes;
  const int units = static_cast<int>(cols / 64);
  const unsigned grid = static_cast<unsigned>((units + 127) / 128);
  if (type == kTypeQ4K) dequant_row_kernel<kTypeQ4K><<<grid, 128, 0, ctx->stream>>>(r, static_cast<int>(cols), out);
  else if (type == kTypeQ5K) dequant_row_kernel<kTypeQ5K><<<grid, 128, 0, ctx->stream>>>(r, static_cast<int>(cols), out);
  else if (type == kTypeQ6K) dequant_row_kernel<kTypeQ6K><<<grid, 128, 0, ctx->stream>>>(r, static_cast<int>(cols), out);
  else return set_error(ctx, KIB_ERR_INVALID_ARGUMENT, "dequantize_row: unsupported type");
  return finish_op(ctx, "dequantize_row");
}

}  // namespace
}  // namespace kib

using namespace kib;

extern "C" {

// ---- host <-> device copies at an offset
int kib_copy_to_buffer_at(kib_ctx* ctx, void* dst, uint64_t dst_offset, const void* src, uint64_t bytes) {
  return kib_copy_to_buffer(ctx, dst, dst_offset, src, bytes);
}
int kib_copy_from_buffer_at(kib_ctx* ctx, const void* src, uint64_t src_offset, void* dst, uint64_t bytes) {
  return kib_copy_from_buffer(ctx, src, src_offset, dst, bytes);
}

// ---- device copies
int kib_copy_f32_region(kib_ctx* ctx, const float* src, float* dst, uint64_t src_offset, uint64_t dst_offset,
                        uint64_t size) {
  KIB_REQUIRE_CTX(ctx);
  KIB_ARG(src && dst && size, "copy_f32_region: invalid arguments");
  copy_region_kernel<<<seam_blocks(size), 256, 0, ctx->stream>>>(src + src_offset, dst + dst_offset, size);
  return finish_op(ctx, "copy_f32_region");
}
int kib_copy_f16_rows(kib_ctx* ctx, const uint16_t* src, uint16_t* dst, uint64_t rows, uint64_t row_size,
                      uint64_t src_stride, uint64_t src_offset, uint64_t dst_stride, uint64_t dst_offset) {
  KIB_REQUIRE_CTX(ctx);
  KIB_ARG(src && dst && rows && row_size && row_size <= src_stride && row_size <= dst_stride,
          "copy_f16_rows: invalid arguments");
  copy_f16_rows_kernel<<<seam_blocks(rows * row_size), 256, 0, ctx->stream>>>(src, dst, rows, row_size, src_stride,
                                                                              src_offset, dst_stride, dst_offset);
  return finish_op(ctx, "copy_f16_rows");
}

// ---- GDN causal conv, the reference's three forms
int kib_ssm_conv_f32(kib_ctx* ctx, const float* input, const float* kernel, uint64_t conv_kernel, uint64_t channels,
                     uint64_t tokens, uint64_t sequences, float* output) {
  KIB_REQUIRE_CTX(ctx);
  KIB_ARG(input && kernel && output && conv_kernel && channels && tokens && sequences,
          "ssm_conv: dimensions must be positive");
  KIB_ARG(conv_kernel - 1 + tokens < (1ull << 32) && channels < (1ull << 32) && sequences < (1ull << 32),
          "ssm_conv: dimensions exceed 32 bits");
  const size_t total = channels * tokens * sequences;
  ssm_conv_window_kernel<<<seam_blocks(total), 256, 0, ctx->stream>>>(
      input, kernel, output, static_cast<unsigned>(conv_kernel), static_cast<unsigned>(channels),
      static_cast<unsigned>(tokens), static_cast<unsigned>(sequences));
  return finish_op(ctx, "ssm_conv");
}
int kib_build_ssm_conv_state_f32(kib_ctx* ctx, float* state, uint64_t state_offset, const float* input,
                                 uint64_t conv_kernel, uint64_t channels, uint64_t tokens, float* conv_input) {
  KIB_REQUIRE_CTX(ctx);
  KIB_ARG(state && input && conv_input && conv_kernel >= 2 && channels && tokens,
          "build_ssm_conv_state: dimensions are invalid");
  KIB_ARG(conv_kernel - 1 + tokens < (1ull << 32) && channels < (1ull << 32), "build_ssm_conv_state: too large");
  build_conv_state_kernel<<<seam_blocks(channels), 256, 0, ctx->stream>>>(
      state + state_offset, input, conv_input, static_cast<unsigned>(conv_kernel), static_cast<unsigned>(channels),
      static_cast<unsigned>(tokens));
  return finish_op(ctx, "build_ssm_conv_state");
}
int kib_ssm_conv1_f32_stateful_at(kib_ctx* ctx, float* state, uint64_t state_offset, const float* input,
                                  const float* kernel, uint64_t conv_kernel, uint64_t channels, float* output) {
  KIB_REQUIRE_CTX(ctx);
  KIB_ARG(state && input && kernel && output && conv_kernel >= 2 && channels && channels < (1ull << 32),
          "ssm_conv1_stateful: dimensions are invalid");
  conv1_stateful_kernel<<<seam_blocks(channels), 256, 0, ctx->stream>>>(
      state + state_offset, input, kernel, output, static_cast<unsigned>(conv_kernel), static_cast<unsigned>(channels));
  return finish_op(ctx, "ssm_conv1_stateful");
}
int kib_ssm_conv1_f32_stateful(kib_ctx* ctx, float* state, const float* input, const float* kernel,
                               uint64_t conv_kernel, uint64_t channels, float* output) {
  return kib_ssm_conv1_f32_stateful_at(ctx, state, 0, input, kernel, conv_kernel, channels, output);
}

// ---- gated delta net: single token and state-offset forms
int kib_gated_delta_net_f32_batched_in_place_at(kib_ctx* ctx, const float* q, const float* k, const float* v,
                                                const float* g, const float* beta, float* state, uint64_t state_offset,
                                                uint64_t tokens, uint64_t key_heads, uint64_t value_heads,
                                                uint64_t head_dim, float* output) {
  KIB_REQUIRE_CTX(ctx);
  KIB_ARG(state, "gated_delta_net: null state");
  return kib_gated_delta_net_f32_batched_in_place(ctx, q, k, v, g, beta, state + state_offset, tokens, key_heads,
                                                  value_heads, head_dim, output);
}
int kib_gated_delta_net_f32_in_place_at(kib_ctx* ctx, const float* q, const float* k, const float* v, const float* g,
                                        const float* beta, float* state, uint64_t state_offset, uint64_t key_heads,
                                        uint64_t value_heads, uint64_t head_dim, float* output) {
  return kib_gated_delta_net_f32_batched_in_place_at(ctx, q, k, v, g, beta, state, state_offset, 1, key_heads,
                                                     value_heads, head_dim, output);
}
int kib_gated_delta_net_f32_in_place(kib_ctx* ctx, const float* q, const float* k, const float* v, const float* g,
                                     const float* beta, float* state, uint64_t key_heads, uint64_t value_heads,
                                     uint64_t head_dim, float* output) {
  return kib_gated_delta_net_f32_batched_in_place_at(ctx, q, k, v, g, beta, state, 0, 1, key_heads, value_heads,
                                                     head_dim, output);
}

// ---- type-named LM heads: argmax, and argmax + p(top1)
int kib_matvec_q4_k_f32_top1(kib_ctx* ctx, const void* w, uint64_t rows, uint64_t cols, const float* in,
                             int32_t* token_out, float* prob_out) {
  KIB_ARG(prob_out, "top1: null probability output");
  return seam_top1(ctx, kTypeQ4K, w, rows, cols, in, token_out, prob_out);
}
int kib_matvec_q5_k_f32_top1(kib_ctx* ctx, const void* w, uint64_t rows, uint64_t cols, const float* in,
                             int32_t* token_out, float* prob_out) {
  KIB_ARG(prob_out, "top1: null probability output");
  return seam_top1(ctx, kTypeQ5K, w, rows, cols, in, token_out, prob_out);
}
int kib_matvec_q6_k_f32_top1(kib_ctx* ctx, const void* w, uint64_t rows, uint64_t cols, const float* in,
                             int32_t* token_out, float* prob_out) {
  KIB_ARG(prob_out, "top1: null probability output");
  return seam_top1(ctx, kTypeQ6K, w, rows, cols, in, token_out, prob_out);
}
int kib_matvec_q4_k_f32_argmax(kib_ctx* ctx, const void* w, uint64_t rows, uint64_t cols, const float* in,
                               int32_t* token_out) {
  return seam_top1(ctx, kTypeQ4K, w, rows, cols, in, token_out, nullptr);
}
int kib_matvec_q5_k_f32_argmax(kib_ctx* ctx, const void* w, uint64_t rows, uint64_t cols, const float* in,
                               int32_t* token_out) {
  return seam_top1(ctx, kTypeQ5K, w, rows, cols, in, token_out, nullptr);
}
int kib_matvec_q6_k_f32_argmax(kib_ctx* ctx, const void* w, uint64_t rows, uint64_t cols, const float* in,
                               int32_t* token_out) {
  return seam_top1(ctx, kTypeQ6K, w, rows, cols, in, token_out, nullptr);
}
int kib_argmax_prob_f32_i32(kib_ctx* ctx, const float* values, uint64_t size, int32_t* token_out, float* prob_out) {
  KIB_ARG(prob_out, "argmax_prob: null probability output");
  return kib_argmax_f32_i32(ctx, values, size, token_out, prob_out);
}

// ---- single-row dequantisation
int kib_dequantize_row_q4_k_f32(kib_ctx* ctx, const void* w, uint64_t row, uint64_t cols, float* out) {
  return dequant_row(ctx, kTypeQ4K, w, row, cols, out);
}
int kib_dequantize_row_q5_k_f32(kib_ctx* ctx, const void* w, uint64_t row, uint64_t cols, float* out) {
  return dequant_row(ctx, kTypeQ5K, w, row, cols, out);
}
int kib_dequantize_row_q6_k_f32(kib_ctx* ctx, const void* w, uint64_t row, uint64_t cols, float* out) {
  return dequant_row(ctx, kTypeQ6K, w, row, cols, out);
}

// ---- non-batched forms (one token)
int kib_rms_norm_f32_f32(kib_ctx* ctx, const float* input, const float* weight, uint64_t size, float eps,
                         float* output) {
  return kib_rms_norm_f32_f32_batched(ctx, input, weight, 1, size, eps, output);
}
int kib_qk_norm_f32_f32(kib_ctx* ctx, float* values, const float* weight, uint64_t heads, uint64_t head_dim,
                        float eps) {
  return kib_qk_norm_f32_f32_batched(ctx, values, weight, 1, heads, head_dim, eps);
}
int kib_attention_f32_f16_kv(kib_ctx* ctx, const float* q, const uint16_t* kc, const uint16_t* vc, uint64_t layer,
                             uint64_t position, uint64_t capacity_tokens, uint64_t heads, uint64_t kv_heads,
                             uint64_t head_dim, float* out) {
  return kib_attention_f32_batched_f16_kv(ctx, q, kc, vc, layer, position, 1, capacity_tokens, heads, kv_heads,
                                          head_dim, out);
}

}  // extern "C"
