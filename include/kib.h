/* kib.h -- C ABI of the B200 (sm_100a) backend for kraken-infer's Qwen3.5
 * decode / MTP-verify hot path.
 *
 * Two levels, both plain C (pointers, sizes, status codes; no C++ or torch
 * types):
 *
 *  1. Op level -- the drop-in twin of the reference's backend seam
 *     toyllm::mps::MpsContext (include/toyllm/backends/mps/mps_backend.hpp:76-428).
 *     Every op takes device pointers the caller allocated (kib_make_buffer or
 *     any cudaMalloc'd memory), validates shapes like the reference
 *     (mps_backend.mm:4006-4308) and enqueues on the context's stream.
 *     Outside kib_begin_graph/kib_commit_graph each op waits for completion
 *     (the reference commits and waits per op, mps_backend.mm:4409-4428);
 *     inside, ops are only enqueued and kib_commit_graph blocks.
 *
 *  2. Runtime level -- the reference's Qwen3.5 entry points
 *     (read_gguf_file + build_qwen35_weight_map + build_qwen35_execution_plan +
 *     generate_qwen35_metal, include/toyllm/runtime/qwen35_runtime.hpp:70-176)
 *     over a GGUF file, with the MTP draft/accept statistics of CpuMtpReport
 *     (include/toyllm/runtime/cpu_inference.hpp:79-94).
 *
 * Status codes mirror toyllm::Status (include/toyllm/core/status.hpp:8-50);
 * kib_last_error() returns the message of the last failing call on a context.
 * A context is not thread-safe (one stream, one pending batch), like MpsContext.
 */
#ifndef KIB_H_
#define KIB_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum kib_status {
  KIB_OK = 0,
  KIB_ERR_INVALID_ARGUMENT = 1, /* Status::invalid_argument */
  KIB_ERR_UNAVAILABLE = 2,      /* Status::unavailable (no device / not built) */
  KIB_ERR_INTERNAL = 3,         /* Status::internal_error (CUDA failure) */
  KIB_ERR_TIMEOUT = 4           /* a bounded device wait gave up */
};

/* GGML tensor types accepted by the K-quant ops (qwen35_runtime.cpp:1391-1403). */
enum kib_ggml_type { KIB_TYPE_F32 = 0, KIB_TYPE_F16 = 1, KIB_TYPE_Q4_K = 12, KIB_TYPE_Q5_K = 13, KIB_TYPE_Q6_K = 14 };

typedef struct kib_ctx kib_ctx;

/* ---------------------------------------------------------------- lifetime */
/* MpsContext::create (mps_backend.hpp:87; mps_backend.mm:5043-5636). */
int kib_create(int device, kib_ctx** out);
/* ~MpsContext. */
void kib_destroy(kib_ctx* ctx);
/* MpsContext::valid (mps_backend.hpp:88). */
int kib_valid(const kib_ctx* ctx);
const char* kib_last_error(const kib_ctx* ctx);
/* MpsContext::begin_graph / commit_graph / abort_graph (mps_backend.hpp:92-94;
 * mps_backend.mm:4430-4467). */
int kib_begin_graph(kib_ctx* ctx);
int kib_commit_graph(kib_ctx* ctx);
int kib_abort_graph(kib_ctx* ctx);
/* The context's CUDA stream (cudaStream_t), for callers that interleave their own work. */
void* kib_stream(kib_ctx* ctx);

/* ------------------------------------------------------------------ memory */
/* MpsContext::make_buffer (mps_backend.hpp:96). */
int kib_make_buffer(kib_ctx* ctx, uint64_t bytes, void** dev_out);
int kib_free_buffer(kib_ctx* ctx, void* dev);
/* copy_to_buffer(_at) / copy_from_buffer(_at) / copy_buffer_region / zero_buffer
 * (mps_backend.hpp:97-114). */
int kib_copy_to_buffer(kib_ctx* ctx, void* dst, uint64_t dst_offset, const void* src_host, uint64_t bytes);
int kib_copy_from_buffer(kib_ctx* ctx, const void* src, uint64_t src_offset, void* dst_host, uint64_t bytes);
int kib_copy_buffer_region(kib_ctx* ctx, const void* src, void* dst, uint64_t src_offset, uint64_t dst_offset,
                           uint64_t bytes);
int kib_zero_buffer(kib_ctx* ctx, void* dev, uint64_t bytes);

/* ----------------------------------------------------------------- K-quant */
/* y[rows] = W . x over raw super-blocks: matvec_q{4,5,6}_k_f32_device
 * (mps_backend.hpp:137, 179; kernels mps_backend.mm:295-463). type is 12/13/14. */
int kib_matvec_kquant_f32(kib_ctx* ctx, int type, const void* weight, uint64_t rows, uint64_t cols,
                          const float* input, float* output);
/* Y[tokens][rows] = X[tokens][cols] . W^T: matmul_q{4,5,6}_k_f32_device
 * (mps_backend.hpp:150, 192; dispatch mps_backend.mm:6336-6454).  Numerics follow
 * the reference's buckets: tokens <= 3 fp32; 4..8 weights rounded to half;
 * > 8 weights and input rounded to half, fp32 accumulation. */
int kib_matmul_kquant_f32(kib_ctx* ctx, int type, const void* weight, uint64_t rows, uint64_t cols,
                          uint64_t tokens, const float* input, float* output);
/* Fused LM head: argmax of W . x without writing logits, ties -> lowest index;
 * with prob_out also p(top1) = 1 / sum exp(l - max):
 * matvec_q{4,5,6}_k_f32_argmax / _top1 (mps_backend.hpp:141-146, 162-167, 183-188; 579-749, 1554-1688). */
int kib_matvec_kquant_f32_argmax(kib_ctx* ctx, int type, const void* weight, uint64_t rows, uint64_t cols,
                                 const float* input, int32_t* token_out, float* prob_out);
/* The same fused LM-head argmax for callers that must not allocate device
 * memory (a host that owns all device memory through its own pool, or that
 * forbids allocations after start-up).  No counterpart in the reference: it
 * exists only in this backend.  Needs no kib_ctx; runs on the current device
 * and on `stream` (a cudaStream_t, NULL for the legacy default stream) and
 * returns once the kernel is queued: synchronise the stream before reading
 * token_out / prob_out.  Its scratch is one fixed array per device inside the
 * library (candidates of up to 1024 CTAs, i.e. devices of up to 1024 SMs;
 * larger devices get KIB_ERR_INVALID_ARGUMENT, as do cols not a multiple of
 * 256 or above 16384).  The first call on a device looks up that array's
 * address; make it before any stream capture.  Every call shares the array:
 * calls whose kernels may overlap on the GPU race and must be ordered by the
 * caller.  The return code covers argument checks and the launch only: a
 * bounded device wait that gives up inside the kernel (reported as
 * KIB_ERR_TIMEOUT by kib_matvec_kquant_f32_argmax) shows here as
 * token_out = -1 and prob_out = 0 once the stream has been synchronised. */
int kib_matvec_kquant_f32_argmax_noalloc(int type, const void* weight, uint64_t rows, uint64_t cols,
                                         const float* input, int32_t* token_out, float* prob_out, void* stream);
/* dequantize_rows_q{4,5,6}_k_f32 / q*_k_get_rows (mps_backend.hpp:201-221;
 * mps_backend.mm:1693-1824): out[i] = row row_ids[i]; out-of-range ids give zeros. */
int kib_dequantize_rows_kquant_f32(kib_ctx* ctx, int type, const void* weight, uint64_t rows,
                                   const int32_t* row_ids, uint64_t count, uint64_t cols, float* output);

/* Type-named forms of the reference (same semantics as the generic calls). */
int kib_matvec_q4_k_f32_device(kib_ctx* ctx, const void* w, uint64_t rows, uint64_t cols, const float* in, float* out);
int kib_matvec_q5_k_f32_device(kib_ctx* ctx, const void* w, uint64_t rows, uint64_t cols, const float* in, float* out);
int kib_matvec_q6_k_f32_device(kib_ctx* ctx, const void* w, uint64_t rows, uint64_t cols, const float* in, float* out);
int kib_matmul_q4_k_f32_device(kib_ctx* ctx, const void* w, uint64_t rows, uint64_t cols, uint64_t tokens,
                               const float* in, float* out);
int kib_matmul_q5_k_f32_device(kib_ctx* ctx, const void* w, uint64_t rows, uint64_t cols, uint64_t tokens,
                               const float* in, float* out);
int kib_matmul_q6_k_f32_device(kib_ctx* ctx, const void* w, uint64_t rows, uint64_t cols, uint64_t tokens,
                               const float* in, float* out);

/* ------------------------------------------------------------------- norms */
/* rms_norm_f32_f32(_batched) (mps_backend.hpp:234-238; mps_backend.mm:1863-1921). */
int kib_rms_norm_f32_f32_batched(kib_ctx* ctx, const float* input, const float* weight, uint64_t tokens,
                                 uint64_t size, float eps, float* output);
/* qk_norm_f32_f32_batched, in place per head (mps_backend.hpp:252; mps_backend.mm:1991-2024). */
int kib_qk_norm_f32_f32_batched(kib_ctx* ctx, float* values, const float* weight, uint64_t tokens, uint64_t heads,
                                uint64_t head_dim, float eps);
/* qwen35_norm_gated_f32_in_place (mps_backend.hpp:258; mps_backend.mm:2026-2063). */
int kib_qwen35_norm_gated_f32_in_place(kib_ctx* ctx, float* values, const float* weight, const float* gate,
                                       uint64_t tokens, uint64_t heads, uint64_t head_dim, float eps);
/* split_qkv_l2_norm_f32_qwen35 (mps_backend.hpp:266; mps_backend.mm:2097-2153). */
int kib_split_qkv_l2_norm_f32_qwen35(kib_ctx* ctx, const float* source, float* query, float* key, float* value,
                                     uint64_t tokens, uint64_t key_heads, uint64_t value_heads, uint64_t head_dim,
                                     float eps);

/* --------------------------------------------------------------------- GDN */
/* build_ssm_conv_state_f32 + ssm_conv_f32 (mps_backend.hpp:301-308;
 * mps_backend.mm:2376-2457): state [channels][K-1] is updated in place,
 * output [tokens][channels] (no activation). */
int kib_ssm_conv_f32_stateful(kib_ctx* ctx, float* state, const float* input, const float* weights,
                              uint64_t conv_kernel, uint64_t channels, uint64_t tokens, float* output);
/* prepare_qwen35_gdn_gate_beta_f32 (mps_backend.hpp:356; mps_backend.mm:2588-2605). */
int kib_prepare_qwen35_gdn_gate_beta_f32(kib_ctx* ctx, float* gate, float* beta, const float* gate_bias,
                                         const float* gate_scale, uint64_t tokens, uint64_t heads);
/* gated_delta_net_f32_batched_in_place(_at) (mps_backend.hpp:291-296;
 * mps_backend.mm:2225-2374): state [value_heads][d][d] updated in place. */
int kib_gated_delta_net_f32_batched_in_place(kib_ctx* ctx, const float* query, const float* key, const float* value,
                                             const float* gate, const float* beta, float* state, uint64_t tokens,
                                             uint64_t key_heads, uint64_t value_heads, uint64_t head_dim,
                                             float* output);

/* --------------------------------------------------------------- attention */
/* mrope_f32_in_place (mps_backend.hpp:331; mps_backend.mm:2482-2527);
 * positions is int32 [4][tokens]. */
int kib_mrope_f32_in_place(kib_ctx* ctx, float* values, const int32_t* positions, uint64_t tokens, uint64_t heads,
                           uint64_t head_dim, uint64_t n_dims, uint64_t s0, uint64_t s1, uint64_t s2, uint64_t s3,
                           float theta);
/* attention_f32_batched_f16_kv (mps_backend.hpp:415; mps_backend.mm:2943-3008,
 * flash256 3398-3643 for tokens >= 64): causal GQA over an F16 cache laid out
 * [layer][capacity][kv_heads*head_dim]. */
int kib_attention_f32_batched_f16_kv(kib_ctx* ctx, const float* query, const uint16_t* key_cache,
                                     const uint16_t* value_cache, uint64_t layer, uint64_t start_position,
                                     uint64_t tokens, uint64_t capacity_tokens, uint64_t heads, uint64_t kv_heads,
                                     uint64_t head_dim, float* output);

/* ------------------------------------------------------ element-wise + misc */
/* add/mul(_row)_f32_in_place, sigmoid/softplus/silu/silu_mul (mps_backend.hpp:342-360;
 * mps_backend.mm:2529-2629).  op: 0 add, 1 mul, 2 add_row, 3 mul_row. */
int kib_binary_f32_in_place(kib_ctx* ctx, int op, float* target, const float* rhs, uint64_t total, uint64_t row_size);
/* op: 0 sigmoid, 1 softplus (passthrough > 20), 2 silu. */
int kib_unary_f32_in_place(kib_ctx* ctx, int op, float* values, uint64_t size);
int kib_silu_mul_f32_in_place(kib_ctx* ctx, float* gate, const float* up, uint64_t size);
/* copy_f32_rows / copy_f32_rows_to_f16 (mps_backend.hpp:366-372; mps_backend.mm:2631-2679). */
int kib_copy_f32_rows(kib_ctx* ctx, const float* source, float* destination, uint64_t rows, uint64_t row_values,
                      uint64_t source_stride, uint64_t source_offset, uint64_t destination_stride,
                      uint64_t destination_offset);
int kib_copy_f32_rows_to_f16(kib_ctx* ctx, const float* source, uint16_t* destination, uint64_t rows,
                             uint64_t row_values, uint64_t source_stride, uint64_t source_offset,
                             uint64_t destination_stride, uint64_t destination_offset);
/* argmax_f32_i32 / argmax_prob_f32_i32 (mps_backend.hpp:384-387; mps_backend.mm:2681-2779). */
int kib_argmax_f32_i32(kib_ctx* ctx, const float* values, uint64_t size, int32_t* token_out, float* prob_out);

/* ------------------------------------------------- named and offset forms
 * The remaining MpsContext members on the Qwen3.5 path, same argument order
 * and meaning (offsets in elements, as the reference's validate_*_region). */
/* copy_to_buffer_at / copy_from_buffer_at (mps_backend.hpp:100-109; mps_backend.mm:5768-5830). */
int kib_copy_to_buffer_at(kib_ctx* ctx, void* buffer, uint64_t destination_offset, const void* data, uint64_t bytes);
int kib_copy_from_buffer_at(kib_ctx* ctx, const void* buffer, uint64_t source_offset, void* data, uint64_t bytes);
/* copy_f32_region (mps_backend.hpp:362-365; mps_backend.mm:2631-2640, 9634):
 * destination[destination_offset + i] = source[source_offset + i], i < size. */
int kib_copy_f32_region(kib_ctx* ctx, const float* source, float* destination, uint64_t source_offset,
                        uint64_t destination_offset, uint64_t size);
/* copy_f16_rows (mps_backend.hpp:377-383; mps_backend.mm:2668-2679, 9900). */
int kib_copy_f16_rows(kib_ctx* ctx, const uint16_t* source, uint16_t* destination, uint64_t rows, uint64_t row_size,
                      uint64_t source_stride, uint64_t source_offset, uint64_t destination_stride,
                      uint64_t destination_offset);
/* ssm_conv_f32 (mps_backend.hpp:301-307; mps_backend.mm:2376-2400, 8703): input
 * [sequences][channels][conv_kernel-1+tokens], kernel [channels][conv_kernel],
 * output [sequences][tokens][channels]; no activation. */
int kib_ssm_conv_f32(kib_ctx* ctx, const float* input, const float* kernel, uint64_t conv_kernel, uint64_t channels,
                     uint64_t tokens, uint64_t sequences, float* output);
/* build_ssm_conv_state_f32 (mps_backend.hpp:308-314; mps_backend.mm:2428-2456, 8801):
 * conv_input[channel] = [state row | the new inputs]; the state row (at
 * state + state_offset, [channels][conv_kernel-1]) becomes the window's tail. */
int kib_build_ssm_conv_state_f32(kib_ctx* ctx, float* state, uint64_t state_offset, const float* input,
                                 uint64_t conv_kernel, uint64_t channels, uint64_t tokens, float* conv_input);
/* ssm_conv1_f32_stateful(_at) (mps_backend.hpp:315-327; mps_backend.mm:2402-2426, 8904-8990). */
int kib_ssm_conv1_f32_stateful(kib_ctx* ctx, float* state, const float* input, const float* kernel,
                               uint64_t conv_kernel, uint64_t channels, float* output);
int kib_ssm_conv1_f32_stateful_at(kib_ctx* ctx, float* state, uint64_t state_offset, const float* input,
                                  const float* kernel, uint64_t conv_kernel, uint64_t channels, float* output);
/* gated_delta_net_f32_in_place(_at), gated_delta_net_f32_batched_in_place_at
 * (mps_backend.hpp:270-300): the batched op with tokens = 1 and/or the state at
 * state + state_offset. */
int kib_gated_delta_net_f32_in_place(kib_ctx* ctx, const float* query, const float* key, const float* value,
                                     const float* gate, const float* beta, float* state, uint64_t key_heads,
                                     uint64_t value_heads, uint64_t head_dim, float* output);
int kib_gated_delta_net_f32_in_place_at(kib_ctx* ctx, const float* query, const float* key, const float* value,
                                        const float* gate, const float* beta, float* state, uint64_t state_offset,
                                        uint64_t key_heads, uint64_t value_heads, uint64_t head_dim, float* output);
int kib_gated_delta_net_f32_batched_in_place_at(kib_ctx* ctx, const float* query, const float* key,
                                                const float* value, const float* gate, const float* beta,
                                                float* state, uint64_t state_offset, uint64_t tokens,
                                                uint64_t key_heads, uint64_t value_heads, uint64_t head_dim,
                                                float* output);
/* matvec_q{4,5,6}_k_f32_top1 / _argmax (mps_backend.hpp:141-149, 162-170, 183-191):
 * the fused LM-head argmax (ties to the lowest row) with and without p(top1). */
int kib_matvec_q4_k_f32_top1(kib_ctx* ctx, const void* weight, uint64_t rows, uint64_t cols, const float* input,
                             int32_t* token_out, float* probability_out);
int kib_matvec_q5_k_f32_top1(kib_ctx* ctx, const void* weight, uint64_t rows, uint64_t cols, const float* input,
                             int32_t* token_out, float* probability_out);
int kib_matvec_q6_k_f32_top1(kib_ctx* ctx, const void* weight, uint64_t rows, uint64_t cols, const float* input,
                             int32_t* token_out, float* probability_out);
int kib_matvec_q4_k_f32_argmax(kib_ctx* ctx, const void* weight, uint64_t rows, uint64_t cols, const float* input,
                               int32_t* token_out);
int kib_matvec_q5_k_f32_argmax(kib_ctx* ctx, const void* weight, uint64_t rows, uint64_t cols, const float* input,
                               int32_t* token_out);
int kib_matvec_q6_k_f32_argmax(kib_ctx* ctx, const void* weight, uint64_t rows, uint64_t cols, const float* input,
                               int32_t* token_out);
/* argmax_prob_f32_i32 (mps_backend.hpp:387-390). */
int kib_argmax_prob_f32_i32(kib_ctx* ctx, const float* values, uint64_t size, int32_t* token_out, float* prob_out);
/* dequantize_row_q{4,5,6}_k_f32 (mps_backend.hpp:196-225; mps_backend.mm:1693-1760): one row. */
int kib_dequantize_row_q4_k_f32(kib_ctx* ctx, const void* weight, uint64_t row, uint64_t cols, float* output);
int kib_dequantize_row_q5_k_f32(kib_ctx* ctx, const void* weight, uint64_t row, uint64_t cols, float* output);
int kib_dequantize_row_q6_k_f32(kib_ctx* ctx, const void* weight, uint64_t row, uint64_t cols, float* output);
/* rms_norm_f32_f32, qk_norm_f32_f32, attention_f32_f16_kv (mps_backend.hpp:230-250, 397-401):
 * the batched ops with one token (attention: the query at `position`). */
int kib_rms_norm_f32_f32(kib_ctx* ctx, const float* input, const float* weight, uint64_t size, float eps,
                         float* output);
int kib_qk_norm_f32_f32(kib_ctx* ctx, float* values, const float* weight, uint64_t heads, uint64_t head_dim,
                        float eps);
int kib_attention_f32_f16_kv(kib_ctx* ctx, const float* query, const uint16_t* key_cache,
                             const uint16_t* value_cache, uint64_t layer, uint64_t position, uint64_t capacity_tokens,
                             uint64_t heads, uint64_t kv_heads, uint64_t head_dim, float* output);

/* ================================================================ runtime */

typedef struct kib_qwen35 kib_qwen35;

/* Qwen35RuntimeOptions (qwen35_runtime.hpp:16-24). */
typedef struct kib_qwen35_options {
  uint64_t context_tokens;       /* 0: sized from the request */
  uint64_t decode_tokens;
  uint64_t prefill_chunk_tokens; /* default 1024 */
  uint64_t sequence_slots;       /* 1 */
  int kv_cache_f16;              /* only 1 is supported (the reference default) */
  int enable_mtp;                /* allocate the MTP/NextN cache if the GGUF has one */
} kib_qwen35_options;

/* Qwen35ExecutionPlan + Qwen35CachePlan (qwen35_runtime.hpp:26-68). */
typedef struct kib_qwen35_plan {
  uint64_t hidden_size, main_layers, total_layers, head_dim, attention_heads, kv_heads;
  uint64_t linear_key_heads, linear_value_heads, linear_key_head_dim, linear_value_head_dim;
  uint64_t linear_inner_size, linear_conv_kernel, linear_conv_channels;
  uint64_t intermediate_size, vocab_size;
  uint64_t attention_capacity_tokens, full_attention_layers, linear_attention_layers, kv_dim;
  uint64_t recurrent_r_elements_per_layer, recurrent_s_elements_per_layer;
  uint64_t kv_cache_bytes, recurrent_r_cache_bytes, recurrent_s_cache_bytes, total_cache_bytes;
  uint64_t weight_bytes;
  int mtp_layers;
  int layer_kinds[64]; /* 0 linear attention, 1 full attention */
} kib_qwen35_plan;

/* CpuMtpReport (cpu_inference.hpp:79-94). */
typedef struct kib_mtp_report {
  int available, enabled;
  uint64_t draft_tokens;
  double p_min;
  uint64_t drafted_tokens, accepted_tokens, verify_steps, confidence_stops;
  uint64_t adaptive_budget, adaptive_changes;
  uint64_t verified_by_position[8];
  uint64_t accepted_by_position[8];
} kib_mtp_report;

/* CpuGenerationRequest subset that reaches the Qwen3.5 path (cpu_inference.hpp:30-53);
 * prompts are token ids (tokenization is outside this backend). */
typedef struct kib_generation_request {
  const int32_t* prompt_tokens;
  uint64_t prompt_count;
  uint64_t max_new_tokens;
  uint64_t prefill_chunk_tokens; /* 0 -> 1024 */
  int enable_mtp;
  uint64_t mtp_draft_tokens;     /* default 3 */
  double mtp_p_min;              /* default 0.30; 0 disables the confidence stop */
  int mtp_adaptive;              /* 1: reference adaptive budget (start 1); 0: fixed budget */
  int ignore_eos;                /* benchmarks: do not stop at EOS */
  uint64_t eos_token_id;         /* in addition to 151643; UINT64_MAX for none */
} kib_generation_request;

/* CpuGenerationResult subset (cpu_inference.hpp:96-115) plus device timings. */
typedef struct kib_generation_result {
  uint64_t prompt_tokens;
  uint64_t generated_tokens;
  int finish_reason_stop; /* 1 "stop", 0 "length" */
  kib_mtp_report mtp;
  uint64_t kv_used_tokens;
  double prefill_ms, decode_ms;
} kib_generation_result;

/* read_gguf_file + build_qwen35_weight_map + build_qwen35_execution_plan +
 * upload_qwen35_metal_weights + allocate_qwen35_metal_cache
 * (gguf_reader.cpp:466-519; qwen35_weight_map.cpp:314-454;
 * qwen35_runtime.cpp:4380-4526, 1252-1528): weights are uploaded as stored. */
int kib_qwen35_load(kib_ctx* ctx, const char* gguf_path, const kib_qwen35_options* options, kib_qwen35** out);
void kib_qwen35_free(kib_qwen35* model);
int kib_qwen35_get_plan(const kib_qwen35* model, kib_qwen35_plan* plan);

/* generate_qwen35_metal (qwen35_runtime.hpp:176; qwen35_runtime.cpp:5239-6714):
 * chunked prefill, then greedy decode or the MTP draft -> verify -> greedy
 * accept loop.  out_tokens receives up to out_capacity generated ids. */
int kib_generate_qwen35(kib_qwen35* model, const kib_generation_request* request, int32_t* out_tokens,
                        uint64_t out_capacity, kib_generation_result* result);

/* Engine steps used by tests and benchmarks (the same calls generate makes). */
/* Reset caches to the empty state (position 0). */
int kib_qwen35_reset(kib_qwen35* model);
/* Chunked prefill of n tokens at the current position; writes the greedy
 * next token (argmax of the last row). */
int kib_qwen35_prefill(kib_qwen35* model, const int32_t* tokens, uint64_t n, uint64_t chunk, int32_t* next_token);
/* One forward over n (1..8) tokens at the current position (no cache reset);
 * writes per-row argmax tokens and, if logits is non-null, [n][vocab] logits.
 * advance != 0 moves the position by n. */
int kib_qwen35_forward(kib_qwen35* model, const int32_t* tokens, uint64_t n, int advance, int32_t* argmax_out,
                       float* logits, float* normed_hidden);
/* `steps` greedy decode steps from `first_token`, each step's input being the
 * previous step's argmax, replayed from one CUDA graph with the token and the
 * position kept on the device.  tokens_out[i] is the argmax after step i. */
int kib_qwen35_decode_greedy(kib_qwen35* model, int32_t first_token, uint64_t steps, int32_t* tokens_out);
/* Current position (tokens in the KV cache). */
uint64_t kib_qwen35_position(const kib_qwen35* model);
int kib_qwen35_set_position(kib_qwen35* model, uint64_t position);
/* Test hook, no counterpart in the reference: lowers the persistent decode
 * kernel's cell-poll limit to poll_limit (0 restores the default) and, when
 * stage >= 0, makes that GEMV stage wait for an input tag no stage writes, so
 * the next decode step's bounded waits run out: the step returns
 * KIB_ERR_TIMEOUT and the model stays usable (state of the aborted step is
 * undefined; reset and prefill again).  stage = -1 restores the stage list. */
int kib_qwen35_debug_stall(kib_qwen35* model, uint32_t poll_limit, int stage);
/* No counterpart in the reference: which bs1 decode path the model runs.
 * Returns the persistent kernel's stage count (> 0), or 0 when decode runs as
 * the per-kernel graph, with the reason (e.g. a matrix type or shape outside
 * the persistent kernel's limits) copied into why (may be null). */
int kib_qwen35_persistent_stages(const kib_qwen35* model, char* why, int why_len);
/* Copies cache state out of (write_into_model = 0) or into (1) the engine: any
 * pointer may be null.  Host buffers; sizes from kib_qwen35_plan. */
int kib_qwen35_state_io(kib_qwen35* model, int write_into_model, uint16_t* k_cache, uint16_t* v_cache,
                        float* r_cache, float* s_cache, uint16_t* mtp_k, uint16_t* mtp_v, float* pending_h);
/* MTP/NextN layer over n tokens at the current position: (ids, h rows) ->
 * normed h_nextn rows and per-row argmax of the LM head; writes the MTP KV cache
 * (run_qwen35_mtp_tokens, qwen35_runtime.cpp:4111-4240). */
int kib_qwen35_mtp_forward(kib_qwen35* model, const int32_t* tokens, const float* h_rows, uint64_t n,
                           uint64_t position, int32_t* argmax_out, float* h_nextn_out);

/* ------------------------------------------------------- batched decode
 * Independent sequences decoded together, one token per sequence per step:
 * the plan's sequence_slots (qwen35_runtime.hpp:20, qwen35_runtime.cpp:
 * 4478-4479), which the reference reserves but does not run.  A batch owns
 * each slot's KV cache (context_tokens positions), conv and delta-rule state;
 * it shares the model's weights and scratch, so calls on one model must not
 * overlap.  The projections of a step are one GEMM over the slots: every slot
 * gets the reference's M > 8 matmul numerics (half-rounded weights and
 * inputs, fp32 accumulation), hence 9 <= slots <= the prefill chunk. */
typedef struct kib_qwen35_batch kib_qwen35_batch;
int kib_qwen35_batch_create(kib_qwen35* model, uint64_t slots, uint64_t context_tokens, uint64_t max_steps,
                            kib_qwen35_batch** out);
void kib_qwen35_batch_free(kib_qwen35_batch* batch);
/* Prefills one slot through the model's own prefill (the model's
 * single-sequence state is reset and then holds this prompt), copies the
 * caches into the slot and returns the prompt's greedy next token. */
int kib_qwen35_batch_prefill(kib_qwen35_batch* batch, uint64_t slot, const int32_t* tokens, uint64_t count,
                             int32_t* next_token);
/* steps greedy steps for every slot, starting from first_tokens[slots];
 * tokens_out[step * slots + slot] receives the argmax of each step. */
int kib_qwen35_batch_decode(kib_qwen35_batch* batch, const int32_t* first_tokens, uint64_t steps,
                            int32_t* tokens_out);
uint64_t kib_qwen35_batch_position(const kib_qwen35_batch* batch, uint64_t slot);
/* The logits of the last batched step, [slots][vocab] (host copy). */
int kib_qwen35_batch_logits(kib_qwen35_batch* batch, float* logits_out);

/* --------------------------------------------------- host prompt cache
 * Qwen35HostPrefixCache (qwen35_runtime.cpp:516-932) on this backend: after
 * each full block of a prefill, the block's K/V rows, the conv and delta-rule
 * state and the block's last hidden row go to host memory under the block's
 * chained hash; kib_qwen35_prefill_cached resets the model, restores the
 * longest stored block-aligned prefix of the prompt into the device caches
 * and prefills only the rest (the whole prompt hit: the next token comes from
 * the restored hidden row).  block_tokens <= the prefill chunk.  Not for use
 * with MTP (the reference disables its prompt cache then too). */
typedef struct kib_qwen35_prefix_cache kib_qwen35_prefix_cache;
int kib_qwen35_prefix_cache_create(kib_qwen35* model, uint64_t block_tokens, uint64_t capacity_blocks,
                                   uint64_t min_reuse_tokens, kib_qwen35_prefix_cache** out);
void kib_qwen35_prefix_cache_free(kib_qwen35_prefix_cache* cache);
/* stored blocks, hit tokens, miss tokens, committed tokens, evicted blocks, block tokens. */
void kib_qwen35_prefix_cache_stats(const kib_qwen35_prefix_cache* cache, uint64_t* out6);
int kib_qwen35_prefill_cached(kib_qwen35* model, kib_qwen35_prefix_cache* cache, const int32_t* tokens,
                              uint64_t count, int32_t* next_token, uint64_t* hit_tokens);

/* Streaming generate (the reference's per-token stream_token callback,
 * emit_generated_token in qwen35_runtime.cpp:6128-6139, which feeds the
 * gateway's SSE responses): as kib_generate_qwen35, and every committed token is passed
 * to cb(user, token, index) as soon as the host has it; a nonzero return
 * cancels (finish_reason_stop stays 0).  cache (may be NULL): prefill through
 * the host prompt cache, its hit length in *cached_tokens. */
typedef int (*kib_token_callback)(void* user, int32_t token, uint64_t index);
int kib_generate_qwen35_stream(kib_qwen35* model, const kib_generation_request* request,
                               kib_qwen35_prefix_cache* cache, kib_token_callback cb, void* user, int32_t* out_tokens,
                               uint64_t out_capacity, kib_generation_result* result, uint64_t* cached_tokens);

/* Synthetic BASELINE-shaped Qwen3.5 GGUF writer (random-init weights, Q4_K_M mix). */
typedef struct kib_synth_config {
  uint64_t hidden, layers, intermediate, vocab, heads, kv_heads, head_dim;
  uint64_t ssm_heads, ssm_head_dim, conv_kernel, full_attention_interval, nextn_layers;
  uint32_t proj_type, down_type, embd_type;
  uint64_t seed;
  double rope_theta, rms_eps;
  int64_t eos_token_id;
  int threads;
  uint32_t qkv_type; /* GDN attn_qkv type; 0: proj_type (Q4_K_M files store it as Q5_K, 13) */
} kib_synth_config;
void kib_synth_default(kib_synth_config* cfg);
int kib_write_synthetic_qwen35(const char* path, const kib_synth_config* cfg, char* err, int err_len);
/* Raw K-quant quantizers used by the writer (n multiple of 256). */
int kib_quantize_kquant(int type, const float* x, uint64_t n, void* out);
/* Opens and validates a GGUF file on the host only (header, metadata, tensor
 * directory, every tensor's data inside the file), as the loader does before
 * it touches the device: KIB_ERR_INVALID_ARGUMENT with the reason in err for a
 * truncated or corrupt file (gguf_reader.cpp's checks). */
int kib_gguf_check(const char* path, char* err, int err_len, uint64_t* n_tensors);

/* ------------------------------------------------------- host prompt cache
 * Exact-prefix block index of the host prefix cache (Qwen35PrefixCacheIndex,
 * include/toyllm/runtime/qwen35_prefix_cache.hpp:52-79;
 * src/runtime/qwen35_prefix_cache.cpp): blocks of block_tokens chained by
 * hash, LRU eviction at capacity_blocks, hits below min_reuse_tokens ignored.
 * Host only (also exported by libkib_gguf.so). */
typedef struct kib_prefix_index kib_prefix_index;
kib_prefix_index* kib_prefix_index_create(uint64_t block_tokens, uint64_t capacity_blocks, uint64_t min_reuse_tokens);
void kib_prefix_index_free(kib_prefix_index* index);
/* Tokens of the longest stored prefix; its block hashes (up to max_hashes) into hashes_out. */
uint64_t kib_prefix_index_lookup(kib_prefix_index* index, const int64_t* tokens, uint64_t count, uint64_t* hashes_out,
                                 uint64_t max_hashes);
/* Commits block [start, start + block_tokens): returns inserted | evicted << 1, -1 on bad arguments. */
int kib_prefix_index_commit(kib_prefix_index* index, const int64_t* tokens, uint64_t count, uint64_t start,
                            uint64_t* hash_out, uint64_t* evicted_hash_out);
/* stored blocks, hit tokens, miss tokens, committed tokens, evicted blocks, block tokens. */
void kib_prefix_index_stats(const kib_prefix_index* index, uint64_t* out6);

/* ------------------------------------------------------- GGUF tokenizer
 * Byte-level BPE from the GGUF's tokenizer.ggml.* metadata, the Qwen3.5
 * pre-tokenizer and chat prompt (GgufTokenizer,
 * include/toyllm/runtime/gguf_tokenizer.hpp:27-66; src/runtime/gguf_tokenizer.cpp).
 * Host only (also exported by libkib_gguf.so).  Calls that produce ids or text
 * return the element count of the full result and write it only when it fits
 * in cap (call with out = NULL, cap = 0 to size the buffer); -1 on error, the
 * reference's message in kib_tokenizer_last_error. */
typedef struct kib_tokenizer kib_tokenizer;
/* load_gguf_tokenizer (gguf_tokenizer.cpp:628-677); NULL on error, reason in kib_tokenizer_load_error(). */
kib_tokenizer* kib_tokenizer_load(const char* gguf_path);
const char* kib_tokenizer_load_error(void);
void kib_tokenizer_free(kib_tokenizer* tok);
const char* kib_tokenizer_last_error(const kib_tokenizer* tok);
/* info9: tokens, merges, bos, eos, pad, add_bos, add_eos, <|im_start|> id, <|im_end|> id (-1 when absent). */
void kib_tokenizer_info(const kib_tokenizer* tok, int64_t* info9);
/* which: 0 tokenizer.ggml.model, 1 tokenizer.ggml.pre, 2 tokenizer.chat_template. */
int64_t kib_tokenizer_meta(const kib_tokenizer* tok, int which, char* out, uint64_t cap);
/* gguf_token_id (gguf_tokenizer.cpp:679-686): -1 when absent. */
int64_t kib_tokenizer_token_id(const kib_tokenizer* tok, const char* text, uint64_t len);
int64_t kib_tokenizer_token_text(const kib_tokenizer* tok, int64_t id, char* out, uint64_t cap);
int64_t kib_tokenizer_token_type(const kib_tokenizer* tok, int64_t id);
/* gguf_token_is_control (gguf_tokenizer.cpp:688-695): control or unused. */
int kib_tokenizer_is_control(const kib_tokenizer* tok, int64_t id);
/* gguf_encode_text (gguf_tokenizer.cpp:697-738). */
int64_t kib_tokenizer_encode(kib_tokenizer* tok, const char* text, uint64_t len, int add_special, int parse_special,
                             int64_t* out, uint64_t cap);
/* gguf_decode_token_text (gguf_tokenizer.cpp:751-775). */
int64_t kib_tokenizer_decode(kib_tokenizer* tok, const int64_t* ids, uint64_t count, int skip_control, char* out,
                             uint64_t cap);
/* format_qwen35_chat_prompt (gguf_tokenizer.cpp:777-809): n messages of (role, content), NUL-terminated. */
int64_t kib_tokenizer_format_chat(kib_tokenizer* tok, const char* const* roles, const char* const* contents,
                                  uint64_t n, int add_generation_prompt, int enable_thinking, char* out, uint64_t cap);
/* gguf_encode_qwen35_chat_prompt (gguf_tokenizer.cpp:740-749). */
int64_t kib_tokenizer_encode_chat(kib_tokenizer* tok, const char* const* roles, const char* const* contents,
                                  uint64_t n, int add_generation_prompt, int enable_thinking, int64_t* out,
                                  uint64_t cap);

#ifdef __cplusplus
}
#endif

#endif /* KIB_H_ */
