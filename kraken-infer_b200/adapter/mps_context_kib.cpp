// mps_context_kib.cpp -- toyllm::mps::MpsContext implemented on the B200
// backend's C ABI (include/kib.h), for kraken-infer builds that select the CUDA
// backend in place of the Metal one.  It defines the same classes the
// reference's src/backends/mps/mps_backend.mm (or mps_backend_stub.cpp)
// defines, against the reference's unchanged header
// include/toyllm/backends/mps/mps_backend.hpp, so the runtime links either one.
//
// Ownership follows the reference's pimpl: an MpsBuffer owns one device
// allocation (kib_make_buffer / kib_free_buffer) of byte_size() bytes; the
// MpsContext owns one kib_ctx (a CUDA stream on one B200).  Shapes are checked
// against the buffers' sizes before any launch, as the reference's
// validate_f32_buffer does, and kib status codes map to Status one to one.
// Members outside the Qwen3.5 decode / verify path (bf16 weights, the
// non-F16 KV attention, rope_f32, the matvec workspace forms) report
// Status::unavailable.
#include <cstring>
#include <string>
#include <utility>
#include <vector>

#include "kib.h"
#include "toyllm/backends/mps/mps_backend.hpp"

namespace toyllm::mps {

struct MpsBuffer::Impl {
  kib_ctx* ctx = nullptr;
  void* dev = nullptr;
  std::size_t bytes = 0;
  ~Impl() {
    if (dev) kib_free_buffer(ctx, dev);
  }
};

MpsBuffer::MpsBuffer() = default;
MpsBuffer::~MpsBuffer() = default;
MpsBuffer::MpsBuffer(MpsBuffer&& other) noexcept = default;
MpsBuffer& MpsBuffer::operator=(MpsBuffer&& other) noexcept = default;
MpsBuffer::MpsBuffer(std::unique_ptr<Impl> impl) : impl_(std::move(impl)) {}
bool MpsBuffer::valid() const { return impl_ && impl_->dev; }
std::size_t MpsBuffer::byte_size() const { return impl_ ? impl_->bytes : 0; }

// MpsContext is MpsBuffer's friend, and so are MpsContext's member classes:
// the buffer accessors live in MpsContext::Impl.
struct MpsContext::Impl {
  kib_ctx* ctx = nullptr;
  ~Impl() {
    if (ctx) kib_destroy(ctx);
  }
  template <typename T>
  static T* dptr(const MpsBuffer& b) {
    return static_cast<T*>(b.impl_ ? b.impl_->dev : nullptr);
  }
  // The buffer holds at least `count` elements of T.
  template <typename T>
  static bool fits(const MpsBuffer& b, std::size_t count) {
    return b.valid() && count <= b.byte_size() / sizeof(T);
  }
  static Status binary(kib_ctx* c, int op, MpsBuffer& target, const MpsBuffer& rhs, std::size_t total,
                       std::size_t row);
};

namespace {

Status to_status(kib_ctx* c, int rc) {
  switch (rc) {
    case KIB_OK: return Status::ok();
    case KIB_ERR_INVALID_ARGUMENT: return Status::invalid_argument(kib_last_error(c));
    case KIB_ERR_UNAVAILABLE: return Status::unavailable(kib_last_error(c));
    case KIB_ERR_TIMEOUT: return Status::internal_error(std::string("device wait timed out: ") + kib_last_error(c));
    default: return Status::internal_error(kib_last_error(c));
  }
}

}  // namespace

MpsContext::MpsContext() = default;
MpsContext::~MpsContext() = default;
MpsContext::MpsContext(MpsContext&& other) noexcept = default;
MpsContext& MpsContext::operator=(MpsContext&& other) noexcept = default;
MpsContext::MpsContext(std::unique_ptr<Impl> impl) : impl_(std::move(impl)) {}

Result<MpsContext> MpsContext::create() {
  auto impl = std::make_unique<Impl>();
  const int rc = kib_create(0, &impl->ctx);
  if (rc != KIB_OK) return Status::unavailable("no sm_100 CUDA device for the B200 backend");
  return MpsContext(std::move(impl));
}

bool MpsContext::valid() const { return impl_ && kib_valid(impl_->ctx); }

#define KIB_CTX_OR_UNAVAILABLE()                                                    \
  if (!valid()) return Status::unavailable("B200 backend context is not initialized"); \
  kib_ctx* c = impl_->ctx

Status MpsContext::begin_graph() const {
  KIB_CTX_OR_UNAVAILABLE();
  return to_status(c, kib_begin_graph(c));
}
Status MpsContext::commit_graph() const {
  KIB_CTX_OR_UNAVAILABLE();
  return to_status(c, kib_commit_graph(c));
}
void MpsContext::abort_graph() const {
  if (valid()) kib_abort_graph(impl_->ctx);
}

Result<MpsBuffer> MpsContext::make_buffer(std::size_t byte_size) const {
  if (!valid()) return Status::unavailable("B200 backend context is not initialized");
  if (byte_size == 0) return Status::invalid_argument("MPS buffer size must be positive");
  auto b = std::make_unique<MpsBuffer::Impl>();
  b->ctx = impl_->ctx;
  b->bytes = byte_size;
  if (int rc = kib_make_buffer(impl_->ctx, byte_size, &b->dev); rc != KIB_OK) return to_status(impl_->ctx, rc);
  if (int rc = kib_zero_buffer(impl_->ctx, b->dev, byte_size); rc != KIB_OK) return to_status(impl_->ctx, rc);
  return MpsBuffer(std::move(b));
}

Status MpsContext::copy_to_buffer(MpsBuffer& buffer, const void* data, std::size_t byte_size) const {
  return copy_to_buffer_at(buffer, 0, data, byte_size);
}
Status MpsContext::copy_to_buffer_at(MpsBuffer& buffer, std::size_t destination_offset, const void* data,
                                     std::size_t byte_size) const {
  KIB_CTX_OR_UNAVAILABLE();
  if (!buffer.valid() || destination_offset > buffer.byte_size() ||
      byte_size > buffer.byte_size() - destination_offset)
    return Status::invalid_argument("MPS buffer copy exceeds buffer size");
  return to_status(c, kib_copy_to_buffer_at(c, Impl::dptr<void>(buffer), destination_offset, data, byte_size));
}
Status MpsContext::copy_from_buffer(const MpsBuffer& buffer, void* data, std::size_t byte_size) const {
  return copy_from_buffer_at(buffer, 0, data, byte_size);
}
Status MpsContext::copy_from_buffer_at(const MpsBuffer& buffer, std::size_t source_offset, void* data,
                                       std::size_t byte_size) const {
  KIB_CTX_OR_UNAVAILABLE();
  if (!buffer.valid() || source_offset > buffer.byte_size() || byte_size > buffer.byte_size() - source_offset)
    return Status::invalid_argument("MPS buffer copy exceeds buffer size");
  return to_status(c, kib_copy_from_buffer_at(c, Impl::dptr<void>(buffer), source_offset, data, byte_size));
}
Status MpsContext::copy_buffer_region(const MpsBuffer& source, MpsBuffer& destination, std::size_t source_offset,
                                      std::size_t destination_offset, std::size_t byte_size) const {
  KIB_CTX_OR_UNAVAILABLE();
  if (!Impl::fits<uint8_t>(source, source_offset + byte_size) || !Impl::fits<uint8_t>(destination, destination_offset + byte_size))
    return Status::invalid_argument("MPS buffer region exceeds buffer size");
  return to_status(c, kib_copy_buffer_region(c, Impl::dptr<void>(source), Impl::dptr<void>(destination), source_offset,
                                             destination_offset, byte_size));
}
Status MpsContext::zero_buffer(MpsBuffer& buffer, std::size_t byte_size) const {
  KIB_CTX_OR_UNAVAILABLE();
  if (!Impl::fits<uint8_t>(buffer, byte_size)) return Status::invalid_argument("MPS zero exceeds buffer size");
  return to_status(c, kib_zero_buffer(c, Impl::dptr<void>(buffer), byte_size));
}

// ---- K-quant
namespace {
constexpr int kQ4K = 12, kQ5K = 13, kQ6K = 14;
std::size_t kquant_bytes(int type, std::size_t rows, std::size_t cols) {
  const std::size_t per = type == kQ4K ? 144 : type == kQ5K ? 176 : 210;
  return rows * (cols / 256) * per;
}
}  // namespace

#define KIB_KQUANT_MEMBERS(NAME, TYPE)                                                                          \
  Status MpsContext::matvec_##NAME##_f32_device(const MpsBuffer& weight, std::size_t rows, std::size_t cols,  \
                                                const MpsBuffer& input, MpsBuffer& output) const {          \
    KIB_CTX_OR_UNAVAILABLE();                                                                                \
    if (cols % 256 || !Impl::fits<uint8_t>(weight, kquant_bytes(TYPE, rows, cols)) || !Impl::fits<float>(input, cols) || \
        !Impl::fits<float>(output, rows))                                                                          \
      return Status::invalid_argument("MPS " #NAME " matvec buffers do not match the shape");               \
    return to_status(c, kib_matvec_kquant_f32(c, TYPE, Impl::dptr<void>(weight), rows, cols, Impl::dptr<float>(input),  \
                                              Impl::dptr<float>(output)));                                         \
  }                                                                                                          \
  Status MpsContext::matmul_##NAME##_f32_device(const MpsBuffer& weight, std::size_t rows, std::size_t cols,  \
                                                std::size_t tokens, const MpsBuffer& input,                  \
                                                MpsBuffer& output) const {                                   \
    KIB_CTX_OR_UNAVAILABLE();                                                                                \
    if (cols % 256 || !Impl::fits<uint8_t>(weight, kquant_bytes(TYPE, rows, cols)) ||                              \
        !Impl::fits<float>(input, cols * tokens) || !Impl::fits<float>(output, rows * tokens))                           \
      return Status::invalid_argument("MPS " #NAME " matmul buffers do not match the shape");               \
    return to_status(c, kib_matmul_kquant_f32(c, TYPE, Impl::dptr<void>(weight), rows, cols, tokens,               \
                                              Impl::dptr<float>(input), Impl::dptr<float>(output)));                     \
  }                                                                                                          \
  Status MpsContext::matvec_##NAME##_f32_top1(const MpsBuffer& weight, std::size_t rows, std::size_t cols,    \
                                              const MpsBuffer& input, MpsBuffer& token_output,               \
                                              MpsBuffer& probability_output) const {                         \
    KIB_CTX_OR_UNAVAILABLE();                                                                                \
    if (cols % 256 || !Impl::fits<uint8_t>(weight, kquant_bytes(TYPE, rows, cols)) || !Impl::fits<float>(input, cols) || \
        !Impl::fits<int32_t>(token_output, 1) || !Impl::fits<float>(probability_output, 1))                              \
      return Status::invalid_argument("MPS " #NAME " top1 buffers do not match the shape");                 \
    return to_status(c, kib_matvec_kquant_f32_argmax(c, TYPE, Impl::dptr<void>(weight), rows, cols,                \
                                                     Impl::dptr<float>(input), Impl::dptr<int32_t>(token_output),        \
                                                     Impl::dptr<float>(probability_output)));                      \
  }                                                                                                          \
  Status MpsContext::matvec_##NAME##_f32_argmax(const MpsBuffer& weight, std::size_t rows, std::size_t cols,  \
                                                const MpsBuffer& input, MpsBuffer& token_output) const {    \
    KIB_CTX_OR_UNAVAILABLE();                                                                                \
    if (cols % 256 || !Impl::fits<uint8_t>(weight, kquant_bytes(TYPE, rows, cols)) || !Impl::fits<float>(input, cols) || \
        !Impl::fits<int32_t>(token_output, 1))                                                                     \
      return Status::invalid_argument("MPS " #NAME " argmax buffers do not match the shape");               \
    return to_status(c, kib_matvec_kquant_f32_argmax(c, TYPE, Impl::dptr<void>(weight), rows, cols,                \
                                                     Impl::dptr<float>(input), Impl::dptr<int32_t>(token_output),        \
                                                     nullptr));                                              \
  }                                                                                                          \
  Status MpsContext::dequantize_rows_##NAME##_f32(const MpsBuffer& weight, std::size_t rows,                  \
                                                  const MpsBuffer& row_ids, std::size_t tokens,              \
                                                  std::size_t cols, MpsBuffer& output) const {               \
    KIB_CTX_OR_UNAVAILABLE();                                                                                \
    if (cols % 256 || !Impl::fits<uint8_t>(weight, kquant_bytes(TYPE, rows, cols)) ||                              \
        !Impl::fits<int32_t>(row_ids, tokens) || !Impl::fits<float>(output, tokens * cols))                              \
      return Status::invalid_argument("MPS " #NAME " get_rows buffers do not match the shape");             \
    return to_status(c, kib_dequantize_rows_kquant_f32(c, TYPE, Impl::dptr<void>(weight), rows,                    \
                                                       Impl::dptr<int32_t>(row_ids), tokens, cols,                 \
                                                       Impl::dptr<float>(output)));                                \
  }                                                                                                          \
  Status MpsContext::dequantize_row_##NAME##_f32(const MpsBuffer& weight, std::size_t row, std::size_t cols,  \
                                                 MpsBuffer& output) const {                                  \
    KIB_CTX_OR_UNAVAILABLE();                                                                                \
    if (cols % 256 || !Impl::fits<uint8_t>(weight, kquant_bytes(TYPE, row + 1, cols)) || !Impl::fits<float>(output, cols)) \
      return Status::invalid_argument("MPS " #NAME " dequantize_row buffers do not match the shape");       \
    return to_status(c, kib_dequantize_row_##NAME##_f32(c, Impl::dptr<void>(weight), row, cols, Impl::dptr<float>(output))); \
  }

KIB_KQUANT_MEMBERS(q4_k, kQ4K)
KIB_KQUANT_MEMBERS(q5_k, kQ5K)
KIB_KQUANT_MEMBERS(q6_k, kQ6K)

// ---- norms
Status MpsContext::rms_norm_f32_f32(const MpsBuffer& input, const MpsBuffer& weight, std::size_t size, float eps,
                                    MpsBuffer& output) const {
  return rms_norm_f32_f32_batched(input, weight, 1, size, eps, output);
}
Status MpsContext::rms_norm_f32_f32_batched(const MpsBuffer& input, const MpsBuffer& weight, std::size_t tokens,
                                            std::size_t size, float eps, MpsBuffer& output) const {
  KIB_CTX_OR_UNAVAILABLE();
  if (!Impl::fits<float>(input, tokens * size) || !Impl::fits<float>(weight, size) || !Impl::fits<float>(output, tokens * size))
    return Status::invalid_argument("MPS RMSNorm buffers do not match the shape");
  return to_status(c, kib_rms_norm_f32_f32_batched(c, Impl::dptr<float>(input), Impl::dptr<float>(weight), tokens, size, eps,
                                                   Impl::dptr<float>(output)));
}
Status MpsContext::qk_norm_f32_f32(MpsBuffer& values, const MpsBuffer& weight, std::size_t heads,
                                   std::size_t head_dim, float eps) const {
  return qk_norm_f32_f32_batched(values, weight, 1, heads, head_dim, eps);
}
Status MpsContext::qk_norm_f32_f32_batched(MpsBuffer& values, const MpsBuffer& weight, std::size_t tokens,
                                           std::size_t heads, std::size_t head_dim, float eps) const {
  KIB_CTX_OR_UNAVAILABLE();
  if (!Impl::fits<float>(values, tokens * heads * head_dim) || !Impl::fits<float>(weight, head_dim))
    return Status::invalid_argument("MPS q/k norm buffers do not match the shape");
  return to_status(c, kib_qk_norm_f32_f32_batched(c, Impl::dptr<float>(values), Impl::dptr<float>(weight), tokens, heads,
                                                  head_dim, eps));
}
Status MpsContext::qwen35_norm_gated_f32_in_place(MpsBuffer& values, const MpsBuffer& weight, const MpsBuffer& gate,
                                                  std::size_t tokens, std::size_t heads, std::size_t head_dim,
                                                  float eps) const {
  KIB_CTX_OR_UNAVAILABLE();
  const std::size_t n = tokens * heads * head_dim;
  if (!Impl::fits<float>(values, n) || !Impl::fits<float>(gate, n) || !Impl::fits<float>(weight, head_dim))
    return Status::invalid_argument("MPS norm-gated buffers do not match the shape");
  return to_status(c, kib_qwen35_norm_gated_f32_in_place(c, Impl::dptr<float>(values), Impl::dptr<float>(weight),
                                                         Impl::dptr<float>(gate), tokens, heads, head_dim, eps));
}
Status MpsContext::split_qkv_l2_norm_f32_qwen35(const MpsBuffer& source, MpsBuffer& query, MpsBuffer& key,
                                                MpsBuffer& value, std::size_t tokens, std::size_t key_heads,
                                                std::size_t value_heads, std::size_t head_dim, float eps) const {
  KIB_CTX_OR_UNAVAILABLE();
  const std::size_t kd = key_heads * head_dim, vd = value_heads * head_dim;
  if (!Impl::fits<float>(source, tokens * (2 * kd + vd)) || !Impl::fits<float>(query, tokens * kd) ||
      !Impl::fits<float>(key, tokens * kd) || !Impl::fits<float>(value, tokens * vd))
    return Status::invalid_argument("MPS split-qkv buffers do not match the shape");
  return to_status(c, kib_split_qkv_l2_norm_f32_qwen35(c, Impl::dptr<float>(source), Impl::dptr<float>(query), Impl::dptr<float>(key),
                                                       Impl::dptr<float>(value), tokens, key_heads, value_heads, head_dim,
                                                       eps));
}

// ---- gated delta net
Status MpsContext::gated_delta_net_f32_batched_in_place_at(const MpsBuffer& query, const MpsBuffer& key,
                                                           const MpsBuffer& value, const MpsBuffer& gate,
                                                           const MpsBuffer& beta, MpsBuffer& state,
                                                           std::size_t state_offset, std::size_t tokens,
                                                           std::size_t key_heads, std::size_t value_heads,
                                                           std::size_t head_dim, MpsBuffer& output) const {
  KIB_CTX_OR_UNAVAILABLE();
  const std::size_t kd = key_heads * head_dim, vd = value_heads * head_dim;
  if (!Impl::fits<float>(query, tokens * kd) || !Impl::fits<float>(key, tokens * kd) || !Impl::fits<float>(value, tokens * vd) ||
      !Impl::fits<float>(gate, tokens * value_heads) || !Impl::fits<float>(beta, tokens * value_heads) ||
      !Impl::fits<float>(state, state_offset + value_heads * head_dim * head_dim) || !Impl::fits<float>(output, tokens * vd))
    return Status::invalid_argument("MPS gated delta net buffers do not match the shape");
  return to_status(c, kib_gated_delta_net_f32_batched_in_place_at(
                          c, Impl::dptr<float>(query), Impl::dptr<float>(key), Impl::dptr<float>(value), Impl::dptr<float>(gate),
                          Impl::dptr<float>(beta), Impl::dptr<float>(state), state_offset, tokens, key_heads, value_heads,
                          head_dim, Impl::dptr<float>(output)));
}
Status MpsContext::gated_delta_net_f32_batched_in_place(const MpsBuffer& query, const MpsBuffer& key,
                                                        const MpsBuffer& value, const MpsBuffer& gate,
                                                        const MpsBuffer& beta, MpsBuffer& state, std::size_t tokens,
                                                        std::size_t key_heads, std::size_t value_heads,
                                                        std::size_t head_dim, MpsBuffer& output) const {
  return gated_delta_net_f32_batched_in_place_at(query, key, value, gate, beta, state, 0, tokens, key_heads,
                                                 value_heads, head_dim, output);
}
Status MpsContext::gated_delta_net_f32_in_place_at(const MpsBuffer& query, const MpsBuffer& key,
                                                   const MpsBuffer& value, const MpsBuffer& gate,
                                                   const MpsBuffer& beta, MpsBuffer& state, std::size_t state_offset,
                                                   std::size_t key_heads, std::size_t value_heads,
                                                   std::size_t head_dim, MpsBuffer& output) const {
  return gated_delta_net_f32_batched_in_place_at(query, key, value, gate, beta, state, state_offset, 1, key_heads,
                                                 value_heads, head_dim, output);
}
Status MpsContext::gated_delta_net_f32_in_place(const MpsBuffer& query, const MpsBuffer& key, const MpsBuffer& value,
                                                const MpsBuffer& gate, const MpsBuffer& beta, MpsBuffer& state,
                                                std::size_t key_heads, std::size_t value_heads,
                                                std::size_t head_dim, MpsBuffer& output) const {
  return gated_delta_net_f32_batched_in_place_at(query, key, value, gate, beta, state, 0, 1, key_heads, value_heads,
                                                 head_dim, output);
}

// ---- causal conv
Status MpsContext::ssm_conv_f32(const MpsBuffer& input, const MpsBuffer& kernel, std::size_t conv_kernel,
                                std::size_t channels, std::size_t tokens, std::size_t sequences,
                                MpsBuffer& output) const {
  KIB_CTX_OR_UNAVAILABLE();
  if (!Impl::fits<float>(input, sequences * channels * (conv_kernel - 1 + tokens)) ||
      !Impl::fits<float>(kernel, channels * conv_kernel) || !Impl::fits<float>(output, sequences * tokens * channels))
    return Status::invalid_argument("MPS SSM conv buffers do not match the shape");
  return to_status(c, kib_ssm_conv_f32(c, Impl::dptr<float>(input), Impl::dptr<float>(kernel), conv_kernel, channels, tokens,
                                       sequences, Impl::dptr<float>(output)));
}
Status MpsContext::build_ssm_conv_state_f32(MpsBuffer& state, std::size_t state_offset, const MpsBuffer& input,
                                            std::size_t conv_kernel, std::size_t channels, std::size_t tokens,
                                            MpsBuffer& conv_input) const {
  KIB_CTX_OR_UNAVAILABLE();
  if (conv_kernel < 2 || !Impl::fits<float>(state, state_offset + (conv_kernel - 1) * channels) ||
      !Impl::fits<float>(input, tokens * channels) || !Impl::fits<float>(conv_input, (conv_kernel - 1 + tokens) * channels))
    return Status::invalid_argument("MPS SSM conv-state buffers do not match the shape");
  return to_status(c, kib_build_ssm_conv_state_f32(c, Impl::dptr<float>(state), state_offset, Impl::dptr<float>(input),
                                                   conv_kernel, channels, tokens, Impl::dptr<float>(conv_input)));
}
Status MpsContext::ssm_conv1_f32_stateful_at(MpsBuffer& state, std::size_t state_offset, const MpsBuffer& input,
                                             const MpsBuffer& kernel, std::size_t conv_kernel, std::size_t channels,
                                             MpsBuffer& output) const {
  KIB_CTX_OR_UNAVAILABLE();
  if (conv_kernel < 2 || !Impl::fits<float>(state, state_offset + (conv_kernel - 1) * channels) ||
      !Impl::fits<float>(input, channels) || !Impl::fits<float>(kernel, conv_kernel * channels) || !Impl::fits<float>(output, channels))
    return Status::invalid_argument("MPS stateful SSM conv buffers do not match the shape");
  return to_status(c, kib_ssm_conv1_f32_stateful_at(c, Impl::dptr<float>(state), state_offset, Impl::dptr<float>(input),
                                                    Impl::dptr<float>(kernel), conv_kernel, channels, Impl::dptr<float>(output)));
}
Status MpsContext::ssm_conv1_f32_stateful(MpsBuffer& state, const MpsBuffer& input, const MpsBuffer& kernel,
                                          std::size_t conv_kernel, std::size_t channels, MpsBuffer& output) const {
  return ssm_conv1_f32_stateful_at(state, 0, input, kernel, conv_kernel, channels, output);
}
Status MpsContext::prepare_qwen35_gdn_gate_beta_f32(MpsBuffer& gate, MpsBuffer& beta, const MpsBuffer& gate_bias,
                                                    const MpsBuffer& gate_scale, std::size_t rows,
                                                    std::size_t row_size) const {
  KIB_CTX_OR_UNAVAILABLE();
  if (!Impl::fits<float>(gate, rows * row_size) || !Impl::fits<float>(beta, rows * row_size) ||
      !Impl::fits<float>(gate_bias, row_size) || !Impl::fits<float>(gate_scale, row_size))
    return Status::invalid_argument("MPS GDN gate/beta buffers do not match the shape");
  return to_status(c, kib_prepare_qwen35_gdn_gate_beta_f32(c, Impl::dptr<float>(gate), Impl::dptr<float>(beta),
                                                           Impl::dptr<float>(gate_bias), Impl::dptr<float>(gate_scale), rows,
                                                           row_size));
}

// ---- attention
Status MpsContext::mrope_f32_in_place(MpsBuffer& values, const MpsBuffer& positions, std::size_t tokens,
                                      std::size_t heads, std::size_t head_dim, std::size_t n_dims,
                                      std::size_t section_0, std::size_t section_1, std::size_t section_2,
                                      std::size_t section_3, float theta) const {
  KIB_CTX_OR_UNAVAILABLE();
  if (!Impl::fits<float>(values, tokens * heads * head_dim) || !Impl::fits<int32_t>(positions, 4 * tokens))
    return Status::invalid_argument("MPS MRoPE buffers do not match the shape");
  return to_status(c, kib_mrope_f32_in_place(c, Impl::dptr<float>(values), Impl::dptr<int32_t>(positions), tokens, heads,
                                             head_dim, n_dims, section_0, section_1, section_2, section_3, theta));
}
Status MpsContext::attention_f32_batched_f16_kv(const MpsBuffer& query, const MpsBuffer& key_cache,
                                                const MpsBuffer& value_cache, std::size_t layer,
                                                std::size_t start_position, std::size_t tokens,
                                                std::size_t capacity_tokens, std::size_t heads,
                                                std::size_t kv_heads, std::size_t head_dim,
                                                MpsBuffer& output) const {
  KIB_CTX_OR_UNAVAILABLE();
  const std::size_t cache = (layer + 1) * capacity_tokens * kv_heads * head_dim;
  if (!Impl::fits<float>(query, tokens * heads * head_dim) || !Impl::fits<uint16_t>(key_cache, cache) ||
      !Impl::fits<uint16_t>(value_cache, cache) || !Impl::fits<float>(output, tokens * heads * head_dim))
    return Status::invalid_argument("MPS attention buffers do not match the shape");
  return to_status(c, kib_attention_f32_batched_f16_kv(c, Impl::dptr<float>(query), Impl::dptr<uint16_t>(key_cache),
                                                       Impl::dptr<uint16_t>(value_cache), layer, start_position, tokens,
                                                       capacity_tokens, heads, kv_heads, head_dim,
                                                       Impl::dptr<float>(output)));
}
Status MpsContext::attention_f32_f16_kv(const MpsBuffer& query, const MpsBuffer& key_cache,
                                        const MpsBuffer& value_cache, std::size_t layer, std::size_t position,
                                        std::size_t capacity_tokens, std::size_t heads, std::size_t kv_heads,
                                        std::size_t head_dim, MpsBuffer& output) const {
  return attention_f32_batched_f16_kv(query, key_cache, value_cache, layer, position, 1, capacity_tokens, heads,
                                      kv_heads, head_dim, output);
}

// ---- element-wise and copies
Status MpsContext::Impl::binary(kib_ctx* c, int op, MpsBuffer& target, const MpsBuffer& rhs, std::size_t total,
                                std::size_t row) {
  if (!Impl::fits<float>(target, total) || !Impl::fits<float>(rhs, op < 2 ? total : row))
    return Status::invalid_argument("MPS element-wise buffers do not match the shape");
  return to_status(c, kib_binary_f32_in_place(c, op, Impl::dptr<float>(target), Impl::dptr<float>(rhs), total, row));
}

Status MpsContext::add_f32_in_place(MpsBuffer& target, const MpsBuffer& delta, std::size_t size) const {
  KIB_CTX_OR_UNAVAILABLE();
  return Impl::binary(c, 0, target, delta, size, 0);
}
Status MpsContext::mul_f32_in_place(MpsBuffer& target, const MpsBuffer& rhs, std::size_t size) const {
  KIB_CTX_OR_UNAVAILABLE();
  return Impl::binary(c, 1, target, rhs, size, 0);
}
Status MpsContext::add_f32_row_in_place(MpsBuffer& target, const MpsBuffer& row, std::size_t rows,
                                        std::size_t row_size) const {
  KIB_CTX_OR_UNAVAILABLE();
  return Impl::binary(c, 2, target, row, rows * row_size, row_size);
}
Status MpsContext::mul_f32_row_in_place(MpsBuffer& target, const MpsBuffer& row, std::size_t rows,
                                        std::size_t row_size) const {
  KIB_CTX_OR_UNAVAILABLE();
  return Impl::binary(c, 3, target, row, rows * row_size, row_size);
}
Status MpsContext::sigmoid_f32_in_place(MpsBuffer& values, std::size_t size) const {
  KIB_CTX_OR_UNAVAILABLE();
  if (!Impl::fits<float>(values, size)) return Status::invalid_argument("MPS sigmoid buffer is too small");
  return to_status(c, kib_unary_f32_in_place(c, 0, Impl::dptr<float>(values), size));
}
Status MpsContext::softplus_f32_in_place(MpsBuffer& values, std::size_t size) const {
  KIB_CTX_OR_UNAVAILABLE();
  if (!Impl::fits<float>(values, size)) return Status::invalid_argument("MPS softplus buffer is too small");
  return to_status(c, kib_unary_f32_in_place(c, 1, Impl::dptr<float>(values), size));
}
Status MpsContext::silu_f32_in_place(MpsBuffer& values, std::size_t size) const {
  KIB_CTX_OR_UNAVAILABLE();
  if (!Impl::fits<float>(values, size)) return Status::invalid_argument("MPS silu buffer is too small");
  return to_status(c, kib_unary_f32_in_place(c, 2, Impl::dptr<float>(values), size));
}
Status MpsContext::silu_mul_f32_in_place(MpsBuffer& gate, const MpsBuffer& up, std::size_t size) const {
  KIB_CTX_OR_UNAVAILABLE();
  if (!Impl::fits<float>(gate, size) || !Impl::fits<float>(up, size))
    return Status::invalid_argument("MPS silu-mul buffers do not match the shape");
  return to_status(c, kib_silu_mul_f32_in_place(c, Impl::dptr<float>(gate), Impl::dptr<float>(up), size));
}
Status MpsContext::copy_f32_region(const MpsBuffer& source, MpsBuffer& destination, std::size_t source_offset,
                                   std::size_t destination_offset, std::size_t size) const {
  KIB_CTX_OR_UNAVAILABLE();
  if (!Impl::fits<float>(source, source_offset + size) || !Impl::fits<float>(destination, destination_offset + size))
    return Status::invalid_argument("MPS copy region exceeds buffer size");
  return to_status(c, kib_copy_f32_region(c, Impl::dptr<float>(source), Impl::dptr<float>(destination), source_offset,
                                          destination_offset, size));
}
Status MpsContext::copy_f32_rows(const MpsBuffer& source, MpsBuffer& destination, std::size_t rows,
                                 std::size_t row_size, std::size_t source_stride, std::size_t source_offset,
                                 std::size_t destination_stride, std::size_t destination_offset) const {
  KIB_CTX_OR_UNAVAILABLE();
  if (rows == 0 || !Impl::fits<float>(source, source_offset + (rows - 1) * source_stride + row_size) ||
      !Impl::fits<float>(destination, destination_offset + (rows - 1) * destination_stride + row_size))
    return Status::invalid_argument("MPS copy rows exceed buffer size");
  return to_status(c, kib_copy_f32_rows(c, Impl::dptr<float>(source), Impl::dptr<float>(destination), rows, row_size,
                                        source_stride, source_offset, destination_stride, destination_offset));
}
Status MpsContext::copy_f32_rows_to_f16(const MpsBuffer& source, MpsBuffer& destination, std::size_t rows,
                                        std::size_t row_size, std::size_t source_stride, std::size_t source_offset,
                                        std::size_t destination_stride, std::size_t destination_offset) const {
  KIB_CTX_OR_UNAVAILABLE();
  if (rows == 0 || !Impl::fits<float>(source, source_offset + (rows - 1) * source_stride + row_size) ||
      !Impl::fits<uint16_t>(destination, destination_offset + (rows - 1) * destination_stride + row_size))
    return Status::invalid_argument("MPS copy rows exceed buffer size");
  return to_status(c, kib_copy_f32_rows_to_f16(c, Impl::dptr<float>(source), Impl::dptr<uint16_t>(destination), rows, row_size,
                                               source_stride, source_offset, destination_stride, destination_offset));
}
Status MpsContext::copy_f16_rows(const MpsBuffer& source, MpsBuffer& destination, std::size_t rows,
                                 std::size_t row_size, std::size_t source_stride, std::size_t source_offset,
                                 std::size_t destination_stride, std::size_t destination_offset) const {
  KIB_CTX_OR_UNAVAILABLE();
  if (rows == 0 || !Impl::fits<uint16_t>(source, source_offset + (rows - 1) * source_stride + row_size) ||
      !Impl::fits<uint16_t>(destination, destination_offset + (rows - 1) * destination_stride + row_size))
    return Status::invalid_argument("MPS copy rows exceed buffer size");
  return to_status(c, kib_copy_f16_rows(c, Impl::dptr<uint16_t>(source), Impl::dptr<uint16_t>(destination), rows, row_size,
                                        source_stride, source_offset, destination_stride, destination_offset));
}
Status MpsContext::argmax_f32_i32(const MpsBuffer& values, std::size_t size, MpsBuffer& output) const {
  KIB_CTX_OR_UNAVAILABLE();
  if (!Impl::fits<float>(values, size) || !Impl::fits<int32_t>(output, 1))
    return Status::invalid_argument("MPS argmax buffers do not match the shape");
  return to_status(c, kib_argmax_f32_i32(c, Impl::dptr<float>(values), size, Impl::dptr<int32_t>(output), nullptr));
}
Status MpsContext::argmax_prob_f32_i32(const MpsBuffer& values, std::size_t size, MpsBuffer& token_output,
                                       MpsBuffer& probability_output) const {
  KIB_CTX_OR_UNAVAILABLE();
  if (!Impl::fits<float>(values, size) || !Impl::fits<int32_t>(token_output, 1) || !Impl::fits<float>(probability_output, 1))
    return Status::invalid_argument("MPS argmax buffers do not match the shape");
  return to_status(c, kib_argmax_prob_f32_i32(c, Impl::dptr<float>(values), size, Impl::dptr<int32_t>(token_output),
                                              Impl::dptr<float>(probability_output)));
}

}  // namespace toyllm::mps
