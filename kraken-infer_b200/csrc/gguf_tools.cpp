// gguf_tools.cpp -- the C ABI of the host-side GGUF tools: the synthetic
// Qwen3.5 writer and the K-quant quantisers.  Plain C++ (no device code); it
// is linked into libkib.so and also built alone as libkib_gguf.so, so that a
// process that must not map the CUDA backend (the CPU reference arm of the
// bench) can still write the benchmark's model file.
#include <cstdint>
#include <cstring>
#include <memory>
#include <string>

#include "gguf.hpp"
#include "kib.h"

using namespace kib;

extern "C" {

void kib_synth_default(kib_synth_config* c) {
  if (!c) return;
  SynthQwen35Config d;
  c->hidden = static_cast<uint64_t>(d.hidden);
  c->layers = static_cast<uint64_t>(d.layers);
  c->intermediate = static_cast<uint64_t>(d.intermediate);
  c->vocab = static_cast<uint64_t>(d.vocab);
  c->heads = static_cast<uint64_t>(d.heads);
  c->kv_heads = static_cast<uint64_t>(d.kv_heads);
  c->head_dim = static_cast<uint64_t>(d.head_dim);
  c->ssm_heads = static_cast<uint64_t>(d.ssm_heads);
  c->ssm_head_dim = static_cast<uint64_t>(d.ssm_head_dim);
  c->conv_kernel = static_cast<uint64_t>(d.conv_kernel);
  c->full_attention_interval = static_cast<uint64_t>(d.full_attention_interval);
  c->nextn_layers = static_cast<uint64_t>(d.nextn_layers);
  c->proj_type = d.proj_type;
  c->down_type = d.down_type;
  c->embd_type = d.embd_type;
  c->seed = d.seed;
  c->rope_theta = d.rope_theta;
  c->rms_eps = d.rms_eps;
  c->eos_token_id = d.eos_token_id;
  c->threads = d.threads;
  c->qkv_type = d.qkv_type;
}

int kib_write_synthetic_qwen35(const char* path, const kib_synth_config* c, char* err, int err_len) {
  if (!path || !c) return KIB_ERR_INVALID_ARGUMENT;
  SynthQwen35Config d;
  d.hidden = static_cast<int64_t>(c->hidden);
  d.layers = static_cast<int64_t>(c->layers);
  d.intermediate = static_cast<int64_t>(c->intermediate);
  d.vocab = static_cast<int64_t>(c->vocab);
  d.heads = static_cast<int64_t>(c->heads);
  d.kv_heads = static_cast<int64_t>(c->kv_heads);
  d.head_dim = static_cast<int64_t>(c->head_dim);
  d.ssm_heads = static_cast<int64_t>(c->ssm_heads);
  d.ssm_head_dim = static_cast<int64_t>(c->ssm_head_dim);
  d.conv_kernel = static_cast<int64_t>(c->conv_kernel);
  d.full_attention_interval = static_cast<int64_t>(c->full_attention_interval);
  d.nextn_layers = static_cast<int64_t>(c->nextn_layers);
  d.proj_type = c->proj_type;
  d.down_type = c->down_type;
  d.embd_type = c->embd_type;
  d.seed = c->seed;
  d.rope_theta = c->rope_theta;
  d.rms_eps = c->rms_eps;
  d.eos_token_id = c->eos_token_id;
  d.threads = c->threads > 0 ? c->threads : 8;
  d.qkv_type = c->qkv_type;
  std::string e;
  if (!write_synthetic_qwen35(path, d, &e)) {
    if (err && err_len > 0) {
      std::strncpy(err, e.c_str(), static_cast<size_t>(err_len - 1));
      err[err_len - 1] = 0;
    }
    return KIB_ERR_INVALID_ARGUMENT;
  }
  return KIB_OK;
}

int kib_quantize_kquant(int type, const float* x, uint64_t n, void* out) {
  if (!x || !out || n == 0 || n % 256) return KIB_ERR_INVALID_ARGUMENT;
  uint8_t* o = static_cast<uint8_t*>(out);
  switch (type) {
    case 12: quantize_q4_k(x, static_cast<int64_t>(n), o); return KIB_OK;
    case 13: quantize_q5_k(x, static_cast<int64_t>(n), o); return KIB_OK;
    case 14: quantize_q6_k(x, static_cast<int64_t>(n), o); return KIB_OK;
    default: return KIB_ERR_INVALID_ARGUMENT;
  }
}

int kib_gguf_check(const char* path, char* err, int err_len, uint64_t* n_tensors) {
  if (!path) return KIB_ERR_INVALID_ARGUMENT;
  std::string e;
  std::unique_ptr<GgufFile> g = GgufFile::open(path, &e);
  if (!g) {
    if (err && err_len > 0) {
      std::strncpy(err, e.c_str(), static_cast<size_t>(err_len - 1));
      err[err_len - 1] = 0;
    }
    return KIB_ERR_INVALID_ARGUMENT;
  }
  if (n_tensors) *n_tensors = static_cast<uint64_t>(g->tensors().size());
  return KIB_OK;
}

}  // extern "C"
