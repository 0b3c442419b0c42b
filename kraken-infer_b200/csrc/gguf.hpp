// gguf.hpp -- GGUF v3 container: mmap reader, writer, K-quant quantizers and
// the synthetic Qwen3.5 model generator.
//
// Reader mirrors the reference's read_gguf_file / GgufMappedData
// (include/toyllm/runtime/gguf_reader.hpp:68-94, src/runtime/gguf_reader.cpp:466-519):
// the tensor directory is parsed once and tensor bytes are served straight from
// the mapping, as stored.
#pragma once

#include <cstdint>
#include <map>
#include <memory>
#include <string>
#include <vector>

namespace kib {

struct GgufTensor {
  std::string name;
  std::vector<uint64_t> shape;  // ne0 (inner, input columns) first
  uint32_t type = 0;
  uint64_t offset = 0;          // relative to the data section
  uint64_t bytes = 0;
  const uint8_t* data = nullptr;
};

struct GgufValue {
  uint32_t type = 0;            // GGUF value type of a scalar / array element type
  bool is_array = false;
  double num = 0.0;
  std::string str;
  std::vector<double> arr;
  std::vector<std::string> strs;  // elements of a string array
};

class GgufFile {
 public:
  ~GgufFile();
  static std::unique_ptr<GgufFile> open(const std::string& path, std::string* err);
  const GgufTensor* tensor(const std::string& name) const;
  const GgufValue* meta(const std::string& key) const;
  double num(const std::string& key, double fallback) const;
  const std::vector<GgufTensor>& tensors() const { return tensors_; }
  uint64_t file_size() const { return size_; }

 private:
  void* map_ = nullptr;
  uint64_t size_ = 0;
  std::vector<GgufTensor> tensors_;
  std::map<std::string, size_t> index_;
  std::map<std::string, GgufValue> meta_;
};

uint64_t ggml_tensor_bytes(uint32_t type, const std::vector<uint64_t>& shape);

// Quantize n (multiple of 256) floats to K-quant super-blocks.
void quantize_q4_k(const float* x, int64_t n, uint8_t* out);
void quantize_q5_k(const float* x, int64_t n, uint8_t* out);
void quantize_q6_k(const float* x, int64_t n, uint8_t* out);

struct SynthQwen35Config {
  int64_t hidden = 1024;
  int64_t layers = 24;          // main layers
  int64_t intermediate = 3584;
  int64_t vocab = 248320;
  int64_t heads = 8;
  int64_t kv_heads = 2;
  int64_t head_dim = 256;
  int64_t ssm_heads = 16;       // key heads == value heads
  int64_t ssm_head_dim = 128;
  int64_t conv_kernel = 4;
  int64_t full_attention_interval = 4;
  int64_t nextn_layers = 0;     // 1 adds an MTP/NextN block
  int64_t context_length = 262144;
  uint32_t proj_type = 12;      // Q4_K for 2-D projections
  uint32_t down_type = 14;      // Q6_K for ffn_down
  uint32_t embd_type = 14;      // Q6_K tied token embedding / LM head
  uint64_t seed = 1234;
  double rope_theta = 1e7;
  double rms_eps = 1e-6;
  int64_t eos_token_id = -1;    // -1: no EOS key
  int threads = 8;
  uint32_t qkv_type = 0;        // GDN attn_qkv; 0: proj_type (the Q4_K_M files store it as Q5_K)
};

// Writes a GGUF whose metadata and tensor names/shapes are those the reference's
// load_model_bundle + build_qwen35_weight_map accept (model_config.cpp:780-870,
// qwen35_weight_map.cpp:61-454).  Weights: 2-D N(0, 0.02), norm vectors
// 1 + N(0, 0.02), conv N(0, 0.02), dt_bias N(0, 0.02), ssm_a = -exp(N(0, 0.5)).
bool write_synthetic_qwen35(const std::string& path, const SynthQwen35Config& cfg, std::string* err);

// Deterministic N(0,1) stream: value `i` of stream `key`.
float synth_normal(uint64_t key, uint64_t i);

}  // namespace kib
