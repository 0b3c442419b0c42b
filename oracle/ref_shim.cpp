// ref_shim.cpp -- TEST INFRASTRUCTURE ONLY.
//
// Exposes a few of the reference's own host routines through a C ABI so the
// parity tests can call them.  The reference translation unit
// src/runtime/qwen35_runtime.cpp is compiled in place (included by path from
// the reference checkout named by -DKIB_REF_ROOT); nothing from it is copied
// into this repository.  Built by oracle/Makefile into oracle/_ref/libkib_ref.so.
#define KIB_STR2(x) #x
#define KIB_STR(x) KIB_STR2(x)
#include KIB_STR(KIB_REF_RUNTIME_TU)

#include <cstring>
#include <map>

#include "toyllm/runtime/gguf_tokenizer.hpp"

extern "C" {

// dequantize_quantized_transposed_f32 (qwen35_runtime.cpp:1084-1241) on a raw
// 2-D tensor; the reference returns the transpose [cols][rows], which this
// wrapper writes back as [rows][cols].
int ref_dequant_tensor(unsigned type, unsigned long long rows, unsigned long long cols,
                       const unsigned char* bytes, unsigned long long nbytes, float* out) {
  toyllm::GgufTensorInfo info;
  info.name = "probe";
  info.shape = {cols, rows};
  info.type = type;
  toyllm::GgufTensorBytes tb;
  tb.data = reinterpret_cast<const std::byte*>(bytes);
  tb.size = static_cast<std::size_t>(nbytes);
  auto result = toyllm::dequantize_quantized_transposed_f32(info, tb);
  if (!result.is_ok()) return -1;
  const auto& t = result.value();
  for (unsigned long long r = 0; r < rows; ++r)
    for (unsigned long long c = 0; c < cols; ++c) out[r * cols + c] = t[c * rows + r];
  return 0;
}

// f16_to_float_cpu (qwen35_runtime.cpp:934-952)
float ref_f16_to_float(unsigned short v) {
  unsigned char b[2] = {static_cast<unsigned char>(v & 0xFF), static_cast<unsigned char>(v >> 8)};
  return toyllm::f16_to_float_cpu(b);
}

// Greedy pick of sample_qwen35_next_token (qwen35_runtime.cpp:3777-3858).
long long ref_greedy_token(const float* logits, unsigned long long n) {
  std::vector<float> v(logits, logits + n);
  std::mt19937 rng(0);
  toyllm::Qwen35EffectiveSamplingConfig cfg;
  cfg.do_sample = false;
  cfg.temperature = 0.0;
  cfg.top_k = 0;
  cfg.top_p = 1.0;
  auto r = toyllm::sample_qwen35_next_token(v, rng, cfg);
  return r.is_ok() ? static_cast<long long>(r.value()) : -1;
}

// load_model_bundle + read_gguf_file + build_qwen35_weight_map +
// build_qwen35_execution_plan over a GGUF file: proves that a synthetic model
// written by this repository is accepted by the reference's own loader.
// Writes hidden, main layers, linear layers, full layers, mtp layers,
// attention capacity, R and S elements per layer into dims[0..7].
int ref_check_gguf(const char* path, unsigned long long context_tokens, long long* dims,
                   char* err, int err_len) {
  auto fail = [&](const std::string& m) {
    if (err && err_len > 0) {
      std::strncpy(err, m.c_str(), static_cast<size_t>(err_len - 1));
      err[err_len - 1] = 0;
    }
    return -1;
  };
  auto bundle = toyllm::load_model_bundle(path);
  if (!bundle.is_ok()) return fail(bundle.status().message());
  auto gguf = toyllm::read_gguf_file(path);
  if (!gguf.is_ok()) return fail(gguf.status().message());
  auto map = toyllm::build_qwen35_weight_map(bundle.value().model, gguf.value());
  if (!map.is_ok()) return fail(map.status().message());
  toyllm::Qwen35RuntimeOptions options;
  options.context_tokens = static_cast<std::size_t>(context_tokens);
  auto plan = toyllm::build_qwen35_execution_plan(bundle.value().model, map.value(), 1, options);
  if (!plan.is_ok()) return fail(plan.status().message());
  const auto& p = plan.value();
  dims[0] = static_cast<long long>(p.hidden_size);
  dims[1] = static_cast<long long>(p.main_layers);
  dims[2] = static_cast<long long>(p.cache.linear_attention_layers);
  dims[3] = static_cast<long long>(p.cache.full_attention_layers);
  dims[4] = static_cast<long long>(map.value().mtp_layers);
  dims[5] = static_cast<long long>(p.cache.attention_capacity_tokens);
  dims[6] = static_cast<long long>(p.cache.recurrent_r_elements_per_layer);
  dims[7] = static_cast<long long>(p.cache.recurrent_s_elements_per_layer);
  return 0;
}

// Qwen35PrefixCacheIndex (src/runtime/qwen35_prefix_cache.cpp) driven by a
// script, to pin the repository's restatement against the reference's own
// index.  ops[i] = 0: lookup of prompt i, 1: commit of the block of prompt i
// at starts[i].  prompts[i] has lens[i] tokens at offs[i] in tokens.  For
// every op, out[2*i] = hit tokens (lookup) or inserted | evicted << 1
// (commit), out[2*i+1] = the last block hash (lookup) or the block hash
// (commit); stats6 = stored, hit, miss, committed, evicted, block tokens.
int ref_prefix_script(unsigned long long block_tokens, unsigned long long capacity, unsigned long long min_reuse,
                      int nops, const int* ops, const long long* tokens, const unsigned long long* offs,
                      const unsigned long long* lens, const unsigned long long* starts, unsigned long long* out,
                      unsigned long long* stats6) {
  toyllm::Qwen35PrefixCacheConfig cfg;
  cfg.enabled = true;
  cfg.block_tokens = block_tokens;
  cfg.capacity_blocks = capacity;
  cfg.min_reuse_tokens = min_reuse;
  toyllm::Qwen35PrefixCacheIndex idx(cfg);
  for (int i = 0; i < nops; ++i) {
    std::vector<std::int64_t> t(tokens + offs[i], tokens + offs[i] + lens[i]);
    if (ops[i] == 0) {
      auto r = idx.lookup(t);
      out[2 * i] = r.hit_tokens;
      out[2 * i + 1] = r.block_hashes.empty() ? 0 : r.block_hashes.back();
    } else {
      auto r = idx.commit_block(t, starts[i]);
      out[2 * i] = (r.inserted ? 1u : 0u) | (r.evicted ? 2u : 0u);
      out[2 * i + 1] = r.hash;
    }
  }
  auto st = idx.stats();
  stats6[0] = st.stored_blocks;
  stats6[1] = st.hit_tokens;
  stats6[2] = st.miss_tokens;
  stats6[3] = st.committed_tokens;
  stats6[4] = st.evicted_blocks;
  stats6[5] = st.block_tokens;
  return 0;
}

// ---- GgufTokenizer (src/runtime/gguf_tokenizer.cpp) over a GGUF file, to pin
// the repository's tokenizer against the reference's own.  ref_tok_load reads
// (or re-reads) the file and keeps the tokenizer for the other calls on the
// same path.  Each call returns its element count or -1 with err filled.
namespace {
std::map<std::string, toyllm::GgufTokenizer> g_ref_toks;

int ref_fail(char* err, int err_len, const std::string& m) {
  if (err && err_len > 0) {
    std::strncpy(err, m.c_str(), static_cast<size_t>(err_len - 1));
    err[err_len - 1] = 0;
  }
  return -1;
}

const toyllm::GgufTokenizer* ref_tok(const char* path, char* err, int err_len, bool reload) {
  auto it = g_ref_toks.find(path);
  if (it != g_ref_toks.end() && !reload) return &it->second;
  auto gguf = toyllm::read_gguf_file(path);
  if (!gguf.is_ok()) {
    ref_fail(err, err_len, gguf.status().message());
    return nullptr;
  }
  auto tok = toyllm::load_gguf_tokenizer(gguf.value());
  if (!tok.is_ok()) {
    ref_fail(err, err_len, tok.status().message());
    return nullptr;
  }
  g_ref_toks[path] = tok.value();
  return &g_ref_toks[path];
}

std::vector<toyllm::ChatMessage> ref_messages(const char* const* roles, const char* const* contents, int n) {
  std::vector<toyllm::ChatMessage> m;
  for (int i = 0; i < n; ++i) m.emplace_back(roles[i], contents[i]);
  return m;
}

long long ref_put_ids(const std::vector<std::int64_t>& ids, long long* out, unsigned long long cap) {
  for (size_t i = 0; i < ids.size() && i < cap; ++i) out[i] = ids[i];
  return static_cast<long long>(ids.size());
}

long long ref_put_text(const std::string& s, char* out, unsigned long long cap) {
  if (s.size() <= cap) std::memcpy(out, s.data(), s.size());
  return static_cast<long long>(s.size());
}
}  // namespace

// info9: tokens, merges, bos, eos, pad, add_bos, add_eos, <|im_start|>, <|im_end|> (-1 when absent)
int ref_tok_load(const char* path, long long* info9, char* err, int err_len) {
  const auto* t = ref_tok(path, err, err_len, true);
  if (!t) return -1;
  const auto im_s = toyllm::gguf_token_id(*t, "<|im_start|>");
  const auto im_e = toyllm::gguf_token_id(*t, "<|im_end|>");
  const long long v[9] = {static_cast<long long>(t->tokens.size()), static_cast<long long>(t->merges.size()),
                          t->bos_token_id, t->eos_token_id, t->pad_token_id, t->add_bos_token, t->add_eos_token,
                          im_s ? *im_s : -1, im_e ? *im_e : -1};
  for (int i = 0; i < 9; ++i) info9[i] = v[i];
  return 0;
}

long long ref_tok_encode(const char* path, const char* text, unsigned long long len, int add_special,
                         int parse_special, long long* out, unsigned long long cap, char* err, int err_len) {
  const auto* t = ref_tok(path, err, err_len, false);
  if (!t) return -1;
  auto r = toyllm::gguf_encode_text(*t, std::string_view(text, len), add_special != 0, parse_special != 0);
  if (!r.is_ok()) return ref_fail(err, err_len, r.status().message());
  return ref_put_ids(r.value(), out, cap);
}

long long ref_tok_decode(const char* path, const long long* ids, unsigned long long n, int skip_control, char* out,
                         unsigned long long cap, char* err, int err_len) {
  const auto* t = ref_tok(path, err, err_len, false);
  if (!t) return -1;
  std::vector<std::int64_t> v(ids, ids + n);
  auto r = toyllm::gguf_decode_token_text(*t, v, skip_control != 0);
  if (!r.is_ok()) return ref_fail(err, err_len, r.status().message());
  return ref_put_text(r.value(), out, cap);
}

long long ref_tok_format_chat(const char* path, const char* const* roles, const char* const* contents, int n,
                              int add_generation_prompt, int enable_thinking, char* out, unsigned long long cap,
                              char* err, int err_len) {
  const auto* t = ref_tok(path, err, err_len, false);
  if (!t) return -1;
  auto r = toyllm::format_qwen35_chat_prompt(*t, ref_messages(roles, contents, n), add_generation_prompt != 0,
                                             enable_thinking != 0);
  if (!r.is_ok()) return ref_fail(err, err_len, r.status().message());
  return ref_put_text(r.value(), out, cap);
}

long long ref_tok_encode_chat(const char* path, const char* const* roles, const char* const* contents, int n,
                              int add_generation_prompt, int enable_thinking, long long* out,
                              unsigned long long cap, char* err, int err_len) {
  const auto* t = ref_tok(path, err, err_len, false);
  if (!t) return -1;
  auto r = toyllm::gguf_encode_qwen35_chat_prompt(*t, ref_messages(roles, contents, n), add_generation_prompt != 0,
                                                  enable_thinking != 0);
  if (!r.is_ok()) return ref_fail(err, err_len, r.status().message());
  return ref_put_ids(r.value(), out, cap);
}

}  // extern "C"
