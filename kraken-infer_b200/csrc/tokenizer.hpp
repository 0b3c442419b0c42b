// tokenizer.hpp -- the GGUF byte-level BPE tokenizer and the Qwen3.5 chat
// prompt, host side of the serving path (prompt text -> token ids -> the
// prefill, sampled ids -> text).
//
// Behaviour follows the reference's GgufTokenizer
// (include/toyllm/runtime/gguf_tokenizer.hpp:27-66,
// src/runtime/gguf_tokenizer.cpp:628-809): the vocabulary, token types,
// merges and special ids come from the GGUF metadata; text is cut into
// user-defined / control tokens and raw fragments, each raw fragment is split
// into words by the Qwen3.5 pre-tokenizer, each word is byte-encoded (GPT-2
// byte -> code point map) and merged by rank.
#pragma once

#include <cstdint>
#include <string>
#include <string_view>
#include <unordered_map>
#include <utility>
#include <vector>

namespace kib {

class GgufFile;

enum class TokenKind : int64_t {  // tokenizer.ggml.token_type values
  undefined = 0,
  normal = 1,
  unknown = 2,
  control = 3,
  user_defined = 4,
  unused = 5,
  byte = 6,
};

struct ChatTurn {
  std::string role;
  std::string content;
};

class Tokenizer {
 public:
  // Reads tokenizer.ggml.* and tokenizer.chat_template.  Returns false with
  // *err set when the token list is missing or the type list disagrees with
  // it (load_gguf_tokenizer, gguf_tokenizer.cpp:628-677).
  bool load(const GgufFile& g, std::string* err);

  // gguf_encode_text (gguf_tokenizer.cpp:697-738).
  bool encode(std::string_view text, bool add_special, bool parse_special, std::vector<int64_t>* out,
              std::string* err) const;
  // gguf_decode_token_text (gguf_tokenizer.cpp:751-775).
  bool decode(const int64_t* ids, size_t n, bool skip_control, std::string* out, std::string* err) const;
  // format_qwen35_chat_prompt (gguf_tokenizer.cpp:777-809).
  bool format_chat(const std::vector<ChatTurn>& turns, bool add_generation_prompt, bool enable_thinking,
                   std::string* out, std::string* err) const;
  // gguf_encode_qwen35_chat_prompt (gguf_tokenizer.cpp:740-749).
  bool encode_chat(const std::vector<ChatTurn>& turns, bool add_generation_prompt, bool enable_thinking,
                   std::vector<int64_t>* out, std::string* err) const;

  int64_t token_id(std::string_view text) const;  // -1 when absent
  bool is_control(int64_t id) const;              // control or unused
  bool valid(int64_t id) const { return id >= 0 && static_cast<size_t>(id) < tokens_.size(); }

  size_t size() const { return tokens_.size(); }
  size_t merge_count() const { return merges_; }
  const std::string& model() const { return model_; }
  const std::string& pre() const { return pre_; }
  const std::string& chat_template() const { return chat_template_; }
  const std::string& token_text(int64_t id) const { return tokens_[static_cast<size_t>(id)]; }
  int64_t token_type(int64_t id) const { return types_[static_cast<size_t>(id)]; }
  int64_t bos() const { return bos_; }
  int64_t eos() const { return eos_; }
  int64_t pad() const { return pad_; }
  bool add_bos() const { return add_bos_; }
  bool add_eos() const { return add_eos_; }

 private:
  void index_specials();
  void bpe_word(std::string_view word, std::vector<int64_t>* out) const;
  int rank(std::string_view a, std::string_view b) const;

  std::string model_, pre_, chat_template_;
  std::vector<std::string> tokens_;
  std::vector<int64_t> types_;
  size_t merges_ = 0;
  std::unordered_map<std::string, int64_t> ids_;
  // merge ranks keyed by pair_key(left, right): the left length as 4 bytes,
  // then both strings (unambiguous for any bytes)
  std::unordered_map<std::string, int> ranks_;
  // special tokens by first byte, longest first then lowest id: [0] user-defined
  // only, [1] user-defined + control + unknown (parse_special)
  std::vector<int64_t> specials_[2][256];
  int64_t bos_ = -1, eos_ = -1, pad_ = -1;
  bool add_bos_ = false, add_eos_ = false;
};

// The Qwen3.5 pre-tokenizer: the byte ranges [start, end) of the words of a raw
// fragment, in order (split_qwen35_words, gguf_tokenizer.cpp:336-455).
std::vector<std::pair<size_t, size_t>> qwen35_word_ranges(std::string_view text);

}  // namespace kib
