// tokenizer.cpp -- GGUF byte-level BPE + the Qwen3.5 pre-tokenizer and chat
// prompt (the reference's src/runtime/gguf_tokenizer.cpp).
//
// Built differently from the reference, with the same results:
//  * merging runs over a linked list of symbols with a min-heap of candidate
//    pairs ordered by (rank, byte offset), so each step takes the lowest-ranked
//    pair and, among equal ranks, the leftmost -- the pair the reference's
//    rescan-per-merge loop picks (bpe_encode_word, gguf_tokenizer.cpp:457-505)
//    -- in O(n log n) rather than O(n^2) string rebuilding;
//  * special tokens are bucketed by first byte, each bucket ordered longest
//    first then lowest id, so the first hit at a position is the reference's
//    longest / lowest-id match (partition_special_tokens, :541-575);
//  * the pre-tokenizer yields byte ranges of the fragment (no per-word copies
//    before the byte encoding).
// Tables that must be the reference's for identical ids: the GPT-2 byte ->
// code point map (build_byte_encoder, :273-298), the code point classes
// (is_unicode_number / _letter / _accent_mark / _whitespace, :194-250), the
// chat framing strings (:769-809) and the error texts.
#include "tokenizer.hpp"

#include <algorithm>
#include <cstring>
#include <queue>

#include "gguf.hpp"

namespace kib {
namespace {

constexpr uint32_t kGgufBool = 7, kGgufString = 8;

// ------------------------------------------------------------ UTF-8 + classes
struct CodePoint {
  uint32_t cp;
  uint32_t len;
};

// Loose UTF-8: a 2/3/4-byte form is taken whenever its continuation bytes are
// 10xxxxxx (overlong forms included); any other byte is U+FFFD of length 1
// (utf8_codepoint_spans, gguf_tokenizer.cpp:116-162).
CodePoint decode_at(std::string_view s, size_t i) {
  const auto b = [&](size_t k) { return static_cast<uint32_t>(static_cast<uint8_t>(s[i + k])); };
  const auto cont = [&](size_t k) { return (b(k) & 0xC0u) == 0x80u; };
  const size_t avail = s.size() - i;
  const uint32_t b0 = b(0);
  if (b0 < 0x80u) return {b0, 1};
  if ((b0 & 0xE0u) == 0xC0u && avail >= 2 && cont(1)) return {((b0 & 0x1Fu) << 6) | (b(1) & 0x3Fu), 2};
  if ((b0 & 0xF0u) == 0xE0u && avail >= 3 && cont(1) && cont(2))
    return {((b0 & 0x0Fu) << 12) | ((b(1) & 0x3Fu) << 6) | (b(2) & 0x3Fu), 3};
  if ((b0 & 0xF8u) == 0xF0u && avail >= 4 && cont(1) && cont(2) && cont(3))
    return {((b0 & 0x07u) << 18) | ((b(1) & 0x3Fu) << 12) | ((b(2) & 0x3Fu) << 6) | (b(3) & 0x3Fu), 4};
  return {0xFFFDu, 1};
}

void put_utf8(std::string* out, uint32_t cp) {
  if (cp < 0x80u) {
    out->push_back(static_cast<char>(cp));
  } else if (cp < 0x800u) {
    out->push_back(static_cast<char>(0xC0u | (cp >> 6)));
    out->push_back(static_cast<char>(0x80u | (cp & 0x3Fu)));
  } else if (cp < 0x10000u) {
    out->push_back(static_cast<char>(0xE0u | (cp >> 12)));
    out->push_back(static_cast<char>(0x80u | ((cp >> 6) & 0x3Fu)));
    out->push_back(static_cast<char>(0x80u | (cp & 0x3Fu)));
  } else {
    out->push_back(static_cast<char>(0xF0u | (cp >> 18)));
    out->push_back(static_cast<char>(0x80u | ((cp >> 12) & 0x3Fu)));
    out->push_back(static_cast<char>(0x80u | ((cp >> 6) & 0x3Fu)));
    out->push_back(static_cast<char>(0x80u | (cp & 0x3Fu)));
  }
}

enum : unsigned { kNum = 1u, kLetter = 2u, kMark = 4u, kSpace = 8u };

struct Range {
  uint32_t lo, hi;
};

// Letter blocks the classifier knows (besides ASCII and Latin-1/Extended
// 0xC0-0x2AF minus the multiplication and division signs).
constexpr Range kLetterBlocks[] = {
    {0x0370u, 0x03FFu}, {0x0400u, 0x052Fu}, {0x0530u, 0x058Fu}, {0x0590u, 0x05FFu},
    {0x0600u, 0x06FFu}, {0x0900u, 0x097Fu}, {0x3040u, 0x30FFu}, {0x3400u, 0x4DBFu},
    {0x4E00u, 0x9FFFu}, {0xAC00u, 0xD7AFu}, {0xF900u, 0xFAFFu}, {0x20000u, 0x2FA1Fu},
};
constexpr Range kMarkBlocks[] = {
    {0x0300u, 0x036Fu}, {0x1AB0u, 0x1AFFu}, {0x1DC0u, 0x1DFFu}, {0x20D0u, 0x20FFu}, {0xFE20u, 0xFE2Fu},
};
constexpr uint32_t kSpaces[] = {0x09u,   0x0Au,   0x0Bu,   0x0Cu,   0x0Du,   0x20u,   0x85u,
                                0xA0u,   0x1680u, 0x2000u, 0x2001u, 0x2002u, 0x2003u, 0x2004u,
                                0x2005u, 0x2006u, 0x2007u, 0x2008u, 0x2009u, 0x200Au, 0x2028u,
                                0x2029u, 0x202Fu, 0x205Fu, 0x3000u};

template <size_t N>
bool in_blocks(uint32_t c, const Range (&r)[N]) {
  for (const Range& x : r)
    if (c >= x.lo && c <= x.hi) return true;
  return false;
}

// The only classes the Qwen3.5 splitter looks at; punctuation and symbols
// carry none (class 0).
unsigned cp_class_slow(uint32_t c) {
  unsigned k = 0;
  if ((c >= '0' && c <= '9') || (c >= 0xFF10u && c <= 0xFF19u)) k |= kNum;
  if ((c >= 'A' && c <= 'Z') || (c >= 'a' && c <= 'z') || (c >= 0xC0u && c <= 0x2AFu && c != 0xD7u && c != 0xF7u) ||
      in_blocks(c, kLetterBlocks))
    k |= kLetter;
  if (in_blocks(c, kMarkBlocks)) k |= kMark;
  if (std::find(std::begin(kSpaces), std::end(kSpaces), c) != std::end(kSpaces)) k |= kSpace;
  return k;
}

struct AsciiClasses {
  uint8_t k[128];
  AsciiClasses() {
    for (uint32_t c = 0; c < 128; ++c) k[c] = static_cast<uint8_t>(cp_class_slow(c));
  }
};

unsigned cp_class(uint32_t c) {
  static const AsciiClasses ascii;
  return c < 128 ? ascii.k[c] : cp_class_slow(c);
}

// ------------------------------------------------------------ byte <-> code point
// GPT-2's map: the printable bytes 33-126, 161-172, 174-255 stand for
// themselves; the other 68 bytes, in increasing order, take 256, 257, ...
struct ByteMap {
  std::string enc[256];  // UTF-8 of each byte's code point
  int16_t dec[256 + 68];  // code point -> byte, -1 for none
  ByteMap() {
    std::fill(std::begin(dec), std::end(dec), int16_t(-1));
    uint32_t extra = 256;
    for (uint32_t byte = 0; byte < 256; ++byte) {
      const bool printable = (byte >= 33 && byte <= 126) || (byte >= 161 && byte <= 172) || byte >= 174;
      const uint32_t cp = printable ? byte : extra++;
      put_utf8(&enc[byte], cp);
      dec[cp] = static_cast<int16_t>(byte);
    }
  }
};

const ByteMap& byte_map() {
  static const ByteMap m;
  return m;
}

void pair_key(std::string* key, std::string_view a, std::string_view b) {
  const uint32_t n = static_cast<uint32_t>(a.size());
  key->assign(reinterpret_cast<const char*>(&n), 4);
  key->append(a.data(), a.size());
  key->append(b.data(), b.size());
}

bool fail(std::string* err, std::string msg) {
  if (err) *err = std::move(msg);
  return false;
}

bool is_int_type(uint32_t t) { return t <= 5 || t == 10 || t == 11; }

std::string meta_string(const GgufFile& g, const char* key) {
  const GgufValue* v = g.meta(key);
  return (v && !v->is_array && v->type == kGgufString) ? v->str : std::string();
}

int64_t meta_int(const GgufFile& g, const char* key, int64_t fallback) {
  const GgufValue* v = g.meta(key);
  return (v && !v->is_array && is_int_type(v->type)) ? static_cast<int64_t>(v->num) : fallback;
}

bool meta_bool(const GgufFile& g, const char* key) {
  const GgufValue* v = g.meta(key);
  return v && !v->is_array && v->type == kGgufBool && v->num != 0.0;
}

}  // namespace

// ------------------------------------------------------------ pre-tokenizer
std::vector<std::pair<size_t, size_t>> qwen35_word_ranges(std::string_view text) {
  std::vector<uint32_t> cps;
  std::vector<size_t> at;  // byte offset of each code point, then the end
  cps.reserve(text.size());
  at.reserve(text.size() + 1);
  for (size_t i = 0; i < text.size();) {
    const CodePoint c = decode_at(text, i);
    cps.push_back(c.cp);
    at.push_back(i);
    i += c.len;
  }
  const size_t n = cps.size();
  at.push_back(text.size());
  const auto cls = [&](size_t i) -> unsigned { return i < n ? cp_class(cps[i]) : 0u; };
  const auto lower = [&](size_t i) -> uint32_t { return (cps[i] >= 'A' && cps[i] <= 'Z') ? cps[i] + 32 : cps[i]; };
  const auto newline = [&](size_t i) { return i < n && (cps[i] == '\r' || cps[i] == '\n'); };

  // End (code point index) of the word that starts at p.  The alternatives of
  // the Qwen3.5 split, in order:
  const auto word_end = [&](size_t p) -> size_t {
    // 's 't 'm 'd 're 've 'll, either case
    if (cps[p] == '\'' && p + 1 < n) {
      const uint32_t a = lower(p + 1);
      if (a == 's' || a == 't' || a == 'm' || a == 'd') return p + 2;
      if (p + 2 < n) {
        const uint32_t b = lower(p + 2);
        if ((a == 'r' && b == 'e') || (a == 'v' && b == 'e') || (a == 'l' && b == 'l')) return p + 3;
      }
    }
    // one optional lead that is neither a newline nor a digit, then letters /
    // marks (the lead itself may be the first letter)
    if (!newline(p) && !(cls(p) & kNum) && ((cls(p) | cls(p + 1)) & (kLetter | kMark))) {
      size_t q = p + 1;
      while (cls(q) & (kLetter | kMark)) ++q;
      return q;
    }
    // a digit stands alone
    if (cls(p) & kNum) return p + 1;
    // The regex's " ?[^\s\p{L}\p{N}]+[\r\n]*" alternative cannot extend past
    // one code point here: with no punctuation class, an unclassified code
    // point never starts a run, and a space before one is emitted alone --
    // which the whitespace rule below does as well.
    // whitespace: up to the last newline of the run; else all but the last
    // space when something follows the run; else the whole run
    size_t w = 0, past_newline = 0;
    while (cls(p + w) & kSpace) {
      if (newline(p + w)) past_newline = p + w + 1;
      ++w;
    }
    if (past_newline) return past_newline;
    if (w > 1 && p + w < n) return p + w - 1;
    if (w > 0) return p + w;
    return p + 1;
  };

  std::vector<std::pair<size_t, size_t>> words;
  for (size_t p = 0; p < n;) {
    const size_t q = word_end(p);
    words.emplace_back(at[p], at[q]);
    p = q;
  }
  return words;
}

// ------------------------------------------------------------ load
bool Tokenizer::load(const GgufFile& g, std::string* err) {
  const GgufValue* toks = g.meta("tokenizer.ggml.tokens");
  if (!toks) return fail(err, "missing GGUF metadata key: tokenizer.ggml.tokens");
  if (!toks->is_array || toks->type != kGgufString)
    return fail(err, "GGUF metadata key is not string array: tokenizer.ggml.tokens");
  model_ = meta_string(g, "tokenizer.ggml.model");
  pre_ = meta_string(g, "tokenizer.ggml.pre");
  chat_template_ = meta_string(g, "tokenizer.chat_template");
  tokens_ = toks->strs;
  types_.assign(tokens_.size(), static_cast<int64_t>(TokenKind::normal));
  if (const GgufValue* t = g.meta("tokenizer.ggml.token_type"); t && t->is_array && is_int_type(t->type)) {
    types_.clear();
    for (double v : t->arr) types_.push_back(static_cast<int64_t>(v));
  }
  bos_ = meta_int(g, "tokenizer.ggml.bos_token_id", -1);
  eos_ = meta_int(g, "tokenizer.ggml.eos_token_id", -1);
  pad_ = meta_int(g, "tokenizer.ggml.padding_token_id", -1);
  add_bos_ = meta_bool(g, "tokenizer.ggml.add_bos_token");
  add_eos_ = meta_bool(g, "tokenizer.ggml.add_eos_token");
  if (types_.size() != tokens_.size()) return fail(err, "tokenizer.ggml.token_type size differs from tokens");

  ranks_.clear();
  merges_ = 0;
  if (const GgufValue* m = g.meta("tokenizer.ggml.merges"); m && m->is_array && m->type == kGgufString) {
    merges_ = m->strs.size();
    ranks_.reserve(m->strs.size());
    std::string key;
    for (size_t i = 0; i < m->strs.size(); ++i) {
      const std::string& s = m->strs[i];
      const size_t sp = s.find(' ', 1);  // a merge may start with a space
      if (sp == std::string::npos) continue;
      pair_key(&key, std::string_view(s).substr(0, sp), std::string_view(s).substr(sp + 1));
      ranks_.emplace(key, static_cast<int>(i));  // the first rank of a repeated pair stays
    }
  }
  ids_.clear();
  ids_.reserve(tokens_.size());
  for (size_t i = 0; i < tokens_.size(); ++i) ids_.emplace(tokens_[i], static_cast<int64_t>(i));
  index_specials();
  return true;
}

void Tokenizer::index_specials() {
  for (auto& set : specials_)
    for (auto& bucket : set) bucket.clear();
  for (size_t i = 0; i < tokens_.size(); ++i) {
    if (tokens_[i].empty()) continue;
    const int64_t t = types_[i];
    const bool user = t == static_cast<int64_t>(TokenKind::user_defined);
    const bool parsed =
        user || t == static_cast<int64_t>(TokenKind::control) || t == static_cast<int64_t>(TokenKind::unknown);
    const uint8_t first = static_cast<uint8_t>(tokens_[i][0]);
    if (user) specials_[0][first].push_back(static_cast<int64_t>(i));
    if (parsed) specials_[1][first].push_back(static_cast<int64_t>(i));
  }
  for (auto& set : specials_)
    for (auto& bucket : set)
      std::sort(bucket.begin(), bucket.end(), [&](int64_t a, int64_t b) {
        const size_t la = tokens_[a].size(), lb = tokens_[b].size();
        return la != lb ? la > lb : a < b;
      });
}

int64_t Tokenizer::token_id(std::string_view text) const {
  const auto it = ids_.find(std::string(text));
  return it == ids_.end() ? -1 : it->second;
}

bool Tokenizer::is_control(int64_t id) const {
  if (!valid(id)) return false;
  const int64_t t = types_[static_cast<size_t>(id)];
  return t == static_cast<int64_t>(TokenKind::control) || t == static_cast<int64_t>(TokenKind::unused);
}

int Tokenizer::rank(std::string_view a, std::string_view b) const {
  thread_local std::string key;
  pair_key(&key, a, b);
  const auto it = ranks_.find(key);
  return it == ranks_.end() ? -1 : it->second;
}

// ------------------------------------------------------------ BPE
void Tokenizer::bpe_word(std::string_view word, std::vector<int64_t>* out) const {
  struct Sym {
    uint32_t start, len;  // bytes of the byte-encoded word; len 0 = merged away
    int prev, next;
  };
  struct Cand {
    int rank;
    uint32_t start;  // byte offset of the left symbol: leftmost first among equal ranks
    int left;
    uint32_t llen, rlen;
    bool operator>(const Cand& o) const { return rank != o.rank ? rank > o.rank : start > o.start; }
  };
  // a final symbol's id; a symbol with no token becomes its single bytes,
  // where the vocabulary has them
  const auto emit = [&](std::string_view t) {
    const auto it = ids_.find(std::string(t));
    if (it != ids_.end()) {
      out->push_back(it->second);
      return;
    }
    for (char ch : t) {
      const auto b = ids_.find(std::string(1, ch));
      if (b != ids_.end()) out->push_back(b->second);
    }
  };
  if (word.empty()) return;
  if (decode_at(word, 0).len == word.size()) {  // one symbol: nothing to merge
    emit(word);
    return;
  }
  thread_local std::vector<Sym> sy;
  sy.clear();
  for (size_t i = 0; i < word.size();) {
    const uint32_t len = decode_at(word, i).len;
    sy.push_back({static_cast<uint32_t>(i), len, static_cast<int>(sy.size()) - 1, static_cast<int>(sy.size()) + 1});
    i += len;
  }
  sy.back().next = -1;
  const auto text = [&](int i) { return word.substr(sy[i].start, sy[i].len); };
  std::priority_queue<Cand, std::vector<Cand>, std::greater<Cand>> heap;
  const auto offer = [&](int l) {
    if (l < 0 || sy[l].next < 0) return;
    const int r = sy[l].next;
    const int k = rank(text(l), text(r));
    if (k >= 0) heap.push({k, sy[l].start, l, sy[l].len, sy[r].len});
  };
  for (int i = 0; i + 1 < static_cast<int>(sy.size()); ++i) offer(i);
  while (!heap.empty()) {
    const Cand c = heap.top();
    heap.pop();
    Sym& l = sy[c.left];
    // stale when either side has merged since the candidate was offered
    if (l.len != c.llen || l.next < 0 || sy[l.next].len != c.rlen) continue;
    Sym& r = sy[l.next];
    l.len += r.len;
    l.next = r.next;
    if (r.next >= 0) sy[r.next].prev = c.left;
    r.len = 0;
    offer(l.prev);
    offer(c.left);
  }
  for (int i = 0; i >= 0; i = sy[i].next) emit(text(i));
}

// ------------------------------------------------------------ encode / decode
bool Tokenizer::encode(std::string_view text, bool add_special, bool parse_special, std::vector<int64_t>* out,
                       std::string* err) const {
  out->clear();
  if (model_ != "gpt2") return fail(err, "GGUF encode currently supports gpt2/BPE tokenizers only");
  if (pre_ != "qwen35") return fail(err, "GGUF encode currently supports tokenizer pre qwen35 only");
  if (add_special && add_bos_) {
    if (!valid(bos_)) return fail(err, "GGUF tokenizer add_bos_token is true but BOS id is invalid");
    out->push_back(bos_);
  }
  const ByteMap& bm = byte_map();
  std::string encoded;
  const auto raw = [&](size_t from, size_t to) {
    const std::string_view frag = text.substr(from, to - from);
    for (const auto& w : qwen35_word_ranges(frag)) {
      encoded.clear();
      for (size_t i = w.first; i < w.second; ++i) encoded += bm.enc[static_cast<uint8_t>(frag[i])];
      bpe_word(encoded, out);
    }
  };
  const auto& specials = specials_[parse_special ? 1 : 0];
  size_t from = 0;
  for (size_t pos = 0; pos < text.size();) {
    int64_t hit = -1;
    for (int64_t id : specials[static_cast<uint8_t>(text[pos])]) {
      const std::string& t = tokens_[static_cast<size_t>(id)];
      if (t.size() <= text.size() - pos && text.compare(pos, t.size(), t) == 0) {
        hit = id;
        break;
      }
    }
    if (hit < 0) {
      ++pos;
      continue;
    }
    if (pos > from) raw(from, pos);
    out->push_back(hit);
    pos += tokens_[static_cast<size_t>(hit)].size();
    from = pos;
  }
  if (from < text.size()) raw(from, text.size());
  if (add_special && add_eos_) {
    if (!valid(eos_)) return fail(err, "GGUF tokenizer add_eos_token is true but EOS id is invalid");
    out->push_back(eos_);
  }
  return true;
}

bool Tokenizer::decode(const int64_t* ids, size_t n, bool skip_control, std::string* out, std::string* err) const {
  out->clear();
  const ByteMap& bm = byte_map();
  for (size_t k = 0; k < n; ++k) {
    const int64_t id = ids[k];
    if (!valid(id)) return fail(err, "GGUF token id out of range: " + std::to_string(id));
    if (skip_control && is_control(id)) continue;
    const std::string& t = tokens_[static_cast<size_t>(id)];
    for (size_t i = 0; i < t.size();) {
      const CodePoint c = decode_at(t, i);
      if (c.cp < 256 + 68 && bm.dec[c.cp] >= 0)
        out->push_back(static_cast<char>(bm.dec[c.cp]));
      else
        out->append(t, i, c.len);
      i += c.len;
    }
  }
  return true;
}

bool Tokenizer::format_chat(const std::vector<ChatTurn>& turns, bool add_generation_prompt, bool enable_thinking,
                            std::string* out, std::string* err) const {
  out->clear();
  if (pre_ != "qwen35") return fail(err, "Qwen3.5 chat formatter requires tokenizer pre qwen35");
  if (token_id("<|im_start|>") < 0 || token_id("<|im_end|>") < 0)
    return fail(err, "Qwen3.5 tokenizer is missing chat control tokens");
  for (const ChatTurn& t : turns) {
    if (t.role != "system" && t.role != "user" && t.role != "assistant")
      return fail(err, "unsupported chat message role: " + t.role);
    *out += "<|im_start|>";
    *out += t.role;
    *out += '\n';
    *out += t.content;
    *out += "<|im_end|>\n";
  }
  if (add_generation_prompt) *out += enable_thinking ? "<|im_start|>assistant\n<think>\n"
                                                     : "<|im_start|>assistant\n<think>\n\n</think>\n\n";
  return true;
}

bool Tokenizer::encode_chat(const std::vector<ChatTurn>& turns, bool add_generation_prompt, bool enable_thinking,
                            std::vector<int64_t>* out, std::string* err) const {
  std::string prompt;
  if (!format_chat(turns, add_generation_prompt, enable_thinking, &prompt, err)) {
    out->clear();
    return false;
  }
  return encode(prompt, false, true, out, err);
}

}  // namespace kib

// ------------------------------------------------------------------ C ABI
// Every call returns the element count it produced (or would produce: a result
// larger than `cap` is not written, the caller retries with a larger buffer),
// or -1 with the message kept for kib_tokenizer_last_error.
#include <memory>

#include "gguf.hpp"

struct kib_tokenizer {
  kib::Tokenizer tok;
  std::string err;
};

namespace {

thread_local std::string g_tok_load_err;

int64_t tok_error(kib_tokenizer* t, const std::string& msg) {
  if (t) t->err = msg;
  return -1;
}

std::vector<kib::ChatTurn> chat_turns(const char* const* roles, const char* const* contents, uint64_t n) {
  std::vector<kib::ChatTurn> turns(n);
  for (uint64_t i = 0; i < n; ++i) {
    turns[i].role = roles[i] ? roles[i] : "";
    turns[i].content = contents[i] ? contents[i] : "";
  }
  return turns;
}

int64_t put_ids(const std::vector<int64_t>& ids, int64_t* out, uint64_t cap) {
  if (out && ids.size() <= cap) std::copy(ids.begin(), ids.end(), out);
  return static_cast<int64_t>(ids.size());
}

int64_t put_text(const std::string& s, char* out, uint64_t cap) {
  if (out && s.size() <= cap) std::memcpy(out, s.data(), s.size());
  return static_cast<int64_t>(s.size());
}

}  // namespace

extern "C" {

kib_tokenizer* kib_tokenizer_load(const char* gguf_path) {
  g_tok_load_err.clear();
  std::string err;
  auto g = kib::GgufFile::open(gguf_path ? gguf_path : "", &err);
  if (!g) {
    g_tok_load_err = err;
    return nullptr;
  }
  std::unique_ptr<kib_tokenizer> t(new kib_tokenizer);
  if (!t->tok.load(*g, &err)) {
    g_tok_load_err = err;
    return nullptr;
  }
  return t.release();
}

const char* kib_tokenizer_load_error(void) { return g_tok_load_err.c_str(); }

void kib_tokenizer_free(kib_tokenizer* t) { delete t; }

const char* kib_tokenizer_last_error(const kib_tokenizer* t) { return t ? t->err.c_str() : "null tokenizer"; }

// info[0..8]: tokens, merges, bos, eos, pad, add_bos, add_eos, <|im_start|>, <|im_end|>
void kib_tokenizer_info(const kib_tokenizer* t, int64_t* info9) {
  if (!t || !info9) return;
  const kib::Tokenizer& k = t->tok;
  const int64_t v[9] = {static_cast<int64_t>(k.size()), static_cast<int64_t>(k.merge_count()), k.bos(), k.eos(),
                        k.pad(), k.add_bos(), k.add_eos(), k.token_id("<|im_start|>"), k.token_id("<|im_end|>")};
  std::copy(v, v + 9, info9);
}

int64_t kib_tokenizer_meta(const kib_tokenizer* t, int which, char* out, uint64_t cap) {
  if (!t) return -1;
  const std::string& s = which == 0 ? t->tok.model() : which == 1 ? t->tok.pre() : t->tok.chat_template();
  return put_text(s, out, cap);
}

int64_t kib_tokenizer_token_id(const kib_tokenizer* t, const char* text, uint64_t len) {
  if (!t || (!text && len)) return -1;
  return t->tok.token_id(std::string_view(text ? text : "", len));
}

int64_t kib_tokenizer_token_text(const kib_tokenizer* t, int64_t id, char* out, uint64_t cap) {
  if (!t || !t->tok.valid(id)) return -1;
  return put_text(t->tok.token_text(id), out, cap);
}

int64_t kib_tokenizer_token_type(const kib_tokenizer* t, int64_t id) {
  if (!t || !t->tok.valid(id)) return -1;
  return t->tok.token_type(id);
}

int kib_tokenizer_is_control(const kib_tokenizer* t, int64_t id) { return t && t->tok.is_control(id) ? 1 : 0; }

int64_t kib_tokenizer_encode(kib_tokenizer* t, const char* text, uint64_t len, int add_special, int parse_special,
                             int64_t* out, uint64_t cap) {
  if (!t) return -1;
  if (!text && len) return tok_error(t, "null text");
  std::vector<int64_t> ids;
  std::string err;
  if (!t->tok.encode(std::string_view(text ? text : "", len), add_special != 0, parse_special != 0, &ids, &err))
    return tok_error(t, err);
  return put_ids(ids, out, cap);
}

int64_t kib_tokenizer_decode(kib_tokenizer* t, const int64_t* ids, uint64_t n, int skip_control, char* out,
                             uint64_t cap) {
  if (!t) return -1;
  if (!ids && n) return tok_error(t, "null ids");
  std::string s, err;
  if (!t->tok.decode(ids, n, skip_control != 0, &s, &err)) return tok_error(t, err);
  return put_text(s, out, cap);
}

int64_t kib_tokenizer_format_chat(kib_tokenizer* t, const char* const* roles, const char* const* contents,
                                  uint64_t n, int add_generation_prompt, int enable_thinking, char* out,
                                  uint64_t cap) {
  if (!t) return -1;
  if ((!roles || !contents) && n) return tok_error(t, "null messages");
  std::string s, err;
  if (!t->tok.format_chat(chat_turns(roles, contents, n), add_generation_prompt != 0, enable_thinking != 0, &s,
                          &err))
    return tok_error(t, err);
  return put_text(s, out, cap);
}

int64_t kib_tokenizer_encode_chat(kib_tokenizer* t, const char* const* roles, const char* const* contents,
                                  uint64_t n, int add_generation_prompt, int enable_thinking, int64_t* out,
                                  uint64_t cap) {
  if (!t) return -1;
  if ((!roles || !contents) && n) return tok_error(t, "null messages");
  std::vector<int64_t> ids;
  std::string err;
  if (!t->tok.encode_chat(chat_turns(roles, contents, n), add_generation_prompt != 0, enable_thinking != 0, &ids,
                          &err))
    return tok_error(t, err);
  return put_ids(ids, out, cap);
}

}  // extern "C"
