// gw_json.hpp -- the JSON the OpenAI-compatible gateway reads and writes.
//
// A recursive-descent reader over a string_view.  Its accepted grammar, its
// number conversion (std::stod of the scanned prefix) and its error texts
// ("<what> at byte <offset>") are those of the reference gateway's parser
// (src/runtime/openai_gateway.cpp:57-302): a client sees the same 400 error
// body for the same malformed request.  \u escapes are decoded one code unit
// at a time (no surrogate pairing), as there.
#pragma once

#include <cstdint>
#include <stdexcept>
#include <string>
#include <string_view>
#include <utility>
#include <vector>

namespace kib::gw {

struct Json {
  enum class Kind { null, boolean, number, string, array, object };
  Kind kind = Kind::null;
  bool b = false;
  double num = 0.0;
  std::string str;
  std::vector<Json> arr;
  std::vector<std::pair<std::string, Json>> obj;  // in document order; lookups take the first match

  const Json* get(std::string_view key) const {
    if (kind != Kind::object) return nullptr;
    for (const auto& kv : obj)
      if (kv.first == key) return &kv.second;
    return nullptr;
  }
  bool is(Kind k) const { return kind == k; }
};

class JsonReader {
 public:
  explicit JsonReader(std::string_view s) : s_(s) {}

  Json document() {
    Json v = value();
    blanks();
    if (at_ < s_.size()) error("unexpected trailing JSON input");
    return v;
  }

 private:
  [[noreturn]] void error(std::string_view what) const {
    throw std::runtime_error(std::string(what) + " at byte " + std::to_string(at_));
  }
  void blanks() {
    while (at_ < s_.size() && (s_[at_] == ' ' || s_[at_] == '\n' || s_[at_] == '\r' || s_[at_] == '\t')) ++at_;
  }
  bool take(char c) {
    blanks();
    if (at_ < s_.size() && s_[at_] == c) {
      ++at_;
      return true;
    }
    return false;
  }
  void need(char c) {
    blanks();
    if (at_ >= s_.size() || s_[at_] != c) error(std::string("expected JSON character ") + c);
    ++at_;
  }
  bool word(std::string_view w) {
    if (s_.substr(at_, w.size()) != w) return false;
    at_ += w.size();
    return true;
  }
  static bool digit(char c) { return c >= '0' && c <= '9'; }

  Json value() {
    blanks();
    if (at_ >= s_.size()) error("unexpected end of JSON");
    Json v;
    const char c = s_[at_];
    if (c == '"') {
      v.kind = Json::Kind::string;
      v.str = string();
    } else if (c == '{') {
      v = object();
    } else if (c == '[') {
      v = array();
    } else if (c == '-' || digit(c)) {
      v = number();
    } else if (word("true")) {
      v.kind = Json::Kind::boolean;
      v.b = true;
    } else if (word("false")) {
      v.kind = Json::Kind::boolean;
    } else if (!word("null")) {
      error("unsupported JSON value");
    }
    return v;
  }

  Json object() {
    need('{');
    Json v;
    v.kind = Json::Kind::object;
    if (take('}')) return v;
    for (;;) {
      std::string key = string();
      need(':');
      Json item = value();
      v.obj.emplace_back(std::move(key), std::move(item));
      if (take('}')) return v;
      need(',');
    }
  }

  Json array() {
    need('[');
    Json v;
    v.kind = Json::Kind::array;
    if (take(']')) return v;
    for (;;) {
      v.arr.push_back(value());
      if (take(']')) return v;
      need(',');
    }
  }

  // sign, digits, optional fraction, optional exponent; the scanned text goes
  // to std::stod (which may reject it, e.g. a lone "-")
  Json number() {
    const size_t from = at_;
    if (at_ < s_.size() && s_[at_] == '-') ++at_;
    while (at_ < s_.size() && digit(s_[at_])) ++at_;
    if (at_ < s_.size() && s_[at_] == '.') {
      ++at_;
      while (at_ < s_.size() && digit(s_[at_])) ++at_;
    }
    if (at_ < s_.size() && (s_[at_] == 'e' || s_[at_] == 'E')) {
      ++at_;
      if (at_ < s_.size() && (s_[at_] == '+' || s_[at_] == '-')) ++at_;
      while (at_ < s_.size() && digit(s_[at_])) ++at_;
    }
    Json v;
    v.kind = Json::Kind::number;
    v.num = std::stod(std::string(s_.substr(from, at_ - from)));
    return v;
  }

  std::string string() {
    need('"');
    std::string out;
    while (at_ < s_.size()) {
      const char c = s_[at_++];
      if (c == '"') return out;
      if (c != '\\') {
        out.push_back(c);
        continue;
      }
      if (at_ >= s_.size()) error("unterminated JSON escape");
      const char e = s_[at_++];
      switch (e) {
        case '"': case '\\': case '/': out.push_back(e); break;
        case 'b': out.push_back('\b'); break;
        case 'f': out.push_back('\f'); break;
        case 'n': out.push_back('\n'); break;
        case 'r': out.push_back('\r'); break;
        case 't': out.push_back('\t'); break;
        case 'u': unit(&out); break;
        default: error("unsupported JSON escape");
      }
    }
    error("unterminated JSON string");
  }

  // one \uXXXX code unit, written as UTF-8 of at most three bytes
  void unit(std::string* out) {
    if (at_ + 4 > s_.size()) error("invalid JSON unicode escape");
    unsigned cp = 0;
    for (int i = 0; i < 4; ++i) {
      const char h = s_[at_++];
      cp <<= 4;
      if (digit(h)) cp += static_cast<unsigned>(h - '0');
      else if (h >= 'a' && h <= 'f') cp += static_cast<unsigned>(h - 'a' + 10);
      else if (h >= 'A' && h <= 'F') cp += static_cast<unsigned>(h - 'A' + 10);
      else error("invalid JSON unicode escape");
    }
    if (cp < 0x80) {
      out->push_back(static_cast<char>(cp));
    } else if (cp < 0x800) {
      out->push_back(static_cast<char>(0xC0 | (cp >> 6)));
      out->push_back(static_cast<char>(0x80 | (cp & 0x3F)));
    } else {
      out->push_back(static_cast<char>(0xE0 | (cp >> 12)));
      out->push_back(static_cast<char>(0x80 | ((cp >> 6) & 0x3F)));
      out->push_back(static_cast<char>(0x80 | (cp & 0x3F)));
    }
  }

  std::string_view s_;
  size_t at_ = 0;
};

inline Json parse_json(std::string_view text) { return JsonReader(text).document(); }

// String contents for a JSON literal: quote, backslash and the control
// characters escaped (\b \f \n \r \t by name, the rest as \u00XX); every
// other byte, UTF-8 included, as is.
inline std::string json_escape(std::string_view text) {
  static const char hex[] = "0123456789abcdef";
  std::string out;
  out.reserve(text.size() + 8);
  for (const char c : text) {
    const auto u = static_cast<unsigned char>(c);
    switch (c) {
      case '"': out += "\\\""; break;
      case '\\': out += "\\\\"; break;
      case '\b': out += "\\b"; break;
      case '\f': out += "\\f"; break;
      case '\n': out += "\\n"; break;
      case '\r': out += "\\r"; break;
      case '\t': out += "\\t"; break;
      default:
        if (u < 0x20) {
          out += "\\u00";
          out.push_back(hex[u >> 4]);
          out.push_back(hex[u & 15]);
        } else {
          out.push_back(c);
        }
    }
  }
  return out;
}

}  // namespace kib::gw
