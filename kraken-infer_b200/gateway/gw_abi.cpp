// gw_abi.cpp -- C entry points of the gateway core (libkib_gateway_core.so),
// so the request parsing, the reasoning split and the response bodies can be
// driven from tests without a server or a GPU.  Each returns the byte length
// of its result and writes it only when it fits in cap.
#include <cstdint>
#include <cstring>
#include <string>

#include "gw_core.hpp"

using namespace kib::gw;

namespace {

int64_t put(const std::string& s, char* out, uint64_t cap) {
  if (out && s.size() <= cap) std::memcpy(out, s.data(), s.size());
  return static_cast<int64_t>(s.size());
}

GatewayConfig test_config() { return GatewayConfig{}; }

Reasoning fmt_of(int f) { return f == 1 ? Reasoning::auto_ : f == 2 ? Reasoning::deepseek : Reasoning::none; }

}  // namespace

extern "C" {

// kind 0: chat completion body, 1: text completion body; the default
// gateway configuration (model id, 16 tokens, MTP on at 3 drafts, p_min 0.30,
// prompt cache on with 16 blocks).
int64_t kib_gw_describe(int kind, const char* body, uint64_t len, char* out, uint64_t cap) {
  const std::string_view b(body ? body : "", len);
  return put(kind == 0 ? describe_chat(b, test_config()) : describe_completion(b, test_config()), out, cap);
}

// {"reasoning_content": ..., "content": ...}; fmt 0 none, 1 auto, 2 deepseek
int64_t kib_gw_split_reasoning(const char* text, uint64_t len, int enable_thinking, int fmt, char* out,
                               uint64_t cap) {
  const ReasoningText r = split_reasoning(std::string_view(text ? text : "", len), enable_thinking != 0, fmt_of(fmt));
  return put("{\"reasoning_content\":\"" + json_escape(r.reasoning) + "\",\"content\":\"" + json_escape(r.content) +
                 "\"}",
             out, cap);
}

// the n pieces (lens[i] bytes each, back to back in text) pushed in order,
// then finish: [[is_reasoning, "text"], ...] of every delta
int64_t kib_gw_stream_reasoning(const char* text, const uint64_t* lens, uint64_t n, int enable_thinking, int fmt,
                                char* out, uint64_t cap) {
  ReasoningStream rs(enable_thinking != 0, fmt_of(fmt));
  std::string s = "[";
  auto add = [&](const std::vector<ReasoningStream::Delta>& ds) {
    for (const auto& d : ds) {
      if (s.size() > 1) s += ',';
      s += std::string("[") + (d.reasoning ? "1" : "0") + ",\"" + json_escape(d.text) + "\"]";
    }
  };
  uint64_t at = 0;
  for (uint64_t i = 0; i < n; ++i) {
    add(rs.push(std::string_view(text + at, lens[i])));
    at += lens[i];
  }
  add(rs.finish());
  return put(s + "]", out, cap);
}

// which: 0 models(s0 model id) 1 error(s0 message, s1 type)
//   2 completion(s0 id, n0 created, s1 model, s2 text, s3 finish, n1 prompt, n2 completion, n3 cached)
//   3 chat(s0 id, n0, s1 model, s2 reasoning, s3 content, s4 finish, n1..n3)
//   4 tool call(s0 id, n0, s1 model, s2 tool)
//   5 completion chunk(s0, n0, s1, s2 text, s3 finish)  6 completion usage chunk(s0, n0, s1, n1..n3)
//   7 chat chunk(s0, n0, s1, s2 content, s3 reasoning, n1 role, s4 finish)  8 chat usage chunk(s0, n0, s1, n1..n3)
//   9 tool chunk(s0, n0, s1, s2 tool, n1 finish)
int64_t kib_gw_body(int which, const char* const* s, const int64_t* n, char* out, uint64_t cap) {
  auto S = [&](int i) { return std::string_view(s[i] ? s[i] : ""); };
  auto U = [&](int i) { return static_cast<uint64_t>(n[i]); };
  GatewayConfig cfg;
  std::string r;
  switch (which) {
    case 0: cfg.model_id = std::string(S(0)); r = models_body(cfg); break;
    case 1: r = error_body(S(0), S(1)); break;
    case 2: r = completion_body(S(0), n[0], S(1), S(2), S(3), U(1), U(2), U(3)); break;
    case 3: r = chat_body(S(0), n[0], S(1), ReasoningText{std::string(S(2)), std::string(S(3))}, S(4), U(1), U(2), U(3)); break;
    case 4: r = tool_call_body(S(0), n[0], S(1), S(2)); break;
    case 5: r = completion_chunk(S(0), n[0], S(1), S(2), S(3)); break;
    case 6: r = completion_usage_chunk(S(0), n[0], S(1), U(1), U(2), U(3)); break;
    case 7: r = chat_chunk(S(0), n[0], S(1), S(2), S(3), n[1] != 0, S(4)); break;
    case 8: r = chat_usage_chunk(S(0), n[0], S(1), U(1), U(2), U(3)); break;
    case 9: r = tool_chunk(S(0), n[0], S(1), S(2), n[1] != 0); break;
    default: return -1;
  }
  return put(r, out, cap);
}

}  // extern "C"
