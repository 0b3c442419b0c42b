// ref_gateway_shim.cpp -- TEST INFRASTRUCTURE ONLY.
//
// The reference gateway's request parsing and response bodies live in an
// anonymous namespace of src/runtime/openai_gateway.cpp; this translation unit
// compiles that file in place (included by path from the reference checkout
// named by -DKIB_REF_GATEWAY_TU) and exposes them, with the reference's
// reasoning parser, through the same C entry points as the repository's
// gateway core (kraken-infer_b200/gateway/gw_abi.cpp), so the tests can feed
// both the same requests.  Nothing from the reference is copied here.
#define KIB_GW_STR2(x) #x
#define KIB_GW_STR(x) KIB_GW_STR2(x)
#include KIB_GW_STR(KIB_REF_GATEWAY_TU)

#include <cstdio>
#include <cstring>

namespace {

int64_t gw_put(const std::string& s, char* out, uint64_t cap) {
  if (out && s.size() <= cap) std::memcpy(out, s.data(), s.size());
  return static_cast<int64_t>(s.size());
}

std::string gw_real(double x) {
  char b[64];
  std::snprintf(b, sizeof b, "%.17g", x);
  return b;
}

const char* gw_device(const toyllm::Device& d) {
  switch (d.kind) {
    case toyllm::DeviceKind::mps: return "mps";
    case toyllm::DeviceKind::mpsgraph: return "mpsgraph";
    default: return "cpu";
  }
}

// the same normalised description the repository's gw_core.cpp writes
template <typename R>
std::string gw_options(const R& r) {
  std::ostringstream s;
  const auto& sm = r.sampling;
  s << "\"max_tokens\":" << r.max_tokens << ",\"prefill_chunk_tokens\":" << r.prefill_chunk_tokens
    << ",\"stream\":" << r.stream << ",\"include_usage\":" << r.stream_include_usage
    << ",\"enable_thinking\":" << r.enable_thinking << ",\"mtp\":" << r.enable_mtp
    << ",\"mtp_draft_tokens\":" << r.mtp_draft_tokens << ",\"mtp_p_min\":" << gw_real(r.mtp_p_min)
    << ",\"cache_prompt\":" << r.cache_prompt << ",\"n_cache_reuse\":" << r.cache_reuse_min_tokens
    << ",\"cache_block_tokens\":" << r.cache_block_tokens << ",\"cache_capacity_blocks\":" << r.cache_capacity_blocks
    << ",\"device\":\"" << gw_device(r.compute_device) << "\",\"do_sample\":" << sm.do_sample
    << ",\"temperature\":" << (sm.temperature_set ? gw_real(sm.temperature) : "null")
    << ",\"top_p\":" << (sm.top_p_set ? gw_real(sm.top_p) : "null")
    << ",\"top_k\":" << (sm.top_k_set ? std::to_string(sm.top_k) : "null")
    << ",\"seed\":" << (sm.seed_set ? std::to_string(sm.seed) : "null");
  return s.str();
}

toyllm::ReasoningFormat gw_fmt(int f) {
  return f == 1 ? toyllm::ReasoningFormat::auto_
                : f == 2 ? toyllm::ReasoningFormat::deepseek : toyllm::ReasoningFormat::none;
}

}  // namespace

extern "C" {

int64_t ref_gw_describe(int kind, const char* body, uint64_t len, char* out, uint64_t cap) {
  const std::string_view b(body ? body : "", len);
  toyllm::OpenAIGatewayConfig cfg;
  try {
    if (kind == 0) {
      const auto r = toyllm::parse_chat_request(b, cfg);
      std::string s = "{\"model\":\"" + toyllm::json_escape(r.model) + "\",\"messages\":[";
      for (size_t i = 0; i < r.messages.size(); ++i) {
        if (i) s += ',';
        s += "[\"" + toyllm::json_escape(r.messages[i].role) + "\",\"" + toyllm::json_escape(r.messages[i].content) +
             "\"," + (toyllm::chat_message_has_image_content(r.messages[i]) ? "1" : "0") + "]";
      }
      s += "]," + gw_options(r) + ",\"reasoning_format\":" + std::to_string(static_cast<int>(r.reasoning_format)) +
           ",\"tools\":[";
      for (size_t i = 0; i < r.tools.size(); ++i) s += (i ? ",\"" : "\"") + toyllm::json_escape(r.tools[i].name) + "\"";
      s += "],\"forced_tool\":" +
           (r.forced_tool ? "\"" + toyllm::json_escape(*r.forced_tool) + "\"" : std::string("null")) + "}";
      return gw_put(s, out, cap);
    }
    const auto r = toyllm::parse_completion_request(b, cfg);
    return gw_put("{\"model\":\"" + toyllm::json_escape(r.model) + "\",\"prompt\":\"" +
                      toyllm::json_escape(r.prompt) + "\"," + gw_options(r) + "}",
                  out, cap);
  } catch (const std::exception& e) {
    return gw_put("{\"error\":\"" + toyllm::json_escape(e.what()) + "\"}", out, cap);
  }
}

int64_t ref_gw_split_reasoning(const char* text, uint64_t len, int enable_thinking, int fmt, char* out,
                               uint64_t cap) {
  const auto m = toyllm::split_reasoning_content(std::string_view(text ? text : "", len), enable_thinking != 0,
                                                 gw_fmt(fmt));
  return gw_put("{\"reasoning_content\":\"" + toyllm::json_escape(m.reasoning_content) + "\",\"content\":\"" +
                    toyllm::json_escape(m.content) + "\"}",
                out, cap);
}

int64_t ref_gw_stream_reasoning(const char* text, const uint64_t* lens, uint64_t n, int enable_thinking, int fmt,
                                char* out, uint64_t cap) {
  toyllm::ReasoningStreamParser p(enable_thinking != 0, gw_fmt(fmt));
  std::string s = "[";
  auto add = [&](const std::vector<toyllm::ReasoningDelta>& ds) {
    for (const auto& d : ds) {
      if (s.size() > 1) s += ',';
      s += std::string("[") + (d.kind == toyllm::ReasoningDelta::Kind::reasoning ? "1" : "0") + ",\"" +
           toyllm::json_escape(d.text) + "\"]";
    }
  };
  uint64_t at = 0;
  for (uint64_t i = 0; i < n; ++i) {
    add(p.push(std::string_view(text + at, lens[i])));
    at += lens[i];
  }
  add(p.finish());
  return gw_put(s + "]", out, cap);
}

int64_t ref_gw_body(int which, const char* const* s, const int64_t* n, char* out, uint64_t cap) {
  auto S = [&](int i) { return std::string_view(s[i] ? s[i] : ""); };
  auto U = [&](int i) { return static_cast<std::size_t>(n[i]); };
  toyllm::OpenAIGatewayConfig cfg;
  std::string r;
  switch (which) {
    case 0: cfg.model_id = std::string(S(0)); r = toyllm::models_body(cfg); break;
    case 1: r = toyllm::error_body(S(0), S(1)); break;
    case 2: r = toyllm::completion_body(S(0), n[0], S(1), S(2), S(3), U(1), U(2), U(3)); break;
    case 3: {
      toyllm::ReasoningMessage m;
      m.reasoning_content = std::string(S(2));
      m.content = std::string(S(3));
      r = toyllm::chat_completion_body(S(0), n[0], S(1), m, S(4), U(1), U(2), U(3));
      break;
    }
    case 4: r = toyllm::tool_call_body(S(0), n[0], S(1), S(2)); break;
    case 5: r = toyllm::completion_stream_chunk(S(0), n[0], S(1), S(2), S(3)); break;
    case 6: r = toyllm::completion_stream_usage_chunk(S(0), n[0], S(1), U(1), U(2), U(3)); break;
    case 7: r = toyllm::stream_chunk(S(0), n[0], S(1), S(2), S(3), n[1] != 0, S(4)); break;
    case 8: r = toyllm::stream_usage_chunk(S(0), n[0], S(1), U(1), U(2), U(3)); break;
    case 9: r = toyllm::tool_stream_chunk(S(0), n[0], S(1), S(2), n[1] != 0); break;
    default: return -1;
  }
  return gw_put(r, out, cap);
}

}  // extern "C"
