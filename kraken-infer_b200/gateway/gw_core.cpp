// gw_core.cpp -- request parsing, reasoning split and response bodies of the
// gateway.  Field names, defaults, parse order (which decides which error a
// bad request reports) and error texts follow the reference gateway
// (src/runtime/openai_gateway.cpp:373-812); the reasoning split follows
// src/runtime/reasoning_parser.cpp.
#include "gw_core.hpp"

#include <cstdio>
#include <limits>
#include <stdexcept>

namespace kib::gw {
namespace {

using K = Json::Kind;

[[noreturn]] void bad(const std::string& what) { throw std::runtime_error(what); }

std::string str_or(const Json* v, std::string_view dflt = {}) {
  return v && v->is(K::string) ? v->str : std::string(dflt);
}
bool bool_or(const Json* v, bool dflt) { return v && v->is(K::boolean) ? v->b : dflt; }
// absent or null: dflt; a boolean: its value; anything else: an error
bool strict_bool(const Json* v, const std::string& name, bool dflt) {
  if (!v || v->is(K::null)) return dflt;
  if (!v->is(K::boolean)) bad(name + " must be a boolean");
  return v->b;
}
// a non-negative number in range, truncated; otherwise "not given"
std::optional<uint64_t> count_of(const Json* v) {
  if (!v || !v->is(K::number) || v->num < 0.0) return std::nullopt;
  if (v->num > static_cast<double>(std::numeric_limits<uint64_t>::max())) return std::nullopt;
  return static_cast<uint64_t>(v->num);
}
std::optional<double> real_of(const Json* v) {
  if (!v || !v->is(K::number)) return std::nullopt;
  return v->num;
}

Message read_message_content(const Json* c, Message m) {
  if (!c || c->is(K::null)) return m;
  if (c->is(K::string)) {
    m.content = c->str;
    return m;
  }
  if (!c->is(K::array)) bad("message content must be a string, null, or content array");
  for (const Json& part : c->arr) {
    if (!part.is(K::object)) bad("message content array entries must be objects");
    const std::string type = str_or(part.get("type"));
    if (type == "text") {
      const Json* t = part.get("text");
      if (!t || !t->is(K::string)) bad("message content text part requires string text");
      m.content += t->str;
    } else if (type == "image_url") {
      const Json* iu = part.get("image_url");
      std::string url;
      if (iu && iu->is(K::string)) {
        url = iu->str;
      } else if (iu && iu->is(K::object)) {
        const Json* u = iu->get("url");
        if (!u || !u->is(K::string)) bad("message content image_url part requires image_url.url");
        url = u->str;
      } else {
        bad("message content image_url part requires image_url");
      }
      if (url.empty()) bad("message content image_url.url must not be empty");
      m.has_image = true;
    } else {
      bad("unsupported message content part type: " + type);
    }
  }
  return m;
}

std::vector<Message> read_messages(const Json* v) {
  if (!v || !v->is(K::array)) bad("messages must be an array");
  std::vector<Message> out;
  for (const Json& item : v->arr) {
    if (!item.is(K::object)) bad("message entries must be objects");
    const std::string role = str_or(item.get("role"));
    Message m = read_message_content(item.get("content"), Message{role, {}, false});
    if (role == "system" || role == "user" || role == "assistant") {
      out.push_back(std::move(m));
    } else if (role == "tool") {
      // a tool result goes back to the model as a user turn
      m.content = "Tool result " + str_or(item.get("tool_call_id"), "tool") + ":\n" + m.content;
      m.role = "user";
      out.push_back(std::move(m));
    } else {
      bad("unsupported message role: " + role);
    }
  }
  if (out.empty()) bad("messages must not be empty");
  return out;
}

Options read_options(const Json& root, const GatewayConfig& cfg) {
  Options o;
  o.max_tokens = cfg.default_max_tokens;
  if (auto n = count_of(root.get("max_tokens"))) o.max_tokens = *n;
  if (auto n = count_of(root.get("max_completion_tokens"))) o.max_tokens = *n;
  o.prefill_chunk_tokens = cfg.prefill_chunk_tokens;
  if (auto n = count_of(root.get("prefill_chunk_tokens"))) o.prefill_chunk_tokens = *n;
  o.stream = bool_or(root.get("stream"), false);
  if (const Json* so = root.get("stream_options"); so && so->is(K::object))
    o.include_usage = strict_bool(so->get("include_usage"), "stream_options.include_usage", false);
  o.enable_thinking = strict_bool(root.get("enable_thinking"), "enable_thinking", false);
  if (const Json* kw = root.get("chat_template_kwargs")) {
    if (!kw->is(K::object)) bad("chat_template_kwargs must be an object");
    o.enable_thinking =
        strict_bool(kw->get("enable_thinking"), "chat_template_kwargs.enable_thinking", o.enable_thinking);
  }
  o.mtp = strict_bool(root.get("mtp"), "mtp", cfg.enable_mtp);
  o.mtp_draft_tokens = cfg.mtp_draft_tokens;
  if (auto n = count_of(root.get("mtp_draft_tokens"))) o.mtp_draft_tokens = *n;
  o.mtp_p_min = cfg.mtp_p_min;
  if (auto x = real_of(root.get("mtp_p_min"))) o.mtp_p_min = *x;
  if (!(o.mtp_p_min >= 0.0 && o.mtp_p_min <= 1.0)) bad("mtp_p_min must be in [0, 1]");
  o.device = str_or(root.get("device"));
  Sampling& s = o.sampling;
  if (auto x = real_of(root.get("temperature"))) s.do_sample = s.temperature_set = true, s.temperature = *x;
  if (auto x = real_of(root.get("top_p"))) s.do_sample = s.top_p_set = true, s.top_p = *x;
  if (auto n = count_of(root.get("top_k"))) s.do_sample = s.top_k_set = true, s.top_k = *n;
  if (auto n = count_of(root.get("seed"))) s.do_sample = s.seed_set = true, s.seed = *n;
  o.cache_prompt = strict_bool(root.get("cache_prompt"), "cache_prompt", cfg.cache_prompt);
  o.cache_reuse_min_tokens = cfg.cache_reuse_min_tokens;
  if (auto n = count_of(root.get("n_cache_reuse"))) o.cache_reuse_min_tokens = *n;
  o.cache_block_tokens = cfg.cache_block_tokens;
  if (auto n = count_of(root.get("cache_block_tokens"))) o.cache_block_tokens = *n;
  o.cache_capacity_blocks = cfg.cache_capacity_blocks;
  if (auto n = count_of(root.get("cache_capacity_blocks"))) o.cache_capacity_blocks = *n;
  return o;
}

Json read_root(std::string_view body) {
  Json root = parse_json(body);
  if (!root.is(K::object)) bad("request body must be a JSON object");
  return root;
}

std::string read_prompt(const Json* v) {
  if (!v) bad("prompt is required");
  if (v->is(K::string)) {
    if (v->str.empty()) bad("prompt must not be empty");
    return v->str;
  }
  if (!v->is(K::array)) bad("prompt must be a string or string array");
  std::string out;
  for (const Json& item : v->arr) {
    if (!item.is(K::string)) bad("prompt array entries must be strings");
    if (!out.empty()) out.push_back('\n');
    out += item.str;
  }
  if (out.empty()) bad("prompt must not be empty");
  return out;
}

}  // namespace

bool ChatRequest::has_images() const {
  for (const Message& m : messages)
    if (m.has_image) return true;
  return false;
}

Reasoning parse_reasoning(std::string_view name) {
  if (name == "none") return Reasoning::none;
  if (name == "auto") return Reasoning::auto_;
  if (name == "deepseek") return Reasoning::deepseek;
  bad("unsupported reasoning_format: " + std::string(name));
}

ChatRequest parse_chat(std::string_view body, const GatewayConfig& cfg) {
  const Json root = read_root(body);
  ChatRequest r;
  r.model = str_or(root.get("model"), cfg.model_id);
  r.messages = read_messages(root.get("messages"));
  r.opt = read_options(root, cfg);
  if (const Json* rf = root.get("reasoning_format"); rf && !rf->is(K::null)) {
    if (!rf->is(K::string)) bad("reasoning_format must be a string");
    r.reasoning = parse_reasoning(rf->str);
  }
  // tools: the named functions; tool_choice "required" or {"function":{"name"}}
  // forces a call without generating (openai_gateway.cpp:548-582)
  if (const Json* tools = root.get("tools"); tools && tools->is(K::array)) {
    for (const Json& t : tools->arr) {
      const Json* fn = t.get("function");
      const Json* name = fn ? fn->get("name") : nullptr;
      if (name && name->is(K::string) && !name->str.empty()) r.tools.push_back(name->str);
    }
  }
  if (const Json* tc = root.get("tool_choice"); tc && !r.tools.empty()) {
    if (tc->is(K::string)) {
      if (tc->str == "required") r.forced_tool = r.tools.front();
    } else {
      const Json* fn = tc->get("function");
      const Json* name = fn ? fn->get("name") : nullptr;
      if (name && name->is(K::string) && !name->str.empty()) r.forced_tool = name->str;
    }
  }
  return r;
}

CompletionRequest parse_completion(std::string_view body, const GatewayConfig& cfg) {
  const Json root = read_root(body);
  CompletionRequest r;
  r.model = str_or(root.get("model"), cfg.model_id);
  r.prompt = read_prompt(root.get("prompt"));
  r.opt = read_options(root, cfg);
  return r;
}

// ------------------------------------------------------------------ reasoning
namespace {

constexpr std::string_view kOpen = "<think>", kClose = "</think>";

bool nl(char c) { return c == '\n' || c == '\r'; }
std::string_view drop_leading_nl(std::string_view t) {
  while (!t.empty() && nl(t.front())) t.remove_prefix(1);
  return t;
}
std::string drop_trailing_nl(std::string_view t) {
  while (!t.empty() && nl(t.back())) t.remove_suffix(1);
  return std::string(t);
}
bool extracts(Reasoning f) { return f == Reasoning::auto_ || f == Reasoning::deepseek; }
// longest proper prefix of tag that ends the text (a tag that may be cut)
size_t partial_tag(std::string_view text, std::string_view tag) {
  for (size_t k = std::min(text.size(), tag.size() - 1); k > 0; --k)
    if (text.substr(text.size() - k) == tag.substr(0, k)) return k;
  return 0;
}

}  // namespace

ReasoningText split_reasoning(std::string_view text, bool enable_thinking, Reasoning fmt) {
  ReasoningText r;
  if (!extracts(fmt)) {
    r.content = std::string(text);
    return r;
  }
  if (!enable_thinking) {
    // the text is content unless it opens a think block somewhere
    const size_t open = text.find(kOpen);
    if (open == std::string_view::npos) {
      r.content = std::string(text);
      return r;
    }
    r.content = std::string(text.substr(0, open));
    text = drop_leading_nl(text.substr(open + kOpen.size()));
  } else if (text.substr(0, kOpen.size()) == kOpen) {
    // thinking: the text starts inside the block (an explicit <think> is skipped)
    text = drop_leading_nl(text.substr(kOpen.size()));
  }
  const size_t close = text.find(kClose);
  r.reasoning = drop_trailing_nl(text.substr(0, close));
  if (close != std::string_view::npos) r.content += std::string(drop_leading_nl(text.substr(close + kClose.size())));
  return r;
}

ReasoningStream::ReasoningStream(bool enable_thinking, Reasoning fmt)
    : fmt_(fmt), in_reasoning_(enable_thinking && extracts(fmt)), skip_reasoning_nl_(in_reasoning_) {}

std::vector<ReasoningStream::Delta> ReasoningStream::push(std::string_view piece) {
  if (done_) return {};
  held_ += piece;
  return drain(false);
}

std::vector<ReasoningStream::Delta> ReasoningStream::finish() {
  if (done_) return {};
  done_ = true;
  return drain(true);
}

std::vector<ReasoningStream::Delta> ReasoningStream::drain(bool final) {
  std::vector<Delta> out;
  auto add = [&](bool reasoning, std::string text) {
    if (text.empty()) return;
    if (!out.empty() && out.back().reasoning == reasoning) out.back().text += text;
    else out.push_back(Delta{reasoning, std::move(text)});
  };
  if (!extracts(fmt_)) {
    add(false, std::move(held_));
    held_.clear();
    return out;
  }
  while (!held_.empty()) {
    if (in_reasoning_) {
      if (skip_reasoning_nl_) {
        held_.erase(0, held_.size() - drop_leading_nl(held_).size());
        skip_reasoning_nl_ = false;
        if (held_.empty()) break;
      }
      if (held_.compare(0, kOpen.size(), kOpen) == 0 && held_.size() >= kOpen.size()) {
        held_.erase(0, kOpen.size());
        skip_reasoning_nl_ = true;
        continue;
      }
      const size_t close = held_.find(kClose);
      if (close != std::string::npos) {
        add(true, drop_trailing_nl(std::string_view(held_).substr(0, close)));
        held_.erase(0, close + kClose.size());
        in_reasoning_ = false;
        skip_content_nl_ = true;
        continue;
      }
      // hold back a possible start of </think> and the newlines before it
      size_t hold = 0;
      if (!final) {
        const size_t tag = partial_tag(held_, kClose);
        const std::string_view before = std::string_view(held_).substr(0, held_.size() - tag);
        size_t nls = 0;
        while (nls < before.size() && nl(before[before.size() - 1 - nls])) ++nls;
        hold = tag + nls;
      }
      if (held_.size() == hold) break;
      std::string piece = held_.substr(0, held_.size() - hold);
      if (final) piece = drop_trailing_nl(piece);
      add(true, std::move(piece));
      held_.erase(0, held_.size() - hold);
      continue;
    }
    if (skip_content_nl_) {
      held_.erase(0, held_.size() - drop_leading_nl(held_).size());
      if (held_.empty()) break;
      skip_content_nl_ = false;
    }
    const size_t open = held_.find(kOpen);
    if (open != std::string::npos) {
      add(false, held_.substr(0, open));
      held_.erase(0, open + kOpen.size());
      in_reasoning_ = true;
      skip_reasoning_nl_ = true;
      continue;
    }
    const size_t hold = final ? 0 : partial_tag(held_, kOpen);
    if (held_.size() == hold) break;
    add(false, held_.substr(0, held_.size() - hold));
    held_.erase(0, held_.size() - hold);
  }
  return out;
}

// ------------------------------------------------------------------ bodies
namespace {

std::string esc(std::string_view s) { return json_escape(s); }

std::string N(uint64_t v) { return std::to_string(v); }

std::string usage(uint64_t prompt, uint64_t completion, uint64_t cached) {
  cached = std::min(cached, prompt);
  return "\"usage\":{\"prompt_tokens\":" + N(prompt) + ",\"completion_tokens\":" + N(completion) +
         ",\"total_tokens\":" + N(prompt + completion) + ",\"prompt_tokens_details\":{\"cached_tokens\":" +
         N(cached) + "}}";
}

std::string head(std::string_view id, std::string_view object, int64_t created, std::string_view model) {
  return "{\"id\":\"" + esc(id) + "\",\"object\":\"" + std::string(object) + "\",\"created\":" +
         std::to_string(created) + ",\"model\":\"" + esc(model) + "\",";
}

std::string finish_field(std::string_view finish) {
  return finish.empty() ? std::string("null") : "\"" + esc(finish) + "\"";
}

}  // namespace

std::string models_body(const GatewayConfig& cfg) {
  return "{\"object\":\"list\",\"data\":[{\"id\":\"" + esc(cfg.model_id) +
         "\",\"object\":\"model\",\"created\":0,\"owned_by\":\"kraken-infer\"}]}";
}

std::string error_body(std::string_view message, std::string_view type) {
  return "{\"error\":{\"message\":\"" + esc(message) + "\",\"type\":\"" + esc(type) +
         "\",\"param\":null,\"code\":null}}";
}

std::string completion_body(std::string_view id, int64_t created, std::string_view model, std::string_view text,
                            std::string_view finish, uint64_t prompt_tokens, uint64_t completion_tokens,
                            uint64_t cached_tokens) {
  return head(id, "text_completion", created, model) + "\"choices\":[{\"index\":0,\"text\":\"" + esc(text) +
         "\",\"finish_reason\":\"" + esc(finish) + "\"}]," + usage(prompt_tokens, completion_tokens, cached_tokens) +
         "}";
}

std::string chat_body(std::string_view id, int64_t created, std::string_view model, const ReasoningText& msg,
                      std::string_view finish, uint64_t prompt_tokens, uint64_t completion_tokens,
                      uint64_t cached_tokens) {
  std::string o = head(id, "chat.completion", created, model) + "\"choices\":[{\"index\":0,\"message\":{\"role\":\"assistant\"";
  if (!msg.reasoning.empty()) o += ",\"reasoning_content\":\"" + esc(msg.reasoning) + "\"";
  o += ",\"content\":\"" + esc(msg.content) + "\"},\"finish_reason\":\"" + esc(finish) + "\"}],";
  return o + usage(prompt_tokens, completion_tokens, cached_tokens) + "}";
}

std::string tool_call_body(std::string_view id, int64_t created, std::string_view model, std::string_view tool) {
  return head(id, "chat.completion", created, model) +
         "\"choices\":[{\"index\":0,\"message\":{\"role\":\"assistant\",\"content\":null,\"tool_calls\":[{\"id\":"
         "\"call_0\",\"type\":\"function\",\"function\":{\"name\":\"" +
         esc(tool) + "\",\"arguments\":\"{}\"}}]},\"finish_reason\":\"tool_calls\"}]," + usage(0, 0, 0) + "}";
}

std::string completion_chunk(std::string_view id, int64_t created, std::string_view model, std::string_view text,
                             std::string_view finish) {
  return head(id, "text_completion", created, model) + "\"choices\":[{\"index\":0,\"text\":\"" + esc(text) +
         "\",\"finish_reason\":" + finish_field(finish) + "}]}";
}

std::string completion_usage_chunk(std::string_view id, int64_t created, std::string_view model,
                                   uint64_t prompt_tokens, uint64_t completion_tokens, uint64_t cached_tokens) {
  return head(id, "text_completion", created, model) + "\"choices\":[]," +
         usage(prompt_tokens, completion_tokens, cached_tokens) + "}";
}

std::string chat_chunk(std::string_view id, int64_t created, std::string_view model, std::string_view content,
                       std::string_view reasoning, bool role, std::string_view finish) {
  std::string delta;
  auto field = [&](const std::string& f) {
    if (!delta.empty()) delta += ',';
    delta += f;
  };
  if (role) field("\"role\":\"assistant\"");
  if (!reasoning.empty()) field("\"reasoning_content\":\"" + esc(reasoning) + "\"");
  if (!content.empty()) field("\"content\":\"" + esc(content) + "\"");
  return head(id, "chat.completion.chunk", created, model) + "\"choices\":[{\"index\":0,\"delta\":{" + delta +
         "},\"finish_reason\":" + finish_field(finish) + "}]}";
}

std::string chat_usage_chunk(std::string_view id, int64_t created, std::string_view model, uint64_t prompt_tokens,
                             uint64_t completion_tokens, uint64_t cached_tokens) {
  return head(id, "chat.completion.chunk", created, model) + "\"choices\":[]," +
         usage(prompt_tokens, completion_tokens, cached_tokens) + "}";
}

std::string tool_chunk(std::string_view id, int64_t created, std::string_view model, std::string_view tool,
                       bool finish) {
  std::string d = finish ? std::string("{}")
                         : "{\"role\":\"assistant\",\"tool_calls\":[{\"index\":0,\"id\":\"call_0\",\"type\":"
                           "\"function\",\"function\":{\"name\":\"" +
                               esc(tool) + "\",\"arguments\":\"{}\"}}]}";
  return head(id, "chat.completion.chunk", created, model) + "\"choices\":[{\"index\":0,\"delta\":" + d +
         ",\"finish_reason\":" + (finish ? "\"tool_calls\"" : "null") + "}]}";
}

// ------------------------------------------------------------------ describe
namespace {

std::string real(double x) {
  char b[64];
  std::snprintf(b, sizeof b, "%.17g", x);
  return b;
}

// the device a request names, as the reference maps it (the B200 gateway
// runs every request on its GPU whatever it names)
const char* device_name(const std::string& d) {
  if (d == "mps" || d == "mps:0") return "mps";
  if (d == "mpsgraph") return "mpsgraph";
  return "cpu";
}

std::string describe_options(const Options& o) {
  auto B = [](bool v) { return std::string(v ? "1" : "0"); };
  const Sampling& m = o.sampling;
  return "\"max_tokens\":" + N(o.max_tokens) + ",\"prefill_chunk_tokens\":" + N(o.prefill_chunk_tokens) +
         ",\"stream\":" + B(o.stream) + ",\"include_usage\":" + B(o.include_usage) +
         ",\"enable_thinking\":" + B(o.enable_thinking) + ",\"mtp\":" + B(o.mtp) + ",\"mtp_draft_tokens\":" +
         N(o.mtp_draft_tokens) + ",\"mtp_p_min\":" + real(o.mtp_p_min) + ",\"cache_prompt\":" + B(o.cache_prompt) +
         ",\"n_cache_reuse\":" + N(o.cache_reuse_min_tokens) + ",\"cache_block_tokens\":" +
         N(o.cache_block_tokens) + ",\"cache_capacity_blocks\":" + N(o.cache_capacity_blocks) + ",\"device\":\"" +
         device_name(o.device) + "\",\"do_sample\":" + B(m.do_sample) +
         ",\"temperature\":" + (m.temperature_set ? real(m.temperature) : "null") +
         ",\"top_p\":" + (m.top_p_set ? real(m.top_p) : "null") +
         ",\"top_k\":" + (m.top_k_set ? N(m.top_k) : "null") + ",\"seed\":" + (m.seed_set ? N(m.seed) : "null");
}

}  // namespace

std::string describe_chat(std::string_view body, const GatewayConfig& cfg) {
  try {
    const ChatRequest r = parse_chat(body, cfg);
    std::string s = "{\"model\":\"" + esc(r.model) + "\",\"messages\":[";
    for (size_t i = 0; i < r.messages.size(); ++i) {
      if (i) s += ',';
      s += "[\"" + esc(r.messages[i].role) + "\",\"" + esc(r.messages[i].content) + "\"," +
           (r.messages[i].has_image ? "1" : "0") + "]";
    }
    s += "]," + describe_options(r.opt) + ",\"reasoning_format\":" +
         std::to_string(static_cast<int>(r.reasoning)) + ",\"tools\":[";
    for (size_t i = 0; i < r.tools.size(); ++i) s += (i ? ",\"" : "\"") + esc(r.tools[i]) + "\"";
    s += "],\"forced_tool\":" + (r.forced_tool ? "\"" + esc(*r.forced_tool) + "\"" : std::string("null")) + "}";
    return s;
  } catch (const std::exception& e) {
    return "{\"error\":\"" + esc(e.what()) + "\"}";
  }
}

std::string describe_completion(std::string_view body, const GatewayConfig& cfg) {
  try {
    const CompletionRequest r = parse_completion(body, cfg);
    return "{\"model\":\"" + esc(r.model) + "\",\"prompt\":\"" + esc(r.prompt) + "\"," + describe_options(r.opt) +
           "}";
  } catch (const std::exception& e) {
    return "{\"error\":\"" + esc(e.what()) + "\"}";
  }
}

}  // namespace kib::gw
