// gw_server.cpp -- kib_gateway: the OpenAI-compatible HTTP gateway over the
// B200 runtime (the reference's `kraken-infer serve`, serve_openai_gateway in
// src/runtime/openai_gateway.cpp).
//
// One process owns one GPU context, one loaded model, its tokenizer and one
// host prompt cache; requests are served one at a time on the accepting thread
// (as the reference does; a request is never run concurrently with another on
// the model's stream).  Routes: GET /health, /v1/health, /v1/models; POST
// /v1/completions and /v1/chat/completions, JSON or SSE (`stream`).  Generation
// is greedy, with MTP speculative decoding when the model has a NextN layer
// and the request allows it; sampling fields are parsed but not applied
// (reported in an X-Kraken-Sampling header).
#include <arpa/inet.h>
#include <netinet/in.h>
#include <signal.h>
#include <sys/socket.h>
#include <unistd.h>

#include <algorithm>
#include <cerrno>
#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <functional>
#include <string>
#include <vector>

#include "gw_core.hpp"
#include "kib.h"

using namespace kib::gw;

namespace {

using Headers = std::vector<std::pair<std::string, std::string>>;

// ------------------------------------------------------------------ HTTP
struct HttpRequest {
  std::string method, path, body;
  Headers headers;  // names lower-cased
  std::string header(const std::string& name) const {
    for (const auto& h : headers)
      if (h.first == name) return h.second;
    return {};
  }
};

bool send_all(int fd, std::string_view data) {
  while (!data.empty()) {
    const ssize_t k = ::send(fd, data.data(), data.size(), MSG_NOSIGNAL);
    if (k <= 0) return false;
    data.remove_prefix(static_cast<size_t>(k));
  }
  return true;
}

const char* status_text(int s) {
  switch (s) {
    case 200: return "OK";
    case 400: return "Bad Request";
    case 404: return "Not Found";
    case 405: return "Method Not Allowed";
    case 413: return "Payload Too Large";
    case 429: return "Too Many Requests";
    case 500: return "Internal Server Error";
    case 501: return "Not Implemented";
    default: return "Error";
  }
}

void send_json(int fd, int status, const std::string& body, const Headers& extra = {}) {
  std::string r = "HTTP/1.1 " + std::to_string(status) + " " + status_text(status) +
                  "\r\nContent-Type: application/json\r\n";
  for (const auto& h : extra) r += h.first + ": " + h.second + "\r\n";
  r += "Content-Length: " + std::to_string(body.size()) + "\r\nConnection: close\r\n\r\n" + body;
  send_all(fd, r);
}

void send_sse_head(int fd, const Headers& extra) {
  std::string r = "HTTP/1.1 200 OK\r\nContent-Type: text/event-stream\r\nCache-Control: no-cache\r\n";
  for (const auto& h : extra) r += h.first + ": " + h.second + "\r\n";
  send_all(fd, r + "Connection: close\r\n\r\n");
}

bool send_sse(int fd, std::string_view json) { return send_all(fd, "data: " + std::string(json) + "\n\n"); }

// Reads one request: the head up to the blank line, then Content-Length bytes.
bool read_request(int fd, HttpRequest* rq, std::string* err) {
  std::string buf;
  char chunk[65536];
  size_t head_end = std::string::npos;
  constexpr size_t kMax = 64u << 20;
  while ((head_end = buf.find("\r\n\r\n")) == std::string::npos) {
    const ssize_t k = ::recv(fd, chunk, sizeof chunk, 0);
    if (k <= 0) return false;
    buf.append(chunk, static_cast<size_t>(k));
    if (buf.size() > kMax) {
      *err = "request head too large";
      return false;
    }
  }
  const std::string head = buf.substr(0, head_end);
  size_t line_end = head.find("\r\n");
  const std::string first = head.substr(0, line_end);
  const size_t sp1 = first.find(' '), sp2 = first.find(' ', sp1 + 1);
  if (sp1 == std::string::npos || sp2 == std::string::npos) {
    *err = "malformed HTTP request line";
    return false;
  }
  rq->method = first.substr(0, sp1);
  rq->path = first.substr(sp1 + 1, sp2 - sp1 - 1);
  if (const size_t q = rq->path.find('?'); q != std::string::npos) rq->path.resize(q);
  size_t at = line_end == std::string::npos ? head.size() : line_end + 2;
  while (at < head.size()) {
    size_t e = head.find("\r\n", at);
    if (e == std::string::npos) e = head.size();
    const std::string line = head.substr(at, e - at);
    if (const size_t c = line.find(':'); c != std::string::npos) {
      std::string name = line.substr(0, c), value = line.substr(c + 1);
      std::transform(name.begin(), name.end(), name.begin(), [](unsigned char ch) { return std::tolower(ch); });
      value.erase(0, value.find_first_not_of(" \t"));
      rq->headers.emplace_back(name, value);
    }
    at = e + 2;
  }
  const size_t want = static_cast<size_t>(std::strtoull(rq->header("content-length").c_str(), nullptr, 10));
  if (want > kMax) {
    *err = "request body too large";
    return false;
  }
  rq->body = buf.substr(head_end + 4);
  while (rq->body.size() < want) {
    const ssize_t k = ::recv(fd, chunk, std::min(sizeof chunk, want - rq->body.size()), 0);
    if (k <= 0) return false;
    rq->body.append(chunk, static_cast<size_t>(k));
  }
  rq->body.resize(std::min(rq->body.size(), want));
  return true;
}

uint64_t micros() {
  return static_cast<uint64_t>(
      std::chrono::duration_cast<std::chrono::microseconds>(std::chrono::steady_clock::now().time_since_epoch())
          .count());
}
int64_t unix_seconds() {
  return std::chrono::duration_cast<std::chrono::seconds>(std::chrono::system_clock::now().time_since_epoch())
      .count();
}

}  // namespace

namespace {

// ------------------------------------------------------------------ the served model
struct Gateway {
  GatewayConfig cfg;
  kib_ctx* ctx = nullptr;
  kib_qwen35* model = nullptr;
  kib_tokenizer* tok = nullptr;
  uint64_t chunk = 1024;  // the model's prefill chunk: the prompt cache's block
  int mtp_layers = 0;
  kib_qwen35_prefix_cache* cache = nullptr;
  uint64_t cache_capacity = 0, cache_min_reuse = 0;
  uint64_t requests = 0;
};

struct Generation {
  int rc = KIB_OK;
  std::string error;
  std::vector<int32_t> ids;
  kib_generation_result res{};
  bool cache_on = false;
  uint64_t cached = 0, committed = 0;
  bool mtp_on = false;
  std::string mtp_off_reason;
  std::string text;  // all generated tokens decoded, control tokens skipped
};

std::string token_text(Gateway& g, const int32_t* ids, size_t n) {
  std::vector<int64_t> v(ids, ids + n);
  const int64_t len = kib_tokenizer_decode(g.tok, v.data(), v.size(), 1, nullptr, 0);
  if (len <= 0) return {};
  std::string s(static_cast<size_t>(len), '\0');
  kib_tokenizer_decode(g.tok, v.data(), v.size(), 1, s.data(), s.size());
  return s;
}

struct StreamCtx {
  Gateway* g;
  std::function<bool(const std::string&)> on_text;  // false: the client is gone
};

int on_token(void* user, int32_t token, uint64_t) {
  auto* s = static_cast<StreamCtx*>(user);
  return s->on_text(token_text(*s->g, &token, 1)) ? 0 : 1;
}

// The generate request of one HTTP request.  MTP and the prompt cache are
// switched as the reference's runtime switches them (qwen35_runtime.cpp:
// 5468-5492 MTP availability, 5521-5542 prompt-cache conditions: the cache
// block is the prefill chunk, and MTP requests bypass the cache).
Generation generate(Gateway& g, const std::vector<int64_t>& prompt, const Options& o,
                    std::function<bool(const std::string&)> on_text) {
  Generation out;
  std::vector<int32_t> p(prompt.begin(), prompt.end());
  if (g.mtp_layers == 0) out.mtp_off_reason = "model_has_no_mtp_layers";
  else if (!o.mtp) out.mtp_off_reason = "request_disabled";
  else if (g.mtp_layers != 1) out.mtp_off_reason = "only_single_mtp_layer_supported";
  else if (o.sampling.do_sample) out.mtp_off_reason = "sampling_not_supported_in_first_mtp_pass";
  else if (o.mtp_draft_tokens == 0) out.mtp_off_reason = "draft_tokens_zero";
  else out.mtp_on = true;
  const uint64_t block = o.cache_block_tokens ? o.cache_block_tokens : g.chunk;
  const uint64_t capacity = o.cache_capacity_blocks ? o.cache_capacity_blocks : 16;
  out.cache_on = o.cache_prompt && block == g.chunk && capacity > 0 && !out.mtp_on;
  if (out.cache_on && (!g.cache || g.cache_capacity != capacity || g.cache_min_reuse != o.cache_reuse_min_tokens)) {
    if (g.cache) kib_qwen35_prefix_cache_free(g.cache);
    g.cache = nullptr;
    if (kib_qwen35_prefix_cache_create(g.model, block, capacity, o.cache_reuse_min_tokens, &g.cache) != KIB_OK) {
      out.cache_on = false;
    } else {
      g.cache_capacity = capacity;
      g.cache_min_reuse = o.cache_reuse_min_tokens;
    }
  }
  uint64_t before[6] = {0, 0, 0, 0, 0, 0};
  if (out.cache_on) kib_qwen35_prefix_cache_stats(g.cache, before);
  kib_generation_request rq{};
  rq.prompt_tokens = p.data();
  rq.prompt_count = p.size();
  rq.max_new_tokens = o.max_tokens;
  rq.prefill_chunk_tokens = o.prefill_chunk_tokens;
  rq.enable_mtp = out.mtp_on ? 1 : 0;
  rq.mtp_draft_tokens = o.mtp_draft_tokens;
  rq.mtp_p_min = o.mtp_p_min;
  rq.mtp_adaptive = 1;
  rq.ignore_eos = 0;
  // the model's own EOS (tokenizer.ggml.eos_token_id of its GGUF) always
  // stops; a separate tokenizer file's EOS stops as well
  int64_t info[9];
  kib_tokenizer_info(g.tok, info);
  rq.eos_token_id = info[3] >= 0 ? static_cast<uint64_t>(info[3]) : UINT64_MAX;
  out.ids.assign(std::max<uint64_t>(1, o.max_tokens), 0);
  StreamCtx sc{&g, std::move(on_text)};
  out.rc = kib_generate_qwen35_stream(g.model, &rq, out.cache_on ? g.cache : nullptr, sc.on_text ? on_token : nullptr,
                                      &sc, out.ids.data(), out.ids.size(), &out.res, &out.cached);
  if (out.rc != KIB_OK) {
    const char* e = kib_last_error(g.ctx);
    out.error = e && *e ? e : "generation failed";
    out.ids.clear();
    return out;
  }
  out.ids.resize(out.res.generated_tokens);
  if (out.cache_on) {
    uint64_t after[6];
    kib_qwen35_prefix_cache_stats(g.cache, after);
    out.committed = after[3] - before[3];
  }
  out.text = token_text(g, out.ids.data(), out.ids.size());
  return out;
}

std::string joined(const uint64_t* v, uint64_t n) {
  std::string s;
  for (uint64_t i = 0; i < n; ++i) s += (i ? "," : "") + std::to_string(v[i]);
  return s;
}

// X-Request-Id, then the prompt-cache and MTP statistics headers
// (request_headers, openai_gateway.cpp:863-930)
Headers stats_headers(const std::string& request_id, const Gateway& g, const Generation& r, const Options& o) {
  Headers h{{"X-Request-Id", request_id}};
  if (r.cache_on) {
    h.push_back({"X-Kraken-Prompt-Cache-Hit-Tokens", std::to_string(r.cached)});
    h.push_back({"X-Kraken-Prompt-Cache-Miss-Tokens", std::to_string(r.res.prompt_tokens - r.cached)});
    h.push_back({"X-Kraken-Prompt-Cache-Committed-Tokens", std::to_string(r.committed)});
  }
  if (g.mtp_layers > 0) {
    const kib_mtp_report& m = r.res.mtp;
    h.push_back({"X-Kraken-MTP-Enabled", r.mtp_on ? "1" : "0"});
    h.push_back({"X-Kraken-MTP-Layers", std::to_string(g.mtp_layers)});
    h.push_back({"X-Kraken-MTP-Draft-Tokens", std::to_string(o.mtp_draft_tokens)});
    h.push_back({"X-Kraken-MTP-P-Min", std::to_string(o.mtp_p_min)});
    h.push_back({"X-Kraken-MTP-Drafted-Tokens", std::to_string(m.drafted_tokens)});
    h.push_back({"X-Kraken-MTP-Accepted-Tokens", std::to_string(m.accepted_tokens)});
    h.push_back({"X-Kraken-MTP-Verify-Steps", std::to_string(m.verify_steps)});
    h.push_back({"X-Kraken-MTP-Confidence-Stops", std::to_string(m.confidence_stops)});
    h.push_back({"X-Kraken-MTP-Adaptive-Budget", std::to_string(r.mtp_on ? m.adaptive_budget : 0)});
    h.push_back({"X-Kraken-MTP-Adaptive-Changes", std::to_string(m.adaptive_changes)});
    if (r.mtp_on) {
      const uint64_t n = std::min<uint64_t>(o.mtp_draft_tokens, 8);
      h.push_back({"X-Kraken-MTP-Verified-By-Position", joined(m.verified_by_position, n)});
      h.push_back({"X-Kraken-MTP-Accepted-By-Position", joined(m.accepted_by_position, n)});
    } else {
      h.push_back({"X-Kraken-MTP-Disabled-Reason", r.mtp_off_reason});
    }
  }
  if (o.sampling.do_sample) h.push_back({"X-Kraken-Sampling", "greedy"});
  return h;
}

const char* finish_of(const Generation& r) { return r.res.finish_reason_stop ? "stop" : "length"; }

void serve_completion(Gateway& g, int fd, const CompletionRequest& rq, const std::string& request_id) {
  const int64_t len = kib_tokenizer_encode(g.tok, rq.prompt.data(), rq.prompt.size(), 0, 0, nullptr, 0);
  if (len < 0) {
    send_json(fd, 500, error_body(kib_tokenizer_last_error(g.tok), "server_error"), {{"X-Request-Id", request_id}});
    return;
  }
  std::vector<int64_t> ids(static_cast<size_t>(len));
  kib_tokenizer_encode(g.tok, rq.prompt.data(), rq.prompt.size(), 0, 0, ids.data(), ids.size());
  const std::string id = "cmpl-" + std::to_string(micros());
  const int64_t created = unix_seconds();
  if (!rq.opt.stream) {
    const Generation r = generate(g, ids, rq.opt, nullptr);
    if (r.rc != KIB_OK) {
      send_json(fd, 500, error_body(r.error, "server_error"), {{"X-Request-Id", request_id}});
      return;
    }
    send_json(fd, 200,
              completion_body(id, created, rq.model, r.text, finish_of(r), r.res.prompt_tokens,
                              r.res.generated_tokens, r.cached),
              stats_headers(request_id, g, r, rq.opt));
    return;
  }
  send_sse_head(fd, {{"X-Request-Id", request_id}});
  const Generation r = generate(g, ids, rq.opt, [&](const std::string& text) {
    return send_sse(fd, completion_chunk(id, created, rq.model, text, ""));
  });
  if (r.rc != KIB_OK) {
    send_sse(fd, error_body(r.error, "server_error"));
  } else {
    send_sse(fd, completion_chunk(id, created, rq.model, "", finish_of(r)));
    if (rq.opt.include_usage)
      send_sse(fd, completion_usage_chunk(id, created, rq.model, r.res.prompt_tokens, r.res.generated_tokens, r.cached));
  }
  send_sse(fd, "[DONE]");
}

void serve_chat(Gateway& g, int fd, const ChatRequest& rq, const std::string& request_id) {
  if (rq.has_images()) {
    // no vision path here: the reference's answer when it runs without --mmproj
    send_json(fd, 400,
              error_body("image input requires starting the gateway with --mmproj pointing to the Qwen3.5 "
                         "conditional mmproj GGUF"),
              {{"X-Request-Id", request_id}});
    return;
  }
  const std::string id = "chatcmpl-" + std::to_string(micros());
  const int64_t created = unix_seconds();
  if (rq.forced_tool) {
    // tool_choice forces the call: answered without generating (openai_gateway.cpp:1582-1598)
    if (!rq.opt.stream) {
      send_json(fd, 200, tool_call_body(id, created, rq.model, *rq.forced_tool), {{"X-Request-Id", request_id}});
      return;
    }
    send_sse_head(fd, {{"X-Request-Id", request_id}});
    send_sse(fd, tool_chunk(id, created, rq.model, *rq.forced_tool, false));
    send_sse(fd, tool_chunk(id, created, rq.model, *rq.forced_tool, true));
    if (rq.opt.include_usage) send_sse(fd, chat_usage_chunk(id, created, rq.model, 0, 0, 0));
    send_sse(fd, "[DONE]");
    return;
  }
  std::vector<const char*> roles, contents;
  for (const Message& m : rq.messages) {
    roles.push_back(m.role.c_str());
    contents.push_back(m.content.c_str());
  }
  const int64_t len = kib_tokenizer_encode_chat(g.tok, roles.data(), contents.data(), roles.size(), 1,
                                                rq.opt.enable_thinking, nullptr, 0);
  if (len < 0) {
    send_json(fd, 500, error_body(kib_tokenizer_last_error(g.tok), "server_error"), {{"X-Request-Id", request_id}});
    return;
  }
  std::vector<int64_t> ids(static_cast<size_t>(len));
  kib_tokenizer_encode_chat(g.tok, roles.data(), contents.data(), roles.size(), 1, rq.opt.enable_thinking, ids.data(),
                            ids.size());
  if (!rq.opt.stream) {
    const Generation r = generate(g, ids, rq.opt, nullptr);
    if (r.rc != KIB_OK) {
      send_json(fd, 500, error_body(r.error, "server_error"), {{"X-Request-Id", request_id}});
      return;
    }
    send_json(fd, 200,
              chat_body(id, created, rq.model, split_reasoning(r.text, rq.opt.enable_thinking, rq.reasoning),
                        finish_of(r), r.res.prompt_tokens, r.res.generated_tokens, r.cached),
              stats_headers(request_id, g, r, rq.opt));
    return;
  }
  send_sse_head(fd, {{"X-Request-Id", request_id}});
  send_sse(fd, chat_chunk(id, created, rq.model, "", "", true, ""));
  ReasoningStream rs(rq.opt.enable_thinking, rq.reasoning);
  auto send_deltas = [&](const std::vector<ReasoningStream::Delta>& ds) {
    bool ok = true;
    for (const auto& d : ds)
      ok = send_sse(fd, d.reasoning ? chat_chunk(id, created, rq.model, "", d.text, false, "")
                                    : chat_chunk(id, created, rq.model, d.text, "", false, "")) && ok;
    return ok;
  };
  const Generation r = generate(g, ids, rq.opt, [&](const std::string& text) { return send_deltas(rs.push(text)); });
  if (r.rc != KIB_OK) {
    send_sse(fd, error_body(r.error, "server_error"));
  } else {
    send_deltas(rs.finish());
    send_sse(fd, chat_chunk(id, created, rq.model, "", "", false, finish_of(r)));
    if (rq.opt.include_usage)
      send_sse(fd, chat_usage_chunk(id, created, rq.model, r.res.prompt_tokens, r.res.generated_tokens, r.cached));
  }
  send_sse(fd, "[DONE]");
}

void handle(Gateway& g, int fd) {
  HttpRequest rq;
  std::string err;
  if (!read_request(fd, &rq, &err)) {
    if (!err.empty()) send_json(fd, 400, error_body(err));
    return;
  }
  const std::string request_id = "req-" + std::to_string(micros());
  try {
    if (rq.path == "/health" || rq.path == "/v1/health") {
      if (rq.method != "GET") return send_json(fd, 405, error_body("method not allowed"));
      return send_json(fd, 200, "{\"status\":\"ok\"}");
    }
    if (rq.path == "/v1/models") {
      if (rq.method != "GET") return send_json(fd, 405, error_body("method not allowed"));
      return send_json(fd, 200, models_body(g.cfg));
    }
    if (rq.path == "/v1/completions") {
      if (rq.method != "POST") return send_json(fd, 405, error_body("method not allowed"));
      return serve_completion(g, fd, parse_completion(rq.body, g.cfg), request_id);
    }
    if (rq.path == "/v1/chat/completions") {
      if (rq.method != "POST") return send_json(fd, 405, error_body("method not allowed"));
      return serve_chat(g, fd, parse_chat(rq.body, g.cfg), request_id);
    }
    send_json(fd, 404, error_body("route not found"));
  } catch (const std::exception& e) {
    send_json(fd, 400, error_body(e.what()));
  }
}

int usage() {
  std::fprintf(stderr,
               "usage: kib_gateway --model model.gguf [--tokenizer tok.gguf] [--host 127.0.0.1] [--port 8080]\n"
               "       [--model-id ID] [--ctx 4096] [--max-tokens 16] [--prefill-chunk 1024] [--no-mtp]\n"
               "       [--mtp-draft-tokens 3] [--mtp-p-min 0.30] [--no-cache-prompt] [--cache-capacity 16]\n"
               "       [--max-requests N] [--device 0]\n");
  return 2;
}

}  // namespace

int main(int argc, char** argv) {
  Gateway g;
  std::string model_path, tok_path, host = "127.0.0.1";
  int port = 8080, device = 0;
  uint64_t ctx_tokens = 4096, max_requests = 0;
  for (int i = 1; i < argc; ++i) {
    const std::string a = argv[i];
    auto next = [&]() -> std::string { return i + 1 < argc ? argv[++i] : std::string(); };
    if (a == "--model") model_path = next();
    else if (a == "--tokenizer") tok_path = next();
    else if (a == "--host") host = next();
    else if (a == "--port") port = std::atoi(next().c_str());
    else if (a == "--model-id") g.cfg.model_id = next();
    else if (a == "--ctx") ctx_tokens = std::strtoull(next().c_str(), nullptr, 10);
    else if (a == "--max-tokens") g.cfg.default_max_tokens = std::strtoull(next().c_str(), nullptr, 10);
    else if (a == "--prefill-chunk") g.chunk = std::strtoull(next().c_str(), nullptr, 10);
    else if (a == "--no-mtp") g.cfg.enable_mtp = false;
    else if (a == "--mtp-draft-tokens") g.cfg.mtp_draft_tokens = std::strtoull(next().c_str(), nullptr, 10);
    else if (a == "--mtp-p-min") g.cfg.mtp_p_min = std::atof(next().c_str());
    else if (a == "--no-cache-prompt") g.cfg.cache_prompt = false;
    else if (a == "--cache-capacity") g.cfg.cache_capacity_blocks = std::strtoull(next().c_str(), nullptr, 10);
    else if (a == "--max-requests") max_requests = std::strtoull(next().c_str(), nullptr, 10);
    else if (a == "--device") device = std::atoi(next().c_str());
    else return usage();
  }
  if (model_path.empty() || port < 0 || port > 65535) return usage();
  if (kib_create(device, &g.ctx) != KIB_OK) {
    std::fprintf(stderr, "kib_gateway: no usable GPU (kib_create failed)\n");
    return 1;
  }
  kib_qwen35_options opt{};
  opt.context_tokens = ctx_tokens;
  opt.decode_tokens = 256;
  opt.prefill_chunk_tokens = g.chunk;
  opt.sequence_slots = 1;
  opt.kv_cache_f16 = 1;
  opt.enable_mtp = 1;
  if (kib_qwen35_load(g.ctx, model_path.c_str(), &opt, &g.model) != KIB_OK) {
    std::fprintf(stderr, "kib_gateway: cannot load %s: %s\n", model_path.c_str(), kib_last_error(g.ctx));
    return 1;
  }
  kib_qwen35_plan plan{};
  kib_qwen35_get_plan(g.model, &plan);
  g.mtp_layers = plan.mtp_layers;
  g.tok = kib_tokenizer_load((tok_path.empty() ? model_path : tok_path).c_str());
  if (!g.tok) {
    std::fprintf(stderr, "kib_gateway: no tokenizer: %s\n", kib_tokenizer_load_error());
    return 1;
  }
  signal(SIGPIPE, SIG_IGN);
  const int srv = ::socket(AF_INET, SOCK_STREAM, 0);
  int one = 1;
  setsockopt(srv, SOL_SOCKET, SO_REUSEADDR, &one, sizeof one);
  sockaddr_in addr{};
  addr.sin_family = AF_INET;
  addr.sin_port = htons(static_cast<uint16_t>(port));
  if (inet_pton(AF_INET, host.c_str(), &addr.sin_addr) != 1 ||
      ::bind(srv, reinterpret_cast<sockaddr*>(&addr), sizeof addr) != 0 || ::listen(srv, 64) != 0) {
    std::fprintf(stderr, "kib_gateway: cannot listen on %s:%d: %s\n", host.c_str(), port, std::strerror(errno));
    return 1;
  }
  socklen_t alen = sizeof addr;
  getsockname(srv, reinterpret_cast<sockaddr*>(&addr), &alen);
  std::printf("kib_gateway listening on %s:%d model=%s\n", host.c_str(), ntohs(addr.sin_port), g.cfg.model_id.c_str());
  std::fflush(stdout);
  while (max_requests == 0 || g.requests < max_requests) {
    const int fd = ::accept(srv, nullptr, nullptr);
    if (fd < 0) {
      if (errno == EINTR) continue;
      break;
    }
    handle(g, fd);
    ::close(fd);
    ++g.requests;
  }
  ::close(srv);
  if (g.cache) kib_qwen35_prefix_cache_free(g.cache);
  kib_tokenizer_free(g.tok);
  kib_qwen35_free(g.model);
  kib_destroy(g.ctx);
  return 0;
}
