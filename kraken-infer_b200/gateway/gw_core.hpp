// gw_core.hpp -- request parsing, reasoning split and response bodies of the
// OpenAI-compatible gateway (host only, no device code).
//
// The gateway is the reference's serving front end for the Qwen3.5 runtime
// (src/runtime/openai_gateway.cpp, src/runtime/reasoning_parser.cpp) rebuilt
// over the kib C ABI.  What a client sees is kept alike so that it is a
// drop-in: the routes, the request fields and their defaults, the error
// texts, the JSON of every response body and SSE chunk, and the X-Kraken-*
// headers.
#pragma once

#include <cstdint>
#include <optional>
#include <string>
#include <string_view>
#include <vector>

#include "gw_json.hpp"

namespace kib::gw {

struct GatewayConfig {
  std::string model_id = "kraken-infer-qwen3-0.6b";
  uint64_t default_max_tokens = 16;
  uint64_t prefill_chunk_tokens = 0;
  bool cache_prompt = true;
  uint64_t cache_reuse_min_tokens = 0;
  uint64_t cache_block_tokens = 0;
  uint64_t cache_capacity_blocks = 16;
  bool enable_mtp = true;
  uint64_t mtp_draft_tokens = 3;
  double mtp_p_min = 0.30;
};

enum class Reasoning { none, auto_, deepseek };

struct Sampling {  // parsed for compatibility; generation here is greedy
  bool do_sample = false;
  bool temperature_set = false, top_p_set = false, top_k_set = false, seed_set = false;
  double temperature = 0.0, top_p = 1.0;
  uint64_t top_k = 0, seed = 0;
};

struct Message {
  std::string role;
  std::string content;
  bool has_image = false;
};

// Fields both endpoints share (parse_common_generation_options,
// openai_gateway.cpp:612-712).
struct Options {
  uint64_t max_tokens = 16;
  uint64_t prefill_chunk_tokens = 0;
  bool stream = false;
  bool include_usage = false;
  bool enable_thinking = false;
  bool mtp = true;
  uint64_t mtp_draft_tokens = 3;
  double mtp_p_min = 0.30;
  bool cache_prompt = false;
  uint64_t cache_reuse_min_tokens = 0;
  uint64_t cache_block_tokens = 0;
  uint64_t cache_capacity_blocks = 0;
  std::string device;
  Sampling sampling;
};

struct ChatRequest {
  std::string model;
  std::vector<Message> messages;
  Options opt;
  Reasoning reasoning = Reasoning::none;
  std::vector<std::string> tools;
  std::optional<std::string> forced_tool;
  bool has_images() const;
};

struct CompletionRequest {
  std::string model;
  std::string prompt;
  Options opt;
};

// Throw std::runtime_error with the reference's message on a bad request.
ChatRequest parse_chat(std::string_view body, const GatewayConfig& cfg);
CompletionRequest parse_completion(std::string_view body, const GatewayConfig& cfg);

Reasoning parse_reasoning(std::string_view name);  // throws "unsupported reasoning_format: ..."
struct ReasoningText {
  std::string reasoning, content;
};
// split_reasoning_content (reasoning_parser.cpp:87-153)
ReasoningText split_reasoning(std::string_view text, bool enable_thinking, Reasoning fmt);

// ReasoningStreamParser (reasoning_parser.cpp:155-275): pieces of generated
// text in, (is_reasoning, text) deltas out; a possible start of a <think> /
// </think> tag (and trailing newlines before one) is held back until the next
// piece decides it.
class ReasoningStream {
 public:
  struct Delta {
    bool reasoning;
    std::string text;
  };
  ReasoningStream(bool enable_thinking, Reasoning fmt);
  std::vector<Delta> push(std::string_view piece);
  std::vector<Delta> finish();

 private:
  std::vector<Delta> drain(bool final);
  Reasoning fmt_;
  bool in_reasoning_;
  bool skip_reasoning_nl_;
  bool skip_content_nl_ = false;
  bool done_ = false;
  std::string held_;
};

// Response bodies (openai_gateway.cpp:1066-1071, 1322-1470).
std::string models_body(const GatewayConfig& cfg);
std::string error_body(std::string_view message, std::string_view type = "invalid_request_error");
std::string completion_body(std::string_view id, int64_t created, std::string_view model, std::string_view text,
                            std::string_view finish, uint64_t prompt_tokens, uint64_t completion_tokens,
                            uint64_t cached_tokens);
std::string chat_body(std::string_view id, int64_t created, std::string_view model, const ReasoningText& msg,
                      std::string_view finish, uint64_t prompt_tokens, uint64_t completion_tokens,
                      uint64_t cached_tokens);
std::string tool_call_body(std::string_view id, int64_t created, std::string_view model, std::string_view tool);
std::string completion_chunk(std::string_view id, int64_t created, std::string_view model, std::string_view text,
                             std::string_view finish);
std::string completion_usage_chunk(std::string_view id, int64_t created, std::string_view model,
                                   uint64_t prompt_tokens, uint64_t completion_tokens, uint64_t cached_tokens);
std::string chat_chunk(std::string_view id, int64_t created, std::string_view model, std::string_view content,
                       std::string_view reasoning, bool role, std::string_view finish);
std::string chat_usage_chunk(std::string_view id, int64_t created, std::string_view model, uint64_t prompt_tokens,
                             uint64_t completion_tokens, uint64_t cached_tokens);
std::string tool_chunk(std::string_view id, int64_t created, std::string_view model, std::string_view tool,
                       bool finish);

// One normalised JSON line describing a parsed request (or {"error": ...}):
// what the tests compare with the reference's parse of the same body.
std::string describe_chat(std::string_view body, const GatewayConfig& cfg);
std::string describe_completion(std::string_view body, const GatewayConfig& cfg);

}  // namespace kib::gw
