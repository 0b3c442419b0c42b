// prefix_cache.hpp -- exact-prefix block index of the host prompt cache
// (prefix_cache.cpp).
#pragma once

#include <cstdint>
#include <vector>

namespace kib {

struct PrefixBlock {
  uint64_t hash = 0, parent = 0, slot = 0, start = 0, tick = 0;
  std::vector<int64_t> tokens;
};

struct PrefixCommit {
  bool inserted = false, evicted = false;
  uint64_t hash = 0, evicted_hash = 0, slot = 0;
};

class PrefixIndex {
 public:
  PrefixIndex(uint64_t block_tokens, uint64_t capacity_blocks, uint64_t min_reuse_tokens);
  bool enabled() const;
  uint64_t block_tokens() const { return block_; }
  // Tokens of the longest stored block-aligned prefix (0 below min_reuse) and
  // the hashes of its blocks in order.
  uint64_t lookup(const int64_t* tokens, uint64_t n, std::vector<uint64_t>* hashes);
  // Records block [start, start + block_tokens) of tokens (LRU eviction when full).
  PrefixCommit commit(const int64_t* tokens, uint64_t n, uint64_t start);
  uint64_t hash_for(const int64_t* tokens, uint64_t start) const { return hash_block(tokens, start, parent_of(tokens, start)); }
  // stored blocks, hit tokens, miss tokens, committed tokens, evicted blocks, block tokens
  void stats(uint64_t out[6]) const;

 private:
  uint64_t hash_block(const int64_t* tokens, uint64_t start, uint64_t parent) const;
  uint64_t parent_of(const int64_t* tokens, uint64_t start) const;
  PrefixBlock* find(uint64_t hash);
  uint64_t block_, capacity_, min_reuse_;
  std::vector<PrefixBlock> blocks_;
  uint64_t tick_ = 0, hit_ = 0, miss_ = 0, committed_ = 0, evicted_ = 0;
};

}  // namespace kib
