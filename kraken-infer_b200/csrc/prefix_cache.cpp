// prefix_cache.cpp -- the exact-prefix block index of the host prompt cache.
//
// Restates Qwen35PrefixCacheIndex (src/runtime/qwen35_prefix_cache.cpp of the
// reference): a prompt is cut into blocks of block_tokens; block b's key is a
// hash chained from block b-1's (FNV-style mixing of the block size, the block
// index and every token id, never 0); lookup walks the chain from the root
// while every block is stored with the same parent and the same tokens,
// refreshing each hit's LRU tick; hits below min_reuse_tokens count as a
// miss; a commit that finds the cache full evicts the least recently used
// block.  The hash arithmetic, the match rules and the LRU policy have to be
// the reference's for a cache that behaves like its (the same prompts hit).
// Host-only C++: linked into libkib.so (with the device payloads in
// engine.cu) and into libkib_gguf.so, so the index is testable without a GPU.
#include "prefix_cache.hpp"

#include <algorithm>

namespace kib {
namespace {

constexpr uint64_t kRoot = 1469598103934665603ull;
constexpr uint64_t kPrime = 1099511628211ull;

uint64_t mix(uint64_t h, uint64_t v) { return (h ^ v) * kPrime; }

}  // namespace

PrefixIndex::PrefixIndex(uint64_t block_tokens, uint64_t capacity_blocks, uint64_t min_reuse_tokens)
    : block_(block_tokens), capacity_(capacity_blocks), min_reuse_(min_reuse_tokens) {}

bool PrefixIndex::enabled() const { return block_ > 0 && capacity_ > 0; }

uint64_t PrefixIndex::hash_block(const int64_t* tokens, uint64_t start, uint64_t parent) const {
  uint64_t h = parent;
  h = mix(h, block_);
  h = mix(h, start / block_);
  for (uint64_t i = 0; i < block_; ++i) h = mix(h, static_cast<uint64_t>(tokens[start + i]));
  return h == 0 ? 1 : h;
}

uint64_t PrefixIndex::parent_of(const int64_t* tokens, uint64_t start) const {
  uint64_t p = kRoot;
  for (uint64_t s = 0; s < start; s += block_) p = hash_block(tokens, s, p);
  return p;
}

PrefixBlock* PrefixIndex::find(uint64_t hash) {
  for (auto& b : blocks_)
    if (b.hash == hash) return &b;
  return nullptr;
}

uint64_t PrefixIndex::lookup(const int64_t* tokens, uint64_t n, std::vector<uint64_t>* hashes) {
  if (hashes) hashes->clear();
  if (!enabled()) {
    miss_ += n;
    return 0;
  }
  uint64_t hit = 0, parent = kRoot;
  std::vector<uint64_t> found;
  for (uint64_t start = 0; start + block_ <= n; start += block_) {
    const uint64_t h = hash_block(tokens, start, parent);
    PrefixBlock* b = find(h);
    if (!b || b->parent != parent || b->tokens.size() != block_) break;
    if (!std::equal(b->tokens.begin(), b->tokens.end(), tokens + start)) break;
    b->tick = ++tick_;
    hit += block_;
    found.push_back(h);
    parent = h;
  }
  if (hit < min_reuse_) {
    hit = 0;
    found.clear();
  }
  hit_ += hit;
  miss_ += n - hit;
  if (hashes) *hashes = found;
  return hit;
}

PrefixCommit PrefixIndex::commit(const int64_t* tokens, uint64_t n, uint64_t start) {
  PrefixCommit r;
  if (!enabled() || start + block_ > n || start % block_) return r;
  const uint64_t parent = parent_of(tokens, start);
  r.hash = hash_block(tokens, start, parent);
  if (PrefixBlock* b = find(r.hash)) {
    b->tick = ++tick_;
    r.slot = b->slot;
    return r;
  }
  if (blocks_.size() < capacity_) {
    r.slot = blocks_.size();
  } else {
    auto victim = blocks_.begin();
    for (auto it = blocks_.begin(); it != blocks_.end(); ++it)
      if (it->tick < victim->tick) victim = it;
    r.slot = victim->slot;
    r.evicted = true;
    r.evicted_hash = victim->hash;
    blocks_.erase(victim);
    ++evicted_;
  }
  PrefixBlock b;
  b.hash = r.hash;
  b.parent = parent;
  b.slot = r.slot;
  b.start = start;
  b.tokens.assign(tokens + start, tokens + start + block_);
  b.tick = ++tick_;
  blocks_.push_back(std::move(b));
  committed_ += block_;
  r.inserted = true;
  return r;
}

void PrefixIndex::stats(uint64_t out[6]) const {
  out[0] = blocks_.size();
  out[1] = hit_;
  out[2] = miss_;
  out[3] = committed_;
  out[4] = evicted_;
  out[5] = block_;
}

}  // namespace kib

// ------------------------------------------------------------------ C ABI
using kib::PrefixIndex;

struct kib_prefix_index {
  PrefixIndex idx;
  kib_prefix_index(uint64_t b, uint64_t c, uint64_t m) : idx(b, c, m) {}
};

extern "C" {

kib_prefix_index* kib_prefix_index_create(uint64_t block_tokens, uint64_t capacity_blocks,
                                          uint64_t min_reuse_tokens) {
  return new kib_prefix_index(block_tokens, capacity_blocks, min_reuse_tokens);
}

void kib_prefix_index_free(kib_prefix_index* p) { delete p; }

uint64_t kib_prefix_index_lookup(kib_prefix_index* p, const int64_t* tokens, uint64_t n, uint64_t* hashes_out,
                                 uint64_t max_hashes) {
  if (!p || (!tokens && n)) return 0;
  std::vector<uint64_t> h;
  const uint64_t hit = p->idx.lookup(tokens, n, &h);
  if (hashes_out)
    for (size_t i = 0; i < h.size() && i < max_hashes; ++i) hashes_out[i] = h[i];
  return hit;
}

int kib_prefix_index_commit(kib_prefix_index* p, const int64_t* tokens, uint64_t n, uint64_t start,
                            uint64_t* hash_out, uint64_t* evicted_hash_out) {
  if (!p || !tokens) return -1;
  const kib::PrefixCommit r = p->idx.commit(tokens, n, start);
  if (hash_out) *hash_out = r.hash;
  if (evicted_hash_out) *evicted_hash_out = r.evicted ? r.evicted_hash : 0;
  return (r.inserted ? 1 : 0) | (r.evicted ? 2 : 0);
}

void kib_prefix_index_stats(const kib_prefix_index* p, uint64_t* out6) {
  if (p && out6) p->idx.stats(out6);
}

}  // extern "C"
