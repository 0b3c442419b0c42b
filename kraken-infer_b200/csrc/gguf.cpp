// gguf.cpp -- GGUF v3 reader (mmap), writer, K-quant quantizers and the
// synthetic Qwen3.5 model generator.  Host code only.
#include "gguf.hpp"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <thread>

namespace kib {

namespace {

enum : uint32_t {
  kU8 = 0, kI8 = 1, kU16 = 2, kI16 = 3, kU32 = 4, kI32 = 5, kF32 = 6, kBool = 7,
  kString = 8, kArray = 9, kU64 = 10, kI64 = 11, kF64 = 12
};

struct Cursor {
  const uint8_t* p;
  const uint8_t* end;
  bool ok = true;
  template <typename T>
  T get() {
    T v{};
    if (static_cast<size_t>(end - p) < sizeof(T)) {
      ok = false;
      return v;
    }
    std::memcpy(&v, p, sizeof(T));
    p += sizeof(T);
    return v;
  }
  std::string str() {
    const uint64_t n = get<uint64_t>();
    if (!ok || static_cast<uint64_t>(end - p) < n) {
      ok = false;
      return {};
    }
    std::string s(reinterpret_cast<const char*>(p), n);
    p += n;
    return s;
  }
};

double read_num(Cursor& c, uint32_t t, bool* ok) {
  *ok = true;
  switch (t) {
    case kU8: return c.get<uint8_t>();
    case kI8: return c.get<int8_t>();
    case kU16: return c.get<uint16_t>();
    case kI16: return c.get<int16_t>();
    case kU32: return c.get<uint32_t>();
    case kI32: return c.get<int32_t>();
    case kF32: return c.get<float>();
    case kBool: return c.get<uint8_t>();
    case kU64: return static_cast<double>(c.get<uint64_t>());
    case kI64: return static_cast<double>(c.get<int64_t>());
    case kF64: return c.get<double>();
    default: *ok = false; return 0.0;
  }
}

// IEEE float -> half bits, round to nearest even.
uint16_t f32_to_f16(float f) {
  uint32_t x;
  std::memcpy(&x, &f, 4);
  const uint32_t sign = (x >> 16) & 0x8000u, a = x & 0x7FFFFFFFu;
  if (a >= 0x7F800000u) return static_cast<uint16_t>(sign | 0x7C00u | (a > 0x7F800000u ? 0x200u : 0u));
  if (a >= 0x477FF000u) return static_cast<uint16_t>(sign | 0x7C00u);
  if (a < 0x38800000u) {
    if (a < 0x33000000u) return static_cast<uint16_t>(sign);
    const uint32_t e = a >> 23, m = (a & 0x7FFFFFu) | 0x800000u, sh = 126u - e;
    uint32_t q = m >> sh;
    const uint32_t rem = m & ((1u << sh) - 1u), hw = 1u << (sh - 1u);
    if (rem > hw || (rem == hw && (q & 1u))) ++q;
    return static_cast<uint16_t>(sign | q);
  }
  uint32_t h = (((a >> 23) - 112u) << 10) | ((a & 0x7FFFFFu) >> 13);
  const uint32_t rem = a & 0x1FFFu;
  if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) ++h;
  return static_cast<uint16_t>(sign | h);
}

float f16_to_f32(uint16_t h) {
  const uint32_t s = (h >> 15) & 1u, e = (h >> 10) & 31u, m = h & 1023u;
  float r;
  if (e == 0) r = std::ldexp(static_cast<float>(m), -24);
  else if (e == 31) r = m ? NAN : INFINITY;
  else r = std::ldexp(1.0f + static_cast<float>(m) / 1024.0f, static_cast<int>(e) - 15);
  return s ? -r : r;
}

int nearest(float v) { return static_cast<int>(std::lrintf(v)); }

// Packs Q4_K/Q5_K 6-bit scales and mins (inverse of q4_k_scale_min,
// mps_backend.mm:282-293).
void pack_scales(const int sc[8], const int mn[8], uint8_t* s) {
  for (int j = 0; j < 4; ++j) {
    s[j] = static_cast<uint8_t>((sc[j] & 63) | ((sc[j + 4] >> 4) << 6));
    s[j + 4] = static_cast<uint8_t>((mn[j] & 63) | ((mn[j + 4] >> 4) << 6));
    s[j + 8] = static_cast<uint8_t>((sc[j + 4] & 15) | ((mn[j + 4] & 15) << 4));
  }
}

// Shared Q4_K/Q5_K quantizer: sub-block affine fit x ~ d*sc*q - dmin*m with
// q in [0, levels].
void quantize_qk_affine(const float* x, uint8_t* blk, int levels, bool q5) {
  float scale[8], minv[8];
  for (int j = 0; j < 8; ++j) {
    float mn = 0.0f, mx = -INFINITY;
    for (int i = 0; i < 32; ++i) {
      mn = std::min(mn, x[32 * j + i]);
      mx = std::max(mx, x[32 * j + i]);
    }
    mx = std::max(mx, mn);
    scale[j] = (mx - mn) / static_cast<float>(levels);
    minv[j] = -mn;
  }
  float ms = 0.0f, mm = 0.0f;
  for (int j = 0; j < 8; ++j) {
    ms = std::max(ms, scale[j]);
    mm = std::max(mm, minv[j]);
  }
  const uint16_t dh = f32_to_f16(ms / 63.0f), mh = f32_to_f16(mm / 63.0f);
  const float d = f16_to_f32(dh), dmin = f16_to_f32(mh);
  int sc[8], mi[8];
  for (int j = 0; j < 8; ++j) {
    sc[j] = d > 0.0f ? std::min(63, std::max(0, nearest(scale[j] / d))) : 0;
    mi[j] = dmin > 0.0f ? std::min(63, std::max(0, nearest(minv[j] / dmin))) : 0;
  }
  std::memcpy(blk, &dh, 2);
  std::memcpy(blk + 2, &mh, 2);
  pack_scales(sc, mi, blk + 4);
  uint8_t q[256];
  for (int j = 0; j < 8; ++j) {
    const float ds = d * static_cast<float>(sc[j]), dm = dmin * static_cast<float>(mi[j]);
    for (int i = 0; i < 32; ++i) {
      int v = ds > 0.0f ? nearest((x[32 * j + i] + dm) / ds) : 0;
      q[32 * j + i] = static_cast<uint8_t>(std::min(levels, std::max(0, v)));
    }
  }
  uint8_t* qh = blk + 16;
  uint8_t* qs = blk + (q5 ? 48 : 16);
  if (q5) std::memset(qh, 0, 32);
  for (int s = 0; s < 4; ++s)
    for (int i = 0; i < 32; ++i) {
      const int lo = q[64 * s + i], hi = q[64 * s + 32 + i];
      qs[32 * s + i] = static_cast<uint8_t>((lo & 15) | ((hi & 15) << 4));
      if (q5) {
        if (lo & 16) qh[i] |= static_cast<uint8_t>(1u << (2 * s));
        if (hi & 16) qh[i] |= static_cast<uint8_t>(2u << (2 * s));
      }
    }
}

// Q6_K: 16 sub-blocks of 16 with signed 8-bit scales, codes q+32 in [0, 63].
void quantize_q6_block(const float* x, uint8_t* blk) {
  float scale[16];
  for (int j = 0; j < 16; ++j) {
    float amax = 0.0f, vmax = 0.0f;
    for (int i = 0; i < 16; ++i) {
      const float v = x[16 * j + i];
      if (std::fabs(v) > amax) {
        amax = std::fabs(v);
        vmax = v;
      }
    }
    scale[j] = amax > 0.0f ? -vmax / 32.0f : 0.0f;
  }
  float ma = 0.0f;
  for (int j = 0; j < 16; ++j) ma = std::max(ma, std::fabs(scale[j]));
  const uint16_t dh = f32_to_f16(ma / 127.0f);
  const float d = f16_to_f32(dh);
  int8_t sc[16];
  for (int j = 0; j < 16; ++j) sc[j] = static_cast<int8_t>(d > 0.0f ? std::min(127, std::max(-128, nearest(scale[j] / d))) : 0);
  uint8_t q[256];
  for (int j = 0; j < 16; ++j) {
    const float ds = d * static_cast<float>(sc[j]);
    for (int i = 0; i < 16; ++i) {
      const int v = ds != 0.0f ? nearest(x[16 * j + i] / ds) : 0;
      q[16 * j + i] = static_cast<uint8_t>(std::min(31, std::max(-32, v)) + 32);
    }
  }
  uint8_t* ql = blk;
  uint8_t* qh = blk + 128;
  for (int c = 0; c < 2; ++c)
    for (int i = 0; i < 32; ++i) {
      const int q1 = q[128 * c + i], q2 = q[128 * c + 32 + i], q3 = q[128 * c + 64 + i], q4 = q[128 * c + 96 + i];
      ql[64 * c + i] = static_cast<uint8_t>((q1 & 15) | ((q3 & 15) << 4));
      ql[64 * c + 32 + i] = static_cast<uint8_t>((q2 & 15) | ((q4 & 15) << 4));
      qh[32 * c + i] = static_cast<uint8_t>((q1 >> 4) | ((q2 >> 4) << 2) | ((q3 >> 4) << 4) | ((q4 >> 4) << 6));
    }
  std::memcpy(blk + 192, sc, 16);
  std::memcpy(blk + 208, &dh, 2);
}

uint64_t splitmix64(uint64_t x) {
  x += 0x9E3779B97F4A7C15ull;
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
  return x ^ (x >> 31);
}

uint64_t name_key(const std::string& s, uint64_t seed) {
  uint64_t h = 1469598103934665603ull ^ seed;
  for (unsigned char c : s) h = (h ^ c) * 1099511628211ull;
  return splitmix64(h);
}

template <typename F>
void parallel_rows(int64_t n, int threads, F&& fn) {
  std::atomic<int64_t> next{0};
  std::vector<std::thread> pool;
  const int t = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(threads, n)));
  for (int w = 0; w < t; ++w)
    pool.emplace_back([&] {
      for (;;) {
        const int64_t i = next.fetch_add(64);
        if (i >= n) break;
        for (int64_t r = i; r < std::min(n, i + 64); ++r) fn(r);
      }
    });
  for (auto& th : pool) th.join();
}

}  // namespace

float synth_normal(uint64_t key, uint64_t i) {
  const uint64_t a = splitmix64(key ^ (i * 0xD1B54A32D192ED03ull));
  const uint64_t b = splitmix64(a);
  const double u1 = (static_cast<double>(a >> 11) + 0.5) * (1.0 / 9007199254740992.0);
  const double u2 = static_cast<double>(b >> 11) * (1.0 / 9007199254740992.0);
  return static_cast<float>(std::sqrt(-2.0 * std::log(u1)) * std::cos(6.283185307179586 * u2));
}

uint64_t ggml_tensor_bytes(uint32_t type, const std::vector<uint64_t>& shape) {
  uint64_t n = 1;
  for (auto d : shape) n *= d;
  switch (type) {
    case 0: return n * 4;
    case 1: return n * 2;
    case 12: return n / 256 * 144;
    case 13: return n / 256 * 176;
    case 14: return n / 256 * 210;
    default: return 0;
  }
}

void quantize_q4_k(const float* x, int64_t n, uint8_t* out) {
  for (int64_t b = 0; b < n / 256; ++b) quantize_qk_affine(x + 256 * b, out + 144 * b, 15, false);
}
void quantize_q5_k(const float* x, int64_t n, uint8_t* out) {
  for (int64_t b = 0; b < n / 256; ++b) quantize_qk_affine(x + 256 * b, out + 176 * b, 31, true);
}
void quantize_q6_k(const float* x, int64_t n, uint8_t* out) {
  for (int64_t b = 0; b < n / 256; ++b) quantize_q6_block(x + 256 * b, out + 210 * b);
}

// ------------------------------------------------------------------ reader
GgufFile::~GgufFile() {
  if (map_) munmap(map_, size_);
}

std::unique_ptr<GgufFile> GgufFile::open(const std::string& path, std::string* err) {
  auto fail = [&](const std::string& m) -> std::unique_ptr<GgufFile> {
    if (err) *err = m;
    return nullptr;
  };
  const int fd = ::open(path.c_str(), O_RDONLY);
  if (fd < 0) return fail("cannot open GGUF file: " + path);
  struct stat st {};
  if (fstat(fd, &st) != 0) {
    ::close(fd);
    return fail("cannot stat GGUF file: " + path);
  }
  std::unique_ptr<GgufFile> g(new GgufFile);
  g->size_ = static_cast<uint64_t>(st.st_size);
  g->map_ = mmap(nullptr, g->size_, PROT_READ, MAP_PRIVATE, fd, 0);
  ::close(fd);
  if (g->map_ == MAP_FAILED) {
    g->map_ = nullptr;
    return fail("mmap failed: " + path);
  }
  const uint8_t* base = static_cast<const uint8_t*>(g->map_);
  Cursor c{base, base + g->size_};
  if (c.get<uint32_t>() != 0x46554747u) return fail("not a GGUF file (bad magic): " + path);
  const uint32_t version = c.get<uint32_t>();
  if (version < 2 || version > 3) return fail("unsupported GGUF version");
  const uint64_t nt = c.get<uint64_t>(), nkv = c.get<uint64_t>();
  if (!c.ok || nt > (1u << 24) || nkv > (1u << 24)) return fail("truncated or corrupt GGUF header");
  for (uint64_t i = 0; i < nkv; ++i) {
    const std::string key = c.str();
    GgufValue v;
    v.type = c.get<uint32_t>();
    if (!c.ok) return fail("truncated GGUF metadata");
    if (v.type == kString) {
      v.str = c.str();
    } else if (v.type == kArray) {
      v.is_array = true;
      v.type = c.get<uint32_t>();
      const uint64_t n = c.get<uint64_t>();
      if (!c.ok || n > g->size_) return fail("corrupt GGUF array");
      for (uint64_t j = 0; j < n && c.ok; ++j) {
        if (v.type == kString) {
          v.strs.push_back(c.str());
        } else {
          bool ok;
          v.arr.push_back(read_num(c, v.type, &ok));
          if (!ok) return fail("unsupported GGUF array element type");
        }
      }
    } else {
      bool ok;
      v.num = read_num(c, v.type, &ok);
      if (!ok) return fail("unsupported GGUF value type");
    }
    if (!c.ok) return fail("truncated GGUF metadata");
    g->meta_[key] = std::move(v);
  }
  uint64_t alignment = 32;
  if (auto* a = g->meta("general.alignment")) alignment = static_cast<uint64_t>(a->num);
  if (alignment == 0 || (alignment & (alignment - 1))) return fail("bad GGUF alignment");
  for (uint64_t i = 0; i < nt; ++i) {
    GgufTensor t;
    t.name = c.str();
    const uint32_t nd = c.get<uint32_t>();
    if (!c.ok || nd > 4) return fail("corrupt GGUF tensor info");
    for (uint32_t d = 0; d < nd; ++d) t.shape.push_back(c.get<uint64_t>());
    t.type = c.get<uint32_t>();
    t.offset = c.get<uint64_t>();
    if (!c.ok) return fail("truncated GGUF tensor directory");
    t.bytes = ggml_tensor_bytes(t.type, t.shape);
    g->tensors_.push_back(std::move(t));
  }
  uint64_t data = static_cast<uint64_t>(c.p - base);
  data = (data + alignment - 1) / alignment * alignment;
  for (size_t i = 0; i < g->tensors_.size(); ++i) {
    auto& t = g->tensors_[i];
    if (t.bytes == 0) return fail("unsupported tensor type for " + t.name);
    if (data + t.offset + t.bytes > g->size_) return fail("tensor data out of file bounds: " + t.name);
    t.data = base + data + t.offset;
    g->index_[t.name] = i;
  }
  return g;
}

const GgufTensor* GgufFile::tensor(const std::string& name) const {
  auto it = index_.find(name);
  return it == index_.end() ? nullptr : &tensors_[it->second];
}

const GgufValue* GgufFile::meta(const std::string& key) const {
  auto it = meta_.find(key);
  return it == meta_.end() ? nullptr : &it->second;
}

double GgufFile::num(const std::string& key, double fallback) const {
  const GgufValue* v = meta(key);
  return (v && !v->is_array && v->type != kString) ? v->num : fallback;
}

// ------------------------------------------------------------------ writer
namespace {

struct PendingTensor {
  std::string name;
  std::vector<uint64_t> shape;
  uint32_t type;
  int kind;  // 0 = 2-D N(0,0.02), 1 = 1 + N(0,0.02), 2 = N(0,0.02) f32, 3 = -exp(N(0,0.5))
};

void put_str(std::vector<uint8_t>& b, const std::string& s) {
  const uint64_t n = s.size();
  b.insert(b.end(), reinterpret_cast<const uint8_t*>(&n), reinterpret_cast<const uint8_t*>(&n) + 8);
  b.insert(b.end(), s.begin(), s.end());
}
template <typename T>
void put(std::vector<uint8_t>& b, T v) {
  b.insert(b.end(), reinterpret_cast<const uint8_t*>(&v), reinterpret_cast<const uint8_t*>(&v) + sizeof(T));
}

}  // namespace

bool write_synthetic_qwen35(const std::string& path, const SynthQwen35Config& cfg, std::string* err) {
  const int64_t H = cfg.hidden, I = cfg.intermediate, V = cfg.vocab;
  const int64_t hd = cfg.head_dim, nh = cfg.heads, nkv = cfg.kv_heads;
  const int64_t sh = cfg.ssm_heads, sd = cfg.ssm_head_dim;
  const int64_t key_dim = sh * sd, value_dim = sh * sd, conv_dim = 2 * key_dim + value_dim;
  const int64_t total_layers = cfg.layers + cfg.nextn_layers;
  if (H % 256 || I % 256 || value_dim % 256 || (nh * hd) % 256) {
    if (err) *err = "synthetic model dimensions must be multiples of 256";
    return false;
  }
  std::vector<PendingTensor> ts;
  auto add = [&](const std::string& n, std::vector<uint64_t> shape, uint32_t type, int kind) {
    ts.push_back({n, std::move(shape), type, kind});
  };
  auto u = [](int64_t v) { return static_cast<uint64_t>(v); };
  add("token_embd.weight", {u(H), u(V)}, cfg.embd_type, 0);
  add("output_norm.weight", {u(H)}, 0, 1);
  for (int64_t l = 0; l < total_layers; ++l) {
    const std::string p = "blk." + std::to_string(l) + ".";
    const bool mtp = l >= cfg.layers;
    const bool full = mtp || ((l + 1) % cfg.full_attention_interval) == 0;
    add(p + "attn_norm.weight", {u(H)}, 0, 1);
    add(p + "post_attention_norm.weight", {u(H)}, 0, 1);
    add(p + "ffn_gate.weight", {u(H), u(I)}, cfg.proj_type, 0);
    add(p + "ffn_up.weight", {u(H), u(I)}, cfg.proj_type, 0);
    add(p + "ffn_down.weight", {u(I), u(H)}, cfg.down_type, 0);
    if (full) {
      add(p + "attn_q.weight", {u(H), u(2 * nh * hd)}, cfg.proj_type, 0);
      add(p + "attn_k.weight", {u(H), u(nkv * hd)}, cfg.proj_type, 0);
      add(p + "attn_v.weight", {u(H), u(nkv * hd)}, cfg.proj_type, 0);
      add(p + "attn_output.weight", {u(nh * hd), u(H)}, cfg.proj_type, 0);
      add(p + "attn_q_norm.weight", {u(hd)}, 0, 1);
      add(p + "attn_k_norm.weight", {u(hd)}, 0, 1);
    } else {
      add(p + "attn_qkv.weight", {u(H), u(conv_dim)}, cfg.qkv_type ? cfg.qkv_type : cfg.proj_type, 0);
      add(p + "attn_gate.weight", {u(H), u(value_dim)}, cfg.proj_type, 0);
      add(p + "ssm_conv1d.weight", {u(cfg.conv_kernel), u(conv_dim)}, 0, 2);
      add(p + "ssm_dt.bias", {u(sh)}, 0, 2);
      add(p + "ssm_a", {u(sh)}, 0, 3);
      add(p + "ssm_beta.weight", {u(H), u(sh)}, cfg.proj_type, 0);
      add(p + "ssm_alpha.weight", {u(H), u(sh)}, cfg.proj_type, 0);
      add(p + "ssm_norm.weight", {u(sd)}, 0, 1);
      add(p + "ssm_out.weight", {u(value_dim), u(H)}, cfg.proj_type, 0);
    }
    if (mtp) {
      add(p + "nextn.eh_proj.weight", {u(2 * H), u(H)}, cfg.proj_type, 0);
      add(p + "nextn.enorm.weight", {u(H)}, 0, 1);
      add(p + "nextn.hnorm.weight", {u(H)}, 0, 1);
      add(p + "nextn.shared_head_norm.weight", {u(H)}, 0, 1);
    }
  }

  std::vector<uint8_t> hdr;
  put<uint32_t>(hdr, 0x46554747u);
  put<uint32_t>(hdr, 3);
  put<uint64_t>(hdr, ts.size());
  std::vector<uint8_t> kv;
  uint64_t nkv_entries = 0;
  auto kv_str = [&](const std::string& k, const std::string& v) {
    put_str(kv, k);
    put<uint32_t>(kv, kString);
    put_str(kv, v);
    ++nkv_entries;
  };
  auto kv_u32 = [&](const std::string& k, uint32_t v) {
    put_str(kv, k);
    put<uint32_t>(kv, kU32);
    put<uint32_t>(kv, v);
    ++nkv_entries;
  };
  auto kv_f32 = [&](const std::string& k, float v) {
    put_str(kv, k);
    put<uint32_t>(kv, kF32);
    put<float>(kv, v);
    ++nkv_entries;
  };
  const std::string a = "qwen35.";
  kv_str("general.architecture", "qwen35");
  kv_str("general.name", "kib-synthetic-qwen35");
  kv_u32("general.alignment", 32);
  kv_u32(a + "context_length", static_cast<uint32_t>(cfg.context_length));
  kv_u32(a + "embedding_length", static_cast<uint32_t>(H));
  kv_u32(a + "feed_forward_length", static_cast<uint32_t>(I));
  kv_u32(a + "vocab_size", static_cast<uint32_t>(V));
  kv_u32(a + "block_count", static_cast<uint32_t>(total_layers));
  kv_u32(a + "nextn_predict_layers", static_cast<uint32_t>(cfg.nextn_layers));
  kv_u32(a + "attention.head_count", static_cast<uint32_t>(nh));
  kv_u32(a + "attention.head_count_kv", static_cast<uint32_t>(nkv));
  kv_u32(a + "attention.key_length", static_cast<uint32_t>(hd));
  kv_u32(a + "attention.value_length", static_cast<uint32_t>(hd));
  kv_f32(a + "attention.layer_norm_rms_epsilon", static_cast<float>(cfg.rms_eps));
  kv_f32(a + "rope.freq_base", static_cast<float>(cfg.rope_theta));
  kv_u32(a + "full_attention_interval", static_cast<uint32_t>(cfg.full_attention_interval));
  kv_u32(a + "ssm.conv_kernel", static_cast<uint32_t>(cfg.conv_kernel));
  kv_u32(a + "ssm.state_size", static_cast<uint32_t>(sd));
  kv_u32(a + "ssm.group_count", static_cast<uint32_t>(sh));
  kv_u32(a + "ssm.time_step_rank", static_cast<uint32_t>(sh));
  kv_u32(a + "ssm.inner_size", static_cast<uint32_t>(value_dim));
  {
    put_str(kv, a + "rope.dimension_sections");
    put<uint32_t>(kv, kArray);
    put<uint32_t>(kv, kI32);
    put<uint64_t>(kv, 4);
    for (int32_t s : {11, 11, 10, 0}) put<int32_t>(kv, s);
    ++nkv_entries;
  }
  if (cfg.eos_token_id >= 0) kv_u32("tokenizer.ggml.eos_token_id", static_cast<uint32_t>(cfg.eos_token_id));
  put<uint64_t>(hdr, nkv_entries);
  hdr.insert(hdr.end(), kv.begin(), kv.end());
  uint64_t off = 0;
  std::vector<uint64_t> offsets;
  for (auto& t : ts) {
    put_str(hdr, t.name);
    put<uint32_t>(hdr, static_cast<uint32_t>(t.shape.size()));
    for (auto d : t.shape) put<uint64_t>(hdr, d);
    put<uint32_t>(hdr, t.type);
    put<uint64_t>(hdr, off);
    offsets.push_back(off);
    off += (ggml_tensor_bytes(t.type, t.shape) + 31) / 32 * 32;
  }
  while (hdr.size() % 32) hdr.push_back(0);

  FILE* f = std::fopen(path.c_str(), "wb");
  if (!f) {
    if (err) *err = "cannot create " + path;
    return false;
  }
  bool ok = std::fwrite(hdr.data(), 1, hdr.size(), f) == hdr.size();
  for (size_t i = 0; i < ts.size() && ok; ++i) {
    const auto& t = ts[i];
    const uint64_t bytes = ggml_tensor_bytes(t.type, t.shape);
    const uint64_t padded = (bytes + 31) / 32 * 32;
    std::vector<uint8_t> buf(padded, 0);
    const uint64_t key = name_key(t.name, cfg.seed);
    if (t.type == 0) {
      uint64_t n = 1;
      for (auto d : t.shape) n *= d;
      float* v = reinterpret_cast<float*>(buf.data());
      for (uint64_t j = 0; j < n; ++j) {
        const float z = synth_normal(key, j);
        v[j] = t.kind == 1 ? 1.0f + 0.02f * z : (t.kind == 3 ? -std::exp(0.5f * z) : 0.02f * z);
      }
    } else {
      const int64_t cols = static_cast<int64_t>(t.shape[0]), rows = static_cast<int64_t>(t.shape[1]);
      const uint64_t row_bytes = ggml_tensor_bytes(t.type, {t.shape[0]});
      parallel_rows(rows, cfg.threads, [&](int64_t r) {
        std::vector<float> x(static_cast<size_t>(cols));
        for (int64_t cidx = 0; cidx < cols; ++cidx)
          x[cidx] = 0.02f * synth_normal(key, static_cast<uint64_t>(r * cols + cidx));
        uint8_t* dst = buf.data() + r * row_bytes;
        if (t.type == 12) quantize_q4_k(x.data(), cols, dst);
        else if (t.type == 13) quantize_q5_k(x.data(), cols, dst);
        else quantize_q6_k(x.data(), cols, dst);
      });
    }
    ok = std::fwrite(buf.data(), 1, buf.size(), f) == buf.size();
  }
  ok = (std::fclose(f) == 0) && ok;
  if (!ok && err) *err = "write failed: " + path;
  return ok;
}

}  // namespace kib
