// kib_oracle.cpp -- CPU restatement of kraken-infer's Qwen3.5 decode / MTP-verify
// hot path.
//
// TEST INFRASTRUCTURE ONLY.  This file is the parity checker for the CUDA
// backend in kraken-infer_b200/.  Only tests/, __graft_entry__.smoke() and the
// cpu_baseline / --impl reference legs of bench.py may load the library built
// from it; the product path never does.
//
// Every function restates one reference kernel or runtime routine and cites the
// reference file:line it follows (paths inside the kraken-infer project):
//   src/backends/mps/mps_backend.mm        -- the Metal kernels (MSL string literals)
//   src/runtime/qwen35_runtime.cpp         -- layer drivers, LM head, MTP loop
//
// Parity pins: the K-quant block decode, the norms, conv, GDN, gate/beta,
// MRoPE, argmax and the attention known-answer vectors of tests/smoke_test.cpp
// are checked in tests/test_oracle_golden.py; the K-quant decode is also
// compared byte-for-byte with the reference's own host decoder compiled from
// its sources (oracle/_ref, see oracle/Makefile).
//
// Numerics follow the reference's matmul buckets (mps_backend.mm:6411-6452):
//   tokens <= 3  : fp32 row reduction (q*_k_matmul, 1268-1446)
//   tokens 4..8  : weights rounded to fp16 per weight, fp32 x (mul_mv_ext, 887-1086)
//   tokens  > 8  : weights and x rounded to fp16, fp32 accumulate (mul_mm_simd, 1088-1266)

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fcntl.h>
#include <limits>
#include <map>
#include <memory>
#include <string>
#include <sys/mman.h>
#include <sys/stat.h>
#include <thread>
#include <unistd.h>
#include <vector>

namespace {

// ---------------------------------------------------------------- fp16 helpers

// f16_to_float_cpu (qwen35_runtime.cpp:934-952): exact IEEE half -> float.
float f16_to_f32(const uint8_t* p) {
  const uint16_t v = static_cast<uint16_t>(p[0] | (p[1] << 8));
  const uint32_t sign = (v >> 15) & 1u, exponent = (v >> 10) & 31u, mantissa = v & 1023u;
  float r;
  if (exponent == 0u) {
    r = std::ldexp(static_cast<float>(mantissa), -24);
  } else if (exponent == 31u) {
    r = mantissa == 0u ? std::numeric_limits<float>::infinity()
                       : std::numeric_limits<float>::quiet_NaN();
  } else {
    r = std::ldexp(1.0f + static_cast<float>(mantissa) / 1024.0f,
                   static_cast<int>(exponent) - 15);
  }
  return sign ? -r : r;
}

float f16_bits_to_f32(uint16_t v) {
  uint8_t b[2] = {static_cast<uint8_t>(v & 0xFF), static_cast<uint8_t>(v >> 8)};
  return f16_to_f32(b);
}

// float -> IEEE half, round to nearest even (the `static_cast<half>` of the
// Metal kernels: mps_backend.mm:866-885, 1148, and the f32->f16 KV write 2655-2666).
uint16_t f32_to_f16_bits(float f) {
  uint32_t x;
  std::memcpy(&x, &f, 4);
  const uint32_t sign = (x >> 16) & 0x8000u;
  const uint32_t absx = x & 0x7FFFFFFFu;
  if (absx >= 0x7F800000u) {  // inf / nan
    return static_cast<uint16_t>(sign | 0x7C00u | (absx > 0x7F800000u ? 0x200u : 0u));
  }
  if (absx >= 0x477FF000u) {  // rounds to >= 65520 -> inf
    return static_cast<uint16_t>(sign | 0x7C00u);
  }
  if (absx < 0x38800000u) {  // below the smallest normal half: subnormal / zero
    if (absx < 0x33000000u) return static_cast<uint16_t>(sign);  // < 2^-25 -> 0
    const uint32_t e = absx >> 23;
    const uint32_t m = (absx & 0x7FFFFFu) | 0x800000u;
    const uint32_t shift = 126u - e;  // value = m * 2^(e-150); half ulp = 2^-24
    uint32_t q = m >> (shift - 0);
    // value / 2^-24 = m * 2^(e-126) = m >> (126-e)
    const uint32_t rem = m & ((1u << shift) - 1u);
    const uint32_t halfway = 1u << (shift - 1u);
    if (rem > halfway || (rem == halfway && (q & 1u))) ++q;
    return static_cast<uint16_t>(sign | q);
  }
  uint32_t e = (absx >> 23) - 112u;  // rebias 127 -> 15
  uint32_t m = absx & 0x7FFFFFu;
  uint32_t h = (e << 10) | (m >> 13);
  const uint32_t rem = m & 0x1FFFu;
  if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) ++h;
  return static_cast<uint16_t>(sign | h);
}

float round_f16(float f) { return f16_bits_to_f32(f32_to_f16_bits(f)); }

// --------------------------------------------------------------- K-quant decode

constexpr int kTypeF32 = 0;
constexpr int kTypeQ4K = 12;
constexpr int kTypeQ5K = 13;
constexpr int kTypeQ6K = 14;

int block_bytes(int type) {
  switch (type) {
    case kTypeQ4K: return 144;
    case kTypeQ5K: return 176;
    case kTypeQ6K: return 210;
    default: return 0;
  }
}

// q4_k_scale_min_cpu (qwen35_runtime.cpp:954-968) / q4_k_scale_min (mps_backend.mm:282-293).
void q4k_scale_min(uint32_t j, const uint8_t* s, uint32_t* sc, uint32_t* m) {
  if (j < 4u) {
    *sc = s[j] & 63u;
    *m = s[j + 4u] & 63u;
  } else {
    *sc = (s[j + 4u] & 0xFu) | ((s[j - 4u] >> 6u) << 4u);
    *m = (s[j + 4u] >> 4u) | ((s[j] >> 6u) << 4u);
  }
}

// Dequantize one 256-weight super-block to fp32, exactly as the reference's
// host decoder dequantize_quantized_transposed_f32 (qwen35_runtime.cpp:1136-1233)
// and the device q*_k_get_row(s) kernels (mps_backend.mm:1448-1549, 1693-1824).
void dequant_block(int type, const uint8_t* b, float* out) {
  if (type == kTypeQ4K || type == kTypeQ5K) {
    const float d = f16_to_f32(b), dmin = f16_to_f32(b + 2);
    const uint8_t* scales = b + 4;
    const uint8_t* qh = b + 16;
    const uint8_t* qs = b + (type == kTypeQ4K ? 16 : 48);
    for (uint32_t s = 0; s < 4u; ++s) {
      uint32_t sc1, m1i, sc2, m2i;
      q4k_scale_min(2u * s, scales, &sc1, &m1i);
      q4k_scale_min(2u * s + 1u, scales, &sc2, &m2i);
      const float d1 = d * static_cast<float>(sc1), m1 = dmin * static_cast<float>(m1i);
      const float d2 = d * static_cast<float>(sc2), m2 = dmin * static_cast<float>(m2i);
      const uint8_t* q = qs + 32u * s;
      for (uint32_t i = 0; i < 32u; ++i) {
        uint32_t lo = q[i] & 0xFu, hi = q[i] >> 4u;
        if (type == kTypeQ5K) {
          lo += (qh[i] & (1u << (2u * s))) ? 16u : 0u;
          hi += (qh[i] & (2u << (2u * s))) ? 16u : 0u;
        }
        out[64u * s + i] = d1 * static_cast<float>(lo) - m1;
        out[64u * s + 32u + i] = d2 * static_cast<float>(hi) - m2;
      }
    }
  } else if (type == kTypeQ6K) {
    const float d = f16_to_f32(b + 208);
    for (uint32_t c = 0; c < 2u; ++c) {
      const uint8_t* ql = b + 64u * c;
      const uint8_t* qh = b + 128u + 32u * c;
      const int8_t* sc = reinterpret_cast<const int8_t*>(b + 192u + 8u * c);
      for (uint32_t i = 0; i < 32u; ++i) {
        const uint32_t si = i / 16u;
        const int q1 = static_cast<int>((ql[i] & 0xFu) | (((qh[i] >> 0u) & 3u) << 4u)) - 32;
        const int q2 = static_cast<int>((ql[i + 32u] & 0xFu) | (((qh[i] >> 2u) & 3u) << 4u)) - 32;
        const int q3 = static_cast<int>((ql[i] >> 4u) | (((qh[i] >> 4u) & 3u) << 4u)) - 32;
        const int q4 = static_cast<int>((ql[i + 32u] >> 4u) | (((qh[i] >> 6u) & 3u) << 4u)) - 32;
        out[128u * c + i] = d * static_cast<float>(sc[si + 0]) * static_cast<float>(q1);
        out[128u * c + 32u + i] = d * static_cast<float>(sc[si + 2]) * static_cast<float>(q2);
        out[128u * c + 64u + i] = d * static_cast<float>(sc[si + 4]) * static_cast<float>(q3);
        out[128u * c + 96u + i] = d * static_cast<float>(sc[si + 6]) * static_cast<float>(q4);
      }
    }
  }
}

// Per-weight fp16 dequant used by the mul_mv_ext / mul_mm_simd paths
// (dequantize_q{4,5,6}_k_mm, mps_backend.mm:780-864): the fp32 value
// dl*q - ml is rounded to half.  For Q4_K/Q5_K dl*q - ml equals the fp32 value
// of dequant_block (the /16, /256 rescalings are exact powers of two); Q6_K
// computes dl0*q' - ml with q' the unsigned 6-bit code, which differs from
// d*sc*(q'-32) by one fp32 rounding.
void dequant_block_f16(int type, const uint8_t* b, float* out) {
  if (type == kTypeQ4K || type == kTypeQ5K) {
    dequant_block(type, b, out);
    for (int i = 0; i < 256; ++i) out[i] = round_f16(out[i]);
    return;
  }
  const float d = f16_to_f32(b + 208);
  for (uint32_t c = 0; c < 2u; ++c) {
    const uint8_t* ql = b + 64u * c;
    const uint8_t* qh = b + 128u + 32u * c;
    const int8_t* sc = reinterpret_cast<const int8_t*>(b + 192u + 8u * c);
    for (uint32_t i = 0; i < 32u; ++i) {
      const uint32_t si = i / 16u;
      const uint32_t u[4] = {(ql[i] & 0xFu) | (((qh[i] >> 0u) & 3u) << 4u),
                             (ql[i + 32u] & 0xFu) | (((qh[i] >> 2u) & 3u) << 4u),
                             (ql[i] >> 4u) | (((qh[i] >> 4u) & 3u) << 4u),
                             (ql[i + 32u] >> 4u) | (((qh[i] >> 6u) & 3u) << 4u)};
      for (uint32_t k = 0; k < 4u; ++k) {
        const float dl0 = d * static_cast<float>(sc[si + 2u * k]);
        const float ml = dl0 * 32.0f;
        out[128u * c + 32u * k + i] = round_f16(dl0 * static_cast<float>(u[k]) - ml);
      }
    }
  }
}

// ------------------------------------------------------------- thread helper

template <typename F>
void pfor(int64_t n, int threads, F&& fn) {
  if (threads <= 1 || n < 2) {
    for (int64_t i = 0; i < n; ++i) fn(i);
    return;
  }
  const int t = static_cast<int>(std::min<int64_t>(threads, n));
  std::atomic<int64_t> next{0};
  std::vector<std::thread> pool;
  pool.reserve(t);
  for (int w = 0; w < t; ++w) {
    pool.emplace_back([&] {
      for (;;) {
        const int64_t i = next.fetch_add(1);
        if (i >= n) break;
        fn(i);
      }
    });
  }
  for (auto& th : pool) th.join();
}

int g_threads = 1;
// Rows the matmul numerics bucket is chosen for, when larger than the actual
// row count (0: the actual count).  A batched decode step multiplies the
// tokens of `slots` sequences in one matmul, so each sequence's rows get the
// bucket of the whole batch; restating one sequence of such a batch sets this.
int64_t g_bucket_rows = 0;

// ------------------------------------------------------------- quant matmul

// Y[t][r] = W[r,:] . X[t,:]; the three reference numerics buckets.
void quant_matmul(int type, const uint8_t* w, int64_t rows, int64_t cols, const float* x,
                  int64_t tokens, float* y) {
  const int64_t bpr = cols / 256;
  const int bb = block_bytes(type);
  const int64_t bucket = tokens > g_bucket_rows ? tokens : g_bucket_rows;
  if (bucket <= 3) {
    // q*_k_matmul (mps_backend.mm:1268-1446): lane b sums block b in order, the
    // 256-wide threadgroup tree-reduces the per-block partials.
    pfor(rows, g_threads, [&](int64_t r) {
      std::vector<float> deq(256);
      std::vector<float> partials(256);
      for (int64_t t = 0; t < tokens; ++t) {
        std::fill(partials.begin(), partials.end(), 0.0f);
        for (int64_t b = 0; b < bpr; ++b) {
          const uint8_t* blk = w + (r * bpr + b) * bb;
          const float* xin = x + t * cols + b * 256;
          float sum = 0.0f;
          if (type == kTypeQ6K) {
            // q6_k_matmul order: for chunk, i: q1,q2,q3,q4 (mps_backend.mm:1405-1434)
            dequant_block(type, blk, deq.data());
            for (int c = 0; c < 2; ++c)
              for (int i = 0; i < 32; ++i)
                for (int k = 0; k < 4; ++k) sum += deq[128 * c + 32 * k + i] * xin[128 * c + 32 * k + i];
          } else {
            // q4/q5: for segment, i: low then high (mps_backend.mm:1296-1306)
            dequant_block(type, blk, deq.data());
            for (int s = 0; s < 4; ++s)
              for (int i = 0; i < 32; ++i) {
                sum += deq[64 * s + i] * xin[64 * s + i];
                sum += deq[64 * s + 32 + i] * xin[64 * s + 32 + i];
              }
          }
          partials[static_cast<size_t>(b % 256)] += sum;
        }
        for (int stride = 128; stride > 0; stride >>= 1)
          for (int l = 0; l < stride; ++l) partials[l] += partials[l + stride];
        y[t * rows + r] = partials[0];
      }
    });
    return;
  }
  const bool round_x = bucket > 8;
  std::vector<float> xr;
  const float* xs = x;
  if (round_x) {
    xr.assign(x, x + tokens * cols);
    for (auto& v : xr) v = round_f16(v);
    xs = xr.data();
  }
  pfor(rows, g_threads, [&](int64_t r) {
    std::vector<float> wrow(static_cast<size_t>(cols));
    for (int64_t b = 0; b < bpr; ++b) dequant_block_f16(type, w + (r * bpr + b) * bb, &wrow[b * 256]);
    for (int64_t t = 0; t < tokens; ++t) {
      const float* xin = xs + t * cols;
      float sum;
      if (!round_x) {
        // mul_mv_ext (mps_backend.mm:887-960): 8 lanes per row, lane tx takes
        // 16-weight chunks tx, tx+8, ...; shuffle-down reduction 4,2,1.
        float part[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        for (int64_t ch = 0; ch * 16 < cols; ++ch) {
          float s = 0.0f;
          for (int q = 0; q < 4; ++q) {
            float d = 0.0f;
            for (int e = 0; e < 4; ++e) d += wrow[ch * 16 + q * 4 + e] * xin[ch * 16 + q * 4 + e];
            s += d;
          }
          part[ch % 8] += s;
        }
        for (int off = 4; off > 0; off >>= 1)
          for (int l = 0; l < off; ++l) part[l] += part[l + off];
        sum = part[0];
      } else {
        // mul_mm_simd (mps_backend.mm:1088-1230): fp16 x fp16 products, fp32 accumulate.
        sum = 0.0f;
        for (int64_t c = 0; c < cols; ++c) sum += wrow[c] * xin[c];
      }
      y[t * rows + r] = sum;
    }
  });
}

// ------------------------------------------------------------- small kernels

// rms_norm_f32_f32_batched (mps_backend.mm:1891-1921): 256-lane strided partial
// sums, tree reduction, scale = rsqrt(mean + eps).
float rms_scale(const float* x, int64_t n, float eps) {
  float partials[256];
  for (int l = 0; l < 256; ++l) {
    float s = 0.0f;
    for (int64_t i = l; i < n; i += 256) s += x[i] * x[i];
    partials[l] = s;
  }
  for (int stride = 128; stride > 0; stride >>= 1)
    for (int l = 0; l < stride; ++l) partials[l] += partials[l + stride];
  return 1.0f / std::sqrt(partials[0] / static_cast<float>(n) + eps);
}

void rms_norm(const float* x, const float* w, int64_t tokens, int64_t n, float eps, float* y) {
  for (int64_t t = 0; t < tokens; ++t) {
    const float s = rms_scale(x + t * n, n, eps);
    for (int64_t i = 0; i < n; ++i) y[t * n + i] = x[t * n + i] * s * w[i];
  }
}

// qk_norm_f32_f32_batched (mps_backend.mm:1991-2024): per-head in-place RMSNorm.
void qk_norm(float* v, const float* w, int64_t tokens, int64_t heads, int64_t d, float eps) {
  for (int64_t t = 0; t < tokens; ++t)
    for (int64_t h = 0; h < heads; ++h) {
      float* p = v + (t * heads + h) * d;
      const float s = rms_scale(p, d, eps);
      for (int64_t i = 0; i < d; ++i) p[i] *= s * w[i];
    }
}

// l2 scale 1/max(sqrt(sum x^2), eps) (split_qkv_l2_norm_f32_qwen35, mps_backend.mm:2097-2153).
float l2_scale(const float* x, int64_t n, float eps) {
  float partials[256];
  for (int l = 0; l < 256; ++l) {
    float s = 0.0f;
    for (int64_t i = l; i < n; i += 256) s += x[i] * x[i];
    partials[l] = s;
  }
  for (int stride = 128; stride > 0; stride >>= 1)
    for (int l = 0; l < stride; ++l) partials[l] += partials[l + stride];
  return 1.0f / std::max(std::sqrt(partials[0]), eps);
}

float silu(float v) { return v / (1.0f + std::exp(-v)); }
float sigmoid(float v) { return 1.0f / (1.0f + std::exp(-v)); }
float softplus20(float v) { return v > 20.0f ? v : std::log(1.0f + std::exp(v)); }

// MRoPE (mrope_f32_in_place, mps_backend.mm:2482-2527): NeoX pairs (p, p+n_dims/2)
// for p < n_dims/2, section chosen by p % sum(sections).
void mrope(float* v, const int32_t* positions, int64_t tokens, int64_t heads, int64_t head_dim,
           int64_t n_dims, const int64_t sec[4], float theta) {
  const int64_t half = n_dims / 2;
  const int64_t total_sec = sec[0] + sec[1] + sec[2] + sec[3];
  if (total_sec == 0) return;
  for (int64_t t = 0; t < tokens; ++t)
    for (int64_t h = 0; h < heads; ++h)
      for (int64_t p = 0; p < half; ++p) {
        const int64_t sector = p % total_sec;
        int idx = 3;
        if (sector < sec[0]) idx = 0;
        else if (sector < sec[0] + sec[1]) idx = 1;
        else if (sector < sec[0] + sec[1] + sec[2]) idx = 2;
        const float pos = static_cast<float>(positions[t + tokens * idx]);
        const float exponent = static_cast<float>(2 * p) / static_cast<float>(n_dims);
        const float freq = 1.0f / std::pow(theta, exponent);
        const float angle = pos * freq;
        const float c = std::cos(angle), s = std::sin(angle);
        float* base = v + (t * heads + h) * head_dim;
        const float x0 = base[p], x1 = base[half + p];
        base[p] = x0 * c - x1 * s;
        base[half + p] = x1 * c + x0 * s;
      }
}

// gated_delta_net_f32_batched_qwen35 (mps_backend.mm:2307-2374): sequential over
// tokens; per state row: decay, sk = S.k, delta = (v - sk) * beta, S += k delta,
// y = S.q * scale.  State layout [head][row v][col k].
void gdn(const float* q, const float* k, const float* v, const float* g, const float* beta,
         float* state, int64_t tokens, int64_t key_heads, int64_t value_heads, int64_t d,
         float* out) {
  const float scale = 1.0f / std::sqrt(static_cast<float>(d));
  for (int64_t h = 0; h < value_heads; ++h) {
    const int64_t kh = h % key_heads;
    for (int64_t row = 0; row < d; ++row) {
      float* s = state + (h * d + row) * d;
      for (int64_t t = 0; t < tokens; ++t) {
        const float* kk = k + (t * key_heads + kh) * d;
        const float* qq = q + (t * key_heads + kh) * d;
        const float ge = std::exp(g[t * value_heads + h]);
        float sk = 0.0f;
        for (int64_t c = 0; c < d; ++c) {
          s[c] *= ge;
          sk += s[c] * kk[c];
        }
        const float delta = (v[(t * value_heads + h) * d + row] - sk) * beta[t * value_heads + h];
        float y = 0.0f;
        for (int64_t c = 0; c < d; ++c) {
          s[c] += kk[c] * delta;
          y += s[c] * qq[c];
        }
        out[(t * value_heads + h) * d + row] = y * scale;
      }
    }
  }
}

// attention_f32_batched_f16_kv (mps_backend.mm:2943-3008): per (query, head)
// sequential online softmax over keys <= query position, f16 K/V.
// flash256 (3398-3643, T >= 64) additionally rounds Q to half.
void attention_f16kv(const float* query, const uint16_t* kcache, const uint16_t* vcache,
                     int64_t start, int64_t tokens, int64_t heads, int64_t kv_heads,
                     int64_t head_dim, bool round_q, float* out) {
  const int64_t group = heads / kv_heads;
  const int64_t kv_dim = kv_heads * head_dim;
  const float scale = 1.0f / std::sqrt(static_cast<float>(head_dim));
  pfor(tokens * heads, g_threads, [&](int64_t idx) {
    const int64_t t = idx / heads, h = idx % heads;
    const int64_t kvh = h / group;
    std::vector<float> qv(head_dim), acc(head_dim, 0.0f);
    for (int64_t i = 0; i < head_dim; ++i) {
      const float qq = query[(t * heads + h) * head_dim + i];
      qv[i] = round_q ? round_f16(qq) : qq;
    }
    float mx = -std::numeric_limits<float>::infinity(), den = 0.0f;
    const int64_t qpos = start + t;
    for (int64_t key = 0; key <= qpos; ++key) {
      const uint16_t* kp = kcache + key * kv_dim + kvh * head_dim;
      const uint16_t* vp = vcache + key * kv_dim + kvh * head_dim;
      float sc = 0.0f;
      for (int64_t i = 0; i < head_dim; ++i) sc += qv[i] * f16_bits_to_f32(kp[i]);
      sc *= scale;
      const float nm = std::max(mx, sc);
      const float ps = std::exp(mx - nm);
      const float wgt = std::exp(sc - nm);
      den = den * ps + wgt;
      for (int64_t i = 0; i < head_dim; ++i) acc[i] = acc[i] * ps + wgt * f16_bits_to_f32(vp[i]);
      mx = nm;
    }
    const float inv = den == 0.0f ? 0.0f : 1.0f / den;
    for (int64_t i = 0; i < head_dim; ++i) out[(t * heads + h) * head_dim + i] = acc[i] * inv;
  });
}

// argmax_f32_i32 (mps_backend.mm:2681-2720): ties -> lowest index.
int64_t argmax(const float* v, int64_t n) {
  int64_t best = n;
  float bv = -std::numeric_limits<float>::infinity();
  for (int64_t i = 0; i < n; ++i)
    if (v[i] > bv || (v[i] == bv && i < best)) {
      bv = v[i];
      best = i;
    }
  return best;
}

// ------------------------------------------------------------------ GGUF read

struct Tensor {
  std::vector<uint64_t> shape;
  uint32_t type = 0;
  const uint8_t* data = nullptr;
};

struct Gguf {
  void* map = nullptr;
  size_t size = 0;
  std::map<std::string, Tensor> tensors;
  std::map<std::string, double> nums;
  std::map<std::string, std::vector<int64_t>> arrays;
  std::map<std::string, std::string> strs;
  ~Gguf() {
    if (map) munmap(map, size);
  }
};

struct Reader {
  const uint8_t* p;
  const uint8_t* end;
  bool ok = true;
  template <typename T>
  T get() {
    T v{};
    if (p + sizeof(T) > end) {
      ok = false;
      return v;
    }
    std::memcpy(&v, p, sizeof(T));
    p += sizeof(T);
    return v;
  }
  std::string str() {
    const uint64_t n = get<uint64_t>();
    if (!ok || p + n > end) {
      ok = false;
      return {};
    }
    std::string s(reinterpret_cast<const char*>(p), n);
    p += n;
    return s;
  }
};

double read_scalar(Reader& r, uint32_t t, bool* is_num) {
  *is_num = true;
  switch (t) {
    case 0: return r.get<uint8_t>();
    case 1: return r.get<int8_t>();
    case 2: return r.get<uint16_t>();
    case 3: return r.get<int16_t>();
    case 4: return r.get<uint32_t>();
    case 5: return r.get<int32_t>();
    case 6: return r.get<float>();
    case 7: return r.get<uint8_t>();
    case 10: return static_cast<double>(r.get<uint64_t>());
    case 11: return static_cast<double>(r.get<int64_t>());
    case 12: return r.get<double>();
    default: *is_num = false; return 0;
  }
}

std::unique_ptr<Gguf> open_gguf(const char* path) {
  auto g = std::make_unique<Gguf>();
  const int fd = ::open(path, O_RDONLY);
  if (fd < 0) return nullptr;
  struct stat st{};
  fstat(fd, &st);
  g->size = static_cast<size_t>(st.st_size);
  g->map = mmap(nullptr, g->size, PROT_READ, MAP_PRIVATE, fd, 0);
  ::close(fd);
  if (g->map == MAP_FAILED) {
    g->map = nullptr;
    return nullptr;
  }
  Reader r{static_cast<const uint8_t*>(g->map), static_cast<const uint8_t*>(g->map) + g->size};
  if (r.get<uint32_t>() != 0x46554747u) return nullptr;  // "GGUF"
  r.get<uint32_t>();
  const uint64_t nt = r.get<uint64_t>(), nkv = r.get<uint64_t>();
  uint64_t alignment = 32;
  for (uint64_t i = 0; i < nkv && r.ok; ++i) {
    const std::string key = r.str();
    const uint32_t t = r.get<uint32_t>();
    if (t == 8) {
      g->strs[key] = r.str();
    } else if (t == 9) {
      const uint32_t et = r.get<uint32_t>();
      const uint64_t n = r.get<uint64_t>();
      std::vector<int64_t> vals;
      for (uint64_t j = 0; j < n && r.ok; ++j) {
        if (et == 8) {
          r.str();
        } else {
          bool num;
          vals.push_back(static_cast<int64_t>(read_scalar(r, et, &num)));
        }
      }
      g->arrays[key] = vals;
    } else {
      bool num;
      g->nums[key] = read_scalar(r, t, &num);
    }
  }
  if (g->nums.count("general.alignment")) alignment = static_cast<uint64_t>(g->nums["general.alignment"]);
  struct Info {
    std::string name;
    std::vector<uint64_t> shape;
    uint32_t type;
    uint64_t off;
  };
  std::vector<Info> infos;
  for (uint64_t i = 0; i < nt && r.ok; ++i) {
    Info inf;
    inf.name = r.str();
    const uint32_t nd = r.get<uint32_t>();
    for (uint32_t d = 0; d < nd; ++d) inf.shape.push_back(r.get<uint64_t>());
    inf.type = r.get<uint32_t>();
    inf.off = r.get<uint64_t>();
    infos.push_back(inf);
  }
  if (!r.ok) return nullptr;
  uint64_t data_off = static_cast<uint64_t>(r.p - static_cast<const uint8_t*>(g->map));
  data_off = (data_off + alignment - 1) / alignment * alignment;
  for (auto& inf : infos) {
    Tensor t;
    t.shape = inf.shape;
    t.type = inf.type;
    t.data = static_cast<const uint8_t*>(g->map) + data_off + inf.off;
    g->tensors[inf.name] = t;
  }
  return g;
}

// ------------------------------------------------------------------ the model

struct Model {
  std::unique_ptr<Gguf> g;
  int64_t hidden = 0, layers_main = 0, layers_total = 0, inter = 0, vocab = 0;
  int64_t heads = 0, kv_heads = 0, head_dim = 0;
  int64_t lk_heads = 0, lv_heads = 0, lhead = 0, conv_k = 0, conv_ch = 0;
  float eps = 1e-6f, theta = 1e7f;
  int64_t sections[4] = {11, 11, 10, 0};
  int64_t eos = -1;
  std::vector<int> kinds;  // 0 = linear, 1 = full attention
  std::vector<int64_t> kind_index;
  int64_t n_full = 0, n_lin = 0, capacity = 0;
  bool has_mtp = false;
  // caches
  std::vector<uint16_t> kcache, vcache, mtp_k, mtp_v;
  std::vector<float> rstate, sstate, pending_h;

  const Tensor& t(const std::string& name) const {
    auto it = g->tensors.find(name);
    if (it == g->tensors.end()) {
      std::fprintf(stderr, "oracle: missing tensor %s\n", name.c_str());
      std::abort();
    }
    return it->second;
  }
  const float* f(const std::string& name) const { return reinterpret_cast<const float*>(t(name).data); }
  std::string L(int64_t l, const char* s) const { return "blk." + std::to_string(l) + "." + s; }
  int64_t kv_dim() const { return kv_heads * head_dim; }

  // run_qwen35_quant_matmul (qwen35_runtime.cpp:1972-2048)
  void matmul(const std::string& name, const float* x, int64_t tokens, float* y) const {
    const Tensor& w = t(name);
    quant_matmul(static_cast<int>(w.type), w.data, static_cast<int64_t>(w.shape[1]),
                 static_cast<int64_t>(w.shape[0]), x, tokens, y);
  }
  int64_t rows(const std::string& name) const { return static_cast<int64_t>(t(name).shape[1]); }

  // q6_k_get_rows embedding (run_qwen35_token_embeddings, qwen35_runtime.cpp:1644-1654;
  // out-of-range ids produce zeros, mps_backend.mm:1772-1824).
  void embed(const int32_t* ids, int64_t tokens, float* out) const {
    const Tensor& e = t("token_embd.weight");
    const int64_t bpr = hidden / 256;
    const int bb = block_bytes(static_cast<int>(e.type));
    for (int64_t i = 0; i < tokens; ++i) {
      if (ids[i] < 0 || ids[i] >= vocab) {
        std::fill(out + i * hidden, out + (i + 1) * hidden, 0.0f);
        continue;
      }
      for (int64_t b = 0; b < bpr; ++b)
        dequant_block(static_cast<int>(e.type), e.data + (ids[i] * bpr + b) * bb, out + i * hidden + b * 256);
    }
  }

  // run_qwen35_linear_layer_chunk (qwen35_runtime.cpp:2634-3144)
  void linear_layer(int64_t l, int64_t li, const float* hidden_in, int64_t T, float* out) {
    const int64_t H = hidden, C = conv_ch, dk = lhead;
    const int64_t key_dim = lk_heads * dk, value_dim = lv_heads * dk;
    std::vector<float> normed(T * H), qkv(T * C);
    rms_norm(hidden_in, f(L(l, "attn_norm.weight")), T, H, eps, normed.data());
    matmul(L(l, "attn_qkv.weight"), normed.data(), T, qkv.data());
    // build_ssm_conv_state_f32 + ssm_conv_f32 + silu (mps_backend.mm:2376-2457, 2610-2618)
    float* R = rstate.data() + li * C * (conv_k - 1);
    const float* cw = f(L(l, "ssm_conv1d.weight"));
    std::vector<float> conv(T * C);
    for (int64_t c = 0; c < C; ++c) {
      std::vector<float> in(conv_k - 1 + T);
      for (int64_t p = 0; p < conv_k - 1; ++p) in[p] = R[c * (conv_k - 1) + p];
      for (int64_t tt = 0; tt < T; ++tt) in[conv_k - 1 + tt] = qkv[tt * C + c];
      for (int64_t p = 0; p < conv_k - 1; ++p) R[c * (conv_k - 1) + p] = in[T + p];
      for (int64_t tt = 0; tt < T; ++tt) {
        float s = 0.0f;
        for (int64_t j = 0; j < conv_k; ++j) s += in[tt + j] * cw[c * conv_k + j];
        conv[tt * C + c] = silu(s);
      }
    }
    // split_qkv_l2_norm_f32_qwen35
    std::vector<float> qv(T * key_dim), kv(T * key_dim), vv(T * value_dim);
    for (int64_t tt = 0; tt < T; ++tt) {
      for (int64_t h = 0; h < lk_heads; ++h) {
        const float* sq = &conv[tt * C + h * dk];
        const float* sk = &conv[tt * C + key_dim + h * dk];
        const float qs = l2_scale(sq, dk, eps), ks = l2_scale(sk, dk, eps);
        for (int64_t i = 0; i < dk; ++i) {
          qv[(tt * lk_heads + h) * dk + i] = sq[i] * qs;
          kv[(tt * lk_heads + h) * dk + i] = sk[i] * ks;
        }
      }
      for (int64_t i = 0; i < value_dim; ++i) vv[tt * value_dim + i] = conv[tt * C + 2 * key_dim + i];
    }
    std::vector<float> z(T * value_dim), beta(T * lv_heads), alpha(T * lv_heads);
    matmul(L(l, "attn_gate.weight"), normed.data(), T, z.data());
    matmul(L(l, "ssm_beta.weight"), normed.data(), T, beta.data());
    matmul(L(l, "ssm_alpha.weight"), normed.data(), T, alpha.data());
    // prepare_qwen35_gdn_gate_beta_f32 (mps_backend.mm:2588-2605)
    const float* dtb = f(L(l, "ssm_dt.bias"));
    const float* sa = f(L(l, "ssm_a"));
    for (int64_t i = 0; i < T * lv_heads; ++i) {
      const int64_t col = i % lv_heads;
      alpha[i] = softplus20(alpha[i] + dtb[col]) * sa[col];
      beta[i] = sigmoid(beta[i]);
    }
    std::vector<float> y(T * value_dim);
    gdn(qv.data(), kv.data(), vv.data(), alpha.data(), beta.data(),
        sstate.data() + li * lv_heads * dk * dk, T, lk_heads, lv_heads, dk, y.data());
    // qk_norm over value heads + silu(gate) * (qwen35_runtime.cpp:2993-3003)
    qk_norm(y.data(), f(L(l, "ssm_norm.weight")), T, lv_heads, dk, eps);
    for (int64_t i = 0; i < T * value_dim; ++i) y[i] *= silu(z[i]);
    std::vector<float> o(T * H);
    matmul(L(l, "ssm_out.weight"), y.data(), T, o.data());
    for (int64_t i = 0; i < T * H; ++i) o[i] += hidden_in[i];
    ffn(l, o.data(), T, out);
  }

  // FFN block shared by both layer kinds (qwen35_runtime.cpp:3054-3140, 3377-3420)
  void ffn(int64_t l, const float* h1, int64_t T, float* out) const {
    const int64_t H = hidden, I = rows(L(l, "ffn_gate.weight"));
    std::vector<float> post(T * H), up(T * I), gate(T * I), down(T * H);
    rms_norm(h1, f(L(l, "post_attention_norm.weight")), T, H, eps, post.data());
    matmul(L(l, "ffn_up.weight"), post.data(), T, up.data());
    matmul(L(l, "ffn_gate.weight"), post.data(), T, gate.data());
    for (int64_t i = 0; i < T * I; ++i) gate[i] = silu(gate[i]) * up[i];
    matmul(L(l, "ffn_down.weight"), gate.data(), T, down.data());
    for (int64_t i = 0; i < T * H; ++i) out[i] = down[i] + h1[i];
  }

  // run_qwen35_full_attention_layer_chunk (qwen35_runtime.cpp:3146-3423)
  void attention_layer(int64_t l, int64_t cache_layer, uint16_t* kc, uint16_t* vc,
                       const float* hidden_in, int64_t T, int64_t pos, float* out) {
    const int64_t H = hidden, hd = head_dim, ad = heads * hd, kd = kv_dim();
    std::vector<float> normed(T * H), qf(T * 2 * ad), q(T * ad), gt(T * ad), k(T * kd), v(T * kd);
    rms_norm(hidden_in, f(L(l, "attn_norm.weight")), T, H, eps, normed.data());
    matmul(L(l, "attn_q.weight"), normed.data(), T, qf.data());
    for (int64_t tt = 0; tt < T; ++tt)
      for (int64_t h = 0; h < heads; ++h)
        for (int64_t i = 0; i < hd; ++i) {
          q[(tt * heads + h) * hd + i] = qf[(tt * heads + h) * 2 * hd + i];
          gt[(tt * heads + h) * hd + i] = qf[(tt * heads + h) * 2 * hd + hd + i];
        }
    qk_norm(q.data(), f(L(l, "attn_q_norm.weight")), T, heads, hd, eps);
    matmul(L(l, "attn_k.weight"), normed.data(), T, k.data());
    matmul(L(l, "attn_v.weight"), normed.data(), T, v.data());
    qk_norm(k.data(), f(L(l, "attn_k_norm.weight")), T, kv_heads, hd, eps);
    std::vector<int32_t> positions(4 * T);
    for (int s = 0; s < 4; ++s)
      for (int64_t tt = 0; tt < T; ++tt) positions[tt + T * s] = static_cast<int32_t>(pos + tt);
    const int64_t n_dims = 2 * (sections[0] + sections[1] + sections[2] + sections[3]);
    mrope(q.data(), positions.data(), T, heads, hd, n_dims, sections, theta);
    mrope(k.data(), positions.data(), T, kv_heads, hd, n_dims, sections, theta);
    uint16_t* kl = kc + cache_layer * capacity * kd;
    uint16_t* vl = vc + cache_layer * capacity * kd;
    for (int64_t tt = 0; tt < T; ++tt)
      for (int64_t i = 0; i < kd; ++i) {
        kl[(pos + tt) * kd + i] = f32_to_f16_bits(k[tt * kd + i]);
        vl[(pos + tt) * kd + i] = f32_to_f16_bits(v[tt * kd + i]);
      }
    std::vector<float> att(T * ad);
    attention_f16kv(q.data(), kl, vl, pos, T, heads, kv_heads, hd, T >= 64, att.data());
    for (int64_t i = 0; i < T * ad; ++i) att[i] *= sigmoid(gt[i]);
    std::vector<float> o(T * H);
    matmul(L(l, "attn_output.weight"), att.data(), T, o.data());
    for (int64_t i = 0; i < T * H; ++i) o[i] += hidden_in[i];
    ffn(l, o.data(), T, out);
  }

  // run_qwen35_decode_tokens (qwen35_runtime.cpp:3860-3936): main layers over T tokens.
  void forward(const int32_t* ids, int64_t T, int64_t pos, std::vector<float>& hidden_out) {
    std::vector<float> h(T * hidden), nxt(T * hidden);
    embed(ids, T, h.data());
    for (int64_t l = 0; l < layers_main; ++l) {
      if (kinds[l] == 0) linear_layer(l, kind_index[l], h.data(), T, nxt.data());
      else attention_layer(l, kind_index[l], kcache.data(), vcache.data(), h.data(), T, pos, nxt.data());
      h.swap(nxt);
    }
    hidden_out = h;
  }

  // output norm (run_qwen35_output_norm, qwen35_runtime.cpp:3461-3503)
  void out_norm(const float* h, int64_t T, const std::string& wname, float* y) const {
    rms_norm(h, f(wname), T, hidden, eps, y);
  }

  // run_qwen35_lm_head_logits (qwen35_runtime.cpp:3505-3647): logits = E . h
  void logits(const float* hn, int64_t T, float* out) const {
    const std::string name = g->tensors.count("output.weight") ? "output.weight" : "token_embd.weight";
    matmul(name, hn, T, out);
  }

  // run_qwen35_mtp_tokens / _from_id_buffer (qwen35_runtime.cpp:3974-4240)
  void mtp(const int32_t* ids, const float* h_rows, int64_t T, int64_t pos, float* h_nextn) {
    const int64_t l = layers_main;
    std::vector<float> e(T * hidden), hn(T * hidden), en(T * hidden), cat(T * 2 * hidden), pr(T * hidden), bo(T * hidden);
    embed(ids, T, e.data());
    rms_norm(h_rows, f(L(l, "nextn.hnorm.weight")), T, hidden, eps, hn.data());
    rms_norm(e.data(), f(L(l, "nextn.enorm.weight")), T, hidden, eps, en.data());
    for (int64_t tt = 0; tt < T; ++tt) {
      std::memcpy(&cat[tt * 2 * hidden], &en[tt * hidden], hidden * 4);
      std::memcpy(&cat[tt * 2 * hidden + hidden], &hn[tt * hidden], hidden * 4);
    }
    matmul(L(l, "nextn.eh_proj.weight"), cat.data(), T, pr.data());
    attention_layer(l, 0, mtp_k.data(), mtp_v.data(), pr.data(), T, pos, bo.data());
    const std::string head_norm = g->tensors.count(L(l, "nextn.shared_head_norm.weight"))
                                    ? L(l, "nextn.shared_head_norm.weight")
                                    : "output_norm.weight";
    out_norm(bo.data(), T, head_norm, h_nextn);
  }
};

bool load_model(Model& m, const char* path, int64_t capacity) {
  m.g = open_gguf(path);
  if (!m.g) return false;
  auto num = [&](const std::string& k, double fb) {
    auto it = m.g->nums.find("qwen35." + k);
    return it == m.g->nums.end() ? fb : it->second;
  };
  m.hidden = static_cast<int64_t>(num("embedding_length", 0));
  m.inter = static_cast<int64_t>(num("feed_forward_length", 0));
  m.layers_total = static_cast<int64_t>(num("block_count", 0));
  const int64_t nextn = static_cast<int64_t>(num("nextn_predict_layers", 0));
  m.layers_main = m.layers_total - nextn;
  m.has_mtp = nextn == 1;
  m.heads = static_cast<int64_t>(num("attention.head_count", 0));
  m.kv_heads = static_cast<int64_t>(num("attention.head_count_kv", 0));
  m.head_dim = static_cast<int64_t>(num("attention.key_length", 0));
  m.eps = static_cast<float>(num("attention.layer_norm_rms_epsilon", 1e-6));
  m.theta = static_cast<float>(num("rope.freq_base", 1e7));
  m.conv_k = static_cast<int64_t>(num("ssm.conv_kernel", 4));
  m.lhead = static_cast<int64_t>(num("ssm.state_size", 128));
  m.lk_heads = static_cast<int64_t>(num("ssm.group_count", 16));
  m.lv_heads = static_cast<int64_t>(num("ssm.time_step_rank", 16));
  const int64_t interval = static_cast<int64_t>(num("full_attention_interval", 4));
  m.vocab = static_cast<int64_t>(m.g->tensors["token_embd.weight"].shape[1]);
  auto sec = m.g->arrays.find("qwen35.rope.dimension_sections");
  if (sec != m.g->arrays.end())
    for (size_t i = 0; i < 4 && i < sec->second.size(); ++i) m.sections[i] = sec->second[i];
  auto eos = m.g->nums.find("tokenizer.ggml.eos_token_id");
  if (eos != m.g->nums.end()) m.eos = static_cast<int64_t>(eos->second);
  m.conv_ch = 2 * m.lk_heads * m.lhead + m.lv_heads * m.lhead;
  for (int64_t l = 0; l < m.layers_main; ++l) {
    const int kind = ((l + 1) % interval) != 0 ? 0 : 1;
    m.kinds.push_back(kind);
    m.kind_index.push_back(kind == 0 ? m.n_lin++ : m.n_full++);
  }
  m.capacity = capacity;
  const int64_t kd = m.kv_dim();
  m.kcache.assign(m.n_full * capacity * kd, 0);
  m.vcache.assign(m.n_full * capacity * kd, 0);
  if (m.has_mtp) {
    m.mtp_k.assign(capacity * kd, 0);
    m.mtp_v.assign(capacity * kd, 0);
  }
  m.rstate.assign(m.n_lin * m.conv_ch * (m.conv_k - 1), 0.0f);
  m.sstate.assign(m.n_lin * m.lv_heads * m.lhead * m.lhead, 0.0f);
  m.pending_h.assign(m.hidden, 0.0f);
  return true;
}

bool is_eos(const Model& m, int64_t tok) { return tok == 151643 || tok == m.eos; }

}  // namespace

// =================================================================== C ABI

extern "C" {

struct orc_mtp_stats {
  int64_t drafted, accepted, verify_steps, confidence_stops, adaptive_budget, adaptive_changes;
  int64_t verified_by_position[8];
  int64_t accepted_by_position[8];
};

void orc_set_threads(int threads) { g_threads = threads < 1 ? 1 : threads; }
void orc_set_bucket_rows(int64_t rows) { g_bucket_rows = rows < 0 ? 0 : rows; }

uint16_t orc_f32_to_f16(float v) { return f32_to_f16_bits(v); }
float orc_f16_to_f32(uint16_t v) { return f16_bits_to_f32(v); }

int orc_dequant_rows(int type, const uint8_t* w, int64_t rows, int64_t cols, float* out) {
  if (block_bytes(type) == 0 || cols % 256) return -1;
  const int64_t bpr = cols / 256;
  for (int64_t r = 0; r < rows; ++r)
    for (int64_t b = 0; b < bpr; ++b) dequant_block(type, w + (r * bpr + b) * block_bytes(type), out + r * cols + b * 256);
  return 0;
}

int orc_quant_matmul(int type, const uint8_t* w, int64_t rows, int64_t cols, const float* x,
                     int64_t tokens, float* y) {
  if (block_bytes(type) == 0 || cols % 256 || tokens < 1) return -1;
  quant_matmul(type, w, rows, cols, x, tokens, y);
  return 0;
}

void orc_rms_norm(const float* x, const float* w, int64_t tokens, int64_t n, float eps, float* y) {
  rms_norm(x, w, tokens, n, eps, y);
}
void orc_qk_norm(float* v, const float* w, int64_t tokens, int64_t heads, int64_t d, float eps) {
  qk_norm(v, w, tokens, heads, d, eps);
}
// qwen35_norm_gated_f32_in_place (mps_backend.mm:2026-2063)
void orc_norm_gated(float* v, const float* w, const float* gate, int64_t tokens, int64_t heads,
                    int64_t d, float eps) {
  for (int64_t t = 0; t < tokens; ++t)
    for (int64_t h = 0; h < heads; ++h) {
      float* p = v + (t * heads + h) * d;
      const float s = rms_scale(p, d, eps);
      for (int64_t i = 0; i < d; ++i) p[i] = p[i] * s * w[i] * silu(gate[(t * heads + h) * d + i]);
    }
}
void orc_split_qkv_l2(const float* src, float* q, float* k, float* v, int64_t tokens,
                      int64_t key_heads, int64_t value_heads, int64_t d, float eps) {
  const int64_t key_dim = key_heads * d, C = 2 * key_dim + value_heads * d;
  for (int64_t t = 0; t < tokens; ++t) {
    for (int64_t h = 0; h < key_heads; ++h) {
      const float* sq = src + t * C + h * d;
      const float* sk = src + t * C + key_dim + h * d;
      const float qs = l2_scale(sq, d, eps), ks = l2_scale(sk, d, eps);
      for (int64_t i = 0; i < d; ++i) {
        q[(t * key_heads + h) * d + i] = sq[i] * qs;
        k[(t * key_heads + h) * d + i] = sk[i] * ks;
      }
    }
    for (int64_t i = 0; i < value_heads * d; ++i) v[t * value_heads * d + i] = src[t * C + 2 * key_dim + i];
  }
}
// build_ssm_conv_state_f32 + ssm_conv_f32 (mps_backend.mm:2376-2457); no activation.
void orc_conv(float* state, const float* input, const float* weights, int64_t conv_k, int64_t channels,
              int64_t tokens, float* out) {
  for (int64_t c = 0; c < channels; ++c) {
    std::vector<float> in(conv_k - 1 + tokens);
    for (int64_t p = 0; p < conv_k - 1; ++p) in[p] = state[c * (conv_k - 1) + p];
    for (int64_t t = 0; t < tokens; ++t) in[conv_k - 1 + t] = input[t * channels + c];
    for (int64_t p = 0; p < conv_k - 1; ++p) state[c * (conv_k - 1) + p] = in[tokens + p];
    for (int64_t t = 0; t < tokens; ++t) {
      float s = 0.0f;
      for (int64_t j = 0; j < conv_k; ++j) s += in[t + j] * weights[c * conv_k + j];
      out[t * channels + c] = s;
    }
  }
}
void orc_gdn(const float* q, const float* k, const float* v, const float* g, const float* beta,
             float* state, int64_t tokens, int64_t key_heads, int64_t value_heads, int64_t d, float* out) {
  gdn(q, k, v, g, beta, state, tokens, key_heads, value_heads, d, out);
}
void orc_prepare_gate_beta(float* gate, float* beta, const float* bias, const float* scale,
                           int64_t tokens, int64_t heads) {
  for (int64_t i = 0; i < tokens * heads; ++i) {
    const int64_t c = i % heads;
    gate[i] = softplus20(gate[i] + bias[c]) * scale[c];
    beta[i] = sigmoid(beta[i]);
  }
}
void orc_mrope(float* v, const int32_t* positions, int64_t tokens, int64_t heads, int64_t head_dim,
               int64_t n_dims, int64_t s0, int64_t s1, int64_t s2, int64_t s3, float theta) {
  const int64_t sec[4] = {s0, s1, s2, s3};
  mrope(v, positions, tokens, heads, head_dim, n_dims, sec, theta);
}
void orc_attention_f16kv(const float* q, const uint16_t* kc, const uint16_t* vc, int64_t start,
                         int64_t tokens, int64_t heads, int64_t kv_heads, int64_t head_dim,
                         int round_q, float* out) {
  attention_f16kv(q, kc, vc, start, tokens, heads, kv_heads, head_dim, round_q != 0, out);
}
int64_t orc_argmax(const float* v, int64_t n) { return argmax(v, n); }
// argmax_prob_f32_i32 (mps_backend.mm:2722-2779): p(top1) = 1 / sum exp(l - max)
float orc_top1_prob(const float* v, int64_t n) {
  const int64_t i = argmax(v, n);
  float s = 0.0f;
  for (int64_t j = 0; j < n; ++j) s += std::exp(v[j] - v[i]);
  return s > 0.0f ? 1.0f / s : 0.0f;
}

// ---- model-level entry points

void* orc_model_open(const char* gguf_path, int64_t capacity) {
  auto* m = new Model;
  if (!load_model(*m, gguf_path, capacity)) {
    delete m;
    return nullptr;
  }
  return m;
}
void orc_model_close(void* h) { delete static_cast<Model*>(h); }

int64_t orc_model_dim(void* h, int which) {
  auto* m = static_cast<Model*>(h);
  switch (which) {
    case 0: return m->hidden;
    case 1: return m->vocab;
    case 2: return m->layers_main;
    case 3: return m->has_mtp ? 1 : 0;
    case 4: return static_cast<int64_t>(m->kcache.size() * 2);
    case 5: return static_cast<int64_t>(m->rstate.size() * 4);
    case 6: return static_cast<int64_t>(m->sstate.size() * 4);
    case 7: return static_cast<int64_t>(m->mtp_k.size() * 2);
    default: return -1;
  }
}

// One main-model forward over T tokens at pos: writes the final (un-normed)
// hidden rows, the output-normed rows and the logits rows (any may be null).
int orc_model_forward(void* h, const int32_t* ids, int64_t T, int64_t pos, float* hidden_out,
                      float* normed_out, float* logits_out) {
  auto* m = static_cast<Model*>(h);
  if (pos + T > m->capacity) return -1;
  std::vector<float> hid;
  m->forward(ids, T, pos, hid);
  if (hidden_out) std::memcpy(hidden_out, hid.data(), hid.size() * 4);
  std::vector<float> hn(T * m->hidden);
  m->out_norm(hid.data(), T, "output_norm.weight", hn.data());
  if (normed_out) std::memcpy(normed_out, hn.data(), hn.size() * 4);
  if (logits_out) m->logits(hn.data(), T, logits_out);
  return 0;
}

// Cache state in/out (KV, R, S, MTP KV, pending h): the GPU engine and the
// oracle start a decode parity run from the same bytes.
int orc_model_state(void* h, int write_into_model, uint16_t* k, uint16_t* v, float* r, float* s,
                    uint16_t* mk, uint16_t* mv, float* pending_h) {
  auto* m = static_cast<Model*>(h);
  auto io = [&](auto& vec, auto* ptr) {
    if (!ptr) return;
    const size_t bytes = vec.size() * sizeof(vec[0]);
    if (write_into_model) std::memcpy(vec.data(), ptr, bytes);
    else std::memcpy(ptr, vec.data(), bytes);
  };
  io(m->kcache, k);
  io(m->vcache, v);
  io(m->rstate, r);
  io(m->sstate, s);
  io(m->mtp_k, mk);
  io(m->mtp_v, mv);
  io(m->pending_h, pending_h);
  return 0;
}

// generate_qwen35_metal's decode loops (qwen35_runtime.cpp:6457-6632) after a
// prefill that ends at `pos` with `first_logits_argmax` already sampled from the
// last prompt row.  mtp_draft_tokens == 0 selects the plain greedy loop.
// Returns the number of generated tokens written to out_tokens.
int64_t orc_generate_from(void* h, int64_t pos, int32_t first_token, int64_t max_new, int mtp_draft_tokens,
                          int adaptive, double p_min, int ignore_eos, int32_t* out_tokens, orc_mtp_stats* stats) {
  auto* m = static_cast<Model*>(h);
  int64_t n = 0;
  std::vector<float> hid, hn, lg;
  const int64_t V = m->vocab, H = m->hidden;
  if (mtp_draft_tokens <= 0 || !m->has_mtp) {
    int32_t tok = first_token;
    for (int64_t step = 0; step < max_new; ++step) {
      if (step > 0) {
        m->forward(&tok, 1, pos, hid);
        ++pos;
        hn.assign(H, 0.0f);
        m->out_norm(hid.data(), 1, "output_norm.weight", hn.data());
        lg.assign(V, 0.0f);
        m->logits(hn.data(), 1, lg.data());
        tok = static_cast<int32_t>(argmax(lg.data(), V));
      }
      if (!ignore_eos && is_eos(*m, tok)) break;
      out_tokens[n++] = tok;
    }
    return n;
  }
  // MTP greedy loop.  Budget control follows update_mtp_adaptive_budget
  // (qwen35_runtime.cpp:6421-6455).  With p_min > 0 a draft whose head p(top1)
  // is below p_min ends the chain and is not drafted (read_mtp_draft_token,
  // qwen35_runtime.cpp:6184-6210; confidence_stops counts these).  The
  // reference runs every forward of the chain before reading the tokens
  // (6339-6364); forwards past the stop only write MTP cache positions that the
  // next chain rewrites before it reads them, so stopping early is equivalent.
  const size_t K = static_cast<size_t>(mtp_draft_tokens);
  size_t budget = adaptive ? 1 : K;
  size_t win_d = 0, win_a = 0;
  std::memset(stats, 0, sizeof(*stats));
  int32_t next_token = first_token;
  std::vector<float> rs = m->rstate, ss = m->sstate;
  while (n < max_new) {
    if (!ignore_eos && is_eos(*m, next_token)) break;
    out_tokens[n++] = next_token;
    if (n >= max_new) break;
    const int64_t vpos = pos;
    const size_t b = std::min<size_t>(budget, static_cast<size_t>(max_new - n));
    // draft_mtp_tokens (6274-6419): chained MTP forwards, h from pending_h then own h_nextn
    std::vector<int32_t> drafts;
    std::vector<float> hin = m->pending_h, hnext(H);
    int32_t dt = next_token;
    for (size_t i = 0; i < b; ++i) {
      m->mtp(&dt, hin.data(), 1, vpos + static_cast<int64_t>(i), hnext.data());
      lg.assign(V, 0.0f);
      const std::string head = m->g->tensors.count("output.weight") ? "output.weight" : "token_embd.weight";
      m->matmul(head, hnext.data(), 1, lg.data());
      dt = static_cast<int32_t>(argmax(lg.data(), V));
      if (p_min > 0.0 && static_cast<double>(orc_top1_prob(lg.data(), V)) < p_min) {
        ++stats->confidence_stops;
        break;
      }
      drafts.push_back(dt);
      ++stats->drafted;
      hin = hnext;
    }
    std::vector<int32_t> verify{next_token};
    verify.insert(verify.end(), drafts.begin(), drafts.end());
    rs = m->rstate;
    ss = m->sstate;  // snapshot_recurrent_state (6154-6167)
    const int64_t T = static_cast<int64_t>(verify.size());
    m->forward(verify.data(), T, vpos, hid);
    hn.assign(T * H, 0.0f);
    m->out_norm(hid.data(), T, "output_norm.weight", hn.data());
    lg.assign(T * V, 0.0f);
    m->logits(hn.data(), T, lg.data());
    size_t acc = 0;
    bool stop = false;
    for (size_t i = 0; i < drafts.size(); ++i) {
      if (n >= max_new) break;
      const int32_t target = static_cast<int32_t>(argmax(&lg[i * V], V));
      ++stats->verify_steps;
      if (i < 8) ++stats->verified_by_position[i];
      if (!ignore_eos && is_eos(*m, target)) {
        stop = true;
        break;
      }
      if (target != drafts[i]) break;
      out_tokens[n++] = drafts[i];
      ++acc;
      ++stats->accepted;
      if (i < 8) ++stats->accepted_by_position[i];
      if (n >= max_new) break;
    }
    if (adaptive && K > 1 && !drafts.empty()) {
      win_d += drafts.size();
      win_a += acc;
      const size_t thr = std::max<size_t>(16, budget * 8);
      if (win_d >= thr) {
        bool changed = false;
        if (budget > 1 && win_a * 4 < win_d * 3) {
          --budget;
          changed = true;
        } else if (budget < K && win_a == win_d) {
          ++budget;
          changed = true;
        }
        if (changed) {
          ++stats->adaptive_changes;
          win_d = win_a = 0;
        } else if (win_d >= thr * 2) {
          win_d = win_a = 0;
        }
      }
    }
    const int64_t committed = 1 + static_cast<int64_t>(acc);
    if (stop) break;
    if (acc == drafts.size()) {
      pos = vpos + committed;
      std::memcpy(m->pending_h.data(), &hn[(committed - 1) * H], H * 4);
      next_token = static_cast<int32_t>(argmax(&lg[(committed - 1) * V], V));
    } else {
      m->rstate = rs;
      m->sstate = ss;  // restore_recurrent_state (6169-6182) and re-run the commit tokens
      std::vector<int32_t> commit(verify.begin(), verify.begin() + committed);
      m->forward(commit.data(), committed, vpos, hid);
      hn.assign(committed * H, 0.0f);
      m->out_norm(hid.data(), committed, "output_norm.weight", hn.data());
      lg.assign(committed * V, 0.0f);
      m->logits(hn.data(), committed, lg.data());
      pos = vpos + committed;
      std::memcpy(m->pending_h.data(), &hn[(committed - 1) * H], H * 4);
      next_token = static_cast<int32_t>(argmax(&lg[(committed - 1) * V], V));
    }
  }
  stats->adaptive_budget = static_cast<int64_t>(budget);
  return n;
}

// MTP layer processing of a prompt chunk (qwen35_runtime.cpp:5894-5961): the MTP
// KV cache is filled with the chunk's tokens and the shifted normed hidden rows;
// pending_h becomes the chunk's last normed row.
int orc_mtp_process_chunk(void* h, const int32_t* ids, const float* normed_rows, int64_t T, int64_t pos) {
  auto* m = static_cast<Model*>(h);
  if (!m->has_mtp) return -1;
  const int64_t H = m->hidden;
  std::vector<float> shifted(T * H), hn(T * H);
  std::memcpy(shifted.data(), m->pending_h.data(), H * 4);
  if (T > 1) std::memcpy(&shifted[H], normed_rows, (T - 1) * H * 4);
  m->mtp(ids, shifted.data(), T, pos, hn.data());
  std::memcpy(m->pending_h.data(), &normed_rows[(T - 1) * H], H * 4);
  return 0;
}

}  // extern "C"
