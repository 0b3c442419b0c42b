// kquant.cuh -- device-side decode of GGUF K-quant super-blocks as stored
// (Q4_K 144 B, Q5_K 176 B, Q6_K 210 B per 256 weights), read from a shared
// memory copy of the raw bytes.
//
// Block formats follow the reference's decoders: q4_k_scale_min and the
// q{4,5,6}_k_matvec kernels (mps_backend.mm:282-463) and the host decoder
// dequantize_quantized_transposed_f32 (qwen35_runtime.cpp:1084-1241).
//
// A "unit" is 64 weights of one row handled by one lane:
//   Q4_K/Q5_K unit s (0..3): quant bytes qs[32s..32s+31]; low nibbles are
//     columns 64s+i (sub-block 2s), high nibbles 64s+32+i (sub-block 2s+1);
//     Q5_K adds qh bit 2s / 2s+1 as the fifth bit.
//   Q6_K unit (c, r) (c = half, r = 0/1): i in [16r, 16r+16) of the reference's
//     32-wide loop; group k (0..3) is column 128c+32k+16r+i with scale
//     sc[8c + r + 2k].
// Every unit therefore covers 64 contiguous input columns starting at
//   Q4/Q5: 64s          Q6: 128c + 16r  (four runs of 16 at stride 32)
// and the x values a lane needs are loaded once into registers.
//
// Integer codes b are materialised as the float 0.5 + b/256 (one PRMT) and
// dotted with x in fp32 (FFMA2); the group sum of b*x is recovered exactly as
// 256*acc - 128*sum(x).  The result equals the reference's fp32 dot product up
// to summation order.
#pragma once

#include "kib_common.cuh"

namespace kib {

// Loads 16 bytes from a 2-byte-aligned shared memory address.
KIB_DEV uint4 lds16_a2(const uint8_t* p) {
  const uintptr_t a = reinterpret_cast<uintptr_t>(p);
  const uint32_t* base = reinterpret_cast<const uint32_t*>(a & ~uintptr_t(3));
  const uint32_t sh = static_cast<uint32_t>(a & 3u) * 8u;
  const uint32_t w0 = base[0], w1 = base[1], w2 = base[2], w3 = base[3], w4 = base[4];
  uint4 r;
  r.x = __funnelshift_r(w0, w1, sh);
  r.y = __funnelshift_r(w1, w2, sh);
  r.z = __funnelshift_r(w2, w3, sh);
  r.w = __funnelshift_r(w3, w4, sh);
  return r;
}

KIB_DEV uint2 lds8_a2(const uint8_t* p) {
  const uintptr_t a = reinterpret_cast<uintptr_t>(p);
  const uint32_t* base = reinterpret_cast<const uint32_t*>(a & ~uintptr_t(3));
  const uint32_t sh = static_cast<uint32_t>(a & 3u) * 8u;
  const uint32_t w0 = base[0], w1 = base[1], w2 = base[2];
  return make_uint2(__funnelshift_r(w0, w1, sh), __funnelshift_r(w1, w2, sh));
}

KIB_DEV uint32_t lds_u16(const uint8_t* p) { return *reinterpret_cast<const uint16_t*>(p); }

// Number of 64-weight units in one 256-weight block.
template <int QT>
struct KQ {
  static constexpr int kBlockBytes = kquant_block_bytes(QT);
  static constexpr int kGroups = QT == kTypeQ6K ? 4 : 2;   // scale groups per unit
  static constexpr int kGroupLen = QT == kTypeQ6K ? 16 : 32;
};

// Column offset (within the block) of element e (0..63) of unit u.
template <int QT>
KIB_DEV int unit_col(int u, int e) {
  if (QT == kTypeQ6K) {
    const int c = u >> 1, r = u & 1, k = e >> 4, i = e & 15;
    return 128 * c + 32 * k + 16 * r + i;
  }
  return 64 * u + e;
}

// Codes of one unit as 16 words of 4 bytes each, ordered so that word w holds
// elements 4w..4w+3 of the unit (element order as unit_col).
// Raw bytes of one unit, as loaded from memory (shared or global):
//   Q4_K: a,b = its 32 quant bytes, h = the 16-byte header (d, dmin, scales)
//   Q5_K: as Q4_K plus qh0,qh1 = the block's 32 high-bit bytes
//   Q6_K: a = ql[64c+16r..], b = ql[64c+32+16r..], h = qh[32c+16r..],
//         s8 = scales[8c..8c+7], d = the fp16 super-block scale
template <int QT>
struct RawUnit {
  uint4 a, b, h;
  uint4 qh0, qh1;
  uint2 s8;
  uint32_t d;
};

template <int QT>
KIB_DEV RawUnit<QT> load_raw(const uint8_t* blk, int u) {
  RawUnit<QT> r;
  if (QT == kTypeQ4K || QT == kTypeQ5K) {
    const uint8_t* qs = blk + (QT == kTypeQ4K ? 16 : 48) + 32 * u;
    r.a = *reinterpret_cast<const uint4*>(qs);
    r.b = *reinterpret_cast<const uint4*>(qs + 16);
    r.h = *reinterpret_cast<const uint4*>(blk);
    if (QT == kTypeQ5K) {
      r.qh0 = *reinterpret_cast<const uint4*>(blk + 16);
      r.qh1 = *reinterpret_cast<const uint4*>(blk + 32);
    }
  } else {
    const int c = u >> 1, rr = u & 1;
    r.a = lds16_a2(blk + 64 * c + 16 * rr);
    r.b = lds16_a2(blk + 64 * c + 32 + 16 * rr);
    r.h = lds16_a2(blk + 128 + 32 * c + 16 * rr);
    r.s8 = lds8_a2(blk + 192 + 8 * c);
    r.d = lds_u16(blk + 208);
  }
  return r;
}

template <int QT>
KIB_DEV void codes_from_raw(const RawUnit<QT>& r, int u, uint32_t (&q)[16]) {
  if (QT == kTypeQ4K || QT == kTypeQ5K) {
    const uint32_t w[8] = {r.a.x, r.a.y, r.a.z, r.a.w, r.b.x, r.b.y, r.b.z, r.b.w};
    if (QT == kTypeQ4K) {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        q[i] = w[i] & 0x0F0F0F0Fu;
        q[8 + i] = (w[i] >> 4) & 0x0F0F0F0Fu;
      }
    } else {
      const uint32_t h[8] = {r.qh0.x, r.qh0.y, r.qh0.z, r.qh0.w, r.qh1.x, r.qh1.y, r.qh1.z, r.qh1.w};
      const int sl = 2 * u, sh = 2 * u + 1;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        q[i] = (w[i] & 0x0F0F0F0Fu) | (((h[i] >> sl) << 4) & 0x10101010u);
        q[8 + i] = ((w[i] >> 4) & 0x0F0F0F0Fu) | (((h[i] >> sh) << 4) & 0x10101010u);
      }
    }
  } else {
    const uint32_t a[4] = {r.a.x, r.a.y, r.a.z, r.a.w}, b[4] = {r.b.x, r.b.y, r.b.z, r.b.w},
                   h[4] = {r.h.x, r.h.y, r.h.z, r.h.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      q[i] = (a[i] & 0x0F0F0F0Fu) | ((h[i] << 4) & 0x30303030u);             // k=0
      q[4 + i] = (b[i] & 0x0F0F0F0Fu) | ((h[i] << 2) & 0x30303030u);         // k=1
      q[8 + i] = ((a[i] >> 4) & 0x0F0F0F0Fu) | (h[i] & 0x30303030u);         // k=2
      q[12 + i] = ((b[i] >> 4) & 0x0F0F0F0Fu) | ((h[i] >> 2) & 0x30303030u); // k=3
    }
  }
}

// Per-group affine coefficients of one unit: value_e = A_g * code_e + B_g.
//   Q4/Q5: A = d*sc, B = -dmin*m          (group 0 = sub-block 2u, 1 = 2u+1)
//   Q6   : A = d*sc, B = -32*d*sc
template <int QT>
KIB_DEV void coeffs_from_raw(const RawUnit<QT>& r, int u, float (&A)[4], float (&B)[4]) {
  if (QT == kTypeQ4K || QT == kTypeQ5K) {
    const uint4 h = r.h;
    const float d = half_bits_to_float(static_cast<uint16_t>(h.x & 0xFFFFu));
    const float dmin = half_bits_to_float(static_cast<uint16_t>(h.x >> 16));
    uint32_t scw, mw;
    int idx;
    if (u < 2) {
      scw = h.y & 0x3F3F3F3Fu;
      mw = h.z & 0x3F3F3F3Fu;
      idx = 2 * u;
    } else {
      scw = (h.w & 0x0F0F0F0Fu) | ((h.y >> 2) & 0x30303030u);
      mw = ((h.w >> 4) & 0x0F0F0F0Fu) | ((h.z >> 2) & 0x30303030u);
      idx = 2 * u - 4;
    }
    const float sc0 = static_cast<float>((scw >> (8 * idx)) & 0xFFu);
    const float sc1 = static_cast<float>((scw >> (8 * idx + 8)) & 0xFFu);
    const float m0 = static_cast<float>((mw >> (8 * idx)) & 0xFFu);
    const float m1 = static_cast<float>((mw >> (8 * idx + 8)) & 0xFFu);
    A[0] = d * sc0;
    B[0] = -(dmin * m0);
    A[1] = d * sc1;
    B[1] = -(dmin * m1);
    A[2] = A[3] = B[2] = B[3] = 0.0f;
  } else {
    const int rr = u & 1;
    const float d = half_bits_to_float(static_cast<uint16_t>(r.d & 0xFFFFu));
    const uint32_t sw[2] = {r.s8.x, r.s8.y};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int idx = rr + 2 * k;  // 0..7
      const int8_t sc = static_cast<int8_t>((sw[idx >> 2] >> (8 * (idx & 3))) & 0xFFu);
      A[k] = d * static_cast<float>(sc);
      B[k] = -32.0f * A[k];
    }
  }
}

template <int QT>
KIB_DEV void unit_codes(const uint8_t* blk, int u, uint32_t (&q)[16]) {
  codes_from_raw<QT>(load_raw<QT>(blk, u), u, q);
}

template <int QT>
KIB_DEV void unit_coeffs(const uint8_t* blk, int u, float (&A)[4], float (&B)[4]) {
  coeffs_from_raw<QT>(load_raw<QT>(blk, u), u, A, B);
}

KIB_DEV float2 code_pair_lo(uint32_t w) {
  return make_float2(byte_as_half_plus(w, kSelByte0), byte_as_half_plus(w, kSelByte1));
}
KIB_DEV float2 code_pair_hi(uint32_t w) {
  return make_float2(byte_as_half_plus(w, kSelByte2), byte_as_half_plus(w, kSelByte3));
}

// x values of one unit for one token: 64 floats as 32 float2 (element order as
// unit_col) plus the per-group sums of x.
template <int QT>
struct UnitX {
  float2 v[32];
  float s[KQ<QT>::kGroups];
};

template <int QT>
KIB_DEV void load_unit_x(const float* xs_block /* x + 256*block */, int u, UnitX<QT>& ux) {
  if (QT == kTypeQ6K) {
    const int c = u >> 1, r = u & 1;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float4* p = reinterpret_cast<const float4*>(xs_block + 128 * c + 32 * k + 16 * r);
      float s = 0.0f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float4 f = p[j];
        ux.v[8 * k + 2 * j] = make_float2(f.x, f.y);
        ux.v[8 * k + 2 * j + 1] = make_float2(f.z, f.w);
        s += (f.x + f.y) + (f.z + f.w);
      }
      ux.s[k] = s;
    }
  } else {
    const float4* p = reinterpret_cast<const float4*>(xs_block + 64 * u);
#pragma unroll
    for (int g = 0; g < 2; ++g) {
      float s = 0.0f;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float4 f = p[8 * g + j];
        ux.v[16 * g + 2 * j] = make_float2(f.x, f.y);
        ux.v[16 * g + 2 * j + 1] = make_float2(f.z, f.w);
        s += (f.x + f.y) + (f.z + f.w);
      }
      ux.s[g] = s;
    }
  }
}

// Dot product of one unit with NT token vectors; adds into out[t].
template <int QT, int NT>
KIB_DEV void unit_dot(const uint8_t* blk, int u, const UnitX<QT> (&ux)[NT], float (&out)[NT]) {
  constexpr int G = KQ<QT>::kGroups;
  constexpr int WPG = 16 / G;  // code words per group
  uint32_t q[16];
  unit_codes<QT>(blk, u, q);
  float A[4], B[4];
  unit_coeffs<QT>(blk, u, A, B);
  float2 acc[NT][G];
#pragma unroll
  for (int t = 0; t < NT; ++t)
#pragma unroll
    for (int g = 0; g < G; ++g) acc[t][g] = make_float2(0.0f, 0.0f);
#pragma unroll
  for (int w = 0; w < 16; ++w) {
    const float2 lo = code_pair_lo(q[w]);
    const float2 hi = code_pair_hi(q[w]);
    const int g = w / WPG;
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      acc[t][g] = ffma2(lo, ux[t].v[2 * w], acc[t][g]);
      acc[t][g] = ffma2(hi, ux[t].v[2 * w + 1], acc[t][g]);
    }
  }
#pragma unroll
  for (int t = 0; t < NT; ++t) {
    float r = 0.0f;
#pragma unroll
    for (int g = 0; g < G; ++g) {
      // sum(code * x) = 256*acc - 128*sum(x); value = A*code + B
      const float cx = fmaf(256.0f, acc[t][g].x + acc[t][g].y, -128.0f * ux[t].s[g]);
      r = fmaf(A[g], cx, fmaf(B[g], ux[t].s[g], r));
    }
    out[t] += r;
  }
}

// Same dot product over a unit already loaded into registers.
template <int QT, int NT>
KIB_DEV void unit_dot_raw(const RawUnit<QT>& raw, int u, const UnitX<QT> (&ux)[NT], float (&out)[NT]) {
  constexpr int G = KQ<QT>::kGroups;
  constexpr int WPG = 16 / G;  // code words per group
  uint32_t q[16];
  codes_from_raw<QT>(raw, u, q);
  float A[4], B[4];
  coeffs_from_raw<QT>(raw, u, A, B);
  float2 acc[NT][G];
#pragma unroll
  for (int t = 0; t < NT; ++t)
#pragma unroll
    for (int g = 0; g < G; ++g) acc[t][g] = make_float2(0.0f, 0.0f);
#pragma unroll
  for (int w = 0; w < 16; ++w) {
    const float2 lo = code_pair_lo(q[w]);
    const float2 hi = code_pair_hi(q[w]);
    const int g = w / WPG;
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      acc[t][g] = ffma2(lo, ux[t].v[2 * w], acc[t][g]);
      acc[t][g] = ffma2(hi, ux[t].v[2 * w + 1], acc[t][g]);
    }
  }
#pragma unroll
  for (int t = 0; t < NT; ++t) {
    float r = 0.0f;
#pragma unroll
    for (int g = 0; g < G; ++g) {
      // sum(code * x) = 256*acc - 128*sum(x); value = A*code + B
      const float cx = fmaf(256.0f, acc[t][g].x + acc[t][g].y, -128.0f * ux[t].s[g]);
      r = fmaf(A[g], cx, fmaf(B[g], ux[t].s[g], r));
    }
    out[t] += r;
  }
}

// Dequantized value of element e of unit u, exactly as the reference
// (d1*q - m1 for Q4/Q5, d*sc*(q-32) for Q6; products are exact in fp32).
template <int QT>
KIB_DEV void unit_dequant(const uint8_t* blk, int u, float (&out)[64]) {
  uint32_t q[16];
  unit_codes<QT>(blk, u, q);
  float A[4], B[4];
  unit_coeffs<QT>(blk, u, A, B);
  constexpr int WPG = 16 / KQ<QT>::kGroups;
#pragma unroll
  for (int w = 0; w < 16; ++w) {
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float code = static_cast<float>((q[w] >> (8 * k)) & 0xFFu);
      const int g = w / WPG;
      if (QT == kTypeQ6K) {
        out[4 * w + k] = A[g] * (code - 32.0f);
      } else {
        out[4 * w + k] = fmaf(A[g], code, B[g]);  // A*q exact, one rounding like a*q - m
      }
    }
  }
}

// Per-weight fp16 value used by the reference's multi-token buckets
// (dequantize_q{4,5,6}_k_mm, mps_backend.mm:780-864): the fp32 value
// dl*q - ml rounded to half.  Q6_K rounds dl0*q' and then subtracts 32*dl0.
// Returned as 32 half2 pairs (element order as unit_col): codes become floats
// by exponent insertion (2^23 + b, exact), each pair is rounded with one packed
// conversion.
template <int QT>
KIB_DEV void unit_dequant_h2(const uint8_t* blk, int u, __half2 (&out)[32]) {
  uint32_t q[16];
  unit_codes<QT>(blk, u, q);
  float A[4], B[4];
  unit_coeffs<QT>(blk, u, A, B);
  constexpr int WPG = 16 / KQ<QT>::kGroups;
#pragma unroll
  for (int w = 0; w < 16; ++w) {
    const int g = w / WPG;
    float v[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float code = __uint_as_float(0x4B000000u | ((q[w] >> (8 * k)) & 0xFFu)) - 8388608.0f;
      if (QT == kTypeQ6K) {
        v[k] = __fsub_rn(__fmul_rn(A[g], code), __fmul_rn(A[g], 32.0f));
      } else {
        v[k] = fmaf(A[g], code, B[g]);
      }
    }
    out[2 * w] = __floats2half2_rn(v[0], v[1]);
    out[2 * w + 1] = __floats2half2_rn(v[2], v[3]);
  }
}

}  // namespace kib
