// ops.cu -- op-level C ABI (the MpsContext twin): context lifetime, memory,
// K-quant matvec/matmul/argmax/get_rows, norms, GDN, conv, MRoPE, attention,
// element-wise ops and copies.  Shape validation follows the reference's
// MpsContext checks (mps_backend.mm:4006-4308): invalid shapes return
// KIB_ERR_INVALID_ARGUMENT with a message, never launch.
#include <cuda_fp16.h>

#include <cstring>
#include <string>

#include "kib_ctx.cuh"
#include "kquant_gemv2.cuh"
#include "layer_kernels.cuh"
#include "gemm_tc.cuh"
#include "kq_skinny.cuh"

#include <cudaTypedefs.h>

using namespace kib;

// =========================================================== small kernels
namespace {

// float4 paths need 16-byte aligned rows (half outputs: 8 bytes)
__device__ __forceinline__ bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
__device__ __forceinline__ bool al8(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 7u) == 0; }

// out16 (may be null): the same values rounded to half, [T][n] packed -- the
// input of the prefill GEMMs, so they need no conversion pass of their own.
__global__ void rms_norm_rows_kernel(const float* in, const float* w, int n, float eps, float* out, __half* out16) {
  __shared__ float red[32];
  const int t = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  pdl_wait();
  pdl_launch_dependents();
  const float* x = in + static_cast<size_t>(t) * n;
  float* y = out + static_cast<size_t>(t) * n;
  __half* y16 = out16 ? out16 + static_cast<size_t>(t) * n : nullptr;
  if (n == 4 * static_cast<int>(blockDim.x) && al16(in) && al16(w) && al16(out) && (!out16 || al8(out16))) {
    // one float4 per thread (the model's hidden width)
    const float4 v = reinterpret_cast<const float4*>(x)[tid];
    float ss = (v.x * v.x + v.y * v.y) + (v.z * v.z + v.w * v.w);
    ss = warp_sum(ss);
    if (lane == 0) red[warp] = ss;
    __syncthreads();
    float tot = 0.0f;
    for (int i = 0; i < static_cast<int>(blockDim.x) / 32; ++i) tot += red[i];
    const float scale = 1.0f / sqrtf(tot / static_cast<float>(n) + eps);
    const float4 g = reinterpret_cast<const float4*>(w)[tid];
    const float4 r = make_float4(v.x * scale * g.x, v.y * scale * g.y, v.z * scale * g.z, v.w * scale * g.w);
    reinterpret_cast<float4*>(y)[tid] = r;
    if (y16) {
      reinterpret_cast<__half2*>(y16)[2 * tid] = __floats2half2_rn(r.x, r.y);
      reinterpret_cast<__half2*>(y16)[2 * tid + 1] = __floats2half2_rn(r.z, r.w);
    }
    return;
  }
  float ss = 0.0f;
  for (int i = tid; i < n; i += blockDim.x) ss += x[i] * x[i];
  ss = warp_sum(ss);
  if (lane == 0) red[warp] = ss;
  __syncthreads();
  float tot = 0.0f;
  for (int i = 0; i < static_cast<int>(blockDim.x) / 32; ++i) tot += red[i];
  const float scale = 1.0f / sqrtf(tot / static_cast<float>(n) + eps);
  for (int i = tid; i < n; i += blockDim.x) {
    const float r = x[i] * scale * w[i];
    y[i] = r;
    if (y16) y16[i] = __float2half_rn(r);
  }
}

// per-head RMSNorm in place; if gate != null also * silu(gate) (norm_gated).
// One warp per (head, token), four per CTA; out16 as for rms_norm_rows_kernel.
// gate rows are gate_ld floats apart (0: heads * d, packed).
__global__ void head_norm_kernel(float* v, const float* w, const float* gate, int heads, int d, float eps,
                                 float* out, __half* out16, int gate_ld) {
  const int h = blockIdx.x * 4 + (threadIdx.x >> 5), t = blockIdx.y, lane = threadIdx.x & 31;
  pdl_wait();
  pdl_launch_dependents();
  if (h >= heads) return;
  const size_t base = (static_cast<size_t>(t) * heads + h) * d;
  if (gate) gate += static_cast<size_t>(t) * (gate_ld ? gate_ld : heads * d) + static_cast<size_t>(h) * d - base;
  float* dst = out ? out : v;
  if (d == 128 && al16(v) && al16(w) && al16(dst) && (!gate || al16(gate)) && (!out16 || al8(out16))) {
    const float4 x = reinterpret_cast<const float4*>(v + base)[lane];
    float ss = (x.x * x.x + x.y * x.y) + (x.z * x.z + x.w * x.w);
    ss = warp_sum(ss);
    const float scale = 1.0f / sqrtf(ss / static_cast<float>(d) + eps);
    const float4 g = reinterpret_cast<const float4*>(w)[lane];
    float4 r;
    if (gate) {
      const float4 z = reinterpret_cast<const float4*>(gate + base)[lane];
      r = make_float4(x.x * scale * g.x * silu_k(z.x), x.y * scale * g.y * silu_k(z.y), x.z * scale * g.z * silu_k(z.z),
                      x.w * scale * g.w * silu_k(z.w));
    } else {
      r = make_float4(x.x * (scale * g.x), x.y * (scale * g.y), x.z * (scale * g.z), x.w * (scale * g.w));
    }
    reinterpret_cast<float4*>(dst + base)[lane] = r;
    if (out16) {
      reinterpret_cast<__half2*>(out16 + base)[2 * lane] = __floats2half2_rn(r.x, r.y);
      reinterpret_cast<__half2*>(out16 + base)[2 * lane + 1] = __floats2half2_rn(r.z, r.w);
    }
    return;
  }
  float ss = 0.0f;
  for (int i = lane; i < d; i += 32) ss += v[base + i] * v[base + i];
  ss = warp_sum(ss);
  const float scale = 1.0f / sqrtf(ss / static_cast<float>(d) + eps);
  for (int i = lane; i < d; i += 32) {
    // qk_norm: v * (scale * w); norm_gated: v * scale * w * silu(gate)
    const float r = gate ? v[base + i] * scale * w[i] * silu_k(gate[base + i]) : v[base + i] * (scale * w[i]);
    dst[base + i] = r;
    if (out16) out16[base + i] = __float2half_rn(r);
  }
}

__global__ void split_qkv_l2_kernel(const float* src, float* q, float* k, float* v, int key_heads, int value_heads,
                                    int d, float eps) {
  const int h = blockIdx.x, t = blockIdx.y, part = blockIdx.z, lane = threadIdx.x;
  const int key_dim = key_heads * d, C = 2 * key_dim + value_heads * d;
  const float* row = src + static_cast<size_t>(t) * C;
  if (part == 2) {
    if (h >= value_heads) return;
    for (int i = lane; i < d; i += 32) v[(static_cast<size_t>(t) * value_heads + h) * d + i] = row[2 * key_dim + h * d + i];
    return;
  }
  if (h >= key_heads) return;
  const float* s = row + part * key_dim + h * d;
  float ss = 0.0f;
  for (int i = lane; i < d; i += 32) ss += s[i] * s[i];
  ss = warp_sum(ss);
  const float scale = 1.0f / fmaxf(sqrtf(ss), eps);
  float* dst = part == 0 ? q : k;
  for (int i = lane; i < d; i += 32) dst[(static_cast<size_t>(t) * key_heads + h) * d + i] = s[i] * scale;
}

// build_ssm_conv_state_f32 + ssm_conv_f32 (+ optional silu), in place or not.
// A CTA owns 32 channels and all T tokens; thread (channel, tile) convolves one
// tile of tokens.  Every thread first reads the K-1 inputs before its tile (the
// carried state for the first tile), then the CTA barrier, then each thread
// reads and overwrites only its own tokens, so tiles run in parallel even when
// out aliases in.  The last tile leaves with the new state in its window.  The
// sum order per output is the reference's (j = 0..K-1).
__global__ void conv_stateful_kernel(float* state, const float* in, int in_ld, const float* w, int K, int C, int T,
                                     float* out, int out_ld, int apply_silu) {
  pdl_wait();
  pdl_launch_dependents();
  const int c = blockIdx.x * 32 + threadIdx.x;
  const int ntiles = blockDim.y, tile = threadIdx.y;
  const int len = (T + ntiles - 1) / ntiles;
  const int t0 = min(tile * len, T), t1 = min(t0 + len, T);
  float win[16], wc[16];
  if (c < C) {
    for (int j = 0; j < K; ++j) wc[j] = w[static_cast<size_t>(c) * K + j];
    for (int j = 0; j < K - 1; ++j) {
      const int t = t0 - (K - 1) + j;
      win[j] = t >= 0 ? in[static_cast<size_t>(t) * in_ld + c] : state[static_cast<size_t>(c) * (K - 1) + (t + K - 1)];
    }
  }
  __syncthreads();
  if (c >= C) return;
  for (int t = t0; t < t1; ++t) {
    win[K - 1] = in[static_cast<size_t>(t) * in_ld + c];
    float s = 0.0f;
    for (int j = 0; j < K; ++j) s += win[j] * wc[j];
    out[static_cast<size_t>(t) * out_ld + c] = apply_silu ? silu_k(s) : s;
    for (int j = 0; j < K - 1; ++j) win[j] = win[j + 1];
  }
  // the tile holding token T-1 ends with the window [.., T-1]; with T < K-1 that
  // is tile 0, whose window also carries the older state entries
  if (t1 == T && t0 < T) for (int j = 0; j < K - 1; ++j) state[static_cast<size_t>(c) * (K - 1) + j] = win[j];
}

// The same with the kernel size fixed at compile time: the window lives in
// registers and four tokens' inputs are loaded together.  Identical sums.
template <int K>
__global__ void conv_stateful_k_kernel(float* state, const float* in, int in_ld, const float* w, int C, int T,
                                       float* out, int out_ld, int apply_silu) {
  pdl_wait();
  pdl_launch_dependents();
  const int c = blockIdx.x * 32 + threadIdx.x;
  const int ntiles = blockDim.y, tile = threadIdx.y;
  const int len = (T + ntiles - 1) / ntiles;
  const int t0 = min(tile * len, T), t1 = min(t0 + len, T);
  float win[K], wc[K];
  if (c < C) {
#pragma unroll
    for (int j = 0; j < K; ++j) wc[j] = w[static_cast<size_t>(c) * K + j];
#pragma unroll
    for (int j = 0; j < K - 1; ++j) {
      const int t = t0 - (K - 1) + j;
      win[j] = t >= 0 ? in[static_cast<size_t>(t) * in_ld + c] : state[static_cast<size_t>(c) * (K - 1) + (t + K - 1)];
    }
  }
  __syncthreads();
  if (c >= C) return;
  constexpr int U = 4;
  int t = t0;
  for (; t + U <= t1; t += U) {
    float x[U];
#pragma unroll
    for (int u = 0; u < U; ++u) x[u] = in[static_cast<size_t>(t + u) * in_ld + c];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      win[K - 1] = x[u];
      float s = 0.0f;
#pragma unroll
      for (int j = 0; j < K; ++j) s += win[j] * wc[j];
      out[static_cast<size_t>(t + u) * out_ld + c] = apply_silu ? silu_k(s) : s;
#pragma unroll
      for (int j = 0; j < K - 1; ++j) win[j] = win[j + 1];
    }
  }
  for (; t < t1; ++t) {
    win[K - 1] = in[static_cast<size_t>(t) * in_ld + c];
    float s = 0.0f;
#pragma unroll
    for (int j = 0; j < K; ++j) s += win[j] * wc[j];
    out[static_cast<size_t>(t) * out_ld + c] = apply_silu ? silu_k(s) : s;
#pragma unroll
    for (int j = 0; j < K - 1; ++j) win[j] = win[j + 1];
  }
  if (t1 == T && t0 < T)
#pragma unroll
    for (int j = 0; j < K - 1; ++j) state[static_cast<size_t>(c) * (K - 1) + j] = win[j];
}

__global__ void prepare_gate_beta_kernel(float* gate, float* beta, const float* bias, const float* scale, int total,
                                         int heads) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= total) return;
  const int c = i % heads;
  gate[i] = softplus20_f(gate[i] + bias[c]) * scale[c];
  beta[i] = sigmoid_f(beta[i]);
}

// Generic delta rule (gated_delta_net_f32_batched_in_place, mps_backend.mm:2225-2305):
// one thread per state row, any head_dim.
__global__ void gdn_generic_kernel(const float* q, const float* k, const float* v, const float* g, const float* beta,
                                   float* state, int T, int key_heads, int value_heads, int d, float* out) {
  const int h = blockIdx.x, row = threadIdx.x + blockIdx.y * blockDim.x;
  if (row >= d) return;
  const int kh = h % key_heads;
  const float scale = 1.0f / sqrtf(static_cast<float>(d));
  float* s = state + (static_cast<size_t>(h) * d + row) * d;
  for (int t = 0; t < T; ++t) {
    const float* kk = k + (static_cast<size_t>(t) * key_heads + kh) * d;
    const float* qq = q + (static_cast<size_t>(t) * key_heads + kh) * d;
    const float ge = expf(g[t * value_heads + h]);
    float sk = 0.0f;
    for (int c = 0; c < d; ++c) {
      s[c] *= ge;
      sk += s[c] * kk[c];
    }
    const float delta = (v[(static_cast<size_t>(t) * value_heads + h) * d + row] - sk) * beta[t * value_heads + h];
    float y = 0.0f;
    for (int c = 0; c < d; ++c) {
      s[c] += kk[c] * delta;
      y += s[c] * qq[c];
    }
    out[(static_cast<size_t>(t) * value_heads + h) * d + row] = y * scale;
  }
}

__global__ void mrope_kernel(float* v, const int* positions, int T, int heads, int hd, int n_dims, int s0, int s1,
                             int s2, int s3, float theta) {
  const int half = n_dims / 2;
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= T * heads * half) return;
  const int pi = idx % half, h = (idx / half) % heads, t = idx / (half * heads);
  const int tot = s0 + s1 + s2 + s3;
  if (tot == 0) return;
  const int sector = pi % tot;
  const int sid = sector < s0 ? 0 : (sector < s0 + s1 ? 1 : (sector < s0 + s1 + s2 ? 2 : 3));
  const float pos = static_cast<float>(positions[t + T * sid]);
  const float freq = 1.0f / powf(theta, static_cast<float>(2 * pi) / static_cast<float>(n_dims));
  float sn, cs;
  sincosf(pos * freq, &sn, &cs);
  float* b = v + (static_cast<size_t>(t) * heads + h) * hd;
  const float x0 = b[pi], x1 = b[half + pi];
  b[pi] = x0 * cs - x1 * sn;
  b[half + pi] = x1 * cs + x0 * sn;
}

// attention_f32_batched_f16_kv (mps_backend.mm:2943-3008): warp per (query, head).
__global__ void attention_generic_kernel(const float* q, const uint16_t* kc, const uint16_t* vc, int start, int T,
                                         int heads, int kv_heads, int hd, int round_q, float* out) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int t = blockIdx.x * 8 + warp, h = blockIdx.y;
  if (t >= T) return;
  const int kvh = h / (heads / kv_heads), kvd = kv_heads * hd;
  const int per = (hd + 31) / 32;
  float qv[8], acc[8];
  for (int i = 0; i < per && i < 8; ++i) {
    const int d = lane + 32 * i;
    const float x = d < hd ? q[(static_cast<size_t>(t) * heads + h) * hd + d] : 0.0f;
    qv[i] = round_q ? round_to_half(x) : x;
    acc[i] = 0.0f;
  }
  const float scale = 1.0f / sqrtf(static_cast<float>(hd));
  float m = -INFINITY, l = 0.0f;
  for (int key = 0; key <= start + t; ++key) {
    float d0 = 0.0f;
    for (int i = 0; i < per && i < 8; ++i) {
      const int d = lane + 32 * i;
      if (d < hd) d0 += qv[i] * half_bits_to_float(kc[static_cast<size_t>(key) * kvd + kvh * hd + d]);
    }
    const float sc = warp_sum(d0) * scale;
    const float nm = fmaxf(m, sc), ps = expf(m - nm), w = expf(sc - nm);
    l = l * ps + w;
    for (int i = 0; i < per && i < 8; ++i) {
      const int d = lane + 32 * i;
      if (d < hd) acc[i] = acc[i] * ps + w * half_bits_to_float(vc[static_cast<size_t>(key) * kvd + kvh * hd + d]);
    }
    m = nm;
  }
  const float inv = l == 0.0f ? 0.0f : 1.0f / l;
  for (int i = 0; i < per && i < 8; ++i) {
    const int d = lane + 32 * i;
    if (d < hd) out[(static_cast<size_t>(t) * heads + h) * hd + d] = acc[i] * inv;
  }
}

__global__ void binary_kernel(int op, float* a, const float* b, size_t n, size_t row) {
  const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n) return;
  switch (op) {
    case 0: a[i] += b[i]; break;
    case 1: a[i] *= b[i]; break;
    case 2: a[i] += b[i % row]; break;
    default: a[i] *= b[i % row]; break;
  }
}

__global__ void unary_kernel(int op, float* v, size_t n) {
  const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const float x = v[i];
  v[i] = op == 0 ? sigmoid_f(x) : (op == 1 ? softplus20_f(x) : silu_k(x));
}

__global__ void silu_mul_kernel(float* g, const float* u, size_t n, __half* out16) {
  pdl_wait();
  pdl_launch_dependents();
  const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (n % 4 == 0 && al16(g) && al16(u) && (!out16 || al8(out16))) {  // float4 per thread
    if (4 * i >= n) return;
    const float4 a = reinterpret_cast<const float4*>(g)[i], b = reinterpret_cast<const float4*>(u)[i];
    const float4 r = make_float4(silu_k(a.x) * b.x, silu_k(a.y) * b.y, silu_k(a.z) * b.z, silu_k(a.w) * b.w);
    reinterpret_cast<float4*>(g)[i] = r;
    if (out16) {
      reinterpret_cast<__half2*>(out16)[2 * i] = __floats2half2_rn(r.x, r.y);
      reinterpret_cast<__half2*>(out16)[2 * i + 1] = __floats2half2_rn(r.z, r.w);
    }
    return;
  }
  if (i < n) {
    g[i] = silu_k(g[i]) * u[i];
    if (out16) out16[i] = __float2half_rn(g[i]);
  }
}

__global__ void copy_rows_kernel(const float* src, float* dst_f, uint16_t* dst_h, size_t rows, size_t rv, size_t ss,
                                 size_t so, size_t ds, size_t dof) {
  const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= rows * rv) return;
  const size_t r = i / rv, c = i % rv;
  const float v = src[r * ss + so + c];
  if (dst_f) dst_f[dof + r * ds + c] = v;
  else dst_h[dof + r * ds + c] = __half_as_ushort(__float2half_rn(v));
}

__global__ void argmax_kernel(const float* v, int n, int* tok, float* prob) {
  __shared__ float bv[256];
  __shared__ int bi[256];
  __shared__ float bs[256];
  const int tid = threadIdx.x;
  float best = -INFINITY;
  int idx = n;
  for (int i = tid; i < n; i += 256)
    if (v[i] > best || (v[i] == best && i < idx)) {
      best = v[i];
      idx = i;
    }
  bv[tid] = best;
  bi[tid] = idx;
  __syncthreads();
  for (int s = 128; s > 0; s >>= 1) {
    if (tid < s) {
      if (bv[tid + s] > bv[tid] || (bv[tid + s] == bv[tid] && bi[tid + s] < bi[tid])) {
        bv[tid] = bv[tid + s];
        bi[tid] = bi[tid + s];
      }
    }
    __syncthreads();
  }
  const float mx = bv[0];
  float sum = 0.0f;
  for (int i = tid; i < n; i += 256) sum += expf(v[i] - mx);
  bs[tid] = sum;
  __syncthreads();
  for (int s = 128; s > 0; s >>= 1) {
    if (tid < s) bs[tid] += bs[tid + s];
    __syncthreads();
  }
  if (tid == 0) {
    *tok = bi[0];
    if (prob) *prob = bs[0] > 0.0f ? 1.0f / bs[0] : 0.0f;
  }
}

unsigned blocks_for(size_t n, unsigned t = 256) { return static_cast<unsigned>((n + t - 1) / t); }

bool kquant_type_ok(int type) { return type == kTypeQ4K || type == kTypeQ5K || type == kTypeQ6K; }

}  // namespace

// ============================================================ GEMV planner
namespace kib {

template <int QT, int NT, bool F16W>
static cudaError_t gemv_instance(const GemvParams& p, int grid, size_t smem, cudaStream_t st) {
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(kquant_gemv_kernel<QT, NT, F16W>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    if (e != cudaSuccess) return e;
    configured = true;
  }
  return launch_pdl(kquant_gemv_kernel<QT, NT, F16W>, dim3(grid), dim3(kGemvThreads), smem, st, p);
}

template <int QT>
static cudaError_t gemv_dispatch(const GemvParams& p, int grid, size_t smem, cudaStream_t st) {
  switch (p.ntok) {
    case 1: return gemv_instance<QT, 1, false>(p, grid, smem, st);
    case 2: return gemv_instance<QT, 2, false>(p, grid, smem, st);
    case 3: return gemv_instance<QT, 3, false>(p, grid, smem, st);
    case 4: return gemv_instance<QT, 4, true>(p, grid, smem, st);  // reductions and epilogues sized to 4
    default: return gemv_instance<QT, 8, true>(p, grid, smem, st);
  }
}

template <int QT, int NT, int PRO>
static cudaError_t gemv2_instance(const GemvParams& p, int grid, size_t smem, cudaStream_t st) {
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(kquant_gemv2_kernel<QT, NT, PRO>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         200 * 1024);
    if (e != cudaSuccess) return e;
    configured = true;
  }
  return launch_pdl(kquant_gemv2_kernel<QT, NT, PRO>, dim3(grid), dim3(kGemvThreads), smem, st, p);
}

template <int QT, int PRO>
static cudaError_t gemv2_dispatch_pro(const GemvParams& p, int grid, size_t smem, cudaStream_t st) {
  switch (p.ntok) {
    case 1: return gemv2_instance<QT, 1, PRO>(p, grid, smem, st);
    case 2: return gemv2_instance<QT, 2, PRO>(p, grid, smem, st);
    default: return gemv2_instance<QT, 3, PRO>(p, grid, smem, st);
  }
}

template <int QT>
static cudaError_t gemv2_dispatch(const GemvParams& p, int grid, size_t smem, cudaStream_t st) {
  switch (p.prologue) {
    case kProRms: return gemv2_dispatch_pro<QT, kProRms>(p, grid, smem, st);
    case kProNormGate: return gemv2_dispatch_pro<QT, kProNormGate>(p, grid, smem, st);
    default: return gemv2_dispatch_pro<QT, kProPlain>(p, grid, smem, st);
  }
}

cudaError_t gemv_launch(const GemvDesc& d, int num_sms, cudaStream_t st, std::string* why) {
  if (!kquant_type_ok(d.type) || d.cols <= 0 || d.cols % 256 || d.cols > 16384 || d.ntok < 1 ||
      d.ntok > kGemvMaxTok || d.nseg < 1 || d.nseg > kGemvMaxSegs) {
    if (why) *why = "GEMV: unsupported type/cols/tokens/segments";
    return cudaErrorInvalidValue;
  }
  GemvParams p = {};
  const int BB = kquant_block_bytes(d.type);
  p.cols = d.cols;
  p.row_bytes = d.cols / 256 * BB;
  const int units = d.cols / 64;
  p.rg = units <= 16 ? 16 : (units <= 32 ? 32 : (units <= 64 ? 64 : (units <= 128 ? 128 : 256)));
  const int groups = kGemvThreads / p.rg;
  const int m = groups > 8 ? groups : 8;
  bool paired = false;
  int total_rows = 0;
  for (int i = 0; i < d.nseg; ++i) {
    total_rows += d.seg[i].rows;
    paired = paired || d.seg[i].epilogue == kEpiSiluMul;
  }
  const int mult = paired ? 2 : 1;
  bool has_conv = false;
  for (int i = 0; i < d.nseg; ++i) has_conv = has_conv || d.seg[i].epilogue == kEpiConv;
  // Two or three tokens (MTP verify) with a norm prologue take the kernel that
  // stages x in shared memory once per CTA: per-lane units would redo the
  // prologue (silu(gate), the RMS sums) once per row group and token.
  const bool compact = d.ntok <= 3 && p.rg <= 128 &&
                       (d.prologue != kProNormGate || (d.ntok == 1 && units == p.rg && d.head_dim == 128)) &&
                       (d.prologue != kProRms || d.ntok == 1) &&
                       (!has_conv || d.conv_k == 4);
  const int km1 = d.conv_k - 1;
  auto count_tiles = [&](int tr) {
    int n = 0;
    for (int i = 0; i < d.nseg; ++i) n += (d.seg[i].rows + tr - 1) / tr;
    return n;
  };
  const int max_stage = 32 * 1024;
  int tr_max = (max_stage / (p.row_bytes * mult)) / m * m;
  if (tr_max < m) tr_max = m;
  int target = (total_rows + num_sms - 1) / num_sms;
  target = (target + m - 1) / m * m;
  int tr = target < tr_max ? target : tr_max;
  if (compact) {
    // one tile per CTA when the matrix fits a single wave of <= 64 KB tiles
    const int cap = ((64 * 1024) / (p.row_bytes * mult)) / m * m;
    int t2 = target;
    while (count_tiles(t2) > num_sms && t2 + m <= cap) t2 += m;
    if (count_tiles(t2) <= num_sms && t2 <= cap) tr = t2;
  }
  p.tile_rows = tr;
  int tiles = 0;
  for (int i = 0; i < d.nseg; ++i) {
    p.seg[i].w = static_cast<const uint8_t*>(d.seg[i].w);
    p.seg[i].w2 = static_cast<const uint8_t*>(d.seg[i].w2);
    p.seg[i].out = d.seg[i].out;
    p.seg[i].rows = d.seg[i].rows;
    p.seg[i].ld = d.seg[i].ld;
    p.seg[i].epilogue = d.seg[i].epilogue;
    p.seg[i].tile_begin = tiles;
    tiles += (d.seg[i].rows + tr - 1) / tr;
  }
  p.nseg = d.nseg;
  p.total_tiles = tiles;
  const int grid = tiles < num_sms ? tiles : num_sms;
  const int half = ((tr * p.row_bytes) + 15) & ~15;
  p.stage_bytes = half * mult;
  p.conv_off = 0;
  if (compact && has_conv && !paired) {
    p.conv_off = p.stage_bytes;
    p.stage_bytes += ((tr * km1 * 4 + 15) & ~15) + ((tr * d.conv_k * 4 + 15) & ~15);
  }
  const int per_cta = (tiles + grid - 1) / grid;
  const bool small_tok = d.ntok <= 3;
  int S = ((small_tok ? 160 : 96) * 1024) / p.stage_bytes;
  if (S < 1) S = 1;
  if (S > per_cta) S = per_cta;
  if (S > 8) S = 8;
  const size_t xs_bytes = compact ? 0 : static_cast<size_t>(d.ntok) * d.cols * sizeof(float);
  while (S > 1 && static_cast<size_t>(S) * p.stage_bytes + xs_bytes > 190 * 1024) --S;
  if (static_cast<size_t>(S) * p.stage_bytes + xs_bytes > 200 * 1024) {
    if (why) *why = "GEMV: shared memory plan exceeds 200 KB";
    return cudaErrorInvalidValue;
  }
  p.stages = S;
  p.ntok = d.ntok;
  p.prologue = d.prologue;
  p.paired = paired ? 1 : 0;
  p.argmax = d.argmax ? 1 : 0;
  p.in = d.in;
  p.in_ld = d.in_ld;
  p.norm_w = d.norm_w;
  p.eps = d.eps;
  p.gate = d.gate;
  p.head_dim = d.head_dim;
  p.resid = d.resid;
  p.conv_state = d.conv_state;
  p.conv_w = d.conv_w;
  p.conv_k = d.conv_k;
  p.cand_max = d.cand_max;
  p.cand_sum = d.cand_sum;
  p.cand_idx = d.cand_idx;
  p.counter = d.counter;
  p.token_out = d.token_out;
  p.prob_out = d.prob_out;
  p.token_log = d.token_log;
  p.step_counter = d.step_counter;
  p.pos_advance = d.pos_advance;
  p.x_out = d.x_out;
  p.err = d.err;
  p.trace = d.trace;
  const size_t smem = static_cast<size_t>(S) * p.stage_bytes + xs_bytes;
  if (compact) {
    switch (d.type) {
      case kTypeQ4K: return gemv2_dispatch<kTypeQ4K>(p, grid, smem, st);
      case kTypeQ5K: return gemv2_dispatch<kTypeQ5K>(p, grid, smem, st);
      default: return gemv2_dispatch<kTypeQ6K>(p, grid, smem, st);
    }
  }
  switch (d.type) {
    case kTypeQ4K: return gemv_dispatch<kTypeQ4K>(p, grid, smem, st);
    case kTypeQ5K: return gemv_dispatch<kTypeQ5K>(p, grid, smem, st);
    default: return gemv_dispatch<kTypeQ6K>(p, grid, smem, st);
  }
}

// M > 8: half-precision GEMM path.
cudaError_t gemm_f16_launch(int type, const void* w, int rows, int cols, const float* x, int x_ld, int T, float* y,
                            int y_ld, const float* resid, cudaStream_t st) {
  GemmParams p;
  p.w = static_cast<const uint8_t*>(w);
  p.rows = rows;
  p.cols = cols;
  p.x = x;
  p.x_ld = x_ld;
  p.T = T;
  p.y = y;
  p.y_ld = y_ld;
  p.resid = resid;
  const size_t smem = kGemmSmem;
  dim3 grid((rows + kGemmTileM - 1) / kGemmTileM, (T + kGemmTileN - 1) / kGemmTileN);
  static bool cfg[3] = {false, false, false};
  switch (type) {
    case kTypeQ4K:
      if (!cfg[0]) { cudaFuncSetAttribute(kquant_gemm_f16_kernel<kTypeQ4K>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)); cfg[0] = true; }
      return launch_pdl(kquant_gemm_f16_kernel<kTypeQ4K>, grid, dim3(256), smem, st, p);
    case kTypeQ5K:
      if (!cfg[1]) { cudaFuncSetAttribute(kquant_gemm_f16_kernel<kTypeQ5K>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)); cfg[1] = true; }
      return launch_pdl(kquant_gemm_f16_kernel<kTypeQ5K>, grid, dim3(256), smem, st, p);
    default:
      if (!cfg[2]) { cudaFuncSetAttribute(kquant_gemm_f16_kernel<kTypeQ6K>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)); cfg[2] = true; }
      return launch_pdl(kquant_gemm_f16_kernel<kTypeQ6K>, grid, dim3(256), smem, st, p);
  }
}

template <int BM, int BN, int WR, int WC>
static cudaError_t gemm_f16w_tile(const GemmF16Params& p, cudaStream_t st) {
  static bool cfg = false;
  constexpr size_t smem = gemm_f16w_smem<BM, BN>();
  if (!cfg) {
    const cudaError_t e =
        cudaFuncSetAttribute(gemm_f16w_kernel<BM, BN, WR, WC>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    cfg = true;
  }
  return launch_pdl(gemm_f16w_kernel<BM, BN, WR, WC>, dim3((p.rows + BM - 1) / BM, (p.T + BN - 1) / BN),
                    dim3(32 * WR * WC), smem, st, p);
}

cudaError_t kquant_to_f16_launch(int type, const void* w, int rows, int cols, __half* out, int num_sms,
                                 cudaStream_t st) {
  if (cols % 256 != 0) return cudaErrorInvalidValue;
  const uint8_t* wb = static_cast<const uint8_t*>(w);
  const size_t units = static_cast<size_t>(rows) * (cols / 256) * 4;
  const int grid = static_cast<int>(std::min<size_t>((units + 255) / 256, static_cast<size_t>(num_sms) * 8));
  switch (type) {
    case kTypeQ4K: return launch_pdl(kquant_to_f16_kernel<kTypeQ4K>, dim3(grid), dim3(256), 0, st, wb, rows, cols, out);
    case kTypeQ5K: return launch_pdl(kquant_to_f16_kernel<kTypeQ5K>, dim3(grid), dim3(256), 0, st, wb, rows, cols, out);
    default: return launch_pdl(kquant_to_f16_kernel<kTypeQ6K>, dim3(grid), dim3(256), 0, st, wb, rows, cols, out);
  }
}

// Prefill GEMM on f16 operands.  w16_resident: the weight's f16 copy made at
// load (nullptr: dequantize into the w16 scratch, rows * cols halves, now).
// convert_x false: x16 (T * cols halves) already holds this x, because the
// previous GEMM read the same input.  The tile is the largest that still
// fills two CTA slots per SM; the two smaller tiles run four warps each.
// ---- tcgen05 GEMM host side: 2-D tensor maps over row-major f16 matrices
namespace tc_host {
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      f = nullptr;
    return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
  }();
  return fn;
}

// [rows][cols] halves, boxes of box_rows x 64 columns, 128-byte swizzle,
// out-of-range rows read as zeros.
bool f16_tensor_map(CUtensorMap* map, const __half* base, int rows, int cols, int box_rows) {
  auto enc = tensor_map_encoder();
  if (!enc || (reinterpret_cast<uintptr_t>(base) & 15u) || (cols * 2) % 16) return false;
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(cols) * 2};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(kTcBK), static_cast<cuuint32_t>(box_rows)};
  const cuuint32_t estr[2] = {1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half*>(base), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool gemm_tc_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("KIB_GEMM_TC");
    return !(v && v[0] == '0');
  }();
  return on;
}

bool gemm_tc_persist_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("KIB_GEMM_TC_PERSIST");
    return !(v && v[0] == '0');
  }();
  return on;
}

template <int BN>
cudaError_t gemm_tc_persist_launch(const __half* w16, const __half* x16, const GemmTcParams& p, int num_sms,
                                   cudaStream_t st) {
  CUtensorMap wm, xm;
  if (!f16_tensor_map(&wm, w16, p.rows, p.cols, kTcBM) || !f16_tensor_map(&xm, x16, p.T, p.cols, BN))
    return cudaErrorInvalidValue;
  static bool cfg = false;
  constexpr size_t smem = gemm_tc_persist_smem<BN>();
  if (!cfg) {
    const cudaError_t e = cudaFuncSetAttribute(gemm_tc_persist_kernel<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    cfg = true;
  }
  const int tiles = ((p.rows + kTcBM - 1) / kTcBM) * ((p.T + BN - 1) / BN);
  return launch_pdl(gemm_tc_persist_kernel<BN>, dim3(std::min(tiles, num_sms)), dim3(kTcThreads), smem, st, wm, xm, p);
}

template <int BN>
cudaError_t gemm_tc_launch(const __half* w16, const __half* x16, const GemmTcParams& p, cudaStream_t st) {
  CUtensorMap wm, xm;
  if (!f16_tensor_map(&wm, w16, p.rows, p.cols, kTcBM) || !f16_tensor_map(&xm, x16, p.T, p.cols, BN))
    return cudaErrorInvalidValue;
  static bool cfg = false;
  constexpr size_t smem = gemm_tc_smem<BN>();
  if (!cfg) {
    const cudaError_t e =
        cudaFuncSetAttribute(gemm_tc_kernel<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    cfg = true;
  }
  return launch_pdl(gemm_tc_kernel<BN>, dim3((p.rows + kTcBM - 1) / kTcBM, (p.T + BN - 1) / BN), dim3(kTcThreads),
                    smem, st, wm, xm, p);
}
}  // namespace tc_host

namespace skinny_host {
template <int QT, int NT>
cudaError_t launch(const SkinnyParams& p, dim3 grid, cudaStream_t st) {
  static bool cfg = false;
  constexpr size_t smem = kq_skinny_smem<NT>();
  if (!cfg) {
    const cudaError_t e = cudaFuncSetAttribute(kq_skinny_gemm_kernel<QT, NT>,
                                               cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    cfg = true;
  }
  if (p.cluster && grid.y > 1)
    return launch_pdl_cluster(kq_skinny_gemm_kernel<QT, NT>, grid, dim3(128), smem, st, dim3(1, grid.y, 1), p);
  return launch_pdl(kq_skinny_gemm_kernel<QT, NT>, grid, dim3(128), smem, st, p);
}
template <int QT>
cudaError_t launch_t(const SkinnyParams& p, dim3 grid, cudaStream_t st) {
  if (p.xrows <= 16) return launch<QT, 2>(p, grid, st);
  if (p.xrows <= 32) return launch<QT, 4>(p, grid, st);
  return launch<QT, 8>(p, grid, st);
}
}  // namespace skinny_host

// Few-token M > 8 projection straight from the K-quant blocks (kq_skinny.cuh).
// Split-K over the super-blocks when the 64-row tiles alone give fewer than
// two CTAs per SM; the partials (ws, nsplit * T * rows floats) are then summed
// in split order by a second kernel.
cudaError_t kq_skinny_launch(int type, const void* w, int rows, int cols, const __half* x16, int T, float* y,
                             int y_ld, const float* resid, float* ws, int num_sms, cudaStream_t st, bool xsplit) {
  static const bool cluster_on = [] {
    const char* v = std::getenv("KIB_SKINNY_CLUSTER");
    return !(v && v[0] == '0');
  }();
  const int bpr = cols / 256;
  const int tiles = (rows + kSkRows - 1) / kSkRows;
  int nsplit = std::min(bpr, std::max(1, (2 * num_sms + tiles - 1) / tiles));
  const int kps = (bpr + nsplit - 1) / nsplit;
  nsplit = (bpr + kps - 1) / kps;
  SkinnyParams p;
  p.w = static_cast<const uint8_t*>(w);
  p.rows = rows;
  p.cols = cols;
  p.T = T;
  p.row_bytes = bpr * kquant_block_bytes(type);
  p.x = x16;
  p.y = y;
  p.y_ld = y_ld;
  p.resid = resid;
  p.ws = ws;
  p.kb_per_split = kps;
  p.xsplit = xsplit ? 1 : 0;
  p.xrows = xsplit ? 16 : T;
  // the 4..8-token bucket (MTP verify) reduces its splits inside one portable
  // cluster through shared memory (measured ~1 % faster there); elsewhere the
  // workspace and the reduce kernel win (batched decode, 32 tokens: 2.65 ms a
  // step against 2.71 ms with clusters, whose co-scheduling leaves SMs idle)
  const bool cluster = cluster_on && xsplit && nsplit <= 8;
  p.cluster = cluster ? 1 : 0;
  const dim3 grid(tiles, nsplit);
  cudaError_t e;
  switch (type) {
    case kTypeQ4K: e = skinny_host::launch_t<kTypeQ4K>(p, grid, st); break;
    case kTypeQ5K: e = skinny_host::launch_t<kTypeQ5K>(p, grid, st); break;
    default: e = skinny_host::launch_t<kTypeQ6K>(p, grid, st); break;
  }
  if (e != cudaSuccess || nsplit == 1 || cluster) return e;
  const size_t n = static_cast<size_t>(T) * rows;
  const int rg = static_cast<int>(std::min<size_t>((n + 255) / 256, static_cast<size_t>(num_sms) * 4));
  return launch_pdl(kq_skinny_reduce_kernel, dim3(rg), dim3(256), 0, st, static_cast<const float*>(ws), nsplit, rows, T,
                    y, y_ld, resid);
}

cudaError_t gemm_f16w_launch(int type, const void* w, const __half* w16_resident, int rows, int cols, const float* x,
                             int x_ld, int T, float* y, int y_ld, const float* resid, __half* w16, __half* x16,
                             bool convert_x, int num_sms, cudaStream_t st, int* err) {
  if (cols % kGfK != 0 || x_ld % 4 != 0) return cudaErrorInvalidValue;
  cudaError_t e;
  static const bool skinny_on = [] {
    const char* v = std::getenv("KIB_GEMM_SKINNY");
    return !(v && v[0] == '0');
  }();
  if (T >= 4 && T <= 8 && cols % 256 == 0 && kquant_type_ok(type) && w16 != nullptr) {
    // the reference's 4..8-token bucket: half weights against fp32 x, as x's
    // high and low halves on the tensor cores
    if (convert_x) {
      const size_t xn = static_cast<size_t>(8) * cols;
      const int x_grid = static_cast<int>(std::min<size_t>((xn + 255) / 256, static_cast<size_t>(num_sms) * 4));
      e = launch_pdl(x_split_f16_kernel, dim3(x_grid), dim3(256), 0, st, x, x_ld, T, cols, x16);
      if (e != cudaSuccess) return e;
    }
    return kq_skinny_launch(type, w, rows, cols, x16, T, y, y_ld, resid, reinterpret_cast<float*>(w16), num_sms, st,
                            true);
  }
  if (skinny_on && T > 8 && T <= 64 && cols % 256 == 0 && kquant_type_ok(type) && w16 != nullptr) {
    // few tokens: dequantise the K-quant blocks in shared memory instead of
    // streaming the f16 copy (same products); w16's scratch holds the split-K
    // partials
    if (convert_x) {
      const size_t xn = static_cast<size_t>(T) * (cols / 4);
      const int x_grid = static_cast<int>(std::min<size_t>((xn + 255) / 256, static_cast<size_t>(num_sms) * 8));
      e = launch_pdl(x_to_f16_kernel, dim3(x_grid), dim3(256), 0, st, x, x_ld, T, cols, x16);
      if (e != cudaSuccess) return e;
    }
    return kq_skinny_launch(type, w, rows, cols, x16, T, y, y_ld, resid, reinterpret_cast<float*>(w16), num_sms, st,
                            false);
  }
  if (!w16_resident) {
    e = kquant_to_f16_launch(type, w, rows, cols, w16, num_sms, st);
    if (e != cudaSuccess) return e;
  }
  if (convert_x) {
    const size_t xn = static_cast<size_t>(T) * (cols / 4);
    const int x_grid = static_cast<int>(std::min<size_t>((xn + 255) / 256, static_cast<size_t>(num_sms) * 8));
    e = launch_pdl(x_to_f16_kernel, dim3(x_grid), dim3(256), 0, st, x, x_ld, T, cols, x16);
    if (e != cudaSuccess) return e;
  }
  const __half* wsrc = w16_resident ? w16_resident : w16;
  if (tc_host::gemm_tc_enabled() && rows >= kTcBM && T >= 128 && cols % kTcBK == 0) {
    // tcgen05 path; the mma.sync tiles below remain for small or unaligned cases
    GemmTcParams tp;
    tp.rows = rows;
    tp.cols = cols;
    tp.T = T;
    tp.y = y;
    tp.y_ld = y_ld;
    tp.resid = resid;
    tp.err = err;
    static const int tc_bn = [] {
      const char* v = std::getenv("KIB_GEMM_TC_BN");
      return v && std::atoi(v) == 256 ? 256 : 128;
    }();
    // tile width by the cost model rounds x width: 64-token tiles when they
    // halve the rounds (narrow matrices whose 128-wide tiles leave SMs idle)
    const int mt = (rows + kTcBM - 1) / kTcBM;
    const int r128 = (mt * ((T + 127) / 128) + num_sms - 1) / num_sms, r64 = (mt * ((T + 63) / 64) + num_sms - 1) / num_sms;
    if (!tc_host::gemm_tc_persist_enabled()) e = tc_host::gemm_tc_launch<128>(wsrc, x16, tp, st);
    else if (tc_bn == 256 && T >= 256) e = tc_host::gemm_tc_persist_launch<256>(wsrc, x16, tp, num_sms, st);
    else if (64 * r64 < 128 * r128) e = tc_host::gemm_tc_persist_launch<64>(wsrc, x16, tp, num_sms, st);
    else e = tc_host::gemm_tc_persist_launch<128>(wsrc, x16, tp, num_sms, st);
    if (e != cudaErrorInvalidValue) return e;
    cudaGetLastError();
  }
  GemmF16Params p;
  p.w = wsrc;
  p.x = x16;
  p.rows = rows;
  p.cols = cols;
  p.T = T;
  p.y = y;
  p.y_ld = y_ld;
  p.resid = resid;
  auto ctas = [&](int bm, int bn) { return ((rows + bm - 1) / bm) * ((T + bn - 1) / bn); };
  const int fill = 2 * num_sms;
  if (ctas(128, 128) >= fill) return gemm_f16w_tile<128, 128, 2, 4>(p, st);
  if (ctas(128, 64) >= fill) return gemm_f16w_tile<128, 64, 2, 2>(p, st);
  // few tokens (batched decode, short chunks): 32 x 32 tiles on two warps give
  // 4x the CTAs of 64 x 64, so narrow matrices still spread over the SMs
  if (T <= 32) return gemm_f16w_tile<32, 32, 2, 1>(p, st);
  return gemm_f16w_tile<64, 64, 2, 2>(p, st);  // 4 warps of 32 x 32, up to four CTAs per SM
}

cudaError_t get_rows_launch(int type, const void* w, int nrows, int cols, const int* ids, int T, float* out,
                            int out_ld, cudaStream_t st) {
  const uint8_t* wb = static_cast<const uint8_t*>(w);
  switch (type) {
    case kTypeQ4K: return launch_pdl(get_rows_kernel<kTypeQ4K>, dim3(T), dim3(64), 0, st, wb, nrows, cols, ids, out, out_ld);
    case kTypeQ5K: return launch_pdl(get_rows_kernel<kTypeQ5K>, dim3(T), dim3(64), 0, st, wb, nrows, cols, ids, out, out_ld);
    default: return launch_pdl(get_rows_kernel<kTypeQ6K>, dim3(T), dim3(64), 0, st, wb, nrows, cols, ids, out, out_ld);
  }
}

cudaError_t rms_rows_launch(const float* in, const float* w, int T, int n, float eps, float* out, cudaStream_t st,
                            __half* out16 = nullptr) {
  return launch_pdl(rms_norm_rows_kernel, dim3(T), dim3(256), 0, st, in, w, n, eps, out, out16);
}

cudaError_t norm_gate_launch(float* v, const float* w, const float* gate, int T, int heads, int d, float eps, float* out,
                             cudaStream_t st, __half* out16 = nullptr, int gate_ld = 0) {
  return launch_pdl(head_norm_kernel, dim3((heads + 3) / 4, T), dim3(128), 0, st, v, w, gate, heads, d, eps, out,
                    out16, gate_ld);
}

cudaError_t conv_launch(float* state, const float* in, int in_ld, const float* w, int K, int C, int T, float* out,
                        int out_ld, int silu, cudaStream_t st) {
  // conv_stateful_kernel keeps the window in 16-entry register arrays
  if (K < 1 || K > 16) return cudaErrorInvalidValue;
  // tiles of >= 16 tokens, at most 32 per CTA (32 x 32 threads)
  const int ntiles = T >= 512 ? 32 : (T + 15) / 16;
  if (K == 4)
    return launch_pdl(conv_stateful_k_kernel<4>, dim3((C + 31) / 32), dim3(32, ntiles), 0, st, state, in, in_ld, w, C, T,
                      out, out_ld, silu);
  return launch_pdl(conv_stateful_kernel, dim3((C + 31) / 32), dim3(32, ntiles), 0, st, state, in, in_ld, w, K, C, T, out,
                    out_ld, silu);
}

// act[t][i] = silu(gu[t][i]) * gu[t][I + i] over a [T][2I] gate | up buffer
// (one GEMM over the concatenated weights); also in half for the next GEMM.
__global__ void silu_mul_cat_kernel(const float* gu, int I, size_t n4, float* act, __half* out16) {
  pdl_wait();
  pdl_launch_dependents();
  const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;  // float4 of act
  if (i >= n4) return;
  const size_t t = (4 * i) / I, c = (4 * i) % I;
  const float4 a = *reinterpret_cast<const float4*>(gu + t * 2 * I + c);
  const float4 b = *reinterpret_cast<const float4*>(gu + t * 2 * I + I + c);
  const float4 r = make_float4(silu_k(a.x) * b.x, silu_k(a.y) * b.y, silu_k(a.z) * b.z, silu_k(a.w) * b.w);
  reinterpret_cast<float4*>(act)[i] = r;
  if (out16) {
    reinterpret_cast<__half2*>(out16)[2 * i] = __floats2half2_rn(r.x, r.y);
    reinterpret_cast<__half2*>(out16)[2 * i + 1] = __floats2half2_rn(r.z, r.w);
  }
}

cudaError_t silu_mul_cat_launch(const float* gu, int T, int I, float* act, cudaStream_t st, __half* out16) {
  if (I % 4 || reinterpret_cast<uintptr_t>(gu) % 16 || reinterpret_cast<uintptr_t>(act) % 16 ||
      reinterpret_cast<uintptr_t>(out16) % 8)
    return cudaErrorInvalidValue;
  const size_t n4 = static_cast<size_t>(T) * I / 4;
  return launch_pdl(silu_mul_cat_kernel, dim3(blocks_for(n4)), dim3(256), 0, st, gu, I, n4, act, out16);
}

cudaError_t silu_mul_launch(float* g, const float* u, size_t n, cudaStream_t st, __half* out16 = nullptr) {
  const bool vec = n % 4 == 0 && (reinterpret_cast<uintptr_t>(g) | reinterpret_cast<uintptr_t>(u)) % 16 == 0 &&
                   reinterpret_cast<uintptr_t>(out16) % 8 == 0;
  const size_t threads = vec ? n / 4 : n;
  return launch_pdl(silu_mul_kernel, dim3(blocks_for(threads)), dim3(256), 0, st, g, u, n, out16);
}

int finish_op(kib_ctx* ctx, const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return check_cuda(ctx, e, what);
  if (ctx->in_graph) return KIB_OK;
  e = cudaStreamSynchronize(ctx->stream);
  if (e != cudaSuccess) return check_cuda(ctx, e, what);
  int err = 0;
  cudaMemcpy(&err, ctx->d_err, sizeof(int), cudaMemcpyDeviceToHost);
  if (err != 0) {
    cudaMemset(ctx->d_err, 0, sizeof(int));
    return set_error(ctx, KIB_ERR_TIMEOUT, std::string(what) + ": a bounded device wait gave up");
  }
  return KIB_OK;
}

}  // namespace kib

// =============================================================== C ABI

extern "C" {

int kib_create(int device, kib_ctx** out) {
  if (!out) return KIB_ERR_INVALID_ARGUMENT;
  *out = nullptr;
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || n <= device || device < 0) return KIB_ERR_UNAVAILABLE;
  auto* ctx = new kib_ctx;
  ctx->device = device;
  cudaSetDevice(device);
  cudaDeviceGetAttribute(&ctx->num_sms, cudaDevAttrMultiProcessorCount, device);
  int major = 0;
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device);
  if (major < 10) {
    delete ctx;
    return KIB_ERR_UNAVAILABLE;
  }
  if (cudaStreamCreateWithFlags(&ctx->stream, cudaStreamNonBlocking) != cudaSuccess ||
      cudaMalloc(&ctx->d_err, sizeof(int)) != cudaSuccess ||
      cudaMalloc(&ctx->d_cand_max, sizeof(float) * 1024 * kGemvMaxTok) != cudaSuccess ||
      cudaMalloc(&ctx->d_cand_sum, sizeof(float) * 1024 * kGemvMaxTok) != cudaSuccess ||
      cudaMalloc(&ctx->d_cand_idx, sizeof(int) * 1024 * kGemvMaxTok) != cudaSuccess ||
      cudaMalloc(&ctx->d_counter, sizeof(unsigned)) != cudaSuccess) {
    kib_destroy(ctx);
    return KIB_ERR_INTERNAL;
  }
  cudaMemset(ctx->d_err, 0, sizeof(int));
  cudaMemset(ctx->d_counter, 0, sizeof(unsigned));
  *out = ctx;
  return KIB_OK;
}

void kib_destroy(kib_ctx* ctx) {
  if (!ctx) return;
  if (ctx->stream) cudaStreamSynchronize(ctx->stream);
  cudaFree(ctx->d_err);
  cudaFree(ctx->d_cand_max);
  cudaFree(ctx->d_cand_sum);
  cudaFree(ctx->d_cand_idx);
  cudaFree(ctx->d_counter);
  if (ctx->stream) cudaStreamDestroy(ctx->stream);
  delete ctx;
}

int kib_valid(const kib_ctx* ctx) { return ctx && ctx->stream ? 1 : 0; }
const char* kib_last_error(const kib_ctx* ctx) { return ctx ? ctx->last_error.c_str() : "no context"; }
void* kib_stream(kib_ctx* ctx) { return ctx ? static_cast<void*>(ctx->stream) : nullptr; }

int kib_begin_graph(kib_ctx* ctx) {
  KIB_REQUIRE_CTX(ctx);
  KIB_ARG(!ctx->in_graph, "graph scope already open");
  ctx->in_graph = true;
  return KIB_OK;
}
int kib_commit_graph(kib_ctx* ctx) {
  KIB_REQUIRE_CTX(ctx);
  KIB_ARG(ctx->in_graph, "no graph scope is open");
  ctx->in_graph = false;
  return finish_op(ctx, "commit_graph");
}
int kib_abort_graph(kib_ctx* ctx) {
  KIB_REQUIRE_CTX(ctx);
  ctx->in_graph = false;
  cudaStreamSynchronize(ctx->stream);
  return KIB_OK;
}

int kib_make_buffer(kib_ctx* ctx, uint64_t bytes, void** dev_out) {
  KIB_REQUIRE_CTX(ctx);
  KIB_ARG(dev_out && bytes > 0, "make_buffer: size must be positive");
  // 256 bytes of tail padding: bulk weight copies round their size up to 16.
  return check_cuda(ctx, cudaMalloc(dev_out, bytes + 256), "make_buffer");
}
int kib_free_buffer(kib_ctx* ctx, void* dev) {
  KIB_REQUIRE_CTX(ctx);
  cudaStreamSynchronize(ctx->stream);
  return check_cuda(ctx, cudaFree(dev), "free_buffer");
}
int kib_copy_to_buffer(kib_ctx* ctx, void* dst, uint64_t off, const void* src, uint64_t bytes) {
  KIB_REQUIRE_CTX(ctx);
  KIB_ARG(dst && src, "copy_to_buffer: null pointer");
  cudaError_t e = cudaMemcpyAsync(static_cast<uint8_t*>(dst) + off, src, bytes, cudaMemcpyHostToDevice, ctx->stream);
  if (e != cudaSuccess) return check_cuda(ctx, e, "copy_to_buffer");
  return finish_op(ctx, "copy_to_buffer");
}
int kib_copy_from_buffer(kib_ctx* ctx, const void* src, uint64_t off, void* dst, uint64_t bytes) {
  KIB_REQUIRE_CTX(ctx);
  KIB_ARG(dst && src, "copy_from_buffer: null pointer");
  cudaError_t e =
      cudaMemcpyAsync(dst, static_cast<const uint8_t*>(src) + off, bytes, cudaMemcpyDeviceToHost, ctx->stream);
  if (e != cudaSuccess) return check_cuda(ctx, e, "copy_from_buffer");
  return check_cuda(ctx, cudaStreamSynchronize(ctx->stream), "copy_from_buffer");
}
int kib_copy_buffer_region(kib_ctx* ctx, const void* src, void* dst, uint64_t so, uint64_t dof, uint64_t bytes) {
  KIB_REQUIRE_CTX(ctx);
  KIB_ARG(dst && src, "copy_buffer_region: null pointer");
  cudaError_t e = cudaMemcpyAsync(static_cast<uint8_t*>(dst) + dof, static_cast<const uint8_t*>(src) + so, bytes,
                                  cudaMemcpyDeviceToDevice, ctx->stream);
  if (e != cudaSuccess) return check_cuda(ctx, e, "copy_buffer_region");
  return finish_op(ctx, "copy_buffer_region");
}
int kib_zero_buffer(kib_ctx* ctx, void* dev, uint64_t bytes) {
  KIB_REQUIRE_CTX(ctx);
  KIB_ARG(dev, "zero_buffer: null pointer");
  cudaError_t e = cudaMemsetAsync(dev, 0, bytes, ctx->stream);
  if (e != cudaSuccess) return check_cuda(ctx, e, "zero_buffer");
  return finish_op(ctx, "zero_buffer");
}

// ---- K-quant
static int kquant_shape_check(kib_ctx* ctx, int type, const void* w, uint64_t rows, uint64_t cols, uint64_t tokens) {
  KIB_ARG(kquant_type_ok(type), "K-quant op: type must be Q4_K(12), Q5_K(13) or Q6_K(14)");
  KIB_ARG(w, "K-quant op: weight buffer is not initialized");
  KIB_ARG(rows > 0 && cols > 0 && tokens > 0, "K-quant op: dimensions must be positive");
  KIB_ARG(cols % 256 == 0, "K-quant op: cols must be a multiple of 256");
  KIB_ARG(rows < (1ull << 31) && cols <= 16384 && tokens < (1ull << 31), "K-quant op: dimensions exceed limits");
  return KIB_OK;
}

int kib_matmul_kquant_f32(kib_ctx* ctx, int type, const void* w, uint64_t rows, uint64_t cols, uint64_t tokens,
                          const float* input, float* output) {
  KIB_REQUIRE_CTX(ctx);
  int st = kquant_shape_check(ctx, type, w, rows, cols, tokens);
  if (st) return st;
  KIB_ARG(input && output, "K-quant matmul: null input/output");
  cudaError_t e;
  if (tokens <= 8) {
    GemvDesc d;
    d.type = type;
    d.cols = static_cast<int>(cols);
    d.ntok = static_cast<int>(tokens);
    d.nseg = 1;
    d.seg[0].w = w;
    d.seg[0].out = output;
    d.seg[0].rows = static_cast<int>(rows);
    d.seg[0].ld = static_cast<int>(rows);
    d.in = input;
    d.in_ld = static_cast<int>(cols);
    d.err = ctx->d_err;
    std::string why;
    e = gemv_launch(d, ctx->num_sms, ctx->stream, &why);
    if (e != cudaSuccess) return set_error(ctx, KIB_ERR_INTERNAL, "matmul: " + why + " " + cudaGetErrorString(e));
  } else {
    e = gemm_f16_launch(type, w, static_cast<int>(rows), static_cast<int>(cols), input, static_cast<int>(cols),
                        static_cast<int>(tokens), output, static_cast<int>(rows), nullptr, ctx->stream);
    if (e != cudaSuccess) return check_cuda(ctx, e, "matmul");
  }
  return finish_op(ctx, "matmul_kquant");
}

int kib_matvec_kquant_f32(kib_ctx* ctx, int type, const void* w, uint64_t rows, uint64_t cols, const float* in,
                          float* out) {
  return kib_matmul_kquant_f32(ctx, type, w, rows, cols, 1, in, out);
}

int kib_matvec_kquant_f32_argmax(kib_ctx* ctx, int type, const void* w, uint64_t rows, uint64_t cols,
                                 const float* input, int32_t* token_out, float* prob_out) {
  KIB_REQUIRE_CTX(ctx);
  int st = kquant_shape_check(ctx, type, w, rows, cols, 1);
  if (st) return st;
  KIB_ARG(input && token_out, "K-quant argmax: null input/output");
  GemvDesc d;
  d.type = type;
  d.cols = static_cast<int>(cols);
  d.ntok = 1;
  d.nseg = 1;
  d.seg[0].w = w;
  d.seg[0].out = nullptr;
  d.seg[0].rows = static_cast<int>(rows);
  d.seg[0].ld = static_cast<int>(rows);
  d.seg[0].epilogue = kEpiArgmax;
  d.in = input;
  d.in_ld = static_cast<int>(cols);
  d.argmax = true;
  d.cand_max = ctx->d_cand_max;
  d.cand_sum = ctx->d_cand_sum;
  d.cand_idx = ctx->d_cand_idx;
  d.counter = ctx->d_counter;
  d.token_out = token_out;
  d.prob_out = prob_out;
  d.err = ctx->d_err;
  std::string why;
  cudaError_t e = gemv_launch(d, ctx->num_sms, ctx->stream, &why);
  if (e != cudaSuccess) return set_error(ctx, KIB_ERR_INTERNAL, "argmax: " + why + " " + cudaGetErrorString(e));
  return finish_op(ctx, "matvec_argmax");
}

int kib_dequantize_rows_kquant_f32(kib_ctx* ctx, int type, const void* w, uint64_t rows, const int32_t* ids,
                                   uint64_t count, uint64_t cols, float* out) {
  KIB_REQUIRE_CTX(ctx);
  int st = kquant_shape_check(ctx, type, w, rows, cols, count);
  if (st) return st;
  KIB_ARG(ids && out, "dequantize_rows: null ids/output");
  cudaError_t e = get_rows_launch(type, w, static_cast<int>(rows), static_cast<int>(cols), ids,
                                  static_cast<int>(count), out, static_cast<int>(cols), ctx->stream);
  if (e != cudaSuccess) return check_cuda(ctx, e, "dequantize_rows");
  return finish_op(ctx, "dequantize_rows");
}

#define KIB_NAMED(q, T)                                                                                     \
  int kib_matvec_##q##_f32_device(kib_ctx* ctx, const void* w, uint64_t r, uint64_t c, const float* i,      \
                                  float* o) {                                                              \
    return kib_matvec_kquant_f32(ctx, T, w, r, c, i, o);                                                    \
  }                                                                                                         \
  int kib_matmul_##q##_f32_device(kib_ctx* ctx, const void* w, uint64_t r, uint64_t c, uint64_t t,          \
                                  const float* i, float* o) {                                              \
    return kib_matmul_kquant_f32(ctx, T, w, r, c, t, i, o);                                                 \
  }
KIB_NAMED(q4_k, 12)
KIB_NAMED(q5_k, 13)
KIB_NAMED(q6_k, 14)

// ---- norms
int kib_rms_norm_f32_f32_batched(kib_ctx* ctx, const float* in, const float* w, uint64_t tokens, uint64_t size,
                                 float eps, float* out) {
  KIB_REQUIRE_CTX(ctx);
  KIB_ARG(in && w && out && tokens > 0 && size > 0, "rms_norm: invalid arguments");
  cudaError_t e = rms_rows_launch(in, w, static_cast<int>(tokens), static_cast<int>(size), eps, out, ctx->stream);
  if (e != cudaSuccess) return check_cuda(ctx, e, "rms_norm");
  return finish_op(ctx, "rms_norm");
}
int kib_qk_norm_f32_f32_batched(kib_ctx* ctx, float* v, const float* w, uint64_t tokens, uint64_t heads,
                                uint64_t hd, float eps) {
  KIB_REQUIRE_CTX(ctx);
  KIB_ARG(v && w && tokens && heads && hd, "qk_norm: invalid arguments");
  cudaError_t e = norm_gate_launch(v, w, nullptr, static_cast<int>(tokens), static_cast<int>(heads),
                                   static_cast<int>(hd), eps, nullptr, ctx->stream);
  if (e != cudaSuccess) return check_cuda(ctx, e, "qk_norm");
  return finish_op(ctx, "qk_norm");
}
int kib_qwen35_norm_gated_f32_in_place(kib_ctx* ctx, float* v, const float* w, const float* gate, uint64_t tokens,
                                       uint64_t heads, uint64_t hd, float eps) {
  KIB_REQUIRE_CTX(ctx);
  KIB_ARG(v && w && gate && tokens && heads && hd, "norm_gated: invalid arguments");
  cudaError_t e = norm_gate_launch(v, w, gate, static_cast<int>(tokens), static_cast<int>(heads),
                                   static_cast<int>(hd), eps, nullptr, ctx->stream);
  if (e != cudaSuccess) return check_cuda(ctx, e, "norm_gated");
  return finish_op(ctx, "norm_gated");
}
int kib_split_qkv_l2_norm_f32_qwen35(kib_ctx* ctx, const float* src, float* q, float* k, float* v, uint64_t tokens,
                                     uint64_t kh, uint64_t vh, uint64_t hd, float eps) {
  KIB_REQUIRE_CTX(ctx);
  KIB_ARG(src && q && k && v && tokens && kh && vh && hd, "split_qkv_l2_norm: invalid arguments");
  const unsigned hmax = static_cast<unsigned>(kh > vh ? kh : vh);
  split_qkv_l2_kernel<<<dim3(hmax, static_cast<unsigned>(tokens), 3), 32, 0, ctx->stream>>>(
      src, q, k, v, static_cast<int>(kh), static_cast<int>(vh), static_cast<int>(hd), eps);
  return finish_op(ctx, "split_qkv_l2_norm");
}

// ---- GDN pieces
int kib_ssm_conv_f32_stateful(kib_ctx* ctx, float* state, const float* in, const float* w, uint64_t K, uint64_t C,
                              uint64_t T, float* out) {
  KIB_REQUIRE_CTX(ctx);
  KIB_ARG(state && in && w && out && K >= 2 && K <= 16 && C && T, "ssm_conv: invalid arguments");
  cudaError_t e = conv_launch(state, in, static_cast<int>(C), w, static_cast<int>(K), static_cast<int>(C),
                              static_cast<int>(T), out, static_cast<int>(C), 0, ctx->stream);
  if (e != cudaSuccess) return check_cuda(ctx, e, "ssm_conv");
  return finish_op(ctx, "ssm_conv");
}
int kib_prepare_qwen35_gdn_gate_beta_f32(kib_ctx* ctx, float* gate, float* beta, const float* bias,
                                         const float* scale, uint64_t tokens, uint64_t heads) {
  KIB_REQUIRE_CTX(ctx);
  KIB_ARG(gate && beta && bias && scale && tokens && heads, "prepare_gate_beta: invalid arguments");
  const size_t n = tokens * heads;
  prepare_gate_beta_kernel<<<blocks_for(n), 256, 0, ctx->stream>>>(gate, beta, bias, scale, static_cast<int>(n),
                                                                    static_cast<int>(heads));
  return finish_op(ctx, "prepare_gate_beta");
}
int kib_gated_delta_net_f32_batched_in_place(kib_ctx* ctx, const float* q, const float* k, const float* v,
                                             const float* g, const float* beta, float* state, uint64_t tokens,
                                             uint64_t kh, uint64_t vh, uint64_t hd, float* out) {
  KIB_REQUIRE_CTX(ctx);
  KIB_ARG(q && k && v && g && beta && state && out && tokens && kh && vh && hd, "gated_delta_net: invalid arguments");
  KIB_ARG(vh % kh == 0, "gated_delta_net: value heads must be a multiple of key heads");
  const unsigned th = static_cast<unsigned>(hd < 256 ? hd : 256);
  gdn_generic_kernel<<<dim3(static_cast<unsigned>(vh), static_cast<unsigned>((hd + th - 1) / th)), th, 0,
                       ctx->stream>>>(q, k, v, g, beta, state, static_cast<int>(tokens), static_cast<int>(kh),
                                      static_cast<int>(vh), static_cast<int>(hd), out);
  return finish_op(ctx, "gated_delta_net");
}

// ---- attention
int kib_mrope_f32_in_place(kib_ctx* ctx, float* v, const int32_t* pos, uint64_t T, uint64_t heads, uint64_t hd,
                           uint64_t n_dims, uint64_t s0, uint64_t s1, uint64_t s2, uint64_t s3, float theta) {
  KIB_REQUIRE_CTX(ctx);
  KIB_ARG(v && pos && T && heads && hd && n_dims && n_dims <= hd && n_dims % 2 == 0, "mrope: invalid arguments");
  const size_t n = T * heads * (n_dims / 2);
  mrope_kernel<<<blocks_for(n), 256, 0, ctx->stream>>>(v, pos, static_cast<int>(T), static_cast<int>(heads),
                                                       static_cast<int>(hd), static_cast<int>(n_dims),
                                                       static_cast<int>(s0), static_cast<int>(s1),
                                                       static_cast<int>(s2), static_cast<int>(s3), theta);
  return finish_op(ctx, "mrope");
}
int kib_attention_f32_batched_f16_kv(kib_ctx* ctx, const float* q, const uint16_t* kc, const uint16_t* vc,
                                     uint64_t layer, uint64_t start, uint64_t T, uint64_t cap, uint64_t heads,
                                     uint64_t kvh, uint64_t hd, float* out) {
  KIB_REQUIRE_CTX(ctx);
  KIB_ARG(q && kc && vc && out && T && heads && kvh && hd && heads % kvh == 0 && hd <= 256,
          "attention: invalid arguments");
  KIB_ARG(start + T <= cap, "attention: positions exceed cache capacity");
  const size_t off = layer * cap * kvh * hd;
  const int round_q = (T >= 64 && hd == 256) ? 1 : 0;
  attention_generic_kernel<<<dim3(static_cast<unsigned>((T + 7) / 8), static_cast<unsigned>(heads)), 256, 0,
                             ctx->stream>>>(q, kc + off, vc + off, static_cast<int>(start), static_cast<int>(T),
                                            static_cast<int>(heads), static_cast<int>(kvh), static_cast<int>(hd),
                                            round_q, out);
  return finish_op(ctx, "attention");
}

// ---- element-wise
int kib_binary_f32_in_place(kib_ctx* ctx, int op, float* a, const float* b, uint64_t total, uint64_t row) {
  KIB_REQUIRE_CTX(ctx);
  KIB_ARG(a && b && total && op >= 0 && op <= 3 && (op < 2 || (row > 0 && total % row == 0)),
          "binary op: invalid arguments");
  binary_kernel<<<blocks_for(total), 256, 0, ctx->stream>>>(op, a, b, total, row ? row : 1);
  return finish_op(ctx, "binary");
}
int kib_unary_f32_in_place(kib_ctx* ctx, int op, float* v, uint64_t n) {
  KIB_REQUIRE_CTX(ctx);
  KIB_ARG(v && n && op >= 0 && op <= 2, "unary op: invalid arguments");
  unary_kernel<<<blocks_for(n), 256, 0, ctx->stream>>>(op, v, n);
  return finish_op(ctx, "unary");
}
int kib_silu_mul_f32_in_place(kib_ctx* ctx, float* g, const float* u, uint64_t n) {
  KIB_REQUIRE_CTX(ctx);
  KIB_ARG(g && u && n, "silu_mul: invalid arguments");
  cudaError_t e = silu_mul_launch(g, u, n, ctx->stream);
  if (e != cudaSuccess) return check_cuda(ctx, e, "silu_mul");
  return finish_op(ctx, "silu_mul");
}
int kib_copy_f32_rows(kib_ctx* ctx, const float* src, float* dst, uint64_t rows, uint64_t rv, uint64_t ss,
                      uint64_t so, uint64_t ds, uint64_t dof) {
  KIB_REQUIRE_CTX(ctx);
  KIB_ARG(src && dst && rows && rv && rv + so <= ss && rv <= ds, "copy_f32_rows: invalid arguments");
  copy_rows_kernel<<<blocks_for(rows * rv), 256, 0, ctx->stream>>>(src, dst, nullptr, rows, rv, ss, so, ds, dof);
  return finish_op(ctx, "copy_f32_rows");
}
int kib_copy_f32_rows_to_f16(kib_ctx* ctx, const float* src, uint16_t* dst, uint64_t rows, uint64_t rv, uint64_t ss,
                             uint64_t so, uint64_t ds, uint64_t dof) {
  KIB_REQUIRE_CTX(ctx);
  KIB_ARG(src && dst && rows && rv && rv + so <= ss && rv <= ds, "copy_f32_rows_to_f16: invalid arguments");
  copy_rows_kernel<<<blocks_for(rows * rv), 256, 0, ctx->stream>>>(src, nullptr, dst, rows, rv, ss, so, ds, dof);
  return finish_op(ctx, "copy_f32_rows_to_f16");
}
int kib_argmax_f32_i32(kib_ctx* ctx, const float* v, uint64_t n, int32_t* tok, float* prob) {
  KIB_REQUIRE_CTX(ctx);
  KIB_ARG(v && tok && n > 0 && n < (1ull << 31), "argmax: invalid arguments");
  argmax_kernel<<<1, 256, 0, ctx->stream>>>(v, static_cast<int>(n), tok, prob);
  return finish_op(ctx, "argmax");
}

}  // extern "C"
