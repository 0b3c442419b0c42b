// layer_kernels.cuh -- the non-GEMV kernels of the Qwen3.5 hybrid decoder:
// fused gated-delta-net core, split-K GQA decode attention with an in-kernel
// combine, prefill attention, token embedding, MTP input preparation and the
// multi-token (M > 8) K-quant GEMM used by chunked prefill.
#pragma once

#include "kib_common.cuh"
#include "kquant.cuh"

namespace kib {

KIB_DEV float sigmoid_f(float v) { return 1.0f / (1.0f + expf(-v)); }
KIB_DEV float softplus20_f(float v) { return v > 20.0f ? v : logf(1.0f + expf(v)); }
KIB_DEV float silu_k(float v) { return v / (1.0f + expf(-v)); }

// ===================================================================== GDN
// One CTA per (value head, group of 16 state rows).  Fuses, per token:
//   split_qkv_l2_norm_f32_qwen35 (mps_backend.mm:2097-2153) for the head's q,k,
//   prepare_qwen35_gdn_gate_beta_f32 (2588-2605),
//   gated_delta_net_f32_batched_qwen35 (2307-2374) for 16 rows of S.
// The conv + silu that precede it run in the qkv GEMV epilogue; the norm-gate
// that follows runs in the ssm_out GEMV prologue.
struct GdnParams {
  const float* conv_out;  // [T][C]: q | k | v after conv+silu
  int C;
  const float* beta_raw;  // [T][ld_ba]
  const float* alpha_raw; // [T][ld_ba]
  int ld_ba;
  const float* dt_bias;   // [Hv]
  const float* ssm_a;     // [Hv]
  float* state;           // [Hv][128][128] (this layer)
  float* out;             // [T][Hv*128]
  int T;
  int key_heads;
  int value_heads;
  float eps;
  unsigned long long* trace;
  // batched decode (gdn_core_kernel only): blockIdx.z is a sequence slot with
  // one token (T = 1); row `slot` of conv_out / alpha / beta / out is its
  // token and its state starts state_slot_stride floats after slot 0's
  int batched;
  size_t state_slot_stride;
};

constexpr int kGdnRows = 16;  // state rows per CTA

static __global__ void __launch_bounds__(128) gdn_core_kernel(const __grid_constant__ GdnParams p) {
  constexpr int D = 128;
  __shared__ __align__(16) float qn[D];
  __shared__ __align__(16) float kn[D];
  __shared__ float red[2][4];
  __shared__ float s_gb[2];
  const int h = blockIdx.x, grp = blockIdx.y;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int kh = h % p.key_heads;
  const int key_dim = p.key_heads * D;
  const int slot = p.batched ? static_cast<int>(blockIdx.z) : 0;
  const float* const conv_out = p.conv_out + static_cast<size_t>(slot) * p.C;
  const float* const alpha_raw = p.alpha_raw + static_cast<size_t>(slot) * p.ld_ba;
  const float* const beta_raw = p.beta_raw + static_cast<size_t>(slot) * p.ld_ba;
  float* const out = p.out + static_cast<size_t>(slot) * p.value_heads * D;
  float* S = p.state + slot * p.state_slot_stride + static_cast<size_t>(h) * D * D;
  // warp w owns rows grp*16 + 4w .. +3; lane owns columns 4*lane .. +3
  trace_entry(p.trace);
  float4 s[4];
#pragma unroll
  for (int r = 0; r < 4; ++r)
    s[r] = *reinterpret_cast<const float4*>(S + static_cast<size_t>(grp * kGdnRows + 4 * warp + r) * D + 4 * lane);

  pdl_wait();
  trace_wait(p.trace);
  pdl_launch_dependents();
  const float scale = 1.0f / sqrtf(static_cast<float>(D));
  // the next token's inputs are loaded while the current one is processed
  // (one global round trip per token would otherwise sit on the sequential path)
  auto load_tok = [&](int t, float& qv, float& kv, float (&vv)[4], float& a, float& b) {
    const float* row = conv_out + static_cast<size_t>(t) * p.C;
    qv = row[kh * D + tid];
    kv = row[key_dim + kh * D + tid];
#pragma unroll
    for (int r = 0; r < 4; ++r) vv[r] = row[2 * key_dim + h * D + grp * kGdnRows + 4 * warp + r];
    a = alpha_raw[static_cast<size_t>(t) * p.ld_ba + h];
    b = beta_raw[static_cast<size_t>(t) * p.ld_ba + h];
  };
  float nq = 0.f, nk = 0.f, nv[4] = {0.f, 0.f, 0.f, 0.f}, na = 0.f, nb = 0.f;
  if (p.T > 0) load_tok(0, nq, nk, nv, na, nb);
  for (int t = 0; t < p.T; ++t) {
    const float qv = nq, kv = nk, a = na, b = nb;
    float vcur[4];
#pragma unroll
    for (int r = 0; r < 4; ++r) vcur[r] = nv[r];
    if (t + 1 < p.T) load_tok(t + 1, nq, nk, nv, na, nb);
    float q2 = warp_sum(qv * qv), k2 = warp_sum(kv * kv);
    if (lane == 0) {
      red[0][warp] = q2;
      red[1][warp] = k2;
    }
    if (tid == 0) {
      s_gb[0] = softplus20_f(a + p.dt_bias[h]) * p.ssm_a[h];
      s_gb[1] = sigmoid_f(b);
    }
    __syncthreads();
    const float qs = 1.0f / fmaxf(sqrtf((red[0][0] + red[0][1]) + (red[0][2] + red[0][3])), p.eps);
    const float ks = 1.0f / fmaxf(sqrtf((red[1][0] + red[1][1]) + (red[1][2] + red[1][3])), p.eps);
    qn[tid] = qv * qs;
    kn[tid] = kv * ks;
    const float ge = expf(s_gb[0]);
    const float beta = s_gb[1];
    __syncthreads();
    const float4 k4 = *reinterpret_cast<const float4*>(kn + 4 * lane);
    const float4 q4 = *reinterpret_cast<const float4*>(qn + 4 * lane);
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int vrow = grp * kGdnRows + 4 * warp + r;
      float4 st = s[r];
      st.x *= ge;
      st.y *= ge;
      st.z *= ge;
      st.w *= ge;
      const float sk = warp_sum(st.x * k4.x + st.y * k4.y + st.z * k4.z + st.w * k4.w);
      const float delta = (vcur[r] - sk) * beta;
      st.x += k4.x * delta;
      st.y += k4.y * delta;
      st.z += k4.z * delta;
      st.w += k4.w * delta;
      const float y = warp_sum(st.x * q4.x + st.y * q4.y + st.z * q4.z + st.w * q4.w);
      if (lane == 0) out[static_cast<size_t>(t) * p.value_heads * D + h * D + vrow] = y * scale;
      s[r] = st;
    }
    __syncthreads();
  }
#pragma unroll
  for (int r = 0; r < 4; ++r)
    *reinterpret_cast<float4*>(S + static_cast<size_t>(grp * kGdnRows + 4 * warp + r) * D + 4 * lane) = s[r];
  trace_exit(p.trace);
}

// Multi-token GDN in two steps.  gdn_prep_kernel does the token-parallel part:
// the L2 norms of each token's q and k head rows (in place in the conv output,
// same reduction order as gdn_core_kernel) and g = softplus(alpha + dt_bias) *
// ssm_a, beta = sigmoid(beta) (in place).  gdn_scan_kernel then runs only the
// sequential delta rule (the recurrence of ggml_gated_delta_net, one value row
// of the state at a time; rows are independent of each other):
//   S_v *= exp(g);  delta = (v_v - S_v . k) * beta;  S_v += delta * k;
//   y_v = (S_v . q) / sqrt(128)
// Eight lanes own one value row (sixteen key columns each, as four float4 at
// columns 32j + 4c, so eight lanes read 128 contiguous bytes of k or q), so
// each dot product ends in three shuffles.  A CTA owns sixteen rows of one
// head; the q, k, v, g and beta of kGdnScanChunk tokens are staged in shared
// memory by cp.async one chunk ahead, so the per-token chain never waits on
// global memory, and the only CTA barrier sits between chunks.
constexpr int kGdnScanRowsPerCta = 16;
constexpr int kGdnScanChunk = 32;
constexpr int kGdnScanStage = kGdnScanChunk * (2 * 128 + kGdnScanRowsPerCta + 2);  // floats per buffer
constexpr int kGdnScanSmem = 2 * kGdnScanStage * 4;

static __global__ void __launch_bounds__(128) gdn_prep_kernel(float* conv_out, int C, float* alpha, float* beta,
                                                               int ld_ba, const float* dt_bias, const float* ssm_a,
                                                               int key_heads, int value_heads, float eps) {
  constexpr int D = 128;
  __shared__ float red[2][4];
  pdl_wait();
  pdl_launch_dependents();
  const int t = blockIdx.x, kh = blockIdx.y;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  float* row = conv_out + static_cast<size_t>(t) * C;
  const int key_dim = key_heads * D;
  const float qv = row[kh * D + tid], kv = row[key_dim + kh * D + tid];
  const float q2 = warp_sum(qv * qv), k2 = warp_sum(kv * kv);
  if (lane == 0) {
    red[0][warp] = q2;
    red[1][warp] = k2;
  }
  __syncthreads();
  const float qs = 1.0f / fmaxf(sqrtf((red[0][0] + red[0][1]) + (red[0][2] + red[0][3])), eps);
  const float ks = 1.0f / fmaxf(sqrtf((red[1][0] + red[1][1]) + (red[1][2] + red[1][3])), eps);
  row[kh * D + tid] = qv * qs;
  row[key_dim + kh * D + tid] = kv * ks;
  // gate/beta of the value heads this key head serves (h % key_heads == kh)
  for (int h = kh + key_heads * tid; h < value_heads; h += key_heads * 128) {
    const size_t o = static_cast<size_t>(t) * ld_ba + h;
    alpha[o] = softplus20_f(alpha[o] + dt_bias[h]) * ssm_a[h];
    beta[o] = sigmoid_f(beta[o]);
  }
}

__device__ __forceinline__ void gs_cp16(void* sdst, const void* gsrc) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(sdst)), "l"(gsrc) : "memory");
}
__device__ __forceinline__ void gs_cp4(void* sdst, const void* gsrc) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(sdst)), "l"(gsrc) : "memory");
}

// Requires C % 4 == 0 and 16-byte aligned conv_out (every row's q/k/v runs are
// copied as 16-byte pieces).
static __global__ void __launch_bounds__(128) gdn_scan_kernel(const __grid_constant__ GdnParams p) {
  constexpr int D = 128, TC = kGdnScanChunk, RC = kGdnScanRowsPerCta;
  extern __shared__ __align__(16) float gs_smem[];
  const int h = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int c = lane & 7;
  const int row_base = blockIdx.y * RC;
  const int row = row_base + warp * 4 + (lane >> 3);
  const int kh = h % p.key_heads;
  const int key_dim = p.key_heads * D;
  float* S = p.state + (static_cast<size_t>(h) * D + row) * D;
  float4 s[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) s[j] = *reinterpret_cast<const float4*>(S + 32 * j + 4 * c);
  pdl_wait();
  pdl_launch_dependents();

  // buffer layout: q[TC][128] | k[TC][128] | v[TC][RC] | g[TC] | beta[TC]
  auto load_chunk = [&](int t0, float* buf) {
    const int n = min(TC, p.T - t0);
    for (int i = tid; i < n * 64; i += 128) {
      const int u = i >> 6, w = i & 63;  // w < 32: q piece, else k piece
      const float* src = p.conv_out + static_cast<size_t>(t0 + u) * p.C + (w < 32 ? kh * D + 4 * w
                                                                                  : key_dim + kh * D + 4 * (w - 32));
      gs_cp16(buf + (w < 32 ? 0 : TC * D) + u * D + 4 * (w & 31), src);
    }
    for (int i = tid; i < n * (RC / 4); i += 128) {
      const int u = i / (RC / 4), w = i % (RC / 4);
      gs_cp16(buf + 2 * TC * D + u * RC + 4 * w,
              p.conv_out + static_cast<size_t>(t0 + u) * p.C + 2 * key_dim + h * D + row_base + 4 * w);
    }
    for (int i = tid; i < 2 * n; i += 128) {
      const int u = i >> 1;
      if (i & 1) gs_cp4(buf + 2 * TC * D + TC * RC + TC + u, p.beta_raw + static_cast<size_t>(t0 + u) * p.ld_ba + h);
      else gs_cp4(buf + 2 * TC * D + TC * RC + u, p.alpha_raw + static_cast<size_t>(t0 + u) * p.ld_ba + h);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };

  const float scale = 1.0f / sqrtf(static_cast<float>(D));
  float* out = p.out + static_cast<size_t>(h) * D + row;
  const size_t out_ld = static_cast<size_t>(p.value_heads) * D;
  const int nchunks = (p.T + TC - 1) / TC;
  load_chunk(0, gs_smem);
  for (int ci = 0; ci < nchunks; ++ci) {
    asm volatile("cp.async.wait_all;" ::: "memory");
    __syncthreads();  // chunk ci landed for all threads; chunk ci-1's buffer is free
    float* buf = gs_smem + (ci & 1) * kGdnScanStage;
    if (ci + 1 < nchunks) load_chunk((ci + 1) * TC, gs_smem + ((ci + 1) & 1) * kGdnScanStage);
    const float* qb = buf;
    const float* kb = buf + TC * D;
    const float* vb = buf + 2 * TC * D + (row - row_base);
    const float* gb = buf + 2 * TC * D + TC * RC;
    const int n = min(TC, p.T - ci * TC);
#pragma unroll 2
    for (int u = 0; u < n; ++u) {
      float4 k4[4], q4[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        k4[j] = *reinterpret_cast<const float4*>(kb + u * D + 32 * j + 4 * c);
        q4[j] = *reinterpret_cast<const float4*>(qb + u * D + 32 * j + 4 * c);
      }
      const float ge = expf(gb[u]), beta = gb[TC + u], v = vb[u * RC];
      float pk[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        s[j].x *= ge;
        s[j].y *= ge;
        s[j].z *= ge;
        s[j].w *= ge;
        pk[j] = s[j].x * k4[j].x + s[j].y * k4[j].y + s[j].z * k4[j].z + s[j].w * k4[j].w;
      }
      float sk = (pk[0] + pk[1]) + (pk[2] + pk[3]);
      sk += __shfl_xor_sync(0xffffffffu, sk, 1);
      sk += __shfl_xor_sync(0xffffffffu, sk, 2);
      sk += __shfl_xor_sync(0xffffffffu, sk, 4);
      const float delta = (v - sk) * beta;
      float pq[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        s[j].x += k4[j].x * delta;
        s[j].y += k4[j].y * delta;
        s[j].z += k4[j].z * delta;
        s[j].w += k4[j].w * delta;
        pq[j] = s[j].x * q4[j].x + s[j].y * q4[j].y + s[j].z * q4[j].z + s[j].w * q4[j].w;
      }
      float y = (pq[0] + pq[1]) + (pq[2] + pq[3]);
      y += __shfl_xor_sync(0xffffffffu, y, 1);
      y += __shfl_xor_sync(0xffffffffu, y, 2);
      y += __shfl_xor_sync(0xffffffffu, y, 4);
      if (c == 0) out[static_cast<size_t>(ci * TC + u) * out_ld] = y * scale;
    }
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) *reinterpret_cast<float4*>(S + 32 * j + 4 * c) = s[j];
}

// =============================================================== attention
struct AttnParams {
  const float* qg;        // [T][heads][2*hd]: q | gate per head (joint projection)
  const float* kp;        // [T][kv_heads*hd]
  const float* vp;        // [T][kv_heads*hd]
  const float* q_norm;    // [hd]
  const float* k_norm;    // [hd]
  uint16_t* kcache;       // [cap][kv_heads*hd] f16, this layer
  uint16_t* vcache;
  const int* pos;         // position of token 0
  int T;
  int heads;
  int kv_heads;
  float eps;
  float theta;
  int n_dims;             // rotated dims (2 * sum of MRoPE sections)
  int sec0, sec1, sec2, sec3;
  int nsplit;
  // batched decode (attn_decode_kernel only): blockIdx.z is a sequence slot
  // with one token (T = 1); pos is then [slots], the caches of slot s start
  // cache_slot_stride halves after the slot-0 pointers, and the qg/kp/vp/out
  // rows, the split partials and the counters are indexed by slot
  int batched;
  size_t cache_slot_stride;
  float* part;            // [nsplit][T][heads][hd + 2]
  unsigned* counters;     // [kv_heads]
  float* out;             // [T][heads*hd]
  float* q_out;           // prefill: normed+roped q [T][heads][hd]
  int round_q;            // prefill T >= 64: Q rounded to half (flash256 numerics)
  unsigned long long* trace;
};

constexpr int kHd = 256;

// qk_norm (mps_backend.mm:1991-2024) then mrope_f32_in_place (2482-2527) on one
// 256-wide head vector held in shared memory; one warp.
KIB_DEV void norm_rope_head(float* v, const float* in, const float* w, float eps, int position,
                            const AttnParams& p, int lane) {
  float ss = 0.0f;
  for (int i = lane; i < kHd; i += 32) {
    const float x = in[i];
    ss += x * x;
  }
  ss = warp_sum(ss);
  const float scale = 1.0f / sqrtf(ss / static_cast<float>(kHd) + p.eps);
  for (int i = lane; i < kHd; i += 32) v[i] = in[i] * (scale * w[i]);
  __syncwarp();
  const int half = p.n_dims / 2;
  const int total = p.sec0 + p.sec1 + p.sec2 + p.sec3;
  for (int pi = lane; pi < half; pi += 32) {
    // text positions: all four MRoPE position streams equal `position`
    (void)total;
    const float exponent = static_cast<float>(2 * pi) / static_cast<float>(p.n_dims);
    const float freq = 1.0f / powf(p.theta, exponent);
    const float angle = static_cast<float>(position) * freq;
    float sn, cs;
    sincosf(angle, &sn, &cs);
    const float x0 = v[pi], x1 = v[half + pi];
    v[pi] = x0 * cs - x1 * sn;
    v[half + pi] = x1 * cs + x0 * sn;
  }
  __syncwarp();
}

// Split-K decode attention for T <= 8 queries over an F16 KV cache.  Grid
// (nsplit, kv_heads); each CTA owns a contiguous key range of one kv head.
// The range's cached keys (positions < pos) are staged into shared memory in
// chunks of 32 keys by cp.async.bulk (K and V rows, 512 B each) -- the first
// two chunks are issued before griddepcontrol.wait, since the cache was written
// by earlier steps.  The CTA owning a new token's position normalises, rotates
// and writes its K/V (single writer) and attends to it from shared memory.
// 8 warps: warp w serves q head (w % 4) of the kv group and every other key
// (w / 4).  The last CTA of each kv head merges all splits and applies
// sigmoid(gate) (attention_f32_batched_f16_kv, mps_backend.mm:2943-3008, plus
// qwen35_runtime.cpp:3347-3351).
constexpr int kAttnChunk = 32;

__host__ __device__ inline size_t attn_decode_smem_bytes(int T) {
  return static_cast<size_t>(2) * kAttnChunk * 2 * kHd * sizeof(uint16_t) +
         (static_cast<size_t>(T) * 4 * kHd + 2 * static_cast<size_t>(T) * kHd + 8 * static_cast<size_t>(T) * (kHd + 2)) *
             sizeof(float);
}

template <int TM>
__global__ void __launch_bounds__(256) attn_decode_kernel(const __grid_constant__ AttnParams p) {
  constexpr int G = 4;  // q heads per kv head
  extern __shared__ __align__(128) uint8_t smraw[];
  uint16_t* kvbuf = reinterpret_cast<uint16_t*>(smraw);  // [2][32 keys][K 256 | V 256] f16
  float* qs = reinterpret_cast<float*>(smraw + 2 * kAttnChunk * 2 * kHd * sizeof(uint16_t));  // [T][G][256]
  float* newk = qs + p.T * G * kHd;     // [T][256] new keys (f16-rounded)
  float* newv = newk + p.T * kHd;       // [T][256]
  float* merge = newv + p.T * kHd;      // [8 warps][T][256 + 2]
  __shared__ uint64_t bar[2];
  __shared__ bool s_last;
  const int split = blockIdx.x, kvh = blockIdx.y;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int kvd = p.kv_heads * kHd;
  const int slot = p.batched ? static_cast<int>(blockIdx.z) : 0;
  uint16_t* const kcache = p.kcache + slot * p.cache_slot_stride;
  uint16_t* const vcache = p.vcache + slot * p.cache_slot_stride;
  const float* const qg = p.qg + static_cast<size_t>(slot) * p.heads * 2 * kHd;
  const float* const kp = p.kp + static_cast<size_t>(slot) * kvd;
  const float* const vp = p.vp + static_cast<size_t>(slot) * kvd;
  float* const part = p.part + static_cast<size_t>(slot) * p.nsplit * p.heads * (kHd + 2);
  unsigned* const counters = p.counters + static_cast<size_t>(slot) * p.kv_heads;
  float* const out = p.out + static_cast<size_t>(slot) * p.heads * kHd;

  // the position was written at least two kernels earlier (host copy or the
  // previous step's LM head), so it and the cached keys are readable now
  trace_entry(p.trace);
  const int pos0 = p.pos[slot];
  const int nkeys = pos0 + p.T;
  int chunk = (nkeys + p.nsplit - 1) / p.nsplit;
  chunk = (chunk + 7) & ~7;
  const int kb = split * chunk, ke = min(kb + chunk, nkeys);
  const int old_end = min(ke, pos0);
  const int nold = max(0, old_end - kb);
  const int nchunks = (nold + kAttnChunk - 1) / kAttnChunk;
  auto issue = [&](int c) {  // warp 0 only
    const int k0 = kb + c * kAttnChunk;
    const int nk = min(kAttnChunk, old_end - k0);
    const int st = c & 1;
    if (lane == 0) mbar_arrive_expect_tx(&bar[st], static_cast<uint32_t>(nk) * 2u * kHd * 2u);
    __syncwarp();
    if (lane < nk) {
      const size_t src = static_cast<size_t>(k0 + lane) * kvd + kvh * kHd;
      uint16_t* dst = kvbuf + (static_cast<size_t>(st) * kAttnChunk + lane) * 2 * kHd;
      bulk_g2s(dst, kcache + src, kHd * 2, &bar[st]);
      bulk_g2s(dst + kHd, vcache + src, kHd * 2, &bar[st]);
    }
  };
  if (warp == 0) {
    if (lane == 0) {
      mbar_init(&bar[0], 1);
      mbar_init(&bar[1], 1);
      fence_mbar_init();
    }
    __syncwarp();
    for (int c = 0; c < min(2, nchunks); ++c) issue(c);
  }
  __syncthreads();

  pdl_wait();
  trace_wait(p.trace);
  pdl_launch_dependents();
  // q prep: warp -> (head, token)
  for (int job = warp; job < G * p.T; job += 8) {
    const int j = job % G, t = job / G;
    const int head = kvh * G + j;
    norm_rope_head(qs + (t * G + j) * kHd, qg + (static_cast<size_t>(t) * p.heads + head) * 2 * kHd, p.q_norm,
                   p.eps, pos0 + t, p, lane);
  }
  // new keys owned by this split
  for (int t = warp; t < p.T; t += 8) {
    const int kpos = pos0 + t;
    if (kpos < kb || kpos >= ke) continue;
    float* kr = newk + t * kHd;
    norm_rope_head(kr, kp + static_cast<size_t>(t) * kvd + kvh * kHd, p.k_norm, p.eps, kpos, p, lane);
    for (int i = lane; i < kHd; i += 32) {
      const __half kh = __float2half_rn(kr[i]);
      const __half vh = __float2half_rn(vp[static_cast<size_t>(t) * kvd + kvh * kHd + i]);
      kcache[static_cast<size_t>(kpos) * kvd + kvh * kHd + i] = __half_as_ushort(kh);
      vcache[static_cast<size_t>(kpos) * kvd + kvh * kHd + i] = __half_as_ushort(vh);
      kr[i] = __half2float(kh);
      newv[t * kHd + i] = __half2float(vh);
    }
  }
  __syncthreads();

  const int j = warp % G, kh2 = warp / G;
  const float scale = 1.0f / sqrtf(static_cast<float>(kHd));
  float m[TM], l[TM], acc[TM][8], qreg[TM][8];
#pragma unroll
  for (int t = 0; t < TM; ++t) {
    m[t] = -INFINITY;
    l[t] = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      acc[t][i] = 0.0f;
      qreg[t][i] = t < p.T ? qs[(t * G + j) * kHd + 8 * lane + i] : 0.0f;
    }
  }
  auto attend = [&](const float (&kf)[8], const float (&vf)[8], int key) {
#pragma unroll
    for (int t = 0; t < TM; ++t) {
      if (t >= p.T) break;
      if (key > pos0 + t) continue;  // causal (uniform across the warp)
      float d = 0.0f;
#pragma unroll
      for (int i = 0; i < 8; ++i) d = fmaf(qreg[t][i], kf[i], d);
      const float sc = warp_sum(d) * scale;
      const float nm = fmaxf(m[t], sc);
      const float ps = expf(m[t] - nm);
      const float w = expf(sc - nm);
      l[t] = l[t] * ps + w;
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[t][i] = acc[t][i] * ps + w * vf[i];
      m[t] = nm;
    }
  };
  // 8 keys per step: the 8 scores reduce independently, then one
  // online-softmax update per step
  constexpr int KB = 8;
#pragma unroll 1
  for (int c = 0; c < nchunks; ++c) {
    const int st = c & 1;
    mbar_wait_bounded(&bar[st], static_cast<uint32_t>((c >> 1) & 1), nullptr);
    const int k0 = kb + c * kAttnChunk;
    const int nk = min(kAttnChunk, old_end - k0);
#pragma unroll 1
    for (int kk0 = kh2 * KB; kk0 < nk; kk0 += 2 * KB) {
      float sc[TM][KB];
      uint4 vraw[KB];
#pragma unroll
      for (int e = 0; e < KB; ++e) {
        const int kk = min(kk0 + e, nk - 1);
        const uint16_t* row = kvbuf + (static_cast<size_t>(st) * kAttnChunk + kk) * 2 * kHd;
        const uint4 kr = *reinterpret_cast<const uint4*>(row + 8 * lane);
        vraw[e] = *reinterpret_cast<const uint4*>(row + kHd + 8 * lane);
        const __half2* kh = reinterpret_cast<const __half2*>(&kr);
        float kf[8];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 a2 = __half22float2(kh[i]);
          kf[2 * i] = a2.x;
          kf[2 * i + 1] = a2.y;
        }
#pragma unroll
        for (int t = 0; t < TM; ++t) {
          float d = 0.0f;
#pragma unroll
          for (int i = 0; i < 8; ++i) d = fmaf(qreg[t][i], kf[i], d);
          sc[t][e] = d;
        }
      }
#pragma unroll
      for (int t = 0; t < TM; ++t)
#pragma unroll
        for (int e = 0; e < KB; ++e) sc[t][e] = warp_sum(sc[t][e]) * scale;
#pragma unroll
      for (int t = 0; t < TM; ++t) {
        if (t >= p.T) break;
        float mx = m[t];
#pragma unroll
        for (int e = 0; e < KB; ++e)
          if (kk0 + e < nk) mx = fmaxf(mx, sc[t][e]);
        const float ps = expf(m[t] - mx);
        l[t] *= ps;
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[t][i] *= ps;
#pragma unroll
        for (int e = 0; e < KB; ++e) {
          if (kk0 + e >= nk) break;
          const float w = expf(sc[t][e] - mx);
          l[t] += w;
          const __half2* vh = reinterpret_cast<const __half2*>(&vraw[e]);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float2 b2 = __half22float2(vh[i]);
            acc[t][2 * i] = fmaf(w, b2.x, acc[t][2 * i]);
            acc[t][2 * i + 1] = fmaf(w, b2.y, acc[t][2 * i + 1]);
          }
        }
        m[t] = mx;
      }
    }
    __syncthreads();  // stage consumed
    if (warp == 0 && c + 2 < nchunks) issue(c + 2);
  }
  // the new keys of this split (positions >= pos0), from shared memory
  if (kh2 == 0) {
    for (int t2 = 0; t2 < p.T; ++t2) {
      const int kpos = pos0 + t2;
      if (kpos < kb || kpos >= ke) continue;
      float kf[8], vf[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        kf[i] = newk[t2 * kHd + 8 * lane + i];
        vf[i] = newv[t2 * kHd + 8 * lane + i];
      }
      attend(kf, vf, kpos);
    }
  }
  // merge the two key halves of each head inside the CTA, then write the split partial
  for (int t = 0; t < p.T; ++t) {
    float* mrow = merge + (warp * p.T + t) * (kHd + 2);
    for (int i = 0; i < 8; ++i) mrow[8 * lane + i] = acc[t][i];
    if (lane == 0) {
      mrow[kHd] = m[t];
      mrow[kHd + 1] = l[t];
    }
  }
  __syncthreads();
  for (int job = tid; job < G * p.T * kHd; job += 256) {
    const int i = job % kHd, jt = job / kHd, jj = jt % G, t = jt / G;
    const float* a = merge + (jj * p.T + t) * (kHd + 2);        // warp jj   (half 0)
    const float* b = merge + ((jj + G) * p.T + t) * (kHd + 2);  // warp jj+4 (half 1)
    const float ma = a[kHd], mb = b[kHd];
    const float M = fmaxf(ma, mb);
    const float ea = ma == -INFINITY ? 0.0f : expf(ma - M);
    const float eb = mb == -INFINITY ? 0.0f : expf(mb - M);
    float* dst = part + ((static_cast<size_t>(split) * p.T + t) * p.heads + kvh * G + jj) * (kHd + 2);
    dst[i] = a[i] * ea + b[i] * eb;
    if (i == 0) {
      dst[kHd] = M;
      dst[kHd + 1] = a[kHd + 1] * ea + b[kHd + 1] * eb;
    }
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) s_last = atomicAdd(&counters[kvh], 1u) == static_cast<unsigned>(p.nsplit - 1);
  __syncthreads();
  trace_exit(p.trace);
  if (!s_last) return;
  __threadfence();
  // merge: per (head, token) pair the split weights exp(m_s - M) go to shared
  // memory once; every output element then sums independent loads.
  const int pairs = G * p.T;
  const int nact = min(p.nsplit, (nkeys + chunk - 1) / chunk);  // splits that saw keys
  float* wsm = merge;                          // [pairs][nsplit]  m, then the weights
  float* lsm = merge + pairs * p.nsplit;       // [pairs][nsplit]  l
  float* dsm = merge + 2 * pairs * p.nsplit;   // [pairs]
  for (int idx = tid; idx < pairs * nact; idx += 256) {
    const int pr = idx / nact, sp = idx % nact;
    const int head = kvh * G + pr % G, t = pr / G;
    const float* src = part + ((static_cast<size_t>(sp) * p.T + t) * p.heads + head) * (kHd + 2) + kHd;
    wsm[pr * p.nsplit + sp] = __ldcg(src);
    lsm[pr * p.nsplit + sp] = __ldcg(src + 1);
  }
  __syncthreads();
  for (int pr = tid; pr < pairs; pr += 256) {
    float M = -INFINITY;
    for (int sp = 0; sp < nact; ++sp) M = fmaxf(M, wsm[pr * p.nsplit + sp]);
    float den = 0.0f;
    for (int sp = 0; sp < nact; ++sp) {
      const float ms = wsm[pr * p.nsplit + sp];
      const float e = ms == -INFINITY ? 0.0f : expf(ms - M);
      wsm[pr * p.nsplit + sp] = e;
      den += lsm[pr * p.nsplit + sp] * e;
    }
    dsm[pr] = den;
  }
  __syncthreads();
  // every thread owns 2 consecutive elements of one (head, token) pair and
  // keeps 16 split loads in flight
  for (int job = tid; job < pairs * (kHd / 2); job += 256) {
    const int i = 2 * (job % (kHd / 2)), pr = job / (kHd / 2), jj = pr % G, t = pr / G;
    const int head = kvh * G + jj;
    const float* src = part + (static_cast<size_t>(t) * p.heads + head) * (kHd + 2) + i;
    const size_t sstride = static_cast<size_t>(p.T) * p.heads * (kHd + 2);
    float n0 = 0.0f, n1 = 0.0f;
#pragma unroll 16
    for (int sp = 0; sp < nact; ++sp) {
      const float2 v = __ldcg(reinterpret_cast<const float2*>(src + sp * sstride));
      const float w = wsm[pr * p.nsplit + sp];
      n0 = fmaf(v.x, w, n0);
      n1 = fmaf(v.y, w, n1);
    }
    const float den = dsm[pr];
    const float inv = den == 0.0f ? 0.0f : 1.0f / den;
    const float* g = qg + (static_cast<size_t>(t) * p.heads + head) * 2 * kHd + kHd + i;
    float* o = out + static_cast<size_t>(t) * p.heads * kHd + head * kHd + i;
    o[0] = n0 * inv * sigmoid_f(g[0]);
    o[1] = n1 * inv * sigmoid_f(g[1]);
  }
  __syncthreads();
  trace_exit(p.trace);
  if (tid == 0) counters[kvh] = 0u;
}

// Prefill step 1: per token, q norm+rope -> q_out, k norm+rope and v -> f16 cache.
// grid T; 8 warps over the heads + kv heads.
static __global__ void __launch_bounds__(256) attn_prep_kernel(const __grid_constant__ AttnParams p) {
  extern __shared__ __align__(16) float sm[];
  const int t = blockIdx.x, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  pdl_wait();
  pdl_launch_dependents();
  const int pos = *p.pos + t;
  const int kvd = p.kv_heads * kHd;
  float* tmp = sm + warp * kHd;
  for (int job = warp; job < p.heads + p.kv_heads; job += 8) {
    if (job < p.heads) {
      norm_rope_head(tmp, p.qg + (static_cast<size_t>(t) * p.heads + job) * 2 * kHd, p.q_norm, p.eps, pos, p, lane);
      for (int i = lane; i < kHd; i += 32) p.q_out[(static_cast<size_t>(t) * p.heads + job) * kHd + i] = tmp[i];
    } else {
      const int kh = job - p.heads;
      norm_rope_head(tmp, p.kp + static_cast<size_t>(t) * kvd + kh * kHd, p.k_norm, p.eps, pos, p, lane);
      for (int i = lane; i < kHd; i += 32) {
        p.kcache[static_cast<size_t>(pos) * kvd + kh * kHd + i] = __half_as_ushort(__float2half_rn(tmp[i]));
        p.vcache[static_cast<size_t>(pos) * kvd + kh * kHd + i] =
            __half_as_ushort(__float2half_rn(p.vp[static_cast<size_t>(t) * kvd + kh * kHd + i]));
      }
    }
    __syncwarp();
  }
}

// Sums 8 values over the warp; every lane ends with the 8 totals.  Three
// halving exchanges leave each lane one value summed over 8 lanes, two more
// finish it, and 8 broadcasts return the totals (17 shuffles instead of 40).
KIB_DEV void warp_sum8(float (&v)[8], int lane) {
  float a[4], b[2];
  const bool h16 = lane & 16, h8 = lane & 8, h4 = lane & 4;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float send = h16 ? v[i] : v[i + 4], keep = h16 ? v[i + 4] : v[i];
    a[i] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
  }
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const float send = h8 ? a[i] : a[i + 2], keep = h8 ? a[i + 2] : a[i];
    b[i] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
  }
  float c = (h4 ? b[1] : b[0]) + __shfl_xor_sync(0xffffffffu, h4 ? b[0] : b[1], 4);
  c += __shfl_xor_sync(0xffffffffu, c, 2);
  c += __shfl_xor_sync(0xffffffffu, c, 1);
  // lane L holds the total of value ((L >> 4) & 1) * 4 + ((L >> 3) & 1) * 2 + ((L >> 2) & 1)
#pragma unroll
  for (int e = 0; e < 8; ++e) v[e] = __shfl_sync(0xffffffffu, c, ((e >> 2) & 1) << 4 | ((e >> 1) & 1) << 3 | (e & 1) << 2);
}

// Prefill step 2: one warp per (query, head), online softmax over keys <= query
// position in blocks of 8 (attention_f32_batched_f16_kv, with the running max
// updated once per block); Q rounded to
// half when round_q (flash256 numerics, mps_backend.mm:3450-3460); output
// multiplied by sigmoid(gate).  grid (ceil(T/8), heads).
static __global__ void __launch_bounds__(256) attn_prefill_kernel(const __grid_constant__ AttnParams p) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int t = blockIdx.x * 8 + warp, head = blockIdx.y;
  pdl_wait();
  pdl_launch_dependents();
  if (t >= p.T) return;
  const int pos0 = *p.pos;
  const int qpos = pos0 + t;
  const int kvd = p.kv_heads * kHd;
  const int kvh = head / (p.heads / p.kv_heads);
  float q[8], acc[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float v = p.q_out[(static_cast<size_t>(t) * p.heads + head) * kHd + 8 * lane + i];
    q[i] = p.round_q ? round_to_half(v) : v;
    acc[i] = 0.0f;
  }
  const float scale = 1.0f / sqrtf(static_cast<float>(kHd));
  float m = -INFINITY, l = 0.0f;
  // blocks of 8 keys: the 8 partial dot products share one butterfly, and the
  // block's K and V rows are loaded together, through L1 (the CTA's eight
  // warps are eight consecutive queries of one head and read the same rows)
  const size_t kbase = static_cast<size_t>(kvh) * kHd + 8 * lane;
  for (int k0 = 0; k0 <= qpos; k0 += 8) {
    uint4 kr[8], vr[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int key = min(k0 + e, qpos);
      kr[e] = __ldg(reinterpret_cast<const uint4*>(p.kcache + static_cast<size_t>(key) * kvd + kbase));
      vr[e] = __ldg(reinterpret_cast<const uint4*>(p.vcache + static_cast<size_t>(key) * kvd + kbase));
    }
    float sc[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const __half2* kh = reinterpret_cast<const __half2*>(&kr[e]);
      float d = 0.0f;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 a = __half22float2(kh[i]);
        d = fmaf(q[2 * i], a.x, d);
        d = fmaf(q[2 * i + 1], a.y, d);
      }
      sc[e] = d;
    }
    warp_sum8(sc, lane);
    float nm = m;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      sc[e] *= scale;
      if (k0 + e <= qpos) nm = fmaxf(nm, sc[e]);
    }
    const float ps = expf(m - nm);
    l *= ps;
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] *= ps;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float w = k0 + e <= qpos ? expf(sc[e] - nm) : 0.0f;
      l += w;
      const __half2* vh = reinterpret_cast<const __half2*>(&vr[e]);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 b = __half22float2(vh[i]);
        acc[2 * i] = fmaf(w, b.x, acc[2 * i]);
        acc[2 * i + 1] = fmaf(w, b.y, acc[2 * i + 1]);
      }
    }
    m = nm;
  }
  const float inv = l == 0.0f ? 0.0f : 1.0f / l;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int d = 8 * lane + i;
    const float g = p.qg[(static_cast<size_t>(t) * p.heads + head) * 2 * kHd + kHd + d];
    p.out[static_cast<size_t>(t) * p.heads * kHd + head * kHd + d] = acc[i] * inv * sigmoid_f(g);
  }
}

// =============================================================== embedding
// q*_k_get_rows (mps_backend.mm:1693-1824): dequantize rows `ids` of a K-quant
// matrix; out-of-range ids produce zeros.  grid T, 256 threads.
template <int QT>
__global__ void __launch_bounds__(256) get_rows_kernel(const uint8_t* w, int nrows, int cols, const int* ids,
                                                       float* out, int out_ld) {
  pdl_wait();
  pdl_launch_dependents();
  const int t = blockIdx.x;
  const int id = ids[t];
  const int units = cols / 64;
  const int bpr = cols / 256;
  float* o = out + static_cast<size_t>(t) * out_ld;
  for (int u = threadIdx.x; u < units; u += blockDim.x) {
    const int blk = u >> 2, unit = u & 3;
    if (id < 0 || id >= nrows) {
      for (int e = 0; e < 64; ++e) o[256 * blk + unit_col<QT>(unit, e)] = 0.0f;
      continue;
    }
    const uint8_t* b = w + (static_cast<size_t>(id) * bpr + blk) * kquant_block_bytes(QT);
    float v[64];
    unit_dequant<QT>(b, unit, v);
#pragma unroll
    for (int e = 0; e < 64; ++e) o[256 * blk + unit_col<QT>(unit, e)] = v[e];
  }
}

// MTP input (qwen35_runtime.cpp:4156-4195): cat[t] = [rms(e_t)*enorm | rms(h_t)*hnorm].
static __global__ void __launch_bounds__(256) mtp_cat_kernel(const float* e, const float* h, const float* enorm,
                                                      const float* hnorm, int H, float eps, float* cat) {
  __shared__ float red[2][8];
  pdl_wait();
  pdl_launch_dependents();
  const int t = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const float* er = e + static_cast<size_t>(t) * H;
  const float* hr = h + static_cast<size_t>(t) * H;
  float se = 0.0f, sh = 0.0f;
  for (int i = tid; i < H; i += 256) {
    se += er[i] * er[i];
    sh += hr[i] * hr[i];
  }
  se = warp_sum(se);
  sh = warp_sum(sh);
  if (lane == 0) {
    red[0][warp] = se;
    red[1][warp] = sh;
  }
  __syncthreads();
  float te = 0.0f, th = 0.0f;
  for (int w = 0; w < 8; ++w) {
    te += red[0][w];
    th += red[1][w];
  }
  const float ce = 1.0f / sqrtf(te / static_cast<float>(H) + eps);
  const float ch = 1.0f / sqrtf(th / static_cast<float>(H) + eps);
  float* c = cat + static_cast<size_t>(t) * 2 * H;
  for (int i = tid; i < H; i += 256) {
    c[i] = er[i] * ce * enorm[i];
    c[H + i] = hr[i] * ch * hnorm[i];
  }
}

// ============================================================ prefill GEMM
// Y[t][r] (+)= W[r,:] . X[t,:] for M > 8 tokens with the reference's mul_mm_simd
// numerics (mps_backend.mm:1088-1230): weights rounded to half per weight
// (dequantize_*_mm), x rounded to half, fp32 accumulation.  Products of two
// halves are exact in fp32, so CUDA-core FMAs reproduce the MMA up to order.
// Tile 64 rows x 64 tokens, K step one super-block (256).
struct GemmParams {
  const uint8_t* w;
  int rows, cols;
  const float* x;   // [T][x_ld]
  int x_ld;
  int T;
  float* y;         // [T][y_ld]
  int y_ld;
  const float* resid;  // optional [T][y_ld]
};

// Multi-token (T > 8) K-quant GEMM on the tensor cores: the reference's M > 8
// numerics (mul_mm_simd: weights and x rounded to fp16, fp32 accumulation).
// CTA tile 128 weight rows x 64 tokens (two CTAs per SM, so one CTA's
// dequantization overlaps the other's MMAs), one 256-column super-block per
// k-step: the 256 threads dequantize the tile's weights into shared memory as
// fp16 (each weight value exactly as unit_dequant_h2 rounds it) and round the
// x tile to fp16; 8 warps (4 along rows x 2 along tokens) each own a 32 x 32
// output tile of mma.sync m16n8k16 f16 x f16 -> f32, fragments by ldmatrix.
// Shared rows are padded to 264 halves so the ldmatrix rows spread over banks.
constexpr int kGemmTileM = 128, kGemmTileN = 64, kGemmLd = 256 + 8;
constexpr int kGemmWarpN = kGemmTileN / 2, kGemmNT = kGemmWarpN / 8;  // warp tile: 32 rows x kGemmWarpN tokens
constexpr size_t kGemmSmem = static_cast<size_t>(kGemmTileM + kGemmTileN) * kGemmLd * 2;

KIB_DEV void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

KIB_DEV void mma_f16_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

template <int QT>
__global__ void __launch_bounds__(256, 2) kquant_gemm_f16_kernel(const __grid_constant__ GemmParams p) {
  extern __shared__ __align__(16) uint8_t gsm_raw[];
  __half* As = reinterpret_cast<__half*>(gsm_raw);        // [128 rows][kGemmLd]
  __half* Bs = As + kGemmTileM * kGemmLd;                 // [128 tokens][kGemmLd]
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int r0 = blockIdx.x * kGemmTileM, t0 = blockIdx.y * kGemmTileN;
  const int bpr = p.cols / 256;
  const int wm = (warp & 3) * 32, wn = (warp >> 2) * kGemmWarpN;  // warp tile origin
  float acc[2][kGemmNT][4];
#pragma unroll
  for (int i = 0; i < 2; ++i)
#pragma unroll
    for (int j = 0; j < kGemmNT; ++j)
#pragma unroll
      for (int c = 0; c < 4; ++c) acc[i][j][c] = 0.0f;
  pdl_wait();
  pdl_launch_dependents();
  const uint32_t as_base = smem_u32(As), bs_base = smem_u32(Bs);
  for (int kb = 0; kb < bpr; ++kb) {
    // weights: 128 rows x 4 units of 64 = 512 units, two per thread
#pragma unroll 1
    for (int job = tid; job < kGemmTileM * 4; job += 256) {
      const int rl = job >> 2, unit = job & 3;
      const int row = r0 + rl;
      __half2 v[32];
      if (row < p.rows) {
        unit_dequant_h2<QT>(p.w + (static_cast<size_t>(row) * bpr + kb) * kquant_block_bytes(QT), unit, v);
      } else {
#pragma unroll
        for (int e = 0; e < 32; ++e) v[e] = __floats2half2_rn(0.0f, 0.0f);
      }
      __half* dst = As + rl * kGemmLd;
#pragma unroll
      for (int e = 0; e < 64; e += 2) {
        // unit_col is contiguous within aligned pairs
        *reinterpret_cast<__half2*>(dst + unit_col<QT>(unit, e)) = v[e / 2];
      }
    }
    // x: 128 tokens x 256 k, rounded to half
#pragma unroll 4
    for (int i = tid; i < kGemmTileN * 64; i += 256) {
      const int tl = i >> 6, k4 = (i & 63) * 4;
      const int t = t0 + tl;
      float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
      if (t < p.T) x = *reinterpret_cast<const float4*>(p.x + static_cast<size_t>(t) * p.x_ld + kb * 256 + k4);
      __half2* dst = reinterpret_cast<__half2*>(Bs + tl * kGemmLd + k4);
      dst[0] = __floats2half2_rn(x.x, x.y);
      dst[1] = __floats2half2_rn(x.z, x.w);
    }
    __syncthreads();
#pragma unroll 2
    for (int k0 = 0; k0 < 256; k0 += 16) {
      uint32_t a[2][4];
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const int row = wm + 16 * i + (lane & 15), col = k0 + (lane >> 4) * 8;
        ldsm_x4(as_base + static_cast<uint32_t>(row * kGemmLd + col) * 2, a[i][0], a[i][1], a[i][2], a[i][3]);
      }
#pragma unroll
      for (int j = 0; j < kGemmNT; j += 2) {
        const int n = wn + 8 * j + (lane & 7) + ((lane >> 4) << 3), col = k0 + ((lane >> 3) & 1) * 8;
        uint32_t b0, b1, b2, b3;
        ldsm_x4(bs_base + static_cast<uint32_t>(n * kGemmLd + col) * 2, b0, b1, b2, b3);
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          mma_f16_16816(acc[i][j], a[i], b0, b1);
          mma_f16_16816(acc[i][j + 1], a[i], b2, b3);
        }
      }
    }
    __syncthreads();
  }
  // D fragment: c0,c1 at (row g, tokens 2q, 2q+1), c2,c3 at row g+8
  const int g = lane >> 2, q = lane & 3;
#pragma unroll
  for (int i = 0; i < 2; ++i)
#pragma unroll
    for (int j = 0; j < kGemmNT; ++j)
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int row = r0 + wm + 16 * i + g + (c >> 1) * 8;
        const int t = t0 + wn + 8 * j + 2 * q + (c & 1);
        if (row < p.rows && t < p.T) {
          float v = acc[i][j][c];
          if (p.resid) v += p.resid[static_cast<size_t>(t) * p.y_ld + row];
          p.y[static_cast<size_t>(t) * p.y_ld + row] = v;
        }
      }
}

// ---- f16-operand GEMM for prefill ---------------------------------------------
// The same products as kquant_gemm_f16_kernel (weights exactly as
// unit_dequant_h2 rounds them, x rounded to half, fp32 accumulation in the same
// k order), with the dequantization taken out of the GEMM: kquant_to_f16_kernel
// writes a weight matrix as f16 [rows][cols] (once at load for the resident
// copies, or per call into scratch), x_to_f16_kernel rounds x once, and
// gemm_f16w_kernel streams both through a three-stage cp.async ring into
// mma.sync m16n8k16.
template <int QT>
__global__ void __launch_bounds__(256) kquant_to_f16_kernel(const uint8_t* w, int rows, int cols, __half* out) {
  pdl_wait();
  pdl_launch_dependents();
  const int bpr = cols / 256;
  const size_t units = static_cast<size_t>(rows) * bpr * 4;
  for (size_t u = blockIdx.x * 256ull + threadIdx.x; u < units; u += static_cast<size_t>(gridDim.x) * 256) {
    const size_t blk = u >> 2;
    const int unit = static_cast<int>(u & 3);
    const size_t row = blk / bpr;
    const int kb = static_cast<int>(blk % bpr);
    __half2 v[32];
    unit_dequant_h2<QT>(w + blk * kquant_block_bytes(QT), unit, v);
    __half* dst = out + row * cols + kb * 256;
#pragma unroll
    for (int e = 0; e < 64; e += 2) *reinterpret_cast<__half2*>(dst + unit_col<QT>(unit, e)) = v[e / 2];
  }
}

static __global__ void __launch_bounds__(256) x_to_f16_kernel(const float* x, int x_ld, int T, int cols, __half* out) {
  pdl_wait();
  pdl_launch_dependents();
  const int q4 = cols / 4;
  const size_t n = static_cast<size_t>(T) * q4;
  for (size_t i = blockIdx.x * 256ull + threadIdx.x; i < n; i += static_cast<size_t>(gridDim.x) * 256) {
    const size_t t = i / q4;
    const int c = static_cast<int>(i % q4) * 4;
    const float4 v = *reinterpret_cast<const float4*>(x + t * x_ld + c);
    __half2* d = reinterpret_cast<__half2*>(out + t * cols + c);
    d[0] = __floats2half2_rn(v.x, v.y);
    d[1] = __floats2half2_rn(v.z, v.w);
  }
}

struct GemmF16Params {
  const __half* w;  // [rows][cols]
  const __half* x;  // [T][cols]
  int rows, cols, T;
  float* y;         // [T][y_ld]
  int y_ld;
  const float* resid;
};

// 16-byte cp.async; src_bytes 0 fills the destination with zeros.
KIB_DEV void cp16_zfill(void* sdst, const void* gsrc, int src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(sdst)), "l"(gsrc), "r"(src_bytes)
               : "memory");
}

// CTA tile BM weight rows x BN tokens, K step 64, WR x WC warps (rows x
// tokens), warp tile BM/WR x BN/WC.  Shared rows of 64 halves are padded to 72
// (144 bytes) so the eight rows of an ldmatrix land on distinct banks.
constexpr int kGfK = 64, kGfLd = 72, kGfStages = 3;
template <int BM, int BN>
constexpr size_t gemm_f16w_smem() {
  return static_cast<size_t>(kGfStages) * (BM + BN) * kGfLd * 2;
}

template <int BM, int BN, int WR, int WC>
__global__ void __launch_bounds__(32 * WR * WC, 16 / (WR * WC)) gemm_f16w_kernel(const __grid_constant__ GemmF16Params p) {
  constexpr int NT = 32 * WR * WC;
  constexpr int WM = BM / WR, WN = BN / WC, MI = WM / 16, NJ = WN / 8;
  static_assert(NJ % 2 == 0, "warp tile needs an even number of n8 tiles");
  extern __shared__ __align__(16) uint16_t gf_sm[];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int r0 = blockIdx.x * BM, t0 = blockIdx.y * BN;
  const int wm = (warp % WR) * WM, wn = (warp / WR) * WN;
  const int nk = p.cols / kGfK;
  pdl_wait();
  pdl_launch_dependents();
  auto stage_ptr = [&](int s) { return gf_sm + static_cast<size_t>(s) * (BM + BN) * kGfLd; };
  auto load = [&](int kt, int s) {
    uint16_t* a = stage_ptr(s);
    uint16_t* b = a + BM * kGfLd;
    const int k0 = kt * kGfK;
#pragma unroll
    for (int i = tid; i < BM * 8; i += NT) {
      const int r = i >> 3, piece = i & 7;
      const int row = r0 + r;
      const bool ok = row < p.rows;
      cp16_zfill(a + r * kGfLd + 8 * piece, p.w + static_cast<size_t>(ok ? row : 0) * p.cols + k0 + 8 * piece,
                 ok ? 16 : 0);
    }
#pragma unroll
    for (int i = tid; i < BN * 8; i += NT) {
      const int r = i >> 3, piece = i & 7;
      const int t = t0 + r;
      const bool ok = t < p.T;
      cp16_zfill(b + r * kGfLd + 8 * piece, p.x + static_cast<size_t>(ok ? t : 0) * p.cols + k0 + 8 * piece,
                 ok ? 16 : 0);
    }
  };
  float acc[MI][NJ][4];
#pragma unroll
  for (int i = 0; i < MI; ++i)
#pragma unroll
    for (int j = 0; j < NJ; ++j) acc[i][j][0] = acc[i][j][1] = acc[i][j][2] = acc[i][j][3] = 0.0f;
#pragma unroll
  for (int s = 0; s < kGfStages - 1; ++s) {
    if (s < nk) load(s, s);
    asm volatile("cp.async.commit_group;" ::: "memory");
  }
  for (int kt = 0; kt < nk; ++kt) {
    asm volatile("cp.async.wait_group %0;" ::"n"(kGfStages - 2) : "memory");
    __syncthreads();  // tile kt landed; the stage loaded below was read at kt-1 by everyone
    if (kt + kGfStages - 1 < nk) load(kt + kGfStages - 1, (kt + kGfStages - 1) % kGfStages);
    asm volatile("cp.async.commit_group;" ::: "memory");
    const uint32_t a_base = smem_u32(stage_ptr(kt % kGfStages));
    const uint32_t b_base = a_base + BM * kGfLd * 2;
#pragma unroll
    for (int k0 = 0; k0 < kGfK; k0 += 16) {
      uint32_t a[MI][4];
#pragma unroll
      for (int i = 0; i < MI; ++i) {
        const int row = wm + 16 * i + (lane & 15), col = k0 + (lane >> 4) * 8;
        ldsm_x4(a_base + static_cast<uint32_t>(row * kGfLd + col) * 2, a[i][0], a[i][1], a[i][2], a[i][3]);
      }
#pragma unroll
      for (int j = 0; j < NJ; j += 2) {
        const int n = wn + 8 * j + (lane & 7) + ((lane >> 4) << 3), col = k0 + ((lane >> 3) & 1) * 8;
        uint32_t b0, b1, b2, b3;
        ldsm_x4(b_base + static_cast<uint32_t>(n * kGfLd + col) * 2, b0, b1, b2, b3);
#pragma unroll
        for (int i = 0; i < MI; ++i) {
          mma_f16_16816(acc[i][j], a[i], b0, b1);
          mma_f16_16816(acc[i][j + 1], a[i], b2, b3);
        }
      }
    }
  }
  asm volatile("cp.async.wait_all;" ::: "memory");
  const int g = lane >> 2, q = lane & 3;
#pragma unroll
  for (int i = 0; i < MI; ++i)
#pragma unroll
    for (int j = 0; j < NJ; ++j)
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int row = r0 + wm + 16 * i + g + (c >> 1) * 8;
        const int t = t0 + wn + 8 * j + 2 * q + (c & 1);
        if (row < p.rows && t < p.T) {
          float v = acc[i][j][c];
          if (p.resid) v += p.resid[static_cast<size_t>(t) * p.y_ld + row];
          p.y[static_cast<size_t>(t) * p.y_ld + row] = v;
        }
      }
}

// ======================================================= prefill attention (tensor cores)
// Prefill step 2 for T >= 64 (flash256 numerics, attention_f32_batched_flash256_f16_kv,
// mps_backend.mm:3398-3640): Q rounded to half, K and V f16 from the cache,
// scores and the online softmax in fp32 (running max and normaliser per block
// of keys, masked keys get weight 0), weights kept in fp32 against f16 V, the
// output divided by the normaliser and multiplied by sigmoid(gate).
// On the tensor cores (mma.sync m16n8k16 f16 x f16 -> f32): S = Q K^T is exact
// per product; P V runs as P_hi V + P_lo V with P_hi = half(P), P_lo =
// half(P - P_hi), so the weights keep ~22 bits against V as in fp32.
// A CTA owns 64 queries of one head (4 warps x 16 rows, the output rows in
// registers); K and V tiles of 32 keys are double-buffered by cp.async.
// Shared rows are padded to 264 halves so the ldmatrix rows spread over banks.
constexpr int kFaQ = 64, kFaK = 32, kFaLd = 264;
constexpr size_t kFaSmem = static_cast<size_t>(kFaQ + 4 * kFaK) * kFaLd * 2;

KIB_DEV void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

KIB_DEV uint32_t h2_bits(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }

static __global__ void __launch_bounds__(128, 2) attn_prefill_mma_kernel(const __grid_constant__ AttnParams p) {
  extern __shared__ __align__(16) uint16_t fa_sm[];
  uint16_t* qs = fa_sm;                   // [64][264]
  uint16_t* ks = fa_sm + kFaQ * kFaLd;    // [2][32][264]
  uint16_t* vs = ks + 2 * kFaK * kFaLd;   // [2][32][264]
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int head = blockIdx.y, q0 = blockIdx.x * kFaQ;
  const int kvh = head / (p.heads / p.kv_heads);
  const int kvd = p.kv_heads * kHd;
  pdl_wait();
  pdl_launch_dependents();
  const int pos0 = *p.pos;
  const int last_q = min(q0 + kFaQ, p.T) - 1;
  const int nkeys = pos0 + last_q + 1;
  const int nblocks = (nkeys + kFaK - 1) / kFaK;
  const uint16_t* kg = p.kcache + static_cast<size_t>(kvh) * kHd;
  const uint16_t* vg = p.vcache + static_cast<size_t>(kvh) * kHd;
  auto load_kv = [&](int b, int stage) {
    uint16_t* kd = ks + stage * kFaK * kFaLd;
    uint16_t* vd = vs + stage * kFaK * kFaLd;
#pragma unroll
    for (int it = 0; it < kFaK * 32 / 128; ++it) {
      const int i = tid + 128 * it, r = i >> 5, piece = i & 31;
      const size_t key = static_cast<size_t>(min(b * kFaK + r, nkeys - 1));
      gs_cp16(kd + r * kFaLd + 8 * piece, kg + key * kvd + 8 * piece);
      gs_cp16(vd + r * kFaLd + 8 * piece, vg + key * kvd + 8 * piece);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  load_kv(0, 0);
  // Q rows, rounded to half (rows past T are zero and never written out)
  for (int i = tid; i < kFaQ * (kHd / 4); i += 128) {
    const int r = i / (kHd / 4), c4 = i % (kHd / 4);
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (q0 + r < p.T)
      v = *reinterpret_cast<const float4*>(p.q_out + (static_cast<size_t>(q0 + r) * p.heads + head) * kHd + 4 * c4);
    __half2* d = reinterpret_cast<__half2*>(qs + r * kFaLd + 4 * c4);
    d[0] = __floats2half2_rn(v.x, v.y);
    d[1] = __floats2half2_rn(v.z, v.w);
  }
  const int g = lane >> 2, c = lane & 3;
  const int qpos0 = pos0 + q0 + 16 * warp + g, qpos1 = qpos0 + 8;
  const int warp_last = pos0 + q0 + 16 * warp + 15;  // last key any row of this warp sees
  const float scale = 1.0f / sqrtf(static_cast<float>(kHd));
  const uint32_t qs_base = smem_u32(qs), ks_base = smem_u32(ks), vs_base = smem_u32(vs);
  float o[kHd / 8][4];
#pragma unroll
  for (int n = 0; n < kHd / 8; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.0f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.0f, l1 = 0.0f;  // l: this lane's share
  for (int b = 0; b < nblocks; ++b) {
    asm volatile("cp.async.wait_all;" ::: "memory");
    __syncthreads();  // block b landed (and Q, at b == 0); the other stage is free
    if (b + 1 < nblocks) load_kv(b + 1, (b + 1) & 1);
    if (b * kFaK > warp_last) continue;
    const uint32_t kst = ks_base + static_cast<uint32_t>((b & 1) * kFaK * kFaLd) * 2;
    const uint32_t vst = vs_base + static_cast<uint32_t>((b & 1) * kFaK * kFaLd) * 2;
    float s[4][4];
#pragma unroll
    for (int j = 0; j < 4; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.0f;
#pragma unroll 4
    for (int k0 = 0; k0 < kHd; k0 += 16) {
      uint32_t a[4];
      ldsm_x4(qs_base + static_cast<uint32_t>((16 * warp + (lane & 15)) * kFaLd + k0 + (lane >> 4) * 8) * 2, a[0], a[1],
              a[2], a[3]);
#pragma unroll
      for (int j = 0; j < 4; j += 2) {
        const int n = 8 * j + (lane & 7) + ((lane >> 4) << 3), col = k0 + ((lane >> 3) & 1) * 8;
        uint32_t b0, b1, b2, b3;
        ldsm_x4(kst + static_cast<uint32_t>(n * kFaLd + col) * 2, b0, b1, b2, b3);
        mma_f16_16816(s[j], a, b0, b1);
        mma_f16_16816(s[j + 1], a, b2, b3);
      }
    }
    float mx0 = m0, mx1 = m1;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int key = b * kFaK + 8 * j + 2 * c;
      s[j][0] = key <= qpos0 ? s[j][0] * scale : -INFINITY;
      s[j][1] = key + 1 <= qpos0 ? s[j][1] * scale : -INFINITY;
      s[j][2] = key <= qpos1 ? s[j][2] * scale : -INFINITY;
      s[j][3] = key + 1 <= qpos1 ? s[j][3] * scale : -INFINITY;
      mx0 = fmaxf(mx0, fmaxf(s[j][0], s[j][1]));
      mx1 = fmaxf(mx1, fmaxf(s[j][2], s[j][3]));
    }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    // key 0 is in block 0 for every row, so the running max is finite from then on
    const float ps0 = expf(m0 - mx0), ps1 = expf(m1 - mx1);
    m0 = mx0;
    m1 = mx1;
    float rs0 = 0.0f, rs1 = 0.0f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      s[j][0] = expf(s[j][0] - m0);
      s[j][1] = expf(s[j][1] - m0);
      s[j][2] = expf(s[j][2] - m1);
      s[j][3] = expf(s[j][3] - m1);
      rs0 += s[j][0] + s[j][1];
      rs1 += s[j][2] + s[j][3];
    }
    l0 = l0 * ps0 + rs0;
    l1 = l1 * ps1 + rs1;
#pragma unroll
    for (int n = 0; n < kHd / 8; ++n) {
      o[n][0] *= ps0;
      o[n][1] *= ps0;
      o[n][2] *= ps1;
      o[n][3] *= ps1;
    }
#pragma unroll
    for (int kk = 0; kk < 2; ++kk) {
      uint32_t ahi[4], alo[4];
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        // a0: row g keys 2c.. of tile 2kk; a1: row g+8; a2/a3: tile 2kk+1
        const float x = s[2 * kk + (h >> 1)][(h & 1) * 2], y = s[2 * kk + (h >> 1)][(h & 1) * 2 + 1];
        const __half2 hi = __floats2half2_rn(x, y);
        const float2 hf = __half22float2(hi);
        ahi[h] = h2_bits(hi);
        alo[h] = h2_bits(__floats2half2_rn(x - hf.x, y - hf.y));
      }
      const int key = 16 * kk + (lane & 7) + ((lane >> 3) & 1) * 8;
#pragma unroll
      for (int nd = 0; nd < kHd / 16; ++nd) {
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(vst + static_cast<uint32_t>(key * kFaLd + 16 * nd + (lane >> 4) * 8) * 2, b0, b1, b2, b3);
        mma_f16_16816(o[2 * nd], ahi, b0, b1);
        mma_f16_16816(o[2 * nd + 1], ahi, b2, b3);
        mma_f16_16816(o[2 * nd], alo, b0, b1);
        mma_f16_16816(o[2 * nd + 1], alo, b2, b3);
      }
    }
  }
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
  const float inv0 = l0 == 0.0f ? 0.0f : 1.0f / l0, inv1 = l1 == 0.0f ? 0.0f : 1.0f / l1;
  const int t0 = q0 + 16 * warp + g, t1 = t0 + 8;
#pragma unroll
  for (int n = 0; n < kHd / 8; ++n) {
    const int d = 8 * n + 2 * c;
    if (t0 < p.T) {
      const float* gt = p.qg + (static_cast<size_t>(t0) * p.heads + head) * 2 * kHd + kHd + d;
      *reinterpret_cast<float2*>(p.out + static_cast<size_t>(t0) * p.heads * kHd + head * kHd + d) =
          make_float2(o[n][0] * inv0 * sigmoid_f(gt[0]), o[n][1] * inv0 * sigmoid_f(gt[1]));
    }
    if (t1 < p.T) {
      const float* gt = p.qg + (static_cast<size_t>(t1) * p.heads + head) * 2 * kHd + kHd + d;
      *reinterpret_cast<float2*>(p.out + static_cast<size_t>(t1) * p.heads * kHd + head * kHd + d) =
          make_float2(o[n][2] * inv1 * sigmoid_f(gt[0]), o[n][3] * inv1 * sigmoid_f(gt[1]));
    }
  }
}

// The same attention with two query heads of one KV head per CTA (8 warps:
// warps 0-3 the even head, 4-7 the odd one, sharing every K/V tile) and the
// key range split over gridDim.z CTAs, so a 1024-token chunk fills the GPU.
// With one split the output is final, as above; with several, each CTA writes
// its unnormalised rows, running max and normaliser to part
// ([split][T][heads][256 + 2]) and attn_prefill_merge_kernel combines them.
// A split may start past some rows' last key: those rows keep max -inf and
// weight 0 until a key of theirs arrives.
constexpr int kFa2Q = 64;  // queries per head per CTA
constexpr int kFa2MaxSplits = 4;
constexpr int kFa2Blk = 2 * kFaK;  // keys per staged block: two 32-key softmax steps per barrier
constexpr size_t kFa2Smem = static_cast<size_t>(2 * kFa2Q + 4 * kFa2Blk) * kFaLd * 2;

static __global__ void __launch_bounds__(256, 1) attn_prefill_mma2_kernel(const __grid_constant__ AttnParams p) {
  extern __shared__ __align__(16) uint16_t fa2_sm[];
  uint16_t* qs = fa2_sm;                    // [2][64][264]
  uint16_t* ks = fa2_sm + 2 * kFa2Q * kFaLd;  // [2][32][264]
  uint16_t* vs = ks + 2 * kFa2Blk * kFaLd;  // [2][64][264]
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int hl = warp >> 2, wq = warp & 3;  // head of the pair, 16-row tile of it
  const int head0 = 2 * blockIdx.y, head = head0 + hl, q0 = blockIdx.x * kFa2Q;
  const int split = blockIdx.z, nsplit = gridDim.z;
  const int kvh = head0 / (p.heads / p.kv_heads);
  const int kvd = p.kv_heads * kHd;
  pdl_wait();
  pdl_launch_dependents();
  const int pos0 = *p.pos;
  const int last_q = min(q0 + kFa2Q, p.T) - 1;
  const int nkeys = pos0 + last_q + 1;
  const int nblocks = (nkeys + kFa2Blk - 1) / kFa2Blk;
  const int b_lo = static_cast<int>(static_cast<long>(nblocks) * split / nsplit);
  const int b_hi = static_cast<int>(static_cast<long>(nblocks) * (split + 1) / nsplit);
  const uint16_t* kg = p.kcache + static_cast<size_t>(kvh) * kHd;
  const uint16_t* vg = p.vcache + static_cast<size_t>(kvh) * kHd;
  auto load_kv = [&](int b, int stage) {
    uint16_t* kd = ks + stage * kFa2Blk * kFaLd;
    uint16_t* vd = vs + stage * kFa2Blk * kFaLd;
#pragma unroll
    for (int it = 0; it < kFa2Blk * 32 / 256; ++it) {
      const int i = tid + 256 * it, r = i >> 5, piece = i & 31;
      const size_t key = static_cast<size_t>(min(b * kFa2Blk + r, nkeys - 1));
      gs_cp16(kd + r * kFaLd + 8 * piece, kg + key * kvd + 8 * piece);
      gs_cp16(vd + r * kFaLd + 8 * piece, vg + key * kvd + 8 * piece);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  if (b_lo < b_hi) load_kv(b_lo, b_lo & 1);
  // Q rows of both heads, rounded to half (rows past T are zero and never written out)
  for (int i = tid; i < 2 * kFa2Q * (kHd / 4); i += 256) {
    const int r = i / (kHd / 4), c4 = i % (kHd / 4), hh = r / kFa2Q, rr = r % kFa2Q;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (q0 + rr < p.T)
      v = *reinterpret_cast<const float4*>(p.q_out + (static_cast<size_t>(q0 + rr) * p.heads + head0 + hh) * kHd +
                                           4 * c4);
    __half2* d = reinterpret_cast<__half2*>(qs + r * kFaLd + 4 * c4);
    d[0] = __floats2half2_rn(v.x, v.y);
    d[1] = __floats2half2_rn(v.z, v.w);
  }
  const int g = lane >> 2, c = lane & 3;
  const int qpos0 = pos0 + q0 + 16 * wq + g, qpos1 = qpos0 + 8;
  const int warp_last = pos0 + q0 + 16 * wq + 15;  // last key any row of this warp sees
  const float scale = 1.0f / sqrtf(static_cast<float>(kHd));
  const uint32_t qs_base = smem_u32(qs + hl * kFa2Q * kFaLd), ks_base = smem_u32(ks), vs_base = smem_u32(vs);
  float o[kHd / 8][4];
#pragma unroll
  for (int n = 0; n < kHd / 8; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.0f;
  // running max starts at a finite floor: a row whose keys all lie beyond this
  // split's blocks keeps weight e^{-inf - floor} = 0 and scale e^0 = 1, and its
  // first key zeroes the (empty) history exactly as a -inf start would
  constexpr float kFloor = -1e30f;
  float m0 = kFloor, m1 = kFloor, l0 = 0.0f, l1 = 0.0f;  // l: this lane's share
  for (int bb = 2 * b_lo; bb < 2 * b_hi; ++bb) {
    const int b = bb >> 1;  // staged block; bb: its 32-key half
    if ((bb & 1) == 0) {
      asm volatile("cp.async.wait_all;" ::: "memory");
      __syncthreads();  // block b landed (and Q, at the first block); the other stage is free
      if (b + 1 < b_hi) load_kv(b + 1, (b + 1) & 1);
    }
    if (bb * kFaK > warp_last) continue;
    const uint32_t kst = ks_base + static_cast<uint32_t>(((b & 1) * kFa2Blk + (bb & 1) * kFaK) * kFaLd) * 2;
    const uint32_t vst = vs_base + static_cast<uint32_t>(((b & 1) * kFa2Blk + (bb & 1) * kFaK) * kFaLd) * 2;
    float s[4][4];
#pragma unroll
    for (int j = 0; j < 4; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.0f;
#pragma unroll 4
    for (int k0 = 0; k0 < kHd; k0 += 16) {
      uint32_t a[4];
      ldsm_x4(qs_base + static_cast<uint32_t>((16 * wq + (lane & 15)) * kFaLd + k0 + (lane >> 4) * 8) * 2, a[0], a[1],
              a[2], a[3]);
#pragma unroll
      for (int j = 0; j < 4; j += 2) {
        const int n = 8 * j + (lane & 7) + ((lane >> 4) << 3), col = k0 + ((lane >> 3) & 1) * 8;
        uint32_t b0, b1, b2, b3;
        ldsm_x4(kst + static_cast<uint32_t>(n * kFaLd + col) * 2, b0, b1, b2, b3);
        mma_f16_16816(s[j], a, b0, b1);
        mma_f16_16816(s[j + 1], a, b2, b3);
      }
    }
    float mx0 = m0, mx1 = m1;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int key = bb * kFaK + 8 * j + 2 * c;
      s[j][0] = key <= qpos0 ? s[j][0] * scale : -INFINITY;
      s[j][1] = key + 1 <= qpos0 ? s[j][1] * scale : -INFINITY;
      s[j][2] = key <= qpos1 ? s[j][2] * scale : -INFINITY;
      s[j][3] = key + 1 <= qpos1 ? s[j][3] * scale : -INFINITY;
      mx0 = fmaxf(mx0, fmaxf(s[j][0], s[j][1]));
      mx1 = fmaxf(mx1, fmaxf(s[j][2], s[j][3]));
    }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    const float ps0 = expf(m0 - mx0), ps1 = expf(m1 - mx1);
    m0 = mx0;
    m1 = mx1;
    float rs0 = 0.0f, rs1 = 0.0f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      s[j][0] = expf(s[j][0] - m0);
      s[j][1] = expf(s[j][1] - m0);
      s[j][2] = expf(s[j][2] - m1);
      s[j][3] = expf(s[j][3] - m1);
      rs0 += s[j][0] + s[j][1];
      rs1 += s[j][2] + s[j][3];
    }
    l0 = l0 * ps0 + rs0;
    l1 = l1 * ps1 + rs1;
#pragma unroll
    for (int n = 0; n < kHd / 8; ++n) {
      o[n][0] *= ps0;
      o[n][1] *= ps0;
      o[n][2] *= ps1;
      o[n][3] *= ps1;
    }
#pragma unroll
    for (int kk = 0; kk < 2; ++kk) {
      uint32_t ahi[4], alo[4];
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        const float x = s[2 * kk + (h >> 1)][(h & 1) * 2], y = s[2 * kk + (h >> 1)][(h & 1) * 2 + 1];
        const __half2 hi = __floats2half2_rn(x, y);
        const float2 hf = __half22float2(hi);
        ahi[h] = h2_bits(hi);
        alo[h] = h2_bits(__floats2half2_rn(x - hf.x, y - hf.y));
      }
      const int key = 16 * kk + (lane & 7) + ((lane >> 3) & 1) * 8;
#pragma unroll
      for (int nd = 0; nd < kHd / 16; ++nd) {
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(vst + static_cast<uint32_t>(key * kFaLd + 16 * nd + (lane >> 4) * 8) * 2, b0, b1, b2, b3);
        mma_f16_16816(o[2 * nd], ahi, b0, b1);
        mma_f16_16816(o[2 * nd + 1], ahi, b2, b3);
        mma_f16_16816(o[2 * nd], alo, b0, b1);
        mma_f16_16816(o[2 * nd + 1], alo, b2, b3);
      }
    }
  }
  asm volatile("cp.async.wait_all;" ::: "memory");
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
  const int t0 = q0 + 16 * wq + g, t1 = t0 + 8;
  if (nsplit == 1) {
    const float inv0 = l0 == 0.0f ? 0.0f : 1.0f / l0, inv1 = l1 == 0.0f ? 0.0f : 1.0f / l1;
#pragma unroll
    for (int n = 0; n < kHd / 8; ++n) {
      const int d = 8 * n + 2 * c;
      if (t0 < p.T) {
        const float* gt = p.qg + (static_cast<size_t>(t0) * p.heads + head) * 2 * kHd + kHd + d;
        *reinterpret_cast<float2*>(p.out + static_cast<size_t>(t0) * p.heads * kHd + head * kHd + d) =
            make_float2(o[n][0] * inv0 * sigmoid_f(gt[0]), o[n][1] * inv0 * sigmoid_f(gt[1]));
      }
      if (t1 < p.T) {
        const float* gt = p.qg + (static_cast<size_t>(t1) * p.heads + head) * 2 * kHd + kHd + d;
        *reinterpret_cast<float2*>(p.out + static_cast<size_t>(t1) * p.heads * kHd + head * kHd + d) =
            make_float2(o[n][2] * inv1 * sigmoid_f(gt[0]), o[n][3] * inv1 * sigmoid_f(gt[1]));
      }
    }
    return;
  }
  float* part = p.part + static_cast<size_t>(split) * p.T * p.heads * (kHd + 2);
  float* r0p = part + (static_cast<size_t>(t0) * p.heads + head) * (kHd + 2);
  float* r1p = part + (static_cast<size_t>(t1) * p.heads + head) * (kHd + 2);
#pragma unroll
  for (int n = 0; n < kHd / 8; ++n) {
    const int d = 8 * n + 2 * c;
    if (t0 < p.T) *reinterpret_cast<float2*>(r0p + d) = make_float2(o[n][0], o[n][1]);
    if (t1 < p.T) *reinterpret_cast<float2*>(r1p + d) = make_float2(o[n][2], o[n][3]);
  }
  if (c == 0) {
    if (t0 < p.T) *reinterpret_cast<float2*>(r0p + kHd) = make_float2(m0, l0);
    if (t1 < p.T) *reinterpret_cast<float2*>(r1p + kHd) = make_float2(m1, l1);
  }
}

// Combines the splits of attn_prefill_mma2_kernel: weights e^{m_s - max m},
// output = sum_s w_s O_s / sum_s w_s l_s, times sigmoid(gate).  One CTA per
// (token, head), one thread per output element.
static __global__ void __launch_bounds__(256) attn_prefill_merge_kernel(const __grid_constant__ AttnParams p,
                                                                        int nsplit) {
  pdl_wait();
  pdl_launch_dependents();
  const int t = blockIdx.x, head = blockIdx.y, d = threadIdx.x;
  const size_t stride = static_cast<size_t>(p.T) * p.heads * (kHd + 2);
  const float* base = p.part + (static_cast<size_t>(t) * p.heads + head) * (kHd + 2);
  float mx = -INFINITY;
  for (int s = 0; s < nsplit; ++s) mx = fmaxf(mx, base[s * stride + kHd]);
  float o = 0.0f, l = 0.0f;
  for (int s = 0; s < nsplit; ++s) {
    // a split that held none of the row's keys reports the floor max and l = 0
    const float ms = base[s * stride + kHd], ls = base[s * stride + kHd + 1];
    const float w = expf(ms - mx);
    o += w * base[s * stride + d];
    l += w * ls;
  }
  const float gt = p.qg[(static_cast<size_t>(t) * p.heads + head) * 2 * kHd + kHd + d];
  p.out[static_cast<size_t>(t) * p.heads * kHd + head * kHd + d] = (l == 0.0f ? 0.0f : o / l) * sigmoid_f(gt);
}

}  // namespace kib
