// gdn_chunk.cuh -- chunked delta rule for prefill (T >= 64 tokens).
//
// The reference runs the gated delta rule token by token
// (gated_delta_net_f32_batched_qwen35, mps_backend.mm:2307-2374):
//   S_v *= exp(g);  u = (v_v - S_v . k) * beta;  S_v += u * k;  y_v = S_v . q / sqrt(128)
// for every value row v of a head's 128 x 128 state.  Over a chunk of C = 64
// tokens with log-decay prefix sums G_i = g_1 + .. + g_i the same recurrence
// has a closed form (the WY / UT representation of a product of rank-one
// updates).  With S0 the state before the chunk,
//   u_i = beta_i (v_i - e^{G_i} S0 k_i - sum_{j<i} e^{G_i - G_j} (k_j . k_i) u_j)
// i.e. (I + L) U = diag(beta) (V - diag(e^G) K S0^T),
//   L_ij = beta_i e^{G_i - G_j} (k_i . k_j) for j < i,
// so with Tb = (I + L)^{-1} diag(beta) and Kt = Tb diag(e^G) K:
//   U   = Tb V - Kt S0^T
//   Y   = (diag(e^G) Q S0^T + P U) / sqrt(128),  P_ij = e^{G_i - G_j} (q_i . k_j), j <= i
//   S_C = e^{G_C} S0 + U^T diag(e^{G_C - G}) K.
// gdn_chunk_prep_kernel computes Tb, P, Kt and G for every (head, chunk) at
// once -- they do not depend on the state -- and gdn_chunk_scan_kernel walks
// the chunks in order for 16 value rows of one head per CTA: the per-token
// dependent chain of the reference becomes 16 steps of small fp32 matrix
// products.  Same arithmetic type (fp32) as the reference; only the order of
// the roundings differs.  Tokens past the end of the prompt are zero (beta = 0
// and g = 0), so they contribute nothing to U, Y or the state.
#pragma once

#include "kib_common.cuh"

namespace kib {

constexpr int kGc = 64;     // tokens per chunk
constexpr int kGcD = 128;   // head dimension (keys and values)
constexpr int kGcRows = 16; // value rows per scan CTA
// workspace per (head, chunk): Tb [64][64], P [64][64], Kt [64][128], G [64],
// then the decayed operands Qg = e^{G_i} q_i and Kd = e^{G_C - G_j} k_j [64][128]
constexpr int kGcWsQg = kGc * kGc * 2 + kGc * kGcD + kGc;
constexpr int kGcWsKd = kGcWsQg + kGc * kGcD;
constexpr int kGcWs = kGcWsKd + kGc * kGcD;  // workspace floats per (head, chunk)

struct GdnChunkParams {
  const float* conv_out;  // [T][C]: q | k (L2-normalised) | v
  int C;
  const float* g;         // [T][ld_ba] log-decay (softplus(alpha + dt_bias) * ssm_a)
  const float* beta;      // [T][ld_ba] sigmoid(beta)
  int ld_ba;
  float* state;           // [value_heads][128][128]
  float* out;             // [T][value_heads * 128]
  float* ws;              // [value_heads][nchunks][kGcWs]
  int T;
  int key_heads;
  int value_heads;
};

// 16-byte global -> shared copy without a register destination; valid false
// writes zeros (source size 0), so every copy of a chunk is in flight at once.
KIB_DEV void gc_cp16(void* sdst, const void* gsrc, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(sdst)), "l"(gsrc), "r"(valid ? 16 : 0)
               : "memory");
}
KIB_DEV void gc_cp_wait() {
  asm volatile("cp.async.commit_group;\n\tcp.async.wait_all;" ::: "memory");
}

// ---------------------------------------------------------------- prep
// One CTA per (value head, chunk), 256 threads.
constexpr int kGcTs = 68;  // padded token stride of the transposed q/k tiles
constexpr size_t kGcPrepSmem = (2 * kGcD * kGcTs + 2 * kGc * kGcD + 2 * kGc * (kGc + 1) + 3 * kGc) * sizeof(float);

__global__ void __launch_bounds__(256) gdn_chunk_prep_kernel(const __grid_constant__ GdnChunkParams p) {
  extern __shared__ __align__(16) float gc_sm[];
  float* kT = gc_sm;                      // [128][68]: k^T
  float* qT = kT + kGcD * kGcTs;          // [128][68]: q^T
  float* kr = qT + kGcD * kGcTs;          // [64][128]: k rows
  float* qr = kr + kGc * kGcD;            // [64][128]: q rows
  float* Lm = qr + kGc * kGcD;            // [64][65]: L, then X = (I + L)^{-1}
  float* Xm = Lm + kGc * (kGc + 1);       // [64][65]
  float* G = Xm + kGc * (kGc + 1);        // [64]
  float* bt = G + kGc;                    // [64]
  float* eG = bt + kGc;                   // [64]
  const int h = blockIdx.x, c = blockIdx.y, tid = threadIdx.x;
  const int kh = h % p.key_heads;
  const int t0 = c * kGc, n = min(kGc, p.T - t0);
  const int key_dim = p.key_heads * kGcD;
  pdl_wait();
  pdl_launch_dependents();
  for (int i = tid; i < kGc * kGcD / 4; i += 256) {
    const int t = i >> 5, d4 = i & 31;
    const bool ok = t < n;
    const float* row = p.conv_out + static_cast<size_t>(t0 + (ok ? t : 0)) * p.C;
    gc_cp16(qr + t * kGcD + 4 * d4, row + kh * kGcD + 4 * d4, ok);
    gc_cp16(kr + t * kGcD + 4 * d4, row + key_dim + kh * kGcD + 4 * d4, ok);
  }
  if (tid < kGc) {
    const bool ok = tid < n;
    G[tid] = ok ? p.g[static_cast<size_t>(t0 + tid) * p.ld_ba + h] : 0.0f;
    bt[tid] = ok ? p.beta[static_cast<size_t>(t0 + tid) * p.ld_ba + h] : 0.0f;
  }
  gc_cp_wait();
  __syncthreads();
  // transposed copies for the K K^T / Q K^T tiles
  for (int i = tid; i < kGc * kGcD; i += 256) {
    const int d = i & 127, t = i >> 7;  // lanes along d: conflict-free reads, 4-way writes (stride 68)
    kT[d * kGcTs + t] = kr[t * kGcD + d];
    qT[d * kGcTs + t] = qr[t * kGcD + d];
  }
  if (tid == 0) {
    float acc = 0.0f;
    for (int i = 0; i < kGc; ++i) {
      acc += G[i];
      G[i] = acc;
    }
  }
  __syncthreads();
  if (tid < kGc) eG[tid] = expf(G[tid]);
  // KK and QK in 4 x 4 register tiles: thread (ti, tj) owns rows 4ti.., cols 4tj..
  const int ti = tid >> 4, tj = tid & 15;
  float kk[4][4], qk[4][4];
#pragma unroll
  for (int a = 0; a < 4; ++a)
#pragma unroll
    for (int b = 0; b < 4; ++b) kk[a][b] = qk[a][b] = 0.0f;
#pragma unroll 4
  for (int d = 0; d < kGcD; ++d) {
    const float4 ki = *reinterpret_cast<const float4*>(kT + d * kGcTs + 4 * ti);
    const float4 qi = *reinterpret_cast<const float4*>(qT + d * kGcTs + 4 * ti);
    const float4 kj = *reinterpret_cast<const float4*>(kT + d * kGcTs + 4 * tj);
    const float kia[4] = {ki.x, ki.y, ki.z, ki.w}, qia[4] = {qi.x, qi.y, qi.z, qi.w};
    const float kja[4] = {kj.x, kj.y, kj.z, kj.w};
#pragma unroll
    for (int a = 0; a < 4; ++a)
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        kk[a][b] = fmaf(kia[a], kja[b], kk[a][b]);
        qk[a][b] = fmaf(qia[a], kja[b], qk[a][b]);
      }
  }
  __syncthreads();
  float* ws = p.ws + (static_cast<size_t>(h) * gridDim.y + c) * kGcWs;
  float* wTb = ws;
  float* wP = ws + kGc * kGc;
  float* wKt = wP + kGc * kGc;
  float* wG = wKt + kGc * kGcD;
#pragma unroll
  for (int a = 0; a < 4; ++a)
#pragma unroll
    for (int b = 0; b < 4; ++b) {
      const int i = 4 * ti + a, j = 4 * tj + b;
      const float dec = j <= i ? expf(G[i] - G[j]) : 0.0f;
      Lm[i * (kGc + 1) + j] = j < i ? bt[i] * dec * kk[a][b] : 0.0f;
      wP[i * kGc + j] = dec * qk[a][b];
    }
  __syncthreads();
  // X = (I + L)^{-1} by forward substitution, row by row: four threads per
  // column split the sum over j < i
  {
    const int col = tid >> 2, part = tid & 3;
    for (int i = 0; i < kGc; ++i) {
      float s = 0.0f;
      for (int j = part; j < i; j += 4) s = fmaf(Lm[i * (kGc + 1) + j], Xm[j * (kGc + 1) + col], s);
      s += __shfl_xor_sync(0xffffffffu, s, 1);
      s += __shfl_xor_sync(0xffffffffu, s, 2);
      if (part == 0) Xm[i * (kGc + 1) + col] = (i == col ? 1.0f : 0.0f) - s;
      __syncthreads();
    }
  }
  // Tb = X diag(beta), then Kt = Tb diag(e^G) K (thread: 4 rows x 8 columns)
  for (int e = tid; e < kGc * kGc; e += 256) {
    const int i = e >> 6, j = e & 63;
    const float v = Xm[i * (kGc + 1) + j] * bt[j];
    wTb[e] = v;
    Lm[i * (kGc + 1) + j] = v * eG[j];  // Tb diag(e^G), reused below
  }
  if (tid < kGc) wG[tid] = G[tid];
  __syncthreads();
  {
    const int ig = tid >> 4, dg = tid & 15;
    float acc[4][8];
#pragma unroll
    for (int a = 0; a < 4; ++a)
#pragma unroll
      for (int b = 0; b < 8; ++b) acc[a][b] = 0.0f;
#pragma unroll 2
    for (int j = 0; j < kGc; ++j) {
      const float4 k0 = *reinterpret_cast<const float4*>(kr + j * kGcD + 8 * dg);
      const float4 k1 = *reinterpret_cast<const float4*>(kr + j * kGcD + 8 * dg + 4);
      const float kv[8] = {k0.x, k0.y, k0.z, k0.w, k1.x, k1.y, k1.z, k1.w};
#pragma unroll
      for (int a = 0; a < 4; ++a) {
        const float t = Lm[(4 * ig + a) * (kGc + 1) + j];
#pragma unroll
        for (int b = 0; b < 8; ++b) acc[a][b] = fmaf(t, kv[b], acc[a][b]);
      }
    }
#pragma unroll
    for (int a = 0; a < 4; ++a) {
      float* o = wKt + (4 * ig + a) * kGcD + 8 * dg;
      *reinterpret_cast<float4*>(o) = make_float4(acc[a][0], acc[a][1], acc[a][2], acc[a][3]);
      *reinterpret_cast<float4*>(o + 4) = make_float4(acc[a][4], acc[a][5], acc[a][6], acc[a][7]);
    }
  }
  // the scan's decayed operands: q rows by e^{G_i}, k rows by e^{G_C - G_j}
  {
    float* wQg = ws + kGcWsQg;
    float* wKd = ws + kGcWsKd;
    const float gend = G[kGc - 1];
    for (int i = tid; i < kGc * kGcD / 4; i += 256) {
      const int t = i >> 5;
      const float fq = expf(G[t]), fk = expf(gend - G[t]);
      const float4 qv = reinterpret_cast<const float4*>(qr)[i], kv = reinterpret_cast<const float4*>(kr)[i];
      reinterpret_cast<float4*>(wQg)[i] = make_float4(qv.x * fq, qv.y * fq, qv.z * fq, qv.w * fq);
      reinterpret_cast<float4*>(wKd)[i] = make_float4(kv.x * fk, kv.y * fk, kv.z * fk, kv.w * fk);
    }
  }
}

// ---------------------------------------------------------------- scan
// One CTA per (value head, 16 value rows), 256 threads; walks the chunks.
constexpr int kGcSr = kGcD + 4;  // padded state row
constexpr size_t kGcScanSmem =
    (3 * kGc * kGcD + 2 * kGc * kGc + kGc * kGcRows * 4 + kGcRows * kGcSr + 2 * kGc) * sizeof(float);

__global__ void __launch_bounds__(256) gdn_chunk_scan_kernel(const __grid_constant__ GdnChunkParams p) {
  extern __shared__ __align__(16) float gs_sm[];
  float* sKt = gs_sm;                 // [64][128]
  float* sKd = sKt + kGc * kGcD;      // [64][128]: e^{G_C - G_j} k_j
  float* sQg = sKd + kGc * kGcD;      // [64][128]: e^{G_i} q_i
  float* sTb = sQg + kGc * kGcD;      // [64][64]
  float* sP = sTb + kGc * kGc;        // [64][64]
  float* sV = sP + kGc * kGc;         // [64][16]
  float* sX1 = sV + kGc * kGcRows;    // [64][16]
  float* sX2 = sX1 + kGc * kGcRows;   // [64][16]
  float* sU = sX2 + kGc * kGcRows;    // [64][16]
  float* sS = sU + kGc * kGcRows;     // [16][132]: the state rows
  float* sG = sS + kGcRows * kGcSr;   // [64]
  float* sE = sG + kGc;               // [64]: e^{G}
  const int h = blockIdx.x, r0 = blockIdx.y * kGcRows, tid = threadIdx.x;
  const int kh = h % p.key_heads;
  const int key_dim = p.key_heads * kGcD;
  const int nchunks = (p.T + kGc - 1) / kGc;
  float* S = p.state + (static_cast<size_t>(h) * kGcD + r0) * kGcD;
  for (int i = tid; i < kGcRows * kGcD / 4; i += 256) {
    const int r = i >> 5, d4 = i & 31;
    *reinterpret_cast<float4*>(sS + r * kGcSr + 4 * d4) = reinterpret_cast<const float4*>(S + r * kGcD)[d4];
  }
  pdl_wait();
  pdl_launch_dependents();
  const float scale = 1.0f / sqrtf(static_cast<float>(kGcD));
  const size_t out_ld = static_cast<size_t>(p.value_heads) * kGcD;
  const int r = tid & 15, ig = tid >> 4;  // output mapping: value row r, chunk rows 4ig..4ig+3
  for (int c = 0; c < nchunks; ++c) {
    const int t0 = c * kGc, n = min(kGc, p.T - t0);
    const float* ws = p.ws + (static_cast<size_t>(h) * nchunks + c) * kGcWs;
    for (int i = tid; i < kGc * kGc / 4; i += 256) {
      gc_cp16(sTb + 4 * i, ws + 4 * i, true);
      gc_cp16(sP + 4 * i, ws + kGc * kGc + 4 * i, true);
    }
    for (int i = tid; i < kGc * kGcD / 4; i += 256) {
      const int t = i >> 5, d4 = i & 31;
      const bool ok = t < n;
      const float* row = p.conv_out + static_cast<size_t>(t0 + (ok ? t : 0)) * p.C;
      gc_cp16(sKt + 4 * i, ws + 2 * kGc * kGc + 4 * i, true);
      gc_cp16(sQg + 4 * i, row + kh * kGcD + 4 * d4, ok);
      gc_cp16(sKd + 4 * i, row + key_dim + kh * kGcD + 4 * d4, ok);
    }
    {
      const int t = tid >> 2, q4 = tid & 3;  // 64 tokens x 4 pieces of the CTA's 16 value rows
      const bool ok = t < n;
      gc_cp16(sV + t * kGcRows + 4 * q4,
              p.conv_out + static_cast<size_t>(t0 + (ok ? t : 0)) * p.C + 2 * key_dim + h * kGcD + r0 + 4 * q4, ok);
    }
    if (tid < kGc / 4) gc_cp16(sG + 4 * tid, ws + 2 * kGc * kGc + kGc * kGcD + 4 * tid, true);
    gc_cp_wait();
    __syncthreads();
    const float gend = sG[kGc - 1];
    if (tid < kGc) sE[tid] = expf(sG[tid]);
    // scale in place: k rows by e^{G_C - G_j}, q rows by e^{G_i}
    for (int i = tid; i < kGc * kGcD / 4; i += 256) {
      const int t = i >> 5;
      const float fk = expf(gend - sG[t]), fq = expf(sG[t]);
      float4 kq = reinterpret_cast<float4*>(sKd)[i], qq = reinterpret_cast<float4*>(sQg)[i];
      reinterpret_cast<float4*>(sKd)[i] = make_float4(kq.x * fk, kq.y * fk, kq.z * fk, kq.w * fk);
      reinterpret_cast<float4*>(sQg)[i] = make_float4(qq.x * fq, qq.y * fq, qq.z * fq, qq.w * fq);
    }
    __syncthreads();
    // X1 = Kt S0^T, X2 = (e^G Q) S0^T for rows 4ig.. and value row r
    {
      float x1[4] = {0.f, 0.f, 0.f, 0.f}, x2[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 4
      for (int d = 0; d < kGcD; d += 4) {
        const float4 s4 = *reinterpret_cast<const float4*>(sS + r * kGcSr + d);
#pragma unroll
        for (int a = 0; a < 4; ++a) {
          const float4 kt = *reinterpret_cast<const float4*>(sKt + (4 * ig + a) * kGcD + d);
          const float4 qg = *reinterpret_cast<const float4*>(sQg + (4 * ig + a) * kGcD + d);
          x1[a] = fmaf(kt.x, s4.x, fmaf(kt.y, s4.y, fmaf(kt.z, s4.z, fmaf(kt.w, s4.w, x1[a]))));
          x2[a] = fmaf(qg.x, s4.x, fmaf(qg.y, s4.y, fmaf(qg.z, s4.z, fmaf(qg.w, s4.w, x2[a]))));
        }
      }
#pragma unroll
      for (int a = 0; a < 4; ++a) {
        sX1[(4 * ig + a) * kGcRows + r] = x1[a];
        sX2[(4 * ig + a) * kGcRows + r] = x2[a];
      }
    }
    __syncthreads();
    // U = Tb V - X1
    {
      float u[4];
#pragma unroll
      for (int a = 0; a < 4; ++a) u[a] = -sX1[(4 * ig + a) * kGcRows + r];
#pragma unroll 4
      for (int j = 0; j < kGc; ++j) {
        const float v = sV[j * kGcRows + r];
#pragma unroll
        for (int a = 0; a < 4; ++a) u[a] = fmaf(sTb[(4 * ig + a) * kGc + j], v, u[a]);
      }
#pragma unroll
      for (int a = 0; a < 4; ++a) sU[(4 * ig + a) * kGcRows + r] = u[a];
    }
    __syncthreads();
    // Y = (X2 + P U) * scale
    {
#pragma unroll
      for (int a = 0; a < 4; ++a) {
        const int i = 4 * ig + a;
        float y = sX2[i * kGcRows + r];
        for (int j = 0; j <= i; ++j) y = fmaf(sP[i * kGc + j], sU[j * kGcRows + r], y);
        if (i < n) p.out[static_cast<size_t>(t0 + i) * out_ld + h * kGcD + r0 + r] = y * scale;
      }
    }
    // S = e^{G_C} S + U^T Kd (thread: value row r, columns 8dg..8dg+7)
    {
      const int dg = tid >> 4;
      const float eg = expf(gend);
      float acc[8];
      const float4 a0 = *reinterpret_cast<const float4*>(sS + r * kGcSr + 8 * dg);
      const float4 a1 = *reinterpret_cast<const float4*>(sS + r * kGcSr + 8 * dg + 4);
      acc[0] = a0.x * eg; acc[1] = a0.y * eg; acc[2] = a0.z * eg; acc[3] = a0.w * eg;
      acc[4] = a1.x * eg; acc[5] = a1.y * eg; acc[6] = a1.z * eg; acc[7] = a1.w * eg;
#pragma unroll 4
      for (int j = 0; j < kGc; ++j) {
        const float u = sU[j * kGcRows + r];
        const float4 k0 = *reinterpret_cast<const float4*>(sKd + j * kGcD + 8 * dg);
        const float4 k1 = *reinterpret_cast<const float4*>(sKd + j * kGcD + 8 * dg + 4);
        acc[0] = fmaf(u, k0.x, acc[0]); acc[1] = fmaf(u, k0.y, acc[1]);
        acc[2] = fmaf(u, k0.z, acc[2]); acc[3] = fmaf(u, k0.w, acc[3]);
        acc[4] = fmaf(u, k1.x, acc[4]); acc[5] = fmaf(u, k1.y, acc[5]);
        acc[6] = fmaf(u, k1.z, acc[6]); acc[7] = fmaf(u, k1.w, acc[7]);
      }
      __syncthreads();  // every thread has read the old state rows (X1/X2 long done; the row is shared by 16 threads)
      *reinterpret_cast<float4*>(sS + r * kGcSr + 8 * dg) = make_float4(acc[0], acc[1], acc[2], acc[3]);
      *reinterpret_cast<float4*>(sS + r * kGcSr + 8 * dg + 4) = make_float4(acc[4], acc[5], acc[6], acc[7]);
    }
    __syncthreads();
  }
  for (int i = tid; i < kGcRows * kGcD / 4; i += 256) {
    const int rr = i >> 5, d4 = i & 31;
    reinterpret_cast<float4*>(S + rr * kGcD)[d4] = *reinterpret_cast<const float4*>(sS + rr * kGcSr + 4 * d4);
  }
}

// ---------------------------------------------------------------- scan on the tensor cores
// The same per-chunk products as gdn_chunk_scan_kernel on mma.sync m16n8k8
// TF32 at fp32 accuracy: every operand is split into a TF32 high part and a
// TF32 remainder, and a product is accumulated as lo*hi + hi*lo + hi*hi
// (the remainder-by-remainder term is below fp32 rounding), in fp32.
// One CTA per (value head, 16 value rows), 8 warps.  Warp w = (m-tile
// mt = w & 3 of the chunk's 64 tokens, k-half kh = w >> 2):
//   X1 = Kt S0^T and X2 = Qg S0^T over its k-half, both n-tiles of the 16
//        value rows; the halves meet in shared memory, after which warp w owns
//        n-tile kh of m-tile mt;
//   U  = Tb V - X1 and Y = X2 + P U for that tile (P lower triangular: k up
//        to the tile's last row);
//   S  = e^{G_C} S + U^T Kd for d columns 16w .. 16w + 15, the state kept in
//        the warp's accumulator registers across chunks (and written back to
//        shared memory split into high and low parts for the next X products).
// The next chunk's tiles stream in with cp.async while the current chunk
// uses the other buffers: Kt / Qg after the X products, Tb / V after U, P /
// Kd / G after the state update.
constexpr int kTcLdK = 132;  // Kt, Qg, S rows: (g * 132 + t) mod 32 distinct over a warp
constexpr int kTcLdKd = 136; // Kd rows read as B (k = token): (t * 136 + g) mod 32 distinct
constexpr int kTcLdT = 68;   // Tb, P rows
constexpr int kTcLdV = 24;   // V, U rows (16 value rows + 8)
constexpr int kTcOffQg = kGc * kTcLdK;
constexpr int kTcOffKd = kTcOffQg + kGc * kTcLdK;
constexpr int kTcOffTb = kTcOffKd + kGc * kTcLdKd;
constexpr int kTcOffP = kTcOffTb + kGc * kTcLdT;
constexpr int kTcOffV = kTcOffP + kGc * kTcLdT;
constexpr int kTcOffUh = kTcOffV + kGc * kTcLdV;
constexpr int kTcOffUl = kTcOffUh + kGc * kTcLdV;
constexpr int kTcOffSh = kTcOffUl + kGc * kTcLdV;
constexpr int kTcOffSl = kTcOffSh + kGcRows * kTcLdK;
constexpr int kTcOffX = kTcOffSl + kGcRows * kTcLdK;
constexpr int kTcOffG = kTcOffX + 8 * 8 * 32;
constexpr size_t kGcScanTcSmem = static_cast<size_t>(kTcOffG + kGc) * sizeof(float);

KIB_DEV uint32_t tf32_rna(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return r;
}
KIB_DEV void tf32_split(float x, uint32_t& hi, uint32_t& lo) {
  hi = tf32_rna(x);
  lo = tf32_rna(x - __uint_as_float(hi));
}
// not volatile: a pure function of its operands, so the compiler may move
// the next k-step's loads and splits ahead of it
KIB_DEV void mma_tf32(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm(
      "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
// d += A B with split operands: the two cross terms first, then the main one
KIB_DEV void mma3(float (&d)[4], const uint32_t (&ah)[4], const uint32_t (&al)[4], uint32_t bh0, uint32_t bh1,
                  uint32_t bl0, uint32_t bl1) {
  mma_tf32(d, al, bh0, bh1);
  mma_tf32(d, ah, bl0, bl1);
  mma_tf32(d, ah, bh0, bh1);
}
// The same with the cross terms in their own accumulator c (added to d by the
// caller once the k loop is done): two shorter dependent chains instead of one
KIB_DEV void mma3s(float (&d)[4], float (&c)[4], const uint32_t (&ah)[4], const uint32_t (&al)[4], uint32_t bh0,
                   uint32_t bh1, uint32_t bl0, uint32_t bl1) {
  mma_tf32(c, al, bh0, bh1);
  mma_tf32(c, ah, bl0, bl1);
  mma_tf32(d, ah, bh0, bh1);
}
KIB_DEV void acc_add(float (&d)[4], const float (&c)[4]) {
#pragma unroll
  for (int e = 0; e < 4; ++e) d[e] += c[e];
}
// A fragment (16 x 8, row-major source, rows m0.., columns k0..) split in two
KIB_DEV void gc_lda(const float* s, int ld, int m0, int k0, int g, int t, uint32_t (&h)[4], uint32_t (&l)[4]) {
  const float* p = s + (m0 + g) * ld + k0 + t;
  tf32_split(p[0], h[0], l[0]);
  tf32_split(p[8 * ld], h[1], l[1]);
  tf32_split(p[4], h[2], l[2]);
  tf32_split(p[8 * ld + 4], h[3], l[3]);
}
// B fragment (8 x 8) from a source stored with k along rows: B[k][n] = s[k * ld + n]
KIB_DEV void gc_ldb_k(const float* s, int ld, int k0, int n0, int g, int t, uint32_t& h0, uint32_t& h1, uint32_t& l0,
                      uint32_t& l1) {
  const float* p = s + (k0 + t) * ld + n0 + g;
  tf32_split(p[0], h0, l0);
  tf32_split(p[4 * ld], h1, l1);
}

// ---------------------------------------------------------------- prep on the tensor cores
// Same outputs as gdn_chunk_prep_kernel.  K K^T, Q K^T and Kt = Tb diag(e^G) K
// run as split-TF32 mma.sync products (fp32 accuracy, see mma3); the unit
// lower-triangular inverse X = (I + L)^{-1} is taken by 16 x 16 blocks: the
// four diagonal blocks by forward substitution inside one warp each, then
// block row b (b = 1..3) as X_ba = -X_bb * sum_{a <= k < b} L_bk X_ka -- three
// CTA-wide steps instead of one barrier per row.
constexpr int kPtLd = 132;  // q / k rows
constexpr int kPtLdT = 68;  // L, X, Tb diag(e^G)
constexpr size_t kGcPrepTcSmem =
    (2 * kGc * kPtLd + 2 * kGc * kPtLdT + 3 * 16 * 16 + 3 * kGc) * sizeof(float);

__global__ void __launch_bounds__(256) gdn_chunk_prep_tc_kernel(const __grid_constant__ GdnChunkParams p) {
  extern __shared__ __align__(16) float pt_sm[];
  float* sK = pt_sm;                    // [64][132]: k rows
  float* sQ = sK + kGc * kPtLd;         // [64][132]: q rows
  float* sL = sQ + kGc * kPtLd;         // [64][68]: L, later Tb diag(e^G)
  float* sX = sL + kGc * kPtLdT;        // [64][68]: X = (I + L)^{-1}
  float* sW = sX + kGc * kPtLdT;        // [3][16][16]: block-row partial sums
  float* G = sW + 3 * 16 * 16;          // [64]
  float* bt = G + kGc;                  // [64]
  float* eG = bt + kGc;                 // [64]
  const int h = blockIdx.x, c = blockIdx.y, tid = threadIdx.x;
  const int lane = tid & 31, warp = tid >> 5, g = lane >> 2, t = lane & 3;
  const int kh = h % p.key_heads;
  const int t0 = c * kGc, n = min(kGc, p.T - t0);
  const int key_dim = p.key_heads * kGcD;
  pdl_wait();
  pdl_launch_dependents();
  for (int i = tid; i < kGc * kGcD / 4; i += 256) {
    const int tk = i >> 5, d4 = i & 31;
    const bool ok = tk < n;
    const float* row = p.conv_out + static_cast<size_t>(t0 + (ok ? tk : 0)) * p.C;
    gc_cp16(sQ + tk * kPtLd + 4 * d4, row + kh * kGcD + 4 * d4, ok);
    gc_cp16(sK + tk * kPtLd + 4 * d4, row + key_dim + kh * kGcD + 4 * d4, ok);
  }
  if (tid < kGc) {
    const bool ok = tid < n;
    G[tid] = ok ? p.g[static_cast<size_t>(t0 + tid) * p.ld_ba + h] : 0.0f;
    bt[tid] = ok ? p.beta[static_cast<size_t>(t0 + tid) * p.ld_ba + h] : 0.0f;
  }
  gc_cp_wait();
  __syncthreads();
  if (tid == 0) {
    float acc = 0.0f;
    for (int i = 0; i < kGc; ++i) {
      acc += G[i];
      G[i] = acc;
    }
  }
  __syncthreads();
  if (tid < kGc) eG[tid] = expf(G[tid]);
  float* ws = p.ws + (static_cast<size_t>(h) * gridDim.y + c) * kGcWs;
  float* wTb = ws;
  float* wP = ws + kGc * kGc;
  float* wKt = wP + kGc * kGc;
  float* wG = wKt + kGc * kGcD;

  // ---- K K^T and Q K^T: warp (m-tile w & 3, n-tiles 4 (w >> 2) .. + 3); tiles
  // wholly above the diagonal are zero
  {
    const int mt = warp & 3, m0 = 16 * mt, nb = 4 * (warp >> 2);
    float kk[4][4], qk[4][4], ck[4][4], cq[4][4];
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) kk[j][e] = qk[j][e] = ck[j][e] = cq[j][e] = 0.0f;
    const int nlive = max(0, min(4, 2 * mt + 2 - nb));  // n-tiles 8nt <= 16mt + 15
#pragma unroll 2
    for (int ks = 0; ks < kGcD / 8; ++ks) {
      const int k0 = 8 * ks;
      uint32_t akh[4], akl[4], aqh[4], aql[4];
      gc_lda(sK, kPtLd, m0, k0, g, t, akh, akl);
      gc_lda(sQ, kPtLd, m0, k0, g, t, aqh, aql);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if (j < nlive) {
          const float* bp = sK + (8 * (nb + j) + g) * kPtLd + k0 + t;  // B[d][j'] = k_j'[d]
          uint32_t b0h, b0l, b1h, b1l;
          tf32_split(bp[0], b0h, b0l);
          tf32_split(bp[4], b1h, b1l);
          mma3s(kk[j], ck[j], akh, akl, b0h, b1h, b0l, b1l);
          mma3s(qk[j], cq[j], aqh, aql, b0h, b1h, b0l, b1l);
        }
      }
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      acc_add(kk[j], ck[j]);
      acc_add(qk[j], cq[j]);
    }
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int i = m0 + g + 8 * (e >> 1), jj = 8 * (nb + j) + 2 * t + (e & 1);
        const float dec = jj <= i ? expf(G[i] - G[jj]) : 0.0f;
        sL[i * kPtLdT + jj] = jj < i ? bt[i] * dec * kk[j][e] : 0.0f;
        wP[i * kGc + jj] = dec * qk[j][e];
      }
  }
  __syncthreads();
  // ---- X = (I + L)^{-1}: diagonal blocks (warp b, lanes 0..15 = columns)
  if (warp < 4) {
    const int b0 = 16 * warp, col = lane & 15;
    for (int i = 0; i < 16; ++i) {
      float s = 0.0f;
      for (int j = col; j < i; ++j) s = fmaf(sL[(b0 + i) * kPtLdT + b0 + j], sX[(b0 + j) * kPtLdT + b0 + col], s);
      if (lane < 16) sX[(b0 + i) * kPtLdT + b0 + col] = col == i ? 1.0f : (col < i ? -s : 0.0f);
      __syncwarp();
    }
  } else {
    // zeros above the diagonal blocks
    for (int e = tid - 128; e < kGc * kGc; e += 128) {
      const int i = e >> 6, j = e & 63;
      if ((j >> 4) > (i >> 4)) sX[i * kPtLdT + j] = 0.0f;
    }
  }
  __syncthreads();
  // block rows 1..3: W_a = sum_{k=a}^{b-1} L_bk X_ka, then X_ba = -X_bb W_a
  for (int b = 1; b < 4; ++b) {
    for (int e = tid; e < b * 256; e += 256) {
      const int a = e >> 8, r = (e >> 4) & 15, cc = e & 15;
      float s = 0.0f;
      for (int k = a; k < b; ++k)
#pragma unroll 4
        for (int q = 0; q < 16; ++q)
          s = fmaf(sL[(16 * b + r) * kPtLdT + 16 * k + q], sX[(16 * k + q) * kPtLdT + 16 * a + cc], s);
      sW[e] = s;
    }
    __syncthreads();
    for (int e = tid; e < b * 256; e += 256) {
      const int a = e >> 8, r = (e >> 4) & 15, cc = e & 15;
      float s = 0.0f;
#pragma unroll 4
      for (int q = 0; q <= r; ++q) s = fmaf(sX[(16 * b + r) * kPtLdT + 16 * b + q], sW[(a * 16 + q) * 16 + cc], s);
      sX[(16 * b + r) * kPtLdT + 16 * a + cc] = -s;
    }
    __syncthreads();
  }
  // ---- Tb = X diag(beta) (to the workspace); Tb diag(e^G) for Kt
  for (int e = tid; e < kGc * kGc; e += 256) {
    const int i = e >> 6, j = e & 63;
    const float v = sX[i * kPtLdT + j] * bt[j];
    wTb[e] = v;
    sL[i * kPtLdT + j] = v * eG[j];
  }
  if (tid < kGc) wG[tid] = G[tid];
  __syncthreads();
  // ---- Kt = (Tb diag(e^G)) K: warp (m-tile w & 3, d columns 64 (w >> 2) ..);
  // Tb is lower triangular, so tokens up to the tile's last row
  {
    const int mt = warp & 3, m0 = 16 * mt, nb = 8 * (warp >> 2);
    float acc[8][4], cacc[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[j][e] = cacc[j][e] = 0.0f;
    for (int ks = 0; ks <= 2 * mt + 1; ++ks) {
      uint32_t ah[4], al[4];
      gc_lda(sL, kPtLdT, m0, 8 * ks, g, t, ah, al);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        uint32_t b0h, b1h, b0l, b1l;
        gc_ldb_k(sK, kPtLd, 8 * ks, 8 * (nb + j), g, t, b0h, b1h, b0l, b1l);
        mma3s(acc[j], cacc[j], ah, al, b0h, b1h, b0l, b1l);
      }
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) acc_add(acc[j], cacc[j]);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int d = 8 * (nb + j) + 2 * t;
      *reinterpret_cast<float2*>(wKt + (m0 + g) * kGcD + d) = make_float2(acc[j][0], acc[j][1]);
      *reinterpret_cast<float2*>(wKt + (m0 + g + 8) * kGcD + d) = make_float2(acc[j][2], acc[j][3]);
    }
  }
  // ---- the scan's decayed operands
  {
    float* wQg = ws + kGcWsQg;
    float* wKd = ws + kGcWsKd;
    const float gend = G[kGc - 1];
    for (int i = tid; i < kGc * kGcD / 4; i += 256) {
      const int tk = i >> 5, d4 = i & 31;
      const float fq = expf(G[tk]), fk = expf(gend - G[tk]);
      const float4 qv = *reinterpret_cast<const float4*>(sQ + tk * kPtLd + 4 * d4);
      const float4 kv = *reinterpret_cast<const float4*>(sK + tk * kPtLd + 4 * d4);
      reinterpret_cast<float4*>(wQg)[i] = make_float4(qv.x * fq, qv.y * fq, qv.z * fq, qv.w * fq);
      reinterpret_cast<float4*>(wKd)[i] = make_float4(kv.x * fk, kv.y * fk, kv.z * fk, kv.w * fk);
    }
  }
}

__global__ void __launch_bounds__(256) gdn_chunk_scan_tc_kernel(const __grid_constant__ GdnChunkParams p) {
  extern __shared__ __align__(16) float tc_sm[];
  float* sKt = tc_sm;
  float* sQg = tc_sm + kTcOffQg;
  float* sKd = tc_sm + kTcOffKd;
  float* sTb = tc_sm + kTcOffTb;
  float* sP = tc_sm + kTcOffP;
  float* sV = tc_sm + kTcOffV;
  float* sUh = tc_sm + kTcOffUh;
  float* sUl = tc_sm + kTcOffUl;
  float* sSh = tc_sm + kTcOffSh;
  float* sSl = tc_sm + kTcOffSl;
  float* sX = tc_sm + kTcOffX;
  float* sG = tc_sm + kTcOffG;
  const int h = blockIdx.x, r0 = blockIdx.y * kGcRows, tid = threadIdx.x;
  const int lane = tid & 31, warp = tid >> 5, g = lane >> 2, t = lane & 3;
  const int mt = warp & 3, kh = warp >> 2, m0 = 16 * mt;
  const int key_dim = p.key_heads * kGcD;
  const int nchunks = (p.T + kGc - 1) / kGc;
  float* S = p.state + (static_cast<size_t>(h) * kGcD + r0) * kGcD;

  // state fragment of warp w: rows g, g + 8 of the CTA's 16, columns
  // 16w + 8nt + 2t (+1)
  float sreg[2][4];
#pragma unroll
  for (int nt = 0; nt < 2; ++nt) {
    const int d = 16 * warp + 8 * nt + 2 * t;
    const float2 a = *reinterpret_cast<const float2*>(S + g * kGcD + d);
    const float2 b = *reinterpret_cast<const float2*>(S + (g + 8) * kGcD + d);
    sreg[nt][0] = a.x;
    sreg[nt][1] = a.y;
    sreg[nt][2] = b.x;
    sreg[nt][3] = b.y;
  }
  auto put_state = [&]() {
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      const int d = 16 * warp + 8 * nt + 2 * t;
      uint32_t hi, lo;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        tf32_split(sreg[nt][e], hi, lo);
        const int o = (g + 8 * (e >> 1)) * kTcLdK + d + (e & 1);
        sSh[o] = __uint_as_float(hi);
        sSl[o] = __uint_as_float(lo);
      }
    }
  };
  put_state();
  pdl_wait();
  pdl_launch_dependents();

  auto ws_of = [&](int c) { return p.ws + (static_cast<size_t>(h) * nchunks + c) * kGcWs; };
  auto issue_ktqg = [&](int c) {
    if (c < nchunks) {
      const float* ws = ws_of(c);
      for (int i = tid; i < kGc * kGcD / 4; i += 256) {
        const int tk = i >> 5, d4 = i & 31;
        gc_cp16(sKt + tk * kTcLdK + 4 * d4, ws + 2 * kGc * kGc + 4 * i, true);
        gc_cp16(sQg + tk * kTcLdK + 4 * d4, ws + kGcWsQg + 4 * i, true);
      }
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  auto issue_tbv = [&](int c) {
    if (c < nchunks) {
      const float* ws = ws_of(c);
      const int t0 = c * kGc, n = min(kGc, p.T - t0);
      for (int i = tid; i < kGc * kGc / 4; i += 256) {
        const int r = i >> 4, j4 = i & 15;
        gc_cp16(sTb + r * kTcLdT + 4 * j4, ws + 4 * i, true);
      }
      const int tk = tid >> 2, q4 = tid & 3;  // 64 tokens x 4 pieces of the 16 value rows
      const bool ok = tk < n;
      gc_cp16(sV + tk * kTcLdV + 4 * q4,
              p.conv_out + static_cast<size_t>(t0 + (ok ? tk : 0)) * p.C + 2 * key_dim + h * kGcD + r0 + 4 * q4, ok);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  auto issue_pkd = [&](int c) {
    if (c < nchunks) {
      const float* ws = ws_of(c);
      for (int i = tid; i < kGc * kGc / 4; i += 256) {
        const int r = i >> 4, j4 = i & 15;
        gc_cp16(sP + r * kTcLdT + 4 * j4, ws + kGc * kGc + 4 * i, true);
      }
      for (int i = tid; i < kGc * kGcD / 4; i += 256) {
        const int tk = i >> 5, d4 = i & 31;
        gc_cp16(sKd + tk * kTcLdKd + 4 * d4, ws + kGcWsKd + 4 * i, true);
      }
      if (tid < kGc / 4) gc_cp16(sG + 4 * tid, ws + 2 * kGc * kGc + kGc * kGcD + 4 * tid, true);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  issue_ktqg(0);
  issue_tbv(0);
  issue_pkd(0);

  const float scale = 1.0f / sqrtf(static_cast<float>(kGcD));
  const size_t out_ld = static_cast<size_t>(p.value_heads) * kGcD;
  const int nt_own = kh;  // n-tile this warp owns after the X exchange
  for (int c = 0; c < nchunks; ++c) {
    const int t0 = c * kGc, n = min(kGc, p.T - t0);
    // ---- X1 = Kt S0^T, X2 = Qg S0^T over this warp's k-half
    asm volatile("cp.async.wait_group 2;" ::: "memory");
    __syncthreads();
    float x1[2][4], x2[2][4], c1[2][4], c2[2][4];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) x1[nt][e] = x2[nt][e] = c1[nt][e] = c2[nt][e] = 0.0f;
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      const int k0 = 64 * kh + 8 * ks;
      uint32_t bh[2][2], bl[2][2];
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        const int o = (8 * nt + g) * kTcLdK + k0 + t;
        bh[nt][0] = __float_as_uint(sSh[o]);
        bh[nt][1] = __float_as_uint(sSh[o + 4]);
        bl[nt][0] = __float_as_uint(sSl[o]);
        bl[nt][1] = __float_as_uint(sSl[o + 4]);
      }
      uint32_t ah[4], al[4];
      gc_lda(sKt, kTcLdK, m0, k0, g, t, ah, al);
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) mma3s(x1[nt], c1[nt], ah, al, bh[nt][0], bh[nt][1], bl[nt][0], bl[nt][1]);
      gc_lda(sQg, kTcLdK, m0, k0, g, t, ah, al);
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) mma3s(x2[nt], c2[nt], ah, al, bh[nt][0], bh[nt][1], bl[nt][0], bl[nt][1]);
    }
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      acc_add(x1[nt], c1[nt]);
      acc_add(x2[nt], c2[nt]);
    }
    // halves meet: the warp keeps n-tile kh, hands the other to warp w ^ 4
    {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        sX[(warp * 8 + e) * 32 + lane] = nt_own ? x1[0][e] : x1[1][e];
        sX[(warp * 8 + 4 + e) * 32 + lane] = nt_own ? x2[0][e] : x2[1][e];
      }
    }
    __syncthreads();
    float X1[4], X2[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float r1 = sX[((warp ^ 4) * 8 + e) * 32 + lane], r2 = sX[((warp ^ 4) * 8 + 4 + e) * 32 + lane];
      // k-half 0 + k-half 1, in that order on both warps
      X1[e] = kh == 0 ? x1[0][e] + r1 : r1 + x1[1][e];
      X2[e] = kh == 0 ? x2[0][e] + r2 : r2 + x2[1][e];
    }
    issue_ktqg(c + 1);
    // ---- U = Tb V - X1 for (mt, nt_own)
    asm volatile("cp.async.wait_group 2;" ::: "memory");
    __syncthreads();
    float u[4] = {-X1[0], -X1[1], -X1[2], -X1[3]}, cu[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      uint32_t ah[4], al[4], b0h, b1h, b0l, b1l;
      gc_lda(sTb, kTcLdT, m0, 8 * ks, g, t, ah, al);
      gc_ldb_k(sV, kTcLdV, 8 * ks, 8 * nt_own, g, t, b0h, b1h, b0l, b1l);
      mma3s(u, cu, ah, al, b0h, b1h, b0l, b1l);
    }
    acc_add(u, cu);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      uint32_t hi, lo;
      tf32_split(u[e], hi, lo);
      const int o = (m0 + g + 8 * (e >> 1)) * kTcLdV + 8 * nt_own + 2 * t + (e & 1);
      sUh[o] = __uint_as_float(hi);
      sUl[o] = __uint_as_float(lo);
    }
    asm volatile("cp.async.wait_group 1;" ::: "memory");  // P, Kd, G of this chunk
    __syncthreads();
    issue_tbv(c + 1);
    // ---- Y = (X2 + P U) / sqrt(128) for (mt, nt_own): tokens up to the tile's last row
    {
      float y[4] = {X2[0], X2[1], X2[2], X2[3]}, cy[4] = {0.f, 0.f, 0.f, 0.f};
      for (int ks = 0; ks <= 2 * mt + 1; ++ks) {
        uint32_t ah[4], al[4];
        gc_lda(sP, kTcLdT, m0, 8 * ks, g, t, ah, al);
        const int o = (8 * ks + t) * kTcLdV + 8 * nt_own + g;
        mma3s(y, cy, ah, al, __float_as_uint(sUh[o]), __float_as_uint(sUh[o + 4 * kTcLdV]), __float_as_uint(sUl[o]),
              __float_as_uint(sUl[o + 4 * kTcLdV]));
      }
      acc_add(y, cy);
      const int col = h * kGcD + r0 + 8 * nt_own + 2 * t;
      const int ra = m0 + g, rb = m0 + g + 8;
      if (ra < n) *reinterpret_cast<float2*>(p.out + static_cast<size_t>(t0 + ra) * out_ld + col) =
          make_float2(y[0] * scale, y[1] * scale);
      if (rb < n) *reinterpret_cast<float2*>(p.out + static_cast<size_t>(t0 + rb) * out_ld + col) =
          make_float2(y[2] * scale, y[3] * scale);
    }
    // ---- S = e^{G_C} S + U^T Kd for columns 16w..16w+15
    {
      const float eg = expf(sG[kGc - 1]);
      float cs[2][4];
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          sreg[nt][e] *= eg;
          cs[nt][e] = 0.0f;
        }
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        const int j0 = 8 * ks;
        uint32_t ah[4], al[4];
        const int o = (j0 + t) * kTcLdV + g;  // A = U^T: A[r][j] = U[j][r]
        ah[0] = __float_as_uint(sUh[o]);
        ah[1] = __float_as_uint(sUh[o + 8]);
        ah[2] = __float_as_uint(sUh[o + 4 * kTcLdV]);
        ah[3] = __float_as_uint(sUh[o + 4 * kTcLdV + 8]);
        al[0] = __float_as_uint(sUl[o]);
        al[1] = __float_as_uint(sUl[o + 8]);
        al[2] = __float_as_uint(sUl[o + 4 * kTcLdV]);
        al[3] = __float_as_uint(sUl[o + 4 * kTcLdV + 8]);
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) {
          uint32_t b0h, b1h, b0l, b1l;
          gc_ldb_k(sKd, kTcLdKd, j0, 16 * warp + 8 * nt, g, t, b0h, b1h, b0l, b1l);
          mma3s(sreg[nt], cs[nt], ah, al, b0h, b1h, b0l, b1l);
        }
      }
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) acc_add(sreg[nt], cs[nt]);
      put_state();  // the X products of the next chunk read it after its barrier
    }
    __syncthreads();  // P, Kd, U free
    issue_pkd(c + 1);
  }
  asm volatile("cp.async.wait_all;" ::: "memory");
#pragma unroll
  for (int nt = 0; nt < 2; ++nt) {
    const int d = 16 * warp + 8 * nt + 2 * t;
    *reinterpret_cast<float2*>(S + g * kGcD + d) = make_float2(sreg[nt][0], sreg[nt][1]);
    *reinterpret_cast<float2*>(S + (g + 8) * kGcD + d) = make_float2(sreg[nt][2], sreg[nt][3]);
  }
}

}  // namespace kib