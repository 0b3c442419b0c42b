// kquant_gemv.cuh -- small-M K-quant matrix-vector products over raw GGUF
// super-blocks, with the neighbouring element-wise work fused in.
//
// Replaces, for M <= 8 tokens, the reference's
//   q{4,5,6}_k_matvec / q*_k_matmul (fp32 row reduction, mps_backend.mm:295-463,
//   1268-1446), q*_k_mul_mv_ext (fp16-rounded weights, 887-1086), the fused
//   LM-head q*_k_matvec_argmax/_top1 + reduce (579-749, 1554-1688) and the
//   surrounding rms_norm / qk_norm+silu+mul / add / silu_mul dispatches of the
//   layer drivers (qwen35_runtime.cpp:2709-3131, 3203-3417).
//
// Data flow per CTA (one CTA per SM, 256 threads):
//   1. thread 0 issues cp.async.bulk copies of its first weight tiles into a
//      ring of shared-memory stages -- before griddepcontrol.wait, because the
//      weights never depend on the previous kernel;
//   2. griddepcontrol.wait; the prologue builds the input vector(s) in shared
//      memory (plain copy, RMSNorm, or per-head RMSNorm * silu(gate));
//   3. each lane owns one 64-weight unit of every row and keeps its x values
//      in registers; a group of RG lanes reduces one row;
//   4. the group leader applies the epilogue (store, + residual, silu(g)*u of a
//      gate/up pair, or a running argmax for the LM head).
#pragma once

#include "kib_common.cuh"
#include "kquant.cuh"

namespace kib {

enum GemvPrologue : int { kProPlain = 0, kProRms = 1, kProNormGate = 2 };
enum GemvEpilogue : int { kEpiStore = 0, kEpiResidual = 1, kEpiSiluMul = 2, kEpiArgmax = 3, kEpiConv = 4 };

constexpr int kGemvThreads = 256;
constexpr int kGemvMaxSegs = 4;
constexpr int kGemvMaxTok = 8;

struct GemvSeg {
  const uint8_t* w;   // raw super-blocks, [rows][cols/256][block]
  const uint8_t* w2;  // second matrix of a gate/up pair (kEpiSiluMul), same shape
  float* out;         // [tok][ld]
  int rows;
  int ld;
  int tile_begin;     // first global tile index of this segment
  int epilogue;       // GemvEpilogue applied to this segment's rows
};

struct GemvParams {
  GemvSeg seg[kGemvMaxSegs];
  int nseg;
  int cols;
  int row_bytes;
  int tile_rows;
  int total_tiles;
  int stages;
  int stage_bytes;
  int rg;               // lanes per row group (16, 32, 64 or 128)
  int ntok;
  int prologue;
  int paired;           // segments carry a gate/up pair (kEpiSiluMul)
  int argmax;           // some segment uses kEpiArgmax
  // prologue inputs
  const float* in;      // [tok][in_ld]
  int in_ld;
  const float* norm_w;  // RMSNorm weight (cols) or per-head norm weight (head_dim)
  float eps;
  const float* gate;    // kProNormGate: z [tok][cols]
  int head_dim;
  // epilogue inputs
  const float* resid;   // kEpiResidual: [tok][ld]
  // kEpiConv: causal depthwise conv (kernel conv_k) over [state | new values],
  // then silu; the state of every channel (row) has exactly one writer, the
  // row's group leader (build_ssm_conv_state_f32 + ssm_conv_f32 + silu,
  // mps_backend.mm:2376-2457, 2610-2618).
  float* conv_state;    // [rows][conv_k-1]
  const float* conv_w;  // [rows][conv_k]
  int conv_k;
  int conv_off;         // compact kernel: byte offset of the staged conv state rows in a stage (0: none)
  // kEpiArgmax: per-CTA candidates, then the last CTA writes token/prob per token
  float* cand_max;      // [grid][tok]
  float* cand_sum;      // [grid][tok]
  int* cand_idx;        // [grid][tok]
  unsigned* counter;
  int* token_out;       // [tok]
  float* prob_out;      // [tok] (may be null)
  int* token_log;       // optional: token_log[*step_counter + t] = token, then ++*step_counter
  int* step_counter;
  int* pos_advance;     // optional: *pos_advance += ntok once the head is done
  float* x_out;         // optional: CTA 0 stores the prologue's input vectors [tok][cols]
  int* err;
  unsigned long long* trace;  // KIB_TRACE slot or null
};

KIB_DEV float silu_f(float v) { return v / (1.0f + expf(-v)); }

// ---------------------------------------------------------------- prologue
// Builds xs[t][0..cols) for t < ntok in shared memory.
KIB_DEV void gemv_prologue(const GemvParams& p, float* xs, float* red) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int cols = p.cols;
  for (int t = 0; t < p.ntok; ++t) {
    const float* in = p.in + static_cast<size_t>(t) * p.in_ld;
    float* x = xs + t * cols;
    if (p.prologue == kProPlain) {
      for (int i = tid * 4; i < cols; i += kGemvThreads * 4)
        *reinterpret_cast<float4*>(x + i) = *reinterpret_cast<const float4*>(in + i);
    } else if (p.prologue == kProRms) {
      // rms_norm_f32_f32_batched (mps_backend.mm:1891-1921): x * rsqrt(mean(x^2)+eps) * w
      float ss = 0.0f;
      for (int i = tid * 4; i < cols; i += kGemvThreads * 4) {
        const float4 v = *reinterpret_cast<const float4*>(in + i);
        *reinterpret_cast<float4*>(x + i) = v;
        ss += (v.x * v.x + v.y * v.y) + (v.z * v.z + v.w * v.w);
      }
      ss = warp_sum(ss);
      if (lane == 0) red[warp] = ss;
      __syncthreads();
      float tot = 0.0f;
#pragma unroll
      for (int w = 0; w < kGemvThreads / 32; ++w) tot += red[w];
      const float scale = 1.0f / sqrtf(tot / static_cast<float>(cols) + p.eps);
      for (int i = tid; i < cols; i += kGemvThreads) x[i] = x[i] * scale * p.norm_w[i];
      __syncthreads();
    } else {
      // qk_norm_f32_f32_batched over heads, silu(gate), mul (qwen35_runtime.cpp:2993-3003)
      const int hd = p.head_dim, heads = cols / hd;
      const float* z = p.gate + static_cast<size_t>(t) * cols;
      for (int h = warp; h < heads; h += kGemvThreads / 32) {
        float ss = 0.0f;
        for (int i = lane; i < hd; i += 32) {
          const float v = in[h * hd + i];
          ss += v * v;
        }
        ss = warp_sum(ss);
        const float scale = 1.0f / sqrtf(ss / static_cast<float>(hd) + p.eps);
        for (int i = lane; i < hd; i += 32) {
          const float v = in[h * hd + i] * (scale * p.norm_w[i]);
          x[h * hd + i] = v * silu_f(z[h * hd + i]);
        }
      }
    }
  }
  __syncthreads();
}

// ------------------------------------------------------------- main kernel
// F16W selects the reference's 4..8-token numerics: every weight is rounded
// to half before the fp32 dot product (x stays fp32 and is read from shared
// memory).
template <int QT, int NT, bool F16W>
__global__ void __launch_bounds__(kGemvThreads, 1) kquant_gemv_kernel(const __grid_constant__ GemvParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ uint64_t full_bar[8];
  __shared__ float red[64];
  __shared__ float s_best[kGemvThreads / 16][kGemvMaxTok];
  __shared__ float s_sum[kGemvThreads / 16][kGemvMaxTok];
  __shared__ int s_idx[kGemvThreads / 16][kGemvMaxTok];
  __shared__ float s_part[kGemvThreads / 32][kGemvMaxTok];
  __shared__ bool s_last;

  constexpr int BB = kquant_block_bytes(QT);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int S = p.stages;
  uint8_t* stage_base = smem;
  float* xs = reinterpret_cast<float*>(smem + static_cast<size_t>(S) * p.stage_bytes);

  // tiles owned by this CTA: blockIdx.x, blockIdx.x + gridDim.x, ...
  const int my_tiles = p.total_tiles > static_cast<int>(blockIdx.x)
                           ? (p.total_tiles - 1 - static_cast<int>(blockIdx.x)) / static_cast<int>(gridDim.x) + 1
                           : 0;
  const bool paired = p.paired != 0;

  auto tile_info = [&](int local, int& seg, int& row0, int& nrows) {
    const int gt = static_cast<int>(blockIdx.x) + local * static_cast<int>(gridDim.x);
    seg = 0;
#pragma unroll
    for (int s = 1; s < kGemvMaxSegs; ++s)
      if (s < p.nseg && gt >= p.seg[s].tile_begin) seg = s;
    row0 = (gt - p.seg[seg].tile_begin) * p.tile_rows;
    nrows = min(p.tile_rows, p.seg[seg].rows - row0);
  };
  auto issue = [&](int local) {
    int seg, row0, nrows;
    tile_info(local, seg, row0, nrows);
    const int st = local % S;
    uint8_t* dst = stage_base + static_cast<size_t>(st) * p.stage_bytes;
    const uint32_t bytes = static_cast<uint32_t>((nrows * p.row_bytes + 15) & ~15);
    const uint8_t* src = p.seg[seg].w + static_cast<size_t>(row0) * p.row_bytes;
    mbar_arrive_expect_tx(&full_bar[st], paired ? 2u * bytes : bytes);
    bulk_g2s(dst, src, bytes, &full_bar[st]);
    if (paired) {
      const uint8_t* src2 = p.seg[seg].w2 + static_cast<size_t>(row0) * p.row_bytes;
      bulk_g2s(dst + p.stage_bytes / 2, src2, bytes, &full_bar[st]);
    }
  };

  if (tid == 0) {
    for (int s = 0; s < S; ++s) mbar_init(&full_bar[s], 1);
    fence_mbar_init();
    for (int i = 0; i < min(S, my_tiles); ++i) issue(i);
  }
  __syncthreads();

  // ---- wait for the producer kernel, then build the input vectors
  pdl_wait();
  gemv_prologue(p, xs, red);
  pdl_launch_dependents();
  if (p.x_out != nullptr && blockIdx.x == 0) {
    for (int i = tid; i < p.ntok * p.cols; i += kGemvThreads) p.x_out[i] = xs[i];
  }

  // ---- per-lane unit and its x values
  const int RG = p.rg;
  const int groups = kGemvThreads / RG;
  const int group = tid / RG;
  const int gl = tid % RG;  // lane within group
  const int units = p.cols / 64;
  const bool active = gl < units;
  const int blk = gl >> 2, unit = gl & 3;
  UnitX<QT> ux[NT];
  if constexpr (!F16W) {
    if (active) {
#pragma unroll
      for (int t = 0; t < NT; ++t) load_unit_x<QT>(xs + t * p.cols + 256 * blk, unit, ux[t]);
    }
  }

  float best[NT], bsum[NT];
  int bidx[NT];
#pragma unroll
  for (int t = 0; t < NT; ++t) {
    best[t] = -INFINITY;
    bsum[t] = 0.0f;
    bidx[t] = 0x7FFFFFFF;
  }

  for (int local = 0; local < my_tiles; ++local) {
    int seg, row0, nrows;
    tile_info(local, seg, row0, nrows);
    const int st = local % S;
    mbar_wait_bounded(&full_bar[st], static_cast<uint32_t>((local / S) & 1), p.err);
    const uint8_t* tile = stage_base + static_cast<size_t>(st) * p.stage_bytes;
    const int passes = (nrows + groups - 1) / groups;
    // F16W: two rows per pass, so every x value read from shared memory
    // serves both (the x of 4..8 tokens does not fit in registers)
    constexpr int PR = F16W ? 2 : 1;
    auto finish = [&](float (&acc)[NT], float (&acc2)[NT], const int rl, const bool row_ok) {
      // ---- reduce across the group
#pragma unroll
      for (int t = 0; t < NT; ++t) {
        const int lim = RG < 32 ? RG : 32;
        for (int o = lim / 2; o > 0; o >>= 1) {
          acc[t] += __shfl_xor_sync(0xffffffffu, acc[t], o);
          if (paired) acc2[t] += __shfl_xor_sync(0xffffffffu, acc2[t], o);
        }
      }
      if (RG > 32) {
        // cross-warp: warps of a group write partials; warp-leader of the group sums.
        if (lane == 0)
#pragma unroll
          for (int t = 0; t < NT; ++t) s_part[warp][t] = acc[t];
        __syncthreads();
        if (gl == 0) {
#pragma unroll
          for (int t = 0; t < NT; ++t) {
            float s = 0.0f;
            for (int w = 0; w < RG / 32; ++w) s += s_part[warp + w][t];
            acc[t] = s;
          }
        }
        if (paired) {
          __syncthreads();
          if (lane == 0)
#pragma unroll
            for (int t = 0; t < NT; ++t) s_part[warp][t] = acc2[t];
          __syncthreads();
          if (gl == 0) {
#pragma unroll
            for (int t = 0; t < NT; ++t) {
              float s = 0.0f;
              for (int w = 0; w < RG / 32; ++w) s += s_part[warp + w][t];
              acc2[t] = s;
            }
          }
        }
        __syncthreads();
      }
      // ---- epilogue by the group leader
      if (gl == 0 && row_ok) {
        const int row = row0 + rl;
        const GemvSeg& sg = p.seg[seg];
        if (sg.epilogue == kEpiConv) {
          const int km1 = p.conv_k - 1;
          float win[8];
          float* st = p.conv_state + static_cast<size_t>(row) * km1;
          for (int j = 0; j < km1; ++j) win[j] = st[j];
          const float* cw = p.conv_w + static_cast<size_t>(row) * p.conv_k;
#pragma unroll
          for (int t = 0; t < NT; ++t) {
            if (t < p.ntok) {
              win[km1] = acc[t];
              float c = 0.0f;
              for (int j = 0; j <= km1; ++j) c += win[j] * cw[j];
              sg.out[static_cast<size_t>(t) * sg.ld + row] = silu_f(c);
              for (int j = 0; j < km1; ++j) win[j] = win[j + 1];
            }
          }
          for (int j = 0; j < km1; ++j) st[j] = win[j];
        } else {
#pragma unroll
          for (int t = 0; t < NT; ++t) {
            if (t >= p.ntok) break;
            float v = acc[t];
            if (sg.epilogue == kEpiResidual) {
              v += p.resid[static_cast<size_t>(t) * sg.ld + row];
            } else if (sg.epilogue == kEpiSiluMul) {
              v = silu_f(acc[t]) * acc2[t];
            }
            if (sg.epilogue == kEpiArgmax) {
              if (v > best[t] || (v == best[t] && row < bidx[t])) {
                bsum[t] = bsum[t] * expf(best[t] - v) + 1.0f;
                best[t] = v;
                bidx[t] = row;
              } else {
                bsum[t] += expf(v - best[t]);
              }
              if (sg.out) sg.out[static_cast<size_t>(t) * sg.ld + row] = v;
            } else {
              sg.out[static_cast<size_t>(t) * sg.ld + row] = v;
            }
          }
        }
      }
        };
#pragma unroll 1
    for (int pass = 0; pass < passes; pass += PR) {
      const int rl = pass * groups + group, rlb = rl + groups;
      const bool row_ok = rl < nrows, rowb_ok = PR == 2 && rlb < nrows;
      float acc[NT], acc2[NT], accb[NT], accb2[NT];
#pragma unroll
      for (int t = 0; t < NT; ++t) acc[t] = acc2[t] = accb[t] = accb2[t] = 0.0f;
      if constexpr (F16W) {
        if (row_ok && active) {
          // weights rounded to half (two per register), x read as float4 runs
          // of unit_col, products accumulated in two fp32 lanes (FFMA2)
          const uint8_t* b0 = tile + static_cast<size_t>(rl) * p.row_bytes + blk * BB;
          const uint8_t* b1 = tile + static_cast<size_t>(rowb_ok ? rlb : rl) * p.row_bytes + blk * BB;
          __half2 wh[32], wh2[32];
#pragma unroll 1
          for (int hh = 0; hh <= static_cast<int>(paired); ++hh) {
            unit_dequant_h2<QT>(b0 + hh * (p.stage_bytes / 2), unit, wh);
            unit_dequant_h2<QT>(b1 + hh * (p.stage_bytes / 2), unit, wh2);
#pragma unroll
            for (int t = 0; t < NT; ++t) {
              if (t >= p.ntok) break;  // xs holds ntok rows only
              const float* xb = xs + t * p.cols + 256 * blk;
              float2 s2 = make_float2(0.0f, 0.0f), s2b = make_float2(0.0f, 0.0f);
#pragma unroll
              for (int e = 0; e < 64; e += 4) {
                const float4 x4 = *reinterpret_cast<const float4*>(xb + unit_col<QT>(unit, e));
                const float2 xa = make_float2(x4.x, x4.y), xc = make_float2(x4.z, x4.w);
                s2 = ffma2(__half22float2(wh[e / 2]), xa, s2);
                s2 = ffma2(__half22float2(wh[e / 2 + 1]), xc, s2);
                s2b = ffma2(__half22float2(wh2[e / 2]), xa, s2b);
                s2b = ffma2(__half22float2(wh2[e / 2 + 1]), xc, s2b);
              }
              if (hh == 0) {
                acc[t] = s2.x + s2.y;
                accb[t] = s2b.x + s2b.y;
              } else {
                acc2[t] = s2.x + s2.y;
                accb2[t] = s2b.x + s2b.y;
              }
            }
          }
        }
      } else {
        if (row_ok && active) {
          const uint8_t* b0 = tile + static_cast<size_t>(rl) * p.row_bytes + blk * BB;
          unit_dot<QT, NT>(b0, unit, ux, acc);
          if (paired) unit_dot<QT, NT>(b0 + p.stage_bytes / 2, unit, ux, acc2);
        }
      }
      finish(acc, acc2, rl, row_ok);
      if (PR == 2) finish(accb, accb2, rlb, rowb_ok);
    }
    __syncthreads();  // stage consumed by every group
    if (tid == 0 && local + S < my_tiles) issue(local + S);
  }

  if (!p.argmax) return;

  // ---- LM-head argmax: CTA reduction, then the last CTA reduces all CTAs
  // (ties -> lowest index, as argmax_f32_i32 / k_quant_top1_reduce).
  if (gl == 0) {
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      s_best[group][t] = best[t];
      s_sum[group][t] = bsum[t];
      s_idx[group][t] = bidx[t];
    }
  }
  __syncthreads();
  if (tid < p.ntok) {
    const int t = tid;
    float m = -INFINITY, s = 0.0f;
    int idx = 0x7FFFFFFF;
    for (int g = 0; g < groups; ++g) {
      const float gm = s_best[g][t];
      const int gi = s_idx[g][t];
      if (gi == 0x7FFFFFFF) continue;
      const float gs = s_sum[g][t];
      if (gm > m || (gm == m && gi < idx)) {
        s = s * expf(m - gm) + gs;
        m = gm;
        idx = gi;
      } else {
        s += gs * expf(gm - m);
      }
    }
    p.cand_max[blockIdx.x * kGemvMaxTok + t] = m;
    p.cand_sum[blockIdx.x * kGemvMaxTok + t] = s;
    p.cand_idx[blockIdx.x * kGemvMaxTok + t] = idx;
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const unsigned done = atomicAdd(p.counter, 1u);
    s_last = done == gridDim.x - 1;
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  if (tid < p.ntok) {
    const int t = tid;
    float m = -INFINITY, s = 0.0f;
    int idx = 0x7FFFFFFF;
    for (unsigned c = 0; c < gridDim.x; ++c) {
      const int gi = __ldcg(&p.cand_idx[c * kGemvMaxTok + t]);
      if (gi == 0x7FFFFFFF) continue;
      const float gm = __ldcg(&p.cand_max[c * kGemvMaxTok + t]);
      const float gs = __ldcg(&p.cand_sum[c * kGemvMaxTok + t]);
      if (gm > m || (gm == m && gi < idx)) {
        s = s * expf(m - gm) + gs;
        m = gm;
        idx = gi;
      } else {
        s += gs * expf(gm - m);
      }
    }
    p.token_out[t] = idx;
    if (p.prob_out) p.prob_out[t] = s > 0.0f ? 1.0f / s : 0.0f;
    if (p.token_log) p.token_log[*p.step_counter + t] = idx;
  }
  __syncthreads();
  if (tid == 0) {
    *p.counter = 0u;
    if (p.token_log) *p.step_counter += p.ntok;
    if (p.pos_advance) *p.pos_advance += p.ntok;
  }
}

}  // namespace kib
