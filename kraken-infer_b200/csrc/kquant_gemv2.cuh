// kquant_gemv2.cuh -- compact K-quant GEMV for 1..3 tokens (the decode and
// small-verify path).
//
// Same contract as kquant_gemv_kernel (GemvParams, prologues, per-segment
// epilogues; replaces the reference's q*_k_matvec / q*_k_matmul row-reduce
// path and the fused LM-head argmax, mps_backend.mm:295-463, 579-749,
// 1268-1446, 1554-1688).  It is built for a short critical path and a small
// instruction footprint, because a bs1 decode step runs ~100 of these
// launches back to back and each one starts with a cold instruction cache:
//   * weight row tiles are staged by one cp.async.bulk per tile, issued before
//     griddepcontrol.wait (the fetch of kernel k+1 overlaps kernel k);
//   * each lane builds the 64 input values of its unit straight from global
//     memory -- the RMSNorm scale is computed by every warp, the per-head
//     norm-gate scale from the neighbouring lane -- so no block barrier
//     precedes the math;
//   * the row loop is not unrolled: the per-row code (one unit dot product,
//     a shuffle reduction, the epilogue) is fetched once and reused.
#pragma once

#include "kquant_gemv.cuh"

namespace kib {

// Input vector of one unit for one token, transformed by the prologue.  The
// normalisation scales are linear factors of the dot product, so they are
// left out here and applied to the result: the RMSNorm scale to the reduced
// row (epilogue), the per-head norm-gate scale to the lane's partial.  This
// lets the input loads and the scale reductions run in one round trip.
//   kProPlain:    x
//   kProRms:      x * w_norm                      (times rsqrt(mean x^2 + eps) later)
//   kProNormGate: y * w_head * silu(z)            (times rsqrt(mean_head y^2 + eps) later)
// Returns this lane's sum of y^2 over its unit (norm-gate) or 0.
template <int QT, int PRO>
KIB_DEV float build_unit_x(const GemvParams& p, int t, int blk, int u, UnitX<QT>& ux) {
  constexpr int GL = KQ<QT>::kGroupLen;
  const float* xr = p.in + static_cast<size_t>(t) * p.in_ld + 256 * blk;
  float ss = 0.0f;
#pragma unroll
  for (int g = 0; g < KQ<QT>::kGroups; ++g) ux.s[g] = 0.0f;
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const int c = unit_col<QT>(u, 4 * j);
    float4 v = *reinterpret_cast<const float4*>(xr + c);
    if constexpr (PRO == kProRms) {
      const float4 w = *reinterpret_cast<const float4*>(p.norm_w + 256 * blk + c);
      v.x *= w.x;
      v.y *= w.y;
      v.z *= w.z;
      v.w *= w.w;
    } else if constexpr (PRO == kProNormGate) {
      ss += (v.x * v.x + v.y * v.y) + (v.z * v.z + v.w * v.w);
      const int hc = (256 * blk + c) % p.head_dim;
      const float4 w = *reinterpret_cast<const float4*>(p.norm_w + hc);
      const float4 z = *reinterpret_cast<const float4*>(p.gate + static_cast<size_t>(t) * p.in_ld + 256 * blk + c);
      v.x = v.x * w.x * silu_f(z.x);
      v.y = v.y * w.y * silu_f(z.y);
      v.z = v.z * w.z * silu_f(z.z);
      v.w = v.w * w.w * silu_f(z.w);
    }
    ux.v[2 * j] = make_float2(v.x, v.y);
    ux.v[2 * j + 1] = make_float2(v.z, v.w);
    ux.s[(4 * j) / GL] += (v.x + v.y) + (v.z + v.w);
  }
  return ss;
}

// Stores the prologue's normalised input (x * scale * w) of this lane's unit.
template <int QT>
KIB_DEV void store_unit_x(const GemvParams& p, int t, int blk, int u, const UnitX<QT>& ux, float scale) {
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const int c = unit_col<QT>(u, 4 * j);
    const float2 a = ux.v[2 * j], b = ux.v[2 * j + 1];
    *reinterpret_cast<float4*>(p.x_out + static_cast<size_t>(t) * p.cols + 256 * blk + c) =
        make_float4(a.x * scale, a.y * scale, b.x * scale, b.y * scale);
  }
}

// Sum of squares of one token's input vector, computed by a whole warp.
KIB_DEV float warp_sumsq(const float* x, int n) {
  float s = 0.0f;
  for (int i = 4 * (threadIdx.x & 31); i < n; i += 128) {
    const float4 v = *reinterpret_cast<const float4*>(x + i);
    s += (v.x * v.x + v.y * v.y) + (v.z * v.z + v.w * v.w);
  }
  return warp_sum(s);
}

// Group leader's epilogue for one row (all tokens).
// conv_s / conv_wt: the row's conv state and weights (staged in shared memory);
// res: the row's residuals (shared memory) or null.
template <int NT>
KIB_DEV void gemv_row_epilogue(const GemvParams& p, const GemvSeg& sg, int row, const float (&acc)[NT],
                               const float (&acc2)[NT], float (&best)[NT], float (&bsum)[NT], int (&bidx)[NT],
                               const float* conv_s, const float* conv_wt, const float* res, int res_ld) {
  if (sg.epilogue == kEpiConv) {
    // kernel size 4 (the host routes other sizes to the generic kernel)
    float w0 = conv_s[0], w1 = conv_s[1], w2 = conv_s[2];
    const float c0 = conv_wt[0], c1 = conv_wt[1], c2 = conv_wt[2], c3 = conv_wt[3];
    float* st = p.conv_state + static_cast<size_t>(row) * 3;
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      const float w3 = acc[t];
      float c = 0.0f;
      c += w0 * c0;
      c += w1 * c1;
      c += w2 * c2;
      c += w3 * c3;
      sg.out[static_cast<size_t>(t) * sg.ld + row] = silu_f(c);
      w0 = w1;
      w1 = w2;
      w2 = w3;
    }
    st[0] = w0;
    st[1] = w1;
    st[2] = w2;
    return;
  }
#pragma unroll
  for (int t = 0; t < NT; ++t) {
    float v = acc[t];
    if (sg.epilogue == kEpiResidual) v += res ? res[t * res_ld] : p.resid[static_cast<size_t>(t) * sg.ld + row];
    if (sg.epilogue == kEpiSiluMul) v = silu_f(acc[t]) * acc2[t];
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

// Copy of segment `i` of the launch parameters with only constant offsets, so
// the parameter block is never indexed dynamically (that would force a local
// memory copy of it).
KIB_DEV GemvSeg seg_at(const GemvParams& p, int i) {
  switch (i) {
    case 0: return p.seg[0];
    case 1: return p.seg[1];
    case 2: return p.seg[2];
    default: return p.seg[3];
  }
}

KIB_DEV int seg_of_tile(const GemvParams& p, int gt) {
  int s = 0;
  if (p.nseg > 1 && gt >= p.seg[1].tile_begin) s = 1;
  if (p.nseg > 2 && gt >= p.seg[2].tile_begin) s = 2;
  if (p.nseg > 3 && gt >= p.seg[3].tile_begin) s = 3;
  return s;
}

template <int QT, int NT, int PRO>
__global__ void __launch_bounds__(kGemvThreads, 1) kquant_gemv2_kernel(const __grid_constant__ GemvParams p) {
  constexpr int kMaxResRows = 256;
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ uint64_t full_bar[8];
  __shared__ float s_part[kGemvThreads / 32][2][NT];
  __shared__ float s_best[kGemvThreads / 16][kGemvMaxTok];
  __shared__ float s_sum[kGemvThreads / 16][kGemvMaxTok];
  __shared__ int s_idx[kGemvThreads / 16][kGemvMaxTok];
  __shared__ float s_res[NT][kMaxResRows];
  __shared__ float s_scale[NT];
  __shared__ bool s_last;
  constexpr int BB = kquant_block_bytes(QT);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int S = p.stages;
  const int my_tiles = p.total_tiles > static_cast<int>(blockIdx.x)
                           ? (p.total_tiles - 1 - static_cast<int>(blockIdx.x)) / static_cast<int>(gridDim.x) + 1
                           : 0;
  const bool paired = p.paired != 0;
  const int km1 = p.conv_k - 1;
  const int conv_w_off = p.conv_off + ((p.tile_rows * km1 * 4 + 15) & ~15);

  auto issue = [&](int local) {
    const int gt = static_cast<int>(blockIdx.x) + local * static_cast<int>(gridDim.x);
    const GemvSeg sg = seg_at(p, seg_of_tile(p, gt));
    const int row0 = (gt - sg.tile_begin) * p.tile_rows;
    const int nrows = min(p.tile_rows, sg.rows - row0);
    const int st = local % S;
    uint8_t* dst = smem + static_cast<size_t>(st) * p.stage_bytes;
    const uint32_t bytes = static_cast<uint32_t>((nrows * p.row_bytes + 15) & ~15);
    const size_t off = static_cast<size_t>(row0) * p.row_bytes;
    const bool conv = sg.epilogue == kEpiConv && p.conv_off > 0;
    const uint32_t cs_bytes = conv ? static_cast<uint32_t>((nrows * km1 * 4 + 15) & ~15) : 0u;
    const uint32_t cw_bytes = conv ? static_cast<uint32_t>((nrows * p.conv_k * 4 + 15) & ~15) : 0u;
    mbar_arrive_expect_tx(&full_bar[st], (paired ? 2u * bytes : bytes) + cs_bytes + cw_bytes);
    bulk_g2s(dst, sg.w + off, bytes, &full_bar[st]);
    if (paired) bulk_g2s(dst + p.stage_bytes / 2, sg.w2 + off, bytes, &full_bar[st]);
    if (conv) {
      // the conv state was written by this kernel's previous step, long complete
      bulk_g2s(dst + p.conv_off, p.conv_state + static_cast<size_t>(row0) * km1, cs_bytes, &full_bar[st]);
      bulk_g2s(dst + conv_w_off, p.conv_w + static_cast<size_t>(row0) * p.conv_k, cw_bytes, &full_bar[st]);
    }
  };

  trace_entry(p.trace);
  if (tid == 0) {
    for (int s = 0; s < S; ++s) mbar_init(&full_bar[s], 1);
    fence_mbar_init();
    for (int i = 0; i < min(S, my_tiles); ++i) issue(i);
  }
  __syncthreads();

  pdl_wait();
  trace_wait(p.trace);
  const int RG = p.rg;
  const int groups = kGemvThreads / RG;
  const int group = tid / RG, gl = tid % RG;
  const bool active = gl < p.cols / 64;
  const int blk = gl >> 2, u = gl & 3;
  // ---- one round trip: residuals of the first tile, the input units and
  // the normalisation sums are all loaded here
  const bool res_smem = p.tile_rows <= kMaxResRows;
  if (res_smem && my_tiles > 0) {
    const GemvSeg sg0 = seg_at(p, seg_of_tile(p, blockIdx.x));
    if (sg0.epilogue == kEpiResidual) {
      const int row00 = (static_cast<int>(blockIdx.x) - sg0.tile_begin) * p.tile_rows;
      const int nrows0 = min(p.tile_rows, sg0.rows - row00);
      for (int i = tid; i < NT * nrows0; i += kGemvThreads) {
        const int t = i / nrows0, r = i % nrows0;
        s_res[t][r] = p.resid[static_cast<size_t>(t) * sg0.ld + row00 + r];
      }
    }
  }
  UnitX<QT> ux[NT];
  float lane_scale[NT];
#pragma unroll
  for (int t = 0; t < NT; ++t) {
    float ss_unit = 0.0f;
    if (active) ss_unit = build_unit_x<QT, PRO>(p, t, blk, u, ux[t]);
    lane_scale[t] = 1.0f;
    if constexpr (PRO == kProRms) {
      const float ss = warp_sumsq(p.in + static_cast<size_t>(t) * p.in_ld, p.cols);
      const float scale = 1.0f / sqrtf(ss / static_cast<float>(p.cols) + p.eps);
      if (tid == 0) s_scale[t] = scale;
      if (p.x_out != nullptr && blockIdx.x == 0 && tid < RG && active) store_unit_x<QT>(p, t, blk, u, ux[t], scale);
    } else if constexpr (PRO == kProNormGate) {
      // the partner unit (lane ^ 1) holds the other half of the 128-wide head
      const float ss = ss_unit + __shfl_xor_sync(0xffffffffu, ss_unit, 1);
      lane_scale[t] = 1.0f / sqrtf(ss / static_cast<float>(p.head_dim) + p.eps);
    } else {
      if (tid == 0) s_scale[t] = 1.0f;
    }
  }
  if (PRO == kProNormGate && tid == 0)
#pragma unroll
    for (int t = 0; t < NT; ++t) s_scale[t] = 1.0f;
  __syncthreads();  // s_res, s_scale
  trace_mark(p.trace, 6);  // prologue (input vectors) done
  pdl_launch_dependents();
  float row_scale[NT];
#pragma unroll
  for (int t = 0; t < NT; ++t) row_scale[t] = s_scale[t];

  float best[NT], bsum[NT];
  int bidx[NT];
#pragma unroll
  for (int t = 0; t < NT; ++t) {
    best[t] = -INFINITY;
    bsum[t] = 0.0f;
    bidx[t] = 0x7FFFFFFF;
  }

#pragma unroll 1
  for (int local = 0; local < my_tiles; ++local) {
    const int gt = static_cast<int>(blockIdx.x) + local * static_cast<int>(gridDim.x);
    const GemvSeg sg = seg_at(p, seg_of_tile(p, gt));
    const int row0 = (gt - sg.tile_begin) * p.tile_rows;
    const int nrows = min(p.tile_rows, sg.rows - row0);
    const int st = local % S;
    mbar_wait_bounded(&full_bar[st], static_cast<uint32_t>((local / S) & 1), p.err);
    if (local == 0) trace_mark(p.trace, 5);
    const uint8_t* tile = smem + static_cast<size_t>(st) * p.stage_bytes;
    const bool res_here = local == 0 && res_smem && sg.epilogue == kEpiResidual;
    const int passes = (nrows + groups - 1) / groups;
#pragma unroll 1
    for (int pass = 0; pass < passes; ++pass) {
      const int rl = pass * groups + group;
      const bool row_ok = rl < nrows;
      float acc[NT], acc2[NT];
#pragma unroll
      for (int t = 0; t < NT; ++t) acc[t] = acc2[t] = 0.0f;
      if (row_ok && active) {
        const uint8_t* b0 = tile + static_cast<size_t>(rl) * p.row_bytes + blk * BB;
        unit_dot<QT, NT>(b0, u, ux, acc);
        if (paired) unit_dot<QT, NT>(b0 + p.stage_bytes / 2, u, ux, acc2);
#pragma unroll
        for (int t = 0; t < NT; ++t) acc[t] *= lane_scale[t];
      }
      const int lim = RG < 32 ? RG : 32;
#pragma unroll
      for (int t = 0; t < NT; ++t)
        for (int o = lim / 2; o > 0; o >>= 1) {
          acc[t] += __shfl_xor_sync(0xffffffffu, acc[t], o);
          if (paired) acc2[t] += __shfl_xor_sync(0xffffffffu, acc2[t], o);
        }
      if (RG > 32) {
        if (lane == 0)
#pragma unroll
          for (int t = 0; t < NT; ++t) {
            s_part[warp][0][t] = acc[t];
            s_part[warp][1][t] = acc2[t];
          }
        __syncthreads();
        if (gl == 0)
#pragma unroll
          for (int t = 0; t < NT; ++t) {
            float a = 0.0f, b = 0.0f;
            for (int w = 0; w < RG / 32; ++w) {
              a += s_part[warp + w][0][t];
              b += s_part[warp + w][1][t];
            }
            acc[t] = a;
            acc2[t] = b;
          }
        __syncthreads();
      }
      if (gl == 0 && row_ok) {
#pragma unroll
        for (int t = 0; t < NT; ++t) {
          acc[t] *= row_scale[t];
          acc2[t] *= row_scale[t];
        }
        const float* cs = reinterpret_cast<const float*>(tile + p.conv_off) + rl * km1;
        const float* cw = reinterpret_cast<const float*>(tile + conv_w_off) + rl * p.conv_k;
        if (p.conv_off == 0) {
          cs = p.conv_state + static_cast<size_t>(row0 + rl) * km1;
          cw = p.conv_w + static_cast<size_t>(row0 + rl) * p.conv_k;
        }
        gemv_row_epilogue<NT>(p, sg, row0 + rl, acc, acc2, best, bsum, bidx, cs, cw,
                              res_here ? &s_res[0][rl] : nullptr, kMaxResRows);
      }
    }
    __syncthreads();  // stage consumed by every group
    if (tid == 0 && local + S < my_tiles) issue(local + S);
  }

  trace_exit(p.trace);
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
  if (tid < NT) {
    const int t = tid;
    float m = -INFINITY, s = 0.0f;
    int idx = 0x7FFFFFFF;
    for (int g = 0; g < groups; ++g) {
      const int gi = s_idx[g][t];
      if (gi == 0x7FFFFFFF) continue;
      const float gm = s_best[g][t], gs = s_sum[g][t];
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
  if (tid == 0) s_last = atomicAdd(p.counter, 1u) == gridDim.x - 1;
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  // A CTA whose bounded tile wait gave up raised *p.err before its fence and
  // ticket, so the last CTA sees it: the token is then -1 (no token), which a
  // caller without a status read-back (the no-allocation entry) can test.
  const bool failed = p.err != nullptr && atomicAdd(p.err, 0) != 0;
  if (tid < NT) {
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
    if (failed) {
      idx = -1;
      s = 0.0f;
    }
    p.token_out[t] = idx;
    if (p.prob_out) p.prob_out[(p.token_log ? *p.step_counter : 0) + t] = s > 0.0f ? 1.0f / s : 0.0f;
    if (p.token_log) p.token_log[*p.step_counter + t] = idx;
  }
  __syncthreads();
  if (tid == 0) {
    *p.counter = 0u;
    if (p.token_log) *p.step_counter += NT;
    if (p.pos_advance) *p.pos_advance += NT;
  }
}

}  // namespace kib
