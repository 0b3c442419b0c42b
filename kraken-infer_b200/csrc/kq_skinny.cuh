// kq_skinny.cuh -- M > 8 bucket projections for few tokens (9..64): batched
// decode steps and short prefill chunks.
//
// Numerics are the reference's M > 8 bucket (q*_k_mul_mm_simd,
// mps_backend.mm:1088-1266): each weight dequantised in fp32 and rounded to
// half, the input rounded to half, products accumulated in fp32 -- the same
// products as the f16-copy GEMMs (unit_dequant_h2 is the routine that writes
// the copies).  What differs is where the weights come from: this kernel
// reads the K-quant super-blocks (0.56 / 0.69 / 0.82 bytes per weight for
// Q4_K / Q5_K / Q6_K instead of 2), so with few tokens per weight the step is
// bound by 3.6x fewer HBM bytes.
//
// A CTA owns 64 weight rows and a range of super-blocks (split-K over
// gridDim.y when the row tiles alone cannot fill the GPU).  Per super-block:
// cp.async brings the 64 rows' raw blocks and the tokens' 256 halves of x into
// a double-buffered shared ring; the CTA dequantises the blocks into a
// [64][256] half tile; each of the four warps runs mma.sync m16n8k16 over its
// 16 rows and all token tiles.  With one split the epilogue writes y (+ the
// residual); with several, fp32 partials go to a workspace that
// kq_skinny_reduce_kernel sums in split order.
#pragma once

#include <cooperative_groups.h>

#include "kquant.cuh"
#include "layer_kernels.cuh"

namespace kib {

constexpr int kSkRows = 64;        // weight rows per CTA
constexpr int kSkLd = 264;         // halves per shared row (256 + 8: ldmatrix rows spread over banks)
constexpr int kSkRawStride = 256;  // bytes per raw block slot (a Q6_K block may start 2 bytes into a 16-byte line)

struct SkinnyParams {
  const uint8_t* w;   // K-quant rows
  int rows, cols, T;
  int row_bytes;
  const __half* x;    // [T][cols] half
  float* y;           // [T][y_ld]
  int y_ld;
  const float* resid; // may alias y
  float* ws;          // split partials [nsplit][T][rows]
  int kb_per_split;
  int xrows;          // rows of x in the shared tile (T, or 16 with xsplit)
  int xsplit;         // x rows 0..7 = half(x), 8..15 = half(x - half(x)): the 4..8 bucket
  int cluster;        // the splits of a row tile are one cluster: partials meet in shared memory
};

template <int NT>
constexpr size_t kq_skinny_smem() {
  return 2 * static_cast<size_t>(kSkRows) * kSkRawStride + static_cast<size_t>(kSkRows) * kSkLd * 2 +
         2 * static_cast<size_t>(8 * NT) * kSkLd * 2;
}

template <int QT, int NT>
__global__ void __launch_bounds__(128) kq_skinny_gemm_kernel(const __grid_constant__ SkinnyParams p) {
  constexpr int BB = kquant_block_bytes(QT);
  constexpr int NTOK = 8 * NT;
  extern __shared__ __align__(16) uint8_t sk_sm[];
  uint8_t* raw = sk_sm;                                                          // [2][64][256 B]
  __half* A = reinterpret_cast<__half*>(sk_sm + 2 * kSkRows * kSkRawStride);     // [64][264]
  __half* X = A + kSkRows * kSkLd;                                               // [2][NTOK][264]
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int row0 = blockIdx.x * kSkRows;
  const int bpr = p.cols / 256;
  const int kb0 = blockIdx.y * p.kb_per_split, kb1 = min(kb0 + p.kb_per_split, bpr);
  pdl_wait();
  pdl_launch_dependents();

  // raw block offsets of this thread's copies: row r's block kb starts at
  // byte (row0 + r) * row_bytes + kb * BB, copied as the 16-byte lines that
  // cover it; the slot keeps the same offset inside its first line
  auto issue = [&](int kb, int buf) {
    uint8_t* rb = raw + static_cast<size_t>(buf) * kSkRows * kSkRawStride;
    // 64 rows x up to 15 lines of 16 bytes
    for (int i = tid; i < kSkRows * 15; i += 128) {
      const int r = i / 15, line = i % 15;
      const int grow = row0 + r;
      const size_t start = static_cast<size_t>(min(grow, p.rows - 1)) * p.row_bytes + static_cast<size_t>(kb) * BB;
      const size_t base = start & ~size_t(15);
      const int nlines = static_cast<int>((start + BB - base + 15) >> 4);
      if (line < nlines)
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(rb + r * kSkRawStride + 16 * line)),
                     "l"(p.w + base + 16 * line)
                     : "memory");
    }
    __half* xb = X + static_cast<size_t>(buf) * NTOK * kSkLd;
    for (int i = tid; i < NTOK * 32; i += 128) {  // 32 pieces of 8 halves per token row
      const int t = i >> 5, piece = i & 31;
      const bool ok = t < p.xrows;
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(xb + t * kSkLd + 8 * piece)),
                   "l"(p.x + static_cast<size_t>(ok ? t : 0) * p.cols + kb * 256 + 8 * piece), "r"(ok ? 16 : 0)
                   : "memory");
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };

  float acc[NT][4];
#pragma unroll
  for (int j = 0; j < NT; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.0f;
  if (kb0 < kb1) issue(kb0, 0);
  for (int kb = kb0; kb < kb1; ++kb) {
    const int buf = (kb - kb0) & 1;
    if (kb + 1 < kb1) {
      issue(kb + 1, buf ^ 1);
      asm volatile("cp.async.wait_group 1;" ::: "memory");
    } else {
      asm volatile("cp.async.wait_group 0;" ::: "memory");
    }
    __syncthreads();  // block kb landed; the A tile of kb-1 is no longer read
    const uint8_t* rb = raw + static_cast<size_t>(buf) * kSkRows * kSkRawStride;
    for (int j = tid; j < kSkRows * 4; j += 128) {
      const int r = j >> 2, unit = j & 3;
      const size_t start = static_cast<size_t>(min(row0 + r, p.rows - 1)) * p.row_bytes + static_cast<size_t>(kb) * BB;
      __half2 v[32];
      unit_dequant_h2<QT>(rb + r * kSkRawStride + (start & 15), unit, v);
      __half* dst = A + r * kSkLd;
#pragma unroll
      for (int e = 0; e < 64; e += 2) *reinterpret_cast<__half2*>(dst + unit_col<QT>(unit, e)) = v[e / 2];
    }
    __syncthreads();
    const uint32_t a_base = smem_u32(A), b_base = smem_u32(X + static_cast<size_t>(buf) * NTOK * kSkLd);
#pragma unroll 4
    for (int k0 = 0; k0 < 256; k0 += 16) {
      uint32_t a[4];
      {
        const int row = 16 * warp + (lane & 15), col = k0 + (lane >> 4) * 8;
        ldsm_x4(a_base + static_cast<uint32_t>(row * kSkLd + col) * 2, a[0], a[1], a[2], a[3]);
      }
#pragma unroll
      for (int j = 0; j < NT; j += 2) {
        const int n = 8 * j + (lane & 7) + ((lane >> 4) << 3), col = k0 + ((lane >> 3) & 1) * 8;
        uint32_t b0, b1, b2, b3;
        ldsm_x4(b_base + static_cast<uint32_t>(n * kSkLd + col) * 2, b0, b1, b2, b3);
        mma_f16_16816(acc[j], a, b0, b1);
        mma_f16_16816(acc[j + 1], a, b2, b3);
      }
    }
  }
  const int g = lane >> 2, q = lane & 3;
  const bool split = gridDim.y > 1;
  if (p.xsplit) {
    // token t's product is the sum of its high-half row (tile 0) and its
    // low-half row (tile 1)
#pragma unroll
    for (int c = 0; c < 4; ++c) acc[0][c] += acc[1 % NT][c];
  }
  if (split && p.cluster) {
    // partial tile [NTOK tokens][64 rows] in this CTA's shared memory (the A
    // tile is no longer read), then every CTA of the cluster sums a slice of
    // the tile over the splits, in split order
    namespace cg = cooperative_groups;
    cg::cluster_group cl = cg::this_cluster();
    __syncthreads();
    float* part = reinterpret_cast<float*>(A);
#pragma unroll
    for (int j = 0; j < NT; ++j)
#pragma unroll
      for (int c = 0; c < 4; ++c)
        part[(8 * j + 2 * q + (c & 1)) * kSkRows + 16 * warp + g + (c >> 1) * 8] = acc[j][c];
    cl.sync();
    const int nsplit = static_cast<int>(gridDim.y), rank = static_cast<int>(cl.block_rank());
    const int ntok = p.xsplit ? 8 : NTOK, total = ntok * kSkRows;
    const int e0 = total * rank / nsplit, e1 = total * (rank + 1) / nsplit;
    for (int e = e0 + tid; e < e1; e += 128) {
      const int t = e / kSkRows, row = row0 + e % kSkRows;
      float v = 0.0f;
      for (int s = 0; s < nsplit; ++s) v += cl.map_shared_rank(part, s)[e];
      if (row < p.rows && t < p.T) {
        const size_t o = static_cast<size_t>(t) * p.y_ld + row;
        if (p.resid) v += p.resid[o];
        p.y[o] = v;
      }
    }
    cl.sync();  // the peers' partials stay in place until every slice is summed
    return;
  }
#pragma unroll
  for (int j = 0; j < NT; ++j)
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const int row = row0 + 16 * warp + g + (c >> 1) * 8;
      const int t = 8 * j + 2 * q + (c & 1);
      if (row < p.rows && t < p.T && !(p.xsplit && j > 0)) {
        if (split) {
          p.ws[(static_cast<size_t>(blockIdx.y) * p.T + t) * p.rows + row] = acc[j][c];
        } else {
          const size_t o = static_cast<size_t>(t) * p.y_ld + row;
          float v = acc[j][c];
          if (p.resid) v += p.resid[o];
          p.y[o] = v;
        }
      }
    }
}

// y[t][row] = sum over splits (in split order) of the partials (+ residual).
static __global__ void __launch_bounds__(256) kq_skinny_reduce_kernel(const float* ws, int nsplit, int rows, int T,
                                                                      float* y, int y_ld, const float* resid) {
  pdl_wait();
  pdl_launch_dependents();
  const size_t n = static_cast<size_t>(T) * rows;
  for (size_t i = blockIdx.x * 256ull + threadIdx.x; i < n; i += static_cast<size_t>(gridDim.x) * 256) {
    const int t = static_cast<int>(i / rows), row = static_cast<int>(i % rows);
    float v = 0.0f;
    for (int s = 0; s < nsplit; ++s) v += ws[static_cast<size_t>(s) * n + i];
    const size_t o = static_cast<size_t>(t) * y_ld + row;
    if (resid) v += resid[o];
    y[o] = v;
  }
}

// The 4..8-token bucket keeps x in fp32 against half weights: x becomes two
// half rows per token, rows 0..7 the rounded value and rows 8..15 the rounding
// remainder, so W_h . x = W_h . x_hi + W_h . x_lo to ~22 bits of x.
static __global__ void __launch_bounds__(256) x_split_f16_kernel(const float* x, int x_ld, int T, int cols,
                                                                 __half* out) {
  pdl_wait();
  pdl_launch_dependents();
  const size_t n = static_cast<size_t>(8) * cols;
  for (size_t i = blockIdx.x * 256ull + threadIdx.x; i < n; i += static_cast<size_t>(gridDim.x) * 256) {
    const int t = static_cast<int>(i / cols), c = static_cast<int>(i % cols);
    const float v = t < T ? x[static_cast<size_t>(t) * x_ld + c] : 0.0f;
    const __half hi = __float2half_rn(v);
    out[i] = hi;
    out[n + i] = __float2half_rn(v - __half2float(hi));
  }
}

}  // namespace kib
