// gemm_tc.cuh -- prefill GEMM on the 5th-generation tensor cores (tcgen05).
//
// Y[t][row] (+= residual) = sum_k W16[row][k] * X16[t][k] for the M > 8
// prefill bucket (weights and input rounded to half, fp32 accumulation:
// q*_k_mul_mm_simd, mps_backend.mm:1088-1266).  Each CTA owns one 128-row x
// BN-token output tile:
//   warp 0      one lane streams W and X tiles of 64 columns (128-byte rows,
//               128-byte swizzle) with 2-D tensor-map TMA into a ring of
//               kTcStages shared-memory stages (full/empty mbarriers);
//   warp 1      allocates BN columns of tensor memory, and one lane issues
//               tcgen05.mma (M = 128, N = BN, K = 16 per instruction, both
//               operands K-major from shared memory, fp32 accumulator in
//               TMEM); tcgen05.commit frees each stage when its MMAs are done
//               and finally signals the accumulator;
//   warps 2-5   read the accumulator back with tcgen05.ld (warp w reads TMEM
//               lanes 32*(w%4)..+31, i.e. 32 consecutive weight rows) and
//               store, for each token, 32 consecutive floats of Y (one
//               128-byte line per warp and token), adding the residual.
// Every wait is bounded; a wait that gives up raises *err (KIB_ERR_TIMEOUT on
// the host) and the CTA still reaches the TMEM release.  No multicast: the
// tensor maps cover this GPU's own memory only.
#pragma once

#include <cuda.h>

#include "kib_common.cuh"

namespace kib {

constexpr int kTcBM = 128;        // weight rows per tile (MMA M)
constexpr int kTcBK = 64;         // columns per stage: 64 halves = one 128-byte swizzle row
constexpr int kTcStages = 3;  // 96 KB of stages at N = 128: two CTAs per SM, one's epilogue under the other's loads
constexpr int kTcThreads = 192;   // producer warp, MMA warp, four epilogue warps

template <int BN>
constexpr size_t gemm_tc_smem() {
  // stages of A (128 x 64 halves) and B (BN x 64 halves), 1024-byte aligned,
  // plus the barriers and the TMEM address
  return static_cast<size_t>(kTcStages) * (kTcBM + BN) * kTcBK * 2 + 1024 + 256;
}

struct GemmTcParams {
  int rows, cols, T;
  float* y;          // [T][y_ld]
  int y_ld;
  const float* resid;  // may alias y (in-place residual add)
  int* err;
};

// ---- tcgen05 / TMA primitives (inline PTX, sm_100a)
KIB_DEV void tma_load_2d(void* smem_dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

KIB_DEV void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// Shared-memory matrix descriptor: K-major operand, rows of 128 bytes with
// the 128-byte swizzle, 8-row groups 1024 bytes apart (SBO), sm_100 version 1.
KIB_DEV uint64_t umma_desc_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);   // start address
  d |= static_cast<uint64_t>(1u) << 16;                 // LBO (unused with this swizzle)
  d |= static_cast<uint64_t>(1024u >> 4) << 32;         // SBO
  d |= static_cast<uint64_t>(1u) << 46;                 // descriptor version (sm_100)
  d |= static_cast<uint64_t>(2u) << 61;                 // SWIZZLE_128B
  return d;
}

// Instruction descriptor: f16 x f16 -> f32, both K-major, M = 128, N = n.
__host__ __device__ constexpr uint32_t umma_idesc_f16(int n) {
  return (1u << 4)                                   // D format f32
         | (0u << 7) | (0u << 10)                    // A, B format f16
         | (static_cast<uint32_t>(n >> 3) << 17)     // N / 8
         | (static_cast<uint32_t>(kTcBM >> 4) << 24);  // M / 16
}

KIB_DEV void umma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

KIB_DEV void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

KIB_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
KIB_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 32 consecutive fp32 columns of this thread's TMEM lane.
KIB_DEV void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// Bounded wait that reports through *err and returns false when it gives up.
KIB_DEV bool tc_wait(uint64_t* bar, uint32_t parity, int* err) {
  #pragma unroll 1
  for (uint32_t i = 0; i < (1u << 20); ++i)
    if (mbar_try_wait(bar, parity)) return true;
  if (err) atomicCAS(err, 0, 2);
  return false;
}

template <int BN>
__global__ void __launch_bounds__(kTcThreads, 2)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap xmap,
                   const __grid_constant__ GemmTcParams p) {
  static_assert(BN % 32 == 0 && BN >= 32 && BN <= 256, "N must be a multiple of 32 up to 256");
  constexpr uint32_t kABytes = kTcBM * kTcBK * 2, kBBytes = BN * kTcBK * 2;
  constexpr uint32_t kTmemCols = BN < 32 ? 32 : BN;  // a power of two >= 32
  static_assert((kTmemCols & (kTmemCols - 1)) == 0, "TMEM allocation must be a power of two");
  extern __shared__ __align__(1024) uint8_t tc_raw[];
  // 1024-byte alignment for the swizzled tiles
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(tc_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* a_st = smem;
  uint8_t* b_st = smem + kTcStages * kABytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(b_st + kTcStages * kBBytes);
  uint64_t* empty = full + kTcStages;
  uint64_t* acc_full = empty + kTcStages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_full + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m0 = blockIdx.x * kTcBM, t0 = blockIdx.y * BN;
  const int nk = p.cols / kTcBK;

  if (warp == 0 && lane == 0) {
    for (int s = 0; s < kTcStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(acc_full, 1);
    fence_mbar_init();
    tma_prefetch_desc(&wmap);
    tma_prefetch_desc(&xmap);
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(tmem_slot);
  // inputs (and a per-call f16 weight copy) come from the previous kernel
  pdl_wait();

  if (warp == 0) {
    if (lane == 0) {
      #pragma unroll 1
      for (int kt = 0; kt < nk; ++kt) {
        const int s = kt % kTcStages;
        if (!tc_wait(&empty[s], static_cast<uint32_t>(((kt / kTcStages) & 1) ^ 1), p.err)) break;
        mbar_arrive_expect_tx(&full[s], kABytes + kBBytes);
        tma_load_2d(a_st + s * kABytes, &wmap, kt * kTcBK, m0, &full[s]);
        tma_load_2d(b_st + s * kBBytes, &xmap, kt * kTcBK, t0, &full[s]);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_f16(BN);
      bool ok = true;
      #pragma unroll 1
      for (int kt = 0; kt < nk && ok; ++kt) {
        const int s = kt % kTcStages;
        ok = tc_wait(&full[s], static_cast<uint32_t>((kt / kTcStages) & 1), p.err);
        if (!ok) break;
        tc_fence_after();
        const uint32_t a0 = smem_u32(a_st + s * kABytes), b0 = smem_u32(b_st + s * kBBytes);
#pragma unroll
        for (int k = 0; k < kTcBK / 16; ++k)
          umma_f16(tmem, umma_desc_sw128(a0 + 32 * k), umma_desc_sw128(b0 + 32 * k), idesc,
                   (kt | k) != 0 ? 1u : 0u);
        umma_commit(&empty[s]);  // the stage is free once these MMAs have read it
      }
      umma_commit(acc_full);  // all MMAs issued so far are done: the accumulator is final
    }
  } else {
    // epilogue: TMEM lane quadrant of this warp
    const int quad = warp & 3;
    const int row = m0 + quad * 32 + lane;
    const bool ok = tc_wait(acc_full, 0u, p.err);
    tc_fence_after();
    if (ok) {
#pragma unroll 1
      for (int c0 = 0; c0 < BN; c0 += 32) {
        float v[32];
        tmem_ld32(tmem + (static_cast<uint32_t>(quad * 32) << 16) + static_cast<uint32_t>(c0), v);
        if (row < p.rows) {
          // all residual loads of the chunk first: y may alias resid, so a
          // load after a store would wait for the store's round trip
          if (p.resid) {
            float r[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const int t = t0 + c0 + j;
              r[j] = t < p.T ? p.resid[static_cast<size_t>(t) * p.y_ld + row] : 0.0f;
            }
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] += r[j];
          }
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const int t = t0 + c0 + j;
            if (t < p.T) p.y[static_cast<size_t>(t) * p.y_ld + row] = v[j];
          }
        }
      }
    }
  }
  pdl_launch_dependents();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
  }
}

// ---------------------------------------------------------------- persistent
// gemm_tc_persist_kernel: the same tile and numerics, one CTA per SM walking
// the tiles t = blockIdx.x, + gridDim.x, ... (row tile fastest).  Two TMEM
// accumulators of BN columns alternate between tiles: the MMA warp fills one
// while the epilogue warps drain the other (acc_full / acc_empty barriers),
// and the TMA ring of kTcPStages stages runs across tile boundaries, so
// neither the epilogue nor the next tile's pipeline fill stalls the tensor
// pipe.
template <int BN>
constexpr int tc_persist_stages() {
  return BN >= 256 ? 4 : (BN >= 128 ? 6 : 8);  // 192 KB of stages in each case
}

template <int BN>
constexpr size_t gemm_tc_persist_smem() {
  return static_cast<size_t>(tc_persist_stages<BN>()) * (kTcBM + BN) * kTcBK * 2 + 1024 + 256;
}

template <int BN>
__global__ void __launch_bounds__(kTcThreads, 1)
    gemm_tc_persist_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap xmap,
                           const __grid_constant__ GemmTcParams p) {
  static_assert(BN % 32 == 0 && BN >= 32 && BN <= 256, "N must be a multiple of 32 up to 256");
  constexpr uint32_t kABytes = kTcBM * kTcBK * 2, kBBytes = BN * kTcBK * 2;
  constexpr uint32_t kTmemCols = 2 * BN;  // two accumulators
  constexpr int kTcPStages = tc_persist_stages<BN>();
  static_assert(kTmemCols <= 512 && (kTmemCols & (kTmemCols - 1)) == 0, "TMEM allocation");
  extern __shared__ __align__(1024) uint8_t tcp_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(tcp_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* a_st = smem;
  uint8_t* b_st = smem + kTcPStages * kABytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(b_st + kTcPStages * kBBytes);
  uint64_t* empty = full + kTcPStages;
  uint64_t* acc_full = empty + kTcPStages;  // [2]
  uint64_t* acc_empty = acc_full + 2;       // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int mt = (p.rows + kTcBM - 1) / kTcBM, nt = (p.T + BN - 1) / BN;
  const int ntiles = mt * nt;
  const int nk = p.cols / kTcBK;

  if (warp == 0 && lane == 0) {
    for (int s = 0; s < kTcPStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 4);  // one arrival per epilogue warp
    }
    fence_mbar_init();
    tma_prefetch_desc(&wmap);
    tma_prefetch_desc(&xmap);
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(tmem_slot);
  pdl_wait();

  if (warp == 0) {
    if (lane == 0) {
      uint32_t it = 0;  // stage uses across all tiles of this CTA
      bool ok = true;
      #pragma unroll 1
      for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x) {
        const int m0 = (tile % mt) * kTcBM, t0 = (tile / mt) * BN;
        #pragma unroll 1
        for (int kt = 0; kt < nk; ++kt, ++it) {
          const int s = static_cast<int>(it % kTcPStages);
          ok = tc_wait(&empty[s], ((it / kTcPStages) & 1) ^ 1, p.err);
          if (!ok) break;
          mbar_arrive_expect_tx(&full[s], kABytes + kBBytes);
          tma_load_2d(a_st + s * kABytes, &wmap, kt * kTcBK, m0, &full[s]);
          tma_load_2d(b_st + s * kBBytes, &xmap, kt * kTcBK, t0, &full[s]);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_f16(BN);
      uint32_t it = 0;
      int local = 0;
      bool ok = true;
      #pragma unroll 1
      for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x, ++local) {
        const int b = local & 1;
        // the epilogue has drained this accumulator (its previous use)
        ok = tc_wait(&acc_empty[b], static_cast<uint32_t>(((local >> 1) & 1) ^ 1), p.err);
        if (!ok) break;
        tc_fence_after();
        const uint32_t acc = tmem + static_cast<uint32_t>(b * BN);
        #pragma unroll 1
        for (int kt = 0; kt < nk; ++kt, ++it) {
          const int s = static_cast<int>(it % kTcPStages);
          ok = tc_wait(&full[s], (it / kTcPStages) & 1, p.err);
          if (!ok) break;
          tc_fence_after();
          const uint32_t a0 = smem_u32(a_st + s * kABytes), b0 = smem_u32(b_st + s * kBBytes);
#pragma unroll
          for (int k = 0; k < kTcBK / 16; ++k)
            umma_f16(acc, umma_desc_sw128(a0 + 32 * k), umma_desc_sw128(b0 + 32 * k), idesc, (kt | k) != 0 ? 1u : 0u);
          umma_commit(&empty[s]);
        }
        umma_commit(&acc_full[b]);
      }
    }
  } else {
    const int quad = warp & 3;
    int local = 0;
    bool ok = true;
    #pragma unroll 1
    for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x, ++local) {
      const int b = local & 1;
      const int m0 = (tile % mt) * kTcBM, t0 = (tile / mt) * BN;
      const int row = m0 + quad * 32 + lane;
      ok = tc_wait(&acc_full[b], static_cast<uint32_t>((local >> 1) & 1), p.err);
      tc_fence_after();
      if (!ok) break;
#pragma unroll 1
      for (int c0 = 0; c0 < BN; c0 += 32) {
        float v[32];
        tmem_ld32(tmem + (static_cast<uint32_t>(quad * 32) << 16) + static_cast<uint32_t>(b * BN + c0), v);
        if (row < p.rows) {
          if (p.resid) {
            float r[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const int t = t0 + c0 + j;
              r[j] = t < p.T ? p.resid[static_cast<size_t>(t) * p.y_ld + row] : 0.0f;
            }
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] += r[j];
          }
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const int t = t0 + c0 + j;
            if (t < p.T) p.y[static_cast<size_t>(t) * p.y_ld + row] = v[j];
          }
        }
      }
      // this accumulator may be overwritten by the tile after next
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[b]);
    }
  }
  pdl_launch_dependents();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
  }
}

}  // namespace kib
