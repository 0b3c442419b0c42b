// decode_persistent.cuh -- one launch per decode token (T = 1).
//
// The bs1 decode step of the hybrid decoder after the token embedding (24
// layers of GDN or attention blocks with their FFNs, the fused LM-head argmax)
// runs as a single persistent grid: one CTA per SM, eight consumer warps and one
// producer warp.  The step is a host-built list of stages (PkStage); between
// dependent stages the consumers meet at a grid barrier.  The producer warp
// walks the same list independently and streams everything the consumers will
// read from HBM -- weight row tiles, the GDN state rows, the cached K/V rows --
// into a ring of shared-memory slots with cp.async.bulk, so the weight stream
// runs ahead across the barriers instead of restarting after every kernel
// boundary.  Weights are constant, so the producer starts them before
// griddepcontrol.wait (overlapping the previous token's tail); everything
// written by the previous step is read only after it.
//
// Stage kinds and the reference ops they carry (the same fused groups as the
// per-kernel path in kquant_gemv2.cuh / layer_kernels.cuh):
//   kPkGemv / kPkHead  K-quant matvec with a prologue (input, RMSNorm or per-head
//                      norm-gate) and
//                      per-segment epilogues (store, residual add, conv+silu,
//                      silu*up, argmax) -- q*_k_matvec, mps_backend.mm:295-463;
//                      rms_norm 1891-1921; ssm_conv 2376-2457; argmax 2681-2779
//   kPkGdn             split_qkv_l2_norm + gate/beta prepare + delta-rule
//                      update of 16 state rows (mps_backend.mm:2097-2153,
//                      2588-2605, 2307-2374)
//   kPkAttn            q/k norm + MRoPE, KV write at pos, split-K attention
//                      over the F16 cache (1991-2024, 2482-2527, 2943-3008)
//   kPkMerge           combine of the splits + sigmoid(gate)
//                      (qwen35_runtime.cpp:3347-3351)
//
// Every wait is bounded: a barrier or mbarrier wait that runs out raises the
// error flag, and all warps then leave the step (the producer first waits,
// again bounded, for the copies it has in flight).
#pragma once

#include "kquant_gemv.cuh"
#include "layer_kernels.cuh"

namespace kib {

constexpr int kPkWarps = 8;                    // consumer warps
constexpr int kPkConsumers = kPkWarps * 32;
// + one producer warpgroup (warps 8-11; warp 8 issues the copies).  The block
// launches at 168 registers a thread (384 x 168 = 64512); the producer
// warpgroup then gives back down to 40 and the consumers take 232:
// 256 x 232 + 128 x 40 = 64512, the launch total.
constexpr int kPkThreads = kPkConsumers + 128;
constexpr int kPkProducerRegs = 40;
constexpr int kPkConsumerRegs = 232;
constexpr int kPkSlots = 6;
constexpr int kPkSlotBytes = 32 * 1024;
constexpr int kPkMaxCols = 4096;
constexpr int kPkMaxSegs = 4;
constexpr int kPkMaxSplits = 128;
constexpr int kPkGdnRows = 16;  // state rows per GDN item
constexpr int kPkMaxTileRows = 256;  // rows of a GEMV tile

enum PkKind : int { kPkGemv = 0, kPkGdn = 1, kPkAttn = 2, kPkMerge = 3, kPkHead = 4 };

struct PkSeg {
  const uint8_t* w;   // this segment's rows (row_bytes each)
  const uint8_t* w2;  // gate/up pair: the up matrix (same rows)
  float* out;         // indexed by the row within the segment
  int row_begin;      // first stage row of the segment
  int rows;
  int epi;            // GemvEpilogue
  int pad;
};

struct __align__(16) PkStage {
  int kind;
  int barrier_after;  // grid barrier between this stage and the next
  // ---- GEMV / head
  int type;
  int cols;
  int row_bytes;
  int rows;           // sum of the segments' rows
  int tile_rows;
  int ntiles;
  int nseg;
  int paired;
  int prologue;
  int rg;             // lanes per row (16, 32 or 64)
  int head_dim;       // norm-gate head size
  float eps;
  PkSeg seg[kPkMaxSegs];
  const float* in;
  const float* norm_w;
  const float* gate;
  const float* resid;  // kEpiResidual: resid[row]
  float* conv_state;   // kEpiConv: [rows][3]
  const float* conv_w; // kEpiConv: [rows][4]
  // ---- GDN (one token)
  const float* conv_out;
  int C;
  const float* beta_raw;
  const float* alpha_raw;
  const float* dt_bias;
  const float* ssm_a;
  float* state;       // [Hv][128][128]
  float* gdn_out;     // [Hv*128]
  int key_heads;
  int value_heads;
  // ---- attention (one token)
  const float* qg;    // [heads][2*256] q | gate
  const float* kp;
  const float* vp;
  const float* q_norm;
  const float* k_norm;
  uint16_t* kcache;   // [cap][kv_heads*256]
  uint16_t* vcache;
  int heads;
  int kv_heads;
  float theta;
  int n_dims;
  int nsplit;         // splits per kv head (kv_heads * nsplit <= grid)
  float* part;        // [nsplit][heads][256 + 2]
  float* att_out;     // [heads*256]
};

struct PkProgram {
  const PkStage* stages;
  int nstages;
  int* pos;           // position of the token being decoded; advanced by the head
  int* token;         // in: the token; out: the argmax
  int* token_log;     // token_log[*step] = argmax, then ++*step
  int* step;
  float* prob_out;    // optional p(top1)
  unsigned* bar_ctr;  // grid barrier ticket (0 at launch; reset by the last CTA)
  unsigned* head_ctr; // LM-head last-CTA ticket
  float* cand_max;    // [grid]
  float* cand_sum;
  int* cand_idx;
  int* err;
  unsigned long long* trace;  // optional: CTA 0's [stage][start, prologue done, first tile, done]
};

struct PkShared {
  uint64_t full[kPkSlots];
  uint64_t empty[kPkSlots];
  PkStage desc[2];
  float red[kPkWarps][2];
  float gb[2];
  float best[16];
  float bsum[16];
  int bidx[16];
  int abort;
  int last;
  float4 ep[kPkMaxTileRows];   // GEMV: per-row epilogue inputs of the tile
  float4 epw[kPkMaxTileRows];
  __align__(16) float xs[kPkMaxCols + kPkMaxCols / 16];  // padded stage input; attention/GDN scratch
  float ws[kPkMaxSplits];
  float ls[kPkMaxSplits];
};

constexpr size_t kPkSmemBytes = static_cast<size_t>(kPkSlots) * kPkSlotBytes + sizeof(PkShared);

// named barrier over the eight consumer warps (the producer never joins)
KIB_DEV void pk_sync() { asm volatile("bar.sync 1, %0;" ::"n"(kPkConsumers) : "memory"); }

KIB_DEV unsigned ld_acquire_u32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// ------------------------------------------------------------------ tiles
// Row granule of a stage: rows per aligned bulk copy (row_bytes * granule is
// a multiple of 16), computed on the host; tiles and segments are multiples.

// Stage rows [r0, r0 + nr) of `stage` copied to dst (paired: the up rows to
// dst + kPkSlotBytes / 2).  Called by one lane per piece.
KIB_DEV uint32_t pk_tile_bytes(const PkStage& S, int r0, int nr) {
  (void)r0;
  const uint32_t b = static_cast<uint32_t>(nr) * static_cast<uint32_t>(S.row_bytes);
  return S.paired ? 2u * b : b;
}

// ------------------------------------------------------------------ producer
struct PkProducer {
  uint8_t* ring;
  PkShared* sh;
  uint32_t seq = 0;
  bool waited = false;
  int lane;
  int* err;
  uint64_t pol;

  // Waits for slot `seq` to be free (bounded); returns its address or null.
  KIB_DEV uint8_t* acquire() {
    const int slot = static_cast<int>(seq % kPkSlots);
    const uint32_t parity = ((seq / kPkSlots) & 1u) ^ 1u;
    int ok = 1;
    if (lane == 0) {
      ok = 0;
      #pragma unroll 1
      for (uint32_t i = 0; i < (1u << 22); ++i) {
        if (mbar_try_wait(&sh->empty[slot], parity)) {
          ok = 1;
          break;
        }
        if ((i & 255u) == 255u && *reinterpret_cast<volatile int*>(&sh->abort)) break;
        __nanosleep(200);  // the ring is full: leave the issue slots to the consumer warps
      }
      if (!ok) {
        if (!*reinterpret_cast<volatile int*>(&sh->abort)) atomicExch(err, 4);
        *reinterpret_cast<volatile int*>(&sh->abort) = 1;
      }
    }
    ok = __shfl_sync(0xffffffffu, ok, 0);
    return ok ? ring + static_cast<size_t>(slot) * kPkSlotBytes : nullptr;
  }
  KIB_DEV void expect(uint32_t bytes) {
    if (lane == 0) mbar_arrive_expect_tx(&sh->full[seq % kPkSlots], bytes);
    __syncwarp();
  }
  KIB_DEV uint64_t* bar() { return &sh->full[seq % kPkSlots]; }
  KIB_DEV void dep_wait() {
    if (!waited) {
      pdl_wait();
      waited = true;
    }
  }
};

KIB_DEV void pk_produce(const PkProgram& P, PkProducer& pr) {
  const int lane = pr.lane;
  const int grid = static_cast<int>(gridDim.x), cta = static_cast<int>(blockIdx.x);
  int pos = -1;
  #pragma unroll 1
  for (int s = 0; s < P.nstages; ++s) {
    const PkStage& S = P.stages[s];
    const int kind = S.kind;
    const uint32_t seq0 = pr.seq;
    unsigned long long* tr = (P.trace && cta == 0 && lane == 0) ? P.trace + 16 * s : nullptr;
    if (tr) tr[6] = gtimer();  // producer reached the stage
    if (kind == kPkGemv || kind == kPkHead) {
      #pragma unroll 1
      for (int t = cta; t < S.ntiles; t += grid) {
        uint8_t* dst = pr.acquire();
        if (!dst) return;
        const int r0 = t * S.tile_rows;
        const int nr = min(S.tile_rows, S.rows - r0);
        pr.expect(pk_tile_bytes(S, r0, nr));
        if (tr && pr.seq == seq0) tr[7] = gtimer();  // first tile issued
        if (lane < S.nseg) {
          const PkSeg& g = S.seg[lane];
          const int a = max(r0, g.row_begin), b = min(r0 + nr, g.row_begin + g.rows);
          if (a < b) {
            const size_t src = static_cast<size_t>(a - g.row_begin) * S.row_bytes;
            const uint32_t bytes = static_cast<uint32_t>(b - a) * static_cast<uint32_t>(S.row_bytes);
            uint8_t* d = dst + static_cast<size_t>(a - r0) * S.row_bytes;
            bulk_g2s_stream(d, g.w + src, bytes, pr.bar(), pr.pol);
            if (S.paired) bulk_g2s_stream(d + kPkSlotBytes / 2, g.w2 + src, bytes, pr.bar(), pr.pol);
          }
        }
        __syncwarp();
        ++pr.seq;
      }
    } else if (kind == kPkGdn) {
      const int items = S.value_heads * (128 / kPkGdnRows);
      #pragma unroll 1
      for (int it = cta; it < items; it += grid) {
        pr.dep_wait();  // the state was written by the previous step
        uint8_t* dst = pr.acquire();
        if (!dst) return;
        constexpr uint32_t bytes = kPkGdnRows * 128 * sizeof(float);
        pr.expect(bytes);
        if (lane == 0) bulk_g2s(dst, S.state + static_cast<size_t>(it) * kPkGdnRows * 128, bytes, pr.bar());
        __syncwarp();
        ++pr.seq;
      }
    } else if (kind == kPkAttn) {
      if (cta >= S.kv_heads * S.nsplit) continue;
      pr.dep_wait();
      if (pos < 0) pos = *P.pos;
      const int kvh = cta / S.nsplit, split = cta % S.nsplit;
      const int nkeys = pos + 1;
      int chunk = (nkeys + S.nsplit - 1) / S.nsplit;
      chunk = (chunk + 7) & ~7;
      const int kb = split * chunk, old_end = min(kb + chunk, pos);
      const int kvd = S.kv_heads * kHd;
      #pragma unroll 1
      for (int k0 = kb; k0 < old_end; k0 += kAttnChunk) {
        uint8_t* dst = pr.acquire();
        if (!dst) return;
        const int nk = min(kAttnChunk, old_end - k0);
        pr.expect(static_cast<uint32_t>(nk) * 2u * kHd * 2u);
        if (lane < nk) {
          const size_t src = static_cast<size_t>(k0 + lane) * kvd + kvh * kHd;
          uint8_t* d = dst + static_cast<size_t>(lane) * 2 * kHd * 2;
          bulk_g2s(d, S.kcache + src, kHd * 2, pr.bar());
          bulk_g2s(d + kHd * 2, S.vcache + src, kHd * 2, pr.bar());
        }
        __syncwarp();
        ++pr.seq;
      }
    }
  }
}

// ------------------------------------------------------------------ consumers
struct PkCons {
  uint8_t* ring;
  PkShared* sh;
  uint32_t seq = 0;
  int* err;
  unsigned long long* tr = nullptr;  // trace of the current stage (CTA 0, thread 0) or null
  bool first = true;

  // Waits for the next ring slot (all consumer threads); null on abort.
  KIB_DEV const uint8_t* take() {
    const int slot = static_cast<int>(seq % kPkSlots);
    if (!mbar_wait_bounded(&sh->full[slot], (seq / kPkSlots) & 1u, err)) {
      sh->abort = 1;
      return nullptr;
    }
    if (tr && first) {
      tr[2] = gtimer();
      first = false;
    }
    return ring + static_cast<size_t>(slot) * kPkSlotBytes;
  }
  // Every consumer thread is done with the slot.
  KIB_DEV void release() {
    pk_sync();
    if (threadIdx.x == 0) mbar_arrive(&sh->empty[seq % kPkSlots]);
    ++seq;
  }
};

// Grid barrier of the consumer warps of all CTAs.  Returns false on abort.
KIB_DEV bool pk_grid_sync(const PkProgram& P, PkShared* sh, unsigned target) {
  pk_sync();  // the CTA's writes happen before thread 0's release below
  if (threadIdx.x == 0) {
    asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(P.bar_ctr) : "memory");
    uint32_t i = 0;
    while (ld_acquire_u32(P.bar_ctr) < target) {
      ++i;
      if ((i & 63u) == 0u && *reinterpret_cast<volatile int*>(P.err) != 0) {
        sh->abort = 1;
        break;
      }
      if (i > (1u << 22)) {
        atomicExch(P.err, 5);
        sh->abort = 1;
        break;
      }
    }
  }
  pk_sync();
  return !*reinterpret_cast<volatile int*>(&sh->abort);
}

KIB_DEV void pk_copy_desc(PkStage* dst, const PkStage* src) {
  constexpr int n = static_cast<int>(sizeof(PkStage) / 16);
  static_assert(sizeof(PkStage) % 16 == 0, "PkStage must be a multiple of 16 bytes");
  static_assert(n <= kPkConsumers, "one descriptor word per consumer thread");
  #pragma unroll 1
  for (int i = threadIdx.x; i < n; i += kPkConsumers)
    reinterpret_cast<uint4*>(dst)[i] = __ldg(reinterpret_cast<const uint4*>(src) + i);
}

// ---- GEMV prologue: the stage's transformed input vector into sh->xs
// The stage input lives in shared memory with 4 floats of padding after every
// 64: the 16 lanes of a row group read their units (64 consecutive inputs for
// Q4_K) at a stride of 68 floats, which spreads them over the banks.
KIB_DEV int xpad(int i) { return i + 4 * (i >> 6); }

// Prologue: every thread issues all of its loads (input, norm weights, gate)
// before the first reduction, so the stage start costs one memory round trip.
KIB_DEV void pk_prologue(const PkStage& S, PkShared* sh) {
  float* xs = sh->xs;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int cols = S.cols;
  if (S.prologue == kProNormGate) {
    // qk_norm over heads of 128 (one warp per head), silu(gate), mul
    // (qwen35_runtime.cpp:2993-3003)
    constexpr int hd = 128;
    const float4 w = *reinterpret_cast<const float4*>(S.norm_w + 4 * lane);
#pragma unroll 1
    for (int base = warp * hd; base < cols; base += kPkWarps * hd) {
      const float4 y = *reinterpret_cast<const float4*>(S.in + base + 4 * lane);
      const float4 z = *reinterpret_cast<const float4*>(S.gate + base + 4 * lane);
      const float ss = warp_sum((y.x * y.x + y.y * y.y) + (y.z * y.z + y.w * y.w));
      const float scale = 1.0f / sqrtf(ss / static_cast<float>(hd) + S.eps);
      float4 o;
      o.x = y.x * (scale * w.x) * silu_f(z.x);
      o.y = y.y * (scale * w.y) * silu_f(z.y);
      o.z = y.z * (scale * w.z) * silu_f(z.z);
      o.w = y.w * (scale * w.w) * silu_f(z.w);
      *reinterpret_cast<float4*>(xs + xpad(base + 4 * lane)) = o;
    }
    pk_sync();
    return;
  }
  constexpr int kPer = kPkMaxCols / (4 * kPkConsumers);  // float4 per thread
  float4 v[kPer], w[kPer];
  float ss = 0.0f;
  const bool rms = S.prologue == kProRms;
#pragma unroll
  for (int k = 0; k < kPer; ++k) {
    const int i = 4 * tid + 4 * kPkConsumers * k;
    if (i < cols) {
      v[k] = *reinterpret_cast<const float4*>(S.in + i);
      if (rms) w[k] = *reinterpret_cast<const float4*>(S.norm_w + i);
    }
  }
#pragma unroll
  for (int k = 0; k < kPer; ++k) {
    const int i = 4 * tid + 4 * kPkConsumers * k;
    if (i < cols) ss += (v[k].x * v[k].x + v[k].y * v[k].y) + (v[k].z * v[k].z + v[k].w * v[k].w);
  }
  float scale = 1.0f;
  if (rms) {
    // rms_norm_f32_f32_batched (mps_backend.mm:1891-1921): x * rsqrt(mean(x^2)+eps) * w
    ss = warp_sum(ss);
    if (lane == 0) sh->red[warp][0] = ss;
    pk_sync();
    float tot = 0.0f;
#pragma unroll
    for (int q = 0; q < kPkWarps; ++q) tot += sh->red[q][0];
    scale = 1.0f / sqrtf(tot / static_cast<float>(cols) + S.eps);
  }
#pragma unroll
  for (int k = 0; k < kPer; ++k) {
    const int i = 4 * tid + 4 * kPkConsumers * k;
    if (i < cols) {
      float4 o = v[k];
      if (rms) {
        o.x = o.x * scale * w[k].x;
        o.y = o.y * scale * w[k].y;
        o.z = o.z * scale * w[k].z;
        o.w = o.w * scale * w[k].w;
      }
      *reinterpret_cast<float4*>(xs + xpad(i)) = o;
    }
  }
  pk_sync();
}

// x values of unit u of block blk from the padded stage input (element order
// as unit_col, group sums as load_unit_x).
template <int QT>
KIB_DEV void pk_load_unit_x(const float* xs, int blk, int u, UnitX<QT>& ux) {
  if (QT == kTypeQ6K) {
    const int c = u >> 1, r = u & 1;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float4* p = reinterpret_cast<const float4*>(xs + 68 * (4 * blk + 2 * c + (k >> 1)) + 32 * (k & 1) + 16 * r);
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
    const float4* p = reinterpret_cast<const float4*>(xs + 68 * (4 * blk + u));
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

struct PkArgmax {
  float best = -INFINITY, bsum = 0.0f;
  int bidx = 0x7FFFFFFF;
  KIB_DEV void push(float v, int row) {
    if (v > best || (v == best && row < bidx)) {
      bsum = bsum * expf(best - v) + 1.0f;
      best = v;
      bidx = row;
    } else {
      bsum += expf(v - best);
    }
  }
};

KIB_DEV int pk_seg_of(const PkStage& S, int r) {
  int s = 0;
  if (S.nseg > 1 && r >= S.seg[1].row_begin) s = 1;
  if (S.nseg > 2 && r >= S.seg[2].row_begin) s = 2;
  if (S.nseg > 3 && r >= S.seg[3].row_begin) s = 3;
  return s;
}

template <int QT>
KIB_DEV bool pk_gemv(const PkStage& S, PkCons& cs, PkArgmax& am) {
  constexpr int BB = kquant_block_bytes(QT);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int RG = S.rg;
  const int groups = kPkConsumers / RG;
  const int group = tid / RG, gl = tid % RG;
  const bool active = gl < S.cols / 64;
  const int blk = gl >> 2, u = gl & 3;
  UnitX<QT> ux[1];
  if (cs.tr) {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t) : "r"(blk));
    cs.tr[8] = t;
  }
  if (active) pk_load_unit_x<QT>(cs.sh->xs, blk, u, ux[0]);
  if (cs.tr) {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t) : "f"(ux[0].v[31].y));
    cs.tr[9] = t;
    UnitX<QT> ux2;
    pk_load_unit_x<QT>(cs.sh->xs, blk, u ^ 1, ux2);
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t) : "f"(ux2.v[31].y));
    cs.tr[10] = t;
  }
  if (cs.tr) {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t) : "f"(ux[0].v[31].y));
    cs.tr[4] = t;
  }
  const int grid = static_cast<int>(gridDim.x);
  #pragma unroll 1
  for (int t = static_cast<int>(blockIdx.x); t < S.ntiles; t += grid) {
    const int r0 = t * S.tile_rows;
    const int nr = min(S.tile_rows, S.rows - r0);
    // the epilogue inputs of every row of the tile (residual, conv state and
    // weights) are loaded at once, before the tile is waited for
    if (tid < nr) {
      const int si = pk_seg_of(S, r0 + tid);
      const int row = r0 + tid - S.seg[si].row_begin;
      const int epi = S.seg[si].epi;
      if (epi == kEpiResidual) {
        cs.sh->ep[tid] = make_float4(S.resid[row], 0.f, 0.f, 0.f);
      } else if (epi == kEpiConv) {
        const float* st = S.conv_state + static_cast<size_t>(row) * 3;
        cs.sh->ep[tid] = make_float4(st[0], st[1], st[2], 0.f);
        cs.sh->epw[tid] = *reinterpret_cast<const float4*>(S.conv_w + static_cast<size_t>(row) * 4);
      }
    }
    const uint8_t* tile = cs.take();
    if (!tile) return false;
    pk_sync();  // ep / epw
    const bool trt = cs.tr && t == static_cast<int>(blockIdx.x);
    if (trt) cs.tr[8] = gtimer();
    const int passes = (nr + groups - 1) / groups;
#pragma unroll 1
    for (int pass = 0; pass < passes; ++pass) {
      const int rl = pass * groups + group;
      const bool ok = rl < nr;
      const int r = r0 + rl;
      int si = 0, row = 0, epi = kEpiStore;
      float pre0 = 0.0f, pre1 = 0.0f, pre2 = 0.0f;
      float4 cw = make_float4(0.f, 0.f, 0.f, 0.f);
      if (gl == 0 && ok) {
        si = pk_seg_of(S, r);
        row = r - S.seg[si].row_begin;
        epi = S.seg[si].epi;
        const float4 e = cs.sh->ep[rl];
        pre0 = e.x;
        pre1 = e.y;
        pre2 = e.z;
        if (epi == kEpiConv) cw = cs.sh->epw[rl];
      }
      float acc[1] = {0.0f}, acc2[1] = {0.0f};
      if (ok && active) {
        const uint8_t* b0 = tile + static_cast<size_t>(rl) * S.row_bytes + blk * BB;
        // gate and up rows of a pair run through one copy of the dot code
#pragma unroll 1
        for (int hh = 0; hh <= S.paired; ++hh) {
          float a[1] = {0.0f};
          unit_dot<QT, 1>(b0 + hh * (kPkSlotBytes / 2), u, ux, a);
          if (hh == 0) acc[0] = a[0]; else acc2[0] = a[0];
        }
      }
      if (trt && pass == 0) {
        unsigned long long tt;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(tt) : "f"(acc[0]));
        cs.tr[9] = tt;
      }
      const int lim = RG < 32 ? RG : 32;
      for (int o = lim / 2; o > 0; o >>= 1) {
        acc[0] += __shfl_xor_sync(0xffffffffu, acc[0], o);
        if (S.paired) acc2[0] += __shfl_xor_sync(0xffffffffu, acc2[0], o);
      }
      if (RG > 32) {
        if (lane == 0) {
          cs.sh->red[warp][0] = acc[0];
          cs.sh->red[warp][1] = acc2[0];
        }
        pk_sync();
        if (gl == 0) {
          #pragma unroll 1
          for (int w = 1; w < RG / 32; ++w) {
            acc[0] += cs.sh->red[warp + w][0];
            acc2[0] += cs.sh->red[warp + w][1];
          }
        }
        pk_sync();
      }
      if (gl == 0 && ok) {
        const PkSeg& g = S.seg[si];
        const float v = acc[0];
        if (epi == kEpiStore) {
          g.out[row] = v;
        } else if (epi == kEpiResidual) {
          g.out[row] = v + pre0;
        } else if (epi == kEpiSiluMul) {
          g.out[row] = silu_f(v) * acc2[0];
        } else if (epi == kEpiConv) {
          // causal depthwise conv of kernel 4 over [state | new], then silu
          float c = 0.0f;
          c += pre0 * cw.x;
          c += pre1 * cw.y;
          c += pre2 * cw.z;
          c += v * cw.w;
          g.out[row] = silu_f(c);
          float* st = S.conv_state + static_cast<size_t>(row) * 3;
          st[0] = pre1;
          st[1] = pre2;
          st[2] = v;
        } else {  // kEpiArgmax
          am.push(v, row);
          if (g.out) g.out[row] = v;
        }
      }
      if (trt && pass == 0) cs.tr[10] = gtimer();
    }
    if (trt) cs.tr[11] = gtimer();
    cs.release();
    if (trt) cs.tr[12] = gtimer();
  }
  return true;
}

// ---- GDN: items of (value head, 16 state rows); warp w updates rows 2w, 2w+1
KIB_DEV bool pk_gdn(const PkStage& S, PkCons& cs) {
  constexpr int D = 128;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  float* qn = cs.sh->xs;
  float* kn = cs.sh->xs + D;
  const int items = S.value_heads * (D / kPkGdnRows);
  const int key_dim = S.key_heads * D;
  const float scale = 1.0f / sqrtf(static_cast<float>(D));
  #pragma unroll 1
  for (int it = static_cast<int>(blockIdx.x); it < items; it += static_cast<int>(gridDim.x)) {
    const int h = it / (D / kPkGdnRows), grp = it % (D / kPkGdnRows);
    const int kh = h % S.key_heads;
    float qv = 0.0f, kv = 0.0f;
    if (tid < D) {
      qv = S.conv_out[kh * D + tid];
      kv = S.conv_out[key_dim + kh * D + tid];
      const float q2 = warp_sum(qv * qv), k2 = warp_sum(kv * kv);
      if (lane == 0) {
        cs.sh->red[warp][0] = q2;
        cs.sh->red[warp][1] = k2;
      }
    }
    if (tid == 0) {
      const float a = S.alpha_raw[h];
      const float b = S.beta_raw[h];
      cs.sh->gb[0] = softplus20_f(a + S.dt_bias[h]) * S.ssm_a[h];
      cs.sh->gb[1] = sigmoid_f(b);
    }
    pk_sync();
    if (tid < D) {
      const float* r0 = &cs.sh->red[0][0];
      const float qsum = (r0[0] + r0[2]) + (r0[4] + r0[6]);
      const float ksum = (r0[1] + r0[3]) + (r0[5] + r0[7]);
      qn[tid] = qv * (1.0f / fmaxf(sqrtf(qsum), S.eps));
      kn[tid] = kv * (1.0f / fmaxf(sqrtf(ksum), S.eps));
    }
    const float ge = expf(cs.sh->gb[0]);
    const float beta = cs.sh->gb[1];
    const uint8_t* tile = cs.take();
    if (!tile) return false;
    pk_sync();  // qn/kn
    const float4 k4 = *reinterpret_cast<const float4*>(kn + 4 * lane);
    const float4 q4 = *reinterpret_cast<const float4*>(qn + 4 * lane);
    const float* srows = reinterpret_cast<const float*>(tile);
#pragma unroll
    for (int rr = 0; rr < 2; ++rr) {
      const int lr = 2 * warp + rr;
      const int vrow = grp * kPkGdnRows + lr;
      float4 st = *reinterpret_cast<const float4*>(srows + lr * D + 4 * lane);
      st.x *= ge;
      st.y *= ge;
      st.z *= ge;
      st.w *= ge;
      const float sk = warp_sum(st.x * k4.x + st.y * k4.y + st.z * k4.z + st.w * k4.w);
      const float v = S.conv_out[2 * key_dim + h * D + vrow];
      const float delta = (v - sk) * beta;
      st.x += k4.x * delta;
      st.y += k4.y * delta;
      st.z += k4.z * delta;
      st.w += k4.w * delta;
      const float y = warp_sum(st.x * q4.x + st.y * q4.y + st.z * q4.z + st.w * q4.w);
      if (lane == 0) S.gdn_out[h * D + vrow] = y * scale;
      *reinterpret_cast<float4*>(S.state + (static_cast<size_t>(h) * D + vrow) * D + 4 * lane) = st;
    }
    cs.release();  // also orders qn/kn reuse
  }
  return true;
}

// Sums 8 values over the warp; every lane ends with the 8 totals.  Three
// halving exchanges leave each lane one value summed over 8 lanes, two more
// finish it, and 8 broadcasts return the totals (17 shuffles instead of 40).
KIB_DEV void pk_warp_sum8(float (&v)[8], int lane) {
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

// qk_norm (mps_backend.mm:1991-2024) then mrope (2482-2527) of one 256-wide
// head vector; text positions (all MRoPE streams equal); one warp.
__device__ __noinline__ void pk_norm_rope(float* v, const float* in, const float* w, float eps, float theta, int n_dims, int position,
                          int lane) {
  float ss = 0.0f;
  #pragma unroll 1
  for (int i = lane; i < kHd; i += 32) {
    const float x = in[i];
    ss += x * x;
  }
  ss = warp_sum(ss);
  const float scale = 1.0f / sqrtf(ss / static_cast<float>(kHd) + eps);
  #pragma unroll 1
  for (int i = lane; i < kHd; i += 32) v[i] = in[i] * (scale * w[i]);
  __syncwarp();
  const int half = n_dims / 2;
  #pragma unroll 1
  for (int pi = lane; pi < half; pi += 32) {
    const float exponent = static_cast<float>(2 * pi) / static_cast<float>(n_dims);
    const float freq = 1.0f / powf(theta, exponent);
    const float angle = static_cast<float>(position) * freq;
    float sn, csn;
    sincosf(angle, &sn, &csn);
    const float x0 = v[pi], x1 = v[half + pi];
    v[pi] = x0 * csn - x1 * sn;
    v[half + pi] = x1 * csn + x0 * sn;
  }
  __syncwarp();
}

// ---- attention: item = (kv head, split); warp w serves q head (w % 4) of the
// group and every other block of 8 keys (w / 4)
KIB_DEV bool pk_attn(const PkStage& S, PkCons& cs, int pos) {
  constexpr int G = 4;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int cta = static_cast<int>(blockIdx.x);
  if (cta >= S.kv_heads * S.nsplit) return true;
  float* qs = cs.sh->xs;               // [4][256]
  float* newk = qs + G * kHd;          // [256]
  float* newv = newk + kHd;            // [256]
  float* merge = newv + kHd;           // [8][258]
  const int kvh = cta / S.nsplit, split = cta % S.nsplit;
  const int kvd = S.kv_heads * kHd;
  const int nkeys = pos + 1;
  int chunk = (nkeys + S.nsplit - 1) / S.nsplit;
  chunk = (chunk + 7) & ~7;
  const int kb = split * chunk, ke = min(kb + chunk, nkeys);
  const int old_end = min(ke, pos);
  const bool owner = pos >= kb && pos < ke;
  if (warp < G) {
    const int head = kvh * G + warp;
    pk_norm_rope(qs + warp * kHd, S.qg + static_cast<size_t>(head) * 2 * kHd, S.q_norm, S.eps, S.theta, S.n_dims, pos,
                 lane);
  } else if (warp == G && owner) {
    pk_norm_rope(newk, S.kp + kvh * kHd, S.k_norm, S.eps, S.theta, S.n_dims, pos, lane);
    #pragma unroll 1
    for (int i = lane; i < kHd; i += 32) {
      const __half kh = __float2half_rn(newk[i]);
      const __half vh = __float2half_rn(S.vp[kvh * kHd + i]);
      S.kcache[static_cast<size_t>(pos) * kvd + kvh * kHd + i] = __half_as_ushort(kh);
      S.vcache[static_cast<size_t>(pos) * kvd + kvh * kHd + i] = __half_as_ushort(vh);
      newk[i] = __half2float(kh);
      newv[i] = __half2float(vh);
    }
  }
  pk_sync();
  const int j = warp % G, kh2 = warp / G;
  const float scale = 1.0f / sqrtf(static_cast<float>(kHd));
  float m = -INFINITY, l = 0.0f, acc[8], qreg[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    acc[i] = 0.0f;
    qreg[i] = qs[j * kHd + 8 * lane + i];
  }
  constexpr int KB = 8;
  #pragma unroll 1
  for (int k0 = kb; k0 < old_end; k0 += kAttnChunk) {
    const uint8_t* tile = cs.take();
    if (!tile) return false;
    const uint16_t* kvbuf = reinterpret_cast<const uint16_t*>(tile);
    const int nk = min(kAttnChunk, old_end - k0);
#pragma unroll 1
    for (int kk0 = kh2 * KB; kk0 < nk; kk0 += 2 * KB) {
      float sc[KB];
      uint4 vraw[KB];
#pragma unroll
      for (int e = 0; e < KB; ++e) {
        const int kk = min(kk0 + e, nk - 1);
        const uint16_t* row = kvbuf + static_cast<size_t>(kk) * 2 * kHd;
        const uint4 kr = *reinterpret_cast<const uint4*>(row + 8 * lane);
        vraw[e] = *reinterpret_cast<const uint4*>(row + kHd + 8 * lane);
        const __half2* kh = reinterpret_cast<const __half2*>(&kr);
        float d = 0.0f;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 a2 = __half22float2(kh[i]);
          d = fmaf(qreg[2 * i], a2.x, d);
          d = fmaf(qreg[2 * i + 1], a2.y, d);
        }
        sc[e] = d;
      }
      pk_warp_sum8(sc, lane);
#pragma unroll
      for (int e = 0; e < KB; ++e) sc[e] *= scale;
      float mx = m;
#pragma unroll
      for (int e = 0; e < KB; ++e)
        if (kk0 + e < nk) mx = fmaxf(mx, sc[e]);
      const float ps = expf(m - mx);
      l *= ps;
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] *= ps;
#pragma unroll
      for (int e = 0; e < KB; ++e) {
        if (kk0 + e >= nk) break;
        const float w = expf(sc[e] - mx);
        l += w;
        const __half2* vh = reinterpret_cast<const __half2*>(&vraw[e]);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 b2 = __half22float2(vh[i]);
          acc[2 * i] = fmaf(w, b2.x, acc[2 * i]);
          acc[2 * i + 1] = fmaf(w, b2.y, acc[2 * i + 1]);
        }
      }
      m = mx;
    }
    cs.release();
  }
  if (owner && kh2 == 0) {  // the new key, from shared memory
    float d = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) d = fmaf(qreg[i], newk[8 * lane + i], d);
    const float sc = warp_sum(d) * scale;
    const float nm = fmaxf(m, sc);
    const float ps = expf(m - nm);
    const float w = expf(sc - nm);
    l = l * ps + w;
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] = acc[i] * ps + w * newv[8 * lane + i];
    m = nm;
  }
  // merge the two key halves of each head, then write the split's partial
  float* mrow = merge + warp * (kHd + 2);
#pragma unroll
  for (int i = 0; i < 8; ++i) mrow[8 * lane + i] = acc[i];
  if (lane == 0) {
    mrow[kHd] = m;
    mrow[kHd + 1] = l;
  }
  pk_sync();
  #pragma unroll 1
  for (int job = tid; job < G * kHd; job += kPkConsumers) {
    const int i = job % kHd, jj = job / kHd;
    const float* a = merge + jj * (kHd + 2);
    const float* b = merge + (jj + G) * (kHd + 2);
    const float ma = a[kHd], mb = b[kHd];
    const float M = fmaxf(ma, mb);
    const float ea = ma == -INFINITY ? 0.0f : expf(ma - M);
    const float eb = mb == -INFINITY ? 0.0f : expf(mb - M);
    float* dst = S.part + (static_cast<size_t>(split) * S.heads + kvh * G + jj) * (kHd + 2);
    dst[i] = a[i] * ea + b[i] * eb;
    if (i == 0) {
      dst[kHd] = M;
      dst[kHd + 1] = a[kHd + 1] * ea + b[kHd + 1] * eb;
    }
  }
  pk_sync();
  return true;
}

// ---- merge: item = (head, 16 output dims); thread = (dim, split lane)
KIB_DEV void pk_merge(const PkStage& S, PkShared* sh) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int items = S.heads * (kHd / 16);
  const int ns = S.nsplit;
  #pragma unroll 1
  for (int it = static_cast<int>(blockIdx.x); it < items; it += static_cast<int>(gridDim.x)) {
    const int h = it / (kHd / 16), d0 = (it % (kHd / 16)) * 16;
    #pragma unroll 1
    for (int s = tid; s < ns; s += kPkConsumers) {
      const float* src = S.part + (static_cast<size_t>(s) * S.heads + h) * (kHd + 2) + kHd;
      sh->ws[s] = __ldcg(src);
      sh->ls[s] = __ldcg(src + 1);
    }
    pk_sync();
    if (warp == 0) {
      float M = -INFINITY;
      #pragma unroll 1
      for (int s = lane; s < ns; s += 32) M = fmaxf(M, sh->ws[s]);
      M = warp_max(M);
      float den = 0.0f;
      #pragma unroll 1
      for (int s = lane; s < ns; s += 32) {
        const float ms = sh->ws[s];
        const float e = ms == -INFINITY ? 0.0f : expf(ms - M);
        sh->ws[s] = e;
        den += sh->ls[s] * e;
      }
      den = warp_sum(den);
      if (lane == 0) sh->gb[0] = den;
    }
    pk_sync();
    const int d = tid & 15, jl = tid >> 4;  // 16 split lanes
    float n = 0.0f;
    #pragma unroll 1
    for (int s = jl; s < ns; s += kPkConsumers / 16)
      n = fmaf(__ldcg(S.part + (static_cast<size_t>(s) * S.heads + h) * (kHd + 2) + d0 + d), sh->ws[s], n);
    n += __shfl_xor_sync(0xffffffffu, n, 16);
    float* part = sh->xs;                     // [8 warps][16]
    if (lane < 16) part[warp * 16 + d] = n;
    pk_sync();
    if (tid < 16) {
      float tot = 0.0f;
#pragma unroll
      for (int w = 0; w < kPkWarps; ++w) tot += part[w * 16 + tid];
      const float den = sh->gb[0];
      const float inv = den == 0.0f ? 0.0f : 1.0f / den;
      const float g = S.qg[static_cast<size_t>(h) * 2 * kHd + kHd + d0 + tid];
      S.att_out[h * kHd + d0 + tid] = tot * inv * sigmoid_f(g);
    }
    pk_sync();
  }
}

// ---- LM head tail: CTA candidate, then the last CTA picks the token
KIB_DEV void pk_head_finish(const PkProgram& P, const PkStage& S, PkShared* sh, const PkArgmax& am) {
  const int tid = threadIdx.x, lane = tid & 31;
  const int groups = kPkConsumers / S.rg;
  const int group = tid / S.rg, gl = tid % S.rg;
  if (gl == 0) {
    sh->best[group] = am.best;
    sh->bsum[group] = am.bsum;
    sh->bidx[group] = am.bidx;
  }
  pk_sync();
  if (tid == 0) {
    float m = -INFINITY, s = 0.0f;
    int idx = 0x7FFFFFFF;
    #pragma unroll 1
    for (int g = 0; g < groups; ++g) {
      const int gi = sh->bidx[g];
      if (gi == 0x7FFFFFFF) continue;
      const float gm = sh->best[g], gs = sh->bsum[g];
      if (gm > m || (gm == m && gi < idx)) {
        s = s * expf(m - gm) + gs;
        m = gm;
        idx = gi;
      } else {
        s += gs * expf(gm - m);
      }
    }
    P.cand_max[blockIdx.x] = m;
    P.cand_sum[blockIdx.x] = s;
    P.cand_idx[blockIdx.x] = idx;
    __threadfence();
    sh->last = atomicAdd(P.head_ctr, 1u) == gridDim.x - 1;
  }
  pk_sync();
  if (!sh->last || tid >= 32) return;
  __threadfence();
  float m = -INFINITY, s = 0.0f;
  int idx = 0x7FFFFFFF;
  #pragma unroll 1
  for (unsigned c = lane; c < gridDim.x; c += 32) {
    const int gi = __ldcg(&P.cand_idx[c]);
    if (gi == 0x7FFFFFFF) continue;
    const float gm = __ldcg(&P.cand_max[c]), gs = __ldcg(&P.cand_sum[c]);
    if (gm > m || (gm == m && gi < idx)) {
      s = s * expf(m - gm) + gs;
      m = gm;
      idx = gi;
    } else {
      s += gs * expf(gm - m);
    }
  }
  for (int o = 16; o > 0; o >>= 1) {
    const float om = __shfl_xor_sync(0xffffffffu, m, o);
    const float os = __shfl_xor_sync(0xffffffffu, s, o);
    const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
    if (oi == 0x7FFFFFFF) continue;
    if (idx == 0x7FFFFFFF || om > m || (om == m && oi < idx)) {
      s = (idx == 0x7FFFFFFF ? 0.0f : s * expf(m - om)) + os;
      m = om;
      idx = oi;
    } else {
      s += os * expf(om - m);
    }
  }
  if (lane == 0) {
    P.token[0] = idx;
    if (P.prob_out) P.prob_out[0] = 1.0f / s;
    if (P.token_log) {
      const int st = *P.step;
      P.token_log[st] = idx;
      *P.step = st + 1;
    }
    *P.pos = *P.pos + 1;
    *P.head_ctr = 0u;
    *P.bar_ctr = 0u;  // every CTA has passed its last barrier
    __threadfence();
  }
}

__global__ void __launch_bounds__(kPkThreads, 1) decode_persistent_kernel(const __grid_constant__ PkProgram P) {
  extern __shared__ __align__(1024) uint8_t pk_smem[];
  uint8_t* ring = pk_smem;
  PkShared* sh = reinterpret_cast<PkShared*>(pk_smem + static_cast<size_t>(kPkSlots) * kPkSlotBytes);
  const int tid = threadIdx.x, warp = tid >> 5;
  if (tid == 0) {
    for (int i = 0; i < kPkSlots; ++i) {
      mbar_init(&sh->full[i], 1);
      mbar_init(&sh->empty[i], 1);
    }
    sh->abort = 0;
    fence_mbar_init();
  }
  __syncthreads();
  if (warp >= kPkWarps) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kPkProducerRegs));
    pdl_launch_dependents();
    if (warp != kPkWarps) return;
    PkProducer pr;
    pr.ring = ring;
    pr.sh = sh;
    pr.lane = tid & 31;
    pr.err = P.err;
    pr.pol = l2_evict_first_policy();
    pk_produce(P, pr);
    // leave only once the copies in flight have landed (bounded)
    if (pr.lane == 0) {
      const uint32_t n = min(pr.seq, static_cast<uint32_t>(kPkSlots));
      #pragma unroll 1
      for (uint32_t q = pr.seq - n; q < pr.seq; ++q) {
        for (uint32_t i = 0; i < (1u << 22); ++i)
          if (mbar_try_wait(&sh->full[q % kPkSlots], (q / kPkSlots) & 1u)) break;
      }
    }
    return;
  }
  // ---------------------------------------------------------------- consumers
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kPkConsumerRegs));
  pdl_wait();
  pdl_launch_dependents();
  const int pos = *P.pos;
  PkCons cs;
  cs.ring = ring;
  cs.sh = sh;
  cs.err = P.err;
  PkArgmax am;
  unsigned barriers = 0;
  pk_copy_desc(&sh->desc[0], &P.stages[0]);
  pk_sync();
  #pragma unroll 1
  for (int s = 0; s < P.nstages; ++s) {
    const PkStage& S = sh->desc[s & 1];
    // the next stage's descriptor: loaded now, stored after this stage's work
    constexpr int kDescWords = static_cast<int>(sizeof(PkStage) / 16);
    uint4 next_desc = make_uint4(0u, 0u, 0u, 0u);
    if (tid < kDescWords && s + 1 < P.nstages) next_desc = __ldg(reinterpret_cast<const uint4*>(&P.stages[s + 1]) + tid);
    cs.tr = (P.trace && blockIdx.x == 0 && tid == 0) ? P.trace + 16 * s : nullptr;
    cs.first = true;
    if (cs.tr) cs.tr[0] = gtimer();
    bool ok = true;
    if (S.kind == kPkGemv || S.kind == kPkHead) {
      pk_prologue(S, sh);
      if (cs.tr) cs.tr[1] = gtimer();
      switch (S.type) {
        // Q5_K matrices are not instantiated here (both 4-bit paths in one
        // kernel push it into local memory); the host routes models that
        // have them to the per-kernel path
        case kTypeQ4K: ok = pk_gemv<kTypeQ4K>(S, cs, am); break;
        default: ok = pk_gemv<kTypeQ6K>(S, cs, am); break;
      }
      if (ok && S.kind == kPkHead) pk_head_finish(P, S, sh, am);
    } else if (S.kind == kPkGdn) {
      ok = pk_gdn(S, cs);
    } else if (S.kind == kPkAttn) {
      ok = pk_attn(S, cs, pos);
    } else {
      pk_merge(S, sh);
    }
    if (!ok) break;
    if (cs.tr) cs.tr[3] = gtimer();
    if (P.trace && tid == 0) atomicMax(P.trace + 16 * s + 5, gtimer());  // slowest CTA done
    if (s + 1 < P.nstages) {
      const bool need_barrier = S.barrier_after != 0;
      if (tid < kDescWords) reinterpret_cast<uint4*>(&sh->desc[(s + 1) & 1])[tid] = next_desc;
      if (need_barrier) {
        ++barriers;
        if (!pk_grid_sync(P, sh, barriers * gridDim.x)) break;
      } else {
        pk_sync();
      }
    }
  }
  if (P.trace && blockIdx.x == 0 && tid == 0) P.trace[16 * P.nstages] = gtimer();
  if (*reinterpret_cast<volatile int*>(&sh->abort) && tid == 0) atomicCAS(P.err, 0, 6);
}

}  // namespace kib
