// decode_persistent.cuh -- one launch per decode token (T = 1).
//
// The bs1 decode step of the hybrid decoder after the token embedding (24
// layers of GDN or attention blocks with their FFNs, the fused LM-head argmax)
// runs as a single persistent grid: one CTA per SM, eight consumer warps and one
// producer warp.  The step is a host-built list of stages (PkStage).  The
// producer warp walks the same list independently and streams everything the
// consumers will read from HBM -- weight row tiles, the GDN state rows, the
// cached K/V rows -- into a ring of shared-memory slots with cp.async.bulk, so
// the weight stream runs ahead of the arithmetic instead of restarting after
// every kernel boundary.  Weights are constant, so the producer starts them
// before griddepcontrol.wait (overlapping the previous token's tail);
// everything written by the previous step is read only after it.
//
// Stages do not meet at grid barriers.  Every activation one CTA hands to
// another inside the step is a *cell*: 8 bytes holding the fp32 value and a
// 32-bit tag (step epoch << 8 | writing stage + 1), written with one 64-bit
// store.  A reader loads the cells it needs and re-loads them until every tag
// is the expected one.  The value and its tag travel in one single-copy-atomic
// access, so no fence is needed on either side, a stage starts as soon as the
// rows it reads exist (a GDN head waits only for its own q/k/v rows), and the
// barrier's fence + ticket + poll round trips disappear from the critical path.
// Every stage writes its own cell array, so no cell is rewritten within a step;
// the epoch advances once per step (by the LM head's last CTA).
//
// Code size is a first-order cost here: every stage runs a different part of
// the kernel once, so instructions come from the instruction cache only if the
// whole step's code fits in it (on B200 a working set above ~64 KB runs at
// several cycles per instruction, fetched from L2).  The kernel therefore keeps
// one copy of each routine: one GEMV for both K-quant types, the slow paths
// (cell polls, transcendental helpers) out of line, and little unrolling
// outside the dot-product core.
//
// Stage kinds and the reference ops they carry (the same fused groups as the
// per-kernel path in kquant_gemv2.cuh / layer_kernels.cuh):
//   kPkGemv / kPkHead  K-quant matvec with a prologue (input, RMSNorm or per-head
//                      norm-gate) and per-segment epilogues (store, residual
//                      add, conv+silu, silu*up, argmax) -- q*_k_matvec,
//                      mps_backend.mm:295-463; rms_norm 1891-1921; ssm_conv
//                      2376-2457; argmax 2681-2779
//   kPkGdn             split_qkv_l2_norm + gate/beta prepare + delta-rule
//                      update of 16 state rows (mps_backend.mm:2097-2153,
//                      2588-2605, 2307-2374)
//   kPkAttn            q/k norm + MRoPE, KV write at pos, split-K attention
//                      over the F16 cache (1991-2024, 2482-2527, 2943-3008)
//   kPkMerge           combine of the splits + sigmoid(gate)
//                      (qwen35_runtime.cpp:3347-3351)
//
// Every wait is bounded: a cell poll or mbarrier wait that runs out raises the
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
// warpgroup then gives back down to kPkProducerRegs and the consumers take
// kPkConsumerRegs: 256 x 232 + 128 x 40 = 64512, the launch total.
constexpr int kPkThreads = kPkConsumers + 128;
constexpr int kPkConsumerRegs = 232;
constexpr int kPkProducerRegs = (kPkThreads * 168 - kPkConsumers * kPkConsumerRegs) / 128;
static_assert(kPkProducerRegs >= 24 && kPkProducerRegs % 8 == 0, "register split");
constexpr int kPkSlots = 6;
constexpr int kPkSlotBytes = 32 * 1024;
constexpr int kPkMaxCols = 4096;
constexpr int kPkMaxSegs = 4;
constexpr int kPkMaxSplits = 128;
constexpr int kPkGdnRows = 16;       // state rows per GDN item
constexpr int kPkMaxTileRows = 256;  // rows of a GEMV tile
constexpr int kPkRows = 2;           // rows a lane dots per pass (independent chains, half the passes)
constexpr int kPkMaxStages = 254;    // stage tags are 1..254 in the low byte
constexpr int kPkRopePairs = 128;    // rotary pairs with a precomputed frequency
constexpr uint32_t kPkPollLimit = 1u << 21;
// Poll limit the kernel uses (kPkPollLimit unless a test lowers it through
// kib_qwen35_debug_stall to make a wait run out on purpose).
__device__ uint32_t g_pk_poll_limit = kPkPollLimit;

enum PkKind : int { kPkGemv = 0, kPkGdn = 1, kPkAttn = 2, kPkMerge = 3, kPkHead = 4 };

// ------------------------------------------------------------------ cells
// A cell is {fp32 value, 32-bit tag} in one aligned 64-bit word.
KIB_DEV void cell_st(uint64_t* p, float v, uint32_t tag) {
  const uint64_t c = (static_cast<uint64_t>(tag) << 32) | __float_as_uint(v);
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(c) : "memory");
}
KIB_DEV ulonglong2 cell_ld2(const uint64_t* p) {
  ulonglong2 r;
  asm volatile("ld.relaxed.gpu.global.v2.u64 {%0, %1}, [%2];" : "=l"(r.x), "=l"(r.y) : "l"(p) : "memory");
  return r;
}
KIB_DEV uint64_t cell_ld1(const uint64_t* p) {
  uint64_t r;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(r) : "l"(p) : "memory");
  return r;
}
KIB_DEV bool cell_ok(uint64_t c, uint32_t tag) { return static_cast<uint32_t>(c >> 32) == tag; }
KIB_DEV float cell_val(uint64_t c) { return __uint_as_float(static_cast<uint32_t>(c)); }

// Asynchronous global -> shared copies (no register destination, so an
// out-of-line call made while they are in flight does not wait for them).
KIB_DEV void cp_async_ca4(void* sdst, const void* gsrc) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(sdst)), "l"(gsrc) : "memory");
}
KIB_DEV void cp_async_ca16(void* sdst, const void* gsrc) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 16;" ::"r"(smem_u32(sdst)), "l"(gsrc) : "memory");
}
// L2 only: for data other CTAs rewrite every step (cells)
KIB_DEV void cp_async_cg16(void* sdst, const void* gsrc) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(sdst)), "l"(gsrc) : "memory");
}
KIB_DEV void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
KIB_DEV void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// Tensor copy (no multicast) of the box at (x, y, 0) of a rank-3 map (the
// instruction's dimension must be the map's rank) into shared memory.
KIB_DEV void pk_tma_kv(void* dst, const void* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(0), "r"(smem_u32(bar))
      : "memory");
}

// Out-of-line poll of one cell: re-loads until it carries `tag`.  Returns the
// cell, or 0 (tag 0 is never a stage tag) when the poll limit runs out or
// another CTA raised the error flag.
__device__ __noinline__ uint64_t pk_poll1(const uint64_t* p, uint32_t tag, const int* err) {
  const uint32_t limit = *reinterpret_cast<const volatile uint32_t*>(&g_pk_poll_limit);
  #pragma unroll 1
  for (uint32_t i = 0; i < limit; ++i) {
    const uint64_t c = cell_ld1(p);
    if (cell_ok(c, tag)) return c;
    if ((i & 255u) == 255u && *reinterpret_cast<const volatile int*>(err) != 0) break;
  }
  return 0;
}
// Loads one cell and waits for it; ok becomes false on a failed wait.
KIB_DEV float pk_cell(const uint64_t* p, uint32_t tag, const int* err, bool& ok) {
  uint64_t c = cell_ld1(p);
  if (!cell_ok(c, tag)) {
    c = pk_poll1(p, tag, err);
    ok = ok && cell_ok(c, tag);
  }
  return cell_val(c);
}

// Waits for a cell whose first load is already in `c` (loads are issued in a
// batch first, then checked: one round trip for the batch instead of one each).
KIB_DEV float pk_cell_chk(const uint64_t* p, uint64_t c, uint32_t tag, const int* err, bool& ok) {
  if (!cell_ok(c, tag)) {
    c = pk_poll1(p, tag, err);
    ok = ok && cell_ok(c, tag);
  }
  return cell_val(c);
}

// Out-of-line copies of the transcendental helpers: each exists once in the kernel.
__device__ __noinline__ float pk_expf(float v) { return expf(v); }
__device__ __noinline__ float pk_silu(float v) { return v / (1.0f + expf(-v)); }
__device__ __noinline__ float pk_sigmoid(float v) { return 1.0f / (1.0f + expf(-v)); }

struct PkSeg {
  const uint8_t* w;   // this segment's rows (row_bytes each)
  const uint8_t* w2;  // gate/up pair: the up matrix (same rows)
  uint64_t* out;      // cells, indexed by the row within the segment
  int row_begin;      // first stage row of the segment
  int rows;
  int epi;            // GemvEpilogue
  int pad;
};

// Input tags: 0 = plain floats written before this launch (the embedding
// row), else the low byte of the writing stage's tag.
struct __align__(16) PkStage {
  int kind;
  int tag;            // low byte of the tags this stage writes (index + 1)
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
  int in_tag;
  int gate_tag;
  int resid_tag;
  int src_tag;        // GDN / attention / merge: the stage that wrote their inputs
  int src2_tag;       // merge: the q|gate projection; GDN: the beta/alpha rows (0: src_tag)
  int pad0;
  PkSeg seg[kPkMaxSegs];
  const void* in;      // cells (in_tag) or floats
  const float* norm_w;
  const uint64_t* gate;  // cells
  const void* resid;   // kEpiResidual: resid[row], cells (resid_tag) or floats
  float* conv_state;   // kEpiConv: [rows][3]
  const float* conv_w; // kEpiConv: [rows][4]
  // ---- GDN (one token)
  const uint64_t* conv_out;  // cells: q | k | v after conv + silu
  const uint64_t* beta_raw;  // cells
  const uint64_t* alpha_raw; // cells
  const float* dt_bias;
  const float* ssm_a;
  float* state;       // [Hv][128][128]
  uint64_t* gdn_out;  // cells [Hv*128]
  int C;
  int key_heads;
  int value_heads;
  int pad1;
  // ---- attention (one token)
  const uint64_t* qg;  // cells [heads][2*256] q | gate
  const uint64_t* kp;  // cells
  const uint64_t* vp;  // cells
  const float* q_norm;
  const float* k_norm;
  const float* rope_freq;  // [n_dims/2] 1/theta^(2p/n_dims), computed on the host
  uint16_t* kcache;   // [cap][kv_heads*256]
  uint16_t* vcache;
  uint64_t* part;     // cells [nsplit][heads][256 + 2]
  uint64_t* att_out;  // cells [heads*256]
  int heads;
  int kv_heads;
  float theta;
  int n_dims;
  int nsplit;         // splits per kv head (kv_heads * nsplit <= grid)
  int pad2;
  const void* tk;     // rank-3 CUtensorMaps (device memory) over kcache / vcache: [1][cap][kv_heads*256],
  const void* tv;     // boxes of 256 columns (one KV head) x 32 positions x 1
};

struct PkProgram {
  const PkStage* stages;
  int nstages;
  int* pos;           // position of the token being decoded; advanced by the head
  int* token;         // in: the token; out: the argmax
  int* token_log;     // token_log[*step] = argmax, then ++*step
  int* step;
  unsigned* head_ctr; // LM-head last-CTA ticket
  unsigned* epoch;    // tag epoch, advanced once per step by the head's last CTA
  float* cand_max;    // [grid]
  int* cand_idx;
  int* err;
  unsigned long long* trace;  // optional: CTA 0's [stage][start, input ready, first tile, end, ...]
};

struct PkShared {
  uint64_t full[kPkSlots];
  uint64_t empty[kPkSlots];
  PkStage desc[2];
  float red[kPkWarps][4 * kPkRows];
  float gb[2];
  float best[kPkWarps];
  int bidx[kPkWarps];
  int abort;
  int last;
  __align__(16) float xs[kPkMaxCols + kPkMaxCols / 16];  // padded stage input; attention/GDN scratch
  __align__(16) uint64_t epi[kPkConsumers][4];  // GEMV: a row owner's epilogue inputs (cp.async)
  float ws[kPkMaxSplits];
  float ls[kPkMaxSplits];
};

constexpr size_t kPkSmemBytes = static_cast<size_t>(kPkSlots) * kPkSlotBytes + sizeof(PkShared);
static_assert(kPkSmemBytes <= 227 * 1024, "persistent kernel shared memory above the per-CTA limit");

// named barrier over the eight consumer warps (the producer never joins)
KIB_DEV void pk_sync() { asm volatile("bar.sync 1, %0;" ::"n"(kPkConsumers) : "memory"); }

// Records a failed wait: the first error code wins, the CTA leaves the step.
__device__ __noinline__ void pk_fail(PkShared* sh, int* err, int code) {
  atomicCAS(err, 0, code);
  *reinterpret_cast<volatile int*>(&sh->abort) = 1;
}

KIB_DEV void pk_mark(unsigned long long* tr, int i) {
  if (tr) tr[i] = gtimer();
}

// Key range of attention split `split` for nkeys keys (shared by producer and
// consumers).
KIB_DEV void pk_split_range(int nkeys, int nsplit, int split, int& kb, int& ke) {
  int chunk = (nkeys + nsplit - 1) / nsplit;
  chunk = (chunk + 7) & ~7;
  kb = split * chunk;
  ke = min(kb + chunk, nkeys);
}

// ------------------------------------------------------------------ producer
// The producer warp's ring position; the empty barriers count one arrival per
// consumer warp.
struct PkProducer {
  uint8_t* ring;
  PkShared* sh;
  uint32_t seq = 0;
  bool waited = false;
  int lane;
  int* err;
  uint64_t pol;
  int nslots = kPkSlots;  // ring slots in use (timing experiments may use fewer)
  int slot = 0;
  uint32_t phase = 0;

  KIB_DEV void advance() {
    __syncwarp();
    ++seq;
    if (++slot == nslots) {
      slot = 0;
      phase ^= 1u;
    }
  }
  // Waits for the current slot to be free (bounded) and arms it for `bytes`;
  // returns its address or null.
  KIB_DEV uint8_t* acquire(uint32_t bytes) {
    int ok = 1;
    if (lane == 0) {
      ok = 0;
      #pragma unroll 1
      for (uint32_t i = 0; i < (1u << 22); ++i) {
        if (mbar_try_wait(&sh->empty[slot], phase ^ 1u)) {
          ok = 1;
          break;
        }
        if ((i & 255u) == 255u && *reinterpret_cast<volatile int*>(&sh->abort)) break;
        __nanosleep(200);  // the ring is full: leave the issue slots to the consumer warps
      }
      if (!ok) {
        if (!*reinterpret_cast<volatile int*>(&sh->abort)) atomicCAS(err, 0, 4);
        *reinterpret_cast<volatile int*>(&sh->abort) = 1;
      } else {
        mbar_arrive_expect_tx(&sh->full[slot], bytes);
      }
    }
    ok = __shfl_sync(0xffffffffu, ok, 0);
    return ok ? ring + static_cast<size_t>(slot) * kPkSlotBytes : nullptr;
  }
  KIB_DEV uint64_t* bar() { return &sh->full[slot]; }
  KIB_DEV void dep_wait() {
    if (!waited) {
      pdl_wait();
      waited = true;
    }
  }
};

__device__ __noinline__ void pk_produce(const PkProgram& P, PkProducer& pr) {
  const int lane = pr.lane;
  const int grid = static_cast<int>(gridDim.x), cta = static_cast<int>(blockIdx.x);
  int pos = -1;
  #pragma unroll 1
  for (int s = 0; s < P.nstages; ++s) {
    const PkStage& S = P.stages[s];
    const int kind = S.kind;
    unsigned long long* tr = (P.trace && cta == 0 && lane == 0) ? P.trace + 16 * s : nullptr;
    pk_mark(tr, 6);  // producer reached the stage
    if (kind == kPkGemv || kind == kPkHead) {
      const int tile_rows = S.tile_rows, rows = S.rows, row_bytes = S.row_bytes, paired = S.paired;
      #pragma unroll 1
      for (int t = cta; t < S.ntiles; t += grid) {
        const int r0 = t * tile_rows;
        const int nr = min(tile_rows, rows - r0);
        const uint32_t b = static_cast<uint32_t>(nr) * static_cast<uint32_t>(row_bytes);
        uint8_t* dst = pr.acquire(paired ? 2u * b : b);
        if (!dst) return;
        if (lane < S.nseg) {
          const PkSeg& g = S.seg[lane];
          const int a = max(r0, g.row_begin), e = min(r0 + nr, g.row_begin + g.rows);
          if (a < e) {
            const size_t src = static_cast<size_t>(a - g.row_begin) * row_bytes;
            const uint32_t bytes = static_cast<uint32_t>(e - a) * static_cast<uint32_t>(row_bytes);
            uint8_t* d = dst + static_cast<size_t>(a - r0) * row_bytes;
            bulk_g2s_stream(d, g.w + src, bytes, pr.bar(), pr.pol);
            if (paired) bulk_g2s_stream(d + kPkSlotBytes / 2, g.w2 + src, bytes, pr.bar(), pr.pol);
          }
        }
        pr.advance();
      }
    } else if (kind == kPkGdn) {
      const int items = S.value_heads * (128 / kPkGdnRows);
      #pragma unroll 1
      for (int it = cta; it < items; it += grid) {
        pr.dep_wait();  // the state was written by the previous step
        constexpr uint32_t bytes = kPkGdnRows * 128 * sizeof(float);
        uint8_t* dst = pr.acquire(bytes);
        if (!dst) return;
        if (lane == 0) bulk_g2s(dst, S.state + static_cast<size_t>(it) * kPkGdnRows * 128, bytes, pr.bar());
        pr.advance();
      }
    } else if (kind == kPkAttn) {
      if (cta >= S.kv_heads * S.nsplit) continue;
      pr.dep_wait();
      if (pos < 0) pos = *P.pos;
      const int kvh = cta / S.nsplit, split = cta % S.nsplit;
      int kb, ke;
      pk_split_range(pos + 1, S.nsplit, split, kb, ke);
      const int old_end = min(ke, pos);
      // one tensor copy per 32-key chunk for K and one for V (per-key bulk
      // copies of 512 B are issue-bound); rows past the split are not read
      #pragma unroll 1
      for (int k0 = kb; k0 < old_end; k0 += kAttnChunk) {
        uint8_t* dst = pr.acquire(static_cast<uint32_t>(kAttnChunk) * 2u * kHd * 2u);
        if (!dst) return;
        if (lane == 0) {
          pk_tma_kv(dst, S.tk, kvh * kHd, k0, pr.bar());
          pk_tma_kv(dst + static_cast<size_t>(kAttnChunk) * kHd * 2, S.tv, kvh * kHd, k0, pr.bar());
        }
        pr.advance();
      }
    }
  }
}

// ------------------------------------------------------------------ consumers
struct PkCons {
  uint8_t* ring;
  PkShared* sh;
  uint32_t tagbase = 0;  // epoch << 8
  int* err;
  unsigned long long* tr = nullptr;  // trace of the current stage (CTA 0, thread 0) or null
  int nslots = kPkSlots;
  int slot = 0;
  uint32_t phase = 0;

  KIB_DEV uint32_t tag(int low) const { return tagbase | static_cast<uint32_t>(low); }
  KIB_DEV void advance() {
    if (++slot == nslots) {
      slot = 0;
      phase ^= 1u;
    }
  }
  // Waits for the next ring slot (every consumer thread); null on abort.
  KIB_DEV const uint8_t* take() {
    if (!mbar_wait_bounded(&sh->full[slot], phase, nullptr)) {
      pk_fail(sh, err, 2);
      return nullptr;
    }
    return ring + static_cast<size_t>(slot) * kPkSlotBytes;
  }
  // The slot after the current one (taken before the current one is released).
  KIB_DEV const uint8_t* take_next() {
    const int s1 = slot + 1 == nslots ? 0 : slot + 1;
    const uint32_t p1 = slot + 1 == nslots ? phase ^ 1u : phase;
    if (!mbar_wait_bounded(&sh->full[s1], p1, nullptr)) {
      pk_fail(sh, err, 2);
      return nullptr;
    }
    return ring + static_cast<size_t>(s1) * kPkSlotBytes;
  }
  // Every consumer thread is done with the slot (CTA barrier, then one arrival
  // per warp).
  KIB_DEV void release() {
    pk_sync();
    if ((threadIdx.x & 31) == 0) mbar_arrive(&sh->empty[slot]);
    advance();
  }
  // This warp is done with the slot.
  KIB_DEV void release_warp() {
    __syncwarp();
    if ((threadIdx.x & 31) == 0) mbar_arrive(&sh->empty[slot]);
    advance();
  }
  KIB_DEV bool aborted() const { return *reinterpret_cast<volatile int*>(&sh->abort) != 0; }
};

// ---- GEMV prologue: the stage's transformed input vector into sh->xs
// The stage input lives in shared memory with 4 floats of padding after every
// 64: the 16 lanes of a row group read their units (64 consecutive inputs for
// Q4_K) at a stride of 68 floats, which spreads them over the banks.
KIB_DEV int xpad(int i) { return i + 4 * (i >> 6); }

// Norm-gate prologue: qk_norm over heads of 128 (one warp per head), silu(gate),
// mul (qwen35_runtime.cpp:2993-3003).
__device__ __noinline__ void pk_prologue_norm_gate(const PkStage& S, PkCons& cs) {
  float* xs = cs.sh->xs;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int cols = S.cols;
  const uint32_t it = cs.tag(S.in_tag), gt = cs.tag(S.gate_tag);
  constexpr int hd = 128;
  const float4 w = *reinterpret_cast<const float4*>(S.norm_w + 4 * lane);
  const float eps = S.eps;
  bool ok = true;
  #pragma unroll 1
  for (int base = warp * hd; base < cols; base += kPkWarps * hd) {
    // the eight cells of this lane are loaded together (one round trip)
    const uint64_t* yc = reinterpret_cast<const uint64_t*>(S.in) + base + 4 * lane;
    const uint64_t* zc = S.gate + base + 4 * lane;
    ulonglong2 ya = cell_ld2(yc), yb = cell_ld2(yc + 2), za = cell_ld2(zc), zb = cell_ld2(zc + 2);
    if (!(cell_ok(ya.x, it) & cell_ok(ya.y, it) & cell_ok(yb.x, it) & cell_ok(yb.y, it) & cell_ok(za.x, gt) &
          cell_ok(za.y, gt) & cell_ok(zb.x, gt) & cell_ok(zb.y, gt))) {
      bool r = true;
      ya.x = cell_ok(ya.x, it) ? ya.x : pk_poll1(yc, it, cs.err);
      ya.y = cell_ok(ya.y, it) ? ya.y : pk_poll1(yc + 1, it, cs.err);
      yb.x = cell_ok(yb.x, it) ? yb.x : pk_poll1(yc + 2, it, cs.err);
      yb.y = cell_ok(yb.y, it) ? yb.y : pk_poll1(yc + 3, it, cs.err);
      za.x = cell_ok(za.x, gt) ? za.x : pk_poll1(zc, gt, cs.err);
      za.y = cell_ok(za.y, gt) ? za.y : pk_poll1(zc + 1, gt, cs.err);
      zb.x = cell_ok(zb.x, gt) ? zb.x : pk_poll1(zc + 2, gt, cs.err);
      zb.y = cell_ok(zb.y, gt) ? zb.y : pk_poll1(zc + 3, gt, cs.err);
      r = cell_ok(ya.x, it) & cell_ok(ya.y, it) & cell_ok(yb.x, it) & cell_ok(yb.y, it) & cell_ok(za.x, gt) &
          cell_ok(za.y, gt) & cell_ok(zb.x, gt) & cell_ok(zb.y, gt);
      ok = ok && r;
    }
    const float y[4] = {cell_val(ya.x), cell_val(ya.y), cell_val(yb.x), cell_val(yb.y)};
    const float z[4] = {cell_val(za.x), cell_val(za.y), cell_val(zb.x), cell_val(zb.y)};
    const float ss = warp_sum((y[0] * y[0] + y[1] * y[1]) + (y[2] * y[2] + y[3] * y[3]));
    const float scale = 1.0f / sqrtf(ss / static_cast<float>(hd) + eps);
    float4 o;
    o.x = y[0] * (scale * w.x) * pk_silu(z[0]);
    o.y = y[1] * (scale * w.y) * pk_silu(z[1]);
    o.z = y[2] * (scale * w.z) * pk_silu(z[2]);
    o.w = y[3] * (scale * w.w) * pk_silu(z[3]);
    *reinterpret_cast<float4*>(xs + xpad(base + 4 * lane)) = o;
  }
  if (!ok) pk_fail(cs.sh, cs.err, 7);
  pk_sync();
}

// Waits for this thread's input cells (up to four groups of four at
// i = 4*tid + 1024*k) and writes their values (times the norm weights) to xs;
// returns the thread's sum of squares.  Every pass loads all of the thread's
// groups at once, so a pass costs one memory round trip; each cell is loaded
// by exactly one thread of the CTA (148 CTAs read every input line, so
// duplicate loads would turn the line into a hot spot), and a pass that finds
// a cell missing backs off briefly before the next.
__device__ __noinline__ float pk_poll_input(const uint64_t* c, uint32_t t, int cols, const float* norm_w, float* xs,
                                            const int* err, bool& ok, unsigned long long* tr) {
  constexpr int kPer = kPkMaxCols / (4 * kPkConsumers);  // float4 per thread
  const int tid = threadIdx.x;
  const int n = (cols - 4 * tid + 4 * kPkConsumers - 1) / (4 * kPkConsumers);  // groups of this thread
  float4 w[kPer];
#pragma unroll
  for (int k = 0; k < kPer; ++k) {
    const int i = 4 * tid + 4 * kPkConsumers * k;
    w[k] = make_float4(1.f, 1.f, 1.f, 1.f);
    if (norm_w && k < n) w[k] = *reinterpret_cast<const float4*>(norm_w + i);
  }
  float ss = 0.0f;
  uint32_t iter = 0;
  const uint32_t limit = *reinterpret_cast<const volatile uint32_t*>(&g_pk_poll_limit);
  #pragma unroll 1
  while (true) {
    bool ready = true;
    ss = 0.0f;
    ulonglong2 a[kPer], b[kPer];
#pragma unroll
    for (int k = 0; k < kPer; ++k) {
      const int i = 4 * tid + 4 * kPkConsumers * k;
      if (k < n) {
        a[k] = cell_ld2(c + i);
        b[k] = cell_ld2(c + i + 2);
      }
    }
#pragma unroll
    for (int k = 0; k < kPer; ++k) {
      const int i = 4 * tid + 4 * kPkConsumers * k;
      if (k < n) {
        ready = ready & cell_ok(a[k].x, t) & cell_ok(a[k].y, t) & cell_ok(b[k].x, t) & cell_ok(b[k].y, t);
        const float4 o = make_float4(cell_val(a[k].x), cell_val(a[k].y), cell_val(b[k].x), cell_val(b[k].y));
        ss += (o.x * o.x + o.y * o.y) + (o.z * o.z + o.w * o.w);
        *reinterpret_cast<float4*>(xs + xpad(i)) = make_float4(o.x * w[k].x, o.y * w[k].y, o.z * w[k].z, o.w * w[k].w);
      }
    }
    if (ready) break;
    if (++iter > limit || ((iter & 255u) == 0u && *reinterpret_cast<const volatile int*>(err) != 0)) {
      ok = false;
      break;
    }
    __nanosleep(32);
  }
  if (tr) tr[12] = iter;
  return ss;
}

// Plain / RMS prologue.  The RMS norm's scalar is not applied here: xs holds
// x * w and every thread folds 1/rms into its own unit registers, so the
// prologue needs a single CTA barrier.  Returns the scale (1
// for the other prologues); on a failed wait the CTA's abort flag is set
// (checked after the barrier).
__device__ __noinline__ float pk_prologue(const PkStage& S, PkCons& cs) {
  if (S.prologue == kProNormGate) {
    pk_prologue_norm_gate(S, cs);
    return 1.0f;
  }
  PkShared* sh = cs.sh;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int cols = S.cols;
  const bool rms = S.prologue == kProRms;
  bool ok = true;
  float ss = 0.0f;
  if (S.in_tag == 0) {
    #pragma unroll 1
    for (int i = 4 * tid; i < cols; i += 4 * kPkConsumers) {
      const float4 o = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(S.in) + i);
      const float4 w = rms ? *reinterpret_cast<const float4*>(S.norm_w + i) : make_float4(1.f, 1.f, 1.f, 1.f);
      ss += (o.x * o.x + o.y * o.y) + (o.z * o.z + o.w * o.w);
      *reinterpret_cast<float4*>(sh->xs + xpad(i)) = make_float4(o.x * w.x, o.y * w.y, o.z * w.z, o.w * w.w);
    }
  } else {
    pk_mark(cs.tr, 13);
    ss = pk_poll_input(reinterpret_cast<const uint64_t*>(S.in), cs.tag(S.in_tag), cols, rms ? S.norm_w : nullptr, sh->xs,
                       cs.err, ok, cs.tr);
  }
  pk_mark(cs.tr, 4);
  // rms_norm_f32_f32_batched (mps_backend.mm:1891-1921): x * rsqrt(mean(x^2)+eps) * w;
  // the weights are applied when the units are loaded
  ss = warp_sum(ss);
  if (lane == 0) sh->red[warp][0] = ss;
  if (!ok) pk_fail(sh, cs.err, 7);
  pk_sync();
  if (!rms) return 1.0f;
  float tot = 0.0f;
  #pragma unroll 1
  for (int q = 0; q < kPkWarps; ++q) tot += sh->red[q][0];
  return 1.0f / sqrtf(tot / static_cast<float>(cols) + S.eps);
}

// x values of one lane's unit in registers: 64 floats as 32 float2 (element
// order as unit_col) and the sums of its four quarters (16 elements each).
struct PkX {
  float2 v[32];
  float s[4];
};

// x values of unit u of block blk from the padded stage input.  Q4_K/Q5_K: quarter q = elements
// 16q..16q+15 of the 64 contiguous columns; Q6_K: quarter k = the 16-column
// run of group k.
KIB_DEV void pk_load_x(int type, const float* xs, int blk, int u, PkX& x) {
  // first column of each quarter's 16-column run
  int col0, cstep;
  if (type == kTypeQ6K) {
    col0 = 256 * blk + 128 * (u >> 1) + 16 * (u & 1);
    cstep = 32;
  } else {
    col0 = 256 * blk + 64 * u;
    cstep = 16;
  }
  #pragma unroll
  for (int q = 0; q < 4; ++q) {
    const float4* p = reinterpret_cast<const float4*>(xs + xpad(col0 + cstep * q));
    float sum = 0.0f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float4 f = p[j];
      x.v[8 * q + 2 * j] = make_float2(f.x, f.y);
      x.v[8 * q + 2 * j + 1] = make_float2(f.z, f.w);
      sum += (f.x + f.y) + (f.z + f.w);
    }
    x.s[q] = sum;
  }
}

// Codes (16 words of 4 byte-codes, element order as unit_col) and per-quarter
// affine coefficients (value = A*code + B) of unit u of one row's block.
template <int QT>
KIB_DEV void pk_decode_t(const uint8_t* blk, int u, uint32_t (&q)[16], float (&A)[4], float (&B)[4]) {
  const RawUnit<QT> raw = load_raw<QT>(blk, u);
  codes_from_raw<QT>(raw, u, q);
  if (QT == kTypeQ6K) {
    coeffs_from_raw<QT>(raw, u, A, B);
  } else {
    float a2[4], b2[4];
    coeffs_from_raw<QT>(raw, u, a2, b2);
    A[0] = A[1] = a2[0];
    A[2] = A[3] = a2[1];
    B[0] = B[1] = b2[0];
    B[2] = B[3] = b2[1];
  }
}

// Dot products of one unit of R rows with the same x: the R rows' codes are
// decoded first and their FMA chains are independent, so loads and arithmetic
// of different rows overlap.  Codes are the floats 0.5 + b/256 (one PRMT);
// sum(b*x) over a quarter is 256*acc - 128*sum(x), exact up to fp32 rounding.
template <int R, int ONLY = 0>  // ONLY: the one K-quant type this call site decodes (0: any)
KIB_DEV void pk_dot_rows(int type, const uint8_t* const (&blk)[R], int u, const PkX& x, float (&out)[R]) {
  uint32_t q[R][16];
  float A[R][4], B[R][4];
  // one type's decodes together: the code a stage runs stays contiguous
  // Q5_K (in Q4_K_M files only the GDN in-projection) runs on the two-row
  // passes alone, laid out off the hot path: the four-row passes (quad stages,
  // the LM head) carry no code for it
  if (ONLY == kTypeQ6K) {
#pragma unroll
    for (int k = 0; k < R; ++k) pk_decode_t<kTypeQ6K>(blk[k], u, q[k], A[k], B[k]);
  } else if (ONLY == kTypeQ4K) {
#pragma unroll
    for (int k = 0; k < R; ++k) pk_decode_t<kTypeQ4K>(blk[k], u, q[k], A[k], B[k]);
  } else if (R == 2 && __builtin_expect(type == kTypeQ5K, 0)) {
#pragma unroll
    for (int k = 0; k < R; ++k) pk_decode_t<kTypeQ5K>(blk[k], u, q[k], A[k], B[k]);
  } else if (type == kTypeQ6K) {
#pragma unroll
    for (int k = 0; k < R; ++k) pk_decode_t<kTypeQ6K>(blk[k], u, q[k], A[k], B[k]);
  } else {
#pragma unroll
    for (int k = 0; k < R; ++k) pk_decode_t<kTypeQ4K>(blk[k], u, q[k], A[k], B[k]);
  }
#pragma unroll
  for (int k = 0; k < R; ++k) {
    float2 acc[4][2];
#pragma unroll
    for (int g = 0; g < 4; ++g) acc[g][0] = acc[g][1] = make_float2(0.0f, 0.0f);
#pragma unroll
    for (int w = 0; w < 16; ++w) {
      const int g = w >> 2, c = w & 1;
      acc[g][c] = ffma2(code_pair_lo(q[k][w]), x.v[2 * w], acc[g][c]);
      acc[g][c] = ffma2(code_pair_hi(q[k][w]), x.v[2 * w + 1], acc[g][c]);
    }
    float r = 0.0f;
#pragma unroll
    for (int g = 0; g < 4; ++g) {
      const float a = (acc[g][0].x + acc[g][0].y) + (acc[g][1].x + acc[g][1].y);
      const float cx = fmaf(256.0f, a, -128.0f * x.s[g]);
      r = fmaf(A[k][g], cx, fmaf(B[k][g], x.s[g], r));
    }
    out[k] = r;
  }
}

// Argmax candidate (max, lowest index at ties).  The persistent path decodes
// greedily and reports only the token; p(top1) (used by the MTP loop's
// adaptive budget) comes from the per-kernel path.
struct PkArgmax {
  float best = -INFINITY;
  int bidx = 0x7FFFFFFF;
  KIB_DEV void push(float v, int row) {
    if (v > best || (v == best && row < bidx)) {
      best = v;
      bidx = row;
    }
  }
  KIB_DEV void merge(float om, int oi) {
    if (oi == 0x7FFFFFFF) return;
    if (bidx == 0x7FFFFFFF || om > best || (om == best && oi < bidx)) {
      best = om;
      bidx = oi;
    }
  }
};

// Epilogue inputs of one output row, loaded by its owner lane before the dot
// products so that their latency hides behind them.
struct PkEpi {
  int epi = kEpiStore;
  int row = 0;
  uint64_t* out = nullptr;
};

// Starts the copies of one output row's epilogue inputs into the owner
// thread's shared-memory slot: the residual cell pair (or plain float pair)
// around the row, or the conv state (3 floats) and conv weights (4 floats).
KIB_DEV void pk_epi_issue(const PkStage& S, PkShared* sh, int r, PkEpi& e) {
  int si = 0;
  if (S.nseg > 1 && r >= S.seg[1].row_begin) si = 1;
  if (S.nseg > 2 && r >= S.seg[2].row_begin) si = 2;
  if (S.nseg > 3 && r >= S.seg[3].row_begin) si = 3;
  const PkSeg& g = S.seg[si];
  e.row = r - g.row_begin;
  e.epi = g.epi;
  e.out = g.out;
  uint64_t* slot = sh->epi[threadIdx.x];
  if (e.epi == kEpiResidual) {
    if (S.resid_tag) cp_async_cg16(slot, reinterpret_cast<const uint64_t*>(S.resid) + (e.row & ~1));
    else cp_async_ca16(slot, reinterpret_cast<const float*>(S.resid) + (e.row & ~3));
  } else if (e.epi == kEpiConv) {
    const float* st = S.conv_state + static_cast<size_t>(e.row) * 3;
    float* d = reinterpret_cast<float*>(slot);
    cp_async_ca4(d, st);
    cp_async_ca4(d + 1, st + 1);
    cp_async_ca4(d + 2, st + 2);
    cp_async_ca16(d + 4, S.conv_w + static_cast<size_t>(e.row) * 4);
  }
  cp_async_commit();
}

// Epilogue of one output row (its owner lane).  Inline: an out-of-line call
// here would save and restore the caller's unit registers on every pass.
KIB_DEV void pk_epi_run(const PkStage& S, PkCons& cs, PkEpi& e, float v, float v2, PkArgmax& am) {
  cp_async_wait_all();
  const uint64_t* slot = cs.sh->epi[threadIdx.x];
  float o;
  if (e.epi == kEpiResidual) {
    float res;
    if (S.resid_tag) {
      const uint32_t rt = cs.tag(S.resid_tag);
      uint64_t c = slot[e.row & 1];
      if (!cell_ok(c, rt)) {
        c = pk_poll1(reinterpret_cast<const uint64_t*>(S.resid) + e.row, rt, cs.err);
        if (!cell_ok(c, rt)) pk_fail(cs.sh, cs.err, 8);
      }
      res = cell_val(c);
    } else {
      res = reinterpret_cast<const float*>(slot)[e.row & 3];
    }
    o = v + res;
  } else if (e.epi == kEpiSiluMul) {
    o = silu_f(v) * v2;
  } else if (e.epi == kEpiConv) {
    // causal depthwise conv of kernel 4 over [state | new], then silu
    const float* f = reinterpret_cast<const float*>(slot);
    const float4 st3 = make_float4(f[0], f[1], f[2], 0.f);
    const float4 cw = *reinterpret_cast<const float4*>(f + 4);
    float c = 0.0f;
    c += st3.x * cw.x;
    c += st3.y * cw.y;
    c += st3.z * cw.z;
    c += v * cw.w;
    o = silu_f(c);
    float* st = S.conv_state + static_cast<size_t>(e.row) * 3;
    st[0] = st3.y;
    st[1] = st3.z;
    st[2] = v;
  } else if (e.epi == kEpiArgmax) {
    am.push(v, e.row);
    return;
  } else {
    o = v;
  }
  cell_st(e.out + e.row, o, cs.tag(S.tag));
}

// Merges the argmax candidates of a warp (butterfly); every lane ends with the total.
KIB_DEV void pk_argmax_warp(PkArgmax& a) {
  #pragma unroll 1
  for (int o = 16; o > 0; o >>= 1) {
    const float om = __shfl_xor_sync(0xffffffffu, a.best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, a.bidx, o);
    a.merge(om, oi);
  }
}

// ---- LM head tail: CTA candidate, then the last CTA picks the token and
// closes the step (token log, position, epoch)
__device__ __noinline__ void pk_head_finish(const PkProgram& P, PkShared* sh, PkArgmax am, uint32_t epoch) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  pk_argmax_warp(am);
  if (lane == 0) {
    sh->best[warp] = am.best;
    sh->bidx[warp] = am.bidx;
  }
  pk_sync();
  if (tid == 0) {
    PkArgmax c;
    #pragma unroll 1
    for (int w = 0; w < kPkWarps; ++w) c.merge(sh->best[w], sh->bidx[w]);
    P.cand_max[blockIdx.x] = c.best;
    P.cand_idx[blockIdx.x] = c.bidx;
    __threadfence();
    sh->last = atomicAdd(P.head_ctr, 1u) == gridDim.x - 1;
  }
  pk_sync();
  if (!sh->last || tid >= 32) return;
  __threadfence();
  PkArgmax c;
  #pragma unroll 1
  for (unsigned i = lane; i < gridDim.x; i += 32) c.merge(__ldcg(&P.cand_max[i]), __ldcg(&P.cand_idx[i]));
  pk_argmax_warp(c);
  if (lane == 0) {
    P.token[0] = c.bidx;
    if (P.token_log) {
      const int st = *P.step;
      P.token_log[st] = c.bidx;
      *P.step = st + 1;
    }
    *P.pos = *P.pos + 1;
    *P.head_ctr = 0u;
    *P.epoch = epoch + 1u;
    __threadfence();
  }
}

// The stage's GEMV: row groups of RG lanes; each lane dots its 64-column unit
// of kPkRows rows per pass, the partial sums are reduced across the group so
// that lane (k * RG/kPkRows) ends with row k's total and runs its epilogue.
// Warps go through the tiles independently: each waits for a tile itself and
// releases it with one arrival per warp (no CTA barrier per tile).
KIB_DEV bool pk_gemv(const PkStage& S, PkCons& cs, const PkProgram& P, uint32_t epoch) {
  constexpr int R = kPkRows;
  constexpr int R_LOG2 = R == 1 ? 0 : R == 2 ? 1 : 2;
  const int tid = threadIdx.x;
  // per-stage constants, in registers
  const int rg_log2 = S.rg == 16 ? 4 : S.rg == 32 ? 5 : 6;
  const int groups = kPkConsumers >> rg_log2;
  const int group = tid >> rg_log2, gl = tid & (S.rg - 1);
  const int lim_log2 = rg_log2 < 5 ? rg_log2 : 5;
  const int lim = 1 << lim_log2;
  const int own_shift = lim_log2 - R_LOG2;
  const int k_own = (gl & (lim - 1)) >> own_shift;
  const bool owner2 = (gl & ((1 << own_shift) - 1)) == 0;  // holds a row total in its warp
  const bool owner = owner2 && gl < 32;                   // writes the row
  const int my_off = k_own * groups + group;
  const int per_pass = groups * R;
  const bool active = gl < (S.cols >> 6);
  const int blk = gl >> 2, u = gl & 3;
  const int type = S.type;
  const int blk_off = blk * kquant_block_bytes(type);
  const int rows = S.rows, tile_rows = S.tile_rows, ntiles = S.ntiles, row_bytes = S.row_bytes;
  const bool paired = S.paired != 0;
  const bool two_warps = rg_log2 > 5;
  const int grid = static_cast<int>(gridDim.x);
  const int cta = static_cast<int>(blockIdx.x);
  PkArgmax am;  // LM head: this thread's rows
  // quad mode: a stage whose single tile per CTA holds 33..64 rows of 1024
  // columns runs as one pass of four rows per lane (the LM head's dot code)
  // instead of two passes of two
  const int nr0 = min(tile_rows, rows - cta * tile_rows);
  // (Q4_K only: the four-row code carries one type's decode)
  const bool quad = S.kind == kPkGemv && type == kTypeQ4K && rg_log2 == 4 && !paired && ntiles <= grid &&
                    nr0 > groups * R && nr0 <= 4 * groups;
  const bool q_owner = (gl & 3) == 0;
  const int q_off = ((gl & 15) >> 2) * groups + group;
  // the first pass's epilogue inputs go out before the prologue's wait
  PkEpi e;
  if (quad) {
    if (q_owner && q_off < nr0) pk_epi_issue(S, cs.sh, cta * tile_rows + q_off, e);
  } else if (owner && my_off < nr0) {
    pk_epi_issue(S, cs.sh, cta * tile_rows + my_off, e);
  }
  const float scale = pk_prologue(S, cs);
  pk_mark(cs.tr, 1);
  if (cs.aborted()) return false;
  PkX ux;  // unscaled: the RMS scale multiplies each row's result instead
  if (active) pk_load_x(type, cs.sh->xs, blk, u, ux);
  if (cs.tr) {
    unsigned long long tt;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(tt) : "f"(ux.v[31].y), "f"(ux.s[3]));
    cs.tr[9] = tt;
  }
  if (quad) {
    const uint8_t* tile = cs.take();
    if (!tile) return false;
    pk_mark(cs.tr, 2);
    const uint8_t* b[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) b[k] = tile + static_cast<size_t>(min(k * groups + group, nr0 - 1)) * row_bytes + blk_off;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    if (active) pk_dot_rows<4, kTypeQ4K>(type, b, u, ux, acc);
    // lanes 0-3 / 4-7 / 8-11 / 12-15 of the group end with rows 0..3
    const bool h1 = gl & 8, h2 = gl & 4;
    const float a0 = (h1 ? acc[2] : acc[0]) + __shfl_xor_sync(0xffffffffu, h1 ? acc[0] : acc[2], 8);
    const float a1 = (h1 ? acc[3] : acc[1]) + __shfl_xor_sync(0xffffffffu, h1 ? acc[1] : acc[3], 8);
    float v = (h2 ? a1 : a0) + __shfl_xor_sync(0xffffffffu, h2 ? a0 : a1, 4);
    v += __shfl_xor_sync(0xffffffffu, v, 2);
    v += __shfl_xor_sync(0xffffffffu, v, 1);
    if (q_owner && q_off < nr0) pk_epi_run(S, cs, e, v * scale, 0.0f, am);
    cs.release_warp();
    return true;
  }
  if (S.kind == kPkHead && type == kTypeQ6K && rg_log2 == 4 && tile_rows == groups * R) {
    // LM head: two tiles per pass (a lane dots rows of both), so each pass has
    // twice the independent work between its waits
    PkArgmax am2;
    const int own2 = (gl & 15) >> 2;  // 0,1: tile A rows group, group+16; 2,3: tile B
    #pragma unroll 1
    for (int t = cta; t < ntiles; t += 2 * grid) {
      const bool two = t + grid < ntiles;
      unsigned long long* ttr = nullptr;  // per-pass times of CTA 0, thread 0 (trace only)
      if (cs.tr && (t - cta) / (2 * grid) < 500) ttr = cs.tr - 16 * (P.nstages - 1) + 8192 + 4 * ((t - cta) / (2 * grid));
      pk_mark(ttr, 0);
      const uint8_t* ta = cs.take();
      if (!ta) return false;
      const uint8_t* tb = two ? cs.take_next() : ta;
      if (!tb) return false;
      pk_mark(ttr, 1);
      const int na = min(tile_rows, rows - t * tile_rows);
      const int nb = two ? min(tile_rows, rows - (t + grid) * tile_rows) : 0;
      const uint8_t* b[4];
      b[0] = ta + static_cast<size_t>(min(group, na - 1)) * row_bytes + blk_off;
      b[1] = ta + static_cast<size_t>(min(group + groups, na - 1)) * row_bytes + blk_off;
      b[2] = tb + static_cast<size_t>(min(group, max(nb, 1) - 1)) * row_bytes + blk_off;
      b[3] = tb + static_cast<size_t>(min(group + groups, max(nb, 1) - 1)) * row_bytes + blk_off;
      float acc[4] = {0.f, 0.f, 0.f, 0.f};
      if (active) pk_dot_rows<4, kTypeQ6K>(type, b, u, ux, acc);
      // lanes 0-3 / 4-7 / 8-11 / 12-15 of the group end with rows 0..3
      const bool h1 = gl & 8, h2 = gl & 4;
      const float a0 = (h1 ? acc[2] : acc[0]) + __shfl_xor_sync(0xffffffffu, h1 ? acc[0] : acc[2], 8);
      const float a1 = (h1 ? acc[3] : acc[1]) + __shfl_xor_sync(0xffffffffu, h1 ? acc[1] : acc[3], 8);
      float v = (h2 ? a1 : a0) + __shfl_xor_sync(0xffffffffu, h2 ? a0 : a1, 4);
      v += __shfl_xor_sync(0xffffffffu, v, 2);
      v += __shfl_xor_sync(0xffffffffu, v, 1);
      if ((gl & 3) == 0) {
        const int tt = own2 < 2 ? t : t + grid;
        const int rl = group + (own2 & 1) * groups;
        if (rl < (own2 < 2 ? na : nb)) am2.push(v * scale, tt * tile_rows + rl);
      }
      pk_mark(ttr, 2);
      cs.release_warp();
      if (two) cs.release_warp();
      pk_mark(ttr, 3);
    }
    pk_head_finish(P, cs.sh, am2, epoch);
    return true;
  }
  bool first = true;
  #pragma unroll 1
  for (int t = cta; t < ntiles; t += grid) {
    const int r0 = t * tile_rows;
    const int nr = min(tile_rows, rows - r0);
    unsigned long long* ttr = nullptr;  // LM head: per-tile times of CTA 0, thread 0 (trace only)
    if (cs.tr && S.kind == kPkHead && (t - cta) / grid < 500) ttr = cs.tr - 16 * (P.nstages - 1) + 8192 + 4 * ((t - cta) / grid);
    pk_mark(ttr, 0);
    const uint8_t* tile = cs.take();
    if (!tile) return false;
    pk_mark(ttr, 1);
    if (first) pk_mark(cs.tr, 2);
    #pragma unroll 1
    for (int p0 = 0; p0 < nr; p0 += per_pass) {
      const int rl = p0 + my_off;
      if (!first && owner && rl < nr) pk_epi_issue(S, cs.sh, r0 + rl, e);
      first = false;
      float acc[R], acc2[R];
      const uint8_t* b[R];
#pragma unroll
      for (int k = 0; k < R; ++k) {
        const int rk = min(p0 + k * groups + group, nr - 1);  // clamped: never past the tile
        b[k] = tile + static_cast<size_t>(rk) * row_bytes + blk_off;
        acc[k] = acc2[k] = 0.0f;
      }
      if (active) {
        // a gate/up pair runs both halves through one copy of the dot code
        #pragma unroll 1
        for (int h = 0; h <= static_cast<int>(paired); ++h) {
          float d[R];
          pk_dot_rows<R>(type, b, u, ux, d);
#pragma unroll
          for (int k = 0; k < R; ++k) {
            if (h == 0) acc[k] = d[k];
            else acc2[k] = d[k];
            b[k] += kPkSlotBytes / 2;
          }
        }
      }
      // transposed reduction: each halving exchange keeps half of the rows on
      // each side (lane bit lim/2 keeps rows {R/2..R-1}, ...); then a plain
      // butterfly over the remaining lane bits
      float v, v2;
      if (R == 4) {
        const bool h1 = gl & (lim >> 1), h2 = gl & (lim >> 2);
        const float a0 = (h1 ? acc[2] : acc[0]) + __shfl_xor_sync(0xffffffffu, h1 ? acc[0] : acc[2], lim >> 1);
        const float a1 = (h1 ? acc[3] : acc[1]) + __shfl_xor_sync(0xffffffffu, h1 ? acc[1] : acc[3], lim >> 1);
        const float c0 = (h1 ? acc2[2] : acc2[0]) + __shfl_xor_sync(0xffffffffu, h1 ? acc2[0] : acc2[2], lim >> 1);
        const float c1 = (h1 ? acc2[3] : acc2[1]) + __shfl_xor_sync(0xffffffffu, h1 ? acc2[1] : acc2[3], lim >> 1);
        v = (h2 ? a1 : a0) + __shfl_xor_sync(0xffffffffu, h2 ? a0 : a1, lim >> 2);
        v2 = (h2 ? c1 : c0) + __shfl_xor_sync(0xffffffffu, h2 ? c0 : c1, lim >> 2);
      } else if (R == 2) {
        const bool hi = gl & (lim >> 1);
        v = (hi ? acc[1] : acc[0]) + __shfl_xor_sync(0xffffffffu, hi ? acc[0] : acc[1], lim >> 1);
        v2 = (hi ? acc2[1] : acc2[0]) + __shfl_xor_sync(0xffffffffu, hi ? acc2[0] : acc2[1], lim >> 1);
      } else {
        v = acc[0];
        v2 = acc2[0];
      }
      #pragma unroll 1
      for (int o = lim >> (1 + R_LOG2); o > 0; o >>= 1) {
        v += __shfl_xor_sync(0xffffffffu, v, o);
        v2 += __shfl_xor_sync(0xffffffffu, v2, o);
      }
      if (two_warps) {
        // two warps per row group: the second warp's totals through shared
        // memory, under a barrier of the pair only
        const int wp = (tid >> 5) & ~1;
        if (owner2 && gl >= 32) {
          cs.sh->red[wp + 1][2 * k_own] = v;
          cs.sh->red[wp + 1][2 * k_own + 1] = v2;
        }
        asm volatile("bar.sync %0, 64;" ::"r"(2 + (wp >> 1)) : "memory");
        if (owner) {
          v += cs.sh->red[wp + 1][2 * k_own];
          v2 += cs.sh->red[wp + 1][2 * k_own + 1];
        }
        asm volatile("bar.sync %0, 64;" ::"r"(2 + (wp >> 1)) : "memory");
      }
      if (owner && rl < nr) pk_epi_run(S, cs, e, v * scale, v2 * scale, am);
    }
    pk_mark(ttr, 2);
    cs.release_warp();
    pk_mark(ttr, 3);
  }
  if (S.kind == kPkHead) pk_head_finish(P, cs.sh, am, epoch);
  return true;
}

// ---- GDN: items of (value head, 16 state rows); warp w updates rows 2w, 2w+1
__device__ __noinline__ bool pk_gdn(const PkStage& S, PkCons& cs) {
  constexpr int D = 128;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  float* qn = cs.sh->xs;
  float* kn = cs.sh->xs + D;
  float* vv = cs.sh->xs + 2 * D;
  const int items = S.value_heads * (D / kPkGdnRows);
  const int key_dim = S.key_heads * D;
  const float scale = 1.0f / sqrtf(static_cast<float>(D));
  const uint32_t in_tag = cs.tag(S.src_tag), otag = cs.tag(S.tag);
  const uint32_t ba_tag = S.src2_tag ? cs.tag(S.src2_tag) : in_tag;
  #pragma unroll 1
  for (int it = static_cast<int>(blockIdx.x); it < items; it += static_cast<int>(gridDim.x)) {
    const int h = it / (D / kPkGdnRows), grp = it % (D / kPkGdnRows);
    const int kh = h % S.key_heads;
    bool ok = true;
    float qv = 0.0f, kv = 0.0f;
    if (tid < D) {
      // this head's q and k rows (and nothing else) must exist
      const uint64_t* qp = S.conv_out + kh * D + tid;
      const uint64_t* kp = S.conv_out + key_dim + kh * D + tid;
      const uint64_t qc = cell_ld1(qp), kc = cell_ld1(kp);
      qv = pk_cell_chk(qp, qc, in_tag, cs.err, ok);
      kv = pk_cell_chk(kp, kc, in_tag, cs.err, ok);
      const float q2 = warp_sum(qv * qv), k2 = warp_sum(kv * kv);
      if (lane == 0) {
        cs.sh->red[warp][0] = q2;
        cs.sh->red[warp][1] = k2;
      }
    } else if (tid < D + kPkGdnRows) {
      const int r = tid - D;
      vv[r] = pk_cell(S.conv_out + 2 * key_dim + h * D + grp * kPkGdnRows + r, in_tag, cs.err, ok);
    } else if (tid == D + kPkGdnRows) {
      const uint64_t ac = cell_ld1(S.alpha_raw + h), bc = cell_ld1(S.beta_raw + h);
      const float a = pk_cell_chk(S.alpha_raw + h, ac, ba_tag, cs.err, ok);
      const float b = pk_cell_chk(S.beta_raw + h, bc, ba_tag, cs.err, ok);
      cs.sh->gb[0] = softplus20_f(a + S.dt_bias[h]) * S.ssm_a[h];
      cs.sh->gb[1] = pk_sigmoid(b);
    }
    if (!ok) pk_fail(cs.sh, cs.err, 9);
    pk_sync();
    if (cs.aborted()) return false;
    if (tid < D) {
      float qsum = 0.0f, ksum = 0.0f;
      #pragma unroll 1
      for (int w = 0; w < D / 32; ++w) {
        qsum += cs.sh->red[w][0];
        ksum += cs.sh->red[w][1];
      }
      qn[tid] = qv * (1.0f / fmaxf(sqrtf(qsum), S.eps));
      kn[tid] = kv * (1.0f / fmaxf(sqrtf(ksum), S.eps));
    }
    const float ge = pk_expf(cs.sh->gb[0]);
    const float beta = cs.sh->gb[1];
    const uint8_t* tile = cs.take();
    if (!tile) return false;
    pk_sync();  // qn/kn
    const float4 k4 = *reinterpret_cast<const float4*>(kn + 4 * lane);
    const float4 q4 = *reinterpret_cast<const float4*>(qn + 4 * lane);
    const float* srows = reinterpret_cast<const float*>(tile);
    #pragma unroll 1
    for (int rr = 0; rr < 2; ++rr) {
      const int lr = 2 * warp + rr;
      const int vrow = grp * kPkGdnRows + lr;
      float4 st = *reinterpret_cast<const float4*>(srows + lr * D + 4 * lane);
      st.x *= ge;
      st.y *= ge;
      st.z *= ge;
      st.w *= ge;
      const float sk = warp_sum(st.x * k4.x + st.y * k4.y + st.z * k4.z + st.w * k4.w);
      const float delta = (vv[lr] - sk) * beta;
      st.x += k4.x * delta;
      st.y += k4.y * delta;
      st.z += k4.z * delta;
      st.w += k4.w * delta;
      const float y = warp_sum(st.x * q4.x + st.y * q4.y + st.z * q4.z + st.w * q4.w);
      if (lane == 0) cell_st(S.gdn_out + h * D + vrow, y * scale, otag);
      *reinterpret_cast<float4*>(S.state + (static_cast<size_t>(h) * D + vrow) * D + 4 * lane) = st;
    }
    cs.release();  // also orders qn/kn/vv reuse
  }
  return true;
}

KIB_DEV void pk_warp_sum8(float (&v)[8], int lane) { warp_sum8(v, lane); }

// qk_norm (mps_backend.mm:1991-2024) then mrope (2482-2527) of one 256-wide
// head vector staged in shared memory; text positions (all MRoPE streams
// equal), frequencies from the host's table; one warp.  Lane l owns elements
// l + 32i; its norm weights and rotary frequency are loaded in one batch.
__device__ __noinline__ void pk_norm_rope(float* v, const float* in, const float* w, const float* freq, float eps,
                                          int n_dims, int position, int lane) {
  constexpr int E = kHd / 32;
  float x[E], wv[E];
  const int half = n_dims / 2;
  const float fr = lane < half ? freq[lane] : 0.0f;  // n_dims/2 <= 32 pairs handled per lane below
#pragma unroll
  for (int i = 0; i < E; ++i) {
    wv[i] = w[lane + 32 * i];
    x[i] = in[lane + 32 * i];
  }
  float ss = 0.0f;
#pragma unroll
  for (int i = 0; i < E; ++i) ss += x[i] * x[i];
  ss = warp_sum(ss);
  const float scale = 1.0f / sqrtf(ss / static_cast<float>(kHd) + eps);
#pragma unroll
  for (int i = 0; i < E; ++i) v[lane + 32 * i] = x[i] * (scale * wv[i]);
  __syncwarp();
  #pragma unroll 1
  for (int pi = lane; pi < half; pi += 32) {
    const float angle = static_cast<float>(position) * (pi == lane ? fr : freq[pi]);
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
__device__ __noinline__ bool pk_attn(const PkStage& S, PkCons& cs, int pos) {
  constexpr int G = 4;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int cta = static_cast<int>(blockIdx.x);
  if (cta >= S.kv_heads * S.nsplit) return true;
  float* qs = cs.sh->xs;               // [4][256]
  float* newk = qs + G * kHd;          // [256]
  float* newv = newk + kHd;            // [256]
  float* merge = newv + kHd;           // [8][258]; first the raw q (4 x 256) and k (256)
  float* qraw = merge;
  const int kvh = cta / S.nsplit, split = cta % S.nsplit;
  const int kvd = S.kv_heads * kHd;
  int kb, ke;
  pk_split_range(pos + 1, S.nsplit, split, kb, ke);
  const int old_end = min(ke, pos);
  const bool owner = pos >= kb && pos < ke;
  const uint32_t in_tag = cs.tag(S.src_tag), otag = cs.tag(S.tag);
  {
    // stage the group's q rows (and, for the owner of the new key, k and v):
    // a thread's (up to three) cell pairs are loaded together, then checked
    bool ok = true;
    const int n = owner ? G * kHd + 2 * kHd : G * kHd;
    const uint64_t* src[3];
    ulonglong2 c[3];
#pragma unroll
    for (int j = 0; j < 3; ++j) {
      const int i = min(2 * tid + 2 * kPkConsumers * j, n - 2);
      if (i < G * kHd) {
        src[j] = S.qg + static_cast<size_t>(kvh * G + i / kHd) * 2 * kHd + i % kHd;
      } else if (i < G * kHd + kHd) {
        src[j] = S.kp + kvh * kHd + (i - G * kHd);
      } else {
        src[j] = S.vp + kvh * kHd + (i - G * kHd - kHd);
      }
      if (2 * tid + 2 * kPkConsumers * j < n) c[j] = cell_ld2(src[j]);
    }
#pragma unroll
    for (int j = 0; j < 3; ++j) {
      const int i = 2 * tid + 2 * kPkConsumers * j;
      if (i < n) {
        const float a = pk_cell_chk(src[j], c[j].x, in_tag, cs.err, ok);
        const float b = pk_cell_chk(src[j] + 1, c[j].y, in_tag, cs.err, ok);
        float* dst = i < G * kHd + kHd ? qraw + i : newv + (i - G * kHd - kHd);
        dst[0] = a;
        dst[1] = b;
      }
    }
    if (!ok) pk_fail(cs.sh, cs.err, 10);
    pk_sync();
    if (cs.aborted()) return false;
  }
  pk_mark(cs.tr, 4);
  if (warp < G) {
    pk_norm_rope(qs + warp * kHd, qraw + warp * kHd, S.q_norm, S.rope_freq, S.eps, S.n_dims, pos, lane);
  } else if (warp == G && owner) {
    pk_norm_rope(newk, qraw + G * kHd, S.k_norm, S.rope_freq, S.eps, S.n_dims, pos, lane);
    #pragma unroll 1
    for (int i = lane; i < kHd; i += 32) {
      const __half kh = __float2half_rn(newk[i]);
      const __half vh = __float2half_rn(newv[i]);
      S.kcache[static_cast<size_t>(pos) * kvd + kvh * kHd + i] = __half_as_ushort(kh);
      S.vcache[static_cast<size_t>(pos) * kvd + kvh * kHd + i] = __half_as_ushort(vh);
      newk[i] = __half2float(kh);
      newv[i] = __half2float(vh);
    }
  }
  pk_sync();
  pk_mark(cs.tr, 9);
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
    const uint16_t* kvbuf = reinterpret_cast<const uint16_t*>(tile);  // [K: 32 keys x 256][V: 32 keys x 256]
    const int nk = min(kAttnChunk, old_end - k0);
    #pragma unroll 1
    for (int kk0 = kh2 * KB; kk0 < nk; kk0 += 2 * KB) {
      float sc[KB];
#pragma unroll
      for (int e = 0; e < KB; ++e) {
        const int kk = min(kk0 + e, nk - 1);
        const uint4 kr = *reinterpret_cast<const uint4*>(kvbuf + static_cast<size_t>(kk) * kHd + 8 * lane);
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
      float mx = m;
#pragma unroll
      for (int e = 0; e < KB; ++e) {
        sc[e] *= scale;
        if (kk0 + e < nk) mx = fmaxf(mx, sc[e]);
      }
      const float ps = expf(m - mx);
      l *= ps;
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] *= ps;
      // the block's V rows are loaded together; keys past the chunk get weight 0
      uint4 vr[KB];
#pragma unroll
      for (int e = 0; e < KB; ++e)
        vr[e] = *reinterpret_cast<const uint4*>(kvbuf + static_cast<size_t>(kAttnChunk + min(kk0 + e, nk - 1)) * kHd +
                                                8 * lane);
#pragma unroll
      for (int e = 0; e < KB; ++e) {
        const float w = kk0 + e < nk ? expf(sc[e] - mx) : 0.0f;
        l += w;
        const __half2* vh = reinterpret_cast<const __half2*>(&vr[e]);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 b2 = __half22float2(vh[i]);
          acc[2 * i] = fmaf(w, b2.x, acc[2 * i]);
          acc[2 * i + 1] = fmaf(w, b2.y, acc[2 * i + 1]);
        }
      }
      m = mx;
    }
    cs.release_warp();
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
  pk_mark(cs.tr, 10);
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
    uint64_t* dst = S.part + (static_cast<size_t>(split) * S.heads + kvh * G + jj) * (kHd + 2);
    cell_st(dst + i, a[i] * ea + b[i] * eb, otag);
    if (i == 0) {
      cell_st(dst + kHd, M, otag);
      cell_st(dst + kHd + 1, a[kHd + 1] * ea + b[kHd + 1] * eb, otag);
    }
  }
  pk_sync();
  return true;
}

// ---- merge: item = (head, 16 output dims); thread = (dim, split lane)
__device__ __noinline__ bool pk_merge(const PkStage& S, PkCons& cs) {
  PkShared* sh = cs.sh;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int items = S.heads * (kHd / 16);
  const int ns = S.nsplit;
  const uint32_t ptag = cs.tag(S.src_tag), gtag = cs.tag(S.src2_tag), otag = cs.tag(S.tag);
  #pragma unroll 1
  for (int it = static_cast<int>(blockIdx.x); it < items; it += static_cast<int>(gridDim.x)) {
    const int h = it / (kHd / 16), d0 = (it % (kHd / 16)) * 16;
    bool ok = true;
    #pragma unroll 1
    for (int s = tid; s < ns; s += kPkConsumers) {
      const uint64_t* src = S.part + (static_cast<size_t>(s) * S.heads + h) * (kHd + 2) + kHd;
      const ulonglong2 c = cell_ld2(src);  // m, l (kHd is even: a 16-byte pair)
      sh->ws[s] = pk_cell_chk(src, c.x, ptag, cs.err, ok);
      sh->ls[s] = pk_cell_chk(src + 1, c.y, ptag, cs.err, ok);
    }
    // the value cells this thread will need, loaded while the weights are formed
    const int d = tid & 15, jl = tid >> 4;  // 16 split lanes
    constexpr int kMaxPer = (kPkMaxSplits + kPkConsumers / 16 - 1) / (kPkConsumers / 16);
    uint64_t vc[kMaxPer];
#pragma unroll
    for (int j = 0; j < kMaxPer; ++j) {
      const int s = jl + j * (kPkConsumers / 16);
      if (s < ns) vc[j] = cell_ld1(S.part + (static_cast<size_t>(s) * S.heads + h) * (kHd + 2) + d0 + d);
    }
    uint64_t gcell = 0;
    if (tid < 16) gcell = cell_ld1(S.qg + static_cast<size_t>(h) * 2 * kHd + kHd + d0 + tid);
    if (!ok) pk_fail(sh, cs.err, 11);
    pk_sync();
    if (cs.aborted()) return false;
    if (warp == 0) {
      float M = -INFINITY;
      #pragma unroll 1
      for (int s = lane; s < ns; s += 32) M = fmaxf(M, sh->ws[s]);
      M = warp_max(M);
      float den = 0.0f;
      #pragma unroll 1
      for (int s = lane; s < ns; s += 32) {
        const float ms = sh->ws[s];
        const float e = ms == -INFINITY ? 0.0f : pk_expf(ms - M);
        sh->ws[s] = e;
        den += sh->ls[s] * e;
      }
      den = warp_sum(den);
      if (lane == 0) sh->gb[0] = den;
    }
    pk_sync();
    float n = 0.0f;
#pragma unroll
    for (int j = 0; j < kMaxPer; ++j) {
      // each value is waited for on its own tag (a split's threads write
      // values, m and l independently)
      const int s = jl + j * (kPkConsumers / 16);
      if (s < ns) {
        const uint64_t* src = S.part + (static_cast<size_t>(s) * S.heads + h) * (kHd + 2) + d0 + d;
        n = fmaf(pk_cell_chk(src, vc[j], ptag, cs.err, ok), sh->ws[s], n);
      }
    }
    n += __shfl_xor_sync(0xffffffffu, n, 16);
    float* part = sh->xs;                     // [8 warps][16]
    if (lane < 16) part[warp * 16 + d] = n;
    float g = 0.0f;
    if (tid < 16) g = pk_cell_chk(S.qg + static_cast<size_t>(h) * 2 * kHd + kHd + d0 + tid, gcell, gtag, cs.err, ok);
    if (!ok) pk_fail(sh, cs.err, 11);
    pk_sync();
    if (cs.aborted()) return false;
    if (tid < 16) {
      float tot = 0.0f;
      #pragma unroll 1
      for (int w = 0; w < kPkWarps; ++w) tot += part[w * 16 + tid];
      const float den = sh->gb[0];
      const float inv = den == 0.0f ? 0.0f : 1.0f / den;
      cell_st(S.att_out + h * kHd + d0 + tid, tot * inv * pk_sigmoid(g), otag);
    }
    pk_sync();
  }
  return true;
}

__global__ void __launch_bounds__(kPkThreads, 1) decode_persistent_kernel(const __grid_constant__ PkProgram P) {
  extern __shared__ __align__(1024) uint8_t pk_smem[];
  uint8_t* ring = pk_smem;
  PkShared* sh = reinterpret_cast<PkShared*>(pk_smem + static_cast<size_t>(kPkSlots) * kPkSlotBytes);
  const int tid = threadIdx.x, warp = tid >> 5;
  if (tid == 0) {
    for (int i = 0; i < kPkSlots; ++i) {
      mbar_init(&sh->full[i], 1);
      mbar_init(&sh->empty[i], kPkWarps);
    }
    sh->abort = 0;
    fence_mbar_init();
  }
  __syncthreads();
  constexpr int nslots = kPkSlots;
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
    pr.nslots = nslots;
    pk_produce(P, pr);
    // leave only once the copies in flight have landed (bounded)
    if (pr.lane == 0) {
      const uint32_t n = min(pr.seq, static_cast<uint32_t>(nslots));
      #pragma unroll 1
      for (uint32_t q = pr.seq - n; q < pr.seq; ++q) {
        const int sl = static_cast<int>(q % static_cast<uint32_t>(nslots));
        const uint32_t ph = (q / static_cast<uint32_t>(nslots)) & 1u;
        #pragma unroll 1
        for (uint32_t i = 0; i < (1u << 22); ++i)
          if (mbar_try_wait(&sh->full[sl], ph)) break;
      }
    }
    return;
  }
  // ---------------------------------------------------------------- consumers
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kPkConsumerRegs));
  pdl_wait();
  pdl_launch_dependents();
  const int pos = *P.pos;
  const uint32_t epoch = *reinterpret_cast<volatile unsigned*>(P.epoch);
  PkCons cs;
  cs.ring = ring;
  cs.sh = sh;
  cs.err = P.err;
  cs.tagbase = epoch << 8;
  cs.nslots = nslots;
  constexpr int kDescWords = static_cast<int>(sizeof(PkStage) / 16);
  static_assert(sizeof(PkStage) % 16 == 0, "PkStage must be a multiple of 16 bytes");
  static_assert(kDescWords <= kPkConsumers, "one descriptor word per consumer thread");
  if (tid < kDescWords) reinterpret_cast<uint4*>(&sh->desc[0])[tid] = __ldg(reinterpret_cast<const uint4*>(P.stages) + tid);
  pk_sync();
  #pragma unroll 1
  for (int s = 0; s < P.nstages; ++s) {
    const PkStage& S = sh->desc[s & 1];
    // the next stage's descriptor goes into the other buffer asynchronously
    // (that buffer's stage ended at the last barrier)
    if (tid < kDescWords && s + 1 < P.nstages) {
      cp_async_cg16(reinterpret_cast<uint4*>(&sh->desc[(s + 1) & 1]) + tid, reinterpret_cast<const uint4*>(&P.stages[s + 1]) + tid);
      cp_async_commit();
    }
    cs.tr = (P.trace && blockIdx.x == 0 && tid == 0) ? P.trace + 16 * s : nullptr;
    pk_mark(cs.tr, 0);
    const int kind = S.kind;
    bool ok = true;
    if (kind == kPkGemv || kind == kPkHead) {
      // CTAs without a tile of this stage skip its input entirely.  One
      // K-quant type per stage (Q4_K, Q5_K or Q6_K): the host splits a
      // projection group of mixed types into one stage per type.
      // (the LM head's finish runs inside pk_gemv; a CTA without a head tile
      // still takes part in the last-CTA ticket)
      if (static_cast<int>(blockIdx.x) < S.ntiles) ok = pk_gemv(S, cs, P, epoch);
      else if (kind == kPkHead) pk_head_finish(P, sh, PkArgmax(), epoch);
    } else if (kind == kPkGdn) {
      ok = pk_gdn(S, cs);
    } else if (kind == kPkAttn) {
      ok = pk_attn(S, cs, pos);
    } else {
      ok = pk_merge(S, cs);
    }
    if (!ok) break;
    if (s + 1 < P.nstages) {
      cp_async_wait_all();
      pk_sync();
    }
    if (cs.tr) {
      pk_mark(cs.tr, 3);
      // slowest CTA done (no return value: a reduction, not a round trip)
      asm volatile("red.relaxed.gpu.global.max.u64 [%0], %1;" ::"l"(P.trace + 16 * s + 5), "l"(gtimer()) : "memory");
    }
  }
  if (P.trace && blockIdx.x == 0 && tid == 0) P.trace[16 * P.nstages] = gtimer();
  if (*reinterpret_cast<volatile int*>(&sh->abort) && tid == 0) atomicCAS(P.err, 0, 6);
}

}  // namespace kib
