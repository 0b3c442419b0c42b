// kib_common.cuh -- device helpers shared by every kernel of the B200 backend.
//
// sm_100a only: programmatic dependent launch (griddepcontrol), the bulk-copy
// engine (cp.async.bulk with an mbarrier transaction count, no multicast), and
// packed fp32x2 arithmetic.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#define KIB_DEV __device__ __forceinline__

namespace kib {

constexpr int kTypeF32 = 0;
constexpr int kTypeQ4K = 12;
constexpr int kTypeQ5K = 13;
constexpr int kTypeQ6K = 14;

__host__ __device__ constexpr int kquant_block_bytes(int type) {
  return type == kTypeQ4K ? 144 : (type == kTypeQ5K ? 176 : (type == kTypeQ6K ? 210 : 0));
}

// ---------------------------------------------------------------------- PDL
// Every kernel launched on the decode chain waits for its predecessor with
// pdl_wait() before touching any activation, and only prefetches read-only
// weights before that point; pdl_launch_dependents() lets the next kernel's
// CTAs start their own weight prefetch while this one finishes.
KIB_DEV void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
KIB_DEV void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" :::); }

// ---------------------------------------------------------- mbarrier + bulk
KIB_DEV uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

KIB_DEV void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

KIB_DEV void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }

KIB_DEV void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

KIB_DEV void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

KIB_DEV bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait: gives up after `limit` polls (each try_wait itself suspends
// for a hardware-defined interval) and raises *err instead of hanging the GPU.
KIB_DEV bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, int* err) {
  for (uint32_t i = 0; i < (1u << 22); ++i) {
    if (mbar_try_wait(bar, parity)) return true;
  }
  if (err) atomicExch(err, 2);
  return false;
}

// Global -> shared bulk copy (TMA engine, 1-D, no multicast).  dst, src and
// bytes must be multiples of 16.
KIB_DEV void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Same copy for data streamed exactly once per step (weights): the lines are
// marked evict-first in L2, so the stream does not push out what the step
// re-reads (activations, KV cache, recurrent state).
KIB_DEV uint64_t l2_evict_first_policy() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}
KIB_DEV void bulk_g2s_stream(void* dst, const void* src, uint32_t bytes, uint64_t* bar, uint64_t pol) {
  asm volatile(
      "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(pol)
      : "memory");
}

KIB_DEV void prefetch_l2(const void* p) { asm volatile("prefetch.global.L2 [%0];" ::"l"(p)); }

// ------------------------------------------------------------------ trace
// Per-launch timeline of one kernel (KIB_TRACE): slot[0] = ~first CTA entry,
// slot[1] = last CTA past griddepcontrol.wait, slot[2] = last CTA exit,
// slot[3] = ~first CTA past the wait (times from %globaltimer, ns; the
// complemented fields turn atomicMax into a minimum).
KIB_DEV unsigned long long gtimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
KIB_DEV void trace_entry(unsigned long long* s) {
  if (s && threadIdx.x == 0) {
    const unsigned long long t = gtimer();
    atomicMax(&s[0], ~t);
    atomicMax(&s[4], t);  // last CTA entry
  }
}
// slot[5]: last CTA whose first staged tile has landed; slot[6]: last CTA
// done with its compute (before the epilogue's final stores).
KIB_DEV void trace_mark(unsigned long long* s, int field) {
  if (s && threadIdx.x == 0) atomicMax(&s[field], gtimer());
}
KIB_DEV void trace_wait(unsigned long long* s) {
  if (s && threadIdx.x == 0) {
    const unsigned long long t = gtimer();
    atomicMax(&s[1], t);
    atomicMax(&s[3], ~t);
  }
}
KIB_DEV void trace_exit(unsigned long long* s) {
  if (s && threadIdx.x == 0) atomicMax(&s[2], gtimer());
}

// ------------------------------------------------------------- reductions
KIB_DEV float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

KIB_DEV float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// ------------------------------------------------------------ conversions
KIB_DEV float half_bits_to_float(uint16_t h) { return __half2float(__ushort_as_half(h)); }
KIB_DEV float round_to_half(float f) { return __half2float(__float2half_rn(f)); }

// Byte b (0..127) of a 32-bit word placed in bits 16..23 of 0x3F00xxxx gives
// the float 0.5 + b/256 exactly; a dot product over such values recovers
// sum(b * x) = 256 * acc - 128 * sum(x) with one PRMT and one FMA per weight.
KIB_DEV float byte_as_half_plus(uint32_t word, uint32_t sel) {
  return __uint_as_float(__byte_perm(word, 0x3F000000u, sel));
}
// selectors that move byte k of `word` to position 2, 0x00 to positions 0,1
// and 0x3F to position 3 (byte_perm indexes {word bytes 0-3, const bytes 4-7}).
constexpr uint32_t kSelByte0 = 0x7044u;
constexpr uint32_t kSelByte1 = 0x7144u;
constexpr uint32_t kSelByte2 = 0x7244u;
constexpr uint32_t kSelByte3 = 0x7344u;

KIB_DEV float2 ffma2(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }

}  // namespace kib

#define KIB_CUDA_CHECK(expr)                                   \
  do {                                                         \
    cudaError_t kib_err_ = (expr);                             \
    if (kib_err_ != cudaSuccess) return kib::cuda_status(kib_err_, #expr, __FILE__, __LINE__); \
  } while (0)
