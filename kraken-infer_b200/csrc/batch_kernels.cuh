// batch_kernels.cuh -- the per-sequence pieces of a batched decode step.
//
// A batched step decodes one token for each of `slots` independent sequences
// (the reference reserves `sequence_slots` in its plan,
// include/toyllm/runtime/qwen35_runtime.hpp:20, qwen35_runtime.cpp:4478-4479).
// Everything token-parallel (norms, projections, FFN, LM head) runs as one
// M = slots GEMM over the batch; what couples a token to its own sequence --
// the causal conv window, the delta-rule state, the KV cache and its position
// -- runs per slot: the conv below, gdn_core_kernel and attn_decode_kernel in
// their batched modes (blockIdx.z = slot).
#pragma once

#include "kib_common.cuh"

namespace kib {

// Causal depthwise conv of one new token per slot (ssm_conv_f32 over
// [state | x], then silu, mps_backend.mm:2376-2400, 2610-2618) and the state
// shift; state is [slots][C][K-1] (this layer's rows of each slot found
// state_slot_stride floats apart), x and out are [slots][ld].
template <int K>
__global__ void __launch_bounds__(256) conv_batched_kernel(float* state, size_t state_slot_stride, const float* x,
                                                           int x_ld, const float* w, int C, float* out, int out_ld) {
  pdl_wait();
  pdl_launch_dependents();
  const int c = blockIdx.x * 256 + threadIdx.x, slot = blockIdx.y;
  if (c >= C) return;
  float* st = state + slot * state_slot_stride + static_cast<size_t>(c) * (K - 1);
  float win[K], wc[K];
#pragma unroll
  for (int j = 0; j < K; ++j) wc[j] = w[static_cast<size_t>(c) * K + j];
#pragma unroll
  for (int j = 0; j < K - 1; ++j) win[j] = st[j];
  win[K - 1] = x[static_cast<size_t>(slot) * x_ld + c];
  float s = 0.0f;
#pragma unroll
  for (int j = 0; j < K; ++j) s += win[j] * wc[j];
  out[static_cast<size_t>(slot) * out_ld + c] = silu_k(s);
#pragma unroll
  for (int j = 0; j < K - 1; ++j) st[j] = win[j + 1];
}

// Greedy token per slot from its logits row (argmax_f32_i32,
// mps_backend.mm:2681-2720: the largest value, ties to the lowest index); the
// token becomes the slot's next input, is logged at log[step][slot], and the
// slot's position advances.
__global__ void __launch_bounds__(256) batch_argmax_kernel(const float* logits, int V, int* token, int* pos,
                                                           int* log, int* step, int slots) {
  pdl_wait();
  pdl_launch_dependents();
  __shared__ float bv[8];
  __shared__ int bi[8];
  const int slot = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const float* row = logits + static_cast<size_t>(slot) * V;
  float best = -INFINITY;
  int idx = 0x7FFFFFFF;
  for (int i = tid; i < V; i += 256) {
    const float v = row[i];
    if (v > best) {  // increasing i: the first of equal values stays
      best = v;
      idx = i;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
    if (ov > best || (ov == best && oi < idx)) {
      best = ov;
      idx = oi;
    }
  }
  if (lane == 0) {
    bv[warp] = best;
    bi[warp] = idx;
  }
  __syncthreads();
  if (tid == 0) {
    for (int w = 1; w < 8; ++w)
      if (bv[w] > best || (bv[w] == best && bi[w] < idx)) {
        best = bv[w];
        idx = bi[w];
      }
    token[slot] = idx;
    log[static_cast<size_t>(*step) * slots + slot] = idx;
    pos[slot] += 1;
  }
}

// Advances the batched step counter once every slot's argmax has been logged.
__global__ void batch_step_kernel(int* step) {
  pdl_wait();
  pdl_launch_dependents();
  if (threadIdx.x == 0) *step += 1;
}

}  // namespace kib
