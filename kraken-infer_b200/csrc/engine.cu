// engine.cu -- the Qwen3.5 runtime on the B200 kernels: GGUF load + weight map +
// execution plan, chunked prefill, graph-replayed greedy decode and the MTP
// draft -> verify -> greedy-accept loop.
//
// Mirrors the reference's runtime (src/runtime/qwen35_runtime.cpp):
//   build_qwen35_execution_plan      4380-4526
//   allocate_qwen35_metal_cache      1252-1389
//   upload_qwen35_metal_weights      1426-1528  (raw GGUF bytes, as stored)
//   run_qwen35_linear_layer_chunk    2634-3144
//   run_qwen35_full_attention_layer_chunk 3146-3423
//   run_qwen35_decode_tokens         3860-3936
//   run_qwen35_mtp_tokens(_from_id_buffer) 4111-4240
//   generate_qwen35_metal            5239-6714 (prefill 5717-6046, MTP loop 6457-6600,
//                                    greedy loop 6601-6632, adaptive budget 6421-6455)
// Per decode step the whole forward is one CUDA graph: 5 kernels per layer
// chained with programmatic dependent launch, the sampled token and the
// position stay on the device.
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <functional>
#include <map>
#include <memory>
#include <string>
#include <vector>

#include "gguf.hpp"
#include "prefix_cache.hpp"
#include "kib_ctx.cuh"
#include "layer_kernels.cuh"
#include "decode_persistent.cuh"
#include "gdn_chunk.cuh"
#include "batch_kernels.cuh"

namespace kib {
cudaError_t gemm_f16_launch(int type, const void* w, int rows, int cols, const float* x, int x_ld, int T, float* y,
                            int y_ld, const float* resid, cudaStream_t st);
cudaError_t gemm_f16w_launch(int type, const void* w, const __half* w16_resident, int rows, int cols, const float* x,
                             int x_ld, int T, float* y, int y_ld, const float* resid, __half* w16, __half* x16,
                             bool convert_x, int num_sms, cudaStream_t st, int* err);
cudaError_t kquant_to_f16_launch(int type, const void* w, int rows, int cols, __half* out, int num_sms,
                                 cudaStream_t st);
cudaError_t kq_skinny_launch(int type, const void* w, int rows, int cols, const __half* x16, int T, float* y,
                             int y_ld, const float* resid, float* ws, int num_sms, cudaStream_t st, bool xsplit);
cudaError_t get_rows_launch(int type, const void* w, int nrows, int cols, const int* ids, int T, float* out,
                            int out_ld, cudaStream_t st);
// out16: also the rows rounded to half (the prefill GEMMs' input), or null
cudaError_t rms_rows_launch(const float* in, const float* w, int T, int n, float eps, float* out, cudaStream_t st,
                            __half* out16 = nullptr);
cudaError_t norm_gate_launch(float* v, const float* w, const float* gate, int T, int heads, int d, float eps,
                             float* out, cudaStream_t st, __half* out16 = nullptr, int gate_ld = 0);
cudaError_t silu_mul_cat_launch(const float* gu, int T, int I, float* act, cudaStream_t st, __half* out16);
cudaError_t conv_launch(float* state, const float* in, int in_ld, const float* w, int K, int C, int T, float* out,
                        int out_ld, int silu, cudaStream_t st);
cudaError_t silu_mul_launch(float* g, const float* u, size_t n, cudaStream_t st, __half* out16 = nullptr);
}  // namespace kib

using namespace kib;

namespace {

constexpr int kMaxSmallT = 8;
constexpr int64_t kQwenEndOfText = 151643;  // qwen_tokenizer.hpp:44

struct DevT {
  uint8_t* p = nullptr;
  __half* h = nullptr;  // K-quant matrices used by prefill GEMMs: resident f16 copy (or nullptr)
  int type = -1;
  std::vector<uint64_t> shape;
  int cols() const { return shape.empty() ? 0 : static_cast<int>(shape[0]); }
  int rows() const { return shape.size() < 2 ? 1 : static_cast<int>(shape[1]); }
  const float* f() const { return reinterpret_cast<const float*>(p); }
  bool ok() const { return p != nullptr; }
};

struct LayerW {
  int kind = 0;  // 0 linear attention, 1 full attention, 2 MTP (full attention block)
  int cache_index = 0;
  DevT attn_norm, post_norm, ffn_gate, ffn_up, ffn_down;
  DevT qkv, zgate, conv1d, dt_bias, ssm_a, beta, alpha, ssm_norm, ssm_out;
  DevT q, k, v, o, q_norm, k_norm;
  DevT eh_proj, enorm, hnorm, shead_norm;
};

}  // namespace

struct kib_qwen35 {
  kib_ctx* ctx = nullptr;
  std::unique_ptr<GgufFile> gguf;
  kib_qwen35_plan plan{};
  // hparams
  int H = 0, I = 0, V = 0, heads = 0, kvh = 0, hd = 0, lkh = 0, lvh = 0, lhd = 0, convk = 0, C = 0, VD = 0;
  int KD = 0, AD = 0;
  float eps = 1e-6f, theta = 1e7f;
  int sections[4] = {11, 11, 10, 0};
  int64_t eos = -1;
  int cap = 0, chunk = 1024, tmax = 1024;
  int nsplit = 64;
  // weights
  uint8_t* d_weights = nullptr;
  uint64_t weight_bytes = 0;
  DevT tok_embd, output_norm, output;
  std::vector<LayerW> layers;
  bool has_mtp = false;
  LayerW mtp;
  // caches
  uint16_t *d_k = nullptr, *d_v = nullptr, *d_mk = nullptr, *d_mv = nullptr;
  float *d_r = nullptr, *d_s = nullptr, *d_r_snap = nullptr, *d_s_snap = nullptr, *d_pending_h = nullptr;
  size_t k_elems = 0, r_elems = 0, s_elems = 0, mk_elems = 0;
  // activations
  float *d_h = nullptr, *d_h1 = nullptr, *d_qkv = nullptr, *d_z = nullptr, *d_beta = nullptr, *d_alpha = nullptr;
  float *d_y = nullptr, *d_act = nullptr, *d_act2 = nullptr, *d_qg = nullptr, *d_kp = nullptr, *d_vp = nullptr;
  float *d_att = nullptr, *d_qout = nullptr, *d_norm = nullptr, *d_norm2 = nullptr, *d_hn = nullptr;
  float *d_logits = nullptr, *d_e = nullptr, *d_cat = nullptr, *d_hm = nullptr, *d_hm1 = nullptr, *d_mtp_h = nullptr;
  float *d_part = nullptr;
  float* d_fa_part = nullptr;
  float* d_proj = nullptr;  // prefill: outputs of one GEMM over concatenated weights [T][sum of rows]  // prefill attention key splits: [split][T][heads][256 + 2]
  __half *d_w16 = nullptr, *d_x16 = nullptr;  // prefill GEMM scratch: one f16 weight matrix, one f16 x
  void* d_w16_all = nullptr;                  // resident f16 prefill weights (DevT::h points inside)
  float* d_gdn_ws = nullptr;                  // chunked delta rule: Tb, P, Kt, G per (value head, 64-token chunk)
  unsigned* d_attn_cnt = nullptr;
  float *d_cand_max = nullptr, *d_cand_sum = nullptr;
  int* d_cand_idx = nullptr;
  unsigned* d_head_cnt = nullptr;
  // d_pos, d_step and d_tokens live in one block d_io (pos at 0, step at 1,
  // tokens from 4), so a decode step's host inputs reach it in one copy
  int* d_io = nullptr;
  int *d_pos = nullptr, *d_mtp_pos = nullptr, *d_tokens = nullptr, *d_argmax = nullptr, *d_log = nullptr,
      *d_step = nullptr, *d_mtp_tok = nullptr;
  float* d_prob = nullptr;
  // host mirrors
  int* h_pin = nullptr;  // pinned scratch (tokens / argmax)
  float* h_pinf = nullptr;
  uint64_t pos = 0;
  // graphs
  cudaGraphExec_t fwd_graph[kMaxSmallT + 1] = {};
  bool fwd_graph_logits[kMaxSmallT + 1] = {};
  cudaGraphExec_t decode_graph = nullptr;
  cudaGraphExec_t mtp_graph = nullptr;
  std::string err;
  // KIB_TRACE=1: per-launch timeline of the decode graph (see trace_* in kib_common.cuh)
  bool trace_on = false;
  unsigned long long* d_trace = nullptr;
  int trace_used = 0;
  std::vector<std::string> trace_names;
  // persistent decode (one launch per token; KIB_PERSISTENT=0 turns it off)
  bool pk_on = false;
  std::string pk_why;
  PkStage* d_pk = nullptr;
  std::vector<PkStage> pk_host;  // host copy of the stage list (kib_qwen35_debug_stall restores from it)
  int pk_n = 0;
  int pk_grid = 0;
  unsigned* d_pk_ctr = nullptr;  // [1] LM-head ticket, [2] cell tag epoch
  uint64_t* d_pk_cells = nullptr;
  float* d_pk_rope = nullptr;  // [kPkRopePairs] rotary inverse frequencies
  CUtensorMap* d_pk_tmaps = nullptr;  // per attention layer: K and V cache tensor maps of the persistent kernel
  float* d_pk_cmax = nullptr;
  int* d_pk_cidx = nullptr;
  unsigned long long* d_pk_trace = nullptr;
  bool pk_coop = true;
  cudaGraphExec_t pk_graph = nullptr;
  cudaGraphExec_t pk_fwd_graph = nullptr;  // one-token forward: step inputs in, embedding, persistent kernel, token + error flag out
};

namespace {

int fail(kib_qwen35* m, int code, const std::string& msg) {
  m->err = msg;
  if (m->ctx) m->ctx->last_error = msg;
  return code;
}

#define ENG_CUDA(expr)                                                                   \
  do {                                                                                   \
    cudaError_t e_ = (expr);                                                             \
    if (e_ != cudaSuccess) return fail(m, KIB_ERR_INTERNAL, std::string(#expr) + ": " + cudaGetErrorString(e_)); \
  } while (0)

template <typename T>
cudaError_t dalloc(T** p, size_t elems) {
  return cudaMalloc(reinterpret_cast<void**>(p), std::max<size_t>(elems, 1) * sizeof(T) + 256);
}

// -------------------------------------------------------------- enqueue ops
struct Enq {
  kib_qwen35* m;
  cudaStream_t st;
  std::string why;
  cudaError_t e = cudaSuccess;
  bool ok() const { return e == cudaSuccess; }
  bool tracing = false;
  unsigned long long* slot(const char* name) {
    if (!tracing || !m->d_trace || m->trace_used >= 4096) return nullptr;
    m->trace_names.push_back(name);
    return m->d_trace + 8 * (m->trace_used++);
  }
  void run(cudaError_t r, const char* what) {
    if (e == cudaSuccess && r != cudaSuccess) {
      e = r;
      if (why.empty()) why = what;
    }
  }
};

GemvDesc base_desc(kib_qwen35* m, int type, int cols, int T) {
  GemvDesc d;
  d.type = type;
  d.cols = cols;
  d.ntok = T;
  d.eps = m->eps;
  d.err = m->ctx->d_err;
  return d;
}

void add_seg(GemvDesc& d, const DevT& w, float* out, int ld, int epi, const DevT* w2 = nullptr) {
  GemvSegDesc& s = d.seg[d.nseg++];
  s.w = w.p;
  s.w2 = w2 ? w2->p : nullptr;
  s.out = out;
  s.rows = w.rows();
  s.ld = ld;
  s.epilogue = epi;
}

// Launches one GEMV over several matrices sharing an input; splits by type
// (segments in one launch must share type and cols).
void gemv_multi(Enq& q, GemvDesc tmpl, const std::vector<std::tuple<const DevT*, float*, int, int>>& segs) {
  std::map<int, GemvDesc> by_type;
  for (auto& s : segs) {
    const DevT* w = std::get<0>(s);
    auto it = by_type.find(w->type);
    if (it == by_type.end()) {
      GemvDesc d = tmpl;
      d.type = w->type;
      d.nseg = 0;
      it = by_type.emplace(w->type, d).first;
    }
    add_seg(it->second, *w, std::get<1>(s), std::get<2>(s), std::get<3>(s));
  }
  for (auto& kv : by_type) {
    if (kv.second.nseg == 0) continue;
    kv.second.trace = q.slot("gemv");
    std::string why;
    q.run(gemv_launch(kv.second, q.m->ctx->num_sms, q.st, &why), "gemv");
    if (!q.ok() && q.why == "gemv") q.why = why;
  }
}

// ---- small-T (<= 8) blocks: every projection is a fused GEMV ----------------

void linear_block_small(Enq& q, const LayerW& L, int T, const float* x_in, float* x_mid) {
  kib_qwen35* m = q.m;
  const int li = L.cache_index;
  GemvDesc d = base_desc(m, L.qkv.type, m->H, T);
  d.prologue = kProRms;
  d.in = x_in;
  d.in_ld = m->H;
  d.norm_w = L.attn_norm.f();
  d.conv_state = m->d_r + static_cast<size_t>(li) * m->C * (m->convk - 1);
  d.conv_w = L.conv1d.f();
  d.conv_k = m->convk;
  gemv_multi(q, d,
             {{&L.qkv, m->d_qkv, m->C, kEpiConv},
              {&L.zgate, m->d_z, m->VD, kEpiStore},
              {&L.beta, m->d_beta, m->lvh, kEpiStore},
              {&L.alpha, m->d_alpha, m->lvh, kEpiStore}});
  GdnParams g = {};
  g.conv_out = m->d_qkv;
  g.C = m->C;
  g.beta_raw = m->d_beta;
  g.alpha_raw = m->d_alpha;
  g.ld_ba = m->lvh;
  g.dt_bias = L.dt_bias.f();
  g.ssm_a = L.ssm_a.f();
  g.state = m->d_s + static_cast<size_t>(li) * m->lvh * m->lhd * m->lhd;
  g.out = m->d_y;
  g.T = T;
  g.key_heads = m->lkh;
  g.value_heads = m->lvh;
  g.eps = m->eps;
  g.trace = q.slot("gdn_core");
  q.run(launch_pdl(gdn_core_kernel, dim3(m->lvh, m->lhd / kGdnRows), dim3(128), 0, q.st, g), "gdn_core");
  GemvDesc o = base_desc(m, L.ssm_out.type, m->VD, T);
  o.prologue = kProNormGate;
  o.in = m->d_y;
  o.in_ld = m->VD;
  o.norm_w = L.ssm_norm.f();
  o.gate = m->d_z;
  o.head_dim = m->lhd;
  o.resid = x_in;
  gemv_multi(q, o, {{&L.ssm_out, x_mid, m->H, kEpiResidual}});
}

AttnParams attn_params(kib_qwen35* m, const LayerW& L, uint16_t* kc, uint16_t* vc, const int* pos, int T) {
  AttnParams a = {};
  a.qg = m->d_qg;
  a.kp = m->d_kp;
  a.vp = m->d_vp;
  a.q_norm = L.q_norm.f();
  a.k_norm = L.k_norm.f();
  a.kcache = kc;
  a.vcache = vc;
  a.pos = pos;
  a.T = T;
  a.heads = m->heads;
  a.kv_heads = m->kvh;
  a.eps = m->eps;
  a.theta = m->theta;
  a.sec0 = m->sections[0];
  a.sec1 = m->sections[1];
  a.sec2 = m->sections[2];
  a.sec3 = m->sections[3];
  a.n_dims = 2 * (a.sec0 + a.sec1 + a.sec2 + a.sec3);
  a.nsplit = m->nsplit;
  a.part = m->d_part;
  a.counters = m->d_attn_cnt;
  a.out = m->d_att;
  a.q_out = m->d_qout;
  a.round_q = T >= 64 ? 1 : 0;
  a.trace = nullptr;
  return a;
}

template <int TM>
cudaError_t launch_attn_decode(const AttnParams& a, int kvh, int nsplit, cudaStream_t st) {
  const size_t smem = attn_decode_smem_bytes(a.T);
  static bool cfg = false;
  if (!cfg) {
    cudaFuncSetAttribute(attn_decode_kernel<TM>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    cfg = true;
  }
  return launch_pdl(attn_decode_kernel<TM>, dim3(nsplit, kvh), dim3(256), smem, st, a);
}

void attention_block_small(Enq& q, const LayerW& L, uint16_t* kc, uint16_t* vc, const int* pos, int T,
                           const float* x_in, float* x_mid) {
  kib_qwen35* m = q.m;
  GemvDesc d = base_desc(m, L.q.type, m->H, T);
  d.prologue = kProRms;
  d.in = x_in;
  d.in_ld = m->H;
  d.norm_w = L.attn_norm.f();
  gemv_multi(q, d,
             {{&L.q, m->d_qg, 2 * m->AD, kEpiStore}, {&L.k, m->d_kp, m->KD, kEpiStore}, {&L.v, m->d_vp, m->KD, kEpiStore}});
  AttnParams a = attn_params(m, L, kc, vc, pos, T);
  a.trace = q.slot("attn_decode");
  // register arrays sized to the token count (verify: 2..5 tokens)
  q.run(T == 1   ? launch_attn_decode<1>(a, m->kvh, m->nsplit, q.st)
        : T == 2 ? launch_attn_decode<2>(a, m->kvh, m->nsplit, q.st)
        : T <= 4 ? launch_attn_decode<4>(a, m->kvh, m->nsplit, q.st)
                 : launch_attn_decode<8>(a, m->kvh, m->nsplit, q.st),
        "attn_decode");
  GemvDesc o = base_desc(m, L.o.type, m->AD, T);
  o.prologue = kProPlain;
  o.in = m->d_att;
  o.in_ld = m->AD;
  o.resid = x_in;
  gemv_multi(q, o, {{&L.o, x_mid, m->H, kEpiResidual}});
}

void ffn_small(Enq& q, const LayerW& L, int T, const float* x_mid, float* x_out) {
  kib_qwen35* m = q.m;
  if (L.ffn_gate.type == L.ffn_up.type) {
    GemvDesc d = base_desc(m, L.ffn_gate.type, m->H, T);
    d.prologue = kProRms;
    d.in = x_mid;
    d.in_ld = m->H;
    d.norm_w = L.post_norm.f();
    d.nseg = 0;
    add_seg(d, L.ffn_gate, m->d_act, m->I, kEpiSiluMul, &L.ffn_up);
    d.trace = q.slot("gemv_ffn_pair");
    std::string why;
    q.run(gemv_launch(d, m->ctx->num_sms, q.st, &why), "ffn_gate_up");
  } else {
    GemvDesc d = base_desc(m, L.ffn_gate.type, m->H, T);
    d.prologue = kProRms;
    d.in = x_mid;
    d.in_ld = m->H;
    d.norm_w = L.post_norm.f();
    gemv_multi(q, d, {{&L.ffn_gate, m->d_act, m->I, kEpiStore}, {&L.ffn_up, m->d_act2, m->I, kEpiStore}});
    q.run(silu_mul_launch(m->d_act, m->d_act2, static_cast<size_t>(T) * m->I, q.st), "silu_mul");
  }
  GemvDesc o = base_desc(m, L.ffn_down.type, m->I, T);
  o.prologue = kProPlain;
  o.in = m->d_act;
  o.in_ld = m->I;
  o.resid = x_mid;
  gemv_multi(q, o, {{&L.ffn_down, x_out, m->H, kEpiResidual}});
}

// LM head over T rows: RMSNorm(norm_w) prologue (rows also stored to x_out),
// fused argmax epilogue (+ logits if requested).
void head_small(Enq& q, int T, const float* x, const DevT& norm_w, const DevT& head, int* token_out, float* prob_out,
                float* x_out, float* logits, int* token_log, int* step, int* pos_adv) {
  kib_qwen35* m = q.m;
  GemvDesc d = base_desc(m, head.type, m->H, T);
  d.prologue = kProRms;
  d.in = x;
  d.in_ld = m->H;
  d.norm_w = norm_w.f();
  d.nseg = 0;
  add_seg(d, head, logits, m->V, kEpiArgmax);
  d.argmax = true;
  d.cand_max = m->d_cand_max;
  d.cand_sum = m->d_cand_sum;
  d.cand_idx = m->d_cand_idx;
  d.counter = m->d_head_cnt;
  d.token_out = token_out;
  d.prob_out = prob_out;
  d.x_out = x_out;
  d.token_log = token_log;
  d.step_counter = step;
  d.pos_advance = pos_adv;
  d.trace = q.slot("lm_head");
  std::string why;
  q.run(gemv_launch(d, m->ctx->num_sms, q.st, &why), "lm_head");
}

// KIB_SMALL_BLOCKS=0: 4..8-token forwards keep the fused GEMV path (A/B runs).
bool small_blocks_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("KIB_SMALL_BLOCKS");
    return !(v && v[0] == '0');
  }();
  return on;
}

// KIB_GDN_CHUNKED=0: prefill keeps the token-by-token delta-rule scan (A/B runs).
bool gdn_chunked_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("KIB_GDN_CHUNKED");
    return !(v && v[0] == '0');
  }();
  return on;
}

void main_layers_small(Enq& q, int T, const int* pos) {
  kib_qwen35* m = q.m;
  for (const LayerW& L : m->layers) {
    if (L.kind == 0) {
      linear_block_small(q, L, T, m->d_h, m->d_h1);
    } else {
      const size_t off = static_cast<size_t>(L.cache_index) * m->cap * m->KD;
      attention_block_small(q, L, m->d_k + off, m->d_v + off, pos, T, m->d_h, m->d_h1);
    }
    ffn_small(q, L, T, m->d_h1, m->d_h);
  }
}

// ---- prefill (T > 8) blocks ----------------------------------------------------

// same_x: x is the input of the previous gemm() call, unchanged since (its f16
// copy is reused).  x16_ready: the kernel that wrote x also wrote its half
// copy into d_x16 ([T][cols] packed), used as is above 8 tokens (the 4..8
// bucket splits x itself).
void gemm(Enq& q, const DevT& w, const float* x, int x_ld, int T, float* y, int y_ld, const float* resid = nullptr,
          bool same_x = false, bool x16_ready = false) {
  if (q.m->d_w16 && w.cols() % 64 == 0 && x_ld % 4 == 0)
    q.run(gemm_f16w_launch(w.type, w.p, w.h, w.rows(), w.cols(), x, x_ld, T, y, y_ld, resid, q.m->d_w16, q.m->d_x16,
                           !same_x && !(x16_ready && T > 8 && x_ld == w.cols()), q.m->ctx->num_sms, q.st,
                           q.m->ctx->d_err),
          "gemm_f16w");
  else
    q.run(gemm_f16_launch(w.type, w.p, w.rows(), w.cols(), x, x_ld, T, y, y_ld, resid, q.st), "gemm");
}

// Several weights with the same input as ONE GEMM above 64 tokens: their
// resident f16 copies were laid out back to back at load time, so rows
// [w0 | w1 | ...] are one matrix; the outputs land side by side in d_proj
// ([T][sum of rows]).  Returns the row stride, or 0 when the copies are not
// contiguous (the caller then runs them one by one).
int gemm_cat(Enq& q, std::initializer_list<const DevT*> ws, const float* x, int x_ld, int T, bool x16_ready) {
  kib_qwen35* m = q.m;
  static const bool on = [] {
    const char* v = std::getenv("KIB_GEMM_CAT");
    return !(v && v[0] == '0');
  }();
  if (!on || T <= 64 || !m->d_w16) return 0;
  const DevT* first = *ws.begin();
  int rows = 0;
  const __half* next = first->h;
  for (const DevT* w : ws) {
    if (!w->h || w->h != next || w->cols() != first->cols() || w->cols() % 64) return 0;
    rows += w->rows();
    const size_t bytes = (static_cast<size_t>(w->rows()) * w->cols() * 2 + 255) & ~static_cast<size_t>(255);
    next = reinterpret_cast<const __half*>(reinterpret_cast<const uint8_t*>(w->h) + bytes);
    if (bytes != static_cast<size_t>(w->rows()) * w->cols() * 2 && w != *(ws.end() - 1)) return 0;  // padding gap
  }
  const int ld = (rows + 3) & ~3;
  q.run(gemm_f16w_launch(first->type, first->p, first->h, rows, first->cols(), x, x_ld, T, m->d_proj, ld, nullptr,
                         m->d_w16, m->d_x16, !(x16_ready && x_ld == first->cols()), m->ctx->num_sms, q.st,
                         m->ctx->d_err),
        "gemm_cat");
  return ld;
}

void linear_block_prefill(Enq& q, const LayerW& L, int T, const float* x_in, float* x_mid) {
  kib_qwen35* m = q.m;
  const int li = L.cache_index;
  q.run(rms_rows_launch(x_in, L.attn_norm.f(), T, m->H, m->eps, m->d_norm, q.st, m->d_x16), "rms");
  // qkv | z | beta | alpha: one GEMM when their copies are contiguous
  float *qkv = m->d_qkv, *z = m->d_z, *beta = m->d_beta, *alpha = m->d_alpha;
  int qkv_ld = m->C, z_ld = m->VD, ld_ba = m->lvh;
  if (const int ld = gemm_cat(q, {&L.qkv, &L.zgate, &L.beta, &L.alpha}, m->d_norm, m->H, T, true)) {
    qkv = m->d_proj;
    z = qkv + L.qkv.rows();
    beta = z + L.zgate.rows();
    alpha = beta + L.beta.rows();
    qkv_ld = z_ld = ld_ba = ld;
  } else {
    gemm(q, L.qkv, m->d_norm, m->H, T, qkv, qkv_ld, nullptr, false, true);
    gemm(q, L.zgate, m->d_norm, m->H, T, z, z_ld, nullptr, true);
    gemm(q, L.beta, m->d_norm, m->H, T, beta, ld_ba, nullptr, true);
    gemm(q, L.alpha, m->d_norm, m->H, T, alpha, ld_ba, nullptr, true);
  }
  q.run(conv_launch(m->d_r + static_cast<size_t>(li) * m->C * (m->convk - 1), qkv, qkv_ld, L.conv1d.f(), m->convk,
                    m->C, T, qkv, qkv_ld, 1, q.st),
        "conv");
  GdnParams g = {};
  g.conv_out = qkv;
  g.C = qkv_ld;
  g.beta_raw = beta;
  g.alpha_raw = alpha;
  g.ld_ba = ld_ba;
  g.dt_bias = L.dt_bias.f();
  g.ssm_a = L.ssm_a.f();
  g.state = m->d_s + static_cast<size_t>(li) * m->lvh * m->lhd * m->lhd;
  g.out = m->d_y;
  g.T = T;
  g.key_heads = m->lkh;
  g.value_heads = m->lvh;
  g.eps = m->eps;
  g.trace = nullptr;
  if (m->lhd == 128 && m->lkh <= m->lvh && m->C % 4 == 0 && T >= kGc && gdn_chunked_enabled()) {
    // token-parallel norms and gate/beta, then the chunked delta rule: the
    // per-chunk matrices for every chunk at once, then the scan over chunks
    q.run(launch_pdl(gdn_prep_kernel, dim3(T, m->lkh), dim3(128), 0, q.st, qkv, qkv_ld, alpha, beta, ld_ba,
                     L.dt_bias.f(), L.ssm_a.f(), m->lkh, m->lvh, m->eps),
          "gdn_prep");
    static bool chunk_cfg = false;
    if (!chunk_cfg) {
      q.run(cudaFuncSetAttribute(gdn_chunk_prep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(kGcPrepSmem)),
            "gdn_chunk_attr");
      q.run(cudaFuncSetAttribute(gdn_chunk_scan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(kGcScanSmem)),
            "gdn_chunk_attr");
      q.run(cudaFuncSetAttribute(gdn_chunk_scan_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(kGcScanTcSmem)),
            "gdn_chunk_attr");
      q.run(cudaFuncSetAttribute(gdn_chunk_prep_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(kGcPrepTcSmem)),
            "gdn_chunk_attr");
      chunk_cfg = true;
    }
    GdnChunkParams gc;
    gc.conv_out = qkv;
    gc.C = qkv_ld;
    gc.g = alpha;
    gc.beta = beta;
    gc.ld_ba = ld_ba;
    gc.state = g.state;
    gc.out = m->d_y;
    gc.ws = m->d_gdn_ws;
    gc.T = T;
    gc.key_heads = m->lkh;
    gc.value_heads = m->lvh;
    static const bool prep_tc = [] {
      const char* v = std::getenv("KIB_GDN_PREP_TC");
      return !(v && v[0] == '0');
    }();
    if (prep_tc)
      q.run(launch_pdl(gdn_chunk_prep_tc_kernel, dim3(m->lvh, (T + kGc - 1) / kGc), dim3(256), kGcPrepTcSmem, q.st,
                       gc),
            "gdn_chunk_prep_tc");
    else
      q.run(launch_pdl(gdn_chunk_prep_kernel, dim3(m->lvh, (T + kGc - 1) / kGc), dim3(256), kGcPrepSmem, q.st, gc),
            "gdn_chunk_prep");
    static const bool scan_tc = [] {
      const char* v = std::getenv("KIB_GDN_SCAN_TC");
      return !(v && v[0] == '0');
    }();
    if (scan_tc)
      q.run(launch_pdl(gdn_chunk_scan_tc_kernel, dim3(m->lvh, kGcD / kGcRows), dim3(256), kGcScanTcSmem, q.st, gc),
            "gdn_chunk_scan_tc");
    else
      q.run(launch_pdl(gdn_chunk_scan_kernel, dim3(m->lvh, kGcD / kGcRows), dim3(256), kGcScanSmem, q.st, gc),
            "gdn_chunk_scan");
  } else if (m->lhd == 128 && m->lkh <= m->lvh && m->C % 4 == 0) {
    // token-parallel norms and gate/beta first, then the sequential scan alone
    q.run(launch_pdl(gdn_prep_kernel, dim3(T, m->lkh), dim3(128), 0, q.st, qkv, qkv_ld, alpha, beta, ld_ba,
                     L.dt_bias.f(), L.ssm_a.f(), m->lkh, m->lvh, m->eps),
          "gdn_prep");
    static bool scan_cfg = false;
    if (!scan_cfg) {
      q.run(cudaFuncSetAttribute(gdn_scan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kGdnScanSmem),
            "gdn_scan_attr");
      scan_cfg = true;
    }
    q.run(launch_pdl(gdn_scan_kernel, dim3(m->lvh, m->lhd / kGdnScanRowsPerCta), dim3(128), kGdnScanSmem, q.st, g),
          "gdn_scan");
  } else {
    q.run(launch_pdl(gdn_core_kernel, dim3(m->lvh, m->lhd / kGdnRows), dim3(128), 0, q.st, g), "gdn_core");
  }
  q.run(norm_gate_launch(m->d_y, L.ssm_norm.f(), z, T, m->lvh, m->lhd, m->eps, m->d_norm2, q.st, m->d_x16, z_ld),
        "norm_gate");
  gemm(q, L.ssm_out, m->d_norm2, m->VD, T, x_mid, m->H, x_in, false, true);
}

void attention_block_prefill(Enq& q, const LayerW& L, uint16_t* kc, uint16_t* vc, const int* pos, int T,
                             const float* x_in, float* x_mid) {
  kib_qwen35* m = q.m;
  q.run(rms_rows_launch(x_in, L.attn_norm.f(), T, m->H, m->eps, m->d_norm, q.st, m->d_x16), "rms");
  gemm(q, L.q, m->d_norm, m->H, T, m->d_qg, 2 * m->AD, nullptr, false, true);
  gemm(q, L.k, m->d_norm, m->H, T, m->d_kp, m->KD, nullptr, true);
  gemm(q, L.v, m->d_norm, m->H, T, m->d_vp, m->KD, nullptr, true);
  const AttnParams a = attn_params(m, L, kc, vc, pos, T);
  q.run(launch_pdl(attn_prep_kernel, dim3(T), dim3(256), 8 * kHd * sizeof(float), q.st, a), "attn_prep");
  static const bool fa2_on = [] {
    const char* v = std::getenv("KIB_FA2");
    return !(v && v[0] == '0');
  }();
  if (a.round_q && fa2_on && m->heads % m->kvh == 0 && (m->heads / m->kvh) % 2 == 0) {
    static bool fa2_cfg = false;
    if (!fa2_cfg) {
      q.run(cudaFuncSetAttribute(attn_prefill_mma2_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(kFa2Smem)),
            "attn_prefill_mma2_attr");
      fa2_cfg = true;
    }
    // key splits so that the (query tile, head pair) CTAs cover the GPU about twice
    const int ctas = ((T + kFa2Q - 1) / kFa2Q) * (m->heads / 2);
    static const int env_splits = [] {
      const char* v = std::getenv("KIB_FA_SPLITS");
      return v ? std::atoi(v) : 0;
    }();
    int ns = env_splits > 0 ? env_splits : (2 * m->ctx->num_sms + ctas - 1) / ctas;
    ns = std::max(1, std::min(ns, kFa2MaxSplits));
    AttnParams a2 = a;
    a2.part = m->d_fa_part;
    q.run(launch_pdl(attn_prefill_mma2_kernel, dim3((T + kFa2Q - 1) / kFa2Q, m->heads / 2, ns), dim3(256), kFa2Smem,
                     q.st, a2),
          "attn_prefill_mma2");
    if (ns > 1)
      q.run(launch_pdl(attn_prefill_merge_kernel, dim3(T, m->heads), dim3(kHd), 0, q.st, a2, ns), "attn_prefill_merge");
  } else if (a.round_q && m->heads % m->kvh == 0) {
    static bool fa_cfg = false;
    if (!fa_cfg) {
      q.run(cudaFuncSetAttribute(attn_prefill_mma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(kFaSmem)),
            "attn_prefill_mma_attr");
      fa_cfg = true;
    }
    q.run(launch_pdl(attn_prefill_mma_kernel, dim3((T + kFaQ - 1) / kFaQ, m->heads), dim3(128), kFaSmem, q.st, a),
          "attn_prefill_mma");
  } else {
    q.run(launch_pdl(attn_prefill_kernel, dim3((T + 7) / 8, m->heads), dim3(256), 0, q.st, a), "attn_prefill");
  }
  gemm(q, L.o, m->d_att, m->AD, T, x_mid, m->H, x_in);
}

void ffn_prefill(Enq& q, const LayerW& L, int T, const float* x_mid, float* x_out) {
  kib_qwen35* m = q.m;
  q.run(rms_rows_launch(x_mid, L.post_norm.f(), T, m->H, m->eps, m->d_norm, q.st, m->d_x16), "rms");
  if (gemm_cat(q, {&L.ffn_gate, &L.ffn_up}, m->d_norm, m->H, T, true) == 2 * m->I) {
    q.run(silu_mul_cat_launch(m->d_proj, T, m->I, m->d_act, q.st, m->d_x16), "silu_mul_cat");
  } else {
    gemm(q, L.ffn_gate, m->d_norm, m->H, T, m->d_act, m->I, nullptr, false, true);
    gemm(q, L.ffn_up, m->d_norm, m->H, T, m->d_act2, m->I, nullptr, true);
    q.run(silu_mul_launch(m->d_act, m->d_act2, static_cast<size_t>(T) * m->I, q.st, m->d_x16), "silu_mul");
  }
  gemm(q, L.ffn_down, m->d_act, m->I, T, x_out, m->H, x_mid, false, true);
}

void main_layers_prefill(Enq& q, int T, const int* pos) {
  kib_qwen35* m = q.m;
  for (const LayerW& L : m->layers) {
    if (L.kind == 0) {
      linear_block_prefill(q, L, T, m->d_h, m->d_h1);
    } else {
      const size_t off = static_cast<size_t>(L.cache_index) * m->cap * m->KD;
      attention_block_prefill(q, L, m->d_k + off, m->d_v + off, pos, T, m->d_h, m->d_h1);
    }
    ffn_prefill(q, L, T, m->d_h1, m->d_h);
  }
}

// 4..8 tokens (MTP verify): the projections as few-token tensor-core GEMMs
// (kq_skinny, x split into halves: the 4..8 bucket numerics), the delta rule
// and the split-K attention of the decode path.
void linear_block_mid(Enq& q, const LayerW& L, int T, const float* x_in, float* x_mid) {
  kib_qwen35* m = q.m;
  const int li = L.cache_index;
  q.run(rms_rows_launch(x_in, L.attn_norm.f(), T, m->H, m->eps, m->d_norm, q.st), "rms");
  gemm(q, L.qkv, m->d_norm, m->H, T, m->d_qkv, m->C);
  q.run(conv_launch(m->d_r + static_cast<size_t>(li) * m->C * (m->convk - 1), m->d_qkv, m->C, L.conv1d.f(), m->convk,
                    m->C, T, m->d_qkv, m->C, 1, q.st),
        "conv");
  gemm(q, L.zgate, m->d_norm, m->H, T, m->d_z, m->VD, nullptr, true);
  gemm(q, L.beta, m->d_norm, m->H, T, m->d_beta, m->lvh, nullptr, true);
  gemm(q, L.alpha, m->d_norm, m->H, T, m->d_alpha, m->lvh, nullptr, true);
  GdnParams g = {};
  g.conv_out = m->d_qkv;
  g.C = m->C;
  g.beta_raw = m->d_beta;
  g.alpha_raw = m->d_alpha;
  g.ld_ba = m->lvh;
  g.dt_bias = L.dt_bias.f();
  g.ssm_a = L.ssm_a.f();
  g.state = m->d_s + static_cast<size_t>(li) * m->lvh * m->lhd * m->lhd;
  g.out = m->d_y;
  g.T = T;
  g.key_heads = m->lkh;
  g.value_heads = m->lvh;
  g.eps = m->eps;
  q.run(launch_pdl(gdn_core_kernel, dim3(m->lvh, m->lhd / kGdnRows), dim3(128), 0, q.st, g), "gdn_core");
  q.run(norm_gate_launch(m->d_y, L.ssm_norm.f(), m->d_z, T, m->lvh, m->lhd, m->eps, m->d_norm2, q.st), "norm_gate");
  gemm(q, L.ssm_out, m->d_norm2, m->VD, T, x_mid, m->H, x_in);
}

void attention_block_mid(Enq& q, const LayerW& L, uint16_t* kc, uint16_t* vc, const int* pos, int T,
                         const float* x_in, float* x_mid) {
  kib_qwen35* m = q.m;
  q.run(rms_rows_launch(x_in, L.attn_norm.f(), T, m->H, m->eps, m->d_norm, q.st), "rms");
  gemm(q, L.q, m->d_norm, m->H, T, m->d_qg, 2 * m->AD);
  gemm(q, L.k, m->d_norm, m->H, T, m->d_kp, m->KD, nullptr, true);
  gemm(q, L.v, m->d_norm, m->H, T, m->d_vp, m->KD, nullptr, true);
  AttnParams a = attn_params(m, L, kc, vc, pos, T);
  q.run(T <= 4 ? launch_attn_decode<4>(a, m->kvh, m->nsplit, q.st) : launch_attn_decode<8>(a, m->kvh, m->nsplit, q.st),
        "attn_decode");
  gemm(q, L.o, m->d_att, m->AD, T, x_mid, m->H, x_in);
}

void main_layers_mid(Enq& q, int T, const int* pos) {
  kib_qwen35* m = q.m;
  for (const LayerW& L : m->layers) {
    if (L.kind == 0) {
      linear_block_mid(q, L, T, m->d_h, m->d_h1);
    } else {
      const size_t off = static_cast<size_t>(L.cache_index) * m->cap * m->KD;
      attention_block_mid(q, L, m->d_k + off, m->d_v + off, pos, T, m->d_h, m->d_h1);
    }
    ffn_prefill(q, L, T, m->d_h1, m->d_h);
  }
}

const DevT& head_weight(kib_qwen35* m) { return m->output.ok() ? m->output : m->tok_embd; }

// ------------------------------------------------------------------ loading
int bind(kib_qwen35* m, const std::map<std::string, DevT>& dev, const std::string& name,
         const std::vector<uint64_t>& shape, DevT& out, bool required = true) {
  auto it = dev.find(name);
  if (it == dev.end()) {
    if (!required) return KIB_OK;
    return fail(m, KIB_ERR_INVALID_ARGUMENT, "missing Qwen3.5 GGUF tensor: " + name);
  }
  if (it->second.shape != shape) return fail(m, KIB_ERR_INVALID_ARGUMENT, "Qwen3.5 GGUF tensor " + name + " has unexpected shape");
  out = it->second;
  return KIB_OK;
}

int capture(kib_qwen35* m, cudaGraphExec_t* exec, const std::function<void(Enq&)>& body, bool tracing = false) {
  cudaStream_t st = m->ctx->stream;
  Enq q{m, st};
  q.tracing = tracing && m->trace_on;
  cudaGraph_t g = nullptr;
  ENG_CUDA(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
  body(q);
  cudaError_t ce = cudaStreamEndCapture(st, &g);
  if (!q.ok()) {
    if (g) cudaGraphDestroy(g);
    return fail(m, KIB_ERR_INTERNAL, "graph capture launch failed: " + q.why + ": " + cudaGetErrorString(q.e));
  }
  if (ce != cudaSuccess) return fail(m, KIB_ERR_INTERNAL, std::string("graph capture: ") + cudaGetErrorString(ce));
  cudaError_t ie = cudaGraphInstantiate(exec, g, 0);
  cudaGraphDestroy(g);
  if (ie != cudaSuccess) *exec = nullptr;
  if (ie != cudaSuccess) return fail(m, KIB_ERR_INTERNAL, std::string("graph instantiate: ") + cudaGetErrorString(ie));
  return KIB_OK;
}

int sync_check(kib_qwen35* m, const char* what) {
  cudaError_t e = cudaStreamSynchronize(m->ctx->stream);
  if (e != cudaSuccess) return fail(m, KIB_ERR_INTERNAL, std::string(what) + ": " + cudaGetErrorString(e));
  int err = 0;
  cudaMemcpy(&err, m->ctx->d_err, sizeof(int), cudaMemcpyDeviceToHost);
  if (err) {
    cudaMemset(m->ctx->d_err, 0, sizeof(int));
    return fail(m, KIB_ERR_TIMEOUT, std::string(what) + ": a bounded device wait gave up");
  }
  return KIB_OK;
}

// As sync_check, with the error flag already copied (in stream order) to *h_err.
int sync_check_flag(kib_qwen35* m, const char* what, const int* h_err) {
  cudaError_t e = cudaStreamSynchronize(m->ctx->stream);
  if (e != cudaSuccess) return fail(m, KIB_ERR_INTERNAL, std::string(what) + ": " + cudaGetErrorString(e));
  if (*reinterpret_cast<const volatile int*>(h_err)) {
    cudaMemset(m->ctx->d_err, 0, sizeof(int));
    return fail(m, KIB_ERR_TIMEOUT, std::string(what) + ": a bounded device wait gave up");
  }
  return KIB_OK;
}

int set_pos(kib_qwen35* m, int* dptr, uint64_t value) {
  m->h_pin[0] = static_cast<int>(value);
  ENG_CUDA(cudaMemcpyAsync(dptr, m->h_pin, sizeof(int), cudaMemcpyHostToDevice, m->ctx->stream));
  ENG_CUDA(cudaStreamSynchronize(m->ctx->stream));
  return KIB_OK;
}

// Forward over T <= 8 tokens already in d_tokens at position *d_pos, through
// the LM head (argmax per row into d_argmax, normed rows into d_hn).
int forward_small(kib_qwen35* m, int T, bool want_logits) {
  if (!m->fwd_graph[T] || m->fwd_graph_logits[T] != want_logits) {
    if (m->fwd_graph[T]) cudaGraphExecDestroy(m->fwd_graph[T]);
    m->fwd_graph[T] = nullptr;
    int rc = capture(m, &m->fwd_graph[T], [&](Enq& q) {
      q.run(get_rows_launch(m->tok_embd.type, m->tok_embd.p, m->V, m->H, m->d_tokens, T, m->d_h, m->H, q.st), "embed");
      // 4..8 tokens (MTP verify): projections on the few-token tensor-core
      // GEMM with x split into halves (the same 4..8 bucket numerics as the
      // GEMV path), delta rule and attention as on the decode path
      if (T >= 4 && m->d_w16 && small_blocks_enabled()) main_layers_mid(q, T, m->d_pos);
      else main_layers_small(q, T, m->d_pos);
      head_small(q, T, m->d_h, m->output_norm, head_weight(m), m->d_argmax, m->d_prob, m->d_hn,
                 want_logits ? m->d_logits : nullptr, nullptr, nullptr, nullptr);
    });
    if (rc) return rc;
    m->fwd_graph_logits[T] = want_logits;
  }
  ENG_CUDA(cudaGraphLaunch(m->fwd_graph[T], m->ctx->stream));
  return KIB_OK;
}

// Prefill chunk with T > 8 tokens (not graph-captured: one-shot).
int forward_prefill(kib_qwen35* m, int T, bool head) {
  Enq q{m, m->ctx->stream};
  q.run(get_rows_launch(m->tok_embd.type, m->tok_embd.p, m->V, m->H, m->d_tokens, T, m->d_h, m->H, q.st), "embed");
  main_layers_prefill(q, T, m->d_pos);
  if (head) {
    head_small(q, 1, m->d_h + static_cast<size_t>(T - 1) * m->H, m->output_norm, head_weight(m), m->d_argmax, m->d_prob,
               nullptr, nullptr, nullptr, nullptr, nullptr);
  }
  if (!q.ok()) return fail(m, KIB_ERR_INTERNAL, "prefill launch: " + q.why + ": " + cudaGetErrorString(q.e));
  return KIB_OK;
}

// MTP layer over T tokens (ids in d_tokens, h rows in h_rows) at *d_mtp_pos:
// writes the MTP KV cache and the normed h_nextn rows into d_mtp_h; with
// head, also the argmax of the LM head per row.
void mtp_enqueue(Enq& q, int T, const int* ids, const float* h_rows, bool head, int* token_out, float* prob_out,
                 int* token_log, int* step, int* pos_adv) {
  kib_qwen35* m = q.m;
  const LayerW& L = m->mtp;
  q.run(get_rows_launch(m->tok_embd.type, m->tok_embd.p, m->V, m->H, ids, T, m->d_e, m->H, q.st), "mtp_embed");
  q.run(launch_pdl(mtp_cat_kernel, dim3(T), dim3(256), 0, q.st, static_cast<const float*>(m->d_e), h_rows,
                   L.enorm.f(), L.hnorm.f(), m->H, m->eps, m->d_cat),
        "mtp_cat");
  if (T <= kMaxSmallT) {
    GemvDesc d = base_desc(m, L.eh_proj.type, 2 * m->H, T);
    d.prologue = kProPlain;
    d.in = m->d_cat;
    d.in_ld = 2 * m->H;
    gemv_multi(q, d, {{&L.eh_proj, m->d_hm, m->H, kEpiStore}});
    attention_block_small(q, L, m->d_mk, m->d_mv, m->d_mtp_pos, T, m->d_hm, m->d_hm1);
    ffn_small(q, L, T, m->d_hm1, m->d_hm);
  } else {
    gemm(q, L.eh_proj, m->d_cat, 2 * m->H, T, m->d_hm, m->H);
    attention_block_prefill(q, L, m->d_mk, m->d_mv, m->d_mtp_pos, T, m->d_hm, m->d_hm1);
    ffn_prefill(q, L, T, m->d_hm1, m->d_hm);
  }
  const DevT& hn = L.shead_norm.ok() ? L.shead_norm : m->output_norm;
  if (head) {
    head_small(q, T, m->d_hm, hn, head_weight(m), token_out, prob_out, m->d_mtp_h, nullptr, token_log, step, pos_adv);
  } else {
    q.run(rms_rows_launch(m->d_hm, hn.f(), T, m->H, m->eps, m->d_mtp_h, q.st), "mtp_head_norm");
  }
}

}  // namespace

// ====================================================================== C ABI
extern "C" {

// ---- persistent decode program ------------------------------------------------

struct PkSegIn {
  const DevT* w;
  const DevT* w2;
  uint64_t* out;  // cells
  int epi;
};

// Fills the GEMV fields of a stage; false (with pk_why) when the shapes do
// not meet the ring's copy rules.
static bool pk_gemv_stage(kib_qwen35* m, PkStage& S, int kind, const std::vector<PkSegIn>& segs, int grid) {
  const int type = segs[0].w->type;
  const int cols = segs[0].w->cols();
  if (type != kTypeQ4K && type != kTypeQ5K && type != kTypeQ6K) {
    m->pk_why = "matrix type other than Q4_K / Q5_K / Q6_K";
    return false;
  }
  if (cols % 256 || cols > kPkMaxCols || static_cast<int>(segs.size()) > kPkMaxSegs) {
    m->pk_why = "unsupported GEMV shape";
    return false;
  }
  const int row_bytes = cols / 256 * kquant_block_bytes(type);
  int g = 1;
  while ((static_cast<long>(g) * row_bytes) % 16) ++g;  // rows per 16-byte aligned piece
  S.kind = kind;
  S.type = type;
  S.cols = cols;
  S.row_bytes = row_bytes;
  S.nseg = 0;
  S.paired = segs[0].w2 != nullptr;
  int rows = 0;
  for (const PkSegIn& in : segs) {
    if (in.w->type != type || in.w->cols() != cols || (in.w2 != nullptr) != (S.paired != 0)) {
      m->pk_why = "segments of one stage differ in type or shape";
      return false;
    }
    const int r = in.w->rows();
    if (r % g || reinterpret_cast<uintptr_t>(in.w->p) % 16 || (in.w2 && reinterpret_cast<uintptr_t>(in.w2->p) % 16)) {
      m->pk_why = "segment rows/base not aligned for bulk copies";
      return false;
    }
    PkSeg& sg = S.seg[S.nseg++];
    sg.w = in.w->p;
    sg.w2 = in.w2 ? in.w2->p : nullptr;
    sg.out = in.out;
    sg.row_begin = rows;
    sg.rows = r;
    sg.epi = in.epi;
    rows += r;
  }
  S.rows = rows;
  const int cap = std::min((kPkSlotBytes / (S.paired ? 2 : 1)) / row_bytes, kPkMaxTileRows) / g * g;
  int want = (rows + grid - 1) / grid;
  want = (want + g - 1) / g * g;
  const int units = cols / 64;
  S.rg = units <= 16 ? 16 : units <= 32 ? 32 : 64;
  S.tile_rows = std::max(g, std::min(cap, want));
  if (want > cap) {
    // several tiles per CTA: make a tile a whole number of passes of the
    // CTA's row groups, so no pass runs part-empty
    const int per_pass = kPkConsumers / S.rg * kPkRows;
    int l = per_pass;
    while (l % g) l += per_pass;  // lcm(per_pass, g)
    if (cap >= l) S.tile_rows = cap / l * l;
  }
  S.ntiles = (rows + S.tile_rows - 1) / S.tile_rows;
  S.eps = m->eps;
  return cap >= g;
}

// Cells of the persistent step: every stage output gets its own array (an
// even number of cells, so pair loads stay 16-byte aligned).
static size_t pk_cells_needed(const kib_qwen35* m, int nsplit) {
  size_t n = 0;
  auto need = [&](size_t c) { n += (c + 1) & ~size_t(1); };
  for (const LayerW& L : m->layers) {
    if (L.kind == 0) {
      need(L.qkv.rows());
      need(L.zgate.rows());
      need(L.beta.rows());
      need(L.alpha.rows());
      need(static_cast<size_t>(m->lvh) * m->lhd);
    } else {
      need(L.q.rows());
      need(L.k.rows());
      need(L.v.rows());
      need(static_cast<size_t>(nsplit) * m->heads * (kHd + 2));
      need(static_cast<size_t>(m->heads) * kHd);
    }
    need(m->H);
    need(L.ffn_gate.rows());
    need(m->H);
  }
  return n;
}

// Tensor map over one attention layer's K or V cache, [positions][kv_dim]
// halves, as a rank-3 map [1][positions][kv_dim] (the persistent kernel issues
// 3-D copies): boxes of one KV head's 256 columns x 32 positions, unswizzled,
// rows past the cache read as zeros.
static bool kv_cache_tensor_map(CUtensorMap* map, const uint16_t* base, int kv_dim, int positions) {
  static PFN_cuTensorMapEncodeTiled_v12000 enc = [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      f = nullptr;
    return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
  }();
  if (!enc || (reinterpret_cast<uintptr_t>(base) & 15u) || kv_dim % kHd) return false;
  const cuuint64_t dims[3] = {static_cast<cuuint64_t>(kv_dim), static_cast<cuuint64_t>(positions), 1};
  const cuuint64_t strides[2] = {static_cast<cuuint64_t>(kv_dim) * 2,
                                 static_cast<cuuint64_t>(kv_dim) * static_cast<cuuint64_t>(positions) * 2};
  const cuuint32_t box[3] = {static_cast<cuuint32_t>(kHd), static_cast<cuuint32_t>(kAttnChunk), 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<uint16_t*>(base), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

static int build_pk(kib_qwen35* m) {
  m->pk_on = false;
  if (const char* e = std::getenv("KIB_PERSISTENT"); e && e[0] == '0') {
    m->pk_why = "disabled by KIB_PERSISTENT=0";
    return KIB_OK;
  }
  const int grid = m->ctx->num_sms;
  if (m->convk != 4 || m->hd != kHd || m->lhd != 128 || m->heads != 4 * m->kvh || m->kvh < 1 ||
      grid / m->kvh > kPkMaxSplits || grid < m->lvh * (128 / kPkGdnRows) / 2) {
    m->pk_why = "model shape outside the persistent kernel's limits";
    return KIB_OK;
  }
  int coop = 0;
  cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, m->ctx->device);
  const int nsplit = grid / m->kvh;
  const int n_dims = 2 * (m->sections[0] + m->sections[1] + m->sections[2] + m->sections[3]);
  if (n_dims / 2 > kPkRopePairs) {
    m->pk_why = "rotary dimensions beyond the persistent kernel's table";
    return KIB_OK;
  }
  if (!m->d_pk_rope) {
    // 1 / theta^(2p / n_dims) in float, the reference's expression (mrope_f32_in_place)
    std::vector<float> fr(kPkRopePairs, 0.0f);
    for (int p = 0; p < n_dims / 2; ++p) {
      const float exponent = static_cast<float>(2 * p) / static_cast<float>(n_dims);
      fr[p] = 1.0f / std::pow(m->theta, exponent);
    }
    if (dalloc(&m->d_pk_rope, kPkRopePairs) != cudaSuccess) return fail(m, KIB_ERR_INTERNAL, "pk rope alloc");
    ENG_CUDA(cudaMemcpy(m->d_pk_rope, fr.data(), fr.size() * sizeof(float), cudaMemcpyHostToDevice));
  }
  if (!m->d_pk_tmaps) {
    // the attention stages stream their K/V rows by tensor copies of 32
    // positions x 256 columns (one KV head)
    const size_t na = m->plan.full_attention_layers;
    std::vector<CUtensorMap> maps(2 * std::max<size_t>(na, 1));
    for (size_t ai = 0; ai < na; ++ai) {
      const size_t off = ai * static_cast<size_t>(m->cap) * m->KD;
      if (!kv_cache_tensor_map(&maps[2 * ai], m->d_k + off, m->KD, m->cap) ||
          !kv_cache_tensor_map(&maps[2 * ai + 1], m->d_v + off, m->KD, m->cap)) {
        m->pk_why = "KV cache tensor maps unavailable";
        return KIB_OK;
      }
    }
    if (cudaMalloc(&m->d_pk_tmaps, maps.size() * sizeof(CUtensorMap)) != cudaSuccess)
      return fail(m, KIB_ERR_INTERNAL, "pk tensor map alloc");
    ENG_CUDA(cudaMemcpy(m->d_pk_tmaps, maps.data(), maps.size() * sizeof(CUtensorMap), cudaMemcpyHostToDevice));
  }
  const size_t ncells = pk_cells_needed(m, nsplit);
  if (!m->d_pk_cells) {
    if (dalloc(&m->d_pk_cells, ncells) != cudaSuccess) return fail(m, KIB_ERR_INTERNAL, "pk cell alloc");
    ENG_CUDA(cudaMemset(m->d_pk_cells, 0, ncells * sizeof(uint64_t)));
  }
  uint64_t* next_cell = m->d_pk_cells;
  auto cells = [&](size_t c) {
    uint64_t* p = next_cell;
    next_cell += (c + 1) & ~size_t(1);
    return p;
  };
  std::vector<PkStage> st;
  // a stage's tag is its index + 1; readers name the tag of the stage that wrote their input
  auto add = [&](PkStage& S) {
    S.tag = static_cast<int>(st.size()) + 1;
    st.push_back(S);
    return S.tag;
  };
  const void* h_in = m->d_h;  // the residual stream entering the layer (layer 0: the embedding row)
  int h_tag = 0;
  for (const LayerW& L : m->layers) {
    const int li = L.cache_index;
    const void* mid = nullptr;  // the stream after the mixer (attention or GDN) block
    int mid_tag = 0;
    if (L.kind == 0) {
      uint64_t* c_qkv = cells(L.qkv.rows());
      uint64_t* c_z = cells(L.zgate.rows());
      uint64_t* c_beta = cells(L.beta.rows());
      uint64_t* c_alpha = cells(L.alpha.rows());
      // the in-projection group (qkv with the conv epilogue, z, beta, alpha):
      // one stage, or -- when the matrices differ in K-quant type, as the
      // Q4_K_M files' Q5_K attn_qkv does -- one stage per type, all reading
      // the same normed input
      const std::vector<PkSegIn> in_segs = {{&L.qkv, nullptr, c_qkv, kEpiConv},
                                            {&L.zgate, nullptr, c_z, kEpiStore},
                                            {&L.beta, nullptr, c_beta, kEpiStore},
                                            {&L.alpha, nullptr, c_alpha, kEpiStore}};
      int seg_tag[4] = {0, 0, 0, 0};
      for (size_t i0 = 0; i0 < in_segs.size();) {
        size_t i1 = i0 + 1;
        while (i1 < in_segs.size() && in_segs[i1].w->type == in_segs[i0].w->type) ++i1;
        PkStage a = {};
        if (!pk_gemv_stage(m, a, kPkGemv, std::vector<PkSegIn>(in_segs.begin() + i0, in_segs.begin() + i1), grid))
          return KIB_OK;
        a.prologue = kProRms;
        a.in = h_in;
        a.in_tag = h_tag;
        a.norm_w = L.attn_norm.f();
        a.conv_state = m->d_r + static_cast<size_t>(li) * m->C * (m->convk - 1);
        a.conv_w = L.conv1d.f();
        const int tg = add(a);
        for (size_t i = i0; i < i1; ++i) seg_tag[i] = tg;
        i0 = i1;
      }
      if (seg_tag[2] != seg_tag[3]) {
        m->pk_why = "ssm beta and alpha types differ";
        return KIB_OK;
      }
      PkStage g = {};
      g.kind = kPkGdn;
      g.conv_out = c_qkv;
      g.C = m->C;
      g.beta_raw = c_beta;
      g.alpha_raw = c_alpha;
      g.src_tag = seg_tag[0];
      g.src2_tag = seg_tag[2] == seg_tag[0] ? 0 : seg_tag[2];
      g.dt_bias = L.dt_bias.f();
      g.ssm_a = L.ssm_a.f();
      g.state = m->d_s + static_cast<size_t>(li) * m->lvh * m->lhd * m->lhd;
      g.gdn_out = cells(static_cast<size_t>(m->lvh) * m->lhd);
      g.key_heads = m->lkh;
      g.value_heads = m->lvh;
      g.eps = m->eps;
      const int g_tag = add(g);
      uint64_t* c_h1 = cells(m->H);
      PkStage o = {};
      if (!pk_gemv_stage(m, o, kPkGemv, {{&L.ssm_out, nullptr, c_h1, kEpiResidual}}, grid)) return KIB_OK;
      o.prologue = kProNormGate;
      o.in = g.gdn_out;
      o.in_tag = g_tag;
      o.gate = c_z;
      o.gate_tag = seg_tag[1];
      o.norm_w = L.ssm_norm.f();
      o.head_dim = m->lhd;
      o.resid = h_in;
      o.resid_tag = h_tag;
      mid_tag = add(o);
      mid = c_h1;
    } else {
      const size_t off = static_cast<size_t>(li) * m->cap * m->KD;
      uint64_t* c_qg = cells(L.q.rows());
      uint64_t* c_k = cells(L.k.rows());
      uint64_t* c_v = cells(L.v.rows());
      PkStage a = {};
      if (!pk_gemv_stage(m, a, kPkGemv,
                         {{&L.q, nullptr, c_qg, kEpiStore},
                          {&L.k, nullptr, c_k, kEpiStore},
                          {&L.v, nullptr, c_v, kEpiStore}},
                         grid))
        return KIB_OK;
      a.prologue = kProRms;
      a.in = h_in;
      a.in_tag = h_tag;
      a.norm_w = L.attn_norm.f();
      const int a_tag = add(a);
      PkStage t = {};
      t.kind = kPkAttn;
      t.qg = c_qg;
      t.kp = c_k;
      t.vp = c_v;
      t.src_tag = a_tag;
      t.q_norm = L.q_norm.f();
      t.k_norm = L.k_norm.f();
      t.kcache = m->d_k + off;
      t.vcache = m->d_v + off;
      t.heads = m->heads;
      t.kv_heads = m->kvh;
      t.eps = m->eps;
      t.theta = m->theta;
      t.n_dims = n_dims;
      t.rope_freq = m->d_pk_rope;
      t.tk = m->d_pk_tmaps + 2 * li;
      t.tv = m->d_pk_tmaps + 2 * li + 1;
      t.nsplit = nsplit;
      t.part = cells(static_cast<size_t>(nsplit) * m->heads * (kHd + 2));
      const int t_tag = add(t);
      PkStage mg = t;
      mg.kind = kPkMerge;
      mg.src_tag = t_tag;
      mg.src2_tag = a_tag;
      mg.att_out = cells(static_cast<size_t>(m->heads) * kHd);
      const int mg_tag = add(mg);
      uint64_t* c_h1 = cells(m->H);
      PkStage o = {};
      if (!pk_gemv_stage(m, o, kPkGemv, {{&L.o, nullptr, c_h1, kEpiResidual}}, grid)) return KIB_OK;
      o.prologue = kProPlain;
      o.in = mg.att_out;
      o.in_tag = mg_tag;
      o.resid = h_in;
      o.resid_tag = h_tag;
      mid_tag = add(o);
      mid = c_h1;
    }
    uint64_t* c_act = cells(L.ffn_gate.rows());
    PkStage f = {};
    if (L.ffn_gate.type != L.ffn_up.type ||
        !pk_gemv_stage(m, f, kPkGemv, {{&L.ffn_gate, &L.ffn_up, c_act, kEpiSiluMul}}, grid)) {
      if (m->pk_why.empty()) m->pk_why = "ffn gate/up types differ";
      return KIB_OK;
    }
    f.prologue = kProRms;
    f.in = mid;
    f.in_tag = mid_tag;
    f.norm_w = L.post_norm.f();
    const int f_tag = add(f);
    uint64_t* c_h = cells(m->H);
    PkStage d = {};
    if (!pk_gemv_stage(m, d, kPkGemv, {{&L.ffn_down, nullptr, c_h, kEpiResidual}}, grid)) return KIB_OK;
    d.prologue = kProPlain;
    d.in = c_act;
    d.in_tag = f_tag;
    d.resid = mid;
    d.resid_tag = mid_tag;
    h_tag = add(d);
    h_in = c_h;
  }
  PkStage h = {};
  if (!pk_gemv_stage(m, h, kPkHead, {{&head_weight(m), nullptr, nullptr, kEpiArgmax}}, grid)) return KIB_OK;
  h.prologue = kProRms;
  h.in = h_in;
  h.in_tag = h_tag;
  h.norm_w = m->output_norm.f();
  add(h);
  if (st.size() > static_cast<size_t>(kPkMaxStages)) {
    m->pk_why = "more stages than the cell tags can name";
    return KIB_OK;
  }
  if (static_cast<size_t>(next_cell - m->d_pk_cells) > ncells) return fail(m, KIB_ERR_INTERNAL, "pk cell arena overrun");
  for (auto& S : st) S.eps = m->eps;
  if (cudaMalloc(&m->d_pk, st.size() * sizeof(PkStage)) != cudaSuccess) return fail(m, KIB_ERR_INTERNAL, "pk alloc");
  ENG_CUDA(cudaMemcpy(m->d_pk, st.data(), st.size() * sizeof(PkStage), cudaMemcpyHostToDevice));
  m->pk_n = static_cast<int>(st.size());
  m->pk_host = st;
  m->pk_grid = grid;
  m->pk_coop = coop != 0;
  ENG_CUDA(cudaFuncSetAttribute(decode_persistent_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                static_cast<int>(kPkSmemBytes)));
  m->pk_on = true;
  m->pk_why.clear();
  return KIB_OK;
}

// After an aborted step: clear the LM-head ticket and move the cell epoch on,
// so cells the aborted step wrote can never pass for the next step's.
static void pk_reset_after_error(kib_qwen35* m) {
  unsigned c[3] = {0u, 0u, 0u};
  cudaMemcpy(c, m->d_pk_ctr, sizeof(c), cudaMemcpyDeviceToHost);
  c[0] = 0u;
  c[1] = 0u;
  c[2] += 1u;
  cudaMemcpy(m->d_pk_ctr, c, sizeof(c), cudaMemcpyHostToDevice);
}

static PkProgram pk_program(kib_qwen35* m) {
  PkProgram P = {};
  P.stages = m->d_pk;
  P.nstages = m->pk_n;
  P.pos = m->d_pos;
  P.token = m->d_tokens;
  P.token_log = m->d_log;
  P.step = m->d_step;
  P.head_ctr = m->d_pk_ctr + 1;
  P.epoch = m->d_pk_ctr + 2;
  P.cand_max = m->d_pk_cmax;
  P.cand_idx = m->d_pk_cidx;
  P.err = m->ctx->d_err;
  P.trace = m->trace_on ? m->d_pk_trace : nullptr;
  return P;
}

static cudaError_t pk_launch(kib_qwen35* m, cudaStream_t st) {
  PkProgram P = pk_program(m);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(m->pk_grid);
  cfg.blockDim = dim3(kPkThreads);
  cfg.dynamicSmemBytes = kPkSmemBytes;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  int n = 0;
  if (pdl_enabled()) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  if (m->pk_coop) {
    attr[n].id = cudaLaunchAttributeCooperative;
    attr[n].val.cooperative = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, decode_persistent_kernel, P);
}

// The per-token graph of the persistent path: the embedding row gather, then
// the persistent decode kernel (programmatic dependent launch between them).
static int ensure_pk_graph(kib_qwen35* m) {
  if (m->pk_graph) return KIB_OK;
  auto body = [&](Enq& q) {
    q.run(get_rows_launch(m->tok_embd.type, m->tok_embd.p, m->V, m->H, m->d_tokens, 1, m->d_h, m->H, q.st), "embed");
    q.run(pk_launch(m, q.st), "decode_persistent");
  };
  int rc = capture(m, &m->pk_graph, body);
  if (rc && m->pk_coop) {  // the cooperative attribute is not accepted together with PDL on every driver
    cudaGetLastError();
    m->pk_coop = false;
    rc = capture(m, &m->pk_graph, body);
  }
  return rc;
}

// The one-token forward of kib_qwen35_forward as a single graph launch: the
// host-to-device copy of the step inputs (pinned h_pin[48..52]), the step, and
// the copies of the token (h_pin[32]) and of the error flag (h_pin[33]).
static int ensure_pk_fwd_graph(kib_qwen35* m) {
  if (m->pk_fwd_graph) return KIB_OK;
  int rc = ensure_pk_graph(m);  // settles the cooperative attribute
  if (rc) return rc;
  return capture(m, &m->pk_fwd_graph, [&](Enq& q) {
    q.run(cudaMemcpyAsync(m->d_io, m->h_pin + 48, 5 * sizeof(int), cudaMemcpyHostToDevice, q.st), "step_inputs");
    q.run(get_rows_launch(m->tok_embd.type, m->tok_embd.p, m->V, m->H, m->d_tokens, 1, m->d_h, m->H, q.st), "embed");
    q.run(pk_launch(m, q.st), "decode_persistent");
    q.run(cudaMemcpyAsync(m->h_pin + 32, m->d_log, sizeof(int), cudaMemcpyDeviceToHost, q.st), "token_out");
    q.run(cudaMemcpyAsync(m->h_pin + 33, m->ctx->d_err, sizeof(int), cudaMemcpyDeviceToHost, q.st), "err_out");
  });
}

int kib_qwen35_load(kib_ctx* ctx, const char* path, const kib_qwen35_options* opt, kib_qwen35** out) {
  if (!ctx || !path || !out) return KIB_ERR_INVALID_ARGUMENT;
  *out = nullptr;
  std::unique_ptr<kib_qwen35> mp(new kib_qwen35);
  kib_qwen35* m = mp.get();
  m->ctx = ctx;
  std::string err;
  m->gguf = GgufFile::open(path, &err);
  if (!m->gguf) return set_error(ctx, KIB_ERR_INVALID_ARGUMENT, err);
  const GgufFile& g = *m->gguf;
  const GgufValue* arch = g.meta("general.architecture");
  if (!arch || arch->str != "qwen35") return set_error(ctx, KIB_ERR_INVALID_ARGUMENT, "unsupported GGUF architecture");
  const std::string a = "qwen35.";
  // load_gguf_bundle hparams (model_config.cpp:808-856)
  m->H = static_cast<int>(g.num(a + "embedding_length", 0));
  m->I = static_cast<int>(g.num(a + "feed_forward_length", 0));
  const int total_layers = static_cast<int>(g.num(a + "block_count", 0));
  const int nextn = static_cast<int>(g.num(a + "nextn_predict_layers", 0));
  const int main_layers = total_layers - nextn;
  m->heads = static_cast<int>(g.num(a + "attention.head_count", 0));
  m->kvh = static_cast<int>(g.num(a + "attention.head_count_kv", 0));
  m->hd = static_cast<int>(g.num(a + "attention.key_length", 0));
  m->eps = static_cast<float>(g.num(a + "attention.layer_norm_rms_epsilon", 1e-6));
  m->theta = static_cast<float>(g.num(a + "rope.freq_base", 1e7));
  m->convk = static_cast<int>(g.num(a + "ssm.conv_kernel", 4));
  m->lhd = static_cast<int>(g.num(a + "ssm.state_size", 128));
  m->lkh = static_cast<int>(g.num(a + "ssm.group_count", 16));
  m->lvh = static_cast<int>(g.num(a + "ssm.time_step_rank", 16));
  const int interval = static_cast<int>(g.num(a + "full_attention_interval", 4));
  if (const GgufValue* s = g.meta(a + "rope.dimension_sections"); s && s->is_array)
    for (size_t i = 0; i < 4 && i < s->arr.size(); ++i) m->sections[i] = static_cast<int>(s->arr[i]);
  m->eos = static_cast<int64_t>(g.num("tokenizer.ggml.eos_token_id", -1));
  const GgufTensor* te = g.tensor("token_embd.weight");
  if (!te || te->shape.size() != 2) return set_error(ctx, KIB_ERR_INVALID_ARGUMENT, "missing Qwen3.5 GGUF tensor: token_embd.weight");
  m->V = static_cast<int>(te->shape[1]);
  if (m->H <= 0 || m->I <= 0 || main_layers <= 0 || main_layers > 64 || m->heads <= 0 || m->kvh <= 0 ||
      m->heads % m->kvh || m->heads / m->kvh != 4 || m->hd != 256 || m->lhd != 128 || m->lvh % m->lkh ||
      m->H % 256 || m->I % 256 || m->convk < 2 || m->convk > 8)
    return set_error(ctx, KIB_ERR_INVALID_ARGUMENT,
                     "Qwen3.5 hparams outside this backend's kernels (need head_dim 256, GQA 4, ssm state 128)");
  m->KD = m->kvh * m->hd;
  m->AD = m->heads * m->hd;
  m->VD = m->lvh * m->lhd;
  m->C = 2 * m->lkh * m->lhd + m->VD;

  // ---- upload every tensor, raw bytes as stored, 256-byte aligned with padding
  uint64_t total = 0;
  for (auto& t : g.tensors()) total += (t.bytes + 511) / 256 * 256;
  m->weight_bytes = total;
  if (cudaMalloc(&m->d_weights, total) != cudaSuccess) return set_error(ctx, KIB_ERR_INTERNAL, "weight allocation failed");
  std::map<std::string, DevT> dev;
  uint64_t off = 0;
  for (auto& t : g.tensors()) {
    DevT d;
    d.p = m->d_weights + off;
    d.type = static_cast<int>(t.type);
    d.shape = t.shape;
    if (cudaMemcpy(d.p, t.data, t.bytes, cudaMemcpyHostToDevice) != cudaSuccess)
      return set_error(ctx, KIB_ERR_INTERNAL, "weight upload failed: " + t.name);
    dev[t.name] = d;
    off += (t.bytes + 511) / 256 * 256;
  }
  // ---- weight map (qwen35_weight_map.cpp:61-454)
  const uint64_t H = static_cast<uint64_t>(m->H), I = static_cast<uint64_t>(m->I), V = static_cast<uint64_t>(m->V);
  const uint64_t hd = static_cast<uint64_t>(m->hd), AD = static_cast<uint64_t>(m->AD), KD = static_cast<uint64_t>(m->KD);
  const uint64_t C = static_cast<uint64_t>(m->C), VD = static_cast<uint64_t>(m->VD);
  const uint64_t lvh = static_cast<uint64_t>(m->lvh), lhd = static_cast<uint64_t>(m->lhd);
  int rc = bind(m, dev, "token_embd.weight", {H, V}, m->tok_embd);
  if (!rc) rc = bind(m, dev, "output_norm.weight", {H}, m->output_norm);
  if (!rc) rc = bind(m, dev, "output.weight", {H, V}, m->output, false);
  if (rc) return set_error(ctx, rc, m->err);
  auto kquant = [](const DevT& t) { return t.type == 12 || t.type == 13 || t.type == 14; };
  if (!kquant(m->tok_embd) || m->output_norm.type != 0 || (m->output.ok() && !kquant(m->output)))
    return set_error(ctx, KIB_ERR_INVALID_ARGUMENT, "token_embd/output must be K-quant and output_norm F32");
  int n_lin = 0, n_full = 0;
  auto bind_full = [&](int l, LayerW& L) {
    const std::string p = "blk." + std::to_string(l) + ".";
    int r = bind(m, dev, p + "attn_q.weight", {H, 2 * AD}, L.q);
    if (!r) r = bind(m, dev, p + "attn_k.weight", {H, KD}, L.k);
    if (!r) r = bind(m, dev, p + "attn_v.weight", {H, KD}, L.v);
    if (!r) r = bind(m, dev, p + "attn_output.weight", {AD, H}, L.o);
    if (!r) r = bind(m, dev, p + "attn_q_norm.weight", {hd}, L.q_norm);
    if (!r) r = bind(m, dev, p + "attn_k_norm.weight", {hd}, L.k_norm);
    return r;
  };
  auto bind_common = [&](int l, LayerW& L) {
    const std::string p = "blk." + std::to_string(l) + ".";
    int r = bind(m, dev, p + "attn_norm.weight", {H}, L.attn_norm);
    if (!r) r = bind(m, dev, p + "post_attention_norm.weight", {H}, L.post_norm);
    if (!r) r = bind(m, dev, p + "ffn_gate.weight", {H, I}, L.ffn_gate);
    if (!r) r = bind(m, dev, p + "ffn_down.weight", {I, H}, L.ffn_down);
    if (!r) r = bind(m, dev, p + "ffn_up.weight", {H, I}, L.ffn_up);
    return r;
  };
  for (int l = 0; l < main_layers; ++l) {
    LayerW L;
    const std::string p = "blk." + std::to_string(l) + ".";
    L.kind = ((l + 1) % interval) != 0 ? 0 : 1;
    rc = bind_common(l, L);
    if (!rc && L.kind == 1) {
      rc = bind_full(l, L);
      L.cache_index = n_full++;
    } else if (!rc) {
      rc = bind(m, dev, p + "attn_qkv.weight", {H, C}, L.qkv);
      if (!rc) rc = bind(m, dev, p + "attn_gate.weight", {H, VD}, L.zgate);
      if (!rc) rc = bind(m, dev, p + "ssm_conv1d.weight", {static_cast<uint64_t>(m->convk), C}, L.conv1d);
      if (!rc) rc = bind(m, dev, p + "ssm_dt.bias", {lvh}, L.dt_bias);
      if (!rc) rc = bind(m, dev, p + "ssm_a", {lvh}, L.ssm_a);
      if (!rc) rc = bind(m, dev, p + "ssm_beta.weight", {H, lvh}, L.beta);
      if (!rc) rc = bind(m, dev, p + "ssm_alpha.weight", {H, lvh}, L.alpha);
      if (!rc) rc = bind(m, dev, p + "ssm_norm.weight", {lhd}, L.ssm_norm);
      if (!rc) rc = bind(m, dev, p + "ssm_out.weight", {VD, H}, L.ssm_out);
      L.cache_index = n_lin++;
    }
    if (rc) return set_error(ctx, rc, m->err);
    m->layers.push_back(L);
  }
  m->has_mtp = nextn == 1 && (!opt || opt->enable_mtp);
  if (m->has_mtp) {
    LayerW& L = m->mtp;
    L.kind = 2;
    const std::string p = "blk." + std::to_string(main_layers) + ".";
    rc = bind_common(main_layers, L);
    if (!rc) rc = bind_full(main_layers, L);
    if (!rc) rc = bind(m, dev, p + "nextn.eh_proj.weight", {2 * H, H}, L.eh_proj);
    if (!rc) rc = bind(m, dev, p + "nextn.enorm.weight", {H}, L.enorm);
    if (!rc) rc = bind(m, dev, p + "nextn.hnorm.weight", {H}, L.hnorm);
    if (!rc) rc = bind(m, dev, p + "nextn.shared_head_norm.weight", {H}, L.shead_norm, false);
    if (rc) return set_error(ctx, rc, m->err);
  }
  // ---- execution plan (qwen35_runtime.cpp:4380-4526)
  const uint64_t context = opt && opt->context_tokens ? opt->context_tokens : 4096;
  const uint64_t decode = opt && opt->decode_tokens ? opt->decode_tokens : 1;
  m->cap = static_cast<int>(context + decode + 8);
  m->chunk = opt && opt->prefill_chunk_tokens ? static_cast<int>(opt->prefill_chunk_tokens) : 1024;
  m->tmax = std::max(m->chunk, kMaxSmallT);
  m->nsplit = std::max(1, std::min(64, (m->cap + 63) / 64));
  auto& P = m->plan;
  P.hidden_size = H;
  P.main_layers = static_cast<uint64_t>(main_layers);
  P.total_layers = static_cast<uint64_t>(total_layers);
  P.head_dim = hd;
  P.attention_heads = static_cast<uint64_t>(m->heads);
  P.kv_heads = static_cast<uint64_t>(m->kvh);
  P.linear_key_heads = static_cast<uint64_t>(m->lkh);
  P.linear_value_heads = lvh;
  P.linear_key_head_dim = lhd;
  P.linear_value_head_dim = lhd;
  P.linear_inner_size = VD;
  P.linear_conv_kernel = static_cast<uint64_t>(m->convk);
  P.linear_conv_channels = C;
  P.intermediate_size = I;
  P.vocab_size = V;
  P.attention_capacity_tokens = static_cast<uint64_t>(m->cap);
  P.full_attention_layers = static_cast<uint64_t>(n_full);
  P.linear_attention_layers = static_cast<uint64_t>(n_lin);
  P.kv_dim = KD;
  P.recurrent_r_elements_per_layer = C * static_cast<uint64_t>(m->convk - 1);
  P.recurrent_s_elements_per_layer = lvh * lhd * lhd;
  P.kv_cache_bytes = 2ull * n_full * m->cap * KD * 2;
  P.recurrent_r_cache_bytes = static_cast<uint64_t>(n_lin) * P.recurrent_r_elements_per_layer * 4;
  P.recurrent_s_cache_bytes = static_cast<uint64_t>(n_lin) * P.recurrent_s_elements_per_layer * 4;
  P.total_cache_bytes = P.kv_cache_bytes + P.recurrent_r_cache_bytes + P.recurrent_s_cache_bytes;
  P.weight_bytes = total;
  P.mtp_layers = m->has_mtp ? 1 : 0;
  for (int l = 0; l < main_layers; ++l) P.layer_kinds[l] = m->layers[l].kind;
  // ---- caches + activations (allocate_qwen35_metal_cache, qwen35_runtime.cpp:1252-1330)
  m->k_elems = static_cast<size_t>(n_full) * m->cap * m->KD;
  m->r_elems = static_cast<size_t>(n_lin) * P.recurrent_r_elements_per_layer;
  m->s_elems = static_cast<size_t>(n_lin) * P.recurrent_s_elements_per_layer;
  m->mk_elems = m->has_mtp ? static_cast<size_t>(m->cap) * m->KD : 0;
  const size_t T = static_cast<size_t>(m->tmax);
  bool ok = dalloc(&m->d_k, m->k_elems) == cudaSuccess && dalloc(&m->d_v, m->k_elems) == cudaSuccess &&
            dalloc(&m->d_r, m->r_elems) == cudaSuccess && dalloc(&m->d_s, m->s_elems) == cudaSuccess &&
            dalloc(&m->d_r_snap, m->r_elems) == cudaSuccess && dalloc(&m->d_s_snap, m->s_elems) == cudaSuccess &&
            dalloc(&m->d_mk, m->mk_elems) == cudaSuccess && dalloc(&m->d_mv, m->mk_elems) == cudaSuccess &&
            dalloc(&m->d_pending_h, H) == cudaSuccess && dalloc(&m->d_h, T * H) == cudaSuccess &&
            dalloc(&m->d_h1, T * H) == cudaSuccess && dalloc(&m->d_qkv, T * C) == cudaSuccess &&
            dalloc(&m->d_z, T * VD) == cudaSuccess && dalloc(&m->d_beta, T * lvh) == cudaSuccess &&
            dalloc(&m->d_alpha, T * lvh) == cudaSuccess && dalloc(&m->d_y, T * VD) == cudaSuccess &&
            dalloc(&m->d_act, T * I) == cudaSuccess && dalloc(&m->d_act2, T * I) == cudaSuccess &&
            dalloc(&m->d_qg, T * 2 * AD) == cudaSuccess && dalloc(&m->d_kp, T * KD) == cudaSuccess &&
            dalloc(&m->d_vp, T * KD) == cudaSuccess && dalloc(&m->d_att, T * AD) == cudaSuccess &&
            dalloc(&m->d_qout, T * AD) == cudaSuccess && dalloc(&m->d_norm, T * 2 * H) == cudaSuccess &&
            dalloc(&m->d_norm2, T * VD) == cudaSuccess && dalloc(&m->d_hn, T * H) == cudaSuccess &&
            dalloc(&m->d_logits, static_cast<size_t>(kMaxSmallT) * V) == cudaSuccess &&
            dalloc(&m->d_e, T * H) == cudaSuccess && dalloc(&m->d_cat, T * 2 * H) == cudaSuccess &&
            dalloc(&m->d_hm, T * H) == cudaSuccess && dalloc(&m->d_hm1, T * H) == cudaSuccess &&
            dalloc(&m->d_mtp_h, T * H) == cudaSuccess &&
            dalloc(&m->d_w16, std::max<uint64_t>({C, 2 * AD, I, VD, H, KD}) * std::max<uint64_t>({H, I, VD, AD})) ==
                cudaSuccess &&
            dalloc(&m->d_x16, T * std::max<uint64_t>({2 * H, I, VD, AD})) == cudaSuccess &&
            dalloc(&m->d_gdn_ws, static_cast<size_t>(lvh) * ((T + kGc - 1) / kGc) * kGcWs) == cudaSuccess &&
            dalloc(&m->d_part, static_cast<size_t>(m->nsplit) * kMaxSmallT * m->heads * (kHd + 2)) == cudaSuccess &&
            dalloc(&m->d_fa_part, static_cast<size_t>(kFa2MaxSplits) * T * m->heads * (kHd + 2)) == cudaSuccess &&
            dalloc(&m->d_proj, T * std::max<uint64_t>({C + VD + 2 * lvh, 2 * I, 2 * AD + 2 * KD})) == cudaSuccess &&
            dalloc(&m->d_attn_cnt, 64) == cudaSuccess && dalloc(&m->d_head_cnt, 4) == cudaSuccess &&
            dalloc(&m->d_cand_max, 1024 * kGemvMaxTok) == cudaSuccess &&
            dalloc(&m->d_cand_sum, 1024 * kGemvMaxTok) == cudaSuccess &&
            dalloc(&m->d_cand_idx, 1024 * kGemvMaxTok) == cudaSuccess && dalloc(&m->d_io, T + 8) == cudaSuccess &&
            dalloc(&m->d_mtp_pos, 4) == cudaSuccess && 
            dalloc(&m->d_argmax, kMaxSmallT) == cudaSuccess && dalloc(&m->d_prob, 4096) == cudaSuccess &&
            dalloc(&m->d_log, 1 << 20) == cudaSuccess && 
            dalloc(&m->d_mtp_tok, 4) == cudaSuccess &&
            cudaMallocHost(&m->h_pin, 4096 * sizeof(int)) == cudaSuccess &&
            cudaMallocHost(&m->h_pinf, 4096 * sizeof(float)) == cudaSuccess;
  if (ok) {
    m->d_pos = m->d_io;
    m->d_step = m->d_io + 1;
    m->d_tokens = m->d_io + 4;
  }
  if (!ok) {
    kib_qwen35_free(mp.release());
    return set_error(ctx, KIB_ERR_INTERNAL, "cache/activation allocation failed");
  }
  cudaMemset(m->d_attn_cnt, 0, 64 * sizeof(unsigned));
  // Resident f16 copies of the prefill GEMM weights (each value as the GEMM
  // rounds it), made once here so prefill GEMMs stream f16 tiles directly;
  // only when they take under a quarter of the free device memory
  // (KIB_PREFILL_F16_WEIGHTS=0 turns them off: per-call dequantization).
  if (const char* ev = std::getenv("KIB_PREFILL_F16_WEIGHTS"); !ev || ev[0] != '0') {
    std::vector<DevT*> ws;
    auto add = [&](LayerW& L) {
      for (DevT* d : {&L.qkv, &L.zgate, &L.beta, &L.alpha, &L.ssm_out, &L.q, &L.k, &L.v, &L.o, &L.ffn_gate, &L.ffn_up,
                      &L.ffn_down, &L.eh_proj})
        if (d->ok() && (d->type == kTypeQ4K || d->type == kTypeQ5K || d->type == kTypeQ6K) && d->cols() % 256 == 0)
          ws.push_back(d);
    };
    for (LayerW& L : m->layers) add(L);
    if (m->has_mtp) add(m->mtp);
    auto bytes = [](const DevT* d) {
      return (static_cast<size_t>(d->rows()) * d->cols() * 2 + 255) & ~static_cast<size_t>(255);
    };
    size_t total = 0;
    for (DevT* d : ws) total += bytes(d);
    size_t free_b = 0, total_b = 0;
    if (!ws.empty() && cudaMemGetInfo(&free_b, &total_b) == cudaSuccess && total < free_b / 4 &&
        cudaMalloc(&m->d_w16_all, total) == cudaSuccess) {
      size_t off = 0;
      cudaError_t e2 = cudaSuccess;
      for (DevT* d : ws) {
        d->h = reinterpret_cast<__half*>(static_cast<uint8_t*>(m->d_w16_all) + off);
        off += bytes(d);
        if (e2 == cudaSuccess)
          e2 = kquant_to_f16_launch(d->type, d->p, d->rows(), d->cols(), d->h, ctx->num_sms, ctx->stream);
      }
      if (e2 == cudaSuccess) e2 = cudaStreamSynchronize(ctx->stream);
      if (e2 != cudaSuccess) {
        for (DevT* d : ws) d->h = nullptr;
        cudaFree(m->d_w16_all);
        m->d_w16_all = nullptr;
        cudaGetLastError();
      }
    }
  }
  if (const char* tr = std::getenv("KIB_TRACE"); tr && tr[0] == '1') {
    m->trace_on = cudaMalloc(&m->d_trace, 4096 * 8 * sizeof(unsigned long long)) == cudaSuccess;
  }
  cudaMemset(m->d_head_cnt, 0, 4 * sizeof(unsigned));
  if (dalloc(&m->d_pk_ctr, 4) != cudaSuccess ||
      dalloc(&m->d_pk_cmax, 1024) != cudaSuccess ||
      dalloc(&m->d_pk_cidx, 1024) != cudaSuccess || dalloc(&m->d_pk_trace, 16 * 4096) != cudaSuccess) {
    kib_qwen35_free(mp.release());
    return set_error(ctx, KIB_ERR_INTERNAL, "persistent decode allocation failed");
  }
  cudaMemset(m->d_pk_ctr, 0, 4 * sizeof(unsigned));
  if (build_pk(m) != KIB_OK) {
    std::string why = m->err;
    kib_qwen35_free(mp.release());
    return set_error(ctx, KIB_ERR_INTERNAL, "persistent decode set-up failed: " + why);
  }
  *out = mp.release();
  return kib_qwen35_reset(*out);
}

void kib_qwen35_free(kib_qwen35* m) {
  if (!m) return;
  if (m->ctx && m->ctx->stream) cudaStreamSynchronize(m->ctx->stream);
  for (auto& g : m->fwd_graph)
    if (g) cudaGraphExecDestroy(g);
  if (m->decode_graph) cudaGraphExecDestroy(m->decode_graph);
  if (m->mtp_graph) cudaGraphExecDestroy(m->mtp_graph);
  if (m->pk_graph) cudaGraphExecDestroy(m->pk_graph);
  if (m->pk_fwd_graph) cudaGraphExecDestroy(m->pk_fwd_graph);
  void* pk_ptrs[] = {m->d_pk, m->d_pk_ctr, m->d_pk_cells, m->d_pk_rope, m->d_pk_cmax, m->d_pk_cidx, m->d_pk_trace,
                     m->d_pk_tmaps};
  for (void* p : pk_ptrs)
    if (p) cudaFree(p);
  void* ptrs[] = {m->d_weights, m->d_k, m->d_v, m->d_mk, m->d_mv, m->d_r, m->d_s, m->d_r_snap, m->d_s_snap,
                  m->d_pending_h, m->d_h, m->d_h1, m->d_qkv, m->d_z, m->d_beta, m->d_alpha, m->d_y, m->d_act,
                  m->d_act2, m->d_qg, m->d_kp, m->d_vp, m->d_att, m->d_qout, m->d_norm, m->d_norm2, m->d_hn,
                  m->d_logits, m->d_e, m->d_cat, m->d_hm, m->d_hm1, m->d_mtp_h, m->d_part, m->d_fa_part, m->d_proj, m->d_attn_cnt,
                  m->d_head_cnt, m->d_cand_max, m->d_cand_sum, m->d_cand_idx, m->d_io, m->d_mtp_pos,
                  m->d_argmax, m->d_prob, m->d_log, m->d_mtp_tok, m->d_trace,
                  m->d_w16, m->d_x16, m->d_w16_all, m->d_gdn_ws};
  for (void* p : ptrs)
    if (p) cudaFree(p);
  if (m->h_pin) cudaFreeHost(m->h_pin);
  if (m->h_pinf) cudaFreeHost(m->h_pinf);
  delete m;
}

int kib_qwen35_get_plan(const kib_qwen35* m, kib_qwen35_plan* plan) {
  if (!m || !plan) return KIB_ERR_INVALID_ARGUMENT;
  *plan = m->plan;
  return KIB_OK;
}

int kib_qwen35_reset(kib_qwen35* m) {
  if (!m) return KIB_ERR_INVALID_ARGUMENT;
  cudaStream_t st = m->ctx->stream;
  ENG_CUDA(cudaMemsetAsync(m->d_k, 0, m->k_elems * 2, st));
  ENG_CUDA(cudaMemsetAsync(m->d_v, 0, m->k_elems * 2, st));
  ENG_CUDA(cudaMemsetAsync(m->d_r, 0, m->r_elems * 4, st));
  ENG_CUDA(cudaMemsetAsync(m->d_s, 0, m->s_elems * 4, st));
  if (m->mk_elems) {
    ENG_CUDA(cudaMemsetAsync(m->d_mk, 0, m->mk_elems * 2, st));
    ENG_CUDA(cudaMemsetAsync(m->d_mv, 0, m->mk_elems * 2, st));
  }
  ENG_CUDA(cudaMemsetAsync(m->d_pending_h, 0, static_cast<size_t>(m->H) * 4, st));
  ENG_CUDA(cudaMemsetAsync(m->d_step, 0, 4, st));
  m->pos = 0;
  return set_pos(m, m->d_pos, 0);
}

uint64_t kib_qwen35_position(const kib_qwen35* m) { return m ? m->pos : 0; }

int kib_qwen35_persistent_stages(const kib_qwen35* m, char* why, int why_len) {
  if (!m) return 0;
  if (why && why_len > 0) {
    std::strncpy(why, m->pk_on ? "" : m->pk_why.c_str(), static_cast<size_t>(why_len - 1));
    why[why_len - 1] = 0;
  }
  return m->pk_on ? m->pk_n : 0;
}

int kib_qwen35_debug_stall(kib_qwen35* m, uint32_t poll_limit, int stage) {
  if (!m) return KIB_ERR_INVALID_ARGUMENT;
  if (!m->pk_on) return fail(m, KIB_ERR_UNAVAILABLE, "debug_stall: the persistent decode kernel is not in use");
  if (stage >= m->pk_n) return fail(m, KIB_ERR_INVALID_ARGUMENT, "debug_stall: no such stage");
  std::vector<PkStage> st = m->pk_host;
  if (stage >= 0) {
    PkStage& S = st[static_cast<size_t>(stage)];
    if (S.kind != kPkGemv || S.in_tag == 0)
      return fail(m, KIB_ERR_INVALID_ARGUMENT, "debug_stall: the stage must be a GEMV reading cells");
    S.in_tag = 255;  // no stage writes tag 255: the input never arrives
  }
  const uint32_t limit = poll_limit ? poll_limit : kPkPollLimit;
  ENG_CUDA(cudaStreamSynchronize(m->ctx->stream));
  ENG_CUDA(cudaMemcpyToSymbol(g_pk_poll_limit, &limit, sizeof(limit)));
  ENG_CUDA(cudaMemcpy(m->d_pk, st.data(), st.size() * sizeof(PkStage), cudaMemcpyHostToDevice));
  return KIB_OK;
}

int kib_qwen35_set_position(kib_qwen35* m, uint64_t position) {
  if (!m || position >= static_cast<uint64_t>(m->cap)) return KIB_ERR_INVALID_ARGUMENT;
  m->pos = position;
  return set_pos(m, m->d_pos, position);
}

// Token ids must name embedding rows (qwen35_runtime.cpp:1575-1578 rejects
// the others as invalid arguments).
static int check_tokens(kib_qwen35* m, const int32_t* t, uint64_t n) {
  for (uint64_t i = 0; i < n; ++i)
    if (t[i] < 0 || t[i] >= m->V) return fail(m, KIB_ERR_INVALID_ARGUMENT, "Qwen3.5 token id is outside embedding rows");
  return KIB_OK;
}

// position, step counter 0 and the token of a decode step: one copy into d_io
static cudaError_t put_step_inputs(kib_qwen35* m, int32_t token, cudaStream_t st) {
  int* h = m->h_pin + 48;
  h[0] = static_cast<int>(m->pos);
  h[1] = 0;
  h[2] = h[3] = 0;
  h[4] = token;
  return cudaMemcpyAsync(m->d_io, h, 5 * sizeof(int), cudaMemcpyHostToDevice, st);
}

int kib_qwen35_forward(kib_qwen35* m, const int32_t* tokens, uint64_t n, int advance, int32_t* argmax_out,
                       float* logits, float* normed_hidden) {
  if (!m || !tokens || n < 1 || n > kMaxSmallT) return KIB_ERR_INVALID_ARGUMENT;
  if (m->pos + n > static_cast<uint64_t>(m->cap)) return fail(m, KIB_ERR_INVALID_ARGUMENT, "forward exceeds cache capacity");
  if (int rc = check_tokens(m, tokens, n)) return rc;
  cudaStream_t st = m->ctx->stream;
  if (n == 1 && !logits && !normed_hidden && m->pk_on) {
    // one token, argmax only: the persistent decode path (its head writes the
    // argmax to the token log and advances the device position)
    int rc = ensure_pk_fwd_graph(m);
    if (rc) return rc;
    int* h = m->h_pin + 48;  // step inputs, read by the graph's first node
    h[0] = static_cast<int>(m->pos);
    h[1] = 0;
    h[2] = h[3] = 0;
    h[4] = tokens[0];
    // one launch: inputs in, the step, token and error flag out (the flag
    // travels with the token instead of a blocking copy after the sync)
    ENG_CUDA(cudaGraphLaunch(m->pk_fwd_graph, st));
    rc = sync_check_flag(m, "forward", m->h_pin + 33);
    if (rc) {
      pk_reset_after_error(m);
      return rc;
    }
    if (argmax_out) argmax_out[0] = m->h_pin[32];
    if (advance) m->pos += 1;
    return KIB_OK;
  }
  std::memcpy(m->h_pin + 16, tokens, n * sizeof(int32_t));
  m->h_pin[0] = static_cast<int>(m->pos);
  ENG_CUDA(cudaMemcpyAsync(m->d_pos, m->h_pin, sizeof(int), cudaMemcpyHostToDevice, st));
  ENG_CUDA(cudaMemcpyAsync(m->d_tokens, m->h_pin + 16, n * sizeof(int), cudaMemcpyHostToDevice, st));
  int rc = forward_small(m, static_cast<int>(n), logits != nullptr);
  if (rc) return rc;
  if (argmax_out) ENG_CUDA(cudaMemcpyAsync(m->h_pin + 32, m->d_argmax, n * sizeof(int), cudaMemcpyDeviceToHost, st));
  if (logits)
    ENG_CUDA(cudaMemcpyAsync(logits, m->d_logits, n * static_cast<size_t>(m->V) * 4, cudaMemcpyDeviceToHost, st));
  if (normed_hidden)
    ENG_CUDA(cudaMemcpyAsync(normed_hidden, m->d_hn, n * static_cast<size_t>(m->H) * 4, cudaMemcpyDeviceToHost, st));
  rc = sync_check(m, "forward");
  if (rc) return rc;
  if (argmax_out) std::memcpy(argmax_out, m->h_pin + 32, n * sizeof(int32_t));
  if (advance) m->pos += n;
  return KIB_OK;
}

int kib_qwen35_prefill(kib_qwen35* m, const int32_t* tokens, uint64_t n, uint64_t chunk, int32_t* next_token) {
  if (!m || !tokens || n == 0) return KIB_ERR_INVALID_ARGUMENT;
  if (m->pos + n > static_cast<uint64_t>(m->cap)) return fail(m, KIB_ERR_INVALID_ARGUMENT, "prefill exceeds cache capacity");
  if (int rc = check_tokens(m, tokens, n)) return rc;
  if (chunk == 0) chunk = static_cast<uint64_t>(m->chunk);
  if (chunk > static_cast<uint64_t>(m->tmax)) chunk = static_cast<uint64_t>(m->tmax);
  cudaStream_t st = m->ctx->stream;
  std::vector<int32_t> staging;
  for (uint64_t s = 0; s < n; s += chunk) {
    const uint64_t T = std::min<uint64_t>(chunk, n - s);
    const bool last = s + T == n;
    m->h_pin[0] = static_cast<int>(m->pos);
    ENG_CUDA(cudaMemcpyAsync(m->d_pos, m->h_pin, sizeof(int), cudaMemcpyHostToDevice, st));
    ENG_CUDA(cudaMemcpyAsync(m->d_tokens, tokens + s, T * sizeof(int32_t), cudaMemcpyHostToDevice, st));
    int rc;
    if (T <= static_cast<uint64_t>(kMaxSmallT)) {
      rc = forward_small(m, static_cast<int>(T), false);
    } else {
      rc = forward_prefill(m, static_cast<int>(T), last);
    }
    if (rc) return rc;
    if (m->has_mtp) {
      // MTP layer over the chunk (qwen35_runtime.cpp:5894-5961): normed rows,
      // shifted by one with pending_h in front.
      Enq q{m, st};
      if (T > static_cast<uint64_t>(kMaxSmallT))
        q.run(rms_rows_launch(m->d_h, m->output_norm.f(), static_cast<int>(T), m->H, m->eps, m->d_hn, st), "norm_rows");
      // shifted rows: [pending_h, normed rows 0..T-2]
      q.run(cudaMemcpyAsync(m->d_norm, m->d_pending_h, static_cast<size_t>(m->H) * 4, cudaMemcpyDeviceToDevice, st),
            "shift");
      if (T > 1)
        q.run(cudaMemcpyAsync(m->d_norm + m->H, m->d_hn, (T - 1) * static_cast<size_t>(m->H) * 4,
                              cudaMemcpyDeviceToDevice, st),
              "shift");
      q.run(cudaMemcpyAsync(m->d_pending_h, m->d_hn + (T - 1) * static_cast<size_t>(m->H),
                            static_cast<size_t>(m->H) * 4, cudaMemcpyDeviceToDevice, st),
            "pending_h");
      q.run(cudaMemcpyAsync(m->d_mtp_pos, m->d_pos, sizeof(int), cudaMemcpyDeviceToDevice, st), "mtp_pos");
      mtp_enqueue(q, static_cast<int>(T), m->d_tokens, m->d_norm, false, nullptr, nullptr, nullptr, nullptr, nullptr);
      if (!q.ok()) return fail(m, KIB_ERR_INTERNAL, "mtp prefill: " + q.why);
    }
    m->pos += T;
    if (last && next_token) {
      // the small path's head ran over all T rows; the last row's argmax is the sample
      const int row = T <= static_cast<uint64_t>(kMaxSmallT) ? static_cast<int>(T) - 1 : 0;
      ENG_CUDA(cudaMemcpyAsync(m->h_pin + 32, m->d_argmax + row, sizeof(int), cudaMemcpyDeviceToHost, st));
    }
    int rc2 = sync_check(m, "prefill");
    if (rc2) return rc2;
    if (last && next_token) *next_token = m->h_pin[32];
  }
  return KIB_OK;
}

int kib_qwen35_decode_greedy(kib_qwen35* m, int32_t first_token, uint64_t steps, int32_t* tokens_out) {
  if (!m || steps == 0) return KIB_ERR_INVALID_ARGUMENT;
  if (m->pos + steps > static_cast<uint64_t>(m->cap)) return fail(m, KIB_ERR_INVALID_ARGUMENT, "decode exceeds cache capacity");
  if (steps > (1u << 20)) return KIB_ERR_INVALID_ARGUMENT;
  if (int rc = check_tokens(m, &first_token, 1)) return rc;
  cudaStream_t st = m->ctx->stream;
  const bool use_pk = m->pk_on;
  if (use_pk) {
    int rc = ensure_pk_graph(m);
    if (rc) return rc;
  }
  if (!use_pk && !m->decode_graph) {
    int rc = capture(m, &m->decode_graph, [&](Enq& q) {
      q.run(get_rows_launch(m->tok_embd.type, m->tok_embd.p, m->V, m->H, m->d_tokens, 1, m->d_h, m->H, q.st), "embed");
      main_layers_small(q, 1, m->d_pos);
      head_small(q, 1, m->d_h, m->output_norm, head_weight(m), m->d_tokens, nullptr, nullptr, nullptr, m->d_log,
                 m->d_step, m->d_pos);
    }, true);
    if (rc) return rc;
  }
  if (m->trace_on && m->d_trace) ENG_CUDA(cudaMemsetAsync(m->d_trace, 0, 4096 * 8 * sizeof(unsigned long long), st));
  if (m->trace_on && m->d_pk_trace) ENG_CUDA(cudaMemsetAsync(m->d_pk_trace, 0, 16 * 4096 * sizeof(unsigned long long), st));
  ENG_CUDA(put_step_inputs(m, first_token, st));
  cudaGraphExec_t g = use_pk ? m->pk_graph : m->decode_graph;
  for (uint64_t i = 0; i < steps; ++i) ENG_CUDA(cudaGraphLaunch(g, st));
  if (tokens_out) ENG_CUDA(cudaMemcpyAsync(tokens_out, m->d_log, steps * sizeof(int32_t), cudaMemcpyDeviceToHost, st));
  int rc = sync_check(m, "decode");
  if (rc) {
    if (use_pk) pk_reset_after_error(m);  // an aborted step leaves its ticket and epoch behind
    return rc;
  }
  m->pos += steps;
  if (use_pk && m->trace_on) {
    // stage start times of CTA 0 in the last step: CSV to $KIB_TRACE_OUT
    std::vector<unsigned long long> h(16 * m->pk_n + 16);
    std::vector<PkStage> stages(m->pk_n);
    cudaMemcpy(h.data(), m->d_pk_trace, h.size() * 8, cudaMemcpyDeviceToHost);
    cudaMemcpy(stages.data(), m->d_pk, stages.size() * sizeof(PkStage), cudaMemcpyDeviceToHost);
    const char* path = std::getenv("KIB_TRACE_OUT");
    FILE* f = path ? std::fopen(path, "w") : nullptr;
    if (f) {
      static const char* names[] = {"gemv", "gdn", "attn", "merge", "head"};
      auto rel = [&](unsigned long long v) { return v ? static_cast<long long>(v - h[0]) : -1ll; };
      std::fprintf(f, "stage,kind,type,rows,cols,start_ns,prologue_ns,first_tile_ns,done_ns,next_ns,max_done_ns,"
                      "prod_stage_ns,prod_issue_ns,ux_ns,p8,p9,p10,p11,p12,p13\n");
      for (int i = 0; i < m->pk_n; ++i) {
        const unsigned long long* t = h.data() + 16 * i;
        std::fprintf(f, "%d,%s,%d,%d,%d", i, names[stages[i].kind], stages[i].type, stages[i].rows, stages[i].cols);
        const int order[] = {0, 1, 2, 3, 16, 5, 6, 7, 4, 8, 9, 10, 11, 12, 13};
        for (int k : order) std::fprintf(f, ",%lld", rel(t[k]));
        std::fprintf(f, "\n");
      }
      std::fclose(f);
    }
    if (const char* p2 = std::getenv("KIB_TRACE_OUT2")) {
      // per-tile times of the LM head on CTA 0: wait start, taken, dots done, released
      std::vector<unsigned long long> t(4 * 500);
      cudaMemcpy(t.data(), m->d_pk_trace + 8192, t.size() * 8, cudaMemcpyDeviceToHost);
      if (FILE* f2 = std::fopen(p2, "w")) {
        for (int j = 0; j < 500 && t[4 * j]; ++j) {
          std::fprintf(f2, "%d", j);
          for (int q = 0; q < 4; ++q) std::fprintf(f2, ",%lld", t[4 * j + q] ? (long long)(t[4 * j + q] - h[0]) : -1ll);
          std::fprintf(f2, "\n");
        }
        std::fclose(f2);
      }
    }
  }
  if (!use_pk && m->trace_on && m->d_trace && m->trace_used > 0) {
    // timeline of the last replayed step(s) merged: CSV to $KIB_TRACE_OUT
    std::vector<unsigned long long> h(8 * static_cast<size_t>(m->trace_used));
    cudaMemcpy(h.data(), m->d_trace, h.size() * 8, cudaMemcpyDeviceToHost);
    const char* path = std::getenv("KIB_TRACE_OUT");
    FILE* f = path ? std::fopen(path, "w") : nullptr;
    if (f) {
      unsigned long long t0 = ~0ull;
      for (int i = 0; i < m->trace_used; ++i) t0 = std::min(t0, ~h[8 * i]);
      auto rel = [&](unsigned long long v) { return v == 0 ? 0ull : v - t0; };
      std::fprintf(f, "idx,kernel,first_entry_ns,first_past_wait_ns,last_past_wait_ns,last_exit_ns,last_entry_ns,"
                      "last_tile_ready_ns,last_prologue_done_ns\n");
      for (int i = 0; i < m->trace_used; ++i)
        std::fprintf(f, "%d,%s,%llu,%llu,%llu,%llu,%llu,%llu,%llu\n", i, m->trace_names[i].c_str(), ~h[8 * i] - t0,
                     ~h[8 * i + 3] - t0, rel(h[8 * i + 1]), rel(h[8 * i + 2]), rel(h[8 * i + 4]), rel(h[8 * i + 5]),
                     rel(h[8 * i + 6]));
      std::fclose(f);
    }
  }
  return KIB_OK;
}

int kib_qwen35_state_io(kib_qwen35* m, int into, uint16_t* k, uint16_t* v, float* r, float* s, uint16_t* mk,
                        uint16_t* mv, float* ph) {
  if (!m) return KIB_ERR_INVALID_ARGUMENT;
  auto io = [&](void* dev, void* host, size_t bytes) -> cudaError_t {
    if (!host || bytes == 0) return cudaSuccess;
    return into ? cudaMemcpy(dev, host, bytes, cudaMemcpyHostToDevice) : cudaMemcpy(host, dev, bytes, cudaMemcpyDeviceToHost);
  };
  cudaStreamSynchronize(m->ctx->stream);
  ENG_CUDA(io(m->d_k, k, m->k_elems * 2));
  ENG_CUDA(io(m->d_v, v, m->k_elems * 2));
  ENG_CUDA(io(m->d_r, r, m->r_elems * 4));
  ENG_CUDA(io(m->d_s, s, m->s_elems * 4));
  ENG_CUDA(io(m->d_mk, mk, m->mk_elems * 2));
  ENG_CUDA(io(m->d_mv, mv, m->mk_elems * 2));
  ENG_CUDA(io(m->d_pending_h, ph, static_cast<size_t>(m->H) * 4));
  return KIB_OK;
}

int kib_qwen35_mtp_forward(kib_qwen35* m, const int32_t* tokens, const float* h_rows, uint64_t n, uint64_t position,
                           int32_t* argmax_out, float* h_nextn_out) {
  if (!m || !tokens || !h_rows || n < 1 || n > kMaxSmallT) return KIB_ERR_INVALID_ARGUMENT;
  if (!m->has_mtp) return fail(m, KIB_ERR_UNAVAILABLE, "model has no MTP/NextN layer");
  if (int rc = check_tokens(m, tokens, n)) return rc;
  cudaStream_t st = m->ctx->stream;
  std::memcpy(m->h_pin + 16, tokens, n * sizeof(int32_t));
  m->h_pin[0] = static_cast<int>(position);
  ENG_CUDA(cudaMemcpyAsync(m->d_mtp_pos, m->h_pin, sizeof(int), cudaMemcpyHostToDevice, st));
  ENG_CUDA(cudaMemcpyAsync(m->d_tokens, m->h_pin + 16, n * sizeof(int), cudaMemcpyHostToDevice, st));
  ENG_CUDA(cudaMemcpyAsync(m->d_norm, h_rows, n * static_cast<size_t>(m->H) * 4, cudaMemcpyHostToDevice, st));
  Enq q{m, st};
  mtp_enqueue(q, static_cast<int>(n), m->d_tokens, m->d_norm, true, m->d_argmax, nullptr, nullptr, nullptr, nullptr);
  if (!q.ok()) return fail(m, KIB_ERR_INTERNAL, "mtp forward: " + q.why);
  if (argmax_out) ENG_CUDA(cudaMemcpyAsync(m->h_pin + 32, m->d_argmax, n * sizeof(int), cudaMemcpyDeviceToHost, st));
  if (h_nextn_out)
    ENG_CUDA(cudaMemcpyAsync(h_nextn_out, m->d_mtp_h, n * static_cast<size_t>(m->H) * 4, cudaMemcpyDeviceToHost, st));
  int rc = sync_check(m, "mtp_forward");
  if (rc) return rc;
  if (argmax_out) std::memcpy(argmax_out, m->h_pin + 32, n * sizeof(int32_t));
  return KIB_OK;
}

// generate_qwen35_metal (qwen35_runtime.cpp:5239-6714), greedy decoding.
int kib_qwen35_prefill_cached(kib_qwen35* m, kib_qwen35_prefix_cache* cache, const int32_t* tokens, uint64_t count,
                              int32_t* next_token, uint64_t* hit_tokens);

// The generate loop behind kib_generate_qwen35 and its streaming form: every
// committed token goes through emit (cb may cancel), and the prompt is
// prefilled through the host prefix cache when one is given.
static int generate_impl(kib_qwen35* m, const kib_generation_request* rq, kib_qwen35_prefix_cache* cache,
                         kib_token_callback cb, void* user, int32_t* out, uint64_t cap_out, kib_generation_result* res,
                         uint64_t* cached_tokens) {
  if (!m || !rq || !rq->prompt_tokens || rq->prompt_count == 0 || !res) return KIB_ERR_INVALID_ARGUMENT;
  std::memset(res, 0, sizeof(*res));
  if (cached_tokens) *cached_tokens = 0;
  bool cancelled = false;
  if (int rc = check_tokens(m, rq->prompt_tokens, rq->prompt_count)) return rc;
  const uint64_t max_new = std::min<uint64_t>(rq->max_new_tokens, cap_out);
  if (rq->prompt_count + max_new + 8 > static_cast<uint64_t>(m->cap))
    return fail(m, KIB_ERR_INVALID_ARGUMENT, "prompt + max_new_tokens exceeds the attention capacity");
  auto is_eos = [&](int64_t t) {
    if (rq->ignore_eos) return false;
    return t == kQwenEndOfText || t == m->eos ||
           (rq->eos_token_id != UINT64_MAX && static_cast<uint64_t>(t) == rq->eos_token_id);
  };
  cudaEvent_t e0, e1, e2;
  cudaEventCreate(&e0);
  cudaEventCreate(&e1);
  cudaEventCreate(&e2);
  cudaStream_t st = m->ctx->stream;
  int rc = kib_qwen35_reset(m);
  if (rc) return rc;
  cudaEventRecord(e0, st);
  int32_t next = 0;
  if (cache) {
    uint64_t hit = 0;
    rc = kib_qwen35_prefill_cached(m, cache, rq->prompt_tokens, rq->prompt_count, &next, &hit);
    if (cached_tokens) *cached_tokens = hit;
  } else {
    rc = kib_qwen35_prefill(m, rq->prompt_tokens, rq->prompt_count, rq->prefill_chunk_tokens, &next);
  }
  if (rc) return rc;
  cudaEventRecord(e1, st);
  res->prompt_tokens = rq->prompt_count;
  uint64_t n = 0;
  bool stop = false;
  // a committed token: stored, then handed to the callback (false: cancelled)
  auto emit = [&](int32_t t) {
    out[n] = t;
    ++n;
    if (cb && cb(user, t, n - 1) != 0) cancelled = true;
    return !cancelled;
  };
  const bool mtp = rq->enable_mtp && m->has_mtp && rq->mtp_draft_tokens > 0;
  kib_mtp_report& R = res->mtp;
  R.available = m->has_mtp ? 1 : 0;
  R.enabled = mtp ? 1 : 0;
  R.draft_tokens = rq->mtp_draft_tokens;
  R.p_min = rq->mtp_p_min;
  if (!mtp) {
    // greedy loop (6601-6632), replayed in device-side batches; tokens past an
    // EOS are discarded
    int32_t tok = next;
    if (is_eos(tok)) {
      stop = true;
    } else if (max_new > 0 && !emit(tok)) {
      stop = true;
    }
    std::vector<int32_t> buf;
    while (!stop && n < max_new) {
      // (smaller device batches when streaming, so tokens reach the client sooner)
      const uint64_t batch = std::min<uint64_t>(cb ? 4 : 32, max_new - n);
      buf.resize(batch);
      rc = kib_qwen35_decode_greedy(m, tok, batch, buf.data());
      if (rc) return rc;
      for (uint64_t i = 0; i < batch; ++i) {
        if (is_eos(buf[i]) || !emit(buf[i])) {
          stop = true;
          break;
        }
      }
      tok = buf[batch - 1];
    }
  } else {
    // MTP loop (6457-6600) with the adaptive budget (6421-6455)
    const uint64_t K = std::min<uint64_t>(rq->mtp_draft_tokens, kMaxSmallT - 1);
    uint64_t budget = rq->mtp_adaptive ? 1 : K;
    uint64_t win_d = 0, win_a = 0;
    int32_t next_token = next;
    while (n < max_new && !stop) {
      if (is_eos(next_token)) {
        stop = true;
        break;
      }
      if (!emit(next_token)) {
        stop = true;
        break;
      }
      if (n >= max_new) break;
      const uint64_t vpos = m->pos;
      const uint64_t b = std::min<uint64_t>(budget, max_new - n);
      // draft chain on the device: token and h stay resident
      m->h_pin[0] = static_cast<int>(vpos);
      m->h_pin[1] = next_token;
      m->h_pin[2] = 0;
      ENG_CUDA(cudaMemcpyAsync(m->d_mtp_pos, m->h_pin, 4, cudaMemcpyHostToDevice, st));
      ENG_CUDA(cudaMemcpyAsync(m->d_mtp_tok, m->h_pin + 1, 4, cudaMemcpyHostToDevice, st));
      ENG_CUDA(cudaMemcpyAsync(m->d_step, m->h_pin + 2, 4, cudaMemcpyHostToDevice, st));
      ENG_CUDA(cudaMemcpyAsync(m->d_mtp_h, m->d_pending_h, static_cast<size_t>(m->H) * 4, cudaMemcpyDeviceToDevice, st));
      if (!m->mtp_graph) {
        rc = capture(m, &m->mtp_graph, [&](Enq& q) {
          // d_mtp_h holds the input h; the head overwrites it with h_nextn
          q.run(cudaMemcpyAsync(m->d_hn, m->d_mtp_h, static_cast<size_t>(m->H) * 4, cudaMemcpyDeviceToDevice, q.st), "h_in");
          mtp_enqueue(q, 1, m->d_mtp_tok, m->d_hn, true, m->d_mtp_tok, m->d_prob, m->d_log, m->d_step, m->d_mtp_pos);
        });
        if (rc) return rc;
      }
      for (uint64_t i = 0; i < b; ++i) ENG_CUDA(cudaGraphLaunch(m->mtp_graph, st));
      ENG_CUDA(cudaMemcpyAsync(m->h_pin + 64, m->d_log, b * 4, cudaMemcpyDeviceToHost, st));
      ENG_CUDA(cudaMemcpyAsync(m->h_pinf, m->d_prob, b * 4, cudaMemcpyDeviceToHost, st));
      rc = sync_check(m, "mtp draft");
      if (rc) return rc;
      std::vector<int32_t> drafts;
      for (uint64_t i = 0; i < b; ++i) {
        if (rq->mtp_p_min > 0.0 && static_cast<double>(m->h_pinf[i]) < rq->mtp_p_min) {
          ++R.confidence_stops;
          break;
        }
        drafts.push_back(m->h_pin[64 + i]);
        ++R.drafted_tokens;
      }
      std::vector<int32_t> verify{next_token};
      verify.insert(verify.end(), drafts.begin(), drafts.end());
      // snapshot_recurrent_state (6154-6167)
      ENG_CUDA(cudaMemcpyAsync(m->d_r_snap, m->d_r, m->r_elems * 4, cudaMemcpyDeviceToDevice, st));
      ENG_CUDA(cudaMemcpyAsync(m->d_s_snap, m->d_s, m->s_elems * 4, cudaMemcpyDeviceToDevice, st));
      std::vector<int32_t> targets(verify.size());
      rc = kib_qwen35_forward(m, verify.data(), verify.size(), 0, targets.data(), nullptr, nullptr);
      if (rc) return rc;
      uint64_t acc = 0;
      for (size_t i = 0; i < drafts.size(); ++i) {
        if (n >= max_new) break;
        ++R.verify_steps;
        if (i < 8) ++R.verified_by_position[i];
        if (is_eos(targets[i])) {
          stop = true;
          break;
        }
        if (targets[i] != drafts[i]) break;
        ++acc;
        if (!emit(drafts[i])) {
          stop = true;
          break;
        }
        ++R.accepted_tokens;
        if (i < 8) ++R.accepted_by_position[i];
        if (n >= max_new) break;
      }
      if (rq->mtp_adaptive && K > 1 && !drafts.empty()) {
        win_d += drafts.size();
        win_a += acc;
        const uint64_t thr = std::max<uint64_t>(16, budget * 8);
        if (win_d >= thr) {
          bool changed = false;
          if (budget > 1 && win_a * 4 < win_d * 3) {
            --budget;
            changed = true;
          } else if (budget < K && win_a == win_d) {
            ++budget;
            changed = true;
          }
          if (changed) {
            ++R.adaptive_changes;
            win_d = win_a = 0;
          } else if (win_d >= thr * 2) {
            win_d = win_a = 0;
          }
        }
      }
      const uint64_t committed = 1 + acc;
      if (stop) {
        m->pos = vpos + committed;
        break;
      }
      if (acc == drafts.size()) {
        m->pos = vpos + committed;
        ENG_CUDA(cudaMemcpyAsync(m->d_pending_h, m->d_hn + (committed - 1) * static_cast<size_t>(m->H),
                                 static_cast<size_t>(m->H) * 4, cudaMemcpyDeviceToDevice, st));
        next_token = targets[committed - 1];
      } else {
        // restore_recurrent_state (6169-6182) and re-run the committed tokens
        ENG_CUDA(cudaMemcpyAsync(m->d_r, m->d_r_snap, m->r_elems * 4, cudaMemcpyDeviceToDevice, st));
        ENG_CUDA(cudaMemcpyAsync(m->d_s, m->d_s_snap, m->s_elems * 4, cudaMemcpyDeviceToDevice, st));
        std::vector<int32_t> commit(verify.begin(), verify.begin() + static_cast<long>(committed));
        std::vector<int32_t> ct(committed);
        m->pos = vpos;
        rc = kib_qwen35_forward(m, commit.data(), committed, 1, ct.data(), nullptr, nullptr);
        if (rc) return rc;
        ENG_CUDA(cudaMemcpyAsync(m->d_pending_h, m->d_hn + (committed - 1) * static_cast<size_t>(m->H),
                                 static_cast<size_t>(m->H) * 4, cudaMemcpyDeviceToDevice, st));
        next_token = ct[committed - 1];
      }
    }
    R.adaptive_budget = budget;
  }
  cudaEventRecord(e2, st);
  cudaEventSynchronize(e2);
  float pf = 0, dc = 0;
  cudaEventElapsedTime(&pf, e0, e1);
  cudaEventElapsedTime(&dc, e1, e2);
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  cudaEventDestroy(e2);
  res->prefill_ms = pf;
  res->decode_ms = dc;
  res->generated_tokens = n;
  res->finish_reason_stop = stop && !cancelled ? 1 : 0;
  res->kv_used_tokens = m->pos;
  return KIB_OK;
}

int kib_generate_qwen35(kib_qwen35* m, const kib_generation_request* rq, int32_t* out, uint64_t cap_out,
                        kib_generation_result* res) {
  return generate_impl(m, rq, nullptr, nullptr, nullptr, out, cap_out, res, nullptr);
}

int kib_generate_qwen35_stream(kib_qwen35* m, const kib_generation_request* rq, kib_qwen35_prefix_cache* cache,
                               kib_token_callback cb, void* user, int32_t* out, uint64_t cap_out,
                               kib_generation_result* res, uint64_t* cached_tokens) {
  return generate_impl(m, rq, cache, cb, user, out, cap_out, res, cached_tokens);
}

}  // extern "C"

// ================================================================ batched decode
// `slots` independent sequences decoded together, one token each per step
// (the plan's sequence_slots, qwen35_runtime.hpp:20 / qwen35_runtime.cpp:4478-4479,
// which the reference reserves but never runs).  The batch owns each slot's
// KV cache, conv state R and delta-rule state S; the model's activation and
// GEMM scratch is shared (one batch step runs at a time on the model's
// stream).  The projections of a step are one GEMM over the slots, so they
// take the reference's M > 8 numerics bucket (weights and inputs rounded to
// half, fp32 accumulation) for every slot.
struct kib_qwen35_batch {
  kib_qwen35* m = nullptr;
  int slots = 0;
  int cap = 0;                // positions per slot
  int nsplit = 8;             // attention key splits per slot
  int max_steps = 0;
  size_t k_slot = 0, r_slot = 0, s_slot = 0;  // elements per slot
  uint16_t *d_k = nullptr, *d_v = nullptr;    // [slot][attention layer][cap][KD]
  float *d_r = nullptr, *d_s = nullptr;       // [slot][linear layer][...]
  float* d_part = nullptr;                    // [slot][nsplit][heads][256 + 2]
  unsigned* d_cnt = nullptr;                  // [slot][kv_heads]
  float* d_logits = nullptr;                  // [slot][vocab]
  int *d_tok = nullptr, *d_pos = nullptr, *d_log = nullptr, *d_step = nullptr;
  std::vector<int> pos;                       // host copy of the slot positions
  cudaGraphExec_t graph = nullptr;
};

namespace {

void linear_block_batch(Enq& q, kib_qwen35_batch* b, const LayerW& L, int S) {
  kib_qwen35* m = q.m;
  const int li = L.cache_index;
  q.run(rms_rows_launch(m->d_h, L.attn_norm.f(), S, m->H, m->eps, m->d_norm, q.st, m->d_x16), "rms");
  gemm(q, L.qkv, m->d_norm, m->H, S, m->d_qkv, m->C, nullptr, false, true);
  q.run(launch_pdl(conv_batched_kernel<4>, dim3((m->C + 255) / 256, S), dim3(256), 0, q.st,
                   b->d_r + static_cast<size_t>(li) * m->C * (m->convk - 1), b->r_slot,
                   static_cast<const float*>(m->d_qkv), m->C, L.conv1d.f(), m->C, m->d_qkv, m->C),
        "conv_batched");
  gemm(q, L.zgate, m->d_norm, m->H, S, m->d_z, m->VD, nullptr, true);
  gemm(q, L.beta, m->d_norm, m->H, S, m->d_beta, m->lvh, nullptr, true);
  gemm(q, L.alpha, m->d_norm, m->H, S, m->d_alpha, m->lvh, nullptr, true);
  GdnParams g = {};
  g.conv_out = m->d_qkv;
  g.C = m->C;
  g.beta_raw = m->d_beta;
  g.alpha_raw = m->d_alpha;
  g.ld_ba = m->lvh;
  g.dt_bias = L.dt_bias.f();
  g.ssm_a = L.ssm_a.f();
  g.state = b->d_s + static_cast<size_t>(li) * m->lvh * m->lhd * m->lhd;
  g.out = m->d_y;
  g.T = 1;
  g.key_heads = m->lkh;
  g.value_heads = m->lvh;
  g.eps = m->eps;
  g.batched = 1;
  g.state_slot_stride = b->s_slot;
  q.run(launch_pdl(gdn_core_kernel, dim3(m->lvh, m->lhd / kGdnRows, S), dim3(128), 0, q.st, g), "gdn_batched");
  q.run(norm_gate_launch(m->d_y, L.ssm_norm.f(), m->d_z, S, m->lvh, m->lhd, m->eps, m->d_norm2, q.st, m->d_x16),
        "norm_gate");
  gemm(q, L.ssm_out, m->d_norm2, m->VD, S, m->d_h1, m->H, m->d_h, false, true);
}

void attention_block_batch(Enq& q, kib_qwen35_batch* b, const LayerW& L, int S) {
  kib_qwen35* m = q.m;
  q.run(rms_rows_launch(m->d_h, L.attn_norm.f(), S, m->H, m->eps, m->d_norm, q.st, m->d_x16), "rms");
  gemm(q, L.q, m->d_norm, m->H, S, m->d_qg, 2 * m->AD, nullptr, false, true);
  gemm(q, L.k, m->d_norm, m->H, S, m->d_kp, m->KD, nullptr, true);
  gemm(q, L.v, m->d_norm, m->H, S, m->d_vp, m->KD, nullptr, true);
  const size_t off = static_cast<size_t>(L.cache_index) * b->cap * m->KD;
  AttnParams a = attn_params(m, L, b->d_k + off, b->d_v + off, b->d_pos, 1);
  a.batched = 1;
  a.cache_slot_stride = b->k_slot;
  a.nsplit = b->nsplit;
  a.part = b->d_part;
  a.counters = b->d_cnt;
  a.round_q = 0;
  static bool cfg = false;
  if (!cfg) {
    q.run(cudaFuncSetAttribute(attn_decode_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024),
          "attn_decode_attr");
    cfg = true;
  }
  q.run(launch_pdl(attn_decode_kernel<1>, dim3(b->nsplit, m->kvh, S), dim3(256), attn_decode_smem_bytes(1), q.st, a),
        "attn_batched");
  gemm(q, L.o, m->d_att, m->AD, S, m->d_h1, m->H, m->d_h);
}

// One step for every slot: embedding of d_tok, the layers, the LM head over
// the batch, argmax per slot into d_tok / d_log, positions advanced.
void batch_step(Enq& q, kib_qwen35_batch* b) {
  kib_qwen35* m = q.m;
  const int S = b->slots;
  q.run(get_rows_launch(m->tok_embd.type, m->tok_embd.p, m->V, m->H, b->d_tok, S, m->d_h, m->H, q.st), "embed");
  for (const LayerW& L : m->layers) {
    if (L.kind == 0) linear_block_batch(q, b, L, S);
    else attention_block_batch(q, b, L, S);
    ffn_prefill(q, L, S, m->d_h1, m->d_h);
  }
  // the head's skinny GEMM reads the half rows the norm writes
  q.run(rms_rows_launch(m->d_h, m->output_norm.f(), S, m->H, m->eps, m->d_hn, q.st, m->d_x16), "head_norm");
  const DevT& hw = head_weight(m);
  if (S <= 64) {
    q.run(kq_skinny_launch(hw.type, hw.p, m->V, m->H, m->d_x16, S, b->d_logits, m->V, nullptr,
                           reinterpret_cast<float*>(m->d_w16), m->ctx->num_sms, q.st, false),
          "lm_head");
  } else {
    q.run(gemm_f16_launch(hw.type, hw.p, m->V, m->H, m->d_hn, m->H, S, b->d_logits, m->V, nullptr, q.st), "lm_head");
  }
  q.run(launch_pdl(batch_argmax_kernel, dim3(S), dim3(256), 0, q.st, static_cast<const float*>(b->d_logits), m->V,
                   b->d_tok, b->d_pos, b->d_log, b->d_step, S),
        "argmax");
  q.run(launch_pdl(batch_step_kernel, dim3(1), dim3(32), 0, q.st, b->d_step), "step");
}

void batch_release(kib_qwen35_batch* b) {
  if (!b) return;
  if (b->graph) cudaGraphExecDestroy(b->graph);
  void* ptrs[] = {b->d_k, b->d_v, b->d_r, b->d_s, b->d_part, b->d_cnt, b->d_logits, b->d_tok, b->d_pos, b->d_log,
                  b->d_step};
  for (void* p : ptrs)
    if (p) cudaFree(p);
  delete b;
}

}  // namespace

extern "C" {

int kib_qwen35_batch_create(kib_qwen35* m, uint64_t slots, uint64_t context_tokens, uint64_t max_steps,
                            kib_qwen35_batch** out) {
  if (!m || !out) return KIB_ERR_INVALID_ARGUMENT;
  *out = nullptr;
  if (slots <= 8 || slots > static_cast<uint64_t>(m->tmax))
    return fail(m, KIB_ERR_INVALID_ARGUMENT, "batched decode needs 9 .. prefill-chunk slots (the M > 8 GEMM bucket)");
  if (context_tokens == 0 || context_tokens > (1u << 20) || max_steps == 0 || max_steps > (1u << 20))
    return fail(m, KIB_ERR_INVALID_ARGUMENT, "batched decode: context_tokens / max_steps out of range");
  if (m->convk != 4 || m->lhd != 128 || m->hd != 256 || !m->d_w16)
    return fail(m, KIB_ERR_UNAVAILABLE, "batched decode needs conv kernel 4, head dims 128/256 and the f16 GEMM scratch");
  auto* b = new kib_qwen35_batch;
  b->m = m;
  b->slots = static_cast<int>(slots);
  b->cap = static_cast<int>(context_tokens);
  b->max_steps = static_cast<int>(max_steps);
  b->nsplit = std::max(1, std::min(32, (b->cap + 255) / 256));
  const size_t n_full = m->plan.full_attention_layers, n_lin = m->plan.linear_attention_layers;
  b->k_slot = n_full * static_cast<size_t>(b->cap) * m->KD;
  b->r_slot = n_lin * static_cast<size_t>(m->C) * (m->convk - 1);
  b->s_slot = n_lin * static_cast<size_t>(m->lvh) * m->lhd * m->lhd;
  const size_t S = slots;
  auto al = [](void** p, size_t bytes) { return cudaMalloc(p, std::max<size_t>(bytes, 16)) == cudaSuccess; };
  bool ok = al(reinterpret_cast<void**>(&b->d_k), S * b->k_slot * 2) && al(reinterpret_cast<void**>(&b->d_v), S * b->k_slot * 2) &&
            al(reinterpret_cast<void**>(&b->d_r), S * b->r_slot * 4) && al(reinterpret_cast<void**>(&b->d_s), S * b->s_slot * 4) &&
            al(reinterpret_cast<void**>(&b->d_part), S * b->nsplit * m->heads * (kHd + 2) * 4) &&
            al(reinterpret_cast<void**>(&b->d_cnt), S * m->kvh * 4) &&
            al(reinterpret_cast<void**>(&b->d_logits), S * static_cast<size_t>(m->V) * 4) &&
            al(reinterpret_cast<void**>(&b->d_tok), S * 4) && al(reinterpret_cast<void**>(&b->d_pos), S * 4) &&
            al(reinterpret_cast<void**>(&b->d_log), S * max_steps * 4) && al(reinterpret_cast<void**>(&b->d_step), 4);
  if (!ok) {
    batch_release(b);
    return fail(m, KIB_ERR_INTERNAL, "batched decode: device allocation failed");
  }
  cudaMemset(b->d_cnt, 0, S * m->kvh * 4);
  cudaMemset(b->d_k, 0, S * b->k_slot * 2);
  cudaMemset(b->d_v, 0, S * b->k_slot * 2);
  cudaMemset(b->d_r, 0, S * b->r_slot * 4);
  cudaMemset(b->d_s, 0, S * b->s_slot * 4);
  b->pos.assign(S, 0);
  *out = b;
  return KIB_OK;
}

void kib_qwen35_batch_free(kib_qwen35_batch* b) {
  if (b && b->m) cudaStreamSynchronize(b->m->ctx->stream);
  batch_release(b);
}

int kib_qwen35_batch_prefill(kib_qwen35_batch* b, uint64_t slot, const int32_t* tokens, uint64_t n,
                             int32_t* next_token) {
  if (!b || !tokens || n == 0 || slot >= static_cast<uint64_t>(b->slots)) return KIB_ERR_INVALID_ARGUMENT;
  kib_qwen35* m = b->m;
  if (n >= static_cast<uint64_t>(b->cap)) return fail(m, KIB_ERR_INVALID_ARGUMENT, "batched prefill exceeds the slot capacity");
  // the model's own single-sequence caches run the prefill, then the slot takes a copy
  if (int rc = kib_qwen35_reset(m)) return rc;
  if (int rc = kib_qwen35_prefill(m, tokens, n, 0, next_token)) return rc;
  cudaStream_t st = m->ctx->stream;
  const size_t n_full = m->plan.full_attention_layers;
  for (size_t l = 0; l < n_full; ++l) {
    const size_t src = l * static_cast<size_t>(m->cap) * m->KD, dst = slot * b->k_slot + l * static_cast<size_t>(b->cap) * m->KD;
    ENG_CUDA(cudaMemcpyAsync(b->d_k + dst, m->d_k + src, n * m->KD * 2, cudaMemcpyDeviceToDevice, st));
    ENG_CUDA(cudaMemcpyAsync(b->d_v + dst, m->d_v + src, n * m->KD * 2, cudaMemcpyDeviceToDevice, st));
  }
  ENG_CUDA(cudaMemcpyAsync(b->d_r + slot * b->r_slot, m->d_r, b->r_slot * 4, cudaMemcpyDeviceToDevice, st));
  ENG_CUDA(cudaMemcpyAsync(b->d_s + slot * b->s_slot, m->d_s, b->s_slot * 4, cudaMemcpyDeviceToDevice, st));
  ENG_CUDA(cudaStreamSynchronize(st));
  b->pos[slot] = static_cast<int>(n);
  return KIB_OK;
}

int kib_qwen35_batch_decode(kib_qwen35_batch* b, const int32_t* first_tokens, uint64_t steps, int32_t* tokens_out) {
  if (!b || !first_tokens || steps == 0) return KIB_ERR_INVALID_ARGUMENT;
  kib_qwen35* m = b->m;
  if (steps > static_cast<uint64_t>(b->max_steps)) return fail(m, KIB_ERR_INVALID_ARGUMENT, "batched decode: more steps than max_steps");
  for (int s = 0; s < b->slots; ++s)
    if (static_cast<uint64_t>(b->pos[s]) + steps > static_cast<uint64_t>(b->cap))
      return fail(m, KIB_ERR_INVALID_ARGUMENT, "batched decode exceeds a slot's capacity");
  if (int rc = check_tokens(m, first_tokens, static_cast<uint64_t>(b->slots))) return rc;
  cudaStream_t st = m->ctx->stream;
  ENG_CUDA(cudaMemcpyAsync(b->d_tok, first_tokens, b->slots * 4, cudaMemcpyHostToDevice, st));
  ENG_CUDA(cudaMemcpyAsync(b->d_pos, b->pos.data(), b->slots * 4, cudaMemcpyHostToDevice, st));
  ENG_CUDA(cudaMemsetAsync(b->d_step, 0, 4, st));
  if (!b->graph) {
    int rc = capture(m, &b->graph, [&](Enq& q) { batch_step(q, b); });
    if (rc) return rc;
  }
  for (uint64_t i = 0; i < steps; ++i) ENG_CUDA(cudaGraphLaunch(b->graph, st));
  if (tokens_out)
    ENG_CUDA(cudaMemcpyAsync(tokens_out, b->d_log, steps * b->slots * 4, cudaMemcpyDeviceToHost, st));
  if (int rc = sync_check(m, "batched decode")) return rc;
  for (int s = 0; s < b->slots; ++s) b->pos[s] += static_cast<int>(steps);
  return KIB_OK;
}

int kib_qwen35_batch_logits(kib_qwen35_batch* b, float* logits_out) {
  if (!b || !logits_out) return KIB_ERR_INVALID_ARGUMENT;
  kib_qwen35* m = b->m;
  ENG_CUDA(cudaMemcpy(logits_out, b->d_logits, static_cast<size_t>(b->slots) * m->V * 4, cudaMemcpyDeviceToHost));
  return KIB_OK;
}

uint64_t kib_qwen35_batch_position(const kib_qwen35_batch* b, uint64_t slot) {
  return (b && slot < static_cast<uint64_t>(b->slots)) ? static_cast<uint64_t>(b->pos[slot]) : 0;
}

}  // extern "C"

// ================================================================ host prompt cache
// The reference's host prefix cache (Qwen35HostPrefixCache,
// qwen35_runtime.cpp:516-932): prompts are prefilled in blocks of
// block_tokens; after each full block the block's K/V rows of every attention
// layer, the whole conv and delta-rule state and the block's last hidden row
// are copied to host memory under the block's chained hash; a later prompt
// with the same block-aligned prefix restores those bytes into the device
// caches and prefills only the rest (or, when the whole prompt hit, samples
// its next token from the restored hidden row).  Restored bytes are the ones
// the prefill computed, so a hit leaves exactly the state of a fresh prefill
// in the same blocks.
struct kib_qwen35_prefix_cache {
  kib_qwen35* m = nullptr;
  std::unique_ptr<kib::PrefixIndex> idx;
  struct Payload {
    std::vector<uint16_t> k, v;  // [attention layer][block_tokens][kv_dim]
    std::vector<float> r, s, h;  // whole R, whole S, last hidden row
  };
  std::map<uint64_t, Payload> payloads;
};

namespace {

int prefix_read_payload(kib_qwen35_prefix_cache* pc, uint64_t start, uint64_t block, int last_row,
                        kib_qwen35_prefix_cache::Payload* out) {
  kib_qwen35* m = pc->m;
  const size_t n_full = m->plan.full_attention_layers, kd = static_cast<size_t>(m->KD);
  out->k.resize(n_full * block * kd);
  out->v.resize(n_full * block * kd);
  for (size_t l = 0; l < n_full; ++l) {
    const size_t src = (l * static_cast<size_t>(m->cap) + start) * kd, dst = l * block * kd;
    ENG_CUDA(cudaMemcpy(out->k.data() + dst, m->d_k + src, block * kd * 2, cudaMemcpyDeviceToHost));
    ENG_CUDA(cudaMemcpy(out->v.data() + dst, m->d_v + src, block * kd * 2, cudaMemcpyDeviceToHost));
  }
  out->r.resize(m->r_elems);
  out->s.resize(m->s_elems);
  out->h.resize(static_cast<size_t>(m->H));
  ENG_CUDA(cudaMemcpy(out->r.data(), m->d_r, m->r_elems * 4, cudaMemcpyDeviceToHost));
  ENG_CUDA(cudaMemcpy(out->s.data(), m->d_s, m->s_elems * 4, cudaMemcpyDeviceToHost));
  ENG_CUDA(cudaMemcpy(out->h.data(), m->d_h + static_cast<size_t>(last_row) * m->H, static_cast<size_t>(m->H) * 4,
                      cudaMemcpyDeviceToHost));
  return KIB_OK;
}

}  // namespace

extern "C" {

int kib_qwen35_prefix_cache_create(kib_qwen35* m, uint64_t block_tokens, uint64_t capacity_blocks,
                                   uint64_t min_reuse_tokens, kib_qwen35_prefix_cache** out) {
  if (!m || !out) return KIB_ERR_INVALID_ARGUMENT;
  *out = nullptr;
  if (block_tokens == 0 || block_tokens > static_cast<uint64_t>(m->tmax) || capacity_blocks == 0)
    return fail(m, KIB_ERR_INVALID_ARGUMENT, "prefix cache: block_tokens must be 1 .. the prefill chunk, capacity > 0");
  auto* pc = new kib_qwen35_prefix_cache;
  pc->m = m;
  pc->idx.reset(new kib::PrefixIndex(block_tokens, capacity_blocks, min_reuse_tokens));
  *out = pc;
  return KIB_OK;
}

void kib_qwen35_prefix_cache_free(kib_qwen35_prefix_cache* pc) { delete pc; }

void kib_qwen35_prefix_cache_stats(const kib_qwen35_prefix_cache* pc, uint64_t* out6) {
  if (pc && out6) pc->idx->stats(out6);
}

int kib_qwen35_prefill_cached(kib_qwen35* m, kib_qwen35_prefix_cache* pc, const int32_t* tokens, uint64_t n,
                              int32_t* next_token, uint64_t* hit_tokens) {
  if (!m || !pc || pc->m != m || !tokens || n == 0 || !next_token) return KIB_ERR_INVALID_ARGUMENT;
  if (n > static_cast<uint64_t>(m->cap)) return fail(m, KIB_ERR_INVALID_ARGUMENT, "prefill exceeds cache capacity");
  if (int rc = check_tokens(m, tokens, n)) return rc;
  const uint64_t block = pc->idx->block_tokens();
  std::vector<int64_t> t64(tokens, tokens + n);
  std::vector<uint64_t> hashes;
  const uint64_t hit = pc->idx->lookup(t64.data(), n, &hashes);
  if (hit_tokens) *hit_tokens = hit;
  if (int rc = kib_qwen35_reset(m)) return rc;
  if (hit > 0) {
    // restore_kv_block per hit block, then the state and hidden row of the last one
    const size_t n_full = m->plan.full_attention_layers, kd = static_cast<size_t>(m->KD);
    for (size_t b = 0; b < hashes.size(); ++b) {
      auto it = pc->payloads.find(hashes[b]);
      if (it == pc->payloads.end()) return fail(m, KIB_ERR_INTERNAL, "prefix cache payload is missing");
      for (size_t l = 0; l < n_full; ++l) {
        const size_t dst = (l * static_cast<size_t>(m->cap) + b * block) * kd, src = l * block * kd;
        ENG_CUDA(cudaMemcpy(m->d_k + dst, it->second.k.data() + src, block * kd * 2, cudaMemcpyHostToDevice));
        ENG_CUDA(cudaMemcpy(m->d_v + dst, it->second.v.data() + src, block * kd * 2, cudaMemcpyHostToDevice));
      }
    }
    const auto& last = pc->payloads.at(hashes.back());
    ENG_CUDA(cudaMemcpy(m->d_r, last.r.data(), m->r_elems * 4, cudaMemcpyHostToDevice));
    ENG_CUDA(cudaMemcpy(m->d_s, last.s.data(), m->s_elems * 4, cudaMemcpyHostToDevice));
    m->pos = hit;
    if (int rc = set_pos(m, m->d_pos, hit)) return rc;
    if (hit == n) {
      // the whole prompt hit: the next token from the restored last hidden row
      ENG_CUDA(cudaMemcpy(m->d_h, last.h.data(), static_cast<size_t>(m->H) * 4, cudaMemcpyHostToDevice));
      Enq q{m, m->ctx->stream};
      head_small(q, 1, m->d_h, m->output_norm, head_weight(m), m->d_argmax, m->d_prob, nullptr, nullptr, nullptr,
                 nullptr, nullptr);
      if (!q.ok()) return fail(m, KIB_ERR_INTERNAL, "prefix cache head: " + q.why);
      ENG_CUDA(cudaMemcpyAsync(m->h_pin, m->d_argmax, 4, cudaMemcpyDeviceToHost, m->ctx->stream));
      if (int rc = sync_check(m, "prefix cache head")) return rc;
      *next_token = m->h_pin[0];
      return KIB_OK;
    }
  }
  // the rest in blocks; every full block is committed with its payload
  for (uint64_t start = hit; start < n; start += block) {
    const uint64_t c = std::min<uint64_t>(block, n - start);
    if (int rc = kib_qwen35_prefill(m, tokens + start, c, c, next_token)) return rc;
    if (c != block) continue;
    const uint64_t h = pc->idx->hash_for(t64.data(), start);
    if (pc->payloads.count(h)) continue;
    kib_qwen35_prefix_cache::Payload pl;
    if (int rc = prefix_read_payload(pc, start, block, static_cast<int>(c) - 1, &pl)) return rc;
    const kib::PrefixCommit cm = pc->idx->commit(t64.data(), n, start);
    if (!cm.inserted) continue;
    if (cm.evicted) pc->payloads.erase(cm.evicted_hash);
    pc->payloads[cm.hash] = std::move(pl);
  }
  return KIB_OK;
}

}  // extern "C"
