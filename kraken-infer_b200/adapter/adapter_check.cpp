// adapter_check.cpp -- drives toyllm::mps::MpsContext as the reference's
// runtime would, through mps_context_kib.cpp and libkib.so: prints
// "unavailable: <reason>" without a B200, else runs a K-quant matvec, an RMS
// norm, the LM-head top1 and a bounds-checked copy, checks them against host
// arithmetic and prints "ok".
#include <cmath>
#include <cstdio>
#include <vector>

#include "kib.h"
#include "toyllm/backends/mps/mps_backend.hpp"

using toyllm::mps::MpsBuffer;
using toyllm::mps::MpsContext;

#define CHECK(expr)                                                            \
  do {                                                                         \
    auto st_ = (expr);                                                         \
    if (!st_.is_ok()) {                                                        \
      std::printf("fail: %s: %s\n", #expr, st_.message().c_str());             \
      return 1;                                                                \
    }                                                                          \
  } while (0)

int main() {
  auto created = MpsContext::create();
  if (!created.is_ok()) {
    std::printf("unavailable: %s\n", created.status().message().c_str());
    return 0;
  }
  MpsContext& ctx = created.value();
  const std::size_t rows = 300, cols = 512;
  std::vector<float> w(rows * cols), x(cols);
  for (std::size_t i = 0; i < w.size(); ++i) w[i] = 0.02f * std::sin(0.37f * static_cast<float>(i));
  for (std::size_t i = 0; i < cols; ++i) x[i] = std::cos(0.11f * static_cast<float>(i));
  std::vector<unsigned char> wq(rows * (cols / 256) * 144);
  if (kib_quantize_kquant(12, w.data(), w.size(), wq.data()) != KIB_OK) return 1;
  auto bw = ctx.make_buffer(wq.size());
  auto bx = ctx.make_buffer(cols * 4);
  auto by = ctx.make_buffer(rows * 4);
  auto brow = ctx.make_buffer(cols * 4);
  auto btok = ctx.make_buffer(4);
  auto bprob = ctx.make_buffer(4);
  if (!bw.is_ok() || !bx.is_ok() || !by.is_ok() || !brow.is_ok() || !btok.is_ok() || !bprob.is_ok()) return 1;
  CHECK(ctx.copy_to_buffer(bw.value(), wq.data(), wq.size()));
  CHECK(ctx.copy_to_buffer(bx.value(), x.data(), cols * 4));
  CHECK(ctx.matvec_q4_k_f32_device(bw.value(), rows, cols, bx.value(), by.value()));
  std::vector<float> y(rows), row(cols);
  CHECK(ctx.copy_from_buffer(by.value(), y.data(), rows * 4));
  double worst = 0.0, scale = 0.0;
  int best = 0;
  for (std::size_t r = 0; r < rows; ++r) {
    CHECK(ctx.dequantize_row_q4_k_f32(bw.value(), r, cols, brow.value()));
    CHECK(ctx.copy_from_buffer(brow.value(), row.data(), cols * 4));
    double ref = 0.0;
    for (std::size_t c = 0; c < cols; ++c) ref += static_cast<double>(row[c]) * x[c];
    worst = std::fmax(worst, std::fabs(ref - y[r]));
    scale = std::fmax(scale, std::fabs(ref));
    if (y[r] > y[best]) best = static_cast<int>(r);
  }
  if (worst > 1e-4 * scale) {  // the matvec tolerance of the parity tests, relative to the largest output
    std::printf("fail: matvec error %g against max |y| %g\n", worst, scale);
    return 1;
  }
  CHECK(ctx.matvec_q4_k_f32_top1(bw.value(), rows, cols, bx.value(), btok.value(), bprob.value()));
  int tok = -1;
  CHECK(ctx.copy_from_buffer(btok.value(), &tok, 4));
  if (tok != best) {
    std::printf("fail: top1 %d vs %d\n", tok, best);
    return 1;
  }
  // rms_norm_f32_f32 against host arithmetic
  auto bn = ctx.make_buffer(cols * 4);
  auto bo = ctx.make_buffer(cols * 4);
  if (!bn.is_ok() || !bo.is_ok()) return 1;
  std::vector<float> nw(cols, 1.5f), o(cols);
  CHECK(ctx.copy_to_buffer(bn.value(), nw.data(), cols * 4));
  CHECK(ctx.rms_norm_f32_f32(bx.value(), bn.value(), cols, 1e-6f, bo.value()));
  CHECK(ctx.copy_from_buffer(bo.value(), o.data(), cols * 4));
  double ss = 0.0;
  for (float v : x) ss += static_cast<double>(v) * v;
  const double sc = 1.0 / std::sqrt(ss / cols + 1e-6);
  for (std::size_t i = 0; i < cols; ++i)
    if (std::fabs(o[i] - x[i] * sc * 1.5) > 1e-5) {
      std::printf("fail: rms_norm at %zu\n", i);
      return 1;
    }
  // a copy past the end is the reference's invalid_argument, not a fault
  auto st = ctx.copy_to_buffer_at(bx.value(), cols * 4 - 4, x.data(), 8);
  if (st.is_ok() || st.code() != toyllm::StatusCode::invalid_argument) {
    std::printf("fail: out-of-bounds copy was not rejected\n");
    return 1;
  }
  std::printf("ok\n");
  return 0;
}
