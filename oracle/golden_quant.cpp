// Pins the C oracle's quantized arithmetic (nbl_oracle.c) to the golden vectors nibble ships, which llama.cpp's own
// reference code produced (tests/data/quant_golden.inc in the reference tree, made by tools/quant_vectors from
// llama.cpp b11715). The inputs are regenerated with the reference's integer-only generators
// (tests/quant_golden_gen.h) and checked against the recorded input hashes first, so a drifted generator cannot
// pass. Both headers are compiled in place from the reference tree (oracle/Makefile, target golden-check); nothing
// of them is copied here.
//
// TEST INFRASTRUCTURE ONLY: tests/test_oracle.py runs the binary (oracle/_ref/nbl_golden_check).
//
// Cases, as nibble's tests/test_quant.cpp uses them:
//   kQuantCases   Q8_0 activation quantizer (scale bits and values) of hand-made rows (ties, extremes)
//   kQ8_1Cases    Q8_1 scale and sum of the same rows
//   kDotCases     Q8_0 x Q8_0 and Q4_0 x Q8_0 dots over random blocks, widths 896 and 4864
//   kDot5Cases    Q5_0 x Q8_0 and Q5_1 x Q8_1 dots
//   kDequant*     Q8_0, Q4_0, Q5_0, Q5_1 dequantization (every float) and Q4_K, Q5_K, Q6_K (hash of the floats)
//   kQ8KCases     Q8_K quantizer on crafted and random rows (hashes of the scales and of values + sums)
//   kKDotCases    Q4_K, Q5_K, Q6_K x Q8_K dots at widths 256 to 8192
// (kQuantCases' Q4_0 fields are the weight quantizer's output, which is not on this path and not restated.)
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <vector>

#include "data/quant_golden.inc"
#include "quant_golden_gen.h"

#include "nbl_oracle.h"

namespace {

int checks = 0, failures = 0;

void expect(bool ok, const char* what, long a = 0, long b = 0) {
  ++checks;
  if (!ok) {
    ++failures;
    std::printf("FAIL %s (%ld, %ld)\n", what, a, b);
  }
}

uint32_t bits(float f) {
  uint32_t u;
  std::memcpy(&u, &f, 4);
  return u;
}

uint16_t rd16(const uint8_t* p) { return static_cast<uint16_t>(p[0] | (p[1] << 8)); }

constexpr int kQ4_0 = 2, kQ5_0 = 6, kQ5_1 = 7, kQ8_0 = 8, kQ4_K = 12, kQ5_K = 13, kQ6_K = 14;

void quantize_cases() {
  for (size_t i = 0; i < std::size(golden::kQuantCases); ++i) {
    const auto& c = golden::kQuantCases[i];
    uint8_t q8[34], q81[36];
    orc_quantize_q8_0(c.x, q8, 32);
    orc_quantize_q8_1(c.x, q81, 32);
    expect(rd16(q8) == c.q8_d, "q8_0 scale", static_cast<long>(i));
    for (int j = 0; j < 32; ++j) expect(static_cast<int8_t>(q8[2 + j]) == c.q8_qs[j], "q8_0 value", static_cast<long>(i), j);
    expect(std::strcmp(golden::kQ8_1Cases[i].name, c.name) == 0, "q8_1 case order", static_cast<long>(i));
    expect(rd16(q81) == golden::kQ8_1Cases[i].d, "q8_1 scale", static_cast<long>(i));
    expect(rd16(q81 + 2) == golden::kQ8_1Cases[i].s, "q8_1 sum", static_cast<long>(i));
    for (int j = 0; j < 32; ++j) expect(q81[4 + j] == q8[2 + j], "q8_1 value", static_cast<long>(i), j);
  }
}

void dot_cases() {
  for (const auto& c : golden::kDotCases) {
    const int nb = c.n / 32;
    std::vector<uint8_t> w8(static_cast<size_t>(nb) * 34), a8(w8.size()), w4(static_cast<size_t>(nb) * 18);
    golden::Rng r{c.seed};
    golden::fill_q8_0(r, w8.data(), nb);
    golden::fill_q8_0(r, a8.data(), nb);
    golden::fill_q4_0(r, w4.data(), nb);
    uint64_t h = golden::fnv1a(w8.data(), w8.size());
    h = golden::fnv1a(a8.data(), a8.size(), h);
    h = golden::fnv1a(w4.data(), w4.size(), h);
    expect(h == c.input_hash, "dot inputs hash", static_cast<long>(c.seed), c.n);
    expect(bits(orc_vec_dot(kQ8_0, w8.data(), a8.data(), nb)) == c.q8q8_bits, "dot q8_0", static_cast<long>(c.seed), c.n);
    expect(bits(orc_vec_dot(kQ4_0, w4.data(), a8.data(), nb)) == c.q4q8_bits, "dot q4_0", static_cast<long>(c.seed), c.n);
  }
  for (const auto& c : golden::kDot5Cases) {
    const int nb = c.n / 32;
    const size_t z = static_cast<size_t>(nb);
    std::vector<uint8_t> w50(z * 22), a80(z * 34), w51(z * 24), a81(z * 36);
    golden::Rng r{c.seed};
    golden::fill_q5_0(r, w50.data(), nb);
    golden::fill_q8_0(r, a80.data(), nb);
    golden::fill_q5_1(r, w51.data(), nb);
    golden::fill_q8_1(r, a81.data(), nb);
    uint64_t h = golden::fnv1a(w50.data(), w50.size());
    h = golden::fnv1a(a80.data(), a80.size(), h);
    h = golden::fnv1a(w51.data(), w51.size(), h);
    h = golden::fnv1a(a81.data(), a81.size(), h);
    expect(h == c.input_hash, "dot5 inputs hash", static_cast<long>(c.seed), c.n);
    expect(bits(orc_vec_dot(kQ5_0, w50.data(), a80.data(), nb)) == c.q5_0_bits, "dot q5_0", static_cast<long>(c.seed), c.n);
    expect(bits(orc_vec_dot(kQ5_1, w51.data(), a81.data(), nb)) == c.q5_1_bits, "dot q5_1", static_cast<long>(c.seed), c.n);
  }
  for (const auto& c : golden::kKDotCases) {
    const int nb = c.n / 256;
    const size_t z = static_cast<size_t>(nb);
    std::vector<uint8_t> w4(z * 144), w5(z * 176), w6(z * 210), a8(z * 292);
    golden::Rng r{c.seed};
    golden::fill_q4_K(r, w4.data(), nb);
    golden::fill_q5_K(r, w5.data(), nb);
    golden::fill_q6_K(r, w6.data(), nb);
    golden::fill_q8_K(r, a8.data(), nb);
    uint64_t h = golden::fnv1a(w4.data(), w4.size());
    h = golden::fnv1a(w5.data(), w5.size(), h);
    h = golden::fnv1a(w6.data(), w6.size(), h);
    h = golden::fnv1a(a8.data(), a8.size(), h);
    expect(h == c.input_hash, "kdot inputs hash", static_cast<long>(c.seed), c.n);
    expect(bits(orc_vec_dot(kQ4_K, w4.data(), a8.data(), nb)) == c.q4k_bits, "dot q4_K", static_cast<long>(c.seed), c.n);
    expect(bits(orc_vec_dot(kQ5_K, w5.data(), a8.data(), nb)) == c.q5k_bits, "dot q5_K", static_cast<long>(c.seed), c.n);
    expect(bits(orc_vec_dot(kQ6_K, w6.data(), a8.data(), nb)) == c.q6k_bits, "dot q6_K", static_cast<long>(c.seed), c.n);
  }
}

void dequant_cases() {
  constexpr int nb = golden::kDequantBlocks;
  std::vector<float> o(nb * 32);
  {
    std::vector<uint8_t> q8(nb * 34), q4(nb * 18);
    golden::Rng r{golden::kDequantSeed};
    golden::fill_q8_0(r, q8.data(), nb);
    golden::fill_q4_0(r, q4.data(), nb);
    orc_dequantize_row(kQ8_0, q8.data(), o.data(), nb * 32);
    for (int i = 0; i < nb * 32; ++i) expect(bits(o[i]) == golden::kDequantQ8_0[i], "dequant q8_0", i);
    orc_dequantize_row(kQ4_0, q4.data(), o.data(), nb * 32);
    for (int i = 0; i < nb * 32; ++i) expect(bits(o[i]) == golden::kDequantQ4_0[i], "dequant q4_0", i);
  }
  {
    std::vector<uint8_t> q50(nb * 22), q51(nb * 24);
    golden::Rng r{golden::kDequantSeed};
    golden::fill_q5_0(r, q50.data(), nb);
    golden::fill_q5_1(r, q51.data(), nb);
    orc_dequantize_row(kQ5_0, q50.data(), o.data(), nb * 32);
    for (int i = 0; i < nb * 32; ++i) expect(bits(o[i]) == golden::kDequantQ5_0[i], "dequant q5_0", i);
    orc_dequantize_row(kQ5_1, q51.data(), o.data(), nb * 32);
    for (int i = 0; i < nb * 32; ++i) expect(bits(o[i]) == golden::kDequantQ5_1[i], "dequant q5_1", i);
  }
  constexpr int nbk = golden::kDequantKBlocks;
  const struct {
    const char* name;
    int dtype, bytes;
    void (*fill)(golden::Rng&, uint8_t*, int64_t);
  } types[] = {{"Q4_K", kQ4_K, 144, golden::fill_q4_K}, {"Q5_K", kQ5_K, 176, golden::fill_q5_K},
               {"Q6_K", kQ6_K, 210, golden::fill_q6_K}};
  for (size_t i = 0; i < 3; ++i) {
    std::vector<uint8_t> q(static_cast<size_t>(nbk * types[i].bytes));
    golden::Rng r{golden::kDequantSeed};
    types[i].fill(r, q.data(), nbk);
    std::vector<float> ok(nbk * 256);
    orc_dequantize_row(types[i].dtype, q.data(), ok.data(), nbk * 256);
    expect(std::strcmp(golden::kDequantK[i].name, types[i].name) == 0, "dequant k case order", static_cast<long>(i));
    expect(golden::fnv1a(reinterpret_cast<const uint8_t*>(ok.data()), ok.size() * 4) == golden::kDequantK[i].hash,
           "dequant k-quant hash", static_cast<long>(i));
  }
}

void q8k_cases() {
  for (const auto& c : golden::kQ8KCases) {
    std::vector<float> x(static_cast<size_t>(c.n));
    if (c.crafted >= 0) {
      golden::crafted_q8k_row(c.crafted, x.data());
    } else {
      golden::Rng r{c.seed};
      golden::q8k_rows(r, x.data(), c.n);
    }
    std::vector<uint8_t> y(static_cast<size_t>(c.n / 256) * 292);
    orc_quantize_q8_K(x.data(), y.data(), c.n);
    uint64_t dh = 0xCBF29CE484222325ull, oh = dh;
    for (size_t b = 0; b < y.size() / 292; ++b) {
      dh = golden::fnv1a(y.data() + b * 292, 4, dh);
      oh = golden::fnv1a(y.data() + b * 292 + 4, 256 + 32, oh);
    }
    expect(dh == c.d_hash, "q8_K scales hash", c.crafted, c.n);
    expect(oh == c.out_hash, "q8_K values and sums hash", c.crafted, c.n);
  }
}

}  // namespace

int main() {
  quantize_cases();
  dot_cases();
  dequant_cases();
  q8k_cases();
  std::printf("%d of %d golden checks passed\n", checks - failures, checks);
  return failures ? 1 : 0;
}
