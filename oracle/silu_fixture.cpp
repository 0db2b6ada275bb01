// silu_fixture.cpp -- TEST INFRASTRUCTURE: the reference's own dealer for the
// SiLU spline gate, writing a JSON fixture for the coefficient-gate kernel.
//
// Built by oracle/Makefile (target `silu`) from the reference's headers and
// src/compiler/suf_to_pfss.cpp where they lie, plus this repository's
// adapter in dealer-only mode (no GPU needed).  It runs, unchanged:
//   gates::make_silu_spec({f, 16})             include/gates/silu_spline_gate.hpp
//   suf::build_silu_suf_from_piecewise(spec)   include/suf/suf_silu_builders.hpp
//   gates::composite_gen_backend_with_masks    include/gates/composite_fss.hpp
// with proto::SufB200Backend as the backend (interval-LUT coefficient mode:
// the gate has no boolean outputs), and prints the compiled coefficient
// program's shape, both parties' interval-LUT keys and r_out shares, the SUF
// table (alpha cutpoints and per-piece coefficient words) and
// suf::eval_suf_ref (include/suf/ref_eval.hpp) on sample inputs.
// Usage: silu_fixture <frac_bits> <seed> <samples>
#include <cstdio>
#include <cstdlib>
#include <random>
#include <vector>

#include "gates/composite_fss.hpp"
#include "gates/silu_spline_gate.hpp"
#include "suf/ref_eval.hpp"
#include "suf/suf_silu_builders.hpp"
#include "sufb200_backend.hpp"

namespace {

void hex(const std::vector<uint8_t>& b) {
  std::printf("\"");
  for (uint8_t c : b) std::printf("%02x", c);
  std::printf("\"");
}

void u64s(const std::vector<uint64_t>& v) {
  std::printf("[");
  for (size_t i = 0; i < v.size(); i++) std::printf("%s\"%llu\"", i ? "," : "", static_cast<unsigned long long>(v[i]));
  std::printf("]");
}

}  // namespace

int main(int argc, char** argv) {
  const int f = argc > 1 ? std::atoi(argv[1]) : 12;
  const uint64_t seed = argc > 2 ? std::strtoull(argv[2], nullptr, 10) : 3;
  const size_t samples = argc > 3 ? std::strtoull(argv[3], nullptr, 10) : 256;

  auto spec = gates::make_silu_spec({f, 16});
  auto F = suf::build_silu_suf_from_piecewise(spec);

  proto::SufB200Backend::Options o;
  o.dealer_only = true;
  o.deterministic = true;
  o.seed = seed * 7919;
  proto::SufB200Backend dealer(o);

  std::mt19937_64 rng(seed);
  const uint64_t r_in = rng();
  std::vector<uint64_t> r_out(static_cast<size_t>(F.r_out));
  for (auto& v : r_out) v = rng();
  auto kp = gates::composite_gen_backend_with_masks(F, dealer, rng, r_in, r_out, samples,
                                                    compiler::GateKind::SiLUSpline);
  const auto& c = kp.k0.compiled;
  if (c.coeff.mode != compiler::CoeffMode::kIntervalLut || kp.k0.coeff_keys.size() != 1) {
    std::fprintf(stderr, "expected one interval-LUT coefficient key\n");
    return 1;
  }

  // sample inputs: Gaussian sigma = 4 at f fractional bits (mt19937_64(seed + 100),
  // std::normal_distribution), plus the spline's breakpoints and the extremes
  std::mt19937_64 xr(seed + 100);
  std::normal_distribution<double> nd(0.0, 4.0);
  std::vector<uint64_t> xs;
  for (double b : {-8.0, -7.0, -0.5, 0.0, 0.5, 7.0, 8.0}) {
    const int64_t q = static_cast<int64_t>(std::llround(b * std::ldexp(1.0, f)));
    xs.push_back(static_cast<uint64_t>(q));
    xs.push_back(static_cast<uint64_t>(q - 1));
  }
  xs.push_back(0x7FFFFFFFFFFFFFFFull);
  xs.push_back(0x8000000000000000ull);
  while (xs.size() < samples)
    xs.push_back(static_cast<uint64_t>(static_cast<int64_t>(std::llround(nd(xr) * std::ldexp(1.0, f)))));

  std::printf("{\"frac_bits\":%d,\"seed\":%llu,\"r_in\":\"%llu\",\"r\":%d,\"degree\":%d,\"out_words\":%d,"
              "\"coeff_in_bits\":%d,\"ring_bits\":64,",
              f, static_cast<unsigned long long>(seed), static_cast<unsigned long long>(r_in), c.r, c.degree,
              c.coeff.out_words, c.coeff.n);
  std::printf("\"r_out\":");
  u64s(r_out);
  std::printf(",\"r_out_share0\":");
  u64s(kp.k0.r_out_share);
  std::printf(",\"r_out_share1\":");
  u64s(kp.k1.r_out_share);
  std::printf(",\"key0\":");
  hex(kp.k0.coeff_keys[0].bytes);
  std::printf(",\"key1\":");
  hex(kp.k1.coeff_keys[0].bytes);
  std::printf(",\"alpha\":");
  u64s(F.alpha);
  std::printf(",\"pieces\":[");
  for (size_t p = 0; p < F.pieces.size(); p++) {
    std::vector<uint64_t> w;
    for (const auto& poly : F.pieces[p].polys) w.push_back(poly.coeffs.empty() ? 0 : poly.coeffs[0]);
    std::printf("%s", p ? "," : "");
    u64s(w);
  }
  std::printf("],\"samples\":[");
  for (size_t i = 0; i < xs.size(); i++) {
    const auto ref = suf::eval_suf_ref(F, xs[i]);
    std::printf("%s{\"x\":\"%llu\",\"expect\":", i ? "," : "", static_cast<unsigned long long>(xs[i]));
    u64s(ref.arith);
    std::printf("}");
  }
  std::printf("]}\n");
  return 0;
}
