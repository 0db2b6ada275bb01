// tape_fixture.cpp -- TEST INFRASTRUCTURE: the reference's own truncation-gate
// dealer and composite tape writer, printing a JSON fixture for the tape
// format of this engine's writer and reader.
//
// Built by oracle/Makefile (target `tape`) from the reference's headers and
// src/compiler/suf_to_pfss.cpp where they lie, plus this repository's adapter
// in dealer-only mode (no GPU needed).  For every case (kind, frac_bits,
// seed) it runs, unchanged:
//   gates::composite_gen_trunc_gate(dealer, mt19937_64(seed), f, kind)
//                                           include/gates/composite_fss.hpp:645
//   gates::composite_write_tapes(kp)        include/gates/composite_fss.hpp:2610
// and checks that gates::read_composite_tape gives back the keys it wrote.
// Output: per case the gate's r_in, the pred-key count and both tapes (hex).
#include <cstdio>
#include <random>
#include <vector>

#include "gates/composite_fss.hpp"
#include "sufb200_backend.hpp"

namespace {

void hex(const std::vector<uint8_t>& b) {
  std::printf("\"");
  for (uint8_t c : b) std::printf("%02x", c);
  std::printf("\"");
}

const char* kind_name(compiler::GateKind k) {
  switch (k) {
    case compiler::GateKind::FaithfulTR: return "tr";
    case compiler::GateKind::FaithfulARS: return "ars";
    default: return "gapars";
  }
}

}  // namespace

int main() {
  struct Case {
    compiler::GateKind kind;
    int f;
    uint64_t seed;
  };
  std::vector<Case> cases;
  for (auto kind : {compiler::GateKind::FaithfulTR, compiler::GateKind::FaithfulARS, compiler::GateKind::GapARS}) {
    for (uint64_t seed : {1ull, 2ull}) cases.push_back({kind, 12, seed});
    // f = 1: seed 3 draws r_low = 1, seed 5 draws r_low = 0, where the dealer
    // drops the carry queries and the wrap share they would bring
    for (uint64_t seed : {3ull, 5ull}) cases.push_back({kind, 1, seed});
  }
  std::printf("{\"cases\":[\n");
  for (size_t c = 0; c < cases.size(); c++) {
    const Case& cs = cases[c];
    proto::SufB200Backend::Options o;
    o.dealer_only = true;
    o.deterministic = true;
    o.seed = cs.seed * 7919;
    proto::SufB200Backend dealer(o);
    std::mt19937_64 rng(cs.seed);
    auto kp = gates::composite_gen_trunc_gate(dealer, rng, cs.f, cs.kind, 1);
    auto tp = gates::composite_write_tapes(kp);
    for (int p = 0; p < 2; p++) {
      const auto& t = p ? tp.t1 : tp.t0;
      const auto& k = p ? kp.k1 : kp.k0;
      auto back = gates::read_composite_tape(t.bytes.data(), t.bytes.size());
      bool same = back.pred_keys.size() == k.pred_keys.size();
      for (size_t q = 0; same && q < k.pred_keys.size(); q++) same = back.pred_keys[q].bytes == k.pred_keys[q].bytes;
      if (!same || back.r_in_share != k.r_in_share) {
        std::fprintf(stderr, "read_composite_tape did not give back the dealt key\n");
        return 1;
      }
    }
    std::printf("{\"kind\":\"%s\",\"frac_bits\":%d,\"seed\":%llu,\"r_in\":\"%llu\",\"bit_order\":%d,\"tape0\":",
                kind_name(cs.kind), cs.f, static_cast<unsigned long long>(cs.seed),
                static_cast<unsigned long long>(kp.k0.compiled.r_in), static_cast<int>(kp.k0.pred_meta.bit_order));
    hex(tp.t0.bytes);
    std::printf(",\"tape1\":");
    hex(tp.t1.bytes);
    std::printf(",\"pred_keys\":%zu}%s\n", kp.k0.pred_keys.size(), c + 1 < cases.size() ? "," : "");
  }
  std::printf("]}\n");
  return 0;
}
