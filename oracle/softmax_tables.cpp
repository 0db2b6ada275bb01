// softmax_tables.cpp -- TEST INFRASTRUCTURE: dumps, as JSON, the SUF programs
// the reference builds for the configs[4] softmax gates, so the device block
// and the plaintext model of the block use the reference's own tables:
//   nexp : gates::make_nexp_spec(NExpGateParams{f, 16}) (include/gates/
//          nexp_gate.hpp:16, tables/nexp_piecewise_table.hpp) expanded by
//          suf::build_silu_suf_from_piecewise, as dealer_make_nexp_task_material
//          does (include/gates/nexp_composite.hpp:107-147);
//   recip: gates::make_recip_affine_init_spec(f, 1024) (tables/
//          recip_piecewise_affine_init.hpp:11) expanded the same way, as
//          dealer_make_recip_task_material does (reciprocal_composite.hpp:55-105);
//   rsqrt: gates::make_rsqrt_affine_init_spec(f, 1/1024, 16) (tables/
//          rsqrt_piecewise_affine_init.hpp) as the affine SUF of
//          oracle/rsqrt_affine_suf.hpp (the LayerNorm block's RsqrtTask init).
// With a second argument `layer` it dumps instead the two further gates of
// the device transformer layer:
//   relu      : gates::make_relu_value_suf_u64() (include/gates/relu_gate.hpp:39),
//               the row-max tournament's ReLU (nn::RowMaxDiffTask);
//   gelu_const: suf::build_gelu_suf_const_from_piecewise(
//               gates::make_gelu_spline_spec(f, 256), 64) (include/suf/
//               suf_gelu_builders.hpp:107), the degree-0 GeLU that
//               mlp_forward uses with SUF_GELU_CONST (the reference bench's
//               GPU default, src/nn/mlp_block.cpp:531-580).
// Built by oracle/Makefile (target `softmax`) into oracle/_ref/; run by
// tests/golden/make_softmax_tables.py.  Usage: softmax_tables <frac_bits> [layer].
#include <cstdio>
#include <cstdlib>

#include "gates/nexp_composite.hpp"
#include "gates/reciprocal_composite.hpp"
#include "gates/relu_gate.hpp"
#include "gates/tables/gelu_spline_table.hpp"
#include "suf/suf_gelu_builders.hpp"
#include <cstring>
#include "gates/tables/rsqrt_piecewise_affine_init.hpp"
#include "rsqrt_affine_suf.hpp"

namespace {

void dump_suf(const char* name, const suf::SUF<uint64_t>& F, bool last) {
  std::printf("  \"%s\": {\"n_bits\": %d, \"r_out\": %d, \"l_out\": %d, \"degree\": %d,\n", name, F.n_bits, F.r_out,
              F.l_out, F.degree);
  std::printf("    \"alpha\": [");
  for (size_t i = 0; i < F.alpha.size(); i++) std::printf("%s\"%llu\"", i ? ", " : "", (unsigned long long)F.alpha[i]);
  std::printf("],\n    \"pieces\": [");
  for (size_t p = 0; p < F.pieces.size(); p++) {
    std::printf("%s[", p ? ",\n      " : "\n      ");
    const auto& polys = F.pieces[p].polys;
    for (size_t j = 0; j < polys.size(); j++) {
      std::printf("%s[", j ? ", " : "");
      for (size_t k = 0; k < polys[j].coeffs.size(); k++)
        std::printf("%s\"%llu\"", k ? ", " : "", (unsigned long long)polys[j].coeffs[k]);
      std::printf("]");
    }
    std::printf("]");
  }
  std::printf("]}%s\n", last ? "" : ",");
}

}  // namespace

int main(int argc, char** argv) {
  const int f = argc > 1 ? std::atoi(argv[1]) : 12;
  if (argc > 2 && std::strcmp(argv[2], "layer") == 0) {
    std::printf("{\n  \"frac_bits\": %d,\n", f);
    dump_suf("relu", gates::make_relu_value_suf_u64(), false);
    dump_suf("gelu_const", suf::build_gelu_suf_const_from_piecewise(gates::make_gelu_spline_spec(f, 256), 64), true);
    std::printf("}\n");
    return 0;
  }
  gates::NExpGateParams np{f, 16};
  const auto nexp = suf::build_silu_suf_from_piecewise(gates::make_nexp_spec(np));
  const auto recip = suf::build_silu_suf_from_piecewise(gates::make_recip_affine_init_spec(f, 1024.0));
  const auto rsqrt = oracle_ref::rsqrt_affine_suf(gates::make_rsqrt_affine_init_spec(f, 1.0 / 1024.0, 16.0));
  std::printf("{\n  \"frac_bits\": %d,\n", f);
  dump_suf("nexp", nexp, false);
  dump_suf("recip", recip, false);
  dump_suf("rsqrt", rsqrt, true);
  std::printf("}\n");
  return 0;
}
