// rsqrt_affine_suf.hpp -- TEST INFRASTRUCTURE (oracle/): the SUF program of
// the affine rsqrt initial guess used by the configs[4] LayerNorm block.
#pragma once

#include <algorithm>
#include <cstdint>

#include "gates/piecewise_poly.hpp"
#include "suf/suf_ir.hpp"

namespace oracle_ref {

// The affine rsqrt-init SUF: per interval [start, end) of the reference's
// spec with pack (a0, a1, offset), the piece outputs c0 = a0 - (a1 offset >>
// frac_in) and c1 = a1, so that c0 + (c1 x >> f) is the chord on x directly;
// a zero piece covers [0, first start).  The construction the reference's
// softmax/norm bench uses for RsqrtTask (src/bench/bench_softmax_norm.cpp:
// 264-311), restated.
inline suf::SUF<uint64_t> rsqrt_affine_suf(const gates::PiecewisePolySpec& spec) {
  suf::SUF<uint64_t> F;
  F.n_bits = 64;
  F.r_out = 2;
  F.l_out = 0;
  F.degree = 0;
  auto iv = spec.intervals;
  std::sort(iv.begin(), iv.end(), [](const auto& a, const auto& b) { return a.start < b.start; });
  if (iv.empty()) return F;
  auto piece = [](uint64_t c0, uint64_t c1) {
    suf::SufPiece<uint64_t> p;
    p.polys.resize(2);
    p.polys[0].coeffs = {c0};
    p.polys[1].coeffs = {c1};
    return p;
  };
  if (iv.front().start != 0) {
    F.alpha.push_back(0);
    F.pieces.push_back(piece(0, 0));
  }
  F.alpha.push_back(iv.front().start);
  for (const auto& v : iv) {
    const int64_t a0 = v.pack.coeffs.empty() ? 0 : v.pack.coeffs[0];
    const int64_t a1 = v.pack.coeffs.size() > 1 ? v.pack.coeffs[1] : 0;
    const int64_t off = static_cast<int64_t>((static_cast<__int128>(a1) * v.pack.offset) >> spec.frac_bits_in);
    F.pieces.push_back(piece(static_cast<uint64_t>(a0 - off), static_cast<uint64_t>(a1)));
    F.alpha.push_back(v.end);
  }
  return F;
}

}  // namespace oracle_ref
