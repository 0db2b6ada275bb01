// dcf_walk.cuh -- the myl7 DCF tree walk (device side, one element per thread).
//
// Restates dcf_eval of third_party/myl7_fss/src/dcf.c:146-193 for the
// adapter key layout of include/proto/myl7_fss_backend.hpp:131-213
//   [in_bits u8][chunks u8][party u8][0][payload_len u32][seed 16]
//   [cw_0 .. cw_{n-1}: s_cw 16 | v_cw 16 | tl<<1|tr][cw_np1 16]
// with two changes that leave every output bit unchanged:
//   * only the child selected by x_i is expanded (2 AES blocks per level
//     instead of 4: the walk never reads the other child's seed or value);
//   * only the low 64 bits of the value accumulator are carried, since the
//     u128 group adds mod 2^127 and 2^64 divides 2^127, and payloads of at
//     most 8 bytes read only those bits.
#pragma once

#include "aes_smem.cuh"

namespace sufb200 {

struct CwLevel {
  Blk s;       // s_cw
  uint64_t v;  // low 64 bits of v_cw
  uint32_t t;  // tl<<1 | tr
};

// One level of the walk.  s/t/v are updated in place; x_bit is bit
// (n-1-i) of the input; party selects the sign of the value share.
template <int GROUP>
SUFB200_DEV void walk_level(const PrgParams& P, uint32_t lb, Blk& s, uint32_t& t, uint64_t& v, uint32_t x_bit,
                            uint32_t party, const CwLevel& cw) {
  const uint32_t xm = 0u - x_bit;
  Blk a;
  uint32_t b0, b1;
  prg_level(P, lb, s, xm, a, b0, b1);
  uint32_t tc = a.w[3] >> 31;
  a.w[3] &= 0x7FFFFFFFu;
  const uint32_t tm = 0u - t;
  a.w[0] ^= cw.s.w[0] & tm;
  a.w[1] ^= cw.s.w[1] & tm;
  a.w[2] ^= cw.s.w[2] & tm;
  a.w[3] ^= cw.s.w[3] & tm;
  // t correction: tl for x=0 (bit 1 of the byte), tr for x=1 (bit 0)
  tc ^= t & ((cw.t >> (1u - x_bit)) & 1u);
  uint64_t vc = (static_cast<uint64_t>(b1) << 32) | b0;
  const uint64_t tm64 = 0ull - static_cast<uint64_t>(t);
  if (GROUP == SUFB200_GROUP_ADD) {
    vc += cw.v & tm64;
    v += party ? (0ull - vc) : vc;
  } else {
    vc ^= cw.v & tm64;
    v ^= vc;
  }
  s = a;
  t = tc;
}

// walk_level split over a lane pair (lanes 2k, 2k+1 of the warp, pmask =
// both lanes' bits, h = lane & 1): each lane computes one of the level's two
// MMO blocks and the pair swaps them, so a level costs one AES block per lane
// instead of two.  Both lanes leave with the same s, t, v as walk_level.
#if !defined(SUFB200_HOST_EMU)
// The round keys come from prg_keys_to_smem's table (sk).
template <int GROUP>
SUFB200_DEV void walk_level_split(const uint4* sk, uint32_t lb, Blk& s, uint32_t& t, uint64_t& v, uint32_t x_bit,
                                  uint32_t party, const CwLevel& cw, uint32_t h, uint32_t pmask) {
  Blk o, e;
  prg_half_sk(sk, lb, s, x_bit, h, o);
#pragma unroll
  for (int c = 0; c < 4; c++) e.w[c] = __shfl_xor_sync(pmask, o.w[c], 1);
  Blk a;
#pragma unroll
  for (int c = 0; c < 4; c++) a.w[c] = h ? e.w[c] : o.w[c];  // block A (half 0)
  const uint32_t b0 = h ? o.w[0] : e.w[0], b1 = h ? o.w[1] : e.w[1];  // low half of block B
  uint32_t tc = a.w[3] >> 31;
  a.w[3] &= 0x7FFFFFFFu;
  const uint32_t tm = 0u - t;
  a.w[0] ^= cw.s.w[0] & tm;
  a.w[1] ^= cw.s.w[1] & tm;
  a.w[2] ^= cw.s.w[2] & tm;
  a.w[3] ^= cw.s.w[3] & tm;
  tc ^= t & ((cw.t >> (1u - x_bit)) & 1u);
  uint64_t vc = (static_cast<uint64_t>(b1) << 32) | b0;
  const uint64_t tm64 = 0ull - static_cast<uint64_t>(t);
  if (GROUP == SUFB200_GROUP_ADD) {
    vc += cw.v & tm64;
    v += party ? (0ull - vc) : vc;
  } else {
    vc ^= cw.v & tm64;
    v ^= vc;
  }
  s = a;
  t = tc;
}
#endif  // !SUFB200_HOST_EMU

// Final correction: v += (-1)^b (s + t * cw_np1) on the low 64 bits.
template <int GROUP>
SUFB200_DEV uint64_t walk_finish(const Blk& s, uint32_t t, uint64_t v, uint32_t party, uint64_t np1_lo) {
  uint64_t sl = (static_cast<uint64_t>(s.w[1]) << 32) | s.w[0];
  const uint64_t tm64 = 0ull - static_cast<uint64_t>(t);
  if (GROUP == SUFB200_GROUP_ADD) {
    sl += np1_lo & tm64;
    return v + (party ? (0ull - sl) : sl);
  }
  sl ^= np1_lo & tm64;
  return v ^ sl;
}

SUFB200_HD uint64_t funnel64(uint64_t lo, uint64_t hi, uint32_t r_bytes) {
  return r_bytes ? ((lo >> (8u * r_bytes)) | (hi << (64u - 8u * r_bytes))) : lo;
}

}  // namespace sufb200
