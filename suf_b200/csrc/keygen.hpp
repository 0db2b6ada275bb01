// keygen.hpp -- dealer-side key generation (keygen.cpp).
#pragma once

#include <cstddef>
#include <cstdint>

#include "../../include/sufb200.h"

namespace sufb200 {
namespace host {

// The four fixed MMO keys' schedules as 44 little-endian words each.
struct PrgHostKeys {
  uint32_t rk[4][44];
};

void myl7_dcf_gen_chunk(const PrgHostKeys& prg, bool add_group, int in_bits, uint64_t alpha, const uint8_t beta[16],
                        const uint8_t seed0[16], const uint8_t seed1[16], uint8_t* cws, uint8_t cw_np1[16]);
size_t myl7_key_bytes(int in_bits, int payload_len);
int myl7_gen_pair(const PrgHostKeys& prg, bool add_group, int in_bits, uint64_t alpha, const uint8_t* payload,
                  int payload_len, const uint8_t* seeds0, const uint8_t* seeds1, uint8_t* key0, uint8_t* key1);
int myl7_gen_batch(const PrgHostKeys& prg, bool add_group, int in_bits, const uint64_t* alphas, size_t n,
                   const uint8_t* payload, int payload_len, const uint8_t* seeds0, const uint8_t* seeds1,
                   uint8_t* keys0, uint8_t* keys1);
// The rotation wrap bits of a truncation gate's rewritten predicates, in the
// compiler's order (compiled.wrap_bits): carry's (when r_low != 0), then
// sign's (FaithfulARS); carry / sign = their index, -1 when absent.
struct TruncWraps {
  int count;
  int carry, sign;
  uint64_t bit[2];
};
// The query plan of a truncation gate with mask r (no randomness): both
// parties' descriptors without shares, the nq thresholds and the wrap bits.
int trunc_plan(int kind, int f, uint64_t r, sufb200_trunc_desc* d0, sufb200_trunc_desc* d1, uint64_t thetas[4],
               TruncWraps* wraps);
int trunc_gen(int kind, int f, uint64_t seed, sufb200_trunc_desc* d0, sufb200_trunc_desc* d1, uint64_t thetas[4],
              uint64_t* r_in_out, uint64_t* r_in_share0 = nullptr);
int trunc_gen_elem(int kind, int f, uint64_t seed, size_t n, sufb200_trunc_desc* shape0, sufb200_trunc_desc* shape1,
                   uint64_t* words0, uint64_t* words1, uint64_t* thetas, uint64_t* r_in);
void seed_from_id(uint64_t id, uint64_t tweak, uint8_t seed[16]);
size_t thr_dcf_build(int in_bits, uint64_t alpha, const uint8_t* payload, int payload_len, uint8_t* out);
size_t packed_lt_build(int party, uint64_t nonce, int in_bits, const uint64_t* thr, int num_thr,
                       const uint8_t seed[16], uint8_t* out);
size_t interval_lut_build(int party, uint64_t nonce, int in_bits, int out_words, const uint64_t* cuts, int intervals,
                          const uint64_t* payload, const uint8_t seed[16], uint8_t* out);

}  // namespace host
}  // namespace sufb200
