// keygen.cpp -- dealer-side (host) key generation.
//
// * myl7 DCF keys: dcf_gen of third_party/myl7_fss/src/dcf.c:42-142 with
//   the AES-128-MMO PRG of src/prg/aes128_mmo.c:41-53, serialized in the
//   adapter layout of include/proto/myl7_fss_backend.hpp:131-213.
// * truncation bundles: the mask / share schedule of composite_gen_trunc_gate
//   (include/gates/composite_fss.hpp:645-833) and the query rewrite of
//   src/compiler/suf_to_pfss.cpp:55-92,443-496 with suf/mask_rewrite.hpp.
// * reference GPU-backend blobs (cuda/pfss_backend_gpu.cu:189-288).
#include <algorithm>
#include <cstring>
#include <random>
#include <vector>

#include "host_aes.hpp"
#include "keygen.hpp"

namespace sufb200 {
namespace host {

namespace {

using u128 = unsigned __int128;
constexpr u128 kM127 = (static_cast<u128>(1) << 127) - 1;

inline u128 load128(const uint8_t* p) {
  uint64_t lo, hi;
  std::memcpy(&lo, p, 8);
  std::memcpy(&hi, p + 8, 8);
  return (static_cast<u128>(hi) << 64) | lo;
}
inline void store128(uint8_t* p, u128 v) {
  const uint64_t lo = static_cast<uint64_t>(v), hi = static_cast<uint64_t>(v >> 64);
  std::memcpy(p, &lo, 8);
  std::memcpy(p + 8, &hi, 8);
}

struct Group {
  bool add;
  u128 plus(u128 a, u128 b) const { return add ? ((a + b) & kM127) : (a ^ b); }
  u128 neg(u128 a) const { return add ? ((static_cast<u128>(0) - a) & kM127) : a; }
};

inline u128 mmo(const PrgHostKeys& prg, int j, u128 seed) {
  uint8_t in[16], out[16];
  store128(in, seed);
  aes128_encrypt(prg.rk[j], in, out);
  return load128(out) ^ seed;
}

}  // namespace

void myl7_dcf_gen_chunk(const PrgHostKeys& prg, bool add_group, int in_bits, uint64_t alpha, const uint8_t beta[16],
                        const uint8_t seed0[16], const uint8_t seed1[16], uint8_t* cws, uint8_t cw_np1[16]) {
  const Group g{add_group};
  u128 s0 = load128(seed0) & kM127, s1 = load128(seed1) & kM127;
  unsigned t0 = 0, t1 = 1;
  u128 v = 0;
  const u128 b = load128(beta) & kM127;
  for (int i = 0; i < in_bits; i++) {
    u128 p0[4], p1[4];
    for (int j = 0; j < 4; j++) {
      p0[j] = mmo(prg, j, s0);
      p1[j] = mmo(prg, j, s1);
    }
    const unsigned t0l = static_cast<unsigned>(p0[0] >> 127), t0r = static_cast<unsigned>(p0[2] >> 127);
    const unsigned t1l = static_cast<unsigned>(p1[0] >> 127), t1r = static_cast<unsigned>(p1[2] >> 127);
    for (int j = 0; j < 4; j++) {
      p0[j] &= kM127;
      p1[j] &= kM127;
    }
    const unsigned a = static_cast<unsigned>((alpha >> (in_bits - 1 - i)) & 1u);
    const int lose = a ? 0 : 2, keep = a ? 2 : 0;
    const u128 s_cw = p0[lose] ^ p1[lose];
    u128 v_cw = g.plus(g.plus(p1[lose + 1], g.neg(p0[lose + 1])), g.neg(v));
    if (t1) v_cw = g.neg(v_cw);
    if (a) v_cw = g.plus(v_cw, t1 ? g.neg(b) : b);  // bound kLtAlpha
    v = g.plus(g.plus(g.plus(v, g.neg(p1[keep + 1])), p0[keep + 1]), t1 ? g.neg(v_cw) : v_cw);
    const unsigned tl_cw = t0l ^ t1l ^ a ^ 1u, tr_cw = t0r ^ t1r ^ a;
    uint8_t* cw = cws + static_cast<size_t>(i) * 33;
    store128(cw, s_cw);
    store128(cw + 16, v_cw);
    cw[32] = static_cast<uint8_t>((tl_cw << 1) | tr_cw);
    const unsigned tk = a ? tr_cw : tl_cw;
    const unsigned t0k = a ? t0r : t0l, t1k = a ? t1r : t1l;
    s0 = p0[keep] ^ (t0 ? s_cw : 0);
    s1 = p1[keep] ^ (t1 ? s_cw : 0);
    t0 = t0k ^ (t0 & tk);
    t1 = t1k ^ (t1 & tk);
  }
  u128 last = g.plus(g.plus(s1, g.neg(s0)), g.neg(v));
  if (t1) last = g.neg(last);
  store128(cw_np1, last);
}

size_t myl7_key_bytes(int in_bits, int payload_len) {
  const size_t chunks = static_cast<size_t>(payload_len + 15) / 16;
  return 8 + chunks * (32 + 33 * static_cast<size_t>(in_bits));
}

int myl7_gen_pair(const PrgHostKeys& prg, bool add_group, int in_bits, uint64_t alpha, const uint8_t* payload,
                  int payload_len, const uint8_t* seeds0, const uint8_t* seeds1, uint8_t* key0, uint8_t* key1) {
  if (in_bits <= 0 || in_bits > 64 || payload_len <= 0) return -1;
  const int chunks = (payload_len + 15) / 16;
  if (chunks > 255) return -1;
  if (in_bits < 64) alpha &= (1ull << in_bits) - 1ull;
  const size_t cw_bytes = 33 * static_cast<size_t>(in_bits), chunk_bytes = 32 + cw_bytes;
  uint8_t* keys[2] = {key0, key1};
  for (int p = 0; p < 2; p++) {
    keys[p][0] = static_cast<uint8_t>(in_bits);
    keys[p][1] = static_cast<uint8_t>(chunks);
    keys[p][2] = static_cast<uint8_t>(p);
    keys[p][3] = 0;
    const uint32_t pl = static_cast<uint32_t>(payload_len);
    std::memcpy(keys[p] + 4, &pl, 4);
  }
  std::vector<uint8_t> cws(cw_bytes);
  for (int c = 0; c < chunks; c++) {
    uint8_t beta[16] = {0};
    const int take = payload_len - 16 * c < 16 ? payload_len - 16 * c : 16;
    std::memcpy(beta, payload + 16 * c, static_cast<size_t>(take));
    beta[15] &= 0x7F;
    uint8_t np1[16];
    myl7_dcf_gen_chunk(prg, add_group, in_bits, alpha, beta, seeds0 + 16 * c, seeds1 + 16 * c, cws.data(), np1);
    const size_t off = 8 + static_cast<size_t>(c) * chunk_bytes;
    std::memcpy(key0 + off, seeds0 + 16 * c, 16);
    std::memcpy(key1 + off, seeds1 + 16 * c, 16);
    std::memcpy(key0 + off + 16, cws.data(), cw_bytes);
    std::memcpy(key1 + off + 16, cws.data(), cw_bytes);
    std::memcpy(key0 + off + 16 + cw_bytes, np1, 16);
    std::memcpy(key1 + off + 16 + cw_bytes, np1, 16);
  }
  return 0;
}

int myl7_gen_batch(const PrgHostKeys& prg, bool add_group, int in_bits, const uint64_t* alphas, size_t n,
                   const uint8_t* payload, int payload_len, const uint8_t* seeds0, const uint8_t* seeds1,
                   uint8_t* keys0, uint8_t* keys1) {
  const size_t kb = myl7_key_bytes(in_bits, payload_len);
  const size_t sb = 16 * static_cast<size_t>((payload_len + 15) / 16);
  int err = 0;
#pragma omp parallel for schedule(dynamic, 256) reduction(| : err)
  for (long long ii = 0; ii < static_cast<long long>(n); ii++) {
    const size_t i = static_cast<size_t>(ii);
    err |= myl7_gen_pair(prg, add_group, in_bits, alphas[i], payload, payload_len, seeds0 + i * sb, seeds1 + i * sb,
                         keys0 + i * kb, keys1 + i * kb) != 0;
  }
  return err ? -1 : 0;
}

// ---- truncation bundles ---------------------------------------------------

int trunc_plan(int kind, int f, uint64_t r, sufb200_trunc_desc* d0, sufb200_trunc_desc* d1, uint64_t thetas[4],
               TruncWraps* wraps) {
  if (kind < 0 || kind > 2 || f < 0 || f > 64) return -1;
  const uint64_t fmask = f >= 64 ? ~0ull : ((1ull << f) - 1ull);
  const uint64_t r_low = r & fmask;
  struct Q {
    int kind;  // 0 = LtU64, 1 = LtLow (RawPredKind order)
    int bits;
    uint64_t theta;
    int tag;  // 0 carry.a 1 carry.b 2 sign.a 3 sign.b 4 wrap
  };
  std::vector<Q> raw;
  TruncWraps w{};
  w.carry = w.sign = -1;
  // carry = NOT(1[x_low < 2^f - r_low]), rewritten by rewrite_ltlow
  if (f > 0 && f < 64 && r_low != 0) {
    const uint64_t gamma = (1ull << f) - r_low;
    const uint64_t th0 = r_low, th1 = (r_low + gamma) & fmask;
    raw.push_back({1, f, th0, 0});
    raw.push_back({1, f, th1, 1});
    w.carry = w.count;
    w.bit[w.count++] = th1 < th0 ? 1u : 0u;
  }
  // sign = MSB(x), rewritten by rewrite_msb_add(r, 0)
  if (kind == SUFB200_TRUNC_FAITHFUL_ARS) {
    const uint64_t th0 = r + (1ull << 63), th1 = th0 + (1ull << 63);
    raw.push_back({0, 64, th0, 2});
    raw.push_back({0, 64, th1, 3});
    w.sign = w.count;
    w.bit[w.count++] = th1 < th0 ? 1u : 0u;
  }
  // wrap = 1[x^ < r_in] for the faithful kinds
  if (kind != SUFB200_TRUNC_GAPARS) raw.push_back({0, 64, r, 4});
  // dedup in first-seen order, then stable sort by (kind, bits, theta)
  std::vector<Q> uq;
  std::vector<int> map(raw.size());
  for (size_t i = 0; i < raw.size(); i++) {
    int found = -1;
    for (size_t j = 0; j < uq.size(); j++)
      if (uq[j].kind == raw[i].kind && uq[j].bits == raw[i].bits && uq[j].theta == raw[i].theta)
        found = static_cast<int>(j);
    if (found < 0) {
      found = static_cast<int>(uq.size());
      uq.push_back(raw[i]);
    }
    map[i] = found;
  }
  std::vector<int> order(uq.size());
  for (size_t i = 0; i < order.size(); i++) order[i] = static_cast<int>(i);
  std::stable_sort(order.begin(), order.end(), [&](int x, int y) {
    const Q &a = uq[x], &b = uq[y];
    if (a.kind != b.kind) return a.kind < b.kind;
    if (a.bits != b.bits) return a.bits < b.bits;
    return a.theta < b.theta;
  });
  std::vector<int> new_of_old(uq.size());
  for (size_t i = 0; i < order.size(); i++) new_of_old[order[i]] = static_cast<int>(i);
  int q_of_tag[5] = {-1, -1, -1, -1, -1};
  for (size_t i = 0; i < raw.size(); i++) q_of_tag[raw[i].tag] = new_of_old[map[i]];

  sufb200_trunc_desc* d[2] = {d0, d1};
  for (int p = 0; p < 2; p++) {
    std::memset(d[p], 0, sizeof(sufb200_trunc_desc));
    d[p]->kind = kind;
    d[p]->frac_bits = f;
    d[p]->party = p;
    d[p]->nq = static_cast<int32_t>(uq.size());
    for (size_t i = 0; i < order.size(); i++) d[p]->q_bits[i] = uq[order[i]].bits;
    d[p]->carry_a = q_of_tag[0];
    d[p]->carry_b = q_of_tag[1];
    d[p]->sign_a = q_of_tag[2];
    d[p]->sign_b = q_of_tag[3];
    d[p]->wrap_q = q_of_tag[4];
  }
  for (int i = 0; i < 4; i++) thetas[i] = i < static_cast<int>(order.size()) ? uq[order[i]].theta : 0ull;
  if (wraps) *wraps = w;
  return 0;
}

int trunc_gen(int kind, int f, uint64_t seed, sufb200_trunc_desc* d0, sufb200_trunc_desc* d1, uint64_t thetas[4],
              uint64_t* r_in_out, uint64_t* r_in_share0) {
  if (kind < 0 || kind > 2 || f < 0 || f > 64) return -1;
  std::mt19937_64 rng(seed);
  const uint64_t r = rng();
  const uint64_t r_hi = f >= 64 ? 0ull : (r >> f);
  TruncWraps w;
  if (trunc_plan(kind, f, r, d0, d1, thetas, &w)) return -1;
  // share splits in composite_gen_trunc_gate order: r_in, r_out, wrap bits, r_hi, m
  const uint64_t rin0 = rng();  // r_in share of party 0; party 1 holds r - rin0
  const uint64_t rout0 = rng();
  d0->haty = rout0;  // base coefficient 0, r_out = 0
  d1->haty = 0ull - rout0;
  for (int k = 0; k < w.count; k++) {
    const uint64_t w0 = rng(), w1 = w.bit[k] - w0;
    if (k == w.carry) {
      d0->carry_w = w0;
      d1->carry_w = w1;
    }
    if (k == w.sign) {
      d0->sign_w = w0;
      d1->sign_w = w1;
    }
  }
  const uint64_t rh0 = rng();
  d0->r_hi = rh0;
  d1->r_hi = r_hi - rh0;
  uint64_t m = 0;
  if (kind == SUFB200_TRUNC_GAPARS && f > 0 && f < 64) m = (r >> 63) ? (1ull << (64 - f)) : 0ull;
  const uint64_t m0 = rng();
  d0->m = kind == SUFB200_TRUNC_GAPARS ? m0 : 0ull;
  d1->m = kind == SUFB200_TRUNC_GAPARS ? (m - m0) : 0ull;
  if (r_in_out) *r_in_out = r;
  if (r_in_share0) *r_in_share0 = rin0;
  return 0;
}

// Per-element masks (SUF_PER_ELEMENT_MASKS=1): every element gets a gate of
// its own, as compiler::lower_truncation_gate does with per_element_masks
// (include/compiler/truncation_lowering.hpp:91-125: one
// composite_gen_trunc_gate per element).  Element i's gate is
// trunc_gen(kind, f, seed_i) with seed_i = seed + i * 0x9E3779B97F4A7C15.
// Its queries fill fixed slots: the 64-bit queries first, then the two f-bit
// carry queries, as trunc_gen sorts them; when an element has no carry
// queries (r_low = 0: the carry is the constant 0 and the reference drops
// the queries) its f-bit slots get keys for threshold 0 and its plan marks
// the carry absent.  Per element and party, words[6] = carry_w, sign_w,
// haty, r_hi, m and the plan: the five query indices carry_a, carry_b,
// sign_a, sign_b, wrap_q, 4 bits each (0xF = absent).  shape gets kind, f,
// party, the slot count and slot widths.
int trunc_gen_elem(int kind, int f, uint64_t seed, size_t n, sufb200_trunc_desc* shape0, sufb200_trunc_desc* shape1,
                   uint64_t* words0, uint64_t* words1, uint64_t* thetas, uint64_t* r_in) {
  if (kind < 0 || kind > 2 || f < 0 || f > 64) return -1;
  const int wide = kind == SUFB200_TRUNC_FAITHFUL_ARS ? 2 : (kind == SUFB200_TRUNC_FAITHFUL_TR ? 1 : 0);
  const int low = (f > 0 && f < 64) ? 2 : 0;
  const int slots = wide + low;
  sufb200_trunc_desc* sh[2] = {shape0, shape1};
  for (int p = 0; p < 2; p++) {
    std::memset(sh[p], 0, sizeof(sufb200_trunc_desc));
    sh[p]->kind = kind;
    sh[p]->frac_bits = f;
    sh[p]->party = p;
    sh[p]->nq = slots;
    for (int q = 0; q < slots; q++) sh[p]->q_bits[q] = q < wide ? 64 : f;
    sh[p]->carry_a = sh[p]->carry_b = sh[p]->sign_a = sh[p]->sign_b = sh[p]->wrap_q = -1;
  }
  int err = 0;
#pragma omp parallel for schedule(static, 4096) reduction(| : err)
  for (long long ii = 0; ii < static_cast<long long>(n); ii++) {
    const size_t i = static_cast<size_t>(ii);
    sufb200_trunc_desc e0, e1;
    uint64_t th[4], r = 0;
    if (trunc_gen(kind, f, seed + static_cast<uint64_t>(i) * 0x9E3779B97F4A7C15ull, &e0, &e1, th, &r)) {
      err |= 1;
      continue;
    }
    // the element's queries are the first e0.nq slots; missing carry slots
    // (r_low = 0) get threshold 0
    if (e0.nq != slots && e0.nq != wide) {
      err |= 2;
      continue;
    }
    for (int q = 0; q < 4; q++) thetas[4 * i + q] = q < e0.nq ? th[q] : 0ull;
    auto nib = [](int32_t v) -> uint64_t { return v < 0 ? 0xFull : static_cast<uint64_t>(v); };
    const uint64_t plan = nib(e0.carry_a) | (nib(e0.carry_b) << 4) | (nib(e0.sign_a) << 8) | (nib(e0.sign_b) << 12) |
                          (nib(e0.wrap_q) << 16);
    const sufb200_trunc_desc* e[2] = {&e0, &e1};
    uint64_t* w[2] = {words0 + 6 * i, words1 + 6 * i};
    for (int p = 0; p < 2; p++) {
      w[p][0] = e[p]->carry_w;
      w[p][1] = e[p]->sign_w;
      w[p][2] = e[p]->haty;
      w[p][3] = e[p]->r_hi;
      w[p][4] = e[p]->m;
      w[p][5] = plan;
    }
    r_in[i] = r;
  }
  return err ? -1 : 0;
}

// ---- reference GPU-backend blobs ------------------------------------------

void seed_from_id(uint64_t id, uint64_t tweak, uint8_t seed[16]) {
  std::mt19937_64 rng(id ^ (tweak * 0x9e3779b97f4a7c15ull));
  for (int i = 0; i < 16; i++) seed[i] = static_cast<uint8_t>(rng() & 0xFFu);
}

static inline uint64_t mask_bits(int bits) { return bits <= 0 ? 0 : (bits >= 64 ? ~0ull : ((1ull << bits) - 1)); }

size_t thr_dcf_build(int in_bits, uint64_t alpha, const uint8_t* payload, int payload_len, uint8_t* out) {
  const size_t bytes = 12 + static_cast<size_t>(payload_len);
  if (!out) return bytes;
  const uint16_t ib = static_cast<uint16_t>(in_bits), pl = static_cast<uint16_t>(payload_len);
  std::memcpy(out, &ib, 2);
  std::memcpy(out + 2, &pl, 2);
  const uint64_t a = alpha & mask_bits(in_bits);
  std::memcpy(out + 4, &a, 8);
  if (payload_len > 0) {
    if (payload) std::memcpy(out + 12, payload, static_cast<size_t>(payload_len));
    else std::memset(out + 12, 0, static_cast<size_t>(payload_len));
  }
  return bytes;
}

size_t packed_lt_build(int party, uint64_t nonce, int in_bits, const uint64_t* thr, int num_thr,
                       const uint8_t seed[16], uint8_t* out) {
  const size_t bytes = 208 + 8 * static_cast<size_t>(num_thr);
  if (!out) return bytes;
  std::memset(out, 0, 208);
  const uint16_t ib = static_cast<uint16_t>(in_bits), nt = static_cast<uint16_t>(num_thr);
  std::memcpy(out, &ib, 2);
  std::memcpy(out + 2, &nt, 2);
  out[4] = static_cast<uint8_t>(party);
  std::memcpy(out + 8, &nonce, 8);
  std::memcpy(out + 16, seed, 16);
  aes128_expand_bytes(seed, out + 32);
  const uint64_t m = mask_bits(in_bits);
  bool sorted = true;
  uint64_t prev = 0;
  for (int i = 0; i < num_thr; i++) {
    const uint64_t v = thr[i] & m;
    std::memcpy(out + 208 + 8 * static_cast<size_t>(i), &v, 8);
    if (i > 0 && v < prev) sorted = false;
    prev = v;
  }
  out[5] = sorted ? 1 : 0;
  return bytes;
}

size_t interval_lut_build(int party, uint64_t nonce, int in_bits, int out_words, const uint64_t* cuts, int intervals,
                          const uint64_t* payload, const uint8_t seed[16], uint8_t* out) {
  const size_t bytes = 216 + 8 * (static_cast<size_t>(intervals) + 1) +
                       8 * static_cast<size_t>(intervals) * static_cast<size_t>(out_words);
  if (!out) return bytes;
  std::memset(out, 0, 216);
  const uint16_t ib = static_cast<uint16_t>(in_bits), ow = static_cast<uint16_t>(out_words);
  const uint32_t iv = static_cast<uint32_t>(intervals);
  std::memcpy(out, &ib, 2);
  std::memcpy(out + 2, &ow, 2);
  std::memcpy(out + 4, &iv, 4);
  out[8] = static_cast<uint8_t>(party);
  std::memcpy(out + 16, &nonce, 8);
  std::memcpy(out + 24, seed, 16);
  aes128_expand_bytes(seed, out + 40);
  std::memcpy(out + 216, cuts, 8 * (static_cast<size_t>(intervals) + 1));
  std::memcpy(out + 216 + 8 * (static_cast<size_t>(intervals) + 1), payload,
              8 * static_cast<size_t>(intervals) * static_cast<size_t>(out_words));
  return bytes;
}

}  // namespace host
}  // namespace sufb200
