// tape.cu -- serialized truncation-gate keys in the reference's composite tape
// format (gates::write_composite_tape / read_composite_tape,
// include/gates/composite_fss.hpp:2458-2608; composite_write_tapes :2610).
//
// A tape is the CompositePartyKey of one party, little-endian:
//   u64 r_in_share | u32 0 (no per-element r_in vector)
//   u32 1, u64 r_out_share | u32 w, u64 wrap_share[w] | u64 r_hi_share
//   u64 wrap_sign_share | u32 2, u64 frac_bits, u64 r_low (extra_params)
//   u8 bit_order, u8 sem, u32 out_bytes (pred) | the same (cut pred)
//   u8 bit_order, u8 sem (coeff)
//   u32 nq, (u32 len, key bytes) per pred key | u32 0 cut keys | u32 0 coeff keys
//   u32 1, u64 base_coeff_share | u32 1, u64 total_delta_share
//   u32 0 triples | u32 0 bit triples
// For the gates composite_gen_trunc_gate deals (include/gates/composite_fss.hpp:
// 645-833): additive (AddU64) 8-byte predicate outputs, one constant-zero
// coefficient word (base 0, no deltas, no coefficient or cut keys), r_out = 0
// split into shares, no Beaver triples.  wrap_share holds the rotation wrap
// bits of the rewritten predicates in the compiler's order (carry's, then
// sign's).  The descriptor's haty is base + r_out share, i.e. the r_out share.
//
// Host: one gate's two tapes from this engine's dealer (sufb200_trunc_gen's
// gate and its keys), and a reader that loads a reference tape into a bundle
// descriptor.  Device: the tapes of per-element gates (sufb200_trunc_gen_elem
// material) assembled by one warp per element straight from the key slots.
#include <cstring>
#include <string>
#include <vector>

#include "kernels.hpp"
#include "keygen.hpp"
#include "sufb200_internal.cuh"

namespace {

int fail(int code, const std::string& msg) { return sufb200::record_error(code, msg); }

constexpr uint8_t kSemAddU64 = 1;  // proto::ShareSemantics::AddU64

// Bytes of a truncation-gate tape with `wraps` wrap shares and pred keys of
// the given sizes.
SUFB200_HD size_t tape_bytes(int wraps, const size_t* key_bytes, int nq) {
  size_t n = 8 + 4 + 4 + 8 + 4 + 8 * static_cast<size_t>(wraps) + 8 + 8 + 4 + 16 + 6 + 6 + 2 + 4;
  for (int q = 0; q < nq; q++) n += 4 + key_bytes[q];
  return n + 4 + 4 + 12 + 12 + 4 + 4;
}

// The fixed fields around the keys; `put` writes n little-endian bytes.
struct TapeFields {
  uint64_t r_in_share, r_out_share, r_hi, wrap_sign, f, r_low;
  uint64_t wrap[2];
  int wraps;
  uint8_t bit_order;
};

// Called with host lambdas by the host writer and device lambdas by the
// kernel; the execution-space check does not apply to either instantiation.
#pragma nv_exec_check_disable
template <typename Put, typename Keys>
SUFB200_HD void emit_tape(const TapeFields& t, int nq, const size_t* key_bytes, const Put& put, const Keys& keys) {
  put(t.r_in_share, 8);
  put(0, 4);
  put(1, 4);
  put(t.r_out_share, 8);
  put(static_cast<uint64_t>(t.wraps), 4);
  for (int w = 0; w < t.wraps; w++) put(t.wrap[w], 8);
  put(t.r_hi, 8);
  put(t.wrap_sign, 8);
  put(2, 4);
  put(t.f, 8);
  put(t.r_low, 8);
  for (int m = 0; m < 2; m++) {  // pred, cut pred
    put(t.bit_order, 1);
    put(kSemAddU64, 1);
    put(8, 4);
  }
  put(t.bit_order, 1);  // coeff
  put(kSemAddU64, 1);
  put(static_cast<uint64_t>(nq), 4);
  for (int q = 0; q < nq; q++) {
    put(key_bytes[q], 4);
    keys(q);
  }
  put(0, 4);  // cut keys
  put(0, 4);  // coeff keys
  put(1, 4);
  put(0, 8);  // base coefficient share (the constant-zero polynomial)
  put(1, 4);
  put(0, 8);  // total delta share
  put(0, 4);  // Beaver triples
  put(0, 4);  // bit triples
}

TapeFields fields_of(const sufb200_trunc_desc& d, uint64_t r_in, uint64_t r_in_share, int bit_order,
                     const sufb200::host::TruncWraps& w) {
  const int f = d.frac_bits;
  TapeFields t{};
  t.r_in_share = r_in_share;
  t.r_out_share = d.haty;
  t.r_hi = d.r_hi;
  t.wrap_sign = d.m;
  t.f = static_cast<uint64_t>(f);
  t.r_low = f <= 0 ? 0ull : (f >= 64 ? r_in : (r_in & ((1ull << f) - 1ull)));
  t.wraps = w.count;
  for (int k = 0; k < w.count; k++) t.wrap[k] = k == w.carry ? d.carry_w : d.sign_w;
  t.bit_order = static_cast<uint8_t>(bit_order);
  return t;
}

// ---- per-element tapes on the device ----------------------------------------

struct ElemTapeLaunch {
  sufb200_trunc_desc shape;
  const uint8_t* keys[4];
  size_t key_bytes[4];
  const uint64_t* words;      // [n][6] this party's dealer words
  const uint64_t* r_in;       // [n]
  const uint64_t* r_in_share; // [n] this party's
  size_t n, stride;
  uint8_t* out;               // [n][stride]
  uint64_t* len;              // [n]
  int bit_order;
};

// One warp per element: lane 0 lays out the fixed fields (a few dozen
// bytes), the warp copies each key's bytes in 32-byte coalesced runs.
__global__ void __launch_bounds__(256) trunc_tapes_elem_kernel(const ElemTapeLaunch a) {
  const size_t warp = (static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const uint32_t lane = threadIdx.x & 31u;
  const size_t nwarps = (static_cast<size_t>(gridDim.x) * blockDim.x) >> 5;
  const int f = a.shape.frac_bits;
  for (size_t i = warp; i < a.n; i += nwarps) {
    const uint64_t* w = a.words + 6 * i;
    const uint64_t plan = w[5];
    const bool carry = (plan & 0xFull) != 0xFull;
    const bool sign = ((plan >> 8) & 0xFull) != 0xFull;
    int nq = 0;
    while (nq < a.shape.nq && (a.shape.q_bits[nq] == 64 || carry)) nq++;
    const uint64_t r = a.r_in[i];
    TapeFields t{};
    t.r_in_share = a.r_in_share[i];
    t.r_out_share = w[2];
    t.r_hi = w[3];
    t.wrap_sign = w[4];
    t.f = static_cast<uint64_t>(f);
    t.r_low = f <= 0 ? 0ull : (f >= 64 ? r : (r & ((1ull << f) - 1ull)));
    t.wraps = 0;
    if (carry) t.wrap[t.wraps++] = w[0];
    if (sign) t.wrap[t.wraps++] = w[1];
    t.bit_order = static_cast<uint8_t>(a.bit_order);
    uint8_t* dst = a.out + i * a.stride;
    size_t off = 0;
    const auto put = [&](uint64_t v, int nb) {
      if (lane == 0)
        for (int b = 0; b < nb; b++) dst[off + b] = static_cast<uint8_t>(v >> (8 * b));
      off += static_cast<size_t>(nb);
    };
    const auto keys = [&](int q) {
      const size_t kb = a.key_bytes[q];
      const uint8_t* src = a.keys[q] + i * kb;
      for (size_t b = lane; b < kb; b += 32) dst[off + b] = src[b];
      off += kb;
    };
    emit_tape(t, nq, a.key_bytes, put, keys);
    if (lane == 0) a.len[i] = off;
  }
}

}  // namespace

extern "C" {

int sufb200_trunc_write_tapes(int kind, int frac_bits, uint64_t rng_seed, int bit_order, const uint8_t* const* keys0,
                              const uint8_t* const* keys1, const size_t* key_bytes, int nkeys, uint8_t* tape0,
                              uint8_t* tape1, size_t cap, size_t* len_out) {
  if (!len_out || (nkeys > 0 && !key_bytes)) return fail(SUFB200_ERR_INVALID, "null pointer");
  if (bit_order != 0 && bit_order != 1) return fail(SUFB200_ERR_INVALID, "bit_order must be 0 (MSB) or 1 (LSB)");
  sufb200_trunc_desc d[2];
  uint64_t thetas[4], r = 0, rin0 = 0;
  if (sufb200::host::trunc_gen(kind, frac_bits, rng_seed, &d[0], &d[1], thetas, &r, &rin0))
    return fail(SUFB200_ERR_INVALID, "bad truncation kind / frac_bits");
  sufb200::host::TruncWraps w;
  sufb200_trunc_desc p0, p1;
  sufb200::host::trunc_plan(kind, frac_bits, r, &p0, &p1, thetas, &w);
  if (nkeys != d[0].nq) return fail(SUFB200_ERR_INVALID, "nkeys differs from the gate's query count");
  for (int q = 0; q < nkeys; q++)
    if (key_bytes[q] != sufb200::host::myl7_key_bytes(d[0].q_bits[q], 8))
      return fail(SUFB200_ERR_KEY, "key size does not match an 8-byte myl7 key of the query's width");
  const size_t len = tape_bytes(w.count, key_bytes, nkeys);
  *len_out = len;
  if (!tape0 && !tape1) return SUFB200_OK;  // size query
  if (cap < len) return fail(SUFB200_ERR_INVALID, "tape buffer smaller than the tape");
  const uint8_t* const* keys[2] = {keys0, keys1};
  uint8_t* out[2] = {tape0, tape1};
  for (int p = 0; p < 2; p++) {
    if (!out[p]) continue;
    if (nkeys > 0 && !keys[p]) return fail(SUFB200_ERR_INVALID, "null key list");
    for (int q = 0; q < nkeys; q++)
      if (!keys[p][q]) return fail(SUFB200_ERR_INVALID, "null key");
    const TapeFields t = fields_of(d[p], r, p ? r - rin0 : rin0, bit_order, w);
    uint8_t* dst = out[p];
    size_t off = 0;
    const auto put = [&](uint64_t v, int nb) {
      for (int b = 0; b < nb; b++) dst[off + b] = static_cast<uint8_t>(v >> (8 * b));
      off += static_cast<size_t>(nb);
    };
    const auto put_key = [&](int q) {
      std::memcpy(dst + off, keys[p][q], key_bytes[q]);
      off += key_bytes[q];
    };
    emit_tape(t, nkeys, key_bytes, put, put_key);
  }
  return SUFB200_OK;
}

int sufb200_trunc_read_tape(const uint8_t* tape, size_t len, int kind, uint64_t r_in, int party,
                            sufb200_trunc_desc* desc, size_t* key_off, size_t* key_bytes, uint64_t* r_in_share) {
  if (!tape || !desc || !key_off || !key_bytes) return fail(SUFB200_ERR_INVALID, "null pointer");
  if (party != 0 && party != 1) return fail(SUFB200_ERR_INVALID, "party must be 0 or 1");
  if (kind < 0 || kind > 2) return fail(SUFB200_ERR_INVALID, "bad truncation kind");
  size_t off = 0;
  bool ok = true;
  const auto get = [&](int nb) -> uint64_t {
    if (!ok || len - off < static_cast<size_t>(nb) || off > len) {
      ok = false;
      return 0;
    }
    uint64_t v = 0;
    for (int b = 0; b < nb; b++) v |= static_cast<uint64_t>(tape[off + b]) << (8 * b);
    off += static_cast<size_t>(nb);
    return v;
  };
  const auto bad = [&](const char* what) { return fail(SUFB200_ERR_KEY, std::string("composite tape: ") + what); };
  const uint64_t rin_share = get(8);
  if (get(4) != 0) return bad("per-element r_in vector is not a truncation gate's");
  if (get(4) != 1) return bad("expected one r_out share");
  const uint64_t rout = get(8);
  const uint64_t nwrap = get(4);
  if (!ok || nwrap > 2) return bad("wrap share count out of range");
  uint64_t wrap[2] = {0, 0};
  for (uint64_t k = 0; k < nwrap; k++) wrap[k] = get(8);
  const uint64_t r_hi = get(8), wrap_sign = get(8);
  if (get(4) != 2) return bad("expected the two truncation parameters (frac_bits, r_low)");
  const uint64_t f = get(8), r_low = get(8);
  if (!ok || f > 64) return bad("frac_bits out of range");
  for (int m = 0; m < 2; m++) {
    get(1);
    if (get(1) != kSemAddU64 || get(4) != 8) return bad("predicate outputs are not additive 8-byte words");
  }
  get(1);
  if (get(1) != kSemAddU64) return bad("coefficient shares are not additive");
  sufb200_trunc_desc d[2];
  uint64_t thetas[4];
  sufb200::host::TruncWraps w;
  if (sufb200::host::trunc_plan(kind, static_cast<int>(f), r_in, &d[0], &d[1], thetas, &w))
    return bad("bad truncation parameters");
  const uint64_t fm = f >= 64 ? ~0ull : ((1ull << f) - 1ull);
  if (r_low != ((f == 0) ? 0ull : (r_in & fm))) return bad("r_low does not match r_in");
  if (nwrap != static_cast<uint64_t>(w.count)) return bad("wrap share count does not match the gate");
  const uint64_t nq = get(4);
  if (!ok || nq != static_cast<uint64_t>(d[0].nq)) return bad("pred key count does not match the gate");
  for (int q = 0; q < static_cast<int>(nq); q++) {
    const uint64_t kb = get(4);
    if (!ok || kb != sufb200::host::myl7_key_bytes(d[0].q_bits[q], 8)) return bad("pred key size mismatch");
    if (len - off < kb) return bad("truncated");
    key_off[q] = off;
    key_bytes[q] = kb;
    off += kb;
  }
  if (get(4) != 0 || get(4) != 0) return bad("cut or coefficient keys are not a truncation gate's");
  if (get(4) != 1) return bad("expected one base coefficient word");
  const uint64_t base = get(8);
  if (get(4) != 1) return bad("expected one total-delta word");
  get(8);
  if (get(4) != 0 || get(4) != 0) return bad("Beaver triples are not a truncation gate's");
  if (!ok) return bad("truncated");
  if (off != len) return bad("trailing bytes");
  sufb200_trunc_desc out = d[party];
  out.haty = base + rout;
  out.carry_w = w.carry >= 0 ? wrap[w.carry] : 0ull;
  out.sign_w = w.sign >= 0 ? wrap[w.sign] : 0ull;
  out.r_hi = r_hi;
  out.m = wrap_sign;
  *desc = out;
  if (r_in_share) *r_in_share = rin_share;
  return SUFB200_OK;
}

int sufb200_trunc_gen_elem_rin_shares(int kind, int frac_bits, uint64_t rng_seed, size_t n, uint64_t* share0) {
  if (n && !share0) return fail(SUFB200_ERR_INVALID, "null pointer");
  int err = 0;
#pragma omp parallel for schedule(static, 4096) reduction(| : err)
  for (long long ii = 0; ii < static_cast<long long>(n); ii++) {
    const size_t i = static_cast<size_t>(ii);
    sufb200_trunc_desc e0, e1;
    uint64_t th[4], r = 0;
    err |= sufb200::host::trunc_gen(kind, frac_bits, rng_seed + static_cast<uint64_t>(i) * 0x9E3779B97F4A7C15ull, &e0,
                                    &e1, th, &r, &share0[i]);
  }
  return err ? fail(SUFB200_ERR_INVALID, "bad truncation kind / frac_bits") : SUFB200_OK;
}

size_t sufb200_trunc_tape_elem_stride(const sufb200_trunc_desc* shape, const size_t* key_bytes) {
  if (!shape || !key_bytes || shape->nq < 0 || shape->nq > 4) return 0;
  const int wraps = (shape->kind == SUFB200_TRUNC_FAITHFUL_ARS ? 1 : 0) + (shape->frac_bits > 0 ? 1 : 0);
  return (tape_bytes(wraps, key_bytes, shape->nq) + 15) / 16 * 16;
}

int sufb200_trunc_write_tapes_elem(sufb200_ctx ctx, const sufb200_trunc_desc* shape, const uint8_t* const* d_keys,
                                   const size_t* key_bytes, const uint64_t* d_words, const uint64_t* d_r_in,
                                   const uint64_t* d_r_in_share, size_t n, int bit_order, uint8_t* d_out,
                                   size_t stride, uint64_t* d_len, void* stream) {
  if (!ctx || !shape || !d_keys || !key_bytes) return fail(SUFB200_ERR_INVALID, "null pointer");
  if (ctx->device < 0) return fail(SUFB200_ERR_UNSUPPORTED, "host-only context: no device");
  if (shape->nq < 0 || shape->nq > 4 || shape->kind < 0 || shape->kind > 2 || shape->frac_bits < 0 ||
      shape->frac_bits > 64)
    return fail(SUFB200_ERR_INVALID, "bad per-element shape");
  if (bit_order != 0 && bit_order != 1) return fail(SUFB200_ERR_INVALID, "bit_order must be 0 (MSB) or 1 (LSB)");
  if (stride < sufb200_trunc_tape_elem_stride(shape, key_bytes))
    return fail(SUFB200_ERR_INVALID, "stride below sufb200_trunc_tape_elem_stride");
  if (n == 0) return SUFB200_OK;
  if (!d_words || !d_r_in || !d_r_in_share || !d_out || !d_len) return fail(SUFB200_ERR_INVALID, "null device pointer");
  ElemTapeLaunch a{};
  a.shape = *shape;
  for (int q = 0; q < shape->nq; q++) {
    if (!d_keys[q]) return fail(SUFB200_ERR_INVALID, "null key slot");
    if (key_bytes[q] != sufb200::host::myl7_key_bytes(shape->q_bits[q], 8))
      return fail(SUFB200_ERR_KEY, "key size does not match an 8-byte myl7 key of the slot's width");
    a.keys[q] = d_keys[q];
    a.key_bytes[q] = key_bytes[q];
  }
  a.words = d_words;
  a.r_in = d_r_in;
  a.r_in_share = d_r_in_share;
  a.n = n;
  a.stride = stride;
  a.out = d_out;
  a.len = d_len;
  a.bit_order = bit_order;
  cudaError_t e = cudaSetDevice(ctx->device);
  if (e != cudaSuccess) return fail(SUFB200_ERR_CUDA, std::string("cudaSetDevice: ") + cudaGetErrorString(e));
  const size_t warps = n;
  size_t blocks = (warps * 32 + 255) / 256;
  const size_t cap = static_cast<size_t>(ctx->sm_count) * 8;
  if (blocks > cap) blocks = cap;
  trunc_tapes_elem_kernel<<<static_cast<int>(blocks), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(a);
  e = cudaGetLastError();
  return e == cudaSuccess ? SUFB200_OK
                          : fail(SUFB200_ERR_CUDA, std::string("per-element tape launch: ") + cudaGetErrorString(e));
}

}  // extern "C"
