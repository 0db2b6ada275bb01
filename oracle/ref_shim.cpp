// ref_shim.cpp -- TEST INFRASTRUCTURE ONLY.
//
// Thin extern "C" shim compiled (by oracle/Makefile) together with the
// reference's own sources, never copied here:
//   third_party/myl7_fss/src/dcf.c, src/prg/aes128_mmo.c and one group file
//   (src/group/u128_le.c -> additive build, src/group/bytes.c -> XOR build),
//   plus the header-only adapter include/proto/myl7_fss_backend.hpp.
// The result, oracle/_ref/libmyl7ref_{add,xor}.so, runs the reference's
// actual DCF code so tests can pin oracle/suf_oracle.c and the CUDA kernels
// per share.  Only tests/ and bench.py's reference leg load it.
#include <omp.h>

#include <cstdint>
#include <cstring>
#include <stdexcept>
#include <vector>

#include <fss/dcf.h>
#include <fss/prg.h>
#include "proto/myl7_fss_backend.hpp"

namespace {
proto::Myl7FssBackend& backend() {
  static proto::Myl7FssBackend b;
  return b;
}
bool g_adapter_seeded = false;
}  // namespace

extern "C" {

// The adapter seeds the PRG once with std::random_device on its first
// gen_dcf (myl7_fss_backend.hpp:116-129).  Trigger that first, then install
// the caller's fixed PRG state so every later gen/eval uses it.
int ref_prg_init(const uint8_t* state, int len) {
  if (len < 128) return -1;
  prg_init(state, len);
  if (!g_adapter_seeded) {
    std::vector<uint8_t> alpha(8, 0);
    try {
      (void)backend().gen_dcf(8, alpha, std::vector<uint8_t>(8, 1));
    } catch (...) {
      return -2;
    }
    g_adapter_seeded = true;
  }
  prg_init(state, len);
  return 0;
}

// Adapter keygen with seeded party seeds: the adapter's serialization
// (myl7_fss_backend.hpp:131-213) around the reference dcf_gen.  seeds0/1 hold
// 16 bytes per payload chunk.
int ref_gen_seeded(int in_bits, uint64_t alpha, const uint8_t* payload, int payload_len,
                   const uint8_t* seeds0, const uint8_t* seeds1, uint8_t* key0, uint8_t* key1) {
  if (in_bits <= 0 || in_bits > 64 || payload_len <= 0) return -1;
  const size_t lambda = 16;
  const size_t chunks = (static_cast<size_t>(payload_len) + lambda - 1) / lambda;
  const size_t cw_bytes = static_cast<size_t>(in_bits) * kDcfCwLen;
  const size_t chunk_bytes = lambda + cw_bytes + lambda;
  std::vector<uint8_t> alpha_bytes((in_bits + 7) / 8, 0);
  for (int i = 0; i < in_bits; i++)
    if ((alpha >> i) & 1u) alpha_bytes[i / 8] |= static_cast<uint8_t>(1u << (i % 8));
  uint8_t* keys[2] = {key0, key1};
  for (int p = 0; p < 2; p++) {
    keys[p][0] = static_cast<uint8_t>(in_bits);
    keys[p][1] = static_cast<uint8_t>(chunks);
    keys[p][2] = static_cast<uint8_t>(p);
    keys[p][3] = 0;
    for (int b = 0; b < 4; b++) keys[p][4 + b] = static_cast<uint8_t>(static_cast<uint32_t>(payload_len) >> (8 * b));
  }
  for (size_t c = 0; c < chunks; c++) {
    size_t take = std::min(lambda, static_cast<size_t>(payload_len) - c * lambda);
    std::vector<uint8_t> padded(lambda, 0);
    std::memcpy(padded.data(), payload + c * lambda, take);
    padded[lambda - 1] &= 0x7Fu;
    std::vector<uint8_t> cws(cw_bytes, 0), np1(lambda, 0), sbuf(10 * lambda, 0);
    std::memcpy(sbuf.data(), seeds0 + c * lambda, lambda);
    std::memcpy(sbuf.data() + lambda, seeds1 + c * lambda, lambda);
    Key key{cws.data(), np1.data()};
    CmpFunc cf;
    cf.point.alpha = Bits{alpha_bytes.data(), in_bits};
    cf.point.beta = padded.data();
    cf.bound = kLtAlpha;
    dcf_gen(key, cf, sbuf.data());
    size_t off = 8 + c * chunk_bytes;
    std::memcpy(key0 + off, seeds0 + c * lambda, lambda);
    std::memcpy(key1 + off, seeds1 + c * lambda, lambda);
    std::memcpy(key0 + off + lambda, cws.data(), cw_bytes);
    std::memcpy(key1 + off + lambda, cws.data(), cw_bytes);
    std::memcpy(key0 + off + lambda + cw_bytes, np1.data(), lambda);
    std::memcpy(key1 + off + lambda + cw_bytes, np1.data(), lambda);
  }
  return 0;
}

// Unseeded keygen through the adapter itself (std::random_device seeds):
// proves that keys produced by the reference code evaluate identically.
int ref_adapter_gen(int in_bits, uint64_t alpha, const uint8_t* payload, int payload_len,
                    uint8_t* key0, uint8_t* key1, size_t key_cap) {
  try {
    auto bits = backend().u64_to_bits_msb(alpha, in_bits);
    auto kp = backend().gen_dcf(in_bits, bits, std::vector<uint8_t>(payload, payload + payload_len));
    if (kp.k0.bytes.size() > key_cap || kp.k1.bytes.size() > key_cap) return -2;
    std::memcpy(key0, kp.k0.bytes.data(), kp.k0.bytes.size());
    std::memcpy(key1, kp.k1.bytes.data(), kp.k1.bytes.size());
    return static_cast<int>(kp.k0.bytes.size());
  } catch (...) {
    return -1;
  }
}

// Per-element (broadcast=0) or broadcast evaluation through the adapter's
// eval_dcf (myl7_fss_backend.hpp:215-256).  outs is [n][out_len].
int ref_adapter_eval_many(int in_bits, const uint8_t* keys, size_t key_bytes, int broadcast,
                          const uint64_t* xs, size_t n, uint8_t* outs, int out_len) {
  try {
    const auto& b = backend();
    for (size_t i = 0; i < n; i++) {
      proto::FssKey k;
      const uint8_t* kp = keys + (broadcast ? 0 : i * key_bytes);
      k.bytes.assign(kp, kp + key_bytes);
      auto out = b.eval_dcf(in_bits, k, b.u64_to_bits_msb(xs[i], in_bits));
      if (static_cast<int>(out.size()) != out_len) return -3;
      std::memcpy(outs + i * static_cast<size_t>(out_len), out.data(), static_cast<size_t>(out_len));
    }
    return 0;
  } catch (...) {
    return -1;
  }
}

// Thread count of the OpenMP loops below (the launcher's OMP_NUM_THREADS, e.g.
// torchrun's default of 1, would otherwise decide it).  Returns the count now
// in effect.
int ref_set_threads(int n) {
  if (n > 0) omp_set_num_threads(n);
  return omp_get_max_threads();
}

// Same walk, run in parallel over elements (the harness-level OpenMP loop the
// CPU baseline uses; each call is the reference dcf_eval on one chunk).
int ref_eval_many_omp(int in_bits, const uint8_t* keys, size_t key_bytes, int broadcast,
                      const uint64_t* xs, size_t n, uint8_t* outs, int out_len) {
  if (in_bits <= 0 || in_bits > 64 || out_len <= 0 || out_len > 16) return -1;
  const size_t cw_bytes = static_cast<size_t>(in_bits) * kDcfCwLen;
  int err = 0;
#pragma omp parallel for schedule(dynamic, 256) reduction(| : err)
  for (long long ii = 0; ii < static_cast<long long>(n); ii++) {
    const size_t i = static_cast<size_t>(ii);
    const uint8_t* kp = keys + (broadcast ? 0 : i * key_bytes);
    if (kp[0] != in_bits || kp[1] != 1) { err |= 1; continue; }
    uint64_t x = xs[i];
    if (in_bits < 64) x &= (uint64_t(1) << in_bits) - 1;
    uint8_t xb[8];
    for (int b = 0; b < 8; b++) xb[b] = static_cast<uint8_t>(x >> (8 * b));
    uint8_t sbuf[6 * 16];
    std::memcpy(sbuf, kp + 8, 16);
    Key key{const_cast<uint8_t*>(kp + 8 + 16), const_cast<uint8_t*>(kp + 8 + 16 + cw_bytes)};
    dcf_eval(sbuf, kp[2], key, Bits{xb, in_bits});
    std::memcpy(outs + i * static_cast<size_t>(out_len), sbuf, static_cast<size_t>(out_len));
  }
  return err ? -2 : 0;
}

}  // extern "C"
