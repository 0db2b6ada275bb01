// host_aes.hpp -- host-side AES-128 for the dealer (keygen) and for building
// the device tables.  Written from FIPS-197: the S-box is derived from the
// multiplicative inverse in GF(2^8) followed by the affine map, and the
// encryption uses little-endian column T-tables derived from it.  The
// AES-NI path (Intel's AESENC/AESENCLAST instructions, used through the
// compiler intrinsics) is taken when the host CPU reports the feature.
#pragma once

#include <array>
#include <cstdint>
#include <cstring>

#if defined(__x86_64__)
#include <immintrin.h>
#endif

namespace sufb200 {
namespace host {

struct AesTables {
  uint8_t sbox[256];
  uint32_t t0[256];  // LE column word 2S | S<<8 | S<<16 | 3S<<24
};

inline uint8_t gf_mul(uint8_t a, uint8_t b) {
  uint8_t r = 0;
  while (b) {
    if (b & 1) r ^= a;
    const uint8_t hi = a & 0x80;
    a = static_cast<uint8_t>(a << 1);
    if (hi) a ^= 0x1b;
    b >>= 1;
  }
  return r;
}

inline const AesTables& aes_tables() {
  static const AesTables tabs = [] {
    AesTables t{};
    // log/antilog tables over generator 3 give the inverse in O(1).
    uint8_t exp_t[256], log_t[256] = {0};
    uint8_t v = 1;
    for (int i = 0; i < 255; i++) {
      exp_t[i] = v;
      log_t[v] = static_cast<uint8_t>(i);
      v = gf_mul(v, 3);
    }
    exp_t[255] = exp_t[0];
    for (int x = 0; x < 256; x++) {
      const uint8_t inv = x ? exp_t[(255 - log_t[x]) % 255] : 0;
      uint8_t s = inv, r = inv;
      for (int k = 0; k < 4; k++) {
        r = static_cast<uint8_t>((r << 1) | (r >> 7));
        s ^= r;
      }
      t.sbox[x] = static_cast<uint8_t>(s ^ 0x63);
    }
    for (int x = 0; x < 256; x++) {
      const uint8_t s = t.sbox[x];
      t.t0[x] = static_cast<uint32_t>(gf_mul(s, 2)) | (static_cast<uint32_t>(s) << 8) |
                (static_cast<uint32_t>(s) << 16) | (static_cast<uint32_t>(gf_mul(s, 3)) << 24);
    }
    return t;
  }();
  return tabs;
}

// FIPS-197 5.2 key expansion into 44 little-endian column words.
inline void aes128_expand_words(const uint8_t key[16], uint32_t w[44]) {
  const auto& T = aes_tables();
  for (int i = 0; i < 4; i++) std::memcpy(&w[i], key + 4 * i, 4);
  uint8_t rcon = 1;
  for (int i = 4; i < 44; i++) {
    uint32_t t = w[i - 1];
    if (i % 4 == 0) {
      // RotWord then SubWord on LE bytes (b0 b1 b2 b3) -> (S b1, S b2, S b3, S b0)
      const uint32_t rot = (t >> 8) | (t << 24);
      t = static_cast<uint32_t>(T.sbox[rot & 0xFF]) | (static_cast<uint32_t>(T.sbox[(rot >> 8) & 0xFF]) << 8) |
          (static_cast<uint32_t>(T.sbox[(rot >> 16) & 0xFF]) << 16) |
          (static_cast<uint32_t>(T.sbox[rot >> 24]) << 24);
      t ^= rcon;
      rcon = gf_mul(rcon, 2);
    }
    w[i] = w[i - 4] ^ t;
  }
}

inline void aes128_expand_bytes(const uint8_t key[16], uint8_t rk[176]) {
  uint32_t w[44];
  aes128_expand_words(key, w);
  std::memcpy(rk, w, 176);
}

inline uint32_t rotl(uint32_t v, int r) { return r ? ((v << r) | (v >> (32 - r))) : v; }

// Portable T-table encryption of one block (LE column words).
inline void aes128_encrypt_portable(const uint32_t rk[44], const uint8_t in[16], uint8_t out[16]) {
  const auto& T = aes_tables();
  uint32_t s[4], t[4];
  std::memcpy(s, in, 16);
  for (int c = 0; c < 4; c++) s[c] ^= rk[c];
  for (int r = 1; r < 10; r++) {
    for (int c = 0; c < 4; c++) {
      t[c] = T.t0[s[c] & 0xFF] ^ rotl(T.t0[(s[(c + 1) & 3] >> 8) & 0xFF], 8) ^
             rotl(T.t0[(s[(c + 2) & 3] >> 16) & 0xFF], 16) ^ rotl(T.t0[s[(c + 3) & 3] >> 24], 24) ^ rk[4 * r + c];
    }
    std::memcpy(s, t, 16);
  }
  for (int c = 0; c < 4; c++) {
    t[c] = static_cast<uint32_t>(T.sbox[s[c] & 0xFF]) | (static_cast<uint32_t>(T.sbox[(s[(c + 1) & 3] >> 8) & 0xFF]) << 8) |
           (static_cast<uint32_t>(T.sbox[(s[(c + 2) & 3] >> 16) & 0xFF]) << 16) |
           (static_cast<uint32_t>(T.sbox[s[(c + 3) & 3] >> 24]) << 24);
    t[c] ^= rk[40 + c];
  }
  std::memcpy(out, t, 16);
}

#if defined(__x86_64__)
__attribute__((target("aes,sse2"))) inline void aes128_encrypt_ni(const uint32_t rk[44], const uint8_t in[16],
                                                                  uint8_t out[16]) {
  __m128i s = _mm_loadu_si128(reinterpret_cast<const __m128i*>(in));
  s = _mm_xor_si128(s, _mm_loadu_si128(reinterpret_cast<const __m128i*>(rk)));
  for (int r = 1; r < 10; r++) s = _mm_aesenc_si128(s, _mm_loadu_si128(reinterpret_cast<const __m128i*>(rk + 4 * r)));
  s = _mm_aesenclast_si128(s, _mm_loadu_si128(reinterpret_cast<const __m128i*>(rk + 40)));
  _mm_storeu_si128(reinterpret_cast<__m128i*>(out), s);
}
#endif

inline bool cpu_has_aesni() {
#if defined(__x86_64__)
  static const bool has = __builtin_cpu_supports("aes");
  return has;
#else
  return false;
#endif
}

inline void aes128_encrypt(const uint32_t rk[44], const uint8_t in[16], uint8_t out[16]) {
#if defined(__x86_64__)
  if (cpu_has_aesni()) {
    aes128_encrypt_ni(rk, in, out);
    return;
  }
#endif
  aes128_encrypt_portable(rk, in, out);
}

}  // namespace host
}  // namespace sufb200
