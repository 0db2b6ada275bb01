/*
 * suf_oracle.c -- TEST INFRASTRUCTURE ONLY (the checker, never the product).
 *
 * A plain-C CPU restatement of the reference (ponyyuhan/SUF) PFSS evaluation
 * path.  Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline /
 * reference legs load this file's shared object; nothing under suf_b200/
 * links or calls it.
 *
 * Pinning: the myl7 DCF functions below are checked against the reference's
 * own third_party/myl7_fss sources compiled into oracle/_ref (oracle/Makefile),
 * the AES-128 core against the FIPS-197 Appendix C.1 example and against
 * OpenSSL's AES through its public API, and the threshold / packed-compare /
 * interval-LUT formats against the fixed vectors of the reference's
 * src/demo/test_pfss_gpu.cpp and src/demo/test_cuda_packed_pfss.cpp
 * (tests/golden/).
 *
 * Every function names the reference file:line it restates.
 */
#include <stdint.h>
#include <stddef.h>
#include <string.h>
#include <stdlib.h>

typedef unsigned __int128 u128;

#define ORC_M127 ((((u128)1) << 127) - 1)

/* ------------------------------------------------------------------------ */
/* mt19937_64 (Matsumoto & Nishimura 2000, the std::mt19937_64 parameters).  */
/* The reference seeds masks and key ids with std::mt19937_64, e.g.          */
/* cuda/pfss_backend_gpu.cu:189-194 and include/gates/composite_fss.hpp:656. */
/* ------------------------------------------------------------------------ */
typedef struct {
  uint64_t mt[312];
  int idx;
} orc_mt64;

void orc_mt64_seed(orc_mt64* g, uint64_t seed) {
  g->mt[0] = seed;
  for (int i = 1; i < 312; i++) {
    uint64_t p = g->mt[i - 1];
    g->mt[i] = 6364136223846793005ULL * (p ^ (p >> 62)) + (uint64_t)i;
  }
  g->idx = 312;
}

static void orc_mt64_twist(orc_mt64* g) {
  const uint64_t lower = 0x7FFFFFFFULL, upper = ~lower;
  for (int i = 0; i < 312; i++) {
    uint64_t x = (g->mt[i] & upper) | (g->mt[(i + 1) % 312] & lower);
    uint64_t xa = x >> 1;
    if (x & 1ULL) xa ^= 0xB5026F5AA96619E9ULL;
    g->mt[i] = g->mt[(i + 156) % 312] ^ xa;
  }
  g->idx = 0;
}

uint64_t orc_mt64_next(orc_mt64* g) {
  if (g->idx >= 312) orc_mt64_twist(g);
  uint64_t y = g->mt[g->idx++];
  y ^= (y >> 29) & 0x5555555555555555ULL;
  y ^= (y << 17) & 0x71D67FFFEDA60000ULL;
  y ^= (y << 37) & 0xFFF7EEE000000000ULL;
  y ^= y >> 43;
  return y;
}

/* Fill out[0..n) with successive draws of mt19937_64(seed). */
void orc_mt64_fill(uint64_t seed, uint64_t* out, size_t n) {
  orc_mt64 g;
  orc_mt64_seed(&g, seed);
  for (size_t i = 0; i < n; i++) out[i] = orc_mt64_next(&g);
}

/* ------------------------------------------------------------------------ */
/* AES-128 from FIPS-197: S-box derived from the GF(2^8) inverse and the     */
/* affine map, byte-oriented rounds.  The reference uses AES-128 as the      */
/* myl7 MMO PRG (third_party/myl7_fss/src/prg/aes128_mmo.c:41-53) and as the */
/* CTR keystream of its GPU key formats (cuda/pfss_kernels.cu:112-165).      */
/* ------------------------------------------------------------------------ */
static uint8_t orc_sbox[256];
static int orc_sbox_ready = 0;

static uint8_t gf_mul(uint8_t a, uint8_t b) {
  uint8_t r = 0;
  while (b) {
    if (b & 1) r ^= a;
    uint8_t hi = a & 0x80;
    a <<= 1;
    if (hi) a ^= 0x1b;
    b >>= 1;
  }
  return r;
}

static void orc_sbox_init(void) {
  if (orc_sbox_ready) return;
  for (int x = 0; x < 256; x++) {
    uint8_t inv = 0;
    if (x) {
      for (int y = 1; y < 256; y++)
        if (gf_mul((uint8_t)x, (uint8_t)y) == 1) { inv = (uint8_t)y; break; }
    }
    uint8_t s = inv;
    uint8_t r = inv;
    for (int k = 1; k <= 4; k++) {
      r = (uint8_t)((r << 1) | (r >> 7));
      s ^= r;
    }
    orc_sbox[x] = s ^ 0x63;
  }
  orc_sbox_ready = 1;
}

uint8_t orc_aes_sbox(uint8_t x) {
  orc_sbox_init();
  return orc_sbox[x];
}

/* FIPS-197 section 5.2 key expansion; rk is 176 bytes (11 round keys). */
void orc_aes128_expand(const uint8_t key[16], uint8_t rk[176]) {
  orc_sbox_init();
  memcpy(rk, key, 16);
  uint8_t rcon = 1;
  for (int i = 4; i < 44; i++) {
    uint8_t t[4];
    memcpy(t, rk + 4 * (i - 1), 4);
    if (i % 4 == 0) {
      uint8_t t0 = t[0];
      t[0] = orc_sbox[t[1]] ^ rcon;
      t[1] = orc_sbox[t[2]];
      t[2] = orc_sbox[t[3]];
      t[3] = orc_sbox[t0];
      rcon = gf_mul(rcon, 2);
    }
    for (int j = 0; j < 4; j++) rk[4 * i + j] = rk[4 * (i - 4) + j] ^ t[j];
  }
}

/* FIPS-197 section 5.1 cipher; state byte i sits at row i%4, column i/4. */
void orc_aes128_encrypt(const uint8_t rk[176], const uint8_t in[16], uint8_t out[16]) {
  orc_sbox_init();
  uint8_t s[16];
  for (int i = 0; i < 16; i++) s[i] = in[i] ^ rk[i];
  for (int round = 1; round <= 10; round++) {
    uint8_t t[16];
    for (int c = 0; c < 4; c++)
      for (int r = 0; r < 4; r++) t[4 * c + r] = orc_sbox[s[4 * ((c + r) % 4) + r]];
    if (round < 10) {
      for (int c = 0; c < 4; c++) {
        uint8_t a0 = t[4 * c], a1 = t[4 * c + 1], a2 = t[4 * c + 2], a3 = t[4 * c + 3];
        t[4 * c + 0] = gf_mul(a0, 2) ^ gf_mul(a1, 3) ^ a2 ^ a3;
        t[4 * c + 1] = a0 ^ gf_mul(a1, 2) ^ gf_mul(a2, 3) ^ a3;
        t[4 * c + 2] = a0 ^ a1 ^ gf_mul(a2, 2) ^ gf_mul(a3, 3);
        t[4 * c + 3] = gf_mul(a0, 3) ^ a1 ^ a2 ^ gf_mul(a3, 2);
      }
    }
    for (int i = 0; i < 16; i++) s[i] = t[i] ^ rk[16 * round + i];
  }
  memcpy(out, s, 16);
}

/* Batch ECB helper for tests: out[i] = AES_key(in[i]). */
void orc_aes128_ecb(const uint8_t key[16], const uint8_t* in, uint8_t* out, size_t blocks) {
  uint8_t rk[176];
  orc_aes128_expand(key, rk);
  for (size_t i = 0; i < blocks; i++) orc_aes128_encrypt(rk, in + 16 * i, out + 16 * i);
}

/* ------------------------------------------------------------------------ */
/* myl7 DCF (third_party/myl7_fss v0.7.1).                                   */
/*   PRG  = AES-128-MMO, block j = AES_{K_j}(seed) xor seed, K_j = state    */
/*          bytes [16j, 16j+16)  (src/prg/aes128_mmo.c:16-53)               */
/*   gen  = src/dcf.c:42-142, eval = src/dcf.c:146-193                      */
/*   group ADD = src/group/u128_le.c (add/neg mod 2^127, MSB cleared)       */
/*   group XOR = src/group/bytes.c (xor, neg is identity)                   */
/*   lambda = 16 bytes; CW record = [s_cw 16][v_cw 16][tl<<1|tr] = 33 bytes */
/* ------------------------------------------------------------------------ */
enum { ORC_GROUP_ADD = 0, ORC_GROUP_XOR = 1 };

typedef struct {
  uint8_t rk[4][176];
} orc_prg;

static orc_prg g_prg;
static int g_prg_ready = 0;

/* prg_init: state is >= 64 bytes (the reference build passes kBlocks*16 = 128). */
void orc_prg_init(const uint8_t* state, size_t len) {
  if (len < 64) return;
  for (int j = 0; j < 4; j++) orc_aes128_expand(state + 16 * j, g_prg.rk[j]);
  g_prg_ready = 1;
}

static u128 ld128(const uint8_t* p) {
  u128 v = 0;
  for (int i = 15; i >= 0; i--) v = (v << 8) | p[i];
  return v;
}
static void st128(uint8_t* p, u128 v) {
  for (int i = 0; i < 16; i++) { p[i] = (uint8_t)v; v >>= 8; }
}

static u128 prg_block(int j, u128 seed) {
  uint8_t in[16], out[16];
  st128(in, seed);
  orc_aes128_encrypt(g_prg.rk[j], in, out);
  return ld128(out) ^ seed;
}

static u128 g_add(int group, u128 a, u128 b) {
  return group == ORC_GROUP_ADD ? ((a + b) & ORC_M127) : (a ^ b);
}
static u128 g_neg(int group, u128 a) {
  return group == ORC_GROUP_ADD ? ((((u128)0) - a) & ORC_M127) : a;
}

static int bit_of(uint64_t x, int i) { return (int)((x >> i) & 1ULL); }

/*
 * dcf_gen restatement.  seed0/seed1 are the initial party seeds (stored
 * verbatim in the keys, MSB included); beta is the 16-byte chunk payload.
 * Output: cws[in_bits*33], cw_np1[16].  Bound is kLtAlpha (the only bound
 * the reference adapter uses, include/proto/myl7_fss_backend.hpp:184).
 */
int orc_myl7_dcf_gen(int group, int in_bits, uint64_t alpha, const uint8_t beta[16],
                     const uint8_t seed0[16], const uint8_t seed1[16],
                     uint8_t* cws, uint8_t cw_np1[16]) {
  if (!g_prg_ready || in_bits <= 0 || in_bits > 64) return -1;
  u128 s0 = ld128(seed0) & ORC_M127, s1 = ld128(seed1) & ORC_M127;
  int t0 = 0, t1 = 1;
  u128 v = 0;
  u128 b128 = ld128(beta) & ORC_M127;
  for (int i = 0; i < in_bits; i++) {
    u128 p0[4], p1[4];
    for (int j = 0; j < 4; j++) { p0[j] = prg_block(j, s0); p1[j] = prg_block(j, s1); }
    int t0l = (int)(p0[0] >> 127), t0r = (int)(p0[2] >> 127);
    int t1l = (int)(p1[0] >> 127), t1r = (int)(p1[2] >> 127);
    for (int j = 0; j < 4; j++) { p0[j] &= ORC_M127; p1[j] &= ORC_M127; }
    int a = bit_of(alpha, in_bits - 1 - i);
    u128 s0_lose = a ? p0[0] : p0[2], s1_lose = a ? p1[0] : p1[2];
    u128 v0_lose = a ? p0[1] : p0[3], v1_lose = a ? p1[1] : p1[3];
    u128 v0_keep = a ? p0[3] : p0[1], v1_keep = a ? p1[3] : p1[1];
    u128 s_cw = s0_lose ^ s1_lose;
    u128 v_cw = g_add(group, g_add(group, v1_lose, g_neg(group, v0_lose)), g_neg(group, v));
    if (t1) v_cw = g_neg(group, v_cw);
    if (a) v_cw = g_add(group, v_cw, t1 ? g_neg(group, b128) : b128);
    v = g_add(group, v, g_neg(group, v1_keep));
    v = g_add(group, v, v0_keep);
    v = g_add(group, v, t1 ? g_neg(group, v_cw) : v_cw);
    int tl_cw = t0l ^ t1l ^ a ^ 1;
    int tr_cw = t0r ^ t1r ^ a;
    uint8_t* cw = cws + (size_t)i * 33;
    st128(cw, s_cw);
    st128(cw + 16, v_cw);
    cw[32] = (uint8_t)((tl_cw << 1) | tr_cw);
    u128 s0_keep = a ? p0[2] : p0[0], s1_keep = a ? p1[2] : p1[0];
    int t0_keep = a ? t0r : t0l, t1_keep = a ? t1r : t1l;
    int tcw_keep = a ? tr_cw : tl_cw;
    s0 = s0_keep ^ (t0 ? s_cw : 0);
    s1 = s1_keep ^ (t1 ? s_cw : 0);
    t0 = t0_keep ^ (t0 & tcw_keep);
    t1 = t1_keep ^ (t1 & tcw_keep);
  }
  u128 last = g_add(group, g_add(group, s1, g_neg(group, s0)), g_neg(group, v));
  if (t1) last = g_neg(group, last);
  st128(cw_np1, last);
  return 0;
}

/* dcf_eval restatement: returns the 16-byte group element in out[16]. */
int orc_myl7_dcf_eval(int group, int party, int in_bits, const uint8_t seed[16],
                      const uint8_t* cws, const uint8_t cw_np1[16], uint64_t x,
                      uint8_t out[16]) {
  if (!g_prg_ready || in_bits <= 0 || in_bits > 64) return -1;
  u128 s = ld128(seed) & ORC_M127;
  int t = party & 1;
  u128 v = 0;
  for (int i = 0; i < in_bits; i++) {
    const uint8_t* cw = cws + (size_t)i * 33;
    int xi = bit_of(x, in_bits - 1 - i);
    /* Only the chosen child is consumed (src/dcf.c:178-186), so the walk
       needs blocks {0,1} for x_i = 0 and {2,3} for x_i = 1. */
    u128 sc = prg_block(xi ? 2 : 0, s);
    u128 vc = prg_block(xi ? 3 : 1, s) & ORC_M127;
    int tc = (int)(sc >> 127);
    sc &= ORC_M127;
    if (t) {
      sc ^= ld128(cw);
      tc ^= xi ? (cw[32] & 1) : ((cw[32] >> 1) & 1);
      vc = g_add(group, vc, ld128(cw + 16));
    }
    if (party) vc = g_neg(group, vc);
    v = g_add(group, v, vc);
    s = sc;
    t = tc;
  }
  if (t) s = g_add(group, s, ld128(cw_np1));
  if (party) s = g_neg(group, s);
  v = g_add(group, v, s);
  st128(out, v);
  return 0;
}

/*
 * Adapter key format, include/proto/myl7_fss_backend.hpp:131-213:
 *   [in_bits u8][num_chunks u8][party u8][0][payload_len u32 LE]
 *   then per 16-byte payload chunk: [seed 16][cws in_bits*33][cw_np1 16]
 * Chunk c uses seeds seeds0[16c..], seeds1[16c..] (the reference draws them
 * from std::random_device; tests pass seeded bytes instead).
 */
size_t orc_myl7_key_bytes(int in_bits, int payload_len) {
  size_t chunks = (size_t)(payload_len + 15) / 16;
  return 8 + chunks * (16 + (size_t)in_bits * 33 + 16);
}

int orc_myl7_gen_key_pair(int group, int in_bits, uint64_t alpha, const uint8_t* payload,
                          int payload_len, const uint8_t* seeds0, const uint8_t* seeds1,
                          uint8_t* key0, uint8_t* key1) {
  if (payload_len <= 0 || (payload_len + 15) / 16 > 255) return -1;
  int chunks = (payload_len + 15) / 16;
  size_t cw_bytes = (size_t)in_bits * 33;
  size_t chunk_bytes = 16 + cw_bytes + 16;
  uint8_t* keys[2] = {key0, key1};
  for (int p = 0; p < 2; p++) {
    uint8_t* k = keys[p];
    k[0] = (uint8_t)in_bits;
    k[1] = (uint8_t)chunks;
    k[2] = (uint8_t)p;
    k[3] = 0;
    uint32_t pl = (uint32_t)payload_len;
    for (int b = 0; b < 4; b++) k[4 + b] = (uint8_t)(pl >> (8 * b));
  }
  uint8_t* cws = (uint8_t*)malloc(cw_bytes);
  if (!cws) return -2;
  for (int c = 0; c < chunks; c++) {
    uint8_t beta[16] = {0};
    int take = payload_len - 16 * c;
    if (take > 16) take = 16;
    memcpy(beta, payload + 16 * c, (size_t)take);
    beta[15] &= 0x7F;
    uint8_t np1[16];
    int rc = orc_myl7_dcf_gen(group, in_bits, alpha, beta, seeds0 + 16 * c, seeds1 + 16 * c, cws, np1);
    if (rc) { free(cws); return rc; }
    size_t off = 8 + (size_t)c * chunk_bytes;
    memcpy(key0 + off, seeds0 + 16 * c, 16);
    memcpy(key1 + off, seeds1 + 16 * c, 16);
    memcpy(key0 + off + 16, cws, cw_bytes);
    memcpy(key1 + off + 16, cws, cw_bytes);
    memcpy(key0 + off + 16 + cw_bytes, np1, 16);
    memcpy(key1 + off + 16 + cw_bytes, np1, 16);
  }
  free(cws);
  return 0;
}

/* Evaluate one adapter-format key at x (include/proto/myl7_fss_backend.hpp:215-256). */
int orc_myl7_eval_key(int group, const uint8_t* key, uint64_t x, uint8_t* out, int out_len) {
  int in_bits = key[0], chunks = key[1], party = key[2];
  uint32_t pl = (uint32_t)key[4] | ((uint32_t)key[5] << 8) | ((uint32_t)key[6] << 16) | ((uint32_t)key[7] << 24);
  if (party != 0 && party != 1) return -3;
  if ((int)pl != out_len) return -4;
  if (in_bits < 64) x &= ((1ULL << in_bits) - 1ULL);
  size_t cw_bytes = (size_t)in_bits * 33;
  size_t chunk_bytes = 16 + cw_bytes + 16;
  int written = 0;
  for (int c = 0; c < chunks; c++) {
    const uint8_t* ck = key + 8 + (size_t)c * chunk_bytes;
    uint8_t v[16];
    int rc = orc_myl7_dcf_eval(group, party, in_bits, ck, ck + 16, ck + 16 + cw_bytes, x, v);
    if (rc) return rc;
    int take = out_len - written;
    if (take > 16) take = 16;
    memcpy(out + written, v, (size_t)take);
    written += take;
  }
  return 0;
}

/* Batched: per-element keys (broadcast=0) or one key for all (broadcast=1). */
int orc_myl7_eval_many(int group, const uint8_t* keys, size_t key_bytes, int broadcast,
                       const uint64_t* xs, size_t n, uint8_t* outs, int out_len) {
  int err = 0;
#pragma omp parallel for schedule(dynamic, 64) reduction(| : err)
  for (long long i = 0; i < (long long)n; i++) {
    const uint8_t* k = keys + (broadcast ? 0 : (size_t)i * key_bytes);
    int rc = orc_myl7_eval_key(group, k, xs[i], outs + (size_t)i * (size_t)out_len, out_len);
    if (rc) err |= 1;
  }
  return err ? -1 : 0;
}

/* ------------------------------------------------------------------------ */
/* Reference GPU-backend key formats (cuda/pfss_backend_gpu.cu).            */
/* ------------------------------------------------------------------------ */

/* seed_from_id, cuda/pfss_backend_gpu.cu:189-194 */
void orc_seed_from_id(uint64_t id, uint64_t tweak, uint8_t seed[16]) {
  orc_mt64 g;
  orc_mt64_seed(&g, id ^ (tweak * 0x9e3779b97f4a7c15ULL));
  for (int i = 0; i < 16; i++) seed[i] = (uint8_t)(orc_mt64_next(&g) & 0xFF);
}

static uint64_t mask_bits(int bits) {
  if (bits <= 0) return 0;
  if (bits >= 64) return ~0ULL;
  return (1ULL << bits) - 1ULL;
}
static uint64_t ld64(const uint8_t* p) { uint64_t v; memcpy(&v, p, 8); return v; }
static void st64(uint8_t* p, uint64_t v) { memcpy(p, &v, 8); }

/*
 * Threshold "DCF" key, DcfKeyHeader (packed, 12 bytes) + payload:
 *   [in_bits u16][payload_len u16][alpha u64]   (cuda/pfss_backend_gpu.cu:69-73,197-221)
 * eval: payload if (x&m) < (alpha&m) else zeros   (:290-311, kernel :386-433)
 */
size_t orc_thr_dcf_build(int in_bits, uint64_t alpha, const uint8_t* payload, int payload_len, uint8_t* out) {
  uint16_t ib = (uint16_t)in_bits, pl = (uint16_t)payload_len;
  memcpy(out, &ib, 2);
  memcpy(out + 2, &pl, 2);
  st64(out + 4, alpha & mask_bits(in_bits));
  if (payload_len > 0 && payload) memcpy(out + 12, payload, (size_t)payload_len);
  else if (payload_len > 0) memset(out + 12, 0, (size_t)payload_len);
  return 12 + (size_t)payload_len;
}

int orc_thr_dcf_eval_many(int in_bits, const uint8_t* keys, size_t key_bytes, int broadcast,
                          const uint64_t* xs, size_t n, int out_bytes, uint8_t* outs) {
  uint64_t m = mask_bits(in_bits);
  for (size_t i = 0; i < n; i++) {
    const uint8_t* k = keys + (broadcast ? 0 : i * key_bytes);
    uint64_t alpha = ld64(k + 4);
    int lt = (xs[i] & m) < (alpha & m);
    uint8_t* o = outs + i * (size_t)out_bytes;
    if (lt) memcpy(o, k + 12, (size_t)out_bytes);
    else memset(o, 0, (size_t)out_bytes);
  }
  return 0;
}

/*
 * Packed-compare key, PackedCmpKeyHeader (packed, 208 bytes):
 *   [in_bits u16][num_thr u16][party u8][flags u8 (bit0 = sorted)][2 pad]
 *   [nonce u64][seed 16][round_keys 176] then thresholds u64[num_thr]
 *   (cuda/pfss_backend_gpu.cu:86-94,257-288)
 */
#define ORC_PACKED_HDR 208
size_t orc_packed_key_build(int party, uint64_t nonce, int in_bits, const uint64_t* thr, int num_thr,
                            const uint8_t seed[16], uint8_t* out) {
  memset(out, 0, ORC_PACKED_HDR);
  uint16_t ib = (uint16_t)in_bits, nt = (uint16_t)num_thr;
  memcpy(out, &ib, 2);
  memcpy(out + 2, &nt, 2);
  out[4] = (uint8_t)party;
  st64(out + 8, nonce);
  memcpy(out + 16, seed, 16);
  orc_aes128_expand(seed, out + 32);
  uint64_t m = mask_bits(in_bits);
  int sorted = 1;
  uint64_t prev = 0;
  for (int i = 0; i < num_thr; i++) {
    uint64_t v = thr[i] & m;
    st64(out + ORC_PACKED_HDR + 8 * (size_t)i, v);
    if (i > 0 && v < prev) sorted = 0;
    prev = v;
  }
  out[5] = (uint8_t)(sorted ? 1 : 0);
  return ORC_PACKED_HDR + 8 * (size_t)num_thr;
}

/* Kernel keystream layout (cuda/pfss_kernels.cu:240-330): one AES block per
   two mask words, ctr = nonce ^ (idx<<32) ^ (w/2), block = [ctr LE][0^8],
   words w, w+1 take the low / high 8 bytes.  idx = idx_base + i. */
static void ctr_block(const uint8_t rk[176], uint64_t ctr, uint64_t* ks0, uint64_t* ks1) {
  uint8_t in[16] = {0}, out[16];
  st64(in, ctr);
  orc_aes128_encrypt(rk, in, out);
  *ks0 = ld64(out);
  *ks1 = ld64(out + 8);
}

int orc_packed_eval_many(const uint8_t* keys, size_t key_bytes, int broadcast, const uint64_t* xs, size_t n,
                         uint64_t idx_base, int out_words, uint64_t* outs) {
  for (size_t i = 0; i < n; i++) {
    const uint8_t* k = keys + (broadcast ? 0 : i * key_bytes);
    uint16_t ib, nt;
    memcpy(&ib, k, 2);
    memcpy(&nt, k + 2, 2);
    int party = k[4];
    uint64_t nonce = ld64(k + 8);
    const uint8_t* rk = k + 32;
    uint64_t m = mask_bits(ib);
    uint64_t x = xs[i] & m;
    int words = (nt + 63) / 64;
    if (words != out_words) return -1;
    uint64_t idx = idx_base + i;
    for (int w = 0; w < words; w += 2) {
      uint64_t word[2] = {0, 0};
      for (int h = 0; h < 2 && w + h < words; h++) {
        int base = (w + h) * 64;
        int lim = base + 64 < nt ? base + 64 : nt;
        for (int b = base; b < lim; b++) {
          uint64_t t = ld64(k + ORC_PACKED_HDR + 8 * (size_t)b) & m;
          if (x < t) word[h] |= 1ULL << (b - base);
        }
      }
      uint64_t ks0, ks1;
      ctr_block(rk, nonce ^ (idx << 32) ^ (uint64_t)(w / 2), &ks0, &ks1);
      outs[i * (size_t)words + (size_t)w] = party == 0 ? ks0 : (word[0] ^ ks0);
      if (w + 1 < words) outs[i * (size_t)words + (size_t)w + 1] = party == 0 ? ks1 : (word[1] ^ ks1);
    }
  }
  return 0;
}

/*
 * Interval-LUT key, IntervalKeyHeader (alignas 8, 216 bytes):
 *   [in_bits u16][out_words u16][intervals u32][party u8][3 pad][4 pad]
 *   [nonce u64 @16][seed 16 @24][round_keys 176 @40]
 *   then cuts u64[intervals+1], payload u64[intervals*out_words]
 *   (cuda/pfss_backend_gpu.cu:75-84,223-255)
 */
#define ORC_IVL_HDR 216
size_t orc_interval_key_build(int party, uint64_t nonce, int in_bits, int out_words, const uint64_t* cuts,
                              int intervals, const uint64_t* payload, const uint8_t seed[16], uint8_t* out) {
  memset(out, 0, ORC_IVL_HDR);
  uint16_t ib = (uint16_t)in_bits, ow = (uint16_t)out_words;
  uint32_t iv = (uint32_t)intervals;
  memcpy(out, &ib, 2);
  memcpy(out + 2, &ow, 2);
  memcpy(out + 4, &iv, 4);
  out[8] = (uint8_t)party;
  st64(out + 16, nonce);
  memcpy(out + 24, seed, 16);
  orc_aes128_expand(seed, out + 40);
  memcpy(out + ORC_IVL_HDR, cuts, 8 * ((size_t)intervals + 1));
  memcpy(out + ORC_IVL_HDR + 8 * ((size_t)intervals + 1), payload, 8 * (size_t)intervals * (size_t)out_words);
  return ORC_IVL_HDR + 8 * ((size_t)intervals + 1) + 8 * (size_t)intervals * (size_t)out_words;
}

/* Kernel layout (cuda/pfss_kernels.cu:545-592): iv = upper_bound(starts, x)-1
   clamped; ctr = nonce ^ (idx<<32) ^ (iv*out_words + w); party0 = ks,
   party1 = payload - ks. */
int orc_interval_eval_many(const uint8_t* keys, size_t key_bytes, int broadcast, const uint64_t* xs, size_t n,
                           uint64_t idx_base, int out_words, uint64_t* outs) {
  for (size_t i = 0; i < n; i++) {
    const uint8_t* k = keys + (broadcast ? 0 : i * key_bytes);
    uint16_t ib, ow;
    uint32_t ivs;
    memcpy(&ib, k, 2);
    memcpy(&ow, k + 2, 2);
    memcpy(&ivs, k + 4, 4);
    if ((int)ow != out_words || ivs == 0) return -1;
    int party = k[8];
    uint64_t nonce = ld64(k + 16);
    const uint8_t* rk = k + 40;
    const uint8_t* cuts = k + ORC_IVL_HDR;
    const uint8_t* pay = cuts + 8 * ((size_t)ivs + 1);
    uint64_t m = mask_bits(ib);
    uint64_t x = xs[i] & m;
    int iv = (int)ivs - 1;
    if (ivs > 1) {
      int lo = 0, hi = (int)ivs;
      while (lo < hi) {
        int mid = (lo + hi) >> 1;
        if ((ld64(cuts + 8 * (size_t)mid) & m) <= x) lo = mid + 1; else hi = mid;
      }
      iv = lo - 1;
      if (iv < 0) iv = 0;
      if (iv >= (int)ivs) iv = (int)ivs - 1;
    }
    uint64_t idx = idx_base + i;
    for (int w = 0; w < ow; w += 2) {
      uint64_t ks0, ks1;
      ctr_block(rk, nonce ^ (idx << 32) ^ ((uint64_t)iv * ow + (uint64_t)w), &ks0, &ks1);
      uint64_t r0 = ld64(pay + 8 * ((size_t)iv * ow + (size_t)w));
      outs[i * (size_t)ow + (size_t)w] = party == 0 ? ks0 : r0 - ks0;
      if (w + 1 < ow) {
        uint64_t r1 = ld64(pay + 8 * ((size_t)iv * ow + (size_t)w + 1));
        outs[i * (size_t)ow + (size_t)w + 1] = party == 0 ? ks1 : r1 - ks1;
      }
    }
  }
  return 0;
}

/* ------------------------------------------------------------------------ */
/* Truncation / ARS bundles.                                                */
/*   keygen masks: include/gates/composite_fss.hpp:645-833                  */
/*   query rewrite: include/suf/mask_rewrite.hpp:13-42,                     */
/*                  src/compiler/suf_to_pfss.cpp:55-92,443-496              */
/*   eval (AddU64 trunc branch): include/gates/composite_fss.hpp:1385-1638  */
/*   postproc: include/gates/postproc_hooks.hpp:173-376                     */
/* ------------------------------------------------------------------------ */
enum { ORC_TR = 0, ORC_ARS = 1, ORC_GAPARS = 2 };

/* Public description of one party's bundle key material (the DCF keys are
   passed separately, one broadcast key per query). */
typedef struct {
  int32_t kind, frac_bits, party, nq;
  int32_t q_bits[4];      /* in_bits of each raw query (64 or f) */
  uint64_t q_theta[4];    /* threshold of each raw query (dealer side only) */
  int32_t carry_a, carry_b;   /* RotXor operands of carry, or -1 = constant 0 */
  int32_t sign_a, sign_b;     /* RotXor operands of sign (ARS), or -1 */
  int32_t wrap_q;             /* query index of wrap = 1[x^ < r_in], or -1 */
  int32_t pad;
  uint64_t carry_w, sign_w;   /* this party's shares of the rotation wrap bits */
  uint64_t haty;              /* base coefficient share + r_out share */
  uint64_t r_hi, m;           /* shares of r_in >> f and of 2^(64-f)*MSB(r_in) */
} orc_trunc_desc;

typedef struct { int kind; uint64_t theta; int bits; int tag; } orc_q;

/*
 * Dealer: draws r = rng() and the share splits in the reference's order
 * (r, r_in split, r_out split, wrap shares, r_hi split, m split), builds
 * the sorted raw query list and both parties' descriptors.  The caller then
 * generates one DCF key per query with AddU64 payload 1.
 * Returns r_in.  out_theta/out_bits receive the sorted queries.
 */
uint64_t orc_trunc_gen(int kind, int f, uint64_t rng_seed, orc_trunc_desc* d0, orc_trunc_desc* d1) {
  orc_mt64 g;
  orc_mt64_seed(&g, rng_seed);
  uint64_t fmask = mask_bits(f);
  uint64_t r = orc_mt64_next(&g);
  uint64_t r_low = r & fmask;
  uint64_t r_hi = f >= 64 ? 0 : (r >> f);
  /* raw queries before canonical sort; tags: 0 carry.a 1 carry.b 2 sign.a 3 sign.b 4 wrap */
  orc_q qs[5];
  int nraw = 0;
  uint64_t wrap_bits[2];
  int nwrap = 0;
  int carry_wi = -1, sign_wi = -1;
  int has_carry = (f > 0) && (r_low != 0) && (f < 64);
  if (has_carry) {
    uint64_t gamma = (1ULL << f) - r_low; /* threshold 2^f - r_low */
    uint64_t th0 = r_low, th1 = (r_low + gamma) & fmask;
    qs[nraw++] = (orc_q){1, th0, f, 0};
    qs[nraw++] = (orc_q){1, th1, f, 1};
    carry_wi = nwrap;
    wrap_bits[nwrap++] = th1 < th0;
  }
  if (kind == ORC_ARS) {
    uint64_t th0 = r + (1ULL << 63);
    uint64_t th1 = th0 + (1ULL << 63);
    qs[nraw++] = (orc_q){0, th0, 64, 2};
    qs[nraw++] = (orc_q){0, th1, 64, 3};
    sign_wi = nwrap;
    wrap_bits[nwrap++] = th1 < th0;
  }
  if (kind == ORC_TR || kind == ORC_ARS) qs[nraw++] = (orc_q){0, r, 64, 4};
  /* dedup on (kind, bits, theta) in first-seen order (suf_to_pfss.cpp:28-36) */
  orc_q uq[5];
  int map[5];
  int nq = 0;
  for (int i = 0; i < nraw; i++) {
    int found = -1;
    for (int j = 0; j < nq; j++)
      if (uq[j].kind == qs[i].kind && uq[j].bits == qs[i].bits && uq[j].theta == qs[i].theta) found = j;
    if (found < 0) { uq[nq] = qs[i]; found = nq++; }
    map[i] = found;
  }
  /* stable sort by (kind, bits, theta) (suf_to_pfss.cpp:458-490) */
  int order[5];
  for (int i = 0; i < nq; i++) order[i] = i;
  for (int i = 1; i < nq; i++) {
    int o = order[i];
    int j = i - 1;
    while (j >= 0) {
      orc_q* a = &uq[order[j]];
      orc_q* b = &uq[o];
      int gt = (a->kind > b->kind) || (a->kind == b->kind && a->bits > b->bits) ||
               (a->kind == b->kind && a->bits == b->bits && a->theta > b->theta);
      if (!gt) break;
      order[j + 1] = order[j];
      j--;
    }
    order[j + 1] = o;
  }
  int new_of_old[5];
  for (int i = 0; i < nq; i++) new_of_old[order[i]] = i;
  int qidx_of_tag[5] = {-1, -1, -1, -1, -1};
  for (int i = 0; i < nraw; i++) qidx_of_tag[qs[i].tag] = new_of_old[map[i]];

  orc_trunc_desc* d[2] = {d0, d1};
  for (int p = 0; p < 2; p++) {
    memset(d[p], 0, sizeof(orc_trunc_desc));
    d[p]->kind = kind;
    d[p]->frac_bits = f;
    d[p]->party = p;
    d[p]->nq = nq;
    for (int i = 0; i < nq; i++) {
      d[p]->q_bits[i] = uq[order[i]].bits;
      d[p]->q_theta[i] = uq[order[i]].theta;
    }
    d[p]->carry_a = qidx_of_tag[0];
    d[p]->carry_b = qidx_of_tag[1];
    d[p]->sign_a = qidx_of_tag[2];
    d[p]->sign_b = qidx_of_tag[3];
    d[p]->wrap_q = qidx_of_tag[4];
  }
  /* share splits, composite_fss.hpp:692-733: split_add(v) = (s0 = rng(), v - s0) */
  uint64_t s;
  s = orc_mt64_next(&g); (void)s; /* r_in share (r0); r1 = r - r0 */
  uint64_t rout0 = orc_mt64_next(&g);
  d0->haty = rout0;
  d1->haty = 0 - rout0; /* r_out = 0, base coefficient = 0 */
  for (int w = 0; w < nwrap; w++) {
    uint64_t w0 = orc_mt64_next(&g);
    uint64_t w1 = wrap_bits[w] - w0;
    if (w == carry_wi) { d0->carry_w = w0; d1->carry_w = w1; }
    if (w == sign_wi) { d0->sign_w = w0; d1->sign_w = w1; }
  }
  uint64_t rh0 = orc_mt64_next(&g);
  d0->r_hi = rh0;
  d1->r_hi = r_hi - rh0;
  uint64_t m = 0;
  if (kind == ORC_GAPARS && f > 0 && f < 64) m = (r >> 63) ? (1ULL << (64 - f)) : 0;
  uint64_t m0 = orc_mt64_next(&g);
  d0->m = kind == ORC_GAPARS ? m0 : 0;
  d1->m = kind == ORC_GAPARS ? (m - m0) : 0;
  return r;
}

/* Combine per-query DCF shares (pred[q*n + i]) into y shares: the AddU64
   bool plan (composite_fss.hpp:1539-1605) then the kind's postproc hook. */
int orc_trunc_combine(const orc_trunc_desc* d, const uint64_t* xhat, const uint64_t* pred, size_t n,
                      uint64_t* y_out, uint64_t* bools_out) {
  int f = d->frac_bits;
  uint64_t one = d->party == 0 ? 1ULL : 0ULL;
  for (size_t i = 0; i < n; i++) {
    uint64_t carry = 0, sign = 0, wrap = 0;
    if (d->carry_a >= 0) {
      uint64_t a = pred[(size_t)d->carry_a * n + i], b = pred[(size_t)d->carry_b * n + i];
      carry = one - ((b - a) + d->carry_w);
    }
    if (d->sign_a >= 0) {
      uint64_t a = pred[(size_t)d->sign_a * n + i], b = pred[(size_t)d->sign_b * n + i];
      sign = (b - a) + d->sign_w;
    }
    if (d->wrap_q >= 0) wrap = pred[(size_t)d->wrap_q * n + i];
    uint64_t y;
    if (d->kind == ORC_GAPARS) {
      uint64_t hb = xhat[i] + (1ULL << 62);
      uint64_t top = 0;
      if (d->party == 0 && f >= 0 && f < 64) top = f == 0 ? hb : (hb >> f);
      y = d->haty + top - d->r_hi - carry;
      if (f > 0 && f < 64 && ((hb >> 63) & 1ULL) == 0) y += d->m;
      if (d->party == 0) y -= (f >= 0 && f <= 62) ? (1ULL << (62 - f)) : 0;
    } else {
      uint64_t top = (d->party == 0 && f < 64) ? (xhat[i] >> f) : 0;
      uint64_t modulus = (f <= 0 || f >= 64) ? 0 : (1ULL << (64 - f));
      y = d->haty + top - d->r_hi - carry;
      if (modulus) y += wrap * modulus;
      if (d->kind == ORC_ARS) {
        uint64_t sign_mask = (f <= 0 || f >= 64) ? 0 : (~0ULL << (64 - f));
        y += sign * sign_mask;
      }
    }
    y_out[i] = y;
    if (bools_out) {
      bools_out[3 * i + 0] = carry;
      bools_out[3 * i + 1] = sign;
      bools_out[3 * i + 2] = wrap;
    }
  }
  return 0;
}

/* ------------------------------------------------------------------------ */
/* Elementwise / row primitives (cuda/cuda_primitives.cu, pfss_kernels.cu).  */
/* ------------------------------------------------------------------------ */

/* pack_eff_bits_host, cuda/pfss_backend_gpu.cu:124-142 */
void orc_pack_eff_bits(const uint64_t* xs, size_t n, int eff_bits, uint64_t* packed, size_t words) {
  memset(packed, 0, words * 8);
  uint64_t m = mask_bits(eff_bits);
  for (size_t i = 0; i < n; i++) {
    uint64_t v = xs[i] & m;
    size_t bit = i * (size_t)eff_bits;
    size_t w = bit >> 6;
    int off = (int)(bit & 63);
    packed[w] |= v << off;
    int spill = off + eff_bits - 64;
    if (spill > 0 && w + 1 < words) packed[w + 1] |= v >> (eff_bits - spill);
  }
}

/* unpack_eff_bits_kernel, cuda/pfss_kernels.cu:722-743 */
void orc_unpack_eff_bits(const uint64_t* packed, size_t n, int eff_bits, uint64_t* out) {
  uint64_t m = mask_bits(eff_bits);
  for (size_t i = 0; i < n; i++) {
    size_t bit = i * (size_t)eff_bits;
    size_t w = bit >> 6;
    int off = (int)(bit & 63);
    uint64_t v = packed[w] >> off;
    int used = 64 - off;
    if (used < eff_bits) v |= packed[w + 1] << used;
    out[i] = eff_bits < 64 ? (v & m) : v;
  }
}

/* beaver_mul_kernel, cuda/cuda_primitives.cu:114-135:
   z = c + d*b + e*a (+ d*e on party 0) mod 2^64 */
void orc_beaver_mul(int party, const uint64_t* a, const uint64_t* b, const uint64_t* c, const uint64_t* d,
                    const uint64_t* e, uint64_t* z, size_t n) {
  for (size_t i = 0; i < n; i++) {
    uint64_t v = c[i] + d[i] * b[i] + e[i] * a[i];
    if (party == 0) v += d[i] * e[i];
    z[i] = v;
  }
}

/* horner_cubic_kernel, cuda/cuda_primitives.cu:254-269 */
void orc_horner_cubic(const uint64_t* x, const uint64_t* c0, const uint64_t* c1, const uint64_t* c2,
                      const uint64_t* c3, uint64_t* out, size_t n) {
  for (size_t i = 0; i < n; i++) out[i] = ((c3[i] * x[i] + c2[i]) * x[i] + c1[i]) * x[i] + c0[i];
}

/* row_sum_kernel, cuda/cuda_primitives.cu:339-362 (valid_lens optional) */
void orc_row_sum(const uint64_t* mat, int rows, int cols, const int* valid, uint64_t* out) {
  for (int r = 0; r < rows; r++) {
    int len = valid ? valid[r] : cols;
    if (len > cols) len = cols;
    uint64_t s = 0;
    for (int c = 0; c < len; c++) s += mat[(size_t)r * cols + c];
    out[r] = s;
  }
}

/* row_variance_kernel, cuda/cuda_primitives.cu:672-707 */
void orc_row_variance(const uint64_t* mat, const uint64_t* mean, int rows, int cols, const int* valid,
                      uint64_t* out) {
  for (int r = 0; r < rows; r++) {
    int len = valid ? valid[r] : cols;
    if (len > cols) len = cols;
    uint64_t s = 0;
    for (int c = 0; c < len; c++) {
      uint64_t dlt = mat[(size_t)r * cols + c] - mean[r];
      s += dlt * dlt;
    }
    out[r] = s;
  }
}
