// aes_smem.cuh -- AES-128 on the shared-memory T-table engine (device side).
//
// State words are little-endian columns: word c holds bytes 4c..4c+3 of the
// 16-byte block, row r of column c at bits 8r..8r+7.  With T0 the column
// word 2S | S<<8 | S<<16 | 3S<<24 of S = Sbox(x), T_k = rotl(T0, 8k), a full
// round is, for output column c,
//     T0[a_c.b0] ^ T1[a_{c+1}.b1] ^ T2[a_{c+2}.b2] ^ T3[a_{c+3}.b3] ^ rk_c
// (SubBytes + ShiftRows + MixColumns, FIPS-197 5.1), and the last round
// picks the S-box byte out of the table entry that already has it in the
// right lane: T2 byte 0, T3 byte 1, T0 byte 2, T1 byte 3.
#pragma once

#include "sufb200_internal.cuh"

// SUFB200_HOST_EMU builds these functions for the host against an emulated
// shared window (used by the CPU test of the table layout and selectors).
#if defined(SUFB200_HOST_EMU)
#define SUFB200_DEV inline
namespace sufb200 {
extern uint8_t* g_emu_smem;  // emulated shared window, >= kTabEnd bytes
extern uint32_t g_emu_lane;
}  // namespace sufb200
#else
#define SUFB200_DEV __device__ __forceinline__
#endif

namespace sufb200 {

// Table offsets relative to kTabBase (see the layout note in
// sufb200_internal.cuh).
constexpr uint32_t kOffT0 = kTabBase + 0x00000u;
constexpr uint32_t kOffT1 = kTabBase + 0x00080u;
constexpr uint32_t kOffT2 = kTabBase + 0x10000u;
constexpr uint32_t kOffT3 = kTabBase + 0x10080u;

// Lookup address for byte r of w: bytes {lb.b0, w.b_r, 0, 0} = (x << 8) | lane*4.
template <int R>
SUFB200_DEV uint32_t tab_addr(uint32_t w, uint32_t lb) {
  return prmt(w, lb, 0x5504u | (static_cast<uint32_t>(R) << 4));
}

template <uint32_t OFF>
SUFB200_DEV uint32_t tab_ld(uint32_t addr) {
#if defined(SUFB200_HOST_EMU)
  uint32_t v;
  memcpy(&v, g_emu_smem + addr + OFF, 4);
  return v;
#else
  uint32_t v;
  asm("ld.shared.u32 %0, [%1+%2];" : "=r"(v) : "r"(addr), "n"(OFF));
  return v;
#endif
}

// Per-lane table base: l * 4.  Read through a volatile asm after the table
// fill barrier so no lookup can be scheduled above that barrier.
SUFB200_DEV uint32_t lane_base() {
#if defined(SUFB200_HOST_EMU)
  return g_emu_lane << 2;
#else
  uint32_t l;
  asm volatile("mov.u32 %0, %%laneid;" : "=r"(l));
  return l << 2;
#endif
}

#if !defined(SUFB200_HOST_EMU)

__device__ __forceinline__ uint32_t dyn_smem_base() {
  extern __shared__ __align__(16) uint8_t sufb200_dyn_smem[];
  return static_cast<uint32_t>(__cvta_generic_to_shared(sufb200_dyn_smem));
}

__device__ __forceinline__ uint32_t dyn_smem_size() {
  uint32_t s;
  asm volatile("mov.u32 %0, %%dynamic_smem_size;" : "=r"(s));
  return s;
}

// True when this CTA's dynamic shared memory covers [kTabBase, kTabEnd).
__device__ __forceinline__ bool aes_layout_ok() {
  const uint32_t base = dyn_smem_base();
  return base <= kTabBase && base + dyn_smem_size() >= kTabEnd;
}

// Fill the four replicated tables from the 256-word global T0.
__device__ __forceinline__ void aes_fill_tables(const uint32_t* __restrict__ g_t0) {
  for (uint32_t idx = threadIdx.x; idx < 4u * 256u * 32u; idx += blockDim.x) {
    const uint32_t lane = idx & 31u, x = (idx >> 5) & 255u, k = idx >> 13;
    const uint32_t v = rotl32(__ldg(g_t0 + x), static_cast<int>(8u * k));
    const uint32_t addr = kTabBase + (k >> 1) * 0x10000u + x * 256u + (k & 1u) * 128u + lane * 4u;
    asm volatile("st.shared.u32 [%0], %1;" ::"r"(addr), "r"(v) : "memory");
  }
}

#endif  // !SUFB200_HOST_EMU

struct Blk {
  uint32_t w[4];
};

// One middle round; k0..k3 are the round-key words.
SUFB200_DEV Blk aes_round(const Blk& a, uint32_t lb, uint32_t k0, uint32_t k1, uint32_t k2,
                                         uint32_t k3) {
  Blk t;
  t.w[0] = tab_ld<kOffT0>(tab_addr<0>(a.w[0], lb)) ^ tab_ld<kOffT1>(tab_addr<1>(a.w[1], lb)) ^
           tab_ld<kOffT2>(tab_addr<2>(a.w[2], lb)) ^ tab_ld<kOffT3>(tab_addr<3>(a.w[3], lb)) ^ k0;
  t.w[1] = tab_ld<kOffT0>(tab_addr<0>(a.w[1], lb)) ^ tab_ld<kOffT1>(tab_addr<1>(a.w[2], lb)) ^
           tab_ld<kOffT2>(tab_addr<2>(a.w[3], lb)) ^ tab_ld<kOffT3>(tab_addr<3>(a.w[0], lb)) ^ k1;
  t.w[2] = tab_ld<kOffT0>(tab_addr<0>(a.w[2], lb)) ^ tab_ld<kOffT1>(tab_addr<1>(a.w[3], lb)) ^
           tab_ld<kOffT2>(tab_addr<2>(a.w[0], lb)) ^ tab_ld<kOffT3>(tab_addr<3>(a.w[1], lb)) ^ k2;
  t.w[3] = tab_ld<kOffT0>(tab_addr<0>(a.w[3], lb)) ^ tab_ld<kOffT1>(tab_addr<1>(a.w[0], lb)) ^
           tab_ld<kOffT2>(tab_addr<2>(a.w[1], lb)) ^ tab_ld<kOffT3>(tab_addr<3>(a.w[2], lb)) ^ k3;
  return t;
}

// Last-round column c (SubBytes + ShiftRows + AddRoundKey).
template <int C>
SUFB200_DEV uint32_t aes_last_col(const Blk& a, uint32_t lb, uint32_t k) {
  const uint32_t v0 = tab_ld<kOffT2>(tab_addr<0>(a.w[C], lb));            // S at byte 0
  const uint32_t v1 = tab_ld<kOffT3>(tab_addr<1>(a.w[(C + 1) & 3], lb));  // S at byte 1
  const uint32_t v2 = tab_ld<kOffT0>(tab_addr<2>(a.w[(C + 2) & 3], lb));  // S at byte 2
  const uint32_t v3 = tab_ld<kOffT1>(tab_addr<3>(a.w[(C + 3) & 3], lb));  // S at byte 3
  const uint32_t lo = prmt(v0, v1, 0x0050u);
  const uint32_t hi = prmt(v2, v3, 0x7200u);
  return prmt(lo, hi, 0x7610u) ^ k;
}

// Key words from a PrgParams half h for round r, column c, chosen per lane:
// key(2x+h) = base[h] ^ (xmask & diff[h]).
#define SUFB200_PRG_KEY(P, H, R, C, XM) ((P).base[H][R][C] ^ ((XM) & (P).diff[H][R][C]))

// The two MMO blocks one tree level needs: A = AES_{K_{2x}}(s) ^ s (full
// block) and the low half of B = AES_{K_{2x+1}}(s) ^ s.
SUFB200_DEV void prg_level(const PrgParams& P, uint32_t lb, const Blk& s, uint32_t xm, Blk& outA,
                                          uint32_t& b0, uint32_t& b1) {
  Blk a, b;
#pragma unroll
  for (int c = 0; c < 4; c++) {
    a.w[c] = s.w[c] ^ SUFB200_PRG_KEY(P, 0, 0, c, xm);
    b.w[c] = s.w[c] ^ SUFB200_PRG_KEY(P, 1, 0, c, xm);
  }
#pragma unroll
  for (int r = 1; r < 10; r++) {
    a = aes_round(a, lb, SUFB200_PRG_KEY(P, 0, r, 0, xm), SUFB200_PRG_KEY(P, 0, r, 1, xm),
                  SUFB200_PRG_KEY(P, 0, r, 2, xm), SUFB200_PRG_KEY(P, 0, r, 3, xm));
    b = aes_round(b, lb, SUFB200_PRG_KEY(P, 1, r, 0, xm), SUFB200_PRG_KEY(P, 1, r, 1, xm),
                  SUFB200_PRG_KEY(P, 1, r, 2, xm), SUFB200_PRG_KEY(P, 1, r, 3, xm));
  }
  outA.w[0] = aes_last_col<0>(a, lb, SUFB200_PRG_KEY(P, 0, 10, 0, xm)) ^ s.w[0];
  outA.w[1] = aes_last_col<1>(a, lb, SUFB200_PRG_KEY(P, 0, 10, 1, xm)) ^ s.w[1];
  outA.w[2] = aes_last_col<2>(a, lb, SUFB200_PRG_KEY(P, 0, 10, 2, xm)) ^ s.w[2];
  outA.w[3] = aes_last_col<3>(a, lb, SUFB200_PRG_KEY(P, 0, 10, 3, xm)) ^ s.w[3];
  b0 = aes_last_col<0>(b, lb, SUFB200_PRG_KEY(P, 1, 10, 0, xm)) ^ s.w[0];
  b1 = aes_last_col<1>(b, lb, SUFB200_PRG_KEY(P, 1, 10, 1, xm)) ^ s.w[1];
}

// Key word of half h (hm = 0 - h) for round r, column c: the per-lane
// choice between the two halves of prg_level, without indexing the
// parameter block by a register.
#define SUFB200_PRG_KEY_H(P, R, C, XM, HM) \
  ((SUFB200_PRG_KEY(P, 0, R, C, XM) & ~(HM)) | (SUFB200_PRG_KEY(P, 1, R, C, XM) & (HM)))

// One of the two MMO blocks of prg_level: out = AES_{K_{2x+h}}(s) ^ s, the
// full block (h = 0 gives prg_level's A, h = 1 its B).
SUFB200_DEV void prg_half(const PrgParams& P, uint32_t lb, const Blk& s, uint32_t xm, uint32_t h, Blk& out) {
  const uint32_t hm = 0u - h;
  Blk a;
#pragma unroll
  for (int c = 0; c < 4; c++) a.w[c] = s.w[c] ^ SUFB200_PRG_KEY_H(P, 0, c, xm, hm);
#pragma unroll
  for (int r = 1; r < 10; r++)
    a = aes_round(a, lb, SUFB200_PRG_KEY_H(P, r, 0, xm, hm), SUFB200_PRG_KEY_H(P, r, 1, xm, hm),
                  SUFB200_PRG_KEY_H(P, r, 2, xm, hm), SUFB200_PRG_KEY_H(P, r, 3, xm, hm));
  out.w[0] = aes_last_col<0>(a, lb, SUFB200_PRG_KEY_H(P, 10, 0, xm, hm)) ^ s.w[0];
  out.w[1] = aes_last_col<1>(a, lb, SUFB200_PRG_KEY_H(P, 10, 1, xm, hm)) ^ s.w[1];
  out.w[2] = aes_last_col<2>(a, lb, SUFB200_PRG_KEY_H(P, 10, 2, xm, hm)) ^ s.w[2];
  out.w[3] = aes_last_col<3>(a, lb, SUFB200_PRG_KEY_H(P, 10, 3, xm, hm)) ^ s.w[3];
}

// The four PRG keys' round keys in shared memory for the lane-split walk:
// sk[j * 11 + r] holds round r of key K_j (j = 2x + h), one 16-byte row per
// round, so a lane with half h at a level with bit x reads each round key
// with one 16-byte load instead of selecting it word by word between the
// halves (three logic ops per word).  The four keys' rows fall in different
// bank groups (176-byte key stride), so a warp's loads are one wavefront.
// Filled once per block by all threads; a barrier must follow.
#if !defined(SUFB200_HOST_EMU)
__device__ __forceinline__ void prg_keys_to_smem(const PrgParams& P, uint4* sk) {
  for (int i = threadIdx.x; i < 44; i += blockDim.x) {
    const int j = i / 11, r = i - 11 * (i / 11), h = j & 1;
    const uint32_t xm = (j >> 1) ? ~0u : 0u;
    sk[i] = make_uint4(SUFB200_PRG_KEY(P, h, r, 0, xm), SUFB200_PRG_KEY(P, h, r, 1, xm),
                       SUFB200_PRG_KEY(P, h, r, 2, xm), SUFB200_PRG_KEY(P, h, r, 3, xm));
  }
}
#endif

// prg_half with the round keys from prg_keys_to_smem.
SUFB200_DEV void prg_half_sk(const uint4* sk, uint32_t lb, const Blk& s, uint32_t x, uint32_t h, Blk& out) {
  const uint4* k = sk + (2u * x + h) * 11u;
  const uint4 k0 = k[0];
  Blk a;
  a.w[0] = s.w[0] ^ k0.x;
  a.w[1] = s.w[1] ^ k0.y;
  a.w[2] = s.w[2] ^ k0.z;
  a.w[3] = s.w[3] ^ k0.w;
#pragma unroll
  for (int r = 1; r < 10; r++) {
    const uint4 kr = k[r];
    a = aes_round(a, lb, kr.x, kr.y, kr.z, kr.w);
  }
  const uint4 kl = k[10];
  out.w[0] = aes_last_col<0>(a, lb, kl.x) ^ s.w[0];
  out.w[1] = aes_last_col<1>(a, lb, kl.y) ^ s.w[1];
  out.w[2] = aes_last_col<2>(a, lb, kl.z) ^ s.w[2];
  out.w[3] = aes_last_col<3>(a, lb, kl.w) ^ s.w[3];
}

// Plain AES-128 of one block under 44 round-key words read from shared
// memory (uniform address across the warp) -- the CTR keystream of the
// reference key formats.
SUFB200_DEV Blk aes_encrypt_smem_rk(const Blk& in, uint32_t lb, const uint32_t* rk) {
  Blk a;
#pragma unroll
  for (int c = 0; c < 4; c++) a.w[c] = in.w[c] ^ rk[c];
#pragma unroll
  for (int r = 1; r < 10; r++) a = aes_round(a, lb, rk[4 * r + 0], rk[4 * r + 1], rk[4 * r + 2], rk[4 * r + 3]);
  Blk o;
  o.w[0] = aes_last_col<0>(a, lb, rk[40]);
  o.w[1] = aes_last_col<1>(a, lb, rk[41]);
  o.w[2] = aes_last_col<2>(a, lb, rk[42]);
  o.w[3] = aes_last_col<3>(a, lb, rk[43]);
  return o;
}

// NB independent blocks under the 11 round keys in shared memory (one
// 16-byte broadcast load per round for all NB), their rounds interleaved:
// NB table-lookup chains in flight per thread and no round-key registers.
// The middle rounds stay a loop (one round of NB blocks is about 64 * NB
// instructions): fully unrolled, four blocks are some 40 KB of code, which
// a warp streams through the instruction cache once per element.
template <int NB>
SUFB200_DEV void aes_encrypt_n_sk(Blk (&b)[NB], uint32_t lb, const uint4* rk) {
  const uint4 k0 = rk[0];
#pragma unroll
  for (int j = 0; j < NB; j++) {
    b[j].w[0] ^= k0.x;
    b[j].w[1] ^= k0.y;
    b[j].w[2] ^= k0.z;
    b[j].w[3] ^= k0.w;
  }
#pragma unroll 1
  for (int r = 1; r < 10; r++) {
    const uint4 kr = rk[r];
#pragma unroll
    for (int j = 0; j < NB; j++) b[j] = aes_round(b[j], lb, kr.x, kr.y, kr.z, kr.w);
  }
  const uint4 kl = rk[10];
#pragma unroll
  for (int j = 0; j < NB; j++) {
    Blk o;
    o.w[0] = aes_last_col<0>(b[j], lb, kl.x);
    o.w[1] = aes_last_col<1>(b[j], lb, kl.y);
    o.w[2] = aes_last_col<2>(b[j], lb, kl.z);
    o.w[3] = aes_last_col<3>(b[j], lb, kl.w);
    b[j] = o;
  }
}

// One block under 44 round-key words held in registers (a row of at most
// two words: one CTR block covers it).
SUFB200_DEV Blk aes_encrypt1_rk(const Blk& in, uint32_t lb, const uint32_t (&rk)[44]) {
  Blk a;
#pragma unroll
  for (int c = 0; c < 4; c++) a.w[c] = in.w[c] ^ rk[c];
#pragma unroll
  for (int r = 1; r < 10; r++) a = aes_round(a, lb, rk[4 * r + 0], rk[4 * r + 1], rk[4 * r + 2], rk[4 * r + 3]);
  Blk o;
  o.w[0] = aes_last_col<0>(a, lb, rk[40]);
  o.w[1] = aes_last_col<1>(a, lb, rk[41]);
  o.w[2] = aes_last_col<2>(a, lb, rk[42]);
  o.w[3] = aes_last_col<3>(a, lb, rk[43]);
  return o;
}

// Two independent blocks under the same 44 round-key words held in
// registers, their rounds interleaved (two table-lookup chains in flight per
// thread, no round-key loads) -- the CTR keystream of a short coefficient row.
SUFB200_DEV void aes_encrypt2_rk(const Blk& in0, const Blk& in1, uint32_t lb, const uint32_t (&rk)[44], Blk& o0,
                                 Blk& o1) {
  Blk a, b;
#pragma unroll
  for (int c = 0; c < 4; c++) {
    a.w[c] = in0.w[c] ^ rk[c];
    b.w[c] = in1.w[c] ^ rk[c];
  }
#pragma unroll
  for (int r = 1; r < 10; r++) {
    a = aes_round(a, lb, rk[4 * r + 0], rk[4 * r + 1], rk[4 * r + 2], rk[4 * r + 3]);
    b = aes_round(b, lb, rk[4 * r + 0], rk[4 * r + 1], rk[4 * r + 2], rk[4 * r + 3]);
  }
  o0.w[0] = aes_last_col<0>(a, lb, rk[40]);
  o0.w[1] = aes_last_col<1>(a, lb, rk[41]);
  o0.w[2] = aes_last_col<2>(a, lb, rk[42]);
  o0.w[3] = aes_last_col<3>(a, lb, rk[43]);
  o1.w[0] = aes_last_col<0>(b, lb, rk[40]);
  o1.w[1] = aes_last_col<1>(b, lb, rk[41]);
  o1.w[2] = aes_last_col<2>(b, lb, rk[42]);
  o1.w[3] = aes_last_col<3>(b, lb, rk[43]);
}

}  // namespace sufb200
