// emu_shim.cpp -- CPU build of the device AES engine and DCF walk
// (suf_b200/csrc/aes_smem.cuh, dcf_walk.cuh) against an emulated shared
// window laid out exactly as the kernels lay it out.  Lets the non-GPU tests
// check the table layout, the byte-permute selectors and the walk against
// the oracle before any kernel runs.
#define SUFB200_HOST_EMU 1
#include <cstring>
#include <vector>

#include "../../suf_b200/csrc/dcf_walk.cuh"
#include "../../suf_b200/csrc/host_aes.hpp"

namespace sufb200 {
uint8_t* g_emu_smem = nullptr;
uint32_t g_emu_lane = 0;
}  // namespace sufb200

using namespace sufb200;

namespace {
std::vector<uint8_t> g_window(kTabEnd, 0);
PrgParams g_prg;

void fill_window() {
  const auto& T = host::aes_tables();
  for (uint32_t k = 0; k < 4; k++)
    for (uint32_t x = 0; x < 256; x++)
      for (uint32_t lane = 0; lane < 32; lane++) {
        const uint32_t v = host::rotl(T.t0[x], static_cast<int>(8 * k));
        const uint32_t addr = kTabBase + (k >> 1) * 0x10000u + x * 256u + (k & 1u) * 128u + lane * 4u;
        std::memcpy(&g_window[addr], &v, 4);
      }
  g_emu_smem = g_window.data();
}
}  // namespace

extern "C" int emu_prg_init(const uint8_t* state) {
  fill_window();
  uint32_t w[4][44];
  for (int j = 0; j < 4; j++) host::aes128_expand_words(state + 16 * j, w[j]);
  for (int h = 0; h < 2; h++)
    for (int r = 0; r < 11; r++)
      for (int c = 0; c < 4; c++) {
        g_prg.base[h][r][c] = w[h][4 * r + c];
        g_prg.diff[h][r][c] = w[h][4 * r + c] ^ w[h + 2][4 * r + c];
      }
  return 0;
}

// Blocks 2x and (low half of) 2x+1 of the MMO PRG on `seed`, as lane `lane`.
extern "C" int emu_prg_level(const uint8_t* seed, int x_bit, int lane, uint8_t* outA, uint8_t* outB8) {
  g_emu_lane = static_cast<uint32_t>(lane);
  Blk s, a;
  std::memcpy(s.w, seed, 16);
  uint32_t b0, b1;
  prg_level(g_prg, lane_base(), s, 0u - static_cast<uint32_t>(x_bit & 1), a, b0, b1);
  std::memcpy(outA, a.w, 16);
  std::memcpy(outB8, &b0, 4);
  std::memcpy(outB8 + 4, &b1, 4);
  return 0;
}

// Plain AES of one block with explicit round keys, as lane `lane`.
extern "C" int emu_aes(const uint8_t* key, const uint8_t* in, int lane, uint8_t* out) {
  fill_window();
  g_emu_lane = static_cast<uint32_t>(lane);
  uint32_t rk[44];
  host::aes128_expand_words(key, rk);
  Blk b;
  std::memcpy(b.w, in, 16);
  Blk o = aes_encrypt_smem_rk(b, lane_base(), rk);
  std::memcpy(out, o.w, 16);
  return 0;
}

// One element of the broadcast-key kernel loop (myl7_dcf.cu) on the CPU.
extern "C" int emu_dcf_eval(int group, const uint8_t* k, int in_bits, uint64_t x, int lane, uint64_t* out) {
  g_emu_lane = static_cast<uint32_t>(lane);
  const uint32_t lb = lane_base();
  if (in_bits < 64) x &= (1ull << in_bits) - 1ull;
  const uint32_t party = k[2];
  Blk s;
  std::memcpy(s.w, k + 8, 16);
  s.w[3] &= 0x7FFFFFFFu;
  uint32_t t = party;
  uint64_t v = 0;
  for (int lv = 0; lv < in_bits; lv++) {
    const uint8_t* c = k + 24 + 33 * lv;
    CwLevel cw;
    std::memcpy(cw.s.w, c, 16);
    std::memcpy(&cw.v, c + 16, 8);
    cw.t = c[32];
    const uint32_t xb = static_cast<uint32_t>((x >> (in_bits - 1 - lv)) & 1ull);
    if (group == 0) walk_level<0>(g_prg, lb, s, t, v, xb, party, cw);
    else walk_level<1>(g_prg, lb, s, t, v, xb, party, cw);
  }
  uint64_t np1;
  std::memcpy(&np1, k + 24 + 33 * in_bits, 8);
  *out = group == 0 ? walk_finish<0>(s, t, v, party, np1) : walk_finish<1>(s, t, v, party, np1);
  return 0;
}

// ---- shared-prefix plan (prefix.cuh) on the CPU --------------------------------
#include "../../suf_b200/csrc/prefix.cuh"

extern "C" int emu_make_plan(uint64_t pivot, uint64_t min_b, uint64_t max_b, int n, uint32_t kmax, uint32_t* depth,
                             uint32_t* count, uint64_t* first) {
  RangeAcc r{min_b, max_b, pivot, 0};
  Plan p = make_plan(r, n, kmax);
  *depth = p.depth;
  *count = p.count;
  *first = p.first;
  return 0;
}

extern "C" uint32_t emu_plan_index(uint32_t depth, uint32_t count, uint64_t first, uint64_t x, int n) {
  Plan p{depth, count, first};
  return plan_index(p, x, n);
}

namespace {
CwLevel key_cw(const uint8_t* k, int lv) {
  const uint8_t* c = k + 24 + 33 * lv;
  CwLevel cw;
  std::memcpy(cw.s.w, c, 16);
  std::memcpy(&cw.v, c + 16, 8);
  cw.t = c[32];
  return cw;
}

template <int GROUP>
void frontier_all(const uint8_t* k, int n, const Plan& plan, uint32_t min_roots, uint64_t* out) {
  const uint32_t lb = lane_base();
  const uint32_t party = k[2];
  Blk seed;
  std::memcpy(seed.w, k + 8, 16);
  seed.w[3] &= 0x7FFFFFFFu;
  uint64_t np1;
  std::memcpy(&np1, k + 24 + 33 * n, 8);
  const int h = expand_height(plan, min_roots);
  const uint64_t roots = root_count(plan, h);
  const bool final_level = static_cast<int>(plan.depth) == n;
  const auto cw_at = [k](int lv) { return key_cw(k, lv); };
  const auto emit = [&](uint64_t slot, const Blk& s, uint32_t t, uint64_t v) {
    uint64_t* e = out + 4 * slot;
    const uint64_t writes = (e[3] >> 32) + 1ull;
    if (final_level) {
      e[0] = e[1] = 0;
      e[2] = walk_finish<GROUP>(s, t, v, party, np1);
      e[3] = 0;
    } else {
      e[0] = (static_cast<uint64_t>(s.w[1]) << 32) | s.w[0];
      e[1] = (static_cast<uint64_t>(s.w[3]) << 32) | s.w[2];
      e[2] = v;
      e[3] = t;
    }
    e[3] |= writes << 32;  // times written: the caller checks every slot was written once
  };
  for (uint64_t j = 0; j < roots; j++) frontier_root<GROUP>(g_prg, lb, seed, party, plan, h, j, cw_at, emit);
}
}  // namespace

// The frontier pass of prefix.cu on the CPU: out[4 * slot ..] = {s lo, s hi,
// v, t | writes << 32} for every entry (final outputs in v when depth == n);
// out must be zeroed.
// Returns the subtree height used.
extern "C" int emu_frontier(int group, const uint8_t* k, int n, uint32_t depth, uint32_t count, uint64_t first,
                            uint32_t min_roots, uint64_t* out) {
  g_emu_lane = 0;
  const Plan p{depth, count, first};
  if (group == 0) frontier_all<0>(k, n, p, min_roots, out);
  else frontier_all<1>(k, n, p, min_roots, out);
  return expand_height(p, min_roots);
}

// Walk state after the top `depth` bits of `prefix` (given as a level-depth
// prefix), or the final output when depth == n: the entry a frontier slot
// must hold.
extern "C" int emu_walk_prefix(int group, const uint8_t* k, int n, uint32_t depth, uint64_t prefix, uint64_t* e) {
  g_emu_lane = 0;
  const uint32_t lb = lane_base();
  const uint32_t party = k[2];
  Blk s;
  std::memcpy(s.w, k + 8, 16);
  s.w[3] &= 0x7FFFFFFFu;
  uint32_t t = party;
  uint64_t v = 0;
  for (uint32_t lv = 0; lv < depth; lv++) {
    const uint32_t xb = static_cast<uint32_t>((prefix >> (depth - 1 - lv)) & 1ull);
    if (group == 0) walk_level<0>(g_prg, lb, s, t, v, xb, party, key_cw(k, static_cast<int>(lv)));
    else walk_level<1>(g_prg, lb, s, t, v, xb, party, key_cw(k, static_cast<int>(lv)));
  }
  if (static_cast<int>(depth) == n) {
    uint64_t np1;
    std::memcpy(&np1, k + 24 + 33 * n, 8);
    e[0] = e[1] = 0;
    e[2] = group == 0 ? walk_finish<0>(s, t, v, party, np1) : walk_finish<1>(s, t, v, party, np1);
    e[3] = 0;
  } else {
    e[0] = (static_cast<uint64_t>(s.w[1]) << 32) | s.w[0];
    e[1] = (static_cast<uint64_t>(s.w[3]) << 32) | s.w[2];
    e[2] = v;
    e[3] = t;
  }
  return 0;
}
