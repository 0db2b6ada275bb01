// prefix.cuh -- shared-prefix evaluation of broadcast DCF keys (device side).
//
// With one key for a whole batch, the walk state after D levels (seed s,
// control bit t, low 64 bits of the value accumulator v) depends only on the
// top D bits of the input.  A batch whose inputs lie in a window [lo, lo + W]
// (mod 2^n) touches few distinct D-bit prefixes, so:
//   1. range_kernel finds the window: signed offsets of every input from a
//      pivot (the first element), min and max, by atomics;
//   2. make_plan picks the deepest D <= n whose prefix count fits a budget;
//   3. a frontier pass computes the state of each of those prefixes (for
//      D = n: the finished output -- a full-domain table when the window
//      covers the whole n-bit space): one thread walks from the root to a
//      subtree root at level D - h, then expands the h levels below it
//      depth-first, both children of every inner node, so a prefix costs
//      about 4 + 2(D - h)/2^h AES blocks instead of 2D (h <= 7);
//   4. the main pass resumes every element from its prefix's state at level D.
// The outputs are the same bits as a walk from the root: step 4 replays the
// identical level sequence, it only skips recomputing shared levels.
#pragma once

#include "dcf_walk.cuh"

namespace sufb200 {

struct RangeAcc {
  unsigned long long min_b;  // min over (x - pivot) as int64, biased by 2^63
  unsigned long long max_b;  // max, biased
  uint64_t pivot;
  uint64_t pad;
};

struct Plan {
  uint32_t depth;  // D
  uint32_t count;  // number of frontier entries
  uint64_t first;  // first D-bit prefix (entries cover first .. first + count - 1 mod 2^D)
};

struct FrontierEntry {  // 32 bytes, one sector
  uint32_t s[4];
  uint64_t v;
  uint32_t t;
  uint32_t pad;
};

SUFB200_HD uint64_t nbit_mask(int n) { return n >= 64 ? ~0ull : ((1ull << n) - 1ull); }

// Deepest D <= n whose prefix count over the window is <= kmax (D = 0 always fits).
// At depth D a prefix is a bucket of 2^(n-D) consecutive n-bit values; the
// window [lo, lo + W] (mod 2^n) starting at offset o inside its first bucket
// crosses floor((o + W) / 2^(n-D)) + 1 buckets, capped at all 2^D of them.
SUFB200_HD Plan make_plan(const RangeAcc& r, int n, uint32_t kmax) {
  const int64_t mn = static_cast<int64_t>(r.min_b - (1ull << 63));
  const int64_t mx = static_cast<int64_t>(r.max_b - (1ull << 63));
  Plan p{0, 1, 0};
  if (r.min_b > r.max_b) return p;  // empty batch
  const uint64_t lo = r.pivot + static_cast<uint64_t>(mn);
  const uint64_t width = static_cast<uint64_t>(mx) - static_cast<uint64_t>(mn);
  const uint64_t lo_n = lo & nbit_mask(n);
  for (int d = n; d >= 1; d--) {
    const int sh = n - d;  // bucket = 2^sh values, sh in [0, 63]
    const uint64_t bm = nbit_mask(sh);
    const uint64_t q = width >> sh;
    const uint64_t carry = ((lo_n & bm) + (width & bm)) >> sh;  // < 2^(sh+1): no overflow
    const uint64_t all = d >= 64 ? 0ull : (1ull << d);           // 0 encodes 2^64
    uint64_t cnt = q + carry + 1ull;                               // 0 on wrap to 2^64
    const bool covers_all = (all != 0) && (cnt == 0 || cnt >= all || q >= all);
    if (covers_all) cnt = all;
    if (cnt != 0 && cnt <= kmax) {
      p.depth = static_cast<uint32_t>(d);
      p.count = static_cast<uint32_t>(cnt);
      p.first = covers_all ? 0ull : (lo_n >> sh);
      return p;
    }
  }
  return p;
}

// Subtree height h of the frontier pass: the largest h <= min(7, D) that still
// leaves at least kMinRoots subtree roots (so the pass fills the GPU).  It
// only decides how the frontier work is split; the entries are the same.  At
// h = 7 an entry costs about 4 + 2(D - 7)/128 AES blocks.
constexpr int kMaxExpand = 7;
constexpr uint32_t kMinRoots = 8192;

SUFB200_HD int expand_height(const Plan& p, uint32_t min_roots = kMinRoots) {
  int h = 0;
  while (h < kMaxExpand && h < static_cast<int>(p.depth) && (p.count >> (h + 1)) >= min_roots) h++;
  return h;
}

// Number of level-(D - h) subtree roots whose subtrees cover the plan's
// prefixes first .. first + count - 1 (mod 2^D).
SUFB200_HD uint64_t root_count(const Plan& p, int h) {
  const uint64_t off = p.first & nbit_mask(h);
  uint64_t c = ((off + p.count - 1ull) >> h) + 1ull;
  const int d0 = static_cast<int>(p.depth) - h;
  if (d0 < 64 && c > (1ull << d0)) c = 1ull << d0;
  return c;
}

// Frontier index of an element, or count (= not covered) when outside.
SUFB200_HD uint32_t plan_index(const Plan& p, uint64_t x, int n) {
  if (p.depth == 0) return 0;
  const uint64_t pre = (x & nbit_mask(n)) >> (n - static_cast<int>(p.depth));
  const uint64_t idx = (pre - p.first) & nbit_mask(static_cast<int>(p.depth));
  return idx < p.count ? static_cast<uint32_t>(idx) : p.count;
}

}  // namespace sufb200

namespace sufb200 {

SUFB200_HD int high_bit(uint32_t x) {  // x != 0
#if defined(__CUDA_ARCH__)
  return 31 - __clz(static_cast<int>(x));
#else
  return 31 - __builtin_clz(x);
#endif
}

// The frontier entries under subtree root j of the frontier pass.  The root
// is R = (first >> h) + j at level d0 = D - h; the walk follows R's bits from
// the seed, then visits the 2^h leaves below R in order, recomputing only
// the levels under the highest bit that changed from the previous leaf (a
// stack holds the states at levels d0 .. D-1), so each child in the subtree
// is computed once.  emit(slot, s, t, v) receives every leaf inside
// first .. first + count - 1 (slot = its index there); cw_at(level) returns
// the correction word of a level.
template <int GROUP, typename CwAt, typename Emit>
SUFB200_DEV void frontier_root(const PrgParams& prg, uint32_t lb, const Blk& seed, uint32_t party, const Plan& plan,
                               int h, uint64_t j, const CwAt& cw_at, const Emit& emit) {
  const int D = static_cast<int>(plan.depth);
  const int d0 = D - h;
  const uint64_t dmask = nbit_mask(D);
  const uint64_t R = ((plan.first >> h) + j) & nbit_mask(d0);
  Blk s = seed;
  uint32_t t = party;
  uint64_t v = 0;
  for (int lv = 0; lv < d0; lv++)
    walk_level<GROUP>(prg, lb, s, t, v, static_cast<uint32_t>((R >> (d0 - 1 - lv)) & 1ull), party, cw_at(lv));
  if (h == 0) {  // R is a level-D prefix and j < count: inside the window
    emit((R - plan.first) & dmask, s, t, v);
    return;
  }
  uint32_t st[kMaxExpand][8];  // s[4], t, v lo, v hi
  st[0][0] = s.w[0];
  st[0][1] = s.w[1];
  st[0][2] = s.w[2];
  st[0][3] = s.w[3];
  st[0][4] = t;
  st[0][5] = static_cast<uint32_t>(v);
  st[0][6] = static_cast<uint32_t>(v >> 32);
  for (uint32_t k = 0; k < (1u << h); k++) {
    const int l0 = k ? (h - 1 - high_bit(k ^ (k - 1u))) : 0;
    s.w[0] = st[l0][0];
    s.w[1] = st[l0][1];
    s.w[2] = st[l0][2];
    s.w[3] = st[l0][3];
    t = st[l0][4];
    v = (static_cast<uint64_t>(st[l0][6]) << 32) | st[l0][5];
    for (int l = l0; l < h; l++) {
      walk_level<GROUP>(prg, lb, s, t, v, (k >> (h - 1 - l)) & 1u, party, cw_at(d0 + l));
      if (l + 1 < h) {
        st[l + 1][0] = s.w[0];
        st[l + 1][1] = s.w[1];
        st[l + 1][2] = s.w[2];
        st[l + 1][3] = s.w[3];
        st[l + 1][4] = t;
        st[l + 1][5] = static_cast<uint32_t>(v);
        st[l + 1][6] = static_cast<uint32_t>(v >> 32);
      }
    }
    const uint64_t slot = ((((R << h) | k) & dmask) - plan.first) & dmask;
    if (slot < plan.count) emit(slot, s, t, v);
  }
}

#if !defined(SUFB200_HOST_EMU)
// frontier_root over a lane pair (lanes 2k and 2k + 1 of a warp, hsel = lane
// & 1, pmask = both lanes' bits; sk: prg_keys_to_smem's round keys): every
// level is walk_level_split, each lane
// computing one of the level's two MMO blocks, so the serial chain of a work
// item is one AES block per level instead of two.  Both lanes hold the same
// states throughout; lane hsel = 0 emits.
template <int GROUP, typename CwAt, typename Emit>
__device__ __forceinline__ void frontier_root_pair(const uint4* sk, uint32_t lb, const Blk& seed,
                                                   uint32_t party, const Plan& plan, int h, uint64_t j,
                                                   const CwAt& cw_at, const Emit& emit, uint32_t hsel,
                                                   uint32_t pmask) {
  const int D = static_cast<int>(plan.depth);
  const int d0 = D - h;
  const uint64_t dmask = nbit_mask(D);
  const uint64_t R = ((plan.first >> h) + j) & nbit_mask(d0);
  Blk s = seed;
  uint32_t t = party;
  uint64_t v = 0;
  for (int lv = 0; lv < d0; lv++)
    walk_level_split<GROUP>(sk, lb, s, t, v, static_cast<uint32_t>((R >> (d0 - 1 - lv)) & 1ull), party, cw_at(lv),
                            hsel, pmask);
  if (h == 0) {
    if (hsel == 0) emit((R - plan.first) & dmask, s, t, v);
    return;
  }
  uint32_t st[kMaxExpand][8];
  st[0][0] = s.w[0];
  st[0][1] = s.w[1];
  st[0][2] = s.w[2];
  st[0][3] = s.w[3];
  st[0][4] = t;
  st[0][5] = static_cast<uint32_t>(v);
  st[0][6] = static_cast<uint32_t>(v >> 32);
  for (uint32_t k = 0; k < (1u << h); k++) {
    const int l0 = k ? (h - 1 - high_bit(k ^ (k - 1u))) : 0;
    s.w[0] = st[l0][0];
    s.w[1] = st[l0][1];
    s.w[2] = st[l0][2];
    s.w[3] = st[l0][3];
    t = st[l0][4];
    v = (static_cast<uint64_t>(st[l0][6]) << 32) | st[l0][5];
    for (int l = l0; l < h; l++) {
      walk_level_split<GROUP>(sk, lb, s, t, v, (k >> (h - 1 - l)) & 1u, party, cw_at(d0 + l), hsel, pmask);
      if (l + 1 < h) {
        st[l + 1][0] = s.w[0];
        st[l + 1][1] = s.w[1];
        st[l + 1][2] = s.w[2];
        st[l + 1][3] = s.w[3];
        st[l + 1][4] = t;
        st[l + 1][5] = static_cast<uint32_t>(v);
        st[l + 1][6] = static_cast<uint32_t>(v >> 32);
      }
    }
    const uint64_t slot = ((((R << h) | k) & dmask) - plan.first) & dmask;
    if (hsel == 0 && slot < plan.count) emit(slot, s, t, v);
  }
}
#endif  // !SUFB200_HOST_EMU

}  // namespace sufb200
