// prefix.cuh -- shared-prefix evaluation of broadcast DCF keys (device side).
//
// With one key for a whole batch, the walk state after D levels (seed s,
// control bit t, low 64 bits of the value accumulator v) depends only on the
// top D bits of the input.  A batch whose inputs lie in a window [lo, lo + W]
// (mod 2^n) touches few distinct D-bit prefixes, so:
//   1. range_kernel finds the window: signed offsets of every input from a
//      pivot (the first element), min and max, by atomics;
//   2. make_plan picks the deepest D <= n whose prefix count fits a budget;
//   3. a frontier pass walks each of those prefixes once from the root and
//      stores its state (for D = n: the finished output -- a full-domain
//      table when the window covers the whole n-bit space);
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

// Frontier index of an element, or count (= not covered) when outside.
SUFB200_HD uint32_t plan_index(const Plan& p, uint64_t x, int n) {
  if (p.depth == 0) return 0;
  const uint64_t pre = (x & nbit_mask(n)) >> (n - static_cast<int>(p.depth));
  const uint64_t idx = (pre - p.first) & nbit_mask(static_cast<int>(p.depth));
  return idx < p.count ? static_cast<uint32_t>(idx) : p.count;
}

}  // namespace sufb200
