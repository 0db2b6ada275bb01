// trunc_bundle.cu -- fused truncation / ARS bundle for sm_100a.
//
// One launch evaluates every raw predicate query of a FaithfulTR /
// FaithfulARS / GapARS gate (broadcast myl7 keys, AddU64 payload 1), folds
// the additive boolean plan of composite_eval_batch_backend
// (include/gates/composite_fss.hpp:1385-1638) and applies the postproc hook
// (include/gates/postproc_hooks.hpp:173-376), writing one y share per
// element.  The reference runs the same steps as nq separate GPU calls, each
// followed by a device-to-host copy, then two OpenMP host loops.
#include "dcf_walk.cuh"
#include "kernels.hpp"
#include "prefix.cuh"

namespace sufb200 {

namespace {

struct QueryKeySmem {
  uint4 cw_s[64];
  uint64_t cw_v[64];
  uint32_t cw_t[64];
  uint4 seed;
  uint64_t np1_lo;
  uint32_t ok;
  uint32_t pad;
};
static_assert(8 * sizeof(QueryKeySmem) % 16 == 0 && 8 * sizeof(QueryKeySmem) + 44 * 16 < kTabBase - 4096,
              "staging (two bundles and the PRG round keys) must fit below the tables");

__device__ __forceinline__ uint32_t ldb32(const uint8_t* p) {
  return static_cast<uint32_t>(p[0]) | (static_cast<uint32_t>(p[1]) << 8) | (static_cast<uint32_t>(p[2]) << 16) |
         (static_cast<uint32_t>(p[3]) << 24);
}
__device__ __forceinline__ uint64_t ldb64(const uint8_t* p) {
  return static_cast<uint64_t>(ldb32(p)) | (static_cast<uint64_t>(ldb32(p + 4)) << 32);
}

__device__ __forceinline__ uint64_t pick4(int q, uint64_t p0, uint64_t p1, uint64_t p2, uint64_t p3) {
  return q == 0 ? p0 : (q == 1 ? p1 : (q == 2 ? p2 : p3));
}

// The AddU64 boolean plan (composite_fss.hpp:1539-1605) and the kind's
// postproc hook (postproc_hooks.hpp:173-376) for one element.
__device__ __forceinline__ void combine_store(const sufb200_trunc_desc& d, uint64_t xh, const uint64_t pr[4],
                                              uint64_t* y_out, uint64_t* bools, size_t i) {
  const uint32_t party = static_cast<uint32_t>(d.party);
  const int f = d.frac_bits;
  const uint64_t one = party == 0 ? 1ull : 0ull;
  uint64_t carry = 0, sign = 0, wrap = 0;
  if (d.carry_a >= 0) {
    const uint64_t qa = pick4(d.carry_a, pr[0], pr[1], pr[2], pr[3]);
    const uint64_t qb = pick4(d.carry_b, pr[0], pr[1], pr[2], pr[3]);
    carry = one - ((qb - qa) + d.carry_w);
  }
  if (d.sign_a >= 0) {
    const uint64_t qa = pick4(d.sign_a, pr[0], pr[1], pr[2], pr[3]);
    const uint64_t qb = pick4(d.sign_b, pr[0], pr[1], pr[2], pr[3]);
    sign = (qb - qa) + d.sign_w;
  }
  if (d.wrap_q >= 0) wrap = pick4(d.wrap_q, pr[0], pr[1], pr[2], pr[3]);
  uint64_t y;
  if (d.kind == SUFB200_TRUNC_GAPARS) {
    // GapArsPostProc::run_batch, postproc_hooks.hpp:324-375
    const uint64_t hb = xh + (1ull << 62);
    uint64_t top = 0;
    if (party == 0 && f >= 0 && f < 64) top = f == 0 ? hb : (hb >> f);
    y = d.haty + top - d.r_hi - carry;
    if (f > 0 && f < 64 && ((hb >> 63) & 1ull) == 0) y += d.m;
    if (party == 0) y -= (f >= 0 && f <= 62) ? (1ull << (62 - f)) : 0ull;
  } else {
    // FaithfulTruncPostProc / FaithfulArsPostProc::run_batch, postproc_hooks.hpp:198-290
    const uint64_t top = (party == 0 && f < 64) ? (xh >> f) : 0ull;
    const uint64_t modulus = (f <= 0 || f >= 64) ? 0ull : (1ull << (64 - f));
    y = d.haty + top - d.r_hi - carry;
    if (modulus) y += wrap * modulus;
    if (d.kind == SUFB200_TRUNC_FAITHFUL_ARS) {
      const uint64_t sign_mask = (f <= 0 || f >= 64) ? 0ull : (~0ull << (64 - f));
      y += sign * sign_mask;
    }
  }
  y_out[i] = y;
  if (bools) {
    bools[3 * i + 0] = carry;
    bools[3 * i + 1] = sign;
    bools[3 * i + 2] = wrap;
  }
}

// Copy every query key of the bundle into shared memory (no barrier).
__device__ __forceinline__ void stage_keys(QueryKeySmem* ks, const TruncLaunch& a) {
  const sufb200_trunc_desc& d = a.desc;
  for (int q = 0; q < d.nq; q++) {
    const uint8_t* k = a.key[q];
    const int nb = d.q_bits[q];
    for (int i = threadIdx.x; i < nb; i += blockDim.x) {
      const uint8_t* c = k + 24 + 33 * i;
      ks[q].cw_s[i] = make_uint4(ldb32(c), ldb32(c + 4), ldb32(c + 8), ldb32(c + 12));
      ks[q].cw_v[i] = ldb64(c + 16);
      ks[q].cw_t[i] = c[32];
    }
    if (threadIdx.x == 0) {
      const uint64_t hdr = ldb64(k);
      const bool ok = (hdr & 0xFF) == static_cast<uint64_t>(nb) && ((hdr >> 8) & 0xFF) == 1 &&
                      ((hdr >> 16) & 0xFF) == static_cast<uint64_t>(d.party) && (hdr >> 32) == 8;
      ks[q].seed = make_uint4(ldb32(k + 8), ldb32(k + 12), ldb32(k + 16), ldb32(k + 20) & 0x7FFFFFFFu);
      ks[q].np1_lo = ldb64(k + 24 + 33 * nb);
      ks[q].ok = ok ? 1u : 0u;
    }
  }
}

// After the barrier: false (status flagged) when a key header did not match.
__device__ __forceinline__ bool keys_ok(const QueryKeySmem* ks, const TruncLaunch& a) {
  for (int q = 0; q < a.desc.nq; q++) {
    if (!ks[q].ok) {
      if (threadIdx.x == 0 && blockIdx.x == 0) atomicOr(a.status, kStatusBadKeyHeader);
      return false;
    }
  }
  return true;
}

// Stage every query key of the bundle into shared memory, fill the AES
// tables; false (status flagged) when a key header does not match.
__device__ __forceinline__ bool stage_bundle(QueryKeySmem* ks, const TruncLaunch& a) {
  aes_fill_tables(a.t0);
  pdl_wait();  // the tables overlap the previous kernel's tail; its outputs are read below
  pdl_trigger();
  stage_keys(ks, a);
  __syncthreads();
  return keys_ok(ks, a);
}

// Walk levels [from, n) of one query from state (s, t, v); returns the share.
__device__ __forceinline__ uint64_t walk_query(const PrgParams& prg, uint32_t lb, const QueryKeySmem& K, int n,
                                               uint64_t x, uint32_t party, Blk s, uint32_t t, uint64_t v, int from) {
  for (int lv = from; lv < n; lv++) {
    CwLevel cw;
    const uint4 cs = K.cw_s[lv];
    cw.s.w[0] = cs.x;
    cw.s.w[1] = cs.y;
    cw.s.w[2] = cs.z;
    cw.s.w[3] = cs.w;
    cw.v = K.cw_v[lv];
    cw.t = K.cw_t[lv];
    walk_level<SUFB200_GROUP_ADD>(prg, lb, s, t, v, static_cast<uint32_t>((x >> (n - 1 - lv)) & 1ull), party, cw);
  }
  return walk_finish<SUFB200_GROUP_ADD>(s, t, v, party, K.np1_lo);
}

// walk_query over a lane pair (walk_level_split): lanes 2k and 2k+1 of the
// warp walk the same query together; both return the share.
__device__ __forceinline__ uint64_t walk_query_split(const uint4* sk, uint32_t lb, const QueryKeySmem& K, int n,
                                                     uint64_t x, uint32_t party, Blk s, uint32_t t, uint64_t v,
                                                     uint32_t h, uint32_t pmask) {
  for (int lv = 0; lv < n; lv++) {
    CwLevel cw;
    const uint4 cs = K.cw_s[lv];
    cw.s.w[0] = cs.x;
    cw.s.w[1] = cs.y;
    cw.s.w[2] = cs.z;
    cw.s.w[3] = cs.w;
    cw.v = K.cw_v[lv];
    cw.t = K.cw_t[lv];
    walk_level_split<SUFB200_GROUP_ADD>(sk, lb, s, t, v, static_cast<uint32_t>((x >> (n - 1 - lv)) & 1ull), party,
                                        cw, h, pmask);
  }
  return walk_finish<SUFB200_GROUP_ADD>(s, t, v, party, K.np1_lo);
}

__device__ __forceinline__ Blk seed_blk(const QueryKeySmem& K) {
  Blk s;
  s.w[0] = K.seed.x;
  s.w[1] = K.seed.y;
  s.w[2] = K.seed.z;
  s.w[3] = K.seed.w;
  return s;
}

__global__ void __launch_bounds__(kAesThreads, 1) trunc_bundle_kernel(const PrgParams prg, const TruncLaunch a) {
  extern __shared__ __align__(16) uint8_t smem[];
  if (!aes_layout_ok()) {
    if (threadIdx.x == 0) atomicOr(a.status, kStatusSmemLayout);
    pdl_wait();
    return;
  }
  const sufb200_trunc_desc& d = a.desc;
  QueryKeySmem* ks = reinterpret_cast<QueryKeySmem*>(smem);
  if (!stage_bundle(ks, a)) return;
  const uint32_t lb = lane_base();
  const uint32_t party = static_cast<uint32_t>(d.party);
  const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
  for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < a.n; i += stride) {
    const uint64_t xh = a.xhat[i];
    uint64_t pr[4] = {0, 0, 0, 0};
#pragma unroll 1
    for (int q = 0; q < d.nq; q++) {
      const int nb = d.q_bits[q];
      const uint64_t x = nb >= 64 ? xh : (xh & ((1ull << nb) - 1ull));
      const uint64_t v = walk_query(prg, lb, ks[q], nb, x, party, seed_blk(ks[q]), party, 0, 0);
      if (q == 0) pr[0] = v;
      else if (q == 1) pr[1] = v;
      else if (q == 2) pr[2] = v;
      else pr[3] = v;
    }
    combine_store(d, xh, pr, a.y, a.bools, i);
  }
}


// Small batches of both parties' bundles over one x^: a lane pair per (party,
// element, query) -- each lane computes one of a tree level's two MMO blocks
// and the pair swaps them (walk_level_split) -- and `lanes` (2, 4 or 8: twice
// the bundle's query count rounded up) lanes per element, so the queries of
// an element run side by side instead of one after another and both parties
// fill one launch; lane 0 of each group gathers the group's shares and folds
// the plan and the postproc.  For batches too small to fill the GPU with one
// lane per element (the row-level truncations of the softmax and LayerNorm
// blocks), which are bound by the latency of the sequential tree levels.
__global__ void __launch_bounds__(kAesThreads, 1)
    trunc_bundle_pair_kernel(const PrgParams prg, const __grid_constant__ TruncLaunch a0,
                             const __grid_constant__ TruncLaunch a1, int lanes) {
  extern __shared__ __align__(16) uint8_t smem[];
  if (!aes_layout_ok()) {
    if (threadIdx.x == 0) atomicOr(a0.status, kStatusSmemLayout);
    pdl_wait();
    return;
  }
  QueryKeySmem* ks = reinterpret_cast<QueryKeySmem*>(smem);  // party p, query q at ks[4 p + q]
  uint4* sk = reinterpret_cast<uint4*>(smem + 8 * sizeof(QueryKeySmem));  // the PRG keys' round keys
  aes_fill_tables(a0.t0);
  prg_keys_to_smem(prg, sk);
  pdl_wait();
  pdl_trigger();
  stage_keys(ks, a0);
  stage_keys(ks + 4, a1);
  __syncthreads();
  if (!keys_ok(ks, a0) || !keys_ok(ks + 4, a1)) return;
  const uint32_t lb = lane_base();
  const int lsh = lanes >= 8 ? 3 : (lanes >= 4 ? 2 : 1);  // lanes per element = 1 << lsh
  const size_t n = a0.n, units = (2 * n) << lsh;           // 2 parties x n elements x lanes
  const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
  const int lane = static_cast<int>(threadIdx.x & 31u), grp = lane & ~((1 << lsh) - 1);
  for (size_t g0 = static_cast<size_t>(blockIdx.x) * blockDim.x; g0 < units; g0 += stride) {
    const size_t g = g0 + threadIdx.x;  // g0 is uniform across the block: every lane reaches the shuffles
    const bool valid = g < units;
    const size_t j = g >> lsh;
    const int u = static_cast<int>(g & ((1u << lsh) - 1u));
    const int q = u >> 1;                      // query of the lane pair
    const uint32_t h = static_cast<uint32_t>(u & 1);  // which MMO block of a level this lane computes
    const uint32_t party = j >= n ? 1u : 0u;
    const size_t i = party ? j - n : j;
    const TruncLaunch* a = party ? &a1 : &a0;
    const sufb200_trunc_desc& d = a->desc;
    const uint64_t xh = valid ? a->xhat[i] : 0ull;
    uint64_t v = 0;
    if (valid && q < d.nq) {
      const int nb = d.q_bits[q];
      const uint64_t x = nb >= 64 ? xh : (xh & ((1ull << nb) - 1ull));
      const QueryKeySmem& K = ks[4 * party + q];
      v = walk_query_split(sk, lb, K, nb, x, party, seed_blk(K), party, 0, h, 3u << (lane & ~1));
    }
    uint64_t pr[4];
#pragma unroll
    for (int k = 0; k < 4; k++) {
      const uint64_t w = __shfl_sync(0xffffffffu, v, grp + (2 * k < (1 << lsh) ? 2 * k : 0));
      pr[k] = 2 * k < (1 << lsh) ? w : 0ull;
    }
    if (valid && u == 0) combine_store(d, xh, pr, a->y, a->bools, i);
  }
}

// Large batches: every query resumes from its frontier entry (prefix.cuh).
struct FrontierSet {
  const FrontierEntry* F[8];  // F[4 p + q]: party slot p's query q
};

// Per-query plan, frontier table and width, staged once per block after the
// keys (the query loop index is uniform across a warp, so these are
// broadcast reads instead of per-thread local-memory copies).
struct QueryPlanSmem {
  Plan plan;
  const FrontierEntry* F;
  int nb;
  int pad;
};
static_assert(8 * sizeof(QueryKeySmem) + 8 * sizeof(QueryPlanSmem) < kTabBase - 4096,
              "staging must fit below the tables");

// NP = 1: one party's bundle; NP = 2: both parties' bundles over one x^ in
// one pass (elements [0, n) party 0, [n, 2n) party 1), so a pair of
// element-level truncations costs one range, one frontier and one main
// launch instead of two of each.
template <int NP>
__global__ void __launch_bounds__(kAesThreads, 1)
    trunc_bundle_prefix_kernel(const PrgParams prg, const __grid_constant__ TruncLaunch a0,
                               const __grid_constant__ TruncLaunch a1, const RangeAcc* acc, uint32_t kmax,
                               const FrontierSet fs) {
  extern __shared__ __align__(16) uint8_t smem[];
  if (!aes_layout_ok()) {
    if (threadIdx.x == 0) atomicOr(a0.status, kStatusSmemLayout);
    pdl_wait();
    return;
  }
  QueryKeySmem* ks = reinterpret_cast<QueryKeySmem*>(smem);
  QueryPlanSmem* qp = reinterpret_cast<QueryPlanSmem*>(smem + 8 * sizeof(QueryKeySmem));
  __shared__ int s_walks;  // 1 when some query resumes above its last level (needs the AES tables)
  pdl_wait();  // the plan reads the range pass's result
  pdl_trigger();
  if (threadIdx.x == 0) {
    int walks = 0;
#pragma unroll
    for (int p = 0; p < NP; p++) {
      const sufb200_trunc_desc& dp = p ? a1.desc : a0.desc;
#pragma unroll
      for (int q = 0; q < 4; q++) {
        const int nb = dp.q_bits[q];
        qp[4 * p + q].plan = q < dp.nq ? make_plan(*acc, nb, kmax) : Plan{0, 1, 0};
        qp[4 * p + q].F = fs.F[4 * p + q];
        qp[4 * p + q].nb = nb;
        qp[4 * p + q].pad = 0;
        if (q < dp.nq && qp[4 * p + q].plan.depth != static_cast<uint32_t>(nb)) walks = 1;
      }
    }
    s_walks = walks;
  }
  stage_keys(ks, a0);
  if (NP == 2) stage_keys(ks + 4, a1);
  __syncthreads();
  // With every query planned at its full depth the pass is table lookups
  // (the plan's window holds every element of the batch), so the AES tables
  // are filled only when some query resumes a walk.
  const bool walks = s_walks != 0;
  if (walks) aes_fill_tables(a0.t0);
  __syncthreads();  // also publishes qp
  if (!keys_ok(ks, a0) || (NP == 2 && !keys_ok(ks + 4, a1))) return;
  const uint32_t lb = lane_base();
  const size_t n = a0.n, total = static_cast<size_t>(NP) * n;
  const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
  for (size_t g = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; g < total; g += stride) {
    const int slot = (NP == 2 && g >= n) ? 1 : 0;
    const size_t i = slot ? g - n : g;
    const TruncLaunch& a = slot ? a1 : a0;
    const sufb200_trunc_desc& d = a.desc;
    const uint32_t party = static_cast<uint32_t>(d.party);
    const QueryKeySmem* kq = ks + 4 * slot;
    const QueryPlanSmem* pq = qp + 4 * slot;
    const uint64_t xh = a.xhat[i];
    uint64_t pr[4] = {0, 0, 0, 0};
#pragma unroll 1
    for (int q = 0; q < d.nq; q++) {
      const int nb = pq[q].nb;
      const uint64_t x = xh & nbit_mask(nb);
      const Plan P = pq[q].plan;
      const uint32_t idx = plan_index(P, x, nb);
      uint64_t v;
      if (idx < P.count) {
        const FrontierEntry e = pq[q].F[idx];
        if (P.depth == static_cast<uint32_t>(nb)) {
          v = e.v;
        } else {
          Blk s;
          s.w[0] = e.s[0];
          s.w[1] = e.s[1];
          s.w[2] = e.s[2];
          s.w[3] = e.s[3];
          v = walk_query(prg, lb, kq[q], nb, x, party, s, e.t, e.v, static_cast<int>(P.depth));
        }
      } else if (walks) {
        v = walk_query(prg, lb, kq[q], nb, x, party, seed_blk(kq[q]), party, 0, 0);
      } else {
        // outside the window of a lookup-only pass: cannot happen for the
        // batch the range was taken over; flagged rather than walked without
        // tables
        atomicOr(a.status, kStatusBadArgument);
        v = 0;
      }
      if (q == 0) pr[0] = v;
      else if (q == 1) pr[1] = v;
      else if (q == 2) pr[2] = v;
      else pr[3] = v;
    }
    combine_store(d, xh, pr, a.y, a.bools, i);
  }
}

// Both parties' bundles over one x^ against full-domain tables (every
// query planned at its whole domain): an element's predicate share is one
// 32-byte frontier entry per query, so the pass needs neither the keys nor
// the AES tables and runs as a plain memory pass, several blocks per SM.
__global__ void __launch_bounds__(256) trunc_bundle_lookup_pair_kernel(const __grid_constant__ TruncLaunch a0,
                                                                       const __grid_constant__ TruncLaunch a1,
                                                                       const RangeAcc* acc, uint32_t kmax,
                                                                       const FrontierSet fs) {
  __shared__ Plan s_plan[8];
  pdl_wait();  // x^ (and the tables) come from earlier work
  pdl_trigger();
  if (threadIdx.x < 8) {
    const int p = threadIdx.x >> 2, q = threadIdx.x & 3;
    const sufb200_trunc_desc& d = p ? a1.desc : a0.desc;
    s_plan[threadIdx.x] = q < d.nq ? make_plan(*acc, d.q_bits[q], kmax) : Plan{0, 1, 0};
  }
  __syncthreads();
  const size_t n = a0.n, total = 2 * n;
  const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
  for (size_t g = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; g < total; g += stride) {
    const int slot = g >= n ? 1 : 0;
    const size_t i = slot ? g - n : g;
    const TruncLaunch& a = slot ? a1 : a0;
    const sufb200_trunc_desc& d = a.desc;
    const uint64_t xh = a.xhat[i];
    uint64_t pr[4] = {0, 0, 0, 0};
#pragma unroll
    for (int q = 0; q < 4; q++) {
      if (q >= d.nq) break;
      const int nb = d.q_bits[q];
      const Plan P = s_plan[4 * slot + q];
      const uint32_t idx = plan_index(P, xh & nbit_mask(nb), nb);
      if (idx < P.count && P.depth == static_cast<uint32_t>(nb)) {
        pr[q] = __ldg(&fs.F[4 * slot + q][idx].v);
      } else {  // not a full-domain table: the caller's tables do not match the bundle
        atomicOr(a.status, kStatusBadArgument);
      }
    }
    combine_store(d, xh, pr, a.y, a.bools, i);
  }
}

}  // namespace

namespace {

// One per-element myl7 key (adapter layout, ADD group, 8-byte payload) walked
// from global memory for input x.  ALIGNED: the key starts 8-byte aligned
// (every key of the array is a multiple of 8 bytes long), so each level's
// 33-byte record comes in three 16-byte loads re-aligned by funnel shifts;
// otherwise byte loads.  A header that does not match flags the status and
// yields 0.
template <bool ALIGNED>
__device__ __forceinline__ uint64_t walk_elem_key(const PrgParams& prg, uint32_t lb, const uint8_t* k, int nb,
                                                  uint64_t x, uint32_t party, uint32_t* status) {
  const uint64_t hdr = ALIGNED ? __ldg(reinterpret_cast<const uint64_t*>(k)) : ldb64(k);
  if ((hdr & 0xFF) != static_cast<uint64_t>(nb) || ((hdr >> 8) & 0xFF) != 1 || ((hdr >> 16) & 0xFF) != party ||
      (hdr >> 32) != 8) {
    atomicOr(status, kStatusBadKeyHeader);
    return 0;
  }
  Blk s;
  if (ALIGNED) {
    const uint64_t s0 = __ldg(reinterpret_cast<const uint64_t*>(k) + 1), s1 = __ldg(reinterpret_cast<const uint64_t*>(k) + 2);
    s.w[0] = static_cast<uint32_t>(s0);
    s.w[1] = static_cast<uint32_t>(s0 >> 32);
    s.w[2] = static_cast<uint32_t>(s1);
    s.w[3] = static_cast<uint32_t>(s1 >> 32);
  } else {
    s.w[0] = ldb32(k + 8);
    s.w[1] = ldb32(k + 12);
    s.w[2] = ldb32(k + 16);
    s.w[3] = ldb32(k + 20);
  }
  s.w[3] &= 0x7FFFFFFFu;
  uint32_t t = party;
  uint64_t v = 0;
  const uintptr_t kaddr = reinterpret_cast<uintptr_t>(k);
  for (int lv = 0; lv < nb; lv++) {
    CwLevel cw;
    if (ALIGNED) {
      // the record lies inside the three aligned 16-byte chunks from its
      // address rounded down to 16 (offset <= 15, 15 + 33 <= 48), all inside
      // the 40 + 33 nb byte key
      const uintptr_t A = kaddr + 24u + 33u * static_cast<uint32_t>(lv);
      const uint4* c = reinterpret_cast<const uint4*>(A & ~static_cast<uintptr_t>(15));
      const uint4 c0 = __ldg(c), c1 = __ldg(c + 1), c2 = __ldg(c + 2);
      const uint32_t r = static_cast<uint32_t>(A & 15u);
      const bool hi = r >= 8u;
      const uint32_t rb = r & 7u;
      const uint64_t w0 = (static_cast<uint64_t>(c0.y) << 32) | c0.x, w1 = (static_cast<uint64_t>(c0.w) << 32) | c0.z;
      const uint64_t w2 = (static_cast<uint64_t>(c1.y) << 32) | c1.x, w3 = (static_cast<uint64_t>(c1.w) << 32) | c1.z;
      const uint64_t w4 = (static_cast<uint64_t>(c2.y) << 32) | c2.x, w5 = (static_cast<uint64_t>(c2.w) << 32) | c2.z;
      const uint64_t q0 = hi ? w1 : w0, q1 = hi ? w2 : w1, q2 = hi ? w3 : w2, q3 = hi ? w4 : w3, q4 = hi ? w5 : w4;
      const uint64_t slo = funnel64(q0, q1, rb), shi = funnel64(q1, q2, rb);
      cw.s.w[0] = static_cast<uint32_t>(slo);
      cw.s.w[1] = static_cast<uint32_t>(slo >> 32);
      cw.s.w[2] = static_cast<uint32_t>(shi);
      cw.s.w[3] = static_cast<uint32_t>(shi >> 32);
      cw.v = funnel64(q2, q3, rb);
      cw.t = static_cast<uint32_t>((q4 >> (8u * rb)) & 0xFFu);
    } else {
      const uint8_t* c = k + 24 + 33 * lv;
      cw.s.w[0] = ldb32(c);
      cw.s.w[1] = ldb32(c + 4);
      cw.s.w[2] = ldb32(c + 8);
      cw.s.w[3] = ldb32(c + 12);
      cw.v = ldb64(c + 16);
      cw.t = c[32];
    }
    walk_level<SUFB200_GROUP_ADD>(prg, lb, s, t, v, static_cast<uint32_t>((x >> (nb - 1 - lv)) & 1ull), party, cw);
  }
  const uint32_t onp = 24u + 33u * static_cast<uint32_t>(nb);
  const uint64_t np1 = ALIGNED ? funnel64(__ldg(reinterpret_cast<const uint64_t*>(k) + (onp >> 3)),
                                          __ldg(reinterpret_cast<const uint64_t*>(k) + (onp >> 3) + 1), onp & 7u)
                               : ldb64(k + onp);
  return walk_finish<SUFB200_GROUP_ADD>(s, t, v, party, np1);
}

// Level-major layout of one slot's n per-element keys, in blocks of
// kSoaBlock elements (the last block may be shorter: m elements); per block:
//   cws [nb][m] uint4   the seed correction word of each level
//   seed [m] uint4      the key's seed (bit 127 set: the key's header failed)
//   cwv [nb][m] u64     the low word of each level's value correction
//   np1 [m] u64         the low word of the final correction
//   cwt [nb][m] u8      each level's two t-bit corrections
// Lanes of a warp (consecutive elements) read one level's words as one
// coalesced run, where the adapter layout spreads them over 32 records
// 33 nb + 40 bytes apart; 25 nb + 24 bytes per key.  The blocks keep a
// walk's levels within a few MB (a level of a block is 256 KB of cws), so a
// wave of the grid touches a few hundred pages of a multi-GB key set
// instead of a page per level per array.
constexpr size_t kSoaBlock = 16384;

struct ElemSoa {
  const uint4* cws;
  const uint4* seed;
  const uint64_t* cwv;
  const uint64_t* np1;
  const uint8_t* cwt;
  size_t m;  // elements in this block (the stride between levels)
  size_t j;  // the element's index in its block
};

__host__ __device__ __forceinline__ ElemSoa elem_soa_view(const uint8_t* base, int nb, size_t n, size_t i) {
  const size_t per = 25 * static_cast<size_t>(nb) + 24;
  const size_t b = i / kSoaBlock;
  ElemSoa v;
  v.j = i - b * kSoaBlock;
  v.m = n - b * kSoaBlock < kSoaBlock ? n - b * kSoaBlock : kSoaBlock;
  const uint8_t* blk = base + b * kSoaBlock * per;
  const size_t L = static_cast<size_t>(nb) * v.m;
  v.cws = reinterpret_cast<const uint4*>(blk);
  v.seed = v.cws + L;
  v.cwv = reinterpret_cast<const uint64_t*>(v.seed + v.m);
  v.np1 = v.cwv + L;
  v.cwt = reinterpret_cast<const uint8_t*>(v.np1 + v.m);
  return v;
}

__device__ __forceinline__ uint64_t walk_elem_soa(const PrgParams& prg, uint32_t lb, const uint8_t* base, size_t i,
                                                  size_t n, int nb, uint64_t x, uint32_t party) {
  const ElemSoa K = elem_soa_view(base, nb, n, i);
  const uint4 sd = __ldg(K.seed + K.j);
  if (sd.w & 0x80000000u) return 0;  // its header failed at the rearrangement (status flagged there)
  Blk s;
  s.w[0] = sd.x;
  s.w[1] = sd.y;
  s.w[2] = sd.z;
  s.w[3] = sd.w;
  uint32_t t = party;
  uint64_t v = 0;
  for (int lv = 0; lv < nb; lv++) {
    const size_t j = static_cast<size_t>(lv) * K.m + K.j;
    const uint4 c = __ldg(K.cws + j);
    CwLevel cw;
    cw.s.w[0] = c.x;
    cw.s.w[1] = c.y;
    cw.s.w[2] = c.z;
    cw.s.w[3] = c.w;
    cw.v = __ldg(K.cwv + j);
    cw.t = __ldg(K.cwt + j);
    walk_level<SUFB200_GROUP_ADD>(prg, lb, s, t, v, static_cast<uint32_t>((x >> (nb - 1 - lv)) & 1ull), party, cw);
  }
  return walk_finish<SUFB200_GROUP_ADD>(s, t, v, party, __ldg(K.np1 + K.j));
}

// Adapter-layout keys [n][key_bytes] of one slot -> the level-major layout;
// one thread per (element, level) record (and the seed / final word at
// level 0), writes coalesced across threads.
__global__ void elem_keys_to_soa_kernel(const uint8_t* __restrict__ keys, size_t kb, int nb, uint32_t party, size_t n,
                                        uint8_t* __restrict__ soa, uint32_t* status) {
  const size_t total = static_cast<size_t>(nb) * n;
  const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
  for (size_t g = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; g < total; g += stride) {
    // g runs element-fastest within a block and level: (block, level, j)
    const size_t b = g / (kSoaBlock * static_cast<size_t>(nb));
    const size_t m = n - b * kSoaBlock < kSoaBlock ? n - b * kSoaBlock : kSoaBlock;
    const size_t r = g - b * kSoaBlock * static_cast<size_t>(nb);
    const size_t lv = r / m, j = r - lv * m, i = b * kSoaBlock + j;
    const ElemSoa K = elem_soa_view(soa, nb, n, i);
    const size_t o = lv * K.m + K.j;
    const uint8_t* k = keys + i * kb;
    const uint8_t* c = k + 24 + 33 * lv;
    const_cast<uint4*>(K.cws)[o] = make_uint4(ldb32(c), ldb32(c + 4), ldb32(c + 8), ldb32(c + 12));
    const_cast<uint64_t*>(K.cwv)[o] = ldb64(c + 16);
    const_cast<uint8_t*>(K.cwt)[o] = c[32];
    uint4* seed = const_cast<uint4*>(K.seed) + K.j;
    uint64_t* np1 = const_cast<uint64_t*>(K.np1) + K.j;
    if (lv == 0) {
      const uint64_t hdr = ldb64(k);
      const bool ok = (hdr & 0xFF) == static_cast<uint64_t>(nb) && ((hdr >> 8) & 0xFF) == 1 &&
                      ((hdr >> 16) & 0xFF) == party && (hdr >> 32) == 8;
      if (!ok) atomicOr(status, kStatusBadKeyHeader);
      *seed = make_uint4(ldb32(k + 8), ldb32(k + 12), ldb32(k + 16),
                         (ldb32(k + 20) & 0x7FFFFFFFu) | (ok ? 0u : 0x80000000u));
      *np1 = ldb64(k + 24 + 33 * static_cast<size_t>(nb));
    }
  }
}

// Per-element masks: element i has its own keys (slot q at keys[q] + i *
// key_bytes[q]), its own descriptor words and plan (words[6 i ..]); one
// thread per element walks every slot and folds the element's plan and
// postproc (the per-element path of compiler::lower_truncation_gate,
// include/compiler/truncation_lowering.hpp:91-125, evaluated by one
// composite_eval_batch_backend per element in the reference).
// MODE: 0 adapter-layout keys read bytewise, 1 adapter-layout keys with
// aligned 16-byte loads, 2 level-major keys (keys[q] = the slot's layout).
template <int MODE>
__global__ void __launch_bounds__(kAesThreads, 1)
    trunc_bundle_elem_kernel(const PrgParams prg, const __grid_constant__ TruncElemLaunch a) {
  if (!aes_layout_ok()) {
    if (threadIdx.x == 0) atomicOr(a.status, kStatusSmemLayout);
    pdl_wait();
    return;
  }
  aes_fill_tables(a.t0);
  __syncthreads();
  const uint32_t lb = lane_base();
  const uint32_t party = static_cast<uint32_t>(a.shape.party);
  const int nq = a.shape.nq;
  const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
  for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < a.n; i += stride) {
    const uint64_t xh = a.xhat[i];
    uint64_t pr[4] = {0, 0, 0, 0};
#pragma unroll
    for (int q = 0; q < 4; q++) {
      if (q < nq) {
        const int nb = a.shape.q_bits[q];
        const uint64_t x = nb >= 64 ? xh : (xh & ((1ull << nb) - 1ull));
        pr[q] = MODE == 2 ? walk_elem_soa(prg, lb, a.keys[q], i, a.n, nb, x, party)
                          : walk_elem_key<MODE == 1>(prg, lb, a.keys[q] + i * a.key_bytes[q], nb, x, party,
                                                     a.status);
      }
    }
    const uint64_t* w = a.words + 6 * i;
    sufb200_trunc_desc d = a.shape;
    d.carry_w = w[0];
    d.sign_w = w[1];
    d.haty = w[2];
    d.r_hi = w[3];
    d.m = w[4];
    const uint64_t plan = w[5];
    int32_t idx[5];
    bool ok = true;
#pragma unroll
    for (int j = 0; j < 5; j++) {
      const int32_t v = static_cast<int32_t>((plan >> (4 * j)) & 0xFu);
      idx[j] = v == 0xF ? -1 : v;
      ok = ok && idx[j] < nq;
    }
    d.carry_a = idx[0];
    d.carry_b = idx[1];
    d.sign_a = idx[2];
    d.sign_b = idx[3];
    d.wrap_q = idx[4];
    if (!ok || (d.carry_a >= 0) != (d.carry_b >= 0) || (d.sign_a >= 0) != (d.sign_b >= 0)) {
      atomicOr(a.status, kStatusBadArgument);
      a.y[i] = 0;
      continue;
    }
    combine_store(d, xh, pr, a.y, a.bools, i);
  }
}

}  // namespace

cudaError_t launch_elem_keys_to_soa(const sufb200_ctx_s* ctx, const uint8_t* keys, size_t kb, int nb, int party,
                                    size_t n, uint8_t* soa, cudaStream_t st) {
  const size_t total = static_cast<size_t>(nb) * n;
  const size_t want = (total + 255) / 256, cap = static_cast<size_t>(ctx->sm_count) * 8;
  elem_keys_to_soa_kernel<<<static_cast<int>(want < cap ? (want ? want : 1) : cap), 256, 0, st>>>(
      keys, kb, nb, static_cast<uint32_t>(party), n, soa, ctx->d_status);
  return cudaGetLastError();
}

size_t elem_soa_bytes(int nb, size_t n) { return n * (25 * static_cast<size_t>(nb) + 24); }

cudaError_t launch_trunc_bundle_elem(const sufb200_ctx_s* ctx, const TruncElemLaunch& a, int mode,
                                     cudaStream_t st) {
  const auto kernel = mode == 2 ? trunc_bundle_elem_kernel<2>
                                : (mode == 1 ? trunc_bundle_elem_kernel<1> : trunc_bundle_elem_kernel<0>);
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(ctx->aes_dyn_bytes));
  if (e != cudaSuccess) return e;
  // One block per 512 elements, not a persistent grid: the scheduler deals
  // blocks out in order, so the keys in use at any time stay those of about
  // one wave.  A 148-block grid-stride loop over 4,194,304 elements ran 30 %
  // slower than the same elements in 262,144-element launches (blocks drift
  // apart over 55 strides and the window of keys in flight widens); the
  // table fill a new block pays is about 0.3 % of its walk.
  const size_t want = (a.n + kAesThreads - 1) / kAesThreads;
  const size_t cap = 0x7FFFFFFFu;
  const int grid = static_cast<int>(want < cap ? (want ? want : 1) : cap);
  kernel<<<grid, kAesThreads, ctx->aes_dyn_bytes, st>>>(ctx->prg, a);
  return cudaGetLastError();
}

cudaError_t launch_trunc_bundle(const sufb200_ctx_s* ctx, const TruncLaunch& a, cudaStream_t st) {
  cudaError_t e = cudaFuncSetAttribute(trunc_bundle_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(ctx->aes_dyn_bytes));
  if (e != cudaSuccess) return e;
  const size_t want = (a.n + kAesThreads - 1) / kAesThreads;
  const int grid = static_cast<int>(want < static_cast<size_t>(ctx->sm_count) ? (want ? want : 1) : ctx->sm_count);
  return launch_pdl(trunc_bundle_kernel, grid, kAesThreads, ctx->aes_dyn_bytes, st, ctx->prg, a);
}

cudaError_t launch_trunc_bundle_pair(const sufb200_ctx_s* ctx, const TruncLaunch& a0, const TruncLaunch& a1,
                                     cudaStream_t st) {
  if (a0.n != a1.n || a0.xhat != a1.xhat) return cudaErrorInvalidValue;
  cudaError_t e = cudaFuncSetAttribute(trunc_bundle_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(ctx->aes_dyn_bytes));
  if (e != cudaSuccess) return e;
  if (a0.desc.nq != a1.desc.nq || a0.desc.nq < 0 || a0.desc.nq > 4) return cudaErrorInvalidValue;  // 0: no query
  const int lanes = 2 * (a0.desc.nq <= 1 ? 1 : (a0.desc.nq <= 2 ? 2 : 4));  // a lane pair per query
  const size_t units = 2 * a0.n * static_cast<size_t>(lanes);
  // The tree levels are sequential and each is hundreds of instructions per
  // lane: a small batch is bound by how many warps share an SM's issue slots,
  // so it is spread over as many SMs as it can use (at least 128 threads per
  // CTA, so the table fill stays short).
  const size_t sms = static_cast<size_t>(ctx->sm_count);
  size_t threads = ((units + sms - 1) / sms + 31) / 32 * 32;
  threads = threads < 128 ? 128 : (threads > static_cast<size_t>(kAesThreads) ? kAesThreads : threads);
  const size_t want = (units + threads - 1) / threads;
  const int grid = static_cast<int>(want < sms ? (want ? want : 1) : sms);
  return launch_pdl(trunc_bundle_pair_kernel, grid, static_cast<unsigned>(threads), ctx->aes_dyn_bytes, st, ctx->prg,
                    a0, a1, lanes);
}

cudaError_t launch_trunc_bundle_prefix(const sufb200_ctx_s* ctx, const TruncLaunch& a, const RangeAcc* acc,
                                       uint32_t kmax, FrontierEntry* const F[4], cudaStream_t st) {
  cudaError_t e = cudaFuncSetAttribute(trunc_bundle_prefix_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(ctx->aes_dyn_bytes));
  if (e != cudaSuccess) return e;
  FrontierSet fs{{F[0], F[1], F[2], F[3], nullptr, nullptr, nullptr, nullptr}};
  const size_t want = (a.n + kAesThreads - 1) / kAesThreads;
  const int grid = static_cast<int>(want < static_cast<size_t>(ctx->sm_count) ? (want ? want : 1) : ctx->sm_count);
  return launch_pdl(trunc_bundle_prefix_kernel<1>, grid, kAesThreads, ctx->aes_dyn_bytes, st, ctx->prg, a, a, acc,
                    kmax, fs);
}

cudaError_t launch_trunc_bundle_lookup_pair(const sufb200_ctx_s* ctx, const TruncLaunch& a0, const TruncLaunch& a1,
                                            const RangeAcc* acc, uint32_t kmax, FrontierEntry* const F[8],
                                            cudaStream_t st) {
  if (a0.n != a1.n || a0.xhat != a1.xhat) return cudaErrorInvalidValue;
  FrontierSet fs{{F[0], F[1], F[2], F[3], F[4], F[5], F[6], F[7]}};
  const size_t want = (2 * a0.n + 255) / 256, cap = static_cast<size_t>(ctx->sm_count) * 8;
  const int grid = static_cast<int>(want < cap ? (want ? want : 1) : cap);
  return launch_pdl(trunc_bundle_lookup_pair_kernel, grid, 256u, 0, st, a0, a1, acc, kmax, fs);
}

cudaError_t launch_trunc_bundle_prefix_pair(const sufb200_ctx_s* ctx, const TruncLaunch& a0, const TruncLaunch& a1,
                                            const RangeAcc* acc, uint32_t kmax, FrontierEntry* const F[8],
                                            cudaStream_t st) {
  if (a0.n != a1.n || a0.xhat != a1.xhat) return cudaErrorInvalidValue;
  cudaError_t e = cudaFuncSetAttribute(trunc_bundle_prefix_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(ctx->aes_dyn_bytes));
  if (e != cudaSuccess) return e;
  FrontierSet fs{{F[0], F[1], F[2], F[3], F[4], F[5], F[6], F[7]}};
  const size_t want = (2 * a0.n + kAesThreads - 1) / kAesThreads;
  const int grid = static_cast<int>(want < static_cast<size_t>(ctx->sm_count) ? (want ? want : 1) : ctx->sm_count);
  return launch_pdl(trunc_bundle_prefix_kernel<2>, grid, kAesThreads, ctx->aes_dyn_bytes, st, ctx->prg, a0, a1, acc,
                    kmax, fs);
}

}  // namespace sufb200
