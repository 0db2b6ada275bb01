// prefix.cu -- range, frontier and resume kernels of the shared-prefix
// evaluation of broadcast myl7 DCF keys (see prefix.cuh for the method).
#include "bcast_key.cuh"
#include "kernels.hpp"
#include "prefix.cuh"

namespace sufb200 {

namespace {

__device__ __forceinline__ uint64_t warp_min_u64(uint64_t v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const uint64_t w = __shfl_xor_sync(0xFFFFFFFFu, v, o);
    v = w < v ? w : v;
  }
  return v;
}
__device__ __forceinline__ uint64_t warp_max_u64(uint64_t v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const uint64_t w = __shfl_xor_sync(0xFFFFFFFFu, v, o);
    v = w > v ? w : v;
  }
  return v;
}

// Signed offsets from the pivot xs[0], biased by flipping the sign bit so
// unsigned order is signed order; one atomic pair per warp.
__global__ void range_kernel(const uint64_t* __restrict__ xs, size_t n, RangeAcc* acc) {
  pdl_wait();
  pdl_trigger();
  const uint64_t pivot = xs[0];
  uint64_t mn = ~0ull, mx = 0ull;
  const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
  for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride) {
    const uint64_t b = (xs[i] - pivot) ^ (1ull << 63);
    mn = b < mn ? b : mn;
    mx = b > mx ? b : mx;
  }
  mn = warp_min_u64(mn);
  mx = warp_max_u64(mx);
  if ((threadIdx.x & 31) == 0) {
    atomicMin(&acc->min_b, static_cast<unsigned long long>(mn));
    atomicMax(&acc->max_b, static_cast<unsigned long long>(mx));
  }
  if (blockIdx.x == 0 && threadIdx.x == 0) acc->pivot = pivot;
}

SUFB200_DEV CwLevel load_cw(const BcastKeySmem* ks, int lv) {
  CwLevel cw;
  const uint4 cs = ks->cw_s[lv];
  cw.s.w[0] = cs.x;
  cw.s.w[1] = cs.y;
  cw.s.w[2] = cs.z;
  cw.s.w[3] = cs.w;
  cw.v = ks->cw_v[lv];
  cw.t = ks->cw_t[lv];
  return cw;
}

template <int GROUP>
SUFB200_DEV void emit_entry(FrontierEntry* out, uint64_t slot, bool final_level, const Blk& s, uint32_t t,
                            uint64_t v, uint32_t party, uint64_t np1_lo) {
  FrontierEntry e;
  if (final_level) {
    e.s[0] = e.s[1] = e.s[2] = e.s[3] = 0;
    e.v = walk_finish<GROUP>(s, t, v, party, np1_lo);
    e.t = 0;
  } else {
    e.s[0] = s.w[0];
    e.s[1] = s.w[1];
    e.s[2] = s.w[2];
    e.s[3] = s.w[3];
    e.v = v;
    e.t = t;
  }
  e.pad = 0;
  // two 16-byte stores: one sector per entry instead of a partial write per field
  uint4* o = reinterpret_cast<uint4*>(out + slot);
  o[0] = make_uint4(e.s[0], e.s[1], e.s[2], e.s[3]);
  o[1] = make_uint4(static_cast<uint32_t>(e.v), static_cast<uint32_t>(e.v >> 32), e.t, 0u);
}

// Per-key parameters of a frontier pass, computed once per block.
struct FrontierKey {
  Plan plan;
  FrontierEntry* out;
  uint64_t roots;   // subtree roots (work items) of this key
  int h;            // subtree height
  int final_level;  // D == n: entries are outputs
};

// Staging area at the start of dynamic shared memory, below the AES tables
// (no static shared memory: it would move the table window).
struct FrontierStage {
  uint4 prg_keys[44];  // prg_keys_to_smem's round keys (the lane-pair walk)
  BcastKeySmem key[kFrontierMaxKeys];
  FrontierKey fk[kFrontierMaxKeys];
  uint64_t first_item[kFrontierMaxKeys + 1];
  int order[kFrontierMaxKeys];
};
static_assert(sizeof(FrontierStage) < kTabBase - 4096, "staging must fit below the tables");

// Frontier pass over all keys of a batch in one wave: every key is staged in
// shared memory and the work items (subtree roots, frontier_root in
// prefix.cuh) of all keys form one list, the most expensive keys' items
// first, dealt out round-robin over the blocks so each SM gets a share of
// each kind.
template <int GROUP>
__global__ void __launch_bounds__(kAesThreads, 1) frontier_kernel(const PrgParams prg, const FrontierBatch b) {
  extern __shared__ __align__(16) uint8_t smem[];
  if (!aes_layout_ok()) {
    if (threadIdx.x == 0) atomicOr(b.q[0].status, kStatusSmemLayout);
    pdl_wait();
    return;
  }
  const int nq = b.nq;
  FrontierStage* fs = reinterpret_cast<FrontierStage*>(smem);
  BcastKeySmem* ks = fs->key;
  FrontierKey* fk = fs->fk;
  int* order = fs->order;
  uint64_t* first_item = fs->first_item;
  aes_fill_tables(b.q[0].t0);
  prg_keys_to_smem(prg, fs->prg_keys);
  pdl_wait();  // the plans read the range pass's result
  pdl_trigger();
#pragma unroll
  for (int q = 0; q < kFrontierMaxKeys; q++)
    if (q < nq) stage_bcast_key(&ks[q], b.q[q].key, b.q[q].in_bits, b.q[q].out_bytes);
  if (threadIdx.x == 0) {
    uint64_t cost[kFrontierMaxKeys];
#pragma unroll
    for (int q = 0; q < kFrontierMaxKeys; q++) {
      if (q >= nq) continue;
      RangeAcc r;
      if (b.q[q].full) {
        r.min_b = 0ull;
        r.max_b = ~0ull;
        r.pivot = 0ull;
        r.pad = 0ull;
        if (blockIdx.x == 0) {
          b.q[q].full->min_b = r.min_b;
          b.q[q].full->max_b = r.max_b;
          b.q[q].full->pivot = r.pivot;
        }
      } else {
        r = *b.q[q].acc;
      }
      const Plan p = make_plan(r, b.q[q].in_bits, b.q[q].kmax);
      const int h = expand_height(p);
      fk[q].plan = p;
      fk[q].out = b.q[q].out;
      fk[q].roots = root_count(p, h);
      fk[q].h = h;
      fk[q].final_level = static_cast<int>(p.depth) == b.q[q].in_bits;
      cost[q] = 2ull * static_cast<uint64_t>(static_cast<int>(p.depth) - h) + 4ull * (1ull << h);
      order[q] = q;
    }
    for (int i = 1; i < nq; i++)  // most expensive items first
      for (int k = i; k > 0 && cost[order[k]] > cost[order[k - 1]]; k--) {
        const int t = order[k];
        order[k] = order[k - 1];
        order[k - 1] = t;
      }
    first_item[0] = 0;
    for (int r = 0; r < nq; r++) first_item[r + 1] = first_item[r] + fk[order[r]].roots;
  }
  __syncthreads();
  for (int q = 0; q < nq; q++)
    if (!ks[q].ok) {
      if (threadIdx.x == 0 && blockIdx.x == 0) atomicOr(b.q[0].status, kStatusBadKeyHeader);
      return;
    }
  const uint32_t lb = lane_base();
  const uint64_t total = first_item[nq];
  // The work item `it` of the merged list, walked by one lane, or by a lane
  // pair (frontier_root_pair) when hsel <= 1.
  const auto item = [&](uint64_t it, uint32_t hsel, uint32_t pmask) {
    int r = 0;
    while (r + 1 < nq && it >= first_item[r + 1]) r++;
    const int q = order[r];
    const BcastKeySmem* k = &ks[q];
    const FrontierKey& f = fk[q];
    Blk seed;
    seed.w[0] = k->seed.x;
    seed.w[1] = k->seed.y;
    seed.w[2] = k->seed.z;
    seed.w[3] = k->seed.w;
    const uint32_t party = k->party;
    const uint64_t np1_lo = k->np1_lo;
    const bool final_level = f.final_level != 0;
    FrontierEntry* out = f.out;
    const auto cw_at = [k](int lv) { return load_cw(k, lv); };
    const auto emit = [=](uint64_t slot, const Blk& s, uint32_t t, uint64_t v) {
      emit_entry<GROUP>(out, slot, final_level, s, t, v, party, np1_lo);
    };
    if (hsel <= 1u)
      frontier_root_pair<GROUP>(fs->prg_keys, lb, seed, party, f.plan, f.h, it - first_item[r], cw_at, emit, hsel,
                                pmask);
    else
      frontier_root<GROUP>(prg, lb, seed, party, f.plan, f.h, it - first_item[r], cw_at, emit);
  };
  const uint64_t lanes = static_cast<uint64_t>(gridDim.x) * blockDim.x;
  if (2 * total <= lanes) {
    // Fewer items than lane pairs (small batches): a lane pair per item
    // halves the serial chain of AES blocks.  Items are dealt round-robin
    // over the blocks, pair by pair; the branch is uniform over the grid.
    const uint32_t lane = threadIdx.x & 31u;
    const uint64_t it = static_cast<uint64_t>(threadIdx.x >> 1) * gridDim.x + blockIdx.x;
    if (it < total) item(it, lane & 1u, 3u << (lane & ~1u));
  } else {
    // Enough items to fill every lane: a lane per item, round-robin over
    // the blocks (the AES tables' throughput, not the chain, bounds this).
    for (uint64_t it = static_cast<uint64_t>(threadIdx.x) * gridDim.x + blockIdx.x; it < total; it += lanes)
      item(it, 2u, 0u);
  }
}

template <int GROUP>
__global__ void __launch_bounds__(kAesThreads, 1)
    myl7_eval_bcast_prefix_kernel(const PrgParams prg, const DcfLaunch a, const RangeAcc* acc, uint32_t kmax,
                                  const FrontierEntry* __restrict__ F) {
  extern __shared__ __align__(16) uint8_t smem[];
  if (!aes_layout_ok()) {
    if (threadIdx.x == 0) atomicOr(a.status, kStatusSmemLayout);
    return;
  }
  BcastKeySmem* ks = reinterpret_cast<BcastKeySmem*>(smem);
  stage_bcast_key(ks, a.keys, a.in_bits, a.out_bytes);
  aes_fill_tables(a.t0);
  __syncthreads();
  if (!ks->ok) {
    if (threadIdx.x == 0 && blockIdx.x == 0) atomicOr(a.status, kStatusBadKeyHeader);
    return;
  }
  const uint32_t lb = lane_base();
  const int n = a.in_bits;
  const Plan plan = make_plan(*acc, n, kmax);
  const uint64_t xmask = nbit_mask(n);
  const uint32_t party = ks->party;
  const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
  for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < a.n; i += stride) {
    const uint64_t x = a.xs[i] & xmask;
    const uint32_t idx = plan_index(plan, x, n);
    Blk s;
    uint32_t t;
    uint64_t v;
    int start;
    if (idx < plan.count) {
      const FrontierEntry e = F[idx];
      if (plan.depth == static_cast<uint32_t>(n)) {
        store_out(a.out, i, a.out_bytes, e.v);
        continue;
      }
      s.w[0] = e.s[0];
      s.w[1] = e.s[1];
      s.w[2] = e.s[2];
      s.w[3] = e.s[3];
      t = e.t;
      v = e.v;
      start = static_cast<int>(plan.depth);
    } else {  // outside the measured window: walk from the root
      s.w[0] = ks->seed.x;
      s.w[1] = ks->seed.y;
      s.w[2] = ks->seed.z;
      s.w[3] = ks->seed.w;
      t = party;
      v = 0;
      start = 0;
    }
    for (int lv = start; lv < n; lv++) {
      CwLevel cw;
      const uint4 cs = ks->cw_s[lv];
      cw.s.w[0] = cs.x;
      cw.s.w[1] = cs.y;
      cw.s.w[2] = cs.z;
      cw.s.w[3] = cs.w;
      cw.v = ks->cw_v[lv];
      cw.t = ks->cw_t[lv];
      walk_level<GROUP>(prg, lb, s, t, v, static_cast<uint32_t>((x >> (n - 1 - lv)) & 1ull), party, cw);
    }
    store_out(a.out, i, a.out_bytes, walk_finish<GROUP>(s, t, v, party, ks->np1_lo));
  }
}

int aes_grid(const sufb200_ctx_s* ctx, size_t work) {
  const size_t want = (work + kAesThreads - 1) / kAesThreads;
  return static_cast<int>(want < static_cast<size_t>(ctx->sm_count) ? (want ? want : 1) : ctx->sm_count);
}

template <typename K>
cudaError_t set_smem(K kernel, const sufb200_ctx_s* ctx) {
  return cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              static_cast<int>(ctx->aes_dyn_bytes));
}

}  // namespace

// Frontier entries allowed per key.  One level deeper saves 2 AES blocks per
// element and costs about 6.4 blocks per added entry (subtree expansion), so
// the best depth has about 0.3 N - 0.6 N entries; 5N/8 keeps a window that
// straddles a bucket boundary at that depth.  Capped at 2^23 entries (256 MB).
uint32_t prefix_budget(size_t n) {
  size_t k = n / 8 * 5;
  if (k < 256) k = 256;
  if (k > (1u << 23)) k = 1u << 23;
  return static_cast<uint32_t>(k);
}

cudaError_t launch_range(const sufb200_ctx_s* ctx, const uint64_t* xs, size_t n, RangeAcc* acc, cudaStream_t st) {
  cudaError_t e = cudaMemsetAsync(&acc->min_b, 0xFF, sizeof(uint64_t), st);
  if (e == cudaSuccess) e = cudaMemsetAsync(&acc->max_b, 0, 2 * sizeof(uint64_t), st);
  if (e != cudaSuccess) return e;
  const size_t want = (n + 255) / 256;
  const size_t cap = static_cast<size_t>(ctx->sm_count) * 4;
  return launch_pdl(range_kernel, static_cast<int>(want < cap ? (want ? want : 1) : cap), 256, 0, st, xs, n, acc);
}

// A range covering every value: make_plan then gives a query its full domain
// whenever 2^n entries fit the budget.  Used instead of the range pass when
// every query of a batch is that narrow (the f-bit carry queries of GapARS
// bundles at shared-prefix sizes): the pass could only shrink tables that are
// already small, and the outputs are the same words either way.
cudaError_t set_full_range(RangeAcc* acc, cudaStream_t st) {
  cudaError_t e = cudaMemsetAsync(&acc->min_b, 0, sizeof(uint64_t), st);
  if (e == cudaSuccess) e = cudaMemsetAsync(&acc->max_b, 0xFF, sizeof(uint64_t), st);
  if (e == cudaSuccess) e = cudaMemsetAsync(&acc->pivot, 0, sizeof(uint64_t), st);
  return e;
}

cudaError_t launch_frontier(const sufb200_ctx_s* ctx, int group, const FrontierBatch& b, cudaStream_t st,
                            int max_grid) {
  if (b.nq < 1 || b.nq > kFrontierMaxKeys) return cudaErrorInvalidValue;
  size_t work = 0;
  for (int q = 0; q < b.nq; q++) work += b.q[q].kmax;
  int grid = aes_grid(ctx, 2 * work);  // up to two lanes per work item
  if (max_grid > 0 && grid > max_grid) grid = max_grid;
  cudaError_t e;
  if (group == SUFB200_GROUP_ADD) {
    if ((e = set_smem(frontier_kernel<SUFB200_GROUP_ADD>, ctx)) != cudaSuccess) return e;
    return launch_pdl(frontier_kernel<SUFB200_GROUP_ADD>, grid, kAesThreads, ctx->aes_dyn_bytes, st, ctx->prg, b);
  }
  if ((e = set_smem(frontier_kernel<SUFB200_GROUP_XOR>, ctx)) != cudaSuccess) return e;
  return launch_pdl(frontier_kernel<SUFB200_GROUP_XOR>, grid, kAesThreads, ctx->aes_dyn_bytes, st, ctx->prg, b);
}

cudaError_t launch_myl7_bcast_prefix(const sufb200_ctx_s* ctx, int group, const DcfLaunch& a, const RangeAcc* acc,
                                     uint32_t kmax, const FrontierEntry* F, cudaStream_t st) {
  cudaError_t e;
  if (group == SUFB200_GROUP_ADD) {
    if ((e = set_smem(myl7_eval_bcast_prefix_kernel<SUFB200_GROUP_ADD>, ctx)) != cudaSuccess) return e;
    myl7_eval_bcast_prefix_kernel<SUFB200_GROUP_ADD>
        <<<aes_grid(ctx, a.n), kAesThreads, ctx->aes_dyn_bytes, st>>>(ctx->prg, a, acc, kmax, F);
  } else {
    if ((e = set_smem(myl7_eval_bcast_prefix_kernel<SUFB200_GROUP_XOR>, ctx)) != cudaSuccess) return e;
    myl7_eval_bcast_prefix_kernel<SUFB200_GROUP_XOR>
        <<<aes_grid(ctx, a.n), kAesThreads, ctx->aes_dyn_bytes, st>>>(ctx->prg, a, acc, kmax, F);
  }
  return cudaGetLastError();
}

}  // namespace sufb200
