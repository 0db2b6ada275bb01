// ref_formats.cu -- the reference GPU backend's own key formats on sm_100a.
//
// Threshold "DCF" (DcfKeyHeader), packed multi-threshold compare
// (PackedCmpKeyHeader) and interval LUT (IntervalKeyHeader) blobs of
// cuda/pfss_backend_gpu.cu:69-94, evaluated with the counter layout of the
// reference kernels (cuda/pfss_kernels.cu:240-719): one AES-128 block masks
// two output words, ctr = nonce ^ (idx << 32) ^ (...), block = [ctr LE][0^8].
// The AES runs on the shared-memory T-table engine; broadcast keys keep
// their round keys, thresholds / cutpoints and payload rows in shared memory.
#include "aes_smem.cuh"
#include "kernels.hpp"

namespace sufb200 {

namespace {

constexpr uint32_t kStageBytes = 48u * 1024u;  // broadcast-key staging budget

__device__ __forceinline__ uint64_t mask_bits(int bits) {
  return bits <= 0 ? 0ull : (bits >= 64 ? ~0ull : ((1ull << bits) - 1ull));
}

__device__ __forceinline__ Blk ctr_block(uint64_t ctr) {
  Blk b;
  b.w[0] = static_cast<uint32_t>(ctr);
  b.w[1] = static_cast<uint32_t>(ctr >> 32);
  b.w[2] = 0;
  b.w[3] = 0;
  return b;
}

// ---- threshold DCF (no AES; HBM-bound) ------------------------------------
__device__ __forceinline__ uint32_t ldb32(const uint8_t* p) {
  return static_cast<uint32_t>(p[0]) | (static_cast<uint32_t>(p[1]) << 8) | (static_cast<uint32_t>(p[2]) << 16) |
         (static_cast<uint32_t>(p[3]) << 24);
}

__global__ void thr_dcf_kernel(const RefFmtLaunch a) {
  const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
  const uint64_t m = mask_bits(a.in_bits);
  for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < a.n; i += stride) {
    const uint8_t* k = a.keys + (a.broadcast ? 0 : i * a.key_bytes);
    const uint32_t h = ldb32(k);
    const uint64_t alpha = static_cast<uint64_t>(ldb32(k + 4)) | (static_cast<uint64_t>(ldb32(k + 8)) << 32);
    if ((h & 0xFFFFu) != static_cast<uint32_t>(a.in_bits) || (h >> 16) != static_cast<uint32_t>(a.out_bytes)) {
      atomicOr(a.status, kStatusBadKeyHeader);
    }
    const bool lt = (a.xs[i] & m) < (alpha & m);
    uint8_t* o = reinterpret_cast<uint8_t*>(a.out) + i * static_cast<size_t>(a.out_bytes);
    if (a.out_bytes == 8) {
      uint64_t p = 0;
      if (lt)
        p = static_cast<uint64_t>(ldb32(k + 12)) | (static_cast<uint64_t>(ldb32(k + 16)) << 32);
      reinterpret_cast<uint64_t*>(a.out)[i] = p;
    } else {
      for (int b = 0; b < a.out_bytes; b++) o[b] = lt ? k[12 + b] : 0;
    }
  }
}

// ---- packed compare ----------------------------------------------------------
__device__ __forceinline__ uint64_t packed_word(int wi, uint64_t x, int num_thr, bool sorted, int pos,
                                                const uint64_t* thr, uint64_t m) {
  const int base = wi * 64;
  const int lim = base + 64 < num_thr ? base + 64 : num_thr;
  uint64_t word = 0;
  if (sorted) {
    const int len = lim - base;
    if (len > 0) {
      const uint64_t bits = len >= 64 ? ~0ull : ((1ull << len) - 1ull);
      if (pos <= base) word = bits;
      else if (pos >= lim) word = 0;
      else word = bits ^ ((1ull << (pos - base)) - 1ull);
    }
  } else {
    for (int b = base; b < lim; b++)
      if (x < (thr[b] & m)) word |= 1ull << (b - base);
  }
  return word;
}

__global__ void __launch_bounds__(kAesThreads, 1) packed_lt_kernel(const RefFmtLaunch a) {
  extern __shared__ __align__(16) uint8_t smem[];
  if (!aes_layout_ok()) {
    if (threadIdx.x == 0) atomicOr(a.status, kStatusSmemLayout);
    return;
  }
  uint32_t* s_rk = reinterpret_cast<uint32_t*>(smem);                 // 176 B
  uint64_t* s_thr = reinterpret_cast<uint64_t*>(smem + 256);          // staged thresholds
  bool thr_in_smem = false;
  if (a.broadcast) {
    const int num_thr = static_cast<int>(reinterpret_cast<const uint16_t*>(a.keys)[1]);
    thr_in_smem = 8u * static_cast<uint32_t>(num_thr) <= kStageBytes;
    for (int i = threadIdx.x; i < 44; i += blockDim.x) s_rk[i] = reinterpret_cast<const uint32_t*>(a.keys + 32)[i];
    if (thr_in_smem)
      for (int i = threadIdx.x; i < num_thr; i += blockDim.x)
        s_thr[i] = reinterpret_cast<const uint64_t*>(a.keys + 208)[i];
  }
  aes_fill_tables(a.t0);
  __syncthreads();
  const uint32_t lb = lane_base();
  const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
  for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < a.n; i += stride) {
    const uint8_t* k = a.keys + (a.broadcast ? 0 : i * a.key_bytes);
    const uint64_t h = *reinterpret_cast<const uint64_t*>(k);
    const int in_bits = static_cast<int>(h & 0xFFFF);
    const int num_thr = static_cast<int>((h >> 16) & 0xFFFF);
    const uint32_t party = static_cast<uint32_t>((h >> 32) & 0xFF);
    const bool sorted = ((h >> 40) & 1ull) != 0;
    const int words = (num_thr + 63) / 64;
    uint64_t* out = reinterpret_cast<uint64_t*>(a.out) + i * static_cast<size_t>(a.out_words);
    if (words != a.out_words || in_bits != a.in_bits || 208u + 8u * static_cast<size_t>(num_thr) > a.key_bytes) {
      atomicOr(a.status, kStatusBadKeyHeader);
      for (int w = 0; w < a.out_words; w++) out[w] = 0;
      continue;
    }
    const uint64_t nonce = *reinterpret_cast<const uint64_t*>(k + 8);
    const uint32_t* rk = a.broadcast ? s_rk : reinterpret_cast<const uint32_t*>(k + 32);
    const uint64_t* thr = (a.broadcast && thr_in_smem) ? s_thr : reinterpret_cast<const uint64_t*>(k + 208);
    const uint64_t m = mask_bits(in_bits);
    const uint64_t x = a.xs[i] & m;
    int pos = 0;
    if (sorted) {
      int lo = 0, hi = num_thr;
      while (lo < hi) {
        const int mid = (lo + hi) >> 1;
        if (x < (thr[mid] & m)) hi = mid; else lo = mid + 1;
      }
      pos = lo;
    }
    const uint64_t idx = a.idx_base + i;
    for (int w = 0; w < words; w += 2) {
      const uint64_t w0 = packed_word(w, x, num_thr, sorted, pos, thr, m);
      const uint64_t w1 = (w + 1 < words) ? packed_word(w + 1, x, num_thr, sorted, pos, thr, m) : 0ull;
      const Blk ks = aes_encrypt_smem_rk(ctr_block(nonce ^ (idx << 32) ^ static_cast<uint64_t>(w / 2)), lb, rk);
      const uint64_t ks0 = (static_cast<uint64_t>(ks.w[1]) << 32) | ks.w[0];
      const uint64_t ks1 = (static_cast<uint64_t>(ks.w[3]) << 32) | ks.w[2];
      out[w] = party == 0 ? ks0 : (w0 ^ ks0);
      if (w + 1 < words) out[w + 1] = party == 0 ? ks1 : (w1 ^ ks1);
    }
  }
}

// ---- interval LUT --------------------------------------------------------
// Round keys and (when it fits `cap` bytes) the cut/payload table of a
// broadcast key into shared memory; true when the table was staged.
__device__ __forceinline__ bool stage_lut_key(const RefFmtLaunch& a, uint32_t* s_rk, uint64_t* s_tab, uint32_t cap) {
  const uint64_t h = *reinterpret_cast<const uint64_t*>(a.keys);
  const uint32_t ivs = static_cast<uint32_t>(h >> 32), ow = static_cast<uint32_t>((h >> 16) & 0xFFFF);
  const size_t words = static_cast<size_t>(ivs) + 1 + static_cast<size_t>(ivs) * ow;
  const bool tab_in_smem = 216u + 8u * words <= a.key_bytes && 8u * words <= cap;
  for (int i = threadIdx.x; i < 44; i += blockDim.x) s_rk[i] = reinterpret_cast<const uint32_t*>(a.keys + 40)[i];
  if (tab_in_smem)
    for (size_t i = threadIdx.x; i < words; i += blockDim.x) s_tab[i] = reinterpret_cast<const uint64_t*>(a.keys + 216)[i];
  return tab_in_smem;
}

// Element i of one interval-LUT launch: interval by binary search over the
// cuts, then the row's share words, one AES-CTR block per two words.
__device__ __forceinline__ void lut_element(const RefFmtLaunch& a, size_t i, const uint32_t* s_rk, const uint64_t* s_tab,
                                            bool tab_in_smem, uint32_t lb) {
  const uint8_t* k = a.keys + (a.broadcast ? 0 : i * a.key_bytes);
  const uint64_t h = *reinterpret_cast<const uint64_t*>(k);
  const int in_bits = static_cast<int>(h & 0xFFFF);
  const int ow = static_cast<int>((h >> 16) & 0xFFFF);
  const uint32_t ivs = static_cast<uint32_t>(h >> 32);
  const uint32_t party = k[8];
  uint64_t* out = reinterpret_cast<uint64_t*>(a.out) + i * static_cast<size_t>(a.out_words);
  const size_t need = 216u + 8u * (static_cast<size_t>(ivs) + 1 + static_cast<size_t>(ivs) * ow);
  if (ow != a.out_words || ivs == 0 || need > a.key_bytes) {
    atomicOr(a.status, kStatusBadKeyHeader);
    for (int w = 0; w < a.out_words; w++) out[w] = 0;
    return;
  }
  const uint64_t nonce = *reinterpret_cast<const uint64_t*>(k + 16);
  const uint32_t* rk = a.broadcast ? s_rk : reinterpret_cast<const uint32_t*>(k + 40);
  const uint64_t* cuts = (a.broadcast && tab_in_smem) ? s_tab : reinterpret_cast<const uint64_t*>(k + 216);
  const uint64_t* pay = cuts + ivs + 1;
  const uint64_t m = mask_bits(in_bits);
  const uint64_t x = a.xs[i] & m;
  int iv = static_cast<int>(ivs) - 1;
  if (ivs > 1) {
    int lo = 0, hi = static_cast<int>(ivs);
    while (lo < hi) {
      const int mid = (lo + hi) >> 1;
      if ((cuts[mid] & m) <= x) lo = mid + 1; else hi = mid;
    }
    iv = lo - 1;
    if (iv < 0) iv = 0;
    if (iv >= static_cast<int>(ivs)) iv = static_cast<int>(ivs) - 1;
  }
  const uint64_t idx = a.idx_base + i;
  const uint64_t* row = pay + static_cast<size_t>(iv) * ow;
  for (int w = 0; w < ow; w += 2) {
    const uint64_t ctr = nonce ^ (idx << 32) ^ (static_cast<uint64_t>(iv) * static_cast<uint64_t>(ow) + w);
    const Blk ks = aes_encrypt_smem_rk(ctr_block(ctr), lb, rk);
    const uint64_t ks0 = (static_cast<uint64_t>(ks.w[1]) << 32) | ks.w[0];
    const uint64_t ks1 = (static_cast<uint64_t>(ks.w[3]) << 32) | ks.w[2];
    out[w] = party == 0 ? ks0 : (row[w] - ks0);
    if (w + 1 < ow) out[w + 1] = party == 0 ? ks1 : (row[w + 1] - ks1);
  }
}

__global__ void __launch_bounds__(kAesThreads, 1) interval_lut_kernel(const RefFmtLaunch a) {
  extern __shared__ __align__(16) uint8_t smem[];
  if (!aes_layout_ok()) {
    if (threadIdx.x == 0) atomicOr(a.status, kStatusSmemLayout);
    return;
  }
  uint32_t* s_rk = reinterpret_cast<uint32_t*>(smem);
  uint64_t* s_tab = reinterpret_cast<uint64_t*>(smem + 256);  // cuts then payload
  const bool tab_in_smem = a.broadcast ? stage_lut_key(a, s_rk, s_tab, kStageBytes) : false;
  aes_fill_tables(a.t0);
  __syncthreads();
  const uint32_t lb = lane_base();
  const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
  for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < a.n; i += stride)
    lut_element(a, i, s_rk, s_tab, tab_in_smem, lb);
}

// True in every thread of the block when two staged broadcast LUT keys
// produce one keystream: the same header, nonce, round keys and cut table.
// The reference's dealer gives both parties of a LUT key one AES key and
// nonce -- party 0's share words are the keystream itself, party 1's the
// payload minus it (cuda/pfss_kernels.cu:545-719) -- so with both parties'
// keys on one GPU each counter block is encrypted once for both outputs.
__device__ __forceinline__ bool lut_keys_share_keystream(const RefFmtLaunch& a0, const RefFmtLaunch& a1,
                                                         const uint32_t* rk0, const uint32_t* rk1) {
  const uint64_t h0 = *reinterpret_cast<const uint64_t*>(a0.keys);
  const uint64_t h1 = *reinterpret_cast<const uint64_t*>(a1.keys);
  const uint32_t ivs = static_cast<uint32_t>(h0 >> 32), ow = static_cast<uint32_t>((h0 >> 16) & 0xFFFF);
  const size_t need = 216u + 8u * (static_cast<size_t>(ivs) + 1 + static_cast<size_t>(ivs) * ow);
  bool same = h0 == h1 && ivs != 0 && ow == static_cast<uint32_t>(a0.out_words) && need <= a0.key_bytes &&
              need <= a1.key_bytes && a0.idx_base == a1.idx_base &&
              *reinterpret_cast<const uint64_t*>(a0.keys + 16) == *reinterpret_cast<const uint64_t*>(a1.keys + 16);
  if (same) {
    for (int i = threadIdx.x; i < 44; i += blockDim.x) same = same && rk0[i] == rk1[i];
    const uint64_t* c0 = reinterpret_cast<const uint64_t*>(a0.keys + 216);
    const uint64_t* c1 = reinterpret_cast<const uint64_t*>(a1.keys + 216);
    for (uint32_t i = threadIdx.x; i <= ivs; i += blockDim.x) same = same && c0[i] == c1[i];
  }
  return __syncthreads_and(same) != 0;
}

// Element i of both parties' gates when their keys share the keystream:
// one interval search and one AES block per two words, two share rows.
__device__ __forceinline__ void lut_element_shared(const RefFmtLaunch& a0, const RefFmtLaunch& a1, size_t i,
                                                   const uint32_t* s_rk, const uint64_t* cuts, const uint64_t* pay0,
                                                   const uint64_t* pay1, uint32_t lb) {
  const uint64_t h = *reinterpret_cast<const uint64_t*>(a0.keys);
  const int in_bits = static_cast<int>(h & 0xFFFF);
  const int ow = static_cast<int>((h >> 16) & 0xFFFF);
  const uint32_t ivs = static_cast<uint32_t>(h >> 32);
  const uint32_t party0 = a0.keys[8], party1 = a1.keys[8];
  const uint64_t nonce = *reinterpret_cast<const uint64_t*>(a0.keys + 16);
  const uint64_t m = mask_bits(in_bits);
  const uint64_t x = a0.xs[i] & m;
  int iv = static_cast<int>(ivs) - 1;
  if (ivs > 1) {
    int lo = 0, hi = static_cast<int>(ivs);
    while (lo < hi) {
      const int mid = (lo + hi) >> 1;
      if ((cuts[mid] & m) <= x) lo = mid + 1; else hi = mid;
    }
    iv = lo - 1;
    if (iv < 0) iv = 0;
    if (iv >= static_cast<int>(ivs)) iv = static_cast<int>(ivs) - 1;
  }
  const uint64_t idx = a0.idx_base + i;
  const uint64_t* row0 = pay0 + static_cast<size_t>(iv) * ow;
  const uint64_t* row1 = pay1 + static_cast<size_t>(iv) * ow;
  uint64_t* out0 = reinterpret_cast<uint64_t*>(a0.out) + i * static_cast<size_t>(ow);
  uint64_t* out1 = reinterpret_cast<uint64_t*>(a1.out) + i * static_cast<size_t>(ow);
  for (int w = 0; w < ow; w += 2) {
    const uint64_t ctr = nonce ^ (idx << 32) ^ (static_cast<uint64_t>(iv) * static_cast<uint64_t>(ow) + w);
    const Blk ks = aes_encrypt_smem_rk(ctr_block(ctr), lb, s_rk);
    const uint64_t ks0 = (static_cast<uint64_t>(ks.w[1]) << 32) | ks.w[0];
    const uint64_t ks1 = (static_cast<uint64_t>(ks.w[3]) << 32) | ks.w[2];
    out0[w] = party0 == 0 ? ks0 : (row0[w] - ks0);
    out1[w] = party1 == 0 ? ks0 : (row1[w] - ks0);
    if (w + 1 < ow) {
      out0[w + 1] = party0 == 0 ? ks1 : (row0[w + 1] - ks1);
      out1[w + 1] = party1 == 0 ? ks1 : (row1[w + 1] - ks1);
    }
  }
}

// Both parties' broadcast-key gates over one x^ in one launch (elements
// [0, n) party 0's key, [n, 2n) party 1's), spread over as many SMs as the
// batch can use: the softmax and LayerNorm blocks' gates on 128 to 99,072
// values, where one launch per party was latency-bound.  When the two keys
// share their keystream the launch covers n items, each serving both
// parties.
__global__ void __launch_bounds__(kAesThreads, 1) interval_lut_pair_kernel(const RefFmtLaunch a0, const RefFmtLaunch a1) {
  extern __shared__ __align__(16) uint8_t smem[];
  if (!aes_layout_ok()) {
    if (threadIdx.x == 0) atomicOr(a0.status, kStatusSmemLayout);
    pdl_wait();
    return;
  }
  uint32_t* s_rk0 = reinterpret_cast<uint32_t*>(smem);
  uint32_t* s_rk1 = reinterpret_cast<uint32_t*>(smem + 256);
  uint64_t* s_tab0 = reinterpret_cast<uint64_t*>(smem + 512);
  uint64_t* s_tab1 = reinterpret_cast<uint64_t*>(smem + 512 + kStageBytes / 2);
  aes_fill_tables(a0.t0);
  pdl_wait();
  pdl_trigger();
  const bool tab0 = stage_lut_key(a0, s_rk0, s_tab0, kStageBytes / 2);
  const bool tab1 = stage_lut_key(a1, s_rk1, s_tab1, kStageBytes / 2);
  __syncthreads();
  const uint32_t lb = lane_base();
  const size_t n = a0.n;
  const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
  if (lut_keys_share_keystream(a0, a1, s_rk0, s_rk1)) {
    const uint32_t ivs = static_cast<uint32_t>(*reinterpret_cast<const uint64_t*>(a0.keys) >> 32);
    const uint64_t* cuts = tab0 ? s_tab0 : reinterpret_cast<const uint64_t*>(a0.keys + 216);
    const uint64_t* pay1 = (tab1 ? s_tab1 : reinterpret_cast<const uint64_t*>(a1.keys + 216)) + ivs + 1;
    // 32-item warp chunks dealt round-robin over the blocks, so the n items
    // spread over every block the launch sized for 2n.
    const size_t first = ((static_cast<size_t>(threadIdx.x >> 5) * gridDim.x + blockIdx.x) << 5) + (threadIdx.x & 31u);
    for (size_t i = first; i < n; i += stride)
      lut_element_shared(a0, a1, i, s_rk0, cuts, cuts + ivs + 1, pay1, lb);
    return;
  }
  for (size_t g = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; g < 2 * n; g += stride) {
    if (g < n)
      lut_element(a0, g, s_rk0, s_tab0, tab0, lb);
    else
      lut_element(a1, g - n, s_rk1, s_tab1, tab1, lb);
  }
}

// One party's gate of a coefficient launch, laid out once per block in
// shared memory.
struct CoeffSide {
  const uint64_t* cuts;  // the interval starts (shared memory when they fit)
  const uint64_t* pay;   // ivs rows of ow words
  uint64_t* out;
  uint64_t nonce, m, ring_mask, idx_base;
  uint64_t r_out[kCoeffMaxOut];
  uint32_t party, ivs;
  int ow, r, d1, ok;
};

// Stage side q's round keys (s_rk, 44 words), its cut/payload table when it
// fits `cap` bytes (s_tab) and its scalars (S, by thread 0).
__device__ __forceinline__ void stage_coeff_side(const RefFmtLaunch& a, const CoeffLutParams& p, uint32_t* s_rk,
                                                 uint64_t* s_tab, uint32_t cap, CoeffSide* S) {
  const uint8_t* key = p.key_in_params ? p.key : a.keys;
  const uint64_t h = *reinterpret_cast<const uint64_t*>(key);
  const int in_bits = static_cast<int>(h & 0xFFFF);
  const int ow = static_cast<int>((h >> 16) & 0xFFFF);
  const uint32_t ivs = static_cast<uint32_t>(h >> 32);
  const size_t words = static_cast<size_t>(ivs) + 1 + static_cast<size_t>(ivs) * ow;
  const bool tab_in_smem = 8u * words <= cap;
  for (int i = threadIdx.x; i < 44; i += blockDim.x) s_rk[i] = reinterpret_cast<const uint32_t*>(key + 40)[i];
  if (tab_in_smem)
    for (size_t i = threadIdx.x; i < words; i += blockDim.x) s_tab[i] = reinterpret_cast<const uint64_t*>(key + 216)[i];
  if (threadIdx.x == 0) {
    const uint64_t* cuts = tab_in_smem ? s_tab : reinterpret_cast<const uint64_t*>(key + 216);
    S->cuts = cuts;
    S->pay = cuts + ivs + 1;
    S->out = reinterpret_cast<uint64_t*>(a.out);
    S->nonce = *reinterpret_cast<const uint64_t*>(key + 16);
    S->m = mask_bits(in_bits);
    S->ring_mask = p.ring_mask;
    S->idx_base = a.idx_base;
    for (int j = 0; j < kCoeffMaxOut; j++) S->r_out[j] = p.r_out[j];
    S->party = key[8];
    S->ivs = ivs;
    S->ow = ow;
    S->r = p.r;
    S->d1 = p.degree + 1;
    S->ok = ow == p.r * (p.degree + 1) && ivs != 0 && 216u + 8u * words <= a.key_bytes;
  }
}

// The interval of x^: the last cut <= x (the first interval below cut 0),
// by a search whose steps depend only on the cut count (the same trip count
// and no branches in every lane; a select per step).
__device__ __forceinline__ int coeff_interval(const CoeffSide& S, uint64_t xh) {
  const uint64_t x = xh & S.m;
  int base = 0, len = static_cast<int>(S.ivs);
  while (len > 1) {
    const int half = len >> 1;
    base = (S.cuts[base + half] & S.m) <= x ? base + half : base;
    len -= half;
  }
  const int ub = base + ((S.cuts[base] & S.m) <= x ? 1 : 0);  // cuts <= x
  return ub - 1 < 0 ? 0 : (ub - 1 >= static_cast<int>(S.ivs) ? static_cast<int>(S.ivs) - 1 : ub - 1);
}

// True in every thread of the block when the two staged sides produce one
// keystream (same round keys, nonce, counter base, cuts and row shape; see
// lut_keys_share_keystream for why the reference's dealt pairs do).
__device__ __forceinline__ bool coeff_sides_share_keystream(const CoeffSide& S0, const CoeffSide& S1,
                                                            const uint32_t* rk0, const uint32_t* rk1) {
  bool same = S0.ok && S1.ok && S0.nonce == S1.nonce && S0.idx_base == S1.idx_base && S0.m == S1.m &&
              S0.ivs == S1.ivs && S0.ow == S1.ow && S0.r == S1.r && S0.d1 == S1.d1;
  if (same) {
    for (int i = threadIdx.x; i < 44; i += blockDim.x) same = same && rk0[i] == rk1[i];
    for (uint32_t i = threadIdx.x; i < S0.ivs; i += blockDim.x) same = same && S0.cuts[i] == S1.cuts[i];
  }
  return __syncthreads_and(same) != 0;
}

// Keystream word w (< 4) of an element from its CTR blocks k0 (words 0, 1)
// and k1 (words 2, 3).
__device__ __forceinline__ uint64_t ks_word(const Blk& k0, const Blk& k1, int w) {
  const uint32_t lo = w == 0 ? k0.w[0] : (w == 1 ? k0.w[2] : (w == 2 ? k1.w[0] : k1.w[2]));
  const uint32_t hi = w == 0 ? k0.w[1] : (w == 1 ? k0.w[3] : (w == 2 ? k1.w[1] : k1.w[3]));
  return (static_cast<uint64_t>(hi) << 32) | lo;
}

// One element's two share rows from its keystream blocks k0 (words 0, 1)
// and k1 (words 2, 3): the polynomial over x^ of each party's share words.
__device__ __forceinline__ void coeff_emit_shared(const CoeffSide& S0, const CoeffSide& S1, size_t i, int iv,
                                                  uint64_t xh, const Blk& k0, const Blk& k1) {
  const int r = S0.r, d1 = S0.d1, ow = S0.ow;
  const uint32_t party0 = S0.party, party1 = S1.party;
  const uint64_t* row0 = S0.pay + static_cast<size_t>(iv) * ow;
  const uint64_t* row1 = S1.pay + static_cast<size_t>(iv) * ow;
  uint64_t* out0 = S0.out + i * static_cast<size_t>(r);
  uint64_t* out1 = S1.out + i * static_cast<size_t>(r);
  if (r == 4 && d1 == 1 &&
      ((reinterpret_cast<uintptr_t>(S0.out) | reinterpret_cast<uintptr_t>(S1.out)) & 15u) == 0) {
    // four degree-0 words: two 16-byte stores a party (32-byte rows from a 16-byte aligned base)
    uint64_t o0[4], o1[4];
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const uint64_t ksw = ks_word(k0, k1, j);
      o0[j] = ((party0 == 0 ? ksw : (row0[j] - ksw)) + S0.r_out[j]) & S0.ring_mask;
      o1[j] = ((party1 == 0 ? ksw : (row1[j] - ksw)) + S1.r_out[j]) & S1.ring_mask;
    }
    reinterpret_cast<ulonglong2*>(out0)[0] = make_ulonglong2(o0[0], o0[1]);
    reinterpret_cast<ulonglong2*>(out0)[1] = make_ulonglong2(o0[2], o0[3]);
    reinterpret_cast<ulonglong2*>(out1)[0] = make_ulonglong2(o1[0], o1[1]);
    reinterpret_cast<ulonglong2*>(out1)[1] = make_ulonglong2(o1[2], o1[3]);
    return;
  }
  int w = 0;
  for (int j = 0; j < r; j++) {
    uint64_t acc0 = 0, acc1 = 0, pw = 1;
    for (int k = 0; k < d1; k++, w++) {
      const uint64_t ksw = ks_word(k0, k1, w);
      acc0 += (party0 == 0 ? ksw : (row0[w] - ksw)) * pw;
      acc1 += (party1 == 0 ? ksw : (row1[w] - ksw)) * pw;
      pw *= xh;
    }
    out0[j] = (acc0 + S0.r_out[j]) & S0.ring_mask;
    out1[j] = (acc1 + S1.r_out[j]) & S1.ring_mask;
  }
}

// Both parties' gates when their keys share the keystream: item i is
// element i of both -- one interval search, one AES block per two words of
// the row, two polynomial rows over the party's share words.  Rows of one
// or two words (one CTR block) take two elements per iteration (i and
// i + step, two chains in flight, round keys read from shared memory);
// rows of three or four words one element with both blocks interleaved
// (round keys in registers, fully unrolled: that measured faster for the
// SiLU gate's four-word rows than two elements of four rolled chains).
__device__ __forceinline__ void coeff_shared_items(const CoeffSide& S0, const CoeffSide& S1, const uint32_t* s_rk,
                                                   const uint64_t* xs, size_t n, size_t first, size_t step,
                                                   uint64_t xh_next, uint32_t lb) {
  const int r = S0.r, d1 = S0.d1, ow = S0.ow;
  const uint32_t party0 = S0.party, party1 = S1.party;
  if (ow <= 2) {
    const uint4* rk4 = reinterpret_cast<const uint4*>(s_rk);
    uint64_t xa_next = xh_next, xb_next = first + step < n ? __ldg(xs + first + step) : 0ull;
    for (size_t i = first; i < n; i += 2 * step) {
      const size_t i2 = i + step;
      const uint64_t xa = xa_next, xb = xb_next;
      xa_next = i + 2 * step < n ? __ldg(xs + i + 2 * step) : 0ull;
      xb_next = i + 3 * step < n ? __ldg(xs + i + 3 * step) : 0ull;
      const int iva = coeff_interval(S0, xa), ivb = coeff_interval(S0, xb);
      Blk k[2] = {ctr_block((S0.nonce ^ ((S0.idx_base + i) << 32)) ^ (static_cast<uint64_t>(iva) * ow)),
                  ctr_block((S0.nonce ^ ((S0.idx_base + i2) << 32)) ^ (static_cast<uint64_t>(ivb) * ow))};
      aes_encrypt_n_sk<2>(k, lb, rk4);
      coeff_emit_shared(S0, S1, i, iva, xa, k[0], k[0]);
      if (i2 < n) coeff_emit_shared(S0, S1, i2, ivb, xb, k[1], k[1]);
    }
    return;
  }
  if (ow <= 4) {
    const uint4* rk4 = reinterpret_cast<const uint4*>(s_rk);
    for (size_t i = first; i < n; i += step) {
      const uint64_t xh = xh_next;
      xh_next = i + step < n ? __ldg(xs + i + step) : 0ull;
      const int iv = coeff_interval(S0, xh);
      const uint64_t base = S0.nonce ^ ((S0.idx_base + i) << 32), w0 = static_cast<uint64_t>(iv) * ow;
      Blk k[2] = {ctr_block(base ^ w0), ctr_block(base ^ (w0 + 2))};
      aes_encrypt_n_sk<2>(k, lb, rk4);
      coeff_emit_shared(S0, S1, i, iv, xh, k[0], k[1]);
    }
    return;
  }
  for (size_t i = first; i < n; i += step) {
    const uint64_t xh = xh_next;
    const size_t in = i + step;
    xh_next = in < n ? __ldg(xs + in) : 0ull;
    const int iv = coeff_interval(S0, xh);
    const uint64_t base = S0.nonce ^ ((S0.idx_base + i) << 32);
    const uint64_t w0 = static_cast<uint64_t>(iv) * static_cast<uint64_t>(ow);
    const uint64_t* row0 = S0.pay + static_cast<size_t>(iv) * ow;
    const uint64_t* row1 = S1.pay + static_cast<size_t>(iv) * ow;
    uint64_t* out0 = S0.out + i * static_cast<size_t>(r);
    uint64_t* out1 = S1.out + i * static_cast<size_t>(r);
    uint64_t ks0 = 0, ks1 = 0;
    int w = 0;
    for (int j = 0; j < r; j++) {
      uint64_t acc0 = 0, acc1 = 0, pw = 1;
      for (int k = 0; k < d1; k++, w++) {
        if ((w & 1) == 0) {
          const Blk ks = aes_encrypt_smem_rk(ctr_block(base ^ (w0 + w)), lb, s_rk);
          ks0 = (static_cast<uint64_t>(ks.w[1]) << 32) | ks.w[0];
          ks1 = (static_cast<uint64_t>(ks.w[3]) << 32) | ks.w[2];
        }
        const uint64_t ksw = (w & 1) ? ks1 : ks0;
        acc0 += (party0 == 0 ? ksw : (row0[w] - ksw)) * pw;
        acc1 += (party1 == 0 ? ksw : (row1[w] - ksw)) * pw;
        pw *= xh;
      }
      out0[j] = (acc0 + S0.r_out[j]) & S0.ring_mask;
      out1[j] = (acc1 + S1.r_out[j]) & S1.ring_mask;
    }
  }
}

// Elements of NP gates over one x^ (NP = 2: both parties; items [0, n) are
// party 0's, [n, 2n) party 1's, or, when the two keys share the keystream,
// item i is element i of both).  Warps take 32-item chunks dealt
// round-robin over the blocks (chunk = warp-in-block * grid + block), so the
// last partial wave spreads over every SM while each warp's x^ loads stay
// coalesced, and each lane loads its next item's x^ before working on the
// current one.
template <int NP>
__device__ __forceinline__ void coeff_lut_body(const RefFmtLaunch& a0, const CoeffLutParams& p0,
                                               const RefFmtLaunch& a1, const CoeffLutParams& p1) {
  extern __shared__ __align__(16) uint8_t smem[];
  if (!aes_layout_ok()) {
    if (threadIdx.x == 0) atomicOr(a0.status, kStatusSmemLayout);
    pdl_wait();
    return;
  }
  const size_t n = a0.n, total = NP * n;
  const uint64_t* xs = a0.xs;
  const uint32_t lane = threadIdx.x & 31u;
  const size_t step = static_cast<size_t>(gridDim.x) * (blockDim.x >> 5) * 32;
  const size_t first = ((static_cast<size_t>(threadIdx.x >> 5) * gridDim.x + blockIdx.x) << 5) + lane;
  aes_fill_tables(a0.t0);
  pdl_wait();  // x^ may come from the previous kernel
  pdl_trigger();
  uint64_t xh_next = first < total ? __ldg(xs + (first < n ? first : first - n)) : 0ull;
  uint32_t* s_rk = reinterpret_cast<uint32_t*>(smem);                 // [NP][44]
  CoeffSide* s_side = reinterpret_cast<CoeffSide*>(smem + 512);       // [NP]
  uint64_t* s_tab = reinterpret_cast<uint64_t*>(smem + 1024);         // [NP][kStageBytes / NP]
  stage_coeff_side(a0, p0, s_rk, s_tab, kStageBytes / NP, &s_side[0]);
  if (NP == 2) stage_coeff_side(a1, p1, s_rk + 44, s_tab + kStageBytes / 16, kStageBytes / 2, &s_side[1]);
  __syncthreads();
  if (threadIdx.x == 0 && blockIdx.x == 0)
    for (int q = 0; q < NP; q++)
      if (!s_side[q].ok) atomicOr(a0.status, kStatusBadKeyHeader);
  const uint32_t lb = lane_base();
  if (NP == 2 && coeff_sides_share_keystream(s_side[0], s_side[1], s_rk, s_rk + 44)) {
    coeff_shared_items(s_side[0], s_side[1], s_rk, xs, n, first, step, xh_next, lb);
    return;
  }
  uint32_t rk[44];
  int cur = -1;
  for (size_t g = first; g < total; g += step) {
    const uint64_t xh = xh_next;
    const size_t gn = g + step;
    xh_next = gn < total ? __ldg(xs + (gn < n ? gn : gn - n)) : 0ull;
    const int q = (NP == 2 && g >= n) ? 1 : 0;
    const size_t i = q ? g - n : g;
    const CoeffSide& S = s_side[q];
    const int r = S.r;
    uint64_t* out = S.out + i * static_cast<size_t>(r);
    if (!S.ok) {
      for (int j = 0; j < r; j++) out[j] = 0;
      continue;
    }
    const int iv = coeff_interval(S, xh);
    const uint64_t base = S.nonce ^ ((S.idx_base + i) << 32);
    const uint64_t w0 = static_cast<uint64_t>(iv) * static_cast<uint64_t>(S.ow);
    const uint64_t* row = S.pay + static_cast<size_t>(iv) * S.ow;
    const uint32_t party = S.party;
    const int d1 = S.d1;
    if (S.ow <= 4) {
      // Rows of at most four words (configs[2]'s SiLU gate: r = 4, degree 0):
      // both CTR blocks of an element at once (one for rows of at most two
      // words), round keys in registers.
      if (q != cur) {
#pragma unroll
        for (int k = 0; k < 44; k++) rk[k] = s_rk[44 * q + k];
        cur = q;
      }
      Blk k0, k1;
      if (S.ow <= 2)
        k0 = k1 = aes_encrypt1_rk(ctr_block(base ^ w0), lb, rk);
      else
        aes_encrypt2_rk(ctr_block(base ^ w0), ctr_block(base ^ (w0 + 2)), lb, rk, k0, k1);
      int w = 0;
      for (int j = 0; j < r; j++) {
        uint64_t acc = 0, pw = 1;
        for (int k = 0; k < d1; k++, w++) {
          const uint64_t ksw = ks_word(k0, k1, w);
          const uint64_t c = party == 0 ? ksw : (row[w] - ksw);
          acc += c * pw;
          pw *= xh;
        }
        out[j] = (acc + S.r_out[j]) & S.ring_mask;
      }
      continue;
    }
    uint64_t ks0 = 0, ks1 = 0;
    int w = 0;
    for (int j = 0; j < r; j++) {
      uint64_t acc = 0, pw = 1;
      for (int k = 0; k < d1; k++, w++) {
        if ((w & 1) == 0) {
          const Blk ks = aes_encrypt_smem_rk(ctr_block(base ^ (w0 + w)), lb, s_rk + 44 * q);
          ks0 = (static_cast<uint64_t>(ks.w[1]) << 32) | ks.w[0];
          ks1 = (static_cast<uint64_t>(ks.w[3]) << 32) | ks.w[2];
        }
        const uint64_t ksw = (w & 1) ? ks1 : ks0;
        const uint64_t c = party == 0 ? ksw : (row[w] - ksw);
        acc += c * pw;
        pw *= xh;
      }
      out[j] = (acc + S.r_out[j]) & S.ring_mask;
    }
  }
}

// ---- coefficient LUT + polynomial over x^ (composite eval, ell = 0) ------
// Restates the two beaver-free branches of composite_eval_batch_backend for a
// gate whose coefficient words come from one broadcast interval LUT:
//   degree 0 (out_words = r): haty[j] = lut[j] + r_out[j]
//     (interval-LUT fast path, include/gates/composite_fss.hpp:1253-1384);
//   degree d > 0: haty[j] = sum_k lut[j*(d+1)+k] * x^^k + r_out[j]
//     (Horner-only path over the public x^, composite_fss.hpp:2066-2130, with
//     the coefficients the compiler shifted to the x^ domain).
// The LUT share words are the reference kernel's (vector_lut_kernel_keyed,
// cuda/pfss_kernels.cu:545-719: one AES block per two words, counter
// nonce ^ (idx << 32) ^ (iv * out_words + w)).  Ring arithmetic mod 2^64,
// reduced to ring_bits at the end (2^ring_bits divides 2^64).
__global__ void __launch_bounds__(kAesThreads, 1)
    coeff_lut_kernel(const RefFmtLaunch a, const __grid_constant__ CoeffLutParams p) {
  coeff_lut_body<1>(a, p, a, p);
}

// Both parties' gates over one x^ in one launch (the parties' halves of one
// GPU's work: one table fill and one launch for the pair).
__global__ void __launch_bounds__(kAesThreads, 1)
    coeff_lut_pair_kernel(const RefFmtLaunch a0, const __grid_constant__ CoeffLutParams p0, const RefFmtLaunch a1,
                          const __grid_constant__ CoeffLutParams p1) {
  coeff_lut_body<2>(a0, p0, a1, p1);
}

int grid_for(const sufb200_ctx_s* ctx, size_t n, int threads, int per_sm) {
  const size_t want = (n + threads - 1) / threads;
  const size_t cap = static_cast<size_t>(ctx->sm_count) * per_sm;
  return static_cast<int>(want < cap ? (want ? want : 1) : cap);
}

}  // namespace

cudaError_t launch_thr_dcf(const sufb200_ctx_s* ctx, const RefFmtLaunch& a, cudaStream_t st) {
  thr_dcf_kernel<<<grid_for(ctx, a.n, 256, 8), 256, 0, st>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_packed_lt(const sufb200_ctx_s* ctx, const RefFmtLaunch& a, cudaStream_t st) {
  cudaError_t e = cudaFuncSetAttribute(packed_lt_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(ctx->aes_dyn_bytes));
  if (e != cudaSuccess) return e;
  packed_lt_kernel<<<grid_for(ctx, a.n, kAesThreads, 1), kAesThreads, ctx->aes_dyn_bytes, st>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_interval_lut(const sufb200_ctx_s* ctx, const RefFmtLaunch& a, cudaStream_t st) {
  cudaError_t e = cudaFuncSetAttribute(interval_lut_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(ctx->aes_dyn_bytes));
  if (e != cudaSuccess) return e;
  interval_lut_kernel<<<grid_for(ctx, a.n, kAesThreads, 1), kAesThreads, ctx->aes_dyn_bytes, st>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_interval_lut_pair(const sufb200_ctx_s* ctx, const RefFmtLaunch& a0, const RefFmtLaunch& a1,
                                     cudaStream_t st) {
  if (!a0.broadcast || !a1.broadcast || a0.n != a1.n || a0.xs != a1.xs || a0.out_words != a1.out_words)
    return cudaErrorInvalidValue;
  cudaError_t e = cudaFuncSetAttribute(interval_lut_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(ctx->aes_dyn_bytes));
  if (e != cudaSuccess) return e;
  const size_t units = 2 * a0.n, sms = static_cast<size_t>(ctx->sm_count);
  size_t threads = ((units + sms - 1) / sms + 31) / 32 * 32;  // as many SMs as the batch can use
  threads = threads < 128 ? 128 : (threads > static_cast<size_t>(kAesThreads) ? kAesThreads : threads);
  const size_t want = (units + threads - 1) / threads;
  const int grid = static_cast<int>(want < sms ? (want ? want : 1) : sms);
  return launch_pdl(interval_lut_pair_kernel, grid, static_cast<unsigned>(threads), ctx->aes_dyn_bytes, st, a0, a1);
}

int interval_lut_pair_eval(const sufb200_ctx_s* ctx, const uint8_t* key0, size_t key_bytes0, const uint8_t* key1,
                           size_t key_bytes1, const uint64_t* xs, size_t n, int out_words, uint64_t* out0,
                           uint64_t* out1, cudaStream_t st) {
  if (n == 0) return SUFB200_OK;
  if (out_words < 1) return record_error(SUFB200_ERR_INVALID, "out_words must be >= 1");
  for (size_t kb : {key_bytes0, key_bytes1})
    if (kb < 216 + 24 || kb % 8) return record_error(SUFB200_ERR_KEY, "interval key_bytes too small or not 8k");
  const void* ptrs[5] = {key0, key1, xs, out0, out1};
  for (const void* q : ptrs)
    if (!q || reinterpret_cast<uintptr_t>(q) % 8) return record_error(SUFB200_ERR_INVALID, "null or misaligned pointer");
  const RefFmtLaunch a0{key0, key_bytes0, 1, xs, n, 0, out0, 0, out_words, 0, ctx->d_t0, ctx->d_status};
  const RefFmtLaunch a1{key1, key_bytes1, 1, xs, n, 0, out1, 0, out_words, 0, ctx->d_t0, ctx->d_status};
  const cudaError_t e = launch_interval_lut_pair(ctx, a0, a1, st);
  return e == cudaSuccess ? SUFB200_OK
                          : record_error(SUFB200_ERR_CUDA, std::string("interval LUT pair launch: ") + cudaGetErrorString(e));
}

cudaError_t launch_coeff_lut(const sufb200_ctx_s* ctx, const RefFmtLaunch& a, const CoeffLutParams& p,
                             cudaStream_t st) {
  cudaError_t e = cudaFuncSetAttribute(coeff_lut_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(ctx->aes_dyn_bytes));
  if (e != cudaSuccess) return e;
  return launch_pdl(coeff_lut_kernel, grid_for(ctx, a.n, kAesThreads, 1), kAesThreads, ctx->aes_dyn_bytes, st, a, p);
}

cudaError_t launch_coeff_lut_pair(const sufb200_ctx_s* ctx, const RefFmtLaunch& a0, const CoeffLutParams& p0,
                                  const RefFmtLaunch& a1, const CoeffLutParams& p1, cudaStream_t st) {
  if (a0.n != a1.n || a0.xs != a1.xs) return cudaErrorInvalidValue;
  cudaError_t e = cudaFuncSetAttribute(coeff_lut_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(ctx->aes_dyn_bytes));
  if (e != cudaSuccess) return e;
  return launch_pdl(coeff_lut_pair_kernel, grid_for(ctx, 2 * a0.n, kAesThreads, 1), kAesThreads, ctx->aes_dyn_bytes,
                    st, a0, p0, a1, p1);
}

}  // namespace sufb200
