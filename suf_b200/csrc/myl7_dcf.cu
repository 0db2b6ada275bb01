// myl7_dcf.cu -- batched myl7 DCF evaluation (PRG tree walk) for sm_100a.
//
// Replaces, for myl7-format keys, the per-element loop of
// Myl7FssBackend::eval_dcf (include/proto/myl7_fss_backend.hpp:215-256) and
// the staged entry points PfssGpuStagedEval::eval_dcf_many_u64_device[_broadcast]
// (include/proto/backend_gpu.hpp:17-38).  One thread walks one element; the
// AES-128-MMO PRG runs on the shared-memory T-table engine (aes_smem.cuh) with
// the four fixed PRG keys as constant-bank kernel parameters.
#include "bcast_key.cuh"
#include "kernels.hpp"

namespace sufb200 {

namespace {

template <int GROUP>
__global__ void __launch_bounds__(kAesThreads, 1)
    myl7_eval_bcast_kernel(const PrgParams prg, const DcfLaunch a) {
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
  const uint64_t xmask = n >= 64 ? ~0ull : ((1ull << n) - 1ull);
  const uint32_t party = ks->party;
  const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
  for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < a.n; i += stride) {
    const uint64_t x = a.xs[i] & xmask;
    Blk s;
    s.w[0] = ks->seed.x;
    s.w[1] = ks->seed.y;
    s.w[2] = ks->seed.z;
    s.w[3] = ks->seed.w;
    uint32_t t = party;
    uint64_t v = 0;
    for (int lv = 0; lv < n; lv++) {
      CwLevel cw;
      const uint4 cs = ks->cw_s[lv];
      cw.s.w[0] = cs.x;
      cw.s.w[1] = cs.y;
      cw.s.w[2] = cs.z;
      cw.s.w[3] = cs.w;
      cw.v = ks->cw_v[lv];
      cw.t = ks->cw_t[lv];
      const uint32_t xb = static_cast<uint32_t>((x >> (n - 1 - lv)) & 1ull);
      walk_level<GROUP>(prg, lb, s, t, v, xb, party, cw);
    }
    store_out(a.out, i, a.out_bytes, walk_finish<GROUP>(s, t, v, party, ks->np1_lo));
  }
}

// Per-element keys, aligned layout (in_bits % 8 == 0 and an 8-byte aligned
// key array): each level's 33-byte record is read with five 8-byte loads and
// re-aligned with funnel shifts (the record offset mod 8 is i mod 8, uniform
// across the warp).
template <int GROUP>
__global__ void __launch_bounds__(kAesThreads, 1)
    myl7_eval_elem_aligned_kernel(const PrgParams prg, const DcfLaunch a) {
  if (!aes_layout_ok()) {
    if (threadIdx.x == 0) atomicOr(a.status, kStatusSmemLayout);
    return;
  }
  aes_fill_tables(a.t0);
  __syncthreads();
  const uint32_t lb = lane_base();
  const int n = a.in_bits;
  const uint64_t xmask = n >= 64 ? ~0ull : ((1ull << n) - 1ull);
  const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
  const size_t kw = a.key_bytes >> 3;
  for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < a.n; i += stride) {
    const uint64_t* k = reinterpret_cast<const uint64_t*>(a.keys) + i * kw;
    const uint64_t hdr = __ldg(k);
    if (!key_header_ok(hdr, n, a.out_bytes)) {
      atomicOr(a.status, kStatusBadKeyHeader);
      store_out(a.out, i, a.out_bytes, 0);
      continue;
    }
    const uint32_t party = static_cast<uint32_t>((hdr >> 16) & 0xFF);
    const uint64_t x = a.xs[i] & xmask;
    const uint64_t s0 = __ldg(k + 1), s1 = __ldg(k + 2);
    Blk s;
    s.w[0] = static_cast<uint32_t>(s0);
    s.w[1] = static_cast<uint32_t>(s0 >> 32);
    s.w[2] = static_cast<uint32_t>(s1);
    s.w[3] = static_cast<uint32_t>(s1 >> 32) & 0x7FFFFFFFu;
    uint32_t t = party;
    uint64_t v = 0;
    const uintptr_t kaddr = reinterpret_cast<uintptr_t>(k);
    for (int lv = 0; lv < n; lv++) {
      // The 33-byte record of level lv lies inside the three aligned 16-byte
      // chunks from its address rounded down to 16 (offset <= 15, 15 + 33 <=
      // 48; the last chunk ends at or before byte 38 + 33n of the 40 + 33n
      // byte key): three 16-byte loads instead of five 8-byte ones.
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
      CwLevel cw;
      const uint64_t slo = funnel64(q0, q1, rb), shi = funnel64(q1, q2, rb);
      cw.s.w[0] = static_cast<uint32_t>(slo);
      cw.s.w[1] = static_cast<uint32_t>(slo >> 32);
      cw.s.w[2] = static_cast<uint32_t>(shi);
      cw.s.w[3] = static_cast<uint32_t>(shi >> 32);
      cw.v = funnel64(q2, q3, rb);
      cw.t = static_cast<uint32_t>((q4 >> (8u * rb)) & 0xFFu);
      const uint32_t xb = static_cast<uint32_t>((x >> (n - 1 - lv)) & 1ull);
      walk_level<GROUP>(prg, lb, s, t, v, xb, party, cw);
    }
    const uint32_t onp = 24u + 33u * static_cast<uint32_t>(n);
    const uint64_t np1 = funnel64(__ldg(k + (onp >> 3)), __ldg(k + (onp >> 3) + 1), onp & 7u);
    store_out(a.out, i, a.out_bytes, walk_finish<GROUP>(s, t, v, party, np1));
  }
}

// Per-element keys, any layout: byte loads (in_bits not a multiple of 8).
template <int GROUP>
__global__ void __launch_bounds__(kAesThreads, 1)
    myl7_eval_elem_bytes_kernel(const PrgParams prg, const DcfLaunch a) {
  if (!aes_layout_ok()) {
    if (threadIdx.x == 0) atomicOr(a.status, kStatusSmemLayout);
    return;
  }
  aes_fill_tables(a.t0);
  __syncthreads();
  const uint32_t lb = lane_base();
  const int n = a.in_bits;
  const uint64_t xmask = n >= 64 ? ~0ull : ((1ull << n) - 1ull);
  const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
  for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < a.n; i += stride) {
    const uint8_t* k = a.keys + i * a.key_bytes;
    const uint64_t hdr = ld_u64_bytes(k);
    if (!key_header_ok(hdr, n, a.out_bytes)) {
      atomicOr(a.status, kStatusBadKeyHeader);
      store_out(a.out, i, a.out_bytes, 0);
      continue;
    }
    const uint32_t party = static_cast<uint32_t>((hdr >> 16) & 0xFF);
    const uint64_t x = a.xs[i] & xmask;
    Blk s;
    s.w[0] = ld_u32_bytes(k + 8);
    s.w[1] = ld_u32_bytes(k + 12);
    s.w[2] = ld_u32_bytes(k + 16);
    s.w[3] = ld_u32_bytes(k + 20) & 0x7FFFFFFFu;
    uint32_t t = party;
    uint64_t v = 0;
    for (int lv = 0; lv < n; lv++) {
      const uint8_t* c = k + 24 + 33 * lv;
      CwLevel cw;
      cw.s.w[0] = ld_u32_bytes(c);
      cw.s.w[1] = ld_u32_bytes(c + 4);
      cw.s.w[2] = ld_u32_bytes(c + 8);
      cw.s.w[3] = ld_u32_bytes(c + 12);
      cw.v = ld_u64_bytes(c + 16);
      cw.t = c[32];
      const uint32_t xb = static_cast<uint32_t>((x >> (n - 1 - lv)) & 1ull);
      walk_level<GROUP>(prg, lb, s, t, v, xb, party, cw);
    }
    store_out(a.out, i, a.out_bytes, walk_finish<GROUP>(s, t, v, party, ld_u64_bytes(k + 24 + 33 * n)));
  }
}

template <typename K>
cudaError_t launch_aes_kernel(K kernel, const sufb200_ctx_s* ctx, const PrgParams& prg, const DcfLaunch& a,
                              cudaStream_t st) {
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(ctx->aes_dyn_bytes));
  if (e != cudaSuccess) return e;
  const size_t want = (a.n + kAesThreads - 1) / kAesThreads;
  const int grid = static_cast<int>(want < static_cast<size_t>(ctx->sm_count) ? (want ? want : 1) : ctx->sm_count);
  kernel<<<grid, kAesThreads, ctx->aes_dyn_bytes, st>>>(prg, a);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_myl7_eval(const sufb200_ctx_s* ctx, int group, const DcfLaunch& a, int broadcast,
                             cudaStream_t st) {
  const PrgParams& prg = ctx->prg;
  const bool aligned = (a.in_bits % 8 == 0) && (a.key_bytes % 8 == 0) &&
                       (reinterpret_cast<uintptr_t>(a.keys) % 8 == 0);
  if (group == SUFB200_GROUP_ADD) {
    if (broadcast) return launch_aes_kernel(myl7_eval_bcast_kernel<SUFB200_GROUP_ADD>, ctx, prg, a, st);
    if (aligned) return launch_aes_kernel(myl7_eval_elem_aligned_kernel<SUFB200_GROUP_ADD>, ctx, prg, a, st);
    return launch_aes_kernel(myl7_eval_elem_bytes_kernel<SUFB200_GROUP_ADD>, ctx, prg, a, st);
  }
  if (broadcast) return launch_aes_kernel(myl7_eval_bcast_kernel<SUFB200_GROUP_XOR>, ctx, prg, a, st);
  if (aligned) return launch_aes_kernel(myl7_eval_elem_aligned_kernel<SUFB200_GROUP_XOR>, ctx, prg, a, st);
  return launch_aes_kernel(myl7_eval_elem_bytes_kernel<SUFB200_GROUP_XOR>, ctx, prg, a, st);
}

}  // namespace sufb200
