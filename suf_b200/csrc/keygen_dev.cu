// keygen_dev.cu -- myl7 DCF key generation on the GPU, one thread per key pair.
//
// Restates dcf_gen (third_party/myl7_fss/src/dcf.c:42-142) in the adapter
// layout of Myl7FssBackend::gen_dcf (include/proto/myl7_fss_backend.hpp:
// 131-213), step for step as the host dealer (keygen.cpp::myl7_dcf_gen_chunk)
// does: per level both parties' seeds are expanded into all four MMO blocks
// (AES-128 under the PRG's K_0..K_3, each XORed with the seed), the losing
// child's seeds and values become the correction word, and the kept child
// continues.  Values are full 128-bit group elements (u128_le: add mod
// 2^127; bytes: XOR).  Party seeds come from the caller, so the keys are
// byte-identical to the host dealer's and the reference's for the same seeds.
#include "aes_smem.cuh"
#include "kernels.hpp"

namespace sufb200 {

namespace {

using u128 = unsigned __int128;
// 384 threads: a key pair's walk holds both parties' four expanded children
// (eight 128-bit values) next to the AES state, which needs more than the 128
// registers a 512-thread block allows.
constexpr int kGenThreads = 384;
constexpr u128 kM127 = (static_cast<u128>(1) << 127) - 1;

__device__ __forceinline__ u128 blk128(const Blk& b) {
  return (static_cast<u128>((static_cast<uint64_t>(b.w[3]) << 32) | b.w[2]) << 64) |
         ((static_cast<uint64_t>(b.w[1]) << 32) | b.w[0]);
}
__device__ __forceinline__ Blk to_blk(u128 v) {
  Blk b;
  b.w[0] = static_cast<uint32_t>(v);
  b.w[1] = static_cast<uint32_t>(v >> 32);
  b.w[2] = static_cast<uint32_t>(v >> 64);
  b.w[3] = static_cast<uint32_t>(v >> 96);
  return b;
}

template <int GROUP>
__device__ __forceinline__ u128 gplus(u128 a, u128 b) {
  return GROUP == SUFB200_GROUP_ADD ? ((a + b) & kM127) : (a ^ b);
}
template <int GROUP>
__device__ __forceinline__ u128 gneg(u128 a) {
  return GROUP == SUFB200_GROUP_ADD ? ((static_cast<u128>(0) - a) & kM127) : a;
}

// Both MMO blocks of one child, in full: A = AES_{K_{2x}}(s) ^ s and
// B = AES_{K_{2x+1}}(s) ^ s, with x chosen by xm (0 or all ones).
__device__ __forceinline__ void prg_child_full(const PrgParams& P, uint32_t lb, const Blk& s, uint32_t xm, Blk& A,
                                               Blk& B) {
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
  A.w[0] = aes_last_col<0>(a, lb, SUFB200_PRG_KEY(P, 0, 10, 0, xm)) ^ s.w[0];
  A.w[1] = aes_last_col<1>(a, lb, SUFB200_PRG_KEY(P, 0, 10, 1, xm)) ^ s.w[1];
  A.w[2] = aes_last_col<2>(a, lb, SUFB200_PRG_KEY(P, 0, 10, 2, xm)) ^ s.w[2];
  A.w[3] = aes_last_col<3>(a, lb, SUFB200_PRG_KEY(P, 0, 10, 3, xm)) ^ s.w[3];
  B.w[0] = aes_last_col<0>(b, lb, SUFB200_PRG_KEY(P, 1, 10, 0, xm)) ^ s.w[0];
  B.w[1] = aes_last_col<1>(b, lb, SUFB200_PRG_KEY(P, 1, 10, 1, xm)) ^ s.w[1];
  B.w[2] = aes_last_col<2>(b, lb, SUFB200_PRG_KEY(P, 1, 10, 2, xm)) ^ s.w[2];
  B.w[3] = aes_last_col<3>(b, lb, SUFB200_PRG_KEY(P, 1, 10, 3, xm)) ^ s.w[3];
}

// Little-endian byte stream into an 8-byte-aligned key, written one aligned
// 64-bit word at a time.
struct KeyWriter {
  uint64_t* dst;
  uint64_t buf;
  int nb;  // bytes pending in buf (0..7)
  __device__ __forceinline__ void u64(uint64_t v) {
    buf |= nb ? (v << (8 * nb)) : v;
    *dst++ = buf;
    buf = nb ? (v >> (64 - 8 * nb)) : 0ull;
  }
  __device__ __forceinline__ void byte(uint32_t v) {
    buf |= static_cast<uint64_t>(v & 0xFFu) << (8 * nb);
    if (++nb == 8) {
      *dst++ = buf;
      buf = 0;
      nb = 0;
    }
  }
  __device__ __forceinline__ void v128(u128 v) {
    u64(static_cast<uint64_t>(v));
    u64(static_cast<uint64_t>(v >> 64));
  }
};

template <int GROUP>
__global__ void __launch_bounds__(kGenThreads, 1) myl7_gen_kernel(const PrgParams prg, const GenLaunch g) {
  if (!aes_layout_ok()) {
    if (threadIdx.x == 0) atomicOr(g.status, kStatusSmemLayout);
    return;
  }
  aes_fill_tables(g.t0);
  __syncthreads();
  const uint32_t lb = lane_base();
  const int n = g.in_bits;
  const uint64_t amask = n >= 64 ? ~0ull : ((1ull << n) - 1ull);
  const u128 beta = (static_cast<u128>(g.beta_hi) << 64 | g.beta_lo) & kM127;
  const uint64_t hdr0 = static_cast<uint64_t>(n) | (1ull << 8) | (static_cast<uint64_t>(g.payload_len) << 32);
  const size_t kw = g.key_bytes / 8;
  const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
  for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < g.n; i += stride) {
    const uint64_t alpha = g.alphas[i] & amask;
    const uint4 q0 = reinterpret_cast<const uint4*>(g.seeds0)[i];
    const uint4 q1 = reinterpret_cast<const uint4*>(g.seeds1)[i];
    KeyWriter w0{reinterpret_cast<uint64_t*>(g.keys0) + i * kw, 0ull, 0};
    KeyWriter w1{reinterpret_cast<uint64_t*>(g.keys1) + i * kw, 0ull, 0};
    w0.u64(hdr0);
    w1.u64(hdr0 | (1ull << 16));  // party byte
    w0.u64((static_cast<uint64_t>(q0.y) << 32) | q0.x);
    w0.u64((static_cast<uint64_t>(q0.w) << 32) | q0.z);
    w1.u64((static_cast<uint64_t>(q1.y) << 32) | q1.x);
    w1.u64((static_cast<uint64_t>(q1.w) << 32) | q1.z);
    Blk s0{{q0.x, q0.y, q0.z, q0.w & 0x7FFFFFFFu}}, s1{{q1.x, q1.y, q1.z, q1.w & 0x7FFFFFFFu}};
    uint32_t t0 = 0, t1 = 1;
    u128 v = 0;
    for (int lv = 0; lv < n; lv++) {
      // Child x of a seed is expanded with keys K_{2x}, K_{2x+1} (constant
      // key selections, so the key words stay constant-bank operands); the
      // kept child is x = alpha's bit, the other one loses.
      const uint32_t a = static_cast<uint32_t>((alpha >> (n - 1 - lv)) & 1ull);
      Blk A, B;
      prg_child_full(prg, lb, s0, 0u, A, B);
      const uint32_t t0l = A.w[3] >> 31;
      const u128 s0l = blk128(A) & kM127, v0l = blk128(B) & kM127;
      prg_child_full(prg, lb, s0, ~0u, A, B);
      const uint32_t t0r = A.w[3] >> 31;
      const u128 s0r = blk128(A) & kM127, v0r = blk128(B) & kM127;
      const u128 s0_lose = a ? s0l : s0r, s0_keep = a ? s0r : s0l;
      const u128 v0_lose = a ? v0l : v0r, v0_keep = a ? v0r : v0l;
      prg_child_full(prg, lb, s1, 0u, A, B);
      const uint32_t t1l = A.w[3] >> 31;
      const u128 s1l = blk128(A) & kM127, v1l = blk128(B) & kM127;
      prg_child_full(prg, lb, s1, ~0u, A, B);
      const uint32_t t1r = A.w[3] >> 31;
      const u128 s1r = blk128(A) & kM127, v1r = blk128(B) & kM127;
      const u128 s1_lose = a ? s1l : s1r, s1_keep = a ? s1r : s1l;
      const u128 v1_lose = a ? v1l : v1r, v1_keep = a ? v1r : v1l;
      const u128 s_cw = s0_lose ^ s1_lose;
      u128 v_cw = gplus<GROUP>(gplus<GROUP>(v1_lose, gneg<GROUP>(v0_lose)), gneg<GROUP>(v));
      if (t1) v_cw = gneg<GROUP>(v_cw);
      if (a) v_cw = gplus<GROUP>(v_cw, t1 ? gneg<GROUP>(beta) : beta);
      v = gplus<GROUP>(gplus<GROUP>(gplus<GROUP>(v, gneg<GROUP>(v1_keep)), v0_keep), t1 ? gneg<GROUP>(v_cw) : v_cw);
      const uint32_t tl_cw = t0l ^ t1l ^ a ^ 1u, tr_cw = t0r ^ t1r ^ a;
      const uint32_t tbyte = (tl_cw << 1) | tr_cw;
      w0.v128(s_cw);
      w0.v128(v_cw);
      w0.byte(tbyte);
      w1.v128(s_cw);
      w1.v128(v_cw);
      w1.byte(tbyte);
      const uint32_t tk = a ? tr_cw : tl_cw;
      const uint32_t t0k = a ? t0r : t0l, t1k = a ? t1r : t1l;
      s0 = to_blk(s0_keep ^ (t0 ? s_cw : static_cast<u128>(0)));
      s1 = to_blk(s1_keep ^ (t1 ? s_cw : static_cast<u128>(0)));
      t0 = t0k ^ (t0 & tk);
      t1 = t1k ^ (t1 & tk);
    }
    u128 last = gplus<GROUP>(gplus<GROUP>(blk128(s1), gneg<GROUP>(blk128(s0))), gneg<GROUP>(v));
    if (t1) last = gneg<GROUP>(last);
    w0.v128(last);
    w1.v128(last);
  }
}

}  // namespace

cudaError_t launch_myl7_gen(const sufb200_ctx_s* ctx, int group, const GenLaunch& g, cudaStream_t st) {
  const size_t want = (g.n + kGenThreads - 1) / kGenThreads;
  const int grid = static_cast<int>(want < static_cast<size_t>(ctx->sm_count) ? (want ? want : 1) : ctx->sm_count);
  cudaError_t e;
  if (group == SUFB200_GROUP_ADD) {
    e = cudaFuncSetAttribute(myl7_gen_kernel<SUFB200_GROUP_ADD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(ctx->aes_dyn_bytes));
    if (e != cudaSuccess) return e;
    myl7_gen_kernel<SUFB200_GROUP_ADD><<<grid, kGenThreads, ctx->aes_dyn_bytes, st>>>(ctx->prg, g);
  } else {
    e = cudaFuncSetAttribute(myl7_gen_kernel<SUFB200_GROUP_XOR>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(ctx->aes_dyn_bytes));
    if (e != cudaSuccess) return e;
    myl7_gen_kernel<SUFB200_GROUP_XOR><<<grid, kGenThreads, ctx->aes_dyn_bytes, st>>>(ctx->prg, g);
  }
  return cudaGetLastError();
}

}  // namespace sufb200
