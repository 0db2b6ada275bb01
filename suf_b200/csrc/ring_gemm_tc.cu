// ring_gemm_tc.cu -- exact Z_2^64 matrix products on the 5th-generation tensor
// cores (tcgen05, kind::i8) by 8-bit limb decomposition.
//
// For u64 operands x = sum_i 2^(8i) x_i and y = sum_j 2^(8j) y_j (bytes),
//   x * y mod 2^64 = sum_{i+j <= 7} 2^(8(i+j)) x_i y_j   (terms with i+j >= 8 vanish).
// A 128 x 64 output tile keeps one int32 accumulator per diagonal s = i + j
// in tensor memory (8 diagonals x 64 columns = all 512 TMEM columns); every
// 32-deep K step issues twelve unsigned 8-bit MMAs (128 x N x 32, N <= 256)
// that together cover the 36 limb pairs (i, j), i + j <= 7, each landing in
// its diagonal, and the epilogue folds
//   acc = sum_s (P_s mod 2^32) << 8s  mod 2^64.
// That is exact as long as P_s is exact wherever bits survive the shift:
// for s <= 3 the diagonal sums stay below 2^31 while K' <= 8192 (P_s <=
// (s+1) K' 255^2), and for s >= 4 only P_s mod 2^(64-8s) | 2^32 matters,
// which the non-saturating accumulator keeps.
//
// A bandwidth-bound pre-pass writes each operand as 8 byte planes already in
// the canonical K-major no-swizzle layout of the UMMA shared-memory
// descriptor (8-row x 16-byte core matrices; leading byte offset 128 between
// the two K halves of a 32-deep step, stride byte offset 256 between 8-row
// groups), tiled so that a CTA's plane block for one step is one contiguous
// range.  The GEMM then runs a 4-stage pipeline: one warp issues two plain
// bulk copies (cp.async.bulk, no multicast) per step, A and B plane blocks,
// against a transaction-count mbarrier, one warp issues the twelve MMAs of
// the step and commits them back to the stage's "empty" mbarrier (one lane of
// each does the issuing), and all warps read the diagonals out of tensor
// memory at the end.  Every wait is bounded.  When B is row-major with
// 16-byte rows, B's planes are instead made inside the GEMM from raw boxes
// loaded by tensor-map TMA (ring_gemm_tc_fused_kernel), so B crosses HBM
// once, as words.
// Contractions too short to fill the GPU are split across the CTAs of one
// thread-block cluster per output tile, which sum their partial tiles through
// distributed shared memory and store the result once.
//
// Serves the reference's Beaver matmul (cuda/cuda_primitives.cu:391-628,
// out = C + D B + A E (+ D E for party 0) as ONE product [D | A] x [B (+E) ; E])
// and the public-weight matmul (src/nn/matmul_gpu.cu:21-117, Y = X W + bias).
#include <atomic>

#include <cuda.h>  // CUtensorMap and its enums (the encoder comes from cudaGetDriverEntryPoint)

#include "kernels.hpp"
#include "ring_common.cuh"

namespace sufb200 {

namespace {

constexpr int kTM = 128;  // output rows per tile (TMEM lanes)
constexpr int kTN = 64;   // output columns per tile (per diagonal)
constexpr int kTK = 32;   // K per MMA (8-bit operands)
constexpr int kThreads = 128;
constexpr int kStages = 4;
constexpr uint32_t kPlaneX = kTM * kTK;                    // 4 KB: one plane of the A tile
constexpr uint32_t kPlaneY = kTN * kTK;                    // 2 KB: one plane of the B tile
constexpr uint32_t kStageBytes = 8 * (kPlaneX + kPlaneY);  // 48 KB
constexpr uint32_t kCtrlOffset = kStages * kStageBytes;    // mbarriers, error flag, TMEM slot
constexpr uint32_t kSmemBytes = kCtrlOffset + 256;         // 192 KB: one CTA per SM, all 512 TMEM columns
constexpr uint32_t kTmemCols = 512;
// idesc for kind::i8 with M = 128 and the given N: D s32 (bits 4-5 = 2), A
// and B unsigned 8-bit, both K-major, N >> 3 at bits 17-22, M >> 4 at 24-28.
__host__ __device__ constexpr uint32_t idesc_n(int n) { return (2u << 4) | (uint32_t(n >> 3) << 17) | (uint32_t(kTM >> 4) << 24); }
constexpr uint32_t kWaitIters = 1u << 26;
constexpr uint64_t kWaitNs = 2000000000ull;  // give up after 2 s of wall time

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// K-major, no swizzle: start >> 4, LBO 128 B, SBO 256 B, version 1.
__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr) {
  return static_cast<uint64_t>((saddr >> 4) & 0x3FFFu) | (static_cast<uint64_t>(128 >> 4) << 16) |
         (static_cast<uint64_t>(256 >> 4) << 32) | (1ull << 46);
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// Bounded wait for the phase with the given parity (iterations and wall
// time, since one try_wait may suspend for an implementation-defined while);
// false on timeout.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
  const uint64_t t0 = global_ns();
  for (uint32_t it = 0; it < kWaitIters; it++) {
    if ((it & 255u) == 255u && global_ns() - t0 > kWaitNs) return false;
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(bar), "r"(parity)
        : "memory");
    if (done) return true;
  }
  return false;
}

__device__ __forceinline__ void umma_i8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}"
      :
      : "r"(d_tmem), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u));
}

__device__ __forceinline__ void umma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

// 16 columns of this warp's 32 lanes; the registers are valid after tmem_wait.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, "
      "[%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
        "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
      : "r"(taddr));
}

// Waits for this thread's outstanding tensor-memory loads; taking the
// registers as operands keeps every use of them after the wait.
__device__ __forceinline__ void tmem_wait(uint32_t (&v)[16]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(v[0]), "+r"(v[1]), "+r"(v[2]), "+r"(v[3]), "+r"(v[4]), "+r"(v[5]), "+r"(v[6]), "+r"(v[7]),
                 "+r"(v[8]), "+r"(v[9]), "+r"(v[10]), "+r"(v[11]), "+r"(v[12]), "+r"(v[13]), "+r"(v[14]), "+r"(v[15])
               :
               : "memory");
}

// Offset of (row r, K half h) inside a plane slab (core-matrix order).
__device__ __forceinline__ uint32_t core_off(int r, int h) {
  return static_cast<uint32_t>((r >> 3) * 256 + h * 128 + (r & 7) * 16);
}

__device__ __forceinline__ void bulk_copy(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "l"(src), "r"(bytes), "r"(bar)
               : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

// Plane i (byte i of every word) of 16 K-consecutive words: 16 bytes.
__device__ __forceinline__ uint4 plane_bytes(const uint64_t (&v)[16], int i) {
  uint32_t w[4];
#pragma unroll
  for (int q = 0; q < 4; q++) {
    const uint32_t a0 = static_cast<uint32_t>(v[4 * q + 0] >> (i < 4 ? 0 : 32));
    const uint32_t a1 = static_cast<uint32_t>(v[4 * q + 1] >> (i < 4 ? 0 : 32));
    const uint32_t a2 = static_cast<uint32_t>(v[4 * q + 2] >> (i < 4 ? 0 : 32));
    const uint32_t a3 = static_cast<uint32_t>(v[4 * q + 3] >> (i < 4 ? 0 : 32));
    const uint32_t sel = static_cast<uint32_t>(i & 3) | (static_cast<uint32_t>(4 + (i & 3)) << 4);
    w[q] = __byte_perm(__byte_perm(a0, a1, sel), __byte_perm(a2, a3, sel), 0x5410);
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}

// The B planes of a stage are consecutive 64-row blocks in core-matrix
// order, so [y_0 | y_1 | y_2 | y_3] is one N = 256 operand.  x_i times it,
// accumulated at column 64 i, lands product (i, j) on column 64 (i + j):
// diagonal i + j.  Twelve MMAs (N = 256 except where the 512 columns end)
// cover the 36 limb pairs; the first two write all 512 columns, so on the
// first step (accumulate = 0) they alone start from zero.
__device__ __forceinline__ void mma_step(const uint32_t (&dt)[8], const uint64_t (&as)[8], const uint64_t (&bs)[8],
                                         uint32_t accumulate) {
  umma_i8(dt[0], as[0], bs[0], idesc_n(256), accumulate);
  umma_i8(dt[4], as[0], bs[4], idesc_n(256), accumulate);
#pragma unroll
  for (int i = 1; i < 8; i++) umma_i8(dt[i], as[i], bs[0], idesc_n(i <= 4 ? 256 : 64 * (8 - i)), 1u);
#pragma unroll
  for (int i = 1; i < 4; i++) umma_i8(dt[i + 4], as[i], bs[4], idesc_n(256 - 64 * i), 1u);
}

// ---- Epilogue: the K-split CTAs of a tile are one thread-block cluster ----
// Every CTA folds its 8 diagonals into a 128 x 64 word tile in its own shared
// memory (the pipeline stages are idle by then); after a cluster barrier each
// of the S ranks sums a 1/S share of the tile's 16-byte chunks over all S
// tiles through distributed shared memory, adds C and the bias, rescales and
// stores it with coalesced rows.  A second barrier keeps every rank's tile
// alive until its readers are done.  S = 1 takes the same path.  (Split
// partials through global memory cost an 8 us epilogue of one-row-per-thread
// stores plus a 6 us reduction kernel per FFN1 call.)
constexpr int kChunks = kTM * kTN / 2;  // 16-byte chunks of a tile

// Chunk c (words 2c, 2c+1) of tile row `row`; chunks XOR-swizzled by row so
// both the row-per-thread fold and the chunk-per-thread reduction are free
// of bank conflicts.
__device__ __forceinline__ uint32_t tile_chunk(int row, int c) {
  return static_cast<uint32_t>(row * (kTN * 8) + ((c ^ (row & 7)) << 4));
}

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile(
      "barrier.cluster.arrive.release.aligned;\n\t"
      "barrier.cluster.wait.acquire.aligned;" ::
          : "memory");
}

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

__device__ __forceinline__ uint32_t cluster_size() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(r));
  return r;
}

// Generic pointer to the same shared-memory object in cluster rank `rank`
// (plain loads through it, so the compiler can keep many in flight; they
// are ordered after the cluster barrier by its memory clobber).
__device__ __forceinline__ const ulonglong2* rank_ptr(const void* p, uint32_t rank) {
  uint64_t a;
  asm("mapa.u64 %0, %1, %2;" : "=l"(a) : "l"(reinterpret_cast<uint64_t>(p)), "r"(rank));
  return reinterpret_cast<const ulonglong2*>(a);
}

// The folded tile, sum_s (P_s mod 2^32) << 8s per word, into this CTA's
// shared memory.  A warp reads the TMEM lanes of its quarter (warp % 4);
// the groups of four warps deal the 16-column blocks among themselves.
__device__ __forceinline__ void fold_tile(uint32_t tmem, int warp, int lane, int nwarps, uint8_t* tile) {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const int quarter = warp & 3, row = quarter * 32 + lane;
  const int groups = nwarps / 4 < kTN / 16 ? nwarps / 4 : kTN / 16;
#pragma unroll 1
  for (int cb = warp >> 2; cb < kTN / 16; cb += groups) {
    uint32_t v[8][16];  // the 8 diagonals of 16 columns, loaded before one wait
#pragma unroll
    for (int s = 0; s < 8; s++)
      tmem_ld16(tmem + (static_cast<uint32_t>(quarter * 32) << 16) + static_cast<uint32_t>(s * kTN + cb * 16), v[s]);
#pragma unroll
    for (int s = 0; s < 8; s++) tmem_wait(v[s]);
#pragma unroll
    for (int q = 0; q < 8; q++) {
      uint64_t a0 = 0, a1 = 0;
#pragma unroll
      for (int s = 0; s < 8; s++) {
        a0 += static_cast<uint64_t>(v[s][2 * q]) << (8 * s);
        a1 += static_cast<uint64_t>(v[s][2 * q + 1]) << (8 * s);
      }
      *reinterpret_cast<ulonglong2*>(tile + tile_chunk(row, cb * 8 + q)) = make_ulonglong2(a0, a1);
    }
  }
}

// Chunks [lo, hi) of the tile are this rank's share of the reduction.
__device__ __forceinline__ void rank_share(int& lo, int& hi) {
  const uint32_t S = cluster_size(), q = cluster_rank();
  lo = static_cast<int>(q * kChunks / S);
  hi = static_cast<int>((q + 1) * kChunks / S);
}

// One warp, during the main loop: the rows of C under this rank's share
// into L2, so the reduction's C loads do not wait on HBM.
__device__ __forceinline__ void prefetch_c_share(const RingGemmLaunch& g, int b, int m0, int n0, int lane) {
  if (!g.c) return;
  int lo, hi;
  rank_share(lo, hi);
  if (hi <= lo) return;
  const int r0 = lo / (kTN / 2), r1 = (hi - 1) / (kTN / 2);
  const uint64_t* C = g.c + static_cast<size_t>(b) * g.cs;
  for (int u = lane; u < (r1 - r0 + 1) * 4; u += 32) {
    const int m = m0 + r0 + u / 4, n = n0 + 16 * (u % 4);  // 128-byte lines of the row
    if (m < g.M && n < g.N) asm volatile("prefetch.global.L2 [%0];" ::"l"(C + static_cast<size_t>(m) * g.N + n));
  }
}

// All threads: this rank's share of the tile, summed over the cluster's
// tiles (addition mod 2^64 commutes), plus C and the bias, rescaled, stored.
// Four chunks per thread at a time, their loads all issued before the first
// use, so the loop pays the load latency once per four chunks.
__device__ __forceinline__ void reduce_tile(const RingGemmLaunch& g, int b, int m0, int n0, const uint8_t* tile, int t,
                                            int nthr) {
  constexpr int kBatch = 4;
  const uint32_t S = cluster_size();
  int lo, hi;
  rank_share(lo, hi);
  const uint64_t* C = g.c ? g.c + static_cast<size_t>(b) * g.cs : nullptr;
  uint64_t* O = g.out + static_cast<size_t>(b) * g.os;
  for (int base = lo + t; base < hi; base += kBatch * nthr) {
    uint64_t s0[kBatch], s1[kBatch];
    size_t o[kBatch];
    int n[kBatch];
    bool ok[kBatch];
#pragma unroll
    for (int u = 0; u < kBatch; u++) {
      const int ch = base + u * nthr;
      const int row = ch / (kTN / 2), c = ch % (kTN / 2);
      const int m = m0 + row;
      n[u] = n0 + 2 * c;
      ok[u] = ch < hi && m < g.M && n[u] < g.N;
      o[u] = static_cast<size_t>(m) * g.N + n[u];
      s0[u] = 0;
      s1[u] = 0;
      if (ok[u]) {
        if (C) {
          s0[u] = C[o[u]];
          if (n[u] + 1 < g.N) s1[u] = C[o[u] + 1];
        }
        if (g.bias) {
          s0[u] += static_cast<uint64_t>(g.bias[n[u]]);
          if (n[u] + 1 < g.N) s1[u] += static_cast<uint64_t>(g.bias[n[u] + 1]);
        }
      }
    }
#pragma unroll
    for (int u = 0; u < kBatch; u++) {
      if (!ok[u]) continue;
      const int ch = base + u * nthr;
      const uint8_t* a = tile + tile_chunk(ch / (kTN / 2), ch % (kTN / 2));
#pragma unroll 4
      for (uint32_t r = 0; r < S; r++) {
        const ulonglong2 xy = *rank_ptr(a, r);
        s0[u] += xy.x;
        s1[u] += xy.y;
      }
    }
#pragma unroll
    for (int u = 0; u < kBatch; u++) {
      if (!ok[u]) continue;
      O[o[u]] = scaled_acc(s0[u], g.has_scale, g.mul_const, g.mul_shift);
      if (n[u] + 1 < g.N) O[o[u] + 1] = scaled_acc(s1[u], g.has_scale, g.mul_const, g.mul_shift);
    }
  }
}

// The common tail of both GEMM kernels: fold, reduce over the cluster, free
// the tensor memory.  Every thread of every rank reaches both cluster
// barriers, on the error path too.
__device__ __forceinline__ void finish_tile(const RingGemmLaunch& g, uint8_t* smem, uint32_t tmem, bool ok, int nsteps,
                                            int warp, int lane, int t, int b, int m0, int n0) {
  const int nwarps = static_cast<int>(blockDim.x) / 32;
  if (ok) {
    if (nsteps > 0) {
      fold_tile(tmem, warp, lane, nwarps, smem);
    } else if (warp < 4) {
      for (int c = 0; c < kTN / 2; c++)
        *reinterpret_cast<ulonglong2*>(smem + tile_chunk(warp * 32 + lane, c)) = make_ulonglong2(0, 0);
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  cluster_sync_all();  // every rank's tile is in its shared memory
  reduce_tile(g, b, m0, n0, smem, t, static_cast<int>(blockDim.x));
  cluster_sync_all();  // every reader of this CTA's tile is done
  if (warp == 0) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
  }
}

// Byte planes of one operand, tiled for the GEMM: for step c and row tile
// (tile rows T = 128 for A, 64 for B) the 8 planes of T rows x 32 bytes in
// core-matrix order, contiguous (one bulk copy per operand per step).
// Unit (c, h, r, q): words 4q..4q+3 of the 16 K-consecutive words of row r,
// K half h of step c; it writes 4 bytes of each plane, and the four units of
// a 16-byte core-matrix row are adjacent threads (short load chains, many
// threads: the pass is latency-bound at configs[4] sizes).
// k_contig: element (row, k) at src[row * K + k], else at src[k * R + row].
__device__ __forceinline__ void split_planes(const PlanesSplit& p, int block, int nblocks, int b) {
  const size_t units = static_cast<size_t>(p.steps) * 2 * static_cast<size_t>(p.rows_pad) * 4;
  const int cpp = (p.K + kTK - 1) / kTK;
  for (size_t u = static_cast<size_t>(block) * blockDim.x + threadIdx.x; u < units;
       u += static_cast<size_t>(nblocks) * blockDim.x) {
    const int q = static_cast<int>(u & 3);
    const size_t w = u >> 2;
    const int r = static_cast<int>(w % static_cast<size_t>(p.rows_pad));
    const int h = static_cast<int>((w / static_cast<size_t>(p.rows_pad)) & 1);
    const int c = static_cast<int>(w / (2 * static_cast<size_t>(p.rows_pad)));
    const bool second = c >= cpp;  // selects, not an indexed copy of the parameter
    const uint64_t* src = (second ? p.piece[1].src : p.piece[0].src) +
                          static_cast<size_t>(b) * (second ? p.piece[1].ss : p.piece[0].ss);
    const uint64_t* add = second ? p.piece[1].add : p.piece[0].add;
    if (add) add += static_cast<size_t>(b) * (second ? p.piece[1].as : p.piece[0].as);
    const int k0 = (c % cpp) * kTK + 16 * h + 4 * q;
    uint64_t v[4];
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const int k = k0 + j;
      uint64_t val = 0;
      if (r < p.R && k < p.K) {
        const size_t idx = p.k_contig ? static_cast<size_t>(r) * p.K + k : static_cast<size_t>(k) * p.R + r;
        val = __ldg(src + idx);
        if (add) val += __ldg(add + idx);
      }
      v[j] = val;
    }
    uint8_t* dst = p.dst + static_cast<size_t>(b) * p.ds;
    const int tiles = p.rows_pad / p.tile_rows, tile = r / p.tile_rows, rr = r % p.tile_rows;
    const size_t plane = static_cast<size_t>(p.tile_rows) * kTK;
    uint8_t* blk = dst + ((static_cast<size_t>(c) * tiles + tile) * 8) * plane + core_off(rr, h) + 4 * q;
#pragma unroll
    for (int i = 0; i < 8; i++) {
      const uint32_t a0 = static_cast<uint32_t>(v[0] >> (i < 4 ? 0 : 32));
      const uint32_t a1 = static_cast<uint32_t>(v[1] >> (i < 4 ? 0 : 32));
      const uint32_t a2 = static_cast<uint32_t>(v[2] >> (i < 4 ? 0 : 32));
      const uint32_t a3 = static_cast<uint32_t>(v[3] >> (i < 4 ? 0 : 32));
      const uint32_t sel = static_cast<uint32_t>(i & 3) | (static_cast<uint32_t>(4 + (i & 3)) << 4);
      *reinterpret_cast<uint32_t*>(blk + i * plane) =
          __byte_perm(__byte_perm(a0, a1, sel), __byte_perm(a2, a3, sel), 0x5410);
    }
  }
}

// The GEMM after it is launched as its programmatic dependent: it may start
// its prologue and B loads at once and waits (griddepcontrol.wait) only
// before it reads the planes written here.
__global__ void split_planes_kernel(const PlanesSplit px, const PlanesSplit py, int xblocks, int xb, int yb) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const int b = blockIdx.y;
  if (static_cast<int>(blockIdx.x) < xblocks) {
    if (b < xb) split_planes(px, blockIdx.x, xblocks, b);
  } else if (b < yb) {
    split_planes(py, blockIdx.x - xblocks, gridDim.x - xblocks, b);
  }
}

__global__ void __launch_bounds__(kThreads, 1) ring_gemm_tc_kernel(const RingGemmLaunch g) {
  extern __shared__ __align__(1024) uint8_t smem[];
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  const int b = blockIdx.z / g.splits, split = blockIdx.z % g.splits;
  const int m0 = blockIdx.y * kTM, n0 = blockIdx.x * kTN;
  const int M = g.M, N = g.N;
  const uint32_t sbase = smem_u32(smem);
  const uint32_t full0 = sbase + kCtrlOffset, empty0 = full0 + 8 * kStages, done = empty0 + 8 * kStages;
  const uint32_t slot = done + 8;
  volatile uint32_t* err = reinterpret_cast<volatile uint32_t*>(smem + kCtrlOffset + 16 * kStages + 16);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kCtrlOffset + 16 * kStages + 8);

  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(slot), "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (t == 0) {
    for (int i = 0; i < kStages; i++) {
      mbar_init(full0 + 8 * i, 1);
      mbar_init(empty0 + 8 * i, 1);
    }
    mbar_init(done, 1);
    *err = 0;
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;

  // this CTA's share of the contraction: steps [c0, c1)
  const int per = (g.steps + g.splits - 1) / g.splits;
  const int c0 = split * per, c1 = c0 + per < g.steps ? c0 + per : g.steps;
  const int nsteps = c1 > c0 ? c1 - c0 : 0;
  const uint8_t* xp = g.xplanes + static_cast<size_t>(b) * g.xps;
  const uint8_t* yp = g.yplanes + static_cast<size_t>(b) * g.yps;
  const int tiles_m = g.m_pad / kTM, tiles_n = g.n_pad / kTN;

  // Roles are warp-uniform: lane 0 waits and issues while the other lanes of
  // its warp sit at the warp's shuffle, so no lane of the issuing warp spins
  // on a different barrier than the one lane 0 is serving.
  if (warp == 0) {  // producer: one bulk copy per operand per step
    asm volatile("griddepcontrol.wait;" ::: "memory");  // the planes of the pre-pass
    for (int li = 0; li < nsteps; li++) {
      const int st = li % kStages;
      const uint32_t sb = sbase + static_cast<uint32_t>(st) * kStageBytes;
      const uint32_t fb = full0 + 8 * st;
      int go = 1;
      if (lane == 0) {
        go = li < kStages || mbar_wait(empty0 + 8 * st, static_cast<uint32_t>(((li / kStages) - 1) & 1));
        if (go) {
          mbar_expect_tx(fb, kStageBytes);
          const size_t c = static_cast<size_t>(c0 + li);
          bulk_copy(sb, xp + (c * tiles_m + blockIdx.y) * (8 * kPlaneX), 8 * kPlaneX, fb);
          bulk_copy(sb + 8 * kPlaneX, yp + (c * tiles_n + blockIdx.x) * (8 * kPlaneY), 8 * kPlaneY, fb);
        } else {
          *err = 1;
        }
      }
      if (!__shfl_sync(0xffffffffu, go, 0)) break;
    }
  } else if (warp == 3) {  // idle in the main loop: C of the epilogue into L2
    prefetch_c_share(g, b, m0, n0, lane);
  } else if (warp == 1) {  // MMA issuer: the 36 limb MMAs of a step, then release the stage
    // Stage 0's plane descriptors and the diagonals' column addresses, once:
    // a stage's descriptors are these plus its byte offset >> 4 in the start
    // field (shared-memory addresses stay below 2^18, so the field never
    // carries), which leaves one instruction per MMA to issue.
    uint64_t ad[8], bd[8];
    uint32_t dt[8];
#pragma unroll
    for (int i = 0; i < 8; i++) {
      ad[i] = umma_desc(sbase + static_cast<uint32_t>(i) * kPlaneX);
      bd[i] = umma_desc(sbase + 8 * kPlaneX + static_cast<uint32_t>(i) * kPlaneY);
      dt[i] = tmem + static_cast<uint32_t>(i * kTN);
    }
    for (int li = 0; li < nsteps; li++) {
      const int st = li % kStages;
      int go = 1;
      if (lane == 0) {
        go = mbar_wait(full0 + 8 * st, static_cast<uint32_t>((li / kStages) & 1));
        if (go) {
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          const uint64_t so = static_cast<uint64_t>((static_cast<uint32_t>(st) * kStageBytes) >> 4);
          uint64_t as[8], bs[8];
#pragma unroll
          for (int i = 0; i < 8; i++) {
            as[i] = ad[i] + so;
            bs[i] = bd[i] + so;
          }
          mma_step(dt, as, bs, li > 0 ? 1u : 0u);
          umma_commit(empty0 + 8 * st);
        } else {
          *err = 1;
        }
      }
      if (!__shfl_sync(0xffffffffu, go, 0)) break;
    }
    if (lane == 0) umma_commit(done);  // arrives once every MMA issued above has completed
    __syncwarp();
  }
  bool ok = mbar_wait(done, 0);
  ok = __syncthreads_and(ok ? 1 : 0) != 0 && *err == 0;
  if (!ok) {
    if (t == 0) atomicOr(g.status, kStatusTimeout);
    mbar_wait(done, 0);  // let whatever was issued drain before the columns are released
  }
  finish_tile(g, smem, tmem, ok, nsteps, warp, lane, t, b, m0, n0);
}

// ---- B split inside the GEMM --------------------------------------------
// For a row-major B (K x N words, N even, 16-byte base) the byte planes of B
// are made inside the GEMM instead of by the pre-pass: warp 0 loads each
// step's raw 32 x 64 words of B (and of the Beaver addend) with one tiled
// tensor-map load per matrix (no multicast; x = n0 is a multiple of 64 words,
// out-of-range rows and columns read as zero) into one of three raw stages;
// warps 4-11 split a landed raw stage into one of two B-plane stages and
// fence them to the async proxy; warp 2 bulk-copies the step's A planes into
// one of three A stages; warp 1 issues the twelve MMAs and commits the A and
// B stages back; warp 3 prefetches the epilogue's C into L2.  B crosses HBM
// once as words instead of being read, written as planes and read again.
// The main loop is bound by the chain raw stage landed -> split -> B planes
// ready -> MMAs: with four converter warps a step took 1.28 us against
// 0.87 us for its MMAs alone; eight (two per SM sub-partition, eight K words
// per thread) took 16 % off the configs[4] layer's four calls, while the
// stage counts (3/2/3, 3/3/2, 3/4/2, 2/3/3) changed them by 1 % at most.
// The counts and the converter warps are compile-time parameters.
#ifndef SUFB200_F_CONV_WARPS
#define SUFB200_F_CONV_WARPS 8
#endif
#ifndef SUFB200_F_A_STAGES
#define SUFB200_F_A_STAGES 3
#endif
#ifndef SUFB200_F_B_STAGES
#define SUFB200_F_B_STAGES 2
#endif
#ifndef SUFB200_F_RAW_STAGES
#define SUFB200_F_RAW_STAGES 3
#endif
constexpr int kFConvWarps = SUFB200_F_CONV_WARPS;  // converter warps (4 or 8)
constexpr int kFThreads = 128 + 32 * kFConvWarps;
constexpr int kFAStages = SUFB200_F_A_STAGES;      // A-plane stages
constexpr int kFBStages = SUFB200_F_B_STAGES;      // B-plane stages
constexpr int kFRawStages = SUFB200_F_RAW_STAGES;  // raw B (+ addend) stages
constexpr int kFConvK = kTK * kTN / (32 * kFConvWarps);  // K words one converter thread splits per step
static_assert(kFConvWarps == 4 || kFConvWarps == 8, "converter split");
constexpr uint32_t kFAStage = 8 * kPlaneX;                            // 32 KB of A planes
constexpr uint32_t kFBStage = 8 * kPlaneY;                            // 16 KB of B planes
constexpr uint32_t kFRawHalf = kTK * kTN * 8;                         // 16 KB: 32 rows x 64 words
constexpr uint32_t kFRawStage = 2 * kFRawHalf;                        // B words, then the addend's
constexpr uint32_t kFBOffset = kFAStages * kFAStage;
constexpr uint32_t kFRawOffset = kFBOffset + kFBStages * kFBStage;
constexpr uint32_t kFCtrl = kFRawOffset + kFRawStages * kFRawStage;
constexpr uint32_t kFSmemBytes = kFCtrl + 256;
static_assert(kFSmemBytes <= 227 * 1024, "dynamic shared memory per CTA");
static_assert(kFCtrl >= kTM * kTN * 8, "the epilogue tile reuses the stages");

// Tensor maps of B and the addend per piece: m[2 p] = B_p, m[2 p + 1] = its
// addend; 3-D {N, K, batch} u64, box {64, 32, 1}, zero fill out of range.
struct alignas(64) BMaps {
  CUtensorMap m[4];
};

// One box of 32 K-rows x 64 words at (n0, k0, batch) into shared memory.
__device__ __forceinline__ void tma_load_box(uint32_t dst, const CUtensorMap* map, int x, int y, int z, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(
          dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(bar)
      : "memory");
}

__global__ void __launch_bounds__(kFThreads, 1)
    ring_gemm_tc_fused_kernel(const __grid_constant__ RingGemmLaunch g, const __grid_constant__ BMaps bm) {
  extern __shared__ __align__(1024) uint8_t smem[];
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  const int b = blockIdx.z / g.splits, split = blockIdx.z % g.splits;
  const int m0 = blockIdx.y * kTM, n0 = blockIdx.x * kTN;
  const uint32_t sbase = smem_u32(smem);
  // control block: full/empty mbarriers of the A, B-plane and raw rings
  constexpr uint32_t kOffAE = 8 * kFAStages, kOffBF = 16 * kFAStages, kOffBE = kOffBF + 8 * kFBStages,
                     kOffRF = kOffBE + 8 * kFBStages, kOffRE = kOffRF + 8 * kFRawStages,
                     kOffDone = kOffRE + 8 * kFRawStages;
  static_assert(kOffDone + 24 <= 256, "control block");
  const uint32_t ctrl = sbase + kFCtrl;
  const uint32_t afull0 = ctrl, aempty0 = ctrl + kOffAE, bfull0 = ctrl + kOffBF, bempty0 = ctrl + kOffBE;
  const uint32_t rfull0 = ctrl + kOffRF, rempty0 = ctrl + kOffRE;
  const uint32_t done = ctrl + kOffDone, slot = done + 8;
  volatile uint32_t* err = reinterpret_cast<volatile uint32_t*>(smem + kFCtrl + kOffDone + 16);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kFCtrl + kOffDone + 8);

  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(slot), "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  } else if (warp == 3 && lane < 2 * g.npieces) {  // the tensor maps this CTA will load through
    if (lane % 2 == 0 || g.piece[lane / 2].y2)
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&bm.m[lane])) : "memory");
  }
  if (t == 0) {
    for (int i = 0; i < kFAStages; i++) {
      mbar_init(afull0 + 8 * i, 1);  // the A copy's arrival (with its transaction bytes)
      mbar_init(aempty0 + 8 * i, 1);
    }
    for (int i = 0; i < kFBStages; i++) {
      mbar_init(bfull0 + 8 * i, kFConvWarps);  // the converter warps
      mbar_init(bempty0 + 8 * i, 1);
    }
    for (int i = 0; i < kFRawStages; i++) {
      mbar_init(rfull0 + 8 * i, 1);
      mbar_init(rempty0 + 8 * i, kFConvWarps);
    }
    mbar_init(done, 1);
    *err = 0;
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;

  const int per = (g.steps + g.splits - 1) / g.splits;
  const int c0 = split * per, c1 = c0 + per < g.steps ? c0 + per : g.steps;
  const int nsteps = c1 > c0 ? c1 - c0 : 0;
  const uint8_t* xp = g.xplanes + static_cast<size_t>(b) * g.xps;
  const int tiles_m = g.m_pad / kTM;
  const int K = g.K, N = g.N, cpp = (K + kTK - 1) / kTK;
  const int cnt = N - n0 < kTN ? N - n0 : kTN;  // valid words of each raw row (the rest read as zero)

  if (warp == 0) {  // raw B (and addend) rows of each step
    for (int li = 0; li < nsteps; li++) {
      const int rs = li % kFRawStages;
      int go = 1;
      if (lane == 0) {
        go = li < kFRawStages || mbar_wait(rempty0 + 8 * rs, static_cast<uint32_t>(((li / kFRawStages) - 1) & 1));
        if (go) {
          const int c = c0 + li;
          const int p = c >= cpp ? 1 : 0;
          const bool add = (p ? g.piece[1].y2 : g.piece[0].y2) != nullptr;
          const int zb = (p ? g.piece[1].ys : g.piece[0].ys) ? b : 0;
          const int za = (p ? g.piece[1].y2s : g.piece[0].y2s) ? b : 0;
          const int k0 = (c % cpp) * kTK;
          const uint32_t rb = sbase + kFRawOffset + static_cast<uint32_t>(rs) * kFRawStage;
          mbar_expect_tx(rfull0 + 8 * rs, add ? kFRawStage : kFRawHalf);
          tma_load_box(rb, &bm.m[2 * p], n0, k0, zb, rfull0 + 8 * rs);
          if (add) tma_load_box(rb + kFRawHalf, &bm.m[2 * p + 1], n0, k0, za, rfull0 + 8 * rs);
        } else {
          *err = 1;
        }
      }
      if (!__shfl_sync(0xffffffffu, go, 0)) break;
    }
  } else if (warp == 2) {  // A planes of each step
    asm volatile("griddepcontrol.wait;" ::: "memory");  // written by the pre-pass
    for (int li = 0; li < nsteps; li++) {
      const int as = li % kFAStages;
      int go = 1;
      if (lane == 0) {
        go = li < kFAStages || mbar_wait(aempty0 + 8 * as, static_cast<uint32_t>(((li / kFAStages) - 1) & 1));
        if (go) {
          mbar_expect_tx(afull0 + 8 * as, kFAStage);
          const size_t c = static_cast<size_t>(c0 + li);
          bulk_copy(sbase + static_cast<uint32_t>(as) * kFAStage, xp + (c * tiles_m + blockIdx.y) * kFAStage,
                    kFAStage, afull0 + 8 * as);
        } else {
          *err = 1;
        }
      }
      if (!__shfl_sync(0xffffffffu, go, 0)) break;
    }
  } else if (warp == 3) {  // idle in the main loop: C of the epilogue into L2
    prefetch_c_share(g, b, m0, n0, lane);
  } else if (warp == 1) {  // MMA issuer
    uint64_t ad[8], bd[8];
    uint32_t dt[8];
#pragma unroll
    for (int i = 0; i < 8; i++) {
      ad[i] = umma_desc(sbase + static_cast<uint32_t>(i) * kPlaneX);
      bd[i] = umma_desc(sbase + kFBOffset + static_cast<uint32_t>(i) * kPlaneY);
      dt[i] = tmem + static_cast<uint32_t>(i * kTN);
    }
    for (int li = 0; li < nsteps; li++) {
      const int as = li % kFAStages, bs = li % kFBStages;
      int go = 1;
      if (lane == 0) {
        go = mbar_wait(afull0 + 8 * as, static_cast<uint32_t>((li / kFAStages) & 1)) &&
             mbar_wait(bfull0 + 8 * bs, static_cast<uint32_t>((li / kFBStages) & 1));
        if (go) {
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          // descriptors of stage 0 plus the stage's byte offset >> 4 (addresses
          // stay below 2^18, so the start field never carries)
          const uint64_t ao = static_cast<uint64_t>((static_cast<uint32_t>(as) * kFAStage) >> 4);
          const uint64_t bo = static_cast<uint64_t>((static_cast<uint32_t>(bs) * kFBStage) >> 4);
          uint64_t a[8], bb[8];
#pragma unroll
          for (int i = 0; i < 8; i++) {
            a[i] = ad[i] + ao;
            bb[i] = bd[i] + bo;
          }
          mma_step(dt, a, bb, li > 0 ? 1u : 0u);
          umma_commit(aempty0 + 8 * as);
          umma_commit(bempty0 + 8 * bs);
        } else {
          *err = 1;
        }
      }
      if (!__shfl_sync(0xffffffffu, go, 0)) break;
    }
    if (lane == 0) umma_commit(done);
    __syncwarp();
  } else if (warp >= 4) {  // converters: a landed raw stage into a B-plane stage
    const int ct = (warp - 4) * 32 + lane;
    const int r = ct % kTN, kq = (ct / kTN) * kFConvK;  // B-tile row (output column n0 + r), first K word
    for (int li = 0; li < nsteps; li++) {
      const int rs = li % kFRawStages, bs = li % kFBStages;
      int go = 1;
      if (lane == 0)
        go = mbar_wait(rfull0 + 8 * rs, static_cast<uint32_t>((li / kFRawStages) & 1)) &&
             (li < kFBStages || mbar_wait(bempty0 + 8 * bs, static_cast<uint32_t>(((li / kFBStages) - 1) & 1)));
      if (!__shfl_sync(0xffffffffu, go, 0)) {
        if (lane == 0) *err = 1;
        break;
      }
      const int c = c0 + li;
      const bool add = (c >= cpp ? g.piece[1].y2 : g.piece[0].y2) != nullptr;
      const int k0 = (c % cpp) * kTK;
      const uint64_t* raw = reinterpret_cast<const uint64_t*>(smem + kFRawOffset + rs * kFRawStage);
      uint64_t v[16];
#pragma unroll
      for (int j = 0; j < 16; j++) {
        const int kk = kq + j;
        uint64_t val = 0;
        if (j < kFConvK && k0 + kk < K && r < cnt) {
          val = raw[kk * kTN + r];
          if (add) val += raw[kFRawHalf / 8 + kk * kTN + r];
        }
        v[j] = val;
      }
      // kFConvK bytes of each plane: a whole 16-byte core-matrix row, or its half
      uint8_t* yt = smem + kFBOffset + static_cast<size_t>(bs) * kFBStage + core_off(r, kq / 16) + (kq % 16);
#pragma unroll
      for (int i = 0; i < 8; i++) {
        const uint4 pb = plane_bytes(v, i);
        if (kFConvK == 16)
          *reinterpret_cast<uint4*>(yt + i * kPlaneY) = pb;
        else
          *reinterpret_cast<uint2*>(yt + i * kPlaneY) = make_uint2(pb.x, pb.y);
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic writes -> tensor core reads
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(rempty0 + 8 * rs);
        mbar_arrive(bfull0 + 8 * bs);
      }
    }
  }
  bool ok = mbar_wait(done, 0);
  ok = __syncthreads_and(ok ? 1 : 0) != 0 && *err == 0;
  if (!ok) {
    if (t == 0) atomicOr(g.status, kStatusTimeout);
    mbar_wait(done, 0);
  }
  finish_tile(g, smem, tmem, ok, nsteps, warp, lane, t, b, m0, n0);
}

using EncodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                 const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiled encode_tiled() {
  static const EncodeTiled fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return static_cast<EncodeTiled>(nullptr);
    return reinterpret_cast<EncodeTiled>(p);
  }();
  return fn;
}

// B (K x N u64, row-major; per-batch stride ys words, 0 = shared) as a 3-D
// tensor map with 32 x 64-word boxes; false when it cannot be encoded.
bool make_b_map(CUtensorMap* m, const uint64_t* y, size_t ys, int N, int K, int batches) {
  const EncodeTiled enc = encode_tiled();
  if (!enc || !y) return false;
  const cuuint64_t dims[3] = {static_cast<cuuint64_t>(N), static_cast<cuuint64_t>(K),
                              static_cast<cuuint64_t>(ys ? batches : 1)};
  const cuuint64_t strides[2] = {static_cast<cuuint64_t>(N) * 8,
                                 static_cast<cuuint64_t>(ys ? ys : static_cast<size_t>(N) * K) * 8};
  const cuuint32_t box[3] = {static_cast<cuuint32_t>(kTN), static_cast<cuuint32_t>(kTK), 1};
  const cuuint32_t es[3] = {1, 1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT64, 3, const_cast<uint64_t*>(y), dims, strides, box, es,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

constexpr int kMaxSplits = 16;  // cluster size; above 8 needs the non-portable opt-in
constexpr int kMaxDevices = 64;
// Fixed cost of one wave of tiles (prologue, first loads, epilogue) in
// pipeline steps, for choosing the split.
constexpr int kWaveSteps = 6;

// Kernel attributes, once per kernel and device: the dynamic shared memory
// and the non-portable cluster sizes.
cudaError_t prepare_kernel(const void* kernel, int which, int device, uint32_t smem) {
  static std::atomic<int> done[kMaxDevices][2];
  if (device < 0 || device >= kMaxDevices) return cudaErrorInvalidDevice;
  if (done[device][which].load(std::memory_order_acquire)) return cudaSuccess;
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e == cudaSuccess) e = cudaFuncSetAttribute(kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
  if (e == cudaSuccess) done[device][which].store(1, std::memory_order_release);
  return e;
}

// How many clusters of S CTAs of the kernel are resident at once (clusters
// stay inside one GPC, so this is below SMs / S where GPCs do not divide
// evenly); 0 when S does not fit.  Cached per kernel, device and S.
int resident_clusters(const void* kernel, int which, int device, int threads, uint32_t smem, int S) {
  static std::atomic<int> cache[kMaxDevices][2][kMaxSplits + 1];
  const int hit = cache[device][which][S].load(std::memory_order_relaxed);
  if (hit) return hit - 1;
  cudaLaunchConfig_t cfg{};
  cudaLaunchAttribute attr{};
  attr.id = cudaLaunchAttributeClusterDimension;
  attr.val.clusterDim.x = 1;
  attr.val.clusterDim.y = 1;
  attr.val.clusterDim.z = static_cast<unsigned>(S);
  cfg.gridDim = dim3(1, 1, static_cast<unsigned>(S));
  cfg.blockDim = dim3(static_cast<unsigned>(threads));
  cfg.dynamicSmemBytes = smem;
  cfg.attrs = &attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, kernel, &cfg) != cudaSuccess) {
    (void)cudaGetLastError();
    n = 0;
  }
  cache[device][which][S].store(n + 1, std::memory_order_relaxed);
  return n;
}

// The split S (cluster size) with the least estimated time: waves of
// resident clusters x (steps per CTA + a wave's fixed cost), keeping at least
// 4 steps per CTA and every split non-empty.
int choose_splits(const void* kernel, int which, int device, int threads, uint32_t smem, long long tiles, int steps,
                  int batches) {
  int best = 1;
  long long best_cost = -1;
  const int smax = steps / 4 < kMaxSplits ? steps / 4 : kMaxSplits;
  for (int S = 1; S <= (smax > 1 ? smax : 1); S++) {
    const int per = (steps + S - 1) / S;
    if ((steps + per - 1) / per != S) continue;  // normalizes to a smaller S
    if (static_cast<long long>(batches) * S > 65535) break;
    const int rc = resident_clusters(kernel, which, device, threads, smem, S);
    if (rc <= 0) continue;
    const long long waves = (tiles + rc - 1) / rc;
    const long long cost = waves * (per + kWaveSteps);
    if (best_cost < 0 || cost < best_cost) {
      best_cost = cost;
      best = S;
    }
  }
  return best;
}

template <typename... KArgs, typename... Args>
cudaError_t launch_clustered(void (*kernel)(KArgs...), dim3 grid, int threads, uint32_t smem, int S, cudaStream_t st,
                             const Args&... args) {
  cudaLaunchConfig_t cfg{};
  cudaLaunchAttribute attr[2]{};
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = static_cast<unsigned>(S);
  // programmatic dependent of the pre-pass launched just before it
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.gridDim = grid;
  cfg.blockDim = dim3(static_cast<unsigned>(threads));
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, kernel, args...);
}

}  // namespace

cudaError_t launch_ring_gemm_tc(const sufb200_ctx_s* ctx, RingGemmLaunch g, int batches, cudaStream_t st) {
  if (g.npieces < 1 || g.npieces > 2 || g.M < 1 || g.N < 1 || g.K < 1 || batches < 1) return cudaErrorInvalidValue;
  const int tiles_n = (g.N + kTN - 1) / kTN, tiles_m = (g.M + kTM - 1) / kTM;
  g.m_pad = tiles_m * kTM;
  g.n_pad = tiles_n * kTN;
  g.steps = ((g.K + kTK - 1) / kTK) * g.npieces;
  const long long tiles = static_cast<long long>(tiles_n) * tiles_m * batches;
  // X planes per batch when any X piece varies per batch, else one copy; same for Y
  bool x_per_batch = false, y_per_batch = false;
  for (int p = 0; p < g.npieces; p++) {
    x_per_batch |= g.piece[p].xs != 0;
    y_per_batch |= g.piece[p].ys != 0 || (g.piece[p].y2 && g.piece[p].y2s != 0);
  }
  const size_t xbytes = static_cast<size_t>(g.steps) * 8 * g.m_pad * kTK;
  const size_t ybytes = static_cast<size_t>(g.steps) * 8 * g.n_pad * kTK;
  // B split inside the GEMM when its rows can be bulk-copied: row-major,
  // N even (16-byte row starts), 16-byte bases and even per-batch strides
  bool fused = !g.trans && g.N % 2 == 0 && g.N >= kTN && g.K >= kTK;
  for (int p = 0; p < g.npieces; p++) {
    fused = fused && (reinterpret_cast<uintptr_t>(g.piece[p].y) & 15u) == 0 && g.piece[p].ys % 2 == 0;
    if (g.piece[p].y2) fused = fused && (reinterpret_cast<uintptr_t>(g.piece[p].y2) & 15u) == 0 && g.piece[p].y2s % 2 == 0;
  }
  BMaps bm{};
  for (int p = 0; p < g.npieces && fused; p++) {
    fused = make_b_map(&bm.m[2 * p], g.piece[p].y, g.piece[p].ys, g.N, g.K, batches);
    if (fused && g.piece[p].y2) fused = make_b_map(&bm.m[2 * p + 1], g.piece[p].y2, g.piece[p].y2s, g.N, g.K, batches);
  }
  const int xb = x_per_batch ? batches : 1, yb = fused ? 0 : (y_per_batch ? batches : 1);
  g.batches = batches;
  const void* kernel = fused ? reinterpret_cast<const void*>(ring_gemm_tc_fused_kernel)
                             : reinterpret_cast<const void*>(ring_gemm_tc_kernel);
  const int which = fused ? 1 : 0, threads = fused ? kFThreads : kThreads;
  const uint32_t smem = fused ? kFSmemBytes : kSmemBytes;
  cudaError_t e = prepare_kernel(kernel, which, ctx->device, smem);
  if (e != cudaSuccess) return e;
  g.splits = choose_splits(kernel, which, ctx->device, threads, smem, tiles, g.steps, batches);
  uint8_t* scratch = nullptr;
  const size_t xoff = 0, yoff = (xbytes * xb + 255) & ~size_t{255};
  e = cudaMallocFromPoolAsync(reinterpret_cast<void**>(&scratch), yoff + ybytes * yb, ctx->pool, st);
  if (e != cudaSuccess) return e;
  g.xplanes = scratch + xoff;
  g.xps = x_per_batch ? xbytes : 0;
  g.yplanes = scratch + yoff;
  g.yps = y_per_batch ? ybytes : 0;
  // the operands as tiled byte planes
  PlanesSplit px{};
  PlanesSplit py{};
  for (int p = 0; p < g.npieces; p++) {
    px.piece[p] = PlanesPiece{g.piece[p].x, nullptr, g.piece[p].xs, 0};
    py.piece[p] = PlanesPiece{g.piece[p].y, g.piece[p].y2, g.piece[p].ys, g.piece[p].y2s};
  }
  px.R = g.M;
  px.K = g.K;
  px.rows_pad = g.m_pad;
  px.tile_rows = kTM;
  px.steps = g.steps;
  px.k_contig = 1;
  px.dst = scratch + xoff;
  px.ds = xbytes;
  py.R = g.N;
  py.K = g.K;
  py.rows_pad = g.n_pad;
  py.tile_rows = kTN;
  py.steps = g.steps;
  py.k_contig = g.trans ? 1 : 0;
  py.dst = scratch + yoff;
  py.ds = ybytes;
  auto split_blocks = [](const PlanesSplit& q) {
    const size_t units = static_cast<size_t>(q.steps) * 2 * q.rows_pad * 4;
    const size_t want = (units + 255) / 256;
    return static_cast<int>(want < 8192 ? (want ? want : 1) : 8192);
  };
  const int xblocks = split_blocks(px), yblocks = fused ? 0 : split_blocks(py);
  if (e == cudaSuccess) {
    const dim3 sgrid(static_cast<unsigned>(xblocks + yblocks), static_cast<unsigned>(xb > yb ? xb : yb));
    split_planes_kernel<<<sgrid, 256, 0, st>>>(px, py, xblocks, xb, yb);
    e = cudaGetLastError();
  }
  const dim3 grid(static_cast<unsigned>(tiles_n), static_cast<unsigned>(tiles_m),
                  static_cast<unsigned>(batches * g.splits));
  if (e == cudaSuccess) {
    const RingGemmLaunch& gc = g;
    const BMaps& bc = bm;
    e = fused ? launch_clustered(ring_gemm_tc_fused_kernel, grid, kFThreads, kFSmemBytes, g.splits, st, gc, bc)
              : launch_clustered(ring_gemm_tc_kernel, grid, kThreads, kSmemBytes, g.splits, st, gc);
  }
  cudaFreeAsync(scratch, st);
  return e;
}

}  // namespace sufb200
