// ring_gemm_tc.cu -- exact Z_2^64 matrix products on the 5th-generation tensor
// cores (tcgen05, kind::i8) by 8-bit limb decomposition.
//
// For u64 operands x = sum_i 2^(8i) x_i and y = sum_j 2^(8j) y_j (bytes),
//   x * y mod 2^64 = sum_{i+j <= 7} 2^(8(i+j)) x_i y_j   (terms with i+j >= 8 vanish).
// A 128 x 64 output tile keeps one int32 accumulator per diagonal s = i + j
// in tensor memory (8 diagonals x 64 columns = all 512 TMEM columns); every
// 32-deep K step issues the 36 unsigned 8-bit MMAs (128 x 64 x 32) of the
// limb pairs into their diagonals, and the epilogue folds
//   acc = sum_s (P_s mod 2^32) << 8s  mod 2^64.
// That is exact as long as P_s is exact wherever bits survive the shift:
// for s <= 3 the diagonal sums stay below 2^31 while K' <= 8192 (P_s <=
// (s+1) K' 255^2), and for s >= 4 only P_s mod 2^(64-8s) | 2^32 matters,
// which the non-saturating accumulator keeps.
//
// Operands are split into byte planes while they are staged into shared
// memory, in the canonical K-major no-swizzle layout of the UMMA shared-memory
// descriptor (8-row x 16-byte core matrices; leading byte offset 128 between
// the two K halves, stride byte offset 256 between 8-row groups), two stages
// deep; one elected thread issues the MMAs and commits each stage to an
// mbarrier that the staging threads wait on (bounded) before reusing it.
//
// Serves the reference's Beaver matmul (cuda/cuda_primitives.cu:391-628,
// out = C + D B + A E (+ D E for party 0) as ONE product [D | A] x [B (+E) ; E])
// and the public-weight matmul (src/nn/matmul_gpu.cu:21-117, Y = X W + bias).
#include "kernels.hpp"
#include "ring_common.cuh"

namespace sufb200 {

namespace {

constexpr int kTM = 128;  // output rows per tile (TMEM lanes)
constexpr int kTN = 64;   // output columns per tile (per diagonal)
constexpr int kTK = 32;   // K per MMA (8-bit operands)
constexpr int kThreads = 128;
constexpr uint32_t kPlaneX = kTM * kTK;             // 4 KB
constexpr uint32_t kPlaneY = kTN * kTK;             // 2 KB
constexpr uint32_t kStageBytes = 8 * (kPlaneX + kPlaneY);  // 48 KB
constexpr uint32_t kCtrlOffset = 2 * kStageBytes;   // mbarriers, TMEM slot
// Requested dynamic shared memory: enough that two CTAs never share an SM,
// so each can own all 512 TMEM columns.
constexpr uint32_t kSmemBytes = 120 * 1024;
constexpr uint32_t kTmemCols = 512;
// idesc for kind::i8: D s32 (bits 4-5 = 2), A and B unsigned 8-bit, both
// K-major, N >> 3 at bits 17-22, M >> 4 at bits 24-28.
constexpr uint32_t kIdesc = (2u << 4) | (uint32_t(kTN >> 3) << 17) | (uint32_t(kTM >> 4) << 24);
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

__device__ __forceinline__ void umma_i8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}"
      :
      : "r"(d_tmem), "l"(adesc), "l"(bdesc), "r"(kIdesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u));
}

__device__ __forceinline__ void umma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, "
      "[%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
        "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Byte i of 16 consecutive words -> 16 bytes of plane i (one row half of a
// core matrix), for all 8 planes.
__device__ __forceinline__ void split_store(const uint64_t (&v)[16], uint32_t base, uint32_t plane_stride) {
#pragma unroll
  for (int i = 0; i < 8; i++) {
    uint32_t w[4];
#pragma unroll
    for (int q = 0; q < 4; q++) {
      const uint32_t a0 = static_cast<uint32_t>(v[4 * q + 0] >> (i < 4 ? 0 : 32));
      const uint32_t a1 = static_cast<uint32_t>(v[4 * q + 1] >> (i < 4 ? 0 : 32));
      const uint32_t a2 = static_cast<uint32_t>(v[4 * q + 2] >> (i < 4 ? 0 : 32));
      const uint32_t a3 = static_cast<uint32_t>(v[4 * q + 3] >> (i < 4 ? 0 : 32));
      const uint32_t sel = static_cast<uint32_t>(i & 3) | (static_cast<uint32_t>(4 + (i & 3)) << 4);
      const uint32_t t01 = __byte_perm(a0, a1, sel);
      const uint32_t t23 = __byte_perm(a2, a3, sel);
      w[q] = __byte_perm(t01, t23, 0x5410);
    }
    asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(base + static_cast<uint32_t>(i) * plane_stride),
                 "r"(w[0]), "r"(w[1]), "r"(w[2]), "r"(w[3])
                 : "memory");
  }
}

// Shared-memory offset of (row r, K half h) inside a plane.
__device__ __forceinline__ uint32_t core_off(int r, int h) {
  return static_cast<uint32_t>((r >> 3) * 256 + h * 128 + (r & 7) * 16);
}

template <bool TRANS>
__global__ void __launch_bounds__(kThreads, 1) ring_gemm_tc_kernel(const RingGemmLaunch g) {
  extern __shared__ __align__(1024) uint8_t smem[];
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  const int b = blockIdx.z;
  const int m0 = blockIdx.y * kTM, n0 = blockIdx.x * kTN;
  const int M = g.M, N = g.N, K = g.K;
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bar0 = sbase + kCtrlOffset, bar1 = bar0 + 8, slot = bar0 + 16;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kCtrlOffset + 16);

  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(slot), "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  if (t == 0) {
    mbar_init(bar0, 1);
    mbar_init(bar1, 1);
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;

  const int cpp = (K + kTK - 1) / kTK;  // K steps per piece
  const int steps = cpp * g.npieces;
  bool ok = true;
  for (int c = 0; c < steps; c++) {
    const int st = c & 1;
    // stage st was last read by the MMAs of step c - 2
    const bool free_ok = c < 2 || mbar_wait(st ? bar1 : bar0, static_cast<uint32_t>(((c >> 1) - 1) & 1));
    const RingGemmPiece& P = g.piece[c / cpp];
    const int kc = (c % cpp) * kTK;
    const uint32_t xs = sbase + static_cast<uint32_t>(st) * kStageBytes;
    const uint32_t ys = xs + 8 * kPlaneX;
    const uint64_t* X = P.x + static_cast<size_t>(b) * P.xs;
    const bool x_vec = (K & 1) == 0 && (reinterpret_cast<uintptr_t>(X) & 15u) == 0;  // 16-byte row loads
    // X tile: unit (row r = t, K half h), 16 words each
#pragma unroll 1
    for (int h = 0; h < 2; h++) {
      const int m = m0 + t, k = kc + 16 * h;
      uint64_t v[16];
      if (m < M && k + 16 <= K && x_vec) {
        const ulonglong2* src = reinterpret_cast<const ulonglong2*>(X + static_cast<size_t>(m) * K + k);
#pragma unroll
        for (int j = 0; j < 8; j++) {
          const ulonglong2 q = __ldg(src + j);
          v[2 * j] = q.x;
          v[2 * j + 1] = q.y;
        }
      } else {
#pragma unroll
        for (int j = 0; j < 16; j++) v[j] = (m < M && k + j < K) ? __ldg(X + static_cast<size_t>(m) * K + k + j) : 0ull;
      }
      split_store(v, xs + core_off(t, h), kPlaneX);
    }
    // Y tile: unit (row r = n, K half h)
    {
      const int r = t & 63, h = t >> 6;  // lanes on consecutive rows: coalesced, conflict-free
      const int n = n0 + r, k = kc + 16 * h;
      const uint64_t* Y = P.y + static_cast<size_t>(b) * P.ys;
      const uint64_t* Y2 = P.y2 ? P.y2 + static_cast<size_t>(b) * P.y2s : nullptr;
      uint64_t v[16];
#pragma unroll
      for (int j = 0; j < 16; j++) {
        const int kk = k + j;
        uint64_t val = 0;
        if (n < N && kk < K) {
          const size_t idx = TRANS ? static_cast<size_t>(n) * K + kk : static_cast<size_t>(kk) * N + n;
          val = __ldg(Y + idx);
          if (Y2) val += __ldg(Y2 + idx);
        }
        v[j] = val;
      }
      split_store(v, ys + core_off(r, h), kPlaneY);
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    ok = __syncthreads_and(free_ok ? 1 : 0) != 0;  // one verdict for the whole block
    if (!ok) break;
    if (t == 0) {
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
#pragma unroll
      for (int i = 0; i < 8; i++) {
        const uint64_t ad = umma_desc(xs + static_cast<uint32_t>(i) * kPlaneX);
#pragma unroll
        for (int j = 0; j + i < 8; j++) {
          const uint64_t bd = umma_desc(ys + static_cast<uint32_t>(j) * kPlaneY);
          umma_i8(tmem + static_cast<uint32_t>((i + j) * kTN), ad, bd, (c > 0 || i > 0) ? 1u : 0u);
        }
      }
      umma_commit(st ? bar1 : bar0);
    }
  }
  // every MMA issued so far has completed once the last commit arrives
  if (ok && steps > 0) {
    const int last = steps - 1;
    ok = __syncthreads_and(mbar_wait((last & 1) ? bar1 : bar0, static_cast<uint32_t>((last >> 1) & 1)) ? 1 : 0) != 0;
  }
  if (!ok) {
    if (t == 0) atomicOr(g.status, kStatusTimeout);
    // let whatever was issued drain before the columns are released
    if (steps > 0) {
      const int last = steps - 1;
      mbar_wait((last & 1) ? bar1 : bar0, static_cast<uint32_t>((last >> 1) & 1));
    }
  } else {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const int m = m0 + warp * 32 + lane;
    const uint64_t* C = g.c ? g.c + static_cast<size_t>(b) * g.cs : nullptr;
    uint64_t* O = g.out + static_cast<size_t>(b) * g.os;
#pragma unroll 1
    for (int cb = 0; cb < kTN / 16; cb++) {
      uint64_t acc[16];
#pragma unroll
      for (int j = 0; j < 16; j++) acc[j] = 0;
#pragma unroll
      for (int s = 0; s < 8; s++) {
        uint32_t v[16];
        tmem_ld16(tmem + (static_cast<uint32_t>(warp * 32) << 16) + static_cast<uint32_t>(s * kTN + cb * 16), v);
#pragma unroll
        for (int j = 0; j < 16; j++) acc[j] += static_cast<uint64_t>(v[j]) << (8 * s);
      }
      if (m < M) {
#pragma unroll
        for (int j = 0; j < 16; j++) {
          const int n = n0 + cb * 16 + j;
          if (n < N) {
            const size_t o = static_cast<size_t>(m) * N + n;
            uint64_t val = acc[j];
            if (C) val += C[o];
            if (g.bias) val += static_cast<uint64_t>(g.bias[n]);
            O[o] = scaled_acc(val, g.has_scale, g.mul_const, g.mul_shift);
          }
        }
      }
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 0) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
  }
}

}  // namespace

cudaError_t launch_ring_gemm_tc(const RingGemmLaunch& g, int batches, cudaStream_t st) {
  if (g.npieces < 1 || g.npieces > 2 || g.M < 1 || g.N < 1 || g.K < 1 || batches < 1) return cudaErrorInvalidValue;
  const dim3 grid(static_cast<unsigned>((g.N + kTN - 1) / kTN), static_cast<unsigned>((g.M + kTM - 1) / kTM),
                  static_cast<unsigned>(batches));
  cudaError_t e;
  if (g.trans) {
    e = cudaFuncSetAttribute(ring_gemm_tc_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
    if (e != cudaSuccess) return e;
    ring_gemm_tc_kernel<true><<<grid, kThreads, kSmemBytes, st>>>(g);
  } else {
    e = cudaFuncSetAttribute(ring_gemm_tc_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
    if (e != cudaSuccess) return e;
    ring_gemm_tc_kernel<false><<<grid, kThreads, kSmemBytes, st>>>(g);
  }
  return cudaGetLastError();
}

}  // namespace sufb200
