// primitives.cu -- elementwise and per-row ring kernels (HBM-bound).
//
// Z_2^64 arithmetic of include/runtime/cuda_primitives.hpp:9-240: Beaver
// multiplication, Horner, truncation postproc, r_out masking, row sums and
// variances, eff-bits packing and the open (unpack + add) step.  Grids are
// sized to a whole number of waves over the SMs with grid-stride loops;
// row reductions use one warp-shuffle tree per row segment.
#include "ring_common.cuh"
#include "kernels.hpp"
#include "primitives.hpp"

namespace sufb200 {

namespace {

constexpr int kThreads = 256;

__device__ __forceinline__ uint64_t mask_low(int bits) {
  return bits <= 0 ? 0ull : (bits >= 64 ? ~0ull : ((1ull << bits) - 1ull));
}

#define SUFB200_GRID_LOOP(i, n)                                                                  \
  for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < (n); \
       i += static_cast<size_t>(gridDim.x) * blockDim.x)

__global__ void beaver_mul_kernel(int party, const uint64_t* __restrict__ a, const uint64_t* __restrict__ b,
                                  const uint64_t* __restrict__ c, const uint64_t* __restrict__ d,
                                  const uint64_t* __restrict__ e, uint64_t* __restrict__ z, size_t n) {
  SUFB200_GRID_LOOP(i, n) {
    const uint64_t dv = d[i], ev = e[i];
    uint64_t v = c[i] + dv * b[i] + ev * a[i];
    if (party == 0) v += dv * ev;
    z[i] = v;
  }
}

__global__ void beaver_mul_aos_kernel(int party, const uint64_t* __restrict__ tri, const uint64_t* __restrict__ d,
                                      const uint64_t* __restrict__ e, uint64_t* __restrict__ z, size_t n) {
  SUFB200_GRID_LOOP(i, n) {
    const uint64_t dv = d[i], ev = e[i];
    uint64_t v = tri[3 * i + 2] + dv * tri[3 * i + 1] + ev * tri[3 * i];
    if (party == 0) v += dv * ev;
    z[i] = v;
  }
}

__global__ void horner_cubic_kernel(const uint64_t* __restrict__ x, const uint64_t* __restrict__ c0,
                                    const uint64_t* __restrict__ c1, const uint64_t* __restrict__ c2,
                                    const uint64_t* __restrict__ c3, uint64_t* __restrict__ out, size_t n) {
  SUFB200_GRID_LOOP(i, n) {
    const uint64_t xv = x[i];
    out[i] = ((c3[i] * xv + c2[i]) * xv + c1[i]) * xv + c0[i];
  }
}

struct PostprocArgs {
  int party, kind_gapars, f;
  uint64_t r_hi, m;
  const uint64_t* hatx;
  const uint64_t* arith;
  size_t arith_stride;
  int arith_idx;
  const uint64_t* bools;
  size_t bool_stride;
  int carry_idx, sign_idx, wrap_idx;
  uint64_t* out;
  size_t n;
};

// launch_trunc_postproc_kernel semantics (cuda/cuda_primitives.cu:179-252).
__global__ void trunc_postproc_kernel(const PostprocArgs p) {
  SUFB200_GRID_LOOP(i, p.n) {
    const uint64_t base = p.arith[static_cast<size_t>(p.arith_idx) + i * p.arith_stride];
    const bool hc = p.bools && p.carry_idx >= 0 && p.carry_idx < static_cast<int>(p.bool_stride);
    const bool hs = p.bools && p.sign_idx >= 0 && p.sign_idx < static_cast<int>(p.bool_stride);
    const bool hw = p.bools && p.wrap_idx >= 0 && p.wrap_idx < static_cast<int>(p.bool_stride);
    const uint64_t carry = hc ? p.bools[static_cast<size_t>(p.carry_idx) + i * p.bool_stride] : 0ull;
    const uint64_t sign = hs ? p.bools[static_cast<size_t>(p.sign_idx) + i * p.bool_stride] : 0ull;
    const uint64_t wrap = hw ? p.bools[static_cast<size_t>(p.wrap_idx) + i * p.bool_stride] : 0ull;
    uint64_t y = base;
    const int f = p.f;
    if (p.kind_gapars) {
      const uint64_t hb = (p.hatx ? p.hatx[i] : 0ull) + (1ull << 62);
      uint64_t top = 0;
      if (p.party == 0) top = f <= 0 ? hb : (f >= 64 ? 0ull : (hb >> f));
      y = y + top - p.r_hi - carry;
      if (f > 0 && f < 64 && ((hb >> 63) & 1ull) == 0) y += p.m;
      if (p.party == 0 && f >= 0 && f <= 62) y -= 1ull << (62 - f);
    } else {
      if (p.party == 0 && f > 0 && f < 64) y += p.hatx ? (p.hatx[i] >> f) : 0ull;
      y = y - p.r_hi - carry;
      if (f > 0 && f < 64) {
        y += wrap * (1ull << (64 - f));
        y += sign * (~0ull << (64 - f));
      }
    }
    p.out[i] = y;
  }
}

struct Rout8 {
  uint64_t r[8];
};

__global__ void add_rout_aos_kernel(uint64_t* __restrict__ out, size_t words, int out_words, int rout_words,
                                    const Rout8 r) {
  SUFB200_GRID_LOOP(i, words) {
    const int j = static_cast<int>(i % static_cast<size_t>(out_words));
    if (j < rout_words) out[i] += r.r[j];
  }
}

__device__ __forceinline__ uint64_t warp_sum(uint64_t v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
  return v;
}

// One CTA per row; sum over [0, len) of row r, then the CTA reduction.
template <bool VAR>
__global__ void row_reduce_kernel(const uint64_t* __restrict__ mat, const uint64_t* __restrict__ mean, int rows,
                                  int cols, const int* __restrict__ valid, uint64_t* __restrict__ out) {
  __shared__ uint64_t part[kThreads / 32];
  for (int r = blockIdx.x; r < rows; r += gridDim.x) {
    int len = valid ? valid[r] : cols;
    if (len > cols) len = cols;
    if (len < 0) len = 0;
    const uint64_t* row = mat + static_cast<size_t>(r) * static_cast<size_t>(cols);
    const uint64_t mu = VAR ? mean[r] : 0ull;
    uint64_t acc = 0;
    for (int c = threadIdx.x; c < len; c += blockDim.x) {
      const uint64_t x = row[c];
      if (VAR) {
        const uint64_t dlt = x - mu;
        acc += dlt * dlt;
      } else {
        acc += x;
      }
    }
    acc = warp_sum(acc);
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = acc;
    __syncthreads();
    if (threadIdx.x < 32) {
      uint64_t v = threadIdx.x < (blockDim.x >> 5) ? part[threadIdx.x] : 0ull;
      v = warp_sum(v);
      if (threadIdx.x == 0) out[r] = v;
    }
    __syncthreads();
  }
}

__global__ void row_sum_ragged_kernel(const uint64_t* __restrict__ vals, const int* __restrict__ offs, int rows,
                                      uint64_t* __restrict__ out) {
  __shared__ uint64_t part[kThreads / 32];
  for (int r = blockIdx.x; r < rows; r += gridDim.x) {
    int start = offs[r], end = offs[r + 1];
    if (start < 0) start = 0;
    if (end < start) end = start;
    uint64_t acc = 0;
    for (int i = start + threadIdx.x; i < end; i += blockDim.x) acc += vals[i];
    acc = warp_sum(acc);
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = acc;
    __syncthreads();
    if (threadIdx.x < 32) {
      uint64_t v = threadIdx.x < (blockDim.x >> 5) ? part[threadIdx.x] : 0ull;
      v = warp_sum(v);
      if (threadIdx.x == 0) out[r] = v;
    }
    __syncthreads();
  }
}

__global__ void row_broadcast_mul_kernel(int party, const uint64_t* __restrict__ A, const uint64_t* __restrict__ B,
                                         const uint64_t* __restrict__ C, const uint64_t* __restrict__ d,
                                         const uint64_t* __restrict__ e, int rows, int cols,
                                         const int* __restrict__ valid, uint64_t* __restrict__ out) {
  const size_t n = static_cast<size_t>(rows) * static_cast<size_t>(cols);
  SUFB200_GRID_LOOP(i, n) {
    const int r = static_cast<int>(i / static_cast<size_t>(cols));
    const int c = static_cast<int>(i - static_cast<size_t>(r) * cols);
    if (valid && c >= valid[r]) {
      out[i] = 0;
      continue;
    }
    const uint64_t dv = d[i], ev = e[r];
    uint64_t z = C[i] + dv * B[r] + ev * A[i];
    if (party == 0) z += dv * ev;
    out[i] = z;
  }
}

// One thread per packed output word (no atomics).
__global__ void pack_eff_bits_kernel(const uint64_t* __restrict__ in, int b, uint64_t* __restrict__ packed, size_t n,
                                     size_t words) {
  const uint64_t m = mask_low(b);
  SUFB200_GRID_LOOP(w, words) {
    const uint64_t bit0 = static_cast<uint64_t>(w) * 64ull;
    size_t idx = static_cast<size_t>(bit0 / static_cast<uint64_t>(b));
    uint64_t word = 0;
    int filled = 0;
    int off = static_cast<int>(bit0 - static_cast<uint64_t>(idx) * static_cast<uint64_t>(b));
    while (filled < 64 && idx < n) {
      const uint64_t v = (in[idx] & m) >> off;
      int avail = b - off;
      if (avail > 64 - filled) avail = 64 - filled;
      const uint64_t take = avail >= 64 ? ~0ull : ((1ull << avail) - 1ull);
      word |= (v & take) << filled;
      filled += avail;
      off = 0;
      idx++;
    }
    packed[w] = word;
  }
}

__device__ __forceinline__ uint64_t unpack_one(const uint64_t* __restrict__ packed, size_t words, int b, size_t i) {
  const size_t bit = i * static_cast<size_t>(b);
  const size_t w = bit >> 6;
  const int off = static_cast<int>(bit & 63);
  const uint64_t lo = w < words ? packed[w] : 0ull;
  const uint64_t hi = (off && w + 1 < words) ? packed[w + 1] : 0ull;
  const uint64_t v = off ? ((lo >> off) | (hi << (64 - off))) : lo;
  return v & mask_low(b);
}

__global__ void unpack_eff_bits_kernel(const uint64_t* __restrict__ packed, int b, uint64_t* __restrict__ out,
                                       size_t n, size_t words) {
  SUFB200_GRID_LOOP(i, n) out[i] = unpack_one(packed, words, b, i);
}

__global__ void unpack_add_mod_kernel(const uint64_t* __restrict__ local, const uint64_t* __restrict__ packed, int b,
                                      uint64_t* __restrict__ out, size_t n, size_t words, uint64_t ring_mask) {
  SUFB200_GRID_LOOP(i, n) out[i] = (local[i] + unpack_one(packed, words, b, i)) & ring_mask;
}

int grid_for(int sm_count, size_t n) {
  const size_t want = (n + kThreads - 1) / kThreads;
  const size_t cap = static_cast<size_t>(sm_count) * 8;
  return static_cast<int>(want < cap ? (want ? want : 1) : cap);
}

}  // namespace

cudaError_t prim_beaver_mul(int sm, int party, const uint64_t* a, const uint64_t* b, const uint64_t* c,
                            const uint64_t* d, const uint64_t* e, uint64_t* z, size_t n, cudaStream_t st) {
  beaver_mul_kernel<<<grid_for(sm, n), kThreads, 0, st>>>(party, a, b, c, d, e, z, n);
  return cudaGetLastError();
}

cudaError_t prim_beaver_mul_aos(int sm, int party, const uint64_t* tri, const uint64_t* d, const uint64_t* e,
                                uint64_t* z, size_t n, cudaStream_t st) {
  beaver_mul_aos_kernel<<<grid_for(sm, n), kThreads, 0, st>>>(party, tri, d, e, z, n);
  return cudaGetLastError();
}

cudaError_t prim_horner_cubic(int sm, const uint64_t* x, const uint64_t* c0, const uint64_t* c1, const uint64_t* c2,
                              const uint64_t* c3, uint64_t* out, size_t n, cudaStream_t st) {
  horner_cubic_kernel<<<grid_for(sm, n), kThreads, 0, st>>>(x, c0, c1, c2, c3, out, n);
  return cudaGetLastError();
}

cudaError_t prim_trunc_postproc(int sm, int party, int kind_gapars, int f, uint64_t r_hi, uint64_t m,
                                const uint64_t* hatx, const uint64_t* arith, size_t arith_stride, int arith_idx,
                                const uint64_t* bools, size_t bool_stride, int carry_idx, int sign_idx, int wrap_idx,
                                uint64_t* out, size_t n, cudaStream_t st) {
  PostprocArgs p{party, kind_gapars, f, r_hi, m, hatx, arith, arith_stride, arith_idx, bools, bool_stride,
                 carry_idx, sign_idx, wrap_idx, out, n};
  trunc_postproc_kernel<<<grid_for(sm, n), kThreads, 0, st>>>(p);
  return cudaGetLastError();
}

cudaError_t prim_add_rout_aos(int sm, uint64_t* out, size_t elems, int out_words, const uint64_t* r_out,
                              size_t r_out_words, cudaStream_t st) {
  Rout8 r{};
  const int rw = static_cast<int>(r_out_words < 8 ? r_out_words : 8);
  for (int j = 0; j < rw; j++) r.r[j] = r_out[j];
  const size_t words = elems * static_cast<size_t>(out_words);
  add_rout_aos_kernel<<<grid_for(sm, words), kThreads, 0, st>>>(out, words, out_words, rw, r);
  return cudaGetLastError();
}

cudaError_t prim_row_sum(int sm, const uint64_t* mat, int rows, int cols, const int* valid, uint64_t* out,
                         cudaStream_t st) {
  const int grid = rows < sm * 8 ? rows : sm * 8;
  row_reduce_kernel<false><<<grid, kThreads, 0, st>>>(mat, nullptr, rows, cols, valid, out);
  return cudaGetLastError();
}

cudaError_t prim_row_variance(int sm, const uint64_t* mat, const uint64_t* mean, int rows, int cols, const int* valid,
                              uint64_t* out, cudaStream_t st) {
  const int grid = rows < sm * 8 ? rows : sm * 8;
  row_reduce_kernel<true><<<grid, kThreads, 0, st>>>(mat, mean, rows, cols, valid, out);
  return cudaGetLastError();
}

cudaError_t prim_row_sum_ragged(int sm, const uint64_t* vals, const int* offs, int rows, uint64_t* out,
                                cudaStream_t st) {
  const int grid = rows < sm * 8 ? rows : sm * 8;
  row_sum_ragged_kernel<<<grid, kThreads, 0, st>>>(vals, offs, rows, out);
  return cudaGetLastError();
}

cudaError_t prim_row_broadcast_mul(int sm, int party, const uint64_t* A, const uint64_t* B, const uint64_t* C,
                                   const uint64_t* d, const uint64_t* e, int rows, int cols, const int* valid,
                                   uint64_t* out, cudaStream_t st) {
  const size_t n = static_cast<size_t>(rows) * static_cast<size_t>(cols);
  row_broadcast_mul_kernel<<<grid_for(sm, n), kThreads, 0, st>>>(party, A, B, C, d, e, rows, cols, valid, out);
  return cudaGetLastError();
}

size_t packed_word_count(size_t n, int b) {
  return static_cast<size_t>((static_cast<unsigned __int128>(n) * static_cast<unsigned>(b) + 63) / 64);
}

cudaError_t prim_pack_eff_bits(int sm, const uint64_t* in, int b, uint64_t* packed, size_t n, cudaStream_t st) {
  const size_t words = packed_word_count(n, b);
  pack_eff_bits_kernel<<<grid_for(sm, words), kThreads, 0, st>>>(in, b, packed, n, words);
  return cudaGetLastError();
}

cudaError_t prim_unpack_eff_bits(int sm, const uint64_t* packed, int b, uint64_t* out, size_t n, cudaStream_t st) {
  unpack_eff_bits_kernel<<<grid_for(sm, n), kThreads, 0, st>>>(packed, b, out, n, packed_word_count(n, b));
  return cudaGetLastError();
}

cudaError_t prim_unpack_add_mod(int sm, const uint64_t* local, const uint64_t* packed, int b, uint64_t* out, size_t n,
                                int ring_bits, cudaStream_t st) {
  const uint64_t rm = ring_bits >= 64 ? ~0ull : ((1ull << ring_bits) - 1ull);
  unpack_add_mod_kernel<<<grid_for(sm, n), kThreads, 0, st>>>(local, packed, b, out, n, packed_word_count(n, b), rm);
  return cudaGetLastError();
}

}  // namespace sufb200

// ---- Beaver matmul, row mean, signed opens, shift (cuda_primitives.hpp:130-240) ----

namespace sufb200 {

namespace {

constexpr int kMT = 32, kKT = 16;

// out = C + D*B + A*E (+ D*E on party 0), mod 2^64, per batch b (D, E and out
// per batch; the triple A, B, C shared), 32 x 32 output tile per CTA, K in
// steps of 16 staged in shared memory.  Sums mod 2^64 are order-free, so the
// tiling is bit-exact with the reference's per-element loop.
template <bool TRANS>
__global__ void __launch_bounds__(256) beaver_matmul_kernel(int party, const uint64_t* __restrict__ D,
                                                            const uint64_t* __restrict__ E,
                                                            const uint64_t* __restrict__ A,
                                                            const uint64_t* __restrict__ B,
                                                            const uint64_t* __restrict__ C, int M, int K, int N,
                                                            int has_scale, int64_t mul_const, int mul_shift,
                                                            uint64_t* __restrict__ out) {
  __shared__ uint64_t sD[kMT][kKT + 1], sA[kMT][kKT + 1], sE[kKT][kMT + 1], sB[kKT][kMT + 1];
  const int b = blockIdx.z;
  const size_t mk = static_cast<size_t>(M) * K, kn = static_cast<size_t>(K) * N, mn = static_cast<size_t>(M) * N;
  const uint64_t* Db = D + b * mk;
  const uint64_t* Eb = E + b * kn;
  const int tx = threadIdx.x, ty = threadIdx.y;  // 32 x 8
  const int m0 = blockIdx.y * kMT, n0 = blockIdx.x * kMT;
  uint64_t acc[4] = {0, 0, 0, 0};
  for (int k0 = 0; k0 < K; k0 += kKT) {
    for (int e = ty * 32 + tx; e < kMT * kKT; e += 256) {
      const int r = e / kKT, c = e % kKT;
      const int m = m0 + r, k = k0 + c;
      const bool ok = m < M && k < K;
      sD[r][c] = ok ? Db[static_cast<size_t>(m) * K + k] : 0ull;
      sA[r][c] = ok ? A[static_cast<size_t>(m) * K + k] : 0ull;
    }
    for (int e = ty * 32 + tx; e < kKT * kMT; e += 256) {
      const int r = e / kMT, c = e % kMT;
      const int k = k0 + r, n = n0 + c;
      const bool ok = k < K && n < N;
      const size_t bi = TRANS ? static_cast<size_t>(n) * K + k : static_cast<size_t>(k) * N + n;
      sE[r][c] = ok ? Eb[bi] : 0ull;
      sB[r][c] = ok ? B[bi] : 0ull;
    }
    __syncthreads();
#pragma unroll 4
    for (int kk = 0; kk < kKT; kk++) {
      const uint64_t e = sE[kk][tx], bb = sB[kk][tx];
#pragma unroll
      for (int r = 0; r < 4; r++) {
        const uint64_t d = sD[ty + 8 * r][kk];
        acc[r] += d * bb + sA[ty + 8 * r][kk] * e + (party == 0 ? d * e : 0ull);
      }
    }
    __syncthreads();
  }
  const int n = n0 + tx;
#pragma unroll
  for (int r = 0; r < 4; r++) {
    const int m = m0 + ty + 8 * r;
    if (m < M && n < N) {
      const size_t o = static_cast<size_t>(m) * N + n;
      out[b * mn + o] = scaled_acc(C[o] + acc[r], has_scale, mul_const, mul_shift);
    }
  }
}

__global__ void row_mean_kernel(const uint64_t* __restrict__ mat, int rows, int cols, const int* __restrict__ valid,
                                uint64_t* __restrict__ out) {
  __shared__ uint64_t part[kThreads / 32];
  for (int r = blockIdx.x; r < rows; r += gridDim.x) {
    int len = valid ? valid[r] : cols;
    if (len > cols) len = cols;
    const uint64_t* row = mat + static_cast<size_t>(r) * static_cast<size_t>(cols);
    uint64_t acc = 0;
    for (int c = threadIdx.x; c < len; c += blockDim.x) acc += row[c];
    acc = warp_sum(acc);
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = acc;
    __syncthreads();
    if (threadIdx.x < 32) {
      uint64_t v = threadIdx.x < (blockDim.x >> 5) ? part[threadIdx.x] : 0ull;
      v = warp_sum(v);
      if (threadIdx.x == 0) out[r] = len > 0 ? v / static_cast<uint64_t>(len) : 0ull;
    }
    __syncthreads();
  }
}

__device__ __forceinline__ uint64_t to_signed_ring(uint64_t v, int ring_bits) {
  if (ring_bits >= 64) return v;
  const uint64_t m = (1ull << ring_bits) - 1ull;
  v &= m;
  if (v & (1ull << (ring_bits - 1))) v |= ~m;
  return v;
}

__global__ void open_add_to_signed_kernel(const uint64_t* __restrict__ local, const uint64_t* __restrict__ remote,
                                          uint64_t* __restrict__ out, size_t n, int ring_bits) {
  SUFB200_GRID_LOOP(i, n) out[i] = to_signed_ring(local[i] + remote[i], ring_bits);
}

__global__ void unpack_add_to_signed_kernel(const uint64_t* __restrict__ local, const uint64_t* __restrict__ packed,
                                            int b, uint64_t* __restrict__ out, size_t n, size_t words, int ring_bits) {
  SUFB200_GRID_LOOP(i, n) out[i] = to_signed_ring(local[i] + unpack_one(packed, words, b, i), ring_bits);
}

__global__ void trunc_shift_kernel(const uint64_t* __restrict__ in, uint64_t* __restrict__ out, int f, size_t n) {
  SUFB200_GRID_LOOP(i, n) out[i] = f <= 0 ? in[i] : (f >= 64 ? 0ull : (in[i] >> f));
}

}  // namespace

cudaError_t prim_beaver_matmul(int party, const uint64_t* D, const uint64_t* E, const uint64_t* A, const uint64_t* B,
                               const uint64_t* C, int batches, int M, int K, int N, int w_transposed, int has_scale,
                               int64_t mul_const, int mul_shift, uint64_t* out, cudaStream_t st) {
  const dim3 grid((N + kMT - 1) / kMT, (M + kMT - 1) / kMT, batches), block(32, 8);
  if (w_transposed)
    beaver_matmul_kernel<true><<<grid, block, 0, st>>>(party, D, E, A, B, C, M, K, N, has_scale, mul_const, mul_shift,
                                                       out);
  else
    beaver_matmul_kernel<false><<<grid, block, 0, st>>>(party, D, E, A, B, C, M, K, N, has_scale, mul_const,
                                                        mul_shift, out);
  return cudaGetLastError();
}

cudaError_t prim_row_mean(int sm, const uint64_t* mat, int rows, int cols, const int* valid, uint64_t* out,
                          cudaStream_t st) {
  const int grid = rows < sm * 8 ? rows : sm * 8;
  row_mean_kernel<<<grid, kThreads, 0, st>>>(mat, rows, cols, valid, out);
  return cudaGetLastError();
}

cudaError_t prim_open_add_to_signed(int sm, const uint64_t* local, const uint64_t* remote, uint64_t* out, size_t n,
                                    int ring_bits, cudaStream_t st) {
  open_add_to_signed_kernel<<<grid_for(sm, n), kThreads, 0, st>>>(local, remote, out, n, ring_bits);
  return cudaGetLastError();
}

cudaError_t prim_unpack_add_to_signed(int sm, const uint64_t* local, const uint64_t* packed, int b, uint64_t* out,
                                      size_t n, int ring_bits, cudaStream_t st) {
  unpack_add_to_signed_kernel<<<grid_for(sm, n), kThreads, 0, st>>>(local, packed, b, out, n,
                                                                      packed_word_count(n, b), ring_bits);
  return cudaGetLastError();
}

cudaError_t prim_trunc_shift(int sm, const uint64_t* in, uint64_t* out, int f, size_t n, cudaStream_t st) {
  trunc_shift_kernel<<<grid_for(sm, n), kThreads, 0, st>>>(in, out, f, n);
  return cudaGetLastError();
}

}  // namespace sufb200
