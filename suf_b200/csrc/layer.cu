// layer.cu -- the glue kernels of the device-resident 2PC transformer layer
// for both parties on one GPU (suf_b200/layer.py drives them; the gates are
// the fused truncation bundles, the coefficient gates and the softmax /
// LayerNorm blocks of the other files).
//
// Each kernel computes every party's share from that party's own material,
// and where the protocol opens a masked value (x^ = x + r_in for the next
// gate, or a Beaver matmul's D = X - A and E = Y - B) the open is the sum of
// the two parties' masked shares, as OpenCollector::flush forms it
// (src/runtime/open_collector.cpp:357-895) when both shares are at hand.
//   * open_masked_pair: x^ = (a0 + r0) + (a1 + r1), the masked input of a
//     truncation or LUT gate after a local product.
//   * beaver_open_pair: per head, both parties' Beaver matmul shares
//     Z_p = C_p + D B_p + A_p E (+ D E for party 0) with D, E opened from the
//     parties' masked operands (nn::matmul_beaver, src/nn/matmul_beaver.cpp,
//     and launch_beaver_matmul2d_kernel, cuda/cuda_primitives.cu:391-628),
//     then the open of the masked result for its truncation: x^ = sum_p
//     (Z_p + r_p).  Strided operands read Q, K, V straight out of the fused
//     QKV rows; a strided output writes heads back into rows.
//   * relu_open_pair / relu_update_pair: one round of the row-max tournament
//     of nn::RowMaxDiffTask (include/nn/row_maxdiff_task.hpp): max(a, b) =
//     b + ReLU(a - b), the ReLU a coefficient gate on the opened difference.
//   * maxdiff_pair: t = max(row) - x per party, the softmax block's input.
//   * add_pair: residual adds, per party.
#include <string>

#include "kernels.hpp"
#include "sufb200_internal.cuh"

namespace {

constexpr int kThreads = 256;
constexpr int kMT = 32;  // output tile of beaver_open_pair_kernel
constexpr int kKT = 16;  // contraction step

int fail(int code, const std::string& msg) { return sufb200::record_error(code, msg); }

int grid_for(size_t n) {
  int dev = 0, sm = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sm, cudaDevAttrMultiProcessorCount, dev);
  const size_t want = (n + kThreads - 1) / kThreads;
  const size_t cap = static_cast<size_t>(sm) * 8;
  return static_cast<int>(want < 1 ? 1 : (want > cap ? cap : want));
}

#define LAYER_GRID_LOOP(i, n) \
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < (n); i += static_cast<size_t>(gridDim.x) * blockDim.x)

__global__ void open_masked_pair_kernel(const uint64_t* __restrict__ a0, const uint64_t* __restrict__ a1, uint64_t r0,
                                        uint64_t r1, uint64_t* __restrict__ xhat, size_t n) {
  sufb200::pdl_trigger();  // a following programmatic launch may start its set-up
  LAYER_GRID_LOOP(i, n) xhat[i] = (a0[i] + r0) + (a1[i] + r1);
}

__global__ void add_pair_kernel(const uint64_t* __restrict__ a0, const uint64_t* __restrict__ b0,
                                const uint64_t* __restrict__ a1, const uint64_t* __restrict__ b1,
                                uint64_t* __restrict__ o0, uint64_t* __restrict__ o1, size_t n) {
  sufb200::pdl_trigger();  // a following programmatic launch may start its set-up
  LAYER_GRID_LOOP(i, n) {
    o0[i] = a0[i] + b0[i];
    o1[i] = a1[i] + b1[i];
  }
}

// Row r of c_p holds w values; pairs (2j, 2j + 1).  x^[r][j] = sum_p
// (c_p[r][2j] - c_p[r][2j+1] + r_p).
__global__ void relu_open_pair_kernel(const uint64_t* __restrict__ c0, const uint64_t* __restrict__ c1, int rows,
                                      int w, uint64_t r0, uint64_t r1, uint64_t* __restrict__ xhat) {
  sufb200::pdl_trigger();  // a following programmatic launch may start its set-up
  const size_t half = static_cast<size_t>(w / 2), n = static_cast<size_t>(rows) * half;
  LAYER_GRID_LOOP(i, n) {
    const size_t r = i / half, j = i % half, at = r * w + 2 * j;
    xhat[i] = (c0[at] - c0[at + 1] + r0) + (c1[at] - c1[at + 1] + r1);
  }
}

// next_p[r][j] = c_p[r][2j+1] + relu_p[r][j]  (= max(c[2j], c[2j+1]) in shares)
__global__ void relu_update_pair_kernel(const uint64_t* __restrict__ c0, const uint64_t* __restrict__ c1,
                                        const uint64_t* __restrict__ relu0, const uint64_t* __restrict__ relu1,
                                        int rows, int w, uint64_t* __restrict__ n0, uint64_t* __restrict__ n1) {
  sufb200::pdl_trigger();  // a following programmatic launch may start its set-up
  const size_t half = static_cast<size_t>(w / 2), n = static_cast<size_t>(rows) * half;
  LAYER_GRID_LOOP(i, n) {
    const size_t r = i / half, j = i % half, at = r * w + 2 * j + 1;
    n0[i] = c0[at] + relu0[i];
    n1[i] = c1[at] + relu1[i];
  }
}

__global__ void maxdiff_pair_kernel(const uint64_t* __restrict__ m0, const uint64_t* __restrict__ m1,
                                    const uint64_t* __restrict__ x0, const uint64_t* __restrict__ x1, int rows,
                                    int cols, uint64_t* __restrict__ t0, uint64_t* __restrict__ t1) {
  sufb200::pdl_trigger();  // a following programmatic launch may start its set-up
  const size_t n = static_cast<size_t>(rows) * cols;
  LAYER_GRID_LOOP(i, n) {
    const size_t r = i / cols;
    t0[i] = m0[r] - x0[i];
    t1[i] = m1[r] - x1[i];
  }
}

struct BeaverPairArgs {
  const uint64_t* x[2];  // left operand shares, element (h, m, k) at x + h*sx + m*ldx + k
  const uint64_t* y[2];  // right operand shares, (h, k, n) at y + h*sy + k*ldy + n (TRANS: n*ldy + k)
  const uint64_t* a[2];  // triple shares A [H][M][K]
  const uint64_t* b[2];  // B [H][K][N] (TRANS: [H][N][K])
  const uint64_t* c[2];  // C = A B, [H][M][N]
  uint64_t r[2];         // the parties' shares of the output's mask
  uint64_t* out;         // x^ (h, m, n) at out + h*so + m*ldo + n
  size_t sx, sy, so;
  int ldx, ldy, ldo, M, K, N;
};

// 32 x 32 output tile per CTA (256 threads, 4 rows each), the contraction in
// steps of 16 staged in shared memory.  The operands' opens D = X - A and
// E = Y - B are formed while staging.  Sums mod 2^64 are order-free.
template <bool TRANS>
__global__ void __launch_bounds__(256) beaver_open_pair_kernel(const BeaverPairArgs p) {
  sufb200::pdl_trigger();  // a following programmatic launch may start its set-up
  __shared__ uint64_t sD[kMT][kKT + 1], sA0[kMT][kKT + 1], sA1[kMT][kKT + 1];
  __shared__ uint64_t sE[kKT][kMT + 1], sB0[kKT][kMT + 1], sB1[kKT][kMT + 1];
  const int h = blockIdx.z;
  const int tx = threadIdx.x, ty = threadIdx.y;
  const int m0 = blockIdx.y * kMT, n0 = blockIdx.x * kMT;
  const int M = p.M, K = p.K, N = p.N;
  const size_t mk = static_cast<size_t>(M) * K, kn = static_cast<size_t>(K) * N, mn = static_cast<size_t>(M) * N;
  const uint64_t *X0 = p.x[0] + h * p.sx, *X1 = p.x[1] + h * p.sx;
  const uint64_t *Y0 = p.y[0] + h * p.sy, *Y1 = p.y[1] + h * p.sy;
  const uint64_t *A0 = p.a[0] + h * mk, *A1 = p.a[1] + h * mk;
  const uint64_t *B0 = p.b[0] + h * kn, *B1 = p.b[1] + h * kn;
  uint64_t z0[4] = {0, 0, 0, 0}, z1[4] = {0, 0, 0, 0};
  for (int k0 = 0; k0 < K; k0 += kKT) {
    for (int e = ty * 32 + tx; e < kMT * kKT; e += 256) {
      const int r = e / kKT, c = e % kKT, m = m0 + r, k = k0 + c;
      uint64_t d = 0, a0 = 0, a1 = 0;
      if (m < M && k < K) {
        const size_t xi = static_cast<size_t>(m) * p.ldx + k, ai = static_cast<size_t>(m) * K + k;
        a0 = A0[ai];
        a1 = A1[ai];
        d = (X0[xi] - a0) + (X1[xi] - a1);
      }
      sD[r][c] = d;
      sA0[r][c] = a0;
      sA1[r][c] = a1;
    }
    for (int e = ty * 32 + tx; e < kKT * kMT; e += 256) {
      const int r = e / kMT, c = e % kMT, k = k0 + r, n = n0 + c;
      uint64_t ev = 0, b0 = 0, b1 = 0;
      if (k < K && n < N) {
        const size_t yi = TRANS ? static_cast<size_t>(n) * p.ldy + k : static_cast<size_t>(k) * p.ldy + n;
        const size_t bi = TRANS ? static_cast<size_t>(n) * K + k : static_cast<size_t>(k) * N + n;
        b0 = B0[bi];
        b1 = B1[bi];
        ev = (Y0[yi] - b0) + (Y1[yi] - b1);
      }
      sE[r][c] = ev;
      sB0[r][c] = b0;
      sB1[r][c] = b1;
    }
    __syncthreads();
#pragma unroll 4
    for (int kk = 0; kk < kKT; kk++) {
      const uint64_t ev = sE[kk][tx], b0 = sB0[kk][tx], b1 = sB1[kk][tx];
#pragma unroll
      for (int q = 0; q < 4; q++) {
        const int r = ty + 8 * q;
        const uint64_t d = sD[r][kk];
        z0[q] += d * b0 + sA0[r][kk] * ev + d * ev;  // party 0 also takes D E
        z1[q] += d * b1 + sA1[r][kk] * ev;
      }
    }
    __syncthreads();
  }
  const int n = n0 + tx;
  if (n >= N) return;
#pragma unroll
  for (int q = 0; q < 4; q++) {
    const int m = m0 + ty + 8 * q;
    if (m >= M) continue;
    const size_t ci = h * mn + static_cast<size_t>(m) * N + n;
    const uint64_t s0 = z0[q] + p.c[0][ci], s1 = z1[q] + p.c[1][ci];
    p.out[h * p.so + static_cast<size_t>(m) * p.ldo + n] = (s0 + p.r[0]) + (s1 + p.r[1]);
  }
}

bool aligned8(const void* q) { return (reinterpret_cast<uintptr_t>(q) & 7u) == 0; }

}  // namespace

extern "C" {

int sufb200_open_masked_pair(const uint64_t* d_a0, const uint64_t* d_a1, uint64_t r0, uint64_t r1, uint64_t* d_xhat,
                             size_t n, void* stream) {
  if (n == 0) return SUFB200_OK;
  if (!d_a0 || !d_a1 || !d_xhat) return fail(SUFB200_ERR_INVALID, "null device pointer");
  open_masked_pair_kernel<<<grid_for(n), kThreads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(d_a0, d_a1, r0, r1,
                                                                                                 d_xhat, n);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? SUFB200_OK : fail(SUFB200_ERR_CUDA, std::string("open_masked_pair: ") + cudaGetErrorString(e));
}

int sufb200_add_pair(const uint64_t* d_a0, const uint64_t* d_b0, const uint64_t* d_a1, const uint64_t* d_b1,
                     uint64_t* d_out0, uint64_t* d_out1, size_t n, void* stream) {
  if (n == 0) return SUFB200_OK;
  if (!d_a0 || !d_b0 || !d_a1 || !d_b1 || !d_out0 || !d_out1) return fail(SUFB200_ERR_INVALID, "null device pointer");
  add_pair_kernel<<<grid_for(n), kThreads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(d_a0, d_b0, d_a1, d_b1,
                                                                                         d_out0, d_out1, n);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? SUFB200_OK : fail(SUFB200_ERR_CUDA, std::string("add_pair: ") + cudaGetErrorString(e));
}

int sufb200_relu_open_pair(const uint64_t* d_c0, const uint64_t* d_c1, int rows, int width, uint64_t r0, uint64_t r1,
                           uint64_t* d_xhat, void* stream) {
  if (rows <= 0) return SUFB200_OK;
  if (width < 2 || (width & 1)) return fail(SUFB200_ERR_INVALID, "relu round: width must be even and >= 2");
  if (!d_c0 || !d_c1 || !d_xhat) return fail(SUFB200_ERR_INVALID, "null device pointer");
  const size_t n = static_cast<size_t>(rows) * (width / 2);
  relu_open_pair_kernel<<<grid_for(n), kThreads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(d_c0, d_c1, rows, width,
                                                                                               r0, r1, d_xhat);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? SUFB200_OK : fail(SUFB200_ERR_CUDA, std::string("relu_open_pair: ") + cudaGetErrorString(e));
}

int sufb200_relu_update_pair(const uint64_t* d_c0, const uint64_t* d_c1, const uint64_t* d_relu0,
                             const uint64_t* d_relu1, int rows, int width, uint64_t* d_next0, uint64_t* d_next1,
                             void* stream) {
  if (rows <= 0) return SUFB200_OK;
  if (width < 2 || (width & 1)) return fail(SUFB200_ERR_INVALID, "relu round: width must be even and >= 2");
  if (!d_c0 || !d_c1 || !d_relu0 || !d_relu1 || !d_next0 || !d_next1)
    return fail(SUFB200_ERR_INVALID, "null device pointer");
  const size_t n = static_cast<size_t>(rows) * (width / 2);
  relu_update_pair_kernel<<<grid_for(n), kThreads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      d_c0, d_c1, d_relu0, d_relu1, rows, width, d_next0, d_next1);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? SUFB200_OK
                          : fail(SUFB200_ERR_CUDA, std::string("relu_update_pair: ") + cudaGetErrorString(e));
}

int sufb200_maxdiff_pair(const uint64_t* d_max0, const uint64_t* d_max1, const uint64_t* d_x0, const uint64_t* d_x1,
                         int rows, int cols, uint64_t* d_t0, uint64_t* d_t1, void* stream) {
  if (rows <= 0 || cols <= 0) return SUFB200_OK;
  if (!d_max0 || !d_max1 || !d_x0 || !d_x1 || !d_t0 || !d_t1) return fail(SUFB200_ERR_INVALID, "null device pointer");
  const size_t n = static_cast<size_t>(rows) * cols;
  maxdiff_pair_kernel<<<grid_for(n), kThreads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(d_max0, d_max1, d_x0,
                                                                                             d_x1, rows, cols, d_t0,
                                                                                             d_t1);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? SUFB200_OK : fail(SUFB200_ERR_CUDA, std::string("maxdiff_pair: ") + cudaGetErrorString(e));
}

int sufb200_beaver_open_pair(const uint64_t* const* d_x, size_t sx, int ldx, const uint64_t* const* d_y, size_t sy,
                             int ldy, int y_transposed, const uint64_t* const* d_a, const uint64_t* const* d_b,
                             const uint64_t* const* d_c, const uint64_t* r, int heads, int M, int K, int N,
                             uint64_t* d_out, size_t so, int ldo, void* stream) {
  if (heads <= 0 || M <= 0 || N <= 0) return SUFB200_OK;
  if (!d_x || !d_y || !d_a || !d_b || !d_c || !r || !d_out || K <= 0)
    return fail(SUFB200_ERR_INVALID, "null pointer or empty contraction");
  if (heads > 65535 || ldx < K || ldo < N || ldy < (y_transposed ? K : N))
    return fail(SUFB200_ERR_INVALID, "beaver_open_pair: bad leading dimension or too many heads");
  BeaverPairArgs a{};
  for (int q = 0; q < 2; q++) {
    if (!d_x[q] || !d_y[q] || !d_a[q] || !d_b[q] || !d_c[q] || !aligned8(d_x[q]) || !aligned8(d_y[q]))
      return fail(SUFB200_ERR_INVALID, "null or misaligned operand");
    a.x[q] = d_x[q];
    a.y[q] = d_y[q];
    a.a[q] = d_a[q];
    a.b[q] = d_b[q];
    a.c[q] = d_c[q];
    a.r[q] = r[q];
  }
  a.out = d_out;
  a.sx = sx;
  a.sy = sy;
  a.so = so;
  a.ldx = ldx;
  a.ldy = ldy;
  a.ldo = ldo;
  a.M = M;
  a.K = K;
  a.N = N;
  const dim3 grid((N + kMT - 1) / kMT, (M + kMT - 1) / kMT, heads), block(32, 8);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (y_transposed)
    beaver_open_pair_kernel<true><<<grid, block, 0, st>>>(a);
  else
    beaver_open_pair_kernel<false><<<grid, block, 0, st>>>(a);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? SUFB200_OK
                          : fail(SUFB200_ERR_CUDA, std::string("beaver_open_pair: ") + cudaGetErrorString(e));
}

}  // extern "C"
