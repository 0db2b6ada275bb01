// layernorm_block.cu -- the configs[4] LayerNorm block (runtime::LayerNormTask
// with RsqrtTask, include/runtime/phase_tasks.hpp:1383-1700, 2186-2600) for
// both parties on one GPU, every open computed on the device.
//
// On shares, in Z_2^64 (T_k = signed floor shift by a truncation bundle):
//   mu = T_f(sum_row(x) invL)                   d = x - mu
//   v  = T_2f(sum_row(d d) invL) + eps          (d d: Beaver squares)
//   c0, c1 = LUT_rsqrt(open(v + r))             y = c0 + T_f(c1 v)
//   y2 = T_f(y y)   g = T_f(v y2)   h = T_1(g)  t = 3 2^(f-1) - h
//   y  = T_f(y t)                               (one Newton step of RsqrtTask)
//   out = T_f(d y[row])                         (MulRowBroadcastTask + TruncTask)
// The reference's RsqrtTask computes its initial guess c0 + (c1 x >> f)
// from the opened input and each party's coefficient shares, and halves
// x y^2 by shifting each share; on additive shares both need the secure
// forms above (a Beaver product with a truncation, a 1-bit truncation),
// which compute the same fixed-point function.
//
// As in softmax_block.cu, both parties' shares are on this GPU, so an open
// is a sum; each kernel ends by writing the masked value the next truncation
// bundle takes.  Row-level stages (rows values) use the one-launch pair
// truncation; the element-level ones the shared-prefix path.
#include <string>

#include "kernels.hpp"
#include "sufb200_internal.cuh"

namespace sufb200 {
namespace {

constexpr int kThreads = 256;
constexpr int kRowThreads = 256;

struct Prod {
  uint64_t z0, z1;
};

__device__ __forceinline__ Prod beaver(uint64_t x0, uint64_t x1, uint64_t y0, uint64_t y1, const uint64_t* t0,
                                       const uint64_t* t1) {
  const uint64_t d = (x0 - t0[0]) + (x1 - t1[0]);
  const uint64_t e = (y0 - t0[1]) + (y1 - t1[1]);
  return Prod{t0[2] + d * t0[1] + e * t0[0] + d * e, t1[2] + d * t1[1] + e * t1[0]};
}

// Sum of a and b over the block (both parties at once); result in thread 0.
__device__ __forceinline__ void block_sum2(uint64_t& a, uint64_t& b) {
  __shared__ uint64_t red[2][kRowThreads / 32];
  for (int o = 16; o > 0; o >>= 1) {
    a += __shfl_xor_sync(0xffffffffu, a, o);
    b += __shfl_xor_sync(0xffffffffu, b, o);
  }
  const int w = threadIdx.x >> 5;
  if ((threadIdx.x & 31) == 0) {
    red[0][w] = a;
    red[1][w] = b;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    a = 0;
    b = 0;
    for (int k = 0; k < kRowThreads / 32; k++) {
      a += red[0][k];
      b += red[1][k];
    }
  }
}

// Row sums times invL, opened with the mean truncation's mask.  One block per row.
__global__ void ln_mean_open_kernel(const uint64_t* __restrict__ x0, const uint64_t* __restrict__ x1, int cols,
                                    uint64_t inv_len, uint64_t rM, uint64_t* __restrict__ xhat) {
  pdl_trigger();  // a following programmatic launch may start its set-up
  const size_t base = static_cast<size_t>(blockIdx.x) * cols;
  uint64_t a = 0, b = 0;
  for (int c = threadIdx.x; c < cols; c += blockDim.x) {
    a += x0[base + c];
    b += x1[base + c];
  }
  block_sum2(a, b);
  if (threadIdx.x == 0) xhat[blockIdx.x] = a * inv_len + b * inv_len + rM;
}

// d = x - mu; the Beaver squares of d, their row sums times invL, opened with
// the variance truncation's mask.  One block per row.
__global__ void ln_var_open_kernel(const uint64_t* __restrict__ x0, const uint64_t* __restrict__ x1,
                                   const uint64_t* __restrict__ mu0, const uint64_t* __restrict__ mu1, int cols,
                                   const uint64_t* __restrict__ tr0, const uint64_t* __restrict__ tr1,
                                   uint64_t inv_len, uint64_t rV, uint64_t* __restrict__ d0,
                                   uint64_t* __restrict__ d1, uint64_t* __restrict__ xhat) {
  pdl_trigger();  // a following programmatic launch may start its set-up
  const int r = blockIdx.x;
  const size_t base = static_cast<size_t>(r) * cols;
  const uint64_t m0 = mu0[r], m1 = mu1[r];
  uint64_t a = 0, b = 0;
  for (int c = threadIdx.x; c < cols; c += blockDim.x) {
    const size_t i = base + c;
    const uint64_t v0 = x0[i] - m0, v1 = x1[i] - m1;
    d0[i] = v0;
    d1[i] = v1;
    const Prod z = beaver(v0, v1, v0, v1, tr0 + 3 * i, tr1 + 3 * i);
    a += z.z0;
    b += z.z1;
  }
  block_sum2(a, b);
  if (threadIdx.x == 0) xhat[r] = a * inv_len + b * inv_len + rV;
}

// v += eps (party 0), opened with the rsqrt LUT gate's mask.
__global__ void ln_rsqrt_open_kernel(uint64_t* __restrict__ v0, const uint64_t* __restrict__ v1, uint64_t eps,
                                     uint64_t rR, uint64_t* __restrict__ xhat, int rows) {
  pdl_trigger();  // a following programmatic launch may start its set-up
  for (int r = blockIdx.x * blockDim.x + threadIdx.x; r < rows; r += gridDim.x * blockDim.x) {
    const uint64_t a = v0[r] + eps;
    v0[r] = a;
    xhat[r] = a + v1[r] + rR;
  }
}

// The row-level Newton stages: stage 0 = c1 * v; 1 = (y = z + c0) * y;
// 2 = v * y2; 3 = the halving's open; 4 = y * (3 2^(f-1) - h).
__global__ void ln_row_stage_kernel(int stage, const uint64_t* __restrict__ in0, const uint64_t* __restrict__ in1,
                                    const uint64_t* __restrict__ lut0, const uint64_t* __restrict__ lut1,
                                    const uint64_t* __restrict__ v0, const uint64_t* __restrict__ v1,
                                    uint64_t* __restrict__ y0, uint64_t* __restrict__ y1,
                                    const uint64_t* __restrict__ tr0, const uint64_t* __restrict__ tr1, int f,
                                    uint64_t rmask, uint64_t* __restrict__ xhat, int rows) {
  pdl_trigger();  // a following programmatic launch may start its set-up
  for (int r = blockIdx.x * blockDim.x + threadIdx.x; r < rows; r += gridDim.x * blockDim.x) {
    const uint64_t* t0 = tr0 + 3 * (static_cast<size_t>(stage < 3 ? stage : 3) * rows + r);
    const uint64_t* t1 = tr1 + 3 * (static_cast<size_t>(stage < 3 ? stage : 3) * rows + r);
    Prod z{0, 0};
    if (stage == 0) {
      z = beaver(lut0[4 * r + 1], lut1[4 * r + 1], v0[r], v1[r], t0, t1);
    } else if (stage == 1) {
      const uint64_t a = in0[r] + lut0[4 * r], b = in1[r] + lut1[4 * r];
      y0[r] = a;
      y1[r] = b;
      z = beaver(a, b, a, b, t0, t1);
    } else if (stage == 2) {
      z = beaver(v0[r], v1[r], in0[r], in1[r], t0, t1);
    } else if (stage == 3) {
      z = Prod{in0[r], in1[r]};
    } else {
      const uint64_t a = (uint64_t{3} << (f - 1)) - in0[r], b = 0ull - in1[r];
      z = beaver(y0[r], y1[r], a, b, t0, t1);
    }
    xhat[r] = z.z0 + z.z1 + rmask;
  }
}

// Row-broadcast Beaver product d * y[row]; writes prod0 + prod1 + rN.  One block per row.
__global__ void ln_norm_kernel(const uint64_t* __restrict__ d0, const uint64_t* __restrict__ d1,
                               const uint64_t* __restrict__ y0, const uint64_t* __restrict__ y1,
                               const uint64_t* __restrict__ A0, const uint64_t* __restrict__ A1,
                               const uint64_t* __restrict__ B0, const uint64_t* __restrict__ B1,
                               const uint64_t* __restrict__ C0, const uint64_t* __restrict__ C1, int cols,
                               uint64_t rN, uint64_t* __restrict__ xhat) {
  pdl_trigger();  // a following programmatic launch may start its set-up
  const int r = blockIdx.x;
  const size_t base = static_cast<size_t>(r) * cols;
  const uint64_t b0 = B0[r], b1 = B1[r];
  const uint64_t dv = (y0[r] - b0) + (y1[r] - b1);
  for (int c = threadIdx.x; c < cols; c += blockDim.x) {
    const size_t i = base + c;
    const uint64_t de = (d0[i] - A0[i]) + (d1[i] - A1[i]);
    xhat[i] = (C0[i] + de * b0 + dv * A0[i] + de * dv) + (C1[i] + de * b1 + dv * A1[i]) + rN;
  }
}

}  // namespace
}  // namespace sufb200

namespace {

int ln_launch_rc(const char* what) {
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? SUFB200_OK
                          : sufb200::record_error(SUFB200_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

int ln_trunc2(sufb200_ctx ctx, const sufb200_layernorm_party* p0, const sufb200_layernorm_party* p1, int k,
              const uint64_t* xhat, size_t n, uint64_t* out0, uint64_t* out1, cudaStream_t st) {
  if (p0->trunc_keys_device && p1->trunc_keys_device && p0->trunc_tables[k] && p1->trunc_tables[k]) {
    if (p0->trunc_ready[k]) {
      const cudaError_t e = cudaStreamWaitEvent(st, static_cast<cudaEvent_t>(p0->trunc_ready[k]), 0);
      if (e != cudaSuccess)
        return sufb200::record_error(SUFB200_ERR_CUDA, std::string("wait for bundle tables: ") + cudaGetErrorString(e));
    }
    return sufb200_trunc_bundle_eval_pair_tables_dev(ctx, &p0->trunc[k], p0->trunc_keys[k], p0->trunc_key_bytes[k],
                                                     p0->trunc_tables[k], &p1->trunc[k], p1->trunc_keys[k],
                                                     p1->trunc_key_bytes[k], p1->trunc_tables[k], xhat, n, out0, out1,
                                                     st);
  }
  if (p0->trunc_keys_device && p1->trunc_keys_device)  // resident keys: no host copy (capturable in a graph)
    return sufb200_trunc_bundle_eval_pair_dev(ctx, &p0->trunc[k], p0->trunc_keys[k], p0->trunc_key_bytes[k],
                                              &p1->trunc[k], p1->trunc_keys[k], p1->trunc_key_bytes[k], xhat, n, out0,
                                              out1, st);
  return sufb200_trunc_bundle_eval_pair(ctx, &p0->trunc[k], p0->trunc_keys[k], p0->trunc_key_bytes[k], &p1->trunc[k],
                                        p1->trunc_keys[k], p1->trunc_key_bytes[k], xhat, n, out0, out1, st);
}

}  // namespace

extern "C" int sufb200_layernorm_block_pair(sufb200_ctx ctx, const sufb200_layernorm_party* p0,
                                            const sufb200_layernorm_party* p1, int rows, int cols,
                                            const uint64_t* d_x0, const uint64_t* d_x1, int frac_bits,
                                            uint64_t inv_len, uint64_t eps, uint64_t* d_out0, uint64_t* d_out1,
                                            void* stream) {
  using namespace sufb200;
  if (!ctx || !p0 || !p1) return record_error(SUFB200_ERR_INVALID, "layernorm block: null context or material");
  if (rows < 1 || cols < 1 || frac_bits < 1 || frac_bits > 30)
    return record_error(SUFB200_ERR_INVALID, "layernorm block: rows, cols >= 1 and 1 <= frac_bits <= 30");
  if (!d_x0 || !d_x1 || !d_out0 || !d_out1) return record_error(SUFB200_ERR_INVALID, "layernorm block: null buffer");
  for (const sufb200_layernorm_party* p : {p0, p1})
    if (!p->d_rsqrt_lut || !p->d_sq_triples || !p->d_row_triples || !p->d_norm_a || !p->d_norm_b || !p->d_norm_c)
      return record_error(SUFB200_ERR_INVALID, "layernorm block: incomplete material");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const size_t R = static_cast<size_t>(rows), n = R * static_cast<size_t>(cols);
  // scratch words: per element 2 (d) + 1 (x^); per row 1 (x^) + 8 (LUT) + 2 x 7
  // (mu, v, z, y, y2, g, h) + 2 (Newton y)
  const size_t words = 3 * n + 25 * R;
  uint64_t* w = nullptr;
  cudaError_t ce = cudaMallocFromPoolAsync(reinterpret_cast<void**>(&w), words * 8, ctx->pool, st);
  if (ce != cudaSuccess)
    return record_error(SUFB200_ERR_CUDA, std::string("layernorm block scratch: ") + cudaGetErrorString(ce));
  uint64_t *d0 = w, *d1 = d0 + n, *xh = d1 + n, *xr = xh + n, *lut0 = xr + R, *lut1 = lut0 + 4 * R;
  uint64_t *mu0 = lut1 + 4 * R, *mu1 = mu0 + R, *v0 = mu1 + R, *v1 = v0 + R, *z0 = v1 + R, *z1 = z0 + R,
           *y0 = z1 + R, *y1 = y0 + R, *q0 = y1 + R, *q1 = q0 + R, *g0 = q1 + R, *g1 = g0 + R, *h0 = g1 + R,
           *h1 = h0 + R, *yn0 = h1 + R, *yn1 = yn0 + R;
  const int f = frac_bits;
  const unsigned gr = static_cast<unsigned>((R + kThreads - 1) / kThreads);
  int rc = SUFB200_OK;
  auto run = [&](int r) {
    if (rc == SUFB200_OK) rc = r;
    return rc == SUFB200_OK;
  };
  auto mask = [&](int k) { return p0->trunc_rin[k] + p1->trunc_rin[k]; };
  auto stage = [&](int s, const uint64_t* a0, const uint64_t* a1, int k) {
    if (rc != SUFB200_OK) return;
    ln_row_stage_kernel<<<gr, kThreads, 0, st>>>(s, a0, a1, lut0, lut1, v0, v1, y0, y1, p0->d_row_triples,
                                                 p1->d_row_triples, f, mask(k), xr, rows);
    run(ln_launch_rc("layernorm row stage"));
  };

  // mean and variance
  ln_mean_open_kernel<<<rows, kRowThreads, 0, st>>>(d_x0, d_x1, cols, inv_len, mask(0), xr);
  run(ln_launch_rc("layernorm mean"));
  if (run(rc)) run(ln_trunc2(ctx, p0, p1, 0, xr, R, mu0, mu1, st));
  if (rc == SUFB200_OK) {
    ln_var_open_kernel<<<rows, kRowThreads, 0, st>>>(d_x0, d_x1, mu0, mu1, cols, p0->d_sq_triples, p1->d_sq_triples,
                                                     inv_len, mask(1), d0, d1, xr);
    run(ln_launch_rc("layernorm variance"));
  }
  if (run(rc)) run(ln_trunc2(ctx, p0, p1, 1, xr, R, v0, v1, st));
  // rsqrt: LUT initial guess, one Newton step
  if (rc == SUFB200_OK) {
    ln_rsqrt_open_kernel<<<gr, kThreads, 0, st>>>(v0, v1, eps, p0->rsqrt_rin + p1->rsqrt_rin, xr, rows);
    run(ln_launch_rc("layernorm rsqrt open"));
  }
  if (run(rc))
    run(sufb200::interval_lut_pair_eval(ctx, p0->d_rsqrt_lut, p0->rsqrt_lut_bytes, p1->d_rsqrt_lut,
                                        p1->rsqrt_lut_bytes, xr, R, 4, lut0, lut1, st));
  stage(0, nullptr, nullptr, 2);  // c1 * v
  if (run(rc)) run(ln_trunc2(ctx, p0, p1, 2, xr, R, z0, z1, st));
  stage(1, z0, z1, 3);  // y = c0 + T_f(c1 v); y * y
  if (run(rc)) run(ln_trunc2(ctx, p0, p1, 3, xr, R, q0, q1, st));
  stage(2, q0, q1, 4);  // v * y2
  if (run(rc)) run(ln_trunc2(ctx, p0, p1, 4, xr, R, g0, g1, st));
  stage(3, g0, g1, 5);  // open g for the halving
  if (run(rc)) run(ln_trunc2(ctx, p0, p1, 5, xr, R, h0, h1, st));
  stage(4, h0, h1, 6);  // y * (3 2^(f-1) - h)
  if (run(rc)) run(ln_trunc2(ctx, p0, p1, 6, xr, R, yn0, yn1, st));
  // normalised output
  if (rc == SUFB200_OK) {
    ln_norm_kernel<<<rows, kRowThreads, 0, st>>>(d0, d1, yn0, yn1, p0->d_norm_a, p1->d_norm_a, p0->d_norm_b,
                                                 p1->d_norm_b, p0->d_norm_c, p1->d_norm_c, cols, mask(7), xh);
    run(ln_launch_rc("layernorm norm product"));
  }
  if (run(rc)) run(ln_trunc2(ctx, p0, p1, 7, xh, n, d_out0, d_out1, st));
  cudaFreeAsync(w, st);
  return rc;
}
