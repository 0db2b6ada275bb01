// softmax_block.cu -- the configs[4] softmax block (nn::SoftmaxBlockTask,
// include/nn/softmax_block_task.hpp) for both parties on one GPU, with every
// open computed on the device instead of through the reference's host
// channel and phase executor.
//
// The block's arithmetic on secret shares (all in Z_2^64, T_k = signed
// floor shift done by a truncation bundle, LUT = interval-LUT coefficient gate):
//   x^ = open(t + r)             c0..c3 = LUT_nexp(x^)
//   p  = (c3 t + c2 2^f) t       p2 = T_f(p)          (CubicPolyTask Mul1, Mul2, Trunc1)
//   r  = (p2 + c1 2^f) t         e  = T_2f(r) + c0    (Mul3, Trunc2; T_2f done
//                                                      as T_f(T_f(r)), the same floor)
//   s  = row sums of e           s^ = open(s + r')    a0, a1 = LUT_recip(s^)
//   y  = T_f(a1 s) + a0                               (RecipTask init)
//   y  = T_f(y (2 2^f - T_f(y s)))                    (one Newton step)
//   prob = T_f(e y[row])                              (MulRowBroadcastTask, TruncTask)
// Products are Beaver products: with d = x - a and e = y - b opened,
// z = c + d b + e a (+ d e on party 0).  Because both parties' shares are on
// this GPU, an open is a per-element sum, so consecutive Beaver rounds with
// no truncation between them fuse into one elementwise kernel; each fused
// kernel ends by writing the masked value x + r_in that the next truncation
// bundle takes as its public input.  Each party's truncation bundle and LUT
// evaluation runs on its own shares and keys, as it would on its own GPU.
//
// 9 fused kernels, 4 LUT launches and 7 truncation stages per block: the
// element-level stages run each party's bundle on the shared-prefix path, the
// row-level ones both parties in one query-parallel launch.
#include <string>

#include "kernels.hpp"
#include "sufb200_internal.cuh"

namespace sufb200 {
namespace {

constexpr int kThreads = 256;
constexpr int kRowThreads = 128;

struct Prod {
  uint64_t z0, z1;
};

// Beaver product of x and y for both parties with triple shares t0, t1
// (a, b, c interleaved).
__device__ __forceinline__ Prod beaver(uint64_t x0, uint64_t x1, uint64_t y0, uint64_t y1, const uint64_t* t0,
                                       const uint64_t* t1) {
  const uint64_t d = (x0 - t0[0]) + (x1 - t1[0]);
  const uint64_t e = (y0 - t0[1]) + (y1 - t1[1]);
  return Prod{t0[2] + d * t0[1] + e * t0[0] + d * e, t1[2] + d * t1[1] + e * t1[0]};
}

// x^ = t0 + t1 + r (the open of the nExp input, masked by its r_in).
__global__ void open_masked_kernel(const uint64_t* __restrict__ a0, const uint64_t* __restrict__ a1, uint64_t r,
                                   uint64_t* __restrict__ out, size_t n) {
  pdl_trigger();  // a following programmatic launch may start its set-up
  for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x)
    out[i] = a0[i] + a1[i] + r;
}

// CubicPolyTask Mul1 + Mul2: p = (c3 t + c2 2^f) t; writes p0 + p1 + rA.
__global__ void nexp_mul12_kernel(const uint64_t* __restrict__ c0, const uint64_t* __restrict__ c1,
                                  const uint64_t* __restrict__ t0, const uint64_t* __restrict__ t1,
                                  const uint64_t* __restrict__ tr0, const uint64_t* __restrict__ tr1, int f,
                                  uint64_t rA, uint64_t* __restrict__ xhat, size_t n) {
  pdl_trigger();  // a following programmatic launch may start its set-up
  for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const uint64_t x0 = t0[i], x1 = t1[i];
    const Prod m = beaver(c0[4 * i + 3], c1[4 * i + 3], x0, x1, tr0 + 3 * i, tr1 + 3 * i);
    const uint64_t u0 = m.z0 + (c0[4 * i + 2] << f), u1 = m.z1 + (c1[4 * i + 2] << f);
    const Prod p = beaver(u0, u1, x0, x1, tr0 + 3 * (n + i), tr1 + 3 * (n + i));
    xhat[i] = p.z0 + p.z1 + rA;
  }
}

// CubicPolyTask Mul3: r = (p2 + c1 2^f) t; writes r0 + r1 + rB.
__global__ void nexp_mul3_kernel(const uint64_t* __restrict__ c0, const uint64_t* __restrict__ c1,
                                 const uint64_t* __restrict__ p20, const uint64_t* __restrict__ p21,
                                 const uint64_t* __restrict__ t0, const uint64_t* __restrict__ t1,
                                 const uint64_t* __restrict__ tr0, const uint64_t* __restrict__ tr1, int f,
                                 uint64_t rB, uint64_t* __restrict__ xhat, size_t n) {
  pdl_trigger();  // a following programmatic launch may start its set-up
  for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const uint64_t q0 = p20[i] + (c0[4 * i + 1] << f), q1 = p21[i] + (c1[4 * i + 1] << f);
    const Prod r = beaver(q0, q1, t0[i], t1[i], tr0 + 3 * (2 * n + i), tr1 + 3 * (2 * n + i));
    xhat[i] = r.z0 + r.z1 + rB;
  }
}

// e = T_2f(r) + c0 per element, row sums of e per party, and the open of the
// reciprocal's input s^ = s0 + s1 + rR.  One block per row.
__global__ void rowsum_open_kernel(const uint64_t* __restrict__ y0, const uint64_t* __restrict__ y1,
                                   const uint64_t* __restrict__ c0, const uint64_t* __restrict__ c1,
                                   const int32_t* __restrict__ row_off, uint64_t rR, uint64_t* __restrict__ e0,
                                   uint64_t* __restrict__ e1, uint64_t* __restrict__ s0, uint64_t* __restrict__ s1,
                                   uint64_t* __restrict__ shat) {
  pdl_trigger();  // a following programmatic launch may start its set-up
  __shared__ uint64_t red[2][kRowThreads / 32];
  const int r = blockIdx.x;
  const int beg = row_off[r], end = row_off[r + 1];
  uint64_t a0 = 0, a1 = 0;
  for (int i = beg + static_cast<int>(threadIdx.x); i < end; i += blockDim.x) {
    const uint64_t v0 = y0[i] + c0[4 * static_cast<size_t>(i)], v1 = y1[i] + c1[4 * static_cast<size_t>(i)];
    e0[i] = v0;
    e1[i] = v1;
    a0 += v0;
    a1 += v1;
  }
  for (int o = 16; o > 0; o >>= 1) {
    a0 += __shfl_xor_sync(0xffffffffu, a0, o);
    a1 += __shfl_xor_sync(0xffffffffu, a1, o);
  }
  const int w = threadIdx.x >> 5;
  if ((threadIdx.x & 31) == 0) {
    red[0][w] = a0;
    red[1][w] = a1;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    uint64_t t0 = 0, t1 = 0;
    for (int k = 0; k < kRowThreads / 32; k++) {
      t0 += red[0][k];
      t1 += red[1][k];
    }
    s0[r] = t0;
    s1[r] = t1;
    shat[r] = t0 + t1 + rR;
  }
}

// RecipTask init multiply: a1 * s; writes z0 + z1 + rC.
__global__ void recip_init_kernel(const uint64_t* __restrict__ a0, const uint64_t* __restrict__ a1,
                                  const uint64_t* __restrict__ s0, const uint64_t* __restrict__ s1,
                                  const uint64_t* __restrict__ tr0, const uint64_t* __restrict__ tr1, uint64_t rC,
                                  uint64_t* __restrict__ xhat, int rows) {
  pdl_trigger();  // a following programmatic launch may start its set-up
  for (int r = blockIdx.x * blockDim.x + threadIdx.x; r < rows; r += gridDim.x * blockDim.x) {
    const Prod z = beaver(a0[4 * r + 1], a1[4 * r + 1], s0[r], s1[r], tr0 + 3 * r, tr1 + 3 * r);
    xhat[r] = z.z0 + z.z1 + rC;
  }
}

// y = T_f(a1 s) + a0, then the Newton step's y * s; keeps y, writes w0 + w1 + rD.
__global__ void recip_nr1_kernel(const uint64_t* __restrict__ z0, const uint64_t* __restrict__ z1,
                                 const uint64_t* __restrict__ a0, const uint64_t* __restrict__ a1,
                                 const uint64_t* __restrict__ s0, const uint64_t* __restrict__ s1,
                                 const uint64_t* __restrict__ tr0, const uint64_t* __restrict__ tr1, uint64_t rD,
                                 uint64_t* __restrict__ y0, uint64_t* __restrict__ y1, uint64_t* __restrict__ xhat,
                                 int rows) {
  pdl_trigger();  // a following programmatic launch may start its set-up
  for (int r = blockIdx.x * blockDim.x + threadIdx.x; r < rows; r += gridDim.x * blockDim.x) {
    const uint64_t v0 = z0[r] + a0[4 * r], v1 = z1[r] + a1[4 * r];
    y0[r] = v0;
    y1[r] = v1;
    const Prod w = beaver(v0, v1, s0[r], s1[r], tr0 + 3 * (rows + r), tr1 + 3 * (rows + r));
    xhat[r] = w.z0 + w.z1 + rD;
  }
}

// d = 2 2^f - T_f(y s) (the constant on party 0), then y * d; writes v0 + v1 + rE.
__global__ void recip_nr2_kernel(const uint64_t* __restrict__ y0, const uint64_t* __restrict__ y1,
                                 const uint64_t* __restrict__ g0, const uint64_t* __restrict__ g1, int f,
                                 const uint64_t* __restrict__ tr0, const uint64_t* __restrict__ tr1, uint64_t rE,
                                 uint64_t* __restrict__ xhat, int rows) {
  pdl_trigger();  // a following programmatic launch may start its set-up
  for (int r = blockIdx.x * blockDim.x + threadIdx.x; r < rows; r += gridDim.x * blockDim.x) {
    const uint64_t d0 = (uint64_t{2} << f) - g0[r], d1 = 0ull - g1[r];
    const Prod v = beaver(y0[r], y1[r], d0, d1, tr0 + 3 * (2 * rows + r), tr1 + 3 * (2 * rows + r));
    xhat[r] = v.z0 + v.z1 + rE;
  }
}

// Row-broadcast Beaver product e * inv[row] with triples (A, B[row], C);
// writes prod0 + prod1 + rF.  One block per row.
__global__ void row_bcast_kernel(const uint64_t* __restrict__ e0, const uint64_t* __restrict__ e1,
                                 const uint64_t* __restrict__ v0, const uint64_t* __restrict__ v1,
                                 const uint64_t* __restrict__ A0, const uint64_t* __restrict__ A1,
                                 const uint64_t* __restrict__ B0, const uint64_t* __restrict__ B1,
                                 const uint64_t* __restrict__ C0, const uint64_t* __restrict__ C1,
                                 const int32_t* __restrict__ row_off, uint64_t rF, uint64_t* __restrict__ xhat) {
  pdl_trigger();  // a following programmatic launch may start its set-up
  const int r = blockIdx.x;
  const int beg = row_off[r], end = row_off[r + 1];
  const uint64_t b0 = B0[r], b1 = B1[r];
  const uint64_t dv = (v0[r] - b0) + (v1[r] - b1);  // the opened row factor
  for (int i = beg + static_cast<int>(threadIdx.x); i < end; i += blockDim.x) {
    const uint64_t de = (e0[i] - A0[i]) + (e1[i] - A1[i]);
    const uint64_t p0 = C0[i] + de * b0 + dv * A0[i] + de * dv;
    const uint64_t p1 = C1[i] + de * b1 + dv * A1[i];
    xhat[i] = p0 + p1 + rF;
  }
}

}  // namespace
}  // namespace sufb200

namespace {

unsigned grid_of(const sufb200_ctx_s* ctx, size_t n) {
  const size_t want = (n + sufb200::kThreads - 1) / sufb200::kThreads;
  const size_t cap = static_cast<size_t>(ctx->sm_count) * 8;
  return static_cast<unsigned>(want < 1 ? 1 : (want < cap ? want : cap));
}

int launch_rc(const char* what) {
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? SUFB200_OK
                          : sufb200::record_error(SUFB200_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

// Both parties' truncation bundle k over x^ (n words) into out0 / out1.
int trunc2(sufb200_ctx ctx, const sufb200_softmax_party* p0, const sufb200_softmax_party* p1, int k,
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

extern "C" int sufb200_softmax_block_pair(sufb200_ctx ctx, const sufb200_softmax_party* p0,
                                          const sufb200_softmax_party* p1, int rows, const int32_t* d_row_off,
                                          const uint64_t* d_t0, const uint64_t* d_t1, size_t n, int frac_bits,
                                          uint64_t* d_prob0, uint64_t* d_prob1, void* stream) {
  using namespace sufb200;
  if (!ctx || !p0 || !p1) return record_error(SUFB200_ERR_INVALID, "softmax block: null context or material");
  if (rows < 1 || frac_bits < 1 || frac_bits > 30)
    return record_error(SUFB200_ERR_INVALID, "softmax block: rows >= 1 and 1 <= frac_bits <= 30");
  if (n == 0) return SUFB200_OK;
  if (!d_row_off || !d_t0 || !d_t1 || !d_prob0 || !d_prob1)
    return record_error(SUFB200_ERR_INVALID, "softmax block: null device buffer");
  for (const sufb200_softmax_party* p : {p0, p1})
    if (!p->d_nexp_lut || !p->d_recip_lut || !p->d_nexp_triples || !p->d_recip_triples || !p->d_row_a ||
        !p->d_row_b || !p->d_row_c)
      return record_error(SUFB200_ERR_INVALID, "softmax block: incomplete material");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const size_t R = static_cast<size_t>(rows);
  // scratch words: per element 8 (LUT) + 1 (x^) + 2 (p2) + 2 (T_f(r)) +
  // 2 (T_2f) + 2 (e); per row 2 (s) + 1 (s^) + 8 (LUT) + 1 (x^) + 2 x 4 (z, y,
  // T(y s), inv)
  const size_t words = 17 * n + 20 * R;
  uint64_t* w = nullptr;
  cudaError_t ce = cudaMallocFromPoolAsync(reinterpret_cast<void**>(&w), words * 8, ctx->pool, st);
  if (ce != cudaSuccess)
    return record_error(SUFB200_ERR_CUDA, std::string("softmax block scratch: ") + cudaGetErrorString(ce));
  uint64_t *lut0 = w, *lut1 = lut0 + 4 * n, *xh = lut1 + 4 * n, *p20 = xh + n, *p21 = p20 + n, *y0 = p21 + n,
           *y1 = y0 + n, *e0 = y1 + n, *e1 = e0 + n;
  uint64_t *h0 = e1 + n, *h1 = h0 + n;  // T_f(r), the first half of T_2f(r)
  uint64_t *s0 = h1 + n, *s1 = s0 + R, *sh = s1 + R, *lr0 = sh + R, *lr1 = lr0 + 4 * R, *xr = lr1 + 4 * R,
           *z0 = xr + R, *z1 = z0 + R, *yr0 = z1 + R, *yr1 = yr0 + R, *g0 = yr1 + R, *g1 = g0 + R, *v0 = g1 + R,
           *v1 = v0 + R;
  const int f = frac_bits;
  const unsigned ge = grid_of(ctx, n), gr = grid_of(ctx, R);
  int rc = SUFB200_OK;
  auto run = [&](int r) {
    if (rc == SUFB200_OK) rc = r;
    return rc == SUFB200_OK;
  };

  // nExp: open t + r, coefficient LUT per party, Horner with two truncations
  open_masked_kernel<<<ge, kThreads, 0, st>>>(d_t0, d_t1, p0->nexp_rin + p1->nexp_rin, xh, n);
  run(launch_rc("softmax open"));
  if (run(rc))
    run(sufb200::interval_lut_pair_eval(ctx, p0->d_nexp_lut, p0->nexp_lut_bytes, p1->d_nexp_lut, p1->nexp_lut_bytes,
                                        xh, n, 4, lut0, lut1, st));
  if (rc == SUFB200_OK) {
    nexp_mul12_kernel<<<ge, kThreads, 0, st>>>(lut0, lut1, d_t0, d_t1, p0->d_nexp_triples, p1->d_nexp_triples, f,
                                               p0->trunc_rin[0] + p1->trunc_rin[0], xh, n);
    run(launch_rc("softmax nExp Mul1/Mul2"));
  }
  if (run(rc)) run(trunc2(ctx, p0, p1, 0, xh, n, p20, p21, st));
  if (rc == SUFB200_OK) {
    nexp_mul3_kernel<<<ge, kThreads, 0, st>>>(lut0, lut1, p20, p21, d_t0, d_t1, p0->d_nexp_triples,
                                              p1->d_nexp_triples, f, p0->trunc_rin[1] + p1->trunc_rin[1], xh, n);
    run(launch_rc("softmax nExp Mul3"));
  }
  if (run(rc)) run(trunc2(ctx, p0, p1, 1, xh, n, h0, h1, st));
  if (rc == SUFB200_OK) {
    open_masked_kernel<<<ge, kThreads, 0, st>>>(h0, h1, p0->trunc_rin[6] + p1->trunc_rin[6], xh, n);
    run(launch_rc("softmax T_2f second half open"));
  }
  if (run(rc)) run(trunc2(ctx, p0, p1, 6, xh, n, y0, y1, st));

  // row sums and the reciprocal (one Newton step) on the rows
  if (rc == SUFB200_OK) {
    rowsum_open_kernel<<<rows, kRowThreads, 0, st>>>(y0, y1, lut0, lut1, d_row_off, p0->recip_rin + p1->recip_rin,
                                                     e0, e1, s0, s1, sh);
    run(launch_rc("softmax row sums"));
  }
  if (run(rc))
    run(sufb200::interval_lut_pair_eval(ctx, p0->d_recip_lut, p0->recip_lut_bytes, p1->d_recip_lut,
                                        p1->recip_lut_bytes, sh, R, 4, lr0, lr1, st));
  if (rc == SUFB200_OK) {
    recip_init_kernel<<<gr, kThreads, 0, st>>>(lr0, lr1, s0, s1, p0->d_recip_triples, p1->d_recip_triples,
                                               p0->trunc_rin[2] + p1->trunc_rin[2], xr, rows);
    run(launch_rc("softmax reciprocal init"));
  }
  if (run(rc)) run(trunc2(ctx, p0, p1, 2, xr, R, z0, z1, st));
  if (rc == SUFB200_OK) {
    recip_nr1_kernel<<<gr, kThreads, 0, st>>>(z0, z1, lr0, lr1, s0, s1, p0->d_recip_triples, p1->d_recip_triples,
                                              p0->trunc_rin[3] + p1->trunc_rin[3], yr0, yr1, xr, rows);
    run(launch_rc("softmax Newton y*s"));
  }
  if (run(rc)) run(trunc2(ctx, p0, p1, 3, xr, R, g0, g1, st));
  if (rc == SUFB200_OK) {
    recip_nr2_kernel<<<gr, kThreads, 0, st>>>(yr0, yr1, g0, g1, f, p0->d_recip_triples, p1->d_recip_triples,
                                              p0->trunc_rin[4] + p1->trunc_rin[4], xr, rows);
    run(launch_rc("softmax Newton y*d"));
  }
  if (run(rc)) run(trunc2(ctx, p0, p1, 4, xr, R, v0, v1, st));

  // probabilities: row-broadcast product and its truncation
  if (rc == SUFB200_OK) {
    row_bcast_kernel<<<rows, kRowThreads, 0, st>>>(e0, e1, v0, v1, p0->d_row_a, p1->d_row_a, p0->d_row_b,
                                                   p1->d_row_b, p0->d_row_c, p1->d_row_c, d_row_off,
                                                   p0->trunc_rin[5] + p1->trunc_rin[5], xh);
    run(launch_rc("softmax row-broadcast product"));
  }
  if (run(rc)) run(trunc2(ctx, p0, p1, 5, xh, n, d_prob0, d_prob1, st));
  cudaFreeAsync(w, st);
  return rc;
}
