// kernels.hpp -- launch helpers shared between the kernel translation units
// and the C ABI (capi.cu).  Internal to the library.
#pragma once

#include <cstddef>
#include <cstdint>
#include <string>
#include <utility>

#include <cuda_runtime.h>

#include "sufb200_internal.cuh"

namespace sufb200 {

// Programmatic dependent launch of kernel k (see pdl_wait in
// sufb200_internal.cuh): the attribute is set unless SUFB200_PDL=0 in the
// environment.  Every kernel launched this way calls pdl_wait() before it
// reads anything an earlier kernel of the stream may still be writing.
bool pdl_enabled();
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*k)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args&&... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, k, std::forward<Args>(args)...);
}

struct DcfLaunch {
  const uint8_t* keys;  // device: [n][key_bytes] or one key (broadcast)
  size_t key_bytes;
  const uint64_t* xs;  // device [n]
  size_t n;
  void* out;  // device [n][out_bytes]
  const uint32_t* t0;
  uint32_t* status;
  int in_bits;
  int out_bytes;
};

cudaError_t launch_myl7_eval(const sufb200_ctx_s* ctx, int group, const DcfLaunch& a, int broadcast,
                             cudaStream_t st);

// Fused truncation bundle (trunc_bundle.cu).
struct TruncLaunch {
  sufb200_trunc_desc desc;
  const uint8_t* key[4];     // device: query q's broadcast myl7 key (any alignment)
  const uint64_t* xhat;      // device [n]
  size_t n;
  uint64_t* y;               // device [n]
  uint64_t* bools;           // device [n][3] (carry, sign, wrap) or nullptr
  const uint32_t* t0;
  uint32_t* status;
};
cudaError_t launch_trunc_bundle(const sufb200_ctx_s* ctx, const TruncLaunch& a, cudaStream_t st);
// Per-element masks: element i's keys for slot q at keys[q] + i * key_bytes[q]
// (device), its words [carry_w, sign_w, haty, r_hi, m, plan] at words[6 i].
struct TruncElemLaunch {
  sufb200_trunc_desc shape;  // kind, frac_bits, party, nq slots, q_bits
  const uint8_t* keys[4];
  uint64_t key_bytes[4];
  const uint64_t* words;
  const uint64_t* xhat;
  size_t n;
  uint64_t* y;
  uint64_t* bools;
  const uint32_t* t0;
  uint32_t* status;
};
// mode: 0 adapter-layout keys (bytewise), 1 adapter-layout keys (aligned
// loads), 2 level-major keys (launch_elem_keys_to_soa's layout).
cudaError_t launch_trunc_bundle_elem(const sufb200_ctx_s* ctx, const TruncElemLaunch& a, int mode,
                                     cudaStream_t st);
// One slot's n adapter-layout keys (key_bytes each, in_bits nb, party) into
// the level-major layout of elem_soa_bytes(nb, n) bytes at soa (device,
// 16-byte aligned); a key whose header does not match is flagged.
cudaError_t launch_elem_keys_to_soa(const sufb200_ctx_s* ctx, const uint8_t* keys, size_t kb, int nb, int party,
                                    size_t n, uint8_t* soa, cudaStream_t st);
size_t elem_soa_bytes(int nb, size_t n);
// A chunk of a job bucket (jobs.cu): job j's words are src[j][0..off[j+1]-off[j])
// (gather) or dst[j][...] (scatter), at batch[base + off[j] ...].
constexpr int kJobsPerLaunch = 48;
struct JobTable {
  const uint64_t* src[kJobsPerLaunch];
  uint64_t* dst[kJobsPerLaunch];
  size_t off[kJobsPerLaunch + 1];
  size_t base;
  int njobs;
};
cudaError_t launch_jobs_copy(const sufb200_ctx_s* ctx, const JobTable& t, uint64_t* batch, bool to_batch,
                             cudaStream_t st);

// Both parties' bundles over the same x^ (a0.xhat == a1.xhat, a0.n == a1.n),
// one lane per (party, element, query): for batches too small to fill the GPU.
cudaError_t launch_trunc_bundle_pair(const sufb200_ctx_s* ctx, const TruncLaunch& a0, const TruncLaunch& a1,
                                     cudaStream_t st);

// Reference GPU-backend key formats (ref_formats.cu).
struct RefFmtLaunch {
  const uint8_t* keys;
  size_t key_bytes;
  int broadcast;
  const uint64_t* xs;
  size_t n;
  uint64_t idx_base;
  void* out;
  int in_bits;
  int out_words;  // packed / LUT
  int out_bytes;  // threshold DCF
  const uint32_t* t0;
  uint32_t* status;
};
cudaError_t launch_thr_dcf(const sufb200_ctx_s* ctx, const RefFmtLaunch& a, cudaStream_t st);
cudaError_t launch_packed_lt(const sufb200_ctx_s* ctx, const RefFmtLaunch& a, cudaStream_t st);
cudaError_t launch_interval_lut(const sufb200_ctx_s* ctx, const RefFmtLaunch& a, cudaStream_t st);
// Both parties' broadcast keys over one x^ (a0 party 0, a1 party 1), one launch.
cudaError_t launch_interval_lut_pair(const sufb200_ctx_s* ctx, const RefFmtLaunch& a0, const RefFmtLaunch& a1,
                                     cudaStream_t st);
// Checked form for the device blocks: both parties' broadcast interval-LUT
// keys (device) over x^, out_words each; a status code (record_error on
// failure).
int interval_lut_pair_eval(const sufb200_ctx_s* ctx, const uint8_t* key0, size_t key_bytes0, const uint8_t* key1,
                           size_t key_bytes1, const uint64_t* xs, size_t n, int out_words, uint64_t* out0,
                           uint64_t* out1, cudaStream_t st);

// Interval-LUT coefficients, the polynomial over the public x^ and the output
// masks in one pass (broadcast key, out_words = r * (degree + 1)).
constexpr int kCoeffMaxOut = 8;
constexpr size_t kCoeffParamKeyBytes = 4096;  // keys up to this size travel in the kernel parameters
struct CoeffLutParams {
  int r;                         // outputs per element
  int degree;                    // coefficients per output = degree + 1
  uint64_t ring_mask;            // results reduced mod 2^ring_bits
  uint64_t r_out[kCoeffMaxOut];  // this party's output-mask shares
  int key_in_params;             // the key is `key` below, not RefFmtLaunch::keys
  alignas(16) uint8_t key[kCoeffParamKeyBytes];
};
cudaError_t launch_coeff_lut(const sufb200_ctx_s* ctx, const RefFmtLaunch& a, const CoeffLutParams& p,
                             cudaStream_t st);
// Both parties' gates over one x^ (a0.xs == a1.xs, equal n) in one launch.
cudaError_t launch_coeff_lut_pair(const sufb200_ctx_s* ctx, const RefFmtLaunch& a0, const CoeffLutParams& p0,
                                  const RefFmtLaunch& a1, const CoeffLutParams& p1, cudaStream_t st);

// Shared-prefix evaluation of broadcast keys (prefix.cu, prefix.cuh).
struct RangeAcc;
struct FrontierEntry;
struct FrontierLaunch {
  const uint8_t* key;  // device: one myl7 key
  int in_bits;
  int out_bytes;
  const RangeAcc* acc;
  uint32_t kmax;
  FrontierEntry* out;  // device [kmax]
  const uint32_t* t0;
  uint32_t* status;
  // Non-null: plan over every value (the range set_full_range writes)
  // without reading acc, and store that range here for the main pass that
  // later reads these tables.
  RangeAcc* full;
};
// The frontier tables of up to eight keys over one batch (one bundle's
// queries, or both parties' bundles), built in one launch (all keys share
// the range accumulator and the status word of q[0]).
constexpr int kFrontierMaxKeys = 16;
struct FrontierBatch {
  FrontierLaunch q[kFrontierMaxKeys];
  int nq;
};
uint32_t prefix_budget(size_t n);
cudaError_t launch_range(const sufb200_ctx_s* ctx, const uint64_t* xs, size_t n, RangeAcc* acc, cudaStream_t st);
// The range of "every value" in place of launch_range (see prefix.cu).
cudaError_t set_full_range(RangeAcc* acc, cudaStream_t st);
// max_grid > 0 caps the blocks (one per SM): a fill meant to run beside
// other work leaves the remaining SMs to it.
cudaError_t launch_frontier(const sufb200_ctx_s* ctx, int group, const FrontierBatch& b, cudaStream_t st,
                            int max_grid = 0);
cudaError_t launch_myl7_bcast_prefix(const sufb200_ctx_s* ctx, int group, const DcfLaunch& a, const RangeAcc* acc,
                                     uint32_t kmax, const FrontierEntry* F, cudaStream_t st);
cudaError_t launch_trunc_bundle_prefix(const sufb200_ctx_s* ctx, const TruncLaunch& a, const RangeAcc* acc,
                                       uint32_t kmax, FrontierEntry* const F[4], cudaStream_t st);
// Both parties' bundles over one x^ in one main pass: F[0..3] party 0's
// queries, F[4..7] party 1's.
// Both parties' bundles against full-domain tables (every query's plan at
// its whole domain): lookups only, no keys or AES tables.
cudaError_t launch_trunc_bundle_lookup_pair(const sufb200_ctx_s* ctx, const TruncLaunch& a0, const TruncLaunch& a1,
                                            const RangeAcc* acc, uint32_t kmax, FrontierEntry* const F[8],
                                            cudaStream_t st);
cudaError_t launch_trunc_bundle_prefix_pair(const sufb200_ctx_s* ctx, const TruncLaunch& a0, const TruncLaunch& a1,
                                            const RangeAcc* acc, uint32_t kmax, FrontierEntry* const F[8],
                                            cudaStream_t st);

// myl7 DCF keygen on the GPU (keygen_dev.cu): one key pair per thread.
struct GenLaunch {
  const uint64_t* alphas;  // device [n]
  const uint8_t* seeds0;   // device [n][16], 16-byte aligned
  const uint8_t* seeds1;
  uint8_t* keys0;          // device [n][key_bytes], 8-byte aligned
  uint8_t* keys1;
  size_t n;
  size_t key_bytes;
  int in_bits;             // multiple of 8
  int payload_len;         // 1..16
  uint64_t beta_lo, beta_hi;
  const uint32_t* t0;
  uint32_t* status;
};
cudaError_t launch_myl7_gen(const sufb200_ctx_s* ctx, int group, const GenLaunch& g, cudaStream_t st);

// Exact Z_2^64 matrix product on the tensor cores (ring_gemm_tc.cu):
// out[b] = scale(C[b] + bias + sum_p X_p[b] (Y_p[b] + Y2_p[b])), X_p [M][K]
// row-major, Y_p [K][N] (or [N][K] when trans), per-batch strides in elements
// (0: shared across batches).
struct RingGemmPiece {
  const uint64_t* x;
  const uint64_t* y;
  const uint64_t* y2;  // optional, added to y element-wise
  size_t xs, ys, y2s;
};
struct RingGemmLaunch {
  RingGemmPiece piece[2];
  int npieces;
  int M, N, K;
  int trans;
  const uint64_t* c;  // optional [M][N]
  size_t cs;
  const int64_t* bias;  // optional [N]
  int has_scale;
  int64_t mul_const;
  int mul_shift;
  uint64_t* out;
  size_t os;
  uint32_t* status;
  // set by the launcher
  int batches;
  int splits;        // contraction split across the CTAs of one cluster
  int steps;         // 32-deep steps over all pieces
  int m_pad, n_pad;  // rows of the plane slabs (multiples of 128 / 64)
  const uint8_t* xplanes;
  size_t xps;  // per-batch stride in bytes (0: shared)
  const uint8_t* yplanes;
  size_t yps;
};

// One operand's byte planes (ring_gemm_tc.cu::split_planes_kernel).
struct PlanesPiece {
  const uint64_t* src;
  const uint64_t* add;  // optional element-wise addend
  size_t ss, as;        // per-batch strides in elements
};
struct PlanesSplit {
  PlanesPiece piece[2];
  int R, K;  // rows (M or N) and depth per piece
  int rows_pad;
  int tile_rows;  // GEMM tile rows of this operand (128 for A, 64 for B)
  int steps;
  int k_contig;  // (row, k) at src[row * K + k]; else src[k * R + row]
  uint8_t* dst;
  size_t ds;  // per-batch stride in bytes
};
cudaError_t launch_ring_gemm_tc(const sufb200_ctx_s* ctx, RingGemmLaunch g, int batches, cudaStream_t st);

// Measured AES-128 block rate of the shared-memory engine (probe.cu).
cudaError_t probe_aes_engine(const sufb200_ctx_s* ctx, double* blocks_per_s);

// Records `msg` as the calling thread's sufb200_last_error() and returns code.
int record_error(int code, const std::string& msg);

// Probe of the dynamic shared-memory base (capi.cu uses it at context setup).
cudaError_t probe_dyn_smem_base(uint32_t* d_out, cudaStream_t st);

}  // namespace sufb200
