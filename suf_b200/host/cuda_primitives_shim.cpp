// cuda_primitives_shim.cpp -- the reference runtime's flat CUDA-primitives
// ABI (include/runtime/cuda_primitives.hpp:9-240, implemented in the
// reference by cuda/cuda_primitives.cu:711-1267) on top of libsufb200.
//
// Linked into the reference in place of cuda/cuda_primitives.cu, it serves the
// launch_* calls of composite_fss.hpp, phase_tasks.hpp, softmax_block_task.hpp,
// open_collector.cpp, pfss_superbatch.cpp and attention_block.cpp.  The
// signatures are the reference's; where the reference launchers return
// silently on a failed launch, these throw std::runtime_error with the engine's
// message (the callers are C++).
#include <cuda_runtime.h>

#include <cstddef>
#include <map>
#include <mutex>
#include <cstdint>
#include <stdexcept>
#include <string>

#include "sufb200.h"

namespace {
void ok(int rc, const char* what) {
  if (rc != SUFB200_OK) throw std::runtime_error(std::string(what) + ": " + sufb200_last_error());
}

// One engine context per device for the launchers that need one (made at
// the first call on the current device, kept until exit).
sufb200_ctx device_ctx() {
  static std::mutex mu;
  static std::map<int, sufb200_ctx> ctxs;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return nullptr;
  std::lock_guard<std::mutex> lk(mu);
  auto it = ctxs.find(dev);
  if (it != ctxs.end()) return it->second;
  sufb200_ctx c = nullptr;
  ok(sufb200_ctx_create(dev, &c), "sufb200_ctx_create");
  ctxs.emplace(dev, c);
  return c;
}
}  // namespace

extern "C" {

void launch_beaver_mul_kernel(int party, const uint64_t* /*d_x*/, const uint64_t* /*d_y*/, const uint64_t* d_a,
                              const uint64_t* d_b, const uint64_t* d_c, const uint64_t* d_d_open,
                              const uint64_t* d_e_open, uint64_t* d_out, size_t n, void* stream) {
  ok(sufb200_beaver_mul(party, d_a, d_b, d_c, d_d_open, d_e_open, d_out, n, stream), "launch_beaver_mul_kernel");
}

void launch_beaver_mul_aos_kernel(int party, const void* d_triples, const uint64_t* d_d_open, const uint64_t* d_e_open,
                                  uint64_t* d_out, size_t n, void* stream) {
  ok(sufb200_beaver_mul_aos(party, static_cast<const uint64_t*>(d_triples), d_d_open, d_e_open, d_out, n, stream),
     "launch_beaver_mul_aos_kernel");
}

void launch_trunc_shift_kernel(const uint64_t* d_in, uint64_t* d_out, int frac_bits, size_t n, void* stream) {
  ok(sufb200_trunc_shift(d_in, d_out, frac_bits, n, stream), "launch_trunc_shift_kernel");
}

void launch_trunc_postproc_kernel(int party, int kind_gapars, int frac_bits, uint64_t r_hi_share, uint64_t m_share,
                                  const uint64_t* d_hatx_public, const uint64_t* d_arith, size_t arith_stride,
                                  int arith_idx, const uint64_t* d_bools, size_t bool_stride, int carry_idx,
                                  int sign_idx, int wrap_idx, uint64_t* d_out, size_t n, void* stream) {
  ok(sufb200_trunc_postproc(party, kind_gapars, frac_bits, r_hi_share, m_share, d_hatx_public, d_arith, arith_stride,
                            arith_idx, d_bools, bool_stride, carry_idx, sign_idx, wrap_idx, d_out, n, stream),
     "launch_trunc_postproc_kernel");
}

void launch_horner_cubic_kernel(const uint64_t* d_x, const uint64_t* d_c0, const uint64_t* d_c1, const uint64_t* d_c2,
                                const uint64_t* d_c3, uint64_t* d_out, size_t n, void* stream) {
  ok(sufb200_horner_cubic(d_x, d_c0, d_c1, d_c2, d_c3, d_out, n, stream), "launch_horner_cubic_kernel");
}

void launch_add_rout_aos_kernel(uint64_t* d_out, size_t elems, int out_words, const uint64_t* r_out,
                                size_t r_out_words, void* stream) {
  ok(sufb200_add_rout_aos(d_out, elems, out_words, r_out, r_out_words, stream), "launch_add_rout_aos_kernel");
}

void launch_row_broadcast_mul_kernel(int party, const uint64_t* d_A, const uint64_t* d_B_rows, const uint64_t* d_C,
                                     const uint64_t* d_d_open, const uint64_t* d_e_open_rows, int rows, int cols,
                                     const int* d_valid_lens, uint64_t* d_out, size_t /*n*/, void* stream) {
  ok(sufb200_row_broadcast_mul(party, d_A, d_B_rows, d_C, d_d_open, d_e_open_rows, rows, cols, d_valid_lens, d_out,
                               stream),
     "launch_row_broadcast_mul_kernel");
}

void launch_row_sum_kernel(const uint64_t* d_mat, int rows, int cols, const int* d_valid_lens, uint64_t* d_out_rows,
                           void* stream) {
  ok(sufb200_row_sum(d_mat, rows, cols, d_valid_lens, d_out_rows, stream), "launch_row_sum_kernel");
}

void launch_row_sum_ragged_kernel(const uint64_t* d_vals, const int* d_row_offsets, int rows, uint64_t* d_out_rows,
                                  void* stream) {
  ok(sufb200_row_sum_ragged(d_vals, d_row_offsets, rows, d_out_rows, stream), "launch_row_sum_ragged_kernel");
}

void launch_beaver_matmul2d_batched_kernel(int party, const uint64_t* d_D_open, const uint64_t* d_E_open,
                                           const uint64_t* d_A_tri_share, const uint64_t* d_B_tri_share,
                                           const uint64_t* d_C_tri_share, int batches, int M, int K, int N,
                                           int w_transposed, int has_scale, int64_t mul_const, int mul_shift,
                                           uint64_t* d_out, void* stream) {
  // The tensor-core form (tcgen05, exact up to contraction depth 2K = 8192)
  // needs an engine context; the launchers have none in their signature, so
  // one per device is made at the first call and kept for the process.  A
  // deeper contraction takes the CUDA-core kernel.
  if (sufb200_ctx ctx = (2 * static_cast<long long>(K) <= 8192) ? device_ctx() : nullptr) {
    ok(sufb200_beaver_matmul2d_tc(ctx, party, d_D_open, d_E_open, d_A_tri_share, d_B_tri_share, d_C_tri_share, batches,
                                  M, K, N, w_transposed, has_scale, mul_const, mul_shift, d_out, stream),
       "launch_beaver_matmul2d_kernel");
    return;
  }
  ok(sufb200_beaver_matmul2d(party, d_D_open, d_E_open, d_A_tri_share, d_B_tri_share, d_C_tri_share, batches, M, K,
                             N, w_transposed, has_scale, mul_const, mul_shift, d_out, stream),
     "launch_beaver_matmul2d_kernel");
}

void launch_beaver_matmul2d_kernel(int party, const uint64_t* d_D_open, const uint64_t* d_E_open,
                                   const uint64_t* d_A_tri_share, const uint64_t* d_B_tri_share,
                                   const uint64_t* d_C_tri_share, int M, int K, int N, int w_transposed,
                                   int has_scale, int64_t mul_const, int mul_shift, uint64_t* d_out, void* stream) {
  launch_beaver_matmul2d_batched_kernel(party, d_D_open, d_E_open, d_A_tri_share, d_B_tri_share, d_C_tri_share, 1, M,
                                        K, N, w_transposed, has_scale, mul_const, mul_shift, d_out, stream);
}

void launch_row_mean_kernel(const uint64_t* d_mat, int rows, int cols, const int* d_valid_lens, uint64_t* d_out_rows,
                            void* stream) {
  ok(sufb200_row_mean(d_mat, rows, cols, d_valid_lens, d_out_rows, stream), "launch_row_mean_kernel");
}

void launch_row_variance_kernel(const uint64_t* d_mat, const uint64_t* d_mean, int rows, int cols,
                                const int* d_valid_lens, uint64_t* d_out_rows, void* stream) {
  ok(sufb200_row_variance(d_mat, d_mean, rows, cols, d_valid_lens, d_out_rows, stream), "launch_row_variance_kernel");
}

void launch_unpack_eff_bits_kernel(const uint64_t* d_packed, int eff_bits, uint64_t* d_out, size_t n, void* stream) {
  ok(sufb200_unpack_eff_bits(d_packed, eff_bits, d_out, n, stream), "launch_unpack_eff_bits_kernel");
}

void launch_pack_eff_bits_kernel(const uint64_t* d_in, int eff_bits, uint64_t* d_packed, size_t n, void* stream) {
  ok(sufb200_pack_eff_bits(d_in, eff_bits, d_packed, n, stream), "launch_pack_eff_bits_kernel");
}

void launch_open_add_to_signed_kernel(const uint64_t* d_local_share, const uint64_t* d_remote_share,
                                      uint64_t* d_out_signed, size_t n, int ring_bits, uint64_t /*ring_mask*/,
                                      void* stream) {
  ok(sufb200_open_add_to_signed(d_local_share, d_remote_share, d_out_signed, n, ring_bits, stream),
     "launch_open_add_to_signed_kernel");
}

void launch_unpack_add_to_signed_kernel(const uint64_t* d_local_share, const uint64_t* d_packed_remote, int eff_bits,
                                        uint64_t* d_out_signed, size_t n, int ring_bits, uint64_t /*ring_mask*/,
                                        void* stream) {
  ok(sufb200_unpack_add_to_signed(d_local_share, d_packed_remote, eff_bits, d_out_signed, n, ring_bits, stream),
     "launch_unpack_add_to_signed_kernel");
}

void launch_unpack_add_mod_kernel(const uint64_t* d_local_share, const uint64_t* d_packed_remote, int eff_bits,
                                  uint64_t* d_out_mod, size_t n, int ring_bits, uint64_t /*ring_mask*/, void* stream) {
  ok(sufb200_unpack_add_mod(d_local_share, d_packed_remote, eff_bits, d_out_mod, n, ring_bits, stream),
     "launch_unpack_add_mod_kernel");
}

}  // extern "C"
