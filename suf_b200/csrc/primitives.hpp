// primitives.hpp -- launchers of the elementwise / row kernels (primitives.cu).
#pragma once

#include <cstddef>
#include <cstdint>

#include <cuda_runtime.h>

namespace sufb200 {

cudaError_t prim_beaver_mul(int sm, int party, const uint64_t* a, const uint64_t* b, const uint64_t* c,
                            const uint64_t* d, const uint64_t* e, uint64_t* z, size_t n, cudaStream_t st);
cudaError_t prim_beaver_mul_aos(int sm, int party, const uint64_t* tri, const uint64_t* d, const uint64_t* e,
                                uint64_t* z, size_t n, cudaStream_t st);
cudaError_t prim_horner_cubic(int sm, const uint64_t* x, const uint64_t* c0, const uint64_t* c1, const uint64_t* c2,
                              const uint64_t* c3, uint64_t* out, size_t n, cudaStream_t st);
cudaError_t prim_trunc_postproc(int sm, int party, int kind_gapars, int f, uint64_t r_hi, uint64_t m,
                                const uint64_t* hatx, const uint64_t* arith, size_t arith_stride, int arith_idx,
                                const uint64_t* bools, size_t bool_stride, int carry_idx, int sign_idx, int wrap_idx,
                                uint64_t* out, size_t n, cudaStream_t st);
cudaError_t prim_add_rout_aos(int sm, uint64_t* out, size_t elems, int out_words, const uint64_t* r_out,
                              size_t r_out_words, cudaStream_t st);
cudaError_t prim_row_sum(int sm, const uint64_t* mat, int rows, int cols, const int* valid, uint64_t* out,
                         cudaStream_t st);
cudaError_t prim_row_variance(int sm, const uint64_t* mat, const uint64_t* mean, int rows, int cols, const int* valid,
                              uint64_t* out, cudaStream_t st);
cudaError_t prim_row_sum_ragged(int sm, const uint64_t* vals, const int* offs, int rows, uint64_t* out,
                                cudaStream_t st);
cudaError_t prim_row_broadcast_mul(int sm, int party, const uint64_t* A, const uint64_t* B, const uint64_t* C,
                                   const uint64_t* d, const uint64_t* e, int rows, int cols, const int* valid,
                                   uint64_t* out, cudaStream_t st);
size_t packed_word_count(size_t n, int b);
cudaError_t prim_pack_eff_bits(int sm, const uint64_t* in, int b, uint64_t* packed, size_t n, cudaStream_t st);
cudaError_t prim_unpack_eff_bits(int sm, const uint64_t* packed, int b, uint64_t* out, size_t n, cudaStream_t st);
cudaError_t prim_unpack_add_mod(int sm, const uint64_t* local, const uint64_t* packed, int b, uint64_t* out, size_t n,
                                int ring_bits, cudaStream_t st);

cudaError_t prim_beaver_matmul(int party, const uint64_t* D, const uint64_t* E, const uint64_t* A, const uint64_t* B,
                               const uint64_t* C, int batches, int M, int K, int N, int w_transposed, int has_scale,
                               int64_t mul_const, int mul_shift, uint64_t* out, cudaStream_t st);
cudaError_t prim_row_mean(int sm, const uint64_t* mat, int rows, int cols, const int* valid, uint64_t* out,
                          cudaStream_t st);
cudaError_t prim_open_add_to_signed(int sm, const uint64_t* local, const uint64_t* remote, uint64_t* out, size_t n,
                                    int ring_bits, cudaStream_t st);
cudaError_t prim_unpack_add_to_signed(int sm, const uint64_t* local, const uint64_t* packed, int b, uint64_t* out,
                                      size_t n, int ring_bits, cudaStream_t st);
cudaError_t prim_trunc_shift(int sm, const uint64_t* in, uint64_t* out, int f, size_t n, cudaStream_t st);

}  // namespace sufb200
