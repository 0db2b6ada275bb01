// ops_harness.cpp -- the hot-path operations timed through the reference's own
// backend interfaces, on whichever backend this binary is linked with:
// proto::make_real_gpu_backend() and the runtime::launch_* primitives ABI
// (include/runtime/cuda_primitives.hpp).  Linked with the reference's
// cuda_pfss it times the reference's GPU build (its kernels compiled for
// sm_100a); linked with libsufb200, the adapter and the primitives shim it
// times this engine behind the same calls.
//
// Operations, at the configs' shapes, x^ staged on the device (the runtime's
// PfssGpuStagedEval path) and results left on the device:
//   dcf      eval_dcf_many_u64_device_broadcast, 64-bit compare, N = 2^20
//   packed   eval_packed_lt_many_device_broadcast, 16 thresholds, N = 2^20
//   lut      eval_interval_lut_many_device_broadcast, 20 intervals x 4 words,
//            N = 393,216 (the configs[2] SiLU gate's shape)
//   postproc launch_trunc_postproc_kernel, GapARS, N = 2^22
//   matmul   launch_beaver_matmul2d_kernel, 128 x 768 x 3072 (FFN1)
//   rowsum   launch_row_sum_kernel, 1,536 rows x 128
// Each: 3 warm-up calls, then --reps calls timed with CUDA events on the
// stream the call runs on (mean per call).  Prints one JSON line.
#include <cuda_runtime.h>

#include <algorithm>
#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <functional>
#include <memory>
#include <random>
#include <stdexcept>
#include <string>
#include <vector>

#include "proto/backend_gpu.hpp"
#include "proto/packed_backend.hpp"
#include "proto/pfss_backend_batch.hpp"
#include "proto/pfss_interval_lut_ext.hpp"
#include "runtime/cuda_primitives.hpp"

namespace {

void ck(cudaError_t e, const char* what) {
  if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

template <typename T>
T* dev_copy(const std::vector<T>& v) {
  T* p = nullptr;
  ck(cudaMalloc(&p, v.size() * sizeof(T)), "cudaMalloc");
  ck(cudaMemcpy(p, v.data(), v.size() * sizeof(T), cudaMemcpyHostToDevice), "H2D");
  return p;
}

// Mean per call of `reps` calls: the device span between CUDA events on the
// call's stream, and the host wall clock to completion (a backend whose calls
// synchronise shows its host gaps in both).
struct Timing {
  double dev_us, wall_us;
};

Timing time_us(cudaStream_t st, int reps, const std::function<void()>& call) {
  for (int i = 0; i < 3; i++) call();
  ck(cudaStreamSynchronize(st), "warm-up sync");
  cudaEvent_t a, b;
  ck(cudaEventCreate(&a), "event");
  ck(cudaEventCreate(&b), "event");
  const auto t0 = std::chrono::steady_clock::now();
  ck(cudaEventRecord(a, st), "record");
  for (int i = 0; i < reps; i++) call();
  ck(cudaEventRecord(b, st), "record");
  ck(cudaEventSynchronize(b), "sync");
  const double wall = std::chrono::duration<double, std::micro>(std::chrono::steady_clock::now() - t0).count();
  float ms = 0;
  ck(cudaEventElapsedTime(&ms, a, b), "elapsed");
  cudaEventDestroy(a);
  cudaEventDestroy(b);
  return {1e3 * ms / reps, wall / reps};
}

std::vector<uint8_t> bits_msb(uint64_t x, int n) {
  std::vector<uint8_t> v(n);
  for (int i = 0; i < n; i++) v[i] = static_cast<uint8_t>((x >> (n - 1 - i)) & 1);
  return v;
}

}  // namespace

int main(int argc, char** argv) {
  try {
    int reps = 10;
    for (int i = 1; i < argc; i++)
      if (std::strncmp(argv[i], "--reps=", 7) == 0) reps = std::atoi(argv[i] + 7);
    std::mt19937_64 g(7);
    auto be = proto::make_real_gpu_backend();
    auto* staged = dynamic_cast<proto::PfssGpuStagedEval*>(be.get());
    auto* packed = dynamic_cast<proto::PackedLtBackend*>(be.get());
    auto* lut = dynamic_cast<proto::PfssIntervalLutExt*>(be.get());
    if (!staged || !packed || !lut) throw std::runtime_error("backend lacks the staged / packed / LUT interfaces");
    cudaStream_t st = reinterpret_cast<cudaStream_t>(staged->device_stream());
    std::printf("{\"reps\": %d", reps);

    // dcf: broadcast 64-bit compare
    {
      const size_t n = size_t{1} << 20;
      std::vector<uint64_t> x(n);
      for (auto& v : x) v = g();
      uint64_t* dx = dev_copy(x);
      std::vector<uint8_t> pay(8, 0);
      pay[0] = 1;
      auto kp = be->gen_dcf(64, bits_msb(g(), 64), pay);
      const auto& k = kp.k0.bytes;
      staged->ensure_output_buffers(n, n);
      const Timing us = time_us(st, reps, [&] {
        staged->eval_dcf_many_u64_device_broadcast(64, k.size(), k.data(), dx, n, 8, nullptr);
      });
      std::printf(", \"dcf_us\": %.2f, \"dcf_wall_us\": %.2f, \"dcf_n\": %zu, \"dcf_key_bytes\": %zu", us.dev_us, us.wall_us, n, k.size());
      cudaFree(dx);
    }
    // packed compare: 16 thresholds
    {
      const size_t n = size_t{1} << 20;
      std::vector<uint64_t> x(n), thr(16);
      for (auto& v : x) v = g();
      for (auto& v : thr) v = g();
      std::sort(thr.begin(), thr.end());
      uint64_t* dx = dev_copy(x);
      auto kp = packed->gen_packed_lt(64, thr);
      const auto& k = kp.k0.bytes;
      staged->ensure_output_buffers(n, n);
      const Timing us = time_us(st, reps, [&] {
        staged->eval_packed_lt_many_device_broadcast(k.size(), k.data(), dx, n, 64, 1, nullptr);
      });
      std::printf(", \"packed_us\": %.2f, \"packed_wall_us\": %.2f, \"packed_n\": %zu", us.dev_us, us.wall_us, n);
      cudaFree(dx);
    }
    // interval LUT: 20 intervals x 4 words (the SiLU gate's shape)
    {
      const size_t n = 393216;
      std::vector<uint64_t> x(n);
      for (auto& v : x) v = g();
      proto::IntervalLutDesc d;
      d.in_bits = 64;
      d.out_words = 4;
      d.cutpoints.resize(21);
      for (auto& v : d.cutpoints) v = g() >> 1;
      std::sort(d.cutpoints.begin(), d.cutpoints.end());
      d.cutpoints.front() = 0;
      d.cutpoints.back() = ~0ull;
      d.payload_flat.resize(20 * 4);
      for (auto& v : d.payload_flat) v = g();
      uint64_t* dx = dev_copy(x);
      auto kp = lut->gen_interval_lut(d);
      const auto& k = kp.k0.bytes;
      staged->ensure_output_buffers(4 * n, n);
      const Timing us = time_us(st, reps, [&] {
        staged->eval_interval_lut_many_device_broadcast(k.size(), k.data(), dx, n, 4, nullptr);
      });
      std::printf(", \"lut_us\": %.2f, \"lut_wall_us\": %.2f, \"lut_n\": %zu", us.dev_us, us.wall_us, n);
      cudaFree(dx);
    }
    // trunc postproc: GapARS over 2^22 elements
    {
      const size_t n = size_t{1} << 22;
      std::vector<uint64_t> x(n), ar(n), bo(2 * n);
      for (auto& v : x) v = g();
      for (auto& v : ar) v = g();
      for (auto& v : bo) v = g() & 1;
      uint64_t *dx = dev_copy(x), *da = dev_copy(ar), *db = dev_copy(bo), *dout = nullptr;
      ck(cudaMalloc(&dout, n * 8), "cudaMalloc");
      const Timing us = time_us(st, reps, [&] {
        launch_trunc_postproc_kernel(0, 1, 12, g(), g(), dx, da, 1, 0, db, 2, 0, -1, 1, dout, n, st);
      });
      std::printf(", \"postproc_us\": %.2f, \"postproc_wall_us\": %.2f, \"postproc_n\": %zu", us.dev_us, us.wall_us, n);
      cudaFree(dx);
      cudaFree(da);
      cudaFree(db);
      cudaFree(dout);
    }
    // Beaver matmul, FFN1 shape
    {
      const int M = 128, K = 768, N = 3072;
      std::vector<uint64_t> D(size_t(M) * K), E(size_t(K) * N), A(size_t(M) * K), B(size_t(K) * N), Cm(size_t(M) * N);
      for (auto* v : {&D, &E, &A, &B, &Cm})
        for (auto& w : *v) w = g();
      uint64_t *dD = dev_copy(D), *dE = dev_copy(E), *dA = dev_copy(A), *dB = dev_copy(B), *dC = dev_copy(Cm),
               *dO = nullptr;
      ck(cudaMalloc(&dO, size_t(M) * N * 8), "cudaMalloc");
      const Timing us = time_us(st, reps, [&] {
        launch_beaver_matmul2d_kernel(0, dD, dE, dA, dB, dC, M, K, N, 0, 0, 0, 0, dO, st);
      });
      std::printf(", \"matmul_us\": %.2f, \"matmul_wall_us\": %.2f, \"matmul_shape\": \"%dx%dx%d\"", us.dev_us, us.wall_us, M, K, N);
      for (auto* p : {dD, dE, dA, dB, dC, dO}) cudaFree(p);
    }
    // row sums: 1,536 rows of 128
    {
      const int rows = 1536, cols = 128;
      std::vector<uint64_t> m(size_t(rows) * cols);
      for (auto& v : m) v = g();
      uint64_t *dm = dev_copy(m), *dr = nullptr;
      ck(cudaMalloc(&dr, rows * 8), "cudaMalloc");
      const Timing us = time_us(st, reps, [&] { launch_row_sum_kernel(dm, rows, cols, nullptr, dr, st); });
      std::printf(", \"rowsum_us\": %.2f, \"rowsum_wall_us\": %.2f", us.dev_us, us.wall_us);
      cudaFree(dm);
      cudaFree(dr);
    }
    ck(cudaStreamSynchronize(st), "final sync");
    std::printf("}\n");
    return 0;
  } catch (const std::exception& e) {
    std::fprintf(stderr, "ops_harness: %s\n", e.what());
    return 1;
  }
}
