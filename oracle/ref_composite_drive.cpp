// ref_composite_drive.cpp -- TEST INFRASTRUCTURE: the reference's own
// composite-FSS truncation pipeline driven through the B200 engine.
//
// Built by oracle/Makefile (target `drive`) from the reference's sources where
// they lie (include/gates/composite_fss.hpp, src/compiler/suf_to_pfss.cpp,
// src/gates/postproc_hooks.cpp, src/runtime/bench_accounting.cpp) plus this
// repository's adapter (suf_b200/host) and libsufb200.so; output goes to
// oracle/_ref/.  For FaithfulTR, FaithfulARS and GapARS it runs, unchanged:
//   composite_gen_trunc_gate(backend, ...)            keygen through our gen_dcf
//   composite_eval_batch_with_postproc(party, ...)    both parties on threads,
//                                                     once with host x^ and once
//                                                     with x^ staged on the device
// with proto::SufB200Backend as the backend, and checks the reconstruction
// against plaintext truncation and against the reference's ClearBackend run
// of the same gate.  Then the SiLU spline gate: the reference's composite
// eval of both parties (interval-LUT coefficients) checked against
// eval_suf_ref, and against the fused sufb200_coeff_lut_eval per party.
// Prints "OK" on success.
#include <condition_variable>
#include <cstdio>
#include <cstdlib>
#include <mutex>
#include <queue>
#include <thread>
#include <vector>

#include "gates/composite_fss.hpp"
#include "gates/postproc_hooks.hpp"
#include "gates/silu_spline_gate.hpp"
#include "suf/ref_eval.hpp"
#include "suf/suf_silu_builders.hpp"
#include "proto/backend_clear.hpp"
#include "proto/channel.hpp"
#include "sufb200_backend.hpp"

namespace {

struct QueueChan : proto::IChannel {
  struct Shared {
    std::mutex m;
    std::condition_variable cv;
    std::queue<std::vector<uint8_t>> q[2];
  };
  Shared* s;
  int me;
  QueueChan(Shared* sh, int p) : s(sh), me(p) {}
  void send_bytes(const void* data, size_t n) override {
    std::vector<uint8_t> b(static_cast<const uint8_t*>(data), static_cast<const uint8_t*>(data) + n);
    std::lock_guard<std::mutex> lk(s->m);
    s->q[1 - me].push(std::move(b));
    s->cv.notify_all();
  }
  void recv_bytes(void* data, size_t n) override {
    std::unique_lock<std::mutex> lk(s->m);
    s->cv.wait(lk, [&] { return !s->q[me].empty(); });
    auto b = std::move(s->q[me].front());
    s->q[me].pop();
    if (b.size() != n) throw std::runtime_error("QueueChan: size mismatch");
    std::memcpy(data, b.data(), n);
  }
};

std::unique_ptr<gates::PostProcHook> make_hook(compiler::GateKind kind, int f) {
  if (kind == compiler::GateKind::FaithfulTR) {
    auto h = std::make_unique<gates::FaithfulTruncPostProc>();
    h->f = f;
    return h;
  }
  if (kind == compiler::GateKind::FaithfulARS) {
    auto h = std::make_unique<gates::FaithfulArsPostProc>();
    h->f = f;
    return h;
  }
  auto h = std::make_unique<gates::GapArsPostProc>();
  h->f = f;
  return h;
}

// Both parties of one composite gate; returns y0 + y1 - r_out.
std::vector<uint64_t> run_pair(proto::PfssBackendBatch& b0, proto::PfssBackendBatch& b1,
                               const gates::CompositeKeyPair& kp, const suf::SUF<uint64_t>& F,
                               compiler::GateKind kind, int f, const std::vector<uint64_t>& hatx,
                               const uint64_t* hatx_dev) {
  QueueChan::Shared sh;
  QueueChan c0(&sh, 0), c1(&sh, 1);
  gates::CompositeBatchInput in{hatx.data(), hatx.size(), hatx_dev};
  auto h0 = make_hook(kind, f), h1 = make_hook(kind, f);
  gates::CompositeBatchOutput o0, o1;
  std::exception_ptr err;
  std::thread t([&] {
    try {
      o1 = gates::composite_eval_batch_with_postproc(1, b1, c1, kp.k1, F, in, *h1);
    } catch (...) {
      err = std::current_exception();
    }
  });
  o0 = gates::composite_eval_batch_with_postproc(0, b0, c0, kp.k0, F, in, *h0);
  t.join();
  if (err) std::rethrow_exception(err);
  const uint64_t rout = kp.k0.r_out_share[0] + kp.k1.r_out_share[0];
  std::vector<uint64_t> rec(hatx.size());
  for (size_t i = 0; i < hatx.size(); i++) rec[i] = o0.haty_share[i] + o1.haty_share[i] - rout;
  return rec;
}

// The SiLU spline gate (configs[2], f = 12): the reference's composite eval of
// both parties on the adapter (interval-LUT coefficient mode), checked
// against eval_suf_ref, and each party's output against the fused
// sufb200_coeff_lut_eval on the same key, r_out share and device x^.
bool run_silu(uint64_t seed, size_t n) {
  auto spec = gates::make_silu_spec({12, 16});
  auto F = suf::build_silu_suf_from_piecewise(spec);
  proto::SufB200Backend::Options o;
  o.deterministic = true;
  o.seed = seed * 131;
  proto::SufB200Backend gen(o), b0(o), b1(o);
  std::mt19937_64 rng(seed);
  const uint64_t r_in = rng();
  std::vector<uint64_t> r_out(static_cast<size_t>(F.r_out));
  for (auto& v : r_out) v = rng();
  auto kp = gates::composite_gen_backend_with_masks(F, gen, rng, r_in, r_out, n, compiler::GateKind::SiLUSpline);
  std::mt19937_64 xr(seed + 7);
  std::normal_distribution<double> nd(0.0, 4.0);
  std::vector<uint64_t> x(n), hatx(n);
  for (size_t i = 0; i < n; i++) {
    x[i] = static_cast<uint64_t>(static_cast<int64_t>(std::llround(nd(xr) * 4096.0)));
    hatx[i] = x[i] + r_in;
  }
  uint64_t* d_hatx = nullptr;
  uint64_t* d_y = nullptr;
  if (cudaMalloc(&d_hatx, n * 8) != cudaSuccess || cudaMalloc(&d_y, n * 32) != cudaSuccess ||
      cudaMemcpy(d_hatx, hatx.data(), n * 8, cudaMemcpyHostToDevice) != cudaSuccess) {
    std::fprintf(stderr, "silu: cuda setup failed\n");
    return false;
  }
  QueueChan::Shared sh;
  QueueChan c0(&sh, 0), c1(&sh, 1);
  gates::CompositeBatchInput in{hatx.data(), n, d_hatx};
  gates::CompositeBatchOutput o0, o1;
  std::exception_ptr err;
  std::thread t([&] {
    try {
      o1 = gates::composite_eval_batch_backend(1, b1, c1, kp.k1, F, in);
    } catch (...) {
      err = std::current_exception();
    }
  });
  o0 = gates::composite_eval_batch_backend(0, b0, c0, kp.k0, F, in);
  t.join();
  if (err) std::rethrow_exception(err);
  bool ok = o0.haty_share.size() == n * 4 && o1.haty_share.size() == n * 4;
  for (size_t i = 0; ok && i < n; i++) {
    const auto ref = suf::eval_suf_ref(F, x[i]);
    for (int j = 0; j < 4; j++) {
      const uint64_t rec = o0.haty_share[i * 4 + j] + o1.haty_share[i * 4 + j] - r_out[static_cast<size_t>(j)];
      if (rec != ref.arith[static_cast<size_t>(j)]) {
        std::fprintf(stderr, "silu: reconstruction differs at %zu/%d\n", i, j);
        ok = false;
        break;
      }
    }
  }
  sufb200_ctx ctx = nullptr;
  ok = ok && sufb200_ctx_create(0, &ctx) == SUFB200_OK;
  for (int p = 0; ok && p < 2; p++) {
    const auto& k = p ? kp.k1 : kp.k0;
    const auto& out = p ? o1 : o0;
    std::vector<uint64_t> y(n * 4);
    ok = sufb200_coeff_lut_eval(ctx, k.coeff_keys[0].bytes.data(), k.coeff_keys[0].bytes.size(), d_hatx, n, 4, 0,
                                k.r_out_share.data(), 64, 0, d_y, nullptr) == SUFB200_OK &&
         sufb200_ctx_sync(ctx, nullptr) == SUFB200_OK &&
         cudaMemcpy(y.data(), d_y, n * 32, cudaMemcpyDeviceToHost) == cudaSuccess;
    if (ok && y != out.haty_share) {
      std::fprintf(stderr, "silu: fused kernel differs from the composite output (party %d)\n", p);
      ok = false;
    }
  }
  if (ctx) sufb200_ctx_destroy(ctx);
  cudaFree(d_hatx);
  cudaFree(d_y);
  return ok;
}

}  // namespace

int main() {
  const int f = 12;
  const size_t n = 20000;
  for (auto kind : {compiler::GateKind::FaithfulTR, compiler::GateKind::FaithfulARS, compiler::GateKind::GapARS}) {
    for (uint64_t seed : {1ull, 2ull}) {
      proto::SufB200Backend::Options o;
      o.deterministic = true;
      o.seed = seed * 7919;
      proto::SufB200Backend gen(o), p0(o), p1(o);
      std::mt19937_64 rng(seed);
      suf::SUF<uint64_t> F;
      auto kp = gates::composite_gen_trunc_gate(gen, rng, f, kind, n, &F);
      proto::ClearBackend clear;
      std::mt19937_64 rng_c(seed);
      suf::SUF<uint64_t> Fc;
      auto kpc = gates::composite_gen_trunc_gate(clear, rng_c, f, kind, n, &Fc);
      if (kp.k0.compiled.r_in != kpc.k0.compiled.r_in) {
        std::fprintf(stderr, "r_in differs between backends\n");
        return 1;
      }
      std::mt19937_64 xr(seed + 100);
      std::vector<int64_t> plain(n);
      for (size_t i = 0; i < n; i++) plain[i] = static_cast<int64_t>(xr() % (1ull << 41)) - (1ll << 40);
      plain[0] = 0;
      plain[1] = -1;
      plain[2] = 1ll << f;
      std::vector<uint64_t> hatx(n);
      for (size_t i = 0; i < n; i++) hatx[i] = static_cast<uint64_t>(plain[i]) + kp.k0.compiled.r_in;
      uint64_t* d_hatx = nullptr;
      if (cudaMalloc(&d_hatx, n * 8) != cudaSuccess ||
          cudaMemcpy(d_hatx, hatx.data(), n * 8, cudaMemcpyHostToDevice) != cudaSuccess) {
        std::fprintf(stderr, "cuda setup failed\n");
        return 1;
      }
      auto rec_host = run_pair(p0, p1, kp, F, kind, f, hatx, nullptr);
      auto rec_dev = run_pair(p0, p1, kp, F, kind, f, hatx, d_hatx);
      auto rec_clear = run_pair(clear, clear, kpc, Fc, kind, f, hatx, nullptr);
      cudaFree(d_hatx);
      for (size_t i = 0; i < n; i++) {
        const uint64_t expect = kind == compiler::GateKind::FaithfulTR ? (static_cast<uint64_t>(plain[i]) >> f)
                                                                       : static_cast<uint64_t>(plain[i] >> f);
        if (rec_host[i] != expect || rec_dev[i] != expect || rec_clear[i] != expect) {
          std::fprintf(stderr, "kind=%d seed=%llu i=%zu plain=%lld host=%llu dev=%llu clear=%llu expect=%llu\n",
                       static_cast<int>(kind), static_cast<unsigned long long>(seed), i,
                       static_cast<long long>(plain[i]), static_cast<unsigned long long>(rec_host[i]),
                       static_cast<unsigned long long>(rec_dev[i]), static_cast<unsigned long long>(rec_clear[i]),
                       static_cast<unsigned long long>(expect));
          return 1;
        }
      }
    }
  }
  for (uint64_t seed : {3ull, 4ull}) {
    if (!run_silu(seed, 5000)) return 1;
  }
  std::printf("OK\n");
  return 0;
}
