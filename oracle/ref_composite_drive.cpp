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
// of the same gate.  Prints "OK" on success.
#include <condition_variable>
#include <cstdio>
#include <cstdlib>
#include <mutex>
#include <queue>
#include <thread>
#include <vector>

#include "gates/composite_fss.hpp"
#include "gates/postproc_hooks.hpp"
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
  std::printf("OK\n");
  return 0;
}
