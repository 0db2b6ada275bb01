// ref_softmax_drive.cpp -- TEST INFRASTRUCTURE: the reference's own softmax
// block run on the reference's CPU backend and on the B200
// engine, outputs compared bit for bit.
//
// Built by oracle/Makefile (target `softmax`) from the reference's sources
// where they lie (include/nn/softmax_block_task.hpp and the runtime it uses:
// src/runtime/{phase_executor,open_collector,pfss_superbatch,
// pfss_gpu_stager_cuda,bench_accounting}.cpp, src/compiler/suf_to_pfss.cpp,
// src/gates/postproc_hooks.cpp) plus this repository's adapter
// (suf_b200/host: proto::make_real_gpu_backend, the cuda_primitives.hpp
// launchers on libsufb200) and libsufb200.so; output goes to oracle/_ref/.
//
// Workload (configs[4] softmax): heads x 128 x 128 attention scores, causal
// (row r of a head has r % cols + 1 valid entries), Gaussian sigma 2.0 at
// f = 12 from mt19937_64(seed); the task's input is the per-row max
// difference t = max - x clamped to [0, 16] (SoftmaxPlan::input_is_max_diff),
// held by party 0 (party 1 holds zeros).  The dealer material is the
// reference's own: gates::dealer_make_nexp_task_material (nExp cubic,
// 16 segments), gates::dealer_make_recip_task_material (affine init + one
// Newton step), prob truncation by the recip material's trunc_fb, and
// row-broadcast Beaver triples made here.
//
// Both parties of each backend run on threads over an in-process channel,
// exactly as nn::SoftmaxBlockTask runs between two processes.  With
// --switches=1 (default) the second run sets the reference's GPU switches
// (SUF_TRUNC_GPU, SUF_MUL_GPU, SUF_RECIP_GPU_KERNELS, SUF_HORNER_GPU,
// SUF_PFSS_CACHE_KEYS/HATX), so its Beaver products, row sums and
// truncations go through the cuda_primitives launchers, i.e. our kernels;
// with --switches=0 only the PFSS gates run on the GPU.  Prints one JSON line
// with both wall times per block and whether the reconstructed probabilities
// are identical; --dump=PATH also writes the input t and the CPU backend's
// reconstruction (raw little-endian u64, rows*cols each).
#include <algorithm>
#include <chrono>
#include <cmath>
#include <condition_variable>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <deque>
#include <mutex>
#include <random>
#include <string>
#include <thread>
#include <vector>

#include "gates/nexp_composite.hpp"
#include "gates/reciprocal_composite.hpp"
#include "mpc/net.hpp"
#include "nn/softmax_block_task.hpp"
#include "proto/backend_gpu.hpp"
#include "proto/reference_backend.hpp"
#include "runtime/pfss_gpu_staging.hpp"
#include "runtime/phase_executor.hpp"
#include "runtime/pfss_superbatch.hpp"
#include "rsqrt_affine_suf.hpp"

namespace {

// Two one-way word pipes between the parties.
struct WordPipes {
  std::mutex m;
  std::condition_variable cv;
  std::deque<uint64_t> q[2];  // q[p]: words waiting for party p
};

struct PipeChan final : net::Chan {
  WordPipes* w;
  int me;
  PipeChan(WordPipes* pipes, int party) : w(pipes), me(party) {}
  void send_u64(uint64_t v) override { send_u64s(&v, 1); }
  uint64_t recv_u64() override {
    uint64_t v;
    recv_u64s(&v, 1);
    return v;
  }
  void send_u64s(const uint64_t* data, size_t n) override {
    std::lock_guard<std::mutex> lk(w->m);
    w->q[1 - me].insert(w->q[1 - me].end(), data, data + n);
    w->cv.notify_all();
  }
  void recv_u64s(uint64_t* data, size_t n) override {
    size_t got = 0;
    std::unique_lock<std::mutex> lk(w->m);
    while (got < n) {
      w->cv.wait(lk, [&] { return !w->q[me].empty(); });
      auto& q = w->q[me];
      const size_t take = std::min(n - got, q.size());
      std::copy(q.begin(), q.begin() + static_cast<std::ptrdiff_t>(take), data + got);
      q.erase(q.begin(), q.begin() + static_cast<std::ptrdiff_t>(take));
      got += take;
    }
  }
};

// Row-broadcast triples: A[rows][cols], B[rows], C = A * B[row], additively
// shared between the parties.
struct RowTriples {
  int rows = 0, cols = 0;
  std::vector<uint64_t> a[2], b[2], c[2];
  RowTriples(int r, int c_, uint64_t seed) : rows(r), cols(c_) {
    std::mt19937_64 g(seed);
    const size_t n = static_cast<size_t>(r) * static_cast<size_t>(c_);
    for (int p = 0; p < 2; p++) {
      a[p].resize(n);
      c[p].resize(n);
      b[p].resize(static_cast<size_t>(r));
    }
    for (int i = 0; i < r; i++) {
      const uint64_t bv = g(), b0 = g();
      b[0][i] = b0;
      b[1][i] = bv - b0;
      for (int j = 0; j < c_; j++) {
        const size_t k = static_cast<size_t>(i) * c_ + j;
        const uint64_t av = g(), a0 = g(), c0 = g();
        a[0][k] = a0;
        a[1][k] = av - a0;
        c[0][k] = c0;
        c[1][k] = av * bv - c0;
      }
    }
  }
};

struct RowTripleSource final : runtime::RowBroadcastTripleProvider {
  const RowTriples& t;
  int party;
  RowTripleSource(const RowTriples& tr, int p) : t(tr), party(p) {}
  runtime::RowBroadcastTriple reserve_mul(int rows, int cols) override {
    if (rows != t.rows || cols != t.cols) throw std::runtime_error("RowTripleSource: shape mismatch");
    return {std::span<const uint64_t>(t.a[party]), std::span<const uint64_t>(t.b[party]),
            std::span<const uint64_t>(t.c[party])};
  }
};

struct Workload {
  int rows, cols, fb;
  std::vector<int> valid;
  std::vector<uint64_t> t;  // max difference, Q(fb), zero outside the valid prefix
  std::vector<double> ref;  // double-precision softmax of the same scores
};

Workload make_workload(int heads, int len, int fb, uint64_t seed) {
  Workload w{heads * len, len, fb, {}, {}, {}};
  std::mt19937_64 g(seed);
  std::normal_distribution<double> nd(0.0, 2.0);
  const size_t n = static_cast<size_t>(w.rows) * len;
  w.t.assign(n, 0);
  w.ref.assign(n, 0.0);
  std::vector<double> x(static_cast<size_t>(len));
  for (int r = 0; r < w.rows; r++) {
    const int L = r % len + 1;
    w.valid.push_back(L);
    for (int c = 0; c < len; c++) x[c] = std::ldexp(std::nearbyint(std::ldexp(nd(g), fb)), -fb);
    const double mx = *std::max_element(x.begin(), x.begin() + L);
    double sum = 0.0;
    for (int c = 0; c < L; c++) {
      const double d = std::min(mx - x[c], 16.0);
      w.t[static_cast<size_t>(r) * len + c] = static_cast<uint64_t>(std::llround(std::ldexp(d, fb)));
      sum += std::exp(-d);
    }
    for (int c = 0; c < L; c++) w.ref[static_cast<size_t>(r) * len + c] = std::exp(-std::min(mx - x[c], 16.0)) / sum;
  }
  return w;
}

struct Material {
  gates::NexpTaskMaterial nexp;
  gates::RecipTaskMaterial recip;
};

Material deal(proto::PfssBackendBatch& be, const Workload& w, uint64_t seed) {
  std::mt19937_64 g(seed);
  const size_t n = static_cast<size_t>(w.rows) * w.cols;
  gates::NExpGateParams np{w.fb, 16};
  // CubicPolyTask's Beaver Horner draws three triples per element whenever the
  // compiled gate outputs coefficients (phase_tasks.hpp: Mul1..Mul3)
  auto nexp = gates::dealer_make_nexp_task_material(be, np, g, 3 * n, n);
  auto recip = gates::dealer_make_recip_task_material(be, w.fb, /*nr_iters=*/1, g, n);
  return Material{std::move(nexp), std::move(recip)};
}

std::vector<uint64_t> run_party(int party, proto::PfssBackendBatch& be, net::Chan& ch, const Workload& w,
                                const Material& mat, runtime::RowBroadcastTripleProvider* rt,
                                std::span<const uint64_t> t) {
  // A GPU backend gets the reference's CUDA stager, as its bench does in device
  // mode: the superbatch then stages x^ on the device and the composite driver
  // takes the broadcast-key device path (pfss_superbatch.cpp:306-339).  It is
  // declared before the executor, which holds a pointer to it.
  std::unique_ptr<runtime::CudaPfssStager> stager;
  if (auto* staged = dynamic_cast<proto::PfssGpuStagedEval*>(&be))
    stager = std::make_unique<runtime::CudaPfssStager>(staged->device_stream());
  runtime::PhaseExecutor pe;
  runtime::PhaseResources R{};
  runtime::ProtoChanFromNet pch(ch);
  R.party = party;
  R.pfss_backend = &be;
  R.pfss_chan = &pch;
  R.net_chan = &ch;
  R.pfss_coeff = &pe.pfss_coeff_batch();
  R.pfss_trunc = &pe.pfss_trunc_batch();
  R.opens = &pe.open_collector();
  if (stager) {
    pe.pfss_coeff_batch().set_gpu_stager(stager.get());
    pe.pfss_trunc_batch().set_gpu_stager(stager.get());
  }

  nn::SoftmaxPlan plan;
  plan.frac_bits = w.fb;
  plan.rows = w.rows;
  plan.cols = w.cols;
  plan.valid_lens = w.valid;
  plan.nexp = gates::make_nexp_cubic_bundle(mat.nexp, w.fb);
  plan.recip = gates::make_recip_bundle(mat.recip);
  plan.prob_trunc.gapars = &mat.recip.trunc_fb;
  plan.prob_trunc.faithful = &mat.recip.trunc_fb;
  plan.prob_trunc.shift_bits = w.fb;
  plan.prob_trunc.signed_value = false;
  plan.row_triples = rt;
  compiler::RangeInterval pr;
  pr.is_signed = true;
  pr.lo = 0;
  pr.hi = static_cast<int64_t>(1ll << w.fb);
  plan.prob_range = pr;

  std::vector<uint64_t> out(t.size(), 0);
  pe.begin_phase(runtime::PhaseExecutor::Phase::kSoftmax);
  pe.add_task(std::make_unique<nn::SoftmaxBlockTask>(plan, t, std::span<uint64_t>(out)));
  pe.run(R);
  return out;
}

// One block, both parties on threads; returns the reconstruction and the wall time.
std::vector<uint64_t> run_block(proto::PfssBackendBatch& be0, proto::PfssBackendBatch& be1, const Workload& w,
                                const Material& mat, const RowTriples& trip, double* ms) {
  WordPipes pipes;
  PipeChan c0(&pipes, 0), c1(&pipes, 1);
  RowTripleSource s0(trip, 0), s1(trip, 1);
  const std::vector<uint64_t> zeros(w.t.size(), 0);
  std::vector<uint64_t> y0, y1;
  std::exception_ptr e1;
  const auto t0 = std::chrono::steady_clock::now();
  std::thread th([&] {
    try {
      y1 = run_party(1, be1, c1, w, mat, &s1, std::span<const uint64_t>(zeros));
    } catch (...) {
      e1 = std::current_exception();
    }
  });
  y0 = run_party(0, be0, c0, w, mat, &s0, std::span<const uint64_t>(w.t));
  th.join();
  if (e1) std::rethrow_exception(e1);
  *ms = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
  std::vector<uint64_t> y(y0.size());
  for (size_t i = 0; i < y.size(); i++) y[i] = y0[i] + y1[i];
  return y;
}

// ---- LayerNorm (configs[4] second half): the reference's runtime::LayerNormTask

struct LnWorkload {
  int rows, cols, fb;
  std::vector<uint64_t> x;  // Q(fb), two's complement
  std::vector<double> ref;  // double-precision LayerNorm (eps 1/1024, no affine)
};

LnWorkload make_ln_workload(int rows, int cols, int fb, uint64_t seed) {
  LnWorkload w{rows, cols, fb, {}, {}};
  std::mt19937_64 g(seed);
  std::normal_distribution<double> nd(0.0, 1.0);
  w.x.resize(static_cast<size_t>(rows) * cols);
  w.ref.resize(w.x.size());
  for (int r = 0; r < rows; r++) {
    double s = 0, s2 = 0;
    for (int c = 0; c < cols; c++) {
      const int64_t q = std::llround(std::ldexp(nd(g), fb));
      w.x[static_cast<size_t>(r) * cols + c] = static_cast<uint64_t>(q);
      s += std::ldexp(static_cast<double>(q), -fb);
    }
    const double mu = s / cols;
    for (int c = 0; c < cols; c++) {
      const double d = std::ldexp(static_cast<double>(static_cast<int64_t>(w.x[static_cast<size_t>(r) * cols + c])), -fb) - mu;
      s2 += d * d;
    }
    const double inv = 1.0 / std::sqrt(s2 / cols + 1.0 / 1024.0);
    for (int c = 0; c < cols; c++) {
      const size_t k = static_cast<size_t>(r) * cols + c;
      w.ref[k] = (std::ldexp(static_cast<double>(static_cast<int64_t>(w.x[k])), -fb) - mu) * inv;
    }
  }
  return w;
}

struct LnMaterial {
  gates::PiecewisePolySpec spec;
  suf::SUF<uint64_t> suf;
  gates::CompositeKeyPair keys;
  compiler::TruncationLoweringResult trunc_f, trunc_2f, mean_t, var_t, norm_t;
  std::vector<proto::BeaverTriple64Share> mul[2];
};

compiler::TruncationLoweringResult lower(proto::PfssBackendBatch& be, std::mt19937_64& g, compiler::GateKind kind,
                                         int f, size_t n) {
  compiler::GateParams p;
  p.kind = kind;
  p.frac_bits = f;
  return compiler::lower_truncation_gate(be, g, p, n);
}

// Signed truncations throughout: the inputs are Gaussian (negative values),
// where a logical shift (FaithfulTR) of the mean or the normalised value
// would be wrong.
std::unique_ptr<LnMaterial> deal_ln(proto::PfssBackendBatch& be, const LnWorkload& w, uint64_t seed) {
  auto m = std::make_unique<LnMaterial>();
  std::mt19937_64 g(seed);
  const size_t R = static_cast<size_t>(w.rows), N = R * w.cols;
  m->spec = gates::make_rsqrt_affine_init_spec(w.fb, 1.0 / 1024.0, 16.0);
  m->suf = oracle_ref::rsqrt_affine_suf(m->spec);
  std::vector<uint64_t> r_out(2, 0ull);
  m->keys = gates::composite_gen_backend_with_masks(m->suf, be, g, g(), r_out, R, compiler::GateKind::Rsqrt);
  m->keys.k0.compiled.gate_kind = compiler::GateKind::Rsqrt;
  m->keys.k1.compiled.gate_kind = compiler::GateKind::Rsqrt;
  gates::ensure_beaver_triples(m->keys, 3 * R, g);  // RsqrtTask: y*y, x*y2, y*t per Newton step
  m->trunc_f = lower(be, g, compiler::GateKind::FaithfulARS, w.fb, R);
  m->trunc_2f = lower(be, g, compiler::GateKind::GapARS, 2 * w.fb, R);
  m->mean_t = lower(be, g, compiler::GateKind::FaithfulARS, w.fb, R);
  m->var_t = lower(be, g, compiler::GateKind::GapARS, 2 * w.fb, R);
  m->norm_t = lower(be, g, compiler::GateKind::FaithfulARS, w.fb, N);
  for (size_t i = 0; i < N; i++) {  // Beaver triples of diff^2
    const uint64_t a = g(), b = g(), c = a * b, a0 = g(), b0 = g(), c0 = g();
    m->mul[0].push_back({a0, b0, c0});
    m->mul[1].push_back({a - a0, b - b0, c - c0});
  }
  return m;
}

std::vector<uint64_t> run_ln_party(int party, proto::PfssBackendBatch& be, net::Chan& ch, const LnWorkload& w,
                                   const LnMaterial& m, runtime::RowBroadcastTripleProvider* rt,
                                   std::span<const uint64_t> x) {
  std::unique_ptr<runtime::CudaPfssStager> stager;
  if (auto* staged = dynamic_cast<proto::PfssGpuStagedEval*>(&be))
    stager = std::make_unique<runtime::CudaPfssStager>(staged->device_stream());
  runtime::PhaseExecutor pe;
  runtime::PhaseResources R{};
  runtime::ProtoChanFromNet pch(ch);
  R.party = party;
  R.pfss_backend = &be;
  R.pfss_chan = &pch;
  R.net_chan = &ch;
  R.pfss_coeff = &pe.pfss_coeff_batch();
  R.pfss_trunc = &pe.pfss_trunc_batch();
  R.opens = &pe.open_collector();
  if (stager) {
    pe.pfss_coeff_batch().set_gpu_stager(stager.get());
    pe.pfss_trunc_batch().set_gpu_stager(stager.get());
  }
  runtime::LayerNormTaskBundle b{};
  b.mean_trunc = {nullptr, &m.mean_t, w.fb, true};
  b.var_trunc = {nullptr, &m.var_t, 2 * w.fb, true};
  b.norm_trunc = {nullptr, &m.norm_t, w.fb, true};
  b.rsqrt = runtime::RsqrtTaskBundle{&m.suf, &m.keys.k0, &m.keys.k1, &m.trunc_f, &m.trunc_2f, &m.spec, w.fb, 1};
  b.inv_len_qf = static_cast<uint64_t>(std::llround(std::ldexp(1.0 / w.cols, w.fb)));
  b.eps_qf = static_cast<uint64_t>(std::llround(std::ldexp(1.0 / 1024.0, w.fb)));
  b.frac_bits = w.fb;
  b.mul_triples = std::span<const proto::BeaverTriple64Share>(m.mul[party]);
  b.row_triples = rt;
  std::vector<uint64_t> out(x.size(), 0);
  pe.add_task(std::make_unique<runtime::LayerNormTask>(b, x, std::span<uint64_t>(out), w.rows, w.cols));
  pe.run(R);
  return out;
}

std::vector<uint64_t> run_ln_block(proto::PfssBackendBatch& be0, proto::PfssBackendBatch& be1, const LnWorkload& w,
                                   const LnMaterial& m, const RowTriples& trip, double* ms) {
  WordPipes pipes;
  PipeChan c0(&pipes, 0), c1(&pipes, 1);
  RowTripleSource s0(trip, 0), s1(trip, 1);
  const std::vector<uint64_t> zeros(w.x.size(), 0);
  std::vector<uint64_t> y0, y1;
  std::exception_ptr e1;
  const auto t0 = std::chrono::steady_clock::now();
  std::thread th([&] {
    try {
      y1 = run_ln_party(1, be1, c1, w, m, &s1, std::span<const uint64_t>(zeros));
    } catch (...) {
      e1 = std::current_exception();
    }
  });
  y0 = run_ln_party(0, be0, c0, w, m, &s0, std::span<const uint64_t>(w.x));
  th.join();
  if (e1) std::rethrow_exception(e1);
  *ms = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
  std::vector<uint64_t> y(y0.size());
  for (size_t i = 0; i < y.size(); i++) y[i] = y0[i] + y1[i];
  return y;
}

double ln_max_err(const LnWorkload& w, const std::vector<uint64_t>& y) {
  double e = 0.0;
  for (size_t k = 0; k < y.size(); k++)
    e = std::max(e, std::fabs(std::ldexp(static_cast<double>(static_cast<int64_t>(y[k])), -w.fb) - w.ref[k]));
  return e;
}

double active_max_err(const Workload& w, const std::vector<uint64_t>& y) {
  double e = 0.0;
  for (int r = 0; r < w.rows; r++)
    for (int c = 0; c < w.valid[r]; c++) {
      const size_t k = static_cast<size_t>(r) * w.cols + c;
      e = std::max(e, std::fabs(std::ldexp(static_cast<double>(static_cast<int64_t>(y[k])), -w.fb) - w.ref[k]));
    }
  return e;
}

}  // namespace

void set_gpu_switches() {
  for (const char* k : {"SUF_PFSS_CACHE_KEYS", "SUF_PFSS_CACHE_HATX", "SUF_TRUNC_GPU", "SUF_MUL_GPU",
                        "SUF_RECIP_GPU_KERNELS", "SUF_HORNER_GPU"})
    setenv(k, "1", 0);
}

bool write_dump(const std::string& path, const std::vector<uint64_t>& a, const std::vector<uint64_t>& b) {
  FILE* fp = std::fopen(path.c_str(), "wb");
  return fp && std::fwrite(a.data(), 8, a.size(), fp) == a.size() && std::fwrite(b.data(), 8, b.size(), fp) == b.size() &&
         std::fclose(fp) == 0;
}

// --block=ln: the LayerNorm block, same legs and output as the softmax block.
int main_ln(int rows, int cols, int fb, int reps, uint64_t seed, const std::string& dump, bool cpu_only,
            bool switches) {
  const LnWorkload w = make_ln_workload(rows, cols, fb, seed);
  const RowTriples trip(rows, cols, seed * 7 + 1);
  proto::ReferenceBackend ref;
  const auto mref = deal_ln(ref, w, seed * 31 + 5);
  double ms = 0.0, ref_ms = 1e30;
  std::vector<uint64_t> yref;
  for (int i = 0; i < reps; i++) {
    yref = run_ln_block(ref, ref, w, *mref, trip, &ms);
    ref_ms = std::min(ref_ms, ms);
  }
  if (!dump.empty() && !write_dump(dump, w.x, yref)) {
    std::printf("{\"error\": \"cannot write %s\"}\n", dump.c_str());
    return 1;
  }
  if (cpu_only) {
    std::printf("{\"workload\": \"configs[4] layernorm block\", \"rows\": %d, \"cols\": %d, \"ref_cpu_ms\": %.3f, "
                "\"ref_max_err_vs_double\": %.6f}\n",
                rows, cols, ref_ms, ln_max_err(w, yref));
    return 0;
  }
  if (switches) set_gpu_switches();
  std::unique_ptr<proto::PfssBackendBatch> g0, g1;
  try {
    g0 = proto::make_real_gpu_backend();
    g1 = proto::make_real_gpu_backend();
  } catch (const std::exception& e) {
    std::printf("{\"workload\": \"configs[4] layernorm block\", \"rows\": %d, \"cols\": %d, \"ref_cpu_ms\": %.3f, "
                "\"ref_max_err_vs_double\": %.6f, \"sufb200\": \"%s\"}\n",
                rows, cols, ref_ms, ln_max_err(w, yref), e.what());
    return 3;
  }
  const auto mgpu = deal_ln(*g0, w, seed * 31 + 5);
  double gpu_ms = 1e30;
  std::vector<uint64_t> ygpu;
  for (int i = 0; i < reps + 1; i++) {
    ygpu = run_ln_block(*g0, *g1, w, *mgpu, trip, &ms);
    if (i > 0) gpu_ms = std::min(gpu_ms, ms);
  }
  size_t diff = 0;
  for (size_t k = 0; k < ygpu.size(); k++) diff += ygpu[k] != yref[k];
  std::printf("{\"workload\": \"configs[4] layernorm block\", \"rows\": %d, \"cols\": %d, \"ref_cpu_ms\": %.3f, "
              "\"sufb200_ms\": %.3f, \"identical\": %s, \"mismatches\": %zu, \"max_err_vs_double\": %.6f, "
              "\"ref_max_err_vs_double\": %.6f}\n",
              rows, cols, ref_ms, gpu_ms, diff == 0 ? "true" : "false", diff, ln_max_err(w, ygpu),
              ln_max_err(w, yref));
  return diff == 0 ? 0 : 2;
}

int main(int argc, char** argv) {
  int heads = 12, len = 128, fb = 12, reps = 3, switches = 1, rows = 128, cols = 768;
  bool ln = false;
  uint64_t seed = 4;
  std::string dump;  // --dump=PATH: t[rows*cols] then the CPU reconstruction, little-endian u64
  bool cpu_only = false;  // --cpu-only: the reference CPU leg alone (the B200 engine is not touched)
  for (int i = 1; i < argc; i++) {
    const std::string a(argv[i]);
    auto val = [&](const char* k) { return a.substr(std::strlen(k)); };
    if (a.rfind("--heads=", 0) == 0) heads = std::stoi(val("--heads="));
    else if (a.rfind("--len=", 0) == 0) len = std::stoi(val("--len="));
    else if (a.rfind("--fb=", 0) == 0) fb = std::stoi(val("--fb="));
    else if (a.rfind("--reps=", 0) == 0) reps = std::stoi(val("--reps="));
    else if (a.rfind("--seed=", 0) == 0) seed = std::stoull(val("--seed="));
    else if (a.rfind("--switches=", 0) == 0) switches = std::stoi(val("--switches="));
    else if (a.rfind("--dump=", 0) == 0) dump = val("--dump=");
    else if (a == "--cpu-only") cpu_only = true;
    else if (a == "--block=ln") ln = true;
    else if (a.rfind("--rows=", 0) == 0) rows = std::stoi(val("--rows="));
    else if (a.rfind("--cols=", 0) == 0) cols = std::stoi(val("--cols="));
  }
  if (ln) return main_ln(rows, cols, fb, reps, seed, dump, cpu_only, switches != 0);
  const Workload w = make_workload(heads, len, fb, seed);
  const RowTriples trip(w.rows, w.cols, seed * 7 + 1);
  size_t active = 0;
  for (int L : w.valid) active += static_cast<size_t>(L);

  // the reference's CPU backend
  proto::ReferenceBackend ref;
  const Material mref = deal(ref, w, seed * 31 + 5);
  double ms = 0.0, ref_ms = 1e30;
  std::vector<uint64_t> yref;
  for (int i = 0; i < reps; i++) {
    yref = run_block(ref, ref, w, mref, trip, &ms);
    ref_ms = std::min(ref_ms, ms);
  }
  if (!dump.empty()) {
    FILE* fp = std::fopen(dump.c_str(), "wb");
    if (!fp || std::fwrite(w.t.data(), 8, w.t.size(), fp) != w.t.size() ||
        std::fwrite(yref.data(), 8, yref.size(), fp) != yref.size() || std::fclose(fp) != 0) {
      std::printf("{\"error\": \"cannot write %s\"}\n", dump.c_str());
      return 1;
    }
  }

  // the B200 engine behind the reference's GPU factory; with --switches=1 the
  // reference's GPU switches route its Beaver products, Horner and
  // truncation postprocessing through the cuda_primitives launchers too
  if (switches)
    for (const char* k : {"SUF_PFSS_CACHE_KEYS", "SUF_PFSS_CACHE_HATX", "SUF_TRUNC_GPU", "SUF_MUL_GPU",
                          "SUF_RECIP_GPU_KERNELS", "SUF_HORNER_GPU"})
      setenv(k, "1", 0);
  if (cpu_only) {
    std::printf("{\"workload\": \"configs[4] softmax block\", \"rows\": %d, \"cols\": %d, \"active\": %zu, "
                "\"ref_cpu_ms\": %.3f, \"ref_max_err_vs_double\": %.6f}\n",
                w.rows, w.cols, active, ref_ms, active_max_err(w, yref));
    return 0;
  }
  std::unique_ptr<proto::PfssBackendBatch> g0, g1;
  try {
    g0 = proto::make_real_gpu_backend();
    g1 = proto::make_real_gpu_backend();
  } catch (const std::exception& e) {
    std::printf("{\"workload\": \"configs[4] softmax block\", \"rows\": %d, \"cols\": %d, \"active\": %zu, "
                "\"ref_cpu_ms\": %.3f, \"ref_max_err_vs_double\": %.6f, \"sufb200\": \"%s\"}\n",
                w.rows, w.cols, active, ref_ms, active_max_err(w, yref), e.what());
    return 3;
  }
  const Material mgpu = deal(*g0, w, seed * 31 + 5);
  double gpu_ms = 1e30;
  std::vector<uint64_t> ygpu;
  for (int i = 0; i < reps + 1; i++) {  // the first run warms the device (module load, pools)
    ygpu = run_block(*g0, *g1, w, mgpu, trip, &ms);
    if (i > 0) gpu_ms = std::min(gpu_ms, ms);
  }

  bool same = ygpu.size() == yref.size();
  size_t diff = 0;
  for (int r = 0; same && r < w.rows; r++)
    for (int c = 0; c < w.valid[r]; c++) {
      const size_t k = static_cast<size_t>(r) * w.cols + c;
      if (ygpu[k] != yref[k]) diff++;
    }
  same = same && diff == 0;
  std::printf(
      "{\"workload\": \"configs[4] softmax block\", \"rows\": %d, \"cols\": %d, \"active\": %zu, \"fb\": %d, "
      "\"gpu_switches\": %d, \"ref_cpu_ms\": %.3f, \"sufb200_ms\": %.3f, \"identical\": %s, \"mismatches\": %zu, "
      "\"max_err_vs_double\": %.6f, \"ref_max_err_vs_double\": %.6f}\n",
      w.rows, w.cols, active, fb, switches, ref_ms, gpu_ms, same ? "true" : "false", diff, active_max_err(w, ygpu),
      active_max_err(w, yref));
  return same ? 0 : 2;
}
