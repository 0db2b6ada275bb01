// test_backend.cpp -- the reference's GPU-backend test scenarios, run through
// proto::SufB200Backend (the drop-in adapter) instead of GpuPfssBackend:
//   src/demo/test_pfss_gpu.cpp:54-120        DCF alpha=5 / interval LUT
//   src/demo/test_cuda_packed_pfss.cpp:33-179 packed compare / vector LUT,
//                                              host and device-broadcast paths
//   src/demo/test_pfss_gpu.cpp:124-204         truncation {16,-8,3,-1}, f=4
// DCF shares are myl7 PRG-tree shares, so the checks reconstruct (the
// reference's party-0 == payload check is specific to its threshold blobs).
// Prints "OK" and exits 0 on success.
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <vector>

#include "sufb200_backend.hpp"

#define REQUIRE(c, ...)                     \
  do {                                      \
    if (!(c)) {                             \
      std::fprintf(stderr, __VA_ARGS__);    \
      std::fprintf(stderr, "\n");           \
      std::exit(1);                         \
    }                                       \
  } while (0)

static std::vector<uint8_t> pack_u64_le(uint64_t v) {
  std::vector<uint8_t> b(8);
  std::memcpy(b.data(), &v, 8);
  return b;
}

int main() {
  using namespace proto;
  SufB200Backend::Options opt;
  opt.deterministic = true;
  opt.seed = 12345;
  SufB200Backend be(opt);

  // DCF: alpha = 5, in_bits 6, payload 0xAA (1-byte, additive group)
  {
    auto kp = be.gen_dcf(6, be.u64_to_bits_msb(5, 6), {0xAA});
    for (uint64_t x : {3ull, 5ull, 7ull, 0ull, 4ull, 63ull}) {
      auto a = be.eval_dcf(6, kp.k0, be.u64_to_bits_msb(x, 6));
      auto b = be.eval_dcf(6, kp.k1, be.u64_to_bits_msb(x, 6));
      REQUIRE(a.size() == 1 && b.size() == 1, "dcf size");
      const uint8_t rec = static_cast<uint8_t>(a[0] + b[0]);
      REQUIRE(rec == (x < 5 ? 0xAA : 0), "dcf x=%llu rec=%u", (unsigned long long)x, rec);
    }
  }
  // batch DCF, per-element keys, AddU64 payload 1
  {
    const size_t n = 1000;
    std::mt19937_64 rng(7);
    std::vector<uint64_t> alphas(n), xs(n);
    std::vector<uint8_t> k0s, k1s;
    size_t kb = 0;
    for (size_t i = 0; i < n; i++) {
      alphas[i] = rng();
      xs[i] = (i % 3 == 0) ? alphas[i] : rng();
      auto kp = be.gen_dcf(64, be.u64_to_bits_msb(alphas[i], 64), pack_u64_le(1));
      kb = kp.k0.bytes.size();
      k0s.insert(k0s.end(), kp.k0.bytes.begin(), kp.k0.bytes.end());
      k1s.insert(k1s.end(), kp.k1.bytes.begin(), kp.k1.bytes.end());
    }
    std::vector<uint64_t> o0(n), o1(n);
    be.eval_dcf_many_u64(64, kb, k0s.data(), xs, 8, reinterpret_cast<uint8_t*>(o0.data()));
    be.eval_dcf_many_u64(64, kb, k1s.data(), xs, 8, reinterpret_cast<uint8_t*>(o1.data()));
    for (size_t i = 0; i < n; i++) REQUIRE(o0[i] + o1[i] == (xs[i] < alphas[i] ? 1u : 0u), "batch dcf i=%zu", i);
    // staged device path, broadcast key, result kept on the device
    uint64_t* d_xs = nullptr;
    REQUIRE(cudaMalloc(&d_xs, n * 8) == cudaSuccess, "cudaMalloc");
    REQUIRE(cudaMemcpy(d_xs, xs.data(), n * 8, cudaMemcpyHostToDevice) == cudaSuccess, "H2D");
    auto kp = be.gen_dcf(64, be.u64_to_bits_msb(alphas[1], 64), pack_u64_le(1));
    be.eval_dcf_many_u64_device_broadcast(64, kp.k0.bytes.size(), kp.k0.bytes.data(), d_xs, n, 8,
                                          reinterpret_cast<uint8_t*>(o0.data()));
    be.eval_dcf_many_u64_device_broadcast(64, kp.k1.bytes.size(), kp.k1.bytes.data(), d_xs, n, 8, nullptr);
    REQUIRE(cudaMemcpy(o1.data(), be.last_device_bools(), n * 8, cudaMemcpyDeviceToHost) == cudaSuccess, "D2H");
    for (size_t i = 0; i < n; i++) REQUIRE(o0[i] + o1[i] == (xs[i] < alphas[1] ? 1u : 0u), "bcast dcf i=%zu", i);
    cudaFree(d_xs);
  }
  // packed compare, host and device-broadcast paths
  {
    std::vector<uint64_t> thr = {5, 12, 33, 48, 60}, xs = {0, 15, 63};
    auto kp = be.gen_packed_lt(6, thr);
    const size_t kb = kp.k0.bytes.size();
    std::vector<uint8_t> f0, f1;
    for (size_t i = 0; i < xs.size(); i++) {
      f0.insert(f0.end(), kp.k0.bytes.begin(), kp.k0.bytes.end());
      f1.insert(f1.end(), kp.k1.bytes.begin(), kp.k1.bytes.end());
    }
    std::vector<uint64_t> o0(3), o1(3), b0(3), b1(3);
    be.eval_packed_lt_many(kb, f0.data(), xs, 6, 1, o0.data());
    be.eval_packed_lt_many(kb, f1.data(), xs, 6, 1, o1.data());
    uint64_t* d_xs = nullptr;
    REQUIRE(cudaMalloc(&d_xs, 24) == cudaSuccess, "cudaMalloc");
    REQUIRE(cudaMemcpy(d_xs, xs.data(), 24, cudaMemcpyHostToDevice) == cudaSuccess, "H2D");
    be.eval_packed_lt_many_device_broadcast(kb, kp.k0.bytes.data(), d_xs, 3, 6, 1, b0.data());
    be.eval_packed_lt_many_device_broadcast(kb, kp.k1.bytes.data(), d_xs, 3, 6, 1, b1.data());
    cudaFree(d_xs);
    for (size_t i = 0; i < 3; i++) {
      uint64_t expect = 0;
      for (size_t j = 0; j < thr.size(); j++) expect |= uint64_t(xs[i] < thr[j]) << j;
      REQUIRE((o0[i] ^ o1[i]) == expect, "packed i=%zu", i);
      REQUIRE((b0[i] ^ b1[i]) == expect, "packed bcast i=%zu", i);
    }
  }
  // interval LUTs: {0,32,64}/{10,20} and {0,20,40,64}/{100..600}, out_words 1 and 2
  {
    struct Case {
      std::vector<uint64_t> cuts, pay, xs;
      int ow;
    } cases[2] = {{{0, 32, 64}, {10, 20}, {0, 15, 40}, 1},
                  {{0, 20, 40, 64}, {100, 200, 300, 400, 500, 600}, {0, 25, 50}, 2}};
    for (auto& c : cases) {
      IntervalLutDesc d;
      d.in_bits = 6;
      d.out_words = c.ow;
      d.cutpoints = c.cuts;
      d.payload_flat = c.pay;
      auto kp = be.gen_interval_lut(d);
      const size_t kb = kp.k0.bytes.size();
      std::vector<uint8_t> f0, f1;
      for (size_t i = 0; i < c.xs.size(); i++) {
        f0.insert(f0.end(), kp.k0.bytes.begin(), kp.k0.bytes.end());
        f1.insert(f1.end(), kp.k1.bytes.begin(), kp.k1.bytes.end());
      }
      std::vector<uint64_t> o0(c.xs.size() * c.ow), o1(o0.size()), b0(o0.size()), b1(o0.size());
      be.eval_interval_lut_many_u64(kb, f0.data(), c.xs, c.ow, o0.data());
      be.eval_interval_lut_many_u64(kb, f1.data(), c.xs, c.ow, o1.data());
      uint64_t* d_xs = nullptr;
      REQUIRE(cudaMalloc(&d_xs, c.xs.size() * 8) == cudaSuccess, "cudaMalloc");
      REQUIRE(cudaMemcpy(d_xs, c.xs.data(), c.xs.size() * 8, cudaMemcpyHostToDevice) == cudaSuccess, "H2D");
      be.eval_interval_lut_many_device_broadcast(kb, kp.k0.bytes.data(), d_xs, c.xs.size(), c.ow, b0.data());
      be.eval_interval_lut_many_device_broadcast(kb, kp.k1.bytes.data(), d_xs, c.xs.size(), c.ow, b1.data());
      cudaFree(d_xs);
      for (size_t i = 0; i < c.xs.size(); i++) {
        size_t iv = 0;
        while (iv + 1 < c.cuts.size() - 1 && c.xs[i] >= c.cuts[iv + 1]) iv++;
        for (int w = 0; w < c.ow; w++) {
          const uint64_t e = c.pay[iv * c.ow + w];
          REQUIRE(o0[i * c.ow + w] + o1[i * c.ow + w] == e, "lut i=%zu w=%d", i, w);
          REQUIRE(b0[i * c.ow + w] + b1[i * c.ow + w] == e, "lut bcast i=%zu w=%d", i, w);
        }
      }
    }
  }
  // fused truncation: plain {16,-8,3,-1}, f = 4, for TR / ARS / GapARS and seeds 1, 2, 12345
  {
    const std::vector<int64_t> plain = {16, -8, 3, -1};
    for (int kind : {SUFB200_TRUNC_FAITHFUL_TR, SUFB200_TRUNC_FAITHFUL_ARS, SUFB200_TRUNC_GAPARS}) {
      for (uint64_t seed : {1ull, 2ull, 12345ull}) {
        sufb200_trunc_desc d[2];
        uint64_t thetas[4], r_in = 0;
        REQUIRE(sufb200_trunc_gen(kind, 4, seed, &d[0], &d[1], thetas, &r_in) == SUFB200_OK, "trunc_gen");
        std::vector<FssKey> keys[2];
        for (int q = 0; q < d[0].nq; q++) {
          auto kp = be.gen_dcf(d[0].q_bits[q], be.u64_to_bits_msb(thetas[q], d[0].q_bits[q]), pack_u64_le(1));
          keys[0].push_back(kp.k0);
          keys[1].push_back(kp.k1);
        }
        std::vector<uint64_t> xh(plain.size());
        for (size_t i = 0; i < plain.size(); i++) xh[i] = static_cast<uint64_t>(plain[i]) + r_in;
        uint64_t* d_x = nullptr;
        REQUIRE(cudaMalloc(&d_x, xh.size() * 8) == cudaSuccess, "cudaMalloc");
        REQUIRE(cudaMemcpy(d_x, xh.data(), xh.size() * 8, cudaMemcpyHostToDevice) == cudaSuccess, "H2D");
        std::vector<uint64_t> y0(xh.size()), y1(xh.size());
        be.eval_trunc_bundle_device(d[0], keys[0], d_x, xh.size(), y0.data());
        be.eval_trunc_bundle_device(d[1], keys[1], d_x, xh.size(), y1.data());
        cudaFree(d_x);
        for (size_t i = 0; i < plain.size(); i++) {
          const uint64_t rec = y0[i] + y1[i];
          const uint64_t expect = kind == SUFB200_TRUNC_FAITHFUL_TR ? (static_cast<uint64_t>(plain[i]) >> 4)
                                                                    : static_cast<uint64_t>(plain[i] >> 4);
          REQUIRE(rec == expect, "trunc kind=%d seed=%llu i=%zu rec=%llu", kind, (unsigned long long)seed, i,
                  (unsigned long long)rec);
        }
      }
    }
  }
  // errors surface as exceptions, not as silent host evaluation
  {
    bool threw = false;
    try {
      std::vector<uint8_t> bad(10, 0);
      std::vector<uint64_t> xs = {1};
      uint8_t out[8];
      be.eval_dcf_many_u64(64, bad.size(), bad.data(), xs, 8, out);
    } catch (const std::runtime_error&) {
      threw = true;
    }
    REQUIRE(threw, "malformed key did not raise");
  }
  std::printf("OK\n");
  return 0;
}
