// sufb200_backend.hpp -- drop-in PFSS backend for the reference runtime.
//
// proto::SufB200Backend implements the interfaces the reference's
// composite-FSS driver and PfssSuperBatch look for with dynamic_cast
// (PfssIntervalLutExt, PackedLtBackend, PfssGpuStagedEval; see
// include/gates/composite_fss.hpp:1203 and src/runtime/pfss_superbatch.cpp:
// 314,487,758) on top of the C ABI of libsufb200.so.  Returned by
// make_real_gpu_backend() (suf_b200/host/make_backend.cpp), it is what
// SUF_PFSS_BACKEND=gpu selects.
//
// Key formats:
//   * DCF keys (gen_dcf / eval_dcf*) use the myl7 PRG-tree layout of
//     Myl7FssBackend (include/proto/myl7_fss_backend.hpp:131-213) and its bit
//     order (LSB_FIRST), so keys made by either backend evaluate on the other;
//     the group is ADD (additive Z_2^64 shares, what AddU64 gates need) unless
//     Options::group says XOR.
//   * packed-compare and interval-LUT keys use the reference GPU backend's
//     blobs (cuda/pfss_backend_gpu.cu:75-94,223-288) with the kernel counter
//     layout of cuda/pfss_kernels.cu.
// Errors throw std::runtime_error carrying sufb200_last_error(), like the
// reference's validation paths; there is no host fallback.
#pragma once

#include <cuda_runtime.h>

#include <cstring>
#include <memory>
#include <mutex>
#include <random>
#include <stdexcept>
#include <string>
#include <vector>

#include "proto_api.hpp"
#include "sufb200.h"

namespace proto {

class SufB200Backend final : public PfssIntervalLutExt, public PackedLtBackend, public PfssGpuStagedEval {
 public:
  struct Options {
    int device = -1;                 // -1: the calling thread's current device
    int group = SUFB200_GROUP_ADD;   // myl7 group of gen_dcf / eval_dcf*
    std::vector<uint8_t> prg_state;  // >= 64 bytes; empty: the process-wide state
    bool deterministic = false;      // party seeds from mt19937_64(seed) instead of std::random_device
    uint64_t seed = 0;
    bool dealer_only = false;        // keygen only, no GPU needed (evaluation calls throw)
  };

  SufB200Backend() : SufB200Backend(Options{}) {}
  explicit SufB200Backend(Options o) : opt_(std::move(o)), rng_(opt_.seed) {
    int dev = SUFB200_HOST_ONLY;
    if (!opt_.dealer_only) {
      dev = opt_.device;
      if (dev < 0 && cudaGetDevice(&dev) != cudaSuccess) throw std::runtime_error("SufB200Backend: no CUDA device");
    }
    check(sufb200_ctx_create(dev, &ctx_), "sufb200_ctx_create");
    const std::vector<uint8_t>& st = opt_.prg_state.empty() ? process_prg_state() : opt_.prg_state;
    check(sufb200_prg_init(ctx_, st.data(), st.size()), "sufb200_prg_init");
    if (!opt_.dealer_only && cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking) != cudaSuccess)
      throw std::runtime_error("SufB200Backend: cudaStreamCreate failed");
  }

  ~SufB200Backend() override {
    for (auto* b : {&keys_buf_, &xs_buf_, &out_buf_, &bool_buf_}) b->release();
    if (stream_) cudaStreamDestroy(stream_);
    sufb200_ctx_destroy(ctx_);
  }

  SufB200Backend(const SufB200Backend&) = delete;
  SufB200Backend& operator=(const SufB200Backend&) = delete;

  // The PRG keys shared by every instance in this process that is not given
  // its own: both parties must use the same fixed AES keys, as the reference
  // adapter's process-global prg_init does (myl7_fss_backend.hpp:116-129).
  static const std::vector<uint8_t>& process_prg_state() {
    static const std::vector<uint8_t> st = [] {
      std::random_device rd;
      std::vector<uint8_t> s(128);
      for (auto& b : s) b = static_cast<uint8_t>(rd());
      return s;
    }();
    return st;
  }

  sufb200_ctx context() const { return ctx_; }

  // ---- PfssBackend -----------------------------------------------------------
  BitOrder bit_order() const override { return BitOrder::LSB_FIRST; }

  std::vector<u8> u64_to_bits_msb(u64 x, int in_bits) const override {
    std::vector<u8> bits(static_cast<size_t>(in_bits));
    for (int i = 0; i < in_bits; i++) bits[static_cast<size_t>(i)] = static_cast<u8>((x >> i) & 1u);
    return bits;
  }

  DcfKeyPair gen_dcf(int in_bits, const std::vector<u8>& alpha_bits, const std::vector<u8>& payload) override {
    if (in_bits <= 0 || in_bits > 64) throw std::runtime_error("SufB200Backend: in_bits out of range");
    if (static_cast<int>(alpha_bits.size()) != in_bits) throw std::runtime_error("SufB200Backend: alpha_bits mismatch");
    if (payload.empty()) throw std::runtime_error("SufB200Backend: empty payload");
    const u64 alpha = bits_to_u64(alpha_bits);
    const size_t chunks = (payload.size() + 15) / 16;
    std::vector<u8> s0(16 * chunks), s1(16 * chunks);
    fill_seeds(s0);
    fill_seeds(s1);
    DcfKeyPair kp;
    const size_t kb = sufb200_myl7_key_bytes(in_bits, static_cast<int>(payload.size()));
    kp.k0.bytes.resize(kb);
    kp.k1.bytes.resize(kb);
    check(sufb200_myl7_gen(ctx_, opt_.group, in_bits, alpha, payload.data(), static_cast<int>(payload.size()),
                           s0.data(), s1.data(), kp.k0.bytes.data(), kp.k1.bytes.data()),
          "gen_dcf");
    return kp;
  }

  std::vector<u8> eval_dcf(int in_bits, const FssKey& kb, const std::vector<u8>& x_bits) const override {
    if (static_cast<int>(x_bits.size()) != in_bits) throw std::runtime_error("SufB200Backend: x_bits mismatch");
    if (kb.bytes.size() < 8) throw std::runtime_error("SufB200Backend: key truncated");
    uint32_t plen;
    std::memcpy(&plen, kb.bytes.data() + 4, 4);
    std::vector<u8> out(plen);
    const u64 x = bits_to_u64(x_bits);
    std::lock_guard<std::mutex> lk(mu_);
    check(sufb200_myl7_dcf_eval_host(ctx_, opt_.group, in_bits, kb.bytes.data(), kb.bytes.size(), 1, &x, 1,
                                     static_cast<int>(plen), out.data()),
          "eval_dcf");
    return out;
  }

  // ---- PfssBackendBatch --------------------------------------------------------
  void eval_dcf_many_u64(int in_bits, size_t key_bytes, const uint8_t* keys_flat, const std::vector<u64>& xs,
                         int out_bytes, uint8_t* outs_flat) const override {
    if (xs.empty()) return;
    const int bc = replicated(keys_flat, key_bytes, xs.size()) ? 1 : 0;
    std::lock_guard<std::mutex> lk(mu_);
    check(sufb200_myl7_dcf_eval_host(ctx_, opt_.group, in_bits, keys_flat, key_bytes, bc, xs.data(), xs.size(),
                                     out_bytes, outs_flat),
          "eval_dcf_many_u64");
  }

  // ---- PackedLtBackend (reference GPU blob) ----------------------------------
  PackedLtKeyPair gen_packed_lt(int in_bits, const std::vector<u64>& thresholds) override {
    if (thresholds.empty()) throw std::runtime_error("SufB200Backend: packed thresholds empty");
    const uint64_t nonce = next_id_++;
    uint8_t seed[16];
    check(sufb200_seed_from_id(nonce, 0, seed), "seed_from_id");
    PackedLtKeyPair kp;
    const int nt = static_cast<int>(thresholds.size());
    for (int p = 0; p < 2; p++) {
      FssKey& k = p ? kp.k1 : kp.k0;
      const size_t n = sufb200_packed_lt_build(p, nonce, in_bits, thresholds.data(), nt, seed, nullptr);
      if (!n) throw std::runtime_error("SufB200Backend: bad packed-compare arguments");
      k.bytes.resize(n);
      sufb200_packed_lt_build(p, nonce, in_bits, thresholds.data(), nt, seed, k.bytes.data());
    }
    return kp;
  }

  void eval_packed_lt_many(size_t key_bytes, const uint8_t* keys_flat, const std::vector<u64>& xs, int in_bits,
                           int out_words, u64* outs) const override {
    if (xs.empty()) return;
    std::lock_guard<std::mutex> lk(mu_);
    const uint64_t* d_xs = upload_xs(xs.data(), xs.size());
    packed_device(key_bytes, keys_flat, false, d_xs, xs.size(), in_bits, out_words, outs);
  }

  // ---- PfssIntervalLutExt (reference GPU blob) --------------------------------
  IntervalLutKeyPair gen_interval_lut(const IntervalLutDesc& desc) override {
    if (desc.out_words <= 0) throw std::runtime_error("SufB200Backend: out_words must be > 0");
    if (desc.cutpoints.size() < 2) throw std::runtime_error("SufB200Backend: need >= 2 cutpoints");
    const int iv = static_cast<int>(desc.cutpoints.size() - 1);
    if (desc.payload_flat.size() != static_cast<size_t>(iv) * static_cast<size_t>(desc.out_words))
      throw std::runtime_error("SufB200Backend: payload size mismatch");
    const uint64_t nonce = next_id_++;
    uint8_t seed[16];
    check(sufb200_seed_from_id(nonce, 7, seed), "seed_from_id");
    IntervalLutKeyPair kp;
    for (int p = 0; p < 2; p++) {
      FssKey& k = p ? kp.k1 : kp.k0;
      const size_t n = sufb200_interval_lut_build(p, nonce, desc.in_bits, desc.out_words, desc.cutpoints.data(), iv,
                                                  desc.payload_flat.data(), seed, nullptr);
      if (!n) throw std::runtime_error("SufB200Backend: bad interval-LUT arguments");
      k.bytes.resize(n);
      sufb200_interval_lut_build(p, nonce, desc.in_bits, desc.out_words, desc.cutpoints.data(), iv,
                                 desc.payload_flat.data(), seed, k.bytes.data());
    }
    return kp;
  }

  void eval_interval_lut_many_u64(size_t key_bytes, const uint8_t* keys_flat, const std::vector<u64>& xs,
                                  int out_words, u64* outs) const override {
    if (xs.empty()) return;
    std::lock_guard<std::mutex> lk(mu_);
    const uint64_t* d_xs = upload_xs(xs.data(), xs.size());
    lut_device(key_bytes, keys_flat, false, d_xs, xs.size(), out_words, outs);
  }

  // ---- PfssGpuStagedEval -------------------------------------------------------
  void eval_dcf_many_u64_device(int in_bits, size_t key_bytes, const uint8_t* keys_flat, const uint64_t* xs_device,
                                size_t N, int out_bytes, uint8_t* outs_flat) const override {
    std::lock_guard<std::mutex> lk(mu_);
    dcf_device(in_bits, key_bytes, keys_flat, false, xs_device, N, out_bytes, outs_flat);
  }

  void eval_dcf_many_u64_device_broadcast(int in_bits, size_t key_bytes, const uint8_t* key, const uint64_t* xs_device,
                                          size_t N, int out_bytes, uint8_t* outs_flat) const override {
    std::lock_guard<std::mutex> lk(mu_);
    dcf_device(in_bits, key_bytes, key, true, xs_device, N, out_bytes, outs_flat);
  }

  void eval_packed_lt_many_device(size_t key_bytes, const uint8_t* keys_flat, const uint64_t* xs_device, size_t N,
                                  int in_bits, int out_words, uint64_t* outs) const override {
    std::lock_guard<std::mutex> lk(mu_);
    packed_device(key_bytes, keys_flat, false, xs_device, N, in_bits, out_words, outs);
  }

  void eval_packed_lt_many_device_broadcast(size_t key_bytes, const uint8_t* key, const uint64_t* xs_device, size_t N,
                                            int in_bits, int out_words, uint64_t* outs) const override {
    std::lock_guard<std::mutex> lk(mu_);
    packed_device(key_bytes, key, true, xs_device, N, in_bits, out_words, outs);
  }

  void eval_interval_lut_many_device(size_t key_bytes, const uint8_t* keys_flat, const uint64_t* xs_device, size_t N,
                                     int out_words, uint64_t* outs) const override {
    std::lock_guard<std::mutex> lk(mu_);
    lut_device(key_bytes, keys_flat, false, xs_device, N, out_words, outs);
  }

  void eval_interval_lut_many_device_broadcast(size_t key_bytes, const uint8_t* key, const uint64_t* xs_device,
                                               size_t N, int out_words, uint64_t* outs) const override {
    std::lock_guard<std::mutex> lk(mu_);
    lut_device(key_bytes, key, true, xs_device, N, out_words, outs);
  }

  void* device_stream() const override { return reinterpret_cast<void*>(stream_); }
  const uint64_t* last_device_output() const override { return reinterpret_cast<const uint64_t*>(out_buf_.ptr); }
  const uint64_t* last_device_bools() const override { return reinterpret_cast<const uint64_t*>(bool_buf_.ptr); }
  void ensure_output_buffers(size_t arith_words, size_t bool_words) const override {
    std::lock_guard<std::mutex> lk(mu_);
    if (arith_words) out_buf_.ensure(arith_words * 8);
    if (bool_words) bool_buf_.ensure(bool_words * 8);
  }

  // ---- beyond the reference interface: the fused truncation bundle ----------
  // One launch for every raw query of a FaithfulTR / FaithfulARS / GapARS gate
  // plus its postproc (replaces the AddU64 branch of composite_eval_batch_backend
  // and the hook's run_batch).  keys[q] is this party's key of query q.
  // y_host may be null: the result then stays in last_device_output().
  void eval_trunc_bundle_device(const sufb200_trunc_desc& desc, const std::vector<FssKey>& keys,
                                const uint64_t* xhat_device, size_t N, uint64_t* y_host) const {
    std::lock_guard<std::mutex> lk(mu_);
    std::vector<const uint8_t*> kp(4, nullptr);
    std::vector<size_t> kb(4, 0);
    for (size_t q = 0; q < keys.size() && q < 4; q++) {
      kp[q] = keys[q].bytes.data();
      kb[q] = keys[q].bytes.size();
    }
    out_buf_.ensure(N * 8);
    check(sufb200_trunc_bundle_eval(ctx_, &desc, kp.data(), kb.data(), xhat_device, N,
                                    reinterpret_cast<uint64_t*>(out_buf_.ptr), nullptr, stream_),
          "trunc bundle");
    if (y_host) cuda(cudaMemcpyAsync(y_host, out_buf_.ptr, N * 8, cudaMemcpyDeviceToHost, stream_), "D2H y");
    check(sufb200_ctx_sync(ctx_, stream_), "trunc bundle");
  }

 private:
  struct DeviceBuffer {
    uint8_t* ptr = nullptr;
    size_t cap = 0;
    void ensure(size_t bytes) {
      if (bytes <= cap) return;
      release();
      if (cudaMalloc(reinterpret_cast<void**>(&ptr), bytes) != cudaSuccess) {
        ptr = nullptr;
        throw std::runtime_error("SufB200Backend: cudaMalloc failed");
      }
      cap = bytes;
    }
    void release() {
      if (ptr) cudaFree(ptr);
      ptr = nullptr;
      cap = 0;
    }
  };

  static void check(int rc, const char* what) {
    if (rc != SUFB200_OK) throw std::runtime_error(std::string("SufB200Backend ") + what + ": " + sufb200_last_error());
  }
  static void cuda(cudaError_t e, const char* what) {
    if (e != cudaSuccess) throw std::runtime_error(std::string("SufB200Backend ") + what + ": " + cudaGetErrorString(e));
  }

  u64 bits_to_u64(const std::vector<u8>& bits) const {
    u64 v = 0;
    for (size_t i = 0; i < bits.size(); i++)
      if (bits[i] & 1u) v |= u64(1) << i;  // LSB_FIRST
    return v;
  }

  void fill_seeds(std::vector<u8>& s) {
    if (opt_.deterministic) {
      for (size_t i = 0; i < s.size(); i += 8) {
        const u64 w = rng_();
        std::memcpy(s.data() + i, &w, std::min<size_t>(8, s.size() - i));
      }
    } else {
      std::random_device rd;
      for (auto& b : s) b = static_cast<u8>(rd());
    }
  }

  // True when all n keys of a per-element key block are byte-identical to the
  // first.  The reference's composite driver, given host x^, copies its one
  // broadcast key n times before calling the batch entry points
  // (composite_fss.hpp:1515-1519); evaluating that block as one broadcast key
  // gives the same shares (every format's per-element counter depends on the
  // element index only) without uploading and walking n copies.
  static bool replicated(const uint8_t* keys, size_t key_bytes, size_t n) {
    if (n < 2 || key_bytes == 0) return false;
    int same = 1;
#pragma omp parallel for schedule(static) reduction(&& : same)
    for (long long i = 1; i < static_cast<long long>(n); i++)
      same = same && std::memcmp(keys + static_cast<size_t>(i) * key_bytes, keys, key_bytes) == 0;
    return same != 0;
  }

  const uint64_t* upload_xs(const u64* xs, size_t n) const {
    xs_buf_.ensure(n * 8);
    cuda(cudaMemcpyAsync(xs_buf_.ptr, xs, n * 8, cudaMemcpyHostToDevice, stream_), "H2D xs");
    return reinterpret_cast<const uint64_t*>(xs_buf_.ptr);
  }

  const uint8_t* upload_keys(const uint8_t* keys, size_t bytes) const {
    keys_buf_.ensure(bytes);
    cuda(cudaMemcpyAsync(keys_buf_.ptr, keys, bytes, cudaMemcpyHostToDevice, stream_), "H2D keys");
    return keys_buf_.ptr;
  }

  void finish(const uint8_t* dev_out, void* host_out, size_t bytes) const {
    if (host_out) cuda(cudaMemcpyAsync(host_out, dev_out, bytes, cudaMemcpyDeviceToHost, stream_), "D2H outs");
    check(sufb200_ctx_sync(ctx_, stream_), "device status");
  }

  void dcf_device(int in_bits, size_t key_bytes, const uint8_t* keys, bool broadcast, const uint64_t* xs, size_t N,
                  int out_bytes, uint8_t* outs) const {
    if (N == 0) return;
    if (!keys || !xs) throw std::runtime_error("SufB200Backend: null keys / xs_device");
    broadcast = broadcast || replicated(keys, key_bytes, N);
    const uint8_t* dk = upload_keys(keys, broadcast ? key_bytes : key_bytes * N);
    bool_buf_.ensure(N * static_cast<size_t>(out_bytes));
    check(sufb200_myl7_dcf_eval(ctx_, opt_.group, in_bits, dk, key_bytes, broadcast ? 1 : 0, xs, N, out_bytes,
                                bool_buf_.ptr, stream_),
          "eval_dcf_many_u64_device");
    finish(bool_buf_.ptr, outs, N * static_cast<size_t>(out_bytes));
  }

  void packed_device(size_t key_bytes, const uint8_t* keys, bool broadcast, const uint64_t* xs, size_t N, int in_bits,
                     int out_words, uint64_t* outs) const {
    if (N == 0) return;
    if (!keys || !xs) throw std::runtime_error("SufB200Backend: null keys / xs");
    broadcast = broadcast || replicated(keys, key_bytes, N);
    const uint8_t* dk = upload_keys(keys, broadcast ? key_bytes : key_bytes * N);
    bool_buf_.ensure(N * static_cast<size_t>(out_words) * 8);
    check(sufb200_packed_lt_eval(ctx_, dk, key_bytes, broadcast ? 1 : 0, xs, N, in_bits, out_words, 0,
                                 reinterpret_cast<uint64_t*>(bool_buf_.ptr), stream_),
          "packed compare");
    finish(bool_buf_.ptr, outs, N * static_cast<size_t>(out_words) * 8);
  }

  void lut_device(size_t key_bytes, const uint8_t* keys, bool broadcast, const uint64_t* xs, size_t N, int out_words,
                  uint64_t* outs) const {
    if (N == 0) return;
    if (!keys || !xs) throw std::runtime_error("SufB200Backend: null keys / xs");
    broadcast = broadcast || replicated(keys, key_bytes, N);
    const uint8_t* dk = upload_keys(keys, broadcast ? key_bytes : key_bytes * N);
    out_buf_.ensure(N * static_cast<size_t>(out_words) * 8);
    check(sufb200_interval_lut_eval(ctx_, dk, key_bytes, broadcast ? 1 : 0, xs, N, out_words, 0,
                                    reinterpret_cast<uint64_t*>(out_buf_.ptr), stream_),
          "interval LUT");
    finish(out_buf_.ptr, outs, N * static_cast<size_t>(out_words) * 8);
  }

  Options opt_;
  sufb200_ctx ctx_ = nullptr;
  cudaStream_t stream_ = nullptr;
  std::mt19937_64 rng_;
  uint64_t next_id_ = 1;
  mutable std::mutex mu_;
  mutable DeviceBuffer keys_buf_, xs_buf_, out_buf_, bool_buf_;
};

}  // namespace proto
