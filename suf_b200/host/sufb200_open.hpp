// sufb200_open.hpp -- C++ handle of the paired-GPU open (sufb200_open_* in
// include/sufb200.h) for the reference runtime's OpenCollector.
//
// OpenCollector::flush's device-pack path (src/runtime/open_collector.cpp,
// the block from the H2D of the send buffer to launch_unpack_add_mod_kernel)
// copies the packed flush to the host, swaps it through net::Chan and copies
// the peer's words back.  With both parties on one node, each party's
// collector holds a PairedOpen and replaces that block with one call:
//   open.exchange(d_send, total_words, eff, ring_bits, false, d_opened, stream);
// which packs, swaps the packed words GPU to GPU and adds them, on `stream`.
// Errors throw std::runtime_error with the engine's message.
#pragma once

#include <cuda_runtime.h>

#include <array>
#include <cstdint>
#include <stdexcept>
#include <string>

#include "sufb200.h"

namespace sufb200 {

class PairedOpen {
 public:
  using Id = std::array<uint8_t, SUFB200_OPEN_ID_BYTES>;

  // Made on one rank and handed to the others out of band.
  static Id unique_id() {
    Id id{};
    check(sufb200_open_unique_id(id.data()), "sufb200_open_unique_id");
    return id;
  }

  // The width OpenCollector packs a flush to: the ring's width when it is
  // below 64 bits and at most max_pack_bits (SUF_OPEN_PACK_MAX_BITS, default
  // 56), else raw 64-bit words (open_collector.cpp, eff_local).
  static int eff_bits_for_ring(int ring_bits, int max_pack_bits = 56) {
    return (ring_bits > 0 && ring_bits < 64 && ring_bits <= max_pack_bits) ? ring_bits : 64;
  }

  // Joins the communicator of all nranks ranks (party 0 on GPUs 0..N/2-1,
  // party 1 on the rest); peer is the rank holding the other party's shares.
  PairedOpen(sufb200_ctx ctx, const Id& id, int nranks, int rank, int peer, double timeout_s = 60.0) : peer_(peer) {
    check(sufb200_open_comm_create(ctx, id.data(), nranks, rank, timeout_s, &comm_), "sufb200_open_comm_create");
  }
  PairedOpen(const PairedOpen&) = delete;
  PairedOpen& operator=(const PairedOpen&) = delete;
  ~PairedOpen() {
    if (comm_) sufb200_open_comm_destroy(comm_);
  }

  // d_out = d_local + peer's shares mod 2^ring_bits (sign-extended when
  // signed_out), both device arrays of n words, enqueued on `stream`.
  void exchange(const uint64_t* d_local, size_t n, int eff_bits, int ring_bits, bool signed_out, uint64_t* d_out,
                cudaStream_t stream) {
    check(sufb200_open_exchange(comm_, peer_, d_local, n, eff_bits, ring_bits, signed_out ? 1 : 0, d_out, stream),
          "sufb200_open_exchange");
  }

  // Ends a pending exchange whose peer has gone (any thread).
  void abort() { sufb200_open_comm_abort(comm_); }

 private:
  static void check(int rc, const char* what) {
    if (rc != SUFB200_OK) throw std::runtime_error(std::string(what) + ": " + sufb200_last_error());
  }
  sufb200_open_comm comm_ = nullptr;
  int peer_;
};

}  // namespace sufb200
