// proto_api.hpp -- the reference's PFSS backend interfaces, declared with the
// same names, signatures and semantics so that SufB200Backend builds and is
// tested without the reference checkout.  Inside the reference tree, define
// SUFB200_WITH_REFERENCE_PROTO and the adapter includes the reference's own
// headers instead (include/proto/pfss_backend.hpp:36-54,
// pfss_backend_batch.hpp:10-29, packed_backend.hpp:11-24,
// pfss_interval_lut_ext.hpp:17-27, backend_gpu.hpp:15-68).
#pragma once

#if defined(SUFB200_WITH_REFERENCE_PROTO)
#include "proto/backend_gpu.hpp"
#include "proto/packed_backend.hpp"
#include "proto/pfss_backend.hpp"
#include "proto/pfss_backend_batch.hpp"
#include "proto/pfss_interval_lut_ext.hpp"
#else

#include <cstddef>
#include <cstdint>
#include <cstring>
#include <stdexcept>
#include <vector>

namespace proto {

using u8 = uint8_t;
using u64 = uint64_t;

struct FssKey {
  std::vector<u8> bytes;
};

struct DcfKeyPair {
  FssKey k0;
  FssKey k1;
};

enum class ShareSemantics : uint8_t { XorBytes, AddU64 };
enum class BitOrder : uint8_t { MSB_FIRST, LSB_FIRST };

// f(x) = payload if x < alpha else 0, two-party shares.
struct PfssBackend {
  virtual ~PfssBackend() = default;
  virtual DcfKeyPair gen_dcf(int in_bits, const std::vector<u8>& alpha_bits, const std::vector<u8>& payload_bytes) = 0;
  virtual std::vector<u8> eval_dcf(int in_bits, const FssKey& kb, const std::vector<u8>& x_bits) const = 0;
  virtual std::vector<u8> u64_to_bits_msb(u64 x, int in_bits) const = 0;
  virtual BitOrder bit_order() const { return BitOrder::MSB_FIRST; }
};

struct PfssBackendBatch : public PfssBackend {
  // keys_flat is [N][key_bytes], outs_flat [N][out_bytes].
  virtual void eval_dcf_many_u64(int in_bits, size_t key_bytes, const uint8_t* keys_flat,
                                 const std::vector<u64>& xs_u64, int out_bytes, uint8_t* outs_flat) const = 0;
};

struct PackedLtKeyPair {
  FssKey k0, k1;
};

class PackedLtBackend {
 public:
  virtual ~PackedLtBackend() = default;
  virtual PackedLtKeyPair gen_packed_lt(int in_bits, const std::vector<u64>& thresholds) = 0;
  virtual void eval_packed_lt_many(size_t key_bytes, const uint8_t* keys_flat, const std::vector<u64>& xs_u64,
                                   int in_bits, int out_words, u64* outs_bitmask) const = 0;
};

struct IntervalLutKeyPair {
  FssKey k0, k1;
};

struct IntervalLutDesc {
  int in_bits = 64;
  int out_words = 0;
  std::vector<u64> cutpoints;     // increasing, masked domain; intervals = size - 1
  std::vector<u64> payload_flat;  // intervals * out_words
};

struct PfssIntervalLutExt : public PfssBackendBatch {
  virtual IntervalLutKeyPair gen_interval_lut(const IntervalLutDesc& desc) = 0;
  virtual void eval_interval_lut_many_u64(size_t key_bytes, const uint8_t* keys_flat, const std::vector<u64>& xs_u64,
                                          int out_words, u64* outs_flat) const = 0;
};

// Device-pointer entry points used by the runtime when x^ is already staged.
struct PfssGpuStagedEval {
  virtual ~PfssGpuStagedEval() = default;
  virtual void eval_dcf_many_u64_device(int in_bits, size_t key_bytes, const uint8_t* keys_flat,
                                        const uint64_t* xs_device, size_t N, int out_bytes,
                                        uint8_t* outs_flat) const = 0;
  virtual void eval_dcf_many_u64_device_broadcast(int in_bits, size_t key_bytes, const uint8_t* key,
                                                  const uint64_t* xs_device, size_t N, int out_bytes,
                                                  uint8_t* outs_flat) const = 0;
  virtual void eval_packed_lt_many_device(size_t key_bytes, const uint8_t* keys_flat, const uint64_t* xs_device,
                                          size_t N, int in_bits, int out_words, uint64_t* outs_bitmask) const = 0;
  virtual void eval_packed_lt_many_device_broadcast(size_t key_bytes, const uint8_t* key, const uint64_t* xs_device,
                                                    size_t N, int in_bits, int out_words,
                                                    uint64_t* outs_bitmask) const = 0;
  virtual void eval_interval_lut_many_device(size_t key_bytes, const uint8_t* keys_flat, const uint64_t* xs_device,
                                             size_t N, int out_words, uint64_t* outs_flat) const = 0;
  virtual void eval_interval_lut_many_device_broadcast(size_t key_bytes, const uint8_t* key,
                                                       const uint64_t* xs_device, size_t N, int out_words,
                                                       uint64_t* outs_flat) const = 0;
  virtual void* device_stream() const = 0;
  virtual const uint64_t* last_device_output() const { return nullptr; }
  virtual const uint64_t* last_device_bools() const { return nullptr; }
  virtual void ensure_output_buffers(size_t /*arith_words*/, size_t /*bool_words*/) const {}
};

}  // namespace proto

#endif  // SUFB200_WITH_REFERENCE_PROTO
