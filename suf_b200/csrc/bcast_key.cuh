// bcast_key.cuh -- staging of one myl7 DCF key (adapter layout,
// include/proto/myl7_fss_backend.hpp:131-213) into shared memory, and the
// header / byte-load helpers shared by the DCF kernels.
#pragma once

#include "dcf_walk.cuh"

namespace sufb200 {

// Broadcast-key staging area at the start of dynamic shared memory.
struct BcastKeySmem {
  uint4 cw_s[64];
  uint64_t cw_v[64];
  uint32_t cw_t[64];
  uint4 seed;
  uint64_t np1_lo;
  uint32_t party;
  uint32_t ok;
};
static_assert(sizeof(BcastKeySmem) < kTabBase - 4096, "staging must fit below the tables");

__device__ __forceinline__ uint32_t ld_u32_bytes(const uint8_t* p) {
  return static_cast<uint32_t>(p[0]) | (static_cast<uint32_t>(p[1]) << 8) | (static_cast<uint32_t>(p[2]) << 16) |
         (static_cast<uint32_t>(p[3]) << 24);
}
__device__ __forceinline__ uint64_t ld_u64_bytes(const uint8_t* p) {
  return static_cast<uint64_t>(ld_u32_bytes(p)) | (static_cast<uint64_t>(ld_u32_bytes(p + 4)) << 32);
}

// Header check shared by all paths (myl7_fss_backend.hpp:222-236 semantics).
__device__ __forceinline__ bool key_header_ok(uint64_t hdr, int in_bits, int out_bytes) {
  const uint32_t kb = static_cast<uint32_t>(hdr & 0xFF), chunks = static_cast<uint32_t>((hdr >> 8) & 0xFF),
                 party = static_cast<uint32_t>((hdr >> 16) & 0xFF), plen = static_cast<uint32_t>(hdr >> 32);
  return kb == static_cast<uint32_t>(in_bits) && chunks == 1u && party <= 1u &&
         plen == static_cast<uint32_t>(out_bytes);
}

__device__ __forceinline__ void store_out(void* out, size_t i, int out_bytes, uint64_t v) {
  if (out_bytes == 8) {
    reinterpret_cast<uint64_t*>(out)[i] = v;
  } else {
    uint8_t* o = reinterpret_cast<uint8_t*>(out) + i * static_cast<size_t>(out_bytes);
    for (int b = 0; b < out_bytes; b++) o[b] = static_cast<uint8_t>(v >> (8 * b));
  }
}

__device__ __forceinline__ void stage_bcast_key(BcastKeySmem* ks, const uint8_t* k, int in_bits, int out_bytes) {
  const uint64_t hdr = ld_u64_bytes(k);
  const bool ok = key_header_ok(hdr, in_bits, out_bytes);
  for (int i = threadIdx.x; i < in_bits; i += blockDim.x) {
    const uint8_t* c = k + 24 + 33 * i;
    ks->cw_s[i] = make_uint4(ld_u32_bytes(c), ld_u32_bytes(c + 4), ld_u32_bytes(c + 8), ld_u32_bytes(c + 12));
    ks->cw_v[i] = ld_u64_bytes(c + 16);
    ks->cw_t[i] = c[32];
  }
  if (threadIdx.x == 0) {
    ks->seed = make_uint4(ld_u32_bytes(k + 8), ld_u32_bytes(k + 12), ld_u32_bytes(k + 16),
                          ld_u32_bytes(k + 20) & 0x7FFFFFFFu);
    ks->np1_lo = ld_u64_bytes(k + 24 + 33 * in_bits);
    ks->party = static_cast<uint32_t>((hdr >> 16) & 0xFF);
    ks->ok = ok ? 1u : 0u;
  }
}


}  // namespace sufb200
