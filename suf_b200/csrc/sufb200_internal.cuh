// sufb200_internal.cuh -- shared definitions for the sm_100a PFSS kernels.
//
// Everything here is product code: the CUDA kernels behind include/sufb200.h.
#pragma once

#include <cstddef>
#include <cstdint>

#include <cuda_runtime.h>

#include "../../include/sufb200.h"

#if defined(__CUDACC__)
#define SUFB200_HD __host__ __device__ __forceinline__
#else
#define SUFB200_HD inline
#endif

namespace sufb200 {

// ---------------------------------------------------------------------------
// Shared-memory AES engine layout.
//
// The four AES T-tables live at a FIXED shared-window address range
// [kTabBase, kTabBase + 128 KB).  For table k, input byte x and lane l:
//     addr = kTabBase + (k >> 1) * 64K + x * 256 + (k & 1) * 128 + l * 4
// Each 256-byte row holds two tables' 32 lane-private copies of one entry,
// so a warp's 32 lookups hit 32 distinct banks whatever the bytes are, and
// the variable part (x << 8 | l * 4) is produced by ONE byte-permute of the
// state word with the per-lane constant l * 4.  The table/region offset rides
// in the load instruction's immediate.  Kernels that use the engine are
// launched with exactly enough dynamic shared memory to reach kTabEnd from
// the dynamic base (measured once per device by a probe kernel) and check
// the base again on entry before touching the tables.
// ---------------------------------------------------------------------------
constexpr uint32_t kTabBase = 0x10000u;
constexpr uint32_t kTabEnd = 0x30000u;
constexpr int kAesThreads = 512;  // threads per CTA of every AES kernel

// Round keys of the four fixed PRG keys of the myl7 AES-128-MMO PRG
// (third_party/myl7_fss/src/prg/aes128_mmo.c:16-53), pre-arranged for the
// per-lane key choice: block index j in {0,1,2,3}; the walk needs j = 2*x+0
// (seed side) and j = 2*x+1 (value side).  base[h] holds key j = h (x = 0),
// diff[h] holds key(h) ^ key(h+2), so key(2x+h) = base[h] ^ (xmask & diff[h]).
// Words are little-endian columns.  Passed by value as a kernel parameter so
// every use is a constant-bank operand.
struct PrgParams {
  uint32_t base[2][11][4];
  uint32_t diff[2][11][4];
};

// Full fixed-key schedules as plain words (for dealer-side kernels that need
// all four blocks).
struct PrgKeys4 {
  uint32_t rk[4][11][4];
};

// Device status word bits (written with atomicOr, read by sufb200_ctx_sync).
enum : uint32_t {
  kStatusBadKeyHeader = 1u << 0,
  kStatusSmemLayout = 1u << 1,
  kStatusBadArgument = 1u << 2,
  kStatusTimeout = 1u << 3,  // a bounded wait inside a kernel gave up
};

SUFB200_HD uint32_t rotl32(uint32_t v, int r) { return (v << r) | (v >> ((32 - r) & 31)); }

// Byte permute with the PTX prmt.b32 default-mode semantics (selector nibbles
// < 8): result byte i = byte sel_i of the 8-byte value {b:a}.
SUFB200_HD uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
#if defined(__CUDA_ARCH__)
  return __byte_perm(a, b, sel);
#else
  uint64_t ab = (static_cast<uint64_t>(b) << 32) | a;
  uint32_t r = 0;
  for (int i = 0; i < 4; i++) {
    uint32_t s = (sel >> (4 * i)) & 7u;
    r |= static_cast<uint32_t>((ab >> (8 * s)) & 0xFFu) << (8 * i);
  }
  return r;
#endif
}

// Programmatic dependent launch.  A kernel launched with the
// programmatic-stream-serialization attribute (launch_pdl) may be scheduled
// while the kernel before it in the stream is still running: pdl_wait()
// blocks until that kernel has completed and its writes are visible (a no-op
// when the kernel was launched without the attribute), so code before it may
// read only constant or resident data (the AES tables' source, resident keys)
// and write only shared memory.  pdl_trigger() lets the next such kernel in
// the stream be scheduled onto SMs as this one's CTAs finish: its table fill
// and set-up then overlap this kernel's last wave.
#if defined(__CUDACC__)
__device__ __forceinline__ void pdl_wait() {
#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ >= 900)
  asm volatile("griddepcontrol.wait;" ::: "memory");
#endif
}
__device__ __forceinline__ void pdl_trigger() {
#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ >= 900)
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
#endif
}
#endif

}  // namespace sufb200

// Host-side context (definition shared by the .cu translation units).
struct sufb200_ctx_s {
  int device = 0;
  int sm_count = 0;
  uint32_t dyn_base = 0;         // shared-window address of dynamic smem
  uint32_t aes_dyn_bytes = 0;    // dynamic smem bytes of AES-engine kernels
  uint32_t* d_t0 = nullptr;      // 256-word T0 table (global), source of the smem fill
  uint32_t* d_status = nullptr;  // device status word
  uint8_t* d_scratch = nullptr;  // staging for small broadcast keys / descriptors
  size_t scratch_bytes = 0;
  cudaMemPool_t pool = nullptr;  // stream-ordered scratch; keeps its memory between calls
  bool prg_ready = false;
  sufb200::PrgParams prg{};
  sufb200::PrgKeys4 prg4{};
};
