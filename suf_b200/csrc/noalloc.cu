// noalloc.cu -- an allocation-free form of the fused truncation bundle.
//
// Some callers cannot allocate device memory at the point where they need a
// truncation: a runtime that hands out all device memory from its own arena
// up front, a process whose allocator must not be re-entered (for example
// from inside an allocator callback or a memory-pool teardown), or a caller
// that must not let the CUDA caching allocator grow during a latency-critical
// phase.  sufb200_trunc_bundle_eval stages the bundle's keys in a buffer it
// takes from a stream-ordered memory pool; the entry point here stages them in
// one fixed array that the library image carries on every device, so the
// call itself allocates nothing on the device or the host.
//
// The array below is g_noalloc_keys: SUFB200_NOALLOC_KEY_BYTES (16 KiB)
// bytes.  A bundle has at most four keys of the myl7 layout, each at most
// 2152 bytes (64-bit input, 8-byte payload; 2160 padded to 16), so 8640
// bytes is the most a valid bundle needs: the size check below is a guard
// with headroom, not a limit a valid bundle reaches.  Every GPU that loads
// the library holds these 16 KiB until the process exits.
//
// Two things on the first call per device are not allocation-free: the
// address lookup, and (with CUDA's lazy module loading, the default since
// CUDA 12.2) loading this library's kernels into the context, which
// allocates device memory.  A caller makes one call at set-up.  The cached
// address is only valid for the context it was looked up in: after
// cudaDeviceReset, or a release and re-creation of the primary context, the
// entry point must not be called again in this process.
#include <cstring>
#include <mutex>
#include <string>

#include "kernels.hpp"
#include "keygen.hpp"
#include "sufb200_internal.cuh"

namespace {

// The key staging area shared by every call on a device.  Host code must
// not use this name as a device address (in host code it names a host-side
// stand-in); it uses the address obtained from cudaGetSymbolAddress below.
static __device__ __align__(256) uint8_t g_noalloc_keys[SUFB200_NOALLOC_KEY_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_setup_mu;
uint8_t* g_keys_addr[kMaxDevices] = {};

// Device address of g_noalloc_keys on the current device, looked up once per
// device (the device must be current; the caller has made it so).
int noalloc_keys_address(int device, uint8_t** out) {
  if (device < 0 || device >= kMaxDevices)
    return sufb200::record_error(SUFB200_ERR_UNSUPPORTED, "device index beyond the staging-address table");
  std::lock_guard<std::mutex> lk(g_setup_mu);
  if (!g_keys_addr[device]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_keys);
    if (e != cudaSuccess || !p)
      return sufb200::record_error(SUFB200_ERR_CUDA,
                                   std::string("cudaGetSymbolAddress(g_noalloc_keys): ") + cudaGetErrorString(e));
    g_keys_addr[device] = static_cast<uint8_t*>(p);
  }
  *out = g_keys_addr[device];
  return SUFB200_OK;
}

int noalloc_fail(int code, const std::string& msg) { return sufb200::record_error(code, msg); }

}  // namespace

// See include/sufb200.h for the contract.  The checks mirror
// sufb200_trunc_bundle_eval; only the key staging differs.
extern "C" int sufb200_trunc_bundle_eval_noalloc(sufb200_ctx ctx, const sufb200_trunc_desc* desc,
                                                 const uint8_t* const* keys, const size_t* key_bytes,
                                                 const uint64_t* d_xhat, size_t n, uint64_t* d_y, uint64_t* d_bools,
                                                 void* stream) {
  if (!ctx) return noalloc_fail(SUFB200_ERR_INVALID, "null context");
  if (ctx->device < 0) return noalloc_fail(SUFB200_ERR_UNSUPPORTED, "host-only context: no device to evaluate on");
  if (!ctx->prg_ready) return noalloc_fail(SUFB200_ERR_NOT_READY, "sufb200_prg_init has not been called");
  if (!desc || !keys || !key_bytes) return noalloc_fail(SUFB200_ERR_INVALID, "null pointer");
  if (desc->nq < 0 || desc->nq > 4) return noalloc_fail(SUFB200_ERR_UNSUPPORTED, "bundle has more than 4 queries");
  if (desc->kind < 0 || desc->kind > 2 || desc->party < 0 || desc->party > 1)
    return noalloc_fail(SUFB200_ERR_INVALID, "bad kind / party");
  if (desc->frac_bits < 0 || desc->frac_bits > 64) return noalloc_fail(SUFB200_ERR_INVALID, "frac_bits out of range");
  const int idx[5] = {desc->carry_a, desc->carry_b, desc->sign_a, desc->sign_b, desc->wrap_q};
  for (int v : idx)
    if (v >= desc->nq) return noalloc_fail(SUFB200_ERR_INVALID, "query index out of range");
  if ((desc->carry_a >= 0) != (desc->carry_b >= 0) || (desc->sign_a >= 0) != (desc->sign_b >= 0))
    return noalloc_fail(SUFB200_ERR_INVALID, "rotation operands must come in pairs");
  // Size and header checks first, so an oversized or mismatched bundle is
  // rejected before anything is written to the shared array.
  sufb200::TruncLaunch a{};
  a.desc = *desc;
  size_t total = 0, off[4] = {0, 0, 0, 0};
  for (int q = 0; q < desc->nq; q++) {
    const int nb = desc->q_bits[q];
    if (nb < 1 || nb > 64) return noalloc_fail(SUFB200_ERR_INVALID, "query in_bits out of range");
    if (!keys[q] || key_bytes[q] != sufb200::host::myl7_key_bytes(nb, 8))
      return noalloc_fail(SUFB200_ERR_KEY, "key size does not match an 8-byte myl7 key");
    const uint8_t* k = keys[q];
    uint32_t pl;
    std::memcpy(&pl, k + 4, 4);
    if (k[0] != nb || k[1] != 1 || k[2] != desc->party || pl != 8)
      return noalloc_fail(SUFB200_ERR_KEY, "key header does not match the bundle");
    off[q] = total;
    total += (key_bytes[q] + 15) & ~static_cast<size_t>(15);
  }
  if (total > SUFB200_NOALLOC_KEY_BYTES)
    return noalloc_fail(SUFB200_ERR_INVALID,
                        "bundle keys exceed the fixed 16 KiB staging array of the allocation-free entry point");
  if (n == 0) return SUFB200_OK;
  if (!d_xhat || !d_y || (reinterpret_cast<uintptr_t>(d_xhat) & 7) || (reinterpret_cast<uintptr_t>(d_y) & 7) ||
      (d_bools && (reinterpret_cast<uintptr_t>(d_bools) & 7)))
    return noalloc_fail(SUFB200_ERR_INVALID, "null or misaligned device pointer");
  cudaError_t e = cudaSetDevice(ctx->device);
  if (e != cudaSuccess) return noalloc_fail(SUFB200_ERR_CUDA, std::string("cudaSetDevice: ") + cudaGetErrorString(e));
  uint8_t* base = nullptr;
  if (int rc = noalloc_keys_address(ctx->device, &base)) return rc;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  // Every byte the kernel reads of each key is written here, so nothing in
  // the array has to start at zero; bytes of an earlier call that are not
  // overwritten (padding, space past this bundle) are never read.
  for (int q = 0; q < desc->nq; q++) {
    e = cudaMemcpyAsync(base + off[q], keys[q], key_bytes[q], cudaMemcpyHostToDevice, st);
    if (e != cudaSuccess)
      return noalloc_fail(SUFB200_ERR_CUDA,
                          std::string("copy of the bundle keys into the staging array: ") + cudaGetErrorString(e));
  }
  for (int q = 0; q < desc->nq; q++) a.key[q] = base + off[q];
  a.xhat = d_xhat;
  a.n = n;
  a.y = d_y;
  a.bools = d_bools;
  a.t0 = ctx->d_t0;
  a.status = ctx->d_status;
  e = sufb200::launch_trunc_bundle(ctx, a, st);
  if (e != cudaSuccess)
    return noalloc_fail(SUFB200_ERR_CUDA, std::string("trunc bundle launch: ") + cudaGetErrorString(e));
  return SUFB200_OK;
}
