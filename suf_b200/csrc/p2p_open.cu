// p2p_open.cu -- the paired-GPU open in one kernel: each party packs its
// shares of a flush to eff_bits-wide words, stores them straight into the
// paired GPU's landing buffer over NVLink (plain peer stores, no copy engine,
// no library call), raises a per-CTA flag there, waits (bounded) for the
// peer's flag on its own landing buffer and adds the peer's words to its own.
//
// It replaces the exchange of OpenCollector::flush
// (src/runtime/open_collector.cpp:722-760: D2H of the packed words, the host
// channel, H2D, unpack_add_mod_kernel) and keeps its wire format: element j's
// low eff_bits bits at bit j * eff_bits of one little-endian bitstream
// (pack_eff_bits_kernel, cuda/pfss_kernels.cu:722-812).  A group of 64
// elements is exactly eff_bits words of that stream, so CTA c owns a
// contiguous run of groups: it packs them, sends them, waits for the peer's
// CTA c (which sent the same groups) and unpacks them -- no CTA waits for
// another CTA of its own grid.
//
// Set-up (sufb200_p2p_open_create / _connect): each rank cudaMallocs one
// landing area [flags: kMaxCtas u64][half 0][half 1] and exports it with
// cudaIpcGetMemHandle; the peer maps it with cudaIpcOpenMemHandle (peer
// access enabled lazily).  Call k (counted on the device, so captured
// exchanges replay with fresh numbers) writes half k & 1 of the peer's area
// and signals flag value k: the peer's kernel of call k + 2 can only run after
// the peer's kernel of call k + 1, which needed this rank's call k + 1 data,
// which this rank sends after finishing call k, so a half is never
// overwritten while it is read (each rank issues its exchanges on one
// stream, in the same order as its peer).
//
// Every wait is bounded by %globaltimer: after timeout_s the CTA records
// kStatusTimeout in the context's status word (sufb200_ctx_sync reports
// it), skips its additions and returns, so a peer that never calls ends the
// kernel instead of hanging the GPU.  Two ranks on one GPU are refused: the
// kernels wait on each other and must run on different devices.  The
// loopback form (sufb200_p2p_open_connect_self) makes an endpoint its own
// peer, so the whole kernel -- pack, stores, flag, wait, unpack and add --
// runs on one device with each CTA waiting only on its own flag.
#include <cstring>
#include <string>

#include "kernels.hpp"
#include "sufb200_internal.cuh"

namespace {

constexpr int kMaxCtas = 1024;
constexpr int kThreads = 512;
constexpr uint32_t kMagic = 0x53423250u;  // "SB2P"

struct HandleBlob {  // what one rank hands its peer (SUFB200_P2P_HANDLE_BYTES)
  uint32_t magic;
  int32_t sm_count;
  uint64_t max_words;
  cudaIpcMemHandle_t ipc;  // 64 bytes
  char pci[40];
};
static_assert(sizeof(HandleBlob) <= SUFB200_P2P_HANDLE_BYTES, "handle blob size");

int fail(int code, const std::string& msg) { return sufb200::record_error(code, msg); }

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void store_release_sys(uint64_t* p, uint64_t v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ uint64_t load_acquire_sys(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ uint64_t elem_masked(const uint64_t* __restrict__ x, size_t n, size_t j, int b) {
  const uint64_t v = j < n ? x[j] : 0ull;
  return b >= 64 ? v : (v & ((1ull << b) - 1ull));
}

struct P2PArgs {
  const uint64_t* local;
  uint64_t* out;
  size_t n;
  int b, ring, sign;
  uint64_t* peer_flags;     // the peer's landing area (mapped)
  uint64_t* peer_halves;    // its two halves, peer_max_words words each
  uint64_t peer_max_words;
  const uint64_t* my_flags;
  const uint64_t* my_halves;
  uint64_t my_max_words;
  uint64_t* calls;          // device: exchanges completed on this endpoint
  uint32_t* arrivals;       // device: CTAs of the running call that have read `calls`
  uint64_t timeout_ns;
  uint32_t* status;
};

// Groups are handled kGroupsPerIter at a time.  Packing stages the masked
// elements in shared memory and computes each output word from the two or
// three elements it covers (group-local indices: 32-bit arithmetic);
// unpacking stages the landed words the same way.  Raw 64-bit words are
// copied straight, four per thread per step.
constexpr int kGroupsPerIter = 32;  // 2,048 elements, 16 KB of staging

__global__ void __launch_bounds__(kThreads) p2p_open_kernel(const P2PArgs a) {
  __shared__ uint64_t s_buf[kGroupsPerIter * 64];
  __shared__ int s_abort;
  __shared__ uint64_t s_seq;
  // The call number comes from the endpoint's device counter, so a captured
  // sequence of exchanges replays with fresh numbers: every CTA reads the
  // counter, then counts itself in; the last CTA in resets the count and
  // advances the counter, after every CTA of this call has read it (the next
  // call starts after this kernel ends: stream order).
  if (threadIdx.x == 0) {
    s_seq = *reinterpret_cast<volatile const uint64_t*>(a.calls) + 1;
    __threadfence();
    if (atomicAdd(a.arrivals, 1u) == gridDim.x - 1) {
      *a.arrivals = 0;
      *a.calls = s_seq;
    }
  }
  __syncthreads();
  const uint64_t seq = s_seq;
  const size_t half = seq & 1;
  uint64_t* const peer_half = a.peer_halves + half * a.peer_max_words;
  const uint64_t* const my_half = a.my_halves + half * a.my_max_words;
  const size_t groups = (a.n + 63) / 64;
  const size_t per = (groups + gridDim.x - 1) / gridDim.x;
  const size_t g0 = static_cast<size_t>(blockIdx.x) * per;
  const size_t g1 = g0 + per < groups ? g0 + per : groups;
  const int b = a.b;
  const uint32_t tid = threadIdx.x, nt = blockDim.x;
  // 1. pack this CTA's groups and store them into the peer's landing half
  if (b == 64) {
    const size_t w0 = g0 * 64, w1 = g1 * 64;
    for (size_t w = w0 + tid; w < w1; w += 4 * static_cast<size_t>(nt)) {
      uint64_t v[4];
#pragma unroll
      for (int u = 0; u < 4; u++) {
        const size_t k = w + static_cast<size_t>(u) * nt;
        v[u] = k < a.n ? a.local[k] : 0ull;
      }
#pragma unroll
      for (int u = 0; u < 4; u++) {
        const size_t k = w + static_cast<size_t>(u) * nt;
        if (k < w1) peer_half[k] = v[u];
      }
    }
  } else {
    for (size_t g = g0; g < g1; g += kGroupsPerIter) {
      const uint32_t ng = static_cast<uint32_t>(g1 - g < kGroupsPerIter ? g1 - g : kGroupsPerIter);
      for (uint32_t k = tid; k < ng * 64; k += nt) s_buf[k] = elem_masked(a.local, a.n, g * 64 + k, b);
      __syncthreads();
      for (uint32_t k = tid; k < ng * static_cast<uint32_t>(b); k += nt) {
        const uint32_t gl = k / b, w = k - gl * b, start = 64u * w;
        const uint64_t* grp = s_buf + gl * 64;
        uint64_t word = 0;
        for (uint32_t e = start / b; e < 64 && e * b < start + 64; e++) {
          const int sh = static_cast<int>(e * b) - static_cast<int>(start);
          word |= sh >= 0 ? (grp[e] << sh) : (grp[e] >> (-sh));
        }
        peer_half[g * b + k] = word;
      }
      __syncthreads();
    }
  }
  __syncthreads();
  if (tid == 0) {
    __threadfence_system();
    store_release_sys(a.peer_flags + blockIdx.x, seq);
    // 2. wait (bounded) for the peer's CTA of the same index
    int abort = 0;
    const uint64_t t0 = globaltimer();
    while (load_acquire_sys(a.my_flags + blockIdx.x) < seq) {
      if (globaltimer() - t0 > a.timeout_ns) {
        atomicOr(a.status, sufb200::kStatusTimeout);
        abort = 1;
        break;
      }
      __nanosleep(32);
    }
    __threadfence();
    s_abort = abort;
  }
  __syncthreads();
  if (s_abort || g0 >= g1) return;
  // 3. unpack the peer's words of these groups and add them to ours
  const uint64_t rmask = a.ring >= 64 ? ~0ull : ((1ull << a.ring) - 1ull);
  const int rb = a.ring;
  const bool sign = a.sign && rb < 64;
  auto finish = [&](uint64_t s) -> uint64_t {
    s &= rmask;
    if (sign && ((s >> (rb - 1)) & 1ull)) s |= ~rmask;
    return s;
  };
  if (b == 64) {
    const size_t e0 = g0 * 64, e1 = (g1 * 64 < a.n) ? g1 * 64 : a.n;
    for (size_t j = e0 + tid; j < e1; j += 4 * static_cast<size_t>(nt)) {
      uint64_t v[4], l[4];
#pragma unroll
      for (int u = 0; u < 4; u++) {
        const size_t k = j + static_cast<size_t>(u) * nt;
        v[u] = k < e1 ? __ldcg(my_half + k) : 0ull;
        l[u] = k < e1 ? a.local[k] : 0ull;
      }
#pragma unroll
      for (int u = 0; u < 4; u++) {
        const size_t k = j + static_cast<size_t>(u) * nt;
        if (k < e1) a.out[k] = finish(l[u] + v[u]);
      }
    }
    return;
  }
  const uint64_t emask = (1ull << b) - 1ull;
  for (size_t g = g0; g < g1; g += kGroupsPerIter) {
    const uint32_t ng = static_cast<uint32_t>(g1 - g < kGroupsPerIter ? g1 - g : kGroupsPerIter);
    for (uint32_t k = tid; k < ng * static_cast<uint32_t>(b); k += nt) s_buf[k] = __ldcg(my_half + g * b + k);
    __syncthreads();
    for (uint32_t k = tid; k < ng * 64; k += nt) {
      const size_t j = g * 64 + k;
      if (j < a.n) {
        const uint32_t bit = k * static_cast<uint32_t>(b), w = bit >> 6, off = bit & 63u;
        uint64_t v = s_buf[w] >> off;
        if (off + b > 64) v |= s_buf[w + 1] << (64 - off);
        a.out[j] = finish(a.local[j] + (v & emask));
      }
    }
    __syncthreads();
  }
}

}  // namespace

struct sufb200_p2p_open_s {
  sufb200_ctx ctx = nullptr;
  uint8_t* area = nullptr;       // this rank's landing area (cudaMalloc)
  uint8_t* peer_area = nullptr;  // the peer's area, mapped
  uint64_t max_words = 0;
  uint64_t peer_max_words = 0;
  int grid_cap = 0;
  uint64_t* d_calls = nullptr;  // [calls (u64), arrivals (u32)], device
  bool loopback = false;        // peer_area is this endpoint's own area
  char pci[40] = {};
};

namespace {

size_t area_bytes(uint64_t max_words) { return kMaxCtas * 8 + 2 * max_words * 8; }

}  // namespace

extern "C" {

int sufb200_p2p_open_create(sufb200_ctx ctx, size_t max_words, sufb200_p2p_open* out, uint8_t* handle_out) {
  if (!ctx || !out || !handle_out) return fail(SUFB200_ERR_INVALID, "null pointer");
  *out = nullptr;
  if (ctx->device < 0) return fail(SUFB200_ERR_INVALID, "dealer-only context: the open needs a GPU");
  if (max_words == 0 || max_words > (size_t{1} << 34)) return fail(SUFB200_ERR_INVALID, "max_words out of range");
  cudaError_t e = cudaSetDevice(ctx->device);
  auto* h = new sufb200_p2p_open_s();
  h->ctx = ctx;
  h->max_words = max_words;
  h->grid_cap = ctx->sm_count < kMaxCtas ? ctx->sm_count : kMaxCtas;
  if (e == cudaSuccess) e = cudaMalloc(reinterpret_cast<void**>(&h->area), area_bytes(max_words));
  if (e == cudaSuccess) e = cudaMemset(h->area, 0, kMaxCtas * 8);
  if (e == cudaSuccess) e = cudaMalloc(reinterpret_cast<void**>(&h->d_calls), 16);
  if (e == cudaSuccess) e = cudaMemset(h->d_calls, 0, 16);
  HandleBlob blob{};
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&blob.ipc, h->area);
  if (e == cudaSuccess) e = cudaDeviceGetPCIBusId(h->pci, sizeof(h->pci), ctx->device);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    if (h->area) cudaFree(h->area);
    if (h->d_calls) cudaFree(h->d_calls);
    delete h;
    return fail(SUFB200_ERR_CUDA, std::string("p2p open set-up: ") + cudaGetErrorString(e));
  }
  blob.magic = kMagic;
  blob.sm_count = h->grid_cap;
  blob.max_words = max_words;
  std::memcpy(blob.pci, h->pci, sizeof(blob.pci));
  std::memset(handle_out, 0, SUFB200_P2P_HANDLE_BYTES);
  std::memcpy(handle_out, &blob, sizeof(blob));
  *out = h;
  return SUFB200_OK;
}

int sufb200_p2p_open_connect(sufb200_p2p_open h, const uint8_t* peer_handle) {
  if (!h || !peer_handle) return fail(SUFB200_ERR_INVALID, "null pointer");
  if (h->peer_area) return fail(SUFB200_ERR_INVALID, "already connected");
  HandleBlob blob;
  std::memcpy(&blob, peer_handle, sizeof(blob));
  if (blob.magic != kMagic) return fail(SUFB200_ERR_INVALID, "not a p2p open handle");
  if (std::strncmp(blob.pci, h->pci, sizeof(blob.pci)) == 0)
    return fail(SUFB200_ERR_UNSUPPORTED, "the peer is on this GPU: the paired kernels wait on each other and need "
                                         "two devices");
  cudaError_t e = cudaSetDevice(h->ctx->device);
  void* p = nullptr;
  if (e == cudaSuccess) e = cudaIpcOpenMemHandle(&p, blob.ipc, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return fail(SUFB200_ERR_CUDA, std::string("cudaIpcOpenMemHandle: ") + cudaGetErrorString(e));
  h->peer_area = static_cast<uint8_t*>(p);
  h->peer_max_words = blob.max_words;
  h->grid_cap = h->grid_cap < blob.sm_count ? h->grid_cap : blob.sm_count;  // both ranks launch the same grid
  return SUFB200_OK;
}

int sufb200_p2p_open_connect_self(sufb200_p2p_open h) {
  if (!h) return fail(SUFB200_ERR_INVALID, "null endpoint");
  if (h->peer_area) return fail(SUFB200_ERR_INVALID, "already connected");
  // CTA c stores into its own landing half, raises its own flag c and waits
  // for that flag: every wait is on a store the same CTA made before it.
  h->peer_area = h->area;
  h->peer_max_words = h->max_words;
  h->loopback = true;
  return SUFB200_OK;
}

int sufb200_p2p_open_exchange(sufb200_p2p_open h, const uint64_t* d_local, size_t n, int eff_bits, int ring_bits,
                              int signed_out, uint64_t* d_out, double timeout_s, void* stream) {
  if (!h) return fail(SUFB200_ERR_INVALID, "null endpoint");
  if (!h->peer_area) return fail(SUFB200_ERR_NOT_READY, "sufb200_p2p_open_connect has not been called");
  if (eff_bits < 1 || eff_bits > 64 || ring_bits < 1 || ring_bits > 64)
    return fail(SUFB200_ERR_INVALID, "eff_bits and ring_bits must be in 1..64");
  if (!(timeout_s > 0) || timeout_s > 3600) return fail(SUFB200_ERR_INVALID, "timeout must be in (0, 3600] s");
  if (n == 0) return SUFB200_OK;
  const uint64_t words = (n + 63) / 64 * static_cast<uint64_t>(eff_bits);
  if (words > h->max_words || words > h->peer_max_words)
    return fail(SUFB200_ERR_INVALID, "flush larger than the landing buffers (max_words at create)");
  if (!d_local || !d_out || (reinterpret_cast<uintptr_t>(d_local) & 7u) || (reinterpret_cast<uintptr_t>(d_out) & 7u))
    return fail(SUFB200_ERR_INVALID, "null or misaligned device pointer");
  cudaError_t e = cudaSetDevice(h->ctx->device);
  if (e != cudaSuccess) return fail(SUFB200_ERR_CUDA, std::string("cudaSetDevice: ") + cudaGetErrorString(e));
  P2PArgs a{};
  a.local = d_local;
  a.out = d_out;
  a.n = n;
  a.b = eff_bits;
  a.ring = ring_bits;
  a.sign = signed_out ? 1 : 0;
  a.peer_flags = reinterpret_cast<uint64_t*>(h->peer_area);
  a.peer_halves = reinterpret_cast<uint64_t*>(h->peer_area + kMaxCtas * 8);
  a.peer_max_words = h->peer_max_words;
  a.my_flags = reinterpret_cast<const uint64_t*>(h->area);
  a.my_halves = reinterpret_cast<const uint64_t*>(h->area + kMaxCtas * 8);
  a.my_max_words = h->max_words;
  a.calls = h->d_calls;
  a.arrivals = reinterpret_cast<uint32_t*>(h->d_calls + 1);
  a.timeout_ns = static_cast<uint64_t>(timeout_s * 1e9);
  a.status = h->ctx->d_status;
  const uint64_t groups = (n + 63) / 64;
  const int grid = static_cast<int>(groups < static_cast<uint64_t>(h->grid_cap) ? groups : h->grid_cap);
  p2p_open_kernel<<<grid, kThreads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(a);
  e = cudaGetLastError();
  return e == cudaSuccess ? SUFB200_OK : fail(SUFB200_ERR_CUDA, std::string("p2p open launch: ") + cudaGetErrorString(e));
}

int sufb200_p2p_open_destroy(sufb200_p2p_open h) {
  if (!h) return SUFB200_OK;
  cudaSetDevice(h->ctx->device);
  cudaError_t e = cudaDeviceSynchronize();
  if (h->peer_area && !h->loopback) cudaIpcCloseMemHandle(h->peer_area);
  if (h->area) cudaFree(h->area);
  if (h->d_calls) cudaFree(h->d_calls);
  delete h;
  return e == cudaSuccess ? SUFB200_OK : fail(SUFB200_ERR_CUDA, std::string("p2p open teardown: ") + cudaGetErrorString(e));
}

}  // extern "C"
