// capi.cu -- the extern "C" boundary of libsufb200.so (include/sufb200.h).
//
// Argument validation, context lifetime, error reporting and the host-buffer
// entry points.  No path here falls back to host evaluation: every
// evaluation runs on the device or returns an error.
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <random>
#include <string>
#include <algorithm>
#include <vector>

#include "host_aes.hpp"
#include "kernels.hpp"
#include "keygen.hpp"
#include "prefix.cuh"
#include "primitives.hpp"
#include "sufb200_internal.cuh"

namespace sufb200 {

bool pdl_enabled() {
  static const bool v = [] {
    const char* e = std::getenv("SUFB200_PDL");
    return !(e && std::string(e) == "0");
  }();
  return v;
}

}  // namespace sufb200

namespace {

thread_local std::string g_err;

int fail(int code, const std::string& msg) {
  g_err = msg;
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(SUFB200_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

#define SUFB200_CHECK_CUDA(expr, what)          \
  do {                                          \
    cudaError_t e_ = (expr);                    \
    if (e_ != cudaSuccess) return cuda_fail(e_, what); \
  } while (0)

cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

__global__ void probe_kernel(uint32_t* out) {
  extern __shared__ __align__(16) uint8_t sufb200_dyn_smem[];
  if (threadIdx.x == 0) out[0] = static_cast<uint32_t>(__cvta_generic_to_shared(sufb200_dyn_smem));
}

bool aligned8(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 7u) == 0; }

// Broadcast-key batches at least this large take the shared-prefix path
// (prefix.cuh); SUFB200_PREFIX=0 in the environment selects the direct walk.
size_t prefix_min_n() {
  static const size_t v = [] {
    const char* e = std::getenv("SUFB200_PREFIX");
    if (e && std::string(e) == "0") return ~static_cast<size_t>(0);
    return static_cast<size_t>(16384);
  }();
  return v;
}

constexpr size_t kAccBytes = 256;  // RangeAcc slot, keeps the frontier 256-byte aligned

// Host-side per-context device buffers for the host-buffer entry points.
struct HostIo {
  std::mutex mu;
  cudaStream_t stream = nullptr;
  cudaStream_t copy = nullptr;    // device-to-host copies of finished chunks
  cudaEvent_t chunk_done = nullptr;
  uint8_t* d_keys = nullptr;
  size_t keys_cap = 0;
  uint64_t* d_xs = nullptr;
  size_t xs_cap = 0;
  uint8_t* d_out = nullptr;
  size_t out_cap = 0;
};

int grow(void** p, size_t* cap, size_t want) {
  if (want <= *cap) return 0;
  if (*p) cudaFree(*p);
  *p = nullptr;
  *cap = 0;
  cudaError_t e = cudaMalloc(p, want);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc (host-io buffer)");
  *cap = want;
  return 0;
}

std::mutex g_io_mu;
std::vector<std::pair<sufb200_ctx, HostIo*>> g_io;

HostIo* io_of(sufb200_ctx ctx, bool create) {
  std::lock_guard<std::mutex> lk(g_io_mu);
  for (auto& kv : g_io)
    if (kv.first == ctx) return kv.second;
  if (!create) return nullptr;
  HostIo* io = new HostIo();
  g_io.emplace_back(ctx, io);
  return io;
}

void io_release(sufb200_ctx ctx) {
  std::lock_guard<std::mutex> lk(g_io_mu);
  for (size_t i = 0; i < g_io.size(); i++) {
    if (g_io[i].first == ctx) {
      HostIo* io = g_io[i].second;
      if (io->d_keys) cudaFree(io->d_keys);
      if (io->d_xs) cudaFree(io->d_xs);
      if (io->d_out) cudaFree(io->d_out);
      if (io->stream) cudaStreamDestroy(io->stream);
      if (io->copy) cudaStreamDestroy(io->copy);
      if (io->chunk_done) cudaEventDestroy(io->chunk_done);
      delete io;
      g_io.erase(g_io.begin() + static_cast<long>(i));
      return;
    }
  }
}

int check_ctx(sufb200_ctx ctx, bool need_prg) {
  if (!ctx) return fail(SUFB200_ERR_INVALID, "null context");
  if (ctx->device < 0) return fail(SUFB200_ERR_UNSUPPORTED, "host-only context: no device to evaluate on");
  if (need_prg && !ctx->prg_ready) return fail(SUFB200_ERR_NOT_READY, "sufb200_prg_init has not been called");
  cudaError_t e = cudaSetDevice(ctx->device);
  if (e != cudaSuccess) return cuda_fail(e, "cudaSetDevice");
  return 0;
}

int myl7_args(sufb200_ctx ctx, int group, int in_bits, const void* keys, size_t key_bytes, const void* xs,
              int out_bytes, const void* out) {
  if (group != SUFB200_GROUP_ADD && group != SUFB200_GROUP_XOR) return fail(SUFB200_ERR_INVALID, "bad group");
  if (in_bits < 1 || in_bits > 64) return fail(SUFB200_ERR_INVALID, "in_bits out of range [1,64]");
  if (out_bytes < 1 || out_bytes > 8)
    return fail(SUFB200_ERR_UNSUPPORTED, "out_bytes must be 1..8 (one 16-byte payload chunk, low 8 bytes)");
  if (key_bytes != sufb200::host::myl7_key_bytes(in_bits, out_bytes))
    return fail(SUFB200_ERR_KEY, "key_bytes does not match in_bits/out_bytes (myl7 layout, one chunk)");
  if (!keys || !xs || !out) return fail(SUFB200_ERR_INVALID, "null pointer");
  if (!aligned8(xs)) return fail(SUFB200_ERR_INVALID, "xs must be 8-byte aligned");
  if (out_bytes == 8 && !aligned8(out)) return fail(SUFB200_ERR_INVALID, "out must be 8-byte aligned");
  (void)ctx;
  return 0;
}

}  // namespace

namespace sufb200 {
int record_error(int code, const std::string& msg) { return fail(code, msg); }

cudaError_t probe_dyn_smem_base(uint32_t* d_out, cudaStream_t st) {
  probe_kernel<<<1, 32, 1024, st>>>(d_out);
  return cudaGetLastError();
}
}  // namespace sufb200

extern "C" {

int sufb200_version(void) { return 10000; }

const char* sufb200_last_error(void) { return g_err.c_str(); }

int sufb200_ctx_create(int device, sufb200_ctx* out) {
  if (!out) return fail(SUFB200_ERR_INVALID, "null out");
  *out = nullptr;
  if (device == SUFB200_HOST_ONLY) {
    auto* ctx = new sufb200_ctx_s();
    ctx->device = SUFB200_HOST_ONLY;
    *out = ctx;
    return SUFB200_OK;
  }
  int ndev = 0;
  cudaError_t e = cudaGetDeviceCount(&ndev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDeviceCount");
  if (device < 0 || device >= ndev) return fail(SUFB200_ERR_INVALID, "device index out of range");
  SUFB200_CHECK_CUDA(cudaSetDevice(device), "cudaSetDevice");
  cudaDeviceProp prop;
  SUFB200_CHECK_CUDA(cudaGetDeviceProperties(&prop, device), "cudaGetDeviceProperties");
  if (prop.major != 10)
    return fail(SUFB200_ERR_UNSUPPORTED, "libsufb200 is built for sm_100a (B200); device is sm_" +
                                             std::to_string(prop.major) + std::to_string(prop.minor));
  auto* ctx = new sufb200_ctx_s();
  ctx->device = device;
  ctx->sm_count = prop.multiProcessorCount;
  const auto& tabs = sufb200::host::aes_tables();
  e = cudaMalloc(&ctx->d_t0, 256 * sizeof(uint32_t));
  if (e == cudaSuccess) e = cudaMemcpy(ctx->d_t0, tabs.t0, 256 * sizeof(uint32_t), cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaMalloc(&ctx->d_status, 2 * sizeof(uint32_t));
  if (e == cudaSuccess) e = cudaMemset(ctx->d_status, 0, 2 * sizeof(uint32_t));
  uint32_t base = 0;
  if (e == cudaSuccess) e = sufb200::probe_dyn_smem_base(ctx->d_status + 1, nullptr);
  if (e == cudaSuccess) e = cudaMemcpy(&base, ctx->d_status + 1, sizeof(uint32_t), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) {
    int rc = cuda_fail(e, "context setup");
    sufb200_ctx_destroy(ctx);
    return rc;
  }
  if (base > sufb200::kTabBase || sufb200::kTabEnd - base > prop.sharedMemPerBlockOptin) {
    sufb200_ctx_destroy(ctx);
    return fail(SUFB200_ERR_UNSUPPORTED, "shared-memory window does not fit the AES table layout (base " +
                                             std::to_string(base) + ")");
  }
  ctx->dyn_base = base;
  ctx->aes_dyn_bytes = sufb200::kTabEnd - base;
  // A private stream-ordered pool for per-call scratch that keeps its memory
  // mapped between calls (the default pool returns it at every sync).
  cudaMemPoolProps pp{};
  pp.allocType = cudaMemAllocationTypePinned;
  pp.location.type = cudaMemLocationTypeDevice;
  pp.location.id = device;
  e = cudaMemPoolCreate(&ctx->pool, &pp);
  if (e == cudaSuccess) {
    uint64_t keep = ~0ull;
    e = cudaMemPoolSetAttribute(ctx->pool, cudaMemPoolAttrReleaseThreshold, &keep);
  }
  if (e != cudaSuccess) {
    int rc = cuda_fail(e, "memory pool setup");
    sufb200_ctx_destroy(ctx);
    return rc;
  }
  *out = ctx;
  return SUFB200_OK;
}

int sufb200_ctx_destroy(sufb200_ctx ctx) {
  if (!ctx) return SUFB200_OK;
  if (ctx->device < 0) {
    delete ctx;
    return SUFB200_OK;
  }
  cudaSetDevice(ctx->device);
  io_release(ctx);
  if (ctx->d_t0) cudaFree(ctx->d_t0);
  if (ctx->d_status) cudaFree(ctx->d_status);
  if (ctx->d_scratch) cudaFree(ctx->d_scratch);
  if (ctx->pool) {
    cudaDeviceSynchronize();
    cudaMemPoolDestroy(ctx->pool);
  }
  delete ctx;
  return SUFB200_OK;
}

int sufb200_ctx_sm_count(sufb200_ctx ctx) { return ctx ? ctx->sm_count : 0; }

int sufb200_probe_aes_engine(sufb200_ctx ctx, double* blocks_per_s) {
  if (int rc = check_ctx(ctx, true)) return rc;
  if (!blocks_per_s) return fail(SUFB200_ERR_INVALID, "null out");
  SUFB200_CHECK_CUDA(sufb200::probe_aes_engine(ctx, blocks_per_s), "AES engine probe");
  return sufb200_ctx_sync(ctx, nullptr);
}

int sufb200_ctx_sync(sufb200_ctx ctx, void* stream) {
  if (int rc = check_ctx(ctx, false)) return rc;
  SUFB200_CHECK_CUDA(cudaStreamSynchronize(as_stream(stream)), "cudaStreamSynchronize");
  uint32_t st = 0;
  SUFB200_CHECK_CUDA(cudaMemcpy(&st, ctx->d_status, sizeof(uint32_t), cudaMemcpyDeviceToHost), "read status");
  if (st) {
    SUFB200_CHECK_CUDA(cudaMemset(ctx->d_status, 0, sizeof(uint32_t)), "clear status");
    if (st & sufb200::kStatusSmemLayout) return fail(SUFB200_ERR_CUDA, "kernel found an unexpected shared-memory layout");
    if (st & sufb200::kStatusBadKeyHeader)
      return fail(SUFB200_ERR_KEY, "a key header did not match the call (in_bits / chunks / party / payload_len)");
    if (st & sufb200::kStatusTimeout) return fail(SUFB200_ERR_CUDA, "a kernel's bounded wait gave up (results invalid)");
    return fail(SUFB200_ERR_INVALID, "device reported a bad argument");
  }
  return SUFB200_OK;
}

int sufb200_prg_init(sufb200_ctx ctx, const uint8_t* state, size_t len) {
  if (!ctx || !state) return fail(SUFB200_ERR_INVALID, "null argument");
  if (len < 64) return fail(SUFB200_ERR_INVALID, "PRG state needs >= 64 bytes (4 AES-128 keys)");
  uint32_t w[4][44];
  for (int j = 0; j < 4; j++) sufb200::host::aes128_expand_words(state + 16 * j, w[j]);
  for (int h = 0; h < 2; h++)
    for (int r = 0; r < 11; r++)
      for (int c = 0; c < 4; c++) {
        ctx->prg.base[h][r][c] = w[h][4 * r + c];
        ctx->prg.diff[h][r][c] = w[h][4 * r + c] ^ w[h + 2][4 * r + c];
      }
  for (int j = 0; j < 4; j++)
    for (int r = 0; r < 11; r++)
      for (int c = 0; c < 4; c++) ctx->prg4.rk[j][r][c] = w[j][4 * r + c];
  ctx->prg_ready = true;
  return SUFB200_OK;
}

size_t sufb200_myl7_key_bytes(int in_bits, int payload_len) {
  if (in_bits < 1 || in_bits > 64 || payload_len < 1) return 0;
  return sufb200::host::myl7_key_bytes(in_bits, payload_len);
}

static sufb200::host::PrgHostKeys host_keys(const sufb200_ctx_s* ctx) {
  sufb200::host::PrgHostKeys k;
  for (int j = 0; j < 4; j++)
    for (int r = 0; r < 11; r++)
      for (int c = 0; c < 4; c++) k.rk[j][4 * r + c] = ctx->prg4.rk[j][r][c];
  return k;
}

int sufb200_myl7_gen(sufb200_ctx ctx, int group, int in_bits, uint64_t alpha, const uint8_t* payload,
                     int payload_len, const uint8_t* seeds0, const uint8_t* seeds1, uint8_t* key0, uint8_t* key1) {
  if (!ctx) return fail(SUFB200_ERR_INVALID, "null context");
  if (!ctx->prg_ready) return fail(SUFB200_ERR_NOT_READY, "sufb200_prg_init has not been called");
  if (!payload || !seeds0 || !seeds1 || !key0 || !key1) return fail(SUFB200_ERR_INVALID, "null pointer");
  if (group != SUFB200_GROUP_ADD && group != SUFB200_GROUP_XOR) return fail(SUFB200_ERR_INVALID, "bad group");
  if (in_bits < 1 || in_bits > 64 || payload_len < 1 || (payload_len + 15) / 16 > 255)
    return fail(SUFB200_ERR_INVALID, "in_bits / payload_len out of range");
  const auto k = host_keys(ctx);
  if (sufb200::host::myl7_gen_pair(k, group == SUFB200_GROUP_ADD, in_bits, alpha, payload, payload_len, seeds0,
                                   seeds1, key0, key1))
    return fail(SUFB200_ERR_INVALID, "myl7 keygen rejected its arguments");
  return SUFB200_OK;
}

int sufb200_myl7_gen_batch(sufb200_ctx ctx, int group, int in_bits, const uint64_t* alphas, size_t n,
                           const uint8_t* payload, int payload_len, const uint8_t* seeds0, const uint8_t* seeds1,
                           uint8_t* keys0, uint8_t* keys1) {
  if (!ctx) return fail(SUFB200_ERR_INVALID, "null context");
  if (!ctx->prg_ready) return fail(SUFB200_ERR_NOT_READY, "sufb200_prg_init has not been called");
  if (n == 0) return SUFB200_OK;
  if (!alphas || !payload || !seeds0 || !seeds1 || !keys0 || !keys1) return fail(SUFB200_ERR_INVALID, "null pointer");
  if (group != SUFB200_GROUP_ADD && group != SUFB200_GROUP_XOR) return fail(SUFB200_ERR_INVALID, "bad group");
  if (in_bits < 1 || in_bits > 64 || payload_len < 1 || (payload_len + 15) / 16 > 255)
    return fail(SUFB200_ERR_INVALID, "in_bits / payload_len out of range");
  const auto k = host_keys(ctx);
  if (sufb200::host::myl7_gen_batch(k, group == SUFB200_GROUP_ADD, in_bits, alphas, n, payload, payload_len, seeds0,
                                    seeds1, keys0, keys1))
    return fail(SUFB200_ERR_INVALID, "myl7 batch keygen failed");
  return SUFB200_OK;
}

int sufb200_myl7_dcf_eval(sufb200_ctx ctx, int group, int in_bits, const uint8_t* d_keys, size_t key_bytes,
                          int broadcast, const uint64_t* d_xs, size_t n, int out_bytes, void* d_out, void* stream) {
  if (int rc = check_ctx(ctx, true)) return rc;
  if (n == 0) return SUFB200_OK;
  if (int rc = myl7_args(ctx, group, in_bits, d_keys, key_bytes, d_xs, out_bytes, d_out)) return rc;
  sufb200::DcfLaunch a{d_keys, key_bytes, d_xs, n, d_out, ctx->d_t0, ctx->d_status, in_bits, out_bytes};
  cudaStream_t st = as_stream(stream);
  if (broadcast && n >= prefix_min_n()) {
    const uint32_t kmax = sufb200::prefix_budget(n);
    uint8_t* scratch = nullptr;
    SUFB200_CHECK_CUDA(cudaMallocFromPoolAsync(reinterpret_cast<void**>(&scratch), kAccBytes + 32ull * kmax,
                                               ctx->pool, st),
                       "prefix scratch allocation");
    auto* acc = reinterpret_cast<sufb200::RangeAcc*>(scratch);
    auto* F = reinterpret_cast<sufb200::FrontierEntry*>(scratch + kAccBytes);
    sufb200::FrontierBatch fb{};
    fb.q[0] = sufb200::FrontierLaunch{d_keys, in_bits, out_bytes, acc, kmax, F, ctx->d_t0, ctx->d_status};
    fb.nq = 1;
    cudaError_t e = sufb200::launch_range(ctx, d_xs, n, acc, st);
    if (e == cudaSuccess) e = sufb200::launch_frontier(ctx, group, fb, st);
    if (e == cudaSuccess) e = sufb200::launch_myl7_bcast_prefix(ctx, group, a, acc, kmax, F, st);
    cudaFreeAsync(scratch, st);
    if (e != cudaSuccess) return cuda_fail(e, "myl7 DCF prefix launch");
    return SUFB200_OK;
  }
  SUFB200_CHECK_CUDA(sufb200::launch_myl7_eval(ctx, group, a, broadcast ? 1 : 0, st), "myl7 DCF eval launch");
  return SUFB200_OK;
}

int sufb200_myl7_dcf_eval_host(sufb200_ctx ctx, int group, int in_bits, const uint8_t* keys, size_t key_bytes,
                               int broadcast, const uint64_t* xs, size_t n, int out_bytes, uint8_t* outs) {
  if (int rc = check_ctx(ctx, true)) return rc;
  if (n == 0) return SUFB200_OK;
  if (int rc = myl7_args(ctx, group, in_bits, keys, key_bytes, xs, out_bytes, outs)) return rc;
  // Host-side header check of every key, as the reference adapter does per element.
  const size_t nk = broadcast ? 1 : n;
  for (size_t i = 0; i < nk; i++) {
    const uint8_t* k = keys + i * key_bytes;
    uint32_t pl;
    std::memcpy(&pl, k + 4, 4);
    if (k[0] != in_bits || k[1] != 1 || k[2] > 1 || pl != static_cast<uint32_t>(out_bytes))
      return fail(SUFB200_ERR_KEY, "key " + std::to_string(i) + ": header does not match in_bits/out_bytes");
  }
  HostIo* io = io_of(ctx, true);
  std::lock_guard<std::mutex> lk(io->mu);
  if (!io->stream) SUFB200_CHECK_CUDA(cudaStreamCreateWithFlags(&io->stream, cudaStreamNonBlocking), "stream");
  if (int rc = grow(reinterpret_cast<void**>(&io->d_keys), &io->keys_cap, nk * key_bytes)) return rc;
  if (int rc = grow(reinterpret_cast<void**>(&io->d_xs), &io->xs_cap, n * 8)) return rc;
  if (int rc = grow(reinterpret_cast<void**>(&io->d_out), &io->out_cap, n * static_cast<size_t>(out_bytes)))
    return rc;
  SUFB200_CHECK_CUDA(cudaMemcpyAsync(io->d_keys, keys, nk * key_bytes, cudaMemcpyHostToDevice, io->stream), "H2D keys");
  SUFB200_CHECK_CUDA(cudaMemcpyAsync(io->d_xs, xs, n * 8, cudaMemcpyHostToDevice, io->stream), "H2D xs");
  sufb200::DcfLaunch a{io->d_keys, key_bytes, io->d_xs, n, io->d_out, ctx->d_t0, ctx->d_status, in_bits, out_bytes};
  SUFB200_CHECK_CUDA(sufb200::launch_myl7_eval(ctx, group, a, broadcast ? 1 : 0, io->stream), "myl7 DCF eval launch");
  SUFB200_CHECK_CUDA(cudaMemcpyAsync(outs, io->d_out, n * static_cast<size_t>(out_bytes), cudaMemcpyDeviceToHost,
                                     io->stream),
                     "D2H outs");
  return sufb200_ctx_sync(ctx, io->stream);
}

int sufb200_trunc_gen(int kind, int frac_bits, uint64_t rng_seed, sufb200_trunc_desc* d0, sufb200_trunc_desc* d1,
                      uint64_t* thetas, uint64_t* r_in_out) {
  if (!d0 || !d1 || !thetas) return fail(SUFB200_ERR_INVALID, "null pointer");
  if (sufb200::host::trunc_gen(kind, frac_bits, rng_seed, d0, d1, thetas, r_in_out))
    return fail(SUFB200_ERR_INVALID, "bad truncation kind / frac_bits");
  return SUFB200_OK;
}

int sufb200_trunc_gen_elem(int kind, int frac_bits, uint64_t rng_seed, size_t n, sufb200_trunc_desc* shape0,
                           sufb200_trunc_desc* shape1, uint64_t* words0, uint64_t* words1, uint64_t* thetas,
                           uint64_t* r_in) {
  if (!shape0 || !shape1 || (n && (!words0 || !words1 || !thetas || !r_in))) return fail(SUFB200_ERR_INVALID, "null pointer");
  if (sufb200::host::trunc_gen_elem(kind, frac_bits, rng_seed, n, shape0, shape1, words0, words1, thetas, r_in))
    return fail(SUFB200_ERR_INVALID, "bad truncation kind / frac_bits");
  return SUFB200_OK;
}

int sufb200_trunc_bundle_eval_elem(sufb200_ctx ctx, const sufb200_trunc_desc* shape, const uint8_t* const* d_keys,
                                   const size_t* key_bytes, const uint64_t* d_words, const uint64_t* d_xhat, size_t n,
                                   uint64_t* d_y, uint64_t* d_bools, void* stream) {
  if (int rc = check_ctx(ctx, true)) return rc;
  if (!shape || !d_keys || !key_bytes) return fail(SUFB200_ERR_INVALID, "null pointer");
  if (shape->nq < 0 || shape->nq > 4) return fail(SUFB200_ERR_UNSUPPORTED, "bundle has more than 4 slots");
  if (shape->kind < 0 || shape->kind > 2 || shape->party < 0 || shape->party > 1 || shape->frac_bits < 0 ||
      shape->frac_bits > 64)
    return fail(SUFB200_ERR_INVALID, "bad kind / party / frac_bits");
  if (n == 0) return SUFB200_OK;
  if (!d_words || !d_xhat || !d_y || !aligned8(d_words) || !aligned8(d_xhat) || !aligned8(d_y) ||
      (d_bools && !aligned8(d_bools)))
    return fail(SUFB200_ERR_INVALID, "null or misaligned device pointer");
  sufb200::TruncElemLaunch a{};
  a.shape = *shape;
  bool aligned = true;
  for (int q = 0; q < shape->nq; q++) {
    const int nb = shape->q_bits[q];
    if (nb < 1 || nb > 64) return fail(SUFB200_ERR_INVALID, "slot in_bits out of range");
    if (!d_keys[q]) return fail(SUFB200_ERR_INVALID, "null key array");
    if (key_bytes[q] != sufb200::host::myl7_key_bytes(nb, 8))
      return fail(SUFB200_ERR_KEY, "key size does not match an 8-byte myl7 key of the slot's width");
    a.keys[q] = d_keys[q];
    a.key_bytes[q] = key_bytes[q];
    aligned = aligned && (key_bytes[q] % 8 == 0) && (reinterpret_cast<uintptr_t>(d_keys[q]) % 8 == 0);
  }
  a.words = d_words;
  a.xhat = d_xhat;
  a.n = n;
  a.y = d_y;
  a.bools = d_bools;
  a.t0 = ctx->d_t0;
  a.status = ctx->d_status;
  const cudaError_t e = sufb200::launch_trunc_bundle_elem(ctx, a, aligned ? 1 : 0, as_stream(stream));
  if (e != cudaSuccess) return cuda_fail(e, "per-element bundle launch");
  return SUFB200_OK;
}

size_t sufb200_elem_keys_soa_bytes(int in_bits, size_t n) {
  if (in_bits < 1 || in_bits > 64) return 0;
  return sufb200::elem_soa_bytes(in_bits, n);
}

int sufb200_elem_keys_to_soa(sufb200_ctx ctx, int in_bits, int party, const uint8_t* d_keys, size_t key_bytes,
                             size_t n, uint8_t* d_soa, void* stream) {
  if (int rc = check_ctx(ctx, false)) return rc;
  if (in_bits < 1 || in_bits > 64 || (party != 0 && party != 1))
    return fail(SUFB200_ERR_INVALID, "in_bits must be 1..64 and party 0 or 1");
  if (key_bytes != sufb200::host::myl7_key_bytes(in_bits, 8))
    return fail(SUFB200_ERR_KEY, "key size does not match an 8-byte myl7 key of this width");
  if (n == 0) return SUFB200_OK;
  if (!d_keys || !d_soa || (reinterpret_cast<uintptr_t>(d_soa) & 15u))
    return fail(SUFB200_ERR_INVALID, "null keys, or a layout buffer that is not 16-byte aligned");
  SUFB200_CHECK_CUDA(sufb200::launch_elem_keys_to_soa(ctx, d_keys, key_bytes, in_bits, party, n, d_soa,
                                                      as_stream(stream)),
                     "per-element key rearrangement launch");
  return SUFB200_OK;
}

int sufb200_trunc_bundle_eval_elem_soa(sufb200_ctx ctx, const sufb200_trunc_desc* shape, const uint8_t* const* d_soa,
                                       const uint64_t* d_words, const uint64_t* d_xhat, size_t n, uint64_t* d_y,
                                       uint64_t* d_bools, void* stream) {
  if (int rc = check_ctx(ctx, true)) return rc;
  if (!shape || !d_soa) return fail(SUFB200_ERR_INVALID, "null pointer");
  if (shape->nq < 0 || shape->nq > 4) return fail(SUFB200_ERR_UNSUPPORTED, "bundle has more than 4 slots");
  if (shape->kind < 0 || shape->kind > 2 || shape->party < 0 || shape->party > 1 || shape->frac_bits < 0 ||
      shape->frac_bits > 64)
    return fail(SUFB200_ERR_INVALID, "bad kind / party / frac_bits");
  if (n == 0) return SUFB200_OK;
  if (!d_words || !d_xhat || !d_y || !aligned8(d_words) || !aligned8(d_xhat) || !aligned8(d_y) ||
      (d_bools && !aligned8(d_bools)))
    return fail(SUFB200_ERR_INVALID, "null or misaligned device pointer");
  sufb200::TruncElemLaunch a{};
  a.shape = *shape;
  for (int q = 0; q < shape->nq; q++) {
    const int nb = shape->q_bits[q];
    if (nb < 1 || nb > 64) return fail(SUFB200_ERR_INVALID, "slot in_bits out of range");
    if (!d_soa[q] || (reinterpret_cast<uintptr_t>(d_soa[q]) & 15u))
      return fail(SUFB200_ERR_INVALID, "null or unaligned key layout");
    a.keys[q] = d_soa[q];
    a.key_bytes[q] = 0;
  }
  a.words = d_words;
  a.xhat = d_xhat;
  a.n = n;
  a.y = d_y;
  a.bools = d_bools;
  a.t0 = ctx->d_t0;
  a.status = ctx->d_status;
  const cudaError_t e = sufb200::launch_trunc_bundle_elem(ctx, a, 2, as_stream(stream));
  if (e != cudaSuccess) return cuda_fail(e, "per-element bundle launch");
  return SUFB200_OK;
}

namespace {

// Where the host entry point wants finished chunks: after the main kernel of
// elements [i0, i1) the results are copied to the caller's host buffers on a
// second stream, overlapping the next chunk's evaluation.
struct ChunkSink {
  cudaStream_t copy;
  cudaEvent_t done;
  uint64_t* y;      // host
  uint64_t* bools;  // host or null
  size_t chunk;     // elements per main-kernel launch
};

int enqueue_chunk_copy(const ChunkSink& k, cudaStream_t st, const uint64_t* d_y, const uint64_t* d_b, size_t i0,
                       size_t i1) {
  SUFB200_CHECK_CUDA(cudaEventRecord(k.done, st), "chunk event");
  SUFB200_CHECK_CUDA(cudaStreamWaitEvent(k.copy, k.done, 0), "chunk wait");
  SUFB200_CHECK_CUDA(cudaMemcpyAsync(k.y + i0, d_y + i0, (i1 - i0) * 8, cudaMemcpyDeviceToHost, k.copy), "D2H y");
  if (k.bools)
    SUFB200_CHECK_CUDA(cudaMemcpyAsync(k.bools + 3 * i0, d_b + 3 * i0, (i1 - i0) * 24, cudaMemcpyDeviceToHost, k.copy),
                       "D2H bools");
  return SUFB200_OK;
}

int trunc_bundle_impl(sufb200_ctx ctx, const sufb200_trunc_desc* desc, const uint8_t* const* keys,
                      const size_t* key_bytes, const uint64_t* d_xhat, size_t n, uint64_t* d_y, uint64_t* d_bools,
                      void* stream, const ChunkSink* sink);
int trunc_pair_core(sufb200_ctx ctx, sufb200::TruncLaunch a0, sufb200::TruncLaunch a1, const uint64_t* d_xhat,
                    size_t n, uint64_t* d_y0, uint64_t* d_y1, cudaStream_t st);

}  // namespace

int sufb200_trunc_bundle_eval(sufb200_ctx ctx, const sufb200_trunc_desc* desc, const uint8_t* const* keys,
                              const size_t* key_bytes, const uint64_t* d_xhat, size_t n, uint64_t* d_y,
                              uint64_t* d_bools, void* stream) {
  return trunc_bundle_impl(ctx, desc, keys, key_bytes, d_xhat, n, d_y, d_bools, stream, nullptr);
}

namespace {

// Descriptor checks of one bundle.
int check_bundle_desc(const sufb200_trunc_desc* desc, const uint8_t* const* keys, const size_t* key_bytes) {
  if (!desc || !keys || !key_bytes) return fail(SUFB200_ERR_INVALID, "null pointer");
  if (desc->nq < 0 || desc->nq > 4) return fail(SUFB200_ERR_UNSUPPORTED, "bundle has more than 4 queries");
  if (desc->kind < 0 || desc->kind > 2 || desc->party < 0 || desc->party > 1)
    return fail(SUFB200_ERR_INVALID, "bad kind / party");
  if (desc->frac_bits < 0 || desc->frac_bits > 64) return fail(SUFB200_ERR_INVALID, "frac_bits out of range");
  const int idx[5] = {desc->carry_a, desc->carry_b, desc->sign_a, desc->sign_b, desc->wrap_q};
  for (int v : idx)
    if (v >= desc->nq) return fail(SUFB200_ERR_INVALID, "query index out of range");
  if ((desc->carry_a >= 0) != (desc->carry_b >= 0) || (desc->sign_a >= 0) != (desc->sign_b >= 0))
    return fail(SUFB200_ERR_INVALID, "rotation operands must come in pairs");
  return SUFB200_OK;
}

// Header checks of the bundle's query keys, appended to `blob` 16-byte
// aligned; key_off[q] receives each key's offset in the blob.
int pack_bundle_keys(const sufb200_trunc_desc& desc, const uint8_t* const* keys, const size_t* key_bytes,
                     std::vector<uint8_t>& blob, uint32_t key_off[4]) {
  for (int q = 0; q < desc.nq; q++) {
    const int nb = desc.q_bits[q];
    if (nb < 1 || nb > 64) return fail(SUFB200_ERR_INVALID, "query in_bits out of range");
    if (!keys[q] || key_bytes[q] != sufb200::host::myl7_key_bytes(nb, 8))
      return fail(SUFB200_ERR_KEY, "query " + std::to_string(q) + ": key size does not match an 8-byte myl7 key");
    const uint8_t* k = keys[q];
    uint32_t pl;
    std::memcpy(&pl, k + 4, 4);
    if (k[0] != nb || k[1] != 1 || k[2] != desc.party || pl != 8)
      return fail(SUFB200_ERR_KEY, "query " + std::to_string(q) + ": key header does not match the bundle");
    key_off[q] = static_cast<uint32_t>(blob.size());
    blob.insert(blob.end(), k, k + key_bytes[q]);
    while (blob.size() % 16) blob.push_back(0);
  }
  return SUFB200_OK;
}

// True when every query of the bundles takes its full domain within the
// shared-prefix budget (2^in_bits <= kmax): no range pass is needed.
bool narrow_queries(const sufb200_trunc_desc* d, int nd, uint32_t kmax) {
  for (int b = 0; b < nd; b++)
    for (int q = 0; q < d[b].nq; q++)
      if (d[b].q_bits[q] >= 32 || (1ull << d[b].q_bits[q]) > kmax) return false;
  return true;
}

// One party's bundle with its keys already on the device (a.key, xhat, n,
// y, bools set): range + frontier + the resuming main pass at shared-prefix
// sizes (scratch for the range and the frontier tables from the pool,
// stream-ordered), else the one-pass kernel.  No host copies.
int single_core(sufb200_ctx ctx, sufb200::TruncLaunch a, cudaStream_t st, const ChunkSink* sink) {
  const size_t n = a.n;
  const sufb200_trunc_desc* desc = &a.desc;
  uint64_t* d_y = a.y;
  uint64_t* d_bools = a.bools;
  a.t0 = ctx->d_t0;
  a.status = ctx->d_status;
  const bool prefix = n >= prefix_min_n() && desc->nq > 0;
  cudaError_t e = cudaSuccess;
  if (!prefix) {
    e = sufb200::launch_trunc_bundle(ctx, a, st);
    if (e == cudaSuccess && sink)
      if (int rc = enqueue_chunk_copy(*sink, st, d_y, d_bools, 0, n)) return rc;
    if (e != cudaSuccess) return cuda_fail(e, "trunc bundle launch");
    return SUFB200_OK;
  }
  const uint32_t kmax = sufb200::prefix_budget(n);
  uint8_t* scratch = nullptr;
  SUFB200_CHECK_CUDA(cudaMallocFromPoolAsync(reinterpret_cast<void**>(&scratch),
                                             kAccBytes + 32ull * kmax * static_cast<size_t>(desc->nq) + 256,
                                             ctx->pool, st),
                     "bundle scratch allocation");
  auto* acc = reinterpret_cast<sufb200::RangeAcc*>(scratch);
  sufb200::FrontierEntry* F[4] = {nullptr, nullptr, nullptr, nullptr};
  sufb200::FrontierBatch fb{};
  fb.nq = desc->nq;
  for (int q = 0; q < desc->nq; q++) {
    F[q] = reinterpret_cast<sufb200::FrontierEntry*>(scratch + kAccBytes + 32ull * kmax * q);
    fb.q[q] = sufb200::FrontierLaunch{a.key[q], desc->q_bits[q], 8, acc, kmax, F[q], ctx->d_t0, ctx->d_status};
  }
  e = narrow_queries(&a.desc, 1, kmax) ? sufb200::set_full_range(acc, st)
                                       : sufb200::launch_range(ctx, a.xhat, n, acc, st);
  if (e == cudaSuccess) e = sufb200::launch_frontier(ctx, SUFB200_GROUP_ADD, fb, st);
  // the main pass, in chunks when a host sink streams results back (the
  // kernel's outputs do not depend on the element index)
  const size_t chunk = sink && sink->chunk ? sink->chunk : n;
  for (size_t i0 = 0; i0 < n && e == cudaSuccess; i0 += chunk) {
    const size_t i1 = n - i0 < chunk ? n : i0 + chunk;
    sufb200::TruncLaunch c = a;
    c.xhat = a.xhat + i0;
    c.n = i1 - i0;
    c.y = d_y + i0;
    c.bools = d_bools ? d_bools + 3 * i0 : nullptr;
    e = sufb200::launch_trunc_bundle_prefix(ctx, c, acc, kmax, F, st);
    if (e == cudaSuccess && sink) {
      if (int rc = enqueue_chunk_copy(*sink, st, d_y, d_bools, i0, i1)) {
        cudaFreeAsync(scratch, st);
        return rc;
      }
    }
  }
  cudaFreeAsync(scratch, st);
  if (e != cudaSuccess) return cuda_fail(e, "trunc bundle launch");
  return SUFB200_OK;
}

// Host keys of the given bundles into one pool buffer (one H2D copy); the
// caller frees *scratch after its launches.
int upload_bundle_keys(sufb200_ctx ctx, const sufb200_trunc_desc* const* desc, const uint8_t* const* const* keys,
                       const size_t* const* key_bytes, int nb, sufb200::TruncLaunch* const* a, cudaStream_t st,
                       uint8_t** scratch) {
  *scratch = nullptr;
  std::vector<uint8_t> blob;
  uint32_t off[2][4] = {};
  for (int b = 0; b < nb; b++)
    if (int rc = pack_bundle_keys(*desc[b], keys[b], key_bytes[b], blob, off[b])) return rc;
  if (blob.empty()) return SUFB200_OK;
  SUFB200_CHECK_CUDA(cudaMallocFromPoolAsync(reinterpret_cast<void**>(scratch), blob.size() + 256, ctx->pool, st),
                     "bundle key staging");
  SUFB200_CHECK_CUDA(cudaMemcpyAsync(*scratch, blob.data(), blob.size(), cudaMemcpyHostToDevice, st), "bundle keys H2D");
  for (int b = 0; b < nb; b++)
    for (int q = 0; q < desc[b]->nq; q++) a[b]->key[q] = *scratch + off[b][q];
  return SUFB200_OK;
}

int trunc_bundle_impl(sufb200_ctx ctx, const sufb200_trunc_desc* desc, const uint8_t* const* keys,
                      const size_t* key_bytes, const uint64_t* d_xhat, size_t n, uint64_t* d_y, uint64_t* d_bools,
                      void* stream, const ChunkSink* sink) {
  if (int rc = check_ctx(ctx, true)) return rc;
  if (int rc = check_bundle_desc(desc, keys, key_bytes)) return rc;
  if (n == 0) return SUFB200_OK;
  if (!d_xhat || !d_y || !aligned8(d_xhat) || !aligned8(d_y) || (d_bools && !aligned8(d_bools)))
    return fail(SUFB200_ERR_INVALID, "null or misaligned device pointer");
  cudaStream_t st = as_stream(stream);
  sufb200::TruncLaunch a{};
  a.desc = *desc;
  a.xhat = d_xhat;
  a.n = n;
  a.y = d_y;
  a.bools = d_bools;
  sufb200::TruncLaunch* pa[1] = {&a};
  uint8_t* scratch = nullptr;
  int rc = upload_bundle_keys(ctx, &desc, &keys, &key_bytes, 1, pa, st, &scratch);
  if (rc == SUFB200_OK) rc = single_core(ctx, a, st, sink);
  if (scratch) cudaFreeAsync(scratch, st);
  return rc;
}

// Both parties' bundles over one x^ with their keys on the device: batches
// below the shared-prefix size in one launch (a lane per party, element and
// query); larger ones on the shared-prefix path with one range pass (x^ is
// common), one frontier launch over both parties' query keys and one main
// pass over both parties' elements; query-free bundles party by party.
int trunc_pair_core(sufb200_ctx ctx, sufb200::TruncLaunch a0, sufb200::TruncLaunch a1, const uint64_t* d_xhat,
                    size_t n, uint64_t* d_y0, uint64_t* d_y1, cudaStream_t st) {
  for (sufb200::TruncLaunch* a : {&a0, &a1}) {
    a->xhat = d_xhat;
    a->n = n;
    a->bools = nullptr;
    a->t0 = ctx->d_t0;
    a->status = ctx->d_status;
  }
  a0.y = d_y0;
  a1.y = d_y1;
  if (n < prefix_min_n()) {
    cudaError_t e = sufb200::launch_trunc_bundle_pair(ctx, a0, a1, st);
    if (e != cudaSuccess) return cuda_fail(e, "pair bundle launch");
    return SUFB200_OK;
  }
  if (a0.desc.nq == 0 || a1.desc.nq == 0) {
    if (int rc = single_core(ctx, a0, st, nullptr)) return rc;
    return single_core(ctx, a1, st, nullptr);
  }
  const uint32_t kmax = sufb200::prefix_budget(n);
  const size_t nqt = static_cast<size_t>(a0.desc.nq + a1.desc.nq);
  uint8_t* scratch = nullptr;
  SUFB200_CHECK_CUDA(cudaMallocFromPoolAsync(reinterpret_cast<void**>(&scratch), kAccBytes + 32ull * kmax * nqt + 256,
                                             ctx->pool, st),
                     "pair bundle scratch allocation");
  auto* acc = reinterpret_cast<sufb200::RangeAcc*>(scratch);
  sufb200::FrontierEntry* F[8] = {nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr};
  sufb200::FrontierBatch fb{};
  fb.nq = static_cast<int>(nqt);
  int k = 0;
  for (int p = 0; p < 2; p++) {
    const sufb200::TruncLaunch& a = p ? a1 : a0;
    for (int q = 0; q < a.desc.nq; q++, k++) {
      F[4 * p + q] = reinterpret_cast<sufb200::FrontierEntry*>(scratch + kAccBytes + 32ull * kmax * k);
      fb.q[k] = sufb200::FrontierLaunch{a.key[q], a.desc.q_bits[q], 8, acc, kmax, F[4 * p + q], ctx->d_t0,
                                        ctx->d_status};
    }
  }
  const sufb200_trunc_desc both[2] = {a0.desc, a1.desc};
  cudaError_t e = narrow_queries(both, 2, kmax) ? sufb200::set_full_range(acc, st)
                                                : sufb200::launch_range(ctx, d_xhat, n, acc, st);
  if (e == cudaSuccess) e = sufb200::launch_frontier(ctx, SUFB200_GROUP_ADD, fb, st);
  if (e == cudaSuccess) e = sufb200::launch_trunc_bundle_prefix_pair(ctx, a0, a1, acc, kmax, F, st);
  cudaFreeAsync(scratch, st);
  if (e != cudaSuccess) return cuda_fail(e, "pair bundle launch");
  return SUFB200_OK;
}

}  // namespace

int sufb200_trunc_bundle_eval_pair(sufb200_ctx ctx, const sufb200_trunc_desc* desc0, const uint8_t* const* keys0,
                                   const size_t* key_bytes0, const sufb200_trunc_desc* desc1,
                                   const uint8_t* const* keys1, const size_t* key_bytes1, const uint64_t* d_xhat,
                                   size_t n, uint64_t* d_y0, uint64_t* d_y1, void* stream) {
  if (int rc = check_ctx(ctx, true)) return rc;
  if (int rc = check_bundle_desc(desc0, keys0, key_bytes0)) return rc;
  if (int rc = check_bundle_desc(desc1, keys1, key_bytes1)) return rc;
  if (desc0->party != 0 || desc1->party != 1) return fail(SUFB200_ERR_INVALID, "desc0 / desc1 must be parties 0 / 1");
  if (n == 0) return SUFB200_OK;
  if (!d_xhat || !d_y0 || !d_y1 || !aligned8(d_xhat) || !aligned8(d_y0) || !aligned8(d_y1))
    return fail(SUFB200_ERR_INVALID, "null or misaligned device pointer");
  cudaStream_t st = as_stream(stream);
  sufb200::TruncLaunch a0{}, a1{};
  a0.desc = *desc0;
  a1.desc = *desc1;
  const sufb200_trunc_desc* descs[2] = {desc0, desc1};
  const uint8_t* const* keys[2] = {keys0, keys1};
  const size_t* kbs[2] = {key_bytes0, key_bytes1};
  sufb200::TruncLaunch* pa[2] = {&a0, &a1};
  uint8_t* scratch = nullptr;
  int rc = upload_bundle_keys(ctx, descs, keys, kbs, 2, pa, st, &scratch);
  if (rc == SUFB200_OK) rc = trunc_pair_core(ctx, a0, a1, d_xhat, n, d_y0, d_y1, st);
  if (scratch) cudaFreeAsync(scratch, st);
  return rc;
}

namespace {

// Checks of a pair of bundles whose keys are device pointers; fills a0 / a1's
// descriptors and key pointers.
// One party's bundle with its keys on the device: desc and key sizes checked.
int dev_launch(sufb200_ctx ctx, const sufb200_trunc_desc* desc, const uint8_t* const* d_keys,
               const size_t* key_bytes, sufb200::TruncLaunch& a) {
  if (int rc = check_ctx(ctx, true)) return rc;
  if (int rc = check_bundle_desc(desc, d_keys, key_bytes)) return rc;
  a = sufb200::TruncLaunch{};
  a.desc = *desc;
  for (int q = 0; q < desc->nq; q++) {
    const int nb = desc->q_bits[q];
    if (nb < 1 || nb > 64) return fail(SUFB200_ERR_INVALID, "query in_bits out of range");
    if (!d_keys[q] || key_bytes[q] != sufb200::host::myl7_key_bytes(nb, 8))
      return fail(SUFB200_ERR_KEY, "query " + std::to_string(q) + ": key size does not match an 8-byte myl7 key");
    a.key[q] = d_keys[q];
  }
  return SUFB200_OK;
}

int dev_pair_launches(sufb200_ctx ctx, const sufb200_trunc_desc* desc0, const uint8_t* const* d_keys0,
                      const size_t* key_bytes0, const sufb200_trunc_desc* desc1, const uint8_t* const* d_keys1,
                      const size_t* key_bytes1, sufb200::TruncLaunch& a0, sufb200::TruncLaunch& a1) {
  if (int rc = dev_launch(ctx, desc0, d_keys0, key_bytes0, a0)) return rc;
  if (int rc = dev_launch(ctx, desc1, d_keys1, key_bytes1, a1)) return rc;
  if (desc0->party != 0 || desc1->party != 1) return fail(SUFB200_ERR_INVALID, "desc0 / desc1 must be parties 0 / 1");
  return SUFB200_OK;
}

// Layout of a pair's full-domain tables: the range record, then query q's
// 2^in_bits entries of 32 bytes, party 0's queries first.
// Tables of one party's bundle whose queries are all at most kTablesMaxBits
// wide: the range word, then each query's 2^bits frontier entries (32
// bytes each).  Returns the size (0 when the bundle does not qualify), the
// entries' offsets and the frontier budget (2^widest bits, at least 256),
// whatever the batch size.
constexpr int kTablesMaxBits = 16;

size_t tables_layout(const sufb200_trunc_desc* d, size_t off[4], uint32_t* kmax) {
  if (!d || d->nq <= 0 || d->nq > 4) return 0;
  int widest = 0;
  for (int q = 0; q < d->nq; q++) {
    if (d->q_bits[q] < 1 || d->q_bits[q] > kTablesMaxBits) return 0;
    widest = d->q_bits[q] > widest ? d->q_bits[q] : widest;
  }
  *kmax = (1u << widest) < 256u ? 256u : (1u << widest);
  size_t at = kAccBytes;
  for (int q = 0; q < d->nq; q++) {
    off[q] = at;
    at += 32ull << d->q_bits[q];
  }
  return at;
}

}  // namespace

int sufb200_trunc_bundle_eval_pair_dev(sufb200_ctx ctx, const sufb200_trunc_desc* desc0,
                                       const uint8_t* const* d_keys0, const size_t* key_bytes0,
                                       const sufb200_trunc_desc* desc1, const uint8_t* const* d_keys1,
                                       const size_t* key_bytes1, const uint64_t* d_xhat, size_t n, uint64_t* d_y0,
                                       uint64_t* d_y1, void* stream) {
  sufb200::TruncLaunch a0, a1;
  if (int rc = dev_pair_launches(ctx, desc0, d_keys0, key_bytes0, desc1, d_keys1, key_bytes1, a0, a1)) return rc;
  if (n == 0) return SUFB200_OK;
  if (!d_xhat || !d_y0 || !d_y1 || !aligned8(d_xhat) || !aligned8(d_y0) || !aligned8(d_y1))
    return fail(SUFB200_ERR_INVALID, "null or misaligned device pointer");
  return trunc_pair_core(ctx, a0, a1, d_xhat, n, d_y0, d_y1, as_stream(stream));
}

size_t sufb200_trunc_tables_bytes(const sufb200_trunc_desc* desc) {
  size_t off[4];
  uint32_t kmax = 0;
  return tables_layout(desc, off, &kmax);
}

int sufb200_trunc_tables_many_dev(sufb200_ctx ctx, int count, const sufb200_trunc_desc* descs,
                                  const uint8_t* const* d_keys, const size_t* key_bytes, void* const* d_tables,
                                  const size_t* tables_bytes, void* stream) {
  if (int rc = check_ctx(ctx, true)) return rc;
  if (count < 0 || (count > 0 && (!descs || !d_keys || !key_bytes || !d_tables || !tables_bytes)))
    return fail(SUFB200_ERR_INVALID, "bad tables list");
  std::vector<sufb200::FrontierLaunch> work;
  for (int i = 0; i < count; i++) {
    if (!d_tables[i]) continue;
    sufb200::TruncLaunch a;
    if (int rc = dev_launch(ctx, &descs[i], d_keys + 4 * i, key_bytes + 4 * i, a)) return rc;
    size_t off[4] = {};
    uint32_t kmax = 0;
    const size_t need = tables_layout(&descs[i], off, &kmax);
    if (need == 0)
      return fail(SUFB200_ERR_UNSUPPORTED,
                  "bundle " + std::to_string(i) + ": no query, or a query wider than the tables' 16 bits");
    if (tables_bytes[i] < need || (reinterpret_cast<uintptr_t>(d_tables[i]) & 255u))
      return fail(SUFB200_ERR_INVALID, "bundle " + std::to_string(i) +
                                           ": tables buffer unaligned (256 bytes) or smaller than sufb200_trunc_tables_bytes");
    uint8_t* base = static_cast<uint8_t*>(d_tables[i]);
    auto* acc = reinterpret_cast<sufb200::RangeAcc*>(base);
    for (int q = 0; q < a.desc.nq; q++)
      work.push_back(sufb200::FrontierLaunch{a.key[q], a.desc.q_bits[q], 8, acc, kmax,
                                             reinterpret_cast<sufb200::FrontierEntry*>(base + off[q]), ctx->d_t0,
                                             ctx->d_status, acc});
  }
  cudaStream_t st = as_stream(stream);
  // Table fills run beside the work that produces x^: a quarter of the SMs
  // each (the frontier kernel holds a whole SM's registers and shared
  // memory per block, so a full-width fill would stall that work).
  const int max_grid = (ctx->sm_count + 3) / 4;
  for (size_t at = 0; at < work.size(); at += sufb200::kFrontierMaxKeys) {
    sufb200::FrontierBatch fb{};
    fb.nq = static_cast<int>(std::min<size_t>(sufb200::kFrontierMaxKeys, work.size() - at));
    for (int q = 0; q < fb.nq; q++) fb.q[q] = work[at + q];
    const cudaError_t e = sufb200::launch_frontier(ctx, SUFB200_GROUP_ADD, fb, st, max_grid);
    if (e != cudaSuccess) return cuda_fail(e, "tables launch");
  }
  return SUFB200_OK;
}

int sufb200_trunc_tables_dev(sufb200_ctx ctx, const sufb200_trunc_desc* desc, const uint8_t* const* d_keys,
                             const size_t* key_bytes, void* d_tables, size_t tables_bytes, void* stream) {
  if (!desc || !d_keys || !key_bytes) return fail(SUFB200_ERR_INVALID, "null descriptor or key list");
  if (!d_tables) return fail(SUFB200_ERR_INVALID, "null tables buffer");
  const uint8_t* keys[4] = {nullptr, nullptr, nullptr, nullptr};
  size_t sizes[4] = {0, 0, 0, 0};
  for (int q = 0; q < desc->nq && q < 4; q++) {
    keys[q] = d_keys[q];
    sizes[q] = key_bytes[q];
  }
  return sufb200_trunc_tables_many_dev(ctx, 1, desc, keys, sizes, &d_tables, &tables_bytes, stream);
}

int sufb200_trunc_bundle_eval_pair_tables_dev(sufb200_ctx ctx, const sufb200_trunc_desc* desc0,
                                              const uint8_t* const* d_keys0, const size_t* key_bytes0,
                                              const void* d_tables0, const sufb200_trunc_desc* desc1,
                                              const uint8_t* const* d_keys1, const size_t* key_bytes1,
                                              const void* d_tables1, const uint64_t* d_xhat, size_t n, uint64_t* d_y0,
                                              uint64_t* d_y1, void* stream) {
  sufb200::TruncLaunch a0, a1;
  if (int rc = dev_pair_launches(ctx, desc0, d_keys0, key_bytes0, desc1, d_keys1, key_bytes1, a0, a1)) return rc;
  size_t off[2][4] = {};
  uint32_t kmax[2] = {0, 0};
  if (tables_layout(desc0, off[0], &kmax[0]) == 0 || tables_layout(desc1, off[1], &kmax[1]) == 0)
    return fail(SUFB200_ERR_UNSUPPORTED, "bundle has a query wider than the tables' 16 bits");
  if (n == 0) return SUFB200_OK;
  if (!d_tables0 || !d_tables1 || !d_xhat || !d_y0 || !d_y1 || !aligned8(d_xhat) || !aligned8(d_y0) ||
      !aligned8(d_y1))
    return fail(SUFB200_ERR_INVALID, "null or misaligned device pointer");
  const uint8_t* base[2] = {static_cast<const uint8_t*>(d_tables0), static_cast<const uint8_t*>(d_tables1)};
  sufb200::FrontierEntry* F[8] = {nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr};
  for (int p = 0; p < 2; p++)
    for (int q = 0; q < (p ? a1 : a0).desc.nq; q++)
      F[4 * p + q] = reinterpret_cast<sufb200::FrontierEntry*>(const_cast<uint8_t*>(base[p]) + off[p][q]);
  for (sufb200::TruncLaunch* a : {&a0, &a1}) {
    a->xhat = d_xhat;
    a->n = n;
    a->bools = nullptr;
    a->t0 = ctx->d_t0;
    a->status = ctx->d_status;
  }
  a0.y = d_y0;
  a1.y = d_y1;
  // Both tables hold the full-domain range word; every query's table covers
  // its whole domain under either budget, so the larger one serves both.
  const cudaError_t e = sufb200::launch_trunc_bundle_lookup_pair(
      ctx, a0, a1, reinterpret_cast<const sufb200::RangeAcc*>(base[0]), kmax[0] > kmax[1] ? kmax[0] : kmax[1], F,
      as_stream(stream));
  return e == cudaSuccess ? SUFB200_OK : cuda_fail(e, "pair bundle launch");
}

int sufb200_trunc_bundle_eval_jobs(sufb200_ctx ctx, const sufb200_trunc_desc* desc, const uint8_t* const* keys,
                                   const size_t* key_bytes, const uint64_t* const* d_xhat, const size_t* n,
                                   uint64_t* const* d_y, int njobs, void* stream) {
  if (int rc = check_ctx(ctx, true)) return rc;
  if (int rc = check_bundle_desc(desc, keys, key_bytes)) return rc;
  if (njobs < 0 || (njobs > 0 && (!d_xhat || !n || !d_y))) return fail(SUFB200_ERR_INVALID, "bad job list");
  size_t total = 0;
  for (int j = 0; j < njobs; j++) {
    if (n[j] && (!d_xhat[j] || !d_y[j] || !aligned8(d_xhat[j]) || !aligned8(d_y[j])))
      return fail(SUFB200_ERR_INVALID, "job " + std::to_string(j) + ": null or misaligned device pointer");
    total += n[j];
  }
  if (total == 0) return SUFB200_OK;
  if (njobs == 1) return trunc_bundle_impl(ctx, desc, keys, key_bytes, d_xhat[0], n[0], d_y[0], nullptr, stream, nullptr);
  cudaStream_t st = as_stream(stream);
  uint64_t* batch = nullptr;
  SUFB200_CHECK_CUDA(cudaMallocFromPoolAsync(reinterpret_cast<void**>(&batch), 2 * total * 8, ctx->pool, st),
                     "job bucket allocation");
  auto copy_all = [&](bool to_batch, uint64_t* buf) {
    size_t base = 0;
    for (int j0 = 0; j0 < njobs; j0 += sufb200::kJobsPerLaunch) {
      sufb200::JobTable t{};
      t.njobs = std::min(sufb200::kJobsPerLaunch, njobs - j0);
      t.base = base;
      t.off[0] = 0;
      for (int k = 0; k < t.njobs; k++) {
        t.src[k] = d_xhat[j0 + k];
        t.dst[k] = d_y[j0 + k];
        t.off[k + 1] = t.off[k] + n[j0 + k];
      }
      const cudaError_t e = sufb200::launch_jobs_copy(ctx, t, buf, to_batch, st);
      if (e != cudaSuccess) return e;
      base += t.off[t.njobs];
    }
    return cudaSuccess;
  };
  cudaError_t e = copy_all(true, batch);
  int rc = SUFB200_OK;
  if (e == cudaSuccess)
    rc = trunc_bundle_impl(ctx, desc, keys, key_bytes, batch, total, batch + total, nullptr, stream, nullptr);
  if (e == cudaSuccess && rc == SUFB200_OK) e = copy_all(false, batch + total);
  cudaFreeAsync(batch, st);
  if (e != cudaSuccess) return cuda_fail(e, "job bucket gather / scatter");
  return rc;
}

int sufb200_trunc_bundle_eval_host(sufb200_ctx ctx, const sufb200_trunc_desc* desc, const uint8_t* const* keys,
                                   const size_t* key_bytes, const uint64_t* xhat, size_t n, uint64_t* y,
                                   uint64_t* bools) {
  if (int rc = check_ctx(ctx, true)) return rc;
  if (n == 0) return SUFB200_OK;
  if (!xhat || !y) return fail(SUFB200_ERR_INVALID, "null host buffer");
  HostIo* io = io_of(ctx, true);
  std::lock_guard<std::mutex> lk(io->mu);
  if (!io->stream) SUFB200_CHECK_CUDA(cudaStreamCreateWithFlags(&io->stream, cudaStreamNonBlocking), "stream");
  const size_t out_bytes = n * 8 * (bools ? 4 : 1);
  if (int rc = grow(reinterpret_cast<void**>(&io->d_xs), &io->xs_cap, n * 8)) return rc;
  if (int rc = grow(reinterpret_cast<void**>(&io->d_out), &io->out_cap, out_bytes)) return rc;
  if (!io->copy) SUFB200_CHECK_CUDA(cudaStreamCreateWithFlags(&io->copy, cudaStreamNonBlocking), "copy stream");
  if (!io->chunk_done)
    SUFB200_CHECK_CUDA(cudaEventCreateWithFlags(&io->chunk_done, cudaEventDisableTiming), "chunk event");
  uint64_t* d_y = reinterpret_cast<uint64_t*>(io->d_out);
  uint64_t* d_b = bools ? d_y + n : nullptr;
  SUFB200_CHECK_CUDA(cudaMemcpyAsync(io->d_xs, xhat, n * 8, cudaMemcpyHostToDevice, io->stream), "H2D xhat");
  // Eight main-kernel launches over large batches, each chunk's results
  // copied back while the next one is evaluated.
  const ChunkSink sink{io->copy, io->chunk_done, y, bools, n >= (1u << 20) ? (n + 7) / 8 : n};
  const int rc = trunc_bundle_impl(ctx, desc, keys, key_bytes, io->d_xs, n, d_y, d_b, io->stream, &sink);
  const cudaError_t ce = cudaStreamSynchronize(io->copy);
  if (rc) return rc;
  SUFB200_CHECK_CUDA(ce, "D2H chunk copies");
  return sufb200_ctx_sync(ctx, io->stream);
}

// ---- reference GPU-backend formats -----------------------------------------

size_t sufb200_thr_dcf_build(int in_bits, uint64_t alpha, const uint8_t* payload, int payload_len, uint8_t* out) {
  if (in_bits < 1 || in_bits > 64 || payload_len < 0 || payload_len > 0xFFFF) return 0;
  return sufb200::host::thr_dcf_build(in_bits, alpha, payload, payload_len, out);
}

int sufb200_thr_dcf_eval(sufb200_ctx ctx, int in_bits, const uint8_t* d_keys, size_t key_bytes, int broadcast,
                         const uint64_t* d_xs, size_t n, int out_bytes, void* d_out, void* stream) {
  if (int rc = check_ctx(ctx, false)) return rc;
  if (n == 0) return SUFB200_OK;
  if (in_bits < 1 || in_bits > 64) return fail(SUFB200_ERR_INVALID, "in_bits out of range");
  if (out_bytes < 0 || key_bytes != 12 + static_cast<size_t>(out_bytes))
    return fail(SUFB200_ERR_KEY, "key_bytes must be 12 + out_bytes");
  if (!d_keys || !d_xs || (!d_out && out_bytes > 0)) return fail(SUFB200_ERR_INVALID, "null pointer");
  if (!aligned8(d_xs) || (out_bytes == 8 && !aligned8(d_out))) return fail(SUFB200_ERR_INVALID, "misaligned pointer");
  sufb200::RefFmtLaunch a{d_keys, key_bytes, broadcast ? 1 : 0, d_xs, n, 0, d_out, in_bits, 0, out_bytes,
                          ctx->d_t0, ctx->d_status};
  SUFB200_CHECK_CUDA(sufb200::launch_thr_dcf(ctx, a, as_stream(stream)), "threshold DCF launch");
  return SUFB200_OK;
}

size_t sufb200_packed_lt_build(int party, uint64_t nonce, int in_bits, const uint64_t* thresholds, int num_thr,
                               const uint8_t* seed, uint8_t* out) {
  if (in_bits < 1 || in_bits > 64 || num_thr < 1 || num_thr > 0xFFFF || party < 0 || party > 1) return 0;
  if (out && (!thresholds || !seed)) return 0;
  return sufb200::host::packed_lt_build(party, nonce, in_bits, thresholds, num_thr, seed, out);
}

int sufb200_packed_lt_eval(sufb200_ctx ctx, const uint8_t* d_keys, size_t key_bytes, int broadcast,
                           const uint64_t* d_xs, size_t n, int in_bits, int out_words, uint64_t idx_base,
                           uint64_t* d_out, void* stream) {
  if (int rc = check_ctx(ctx, false)) return rc;
  if (n == 0) return SUFB200_OK;
  if (in_bits < 1 || in_bits > 64 || out_words < 1) return fail(SUFB200_ERR_INVALID, "in_bits / out_words");
  if (key_bytes < 208 + 8 || key_bytes % 8) return fail(SUFB200_ERR_KEY, "packed key_bytes too small or not 8k");
  if (!d_keys || !d_xs || !d_out || !aligned8(d_keys) || !aligned8(d_xs) || !aligned8(d_out))
    return fail(SUFB200_ERR_INVALID, "null or misaligned pointer");
  sufb200::RefFmtLaunch a{d_keys, key_bytes, broadcast ? 1 : 0, d_xs, n, idx_base, d_out, in_bits, out_words, 0,
                          ctx->d_t0, ctx->d_status};
  SUFB200_CHECK_CUDA(sufb200::launch_packed_lt(ctx, a, as_stream(stream)), "packed compare launch");
  return SUFB200_OK;
}

size_t sufb200_interval_lut_build(int party, uint64_t nonce, int in_bits, int out_words, const uint64_t* cuts,
                                  int intervals, const uint64_t* payload, const uint8_t* seed, uint8_t* out) {
  if (in_bits < 1 || in_bits > 64 || out_words < 1 || out_words > 0xFFFF || intervals < 1 || party < 0 || party > 1)
    return 0;
  if (out && (!cuts || !payload || !seed)) return 0;
  return sufb200::host::interval_lut_build(party, nonce, in_bits, out_words, cuts, intervals, payload, seed, out);
}

int sufb200_interval_lut_eval(sufb200_ctx ctx, const uint8_t* d_keys, size_t key_bytes, int broadcast,
                              const uint64_t* d_xs, size_t n, int out_words, uint64_t idx_base, uint64_t* d_out,
                              void* stream) {
  if (int rc = check_ctx(ctx, false)) return rc;
  if (n == 0) return SUFB200_OK;
  if (out_words < 1) return fail(SUFB200_ERR_INVALID, "out_words must be >= 1");
  if (key_bytes < 216 + 24 || key_bytes % 8) return fail(SUFB200_ERR_KEY, "interval key_bytes too small or not 8k");
  if (!d_keys || !d_xs || !d_out || !aligned8(d_keys) || !aligned8(d_xs) || !aligned8(d_out))
    return fail(SUFB200_ERR_INVALID, "null or misaligned pointer");
  sufb200::RefFmtLaunch a{d_keys, key_bytes, broadcast ? 1 : 0, d_xs, n, idx_base, d_out, 0, out_words, 0,
                          ctx->d_t0, ctx->d_status};
  SUFB200_CHECK_CUDA(sufb200::launch_interval_lut(ctx, a, as_stream(stream)), "interval LUT launch");
  return SUFB200_OK;
}

int sufb200_myl7_gen_batch_device(sufb200_ctx ctx, int group, int in_bits, const uint64_t* d_alphas, size_t n,
                                  const uint8_t* payload, int payload_len, const uint8_t* d_seeds0,
                                  const uint8_t* d_seeds1, uint8_t* d_keys0, uint8_t* d_keys1, void* stream) {
  if (int rc = check_ctx(ctx, true)) return rc;
  if (group != SUFB200_GROUP_ADD && group != SUFB200_GROUP_XOR) return fail(SUFB200_ERR_INVALID, "bad group");
  if (in_bits < 8 || in_bits > 64 || in_bits % 8)
    return fail(SUFB200_ERR_UNSUPPORTED, "device keygen needs in_bits in 8..64, a multiple of 8");
  if (payload_len < 1 || payload_len > 16 || !payload)
    return fail(SUFB200_ERR_UNSUPPORTED, "device keygen takes a payload of 1..16 bytes (one chunk)");
  if (n == 0) return SUFB200_OK;
  auto al = [](const void* p, uintptr_t a) { return p && (reinterpret_cast<uintptr_t>(p) % a) == 0; };
  if (!al(d_alphas, 8) || !al(d_seeds0, 16) || !al(d_seeds1, 16) || !al(d_keys0, 8) || !al(d_keys1, 8))
    return fail(SUFB200_ERR_INVALID, "null or misaligned device pointer (seeds 16-byte, keys 8-byte aligned)");
  uint8_t beta[16] = {0};
  std::memcpy(beta, payload, static_cast<size_t>(payload_len));
  beta[15] &= 0x7F;
  sufb200::GenLaunch g{};
  g.alphas = d_alphas;
  g.seeds0 = d_seeds0;
  g.seeds1 = d_seeds1;
  g.keys0 = d_keys0;
  g.keys1 = d_keys1;
  g.n = n;
  g.key_bytes = sufb200::host::myl7_key_bytes(in_bits, payload_len);
  g.in_bits = in_bits;
  g.payload_len = payload_len;
  std::memcpy(&g.beta_lo, beta, 8);
  std::memcpy(&g.beta_hi, beta + 8, 8);
  g.t0 = ctx->d_t0;
  g.status = ctx->d_status;
  SUFB200_CHECK_CUDA(sufb200::launch_myl7_gen(ctx, group, g, as_stream(stream)), "myl7 keygen launch");
  return SUFB200_OK;
}

// Checks one party's coefficient-gate key against r / degree and fills the
// launch parameters (the key rides in them when it fits, else it is staged
// in a pool buffer returned through *scratch, freed by the caller after the
// launch).
static int coeff_prepare(sufb200_ctx ctx, const uint8_t* key, size_t key_bytes, int r, int degree,
                         const uint64_t* r_out, int ring_bits, sufb200::CoeffLutParams& p, uint8_t** scratch,
                         cudaStream_t st) {
  *scratch = nullptr;
  if (r < 1 || r > sufb200::kCoeffMaxOut || degree < 0 || degree > 15 || ring_bits < 1 || ring_bits > 64)
    return fail(SUFB200_ERR_INVALID, "need 1 <= r <= 8, 0 <= degree <= 15, 1 <= ring_bits <= 64");
  if (!key || key_bytes < 216 + 24) return fail(SUFB200_ERR_KEY, "interval key missing or too small");
  uint64_t hdr;
  std::memcpy(&hdr, key, 8);
  const uint64_t ow = (hdr >> 16) & 0xFFFF, ivs = hdr >> 32, in_bits = hdr & 0xFFFF;
  if (in_bits < 1 || in_bits > 64 || ivs < 1 || ow != static_cast<uint64_t>(r) * static_cast<uint64_t>(degree + 1))
    return fail(SUFB200_ERR_KEY, "interval key header does not match r * (degree + 1) output words");
  if (key_bytes < 216 + 8 * (ivs + 1 + ivs * ow)) return fail(SUFB200_ERR_KEY, "interval key shorter than its table");
  p.r = r;
  p.degree = degree;
  p.ring_mask = ring_bits >= 64 ? ~0ull : ((1ull << ring_bits) - 1ull);
  for (int j = 0; j < sufb200::kCoeffMaxOut; j++) p.r_out[j] = (r_out && j < r) ? r_out[j] : 0ull;
  p.key_in_params = key_bytes <= sufb200::kCoeffParamKeyBytes ? 1 : 0;
  if (p.key_in_params) {
    std::memcpy(p.key, key, key_bytes);
    return SUFB200_OK;
  }
  SUFB200_CHECK_CUDA(cudaMallocFromPoolAsync(reinterpret_cast<void**>(scratch), (key_bytes + 255) & ~size_t{255},
                                             ctx->pool, st),
                     "coefficient key staging");
  SUFB200_CHECK_CUDA(cudaMemcpyAsync(*scratch, key, key_bytes, cudaMemcpyHostToDevice, st), "coefficient key H2D");
  return SUFB200_OK;
}

int sufb200_coeff_lut_eval(sufb200_ctx ctx, const uint8_t* key, size_t key_bytes, const uint64_t* d_xhat, size_t n,
                           int r, int degree, const uint64_t* r_out, int ring_bits, uint64_t idx_base,
                           uint64_t* d_out, void* stream) {
  if (int rc = check_ctx(ctx, false)) return rc;
  cudaStream_t st = as_stream(stream);
  static thread_local sufb200::CoeffLutParams p;  // 4 KB: not on the stack
  uint8_t* scratch = nullptr;
  if (n == 0) {
    if (int rc = coeff_prepare(ctx, key, key_bytes, r, degree, r_out, ring_bits, p, &scratch, nullptr)) return rc;
    return SUFB200_OK;
  }
  if (!d_xhat || !d_out || !aligned8(d_xhat) || !aligned8(d_out))
    return fail(SUFB200_ERR_INVALID, "null or misaligned device pointer");
  if (int rc = coeff_prepare(ctx, key, key_bytes, r, degree, r_out, ring_bits, p, &scratch, st)) {
    if (scratch) cudaFreeAsync(scratch, st);
    return rc;
  }
  sufb200::RefFmtLaunch a{scratch, key_bytes, 1, d_xhat, n, idx_base, d_out, 0, r * (degree + 1), 0, ctx->d_t0,
                          ctx->d_status};
  cudaError_t e = sufb200::launch_coeff_lut(ctx, a, p, st);
  if (scratch) cudaFreeAsync(scratch, st);
  if (e != cudaSuccess) return cuda_fail(e, "coefficient LUT launch");
  return SUFB200_OK;
}

int sufb200_coeff_lut_eval_pair(sufb200_ctx ctx, const uint8_t* key0, size_t key_bytes0, const uint8_t* key1,
                                size_t key_bytes1, const uint64_t* d_xhat, size_t n, int r, int degree,
                                const uint64_t* r_out0, const uint64_t* r_out1, int ring_bits, uint64_t idx_base,
                                uint64_t* d_out0, uint64_t* d_out1, void* stream) {
  if (int rc = check_ctx(ctx, false)) return rc;
  cudaStream_t st = as_stream(stream);
  static thread_local sufb200::CoeffLutParams p[2];
  uint8_t* scratch[2] = {nullptr, nullptr};
  const uint8_t* keys[2] = {key0, key1};
  const size_t kb[2] = {key_bytes0, key_bytes1};
  const uint64_t* ro[2] = {r_out0, r_out1};
  if (n != 0 && (!d_xhat || !d_out0 || !d_out1 || !aligned8(d_xhat) || !aligned8(d_out0) || !aligned8(d_out1)))
    return fail(SUFB200_ERR_INVALID, "null or misaligned device pointer");
  int rc = SUFB200_OK;
  for (int q = 0; q < 2 && rc == SUFB200_OK; q++)
    rc = coeff_prepare(ctx, keys[q], kb[q], r, degree, ro[q], ring_bits, p[q], &scratch[q], n ? st : nullptr);
  cudaError_t e = cudaSuccess;
  if (rc == SUFB200_OK && n != 0) {
    sufb200::RefFmtLaunch a0{scratch[0], kb[0], 1, d_xhat, n, idx_base, d_out0, 0, r * (degree + 1), 0, ctx->d_t0,
                             ctx->d_status};
    sufb200::RefFmtLaunch a1{scratch[1], kb[1], 1, d_xhat, n, idx_base, d_out1, 0, r * (degree + 1), 0, ctx->d_t0,
                             ctx->d_status};
    e = sufb200::launch_coeff_lut_pair(ctx, a0, p[0], a1, p[1], st);
  }
  for (int q = 0; q < 2; q++)
    if (scratch[q]) cudaFreeAsync(scratch[q], st);
  if (rc != SUFB200_OK) return rc;
  if (e != cudaSuccess) return cuda_fail(e, "coefficient LUT pair launch");
  return SUFB200_OK;
}

// ---- ring matmuls on the tensor cores (ring_gemm_tc.cu) ---------------------
// K' (summed over the product's pieces) up to 8192 keeps every limb diagonal
// exact in its 32-bit accumulator.
constexpr int kRingMaxK = 8192;

int sufb200_ring_matmul(sufb200_ctx ctx, const uint64_t* d_x, const int64_t* d_w, const int64_t* d_bias,
                        uint64_t* d_y, size_t batch, int M, int K, int N, int w_transposed, void* stream) {
  if (int rc = check_ctx(ctx, false)) return rc;
  if (batch == 0 || M == 0 || N == 0) return SUFB200_OK;
  if (M < 0 || N < 0 || K < 1 || batch > 65535) return fail(SUFB200_ERR_INVALID, "bad shape");
  if (K > kRingMaxK) return fail(SUFB200_ERR_UNSUPPORTED, "K above 8192 (split the contraction)");
  if (!d_x || !d_w || !d_y || !aligned8(d_x) || !aligned8(d_w) || !aligned8(d_y) || (d_bias && !aligned8(d_bias)))
    return fail(SUFB200_ERR_INVALID, "null or misaligned device pointer");
  sufb200::RingGemmLaunch g{};
  g.piece[0] = sufb200::RingGemmPiece{d_x, reinterpret_cast<const uint64_t*>(d_w), nullptr,
                                      static_cast<size_t>(M) * K, 0, 0};
  g.npieces = 1;
  g.M = M;
  g.N = N;
  g.K = K;
  g.trans = w_transposed ? 1 : 0;
  g.bias = d_bias;
  g.out = d_y;
  g.os = static_cast<size_t>(M) * N;
  g.status = ctx->d_status;
  SUFB200_CHECK_CUDA(sufb200::launch_ring_gemm_tc(ctx, g, static_cast<int>(batch), as_stream(stream)), "ring matmul launch");
  return SUFB200_OK;
}

int sufb200_beaver_matmul2d_tc(sufb200_ctx ctx, int party, const uint64_t* d_D_open, const uint64_t* d_E_open,
                               const uint64_t* d_A, const uint64_t* d_B, const uint64_t* d_C, int batches, int M,
                               int K, int N, int w_transposed, int has_scale, int64_t mul_const, int mul_shift,
                               uint64_t* d_out, void* stream) {
  if (int rc = check_ctx(ctx, false)) return rc;
  if (batches <= 0 || M <= 0 || N <= 0) return SUFB200_OK;
  if (K < 1 || batches > 65535 || (party != 0 && party != 1)) return fail(SUFB200_ERR_INVALID, "bad shape or party");
  if (2 * K > kRingMaxK) return fail(SUFB200_ERR_UNSUPPORTED, "K above 4096 (split the contraction)");
  const void* ptrs[6] = {d_D_open, d_E_open, d_A, d_B, d_C, d_out};
  for (const void* p : ptrs)
    if (!p || !aligned8(p)) return fail(SUFB200_ERR_INVALID, "null or misaligned device pointer");
  const size_t mk = static_cast<size_t>(M) * K, kn = static_cast<size_t>(K) * N;
  sufb200::RingGemmLaunch g{};
  // [D | A] x [B (+ E for party 0) ; E]: one product of depth 2K
  g.piece[0] = sufb200::RingGemmPiece{d_D_open, d_B, party == 0 ? d_E_open : nullptr, mk, 0, kn};
  g.piece[1] = sufb200::RingGemmPiece{d_A, d_E_open, nullptr, 0, kn, 0};
  g.npieces = 2;
  g.M = M;
  g.N = N;
  g.K = K;
  g.trans = w_transposed ? 1 : 0;
  g.c = d_C;
  g.cs = 0;
  g.has_scale = has_scale;
  g.mul_const = mul_const;
  g.mul_shift = mul_shift;
  g.out = d_out;
  g.os = static_cast<size_t>(M) * N;
  g.status = ctx->d_status;
  SUFB200_CHECK_CUDA(sufb200::launch_ring_gemm_tc(ctx, g, batches, as_stream(stream)), "Beaver matmul launch");
  return SUFB200_OK;
}

int sufb200_seed_from_id(uint64_t id, uint64_t tweak, uint8_t* seed16) {
  if (!seed16) return fail(SUFB200_ERR_INVALID, "null seed");
  sufb200::host::seed_from_id(id, tweak, seed16);
  return SUFB200_OK;
}

// ---- primitives -------------------------------------------------------------

static int prim_rc(cudaError_t e, const char* what) { return e == cudaSuccess ? SUFB200_OK : cuda_fail(e, what); }

static int cur_sm() {
  int dev = 0, sm = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sm, cudaDevAttrMultiProcessorCount, dev);
  return sm;
}

int sufb200_beaver_mul(int party, const uint64_t* d_a, const uint64_t* d_b, const uint64_t* d_c,
                       const uint64_t* d_d_open, const uint64_t* d_e_open, uint64_t* d_out, size_t n, void* stream) {
  if (n == 0) return SUFB200_OK;
  if (!d_a || !d_b || !d_c || !d_d_open || !d_e_open || !d_out) return fail(SUFB200_ERR_INVALID, "null pointer");
  return prim_rc(sufb200::prim_beaver_mul(cur_sm(), party, d_a, d_b, d_c, d_d_open, d_e_open, d_out, n,
                                          as_stream(stream)),
                 "beaver_mul");
}

int sufb200_beaver_mul_aos(int party, const uint64_t* d_triples, const uint64_t* d_d_open, const uint64_t* d_e_open,
                           uint64_t* d_out, size_t n, void* stream) {
  if (n == 0) return SUFB200_OK;
  if (!d_triples || !d_d_open || !d_e_open || !d_out) return fail(SUFB200_ERR_INVALID, "null pointer");
  return prim_rc(sufb200::prim_beaver_mul_aos(cur_sm(), party, d_triples, d_d_open, d_e_open, d_out, n,
                                              as_stream(stream)),
                 "beaver_mul_aos");
}

int sufb200_horner_cubic(const uint64_t* d_x, const uint64_t* d_c0, const uint64_t* d_c1, const uint64_t* d_c2,
                         const uint64_t* d_c3, uint64_t* d_out, size_t n, void* stream) {
  if (n == 0) return SUFB200_OK;
  if (!d_x || !d_c0 || !d_c1 || !d_c2 || !d_c3 || !d_out) return fail(SUFB200_ERR_INVALID, "null pointer");
  return prim_rc(sufb200::prim_horner_cubic(cur_sm(), d_x, d_c0, d_c1, d_c2, d_c3, d_out, n, as_stream(stream)),
                 "horner_cubic");
}

int sufb200_trunc_postproc(int party, int kind_gapars, int frac_bits, uint64_t r_hi_share, uint64_t m_share,
                           const uint64_t* d_hatx, const uint64_t* d_arith, size_t arith_stride, int arith_idx,
                           const uint64_t* d_bools, size_t bool_stride, int carry_idx, int sign_idx, int wrap_idx,
                           uint64_t* d_out, size_t n, void* stream) {
  if (n == 0) return SUFB200_OK;
  if (!d_arith || !d_out || arith_idx < 0 || static_cast<size_t>(arith_idx) >= arith_stride)
    return fail(SUFB200_ERR_INVALID, "bad arith operand");
  return prim_rc(sufb200::prim_trunc_postproc(cur_sm(), party, kind_gapars, frac_bits, r_hi_share, m_share, d_hatx,
                                              d_arith, arith_stride, arith_idx, d_bools, bool_stride, carry_idx,
                                              sign_idx, wrap_idx, d_out, n, as_stream(stream)),
                 "trunc_postproc");
}

int sufb200_add_rout_aos(uint64_t* d_out, size_t elems, int out_words, const uint64_t* r_out, size_t r_out_words,
                         void* stream) {
  if (elems == 0) return SUFB200_OK;
  if (!d_out || !r_out || out_words < 1) return fail(SUFB200_ERR_INVALID, "bad argument");
  if (out_words > 8 || r_out_words > 8) return fail(SUFB200_ERR_UNSUPPORTED, "add_rout_aos supports <= 8 words");
  return prim_rc(sufb200::prim_add_rout_aos(cur_sm(), d_out, elems, out_words, r_out, r_out_words, as_stream(stream)),
                 "add_rout_aos");
}

int sufb200_row_sum(const uint64_t* d_mat, int rows, int cols, const int* d_valid_lens, uint64_t* d_out_rows,
                    void* stream) {
  if (rows <= 0) return SUFB200_OK;
  if (!d_mat || !d_out_rows || cols < 0) return fail(SUFB200_ERR_INVALID, "bad argument");
  return prim_rc(sufb200::prim_row_sum(cur_sm(), d_mat, rows, cols, d_valid_lens, d_out_rows, as_stream(stream)),
                 "row_sum");
}

int sufb200_row_sum_ragged(const uint64_t* d_vals, const int* d_row_offsets, int rows, uint64_t* d_out_rows,
                           void* stream) {
  if (rows <= 0) return SUFB200_OK;
  if (!d_vals || !d_row_offsets || !d_out_rows) return fail(SUFB200_ERR_INVALID, "bad argument");
  return prim_rc(sufb200::prim_row_sum_ragged(cur_sm(), d_vals, d_row_offsets, rows, d_out_rows, as_stream(stream)),
                 "row_sum_ragged");
}

int sufb200_row_variance(const uint64_t* d_mat, const uint64_t* d_mean, int rows, int cols, const int* d_valid_lens,
                         uint64_t* d_out_rows, void* stream) {
  if (rows <= 0) return SUFB200_OK;
  if (!d_mat || !d_mean || !d_out_rows || cols < 0) return fail(SUFB200_ERR_INVALID, "bad argument");
  return prim_rc(sufb200::prim_row_variance(cur_sm(), d_mat, d_mean, rows, cols, d_valid_lens, d_out_rows,
                                            as_stream(stream)),
                 "row_variance");
}

int sufb200_row_broadcast_mul(int party, const uint64_t* d_A, const uint64_t* d_B_rows, const uint64_t* d_C,
                              const uint64_t* d_d_open, const uint64_t* d_e_open_rows, int rows, int cols,
                              const int* d_valid_lens, uint64_t* d_out, void* stream) {
  if (rows <= 0 || cols <= 0) return SUFB200_OK;
  if (!d_A || !d_B_rows || !d_C || !d_d_open || !d_e_open_rows || !d_out) return fail(SUFB200_ERR_INVALID, "null");
  return prim_rc(sufb200::prim_row_broadcast_mul(cur_sm(), party, d_A, d_B_rows, d_C, d_d_open, d_e_open_rows, rows,
                                                 cols, d_valid_lens, d_out, as_stream(stream)),
                 "row_broadcast_mul");
}

int sufb200_pack_eff_bits(const uint64_t* d_in, int eff_bits, uint64_t* d_packed, size_t n, void* stream) {
  if (n == 0) return SUFB200_OK;
  if (!d_in || !d_packed || eff_bits < 1 || eff_bits > 64) return fail(SUFB200_ERR_INVALID, "bad argument");
  return prim_rc(sufb200::prim_pack_eff_bits(cur_sm(), d_in, eff_bits, d_packed, n, as_stream(stream)), "pack");
}

int sufb200_unpack_eff_bits(const uint64_t* d_packed, int eff_bits, uint64_t* d_out, size_t n, void* stream) {
  if (n == 0) return SUFB200_OK;
  if (!d_packed || !d_out || eff_bits < 1 || eff_bits > 64) return fail(SUFB200_ERR_INVALID, "bad argument");
  return prim_rc(sufb200::prim_unpack_eff_bits(cur_sm(), d_packed, eff_bits, d_out, n, as_stream(stream)), "unpack");
}

int sufb200_unpack_add_mod(const uint64_t* d_local, const uint64_t* d_packed_remote, int eff_bits, uint64_t* d_out,
                           size_t n, int ring_bits, void* stream) {
  if (n == 0) return SUFB200_OK;
  if (!d_local || !d_packed_remote || !d_out || eff_bits < 1 || eff_bits > 64 || ring_bits < 1 || ring_bits > 64)
    return fail(SUFB200_ERR_INVALID, "bad argument");
  return prim_rc(sufb200::prim_unpack_add_mod(cur_sm(), d_local, d_packed_remote, eff_bits, d_out, n, ring_bits,
                                              as_stream(stream)),
                 "unpack_add_mod");
}

int sufb200_unpack_add_to_signed(const uint64_t* d_local, const uint64_t* d_packed_remote, int eff_bits,
                                 uint64_t* d_out, size_t n, int ring_bits, void* stream) {
  if (n == 0) return SUFB200_OK;
  if (!d_local || !d_packed_remote || !d_out || eff_bits < 1 || eff_bits > 64 || ring_bits < 1 || ring_bits > 64)
    return fail(SUFB200_ERR_INVALID, "bad argument");
  return prim_rc(sufb200::prim_unpack_add_to_signed(cur_sm(), d_local, d_packed_remote, eff_bits, d_out, n, ring_bits,
                                                    as_stream(stream)),
                 "unpack_add_to_signed");
}

int sufb200_open_add_to_signed(const uint64_t* d_local, const uint64_t* d_remote, uint64_t* d_out, size_t n,
                               int ring_bits, void* stream) {
  if (n == 0) return SUFB200_OK;
  if (!d_local || !d_remote || !d_out || ring_bits < 1 || ring_bits > 64) return fail(SUFB200_ERR_INVALID, "bad argument");
  return prim_rc(sufb200::prim_open_add_to_signed(cur_sm(), d_local, d_remote, d_out, n, ring_bits, as_stream(stream)),
                 "open_add_to_signed");
}

int sufb200_row_mean(const uint64_t* d_mat, int rows, int cols, const int* d_valid_lens, uint64_t* d_out_rows,
                     void* stream) {
  if (rows <= 0) return SUFB200_OK;
  if (!d_mat || !d_out_rows || cols < 0) return fail(SUFB200_ERR_INVALID, "bad argument");
  return prim_rc(sufb200::prim_row_mean(cur_sm(), d_mat, rows, cols, d_valid_lens, d_out_rows, as_stream(stream)),
                 "row_mean");
}

int sufb200_trunc_shift(const uint64_t* d_in, uint64_t* d_out, int frac_bits, size_t n, void* stream) {
  if (n == 0) return SUFB200_OK;
  if (!d_in || !d_out) return fail(SUFB200_ERR_INVALID, "null pointer");
  return prim_rc(sufb200::prim_trunc_shift(cur_sm(), d_in, d_out, frac_bits, n, as_stream(stream)), "trunc_shift");
}

int sufb200_beaver_matmul2d(int party, const uint64_t* d_D_open, const uint64_t* d_E_open, const uint64_t* d_A,
                            const uint64_t* d_B, const uint64_t* d_C, int batches, int M, int K, int N,
                            int w_transposed, int has_scale, int64_t mul_const, int mul_shift, uint64_t* d_out,
                            void* stream) {
  if (batches <= 0 || M <= 0 || K <= 0 || N <= 0) return SUFB200_OK;
  if (batches > 65535) return fail(SUFB200_ERR_UNSUPPORTED, "more than 65535 batches");
  if (!d_D_open || !d_E_open || !d_A || !d_B || !d_C || !d_out) return fail(SUFB200_ERR_INVALID, "null pointer");
  return prim_rc(sufb200::prim_beaver_matmul(party, d_D_open, d_E_open, d_A, d_B, d_C, batches, M, K, N,
                                             w_transposed ? 1 : 0, has_scale, mul_const, mul_shift, d_out,
                                             as_stream(stream)),
                 "beaver_matmul2d");
}

int sufb200_host_mt19937_64(uint64_t seed, uint64_t* out, size_t n) {
  if (!out && n) return fail(SUFB200_ERR_INVALID, "null out");
  std::mt19937_64 rng(seed);
  for (size_t i = 0; i < n; i++) out[i] = rng();
  return SUFB200_OK;
}

}  // extern "C"
