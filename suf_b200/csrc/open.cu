// open.cu -- the paired-GPU open: each party's shares of a flush, packed to
// eff_bits-wide words, cross NVLink to the other party's GPU in one NCCL
// group call, and each side adds the peer's words to its own.
//
// Restates the packed path of OpenCollector::flush
// (src/runtime/open_collector.cpp:357-895): one bit-width for the whole flush
// (ring_bits when below 64 and at most SUF_OPEN_PACK_MAX_BITS, else raw
// 64-bit words), a dense little-endian bitstream (pack_eff_bits_kernel,
// cuda/pfss_kernels.cu:722-812), and opened = add_mod(local, remote) in
// Z_2^ring, optionally sign-extended (unpack_add_mod_kernel /
// unpack_add_to_signed_kernel, cuda/cuda_primitives.cu:87-112).  The
// reference moves the packed words device -> host -> channel -> host ->
// device; here they go GPU to GPU, and pack, exchange and add are enqueued
// on the caller's stream with no host synchronisation.
#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <condition_variable>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <mutex>
#include <string>
#include <thread>

#include "kernels.hpp"
#include "primitives.hpp"

namespace {

// NCCL is opened at the first open-communicator call, not linked: a process
// that already holds libnccl.so.2 (torch loads its own copy) keeps using that
// one, so only one NCCL lives in the process.  SUFB200_NCCL_LIB names a
// different library file.
struct Nccl {
  ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
  ncclResult_t (*CommInitRankConfig)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*) = nullptr;
  ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*) = nullptr;
  ncclResult_t (*CommFinalize)(ncclComm_t) = nullptr;
  ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
  ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
  ncclResult_t (*GroupStart)() = nullptr;
  ncclResult_t (*GroupEnd)() = nullptr;
  ncclResult_t (*Send)(const void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*Recv)(void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  const char* (*GetErrorString)(ncclResult_t) = nullptr;
  std::string error;
};

Nccl& nccl_state() {
  static Nccl n;
  return n;
}

const Nccl* nccl() {
  Nccl& n = nccl_state();
  static std::once_flag once;
  std::call_once(once, [&n] {
    const char* path = std::getenv("SUFB200_NCCL_LIB");
    void* h = dlopen(path && *path ? path : "libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) {
      const char* e = dlerror();
      n.error = std::string("cannot load NCCL: ") + (e ? e : "unknown error");
      return;
    }
    bool ok = true;
    auto get = [&](auto& fn, const char* name) {
      fn = reinterpret_cast<std::remove_reference_t<decltype(fn)>>(dlsym(h, name));
      ok = ok && fn != nullptr;
    };
    get(n.GetUniqueId, "ncclGetUniqueId");
    get(n.CommInitRankConfig, "ncclCommInitRankConfig");
    get(n.CommGetAsyncError, "ncclCommGetAsyncError");
    get(n.CommFinalize, "ncclCommFinalize");
    get(n.CommDestroy, "ncclCommDestroy");
    get(n.CommAbort, "ncclCommAbort");
    get(n.GroupStart, "ncclGroupStart");
    get(n.GroupEnd, "ncclGroupEnd");
    get(n.Send, "ncclSend");
    get(n.Recv, "ncclRecv");
    get(n.GetErrorString, "ncclGetErrorString");
    if (!ok) {
      n.GetUniqueId = nullptr;
      n.error = "the loaded NCCL lacks a required entry point (NCCL >= 2.14 needed)";
    }
  });
  return n.GetUniqueId ? &n : nullptr;
}

int nccl_unavailable() { return sufb200::record_error(SUFB200_ERR_COMM, nccl_state().error); }

}  // namespace

struct sufb200_open_comm_s {
  sufb200_ctx ctx = nullptr;
  ncclComm_t comm = nullptr;  // blocking communicator
  int nranks = 0;
  int rank = 0;
};

namespace {

int nccl_fail(ncclResult_t r, const char* what) {
  const Nccl* N = nccl();
  if (!N) return sufb200::record_error(SUFB200_ERR_COMM, what);
  return sufb200::record_error(SUFB200_ERR_COMM, std::string(what) + ": " + N->GetErrorString(r));
}

// Wait (bounded) until a non-blocking communicator has finished the last
// operation it started; ncclInProgress on timeout.
ncclResult_t settle(const Nccl* N, ncclComm_t comm, double timeout_s) {
  const auto t0 = std::chrono::steady_clock::now();
  ncclResult_t state = ncclInProgress;
  for (;;) {
    const ncclResult_t r = N->CommGetAsyncError(comm, &state);
    if (r != ncclSuccess) return r;
    if (state != ncclInProgress) return state;
    const double dt = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    if (dt > timeout_s) return ncclInProgress;
    // an enqueue usually settles within microseconds: spin first, then back off
    if (dt < 2e-3) std::this_thread::yield();
    else std::this_thread::sleep_for(std::chrono::microseconds(100));
  }
}

}  // namespace

extern "C" {

int sufb200_open_unique_id(uint8_t* id) {
  if (!id) return sufb200::record_error(SUFB200_ERR_INVALID, "null id buffer");
  const Nccl* N = nccl();
  if (!N) return nccl_unavailable();
  static_assert(sizeof(ncclUniqueId) == SUFB200_OPEN_ID_BYTES, "NCCL unique id size");
  ncclUniqueId u;
  const ncclResult_t r = N->GetUniqueId(&u);
  if (r != ncclSuccess) return nccl_fail(r, "ncclGetUniqueId");
  std::memcpy(id, &u, sizeof(u));
  return SUFB200_OK;
}

int sufb200_open_comm_create(sufb200_ctx ctx, const uint8_t* id, int nranks, int rank, double timeout_s,
                             sufb200_open_comm* out) {
  if (!ctx || !id || !out) return sufb200::record_error(SUFB200_ERR_INVALID, "null pointer");
  *out = nullptr;
  if (ctx->device < 0)
    return sufb200::record_error(SUFB200_ERR_INVALID, "dealer-only context: the open needs a GPU");
  if (nranks < 2 || rank < 0 || rank >= nranks)
    return sufb200::record_error(SUFB200_ERR_INVALID, "need 2 <= nranks and 0 <= rank < nranks");
  if (!(timeout_s > 0)) return sufb200::record_error(SUFB200_ERR_INVALID, "timeout must be positive");
  const Nccl* N = nccl();
  if (!N) return nccl_unavailable();
  ncclUniqueId u;
  std::memcpy(&u, id, sizeof(u));
  // A blocking communicator (on a non-blocking one NCCL hands every group
  // call to a helper thread: tens of microseconds per exchange), joined on a
  // helper thread so the caller can give up after timeout_s.  If the peers
  // never come, that thread stays in NCCL's bootstrap and aborts the
  // communicator should the join ever complete; nothing runs on the GPU.
  struct Join {
    std::mutex m;
    std::condition_variable cv;
    bool done = false, abandoned = false;
    ncclResult_t r = ncclInternalError;
    ncclComm_t comm = nullptr;
  };
  auto job = std::make_shared<Join>();
  const int dev = ctx->device;
  std::thread([job, N, nranks, u, rank, dev] {
    ncclComm_t c = nullptr;
    ncclResult_t r = cudaSetDevice(dev) == cudaSuccess ? ncclSuccess : ncclUnhandledCudaError;
    if (r == ncclSuccess) {
      ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
      cfg.blocking = 1;
      r = N->CommInitRankConfig(&c, nranks, u, rank, &cfg);
    }
    std::lock_guard<std::mutex> lk(job->m);
    job->r = r;
    job->comm = c;
    job->done = true;
    if (job->abandoned && c) N->CommAbort(c);
    job->cv.notify_all();
  }).detach();
  ncclComm_t comm = nullptr;
  {
    std::unique_lock<std::mutex> lk(job->m);
    const auto deadline =
        std::chrono::steady_clock::now() +
        std::chrono::duration_cast<std::chrono::steady_clock::duration>(std::chrono::duration<double>(timeout_s));
    if (!job->cv.wait_until(lk, deadline, [&] { return job->done; })) {
      job->abandoned = true;
      return sufb200::record_error(SUFB200_ERR_COMM, "ncclCommInitRankConfig: peers did not join in time");
    }
    if (job->r != ncclSuccess) {
      if (job->comm) N->CommAbort(job->comm);
      return nccl_fail(job->r, "ncclCommInitRankConfig");
    }
    comm = job->comm;
  }
  auto* c = new sufb200_open_comm_s();
  c->ctx = ctx;
  c->comm = comm;
  c->nranks = nranks;
  c->rank = rank;
  *out = c;
  return SUFB200_OK;
}

int sufb200_open_comm_destroy(sufb200_open_comm comm) {
  if (!comm) return SUFB200_OK;
  const Nccl* N = nccl();
  if (!N) {
    delete comm;
    return nccl_unavailable();
  }
  ncclResult_t r = ncclSuccess;
  if (comm->comm) {
    r = N->CommFinalize(comm->comm);
    if (r == ncclSuccess) r = N->CommDestroy(comm->comm);
    else N->CommAbort(comm->comm);
    comm->comm = nullptr;
  }
  delete comm;
  return r == ncclSuccess ? SUFB200_OK : nccl_fail(r, "closing the open communicator");
}

int sufb200_open_comm_abort(sufb200_open_comm comm) {
  if (!comm || !comm->comm) return SUFB200_OK;
  const Nccl* N = nccl();
  if (!N) return nccl_unavailable();
  const ncclResult_t r = N->CommAbort(comm->comm);
  comm->comm = nullptr;
  return r == ncclSuccess ? SUFB200_OK : nccl_fail(r, "ncclCommAbort");
}

int sufb200_open_exchange(sufb200_open_comm comm, int peer, const uint64_t* d_local, size_t n, int eff_bits,
                          int ring_bits, int signed_out, uint64_t* d_out, void* stream) {
  if (!comm || !comm->comm) return sufb200::record_error(SUFB200_ERR_INVALID, "no open communicator");
  const Nccl* N = nccl();
  if (!N) return nccl_unavailable();
  if (peer < 0 || peer >= comm->nranks || peer == comm->rank)
    return sufb200::record_error(SUFB200_ERR_INVALID, "peer must be another rank of the communicator");
  if (eff_bits < 1 || eff_bits > 64 || ring_bits < 1 || ring_bits > 64)
    return sufb200::record_error(SUFB200_ERR_INVALID, "eff_bits and ring_bits must be in 1..64");
  if (n == 0) return SUFB200_OK;
  if (!d_local || !d_out || (reinterpret_cast<uintptr_t>(d_local) & 7u) || (reinterpret_cast<uintptr_t>(d_out) & 7u))
    return sufb200::record_error(SUFB200_ERR_INVALID, "null or misaligned device pointer");
  const int dev = comm->ctx->device;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int sm = comm->ctx->sm_count;
  const size_t words = sufb200::packed_word_count(n, eff_bits);
  // send buffer (not needed for raw 64-bit words) + receive buffer, stream-ordered
  const bool raw = eff_bits == 64;
  uint64_t* scratch = nullptr;
  cudaError_t ce = cudaSetDevice(dev);
  if (ce == cudaSuccess)
    ce = cudaMallocFromPoolAsync(reinterpret_cast<void**>(&scratch), (raw ? 1 : 2) * words * 8,
                                 comm->ctx->pool, st);
  if (ce != cudaSuccess)
    return sufb200::record_error(SUFB200_ERR_CUDA, std::string("open scratch: ") + cudaGetErrorString(ce));
  uint64_t* recv = scratch;
  const uint64_t* send = d_local;
  if (!raw) {
    uint64_t* packed = scratch + words;
    ce = sufb200::prim_pack_eff_bits(sm, d_local, eff_bits, packed, n, st);
    send = packed;
  }
  int rc = SUFB200_OK;
  if (ce != cudaSuccess) {
    rc = sufb200::record_error(SUFB200_ERR_CUDA, std::string("open pack: ") + cudaGetErrorString(ce));
  } else {
    ncclResult_t r = N->GroupStart();
    if (r == ncclSuccess) r = N->Send(send, words, ncclUint64, peer, comm->comm, st);
    if (r == ncclSuccess) r = N->Recv(recv, words, ncclUint64, peer, comm->comm, st);
    const ncclResult_t re = N->GroupEnd();
    if (r == ncclSuccess) r = re;
    if (r == ncclInProgress) r = settle(N, comm->comm, 30.0);
    if (r != ncclSuccess) {
      rc = r == ncclInProgress ? sufb200::record_error(SUFB200_ERR_COMM, "open exchange: NCCL did not settle")
                               : nccl_fail(r, "open exchange");
    } else {
      ce = signed_out ? sufb200::prim_unpack_add_to_signed(sm, d_local, recv, eff_bits, d_out, n, ring_bits, st)
                      : sufb200::prim_unpack_add_mod(sm, d_local, recv, eff_bits, d_out, n, ring_bits, st);
      if (ce != cudaSuccess)
        rc = sufb200::record_error(SUFB200_ERR_CUDA, std::string("open add: ") + cudaGetErrorString(ce));
    }
  }
  cudaFreeAsync(scratch, st);
  return rc;
}

}  // extern "C"
