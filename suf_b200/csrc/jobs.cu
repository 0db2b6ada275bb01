// jobs.cu -- gather / scatter of several jobs' words into one contiguous
// device batch, for evaluating one broadcast-key bundle over a bucket of jobs
// in one pass (the bucket step of PfssSuperBatch::flush_eval,
// src/runtime/pfss_superbatch.cpp:251-975, whose device path concatenates
// the jobs' x^ with one device memcpy per job, :801-845).  The job table
// travels as a kernel parameter, kJobsPerLaunch jobs per launch.
#include "kernels.hpp"

namespace sufb200 {
namespace {

__device__ __forceinline__ int job_of(const JobTable& t, size_t i) {
  int lo = 0, hi = t.njobs;  // last job with off <= i
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (t.off[mid] <= i) lo = mid; else hi = mid;
  }
  return lo;
}

// gather: batch[base + i] = job j's word i - off[j]; scatter: the reverse.
__global__ void jobs_copy_kernel(const __grid_constant__ JobTable t, uint64_t* batch, int to_batch) {
  const size_t n = t.off[t.njobs];
  for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const int j = job_of(t, i);
    const size_t k = i - t.off[j];
    if (to_batch) batch[t.base + i] = t.src[j][k];
    else t.dst[j][k] = batch[t.base + i];
  }
}

}  // namespace

cudaError_t launch_jobs_copy(const sufb200_ctx_s* ctx, const JobTable& t, uint64_t* batch, bool to_batch,
                             cudaStream_t st) {
  const size_t n = t.off[t.njobs];
  if (n == 0) return cudaSuccess;
  const size_t want = (n + 255) / 256, cap = static_cast<size_t>(ctx->sm_count) * 8;
  jobs_copy_kernel<<<static_cast<unsigned>(want < cap ? want : cap), 256, 0, st>>>(t, batch, to_batch ? 1 : 0);
  return cudaGetLastError();
}

}  // namespace sufb200
