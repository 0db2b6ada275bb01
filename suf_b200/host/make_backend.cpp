// make_backend.cpp -- the factory the reference runtime calls for
// SUF_PFSS_BACKEND=gpu (declared in include/proto/backend_gpu.hpp:70-72 of the
// reference, defined there in cuda/pfss_backend_gpu.cu:1512).  Built into the
// reference in place of its cuda_pfss target, it returns the B200 engine.
#include <memory>

#include "sufb200_backend.hpp"

namespace proto {

std::unique_ptr<PfssBackendBatch> make_real_gpu_backend() { return std::make_unique<SufB200Backend>(); }

}  // namespace proto
