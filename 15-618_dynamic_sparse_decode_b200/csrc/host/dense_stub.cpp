// The dense GPU baseline is not part of this build; see cuda_dense_attention.h.
#include <stdexcept>

#include "dsd/cuda_dense_attention.h"

namespace dsd {

namespace {
[[noreturn]] void Unavailable() {
  throw std::runtime_error("the dense GPU baseline (DenseCudaContext) is not part of this build");
}
}  // namespace

bool DenseAttentionCudaAvailable() { return false; }
DenseCudaContext::DenseCudaContext(const PagedKvCache&, const ModelConfig&) { Unavailable(); }
DenseBatchResult DenseCudaContext::RunBatch(const std::vector<RequestState>&) { Unavailable(); }
DenseBatchResult DenseAttentionCudaBatch(const PagedKvCache&, const std::vector<RequestState>&,
                                         const ModelConfig&) {
  Unavailable();
}

}  // namespace dsd
