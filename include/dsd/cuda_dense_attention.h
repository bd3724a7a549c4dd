// The reference's dense GPU baseline (DenseCudaContext) is outside the scope
// of this build (the sparse path is).  The symbols exist so callers link;
// DenseAttentionCudaAvailable() returns false and the rest throw
// std::runtime_error.
#pragma once

#include <vector>

#include "dsd/config.h"
#include "dsd/paged_kv_cache.h"
#include "dsd/types.h"

namespace dsd {

bool DenseAttentionCudaAvailable();

class DenseCudaContext {
 public:
  DenseCudaContext(const PagedKvCache& cache, const ModelConfig& config);
  DenseBatchResult RunBatch(const std::vector<RequestState>& requests);
};

DenseBatchResult DenseAttentionCudaBatch(const PagedKvCache& cache,
                                         const std::vector<RequestState>& requests,
                                         const ModelConfig& config);

}  // namespace dsd
