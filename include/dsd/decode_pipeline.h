// Decode facade (drop-in for include/dsd/decode_pipeline.h:14-54).
#pragma once

#include <vector>

#include "dsd/config.h"
#include "dsd/cuda_dense_attention.h"
#include "dsd/cuda_sparse_attention.h"
#include "dsd/paged_kv_cache.h"
#include "dsd/reference_kernels.h"
#include "dsd/types.h"

namespace dsd {

class DecodePipeline {
 public:
  explicit DecodePipeline(ModelConfig config) : config_(config) {}

  // sparse_cpu: score, top-k, gather, attend on the host, each stage timed.
  SparseDecodeResult RunNaiveSparseStep(const PagedKvCache& cache,
                                        const RequestState& request) const;
  AttentionResult RunDenseStep(const PagedKvCache& cache, const RequestState& request) const;
  AttentionResult RunDenseStepCuda(const PagedKvCache& cache, const RequestState& request) const;
  SparseDecodeResult RunNaiveSparseStepCuda(const PagedKvCache& cache,
                                            const RequestState& request) const;
  DenseBatchResult RunDenseBatchCuda(const PagedKvCache& cache,
                                     const std::vector<RequestState>& requests) const;
  DenseBatchResult RunDenseBatchCuda(DenseCudaContext& context,
                                     const std::vector<RequestState>& requests) const;
  // sparse_gpu with debug tensors (scores and selected ids) returned.
  SparseBatchCudaResult RunNaiveSparseBatchCuda(SparseCudaContext& context,
                                                const std::vector<RequestState>& requests) const;
  BatchDecodeResult RunNaiveSparseBatch(const PagedKvCache& cache,
                                        const std::vector<RequestState>& requests) const;

  const ModelConfig& config() const { return config_; }

 private:
  ModelConfig config_;
};

}  // namespace dsd
