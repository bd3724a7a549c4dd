// Dense GPU decode baseline (drop-in for include/dsd/cuda_dense_attention.h
// of the reference): every request attends over ALL its candidate pages on
// the GPU.  Built on the same pool and split-K attention kernels as the
// sparse path, with scoring and top-k switched off.
#pragma once

#include <memory>
#include <vector>

#include "dsd/config.h"
#include "dsd/paged_kv_cache.h"
#include "dsd/types.h"

namespace dsd {

class SparseCudaContext;

bool DenseAttentionCudaAvailable();

class DenseCudaContext {
 public:
  DenseCudaContext(const PagedKvCache& cache, const ModelConfig& config);
  ~DenseCudaContext();
  DenseCudaContext(const DenseCudaContext&) = delete;
  DenseCudaContext& operator=(const DenseCudaContext&) = delete;

  DenseBatchResult RunBatch(const std::vector<RequestState>& requests);

  void SyncPageFromCache(const PagedKvCache& cache, PageId page_id);
  void SyncPagesFromCache(const PagedKvCache& cache, const std::vector<PageId>& page_ids);
  void SyncAppendedToken(const PagedKvCache& cache, const AppendTokenResult& result);
  void SyncAppendedTokens(const PagedKvCache& cache, const std::vector<AppendTokenResult>& results);
  void SyncFreedPages(const std::vector<PageId>& page_ids);

 private:
  std::unique_ptr<SparseCudaContext> impl_;
};

DenseBatchResult DenseAttentionCudaBatch(const PagedKvCache& cache,
                                         const std::vector<RequestState>& requests,
                                         const ModelConfig& config);

}  // namespace dsd
