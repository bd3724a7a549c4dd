// Dense GPU decode baseline over the sparse context with dense attention
// (dsd_set_attention_mode): no scoring, no top-k, every candidate attended.
#include <algorithm>
#include <stdexcept>

#include "capi_error.h"
#include "dsd/cuda_dense_attention.h"
#include "dsd/cuda_sparse_attention.h"
#include "dsd_b200.h"

namespace dsd {

bool DenseAttentionCudaAvailable() { return SparseAttentionCudaAvailable(); }

DenseCudaContext::DenseCudaContext(const PagedKvCache& cache, const ModelConfig& config) {
  // every page can be a candidate of one request per step
  const int cap = std::max(1, cache.CapacityPages());
  impl_.reset(new SparseCudaContext(cache, config, 1024, cap, cap));
  detail::ThrowIf(dsd_set_attention_mode(impl_->handle(), 1));
}

DenseCudaContext::~DenseCudaContext() = default;

DenseBatchResult DenseCudaContext::RunBatch(const std::vector<RequestState>& requests) {
  auto r = impl_->RunBatch(requests, SparseBatchOutputMode::kOutputsOnly);
  DenseBatchResult out;
  out.kernel_ms = r.aggregate_timings.attention_ms;
  out.runtime_overheads = r.runtime_overheads;
  for (auto& p : r.per_request) out.outputs.push_back(std::move(p.output));
  return out;
}

void DenseCudaContext::SyncPageFromCache(const PagedKvCache& cache, PageId page_id) {
  impl_->SyncPageFromCache(cache, page_id);
}
void DenseCudaContext::SyncPagesFromCache(const PagedKvCache& cache,
                                          const std::vector<PageId>& page_ids) {
  impl_->SyncPagesFromCache(cache, page_ids);
}
void DenseCudaContext::SyncAppendedToken(const PagedKvCache& cache,
                                         const AppendTokenResult& result) {
  impl_->SyncAppendedToken(cache, result);
}
void DenseCudaContext::SyncAppendedTokens(const PagedKvCache& cache,
                                          const std::vector<AppendTokenResult>& results) {
  impl_->SyncAppendedTokens(cache, results);
}
void DenseCudaContext::SyncFreedPages(const std::vector<PageId>& page_ids) {
  impl_->SyncFreedPages(page_ids);
}

DenseBatchResult DenseAttentionCudaBatch(const PagedKvCache& cache,
                                         const std::vector<RequestState>& requests,
                                         const ModelConfig& config) {
  DenseCudaContext ctx(cache, config);
  return ctx.RunBatch(requests);
}

}  // namespace dsd
