// DecodePipeline facade (reference: src/decode_pipeline.cpp:13-107).
#include "dsd/decode_pipeline.h"

#include "dsd/profiler.h"

namespace dsd {

SparseDecodeResult DecodePipeline::RunNaiveSparseStep(const PagedKvCache& cache,
                                                      const RequestState& request) const {
  SparseDecodeResult r;
  r.request_id = request.request_id;
  GatheredPages g;
  {
    ScopedStageTimer total(&r.timings.total_ms);
    {
      ScopedStageTimer t(&r.timings.page_scoring_ms);
      r.scores = ScorePagesCpu(cache, request, config_);
    }
    {
      ScopedStageTimer t(&r.timings.topk_ms);
      r.selected_page_ids = SelectTopKPagesCpu(r.scores, config_.top_k_pages);
    }
    {
      ScopedStageTimer t(&r.timings.gather_ms);
      g = GatherPagesCpu(cache, r.selected_page_ids, config_);
    }
    {
      ScopedStageTimer t(&r.timings.attention_ms);
      r.output = SparseAttentionCpu(request.query, g, config_);
    }
  }
  return r;
}

AttentionResult DecodePipeline::RunDenseStep(const PagedKvCache& cache,
                                             const RequestState& request) const {
  return DenseAttentionCpu(cache, request, config_);
}

AttentionResult DecodePipeline::RunDenseStepCuda(const PagedKvCache& cache,
                                                 const RequestState& request) const {
  auto b = DenseAttentionCudaBatch(cache, {request}, config_);
  return b.outputs.empty() ? AttentionResult{} : b.outputs.front();
}

SparseDecodeResult DecodePipeline::RunNaiveSparseStepCuda(const PagedKvCache& cache,
                                                          const RequestState& request) const {
  return SparseDecodeCuda(cache, request, config_);
}

DenseBatchResult DecodePipeline::RunDenseBatchCuda(const PagedKvCache& cache,
                                                   const std::vector<RequestState>& requests) const {
  return DenseAttentionCudaBatch(cache, requests, config_);
}

DenseBatchResult DecodePipeline::RunDenseBatchCuda(DenseCudaContext& context,
                                                   const std::vector<RequestState>& requests) const {
  return context.RunBatch(requests);
}

SparseBatchCudaResult DecodePipeline::RunNaiveSparseBatchCuda(
    SparseCudaContext& context, const std::vector<RequestState>& requests) const {
  return context.RunBatch(requests, SparseBatchOutputMode::kDebugTensors);
}

BatchDecodeResult DecodePipeline::RunNaiveSparseBatch(const PagedKvCache& cache,
                                                      const std::vector<RequestState>& requests) const {
  BatchDecodeResult out;
  for (const auto& req : requests) {
    auto r = RunNaiveSparseStep(cache, req);
    out.aggregate_timings.page_scoring_ms += r.timings.page_scoring_ms;
    out.aggregate_timings.topk_ms += r.timings.topk_ms;
    out.aggregate_timings.gather_ms += r.timings.gather_ms;
    out.aggregate_timings.attention_ms += r.timings.attention_ms;
    out.aggregate_timings.total_ms += r.timings.total_ms;
    out.per_request.push_back(std::move(r));
  }
  return out;
}

}  // namespace dsd
