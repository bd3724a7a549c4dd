// SparseCudaContext over the C ABI (reference: src/cuda/sparse_batched_attention.cu:444-966).
// RunBatch packs the step's queries and candidate CSR into one upload and
// calls dsd_decode_batch; RunStep calls dsd_decode_step, whose candidates are
// the device request page tables (no host packing of candidate ids).
#include "dsd/cuda_sparse_attention.h"

#include <algorithm>
#include <chrono>
#include <cmath>
#include <stdexcept>

#include "capi_error.h"
#include "worker_pool.h"
#include "dsd_b200.h"
#include "dsd/profiler.h"

namespace dsd {

using detail::ThrowIf;

bool SparseAttentionCudaAvailable() { return dsd_available() != 0; }

SparseCudaContext::SparseCudaContext(const PagedKvCache& cache, const ModelConfig& config,
                                     int max_batch_size, int max_total_candidates,
                                     int max_total_selected_pages, int max_requests,
                                     int max_pages_per_request, int device, int kv_format)
    : cache_(&cache),
      config_(config),
      elements_per_token_(config.num_heads * config.head_dim),
      max_batch_size_(max_batch_size),
      max_total_candidates_(max_total_candidates),
      max_total_selected_pages_(max_total_selected_pages),
      max_requests_(max_requests) {
  if (max_batch_size < 0 || max_total_candidates < 0 || max_total_selected_pages < 0)
    throw std::invalid_argument("sparse CUDA context capacities must be non-negative");
  if (!SparseAttentionCudaAvailable())
    throw std::runtime_error("Sparse CUDA attention requires a visible sm_100 GPU (B200)");
  dsd_model_config mc{config.num_heads, config.head_dim, config.page_size, config.top_k_pages};
  dsd_ctx_options opt{cache.CapacityPages(), max_batch_size, max_total_candidates,
                      max_total_selected_pages, max_requests, max_pages_per_request};
  ThrowIf(dsd_ctx_create_ex(device, &mc, &opt, kv_format, &ctx_));
  pool_.reset(new DevicePagePool(config, ctx_, cache.CapacityPages()));
  try {
    pool_->UploadActivePagesFromCache(cache);
  } catch (...) {
    pool_.reset();
    dsd_ctx_destroy(ctx_);
    throw;
  }
  // queries are packed straight into the context's pinned staging and
  // outputs read from it: no extra host copy per step.  A head_dim the
  // device pads (not a power of two >= 4) has no such buffers: rows then go
  // through host vectors that the C ABI widens and narrows.
  if (dsd_step_host_buffers(ctx_, &host_queries_, &host_outputs_) != DSD_OK) {
    const std::size_t rows = static_cast<std::size_t>(std::max(1, max_batch_size));
    own_queries_.assign(rows * static_cast<std::size_t>(elements_per_token_), 0.0f);
    own_outputs_.assign(rows * static_cast<std::size_t>(elements_per_token_), 0.0f);
    host_queries_ = own_queries_.data();
    host_outputs_ = own_outputs_.data();
  }
  const unsigned hw = std::max(1u, std::thread::hardware_concurrency());
  pack_pool_.reset(new detail::WorkerPool(static_cast<int>(std::min(4u, hw) - 1)));
}

// Copies every request's query into the pinned step staging; large batches
// are split over the pack pool (the host copy is memory-bound).
void SparseCudaContext::PackQueries(const std::vector<const RequestState*>& requests,
                                    const std::vector<const float*>* query_rows) {
  const int B = static_cast<int>(requests.size());
  const int ept = elements_per_token_;
  auto copy_one = [&](int r) {
    const float* row = query_rows ? (*query_rows)[static_cast<std::size_t>(r)] : nullptr;
    if (row == nullptr) row = requests[static_cast<std::size_t>(r)]->query.data();
    std::copy(row, row + ept, host_queries_ + static_cast<std::size_t>(r) * ept);
  };
  if (static_cast<std::size_t>(B) * ept < (std::size_t(1) << 17)) {
    for (int r = 0; r < B; ++r) copy_one(r);
  } else {
    pack_pool_->ParallelFor(B, copy_one);
  }
}

SparseCudaContext::~SparseCudaContext() {
  pack_pool_.reset();
  pool_.reset();
  if (ctx_) dsd_ctx_destroy(ctx_);
}

SparseBatchCudaResult SparseCudaContext::RunBatch(const std::vector<RequestState>& requests,
                                                  SparseBatchOutputMode output_mode) {
  SparseRunBatchOptions o;
  o.output_mode = output_mode;
  o.timing_mode = SparseBatchTimingMode::kKernelEvents;
  return RunBatch(requests, o);
}

SparseBatchCudaResult SparseCudaContext::RunBatch(const std::vector<RequestState>& requests,
                                                  SparseRunBatchOptions options) {
  ptr_scratch_.clear();
  for (const auto& r : requests) ptr_scratch_.push_back(&r);
  return Run(ptr_scratch_, options, false);
}

SparseBatchCudaResult SparseCudaContext::RunBatch(const std::vector<const RequestState*>& requests,
                                                  SparseRunBatchOptions options) {
  return Run(requests, options, false);
}

SparseBatchCudaResult SparseCudaContext::RunStep(const std::vector<const RequestState*>& requests,
                                                 SparseRunBatchOptions options) {
  if (!HasRequestTables())
    throw std::invalid_argument("context was created without device request page tables");
  return Run(requests, options, true);
}

SparseBatchCudaResult SparseCudaContext::Run(const std::vector<const RequestState*>& requests,
                                             SparseRunBatchOptions options, bool tables) {
  SparseBatchCudaResult result;
  if (requests.empty()) return result;
  const bool debug = options.output_mode == SparseBatchOutputMode::kDebugTensors;
  const bool outputs = options.output_mode != SparseBatchOutputMode::kNoOutputs;
  const bool timed = options.timing_mode == SparseBatchTimingMode::kKernelEvents;
  const int B = static_cast<int>(requests.size());
  const int ept = elements_per_token_;
  if (B > max_batch_size_)
    throw std::invalid_argument("request batch exceeds sparse CUDA context capacity");
  const auto wall0 = std::chrono::steady_clock::now();

  double* prep = timed ? &result.runtime_overheads.time_prepare_sparse_layout_ms : nullptr;
  std::vector<int> sel_off(static_cast<std::size_t>(B) + 1, 0);
  int total_cand = 0;
  {
    ScopedStageTimer t(prep);
    offsets_.assign(1, 0);
    ids_.clear();
    request_ids_.clear();
    for (int r = 0; r < B; ++r) {
      const RequestState* q = requests[static_cast<std::size_t>(r)];
      if (!q) throw std::invalid_argument("request pointer must be non-null");
      if (static_cast<int>(q->query.size()) != ept)
        throw std::invalid_argument("query length does not match model config");
      int n;
      if (tables) {
        request_ids_.push_back(q->request_id);
        n = std::max(0, dsd_request_num_pages(ctx_, q->request_id));
      } else {
        ids_.insert(ids_.end(), q->candidate_page_ids.begin(), q->candidate_page_ids.end());
        n = static_cast<int>(q->candidate_page_ids.size());
      }
      offsets_.push_back(offsets_.back() + n);
      sel_off[static_cast<std::size_t>(r) + 1] =
          sel_off[static_cast<std::size_t>(r)] + std::max(0, std::min(config_.top_k_pages, n));
    }
    total_cand = offsets_.back();
    ThrowIf(dsd_step_staging_wait(ctx_));   // a queued step may still read the staging
    PackQueries(requests);
  }
  const int total_sel = sel_off.back();
  if (B > max_batch_size_)
    throw std::invalid_argument("request batch exceeds sparse CUDA context capacity");
  if (total_cand > max_total_candidates_)
    throw std::invalid_argument("candidate page count exceeds sparse CUDA context capacity");
  if (total_sel > max_total_selected_pages_)
    throw std::invalid_argument("selected page count exceeds sparse CUDA context capacity");

  const int mode = options.output_mode == SparseBatchOutputMode::kNoOutputs ? DSD_OUTPUT_NONE
                   : debug ? DSD_OUTPUT_DEBUG : DSD_OUTPUT_OUTPUTS;
  scores_.resize(static_cast<std::size_t>(std::max(1, total_cand)));
  selected_.resize(static_cast<std::size_t>(std::max(1, total_sel)));
  dsd_step_timing st{};
  if (tables) {
    ThrowIf(dsd_decode_step(ctx_, request_ids_.data(), B, host_queries_, mode, timed ? 1 : 0,
                            host_outputs_, scores_.data(), selected_.data(), &st));
  } else {
    ThrowIf(dsd_decode_batch(ctx_, B, host_queries_, offsets_.data(), ids_.data(), mode,
                             timed ? 1 : 0, host_outputs_, scores_.data(), selected_.data(), &st));
  }
  if (timed) {
    result.aggregate_timings.page_scoring_ms = st.score_ms;
    result.aggregate_timings.topk_ms = st.topk_ms;
    result.aggregate_timings.attention_ms = st.attention_ms;
    result.aggregate_timings.gather_ms = 0.0;   // fused into attention
    result.aggregate_timings.total_ms = st.score_ms + st.topk_ms + st.attention_ms;
    result.kernel_ms = result.aggregate_timings.total_ms;
    const double wall =
        std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - wall0).count();
    // the C ABI call copies, launches and waits in one go; its host time
    // beyond the kernels is reported as synchronisation overhead
    result.runtime_overheads.time_sync_ms =
        std::max(0.0, wall - result.runtime_overheads.time_prepare_sparse_layout_ms - result.kernel_ms);
  }
  if (!outputs) return result;
  result.per_request.reserve(static_cast<std::size_t>(B));
  for (int r = 0; r < B; ++r) {
    SparseDecodeResult one;
    one.request_id = requests[static_cast<std::size_t>(r)]->request_id;
    if (debug) {
      for (int c = offsets_[static_cast<std::size_t>(r)]; c < offsets_[static_cast<std::size_t>(r) + 1]; ++c) {
        const int page = tables ? -1 : ids_[static_cast<std::size_t>(c)];
        one.scores.push_back(PageScore{page, scores_[static_cast<std::size_t>(c)]});
      }
      one.selected_page_ids.assign(selected_.begin() + sel_off[static_cast<std::size_t>(r)],
                                   selected_.begin() + sel_off[static_cast<std::size_t>(r) + 1]);
    }
    one.output.output.assign(host_outputs_ + static_cast<std::ptrdiff_t>(r) * ept,
                             host_outputs_ + static_cast<std::ptrdiff_t>(r + 1) * ept);
    result.per_request.push_back(std::move(one));
  }
  if (debug && tables) {
    // page ids of the scores come from the requests' own candidate lists
    for (int r = 0; r < B; ++r) {
      const auto& cand = requests[static_cast<std::size_t>(r)]->candidate_page_ids;
      auto& sc = result.per_request[static_cast<std::size_t>(r)].scores;
      for (std::size_t i = 0; i < sc.size() && i < cand.size(); ++i) sc[i].page_id = cand[i];
    }
  }
  return result;
}

void SparseCudaContext::BeginStep(const std::vector<const RequestState*>& requests,
                                  SparseRunBatchOptions options) {
  BeginStep(requests, options, nullptr);
}

void SparseCudaContext::BeginStep(const std::vector<const RequestState*>& requests,
                                  SparseRunBatchOptions options,
                                  const std::vector<const float*>* query_rows) {
  if (query_rows && query_rows->size() != requests.size())
    throw std::invalid_argument("one query row per request");
  if (!HasRequestTables())
    throw std::invalid_argument("context was created without device request page tables");
  if (pending_.size() >= 2) throw std::invalid_argument("two steps are already pending");
  const int B = static_cast<int>(requests.size());
  if (B == 0) throw std::invalid_argument("empty batch");
  if (B > max_batch_size_)
    throw std::invalid_argument("request batch exceeds sparse CUDA context capacity");
  const int ept = elements_per_token_;
  const bool debug = options.output_mode == SparseBatchOutputMode::kDebugTensors;
  const auto t0 = std::chrono::steady_clock::now();
  PendingStep ps;
  ps.options = options;
  ps.sel_off.assign(static_cast<std::size_t>(B) + 1, 0);
  ps.cand_off.assign(1, 0);
  for (int r = 0; r < B; ++r) {
    const RequestState* q = requests[static_cast<std::size_t>(r)];
    if (!q) throw std::invalid_argument("request pointer must be non-null");
    const bool row = query_rows && (*query_rows)[static_cast<std::size_t>(r)] != nullptr;
    if (!row && static_cast<int>(q->query.size()) != ept)
      throw std::invalid_argument("query length does not match model config");
    ps.request_ids.push_back(q->request_id);
    if (debug) ps.candidates.push_back(q->candidate_page_ids);
    const int n = std::max(0, dsd_request_num_pages(ctx_, q->request_id));
    ps.cand_off.push_back(ps.cand_off.back() + n);
    ps.sel_off[static_cast<std::size_t>(r) + 1] =
        ps.sel_off[static_cast<std::size_t>(r)] + std::min(config_.top_k_pages, n);
  }
  if (ps.cand_off.back() > max_total_candidates_)
    throw std::invalid_argument("candidate page count exceeds sparse CUDA context capacity");
  if (ps.sel_off.back() > max_total_selected_pages_)
    throw std::invalid_argument("selected page count exceeds sparse CUDA context capacity");
  ThrowIf(dsd_step_staging_wait(ctx_));   // the staging may still feed the previous step
  PackQueries(requests, query_rows);
  ps.prep_ms =
      std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
  const int mode = options.output_mode == SparseBatchOutputMode::kNoOutputs ? DSD_OUTPUT_NONE
                   : debug ? DSD_OUTPUT_DEBUG : DSD_OUTPUT_OUTPUTS;
  const bool timed = options.timing_mode == SparseBatchTimingMode::kKernelEvents;
  ThrowIf(dsd_decode_step_begin(ctx_, ps.request_ids.data(), B, host_queries_, mode,
                                timed ? 1 : 0));
  pending_.push_back(std::move(ps));
}

SparseBatchCudaResult SparseCudaContext::FinishStep() { return FinishStep(true); }

SparseBatchCudaResult SparseCudaContext::FinishStep(bool copy_outputs) {
  if (pending_.empty()) throw std::invalid_argument("no step is pending");
  PendingStep ps = std::move(pending_.front());
  pending_.erase(pending_.begin());
  const int B = static_cast<int>(ps.request_ids.size());
  const int ept = elements_per_token_;
  const bool debug = ps.options.output_mode == SparseBatchOutputMode::kDebugTensors;
  const bool timed = ps.options.timing_mode == SparseBatchTimingMode::kKernelEvents;
  scores_.resize(static_cast<std::size_t>(std::max(1, ps.cand_off.back())));
  selected_.resize(static_cast<std::size_t>(std::max(1, ps.sel_off.back())));
  finish_outputs_.resize(static_cast<std::size_t>(B) * ept);
  dsd_step_timing st{};
  const auto t0 = std::chrono::steady_clock::now();
  ThrowIf(dsd_decode_step_end(ctx_, copy_outputs ? finish_outputs_.data() : nullptr,
                              scores_.data(), selected_.data(), &st));
  SparseBatchCudaResult result;
  if (timed) {
    result.aggregate_timings.page_scoring_ms = st.score_ms;
    result.aggregate_timings.topk_ms = st.topk_ms;
    result.aggregate_timings.attention_ms = st.attention_ms;
    result.aggregate_timings.total_ms = st.score_ms + st.topk_ms + st.attention_ms;
    result.kernel_ms = result.aggregate_timings.total_ms;
    result.runtime_overheads.time_prepare_sparse_layout_ms = ps.prep_ms;
    result.runtime_overheads.time_sync_ms =
        std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
  }
  if (ps.options.output_mode == SparseBatchOutputMode::kNoOutputs) return result;
  result.per_request.reserve(static_cast<std::size_t>(B));
  for (int r = 0; r < B; ++r) {
    SparseDecodeResult one;
    one.request_id = ps.request_ids[static_cast<std::size_t>(r)];
    if (debug) {
      const auto& cand = ps.candidates[static_cast<std::size_t>(r)];
      const int c0 = ps.cand_off[static_cast<std::size_t>(r)];
      for (int c = c0; c < ps.cand_off[static_cast<std::size_t>(r) + 1]; ++c) {
        const std::size_t i = static_cast<std::size_t>(c - c0);
        one.scores.push_back(PageScore{i < cand.size() ? cand[i] : -1, scores_[static_cast<std::size_t>(c)]});
      }
      one.selected_page_ids.assign(selected_.begin() + ps.sel_off[static_cast<std::size_t>(r)],
                                   selected_.begin() + ps.sel_off[static_cast<std::size_t>(r) + 1]);
    }
    if (copy_outputs)
      one.output.output.assign(finish_outputs_.begin() + static_cast<std::ptrdiff_t>(r) * ept,
                               finish_outputs_.begin() + static_cast<std::ptrdiff_t>(r + 1) * ept);
    result.per_request.push_back(std::move(one));
  }
  return result;
}

void SparseCudaContext::SyncPageFromCache(const PagedKvCache& cache, PageId page_id) {
  SyncPagesFromCache(cache, {page_id});
}
void SparseCudaContext::SyncPagesFromCache(const PagedKvCache& cache,
                                           const std::vector<PageId>& page_ids) {
  cache_ = &cache;
  pool_->UploadPagesFromCache(cache, page_ids);
}
void SparseCudaContext::SyncPromptDirect(const PagedKvCache& cache,
                                         const std::vector<PageId>& page_ids,
                                         const std::vector<int>& token_counts,
                                         const float* prompt_keys, const float* prompt_values) {
  cache_ = &cache;
  pool_->UploadPromptDirect(cache, page_ids, token_counts, prompt_keys, prompt_values);
}
void SparseCudaContext::PrefillPromptSynthetic(const PagedKvCache& cache,
                                               const std::vector<PageId>& page_ids,
                                               const std::vector<int>& token_counts,
                                               int request_id) {
  cache_ = &cache;
  pool_->PrefillPromptSynthetic(cache, page_ids, token_counts, request_id);
}
void SparseCudaContext::SyncAppendedToken(const PagedKvCache& cache,
                                          const AppendTokenResult& result) {
  SyncAppendedTokens(cache, {result});
}
void SparseCudaContext::SyncAppendedTokens(const PagedKvCache& cache,
                                           const std::vector<AppendTokenResult>& results) {
  cache_ = &cache;
  pool_->UploadTokensFromCache(cache, results);
}
void SparseCudaContext::SyncAppendedTokensDirect(const PagedKvCache& cache,
                                                 const std::vector<AppendTokenResult>& results,
                                                 const std::vector<float>& token_keys,
                                                 const std::vector<float>& token_values) {
  cache_ = &cache;
  pool_->UploadTokensDirect(cache, results, token_keys, token_values);
}
void SparseCudaContext::AppendSyntheticTokens(const PagedKvCache& cache,
                                              const std::vector<AppendTokenResult>& results,
                                              const std::vector<int>& request_ids,
                                              const std::vector<int>& decode_steps) {
  cache_ = &cache;
  pool_->AppendTokensSynthetic(cache, results, request_ids, decode_steps);
}
void SparseCudaContext::SyncFreedPages(const std::vector<PageId>& page_ids) {
  pool_->MarkPagesFree(page_ids);
}
void SparseCudaContext::ResetDeviceTransferStats() { pool_->ResetTransferStats(); }
DeviceTransferStats SparseCudaContext::DeviceTransfers() const { return pool_->transfer_stats(); }

void SparseCudaContext::SetRequestPages(int request_id, const std::vector<PageId>& page_ids) {
  ThrowIf(dsd_request_set_pages(ctx_, request_id, page_ids.data(),
                                static_cast<int>(page_ids.size())));
}
void SparseCudaContext::AppendRequestPages(int request_id, const std::vector<PageId>& page_ids) {
  ThrowIf(dsd_request_append_pages(ctx_, request_id, page_ids.data(),
                                   static_cast<int>(page_ids.size())));
}
void SparseCudaContext::AppendRequestPages(const std::vector<int>& request_ids,
                                           const std::vector<PageId>& page_ids) {
  if (request_ids.size() != page_ids.size())
    throw std::invalid_argument("one request id per page");
  ThrowIf(dsd_request_append_pages_multi(ctx_, request_ids.data(), page_ids.data(),
                                         static_cast<int>(page_ids.size())));
}
void SparseCudaContext::ReleaseRequestPages(int request_id, bool free_pages) {
  ThrowIf(dsd_request_release(ctx_, request_id, free_pages ? 1 : 0));
}

SparseDecodeResult SparseDecodeCuda(const PagedKvCache& cache, const RequestState& request,
                                    const ModelConfig& config) {
  const int n = static_cast<int>(request.candidate_page_ids.size());
  SparseCudaContext ctx(cache, config, 1, n, std::min(config.top_k_pages, n));
  auto batch = ctx.RunBatch(std::vector<RequestState>{request}, SparseBatchOutputMode::kDebugTensors);
  SparseDecodeResult r;
  if (!batch.per_request.empty()) r = std::move(batch.per_request.front());
  r.request_id = request.request_id;
  r.timings = batch.aggregate_timings;
  r.runtime_overheads = batch.runtime_overheads;
  return r;
}

AttentionResult SparseAttentionCuda(const PagedKvCache& cache, const std::vector<float>& query,
                                    const std::vector<PageId>& selected_page_ids,
                                    const ModelConfig& config, double* gather_ms,
                                    double* attention_ms,
                                    RuntimeOverheadTimings* runtime_overheads) {
  RequestState req;
  req.request_id = 0;
  req.query = query;
  req.candidate_page_ids = selected_page_ids;
  req.context_tokens = static_cast<int>(selected_page_ids.size()) * config.page_size;
  ModelConfig local = config;
  local.top_k_pages = static_cast<int>(selected_page_ids.size());
  const auto r = SparseDecodeCuda(cache, req, local);
  if (gather_ms) *gather_ms = r.timings.gather_ms;
  if (attention_ms) *attention_ms = r.timings.attention_ms;
  if (runtime_overheads) *runtime_overheads = r.runtime_overheads;
  return r.output;
}

}  // namespace dsd
