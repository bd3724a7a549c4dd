// Batched sparse decode on the GPU (drop-in for
// include/dsd/cuda_sparse_attention.h:17-151) over the C ABI.
// RunBatch scores every candidate page of each request against its query
// (one score per page over all heads), selects min(top_k, n) pages by
// (score desc, page id asc) and attends over their tokens for every head.
// Selection is bit-identical to the CPU reference; outputs match it within
// 1e-4.  Errors: std::invalid_argument (sizes, capacities),
// std::out_of_range (page ids), std::runtime_error (CUDA, no GPU).
#pragma once

#include <cstdint>
#include <memory>
#include <vector>

#include "dsd/config.h"
#include "dsd/device_page_pool.h"
#include "dsd/paged_kv_cache.h"
#include "dsd/types.h"

struct dsd_ctx;

namespace dsd {

namespace detail {
class WorkerPool;
}

bool SparseAttentionCudaAvailable();

enum class SparseBatchOutputMode { kNoOutputs, kOutputsOnly, kDebugTensors };
enum class SparseBatchTimingMode { kNone, kKernelEvents };

struct SparseRunBatchOptions {
  SparseBatchOutputMode output_mode = SparseBatchOutputMode::kOutputsOnly;
  SparseBatchTimingMode timing_mode = SparseBatchTimingMode::kKernelEvents;
};

// Kept for API compatibility; the GPU path packs on the device.
struct PackedSparseBatch {
  std::vector<float> queries;
  std::vector<int> request_candidate_offsets;
  std::vector<int> candidate_page_ids;
  std::vector<int> selected_offsets;
  std::vector<int> selected_counts;
  int num_requests = 0;
  int total_candidates = 0;
  int total_selected_pages = 0;
  int num_heads = 0;
  int head_dim = 0;
  int elements_per_token = 0;
  int max_candidates_per_request = 0;
};

class SparseCudaContext {
 public:
  // Uploads every active page of `cache` (K, V and its summaries verbatim).
  // max_requests / max_pages_per_request > 0 also create device request page
  // tables for RunStep (the continuous-batching path).  kv_format (this
  // build) selects the device page format: DSD_KV_F32 (default, the
  // reference's) or DSD_KV_BF16.
  SparseCudaContext(const PagedKvCache& cache, const ModelConfig& config, int max_batch_size,
                    int max_total_candidates, int max_total_selected_pages,
                    int max_requests = 0, int max_pages_per_request = 0, int device = 0,
                    int kv_format = 0);
  ~SparseCudaContext();
  SparseCudaContext(const SparseCudaContext&) = delete;
  SparseCudaContext& operator=(const SparseCudaContext&) = delete;

  SparseBatchCudaResult RunBatch(
      const std::vector<RequestState>& requests,
      SparseBatchOutputMode output_mode = SparseBatchOutputMode::kOutputsOnly);
  SparseBatchCudaResult RunBatch(const std::vector<RequestState>& requests,
                                 SparseRunBatchOptions options);
  SparseBatchCudaResult RunBatch(const std::vector<const RequestState*>& requests,
                                 SparseRunBatchOptions options);

  // Device page-table step: candidates are each request's device page list
  // (maintained by Sync*/Append*/Release calls with tables enabled); only the
  // queries go up and the outputs come back.
  SparseBatchCudaResult RunStep(const std::vector<const RequestState*>& requests,
                                SparseRunBatchOptions options);

  // RunStep split in two: BeginStep uploads the queries and queues the step;
  // host work and further uploads on this context (appends, frees, the next
  // BeginStep) may follow before FinishStep waits for the OLDEST pending
  // step's results.  Up to two steps may be pending; the requests are copied
  // as needed, so they may change after BeginStep returns.
  void BeginStep(const std::vector<const RequestState*>& requests, SparseRunBatchOptions options);
  SparseBatchCudaResult FinishStep();
  // This build: BeginStep whose request r takes its query from query_rows[r]
  // when that is non-null (num_heads*head_dim floats, read before the call
  // returns) instead of requests[r]->query -- the serving loop's precomputed
  // queries go straight into the pinned staging.  FinishStep(false) leaves
  // per_request[r].output empty: the outputs still come back to the host
  // staging, but are not copied out for a caller that does not read them.
  void BeginStep(const std::vector<const RequestState*>& requests, SparseRunBatchOptions options,
                 const std::vector<const float*>* query_rows);
  SparseBatchCudaResult FinishStep(bool copy_outputs);

  void SyncPageFromCache(const PagedKvCache& cache, PageId page_id);
  void SyncPagesFromCache(const PagedKvCache& cache, const std::vector<PageId>& page_ids);
  void SyncPromptDirect(const PagedKvCache& cache, const std::vector<PageId>& page_ids,
                        const std::vector<int>& token_counts, const float* prompt_keys,
                        const float* prompt_values);
  void PrefillPromptSynthetic(const PagedKvCache& cache, const std::vector<PageId>& page_ids,
                              const std::vector<int>& token_counts, int request_id);
  void SyncAppendedToken(const PagedKvCache& cache, const AppendTokenResult& result);
  void SyncAppendedTokens(const PagedKvCache& cache, const std::vector<AppendTokenResult>& results);
  void SyncAppendedTokensDirect(const PagedKvCache& cache,
                                const std::vector<AppendTokenResult>& results,
                                const std::vector<float>& token_keys,
                                const std::vector<float>& token_values);
  void AppendSyntheticTokens(const PagedKvCache& cache,
                             const std::vector<AppendTokenResult>& results,
                             const std::vector<int>& request_ids,
                             const std::vector<int>& decode_steps);
  void SyncFreedPages(const std::vector<PageId>& page_ids);
  void ResetDeviceTransferStats();
  DeviceTransferStats DeviceTransfers() const;

  // device request page tables
  void SetRequestPages(int request_id, const std::vector<PageId>& page_ids);
  void AppendRequestPages(int request_id, const std::vector<PageId>& page_ids);
  // one upload for new pages of several requests (request_ids[i] gets page_ids[i])
  void AppendRequestPages(const std::vector<int>& request_ids, const std::vector<PageId>& page_ids);
  void ReleaseRequestPages(int request_id, bool free_pages);
  bool HasRequestTables() const { return max_requests_ > 0; }
  int PendingSteps() const { return static_cast<int>(pending_.size()); }

  DevicePagePool& device_pool() { return *pool_; }
  dsd_ctx* handle() const { return ctx_; }

 private:
  SparseBatchCudaResult Run(const std::vector<const RequestState*>& requests,
                            SparseRunBatchOptions options, bool tables);
  const PagedKvCache* cache_ = nullptr;
  ModelConfig config_{};
  int elements_per_token_ = 0;
  int max_batch_size_ = 0;
  int max_total_candidates_ = 0;
  int max_total_selected_pages_ = 0;
  int max_requests_ = 0;
  dsd_ctx* ctx_ = nullptr;
  std::unique_ptr<DevicePagePool> pool_;
  std::vector<const RequestState*> ptr_scratch_;
  float* host_queries_ = nullptr;   // pinned step staging owned by the context
  float* host_outputs_ = nullptr;
  std::vector<float> own_queries_, own_outputs_;   // used when the device pads head_dim
  std::vector<int> offsets_, ids_, request_ids_, selected_;
  std::vector<float> scores_;
  std::vector<float> finish_outputs_;
  // steps queued by BeginStep, oldest first
  struct PendingStep {
    std::vector<int> request_ids;
    std::vector<std::vector<PageId>> candidates;   // debug mode only
    std::vector<int> cand_off, sel_off;
    SparseRunBatchOptions options;
    double prep_ms = 0.0;
  };
  std::vector<PendingStep> pending_;
  std::unique_ptr<detail::WorkerPool> pack_pool_;   // parallel query packing
  void PackQueries(const std::vector<const RequestState*>& requests,
                   const std::vector<const float*>* query_rows = nullptr);
};

SparseDecodeResult SparseDecodeCuda(const PagedKvCache& cache, const RequestState& request,
                                    const ModelConfig& config);

AttentionResult SparseAttentionCuda(const PagedKvCache& cache, const std::vector<float>& query,
                                    const std::vector<PageId>& selected_page_ids,
                                    const ModelConfig& config, double* gather_ms = nullptr,
                                    double* attention_ms = nullptr,
                                    RuntimeOverheadTimings* runtime_overheads = nullptr);

}  // namespace dsd
