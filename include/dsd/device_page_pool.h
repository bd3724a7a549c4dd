// GPU-resident page pool (drop-in for include/dsd/device_page_pool.h:17-140)
// over the C ABI (include/dsd_b200.h).  Layout in HBM: page-major K and V
// [capacity][page_size][H*D] fp32, summaries chunk-major in 128-page groups
// (see include/dsd_b200.h), token counts,
// live flags.  Page offsets are derived (page * page_size * H*D), so the
// reference's per-page offset tables do not exist: page_k/v_offsets_device()
// return nullptr.
#pragma once

#include <cstdint>
#include <vector>

#include "dsd/config.h"
#include "dsd/paged_kv_cache.h"
#include "dsd/types.h"

struct dsd_ctx;

namespace dsd {

class DevicePagePool {
 public:
  DevicePagePool(ModelConfig config, int capacity_pages);
  // A pool that shares an existing context (used by SparseCudaContext).
  DevicePagePool(ModelConfig config, dsd_ctx* shared_ctx, int capacity_pages);
  ~DevicePagePool();
  DevicePagePool(const DevicePagePool&) = delete;
  DevicePagePool& operator=(const DevicePagePool&) = delete;
  DevicePagePool(DevicePagePool&& other) noexcept;
  DevicePagePool& operator=(DevicePagePool&& other) noexcept;

  void Reset();
  void UploadPage(PageId page_id, const float* host_keys, const float* host_values,
                  int token_count);
  void UploadPageFromCache(const PagedKvCache& cache, PageId page_id);
  void UploadPagesFromCache(const PagedKvCache& cache, const std::vector<PageId>& page_ids);
  void UploadActivePagesFromCache(const PagedKvCache& cache);
  void UploadPromptDirect(const PagedKvCache& cache, const std::vector<PageId>& page_ids,
                          const std::vector<int>& token_counts, const float* prompt_keys,
                          const float* prompt_values);
  void PrefillPromptSynthetic(const PagedKvCache& cache, const std::vector<PageId>& page_ids,
                              const std::vector<int>& token_counts, int request_id);
  void UploadTokenFromCache(const PagedKvCache& cache, PageId page_id, int token_offset);
  void UploadTokensFromCache(const PagedKvCache& cache,
                             const std::vector<AppendTokenResult>& results);
  void UploadTokensDirect(const PagedKvCache& cache, const std::vector<AppendTokenResult>& results,
                          const std::vector<float>& token_keys,
                          const std::vector<float>& token_values);
  void AppendTokensSynthetic(const PagedKvCache& cache,
                             const std::vector<AppendTokenResult>& results,
                             const std::vector<int>& request_ids,
                             const std::vector<int>& decode_steps);
  void MarkPageFree(PageId page_id);
  void MarkPagesFree(const std::vector<PageId>& page_ids);
  void DownloadPage(PageId page_id, std::vector<float>* host_keys,
                    std::vector<float>* host_values) const;
  void DownloadMetadata(std::vector<int>* token_counts, std::vector<std::uint8_t>* live_mask) const;
  void UploadAllFromCache(const PagedKvCache& cache);

  void ResetTransferStats();
  DeviceTransferStats transfer_stats() const;

  int capacity_pages() const { return capacity_pages_; }
  int elements_per_token() const { return config_.num_heads * config_.head_dim; }
  int elements_per_page() const { return config_.page_size * elements_per_token(); }

  const float* key_base_device() const;
  const float* value_base_device() const;
  const float* page_summary_base_device() const;
  const int* page_token_counts_device() const;
  const std::uint8_t* page_live_mask_device() const { return nullptr; }
  const std::uint64_t* page_k_offsets_device() const { return nullptr; }
  const std::uint64_t* page_v_offsets_device() const { return nullptr; }

  dsd_ctx* handle() const { return ctx_; }

 private:
  void CheckCache(const PagedKvCache& cache) const;
  ModelConfig config_;
  int capacity_pages_ = 0;
  dsd_ctx* ctx_ = nullptr;
  bool owns_ctx_ = false;
};

}  // namespace dsd
