// Host paged KV cache (drop-in for include/dsd/paged_kv_cache.h:13-122):
// request -> ordered page list, per-page descriptors, K/V storage (optional:
// metadata-only caches mirror a GPU-resident pool) and the per-page key
// summary that page scoring reads.  Summary formulas are part of the parity
// contract: AppendPage = token-order sum then * (1/n); AppendToken = running
// mean (s*old + k)/(old+1).
#pragma once

#include <cstddef>
#include <cstdint>
#include <unordered_map>
#include <vector>

#include "dsd/config.h"
#include "dsd/page_pool.h"
#include "dsd/types.h"

namespace dsd {

struct PageDescriptor {
  PageId id = -1;
  int request_id = -1;
  int start_token = 0;
  int token_count = 0;
  std::size_t k_offset = 0;
  std::size_t v_offset = 0;
};

class PagedKvCache {
 public:
  explicit PagedKvCache(ModelConfig config, int capacity_pages = 1024,
                        bool allocate_kv_storage = true);

  PageId AppendPage(int request_id, const std::vector<float>& keys,
                    const std::vector<float>& values, int token_count);
  PageId AppendPage(int request_id, const float* keys, const float* values, int token_count);
  PageId AppendPage(int request_id, const float* keys, const float* values, int token_count,
                    bool compute_summary);

  // Allocates one page per entry, ids sorted ascending, summaries zero.
  std::vector<PageId> ReservePagesForRequest(int request_id, const std::vector<int>& token_counts);

  AppendTokenResult AppendToken(int request_id, const std::vector<float>& key,
                                const std::vector<float>& value);
  AppendTokenResult AppendToken(int request_id, const std::vector<float>& key,
                                const std::vector<float>& value, bool force_new_page);
  AppendTokenResult AppendToken(int request_id, const float* key, const float* value,
                                bool force_new_page);
  AppendTokenResult AppendTokenMetadataOnly(int request_id, const std::vector<float>& key,
                                            bool force_new_page);
  AppendTokenResult AppendTokenMetadataOnly(int request_id, const float* key,
                                            bool force_new_page);
  AppendTokenResult AppendTokenMetadataOnly(int request_id, bool force_new_page);

  // Frees the request's pages (LIFO reuse).  Their raw PageSummaryPool()
  // rows are left as they were; a free page reads as zeros through
  // CopyPageSummary / BuildPageSummary and is cleared when reallocated.
  std::vector<PageId> ReleaseRequest(int request_id);
  void Reset();

  const PageDescriptor& GetPage(PageId page_id) const;
  const std::vector<PageId>& GetRequestPages(int request_id) const;
  const std::vector<PageDescriptor>& Pages() const { return pages_; }
  const std::vector<float>& KeyPool() const { return pool_.key_storage(); }
  const std::vector<float>& ValuePool() const { return pool_.value_storage(); }
  const std::vector<float>& PageSummaryPool() const { return summaries_; }

  std::vector<float> CopyPageKeys(PageId page_id) const;
  std::vector<float> CopyPageValues(PageId page_id) const;
  void CopyPageToken(PageId page_id, int token_offset, std::vector<float>* key,
                     std::vector<float>* value) const;
  std::vector<float> CopyPageSummary(PageId page_id) const;
  std::vector<float> BuildPageSummary(PageId page_id) const;

  int TotalPages() const { return active_pages_; }
  int CapacityPages() const { return pool_.capacity_pages(); }
  int ElementsPerToken() const { return config_.num_heads * config_.head_dim; }
  int ElementsPerPage() const { return config_.page_size * ElementsPerToken(); }
  bool HasKvStorage() const { return pool_.has_storage(); }

 private:
  PageDescriptor FreeDescriptor(PageId page_id) const;
  int NextStartToken(int request_id) const;
  float* Summary(PageId page_id);
  const float* Summary(PageId page_id) const;
  PageId TailForAppend(int request_id, bool force_new_page, bool* allocated);
  void ClearSummary(PageId page_id);

  ModelConfig config_;
  PagePool pool_;
  std::vector<PageDescriptor> pages_;
  std::vector<float> summaries_;
  std::vector<std::uint8_t> summary_dirty_;   // row may hold non-zero values
  std::unordered_map<int, std::vector<PageId>> request_pages_;
  int active_pages_ = 0;
};

}  // namespace dsd
