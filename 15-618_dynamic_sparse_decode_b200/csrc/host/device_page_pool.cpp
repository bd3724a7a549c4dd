// DevicePagePool over the C ABI (reference: src/device_page_pool.cpp).
// Differences by design: summaries uploaded from a host cache are copied
// verbatim (the device then holds exactly what sparse_cpu reads), and
// summaries computed on the device use the host cache's formulas, so the GPU
// and CPU paths never disagree on a summary.
#include "dsd/device_page_pool.h"

#include <algorithm>
#include <stdexcept>

#include "capi_error.h"
#include "dsd_b200.h"

namespace dsd {

using detail::ThrowIf;

DevicePagePool::DevicePagePool(ModelConfig config, int capacity_pages)
    : config_(config), capacity_pages_(capacity_pages), owns_ctx_(true) {
  if (capacity_pages < 0) throw std::invalid_argument("capacity_pages must be non-negative");
  dsd_model_config mc{config.num_heads, config.head_dim, config.page_size, config.top_k_pages};
  dsd_ctx_options opt{capacity_pages, 0, 0, 0, 0, 0};
  ThrowIf(dsd_ctx_create(0, &mc, &opt, &ctx_));
}

DevicePagePool::DevicePagePool(ModelConfig config, dsd_ctx* shared_ctx, int capacity_pages)
    : config_(config), capacity_pages_(capacity_pages), ctx_(shared_ctx), owns_ctx_(false) {}

DevicePagePool::~DevicePagePool() {
  if (owns_ctx_ && ctx_) dsd_ctx_destroy(ctx_);
}

DevicePagePool::DevicePagePool(DevicePagePool&& o) noexcept
    : config_(o.config_), capacity_pages_(o.capacity_pages_), ctx_(o.ctx_), owns_ctx_(o.owns_ctx_) {
  o.ctx_ = nullptr;
  o.owns_ctx_ = false;
}

DevicePagePool& DevicePagePool::operator=(DevicePagePool&& o) noexcept {
  if (this != &o) {
    if (owns_ctx_ && ctx_) dsd_ctx_destroy(ctx_);
    config_ = o.config_;
    capacity_pages_ = o.capacity_pages_;
    ctx_ = o.ctx_;
    owns_ctx_ = o.owns_ctx_;
    o.ctx_ = nullptr;
    o.owns_ctx_ = false;
  }
  return *this;
}

void DevicePagePool::CheckCache(const PagedKvCache& cache) const {
  if (cache.CapacityPages() != capacity_pages_)
    throw std::invalid_argument("cache capacity does not match device page pool");
}

void DevicePagePool::Reset() { ThrowIf(dsd_pool_reset(ctx_)); }

void DevicePagePool::UploadPage(PageId page_id, const float* host_keys, const float* host_values,
                                int token_count) {
  if (page_id < 0 || page_id >= capacity_pages_) throw std::out_of_range("invalid page id");
  if (token_count <= 0 || token_count > config_.page_size)
    throw std::invalid_argument("token_count must be in (0, page_size]");
  if (!host_keys || !host_values)
    throw std::invalid_argument("host page payload pointers must be non-null");
  ThrowIf(dsd_pool_upload_pages(ctx_, &page_id, &token_count, 1, host_keys, host_values, 1));
}

void DevicePagePool::UploadPageFromCache(const PagedKvCache& cache, PageId page_id) {
  UploadPagesFromCache(cache, {page_id});
}

void DevicePagePool::UploadPagesFromCache(const PagedKvCache& cache,
                                          const std::vector<PageId>& page_ids) {
  CheckCache(cache);
  if (page_ids.empty()) return;
  std::vector<PageId> ids = page_ids;
  std::sort(ids.begin(), ids.end());
  ids.erase(std::unique(ids.begin(), ids.end()), ids.end());
  const int ept = elements_per_token();
  std::vector<int> counts;
  std::vector<float> keys, values, summaries;
  for (PageId id : ids) {
    if (id < 0 || id >= capacity_pages_) throw std::out_of_range("invalid page id");
    const auto& page = cache.GetPage(id);
    if (page.request_id == -1 || page.token_count == 0)
      throw std::invalid_argument("cannot upload a free or empty page from cache");
    counts.push_back(page.token_count);
    const auto k = cache.CopyPageKeys(id);
    const auto v = cache.CopyPageValues(id);
    keys.insert(keys.end(), k.begin(), k.end());
    values.insert(values.end(), v.begin(), v.end());
    const float* s = cache.PageSummaryPool().data() + static_cast<std::size_t>(id) * ept;
    summaries.insert(summaries.end(), s, s + ept);
  }
  ThrowIf(dsd_pool_upload_pages(ctx_, ids.data(), counts.data(), static_cast<int>(ids.size()),
                                keys.data(), values.data(), 0));
  ThrowIf(dsd_pool_upload_summaries(ctx_, ids.data(), static_cast<int>(ids.size()),
                                    summaries.data()));
}

void DevicePagePool::UploadActivePagesFromCache(const PagedKvCache& cache) {
  std::vector<PageId> ids;
  for (const auto& p : cache.Pages())
    if (p.request_id != -1 && p.token_count > 0) ids.push_back(p.id);
  UploadPagesFromCache(cache, ids);
}

void DevicePagePool::UploadAllFromCache(const PagedKvCache& cache) {
  Reset();
  UploadActivePagesFromCache(cache);
}

void DevicePagePool::UploadPromptDirect(const PagedKvCache& cache,
                                        const std::vector<PageId>& page_ids,
                                        const std::vector<int>& token_counts,
                                        const float* prompt_keys, const float* prompt_values) {
  CheckCache(cache);
  if (page_ids.size() != token_counts.size())
    throw std::invalid_argument("page_ids and token_counts sizes must match");
  if (page_ids.empty()) return;
  for (std::size_t i = 0; i < page_ids.size(); ++i) {
    if (page_ids[i] < 0 || page_ids[i] >= capacity_pages_) throw std::out_of_range("invalid page id");
    if (token_counts[i] <= 0 || token_counts[i] > config_.page_size)
      throw std::invalid_argument("token_count must be in (0, page_size]");
    const auto& page = cache.GetPage(page_ids[i]);
    if (page.request_id == -1 || page.token_count != token_counts[i])
      throw std::invalid_argument("reserved prompt page metadata is inconsistent");
  }
  if (!prompt_keys || !prompt_values)
    throw std::invalid_argument("prompt payload pointers must be non-null");
  ThrowIf(dsd_pool_upload_pages(ctx_, page_ids.data(), token_counts.data(),
                                static_cast<int>(page_ids.size()), prompt_keys, prompt_values, 1));
}

void DevicePagePool::PrefillPromptSynthetic(const PagedKvCache& cache,
                                            const std::vector<PageId>& page_ids,
                                            const std::vector<int>& token_counts, int request_id) {
  CheckCache(cache);
  if (page_ids.size() != token_counts.size())
    throw std::invalid_argument("page_ids and token_counts sizes must match");
  if (page_ids.empty()) return;
  for (std::size_t i = 0; i < page_ids.size(); ++i) {
    const auto& page = cache.GetPage(page_ids[i]);
    if (page.request_id == -1 || page.token_count != token_counts[i])
      throw std::invalid_argument("reserved prompt page metadata is inconsistent");
  }
  ThrowIf(dsd_pool_prefill_synthetic(ctx_, page_ids.data(), token_counts.data(),
                                     static_cast<int>(page_ids.size()), request_id));
}

void DevicePagePool::UploadTokenFromCache(const PagedKvCache& cache, PageId page_id,
                                          int token_offset) {
  UploadTokensFromCache(cache, {AppendTokenResult{page_id, token_offset, false}});
}

void DevicePagePool::UploadTokensFromCache(const PagedKvCache& cache,
                                           const std::vector<AppendTokenResult>& results) {
  CheckCache(cache);
  if (results.empty()) return;
  const int ept = elements_per_token();
  std::vector<int> ids, offs;
  std::vector<float> keys, values, k, v;
  for (const auto& r : results) {
    if (r.page_id < 0 || r.page_id >= capacity_pages_) throw std::out_of_range("invalid page id");
    cache.CopyPageToken(r.page_id, r.token_offset, &k, &v);
    ids.push_back(r.page_id);
    offs.push_back(r.token_offset);
    keys.insert(keys.end(), k.begin(), k.end());
    values.insert(values.end(), v.begin(), v.end());
  }
  ThrowIf(dsd_append_tokens(ctx_, ids.data(), offs.data(), nullptr, static_cast<int>(ids.size()),
                            keys.data(), values.data()));
  // the device now holds the cache's summaries exactly
  std::vector<int> uniq = ids;
  std::sort(uniq.begin(), uniq.end());
  uniq.erase(std::unique(uniq.begin(), uniq.end()), uniq.end());
  std::vector<float> summ;
  for (int id : uniq) {
    const float* s = cache.PageSummaryPool().data() + static_cast<std::size_t>(id) * ept;
    summ.insert(summ.end(), s, s + ept);
  }
  ThrowIf(dsd_pool_upload_summaries(ctx_, uniq.data(), static_cast<int>(uniq.size()), summ.data()));
}

void DevicePagePool::UploadTokensDirect(const PagedKvCache& cache,
                                        const std::vector<AppendTokenResult>& results,
                                        const std::vector<float>& token_keys,
                                        const std::vector<float>& token_values) {
  CheckCache(cache);
  if (results.empty()) return;
  const std::size_t n = results.size() * static_cast<std::size_t>(elements_per_token());
  if (token_keys.size() != n || token_values.size() != n)
    throw std::invalid_argument("direct token payload size does not match results");
  std::vector<int> ids, offs;
  for (const auto& r : results) {
    if (r.page_id < 0 || r.page_id >= capacity_pages_) throw std::out_of_range("invalid page id");
    const auto& page = cache.GetPage(r.page_id);
    if (page.request_id == -1 || page.token_count == 0)
      throw std::invalid_argument("cannot upload a token to a free cache page");
    if (r.token_offset < 0 || r.token_offset >= page.token_count)
      throw std::out_of_range("token_offset is outside the valid page prefix");
    ids.push_back(r.page_id);
    offs.push_back(r.token_offset);
  }
  ThrowIf(dsd_append_tokens(ctx_, ids.data(), offs.data(), nullptr, static_cast<int>(ids.size()),
                            token_keys.data(), token_values.data()));
}

void DevicePagePool::AppendTokensSynthetic(const PagedKvCache& cache,
                                           const std::vector<AppendTokenResult>& results,
                                           const std::vector<int>& request_ids,
                                           const std::vector<int>& decode_steps) {
  CheckCache(cache);
  if (results.empty()) return;
  if (request_ids.size() != results.size() || decode_steps.size() != results.size())
    throw std::invalid_argument("synthetic append metadata size mismatch");
  std::vector<int> ids, offs;
  for (std::size_t i = 0; i < results.size(); ++i) {
    const auto& r = results[i];
    const auto& page = cache.GetPage(r.page_id);
    if (page.request_id == -1 || page.token_count == 0)
      throw std::invalid_argument("cannot append a synthetic token to a free page");
    if (r.token_offset < 0 || r.token_offset >= page.token_count)
      throw std::out_of_range("token_offset is outside the valid page prefix");
    if (page.request_id != request_ids[i])
      throw std::invalid_argument("synthetic append request_id mismatch");
    ids.push_back(r.page_id);
    offs.push_back(r.token_offset);
  }
  ThrowIf(dsd_append_tokens_synthetic(ctx_, ids.data(), offs.data(), request_ids.data(),
                                      decode_steps.data(), static_cast<int>(ids.size())));
}

void DevicePagePool::MarkPageFree(PageId page_id) { MarkPagesFree({page_id}); }

void DevicePagePool::MarkPagesFree(const std::vector<PageId>& page_ids) {
  if (page_ids.empty()) return;
  std::vector<PageId> ids = page_ids;
  std::sort(ids.begin(), ids.end());
  ids.erase(std::unique(ids.begin(), ids.end()), ids.end());
  ThrowIf(dsd_pool_free_pages(ctx_, ids.data(), static_cast<int>(ids.size())));
}

void DevicePagePool::DownloadPage(PageId page_id, std::vector<float>* host_keys,
                                  std::vector<float>* host_values) const {
  if (!host_keys || !host_values) throw std::invalid_argument("download outputs must be non-null");
  if (page_id < 0 || page_id >= capacity_pages_) throw std::out_of_range("invalid page id");
  const std::size_t pf = static_cast<std::size_t>(elements_per_page());
  std::vector<float> k(pf), v(pf);
  int count = 0;
  ThrowIf(dsd_download_page(ctx_, page_id, k.data(), v.data(), nullptr, &count));
  if (count == 0) throw std::runtime_error("cannot download a free device page");
  const std::size_t n = static_cast<std::size_t>(count) * elements_per_token();
  host_keys->assign(k.begin(), k.begin() + static_cast<std::ptrdiff_t>(n));
  host_values->assign(v.begin(), v.begin() + static_cast<std::ptrdiff_t>(n));
}

void DevicePagePool::DownloadMetadata(std::vector<int>* token_counts,
                                      std::vector<std::uint8_t>* live_mask) const {
  if (!token_counts || !live_mask) throw std::invalid_argument("metadata outputs must be non-null");
  token_counts->resize(static_cast<std::size_t>(capacity_pages_));
  live_mask->resize(static_cast<std::size_t>(capacity_pages_));
  ThrowIf(dsd_download_metadata(ctx_, token_counts->data(), live_mask->data()));
}

void DevicePagePool::ResetTransferStats() { ThrowIf(dsd_reset_transfer_stats(ctx_)); }

DeviceTransferStats DevicePagePool::transfer_stats() const {
  dsd_transfer_stats s{};
  ThrowIf(dsd_get_transfer_stats(ctx_, &s));
  return DeviceTransferStats{s.h2d_bytes, s.d2h_bytes, s.h2d_calls,
                             s.d2h_calls, s.h2d_large_calls, s.d2h_large_calls};
}

const float* DevicePagePool::key_base_device() const {
  float* p = nullptr;
  ThrowIf(dsd_ctx_device_pointers(ctx_, &p, nullptr, nullptr, nullptr));
  return p;
}
const float* DevicePagePool::value_base_device() const {
  float* p = nullptr;
  ThrowIf(dsd_ctx_device_pointers(ctx_, nullptr, &p, nullptr, nullptr));
  return p;
}
const float* DevicePagePool::page_summary_base_device() const {
  float* p = nullptr;
  ThrowIf(dsd_ctx_device_pointers(ctx_, nullptr, nullptr, &p, nullptr));
  return p;
}
const int* DevicePagePool::page_token_counts_device() const {
  int* p = nullptr;
  ThrowIf(dsd_ctx_device_pointers(ctx_, nullptr, nullptr, nullptr, &p));
  return p;
}

}  // namespace dsd
