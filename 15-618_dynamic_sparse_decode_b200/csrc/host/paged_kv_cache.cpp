// PagedKvCache (reference: src/paged_kv_cache.cpp).  Summary arithmetic is
// kept operation for operation (AppendPage :88-99, AppendToken :231-238)
// because the GPU path reproduces it bit for bit.
#include "dsd/paged_kv_cache.h"

#include <algorithm>
#include <stdexcept>

namespace dsd {

namespace {
const std::vector<PageId>& NoPages() {
  static const std::vector<PageId> empty;
  return empty;
}
}  // namespace

PagedKvCache::PagedKvCache(ModelConfig config, int capacity_pages, bool allocate_kv_storage)
    : config_(config), pool_(config, capacity_pages, allocate_kv_storage) {
  summaries_.assign(static_cast<std::size_t>(capacity_pages) * ElementsPerToken(), 0.0f);
  summary_dirty_.assign(static_cast<std::size_t>(capacity_pages), 0);
  pages_.reserve(static_cast<std::size_t>(capacity_pages));
  for (PageId p = 0; p < capacity_pages; ++p) pages_.push_back(FreeDescriptor(p));
}

PageDescriptor PagedKvCache::FreeDescriptor(PageId page_id) const {
  const std::size_t off = static_cast<std::size_t>(page_id) * ElementsPerPage();
  return PageDescriptor{page_id, -1, 0, 0, off, off};
}

int PagedKvCache::NextStartToken(int request_id) const {
  auto it = request_pages_.find(request_id);
  if (it == request_pages_.end() || it->second.empty()) return 0;
  const auto& last = GetPage(it->second.back());
  return last.start_token + last.token_count;
}

float* PagedKvCache::Summary(PageId page_id) {
  if (page_id < 0 || page_id >= static_cast<PageId>(pages_.size()))
    throw std::out_of_range("invalid page id");
  return summaries_.data() + static_cast<std::ptrdiff_t>(page_id) * ElementsPerToken();
}

const float* PagedKvCache::Summary(PageId page_id) const {
  if (page_id < 0 || page_id >= static_cast<PageId>(pages_.size()))
    throw std::out_of_range("invalid page id");
  return summaries_.data() + static_cast<std::ptrdiff_t>(page_id) * ElementsPerToken();
}

// Clears a page's summary row unless it is known to be zero already: rows of
// pages that were only reserved for GPU-resident prompts are never written
// on the host, so admission does not memset 16 KiB per reserved page.
void PagedKvCache::ClearSummary(PageId page_id) {
  float* s = Summary(page_id);
  auto& dirty = summary_dirty_[static_cast<std::size_t>(page_id)];
  if (dirty) std::fill(s, s + ElementsPerToken(), 0.0f);
  dirty = 0;
}

PageId PagedKvCache::AppendPage(int request_id, const std::vector<float>& keys,
                                const std::vector<float>& values, int token_count) {
  if (token_count <= 0 || token_count > config_.page_size)
    throw std::invalid_argument("token_count must be in (0, page_size]");
  const std::size_t n = static_cast<std::size_t>(token_count) * ElementsPerToken();
  if (keys.size() != n || values.size() != n)
    throw std::invalid_argument("page payload does not match expected size");
  return AppendPage(request_id, keys.data(), values.data(), token_count, true);
}

PageId PagedKvCache::AppendPage(int request_id, const float* keys, const float* values,
                                int token_count) {
  return AppendPage(request_id, keys, values, token_count, true);
}

PageId PagedKvCache::AppendPage(int request_id, const float* keys, const float* values,
                                int token_count, bool compute_summary) {
  if (token_count <= 0 || token_count > config_.page_size)
    throw std::invalid_argument("token_count must be in (0, page_size]");
  const int ept = ElementsPerToken();
  const std::size_t n = static_cast<std::size_t>(token_count) * ept;
  if (n == 0) throw std::invalid_argument("page payload does not match expected size");
  if (keys == nullptr || values == nullptr)
    throw std::invalid_argument("page payload pointers must be non-null");

  const PageId id = pool_.allocate_page();
  const int start = NextStartToken(request_id);
  std::copy(keys, keys + n, pool_.get_k_page_ptr(id));
  std::copy(values, values + n, pool_.get_v_page_ptr(id));
  ClearSummary(id);
  float* s = Summary(id);
  if (compute_summary) {
    summary_dirty_[static_cast<std::size_t>(id)] = 1;
    for (int t = 0; t < token_count; ++t) {
      const float* k = keys + static_cast<std::size_t>(t) * ept;
      for (int i = 0; i < ept; ++i) s[i] += k[i];
    }
    const float inv = 1.0f / static_cast<float>(token_count);
    for (int i = 0; i < ept; ++i) s[i] *= inv;
  }
  const std::size_t off = static_cast<std::size_t>(id) * ElementsPerPage();
  pages_[static_cast<std::size_t>(id)] = PageDescriptor{id, request_id, start, token_count, off, off};
  request_pages_[request_id].push_back(id);
  ++active_pages_;
  return id;
}

std::vector<PageId> PagedKvCache::ReservePagesForRequest(int request_id,
                                                         const std::vector<int>& token_counts) {
  std::vector<PageId> ids;
  if (token_counts.empty()) return ids;
  for (int c : token_counts)
    if (c <= 0 || c > config_.page_size)
      throw std::invalid_argument("token_count must be in (0, page_size]");
  for (std::size_t i = 0; i < token_counts.size(); ++i) ids.push_back(pool_.allocate_page());
  std::sort(ids.begin(), ids.end());
  int start = NextStartToken(request_id);
  auto& list = request_pages_[request_id];
  for (std::size_t i = 0; i < ids.size(); ++i) {
    const PageId id = ids[i];
    ClearSummary(id);
    const std::size_t off = static_cast<std::size_t>(id) * ElementsPerPage();
    pages_[static_cast<std::size_t>(id)] = PageDescriptor{id, request_id, start, token_counts[i], off, off};
    list.push_back(id);
    start += token_counts[i];
    ++active_pages_;
  }
  return ids;
}

// Chooses the page the next token of `request_id` goes to, allocating a
// fresh (zero-summary) page when forced, when the request has none, or when
// its tail page is full.
PageId PagedKvCache::TailForAppend(int request_id, bool force_new_page, bool* allocated) {
  auto& list = request_pages_[request_id];
  *allocated = false;
  PageId id;
  if (force_new_page || list.empty() ||
      pages_[static_cast<std::size_t>(list.back())].token_count >= config_.page_size) {
    id = pool_.allocate_page();
    const std::size_t off = static_cast<std::size_t>(id) * ElementsPerPage();
    pages_[static_cast<std::size_t>(id)] =
        PageDescriptor{id, request_id, NextStartToken(request_id), 0, off, off};
    ClearSummary(id);
    list.push_back(id);
    ++active_pages_;
    *allocated = true;
  } else {
    id = list.back();
  }
  const auto& page = pages_[static_cast<std::size_t>(id)];
  if (page.request_id != request_id || page.token_count < 0 ||
      page.token_count >= config_.page_size)
    throw std::runtime_error("request tail page is inconsistent");
  return id;
}

AppendTokenResult PagedKvCache::AppendToken(int request_id, const std::vector<float>& key,
                                            const std::vector<float>& value) {
  return AppendToken(request_id, key, value, false);
}

AppendTokenResult PagedKvCache::AppendToken(int request_id, const std::vector<float>& key,
                                            const std::vector<float>& value,
                                            bool force_new_page) {
  const int ept = ElementsPerToken();
  if (static_cast<int>(key.size()) != ept || static_cast<int>(value.size()) != ept)
    throw std::invalid_argument("token payload does not match expected size");
  return AppendToken(request_id, key.data(), value.data(), force_new_page);
}

AppendTokenResult PagedKvCache::AppendToken(int request_id, const float* key, const float* value,
                                            bool force_new_page) {
  if (key == nullptr || value == nullptr)
    throw std::invalid_argument("token payload pointers must be non-null");
  bool allocated = false;
  const PageId id = TailForAppend(request_id, force_new_page, &allocated);
  auto& page = pages_[static_cast<std::size_t>(id)];
  const int ept = ElementsPerToken();
  const int off = page.token_count;
  std::copy(key, key + ept, pool_.get_k_page_ptr(id) + static_cast<std::ptrdiff_t>(off) * ept);
  std::copy(value, value + ept, pool_.get_v_page_ptr(id) + static_cast<std::ptrdiff_t>(off) * ept);
  float* s = Summary(id);
  summary_dirty_[static_cast<std::size_t>(id)] = 1;
  const float old_c = static_cast<float>(page.token_count);
  const float new_c = old_c + 1.0f;
  for (int i = 0; i < ept; ++i) s[i] = (s[i] * old_c + key[i]) / new_c;
  ++page.token_count;
  return AppendTokenResult{id, off, allocated};
}

AppendTokenResult PagedKvCache::AppendTokenMetadataOnly(int request_id,
                                                        const std::vector<float>& key,
                                                        bool force_new_page) {
  if (static_cast<int>(key.size()) != ElementsPerToken())
    throw std::invalid_argument("token payload does not match expected size");
  return AppendTokenMetadataOnly(request_id, key.data(), force_new_page);
}

AppendTokenResult PagedKvCache::AppendTokenMetadataOnly(int request_id, const float* key,
                                                        bool force_new_page) {
  if (key == nullptr) throw std::invalid_argument("token payload pointer must be non-null");
  bool allocated = false;
  const PageId id = TailForAppend(request_id, force_new_page, &allocated);
  auto& page = pages_[static_cast<std::size_t>(id)];
  const int off = page.token_count;
  float* s = Summary(id);
  summary_dirty_[static_cast<std::size_t>(id)] = 1;
  const float old_c = static_cast<float>(page.token_count);
  const float new_c = old_c + 1.0f;
  for (int i = 0; i < ElementsPerToken(); ++i) s[i] = (s[i] * old_c + key[i]) / new_c;
  ++page.token_count;
  return AppendTokenResult{id, off, allocated};
}

AppendTokenResult PagedKvCache::AppendTokenMetadataOnly(int request_id, bool force_new_page) {
  bool allocated = false;
  const PageId id = TailForAppend(request_id, force_new_page, &allocated);
  auto& page = pages_[static_cast<std::size_t>(id)];
  const int off = page.token_count;
  ++page.token_count;
  return AppendTokenResult{id, off, allocated};
}

std::vector<PageId> PagedKvCache::ReleaseRequest(int request_id) {
  auto it = request_pages_.find(request_id);
  if (it == request_pages_.end()) return {};
  std::vector<PageId> released = it->second;
  for (PageId id : released) {
    if (pages_[static_cast<std::size_t>(id)].request_id != request_id)
      throw std::runtime_error("request page mapping is inconsistent");
    // The summary row is not cleared here: every allocation path clears it
    // before use, and a free page (token_count 0) reads as zeros through
    // CopyPageSummary.  Skipping the 16 KiB clear per page keeps release
    // O(pages) instead of O(pages * H * D) in the serving loop.
    pages_[static_cast<std::size_t>(id)] = FreeDescriptor(id);
    pool_.free_page(id);
    --active_pages_;
  }
  request_pages_.erase(it);
  return released;
}

void PagedKvCache::Reset() {
  request_pages_.clear();
  active_pages_ = 0;
  pool_.reset_pool();
  for (PageId p = 0; p < static_cast<PageId>(pages_.size()); ++p) ClearSummary(p);
  for (PageId p = 0; p < static_cast<PageId>(pages_.size()); ++p)
    pages_[static_cast<std::size_t>(p)] = FreeDescriptor(p);
}

const PageDescriptor& PagedKvCache::GetPage(PageId page_id) const {
  if (page_id < 0 || page_id >= static_cast<PageId>(pages_.size()))
    throw std::out_of_range("invalid page id");
  return pages_[static_cast<std::size_t>(page_id)];
}

const std::vector<PageId>& PagedKvCache::GetRequestPages(int request_id) const {
  auto it = request_pages_.find(request_id);
  return it == request_pages_.end() ? NoPages() : it->second;
}

std::vector<float> PagedKvCache::CopyPageKeys(PageId page_id) const {
  const auto& page = GetPage(page_id);
  const std::size_t n = static_cast<std::size_t>(page.token_count) * ElementsPerToken();
  if (n == 0) return {};
  const float* k = pool_.get_k_page_ptr(page_id);
  return std::vector<float>(k, k + n);
}

std::vector<float> PagedKvCache::CopyPageValues(PageId page_id) const {
  const auto& page = GetPage(page_id);
  const std::size_t n = static_cast<std::size_t>(page.token_count) * ElementsPerToken();
  if (n == 0) return {};
  const float* v = pool_.get_v_page_ptr(page_id);
  return std::vector<float>(v, v + n);
}

void PagedKvCache::CopyPageToken(PageId page_id, int token_offset, std::vector<float>* key,
                                 std::vector<float>* value) const {
  if (key == nullptr || value == nullptr)
    throw std::invalid_argument("token copy outputs must be non-null");
  const auto& page = GetPage(page_id);
  if (page.request_id == -1 || page.token_count == 0)
    throw std::invalid_argument("cannot copy a token from a free page");
  if (token_offset < 0 || token_offset >= page.token_count)
    throw std::out_of_range("token_offset is outside the valid page prefix");
  const int ept = ElementsPerToken();
  const float* k = pool_.get_k_page_ptr(page_id) + static_cast<std::ptrdiff_t>(token_offset) * ept;
  const float* v = pool_.get_v_page_ptr(page_id) + static_cast<std::ptrdiff_t>(token_offset) * ept;
  key->assign(k, k + ept);
  value->assign(v, v + ept);
}

std::vector<float> PagedKvCache::CopyPageSummary(PageId page_id) const {
  const auto& page = GetPage(page_id);
  if (page.token_count == 0) return std::vector<float>(static_cast<std::size_t>(ElementsPerToken()), 0.0f);
  const float* s = Summary(page_id);
  return std::vector<float>(s, s + ElementsPerToken());
}

std::vector<float> PagedKvCache::BuildPageSummary(PageId page_id) const {
  return CopyPageSummary(page_id);
}

}  // namespace dsd
