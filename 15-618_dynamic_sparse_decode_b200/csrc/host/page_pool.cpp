// PagePool: LIFO slot allocator (src/page_pool.cpp:18-128 in the reference).
#include "dsd/page_pool.h"

#include <algorithm>
#include <stdexcept>

namespace dsd {

PagePool::PagePool(ModelConfig config, int capacity_pages, bool allocate_storage)
    : config_(config), has_storage_(allocate_storage) {
  if (capacity_pages < 0) throw std::invalid_argument("capacity_pages must be non-negative");
  capacity_pages_ = capacity_pages;
  live_.assign(static_cast<std::size_t>(capacity_pages_), 0);
  if (allocate_storage) {
    const std::size_t n = static_cast<std::size_t>(capacity_pages_) * elements_per_page();
    keys_.assign(n, 0.0f);
    values_.assign(n, 0.0f);
  }
  reset_pool();
}

PageId PagePool::allocate_page() {
  if (free_.empty()) throw std::runtime_error("page pool is exhausted");
  const PageId id = free_.back();
  free_.pop_back();
  live_[static_cast<std::size_t>(id)] = 1;
  return id;
}

void PagePool::free_page(PageId page_id) {
  CheckId(page_id);
  CheckLive(page_id);
  live_[static_cast<std::size_t>(page_id)] = 0;
  free_.push_back(page_id);
}

void PagePool::CheckId(PageId page_id) const {
  if (page_id < 0 || page_id >= capacity_pages_) throw std::out_of_range("invalid page id");
}

void PagePool::CheckLive(PageId page_id) const {
  if (!live_[static_cast<std::size_t>(page_id)])
    throw std::runtime_error("page is not currently allocated");
}

float* PagePool::Slot(std::vector<float>& pool, PageId page_id) {
  CheckId(page_id);
  CheckLive(page_id);
  if (!has_storage_) throw std::runtime_error("page pool KV storage is disabled");
  return pool.data() + static_cast<std::ptrdiff_t>(page_id) * elements_per_page();
}

const float* PagePool::Slot(const std::vector<float>& pool, PageId page_id) const {
  CheckId(page_id);
  CheckLive(page_id);
  if (!has_storage_) throw std::runtime_error("page pool KV storage is disabled");
  return pool.data() + static_cast<std::ptrdiff_t>(page_id) * elements_per_page();
}

float* PagePool::get_k_page_ptr(PageId page_id) { return Slot(keys_, page_id); }
const float* PagePool::get_k_page_ptr(PageId page_id) const { return Slot(keys_, page_id); }
float* PagePool::get_v_page_ptr(PageId page_id) { return Slot(values_, page_id); }
const float* PagePool::get_v_page_ptr(PageId page_id) const { return Slot(values_, page_id); }

void PagePool::reset_pool() {
  std::fill(live_.begin(), live_.end(), 0);
  free_.resize(static_cast<std::size_t>(capacity_pages_));
  for (PageId i = 0; i < capacity_pages_; ++i) free_[static_cast<std::size_t>(i)] = i;
}

bool PagePool::is_allocated(PageId page_id) const {
  CheckId(page_id);
  return live_[static_cast<std::size_t>(page_id)] != 0;
}

}  // namespace dsd
