// Host page allocator (drop-in for include/dsd/page_pool.h:11-48).
// The free list starts as 0..N-1 and pops from the back, so the first
// allocation returns N-1 (LIFO); freed pages are reused first.  Page ids
// decide top-k tie-breaks, so this order is part of the parity contract.
#pragma once

#include <cstdint>
#include <vector>

#include "dsd/config.h"
#include "dsd/types.h"

namespace dsd {

class PagePool {
 public:
  PagePool(ModelConfig config, int capacity_pages, bool allocate_storage = true);

  PageId allocate_page();              // std::runtime_error when exhausted
  void free_page(PageId page_id);      // out_of_range / runtime_error on misuse

  float* get_k_page_ptr(PageId page_id);
  const float* get_k_page_ptr(PageId page_id) const;
  float* get_v_page_ptr(PageId page_id);
  const float* get_v_page_ptr(PageId page_id) const;

  void reset_pool();

  int capacity_pages() const { return capacity_pages_; }
  bool is_allocated(PageId page_id) const;
  int elements_per_token() const { return config_.num_heads * config_.head_dim; }
  int elements_per_page() const { return config_.page_size * elements_per_token(); }

  const std::vector<float>& key_storage() const { return keys_; }
  const std::vector<float>& value_storage() const { return values_; }
  bool has_storage() const { return has_storage_; }

 private:
  void CheckId(PageId page_id) const;
  void CheckLive(PageId page_id) const;
  float* Slot(std::vector<float>& pool, PageId page_id);
  const float* Slot(const std::vector<float>& pool, PageId page_id) const;

  ModelConfig config_;
  int capacity_pages_ = 0;
  std::vector<PageId> free_;
  std::vector<std::uint8_t> live_;
  std::vector<float> keys_;
  std::vector<float> values_;
  bool has_storage_ = true;
};

}  // namespace dsd
