// Host page pool and paged cache behaviour the reference's CPU tests pin
// (tests/test_page_pool.cpp, tests/test_reference.cpp), on this build's API.
#include <cmath>
#include <vector>

#include "check.h"
#include "dsd/decode_pipeline.h"
#include "dsd/page_pool.h"
#include "dsd/paged_kv_cache.h"
#include "dsd/reference_kernels.h"
#include "dsd/synthetic_data.h"

namespace {

std::vector<float> Seq(int n, float start) {
  std::vector<float> v(static_cast<std::size_t>(n));
  for (int i = 0; i < n; ++i) v[static_cast<std::size_t>(i)] = start + static_cast<float>(i);
  return v;
}

void PagePoolOrder() {
  dsd::ModelConfig c;
  c.num_heads = 2; c.head_dim = 4; c.page_size = 4;
  dsd::PagePool pool(c, 3);
  CHECK(pool.allocate_page() == 2 && pool.allocate_page() == 1 && pool.allocate_page() == 0,
        "LIFO allocation order must be 2,1,0");
  CHECK(Throws<std::runtime_error>([&] { pool.allocate_page(); }), "exhaustion must throw");
  CHECK(pool.get_k_page_ptr(1) - pool.get_k_page_ptr(0) == pool.elements_per_page(),
        "page slots are contiguous");
  pool.free_page(1);
  CHECK(pool.allocate_page() == 1, "freed page is reused first");
  CHECK(Throws<std::out_of_range>([&] { pool.free_page(7); }), "invalid id must throw");
  pool.free_page(0);
  CHECK(Throws<std::runtime_error>([&] { pool.free_page(0); }), "double free must throw");
  pool.reset_pool();
  CHECK(pool.allocate_page() == 2, "reset restores the free list");
}

void AppendAndRelease() {
  dsd::ModelConfig c;
  c.num_heads = 2; c.head_dim = 4; c.page_size = 4;
  const int ept = 8;
  dsd::PagedKvCache cache(c, 4);
  const auto k0 = Seq(3 * ept, 1.0f), v0 = Seq(3 * ept, 101.0f);
  const auto p0 = cache.AppendPage(7, k0, v0, 3);
  auto r = cache.AppendToken(7, Seq(ept, 500.0f), Seq(ept, 600.0f));
  CHECK(r.page_id == p0 && r.token_offset == 3 && !r.allocated_new_page, "token goes into the tail");
  // summary is the running mean of the 4 keys
  std::vector<float> mean(ept, 0.0f);
  for (int t = 0; t < 3; ++t)
    for (int i = 0; i < ept; ++i) mean[i] += k0[static_cast<std::size_t>(t * ept + i)];
  for (int i = 0; i < ept; ++i) mean[i] = (mean[i] + 500.0f + i) / 4.0f;
  CHECK(dsd::MaxAbsDiff(cache.CopyPageSummary(p0), mean) <= 1e-5f, "incremental summary");
  r = cache.AppendToken(7, Seq(ept, 700.0f), Seq(ept, 800.0f));
  CHECK(r.allocated_new_page && r.token_offset == 0, "full tail page opens a new page");
  CHECK(cache.GetPage(r.page_id).start_token == 4, "start_token continues the request");
  r = cache.AppendToken(7, Seq(ept, 900.0f), Seq(ept, 950.0f), true);
  CHECK(r.allocated_new_page, "force_new_page opens a page");
  const auto released = cache.ReleaseRequest(7);
  CHECK(released.size() == 3 && cache.TotalPages() == 0, "release frees every page");
  const auto reuse = cache.AppendToken(9, Seq(ept, 1.0f), Seq(ept, 2.0f));
  CHECK(reuse.page_id == released.back(), "released pages are reused LIFO");
  CHECK(cache.CopyPageSummary(released.front())[0] == 0.0f, "released summaries are zero");
}

void PayloadRoundTrip() {
  dsd::ModelConfig c;
  c.num_heads = 2; c.head_dim = 4; c.page_size = 4;
  dsd::PagedKvCache cache(c, 4);
  const auto k = Seq(32, 1.0f), v = Seq(32, 101.0f);
  const auto id = cache.AppendPage(9, k, v, 4);
  CHECK(cache.CopyPageKeys(id) == k && cache.CopyPageValues(id) == v, "payload copy-back");
  std::vector<float> s(8, 0.0f);
  for (int t = 0; t < 4; ++t)
    for (int i = 0; i < 8; ++i) s[i] += k[static_cast<std::size_t>(t * 8 + i)];
  for (float& x : s) x /= 4.0f;
  CHECK(dsd::MaxAbsDiff(cache.CopyPageSummary(id), s) <= 1e-6f, "summary is the key mean");
  cache.Reset();
  CHECK(cache.TotalPages() == 0 && cache.GetRequestPages(9).empty(), "reset clears state");
  for (float x : cache.PageSummaryPool()) CHECK(x == 0.0f, "reset clears summaries");
  CHECK(cache.AppendPage(5, Seq(16, 0.0f), Seq(16, 0.0f), 2) == 3, "reset restores LIFO order");
  CHECK(Throws<std::invalid_argument>([&] { cache.AppendPage(5, Seq(16, 0.0f), Seq(16, 0.0f), 5); }),
        "token_count beyond page_size must throw");
  const auto ids = cache.ReservePagesForRequest(6, {4, 4, 1});
  CHECK(ids.size() == 3 && ids[0] < ids[1] && ids[1] < ids[2], "reserved ids ascend");
}

void SparseEqualsDenseWhenKCoversAll() {
  dsd::ModelConfig c;
  c.num_heads = 2; c.head_dim = 8; c.page_size = 4; c.top_k_pages = 64;
  const auto b = dsd::BuildSyntheticBatch(c, 3, 12, 12, 123);
  dsd::DecodePipeline p(c);
  for (const auto& r : b.requests) {
    const auto s = p.RunNaiveSparseStep(b.cache, r);
    const auto d = p.RunDenseStep(b.cache, r);
    CHECK(dsd::MaxAbsDiff(s.output.output, d.output) <= 1e-5f, "sparse == dense when k >= pages");
  }
  int pages = 0;
  const auto b2 = dsd::BuildSyntheticBatch(c, 5, 7, 13, 42);
  for (const auto& r : b2.requests) pages += (r.context_tokens + 3) / 4;
  CHECK(b2.cache.TotalPages() == pages, "synthetic capacity equals the page count");
  CHECK(dsd::SelectTopKPagesCpu(dsd::ScorePagesCpu(b.cache, b.requests[0], c), 2).size() == 2,
        "top-k count");
}

}  // namespace

int main() {
  PagePoolOrder();
  AppendAndRelease();
  PayloadRoundTrip();
  SparseEqualsDenseWhenKCoversAll();
  std::cout << "host cache tests passed\n";
  return 0;
}
