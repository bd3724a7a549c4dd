// GPU tests of the drop-in C++ API against its CPU backend on the same cache:
// the reference's sparse CUDA test cases (tests/test_sparse_cuda.cpp) plus
// the device-pool round trips (tests/test_device_page_pool.cpp) and a
// continuous append/release/reuse sequence (tests/test_continuous_batching.cpp).
#include <algorithm>
#include <vector>

#include "check.h"
#include "dsd/continuous_batching.h"
#include "dsd/cuda_dense_attention.h"
#include "dsd/cuda_sparse_attention.h"
#include "dsd/decode_pipeline.h"
#include "dsd/device_page_pool.h"
#include "dsd/synthetic_data.h"

namespace {

dsd::ModelConfig Cfg(int h, int d, int p, int k) {
  dsd::ModelConfig c;
  c.num_heads = h; c.head_dim = d; c.page_size = p; c.top_k_pages = k;
  return c;
}

std::vector<float> Seq(int n, float start) {
  std::vector<float> v(static_cast<std::size_t>(n));
  for (int i = 0; i < n; ++i) v[static_cast<std::size_t>(i)] = start + 0.5f * static_cast<float>(i);
  return v;
}

void SyntheticCase(dsd::ModelConfig c, int batch, int lo, int hi, int seed, float tol) {
  const auto b = dsd::BuildSyntheticBatch(c, batch, lo, hi, seed);
  int cand = 0, sel = 0;
  for (const auto& r : b.requests) {
    cand += static_cast<int>(r.candidate_page_ids.size());
    sel += std::min<int>(c.top_k_pages, static_cast<int>(r.candidate_page_ids.size()));
  }
  dsd::SparseCudaContext ctx(b.cache, c, batch, cand, sel);
  const auto g = ctx.RunBatch(b.requests, dsd::SparseBatchOutputMode::kDebugTensors);
  CHECK(g.per_request.size() == b.requests.size(), "one result per request");
  CHECK(g.aggregate_timings.gather_ms == 0.0, "gather is fused into attention");
  dsd::DecodePipeline p(c);
  for (std::size_t i = 0; i < b.requests.size(); ++i) {
    const auto cpu = p.RunNaiveSparseStep(b.cache, b.requests[i]);
    CHECK(cpu.selected_page_ids == g.per_request[i].selected_page_ids, "selected pages differ");
    CHECK(dsd::MaxAbsDiff(cpu.output.output, g.per_request[i].output.output) <= tol,
          "output differs beyond tolerance");
    for (std::size_t j = 0; j < cpu.scores.size(); ++j)
      CHECK(cpu.scores[j].score == g.per_request[i].scores[j].score &&
                cpu.scores[j].page_id == g.per_request[i].scores[j].page_id,
            "scores differ");
  }
  // no-output fast path (tests/test_sparse_cuda.cpp:171-205)
  dsd::SparseRunBatchOptions o;
  o.output_mode = dsd::SparseBatchOutputMode::kNoOutputs;
  o.timing_mode = dsd::SparseBatchTimingMode::kNone;
  const auto none = ctx.RunBatch(b.requests, o);
  CHECK(none.per_request.empty() && none.kernel_ms == 0.0, "no-output mode returns nothing");
}

// dense_gpu vs dense_cpu (tests/test_dense_cuda.cpp:21-156) incl. a request with no pages
void DenseBaseline() {
  const auto c = Cfg(4, 32, 8, 4);
  auto b = dsd::BuildSyntheticBatch(c, 3, 40, 120, 5);
  dsd::RequestState empty;
  empty.request_id = 99;
  empty.query = b.requests[0].query;
  b.requests.push_back(empty);
  dsd::DenseCudaContext ctx(b.cache, c);
  const auto g = ctx.RunBatch(b.requests);
  dsd::DecodePipeline p(c);
  CHECK(g.outputs.size() == b.requests.size(), "one dense output per request");
  for (std::size_t i = 0; i < b.requests.size(); ++i)
    CHECK(dsd::MaxAbsDiff(p.RunDenseStep(b.cache, b.requests[i]).output, g.outputs[i].output) <= 5e-5f,
          "dense output differs");
}

void TopKZero() {
  const auto c = Cfg(2, 8, 4, 0);
  const auto b = dsd::BuildSyntheticBatch(c, 3, 5, 19, 11);
  int cand = 0;
  for (const auto& r : b.requests) cand += static_cast<int>(r.candidate_page_ids.size());
  dsd::SparseCudaContext ctx(b.cache, c, 3, cand, 0);
  const auto g = ctx.RunBatch(b.requests, dsd::SparseBatchOutputMode::kDebugTensors);
  for (const auto& r : g.per_request) {
    CHECK(r.selected_page_ids.empty(), "k=0 selects nothing");
    for (float x : r.output.output) CHECK(x == 0.0f, "k=0 gives a zero output");
  }
}

void TieBreak() {
  const auto c = Cfg(2, 8, 4, 2);
  dsd::PagedKvCache cache(c, 4);
  const std::vector<float> zeros(4 * 16, 0.0f);
  for (int i = 0; i < 4; ++i) cache.AppendPage(0, zeros, Seq(64, float(i)), 4);
  dsd::RequestState r;
  r.request_id = 0;
  r.query = Seq(16, 1.0f);
  r.candidate_page_ids = {3, 2, 1, 0};
  dsd::SparseCudaContext ctx(cache, c, 1, 4, 2);
  const auto g = ctx.RunBatch({r}, dsd::SparseBatchOutputMode::kDebugTensors);
  CHECK((g.per_request[0].selected_page_ids == std::vector<int>{0, 1}), "ties go to lower ids");
}

void DevicePoolRoundTrip() {
  const auto c = Cfg(2, 4, 4, 2);
  dsd::PagedKvCache cache(c, 3);
  const auto a = cache.AppendPage(1, Seq(32, 1.0f), Seq(32, 100.0f), 4);
  const auto b = cache.AppendPage(1, Seq(16, 200.0f), Seq(16, 300.0f), 2);
  dsd::DevicePagePool pool(c, 3);
  pool.UploadPagesFromCache(cache, {b, a});
  std::vector<float> k, v;
  pool.DownloadPage(a, &k, &v);
  CHECK(k == cache.CopyPageKeys(a) && v == cache.CopyPageValues(a), "page round trip");
  pool.DownloadPage(b, &k, &v);
  CHECK(k.size() == 16 && k == cache.CopyPageKeys(b), "partial page round trip");
  std::vector<int> counts;
  std::vector<std::uint8_t> live;
  pool.DownloadMetadata(&counts, &live);
  CHECK(counts[a] == 4 && counts[b] == 2 && live[a] == 1 && live[0] == 0, "metadata");
  CHECK(Throws<std::out_of_range>([&] { pool.DownloadPage(9, &k, &v); }), "bad id throws");
  CHECK(Throws<std::runtime_error>([&] { pool.DownloadPage(0, &k, &v); }), "free page throws");
  CHECK(Throws<std::invalid_argument>([&] { pool.UploadPagesFromCache(cache, {0}); }),
        "uploading a free page throws");
  // tokens appended into the same page in one batch, then freed
  auto r1 = cache.AppendToken(1, Seq(8, 9.0f), Seq(8, 19.0f));
  auto r2 = cache.AppendToken(1, Seq(8, 29.0f), Seq(8, 39.0f));
  pool.UploadTokensFromCache(cache, {r1, r2});
  pool.DownloadPage(b, &k, &v);
  CHECK(k == cache.CopyPageKeys(b), "appended tokens on device");
  pool.MarkPagesFree({a, b});
  pool.DownloadMetadata(&counts, &live);
  CHECK(counts[a] == 0 && live[b] == 0, "freed pages are cleared");
  pool.Reset();
  // direct prompt upload
  dsd::PagedKvCache meta(c, 3, false);
  const auto ids = meta.ReservePagesForRequest(4, {4, 3});
  const auto pk = Seq(7 * 8, 1.0f), pv = Seq(7 * 8, 50.0f);
  pool.UploadPromptDirect(meta, ids, {4, 3}, pk.data(), pv.data());
  pool.DownloadPage(ids[1], &k, &v);
  CHECK(k.size() == 24 && k[0] == pk[32] && v[23] == pv[55], "direct prompt payload");
  pool.PrefillPromptSynthetic(meta, ids, {4, 3}, 4);
  pool.DownloadMetadata(&counts, &live);
  CHECK(counts[ids[0]] == 4 && counts[ids[1]] == 3, "synthetic prefill metadata");
}

// Manual continuous sequence with device page tables: steps, token appends,
// release and LIFO reuse; GPU selection and outputs vs the CPU backend.
void ContinuousSequence() {
  const auto c = Cfg(4, 16, 4, 3);
  const int ept = 64;
  dsd::PagedKvCache cache(c, 64);
  dsd::SparseCudaContext ctx(cache, c, 4, 64, 12, 8, 32);
  dsd::DecodePipeline cpu(c);
  std::vector<dsd::RequestState> reqs;
  for (int r = 0; r < 3; ++r) {
    const int tokens = 9 + 4 * r;
    std::vector<dsd::PageId> pages;
    for (int t = 0; t < tokens; t += 4) {
      const int n = std::min(4, tokens - t);
      pages.push_back(cache.AppendPage(r, dsd::DeterministicTokenVector(n * ept, r, 100 + t, 1),
                                       dsd::DeterministicTokenVector(n * ept, r, 100 + t, 2), n));
    }
    ctx.SyncPagesFromCache(cache, pages);
    ctx.SetRequestPages(r, pages);
    reqs.push_back(dsd::MakeRequestState(r, dsd::DeterministicTokenVector(ept, r, 0, 0), cache, tokens));
  }
  for (int step = 0; step < 9; ++step) {
    std::vector<const dsd::RequestState*> ptrs;
    for (const auto& r : reqs) ptrs.push_back(&r);
    dsd::SparseRunBatchOptions o;
    o.output_mode = dsd::SparseBatchOutputMode::kDebugTensors;
    const auto g = ctx.RunStep(ptrs, o);
    for (std::size_t i = 0; i < reqs.size(); ++i) {
      const auto want = cpu.RunNaiveSparseStep(cache, reqs[i]);
      CHECK(want.selected_page_ids == g.per_request[i].selected_page_ids, "continuous selection");
      CHECK(dsd::MaxAbsDiff(want.output.output, g.per_request[i].output.output) <= 1e-5f,
            "continuous output");
    }
    std::vector<dsd::AppendTokenResult> appended;
    for (auto& r : reqs) {
      const auto k = dsd::DeterministicTokenVector(ept, r.request_id, step, 1);
      const auto v = dsd::DeterministicTokenVector(ept, r.request_id, step, 2);
      const auto res = cache.AppendToken(r.request_id, k, v, step == 0);
      appended.push_back(res);
      if (res.allocated_new_page) ctx.AppendRequestPages(r.request_id, {res.page_id});
      const auto& pages = cache.GetRequestPages(r.request_id);
      r.candidate_page_ids.assign(pages.begin(), pages.end());
      r.query = dsd::DeterministicTokenVector(ept, r.request_id, step + 1, 0);
    }
    ctx.SyncAppendedTokens(cache, appended);
    if (step == 4) {  // release request 1, admit request 7 on the recycled pages
      const auto freed = cache.ReleaseRequest(1);
      ctx.SyncFreedPages(freed);
      ctx.ReleaseRequestPages(1, false);
      std::vector<dsd::PageId> pages;
      for (int t = 0; t < 6; t += 4)
        pages.push_back(cache.AppendPage(7, dsd::DeterministicTokenVector(std::min(4, 6 - t) * ept, 7, t, 5),
                                         dsd::DeterministicTokenVector(std::min(4, 6 - t) * ept, 7, t, 6),
                                         std::min(4, 6 - t)));
      CHECK(pages[0] == freed.back(), "released pages are reused LIFO");
      ctx.SyncPagesFromCache(cache, pages);
      ctx.SetRequestPages(7, pages);
      reqs[1] = dsd::MakeRequestState(7, dsd::DeterministicTokenVector(ept, 7, 0, 0), cache, 6);
    }
  }
}

}  // namespace

int main() {
  if (!dsd::SparseAttentionCudaAvailable()) {
    std::cout << "no sm_100 GPU visible; skipped\n";
    return 0;
  }
  SyntheticCase(Cfg(2, 8, 4, 2), 3, 5, 19, 11, 1e-5f);
  SyntheticCase(Cfg(4, 16, 16, 3), 4, 33, 97, 7, 2e-5f);
  SyntheticCase(Cfg(2, 64, 8, 4), 2, 17, 45, 17, 5e-5f);
  SyntheticCase(Cfg(2, 16, 8, 8), 2, 160, 184, 123, 3e-5f);
  SyntheticCase(Cfg(32, 128, 16, 8), 16, 512, 2048, 7, 1e-4f);
  TopKZero();
  DenseBaseline();
  TieBreak();
  DevicePoolRoundTrip();
  ContinuousSequence();
  std::cout << "sparse GPU C++ API tests passed\n";
  return 0;
}
