// ref_shim.cpp -- flat C entry points over the UNMODIFIED reference CPU code.
//
// TEST INFRASTRUCTURE ONLY.  oracle/Makefile compiles this file together with
// the reference's own CPU sources (page_pool, paged_kv_cache,
// reference_kernels, decode_pipeline, synthetic_data, continuous_batching and
// the CPU stubs of the CUDA contexts) into oracle/_ref/libdsd_ref.so.  It is
// used to pin the restatement in dsd_oracle.cpp and, in `bench.py --impl
// reference`, to time the reference's own sparse_cpu path.

#include <algorithm>
#include <chrono>
#include <cstring>
#include <thread>
#include <vector>

#include "dsd/config.h"
#include "dsd/decode_pipeline.h"
#include "dsd/paged_kv_cache.h"
#include "dsd/reference_kernels.h"
#include "dsd/synthetic_data.h"

namespace {

dsd::ModelConfig MakeConfig(int h, int d, int p, int k) {
  dsd::ModelConfig c;
  c.num_heads = h;
  c.head_dim = d;
  c.page_size = p;
  c.top_k_pages = k;
  return c;
}

struct RefBatch {
  dsd::ModelConfig config;
  dsd::SyntheticBatch batch;
  RefBatch(const dsd::ModelConfig& c, int b, int lo, int hi, int seed)
      : config(c), batch(dsd::BuildSyntheticBatch(c, b, lo, hi, seed)) {}
};

}  // namespace

extern "C" {

// BuildSyntheticBatch (src/synthetic_data.cpp:23-69) kept alive behind a handle.
void* ref_batch_create(int h, int d, int p, int k, int batch, int lo, int hi, int seed) {
  return new RefBatch(MakeConfig(h, d, p, k), batch, lo, hi, seed);
}

void ref_batch_destroy(void* handle) { delete static_cast<RefBatch*>(handle); }

int ref_batch_capacity(void* handle) {
  return static_cast<RefBatch*>(handle)->batch.cache.CapacityPages();
}

int ref_batch_total_candidates(void* handle) {
  int total = 0;
  for (const auto& r : static_cast<RefBatch*>(handle)->batch.requests)
    total += static_cast<int>(r.candidate_page_ids.size());
  return total;
}

// Copies the reference cache out as flat arrays (same layout as the oracle).
void ref_batch_export(void* handle, float* key_pool, float* value_pool, float* summaries,
                      int* token_counts, float* queries, int* cand_offsets, int* cand_ids) {
  auto* rb = static_cast<RefBatch*>(handle);
  const auto& cache = rb->batch.cache;
  std::memcpy(key_pool, cache.KeyPool().data(), cache.KeyPool().size() * sizeof(float));
  std::memcpy(value_pool, cache.ValuePool().data(), cache.ValuePool().size() * sizeof(float));
  std::memcpy(summaries, cache.PageSummaryPool().data(),
              cache.PageSummaryPool().size() * sizeof(float));
  for (const auto& page : cache.Pages()) token_counts[page.id] = page.token_count;
  const int ept = rb->config.num_heads * rb->config.head_dim;
  int c = 0;
  cand_offsets[0] = 0;
  for (std::size_t r = 0; r < rb->batch.requests.size(); ++r) {
    const auto& req = rb->batch.requests[r];
    std::memcpy(queries + r * static_cast<std::size_t>(ept), req.query.data(),
                static_cast<std::size_t>(ept) * sizeof(float));
    for (int id : req.candidate_page_ids) cand_ids[c++] = id;
    cand_offsets[r + 1] = c;
  }
}

// DecodePipeline::RunNaiveSparseStep (src/decode_pipeline.cpp:13-46) for every
// request.  Selected ids are packed by min(k, n) per request.
void ref_batch_sparse_cpu(void* handle, int* selected_out, float* outputs, float* scores_out) {
  auto* rb = static_cast<RefBatch*>(handle);
  dsd::DecodePipeline pipeline(rb->config);
  const int ept = rb->config.num_heads * rb->config.head_dim;
  int s = 0, c = 0;
  for (std::size_t r = 0; r < rb->batch.requests.size(); ++r) {
    const auto res = pipeline.RunNaiveSparseStep(rb->batch.cache, rb->batch.requests[r]);
    for (int id : res.selected_page_ids) selected_out[s++] = id;
    std::memcpy(outputs + r * static_cast<std::size_t>(ept), res.output.output.data(),
                static_cast<std::size_t>(ept) * sizeof(float));
    for (const auto& sc : res.scores) scores_out[c++] = sc.score;
  }
}

// DecodePipeline::RunDenseStep for every request (src/reference_kernels.cpp:196-203).
void ref_batch_dense_cpu(void* handle, float* outputs) {
  auto* rb = static_cast<RefBatch*>(handle);
  dsd::DecodePipeline pipeline(rb->config);
  const int ept = rb->config.num_heads * rb->config.head_dim;
  for (std::size_t r = 0; r < rb->batch.requests.size(); ++r) {
    const auto res = pipeline.RunDenseStep(rb->batch.cache, rb->batch.requests[r]);
    std::memcpy(outputs + r * static_cast<std::size_t>(ept), res.output.data(),
                static_cast<std::size_t>(ept) * sizeof(float));
  }
}

// Times `items` reference decode steps spread over n_threads host threads:
// item i decodes request (i mod batch) of the batch, so a small resident
// sample keeps every thread busy without materialising more requests (the
// reference code is single threaded per request; requests are independent).
// dense = 0: DecodePipeline::RunNaiveSparseStep (sparse_cpu,
// src/decode_pipeline.cpp:13-46); dense = 1: DecodePipeline::RunDenseStep
// (dense_cpu, src/decode_pipeline.cpp:47-51).  Returns the wall ms.
double ref_batch_time_cpu(void* handle, int items, int n_threads, int dense) {
  auto* rb = static_cast<RefBatch*>(handle);
  dsd::DecodePipeline pipeline(rb->config);
  const int batch = static_cast<int>(rb->batch.requests.size());
  n_threads = std::max(1, std::min(n_threads, items));
  const auto t0 = std::chrono::steady_clock::now();
  std::vector<std::thread> pool;
  for (int t = 0; t < n_threads; ++t) {
    pool.emplace_back([&, t]() {
      for (int i = t; i < items; i += n_threads) {
        const auto& req = rb->batch.requests[static_cast<std::size_t>(i % batch)];
        volatile float sink = dense ? pipeline.RunDenseStep(rb->batch.cache, req).output[0]
                                    : pipeline.RunNaiveSparseStep(rb->batch.cache, req)
                                          .output.output[0];
        (void)sink;
      }
    });
  }
  for (auto& th : pool) th.join();
  const auto t1 = std::chrono::steady_clock::now();
  return std::chrono::duration<double, std::milli>(t1 - t0).count();
}

}  // extern "C"
