// BuildSyntheticBatch (reference: src/synthetic_data.cpp:23-69).  The draw
// order is part of the input contract: all context lengths first, then per
// request per page keys then values, then the query.
#include "dsd/synthetic_data.h"

#include <algorithm>
#include <random>

#include "dsd/reference_kernels.h"

namespace dsd {

namespace {
std::vector<float> Uniform(int count, std::mt19937& rng) {
  std::uniform_real_distribution<float> dist(-1.0f, 1.0f);
  std::vector<float> v(static_cast<std::size_t>(count));
  for (float& x : v) x = dist(rng);
  return v;
}
}  // namespace

SyntheticBatch BuildSyntheticBatch(const ModelConfig& config, int batch_size,
                                   int min_context_tokens, int max_context_tokens, int seed) {
  std::mt19937 rng(static_cast<std::uint32_t>(seed));
  std::uniform_int_distribution<int> ctx_dist(min_context_tokens, max_context_tokens);
  std::vector<int> ctx(static_cast<std::size_t>(batch_size));
  int pages = 0;
  for (int& c : ctx) {
    c = ctx_dist(rng);
    pages += (c + config.page_size - 1) / config.page_size;
  }
  SyntheticBatch batch(config, pages);
  const int ept = config.num_heads * config.head_dim;
  for (int r = 0; r < batch_size; ++r) {
    const int tokens = ctx[static_cast<std::size_t>(r)];
    const int n_pages = (tokens + config.page_size - 1) / config.page_size;
    for (int p = 0; p < n_pages; ++p) {
      const int n = std::min(config.page_size, tokens - p * config.page_size);
      const auto k = Uniform(n * ept, rng);
      const auto v = Uniform(n * ept, rng);
      batch.cache.AppendPage(r, k, v, n);
    }
    batch.requests.push_back(MakeRequestState(r, Uniform(ept, rng), batch.cache, tokens));
  }
  return batch;
}

}  // namespace dsd
