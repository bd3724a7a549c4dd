// CPU backends of the API (sparse_cpu / dense_cpu).  Operation order follows
// the reference (src/reference_kernels.cpp:13-217): sequential fp32 dot,
// max-subtracted std::exp softmax, weighted V sum in token order.  Build with
// -ffp-contract=off so nothing is fused.
#include "dsd/reference_kernels.h"

#include <algorithm>
#include <cmath>
#include <limits>
#include <stdexcept>

namespace dsd {

namespace {

float SeqDot(const float* a, const float* b, int n) {
  float acc = 0.0f;
  for (int i = 0; i < n; ++i) acc += a[i] * b[i];
  return acc;
}

}  // namespace

RequestState MakeRequestState(int request_id, std::vector<float> query,
                              const PagedKvCache& cache, int context_tokens) {
  RequestState r;
  r.request_id = request_id;
  r.query = std::move(query);
  r.context_tokens = context_tokens;
  const auto& pages = cache.GetRequestPages(request_id);
  r.candidate_page_ids.assign(pages.begin(), pages.end());
  return r;
}

std::vector<PageScore> ScorePagesCpu(const PagedKvCache& cache, const RequestState& request,
                                     const ModelConfig& config) {
  const int ept = config.num_heads * config.head_dim;
  if (static_cast<int>(request.query.size()) != ept)
    throw std::invalid_argument("query length does not match model config");
  const float scale = 1.0f / std::sqrt(static_cast<float>(config.head_dim));
  std::vector<PageScore> out;
  out.reserve(request.candidate_page_ids.size());
  for (PageId id : request.candidate_page_ids) {
    const auto summary = cache.BuildPageSummary(id);
    out.push_back(PageScore{id, SeqDot(request.query.data(), summary.data(), ept) * scale});
  }
  return out;
}

std::vector<PageId> SelectTopKPagesCpu(std::vector<PageScore> scores, int top_k) {
  if (top_k <= 0 || scores.empty()) return {};
  const int k = std::min(top_k, static_cast<int>(scores.size()));
  std::partial_sort(scores.begin(), scores.begin() + k, scores.end(),
                    [](const PageScore& a, const PageScore& b) {
                      return a.score == b.score ? a.page_id < b.page_id : a.score > b.score;
                    });
  std::vector<PageId> ids;
  ids.reserve(static_cast<std::size_t>(k));
  for (int i = 0; i < k; ++i) ids.push_back(scores[static_cast<std::size_t>(i)].page_id);
  return ids;
}

GatheredPages GatherPagesCpu(const PagedKvCache& cache, const std::vector<PageId>& page_ids,
                             const ModelConfig& config) {
  GatheredPages g;
  g.page_ids = page_ids;
  int running = 0;
  for (PageId id : page_ids) {
    const auto& page = cache.GetPage(id);
    g.token_offsets.push_back(running);
    g.token_counts.push_back(page.token_count);
    running += page.token_count;
    const auto k = cache.CopyPageKeys(id);
    const auto v = cache.CopyPageValues(id);
    g.keys.insert(g.keys.end(), k.begin(), k.end());
    g.values.insert(g.values.end(), v.begin(), v.end());
  }
  const std::size_t expect = static_cast<std::size_t>(running) * config.num_heads * config.head_dim;
  if (g.keys.size() != expect || g.values.size() != expect)
    throw std::runtime_error("gather stage produced an inconsistent layout");
  return g;
}

AttentionResult SparseAttentionCpu(const std::vector<float>& query, const GatheredPages& gathered,
                                   const ModelConfig& config) {
  const int ept = config.num_heads * config.head_dim;
  if (static_cast<int>(query.size()) != ept)
    throw std::invalid_argument("query length does not match model config");
  AttentionResult res;
  res.output.assign(static_cast<std::size_t>(ept), 0.0f);
  const int tokens = static_cast<int>(gathered.keys.size() / static_cast<std::size_t>(ept));
  if (tokens == 0) return res;
  const float scale = 1.0f / std::sqrt(static_cast<float>(config.head_dim));
  std::vector<float> logit(static_cast<std::size_t>(tokens)), w(static_cast<std::size_t>(tokens));
  for (int h = 0; h < config.num_heads; ++h) {
    const int hb = h * config.head_dim;
    for (int t = 0; t < tokens; ++t)
      logit[static_cast<std::size_t>(t)] =
          SeqDot(query.data() + hb, gathered.keys.data() + static_cast<std::size_t>(t) * ept + hb,
                 config.head_dim) * scale;
    const float mx = *std::max_element(logit.begin(), logit.end());
    float sum = 0.0f;
    for (int t = 0; t < tokens; ++t) {
      w[static_cast<std::size_t>(t)] = std::exp(logit[static_cast<std::size_t>(t)] - mx);
      sum += w[static_cast<std::size_t>(t)];
    }
    for (float& x : w) x /= sum;
    for (int t = 0; t < tokens; ++t) {
      const float* v = gathered.values.data() + static_cast<std::size_t>(t) * ept + hb;
      for (int d = 0; d < config.head_dim; ++d) res.output[static_cast<std::size_t>(hb + d)] += w[static_cast<std::size_t>(t)] * v[d];
    }
  }
  return res;
}

AttentionResult DenseAttentionCpu(const PagedKvCache& cache, const RequestState& request,
                                  const ModelConfig& config) {
  return SparseAttentionCpu(request.query, GatherPagesCpu(cache, request.candidate_page_ids, config),
                            config);
}

float MaxAbsDiff(const std::vector<float>& lhs, const std::vector<float>& rhs) {
  if (lhs.size() != rhs.size()) return std::numeric_limits<float>::infinity();
  float d = 0.0f;
  for (std::size_t i = 0; i < lhs.size(); ++i) d = std::max(d, std::fabs(lhs[i] - rhs[i]));
  return d;
}

}  // namespace dsd
