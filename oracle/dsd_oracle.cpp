// dsd_oracle.cpp -- CPU restatement of the reference sparse-decode path.
//
// TEST INFRASTRUCTURE ONLY.  This file is the checker the parity tests,
// `__graft_entry__.smoke()` and the `cpu_baseline` leg of `bench.py` compare
// the CUDA path against.  Nothing in the product library links or calls it.
//
// Every function restates one reference function and cites it
// (JudySun233/15-618_Dynamic_Sparse_Decode, paths relative to the repo root).
// The order of floating-point operations is kept identical to the reference,
// so a correct restatement reproduces the reference bit for bit; the
// restatement is pinned against the reference itself (oracle/_ref, built by
// oracle/Makefile) and against the reference tests' known answers.
//
// Build (see oracle/Makefile):  g++ -O2 -std=c++17 -ffp-contract=off -fPIC -shared
// The x86-64 baseline ISA has no FMA, and -ffp-contract=off keeps it that way
// even where the compiler could contract, exactly like the reference Release
// build (no -march=native, no fast-math).

#include <algorithm>
#include <array>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <random>
#include <thread>
#include <vector>

namespace {

struct Cfg {
  int num_heads;
  int head_dim;
  int page_size;
  int top_k_pages;
  int ept() const { return num_heads * head_dim; }
  long long epp() const { return static_cast<long long>(page_size) * ept(); }
};

// Dot: src/reference_kernels.cpp:13-19 (sequential fp32 accumulate).
float Dot(const float* lhs, const float* rhs, int count) {
  float acc = 0.0f;
  for (int i = 0; i < count; ++i) {
    acc += lhs[i] * rhs[i];
  }
  return acc;
}

// Softmax: src/reference_kernels.cpp:21-40 (max-subtract, std::exp, divide).
void Softmax(const std::vector<float>& logits, std::vector<float>* weights) {
  weights->assign(logits.size(), 0.0f);
  if (logits.empty()) return;
  const float max_logit = *std::max_element(logits.begin(), logits.end());
  float sum = 0.0f;
  for (std::size_t i = 0; i < logits.size(); ++i) {
    (*weights)[i] = std::exp(logits[i] - max_logit);
    sum += (*weights)[i];
  }
  for (float& w : *weights) w /= sum;
}

struct Scored {
  int page_id;
  float score;
};

// SelectTopKPagesCpu: src/reference_kernels.cpp:82-107.  Order is score
// descending, ties by lower page id; the first min(k, n) are returned.
void SelectTopK(std::vector<Scored> scores, int top_k, std::vector<int>* out) {
  out->clear();
  if (top_k <= 0 || scores.empty()) return;
  const int k = std::min(top_k, static_cast<int>(scores.size()));
  std::partial_sort(scores.begin(), scores.begin() + k, scores.end(),
                    [](const Scored& a, const Scored& b) {
                      if (a.score == b.score) return a.page_id < b.page_id;
                      return a.score > b.score;
                    });
  for (int i = 0; i < k; ++i) out->push_back(scores[static_cast<std::size_t>(i)].page_id);
}

// GatherPagesCpu + SparseAttentionCpu: src/reference_kernels.cpp:109-194.
// Tokens are visited in selected-page order, then token order in the page;
// per head: logits = dot * scale, softmax, out += w * v (sequential).
void SparseAttention(const Cfg& cfg, const float* query, const float* key_pool,
                     const float* value_pool, const int* token_counts,
                     const std::vector<int>& pages, float* out) {
  const int ept = cfg.ept();
  std::vector<float> keys, values;
  for (int page : pages) {
    const int n = token_counts[page];
    const float* k = key_pool + static_cast<long long>(page) * cfg.epp();
    const float* v = value_pool + static_cast<long long>(page) * cfg.epp();
    keys.insert(keys.end(), k, k + static_cast<long long>(n) * ept);
    values.insert(values.end(), v, v + static_cast<long long>(n) * ept);
  }
  std::fill(out, out + ept, 0.0f);
  const int total_tokens = static_cast<int>(keys.size() / static_cast<std::size_t>(ept));
  if (total_tokens == 0) return;
  const float scale = 1.0f / std::sqrt(static_cast<float>(cfg.head_dim));
  std::vector<float> logits(static_cast<std::size_t>(total_tokens));
  std::vector<float> weights;
  for (int head = 0; head < cfg.num_heads; ++head) {
    const int hb = head * cfg.head_dim;
    for (int t = 0; t < total_tokens; ++t) {
      logits[static_cast<std::size_t>(t)] =
          Dot(query + hb, keys.data() + static_cast<std::size_t>(t) * ept + hb, cfg.head_dim) *
          scale;
    }
    Softmax(logits, &weights);
    for (int t = 0; t < total_tokens; ++t) {
      const float w = weights[static_cast<std::size_t>(t)];
      const float* v = values.data() + static_cast<std::size_t>(t) * ept + hb;
      for (int d = 0; d < cfg.head_dim; ++d) out[hb + d] += w * v[d];
    }
  }
}

// One request of DecodePipeline::RunNaiveSparseStep (src/decode_pipeline.cpp:13-46):
// ScorePagesCpu (src/reference_kernels.cpp:59-80) -> SelectTopKPagesCpu ->
// GatherPagesCpu -> SparseAttentionCpu.  A page whose token_count is 0 scores
// with a zero summary (PagedKvCache::CopyPageSummary, src/paged_kv_cache.cpp:449-456).
void SparseStep(const Cfg& cfg, const float* query, const float* key_pool,
                const float* value_pool, const float* summaries, const int* token_counts,
                const int* cand, int n_cand, int* sel_out, float* out, float* scores_out) {
  const int ept = cfg.ept();
  const float scale = 1.0f / std::sqrt(static_cast<float>(cfg.head_dim));
  std::vector<Scored> scores;
  scores.reserve(static_cast<std::size_t>(n_cand));
  std::vector<float> zero(static_cast<std::size_t>(ept), 0.0f);
  for (int c = 0; c < n_cand; ++c) {
    const int page = cand[c];
    const float* s = token_counts[page] == 0
                         ? zero.data()
                         : summaries + static_cast<long long>(page) * ept;
    const float score = Dot(query, s, ept) * scale;
    scores.push_back(Scored{page, score});
    if (scores_out) scores_out[c] = score;
  }
  std::vector<int> selected;
  SelectTopK(scores, cfg.top_k_pages, &selected);
  for (std::size_t i = 0; i < selected.size(); ++i) sel_out[i] = selected[i];
  SparseAttention(cfg, query, key_pool, value_pool, token_counts, selected, out);
}

// std::uniform_real_distribution<float>(-1, 1) over std::mt19937, as used by
// RandomVector (src/synthetic_data.cpp:12-19, src/continuous_batching.cpp:35-42).
void RandomFill(float* dst, long long count, std::mt19937& rng) {
  std::uniform_real_distribution<float> dist(-1.0f, 1.0f);
  for (long long i = 0; i < count; ++i) dst[i] = dist(rng);
}

// MixSeed: src/continuous_batching.cpp:44-50.
std::uint32_t MixSeed(int request_id, int decode_step, int stream) {
  std::uint32_t x = 0x9e3779b9u;
  x ^= static_cast<std::uint32_t>(request_id + 0x85ebca6b) + (x << 6) + (x >> 2);
  x ^= static_cast<std::uint32_t>(decode_step + 0xc2b2ae35) + (x << 6) + (x >> 2);
  x ^= static_cast<std::uint32_t>(stream + 0x27d4eb2f) + (x << 6) + (x >> 2);
  return x;
}

// Counter-based normal generator used for the long-context workloads that
// are generated on the device (no reference counterpart: the reference
// materialises everything on the host with mt19937).  Restated here so the
// device generator can be checked bit for bit.  Irwin-Hall(4) over 16-bit
// uniforms: integer sum (exact), one float conversion, one multiply.
inline std::uint64_t Mix64(std::uint64_t z) {
  z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ULL;
  z = (z ^ (z >> 27)) * 0x94d049bb133111ebULL;
  return z ^ (z >> 31);
}

}  // namespace

extern "C" {

// -------- summaries (PagedKvCache formulas) -----------------------------------

// PagedKvCache::AppendPage summary: src/paged_kv_cache.cpp:88-99.
// sum_t k[t][i] in token order, then * (1.0f / token_count).
void orc_page_summary(const float* keys, int token_count, int ept, float* out) {
  for (int i = 0; i < ept; ++i) out[i] = 0.0f;
  for (int t = 0; t < token_count; ++t)
    for (int i = 0; i < ept; ++i) out[i] += keys[static_cast<long long>(t) * ept + i];
  const float inv = 1.0f / static_cast<float>(token_count);
  for (int i = 0; i < ept; ++i) out[i] *= inv;
}

// PagedKvCache::AppendToken running mean: src/paged_kv_cache.cpp:231-238.
void orc_running_mean_append(float* summary, const float* key, int old_count, int ept) {
  const float old_c = static_cast<float>(old_count);
  const float new_c = old_c + 1.0f;
  for (int i = 0; i < ept; ++i) summary[i] = (summary[i] * old_c + key[i]) / new_c;
}

// -------- the decode step ------------------------------------------------------

// Batched sparse decode exactly as sparse_cpu runs it (RunNaiveSparseBatch,
// src/decode_pipeline.cpp:90-107), one request after another.
// Pools: keys/values [capacity][page_size][H*D], summaries [capacity][H*D].
// Candidates in CSR (cand_offsets[B+1], cand_ids).  Selected ids are written
// at sel_offsets[r] = sum_{j<r} min(k, n_j).  scores_out (nullable) is [C].
// n_threads > 1 runs independent requests on that many host threads.
void orc_sparse_decode(int num_heads, int head_dim, int page_size, int top_k,
                       const float* key_pool, const float* value_pool,
                       const float* summaries, const int* token_counts, int batch,
                       const float* queries, const int* cand_offsets, const int* cand_ids,
                       int* selected_out, float* outputs, float* scores_out,
                       int n_threads) {
  const Cfg cfg{num_heads, head_dim, page_size, top_k};
  std::vector<int> sel_off(static_cast<std::size_t>(batch) + 1, 0);
  for (int r = 0; r < batch; ++r) {
    const int n = cand_offsets[r + 1] - cand_offsets[r];
    sel_off[r + 1] = sel_off[r] + std::max(0, std::min(top_k, n));
  }
  auto run = [&](int r) {
    const int b = cand_offsets[r];
    SparseStep(cfg, queries + static_cast<long long>(r) * cfg.ept(), key_pool, value_pool,
               summaries, token_counts, cand_ids + b, cand_offsets[r + 1] - b,
               selected_out + sel_off[r], outputs + static_cast<long long>(r) * cfg.ept(),
               scores_out ? scores_out + b : nullptr);
  };
  if (n_threads <= 1) {
    for (int r = 0; r < batch; ++r) run(r);
    return;
  }
  std::vector<std::thread> pool;
  for (int t = 0; t < n_threads; ++t) {
    pool.emplace_back([&, t]() {
      for (int r = t; r < batch; r += n_threads) run(r);
    });
  }
  for (auto& th : pool) th.join();
}

// DenseAttentionCpu: src/reference_kernels.cpp:196-203 (all candidates, in order).
void orc_dense_decode(int num_heads, int head_dim, int page_size, const float* key_pool,
                      const float* value_pool, const int* token_counts, int batch,
                      const float* queries, const int* cand_offsets, const int* cand_ids,
                      float* outputs) {
  const Cfg cfg{num_heads, head_dim, page_size, 0};
  for (int r = 0; r < batch; ++r) {
    std::vector<int> pages(cand_ids + cand_offsets[r], cand_ids + cand_offsets[r + 1]);
    SparseAttention(cfg, queries + static_cast<long long>(r) * cfg.ept(), key_pool, value_pool,
                    token_counts, pages, outputs + static_cast<long long>(r) * cfg.ept());
  }
}

// -------- inputs -----------------------------------------------------------------

// BuildSyntheticBatch, phase 1: src/synthetic_data.cpp:23-41.  All context
// lengths are drawn first.  Returns the total page count (= cache capacity).
int orc_synthetic_batch_contexts(int page_size, int batch, int min_ctx, int max_ctx, int seed,
                                 int* context_tokens) {
  std::mt19937 rng(static_cast<std::uint32_t>(seed));
  std::uniform_int_distribution<int> dist(min_ctx, max_ctx);
  int total = 0;
  for (int r = 0; r < batch; ++r) {
    context_tokens[r] = dist(rng);
    total += (context_tokens[r] + page_size - 1) / page_size;
  }
  return total;
}

// BuildSyntheticBatch, phase 2: src/synthetic_data.cpp:43-69.  Per request,
// per page: keys then values, then the query, all U(-1,1) from the same
// mt19937 stream.  Pages come from a PagePool of capacity = total pages whose
// free list pops from the back (src/page_pool.cpp:36-45, :122-128), so the
// first page gets id capacity-1.  Summaries follow AppendPage.
// Outputs: key_pool/value_pool [cap][P][E] (zero-filled by the caller),
// summaries [cap][E], token_counts [cap], queries [B][E],
// cand_offsets [B+1], cand_ids [cap].
void orc_synthetic_batch_fill(int num_heads, int head_dim, int page_size, int batch,
                              int min_ctx, int max_ctx, int seed, float* key_pool,
                              float* value_pool, float* summaries, int* token_counts,
                              float* queries, int* cand_offsets, int* cand_ids) {
  const Cfg cfg{num_heads, head_dim, page_size, 0};
  const int ept = cfg.ept();
  std::mt19937 rng(static_cast<std::uint32_t>(seed));
  std::uniform_int_distribution<int> dist(min_ctx, max_ctx);
  std::vector<int> ctx(static_cast<std::size_t>(batch));
  int capacity = 0;
  for (int r = 0; r < batch; ++r) {
    ctx[static_cast<std::size_t>(r)] = dist(rng);
    capacity += (ctx[static_cast<std::size_t>(r)] + page_size - 1) / page_size;
  }
  for (int p = 0; p < capacity; ++p) token_counts[p] = 0;
  int next_free = capacity - 1;
  int c = 0;
  cand_offsets[0] = 0;
  for (int r = 0; r < batch; ++r) {
    const int tokens = ctx[static_cast<std::size_t>(r)];
    const int pages = (tokens + page_size - 1) / page_size;
    for (int p = 0; p < pages; ++p) {
      const int n = std::min(page_size, tokens - p * page_size);
      const int id = next_free--;
      float* k = key_pool + static_cast<long long>(id) * cfg.epp();
      float* v = value_pool + static_cast<long long>(id) * cfg.epp();
      RandomFill(k, static_cast<long long>(n) * ept, rng);
      RandomFill(v, static_cast<long long>(n) * ept, rng);
      orc_page_summary(k, n, ept, summaries + static_cast<long long>(id) * ept);
      token_counts[id] = n;
      cand_ids[c++] = id;
    }
    RandomFill(queries + static_cast<long long>(r) * ept, ept, rng);
    cand_offsets[r + 1] = c;
  }
}

// DeterministicTokenVector: src/continuous_batching.cpp:52-59.
void orc_deterministic_token_vector(int count, int request_id, int decode_step, int stream,
                                    float* out) {
  std::mt19937 rng(MixSeed(request_id, decode_step, stream));
  RandomFill(out, count, rng);
}

// BuildSyntheticContinuousWorkload spec draws: src/continuous_batching.cpp:336-381.
// The payloads are drawn from the same stream between the integer draws, so
// they are generated (into a scratch buffer) to keep the stream aligned.
// Writes request_id, arrival_step, prompt_tokens, decode_steps per request in
// the reference's final (arrival, id) order.  When prompt_keys/prompt_values/
// initial_queries are non-null they receive the payloads in that same order,
// packed: prompts back to back ([sum prompt_tokens][E]) and queries [N][E].
void orc_continuous_workload(int num_heads, int head_dim, int num_requests, int arrival_window,
                             int min_prompt, int max_prompt, int min_decode, int max_decode,
                             int seed, int* request_ids, int* arrival_steps,
                             int* prompt_tokens, int* decode_steps, float* prompt_keys,
                             float* prompt_values, float* initial_queries) {
  const int ept = num_heads * head_dim;
  std::mt19937 rng(static_cast<std::uint32_t>(seed));
  std::uniform_int_distribution<int> arrival_dist(0, std::max(0, arrival_window));
  std::uniform_int_distribution<int> prompt_dist(min_prompt, max_prompt);
  std::uniform_int_distribution<int> decode_dist(min_decode, max_decode);
  struct Spec {
    int id, arrival, prompt, decode;
    std::vector<float> k, v, q;
  };
  const bool keep = prompt_keys != nullptr;
  std::vector<Spec> specs;
  std::vector<float> scratch;
  for (int r = 0; r < num_requests; ++r) {
    Spec s;
    s.id = r;
    s.arrival = arrival_dist(rng);
    s.prompt = prompt_dist(rng);
    s.decode = decode_dist(rng);
    const long long n = static_cast<long long>(s.prompt) * ept;
    if (keep) {
      s.k.resize(static_cast<std::size_t>(n));
      s.v.resize(static_cast<std::size_t>(n));
      s.q.resize(static_cast<std::size_t>(ept));
      RandomFill(s.k.data(), n, rng);
      RandomFill(s.v.data(), n, rng);
      RandomFill(s.q.data(), ept, rng);
    } else {
      scratch.resize(static_cast<std::size_t>(std::max<long long>(n, ept)));
      RandomFill(scratch.data(), n, rng);
      RandomFill(scratch.data(), n, rng);
      RandomFill(scratch.data(), ept, rng);
    }
    specs.push_back(std::move(s));
  }
  std::stable_sort(specs.begin(), specs.end(), [](const Spec& a, const Spec& b) {
    if (a.arrival == b.arrival) return a.id < b.id;
    return a.arrival < b.arrival;
  });
  long long off = 0;
  for (int i = 0; i < num_requests; ++i) {
    const Spec& s = specs[static_cast<std::size_t>(i)];
    request_ids[i] = s.id;
    arrival_steps[i] = s.arrival;
    prompt_tokens[i] = s.prompt;
    decode_steps[i] = s.decode;
    if (keep) {
      std::memcpy(prompt_keys + off, s.k.data(), s.k.size() * sizeof(float));
      std::memcpy(prompt_values + off, s.v.data(), s.v.size() * sizeof(float));
      std::memcpy(initial_queries + static_cast<long long>(i) * ept, s.q.data(),
                  s.q.size() * sizeof(float));
      off += static_cast<long long>(s.k.size());
    }
  }
}

// Spec draws without payloads: the lengths-only generator this build uses
// where prompt payloads cannot be held on the host (BuildSyntheticContinuousSpecs
// of the C++ API; no reference counterpart -- the reference always draws the
// payloads, so its lengths at the same seed differ).  mt19937(seed), per
// request arrival in [0, window], prompt and decode lengths, nothing else;
// sorted by (arrival, id).
void orc_continuous_specs_only(int num_requests, int arrival_window, int min_prompt,
                               int max_prompt, int min_decode, int max_decode, int seed,
                               int* request_ids, int* arrival_steps, int* prompt_tokens,
                               int* decode_steps) {
  std::mt19937 rng(static_cast<std::uint32_t>(seed));
  std::uniform_int_distribution<int> arrival_dist(0, std::max(0, arrival_window));
  std::uniform_int_distribution<int> prompt_dist(min_prompt, max_prompt);
  std::uniform_int_distribution<int> decode_dist(min_decode, max_decode);
  std::vector<std::array<int, 4>> specs;
  for (int r = 0; r < num_requests; ++r) {
    const int a = arrival_dist(rng);
    const int p = prompt_dist(rng);
    const int d = decode_dist(rng);
    specs.push_back({a, r, p, d});
  }
  std::stable_sort(specs.begin(), specs.end(), [](const auto& x, const auto& y) {
    return x[0] == y[0] ? x[1] < y[1] : x[0] < y[0];
  });
  for (int i = 0; i < num_requests; ++i) {
    arrival_steps[i] = specs[static_cast<std::size_t>(i)][0];
    request_ids[i] = specs[static_cast<std::size_t>(i)][1];
    prompt_tokens[i] = specs[static_cast<std::size_t>(i)][2];
    decode_steps[i] = specs[static_cast<std::size_t>(i)][3];
  }
}

// Device workload generator restatement (see Mix64 above).  Element `index`
// of stream (seed, kind) where kind 0 = query, 1 = key, 2 = value.
float orc_normal_value(std::uint64_t seed, int kind, std::uint64_t index) {
  const std::uint64_t h =
      Mix64(index ^ Mix64(seed * 0x9e3779b97f4a7c15ULL + static_cast<std::uint64_t>(kind)));
  const int sum = static_cast<int>(h & 0xffff) + static_cast<int>((h >> 16) & 0xffff) +
                  static_cast<int>((h >> 32) & 0xffff) + static_cast<int>((h >> 48) & 0xffff);
  return static_cast<float>(sum - 131070) * 2.6429e-5f;
}

void orc_normal_fill(std::uint64_t seed, int kind, std::uint64_t first_index, long long count,
                     float* out) {
  for (long long i = 0; i < count; ++i)
    out[i] = orc_normal_value(seed, kind, first_index + static_cast<std::uint64_t>(i));
}

// SyntheticPromptValue / SyntheticDecodeValue of the reference's GPU
// admission mode 2 (src/device_page_pool.cpp:102-138): boost-style hash
// combine of the indices, 32-bit finaliser, (x % 2001 - 1000) / 1000.
static std::uint32_t HashCombine(std::uint32_t x, int v, std::uint32_t salt) {
  return x ^ (static_cast<std::uint32_t>(v + static_cast<int>(salt)) + (x << 6) + (x >> 2));
}
static float HashUnit(std::uint32_t x) {
  x ^= x >> 16;
  x *= 0x7feb352du;
  x ^= x >> 15;
  x *= 0x846ca68bu;
  x ^= x >> 16;
  return static_cast<float>(static_cast<int>(x % 2001u) - 1000) / 1000.0f;
}

// tokens [0, n) of prompt page `page_idx` of `request`, stream 1 = key, 2 = value
void orc_synthetic_prompt_fill(int request, int page_idx, int n, int ept, int stream, float* out) {
  for (int t = 0; t < n; ++t)
    for (int e = 0; e < ept; ++e) {
      std::uint32_t x = 0x9e3779b9u;
      x = HashCombine(x, request, 0x85ebca6bu);
      x = HashCombine(x, page_idx, 0xc2b2ae35u);
      x = HashCombine(x, t, 0x27d4eb2fu);
      x = HashCombine(x, e, 0x165667b1u);
      x = HashCombine(x, stream, 0xd3a2646cu);
      out[static_cast<long long>(t) * ept + e] = HashUnit(x);
    }
}

void orc_synthetic_decode_fill(int request, int step, int ept, int stream, float* out) {
  for (int e = 0; e < ept; ++e) {
    std::uint32_t x = 0x9e3779b9u;
    x = HashCombine(x, request, 0x85ebca6bu);
    x = HashCombine(x, step, 0xc2b2ae35u);
    x = HashCombine(x, e, 0x165667b1u);
    x = HashCombine(x, stream, 0xd3a2646cu);
    out[e] = HashUnit(x);
  }
}

}  // extern "C"
