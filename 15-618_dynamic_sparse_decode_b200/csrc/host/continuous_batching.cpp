// Continuous-batching sparse decode (reference: src/continuous_batching.cpp:336-1039).
// The loop, admission policy and statistics follow the reference.  What
// changes: with device_page_tables (the default) each request's page list
// lives on the GPU -- set at admission, extended by the token-append upload
// when a token opens a new page, dropped at release -- so a step uploads only
// the queries, and the host no longer re-packs every candidate id per step.
#include "dsd/continuous_batching.h"

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdint>
#include <deque>
#include <numeric>
#include <random>
#include <stdexcept>
#include <atomic>
#include <condition_variable>
#include <functional>
#include <mutex>
#include <thread>
#include <unordered_set>

#include "capi_error.h"
#include "worker_pool.h"
#include "dsd_b200.h"
#include "dsd/paged_kv_cache.h"
#include "dsd/reference_kernels.h"

namespace dsd {

namespace {

using Clock = std::chrono::steady_clock;

double Ms(Clock::time_point a, Clock::time_point b) {
  return std::chrono::duration<double, std::milli>(b - a).count();
}

int Ept(const ModelConfig& c) { return c.num_heads * c.head_dim; }

int PagesFor(const ModelConfig& c, int tokens) {
  return tokens <= 0 ? 0 : (tokens + c.page_size - 1) / c.page_size;
}

void FillUniform(float* dst, std::size_t n, std::mt19937& rng) {
  std::uniform_real_distribution<float> dist(-1.0f, 1.0f);
  for (std::size_t i = 0; i < n; ++i) dst[i] = dist(rng);
}

// MixSeed (src/continuous_batching.cpp:44-50): combine (request, step, stream).
std::uint32_t MixSeed(int request_id, int decode_step, int stream) {
  std::uint32_t x = 0x9e3779b9u;
  x ^= static_cast<std::uint32_t>(request_id + 0x85ebca6b) + (x << 6) + (x >> 2);
  x ^= static_cast<std::uint32_t>(decode_step + 0xc2b2ae35) + (x << 6) + (x >> 2);
  x ^= static_cast<std::uint32_t>(stream + 0x27d4eb2f) + (x << 6) + (x >> 2);
  return x;
}

std::vector<ContinuousRequestSpec> BuildSpecs(const ModelConfig& config, int num_requests,
                                              int arrival_window, int min_prompt, int max_prompt,
                                              int min_decode, int max_decode, int seed,
                                              bool payloads) {
  if (num_requests < 0 || arrival_window < 0 || min_prompt < 0 || max_prompt < min_prompt ||
      min_decode < 0 || max_decode < min_decode)
    throw std::invalid_argument("invalid continuous workload parameters");
  std::mt19937 rng(static_cast<std::uint32_t>(seed));
  std::uniform_int_distribution<int> arrival(0, std::max(0, arrival_window));
  std::uniform_int_distribution<int> prompt(min_prompt, max_prompt);
  std::uniform_int_distribution<int> decode(min_decode, max_decode);
  const int ept = Ept(config);
  std::vector<ContinuousRequestSpec> specs;
  specs.reserve(static_cast<std::size_t>(num_requests));
  for (int r = 0; r < num_requests; ++r) {
    ContinuousRequestSpec s;
    s.request_id = r;
    s.arrival_step = arrival(rng);
    s.prompt_tokens = prompt(rng);
    s.decode_steps = decode(rng);
    s.initial_query.resize(static_cast<std::size_t>(ept));
    if (payloads) {
      const std::size_t n = static_cast<std::size_t>(s.prompt_tokens) * ept;
      s.prompt_keys.resize(n);
      s.prompt_values.resize(n);
      FillUniform(s.prompt_keys.data(), n, rng);
      FillUniform(s.prompt_values.data(), n, rng);
      FillUniform(s.initial_query.data(), s.initial_query.size(), rng);
    } else {
      std::mt19937 qrng(MixSeed(r, 0, 0));
      FillUniform(s.initial_query.data(), s.initial_query.size(), qrng);
    }
    specs.push_back(std::move(s));
  }
  std::sort(specs.begin(), specs.end(), [](const ContinuousRequestSpec& a,
                                           const ContinuousRequestSpec& b) {
    return a.arrival_step == b.arrival_step ? a.request_id < b.request_id
                                            : a.arrival_step < b.arrival_step;
  });
  return specs;
}

double Percentile(std::vector<double> v, double p) {
  if (v.empty()) return 0.0;
  std::sort(v.begin(), v.end());
  const double pos = p * static_cast<double>(v.size() - 1);
  const auto lo = static_cast<std::size_t>(std::floor(pos));
  const auto hi = static_cast<std::size_t>(std::ceil(pos));
  if (lo == hi) return v[lo];
  const double f = pos - static_cast<double>(lo);
  return v[lo] * (1.0 - f) + v[hi] * f;
}

void Add(StageTimings* d, const StageTimings& s) {
  d->page_scoring_ms += s.page_scoring_ms;
  d->topk_ms += s.topk_ms;
  d->gather_ms += s.gather_ms;
  d->attention_ms += s.attention_ms;
  d->total_ms += s.total_ms;
}

void Add(RuntimeOverheadTimings* d, const RuntimeOverheadTimings& s) {
  d->time_malloc_ms += s.time_malloc_ms;
  d->time_memcpy_h2d_ms += s.time_memcpy_h2d_ms;
  d->time_memcpy_d2h_ms += s.time_memcpy_d2h_ms;
  d->time_free_ms += s.time_free_ms;
  d->time_kernel_launch_ms += s.time_kernel_launch_ms;
  d->time_sync_ms += s.time_sync_ms;
  d->time_prepare_sparse_layout_ms += s.time_prepare_sparse_layout_ms;
}

void Validate(const ModelConfig& config, const ContinuousRequestSpec& s, bool need_payload) {
  if (s.request_id < 0) throw std::invalid_argument("request_id must be non-negative");
  if (s.arrival_step < 0 || s.prompt_tokens < 0 || s.decode_steps < 0)
    throw std::invalid_argument("continuous request counts must be non-negative");
  const std::size_t n = static_cast<std::size_t>(s.prompt_tokens) * Ept(config);
  if (need_payload && (s.prompt_keys.size() != n || s.prompt_values.size() != n))
    throw std::invalid_argument("prompt payload size does not match prompt_tokens");
  if (static_cast<int>(s.initial_query.size()) != Ept(config))
    throw std::invalid_argument("initial query size does not match model config");
}

std::vector<int> PromptCounts(const ModelConfig& c, int prompt_tokens) {
  std::vector<int> counts;
  for (int t = 0; t < prompt_tokens; t += c.page_size) counts.push_back(std::min(c.page_size, prompt_tokens - t));
  return counts;
}

// Admission (reference AdmitPrompt, :208-239) plus the device page table.
void Admit(const ModelConfig& config, const ContinuousRequestSpec& spec,
           ContinuousPromptAdmissionMode mode, PagedKvCache* cache, SparseCudaContext* ctx,
           bool tables) {
  std::vector<PageId> pages;
  if (mode == ContinuousPromptAdmissionMode::kCpuCache) {
    const int ept = Ept(config);
    for (int t = 0; t < spec.prompt_tokens; t += config.page_size) {
      const int n = std::min(config.page_size, spec.prompt_tokens - t);
      const bool tail = t + n == spec.prompt_tokens;
      // the reference computes the summary only for a partial tail page that
      // decode tokens will be appended into (:181-186)
      const bool summary = tail && n < config.page_size && spec.decode_steps > 0;
      pages.push_back(cache->AppendPage(spec.request_id,
                                        spec.prompt_keys.data() + static_cast<std::size_t>(t) * ept,
                                        spec.prompt_values.data() + static_cast<std::size_t>(t) * ept,
                                        n, summary));
    }
    ctx->SyncPagesFromCache(*cache, pages);
  } else {
    const auto counts = PromptCounts(config, spec.prompt_tokens);
    pages = cache->ReservePagesForRequest(spec.request_id, counts);
    if (mode == ContinuousPromptAdmissionMode::kDirectGpuUpload) {
      ctx->SyncPromptDirect(*cache, pages, counts, spec.prompt_keys.data(),
                            spec.prompt_values.data());
    } else {
      ctx->PrefillPromptSynthetic(*cache, pages, counts, spec.request_id);
    }
  }
  if (tables) ctx->SetRequestPages(spec.request_id, pages);
}

}  // namespace

std::vector<float> DeterministicTokenVector(int count, int request_id, int decode_step,
                                            int stream) {
  std::mt19937 rng(MixSeed(request_id, decode_step, stream));
  std::vector<float> v(static_cast<std::size_t>(count));
  FillUniform(v.data(), v.size(), rng);
  return v;
}

std::vector<ContinuousRequestSpec> BuildSyntheticContinuousWorkload(
    const ModelConfig& config, int num_requests, int arrival_window, int min_prompt_tokens,
    int max_prompt_tokens, int min_decode_steps, int max_decode_steps, int seed) {
  return BuildSpecs(config, num_requests, arrival_window, min_prompt_tokens, max_prompt_tokens,
                    min_decode_steps, max_decode_steps, seed, true);
}

std::vector<ContinuousRequestSpec> BuildSyntheticContinuousSpecs(
    const ModelConfig& config, int num_requests, int arrival_window, int min_prompt_tokens,
    int max_prompt_tokens, int min_decode_steps, int max_decode_steps, int seed) {
  return BuildSpecs(config, num_requests, arrival_window, min_prompt_tokens, max_prompt_tokens,
                    min_decode_steps, max_decode_steps, seed, false);
}

ContinuousBatchStats RunContinuousSparseDecode(const ModelConfig& config,
                                               const std::vector<ContinuousRequestSpec>& requests,
                                               int max_active_requests) {
  ContinuousDecodeOptions o;
  o.max_active_requests = max_active_requests;
  return RunContinuousSparseDecode(config, requests, o);
}

namespace {
ContinuousBatchStats RunContinuous(const ModelConfig& config,
                                   const std::vector<ContinuousRequestSpec>& specs,
                                   const ContinuousDecodeOptions& options, bool dense);
}  // namespace

ContinuousBatchStats RunContinuousSparseDecode(const ModelConfig& config,
                                               const std::vector<ContinuousRequestSpec>& specs,
                                               const ContinuousDecodeOptions& options) {
  return RunContinuous(config, specs, options, false);
}

namespace {

// The serving loop of both backends; `dense` attends over every page of each
// active request (the dense GPU baseline) instead of the top-k pages.
ContinuousBatchStats RunContinuous(const ModelConfig& config,
                                   const std::vector<ContinuousRequestSpec>& specs,
                                   const ContinuousDecodeOptions& options, bool dense) {
  using Mode = ContinuousPromptAdmissionMode;
  if (options.max_active_requests <= 0)
    throw std::invalid_argument("max_active_requests must be positive");
  if (!SparseAttentionCudaAvailable())
    throw std::runtime_error("continuous sparse decode requires a visible sm_100 GPU");
  if (options.gpu_synthetic_decode_append && options.prompt_admission_mode == Mode::kCpuCache)
    throw std::invalid_argument(
        "gpu_synthetic_decode_append requires a GPU-resident prompt admission mode");
  const bool need_payload = options.prompt_admission_mode != Mode::kSyntheticGpuPrefill;
  std::unordered_set<int> seen;
  for (const auto& s : specs) {
    Validate(config, s, need_payload);
    if (!seen.insert(s.request_id).second)
      throw std::invalid_argument("continuous workload request_id values must be unique");
  }

  int total_pages = 0, max_pages = 1;
  for (const auto& s : specs) {
    const int p = PagesFor(config, s.prompt_tokens) + PagesFor(config, std::max(0, s.decode_steps));
    total_pages += p;
    max_pages = std::max(max_pages, p);
  }
  total_pages = std::max(total_pages, 1);
  const int window = std::max(1, options.max_active_requests * max_pages);
  const int capacity = options.preadmit_prompts ? total_pages : std::min(total_pages, window);
  const int max_cand = options.max_active_requests * max_pages;
  const int max_sel =
      dense ? max_cand : options.max_active_requests * std::min(config.top_k_pages, max_pages);
  const bool metadata_only = options.prompt_admission_mode != Mode::kCpuCache;
  const bool tables = options.device_page_tables;
  const int table_slots = options.preadmit_prompts ? static_cast<int>(specs.size())
                                                   : options.max_active_requests;

  PagedKvCache cache(config, capacity, !metadata_only);
  SparseCudaContext ctx(cache, config, options.max_active_requests, max_cand, max_sel,
                        tables ? std::max(1, table_slots) : 0, tables ? max_pages : 0,
                        options.device, options.kv_format);
  if (dense) detail::ThrowIf(dsd_set_attention_mode(ctx.handle(), 1));
  ctx.ResetDeviceTransferStats();
  const int ept = Ept(config);

  ContinuousBatchStats stats;
  // precomputed decode payloads: next queries and (unless appended on the GPU) K/V
  std::vector<std::vector<float>> pre_q, pre_k, pre_v;
  if (options.precompute_decode_payloads) {
    const auto t0 = Clock::now();
    pre_q.resize(specs.size());
    if (!options.gpu_synthetic_decode_append) {
      pre_k.resize(specs.size());
      pre_v.resize(specs.size());
    }
    for (std::size_t i = 0; i < specs.size(); ++i) {
      for (int d = 0; d < specs[i].decode_steps; ++d) {
        auto q = DeterministicTokenVector(ept, specs[i].request_id, d + 1, 0);
        pre_q[i].insert(pre_q[i].end(), q.begin(), q.end());
        if (!options.gpu_synthetic_decode_append) {
          auto k = DeterministicTokenVector(ept, specs[i].request_id, d, 1);
          auto v = DeterministicTokenVector(ept, specs[i].request_id, d, 2);
          pre_k[i].insert(pre_k[i].end(), k.begin(), k.end());
          pre_v[i].insert(pre_v[i].end(), v.begin(), v.end());
        }
      }
    }
    stats.decode_payload_prep_ms = Ms(t0, Clock::now());
  }

  std::vector<double> step_ms;
  StageTimings timings_sum;
  RuntimeOverheadTimings overhead_sum;
  int nonempty = 0, active_sum = 0;
  std::deque<std::size_t> pending;
  std::vector<ActiveDecodeRequest> active;
  active.reserve(static_cast<std::size_t>(options.max_active_requests));
  std::vector<const RequestState*> batch;
  std::vector<const float*> query_rows;
  std::vector<std::uint8_t> admitted(specs.size(), 0);

  if (options.preadmit_prompts) {
    for (std::size_t i = 0; i < specs.size(); ++i) {
      const auto t0 = Clock::now();
      Admit(config, specs[i], options.prompt_admission_mode, &cache, &ctx, tables);
      const double ms = Ms(t0, Clock::now());
      stats.admission_ms += ms;
      stats.prompt_preadmit_ms += ms;
      admitted[i] = 1;
    }
    stats.admission_device_transfer_stats = ctx.DeviceTransfers();
    ctx.ResetDeviceTransferStats();
  }

  SparseRunBatchOptions run_opts;
  run_opts.output_mode = options.run_batch_output_mode;
  run_opts.timing_mode = options.run_batch_timing_mode;

  std::size_t next = 0;
  int step = 0;
  std::deque<Clock::time_point> step_starts;
  // Waits for the oldest queued step; its wall time runs from its BeginStep
  // to the moment its results are back on the host.
  // step records awaiting their results (step_observer only)
  std::deque<ContinuousStepRecord> records;
  int step_index = 0;
  auto record_step = [&]() {
    if (!options.step_observer) return;
    ContinuousStepRecord rec;
    rec.step_index = step_index;
    for (const auto& a : active) {
      rec.request_ids.push_back(a.state.request_id);
      rec.context_tokens.push_back(a.state.context_tokens);
      rec.candidate_page_ids.push_back(a.state.candidate_page_ids);
      rec.queries.push_back(a.query_row ? std::vector<float>(a.query_row, a.query_row + ept)
                                        : a.state.query);
    }
    records.push_back(std::move(rec));
  };
  auto observe = [&](const SparseBatchCudaResult& out) {
    if (!options.step_observer) return;
    records.front().result = &out;
    options.step_observer(records.front());
    records.pop_front();
  };
  auto finish_oldest = [&]() {
    // the loop reads only the timings: outputs are copied out for an observer only
    const auto out = ctx.FinishStep(static_cast<bool>(options.step_observer));
    observe(out);
    const double ms = Ms(step_starts.front(), Clock::now());
    step_starts.pop_front();
    stats.run_batch_wall_ms += ms;
    step_ms.push_back(ms);
    Add(&timings_sum, out.aggregate_timings);
    Add(&overhead_sum, out.runtime_overheads);
  };
  const auto wall0 = Clock::now();
  std::vector<int> up_pages, up_offs, up_reqs, up_steps;
  std::vector<float> up_k, up_v;
  std::vector<AppendTokenResult> results;
  std::vector<std::vector<float>> gen_k, gen_v;
  const int pool_threads = static_cast<int>(
      std::min<unsigned>(8, std::max(1u, std::thread::hardware_concurrency())) - 1);
  detail::WorkerPool pool(pool_threads);
  std::vector<std::pair<int, PageId>> new_pages;
  std::vector<int> np_reqs;
  std::vector<PageId> np_pages;
  while (next < specs.size() || !pending.empty() || !active.empty()) {
    if (active.empty() && pending.empty() && next < specs.size() &&
        step < specs[next].arrival_step)
      step = specs[next].arrival_step;
    while (next < specs.size() && specs[next].arrival_step <= step) pending.push_back(next++);
    while (static_cast<int>(active.size()) < options.max_active_requests && !pending.empty()) {
      const std::size_t i = pending.front();
      pending.pop_front();
      const auto& spec = specs[i];
      if (!admitted[i]) {
        const auto t0 = Clock::now();
        Admit(config, spec, options.prompt_admission_mode, &cache, &ctx, tables);
        const double ms = Ms(t0, Clock::now());
        stats.admission_ms += ms;
        stats.runtime_admission_ms += ms;
        admitted[i] = 1;
      }
      if (spec.decode_steps > 0) {
        ActiveDecodeRequest a;
        a.state = MakeRequestState(spec.request_id, spec.initial_query, cache, spec.prompt_tokens);
        a.remaining_decode_steps = spec.decode_steps;
        a.spec_index = i;
        active.push_back(std::move(a));
      } else {
        const auto freed = cache.ReleaseRequest(spec.request_id);
        if (tables) ctx.ReleaseRequestPages(spec.request_id, false);
        if (!options.lazy_release) ctx.SyncFreedPages(freed);
      }
    }
    if (active.empty()) {
      ++step;
      continue;
    }

    batch.clear();
    query_rows.clear();
    for (const auto& a : active) {
      batch.push_back(&a.state);
      query_rows.push_back(a.query_row);
    }
    // With device page tables steps are queued asynchronously and up to two
    // are in flight: the host bookkeeping of this step's token appends, its
    // releases and the next step's admission overlap the GPU work (every
    // upload is ordered after the step on the context stream).
    record_step();
    ++step_index;
    if (tables) {
      step_starts.push_back(Clock::now());
      ctx.BeginStep(batch, run_opts, &query_rows);
    } else {
      const auto s0 = Clock::now();
      const auto out = ctx.RunBatch(batch, run_opts);
      observe(out);
      const double ms = Ms(s0, Clock::now());
      stats.run_batch_wall_ms += ms;
      step_ms.push_back(ms);
      Add(&timings_sum, out.aggregate_timings);
      Add(&overhead_sum, out.runtime_overheads);
    }
    ++nonempty;
    active_sum += static_cast<int>(active.size());

    // append this step's token of every active request
    results.clear();
    up_pages.clear(); up_offs.clear(); up_reqs.clear(); up_steps.clear();
    up_k.clear(); up_v.clear();
    new_pages.clear();
    // payloads of this step (K/V of the token, the next query): independent
    // per request, generated on the worker pool
    const bool gen_kv = !options.gpu_synthetic_decode_append && !options.precompute_decode_payloads;
    if (gen_kv) {
      gen_k.resize(active.size());
      gen_v.resize(active.size());
    }
    auto next_payload = [&](int i) {
      auto& a = active[static_cast<std::size_t>(i)];
      const int rid = a.state.request_id;
      const int d = a.decode_step_index;
      if (gen_kv) {
        gen_k[static_cast<std::size_t>(i)] = DeterministicTokenVector(ept, rid, d, 1);
        gen_v[static_cast<std::size_t>(i)] = DeterministicTokenVector(ept, rid, d, 2);
      }
      if (options.precompute_decode_payloads) {
        const float* q = pre_q[a.spec_index].data() + static_cast<std::size_t>(d) * ept;
        // queued steps pack it straight from the payload store
        if (tables) a.query_row = q; else a.state.query.assign(q, q + ept);
      } else {
        a.state.query = DeterministicTokenVector(ept, rid, d + 1, 0);
      }
    };
    // generation is spread over the worker pool; pointing at precomputed rows
    // is not worth a dispatch
    if (gen_kv || !options.precompute_decode_payloads)
      pool.ParallelFor(static_cast<int>(active.size()), next_payload);
    else
      for (int i = 0; i < static_cast<int>(active.size()); ++i) next_payload(i);
    for (std::size_t ai = 0; ai < active.size(); ++ai) {
      auto& a = active[ai];
      const int rid = a.state.request_id;
      const int d = a.decode_step_index;
      const float* kp = nullptr;
      const float* vp = nullptr;
      if (!options.gpu_synthetic_decode_append) {
        if (options.precompute_decode_payloads) {
          kp = pre_k[a.spec_index].data() + static_cast<std::size_t>(d) * ept;
          vp = pre_v[a.spec_index].data() + static_cast<std::size_t>(d) * ept;
        } else {
          kp = gen_k[ai].data();
          vp = gen_v[ai].data();
        }
      }
      // GPU admission modes open a new page for the first decoded token (:614-616)
      const bool force_new = options.prompt_admission_mode != Mode::kCpuCache && d == 0;
      const AppendTokenResult r =
          options.gpu_synthetic_decode_append ? cache.AppendTokenMetadataOnly(rid, force_new)
          : metadata_only ? cache.AppendTokenMetadataOnly(rid, kp, force_new)
                          : cache.AppendToken(rid, kp, vp, force_new);
      if (r.allocated_new_page) a.state.candidate_page_ids.push_back(r.page_id);
      // the token of a request's last step is never read again (:625)
      if (a.remaining_decode_steps > 1) {
        results.push_back(r);
        up_pages.push_back(r.page_id);
        up_offs.push_back(r.token_offset);
        up_reqs.push_back(rid);
        up_steps.push_back(d);
        if (!options.gpu_synthetic_decode_append) {
          up_k.insert(up_k.end(), kp, kp + ept);
          up_v.insert(up_v.end(), vp, vp + ept);
        }
        if (r.allocated_new_page) new_pages.emplace_back(rid, r.page_id);
      }
      ++a.state.context_tokens;
      if (!tables) {
        const auto& pages = cache.GetRequestPages(rid);
        a.state.candidate_page_ids.assign(pages.begin(), pages.end());
      }
      ++a.decode_step_index;
      --a.remaining_decode_steps;
      ++stats.total_generated_tokens;
    }
    const auto a0 = Clock::now();
    if (!results.empty()) {
      if (options.gpu_synthetic_decode_append) {
        ctx.AppendSyntheticTokens(cache, results, up_reqs, up_steps);
      } else if (metadata_only) {
        if (tables) {
          // K/V, running-mean summaries and the new page-table entries in one upload
          detail::ThrowIf(dsd_append_tokens(ctx.handle(), up_pages.data(), up_offs.data(),
                                            up_reqs.data(), static_cast<int>(up_pages.size()),
                                            up_k.data(), up_v.data()));
          new_pages.clear();
        } else {
          ctx.SyncAppendedTokensDirect(cache, results, up_k, up_v);
        }
      } else {
        ctx.SyncAppendedTokens(cache, results);
      }
      if (tables && !new_pages.empty()) {
        np_reqs.clear();
        np_pages.clear();
        for (const auto& np : new_pages) {
          np_reqs.push_back(np.first);
          np_pages.push_back(np.second);
        }
        ctx.AppendRequestPages(np_reqs, np_pages);   // one upload for all of them
      }
    }
    stats.append_sync_ms += Ms(a0, Clock::now());
    if (tables && ctx.PendingSteps() == 2) finish_oldest();

    std::vector<PageId> released;
    active.erase(std::remove_if(active.begin(), active.end(),
                                [&](const ActiveDecodeRequest& a) {
                                  if (a.remaining_decode_steps > 0) return false;
                                  auto p = cache.ReleaseRequest(a.state.request_id);
                                  released.insert(released.end(), p.begin(), p.end());
                                  if (tables) ctx.ReleaseRequestPages(a.state.request_id, false);
                                  return true;
                                }),
                 active.end());
    const auto r0 = Clock::now();
    if (!options.lazy_release) ctx.SyncFreedPages(released);
    stats.release_sync_ms += Ms(r0, Clock::now());
    ++step;
  }

  while (tables && ctx.PendingSteps() > 0) finish_oldest();
  stats.total_wall_ms = Ms(wall0, Clock::now());
  stats.tokens_per_second = stats.total_wall_ms > 0.0
                                ? stats.total_generated_tokens / (stats.total_wall_ms / 1000.0)
                                : 0.0;
  stats.outside_run_batch_ms = std::max(0.0, stats.total_wall_ms - stats.run_batch_wall_ms);
  stats.serving_loop_other_ms =
      std::max(0.0, stats.total_wall_ms - stats.run_batch_wall_ms - stats.runtime_admission_ms -
                        stats.append_sync_ms - stats.release_sync_ms);
  stats.measured_end_to_end_ms =
      stats.decode_payload_prep_ms + stats.prompt_preadmit_ms + stats.total_wall_ms;
  stats.device_transfer_stats = ctx.DeviceTransfers();
  stats.avg_step_ms =
      step_ms.empty() ? 0.0
                      : std::accumulate(step_ms.begin(), step_ms.end(), 0.0) / step_ms.size();
  stats.p50_step_ms = Percentile(step_ms, 0.50);
  stats.p95_step_ms = Percentile(step_ms, 0.95);
  stats.avg_active_batch_size = nonempty > 0 ? static_cast<double>(active_sum) / nonempty : 0.0;
  if (nonempty > 0) {
    const double inv = 1.0 / nonempty;
    stats.avg_sparse_timings = timings_sum;
    stats.avg_sparse_timings.page_scoring_ms *= inv;
    stats.avg_sparse_timings.topk_ms *= inv;
    stats.avg_sparse_timings.gather_ms *= inv;
    stats.avg_sparse_timings.attention_ms *= inv;
    stats.avg_sparse_timings.total_ms *= inv;
    stats.avg_runtime_overheads = overhead_sum;
    RuntimeOverheadTimings& o = stats.avg_runtime_overheads;
    o.time_malloc_ms *= inv; o.time_memcpy_h2d_ms *= inv; o.time_memcpy_d2h_ms *= inv;
    o.time_free_ms *= inv; o.time_kernel_launch_ms *= inv; o.time_sync_ms *= inv;
    o.time_prepare_sparse_layout_ms *= inv;
  }
  return stats;
}

}  // namespace

ContinuousBatchStats RunContinuousDenseGpuDecode(const ModelConfig& config,
                                                 const std::vector<ContinuousRequestSpec>& specs,
                                                 int max_active_requests) {
  ContinuousDecodeOptions o;
  o.max_active_requests = max_active_requests;
  return RunContinuousDenseGpuDecode(config, specs, o);
}

ContinuousBatchStats RunContinuousDenseGpuDecode(const ModelConfig& config,
                                                 const std::vector<ContinuousRequestSpec>& specs,
                                                 const ContinuousDecodeOptions& options) {
  return RunContinuous(config, specs, options, true);
}

ContinuousBenchmarkResult RunContinuousSparseBenchmark(
    const ModelConfig& config, const std::vector<ContinuousRequestSpec>& requests,
    int max_active_requests) {
  ContinuousDecodeOptions o;
  o.max_active_requests = max_active_requests;
  return RunContinuousSparseBenchmark(config, requests, o);
}

ContinuousBenchmarkResult RunContinuousSparseBenchmark(
    const ModelConfig& config, const std::vector<ContinuousRequestSpec>& requests,
    const ContinuousDecodeOptions& options) {
  ContinuousBenchmarkResult r;
  r.continuous_sparse = RunContinuousSparseDecode(config, requests, options);
  ContinuousDecodeOptions serial = options;
  serial.max_active_requests = 1;
  r.serial_sparse = RunContinuousSparseDecode(config, requests, serial);
  r.continuous_vs_serial_speedup =
      r.serial_sparse.tokens_per_second > 0.0
          ? r.continuous_sparse.tokens_per_second / r.serial_sparse.tokens_per_second
          : 0.0;
  return r;
}

}  // namespace dsd
