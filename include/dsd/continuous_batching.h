// Continuous-batching decode loop (drop-in for include/dsd/continuous_batching.h:12-117).
// Requests arrive at arrival_step, are admitted while fewer than
// max_active_requests are decoding, decode one token per step (the sparse
// step on the GPU, then the new K/V token is appended on the device) and
// release their pages when done.
#pragma once

#include <cstddef>
#include <functional>
#include <vector>

#include "dsd/config.h"
#include "dsd/cuda_sparse_attention.h"
#include "dsd/types.h"

namespace dsd {

struct ContinuousRequestSpec {
  int request_id = -1;
  int arrival_step = 0;
  int prompt_tokens = 0;
  int decode_steps = 0;
  std::vector<float> prompt_keys;    // [prompt_tokens][H*D]; empty for synthetic prefill
  std::vector<float> prompt_values;
  std::vector<float> initial_query;  // [H*D]
};

struct ActiveDecodeRequest {
  RequestState state;
  int remaining_decode_steps = 0;
  int decode_step_index = 0;
  std::size_t spec_index = 0;
  // This build: when non-null, the step's query (a precomputed payload row)
  // used in place of state.query
  const float* query_row = nullptr;
};

enum class ContinuousPromptAdmissionMode { kCpuCache, kDirectGpuUpload, kSyntheticGpuPrefill };

// This build: one decode step of the serving loop as the step observer sees
// it -- the batch in launch order (request id, context tokens, the page list
// the step selected from and the query the host handed over) and the step's
// result (per_request outputs; selected ids and scores in kDebugTensors mode).
struct ContinuousStepRecord {
  int step_index = 0;
  std::vector<int> request_ids;
  std::vector<int> context_tokens;
  std::vector<std::vector<PageId>> candidate_page_ids;
  std::vector<std::vector<float>> queries;
  const SparseBatchCudaResult* result = nullptr;
};

struct ContinuousDecodeOptions {
  int max_active_requests = 1;
  ContinuousPromptAdmissionMode prompt_admission_mode =
      ContinuousPromptAdmissionMode::kDirectGpuUpload;
  bool preadmit_prompts = false;
  bool precompute_decode_payloads = false;
  bool gpu_synthetic_decode_append = false;
  bool lazy_release = false;
  SparseBatchOutputMode run_batch_output_mode = SparseBatchOutputMode::kOutputsOnly;
  SparseBatchTimingMode run_batch_timing_mode = SparseBatchTimingMode::kKernelEvents;
  // This build: candidates come from the device request page tables (no host
  // CSR packing per step).  false = the reference's explicit-candidate RunBatch.
  bool device_page_tables = true;
  int device = 0;
  // This build: page element format of the device pool (DSD_KV_F32, the
  // reference's, or DSD_KV_BF16: bf16 pages and summaries, fp32 arithmetic).
  int kv_format = 0;
  // This build: called once per decode step, in step order, when the step's
  // results are on the host (tracing and step-by-step checking).  Unset by
  // default; the record and its result are valid during the call only.
  std::function<void(const ContinuousStepRecord&)> step_observer;
};

struct ContinuousBatchStats {
  int total_generated_tokens = 0;
  double total_wall_ms = 0.0;
  double avg_step_ms = 0.0;
  double p50_step_ms = 0.0;
  double p95_step_ms = 0.0;
  double tokens_per_second = 0.0;
  double avg_active_batch_size = 0.0;
  double admission_ms = 0.0;
  double prompt_preadmit_ms = 0.0;
  double runtime_admission_ms = 0.0;
  double append_sync_ms = 0.0;
  double release_sync_ms = 0.0;
  double decode_payload_prep_ms = 0.0;
  double run_batch_wall_ms = 0.0;
  double outside_run_batch_ms = 0.0;
  double serving_loop_other_ms = 0.0;
  double measured_end_to_end_ms = 0.0;
  StageTimings avg_sparse_timings;
  RuntimeOverheadTimings avg_runtime_overheads;
  DeviceTransferStats device_transfer_stats;
  DeviceTransferStats admission_device_transfer_stats;
};

struct ContinuousBenchmarkResult {
  ContinuousBatchStats continuous_sparse;
  ContinuousBatchStats serial_sparse;
  double continuous_vs_serial_speedup = 0.0;
};

// The reference generator: mt19937(seed); per request arrival in
// [0, arrival_window] (inclusive), prompt and decode lengths, then prompt K,
// prompt V and the initial query (U(-1,1)); sorted by (arrival, id).
std::vector<ContinuousRequestSpec> BuildSyntheticContinuousWorkload(
    const ModelConfig& config, int num_requests, int arrival_window, int min_prompt_tokens,
    int max_prompt_tokens, int min_decode_steps, int max_decode_steps, int seed);

// Same lengths and arrivals without prompt payloads (for synthetic GPU
// prefill at sizes whose payloads cannot be held on the host).  The payload
// draws are skipped, so the lengths differ from the full generator's.
std::vector<ContinuousRequestSpec> BuildSyntheticContinuousSpecs(
    const ModelConfig& config, int num_requests, int arrival_window, int min_prompt_tokens,
    int max_prompt_tokens, int min_decode_steps, int max_decode_steps, int seed);

// DeterministicTokenVector: U(-1,1) from mt19937(mix(request, step, stream)).
std::vector<float> DeterministicTokenVector(int count, int request_id, int decode_step,
                                            int stream);

ContinuousBatchStats RunContinuousSparseDecode(const ModelConfig& config,
                                               const std::vector<ContinuousRequestSpec>& requests,
                                               int max_active_requests);
ContinuousBatchStats RunContinuousSparseDecode(const ModelConfig& config,
                                               const std::vector<ContinuousRequestSpec>& requests,
                                               const ContinuousDecodeOptions& options);
ContinuousBatchStats RunContinuousDenseGpuDecode(const ModelConfig& config,
                                                 const std::vector<ContinuousRequestSpec>& requests,
                                                 int max_active_requests);
ContinuousBatchStats RunContinuousDenseGpuDecode(const ModelConfig& config,
                                                 const std::vector<ContinuousRequestSpec>& requests,
                                                 const ContinuousDecodeOptions& options);
ContinuousBenchmarkResult RunContinuousSparseBenchmark(
    const ModelConfig& config, const std::vector<ContinuousRequestSpec>& requests,
    int max_active_requests);
ContinuousBenchmarkResult RunContinuousSparseBenchmark(
    const ModelConfig& config, const std::vector<ContinuousRequestSpec>& requests,
    const ContinuousDecodeOptions& options);

}  // namespace dsd
