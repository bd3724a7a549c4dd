// dsd_continuous_bench -- continuous-batching benchmark, argv- and
// key=value-compatible with the reference CLI
// (benchmarks/bench_continuous_decode.cpp:178-291):
//   1 num_requests=128 2 max_active=32 3 arrival_window=64 4 min_prompt=1024
//   5 max_prompt=4096 6 min_decode=16 7 max_decode=64 8 seed=7 9 heads=32
//   10 head_dim=128 11 page_size=16 12 top_k=8 13 admission (0 cpu_cache,
//   1 direct_gpu_upload, 2 synthetic_gpu_prefill) 14 preadmit 15 precompute
//   16 gpu_synthetic_append 17 lazy_release 18 output_mode (0 none, 1 outputs,
//   2 debug) 19 timing (0 none, 1 kernel_events) 20 benchmark_mode (0 sparse,
//   1 dense_gpu)
// Added: 21 device_page_tables (default 1), 22 skip the serial run (default 0),
// 23 shard_world (default 1), 24 shard_rank (default 0): serve only requests
// with request_id % shard_world == shard_rank (one process per GPU),
// 25 repeats (default 1): serve the workload this many times (a fresh
// context each time) and print every repeat's tokens/s; the stats printed
// are the median repeat's.  26 kv_format (default 0 = fp32 pages, the
// reference's; 1 = bf16, 2 = fp8 e4m3 pages and summaries, fp32 arithmetic).
#include <algorithm>
#include <cstdlib>
#include <vector>
#include <iomanip>
#include <iostream>
#include <stdexcept>
#include <string>

#include "dsd/config.h"
#include "dsd/continuous_batching.h"
#include "dsd/cuda_sparse_attention.h"

namespace {

int Arg(int argc, char** argv, int i, int dflt) { return argc > i ? std::atoi(argv[i]) : dflt; }

void Print(const std::string& p, const dsd::ContinuousBatchStats& s) {
  auto kv = [&](const char* k, double v) { std::cout << p << "_" << k << "=" << v << "\n"; };
  kv("total_ms", s.total_wall_ms);
  kv("measured_end_to_end_ms", s.measured_end_to_end_ms);
  kv("tokens_per_second", s.tokens_per_second);
  kv("admission_ms", s.admission_ms);
  kv("prompt_preadmit_ms", s.prompt_preadmit_ms);
  kv("runtime_admission_ms", s.runtime_admission_ms);
  kv("append_sync_ms", s.append_sync_ms);
  kv("release_sync_ms", s.release_sync_ms);
  kv("decode_payload_prep_ms", s.decode_payload_prep_ms);
  kv("run_batch_wall_ms", s.run_batch_wall_ms);
  kv("outside_run_batch_ms", s.outside_run_batch_ms);
  kv("serving_loop_other_ms", s.serving_loop_other_ms);
  kv("avg_step_ms", s.avg_step_ms);
  kv("p50_step_ms", s.p50_step_ms);
  kv("p95_step_ms", s.p95_step_ms);
  kv("avg_active_batch_size", s.avg_active_batch_size);
  kv("avg_score_ms", s.avg_sparse_timings.page_scoring_ms);
  kv("avg_topk_ms", s.avg_sparse_timings.topk_ms);
  kv("avg_gather_ms", s.avg_sparse_timings.gather_ms);
  kv("avg_attention_ms", s.avg_sparse_timings.attention_ms);
  kv("avg_kernel_ms", s.avg_sparse_timings.total_ms);
  kv("avg_h2d_ms", s.avg_runtime_overheads.time_memcpy_h2d_ms);
  kv("avg_d2h_ms", s.avg_runtime_overheads.time_memcpy_d2h_ms);
  kv("avg_launch_ms", s.avg_runtime_overheads.time_kernel_launch_ms);
  kv("avg_sync_ms", s.avg_runtime_overheads.time_sync_ms);
  kv("avg_prepare_sparse_layout_ms", s.avg_runtime_overheads.time_prepare_sparse_layout_ms);
  std::cout << p << "_device_h2d_bytes=" << s.device_transfer_stats.h2d_bytes << "\n"
            << p << "_device_d2h_bytes=" << s.device_transfer_stats.d2h_bytes << "\n"
            << p << "_device_h2d_calls=" << s.device_transfer_stats.h2d_calls << "\n"
            << p << "_device_d2h_calls=" << s.device_transfer_stats.d2h_calls << "\n"
            << p << "_device_h2d_large_calls=" << s.device_transfer_stats.h2d_large_calls << "\n"
            << p << "_device_d2h_large_calls=" << s.device_transfer_stats.d2h_large_calls << "\n"
            << p << "_admission_device_h2d_bytes=" << s.admission_device_transfer_stats.h2d_bytes << "\n"
            << p << "_admission_device_h2d_calls=" << s.admission_device_transfer_stats.h2d_calls << "\n"
            << p << "_admission_device_h2d_large_calls="
            << s.admission_device_transfer_stats.h2d_large_calls << "\n";
}

}  // namespace

int main(int argc, char** argv) try {
  dsd::ModelConfig config;
  const int num_requests = Arg(argc, argv, 1, 128);
  const int max_active = Arg(argc, argv, 2, 32);
  const int arrival_window = Arg(argc, argv, 3, 64);
  const int min_prompt = Arg(argc, argv, 4, 1024);
  const int max_prompt = Arg(argc, argv, 5, 4096);
  const int min_decode = Arg(argc, argv, 6, 16);
  const int max_decode = Arg(argc, argv, 7, 64);
  const int seed = Arg(argc, argv, 8, 7);
  config.num_heads = Arg(argc, argv, 9, 32);
  config.head_dim = Arg(argc, argv, 10, 128);
  config.page_size = Arg(argc, argv, 11, 16);
  config.top_k_pages = Arg(argc, argv, 12, 8);
  const int admission = Arg(argc, argv, 13, 1);
  dsd::ContinuousDecodeOptions o;
  o.max_active_requests = max_active;
  if (admission < 0 || admission > 2)
    throw std::invalid_argument(
        "admission_mode must be 0=cpu_cache, 1=direct_gpu_upload, or 2=synthetic_gpu_prefill");
  o.prompt_admission_mode = static_cast<dsd::ContinuousPromptAdmissionMode>(admission);
  o.preadmit_prompts = Arg(argc, argv, 14, 0) != 0;
  o.precompute_decode_payloads = Arg(argc, argv, 15, 0) != 0;
  o.gpu_synthetic_decode_append = Arg(argc, argv, 16, 0) != 0;
  o.lazy_release = Arg(argc, argv, 17, 0) != 0;
  const int out_mode = Arg(argc, argv, 18, 1);
  o.run_batch_output_mode = out_mode == 0 ? dsd::SparseBatchOutputMode::kNoOutputs
                            : out_mode == 2 ? dsd::SparseBatchOutputMode::kDebugTensors
                                            : dsd::SparseBatchOutputMode::kOutputsOnly;
  o.run_batch_timing_mode = Arg(argc, argv, 19, 1) ? dsd::SparseBatchTimingMode::kKernelEvents
                                                   : dsd::SparseBatchTimingMode::kNone;
  const int bench_mode = Arg(argc, argv, 20, 0);
  o.device_page_tables = Arg(argc, argv, 21, 1) != 0;
  const bool skip_serial = Arg(argc, argv, 22, 0) != 0;
  const int shard_world = Arg(argc, argv, 23, 1);
  const int shard_rank = Arg(argc, argv, 24, 0);
  const int repeats = std::max(1, Arg(argc, argv, 25, 1));
  o.kv_format = Arg(argc, argv, 26, 0);
  if (shard_world < 1 || shard_rank < 0 || shard_rank >= shard_world)
    throw std::invalid_argument("shard_rank must be in [0, shard_world)");
  const char* adm[] = {"cpu_cache", "direct_gpu_upload", "synthetic_gpu_prefill"};
  const char* outn[] = {"no_outputs", "outputs_only", "debug_tensors"};

  std::cout << std::fixed << std::setprecision(6);
  std::cout << "num_requests=" << num_requests << "\nmax_active_requests=" << max_active
            << "\narrival_window=" << arrival_window << "\nmin_prompt_tokens=" << min_prompt
            << "\nmax_prompt_tokens=" << max_prompt << "\nmin_decode_steps=" << min_decode
            << "\nmax_decode_steps=" << max_decode << "\nseed=" << seed
            << "\nnum_heads=" << config.num_heads << "\nhead_dim=" << config.head_dim
            << "\npage_size=" << config.page_size << "\ntop_k_pages=" << config.top_k_pages
            << "\nadmission_mode=" << adm[admission]
            << "\npreadmit_prompts=" << o.preadmit_prompts
            << "\nprecompute_decode_payloads=" << o.precompute_decode_payloads
            << "\ngpu_synthetic_decode_append=" << o.gpu_synthetic_decode_append
            << "\nlazy_release=" << o.lazy_release
            << "\nrun_batch_output_mode=" << outn[out_mode < 0 || out_mode > 2 ? 1 : out_mode]
            << "\nrun_batch_timing_mode="
            << (o.run_batch_timing_mode == dsd::SparseBatchTimingMode::kNone ? "none" : "kernel_events")
            << "\nbenchmark_mode=" << (bench_mode == 1 ? "dense_gpu" : "sparse")
            << "\ndevice_page_tables=" << o.device_page_tables << "\nshard_world=" << shard_world
            << "\nshard_rank=" << shard_rank << "\n";
  std::cout << "kv_format="
            << (o.kv_format == 2 ? "fp8" : o.kv_format == 1 ? "bf16" : "fp32") << "\n";

  const char* avail = bench_mode == 1 ? "continuous_dense_gpu_available" : "continuous_sparse_available";
  if (!dsd::SparseAttentionCudaAvailable()) {
    std::cout << avail << "=0\ncontinuous benchmark skipped: no visible sm_100 GPU\n";
    return 0;
  }
  std::cout << avail << "=1\n";
  auto specs =
      admission == 2
          ? dsd::BuildSyntheticContinuousSpecs(config, num_requests, arrival_window, min_prompt,
                                               max_prompt, min_decode, max_decode, seed)
          : dsd::BuildSyntheticContinuousWorkload(config, num_requests, arrival_window, min_prompt,
                                                  max_prompt, min_decode, max_decode, seed);
  if (shard_world > 1) {
    decltype(specs) mine;
    for (auto& sp : specs)
      if (sp.request_id % shard_world == shard_rank) mine.push_back(std::move(sp));
    specs.swap(mine);
  }
  std::cout << "shard_requests=" << specs.size() << "\n";
  if (bench_mode == 1) {
    const auto d = dsd::RunContinuousDenseGpuDecode(config, specs, o);
    std::cout << "total_generated_tokens=" << d.total_generated_tokens << "\n";
    Print("continuous_dense_gpu", d);
    return 0;
  }
  if (skip_serial) {
    std::vector<dsd::ContinuousBatchStats> runs;
    for (int i = 0; i < repeats; ++i) {
      runs.push_back(dsd::RunContinuousSparseDecode(config, specs, o));
      std::cout << "continuous_sparse_repeat_tokens_per_second=" << runs.back().tokens_per_second
                << "\n";
    }
    std::sort(runs.begin(), runs.end(), [](const auto& a, const auto& b) {
      return a.tokens_per_second < b.tokens_per_second;
    });
    const auto& s = runs[runs.size() / 2];
    std::cout << "total_generated_tokens=" << s.total_generated_tokens << "\n";
    Print("continuous_sparse", s);
    return 0;
  }
  const auto r = dsd::RunContinuousSparseBenchmark(config, specs, o);
  std::cout << "total_generated_tokens=" << r.continuous_sparse.total_generated_tokens << "\n";
  Print("continuous_sparse", r.continuous_sparse);
  Print("serial_sparse", r.serial_sparse);
  std::cout << "continuous_vs_serial_speedup=" << r.continuous_vs_serial_speedup << "\n";
  return 0;
} catch (const std::exception& e) {
  std::cerr << "error: " << e.what() << "\n";
  return 1;
}
