// dsd_bench -- one-step batched decode benchmark, argv- and output-compatible
// with the reference CLI (benchmarks/bench_decode.cpp:336-657):
//   dsd_bench [top_k=8] [batch=16] [min_ctx=512] [max_ctx=2048] [seed=7]
//             [iterations=5] [warmup=1] [num_heads=8] [head_dim=16] [page_size=16]
// Sections and row names match, so the reference's experiment scripts parse
// it.  Added keys: sparse_gpu_hbm_gbps, sparse_gpu_roofline_frac (against the
// HBM bandwidth HbmBytesPerSec finds), sparse_gpu_roofline_peak_gbps and
// _peak_source, sparse_gpu_selection_exact.
#include <algorithm>
#include <chrono>
#include <cstdint>
#include <cstdlib>
#include <fstream>
#include <iterator>
#include <iomanip>
#include <iostream>
#include <memory>
#include <string>
#include <vector>

#include "dsd/config.h"
#include "dsd/cuda_dense_attention.h"
#include "dsd/cuda_sparse_attention.h"
#include "dsd/decode_pipeline.h"
#include "dsd/reference_kernels.h"
#include "dsd/synthetic_data.h"

namespace {

using Clock = std::chrono::steady_clock;
constexpr double kFp32FlopsPerSec = 75e12;      // B200 fp32 CUDA-core figure (context only)

// HBM bandwidth the roofline fractions are quoted against, in bytes/s, and
// where it came from: $DSD_HBM_GBS, else "hbm_gbs" of MEASURED_PEAKS.json
// (the copy bandwidth measured on the machine, looked for in the working
// directory and two levels above this executable), else a nominal 6.65 TB/s.
std::string g_hbm_source = "fallback";
double HbmBytesPerSec(const char* argv0) {
  if (const char* env = std::getenv("DSD_HBM_GBS")) {
    g_hbm_source = "DSD_HBM_GBS";
    return std::atof(env) * 1e9;
  }
  std::string exe = argv0 ? argv0 : "";
  const auto slash = exe.find_last_of('/');
  const std::string dir = slash == std::string::npos ? "." : exe.substr(0, slash);
  for (const std::string& path : {std::string("MEASURED_PEAKS.json"),
                                 dir + "/../../MEASURED_PEAKS.json"}) {
    std::ifstream f(path);
    if (!f) continue;
    const std::string text((std::istreambuf_iterator<char>(f)), std::istreambuf_iterator<char>());
    const auto key = text.find("\"hbm_gbs\"");
    if (key == std::string::npos) continue;
    const auto colon = text.find(':', key);
    if (colon == std::string::npos) continue;
    const double gbs = std::atof(text.c_str() + colon + 1);
    if (gbs > 0) {
      g_hbm_source = "measured";
      return gbs * 1e9;
    }
  }
  return 6650e9;
}
double kHbmBytesPerSec = 6650e9;

int Arg(int argc, char** argv, int i, int dflt) { return argc > i ? std::atoi(argv[i]) : dflt; }

double Ms(Clock::time_point a, Clock::time_point b) {
  return std::chrono::duration<double, std::milli>(b - a).count();
}

double OverheadMs(const dsd::RuntimeOverheadTimings& t) {
  return t.time_malloc_ms + t.time_memcpy_h2d_ms + t.time_memcpy_d2h_ms + t.time_free_ms +
         t.time_kernel_launch_ms + t.time_sync_ms + t.time_prepare_sparse_layout_ms;
}

void AnalyticalRow(const std::string& name, double bytes, double flops) {
  std::cout << std::left << std::setw(16) << name << std::right << std::fixed
            << std::setprecision(3) << std::setw(12) << bytes / 1e6 << std::setw(12)
            << flops / 1e6 << std::setw(12) << (bytes > 0 ? flops / bytes : 0.0) << std::setw(14)
            << bytes / kHbmBytesPerSec * 1e6 << std::setw(14) << flops / kFp32FlopsPerSec * 1e6
            << "\n";
}

}  // namespace

int main(int argc, char** argv) {
  kHbmBytesPerSec = HbmBytesPerSec(argc > 0 ? argv[0] : nullptr);
  dsd::ModelConfig config;
  config.top_k_pages = Arg(argc, argv, 1, 8);
  config.num_heads = Arg(argc, argv, 8, 8);
  config.head_dim = Arg(argc, argv, 9, 16);
  config.page_size = Arg(argc, argv, 10, 16);
  const int batch_size = Arg(argc, argv, 2, 16);
  const int min_ctx = Arg(argc, argv, 3, 512);
  const int max_ctx = Arg(argc, argv, 4, 2048);
  const int seed = Arg(argc, argv, 5, 7);
  const int iterations = Arg(argc, argv, 6, 5);
  const int warmup = Arg(argc, argv, 7, 1);

  const auto batch = dsd::BuildSyntheticBatch(config, batch_size, min_ctx, max_ctx, seed);
  dsd::DecodePipeline pipeline(config);
  const std::uint64_t ept = static_cast<std::uint64_t>(config.num_heads * config.head_dim);
  std::uint64_t ctx_tokens = 0, cand = 0, sel_tokens_nominal = 0;
  int total_sel = 0;
  for (const auto& r : batch.requests) {
    ctx_tokens += static_cast<std::uint64_t>(std::max(0, r.context_tokens));
    cand += r.candidate_page_ids.size();
    const int k = std::min<int>(config.top_k_pages, static_cast<int>(r.candidate_page_ids.size()));
    total_sel += k;
    sel_tokens_nominal += static_cast<std::uint64_t>(k) * config.page_size;
  }

  std::unique_ptr<dsd::SparseCudaContext> gpu;
  std::unique_ptr<dsd::DenseCudaContext> dense_gpu;
  const bool gpu_ok = dsd::SparseAttentionCudaAvailable();
  if (gpu_ok) {
    gpu.reset(new dsd::SparseCudaContext(batch.cache, config, batch_size, static_cast<int>(cand),
                                         total_sel));
    dense_gpu.reset(new dsd::DenseCudaContext(batch.cache, config));
  }

  double dense_total = 0, sparse_total = 0, s_score = 0, s_topk = 0, s_gather = 0, s_attn = 0;
  double g_total = 0, g_score = 0, g_topk = 0, g_attn = 0, g_kernel = 0;
  double dg_total = 0, dg_kernel = 0;
  dsd::DenseBatchResult dense_gpu_out;
  dsd::RuntimeOverheadTimings g_oh;
  std::vector<dsd::AttentionResult> dense_out;
  dsd::BatchDecodeResult cpu_out;
  dsd::SparseBatchCudaResult gpu_out;
  for (int it = 0; it < warmup + iterations; ++it) {
    const bool timed = it >= warmup;
    const auto d0 = Clock::now();
    dense_out.clear();
    for (const auto& r : batch.requests) dense_out.push_back(pipeline.RunDenseStep(batch.cache, r));
    const auto d1 = Clock::now();
    cpu_out = pipeline.RunNaiveSparseBatch(batch.cache, batch.requests);
    if (timed) {
      dense_total += Ms(d0, d1);
      sparse_total += cpu_out.aggregate_timings.total_ms;
      s_score += cpu_out.aggregate_timings.page_scoring_ms;
      s_topk += cpu_out.aggregate_timings.topk_ms;
      s_gather += cpu_out.aggregate_timings.gather_ms;
      s_attn += cpu_out.aggregate_timings.attention_ms;
    }
    if (gpu_ok) {
      const auto h0 = Clock::now();
      dense_gpu_out = dense_gpu->RunBatch(batch.requests);
      const auto h1 = Clock::now();
      if (timed) {
        dg_total += Ms(h0, h1);
        dg_kernel += dense_gpu_out.kernel_ms;
      }
      const auto g0 = Clock::now();
      gpu_out = gpu->RunBatch(batch.requests, dsd::SparseBatchOutputMode::kDebugTensors);
      const auto g1 = Clock::now();
      if (timed) {
        g_total += Ms(g0, g1);
        g_score += gpu_out.aggregate_timings.page_scoring_ms;
        g_topk += gpu_out.aggregate_timings.topk_ms;
        g_attn += gpu_out.aggregate_timings.attention_ms;
        g_kernel += gpu_out.kernel_ms;
        g_oh.time_sync_ms += gpu_out.runtime_overheads.time_sync_ms;
        g_oh.time_prepare_sparse_layout_ms += gpu_out.runtime_overheads.time_prepare_sparse_layout_ms;
      }
    }
  }
  const double n = std::max(1, iterations);
  dense_total /= n; sparse_total /= n; s_score /= n; s_topk /= n; s_gather /= n; s_attn /= n;
  g_total /= n; g_score /= n; g_topk /= n; g_attn /= n; g_kernel /= n;
  dg_total /= n; dg_kernel /= n;
  g_oh.time_sync_ms /= n; g_oh.time_prepare_sparse_layout_ms /= n;

  std::cout << "\n== Decode Benchmark ==\n";
  std::cout << "batch_size=" << batch_size << " total_pages=" << batch.cache.TotalPages()
            << " top_k_pages=" << config.top_k_pages << " num_heads=" << config.num_heads
            << " head_dim=" << config.head_dim << " page_size=" << config.page_size
            << " min_ctx=" << min_ctx << " max_ctx=" << max_ctx << " seed=" << seed
            << " iterations=" << iterations << " warmup=" << warmup << "\n";

  const double bpt = static_cast<double>(ept) * 4.0;
  const double dense_bytes = 2.0 * ctx_tokens * bpt;
  const double cur_bytes = (ctx_tokens + 6.0 * sel_tokens_nominal) * bpt;
  const double tgt_bytes = (cand + 2.0 * sel_tokens_nominal) * bpt;
  const double dense_flops = 4.0 * ctx_tokens * ept;
  const double sparse_flops = 2.0 * cand * ept + 4.0 * sel_tokens_nominal * ept;
  std::cout << "\n== Analytical Ceiling ==\n";
  std::cout << "total_context_tokens=" << ctx_tokens << " total_candidate_pages=" << cand
            << " total_selected_tokens=" << sel_tokens_nominal << "\n";
  std::cout << std::left << std::setw(16) << "Path" << std::right << std::setw(12) << "Bytes(MB)"
            << std::setw(12) << "FLOPs(M)" << std::setw(12) << "AI" << std::setw(14)
            << "BwFloor(us)" << std::setw(14) << "CmpFloor(us)" << "\n"
            << std::string(80, '-') << "\n";
  AnalyticalRow("dense", dense_bytes, dense_flops);
  AnalyticalRow("sparse_current", cur_bytes, sparse_flops);
  AnalyticalRow("sparse_target", tgt_bytes, sparse_flops);
  std::cout << std::fixed << std::setprecision(3) << "sparse_current_over_dense_bytes="
            << (dense_bytes > 0 ? cur_bytes / dense_bytes : 0.0)
            << " sparse_target_over_dense_bytes="
            << (dense_bytes > 0 ? tgt_bytes / dense_bytes : 0.0) << "\n";

  auto e2e = [&](const char* name, double ms, bool ok, const char* note) {
    std::cout << std::left << std::setw(12) << name << std::right << std::setw(14)
              << (ok ? ms : 0.0) << std::setw(14) << (ok && ms > 0 ? dense_total / ms : 0.0)
              << "  " << note << "\n";
  };
  std::cout << "\n== End-to-End ==\n";
  std::cout << std::left << std::setw(12) << "Path" << std::right << std::setw(14) << "Total(ms)"
            << std::setw(14) << "Speedup" << "  Note\n" << std::string(72, '-') << "\n";
  e2e("dense_cpu", dense_total, true, "reference wall time");
  e2e("sparse_cpu", sparse_total, true, "naive sparse pipeline");
  e2e("dense_gpu", dg_total, gpu_ok, gpu_ok ? "dense split-K attention (all pages)" : "unavailable");
  e2e("sparse_gpu", g_total, gpu_ok, gpu_ok ? "B200 sparse path (RunBatch)" : "unavailable");

  auto brk = [&](const char* name, double a, double b, double c, double d, double k, bool ok,
                 const char* note) {
    std::cout << std::left << std::setw(12) << name << std::right << std::setw(12) << (ok ? a : 0.0)
              << std::setw(12) << (ok ? b : 0.0) << std::setw(12) << (ok ? c : 0.0) << std::setw(12)
              << (ok ? d : 0.0) << std::setw(14) << (ok ? k : 0.0) << "  " << note << "\n";
  };
  std::cout << "\n== Stage / Kernel Breakdown ==\n";
  std::cout << std::left << std::setw(12) << "Path" << std::right << std::setw(12) << "Score"
            << std::setw(12) << "TopK" << std::setw(12) << "Gather" << std::setw(12) << "Attend"
            << std::setw(14) << "GPUKernel" << "  Note\n" << std::string(86, '-') << "\n";
  brk("dense_cpu", 0, 0, 0, dense_total, 0, true, "attention only");
  brk("sparse_cpu", s_score, s_topk, s_gather, s_attn, 0, true, "full CPU stage split");
  brk("dense_gpu", 0, 0, 0, dg_kernel, dg_kernel, gpu_ok, "attention kernel only");
  brk("sparse_gpu", g_score, g_topk, 0, g_attn, g_kernel, gpu_ok,
      gpu_ok ? "gather fused into attention" : "unavailable");

  std::cout << "\n== Runtime Overheads ==\n";
  std::cout << std::left << std::setw(12) << "Path" << std::right << std::setw(12) << "Malloc"
            << std::setw(12) << "H2D" << std::setw(12) << "D2H" << std::setw(12) << "Free"
            << std::setw(14) << "Launch" << std::setw(12) << "Sync" << std::setw(14)
            << "SparseLayout" << std::setw(12) << "TotalOH" << "  Note\n"
            << std::string(122, '-') << "\n";
  auto oh = [&](const char* name, const dsd::RuntimeOverheadTimings& t, bool ok, const char* note) {
    std::cout << std::left << std::setw(12) << name << std::right << std::setw(12)
              << t.time_malloc_ms << std::setw(12) << t.time_memcpy_h2d_ms << std::setw(12)
              << t.time_memcpy_d2h_ms << std::setw(12) << t.time_free_ms << std::setw(14)
              << t.time_kernel_launch_ms << std::setw(12) << t.time_sync_ms << std::setw(14)
              << t.time_prepare_sparse_layout_ms << std::setw(12) << (ok ? OverheadMs(t) : 0.0)
              << "  " << note << "\n";
  };
  const dsd::RuntimeOverheadTimings none;
  oh("dense_cpu", none, true, "host only");
  oh("sparse_cpu", none, true, "host only");
  oh("dense_gpu", dense_gpu_out.runtime_overheads, gpu_ok, "copies+launch+wait in one call");
  oh("sparse_gpu", g_oh, gpu_ok, "copies+launch+wait are one C ABI call (Sync)");

  // accuracy against dense_cpu and sparse_cpu; selection exactness
  double cpu_vs_dense = 0, gpu_vs_cpu = 0, gpu_vs_dense = 0, dgpu_vs_dense = 0;
  bool exact = true;
  for (std::size_t i = 0; i < batch.requests.size(); ++i) {
    cpu_vs_dense += dsd::MaxAbsDiff(cpu_out.per_request[i].output.output, dense_out[i].output);
    if (gpu_ok) {
      gpu_vs_cpu += dsd::MaxAbsDiff(gpu_out.per_request[i].output.output,
                                    cpu_out.per_request[i].output.output);
      gpu_vs_dense += dsd::MaxAbsDiff(gpu_out.per_request[i].output.output, dense_out[i].output);
      dgpu_vs_dense += dsd::MaxAbsDiff(dense_gpu_out.outputs[i].output, dense_out[i].output);
      exact = exact && gpu_out.per_request[i].selected_page_ids ==
                           cpu_out.per_request[i].selected_page_ids;
    }
  }
  const double nb = std::max<std::size_t>(1, batch.requests.size());
  std::cout << "\n== Accuracy ==\n" << std::scientific << std::setprecision(6);
  std::cout << "avg_max_abs_diff_sparse_cpu_vs_dense_cpu=" << cpu_vs_dense / nb << "\n";
  if (gpu_ok) {
    std::cout << "avg_max_abs_diff_sparse_gpu_vs_sparse_cpu=" << gpu_vs_cpu / nb << "\n";
    std::cout << "avg_max_abs_diff_sparse_gpu_vs_dense_cpu=" << gpu_vs_dense / nb << "\n";
    std::cout << "avg_max_abs_diff_dense_gpu_vs_dense_cpu=" << dgpu_vs_dense / nb << "\n";
    std::cout << "sparse_gpu_selection_exact=" << (exact ? 1 : 0) << "\n";
    // algorithmic bytes of one GPU step over its kernel time
    std::uint64_t sel_tokens = 0;
    for (const auto& r : gpu_out.per_request)
      for (int p : r.selected_page_ids) sel_tokens += batch.cache.GetPage(p).token_count;
    const double step_bytes = 4.0 * ept * cand + 8.0 * ept * sel_tokens + 8.0 * ept * batch_size +
                              4.0 * (cand + 2.0 * total_sel + 3.0 * batch_size + 3.0);
    const double gbps = g_kernel > 0 ? step_bytes / (g_kernel * 1e-3) / 1e9 : 0.0;
    std::cout << std::fixed << std::setprecision(3) << "sparse_gpu_hbm_gbps=" << gbps << "\n"
              << "sparse_gpu_roofline_frac=" << gbps * 1e9 / kHbmBytesPerSec << "\n"
              << "sparse_gpu_roofline_peak_gbps=" << kHbmBytesPerSec / 1e9 << "\n"
              << "sparse_gpu_roofline_peak_source=" << g_hbm_source << "\n";
  }
  std::cout << "\n== Reading Guide ==\n"
            << "End-to-End Total(ms) is the full wall time for that path.\n"
            << "Speedup is dense_cpu_total_ms / path_total_ms.\n"
            << "For sparse_gpu, Gather is fused into attention, so gather_ms is zero.\n"
            << "Analytical floors use the measured B200 HBM copy bandwidth (6537 GB/s).\n";
  return 0;
}
