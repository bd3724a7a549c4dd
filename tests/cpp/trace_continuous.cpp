// Runs this build's continuous serving loop (RunContinuousSparseDecode, the
// dsd_continuous_bench path) with a step observer and writes every step to a
// binary trace, so that a test can check each step against the oracle.
//
//   trace_continuous OUT N max_active window min_prompt max_prompt min_decode
//                    max_decode seed H D P K admission preadmit precompute
//                    gpu_append lazy_release kv_format
//
// admission: 1 direct GPU upload of the reference generator's payloads,
// 2 synthetic GPU prefill (specs without payloads).  Output mode is
// kDebugTensors (selected ids and scores come back).  Trace, all int32 /
// float32 little endian: per step
//   B, then per request: request_id, context_tokens, n_pages, pages[n_pages],
//   query[E], n_sel, selected[n_sel], scores[n_pages], output[E]
// terminated by B = -1; then generated tokens as one int32.
#include <cstdio>
#include <cstdlib>
#include <vector>

#include "dsd/continuous_batching.h"

namespace {
std::FILE* g_out = nullptr;
void W(const void* p, std::size_t bytes) {
  if (bytes && std::fwrite(p, 1, bytes, g_out) != bytes) {
    std::perror("fwrite");
    std::exit(1);
  }
}
void Wi(int v) { W(&v, 4); }
}  // namespace

int main(int argc, char** argv) {
  if (argc != 20) {
    std::fprintf(stderr, "usage: see the header of trace_continuous.cpp\n");
    return 2;
  }
  int a[19];
  for (int i = 0; i < 18; ++i) a[i] = std::atoi(argv[2 + i]);
  dsd::ModelConfig c;
  c.num_heads = a[8];
  c.head_dim = a[9];
  c.page_size = a[10];
  c.top_k_pages = a[11];
  const int admission = a[12];
  const auto specs =
      admission == 2
          ? dsd::BuildSyntheticContinuousSpecs(c, a[0], a[2], a[3], a[4], a[5], a[6], a[7])
          : dsd::BuildSyntheticContinuousWorkload(c, a[0], a[2], a[3], a[4], a[5], a[6], a[7]);
  dsd::ContinuousDecodeOptions o;
  o.max_active_requests = a[1];
  o.prompt_admission_mode = admission == 2
                                ? dsd::ContinuousPromptAdmissionMode::kSyntheticGpuPrefill
                                : dsd::ContinuousPromptAdmissionMode::kDirectGpuUpload;
  o.preadmit_prompts = a[13] != 0;
  o.precompute_decode_payloads = a[14] != 0;
  o.gpu_synthetic_decode_append = a[15] != 0;
  o.lazy_release = a[16] != 0;
  o.kv_format = a[17];
  o.run_batch_output_mode = dsd::SparseBatchOutputMode::kDebugTensors;
  g_out = std::fopen(argv[1], "wb");
  if (!g_out) return 1;
  o.step_observer = [](const dsd::ContinuousStepRecord& r) {
    const int b = static_cast<int>(r.request_ids.size());
    Wi(b);
    for (int i = 0; i < b; ++i) {
      const auto& res = r.result->per_request[static_cast<std::size_t>(i)];
      const auto& pages = r.candidate_page_ids[static_cast<std::size_t>(i)];
      Wi(r.request_ids[static_cast<std::size_t>(i)]);
      Wi(r.context_tokens[static_cast<std::size_t>(i)]);
      Wi(static_cast<int>(pages.size()));
      W(pages.data(), pages.size() * 4);
      const auto& q = r.queries[static_cast<std::size_t>(i)];
      W(q.data(), q.size() * 4);
      Wi(static_cast<int>(res.selected_page_ids.size()));
      W(res.selected_page_ids.data(), res.selected_page_ids.size() * 4);
      if (res.scores.size() != pages.size()) {
        std::fprintf(stderr, "score count %zu != pages %zu\n", res.scores.size(), pages.size());
        std::exit(1);
      }
      for (const auto& s : res.scores) W(&s.score, 4);
      W(res.output.output.data(), res.output.output.size() * 4);
    }
  };
  const auto stats = dsd::RunContinuousSparseDecode(c, specs, o);
  Wi(-1);
  Wi(stats.total_generated_tokens);
  std::fclose(g_out);
  std::printf("generated=%d\n", stats.total_generated_tokens);
  return 0;
}
