// Writes this build's continuous workload generator output to a file, so the
// Python tests can compare it with the oracle, the reference and the golden
// fixtures byte for byte.
//
//   dump_workload specs  H D N window min_prompt max_prompt min_decode max_decode seed OUT
//       int32 ids[N], arrivals[N], prompt_tokens[N], decode_steps[N], then
//       float32 prompt keys (packed), prompt values (packed), initial queries [N][E]
//   dump_workload specs_only ...same arguments...
//       the same layout from BuildSyntheticContinuousSpecs (no prompt payloads)
//   dump_workload tokens COUNT REQUEST STEP STREAM OUT
//       float32 DeterministicTokenVector(COUNT, REQUEST, STEP, STREAM)
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <vector>

#include "dsd/continuous_batching.h"

namespace {

void Write(std::FILE* f, const void* p, std::size_t bytes) {
  if (bytes != 0 && std::fwrite(p, 1, bytes, f) != bytes) {
    std::perror("fwrite");
    std::exit(1);
  }
}

}  // namespace

int main(int argc, char** argv) {
  const bool specs_only = argc == 12 && std::strcmp(argv[1], "specs_only") == 0;
  if (argc == 12 && (specs_only || std::strcmp(argv[1], "specs") == 0)) {
    int a[9];
    for (int i = 0; i < 9; ++i) a[i] = std::atoi(argv[2 + i]);
    dsd::ModelConfig c;
    c.num_heads = a[0];
    c.head_dim = a[1];
    const auto specs =
        specs_only
            ? dsd::BuildSyntheticContinuousSpecs(c, a[2], a[3], a[4], a[5], a[6], a[7], a[8])
            : dsd::BuildSyntheticContinuousWorkload(c, a[2], a[3], a[4], a[5], a[6], a[7], a[8]);
    std::FILE* f = std::fopen(argv[11], "wb");
    if (f == nullptr) return 1;
    std::vector<int> col(specs.size());
    for (int field = 0; field < 4; ++field) {
      for (std::size_t i = 0; i < specs.size(); ++i) {
        const auto& s = specs[i];
        col[i] = field == 0 ? s.request_id
               : field == 1 ? s.arrival_step
               : field == 2 ? s.prompt_tokens
                            : s.decode_steps;
      }
      Write(f, col.data(), col.size() * sizeof(int));
    }
    for (const auto& s : specs) Write(f, s.prompt_keys.data(), s.prompt_keys.size() * 4);
    for (const auto& s : specs) Write(f, s.prompt_values.data(), s.prompt_values.size() * 4);
    for (const auto& s : specs) Write(f, s.initial_query.data(), s.initial_query.size() * 4);
    std::fclose(f);
    return 0;
  }
  if (argc == 7 && std::strcmp(argv[1], "tokens") == 0) {
    const auto v = dsd::DeterministicTokenVector(std::atoi(argv[2]), std::atoi(argv[3]),
                                                 std::atoi(argv[4]), std::atoi(argv[5]));
    std::FILE* f = std::fopen(argv[6], "wb");
    if (f == nullptr) return 1;
    Write(f, v.data(), v.size() * 4);
    std::fclose(f);
    return 0;
  }
  std::fprintf(stderr, "usage: dump_workload specs H D N W minp maxp mind maxd seed OUT | "
                       "tokens COUNT REQ STEP STREAM OUT\n");
  return 2;
}
