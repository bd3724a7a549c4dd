// ref_cb_shim.cpp -- flat C entry points over the reference's continuous
// workload generator.
//
// TEST INFRASTRUCTURE ONLY.  The reference keeps MixSeed and
// DeterministicTokenVector in an anonymous namespace of
// src/continuous_batching.cpp (:44-59), so they cannot be linked from another
// translation unit.  This file compiles that source file, unmodified and where
// it lies (oracle/Makefile passes -I<reference root>), into the same
// translation unit and exports:
//   ref_deterministic_token_vector  DeterministicTokenVector (:52-59)
//   ref_continuous_workload         BuildSyntheticContinuousWorkload (:336-381)
// with the argument layout of the oracle's orc_* restatements, so that tests
// can compare the two bit for bit.  oracle/Makefile links this object in place
// of the separately compiled continuous_batching.o.

#include "src/continuous_batching.cpp"

#include <cstring>

extern "C" {

void ref_deterministic_token_vector(int count, int request_id, int decode_step, int stream,
                                    float* out) {
  const auto v = dsd::DeterministicTokenVector(count, request_id, decode_step, stream);
  std::memcpy(out, v.data(), v.size() * sizeof(float));
}

// Specs in the reference's (arrival, id) order.  Payload pointers may be null
// (sizes only); otherwise prompts are packed back to back ([sum prompt][E])
// and initial queries [N][E], in the same order.
void ref_continuous_workload(int num_heads, int head_dim, int num_requests, int arrival_window,
                             int min_prompt, int max_prompt, int min_decode, int max_decode,
                             int seed, int* request_ids, int* arrival_steps, int* prompt_tokens,
                             int* decode_steps, float* prompt_keys, float* prompt_values,
                             float* initial_queries) {
  dsd::ModelConfig c;
  c.num_heads = num_heads;
  c.head_dim = head_dim;
  const auto specs = dsd::BuildSyntheticContinuousWorkload(
      c, num_requests, arrival_window, min_prompt, max_prompt, min_decode, max_decode, seed);
  long long off = 0;
  const int ept = num_heads * head_dim;
  for (std::size_t i = 0; i < specs.size(); ++i) {
    const auto& s = specs[i];
    request_ids[i] = s.request_id;
    arrival_steps[i] = s.arrival_step;
    prompt_tokens[i] = s.prompt_tokens;
    decode_steps[i] = s.decode_steps;
    if (prompt_keys != nullptr) {
      std::memcpy(prompt_keys + off, s.prompt_keys.data(), s.prompt_keys.size() * sizeof(float));
      std::memcpy(prompt_values + off, s.prompt_values.data(),
                  s.prompt_values.size() * sizeof(float));
      std::memcpy(initial_queries + static_cast<long long>(i) * ept, s.initial_query.data(),
                  s.initial_query.size() * sizeof(float));
      off += static_cast<long long>(s.prompt_keys.size());
    }
  }
}

}  // extern "C"
