// Model and runtime configuration of the drop-in C++ API.
// Same fields and defaults as the reference's ModelConfig / RuntimeConfig
// (include/dsd/config.h:5-17) so existing callers compile unchanged.
#pragma once

namespace dsd {

struct ModelConfig {
  int num_heads = 4;
  int head_dim = 16;
  int page_size = 16;
  int top_k_pages = 4;
};

struct RuntimeConfig {
  int batch_size = 8;
  int seed = 7;
  bool enable_reordering = false;
  bool print_per_request = false;
};

}  // namespace dsd
