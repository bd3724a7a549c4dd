// Maps C ABI status codes onto the exception types the reference API throws.
#pragma once

#include <stdexcept>
#include <string>

#include "dsd_b200.h"

namespace dsd {
namespace detail {

inline void ThrowIf(int rc) {
  if (rc == DSD_OK) return;
  const std::string msg = dsd_last_error();
  if (rc == DSD_EINVAL) throw std::invalid_argument(msg);
  if (rc == DSD_ERANGE) throw std::out_of_range(msg);
  throw std::runtime_error(msg);
}

}  // namespace detail
}  // namespace dsd
