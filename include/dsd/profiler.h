// Host wall-clock helpers (the reference's ScopedStageTimer and TimeHostMs,
// include/dsd/profiler.h:7-27, include/dsd/cuda_utils.h:16-41).
#pragma once

#include <chrono>
#include <type_traits>

namespace dsd {

// Adds the lifetime of the object, in ms, to *sink_ms (nothing when null).
class ScopedStageTimer {
 public:
  explicit ScopedStageTimer(double* sink_ms)
      : sink_ms_(sink_ms), start_(std::chrono::steady_clock::now()) {}
  ~ScopedStageTimer() {
    if (sink_ms_)
      *sink_ms_ += std::chrono::duration<double, std::milli>(
                       std::chrono::steady_clock::now() - start_).count();
  }
  ScopedStageTimer(const ScopedStageTimer&) = delete;
  ScopedStageTimer& operator=(const ScopedStageTimer&) = delete;

 private:
  double* sink_ms_;
  std::chrono::steady_clock::time_point start_;
};

// Runs fn() and adds its wall time to *sink_ms when sink_ms is not null.
template <typename Fn>
auto TimeHostMs(double* sink_ms, Fn&& fn) -> decltype(fn()) {
  ScopedStageTimer timer(sink_ms);
  return fn();
}

}  // namespace dsd
