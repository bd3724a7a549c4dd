// Minimal check helpers for the C++ test programs (exit code 1 on failure).
#pragma once

#include <cstdlib>
#include <iostream>
#include <string>

#define CHECK(cond, msg)                                                             \
  do {                                                                               \
    if (!(cond)) {                                                                   \
      std::cerr << __FILE__ << ":" << __LINE__ << ": " << (msg) << "\n";             \
      std::exit(1);                                                                  \
    }                                                                                \
  } while (0)

template <typename Ex, typename Fn>
bool Throws(Fn&& fn) {
  try {
    fn();
  } catch (const Ex&) {
    return true;
  } catch (...) {
    return false;
  }
  return false;
}
