// Process-wide count of mtorus kernel launches (shared by every translation unit
// of the kernel extension; read by the benchmark for its launch count).
#pragma once
#include <cstdint>

namespace mtorus {
inline int64_t& launch_counter() {
  static int64_t n = 0;
  return n;
}
}  // namespace mtorus
