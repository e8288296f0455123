// planner_shim.hpp -- host stand-in for the nanobind CPU int64 array the reference's raw-byte run
// planner takes (test infrastructure only), so the planner compiles without nanobind / TTNN.
#pragma once

#include <cstddef>
#include <cstdint>
#include <cstring>
#include <limits>
#include <optional>
#include <vector>

struct CpuInt64Tensor {
  const int64_t *ptr;
  size_t n;
  size_t ndim() const { return 1; }
  size_t shape(size_t) const { return n; }
  const int64_t *data() const { return ptr; }
};
