// fiber.h — NDRange executor for kernels compiled through clshim.h.
// TEST INFRASTRUCTURE ONLY.
#pragma once
#include <functional>
#include "clshim.h"

namespace clshim {
// Runs `call` (which invokes one kernel with its arguments) for every
// work-item of an NDRange: global[d] must be a multiple of local[d]; dims <= 2.
// Work-groups are spread over OpenMP threads; the work-items of a group run as
// fibers on one thread.
void run_ndrange(const size_t global[2], const size_t local[2], const std::function<void()>& call);
// The same over three dimensions.
void run_ndrange3(const size_t global[3], const size_t local[3], const std::function<void()>& call);
}  // namespace clshim
