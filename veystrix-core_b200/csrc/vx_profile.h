// Stage timing hooks used by the entry points (no-ops unless enabled).
#pragma once

#include <cuda_runtime.h>

namespace vx {
bool profile_on();
// Record an event on `st`; `label` names the stage that ends here, an empty
// label opens a new call.
void profile_mark(cudaStream_t st, const char* label);
}  // namespace vx
