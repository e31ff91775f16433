// Launch counter of the _gemm extension.
#include "common.cuh"

namespace pd {
long long launches() { return launch_counter().load(); }
}  // namespace pd
