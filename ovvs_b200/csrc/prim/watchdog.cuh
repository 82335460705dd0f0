// Kernel watchdog self test (see watchdog.cu).
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace ovvs {
namespace prim {

constexpr int kErrSelfTest = 0x201;

cudaError_t launch_watchdog_selftest(int* err, uint64_t limit_ns, cudaStream_t stream);

}  // namespace prim
}  // namespace ovvs
