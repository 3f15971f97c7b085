// NVLink / NVSwitch collective kernels over symmetric memory (see comm.cu).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace b200 {
}  // namespace b200
