// Host-side launch helpers shared by the kernel files and the C ABI layer.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace exf {

// Blocks that fill every SM of the current device at the kernel's occupancy (cached per
// device and kernel); 0 if the query fails.
int persistent_grid(const void* kernel, int threads, size_t dynamic_smem);
int sm_count();

}  // namespace exf
