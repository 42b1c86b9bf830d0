// Host-callable launchers of the device kernels (no torch dependency).
#pragma once

#include <cuda_runtime.h>

#include "nab_params.h"

namespace nab {

int allreduce_threads();

// Launches one allreduce kernel. grid.y must be 1 for a real launch and ws for
// a single-GPU emulation launch (which must also be cooperative).
cudaError_t launch_allreduce(int algo, int dtype, const ARParams& p, dim3 grid, cudaStream_t s,
                             bool cooperative);

}  // namespace nab
