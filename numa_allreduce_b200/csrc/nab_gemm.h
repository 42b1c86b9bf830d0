// tcgen05 GEMM entry points (see nab_gemm_sm100.cu).
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

#include "nab_comm.h"

namespace nab {

// y[T, N] = x[T, K] . wt[N, K]^T in bf16 with fp32 accumulation. N must be a
// multiple of 128 and K of 64. With splits > 1 the K loop is split over that
// many CTAs per tile; splitk_ws must then hold splits * T * N floats.
void gemm_bf16(cudaStream_t s, const void* wt, const void* x, void* y, int T, int N, int K, float* splitk_ws,
               int64_t splitk_ws_floats, int splits);

// Split count that gives enough CTAs to stream the weight from every SM.
int gemm_splits_for(int T, int N, int K, int sms);

// Row-parallel layer tail in two launches: the GEMM whose epilogue stores its
// bf16 partial tiles into every rank's slot over NVLink (with a per-tile flag
// exchange), then the rank-order sum + residual add + RMSNorm from the slots.
// residual is updated in place; out receives the normalised activations.
// splits <= 0 picks the split-K factor; with more than one split the
// partials travel in fp32 (one per split), otherwise in bf16. Returns the
// split count used.
int gemm_allreduce_rmsnorm(Communicator& c, cudaStream_t s, const void* wt, const void* x, void* residual,
                           const void* weight, void* out, int T, int N, int K, float eps, int splits);

}  // namespace nab
