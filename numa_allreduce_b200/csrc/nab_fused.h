// Fused tensor-parallel layer tail: allreduce of the row-parallel partial
// output, residual add and RMSNorm in one kernel (bf16).
//
//   z        = sum over ranks of inp  (fp32, rank order) + residual
//   residual = bf16(z)
//   out      = bf16(residual * rsqrt(mean(residual^2) + eps) * weight)
//
// No counterpart in the reference (it has no fused ops); this is the B200
// build's TP-layer path. The norm is computed from the bf16 residual, as an
// unfused "allreduce, then add, then RMSNorm" sequence would, so every rank
// can recompute it from gathered residual rows and all ranks agree bit for bit.
#pragma once

#include <cuda_runtime.h>

#include <vector>

#include "nab_comm.h"

namespace nab {

enum FusedAlgo : int { kFusedAuto = 0, kFusedOneshot = 1, kFusedTwoshot = 2 };

// Returns the protocol used.
int fused_allreduce_rmsnorm(Communicator& c, cudaStream_t s, const void* inp, void* residual,
                            const void* weight, void* out, int64_t T, int64_t H, float eps, int algo);

// Single-GPU emulation of the fused op over ws ranks (cooperative launch).
int emulate_fused_allreduce_rmsnorm(const std::vector<Communicator*>& comms, cudaStream_t s,
                                    const std::vector<const void*>& ins,
                                    const std::vector<void*>& residuals,
                                    const std::vector<const void*>& weights,
                                    const std::vector<void*>& outs, int64_t T, int64_t H, float eps,
                                    int algo);

// Second half of the fused GEMM + allreduce: every rank's bf16 [T, H] GEMM
// output lands in this rank's fused slots (written by the GEMM epilogues of
// the call whose epoch the signal pad holds), one flag per 128-feature x
// `tile_tokens`-token tile and rank; waits for the flags of each row's tiles
// (bounded), adds the ranks' rows in rank order with the residual and
// applies RMSNorm. tile_tokens == 0 skips the waits (slots already complete).
void slots_rmsnorm(Communicator& c, cudaStream_t s, void* residual, const void* weight, void* out, int64_t T,
                   int64_t H, float eps, int tile_tokens);

// Second half of the reduce-scatter GEMM + allreduce: this rank's slots hold
// every rank's partial of the rows it owns (t % ws == rank); reduces them in
// rank order + residual + RMSNorm, publishes the new residual rows in place,
// exchanges a flag with every peer and pulls the other owners' residual rows
// (recomputing their norm locally).
void slots_rs_rmsnorm(Communicator& c, cudaStream_t s, void* residual, const void* weight, void* out, int64_t T,
                      int64_t H, float eps, int tile_tokens);

// Local residual add + RMSNorm (no communication): the world-size-1 path and
// the norm of the unfused baseline.
void rmsnorm_residual(cudaStream_t s, const void* inp, void* residual, const void* weight, void* out,
                      int64_t T, int64_t H, float eps);

}  // namespace nab
