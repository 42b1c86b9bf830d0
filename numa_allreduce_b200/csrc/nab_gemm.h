// tcgen05 GEMM entry points (see nab_gemm_sm100.cu).
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

#include "nab_comm.h"

namespace nab {

// y[T, N] = x[T, K] . wt[N, K]^T in bf16 with fp32 accumulation. N must be a
// multiple of 128 and K of 64. With splits > 1 the K loop of each output tile
// is split over that many CTAs (at most 16), launched as one thread-block
// cluster that adds the fp32 partials in split order over distributed
// shared memory; splits <= 0 picks the count (gemm_splits_for).
// packed: wt is in the tiled layout of pack_weight_tiles — [N/128][K/64] tiles
// of 128 rows x 64 columns, each 16 KB contiguous — so every weight TMA load
// reads one contiguous block of HBM instead of 128 rows 2K bytes apart.
// Launched as a programmatic dependent launch: the weight loads may start
// while the kernel before it in the stream still runs, if that kernel is one
// of this library's (they allow early launch); such a kernel must not write
// wt. Activations are read only after it completed.
// swiglu: every 128-row tile of wt holds 64 gate rows followed by the 64
// matching up rows (interleave_gate_up); y is then [T, N/2] with
// y = silu(gate) * up computed from the fp32 accumulators.
void gemm_bf16(cudaStream_t s, const void* wt, const void* x, void* y, int T, int N, int K, int splits,
               bool packed = false, bool swiglu = false);

// Split count that balances the CTAs over the SMs.
int gemm_splits_for(int T, int N, int K, int sms);
// Clusters of cs CTAs of the bn-token-wide kernel the device runs at once.
int gemm_active_clusters(int bn, int cs);

// Row-parallel layer tail in two launches, in one of two modes:
//  one-shot        the GEMM's epilogue stores each finished bf16 output tile
//                  into this rank's slot on every rank over NVLink and raises
//                  the tile's flag there; the second kernel waits for each
//                  row's tiles and does the rank-order sum + residual add +
//                  RMSNorm of every row;
//  reduce-scatter  the epilogue stores token row t only into its owner rank
//                  t % ws; the second kernel reduces the owned rows (rank
//                  order) + residual + RMSNorm, publishes each new residual
//                  row in place, and every rank pulls the other owners'
//                  residual rows and recomputes the norm locally:
//                  2 (ws - 1) / ws of the output crosses NVLink instead of
//                  (ws - 1) times it.
// residual is updated in place; out receives the normalised activations.
// splits as for gemm_bf16 (split partials are added on this GPU, so only
// bf16 tiles cross NVLink). Returns the split count used.
enum GemmArMode : int { kGemmArAuto = 0, kGemmArOneshot = 1, kGemmArReduceScatter = 2 };
int gemm_allreduce_rmsnorm(Communicator& c, cudaStream_t s, const void* wt, const void* x, void* residual,
                           const void* weight, void* out, int T, int N, int K, float eps, int splits,
                           bool packed = false, int mode = kGemmArAuto);
// The mode kGemmArAuto picks for T tokens on ws ranks.
int gemm_ar_mode_for(int T, int ws);

}  // namespace nab
