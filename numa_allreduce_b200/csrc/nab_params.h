// Kernel parameter block shared by the host runtime and the device kernels.
//
// One RankView describes everything a rank needs. A real multi-process launch
// fills v[0] and uses gridDim.y == 1. A single-GPU emulation launch fills
// v[0..ws) with one view per emulated rank (all buffers on the same GPU) and
// uses gridDim.y == ws with a cooperative launch, so the CTAs of different
// emulated ranks that wait on each other are guaranteed to be co-resident.
#pragma once

#include <cstdint>

#include "nab_common.h"

namespace nab {

struct RankView {
  const char* in;
  char* out;
  char* wsp[kMaxRanks];  // IPC workspace base of every rank, as mapped here
  const RankData* reg;   // peers' registered input pointers (pull protocol)
  const RankData* reg_end;  // end of this rank's RankData registry (debug bounds checks)
  char* mc;              // multicast address of the NVLS workspace (or null)
  char* uc;              // this rank's own unicast view of the NVLS workspace
  int rank;
  int pad_;
};

// Byte offsets inside the IPC workspace (ws_*) and the NVLS workspace (mc_*).
struct Layout {
  int64_t oneshot_off;    // [2 parities][ws slots][oneshot_max]
  int64_t oneshot_max;    // bytes per slot
  int64_t twoshot_off;    // [cta][ws rs slots + 1 result][chunk_max]
  int64_t hier_off;       // [cta][gsize rs + 2*ngroups*2 fp32 partials + 1 result][hier_chunk]
  int64_t pipe_off;       // pipelined two-shot: [cta][ring slot][ws rs + ws ag chunks][pipe_chunk]
  int64_t pipe_chunk;     // bytes per owner chunk in a ring slot
  int64_t fused_off;      // fused one-shot: [2 parities][ws slots][fused_bytes]
  int64_t fused_bytes;    // bytes per fused one-shot slot
  int64_t fused2_off;     // fused two-shot: [cta][ws rs rows + 1 result row][kFusedMaxHidden*2]
  int64_t chunk_max;      // bytes per owner chunk per round (two-shot protocols)
  int64_t hier_chunk;     // bytes per owner chunk per round (hierarchical protocol)
  int64_t ws_bytes;       // total IPC workspace bytes
  int64_t mc_oneshot_off; // [2 parities][oneshot_max]
  int64_t mc_twoshot_off; // [cta][ring slot][ws chunks][nvls_chunk]
  int64_t nvls_chunk;     // bytes per owner chunk in a ring slot
  int64_t mc_bytes;
  int max_ctas;           // CTA slots the workspace was sized for
  int hier_ctas;          // CTA slots of the hierarchical region
  int pipe_ctas;          // CTA slots of the pipelined two-shot ring
  int pad2_;
};

struct ARParams {
  RankView v[kMaxRanks];
  ErrorState* err;
  uint32_t* err_host;
  int64_t npacks;        // message size in 16-byte packs
  uint64_t timeout_ns;
  int ws;
  int chunk_packs;       // packs per owner chunk per round
  int rounds;            // rounds per CTA
  int ngroups;           // hierarchical: number of groups
  int gsize;             // hierarchical: ranks per group
  int hyb_ctas;          // hybrid: CTAs [0, hyb_ctas) run the P2P part
  int chunk_packs2;      // hybrid: packs per owner chunk of the NVLS part
  int pad3_;
  int64_t split_packs;   // hybrid: packs [0, split_packs) go P2P, the rest NVLS
  int64_t seg_stride;    // reduce-scatter input / all-gather output: packs between rank segments
  int8_t group_of[kMaxRanks];
  int8_t lidx_of[kMaxRanks];
  int8_t member[kMaxRanks][kMaxRanks];  // [group][local index] -> rank
  Layout L;
};

}  // namespace nab
