// Common definitions shared by host and device code of the native allreduce core.
//
// Capability parity: the reference's constants kMaxBlocks/kMaxGPUs and its
// Signal/RankData structs (src/numa_all_reduce.cu:39-72). This build sizes the
// flag arrays for a full B200 (148 SMs) instead of 36 blocks, keeps one flag
// array per protocol so protocols never share epochs, and adds an error word
// that bounded waits write instead of hanging.
#pragma once

#include <cstddef>
#include <cstdint>

namespace nab {

constexpr int kMaxRanks = 8;
// Flag slots per protocol: one per CTA index. 160 >= 148 SMs of a B200.
constexpr int kMaxBlocks = 160;
// Output tiles (128 features x up to 256 tokens) of one GEMM + allreduce call.
constexpr int kGemmMaxTiles = 1024;

enum DType : int { kF32 = 0, kF16 = 1, kBF16 = 2 };

// Algorithm identifiers. The numeric values are part of the C ABI and of the
// tuning-table file format, so they never change meaning.
enum Algo : int {
  kAlgoAuto = 0,
  kAlgoOneshot = 1,      // push whole input to every peer, each rank reduces all
  kAlgoTwoshot = 2,      // push reduce-scatter, pull all-gather, tiled rounds
  kAlgoNvlsOneshot = 3,  // multimem.ld_reduce of the whole message
  kAlgoNvlsTwoshot = 4,  // multimem.ld_reduce own slice + multimem.st broadcast
  kAlgoHier = 5,         // 3-stage: intra-group RS, inter-group AR, intra-group AG
  kAlgoOneshotPull = 6,  // registered inputs: read peers' buffers directly
  kAlgoCopy = 7,         // world size 1: out = in
  kAlgoTwoshotPipe = 8,  // two-shot, warp-specialised and pipelined over a slot ring
  kAlgoHybrid = 9,       // one launch: P2P pipelined two-shot on a prefix, NVLS two-shot on the rest
  kAlgoCount = 10,
  // Not allreduce protocols (never in a tuning table): the contiguous-segment
  // reduce-scatter and all-gather collectives on the one-shot slots.
  kAlgoReduceScatter = 20,
  kAlgoAllGather = 21,
  kAlgoNccl = 100,       // selector result only: the caller should use NCCL
};

// Error codes written into ErrorState::code by device code.
enum ErrCode : uint32_t {
  kErrNone = 0,
  kErrTimeout = 1,       // a bounded wait on a peer flag ran out
  kErrBadLaunch = 2,     // launch-time argument check failed on device
};

// Stage tags recorded with a timeout so the host can say where it happened.
enum Stage : uint32_t {
  kStageOneshot = 1,
  kStageRS = 2,
  kStageAG = 3,
  kStageHierX = 4,
  kStagePullStart = 5,
  kStagePullEnd = 6,
  kStageNvls1 = 7,
  kStageNvls2 = 8,
  kStageFused = 9,
  kStageGemmAR = 10,
  kStageGemm = 11,       // plain GEMM: its own TMA / tensor-core mbarriers
  kStageAttn = 12,       // decode attention: its own bulk-copy mbarriers
  kStageBounds = 13,     // debug builds: an index failed a bounds check
  kStageReduceScatter = 14,
  kStageAllGather = 15,
};

// Lives in host-mapped pinned memory so the host can read it at any time, even
// when the stream has not been synchronised.
struct ErrorState {
  uint32_t code;
  uint32_t rank;
  uint32_t peer;
  uint32_t stage;
  uint32_t block;
  uint32_t epoch;
  uint32_t observed;
  uint32_t count;  // number of waits that gave up (all CTAs)
};

// Flag arrays of one rank, in its IPC-shared workspace. Peers write into
// [block][their rank]; the owner polls its own copy. Values are 64-bit
// sequence numbers ((epoch << 20) | round) that only ever grow, so a flag
// left over from an old call can never look current.
struct alignas(128) FlagArray {
  uint64_t v[kMaxBlocks][kMaxRanks];
};

enum FlagKind : int {
  kFlagOneshot = 0,
  kFlagRS,
  kFlagAG,
  kFlagHierRS,
  kFlagHierX,
  kFlagHierAG,
  kFlagPullStart,
  kFlagPullEnd,
  kFlagFused,
  kFlagFusedRS,
  kFlagFusedAG,
  kFlagPipeRS,  // pipelined two-shot: tiles pushed to this rank, per CTA
  kFlagPipeAG,  // pipelined two-shot: tiles reduced by the owner, per CTA
  kFlagScatter, // reduce-scatter collective: segments pushed to their owners
  kFlagGather,  // all-gather collective: this rank's segment pushed to every peer
  kFlagCount,
};

struct alignas(128) SignalPad {
  FlagArray flags[kFlagCount];
  // Per-call epoch: read by every CTA at kernel start, advanced by the last
  // CTA to finish. One counter for all protocols, so a protocol switch
  // between calls never reuses a double-buffer parity too early.
  alignas(128) uint32_t epoch;
  uint32_t done_ctas;
  // Set by a CTA whose wait gave up; every later wait of this rank returns at
  // once. Cleared only by the host (Communicator::reset).
  uint32_t abort;
  uint32_t pad_[29];
  // Rounds each CTA index has completed in the hierarchical protocol; the
  // same on every rank. Its parity picks the double-buffered stage-2 slots.
  alignas(128) uint32_t hier_rounds[kMaxBlocks];
  // GEMM + allreduce: rank r raises [tile][r] on every rank once its output
  // tile is in every rank's slot.
  alignas(128) uint64_t gemm_flags[kGemmMaxTiles][kMaxRanks];
};

// Header of the NVLS (multicast) workspace. The counters are incremented on
// every GPU at once with multimem.red; `rounds` is local bookkeeping: how many
// rounds each CTA index has completed, identical on every rank.
struct alignas(128) NvlsPad {
  // [cta][counter], 32 B apart: 0 and 1 are the two arrival phases of the
  // two-shot protocol, 2 the one-shot arrival. Each protocol owns its
  // counters because each tracks its own expected count in `rounds`.
  uint32_t cnt[kMaxBlocks][3][8];
  uint32_t rounds[kMaxBlocks][2];  // [cta][0]=twoshot rounds, [cta][1]=oneshot calls
  // Pipelined two-shot: arrival counters per [cta][ring slot][phase] (phase 0:
  // tile copied in on every GPU, 1: tile reduced and broadcast by every owner)
  // and the number of tiles each CTA index has pushed through its ring.
  uint32_t pipe[kMaxBlocks][4][2][8];
  uint32_t pipe_tiles[kMaxBlocks];
};

// Ring depth, CTA count and tile size of the pipelined P2P two-shot kernel.
constexpr int kPipeSlots = 4;
constexpr int kPipeCtas = 128;
constexpr int64_t kPipeTileBytes = 256 << 10;

// Ring depth and CTA count of the pipelined NVLS two-shot kernel.
constexpr int kNvlsSlots = 4;
constexpr int kNvlsCtas = 128;
constexpr int64_t kNvlsTileBytes = 256 << 10;  // one ring slot: ws chunks

// Default split of the hybrid protocol (P2P share of the message in per
// mille, CTAs of each part; their sum stays below the 148 SMs so every CTA of
// the launch is resident at once).
constexpr int kHybridP2pPermille = 400;
constexpr int kHybridP2pCtas = 64;
constexpr int kHybridNvlsCtas = 80;

constexpr uint64_t kSeqShift = 20;  // rounds per call < 2^20

// Largest row (hidden size) of the fused allreduce + RMSNorm kernels.
constexpr int kFusedMaxHidden = 16384;

// Peer pointers of one registered buffer (the reference's RankData).
struct alignas(16) RankData {
  const void* ptrs[kMaxRanks];
};

}  // namespace nab
