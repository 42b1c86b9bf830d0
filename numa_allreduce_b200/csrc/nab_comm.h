// Host runtime of the allreduce library (no torch dependency).
//
// Capability parity: the reference's host class NumaAwareAllReduceImpl
// (src/numa_all_reduce.cu:347-556: rank/NUMA maps, RankData registry,
// per-stage launchers) and the buffer/graph bookkeeping it delegates to
// vllm::CustomAllreduce (src/numa_all_reduce.cu:577-691). Here the
// three-stage schedule is real (groups may be any equal-size partition, not
// only contiguous ranks), and every launch carries a timeout and an error
// word instead of spinning forever.
#pragma once

#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>
#include <map>
#include <string>
#include <unordered_map>
#include <utility>
#include <vector>

#include "nab_common.h"
#include "nab_device_flags.h"
#include "nab_params.h"

namespace nab {

struct CommConfig {
  int64_t oneshot_max = 1 << 20;  // largest message of the one-shot protocols
  // Bytes per owner chunk per round of the two-shot protocols; 0 picks
  // 512 KiB / world size (a CTA moves ~512 KiB per round at any world size).
  int64_t chunk_max = 0;
  int max_ctas = 128;             // CTAs of the round-based tiled protocols
  // One-shot launch shape: a CTA per oneshot_grain packs (16 B), at most
  // oneshot_ctas (measured on 8 B200s: 512 x 64 was at least as fast as any
  // other shape at every size up to 1 MiB, eager and in CUDA graphs)
  int oneshot_ctas = 64;
  int oneshot_grain = 512;
  int64_t fused_bytes = 512 << 10;  // fused one-shot slot (allreduce + norm)
  uint64_t timeout_ns = 5000000000ull;
  int pipe_ctas = kPipeCtas;             // CTAs of the pipelined two-shot
  int64_t pipe_tile = kPipeTileBytes;    // bytes per ring slot of the pipelined two-shot
  // Hybrid protocol: share of the message (per mille) that takes the P2P
  // two-shot, and the CTA budget of each part (the rest goes through NVLS).
  int hybrid_p2p_permille = kHybridP2pPermille;
  int hybrid_p2p_ctas = kHybridP2pCtas;
  int hybrid_nvls_ctas = kHybridNvlsCtas;
};

// Config from a flat list: [oneshot_max, chunk_max, max_ctas, oneshot_ctas,
// fused_bytes, timeout_ns, pipe_ctas, pipe_tile, hybrid_p2p_permille,
// hybrid_p2p_ctas, hybrid_nvls_ctas, oneshot_grain]; missing or negative
// entries keep their defaults.
CommConfig config_from_list(const std::vector<int64_t>& v);

// Protocol steps of the automatic choice for one dtype: the first step whose
// max_bytes >= the message size gives the protocol; a larger message gets
// `fallback` (kAlgoNccl: the caller should use NCCL). The Python selector
// (parallel/select.py) loads the same table and hands it to the communicator,
// so both make the same choice; without a table both use builtin_auto_table().
struct AutoStep {
  int64_t max_bytes;
  int algo;
};
struct AutoTable {
  std::vector<AutoStep> steps;
  int fallback = kAlgoNccl;
};

// Built-in steps for a world size (used when no measured table covers it).
AutoTable builtin_auto_table(int ws, bool has_nvls);
// The protocol the table picks, after substituting what this communicator
// cannot run (NVLS and hybrid need a multicast workspace, hier needs groups).
// kAlgoNccl means "use NCCL"; kAlgoCopy for world size 1.
int choose_auto(const AutoTable& t, int ws, int64_t nbytes, bool has_nvls, bool has_groups);

// Computes where everything lives in the IPC and NVLS workspaces.
Layout make_layout(int ws, const CommConfig& cfg);

struct LaunchPlan {
  int algo = kAlgoAuto;
  dim3 grid{1, 1, 1};
  int chunk_packs = 0;
  int rounds = 0;
  int hyb_ctas = 0;       // hybrid only
  int chunk_packs2 = 0;
  int64_t split_packs = 0;
};

class Communicator {
 public:
  // wsp: IPC workspace base of every rank as mapped in this process (each was
  // sized with make_layout(ws, cfg).ws_bytes and zero-initialised).
  // rank_data: device memory for the RankData registry.
  Communicator(int rank, int ws, const std::vector<char*>& wsp, void* rank_data,
               size_t rank_data_bytes, const CommConfig& cfg, bool full_nvlink);
  ~Communicator();
  Communicator(const Communicator&) = delete;
  Communicator& operator=(const Communicator&) = delete;

  int rank() const { return rank_; }
  int world_size() const { return ws_; }
  const Layout& layout() const { return L_; }
  const CommConfig& config() const { return cfg_; }
  bool has_nvls() const { return mc_ != nullptr; }
  bool has_groups() const { return ngroups_ > 0; }

  // Replaces the automatic-choice table of one dtype (kF32/kF16/kBF16).
  void set_auto_table(int dtype, const AutoTable& t);
  const AutoTable& auto_table(int dtype) const;
  // Changes the hybrid protocol's split at run time (tuning sweeps).
  void set_hybrid(int p2p_permille, int p2p_ctas, int nvls_ctas);

  // Hierarchical groups: equal-size partition of the ranks.
  void set_groups(const std::vector<std::vector<int>>& groups);
  // NVLS workspace: multicast VA and this rank's own unicast VA of it.
  void attach_nvls(char* mc, char* uc, int64_t bytes);

  // Registers an IPC-shared buffer (ptrs[rank] is local) for the pull path.
  void register_buffer(const std::vector<void*>& ptrs);
  // During CUDA-graph capture, pull launches on unregistered inputs reserve a
  // RankData slot; these two fill the slots after capture (reference
  // src/numa_all_reduce.cu:673-691 and src/numa_all_reduce.py:395-413).
  std::pair<std::string, std::vector<int64_t>> graph_buffer_ipc_meta();
  void register_graph_buffers(const std::vector<std::string>& handles,
                              const std::vector<std::vector<int64_t>>& offsets);
  size_t num_graph_buffers() const { return graph_unreg_.size(); }

  // Chooses the protocol when algo == kAlgoAuto and sizes the launch. A
  // message the table hands to NCCL gets the table's last custom protocol
  // here: a caller of the C ABI has no NCCL to fall back to.
  LaunchPlan plan(int64_t nbytes, int algo, bool registered, int dtype = kBF16) const;
  // Fills the view of this rank for a launch.
  RankView view(const void* in, void* out, const RankData* reg) const;
  // Fills everything but the views.
  void fill_params(ARParams& p, const LaunchPlan& pl, int64_t nbytes) const;

  // out = sum over ranks of in. Returns the protocol used. Throws
  // std::runtime_error on bad arguments or launch failure.
  int allreduce(cudaStream_t s, const void* in, void* out, int64_t nbytes, int dtype, int algo,
                bool registered);

  // Contiguous-segment collectives; seg_bytes is one rank's segment (a
  // positive multiple of 16). reduce_scatter: in holds ws segments, out gets
  // the sum of every rank's segment [rank]. all_gather: in is one segment,
  // out gets the ws ranks' segments in rank order. One launch per piece of at
  // most oneshot_max bytes per segment; returns the number of launches.
  int reduce_scatter(cudaStream_t s, const void* in, void* out, int64_t seg_bytes, int dtype);
  int all_gather(cudaStream_t s, const void* in, void* out, int64_t seg_bytes, int dtype);
  // Launch shape of one piece of those collectives (grid.x CTAs).
  dim3 collective_grid(int64_t piece_bytes) const;

  // Error state written by bounded waits.
  uint32_t error_code() const;  // from host-mapped memory, no sync
  ErrorState error_state() const;  // synchronous copy of the full record
  // Clears the error record, the abort word and all flags/epochs of this
  // rank's signal pad. All ranks must do this together (host barrier) before
  // the next launch.
  void reset();

  int64_t launches() const { return launches_.load(); }
  void count_launch() { launches_.fetch_add(1); }

  // Used by the fused kernels.
  ErrorState* err_dev() const { return err_dev_; }
  uint32_t* err_host() const { return err_host_; }
  char* wsp(int r) const { return wsp_[r]; }
  char* mc() const { return mc_; }
  char* uc() const { return uc_; }

 private:
  RankData* reserve_rank_data();

  int rank_;
  int ws_;
  int device_;
  CommConfig cfg_;
  Layout L_;
  bool full_nvlink_;
  std::vector<char*> wsp_;
  char* mc_ = nullptr;
  char* uc_ = nullptr;
  int64_t mc_bytes_ = 0;
  int ngroups_ = 0, gsize_ = 0;
  int8_t group_of_[kMaxRanks] = {};
  int8_t lidx_of_[kMaxRanks] = {};
  int8_t member_[kMaxRanks][kMaxRanks] = {};
  AutoTable auto_[3];  // per dtype
  RankData* rd_base_;
  RankData* rd_cur_;
  RankData* rd_end_;
  std::unordered_map<const void*, RankData*> buffers_;
  std::vector<const void*> graph_unreg_;
  std::map<std::string, char*> opened_;  // IPC handle bytes -> mapped base
  ErrorState* err_dev_ = nullptr;
  uint32_t* err_host_ = nullptr;
  std::atomic<int64_t> launches_{0};
};

// Launches one allreduce over ws emulated ranks that all live on the current
// GPU (one cooperative launch, grid.y = ws). ins/outs are per emulated rank.
// participants < ws launches only the first ranks: the others never signal,
// which is how tests make a bounded wait run out without faulting anything.
int emulate_allreduce(const std::vector<Communicator*>& comms, cudaStream_t s,
                      const std::vector<const void*>& ins, const std::vector<void*>& outs,
                      int64_t nbytes, int dtype, int algo, int participants = -1);

// The reduce-scatter (kAlgoReduceScatter) or all-gather (kAlgoAllGather)
// collective over ws emulated ranks on the current GPU, piece by piece like
// Communicator::reduce_scatter / all_gather. Returns the number of launches.
int emulate_collective(const std::vector<Communicator*>& comms, cudaStream_t s,
                       const std::vector<const void*>& ins, const std::vector<void*>& outs,
                       int64_t seg_bytes, int dtype, int kind, int participants = -1);

#if NAB_DEBUG_BOUNDS
// Debug builds only: the same launch with emulated rank 0's view claiming an
// out-of-range rank, so that the device bounds check must catch it before
// that rank touches any memory (tests of the check itself).
int emulate_allreduce_bad_rank(const std::vector<Communicator*>& comms, cudaStream_t s,
                               const std::vector<const void*>& ins, const std::vector<void*>& outs,
                               int64_t nbytes, int dtype, int algo);
#endif

// Legacy CUDA IPC helpers (reference src/numa_all_reduce.cu:693-734).
void* ipc_alloc_shared(size_t bytes, cudaStream_t s, std::string* handle_out);
void* ipc_open(const std::string& handle);
void ipc_close(void* ptr);
void ipc_free(void* ptr);

std::string cuda_error_string(cudaError_t e);

}  // namespace nab
