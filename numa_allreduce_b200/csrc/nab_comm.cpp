// Host runtime of the allreduce library. See nab_comm.h.
#include "nab_comm.h"

#include <algorithm>
#include <cstring>
#include <stdexcept>
#include <string>

#include "nab_driver.h"
#include "nab_kernels.h"

namespace nab {

namespace {

constexpr int64_t kAlign = 4096;

int64_t round_up(int64_t x, int64_t a) { return (x + a - 1) / a * a; }

int64_t ceil_div_host(int64_t a, int64_t b) { return (a + b - 1) / b; }

template <typename T>
T clampv(T v, T lo, T hi) {
  return std::max(lo, std::min(v, hi));
}

}  // namespace

std::string cuda_error_string(cudaError_t e) { return cudaGetErrorString(e); }

// Entry points are requested as of CUDA 12.5: the multicast (NVLS) calls
// appeared in 12.1, so an older version would report them as missing.
void* driver_entry(const char* name) {
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q;
  cudaError_t e = cudaGetDriverEntryPointByVersion(name, &fn, 12050, cudaEnableDefault, &q);
  if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || fn == nullptr)
    throw std::runtime_error(std::string("CUDA driver entry point unavailable: ") + name);
  return fn;
}

std::string cu_error_string(CUresult r) {
  using Fn = CUresult (*)(CUresult, const char**);
  const char* s = nullptr;
  try {
    driver_fn<Fn>("cuGetErrorString")(r, &s);
  } catch (...) {
  }
  return s ? std::string(s) : ("CUresult " + std::to_string(static_cast<int>(r)));
}

CommConfig config_from_list(const std::vector<int64_t>& v) {
  CommConfig c;
  auto at = [&](size_t i, int64_t d) { return i < v.size() && v[i] >= 0 ? v[i] : d; };
  c.oneshot_max = at(0, c.oneshot_max);
  c.chunk_max = at(1, c.chunk_max);
  c.max_ctas = static_cast<int>(at(2, c.max_ctas));
  c.oneshot_ctas = static_cast<int>(at(3, c.oneshot_ctas));
  c.fused_bytes = at(4, c.fused_bytes);
  c.timeout_ns = static_cast<uint64_t>(at(5, static_cast<int64_t>(c.timeout_ns)));
  c.pipe_ctas = static_cast<int>(at(6, c.pipe_ctas));
  c.pipe_tile = at(7, c.pipe_tile);
  c.hybrid_p2p_permille = static_cast<int>(at(8, c.hybrid_p2p_permille));
  c.hybrid_p2p_ctas = static_cast<int>(at(9, c.hybrid_p2p_ctas));
  c.hybrid_nvls_ctas = static_cast<int>(at(10, c.hybrid_nvls_ctas));
  c.oneshot_grain = static_cast<int>(at(11, c.oneshot_grain));
  return c;
}

AutoTable builtin_auto_table(int ws, bool has_nvls) {
  (void)has_nvls;
  AutoTable t;
  if (ws <= 1) {
    t.steps = {{int64_t(1) << 62, kAlgoCopy}};
    return t;
  }
  // push one-shot for latency-bound sizes, the pipelined store two-shot above
  // (measured fastest of this library's protocols at 2, 4 and 8 B200s; the
  // NVLS and hybrid protocols trailed it at every size)
  t.steps.push_back({512 << 10, kAlgoOneshot});
  t.steps.push_back({int64_t(1) << 62, kAlgoTwoshotPipe});
  t.fallback = kAlgoNccl;
  return t;
}

int choose_auto(const AutoTable& t, int ws, int64_t nbytes, bool has_nvls, bool has_groups) {
  if (ws <= 1) return kAlgoCopy;
  int algo = t.fallback;
  for (const AutoStep& st : t.steps) {
    if (nbytes <= st.max_bytes) {
      algo = st.algo;
      break;
    }
  }
  if (!has_nvls) {
    if (algo == kAlgoNvlsTwoshot) algo = kAlgoTwoshot;
    if (algo == kAlgoNvlsOneshot) algo = kAlgoOneshot;
    if (algo == kAlgoHybrid) algo = kAlgoTwoshotPipe;
  }
  if (algo == kAlgoHier && !has_groups) algo = kAlgoTwoshot;
  return algo;
}

Layout make_layout(int ws, const CommConfig& cfg) {
  if (ws < 1 || ws > kMaxRanks) throw std::invalid_argument("world size must be in [1, 8]");
  if (cfg.max_ctas < 1 || cfg.max_ctas > kMaxBlocks || cfg.oneshot_ctas < 1 ||
      cfg.oneshot_ctas > kMaxBlocks)
    throw std::invalid_argument("CTA counts must be in [1, 160]");
  if (cfg.oneshot_grain < 32 || cfg.oneshot_grain > (1 << 20))
    throw std::invalid_argument("oneshot_grain must be in [32, 2^20] packs");
  if (cfg.chunk_max != 0 && (cfg.chunk_max < 16 * 512 || cfg.chunk_max % 16 != 0))
    throw std::invalid_argument("chunk_max must be 0 (auto) or a multiple of 16 and >= 8 KiB");
  if (cfg.oneshot_max % 16 != 0) throw std::invalid_argument("oneshot_max must be a multiple of 16");
  if (cfg.pipe_ctas < 1 || cfg.pipe_ctas > kMaxBlocks) throw std::invalid_argument("pipe_ctas must be in [1, 160]");
  if (cfg.pipe_tile < (64 << 10) || cfg.pipe_tile > (4 << 20))
    throw std::invalid_argument("pipe_tile must be in [64 KiB, 4 MiB]");
  if (cfg.hybrid_p2p_permille < 0 || cfg.hybrid_p2p_permille > 1000 || cfg.hybrid_p2p_ctas < 1 ||
      cfg.hybrid_p2p_ctas > kMaxBlocks || cfg.hybrid_nvls_ctas < 1 || cfg.hybrid_nvls_ctas > kNvlsCtas)
    throw std::invalid_argument("hybrid split: permille in [0, 1000], P2P CTAs in [1, 160], NVLS CTAs in [1, 128]");
  Layout L{};
  int64_t off = round_up(static_cast<int64_t>(sizeof(SignalPad)), kAlign);
  L.oneshot_off = off;
  L.oneshot_max = cfg.oneshot_max;
  off += round_up(2 * ws * cfg.oneshot_max, kAlign);
  const int64_t chunk = cfg.chunk_max != 0
                            ? cfg.chunk_max
                            : std::max<int64_t>(32 << 10, std::min<int64_t>(256 << 10, (512 << 10) / ws / 4096 * 4096));
  L.chunk_max = chunk;
  L.max_ctas = cfg.max_ctas;
  L.twoshot_off = off;
  off += round_up(static_cast<int64_t>(cfg.max_ctas) * (ws + 1) * chunk, kAlign);
  // The hierarchical protocol exists to cut cross-group traffic, not for peak
  // bandwidth on NVSwitch, so it gets a smaller region: at most 64 CTAs and
  // 32 KiB chunks. Per CTA: gsize rs slots + 2 parities x ngroups fp32 partial
  // slots (two chunk widths each) + 1 result; gsize + 4 * ngroups + 1 <= 4 * ws + 2.
  L.hier_ctas = std::min(cfg.max_ctas, 64);
  L.hier_chunk = std::min<int64_t>(chunk, 32 << 10);
  L.hier_off = off;
  off += round_up(static_cast<int64_t>(L.hier_ctas) * (4 * ws + 2) * L.hier_chunk, kAlign);
  L.pipe_off = off;
  L.pipe_chunk = std::max<int64_t>(16 << 10, cfg.pipe_tile / ws / 4096 * 4096);
  L.pipe_ctas = cfg.pipe_ctas;
  off += round_up(static_cast<int64_t>(cfg.pipe_ctas) * kPipeSlots * 2 * ws * L.pipe_chunk, kAlign);
  L.fused_off = off;
  L.fused_bytes = round_up(cfg.fused_bytes, kAlign);
  off += 2 * ws * L.fused_bytes;
  L.fused2_off = off;
  off += static_cast<int64_t>(cfg.max_ctas) * (ws + 1) * kFusedMaxHidden * 2;
  L.ws_bytes = off;
  int64_t moff = round_up(static_cast<int64_t>(sizeof(NvlsPad)), kAlign);
  L.mc_oneshot_off = moff;
  moff += round_up(2 * cfg.oneshot_max, kAlign);
  L.mc_twoshot_off = moff;
  L.nvls_chunk = std::max<int64_t>(16 << 10, kNvlsTileBytes / ws / 4096 * 4096);
  moff += round_up(static_cast<int64_t>(kNvlsCtas) * kNvlsSlots * ws * L.nvls_chunk, kAlign);
  L.mc_bytes = moff;
  return L;
}

Communicator::Communicator(int rank, int ws, const std::vector<char*>& wsp, void* rank_data,
                           size_t rank_data_bytes, const CommConfig& cfg, bool full_nvlink)
    : rank_(rank), ws_(ws), cfg_(cfg), L_(make_layout(ws, cfg)), full_nvlink_(full_nvlink),
      wsp_(wsp) {
  if (rank < 0 || rank >= ws) throw std::invalid_argument("rank out of range");
  if (static_cast<int>(wsp.size()) != ws)
    throw std::invalid_argument("need one workspace pointer per rank");
  for (auto* p : wsp)
    if (p == nullptr || reinterpret_cast<uintptr_t>(p) % 256 != 0)
      throw std::invalid_argument("workspace pointers must be non-null and 256-byte aligned");
  NAB_CUDA_CHECK(cudaGetDevice(&device_));
  rd_base_ = rd_cur_ = reinterpret_cast<RankData*>(rank_data);
  rd_end_ = rd_base_ + (rank_data ? rank_data_bytes / sizeof(RankData) : 0);
  NAB_CUDA_CHECK(cudaMalloc(&err_dev_, sizeof(ErrorState)));
  NAB_CUDA_CHECK(cudaMemset(err_dev_, 0, sizeof(ErrorState)));
  NAB_CUDA_CHECK(cudaHostAlloc(&err_host_, 64, cudaHostAllocMapped | cudaHostAllocPortable));
  std::memset(err_host_, 0, 64);
  for (auto& t : auto_) t = builtin_auto_table(ws_, false);
}

void Communicator::set_auto_table(int dtype, const AutoTable& t) {
  if (dtype < kF32 || dtype > kBF16) throw std::invalid_argument("dtype must be 0, 1 or 2");
  int64_t prev = -1;
  for (const AutoStep& st : t.steps) {
    if (st.max_bytes <= prev) throw std::invalid_argument("table steps must be strictly ascending");
    if (st.algo <= kAlgoAuto || (st.algo >= kAlgoCount && st.algo != kAlgoNccl))
      throw std::invalid_argument("unknown protocol in table: " + std::to_string(st.algo));
    prev = st.max_bytes;
  }
  auto_[dtype] = t;
}

const AutoTable& Communicator::auto_table(int dtype) const {
  if (dtype < kF32 || dtype > kBF16) throw std::invalid_argument("dtype must be 0, 1 or 2");
  return auto_[dtype];
}

void Communicator::set_hybrid(int p2p_permille, int p2p_ctas, int nvls_ctas) {
  if (p2p_ctas > cfg_.pipe_ctas)
    throw std::invalid_argument("hybrid split: more P2P CTAs than the pipelined ring has slots (pipe_ctas)");
  CommConfig c = cfg_;
  c.hybrid_p2p_permille = p2p_permille;
  c.hybrid_p2p_ctas = p2p_ctas;
  c.hybrid_nvls_ctas = nvls_ctas;
  make_layout(ws_, c);  // validates; the layout itself does not depend on the split
  cfg_ = c;
}

Communicator::~Communicator() {
  for (auto& kv : opened_) cudaIpcCloseMemHandle(kv.second);
  if (err_dev_) cudaFree(err_dev_);
  if (err_host_) cudaFreeHost(err_host_);
}

void Communicator::set_groups(const std::vector<std::vector<int>>& groups) {
  const int ng = static_cast<int>(groups.size());
  if (ng < 1 || ng > ws_) throw std::invalid_argument("bad number of groups");
  const int gs = static_cast<int>(groups[0].size());
  if (gs * ng != ws_) throw std::invalid_argument("groups must partition the ranks equally");
  std::vector<int> seen(ws_, 0);
  for (int g = 0; g < ng; ++g) {
    if (static_cast<int>(groups[g].size()) != gs)
      throw std::invalid_argument("all groups must have the same size");
    for (int l = 0; l < gs; ++l) {
      const int r = groups[g][l];
      if (r < 0 || r >= ws_ || seen[r]++) throw std::invalid_argument("groups must partition ranks");
      group_of_[r] = static_cast<int8_t>(g);
      lidx_of_[r] = static_cast<int8_t>(l);
      member_[g][l] = static_cast<int8_t>(r);
    }
  }
  ngroups_ = ng;
  gsize_ = gs;
}

void Communicator::attach_nvls(char* mc, char* uc, int64_t bytes) {
  if (bytes < L_.mc_bytes) throw std::invalid_argument("NVLS workspace too small");
  mc_ = mc;
  uc_ = uc;
  mc_bytes_ = bytes;
  // the built-in steps depend on multicast support; a table set later wins
  for (auto& t : auto_) t = builtin_auto_table(ws_, true);
}

RankData* Communicator::reserve_rank_data() {
  if (rd_cur_ >= rd_end_) throw std::runtime_error("RankData registry is full");
  return rd_cur_++;
}

void Communicator::register_buffer(const std::vector<void*>& ptrs) {
  if (static_cast<int>(ptrs.size()) != ws_) throw std::invalid_argument("need one pointer per rank");
  RankData rd{};
  for (int i = 0; i < ws_; ++i) rd.ptrs[i] = ptrs[i];
  RankData* slot = reserve_rank_data();
  NAB_CUDA_CHECK(cudaMemcpy(slot, &rd, sizeof(rd), cudaMemcpyHostToDevice));
  buffers_[ptrs[rank_]] = slot;
}

std::pair<std::string, std::vector<int64_t>> Communicator::graph_buffer_ipc_meta() {
  using GetAttr = CUresult (*)(void*, CUpointer_attribute, CUdeviceptr);
  auto get_attr = driver_fn<GetAttr>("cuPointerGetAttribute");
  std::string handles;
  handles.reserve(graph_unreg_.size() * sizeof(cudaIpcMemHandle_t));
  std::vector<int64_t> offsets;
  offsets.reserve(graph_unreg_.size());
  for (const void* ptr : graph_unreg_) {
    CUdeviceptr base = 0;
    NAB_CU_CHECK(get_attr(&base, CU_POINTER_ATTRIBUTE_RANGE_START_ADDR,
                          reinterpret_cast<CUdeviceptr>(ptr)));
    cudaIpcMemHandle_t h;
    NAB_CUDA_CHECK(cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base)));
    handles.append(reinterpret_cast<const char*>(&h), sizeof(h));
    offsets.push_back(reinterpret_cast<const char*>(ptr) - reinterpret_cast<const char*>(base));
  }
  return {handles, offsets};
}

void Communicator::register_graph_buffers(const std::vector<std::string>& handles,
                                          const std::vector<std::vector<int64_t>>& offsets) {
  const size_t n = graph_unreg_.size();
  if (static_cast<int>(handles.size()) != ws_ || static_cast<int>(offsets.size()) != ws_)
    throw std::invalid_argument("need handles and offsets from every rank");
  std::vector<RankData> rds(n);
  for (int j = 0; j < ws_; ++j) {
    if (handles[j].size() != n * sizeof(cudaIpcMemHandle_t) || offsets[j].size() != n)
      throw std::invalid_argument("ranks captured different numbers of buffers");
    for (size_t i = 0; i < n; ++i) {
      if (j == rank_) {
        rds[i].ptrs[j] = graph_unreg_[i];
        continue;
      }
      const std::string h = handles[j].substr(i * sizeof(cudaIpcMemHandle_t), sizeof(cudaIpcMemHandle_t));
      auto it = opened_.find(h);
      char* base;
      if (it == opened_.end()) {
        base = static_cast<char*>(ipc_open(h));
        opened_[h] = base;
      } else {
        base = it->second;
      }
      rds[i].ptrs[j] = base + offsets[j][i];
    }
  }
  for (size_t i = 0; i < n; ++i)
    NAB_CUDA_CHECK(cudaMemcpy(buffers_.at(graph_unreg_[i]), &rds[i], sizeof(RankData),
                              cudaMemcpyHostToDevice));
  graph_unreg_.clear();
}

LaunchPlan Communicator::plan(int64_t nbytes, int algo, bool registered, int dtype) const {
  (void)registered;
  LaunchPlan pl;
  const int64_t npacks = nbytes / 16;
  if (ws_ == 1) {
    pl.algo = kAlgoCopy;
    pl.grid = dim3(static_cast<unsigned>(clampv<int64_t>(ceil_div_host(npacks, 4 * 512), 1, 148 * 4)));
    return pl;
  }
  if (algo == kAlgoAuto) {
    const AutoTable& t = auto_table(dtype);
    algo = choose_auto(t, ws_, nbytes, mc_ != nullptr, ngroups_ > 0);
    if (algo == kAlgoNccl) {
      // no NCCL here: the last custom protocol of the table takes the message
      algo = kAlgoTwoshotPipe;
      for (auto it = t.steps.rbegin(); it != t.steps.rend(); ++it)
        if (it->algo != kAlgoNccl) {
          algo = choose_auto(AutoTable{{{int64_t(1) << 62, it->algo}}, kAlgoNccl}, ws_, nbytes, mc_ != nullptr,
                             ngroups_ > 0);
          break;
        }
    }
    if ((algo == kAlgoOneshot || algo == kAlgoNvlsOneshot) && nbytes > cfg_.oneshot_max) algo = kAlgoTwoshotPipe;
  }
  if (algo == kAlgoHybrid && mc_ == nullptr)
    throw std::invalid_argument("hybrid protocol requested but no multicast workspace attached");
  // too small to split: the whole message takes the P2P part
  if (algo == kAlgoHybrid && npacks < 2 * 32 * ws_) algo = kAlgoTwoshotPipe;
  if ((algo == kAlgoNvlsOneshot || algo == kAlgoNvlsTwoshot) && mc_ == nullptr)
    throw std::invalid_argument("NVLS protocol requested but no multicast workspace attached");
  if (algo == kAlgoHier && ngroups_ == 0)
    throw std::invalid_argument("hierarchical protocol requested but no groups set");
  pl.algo = algo;
  switch (algo) {
    case kAlgoOneshot:
    case kAlgoNvlsOneshot:
    case kAlgoOneshotPull: {
      if (algo != kAlgoOneshotPull && nbytes > cfg_.oneshot_max)
        throw std::invalid_argument("message exceeds the one-shot workspace");
      const int64_t b = clampv<int64_t>(ceil_div_host(npacks, cfg_.oneshot_grain), 1, cfg_.oneshot_ctas);
      pl.grid = dim3(static_cast<unsigned>(b));
      break;
    }
    case kAlgoTwoshotPipe:
    case kAlgoNvlsTwoshot: {
      // pipelined: tiles of ws chunks flow through each CTA's ring; small
      // tiles for small messages so that they still spread over all CTAs
      const bool nv = algo == kAlgoNvlsTwoshot;
      const int64_t chunk_cap = (nv ? L_.nvls_chunk : L_.pipe_chunk) / 16;
      const int kctas = nv ? kNvlsCtas : L_.pipe_ctas;
      const int64_t chp = std::min(chunk_cap, std::max<int64_t>(32, ceil_div_host(npacks, ws_ * kctas)));
      const int64_t ntiles = ceil_div_host(npacks, ws_ * chp);
      const int64_t C = clampv<int64_t>(ntiles, 1, kctas);
      const int64_t per_cta = ceil_div_host(ntiles, C);
      if (per_cta >= (int64_t(1) << 30)) throw std::invalid_argument("message too large");
      pl.grid = dim3(static_cast<unsigned>(C));
      pl.chunk_packs = static_cast<int>(chp);
      pl.rounds = static_cast<int>(per_cta);
      break;
    }
    case kAlgoHybrid: {
      // P2P share of the message and CTA budget of each part from the config;
      // the split point is a multiple of 16 packs (256 B) and both parts are
      // non-empty
      const int64_t permille = clampv<int64_t>(cfg_.hybrid_p2p_permille, 1, 999);
      const int cp_max = std::min(cfg_.hybrid_p2p_ctas, L_.pipe_ctas);
      const int cn_max = cfg_.hybrid_nvls_ctas;
      const int64_t split = clampv<int64_t>((npacks * permille / 1000) / 16 * 16, 16, (npacks - 1) / 16 * 16);
      const int64_t rest = npacks - split;
      auto part = [&](int64_t n, int64_t cap_bytes, int cmax, int& ctas) {
        const int64_t chp = std::min(cap_bytes / 16, std::max<int64_t>(32, ceil_div_host(n, ws_ * cmax)));
        ctas = static_cast<int>(clampv<int64_t>(ceil_div_host(n, ws_ * chp), 1, cmax));
        return static_cast<int>(chp);
      };
      int cp = 0, cn = 0;
      pl.chunk_packs = part(split, L_.pipe_chunk, cp_max, cp);
      pl.chunk_packs2 = part(rest, L_.nvls_chunk, cn_max, cn);
      pl.hyb_ctas = cp;
      pl.split_packs = split;
      pl.grid = dim3(static_cast<unsigned>(cp + cn));
      pl.rounds = 1;
      break;
    }
    case kAlgoTwoshot:
    case kAlgoHier: {
      const bool hier = algo == kAlgoHier;
      const int parts = hier ? gsize_ : ws_;
      const int64_t chunk_cap = (hier ? L_.hier_chunk : L_.chunk_max) / 16;
      const int64_t C = clampv<int64_t>(ceil_div_host(npacks, static_cast<int64_t>(parts) * 512), 1,
                                        hier ? L_.hier_ctas : cfg_.max_ctas);
      const int64_t chp = std::min(chunk_cap, std::max<int64_t>(1, ceil_div_host(npacks, C * parts)));
      const int64_t rounds = ceil_div_host(npacks, C * parts * chp);
      if (rounds >= (int64_t(1) << kSeqShift)) throw std::invalid_argument("message too large");
      pl.grid = dim3(static_cast<unsigned>(C));
      pl.chunk_packs = static_cast<int>(chp);
      pl.rounds = static_cast<int>(rounds);
      break;
    }
    default:
      throw std::invalid_argument("unknown allreduce algorithm " + std::to_string(algo));
  }
  return pl;
}

RankView Communicator::view(const void* in, void* out, const RankData* reg) const {
  RankView v{};
  v.in = static_cast<const char*>(in);
  v.out = static_cast<char*>(out);
  for (int i = 0; i < ws_; ++i) v.wsp[i] = wsp_[i];
  v.reg = reg;
  v.reg_end = rd_end_;
  v.mc = mc_;
  v.uc = uc_;
  v.rank = rank_;
  return v;
}

void Communicator::fill_params(ARParams& p, const LaunchPlan& pl, int64_t nbytes) const {
  p.err = err_dev_;
  p.err_host = err_host_;
  p.npacks = nbytes / 16;
  p.timeout_ns = cfg_.timeout_ns;
  p.ws = ws_;
  p.chunk_packs = pl.chunk_packs;
  p.rounds = pl.rounds;
  p.hyb_ctas = pl.hyb_ctas;
  p.chunk_packs2 = pl.chunk_packs2;
  p.split_packs = pl.split_packs;
  p.ngroups = ngroups_;
  p.gsize = gsize_;
  std::memcpy(p.group_of, group_of_, sizeof(group_of_));
  std::memcpy(p.lidx_of, lidx_of_, sizeof(lidx_of_));
  std::memcpy(p.member, member_, sizeof(member_));
  p.L = L_;
}

int Communicator::allreduce(cudaStream_t s, const void* in, void* out, int64_t nbytes, int dtype,
                            int algo, bool registered) {
  if (nbytes <= 0 || nbytes % 16 != 0)
    throw std::invalid_argument("allreduce size must be a positive multiple of 16 bytes");
  if (dtype != kF32 && dtype != kF16 && dtype != kBF16)
    throw std::invalid_argument("allreduce supports float32, float16 and bfloat16");
  if (reinterpret_cast<uintptr_t>(in) % 16 || reinterpret_cast<uintptr_t>(out) % 16)
    throw std::invalid_argument("allreduce buffers must be 16-byte aligned");
  if (ws_ == 1 && in == out) return kAlgoCopy;  // nothing to do
  const LaunchPlan pl = plan(nbytes, algo, registered, dtype);
  const RankData* reg = nullptr;
  if (pl.algo == kAlgoOneshotPull) {
    auto it = buffers_.find(in);
    if (it != buffers_.end()) {
      reg = it->second;
    } else {
      cudaStreamCaptureStatus st;
      NAB_CUDA_CHECK(cudaStreamIsCapturing(s, &st));
      if (st != cudaStreamCaptureStatusActive)
        throw std::invalid_argument("pull protocol needs a registered input buffer");
      RankData* slot = reserve_rank_data();
      buffers_[in] = slot;
      graph_unreg_.push_back(in);
      reg = slot;
    }
  }
  ARParams p{};
  fill_params(p, pl, nbytes);
  p.v[0] = view(in, out, reg);
  const cudaError_t e = launch_allreduce(pl.algo, dtype, p, pl.grid, s, false);
  if (e != cudaSuccess)
    throw std::runtime_error(std::string("allreduce launch failed: ") + cudaGetErrorString(e));
  count_launch();
  return pl.algo;
}

dim3 Communicator::collective_grid(int64_t piece_bytes) const {
  const int64_t b = clampv<int64_t>(ceil_div_host(piece_bytes / 16, cfg_.oneshot_grain), 1, cfg_.max_ctas);
  return dim3(static_cast<unsigned>(b));
}

namespace {

void check_collective_args(const void* in, const void* out, int64_t seg_bytes, int dtype) {
  if (seg_bytes <= 0 || seg_bytes % 16 != 0)
    throw std::invalid_argument("segment size must be a positive multiple of 16 bytes");
  if (dtype != kF32 && dtype != kF16 && dtype != kBF16)
    throw std::invalid_argument("collectives support float32, float16 and bfloat16");
  if (reinterpret_cast<uintptr_t>(in) % 16 || reinterpret_cast<uintptr_t>(out) % 16)
    throw std::invalid_argument("collective buffers must be 16-byte aligned");
  if (in == out) throw std::invalid_argument("collectives need distinct input and output buffers");
}

// Byte offsets of piece k in the segmented buffer (reduce-scatter input /
// all-gather output) and in the one-segment buffer.
struct Piece {
  int64_t off;    // into every segment
  int64_t bytes;  // this piece
};

std::vector<Piece> pieces_of(int64_t seg_bytes, int64_t cap) {
  std::vector<Piece> v;
  for (int64_t off = 0; off < seg_bytes; off += cap) v.push_back({off, std::min(cap, seg_bytes - off)});
  return v;
}

}  // namespace

int Communicator::reduce_scatter(cudaStream_t s, const void* in, void* out, int64_t seg_bytes, int dtype) {
  check_collective_args(in, out, seg_bytes, dtype);
  const char* src = static_cast<const char*>(in);
  char* dst = static_cast<char*>(out);
  int n = 0;
  for (const Piece& pc : pieces_of(seg_bytes, cfg_.oneshot_max)) {
    ARParams p{};
    LaunchPlan pl;
    pl.algo = ws_ == 1 ? kAlgoCopy : kAlgoReduceScatter;
    pl.grid = ws_ == 1 ? dim3(static_cast<unsigned>(clampv<int64_t>(ceil_div_host(pc.bytes / 16, 4 * 512), 1, 148)))
                       : collective_grid(pc.bytes);
    fill_params(p, pl, pc.bytes);
    p.seg_stride = seg_bytes / 16;
    p.v[0] = view(src + pc.off, dst + pc.off, nullptr);
    const cudaError_t e = launch_allreduce(pl.algo, dtype, p, pl.grid, s, false);
    if (e != cudaSuccess)
      throw std::runtime_error(std::string("reduce-scatter launch failed: ") + cudaGetErrorString(e));
    count_launch();
    ++n;
  }
  return n;
}

int Communicator::all_gather(cudaStream_t s, const void* in, void* out, int64_t seg_bytes, int dtype) {
  check_collective_args(in, out, seg_bytes, dtype);
  const char* src = static_cast<const char*>(in);
  char* dst = static_cast<char*>(out);
  int n = 0;
  for (const Piece& pc : pieces_of(seg_bytes, cfg_.oneshot_max)) {
    ARParams p{};
    LaunchPlan pl;
    pl.algo = ws_ == 1 ? kAlgoCopy : kAlgoAllGather;
    pl.grid = ws_ == 1 ? dim3(static_cast<unsigned>(clampv<int64_t>(ceil_div_host(pc.bytes / 16, 4 * 512), 1, 148)))
                       : collective_grid(pc.bytes);
    fill_params(p, pl, pc.bytes);
    p.seg_stride = seg_bytes / 16;
    p.v[0] = view(src + pc.off, dst + pc.off, nullptr);
    const cudaError_t e = launch_allreduce(pl.algo, dtype, p, pl.grid, s, false);
    if (e != cudaSuccess)
      throw std::runtime_error(std::string("all-gather launch failed: ") + cudaGetErrorString(e));
    count_launch();
    ++n;
  }
  return n;
}

uint32_t Communicator::error_code() const {
  return *reinterpret_cast<volatile uint32_t*>(err_host_);
}

ErrorState Communicator::error_state() const {
  ErrorState st{};
  NAB_CUDA_CHECK(cudaMemcpy(&st, err_dev_, sizeof(st), cudaMemcpyDeviceToHost));
  return st;
}

void Communicator::reset() {
  NAB_CUDA_CHECK(cudaDeviceSynchronize());
  NAB_CUDA_CHECK(cudaMemset(wsp_[rank_], 0, sizeof(SignalPad)));
  if (uc_) NAB_CUDA_CHECK(cudaMemset(uc_, 0, sizeof(NvlsPad)));
  NAB_CUDA_CHECK(cudaMemset(err_dev_, 0, sizeof(ErrorState)));
  NAB_CUDA_CHECK(cudaDeviceSynchronize());
  std::memset(err_host_, 0, 64);
}

namespace {

int emulate_impl(const std::vector<Communicator*>& comms, cudaStream_t s, const std::vector<const void*>& ins,
                 const std::vector<void*>& outs, int64_t nbytes, int dtype, int algo, int participants,
                 bool bad_rank) {
  const int ws = static_cast<int>(comms.size());
  if (participants < 0) participants = ws;
  if (participants < 1 || participants > ws) throw std::invalid_argument("bad participant count");
  if (ws < 2 || ws > kMaxRanks || static_cast<int>(ins.size()) != ws ||
      static_cast<int>(outs.size()) != ws)
    throw std::invalid_argument("emulation needs 2..8 communicators and one buffer per rank");
  if (nbytes <= 0 || nbytes % 16 != 0)
    throw std::invalid_argument("allreduce size must be a positive multiple of 16 bytes");
  if (algo == kAlgoNvlsOneshot || algo == kAlgoNvlsTwoshot || algo == kAlgoOneshotPull || algo == kAlgoHybrid)
    throw std::invalid_argument("NVLS, hybrid and pull protocols cannot be emulated on one GPU");
  Communicator* c0 = comms[0];
  LaunchPlan pl = c0->plan(nbytes, algo, false);
  // Every CTA of every emulated rank must be resident at once: cap the grid
  // at one 512-thread CTA per SM and re-plan the tiling for that grid.
  int dev = 0, sms = 0;
  NAB_CUDA_CHECK(cudaGetDevice(&dev));
  NAB_CUDA_CHECK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  const int64_t cap = std::max(1, sms / ws);
  if (pl.grid.x > cap) {
    const int64_t npacks = nbytes / 16;
    pl.grid.x = static_cast<unsigned>(cap);
    // round-based protocols re-plan their tiling for the smaller grid; the
    // pipelined one just gives each CTA more tiles
    if (pl.rounds > 0 && (pl.algo == kAlgoTwoshot || pl.algo == kAlgoHier)) {
      ARParams tmp{};
      c0->fill_params(tmp, pl, nbytes);
      const int parts = (pl.algo == kAlgoHier) ? tmp.gsize : ws;
      const int64_t chunk_cap =
          (pl.algo == kAlgoHier ? c0->layout().hier_chunk : c0->layout().chunk_max) / 16;
      const int64_t chp = std::min(chunk_cap, std::max<int64_t>(1, ceil_div_host(npacks, cap * parts)));
      pl.chunk_packs = static_cast<int>(chp);
      pl.rounds = static_cast<int>(ceil_div_host(npacks, cap * parts * chp));
    }
  }
  ARParams p{};
  c0->fill_params(p, pl, nbytes);
  for (int r = 0; r < ws; ++r) {
    if (comms[r]->rank() != r) throw std::invalid_argument("communicators must be in rank order");
    p.v[r] = comms[r]->view(ins[r], outs[r], nullptr);
  }
  if (bad_rank) p.v[0].rank = ws;  // caught by the device bounds check of debug builds
  pl.grid.y = participants;
  const cudaError_t e = launch_allreduce(pl.algo, dtype, p, pl.grid, s, true);
  if (e != cudaSuccess)
    throw std::runtime_error(std::string("emulated allreduce launch failed: ") + cudaGetErrorString(e));
  for (int r = 0; r < participants; ++r) comms[r]->count_launch();
  return pl.algo;
}

}  // namespace

int emulate_allreduce(const std::vector<Communicator*>& comms, cudaStream_t s,
                      const std::vector<const void*>& ins, const std::vector<void*>& outs,
                      int64_t nbytes, int dtype, int algo, int participants) {
  return emulate_impl(comms, s, ins, outs, nbytes, dtype, algo, participants, false);
}

int emulate_collective(const std::vector<Communicator*>& comms, cudaStream_t s,
                       const std::vector<const void*>& ins, const std::vector<void*>& outs,
                       int64_t seg_bytes, int dtype, int kind, int participants) {
  const int ws = static_cast<int>(comms.size());
  if (participants < 0) participants = ws;
  if (participants < 1 || participants > ws) throw std::invalid_argument("bad participant count");
  if (ws < 2 || ws > kMaxRanks || static_cast<int>(ins.size()) != ws || static_cast<int>(outs.size()) != ws)
    throw std::invalid_argument("emulation needs 2..8 communicators and one buffer per rank");
  if (kind != kAlgoReduceScatter && kind != kAlgoAllGather)
    throw std::invalid_argument("emulated collective must be reduce-scatter or all-gather");
  for (int r = 0; r < ws; ++r) {
    check_collective_args(ins[r], outs[r], seg_bytes, dtype);
    if (comms[r]->rank() != r) throw std::invalid_argument("communicators must be in rank order");
  }
  Communicator* c0 = comms[0];
  // every CTA of every emulated rank resident at once (cooperative launch)
  int dev = 0, sms = 0;
  NAB_CUDA_CHECK(cudaGetDevice(&dev));
  NAB_CUDA_CHECK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  const unsigned cap = static_cast<unsigned>(std::max(1, sms / ws));
  int n = 0;
  for (const Piece& pc : pieces_of(seg_bytes, c0->config().oneshot_max)) {
    LaunchPlan pl;
    pl.algo = kind;
    pl.grid = c0->collective_grid(pc.bytes);
    pl.grid.x = std::min(pl.grid.x, cap);
    ARParams p{};
    c0->fill_params(p, pl, pc.bytes);
    p.seg_stride = seg_bytes / 16;
    for (int r = 0; r < ws; ++r)
      p.v[r] = comms[r]->view(static_cast<const char*>(ins[r]) + pc.off, static_cast<char*>(outs[r]) + pc.off,
                              nullptr);
    pl.grid.y = participants;
    const cudaError_t e = launch_allreduce(kind, dtype, p, pl.grid, s, true);
    if (e != cudaSuccess)
      throw std::runtime_error(std::string("emulated collective launch failed: ") + cudaGetErrorString(e));
    for (int r = 0; r < participants; ++r) comms[r]->count_launch();
    ++n;
  }
  return n;
}

#if NAB_DEBUG_BOUNDS
int emulate_allreduce_bad_rank(const std::vector<Communicator*>& comms, cudaStream_t s,
                               const std::vector<const void*>& ins, const std::vector<void*>& outs,
                               int64_t nbytes, int dtype, int algo) {
  return emulate_impl(comms, s, ins, outs, nbytes, dtype, algo, -1, true);
}
#endif

void* ipc_alloc_shared(size_t bytes, cudaStream_t s, std::string* handle_out) {
  void* buf = nullptr;
  cudaStreamCaptureMode mode = cudaStreamCaptureModeRelaxed;
  NAB_CUDA_CHECK(cudaThreadExchangeStreamCaptureMode(&mode));
  cudaError_t e = cudaMalloc(&buf, bytes);
  if (e == cudaSuccess) e = cudaMemsetAsync(buf, 0, bytes, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  cudaThreadExchangeStreamCaptureMode(&mode);
  if (e != cudaSuccess) {
    if (buf) cudaFree(buf);
    throw std::runtime_error(std::string("shared buffer allocation failed: ") + cudaGetErrorString(e));
  }
  if (handle_out) {
    cudaIpcMemHandle_t h;
    NAB_CUDA_CHECK(cudaIpcGetMemHandle(&h, buf));
    handle_out->assign(reinterpret_cast<const char*>(&h), sizeof(h));
  }
  return buf;
}

void* ipc_open(const std::string& handle) {
  if (handle.size() != sizeof(cudaIpcMemHandle_t)) throw std::invalid_argument("bad IPC handle size");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle.data(), sizeof(h));
  void* p = nullptr;
  NAB_CUDA_CHECK(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
  return p;
}

void ipc_close(void* ptr) { NAB_CUDA_CHECK(cudaIpcCloseMemHandle(ptr)); }

void ipc_free(void* ptr) { NAB_CUDA_CHECK(cudaFree(ptr)); }

}  // namespace nab
