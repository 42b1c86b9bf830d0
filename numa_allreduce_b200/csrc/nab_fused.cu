// Fused allreduce + residual add + RMSNorm kernels. See nab_fused.h.
//
// oneshot: every rank pushes its [T, H] partial into every peer's slot
//          (double-buffered by call parity), one flag exchange per CTA, then
//          every rank reduces all rows and applies residual + norm itself.
// twoshot: rows are dealt round-robin to owners; each owner reduces its rows,
//          applies residual + norm, and publishes the new residual row; the
//          others pull that row and recompute the norm locally.
#include <cuda_runtime.h>

#include <stdexcept>
#include <string>

#include "nab_device.cuh"
#include "nab_fused.h"
#include "nab_proto.cuh"

namespace nab {

namespace {

constexpr int kFThreads = 256;
constexpr int kRowMaxPacks = kFusedMaxHidden * 2 / 16;

struct FusedView {
  const char* in;
  char* residual;
  const char* weight;
  char* out;
  char* wsp[kMaxRanks];
  int rank;
  int pad_;
};

struct FusedParams {
  FusedView v[kMaxRanks];
  ErrorState* err;
  uint32_t* err_host;
  uint64_t timeout_ns;
  int ws;
  int T;
  int H;
  int rounds;
  float eps;
  int pad_;
  Layout L;
};

NAB_DINLINE float block_sum(float v) {
  __shared__ float s_part[kFThreads / 32];
  __shared__ float s_total;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) s_part[warp] = v;
  __syncthreads();
  if (warp == 0) {
    float t = lane < kFThreads / 32 ? s_part[lane] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    if (lane == 0) s_total = t;
  }
  __syncthreads();
  const float r = s_total;
  __syncthreads();
  return r;
}

NAB_DINLINE void unpack_bf16(uint4 x, float* f) {
  const uint32_t w[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    f[2 * k] = __uint_as_float(w[k] << 16);
    f[2 * k + 1] = __uint_as_float(w[k] & 0xffff0000u);
  }
}

// z holds the bf16-rounded residual row (as floats) for this thread's packs.
template <int PPT>
NAB_DINLINE void norm_store(const float (&z)[PPT][8], float ss, const uint4* w, uint4* out_row, int hp,
                            int H, float eps) {
  const float inv = rsqrtf(block_sum(ss) / static_cast<float>(H) + eps);
#pragma unroll
  for (int k = 0; k < PPT; ++k) {
    const int idx = threadIdx.x + k * kFThreads;
    if (idx < hp) {
      float wf[8];
      unpack_bf16(ld_plain(w + idx), wf);
      uint4 y;
      y.x = pack_bf16x2(z[k][0] * inv * wf[0], z[k][1] * inv * wf[1]);
      y.y = pack_bf16x2(z[k][2] * inv * wf[2], z[k][3] * inv * wf[3]);
      y.z = pack_bf16x2(z[k][4] * inv * wf[4], z[k][5] * inv * wf[5]);
      y.w = pack_bf16x2(z[k][6] * inv * wf[6], z[k][7] * inv * wf[7]);
      st_plain(out_row + idx, y);
    }
  }
}

// Adds the residual pack to the reduced sum, rounds to bf16, writes the new
// residual and returns the rounded values and their sum of squares.
NAB_DINLINE float finish_pack(Acc<__nv_bfloat16>& a, uint4 res, uint4* res_dst, uint4* extra_dst,
                              float* z) {
  acc_add(a, res);
  const uint4 zb = acc_pack(a);
  st_plain(res_dst, zb);
  if (extra_dst) st_plain(extra_dst, zb);
  unpack_bf16(zb, z);
  float ss = 0.f;
#pragma unroll
  for (int e = 0; e < 8; ++e) ss += z[e] * z[e];
  return ss;
}

template <int PPT>
__global__ void __launch_bounds__(kFThreads) k_rmsnorm(const uint4* __restrict__ in, uint4* residual,
                                                       const uint4* __restrict__ w, uint4* out, int T,
                                                       int H, float eps) {
  pdl_wait();
  pdl_trigger();
  const int hp = H / 8;
  for (int t = blockIdx.x; t < T; t += gridDim.x) {
    float z[PPT][8];
    float ss = 0.f;
#pragma unroll
    for (int k = 0; k < PPT; ++k) {
      const int idx = threadIdx.x + k * kFThreads;
      if (idx < hp) {
        Acc<__nv_bfloat16> a;
        acc_set(a, ld_plain(in + static_cast<int64_t>(t) * hp + idx));
        ss += finish_pack(a, ld_plain(residual + static_cast<int64_t>(t) * hp + idx),
                          residual + static_cast<int64_t>(t) * hp + idx, nullptr, z[k]);
      }
    }
    norm_store<PPT>(z, ss, w, out + static_cast<int64_t>(t) * hp, hp, H, eps);
  }
}

template <int WS, int PPT>
__global__ void __launch_bounds__(kFThreads) k_fused_oneshot(const __grid_constant__ FusedParams p) {
  pdl_trigger();
  const FusedView& me = p.v[blockIdx.y];
  const int rank = me.rank;
  const uint32_t epoch = begin_call(me.wsp, rank);
  const WaitCtx wc = make_wait(p.err, p.err_host, p.timeout_ns, me.wsp, rank, epoch);
  const int parity = epoch & 1;
  const int hp = p.H / 8;
  const int64_t slot_packs = p.L.fused_bytes / 16;
  const uint4* in = reinterpret_cast<const uint4*>(me.in);
  uint4* res = reinterpret_cast<uint4*>(me.residual);
  auto slot = [&](int owner, int src) -> uint4* {
    return reinterpret_cast<uint4*>(me.wsp[owner] + p.L.fused_off) +
           (static_cast<int64_t>(parity) * WS + src) * slot_packs;
  };
  // 1. push my partial rows to every peer
  for (int t = blockIdx.x; t < p.T; t += gridDim.x) {
    for (int idx = threadIdx.x; idx < hp; idx += kFThreads) {
      const int64_t o = static_cast<int64_t>(t) * hp + idx;
      const uint4 x = ld_plain(in + o);
#pragma unroll
      for (int k = 1; k < WS; ++k) st_plain(slot((rank + k) % WS, rank) + o, x);
    }
  }
  int peers[WS - 1];
  all_peers<WS>(rank, peers);
  const bool ok = exchange(me.wsp, rank, kFlagFused, blockIdx.x, make_seq(epoch, 0), peers, WS - 1, wc,
                           kStageFused);
  if (ok) {
    for (int t = blockIdx.x; t < p.T; t += gridDim.x) {
      float z[PPT][8];
      float ss = 0.f;
#pragma unroll
      for (int k = 0; k < PPT; ++k) {
        const int idx = threadIdx.x + k * kFThreads;
        if (idx < hp) {
          const int64_t o = static_cast<int64_t>(t) * hp + idx;
          uint4 x[WS];
#pragma unroll
          for (int q = 0; q < WS; ++q) x[q] = (q == rank) ? ld_plain(in + o) : ld_cg(slot(rank, q) + o);
          Acc<__nv_bfloat16> a;
          acc_set(a, x[0]);
#pragma unroll
          for (int q = 1; q < WS; ++q) acc_add(a, x[q]);
          ss += finish_pack(a, ld_plain(res + o), res + o, nullptr, z[k]);
        }
      }
      norm_store<PPT>(z, ss, reinterpret_cast<const uint4*>(me.weight),
                      reinterpret_cast<uint4*>(me.out) + static_cast<int64_t>(t) * hp, hp, p.H, p.eps);
    }
  }
  end_call(me.wsp, rank, epoch);
}

template <int WS, int PPT>
__global__ void __launch_bounds__(kFThreads) k_fused_twoshot(const __grid_constant__ FusedParams p) {
  pdl_trigger();
  const FusedView& me = p.v[blockIdx.y];
  const int rank = me.rank;
  const uint32_t epoch = begin_call(me.wsp, rank);
  const WaitCtx wc = make_wait(p.err, p.err_host, p.timeout_ns, me.wsp, rank, epoch);
  const int c = blockIdx.x;
  const int hp = p.H / 8;
  const uint4* in = reinterpret_cast<const uint4*>(me.in);
  uint4* res = reinterpret_cast<uint4*>(me.residual);
  uint4* out = reinterpret_cast<uint4*>(me.out);
  const uint4* w = reinterpret_cast<const uint4*>(me.weight);
  auto region = [&](int r) -> uint4* {
    return reinterpret_cast<uint4*>(me.wsp[r] + p.L.fused2_off) +
           static_cast<int64_t>(c) * (WS + 1) * kRowMaxPacks;
  };
  int peers[WS - 1];
  all_peers<WS>(rank, peers);
  bool ok = true;
  for (int r = 0; r < p.rounds && ok; ++r) {
    const int base_row = (r * gridDim.x + c) * WS;
    const uint64_t seq = make_seq(epoch, r + 1);
    // 1. push the rows other ranks own
    for (int k = 0; k < WS - 1; ++k) {
      const int t = base_row + peers[k];
      if (t >= p.T) continue;
      uint4* dst = region(peers[k]) + rank * kRowMaxPacks;
      for (int idx = threadIdx.x; idx < hp; idx += kFThreads)
        st_plain(dst + idx, ld_plain(in + static_cast<int64_t>(t) * hp + idx));
    }
    ok = exchange(me.wsp, rank, kFlagFusedRS, c, seq, peers, WS - 1, wc, kStageRS);
    if (!ok) break;
    // 2. reduce + residual + norm of my row; publish the new residual row
    const int tm = base_row + rank;
    if (tm < p.T) {
      uint4* mine = region(rank);
      float z[PPT][8];
      float ss = 0.f;
#pragma unroll
      for (int k = 0; k < PPT; ++k) {
        const int idx = threadIdx.x + k * kFThreads;
        if (idx < hp) {
          const int64_t o = static_cast<int64_t>(tm) * hp + idx;
          uint4 x[WS];
#pragma unroll
          for (int q = 0; q < WS; ++q) x[q] = (q == rank) ? ld_plain(in + o) : ld_cg(mine + q * kRowMaxPacks + idx);
          Acc<__nv_bfloat16> a;
          acc_set(a, x[0]);
#pragma unroll
          for (int q = 1; q < WS; ++q) acc_add(a, x[q]);
          ss += finish_pack(a, ld_plain(res + o), res + o, mine + WS * kRowMaxPacks + idx, z[k]);
        }
      }
      norm_store<PPT>(z, ss, w, out + static_cast<int64_t>(tm) * hp, hp, p.H, p.eps);
    }
    ok = exchange(me.wsp, rank, kFlagFusedAG, c, seq, peers, WS - 1, wc, kStageAG);
    if (!ok) break;
    // 3. pull the other owners' residual rows and apply the norm locally
    for (int k = 0; k < WS - 1; ++k) {
      const int t = base_row + peers[k];
      if (t >= p.T) continue;
      const uint4* src = region(peers[k]) + WS * kRowMaxPacks;
      float z[PPT][8];
      float ss = 0.f;
#pragma unroll
      for (int kk = 0; kk < PPT; ++kk) {
        const int idx = threadIdx.x + kk * kFThreads;
        if (idx < hp) {
          const uint4 zb = ld_cg(src + idx);
          st_plain(res + static_cast<int64_t>(t) * hp + idx, zb);
          unpack_bf16(zb, z[kk]);
#pragma unroll
          for (int e = 0; e < 8; ++e) ss += z[kk][e] * z[kk][e];
        }
      }
      norm_store<PPT>(z, ss, w, out + static_cast<int64_t>(t) * hp, hp, p.H, p.eps);
    }
  }
  end_call(me.wsp, rank, epoch);
}

// Rank-order sum of the ws partial rows in this rank's one-shot slots, plus
// the residual, then RMSNorm. The slot parity comes from the epoch of the
// last completed call (the GEMM that filled the slots).
template <int PPT>
__global__ void __launch_bounds__(kFThreads) k_slots_rmsnorm(const char* base, int64_t slot_off, int64_t slot_bytes,
                                                             int ws, int tile_tokens, int m_tiles, WaitCtx w,
                                                             uint4* residual, const uint4* wgt, uint4* out, int T,
                                                             int H, float eps) {
  pdl_wait();
  pdl_trigger();
  const SignalPad* pad = reinterpret_cast<const SignalPad*>(base);
  const uint32_t epoch = ld_volatile_u32(&pad->epoch);
  const int parity = epoch & 1;
  const uint64_t seq = make_seq(epoch, 0);
  w.epoch = epoch;
  const int hp = H / 8;
  auto slot = [&](int q) -> const char* {
    return base + slot_off + (static_cast<int64_t>(parity) * ws + q) * slot_bytes;
  };
  int ready_tile = -1;
  for (int t = blockIdx.x; t < T; t += gridDim.x) {
    if (tile_tokens > 0 && t / tile_tokens != ready_tile) {
      // every rank's output tiles covering row t must have landed here
      ready_tile = t / tile_tokens;
      bool ok = true;
      for (int i = threadIdx.x; i < m_tiles * ws; i += kFThreads) {
        const int m = i / ws, q = i % ws;
        ok &= wait_geq(&pad->gemm_flags[ready_tile * m_tiles + m][q], seq, w, static_cast<uint32_t>(q),
                       kStageGemmAR);
      }
      if (!__syncthreads_and(ok)) return;
    }
    float z[PPT][8];
    float ss = 0.f;
#pragma unroll
    for (int k = 0; k < PPT; ++k) {
      const int idx = threadIdx.x + k * kFThreads;
      if (idx < hp) {
        const int64_t o = static_cast<int64_t>(t) * hp + idx;
        uint4 v[kMaxRanks];
#pragma unroll
        for (int q = 0; q < kMaxRanks; ++q)
          if (q < ws) v[q] = ld_cg(reinterpret_cast<const uint4*>(slot(q)) + o);
        Acc<__nv_bfloat16> a;
        acc_set(a, v[0]);
#pragma unroll
        for (int q = 1; q < kMaxRanks; ++q)
          if (q < ws) acc_add(a, v[q]);
        ss += finish_pack(a, ld_plain(residual + o), residual + o, nullptr, z[k]);
      }
    }
    norm_store<PPT>(z, ss, wgt, out + static_cast<int64_t>(t) * hp, hp, H, eps);
  }
}

// Second half of the reduce-scatter GEMM + allreduce. Row t is owned by rank
// t % ws and its partials from every rank are in the owner's slots. Row
// blocks k hold rows [k ws, (k + 1) ws); CTA c takes blocks c, c + C, ...
//   phase A  for the owned row of each block: wait (bounded) for every rank's
//            tiles covering it, add the ws partials in rank order and the
//            residual -> z (bf16); residual = z, out = norm(z); z is stored
//            into row t of slot [this rank] on every rank (a row no GEMM
//            epilogue writes there: only the owner receives row t);
//   exchange release this CTA's flag on every peer, acquire every peer's;
//   phase B  for the other owners' rows of the same blocks: read z from this
//            rank's own slot [owner], residual = z, out = norm(z).
// All NVLink traffic is stores (posted writes; no load round trips).
// Every rank computes the norm from the same bf16 z, so all hold the same
// bits. A slot's parity is reused two calls later; by then every peer has
// passed this call's exchange of the next call, so nobody still reads it.
struct RsNormArgs {
  char* wsp[kMaxRanks];
  int64_t slot_off;
  int64_t slot_bytes;
  int ws;
  int rank;
  int tile_tokens;
  int m_tiles;
  WaitCtx w;
  uint4* residual;
  const uint4* wgt;
  uint4* out;
  int T;
  int H;
  float eps;
};

template <int PPT>
__global__ void __launch_bounds__(kFThreads) k_slots_rs_rmsnorm(const __grid_constant__ RsNormArgs a) {
  pdl_wait();
  pdl_trigger();
  const int rank = a.rank, ws = a.ws;
  const SignalPad* pad = reinterpret_cast<const SignalPad*>(a.wsp[rank]);
  const uint32_t epoch = ld_volatile_u32(&pad->epoch);
  const int parity = epoch & 1;
  WaitCtx w = a.w;
  w.epoch = epoch;
  const int hp = a.H / 8;
  const int nblocks = (a.T + ws - 1) / ws;
  auto slot_row = [&](int owner, int src, int t) -> uint4* {
    return reinterpret_cast<uint4*>(a.wsp[owner] + a.slot_off + (static_cast<int64_t>(parity) * ws + src) * a.slot_bytes) +
           static_cast<int64_t>(t) * hp;
  };
  // ---- phase A: owned rows
  int ready_tile = -1;
  bool ok = true;
  for (int k = blockIdx.x; k < nblocks && ok; k += gridDim.x) {
    const int t = k * ws + rank;
    if (t >= a.T) continue;
    if (t / a.tile_tokens != ready_tile) {
      ready_tile = t / a.tile_tokens;
      bool fine = true;
      for (int i = threadIdx.x; i < a.m_tiles * ws; i += kFThreads) {
        const int m = i / ws, q = i % ws;
        fine &= wait_geq(&pad->gemm_flags[ready_tile * a.m_tiles + m][q], make_seq(epoch, 0), w,
                         static_cast<uint32_t>(q), kStageGemmAR);
      }
      ok = __syncthreads_and(fine) != 0;
      if (!ok) break;
    }
    float z[PPT][8];
    float ss = 0.f;
    const int64_t o = static_cast<int64_t>(t) * hp;
#pragma unroll
    for (int kk = 0; kk < PPT; ++kk) {
      const int idx = threadIdx.x + kk * kFThreads;
      if (idx < hp) {
        uint4 v[kMaxRanks];
#pragma unroll
        for (int q = 0; q < kMaxRanks; ++q)
          if (q < ws) v[q] = ld_cg(slot_row(rank, q, t) + idx);
        Acc<__nv_bfloat16> acc;
        acc_set(acc, v[0]);
#pragma unroll
        for (int q = 1; q < kMaxRanks; ++q)
          if (q < ws) acc_add(acc, v[q]);
        ss += finish_pack(acc, ld_plain(a.residual + o + idx), a.residual + o + idx, nullptr, z[kk]);
        // publish z on every peer (staggered by rank)
        const uint4 zb = ld_plain(a.residual + o + idx);
        for (int j = 1; j < ws; ++j) st_plain(slot_row((rank + j) % ws, rank, t) + idx, zb);
      }
    }
    norm_store<PPT>(z, ss, a.wgt, a.out + o, hp, a.H, a.eps);
  }
  // ---- exchange with every peer (the same CTA index), then phase B
  int peers[kMaxRanks];
  all_peers_rt(ws, rank, peers);
  ok = exchange(a.wsp, rank, kFlagFusedAG, blockIdx.x, make_seq(epoch, 1), peers, ok ? ws - 1 : 0, w, kStageAG) &&
       ok;
  if (!ok) return;
  for (int k = blockIdx.x; k < nblocks; k += gridDim.x) {
    for (int j = 0; j < ws - 1; ++j) {
      const int q = peers[j];
      const int t = k * ws + q;
      if (t >= a.T) continue;
      const uint4* src = slot_row(rank, q, t);
      const int64_t o = static_cast<int64_t>(t) * hp;
      float z[PPT][8];
      float ss = 0.f;
#pragma unroll
      for (int kk = 0; kk < PPT; ++kk) {
        const int idx = threadIdx.x + kk * kFThreads;
        if (idx < hp) {
          const uint4 zb = ld_cg(src + idx);
          st_plain(a.residual + o + idx, zb);
          unpack_bf16(zb, z[kk]);
#pragma unroll
          for (int e = 0; e < 8; ++e) ss += z[kk][e] * z[kk][e];
        }
      }
      norm_store<PPT>(z, ss, a.wgt, a.out + o, hp, a.H, a.eps);
    }
  }
}

template <int WS, int PPT>
void* pick_kernel(int algo) {
  return algo == kFusedOneshot ? reinterpret_cast<void*>(&k_fused_oneshot<WS, PPT>)
                               : reinterpret_cast<void*>(&k_fused_twoshot<WS, PPT>);
}

template <int WS>
void* pick_ppt(int algo, int ppt) {
  switch (ppt) {
    case 1: return pick_kernel<WS, 1>(algo);
    case 2: return pick_kernel<WS, 2>(algo);
    case 4: return pick_kernel<WS, 4>(algo);
    default: return pick_kernel<WS, 8>(algo);
  }
}

void* pick(int ws, int algo, int ppt) {
  switch (ws) {
    case 2: return pick_ppt<2>(algo, ppt);
    case 3: return pick_ppt<3>(algo, ppt);
    case 4: return pick_ppt<4>(algo, ppt);
    case 5: return pick_ppt<5>(algo, ppt);
    case 6: return pick_ppt<6>(algo, ppt);
    case 7: return pick_ppt<7>(algo, ppt);
    case 8: return pick_ppt<8>(algo, ppt);
    default: throw std::invalid_argument("fused allreduce needs a world size in [2, 8]");
  }
}

int ppt_for(int64_t H) {
  const int64_t hp = H / 8;
  if (hp <= kFThreads) return 1;
  if (hp <= 2 * kFThreads) return 2;
  if (hp <= 4 * kFThreads) return 4;
  return 8;
}

void check_shape(int64_t T, int64_t H) {
  if (T < 1 || T > (int64_t(1) << 30)) throw std::invalid_argument("fused rmsnorm: bad token count");
  if (H < 8 || H % 8 != 0 || H > kFusedMaxHidden)
    throw std::invalid_argument("fused rmsnorm: hidden size must be a multiple of 8 up to 16384");
}

struct FusedPlan {
  int algo;
  dim3 grid;
  int rounds;
};

FusedPlan plan_fused(const Communicator& c, int64_t T, int64_t H, int algo) {
  const int ws = c.world_size();
  const int64_t bytes = T * H * 2;
  if (algo == kFusedAuto)
    algo = (bytes <= c.layout().fused_bytes && T <= 4 * static_cast<int64_t>(ws)) ? kFusedOneshot
                                                                                  : kFusedTwoshot;
  FusedPlan pl{algo, dim3(1), 0};
  if (algo == kFusedOneshot) {
    if (bytes > c.layout().fused_bytes) throw std::invalid_argument("fused one-shot: message too large");
    pl.grid = dim3(static_cast<unsigned>(std::min<int64_t>(T, c.config().oneshot_ctas)));
  } else if (algo == kFusedTwoshot) {
    const int64_t tiles = (T + ws - 1) / ws;
    const int64_t C = std::min<int64_t>(tiles, c.config().max_ctas);
    pl.grid = dim3(static_cast<unsigned>(C));
    pl.rounds = static_cast<int>((tiles + C - 1) / C);
  } else {
    throw std::invalid_argument("unknown fused allreduce algorithm");
  }
  return pl;
}

void fill(FusedParams& p, const Communicator& c, const FusedPlan& pl, int64_t T, int64_t H, float eps) {
  p.err = c.err_dev();
  p.err_host = c.err_host();
  p.timeout_ns = c.config().timeout_ns;
  p.ws = c.world_size();
  p.T = static_cast<int>(T);
  p.H = static_cast<int>(H);
  p.rounds = pl.rounds;
  p.eps = eps;
  p.L = c.layout();
}

FusedView make_view(const Communicator& c, const void* in, void* residual, const void* weight, void* out) {
  FusedView v{};
  v.in = static_cast<const char*>(in);
  v.residual = static_cast<char*>(residual);
  v.weight = static_cast<const char*>(weight);
  v.out = static_cast<char*>(out);
  for (int i = 0; i < c.world_size(); ++i) v.wsp[i] = c.wsp(i);
  v.rank = c.rank();
  return v;
}

// Launch as a programmatic dependent launch: the CTAs become resident while
// the kernel before is still running and start at its completion
// (griddepcontrol.wait at the top of the kernel).
template <typename... KArgs, typename... Args>
void launch_pdl(void (*kernel)(KArgs...), int grid, int block, cudaStream_t s, Args... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(block);
  cfg.stream = s;
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr.val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = &attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
  if (e != cudaSuccess) throw std::runtime_error(std::string("norm launch failed: ") + cudaGetErrorString(e));
}

void check_ptrs(const void* a, const void* b, const void* c, const void* d) {
  for (const void* x : {a, b, c, d})
    if (reinterpret_cast<uintptr_t>(x) % 16 != 0) throw std::invalid_argument("fused rmsnorm: 16-byte alignment");
}

}  // namespace

void slots_rmsnorm(Communicator& c, cudaStream_t s, void* residual, const void* weight, void* out, int64_t T,
                   int64_t H, float eps, int tile_tokens) {
  check_shape(T, H);
  if (reinterpret_cast<uintptr_t>(residual) % 16 || reinterpret_cast<uintptr_t>(weight) % 16 ||
      reinterpret_cast<uintptr_t>(out) % 16)
    throw std::invalid_argument("slots rmsnorm: 16-byte alignment");
  if (H % 128 != 0 && tile_tokens > 0) throw std::invalid_argument("slots rmsnorm: H must be a multiple of 128");
  const Layout& L = c.layout();
  const char* base = c.wsp(c.rank());
  WaitCtx w{};
  w.err = c.err_dev();
  w.err_host = c.err_host();
  w.abort = &reinterpret_cast<SignalPad*>(c.wsp(c.rank()))->abort;
  w.timeout_ns = c.config().timeout_ns;
  w.rank = static_cast<uint32_t>(c.rank());
  const int grid = static_cast<int>(std::min<int64_t>(T, 148 * 4));
  auto* r4 = static_cast<uint4*>(residual);
  const auto* w4 = static_cast<const uint4*>(weight);
  auto* o4 = static_cast<uint4*>(out);
  const int t = static_cast<int>(T), h = static_cast<int>(H), ws = c.world_size();
  const int m_tiles = h / 128;
  switch (ppt_for(H)) {
    case 1: launch_pdl(k_slots_rmsnorm<1>, grid, kFThreads, s, base, L.fused_off, L.fused_bytes, ws, tile_tokens, m_tiles, w, r4, w4, o4, t, h, eps); break;
    case 2: launch_pdl(k_slots_rmsnorm<2>, grid, kFThreads, s, base, L.fused_off, L.fused_bytes, ws, tile_tokens, m_tiles, w, r4, w4, o4, t, h, eps); break;
    case 4: launch_pdl(k_slots_rmsnorm<4>, grid, kFThreads, s, base, L.fused_off, L.fused_bytes, ws, tile_tokens, m_tiles, w, r4, w4, o4, t, h, eps); break;
    default: launch_pdl(k_slots_rmsnorm<8>, grid, kFThreads, s, base, L.fused_off, L.fused_bytes, ws, tile_tokens, m_tiles, w, r4, w4, o4, t, h, eps); break;
  }
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) throw std::runtime_error(std::string("slots rmsnorm launch failed: ") + cudaGetErrorString(e));
  c.count_launch();
}

void slots_rs_rmsnorm(Communicator& c, cudaStream_t s, void* residual, const void* weight, void* out, int64_t T,
                      int64_t H, float eps, int tile_tokens) {
  check_shape(T, H);
  if (reinterpret_cast<uintptr_t>(residual) % 16 || reinterpret_cast<uintptr_t>(weight) % 16 ||
      reinterpret_cast<uintptr_t>(out) % 16)
    throw std::invalid_argument("slots rmsnorm: 16-byte alignment");
  if (H % 128 != 0 || tile_tokens < 1) throw std::invalid_argument("slots rmsnorm: H must be a multiple of 128");
  const int ws = c.world_size();
  const Layout& L = c.layout();
  RsNormArgs a{};
  for (int r = 0; r < ws; ++r) a.wsp[r] = c.wsp(r);
  a.slot_off = L.fused_off;
  a.slot_bytes = L.fused_bytes;
  a.ws = ws;
  a.rank = c.rank();
  a.tile_tokens = tile_tokens;
  a.m_tiles = static_cast<int>(H / 128);
  a.w.err = c.err_dev();
  a.w.err_host = c.err_host();
  a.w.abort = &reinterpret_cast<SignalPad*>(c.wsp(c.rank()))->abort;
  a.w.timeout_ns = c.config().timeout_ns;
  a.w.rank = static_cast<uint32_t>(c.rank());
  a.residual = static_cast<uint4*>(residual);
  a.wgt = static_cast<const uint4*>(weight);
  a.out = static_cast<uint4*>(out);
  a.T = static_cast<int>(T);
  a.H = static_cast<int>(H);
  a.eps = eps;
  // one CTA per row block, at most one per flag slot; every CTA of every
  // rank must be resident at once (they wait on each other): 256 threads,
  // no dynamic shared memory, far below the device's capacity
  const int grid = static_cast<int>(std::min<int64_t>((T + ws - 1) / ws, 148));
  switch (ppt_for(H)) {
    case 1: launch_pdl(k_slots_rs_rmsnorm<1>, grid, kFThreads, s, a); break;
    case 2: launch_pdl(k_slots_rs_rmsnorm<2>, grid, kFThreads, s, a); break;
    case 4: launch_pdl(k_slots_rs_rmsnorm<4>, grid, kFThreads, s, a); break;
    default: launch_pdl(k_slots_rs_rmsnorm<8>, grid, kFThreads, s, a); break;
  }
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) throw std::runtime_error(std::string("slots rs rmsnorm launch failed: ") + cudaGetErrorString(e));
  c.count_launch();
}

void rmsnorm_residual(cudaStream_t s, const void* inp, void* residual, const void* weight, void* out,
                      int64_t T, int64_t H, float eps) {
  check_shape(T, H);
  check_ptrs(inp, residual, weight, out);
  const int grid = static_cast<int>(std::min<int64_t>(T, 148 * 8));
  const auto* i4 = static_cast<const uint4*>(inp);
  auto* r4 = static_cast<uint4*>(residual);
  const auto* w4 = static_cast<const uint4*>(weight);
  auto* o4 = static_cast<uint4*>(out);
  const int t = static_cast<int>(T), h = static_cast<int>(H);
  switch (ppt_for(H)) {
    case 1: launch_pdl(k_rmsnorm<1>, grid, kFThreads, s, i4, r4, w4, o4, t, h, eps); break;
    case 2: launch_pdl(k_rmsnorm<2>, grid, kFThreads, s, i4, r4, w4, o4, t, h, eps); break;
    case 4: launch_pdl(k_rmsnorm<4>, grid, kFThreads, s, i4, r4, w4, o4, t, h, eps); break;
    default: launch_pdl(k_rmsnorm<8>, grid, kFThreads, s, i4, r4, w4, o4, t, h, eps); break;
  }
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) throw std::runtime_error(std::string("rmsnorm launch failed: ") + cudaGetErrorString(e));
}

int fused_allreduce_rmsnorm(Communicator& c, cudaStream_t s, const void* inp, void* residual,
                            const void* weight, void* out, int64_t T, int64_t H, float eps, int algo) {
  check_shape(T, H);
  check_ptrs(inp, residual, weight, out);
  if (c.world_size() == 1) {
    rmsnorm_residual(s, inp, residual, weight, out, T, H, eps);
    c.count_launch();
    return kFusedAuto;
  }
  const FusedPlan pl = plan_fused(c, T, H, algo);
  FusedParams p{};
  fill(p, c, pl, T, H, eps);
  p.v[0] = make_view(c, inp, residual, weight, out);
  void* fn = pick(c.world_size(), pl.algo, ppt_for(H));
  void* args[] = {&p};
  const cudaError_t e = cudaLaunchKernel(fn, pl.grid, dim3(kFThreads), args, 0, s);
  if (e != cudaSuccess) throw std::runtime_error(std::string("fused launch failed: ") + cudaGetErrorString(e));
  c.count_launch();
  return pl.algo;
}

int emulate_fused_allreduce_rmsnorm(const std::vector<Communicator*>& comms, cudaStream_t s,
                                    const std::vector<const void*>& ins,
                                    const std::vector<void*>& residuals,
                                    const std::vector<const void*>& weights,
                                    const std::vector<void*>& outs, int64_t T, int64_t H, float eps,
                                    int algo) {
  const int ws = static_cast<int>(comms.size());
  if (ws < 2 || ws > kMaxRanks || static_cast<int>(ins.size()) != ws ||
      static_cast<int>(residuals.size()) != ws || static_cast<int>(weights.size()) != ws ||
      static_cast<int>(outs.size()) != ws)
    throw std::invalid_argument("fused emulation needs 2..8 ranks with one buffer set each");
  check_shape(T, H);
  FusedPlan pl = plan_fused(*comms[0], T, H, algo);
  int dev = 0, sms = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const unsigned cap = static_cast<unsigned>(std::max(1, sms / ws));
  if (pl.grid.x > cap) {
    pl.grid.x = cap;
    if (pl.algo == kFusedTwoshot) {
      const int64_t tiles = (T + ws - 1) / ws;
      pl.rounds = static_cast<int>((tiles + cap - 1) / cap);
    }
  }
  FusedParams p{};
  fill(p, *comms[0], pl, T, H, eps);
  for (int r = 0; r < ws; ++r) {
    check_ptrs(ins[r], residuals[r], weights[r], outs[r]);
    p.v[r] = make_view(*comms[r], ins[r], residuals[r], weights[r], outs[r]);
  }
  pl.grid.y = ws;
  void* fn = pick(ws, pl.algo, ppt_for(H));
  void* args[] = {&p};
  const cudaError_t e = cudaLaunchCooperativeKernel(fn, pl.grid, dim3(kFThreads), args, 0, s);
  if (e != cudaSuccess)
    throw std::runtime_error(std::string("fused emulation launch failed: ") + cudaGetErrorString(e));
  for (auto* c : comms) c->count_launch();
  return pl.algo;
}

}  // namespace nab
