// Allreduce kernels for B200 over NVLink 5 / NVSwitch, and their launcher.
//
// Every kernel reduces in fp32 in ascending rank order and rounds once, so all
// ranks produce bit-identical results and a CPU fp32 sum in rank order is an
// exact oracle.
//
// Protocols (capability parity with the reference's effective kernel, vLLM's
// one-/two-shot custom allreduce reached through ops.all_reduce in
// src/numa_all_reduce.py:354-357, and with its dead three-stage kernels in
// src/numa_all_reduce.cu:228-344):
//   oneshot       push the whole input into every peer's slot (double
//                 buffered by call parity), one flag exchange, every rank
//                 reduces everything. No end barrier.
//   twoshot       tiled rounds per CTA: push chunk j to owner j (reduce-
//                 scatter by stores), owner reduces, peers pull the result
//                 (all-gather by loads). Workspace is independent of message
//                 size; no start or end barrier.
//   hier          the reference's three stages done right: intra-group RS,
//                 exchange of partial sums between same-slice owners of other
//                 groups, intra-group AG.
//   oneshot_pull  registered inputs (CUDA-graph path): read peers' buffers
//                 in place between a start and an end barrier.
//   nvls_oneshot  copy into the multicast-bound workspace, one arrival
//                 counter, multimem.ld_reduce of the whole message.
//   nvls_twoshot  tiled rounds: copy in, multimem.ld_reduce own chunk,
//                 multimem.st of the result to every GPU, copy out.
//   copy          world size 1.
#include <cuda_runtime.h>

#include <cstdio>

#include "nab_device.cuh"
#include "nab_kernels.h"
#include "nab_params.h"
#include "nab_proto.cuh"

namespace nab {

namespace {

constexpr int kThreads = 512;

NAB_DINLINE SignalPad* pad_of(const RankView& me, int r) { return pad_at(me.wsp, r); }

NAB_DINLINE uint32_t begin_call(const RankView& me) { return ::nab::begin_call(me.wsp, me.rank); }

NAB_DINLINE void end_call(const RankView& me, uint32_t epoch) { ::nab::end_call(me.wsp, me.rank, epoch); }

NAB_DINLINE WaitCtx make_wait(const ARParams& p, const RankView& me, uint32_t epoch) {
  return ::nab::make_wait(p.err, p.err_host, p.timeout_ns, me.wsp, me.rank, epoch);
}

NAB_DINLINE bool exchange(const RankView& me, int kind, int slot, uint64_t seq, const int* peers,
                          int npeers, const WaitCtx& w, uint32_t stage) {
  return ::nab::exchange(me.wsp, me.rank, kind, slot, seq, peers, npeers, w, stage);
}

// Debug builds: checks of a launch made by every CTA before it touches any
// memory (the rank, the world size, the flag slot of this CTA, 16-byte
// aligned buffers and, through region_ok, that this CTA's slots lie inside
// the workspace). A CTA whose check fails records it and returns; its peers'
// bounded waits then run out. Always true in release builds.
NAB_DINLINE bool launch_ok(const ARParams& p, const RankView& me, int ws, bool region_ok) {
  if (!NAB_DEBUG_BOUNDS) return true;
  const bool ok = me.rank >= 0 && me.rank < ws && p.ws == ws && blockIdx.x < kMaxBlocks && p.npacks > 0 &&
                  ((reinterpret_cast<uintptr_t>(me.in) | reinterpret_cast<uintptr_t>(me.out)) & 15u) == 0 &&
                  region_ok;
  return dbg_ok(ok, p.err, p.err_host, static_cast<uint32_t>(me.rank));
}

// Debug builds: a pack index below its bound (records and skips the access
// otherwise).
#define NAB_DBG_IDX(idx, n) (!NAB_DEBUG_BOUNDS || dbg_ok((idx) < (n), p.err, p.err_host, static_cast<uint32_t>(idx)))

// Slot regions of CTA c inside the IPC / multicast workspaces (debug checks).
template <int WS>
NAB_DINLINE bool pipe_region_ok(const ARParams& p, int c, int chp) {
  return c < p.L.pipe_ctas && static_cast<int64_t>(chp) * 16 <= p.L.pipe_chunk &&
         p.L.pipe_off + static_cast<int64_t>(c + 1) * kPipeSlots * 2 * WS * p.L.pipe_chunk <= p.L.ws_bytes;
}
template <int WS>
NAB_DINLINE bool nvls_region_ok(const ARParams& p, const RankView& me, int c, int chp) {
  return me.mc != nullptr && me.uc != nullptr && c < kNvlsCtas && static_cast<int64_t>(chp) * 16 <= p.L.nvls_chunk &&
         p.L.mc_twoshot_off + static_cast<int64_t>(c + 1) * kNvlsSlots * WS * p.L.nvls_chunk <= p.L.mc_bytes;
}

// ------------------------------------------------------------------ copy ----
__global__ void __launch_bounds__(kThreads) k_copy(const __grid_constant__ ARParams p) {
  const RankView& me = p.v[blockIdx.y];
  const uint4* src = reinterpret_cast<const uint4*>(me.in);
  uint4* dst = reinterpret_cast<uint4*>(me.out);
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  for (; i + 3 * stride < p.npacks; i += 4 * stride) {
    uint4 a = ld_plain(src + i), b = ld_plain(src + i + stride);
    uint4 c = ld_plain(src + i + 2 * stride), d = ld_plain(src + i + 3 * stride);
    st_plain(dst + i, a);
    st_plain(dst + i + stride, b);
    st_plain(dst + i + 2 * stride, c);
    st_plain(dst + i + 3 * stride, d);
  }
  for (; i < p.npacks; i += stride) st_plain(dst + i, ld_plain(src + i));
}

NAB_DINLINE void named_barrier(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// Loads in flight per thread: each phase issues all of its loads for U
// consecutive packs before the first store, so a warp keeps ~8 independent
// 16-byte requests outstanding (NVLink round trips are ~1-2 us).
template <int WS>
struct Unroll {
  static constexpr int kPeer = (WS - 1) >= 8 ? 1 : 8 / (WS - 1);  // one load per peer per pack
  static constexpr int kRed = WS >= 8 ? 1 : 8 / WS;               // WS loads per pack
};

// --------------------------------------------------------------- oneshot ----
template <typename T, int WS>
__global__ void __launch_bounds__(kThreads, 2) k_oneshot(const __grid_constant__ ARParams p) {
  constexpr int U = 4;
  constexpr int UR = Unroll<WS>::kRed;
  const RankView& me = p.v[blockIdx.y];
  if (!launch_ok(p, me, WS, p.npacks * 16 <= p.L.oneshot_max &&
                                p.L.oneshot_off + 2 * WS * p.L.oneshot_max <= p.L.ws_bytes))
    return;
  const int rank = me.rank;
  const uint32_t epoch = begin_call(me);
  const WaitCtx w = make_wait(p, me, epoch);
  const int parity = epoch & 1;
  const int64_t per = ceil_div<int64_t>(p.npacks, gridDim.x);
  const int64_t beg = per * blockIdx.x;
  const int64_t end = min(p.npacks, beg + per);
  const uint4* src = reinterpret_cast<const uint4*>(me.in);
  const int64_t slot_packs = p.L.oneshot_max / 16;
  auto slot = [&](int owner_rank, int src_rank) -> uint4* {
    return reinterpret_cast<uint4*>(me.wsp[owner_rank] + p.L.oneshot_off) +
           (static_cast<int64_t>(parity) * WS + src_rank) * slot_packs;
  };
  // 1. push my input into slot [rank] of every peer
  for (int64_t i0 = beg + threadIdx.x; i0 < end; i0 += static_cast<int64_t>(blockDim.x) * U) {
    uint4 x[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t i = i0 + static_cast<int64_t>(u) * blockDim.x;
      if (i < end) x[u] = ld_plain(src + i);
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t i = i0 + static_cast<int64_t>(u) * blockDim.x;
      if (i < end && NAB_DBG_IDX(i, slot_packs)) {
#pragma unroll
        for (int k = 1; k < WS; ++k) st_plain(slot((rank + k) % WS, rank) + i, x[u]);
      }
    }
  }
  int peers[WS > 1 ? WS - 1 : 1];
  all_peers<WS>(rank, peers);
  const bool ok = exchange(me, kFlagOneshot, blockIdx.x, make_seq(epoch, 0), peers, WS - 1, w,
                           kStageOneshot);
  // 2. reduce all WS contributions in rank order
  if (ok) {
    uint4* dst = reinterpret_cast<uint4*>(me.out);
    for (int64_t i0 = beg + threadIdx.x; i0 < end; i0 += static_cast<int64_t>(blockDim.x) * UR) {
      uint4 x[UR][WS];
#pragma unroll
      for (int u = 0; u < UR; ++u) {
        const int64_t i = i0 + static_cast<int64_t>(u) * blockDim.x;
        if (i < end) {
#pragma unroll
          for (int q = 0; q < WS; ++q) x[u][q] = (q == rank) ? ld_plain(src + i) : ld_cg(slot(rank, q) + i);
        }
      }
#pragma unroll
      for (int u = 0; u < UR; ++u) {
        const int64_t i = i0 + static_cast<int64_t>(u) * blockDim.x;
        if (i < end) {
          Acc<T> a;
          acc_set(a, x[u][0]);
#pragma unroll
          for (int q = 1; q < WS; ++q) acc_add(a, x[u][q]);
          st_plain(dst + i, acc_pack(a));
        }
      }
    }
  }
  end_call(me, epoch);
}

// --------------------------------------------------------------- twoshot ----
template <typename T, int WS>
__global__ void __launch_bounds__(kThreads, 1) k_twoshot(const __grid_constant__ ARParams p) {
  constexpr int UP = Unroll<WS>::kPeer;
  constexpr int UR = Unroll<WS>::kRed;
  const RankView& me = p.v[blockIdx.y];
  if (!launch_ok(p, me, WS, static_cast<int>(blockIdx.x) < p.L.max_ctas &&
                                static_cast<int64_t>(p.chunk_packs) * 16 <= p.L.chunk_max &&
                                p.L.twoshot_off + static_cast<int64_t>(blockIdx.x + 1) * (WS + 1) * p.L.chunk_max <=
                                    p.L.ws_bytes))
    return;
  const int rank = me.rank;
  const uint32_t epoch = begin_call(me);
  const WaitCtx w = make_wait(p, me, epoch);
  const int c = blockIdx.x;
  const int chp = p.chunk_packs;
  const int64_t tile = static_cast<int64_t>(WS) * chp;
  const int64_t stripe = tile * gridDim.x;
  const int64_t slot_stride = p.L.chunk_max / 16;
  const int64_t cta_packs = (WS + 1) * slot_stride;
  const uint4* src = reinterpret_cast<const uint4*>(me.in);
  uint4* dst = reinterpret_cast<uint4*>(me.out);
  // CTA c's region in rank r's workspace: [WS rs slots][result]
  auto region = [&](int r) -> uint4* {
    return reinterpret_cast<uint4*>(me.wsp[r] + p.L.twoshot_off) + c * cta_packs;
  };
  int peers[WS - 1];
  all_peers<WS>(rank, peers);
  const int stride = blockDim.x;
  bool ok = true;
  for (int r = 0; r < p.rounds && ok; ++r) {
    const int64_t tbase = r * stripe + c * tile;
    const uint64_t seq = make_seq(epoch, r + 1);
    // valid packs of each owner's chunk in this round (the last round is ragged)
    auto chunk_len = [&](int owner) -> int {
      const int64_t b = tbase + static_cast<int64_t>(owner) * chp;
      return static_cast<int>(span_len(chp, p.npacks - b));
    };
    // 1. reduce-scatter by stores: chunk j -> owner j, slot [rank]
    {
      int len[WS - 1];
#pragma unroll
      for (int k = 0; k < WS - 1; ++k) len[k] = chunk_len(peers[k]);
      for (int i0 = threadIdx.x; i0 < chp; i0 += stride * UP) {
        uint4 x[UP][WS - 1];
#pragma unroll
        for (int u = 0; u < UP; ++u) {
          const int i = i0 + u * stride;
#pragma unroll
          for (int k = 0; k < WS - 1; ++k)
            if (i < len[k]) x[u][k] = ld_plain(src + tbase + static_cast<int64_t>(peers[k]) * chp + i);
        }
#pragma unroll
        for (int u = 0; u < UP; ++u) {
          const int i = i0 + u * stride;
#pragma unroll
          for (int k = 0; k < WS - 1; ++k)
            if (i < len[k]) st_plain(region(peers[k]) + rank * slot_stride + i, x[u][k]);
        }
      }
    }
    ok = exchange(me, kFlagRS, c, seq, peers, WS - 1, w, kStageRS);
    if (!ok) break;
    // 2. reduce my chunk; publish it in my result slot and in my output
    {
      uint4* mine = region(rank);
      const int mlen = chunk_len(rank);
      const int64_t mbase = tbase + static_cast<int64_t>(rank) * chp;
      for (int i0 = threadIdx.x; i0 < mlen; i0 += stride * UR) {
        uint4 x[UR][WS];
#pragma unroll
        for (int u = 0; u < UR; ++u) {
          const int i = i0 + u * stride;
          if (i < mlen) {
#pragma unroll
            for (int q = 0; q < WS; ++q)
              x[u][q] = (q == rank) ? ld_plain(src + mbase + i) : ld_cg(mine + q * slot_stride + i);
          }
        }
#pragma unroll
        for (int u = 0; u < UR; ++u) {
          const int i = i0 + u * stride;
          if (i < mlen) {
            Acc<T> a;
            acc_set(a, x[u][0]);
#pragma unroll
            for (int q = 1; q < WS; ++q) acc_add(a, x[u][q]);
            const uint4 y = acc_pack(a);
            st_plain(mine + WS * slot_stride + i, y);
            st_plain(dst + mbase + i, y);
          }
        }
      }
    }
    ok = exchange(me, kFlagAG, c, seq, peers, WS - 1, w, kStageAG);
    if (!ok) break;
    // 3. all-gather by loads from every owner's result slot
    {
      int len[WS - 1];
#pragma unroll
      for (int k = 0; k < WS - 1; ++k) len[k] = chunk_len(peers[k]);
      for (int i0 = threadIdx.x; i0 < chp; i0 += stride * UP) {
        uint4 x[UP][WS - 1];
#pragma unroll
        for (int u = 0; u < UP; ++u) {
          const int i = i0 + u * stride;
#pragma unroll
          for (int k = 0; k < WS - 1; ++k)
            if (i < len[k]) x[u][k] = ld_cg(region(peers[k]) + WS * slot_stride + i);
        }
#pragma unroll
        for (int u = 0; u < UP; ++u) {
          const int i = i0 + u * stride;
#pragma unroll
          for (int k = 0; k < WS - 1; ++k)
            if (i < len[k]) st_plain(dst + tbase + static_cast<int64_t>(peers[k]) * chp + i, x[u][k]);
        }
      }
    }
  }
  end_call(me, epoch);
}

// --------------------------------------------------------- twoshot pipe ----
// Pipelined, warp-specialised two-shot with both phases done by stores (an
// NVLink write carries its data in one packet; a read needs a request and a
// response). Tiles of WS chunks flow through a ring of kPipeSlots slots per
// CTA; every rank holds, per slot, WS reduce-scatter chunks and WS
// all-gather chunks (one of each per source rank).
//   pusher warps   store chunk j of tile k into owner j's slot, then release
//                  the owner's per-CTA "pushed" flag (value: tile k + 1);
//   reducer warps  acquire every peer's "pushed" flag, reduce the own chunk,
//                  write it to the output and store it into every peer's
//                  all-gather chunk, then release the peers' "reduced" flag;
//   copier warps   acquire every owner's "reduced" flag, copy the gathered
//                  chunks from the local slot into the output, free the slot.
// Flags are monotonic per CTA and peer ((epoch << 20) | tile + 1), so one
// flag covers every slot. A slot is reused by tile k + S only after this
// rank's copiers finished tile k; every peer pushes tile k + S (and thus
// overwrites this rank's chunks of tile k) only after its own copiers
// finished tile k, which needed this rank's reduction of tile k.
constexpr int kPushWarps = 4, kReduceWarps = 4, kPullWarps = 8;
static_assert((kPushWarps + kReduceWarps + kPullWarps) * 32 == kThreads, "warp groups must fill the CTA");

NAB_DINLINE bool wait_geq_cta(const uint64_t* addr, uint64_t target, const WaitCtx& w, uint32_t peer,
                              uint32_t stage, volatile int* s_abort) {
  uint64_t v = ld_acquire_sys(addr);
  if (static_cast<int64_t>(v - target) >= 0) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t it = 1;; ++it) {
    v = ld_acquire_sys(addr);
    if (static_cast<int64_t>(v - target) >= 0) return true;
    if ((it & 127u) == 0u) {
      if (*s_abort || ld_volatile_u32(w.abort) != 0u) return false;
      if (globaltimer_ns() - t0 > w.timeout_ns) {
        record_failure(w, kErrTimeout, peer, stage, static_cast<uint32_t>(v));
        return false;
      }
    }
  }
}

// Body of the pipelined P2P two-shot for CTA c of C on packs [0, npacks) of
// src/dst (a hybrid launch passes a prefix of the message).
template <typename T, int WS>
__device__ __forceinline__ void twoshot_pipe_body(const ARParams& p, const RankView& me, uint32_t epoch,
                                                  const WaitCtx& w, int c, int C, const uint4* src, uint4* dst,
                                                  int64_t npacks, int chp) {
  constexpr int S = kPipeSlots;
  constexpr int UP = Unroll<WS>::kPeer;
  constexpr int UR = Unroll<WS>::kRed;
  const int rank = me.rank;
  const int64_t tile = static_cast<int64_t>(WS) * chp;
  const int64_t ntiles = (npacks + tile - 1) / tile;
  const int64_t my_tiles = ntiles > c ? (ntiles - c + C - 1) / C : 0;
  const int64_t cstride = p.L.pipe_chunk / 16;
  const int64_t slot_packs = 2 * WS * cstride;  // [WS rs chunks][WS ag chunks]
  auto ring = [&](int r) -> uint4* {
    return reinterpret_cast<uint4*>(me.wsp[r] + p.L.pipe_off) + static_cast<int64_t>(c) * S * slot_packs;
  };
  SignalPad* mypad = pad_of(me, rank);
  int peers[WS - 1];
  all_peers<WS>(rank, peers);

  __shared__ int s_abort;
  __shared__ int64_t s_done;  // tiles the pullers have finished (in order)
  if (threadIdx.x == 0) {
    s_abort = 0;
    s_done = 0;
  }
  __syncthreads();
  volatile int* abort_flag = &s_abort;
  volatile int64_t* done = &s_done;
  const int warp = threadIdx.x >> 5;
  auto chunk_len = [&](int64_t tb, int owner) -> int {
    return static_cast<int>(span_len(chp, npacks - (tb + static_cast<int64_t>(owner) * chp)));
  };

  if (warp < kPushWarps) {
    // -------------------------------------------------------------- pushers
    const int t = threadIdx.x, nt = kPushWarps * 32;
    for (int64_t k = 0; k < my_tiles; ++k) {
      const int slot = static_cast<int>(k % S);
      if (t == 0 && k >= S) {
        const uint64_t t0 = globaltimer_ns();
        while (*done < k - S + 1 && !*abort_flag) {
          if (globaltimer_ns() - t0 > w.timeout_ns) {
            record_failure(w, kErrTimeout, 0xffffffffu, kStageRS, static_cast<uint32_t>(*done));
            *abort_flag = 1;
          }
        }
      }
      if (named_barrier_or(1, nt, *abort_flag != 0)) break;
      const int64_t tb = (c + k * C) * tile;
      int len[WS - 1];
#pragma unroll
      for (int q = 0; q < WS - 1; ++q) len[q] = chunk_len(tb, peers[q]);
      for (int i0 = t; i0 < chp; i0 += nt * UP) {
        uint4 x[UP][WS - 1];
#pragma unroll
        for (int u = 0; u < UP; ++u) {
          const int i = i0 + u * nt;
#pragma unroll
          for (int q = 0; q < WS - 1; ++q)
            if (i < len[q]) x[u][q] = ld_plain(src + tb + static_cast<int64_t>(peers[q]) * chp + i);
        }
#pragma unroll
        for (int u = 0; u < UP; ++u) {
          const int i = i0 + u * nt;
#pragma unroll
          for (int q = 0; q < WS - 1; ++q)
            if (i < len[q] && NAB_DBG_IDX(tb + static_cast<int64_t>(peers[q]) * chp + i, npacks))
              st_plain(ring(peers[q]) + slot * slot_packs + rank * cstride + i, x[u][q]);
        }
      }
      named_barrier(1, nt);
      if (t < WS - 1) st_release_sys(&pad_at(me.wsp, peers[t])->flags[kFlagPipeRS].v[c][rank], make_seq(epoch, k + 1));
    }
  } else if (warp < kPushWarps + kReduceWarps) {
    // ------------------------------------------------------------- reducers
    const int t = threadIdx.x - kPushWarps * 32, nt = kReduceWarps * 32;
    for (int64_t k = 0; k < my_tiles; ++k) {
      const int slot = static_cast<int>(k % S);
      bool ok = true;
      if (t < WS - 1)
        ok = wait_geq_cta(&mypad->flags[kFlagPipeRS].v[c][peers[t]], make_seq(epoch, k + 1), w, peers[t], kStageRS,
                          abort_flag);
      if (!ok) *abort_flag = 1;
      if (named_barrier_or(2, nt, *abort_flag != 0)) break;
      const int64_t tb = (c + k * C) * tile;
      const int64_t mb = tb + static_cast<int64_t>(rank) * chp;
      const int mlen = chunk_len(tb, rank);
      uint4* mine = ring(rank) + slot * slot_packs;
      for (int i0 = t; i0 < mlen; i0 += nt * UR) {
        uint4 x[UR][WS];
#pragma unroll
        for (int u = 0; u < UR; ++u) {
          const int i = i0 + u * nt;
          if (i < mlen) {
#pragma unroll
            for (int q = 0; q < WS; ++q) x[u][q] = (q == rank) ? ld_plain(src + mb + i) : ld_cg(mine + q * cstride + i);
          }
        }
#pragma unroll
        for (int u = 0; u < UR; ++u) {
          const int i = i0 + u * nt;
          if (i < mlen && NAB_DBG_IDX(mb + i, npacks)) {
            Acc<T> a;
            acc_set(a, x[u][0]);
#pragma unroll
            for (int q = 1; q < WS; ++q) acc_add(a, x[u][q]);
            const uint4 y = acc_pack(a);
            st_plain(dst + mb + i, y);
#pragma unroll
            for (int q = 0; q < WS - 1; ++q)
              st_plain(ring(peers[q]) + slot * slot_packs + (WS + rank) * cstride + i, y);
          }
        }
      }
      named_barrier(2, nt);
      if (t < WS - 1) st_release_sys(&pad_at(me.wsp, peers[t])->flags[kFlagPipeAG].v[c][rank], make_seq(epoch, k + 1));
    }
  } else {
    // -------------------------------------------------------------- copiers
    const int t = threadIdx.x - (kPushWarps + kReduceWarps) * 32, nt = kPullWarps * 32;
    for (int64_t k = 0; k < my_tiles; ++k) {
      const int slot = static_cast<int>(k % S);
      bool ok = true;
      if (t < WS - 1)
        ok = wait_geq_cta(&mypad->flags[kFlagPipeAG].v[c][peers[t]], make_seq(epoch, k + 1), w, peers[t], kStageAG,
                          abort_flag);
      if (!ok) *abort_flag = 1;
      if (named_barrier_or(3, nt, *abort_flag != 0)) break;
      const int64_t tb = (c + k * C) * tile;
      int len[WS - 1];
#pragma unroll
      for (int q = 0; q < WS - 1; ++q) len[q] = chunk_len(tb, peers[q]);
      for (int i0 = t; i0 < chp; i0 += nt * UP) {
        uint4 x[UP][WS - 1];
#pragma unroll
        for (int u = 0; u < UP; ++u) {
          const int i = i0 + u * nt;
#pragma unroll
          for (int q = 0; q < WS - 1; ++q)
            if (i < len[q]) x[u][q] = ld_cg(ring(rank) + slot * slot_packs + (WS + peers[q]) * cstride + i);
        }
#pragma unroll
        for (int u = 0; u < UP; ++u) {
          const int i = i0 + u * nt;
#pragma unroll
          for (int q = 0; q < WS - 1; ++q)
            if (i < len[q] && NAB_DBG_IDX(tb + static_cast<int64_t>(peers[q]) * chp + i, npacks))
              st_plain(dst + tb + static_cast<int64_t>(peers[q]) * chp + i, x[u][q]);
        }
      }
      named_barrier(3, nt);
      if (t == 0) {
        __threadfence_block();
        *done = k + 1;
      }
    }
  }
}

template <typename T, int WS>
__global__ void __launch_bounds__(kThreads, 1) k_twoshot_pipe(const __grid_constant__ ARParams p) {
  const RankView& me = p.v[blockIdx.y];
  if (!launch_ok(p, me, WS, pipe_region_ok<WS>(p, blockIdx.x, p.chunk_packs))) return;
  const uint32_t epoch = begin_call(me);
  const WaitCtx w = make_wait(p, me, epoch);
  twoshot_pipe_body<T, WS>(p, me, epoch, w, blockIdx.x, gridDim.x, reinterpret_cast<const uint4*>(me.in),
                           reinterpret_cast<uint4*>(me.out), p.npacks, p.chunk_packs);
  end_call(me, epoch);
}

// ------------------------------------------------------------------ hier ----
// Stage 1: reduce-scatter inside the group (chunk l -> local index l).
// Stage 2: the owners of chunk l in all groups exchange their partial sums in
//          fp32 (double-buffered by the CTA's global round parity) and each
//          adds them in group order, so the result is rounded exactly once.
// Stage 3: all-gather inside the group by loads.
template <typename T>
__global__ void __launch_bounds__(kThreads) k_hier(const __grid_constant__ ARParams p) {
  constexpr int XW = AccWords<T>::kW;
  const RankView& me = p.v[blockIdx.y];
  if (!launch_ok(p, me, p.ws, p.gsize * p.ngroups == p.ws && static_cast<int>(blockIdx.x) < p.L.hier_ctas &&
                                  static_cast<int64_t>(p.chunk_packs) * 16 <= p.L.hier_chunk &&
                                  p.L.hier_off + static_cast<int64_t>(blockIdx.x + 1) * (p.gsize + 4 * p.ngroups + 1) *
                                                     p.L.hier_chunk <= p.L.ws_bytes))
    return;
  const int rank = me.rank;
  const uint32_t epoch = begin_call(me);
  const WaitCtx w = make_wait(p, me, epoch);
  const int c = blockIdx.x;
  const int G = p.gsize, NG = p.ngroups;
  const int g = p.group_of[rank], l = p.lidx_of[rank];
  const int chp = p.chunk_packs;
  const int64_t tile = static_cast<int64_t>(G) * chp;
  const int64_t stripe = tile * gridDim.x;
  const int64_t slot_stride = p.L.hier_chunk / 16;
  // per CTA: [G rs slots][2 parities x NG groups x 2 widths of fp32 partials][result]
  const int64_t cta_packs = (G + 4 * NG + 1) * slot_stride;
  const int64_t res_off = (G + 4 * NG) * slot_stride;
  const uint4* src = reinterpret_cast<const uint4*>(me.in);
  uint4* dst = reinterpret_cast<uint4*>(me.out);
  auto region = [&](int r) -> uint4* {
    return reinterpret_cast<uint4*>(me.wsp[r] + p.L.hier_off) + c * cta_packs;
  };
  auto xslot = [&](int par, int h) -> int64_t { return (G + 2 * (par * NG + h)) * slot_stride; };
  int gpeers[kMaxRanks], xpeers[kMaxRanks];
  int ng = 0, nx = 0;
  for (int m = 0; m < G; ++m)
    if (m != l) gpeers[ng++] = p.member[g][m];
  for (int h = 0; h < NG; ++h)
    if (h != g) xpeers[nx++] = p.member[h][l];
  __shared__ uint32_t s_base;
  if (threadIdx.x == 0) s_base = ld_volatile_u32(&pad_of(me, rank)->hier_rounds[c]);
  __syncthreads();
  const uint32_t base_rounds = s_base;
  bool ok = true;
  for (int r = 0; r < p.rounds && ok; ++r) {
    const int64_t tbase = r * stripe + c * tile;
    const uint64_t seq = make_seq(epoch, r + 1);
    const int par = (base_rounds + r) & 1;
    // 1. intra-group reduce-scatter by stores
    for (int i = threadIdx.x; i < chp; i += blockDim.x) {
      for (int m = 0; m < G; ++m) {
        if (m == l) continue;
        const int64_t gi = tbase + static_cast<int64_t>(m) * chp + i;
        if (gi < p.npacks) st_plain(region(p.member[g][m]) + l * slot_stride + i, ld_plain(src + gi));
      }
    }
    ok = exchange(me, kFlagHierRS, c, seq, gpeers, ng, w, kStageRS);
    if (!ok) break;
    // 2a. fp32 group partial of chunk l -> my own slot and the same-slice owners
    uint4* mine = region(rank);
    for (int i = threadIdx.x; i < chp; i += blockDim.x) {
      const int64_t gi = tbase + static_cast<int64_t>(l) * chp + i;
      if (gi < p.npacks) {
        Acc<T> a;
        for (int m = 0; m < G; ++m) {
          const uint4 x = (m == l) ? ld_plain(src + gi) : ld_cg(mine + m * slot_stride + i);
          if (m == 0) acc_set(a, x); else acc_add(a, x);
        }
        const int64_t xs = xslot(par, g) + static_cast<int64_t>(i) * XW;
        acc_store_f32(mine + xs, a);
        for (int h = 0; h < NG; ++h)
          if (h != g) acc_store_f32(region(p.member[h][l]) + xs, a);
      }
    }
    ok = exchange(me, kFlagHierX, c, seq, xpeers, nx, w, kStageHierX);
    if (!ok) break;
    // 2b. add the group partials in group order, round once -> result slot and output
    for (int i = threadIdx.x; i < chp; i += blockDim.x) {
      const int64_t gi = tbase + static_cast<int64_t>(l) * chp + i;
      if (gi < p.npacks) {
        Acc<T> a;
        for (int h = 0; h < NG; ++h) acc_accum_f32(a, mine + xslot(par, h) + static_cast<int64_t>(i) * XW, h == 0);
        const uint4 y = acc_pack(a);
        st_plain(mine + res_off + i, y);
        st_plain(dst + gi, y);
      }
    }
    ok = exchange(me, kFlagHierAG, c, seq, gpeers, ng, w, kStageAG);
    if (!ok) break;
    // 3. intra-group all-gather by loads
    for (int i = threadIdx.x; i < chp; i += blockDim.x) {
      for (int m = 0; m < G; ++m) {
        if (m == l) continue;
        const int64_t gi = tbase + static_cast<int64_t>(m) * chp + i;
        if (gi < p.npacks) st_plain(dst + gi, ld_cg(region(p.member[g][m]) + res_off + i));
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) st_volatile_u32(&pad_of(me, rank)->hier_rounds[c], base_rounds + p.rounds);
  end_call(me, epoch);
}

// ---------------------------------------------------------- oneshot pull ----
template <typename T, int WS>
__global__ void __launch_bounds__(kThreads) k_oneshot_pull(const __grid_constant__ ARParams p) {
  const RankView& me = p.v[blockIdx.y];
  // the RankData slot must lie inside the registry
  if (!launch_ok(p, me, WS, me.reg != nullptr && me.reg < me.reg_end)) return;
  const int rank = me.rank;
  const uint32_t epoch = begin_call(me);
  const WaitCtx w = make_wait(p, me, epoch);
  const int64_t per = ceil_div<int64_t>(p.npacks, gridDim.x);
  const int64_t beg = per * blockIdx.x;
  const int64_t end = min(p.npacks, beg + per);
  int peers[WS - 1];
  all_peers<WS>(rank, peers);
  const uint64_t seq = make_seq(epoch, 0);
  bool ok = exchange(me, kFlagPullStart, blockIdx.x, seq, peers, WS - 1, w, kStagePullStart);
  if (ok) {
    const RankData rd = *me.reg;
    uint4* dst = reinterpret_cast<uint4*>(me.out);
    for (int64_t i = beg + threadIdx.x; i < end; i += blockDim.x) {
      uint4 x[WS];
#pragma unroll
      for (int q = 0; q < WS; ++q) x[q] = ld_cg(reinterpret_cast<const uint4*>(rd.ptrs[q]) + i);
      Acc<T> a;
      acc_set(a, x[0]);
#pragma unroll
      for (int q = 1; q < WS; ++q) acc_add(a, x[q]);
      st_plain(dst + i, acc_pack(a));
    }
    // nobody may overwrite its input while a peer still reads it
    exchange(me, kFlagPullEnd, blockIdx.x, seq, peers, WS - 1, w, kStagePullEnd);
  }
  end_call(me, epoch);
}

// ------------------------------------------ reduce-scatter / all-gather ----
// Contiguous-segment collectives, one launch per piece of at most
// oneshot_max bytes per segment (the host walks longer segments piece by
// piece). Both use the one-shot slots, double buffered by call parity: a rank
// can only start call e + 2 after every peer has arrived at call e + 1, which
// each does after its call e has finished reading, so no end barrier.
//   reduce-scatter: the input holds WS segments seg_stride packs apart; rank
//     r pushes segment j into slot [r] of rank j, then sums its own segment
//     over the WS contributions in rank order (fp32, one rounding).
//   all-gather: rank r pushes its input into slot [r] of every peer, then
//     copies the WS segments (its own from the input) into the output,
//     seg_stride packs apart.
// Capability parity: the reduce-scatter and all-gather stages of the
// reference's dead three-stage path (src/numa_all_reduce.cu:228-268, 318-344),
// here as standalone collectives over all ranks.
template <typename T, int WS>
__global__ void __launch_bounds__(kThreads, 1) k_reduce_scatter(const __grid_constant__ ARParams p) {
  constexpr int UP = Unroll<WS>::kPeer;
  constexpr int UR = Unroll<WS>::kRed;
  const RankView& me = p.v[blockIdx.y];
  if (!launch_ok(p, me, WS, p.npacks * 16 <= p.L.oneshot_max && p.seg_stride >= p.npacks &&
                                p.L.oneshot_off + 2 * WS * p.L.oneshot_max <= p.L.ws_bytes))
    return;
  const int rank = me.rank;
  const uint32_t epoch = begin_call(me);
  const WaitCtx w = make_wait(p, me, epoch);
  const int parity = epoch & 1;
  const int64_t per = ceil_div<int64_t>(p.npacks, gridDim.x);
  const int64_t beg = per * blockIdx.x;
  const int64_t end = min(p.npacks, beg + per);
  const uint4* src = reinterpret_cast<const uint4*>(me.in);
  const int64_t stride = p.seg_stride;
  const int64_t slot_packs = p.L.oneshot_max / 16;
  auto slot = [&](int owner_rank, int src_rank) -> uint4* {
    return reinterpret_cast<uint4*>(me.wsp[owner_rank] + p.L.oneshot_off) +
           (static_cast<int64_t>(parity) * WS + src_rank) * slot_packs;
  };
  // 1. segment j of my input -> slot [rank] of rank j
  for (int64_t i0 = beg + threadIdx.x; i0 < end; i0 += static_cast<int64_t>(blockDim.x) * UP) {
    uint4 x[UP][WS - 1];
#pragma unroll
    for (int u = 0; u < UP; ++u) {
      const int64_t i = i0 + static_cast<int64_t>(u) * blockDim.x;
      if (i < end) {
#pragma unroll
        for (int k = 1; k < WS; ++k) x[u][k - 1] = ld_plain(src + ((rank + k) % WS) * stride + i);
      }
    }
#pragma unroll
    for (int u = 0; u < UP; ++u) {
      const int64_t i = i0 + static_cast<int64_t>(u) * blockDim.x;
      if (i < end && NAB_DBG_IDX(i, slot_packs)) {
#pragma unroll
        for (int k = 1; k < WS; ++k) st_plain(slot((rank + k) % WS, rank) + i, x[u][k - 1]);
      }
    }
  }
  int peers[WS - 1];
  all_peers<WS>(rank, peers);
  const bool ok = exchange(me, kFlagScatter, blockIdx.x, make_seq(epoch, 0), peers, WS - 1, w,
                           kStageReduceScatter);
  // 2. my segment: the WS contributions in rank order
  if (ok) {
    uint4* dst = reinterpret_cast<uint4*>(me.out);
    const uint4* own = src + rank * stride;
    for (int64_t i0 = beg + threadIdx.x; i0 < end; i0 += static_cast<int64_t>(blockDim.x) * UR) {
      uint4 x[UR][WS];
#pragma unroll
      for (int u = 0; u < UR; ++u) {
        const int64_t i = i0 + static_cast<int64_t>(u) * blockDim.x;
        if (i < end) {
#pragma unroll
          for (int q = 0; q < WS; ++q) x[u][q] = (q == rank) ? ld_plain(own + i) : ld_cg(slot(rank, q) + i);
        }
      }
#pragma unroll
      for (int u = 0; u < UR; ++u) {
        const int64_t i = i0 + static_cast<int64_t>(u) * blockDim.x;
        if (i < end) {
          Acc<T> a;
          acc_set(a, x[u][0]);
#pragma unroll
          for (int q = 1; q < WS; ++q) acc_add(a, x[u][q]);
          st_plain(dst + i, acc_pack(a));
        }
      }
    }
  }
  end_call(me, epoch);
}

template <int WS>
__global__ void __launch_bounds__(kThreads, 1) k_all_gather(const __grid_constant__ ARParams p) {
  constexpr int U = 4;
  constexpr int UR = Unroll<WS>::kRed;
  const RankView& me = p.v[blockIdx.y];
  if (!launch_ok(p, me, WS, p.npacks * 16 <= p.L.oneshot_max && p.seg_stride >= p.npacks &&
                                p.L.oneshot_off + 2 * WS * p.L.oneshot_max <= p.L.ws_bytes))
    return;
  const int rank = me.rank;
  const uint32_t epoch = begin_call(me);
  const WaitCtx w = make_wait(p, me, epoch);
  const int parity = epoch & 1;
  const int64_t per = ceil_div<int64_t>(p.npacks, gridDim.x);
  const int64_t beg = per * blockIdx.x;
  const int64_t end = min(p.npacks, beg + per);
  const uint4* src = reinterpret_cast<const uint4*>(me.in);
  const int64_t stride = p.seg_stride;
  const int64_t slot_packs = p.L.oneshot_max / 16;
  auto slot = [&](int owner_rank, int src_rank) -> uint4* {
    return reinterpret_cast<uint4*>(me.wsp[owner_rank] + p.L.oneshot_off) +
           (static_cast<int64_t>(parity) * WS + src_rank) * slot_packs;
  };
  uint4* dst = reinterpret_cast<uint4*>(me.out);
  // 1. my input -> slot [rank] of every peer, and -> my own output segment
  for (int64_t i0 = beg + threadIdx.x; i0 < end; i0 += static_cast<int64_t>(blockDim.x) * U) {
    uint4 x[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t i = i0 + static_cast<int64_t>(u) * blockDim.x;
      if (i < end) x[u] = ld_plain(src + i);
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t i = i0 + static_cast<int64_t>(u) * blockDim.x;
      if (i < end && NAB_DBG_IDX(i, slot_packs)) {
#pragma unroll
        for (int k = 1; k < WS; ++k) st_plain(slot((rank + k) % WS, rank) + i, x[u]);
        st_plain(dst + rank * stride + i, x[u]);
      }
    }
  }
  int peers[WS - 1];
  all_peers<WS>(rank, peers);
  const bool ok = exchange(me, kFlagGather, blockIdx.x, make_seq(epoch, 0), peers, WS - 1, w,
                           kStageAllGather);
  // 2. the peers' segments from my slots into the output
  if (ok) {
    for (int64_t i0 = beg + threadIdx.x; i0 < end; i0 += static_cast<int64_t>(blockDim.x) * UR) {
      uint4 x[UR][WS - 1];
#pragma unroll
      for (int u = 0; u < UR; ++u) {
        const int64_t i = i0 + static_cast<int64_t>(u) * blockDim.x;
        if (i < end) {
#pragma unroll
          for (int k = 1; k < WS; ++k) x[u][k - 1] = ld_cg(slot(rank, (rank + k) % WS) + i);
        }
      }
#pragma unroll
      for (int u = 0; u < UR; ++u) {
        const int64_t i = i0 + static_cast<int64_t>(u) * blockDim.x;
        if (i < end) {
#pragma unroll
          for (int k = 1; k < WS; ++k) st_plain(dst + ((rank + k) % WS) * stride + i, x[u][k - 1]);
        }
      }
    }
  }
  end_call(me, epoch);
}

// ---------------------------------------------------------- NVLS oneshot ----
template <typename T, int WS>
__global__ void __launch_bounds__(kThreads, 2) k_nvls_oneshot(const __grid_constant__ ARParams p) {
  constexpr int U = 4;
  const RankView& me = p.v[blockIdx.y];
  if (!launch_ok(p, me, WS, me.mc != nullptr && blockIdx.x < kMaxBlocks && p.npacks * 16 <= p.L.oneshot_max &&
                                p.L.mc_oneshot_off + 2 * p.L.oneshot_max <= p.L.mc_bytes))
    return;
  const uint32_t epoch = begin_call(me);
  const WaitCtx w = make_wait(p, me, epoch);
  const int b = blockIdx.x;
  const int parity = epoch & 1;
  const int64_t per = ceil_div<int64_t>(p.npacks, gridDim.x);
  const int64_t beg = per * b;
  const int64_t end = min(p.npacks, beg + per);
  const uint4* src = reinterpret_cast<const uint4*>(me.in);
  uint4* dst = reinterpret_cast<uint4*>(me.out);
  const int64_t off = p.L.mc_oneshot_off + parity * p.L.oneshot_max;
  uint4* uc = reinterpret_cast<uint4*>(me.uc + off);
  const uint4* mc = reinterpret_cast<const uint4*>(me.mc + off);
  NvlsPad* upad = reinterpret_cast<NvlsPad*>(me.uc);
  NvlsPad* mpad = reinterpret_cast<NvlsPad*>(me.mc);
  const int64_t stride = blockDim.x;
  for (int64_t i0 = beg + threadIdx.x; i0 < end; i0 += stride * U) {
    uint4 x[U];
#pragma unroll
    for (int u = 0; u < U; ++u)
      if (i0 + u * stride < end) x[u] = ld_plain(src + i0 + u * stride);
#pragma unroll
    for (int u = 0; u < U; ++u)
      if (i0 + u * stride < end) st_plain(uc + i0 + u * stride, x[u]);
  }
  fence_proxy_alias();  // unicast stores before the multicast arrival
  __syncthreads();
  __shared__ int s_ok;
  if (threadIdx.x == 0) {
    const uint32_t calls = upad->rounds[b][1] + 1u;
    mm_red_add_release(&mpad->cnt[b][2][0], 1u);
    s_ok = wait_geq_u32(&upad->cnt[b][2][0], calls * WS, w, kStageNvls1);
    upad->rounds[b][1] = calls;
  }
  __syncthreads();
  fence_proxy_alias();  // unicast acquire before multicast loads
  if (s_ok) {
    for (int64_t i0 = beg + threadIdx.x; i0 < end; i0 += stride * U) {
      uint4 y[U];
#pragma unroll
      for (int u = 0; u < U; ++u)
        if (i0 + u * stride < end) y[u] = mm_ld_reduce<T>(mc + i0 + u * stride);
#pragma unroll
      for (int u = 0; u < U; ++u)
        if (i0 + u * stride < end) st_plain(dst + i0 + u * stride, y[u]);
    }
  }
  end_call(me, epoch);
}

// ---------------------------------------------------------- NVLS twoshot ----
// Pipelined and warp-specialised. Tiles of WS chunks (chunk j owned by rank j)
// flow through a ring of kNvlsSlots slots in the CTA's part of the multicast
// workspace:
//   producer warps  copy tile k of the input into slot k % S (unicast address)
//                   and arrive on the slot's phase-0 counter of every GPU;
//   reducer warps   wait until every GPU copied tile k in, multimem.ld_reduce
//                   their own chunk, multimem.st the result into the slot of
//                   every GPU (and into their own output), arrive on phase 1;
//   consumer warps  wait until every owner broadcast, copy the other chunks
//                   out and hand the slot back to the producers.
// Up to S tiles are in flight, so the local copies, the switch traffic and
// the cross-GPU arrivals overlap. Counters are monotonic per slot: the n-th
// use of a slot waits for WS * n arrivals. Every wait is bounded; a wait that
// gives up sets a CTA-wide abort flag that every group checks.
constexpr int kProdWarps = 4, kRedWarps = 8, kConsWarps = 4;
static_assert((kProdWarps + kRedWarps + kConsWarps) * 32 == kThreads, "warp groups must fill the CTA");

// One thread spins on a local counter (arrivals from every GPU) with a
// deadline; also gives up when the CTA-wide abort flag is set.
NAB_DINLINE bool pipe_wait(const uint32_t* ctr, uint32_t target, const WaitCtx& w, volatile int* s_abort,
                           uint32_t stage) {
  uint32_t v = ld_acquire_sys_u32(ctr);
  if (static_cast<int32_t>(v - target) >= 0) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t it = 1;; ++it) {
    v = ld_acquire_sys_u32(ctr);
    if (static_cast<int32_t>(v - target) >= 0) return true;
    if ((it & 127u) == 0u) {
      if (*s_abort || ld_volatile_u32(w.abort) != 0u) return false;
      if (globaltimer_ns() - t0 > w.timeout_ns) {
        record_failure(w, kErrTimeout, 0xffffffffu, stage, v);
        return false;
      }
    }
  }
}

// Body of the pipelined NVLS two-shot for CTA c of C on packs [0, npacks)
// of src/dst (a hybrid launch passes the message's suffix).
template <typename T, int WS>
__device__ __forceinline__ void nvls_twoshot_body(const ARParams& p, const RankView& me, uint32_t epoch,
                                                  const WaitCtx& w, int c, int C, const uint4* src, uint4* dst,
                                                  int64_t npacks, int chp) {
  constexpr int S = kNvlsSlots;
  constexpr int U = 8;
  constexpr int UL = 8;  // multimem.ld_reduce requests in flight per reducer thread
  const int rank = me.rank;
  const int64_t tile = static_cast<int64_t>(WS) * chp;
  const int64_t ntiles = (npacks + tile - 1) / tile;
  const int64_t my_tiles = ntiles > c ? (ntiles - c + C - 1) / C : 0;
  const int64_t cstride = p.L.nvls_chunk / 16;  // packs between chunks of a slot
  const int64_t slot_packs = WS * cstride;
  const int64_t cta_off = p.L.mc_twoshot_off + static_cast<int64_t>(c) * S * WS * p.L.nvls_chunk;
  uint4* ucb = reinterpret_cast<uint4*>(me.uc + cta_off);
  uint4* mcb = reinterpret_cast<uint4*>(me.mc + cta_off);
  NvlsPad* upad = reinterpret_cast<NvlsPad*>(me.uc);
  NvlsPad* mpad = reinterpret_cast<NvlsPad*>(me.mc);

  __shared__ uint32_t s_base;
  __shared__ int s_abort;
  __shared__ int64_t s_done;  // tiles the consumers have finished (in order)
  if (threadIdx.x == 0) {
    s_base = upad->pipe_tiles[c];
    s_abort = 0;
    s_done = 0;
  }
  __syncthreads();
  const uint32_t base = s_base;
  volatile int* abort_flag = &s_abort;
  volatile int64_t* done = &s_done;
  const int warp = threadIdx.x >> 5;

  if (warp < kProdWarps) {
    // ------------------------------------------------------------ producers
    const int t = threadIdx.x, nt = kProdWarps * 32;
    for (int64_t k = 0; k < my_tiles; ++k) {
      const uint32_t g = base + static_cast<uint32_t>(k);
      const int slot = g % S;
      if (t == 0 && k >= S) {  // the slot's previous tile must be consumed here
        const uint64_t t0 = globaltimer_ns();
        while (*done < k - S + 1 && !*abort_flag) {
          if (globaltimer_ns() - t0 > w.timeout_ns) {
            record_failure(w, kErrTimeout, 0xffffffffu, kStageNvls1, static_cast<uint32_t>(*done));
            *abort_flag = 1;
          }
        }
      }
      if (named_barrier_or(1, nt, *abort_flag != 0)) break;
      const int64_t tb = (c + k * C) * tile;
      const int tlen = static_cast<int>(span_len(tile, npacks - tb));
      uint4* us = ucb + slot * slot_packs;
      for (int i0 = t; i0 < tlen; i0 += nt * U) {
        uint4 x[U];
#pragma unroll
        for (int u = 0; u < U; ++u)
          if (i0 + u * nt < tlen) x[u] = ld_plain(src + tb + i0 + u * nt);
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int i = i0 + u * nt;
          if (i < tlen) st_plain(us + (i / chp) * cstride + (i % chp), x[u]);
        }
      }
      fence_proxy_alias();  // unicast stores before the multicast arrival
      named_barrier(1, nt);
      if (t == 0) mm_red_add_release(&mpad->pipe[c][slot][0][0], 1u);
    }
  } else if (warp < kProdWarps + kRedWarps) {
    // ------------------------------------------------------------- reducers
    const int t = threadIdx.x - kProdWarps * 32, nt = kRedWarps * 32;
    for (int64_t k = 0; k < my_tiles; ++k) {
      const uint32_t g = base + static_cast<uint32_t>(k);
      const int slot = g % S;
      const uint32_t target = WS * (g / S + 1u);
      if (t == 0 && !pipe_wait(&upad->pipe[c][slot][0][0], target, w, abort_flag, kStageNvls1)) *abort_flag = 1;
      if (named_barrier_or(2, nt, *abort_flag != 0)) break;
      fence_proxy_alias();  // unicast acquire before multicast loads
      const int64_t mb = (c + k * C) * tile + static_cast<int64_t>(rank) * chp;
      const int mlen = static_cast<int>(span_len(chp, npacks - mb));
      uint4* mchunk = mcb + slot * slot_packs + rank * cstride;
      for (int i0 = t; i0 < mlen; i0 += nt * UL) {
        uint4 y[UL];
#pragma unroll
        for (int u = 0; u < UL; ++u)
          if (i0 + u * nt < mlen) y[u] = mm_ld_reduce<T>(mchunk + i0 + u * nt);
#pragma unroll
        for (int u = 0; u < UL; ++u) {
          const int i = i0 + u * nt;
          if (i < mlen) {
            mm_st<T>(mchunk + i, y[u]);
            st_plain(dst + mb + i, y[u]);
          }
        }
      }
      fence_proxy_alias();
      named_barrier(2, nt);
      if (t == 0) mm_red_add_release(&mpad->pipe[c][slot][1][0], 1u);
    }
  } else {
    // ------------------------------------------------------------ consumers
    const int t = threadIdx.x - (kProdWarps + kRedWarps) * 32, nt = kConsWarps * 32;
    for (int64_t k = 0; k < my_tiles; ++k) {
      const uint32_t g = base + static_cast<uint32_t>(k);
      const int slot = g % S;
      const uint32_t target = WS * (g / S + 1u);
      if (t == 0 && !pipe_wait(&upad->pipe[c][slot][1][0], target, w, abort_flag, kStageNvls2)) *abort_flag = 1;
      if (named_barrier_or(3, nt, *abort_flag != 0)) break;
      fence_proxy_alias();  // the owners' multicast stores before unicast loads
      const int64_t tb = (c + k * C) * tile;
      const int tlen = static_cast<int>(span_len(tile, npacks - tb));
      const uint4* us = ucb + slot * slot_packs;
      for (int i0 = t; i0 < tlen; i0 += nt * U) {
        uint4 x[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int i = i0 + u * nt;
          if (i < tlen && i / chp != rank) x[u] = ld_cg(us + (i / chp) * cstride + (i % chp));
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int i = i0 + u * nt;
          if (i < tlen && i / chp != rank) st_plain(dst + tb + i, x[u]);
        }
      }
      named_barrier(3, nt);
      if (t == 0) {
        __threadfence_block();
        *done = k + 1;
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) upad->pipe_tiles[c] = base + static_cast<uint32_t>(my_tiles);
}

template <typename T, int WS>
__global__ void __launch_bounds__(kThreads, 1) k_nvls_twoshot(const __grid_constant__ ARParams p) {
  const RankView& me = p.v[blockIdx.y];
  if (!launch_ok(p, me, WS, nvls_region_ok<WS>(p, me, blockIdx.x, p.chunk_packs))) return;
  const uint32_t epoch = begin_call(me);
  const WaitCtx w = make_wait(p, me, epoch);
  nvls_twoshot_body<T, WS>(p, me, epoch, w, blockIdx.x, gridDim.x, reinterpret_cast<const uint4*>(me.in),
                           reinterpret_cast<uint4*>(me.out), p.npacks, p.chunk_packs);
  end_call(me, epoch);
}

// ---------------------------------------------------------------- hybrid ----
// One launch, two protocols on disjoint parts of the message: CTAs
// [0, hyb_ctas) run the P2P pipelined two-shot on packs [0, split_packs)
// (link-bound: 1.75 S per direction of each GPU's NVLink at 8 ranks), the
// rest run the NVLS two-shot on the remainder (about 1.125 S per direction,
// bound by the switch's reduction rate). Their rings, flags and counters are
// disjoint, so they share only the call's epoch.
template <typename T, int WS>
__global__ void __launch_bounds__(kThreads, 1) k_hybrid(const __grid_constant__ ARParams p) {
  const RankView& me = p.v[blockIdx.y];
  const int cb = static_cast<int>(blockIdx.x);
  if (!launch_ok(p, me, WS,
                 p.split_packs > 0 && p.split_packs < p.npacks &&
                     (cb < p.hyb_ctas ? pipe_region_ok<WS>(p, cb, p.chunk_packs)
                                      : nvls_region_ok<WS>(p, me, cb - p.hyb_ctas, p.chunk_packs2))))
    return;
  const uint32_t epoch = begin_call(me);
  const WaitCtx w = make_wait(p, me, epoch);
  const uint4* src = reinterpret_cast<const uint4*>(me.in);
  uint4* dst = reinterpret_cast<uint4*>(me.out);
  const int c = blockIdx.x;
  if (c < p.hyb_ctas)
    twoshot_pipe_body<T, WS>(p, me, epoch, w, c, p.hyb_ctas, src, dst, p.split_packs, p.chunk_packs);
  else
    nvls_twoshot_body<T, WS>(p, me, epoch, w, c - p.hyb_ctas, gridDim.x - p.hyb_ctas, src + p.split_packs,
                             dst + p.split_packs, p.npacks - p.split_packs, p.chunk_packs2);
  end_call(me, epoch);
}

template <typename T, int WS>
cudaError_t launch_ws(int algo, const ARParams& p, dim3 grid, cudaStream_t s, bool coop) {
  void* fn = nullptr;
  switch (algo) {
    case kAlgoOneshot: fn = reinterpret_cast<void*>(&k_oneshot<T, WS>); break;
    case kAlgoTwoshot: fn = reinterpret_cast<void*>(&k_twoshot<T, WS>); break;
    case kAlgoTwoshotPipe: fn = reinterpret_cast<void*>(&k_twoshot_pipe<T, WS>); break;
    case kAlgoHier: fn = reinterpret_cast<void*>(&k_hier<T>); break;
    case kAlgoOneshotPull: fn = reinterpret_cast<void*>(&k_oneshot_pull<T, WS>); break;
    case kAlgoNvlsOneshot: fn = reinterpret_cast<void*>(&k_nvls_oneshot<T, WS>); break;
    case kAlgoNvlsTwoshot: fn = reinterpret_cast<void*>(&k_nvls_twoshot<T, WS>); break;
    case kAlgoHybrid: fn = reinterpret_cast<void*>(&k_hybrid<T, WS>); break;
    case kAlgoReduceScatter: fn = reinterpret_cast<void*>(&k_reduce_scatter<T, WS>); break;
    case kAlgoAllGather: fn = reinterpret_cast<void*>(&k_all_gather<WS>); break;
    default: return cudaErrorInvalidValue;
  }
  void* args[] = {const_cast<ARParams*>(&p)};
  if (coop) return cudaLaunchCooperativeKernel(fn, grid, dim3(kThreads), args, 0, s);
  return cudaLaunchKernel(fn, grid, dim3(kThreads), args, 0, s);
}

template <typename T>
cudaError_t launch_t(int algo, const ARParams& p, dim3 grid, cudaStream_t s, bool coop) {
  switch (p.ws) {
    case 2: return launch_ws<T, 2>(algo, p, grid, s, coop);
    case 3: return launch_ws<T, 3>(algo, p, grid, s, coop);
    case 4: return launch_ws<T, 4>(algo, p, grid, s, coop);
    case 5: return launch_ws<T, 5>(algo, p, grid, s, coop);
    case 6: return launch_ws<T, 6>(algo, p, grid, s, coop);
    case 7: return launch_ws<T, 7>(algo, p, grid, s, coop);
    case 8: return launch_ws<T, 8>(algo, p, grid, s, coop);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace

int allreduce_threads() { return kThreads; }

cudaError_t launch_allreduce(int algo, int dtype, const ARParams& p, dim3 grid, cudaStream_t s,
                             bool cooperative) {
  if (algo == kAlgoCopy) {
    void* args[] = {const_cast<ARParams*>(&p)};
    void* fn = reinterpret_cast<void*>(&k_copy);
    if (cooperative) return cudaLaunchCooperativeKernel(fn, grid, dim3(kThreads), args, 0, s);
    return cudaLaunchKernel(fn, grid, dim3(kThreads), args, 0, s);
  }
  switch (dtype) {
    case kF32: return launch_t<float>(algo, p, grid, s, cooperative);
    case kF16: return launch_t<__half>(algo, p, grid, s, cooperative);
    case kBF16: return launch_t<__nv_bfloat16>(algo, p, grid, s, cooperative);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace nab
