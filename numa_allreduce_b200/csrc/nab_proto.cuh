// Protocol helpers shared by every cross-GPU kernel: the per-call epoch, the
// release/acquire flag exchange between a CTA and the same CTA index on its
// peers, and the bounded-wait context.
#pragma once

#include "nab_device.cuh"

namespace nab {

NAB_DINLINE SignalPad* pad_at(char* const* wsp, int r) { return reinterpret_cast<SignalPad*>(wsp[r]); }

NAB_DINLINE uint64_t make_seq(uint32_t epoch, int round) {
  return (static_cast<uint64_t>(epoch) << kSeqShift) + static_cast<uint64_t>(round);
}

// Reads the per-call epoch (thread 0) and broadcasts it to the CTA.
NAB_DINLINE uint32_t begin_call(char* const* wsp, int rank) {
  __shared__ uint32_t s_epoch;
  if (threadIdx.x == 0) s_epoch = ld_volatile_u32(&pad_at(wsp, rank)->epoch) + 1u;
  __syncthreads();
  return s_epoch;
}

// The last CTA of this rank to finish publishes the epoch for the next call.
NAB_DINLINE void end_call(char* const* wsp, int rank, uint32_t epoch) {
  __syncthreads();
  if (threadIdx.x == 0) {
    SignalPad* my = pad_at(wsp, rank);
    __threadfence();
    const uint32_t prev = atomicAdd(&my->done_ctas, 1u);
    if (prev == gridDim.x - 1) {
      st_volatile_u32(&my->done_ctas, 0u);
      st_volatile_u32(&my->epoch, epoch);
    }
  }
}

NAB_DINLINE WaitCtx make_wait(ErrorState* err, uint32_t* err_host, uint64_t timeout_ns,
                              char* const* wsp, int rank, uint32_t epoch) {
  WaitCtx w;
  w.err = err;
  w.err_host = err_host;
  w.abort = &pad_at(wsp, rank)->abort;
  w.timeout_ns = timeout_ns;
  w.rank = static_cast<uint32_t>(rank);
  w.epoch = epoch;
  return w;
}

// Threads [0, npeers) each signal one peer (release) and then wait for that
// peer's signal (acquire). The leading bar.sync orders all of the CTA's
// earlier stores before the release; the trailing one orders every thread's
// later loads after the acquires. Returns false on every thread if any wait
// gave up.
NAB_DINLINE bool exchange(char* const* wsp, int rank, int kind, int slot, uint64_t seq,
                          const int* peers, int npeers, const WaitCtx& w, uint32_t stage) {
  __syncthreads();
  bool ok = true;
  const int t = threadIdx.x;
  if (t < npeers) {
    const int peer = peers[t];
    st_release_sys(&pad_at(wsp, peer)->flags[kind].v[slot][rank], seq);
    ok = wait_geq(&pad_at(wsp, rank)->flags[kind].v[slot][peer], seq, w, static_cast<uint32_t>(peer),
                  stage);
  }
  return __syncthreads_and(ok) != 0;
}

template <int WS>
NAB_DINLINE void all_peers(int rank, int* peers) {
#pragma unroll
  for (int k = 0; k < WS - 1; ++k) peers[k] = (rank + 1 + k) % WS;
}

NAB_DINLINE void all_peers_rt(int ws, int rank, int* peers) {
  for (int k = 0; k < ws - 1; ++k) peers[k] = (rank + 1 + k) % ws;
}

}  // namespace nab
