// Plain C ABI of the allreduce library, usable without Python or torch.
//
// Capability parity: the reference's extern "C" block
// (src/numa_all_reduce.cu:736-808: numa_all_reduce_init / _dispose /
// _register_buffer / _fp16 / _fp32 / _bf16). The same names and argument
// lists are kept so a caller of the reference's C ABI links unchanged; the
// functions return 0 on success and a non-zero status on failure (the
// reference returned void and exited the process on CUDA errors), with the
// message available from nab_last_error. `signals` are the per-rank
// workspaces (nab_workspace_bytes(world_size) bytes each, zero-initialised,
// IPC-mapped), and `nnuma` splits the ranks into that many contiguous groups
// for the hierarchical protocol, as the reference's build_numa_mappings did.
// C declarations: nab_capi.h.
#include <cuda_runtime.h>

#include <cstring>
#include <exception>
#include <stdexcept>
#include <string>
#include <vector>

#include "nab_capi.h"
#include "nab_comm.h"

#define NAB_API extern "C" __attribute__((visibility("default")))

namespace {

thread_local std::string g_last_error;

template <typename F>
int guarded(F&& f) {
  try {
    f();
    return 0;
  } catch (const std::exception& e) {
    g_last_error = e.what();
  } catch (...) {
    g_last_error = "unknown error";
  }
  return 1;
}

nab::Communicator* C(void* p) { return static_cast<nab::Communicator*>(p); }

int do_allreduce(void* ptr, cudaStream_t stream, const void* in, void* out, int64_t numel, int dtype,
                 int algo) {
  return guarded([&] {
    if (!ptr) throw std::invalid_argument("null communicator");
    const int64_t esize = dtype == nab::kF32 ? 4 : 2;
    C(ptr)->allreduce(stream, in, out, numel * esize, dtype, algo, false);
  });
}

}  // namespace

NAB_API int nab_last_error(char* buf, int len) {
  if (!buf || len <= 0) return static_cast<int>(g_last_error.size());
  std::strncpy(buf, g_last_error.c_str(), static_cast<size_t>(len) - 1);
  buf[len - 1] = '\0';
  return static_cast<int>(g_last_error.size());
}

NAB_API int64_t nab_workspace_bytes(int world_size) {
  try {
    return nab::make_layout(world_size, nab::CommConfig{}).ws_bytes;
  } catch (const std::exception& e) {
    g_last_error = e.what();
    return -1;
  }
}

NAB_API void* numa_all_reduce_init(void** signals, void* rank_data, size_t rank_data_sz, int rank,
                                   int world_size, int nnuma) {
  nab::Communicator* c = nullptr;
  const int rc = guarded([&] {
    std::vector<char*> ws;
    for (int i = 0; i < world_size; ++i) ws.push_back(static_cast<char*>(signals[i]));
    c = new nab::Communicator(rank, world_size, ws, rank_data, rank_data_sz, nab::CommConfig{}, true);
    if (nnuma > 1) {
      if (world_size % nnuma != 0) throw std::invalid_argument("world size not divisible by nnuma");
      const int per = world_size / nnuma;
      std::vector<std::vector<int>> groups(nnuma);
      for (int r = 0; r < world_size; ++r) groups[r / per].push_back(r);
      c->set_groups(groups);
    }
  });
  if (rc != 0) {
    delete c;
    return nullptr;
  }
  return c;
}

NAB_API int numa_all_reduce_dispose(void* ptr) {
  return guarded([&] { delete C(ptr); });
}

NAB_API int numa_all_reduce_register_buffer(void* ptr, void** ptrs) {
  return guarded([&] {
    std::vector<void*> v(ptrs, ptrs + C(ptr)->world_size());
    C(ptr)->register_buffer(v);
  });
}

NAB_API int numa_all_reduce_fp16(void* ptr, cudaStream_t stream, void* input, void* output, int size) {
  return do_allreduce(ptr, stream, input, output, size, nab::kF16, nab::kAlgoAuto);
}

NAB_API int numa_all_reduce_fp32(void* ptr, cudaStream_t stream, void* input, void* output, int size) {
  return do_allreduce(ptr, stream, input, output, size, nab::kF32, nab::kAlgoAuto);
}

NAB_API int numa_all_reduce_bf16(void* ptr, cudaStream_t stream, void* input, void* output, int size) {
  return do_allreduce(ptr, stream, input, output, size, nab::kBF16, nab::kAlgoAuto);
}

// Explicit protocol choice (nab::Algo values) and 64-bit element counts.
NAB_API int nab_allreduce(void* ptr, cudaStream_t stream, const void* input, void* output, int64_t numel,
                          int dtype, int algo) {
  return do_allreduce(ptr, stream, input, output, numel, dtype, algo);
}

// Contiguous-segment collectives; seg_numel elements per rank segment.
// Reduce-scatter: input holds world_size segments, output one (the sum of
// every rank's segment [rank]). All-gather: input one segment, output
// world_size (rank order).
NAB_API int nab_reduce_scatter(void* ptr, cudaStream_t stream, const void* input, void* output, int64_t seg_numel,
                               int dtype) {
  return guarded([&] {
    if (!ptr) throw std::invalid_argument("null communicator");
    C(ptr)->reduce_scatter(stream, input, output, seg_numel * (dtype == nab::kF32 ? 4 : 2), dtype);
  });
}

NAB_API int nab_all_gather(void* ptr, cudaStream_t stream, const void* input, void* output, int64_t seg_numel,
                           int dtype) {
  return guarded([&] {
    if (!ptr) throw std::invalid_argument("null communicator");
    C(ptr)->all_gather(stream, input, output, seg_numel * (dtype == nab::kF32 ? 4 : 2), dtype);
  });
}

// Replaces the automatic choice's steps for one dtype (0 fp32, 1 fp16, 2
// bf16): n ascending byte limits with their protocol ids, and the protocol of
// larger messages (100 = NCCL, which this ABI cannot call: such messages take
// the last custom protocol of the steps). The Python package hands the same
// steps to its communicators, from its tuning table or the built-in ones.
NAB_API int nab_set_auto_table(void* ptr, int dtype, int n, const int64_t* max_bytes, const int* algos,
                               int fallback) {
  return guarded([&] {
    if (!ptr) throw std::invalid_argument("null communicator");
    if (n < 0 || (n > 0 && (!max_bytes || !algos))) throw std::invalid_argument("bad step arrays");
    nab::AutoTable t;
    for (int i = 0; i < n; ++i) t.steps.push_back({max_bytes[i], algos[i]});
    t.fallback = fallback;
    C(ptr)->set_auto_table(dtype, t);
  });
}

// Hybrid protocol split: per mille of each message on the P2P part, and the
// CTAs of the P2P and NVLS parts.
NAB_API int nab_set_hybrid(void* ptr, int p2p_permille, int p2p_ctas, int nvls_ctas) {
  return guarded([&] {
    if (!ptr) throw std::invalid_argument("null communicator");
    C(ptr)->set_hybrid(p2p_permille, p2p_ctas, nvls_ctas);
  });
}

// The protocol the automatic choice launches for a message (negative on error).
NAB_API int nab_auto_protocol(void* ptr, int64_t nbytes, int dtype) {
  int algo = -1;
  guarded([&] {
    if (!ptr) throw std::invalid_argument("null communicator");
    algo = C(ptr)->plan(nbytes, nab::kAlgoAuto, false, dtype).algo;
  });
  return algo;
}

NAB_API uint32_t nab_error_code(void* ptr) { return ptr ? C(ptr)->error_code() : 0u; }

NAB_API int nab_reset(void* ptr) {
  return guarded([&] { C(ptr)->reset(); });
}
