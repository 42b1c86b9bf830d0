// Torch bindings: every entry point is a TORCH_LIBRARY op (torch.ops.nab.*),
// so the allreduce can be captured in CUDA graphs from Python.
//
// Capability parity: the reference's torch-facing wrappers
// (src/numa_all_reduce.cu:579-734: init_numa_ar, numa_ar_allreduce,
// numa_ar_dispose, numa_ar_register_buffer, numa_ar_meta_size,
// numa_ar_get_graph_buffer_ipc_meta, numa_ar_register_graph_buffers,
// numa_ar_allocate_shared_buffer_and_handle, numa_ar_open_mem_handle,
// numa_ar_free_shared_buffer), which the reference never registered with
// torch. Handles are int64 pointers as in the reference (fptr_t).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/library.h>
#include <torch/torch.h>

#include <stdexcept>
#include <string>
#include <tuple>
#include <vector>

#include "nab_comm.h"
#include "nab_fused.h"
#include "nab_gemm.h"
#include "nab_kerr.h"
#include "nab_llama.h"
#include "nab_nvls.h"

namespace {

using nab::Communicator;
using fptr_t = int64_t;
static_assert(sizeof(void*) == sizeof(fptr_t), "pointer size");

Communicator* C(fptr_t fa) {
  TORCH_CHECK(fa != 0, "allreduce communicator is closed");
  return reinterpret_cast<Communicator*>(fa);
}

int dtype_of(const at::Tensor& t) {
  switch (t.scalar_type()) {
    case at::kFloat: return nab::kF32;
    case at::kHalf: return nab::kF16;
    case at::kBFloat16: return nab::kBF16;
    default: TORCH_CHECK(false, "allreduce supports float32, float16 and bfloat16, got ", t.scalar_type());
  }
  return -1;
}

// Weakly contiguous: the tensor's bytes are exactly the tail of its storage
// (reference src/numa_all_reduce.cu:565-569).
bool weak_contiguous(const at::Tensor& t) {
  return t.is_contiguous() ||
         (t.storage().nbytes() - t.storage_offset() * t.element_size() == t.numel() * t.element_size());
}

std::vector<int64_t> layout(int64_t ws, const std::vector<int64_t>& cfg) {
  const nab::Layout L = nab::make_layout(static_cast<int>(ws), nab::config_from_list(cfg));
  return {L.ws_bytes, L.mc_bytes, L.oneshot_off, L.twoshot_off, L.hier_off, L.fused_off, L.pipe_off};
}

int64_t meta_size() { return static_cast<int64_t>(sizeof(nab::SignalPad)); }

fptr_t init(const std::vector<int64_t>& ws_ptrs, at::Tensor& rank_data, int64_t rank,
            bool full_nvlink, const std::vector<int64_t>& cfg) {
  TORCH_CHECK(rank_data.is_cuda(), "rank_data must be a CUDA tensor");
  const at::cuda::OptionalCUDAGuard guard(rank_data.device());
  std::vector<char*> ptrs;
  for (int64_t p : ws_ptrs) ptrs.push_back(reinterpret_cast<char*>(p));
  auto* c = new Communicator(static_cast<int>(rank), static_cast<int>(ws_ptrs.size()), ptrs,
                             rank_data.data_ptr(), rank_data.numel() * rank_data.element_size(),
                             nab::config_from_list(cfg), full_nvlink);
  return reinterpret_cast<fptr_t>(c);
}

void dispose(fptr_t fa) { delete reinterpret_cast<Communicator*>(fa); }

void set_groups(fptr_t fa, const std::vector<int64_t>& flat, int64_t ngroups) {
  TORCH_CHECK(ngroups > 0 && static_cast<int64_t>(flat.size()) % ngroups == 0, "bad groups");
  const int64_t gs = static_cast<int64_t>(flat.size()) / ngroups;
  std::vector<std::vector<int>> g(ngroups);
  for (int64_t i = 0; i < ngroups; ++i)
    for (int64_t j = 0; j < gs; ++j) g[i].push_back(static_cast<int>(flat[i * gs + j]));
  C(fa)->set_groups(g);
}

void attach_nvls(fptr_t fa, int64_t mc, int64_t uc, int64_t bytes) {
  C(fa)->attach_nvls(reinterpret_cast<char*>(mc), reinterpret_cast<char*>(uc), bytes);
}

void register_buffer(fptr_t fa, const std::vector<int64_t>& ptrs) {
  std::vector<void*> p;
  for (int64_t x : ptrs) p.push_back(reinterpret_cast<void*>(x));
  C(fa)->register_buffer(p);
}

void check_io(const at::Tensor& inp, const at::Tensor& out) {
  TORCH_CHECK(inp.is_cuda() && out.is_cuda(), "allreduce tensors must be on a CUDA device");
  TORCH_CHECK(inp.scalar_type() == out.scalar_type(), "input and output dtypes differ");
  TORCH_CHECK(inp.numel() == out.numel(), "input and output sizes differ");
  TORCH_CHECK(weak_contiguous(inp) && weak_contiguous(out), "allreduce tensors must be weakly contiguous");
}

// Reference-compatible entry point (src/numa_all_reduce.cu:604-653): a
// non-zero reg_buffer means "input is not registered". No staging copy is
// made: the push protocols read the local input directly.
void all_reduce(fptr_t fa, const at::Tensor& inp, at::Tensor& out, fptr_t reg_buffer,
                int64_t reg_buffer_sz_bytes) {
  check_io(inp, out);
  const int64_t bytes = inp.numel() * inp.element_size();
  if (reg_buffer) TORCH_CHECK(bytes <= reg_buffer_sz_bytes, "input larger than the registered buffer");
  const at::cuda::OptionalCUDAGuard guard(inp.device());
  auto stream = at::cuda::getCurrentCUDAStream().stream();
  C(fa)->allreduce(stream, inp.data_ptr(), out.data_ptr(), bytes, dtype_of(inp), nab::kAlgoAuto,
                   reg_buffer == 0);
}

void all_reduce_algo(fptr_t fa, const at::Tensor& inp, at::Tensor& out, int64_t algo,
                     bool registered) {
  check_io(inp, out);
  const at::cuda::OptionalCUDAGuard guard(inp.device());
  auto stream = at::cuda::getCurrentCUDAStream().stream();
  C(fa)->allreduce(stream, inp.data_ptr(), out.data_ptr(), inp.numel() * inp.element_size(),
                   dtype_of(inp), static_cast<int>(algo), registered);
}

// Reduce-scatter / all-gather: `big` holds ws segments of `small`'s size.
void check_collective_io(const at::Tensor& small, const at::Tensor& big, int ws) {
  TORCH_CHECK(small.is_cuda() && big.is_cuda(), "collective tensors must be on a CUDA device");
  TORCH_CHECK(small.scalar_type() == big.scalar_type(), "input and output dtypes differ");
  TORCH_CHECK(big.numel() == small.numel() * ws, "the segmented tensor must hold world_size segments");
  TORCH_CHECK(small.is_contiguous() && big.is_contiguous(), "collective tensors must be contiguous");
}

void reduce_scatter(fptr_t fa, const at::Tensor& inp, at::Tensor& out) {
  check_collective_io(out, inp, C(fa)->world_size());
  const at::cuda::OptionalCUDAGuard guard(inp.device());
  auto stream = at::cuda::getCurrentCUDAStream().stream();
  C(fa)->reduce_scatter(stream, inp.data_ptr(), out.data_ptr(), out.numel() * out.element_size(), dtype_of(inp));
}

void all_gather(fptr_t fa, const at::Tensor& inp, at::Tensor& out) {
  check_collective_io(inp, out, C(fa)->world_size());
  const at::cuda::OptionalCUDAGuard guard(inp.device());
  auto stream = at::cuda::getCurrentCUDAStream().stream();
  C(fa)->all_gather(stream, inp.data_ptr(), out.data_ptr(), inp.numel() * inp.element_size(), dtype_of(inp));
}

// kind: 0 reduce-scatter (ins segmented, outs one segment), 1 all-gather.
int64_t emulate_collective(const std::vector<int64_t>& fas, const std::vector<at::Tensor>& ins,
                           const std::vector<at::Tensor>& outs, int64_t kind, int64_t participants) {
  TORCH_CHECK(fas.size() == ins.size() && ins.size() == outs.size(), "one tensor pair per rank");
  TORCH_CHECK(kind == 0 || kind == 1, "kind is 0 (reduce-scatter) or 1 (all-gather)");
  const int ws = static_cast<int>(fas.size());
  std::vector<Communicator*> cs;
  std::vector<const void*> in_ptrs;
  std::vector<void*> out_ptrs;
  for (size_t i = 0; i < fas.size(); ++i) {
    if (kind == 0)
      check_collective_io(outs[i], ins[i], ws);
    else
      check_collective_io(ins[i], outs[i], ws);
    TORCH_CHECK(ins[i].numel() == ins[0].numel() && ins[i].scalar_type() == ins[0].scalar_type(),
                "all ranks must use the same shape and dtype");
    cs.push_back(C(fas[i]));
    in_ptrs.push_back(ins[i].data_ptr());
    out_ptrs.push_back(outs[i].data_ptr());
  }
  const at::Tensor& seg = kind == 0 ? outs[0] : ins[0];
  const at::cuda::OptionalCUDAGuard guard(ins[0].device());
  auto stream = at::cuda::getCurrentCUDAStream().stream();
  return nab::emulate_collective(cs, stream, in_ptrs, out_ptrs, seg.numel() * seg.element_size(), dtype_of(seg),
                                 kind == 0 ? nab::kAlgoReduceScatter : nab::kAlgoAllGather,
                                 static_cast<int>(participants));
}

int64_t plan_algo(fptr_t fa, int64_t nbytes, int64_t algo, bool registered, int64_t dtype) {
  if (C(fa)->world_size() == 1) return nab::kAlgoCopy;
  return C(fa)->plan(nbytes, static_cast<int>(algo), registered, static_cast<int>(dtype)).algo;
}

std::vector<int64_t> plan(fptr_t fa, int64_t nbytes, int64_t algo, bool registered, int64_t dtype) {
  const nab::LaunchPlan p = C(fa)->plan(nbytes, static_cast<int>(algo), registered, static_cast<int>(dtype));
  return {p.algo, p.grid.x, p.chunk_packs, p.rounds, p.hyb_ctas, p.chunk_packs2, p.split_packs};
}

nab::AutoTable make_table(const std::vector<int64_t>& limits, const std::vector<int64_t>& algos, int64_t fallback) {
  TORCH_CHECK(limits.size() == algos.size(), "one protocol per step");
  nab::AutoTable t;
  for (size_t i = 0; i < limits.size(); ++i) t.steps.push_back({limits[i], static_cast<int>(algos[i])});
  t.fallback = static_cast<int>(fallback);
  return t;
}

void set_auto_table(fptr_t fa, int64_t dtype, const std::vector<int64_t>& limits, const std::vector<int64_t>& algos,
                    int64_t fallback) {
  C(fa)->set_auto_table(static_cast<int>(dtype), make_table(limits, algos, fallback));
}

std::tuple<std::vector<int64_t>, std::vector<int64_t>, int64_t> table_lists(const nab::AutoTable& t) {
  std::vector<int64_t> limits, algos;
  for (const auto& st : t.steps) {
    limits.push_back(st.max_bytes);
    algos.push_back(st.algo);
  }
  return {limits, algos, t.fallback};
}

std::tuple<std::vector<int64_t>, std::vector<int64_t>, int64_t> get_auto_table(fptr_t fa, int64_t dtype) {
  return table_lists(C(fa)->auto_table(static_cast<int>(dtype)));
}

std::tuple<std::vector<int64_t>, std::vector<int64_t>, int64_t> builtin_auto_table(int64_t ws, bool has_nvls) {
  return table_lists(nab::builtin_auto_table(static_cast<int>(ws), has_nvls));
}

int64_t choose_auto(int64_t ws, int64_t nbytes, bool has_nvls, bool has_groups, const std::vector<int64_t>& limits,
                    const std::vector<int64_t>& algos, int64_t fallback) {
  return nab::choose_auto(make_table(limits, algos, fallback), static_cast<int>(ws), nbytes, has_nvls, has_groups);
}

// Error record of the kernels without a communicator (GEMM, attention) on the
// current device: [code, rank, peer, stage, block, epoch, observed, count].
std::vector<int64_t> kernel_error_state() {
  const nab::ErrorState st = nab::kernel_error_state();
  return {st.code, st.rank, st.peer, st.stage, st.block, st.epoch, st.observed, st.count};
}

int64_t kernel_error_code() { return nab::kernel_error_code(); }

void kernel_error_reset() { nab::kernel_error_reset(); }

void set_hybrid(fptr_t fa, int64_t permille, int64_t p2p_ctas, int64_t nvls_ctas) {
  C(fa)->set_hybrid(static_cast<int>(permille), static_cast<int>(p2p_ctas), static_cast<int>(nvls_ctas));
}

void emulate_all_reduce(const std::vector<int64_t>& fas, const std::vector<at::Tensor>& ins,
                        const std::vector<at::Tensor>& outs, int64_t algo, int64_t participants) {
  TORCH_CHECK(fas.size() == ins.size() && ins.size() == outs.size(), "one tensor pair per rank");
  std::vector<Communicator*> cs;
  std::vector<const void*> in_ptrs;
  std::vector<void*> out_ptrs;
  for (size_t i = 0; i < fas.size(); ++i) {
    check_io(ins[i], outs[i]);
    TORCH_CHECK(ins[i].numel() == ins[0].numel() && ins[i].scalar_type() == ins[0].scalar_type(),
                "all ranks must reduce the same shape and dtype");
    cs.push_back(C(fas[i]));
    in_ptrs.push_back(ins[i].data_ptr());
    out_ptrs.push_back(outs[i].data_ptr());
  }
  const at::cuda::OptionalCUDAGuard guard(ins[0].device());
  auto stream = at::cuda::getCurrentCUDAStream().stream();
  nab::emulate_allreduce(cs, stream, in_ptrs, out_ptrs, ins[0].numel() * ins[0].element_size(),
                         dtype_of(ins[0]), static_cast<int>(algo), static_cast<int>(participants));
}

#if NAB_DEBUG_BOUNDS
void debug_emulate_bad_rank(const std::vector<int64_t>& fas, const std::vector<at::Tensor>& ins,
                            const std::vector<at::Tensor>& outs, int64_t algo) {
  TORCH_CHECK(fas.size() == ins.size() && ins.size() == outs.size(), "one tensor pair per rank");
  std::vector<Communicator*> cs;
  std::vector<const void*> in_ptrs;
  std::vector<void*> out_ptrs;
  for (size_t i = 0; i < fas.size(); ++i) {
    check_io(ins[i], outs[i]);
    cs.push_back(C(fas[i]));
    in_ptrs.push_back(ins[i].data_ptr());
    out_ptrs.push_back(outs[i].data_ptr());
  }
  const at::cuda::OptionalCUDAGuard guard(ins[0].device());
  auto stream = at::cuda::getCurrentCUDAStream().stream();
  nab::emulate_allreduce_bad_rank(cs, stream, in_ptrs, out_ptrs, ins[0].numel() * ins[0].element_size(),
                                  dtype_of(ins[0]), static_cast<int>(algo));
}
#endif

bool debug_bounds_build() { return NAB_DEBUG_BOUNDS != 0; }

std::tuple<std::vector<int64_t>, std::vector<int64_t>> get_graph_buffer_ipc_meta(fptr_t fa) {
  auto [handles, offsets] = C(fa)->graph_buffer_ipc_meta();
  std::vector<int64_t> bytes(handles.begin(), handles.end());
  return {bytes, offsets};
}

void register_graph_buffers(fptr_t fa, const std::vector<std::vector<int64_t>>& handles,
                            const std::vector<std::vector<int64_t>>& offsets) {
  std::vector<std::string> h;
  for (const auto& v : handles) {
    std::string s;
    for (int64_t b : v) s.push_back(static_cast<char>(b));
    h.push_back(std::move(s));
  }
  C(fa)->register_graph_buffers(h, offsets);
}

int64_t num_graph_buffers(fptr_t fa) { return static_cast<int64_t>(C(fa)->num_graph_buffers()); }

std::tuple<fptr_t, at::Tensor> allocate_shared_buffer_and_handle(int64_t size) {
  auto stream = at::cuda::getCurrentCUDAStream().stream();
  std::string h;
  void* p = nab::ipc_alloc_shared(static_cast<size_t>(size), stream, &h);
  auto handle = torch::empty({static_cast<int64_t>(h.size())}, torch::dtype(torch::kUInt8));
  std::memcpy(handle.data_ptr(), h.data(), h.size());
  return {reinterpret_cast<fptr_t>(p), handle};
}

fptr_t open_mem_handle(const at::Tensor& mem_handle) {
  TORCH_CHECK(mem_handle.device().is_cpu() && mem_handle.scalar_type() == at::kByte, "bad handle");
  std::string h(reinterpret_cast<const char*>(mem_handle.data_ptr()), mem_handle.numel());
  return reinterpret_cast<fptr_t>(nab::ipc_open(h));
}

void close_mem_handle(fptr_t p) { nab::ipc_close(reinterpret_cast<void*>(p)); }
void free_shared_buffer(fptr_t p) { nab::ipc_free(reinterpret_cast<void*>(p)); }

int64_t error_code(fptr_t fa) { return C(fa)->error_code(); }
std::vector<int64_t> error_state(fptr_t fa) {
  const nab::ErrorState s = C(fa)->error_state();
  return {s.code, s.rank, s.peer, s.stage, s.block, s.epoch, s.observed, s.count};
}
void reset(fptr_t fa) { C(fa)->reset(); }
int64_t launches(fptr_t fa) { return C(fa)->launches(); }

// NVLS
bool nvls_supported(int64_t dev) { return nab::nvls_supported(static_cast<int>(dev)); }
int64_t nvls_new(int64_t dev, int64_t ws, int64_t bytes) {
  return reinterpret_cast<int64_t>(new nab::NvlsBuffer(static_cast<int>(dev), static_cast<int>(ws),
                                                       static_cast<size_t>(bytes)));
}
nab::NvlsBuffer* N(int64_t h) {
  TORCH_CHECK(h != 0, "NVLS buffer is closed");
  return reinterpret_cast<nab::NvlsBuffer*>(h);
}
int64_t nvls_bytes(int64_t h) { return static_cast<int64_t>(N(h)->bytes()); }
int64_t nvls_create(int64_t h) { return N(h)->create(); }
void nvls_import(int64_t h, int64_t fd) { N(h)->import_fd(static_cast<int>(fd)); }
void nvls_add_device(int64_t h) { N(h)->add_device(); }
void nvls_bind(int64_t h) { N(h)->bind_and_map(); }
std::vector<int64_t> nvls_ptrs(int64_t h) {
  return {static_cast<int64_t>(N(h)->mc_ptr()), static_cast<int64_t>(N(h)->uc_ptr())};
}
void nvls_release(int64_t h) { N(h)->release(); }
void nvls_free(int64_t h) { delete reinterpret_cast<nab::NvlsBuffer*>(h); }

int64_t sock_listen(const std::string& name) { return nab::sock_listen(name); }
void sock_send_fd(const std::string& name, int64_t fd, int64_t timeout_ms) {
  nab::sock_send_fd(name, static_cast<int>(fd), static_cast<int>(timeout_ms));
}
int64_t sock_recv_fd(int64_t lfd, int64_t timeout_ms) {
  return nab::sock_recv_fd(static_cast<int>(lfd), static_cast<int>(timeout_ms));
}
void sock_close(int64_t fd) { nab::sock_close(static_cast<int>(fd)); }

// Fused allreduce + residual add + RMSNorm.
void fused_ar_rmsnorm(fptr_t fa, const at::Tensor& inp, at::Tensor& residual, const at::Tensor& weight,
                      at::Tensor& out, double eps, int64_t algo) {
  TORCH_CHECK(inp.is_cuda() && inp.is_contiguous() && residual.is_contiguous() && out.is_contiguous() &&
                  weight.is_contiguous(),
              "fused allreduce+rmsnorm needs contiguous CUDA tensors");
  TORCH_CHECK(inp.dim() == 2 && residual.sizes() == inp.sizes() && out.sizes() == inp.sizes(),
              "fused allreduce+rmsnorm expects [tokens, hidden] tensors of one shape");
  TORCH_CHECK(weight.dim() == 1 && weight.size(0) == inp.size(1), "weight must be [hidden]");
  TORCH_CHECK(inp.scalar_type() == at::kBFloat16 && residual.scalar_type() == at::kBFloat16 &&
                  out.scalar_type() == at::kBFloat16 && weight.scalar_type() == at::kBFloat16,
              "fused allreduce+rmsnorm supports bfloat16");
  const at::cuda::OptionalCUDAGuard guard(inp.device());
  auto stream = at::cuda::getCurrentCUDAStream().stream();
  nab::fused_allreduce_rmsnorm(*C(fa), stream, inp.data_ptr(), residual.data_ptr(), weight.data_ptr(),
                               out.data_ptr(), inp.size(0), inp.size(1), static_cast<float>(eps),
                               static_cast<int>(algo));
}

void rmsnorm_residual(const at::Tensor& inp, at::Tensor& residual, const at::Tensor& weight,
                      at::Tensor& out, double eps) {
  TORCH_CHECK(inp.is_cuda() && inp.dim() == 2 && inp.is_contiguous() && residual.is_contiguous() &&
                  out.is_contiguous() && weight.is_contiguous(),
              "rmsnorm expects contiguous [tokens, hidden] CUDA tensors");
  TORCH_CHECK(inp.scalar_type() == at::kBFloat16, "rmsnorm supports bfloat16");
  const at::cuda::OptionalCUDAGuard guard(inp.device());
  auto stream = at::cuda::getCurrentCUDAStream().stream();
  nab::rmsnorm_residual(stream, inp.data_ptr(), residual.data_ptr(), weight.data_ptr(), out.data_ptr(),
                        inp.size(0), inp.size(1), static_cast<float>(eps));
}

void emulate_fused_ar_rmsnorm(const std::vector<int64_t>& fas, const std::vector<at::Tensor>& ins,
                              const std::vector<at::Tensor>& residuals, const std::vector<at::Tensor>& weights,
                              const std::vector<at::Tensor>& outs, double eps, int64_t algo) {
  const size_t n = fas.size();
  TORCH_CHECK(ins.size() == n && residuals.size() == n && weights.size() == n && outs.size() == n,
              "one tensor set per emulated rank");
  std::vector<nab::Communicator*> cs;
  std::vector<const void*> i, w;
  std::vector<void*> r, o;
  for (size_t k = 0; k < n; ++k) {
    TORCH_CHECK(ins[k].dim() == 2 && ins[k].sizes() == ins[0].sizes() && residuals[k].sizes() == ins[0].sizes() &&
                    outs[k].sizes() == ins[0].sizes() && ins[k].is_contiguous() && residuals[k].is_contiguous() &&
                    outs[k].is_contiguous() && weights[k].is_contiguous(),
                "fused emulation expects contiguous [tokens, hidden] tensors of one shape");
    TORCH_CHECK(ins[k].scalar_type() == at::kBFloat16 && residuals[k].scalar_type() == at::kBFloat16 &&
                    outs[k].scalar_type() == at::kBFloat16 && weights[k].scalar_type() == at::kBFloat16,
                "fused allreduce+rmsnorm supports bfloat16");
    cs.push_back(C(fas[k]));
    i.push_back(ins[k].data_ptr());
    r.push_back(residuals[k].data_ptr());
    w.push_back(weights[k].data_ptr());
    o.push_back(outs[k].data_ptr());
  }
  const at::cuda::OptionalCUDAGuard guard(ins[0].device());
  auto stream = at::cuda::getCurrentCUDAStream().stream();
  nab::emulate_fused_allreduce_rmsnorm(cs, stream, i, r, w, o, ins[0].size(0), ins[0].size(1),
                                       static_cast<float>(eps), static_cast<int>(algo));
}

void check_gemm_operand(const at::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda() && t.is_contiguous() && t.dim() == 2 && t.scalar_type() == at::kBFloat16, name,
              " must be a contiguous 2-D bfloat16 CUDA tensor");
}

// y[T, N] = x[T, K] . wt[N, K]^T on the tcgen05 tensor cores.
// wt: [N, K] row-major, or (packed) the tiled layout [N * K / 64, 64]; N is
// y's width (twice that with the SwiGLU epilogue).
void gemm(const at::Tensor& x, const at::Tensor& wt, at::Tensor& y, int64_t splits, bool packed, bool swiglu) {
  check_gemm_operand(x, "x");
  check_gemm_operand(wt, "wt");
  check_gemm_operand(y, "y");
  const int64_t N = y.size(1) * (swiglu ? 2 : 1), K = x.size(1);
  TORCH_CHECK(y.size(0) == x.size(0), "GEMM shape mismatch");
  if (packed) {
    TORCH_CHECK(wt.size(1) == 64 && wt.size(0) * 64 == N * K, "packed weight must be [N * K / 64, 64]");
  } else {
    TORCH_CHECK(wt.size(1) == K && wt.size(0) == N, "GEMM shape mismatch");
  }
  const at::cuda::OptionalCUDAGuard guard(x.device());
  auto stream = at::cuda::getCurrentCUDAStream().stream();
  nab::gemm_bf16(stream, wt.data_ptr(), x.data_ptr(), y.data_ptr(), static_cast<int>(x.size(0)), static_cast<int>(N),
                 static_cast<int>(K), static_cast<int>(splits), packed, swiglu);
}


int64_t gemm_active_clusters(int64_t bn, int64_t cs) {
  return nab::gemm_active_clusters(static_cast<int>(bn), static_cast<int>(cs));
}

int64_t gemm_splits(int64_t T, int64_t N, int64_t K) {
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return nab::gemm_splits_for(static_cast<int>(T), static_cast<int>(N), static_cast<int>(K), sms);
}

void gemm_ar_rmsnorm(fptr_t fa, const at::Tensor& x, const at::Tensor& wt, at::Tensor& residual,
                     const at::Tensor& weight, at::Tensor& out, double eps, int64_t splits, bool packed,
                     int64_t mode) {
  check_gemm_operand(x, "x");
  check_gemm_operand(wt, "wt");
  check_gemm_operand(residual, "residual");
  check_gemm_operand(out, "out");
  const int64_t N = residual.size(1), K = x.size(1);
  TORCH_CHECK(residual.size(0) == x.size(0) && out.sizes() == residual.sizes(), "GEMM+allreduce shape mismatch");
  if (packed) {
    TORCH_CHECK(wt.size(1) == 64 && wt.size(0) * 64 == N * K, "packed weight must be [N * K / 64, 64]");
  } else {
    TORCH_CHECK(wt.size(1) == K && wt.size(0) == N, "GEMM+allreduce shape mismatch");
  }
  TORCH_CHECK(weight.is_contiguous() && weight.numel() == N && weight.scalar_type() == at::kBFloat16,
              "norm weight must be [N] bfloat16");
  const at::cuda::OptionalCUDAGuard guard(x.device());
  auto stream = at::cuda::getCurrentCUDAStream().stream();
  nab::gemm_allreduce_rmsnorm(*C(fa), stream, wt.data_ptr(), x.data_ptr(), residual.data_ptr(), weight.data_ptr(),
                              out.data_ptr(), static_cast<int>(x.size(0)), static_cast<int>(N), static_cast<int>(K),
                              static_cast<float>(eps), static_cast<int>(splits), packed, static_cast<int>(mode));
}

int64_t gemm_ar_mode(int64_t T, int64_t ws) { return nab::gemm_ar_mode_for(static_cast<int>(T), static_cast<int>(ws)); }

void rope_append_op(const at::Tensor& qkv, const at::Tensor& cos_t, const at::Tensor& sin_t, const at::Tensor& pos,
                    at::Tensor& q_out, at::Tensor& k_cache, at::Tensor& v_cache, int64_t Hq, int64_t Hkv) {
  TORCH_CHECK(qkv.is_contiguous() && q_out.is_contiguous() && k_cache.is_contiguous() && v_cache.is_contiguous(),
              "rope_append: contiguous tensors");
  TORCH_CHECK(k_cache.dim() == 4 && k_cache.size(3) == 128 && pos.scalar_type() == at::kInt, "rope_append: shapes");
  TORCH_CHECK(cos_t.scalar_type() == at::kFloat && sin_t.scalar_type() == at::kFloat, "rope tables must be fp32");
  const at::cuda::OptionalCUDAGuard guard(qkv.device());
  nab::rope_append(at::cuda::getCurrentCUDAStream().stream(), qkv.data_ptr(), cos_t.data_ptr<float>(),
                   sin_t.data_ptr<float>(), pos.data_ptr<int>(), q_out.data_ptr(), k_cache.data_ptr(),
                   v_cache.data_ptr(), static_cast<int>(qkv.size(0)), static_cast<int>(Hq), static_cast<int>(Hkv),
                   static_cast<int>(k_cache.size(2)));
}

void decode_attention_op(const at::Tensor& q, const at::Tensor& k_cache, const at::Tensor& v_cache,
                         const at::Tensor& pos, at::Tensor& out, int64_t splits) {
  TORCH_CHECK(q.dim() == 3 && q.size(2) == 128 && k_cache.dim() == 4 && q.is_contiguous(), "decode_attention: shapes");
  const int64_t B = q.size(0), Hq = q.size(1), Hkv = k_cache.size(1);
  const at::cuda::OptionalCUDAGuard guard(q.device());
  nab::decode_attention(at::cuda::getCurrentCUDAStream().stream(), q.data_ptr(), k_cache.data_ptr(),
                        v_cache.data_ptr(), pos.data_ptr<int>(), out.data_ptr(), static_cast<int>(B),
                        static_cast<int>(Hq), static_cast<int>(Hkv), static_cast<int>(k_cache.size(2)),
                        static_cast<int>(splits));
}

void rope_attention_op(const at::Tensor& qkv, const at::Tensor& cos, const at::Tensor& sin, const at::Tensor& pos,
                       at::Tensor& k_cache, at::Tensor& v_cache, at::Tensor& out, int64_t Hq, int64_t Hkv,
                       int64_t splits) {
  TORCH_CHECK(qkv.dim() == 2 && qkv.size(1) == (Hq + 2 * Hkv) * 128 && qkv.is_contiguous(), "rope_attention: qkv");
  TORCH_CHECK(k_cache.dim() == 4 && k_cache.size(1) == Hkv && cos.scalar_type() == at::kFloat, "rope_attention: shapes");
  const at::cuda::OptionalCUDAGuard guard(qkv.device());
  nab::rope_attention(at::cuda::getCurrentCUDAStream().stream(), qkv.data_ptr(), cos.data_ptr<float>(),
                      sin.data_ptr<float>(), pos.data_ptr<int>(), k_cache.data_ptr(), v_cache.data_ptr(),
                      out.data_ptr(), static_cast<int>(qkv.size(0)), static_cast<int>(Hq), static_cast<int>(Hkv),
                      static_cast<int>(k_cache.size(2)), static_cast<int>(splits));
}

void decode_attention_tc_op(const at::Tensor& q, const at::Tensor& k_cache, const at::Tensor& v_cache,
                            const at::Tensor& pos, at::Tensor& out, int64_t splits) {
  TORCH_CHECK(q.dim() == 3 && q.size(2) == 128 && k_cache.dim() == 4 && k_cache.size(3) == 128 && q.is_contiguous() &&
                  k_cache.is_contiguous() && v_cache.is_contiguous() && v_cache.sizes() == k_cache.sizes(),
              "decode_attention_tc: shapes");
  const int64_t B = q.size(0), Hq = q.size(1), Hkv = k_cache.size(1);
  const at::cuda::OptionalCUDAGuard guard(q.device());
  nab::decode_attention_tc(at::cuda::getCurrentCUDAStream().stream(), q.data_ptr(), k_cache.data_ptr(),
                           v_cache.data_ptr(), pos.data_ptr<int>(), out.data_ptr(), static_cast<int>(B),
                           static_cast<int>(Hq), static_cast<int>(Hkv), static_cast<int>(k_cache.size(2)),
                           static_cast<int>(splits));
}

void rope_attention_tc_op(const at::Tensor& qkv, const at::Tensor& cos, const at::Tensor& sin, const at::Tensor& pos,
                          at::Tensor& k_cache, at::Tensor& v_cache, at::Tensor& out, int64_t Hq, int64_t Hkv,
                          int64_t splits) {
  TORCH_CHECK(qkv.dim() == 2 && qkv.size(1) == (Hq + 2 * Hkv) * 128 && qkv.is_contiguous(), "rope_attention_tc: qkv");
  TORCH_CHECK(k_cache.dim() == 4 && k_cache.size(1) == Hkv && k_cache.size(3) == 128 && k_cache.is_contiguous() &&
                  v_cache.is_contiguous() && v_cache.sizes() == k_cache.sizes() && cos.scalar_type() == at::kFloat,
              "rope_attention_tc: shapes");
  const at::cuda::OptionalCUDAGuard guard(qkv.device());
  nab::rope_attention_tc(at::cuda::getCurrentCUDAStream().stream(), qkv.data_ptr(), cos.data_ptr<float>(),
                         sin.data_ptr<float>(), pos.data_ptr<int>(), k_cache.data_ptr(), v_cache.data_ptr(),
                         out.data_ptr(), static_cast<int>(qkv.size(0)), static_cast<int>(Hq), static_cast<int>(Hkv),
                         static_cast<int>(k_cache.size(2)), static_cast<int>(splits));
}

int64_t attention_splits_tc(int64_t B, int64_t Hkv, int64_t context) {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return nab::attention_splits_tc(static_cast<int>(B), static_cast<int>(Hkv), static_cast<int>(context), sms);
}

int64_t attention_splits(int64_t B, int64_t Hkv, int64_t context) {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return nab::attention_splits(static_cast<int>(B), static_cast<int>(Hkv), static_cast<int>(context), sms);
}

void silu_mul_op(const at::Tensor& gu, at::Tensor& out) {
  TORCH_CHECK(gu.is_contiguous() && out.is_contiguous() && gu.dim() == 2 && gu.size(1) == 2 * out.size(1),
              "silu_mul: shapes");
  const at::cuda::OptionalCUDAGuard guard(gu.device());
  nab::silu_mul(at::cuda::getCurrentCUDAStream().stream(), gu.data_ptr(), out.data_ptr(),
                static_cast<int>(gu.size(0)), static_cast<int>(out.size(1)));
}

}  // namespace

TORCH_LIBRARY(nab, m) {
  m.def("meta_size() -> int", &meta_size);
  // cfg: [oneshot_max, chunk_max, max_ctas, oneshot_ctas, fused_bytes, timeout_ns, pipe_ctas, pipe_tile,
  //       hybrid_p2p_permille, hybrid_p2p_ctas, hybrid_nvls_ctas, oneshot_grain]; negative = default
  m.def("layout(int ws, int[] cfg) -> int[]", &layout);
  m.def("init(int[] ws_ptrs, Tensor rank_data, int rank, bool full_nvlink, int[] cfg) -> int", &init);
  m.def("dispose(int fa) -> ()", &dispose);
  m.def("set_groups(int fa, int[] flat, int ngroups) -> ()", &set_groups);
  m.def("attach_nvls(int fa, int mc, int uc, int bytes) -> ()", &attach_nvls);
  m.def("register_buffer(int fa, int[] ptrs) -> ()", &register_buffer);
  m.def("all_reduce(int fa, Tensor inp, Tensor(a!) out, int reg_buffer, int reg_buffer_sz_bytes) -> ()");
  m.impl("all_reduce", c10::kCUDA, &all_reduce);
  m.def("all_reduce_algo(int fa, Tensor inp, Tensor(a!) out, int algo, bool registered) -> ()");
  m.impl("all_reduce_algo", c10::kCUDA, &all_reduce_algo);
  m.def("reduce_scatter(int fa, Tensor inp, Tensor(a!) out) -> ()");
  m.impl("reduce_scatter", c10::kCUDA, &reduce_scatter);
  m.def("all_gather(int fa, Tensor inp, Tensor(a!) out) -> ()");
  m.impl("all_gather", c10::kCUDA, &all_gather);
  m.def("emulate_collective(int[] fas, Tensor[] ins, Tensor(a!)[] outs, int kind, int participants=-1) -> int");
  m.impl("emulate_collective", c10::kCUDA, &emulate_collective);
  m.def("plan_algo(int fa, int nbytes, int algo, bool registered, int dtype=2) -> int", &plan_algo);
  m.def("plan(int fa, int nbytes, int algo, bool registered, int dtype=2) -> int[]", &plan);
  m.def("set_auto_table(int fa, int dtype, int[] limits, int[] algos, int fallback) -> ()", &set_auto_table);
  m.def("get_auto_table(int fa, int dtype) -> (int[], int[], int)", &get_auto_table);
  m.def("builtin_auto_table(int ws, bool has_nvls) -> (int[], int[], int)", &builtin_auto_table);
  m.def("choose_auto(int ws, int nbytes, bool has_nvls, bool has_groups, int[] limits, int[] algos, int fallback) "
        "-> int", &choose_auto);
  m.def("set_hybrid(int fa, int permille, int p2p_ctas, int nvls_ctas) -> ()", &set_hybrid);
  m.def("kernel_error_state() -> int[]", &kernel_error_state);
  m.def("debug_bounds_build() -> bool", &debug_bounds_build);
#if NAB_DEBUG_BOUNDS
  m.def("debug_emulate_bad_rank(int[] fas, Tensor[] ins, Tensor(a!)[] outs, int algo) -> ()");
  m.impl("debug_emulate_bad_rank", c10::kCUDA, &debug_emulate_bad_rank);
#endif
  m.def("kernel_error_code() -> int", &kernel_error_code);
  m.def("kernel_error_reset() -> ()", &kernel_error_reset);
  m.def("emulate_all_reduce(int[] fas, Tensor[] ins, Tensor(a!)[] outs, int algo, int participants=-1) -> ()");
  m.impl("emulate_all_reduce", c10::kCUDA, &emulate_all_reduce);
  m.def("get_graph_buffer_ipc_meta(int fa) -> (int[], int[])", &get_graph_buffer_ipc_meta);
  m.def("register_graph_buffers(int fa, int[][] handles, int[][] offsets) -> ()", &register_graph_buffers);
  m.def("num_graph_buffers(int fa) -> int", &num_graph_buffers);
  m.def("allocate_shared_buffer_and_handle(int size) -> (int, Tensor)", &allocate_shared_buffer_and_handle);
  m.def("open_mem_handle(Tensor mem_handle) -> int", &open_mem_handle);
  m.def("close_mem_handle(int ptr) -> ()", &close_mem_handle);
  m.def("free_shared_buffer(int ptr) -> ()", &free_shared_buffer);
  m.def("error_code(int fa) -> int", &error_code);
  m.def("error_state(int fa) -> int[]", &error_state);
  m.def("reset(int fa) -> ()", &reset);
  m.def("launches(int fa) -> int", &launches);
  m.def("nvls_supported(int dev) -> bool", &nvls_supported);
  m.def("nvls_new(int dev, int ws, int bytes) -> int", &nvls_new);
  m.def("nvls_bytes(int h) -> int", &nvls_bytes);
  m.def("nvls_create(int h) -> int", &nvls_create);
  m.def("nvls_import(int h, int fd) -> ()", &nvls_import);
  m.def("nvls_add_device(int h) -> ()", &nvls_add_device);
  m.def("nvls_bind(int h) -> ()", &nvls_bind);
  m.def("nvls_ptrs(int h) -> int[]", &nvls_ptrs);
  m.def("nvls_release(int h) -> ()", &nvls_release);
  m.def("nvls_free(int h) -> ()", &nvls_free);
  m.def("sock_listen(str name) -> int", &sock_listen);
  m.def("sock_send_fd(str name, int fd, int timeout_ms) -> ()", &sock_send_fd);
  m.def("sock_recv_fd(int lfd, int timeout_ms) -> int", &sock_recv_fd);
  m.def("sock_close(int fd) -> ()", &sock_close);
  m.def("fused_ar_rmsnorm(int fa, Tensor inp, Tensor(a!) residual, Tensor weight, Tensor(b!) out, float eps, "
        "int algo) -> ()");
  m.impl("fused_ar_rmsnorm", c10::kCUDA, &fused_ar_rmsnorm);
  m.def("emulate_fused_ar_rmsnorm(int[] fas, Tensor[] ins, Tensor(a!)[] residuals, Tensor[] weights, "
        "Tensor(b!)[] outs, float eps, int algo) -> ()");
  m.impl("emulate_fused_ar_rmsnorm", c10::kCUDA, &emulate_fused_ar_rmsnorm);
  m.def("gemm(Tensor x, Tensor wt, Tensor(a!) y, int splits=0, bool packed=False, bool swiglu=False) -> ()");
  m.impl("gemm", c10::kCUDA, &gemm);
  m.def("gemm_splits(int T, int N, int K) -> int", &gemm_splits);
  m.def("gemm_active_clusters(int bn, int cs) -> int", &gemm_active_clusters);
  m.def("gemm_ar_rmsnorm(int fa, Tensor x, Tensor wt, Tensor(a!) residual, Tensor weight, Tensor(b!) out, "
        "float eps, int splits=0, bool packed=False, int mode=0) -> ()");
  m.def("gemm_ar_mode(int T, int ws) -> int", &gemm_ar_mode);
  m.impl("gemm_ar_rmsnorm", c10::kCUDA, &gemm_ar_rmsnorm);
  m.def("rope_append(Tensor qkv, Tensor cos, Tensor sin, Tensor pos, Tensor(a!) q_out, Tensor(b!) k_cache, "
        "Tensor(c!) v_cache, int Hq, int Hkv) -> ()");
  m.impl("rope_append", c10::kCUDA, &rope_append_op);
  m.def("decode_attention(Tensor q, Tensor k_cache, Tensor v_cache, Tensor pos, Tensor(a!) out, int splits) -> ()");
  m.def("rope_attention(Tensor qkv, Tensor cos, Tensor sin, Tensor pos, Tensor(a!) k_cache, Tensor(b!) v_cache, "
        "Tensor(c!) out, int Hq, int Hkv, int splits) -> ()");
  m.impl("rope_attention", c10::kCUDA, &rope_attention_op);
  m.def("attention_splits(int B, int Hkv, int context) -> int", &attention_splits);
  m.impl("decode_attention", c10::kCUDA, &decode_attention_op);
  m.def("decode_attention_tc(Tensor q, Tensor k_cache, Tensor v_cache, Tensor pos, Tensor(a!) out, int splits) -> ()");
  m.impl("decode_attention_tc", c10::kCUDA, &decode_attention_tc_op);
  m.def("rope_attention_tc(Tensor qkv, Tensor cos, Tensor sin, Tensor pos, Tensor(a!) k_cache, Tensor(b!) v_cache, "
        "Tensor(c!) out, int Hq, int Hkv, int splits) -> ()");
  m.impl("rope_attention_tc", c10::kCUDA, &rope_attention_tc_op);
  m.def("attention_splits_tc(int B, int Hkv, int context) -> int", &attention_splits_tc);
  m.def("silu_mul(Tensor gu, Tensor(a!) out) -> ()");
  m.impl("silu_mul", c10::kCUDA, &silu_mul_op);
  m.def("rmsnorm_residual(Tensor inp, Tensor(a!) residual, Tensor weight, Tensor(b!) out, float eps) -> ()");
  m.impl("rmsnorm_residual", c10::kCUDA, &rmsnorm_residual);
}
