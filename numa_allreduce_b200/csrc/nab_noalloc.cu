// Allocation-free entry point (no counterpart in the reference); declared in
// nab_noalloc.h.
//
//   int nab_noalloc_emulated_allreduce(const void* const* inputs,
//                                      void* const* outputs, int world_size,
//                                      int64_t numel, int dtype, void* stream);
//   int nab_noalloc_last_error(uint32_t* record);
//
// Runs the two-shot allreduce kernel for `world_size` ranks whose buffers all
// live on the current GPU (the same single-GPU emulation the library's tests
// use: one cooperative launch, one grid row per rank), and allocates nothing:
// the signal pads, reduce-scatter slots and error record live in a static
// device array owned by this file.
//
// Who needs this: callers that cannot call cudaMalloc at the point where they
// reduce, for example code that runs while another allocator has reserved all
// device memory, real-time paths that must not enter the driver's allocator,
// or host code that is not allowed to own device allocations at all (plugins
// and firmware-style runtimes). Such a caller passes its inputs and outputs
// and nothing else.
//
// Limits and contract:
// * The scratch is kNoAllocScratchBytes (12 MiB) per GPU. Every GPU that loads
//   libnab.so holds it until the process exits. It serves up to 8 ranks; a
//   call whose layout would not fit is rejected with an error (message size
//   is not limited: the kernel loops over rounds).
// * The first call on each device looks up the array's device address
//   (cudaGetSymbolAddress, with that device current) and caches it; make that
//   first call before any stream capture.
// * Every call shares the array and leaves its contents behind: each call
//   clears the signal pads and the error record on its stream first. Calls
//   that overlap on the GPU (different streams, or different host threads on
//   the same device without ordering) race on the array; order them.
// * The return code covers the argument checks and the launch only: 0 when
//   the kernel was launched, 1 for a rejected argument, 2 when the world size
//   needs more scratch than the static array holds, 3 for a CUDA error; a
//   one-line reason goes to stderr (formatted in a fixed buffer, no heap).
//   A bounded wait inside the kernel that gives up (after NAB_TIMEOUT_NS,
//   default 5 s, read from the environment on every call) leaves the output
//   partly written and records the failure in the array's error record;
//   nab_noalloc_last_error copies that record out after the caller has
//   synchronized the stream.
// * numel * element size must be a positive multiple of 16 bytes and every
//   pointer 16-byte aligned; dtype is 0 (fp32), 1 (fp16) or 2 (bf16).
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <mutex>

#include <cstdlib>

#include "nab_kernels.h"
#include "nab_noalloc.h"
#include "nab_params.h"

namespace {

constexpr size_t kNoAllocScratchBytes = NAB_NOALLOC_SCRATCH_BYTES;
constexpr int kNoAllocMaxCtas = 8;              // CTAs per emulated rank
constexpr int64_t kNoAllocChunk = 16 << 10;     // bytes per owner chunk per round
constexpr int64_t kHeaderBytes = 4096;          // error record
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

char* g_scratch_addr[kMaxDevices] = {};
std::mutex g_setup_mu;
enum : int { kOk = 0, kBadArgument = 1, kScratchTooSmall = 2, kCudaError = 3 };

int fail(int code, const char* fmt, ...) {
  char msg[256];
  va_list ap;
  va_start(ap, fmt);
  std::vsnprintf(msg, sizeof(msg), fmt, ap);
  va_end(ap);
  std::fprintf(stderr, "nab_noalloc_emulated_allreduce: %s\n", msg);
  return code;
}

int64_t round_up(int64_t x, int64_t a) { return (x + a - 1) / a * a; }

// Bound of every device-side wait: NAB_TIMEOUT_NS if set (getenv and strtoull
// allocate nothing), else 5 s.
uint64_t timeout_ns() {
  const char* v = std::getenv("NAB_TIMEOUT_NS");
  if (v != nullptr && *v != '\0') {
    char* end = nullptr;
    const unsigned long long t = std::strtoull(v, &end, 0);
    if (end != v && t > 0) return static_cast<uint64_t>(t);
  }
  return 5000000000ull;
}

}  // namespace

extern "C" __attribute__((visibility("default"))) int nab_noalloc_emulated_allreduce(
    const void* const* inputs, void* const* outputs, int world_size, int64_t numel, int dtype, void* stream) {
  using namespace nab;
  if (world_size < 2 || world_size > kMaxRanks) return fail(kBadArgument, "world_size must be in [2, 8], got %d", world_size);
  if (dtype != kF32 && dtype != kF16 && dtype != kBF16) return fail(kBadArgument, "dtype must be 0, 1 or 2, got %d", dtype);
  if (!inputs || !outputs) return fail(kBadArgument, "inputs and outputs must not be null");
  const int64_t esize = dtype == kF32 ? 4 : 2;
  const int64_t nbytes = numel * esize;
  if (numel <= 0 || nbytes % 16 != 0) return fail(kBadArgument, "message must be a positive multiple of 16 bytes");
  for (int r = 0; r < world_size; ++r) {
    if (!inputs[r] || !outputs[r] || reinterpret_cast<uintptr_t>(inputs[r]) % 16 ||
        reinterpret_cast<uintptr_t>(outputs[r]) % 16)
      return fail(kBadArgument, "buffer of rank %d is null or not 16-byte aligned", r);
  }

  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(kCudaError, "cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return fail(kBadArgument, "device ordinal %d out of range", dev);
  char* base;
  {
    std::lock_guard<std::mutex> lock(g_setup_mu);
    if (g_scratch_addr[dev] == nullptr) {
      void* p = nullptr;
      e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
      if (e != cudaSuccess || p == nullptr)
        return fail(kCudaError, "cudaGetSymbolAddress of the scratch array failed: %s", cudaGetErrorString(e));
      g_scratch_addr[dev] = static_cast<char*>(p);
    }
    base = g_scratch_addr[dev];
  }

  // Layout: [error record][rank 0: signal pad | two-shot slots] ... [rank ws-1]
  int sms = 0;
  e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return fail(kCudaError, "cudaDeviceGetAttribute: %s", cudaGetErrorString(e));
  const int64_t npacks = nbytes / 16;
  const int64_t chunk_packs_cap = kNoAllocChunk / 16;
  int64_t C = (npacks + static_cast<int64_t>(world_size) * 512 - 1) / (static_cast<int64_t>(world_size) * 512);
  C = C < 1 ? 1 : C;
  C = C > kNoAllocMaxCtas ? kNoAllocMaxCtas : C;
  if (C > sms / world_size) C = sms / world_size;  // every CTA of every rank resident at once
  if (C < 1) return fail(kBadArgument, "device has too few SMs for %d emulated ranks", world_size);
  const int64_t pad_bytes = round_up(static_cast<int64_t>(sizeof(SignalPad)), 4096);
  const int64_t rank_bytes = pad_bytes + kNoAllocMaxCtas * (world_size + 1) * kNoAllocChunk;
  const int64_t need = kHeaderBytes + world_size * rank_bytes;
  if (need > static_cast<int64_t>(kNoAllocScratchBytes))
    return fail(kScratchTooSmall, "%d ranks need %lld scratch bytes; the static scratch holds %lld", world_size,
                static_cast<long long>(need), static_cast<long long>(kNoAllocScratchBytes));
  int64_t chp = (npacks + C * world_size - 1) / (C * world_size);
  chp = chp > chunk_packs_cap ? chunk_packs_cap : chp;
  chp = chp < 1 ? 1 : chp;
  const int64_t rounds = (npacks + C * world_size * chp - 1) / (C * world_size * chp);
  if (rounds >= (int64_t(1) << kSeqShift)) return fail(kBadArgument, "message too large");

  // Clear what must start at zero: the error record and every rank's pad.
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  e = cudaMemsetAsync(base, 0, kHeaderBytes, s);
  for (int r = 0; r < world_size && e == cudaSuccess; ++r)
    e = cudaMemsetAsync(base + kHeaderBytes + r * rank_bytes, 0, pad_bytes, s);
  if (e != cudaSuccess) return fail(kCudaError, "clearing the scratch failed: %s", cudaGetErrorString(e));

  ARParams p{};
  p.err = reinterpret_cast<ErrorState*>(base);
  p.err_host = nullptr;
  p.npacks = npacks;
  p.timeout_ns = timeout_ns();
  p.ws = world_size;
  p.chunk_packs = static_cast<int>(chp);
  p.rounds = static_cast<int>(rounds);
  p.L.twoshot_off = pad_bytes;
  p.L.chunk_max = kNoAllocChunk;
  p.L.max_ctas = kNoAllocMaxCtas;
  for (int r = 0; r < world_size; ++r) {
    RankView& v = p.v[r];
    v.in = static_cast<const char*>(inputs[r]);
    v.out = static_cast<char*>(outputs[r]);
    for (int q = 0; q < world_size; ++q) v.wsp[q] = base + kHeaderBytes + q * rank_bytes;
    v.rank = r;
  }
  e = launch_allreduce(kAlgoTwoshot, dtype, p, dim3(static_cast<unsigned>(C), static_cast<unsigned>(world_size)), s,
                       /*cooperative=*/true);
  if (e != cudaSuccess) return fail(kCudaError, "launch failed: %s", cudaGetErrorString(e));
  return kOk;
}

extern "C" __attribute__((visibility("default"))) int nab_noalloc_last_error(uint32_t* record) {
  static_assert(sizeof(nab::ErrorState) == 8 * sizeof(uint32_t), "record layout");
  if (record == nullptr) return fail(kBadArgument, "record must not be null");
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(kCudaError, "cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return fail(kBadArgument, "device ordinal %d out of range", dev);
  char* base;
  {
    std::lock_guard<std::mutex> lock(g_setup_mu);
    base = g_scratch_addr[dev];
  }
  if (base == nullptr) return kBadArgument;  // no call on this device yet: nothing recorded
  // the error record sits at the start of the array (see the layout above)
  e = cudaMemcpy(record, base, sizeof(nab::ErrorState), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return fail(kCudaError, "reading the error record failed: %s", cudaGetErrorString(e));
  return kOk;
}
