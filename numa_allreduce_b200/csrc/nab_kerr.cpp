// Per-device error record of the GEMM and attention kernels. See nab_kerr.h.
#include "nab_kerr.h"

#include <cuda_runtime.h>

#include <cstdlib>
#include <cstring>
#include <mutex>
#include <stdexcept>
#include <string>

#include "nab_driver.h"

namespace nab {

namespace {

constexpr int kMaxDevices = 64;
std::mutex g_mu;
KernelErrorRecord g_rec[kMaxDevices] = {};

int current_device() {
  int dev = 0;
  NAB_CUDA_CHECK(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) throw std::runtime_error("device ordinal out of range");
  return dev;
}

}  // namespace

KernelErrorRecord kernel_error_record() {
  const int dev = current_device();
  std::lock_guard<std::mutex> lock(g_mu);
  KernelErrorRecord& r = g_rec[dev];
  if (r.dev == nullptr) {
    cudaStreamCaptureMode mode = cudaStreamCaptureModeRelaxed;
    NAB_CUDA_CHECK(cudaThreadExchangeStreamCaptureMode(&mode));
    ErrorState* d = nullptr;
    uint32_t* h = nullptr;
    cudaError_t e = cudaMalloc(&d, sizeof(ErrorState));
    if (e == cudaSuccess) e = cudaMemset(d, 0, sizeof(ErrorState));
    if (e == cudaSuccess) e = cudaHostAlloc(&h, 64, cudaHostAllocMapped | cudaHostAllocPortable);
    cudaThreadExchangeStreamCaptureMode(&mode);
    if (e != cudaSuccess) {
      if (d) cudaFree(d);
      throw std::runtime_error(std::string("kernel error record: ") + cudaGetErrorString(e));
    }
    std::memset(h, 0, 64);
    r.dev = d;
    r.host = h;
  }
  return r;
}

uint64_t kernel_timeout_ns() {
  static const uint64_t t = [] {
    const char* v = std::getenv("NAB_TIMEOUT_NS");
    if (v != nullptr && *v != '\0') {
      char* end = nullptr;
      const unsigned long long x = std::strtoull(v, &end, 0);
      if (end != v && x > 0) return static_cast<uint64_t>(x);
    }
    return uint64_t(5000000000ull);
  }();
  return t;
}

uint32_t kernel_error_code() {
  const KernelErrorRecord r = kernel_error_record();
  return *reinterpret_cast<volatile uint32_t*>(r.host);
}

ErrorState kernel_error_state() {
  const KernelErrorRecord r = kernel_error_record();
  ErrorState st{};
  NAB_CUDA_CHECK(cudaMemcpy(&st, r.dev, sizeof(st), cudaMemcpyDeviceToHost));
  return st;
}

void kernel_error_reset() {
  const KernelErrorRecord r = kernel_error_record();
  NAB_CUDA_CHECK(cudaDeviceSynchronize());
  NAB_CUDA_CHECK(cudaMemset(r.dev, 0, sizeof(ErrorState)));
  NAB_CUDA_CHECK(cudaDeviceSynchronize());
  std::memset(r.host, 0, 64);
}

}  // namespace nab
