// Access to CUDA driver API entry points without linking libcuda: the entry
// points are fetched through the runtime, so the library also loads on hosts
// that have no GPU driver (CPU-only test machines).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <stdexcept>
#include <string>

namespace nab {

void* driver_entry(const char* name);  // throws if unavailable

template <typename F>
F driver_fn(const char* name) {
  return reinterpret_cast<F>(driver_entry(name));
}

std::string cu_error_string(CUresult r);

#define NAB_CU_CHECK(expr)                                                          \
  do {                                                                              \
    CUresult _r = (expr);                                                           \
    if (_r != CUDA_SUCCESS)                                                         \
      throw std::runtime_error(std::string("CUDA driver error in ") + #expr + ": " + \
                               ::nab::cu_error_string(_r));                         \
  } while (0)

#define NAB_CUDA_CHECK(expr)                                                         \
  do {                                                                               \
    cudaError_t _e = (expr);                                                         \
    if (_e != cudaSuccess)                                                           \
      throw std::runtime_error(std::string("CUDA error in ") + #expr + ": " +         \
                               cudaGetErrorString(_e));                              \
  } while (0)

}  // namespace nab
