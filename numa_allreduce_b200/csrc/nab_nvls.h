// NVLink SHARP (NVLS) workspace: one multicast object per communicator with a
// physical allocation of every GPU bound to it. Kernels use the multicast
// address for multimem.ld_reduce / multimem.st / multimem.red and their own
// unicast address for plain local loads and stores.
//
// The multicast handle crosses processes as a POSIX file descriptor, passed
// over an abstract-namespace Unix socket (SCM_RIGHTS). Python drives the
// steps and the host barriers between them.
//
// No counterpart in the reference (its data plane is legacy CUDA IPC only);
// this is the B200 path the build targets.
#pragma once

#include <cuda.h>

#include <cstddef>
#include <cstdint>
#include <string>

namespace nab {

bool nvls_supported(int device);

class NvlsBuffer {
 public:
  NvlsBuffer(int device, int world_size, size_t min_bytes);
  ~NvlsBuffer();
  NvlsBuffer(const NvlsBuffer&) = delete;
  NvlsBuffer& operator=(const NvlsBuffer&) = delete;

  size_t bytes() const { return bytes_; }
  std::string describe() const;
  // Root only: creates the multicast object and returns a FD that refers to
  // it (owned by this object; the caller sends it to the other ranks).
  int create();
  // Non-root: adopts the multicast object from a received FD.
  void import_fd(int fd);
  // Every rank, after create/import, before any rank binds memory.
  void add_device();
  // Every rank, after all ranks added their device: allocates this GPU's
  // physical memory, binds it and maps both addresses (zero-filled).
  void bind_and_map();
  uintptr_t mc_ptr() const { return reinterpret_cast<uintptr_t>(mc_va_); }
  uintptr_t uc_ptr() const { return reinterpret_cast<uintptr_t>(uc_va_); }
  // Unmaps and unbinds; all ranks should reach this together.
  void release();

 private:
  int device_;
  int ws_;
  size_t bytes_;
  size_t mc_gran_ = 0, alloc_gran_ = 0;
  CUmemGenericAllocationHandle mc_ = 0;
  CUmemGenericAllocationHandle phys_ = 0;
  bool have_mc_ = false, have_phys_ = false, bound_ = false, added_ = false;
  void* mc_va_ = nullptr;
  void* uc_va_ = nullptr;
  int export_fd_ = -1;
};

// Abstract Unix sockets for passing file descriptors between local processes.
int sock_listen(const std::string& name);
void sock_send_fd(const std::string& name, int fd, int timeout_ms);
int sock_recv_fd(int listen_fd, int timeout_ms);
void sock_close(int fd);

}  // namespace nab
