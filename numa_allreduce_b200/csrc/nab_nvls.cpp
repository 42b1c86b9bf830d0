// NVLS workspace and file-descriptor passing. See nab_nvls.h.
#include "nab_nvls.h"

#include <poll.h>
#include <sys/socket.h>
#include <sys/un.h>
#include <unistd.h>

#include <cerrno>
#include <chrono>
#include <cstring>
#include <stdexcept>
#include <thread>

#include "nab_driver.h"

namespace nab {

namespace {

using PFN_DevGetAttr = CUresult (*)(int*, CUdevice_attribute, CUdevice);
using PFN_DevGet = CUresult (*)(CUdevice*, int);
using PFN_McGran = CUresult (*)(size_t*, const CUmulticastObjectProp*, CUmulticastGranularity_flags);
using PFN_McCreate = CUresult (*)(CUmemGenericAllocationHandle*, const CUmulticastObjectProp*);
using PFN_McAdd = CUresult (*)(CUmemGenericAllocationHandle, CUdevice);
using PFN_McBind = CUresult (*)(CUmemGenericAllocationHandle, size_t, CUmemGenericAllocationHandle,
                                size_t, size_t, unsigned long long);
using PFN_McUnbind = CUresult (*)(CUmemGenericAllocationHandle, CUdevice, size_t, size_t);
using PFN_MemCreate = CUresult (*)(CUmemGenericAllocationHandle*, size_t, const CUmemAllocationProp*,
                                   unsigned long long);
using PFN_MemGran = CUresult (*)(size_t*, const CUmemAllocationProp*, CUmemAllocationGranularity_flags);
using PFN_MemRelease = CUresult (*)(CUmemGenericAllocationHandle);
using PFN_Export = CUresult (*)(void*, CUmemGenericAllocationHandle, CUmemAllocationHandleType,
                                unsigned long long);
using PFN_Import = CUresult (*)(CUmemGenericAllocationHandle*, void*, CUmemAllocationHandleType);
using PFN_Reserve = CUresult (*)(CUdeviceptr*, size_t, size_t, CUdeviceptr, unsigned long long);
using PFN_Free = CUresult (*)(CUdeviceptr, size_t);
using PFN_Map = CUresult (*)(CUdeviceptr, size_t, size_t, CUmemGenericAllocationHandle, unsigned long long);
using PFN_Unmap = CUresult (*)(CUdeviceptr, size_t);
using PFN_SetAccess = CUresult (*)(CUdeviceptr, size_t, const CUmemAccessDesc*, size_t);

CUdevice cu_device(int ordinal) {
  CUdevice d;
  NAB_CU_CHECK(driver_fn<PFN_DevGet>("cuDeviceGet")(&d, ordinal));
  return d;
}

size_t round_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

sockaddr_un abstract_addr(const std::string& name, socklen_t* len) {
  sockaddr_un a;
  std::memset(&a, 0, sizeof(a));
  a.sun_family = AF_UNIX;
  if (name.size() + 1 > sizeof(a.sun_path)) throw std::invalid_argument("socket name too long");
  a.sun_path[0] = '\0';  // abstract namespace: no file system entry
  std::memcpy(a.sun_path + 1, name.data(), name.size());
  *len = static_cast<socklen_t>(offsetof(sockaddr_un, sun_path) + 1 + name.size());
  return a;
}

}  // namespace

bool nvls_supported(int device) {
  try {
    int v = 0;
    NAB_CU_CHECK(driver_fn<PFN_DevGetAttr>("cuDeviceGetAttribute")(
        &v, CU_DEVICE_ATTRIBUTE_MULTICAST_SUPPORTED, cu_device(device)));
    return v != 0;
  } catch (...) {
    return false;
  }
}

static CUmemAllocationProp phys_prop(int device) {
  CUmemAllocationProp ap{};
  ap.type = CU_MEM_ALLOCATION_TYPE_PINNED;
  ap.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
  ap.location.id = device;
  // same shareable handle type as the multicast object
  ap.requestedHandleTypes = CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR;
  return ap;
}

NvlsBuffer::NvlsBuffer(int device, int world_size, size_t min_bytes)
    : device_(device), ws_(world_size) {
  CUmulticastObjectProp mp{};
  mp.numDevices = static_cast<unsigned>(world_size);
  mp.size = min_bytes;
  mp.handleTypes = CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR;
  NAB_CU_CHECK(driver_fn<PFN_McGran>("cuMulticastGetGranularity")(&mc_gran_, &mp,
                                                                   CU_MULTICAST_GRANULARITY_RECOMMENDED));
  const CUmemAllocationProp ap = phys_prop(device);
  NAB_CU_CHECK(driver_fn<PFN_MemGran>("cuMemGetAllocationGranularity")(
      &alloc_gran_, &ap, CU_MEM_ALLOC_GRANULARITY_RECOMMENDED));
  const size_t gran = std::max(mc_gran_, alloc_gran_);
  bytes_ = round_up(min_bytes, gran);
}

std::string NvlsBuffer::describe() const {
  return "bytes=" + std::to_string(bytes_) + " multicast_granularity=" + std::to_string(mc_gran_) +
         " allocation_granularity=" + std::to_string(alloc_gran_) + " device=" + std::to_string(device_) +
         " world=" + std::to_string(ws_);
}

NvlsBuffer::~NvlsBuffer() {
  try {
    release();
  } catch (...) {
  }
}

int NvlsBuffer::create() {
  CUmulticastObjectProp mp{};
  mp.numDevices = static_cast<unsigned>(ws_);
  mp.size = bytes_;
  mp.handleTypes = CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR;
  NAB_CU_CHECK(driver_fn<PFN_McCreate>("cuMulticastCreate")(&mc_, &mp));
  have_mc_ = true;
  int fd = -1;
  NAB_CU_CHECK(driver_fn<PFN_Export>("cuMemExportToShareableHandle")(
      &fd, mc_, CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR, 0));
  export_fd_ = fd;
  return fd;
}

void NvlsBuffer::import_fd(int fd) {
  NAB_CU_CHECK(driver_fn<PFN_Import>("cuMemImportFromShareableHandle")(
      &mc_, reinterpret_cast<void*>(static_cast<uintptr_t>(fd)),
      CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR));
  have_mc_ = true;
  ::close(fd);
}

void NvlsBuffer::add_device() {
  if (!have_mc_) throw std::runtime_error("multicast object not created or imported");
  NAB_CU_CHECK(driver_fn<PFN_McAdd>("cuMulticastAddDevice")(mc_, cu_device(device_)));
  added_ = true;
}

void NvlsBuffer::bind_and_map() {
  if (!added_) throw std::runtime_error("add_device must precede bind_and_map");
  const CUmemAllocationProp ap = phys_prop(device_);
  NAB_CU_CHECK(driver_fn<PFN_MemCreate>("cuMemCreate")(&phys_, bytes_, &ap, 0));
  have_phys_ = true;
  const CUresult r = driver_fn<PFN_McBind>("cuMulticastBindMem")(mc_, 0, phys_, 0, bytes_, 0);
  if (r != CUDA_SUCCESS)
    throw std::runtime_error("cuMulticastBindMem failed: " + cu_error_string(r) + " (" + describe() + ")");
  bound_ = true;
  CUmemAccessDesc ad{};
  ad.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
  ad.location.id = device_;
  ad.flags = CU_MEM_ACCESS_FLAGS_PROT_READWRITE;
  auto reserve = driver_fn<PFN_Reserve>("cuMemAddressReserve");
  auto map = driver_fn<PFN_Map>("cuMemMap");
  auto access = driver_fn<PFN_SetAccess>("cuMemSetAccess");
  CUdeviceptr uc = 0, mc = 0;
  NAB_CU_CHECK(reserve(&uc, bytes_, 0, 0, 0));
  NAB_CU_CHECK(map(uc, bytes_, 0, phys_, 0));
  NAB_CU_CHECK(access(uc, bytes_, &ad, 1));
  uc_va_ = reinterpret_cast<void*>(uc);
  NAB_CU_CHECK(reserve(&mc, bytes_, 0, 0, 0));
  NAB_CU_CHECK(map(mc, bytes_, 0, mc_, 0));
  NAB_CU_CHECK(access(mc, bytes_, &ad, 1));
  mc_va_ = reinterpret_cast<void*>(mc);
  NAB_CUDA_CHECK(cudaMemset(uc_va_, 0, bytes_));
  NAB_CUDA_CHECK(cudaDeviceSynchronize());
}

void NvlsBuffer::release() {
  auto unmap = driver_fn<PFN_Unmap>("cuMemUnmap");
  auto vfree = driver_fn<PFN_Free>("cuMemAddressFree");
  auto rel = driver_fn<PFN_MemRelease>("cuMemRelease");
  if (mc_va_ || uc_va_) cudaDeviceSynchronize();
  if (mc_va_) {
    unmap(reinterpret_cast<CUdeviceptr>(mc_va_), bytes_);
    vfree(reinterpret_cast<CUdeviceptr>(mc_va_), bytes_);
    mc_va_ = nullptr;
  }
  if (uc_va_) {
    unmap(reinterpret_cast<CUdeviceptr>(uc_va_), bytes_);
    vfree(reinterpret_cast<CUdeviceptr>(uc_va_), bytes_);
    uc_va_ = nullptr;
  }
  if (bound_) {
    driver_fn<PFN_McUnbind>("cuMulticastUnbind")(mc_, cu_device(device_), 0, bytes_);
    bound_ = false;
  }
  if (have_phys_) {
    rel(phys_);
    have_phys_ = false;
  }
  if (have_mc_) {
    rel(mc_);
    have_mc_ = false;
  }
  if (export_fd_ >= 0) {
    ::close(export_fd_);
    export_fd_ = -1;
  }
}

int sock_listen(const std::string& name) {
  const int fd = ::socket(AF_UNIX, SOCK_STREAM | SOCK_CLOEXEC, 0);
  if (fd < 0) throw std::runtime_error(std::string("socket: ") + std::strerror(errno));
  socklen_t len;
  sockaddr_un a = abstract_addr(name, &len);
  if (::bind(fd, reinterpret_cast<sockaddr*>(&a), len) != 0 || ::listen(fd, 16) != 0) {
    const int err = errno;
    ::close(fd);
    throw std::runtime_error(std::string("bind/listen on abstract socket: ") + std::strerror(err));
  }
  return fd;
}

void sock_send_fd(const std::string& name, int fd_to_send, int timeout_ms) {
  socklen_t len;
  sockaddr_un a = abstract_addr(name, &len);
  const auto deadline = std::chrono::steady_clock::now() + std::chrono::milliseconds(timeout_ms);
  int s = -1;
  while (true) {
    s = ::socket(AF_UNIX, SOCK_STREAM | SOCK_CLOEXEC, 0);
    if (s < 0) throw std::runtime_error(std::string("socket: ") + std::strerror(errno));
    if (::connect(s, reinterpret_cast<sockaddr*>(&a), len) == 0) break;
    ::close(s);
    if (std::chrono::steady_clock::now() > deadline)
      throw std::runtime_error("timed out connecting to peer socket " + name);
    std::this_thread::sleep_for(std::chrono::milliseconds(5));
  }
  char byte = 'F';
  iovec iov{&byte, 1};
  char ctrl[CMSG_SPACE(sizeof(int))];
  std::memset(ctrl, 0, sizeof(ctrl));
  msghdr msg{};
  msg.msg_iov = &iov;
  msg.msg_iovlen = 1;
  msg.msg_control = ctrl;
  msg.msg_controllen = sizeof(ctrl);
  cmsghdr* c = CMSG_FIRSTHDR(&msg);
  c->cmsg_level = SOL_SOCKET;
  c->cmsg_type = SCM_RIGHTS;
  c->cmsg_len = CMSG_LEN(sizeof(int));
  std::memcpy(CMSG_DATA(c), &fd_to_send, sizeof(int));
  const ssize_t n = ::sendmsg(s, &msg, 0);
  const int err = errno;
  ::close(s);
  if (n != 1) throw std::runtime_error(std::string("sendmsg: ") + std::strerror(err));
}

int sock_recv_fd(int listen_fd, int timeout_ms) {
  pollfd pfd{listen_fd, POLLIN, 0};
  const int pr = ::poll(&pfd, 1, timeout_ms);
  if (pr <= 0) throw std::runtime_error("timed out waiting for a file descriptor from a peer");
  const int s = ::accept4(listen_fd, nullptr, nullptr, SOCK_CLOEXEC);
  if (s < 0) throw std::runtime_error(std::string("accept: ") + std::strerror(errno));
  char byte = 0;
  iovec iov{&byte, 1};
  char ctrl[CMSG_SPACE(sizeof(int))];
  msghdr msg{};
  msg.msg_iov = &iov;
  msg.msg_iovlen = 1;
  msg.msg_control = ctrl;
  msg.msg_controllen = sizeof(ctrl);
  pollfd p2{s, POLLIN, 0};
  if (::poll(&p2, 1, timeout_ms) <= 0) {
    ::close(s);
    throw std::runtime_error("timed out receiving a file descriptor");
  }
  const ssize_t n = ::recvmsg(s, &msg, 0);
  ::close(s);
  if (n != 1) throw std::runtime_error("recvmsg failed");
  cmsghdr* c = CMSG_FIRSTHDR(&msg);
  if (!c || c->cmsg_type != SCM_RIGHTS) throw std::runtime_error("no file descriptor received");
  int fd;
  std::memcpy(&fd, CMSG_DATA(c), sizeof(int));
  return fd;
}

void sock_close(int fd) {
  if (fd >= 0) ::close(fd);
}

}  // namespace nab
