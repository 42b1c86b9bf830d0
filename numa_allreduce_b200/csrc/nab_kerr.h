// Error record of the kernels that do not belong to a communicator (the
// plain GEMM and the decode attention). Their only waits are on their own
// mbarriers (TMA and tensor-core completions), which run out only on a
// defect; such a wait records where it gave up here instead of hanging, and
// the kernel returns with a partial output. One record per device, in device
// memory plus a host-mapped copy of the error code, allocated on first use.
#pragma once

#include <cstdint>

#include "nab_common.h"

namespace nab {

struct KernelErrorRecord {
  ErrorState* dev;   // device memory, written by the kernels
  uint32_t* host;    // host-mapped copy of ErrorState::code
};

// The current device's record (allocated on the first call; the allocation
// is made in relaxed capture mode, so a first call during stream capture works).
KernelErrorRecord kernel_error_record();
// Bound of those waits: NAB_TIMEOUT_NS if set, else 5 s.
uint64_t kernel_timeout_ns();
// Error code from host-mapped memory (no synchronisation).
uint32_t kernel_error_code();
// Synchronous copy of the current device's full record.
ErrorState kernel_error_state();
// Clears the current device's record (synchronises the device first).
void kernel_error_reset();

}  // namespace nab
