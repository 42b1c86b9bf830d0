// C declarations of libnab.so's allocation-free entry points (no counterpart
// in the reference).
//
// These are for callers that cannot call cudaMalloc at the point where they
// reduce: code that runs while another allocator has reserved all device
// memory, real-time paths that must not enter the driver's allocator, and
// host runtimes (plugins, firmware-style loaders) that may not own device
// allocations. Their scratch lives in a static device array of
// NAB_NOALLOC_SCRATCH_BYTES that every GPU loading libnab.so holds until the
// process exits. Calls share that array: calls that overlap on the GPU race,
// so order them on one stream.
#pragma once

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define NAB_NOALLOC_SCRATCH_BYTES (12u << 20)

// Two-shot allreduce of `world_size` (2..8) emulated ranks whose buffers all
// live on the current GPU: outputs[r] = sum over q of inputs[q], accumulated
// in fp32 in rank order. numel * element size must be a positive multiple of
// 16 bytes and every pointer 16-byte aligned; dtype is 0 (fp32), 1 (fp16) or
// 2 (bf16). The first call on a device looks up the scratch array's address
// with that device current; make it before any stream capture.
//
// The return code covers the argument checks and the launch only: 0 launched,
// 1 rejected argument, 2 the world size needs more scratch than the array
// holds, 3 CUDA error (a one-line reason goes to stderr). A bounded wait in
// the kernel that gives up (NAB_TIMEOUT_NS, default 5 s) is recorded in the
// scratch array's error record: read it with nab_noalloc_last_error after
// synchronizing the stream.
int nab_noalloc_emulated_allreduce(const void* const* inputs, void* const* outputs, int world_size,
                                   int64_t numel, int dtype, void* stream);

// Copies the current device's error record of the last call into record[8]:
// code (0 = none, 1 = a wait timed out), rank, peer, stage, CTA, call epoch,
// observed flag value, number of waits that gave up. Synchronous; call it
// after the stream of the allreduce has been synchronized. Returns 0 on
// success, 1 when no call has been made on this device yet, 3 on a CUDA error.
int nab_noalloc_last_error(uint32_t* record);

#ifdef __cplusplus
}
#endif
