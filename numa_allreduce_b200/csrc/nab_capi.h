// C declarations of libnab.so, the allreduce library without Python or torch.
//
// The first six functions keep the names and argument lists of the
// reference's C ABI (src/numa_all_reduce.cu:736-808), so a caller of that ABI
// links unchanged. They return 0 on success and 1 on failure (the reference
// returned void and exited the process on CUDA errors); nab_last_error gives
// the message of the calling thread's last failure. The allocation-free entry
// points are declared in nab_noalloc.h.
//
// Set-up, per process and GPU (one process per GPU):
//   1. allocate nab_workspace_bytes(world_size) bytes of device memory, zero
//      it, and exchange CUDA IPC handles so that every rank maps every other
//      rank's workspace ("signals" below, indexed by rank);
//   2. allocate a device buffer for the registry of registered inputs
//      ("rank_data", a few KiB per registered buffer);
//   3. numa_all_reduce_init on every rank, then the allreduce calls, all
//      ranks issuing the same calls in the same order;
//   4. numa_all_reduce_dispose.
#pragma once

#include <cuda_runtime_api.h>
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

// Copies the calling thread's last error message into buf (at most len - 1
// characters and a terminating zero); returns the message length.
int nab_last_error(char* buf, int len);

// Bytes of the IPC workspace each rank allocates for world_size ranks (1..8);
// -1 for an unsupported world size.
int64_t nab_workspace_bytes(int world_size);

// Creates the communicator of `rank` among `world_size` ranks. signals[r] is
// rank r's workspace as mapped in this process. nnuma > 1 splits the ranks
// into that many contiguous groups for the hierarchical protocol. Returns
// NULL on failure.
void* numa_all_reduce_init(void** signals, void* rank_data, size_t rank_data_sz, int rank, int world_size,
                           int nnuma);
int numa_all_reduce_dispose(void* ptr);

// Registers an IPC-shared input buffer (ptrs[r]: rank r's copy as mapped
// here) for the pull protocol.
int numa_all_reduce_register_buffer(void* ptr, void** ptrs);

// output = sum over ranks of input, `size` elements, the protocol chosen by
// the communicator's table (a message the table hands to NCCL takes the last
// custom protocol: this ABI has no NCCL to fall back to).
int numa_all_reduce_fp16(void* ptr, cudaStream_t stream, void* input, void* output, int size);
int numa_all_reduce_fp32(void* ptr, cudaStream_t stream, void* input, void* output, int size);
int numa_all_reduce_bf16(void* ptr, cudaStream_t stream, void* input, void* output, int size);

// The same with 64-bit element counts and an explicit protocol (0 automatic,
// 1 one-shot, 2 two-shot, 3 NVLS one-shot, 4 NVLS two-shot, 5 hierarchical,
// 6 pull one-shot, 8 pipelined two-shot, 9 hybrid); dtype 0 fp32, 1 fp16,
// 2 bf16.
int nab_allreduce(void* ptr, cudaStream_t stream, const void* input, void* output, int64_t numel, int dtype,
                  int algo);

// Contiguous-segment collectives, seg_numel elements per rank segment.
// Reduce-scatter: input holds world_size segments; output gets the sum over
// ranks of segment [rank]. All-gather: input is one segment; output gets the
// world_size ranks' segments in rank order.
int nab_reduce_scatter(void* ptr, cudaStream_t stream, const void* input, void* output, int64_t seg_numel,
                       int dtype);
int nab_all_gather(void* ptr, cudaStream_t stream, const void* input, void* output, int64_t seg_numel,
                   int dtype);

// Replaces the automatic choice's steps for one dtype: n ascending byte
// limits with their protocol ids, and the protocol of larger messages.
int nab_set_auto_table(void* ptr, int dtype, int n, const int64_t* max_bytes, const int* algos, int fallback);
// Hybrid protocol split: per mille of each message on the P2P part, and the
// CTAs of the P2P and NVLS parts.
int nab_set_hybrid(void* ptr, int p2p_permille, int p2p_ctas, int nvls_ctas);
// The protocol the automatic choice launches for a message (negative on error).
int nab_auto_protocol(void* ptr, int64_t nbytes, int dtype);

// Non-zero once a bounded device wait of this rank gave up (1 a timeout, 2 a
// failed launch check); reads host-mapped memory, no synchronisation.
uint32_t nab_error_code(void* ptr);
// Clears the error record and all flags and epochs of this rank. Every rank
// must reset together, with no call in flight.
int nab_reset(void* ptr);

#ifdef __cplusplus
}
#endif
