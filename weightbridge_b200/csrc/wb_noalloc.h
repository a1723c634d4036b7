// No-allocation entry point of the transfer kernel.
//
// This entry point has no counterpart in the reference project (which ships no native code);
// it exists for callers of this library that cannot allocate GPU memory themselves.
//
// Who needs it: a rollout engine that hands all free GPU memory to its own allocator (for
// instance a KV-cache pool sized to "everything that is left", or an allocator that tags
// every cudaMalloc so it can release and restore memory around weight updates), and plain
// C/C++ hosts with no tensor framework to allocate from.  For them a weight update must not
// call cudaMalloc: a new allocation either fails because the memory is already reserved, or
// escapes the engine's bookkeeping.  Such a caller passes its work table in host memory and
// the destination/source buffers it already owns; the library keeps the little device-side
// state the kernel needs (the staged work table, the flag-address table, the epoch word and
// the completion counter) in a fixed-size array that is part of the loaded module.
//
// The scratch array lives in device memory of every GPU that loads this library, from load
// until process exit, whether or not this entry point is ever called.  Its size is fixed at
// build time by the two limits below (about 400 KB); a host staging block of the same size,
// also part of the library, carries the arguments over.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#define WB_NOALLOC_MAX_ITEMS 8192u  // work items per call (48 bytes each, host layout wb::Item)
#define WB_NOALLOC_MAX_FLAGS 64u    // flag words per call

// Error codes returned in addition to cudaError_t values (which are >= 0).
#define WB_NOALLOC_ERR_TOO_MANY_ITEMS (-1)  // n_items > WB_NOALLOC_MAX_ITEMS; nothing was launched
#define WB_NOALLOC_ERR_TOO_MANY_FLAGS (-2)  // n_flags > WB_NOALLOC_MAX_FLAGS; nothing was launched
#define WB_NOALLOC_ERR_NULL_ARGUMENT (-3)   // a count is non-zero but its host pointer is NULL

#ifdef __cplusplus
extern "C" {
#endif

// Copy/cast the regions described by `host_items` (n_items rows of the 48-byte wb::Item layout
// from wb_common.h, living in HOST memory; their src/dst fields are device addresses the
// caller owns, including CUDA IPC mappings of peer GPUs) on `stream`, on the current device.
// When the last block finishes, every address in `host_flag_addrs` (host array of n_flags
// device addresses of 8-byte words) receives `epoch` with a system-scope release store.
// Kernel errors set bits in *status (a device word owned by the caller; may be NULL).
//
// Allocates nothing: no cudaMalloc, cudaFree or allocating library call.  The work table,
// flag table and epoch are first copied into a fixed staging block in the library's own host
// memory and then sent with ONE cudaMemcpyAsync on `stream` into the library's fixed device
// scratch array (the same copy zeroes the completion counter).  Because that staging block is
// ordinary pageable memory, the copy has read it before cudaMemcpyAsync returns, so the
// caller's host arrays may be reused as soon as this call returns, whether they are pageable,
// pinned or registered memory.  A host-to-device copy from pageable memory also waits for the
// work already queued on `stream`: this call blocks the calling thread until that work is done.
//
// The first call on a device (with that device current) looks up the scratch array's device
// address (cudaGetSymbolAddress) and caches it per device and driver context; make that first
// call before any stream capture on the device, and do not reset the device (cudaDeviceReset)
// between calls.  All calls share the one scratch array and it keeps the contents of the last
// call.  Calls from several host threads are serialised while they stage and enqueue, but two
// calls whose work overlaps on the GPU (different streams, or the same device driven by
// several threads without ordering) race on the scratch and must be serialised by the caller.
//
// Returns 0 on success, a WB_NOALLOC_ERR_* code for rejected arguments, or the cudaError_t
// of the failing CUDA runtime call.
int wb_transfer_noalloc(const void* host_items, uint32_t n_items, const uint64_t* host_flag_addrs,
                        uint32_t n_flags, uint64_t epoch, uint32_t* status, cudaStream_t stream);

#ifdef __cplusplus
}
#endif
