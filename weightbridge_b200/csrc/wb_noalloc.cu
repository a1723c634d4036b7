// No-allocation entry point of the transfer kernel (declared in wb_noalloc.h, which explains
// which callers need it).  It launches the same transfer kernel as the regular path, with
// every piece of device-side state the launch needs placed in one file-scope scratch array.
#include "wb_noalloc.h"

#include <cuda_runtime.h>

#include <mutex>

#include "wb_common.h"
#include "wb_transfer.h"

namespace {

// Scratch layout (bytes):
//   [0, 4)     completion counter (cleared by every call)
//   [8, 16)    epoch published to the flags
//   [256, ...) flag-address table, WB_NOALLOC_MAX_FLAGS x 8 bytes
//   [kItems..) work items, WB_NOALLOC_MAX_ITEMS x sizeof(wb::Item)
constexpr size_t kCounterOff = 0;
constexpr size_t kEpochOff = 8;
constexpr size_t kFlagsOff = 256;
constexpr size_t kItemsOff = kFlagsOff + 8 * WB_NOALLOC_MAX_FLAGS;
constexpr size_t kScratchBytes = kItemsOff + sizeof(wb::Item) * WB_NOALLOC_MAX_ITEMS;
static_assert(kItemsOff % 16 == 0, "items must be 16-byte aligned");

constexpr int kMaxDevices = 64;
std::mutex g_mu;
unsigned char* g_scratch_ptr[kMaxDevices] = {};  // device address of the array, per device

}  // namespace

static __device__ __align__(256) unsigned char g_wb_noalloc_scratch[kScratchBytes];

// Device address of the scratch array on the current device (looked up once per device).
static cudaError_t scratch_on_current_device(unsigned char** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_mu);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_wb_noalloc_scratch);
    if (e != cudaSuccess) return e;
    g_scratch_ptr[dev] = static_cast<unsigned char*>(p);
  }
  *out = g_scratch_ptr[dev];
  return cudaSuccess;
}

extern "C" __attribute__((visibility("default"))) int wb_transfer_noalloc(
    const void* host_items, uint32_t n_items, const uint64_t* host_flag_addrs, uint32_t n_flags, uint64_t epoch,
    uint32_t* status, cudaStream_t stream) {
  if (n_items > WB_NOALLOC_MAX_ITEMS) return WB_NOALLOC_ERR_TOO_MANY_ITEMS;
  if (n_flags > WB_NOALLOC_MAX_FLAGS) return WB_NOALLOC_ERR_TOO_MANY_FLAGS;
  if ((n_items && host_items == nullptr) || (n_flags && host_flag_addrs == nullptr))
    return WB_NOALLOC_ERR_NULL_ARGUMENT;

  unsigned char* s = nullptr;
  cudaError_t e = scratch_on_current_device(&s);
  if (e != cudaSuccess) return static_cast<int>(e);

  // The counter must start at zero; the rest is overwritten for this call.  Host sources are
  // pageable: cudaMemcpyAsync has staged them before it returns, so stack values are fine.
  e = cudaMemsetAsync(s + kCounterOff, 0, 8, stream);
  if (e != cudaSuccess) return static_cast<int>(e);
  e = cudaMemcpyAsync(s + kEpochOff, &epoch, sizeof(epoch), cudaMemcpyHostToDevice, stream);
  if (e != cudaSuccess) return static_cast<int>(e);
  if (n_flags) {
    e = cudaMemcpyAsync(s + kFlagsOff, host_flag_addrs, 8u * n_flags, cudaMemcpyHostToDevice, stream);
    if (e != cudaSuccess) return static_cast<int>(e);
  }
  if (n_items) {
    e = cudaMemcpyAsync(s + kItemsOff, host_items, sizeof(wb::Item) * n_items, cudaMemcpyHostToDevice, stream);
    if (e != cudaSuccess) return static_cast<int>(e);
  }

  int dev = 0, sms = 0;
  e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return static_cast<int>(e);
  e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return static_cast<int>(e);
  int grid = sms * 4;
  if (n_items > 0 && static_cast<uint32_t>(grid) > n_items) grid = static_cast<int>(n_items);
  if (grid < 1) grid = 1;

  wb::TransferArgs a{};
  a.items = reinterpret_cast<const wb::Item*>(s + kItemsOff);
  a.n_items = n_items;
  a.piece_bytes = 16384;
  a.mbar_spin_limit = 1u << 26;
  a.sig.counter = reinterpret_cast<uint32_t*>(s + kCounterOff);
  a.sig.flag_addrs = reinterpret_cast<const uint64_t*>(s + kFlagsOff);
  a.sig.n_flags = n_flags;
  a.sig.epoch = reinterpret_cast<const uint64_t*>(s + kEpochOff);
  a.sig.status = status;
  return static_cast<int>(wb::launch_transfer(a, /*mode=*/0, grid, stream));
}
