// No-allocation entry point of the transfer kernel (declared in wb_noalloc.h, which explains
// which callers need it).  It launches the same transfer kernel as the regular path, with
// every piece of device-side state the launch needs placed in one file-scope scratch array.
#include "wb_noalloc.h"

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstring>
#include <mutex>

#include "wb_common.h"
#include "wb_transfer.h"

namespace {

// Scratch layout (bytes), identical on the host staging block and on the device array:
//   [0, 8)     completion counter (the kernel reads the low 4 bytes; zero in every call)
//   [8, 16)    epoch published to the flags
//   [256, ...) flag-address table, WB_NOALLOC_MAX_FLAGS x 8 bytes
//   [kItems..) work items, WB_NOALLOC_MAX_ITEMS x sizeof(wb::Item)
constexpr size_t kCounterOff = 0;
constexpr size_t kEpochOff = 8;
constexpr size_t kFlagsOff = 256;
constexpr size_t kItemsOff = kFlagsOff + 8 * WB_NOALLOC_MAX_FLAGS;
constexpr size_t kScratchBytes = kItemsOff + sizeof(wb::Item) * WB_NOALLOC_MAX_ITEMS;
static_assert(kItemsOff % 16 == 0, "items must be 16-byte aligned");

// One call at a time stages its arguments here (ordinary pageable host memory owned by the
// library, so cudaMemcpyAsync has copied it out before it returns, whatever kind of memory the
// caller's arrays are in) and then issues one host-to-device copy of the used prefix.
std::mutex g_mu;
alignas(256) unsigned char g_host_stage[kScratchBytes];

// Cached device address of the scratch array, per (device, context).
constexpr int kMaxCached = 64;
struct Cached {
  int device;
  void* ctx;
  unsigned char* ptr;
};
Cached g_cache[kMaxCached];
int g_cached = 0;

using CtxGetCurrent = CUresult (*)(CUcontext*);

// The current driver context, resolved through the runtime's driver entry-point query so this
// file links against the CUDA runtime only.  nullptr when the query is unavailable.
void* current_context() {
  static CtxGetCurrent fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &p, CUDA_VERSION, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      p = nullptr;
    return reinterpret_cast<CtxGetCurrent>(p);
  }();
  CUcontext c = nullptr;
  if (fn == nullptr || fn(&c) != CUDA_SUCCESS) return nullptr;
  return c;
}

}  // namespace

static __device__ __align__(256) unsigned char g_wb_noalloc_scratch[kScratchBytes];

// Device address of the scratch array in the current device's current context (looked up
// once per device and context; the caller holds g_mu).
static cudaError_t scratch_on_current_device(unsigned char** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  void* ctx = current_context();
  for (int i = 0; i < g_cached; ++i) {
    if (g_cache[i].device == dev && g_cache[i].ctx == ctx) {
      *out = g_cache[i].ptr;
      return cudaSuccess;
    }
  }
  void* p = nullptr;
  e = cudaGetSymbolAddress(&p, g_wb_noalloc_scratch);
  if (e != cudaSuccess) return e;
  if (g_cached < kMaxCached) g_cache[g_cached++] = Cached{dev, ctx, static_cast<unsigned char*>(p)};
  *out = static_cast<unsigned char*>(p);
  return cudaSuccess;
}

extern "C" __attribute__((visibility("default"))) int wb_transfer_noalloc(
    const void* host_items, uint32_t n_items, const uint64_t* host_flag_addrs, uint32_t n_flags, uint64_t epoch,
    uint32_t* status, cudaStream_t stream) {
  if (n_items > WB_NOALLOC_MAX_ITEMS) return WB_NOALLOC_ERR_TOO_MANY_ITEMS;
  if (n_flags > WB_NOALLOC_MAX_FLAGS) return WB_NOALLOC_ERR_TOO_MANY_FLAGS;
  if ((n_items && host_items == nullptr) || (n_flags && host_flag_addrs == nullptr))
    return WB_NOALLOC_ERR_NULL_ARGUMENT;

  std::lock_guard<std::mutex> lock(g_mu);
  unsigned char* s = nullptr;
  cudaError_t e = scratch_on_current_device(&s);
  if (e != cudaSuccess) return static_cast<int>(e);

  // Stage everything into the library's host block, then one copy of the used prefix: the
  // counter goes down as zero, the epoch, flag table and items after it.
  std::memset(g_host_stage, 0, kFlagsOff);
  std::memcpy(g_host_stage + kEpochOff, &epoch, sizeof(epoch));
  if (n_flags) std::memcpy(g_host_stage + kFlagsOff, host_flag_addrs, 8u * n_flags);
  if (n_items) std::memcpy(g_host_stage + kItemsOff, host_items, sizeof(wb::Item) * n_items);
  const size_t used = kItemsOff + sizeof(wb::Item) * n_items;
  e = cudaMemcpyAsync(s, g_host_stage, used, cudaMemcpyHostToDevice, stream);
  if (e != cudaSuccess) return static_cast<int>(e);

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
