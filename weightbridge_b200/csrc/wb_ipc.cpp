// Cross-process GPU memory: CUDA IPC for caching-allocator tensors, VMM allocations that
// export POSIX file descriptors, and NVLink multicast objects for one-to-many fan-out.
//
// Driver-API entry points are resolved at run time with cudaGetDriverEntryPointByVersion,
// so the extension links only against the CUDA runtime and imports on machines without a
// GPU driver.
#include "wb_ipc.h"
#include "wb_driver.h"

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstring>
#include <mutex>
#include <stdexcept>
#include <string>

namespace wb {
namespace {

void check_rt(cudaError_t e, const char* what) {
  if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

using drv::entry;

void check_drv(CUresult r, const char* what) { drv::check(r, what); }

}  // namespace

AddrRange addr_range(uint64_t ptr) {
  using Fn = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);
  static Fn fn = entry<Fn>("cuMemGetAddressRange");
  CUdeviceptr base = 0;
  size_t size = 0;
  check_drv(fn(&base, &size, (CUdeviceptr)ptr), "cuMemGetAddressRange");
  return AddrRange{(uint64_t)base, (uint64_t)size};
}

std::string ipc_handle(uint64_t base) {
  cudaIpcMemHandle_t h;
  check_rt(cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base)), "cudaIpcGetMemHandle");
  return std::string(reinterpret_cast<const char*>(&h), sizeof(h));
}

uint64_t ipc_open(const std::string& handle) {
  if (handle.size() != sizeof(cudaIpcMemHandle_t)) throw std::invalid_argument("bad IPC handle size");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle.data(), sizeof(h));
  void* p = nullptr;
  check_rt(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
  return reinterpret_cast<uint64_t>(p);
}

void ipc_close(uint64_t ptr) { check_rt(cudaIpcCloseMemHandle(reinterpret_cast<void*>(ptr)), "cudaIpcCloseMemHandle"); }

std::string device_uuid(int device) {
  cudaDeviceProp prop;
  check_rt(cudaGetDeviceProperties(&prop, device), "cudaGetDeviceProperties");
  return std::string(prop.uuid.bytes, sizeof(prop.uuid.bytes));
}

bool can_access_peer(int a, int b) {
  if (a == b) return true;
  int ok = 0;
  check_rt(cudaDeviceCanAccessPeer(&ok, a, b), "cudaDeviceCanAccessPeer");
  return ok != 0;
}

void enable_peer_access(int peer) {
  cudaError_t e = cudaDeviceEnablePeerAccess(peer, 0);
  if (e == cudaErrorPeerAccessAlreadyEnabled) {
    cudaGetLastError();
    return;
  }
  check_rt(e, "cudaDeviceEnablePeerAccess");
}

// ---------------------------------------------------------------------------------------
// VMM allocations exported as POSIX file descriptors
// ---------------------------------------------------------------------------------------
namespace {
CUmemAllocationProp vmm_prop(int device, bool multicast_ready) {
  CUmemAllocationProp p;
  std::memset(&p, 0, sizeof(p));
  p.type = CU_MEM_ALLOCATION_TYPE_PINNED;
  p.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
  p.location.id = device;
  p.requestedHandleTypes = CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR;
  (void)multicast_ready;
  return p;
}

void map_rw(CUdeviceptr va, size_t size, int device) {
  using SetAccess = CUresult (*)(CUdeviceptr, size_t, const CUmemAccessDesc*, size_t);
  static SetAccess set_access = entry<SetAccess>("cuMemSetAccess");
  CUmemAccessDesc acc;
  std::memset(&acc, 0, sizeof(acc));
  acc.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
  acc.location.id = device;
  acc.flags = CU_MEM_ACCESS_FLAGS_PROT_READWRITE;
  check_drv(set_access(va, size, &acc, 1), "cuMemSetAccess");
}
}  // namespace

uint64_t vmm_granularity(int device, bool multicast) {
  if (multicast) {
    using Fn = CUresult (*)(size_t*, const CUmulticastObjectProp*, CUmulticastGranularity_flags);
    static Fn fn = entry<Fn>("cuMulticastGetGranularity");
    CUmulticastObjectProp mp;
    std::memset(&mp, 0, sizeof(mp));
    mp.numDevices = 1;
    mp.size = 1;
    mp.handleTypes = CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR;
    size_t g = 0;
    check_drv(fn(&g, &mp, CU_MULTICAST_GRANULARITY_RECOMMENDED), "cuMulticastGetGranularity");
    return g;
  }
  using Fn = CUresult (*)(size_t*, const CUmemAllocationProp*, CUmemAllocationGranularity_flags);
  static Fn fn = entry<Fn>("cuMemGetAllocationGranularity");
  CUmemAllocationProp p = vmm_prop(device, false);
  size_t g = 0;
  check_drv(fn(&g, &p, CU_MEM_ALLOC_GRANULARITY_RECOMMENDED), "cuMemGetAllocationGranularity");
  return g;
}

VmmAlloc vmm_alloc(size_t size, int device) {
  using Create = CUresult (*)(CUmemGenericAllocationHandle*, size_t, const CUmemAllocationProp*, unsigned long long);
  using Reserve = CUresult (*)(CUdeviceptr*, size_t, size_t, CUdeviceptr, unsigned long long);
  using Map = CUresult (*)(CUdeviceptr, size_t, size_t, CUmemGenericAllocationHandle, unsigned long long);
  static Create create = entry<Create>("cuMemCreate");
  static Reserve reserve = entry<Reserve>("cuMemAddressReserve");
  static Map map = entry<Map>("cuMemMap");
  const size_t g = vmm_granularity(device, false);
  size = (size + g - 1) / g * g;
  CUmemAllocationProp p = vmm_prop(device, false);
  CUmemGenericAllocationHandle h = 0;
  check_drv(create(&h, size, &p, 0), "cuMemCreate");
  CUdeviceptr va = 0;
  check_drv(reserve(&va, size, g, 0, 0), "cuMemAddressReserve");
  check_drv(map(va, size, 0, h, 0), "cuMemMap");
  map_rw(va, size, device);
  return VmmAlloc{(uint64_t)va, (uint64_t)size, (uint64_t)h};
}

int vmm_export_fd(uint64_t handle) {
  using Fn = CUresult (*)(void*, CUmemGenericAllocationHandle, CUmemAllocationHandleType, unsigned long long);
  static Fn fn = entry<Fn>("cuMemExportToShareableHandle");
  int fd = -1;
  check_drv(fn(&fd, (CUmemGenericAllocationHandle)handle, CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR, 0),
            "cuMemExportToShareableHandle");
  return fd;
}

VmmAlloc vmm_import_fd(int fd, size_t size, int device) {
  using Import = CUresult (*)(CUmemGenericAllocationHandle*, void*, CUmemAllocationHandleType);
  using Reserve = CUresult (*)(CUdeviceptr*, size_t, size_t, CUdeviceptr, unsigned long long);
  using Map = CUresult (*)(CUdeviceptr, size_t, size_t, CUmemGenericAllocationHandle, unsigned long long);
  static Import imp = entry<Import>("cuMemImportFromShareableHandle");
  static Reserve reserve = entry<Reserve>("cuMemAddressReserve");
  static Map map = entry<Map>("cuMemMap");
  CUmemGenericAllocationHandle h = 0;
  check_drv(imp(&h, reinterpret_cast<void*>(static_cast<intptr_t>(fd)), CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR),
            "cuMemImportFromShareableHandle");
  const size_t g = vmm_granularity(device, false);
  CUdeviceptr va = 0;
  check_drv(reserve(&va, size, g, 0, 0), "cuMemAddressReserve");
  check_drv(map(va, size, 0, h, 0), "cuMemMap");
  map_rw(va, size, device);
  return VmmAlloc{(uint64_t)va, (uint64_t)size, (uint64_t)h};
}

void vmm_free(const VmmAlloc& a) {
  using Unmap = CUresult (*)(CUdeviceptr, size_t);
  using Free = CUresult (*)(CUdeviceptr, size_t);
  using Release = CUresult (*)(CUmemGenericAllocationHandle);
  static Unmap unmap = entry<Unmap>("cuMemUnmap");
  static Free afree = entry<Free>("cuMemAddressFree");
  static Release release = entry<Release>("cuMemRelease");
  check_drv(unmap((CUdeviceptr)a.ptr, a.size), "cuMemUnmap");
  check_drv(afree((CUdeviceptr)a.ptr, a.size), "cuMemAddressFree");
  check_drv(release((CUmemGenericAllocationHandle)a.handle), "cuMemRelease");
}

// ---------------------------------------------------------------------------------------
// NVLink multicast objects
// ---------------------------------------------------------------------------------------
bool multicast_supported(int device) {
  using Fn = CUresult (*)(int*, CUdevice_attribute, CUdevice);
  static Fn fn = entry<Fn>("cuDeviceGetAttribute");
  int v = 0;
  check_drv(fn(&v, CU_DEVICE_ATTRIBUTE_MULTICAST_SUPPORTED, (CUdevice)device), "cuDeviceGetAttribute");
  return v != 0;
}

uint64_t mc_create(size_t size, int num_devices) {
  using Fn = CUresult (*)(CUmemGenericAllocationHandle*, const CUmulticastObjectProp*);
  static Fn fn = entry<Fn>("cuMulticastCreate");
  CUmulticastObjectProp mp;
  std::memset(&mp, 0, sizeof(mp));
  mp.numDevices = (unsigned)num_devices;
  mp.size = size;
  mp.handleTypes = CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR;
  CUmemGenericAllocationHandle h = 0;
  check_drv(fn(&h, &mp), "cuMulticastCreate");
  return (uint64_t)h;
}

uint64_t mc_import_fd(int fd) {
  using Import = CUresult (*)(CUmemGenericAllocationHandle*, void*, CUmemAllocationHandleType);
  static Import imp = entry<Import>("cuMemImportFromShareableHandle");
  CUmemGenericAllocationHandle h = 0;
  check_drv(imp(&h, reinterpret_cast<void*>(static_cast<intptr_t>(fd)), CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR),
            "cuMemImportFromShareableHandle(multicast)");
  return (uint64_t)h;
}

void mc_add_device(uint64_t mc, int device) {
  using Fn = CUresult (*)(CUmemGenericAllocationHandle, CUdevice);
  static Fn fn = entry<Fn>("cuMulticastAddDevice");
  check_drv(fn((CUmemGenericAllocationHandle)mc, (CUdevice)device), "cuMulticastAddDevice");
}

void mc_bind_mem(uint64_t mc, size_t mc_offset, uint64_t mem_handle, size_t mem_offset, size_t size) {
  using Fn = CUresult (*)(CUmemGenericAllocationHandle, size_t, CUmemGenericAllocationHandle, size_t, size_t,
                          unsigned long long);
  static Fn fn = entry<Fn>("cuMulticastBindMem");
  check_drv(fn((CUmemGenericAllocationHandle)mc, mc_offset, (CUmemGenericAllocationHandle)mem_handle, mem_offset,
               size, 0),
            "cuMulticastBindMem");
}

void mc_unbind(uint64_t mc, int device, size_t mc_offset, size_t size) {
  using Fn = CUresult (*)(CUmemGenericAllocationHandle, CUdevice, size_t, size_t);
  static Fn fn = entry<Fn>("cuMulticastUnbind");
  check_drv(fn((CUmemGenericAllocationHandle)mc, (CUdevice)device, mc_offset, size), "cuMulticastUnbind");
}

void mem_release(uint64_t handle) {
  using Fn = CUresult (*)(CUmemGenericAllocationHandle);
  static Fn fn = entry<Fn>("cuMemRelease");
  check_drv(fn((CUmemGenericAllocationHandle)handle), "cuMemRelease");
}

void va_unmap(uint64_t ptr, size_t size) {
  using Unmap = CUresult (*)(CUdeviceptr, size_t);
  using Free = CUresult (*)(CUdeviceptr, size_t);
  static Unmap unmap = entry<Unmap>("cuMemUnmap");
  static Free afree = entry<Free>("cuMemAddressFree");
  check_drv(unmap((CUdeviceptr)ptr, size), "cuMemUnmap");
  check_drv(afree((CUdeviceptr)ptr, size), "cuMemAddressFree");
}

VmmAlloc mc_map(uint64_t mc, size_t size, int device) {
  using Reserve = CUresult (*)(CUdeviceptr*, size_t, size_t, CUdeviceptr, unsigned long long);
  using Map = CUresult (*)(CUdeviceptr, size_t, size_t, CUmemGenericAllocationHandle, unsigned long long);
  static Reserve reserve = entry<Reserve>("cuMemAddressReserve");
  static Map map = entry<Map>("cuMemMap");
  const size_t g = vmm_granularity(device, true);
  CUdeviceptr va = 0;
  check_drv(reserve(&va, size, g, 0, 0), "cuMemAddressReserve(multicast)");
  check_drv(map(va, size, 0, (CUmemGenericAllocationHandle)mc, 0), "cuMemMap(multicast)");
  map_rw(va, size, device);
  return VmmAlloc{(uint64_t)va, (uint64_t)size, mc};
}

}  // namespace wb
