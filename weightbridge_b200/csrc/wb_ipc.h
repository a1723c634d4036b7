// Cross-process GPU memory helpers (wb_ipc.cpp).
#pragma once
#include <cstddef>
#include <cstdint>
#include <string>

namespace wb {

struct AddrRange {
  uint64_t base;
  uint64_t size;
};

struct VmmAlloc {
  uint64_t ptr;
  uint64_t size;
  uint64_t handle;  // CUmemGenericAllocationHandle
};

AddrRange addr_range(uint64_t ptr);
std::string ipc_handle(uint64_t base);
uint64_t ipc_open(const std::string& handle);
void ipc_close(uint64_t ptr);
std::string device_uuid(int device);
bool can_access_peer(int a, int b);
void enable_peer_access(int peer);

uint64_t vmm_granularity(int device, bool multicast);
VmmAlloc vmm_alloc(size_t size, int device);
int vmm_export_fd(uint64_t handle);
VmmAlloc vmm_import_fd(int fd, size_t size, int device);
void vmm_free(const VmmAlloc& a);

bool multicast_supported(int device);
uint64_t mc_create(size_t size, int num_devices);
uint64_t mc_import_fd(int fd);
void mc_add_device(uint64_t mc, int device);
void mc_bind_mem(uint64_t mc, size_t mc_offset, uint64_t mem_handle, size_t mem_offset, size_t size);
void mc_unbind(uint64_t mc, int device, size_t mc_offset, size_t size);
VmmAlloc mc_map(uint64_t mc, size_t size, int device);
void mem_release(uint64_t handle);
void va_unmap(uint64_t ptr, size_t size);

}  // namespace wb
