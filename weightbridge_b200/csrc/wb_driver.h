// Driver-API entry points resolved at run time with cudaGetDriverEntryPointByVersion, so the
// extension links only against the CUDA runtime and imports on machines without a GPU driver.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

#include <stdexcept>
#include <string>

namespace wb {
namespace drv {

// The ABI version every entry point is requested at: the one of the cuda.h these typedefs
// were written against.  (A symbol newer than the requested version - the multicast API is
// 12.1 - is reported as not found.)
constexpr unsigned kDriverAbi = CUDA_VERSION;

template <typename F>
F entry(const char* name) {
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
  cudaError_t e = cudaGetDriverEntryPointByVersion(name, &fn, kDriverAbi, cudaEnableDefault, &q);
  if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || fn == nullptr)
    throw std::runtime_error(std::string("driver entry point unavailable: ") + name);
  return reinterpret_cast<F>(fn);
}

inline void check(CUresult r, const char* what) {
  if (r == CUDA_SUCCESS) return;
  using GetErr = CUresult (*)(CUresult, const char**);
  const char* msg = nullptr;
  try {
    entry<GetErr>("cuGetErrorString")(r, &msg);
  } catch (...) {
  }
  throw std::runtime_error(std::string(what) + ": CUresult " + std::to_string((int)r) + (msg ? std::string(" ") + msg : ""));
}

}  // namespace drv
}  // namespace wb
