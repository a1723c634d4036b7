// Synthetic N(0, std) weights written straight into (strided) parameter views on the GPU.
//
// The value of every element depends only on (tensor key, flat logical index in the full HF
// tensor): a 32-bit integer mixing hash of the index gives two uniforms, and the Box-Muller
// transform turns them into a normal sample.  The arithmetic is done in double precision in
// the same order as the PyTorch restatement in weightbridge_b200/models/synthetic.py
// (synth_values), and the result is rounded double -> float -> target type as PyTorch's
// conversion does, so the kernel writes exactly what that code writes on a CUDA device.  One
// launch fills one view of any rank up to kMaxDims, replacing the dozens of elementwise
// launches per chunk of the tensor-op version.
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cstdint>

#include "wb_common.h"
#include "wb_synth.h"

namespace wb {

namespace {

__device__ __forceinline__ uint64_t mix32(uint64_t x) {
  constexpr uint64_t kM = 0x45D9F3Bull, kMask = 0xFFFFFFFFull;
  x = (((x >> 16) ^ x) * kM) & kMask;
  x = (((x >> 16) ^ x) * kM) & kMask;
  return (x >> 16) ^ x;
}

__device__ __forceinline__ double synth_value(uint64_t lidx, uint64_t key, double std) {
  const uint64_t hi = mix32((lidx >> 32) ^ key);
  const uint64_t h1 = mix32((lidx & 0xFFFFFFFFull) ^ hi);
  const uint64_t h2 = mix32(h1 ^ 0x68E31DA4ull);
  const double u1 = ((double)h1 + 1.0) / 4294967297.0;
  const double u2 = (double)h2 / 4294967296.0;
  const double two_pi = 6.283185307179586;     // the double nearest 2 pi (Python's 2.0 * math.pi)
  const double z = sqrt(-2.0 * log(u1)) * cos(two_pi * u2);
  return z * std;
}

__global__ void synth_fill_kernel(SynthDesc d, uint64_t n) {
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    uint64_t rem = i;
    int64_t off = 0;
    uint64_t lidx = 0;
    for (int k = d.ndim - 1; k >= 0; --k) {
      const uint64_t e = (uint64_t)d.ext[k];
      const uint64_t c = k ? rem % e : rem;
      rem = k ? rem / e : 0;
      off += (int64_t)c * d.vstride[k];
      lidx += (uint64_t)(d.lo[k] + (int64_t)c) * (uint64_t)d.lstride[k];
    }
    const double v = synth_value(lidx, d.key, d.std);
    switch (d.dtype) {
      case DT_F32: reinterpret_cast<float*>(d.dst)[off] = (float)v; break;
      case DT_BF16: reinterpret_cast<__nv_bfloat16*>(d.dst)[off] = __float2bfloat16_rn((float)v); break;
      case DT_F16: reinterpret_cast<__half*>(d.dst)[off] = __float2half_rn((float)v); break;
      case DT_F64: reinterpret_cast<double*>(d.dst)[off] = v; break;
      default: break;
    }
  }
}

}  // namespace

bool synth_dtype_supported(uint32_t code) {
  return code == DT_F32 || code == DT_BF16 || code == DT_F16 || code == DT_F64;
}

cudaError_t launch_synth_fill(const SynthDesc& d, cudaStream_t stream) {
  if (d.ndim < 1 || d.ndim > kSynthMaxDims || !synth_dtype_supported(d.dtype)) return cudaErrorInvalidValue;
  uint64_t n = 1;
  for (int k = 0; k < d.ndim; ++k) {
    if (d.ext[k] < 0) return cudaErrorInvalidValue;
    n *= (uint64_t)d.ext[k];
  }
  if (n == 0) return cudaSuccess;
  int dev = 0, sms = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return e;
  constexpr int kThreadsPerBlock = 256;
  const uint64_t blocks_needed = (n + kThreadsPerBlock - 1) / kThreadsPerBlock;
  const uint64_t cap = (uint64_t)sms * 8;
  const int grid = (int)(blocks_needed < cap ? blocks_needed : cap);
  synth_fill_kernel<<<grid, kThreadsPerBlock, 0, stream>>>(d, n);
  return cudaGetLastError();
}

}  // namespace wb
