// Split-block fp8 quantisation (sm_100a).
//
// A 128 x 128 block of a block-quantised destination whose rows or columns come from several
// senders cannot be quantised by any one of them: the scale needs the whole block's amax.
// Each sender runs split_amax over its parts (pieces) of such blocks, the senders exchange
// the per-block maxima through the host session, and each then runs split_quant, which
// quantises its pieces with the common amax and writes the block's scale (every sender of
// the block writes the same value).  The arithmetic matches the transfer kernel's quant
// path: scale = amax / 448 (IEEE division), inv = RN(1 / scale), q = satfinite_e4m3(x * inv).
//
// Pieces are a small share of a sync (the fringe rows or columns of a shard), so these are
// plain one-CTA-per-piece kernels with element loads and stores; nothing waits on another
// kernel or rank.
#include "wb_splitq.h"

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>

namespace wb {
namespace {

constexpr int kThreads = 256;

__device__ __forceinline__ uint32_t code_bytes(uint32_t c) {
  return c == DT_F32 ? 4u : (c == DT_BF16 || c == DT_F16) ? 2u : 0u;
}

__device__ __forceinline__ float load_f32(const uint8_t* p, uint32_t c) {
  if (c == DT_F32) return *reinterpret_cast<const float*>(p);
  if (c == DT_BF16) return __bfloat162float(*reinterpret_cast<const __nv_bfloat16*>(p));
  return __half2float(*reinterpret_cast<const __half*>(p));
}

__device__ __forceinline__ float cta_max(float v, float* red) {
  #pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();  // red[] may still be read for the previous piece
  if (l == 0) red[w] = v;
  __syncthreads();
  if (w == 0) {
    float x = l < (kThreads >> 5) ? red[l] : 0.f;
    #pragma unroll
    for (int o = 16; o > 0; o >>= 1) x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, o));
    if (l == 0) red[32] = x;
  }
  __syncthreads();
  return red[32];
}

__global__ void __launch_bounds__(kThreads) split_amax_kernel(const SplitPiece* __restrict__ pieces, uint32_t n,
                                                              float* __restrict__ partial) {
  __shared__ float red[33];
  for (uint32_t i = blockIdx.x; i < n; i += gridDim.x) {
    const SplitPiece p = pieces[i];
    const uint32_t es = code_bytes(p.src_code);
    const uint8_t* src = reinterpret_cast<const uint8_t*>(p.src);
    const uint32_t total = es ? p.rows * p.cols : 0u;
    float m = 0.f;
    for (uint32_t k = threadIdx.x; k < total; k += kThreads) {
      const uint32_t r = k / p.cols, c = k - r * p.cols;
      m = fmaxf(m, fabsf(load_f32(src + (int64_t)r * p.src_pitch + (uint64_t)c * es, p.src_code)));
    }
    m = cta_max(m, red);
    if (threadIdx.x == 0) partial[i] = m;
  }
}

__global__ void __launch_bounds__(kThreads) split_quant_kernel(const SplitPiece* __restrict__ pieces, uint32_t n,
                                                               const float* __restrict__ amax) {
  for (uint32_t i = blockIdx.x; i < n; i += gridDim.x) {
    const SplitPiece p = pieces[i];
    const uint32_t es = code_bytes(p.src_code);
    if (es == 0) continue;
    const float a = amax[i];
    const float scale = a > 0.f ? __fdiv_rn(a, kE4M3Max) : 1.f;
    const float inv = __frcp_rn(scale);
    const uint8_t* src = reinterpret_cast<const uint8_t*>(p.src);
    uint8_t* dst = reinterpret_cast<uint8_t*>(p.dst);
    const uint32_t total = p.rows * p.cols;
    for (uint32_t k = threadIdx.x; k < total; k += kThreads) {
      const uint32_t r = k / p.cols, c = k - r * p.cols;
      const float x = load_f32(src + (int64_t)r * p.src_pitch + (uint64_t)c * es, p.src_code);
      dst[(int64_t)r * p.dst_pitch + c] = __nv_cvt_float_to_fp8(__fmul_rn(x, inv), __NV_SATFINITE, __NV_E4M3);
    }
    if (threadIdx.x == 0) *reinterpret_cast<float*>(p.scale) = scale;
  }
}

int grid_for(uint32_t n) {
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const uint32_t cap = (uint32_t)sms * 8u;
  return (int)(n < cap ? n : cap);
}

}  // namespace

cudaError_t launch_split_amax(const SplitPiece* pieces, uint32_t n, float* partial, cudaStream_t stream) {
  if (n == 0) return cudaSuccess;
  split_amax_kernel<<<grid_for(n), kThreads, 0, stream>>>(pieces, n, partial);
  return cudaGetLastError();
}

cudaError_t launch_split_quant(const SplitPiece* pieces, uint32_t n, const float* amax, cudaStream_t stream) {
  if (n == 0) return cudaSuccess;
  split_quant_kernel<<<grid_for(n), kThreads, 0, stream>>>(pieces, n, amax);
  return cudaGetLastError();
}

}  // namespace wb
