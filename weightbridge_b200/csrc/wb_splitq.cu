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
// One CTA per piece.  A piece with 16-bit source, a multiple of 16 columns and 16-byte aligned
// rows (expert-TP or FSDP slices cutting block rows or columns) takes the vector path of the
// transfer kernel's quant blocks: cols / 16 threads span a row, 32-byte loads, 16-byte stores;
// other pieces go element by element.  Nothing waits on another kernel or rank.
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

__device__ __forceinline__ uint4 ld16(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}

__device__ __forceinline__ void st16(void* p, uint4 v) {
  asm volatile("st.global.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w) : "memory");
}

// The vector path: 16-bit source, a multiple of 16 columns (at most 128), 16-byte aligned rows
// on both sides.  cols / 16 threads span a row (32 source bytes, 16 e4m3 bytes each).
__device__ __forceinline__ bool vec_ok(const SplitPiece& p) {
  return (p.src_code == DT_BF16 || p.src_code == DT_F16) && p.cols % 16 == 0 && p.cols >= 16 && p.cols <= 128 &&
         ((p.src | p.dst | (uint64_t)p.src_pitch | (uint64_t)p.dst_pitch) & 15) == 0;
}

__device__ __forceinline__ float2 unpack2(uint32_t w, bool bf16) {
  if (bf16) return __bfloat1622float2(*reinterpret_cast<__nv_bfloat162*>(&w));
  return __half22float2(*reinterpret_cast<__half2*>(&w));
}

// max |x| of 8 packed 16-bit values
__device__ __forceinline__ float amax8(const uint4 v, bool bf16) {
  float m = 0.f;
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
  #pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 f = unpack2(w[j], bf16);
    m = fmaxf(m, fmaxf(fabsf(f.x), fabsf(f.y)));
  }
  return m;
}

__device__ __forceinline__ uint32_t pack4(float a, float b, float c, float d, float inv) {
  const __nv_fp8x2_storage_t lo =
      __nv_cvt_float2_to_fp8x2(make_float2(__fmul_rn(a, inv), __fmul_rn(b, inv)), __NV_SATFINITE, __NV_E4M3);
  const __nv_fp8x2_storage_t hi =
      __nv_cvt_float2_to_fp8x2(make_float2(__fmul_rn(c, inv), __fmul_rn(d, inv)), __NV_SATFINITE, __NV_E4M3);
  return (uint32_t)lo | ((uint32_t)hi << 16);
}

// 8 source values -> 8 e4m3 bytes
__device__ __forceinline__ uint2 quant8(const uint4 v, bool bf16, float inv) {
  const float2 a = unpack2(v.x, bf16), b = unpack2(v.y, bf16), c = unpack2(v.z, bf16), e = unpack2(v.w, bf16);
  return make_uint2(pack4(a.x, a.y, b.x, b.y, inv), pack4(c.x, c.y, e.x, e.y, inv));
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
    float m = 0.f;
    if (vec_ok(p)) {
      const bool bf16 = p.src_code == DT_BF16;
      const uint32_t tpr = p.cols / 16, rpp = kThreads / tpr;    // threads per row, rows per pass
      if (threadIdx.x < tpr * rpp) {
        const uint32_t col = threadIdx.x % tpr;
        for (uint32_t r = threadIdx.x / tpr; r < p.rows; r += rpp) {
          const uint8_t* q = src + (int64_t)r * p.src_pitch + col * 32u;
          m = fmaxf(m, fmaxf(amax8(ld16(q), bf16), amax8(ld16(q + 16), bf16)));
        }
      }
    } else {
      const uint32_t total = es ? p.rows * p.cols : 0u;
      for (uint32_t k = threadIdx.x; k < total; k += kThreads) {
        const uint32_t r = k / p.cols, c = k - r * p.cols;
        m = fmaxf(m, fabsf(load_f32(src + (int64_t)r * p.src_pitch + (uint64_t)c * es, p.src_code)));
      }
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
    if (vec_ok(p)) {
      const bool bf16 = p.src_code == DT_BF16;
      const uint32_t tpr = p.cols / 16, rpp = kThreads / tpr;
      if (threadIdx.x < tpr * rpp) {
        const uint32_t col = threadIdx.x % tpr;
        for (uint32_t r = threadIdx.x / tpr; r < p.rows; r += rpp) {
          const uint8_t* q = src + (int64_t)r * p.src_pitch + col * 32u;
          const uint2 lo = quant8(ld16(q), bf16, inv), hi = quant8(ld16(q + 16), bf16, inv);
          st16(dst + (int64_t)r * p.dst_pitch + col * 16u, make_uint4(lo.x, lo.y, hi.x, hi.y));
        }
      }
    } else {
      const uint32_t total = p.rows * p.cols;
      for (uint32_t k = threadIdx.x; k < total; k += kThreads) {
        const uint32_t r = k / p.cols, c = k - r * p.cols;
        const float x = load_f32(src + (int64_t)r * p.src_pitch + (uint64_t)c * es, p.src_code);
        dst[(int64_t)r * p.dst_pitch + c] = __nv_cvt_float_to_fp8(__fmul_rn(x, inv), __NV_SATFINITE, __NV_E4M3);
      }
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
