// sm_100a transfer kernel: one persistent launch walks the plan's work tables and stores
// straight into the destination parameter memory (this GPU, a peer GPU through a CUDA IPC
// mapping, or an NVLink multicast address), then publishes the sync epoch to every
// receiver's flag word.
//
// Three kinds of work share the launch:
//   * generic items  - 2-D strided copies / float casts, all threads, widest aligned vector;
//   * quant blocks   - 128 x 128 bf16/fp16/fp32 -> e4m3 with an fp32 block scale, fused with
//                      the (peer) store of the quantised block and its scale.  In the TMA
//                      modes a block whose matrix has a tensor map arrives in shared memory
//                      with one cp.async.bulk.tensor.2d load (a ring of 32 KiB stages, loads
//                      issued ahead by one thread); others are loaded into registers;
//   * bulk items     - 16-byte aligned copies moved by the TMA engine: one elected thread
//                      streams pieces global -> shared (cp.async.bulk + mbarrier) and
//                      shared -> destination (cp.async.bulk bulk_group), S stages deep.
//                      Bulk loads may read a peer GPU's memory (the pull direction runs
//                      this kernel on the receiver with sources in the sender's IPC
//                      mapping); no load or store here uses .multicast::cluster.
//
// Completion: every CTA fences at system scope and bumps a scratch counter; the last CTA
// writes the epoch with st.release.sys to each flag and resets the counter.  Every wait in
// this file is bounded and reports through the status word instead of trapping.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cstdint>
#include <cstring>

#include "wb_common.h"
#include "wb_driver.h"
#include "wb_transfer.h"

namespace wb {

constexpr int kThreads = 256;     // threads per CTA of the transfer kernel

// ------------------------------------------------------------------------------------
// memory helpers
// ------------------------------------------------------------------------------------
__device__ __forceinline__ uint4 ld_nc16(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}
__device__ __forceinline__ void st16(void* p, uint4 v) {
  asm volatile("st.global.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}
__device__ __forceinline__ void st_mc16(void* p, uint4 v) {
  asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1,%2,%3,%4};" ::"l"(p),
               "f"(__uint_as_float(v.x)), "f"(__uint_as_float(v.y)), "f"(__uint_as_float(v.z)),
               "f"(__uint_as_float(v.w))
               : "memory");
}
__device__ __forceinline__ void st_release_sys(uint64_t* p, uint64_t v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
// release store of a flag word through an NVLink multicast address: every replica's copy of
// the word receives it, ordered after this thread's earlier multimem stores
__device__ __forceinline__ void st_mc_release_sys(uint64_t* p, uint64_t v) {
  asm volatile("multimem.st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t ld_acquire_sys(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

template <int G> struct Vec;
template <> struct Vec<16> { using T = uint4; };
template <> struct Vec<8> { using T = uint2; };
template <> struct Vec<4> { using T = uint32_t; };
template <> struct Vec<2> { using T = uint16_t; };
template <> struct Vec<1> { using T = uint8_t; };

template <int G>
__device__ __forceinline__ typename Vec<G>::T vload(const typename Vec<G>::T* p) {
  if constexpr (G == 16) return ld_nc16(p);
  else return __ldg(p);
}
template <int G>
__device__ __forceinline__ void vstore(typename Vec<G>::T* p, typename Vec<G>::T v) {
  if constexpr (G == 16) st16(p, v);
  else *p = v;
}

// ------------------------------------------------------------------------------------
// generic items: copy
// ------------------------------------------------------------------------------------
template <int G, bool MC>
__device__ __forceinline__ void copy_item(const Item& it) {
  using T = typename Vec<G>::T;
  const uint32_t per_row = it.row_bytes / G;
  const uint32_t n = per_row * it.rows;
  const uint32_t B = blockDim.x;
  const uint8_t* s8 = reinterpret_cast<const uint8_t*>(it.src);
  uint8_t* d8 = reinterpret_cast<uint8_t*>(it.dst);
  auto put = [&](T* p, T v) {
    if constexpr (MC) st_mc16(p, v);
    else vstore<G>(p, v);
  };
  const bool flat = it.rows == 1 || (it.src_pitch == (int64_t)it.row_bytes && it.dst_pitch == (int64_t)it.row_bytes);
  if (flat) {
    const T* s = reinterpret_cast<const T*>(s8);
    T* d = reinterpret_cast<T*>(d8);
    uint32_t i = threadIdx.x;
    for (; i + 3 * B < n; i += 4 * B) {
      T a = vload<G>(s + i), b = vload<G>(s + i + B), c = vload<G>(s + i + 2 * B), e = vload<G>(s + i + 3 * B);
      put(d + i, a); put(d + i + B, b); put(d + i + 2 * B, c); put(d + i + 3 * B, e);
    }
    for (; i < n; i += B) put(d + i, vload<G>(s + i));
    return;
  }
  uint32_t i = threadIdx.x;
  for (; i + B < n; i += 2 * B) {
    const uint32_t r0 = i / per_row, c0 = i - r0 * per_row;
    const uint32_t j = i + B;
    const uint32_t r1 = j / per_row, c1 = j - r1 * per_row;
    T a = vload<G>(reinterpret_cast<const T*>(s8 + r0 * it.src_pitch) + c0);
    T b = vload<G>(reinterpret_cast<const T*>(s8 + r1 * it.src_pitch) + c1);
    put(reinterpret_cast<T*>(d8 + r0 * it.dst_pitch) + c0, a);
    put(reinterpret_cast<T*>(d8 + r1 * it.dst_pitch) + c1, b);
  }
  for (; i < n; i += B) {
    const uint32_t r = i / per_row, c = i - r * per_row;
    put(reinterpret_cast<T*>(d8 + r * it.dst_pitch) + c, vload<G>(reinterpret_cast<const T*>(s8 + r * it.src_pitch) + c));
  }
}

__device__ __forceinline__ int item_granularity(const Item& it) {
  const uint64_t bits = it.src | it.dst | (uint64_t)it.src_pitch | (uint64_t)it.dst_pitch | (uint64_t)it.row_bytes;
  if ((bits & 15) == 0) return 16;
  if ((bits & 7) == 0) return 8;
  if ((bits & 3) == 0) return 4;
  if ((bits & 1) == 0) return 2;
  return 1;
}

// ------------------------------------------------------------------------------------
// generic items: float casts (round to nearest even)
// ------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t dt_size(uint32_t c) {
  return c == DT_F32 ? 4u : (c == DT_BF16 || c == DT_F16) ? 2u : 0u;
}
__device__ __forceinline__ float ld_as_f32(const uint8_t* p, uint32_t c) {
  if (c == DT_F32) return *reinterpret_cast<const float*>(p);
  if (c == DT_BF16) return __bfloat162float(*reinterpret_cast<const __nv_bfloat16*>(p));
  return __half2float(*reinterpret_cast<const __half*>(p));
}
__device__ __forceinline__ void st_from_f32(uint8_t* p, uint32_t c, float v) {
  if (c == DT_F32) *reinterpret_cast<float*>(p) = v;
  else if (c == DT_BF16) *reinterpret_cast<__nv_bfloat16*>(p) = __float2bfloat16_rn(v);
  else *reinterpret_cast<__half*>(p) = __float2half_rn(v);
}

__device__ void cast_item(const Item& it, uint32_t* status) {
  const uint32_t sc = op_src(it.op), dc = op_dst(it.op);
  const uint32_t ss = dt_size(sc), ds = dt_size(dc);
  if (ss == 0 || ds == 0) {
    if (threadIdx.x == 0 && status) atomicOr(status, ST_BAD_ITEM);
    return;
  }
  const uint32_t per_row = it.row_bytes / ss;
  const uint32_t n = per_row * it.rows;
  const uint8_t* s8 = reinterpret_cast<const uint8_t*>(it.src);
  uint8_t* d8 = reinterpret_cast<uint8_t*>(it.dst);
  for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) {
    const uint32_t r = i / per_row, c = i - r * per_row;
    st_from_f32(d8 + r * it.dst_pitch + (uint64_t)c * ds, dc, ld_as_f32(s8 + r * it.src_pitch + (uint64_t)c * ss, sc));
  }
}

// ------------------------------------------------------------------------------------
// generic items: transposes (a destination whose contiguous dimension is the source's rows,
// e.g. MLA's w_kc written from kv_b_proj).  2-byte elements go through a 64 x 64 tile in
// shared memory so that both the loads (along source rows) and the stores (along destination
// rows) are coalesced 128-byte warp accesses; other sizes take an element loop.
// ------------------------------------------------------------------------------------
constexpr int kTp = 64;         // tile edge, elements
constexpr int kTpPitch = 66;    // tile row pitch, elements: 33 words, so the 32-bit writes of a
                                // warp (4 rows x 8 lanes) hit 32 banks and the column reads 2-way

// One 64 x 64 tile of 2-byte elements: each of the 256 threads holds two 16-byte pieces of
// source rows (eight lanes span a 128-byte row segment, a warp four rows), written to shared
// memory as 32-bit words.  Loads of the next tile are issued before the current tile's
// stores, so they overlap.
struct TpRegs {
  uint4 v[2];
};

__device__ __forceinline__ void tp_load(const uint8_t* s8, int64_t pitch, uint32_t R, uint32_t C, uint32_t r0,
                                        uint32_t c0, TpRegs& g) {
  #pragma unroll
  for (int k = 0; k < 2; ++k) {
    const uint32_t idx = threadIdx.x + 256u * k;          // 512 pieces of 8 elements
    const uint32_t r = idx >> 3, c = (idx & 7) * 8;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (r0 + r < R) {
      const uint8_t* p = s8 + (r0 + r) * pitch + (uint64_t)(c0 + c) * 2;
      if (c0 + c + 8 <= C && (reinterpret_cast<uint64_t>(p) & 15) == 0) {
        v = ld_nc16(p);
      } else {
        uint16_t e[8];
        #pragma unroll
        for (int j = 0; j < 8; ++j) e[j] = (c0 + c + j < C) ? __ldg(reinterpret_cast<const uint16_t*>(p) + j) : 0;
        v = make_uint4(e[0] | ((uint32_t)e[1] << 16), e[2] | ((uint32_t)e[3] << 16), e[4] | ((uint32_t)e[5] << 16),
                       e[6] | ((uint32_t)e[7] << 16));
      }
    }
    g.v[k] = v;
  }
}

__device__ void transpose_item(const Item& it, uint16_t* tile, uint32_t* status) {
  const uint32_t es = dtype_bytes(op_src(it.op));
  if (es == 0 || it.row_bytes % es) {
    if (threadIdx.x == 0 && status) atomicOr(status, ST_BAD_ITEM);
    return;
  }
  const uint32_t R = it.rows, C = it.row_bytes / es;
  const uint8_t* s8 = reinterpret_cast<const uint8_t*>(it.src);
  uint8_t* d8 = reinterpret_cast<uint8_t*>(it.dst);
  if (es != 2 || blockDim.x != 256) {
    const uint64_t n = (uint64_t)R * C;
    for (uint64_t i = threadIdx.x; i < n; i += blockDim.x) {
      const uint32_t c = (uint32_t)(i / R), r = (uint32_t)(i - (uint64_t)c * R);   // r fastest: dst rows
      const uint8_t* sp = s8 + r * it.src_pitch + (uint64_t)c * es;
      uint8_t* dp = d8 + c * it.dst_pitch + (uint64_t)r * es;
      for (uint32_t b = 0; b < es; ++b) dp[b] = sp[b];
    }
    return;
  }
  const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint32_t tr = (R + kTp - 1) / kTp, tc = (C + kTp - 1) / kTp, nt = tr * tc;
  TpRegs g;
  tp_load(s8, it.src_pitch, R, C, 0, 0, g);
  for (uint32_t t = 0; t < nt; ++t) {
    const uint32_t r0 = (t / tc) * kTp, c0 = (t % tc) * kTp;
    const uint32_t nr = min((uint32_t)kTp, R - r0), nc = min((uint32_t)kTp, C - c0);
    __syncthreads();                        // the previous tile's stores have read the tile
    #pragma unroll
    for (int k = 0; k < 2; ++k) {
      const uint32_t idx = threadIdx.x + 256u * k;
      uint32_t* w = reinterpret_cast<uint32_t*>(tile + (idx >> 3) * kTpPitch + (idx & 7) * 8);
      w[0] = g.v[k].x;
      w[1] = g.v[k].y;
      w[2] = g.v[k].z;
      w[3] = g.v[k].w;
    }
    __syncthreads();
    if (t + 1 < nt) tp_load(s8, it.src_pitch, R, C, ((t + 1) / tc) * kTp, ((t + 1) % tc) * kTp, g);
    // store: a warp takes one destination row (source column) at a time, two elements per lane
    for (uint32_t c = warp; c < nc; c += 8) {
      uint8_t* row = d8 + (c0 + c) * it.dst_pitch + (uint64_t)r0 * 2;
      const uint32_t r = 2 * lane;
      const uint16_t lo = r < nr ? tile[r * kTpPitch + c] : 0;
      const uint16_t hi = r + 1 < nr ? tile[(r + 1) * kTpPitch + c] : 0;
      if (r + 1 < nr && (reinterpret_cast<uint64_t>(row) & 3) == 0) {
        reinterpret_cast<uint32_t*>(row)[lane] = (uint32_t)lo | ((uint32_t)hi << 16);
      } else {
        if (r < nr) reinterpret_cast<uint16_t*>(row)[r] = lo;
        if (r + 1 < nr) reinterpret_cast<uint16_t*>(row)[r + 1] = hi;
      }
    }
  }
}

__device__ void generic_item(const Item& it, uint16_t* tile, uint32_t* status) {
  const uint32_t k = op_kind(it.op);
  if (k == OP_CAST) {
    cast_item(it, status);
    return;
  }
  if (k == OP_TRANSPOSE) {
    transpose_item(it, tile, status);
    return;
  }
  const int g = item_granularity(it);
  if (k == OP_COPY_MC) {
    if (g != 16) {
      if (threadIdx.x == 0 && status) atomicOr(status, ST_BAD_ITEM);
      return;
    }
    copy_item<16, true>(it);
    return;
  }
  if (k != OP_COPY) {
    if (threadIdx.x == 0 && status) atomicOr(status, ST_BAD_ITEM);
    return;
  }
  switch (g) {
    case 16: copy_item<16, false>(it); break;
    case 8: copy_item<8, false>(it); break;
    case 4: copy_item<4, false>(it); break;
    case 2: copy_item<2, false>(it); break;
    default: copy_item<1, false>(it); break;
  }
}

// ------------------------------------------------------------------------------------
// quant blocks: 128 x 128 -> e4m3 + fp32 scale (scale = amax / 448, q = satfinite(x * RN(1 / scale)))
// ------------------------------------------------------------------------------------
__device__ __forceinline__ float block_max(float v, float* red) {
  #pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();  // red[] may still be read from the previous block
  if (l == 0) red[w] = v;
  __syncthreads();
  if (w == 0) {
    const int nw = (blockDim.x + 31) >> 5;
    float x = l < nw ? red[l] : 0.f;
    #pragma unroll
    for (int o = 16; o > 0; o >>= 1) x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, o));
    if (l == 0) red[32] = x;
  }
  __syncthreads();
  return red[32];
}

__device__ __forceinline__ float2 unpack2(uint32_t w, bool bf16) {
  if (bf16) {
    __nv_bfloat162 h = *reinterpret_cast<__nv_bfloat162*>(&w);
    return __bfloat1622float2(h);
  }
  __half2 h = *reinterpret_cast<__half2*>(&w);
  return __half22float2(h);
}

__device__ __forceinline__ uint32_t pack4_e4m3(float a, float b, float c, float d, float inv) {
  const __nv_fp8x2_storage_t lo = __nv_cvt_float2_to_fp8x2(make_float2(__fmul_rn(a, inv), __fmul_rn(b, inv)),
                                                           __NV_SATFINITE, __NV_E4M3);
  const __nv_fp8x2_storage_t hi = __nv_cvt_float2_to_fp8x2(make_float2(__fmul_rn(c, inv), __fmul_rn(d, inv)),
                                                           __NV_SATFINITE, __NV_E4M3);
  return (uint32_t)lo | ((uint32_t)hi << 16);
}

// amax of 8 packed 16-bit floats (bf16 or fp16) without unpacking: max of |x| is exact in
// the source format.
__device__ __forceinline__ float amax8(const uint4 v, bool bf16) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
  if (bf16) {
    __nv_bfloat162 m = __float2bfloat162_rn(0.f);
    #pragma unroll
    for (int j = 0; j < 4; ++j) m = __hmax2(m, __habs2(*reinterpret_cast<const __nv_bfloat162*>(&w[j])));
    const float2 f = __bfloat1622float2(m);
    return fmaxf(f.x, f.y);
  }
  __half2 m = __float2half2_rn(0.f);
  #pragma unroll
  for (int j = 0; j < 4; ++j) m = __hmax2(m, __habs2(*reinterpret_cast<const __half2*>(&w[j])));
  const float2 f = __half22float2(m);
  return fmaxf(f.x, f.y);
}

// 8 source values (one uint4) -> 8 e4m3 bytes (one uint2)
__device__ __forceinline__ uint2 quant8(const uint4 v, bool bf16, float inv) {
  const float2 a = unpack2(v.x, bf16), b = unpack2(v.y, bf16), c = unpack2(v.z, bf16), e = unpack2(v.w, bf16);
  return make_uint2(pack4_e4m3(a.x, a.y, b.x, b.y, inv), pack4_e4m3(c.x, c.y, e.x, e.y, inv));
}

// One block of a block-quantised matrix: scale = amax / 448 (IEEE division), inv = RN(1 / scale),
// q = satfinite_e4m3(x * inv) with round-to-nearest-even; the block's scale goes to the scale grid.
__device__ void quant_block(const QuantDesc& d, uint32_t block, float* red, uint32_t* status) {
  const uint32_t bn = d.bn, bk = d.bk;
  const uint32_t nbc = (d.cols + bk - 1) / bk;
  const uint32_t br = block / nbc, bc = block - br * nbc;
  const uint32_t r0 = br * bn, c0 = bc * bk;
  const uint32_t nr = min(bn, d.rows - r0), nc = min(bk, d.cols - c0);
  const uint32_t es = dt_size(d.src_code);
  if (es == 0 || bn == 0 || bk == 0) {
    if (threadIdx.x == 0 && status) atomicOr(status, ST_BAD_QUANT);
    return;
  }
  const uint8_t* src = reinterpret_cast<const uint8_t*>(d.src) + r0 * d.src_pitch + (uint64_t)c0 * es;
  uint8_t* dst = reinterpret_cast<uint8_t*>(d.dst) + r0 * d.dst_pitch + c0;
  float scale;
  const bool fast = es == 2 && bk == 128 && bn <= 128 && nc == 128 && blockDim.x == 256 &&
                    ((reinterpret_cast<uint64_t>(src) | (uint64_t)d.src_pitch) & 15) == 0 &&
                    ((reinterpret_cast<uint64_t>(dst) | (uint64_t)d.dst_pitch) & 15) == 0;
  if (fast) {
    // 8 threads span a 128-column row (16 columns = 32 source bytes each); 32 rows per pass,
    // 4 passes.  Every thread ends with one 16-byte store per row it owns.
    const uint32_t col = threadIdx.x & 7, rg = threadIdx.x >> 3;
    const bool bf16 = d.src_code == DT_BF16;
    uint4 v[4][2];
    #pragma unroll
    for (int k = 0; k < 4; ++k) {
      const uint32_t r = rg + 32u * k;
      if (r < nr) {
        const uint8_t* p = src + r * d.src_pitch + col * 32u;
        v[k][0] = ld_nc16(p);
        v[k][1] = ld_nc16(p + 16);
      } else {
        v[k][0] = v[k][1] = make_uint4(0, 0, 0, 0);
      }
    }
    float amax = 0.f;
    #pragma unroll
    for (int k = 0; k < 4; ++k) amax = fmaxf(amax, fmaxf(amax8(v[k][0], bf16), amax8(v[k][1], bf16)));
    amax = block_max(amax, red);
    scale = amax > 0.f ? __fdiv_rn(amax, kE4M3Max) : 1.f;
    const float inv = __frcp_rn(scale);
    #pragma unroll
    for (int k = 0; k < 4; ++k) {
      const uint32_t r = rg + 32u * k;
      if (r >= nr) continue;
      const uint2 lo = quant8(v[k][0], bf16, inv), hi = quant8(v[k][1], bf16, inv);
      st16(dst + r * d.dst_pitch + col * 16u, make_uint4(lo.x, lo.y, hi.x, hi.y));
    }
  } else {
    float amax = 0.f;
    const uint32_t n = nr * nc;
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) {
      const uint32_t r = i / nc, c = i - r * nc;
      amax = fmaxf(amax, fabsf(ld_as_f32(src + r * d.src_pitch + (uint64_t)c * es, d.src_code)));
    }
    amax = block_max(amax, red);
    scale = amax > 0.f ? __fdiv_rn(amax, kE4M3Max) : 1.f;
    const float inv = __frcp_rn(scale);
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) {
      const uint32_t r = i / nc, c = i - r * nc;
      const float x = ld_as_f32(src + r * d.src_pitch + (uint64_t)c * es, d.src_code);
      dst[r * d.dst_pitch + c] = __nv_cvt_float_to_fp8(__fmul_rn(x, inv), __NV_SATFINITE, __NV_E4M3);
    }
  }
  if (threadIdx.x == 0)
    *reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(d.scale) + br * d.scale_pitch + bc * 4u) = scale;
}

// ------------------------------------------------------------------------------------
// quant blocks from shared memory (TMA modes): the 128 x 128 source block was loaded by one
// tensor-map copy (rows at a 256-byte pitch; rows and columns past the matrix read as zero,
// which leaves the amax unchanged).  Thread t holds elements [8c, 8c + 8) and [64 + 8c, 72 + 8c)
// of rows t / 8 + 32k (c = t % 8): each quarter-warp reads 128 contiguous bytes, no bank
// conflicts.  Same arithmetic as quant_block, so the output is identical.
// ------------------------------------------------------------------------------------
__device__ __forceinline__ void st8(void* p, uint2 v) {
  asm volatile("st.global.v2.u32 [%0], {%1,%2};" ::"l"(p), "r"(v.x), "r"(v.y) : "memory");
}

__device__ void quant_block_smem(const QuantDesc& d, uint32_t block, const uint8_t* tile, float* red) {
  const uint32_t nbc = (d.cols + 127u) / 128u;
  const uint32_t br = block / nbc, bc = block - br * nbc;
  const uint32_t r0 = br * 128u, c0 = bc * 128u;
  const uint32_t nr = min(128u, d.rows - r0), nc = min(128u, d.cols - c0);
  const bool bf16 = d.src_code == DT_BF16;
  const uint32_t cc = threadIdx.x & 7u, rg = threadIdx.x >> 3;
  uint4 v[4][2];
  #pragma unroll
  for (int k = 0; k < 4; ++k) {
    const uint4* p = reinterpret_cast<const uint4*>(tile + (rg + 32u * k) * 256u + cc * 16u);
    v[k][0] = p[0];
    v[k][1] = p[8];
  }
  float amax = 0.f;
  #pragma unroll
  for (int k = 0; k < 4; ++k) amax = fmaxf(amax, fmaxf(amax8(v[k][0], bf16), amax8(v[k][1], bf16)));
  // block max with one barrier: every warp posts its max, every thread folds the eight
  // (the caller's barrier after the previous block guards `red` against reuse)
  #pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  if ((threadIdx.x & 31u) == 0) red[threadIdx.x >> 5] = amax;
  __syncthreads();
  #pragma unroll
  for (int w = 0; w < kThreads / 32; ++w) amax = fmaxf(amax, red[w]);
  const float scale = amax > 0.f ? __fdiv_rn(amax, kE4M3Max) : 1.f;
  const float inv = __frcp_rn(scale);
  uint8_t* dst = reinterpret_cast<uint8_t*>(d.dst) + r0 * d.dst_pitch + c0;
  // 16-byte stores where the destination allows: lane pairs (c, c ^ 1) swap one 8-byte half,
  // so the even lane stores columns [16m, 16m + 16) and the odd lane [64 + 16m, 80 + 16m)
  // (c = 2m, 2m + 1): one warp instruction writes each of its rows as 128 contiguous bytes,
  // whole lines on NVLink when the destination is a peer GPU
  const bool wide = ((reinterpret_cast<uint64_t>(dst) | (uint64_t)d.dst_pitch) & 15) == 0;
  const bool odd = cc & 1u;
  #pragma unroll
  for (int k = 0; k < 4; ++k) {
    const uint32_t r = rg + 32u * k;
    const uint2 lo = quant8(v[k][0], bf16, inv), hi = quant8(v[k][1], bf16, inv);
    const uint2 give = odd ? lo : hi;
    const uint2 got = make_uint2(__shfl_xor_sync(0xffffffffu, give.x, 1), __shfl_xor_sync(0xffffffffu, give.y, 1));
    if (r >= nr) continue;
    uint8_t* row = dst + r * d.dst_pitch;
    if (wide) {
      const uint32_t col = odd ? 64u + 8u * (cc - 1u) : 8u * cc;          // 16-byte aligned
      const uint4 v16 = odd ? make_uint4(got.x, got.y, hi.x, hi.y) : make_uint4(lo.x, lo.y, got.x, got.y);
      if (col + 16u <= nc) st16(row + col, v16);
      else if (col + 8u <= nc) st8(row + col, make_uint2(v16.x, v16.y));
    } else {
      if (cc * 8u < nc) st8(row + cc * 8u, lo);
      if (64u + cc * 8u < nc) st8(row + 64u + cc * 8u, hi);
    }
  }
  if (threadIdx.x == 0)
    *reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(d.scale) + br * d.scale_pitch + bc * 4u) = scale;
}

// ------------------------------------------------------------------------------------
// bulk items: TMA pipeline driven by one thread
// ------------------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait: false once `limit` polls have passed without the phase completing.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, uint32_t limit) {
  for (uint32_t i = 0; i < limit; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  return false;
}
__device__ __forceinline__ void bulk_g2s(void* smem, const void* gsrc, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(smem)),
               "l"(gsrc), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void bulk_s2g(void* gdst, const void* smem, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(gdst), "r"(smem_u32(smem)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

struct PieceCursor {
  const Item* items;
  uint32_t n, idx, row, off;
  Item it;
  __device__ void start(const Item* items_, uint32_t n_) {
    items = items_;
    n = n_;
    idx = blockIdx.x;
    row = off = 0;
    if (idx < n) it = items[idx];
  }
  // next piece of at most `piece` bytes: false when this CTA's items are exhausted
  __device__ bool next(uint32_t piece, uint64_t& s, uint64_t& d, uint32_t& b) {
    while (idx < n) {
      if (row < it.rows && it.row_bytes > 0) {
        b = min(piece, it.row_bytes - off);
        s = it.src + (uint64_t)(row * it.src_pitch) + off;
        d = it.dst + (uint64_t)(row * it.dst_pitch) + off;
        off += b;
        if (off >= it.row_bytes) {
          off = 0;
          ++row;
        }
        return true;
      }
      idx += gridDim.x;
      row = off = 0;
      if (idx < n) it = items[idx];
    }
    return false;
  }
};

template <int S, int KST>
__device__ void bulk_pipeline(const Item* items, uint32_t n_items, uint8_t* stage_mem, uint32_t piece,
                              uint64_t* bars, uint64_t* ring_dst, uint32_t* ring_bytes, uint32_t spin_limit,
                              uint32_t* status) {
  constexpr int KLD = S - KST;
  static_assert(KLD >= 1 && KST >= 0, "stage split");
  for (int s = 0; s < S; ++s) mbar_init(&bars[s], 1);
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");

  PieceCursor cur;
  cur.start(items, n_items);
  uint32_t loaded = 0, stored = 0;
  uint64_t src, dst;
  uint32_t bytes;
  auto issue = [&](uint32_t p) -> bool {
    if (!cur.next(piece, src, dst, bytes)) return false;
    if (((src | dst | bytes) & 15) != 0) {  // never issue a misaligned bulk copy
      if (status) atomicOr(status, ST_BAD_ITEM);
      return false;
    }
    const uint32_t s = p % S;
    ring_dst[s] = dst;
    ring_bytes[s] = bytes;
    mbar_expect_tx(&bars[s], bytes);
    bulk_g2s(stage_mem + (size_t)s * piece, reinterpret_cast<const void*>(src), bytes, &bars[s]);
    return true;
  };
  while (loaded < (uint32_t)KLD && issue(loaded)) ++loaded;
  bool failed = false;
  while (stored < loaded) {
    const uint32_t s = stored % S;
    if (!mbar_wait_bounded(&bars[s], (stored / S) & 1u, spin_limit)) {
      if (status) atomicOr(status, ST_MBAR_TIMEOUT);
      failed = true;
      break;
    }
    bulk_s2g(reinterpret_cast<void*>(ring_dst[s]), stage_mem + (size_t)s * piece, ring_bytes[s]);
    bulk_commit();
    ++stored;
    bulk_wait_read<KST>();
    if (issue(loaded)) ++loaded;
  }
  if (failed) {
    // drain: give the loads still in flight a bounded chance to land before smem goes away
    for (uint32_t p = stored + 1; p < loaded; ++p) mbar_wait_bounded(&bars[p % S], (p / S) & 1u, spin_limit);
  }
  bulk_wait_all();
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

// ------------------------------------------------------------------------------------
// quant phase of the TMA modes: the dynamic shared memory is a ring of `qs` block stages.
// Thread 0 keeps `qs` tensor-map loads in flight (the CTA's next TMA-eligible blocks, in the
// order the consumers take them); all 256 threads wait on a stage's mbarrier, quantise it
// from shared memory, and after a barrier thread 0 refills the stage.  Blocks without a valid
// map take the register path in the same walk.  A wait that runs out of polls sets
// ST_MBAR_TIMEOUT; the CTA then lets its loads in flight land (bounded) and skips its
// remaining blocks.
// ------------------------------------------------------------------------------------
constexpr int kMaxQStages = 8;

__device__ __forceinline__ void tma_load_2d(void* smem, const void* tmap, int32_t x, int32_t y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(smem)),
      "l"(tmap), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

__device__ void quant_tma_phase(const TransferArgs& a, uint8_t* smem, uint32_t qs, uint64_t* qbars, float* red) {
  if (threadIdx.x == 0) {
    for (uint32_t s = 0; s < qs; ++s) mbar_init(&qbars[s], 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  uint32_t pi = blockIdx.x, issued = 0;      // producer cursor (thread 0)
  auto issue_next = [&]() {
    while (pi < a.n_qwork) {
      const QuantWork w = a.qwork[pi];
      pi += gridDim.x;
      if (!a.qtma[w.desc]) continue;
      const uint32_t cols = a.qdescs[w.desc].cols;
      const uint32_t nbc = (cols + 127u) / 128u;
      const uint32_t br = w.block / nbc, bc = w.block - br * nbc;
      const uint32_t s = issued % qs;
      mbar_expect_tx(&qbars[s], kQBlockBytes);
      tma_load_2d(smem + (size_t)s * kQBlockBytes, a.qmaps + (size_t)w.desc * 128u, (int32_t)(bc * 128u),
                  (int32_t)(br * 128u), &qbars[s]);
      ++issued;
      return;
    }
  };
  if (threadIdx.x == 0) {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    for (uint32_t k = 0; k < qs; ++k) issue_next();
  }
  uint32_t consumed = 0;
  for (uint32_t i = blockIdx.x; i < a.n_qwork; i += gridDim.x) {
    const QuantWork w = a.qwork[i];
    const QuantDesc d = a.qdescs[w.desc];
    if (!a.qtma[w.desc]) {
      quant_block(d, w.block, red, a.sig.status);
      continue;
    }
    const uint32_t s = consumed % qs;
    const bool ok = mbar_wait_bounded(&qbars[s], (consumed / qs) & 1u, a.mbar_spin_limit);
    if (__syncthreads_or(!ok)) {
      if (threadIdx.x == 0) {
        if (a.sig.status) atomicOr(a.sig.status, ST_MBAR_TIMEOUT);
        for (uint32_t k = consumed; k < issued; ++k) mbar_wait_bounded(&qbars[k % qs], (k / qs) & 1u, a.mbar_spin_limit);
      }
      __syncthreads();
      return;
    }
    quant_block_smem(d, w.block, smem + (size_t)s * kQBlockBytes, red);
    __syncthreads();                       // every thread is done reading stage s
    if (threadIdx.x == 0) {
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      issue_next();
    }
    ++consumed;
  }
}

// ------------------------------------------------------------------------------------
// completion signal
// ------------------------------------------------------------------------------------
__device__ void signal_done(const Signal& sg, uint32_t* s_last) {
  if (sg.counter == nullptr) return;
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    const uint32_t prev = atomicAdd(sg.counter, 1u);
    *s_last = (prev == gridDim.x - 1) ? 1u : 0u;
  }
  __syncthreads();
  if (*s_last && threadIdx.x == 0) {
    __threadfence_system();
    const uint64_t e = *reinterpret_cast<volatile const uint64_t*>(sg.epoch);
    for (uint32_t i = 0; i < sg.n_flags; ++i) {
      const uint64_t a = sg.flag_addrs[i];     // bit 0 set: a multicast address (replica group)
      if (a & 1ull) st_mc_release_sys(reinterpret_cast<uint64_t*>(a & ~1ull), e);
      else st_release_sys(reinterpret_cast<uint64_t*>(a), e);
    }
    *reinterpret_cast<volatile uint32_t*>(sg.counter) = 0u;
    __threadfence();
  }
}

// ------------------------------------------------------------------------------------
// kernels
// ------------------------------------------------------------------------------------

template <bool BULK, int S, int KST>
__global__ void __launch_bounds__(kThreads) transfer_kernel(TransferArgs a) {
  extern __shared__ __align__(1024) uint8_t dyn_smem[];
  __shared__ float red[33];
  __shared__ __align__(16) uint16_t tile[kTp * kTpPitch];
  __shared__ uint32_t s_last;
  __shared__ uint64_t bars[S > 0 ? S : 1];
  __shared__ uint64_t ring_dst[S > 0 ? S : 1];
  __shared__ uint32_t ring_bytes[S > 0 ? S : 1];
  __shared__ uint64_t qbars[BULK ? kMaxQStages : 1];

  for (uint32_t i = blockIdx.x; i < a.n_items; i += gridDim.x) {
    const Item it = a.items[i];
    generic_item(it, tile, a.sig.status);
  }
  uint32_t qs = 0;                          // quant stages in shared memory (TMA modes)
  if constexpr (BULK) {
    if (a.qmaps != nullptr && a.qtma != nullptr)
      qs = min((uint32_t)kMaxQStages, (uint32_t)(((uint64_t)S * a.piece_bytes) / kQBlockBytes));
  }
  if (qs > 0 && a.n_qwork > 0) {
    if constexpr (BULK) quant_tma_phase(a, dyn_smem, qs, qbars, red);
  } else {
    for (uint32_t i = blockIdx.x; i < a.n_qwork; i += gridDim.x) {
      const QuantWork w = a.qwork[i];
      const QuantDesc d = a.qdescs[w.desc];
      quant_block(d, w.block, red, a.sig.status);
    }
  }
  if constexpr (BULK) {
    if (a.n_bulk > 0 && threadIdx.x == 0)
      bulk_pipeline<S, KST>(a.bulk_items, a.n_bulk, dyn_smem, a.piece_bytes, bars, ring_dst, ring_bytes,
                            a.mbar_spin_limit, a.sig.status);
  }
  signal_done(a.sig, &s_last);
}

__global__ void wait_flags_kernel(const uint64_t* flags, uint32_t n, const uint64_t* epoch, uint64_t timeout_ns,
                                  uint32_t* status, uint32_t* where) {
  if (threadIdx.x >= 32) return;
  const uint64_t e = *reinterpret_cast<volatile const uint64_t*>(epoch);
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t i = threadIdx.x; i < n; i += 32) {
    uint64_t v;
    while ((v = ld_acquire_sys(flags + i)) < e) {
      if (globaltimer_ns() - t0 > timeout_ns) {
        atomicOr(status, ST_FLAG_TIMEOUT);
        if (where) atomicMin(where, i);
        return;
      }
      __nanosleep(256);
    }
    if (v != e) atomicOr(status, ST_FLAG_STALE);
  }
}

// ------------------------------------------------------------------------------------
// host launchers
// ------------------------------------------------------------------------------------
namespace {
template <bool BULK, int S, int KST>
cudaError_t launch_impl(const TransferArgs& a, int grid, size_t smem, cudaStream_t stream) {
  auto k = transfer_kernel<BULK, S, KST>;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
  k<<<grid, kThreads, smem, stream>>>(a);
  return cudaGetLastError();
}
}  // namespace

int bulk_stages(int mode) {
  switch (mode) {
    case 1: return 8;
    case 2: return 12;
    case 3: return 4;
    default: return 0;
  }
}

cudaError_t launch_transfer(const TransferArgs& a, int mode, int grid, cudaStream_t stream) {
  if (grid <= 0) return cudaErrorInvalidValue;
  const size_t smem = (size_t)bulk_stages(mode) * a.piece_bytes;
  switch (mode) {
    case 0: return launch_impl<false, 0, 0>(a, grid, 0, stream);
    case 1: return launch_impl<true, 8, 4>(a, grid, smem, stream);
    case 2: return launch_impl<true, 12, 6>(a, grid, smem, stream);
    case 3: return launch_impl<true, 4, 2>(a, grid, smem, stream);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_wait_flags(const uint64_t* flags, uint32_t n, const uint64_t* epoch, uint64_t timeout_ns,
                              uint32_t* status, uint32_t* where, cudaStream_t stream) {
  wait_flags_kernel<<<1, 32, 0, stream>>>(flags, n, epoch, timeout_ns, status, where);
  return cudaGetLastError();
}

uint32_t encode_quant_maps(const QuantDesc* descs, uint32_t n, uint8_t* maps, uint8_t* valid) {
  using Encode = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                              const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                              CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
  static Encode encode = drv::entry<Encode>("cuTensorMapEncodeTiled");
  static_assert(sizeof(CUtensorMap) == 128, "tensor map size");
  uint32_t ok = 0;
  for (uint32_t i = 0; i < n; ++i) {
    const QuantDesc& d = descs[i];
    CUtensorMap* m = reinterpret_cast<CUtensorMap*>(maps + (size_t)i * 128u);
    std::memset(m, 0, sizeof(CUtensorMap));
    valid[i] = 0;
    const bool fits = (d.src_code == DT_BF16 || d.src_code == DT_F16) && d.bn == 128 && d.bk == 128 && d.rows > 0 &&
                      d.cols > 0 && d.cols % 8 == 0 && d.src % 16 == 0 && d.src_pitch > 0 && d.src_pitch % 16 == 0 &&
                      (uint64_t)d.src_pitch >= 2ull * d.cols && (uint64_t)d.src_pitch < (1ull << 40) &&
                      d.dst % 8 == 0 && d.dst_pitch % 8 == 0;
    if (!fits) continue;
    const cuuint64_t dims[2] = {d.cols, d.rows};
    const cuuint64_t strides[1] = {(cuuint64_t)d.src_pitch};
    const cuuint32_t box[2] = {128u, 128u};
    const cuuint32_t estr[2] = {1u, 1u};
    const CUresult r = encode(m, d.src_code == DT_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                              2, reinterpret_cast<void*>(d.src), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                              CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r == CUDA_SUCCESS) {
      valid[i] = 1;
      ++ok;
    }
  }
  return ok;
}

}  // namespace wb
