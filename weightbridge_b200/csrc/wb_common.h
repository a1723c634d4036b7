// Work-table layouts shared by the sm_100a transfer kernel, the CPU executor and the
// Python planner (weightbridge_b200/core/plan.py declares the same byte layouts).
#pragma once
#include <cstdint>

#if defined(__CUDACC__)
#define WB_HD __host__ __device__
#else
#define WB_HD
#endif

namespace wb {

// dtype wire codes (weightbridge_b200/utils/dtypes.py: DTYPE_CODES)
enum DType : uint32_t {
  DT_U8 = 0, DT_I8 = 1, DT_F16 = 2, DT_BF16 = 3, DT_F32 = 4, DT_E4M3 = 5,
  DT_I32 = 6, DT_I64 = 7, DT_F64 = 8, DT_BOOL = 9, DT_I16 = 10, DT_E5M2 = 11,
};

// op word: bits 0-7 kind, 8-15 source dtype, 16-23 destination dtype
// OP_TRANSPOSE: `rows` source rows of `row_bytes` (same dtype both sides); destination row c
// (at dst + c * dst_pitch, `dst_row_bytes` long) holds source column c.
enum OpKind : uint32_t { OP_COPY = 0, OP_CAST = 1, OP_COPY_MC = 2, OP_TRANSPOSE = 3 };

inline WB_HD uint32_t op_kind(uint32_t w) { return w & 0xffu; }
inline WB_HD uint32_t op_src(uint32_t w) { return (w >> 8) & 0xffu; }
inline WB_HD uint32_t op_dst(uint32_t w) { return (w >> 16) & 0xffu; }

// bytes per element of a dtype code (0: unknown)
inline WB_HD uint32_t dtype_bytes(uint32_t c) {
  switch (c) {
    case DT_U8: case DT_I8: case DT_E4M3: case DT_BOOL: case DT_E5M2: return 1u;
    case DT_F16: case DT_BF16: case DT_I16: return 2u;
    case DT_F32: case DT_I32: return 4u;
    case DT_I64: case DT_F64: return 8u;
    default: return 0u;
  }
}

// One unit of copy work: `rows` rows of `row_bytes` source bytes.
struct alignas(16) Item {
  uint64_t src;
  uint64_t dst;
  int64_t src_pitch;       // bytes between source rows
  int64_t dst_pitch;       // bytes between destination rows
  uint32_t row_bytes;      // source bytes per row
  uint32_t rows;
  uint32_t op;             // op word
  uint32_t dst_row_bytes;  // destination bytes per row (differs from row_bytes for casts)
};
static_assert(sizeof(Item) == 48, "Item layout");

// One block-quantised matrix: rows x cols source elements -> e4m3 + fp32 block scales.
struct alignas(16) QuantDesc {
  uint64_t src;
  uint64_t dst;
  uint64_t scale;
  int64_t src_pitch;       // bytes
  int64_t dst_pitch;       // bytes
  int64_t scale_pitch;     // bytes between scale rows; scale columns are contiguous fp32
  uint32_t rows;
  uint32_t cols;
  uint32_t src_code;       // DT_BF16 / DT_F16 / DT_F32
  uint16_t bn;             // block rows
  uint16_t bk;             // block cols
};
static_assert(sizeof(QuantDesc) == 64, "QuantDesc layout");

struct QuantWork {
  uint32_t desc;
  uint32_t block;          // row-major block index inside the matrix
};
static_assert(sizeof(QuantWork) == 8, "QuantWork layout");

// One sender's part of a 128 x 128 quantisation block whose rows or columns are spread over
// several senders (a "split block"): the block's scale needs the amax of every part, so the
// senders first reduce their parts (split_amax), exchange the maxima on the host, then
// quantise their parts with the common amax (split_quant).
struct alignas(16) SplitPiece {
  uint64_t src;
  uint64_t dst;            // e4m3 destination of the part
  uint64_t scale;          // the block's fp32 scale cell
  int64_t src_pitch;       // bytes
  int64_t dst_pitch;       // bytes
  uint32_t rows;           // at most one block
  uint32_t cols;
  uint32_t src_code;       // DT_BF16 / DT_F16 / DT_F32
  uint32_t reserved[3];
};
static_assert(sizeof(SplitPiece) == 64, "SplitPiece layout");

// Status bits a kernel reports through its status word.
enum Status : uint32_t {
  ST_OK = 0,
  ST_MBAR_TIMEOUT = 1u << 0,   // a TMA load never completed within the wait limit
  ST_FLAG_TIMEOUT = 1u << 1,   // a peer's flag never reached the expected epoch
  ST_FLAG_STALE = 1u << 2,     // a flag holds an epoch other than the expected one
  ST_BAD_ITEM = 1u << 3,       // an item violated the kernel's alignment contract
  ST_BAD_QUANT = 1u << 4,      // a quant descriptor the kernel cannot handle
};

constexpr float kE4M3Max = 448.0f;

}  // namespace wb
