// CPU executor for the same work tables the sm_100a kernel walks.  It runs the gloo
// (cpu_direct) transfer path - pack local shards into a wire buffer, unpack a received
// buffer into local shards - and is the oracle the GPU tests compare against.
//
// Casts round to nearest even (c10::BFloat16 / c10::Half); block fp8 computes
// scale = amax / 448, inv = 1 / scale and q = e4m3(clamp(x * inv, +-448)) in IEEE float, the
// same arithmetic as the device kernel.
#include "wb_cpu.h"

#include <ATen/Parallel.h>
#include <c10/util/BFloat16.h>
#include <c10/util/Float8_e4m3fn.h>
#include <c10/util/Half.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <stdexcept>

namespace wb {
namespace {

inline uint32_t dsize(uint32_t c) { return c == DT_F32 ? 4u : (c == DT_BF16 || c == DT_F16) ? 2u : 0u; }

inline float load_f(const uint8_t* p, uint32_t c) {
  if (c == DT_F32) {
    float v;
    std::memcpy(&v, p, 4);
    return v;
  }
  uint16_t bits;
  std::memcpy(&bits, p, 2);
  if (c == DT_BF16) return static_cast<float>(c10::BFloat16(bits, c10::BFloat16::from_bits()));
  return static_cast<float>(c10::Half(bits, c10::Half::from_bits()));
}

inline void store_f(uint8_t* p, uint32_t c, float v) {
  if (c == DT_F32) {
    std::memcpy(p, &v, 4);
  } else if (c == DT_BF16) {
    const uint16_t b = c10::BFloat16(v).x;
    std::memcpy(p, &b, 2);
  } else {
    const uint16_t b = c10::Half(v).x;
    std::memcpy(p, &b, 2);
  }
}

void run_item(const Item& it) {
  const uint8_t* s = reinterpret_cast<const uint8_t*>(it.src);
  uint8_t* d = reinterpret_cast<uint8_t*>(it.dst);
  const uint32_t k = op_kind(it.op);
  if (k == OP_CAST) {
    const uint32_t sc = op_src(it.op), dc = op_dst(it.op);
    const uint32_t ss = dsize(sc), ds = dsize(dc);
    if (!ss || !ds) throw std::invalid_argument("cast item with unsupported dtype");
    const uint32_t n = it.row_bytes / ss;
    for (uint32_t r = 0; r < it.rows; ++r)
      for (uint32_t c = 0; c < n; ++c) store_f(d + r * it.dst_pitch + (uint64_t)c * ds, dc, load_f(s + r * it.src_pitch + (uint64_t)c * ss, sc));
    return;
  }
  if (k == OP_COPY_MC) throw std::invalid_argument("multicast items have no CPU execution");
  if (k == OP_TRANSPOSE) {
    const uint32_t es = dtype_bytes(op_src(it.op));
    if (!es || it.row_bytes % es) throw std::invalid_argument("transpose item with unsupported dtype");
    const uint32_t cols = it.row_bytes / es;
    for (uint32_t r = 0; r < it.rows; ++r)
      for (uint32_t c = 0; c < cols; ++c)
        std::memcpy(d + c * it.dst_pitch + (uint64_t)r * es, s + r * it.src_pitch + (uint64_t)c * es, es);
    return;
  }
  if (k != OP_COPY) throw std::invalid_argument("work row with an unknown op kind");
  for (uint32_t r = 0; r < it.rows; ++r) std::memcpy(d + r * it.dst_pitch, s + r * it.src_pitch, it.row_bytes);
}

void run_quant(const QuantDesc& q, uint32_t block) {
  const uint32_t es = dsize(q.src_code);
  if (!es || !q.bn || !q.bk) throw std::invalid_argument("bad quant descriptor");
  const uint32_t nbc = (q.cols + q.bk - 1) / q.bk;
  const uint32_t br = block / nbc, bc = block % nbc;
  const uint32_t r0 = br * q.bn, c0 = bc * q.bk;
  const uint32_t nr = std::min<uint32_t>(q.bn, q.rows - r0), nc = std::min<uint32_t>(q.bk, q.cols - c0);
  const uint8_t* src = reinterpret_cast<const uint8_t*>(q.src) + r0 * q.src_pitch + (uint64_t)c0 * es;
  uint8_t* dst = reinterpret_cast<uint8_t*>(q.dst) + r0 * q.dst_pitch + c0;
  float amax = 0.f;
  for (uint32_t r = 0; r < nr; ++r)
    for (uint32_t c = 0; c < nc; ++c) amax = std::max(amax, std::fabs(load_f(src + r * q.src_pitch + (uint64_t)c * es, q.src_code)));
  const float scale = amax > 0.f ? amax / kE4M3Max : 1.f;
  const float inv = 1.f / scale;
  for (uint32_t r = 0; r < nr; ++r)
    for (uint32_t c = 0; c < nc; ++c) {
      float x = load_f(src + r * q.src_pitch + (uint64_t)c * es, q.src_code) * inv;
      x = std::min(std::max(x, -kE4M3Max), kE4M3Max);
      dst[r * q.dst_pitch + c] = c10::Float8_e4m3fn(x).x;
    }
  float* sp = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(q.scale) + br * q.scale_pitch + bc * 4u);
  *sp = scale;
}

float piece_amax(const SplitPiece& p) {
  const uint32_t es = dsize(p.src_code);
  if (!es) throw std::invalid_argument("split piece with unsupported dtype");
  const uint8_t* src = reinterpret_cast<const uint8_t*>(p.src);
  float amax = 0.f;
  for (uint32_t r = 0; r < p.rows; ++r)
    for (uint32_t c = 0; c < p.cols; ++c)
      amax = std::max(amax, std::fabs(load_f(src + (int64_t)r * p.src_pitch + (uint64_t)c * es, p.src_code)));
  return amax;
}

void piece_quant(const SplitPiece& p, float amax) {
  const uint32_t es = dsize(p.src_code);
  if (!es) throw std::invalid_argument("split piece with unsupported dtype");
  const uint8_t* src = reinterpret_cast<const uint8_t*>(p.src);
  uint8_t* dst = reinterpret_cast<uint8_t*>(p.dst);
  const float scale = amax > 0.f ? amax / kE4M3Max : 1.f;
  const float inv = 1.f / scale;
  for (uint32_t r = 0; r < p.rows; ++r)
    for (uint32_t c = 0; c < p.cols; ++c) {
      float x = load_f(src + (int64_t)r * p.src_pitch + (uint64_t)c * es, p.src_code) * inv;
      x = std::min(std::max(x, -kE4M3Max), kE4M3Max);
      dst[(int64_t)r * p.dst_pitch + c] = c10::Float8_e4m3fn(x).x;
    }
  std::memcpy(reinterpret_cast<void*>(p.scale), &scale, 4);
}

}  // namespace

void cpu_split_amax(const SplitPiece* pieces, size_t n, float* partial) {
  at::parallel_for(0, (int64_t)n, 4, [&](int64_t b, int64_t e) {
    for (int64_t i = b; i < e; ++i) partial[i] = piece_amax(pieces[i]);
  });
}

void cpu_split_quant(const SplitPiece* pieces, size_t n, const float* amax) {
  at::parallel_for(0, (int64_t)n, 4, [&](int64_t b, int64_t e) {
    for (int64_t i = b; i < e; ++i) piece_quant(pieces[i], amax[i]);
  });
}

void cpu_execute(const Item* items, size_t n_items, const QuantDesc* qdescs, const QuantWork* qwork,
                 size_t n_qwork) {
  at::parallel_for(0, (int64_t)n_items, 16, [&](int64_t b, int64_t e) {
    for (int64_t i = b; i < e; ++i) run_item(items[i]);
  });
  at::parallel_for(0, (int64_t)n_qwork, 4, [&](int64_t b, int64_t e) {
    for (int64_t i = b; i < e; ++i) run_quant(qdescs[qwork[i].desc], qwork[i].block);
  });
}

}  // namespace wb
