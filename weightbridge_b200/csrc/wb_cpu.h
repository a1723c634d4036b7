// CPU executor of the transfer work tables (wb_cpu.cpp).
#pragma once
#include <cstddef>

#include "wb_common.h"

namespace wb {
void cpu_execute(const Item* items, size_t n_items, const QuantDesc* qdescs, const QuantWork* qwork,
                 size_t n_qwork);
// Split-block quantisation on the host (the same arithmetic as wb_splitq.cu).
void cpu_split_amax(const SplitPiece* pieces, size_t n, float* partial);
void cpu_split_quant(const SplitPiece* pieces, size_t n, const float* amax);
}  // namespace wb
