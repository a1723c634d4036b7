// CPU executor of the transfer work tables (wb_cpu.cpp).
#pragma once
#include <cstddef>

#include "wb_common.h"

namespace wb {
void cpu_execute(const Item* items, size_t n_items, const QuantDesc* qdescs, const QuantWork* qwork,
                 size_t n_qwork);
}  // namespace wb
