// Shared-memory handshake words (wb_board.cpp).  A slot is a group of int64 words at word
// offset `off` from `base`: word 0 is the slot's epoch, the rest its fields.
#pragma once
#include <cstdint>
#include <vector>

namespace wb {

// Store `fields` into words off+1.. and then `epoch` into word off with release ordering.
void board_publish(uint64_t base, int64_t off, const std::vector<int64_t>& fields, int64_t epoch);
// Wait (acquire loads) until the epoch word of every slot in `offs` is >= `target`; false if
// `max_ns` passed first.
bool board_wait(uint64_t base, const std::vector<int64_t>& offs, int64_t target, int64_t max_ns);
// The epoch (acquire) and the n - 1 field words of one slot.
std::vector<int64_t> board_read(uint64_t base, int64_t off, int64_t n);

}  // namespace wb
