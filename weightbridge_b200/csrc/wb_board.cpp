// Per-sync handshake words in shared memory, for senders and workers on one host.
//
// A sync needs two notifications per (sender, worker) pair - the sender's "done" (its
// parameters are final; in the pull direction the worker may load them) and the worker's
// "pulled" or "ready" - which otherwise cost a session-store round trip each.  Here every
// notification is a group of 64-bit words in one shared-memory file: the writer stores the
// fields and then the epoch with release ordering; a waiter polls the epoch words with acquire
// loads (spinning, then yielding the core between polls) until all of them reach the target,
// with the GIL released.  Errors do not travel here: they stay in the session store, which the
// caller checks between bounded waits.
#include "wb_board.h"

#include <atomic>
#include <chrono>
#include <cstring>
#include <stdexcept>
#include <thread>

namespace wb {

namespace {
inline std::atomic<int64_t>* word(uint64_t base, int64_t off) {
  return reinterpret_cast<std::atomic<int64_t>*>(base + 8 * static_cast<uint64_t>(off));
}
}  // namespace

void board_publish(uint64_t base, int64_t off, const std::vector<int64_t>& fields, int64_t epoch) {
  if (base == 0 || (base & 7)) throw std::invalid_argument("board: base must be a non-null 8-byte aligned address");
  for (size_t i = 0; i < fields.size(); ++i) word(base, off + 1 + (int64_t)i)->store(fields[i], std::memory_order_relaxed);
  word(base, off)->store(epoch, std::memory_order_release);
}

bool board_wait(uint64_t base, const std::vector<int64_t>& offs, int64_t target, int64_t max_ns) {
  if (base == 0 || (base & 7)) throw std::invalid_argument("board: base must be a non-null 8-byte aligned address");
  using clock = std::chrono::steady_clock;
  const auto t0 = clock::now();
  const auto limit = std::chrono::nanoseconds(max_ns);
  size_t next = 0;
  for (uint64_t polls = 0;; ++polls) {
    while (next < offs.size() && word(base, offs[next])->load(std::memory_order_acquire) >= target) ++next;
    if (next == offs.size()) return true;
    if ((polls & 63) == 0 && clock::now() - t0 >= limit) return false;
    // spin first; then yield the core between polls (a sleep would wake late: the kernel's
    // timer slack rounds short sleeps up to ~50 us, which a sync would pay at every handshake)
    if (polls > 4096) std::this_thread::yield();
  }
}

std::vector<int64_t> board_read(uint64_t base, int64_t off, int64_t n) {
  if (base == 0 || (base & 7)) throw std::invalid_argument("board: base must be a non-null 8-byte aligned address");
  std::vector<int64_t> out(static_cast<size_t>(n));
  const int64_t e = word(base, off)->load(std::memory_order_acquire);
  out[0] = e;
  for (int64_t i = 1; i < n; ++i) out[static_cast<size_t>(i)] = word(base, off + i)->load(std::memory_order_relaxed);
  return out;
}

}  // namespace wb
