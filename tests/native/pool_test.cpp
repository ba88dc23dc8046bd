// Host-only test of CompletedBufferPool with a fake allocator: best-fit reuse,
// budget and per-buffer cap bypasses, quarantine of leases whose work did not
// complete, Close() drain report and Snapshot counters.
#include <cstdlib>
#include <map>

#include "completed_buffer_pool.h"

using statecentric::CompletedBufferPool;

int main() {
  std::map<void*, std::size_t> live;
  bool fail_next = false;
  auto alloc = [&](std::size_t bytes) -> void* {
    if (fail_next) { fail_next = false; return nullptr; }
    void* p = std::malloc(bytes);
    live[p] = bytes;
    return p;
  };
  auto release = [&](void* p) {
    live.erase(p);
    std::free(p);
    return true;
  };
  {
    CompletedBufferPool pool(1000, 600, alloc, release);
    auto a = pool.Borrow(1, 400);
    if (!a || a->bytes != 400) return 1;
    auto b = pool.Borrow(2, 500);
    if (!b) return 2;
    if (pool.Borrow(3, 200)) return 3;            // budget: 900 + 200 > 1000
    if (pool.Borrow(3, 700)) return 4;            // per-buffer cap
    auto s = pool.Snapshot();
    if (s.owned_bytes != 900 || s.active_leases != 2 || s.allocations != 2 ||
        s.budget_bypasses != 2)
      return 5;
    pool.Retire(*a, true);
    auto c = pool.Borrow(4, 300);                 // reuses the 400-byte buffer
    if (!c || c->pointer != a->pointer || pool.Snapshot().reuses != 1) return 6;
    pool.Retire(*b, false);                       // incomplete: quarantined
    s = pool.Snapshot();
    if (s.quarantined_buffers != 1 || s.active_leases != 1) return 7;
    auto d = pool.Borrow(5, 101);                 // 400 in use + 500 quarantined + 101 > budget
    if (d) return 8;
    pool.Retire(*c, true);
    auto e = pool.Borrow(6, 100);                 // best fit: the free 400-byte buffer
    if (!e || e->pointer != a->pointer) return 9;
    pool.Retire(*e, true);
    fail_next = true;
    auto f = pool.Borrow(7, 50);                  // a free buffer serves it: no allocation
    if (!f || !fail_next) return 18;
    fail_next = false;
    pool.Retire(*f, true);
    if (pool.Close()) return 10;                  // quarantine keeps it from draining
    if (pool.Borrow(8, 10)) return 11;            // closed
  }
  {
    CompletedBufferPool pool(1000, 1000, alloc, release);
    auto a = pool.Borrow(1, 300);
    pool.Retire(*a, true);
    auto b = pool.Borrow(2, 800);                 // frees the idle 300 to fit the budget
    if (!b || pool.Snapshot().owned_bytes != 800) return 12;
    pool.Retire(*b, true);
    if (!pool.Close()) return 13;
    if (pool.Snapshot().owned_bytes != 0 || pool.Snapshot().peak_owned_bytes != 800) return 14;
  }
  {
    CompletedBufferPool pool(1000, 1000, alloc, release);
    fail_next = true;
    if (pool.Borrow(1, 10)) return 15;            // allocation failure -> bypass
    if (pool.Snapshot().budget_bypasses != 1) return 16;
  }
  // Everything except the quarantined buffer went back to the allocator.
  return live.size() == 1 ? 0 : 17;
}
