// CompletedBufferPool: device scratch buffers leased per submission and
// returned when the submission's event is released.
//
// The reference provider includes "statecentric/completed_buffer_pool.h",
// which is not in the reference repository; the contract below is the one its
// call sites rely on (qwen38_geometry_normalized_gdn_provider.cpp):
//   construction with a byte budget, a per-buffer cap and allocate/free
//   callbacks (P:2207-2216); Borrow(owner, bytes) returning a lease or
//   nothing, in which case the caller allocates privately (P:494-503);
//   Retire(lease, completed) at event release, where leases of work that did
//   not complete are quarantined instead of reused (P:551-554);
//   Close() reporting whether everything drained, and Snapshot() with
//   owned/peak bytes, active leases, quarantined buffers, allocations, reuses
//   and budget bypasses (P:2230-2245).
// The allocator callbacks make the pool testable on the host with fakes.
#pragma once

#include <cstddef>
#include <cstdint>
#include <functional>
#include <mutex>
#include <optional>
#include <vector>

namespace statecentric {

class CompletedBufferPool {
 public:
  struct Lease {
    void* pointer = nullptr;
    std::size_t bytes = 0;        // capacity of the leased buffer
    std::uintptr_t owner = 0;
    std::uint64_t id = 0;
  };
  struct Stats {
    std::size_t owned_bytes = 0;
    std::size_t peak_owned_bytes = 0;
    std::size_t active_leases = 0;
    std::size_t quarantined_buffers = 0;
    std::uint64_t allocations = 0;
    std::uint64_t reuses = 0;
    std::uint64_t budget_bypasses = 0;
  };
  using AllocateFn = std::function<void*(std::size_t)>;
  using FreeFn = std::function<bool(void*)>;

  CompletedBufferPool(std::size_t budget_bytes, std::size_t max_buffer_bytes,
                      AllocateFn allocate, FreeFn release)
      : budget_(budget_bytes), max_buffer_(max_buffer_bytes),
        allocate_(std::move(allocate)), free_(std::move(release)) {}

  CompletedBufferPool(const CompletedBufferPool&) = delete;
  CompletedBufferPool& operator=(const CompletedBufferPool&) = delete;
  ~CompletedBufferPool() { Close(); }

  // Smallest free buffer that fits, else a new one within the budget.
  // Returns nothing (and counts a bypass) when the request exceeds the
  // per-buffer cap or the budget, or when the pool is closed.
  std::optional<Lease> Borrow(std::uintptr_t owner, std::size_t bytes) {
    std::scoped_lock lock(mutex_);
    if (closed_ || bytes == 0 || bytes > max_buffer_) {
      ++stats_.budget_bypasses;
      return std::nullopt;
    }
    std::size_t best = free_list_.size();
    for (std::size_t i = 0; i < free_list_.size(); ++i) {
      if (free_list_[i].bytes >= bytes &&
          (best == free_list_.size() || free_list_[i].bytes < free_list_[best].bytes)) {
        best = i;
      }
    }
    if (best != free_list_.size()) {
      Buffer b = free_list_[best];
      free_list_.erase(free_list_.begin() + static_cast<std::ptrdiff_t>(best));
      ++stats_.reuses;
      return Activate(b, owner);
    }
    if (stats_.owned_bytes + bytes > budget_) {
      // Make room by releasing idle buffers before giving up.
      while (!free_list_.empty() && stats_.owned_bytes + bytes > budget_) {
        Buffer b = free_list_.back();
        free_list_.pop_back();
        free_(b.pointer);
        stats_.owned_bytes -= b.bytes;
      }
      if (stats_.owned_bytes + bytes > budget_) {
        ++stats_.budget_bypasses;
        return std::nullopt;
      }
    }
    void* p = allocate_(bytes);
    if (p == nullptr) {
      ++stats_.budget_bypasses;
      return std::nullopt;
    }
    ++stats_.allocations;
    stats_.owned_bytes += bytes;
    if (stats_.owned_bytes > stats_.peak_owned_bytes) stats_.peak_owned_bytes = stats_.owned_bytes;
    return Activate(Buffer{p, bytes}, owner);
  }

  // completed == false quarantines the buffer: the device may still use it.
  void Retire(const Lease& lease, bool completed) {
    std::scoped_lock lock(mutex_);
    for (std::size_t i = 0; i < active_.size(); ++i) {
      if (active_[i].id == lease.id) {
        Buffer b{active_[i].pointer, active_[i].bytes};
        active_.erase(active_.begin() + static_cast<std::ptrdiff_t>(i));
        --stats_.active_leases;
        if (!completed) {
          quarantine_.push_back(b);
          ++stats_.quarantined_buffers;
        } else if (closed_) {
          free_(b.pointer);
          stats_.owned_bytes -= b.bytes;
        } else {
          free_list_.push_back(b);
        }
        return;
      }
    }
  }

  // Frees idle buffers; quarantined buffers are kept (never handed out).
  // Returns true when no lease is active and nothing is quarantined.
  bool Close() {
    std::scoped_lock lock(mutex_);
    closed_ = true;
    for (const Buffer& b : free_list_) {
      free_(b.pointer);
      stats_.owned_bytes -= b.bytes;
    }
    free_list_.clear();
    return active_.empty() && quarantine_.empty();
  }

  Stats Snapshot() const {
    std::scoped_lock lock(mutex_);
    return stats_;
  }

 private:
  struct Buffer {
    void* pointer;
    std::size_t bytes;
  };
  Lease Activate(const Buffer& b, std::uintptr_t owner) {
    Lease l{b.pointer, b.bytes, owner, ++next_id_};
    active_.push_back(l);
    ++stats_.active_leases;
    return l;
  }

  const std::size_t budget_;
  const std::size_t max_buffer_;
  AllocateFn allocate_;
  FreeFn free_;
  mutable std::mutex mutex_;
  bool closed_ = false;
  std::uint64_t next_id_ = 0;
  std::vector<Buffer> free_list_;
  std::vector<Lease> active_;
  std::vector<Buffer> quarantine_;
  Stats stats_;
};

}  // namespace statecentric
