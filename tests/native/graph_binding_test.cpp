// Host-only test of the graph-slot binding rules (csrc/gdn_graph_binding.h),
// in the manner of the reference's policy test: a distinct exit code for
// every failing clause.  The copy callable is a fake that records the
// transfers it was asked for.
#include <cstdint>
#include <cstring>
#include <span>
#include <vector>

#include "gdn_graph_binding.h"

namespace {

struct Transfer {
  std::uintptr_t dst;
  std::uint64_t bytes;
  std::uintptr_t src;
};

constexpr std::uintptr_t kArena = 0x100000;
constexpr std::uint64_t kArenaBytes = 1 << 20;
constexpr std::uint64_t kConv = 4096, kRec = 65536;
constexpr std::uintptr_t kPackedConv = 0x900000, kPackedRec = 0xA00000;

statecentric_qwen38_gdn_layout_workspace_v1 Layout(std::uint32_t rows, std::uint32_t mode) {
  statecentric_qwen38_gdn_layout_workspace_v1 l;
  std::memset(&l, 0, sizeof l);
  l.size = sizeof l;
  l.abi_version = STATECENTRIC_QWEN38_PROVIDER_ABI_V1;
  l.batch_size = rows;
  l.binding_mode = mode;
  l.arena = kArena;
  l.arena_bytes = kArenaBytes;
  l.required_arena_bytes = kArenaBytes;
  l.conv_bytes_per_row = kConv;
  l.recurrent_bytes_per_row = kRec;
  for (std::uint32_t r = 0; r < STATECENTRIC_QWEN38_GDN_GRAPH_MAX_ROWS; ++r) {
    l.conv_row_addresses[r] = kArena + r * kConv;
    l.recurrent_row_addresses[r] = kArena + 0x40000 + r * kRec;
  }
  return l;
}

const char* Run(const statecentric_qwen38_gdn_layout_workspace_v1& l, std::size_t rows,
                bool gather, std::vector<Transfer>* log,
                std::uintptr_t packed_conv = kPackedConv, std::uint64_t conv = kConv) {
  return gdn_b200::CopyGraphRows(l, rows, conv, kRec, packed_conv, kPackedRec, gather,
                                 [&](std::uintptr_t d, std::uint64_t b, std::uintptr_t s) {
                                   log->push_back({d, b, s});
                                 });
}

}  // namespace

int main() {
  std::vector<Transfer> log;
  // Gather: conv row then recurrent row, row by row, state -> packed.
  auto l = Layout(3, STATECENTRIC_QWEN38_GDN_BINDING_COPY_V1);
  if (Run(l, 3, true, &log) != nullptr || log.size() != 6) return 1;
  for (int r = 0; r < 3; ++r) {
    const Transfer& c = log[2 * r];
    const Transfer& s = log[2 * r + 1];
    if (c.dst != kPackedConv + r * kConv || c.src != l.conv_row_addresses[r] || c.bytes != kConv)
      return 2;
    if (s.dst != kPackedRec + r * kRec || s.src != l.recurrent_row_addresses[r] || s.bytes != kRec)
      return 3;
  }
  // Scatter: packed -> state, same order.
  log.clear();
  if (Run(l, 3, false, &log) != nullptr || log.size() != 6) return 4;
  if (log[0].dst != l.conv_row_addresses[0] || log[0].src != kPackedConv) return 5;
  // DIRECT layouts expose row addresses too.
  log.clear();
  if (Run(Layout(2, STATECENTRIC_QWEN38_GDN_BINDING_DIRECT_V1), 2, true, &log) != nullptr ||
      log.size() != 4)
    return 6;

  // Refusals, each with no transfer issued.
  struct Case {
    int code;
    statecentric_qwen38_gdn_layout_workspace_v1 layout;
    std::size_t rows;
    std::uintptr_t packed_conv;
    std::uint64_t conv;
    bool row_error;
  };
  std::vector<Case> cases;
  auto base = Layout(2, STATECENTRIC_QWEN38_GDN_BINDING_COPY_V1);
  cases.push_back({10, base, 0, kPackedConv, kConv, false});             // empty batch
  cases.push_back({11, Layout(4, 1), 5, kPackedConv, kConv, false});     // more than four rows
  cases.push_back({12, base, 3, kPackedConv, kConv, false});             // batch size mismatch
  auto bad = base; bad.binding_mode = 7;
  cases.push_back({13, bad, 2, kPackedConv, kConv, false});              // unknown mode
  bad = base; bad.required_arena_bytes = kArenaBytes + 1;
  cases.push_back({14, bad, 2, kPackedConv, kConv, false});              // arena size mismatch
  cases.push_back({15, base, 2, kPackedConv, kConv + 16, false});        // row width mismatch
  cases.push_back({16, base, 2, 0, kConv, false});                       // no packed buffer
  bad = base; bad.abi_version = 2;
  cases.push_back({17, bad, 2, kPackedConv, kConv, false});              // ABI
  bad = base; bad.size = 8;
  cases.push_back({18, bad, 2, kPackedConv, kConv, false});              // struct size
  bad = base; bad.recurrent_row_addresses[1] = kArena + kArenaBytes - kRec + 16;
  cases.push_back({19, bad, 2, kPackedConv, kConv, true});               // row past the arena
  bad = base; bad.conv_row_addresses[0] = kArena - 16;
  cases.push_back({20, bad, 2, kPackedConv, kConv, true});               // row before the arena
  bad = base; bad.arena = 0;
  cases.push_back({21, bad, 2, kPackedConv, kConv, true});               // no arena
  for (const Case& c : cases) {
    log.clear();
    const char* why = Run(c.layout, c.rows, true, &log, c.packed_conv, c.conv);
    if (why == nullptr || !log.empty()) return c.code;
    const bool row_msg = std::strstr(why, "out of bounds") != nullptr;
    if (row_msg != c.row_error) return c.code + 20;
  }

  // Slot matching: DIRECT needs the same rows in the same order, COPY only
  // the same batch width.
  const std::uintptr_t a[3] = {1, 2, 3}, b[3] = {1, 3, 2}, c[2] = {1, 2};
  std::span<const std::uintptr_t> sa(a), sb(b), sc(c);
  if (!gdn_b200::GraphSlotsMatch(sa, sa, true)) return 50;
  if (gdn_b200::GraphSlotsMatch(sa, sb, true)) return 51;
  if (!gdn_b200::GraphSlotsMatch(sa, sb, false)) return 52;
  if (gdn_b200::GraphSlotsMatch(sa, sc, false)) return 53;
  return 0;
}
