// Graph-slot binding of the GDN state rows: the B200 counterpart of the
// reference's qwen38_gdn_graph_binding.h (GB.h:15-73), with the same
// acceptance rules and copy order, reporting a reason instead of throwing
// (nothing may throw across the C ABI).
//
// A graph captured with DIRECT binding embeds the exact ordered row addresses
// and can only be replayed against the same rows; a COPY capture runs on
// private packed buffers, so it can be replayed against any rows of the same
// batch width once they are gathered into those buffers (and scattered back
// afterwards).  On B200 the decode kernel can also read every row through a
// device table of row addresses (gdn_b200_decode_step_rows): a graph captured
// that way is rebound by rewriting the table, without copies.
#pragma once

#include <cstddef>
#include <cstdint>
#include <limits>
#include <span>

#include "statecentric_qwen38_provider_api_v1.h"

namespace gdn_b200 {

// DIRECT: the same rows in the same order; COPY: the same batch width.
template <typename CapturedSlot, typename CurrentSlot>
bool GraphSlotsMatch(std::span<const CapturedSlot> captured,
                     std::span<const CurrentSlot> current, bool direct) noexcept {
  if (captured.size() != current.size()) return false;
  if (!direct) return true;
  for (std::size_t i = 0; i < captured.size(); ++i)
    if (!(captured[i] == current[i])) return false;
  return true;
}

// Gathers (gather = true: state rows -> packed buffers) or scatters the conv
// and recurrent rows of a COPY or DIRECT layout through copy(destination,
// bytes, source), row by row, conv row first.  Every row is checked against
// the arena before the first copy is issued.  Returns nullptr on success or
// the reason the binding was refused (then no copy was issued).
template <typename Copy>
const char* CopyGraphRows(const statecentric_qwen38_gdn_layout_workspace_v1& layout,
                          std::size_t batch_size, std::uint64_t conv_bytes,
                          std::uint64_t recurrent_bytes, std::uintptr_t packed_conv,
                          std::uintptr_t packed_recurrent, bool gather, Copy&& copy) {
  // [address, address + bytes) inside [base, base + capacity), without
  // overflowing uintptr_t anywhere.
  const auto inside = [](std::uintptr_t base, std::uint64_t capacity, std::uintptr_t address,
                         std::uint64_t bytes) {
    return base != 0 && address >= base && bytes > 0 && bytes <= capacity &&
           capacity <= std::numeric_limits<std::uintptr_t>::max() - base &&
           address - base <= capacity - bytes;
  };
  const auto max_rows = static_cast<std::size_t>(STATECENTRIC_QWEN38_GDN_GRAPH_MAX_ROWS);
  if (layout.size < sizeof(layout) || layout.abi_version != STATECENTRIC_QWEN38_PROVIDER_ABI_V1 ||
      batch_size == 0 || batch_size > max_rows || layout.batch_size != batch_size ||
      (layout.binding_mode != STATECENTRIC_QWEN38_GDN_BINDING_COPY_V1 &&
       layout.binding_mode != STATECENTRIC_QWEN38_GDN_BINDING_DIRECT_V1) ||
      layout.required_arena_bytes != layout.arena_bytes ||
      layout.conv_bytes_per_row != conv_bytes ||
      layout.recurrent_bytes_per_row != recurrent_bytes ||
      conv_bytes > std::numeric_limits<std::uintptr_t>::max() / batch_size ||
      recurrent_bytes > std::numeric_limits<std::uintptr_t>::max() / batch_size ||
      !inside(packed_conv, batch_size * conv_bytes, packed_conv, conv_bytes) ||
      !inside(packed_recurrent, batch_size * recurrent_bytes, packed_recurrent,
              recurrent_bytes))
    return "Qwen3.8 graph GDN copy binding is invalid";
  for (std::size_t row = 0; row < batch_size; ++row) {
    if (!inside(layout.arena, layout.arena_bytes, layout.conv_row_addresses[row], conv_bytes) ||
        !inside(layout.arena, layout.arena_bytes, layout.recurrent_row_addresses[row],
                recurrent_bytes))
      return "Qwen3.8 graph GDN copy row is out of bounds";
  }
  for (std::size_t row = 0; row < batch_size; ++row) {
    const std::uintptr_t pc = packed_conv + row * conv_bytes;
    const std::uintptr_t pr = packed_recurrent + row * recurrent_bytes;
    const std::uintptr_t sc = layout.conv_row_addresses[row];
    const std::uintptr_t sr = layout.recurrent_row_addresses[row];
    if (gather) {
      copy(pc, conv_bytes, sc);
      copy(pr, recurrent_bytes, sr);
    } else {
      copy(sc, conv_bytes, pc);
      copy(sr, recurrent_bytes, pr);
    }
  }
  return nullptr;
}

}  // namespace gdn_b200
