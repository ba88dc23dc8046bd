// plan_probe.cpp -- exhaustive truth tables of the admission plans, feature
// predicates, the chunk-vs-recurrent rule and the graph-row COPY binding.
//
// TEST INFRASTRUCTURE ONLY.  Built twice by oracle/Makefile:
//  * with -DPROBE_REFERENCE against the reference's own headers where they
//    lie (native/include/statecentric/qwen38_gdn_dual_sequence_tail_policy.h,
//    qwen38_gdn_geometry_policy.h, qwen38_gdn_graph_binding.h; the last one
//    through oracle/ref_shim/ against this repository's reconstruction of the
//    provider ABI header, so the reconstructed layout_workspace_v1 has to
//    provide every field the reference reads), into oracle/_ref/;
//  * against this build's csrc/gdn_plan.h and csrc/gdn_graph_binding.h.
// tests/test_native_host.py runs both and requires identical output.
// Every line is a case and its answer; the graph-binding cases record the
// refusal message or every copy (destination, bytes, source) in order.
#include <cstdint>
#include <cstdio>
#include <span>
#include <stdexcept>
#include <string>
#include <vector>

#ifdef PROBE_REFERENCE
#include "statecentric/qwen38_gdn_dual_sequence_tail_policy.h"
#include "statecentric/qwen38_gdn_geometry_policy.h"
#include "statecentric/qwen38_gdn_graph_binding.h"
#else
#include "gdn_graph_binding.h"
#include "gdn_plan.h"
#endif

using namespace statecentric;

namespace {

uint64_t g_hash = 1469598103934665603ull;
void mix(uint64_t v) {
  for (int i = 0; i < 8; ++i) {
    g_hash ^= (v >> (8 * i)) & 0xFF;
    g_hash *= 1099511628211ull;
  }
}

struct Copy {
  uintptr_t dst;
  uint64_t bytes;
  uintptr_t src;
};

// The binding under test: nullptr on success (copies in `out`), else the
// refusal message.
std::string bind(const statecentric_qwen38_gdn_layout_workspace_v1& layout, size_t batch,
                 uint64_t conv_bytes, uint64_t rec_bytes, uintptr_t packed_conv,
                 uintptr_t packed_rec, bool gather, std::vector<Copy>* out) {
  auto copy = [&](uintptr_t d, uint64_t b, uintptr_t s) { out->push_back({d, b, s}); };
#ifdef PROBE_REFERENCE
  try {
    CopyQwen38GdnGraphRows(layout, batch, conv_bytes, rec_bytes, packed_conv, packed_rec,
                           gather, copy);
  } catch (const std::runtime_error& e) {
    return e.what();
  }
  return "";
#else
  const char* why = gdn_b200::CopyGraphRows(layout, batch, conv_bytes, rec_bytes, packed_conv,
                                            packed_rec, gather, copy);
  return why ? why : "";
#endif
}

bool slots_match(std::span<const uintptr_t> a, std::span<const uintptr_t> b, bool direct) {
#ifdef PROBE_REFERENCE
  return Qwen38GdnGraphSlotsMatch(a, b, direct);
#else
  return gdn_b200::GraphSlotsMatch(a, b, direct);
#endif
}

uint64_t rng_state = 0x9E3779B97F4A7C15ull;
uint64_t next_u64() {
  rng_state += 0x9E3779B97F4A7C15ull;
  uint64_t x = rng_state;
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
  return x ^ (x >> 31);
}

}  // namespace

int main() {
  // Feature predicates over every flag combination.
  for (int m = 0; m < 64; ++m) {
    const bool f[6] = {bool(m & 1), bool(m & 2), bool(m & 4), bool(m & 8), bool(m & 16),
                       bool(m & 32)};
    if (m < 4) std::printf("dual_tail_valid %d -> %d\n", m, Qwen38GdnDualSequenceTailFeaturesValid(f[0], f[1]));
    if (m < 8) {
      std::printf("projection_only_valid %d -> %d\n", m,
                  Qwen38GdnProjectionOnlyTailFeaturesValid(f[0], f[1], f[2]));
      std::printf("constants_required %d -> %d\n", m,
                  Qwen38GdnPackedDecodeConstantsRequired(f[0], f[1], f[2]));
    }
    if (m < 4)
      std::printf("layout_ready %d -> %d\n", m, Qwen38GdnPackedDecodeLayoutReady(f[0], f[1]));
    if (m < 16)
      std::printf("packed_decode_valid %d -> %d\n", m,
                  Qwen38GdnPackedDecodeFeaturesValid(f[0], f[1], f[2], f[3]));
    if (m < 32)
      std::printf("lane_local_valid %d -> %d\n", m,
                  Qwen38GdnLaneLocalPackedDecodeFeaturesValid(f[0], f[1], f[2], f[3], f[4]));
    std::printf("lane_anchored_valid %d -> %d\n", m,
                Qwen38GdnLaneAnchoredPackedDecodeFeaturesValid(f[0], f[1], f[2], f[3], f[4],
                                                               f[5]));
  }

  // Chunk-vs-recurrent rule.
  const uint32_t lens[] = {0u, 1u, 7u, 8u, 9u, 10u, 32u, 63u, 64u, 65u, 128u, 4096u, 0xFFFFFFFFu};
  for (int m = 0; m < 8; ++m)
    for (uint32_t n : lens)
      std::printf("chunk_rule %d %u -> %d\n", m, n,
                  UsePackedSequenceChunkGdn(m & 1, m & 2, m & 4, n));

  // Plans: every gate combination x token-count vectors of length 0-4 over
  // {0, 1, 2, 63, 64, 65, 128} x state counts and totals around them.
  // Admitted cases are printed; every answer goes into the hash.
  const uint32_t vals[] = {0u, 1u, 2u, 63u, 64u, 65u, 128u};
  uint64_t cases = 0, admitted = 0;
  for (int len = 0; len <= 4; ++len) {
    int combos = 1;
    for (int i = 0; i < len; ++i) combos *= 7;
    for (int c = 0; c < combos; ++c) {
      std::vector<uint32_t> counts(len);
      uint64_t sum = 0;
      for (int i = 0, x = c; i < len; ++i, x /= 7) {
        counts[i] = vals[x % 7];
        sum += counts[i];
      }
      const std::span<const uint32_t> span(counts.data(), counts.size());
      const uint64_t states[] = {uint64_t(len), uint64_t(len) + 1, len ? uint64_t(len) - 1 : 3u, 2u};
      const uint64_t totals[] = {sum, sum + 1, sum ? sum - 1 : 5u, 128u, 2u};
      for (int g = 0; g < 16; ++g) {
        for (uint64_t sc : states) {
          for (uint64_t tt : totals) {
            const bool e = g & 1, ms = g & 2, pc = g & 4, bp = g & 8;
            const auto d = PlanQwen38GdnDualSequenceTail(e, ms, pc, bp, sc, tt, span);
            const auto p = PlanQwen38GdnProjectionOnlyTail(e, ms, pc, bp, sc, tt, span);
            const auto k = PlanQwen38GdnPackedDecode(e, ms, pc, bp, sc, tt, span);
            const auto l = PlanQwen38GdnLaneLocalPackedDecode(e, ms, pc, bp, sc, tt, span);
            const auto a = PlanQwen38GdnLaneAnchoredPackedDecode(e, ms, pc, bp, sc, tt, span);
            const uint64_t word =
                uint64_t(d.batch) | uint64_t(d.tokens_per_sequence) << 8 |
                uint64_t(d.batch_rms_norm) << 16 | uint64_t(d.batch_elementwise) << 17 |
                uint64_t(d.batch_output_projection) << 18 | uint64_t(p.batch) << 20 |
                uint64_t(p.tokens_per_sequence) << 24 | uint64_t(p.batch_rms_norm) << 32 |
                uint64_t(p.batch_elementwise) << 33 | uint64_t(p.batch_output_projection) << 34 |
                uint64_t(k.batch) << 36 | uint64_t(k.tokens_per_sequence) << 40 |
                uint64_t(k.packed_recurrent) << 44 | uint64_t(l.batch) << 45 |
                uint64_t(l.tokens_per_sequence) << 48 | uint64_t(l.lane_prepare) << 52 |
                uint64_t(l.packed_recurrent) << 53 | uint64_t(l.lane_output_tail) << 54 |
                uint64_t(a.batch) << 55 | uint64_t(a.tokens_per_sequence) << 58 |
                uint64_t(a.lane_prepare) << 61 | uint64_t(a.packed_recurrent) << 62 |
                uint64_t(a.lane_output_tail) << 63;
            // Every field into the hash on its own (the packed word above is
            // only the printed summary).
            for (uint64_t v : {uint64_t(d.batch), uint64_t(d.tokens_per_sequence),
                               uint64_t(d.batch_rms_norm), uint64_t(d.batch_elementwise),
                               uint64_t(d.batch_output_projection), uint64_t(p.batch),
                               uint64_t(p.tokens_per_sequence), uint64_t(p.batch_rms_norm),
                               uint64_t(p.batch_elementwise),
                               uint64_t(p.batch_output_projection), uint64_t(k.batch),
                               uint64_t(k.tokens_per_sequence), uint64_t(k.packed_recurrent),
                               uint64_t(l.batch), uint64_t(l.tokens_per_sequence),
                               uint64_t(l.lane_prepare), uint64_t(l.packed_recurrent),
                               uint64_t(l.lane_output_tail), uint64_t(a.batch),
                               uint64_t(a.tokens_per_sequence), uint64_t(a.lane_prepare),
                               uint64_t(a.packed_recurrent), uint64_t(a.lane_output_tail)})
              mix(v);
            ++cases;
            if (word != 0) {
              ++admitted;
              std::printf("plan g=%d sc=%llu tt=%llu counts=", g, (unsigned long long)sc,
                          (unsigned long long)tt);
              for (uint32_t v : counts) std::printf("%u,", v);
              std::printf(" -> %016llx\n", (unsigned long long)word);
            }
          }
        }
      }
    }
  }
  std::printf("plans cases=%llu admitted=%llu hash=%016llx\n", (unsigned long long)cases,
              (unsigned long long)admitted, (unsigned long long)g_hash);

  // Slot matching.
  const uintptr_t s1[] = {16, 32, 48}, s2[] = {16, 32, 48}, s3[] = {16, 48, 32};
  for (int direct = 0; direct < 2; ++direct) {
    std::printf("slots %d same=%d permuted=%d shorter=%d empty=%d\n", direct,
                slots_match(s1, s2, direct), slots_match(s1, s3, direct),
                slots_match(std::span<const uintptr_t>(s1, 2), s2, direct),
                slots_match(std::span<const uintptr_t>(), std::span<const uintptr_t>(), direct));
  }

  // COPY binding: structured cases around every acceptance rule plus seeded
  // random layouts.
  const uintptr_t arena = 0x100000;
  for (int i = 0; i < 20000; ++i) {
    statecentric_qwen38_gdn_layout_workspace_v1 L{};
    L.size = sizeof(L);
    L.abi_version = STATECENTRIC_QWEN38_PROVIDER_ABI_V1;
    size_t batch = 1 + next_u64() % 4;
    L.batch_size = static_cast<uint32_t>(batch);
    L.binding_mode = (next_u64() & 1) ? STATECENTRIC_QWEN38_GDN_BINDING_COPY_V1
                                      : STATECENTRIC_QWEN38_GDN_BINDING_DIRECT_V1;
    uint64_t conv = 64 * (1 + next_u64() % 4), rec = 256 * (1 + next_u64() % 4);
    L.arena = arena;
    L.arena_bytes = batch * (conv + rec) + (next_u64() % 3) * 64;
    L.required_arena_bytes = L.arena_bytes;
    L.conv_bytes_per_row = conv;
    L.recurrent_bytes_per_row = rec;
    for (size_t r = 0; r < STATECENTRIC_QWEN38_GDN_GRAPH_MAX_ROWS; ++r) {
      L.conv_row_addresses[r] = arena + r * conv;
      L.recurrent_row_addresses[r] = arena + batch * conv + r * rec;
    }
    uintptr_t pc = 0x900000, pr = 0xA00000;
    bool gather = next_u64() & 1;
    // Break up to two rules, each with probability 1/3 (row indexes stay
    // inside the four-row arrays whatever the batch).
    const auto row = [&](uint64_t x) { return static_cast<size_t>(x % 4); };
    for (int k = 0; k < 2; ++k) {
      switch (next_u64() % 72) {
        case 1: L.size = sizeof(L) - 8; break;
        case 2: L.abi_version = 2; break;
        case 3: batch = 0; break;
        case 4: batch = 5; L.batch_size = 5; break;
        case 5: L.batch_size = static_cast<uint32_t>(batch) + 1; break;
        case 6: L.binding_mode = 0; break;
        case 7: L.binding_mode = 3; break;
        case 8: L.required_arena_bytes += 64; break;
        case 9: L.conv_bytes_per_row += 64; break;
        case 10: L.recurrent_bytes_per_row -= 64; break;
        case 11: pc = 0; break;
        case 12: pr = 0; break;
        case 13: L.arena = 0; break;
        case 14: L.conv_row_addresses[row(next_u64() % (batch ? batch : 1))] += L.arena_bytes; break;
        case 15: L.recurrent_row_addresses[row(next_u64() % (batch ? batch : 1))] = arena - 1; break;
        case 16: L.recurrent_row_addresses[row(batch ? batch - 1 : 0)] = arena + L.arena_bytes - rec + 1; break;
        case 17: L.conv_row_addresses[0] = arena + L.arena_bytes - conv; break;
        case 18: conv = 0; L.conv_bytes_per_row = 0; break;
        case 19: L.arena_bytes = ~uint64_t(0) - 8; L.required_arena_bytes = L.arena_bytes; break;
        case 20: conv = ~uint64_t(0) / 2; L.conv_bytes_per_row = conv; break;
        case 21: pc = ~uintptr_t(0) - 16; break;
        case 22: L.conv_row_addresses[row(batch)] = 0; break;
        case 23: gather = !gather; break;
        default: break;
      }
    }
    std::vector<Copy> copies;
    const std::string why = bind(L, batch, conv, rec, pc, pr, gather, &copies);
    std::printf("bind %d: [%s]", i, why.c_str());
    for (const Copy& c : copies)
      std::printf(" (%llx,%llu,%llx)", (unsigned long long)c.dst, (unsigned long long)c.bytes,
                  (unsigned long long)c.src);
    std::printf("\n");
  }
  return 0;
}
