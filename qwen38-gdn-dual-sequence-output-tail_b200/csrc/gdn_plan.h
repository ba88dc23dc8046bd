// Admission planning for GDN submissions.
//
// Two layers:
//  * statecentric::PlanQwen38Gdn* and the *FeaturesValid predicates keep the
//    reference's admission semantics (native/include/statecentric/
//    qwen38_gdn_dual_sequence_tail_policy.h:30-148 and
//    qwen38_gdn_geometry_policy.h:10-16), so a host that reasons about the
//    reference's exact 2x64 dual tail and 1+1 packed decode gets the same
//    answers.  The truth tables are identical by design; the code is this
//    build's own.
//  * PlanGdnB200Submission is what the B200 provider executes: it admits any
//    packed multi-sequence batch.  Every sequence of a batch goes through one
//    chunked-prefill launch (any length, chunk 64) unless every sequence has
//    exactly one token, in which case the packed decode kernel runs; the
//    output tail is always one flattened GEMM over all rows.
#pragma once

#include <cstdint>
#include <span>

namespace statecentric {

struct Qwen38GdnDualSequenceTailPlan {
  std::uint32_t batch = 0;
  std::uint32_t tokens_per_sequence = 0;
  bool batch_rms_norm = false;
  bool batch_elementwise = false;
  bool batch_output_projection = false;
};

struct Qwen38GdnPackedDecodePlan {
  std::uint32_t batch = 0;
  std::uint32_t tokens_per_sequence = 0;
  bool packed_recurrent = false;
};

struct Qwen38GdnLaneLocalPackedDecodePlan {
  std::uint32_t batch = 0;
  std::uint32_t tokens_per_sequence = 0;
  bool lane_prepare = false;
  bool packed_recurrent = false;
  bool lane_output_tail = false;
};

// Feature dependencies: a later feature requires batched projections and
// excludes every earlier exclusive feature.
constexpr bool Qwen38GdnDualSequenceTailFeaturesValid(bool batched_projection_v1,
                                                      bool dual_sequence_tail_v10) {
  return batched_projection_v1 || !dual_sequence_tail_v10;
}

constexpr bool Qwen38GdnProjectionOnlyTailFeaturesValid(bool batched_projection_v1,
                                                        bool dual_sequence_tail_v10,
                                                        bool projection_only_tail_v11) {
  if (!projection_only_tail_v11) return true;
  return batched_projection_v1 && !dual_sequence_tail_v10;
}

constexpr bool Qwen38GdnPackedDecodeFeaturesValid(bool batched_projection_v1,
                                                  bool dual_sequence_tail_v10,
                                                  bool projection_only_tail_v11,
                                                  bool packed_decode_recurrent_v12) {
  if (!packed_decode_recurrent_v12) return true;
  return batched_projection_v1 && !(dual_sequence_tail_v10 || projection_only_tail_v11);
}

constexpr bool Qwen38GdnLaneLocalPackedDecodeFeaturesValid(
    bool batched_projection_v1, bool dual_sequence_tail_v10, bool projection_only_tail_v11,
    bool packed_decode_recurrent_v12, bool lane_local_packed_recurrent_v13) {
  if (!lane_local_packed_recurrent_v13) return true;
  return batched_projection_v1 &&
         !(dual_sequence_tail_v10 || projection_only_tail_v11 || packed_decode_recurrent_v12);
}

constexpr bool Qwen38GdnLaneAnchoredPackedDecodeFeaturesValid(
    bool batched_projection_v1, bool dual_sequence_tail_v10, bool projection_only_tail_v11,
    bool packed_decode_recurrent_v12, bool lane_local_packed_recurrent_v13,
    bool lane_anchored_packed_recurrent_v14) {
  if (!lane_anchored_packed_recurrent_v14) return true;
  return batched_projection_v1 &&
         !(dual_sequence_tail_v10 || projection_only_tail_v11 || packed_decode_recurrent_v12 ||
           lane_local_packed_recurrent_v13);
}

constexpr bool Qwen38GdnPackedDecodeLayoutReady(bool post_conv_pack_v5, bool decode_forward_v1) {
  return decode_forward_v1 || post_conv_pack_v5;
}

constexpr bool Qwen38GdnPackedDecodeConstantsRequired(bool packed_decode_recurrent_v12,
                                                      bool lane_local_packed_recurrent_v13,
                                                      bool lane_anchored_packed_recurrent_v14) {
  return lane_anchored_packed_recurrent_v14 || lane_local_packed_recurrent_v13 ||
         packed_decode_recurrent_v12;
}

namespace detail {
// The reference admits a plan only for exactly two sequences of the given
// per-sequence token count with every gate enabled.
constexpr bool ExactPair(bool enabled, bool multistate, bool post_conv_pack_v5,
                         bool batched_projection_v1, std::uint64_t state_count,
                         std::uint64_t total_tokens, std::span<const std::uint32_t> counts,
                         std::uint32_t per_sequence) {
  if (!(enabled && multistate && post_conv_pack_v5 && batched_projection_v1)) return false;
  if (state_count != 2 || counts.size() != 2) return false;
  if (total_tokens != 2ull * per_sequence) return false;
  return counts[0] == per_sequence && counts[1] == per_sequence;
}
}  // namespace detail

inline Qwen38GdnDualSequenceTailPlan PlanQwen38GdnDualSequenceTail(
    bool enabled, bool multistate, bool post_conv_pack_v5, bool batched_projection_v1,
    std::uint64_t state_count, std::uint64_t total_tokens,
    std::span<const std::uint32_t> token_counts) {
  Qwen38GdnDualSequenceTailPlan plan;
  if (detail::ExactPair(enabled, multistate, post_conv_pack_v5, batched_projection_v1,
                        state_count, total_tokens, token_counts, 64)) {
    plan.batch = 2;
    plan.tokens_per_sequence = 64;
    plan.batch_rms_norm = plan.batch_elementwise = plan.batch_output_projection = true;
  }
  return plan;
}

inline Qwen38GdnDualSequenceTailPlan PlanQwen38GdnProjectionOnlyTail(
    bool enabled, bool multistate, bool post_conv_pack_v5, bool batched_projection_v1,
    std::uint64_t state_count, std::uint64_t total_tokens,
    std::span<const std::uint32_t> token_counts) {
  Qwen38GdnDualSequenceTailPlan plan;
  if (detail::ExactPair(enabled, multistate, post_conv_pack_v5, batched_projection_v1,
                        state_count, total_tokens, token_counts, 64)) {
    plan.batch = 2;
    plan.tokens_per_sequence = 64;
    plan.batch_output_projection = true;
  }
  return plan;
}

inline Qwen38GdnPackedDecodePlan PlanQwen38GdnPackedDecode(
    bool enabled, bool multistate, bool post_conv_pack_v5, bool batched_projection_v1,
    std::uint64_t state_count, std::uint64_t total_tokens,
    std::span<const std::uint32_t> token_counts) {
  Qwen38GdnPackedDecodePlan plan;
  if (detail::ExactPair(enabled, multistate, post_conv_pack_v5, batched_projection_v1,
                        state_count, total_tokens, token_counts, 1)) {
    plan.batch = 2;
    plan.tokens_per_sequence = 1;
    plan.packed_recurrent = true;
  }
  return plan;
}

inline Qwen38GdnLaneLocalPackedDecodePlan PlanQwen38GdnLaneLocalPackedDecode(
    bool enabled, bool multistate, bool post_conv_pack_v5, bool batched_projection_v1,
    std::uint64_t state_count, std::uint64_t total_tokens,
    std::span<const std::uint32_t> token_counts) {
  Qwen38GdnLaneLocalPackedDecodePlan plan;
  if (detail::ExactPair(enabled, multistate, post_conv_pack_v5, batched_projection_v1,
                        state_count, total_tokens, token_counts, 1)) {
    plan.batch = 2;
    plan.tokens_per_sequence = 1;
    plan.lane_prepare = plan.packed_recurrent = plan.lane_output_tail = true;
  }
  return plan;
}

// The anchored variant admits exactly what the lane-local one admits.
inline Qwen38GdnLaneLocalPackedDecodePlan PlanQwen38GdnLaneAnchoredPackedDecode(
    bool enabled, bool multistate, bool post_conv_pack_v5, bool batched_projection_v1,
    std::uint64_t state_count, std::uint64_t total_tokens,
    std::span<const std::uint32_t> token_counts) {
  return PlanQwen38GdnLaneLocalPackedDecode(enabled, multistate, post_conv_pack_v5,
                                            batched_projection_v1, state_count, total_tokens,
                                            token_counts);
}

// Reference chunk-vs-recurrent rule for one packed sequence: its chunk
// operator handles one chunk of 9..64 tokens.
constexpr bool UsePackedSequenceChunkGdn(bool multistate, bool prefill_post_conv_pack_v5,
                                         bool recurrent_prefill_always_recurrent,
                                         std::uint32_t sequence_tokens) {
  if (!multistate || !prefill_post_conv_pack_v5 || recurrent_prefill_always_recurrent)
    return false;
  return sequence_tokens >= 9 && sequence_tokens <= 64;
}

// ------------------------------------------------------------- B200 ----

enum class GdnB200Core : std::uint8_t { kNone = 0, kPackedDecode = 1, kChunked = 2 };

struct GdnB200Plan {
  bool admitted = false;
  GdnB200Core core = GdnB200Core::kNone;
  std::uint32_t sequences = 0;
  std::uint64_t rows = 0;            // flattened output-tail rows
  std::uint64_t chunks = 0;          // chunk-64 work units of the prefill core
  bool flattened_output_tail = false;
};

// token_counts: one entry per sequence (packed in order); max_tokens is the
// create-time limit; max_sequences the kernel table limit.
inline GdnB200Plan PlanGdnB200Submission(std::span<const std::uint32_t> token_counts,
                                         std::uint64_t max_tokens,
                                         std::uint32_t max_sequences) {
  GdnB200Plan plan;
  if (token_counts.empty() || token_counts.size() > max_sequences) return plan;
  std::uint64_t rows = 0, chunks = 0;
  bool all_single = true;
  for (const std::uint32_t n : token_counts) {
    if (n == 0) return plan;
    rows += n;
    chunks += (n + 63u) / 64u;
    all_single = all_single && n == 1;
  }
  if (rows > max_tokens) return plan;
  plan.admitted = true;
  plan.core = all_single ? GdnB200Core::kPackedDecode : GdnB200Core::kChunked;
  plan.sequences = static_cast<std::uint32_t>(token_counts.size());
  plan.rows = rows;
  plan.chunks = all_single ? 0 : chunks;
  plan.flattened_output_tail = true;
  return plan;
}

}  // namespace statecentric
