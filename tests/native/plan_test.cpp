// Host-only truth tables for the admission plans (gdn_plan.h).  The first
// block mirrors the reference's policy test
// (native/tests/qwen38_gdn_dual_sequence_tail_policy_test.cpp): exact 2x64
// dual tail and 1+1 packed decode admitted, ragged and disabled cases
// rejected, each failing clause with its own exit code.  The second block
// covers the B200 planner, which admits any packed batch.
#include <array>
#include <cstdint>
#include <vector>

#include "gdn_plan.h"

using namespace statecentric;

int main() {
  // Feature dependency predicates.
  if (!Qwen38GdnDualSequenceTailFeaturesValid(false, false) ||
      !Qwen38GdnDualSequenceTailFeaturesValid(true, false) ||
      !Qwen38GdnDualSequenceTailFeaturesValid(true, true) ||
      Qwen38GdnDualSequenceTailFeaturesValid(false, true))
    return 1;
  if (!Qwen38GdnProjectionOnlyTailFeaturesValid(false, false, false) ||
      !Qwen38GdnProjectionOnlyTailFeaturesValid(true, false, true) ||
      Qwen38GdnProjectionOnlyTailFeaturesValid(false, false, true) ||
      Qwen38GdnProjectionOnlyTailFeaturesValid(true, true, true))
    return 4;
  if (!Qwen38GdnPackedDecodeFeaturesValid(false, false, false, false) ||
      !Qwen38GdnPackedDecodeFeaturesValid(true, false, false, true) ||
      Qwen38GdnPackedDecodeFeaturesValid(false, false, false, true) ||
      Qwen38GdnPackedDecodeFeaturesValid(true, true, false, true) ||
      Qwen38GdnPackedDecodeFeaturesValid(true, false, true, true))
    return 6;
  if (!Qwen38GdnLaneLocalPackedDecodeFeaturesValid(false, false, false, false, false) ||
      !Qwen38GdnLaneLocalPackedDecodeFeaturesValid(true, false, false, false, true) ||
      Qwen38GdnLaneLocalPackedDecodeFeaturesValid(false, false, false, false, true) ||
      Qwen38GdnLaneLocalPackedDecodeFeaturesValid(true, true, false, false, true) ||
      Qwen38GdnLaneLocalPackedDecodeFeaturesValid(true, false, true, false, true) ||
      Qwen38GdnLaneLocalPackedDecodeFeaturesValid(true, false, false, true, true))
    return 8;
  if (!Qwen38GdnLaneAnchoredPackedDecodeFeaturesValid(false, false, false, false, false, false) ||
      !Qwen38GdnLaneAnchoredPackedDecodeFeaturesValid(true, false, false, false, false, true) ||
      Qwen38GdnLaneAnchoredPackedDecodeFeaturesValid(false, false, false, false, false, true) ||
      Qwen38GdnLaneAnchoredPackedDecodeFeaturesValid(true, true, false, false, false, true) ||
      Qwen38GdnLaneAnchoredPackedDecodeFeaturesValid(true, false, true, false, false, true) ||
      Qwen38GdnLaneAnchoredPackedDecodeFeaturesValid(true, false, false, true, false, true) ||
      Qwen38GdnLaneAnchoredPackedDecodeFeaturesValid(true, false, false, false, true, true))
    return 10;
  if (Qwen38GdnPackedDecodeLayoutReady(false, false) || !Qwen38GdnPackedDecodeLayoutReady(true, false) ||
      !Qwen38GdnPackedDecodeLayoutReady(false, true) || !Qwen38GdnPackedDecodeLayoutReady(true, true))
    return 12;
  if (Qwen38GdnPackedDecodeConstantsRequired(false, false, false) ||
      !Qwen38GdnPackedDecodeConstantsRequired(true, false, false) ||
      !Qwen38GdnPackedDecodeConstantsRequired(false, true, false) ||
      !Qwen38GdnPackedDecodeConstantsRequired(false, false, true))
    return 13;

  // Exact 2x64 dual tail.
  constexpr std::array<std::uint32_t, 2> exact{64, 64};
  constexpr std::array<std::uint32_t, 2> ragged{63, 65};
  const auto admitted = PlanQwen38GdnDualSequenceTail(true, true, true, true, 2, 128, exact);
  if (admitted.batch != 2 || admitted.tokens_per_sequence != 64 || !admitted.batch_rms_norm ||
      !admitted.batch_elementwise || !admitted.batch_output_projection)
    return 2;
  if (PlanQwen38GdnDualSequenceTail(false, true, true, true, 2, 128, exact).batch != 0 ||
      PlanQwen38GdnDualSequenceTail(true, false, true, true, 2, 128, exact).batch != 0 ||
      PlanQwen38GdnDualSequenceTail(true, true, false, true, 2, 128, exact).batch != 0 ||
      PlanQwen38GdnDualSequenceTail(true, true, true, false, 2, 128, exact).batch != 0 ||
      PlanQwen38GdnDualSequenceTail(true, true, true, true, 2, 127, exact).batch != 0 ||
      PlanQwen38GdnDualSequenceTail(true, true, true, true, 2, 128, ragged).batch != 0)
    return 3;
  const auto proj = PlanQwen38GdnProjectionOnlyTail(true, true, true, true, 2, 128, exact);
  if (proj.batch != 2 || proj.tokens_per_sequence != 64 || proj.batch_rms_norm ||
      proj.batch_elementwise || !proj.batch_output_projection ||
      PlanQwen38GdnProjectionOnlyTail(true, true, true, true, 2, 128, ragged).batch != 0)
    return 5;

  // 1 + 1 packed decode.
  constexpr std::array<std::uint32_t, 2> d_exact{1, 1};
  constexpr std::array<std::uint32_t, 2> d_ragged{1, 2};
  const auto pd = PlanQwen38GdnPackedDecode(true, true, true, true, 2, 2, d_exact);
  if (pd.batch != 2 || pd.tokens_per_sequence != 1 || !pd.packed_recurrent ||
      PlanQwen38GdnPackedDecode(false, true, true, true, 2, 2, d_exact).packed_recurrent ||
      PlanQwen38GdnPackedDecode(true, false, true, true, 2, 2, d_exact).packed_recurrent ||
      PlanQwen38GdnPackedDecode(true, true, false, true, 2, 2, d_exact).packed_recurrent ||
      PlanQwen38GdnPackedDecode(true, true, true, false, 2, 2, d_exact).packed_recurrent ||
      PlanQwen38GdnPackedDecode(true, true, true, true, 2, 3, d_ragged).packed_recurrent)
    return 7;
  const auto ll = PlanQwen38GdnLaneLocalPackedDecode(true, true, true, true, 2, 2, d_exact);
  if (ll.batch != 2 || ll.tokens_per_sequence != 1 || !ll.lane_prepare || !ll.packed_recurrent ||
      !ll.lane_output_tail ||
      PlanQwen38GdnLaneLocalPackedDecode(true, true, true, true, 2, 3, d_ragged).packed_recurrent)
    return 9;
  const auto la = PlanQwen38GdnLaneAnchoredPackedDecode(true, true, true, true, 2, 2, d_exact);
  if (la.batch != 2 || !la.lane_prepare || !la.packed_recurrent || !la.lane_output_tail ||
      PlanQwen38GdnLaneAnchoredPackedDecode(true, true, true, true, 2, 3, d_ragged).packed_recurrent)
    return 11;

  // Reference chunk-vs-recurrent rule: 9..64 tokens on the chunk operator.
  if (UsePackedSequenceChunkGdn(true, true, false, 8) || !UsePackedSequenceChunkGdn(true, true, false, 9) ||
      !UsePackedSequenceChunkGdn(true, true, false, 64) || UsePackedSequenceChunkGdn(true, true, false, 65) ||
      UsePackedSequenceChunkGdn(false, true, false, 32) || UsePackedSequenceChunkGdn(true, false, false, 32) ||
      UsePackedSequenceChunkGdn(true, true, true, 32))
    return 14;

  // B200 planner: any packed batch; decode when every sequence has 1 token.
  {
    const std::vector<std::uint32_t> dual{64, 64};
    const auto p = PlanGdnB200Submission(dual, 1 << 20, 1024);
    if (!p.admitted || p.core != GdnB200Core::kChunked || p.rows != 128 || p.chunks != 2 ||
        !p.flattened_output_tail || p.sequences != 2)
      return 20;
    const std::vector<std::uint32_t> rag{63, 65};
    const auto r = PlanGdnB200Submission(rag, 1 << 20, 1024);
    if (!r.admitted || r.core != GdnB200Core::kChunked || r.rows != 128 || r.chunks != 3) return 21;
    std::vector<std::uint32_t> dec(64, 1);
    const auto d = PlanGdnB200Submission(dec, 1 << 20, 1024);
    if (!d.admitted || d.core != GdnB200Core::kPackedDecode || d.rows != 64 || d.chunks != 0)
      return 22;
    const std::vector<std::uint32_t> mixed{1, 2};
    if (PlanGdnB200Submission(mixed, 1 << 20, 1024).core != GdnB200Core::kChunked) return 23;
    const std::vector<std::uint32_t> zero{4, 0};
    if (PlanGdnB200Submission(zero, 1 << 20, 1024).admitted) return 24;
    const std::vector<std::uint32_t> big{4096, 4096};
    if (PlanGdnB200Submission(big, 8191, 1024).admitted) return 25;
    if (!PlanGdnB200Submission(big, 8192, 1024).admitted) return 26;
    std::vector<std::uint32_t> many(1025, 1);
    if (PlanGdnB200Submission(many, 1 << 20, 1024).admitted) return 27;
    if (PlanGdnB200Submission(std::vector<std::uint32_t>{}, 1 << 20, 1024).admitted) return 28;
  }
  return 0;
}
