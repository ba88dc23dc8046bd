// Tile geometry and host helpers shared by the output-tail GEMM kernels
// (gdn_tail.cu: one GPU; gdn_tail_allreduce.cu: head-parallel ranks with the
// rank reduction fused in).
#pragma once

#include "gdn_common.cuh"

namespace gdn {

constexpr int kGemmBM = 128;
constexpr int kGemmBK = 64;
constexpr int kGemmStages = 4;
constexpr int kGemmThreads = 192;

// Stage ring of a GEMM with BN-wide N tiles: a 128x64 A tile and a BNx64 B
// tile per stage, both 128-byte swizzled K-major as TMA writes them.
template <int BN>
struct GemmSmem {
  static constexpr uint32_t kABytes = kGemmBM * kGemmBK * 2;
  static constexpr uint32_t kBBytes = BN * kGemmBK * 2;
  static constexpr uint32_t kStageBytes = kABytes + kBBytes;
  static constexpr uint32_t kBarrierOffset = kGemmStages * kStageBytes;
  static constexpr uint32_t kTotal = kBarrierOffset + 256 + 1024;  // + alignment slack
};

// Row-major bf16 matrix [rows, cols] (cols contiguous), box [box_rows, 64]
// with 128-byte swizzle; rows beyond the matrix read as zero.
bool make_tmap_bf16(CUtensorMap* map, const void* base, int64_t rows, int64_t cols,
                    int box_rows);

// Streaming multiprocessors of the current device.
int sm_count();

}  // namespace gdn
