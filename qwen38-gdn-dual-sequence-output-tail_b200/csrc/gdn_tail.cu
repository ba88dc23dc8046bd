// Dual-sequence output tail: gated RMSNorm prologue + one flattened out_proj
// GEMM on tcgen05.
//
// Replaces BatchGdnOutputTail (reference provider P:1434-1498; the flattened
// Matmul of patches/0001-feat-qwen38-flatten-dual-tail-output-projection.patch
// :179-184), LaneGdnOutputTailV13 (P:1371-1432) and the single-sequence tail
// (P:3498-3547).  The reference runs RmsNorm, Silu, Mul and Matmul as four
// aclnn operators with four workspace allocations; here the rows of every
// sequence are flattened into one GEMM M = sum of rows, K = Hv*128, N = hidden.
//
// GEMM design (sm_100a): persistent CTAs, one per SM; warp 0 issues TMA
// loads of 128x64 A and BNx64 B tiles (128-byte swizzle) into a 4-stage ring;
// warp 1 issues tcgen05.mma (M=128, N=BN, K=16) from one thread with the f32
// accumulator in TMEM (two accumulators so the epilogue of one tile overlaps
// the main loop of the next); warps 2-5 drain TMEM with tcgen05.ld and store
// bf16.  For M <= 128 (decode rows, the 2x64 tail) the K dimension is split
// over the CTAs of a thread-block cluster that reduce their f32 partial
// tiles through distributed shared memory in split order; for other shapes
// with fewer output tiles than SMs each split writes an f32 partial tile and
// a small pass sums the splits in a fixed order.  Either way the result does
// not depend on scheduling.
#include <vector>

#include "gdn_internal.h"
#include "gdn_tail_gemm.cuh"

namespace gdn {

// ------------------------------------------------------------ prologue --

// gated[r, h*128 + j] = bf16( bf16(o*rstd*gamma) * bf16(SiLU(z)) ); the
// rounding points are the aclnn operator boundaries.  Sixteen threads per
// (row, head), eight elements (16 bytes) each; for large inputs every
// thread takes kPairs (row, head) pairs kPrologueStride apart and issues all
// of their loads before the first use, so more bytes are in flight per
// thread (small inputs keep one pair per thread and twice the blocks).
constexpr int kPrologueStride = 16;          // pairs per block per round (256 threads / 16)
constexpr int64_t kPrologueTwoPairs = 65536; // from this many pairs on, two per thread

template <int kProloguePairs>
__global__ void __launch_bounds__(256)
tail_prologue_kernel(const uint16_t* __restrict__ o, const uint16_t* __restrict__ z,
                     const uint16_t* __restrict__ gamma, uint16_t* __restrict__ gated,
                     int64_t pairs, float eps, uint32_t* __restrict__ clear_err) {
  // Launched to overlap the kernel before it (which writes o): wait for it
  // (a no-op for an ordinary launch).
  griddep_wait();
  // The call's error word starts at zero: cleared here, before the GEMM is
  // let in, instead of by a separate memset (only the GEMM records errors,
  // after a bounded wait of seconds).
  if (clear_err != nullptr && blockIdx.x == 0 && threadIdx.x == 0) *clear_err = 0u;
  griddep_launch_dependents();   // the tail GEMM may start streaming W now
  const int64_t first = static_cast<int64_t>(blockIdx.x) * kPrologueStride * kProloguePairs +
                        (threadIdx.x >> 4);
  const int sub = threadIdx.x & 15;
  uint4 ov[kProloguePairs], zv[kProloguePairs];
  int64_t base[kProloguePairs];
  bool live[kProloguePairs];
#pragma unroll
  for (int i = 0; i < kProloguePairs; ++i) {
    const int64_t pair = first + i * kPrologueStride;
    live[i] = pair < pairs;
    base[i] = (live[i] ? pair : 0) * kHeadDim + sub * 8;
    ov[i] = *reinterpret_cast<const uint4*>(o + base[i]);
    zv[i] = *reinterpret_cast<const uint4*>(z + base[i]);
  }
  const uint4 gv = *reinterpret_cast<const uint4*>(gamma + sub * 8);
  const uint32_t gw[4] = {gv.x, gv.y, gv.z, gv.w};
#pragma unroll
  for (int i = 0; i < kProloguePairs; ++i) {
    const uint32_t ow[4] = {ov[i].x, ov[i].y, ov[i].z, ov[i].w};
    const uint32_t zw[4] = {zv[i].x, zv[i].y, zv[i].z, zv[i].w};
    const float rstd = rsqrtf(gate_sumsq16(ow) * (1.0f / 128.0f) + eps);
    const uint4 res = gate8(ow, zw, gw, rstd);
    if (live[i]) *reinterpret_cast<uint4*>(gated + base[i]) = res;
  }
}

// ---------------------------------------------------------------- GEMM --

// Unit -> output tile.  Units below full_units are whole BM x BN tiles (unit
// = tile * splits + split); when the last wave of tiles would leave SMs idle,
// each remaining tile runs as two BM x BN/2 halves (units full_units + 2 r
// and + 1), so that wave takes about half as long.
struct TileRef {
  int tm, tn, split, col0, width;
};
template <int BN>
__device__ __forceinline__ TileRef tile_of(int unit, int tiles_n, int splits, int full_units) {
  TileRef t;
  int tile, half = -1;
  if (unit < full_units) {
    t.split = unit % splits;
    tile = unit / splits;
  } else {
    t.split = 0;
    tile = full_units / splits + ((unit - full_units) >> 1);
    half = (unit - full_units) & 1;
  }
  t.tn = tile % tiles_n;
  t.tm = tile / tiles_n;
  t.col0 = t.tn * BN + (half > 0 ? BN / 2 : 0);
  t.width = half >= 0 ? BN / 2 : BN;
  return t;
}

template <int BN>
__global__ void __launch_bounds__(kGemmThreads, 1)
tail_gemm_kernel(const __grid_constant__ CUtensorMap tmap_a,
                 const __grid_constant__ CUtensorMap tmap_b,
                 const __grid_constant__ CUtensorMap tmap_b_half, uint16_t* __restrict__ out,
                 float* __restrict__ out_f32, int M, int N, int tiles_m, int tiles_n, int splits,
                 int kblocks_total, int kblocks_per_split, int full_units, int total_units,
                 uint32_t* err) {
  using L = GemmSmem<BN>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::kBarrierOffset);
  uint64_t* empty = full + kGemmStages;
  uint64_t* tfull = empty + kGemmStages;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kGemmStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&tfull[s], 1);
      mbar_init(&tempty[s], 128);
    }
    fence_barrier_init();
    tma_prefetch_desc(&tmap_a);
    tma_prefetch_desc(&tmap_b);
    if (full_units < total_units) tma_prefetch_desc(&tmap_b_half);
  }
  if (warp == 1) tmem_alloc(tmem_slot, 2 * BN);
  tmem_fence_before();
  __syncthreads();
  tmem_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int unit = blockIdx.x; unit < total_units && ok; unit += gridDim.x) {
        const TileRef t = tile_of<BN>(unit, tiles_n, splits, full_units);
        const bool whole = t.width == BN;
        const int kb0 = t.split * kblocks_per_split;
        const int kb1 = min(kb0 + kblocks_per_split, kblocks_total);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, err)) { ok = false; break; }
          mbar_arrive_expect_tx(&full[stage], whole ? L::kStageBytes
                                                    : L::kABytes + L::kBBytes / 2);
          uint8_t* sa = smem + stage * L::kStageBytes;
          tma_load_2d(sa, &tmap_a, &full[stage], kb * kGemmBK, t.tm * kGemmBM);
          tma_load_2d(sa + L::kABytes, whole ? &tmap_b : &tmap_b_half, &full[stage],
                      kb * kGemmBK, t.col0);
          if (++stage == kGemmStages) { stage = 0; phase ^= 1u; }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc_whole = umma_idesc_bf16(kGemmBM, BN, false, false);
      constexpr uint32_t idesc_half = umma_idesc_bf16(kGemmBM, BN / 2, false, false);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int unit = blockIdx.x; unit < total_units && ok; unit += gridDim.x) {
        const TileRef t = tile_of<BN>(unit, tiles_n, splits, full_units);
        const uint32_t idesc = t.width == BN ? idesc_whole : idesc_half;
        const int kb0 = t.split * kblocks_per_split;
        const int kb1 = min(kb0 + kblocks_per_split, kblocks_total);
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1u, err)) break;
        tmem_fence_after();
        const uint32_t d = tmem_base + static_cast<uint32_t>(acc * BN);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full[stage], phase, err)) { ok = false; break; }
          tmem_fence_after();
          const uint32_t sa = smem_u32(smem + stage * L::kStageBytes);
          const uint32_t sb = sa + L::kABytes;
#pragma unroll
          for (int kk = 0; kk < kGemmBK / 16; ++kk) {
            umma_bf16(d, umma_sdesc(sa + kk * 32, 16, 1024), umma_sdesc(sb + kk * 32, 16, 1024),
                      idesc, (kb > kb0 || kk > 0) ? 1u : 0u);
          }
          umma_commit(&empty[stage]);
          if (++stage == kGemmStages) { stage = 0; phase ^= 1u; }
        }
        umma_commit(&tfull[acc]);
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1u;
      }
    }
  } else {
    // Epilogue warps 2..5: warp w drains TMEM lanes 32*(w%4) .. +31.
    const int quarter = warp & 3;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int unit = blockIdx.x; unit < total_units; unit += gridDim.x) {
      const TileRef t = tile_of<BN>(unit, tiles_n, splits, full_units);
      if (!mbar_wait(&tfull[acc], acc_phase, err)) break;
      tmem_fence_after();
      const int row = t.tm * kGemmBM + quarter * 32 + lane;
      const uint32_t tbase = tmem_addr(tmem_base, quarter * 32, acc * BN);
#pragma unroll 1
      for (int c = 0; c < t.width; c += 16) {
        uint32_t r[16];
        tmem_ld16(tbase + c, r);
        tmem_ld_wait();
        if (row < M) {
          const int64_t off = static_cast<int64_t>(row) * N + t.col0 + c;
          if (splits == 1) {
            uint4 w0, w1;
            w0.x = pack_bf16x2(__uint_as_float(r[0]), __uint_as_float(r[1]));
            w0.y = pack_bf16x2(__uint_as_float(r[2]), __uint_as_float(r[3]));
            w0.z = pack_bf16x2(__uint_as_float(r[4]), __uint_as_float(r[5]));
            w0.w = pack_bf16x2(__uint_as_float(r[6]), __uint_as_float(r[7]));
            w1.x = pack_bf16x2(__uint_as_float(r[8]), __uint_as_float(r[9]));
            w1.y = pack_bf16x2(__uint_as_float(r[10]), __uint_as_float(r[11]));
            w1.z = pack_bf16x2(__uint_as_float(r[12]), __uint_as_float(r[13]));
            w1.w = pack_bf16x2(__uint_as_float(r[14]), __uint_as_float(r[15]));
            reinterpret_cast<uint4*>(out + off)[0] = w0;
            reinterpret_cast<uint4*>(out + off)[1] = w1;
          } else {
            // Split-K partial: slice `split` of the [splits, M, N] f32 scratch,
            // summed in a fixed order afterwards (deterministic).
            float4* dst = reinterpret_cast<float4*>(out_f32 + static_cast<int64_t>(t.split) * M * N + off);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              dst[j] = make_float4(__uint_as_float(r[4 * j]), __uint_as_float(r[4 * j + 1]),
                                   __uint_as_float(r[4 * j + 2]), __uint_as_float(r[4 * j + 3]));
            }
          }
        }
      }
      tmem_fence_before();
      mbar_arrive(&tempty[acc]);
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1u;
    }
  }
  tmem_fence_before();
  __syncthreads();
  if (warp == 1) {
    tmem_fence_after();
    tmem_dealloc(tmem_base, 2 * BN);
  }
}

// ------------------------------------------------- split-K in a cluster --
// For M <= 128 (decode rows, the 2x64 dual tail) the K dimension is split
// over the CTAs of one thread-block cluster (one CTA per split, up to 4) and
// N into 64-column tiles, so a 2048-wide output runs as 32 clusters of 4 =
// 128 CTAs, one per SM and all resident at once, each streaming an equal
// share of W (the HBM stream).  Each CTA drains its f32 partial tile from
// TMEM into its own shared memory; after a cluster barrier it pushes row
// slice p of that tile to CTA p of the cluster with one bulk shared->shared
// copy (the bytes are counted on p's mbarrier), and CTA p sums its slice over
// the splits in split order (deterministic) and writes bf16.  No partial
// leaves the SMs and no second kernel runs.
//
// The shape follows measured limits: the SM-to-SM network moves about 25-30
// GB/s per SM, so the exchanged volume ((splits-1)/splits of a 128 x BN f32
// tile) has to stay small, and at most 15 clusters of 8 CTAs of this size are
// resident on a 148-SM B200, so 8-way splits of 128-column tiles would run
// in two waves.
constexpr int kClusterBN = 64;
constexpr int kClusterStages = 8;
constexpr int kClusterMaxSplits = 4;

template <int BN, int Stages>
struct ClusterGemmSmem {
  static constexpr int kPartStride = BN + 4;   // f32 per partial-tile row (padded)
  static constexpr uint32_t kABytes = kGemmBM * kGemmBK * 2;
  static constexpr uint32_t kBBytes = BN * kGemmBK * 2;
  static constexpr uint32_t kStageBytes = kABytes + kBBytes;
  // After the main loop: the partial tile at 0, then the slices received
  // from the other splits ([splits][slice rows][kPartStride], at most one
  // tile's worth: splits * ceil(M / splits) <= 128 for splits dividing 128).
  static constexpr uint32_t kPartBytes = kGemmBM * kPartStride * 4;
  static constexpr uint32_t kRecvOffset = kPartBytes;
  static constexpr uint32_t kBarrierOffset = Stages * kStageBytes;
  static constexpr uint32_t kTotal = kBarrierOffset + 256 + 1024;
  static_assert(2 * kPartBytes <= kBarrierOffset, "partial tile and slices fit the stages");
};

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_size() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(r));
  return r;
}
// Every thread of every CTA of the cluster; the CTAs of a cluster are
// co-scheduled and reach it after bounded work only.
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\t"
               "barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

template <int BN, int Stages>
__global__ void __launch_bounds__(kGemmThreads, 1)
tail_gemm_cluster_kernel(const __grid_constant__ CUtensorMap tmap_a,
                         const __grid_constant__ CUtensorMap tmap_b, uint16_t* __restrict__ out,
                         int M, int N, int kblocks_total, int kblocks_per_split, int weights_first,
                         uint32_t* err) {
  using L = ClusterGemmSmem<BN, Stages>;
  constexpr int kPartStride = L::kPartStride;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::kBarrierOffset);
  uint64_t* empty = full + Stages;
  uint64_t* tfull = empty + Stages;
  uint64_t* recv = tfull + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(recv + 1);
  float* part = reinterpret_cast<float*>(smem);   // reuses the stages once the MMAs are done
  float* slices = reinterpret_cast<float*>(smem + L::kRecvOffset);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t split = cluster_rank();
  const uint32_t splits = cluster_size();
  const int tn = blockIdx.x / splits;
  const int kb0 = static_cast<int>(split) * kblocks_per_split;
  const int kb1 = min(kb0 + kblocks_per_split, kblocks_total);
  // Rows per slice: M spread evenly over the splits.
  const int rows_per = (M + static_cast<int>(splits) - 1) / static_cast<int>(splits);

  if (threadIdx.x == 0) {
    for (int s = 0; s < Stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(tfull, 1);
    mbar_init(recv, 1);
    fence_barrier_init();
    tma_prefetch_desc(&tmap_a);
    tma_prefetch_desc(&tmap_b);
  }
  if (warp == 1) tmem_alloc(tmem_slot, BN);
  tmem_fence_before();
  __syncthreads();
  tmem_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int kb = kb0;
      if (weights_first) {
        // Launched to overlap the kernel before it on the stream, which
        // wrote A but not W: fill the ring's W halves first, then wait for
        // that kernel and load the A halves.
        const int pre = min(Stages, kb1 - kb0);
        for (int i = 0; i < pre; ++i) {
          mbar_arrive_expect_tx(&full[i], L::kStageBytes);
          tma_load_2d(smem + i * L::kStageBytes + L::kABytes, &tmap_b, &full[i],
                      (kb0 + i) * kGemmBK, tn * BN);
        }
        griddep_wait();
        for (int i = 0; i < pre; ++i)
          tma_load_2d(smem + i * L::kStageBytes, &tmap_a, &full[i], (kb0 + i) * kGemmBK, 0);
        kb = kb0 + pre;
        stage = pre % Stages;
        phase = pre == Stages ? 1u : 0u;
      }
      for (; kb < kb1; ++kb) {
        if (!mbar_wait(&empty[stage], phase ^ 1u, err)) break;
        mbar_arrive_expect_tx(&full[stage], L::kStageBytes);
        uint8_t* sa = smem + stage * L::kStageBytes;
        tma_load_2d(sa, &tmap_a, &full[stage], kb * kGemmBK, 0);
        tma_load_2d(sa + L::kABytes, &tmap_b, &full[stage], kb * kGemmBK, tn * BN);
        if (++stage == Stages) { stage = 0; phase ^= 1u; }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_bf16(kGemmBM, BN, false, false);
      int stage = 0;
      uint32_t phase = 0;
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!mbar_wait(&full[stage], phase, err)) break;
        tmem_fence_after();
        const uint32_t sa = smem_u32(smem + stage * L::kStageBytes);
        const uint32_t sb = sa + L::kABytes;
#pragma unroll
        for (int kk = 0; kk < kGemmBK / 16; ++kk)
          umma_bf16(tmem_base, umma_sdesc(sa + kk * 32, 16, 1024), umma_sdesc(sb + kk * 32, 16, 1024),
                    idesc, (kb > kb0 || kk > 0) ? 1u : 0u);
        umma_commit(&empty[stage]);
        if (++stage == Stages) { stage = 0; phase ^= 1u; }
      }
      umma_commit(tfull);   // also covers a split with no k-block
    }
    __syncwarp();
  } else {
    // Warps 2..5: TMEM lanes 32*(w%4) .. +31 -> rows of the partial tile;
    // rows at or beyond M are never summed and are left alone.
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const bool done = mbar_wait(tfull, 0, err);
    tmem_fence_after();
    if (quarter * 32 < M) {
      float* prow = part + row * kPartStride;
      const bool live = done && kb1 > kb0;
#pragma unroll 1
      for (int c = 0; c < BN; c += 16) {
        uint32_t r[16];
        tmem_ld16(tmem_addr(tmem_base, quarter * 32, c), r);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 4; ++j)
          reinterpret_cast<float4*>(prow + c)[j] =
              live ? make_float4(__uint_as_float(r[4 * j]), __uint_as_float(r[4 * j + 1]),
                                 __uint_as_float(r[4 * j + 2]), __uint_as_float(r[4 * j + 3]))
                   : make_float4(0.f, 0.f, 0.f, 0.f);
      }
      fence_proxy_async_smem();   // the bulk copies below read these rows
    }
  }
  cluster_sync_all();   // every partial tile written, every CTA's stages idle

  // Slice p = rows [p * rows_per, +rows_per) of the tile belongs to CTA p
  // (rows at or beyond M ride along and are not written).
  const int r0 = static_cast<int>(split) * rows_per;
  const uint32_t slice_floats = static_cast<uint32_t>(rows_per * kPartStride);
  const uint32_t slice_bytes = slice_floats * 4u;
  if (threadIdx.x == 0) {
    if (r0 < M && splits > 1) mbar_arrive_expect_tx(recv, (splits - 1u) * slice_bytes);
    for (uint32_t p = 0; p < splits; ++p) {
      if (p == split || static_cast<int>(p) * rows_per >= M) continue;
      bulk_push_cluster(cluster_map(smem_u32(slices + split * slice_floats), p),
                        part + p * slice_floats, slice_bytes, cluster_map(smem_u32(recv), p));
    }
  }
  if (r0 < M) {
    const bool got = splits == 1 || mbar_wait(recv, 0, err);
    const int rows = min(rows_per, M - r0);
    for (int idx = threadIdx.x; idx < rows * (BN / 4); idx += kGemmThreads) {
      const int rr = idx / (BN / 4);
      const int c4 = idx % (BN / 4);
      // All splits' values loaded, then the sum in split order.
      float4 v[kClusterMaxSplits];
#pragma unroll
      for (uint32_t s = 0; s < static_cast<uint32_t>(kClusterMaxSplits); ++s) {
        const float* src = (s == split) ? part + (r0 + rr) * kPartStride
                                        : slices + s * slice_floats + rr * kPartStride;
        v[s] = (s < splits) ? reinterpret_cast<const float4*>(src)[c4]
                            : make_float4(0.f, 0.f, 0.f, 0.f);
      }
      float4 acc = v[0];
#pragma unroll
      for (uint32_t s = 1; s < static_cast<uint32_t>(kClusterMaxSplits); ++s) {
        if (s < splits) { acc.x += v[s].x; acc.y += v[s].y; acc.z += v[s].z; acc.w += v[s].w; }
      }
      if (got) {
        uint2 w;
        w.x = pack_bf16x2(acc.x, acc.y);
        w.y = pack_bf16x2(acc.z, acc.w);
        *reinterpret_cast<uint2*>(out + static_cast<int64_t>(r0 + rr) * N + tn * BN + c4 * 4) = w;
      }
    }
  }
  cluster_sync_all();   // every push has landed before any CTA leaves

  tmem_fence_before();
  __syncthreads();
  if (warp == 1) {
    tmem_fence_after();
    tmem_dealloc(tmem_base, BN);
  }
}

// out = bf16(sum over splits of ws[split]) in split order.
__global__ void splitk_reduce_kernel(const float* __restrict__ ws, uint16_t* __restrict__ out,
                                     int64_t n4, int splits) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n4) return;
  float4 acc = reinterpret_cast<const float4*>(ws)[i];
  for (int s = 1; s < splits; ++s) {
    const float4 v = reinterpret_cast<const float4*>(ws)[s * n4 + i];
    acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
  }
  uint2 w;
  w.x = pack_bf16x2(acc.x, acc.y);
  w.y = pack_bf16x2(acc.z, acc.w);
  reinterpret_cast<uint2*>(out)[i] = w;
}

// ------------------------------------------------------------- host side --

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_tiled_fn() {
  static EncodeTiledFn fn = nullptr;
  if (fn == nullptr) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
    }
  }
  return fn;
}

bool make_tmap_bf16(CUtensorMap* map, const void* base, int64_t rows, int64_t cols,
                           int box_rows) {
  EncodeTiledFn fn = encode_tiled_fn();
  if (fn == nullptr) return false;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(cols) * 2};
  cuuint32_t box[2] = {64, static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box,
            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) ==
         CUDA_SUCCESS;
}

struct TailGemmPlan {
  int bn, tiles_m, tiles_n, splits, kblocks_total, kblocks_per_split, grid;
  int full_units, total_units;   // persistent kernel: whole tiles, all units
  bool cluster;   // split-K reduced inside a thread-block cluster (M <= 128)
};

int sm_count() {
  static int count = 0;
  if (count == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    if (cudaDeviceGetAttribute(&count, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
        count <= 0)
      count = 148;
  }
  return count;
}

TailGemmPlan plan_tail_gemm(int64_t M, int N, int K) {
  TailGemmPlan p{};
  if (M <= kGemmBM && N % kClusterBN == 0) {
    // One row tile: N tiles of kClusterBN columns, K split over a cluster of
    // up to kClusterMaxSplits CTAs (the largest power of two that divides
    // the k-blocks).
    p.cluster = true;
    p.bn = kClusterBN;
    p.tiles_m = 1;
    p.tiles_n = N / kClusterBN;
    p.kblocks_total = K / kGemmBK;
    p.splits = 1;
    for (int sp = kClusterMaxSplits; sp >= 2; sp >>= 1) {
      if (p.kblocks_total % sp == 0) { p.splits = sp; break; }
    }
    p.kblocks_per_split = p.kblocks_total / p.splits;
    p.grid = p.tiles_n * p.splits;
    return p;
  }
  p.cluster = false;
  p.bn = (N % 256 == 0) ? 256 : (N % 128 == 0 ? 128 : 64);
  p.tiles_m = static_cast<int>((M + kGemmBM - 1) / kGemmBM);
  p.tiles_n = N / p.bn;
  p.kblocks_total = K / kGemmBK;
  const int sms = sm_count();
  const int tiles = p.tiles_m * p.tiles_n;
  p.splits = 1;
  if (tiles * 2 <= sms) {
    int want = sms / tiles;
    if (want > p.kblocks_total) want = p.kblocks_total;
    // keep at least 2 k-blocks per split so TMA and MMA overlap
    while (want > 1 && p.kblocks_total / want < 2) --want;
    p.splits = want;
  }
  p.kblocks_per_split = (p.kblocks_total + p.splits - 1) / p.splits;
  p.splits = (p.kblocks_total + p.kblocks_per_split - 1) / p.kblocks_per_split;
  const int units = tiles * p.splits;
  p.grid = units < sms ? units : sms;
  p.full_units = units;
  p.total_units = units;
  // A last wave of whole tiles that would fill at most half of the CTAs
  // runs as twice as many half-width tiles instead.
  const int rem = units % p.grid;
  if (p.splits == 1 && p.bn == 256 && units > p.grid && rem > 0 && 2 * rem <= p.grid) {
    p.full_units = units - rem;
    p.total_units = p.full_units + 2 * rem;
  }
  return p;
}

uint64_t tail_gemm_workspace_bytes(int64_t M, int N, int K) {
  const TailGemmPlan p = plan_tail_gemm(M, N, K);
  return (p.splits > 1 && !p.cluster) ? static_cast<uint64_t>(p.splits) * M * N * sizeof(float) : 0;
}

cudaError_t launch_tail_prologue(const uint16_t* o, const uint16_t* z, const uint16_t* gamma,
                                 uint16_t* gated, int64_t rows, int value_heads, float eps,
                                 cudaStream_t stream, uint32_t* clear_err) {
  const int64_t pairs = rows * value_heads;
  if (pairs == 0) return cudaSuccess;
  // Small tails are launched to overlap the kernel before it on the stream
  // (the state pass of a layer): the kernel waits for that grid before it
  // reads o.  (For large tails this measured slower: the 2 x 4096 step
  // 0.389 -> 0.395 ms, and 0.388 -> 0.391 ms with the state pass letting
  // it launch only at its last chunk.)
  cudaLaunchConfig_t cfg = {};
  cfg.blockDim = dim3(256, 1, 1);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pairs < kPrologueTwoPairs ? 1 : 0;
  cudaError_t e;
  if (pairs >= kPrologueTwoPairs) {
    cfg.gridDim = dim3(static_cast<unsigned>((pairs + 2 * kPrologueStride - 1) /
                                             (2 * kPrologueStride)), 1, 1);
    e = cudaLaunchKernelEx(&cfg, tail_prologue_kernel<2>, o, z, gamma, gated, pairs, eps,
                           clear_err);
  } else {
    cfg.gridDim = dim3(static_cast<unsigned>((pairs + kPrologueStride - 1) / kPrologueStride), 1, 1);
    e = cudaLaunchKernelEx(&cfg, tail_prologue_kernel<1>, o, z, gamma, gated, pairs, eps,
                           clear_err);
  }
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e == cudaSuccess) note_launches();
  return e;
}

template <int BN>
static cudaError_t launch_gemm_bn(const CUtensorMap& ta, const CUtensorMap& tb,
                                  const CUtensorMap& tb_half, uint16_t* out, float* ws, int64_t M,
                                  int N, const TailGemmPlan& p, uint32_t* err,
                                  cudaStream_t stream) {
  const uint32_t smem = GemmSmem<BN>::kTotal;
  cudaError_t e = cudaFuncSetAttribute(tail_gemm_kernel<BN>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  tail_gemm_kernel<BN><<<p.grid, kGemmThreads, smem, stream>>>(
      ta, tb, tb_half, out, ws, static_cast<int>(M), N, p.tiles_m, p.tiles_n, p.splits,
      p.kblocks_total, p.kblocks_per_split, p.full_units, p.total_units, err);
  e = cudaGetLastError();
  if (e == cudaSuccess) note_launches();
  return e;
}

// out[M, N] = a[M, K] @ w[N, K]^T  (bf16 in, f32 accumulate, bf16 out).
// ws: f32 [M, N] scratch when the plan splits K (tail_gemm_workspace_bytes).
cudaError_t launch_tail_gemm(const uint16_t* a, const uint16_t* w, uint16_t* out, float* ws,
                             int64_t M, int N, int K, uint32_t* err, cudaStream_t stream,
                             bool overlap_previous) {
  if (M == 0) return cudaSuccess;
  const TailGemmPlan p = plan_tail_gemm(M, N, K);
  CUtensorMap ta, tb;
  if (!make_tmap_bf16(&ta, a, M, K, kGemmBM) || !make_tmap_bf16(&tb, w, N, K, p.bn))
    return cudaErrorInvalidValue;
  if (p.cluster) {
    const uint32_t smem = ClusterGemmSmem<kClusterBN, kClusterStages>::kTotal;
    cudaError_t ec = cudaFuncSetAttribute(tail_gemm_cluster_kernel<kClusterBN, kClusterStages>,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (ec != cudaSuccess) return ec;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(p.grid), 1, 1);
    cfg.blockDim = dim3(kGemmThreads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = static_cast<unsigned>(p.splits);
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = overlap_previous ? 2 : 1;
    ec = cudaLaunchKernelEx(&cfg, tail_gemm_cluster_kernel<kClusterBN, kClusterStages>, ta, tb,
                            out, static_cast<int>(M), N, p.kblocks_total, p.kblocks_per_split,
                            overlap_previous ? 1 : 0, err);
    if (ec == cudaSuccess) note_launches();
    return ec;
  }
  // Half-width B tiles for a split last wave (the same map when unused).
  CUtensorMap tb_half = tb;
  if (p.total_units > p.full_units && !make_tmap_bf16(&tb_half, w, N, K, p.bn / 2))
    return cudaErrorInvalidValue;
  cudaError_t e =
      (p.bn == 256)   ? launch_gemm_bn<256>(ta, tb, tb_half, out, ws, M, N, p, err, stream)
      : (p.bn == 128) ? launch_gemm_bn<128>(ta, tb, tb_half, out, ws, M, N, p, err, stream)
                      : launch_gemm_bn<64>(ta, tb, tb_half, out, ws, M, N, p, err, stream);
  if (e != cudaSuccess) return e;
  if (p.splits > 1) {
    const int64_t n4 = M * N / 4;
    splitk_reduce_kernel<<<static_cast<unsigned>((n4 + 255) / 256), 256, 0, stream>>>(ws, out, n4,
                                                                                   p.splits);
    e = cudaGetLastError();
    if (e == cudaSuccess) note_launches();
  }
  return e;
}

}  // namespace gdn
