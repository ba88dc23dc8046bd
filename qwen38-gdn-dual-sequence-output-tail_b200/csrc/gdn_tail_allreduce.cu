// Head-parallel output tail with the rank reduction fused into the GEMM.
//
// With the value heads split over W GPUs (rank r holds Hv/W heads and the
// matching K columns of w_out), each rank's tail GEMM yields a partial
// [rows, hidden] that has to be summed over the ranks.  The reference hands
// this rank-partial to its engine (provider P:3541-3547), which all-reduces
// it after the operator.  Here the sum happens inside the GEMM kernel, over
// NVLink peer memory, tile by tile, while the tensor cores work on the next
// tile:
//
//  * Output tile t (128 rows x 256 columns) is owned by rank
//    (t / grid) % W, so along each CTA's tile sequence the owner rotates.
//  * A rank that does not own t rounds its partial to bf16 and writes it
//    with coalesced 16-byte stores through the NVLink mapping into the
//    owner's staging area, then raises one flag per (tile, rank, epilogue
//    warp) with a system-scope release.
//  * On the owner the TMA warp waits for those flags, loads each staged
//    partial by TMA from its own memory, and the MMA warp adds it to the f32
//    TMEM accumulator with identity-matrix MMAs (D[:, n] += P[:, n], one
//    nonzero product per element, so exact before the f32 rounding), in rank
//    order.  The epilogue rounds once and writes the tile to every rank's
//    output.
//  * At the end every CTA meets the CTAs with the same index on the other
//    ranks (done flags): when the kernel has finished on a rank, every peer
//    has written its share of that rank's output and has stopped reading
//    this call's staging.
//
// out = bf16( f32(owner's partial) + sum over the other ranks, in rank
// order, of bf16(their partial) ), the same bits on every rank and
// deterministic.  Each rank sends 2 (W-1)/W of the output over NVLink (the
// volume of a reduce-scatter plus all-gather) while its main loops run.
//
// Waits are bounded (2 s) like every wait in this library.  Kernels on
// different ranks wait for one another, so one launch per GPU: every rank
// enqueues this kernel with the same rows, hidden, grid and epoch.
#include "gdn_internal.h"
#include "gdn_tail_gemm.cuh"

namespace gdn {

namespace {

constexpr int kArBN = 256;
constexpr uint32_t kArTileBytes = kGemmBM * kArBN * 2;  // one bf16 output tile

struct ArSmem {
  using G = GemmSmem<kArBN>;
  static constexpr uint32_t kStageBytes = G::kStageBytes;
  static constexpr uint32_t kABytes = G::kABytes;
  // 64x64 bf16 identity, K-major 128-byte swizzled (B operand of the
  // reduction MMAs).
  static constexpr uint32_t kIdentOffset = kGemmStages * kStageBytes;
  // Per epilogue warp: 32 rows x 64 columns of bf16 on their way out.
  static constexpr uint32_t kStagingOffset = kIdentOffset + 64 * 64 * 2;
  static constexpr uint32_t kBarrierOffset = kStagingOffset + 4 * 32 * 128;
  static constexpr uint32_t kTotal = kBarrierOffset + 256 + 1024;
};
static_assert(ArSmem::kTotal <= 232448, "shared memory budget");

struct ArParams {
  int rank, M, N, tiles_n, total_tiles, kblocks;
  uint32_t epoch;
  uint64_t staging_off, flags_off, done_off;
};

__device__ __forceinline__ uint32_t* tile_flag(uint8_t* region, const ArParams& p, int world,
                                               int tile, int src, int warp) {
  return reinterpret_cast<uint32_t*>(region + p.flags_off) +
         ((static_cast<uint64_t>(tile) * world + src) * 4 + warp);
}
__device__ __forceinline__ uint32_t* done_flag(uint8_t* region, const ArParams& p, int world,
                                               int cta, int src) {
  return reinterpret_cast<uint32_t*>(region + p.done_off) +
         (static_cast<uint64_t>(cta) * world + src);
}

template <int W>
__global__ void __launch_bounds__(kGemmThreads, 1)
tail_gemm_allreduce_kernel(const __grid_constant__ CUtensorMap tmap_a,
                           const __grid_constant__ CUtensorMap tmap_b,
                           const __grid_constant__ CUtensorMap tmap_stage,
                           const __grid_constant__ TailPeerRegions peers,
                           const __grid_constant__ ArParams p, uint32_t* err) {
  using L = ArSmem;
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
  uint8_t* const mine = peers.region[p.rank];

  // Identity operand: element (n, k) = (n == k), 8 bf16 per 16-byte chunk.
  for (int i = threadIdx.x; i < 64 * 8; i += blockDim.x) {
    const int n = i >> 3, kc = i & 7;
    uint32_t w4[4] = {0u, 0u, 0u, 0u};
    if ((n >> 3) == kc) w4[(n & 7) >> 1] = (n & 1) ? 0x3F800000u : 0x00003F80u;
    *reinterpret_cast<uint4*>(smem + L::kIdentOffset + (n >> 3) * 1024 + (n & 7) * 128 +
                              (((kc ^ n) & 7) << 4)) = make_uint4(w4[0], w4[1], w4[2], w4[3]);
  }
  fence_proxy_async_smem();
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
    if (W > 1) tma_prefetch_desc(&tmap_stage);
  }
  if (warp == 1) tmem_alloc(tmem_slot, 2 * kArBN);
  tmem_fence_before();
  __syncthreads();
  tmem_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // Producer: the K blocks of every tile; for an owned tile, after the
      // other ranks' flags, the 4 column blocks of each staged partial.
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int unit = blockIdx.x; unit < p.total_tiles && ok; unit += gridDim.x) {
        const int tn = unit % p.tiles_n;
        const int tm = unit / p.tiles_n;
        const int round = unit / gridDim.x;
        for (int kb = 0; kb < p.kblocks; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, err)) { ok = false; break; }
          mbar_arrive_expect_tx(&full[stage], L::kStageBytes);
          uint8_t* sa = smem + stage * L::kStageBytes;
          tma_load_2d(sa, &tmap_a, &full[stage], kb * kGemmBK, tm * kGemmBM);
          tma_load_2d(sa + L::kABytes, &tmap_b, &full[stage], kb * kGemmBK, tn * kArBN);
          if (++stage == kGemmStages) { stage = 0; phase ^= 1u; }
        }
        if (!ok || W == 1 || round % W != p.rank) continue;
        const int64_t slot = static_cast<int64_t>(round / W) * gridDim.x + blockIdx.x;
        for (int src = 0; src < W && ok; ++src) {
          if (src == p.rank) continue;
          for (int w = 0; w < 4 && ok; ++w)
            ok = wait_flag_reached(tile_flag(mine, p, W, unit, src, w), p.epoch, err);
          if (!ok) break;
          fence_proxy_async_global();
          const int row0 = static_cast<int>((slot * W + src) * kGemmBM);
          for (int cb = 0; cb < 4; ++cb) {
            if (!mbar_wait(&empty[stage], phase ^ 1u, err)) { ok = false; break; }
            mbar_arrive_expect_tx(&full[stage], L::kABytes);
            tma_load_2d(smem + stage * L::kStageBytes, &tmap_stage, &full[stage], cb * 64, row0);
            if (++stage == kGemmStages) { stage = 0; phase ^= 1u; }
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_bf16(kGemmBM, kArBN, false, false);
      constexpr uint32_t idesc64 = umma_idesc_bf16(kGemmBM, 64, false, false);
      const uint32_t ident = smem_u32(smem + L::kIdentOffset);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int unit = blockIdx.x; unit < p.total_tiles && ok; unit += gridDim.x) {
        const int round = unit / gridDim.x;
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1u, err)) break;
        tmem_fence_after();
        const uint32_t d = tmem_base + static_cast<uint32_t>(acc * kArBN);
        for (int kb = 0; kb < p.kblocks; ++kb) {
          if (!mbar_wait(&full[stage], phase, err)) { ok = false; break; }
          tmem_fence_after();
          const uint32_t sa = smem_u32(smem + stage * L::kStageBytes);
          const uint32_t sb = sa + L::kABytes;
#pragma unroll
          for (int kk = 0; kk < kGemmBK / 16; ++kk) {
            umma_bf16(d, umma_sdesc(sa + kk * 32, 16, 1024), umma_sdesc(sb + kk * 32, 16, 1024),
                      idesc, (kb > 0 || kk > 0) ? 1u : 0u);
          }
          umma_commit(&empty[stage]);
          if (++stage == kGemmStages) { stage = 0; phase ^= 1u; }
        }
        if (ok && W > 1 && round % W == p.rank) {
          // D[:, 64 cb + n] += P_src[:, 64 cb + n], sources in rank order.
          for (int src = 0; src < W && ok; ++src) {
            if (src == p.rank) continue;
            for (int cb = 0; cb < 4; ++cb) {
              if (!mbar_wait(&full[stage], phase, err)) { ok = false; break; }
              tmem_fence_after();
              const uint32_t sa = smem_u32(smem + stage * L::kStageBytes);
#pragma unroll
              for (int kk = 0; kk < 4; ++kk) {
                umma_bf16(d + static_cast<uint32_t>(cb * 64), umma_sdesc(sa + kk * 32, 16, 1024),
                          umma_sdesc(ident + kk * 32, 16, 1024), idesc64, 1u);
              }
              umma_commit(&empty[stage]);
              if (++stage == kGemmStages) { stage = 0; phase ^= 1u; }
            }
          }
        }
        umma_commit(&tfull[acc]);
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1u;
      }
    }
  } else {
    // Epilogue warps 2..5: warp w drains TMEM lanes 32*(w%4) .. +31, i.e.
    // rows 32*(w%4) .. +31 of the tile, 64 columns per pass through a
    // swizzled shared-memory block so that global stores are row-contiguous
    // (8 lanes x 16 bytes per 128-byte row segment).
    const int q = warp & 3;
    uint8_t* const wst = smem + L::kStagingOffset + q * (32 * 128);
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int unit = blockIdx.x; unit < p.total_tiles; unit += gridDim.x) {
      const int tn = unit % p.tiles_n;
      const int tm = unit / p.tiles_n;
      const int round = unit / gridDim.x;
      const int owner = W == 1 ? 0 : round % W;
      const bool own = owner == p.rank;
      if (!mbar_wait(&tfull[acc], acc_phase, err)) break;
      tmem_fence_after();
      const uint32_t tb = tmem_addr(tmem_base, q * 32, acc * kArBN);
      int rows_valid;
      uint64_t dst_off, stride;
      if (own) {
        const int64_t r0 = static_cast<int64_t>(tm) * kGemmBM + q * 32;
        rows_valid = p.M - r0 < 32 ? static_cast<int>(p.M - r0) : 32;
        dst_off = (static_cast<uint64_t>(r0) * p.N + static_cast<uint64_t>(tn) * kArBN) * 2;
        stride = static_cast<uint64_t>(p.N) * 2;
      } else {
        const int64_t slot = static_cast<int64_t>(round / W) * gridDim.x + blockIdx.x;
        rows_valid = 32;
        dst_off = p.staging_off +
                  (static_cast<uint64_t>(slot * W + p.rank) * kGemmBM + q * 32) * (kArBN * 2);
        stride = kArBN * 2;
      }
#pragma unroll 1
      for (int pass = 0; pass < 4; ++pass) {
        uint32_t r[4][16];
#pragma unroll
        for (int j = 0; j < 4; ++j) tmem_ld16(tb + pass * 64 + j * 16, r[j]);
        tmem_ld_wait();
        uint4* rowp = reinterpret_cast<uint4*>(wst + lane * 128);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          uint4 lo, hi;
          lo.x = pack_bf16x2(__uint_as_float(r[j][0]), __uint_as_float(r[j][1]));
          lo.y = pack_bf16x2(__uint_as_float(r[j][2]), __uint_as_float(r[j][3]));
          lo.z = pack_bf16x2(__uint_as_float(r[j][4]), __uint_as_float(r[j][5]));
          lo.w = pack_bf16x2(__uint_as_float(r[j][6]), __uint_as_float(r[j][7]));
          hi.x = pack_bf16x2(__uint_as_float(r[j][8]), __uint_as_float(r[j][9]));
          hi.y = pack_bf16x2(__uint_as_float(r[j][10]), __uint_as_float(r[j][11]));
          hi.z = pack_bf16x2(__uint_as_float(r[j][12]), __uint_as_float(r[j][13]));
          hi.w = pack_bf16x2(__uint_as_float(r[j][14]), __uint_as_float(r[j][15]));
          rowp[(2 * j) ^ (lane & 7)] = lo;
          rowp[(2 * j + 1) ^ (lane & 7)] = hi;
        }
        __syncwarp();
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int rr = i * 4 + (lane >> 3);
          const int c = lane & 7;
          const uint4 v = reinterpret_cast<const uint4*>(wst + rr * 128)[c ^ (rr & 7)];
          if (rr < rows_valid) {
            const uint64_t off = dst_off + rr * stride + pass * 128 + c * 16;
            if (own) {
#pragma unroll
              for (int dst = 0; dst < W; ++dst)
                *reinterpret_cast<uint4*>(peers.region[dst] + off) = v;
            } else {
              *reinterpret_cast<uint4*>(peers.region[owner] + off) = v;
            }
          }
        }
        __syncwarp();
      }
      tmem_fence_before();
      mbar_arrive(&tempty[acc]);
      if (W > 1 && !own) {
        fence_acq_rel_sys();
        __syncwarp();
        if (lane == 0)
          st_release_sys(tile_flag(peers.region[owner], p, W, unit, p.rank, q), p.epoch);
      }
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1u;
    }
    if (W > 1) {
      // Meet the CTAs with this index on the other ranks.
      fence_acq_rel_sys();
      named_barrier_sync(1, 128);
      if (warp == 2 && lane == 0) {
        for (int dst = 0; dst < W; ++dst)
          if (dst != p.rank)
            st_release_sys(done_flag(peers.region[dst], p, W, blockIdx.x, p.rank), p.epoch);
        for (int src = 0; src < W; ++src)
          if (src != p.rank &&
              !wait_flag_reached(done_flag(mine, p, W, blockIdx.x, src), p.epoch, err))
            break;
      }
    }
  }
  tmem_fence_before();
  __syncthreads();
  if (warp == 1) {
    tmem_fence_after();
    tmem_dealloc(tmem_base, 2 * kArBN);
  }
}

int64_t ar_tiles(int64_t rows, int hidden) {
  return ((rows + kGemmBM - 1) / kGemmBM) * (hidden / kArBN);
}

int ar_grid(int64_t tiles) { return static_cast<int>(tiles < kTailArGrid ? tiles : kTailArGrid); }

template <int W>
cudaError_t launch_ar(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& ts,
                      const TailPeerRegions& peers, const ArParams& p, int grid, uint32_t* err,
                      cudaStream_t stream) {
  const uint32_t smem = ArSmem::kTotal;
  cudaError_t e = cudaFuncSetAttribute(tail_gemm_allreduce_kernel<W>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  tail_gemm_allreduce_kernel<W><<<grid, kGemmThreads, smem, stream>>>(ta, tb, ts, peers, p, err);
  return cudaGetLastError();
}

}  // namespace

bool tail_exchange_layout(int64_t max_rows, int hidden, int world, TailExchangeLayout* out) {
  if (max_rows <= 0 || hidden <= 0 || hidden % kArBN != 0 ||
      (world != 1 && world != 2 && world != 4 && world != 8))
    return false;
  const int64_t tiles = ar_tiles(max_rows, hidden);
  const int64_t grid = ar_grid(tiles);
  const int64_t rounds = (tiles + grid - 1) / grid;
  const int64_t slots = ((rounds + world - 1) / world) * grid;
  auto r256 = [](uint64_t x) { return (x + 255u) & ~static_cast<uint64_t>(255u); };
  TailExchangeLayout L{};
  L.out_bytes = static_cast<uint64_t>(max_rows) * hidden * 2;
  L.staging_off = r256(L.out_bytes);
  L.staging_rows = world > 1 ? static_cast<uint64_t>(slots) * world * kGemmBM : 0;
  L.flags_off = L.staging_off + L.staging_rows * kArBN * 2;
  const uint64_t flag_bytes = world > 1 ? r256(static_cast<uint64_t>(tiles) * world * 16) : 0;
  L.done_off = L.flags_off + flag_bytes;
  const uint64_t done_bytes = world > 1 ? r256(static_cast<uint64_t>(kTailArGrid) * world * 4) : 0;
  L.total = L.done_off + done_bytes;
  *out = L;
  return true;
}

cudaError_t launch_tail_gemm_allreduce(const uint16_t* a, const uint16_t* w, int64_t M, int N,
                                       int K, const TailPeerRegions& peers, int rank, int world,
                                       const TailExchangeLayout& layout, uint32_t epoch,
                                       uint32_t* err, cudaStream_t stream) {
  if (M == 0) return cudaSuccess;
  const int64_t tiles = ar_tiles(M, N);
  const int grid = ar_grid(tiles);
  ArParams p{};
  p.rank = rank;
  p.M = static_cast<int>(M);
  p.N = N;
  p.tiles_n = N / kArBN;
  p.total_tiles = static_cast<int>(tiles);
  p.kblocks = K / kGemmBK;
  p.epoch = epoch;
  p.staging_off = layout.staging_off;
  p.flags_off = layout.flags_off;
  p.done_off = layout.done_off;
  CUtensorMap ta, tb, ts;
  if (!make_tmap_bf16(&ta, a, M, K, kGemmBM) || !make_tmap_bf16(&tb, w, N, K, kArBN))
    return cudaErrorInvalidValue;
  if (world > 1) {
    if (!make_tmap_bf16(&ts, peers.region[rank] + layout.staging_off,
                        static_cast<int64_t>(layout.staging_rows), kArBN, kGemmBM))
      return cudaErrorInvalidValue;
  } else {
    ts = ta;  // not read
  }
  switch (world) {
    case 1: return launch_ar<1>(ta, tb, ts, peers, p, grid, err, stream);
    case 2: return launch_ar<2>(ta, tb, ts, peers, p, grid, err, stream);
    case 4: return launch_ar<4>(ta, tb, ts, peers, p, grid, err, stream);
    case 8: return launch_ar<8>(ta, tb, ts, peers, p, grid, err, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace gdn
