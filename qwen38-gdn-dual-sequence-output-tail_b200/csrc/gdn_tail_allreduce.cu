// Head-parallel output tail with the rank reduction fused into the GEMM.
//
// With the value heads split over W GPUs (rank r holds Hv/W heads and the
// matching K columns of w_out), each rank's tail GEMM yields a partial
// [rows, hidden] that has to be summed over the ranks.  The reference hands
// this rank-partial to its engine (provider P:3541-3547), which all-reduces
// it after the operator.  Here the sum happens inside the GEMM kernel, over
// NVLink peer memory, tile by tile, while the tensor cores work on the next
// tiles:
//
//  * The TMA and MMA warps run the plain persistent GEMM (128 x 256 tiles,
//    4-stage ring, two TMEM accumulators); they never wait for another GPU.
//  * Output tile t is owned by rank (t / grid) % W, so along each CTA's tile
//    sequence the owner rotates.  The epilogue rounds every tile's partial to
//    bf16 and stores it, row-contiguous, into the owner's staging slot for
//    this rank (through the NVLink mapping when the owner is another GPU),
//    releases TMEM, and raises a per-(tile, rank, warp) flag on the owner
//    with a system-scope release.
//  * One tile later the owner's epilogue warps reduce each owned tile: wait
//    for the other ranks' flags, read the W staged partials (this rank's own
//    is staged the same way, locally; 512-byte rows per warp instruction),
//    add them in f32 in rank order, round, and store each row into every
//    rank's output.  TMEM is released before the reduction starts.
//    (Measured on two GPUs: handing the reductions to four extra warps that
//    run beside the epilogue was slower, 268 against 233 us for the
//    16384-row tail, because more NVLink stores were in flight at once and
//    the main loop's TMA loads slowed down more.)
//  * At the end every CTA meets the CTAs with the same index on the other
//    ranks (done flags): when the kernel has finished on a rank, every peer
//    has written its share of that rank's output and has stopped reading
//    this call's staging.
//
// out = bf16( sum over ranks, in rank order, in f32, of bf16(partial) ): the
// same bits on every rank, deterministic, and equal to a bf16 all-reduce of
// the rank-partial outputs with f32 accumulation.  Each rank sends
// 2 (W-1)/W of the output over NVLink (the volume of a reduce-scatter plus an
// all-gather) while its main loops run.
//
// Waits are bounded (2 s) like every wait in this library.  Kernels on
// different ranks wait for one another, so one launch per GPU: every rank
// enqueues this kernel with the same rows, hidden, grid and epoch.
#include "gdn_internal.h"
#include "gdn_tail_gemm.cuh"

namespace gdn {

namespace {

constexpr int kArBN = 256;
// warp 0 TMA, warp 1 MMA, warps 2-5 epilogue and reductions
constexpr int kArThreads = 192;
constexpr uint32_t kArRowBytes = kArBN * 2;                 // one bf16 tile row
constexpr uint32_t kArTileBytes = kGemmBM * kArRowBytes;    // one bf16 tile

struct ArSmem {
  using G = GemmSmem<kArBN>;
  static constexpr uint32_t kStageBytes = G::kStageBytes;
  static constexpr uint32_t kABytes = G::kABytes;
  // Per epilogue warp: 32 rows x 64 columns of bf16 on their way out.
  static constexpr uint32_t kStagingOffset = kGemmStages * kStageBytes;
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

__device__ __forceinline__ void add_bf16x8(float (&s)[8], const uint4& v) {
  s[0] += bf16lo_f32(v.x); s[1] += bf16hi_f32(v.x);
  s[2] += bf16lo_f32(v.y); s[3] += bf16hi_f32(v.y);
  s[4] += bf16lo_f32(v.z); s[5] += bf16hi_f32(v.z);
  s[6] += bf16lo_f32(v.w); s[7] += bf16hi_f32(v.w);
}

// Rows 32q .. 32q+31 of owned tile `tile` (staging slot `slot`), by one
// warp: lane l holds columns 8l .. 8l+7 of a row, so every load and store of
// the warp covers one whole 512-byte row.  RB rows are loaded before any is
// stored (the stores may alias nothing that is loaded, but the compiler
// cannot know that).
template <int W>
__device__ __forceinline__ bool reduce_owned_rows(const TailPeerRegions& peers, const ArParams& p,
                                                  int tile, int64_t slot, int q, int lane,
                                                  uint32_t* err) {
  constexpr int RB = W >= 8 ? 2 : (W >= 4 ? 4 : 8);
  uint8_t* const mine = peers.region[p.rank];
  for (int src = 0; src < W; ++src) {
    if (src != p.rank && !wait_flag_reached(tile_flag(mine, p, W, tile, src, q), p.epoch, err))
      return false;
  }
  const int tn = tile % p.tiles_n;
  const int tm = tile / p.tiles_n;
  const int64_t r0 = static_cast<int64_t>(tm) * kGemmBM + q * 32;
  const int rows = p.M - r0 < 32 ? static_cast<int>(p.M - r0) : 32;
  const uint8_t* stg = mine + p.staging_off + static_cast<uint64_t>(slot) * W * kArTileBytes +
                       static_cast<uint64_t>(q * 32) * kArRowBytes + lane * 16;
  const uint64_t out0 = (static_cast<uint64_t>(r0) * p.N + static_cast<uint64_t>(tn) * kArBN) * 2 +
                        lane * 16;
  const uint64_t out_row = static_cast<uint64_t>(p.N) * 2;
  for (int rb = 0; rb < rows; rb += RB) {
    uint4 v[RB][W];
#pragma unroll
    for (int i = 0; i < RB; ++i) {
#pragma unroll
      for (int src = 0; src < W; ++src)
        v[i][src] = __ldcg(reinterpret_cast<const uint4*>(stg + src * kArTileBytes +
                                                          (rb + i) * kArRowBytes));
    }
#pragma unroll
    for (int i = 0; i < RB; ++i) {
      float s[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int src = 0; src < W; ++src) add_bf16x8(s, v[i][src]);
      const uint4 o = make_uint4(pack_bf16x2(s[0], s[1]), pack_bf16x2(s[2], s[3]),
                                 pack_bf16x2(s[4], s[5]), pack_bf16x2(s[6], s[7]));
      if (rb + i < rows) {
#pragma unroll
        for (int dst = 0; dst < W; ++dst)
          *reinterpret_cast<uint4*>(peers.region[dst] + out0 + (rb + i) * out_row) = o;
      }
    }
  }
  return true;
}

template <int W>
__global__ void __launch_bounds__(kArThreads, 1)
tail_gemm_allreduce_kernel(const __grid_constant__ CUtensorMap tmap_a,
                           const __grid_constant__ CUtensorMap tmap_b,
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
  }
  if (warp == 1) tmem_alloc(tmem_slot, 2 * kArBN);
  tmem_fence_before();
  __syncthreads();
  tmem_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int unit = blockIdx.x; unit < p.total_tiles && ok; unit += gridDim.x) {
        const int tn = unit % p.tiles_n;
        const int tm = unit / p.tiles_n;
        for (int kb = 0; kb < p.kblocks; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, err)) { ok = false; break; }
          mbar_arrive_expect_tx(&full[stage], L::kStageBytes);
          uint8_t* sa = smem + stage * L::kStageBytes;
          tma_load_2d(sa, &tmap_a, &full[stage], kb * kGemmBK, tm * kGemmBM);
          tma_load_2d(sa + L::kABytes, &tmap_b, &full[stage], kb * kGemmBK, tn * kArBN);
          if (++stage == kGemmStages) { stage = 0; phase ^= 1u; }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_bf16(kGemmBM, kArBN, false, false);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int unit = blockIdx.x; unit < p.total_tiles && ok; unit += gridDim.x) {
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
        umma_commit(&tfull[acc]);
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1u;
      }
    }
  } else {
    // Epilogue warps 2..5: warp w drains TMEM lanes 32*(w%4) .. +31, i.e.
    // rows 32*(w%4) .. +31 of the tile, 64 columns per pass through a
    // swizzled shared-memory block so that global stores are row-contiguous
    // (8 lanes x 16 bytes per 128-byte row segment).  With one rank the tile
    // goes straight to the output; otherwise to the owner's staging slot.
    const int q = warp & 3;
    uint8_t* const wst = smem + L::kStagingOffset + q * (32 * 128);
    int acc = 0;
    uint32_t acc_phase = 0;
    int pending = -1;  // owned tile waiting for its reduction
    int64_t pending_slot = 0;
    bool ok = true;
    for (int unit = blockIdx.x; unit < p.total_tiles; unit += gridDim.x) {
      const int tn = unit % p.tiles_n;
      const int tm = unit / p.tiles_n;
      const int round = unit / gridDim.x;
      const int owner = W == 1 ? 0 : round % W;
      const int64_t slot = static_cast<int64_t>(round / W) * gridDim.x + blockIdx.x;
      if (!mbar_wait(&tfull[acc], acc_phase, err)) { ok = false; break; }
      tmem_fence_after();
      const uint32_t tb = tmem_addr(tmem_base, q * 32, acc * kArBN);
      uint8_t* base;
      uint64_t stride;
      int rows_valid;
      if (W == 1) {
        const int64_t r0 = static_cast<int64_t>(tm) * kGemmBM + q * 32;
        rows_valid = p.M - r0 < 32 ? static_cast<int>(p.M - r0) : 32;
        base = peers.region[0] +
               (static_cast<uint64_t>(r0) * p.N + static_cast<uint64_t>(tn) * kArBN) * 2;
        stride = static_cast<uint64_t>(p.N) * 2;
      } else {
        rows_valid = 32;
        base = peers.region[owner] + p.staging_off +
               (static_cast<uint64_t>(slot * W + p.rank) * kGemmBM + q * 32) * kArRowBytes;
        stride = kArRowBytes;
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
          if (rr < rows_valid)
            *reinterpret_cast<uint4*>(base + rr * stride + pass * 128 + c * 16) = v;
        }
        __syncwarp();
      }
      tmem_fence_before();
      mbar_arrive(&tempty[acc]);
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1u;
      if (W == 1) continue;
      if (owner != p.rank) {
        fence_acq_rel_sys();
        __syncwarp();
        if (lane == 0)
          st_release_sys(tile_flag(peers.region[owner], p, W, unit, p.rank, q), p.epoch);
      } else {
        __syncwarp();
      }
      if (pending >= 0) {
        ok = reduce_owned_rows<W>(peers, p, pending, pending_slot, q, lane, err);
        pending = -1;
        if (!ok) break;
      }
      if (owner == p.rank) {
        pending = unit;
        pending_slot = slot;
      }
    }
    if (W > 1 && ok && pending >= 0)
      reduce_owned_rows<W>(peers, p, pending, pending_slot, q, lane, err);
  }
  if (W > 1 && warp >= 2) {
    // Epilogue warps: meet the CTAs with this index on the other ranks.
    fence_acq_rel_sys();
    named_barrier_sync(1, kArThreads - 64);
    if (warp == 2 && lane == 0) {
      uint8_t* const mine = peers.region[p.rank];
      for (int dst = 0; dst < W; ++dst)
        if (dst != p.rank)
          st_release_sys(done_flag(peers.region[dst], p, W, blockIdx.x, p.rank), p.epoch);
      for (int src = 0; src < W; ++src)
        if (src != p.rank &&
            !wait_flag_reached(done_flag(mine, p, W, blockIdx.x, src), p.epoch, err))
          break;
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
cudaError_t launch_ar(const CUtensorMap& ta, const CUtensorMap& tb, const TailPeerRegions& peers,
                      const ArParams& p, int grid, uint32_t* err, cudaStream_t stream) {
  const uint32_t smem = ArSmem::kTotal;
  cudaError_t e = cudaFuncSetAttribute(tail_gemm_allreduce_kernel<W>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  tail_gemm_allreduce_kernel<W><<<grid, kArThreads, smem, stream>>>(ta, tb, peers, p, err);
  e = cudaGetLastError();
  if (e == cudaSuccess) note_launches();
  return e;
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
  CUtensorMap ta, tb;
  if (!make_tmap_bf16(&ta, a, M, K, kGemmBM) || !make_tmap_bf16(&tb, w, N, K, kArBN))
    return cudaErrorInvalidValue;
  switch (world) {
    case 1: return launch_ar<1>(ta, tb, peers, p, grid, err, stream);
    case 2: return launch_ar<2>(ta, tb, peers, p, grid, err, stream);
    case 4: return launch_ar<4>(ta, tb, peers, p, grid, err, stream);
    case 8: return launch_ar<8>(ta, tb, peers, p, grid, err, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace gdn
