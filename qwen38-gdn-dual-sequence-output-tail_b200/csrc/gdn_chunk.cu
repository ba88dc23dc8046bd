// Chunked (C = 64) gated delta rule for packed variable-length sequences.
//
// Replaces ChunkGdn (reference provider P:1641-1838): there, one chunk of at
// most 64 tokens per call runs as cumsum -> KK^T (AOT) -> 16x16 solve (AOT)
// -> 64x64 merge (AOT) -> W,U (AOT) -> ChunkGatedDeltaRuleFwdH -> ChunkFwdO
// with eight permutes and seventeen allocations, and longer prompts fall back
// to 8-token recurrent slices (run_sequence, P:3387-3469).  Here every chunk
// of every sequence is processed in two launches:
//
//  1. gdn_chunk_prep_kernel, chunk-parallel, one CTA per (chunk, q/k head):
//     L2-norm of k, gating g and beta, in-chunk cumsum G, K K^T on tcgen05,
//     A = beta_i (K K^T)_ij exp(G_i - G_j) (strictly lower) and
//     T = (I + A)^-1 by a blocked 16x16 forward substitution in fp32.  T is
//     stored as a bf16 hi/lo pair, already in the 128-byte-swizzled operand
//     layout the second kernel feeds to tcgen05, with G and beta.
//  2. gdn_chunk_state_kernel, sequential over the chunks of one sequence,
//     one CTA per (sequence, v-head, half of the value dimension); column j
//     of v_new, S and O depends only on column j of S, so the split is exact.
//     A loader warp streams raw q/k/v tiles (TMA) and the prep record (bulk
//     copy) two chunks ahead; four compute warps run per chunk
//       D1 = [K;Q] S            (K S for v_new, Q S for the output)
//       D2 = [K;Q] K^T          (Q K^T for the intra-chunk term)
//       R  = beta (V - exp(G) K S)
//       v_new = T R             (T and R as bf16 hi+lo pairs: ~fp32 accuracy)
//       O  = scale (exp(G) Q S + (Q K^T . Gamma) v_new)
//       S  = exp(G_C) S + K^T (v_new exp(G_C - G))   (v_new as hi+lo pair)
//     with every contraction on tcgen05 (TMEM accumulators) and the f32 state
//     held in registers (thread t owns key row t of its 64 value columns).
//
// The W = T (beta exp(G) K) of the reference is never formed: v_new =
// U - W S = T (beta V - beta exp(G) (K S)) uses one product with T.
// Decay factors are always formed as exp of a non-positive difference.
#include <vector>

#include "gdn_common.cuh"
#include "gdn_internal.h"

namespace gdn {

// Per (chunk, v-head) record written by the prep kernel.
constexpr uint32_t kRecTHi = 0;          // bf16 [64 x 64], K-major SW128 image
constexpr uint32_t kRecTLo = 8192;       // bf16 [64 x 64], K-major SW128 image
constexpr uint32_t kRecG = 16384;        // f32 [64] in-chunk cumsum of g
constexpr uint32_t kRecBeta = 16640;     // f32 [64] beta (bf16 value)
constexpr uint32_t kRecBytes = 16896;

__device__ __forceinline__ int find_seq(const ChunkTable& tab, int chunk) {
  int lo = 0, hi = tab.num_seqs - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (tab.chunk_start[mid] <= chunk) lo = mid; else hi = mid - 1;
  }
  return lo;
}

__device__ __forceinline__ float softplus20(float x) { return x > 20.0f ? x : log1pf(expf(x)); }

// ============================================================ prep =====

constexpr int kPrepThreads = 256;

struct PrepSmem {
  uint8_t ktile[16384];          // K-major SW128 [64 tokens x 128], 2 slabs
  float kk[64][65];              // K K^T
  float amat[2][64][65];         // A, then T, per v-head of the pair
  float xs[2][16][49];           // merge temporaries
  float gs[2][64];
  float bs[2][64];
  uint64_t bar;
  uint32_t tmem;
};

__global__ void __launch_bounds__(kPrepThreads)
gdn_chunk_prep_kernel(const __grid_constant__ ChunkTable tab, const uint16_t* __restrict__ k,
                      const uint16_t* __restrict__ a, const uint16_t* __restrict__ b,
                      const float* __restrict__ A_log, const float* __restrict__ dt_bias,
                      uint8_t* __restrict__ records, int qk_heads, int value_heads,
                      uint32_t* err) {
  extern __shared__ uint8_t smem_raw[];
  PrepSmem& sm = *reinterpret_cast<PrepSmem*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int chunk = blockIdx.x;
  const int kh = blockIdx.y;
  if (chunk >= tab.total_chunks) return;
  const int seq = find_seq(tab, chunk);
  const int t0 = tab.cu[seq] + (chunk - tab.chunk_start[seq]) * kChunk;
  const int n = min(kChunk, tab.cu[seq + 1] - t0);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int group = value_heads / qk_heads;

  if (threadIdx.x == 0) {
    mbar_init(&sm.bar, 1);
    fence_barrier_init();
  }
  if (warp == 0) tmem_alloc(&sm.tmem, 64);

  // k rows -> L2 norm -> bf16 -> swizzled operand tile (zero rows past n).
  const float l2gamma = round_bf16(0.08838834764831845f);
  for (int r = warp; r < kChunk; r += 8) {
    float x[4] = {0.f, 0.f, 0.f, 0.f};
    if (r < n) {
      const uint2 raw = *reinterpret_cast<const uint2*>(
          k + (static_cast<int64_t>(t0 + r) * qk_heads + kh) * kHeadDim + lane * 4);
      x[0] = bf16_bits_to_f32(raw.x & 0xFFFFu);
      x[1] = bf16_bits_to_f32(raw.x >> 16);
      x[2] = bf16_bits_to_f32(raw.y & 0xFFFFu);
      x[3] = bf16_bits_to_f32(raw.y >> 16);
    }
    float ss = x[0] * x[0] + x[1] * x[1] + x[2] * x[2] + x[3] * x[3];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float rstd = rsqrtf(ss * (1.0f / 128.0f) + 1.0e-6f / 128.0f);
    uint2 w;
    w.x = pack_bf16x2(x[0] * rstd * l2gamma, x[1] * rstd * l2gamma);
    w.y = pack_bf16x2(x[2] * rstd * l2gamma, x[3] * rstd * l2gamma);
    *reinterpret_cast<uint2*>(sm.ktile + kmajor_offset(r, lane * 4, 64)) = w;
  }
  fence_proxy_async_smem();
  tmem_fence_before();
  __syncthreads();
  tmem_fence_after();
  const uint32_t tmem = sm.tmem;

  if (threadIdx.x == 0) {
    constexpr uint32_t idesc = umma_idesc_bf16(64, 64, false, false);
    const uint32_t kt = smem_u32(sm.ktile);
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      const uint32_t off = (kk >> 2) * 8192u + (kk & 3) * 32u;
      umma_bf16(tmem, umma_sdesc(kt + off, 16, 1024), umma_sdesc(kt + off, 16, 1024), idesc,
                kk > 0 ? 1u : 0u);
    }
    umma_commit(&sm.bar);
  }

  // Gating for the v-heads of this q/k head, two at a time (warps 0-3 and
  // 4-7), while the MMA runs.
  const int half = threadIdx.x >> 7;   // which v-head of the pair
  const int u = threadIdx.x & 127;

  const bool ok = mbar_wait(&sm.bar, 0, err);
  tmem_fence_after();
  if (ok && warp < 4) {
    // M = 64 accumulator: row m lives in TMEM lane (m % 16) + 32 * (m / 16).
    const uint32_t base = tmem_addr(tmem, warp * 32, 0);
#pragma unroll
    for (int c = 0; c < 64; c += 16) {
      uint32_t r[16];
      tmem_ld16(base + c, r);
      tmem_ld_wait();
      if (lane < 16) {
        const int row = warp * 16 + lane;
#pragma unroll
        for (int j = 0; j < 16; ++j) sm.kk[row][c + j] = __uint_as_float(r[j]);
      }
    }
  }
  tmem_fence_before();
  __syncthreads();

  for (int hp = 0; hp < group; hp += 2) {
    const int hl = hp + half;
    const bool active = ok && hl < group;
    const int h = kh * group + hl;
    float (*T)[65] = sm.amat[half];
    if (active && u < 64) {
      float g = 0.f, bt = 0.f;
      if (u < n) {
        const int64_t gi = static_cast<int64_t>(t0 + u) * value_heads + h;
        g = -expf(A_log[h]) * softplus20(bf16_bits_to_f32(a[gi]) + dt_bias[h]);
        bt = round_bf16(1.0f / (1.0f + expf(-bf16_bits_to_f32(b[gi]))));
      }
      sm.gs[half][u] = g;
      sm.bs[half][u] = bt;
    }
    __syncthreads();
    float gcum = 0.f;
    if (active && u < 64) {
      for (int j = 0; j <= u; ++j) gcum += sm.gs[half][j];
    }
    __syncthreads();
    if (active && u < 64) sm.gs[half][u] = gcum;
    __syncthreads();
    // A (strictly lower, zero past n)
    if (active) {
      for (int e = u; e < 64 * 64; e += 128) {
        const int i = e >> 6, j = e & 63;
        float val = 0.f;
        if (j < i && i < n) val = sm.bs[half][i] * sm.kk[i][j] * expf(sm.gs[half][i] - sm.gs[half][j]);
        T[i][j] = val;
      }
    }
    __syncthreads();
    // Diagonal 16x16 blocks: column c of block bl by forward substitution.
    float x[16];
    if (active && u < 64) {
      const int bl = u >> 4, c = u & 15, o = bl * 16;
#pragma unroll
      for (int r = 0; r < 16; ++r) {
        float acc = (r == c) ? 1.f : 0.f;
#pragma unroll
        for (int m = 0; m < r; ++m) acc -= T[o + r][o + m] * x[m];
        x[r] = acc;
      }
    }
    __syncthreads();  // all reads of the diagonal A blocks are done
    if (active && u < 64) {
      const int bl = u >> 4, c = u & 15, o = bl * 16;
#pragma unroll
      for (int r = 0; r < 16; ++r) T[o + r][o + c] = x[r];
    }
    __syncthreads();
    // Off-diagonal blocks, block row I: T_IJ = -T_II sum_{K=J}^{I-1} A_IK T_KJ.
    // Block row I of A is still intact (only its diagonal block was
    // replaced), block rows < I already hold T.
    for (int I = 1; I < 4; ++I) {
      const int cols = 16 * I;
      if (active) {
        for (int e = u; e < 16 * cols; e += 128) {
          const int r = e / cols, cc = e % cols;   // cc = global column < 16 I
          const int J = cc >> 4;
          float acc = 0.f;
          for (int m = 16 * J; m < 16 * I; ++m) acc += T[16 * I + r][m] * T[m][cc];
          sm.xs[half][r][cc] = acc;
        }
      }
      __syncthreads();
      if (active) {
        for (int e = u; e < 16 * cols; e += 128) {
          const int r = e / cols, cc = e % cols;
          float acc = 0.f;
#pragma unroll
          for (int m = 0; m < 16; ++m) acc += T[16 * I + r][16 * I + m] * sm.xs[half][m][cc];
          T[16 * I + r][cc] = -acc;
        }
      }
      __syncthreads();
    }
    // Upper triangle is zero.
    if (active) {
      for (int e = u; e < 64 * 64; e += 128) {
        const int i = e >> 6, j = e & 63;
        if (j > i) T[i][j] = 0.f;
      }
    }
    __syncthreads();
    // Store T as hi/lo bf16 operand images, plus G and beta.
    if (active) {
      uint8_t* rec = records + (static_cast<int64_t>(chunk) * value_heads + h) * kRecBytes;
      const int row = u >> 1;
      const int cbase = (u & 1) * 32;
#pragma unroll
      for (int q4 = 0; q4 < 4; ++q4) {
        const int c0 = cbase + q4 * 8;
        uint32_t hi[4], lo[4];
#pragma unroll
        for (int p = 0; p < 4; ++p) {
          const float v0 = T[row][c0 + 2 * p], v1 = T[row][c0 + 2 * p + 1];
          const float h0 = round_bf16(v0), h1 = round_bf16(v1);
          hi[p] = pack_bf16x2(h0, h1);
          lo[p] = pack_bf16x2(v0 - h0, v1 - h1);
        }
        const uint32_t off = sw128_chunk(row, c0 >> 3);
        *reinterpret_cast<uint4*>(rec + kRecTHi + off) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
        *reinterpret_cast<uint4*>(rec + kRecTLo + off) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
      }
      if (u < 64) {
        reinterpret_cast<float*>(rec + kRecG)[u] = sm.gs[half][u];
        reinterpret_cast<float*>(rec + kRecBeta)[u] = sm.bs[half][u];
      }
    }
    __syncthreads();
  }
  __syncthreads();
  if (warp == 0) {
    __syncwarp();
    tmem_dealloc(tmem, 64);
  }
}

// =========================================================== state =====

constexpr int kStateThreads = 160;  // warps 0-3 compute, warp 4 loads
constexpr int kDvHalf = 64;

// One load stage: prep record (1024-aligned, holds the T operands), raw q
// and raw k ([64 tokens x 128] bf16 as two 128-byte-swizzled 64-column
// slabs of 8 KB) and raw v ([64 x 64] bf16, one swizzled slab).
constexpr uint32_t kStRec = 0;
constexpr uint32_t kStQ = 17408;
constexpr uint32_t kStK = kStQ + 16384;
constexpr uint32_t kStV = kStK + 16384;
constexpr uint32_t kStageBytes = kStV + 8192;  // 58368, multiple of 1024
constexpr uint32_t kStageTx = kRecBytes + 16384 + 16384 + 8192;

struct StateSmemLayout {
  static constexpr uint32_t kStage0 = 0;
  static constexpr uint32_t kStage1 = kStageBytes;
  static constexpr uint32_t kKQ = 2 * kStageBytes;        // K-major [128 x 128], 32 KB
  static constexpr uint32_t kSop = kKQ + 32768;           // MN-major [128 dk x 64 dv], 16 KB
  static constexpr uint32_t kRhi = kSop + 16384;          // MN-major [64 tok x 64 dv]
  static constexpr uint32_t kRlo = kRhi + 8192;
  static constexpr uint32_t kP = kRlo + 8192;             // K-major [128 x 64]: rows 0-63 zero
  static constexpr uint32_t kVn = kP + 16384;             // MN-major [64 tok x 64 dv]
  static constexpr uint32_t kVdhi = kVn + 8192;
  static constexpr uint32_t kVdlo = kVdhi + 8192;
  static constexpr uint32_t kFactors = kVdlo + 8192;      // f32 G, beta, exp(G), exp(G_C-G)
  static constexpr uint32_t kBars = kFactors + 4 * 64 * 4;
  static constexpr uint32_t kTotal = kBars + 64 + 1024;
};

// TMEM columns: D1 [K;Q] S, D2 [K;Q] K^T, D3 T R (M=64), D4 [0;P] v_new,
// D5 K^T Vd.
constexpr uint32_t kTmD1 = 0, kTmD2 = 64, kTmD3 = 128, kTmD4 = 192, kTmD5 = 256;

__device__ __forceinline__ void named_barrier_compute() {
  asm volatile("bar.sync 1, 128;" ::: "memory");
}

// Wait used by the four compute warps: thread 0 waits (bounded), the result
// is broadcast through shared memory behind the compute barrier, so every
// compute thread takes the same branch and no thread is left at a barrier.
__device__ __forceinline__ bool compute_wait(uint64_t* bar, uint32_t parity, uint32_t* err,
                                             volatile uint32_t* flag) {
  if (threadIdx.x == 0) *flag = mbar_wait(bar, parity, err) ? 1u : 0u;
  named_barrier_compute();
  return *flag != 0u;
}

__global__ void __launch_bounds__(kStateThreads, 1)
gdn_chunk_state_kernel(const __grid_constant__ ChunkTable tab,
                       const __grid_constant__ CUtensorMap tm_q,
                       const __grid_constant__ CUtensorMap tm_k,
                       const __grid_constant__ CUtensorMap tm_v,
                       const uint8_t* __restrict__ records, float* __restrict__ state,
                       uint16_t* __restrict__ o_out, int qk_heads, int value_heads,
                       uint32_t* err) {
  using L = StateSmemLayout;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::kBars);
  uint64_t* empty = full + 2;
  uint64_t* mma_bar = empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_bar + 1);
  volatile uint32_t* wait_flag = tmem_slot + 1;
  float* fG = reinterpret_cast<float*>(smem + L::kFactors);
  float* fB = fG + 64;
  float* fEG = fB + 64;
  float* fED = fEG + 64;

  const int dvh = blockIdx.x;          // which half of the value dim
  const int h = blockIdx.y;
  const int seq = blockIdx.z;
  const int kh = h / (value_heads / qk_heads);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int tid = threadIdx.x;
  const int seq_t0 = tab.cu[seq];
  const int seq_len = tab.cu[seq + 1] - seq_t0;
  const int nchunks = (seq_len + kChunk - 1) / kChunk;
  const int chunk0 = tab.chunk_start[seq];

  if (tid == 0) {
    mbar_init(&full[0], 1);
    mbar_init(&full[1], 1);
    mbar_init(&empty[0], 1);
    mbar_init(&empty[1], 1);
    mbar_init(mma_bar, 1);
    fence_barrier_init();
    tma_prefetch_desc(&tm_q);
    tma_prefetch_desc(&tm_k);
    tma_prefetch_desc(&tm_v);
  }
  if (warp == 0) tmem_alloc(tmem_slot, 512);
  tmem_fence_before();
  __syncthreads();
  tmem_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 4) {
    // ------------------------------------------------------ loader warp --
    if (lane == 0) {
      int issued = 0;
      for (int c = 0; c < nchunks; ++c) {
        const int st = c & 1;
        const uint32_t par = ((c >> 1) & 1) ^ 1u;
        if (!mbar_wait(&empty[st], par, err)) break;
        uint8_t* sbase = smem + (st ? L::kStage1 : L::kStage0);
        const int t0 = seq_t0 + c * kChunk;
        mbar_arrive_expect_tx(&full[st], kStageTx);
        bulk_load(sbase + kStRec,
                  records + (static_cast<int64_t>(chunk0 + c) * value_heads + h) * kRecBytes,
                  kRecBytes, &full[st]);
        // 3-D maps {d, head, token}, box {64, 1, 64}, 128-byte swizzle:
        // q and k land as two 64-column slabs, v as one.
        const uint32_t fb = smem_u32(&full[st]);
        const uint64_t mq = reinterpret_cast<uint64_t>(&tm_q);
        const uint64_t mk = reinterpret_cast<uint64_t>(&tm_k);
        const uint64_t mv = reinterpret_cast<uint64_t>(&tm_v);
#pragma unroll
        for (int sl = 0; sl < 2; ++sl) {
          asm volatile(
              "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
              " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(sbase + kStQ + sl * 8192)),
              "l"(mq), "r"(fb), "r"(sl * 64), "r"(kh), "r"(t0)
              : "memory");
          asm volatile(
              "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
              " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(sbase + kStK + sl * 8192)),
              "l"(mk), "r"(fb), "r"(sl * 64), "r"(kh), "r"(t0)
              : "memory");
        }
        asm volatile(
            "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
            " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(sbase + kStV)),
            "l"(mv), "r"(fb), "r"(dvh * kDvHalf), "r"(h), "r"(t0)
            : "memory");
        issued = c + 1;
      }
      // If the launch failed, let copies still in flight land before exit.
      if (err != nullptr && *reinterpret_cast<volatile uint32_t*>(err) != 0) {
        for (int c = (issued > 2 ? issued - 2 : 0); c < issued; ++c) {
          const unsigned long long t_start = global_ns();
          while (!mbar_try_wait(&full[c & 1], (c >> 1) & 1) &&
                 global_ns() - t_start < kWaitLimitNs) {
          }
        }
      }
    }
  } else {
    // ---------------------------------------------------- compute warps --
    const float scale = 0.08838834764831845f;
    const float l2gamma = round_bf16(0.08838834764831845f);
    uint8_t* kq = smem + L::kKQ;
    uint8_t* sop = smem + L::kSop;
    uint8_t* rhi = smem + L::kRhi;
    uint8_t* rlo = smem + L::kRlo;
    uint8_t* pt = smem + L::kP;
    uint8_t* vn = smem + L::kVn;
    uint8_t* vdhi = smem + L::kVdhi;
    uint8_t* vdlo = smem + L::kVdlo;
    const int quarter = warp;  // TMEM lane quarter of this warp
    // Thread tid owns key row tid of the state for value columns
    // [64*dvh, 64*dvh + 64): S[v][k] -> s[v - 64*dvh] at k = tid.
    float s[kDvHalf];
    float* sg = state + (static_cast<int64_t>(seq) * value_heads + h) * kHeadDim * kHeadDim;
#pragma unroll
    for (int j = 0; j < kDvHalf; ++j) s[j] = sg[(dvh * kDvHalf + j) * kHeadDim + tid];

    // P rows 0..63 stay zero: D4 = [0; P] v_new puts P v_new in lanes 64..127.
    for (int e = tid; e < 8192 / 16; e += 128) reinterpret_cast<uint4*>(pt)[e] = make_uint4(0, 0, 0, 0);

    auto write_sop = [&]() {
      // bf16(S) as MN-major [K = dk rows x N = 64 dv]: row tid, 8 chunks.
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        uint4 w;
        w.x = pack_bf16x2(s[8 * j + 0], s[8 * j + 1]);
        w.y = pack_bf16x2(s[8 * j + 2], s[8 * j + 3]);
        w.z = pack_bf16x2(s[8 * j + 4], s[8 * j + 5]);
        w.w = pack_bf16x2(s[8 * j + 6], s[8 * j + 7]);
        *reinterpret_cast<uint4*>(sop + sw128_chunk(tid, j)) = w;
      }
    };
    write_sop();

    uint32_t mma_phase = 0;
    bool ok = true;
    for (int c = 0; c < nchunks && ok; ++c) {
      const int st = c & 1;
      const uint8_t* sbase = smem + (st ? L::kStage1 : L::kStage0);
      const int t0 = seq_t0 + c * kChunk;
      const int n = min(kChunk, seq_t0 + seq_len - t0);
      if (!compute_wait(&full[st], (c >> 1) & 1, err, wait_flag)) { ok = false; break; }

      // Phase 1: normalise K (rows 0-63) and Q (rows 64-127) into the
      // K-major operand tile; per-token factors.
      {
        const int r = tid & 63;
        const uint8_t* src = sbase + (tid < 64 ? kStK : kStQ);
        uint4 raw[16];
        float ss = 0.f;
#pragma unroll
        for (int j = 0; j < 16; ++j)
          raw[j] = *reinterpret_cast<const uint4*>(src + (j >> 3) * 8192 + sw128_chunk(r, j & 7));
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const uint32_t w[4] = {raw[j].x, raw[j].y, raw[j].z, raw[j].w};
#pragma unroll
          for (int p = 0; p < 4; ++p) {
            const float x0 = bf16_bits_to_f32(w[p] & 0xFFFFu), x1 = bf16_bits_to_f32(w[p] >> 16);
            ss += x0 * x0 + x1 * x1;
          }
        }
        const float rs = (r < n) ? rsqrtf(ss * (1.0f / 128.0f) + 1.0e-6f / 128.0f) * l2gamma : 0.f;
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const uint32_t w[4] = {raw[j].x, raw[j].y, raw[j].z, raw[j].w};
          uint4 o;
          uint32_t* op = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
          for (int p = 0; p < 4; ++p)
            op[p] = pack_bf16x2(bf16_bits_to_f32(w[p] & 0xFFFFu) * rs,
                                bf16_bits_to_f32(w[p] >> 16) * rs);
          *reinterpret_cast<uint4*>(kq + (j >> 3) * 16384 + sw128_chunk(tid, j & 7)) = o;
        }
        if (tid < 64) {
          const float* rg = reinterpret_cast<const float*>(sbase + kStRec + kRecG);
          const float* rb = reinterpret_cast<const float*>(sbase + kStRec + kRecBeta);
          const float gi = rg[tid];
          const float glast = rg[n - 1];
          fG[tid] = gi;
          fB[tid] = rb[tid];
          fEG[tid] = expf(gi);
          fED[tid] = expf(glast - gi);
        }
      }
      fence_proxy_async_smem();
      tmem_fence_before();
      named_barrier_compute();
      tmem_fence_after();

      // Phase 2: D1 = [K;Q] S, D2 = [K;Q] K^T.
      if (tid == 0) {
        constexpr uint32_t id_s = umma_idesc_bf16(128, 64, false, true);
        constexpr uint32_t id_k = umma_idesc_bf16(128, 64, false, false);
        const uint32_t akq = smem_u32(kq);
        const uint32_t bs = smem_u32(sop);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t aoff = (kk >> 2) * 16384u + (kk & 3) * 32u;
          umma_bf16(tmem + kTmD1, umma_sdesc(akq + aoff, 16, 1024),
                    umma_sdesc(bs + kk * 2048u, 16384, 1024), id_s, kk > 0 ? 1u : 0u);
          umma_bf16(tmem + kTmD2, umma_sdesc(akq + aoff, 16, 1024),
                    umma_sdesc(akq + aoff, 16, 1024), id_k, kk > 0 ? 1u : 0u);
        }
        umma_commit(mma_bar);
      }
      if (!compute_wait(mma_bar, mma_phase, err, wait_flag)) { ok = false; break; }
      mma_phase ^= 1u;
      tmem_fence_after();

      // Phase 3: R = beta (V - exp(G) K S) -> hi/lo (rows 0-63);
      //          P = Q K^T . exp(G_i - G_j), j <= i < n (rows 64-127).
      {
        const uint32_t lane_base = tmem_addr(tmem, quarter * 32, 0);
        if (tid < 64) {
          const int i = tid;
          const float bi = fB[i], egi = fEG[i];
          const uint8_t* vtile = sbase + kStV;
#pragma unroll
          for (int c16 = 0; c16 < 4; ++c16) {
            uint32_t r[16];
            tmem_ld16(lane_base + kTmD1 + c16 * 16, r);
            tmem_ld_wait();
#pragma unroll
            for (int half8 = 0; half8 < 2; ++half8) {
              const int j = c16 * 2 + half8;            // 8-element chunk index
              const uint4 vv = *reinterpret_cast<const uint4*>(vtile + sw128_chunk(i, j));
              const uint32_t vw[4] = {vv.x, vv.y, vv.z, vv.w};
              uint32_t hi[4], lo[4];
#pragma unroll
              for (int p = 0; p < 4; ++p) {
                const float v0 = bf16_bits_to_f32(vw[p] & 0xFFFFu);
                const float v1 = bf16_bits_to_f32(vw[p] >> 16);
                const float r0 = bi * (v0 - egi * __uint_as_float(r[half8 * 8 + 2 * p]));
                const float r1 = bi * (v1 - egi * __uint_as_float(r[half8 * 8 + 2 * p + 1]));
                const float h0 = round_bf16(r0), h1 = round_bf16(r1);
                hi[p] = pack_bf16x2(h0, h1);
                lo[p] = pack_bf16x2(r0 - h0, r1 - h1);
              }
              *reinterpret_cast<uint4*>(rhi + sw128_chunk(i, j)) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
              *reinterpret_cast<uint4*>(rlo + sw128_chunk(i, j)) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
            }
          }
        } else {
          const int i = tid - 64;
          const float gi = fG[i];
#pragma unroll
          for (int c16 = 0; c16 < 4; ++c16) {
            uint32_t r[16];
            tmem_ld16(lane_base + kTmD2 + c16 * 16, r);
            tmem_ld_wait();
#pragma unroll
            for (int half8 = 0; half8 < 2; ++half8) {
              const int j8 = c16 * 2 + half8;
              uint32_t w[4];
#pragma unroll
              for (int p = 0; p < 4; ++p) {
                const int j0 = j8 * 8 + 2 * p;
                const float p0 = (j0 <= i && i < n) ? __uint_as_float(r[half8 * 8 + 2 * p]) * expf(gi - fG[j0]) : 0.f;
                const float p1 = (j0 + 1 <= i && i < n) ? __uint_as_float(r[half8 * 8 + 2 * p + 1]) * expf(gi - fG[j0 + 1]) : 0.f;
                w[p] = pack_bf16x2(p0, p1);
              }
              // row 64 + i of the [128 x 64] K-major P tile
              *reinterpret_cast<uint4*>(pt + sw128_chunk(64 + i, j8)) = make_uint4(w[0], w[1], w[2], w[3]);
            }
          }
        }
      }
      fence_proxy_async_smem();
      tmem_fence_before();
      named_barrier_compute();
      tmem_fence_after();

      // Phase 4: D3 = T_hi R_hi + T_lo R_hi + T_hi R_lo  (M = 64).
      if (tid == 0) {
        constexpr uint32_t id = umma_idesc_bf16(64, 64, false, true);
        const uint32_t thi = smem_u32(sbase + kStRec + kRecTHi);
        const uint32_t tlo = smem_u32(sbase + kStRec + kRecTLo);
        const uint32_t bh = smem_u32(rhi), bl = smem_u32(rlo);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          umma_bf16(tmem + kTmD3, umma_sdesc(thi + kk * 32, 16, 1024),
                    umma_sdesc(bh + kk * 2048, 8192, 1024), id, kk > 0 ? 1u : 0u);
        }
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          umma_bf16(tmem + kTmD3, umma_sdesc(tlo + kk * 32, 16, 1024),
                    umma_sdesc(bh + kk * 2048, 8192, 1024), id, 1u);
          umma_bf16(tmem + kTmD3, umma_sdesc(thi + kk * 32, 16, 1024),
                    umma_sdesc(bl + kk * 2048, 8192, 1024), id, 1u);
        }
        umma_commit(mma_bar);
      }
      if (!compute_wait(mma_bar, mma_phase, err, wait_flag)) { ok = false; break; }
      mma_phase ^= 1u;
      tmem_fence_after();
      // The stage (record, raw q/k/v) is no longer read: release it.
      if (tid == 0) mbar_arrive(&empty[st]);

      // Phase 5: v_new rows (M = 64 layout: row 16*quarter + lane, lane < 16)
      // -> bf16 v_new and hi/lo of v_new * exp(G_C - G).
      {
        const uint32_t lane_base = tmem_addr(tmem, quarter * 32, 0);
        const int i = quarter * 16 + lane;
        const float edi = (lane < 16) ? fED[i] : 0.f;
#pragma unroll
        for (int c16 = 0; c16 < 4; ++c16) {
          uint32_t r[16];
          tmem_ld16(lane_base + kTmD3 + c16 * 16, r);
          tmem_ld_wait();
          if (lane < 16) {
#pragma unroll
            for (int half8 = 0; half8 < 2; ++half8) {
              const int j = c16 * 2 + half8;
              uint32_t vb[4], dh[4], dl[4];
#pragma unroll
              for (int p = 0; p < 4; ++p) {
                const float v0 = __uint_as_float(r[half8 * 8 + 2 * p]);
                const float v1 = __uint_as_float(r[half8 * 8 + 2 * p + 1]);
                vb[p] = pack_bf16x2(v0, v1);
                const float d0 = v0 * edi, d1 = v1 * edi;
                const float h0 = round_bf16(d0), h1 = round_bf16(d1);
                dh[p] = pack_bf16x2(h0, h1);
                dl[p] = pack_bf16x2(d0 - h0, d1 - h1);
              }
              *reinterpret_cast<uint4*>(vn + sw128_chunk(i, j)) = make_uint4(vb[0], vb[1], vb[2], vb[3]);
              *reinterpret_cast<uint4*>(vdhi + sw128_chunk(i, j)) = make_uint4(dh[0], dh[1], dh[2], dh[3]);
              *reinterpret_cast<uint4*>(vdlo + sw128_chunk(i, j)) = make_uint4(dl[0], dl[1], dl[2], dl[3]);
            }
          }
        }
      }
      fence_proxy_async_smem();
      tmem_fence_before();
      named_barrier_compute();
      tmem_fence_after();

      // Phase 6: D4 = [0;P] v_new (M=128), D5 = K^T (Vd_hi + Vd_lo) (M=128).
      if (tid == 0) {
        constexpr uint32_t id_o = umma_idesc_bf16(128, 64, false, true);
        constexpr uint32_t id_s = umma_idesc_bf16(128, 64, true, true);
        const uint32_t ap = smem_u32(pt), bv = smem_u32(vn);
        const uint32_t akt = smem_u32(kq);
        const uint32_t bdh = smem_u32(vdhi), bdl = smem_u32(vdlo);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          umma_bf16(tmem + kTmD4, umma_sdesc(ap + kk * 32, 16, 1024),
                    umma_sdesc(bv + kk * 2048, 8192, 1024), id_o, kk > 0 ? 1u : 0u);
        }
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          // A = K^T: MN-major view of KQ rows 0..63 (tokens), dk slabs 16 KB apart.
          umma_bf16(tmem + kTmD5, umma_sdesc(akt + kk * 2048, 16384, 1024),
                    umma_sdesc(bdh + kk * 2048, 8192, 1024), id_s, kk > 0 ? 1u : 0u);
          umma_bf16(tmem + kTmD5, umma_sdesc(akt + kk * 2048, 16384, 1024),
                    umma_sdesc(bdl + kk * 2048, 8192, 1024), id_s, 1u);
        }
        umma_commit(mma_bar);
      }
      if (!compute_wait(mma_bar, mma_phase, err, wait_flag)) { ok = false; break; }
      mma_phase ^= 1u;
      tmem_fence_after();

      // Phase 7: output rows (lanes 64..127) and state update (all lanes).
      {
        const uint32_t lane_base = tmem_addr(tmem, quarter * 32, 0);
        if (tid >= 64) {
          const int i = tid - 64;
          const float egi = fEG[i];
          uint16_t* orow = o_out + (static_cast<int64_t>(t0 + i) * value_heads + h) * kHeadDim + dvh * kDvHalf;
#pragma unroll
          for (int c16 = 0; c16 < 4; ++c16) {
            uint32_t rq[16], rp[16];
            tmem_ld16(lane_base + kTmD1 + c16 * 16, rq);
            tmem_ld16(lane_base + kTmD4 + c16 * 16, rp);
            tmem_ld_wait();
            if (i < n) {
              uint32_t w[8];
#pragma unroll
              for (int p = 0; p < 8; ++p) {
                const float o0 = scale * (egi * __uint_as_float(rq[2 * p]) + __uint_as_float(rp[2 * p]));
                const float o1 = scale * (egi * __uint_as_float(rq[2 * p + 1]) + __uint_as_float(rp[2 * p + 1]));
                w[p] = pack_bf16x2(o0, o1);
              }
              reinterpret_cast<uint4*>(orow + c16 * 16)[0] = make_uint4(w[0], w[1], w[2], w[3]);
              reinterpret_cast<uint4*>(orow + c16 * 16)[1] = make_uint4(w[4], w[5], w[6], w[7]);
            }
          }
        }
        const float dl = expf(fG[n - 1]);
#pragma unroll
        for (int c16 = 0; c16 < 4; ++c16) {
          uint32_t r[16];
          tmem_ld16(lane_base + kTmD5 + c16 * 16, r);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 16; ++j) s[c16 * 16 + j] = dl * s[c16 * 16 + j] + __uint_as_float(r[j]);
        }
        write_sop();
      }
      fence_proxy_async_smem();
      tmem_fence_before();
      named_barrier_compute();
      tmem_fence_after();
    }
    if (ok) {
#pragma unroll
      for (int j = 0; j < kDvHalf; ++j) sg[(dvh * kDvHalf + j) * kHeadDim + tid] = s[j];
    }
  }
  tmem_fence_before();
  __syncthreads();
  if (warp == 0) {
    __syncwarp();
    tmem_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ============================================================= host ====

using EncodeTiledFn3 = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                    const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                    const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                    CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn3 encode_fn3() {
  static EncodeTiledFn3 fn = nullptr;
  if (fn == nullptr) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      fn = reinterpret_cast<EncodeTiledFn3>(ptr);
    }
  }
  return fn;
}

// bf16 [tokens, heads, 128] viewed as {d, head, token}; box {box_d, 1, 64}.
static bool make_tmap_thd(CUtensorMap* map, const void* base, int64_t tokens, int heads,
                          int box_d) {
  EncodeTiledFn3 fn = encode_fn3();
  if (fn == nullptr) return false;
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(kHeadDim), static_cast<cuuint64_t>(heads),
                        static_cast<cuuint64_t>(tokens)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(kHeadDim) * 2,
                           static_cast<cuuint64_t>(heads) * kHeadDim * 2};
  cuuint32_t box[3] = {static_cast<cuuint32_t>(box_d), 1, static_cast<cuuint32_t>(kChunk)};
  cuuint32_t estr[3] = {1, 1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box,
            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) ==
         CUDA_SUCCESS;
}

bool build_chunk_table(const int32_t* cu_seqlens, int num_seqs, ChunkTable* tab) {
  if (num_seqs < 1 || num_seqs > kMaxSeqsInternal || cu_seqlens[0] != 0) return false;
  tab->num_seqs = num_seqs;
  int chunks = 0;
  for (int s = 0; s <= num_seqs; ++s) {
    tab->cu[s] = cu_seqlens[s];
    tab->chunk_start[s] = chunks;
    if (s < num_seqs) {
      const int len = cu_seqlens[s + 1] - cu_seqlens[s];
      if (len < 0) return false;
      chunks += (len + kChunk - 1) / kChunk;
    }
  }
  tab->total_chunks = chunks;
  return true;
}

uint64_t chunk_workspace_bytes(const ChunkTable& tab, int value_heads) {
  return static_cast<uint64_t>(tab.total_chunks) * value_heads * kRecBytes;
}

cudaError_t launch_chunk_prefill(const ChunkTable& tab, const uint16_t* q, const uint16_t* k,
                                 const uint16_t* v, const uint16_t* a, const uint16_t* b,
                                 const float* A_log, const float* dt_bias, float* state,
                                 uint16_t* o_out, int qk_heads, int value_heads,
                                 uint8_t* records, uint32_t* err, cudaStream_t stream) {
  if (tab.total_chunks == 0) return cudaSuccess;
  const int64_t tokens = tab.cu[tab.num_seqs];
  const uint32_t prep_smem = sizeof(PrepSmem) + 1024;
  cudaError_t e = cudaFuncSetAttribute(gdn_chunk_prep_kernel,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, prep_smem);
  if (e != cudaSuccess) return e;
  dim3 pgrid(tab.total_chunks, qk_heads);
  gdn_chunk_prep_kernel<<<pgrid, kPrepThreads, prep_smem, stream>>>(
      tab, k, a, b, A_log, dt_bias, records, qk_heads, value_heads, err);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;

  CUtensorMap tq, tk, tv;
  if (!make_tmap_thd(&tq, q, tokens, qk_heads, 64) ||
      !make_tmap_thd(&tk, k, tokens, qk_heads, 64) ||
      !make_tmap_thd(&tv, v, tokens, value_heads, kDvHalf))
    return cudaErrorInvalidValue;
  const uint32_t st_smem = StateSmemLayout::kTotal;
  e = cudaFuncSetAttribute(gdn_chunk_state_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           st_smem);
  if (e != cudaSuccess) return e;
  dim3 sgrid(kHeadDim / kDvHalf, value_heads, tab.num_seqs);
  gdn_chunk_state_kernel<<<sgrid, kStateThreads, st_smem, stream>>>(
      tab, tq, tk, tv, records, state, o_out, qk_heads, value_heads, err);
  return cudaGetLastError();
}

}  // namespace gdn
