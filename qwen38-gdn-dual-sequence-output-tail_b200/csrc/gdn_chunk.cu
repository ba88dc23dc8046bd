// Chunked (C = 64) gated delta rule for packed variable-length sequences.
//
// Replaces ChunkGdn (reference provider P:1641-1838): there, one chunk of at
// most 64 tokens per call runs as cumsum -> KK^T (AOT) -> 16x16 solve (AOT)
// -> 64x64 merge (AOT) -> W,U (AOT) -> ChunkGatedDeltaRuleFwdH -> ChunkFwdO
// with eight permutes and seventeen allocations, and longer prompts fall back
// to 8-token recurrent slices (run_sequence, P:3387-3469).  Here every chunk
// of every sequence is processed in two launches (the second launched to
// overlap the first's last CTAs).
//
// 1. gdn_chunk_prep_kernel: chunk-parallel and persistent (three CTAs per SM,
//    units of one chunk x one q/k head, the next unit's q/k tile on its way
//    by TMA), everything that does not depend on the recurrent state:
//      q, k L2-norm -> the bf16 [K;Q] operand image (shared by the v-heads),
//      [K;Q] K^T on tcgen05 (K K^T and Q K^T in one M=128 MMA),
//      per v-head: gating g, beta, in-chunk cumsum G (warp scans),
//      A = beta_i (K K^T)_ij exp(G_i - G_j) (strictly lower),
//      T = (I + A)^-1 in f32: 16x16 diagonal blocks by forward substitution,
//      then block doubling 16 -> 32 -> 64,
//      P = (Q K^T)_ij exp(G_i - G_j) (j <= i),
//    stored as 128-byte-swizzled operand images the second kernel feeds
//    straight to tcgen05: T as a bf16 hi/lo pair (about 16 mantissa bits),
//    P in bf16, plus per-token factors.
// 2. gdn_chunk_state_kernel: sequential over the chunks of one sequence,
//    one CTA per (sequence, v-head, half of the value dimension) -- column j
//    of v_new, S and O depends only on column j of S, so the split is exact.
//    Eight compute warps, an MMA-issuing warp and a loader warp, handing over
//    through mbarriers; per chunk
//      D1 = [S^T;S^T] K^T, [S^T;S^T] Q^T    ((K S)^T, (Q S)^T)
//      R^T = (beta V - beta exp(G) (K S))^T -> bf16 hi/lo
//      D3 = [T;T] [R_hi | R_lo] + [T_lo;T_lo] R_hi,   v_new = sum of halves
//      D5 = K^T [Vd_hi | Vd_lo],  Vd = v_new exp(G_C - G)
//      S = exp(G_C) S + D5
//    and, off that chain, D4 = [Vn^T;Vn^T] P^T = (P v_new)^T and
//    O = scale (exp(G) (Q S) + P v_new), stored by TMA, with the f32 state
//    in registers (thread t owns key row t).
// The reference's W = T (beta exp(G) K) is never formed:
// v_new = U - W S = T (beta V - beta exp(G) (K S)) needs one product with T.
// Decay factors are always exp of a non-positive difference.
#include <algorithm>
#include <vector>

#include "gdn_common.cuh"
#include "gdn_internal.h"

namespace gdn {

// Per (chunk, q/k head): [K;Q] image, K-major [128 rows x 128 cols] bf16,
// 64-column slab s at s * 16 KB; rows 0-63 = normalised K, 64-127 = Q
// (rows past the chunk length are zero).
constexpr uint32_t kKQBytes = 32768;
// Per (chunk, v-head) record.
constexpr uint32_t kRecP = 0;          // P, K-major [64 i x 64 j] bf16
constexpr uint32_t kRecTHi = 8192;     // T hi, MN-major [K = j][M = i] bf16
constexpr uint32_t kRecTLo = 16384;    // T lo
constexpr uint32_t kRecF = 24576;      // f32 factors, see kF*
constexpr uint32_t kRecBytes = 25856;
// Factor offsets (floats) inside kRecF.
constexpr int kFBeta = 0, kFBetaEG = 64, kFEG = 128, kFED = 192, kFELast = 256;

__device__ __forceinline__ int find_seq(const ChunkTable& tab, int chunk) {
  int lo = 0, hi = tab.num_seqs - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (tab.chunk_start[mid] <= chunk) lo = mid; else hi = mid - 1;
  }
  return lo;
}

__device__ __forceinline__ float softplus20(float x) { return x > 20.0f ? x : log1pf(expf(x)); }

__device__ __forceinline__ void group_barrier(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// ============================================================ prep =====

// T = (I + A)^-1 by block doubling, once the four 16x16 diagonal blocks of T
// are in place (M holds A below them).  For a unit lower-triangular
// [[M1, 0], [M21, M2]] the inverse is [[T1, 0], [-T2 M21 T1, T2]], so
//   level 1: T_10 = -T_11 (A_10 T_00),  T_32 = -T_33 (A_32 T_22)
//   level 2: X = [A_20 A_21; A_30 A_31] [T_00 0; T_10 T_11]   (32 x 32)
//            [T_20 T_21; T_30 T_31] = -[T_22 0; T_32 T_33] X
// in four phases of one group of 128 threads.  The products X go to the
// strictly upper blocks of M, which the inverse never reads (the T store
// masks them to zero).  Warp w of the group takes rows w + 4 (lane / 16) and
// that + 8 of every output block, lane % 16 its column: all 128 threads carry
// the same number of multiply-adds in every phase, the loop bounds are
// warp-uniform, and the two rows of an instruction are 4 apart (16 banks).
// Products run on f32x2 pairs along the summation index (even and odd terms).
__device__ __forceinline__ float2 col_pair(float (*M)[68], int m, int c) {
  return make_float2(M[m][c], M[m + 1][c]);
}
// M[r][m .. m+3] as two pairs (one 16-byte load; m % 4 == 0).
__device__ __forceinline__ void row_quad(float (*M)[68], int r, int m, float2& lo, float2& hi) {
  const float4 q = *reinterpret_cast<const float4*>(&M[r][m]);
  lo = make_float2(q.x, q.y);
  hi = make_float2(q.z, q.w);
}
__device__ __forceinline__ float pair_sum(float2 v) { return v.x + v.y; }
// acc += M[r][m .. m+3] . (b0, b1), b0 = column values at m, m+1 and b1 at m+2, m+3.
__device__ __forceinline__ float2 quad_fma(float (*M)[68], int r, int m, float2 b0, float2 b1,
                                           float2 acc) {
  float2 lo, hi;
  row_quad(M, r, m, lo, hi);
  return ffma2(hi, b1, ffma2(lo, b0, acc));
}

__device__ __forceinline__ void invert_by_doubling(float (*M)[68], int u, int grp, bool live) {
  const int c = u & 15;
  const int r0 = (u >> 5) + 4 * ((u >> 4) & 1);
  // Level 1, products: X_10 -> block (0, 1), X_32 -> block (2, 3).
  if (live) {
    float2 acc[2][2] = {};
#pragma unroll
    for (int m = 0; m < 16; m += 4) {
      const float2 t00a = col_pair(M, m, c), t00b = col_pair(M, m + 2, c);
      const float2 t22a = col_pair(M, 32 + m, 32 + c), t22b = col_pair(M, 34 + m, 32 + c);
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        const int r = r0 + 8 * k;
        acc[k][0] = quad_fma(M, 16 + r, m, t00a, t00b, acc[k][0]);
        acc[k][1] = quad_fma(M, 48 + r, 32 + m, t22a, t22b, acc[k][1]);
      }
    }
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      M[r0 + 8 * k][16 + c] = pair_sum(acc[k][0]);
      M[32 + r0 + 8 * k][48 + c] = pair_sum(acc[k][1]);
    }
  }
  group_barrier(1 + grp, 128);
  // Level 1, T_10 = -T_11 X_10 and T_32 = -T_33 X_32 (over A_10, A_32).
  if (live) {
    float2 acc[2][2] = {};
#pragma unroll
    for (int m = 0; m < 16; m += 4) {
      const float2 x10a = col_pair(M, m, 16 + c), x10b = col_pair(M, m + 2, 16 + c);
      const float2 x32a = col_pair(M, 32 + m, 48 + c), x32b = col_pair(M, 34 + m, 48 + c);
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        const int r = r0 + 8 * k;
        acc[k][0] = quad_fma(M, 16 + r, 16 + m, x10a, x10b, acc[k][0]);
        acc[k][1] = quad_fma(M, 48 + r, 48 + m, x32a, x32b, acc[k][1]);
      }
    }
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      M[16 + r0 + 8 * k][c] = -pair_sum(acc[k][0]);
      M[48 + r0 + 8 * k][32 + c] = -pair_sum(acc[k][1]);
    }
  }
  group_barrier(1 + grp, 128);
  // Level 2, products: X_20 -> (0, 2), X_21 -> (0, 3), X_30 -> (1, 2),
  // X_31 -> (1, 3).
  if (live) {
    float2 acc[2][4] = {};
#pragma unroll
    for (int m = 0; m < 32; m += 4) {
      const float2 ta = col_pair(M, m, c), tb = col_pair(M, m + 2, c);   // [T_00; T_10]
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        const int r = r0 + 8 * k;
        acc[k][0] = quad_fma(M, 32 + r, m, ta, tb, acc[k][0]);
        acc[k][2] = quad_fma(M, 48 + r, m, ta, tb, acc[k][2]);
      }
    }
#pragma unroll
    for (int m = 0; m < 16; m += 4) {
      const float2 ta = col_pair(M, 16 + m, 16 + c), tb = col_pair(M, 18 + m, 16 + c);   // T_11
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        const int r = r0 + 8 * k;
        acc[k][1] = quad_fma(M, 32 + r, 16 + m, ta, tb, acc[k][1]);
        acc[k][3] = quad_fma(M, 48 + r, 16 + m, ta, tb, acc[k][3]);
      }
    }
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int r = r0 + 8 * k;
      M[r][32 + c] = pair_sum(acc[k][0]);
      M[r][48 + c] = pair_sum(acc[k][1]);
      M[16 + r][32 + c] = pair_sum(acc[k][2]);
      M[16 + r][48 + c] = pair_sum(acc[k][3]);
    }
  }
  group_barrier(1 + grp, 128);
  // Level 2, the lower-left 32 x 32 block of T (over A_20 .. A_31).
  if (live) {
    float2 acc[2][4] = {};
#pragma unroll
    for (int m = 0; m < 16; m += 4) {
      const float2 x20a = col_pair(M, m, 32 + c), x20b = col_pair(M, m + 2, 32 + c);
      const float2 x21a = col_pair(M, m, 48 + c), x21b = col_pair(M, m + 2, 48 + c);
      const float2 x30a = col_pair(M, 16 + m, 32 + c), x30b = col_pair(M, 18 + m, 32 + c);
      const float2 x31a = col_pair(M, 16 + m, 48 + c), x31b = col_pair(M, 18 + m, 48 + c);
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        const int r = r0 + 8 * k;
        float2 t22a, t22b, t32a, t32b, t33a, t33b;
        row_quad(M, 32 + r, 32 + m, t22a, t22b);
        row_quad(M, 48 + r, 32 + m, t32a, t32b);
        row_quad(M, 48 + r, 48 + m, t33a, t33b);
        acc[k][0] = ffma2(t22b, x20b, ffma2(t22a, x20a, acc[k][0]));
        acc[k][1] = ffma2(t22b, x21b, ffma2(t22a, x21a, acc[k][1]));
        acc[k][2] = ffma2(t33b, x30b, ffma2(t33a, x30a, ffma2(t32b, x20b, ffma2(t32a, x20a, acc[k][2]))));
        acc[k][3] = ffma2(t33b, x31b, ffma2(t33a, x31a, ffma2(t32b, x21b, ffma2(t32a, x21a, acc[k][3]))));
      }
    }
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int r = r0 + 8 * k;
      M[32 + r][c] = -pair_sum(acc[k][0]);
      M[32 + r][16 + c] = -pair_sum(acc[k][1]);
      M[48 + r][c] = -pair_sum(acc[k][2]);
      M[48 + r][16 + c] = -pair_sum(acc[k][3]);
    }
  }
  group_barrier(1 + grp, 128);
}


constexpr int kPrepThreads = 256;

struct PrepSmem {
  uint8_t kq[kKQBytes];     // [K;Q] tile (1024-aligned): raw q/k land here by TMA
                            // and are normalised in place
  float amat[2][64][68];    // A, overwritten in place by T = (I + A)^-1; the
                            // strictly upper blocks hold the inverse's products
  float g[2][64];           // cumsum G
  float e1[2][64];          // exp(g_t) = exp(G_t - G_{t-1})
  float beta[2][64];
  float carry[2];
  uint64_t full;            // raw tile of the current unit has landed
  uint64_t mma;             // [K;Q] K^T of the current unit has completed
  uint32_t tmem;
};
// Three CTAs per SM: 3 x (this + 1 KB alignment slack + 1 KB reserved) must
// fit in the SM's 228 KB.
static_assert(sizeof(PrepSmem) + 1024 <= 228 * 1024 / 3 - 1024, "prep shared memory");

// Persistent: CTA x handles units x, x + gridDim.x, ... (unit = chunk * Hk +
// q/k head).  The finished [K;Q] image goes back to global memory as one bulk
// store; once that store and the unit's MMA have read the tile buffer, the
// raw q/k tile of the next unit is loaded into it by TMA while the rest of the
// unit (A, P and the inverse, most of its time) runs.  Three CTAs per SM.
__global__ void __launch_bounds__(kPrepThreads, 3)
gdn_chunk_prep_kernel(const __grid_constant__ ChunkTable tab,
                      const __grid_constant__ CUtensorMap tm_q,
                      const __grid_constant__ CUtensorMap tm_k,
                      const uint16_t* __restrict__ a,
                      const uint16_t* __restrict__ b, const float* __restrict__ A_log,
                      const float* __restrict__ dt_bias, uint8_t* __restrict__ kq_records,
                      uint8_t* __restrict__ records, int qk_heads, int value_heads,
                      uint32_t* err, int clear_err) {
  // With clear_err the call's error word starts at zero here instead of by a
  // separate memset (errors are recorded only after bounded waits of seconds).
  if (clear_err && blockIdx.x == 0 && threadIdx.x == 0) *err = 0u;
  // A state pass launched to overlap this kernel may start its set-up now
  // (it waits for this grid before it reads a record).
  griddep_launch_dependents();
  extern __shared__ uint8_t smem_raw[];
  PrepSmem& sm = *reinterpret_cast<PrepSmem*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int units = tab.total_chunks * qk_heads;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int group = value_heads / qk_heads;
  const int grp = threadIdx.x >> 7;     // v-head of the pair handled by this group
  const int u = threadIdx.x & 127;
  const int quarter = warp & 3;         // TMEM lane quarter of this warp

  // Raw q/k tile of a unit: K rows 0-63 and Q rows 64-127 of both 64-column
  // slabs, four 8 KB boxes (tokens past the tensor read as zero).
  auto load_unit = [&](int unit) {
    const int chunk = unit / qk_heads;
    const int kh = unit - chunk * qk_heads;
    const int seq = find_seq(tab, chunk);
    const int t0 = tab.cu[seq] + (chunk - tab.chunk_start[seq]) * kChunk;
    uint8_t* dst = sm.kq;
    mbar_arrive_expect_tx(&sm.full, kKQBytes);
    tma_load_3d(dst, &tm_k, &sm.full, 0, kh, t0);
    tma_load_3d(dst + 16384, &tm_k, &sm.full, 64, kh, t0);
    tma_load_3d(dst + 8192, &tm_q, &sm.full, 0, kh, t0);
    tma_load_3d(dst + 16384 + 8192, &tm_q, &sm.full, 64, kh, t0);
  };

  if (threadIdx.x == 0) {
    mbar_init(&sm.full, 1);
    mbar_init(&sm.mma, 1);
    fence_barrier_init();
    tma_prefetch_desc(&tm_q);
    tma_prefetch_desc(&tm_k);
    if (static_cast<int>(blockIdx.x) < units) load_unit(blockIdx.x);
  }
  if (warp == 0) tmem_alloc(&sm.tmem, 64);
  tmem_fence_before();
  __syncthreads();
  tmem_fence_after();
  const uint32_t tmem = sm.tmem;

  int it = 0;
  for (int unit = blockIdx.x; unit < units; unit += gridDim.x, ++it) {
    const int chunk = unit / qk_heads;
    const int kh = unit - chunk * qk_heads;
    const int seq = find_seq(tab, chunk);
    const int t0 = tab.cu[seq] + (chunk - tab.chunk_start[seq]) * kChunk;
    const int n = min(kChunk, tab.cu[seq + 1] - t0);

    // Gate inputs of the first v-head pair, fetched before the tile wait.
    float pre_a = 0.f, pre_b = 0.f, pre_alog = 0.f, pre_dt = 0.f;
    if (grp < group && u < 64) {
      pre_alog = A_log[kh * group + grp];
      pre_dt = dt_bias[kh * group + grp];
      if (u < n) {
        const int64_t gi = static_cast<int64_t>(t0 + u) * value_heads + kh * group + grp;
        pre_a = bf16_bits_to_f32(a[gi]);
        pre_b = bf16_bits_to_f32(b[gi]);
      }
    }

    // q/k rows -> RmsNorm L2-norm (gamma bf16(1/sqrt(128)), eps 1e-6/128) ->
    // bf16, in place.  Two threads per row (row r = tid / 2, half = tid % 2:
    // the 64-column slab `half`, eight 16-byte chunks); rows past the chunk
    // are zeroed.
    bool landed = mbar_wait(&sm.full, it & 1, err);
    {
      uint8_t* tile = sm.kq;
      const float l2gamma = round_bf16(0.08838834764831845f);
      const int r = threadIdx.x >> 1;
      const int half = threadIdx.x & 1;
      const int tok = r & 63;
      // Two passes over the row's chunks (sum of squares, then scale): the
      // tile is read twice from shared memory instead of being held in
      // registers.
      const bool live_row = landed && tok < n;
      // Sum of squares on f32x2 pairs (the two halves of each bf16x2 word).
      float2 ss2 = make_float2(0.f, 0.f);
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const uint4 v = live_row
                            ? *reinterpret_cast<const uint4*>(tile + half * 16384u + sw128_chunk(r, c))
                            : make_uint4(0u, 0u, 0u, 0u);
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int p = 0; p < 4; ++p) {
          const float2 x = bf16x2_f32x2(w[p]);
          ss2 = ffma2(x, x, ss2);
        }
      }
      float ss = ss2.x + ss2.y;
      ss += __shfl_xor_sync(0xffffffffu, ss, 1);
      const float rs = rsqrtf(ss * (1.0f / 128.0f) + 1.0e-6f / 128.0f) * l2gamma;
      const float2 rs2 = make_float2(rs, rs);
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const uint4 v = live_row
                            ? *reinterpret_cast<const uint4*>(tile + half * 16384u + sw128_chunk(r, c))
                            : make_uint4(0u, 0u, 0u, 0u);
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
        uint32_t ow[4];
#pragma unroll
        for (int p = 0; p < 4; ++p) {
          const float2 y = fmul2(bf16x2_f32x2(w[p]), rs2);
          ow[p] = pack_bf16x2(y.x, y.y);
        }
        *reinterpret_cast<uint4*>(tile + half * 16384u + sw128_chunk(r, c)) =
            make_uint4(ow[0], ow[1], ow[2], ow[3]);
      }
    }
    fence_proxy_async_smem();
    tmem_fence_before();
    __syncthreads();
    tmem_fence_after();

    if (threadIdx.x == 0) {
      // D[128 x 64] = [K;Q] K^T: lanes 0-63 hold K K^T, lanes 64-127 Q K^T.
      constexpr uint32_t idesc = umma_idesc_bf16(128, 64, false, false);
      const uint32_t t = smem_u32(sm.kq);
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        const uint32_t off = (kk >> 2) * 16384u + (kk & 3) * 32u;
        umma_bf16(tmem, umma_sdesc(t + off, 16, 1024), umma_sdesc(t + off, 16, 1024), idesc,
                  kk > 0 ? 1u : 0u);
      }
      umma_commit(&sm.mma);
      // The [K;Q] image to its record.
      bulk_store(kq_records + static_cast<int64_t>(unit) * kKQBytes, sm.kq, kKQBytes);
      bulk_commit();
    }

    bool ok = true;
    bool waited = false;
    // T overwrites A in place: block row I of A is last read while block row
    // I of T is formed, and T's strictly upper part equals A's (zero).
    float (*A)[68] = sm.amat[grp];
    float (*T)[68] = sm.amat[grp];

    for (int hp = 0; hp < group; hp += 2) {
      const int hl = hp + grp;
      const bool active = hl < group;
      const int h = kh * group + (active ? hl : 0);
      uint8_t* rec = records + (static_cast<int64_t>(chunk) * value_heads + h) * kRecBytes;
      float* fac = reinterpret_cast<float*>(rec + kRecF);

      // Gating (aclnnFusedGdnGating: softplus beta 1, threshold 20) and the
      // in-chunk cumsum as two warp scans.
      if (active && u < 64) {
        float ga = pre_a, gb = pre_b, alog = pre_alog, dtb = pre_dt;
        if (hp > 0) {
          alog = A_log[h];
          dtb = dt_bias[h];
          if (u < n) {
            const int64_t gi = static_cast<int64_t>(t0 + u) * value_heads + h;
            ga = bf16_bits_to_f32(a[gi]);
            gb = bf16_bits_to_f32(b[gi]);
          }
        }
        float g = 0.f, bt = 0.f;
        if (u < n) {
          g = -expf(alog) * softplus20(ga + dtb);
          bt = round_bf16(1.0f / (1.0f + expf(-gb)));
        }
        sm.e1[grp][u] = __expf(g);
  #pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const float y = __shfl_up_sync(0xffffffffu, g, o);
          if (lane >= o) g += y;
        }
        if (u == 31) sm.carry[grp] = g;
        sm.beta[grp][u] = bt;
        sm.g[grp][u] = g;
      }
      group_barrier(1 + grp, 128);
      if (active && u >= 32 && u < 64) sm.g[grp][u] += sm.carry[grp];
      group_barrier(1 + grp, 128);
      if (active && u < 64) {
        const float gi = sm.g[grp][u];
        const float glast = sm.g[grp][n - 1];
        const float bt = sm.beta[grp][u];
        const float egi = __expf(gi);
        fac[kFBeta + u] = bt;
        fac[kFBetaEG + u] = bt * egi;
        fac[kFEG + u] = egi;
        fac[kFED + u] = __expf(glast - gi);
        if (u == 0) fac[kFELast] = __expf(glast);
      }

      if (!waited) {
        ok = mbar_wait(&sm.mma, it & 1, err);
        waited = true;
      }
      tmem_fence_after();
      if (active && ok) {
        // TMEM row of this lane, 16 columns at a time.
        const uint32_t base = tmem_addr(tmem, quarter * 32, 0);
        if (u < 64) {
          // Lane u holds row u of K K^T: A[u][j] = beta_u KK_uj exp(G_u - G_j)
          // for j < u (beta_u = 0 past the chunk), the decay a running
          // product of the per-token exp(g) towards smaller j; each
          // 16-column piece goes to row u of A as four 16-byte stores.
          const float bu = sm.beta[grp][u];
          float d = 1.f;
          float e1_up = 1.f;                 // exp(g) of the token after the piece
  #pragma unroll
          for (int c = 48; c >= 0; c -= 16) {
            uint32_t r[16];
            tmem_ld16(base + c, r);
            float e1v[16];
  #pragma unroll
            for (int q4 = 0; q4 < 4; ++q4) {
              const float4 ev = *reinterpret_cast<const float4*>(&sm.e1[grp][c + 4 * q4]);
              e1v[4 * q4] = ev.x; e1v[4 * q4 + 1] = ev.y; e1v[4 * q4 + 2] = ev.z; e1v[4 * q4 + 3] = ev.w;
            }
            tmem_ld_wait();
            float av[16];
  #pragma unroll
            for (int jj = 15; jj >= 0; --jj) {
              const int j = c + jj;
              d = (j < u) ? d * (jj == 15 ? e1_up : e1v[jj + 1]) : 1.f;
              av[jj] = (j < u) ? bu * __uint_as_float(r[jj]) * d : 0.f;
            }
            e1_up = e1v[0];
  #pragma unroll
            for (int q4 = 0; q4 < 4; ++q4)
              *reinterpret_cast<float4*>(&A[u][c + 4 * q4]) =
                  make_float4(av[4 * q4], av[4 * q4 + 1], av[4 * q4 + 2], av[4 * q4 + 3]);
          }
        } else {
          // Lane 64+i holds row i of Q K^T: P[i][j] = QK_ij exp(G_i - G_j),
          // j <= i < n, decay as a running product towards smaller j; each
          // 16-column piece goes to the record as two 16-byte chunks.
          const int i = u - 64;
          float d = 1.f;
  #pragma unroll
          for (int c = 48; c >= 0; c -= 16) {
            uint32_t r[16];
            tmem_ld16(base + c, r);
            float e1v[16];
  #pragma unroll
            for (int q4 = 0; q4 < 4; ++q4) {
              const float4 ev = *reinterpret_cast<const float4*>(&sm.e1[grp][c + 4 * q4]);
              e1v[4 * q4] = ev.x; e1v[4 * q4 + 1] = ev.y; e1v[4 * q4 + 2] = ev.z; e1v[4 * q4 + 3] = ev.w;
            }
            tmem_ld_wait();
            uint32_t w[8];
  #pragma unroll
            for (int jj = 15; jj >= 0; --jj) {
              const int j = c + jj;
              const float pj = (j <= i && i < n) ? __uint_as_float(r[jj]) * d : 0.f;
              d = (j <= i) ? d * e1v[jj] : 1.f;
              if (jj & 1) w[jj >> 1] = __float_as_uint(pj);
              else w[jj >> 1] = pack_bf16x2(pj, __uint_as_float(w[jj >> 1]));
            }
            *reinterpret_cast<uint4*>(rec + kRecP + sw128_chunk(i, c >> 3)) =
                make_uint4(w[0], w[1], w[2], w[3]);
            *reinterpret_cast<uint4*>(rec + kRecP + sw128_chunk(i, (c >> 3) + 1)) =
                make_uint4(w[4], w[5], w[6], w[7]);
          }
        }
      }
      group_barrier(1 + grp, 128);
      if (hp == 0 && threadIdx.x == 0) {
        // The unit's MMA and [K;Q] store have read the tile buffer (the MMA
        // was waited for above): the next unit's tile can land in it now.
        bulk_wait_read<0>();
        const int next = unit + gridDim.x;
        if (next < units) load_unit(next);
      }

      // T = (I + A)^-1: the 16x16 diagonal blocks by forward substitution
      // (one thread per block column; x[rr] = 0 above the diagonal), then
      // block doubling (invert_by_doubling).  The substitution sums run on
      // f32x2 pairs (even and odd terms), halving the dependent chain.
      const bool diag = active && ok && u < 64;
      const int bl = u >> 4, dc = u & 15, o = bl * 16;
      float2 x2[8];
      if (diag) {
  #pragma unroll
        for (int rr = 0; rr < 16; ++rr) {
          float2 sacc = make_float2(0.f, 0.f);
  #pragma unroll
          for (int m = 0; m + 1 < rr; m += 2)
            sacc = ffma2(*reinterpret_cast<const float2*>(&A[o + rr][o + m]), x2[m >> 1], sacc);
          float v = ((rr == dc) ? 1.f : 0.f) - (sacc.x + sacc.y);
          if (rr & 1) v -= A[o + rr][o + rr - 1] * x2[(rr - 1) >> 1].x;
          if (rr & 1) x2[rr >> 1].y = v; else x2[rr >> 1].x = v;
        }
      }
      group_barrier(1 + grp, 128);  // every read of the diagonal A blocks is done
      if (diag) {
  #pragma unroll
        for (int rr = 0; rr < 16; rr += 2) {
          T[o + rr][o + dc] = x2[rr >> 1].x;
          T[o + rr + 1][o + dc] = x2[rr >> 1].y;
        }
      }
      group_barrier(1 + grp, 128);
      invert_by_doubling(T, u, grp, active && ok);
      // Store T as K-rows j of the MN-major operand image (hi/lo pair):
      // thread -> column j = u / 2, rows [32 (u % 2), +32); entries above the
      // diagonal are zero (the upper blocks of M hold scratch).
      if (active && ok) {
        const int j = u >> 1;
        const int i0 = (u & 1) * 32;
  #pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t hi[4], lo[4];
  #pragma unroll
          for (int p = 0; p < 4; ++p) {
            const int i = i0 + 8 * c + 2 * p;
            split_bf16x2(i >= j ? T[i][j] : 0.f, i + 1 >= j ? T[i + 1][j] : 0.f, hi[p], lo[p]);
          }
          const uint32_t off = sw128_chunk(j, (i0 >> 3) + c);
          *reinterpret_cast<uint4*>(rec + kRecTHi + off) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
          *reinterpret_cast<uint4*>(rec + kRecTLo + off) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
        }
      }
      group_barrier(1 + grp, 128);
    }
    __syncthreads();   // shared scratch is reused by the next unit
  }
  if (threadIdx.x == 0) bulk_wait_all();
  tmem_fence_before();
  __syncthreads();
  if (warp == 0) {
    __syncwarp();
    tmem_fence_after();
    tmem_dealloc(tmem, 64);
  }
}

// =========================================================== state =====

// Eight compute warps, an MMA issuer warp and a loader warp, handing over
// through mbarriers only (every wait bounded): the compute warps arrive on
// `rdy` when a phase's operands are written and wait on the tensor core's
// commit barrier themselves; lane 0 of warp 8 waits on `rdy` and issues the
// MMAs; lane 0 of warp 9 issues the stage loads, the L2 prefetch and the
// output stores.
constexpr int kStateThreads = 320;
constexpr int kComputeThreads = 256;
constexpr int kDvHalf = 64;         // value columns per CTA
constexpr int kDvGroup = 32;        // value columns per thread in the state update

// One load stage: [K;Q] image, the prep record, then v ([64 tokens x 64]
// bf16, one 128-byte-swizzled TMA box).
constexpr uint32_t kStKQ = 0;
constexpr uint32_t kStRec = kKQBytes;               // 32768
constexpr uint32_t kStV = 59392;                    // 58 KB, after the record
constexpr uint32_t kStageBytes = kStV + 8192;       // 67584
constexpr uint32_t kStageTx = kKQBytes + kRecBytes + 8192;
static_assert(kStRec + kRecBytes <= kStV, "stage layout");

// Operand images, all 128-byte swizzled:
//   S    MN-major [128 dk x 64 dv]     A of [S^T; S^T] [K;Q]^T (dv = M)
//   R    K-major  [128 x 64 tokens]    rows 0-63 R_hi^T, 64-127 R_lo^T (dv rows)
//   Vn   MN-major [64 tokens x 64 dv]  A of [Vn^T; Vn^T] P^T (dv = M)
//   Vd   MN-major [64 tokens x 64 dv]  hi, then lo 8 KB later (one N=128 B)
//   O    [64 tokens x 64 dv] bf16, two buffers: the output tile of a chunk,
//        written to global memory by a TMA store
struct StateSmemLayout {
  static constexpr uint32_t kStage0 = 0;
  static constexpr uint32_t kStage1 = kStageBytes;
  static constexpr uint32_t kSop = 2 * kStageBytes;   // 135168
  static constexpr uint32_t kR = kSop + 16384;
  static constexpr uint32_t kVn = kR + 16384;
  static constexpr uint32_t kVdhi = kVn + 8192;
  static constexpr uint32_t kVdlo = kVdhi + 8192;
  static constexpr uint32_t kOut = kVdlo + 8192;      // two 8 KB tiles
  static constexpr uint32_t kEg = kOut + 16384;       // exp(G) of the chunk awaiting output
  static constexpr uint32_t kBars = kEg + 256;
  static constexpr uint32_t kTotal = kBars + 128 + 1024;
};
static_assert(StateSmemLayout::kSop % 1024 == 0 && StateSmemLayout::kOut % 1024 == 0,
              "operand alignment");

// TMEM columns.  The S^T and v_new^T products use M=128 with the MN-major A
// descriptor's LBO = 0, so both 64-row halves of the accumulator hold the
// same 64 rows: all 128 lanes carry data and the register work of a phase
// spreads over the four SM sub-partitions.
//   D1[2] (0, 128): [S^T;S^T] [K;Q]^T, rows dv, cols 0-63 (K S)^T, 64-127 (Q S)^T
//   D3 (256):       [T;T] [R_hi | R_lo] + [T_lo;T_lo] R_hi, rows tokens
//   D4 (320):       [Vn^T;Vn^T] P^T = (P v_new)^T, rows dv; shares D3's
//                   columns 64-127 once v_new has been read
//   D5 (384):       K^T [Vd_hi | Vd_lo], rows dk
constexpr uint32_t kTmD1 = 0, kTmD3 = 256, kTmD4 = 320, kTmD5 = 384;


__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, const void* smem_src,
                                             int32_t c0, int32_t c1, int32_t c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(smem_u32(smem_src)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

__global__ void __launch_bounds__(kStateThreads, 1)
gdn_chunk_state_kernel(const __grid_constant__ ChunkTable tab,
                       const __grid_constant__ CUtensorMap tm_v,
                       const __grid_constant__ CUtensorMap tm_o,
                       const uint8_t* __restrict__ kq_records,
                       const uint8_t* __restrict__ records, float* __restrict__ state,
                       uint16_t* __restrict__ o_out, int qk_heads, int value_heads,
                       uint32_t* err) {
  using L = StateSmemLayout;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::kBars);
  uint64_t* smma = full + 2;       // per stage: the tensor core is done with it
  uint64_t* mma_bar = smma + 2;
  uint64_t* stage_free = mma_bar + 1;  // per stage: ready for the next load
  uint64_t* tile_ready = stage_free + 2;  // per output tile: written, store it
  uint64_t* tile_free = tile_ready + 2;   // per output tile: stored, reuse it
  uint64_t* rdy = tile_free + 2;          // compute -> issuer: operands written
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(rdy + 1);
  float* eg_prev = reinterpret_cast<float*>(smem + L::kEg);

  const int dvh = blockIdx.x;
  const int h = blockIdx.y;
  const int seq = blockIdx.z;
  const int kh = h / (value_heads / qk_heads);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int tid = threadIdx.x;
  const int seq_t0 = tab.cu[seq];
  griddep_launch_dependents();   // the tail prologue may launch (it waits for this grid)
  const int seq_len = tab.cu[seq + 1] - seq_t0;
  const int nchunks = (seq_len + kChunk - 1) / kChunk;
  const int chunk0 = tab.chunk_start[seq];
  const int last_n = seq_len - (nchunks - 1) * kChunk;   // tokens in the last chunk

  if (tid == 0) {
    mbar_init(&full[0], 1);
    mbar_init(&full[1], 1);
    mbar_init(&smma[0], 1);
    mbar_init(&smma[1], 1);
    mbar_init(mma_bar, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&stage_free[i], 1);
      mbar_init(&tile_ready[i], kComputeThreads / 32);
      mbar_init(&tile_free[i], 1);
    }
    mbar_init(rdy, kComputeThreads / 32);
    fence_barrier_init();
  }
  if (warp == 0) tmem_alloc(tmem_slot, 512);
  tmem_fence_before();
  __syncthreads();
  tmem_fence_after();
  const uint32_t tmem = *tmem_slot;
  uint8_t* sop = smem + L::kSop;
  uint8_t* rimg = smem + L::kR;
  uint8_t* vn = smem + L::kVn;
  uint8_t* vdhi = smem + L::kVdhi;
  uint8_t* vdlo = smem + L::kVdlo;
  uint8_t* otile = smem + L::kOut;

  if (warp == 8) {
    // ======================================================= MMA issuer ==
    if (lane == 0) {
      uint32_t rdy_phase = 0;
      auto wait_rdy = [&]() -> bool {
        const bool r = mbar_wait(rdy, rdy_phase, err);
        rdy_phase ^= 1u;
        tmem_fence_after();
        return r;
      };
      bool ok = true;
      for (int c = 0; c < nchunks && ok; ++c) {
        const int st = c & 1;
        uint8_t* sb = smem + (st ? L::kStage1 : L::kStage0);
        const uint32_t d1 = tmem + kTmD1 + (c & 1) * 128;
        // D1 = [S^T; S^T] [K;Q]^T (M=128 with LBO 0, N=128, K=128 dk), once S
        // of this chunk is written and the stage has landed.
        if (!(ok = wait_rdy() && mbar_wait(&full[st], (c >> 1) & 1, err))) break;
        {
          constexpr uint32_t id = umma_idesc_bf16(128, 128, true, false);
          const uint32_t akq = smem_u32(sb + kStKQ);
          const uint32_t as = smem_u32(sop);
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            umma_bf16(d1, umma_sdesc(as + kk * 2048u, 0, 1024),
                      umma_sdesc(akq + (kk >> 2) * 16384u + (kk & 3) * 32u, 16, 1024), id,
                      kk > 0 ? 1u : 0u);
          umma_commit(mma_bar);
        }
        // The stage of chunk c - 1 takes chunk c + 1 once its last MMA
        // ((P v_new)^T) completed (every thread finished with it: the rdy of
        // the state update above).
        if (c >= 1) {
          if (!(ok = mbar_wait(&smma[st ^ 1], ((c - 1) >> 1) & 1, err))) break;
          mbar_arrive(&stage_free[st ^ 1]);
        }
        // D3[:, 0:64] = T_hi R_hi + T_lo R_hi, D3[:, 64:128] = T_hi R_lo
        // (M=128 as [T;T] with LBO 0, B = R^T rows K-major).
        if (!(ok = wait_rdy())) break;
        {
          constexpr uint32_t id_w = umma_idesc_bf16(128, 128, true, false);
          constexpr uint32_t id_n = umma_idesc_bf16(128, 64, true, false);
          const uint32_t thi = smem_u32(sb + kStRec + kRecTHi);
          const uint32_t tlo = smem_u32(sb + kStRec + kRecTLo);
          const uint32_t br = smem_u32(rimg);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_bf16(tmem + kTmD3, umma_sdesc(thi + kk * 2048, 0, 1024),
                      umma_sdesc(br + kk * 32, 16, 1024), id_w, kk > 0 ? 1u : 0u);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_bf16(tmem + kTmD3, umma_sdesc(tlo + kk * 2048, 0, 1024),
                      umma_sdesc(br + kk * 32, 16, 1024), id_n, 1u);
          umma_commit(mma_bar);
        }
        // D5 = K^T [Vd_hi | Vd_lo] (the state chain), then D4 = [Vn^T; Vn^T]
        // P^T = (P v_new)^T, completed behind a commit to the stage barrier.
        if (!(ok = wait_rdy())) break;
        {
          constexpr uint32_t id_s = umma_idesc_bf16(128, 128, true, true);
          constexpr uint32_t id_o = umma_idesc_bf16(128, 64, true, false);
          const uint32_t akt = smem_u32(sb + kStKQ);
          const uint32_t ap = smem_u32(sb + kStRec + kRecP);
          const uint32_t bv = smem_u32(vn), bd = smem_u32(vdhi);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            // A = K^T: MN-major view of the [K;Q] rows 0..63, dk slabs 16 KB apart.
            umma_bf16(tmem + kTmD5, umma_sdesc(akt + kk * 2048, 16384, 1024),
                      umma_sdesc(bd + kk * 2048, 8192, 1024), id_s, kk > 0 ? 1u : 0u);
          umma_commit(mma_bar);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_bf16(tmem + kTmD4, umma_sdesc(bv + kk * 2048, 0, 1024),
                      umma_sdesc(ap + kk * 32, 16, 1024), id_o, kk > 0 ? 1u : 0u);
          umma_commit(&smma[st]);
        }
      }
      // Drain: every MMA issued completes before TMEM is released (the
      // compute warps wait on the same commit before the last output).
      umma_commit(mma_bar);
    }
  } else if (warp == 9) {
    // =========================================================== loader ==
    // Stage loads, L2 prefetch and output stores, so that no copy issue sits
    // in front of an MMA.
    if (lane == 0) {
      auto load_stage = [&](int c) {
        const int st = c & 1;
        uint8_t* sb = smem + (st ? L::kStage1 : L::kStage0);
        const int chunk = chunk0 + c;
        mbar_arrive_expect_tx(&full[st], kStageTx);
        bulk_load(sb + kStKQ, kq_records + (static_cast<int64_t>(chunk) * qk_heads + kh) * kKQBytes,
                  kKQBytes, &full[st]);
        bulk_load(sb + kStRec, records + (static_cast<int64_t>(chunk) * value_heads + h) * kRecBytes,
                  kRecBytes, &full[st]);
        tma_load_3d(sb + kStV, &tm_v, &full[st], dvh * kDvHalf, h, seq_t0 + c * kChunk);
      };
      auto prefetch_stage = [&](int c) {
        const int chunk = chunk0 + c;
        prefetch_l2(kq_records + (static_cast<int64_t>(chunk) * qk_heads + kh) * kKQBytes, kKQBytes);
        prefetch_l2(records + (static_cast<int64_t>(chunk) * value_heads + h) * kRecBytes, kRecBytes);
        prefetch_l2_3d(&tm_v, dvh * kDvHalf, h, seq_t0 + c * kChunk);
      };
      tma_prefetch_desc(&tm_v);
      tma_prefetch_desc(&tm_o);
      // Launched to overlap the prep kernel: its records are complete and
      // visible after this (a no-op for an ordinary launch).
      griddep_wait();
      int issued = 0;
      for (; issued < 2 && issued < nchunks; ++issued) load_stage(issued);
      if (nchunks > 2) prefetch_stage(2);
      bool ok = true;
      for (int c = 1; c < nchunks && ok; ++c) {
        // Chunk c + 1 into the stage chunk c - 1 used, once the MMA issuer
        // saw that stage's last MMA complete (at its chunk c).
        if (c + 1 < nchunks) {
          ok = mbar_wait(&stage_free[(c + 1) & 1], ((c - 1) >> 1) & 1, err);
          if (!ok) break;
          load_stage(c + 1);
          issued = c + 2;
          if (c + 2 < nchunks) prefetch_stage(c + 2);
        }
        // The output tile of chunk c - 1, once written (after R of chunk c).
        ok = mbar_wait(&tile_ready[(c - 1) & 1], ((c - 1) >> 1) & 1, err);
        if (!ok) break;
        tma_store_3d(&tm_o, otile + ((c - 1) & 1) * 8192, dvh * kDvHalf, h,
                     seq_t0 + (c - 1) * kChunk);
        bulk_commit();
        if (c >= 2) {
          bulk_wait_read<1>();                    // the store of chunk c - 2 has read its tile
          mbar_arrive(&tile_free[(c - 2) & 1]);
        }
      }
      // The last tile, when it is a full chunk (a shorter one was written
      // row by row).
      if (ok && nchunks > 0 && last_n == kChunk &&
          mbar_wait(&tile_ready[(nchunks - 1) & 1], ((nchunks - 1) >> 1) & 1, err)) {
        tma_store_3d(&tm_o, otile + ((nchunks - 1) & 1) * 8192, dvh * kDvHalf, h,
                     seq_t0 + (nchunks - 1) * kChunk);
        bulk_commit();
      }
      bulk_wait_all();
      // Let stage copies still in flight land before exit (a completed
      // phase returns at once).
      for (int c = (issued > 2 ? issued - 2 : 0); c < issued; ++c) {
        const unsigned long long t_start = global_ns();
        while (!mbar_try_wait(&full[c & 1], (c >> 1) & 1) && global_ns() - t_start < kWaitLimitNs) {
        }
      }
    }
  } else {
    // ============================================================ compute ==
    const float scale = 0.08838834764831845f;
    const int quarter = warp & 3;          // TMEM lane quarter
    const int lrow = quarter * 32 + lane;  // TMEM lane of this thread
    const int cg = warp >> 2;
    const int c0 = cg * kDvGroup;          // state update: value columns [c0, c0 + 32)
    const int half = lrow >> 6;            // which copy of a duplicated 64-row accumulator
    const int r64 = lrow & 63;             // row inside it (dv or token)
    const int seg = 32 * half + 16 * cg;   // the 16 columns this thread takes from it

    uint32_t mma_phase = 0;
    auto wait_mma = [&]() -> bool {
      const bool r = mbar_wait(mma_bar, mma_phase, err);
      mma_phase ^= 1u;
      tmem_fence_after();
      return r;
    };
    // One arrival per compute warp (after every lane's fences and a warp
    // barrier): 8 arrivals instead of 256 on the same mbarrier word.
    auto ready = [&]() {
      fence_proxy_async_smem();
      tmem_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(rdy);
    };

    // State: thread owns key row lrow, value columns dvh*64 + c0 + [0, 32).
    float s[kDvGroup];
    float* sg = state + (static_cast<int64_t>(seq) * value_heads + h) * kHeadDim * kHeadDim;
#pragma unroll
    for (int j = 0; j < kDvGroup; ++j) s[j] = sg[(dvh * kDvHalf + c0 + j) * kHeadDim + lrow];

    auto write_sop = [&]() {
#pragma unroll
      for (int cc = 0; cc < 4; ++cc) {
        uint4 w;
        w.x = pack_bf16x2(s[8 * cc + 0], s[8 * cc + 1]);
        w.y = pack_bf16x2(s[8 * cc + 2], s[8 * cc + 3]);
        w.z = pack_bf16x2(s[8 * cc + 4], s[8 * cc + 5]);
        w.w = pack_bf16x2(s[8 * cc + 6], s[8 * cc + 7]);
        *reinterpret_cast<uint4*>(sop + sw128_chunk(lrow, (c0 >> 3) + cc)) = w;
      }
    };

    // Output of a finished chunk, transposed: this thread has value column
    // d = r64 and tokens [seg, seg + 16): O = scale (exp(G) (Q S) + P v_new),
    // into the 128-byte-swizzled tile (a TMA store writes it out) or, for a
    // last chunk shorter than 64 tokens, straight to its rows.
    int prev_t0 = 0;
    auto write_output = [&](uint32_t d1, int buf, int rows) {
      uint32_t rq[16], rp[16];
      tmem_ld16(tmem_addr(d1, quarter * 32, 64 + seg), rq);
      tmem_ld16(tmem_addr(tmem + kTmD4, quarter * 32, seg), rp);
      float eg[16];
#pragma unroll
      for (int q4 = 0; q4 < 4; ++q4) {
        const float4 e4 = *reinterpret_cast<const float4*>(eg_prev + seg + 4 * q4);
        eg[4 * q4] = e4.x; eg[4 * q4 + 1] = e4.y; eg[4 * q4 + 2] = e4.z; eg[4 * q4 + 3] = e4.w;
      }
      tmem_ld_wait();
      if (rows == kChunk) {
        uint8_t* tile = otile + buf * 8192;
#pragma unroll
        for (int t = 0; t < 16; ++t) {
          const float o = scale * (eg[t] * __uint_as_float(rq[t]) + __uint_as_float(rp[t]));
          *reinterpret_cast<uint16_t*>(tile + sw128_chunk(seg + t, r64 >> 3) + (r64 & 7) * 2) =
              f32_to_bf16_bits(o);
        }
      } else {
        uint16_t* ocol = o_out + (static_cast<int64_t>(prev_t0 + seg) * value_heads + h) * kHeadDim +
                         dvh * kDvHalf + r64;
        const int64_t tstride = static_cast<int64_t>(value_heads) * kHeadDim;
#pragma unroll
        for (int t = 0; t < 16; ++t) {
          if (seg + t < rows) {
            const float o = scale * (eg[t] * __uint_as_float(rq[t]) + __uint_as_float(rp[t]));
            ocol[t * tstride] = f32_to_bf16_bits(o);
          }
        }
      }
    };

    write_sop();
    ready();                                   // S of chunk 0 written
    bool ok = true;
    for (int c = 0; c < nchunks; ++c) {
      const int st = c & 1;
      uint8_t* sb = smem + (st ? L::kStage1 : L::kStage0);
      const float* fac = reinterpret_cast<const float*>(sb + kStRec + kRecF);
      const uint32_t d1 = tmem + kTmD1 + (c & 1) * 128;
      const uint32_t d1_prev = tmem + kTmD1 + ((c & 1) ^ 1) * 128;

      // Output of chunk c - 1 while D1 forms: every thread's state update of
      // chunk c - 1 is done (exp(G) saved; rdy phase 3c: the initial S, then
      // three per chunk), its (P v_new)^T has completed and the store of
      // chunk c - 3 has read the tile buffer.
      if (c > 0) {
        if (!mbar_wait(rdy, c & 1, err) ||
            !mbar_wait(&smma[(c - 1) & 1], ((c - 1) >> 1) & 1, err) ||
            (c >= 3 && !mbar_wait(&tile_free[(c - 1) & 1], ((c - 3) >> 1) & 1, err))) {
          ok = false;
          break;
        }
        tmem_fence_after();
        write_output(d1_prev, (c - 1) & 1, kChunk);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tile_ready[(c - 1) & 1]);
      }
      if (!mbar_wait(&full[st], (c >> 1) & 1, err) || !wait_mma()) { ok = false; break; }

      // R^T = (beta V - beta exp(G) (K S))^T, hi/lo, for value column d = r64
      // and tokens [seg, seg + 16): K-major rows d (hi) and 64 + d (lo).
      {
        uint32_t rk[16];
        tmem_ld16(tmem_addr(d1, quarter * 32, seg), rk);
        float bv[16], bg[16];
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4) {
          const float4 b4 = *reinterpret_cast<const float4*>(fac + kFBeta + seg + 4 * q4);
          const float4 g4 = *reinterpret_cast<const float4*>(fac + kFBetaEG + seg + 4 * q4);
          bv[4 * q4] = b4.x; bv[4 * q4 + 1] = b4.y; bv[4 * q4 + 2] = b4.z; bv[4 * q4 + 3] = b4.w;
          bg[4 * q4] = g4.x; bg[4 * q4 + 1] = g4.y; bg[4 * q4 + 2] = g4.z; bg[4 * q4 + 3] = g4.w;
        }
        float vv[16];
        const uint8_t* vt = sb + kStV;
#pragma unroll
        for (int t = 0; t < 16; ++t)
          vv[t] = bf16_bits_to_f32(*reinterpret_cast<const uint16_t*>(
              vt + sw128_chunk(seg + t, r64 >> 3) + (r64 & 7) * 2));
        tmem_ld_wait();
        uint32_t hi[8], lo[8];
#pragma unroll
        for (int p = 0; p < 8; ++p) {
          const float x0 = bv[2 * p] * vv[2 * p] - bg[2 * p] * __uint_as_float(rk[2 * p]);
          const float x1 = bv[2 * p + 1] * vv[2 * p + 1] - bg[2 * p + 1] * __uint_as_float(rk[2 * p + 1]);
          split_bf16x2(x0, x1, hi[p], lo[p]);
        }
        const int ch = seg >> 3;
        *reinterpret_cast<uint4*>(rimg + sw128_chunk(r64, ch)) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
        *reinterpret_cast<uint4*>(rimg + sw128_chunk(r64, ch + 1)) = make_uint4(hi[4], hi[5], hi[6], hi[7]);
        *reinterpret_cast<uint4*>(rimg + 8192 + sw128_chunk(r64, ch)) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
        *reinterpret_cast<uint4*>(rimg + 8192 + sw128_chunk(r64, ch + 1)) = make_uint4(lo[4], lo[5], lo[6], lo[7]);
      }
      ready();
      if (!wait_mma()) { ok = false; break; }   // D3 complete

      // v_new for token i = r64 and value columns [seg, seg + 16): bf16 v_new
      // and v_new exp(G_C - G) as a hi/lo pair (MN-major rows i).
      {
        uint32_t ra[16], rb[16];
        tmem_ld16(tmem_addr(tmem + kTmD3, quarter * 32, seg), ra);
        tmem_ld16(tmem_addr(tmem + kTmD3, quarter * 32, 64 + seg), rb);
        const float edi = fac[kFED + r64];
        tmem_ld_wait();
        uint32_t vb[8], dh[8], dl[8];
#pragma unroll
        for (int p = 0; p < 8; ++p) {
          const float v0 = __uint_as_float(ra[2 * p]) + __uint_as_float(rb[2 * p]);
          const float v1 = __uint_as_float(ra[2 * p + 1]) + __uint_as_float(rb[2 * p + 1]);
          vb[p] = pack_bf16x2(v0, v1);
          split_bf16x2(v0 * edi, v1 * edi, dh[p], dl[p]);
        }
        const int ch = seg >> 3;
#pragma unroll
        for (int k2 = 0; k2 < 2; ++k2) {
          const uint32_t off = sw128_chunk(r64, ch + k2);
          *reinterpret_cast<uint4*>(vn + off) = make_uint4(vb[4 * k2], vb[4 * k2 + 1], vb[4 * k2 + 2], vb[4 * k2 + 3]);
          *reinterpret_cast<uint4*>(vdhi + off) = make_uint4(dh[4 * k2], dh[4 * k2 + 1], dh[4 * k2 + 2], dh[4 * k2 + 3]);
          *reinterpret_cast<uint4*>(vdlo + off) = make_uint4(dl[4 * k2], dl[4 * k2 + 1], dl[4 * k2 + 2], dl[4 * k2 + 3]);
        }
      }
      ready();
      if (!wait_mma()) { ok = false; break; }   // D5 complete

      // State update (every lane): S = exp(G_C) S + K^T Vd_hi + K^T Vd_lo.
      {
        uint32_t ra[2][16], rb[2][16];
        tmem_ld16(tmem_addr(tmem + kTmD5, quarter * 32, c0), ra[0]);
        tmem_ld16(tmem_addr(tmem + kTmD5, quarter * 32, c0 + 16), ra[1]);
        tmem_ld16(tmem_addr(tmem + kTmD5, quarter * 32, 64 + c0), rb[0]);
        tmem_ld16(tmem_addr(tmem + kTmD5, quarter * 32, 64 + c0 + 16), rb[1]);
        const float dl = fac[kFELast];
        if (tid < 64) eg_prev[tid] = fac[kFEG + tid];
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < kDvGroup; ++j)
          s[j] = dl * s[j] + (__uint_as_float(ra[j >> 4][j & 15]) + __uint_as_float(rb[j >> 4][j & 15]));
        write_sop();
      }
      prev_t0 = seq_t0 + c * kChunk;
      ready();
    }
    // The last output (after the issuer's drain commit and every thread's
    // last state update: rdy phase 3 nchunks) and the state.
    if (ok && wait_mma() && mbar_wait(rdy, nchunks & 1, err) &&
        (nchunks < 3 || last_n < kChunk ||
         mbar_wait(&tile_free[(nchunks - 1) & 1], ((nchunks - 3) >> 1) & 1, err))) {
      if (nchunks > 0) {
        write_output(tmem + kTmD1 + ((nchunks - 1) & 1) * 128, (nchunks - 1) & 1, last_n);
        if (last_n == kChunk) {
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) mbar_arrive(&tile_ready[(nchunks - 1) & 1]);
        }
      }
#pragma unroll
      for (int j = 0; j < kDvGroup; ++j) sg[(dvh * kDvHalf + c0 + j) * kHeadDim + lrow] = s[j];
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

// bf16 [tokens, heads, 128] viewed as {d, head, token}; box {64, 1, 64} with
// 128-byte swizzle.
static bool make_tmap_thd(CUtensorMap* map, const void* base, int64_t tokens, int heads) {
  EncodeTiledFn3 fn = encode_fn3();
  if (fn == nullptr) return false;
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(kHeadDim), static_cast<cuuint64_t>(heads),
                        static_cast<cuuint64_t>(tokens)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(kHeadDim) * 2,
                           static_cast<cuuint64_t>(heads) * kHeadDim * 2};
  cuuint32_t box[3] = {64, 1, static_cast<cuuint32_t>(kChunk)};
  cuuint32_t estr[3] = {1, 1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box,
            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) ==
         CUDA_SUCCESS;
}

bool build_chunk_table(const int32_t* cu_seqlens, int num_seqs, ChunkTable* tab) {
  if (num_seqs < 1 || num_seqs > kMaxSeqsInternal || cu_seqlens[0] != 0) return false;
  tab->num_seqs = num_seqs;
  int64_t chunks = 0;
  for (int s = 0; s <= num_seqs; ++s) {
    tab->cu[s] = cu_seqlens[s];
    tab->chunk_start[s] = static_cast<int32_t>(chunks);
    if (s < num_seqs) {
      const int64_t len = static_cast<int64_t>(cu_seqlens[s + 1]) - cu_seqlens[s];
      if (len < 0) return false;
      chunks += (len + kChunk - 1) / kChunk;
    }
  }
  if (chunks > (1 << 30)) return false;
  tab->total_chunks = static_cast<int32_t>(chunks);
  return true;
}

uint64_t chunk_workspace_bytes(const ChunkTable& tab, int qk_heads, int value_heads) {
  return static_cast<uint64_t>(tab.total_chunks) *
         (static_cast<uint64_t>(qk_heads) * kKQBytes + static_cast<uint64_t>(value_heads) * kRecBytes);
}

cudaError_t launch_chunk_prefill(const ChunkTable& tab, const uint16_t* q, const uint16_t* k,
                                 const uint16_t* v, const uint16_t* a, const uint16_t* b,
                                 const float* A_log, const float* dt_bias, float* state,
                                 uint16_t* o_out, int qk_heads, int value_heads,
                                 uint8_t* scratch, uint32_t* err, cudaStream_t stream,
                                 bool clear_err) {
  if (tab.total_chunks == 0) {
    return clear_err ? cudaMemsetAsync(err, 0, sizeof(uint32_t), stream) : cudaSuccess;
  }
  const int64_t tokens = tab.cu[tab.num_seqs];
  uint8_t* kq_records = scratch;
  uint8_t* records = scratch + static_cast<uint64_t>(tab.total_chunks) * qk_heads * kKQBytes;
  CUtensorMap tq, tk, tv;
  if (!make_tmap_thd(&tq, q, tokens, qk_heads) || !make_tmap_thd(&tk, k, tokens, qk_heads) ||
      !make_tmap_thd(&tv, v, tokens, value_heads))
    return cudaErrorInvalidValue;
  const uint32_t prep_smem = sizeof(PrepSmem) + 1024;
  cudaError_t e = cudaFuncSetAttribute(gdn_chunk_prep_kernel,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, prep_smem);
  if (e != cudaSuccess) return e;
  // All of L1 as shared memory, so that three CTAs fit on an SM.
  e = cudaFuncSetAttribute(gdn_chunk_prep_kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                           100);
  if (e != cudaSuccess) return e;
  // Persistent grid: three CTAs per SM (at most 85 registers x 256 threads and
  // about 75 KB of shared memory each), at most one per unit.  CTAs never
  // wait on one another, so fewer resident slots only means a second wave.
  int device = 0, sms = 0;
  if ((e = cudaGetDevice(&device)) != cudaSuccess) return e;
  if ((e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device)) != cudaSuccess) return e;
  const int64_t units = static_cast<int64_t>(tab.total_chunks) * qk_heads;
  const int pgrid = static_cast<int>(std::min<int64_t>(units, 3 * static_cast<int64_t>(sms)));
  gdn_chunk_prep_kernel<<<pgrid, kPrepThreads, prep_smem, stream>>>(
      tab, tq, tk, a, b, A_log, dt_bias, kq_records, records, qk_heads, value_heads, err,
      clear_err ? 1 : 0);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  note_launches();

  const uint32_t st_smem = StateSmemLayout::kTotal;
  e = cudaFuncSetAttribute(gdn_chunk_state_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           st_smem);
  if (e != cudaSuccess) return e;
  dim3 sgrid(kHeadDim / kDvHalf, value_heads, tab.num_seqs);
  CUtensorMap to;
  if (!make_tmap_thd(&to, o_out, tokens, value_heads)) return cudaErrorInvalidValue;
  // The state pass is launched to overlap the prep kernel: its CTAs take
  // SMs as prep CTAs leave (at once on the SMs a short input leaves idle),
  // allocate TMEM, load their initial state and wait for the prep grid only
  // before the first record (2 x 4096 chunk core 0.255 -> 0.252 ms).
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = sgrid;
  cfg.blockDim = dim3(kStateThreads, 1, 1);
  cfg.dynamicSmemBytes = st_smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, gdn_chunk_state_kernel, tab, tv, to, kq_records, records, state,
                         o_out, qk_heads, value_heads, err);
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e == cudaSuccess) note_launches();
  return e;
}

}  // namespace gdn
