// Single-token recurrent GDN step for B packed sequences (decode).
//
// Replaces PackedDecodeRecurrentV12 (reference provider P:1308-1369: one
// aclnnRecurrentGatedDeltaRule over the packed states) together with the
// gating (aclnnFusedGdnGating, P:3310-3339) and the q/k RmsNorm L2-norm
// (P:3249-3308) that precede it, and optionally the gated-RMSNorm prologue of
// the output tail (P:1434-1494).
//
// Layout and roofline: the state is f32 [B, Hv, 128(v), 128(k)]; the block
// of one (sequence, head) -- a unit -- is 64 KB, read once and written once,
// so the step is HBM-bound at 2 * B * Hv * 64 KB.
//
// Persistent design: one CTA per SM walks the units u = blockIdx.x + i *
// gridDim.x.  Warp 0 drives the copy engine: it bulk-loads each unit's 64 KB
// block into a three-deep shared-memory ring and bulk-stores it back once
// updated, so two blocks stream in while the third is worked on and no
// thread waits on HBM latency.  Warps 1-16 update the block in shared
// memory: warp w owns value rows 8(w-1)..+7, lane l keys 4l..4l+3 of each row
// (one float4), the two dot products per row (S k and S q) are warp-shuffle
// reductions; sixteen warps keep enough of these dependent chains in flight
// that the update is faster than the block's HBM traffic.  The small per-unit
// inputs (q, k, v, z rows, a, b, dt_bias, A_log) are loaded into registers
// one unit ahead by the compute warps, which keeps their 8-byte alignment
// contract.
#include "gdn_common.cuh"
#include "gdn_internal.h"

namespace gdn {

constexpr int kDecodeComputeWarps = 16;
constexpr int kDecodeThreads = 32 * (1 + kDecodeComputeWarps);
constexpr int kDecodeRowsPerWarp = kHeadDim / kDecodeComputeWarps;   // 8
constexpr int kDecodeStages = 3;
constexpr uint32_t kUnitBytes = kHeadDim * kHeadDim * 4;             // 64 KB
constexpr uint32_t kUnitPieces = 4;                                  // bulk copies per unit
constexpr int kComputeBarrier = 1;                                   // named barrier id

struct DecodeSmem {
  float state[kDecodeStages][kHeadDim * kHeadDim];
  float q[kHeadDim];        // L2-normalised, bf16-rounded
  float k[kHeadDim];
  float v[kHeadDim];
  float z[2][kHeadDim];     // double-buffered: read by the output step of a unit
                            // while the next unit's row is published
  float o[kHeadDim];        // bf16-rounded attention output of the unit
  float gamma[kHeadDim];
  float gate[2];            // decay, beta
  uint64_t full[kDecodeStages];
  uint64_t done[kDecodeStages];
};

__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}

__device__ __forceinline__ void bf16x4_to_f32(uint2 raw, float* x) {
  x[0] = bf16_bits_to_f32(raw.x & 0xFFFFu);
  x[1] = bf16_bits_to_f32(raw.x >> 16);
  x[2] = bf16_bits_to_f32(raw.y & 0xFFFFu);
  x[3] = bf16_bits_to_f32(raw.y >> 16);
}

// q/k RmsNorm with gamma = bf16(1/sqrt(128)) and eps = 1e-6/128, output
// rounded to bf16 as the reference's RmsNorm output tensor is bf16.
__device__ __forceinline__ void l2norm_row_warp(uint2 raw, float* dst, int lane) {
  float x[4];
  bf16x4_to_f32(raw, x);
  const float ss = warp_sum(x[0] * x[0] + x[1] * x[1] + x[2] * x[2] + x[3] * x[3]);
  const float gamma = round_bf16(0.08838834764831845f);
  const float rstd = rsqrtf(ss * (1.0f / 128.0f) + 1.0e-6f / 128.0f);
#pragma unroll
  for (int i = 0; i < 4; ++i) dst[lane * 4 + i] = round_bf16(x[i] * rstd * gamma);
}

struct UnitIndex {
  int seq, h, kh;
};
__device__ __forceinline__ UnitIndex unit_index(int u, int qk_heads, int value_heads) {
  UnitIndex x;
  x.seq = u / value_heads;
  x.h = u - x.seq * value_heads;
  x.kh = x.h / (value_heads / qk_heads);
  return x;
}

__device__ __forceinline__ float* unit_state(const UnitIndex& x, float* state,
                                             const uint64_t* state_rows, int value_heads) {
  float* row = state_rows != nullptr
                   ? reinterpret_cast<float*>(state_rows[x.seq])
                   : state + static_cast<int64_t>(x.seq) * value_heads * kHeadDim * kHeadDim;
  return row + static_cast<int64_t>(x.h) * kHeadDim * kHeadDim;
}

__global__ void __launch_bounds__(kDecodeThreads, 1)
gdn_decode_kernel(const uint16_t* __restrict__ q, const uint16_t* __restrict__ k,
                  const uint16_t* __restrict__ v, const uint16_t* __restrict__ a,
                  const uint16_t* __restrict__ b, const float* __restrict__ A_log,
                  const float* __restrict__ dt_bias, float* __restrict__ state,
                  uint16_t* __restrict__ o_out, const uint16_t* __restrict__ z,
                  const uint16_t* __restrict__ gamma, uint16_t* __restrict__ gated_out,
                  const uint64_t* __restrict__ state_rows, int units, int qk_heads,
                  int value_heads, const uint8_t* __restrict__ l2_pre, uint64_t l2_pre_bytes,
                  uint32_t* err, int clear_err) {
  // With clear_err the call's error word starts at zero here instead of by a
  // separate memset, before the tail GEMM is let in (errors are recorded only
  // after bounded waits of seconds, or for a misaligned slot-table row, which
  // this mode never receives).
  if (clear_err && blockIdx.x == 0 && threadIdx.x == 0) *err = 0u;
  griddep_launch_dependents();   // the tail GEMM may start streaming W now
  extern __shared__ uint8_t smem_raw[];
  DecodeSmem& sm = *reinterpret_cast<DecodeSmem*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~static_cast<uintptr_t>(127));
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int n = units > static_cast<int>(blockIdx.x)
                    ? (units - 1 - static_cast<int>(blockIdx.x)) / static_cast<int>(gridDim.x) + 1
                    : 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kDecodeStages; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.done[s], 1);
    }
    fence_barrier_init();
  }
  if (gated_out != nullptr && threadIdx.x < kHeadDim)
    sm.gamma[threadIdx.x] = bf16_bits_to_f32(gamma[threadIdx.x]);
  __syncthreads();

  if (warp == 0) {
    // ------------------------------------------------ copy-engine driver --
    if (lane == 0) {
      for (int i = 0; i < n + kDecodeStages; ++i) {
        // Store unit i - S once its update is done, which frees its stage.
        const int j = i - kDecodeStages;
        if (j >= 0 && j < n) {
          const int s = j % kDecodeStages;
          if (!mbar_wait(&sm.done[s], static_cast<uint32_t>(j / kDecodeStages) & 1u, err)) break;
          const UnitIndex x = unit_index(static_cast<int>(blockIdx.x) + j * gridDim.x, qk_heads,
                                         value_heads);
          float* g = unit_state(x, state, state_rows, value_heads);
          if ((reinterpret_cast<uintptr_t>(g) & 15u) == 0) {
            for (uint32_t p = 0; p < kUnitPieces; ++p)
              bulk_store(reinterpret_cast<uint8_t*>(g) + p * (kUnitBytes / kUnitPieces),
                         reinterpret_cast<uint8_t*>(sm.state[s]) + p * (kUnitBytes / kUnitPieces),
                         kUnitBytes / kUnitPieces);
            bulk_commit();
            bulk_wait_read<0>();
          }
        }
        if (i < n) {
          const int s = i % kDecodeStages;
          const UnitIndex x = unit_index(static_cast<int>(blockIdx.x) + i * gridDim.x, qk_heads,
                                         value_heads);
          const float* g = unit_state(x, state, state_rows, value_heads);
          if ((reinterpret_cast<uintptr_t>(g) & 15u) != 0) {
            record_error(err, kErrMisaligned);   // block left alone; the phase still completes
            mbar_arrive(&sm.full[s]);
            continue;
          }
          mbar_arrive_expect_tx(&sm.full[s], kUnitBytes);
          for (uint32_t p = 0; p < kUnitPieces; ++p)
            bulk_load(reinterpret_cast<uint8_t*>(sm.state[s]) + p * (kUnitBytes / kUnitPieces),
                      reinterpret_cast<const uint8_t*>(g) + p * (kUnitBytes / kUnitPieces),
                      kUnitBytes / kUnitPieces, &sm.full[s]);
          if (i == n - 1 && l2_pre != nullptr) {
            // Last state load issued: warm L2 with this CTA's share of the
            // buffer the next kernel reads (the tail GEMM's weight), while
            // the remaining units drain.
            const uint64_t per = ((l2_pre_bytes + gridDim.x - 1) / gridDim.x + 15) & ~15ull;
            const uint64_t lim = per * (blockIdx.x + 1);
            const uint64_t end = l2_pre_bytes < lim ? l2_pre_bytes : lim;
            for (uint64_t off = per * blockIdx.x; off + 16 <= end; off += 32768) {
              const uint64_t len = (end - off < 32768ull ? end - off : 32768ull) & ~15ull;
              prefetch_l2(l2_pre + off, static_cast<uint32_t>(len));
            }
          }
        }
      }
      bulk_wait_all();   // every store has landed before the CTA leaves
    }
    __syncwarp();
    return;
  }

  // --------------------------------------------------- compute warps 1-16 --
  const int cw = warp - 1;
  // Per-role prefetch of the next unit's small inputs (one unit ahead).
  uint2 pre = make_uint2(0u, 0u);
  uint16_t pre_a = 0, pre_b = 0;
  float pre_dt = 0.f, pre_alog = 0.f;
  auto prefetch = [&](int i) {
    if (i >= n) return;
    const UnitIndex x = unit_index(static_cast<int>(blockIdx.x) + i * gridDim.x, qk_heads,
                                   value_heads);
    const int64_t qk_row = (static_cast<int64_t>(x.seq) * qk_heads + x.kh) * kHeadDim;
    const int64_t v_row = (static_cast<int64_t>(x.seq) * value_heads + x.h) * kHeadDim;
    if (cw == 0) pre = *reinterpret_cast<const uint2*>(q + qk_row + lane * 4);
    else if (cw == 1) pre = *reinterpret_cast<const uint2*>(k + qk_row + lane * 4);
    else if (cw == 2) pre = *reinterpret_cast<const uint2*>(v + v_row + lane * 4);
    else if (cw == 3 && gated_out != nullptr)
      pre = *reinterpret_cast<const uint2*>(z + v_row + lane * 4);
    else if (cw == 4 && lane == 0) {
      const int64_t gi = static_cast<int64_t>(x.seq) * value_heads + x.h;
      pre_a = a[gi];
      pre_b = b[gi];
      pre_dt = dt_bias[x.h];
      pre_alog = A_log[x.h];
    }
  };
  prefetch(0);

  const float scale = 0.08838834764831845f;
  const int row0 = cw * kDecodeRowsPerWarp;
  for (int i = 0; i < n; ++i) {
    const UnitIndex x = unit_index(static_cast<int>(blockIdx.x) + i * gridDim.x, qk_heads,
                                   value_heads);
    const int s = i % kDecodeStages;
    // Publish this unit's small inputs, then fetch the next unit's.
    if (cw == 0) {
      l2norm_row_warp(pre, sm.q, lane);
    } else if (cw == 1) {
      l2norm_row_warp(pre, sm.k, lane);
    } else if (cw == 2) {
      bf16x4_to_f32(pre, sm.v + lane * 4);
    } else if (cw == 3) {
      if (gated_out != nullptr) bf16x4_to_f32(pre, sm.z[i & 1] + lane * 4);
    } else if (cw == 4 && lane == 0) {
      // aclnnFusedGdnGating: softplus with beta 1, threshold 20.
      const float xx = bf16_bits_to_f32(pre_a) + pre_dt;
      const float sp = xx > 20.0f ? xx : log1pf(expf(xx));
      const float gl = -expf(pre_alog) * sp;
      sm.gate[0] = expf(gl);
      sm.gate[1] = round_bf16(1.0f / (1.0f + expf(-bf16_bits_to_f32(pre_b))));
    }
    prefetch(i + 1);
    const bool landed = mbar_wait(&sm.full[s], static_cast<uint32_t>(i / kDecodeStages) & 1u, err);
    named_barrier_sync(kComputeBarrier, 32 * kDecodeComputeWarps);

    float* blk = sm.state[s];
    const float decay = sm.gate[0];
    const float beta = sm.gate[1];
    const float4 kk = reinterpret_cast<const float4*>(sm.k)[lane];
    const float4 qq = reinterpret_cast<const float4*>(sm.q)[lane];
    float4 r[kDecodeRowsPerWarp];
#pragma unroll
    for (int t = 0; t < kDecodeRowsPerWarp; ++t)
      r[t] = reinterpret_cast<const float4*>(blk + (row0 + t) * kHeadDim)[lane];
#pragma unroll
    for (int t = 0; t < kDecodeRowsPerWarp; ++t) {
      float4 rr = r[t];
      rr.x *= decay; rr.y *= decay; rr.z *= decay; rr.w *= decay;
      const float kv = warp_sum(rr.x * kk.x + rr.y * kk.y + rr.z * kk.z + rr.w * kk.w);
      const float delta = beta * (sm.v[row0 + t] - kv);
      rr.x += delta * kk.x; rr.y += delta * kk.y; rr.z += delta * kk.z; rr.w += delta * kk.w;
      const float oq = warp_sum(rr.x * qq.x + rr.y * qq.y + rr.z * qq.z + rr.w * qq.w);
      reinterpret_cast<float4*>(blk + (row0 + t) * kHeadDim)[lane] = rr;
      if (lane == 0) sm.o[row0 + t] = round_bf16(scale * oq);
    }
    fence_proxy_async_smem();   // the bulk store reads the updated block
    named_barrier_sync(kComputeBarrier, 32 * kDecodeComputeWarps);
    if (cw == 0) {
      if (lane == 0 && landed) mbar_arrive(&sm.done[s]);
      const int64_t v_row = (static_cast<int64_t>(x.seq) * value_heads + x.h) * kHeadDim;
      float xo[4];
#pragma unroll
      for (int t = 0; t < 4; ++t) xo[t] = sm.o[lane * 4 + t];
      if (o_out != nullptr) {
        uint2 w;
        w.x = pack_bf16x2(xo[0], xo[1]);
        w.y = pack_bf16x2(xo[2], xo[3]);
        *reinterpret_cast<uint2*>(o_out + v_row + lane * 4) = w;
      }
      if (gated_out != nullptr) {
        // Tail prologue with the reference's rounding points:
        // bf16(RmsNorm(o) * gamma), bf16(SiLU(z)), bf16(product).
        const float ss = warp_sum(xo[0] * xo[0] + xo[1] * xo[1] + xo[2] * xo[2] + xo[3] * xo[3]);
        const float rstd = rsqrtf(ss * (1.0f / 128.0f) + 1.0e-6f);
        float res[4];
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          const float zz = sm.z[i & 1][lane * 4 + t];
          const float nrm = round_bf16(xo[t] * rstd * sm.gamma[lane * 4 + t]);
          const float sl = round_bf16(__fdividef(zz, 1.0f + __expf(-zz)));
          res[t] = nrm * sl;
        }
        uint2 w;
        w.x = pack_bf16x2(res[0], res[1]);
        w.y = pack_bf16x2(res[2], res[3]);
        *reinterpret_cast<uint2*>(gated_out + v_row + lane * 4) = w;
      }
    }
    if (!landed) break;
  }
}

static uint32_t decode_smem_bytes() { return sizeof(DecodeSmem) + 128; }

cudaError_t launch_decode(const uint16_t* q, const uint16_t* k, const uint16_t* v,
                          const uint16_t* a, const uint16_t* b, const float* A_log,
                          const float* dt_bias, float* state, uint16_t* o_out,
                          const uint16_t* z, const uint16_t* gamma, uint16_t* gated_out,
                          int batch, int qk_heads, int value_heads, cudaStream_t stream,
                          const uint64_t* state_rows, uint32_t* err, const void* l2_prefetch,
                          uint64_t l2_prefetch_bytes, bool clear_err) {
  const int units = batch * value_heads;
  if (units <= 0) return cudaSuccess;
  const uint32_t smem = decode_smem_bytes();
  cudaError_t e = cudaFuncSetAttribute(gdn_decode_kernel,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  const int grid = units < sm_count() ? units : sm_count();
  gdn_decode_kernel<<<grid, kDecodeThreads, smem, stream>>>(
      q, k, v, a, b, A_log, dt_bias, state, o_out, z, gamma, gated_out, state_rows, units,
      qk_heads, value_heads, static_cast<const uint8_t*>(l2_prefetch), l2_prefetch_bytes, err,
      clear_err && state_rows == nullptr ? 1 : 0);
  e = cudaGetLastError();
  if (e == cudaSuccess) note_launches();
  return e;
}

}  // namespace gdn
