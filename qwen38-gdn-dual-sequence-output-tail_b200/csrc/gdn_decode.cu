// Single-token recurrent GDN step for B packed sequences (decode).
//
// Replaces PackedDecodeRecurrentV12 (reference provider P:1308-1369: one
// aclnnRecurrentGatedDeltaRule over the packed states) together with the
// gating (aclnnFusedGdnGating, P:3310-3339) and the q/k RmsNorm L2-norm
// (P:3249-3308) that precede it, and optionally the gated-RMSNorm prologue of
// the output tail (P:1434-1494).
//
// Layout and roofline: the state is f32 [B, Hv, 128(v), 128(k)], one 512-byte
// row per value index.  Each row is read once and written once, so the step
// is HBM-bound at 2 * B * Hv * 128 * 128 * 4 bytes.  One warp owns 16 rows:
// lane l holds keys 4l..4l+3 of every row as a float4 (128-bit coalesced
// access, 512 contiguous bytes per warp instruction), the two dot products
// per row (S k and S q) are warp-shuffle reductions, and the row update is
// done in registers between the load and the store.
#include "gdn_common.cuh"
#include "gdn_internal.h"

namespace gdn {

constexpr int kDecodeThreads = 256;          // 8 warps
constexpr int kDecodeRowsPerWarp = 16;       // 8 * 16 = 128 value rows

__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}

// q/k RmsNorm with gamma = bf16(1/sqrt(128)) and eps = 1e-6/128, output
// rounded to bf16 as the reference's RmsNorm output tensor is bf16.
__device__ __forceinline__ void l2norm_row_warp(const uint16_t* src, float* dst, int lane) {
  const uint2 raw = *reinterpret_cast<const uint2*>(src + lane * 4);
  float x[4] = {bf16_bits_to_f32(raw.x & 0xFFFFu), bf16_bits_to_f32(raw.x >> 16),
                bf16_bits_to_f32(raw.y & 0xFFFFu), bf16_bits_to_f32(raw.y >> 16)};
  const float ss = warp_sum(x[0] * x[0] + x[1] * x[1] + x[2] * x[2] + x[3] * x[3]);
  const float gamma = round_bf16(0.08838834764831845f);
  const float rstd = rsqrtf(ss * (1.0f / 128.0f) + 1.0e-6f / 128.0f);
#pragma unroll
  for (int i = 0; i < 4; ++i) dst[lane * 4 + i] = round_bf16(x[i] * rstd * gamma);
}

__global__ void __launch_bounds__(kDecodeThreads, 2)
gdn_decode_kernel(const uint16_t* __restrict__ q, const uint16_t* __restrict__ k,
                  const uint16_t* __restrict__ v, const uint16_t* __restrict__ a,
                  const uint16_t* __restrict__ b, const float* __restrict__ A_log,
                  const float* __restrict__ dt_bias, float* __restrict__ state,
                  uint16_t* __restrict__ o_out, const uint16_t* __restrict__ z,
                  const uint16_t* __restrict__ gamma, uint16_t* __restrict__ gated_out,
                  const uint64_t* __restrict__ state_rows, int qk_heads, int value_heads) {
  griddep_launch_dependents();   // the tail GEMM may start streaming W now
  const int h = blockIdx.x;
  const int seq = blockIdx.y;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int kh = h / (value_heads / qk_heads);

  __shared__ __align__(16) float s_q[kHeadDim];
  __shared__ __align__(16) float s_k[kHeadDim];
  __shared__ __align__(16) float s_v[kHeadDim];
  __shared__ __align__(16) float s_o[kHeadDim];
  __shared__ float s_gate[2];

  const int64_t qk_row = (static_cast<int64_t>(seq) * qk_heads + kh) * kHeadDim;
  const int64_t v_row = (static_cast<int64_t>(seq) * value_heads + h) * kHeadDim;
  // The sequence's state: row `seq` of the contiguous [S, Hv, 128, 128]
  // state, or the [Hv, 128, 128] row at the address given for it (slot
  // binding: the rows can sit anywhere in a state pool).
  float* srow0 = (state_rows != nullptr
                      ? reinterpret_cast<float*>(state_rows[seq])
                      : state + static_cast<int64_t>(seq) * value_heads * kHeadDim * kHeadDim) +
                 static_cast<int64_t>(h) * kHeadDim * kHeadDim;

  // Issue the state loads first: they are the long-latency stream.
  float4 s[kDecodeRowsPerWarp];
  const int row0 = warp * kDecodeRowsPerWarp;
#pragma unroll
  for (int i = 0; i < kDecodeRowsPerWarp; ++i) {
    s[i] = __ldcs(reinterpret_cast<const float4*>(srow0 + (row0 + i) * kHeadDim) + lane);
  }

  if (warp == 0) {
    l2norm_row_warp(q + qk_row, s_q, lane);
  } else if (warp == 1) {
    l2norm_row_warp(k + qk_row, s_k, lane);
  } else if (warp == 2) {
    const uint2 raw = *reinterpret_cast<const uint2*>(v + v_row + lane * 4);
    s_v[lane * 4 + 0] = bf16_bits_to_f32(raw.x & 0xFFFFu);
    s_v[lane * 4 + 1] = bf16_bits_to_f32(raw.x >> 16);
    s_v[lane * 4 + 2] = bf16_bits_to_f32(raw.y & 0xFFFFu);
    s_v[lane * 4 + 3] = bf16_bits_to_f32(raw.y >> 16);
  } else if (warp == 3 && lane == 0) {
    // aclnnFusedGdnGating: softplus with beta 1, threshold 20.
    const int64_t gi = static_cast<int64_t>(seq) * value_heads + h;
    const float x = bf16_bits_to_f32(a[gi]) + dt_bias[h];
    const float sp = x > 20.0f ? x : log1pf(expf(x));
    const float g = -expf(A_log[h]) * sp;
    s_gate[0] = expf(g);
    s_gate[1] = round_bf16(1.0f / (1.0f + expf(-bf16_bits_to_f32(b[gi]))));
  }
  __syncthreads();

  const float decay = s_gate[0];
  const float beta = s_gate[1];
  const float4 kk = reinterpret_cast<const float4*>(s_k)[lane];
  const float4 qq = reinterpret_cast<const float4*>(s_q)[lane];
  const float scale = 0.08838834764831845f;
#pragma unroll
  for (int i = 0; i < kDecodeRowsPerWarp; ++i) {
    float4 r = s[i];
    r.x *= decay; r.y *= decay; r.z *= decay; r.w *= decay;
    const float kv = warp_sum(r.x * kk.x + r.y * kk.y + r.z * kk.z + r.w * kk.w);
    const float delta = beta * (s_v[row0 + i] - kv);
    r.x += delta * kk.x; r.y += delta * kk.y; r.z += delta * kk.z; r.w += delta * kk.w;
    const float oq = warp_sum(r.x * qq.x + r.y * qq.y + r.z * qq.z + r.w * qq.w);
    __stcs(reinterpret_cast<float4*>(srow0 + (row0 + i) * kHeadDim) + lane, r);
    if (lane == 0) s_o[row0 + i] = round_bf16(scale * oq);
  }
  __syncthreads();

  if (warp == 0) {
    float x[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) x[i] = s_o[lane * 4 + i];
    if (o_out != nullptr) {
      uint2 w;
      w.x = pack_bf16x2(x[0], x[1]);
      w.y = pack_bf16x2(x[2], x[3]);
      *reinterpret_cast<uint2*>(o_out + v_row + lane * 4) = w;
    }
    if (gated_out != nullptr) {
      // Tail prologue with the reference's rounding points:
      // bf16(RmsNorm(o) * gamma), bf16(SiLU(z)), bf16(product).
      const float ss = warp_sum(x[0] * x[0] + x[1] * x[1] + x[2] * x[2] + x[3] * x[3]);
      const float rstd = rsqrtf(ss * (1.0f / 128.0f) + 1.0e-6f);
      const uint2 zr = *reinterpret_cast<const uint2*>(z + v_row + lane * 4);
      const uint2 gr = *reinterpret_cast<const uint2*>(gamma + lane * 4);
      const float zz[4] = {bf16_bits_to_f32(zr.x & 0xFFFFu), bf16_bits_to_f32(zr.x >> 16),
                           bf16_bits_to_f32(zr.y & 0xFFFFu), bf16_bits_to_f32(zr.y >> 16)};
      const float gg[4] = {bf16_bits_to_f32(gr.x & 0xFFFFu), bf16_bits_to_f32(gr.x >> 16),
                           bf16_bits_to_f32(gr.y & 0xFFFFu), bf16_bits_to_f32(gr.y >> 16)};
      float out[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float n = round_bf16(x[i] * rstd * gg[i]);
        const float sl = round_bf16(__fdividef(zz[i], 1.0f + __expf(-zz[i])));
        out[i] = n * sl;
      }
      uint2 w;
      w.x = pack_bf16x2(out[0], out[1]);
      w.y = pack_bf16x2(out[2], out[3]);
      *reinterpret_cast<uint2*>(gated_out + v_row + lane * 4) = w;
    }
  }
}

cudaError_t launch_decode(const uint16_t* q, const uint16_t* k, const uint16_t* v,
                          const uint16_t* a, const uint16_t* b, const float* A_log,
                          const float* dt_bias, float* state, uint16_t* o_out,
                          const uint16_t* z, const uint16_t* gamma, uint16_t* gated_out,
                          int batch, int qk_heads, int value_heads, cudaStream_t stream,
                          const uint64_t* state_rows) {
  dim3 grid(value_heads, batch);
  gdn_decode_kernel<<<grid, kDecodeThreads, 0, stream>>>(q, k, v, a, b, A_log, dt_bias, state,
                                                         o_out, z, gamma, gated_out, state_rows,
                                                         qk_heads, value_heads);
  return cudaGetLastError();
}

}  // namespace gdn
