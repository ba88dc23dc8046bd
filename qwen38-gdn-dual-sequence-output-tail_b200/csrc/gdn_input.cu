// Input side of the layer: x -> q, k, v, z, a, b.
//
// Replaces the reference's projections and causal conv (provider P:3101-3247):
// four aclnnMatmul calls (qkv, z, a, b), aclnnCausalConv1d over qkv with the
// conv-state update, then a Q/K/V split by memcpy/slice/pack kernels.  Here
// the projections run on the tcgen05 GEMM of gdn_tail.cu (a and b as one
// GEMM over the stacked, zero-padded [w_a; w_b]), and one memory-bound kernel
// does the depthwise causal conv (width 4, history 3) + SiLU for every token
// and writes q, k and v in place of the split; a second kernel writes the
// new conv state and a third splits a and b.
//
// Conv arithmetic (the CPU restatement sums the same way): for channel c and
// token t, acc = w0 x[t-3]; acc = fma(w1, x[t-2], acc); acc = fma(w2,
// x[t-1], acc); acc = fma(w3, x[t], acc); out = bf16(acc / (1 + exp(-acc)))
// with the fast exp and divide (as the tail prologue's SiLU), rows before a
// sequence taken from its conv state (zero when the call has no context).
#include <algorithm>

#include "gdn_common.cuh"
#include "gdn_internal.h"

namespace gdn {

namespace {

__device__ __forceinline__ int seq_of_chunk(const ChunkTable& tab, int chunk) {
  int lo = 0, hi = tab.num_seqs - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (tab.chunk_start[mid] <= chunk) lo = mid; else hi = mid - 1;
  }
  return lo;
}

__device__ __forceinline__ void unpack8(const uint4& v, float (&f)[8]) {
  f[0] = bf16lo_f32(v.x); f[1] = bf16hi_f32(v.x);
  f[2] = bf16lo_f32(v.y); f[3] = bf16hi_f32(v.y);
  f[4] = bf16lo_f32(v.z); f[5] = bf16hi_f32(v.z);
  f[6] = bf16lo_f32(v.w); f[7] = bf16hi_f32(v.w);
}

// Tokens per thread: a quarter of a 64-token chunk, all of its rows loaded
// before the first is used (16 loads in flight per thread).
constexpr int kConvRun = 16;

// One thread: 8 channels (16 bytes) x a run of kConvRun tokens of one chunk of
// a sequence, with a sliding window of the three previous rows.
// grid (channels / 8 / blockDim.x, chunks * 64 / kConvRun).
__global__ void __launch_bounds__(128)
causal_conv_split_kernel(const __grid_constant__ ChunkTable tab,
                         const uint16_t* __restrict__ qkv, const uint16_t* __restrict__ w,
                         const uint16_t* __restrict__ conv_state, int use_state,
                         uint16_t* __restrict__ q, uint16_t* __restrict__ k,
                         uint16_t* __restrict__ v, int qk_dim, int v_dim) {
  const int channels = 2 * qk_dim + v_dim;
  const int c8 = (blockIdx.x * blockDim.x + threadIdx.x) * 8;
  if (c8 >= channels) return;
  constexpr int kRunsPerChunk = kChunk / kConvRun;
  const int chunk = blockIdx.y / kRunsPerChunk;
  const int seq = seq_of_chunk(tab, chunk);
  const int s0 = tab.cu[seq];
  const int t0 = s0 + (chunk - tab.chunk_start[seq]) * kChunk +
                 (blockIdx.y % kRunsPerChunk) * kConvRun;
  const int t1 = min(t0 + kConvRun, tab.cu[seq + 1]);
  if (t0 >= t1) return;
  uint4 rows[kConvRun];
#pragma unroll
  for (int i = 0; i < kConvRun; ++i)
    rows[i] = t0 + i < t1
                  ? *reinterpret_cast<const uint4*>(qkv + static_cast<int64_t>(t0 + i) * channels + c8)
                  : make_uint4(0u, 0u, 0u, 0u);

  float wt[4][8];
#pragma unroll
  for (int kk = 0; kk < 4; ++kk)
    unpack8(*reinterpret_cast<const uint4*>(w + static_cast<int64_t>(kk) * channels + c8), wt[kk]);
  // History rows t0-3, t0-2, t0-1: inside the sequence from qkv, before it
  // from the state (row 2 = the most recent) or zero.
  float h[3][8];
#pragma unroll
  for (int j = 0; j < 3; ++j) {
    const int r = t0 - 3 + j;
    uint4 raw = make_uint4(0u, 0u, 0u, 0u);
    if (r >= s0) {
      raw = *reinterpret_cast<const uint4*>(qkv + static_cast<int64_t>(r) * channels + c8);
    } else if (use_state) {
      const int idx = 3 - (s0 - r);
      raw = *reinterpret_cast<const uint4*>(
          conv_state + (static_cast<int64_t>(seq) * 3 + idx) * channels + c8);
    }
    unpack8(raw, h[j]);
  }
  uint16_t* dst;
  int64_t dst_stride;
  int col;
  if (c8 < qk_dim) { dst = q; dst_stride = qk_dim; col = c8; }
  else if (c8 < 2 * qk_dim) { dst = k; dst_stride = qk_dim; col = c8 - qk_dim; }
  else { dst = v; dst_stride = v_dim; col = c8 - 2 * qk_dim; }

#pragma unroll
  for (int i = 0; i < kConvRun; ++i) {
    const int t = t0 + i;
    if (t >= t1) break;
    float x[8];
    unpack8(rows[i], x);
    float y[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      float acc = wt[0][e] * h[0][e];
      acc = fmaf(wt[1][e], h[1][e], acc);
      acc = fmaf(wt[2][e], h[2][e], acc);
      acc = fmaf(wt[3][e], x[e], acc);
      y[e] = __fdividef(acc, 1.0f + __expf(-acc));
      h[0][e] = h[1][e];
      h[1][e] = h[2][e];
      h[2][e] = x[e];
    }
    *reinterpret_cast<uint4*>(dst + static_cast<int64_t>(t) * dst_stride + col) =
        make_uint4(pack_bf16x2(y[0], y[1]), pack_bf16x2(y[2], y[3]), pack_bf16x2(y[4], y[5]),
                   pack_bf16x2(y[6], y[7]));
  }
}

// New conv state: the last three rows of [history; x] of each sequence.
// Runs after the conv kernel (which reads the old state).  grid (channel
// groups, sequences).
__global__ void __launch_bounds__(128)
conv_state_update_kernel(const __grid_constant__ ChunkTable tab,
                         const uint16_t* __restrict__ qkv, uint16_t* __restrict__ conv_state,
                         int use_state, int channels) {
  const int c8 = (blockIdx.x * blockDim.x + threadIdx.x) * 8;
  if (c8 >= channels) return;
  const int seq = blockIdx.y;
  const int s0 = tab.cu[seq];
  const int len = tab.cu[seq + 1] - s0;
  uint16_t* st = conv_state + static_cast<int64_t>(seq) * 3 * channels + c8;
  uint4 rows[3];
#pragma unroll
  for (int i = 0; i < 3; ++i) {
    const int e = len + i;  // row of [history (3 rows); x (len rows)]
    if (e >= 3) {
      rows[i] = *reinterpret_cast<const uint4*>(qkv + static_cast<int64_t>(s0 + e - 3) * channels + c8);
    } else {
      rows[i] = use_state ? *reinterpret_cast<const uint4*>(st + static_cast<int64_t>(e) * channels)
                          : make_uint4(0u, 0u, 0u, 0u);
    }
  }
#pragma unroll
  for (int i = 0; i < 3; ++i)
    *reinterpret_cast<uint4*>(st + static_cast<int64_t>(i) * channels) = rows[i];
}

// a = ab[:, 0:hv], b = ab[:, hv:2 hv] (ab row stride n_ab), one element per
// thread.
__global__ void split_gates_kernel(const uint16_t* __restrict__ ab, uint16_t* __restrict__ a,
                                   uint16_t* __restrict__ b, int64_t tokens, int hv, int n_ab) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= tokens * hv) return;
  const int64_t t = i / hv;
  const int h = static_cast<int>(i - t * hv);
  a[i] = ab[t * n_ab + h];
  b[i] = ab[t * n_ab + hv + h];
}

}  // namespace

int input_gate_width(int value_heads) { return ((2 * value_heads + 63) / 64) * 64; }

uint64_t input_side_scratch_bytes(int64_t tokens, int qk_heads, int value_heads, int hidden) {
  auto r256 = [](uint64_t x) { return (x + 255u) & ~static_cast<uint64_t>(255u); };
  const int64_t channels = static_cast<int64_t>(2 * qk_heads + value_heads) * kHeadDim;
  const int n_ab = input_gate_width(value_heads);
  uint64_t gemm_ws = tail_gemm_workspace_bytes(tokens, static_cast<int>(channels), hidden);
  gemm_ws = std::max<uint64_t>(gemm_ws, tail_gemm_workspace_bytes(tokens, value_heads * kHeadDim, hidden));
  gemm_ws = std::max<uint64_t>(gemm_ws, tail_gemm_workspace_bytes(tokens, n_ab, hidden));
  return r256(static_cast<uint64_t>(tokens) * channels * 2) +          // qkv
         r256(static_cast<uint64_t>(tokens) * n_ab * 2) +              // ab
         r256(static_cast<uint64_t>(n_ab) * hidden * 2) +              // [w_a; w_b; 0]
         r256(gemm_ws);
}

cudaError_t launch_input_side(const ChunkTable& tab, const uint16_t* x, const uint16_t* w_qkv,
                              const uint16_t* w_z, const uint16_t* w_a, const uint16_t* w_b,
                              const uint16_t* conv_w, uint16_t* conv_state, int use_state,
                              uint16_t* q, uint16_t* k, uint16_t* v, uint16_t* z, uint16_t* a,
                              uint16_t* b, int qk_heads, int value_heads, int hidden,
                              uint8_t* scratch, uint32_t* err, cudaStream_t stream) {
  auto r256 = [](uint64_t x_) { return (x_ + 255u) & ~static_cast<uint64_t>(255u); };
  const int64_t tokens = tab.cu[tab.num_seqs];
  const int qk_dim = qk_heads * kHeadDim, v_dim = value_heads * kHeadDim;
  const int channels = 2 * qk_dim + v_dim;
  const int n_ab = input_gate_width(value_heads);
  uint8_t* p = scratch;
  uint16_t* qkv = reinterpret_cast<uint16_t*>(p);
  p += r256(static_cast<uint64_t>(tokens) * channels * 2);
  uint16_t* ab = reinterpret_cast<uint16_t*>(p);
  p += r256(static_cast<uint64_t>(tokens) * n_ab * 2);
  uint16_t* w_ab = reinterpret_cast<uint16_t*>(p);
  p += r256(static_cast<uint64_t>(n_ab) * hidden * 2);
  float* gemm_ws = reinterpret_cast<float*>(p);

  const int groups = channels / 8;
  cudaError_t e = cudaSuccess;
  if (tokens > 0) {
    const size_t wrow = static_cast<size_t>(hidden) * 2;
    e = cudaMemcpyAsync(w_ab, w_a, value_heads * wrow, cudaMemcpyDeviceToDevice, stream);
    if (e != cudaSuccess) return e;
    e = cudaMemcpyAsync(w_ab + static_cast<size_t>(value_heads) * hidden, w_b, value_heads * wrow,
                        cudaMemcpyDeviceToDevice, stream);
    if (e != cudaSuccess) return e;
    if (n_ab > 2 * value_heads) {
      e = cudaMemsetAsync(w_ab + static_cast<size_t>(2 * value_heads) * hidden, 0,
                          (n_ab - 2 * value_heads) * wrow, stream);
      if (e != cudaSuccess) return e;
    }
    e = launch_tail_gemm(x, w_qkv, qkv, gemm_ws, tokens, channels, hidden, err, stream);
    if (e != cudaSuccess) return e;
    e = launch_tail_gemm(x, w_z, z, gemm_ws, tokens, v_dim, hidden, err, stream);
    if (e != cudaSuccess) return e;
    e = launch_tail_gemm(x, w_ab, ab, gemm_ws, tokens, n_ab, hidden, err, stream);
    if (e != cudaSuccess) return e;
    dim3 cgrid((groups + 127) / 128, tab.total_chunks * (kChunk / kConvRun));
    causal_conv_split_kernel<<<cgrid, 128, 0, stream>>>(tab, qkv, conv_w, conv_state, use_state,
                                                        q, k, v, qk_dim, v_dim);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    note_launches();
  }
  // The state of every sequence (an empty one keeps its history, or zeros
  // when the call has no context), after the conv has read the old state.
  dim3 sgrid((groups + 127) / 128, tab.num_seqs);
  conv_state_update_kernel<<<sgrid, 128, 0, stream>>>(tab, qkv, conv_state, use_state, channels);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  note_launches();
  const int64_t n = tokens * value_heads;
  if (n == 0) return cudaSuccess;
  split_gates_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, stream>>>(
      ab, a, b, tokens, value_heads, n_ab);
  e = cudaGetLastError();
  if (e == cudaSuccess) note_launches();
  return e;
}

}  // namespace gdn
