// Internal launch interface between the C-ABI layer and the kernel files.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace gdn {

constexpr int kMaxSeqsInternal = 1024;

struct ChunkTable {
  int32_t num_seqs;
  int32_t total_chunks;
  int32_t cu[kMaxSeqsInternal + 1];
  int32_t chunk_start[kMaxSeqsInternal + 1];
};

bool build_chunk_table(const int32_t* cu_seqlens, int num_seqs, ChunkTable* tab);
uint64_t chunk_workspace_bytes(const ChunkTable& tab, int qk_heads, int value_heads);
cudaError_t launch_chunk_prefill(const ChunkTable& tab, const uint16_t* q, const uint16_t* k,
                                 const uint16_t* v, const uint16_t* a, const uint16_t* b,
                                 const float* A_log, const float* dt_bias, float* state,
                                 uint16_t* o_out, int qk_heads, int value_heads,
                                 uint8_t* scratch, uint32_t* err, cudaStream_t stream);

cudaError_t launch_decode(const uint16_t* q, const uint16_t* k, const uint16_t* v,
                          const uint16_t* a, const uint16_t* b, const float* A_log,
                          const float* dt_bias, float* state, uint16_t* o_out,
                          const uint16_t* z, const uint16_t* gamma, uint16_t* gated_out,
                          int batch, int qk_heads, int value_heads, cudaStream_t stream);

uint64_t tail_gemm_workspace_bytes(int64_t M, int N, int K);
cudaError_t launch_tail_prologue(const uint16_t* o, const uint16_t* z, const uint16_t* gamma,
                                 uint16_t* gated, int64_t rows, int value_heads, float eps,
                                 cudaStream_t stream);
cudaError_t launch_tail_gemm(const uint16_t* a, const uint16_t* w, uint16_t* out, float* ws,
                             int64_t M, int N, int K, uint32_t* err, cudaStream_t stream);

}  // namespace gdn
