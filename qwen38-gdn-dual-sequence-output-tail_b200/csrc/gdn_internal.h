// Internal launch interface between the C-ABI layer and the kernel files.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

namespace gdn {

// Status reporting shared by every C-ABI entry point: api_fail records the
// message that gdn_b200_last_error() returns on this thread, api_ok clears it.
int32_t api_fail(int32_t status, const std::string& message);
int32_t api_ok();
// Synchronises `stream`, then reads the device error word at `word_address`
// and turns it into a status (OK, or INTERNAL with the reason).
int32_t read_error_word(const void* word_address, cudaStream_t stream);
// Counts kernel launches made by this library (gdn_b200_kernel_launches()).
void note_launches(int n = 1);

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
                                 uint8_t* scratch, uint32_t* err, cudaStream_t stream,
                                 bool clear_err = false);

cudaError_t launch_decode(const uint16_t* q, const uint16_t* k, const uint16_t* v,
                          const uint16_t* a, const uint16_t* b, const float* A_log,
                          const float* dt_bias, float* state, uint16_t* o_out,
                          const uint16_t* z, const uint16_t* gamma, uint16_t* gated_out,
                          int batch, int qk_heads, int value_heads, cudaStream_t stream,
                          const uint64_t* state_rows = nullptr, uint32_t* err = nullptr,
                          const void* l2_prefetch = nullptr, uint64_t l2_prefetch_bytes = 0,
                          bool clear_err = false);
// l2_prefetch: a buffer (16-byte aligned) the next kernel on the stream reads,
// brought into L2 by the decode CTAs once their last state block is loading.

// Streaming multiprocessors of the current device.
int sm_count();

uint64_t tail_gemm_workspace_bytes(int64_t M, int N, int K);
cudaError_t launch_tail_prologue(const uint16_t* o, const uint16_t* z, const uint16_t* gamma,
                                 uint16_t* gated, int64_t rows, int value_heads, float eps,
                                 cudaStream_t stream,
                                 uint32_t* clear_err = nullptr);
// overlap_previous: the previous launch on `stream` is one of this
// library's kernels (tail prologue or decode) that writes `a` but not `w`;
// for M <= 128 the GEMM then starts while it runs and streams W early.
cudaError_t launch_tail_gemm(const uint16_t* a, const uint16_t* w, uint16_t* out, float* ws,
                             int64_t M, int N, int K, uint32_t* err, cudaStream_t stream,
                             bool overlap_previous = false);

// Input side: projections, causal conv + SiLU, q/k/v split, conv-state
// update (gdn_input.cu).  a, b come from one GEMM over [w_a; w_b] padded to
// input_gate_width(value_heads) rows.
int input_gate_width(int value_heads);
uint64_t input_side_scratch_bytes(int64_t tokens, int qk_heads, int value_heads, int hidden);
cudaError_t launch_input_side(const ChunkTable& tab, const uint16_t* x, const uint16_t* w_qkv,
                              const uint16_t* w_z, const uint16_t* w_a, const uint16_t* w_b,
                              const uint16_t* conv_w, uint16_t* conv_state, int use_state,
                              uint16_t* q, uint16_t* k, uint16_t* v, uint16_t* z, uint16_t* a,
                              uint16_t* b, int qk_heads, int value_heads, int hidden,
                              uint8_t* scratch, uint32_t* err, cudaStream_t stream);

// Head-parallel tail with the rank reduction fused in (gdn_tail_allreduce.cu).
constexpr int kTailMaxRanks = 8;
constexpr int kTailArGrid = 148;  // CTAs per rank (same on every rank)

// Every rank's exchange region as mapped in this process.
struct TailPeerRegions {
  uint8_t* region[kTailMaxRanks];
};

// Exchange region of one rank, sized for up to max_rows rows: the rank's
// output [max_rows, hidden] bf16 at offset 0, then the staging area for the
// partial tiles other ranks send it ([slots * world * 128, 256] bf16), the
// per-(tile, source rank, warp) flags and the per-(CTA, source rank) done
// flags (u32, zero at allocation).
struct TailExchangeLayout {
  uint64_t out_bytes, staging_off, staging_rows, flags_off, done_off, total;
};
bool tail_exchange_layout(int64_t max_rows, int hidden, int world, TailExchangeLayout* out);
cudaError_t launch_tail_gemm_allreduce(const uint16_t* a, const uint16_t* w, int64_t M, int N,
                                       int K, const TailPeerRegions& peers, int rank, int world,
                                       const TailExchangeLayout& layout, uint32_t epoch,
                                       uint32_t* err, cudaStream_t stream);

}  // namespace gdn
