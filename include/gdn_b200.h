/*
 * gdn_b200: B200 (sm_100a) kernels for the Qwen3.8 / Qwen3-Next gated delta
 * net (GDN) layer hot path, behind a plain C ABI.
 *
 * Every entry point takes device pointers, sizes and a cudaStream_t passed as
 * void*, enqueues its kernels on that stream and returns without waiting.
 * The compute entry points allocate no device memory: scratch space is passed
 * in by the caller (query its size with the matching *_workspace_bytes
 * function).  The one exception is gdn_b200_exchange_alloc(), which exists to
 * allocate the IPC-shareable exchange region of the head-parallel tail.
 * Return values are the STATECENTRIC_QWEN38_* status codes of
 * statecentric_qwen38_provider_api_v1.h; gdn_b200_last_error() returns the
 * message of the last failure on the calling thread.
 *
 * Citations name the reference operator each entry point replaces
 * (P = native/src/qwen38_geometry_normalized_gdn_provider.cpp).
 *
 * Tensor layouts (row-major, contiguous):
 *   q, k        bf16 [T, Hk, 128]   raw (not yet L2-normalised)
 *   v, z, o     bf16 [T, Hv, 128]
 *   a, b        bf16 [T, Hv]        gate inputs: g = -exp(A_log)*softplus(a+dt_bias),
 *                                   beta = sigmoid(b)
 *   A_log, dt_bias  f32 [Hv]
 *   gamma       bf16 [128]          output RMSNorm weight (eps 1e-6)
 *   w_out       bf16 [hidden, Hv*128]  (reference input 9: dims {value, hidden},
 *                                   strides {1, value}, P:2405-2406)
 *   state       f32 [S, Hv, 128(v), 128(k)]  recurrent state, row = value
 *                                   index, contiguous along key; updated in place
 *   out         bf16 [T, hidden]    rank-partial when heads are sharded
 *   cu_seqlens  int32 host array [S+1], packed prefix sums of sequence lengths
 * Sequence s owns tokens [cu_seqlens[s], cu_seqlens[s+1]) and state row s.
 * v-head h reads q/k head h / (Hv / Hk).
 */
#ifndef GDN_B200_H_
#define GDN_B200_H_

#include <stdint.h>

#include "statecentric_qwen38_provider_api_v1.h"

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define GDN_B200_API __attribute__((visibility("default")))
#else
#define GDN_B200_API
#endif

#define GDN_B200_HEAD_DIM 128
#define GDN_B200_CHUNK 64
#define GDN_B200_MAX_SEQUENCES 1024

/* Message of the last failed call on this thread ("" when none). */
GDN_B200_API const char* gdn_b200_last_error(void);

/* Number of kernels this library has launched in this process (all devices,
 * all threads; a monotonically increasing count taken at each successful
 * launch).  No counterpart in the reference: it lets a caller check how many
 * device launches a step costs. */
GDN_B200_API uint64_t gdn_b200_kernel_launches(void);

/* Every entry point that takes a workspace keeps a device error word in its
 * first 256 bytes.  Kernels never spin without a time limit: a wait that runs
 * out records an error there and the kernel exits.  This call synchronises
 * `stream` and returns OK, or INTERNAL with the reason. */
GDN_B200_API int32_t gdn_b200_workspace_status(const void* workspace, void* stream);

/* Output tail: out = bf16( bf16(bf16(RMSNorm_head(o)*gamma) * bf16(SiLU(z))) @ w_out^T ).
 * Replaces BatchGdnOutputTail (P:1434-1498; flattened matmul since
 * patches/0001-feat-qwen38-flatten-dual-tail-output-projection.patch:179-184),
 * LaneGdnOutputTailV13 (P:1371-1432) and the single-sequence tail (P:3498-3547):
 * rows = B*T of every sequence, flattened into one GEMM. */
GDN_B200_API uint64_t gdn_b200_output_tail_workspace_bytes(int64_t rows, int32_t value_heads,
                                              int32_t hidden);
GDN_B200_API int32_t gdn_b200_output_tail(const void* o, const void* z, const void* gamma,
                             const void* w_out, void* out, int64_t rows,
                             int32_t value_heads, int32_t hidden, float eps,
                             void* workspace, uint64_t workspace_bytes,
                             void* stream);

/* Output tail that allocates nothing and takes no workspace: for callers that
 * cannot provide device scratch (an operator interface that passes only
 * inputs and outputs, or a serving loop bound to a memory plan frozen at
 * start-up, where cudaMalloc is not allowed).  This entry point has no
 * counterpart in the reference.  Its scratch is a static device array of
 * GDN_B200_NO_ALLOC_SCRATCH_BYTES held by every GPU that loads the library;
 * sizes are limited to rows <= 128, value_heads * 128 <= 4096, hidden <= 2048
 * (larger sizes return INVALID_ARGUMENT).  All calls on a device share the
 * array: calls that overlap on the GPU race and must be serialised.  The
 * first call in each CUDA context (per device, and again after
 * cudaDeviceReset) resolves the array's device address; make it before any
 * stream capture.  Argument errors are reported like every other entry point
 * (status + gdn_b200_last_error()). */
#define GDN_B200_NO_ALLOC_MAX_ROWS 128
#define GDN_B200_NO_ALLOC_MAX_VALUE 4096
#define GDN_B200_NO_ALLOC_MAX_HIDDEN 2048
#define GDN_B200_NO_ALLOC_SCRATCH_BYTES (256ull + 128ull * 4096ull * 2ull + 16ull * 128ull * 2048ull * 4ull)
GDN_B200_API int32_t gdn_b200_output_tail_no_alloc(const void* o, const void* z,
                                                   const void* gamma, const void* w_out,
                                                   void* out, int64_t rows,
                                                   int32_t value_heads, int32_t hidden,
                                                   float eps, void* stream);

/* Device-side status of the last gdn_b200_output_tail_no_alloc() call in the
 * current context: synchronises `stream`, then reads the error word the
 * kernels record in the static scratch (a bounded wait that ran out, a failed
 * TMEM allocation).  Returns OK when nothing was recorded or no call has run
 * in this context, INTERNAL with gdn_b200_last_error() naming the reason
 * otherwise.  It is the no-workspace counterpart of
 * gdn_b200_workspace_status() and allocates nothing either. */
GDN_B200_API int32_t gdn_b200_output_tail_no_alloc_status(void* stream);

/* One decode step for `batch` sequences of one token each: gating, q/k
 * L2-norm, S <- exp(g) S; S += beta k (v - S^T k)^T; o = scale S^T q,
 * scale = 128^-1/2.  Replaces PackedDecodeRecurrentV12 (P:1308-1369) with the
 * gating (P:3310-3339) and q/k RmsNorm (P:3249-3308) fused in.  o_out may be
 * NULL.  When z and gated_out are not NULL the tail prologue
 * bf16(bf16(RMSNorm(o)*gamma)*bf16(SiLU(z))) is fused too and written to
 * gated_out [batch, Hv*128]. */
GDN_B200_API int32_t gdn_b200_decode_step(const void* q, const void* k, const void* v,
                             const void* a, const void* b, const float* A_log,
                             const float* dt_bias, float* state, void* o_out,
                             const void* z, const void* gamma, void* gated_out,
                             int32_t batch, int32_t qk_heads,
                             int32_t value_heads, void* stream);

/* Decode with the state of sequence i at the device address state_rows[i]
 * (a device array of `batch` uint64 addresses, each a 16-byte aligned f32
 * [Hv, 128(v), 128(k)] row): slot binding, so the rows can live anywhere in a
 * state pool.  A CUDA graph captured around this call is rebound to other
 * slots by rewriting state_rows (the DIRECT binding of the reference's
 * qwen38_gdn_graph_binding.h without the exact-address restriction).  The
 * kernel trusts the addresses.  Otherwise as gdn_b200_decode_step. */
GDN_B200_API int32_t gdn_b200_decode_step_rows(const void* q, const void* k, const void* v,
                                               const void* a, const void* b,
                                               const float* A_log, const float* dt_bias,
                                               const uint64_t* state_rows, void* o_out,
                                               const void* z, const void* gamma,
                                               void* gated_out, int32_t batch,
                                               int32_t qk_heads, int32_t value_heads,
                                               void* stream);

/* COPY graph binding (reference qwen38_gdn_graph_binding.h:27-73): gathers
 * (gather != 0: state rows -> packed buffers) or scatters the conv and
 * recurrent rows of `layout` with one cudaMemcpyAsync per row on `stream`,
 * conv row first.  Every row is checked against the layout's arena before
 * any copy is enqueued; a refused binding returns INVALID_ARGUMENT with the
 * reference's reason and issues no copy.  packed_conv / packed_recurrent are
 * device addresses of batch_size rows each. */
GDN_B200_API int32_t gdn_b200_copy_graph_rows(
    const statecentric_qwen38_gdn_layout_workspace_v1* layout, uint64_t batch_size,
    uint64_t conv_bytes, uint64_t recurrent_bytes, uint64_t packed_conv,
    uint64_t packed_recurrent, int32_t gather, void* stream);

/* Chunked (C = 64) gated delta rule over packed variable-length sequences.
 * Replaces ChunkGdn (P:1641-1838) and the token-serial run_sequence
 * (P:3387-3469): every sequence length, any number of chunks, one call. */
GDN_B200_API uint64_t gdn_b200_chunk_prefill_workspace_bytes(const int32_t* cu_seqlens,
                                                             int32_t num_seqs,
                                                             int32_t qk_heads,
                                                             int32_t value_heads);
GDN_B200_API int32_t gdn_b200_chunk_prefill(const void* q, const void* k, const void* v,
                               const void* a, const void* b,
                               const float* A_log, const float* dt_bias,
                               float* state, void* o_out,
                               const int32_t* cu_seqlens, int32_t num_seqs,
                               int32_t qk_heads, int32_t value_heads,
                               void* workspace, uint64_t workspace_bytes,
                               void* stream);

/* Whole post-projection layer: core (decode kernel when every sequence has
 * one token, chunk kernels otherwise) then the flattened output tail.
 * Replaces the Submit path after the projections (P:3249-3547). */
GDN_B200_API uint64_t gdn_b200_layer_forward_workspace_bytes(const int32_t* cu_seqlens,
                                                             int32_t num_seqs,
                                                             int32_t qk_heads,
                                                             int32_t value_heads,
                                                             int32_t hidden);
GDN_B200_API int32_t gdn_b200_layer_forward(const void* q, const void* k, const void* v,
                               const void* a, const void* b, const void* z,
                               const float* A_log, const float* dt_bias,
                               const void* gamma, const void* w_out,
                               float* state, void* out,
                               const int32_t* cu_seqlens, int32_t num_seqs,
                               int32_t qk_heads, int32_t value_heads,
                               int32_t hidden, void* workspace,
                               uint64_t workspace_bytes, void* stream);

/* ----------------------------------------------------------------------
 * Input side of the layer: x -> q, k, v, z, a, b.  Replaces the reference's
 * projections (four aclnnMatmul calls, P:3101-3130), aclnnCausalConv1d with
 * the conv-state update (P:3132-3179) and the Q/K/V split (P:3186-3247).
 *   x        bf16 [T, hidden]   the normalised layer input (reference input 0)
 *   w_qkv    bf16 [(2 Hk + Hv) 128, hidden], w_z bf16 [Hv 128, hidden],
 *   w_a, w_b bf16 [Hv, hidden]  (reference inputs 1-4: dims {hidden, N},
 *                               strides {1, hidden})
 *   conv_w   bf16 [4, (2 Hk + Hv) 128]   (input 5: tap k multiplies x[t-3+k])
 *   conv_state bf16 [S, 3, (2 Hk + Hv) 128]  (region gdn.conv: the last three
 *            projected rows of each sequence), updated in place; with
 *            use_conv_state = 0 the history is taken as zero (a submission
 *            without context) and the state is still written.
 * q, k, v are the conv output (SiLU applied) split at Hk 128 and 2 Hk 128;
 * z, a, b are the projections.  L2-norm and gating follow in the layer. */
GDN_B200_API uint64_t gdn_b200_input_side_workspace_bytes(const int32_t* cu_seqlens,
                                                          int32_t num_seqs, int32_t qk_heads,
                                                          int32_t value_heads, int32_t hidden);
GDN_B200_API int32_t gdn_b200_input_side(const void* x, const void* w_qkv, const void* w_z,
                                         const void* w_a, const void* w_b, const void* conv_w,
                                         void* conv_state, const int32_t* cu_seqlens,
                                         int32_t num_seqs, int32_t qk_heads,
                                         int32_t value_heads, int32_t hidden,
                                         int32_t use_conv_state, void* q, void* k, void* v,
                                         void* z, void* a, void* b, void* workspace,
                                         uint64_t workspace_bytes, void* stream);

/* The whole layer from x: input side, then gdn_b200_layer_forward's path
 * (the reference's Submit with GDN_FORWARD_V1 on x, P:3083-3547). */
GDN_B200_API uint64_t gdn_b200_layer_forward_x_workspace_bytes(const int32_t* cu_seqlens,
                                                               int32_t num_seqs,
                                                               int32_t qk_heads,
                                                               int32_t value_heads,
                                                               int32_t hidden);
GDN_B200_API int32_t gdn_b200_layer_forward_x(const void* x, const void* w_qkv, const void* w_z,
                                              const void* w_a, const void* w_b,
                                              const void* conv_w, void* conv_state,
                                              const float* A_log, const float* dt_bias,
                                              const void* gamma, const void* w_out,
                                              float* state, void* out,
                                              const int32_t* cu_seqlens, int32_t num_seqs,
                                              int32_t qk_heads, int32_t value_heads,
                                              int32_t hidden, int32_t use_conv_state,
                                              void* workspace, uint64_t workspace_bytes,
                                              void* stream);

/* ----------------------------------------------------------------------
 * Head-parallel output tail with the rank reduction fused in.
 *
 * With the value heads split over world_size GPUs of one node (rank r holds
 * value_heads = Hv / world_size heads, the matching o and z columns and the
 * w_out columns [r * value_heads * 128, (r + 1) * value_heads * 128)), each
 * rank's tail yields a partial [rows, hidden].  The reference returns that
 * rank-partial (P:3541-3547) and leaves the sum to its engine; this entry
 * point (no counterpart in the reference) sums it inside the tail GEMM
 * kernel over NVLink peer memory, tile by tile, and leaves the full output
 * on every rank:
 *   out = bf16( sum over ranks, in rank order, in f32, of bf16(partial) ),
 * the same bits on every rank (a bf16 all-reduce of the rank-partial outputs
 * with f32 accumulation).
 *
 * Each rank owns an exchange region of gdn_b200_tail_exchange_bytes bytes
 * (gdn_b200_exchange_alloc: zero-filled device memory of the current
 * device).  It holds the rank's output at offset 0 ([max_rows, hidden] bf16;
 * the first rows * hidden elements are valid after a call) and the staging
 * space and flags of the exchange.  Ranks map one another's regions with
 * gdn_b200_exchange_export / gdn_b200_exchange_open (CUDA IPC: the handle is
 * GDN_B200_EXCHANGE_HANDLE_BYTES plain bytes, passed between the processes by
 * any means) and list them, by rank, in a gdn_b200_tail_group_v1.
 *
 * Every rank calls gdn_b200_output_tail_allreduce with the same rows, hidden,
 * max_rows and epoch; epochs start at 1 and grow by one per call.  The
 * kernels of the ranks wait for one another, bounded: if a rank does not take
 * part, the others end with a device error (gdn_b200_workspace_status) after
 * 2 s.  After a failed call the regions must be freed and allocated again.
 */
#define GDN_B200_MAX_RANKS 8
#define GDN_B200_EXCHANGE_HANDLE_BYTES 64

typedef struct gdn_b200_tail_group_v1 {
  int32_t rank;
  int32_t world_size;                /* 1, 2, 4 or 8 */
  int64_t max_rows;                  /* rows the regions were sized for */
  int32_t hidden;                    /* a multiple of 256 */
  int32_t reserved;                  /* must be 0 */
  void* region[GDN_B200_MAX_RANKS];  /* rank i's exchange region as mapped here */
} gdn_b200_tail_group_v1;

GDN_B200_API uint64_t gdn_b200_tail_exchange_bytes(int64_t max_rows, int32_t hidden,
                                                   int32_t world_size);
GDN_B200_API int32_t gdn_b200_exchange_alloc(uint64_t bytes, void** region);
GDN_B200_API int32_t gdn_b200_exchange_free(void* region);
GDN_B200_API int32_t gdn_b200_exchange_export(const void* region, void* handle);
GDN_B200_API int32_t gdn_b200_exchange_open(const void* handle, void** region);
GDN_B200_API int32_t gdn_b200_exchange_close(void* region);
/* Rank sum of the head-parallel layer's rank-partial outputs over the copy
 * engines: a reduce-scatter.  No counterpart in the reference, which returns
 * the rank-partial (P:3541-3547) and leaves the sum to its engine; this is
 * the B200 form of that engine step.  Every rank ends with its row shard
 *   shard_r = bf16( sum over ranks q, in rank order, in f32, of
 *                   partial_q[rows r*rows/W .. (r+1)*rows/W) )
 * (W = world_size); the rows move as cudaMemcpyAsync peer copies, i.e. on the
 * copy engines over NVLink, so no SM takes part in the transfer and it
 * overlaps the next layer step.  A consumer that needs every row on every
 * rank gathers the shards afterwards.
 *
 * Each rank owns a region of gdn_b200_rank_sum_bytes bytes
 * (gdn_b200_exchange_alloc: zero-filled), exported and opened like the fused
 * tail's regions and listed by rank in a gdn_b200_tail_group_v1 (max_rows a
 * multiple of world_size, hidden a multiple of 8).  Per epoch (1, 2, 3 ...,
 * the same on every rank):
 *   gdn_b200_rank_sum_acquire(group, e, err, stream)   before the layer
 *   the layer writes its [rows, hidden] bf16 rank-partial to
 *       gdn_b200_rank_sum_part(group, e) on `stream`
 *   gdn_b200_rank_sum(group, e, rows, shard_out, err, stream, comm_stream)
 * Acquire waits (on `stream`) until every rank has copied out this rank's
 * part of epoch e - 2, whose buffer the layer of epoch e reuses.  The sum
 * publishes the part (on `stream`), then on `comm_stream` waits for every
 * rank's part of epoch e, copies this rank's rows of each, tells every rank
 * they are out, and writes shard_out [rows / world_size, hidden] bf16.
 * Waits are bounded (2 s): a rank that does not take part leaves
 * kErrWaitTimeout in *err (a device word, read with
 * gdn_b200_workspace_status). */
GDN_B200_API uint64_t gdn_b200_rank_sum_bytes(int64_t max_rows, int32_t hidden,
                                              int32_t world_size);
GDN_B200_API void* gdn_b200_rank_sum_part(const gdn_b200_tail_group_v1* group, uint32_t epoch);
GDN_B200_API int32_t gdn_b200_rank_sum_acquire(const gdn_b200_tail_group_v1* group,
                                               uint32_t epoch, uint32_t* err, void* stream);
GDN_B200_API int32_t gdn_b200_rank_sum(const gdn_b200_tail_group_v1* group, uint32_t epoch,
                                       int64_t rows, void* shard_out, uint32_t* err,
                                       void* stream, void* comm_stream);

GDN_B200_API uint64_t gdn_b200_output_tail_allreduce_workspace_bytes(int64_t rows,
                                                                     int32_t value_heads);
GDN_B200_API int32_t gdn_b200_output_tail_allreduce(const void* o, const void* z,
                                                    const void* gamma, const void* w_out,
                                                    int64_t rows, int32_t value_heads,
                                                    int32_t hidden, float eps,
                                                    const gdn_b200_tail_group_v1* group,
                                                    uint32_t epoch, void* workspace,
                                                    uint64_t workspace_bytes, void* stream);

/* Seeded synthetic inputs (host side, used by benchmarks and tests).
 * Element i of tensor `tensor_id` under `seed` is a pure function of
 * (seed, tensor_id, i): SplitMix64 counters, Box-Muller for normals.
 * distribution: 0 = normal(p0 = mean, p1 = std), 1 = uniform[p0, p1),
 *               2 = log(uniform(p0, p1)).
 * out_dtype: 1 = bf16 (round to nearest even), 2 = f32. */
GDN_B200_API int32_t gdn_b200_fill_synthetic(uint64_t seed, uint64_t tensor_id,
                                uint64_t count, int32_t distribution, float p0,
                                float p1, int32_t out_dtype, void* host_out);

#ifdef __cplusplus
}
#endif

#endif /* GDN_B200_H_ */
