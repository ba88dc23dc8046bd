// C-ABI entry points of include/gdn_b200.h: argument validation, workspace
// carving and kernel launches.  Host code only; kernels live in
// gdn_decode.cu, gdn_tail.cu and gdn_chunk.cu.
#include <atomic>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <string>

#include "gdn_b200.h"
#include "gdn_common.cuh"
#include "gdn_graph_binding.h"
#include "gdn_internal.h"

namespace {

thread_local std::string g_last_error;

int32_t fail(int32_t status, const std::string& message) {
  g_last_error = message;
  return status;
}

int32_t ok() {
  g_last_error.clear();
  return STATECENTRIC_QWEN38_OK;
}

int32_t cuda_status(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return ok();
  return fail(STATECENTRIC_QWEN38_INTERNAL,
              std::string(what) + ": " + cudaGetErrorString(e));
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

constexpr uint64_t kErrBytes = 256;

uint64_t round256(uint64_t x) { return (x + 255u) & ~static_cast<uint64_t>(255u); }

bool heads_ok(int32_t qk_heads, int32_t value_heads) {
  return qk_heads > 0 && value_heads > 0 && value_heads % qk_heads == 0 && value_heads <= 4096;
}

// Validates host cu_seqlens; fills the chunk table.
int32_t check_seqlens(const int32_t* cu, int32_t num_seqs, gdn::ChunkTable* tab) {
  if (cu == nullptr) return fail(STATECENTRIC_QWEN38_INVALID_ARGUMENT, "cu_seqlens is null");
  if (num_seqs < 1 || num_seqs > GDN_B200_MAX_SEQUENCES)
    return fail(STATECENTRIC_QWEN38_INVALID_ARGUMENT,
                "num_seqs must be in [1, " + std::to_string(GDN_B200_MAX_SEQUENCES) + "]");
  if (cu[0] != 0) return fail(STATECENTRIC_QWEN38_INVALID_ARGUMENT, "cu_seqlens[0] must be 0");
  for (int32_t s = 0; s < num_seqs; ++s) {
    if (cu[s + 1] < cu[s])
      return fail(STATECENTRIC_QWEN38_INVALID_ARGUMENT, "cu_seqlens must be non-decreasing");
  }
  if (!gdn::build_chunk_table(cu, num_seqs, tab))
    return fail(STATECENTRIC_QWEN38_INVALID_ARGUMENT, "invalid cu_seqlens");
  return ok();
}

}  // namespace

namespace gdn {

int32_t api_fail(int32_t status, const std::string& message) { return fail(status, message); }

int32_t api_ok() { return ok(); }

namespace {
std::atomic<uint64_t> g_kernel_launches{0};
}  // namespace

void note_launches(int n) { g_kernel_launches.fetch_add(static_cast<uint64_t>(n), std::memory_order_relaxed); }

int32_t read_error_word(const void* word_address, cudaStream_t stream) {
  cudaError_t e = cudaStreamSynchronize(stream);
  if (e != cudaSuccess) return cuda_status(e, "cudaStreamSynchronize");
  uint32_t word = 0;
  e = cudaMemcpy(&word, word_address, sizeof(word), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_status(e, "cudaMemcpy(error word)");
  if (word == kErrNone) return ok();
  const char* what = word == kErrWaitTimeout  ? "a kernel wait ran out of time"
                     : word == kErrTmemAlloc  ? "TMEM allocation failed"
                     : word == kErrMisaligned ? "a state row address is not 16-byte aligned"
                                              : "kernel reported a geometry error";
  return fail(STATECENTRIC_QWEN38_INTERNAL, std::string("device error: ") + what);
}

}  // namespace gdn

extern "C" {

const char* gdn_b200_last_error(void) { return g_last_error.c_str(); }

uint64_t gdn_b200_kernel_launches(void) {
  return gdn::g_kernel_launches.load(std::memory_order_relaxed);
}

int32_t gdn_b200_workspace_status(const void* workspace, void* stream) {
  if (workspace == nullptr) return fail(STATECENTRIC_QWEN38_INVALID_ARGUMENT, "workspace is null");
  return gdn::read_error_word(workspace, static_cast<cudaStream_t>(stream));
}

// ------------------------------------------------------------- tail ----

uint64_t gdn_b200_output_tail_workspace_bytes(int64_t rows, int32_t value_heads,
                                              int32_t hidden) {
  if (rows < 0 || value_heads <= 0 || hidden <= 0) return 0;
  const int64_t K = static_cast<int64_t>(value_heads) * GDN_B200_HEAD_DIM;
  return kErrBytes + round256(static_cast<uint64_t>(rows) * K * 2) +
         round256(gdn::tail_gemm_workspace_bytes(rows, hidden, static_cast<int>(K)));
}

int32_t gdn_b200_output_tail(const void* o, const void* z, const void* gamma, const void* w_out,
                             void* out, int64_t rows, int32_t value_heads, int32_t hidden,
                             float eps, void* workspace, uint64_t workspace_bytes,
                             void* stream) {
  if (rows < 0 || value_heads <= 0 || hidden <= 0)
    return fail(STATECENTRIC_QWEN38_INVALID_ARGUMENT, "rows, value_heads and hidden must be positive");
  if (hidden % 128 != 0)
    return fail(STATECENTRIC_QWEN38_INVALID_ARGUMENT, "hidden must be a multiple of 128");
  if (rows > (int64_t{1} << 31) / 2)
    return fail(STATECENTRIC_QWEN38_INVALID_ARGUMENT, "too many rows");
  if (!(eps > 0.0f) || !std::isfinite(eps))
    return fail(STATECENTRIC_QWEN38_INVALID_ARGUMENT, "eps must be positive");
  if (o == nullptr || z == nullptr || gamma == nullptr || w_out == nullptr || out == nullptr ||
      workspace == nullptr)
    return fail(STATECENTRIC_QWEN38_INVALID_ARGUMENT, "null pointer argument");
  if (!aligned16(o) || !aligned16(z) || !aligned16(w_out) || !aligned16(out) ||
      !aligned16(workspace) || !aligned16(gamma))
    return fail(STATECENTRIC_QWEN38_INVALID_ARGUMENT, "tensors must be 16-byte aligned");
  const uint64_t need = gdn_b200_output_tail_workspace_bytes(rows, value_heads, hidden);
  if (workspace_bytes < need)
    return fail(STATECENTRIC_QWEN38_INVALID_ARGUMENT,
                "workspace too small: need " + std::to_string(need) + " bytes");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  uint32_t* err = reinterpret_cast<uint32_t*>(ws);
  const int K = value_heads * GDN_B200_HEAD_DIM;
  uint16_t* gated = reinterpret_cast<uint16_t*>(ws + kErrBytes);
  float* gemm_ws = reinterpret_cast<float*>(ws + kErrBytes + round256(static_cast<uint64_t>(rows) * K * 2));
  cudaError_t e;
  if (rows == 0) {
    e = cudaMemsetAsync(err, 0, sizeof(uint32_t), s);
    return e == cudaSuccess ? ok() : cuda_status(e, "cudaMemsetAsync");
  }
  // The prologue clears the error word (no separate memset on the stream).
  e = gdn::launch_tail_prologue(static_cast<const uint16_t*>(o), static_cast<const uint16_t*>(z),
                                static_cast<const uint16_t*>(gamma), gated, rows, value_heads,
                                eps, s, err);
  if (e != cudaSuccess) return cuda_status(e, "tail prologue launch");
  e = gdn::launch_tail_gemm(gated, static_cast<const uint16_t*>(w_out),
                            static_cast<uint16_t*>(out), gemm_ws, rows, hidden, K, err, s,
                            /*overlap_previous=*/true);
  return cuda_status(e, "tail GEMM launch");
}

// ------------------------------------------- head-parallel fused tail ----

static_assert(GDN_B200_MAX_RANKS == gdn::kTailMaxRanks, "rank limit");
static_assert(GDN_B200_EXCHANGE_HANDLE_BYTES == sizeof(cudaIpcMemHandle_t), "IPC handle size");

uint64_t gdn_b200_tail_exchange_bytes(int64_t max_rows, int32_t hidden, int32_t world_size) {
  gdn::TailExchangeLayout L;
  if (!gdn::tail_exchange_layout(max_rows, hidden, world_size, &L)) return 0;
  return L.total;
}

int32_t gdn_b200_exchange_alloc(uint64_t bytes, void** region) {
  if (region == nullptr) return fail(STATECENTRIC_QWEN38_INVALID_ARGUMENT, "region is null");
  *region = nullptr;
  if (bytes == 0) return fail(STATECENTRIC_QWEN38_INVALID_ARGUMENT, "bytes must be positive");
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) return cuda_status(e, "cudaMalloc(exchange region)");
  e = cudaMemset(p, 0, bytes);
  if (e != cudaSuccess) {
    cudaFree(p);
    return cuda_status(e, "cudaMemset(exchange region)");
  }
  *region = p;
  return ok();
}

int32_t gdn_b200_exchange_free(void* region) {
  if (region == nullptr) return ok();
  return cuda_status(cudaFree(region), "cudaFree(exchange region)");
}

int32_t gdn_b200_exchange_export(const void* region, void* handle) {
  if (region == nullptr || handle == nullptr)
    return fail(STATECENTRIC_QWEN38_INVALID_ARGUMENT, "null pointer argument");
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, const_cast<void*>(region));
  if (e != cudaSuccess) return cuda_status(e, "cudaIpcGetMemHandle");
  std::memcpy(handle, &h, sizeof(h));
  return ok();
}

int32_t gdn_b200_exchange_open(const void* handle, void** region) {
  if (handle == nullptr || region == nullptr)
    return fail(STATECENTRIC_QWEN38_INVALID_ARGUMENT, "null pointer argument");
  *region = nullptr;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  void* p = nullptr;
  const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return cuda_status(e, "cudaIpcOpenMemHandle");
  *region = p;
  return ok();
}

int32_t gdn_b200_exchange_close(void* region) {
  if (region == nullptr) return ok();
  return cuda_status(cudaIpcCloseMemHandle(region), "cudaIpcCloseMemHandle");
}

uint64_t gdn_b200_output_tail_allreduce_workspace_bytes(int64_t rows, int32_t value_heads) {
  if (rows < 0 || value_heads <= 0) return 0;
  return kErrBytes + round256(static_cast<uint64_t>(rows) * value_heads * GDN_B200_HEAD_DIM * 2);
}

int32_t gdn_b200_output_tail_allreduce(const void* o, const void* z, const void* gamma,
                                       const void* w_out, int64_t rows, int32_t value_heads,
                                       int32_t hidden, float eps,
                                       const gdn_b200_tail_group_v1* group, uint32_t epoch,
                                       void* workspace, uint64_t workspace_bytes,
                                       void* stream) {
  if (rows < 0 || value_heads <= 0 || hidden <= 0)
    return fail(STATECENTRIC_QWEN38_INVALID_ARGUMENT, "rows, value_heads and hidden must be positive");
  if (hidden % 256 != 0)
    return fail(STATECENTRIC_QWEN38_INVALID_ARGUMENT, "hidden must be a multiple of 256");
  if (rows > (int64_t{1} << 31) / 2)
    return fail(STATECENTRIC_QWEN38_INVALID_ARGUMENT, "too many rows");
  if (!(eps > 0.0f) || !std::isfinite(eps))
    return fail(STATECENTRIC_QWEN38_INVALID_ARGUMENT, "eps must be positive");
  if (o == nullptr || z == nullptr || gamma == nullptr || w_out == nullptr ||
      workspace == nullptr || group == nullptr)
    return fail(STATECENTRIC_QWEN38_INVALID_ARGUMENT, "null pointer argument");
  if (!aligned16(o) || !aligned16(z) || !aligned16(w_out) || !aligned16(workspace) ||
      !aligned16(gamma))
    return fail(STATECENTRIC_QWEN38_INVALID_ARGUMENT, "tensors must be 16-byte aligned");
  const int world = group->world_size;
  if (world != 1 && world != 2 && world != 4 && world != 8)
    return fail(STATECENTRIC_QWEN38_INVALID_ARGUMENT, "group world_size must be 1, 2, 4 or 8");
  if (group->rank < 0 || group->rank >= world)
    return fail(STATECENTRIC_QWEN38_INVALID_ARGUMENT, "group rank out of range");
  if (group->reserved != 0)
    return fail(STATECENTRIC_QWEN38_INVALID_ARGUMENT, "group reserved field must be 0");
  if (group->hidden != hidden)
    return fail(STATECENTRIC_QWEN38_INVALID_ARGUMENT, "hidden differs from the group's");
  if (rows > group->max_rows)
    return fail(STATECENTRIC_QWEN38_INVALID_ARGUMENT, "rows exceed the group's max_rows");
  gdn::TailExchangeLayout layout;
  if (!gdn::tail_exchange_layout(group->max_rows, hidden, world, &layout))
    return fail(STATECENTRIC_QWEN38_INVALID_ARGUMENT, "invalid group geometry");
  gdn::TailPeerRegions peers{};
  for (int i = 0; i < world; ++i) {
    if (group->region[i] == nullptr)
      return fail(STATECENTRIC_QWEN38_INVALID_ARGUMENT, "group region is null");
    if ((reinterpret_cast<uintptr_t>(group->region[i]) & 255u) != 0)
      return fail(STATECENTRIC_QWEN38_INVALID_ARGUMENT, "group regions must be 256-byte aligned");
    peers.region[i] = static_cast<uint8_t*>(group->region[i]);
  }
  if (epoch == 0) return fail(STATECENTRIC_QWEN38_INVALID_ARGUMENT, "epoch must start at 1");
  const uint64_t need = gdn_b200_output_tail_allreduce_workspace_bytes(rows, value_heads);
  if (workspace_bytes < need)
    return fail(STATECENTRIC_QWEN38_INVALID_ARGUMENT,
                "workspace too small: need " + std::to_string(need) + " bytes");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  uint32_t* err = reinterpret_cast<uint32_t*>(ws);
  uint16_t* gated = reinterpret_cast<uint16_t*>(ws + kErrBytes);
  const int K = value_heads * GDN_B200_HEAD_DIM;
  cudaError_t e = cudaMemsetAsync(err, 0, sizeof(uint32_t), s);
  if (e != cudaSuccess) return cuda_status(e, "cudaMemsetAsync");
  if (rows == 0) return ok();
  e = gdn::launch_tail_prologue(static_cast<const uint16_t*>(o), static_cast<const uint16_t*>(z),
                                static_cast<const uint16_t*>(gamma), gated, rows, value_heads,
                                eps, s);
  if (e != cudaSuccess) return cuda_status(e, "tail prologue launch");
  e = gdn::launch_tail_gemm_allreduce(gated, static_cast<const uint16_t*>(w_out), rows, hidden, K,
                                      peers, group->rank, world, layout, epoch, err, s);
  return cuda_status(e, "fused tail launch");
}

// ----------------------------------------------------------- decode ----

// Decode on validated arguments: the state is either contiguous (`state`)
// or addressed per sequence through the device table `state_rows`.
static int32_t decode_impl(const void* q, const void* k, const void* v, const void* a,
                           const void* b, const float* A_log, const float* dt_bias, float* state,
                           const uint64_t* state_rows, void* o_out, const void* z,
                           const void* gamma, void* gated_out, int32_t batch, int32_t qk_heads,
                           int32_t value_heads, void* stream) {
  if (batch < 0 || batch > 65535)
    return fail(STATECENTRIC_QWEN38_INVALID_ARGUMENT, "batch must be in [0, 65535]");
  if (!heads_ok(qk_heads, value_heads))
    return fail(STATECENTRIC_QWEN38_INVALID_ARGUMENT,
                "value_heads must be a positive multiple of qk_heads");
  if (batch == 0) return ok();
  if (q == nullptr || k == nullptr || v == nullptr || a == nullptr || b == nullptr ||
      A_log == nullptr || dt_bias == nullptr || (state == nullptr && state_rows == nullptr))
    return fail(STATECENTRIC_QWEN38_INVALID_ARGUMENT, "null pointer argument");
  if ((gated_out != nullptr) && (z == nullptr || gamma == nullptr))
    return fail(STATECENTRIC_QWEN38_INVALID_ARGUMENT, "gated_out needs z and gamma");
  if ((state && !aligned16(state)) || (reinterpret_cast<uintptr_t>(state_rows) & 7u) ||
      (reinterpret_cast<uintptr_t>(q) & 7u) || (reinterpret_cast<uintptr_t>(k) & 7u) ||
      (reinterpret_cast<uintptr_t>(v) & 7u) || (o_out && (reinterpret_cast<uintptr_t>(o_out) & 7u)) ||
      (gated_out && ((reinterpret_cast<uintptr_t>(gated_out) & 7u) || (reinterpret_cast<uintptr_t>(z) & 7u) ||
                     (reinterpret_cast<uintptr_t>(gamma) & 7u))))
    return fail(STATECENTRIC_QWEN38_INVALID_ARGUMENT, "misaligned tensor");
  cudaError_t e = gdn::launch_decode(
      static_cast<const uint16_t*>(q), static_cast<const uint16_t*>(k),
      static_cast<const uint16_t*>(v), static_cast<const uint16_t*>(a),
      static_cast<const uint16_t*>(b), A_log, dt_bias, state, static_cast<uint16_t*>(o_out),
      static_cast<const uint16_t*>(z), static_cast<const uint16_t*>(gamma),
      static_cast<uint16_t*>(gated_out), batch, qk_heads, value_heads,
      static_cast<cudaStream_t>(stream), state_rows);
  return cuda_status(e, "decode launch");
}

int32_t gdn_b200_decode_step(const void* q, const void* k, const void* v, const void* a,
                             const void* b, const float* A_log, const float* dt_bias,
                             float* state, void* o_out, const void* z, const void* gamma,
                             void* gated_out, int32_t batch, int32_t qk_heads,
                             int32_t value_heads, void* stream) {
  if (batch > 0 && state == nullptr)
    return fail(STATECENTRIC_QWEN38_INVALID_ARGUMENT, "null pointer argument");
  return decode_impl(q, k, v, a, b, A_log, dt_bias, state, nullptr, o_out, z, gamma, gated_out,
                     batch, qk_heads, value_heads, stream);
}

int32_t gdn_b200_decode_step_rows(const void* q, const void* k, const void* v, const void* a,
                                  const void* b, const float* A_log, const float* dt_bias,
                                  const uint64_t* state_rows, void* o_out, const void* z,
                                  const void* gamma, void* gated_out, int32_t batch,
                                  int32_t qk_heads, int32_t value_heads, void* stream) {
  if (batch > 0 && state_rows == nullptr)
    return fail(STATECENTRIC_QWEN38_INVALID_ARGUMENT, "null pointer argument");
  return decode_impl(q, k, v, a, b, A_log, dt_bias, nullptr, state_rows, o_out, z, gamma,
                     gated_out, batch, qk_heads, value_heads, stream);
}

// ------------------------------------------------------------ chunk ----

uint64_t gdn_b200_chunk_prefill_workspace_bytes(const int32_t* cu_seqlens, int32_t num_seqs,
                                                int32_t qk_heads, int32_t value_heads) {
  gdn::ChunkTable tab;
  if (!heads_ok(qk_heads, value_heads) ||
      check_seqlens(cu_seqlens, num_seqs, &tab) != STATECENTRIC_QWEN38_OK)
    return 0;
  return kErrBytes + round256(gdn::chunk_workspace_bytes(tab, qk_heads, value_heads));
}

static int32_t chunk_prefill_impl(const gdn::ChunkTable& tab, const void* q, const void* k,
                                  const void* v, const void* a, const void* b,
                                  const float* A_log, const float* dt_bias, float* state,
                                  void* o_out, int32_t qk_heads, int32_t value_heads,
                                  uint8_t* scratch, uint32_t* err, cudaStream_t s,
                                  bool clear_err = false) {
  cudaError_t e = gdn::launch_chunk_prefill(
      tab, static_cast<const uint16_t*>(q), static_cast<const uint16_t*>(k),
      static_cast<const uint16_t*>(v), static_cast<const uint16_t*>(a),
      static_cast<const uint16_t*>(b), A_log, dt_bias, state, static_cast<uint16_t*>(o_out),
      qk_heads, value_heads, scratch, err, s, clear_err);
  return cuda_status(e, "chunk prefill launch");
}

int32_t gdn_b200_chunk_prefill(const void* q, const void* k, const void* v, const void* a,
                               const void* b, const float* A_log, const float* dt_bias,
                               float* state, void* o_out, const int32_t* cu_seqlens,
                               int32_t num_seqs, int32_t qk_heads, int32_t value_heads,
                               void* workspace, uint64_t workspace_bytes, void* stream) {
  if (!heads_ok(qk_heads, value_heads))
    return fail(STATECENTRIC_QWEN38_INVALID_ARGUMENT,
                "value_heads must be a positive multiple of qk_heads");
  gdn::ChunkTable tab;
  const int32_t st = check_seqlens(cu_seqlens, num_seqs, &tab);
  if (st != STATECENTRIC_QWEN38_OK) return st;
  if (q == nullptr || k == nullptr || v == nullptr || a == nullptr || b == nullptr ||
      A_log == nullptr || dt_bias == nullptr || state == nullptr || o_out == nullptr ||
      workspace == nullptr)
    return fail(STATECENTRIC_QWEN38_INVALID_ARGUMENT, "null pointer argument");
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(o_out) ||
      !aligned16(state) || !aligned16(workspace))
    return fail(STATECENTRIC_QWEN38_INVALID_ARGUMENT, "tensors must be 16-byte aligned");
  const uint64_t need = kErrBytes + round256(gdn::chunk_workspace_bytes(tab, qk_heads, value_heads));
  if (workspace_bytes < need)
    return fail(STATECENTRIC_QWEN38_INVALID_ARGUMENT,
                "workspace too small: need " + std::to_string(need) + " bytes");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  uint32_t* err = reinterpret_cast<uint32_t*>(ws);
  // The prep kernel clears the error word (no separate memset).
  return chunk_prefill_impl(tab, q, k, v, a, b, A_log, dt_bias, state, o_out, qk_heads,
                            value_heads, ws + kErrBytes, err, s, /*clear_err=*/true);
}

// ------------------------------------------------------------ layer ----

static bool all_single_token(const gdn::ChunkTable& tab) {
  for (int s = 0; s < tab.num_seqs; ++s)
    if (tab.cu[s + 1] - tab.cu[s] != 1) return false;
  return true;
}

// Post-projection layer on validated arguments: core (decode kernel when
// every sequence has one token, chunk kernels otherwise), then the tail.
// `ws` is the workspace after its error word.
static int32_t layer_forward_impl(const gdn::ChunkTable& tab, const void* q, const void* k,
                                  const void* v, const void* a, const void* b, const void* z,
                                  const float* A_log, const float* dt_bias, const void* gamma,
                                  const void* w_out, float* state, void* out, int32_t qk_heads,
                                  int32_t value_heads, int32_t hidden, uint8_t* ws, uint32_t* err,
                                  cudaStream_t s, bool clear_err = false) {
  const int64_t T = tab.cu[tab.num_seqs];
  const int64_t K = static_cast<int64_t>(value_heads) * GDN_B200_HEAD_DIM;
  uint64_t off = 0;
  uint16_t* o = reinterpret_cast<uint16_t*>(ws + off);
  off += round256(static_cast<uint64_t>(T) * K * 2);
  uint16_t* gated = reinterpret_cast<uint16_t*>(ws + off);
  off += round256(static_cast<uint64_t>(T) * K * 2);
  const bool decode = all_single_token(tab);
  uint8_t* records = ws + off;
  if (!decode) off += round256(gdn::chunk_workspace_bytes(tab, qk_heads, value_heads));
  float* gemm_ws = reinterpret_cast<float*>(ws + off);
  if (T == 0) {
    if (!clear_err) return ok();
    const cudaError_t e0 = cudaMemsetAsync(err, 0, sizeof(uint32_t), s);
    return e0 == cudaSuccess ? ok() : cuda_status(e0, "cudaMemsetAsync");
  }
  cudaError_t e;
  if (decode) {
    e = gdn::launch_decode(static_cast<const uint16_t*>(q), static_cast<const uint16_t*>(k),
                           static_cast<const uint16_t*>(v), static_cast<const uint16_t*>(a),
                           static_cast<const uint16_t*>(b), A_log, dt_bias, state, nullptr,
                           static_cast<const uint16_t*>(z), static_cast<const uint16_t*>(gamma),
                           gated, tab.num_seqs, qk_heads, value_heads, s, nullptr, err,
                           w_out, static_cast<uint64_t>(hidden) * K * 2, clear_err);
    if (e != cudaSuccess) return cuda_status(e, "decode launch");
  } else {
    const int32_t r = chunk_prefill_impl(tab, q, k, v, a, b, A_log, dt_bias, state, o, qk_heads,
                                         value_heads, records, err, s, clear_err);
    if (r != STATECENTRIC_QWEN38_OK) return r;
    e = gdn::launch_tail_prologue(o, static_cast<const uint16_t*>(z),
                                  static_cast<const uint16_t*>(gamma), gated, T, value_heads,
                                  1.0e-6f, s);
    if (e != cudaSuccess) return cuda_status(e, "tail prologue launch");
  }
  e = gdn::launch_tail_gemm(gated, static_cast<const uint16_t*>(w_out),
                            static_cast<uint16_t*>(out), gemm_ws, T, hidden, static_cast<int>(K),
                            err, s, /*overlap_previous=*/true);
  return cuda_status(e, "tail GEMM launch");
}

static uint64_t layer_scratch_bytes(const gdn::ChunkTable& tab, int32_t qk_heads,
                                    int32_t value_heads, int32_t hidden) {
  const int64_t T = tab.cu[tab.num_seqs];
  const int64_t K = static_cast<int64_t>(value_heads) * GDN_B200_HEAD_DIM;
  uint64_t bytes = 0;
  bytes += round256(static_cast<uint64_t>(T) * K * 2);  // o
  bytes += round256(static_cast<uint64_t>(T) * K * 2);  // gated
  if (!all_single_token(tab))
    bytes += round256(gdn::chunk_workspace_bytes(tab, qk_heads, value_heads));
  bytes += round256(gdn::tail_gemm_workspace_bytes(T, hidden, static_cast<int>(K)));
  return bytes;
}

uint64_t gdn_b200_layer_forward_workspace_bytes(const int32_t* cu_seqlens, int32_t num_seqs,
                                                int32_t qk_heads, int32_t value_heads,
                                                int32_t hidden) {
  gdn::ChunkTable tab;
  if (!heads_ok(qk_heads, value_heads) || hidden <= 0 ||
      check_seqlens(cu_seqlens, num_seqs, &tab) != STATECENTRIC_QWEN38_OK)
    return 0;
  return kErrBytes + layer_scratch_bytes(tab, qk_heads, value_heads, hidden);
}

int32_t gdn_b200_layer_forward(const void* q, const void* k, const void* v, const void* a,
                               const void* b, const void* z, const float* A_log,
                               const float* dt_bias, const void* gamma, const void* w_out,
                               float* state, void* out, const int32_t* cu_seqlens,
                               int32_t num_seqs, int32_t qk_heads, int32_t value_heads,
                               int32_t hidden, void* workspace, uint64_t workspace_bytes,
                               void* stream) {
  if (!heads_ok(qk_heads, value_heads))
    return fail(STATECENTRIC_QWEN38_INVALID_ARGUMENT,
                "value_heads must be a positive multiple of qk_heads");
  if (hidden <= 0 || hidden % 128 != 0)
    return fail(STATECENTRIC_QWEN38_INVALID_ARGUMENT, "hidden must be a positive multiple of 128");
  gdn::ChunkTable tab;
  const int32_t st = check_seqlens(cu_seqlens, num_seqs, &tab);
  if (st != STATECENTRIC_QWEN38_OK) return st;
  if (q == nullptr || k == nullptr || v == nullptr || a == nullptr || b == nullptr ||
      z == nullptr || A_log == nullptr || dt_bias == nullptr || gamma == nullptr ||
      w_out == nullptr || state == nullptr || out == nullptr || workspace == nullptr)
    return fail(STATECENTRIC_QWEN38_INVALID_ARGUMENT, "null pointer argument");
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(z) || !aligned16(w_out) ||
      !aligned16(out) || !aligned16(state) || !aligned16(workspace) ||
      !aligned16(gamma))
    return fail(STATECENTRIC_QWEN38_INVALID_ARGUMENT, "tensors must be 16-byte aligned");
  const uint64_t need =
      gdn_b200_layer_forward_workspace_bytes(cu_seqlens, num_seqs, qk_heads, value_heads, hidden);
  if (workspace_bytes < need)
    return fail(STATECENTRIC_QWEN38_INVALID_ARGUMENT,
                "workspace too small: need " + std::to_string(need) + " bytes");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  uint32_t* err = reinterpret_cast<uint32_t*>(ws);
  // The layer's first kernel clears the error word (no separate memset).
  return layer_forward_impl(tab, q, k, v, a, b, z, A_log, dt_bias, gamma, w_out, state, out,
                            qk_heads, value_heads, hidden, ws + kErrBytes, err, s,
                            /*clear_err=*/true);
}

// ------------------------------------------------------- input side ----

uint64_t gdn_b200_input_side_workspace_bytes(const int32_t* cu_seqlens, int32_t num_seqs,
                                             int32_t qk_heads, int32_t value_heads,
                                             int32_t hidden) {
  gdn::ChunkTable tab;
  if (!heads_ok(qk_heads, value_heads) || hidden <= 0 ||
      check_seqlens(cu_seqlens, num_seqs, &tab) != STATECENTRIC_QWEN38_OK)
    return 0;
  return kErrBytes + round256(gdn::input_side_scratch_bytes(tab.cu[num_seqs], qk_heads,
                                                            value_heads, hidden));
}

static int32_t check_input_side(const void* x, const void* w_qkv, const void* w_z,
                                const void* w_a, const void* w_b, const void* conv_w,
                                const void* conv_state, int32_t qk_heads, int32_t value_heads,
                                int32_t hidden) {
  if (!heads_ok(qk_heads, value_heads))
    return fail(STATECENTRIC_QWEN38_INVALID_ARGUMENT,
                "value_heads must be a positive multiple of qk_heads");
  if (hidden <= 0 || hidden % 128 != 0)
    return fail(STATECENTRIC_QWEN38_INVALID_ARGUMENT, "hidden must be a positive multiple of 128");
  if (x == nullptr || w_qkv == nullptr || w_z == nullptr || w_a == nullptr || w_b == nullptr ||
      conv_w == nullptr || conv_state == nullptr)
    return fail(STATECENTRIC_QWEN38_INVALID_ARGUMENT, "null pointer argument");
  if (!aligned16(x) || !aligned16(w_qkv) || !aligned16(w_z) || !aligned16(w_a) ||
      !aligned16(w_b) || !aligned16(conv_w) || !aligned16(conv_state))
    return fail(STATECENTRIC_QWEN38_INVALID_ARGUMENT, "tensors must be 16-byte aligned");
  return ok();
}

int32_t gdn_b200_input_side(const void* x, const void* w_qkv, const void* w_z, const void* w_a,
                            const void* w_b, const void* conv_w, void* conv_state,
                            const int32_t* cu_seqlens, int32_t num_seqs, int32_t qk_heads,
                            int32_t value_heads, int32_t hidden, int32_t use_conv_state,
                            void* q, void* k, void* v, void* z, void* a, void* b,
                            void* workspace, uint64_t workspace_bytes, void* stream) {
  int32_t st = check_input_side(x, w_qkv, w_z, w_a, w_b, conv_w, conv_state, qk_heads,
                                value_heads, hidden);
  if (st != STATECENTRIC_QWEN38_OK) return st;
  gdn::ChunkTable tab;
  st = check_seqlens(cu_seqlens, num_seqs, &tab);
  if (st != STATECENTRIC_QWEN38_OK) return st;
  if (q == nullptr || k == nullptr || v == nullptr || z == nullptr || a == nullptr ||
      b == nullptr || workspace == nullptr)
    return fail(STATECENTRIC_QWEN38_INVALID_ARGUMENT, "null pointer argument");
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(z) || !aligned16(workspace))
    return fail(STATECENTRIC_QWEN38_INVALID_ARGUMENT, "tensors must be 16-byte aligned");
  const uint64_t need = gdn_b200_input_side_workspace_bytes(cu_seqlens, num_seqs, qk_heads,
                                                            value_heads, hidden);
  if (workspace_bytes < need)
    return fail(STATECENTRIC_QWEN38_INVALID_ARGUMENT,
                "workspace too small: need " + std::to_string(need) + " bytes");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  uint32_t* err = reinterpret_cast<uint32_t*>(ws);
  cudaError_t e = cudaMemsetAsync(err, 0, sizeof(uint32_t), s);
  if (e != cudaSuccess) return cuda_status(e, "cudaMemsetAsync");
  e = gdn::launch_input_side(
      tab, static_cast<const uint16_t*>(x), static_cast<const uint16_t*>(w_qkv),
      static_cast<const uint16_t*>(w_z), static_cast<const uint16_t*>(w_a),
      static_cast<const uint16_t*>(w_b), static_cast<const uint16_t*>(conv_w),
      static_cast<uint16_t*>(conv_state), use_conv_state != 0, static_cast<uint16_t*>(q),
      static_cast<uint16_t*>(k), static_cast<uint16_t*>(v), static_cast<uint16_t*>(z),
      static_cast<uint16_t*>(a), static_cast<uint16_t*>(b), qk_heads, value_heads, hidden,
      ws + kErrBytes, err, s);
  return cuda_status(e, "input side launch");
}

// Layout after the error word: q, k, v, z, a, b, the input-side scratch, then
// the post-projection layer's scratch.
uint64_t gdn_b200_layer_forward_x_workspace_bytes(const int32_t* cu_seqlens, int32_t num_seqs,
                                                  int32_t qk_heads, int32_t value_heads,
                                                  int32_t hidden) {
  gdn::ChunkTable tab;
  if (!heads_ok(qk_heads, value_heads) || hidden <= 0 ||
      check_seqlens(cu_seqlens, num_seqs, &tab) != STATECENTRIC_QWEN38_OK)
    return 0;
  const uint64_t T = static_cast<uint64_t>(tab.cu[num_seqs]);
  const uint64_t qk = T * qk_heads * GDN_B200_HEAD_DIM * 2;
  const uint64_t vv = T * value_heads * GDN_B200_HEAD_DIM * 2;
  const uint64_t gate = T * value_heads * 2;
  return kErrBytes + 2 * round256(qk) + 2 * round256(vv) + 2 * round256(gate) +
         round256(gdn::input_side_scratch_bytes(T, qk_heads, value_heads, hidden)) +
         layer_scratch_bytes(tab, qk_heads, value_heads, hidden);
}

int32_t gdn_b200_layer_forward_x(const void* x, const void* w_qkv, const void* w_z,
                                 const void* w_a, const void* w_b, const void* conv_w,
                                 void* conv_state, const float* A_log, const float* dt_bias,
                                 const void* gamma, const void* w_out, float* state, void* out,
                                 const int32_t* cu_seqlens, int32_t num_seqs, int32_t qk_heads,
                                 int32_t value_heads, int32_t hidden, int32_t use_conv_state,
                                 void* workspace, uint64_t workspace_bytes, void* stream) {
  int32_t st = check_input_side(x, w_qkv, w_z, w_a, w_b, conv_w, conv_state, qk_heads,
                                value_heads, hidden);
  if (st != STATECENTRIC_QWEN38_OK) return st;
  gdn::ChunkTable tab;
  st = check_seqlens(cu_seqlens, num_seqs, &tab);
  if (st != STATECENTRIC_QWEN38_OK) return st;
  if (A_log == nullptr || dt_bias == nullptr || gamma == nullptr || w_out == nullptr ||
      state == nullptr || out == nullptr || workspace == nullptr)
    return fail(STATECENTRIC_QWEN38_INVALID_ARGUMENT, "null pointer argument");
  if (!aligned16(gamma) || !aligned16(w_out) || !aligned16(state) || !aligned16(out) ||
      !aligned16(workspace))
    return fail(STATECENTRIC_QWEN38_INVALID_ARGUMENT, "tensors must be 16-byte aligned");
  const uint64_t need = gdn_b200_layer_forward_x_workspace_bytes(cu_seqlens, num_seqs, qk_heads,
                                                                 value_heads, hidden);
  if (workspace_bytes < need)
    return fail(STATECENTRIC_QWEN38_INVALID_ARGUMENT,
                "workspace too small: need " + std::to_string(need) + " bytes");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  uint32_t* err = reinterpret_cast<uint32_t*>(ws);
  const uint64_t T = static_cast<uint64_t>(tab.cu[num_seqs]);
  const uint64_t qk = T * qk_heads * GDN_B200_HEAD_DIM * 2;
  const uint64_t vv = T * value_heads * GDN_B200_HEAD_DIM * 2;
  const uint64_t gate = T * value_heads * 2;
  uint64_t off = kErrBytes;
  auto take = [&](uint64_t bytes) {
    uint16_t* p = reinterpret_cast<uint16_t*>(ws + off);
    off += round256(bytes);
    return p;
  };
  uint16_t* q = take(qk);
  uint16_t* k = take(qk);
  uint16_t* v = take(vv);
  uint16_t* z = take(vv);
  uint16_t* a = take(gate);
  uint16_t* b = take(gate);
  uint8_t* in_scratch = ws + off;
  off += round256(gdn::input_side_scratch_bytes(T, qk_heads, value_heads, hidden));
  cudaError_t e = cudaMemsetAsync(err, 0, sizeof(uint32_t), s);
  if (e != cudaSuccess) return cuda_status(e, "cudaMemsetAsync");
  e = gdn::launch_input_side(tab, static_cast<const uint16_t*>(x),
                             static_cast<const uint16_t*>(w_qkv), static_cast<const uint16_t*>(w_z),
                             static_cast<const uint16_t*>(w_a), static_cast<const uint16_t*>(w_b),
                             static_cast<const uint16_t*>(conv_w),
                             static_cast<uint16_t*>(conv_state), use_conv_state != 0, q, k, v, z,
                             a, b, qk_heads, value_heads, hidden, in_scratch, err, s);
  if (e != cudaSuccess) return cuda_status(e, "input side launch");
  return layer_forward_impl(tab, q, k, v, a, b, z, A_log, dt_bias, gamma, w_out, state, out,
                            qk_heads, value_heads, hidden, ws + off, err, s);
}

// ---------------------------------------------------- graph binding ----

int32_t gdn_b200_copy_graph_rows(const statecentric_qwen38_gdn_layout_workspace_v1* layout,
                                 uint64_t batch_size, uint64_t conv_bytes,
                                 uint64_t recurrent_bytes, uint64_t packed_conv,
                                 uint64_t packed_recurrent, int32_t gather, void* stream) {
  if (layout == nullptr) return fail(STATECENTRIC_QWEN38_INVALID_ARGUMENT, "layout is null");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t first = cudaSuccess;
  const char* refused = gdn_b200::CopyGraphRows(
      *layout, static_cast<std::size_t>(batch_size), conv_bytes, recurrent_bytes,
      static_cast<uintptr_t>(packed_conv), static_cast<uintptr_t>(packed_recurrent), gather != 0,
      [&](uintptr_t dst, uint64_t bytes, uintptr_t src) {
        if (first == cudaSuccess)
          first = cudaMemcpyAsync(reinterpret_cast<void*>(dst), reinterpret_cast<const void*>(src),
                                  bytes, cudaMemcpyDeviceToDevice, s);
      });
  if (refused != nullptr) return fail(STATECENTRIC_QWEN38_INVALID_ARGUMENT, refused);
  return cuda_status(first, "cudaMemcpyAsync(graph rows)");
}

// -------------------------------------------------- synthetic inputs ----

static inline uint64_t splitmix64(uint64_t x) {
  x += 0x9E3779B97F4A7C15ull;
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
  return x ^ (x >> 31);
}

static inline uint16_t host_bf16(float f) {
  uint32_t u;
  std::memcpy(&u, &f, sizeof u);
  if ((u & 0x7F800000u) == 0x7F800000u && (u & 0x007FFFFFu) != 0) return static_cast<uint16_t>((u >> 16) | 0x40u);
  u += 0x7FFFu + ((u >> 16) & 1u);
  return static_cast<uint16_t>(u >> 16);
}

int32_t gdn_b200_fill_synthetic(uint64_t seed, uint64_t tensor_id, uint64_t count,
                                int32_t distribution, float p0, float p1, int32_t out_dtype,
                                void* host_out) {
  if (host_out == nullptr && count > 0)
    return fail(STATECENTRIC_QWEN38_INVALID_ARGUMENT, "null output");
  if (distribution < 0 || distribution > 2 || (out_dtype != 1 && out_dtype != 2))
    return fail(STATECENTRIC_QWEN38_INVALID_ARGUMENT, "bad distribution or dtype");
  const uint64_t key = splitmix64(splitmix64(seed) ^ (tensor_id * 0xD1B54A32D192ED03ull));
  const double two_pi = 6.283185307179586476925286766559;
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < static_cast<int64_t>(count); ++i) {
    const uint64_t r1 = splitmix64(key + 2 * static_cast<uint64_t>(i));
    const uint64_t r2 = splitmix64(key + 2 * static_cast<uint64_t>(i) + 1);
    const double u1 = (static_cast<double>(r1 >> 11) + 1.0) * (1.0 / 9007199254740992.0);  // (0,1]
    const double u2 = static_cast<double>(r2 >> 11) * (1.0 / 9007199254740992.0);          // [0,1)
    double val;
    if (distribution == 0) {
      val = p0 + p1 * std::sqrt(-2.0 * std::log(u1)) * std::cos(two_pi * u2);
    } else if (distribution == 1) {
      val = p0 + (p1 - p0) * u2;
    } else {
      val = std::log(p0 + (p1 - p0) * u1);
    }
    if (out_dtype == 1) {
      static_cast<uint16_t*>(host_out)[i] = host_bf16(static_cast<float>(val));
    } else {
      static_cast<float*>(host_out)[i] = static_cast<float>(val);
    }
  }
  return ok();
}

}  // extern "C"
