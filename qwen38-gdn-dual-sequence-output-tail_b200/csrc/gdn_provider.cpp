// Provider C ABI (include/statecentric_qwen38_provider_api_v1.h) on top of
// the B200 kernels.
//
// Mirrors the reference provider's entry points and error behaviour
// (native/src/qwen38_geometry_normalized_gdn_provider.cpp, "P"):
//   query      P:3662-3694   descriptor with eight function pointers
//   Create     P:1865-2226   contract + configuration validation
//   Submit     P:2249-3559   execution/tensor validation, deadline, enqueue
//   Poll       P:3570-3596   OK when complete, NOT_READY otherwise
//   Wait       P:3598-3629   bounded wait, TIMEOUT at the deadline
//   Cancel     P:3631-3637   always UNSUPPORTED
//   ReleaseEvent P:3639-3654 synchronise if needed, then free
//   ReleaseError P:3656-3658
// Exceptions never cross the ABI: every failure is a status plus an owned
// error message.  Work is enqueued on the caller's stream; completion is a
// CUDA event recorded after the last kernel of the submission.
//
// Executed paths (flags always include GDN_FORWARD_V1):
//   GDN_FORWARD_V1 alone or with a split variant (PREFILL_SPLIT_V2/V3,
//     STRIDED_QKV_V4, POST_CONV_PACK_V5; the variants only change how the
//     reference splits q/k/v, P:3186-3247): the reference's x-based layer,
//     inputs x, w_qkv, w_z, w_a, w_b, conv_w, A_log, dt_bias, gamma, w_out
//     (P:2387-2410); mutable state gdn.conv then gdn.recurrent (P:2313-2314);
//     zero conv history when context_tokens is 0 (P:3163-3173).
//   GDN_POST_PROJECTION_V6: inputs q, k, v, a, b, z, A_log, dt_bias, gamma,
//     w_out; mutable state gdn.conv (validated, untouched) and gdn.recurrent;
//     one packed decode launch when every sequence has one token, one
//     chunked-prefill launch otherwise, then the flattened output tail.
//   GDN_OUTPUT_TAIL_V7: inputs o, z, gamma, w_out; only the output tail.
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <mutex>
#include <new>
#include <string>
#include <thread>
#include <vector>

#include "completed_buffer_pool.h"
#include "gdn_b200.h"
#include "gdn_plan.h"
#include "statecentric_qwen38_provider_api_v1.h"

struct statecentric_qwen38_provider_handle_v1 {
  const statecentric_qwen38_host_v1* host = nullptr;
  uint32_t rank = 0;
  uint32_t world_size = 1;
  int32_t device = 0;
  uint32_t hidden = 0;
  uint32_t qkv = 0;
  uint32_t value = 0;
  uint32_t qk_heads = 0;
  uint32_t value_heads = 0;
  uint32_t max_tokens = 0;
  std::unique_ptr<statecentric::CompletedBufferPool> pool;
  std::atomic<uint64_t> submissions{0};
  std::atomic<uint64_t> private_allocations{0};
  // Admission telemetry (the reference's first-admission lines, P:590-723,
  // for the paths that exist here): every validated GDN submission is a
  // submit call; each executed path counts its admissions and writes one
  // line to stderr at its first.
  std::atomic<uint64_t> gdn_submit_calls{0};
  std::atomic<uint64_t> packed_decode_admitted{0};
  std::atomic<uint64_t> chunk_prefill_admitted{0};
  std::atomic<uint64_t> input_side_admitted{0};
  std::atomic<bool> packed_decode_emitted{false};
  std::atomic<bool> decode_flat_output_emitted{false};
  std::atomic<bool> chunk_prefill_emitted{false};
  std::atomic<bool> input_side_emitted{false};
};

struct statecentric_qwen38_event_v1 {
  cudaStream_t stream = nullptr;
  cudaEvent_t done = nullptr;
  uint64_t submitted_ns = 0;
  bool complete = false;
  statecentric::CompletedBufferPool* pool = nullptr;
  std::vector<statecentric::CompletedBufferPool::Lease> leases;
  std::vector<void*> allocations;  // private cudaMalloc fallbacks
  void* workspace = nullptr;       // holds the device error word
};

namespace {

constexpr uint32_t kAbi = STATECENTRIC_QWEN38_PROVIDER_ABI_V1;

// One telemetry line, written once per handle (`flag` guards it).
void EmitOnce(std::atomic<bool>& flag, const char* line) {
  bool expected = false;
  if (flag.compare_exchange_strong(expected, true, std::memory_order_acq_rel,
                                   std::memory_order_relaxed)) {
    std::fputs(line, stderr);
    std::fflush(stderr);
  }
}

void RecordAdmission(statecentric_qwen38_provider_handle_v1* h, bool from_x, bool decode,
                     uint64_t sequences, uint64_t rows, uint64_t chunks) {
  const auto submits = static_cast<unsigned long long>(h->gdn_submit_calls.load());
  char line[320];
  if (from_x) {
    const auto n = static_cast<unsigned long long>(h->input_side_admitted.fetch_add(1) + 1);
    std::snprintf(line, sizeof line,
                  "STATECENTRIC_QWEN38_GDN_B200_INPUT_SIDE_TELEMETRY_V1="
                  "{\"rank\":%u,\"submit_calls\":%llu,\"admitted_calls\":%llu}\n",
                  h->rank, submits, n);
    EmitOnce(h->input_side_emitted, line);
  }
  if (decode) {
    const auto n = static_cast<unsigned long long>(h->packed_decode_admitted.fetch_add(1) + 1);
    std::snprintf(line, sizeof line,
                  "STATECENTRIC_QWEN38_GDN_PACKED_DECODE_TELEMETRY_V12="
                  "{\"rank\":%u,\"submit_calls\":%llu,\"admitted_calls\":%llu}\n",
                  h->rank, submits, n);
    EmitOnce(h->packed_decode_emitted, line);
    std::snprintf(line, sizeof line,
                  "STATECENTRIC_QWEN38_GDN_DECODE_FLAT_OUTPUT_PROJECTION_V18="
                  "{\"rank\":%u,\"admitted_calls\":%llu,\"rows\":%llu}\n",
                  h->rank, n, static_cast<unsigned long long>(rows));
    EmitOnce(h->decode_flat_output_emitted, line);
  } else {
    const auto n = static_cast<unsigned long long>(h->chunk_prefill_admitted.fetch_add(1) + 1);
    std::snprintf(line, sizeof line,
                  "STATECENTRIC_QWEN38_GDN_B200_CHUNK_PREFILL_TELEMETRY_V1="
                  "{\"rank\":%u,\"submit_calls\":%llu,\"admitted_calls\":%llu,"
                  "\"sequences\":%llu,\"chunks\":%llu}\n",
                  h->rank, submits, n, static_cast<unsigned long long>(sequences),
                  static_cast<unsigned long long>(chunks));
    EmitOnce(h->chunk_prefill_emitted, line);
  }
}
constexpr uint32_t kHeadDim = GDN_B200_HEAD_DIM;
constexpr uint64_t kMaxTokensLimit = 1ull << 22;

struct OwnedError {
  statecentric_qwen38_error_v1 value{};
  std::string message;
};

int32_t Fail(int32_t status, std::string message, statecentric_qwen38_error_v1** out_error) {
  if (out_error != nullptr) {
    auto* owned = new (std::nothrow) OwnedError;
    if (owned != nullptr) {
      owned->message = std::move(message);
      owned->value = {sizeof(statecentric_qwen38_error_v1), kAbi, status, 0,
                      owned->message.c_str(), nullptr};
      *out_error = &owned->value;
    }
  }
  return status;
}

class DeviceGuard {
 public:
  explicit DeviceGuard(int device) {
    if (cudaGetDevice(&previous_) != cudaSuccess) previous_ = -1;
    if (previous_ != device) ok_ = cudaSetDevice(device) == cudaSuccess;
  }
  ~DeviceGuard() {
    if (previous_ >= 0) cudaSetDevice(previous_);
  }
  bool ok() const { return ok_; }

 private:
  int previous_ = -1;
  bool ok_ = true;
};

// Tensor view check in the manner of TensorGeometry (P:1840-1863).
bool TensorGeometry(const statecentric_qwen38_tensor_v1& t, int32_t device, uint32_t scalar,
                    std::initializer_list<uint64_t> dims, std::initializer_list<int64_t> strides,
                    uint64_t element_bytes) {
  if (t.size < sizeof(t) || t.abi_version != kAbi || t.data == 0 || t.scalar_type != scalar ||
      t.memory_kind != STATECENTRIC_QWEN38_MEMORY_DEVICE || t.device_ordinal != device ||
      t.rank != dims.size() || dims.size() > STATECENTRIC_QWEN38_MAX_TENSOR_RANK)
    return false;
  uint64_t elements = 1;
  size_t i = 0;
  auto st = strides.begin();
  for (const uint64_t d : dims) {
    if (t.dimensions[i] != d || t.strides[i] != *st) return false;
    elements *= d;
    ++i;
    ++st;
  }
  return t.byte_length == elements * element_bytes;
}

bool StateRegion(const statecentric_qwen38_state_region_v1& r, uint32_t layer, const char* kind) {
  return r.size >= sizeof(r) && r.abi_version == kAbi && r.layer_index == layer &&
         r.state_kind != nullptr && std::strcmp(r.state_kind, kind) == 0;
}

void* PoolAllocate(size_t bytes) {
  void* p = nullptr;
  return cudaMalloc(&p, bytes) == cudaSuccess ? p : nullptr;
}
bool PoolFree(void* p) { return cudaFree(p) == cudaSuccess; }

void FreeEvent(statecentric_qwen38_event_v1* event) {
  if (event == nullptr) return;
  for (const auto& lease : event->leases) event->pool->Retire(lease, event->complete);
  event->leases.clear();
  for (void* p : event->allocations) {
    if (event->complete) {
      cudaFree(p);
    }
    // Memory of work that did not complete is leaked rather than freed under
    // the device: the reference quarantines for the same reason (P:551-554).
  }
  event->allocations.clear();
  if (event->done != nullptr) cudaEventDestroy(event->done);
  delete event;
}

// Scratch for one submission: a pool lease, else a private allocation.
void* AcquireWorkspace(statecentric_qwen38_provider_handle_v1* h,
                       statecentric_qwen38_event_v1* ev, uint64_t bytes) {
  if (bytes == 0) bytes = 256;
  if (h->pool) {
    auto lease = h->pool->Borrow(reinterpret_cast<uintptr_t>(ev), bytes);
    if (lease) {
      ev->leases.push_back(*lease);
      return lease->pointer;
    }
  }
  void* p = nullptr;
  if (cudaMalloc(&p, bytes) != cudaSuccess) return nullptr;
  ev->allocations.push_back(p);
  h->private_allocations.fetch_add(1, std::memory_order_relaxed);
  return p;
}

int32_t Create(const statecentric_qwen38_host_v1* host, const statecentric_qwen38_create_v1* create,
               statecentric_qwen38_provider_handle_v1** out_handle,
               statecentric_qwen38_error_v1** out_error) {
  if (host == nullptr || create == nullptr || out_handle == nullptr || host->size < sizeof(*host) ||
      host->abi_version != kAbi || host->monotonic_time_ns == nullptr ||
      create->size < sizeof(*create) || create->abi_version != kAbi ||
      !(create->world_size == 1 || create->world_size == 2 || create->world_size == 4 ||
        create->world_size == 8) ||
      create->rank >= create->world_size || create->device_ordinal < 0 ||
      create->assembly_fingerprint_sha256 == nullptr ||
      create->assembly_fingerprint_length != 32 || create->configuration == nullptr ||
      create->configuration_length <
          offsetof(statecentric_qwen38_gdn_create_config_v1, prefill_qkv_split_variant)) {
    return Fail(STATECENTRIC_QWEN38_INVALID_ARGUMENT, "invalid Qwen3.8 GDN create contract",
                out_error);
  }
  statecentric_qwen38_gdn_create_config_v1 config{};
  std::memcpy(&config, create->configuration,
              std::min<uint64_t>(create->configuration_length, sizeof(config)));
  const uint64_t min_size =
      offsetof(statecentric_qwen38_gdn_create_config_v1, prefill_qkv_split_variant);
  const bool heads_ok = config.query_heads_per_rank > 0 && config.value_heads_per_rank > 0 &&
                        config.value_heads_per_rank % config.query_heads_per_rank == 0 &&
                        config.gate_heads_per_rank == config.value_heads_per_rank &&
                        config.value_size_per_rank == config.value_heads_per_rank * kHeadDim &&
                        config.qkv_size_per_rank ==
                            2 * config.query_heads_per_rank * kHeadDim +
                                config.value_size_per_rank;
  if (config.size < min_size || config.size > create->configuration_length ||
      config.abi_version != kAbi || config.hidden_size == 0 || config.hidden_size % 128 != 0 ||
      config.head_dim != kHeadDim || !heads_ok || config.max_tokens_per_submission == 0 ||
      config.max_tokens_per_submission > kMaxTokensLimit ||
      config.prefill_qkv_split_variant > 7 || config.reserved != 0) {
    return Fail(STATECENTRIC_QWEN38_INVALID_ARGUMENT, "invalid Qwen3.8 GDN configuration",
                out_error);
  }
  int count = 0;
  if (cudaGetDeviceCount(&count) != cudaSuccess || create->device_ordinal >= count) {
    cudaGetLastError();
    return Fail(STATECENTRIC_QWEN38_INTERNAL, "CUDA device is not available", out_error);
  }
  auto* handle = new (std::nothrow) statecentric_qwen38_provider_handle_v1;
  if (handle == nullptr)
    return Fail(STATECENTRIC_QWEN38_INTERNAL, "cannot allocate Qwen3.8 GDN provider", out_error);
  handle->host = host;
  handle->rank = create->rank;
  handle->world_size = create->world_size;
  handle->device = create->device_ordinal;
  handle->hidden = config.hidden_size;
  handle->qkv = config.qkv_size_per_rank;
  handle->value = config.value_size_per_rank;
  handle->qk_heads = config.query_heads_per_rank;
  handle->value_heads = config.value_heads_per_rank;
  handle->max_tokens = config.max_tokens_per_submission;
  // Budget: the reference pool is 64 MiB with an 8 MiB per-buffer cap
  // (P:2207-2216).  Whole submissions here take one scratch buffer, so both
  // limits grow to the largest submission the configuration admits.
  std::vector<int32_t> cu{0, static_cast<int32_t>(handle->max_tokens)};
  const uint64_t need = gdn_b200_layer_forward_workspace_bytes(
      cu.data(), 1, static_cast<int32_t>(handle->qk_heads),
      static_cast<int32_t>(handle->value_heads), static_cast<int32_t>(handle->hidden));
  const uint64_t budget = std::max<uint64_t>(64ull << 20, 2 * need);
  const uint64_t cap = std::max<uint64_t>(8ull << 20, need + (1ull << 20));
  handle->pool = std::make_unique<statecentric::CompletedBufferPool>(
      budget, cap, [dev = handle->device](size_t bytes) {
        DeviceGuard g(dev);
        return PoolAllocate(bytes);
      },
      [dev = handle->device](void* p) {
        DeviceGuard g(dev);
        return PoolFree(p);
      });
  *out_handle = handle;
  return STATECENTRIC_QWEN38_OK;
}

void Destroy(statecentric_qwen38_provider_handle_v1* handle) {
  if (handle == nullptr) return;
  if (handle->pool) {
    DeviceGuard g(handle->device);
    const bool drained = handle->pool->Close();
    const auto s = handle->pool->Snapshot();
    const char* telemetry = std::getenv("STATECENTRIC_QWEN38_GDN_POOL_TELEMETRY");
    if (telemetry != nullptr && std::strcmp(telemetry, "1") == 0) {
      std::fprintf(stderr,
                   "STATECENTRIC_GDN_B200_POOL={\"rank\":%u,\"drained\":%s,\"owned_bytes\":%zu,"
                   "\"peak_owned_bytes\":%zu,\"active_leases\":%zu,\"quarantined_buffers\":%zu,"
                   "\"allocations\":%llu,\"reuses\":%llu,\"budget_bypasses\":%llu,"
                   "\"submissions\":%llu}\n",
                   handle->rank, drained ? "true" : "false", s.owned_bytes, s.peak_owned_bytes,
                   s.active_leases, s.quarantined_buffers,
                   static_cast<unsigned long long>(s.allocations),
                   static_cast<unsigned long long>(s.reuses),
                   static_cast<unsigned long long>(s.budget_bypasses),
                   static_cast<unsigned long long>(handle->submissions.load()));
    }
    handle->pool.reset();
  }
  delete handle;
}

struct Validated {
  uint64_t tokens = 0;
  uint64_t states = 1;
  std::vector<int32_t> cu;
  std::vector<uint32_t> counts;
};

int32_t Submit(statecentric_qwen38_provider_handle_v1* handle,
               const statecentric_qwen38_execution_v1* execution, uint64_t deadline_monotonic_ns,
               statecentric_qwen38_event_v1** out_event, statecentric_qwen38_error_v1** out_error) {
  constexpr uint32_t kV6 = STATECENTRIC_QWEN38_GDN_FORWARD_V1 | STATECENTRIC_QWEN38_GDN_POST_PROJECTION_V6;
  constexpr uint32_t kV7 = STATECENTRIC_QWEN38_GDN_FORWARD_V1 | STATECENTRIC_QWEN38_GDN_OUTPUT_TAIL_V7;
  if (handle == nullptr || execution == nullptr || out_event == nullptr ||
      execution->size < sizeof(*execution) || execution->abi_version != kAbi ||
      execution->rank != handle->rank || execution->world_size != handle->world_size ||
      execution->device_ordinal != handle->device ||
      execution->stage != STATECENTRIC_QWEN38_STAGE_GDN || execution->layer_index >= 64 ||
      execution->layer_index % 4 == 3 || execution->token_count == 0 ||
      execution->token_count > handle->max_tokens || execution->stream == 0 ||
      execution->inputs == nullptr || execution->outputs == nullptr ||
      execution->output_count != 1) {
    return Fail(STATECENTRIC_QWEN38_INVALID_ARGUMENT, "invalid Qwen3.8 GDN submission", out_error);
  }
  const uint32_t flags = execution->flags;
  const bool known_reference_flag =
      flags == STATECENTRIC_QWEN38_GDN_FORWARD_V1 ||
      flags == (STATECENTRIC_QWEN38_GDN_FORWARD_V1 | STATECENTRIC_QWEN38_GDN_PREFILL_SPLIT_V2) ||
      flags == (STATECENTRIC_QWEN38_GDN_FORWARD_V1 | STATECENTRIC_QWEN38_GDN_PREFILL_SPLIT_V3) ||
      flags == (STATECENTRIC_QWEN38_GDN_FORWARD_V1 | STATECENTRIC_QWEN38_GDN_PREFILL_STRIDED_QKV_V4) ||
      flags == (STATECENTRIC_QWEN38_GDN_FORWARD_V1 | STATECENTRIC_QWEN38_GDN_PREFILL_POST_CONV_PACK_V5);
  if (!known_reference_flag && flags != kV6 && flags != kV7) {
    return Fail(STATECENTRIC_QWEN38_INVALID_ARGUMENT, "invalid Qwen3.8 GDN submission flags",
                out_error);
  }
  const bool from_x = known_reference_flag;
  const bool tail_only = flags == kV7;
  if ((tail_only && (execution->input_count != 4 || execution->mutable_state_count != 0)) ||
      (from_x && (execution->input_count != 10 || execution->mutable_state == nullptr ||
                  execution->mutable_state_count != 2)) ||
      (!tail_only && !from_x &&
       (execution->input_count != 10 || execution->mutable_state == nullptr ||
        (execution->mutable_state_count != 1 && execution->mutable_state_count != 2)))) {
    return Fail(STATECENTRIC_QWEN38_INVALID_ARGUMENT, "invalid Qwen3.8 GDN submission counts",
                out_error);
  }

  const uint64_t tokens = execution->token_count;
  const int32_t dev = handle->device;
  const uint64_t hk = handle->qk_heads, hv = handle->value_heads, value = handle->value;
  const uint64_t hidden = handle->hidden, D = kHeadDim;
  const auto& in = execution->inputs;

  // Sequences: the packed gdn_batch_v1 metadata (P:2321-2350) when several
  // states are present, one sequence otherwise.
  Validated v;
  v.tokens = tokens;
  const statecentric_qwen38_state_region_v1* recurrent = nullptr;
  const statecentric_qwen38_state_region_v1* conv = nullptr;
  if (!tail_only) {
    recurrent = &execution->mutable_state[execution->mutable_state_count - 1];
    if (execution->mutable_state_count == 2) conv = &execution->mutable_state[0];
    v.states = recurrent->tensor.dimensions[0];
  }
  if (execution->workspace != 0) {
    if (execution->workspace_length != sizeof(statecentric_qwen38_gdn_batch_v1))
      return Fail(STATECENTRIC_QWEN38_INVALID_ARGUMENT,
                  "Qwen3.8 multi-state GDN metadata is invalid", out_error);
    const auto* batch = reinterpret_cast<const statecentric_qwen38_gdn_batch_v1*>(execution->workspace);
    if (batch->size < sizeof(*batch) || batch->abi_version != kAbi || batch->reserved != 0 ||
        batch->token_offsets == nullptr || batch->token_counts == nullptr ||
        batch->state_count == 0 || batch->state_count > GDN_B200_MAX_SEQUENCES ||
        (!tail_only && batch->state_count != v.states))
      return Fail(STATECENTRIC_QWEN38_INVALID_ARGUMENT,
                  "Qwen3.8 multi-state GDN metadata is invalid", out_error);
    v.states = batch->state_count;
    uint64_t expected = 0;
    v.cu.push_back(0);
    for (uint64_t s = 0; s < v.states; ++s) {
      if (batch->token_offsets[s] != expected || batch->token_counts[s] == 0)
        return Fail(STATECENTRIC_QWEN38_INVALID_ARGUMENT,
                    "Qwen3.8 multi-state GDN ranges are not packed", out_error);
      expected += batch->token_counts[s];
      v.counts.push_back(batch->token_counts[s]);
      v.cu.push_back(static_cast<int32_t>(expected));
    }
    if (expected != tokens)
      return Fail(STATECENTRIC_QWEN38_INVALID_ARGUMENT,
                  "Qwen3.8 multi-state GDN ranges do not cover tokens", out_error);
  } else {
    if (execution->workspace_length != 0 || (!tail_only && v.states != 1))
      return Fail(STATECENTRIC_QWEN38_INVALID_ARGUMENT,
                  "Qwen3.8 multi-state GDN metadata is missing", out_error);
    v.states = 1;
    v.cu = {0, static_cast<int32_t>(tokens)};
    v.counts = {static_cast<uint32_t>(tokens)};
  }
  if (!tail_only) handle->gdn_submit_calls.fetch_add(1, std::memory_order_relaxed);
  const auto plan = statecentric::PlanGdnB200Submission(v.counts, handle->max_tokens,
                                                        GDN_B200_MAX_SEQUENCES);
  if (!plan.admitted)
    return Fail(STATECENTRIC_QWEN38_INVALID_ARGUMENT, "Qwen3.8 GDN submission was not admitted",
                out_error);

  bool tensors_valid;
  const auto& out = execution->outputs[0];
  const uint64_t qkv = handle->qkv;
  if (from_x) {
    const uint64_t S = v.states;
    tensors_valid =
        TensorGeometry(in[0], dev, STATECENTRIC_QWEN38_SCALAR_BF16, {tokens, hidden}, {int64_t(hidden), 1}, 2) &&
        TensorGeometry(in[1], dev, STATECENTRIC_QWEN38_SCALAR_BF16, {hidden, qkv}, {1, int64_t(hidden)}, 2) &&
        TensorGeometry(in[2], dev, STATECENTRIC_QWEN38_SCALAR_BF16, {hidden, value}, {1, int64_t(hidden)}, 2) &&
        TensorGeometry(in[3], dev, STATECENTRIC_QWEN38_SCALAR_BF16, {hidden, hv}, {1, int64_t(hidden)}, 2) &&
        TensorGeometry(in[4], dev, STATECENTRIC_QWEN38_SCALAR_BF16, {hidden, hv}, {1, int64_t(hidden)}, 2) &&
        TensorGeometry(in[5], dev, STATECENTRIC_QWEN38_SCALAR_BF16, {4, qkv}, {int64_t(qkv), 1}, 2) &&
        TensorGeometry(in[6], dev, STATECENTRIC_QWEN38_SCALAR_F32, {hv}, {1}, 4) &&
        TensorGeometry(in[7], dev, STATECENTRIC_QWEN38_SCALAR_F32, {hv}, {1}, 4) &&
        TensorGeometry(in[8], dev, STATECENTRIC_QWEN38_SCALAR_BF16, {D}, {1}, 2) &&
        TensorGeometry(in[9], dev, STATECENTRIC_QWEN38_SCALAR_BF16, {value, hidden}, {1, int64_t(value)}, 2) &&
        TensorGeometry(out, dev, STATECENTRIC_QWEN38_SCALAR_BF16, {tokens, hidden}, {int64_t(hidden), 1}, 2) &&
        StateRegion(*conv, execution->layer_index, "gdn.conv") &&
        TensorGeometry(conv->tensor, dev, STATECENTRIC_QWEN38_SCALAR_BF16, {S, 3, qkv},
                       {int64_t(3 * qkv), int64_t(qkv), 1}, 2) &&
        StateRegion(*recurrent, execution->layer_index, "gdn.recurrent") &&
        TensorGeometry(recurrent->tensor, dev, STATECENTRIC_QWEN38_SCALAR_F32, {S, hv, D, D},
                       {int64_t(hv * D * D), int64_t(D * D), int64_t(D), 1}, 4);
  } else if (tail_only) {
    tensors_valid =
        TensorGeometry(in[0], dev, STATECENTRIC_QWEN38_SCALAR_BF16, {tokens, value}, {int64_t(value), 1}, 2) &&
        TensorGeometry(in[1], dev, STATECENTRIC_QWEN38_SCALAR_BF16, {tokens, value}, {int64_t(value), 1}, 2) &&
        TensorGeometry(in[2], dev, STATECENTRIC_QWEN38_SCALAR_BF16, {D}, {1}, 2) &&
        TensorGeometry(in[3], dev, STATECENTRIC_QWEN38_SCALAR_BF16, {value, hidden}, {1, int64_t(value)}, 2) &&
        TensorGeometry(out, dev, STATECENTRIC_QWEN38_SCALAR_BF16, {tokens, hidden}, {int64_t(hidden), 1}, 2);
  } else {
    const uint64_t S = v.states;
    tensors_valid =
        TensorGeometry(in[0], dev, STATECENTRIC_QWEN38_SCALAR_BF16, {tokens, hk * D}, {int64_t(hk * D), 1}, 2) &&
        TensorGeometry(in[1], dev, STATECENTRIC_QWEN38_SCALAR_BF16, {tokens, hk * D}, {int64_t(hk * D), 1}, 2) &&
        TensorGeometry(in[2], dev, STATECENTRIC_QWEN38_SCALAR_BF16, {tokens, value}, {int64_t(value), 1}, 2) &&
        TensorGeometry(in[3], dev, STATECENTRIC_QWEN38_SCALAR_BF16, {tokens, hv}, {int64_t(hv), 1}, 2) &&
        TensorGeometry(in[4], dev, STATECENTRIC_QWEN38_SCALAR_BF16, {tokens, hv}, {int64_t(hv), 1}, 2) &&
        TensorGeometry(in[5], dev, STATECENTRIC_QWEN38_SCALAR_BF16, {tokens, value}, {int64_t(value), 1}, 2) &&
        TensorGeometry(in[6], dev, STATECENTRIC_QWEN38_SCALAR_F32, {hv}, {1}, 4) &&
        TensorGeometry(in[7], dev, STATECENTRIC_QWEN38_SCALAR_F32, {hv}, {1}, 4) &&
        TensorGeometry(in[8], dev, STATECENTRIC_QWEN38_SCALAR_BF16, {D}, {1}, 2) &&
        TensorGeometry(in[9], dev, STATECENTRIC_QWEN38_SCALAR_BF16, {value, hidden}, {1, int64_t(value)}, 2) &&
        TensorGeometry(out, dev, STATECENTRIC_QWEN38_SCALAR_BF16, {tokens, hidden}, {int64_t(hidden), 1}, 2) &&
        StateRegion(*recurrent, execution->layer_index, "gdn.recurrent") &&
        TensorGeometry(recurrent->tensor, dev, STATECENTRIC_QWEN38_SCALAR_F32, {S, hv, D, D},
                       {int64_t(hv * D * D), int64_t(D * D), int64_t(D), 1}, 4) &&
        (conv == nullptr ||
         (StateRegion(*conv, execution->layer_index, "gdn.conv") &&
          TensorGeometry(conv->tensor, dev, STATECENTRIC_QWEN38_SCALAR_BF16, {S, 3, handle->qkv},
                         {int64_t(3 * handle->qkv), int64_t(handle->qkv), 1}, 2)));
  }
  if (!tensors_valid)
    return Fail(STATECENTRIC_QWEN38_INVALID_ARGUMENT, "invalid Qwen3.8 GDN tensor or state geometry",
                out_error);

  const uint64_t started = handle->host->monotonic_time_ns(handle->host->context);
  if (deadline_monotonic_ns <= started)
    return Fail(STATECENTRIC_QWEN38_TIMEOUT, "Qwen3.8 GDN deadline expired", out_error);

  DeviceGuard guard(dev);
  if (!guard.ok())
    return Fail(STATECENTRIC_QWEN38_INTERNAL, "cudaSetDevice failed", out_error);
  auto* event = new (std::nothrow) statecentric_qwen38_event_v1;
  if (event == nullptr)
    return Fail(STATECENTRIC_QWEN38_INTERNAL, "cannot allocate Qwen3.8 GDN event", out_error);
  event->stream = reinterpret_cast<cudaStream_t>(execution->stream);
  event->submitted_ns = started;
  event->pool = handle->pool.get();
  if (cudaEventCreateWithFlags(&event->done, cudaEventDisableTiming) != cudaSuccess) {
    event->done = nullptr;
    event->complete = true;
    FreeEvent(event);
    return Fail(STATECENTRIC_QWEN38_INTERNAL, "cudaEventCreate failed", out_error);
  }

  const int32_t nseq = static_cast<int32_t>(v.states);
  uint64_t ws_bytes =
      tail_only ? gdn_b200_output_tail_workspace_bytes(static_cast<int64_t>(tokens),
                                                       static_cast<int32_t>(hv),
                                                       static_cast<int32_t>(hidden))
      : from_x  ? gdn_b200_layer_forward_x_workspace_bytes(v.cu.data(), nseq,
                                                           static_cast<int32_t>(hk),
                                                           static_cast<int32_t>(hv),
                                                           static_cast<int32_t>(hidden))
                : gdn_b200_layer_forward_workspace_bytes(v.cu.data(), nseq,
                                                         static_cast<int32_t>(hk),
                                                         static_cast<int32_t>(hv),
                                                         static_cast<int32_t>(hidden));
  void* ws = AcquireWorkspace(handle, event, ws_bytes);
  if (ws == nullptr) {
    event->complete = true;
    FreeEvent(event);
    return Fail(STATECENTRIC_QWEN38_INTERNAL, "cannot allocate GDN workspace", out_error);
  }
  event->workspace = ws;
  void* stream = reinterpret_cast<void*>(execution->stream);
  int32_t status;
  if (from_x) {
    status = gdn_b200_layer_forward_x(
        reinterpret_cast<const void*>(in[0].data), reinterpret_cast<const void*>(in[1].data),
        reinterpret_cast<const void*>(in[2].data), reinterpret_cast<const void*>(in[3].data),
        reinterpret_cast<const void*>(in[4].data), reinterpret_cast<const void*>(in[5].data),
        reinterpret_cast<void*>(conv->tensor.data), reinterpret_cast<const float*>(in[6].data),
        reinterpret_cast<const float*>(in[7].data), reinterpret_cast<const void*>(in[8].data),
        reinterpret_cast<const void*>(in[9].data),
        reinterpret_cast<float*>(recurrent->tensor.data), reinterpret_cast<void*>(out.data),
        v.cu.data(), nseq, static_cast<int32_t>(hk), static_cast<int32_t>(hv),
        static_cast<int32_t>(hidden), execution->context_tokens != 0 ? 1 : 0, ws, ws_bytes,
        stream);
  } else if (tail_only) {
    status = gdn_b200_output_tail(reinterpret_cast<const void*>(in[0].data),
                                  reinterpret_cast<const void*>(in[1].data),
                                  reinterpret_cast<const void*>(in[2].data),
                                  reinterpret_cast<const void*>(in[3].data),
                                  reinterpret_cast<void*>(out.data), static_cast<int64_t>(tokens),
                                  static_cast<int32_t>(hv), static_cast<int32_t>(hidden), 1.0e-6f,
                                  ws, ws_bytes, stream);
  } else {
    status = gdn_b200_layer_forward(
        reinterpret_cast<const void*>(in[0].data), reinterpret_cast<const void*>(in[1].data),
        reinterpret_cast<const void*>(in[2].data), reinterpret_cast<const void*>(in[3].data),
        reinterpret_cast<const void*>(in[4].data), reinterpret_cast<const void*>(in[5].data),
        reinterpret_cast<const float*>(in[6].data), reinterpret_cast<const float*>(in[7].data),
        reinterpret_cast<const void*>(in[8].data), reinterpret_cast<const void*>(in[9].data),
        reinterpret_cast<float*>(recurrent->tensor.data), reinterpret_cast<void*>(out.data),
        v.cu.data(), nseq, static_cast<int32_t>(hk), static_cast<int32_t>(hv),
        static_cast<int32_t>(hidden), ws, ws_bytes, stream);
  }
  if (status == STATECENTRIC_QWEN38_OK &&
      cudaEventRecord(event->done, event->stream) != cudaSuccess)
    status = STATECENTRIC_QWEN38_INTERNAL;
  if (status != STATECENTRIC_QWEN38_OK) {
    std::string msg = std::string("Qwen3.8 GDN submission failed: ") + gdn_b200_last_error();
    event->complete = cudaStreamSynchronize(event->stream) == cudaSuccess;
    FreeEvent(event);
    return Fail(STATECENTRIC_QWEN38_INTERNAL, msg, out_error);
  }
  handle->submissions.fetch_add(1, std::memory_order_relaxed);
  if (!tail_only)
    RecordAdmission(handle, from_x, plan.core == statecentric::GdnB200Core::kPackedDecode,
                    plan.sequences, plan.rows, plan.chunks);
  *out_event = event;
  return STATECENTRIC_QWEN38_OK;
}

void FillCompletion(statecentric_qwen38_completion_v1* c, uint32_t phase, uint64_t submitted,
                    uint64_t completed) {
  *c = {sizeof(*c), kAbi, phase, 0, completed >= submitted ? completed - submitted : 0, completed};
}

// After completion: surface a device-side error recorded by a kernel.
int32_t CheckDeviceError(statecentric_qwen38_event_v1* event,
                         statecentric_qwen38_error_v1** out_error) {
  uint32_t word = 0;
  if (event->workspace != nullptr &&
      cudaMemcpy(&word, event->workspace, sizeof(word), cudaMemcpyDeviceToHost) != cudaSuccess)
    return Fail(STATECENTRIC_QWEN38_INTERNAL, "cannot read GDN device status", out_error);
  if (word != 0)
    return Fail(STATECENTRIC_QWEN38_INTERNAL,
                "GDN kernel reported device error " + std::to_string(word), out_error);
  return STATECENTRIC_QWEN38_OK;
}

int32_t Poll(statecentric_qwen38_provider_handle_v1* handle, statecentric_qwen38_event_v1* event,
             statecentric_qwen38_completion_v1* completion, statecentric_qwen38_error_v1** out_error) {
  if (handle == nullptr || event == nullptr || completion == nullptr)
    return Fail(STATECENTRIC_QWEN38_INVALID_ARGUMENT, "invalid Qwen3.8 GDN event poll", out_error);
  DeviceGuard guard(handle->device);
  const cudaError_t q = cudaEventQuery(event->done);
  if (q != cudaSuccess && q != cudaErrorNotReady) {
    cudaGetLastError();
    return Fail(STATECENTRIC_QWEN38_INTERNAL,
                std::string("cudaEventQuery(GDN) failed: ") + cudaGetErrorString(q), out_error);
  }
  const uint64_t now = handle->host->monotonic_time_ns(handle->host->context);
  if (q == cudaSuccess) {
    event->complete = true;
    FillCompletion(completion, STATECENTRIC_QWEN38_EVENT_COMPLETE, event->submitted_ns, now);
    return CheckDeviceError(event, out_error);
  }
  FillCompletion(completion, STATECENTRIC_QWEN38_EVENT_PENDING, event->submitted_ns, 0);
  return STATECENTRIC_QWEN38_NOT_READY;
}

// Bounded host wait: polls the completion event until the deadline of the
// host clock passes (the reference converts the deadline into a stream
// synchronisation timeout, P:3598-3629).
int32_t Wait(statecentric_qwen38_provider_handle_v1* handle, statecentric_qwen38_event_v1* event,
             uint64_t deadline_monotonic_ns, statecentric_qwen38_completion_v1* completion,
             statecentric_qwen38_error_v1** out_error) {
  if (handle == nullptr || event == nullptr || completion == nullptr)
    return Fail(STATECENTRIC_QWEN38_INVALID_ARGUMENT, "invalid Qwen3.8 GDN event wait", out_error);
  uint64_t now = handle->host->monotonic_time_ns(handle->host->context);
  if (deadline_monotonic_ns <= now)
    return Fail(STATECENTRIC_QWEN38_TIMEOUT, "Qwen3.8 GDN event deadline expired", out_error);
  DeviceGuard guard(handle->device);
  uint32_t spins = 0;
  while (true) {
    const cudaError_t q = cudaEventQuery(event->done);
    if (q == cudaSuccess) break;
    if (q != cudaErrorNotReady) {
      cudaGetLastError();
      return Fail(STATECENTRIC_QWEN38_INTERNAL,
                  std::string("cudaEventQuery(GDN) failed: ") + cudaGetErrorString(q), out_error);
    }
    now = handle->host->monotonic_time_ns(handle->host->context);
    if (now >= deadline_monotonic_ns)
      return Fail(STATECENTRIC_QWEN38_TIMEOUT, "Qwen3.8 GDN event wait timed out", out_error);
    if (++spins > 64) std::this_thread::sleep_for(std::chrono::microseconds(20));
  }
  event->complete = true;
  const uint64_t completed = handle->host->monotonic_time_ns(handle->host->context);
  FillCompletion(completion, STATECENTRIC_QWEN38_EVENT_COMPLETE, event->submitted_ns, completed);
  return CheckDeviceError(event, out_error);
}

int32_t Cancel(statecentric_qwen38_provider_handle_v1*, statecentric_qwen38_event_v1*,
               statecentric_qwen38_error_v1** out_error) {
  return Fail(STATECENTRIC_QWEN38_UNSUPPORTED,
              "submitted Qwen3.8 GDN work cannot be cancelled safely", out_error);
}

void ReleaseEvent(statecentric_qwen38_provider_handle_v1* handle,
                  statecentric_qwen38_event_v1* event) {
  if (event == nullptr) return;
  DeviceGuard guard(handle != nullptr ? handle->device : 0);
  if (!event->complete) event->complete = cudaEventSynchronize(event->done) == cudaSuccess;
  FreeEvent(event);
}

void ReleaseError(statecentric_qwen38_error_v1* error) {
  delete reinterpret_cast<OwnedError*>(error);
}

}  // namespace

extern "C" int32_t statecentric_qwen38_provider_query_v1(
    uint32_t host_abi_version, uint32_t host_descriptor_size,
    statecentric_qwen38_provider_descriptor_v1* out_descriptor,
    statecentric_qwen38_error_v1** out_error) {
  if (host_abi_version != kAbi ||
      host_descriptor_size < STATECENTRIC_QWEN38_PROVIDER_DESCRIPTOR_V1_MIN_SIZE ||
      out_descriptor == nullptr) {
    return Fail(STATECENTRIC_QWEN38_ABI_MISMATCH, "Qwen3.8 GDN provider query ABI mismatch",
                out_error);
  }
  statecentric_qwen38_provider_descriptor_v1 d{};
  d.size = sizeof(d);
  d.abi_version = kAbi;
  d.provider_id = "org.statecentric.qwen38.gdn";
  d.provider_version = "1.0.0";
  d.operator_name = "operator.qwen38.gdn";
  d.operator_version = 1;
  d.stage = STATECENTRIC_QWEN38_STAGE_GDN;
  d.flags = STATECENTRIC_QWEN38_PROVIDER_FLAG_NO_PYTHON_IPC_V1;
  d.create = Create;
  d.destroy = Destroy;
  d.submit = Submit;
  d.poll = Poll;
  d.wait = Wait;
  d.cancel = Cancel;
  d.release_event = ReleaseEvent;
  d.release_error = ReleaseError;
  const size_t n = std::min<size_t>(host_descriptor_size, sizeof(d));
  std::memcpy(out_descriptor, &d, n);
  return STATECENTRIC_QWEN38_OK;
}
