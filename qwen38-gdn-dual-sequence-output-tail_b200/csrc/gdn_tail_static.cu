// Output tail for callers that cannot allocate device memory.
//
// gdn_b200_output_tail() needs a caller-provided workspace for the gated
// activations, the split-K partial sums and the device error word.  Some
// callers have no way to provide one: host engines whose operator interface
// hands an operator only its inputs and outputs (no scratch buffer), and
// serving loops that run against a memory plan frozen at start-up, where a
// cudaMalloc (or an allocating library call) after start-up is forbidden or
// would break the plan.  gdn_b200_output_tail_no_alloc() serves them with
// scratch that lives in this file-scope device array instead.
//
// Limits: rows <= 128 (one 2 x 64 dual-sequence tail or up to 128 decode
// rows), value_heads * 128 <= 4096, hidden <= 2048.  The array is
// GDN_B200_NO_ALLOC_SCRATCH_BYTES (17 MiB + 256 B) and every GPU that loads
// the library holds it until the process exits.
//
// Every call on a device shares the one array and it keeps the last call's
// contents; the error word is cleared at each call and everything else is
// fully rewritten before it is read.  Calls whose work overlaps on the GPU
// (different streams, or different host threads using one device) race on
// the array: serialise them.  gdn_b200_output_tail_no_alloc_status() reads
// the error word that the kernels of the last call on the current device
// recorded (a bounded wait that ran out, a failed TMEM allocation).
//
// Host code must not use the array's name as a device address (in host code
// it names a host-side stand-in).  The first call in each CUDA context looks
// up the array's device address with cudaGetSymbolAddress while that
// context's device is current and caches it under the context's unique id,
// so a context created after cudaDeviceReset resolves the address again;
// make that first call before any stream capture.
#include <cmath>
#include <mutex>
#include <string>

#include "gdn_b200.h"
#include "gdn_common.cuh"
#include "gdn_internal.h"

namespace {

constexpr int64_t kMaxRows = GDN_B200_NO_ALLOC_MAX_ROWS;
constexpr int32_t kMaxK = GDN_B200_NO_ALLOC_MAX_VALUE;
constexpr int32_t kMaxHidden = GDN_B200_NO_ALLOC_MAX_HIDDEN;
constexpr uint64_t kErrBytes = 256;
constexpr uint64_t kGatedBytes = static_cast<uint64_t>(kMaxRows) * kMaxK * 2;
constexpr uint64_t kScratchBytes = GDN_B200_NO_ALLOC_SCRATCH_BYTES;

__device__ __align__(256) static uint8_t g_no_alloc_scratch[kScratchBytes];

// The array's device address per CUDA context, keyed by the context's unique
// id (cuCtxGetId: never reused within a process, unlike context handles).
constexpr int kMaxContexts = 64;
struct ContextEntry {
  unsigned long long id;
  void* scratch;
};
std::mutex g_mutex;
ContextEntry g_contexts[kMaxContexts] = {};
int g_num_contexts = 0;

using CtxGetCurrentFn = int (*)(void**);
using CtxGetIdFn = int (*)(void*, unsigned long long*);

// Unique id of the CUDA context current on this host thread.
cudaError_t current_context_id(unsigned long long* id) {
  static CtxGetCurrentFn get_current = nullptr;
  static CtxGetIdFn get_id = nullptr;
  if (get_current == nullptr || get_id == nullptr) {
    void* p1 = nullptr;
    void* p2 = nullptr;
    cudaDriverEntryPointQueryResult q1, q2;
    cudaError_t e = cudaGetDriverEntryPoint("cuCtxGetCurrent", &p1, cudaEnableDefault, &q1);
    if (e != cudaSuccess || q1 != cudaDriverEntryPointSuccess || p1 == nullptr)
      return cudaErrorNotSupported;
    e = cudaGetDriverEntryPoint("cuCtxGetId", &p2, cudaEnableDefault, &q2);
    if (e != cudaSuccess || q2 != cudaDriverEntryPointSuccess || p2 == nullptr)
      return cudaErrorNotSupported;
    get_current = reinterpret_cast<CtxGetCurrentFn>(p1);
    get_id = reinterpret_cast<CtxGetIdFn>(p2);
  }
  void* ctx = nullptr;
  if (get_current(&ctx) != 0) return cudaErrorDeviceUninitialized;
  if (ctx == nullptr) {
    // No context bound to this host thread yet: let the runtime bind the
    // current device's primary context.
    const cudaError_t e = cudaFree(nullptr);
    if (e != cudaSuccess) return e;
    if (get_current(&ctx) != 0 || ctx == nullptr) return cudaErrorDeviceUninitialized;
  }
  if (get_id(ctx, id) != 0) return cudaErrorDeviceUninitialized;
  return cudaSuccess;
}

// The array's device address in the current context; resolved on first use.
// `resolve` false only looks it up (nullptr when no call has run here).
int32_t scratch_address(bool resolve, void** out) {
  unsigned long long id = 0;
  cudaError_t e = current_context_id(&id);
  if (e != cudaSuccess)
    return gdn::api_fail(STATECENTRIC_QWEN38_INTERNAL,
                         std::string("no current CUDA context: ") + cudaGetErrorString(e));
  std::scoped_lock lock(g_mutex);
  for (int i = 0; i < g_num_contexts; ++i) {
    if (g_contexts[i].id == id) {
      *out = g_contexts[i].scratch;
      return STATECENTRIC_QWEN38_OK;
    }
  }
  *out = nullptr;
  if (!resolve) return STATECENTRIC_QWEN38_OK;
  void* ptr = nullptr;
  e = cudaGetSymbolAddress(&ptr, g_no_alloc_scratch);
  if (e != cudaSuccess || ptr == nullptr)
    return gdn::api_fail(STATECENTRIC_QWEN38_INTERNAL,
                         std::string("cudaGetSymbolAddress failed: ") + cudaGetErrorString(e));
  if (g_num_contexts == kMaxContexts) {
    // Oldest entry out: its context is most likely gone.
    for (int i = 1; i < kMaxContexts; ++i) g_contexts[i - 1] = g_contexts[i];
    --g_num_contexts;
  }
  g_contexts[g_num_contexts++] = ContextEntry{id, ptr};
  *out = ptr;
  return STATECENTRIC_QWEN38_OK;
}

}  // namespace

extern "C" GDN_B200_API int32_t gdn_b200_output_tail_no_alloc(
    const void* o, const void* z, const void* gamma, const void* w_out, void* out, int64_t rows,
    int32_t value_heads, int32_t hidden, float eps, void* stream) {
  const int64_t K = static_cast<int64_t>(value_heads) * GDN_B200_HEAD_DIM;
  if (rows < 0 || value_heads <= 0 || hidden <= 0 || hidden % 128 != 0 || !(eps > 0.0f) ||
      !std::isfinite(eps))
    return gdn::api_fail(STATECENTRIC_QWEN38_INVALID_ARGUMENT,
                "rows, value_heads, hidden (multiple of 128) and eps must be positive");
  if (rows > kMaxRows || K > kMaxK || hidden > kMaxHidden)
    return gdn::api_fail(STATECENTRIC_QWEN38_INVALID_ARGUMENT,
                "size beyond the static scratch: rows <= " + std::to_string(kMaxRows) +
                    ", value_heads*128 <= " + std::to_string(kMaxK) + ", hidden <= " +
                    std::to_string(kMaxHidden));
  if (o == nullptr || z == nullptr || gamma == nullptr || w_out == nullptr || out == nullptr)
    return gdn::api_fail(STATECENTRIC_QWEN38_INVALID_ARGUMENT, "null pointer argument");
  const auto misaligned = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) != 0; };
  if (misaligned(o) || misaligned(z) || misaligned(gamma) || misaligned(w_out) || misaligned(out))
    return gdn::api_fail(STATECENTRIC_QWEN38_INVALID_ARGUMENT, "tensors must be 16-byte aligned");
  const uint64_t partial_bytes = gdn::tail_gemm_workspace_bytes(rows, hidden, static_cast<int>(K));
  if (kErrBytes + kGatedBytes + partial_bytes > kScratchBytes)
    return gdn::api_fail(STATECENTRIC_QWEN38_INVALID_ARGUMENT, "split-K partials exceed the static scratch");

  void* base = nullptr;
  const int32_t st = scratch_address(/*resolve=*/true, &base);
  if (st != STATECENTRIC_QWEN38_OK) return st;
  uint8_t* scratch = static_cast<uint8_t*>(base);
  uint32_t* err = reinterpret_cast<uint32_t*>(scratch);
  uint16_t* gated = reinterpret_cast<uint16_t*>(scratch + kErrBytes);
  float* partials = reinterpret_cast<float*>(scratch + kErrBytes + kGatedBytes);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemsetAsync(err, 0, sizeof(uint32_t), s);
  if (e != cudaSuccess) return gdn::api_fail(STATECENTRIC_QWEN38_INTERNAL, "cudaMemsetAsync failed");
  if (rows == 0) return gdn::api_ok();
  e = gdn::launch_tail_prologue(static_cast<const uint16_t*>(o), static_cast<const uint16_t*>(z),
                                static_cast<const uint16_t*>(gamma), gated, rows, value_heads,
                                eps, s);
  if (e != cudaSuccess)
    return gdn::api_fail(STATECENTRIC_QWEN38_INTERNAL, std::string("launch: ") + cudaGetErrorString(e));
  e = gdn::launch_tail_gemm(gated, static_cast<const uint16_t*>(w_out), static_cast<uint16_t*>(out),
                            partials, rows, hidden, static_cast<int>(K), err, s,
                            /*overlap_previous=*/true);
  if (e != cudaSuccess)
    return gdn::api_fail(STATECENTRIC_QWEN38_INTERNAL, std::string("launch: ") + cudaGetErrorString(e));
  return gdn::api_ok();
}

extern "C" GDN_B200_API int32_t gdn_b200_output_tail_no_alloc_status(void* stream) {
  void* base = nullptr;
  const int32_t st = scratch_address(/*resolve=*/false, &base);
  if (st != STATECENTRIC_QWEN38_OK) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (base == nullptr) {
    // No call has run in this context: nothing can have failed.
    const cudaError_t e = cudaStreamSynchronize(s);
    if (e != cudaSuccess)
      return gdn::api_fail(STATECENTRIC_QWEN38_INTERNAL,
                           std::string("cudaStreamSynchronize: ") + cudaGetErrorString(e));
    return gdn::api_ok();
  }
  return gdn::read_error_word(base, s);
}
