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
// the array: serialise them.
//
// Host code must not use the array's name as a device address (in host code
// it names a host-side stand-in).  The first call on each device looks up the
// array's device address with cudaGetSymbolAddress while that device is
// current and caches it; make that first call before any stream capture.
#include <cstdio>
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

constexpr int kMaxDevices = 64;
std::mutex g_mutex;
void* g_scratch_ptr[kMaxDevices] = {};

thread_local std::string g_message;

int32_t fail(int32_t status, std::string message) {
  g_message = std::move(message);
  std::fprintf(stderr, "gdn_b200_output_tail_no_alloc: %s\n", g_message.c_str());
  return status;
}

}  // namespace

extern "C" GDN_B200_API int32_t gdn_b200_output_tail_no_alloc(
    const void* o, const void* z, const void* gamma, const void* w_out, void* out, int64_t rows,
    int32_t value_heads, int32_t hidden, float eps, void* stream) {
  const int64_t K = static_cast<int64_t>(value_heads) * GDN_B200_HEAD_DIM;
  if (rows < 0 || value_heads <= 0 || hidden <= 0 || hidden % 128 != 0 || !(eps > 0.0f))
    return fail(STATECENTRIC_QWEN38_INVALID_ARGUMENT,
                "rows, value_heads, hidden (multiple of 128) and eps must be positive");
  if (rows > kMaxRows || K > kMaxK || hidden > kMaxHidden)
    return fail(STATECENTRIC_QWEN38_INVALID_ARGUMENT,
                "size beyond the static scratch: rows <= " + std::to_string(kMaxRows) +
                    ", value_heads*128 <= " + std::to_string(kMaxK) + ", hidden <= " +
                    std::to_string(kMaxHidden));
  if (o == nullptr || z == nullptr || gamma == nullptr || w_out == nullptr || out == nullptr)
    return fail(STATECENTRIC_QWEN38_INVALID_ARGUMENT, "null pointer argument");
  const auto misaligned = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) != 0; };
  if (misaligned(o) || misaligned(z) || misaligned(gamma) || misaligned(w_out) || misaligned(out))
    return fail(STATECENTRIC_QWEN38_INVALID_ARGUMENT, "tensors must be 16-byte aligned");
  const uint64_t partial_bytes = gdn::tail_gemm_workspace_bytes(rows, hidden, static_cast<int>(K));
  if (kErrBytes + kGatedBytes + partial_bytes > kScratchBytes)
    return fail(STATECENTRIC_QWEN38_INVALID_ARGUMENT, "split-K partials exceed the static scratch");

  int device = 0;
  cudaError_t e = cudaGetDevice(&device);
  if (e != cudaSuccess || device < 0 || device >= kMaxDevices)
    return fail(STATECENTRIC_QWEN38_INTERNAL, "cudaGetDevice failed");
  void* base = nullptr;
  {
    std::scoped_lock lock(g_mutex);
    if (g_scratch_ptr[device] == nullptr) {
      void* ptr = nullptr;
      e = cudaGetSymbolAddress(&ptr, g_no_alloc_scratch);
      if (e != cudaSuccess || ptr == nullptr)
        return fail(STATECENTRIC_QWEN38_INTERNAL,
                    std::string("cudaGetSymbolAddress failed: ") + cudaGetErrorString(e));
      g_scratch_ptr[device] = ptr;
    }
    base = g_scratch_ptr[device];
  }
  uint8_t* scratch = static_cast<uint8_t*>(base);
  uint32_t* err = reinterpret_cast<uint32_t*>(scratch);
  uint16_t* gated = reinterpret_cast<uint16_t*>(scratch + kErrBytes);
  float* partials = reinterpret_cast<float*>(scratch + kErrBytes + kGatedBytes);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  e = cudaMemsetAsync(err, 0, sizeof(uint32_t), s);
  if (e != cudaSuccess) return fail(STATECENTRIC_QWEN38_INTERNAL, "cudaMemsetAsync failed");
  if (rows == 0) return STATECENTRIC_QWEN38_OK;
  e = gdn::launch_tail_prologue(static_cast<const uint16_t*>(o), static_cast<const uint16_t*>(z),
                                static_cast<const uint16_t*>(gamma), gated, rows, value_heads,
                                eps, s);
  if (e != cudaSuccess)
    return fail(STATECENTRIC_QWEN38_INTERNAL, std::string("launch: ") + cudaGetErrorString(e));
  e = gdn::launch_tail_gemm(gated, static_cast<const uint16_t*>(w_out), static_cast<uint16_t*>(out),
                            partials, rows, hidden, static_cast<int>(K), err, s,
                            /*overlap_previous=*/true);
  if (e != cudaSuccess)
    return fail(STATECENTRIC_QWEN38_INTERNAL, std::string("launch: ") + cudaGetErrorString(e));
  return STATECENTRIC_QWEN38_OK;
}
