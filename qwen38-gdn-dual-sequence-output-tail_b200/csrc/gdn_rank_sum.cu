// Rank sum of the head-parallel layer's rank-partial outputs, moved by the
// copy engines.
//
// With the value heads split over the ranks, every rank's layer yields a
// partial [rows, hidden] out_proj output; the reference returns it
// (P:3541-3547) and its engine reduces it.  Here every rank ends with its
// row shard of the reduced output (a reduce-scatter):
//   shard_r = bf16( sum over ranks q, in rank order, in f32, of partial_q[rows of r] ).
// The partial rows travel as plain cudaMemcpyAsync peer copies, which run
// on the copy engines over NVLink: no SM takes part in the transfer, so it
// overlaps the next step's kernels almost for free (measured on two B200s:
// 742 GB/s for one 256 MB copy, and the layer step 0.415 -> 0.425 ms while
// 2 GB were copied).  The SMs only run three one-thread flag kernels and
// the summing kernel.
//
// Region of each rank (all offsets 256-byte aligned):
//   part[2]          [max_rows, hidden] bf16: the layer's output of epoch e
//                    goes to part[e & 1]
//   staging[2][W]    [max_rows / W, hidden] bf16: slot q holds the rows of
//                    this rank's shard pulled from rank q
//   flags            ready (epoch of the newest part written here),
//                    pulled[W] (pulled[q] = newest epoch of this rank's part
//                    that rank q has copied out)
// Flags only grow (epochs), so they are never reset; every wait on them is
// bounded (2 s) and records kErrWaitTimeout in the caller's error word.  A
// flag kernel only ever waits for flags that other GPUs write; ordering on
// this GPU (the communication stream after the layer's stream) is a CUDA
// event.
#include <algorithm>
#include <string>

#include "gdn_b200.h"
#include "gdn_common.cuh"
#include "gdn_internal.h"

namespace gdn {
namespace {

struct RankSumLayout {
  uint64_t part_bytes, slot_bytes, shard_rows, staging_off, flags_off, total;
};

uint64_t r256(uint64_t x) { return (x + 255u) & ~uint64_t{255}; }

bool rank_sum_layout(int64_t max_rows, int hidden, int world, RankSumLayout* L) {
  if (max_rows <= 0 || hidden <= 0 || hidden % 8 != 0 || world < 1 || world > kTailMaxRanks ||
      max_rows % world != 0)
    return false;
  L->shard_rows = static_cast<uint64_t>(max_rows / world);
  L->part_bytes = r256(static_cast<uint64_t>(max_rows) * hidden * 2);
  L->slot_bytes = r256(L->shard_rows * hidden * 2);
  L->staging_off = 2 * L->part_bytes;
  L->flags_off = L->staging_off + 2 * static_cast<uint64_t>(world) * L->slot_bytes;
  L->total = L->flags_off + 256;
  return true;
}

struct FlagList {
  uint32_t* flag[kTailMaxRanks];
  int count;
};

// Waits until every listed flag (any rank's memory) has reached `epoch`.
__global__ void rank_flags_wait_kernel(const FlagList flags, uint32_t epoch, uint32_t* err) {
  if (threadIdx.x != 0) return;
  for (int i = 0; i < flags.count; ++i)
    if (!wait_flag_reached(flags.flag[i], epoch, err)) return;
}

// Publishes `epoch` in every listed flag after the earlier work of the stream.
__global__ void rank_flags_set_kernel(const FlagList flags, uint32_t epoch) {
  if (threadIdx.x != 0) return;
  fence_acq_rel_sys();
  for (int i = 0; i < flags.count; ++i) st_release_sys(flags.flag[i], epoch);
}

struct PartList {
  const uint16_t* part[kTailMaxRanks];
  int count;
};

// out = bf16(sum over q of parts[q], in q order, in f32); 8 elements a thread.
__global__ void __launch_bounds__(256) rank_sum_kernel(const PartList parts, uint16_t* out,
                                                       int64_t n8) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n8;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    uint4 v[kTailMaxRanks];
#pragma unroll
    for (int q = 0; q < kTailMaxRanks; ++q)
      if (q < parts.count) v[q] = reinterpret_cast<const uint4*>(parts.part[q])[i];
#pragma unroll
    for (int q = 0; q < kTailMaxRanks; ++q) {
      if (q < parts.count) {
        const uint32_t w[4] = {v[q].x, v[q].y, v[q].z, v[q].w};
#pragma unroll
        for (int p = 0; p < 4; ++p) {
          acc[2 * p] += bf16lo_f32(w[p]);
          acc[2 * p + 1] += bf16hi_f32(w[p]);
        }
      }
    }
    reinterpret_cast<uint4*>(out)[i] =
        make_uint4(pack_bf16x2(acc[0], acc[1]), pack_bf16x2(acc[2], acc[3]),
                   pack_bf16x2(acc[4], acc[5]), pack_bf16x2(acc[6], acc[7]));
  }
}

bool group_ok(const gdn_b200_tail_group_v1* g, RankSumLayout* L) {
  if (g == nullptr || g->reserved != 0 || g->world_size < 1 || g->world_size > kTailMaxRanks ||
      g->rank < 0 || g->rank >= g->world_size)
    return false;
  if (!rank_sum_layout(g->max_rows, g->hidden, g->world_size, L)) return false;
  for (int q = 0; q < g->world_size; ++q)
    if (g->region[q] == nullptr || (reinterpret_cast<uintptr_t>(g->region[q]) & 255u) != 0)
      return false;
  return true;
}

uint8_t* region(const gdn_b200_tail_group_v1* g, int q) { return static_cast<uint8_t*>(g->region[q]); }
uint32_t* flag_ready(const gdn_b200_tail_group_v1* g, const RankSumLayout& L, int q) {
  return reinterpret_cast<uint32_t*>(region(g, q) + L.flags_off);
}
uint32_t* flag_pulled(const gdn_b200_tail_group_v1* g, const RankSumLayout& L, int q, int by) {
  return reinterpret_cast<uint32_t*>(region(g, q) + L.flags_off) + 1 + by;
}

}  // namespace
}  // namespace gdn

extern "C" {

uint64_t gdn_b200_rank_sum_bytes(int64_t max_rows, int32_t hidden, int32_t world_size) {
  gdn::RankSumLayout L;
  return gdn::rank_sum_layout(max_rows, hidden, world_size, &L) ? L.total : 0;
}

void* gdn_b200_rank_sum_part(const gdn_b200_tail_group_v1* group, uint32_t epoch) {
  gdn::RankSumLayout L;
  if (!gdn::group_ok(group, &L) || epoch == 0) return nullptr;
  return gdn::region(group, group->rank) + (epoch & 1u) * L.part_bytes;
}

int32_t gdn_b200_rank_sum_acquire(const gdn_b200_tail_group_v1* group, uint32_t epoch,
                                  uint32_t* err, void* stream) {
  gdn::RankSumLayout L;
  if (!gdn::group_ok(group, &L))
    return gdn::api_fail(STATECENTRIC_QWEN38_INVALID_ARGUMENT, "invalid rank-sum group");
  if (epoch == 0 || err == nullptr)
    return gdn::api_fail(STATECENTRIC_QWEN38_INVALID_ARGUMENT, "epochs start at 1; err is required");
  if (epoch <= 2 || group->world_size == 1) return gdn::api_ok();
  // part[epoch & 1] last held epoch - 2: every other rank must have copied
  // its rows out (their pulled flags live in this rank's region).
  gdn::FlagList f{};
  for (int q = 0; q < group->world_size; ++q)
    if (q != group->rank) f.flag[f.count++] = gdn::flag_pulled(group, L, group->rank, q);
  gdn::rank_flags_wait_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(f, epoch - 2, err);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess)
    return gdn::api_fail(STATECENTRIC_QWEN38_INTERNAL, std::string("launch: ") + cudaGetErrorString(e));
  gdn::note_launches();
  return gdn::api_ok();
}

int32_t gdn_b200_rank_sum(const gdn_b200_tail_group_v1* group, uint32_t epoch, int64_t rows,
                          void* shard_out, uint32_t* err, void* stream, void* comm_stream) {
  gdn::RankSumLayout L;
  if (!gdn::group_ok(group, &L))
    return gdn::api_fail(STATECENTRIC_QWEN38_INVALID_ARGUMENT, "invalid rank-sum group");
  const int W = group->world_size, me = group->rank;
  if (epoch == 0 || err == nullptr || shard_out == nullptr)
    return gdn::api_fail(STATECENTRIC_QWEN38_INVALID_ARGUMENT,
                         "epochs start at 1; err and shard_out are required");
  if (rows < 0 || rows > group->max_rows || rows % W != 0)
    return gdn::api_fail(STATECENTRIC_QWEN38_INVALID_ARGUMENT,
                         "rows must be a multiple of world_size, at most max_rows");
  if ((reinterpret_cast<uintptr_t>(shard_out) & 15u) != 0)
    return gdn::api_fail(STATECENTRIC_QWEN38_INVALID_ARGUMENT, "shard_out must be 16-byte aligned");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaStream_t c = static_cast<cudaStream_t>(comm_stream);
  const uint64_t shard_rows = static_cast<uint64_t>(rows / W);
  const uint64_t shard_bytes = shard_rows * group->hidden * 2;
  const uint32_t b = epoch & 1u;
  const auto launch_check = [](const char* what) -> int32_t {
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess)
      return gdn::api_fail(STATECENTRIC_QWEN38_INTERNAL, std::string(what) + ": " + cudaGetErrorString(e));
    gdn::note_launches();
    return STATECENTRIC_QWEN38_OK;
  };
  int32_t st;
  // 1. The layer of this epoch is done on `stream`: publish this rank's part.
  gdn::FlagList mine{};
  mine.flag[mine.count++] = gdn::flag_ready(group, L, me);
  gdn::rank_flags_set_kernel<<<1, 32, 0, s>>>(mine, epoch);
  if ((st = launch_check("ready flag")) != STATECENTRIC_QWEN38_OK) return st;
  if (W == 1) {
    // One rank: the shard is the whole (already reduced) output.
    const cudaError_t e = cudaMemcpyAsync(shard_out, gdn::region(group, me) + b * L.part_bytes,
                                          shard_bytes, cudaMemcpyDeviceToDevice, s);
    if (e != cudaSuccess)
      return gdn::api_fail(STATECENTRIC_QWEN38_INTERNAL, std::string("copy: ") + cudaGetErrorString(e));
    return gdn::api_ok();
  }
  // 2. On the communication stream: after this rank's own layer (an event:
  // no kernel waits on another kernel of the same GPU), every other rank's
  // part of this epoch...
  {
    cudaEvent_t ev;
    cudaError_t e = cudaEventCreateWithFlags(&ev, cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventRecord(ev, s);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(c, ev, 0);
    cudaEventDestroy(ev);   // released once the recorded work completes
    if (e != cudaSuccess)
      return gdn::api_fail(STATECENTRIC_QWEN38_INTERNAL, std::string("event: ") + cudaGetErrorString(e));
  }
  gdn::FlagList ready{};
  for (int q = 0; q < W; ++q)
    if (q != me) ready.flag[ready.count++] = gdn::flag_ready(group, L, q);
  gdn::rank_flags_wait_kernel<<<1, 32, 0, c>>>(ready, epoch, err);
  if ((st = launch_check("ready wait")) != STATECENTRIC_QWEN38_OK) return st;
  // 3. ...this rank's rows of it, pulled by the copy engines, starting at
  // the next rank: at every point of the sequence each rank's memory serves
  // one puller instead of all of them reading rank 0, then rank 1, ...
  uint8_t* staging = gdn::region(group, me) + L.staging_off + b * W * L.slot_bytes;
  for (int step = 1; step < W; ++step) {
    const int q = (me + step) % W;
    const uint8_t* src = gdn::region(group, q) + b * L.part_bytes +
                         static_cast<uint64_t>(me) * shard_bytes;
    const cudaError_t e = cudaMemcpyAsync(staging + q * L.slot_bytes, src, shard_bytes,
                                          cudaMemcpyDeviceToDevice, c);
    if (e != cudaSuccess)
      return gdn::api_fail(STATECENTRIC_QWEN38_INTERNAL, std::string("peer copy: ") + cudaGetErrorString(e));
  }
  // 4. ...tell every rank its rows are out (they may overwrite that part at
  // epoch + 2)...
  gdn::FlagList pulled{};
  for (int q = 0; q < W; ++q)
    if (q != me) pulled.flag[pulled.count++] = gdn::flag_pulled(group, L, q, me);
  gdn::rank_flags_set_kernel<<<1, 32, 0, c>>>(pulled, epoch);
  if ((st = launch_check("pulled flags")) != STATECENTRIC_QWEN38_OK) return st;
  // 5. ...and sum them in rank order.
  gdn::PartList parts{};
  for (int q = 0; q < W; ++q)
    parts.part[q] = reinterpret_cast<const uint16_t*>(
        q == me ? gdn::region(group, me) + b * L.part_bytes + static_cast<uint64_t>(me) * shard_bytes
                : staging + q * L.slot_bytes);
  parts.count = W;
  const int64_t n8 = static_cast<int64_t>(shard_rows) * group->hidden / 8;
  if (n8 > 0) {
    const int grid = static_cast<int>(std::min<int64_t>((n8 + 255) / 256, 2 * gdn::sm_count()));
    gdn::rank_sum_kernel<<<grid, 256, 0, c>>>(parts, static_cast<uint16_t*>(shard_out), n8);
    if ((st = launch_check("rank sum")) != STATECENTRIC_QWEN38_OK) return st;
  }
  return gdn::api_ok();
}

}  // extern "C"
