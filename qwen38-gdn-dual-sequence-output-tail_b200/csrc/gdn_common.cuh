// Shared device helpers for the sm_100a GDN kernels: bf16 conversion,
// mbarriers with bounded waits, TMA, and tcgen05 (UMMA + TMEM) wrappers.
//
// Every spin in this library is bounded by a wall-clock limit read from
// %globaltimer.  A wait that runs out records an error code in the error
// word the kernel was given and returns false; the caller then skips the
// rest of its work, releases TMEM and exits, so a malformed launch ends with
// an error status on the host instead of a hung GPU.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace gdn {

constexpr int kHeadDim = 128;
constexpr int kChunk = 64;
constexpr unsigned long long kWaitLimitNs = 2000000000ull;  // 2 s

// Error codes written to the per-launch error word.
enum : uint32_t {
  kErrNone = 0,
  kErrWaitTimeout = 1,
  kErrTmemAlloc = 2,
  kErrBadGeometry = 3,
  kErrMisaligned = 4,   // a device-side address (a state row) not 16-byte aligned
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void record_error(uint32_t* err, uint32_t code) {
  if (err != nullptr) atomicCAS(err, 0u, code);
}

// ------------------------------------------------- cross-GPU signalling --
// Flags that live in one GPU's memory and are written by another GPU over an
// NVLink mapping.  A writer makes its earlier stores visible with a
// system-scope release; a reader acquires the flag before it reads the data.
// Flags carry a call epoch that only grows, so they are never reset.

__device__ __forceinline__ void fence_acq_rel_sys() {
  asm volatile("fence.acq_rel.sys;" ::: "memory");
}
__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
// Orders this thread's earlier generic-proxy accesses of global memory
// before its later TMA (async-proxy) reads.
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}
__device__ __forceinline__ void named_barrier_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// Programmatic dependent launch.  A kernel launched with programmatic stream
// serialization may start while the previous kernel on its stream still
// runs; griddep_wait() returns once that kernel has completed and its
// writes are visible (a no-op for an ordinary launch).
// griddep_launch_dependents() lets such a next kernel start early.
__device__ __forceinline__ void griddep_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void griddep_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Waits until the flag has reached `epoch` (wrap-safe comparison), bounded
// by the same wall-clock limit as every other wait; on expiry records
// kErrWaitTimeout and returns false.
__device__ __forceinline__ bool wait_flag_reached(const uint32_t* flag, uint32_t epoch,
                                                  uint32_t* err) {
  if (static_cast<int32_t>(ld_acquire_sys(flag) - epoch) >= 0) return true;
  const unsigned long long start = global_ns();
  for (uint32_t poll = 1;; ++poll) {
    if (static_cast<int32_t>(ld_acquire_sys(flag) - epoch) >= 0) return true;
    if ((poll & 15u) == 0u) {
      if (global_ns() - start > kWaitLimitNs) {
        record_error(err, kErrWaitTimeout);
        return false;
      }
      if (err != nullptr && *reinterpret_cast<volatile uint32_t*>(err) != 0) return false;
    }
    __nanosleep(40);
  }
}

// ------------------------------------------------------------- bf16 -----

__device__ __forceinline__ float bf16_bits_to_f32(uint16_t h) {
  return __uint_as_float(static_cast<uint32_t>(h) << 16);
}
__device__ __forceinline__ uint16_t f32_to_bf16_bits(float f) {
  return __bfloat16_as_ushort(__float2bfloat16_rn(f));
}
// Round to the nearest bf16 value (ties to even), result as f32.  Integer
// arithmetic keeps this off the transcendental/conversion pipe; inputs are
// finite (NaN payloads are not preserved).
__device__ __forceinline__ float round_bf16(float f) {
  uint32_t u = __float_as_uint(f);
  u += 0x7FFFu + ((u >> 16) & 1u);
  return __uint_as_float(u & 0xFFFF0000u);
}
// Two floats -> packed bf16x2 (round to nearest even; low half = first),
// one cvt.rn.bf16x2.f32.
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}
// Low / high bf16 of a packed pair, as f32.
__device__ __forceinline__ float bf16lo_f32(uint32_t p) { return __uint_as_float(p << 16); }
__device__ __forceinline__ float bf16hi_f32(uint32_t p) { return __uint_as_float(p & 0xFFFF0000u); }
// x ~= hi + lo with hi = bf16(x), lo = bf16(x - hi): two bf16 operands that
// carry about 16 mantissa bits of x.  Returns packed (hi0,hi1) and (lo0,lo1).
__device__ __forceinline__ void split_bf16x2(float x0, float x1, uint32_t& hi, uint32_t& lo) {
  hi = pack_bf16x2(x0, x1);
  lo = pack_bf16x2(x0 - bf16lo_f32(hi), x1 - bf16hi_f32(hi));
}

// ------------------------------------------------- output-tail gating -----
// The output tail's gate for eight elements of one (row, head) pair, the
// reference's RmsNorm -> Silu -> Mul operator chain with a bf16 rounding at
// each operator boundary (P:1443-1497):
//   gated = bf16( bf16(o * rstd * gamma) * bf16(SiLU(z)) ).
// Sixteen consecutive lanes hold the 128 elements of a pair (8 each):
// gate_sumsq16 returns the pair's sum of o^2 in every one of those lanes.
__device__ __forceinline__ float gate_sumsq16(const uint32_t (&ow)[4]) {
  float ss = 0.f;
#pragma unroll
  for (int p = 0; p < 4; ++p) {
    const float x0 = bf16lo_f32(ow[p]), x1 = bf16hi_f32(ow[p]);
    ss += x0 * x0 + x1 * x1;
  }
#pragma unroll
  for (int off = 8; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
  return ss;
}
__device__ __forceinline__ uint4 gate8(const uint32_t (&ow)[4], const uint32_t (&zw)[4],
                                       const uint32_t (&gw)[4], float rstd) {
  uint32_t res[4];
#pragma unroll
  for (int p = 0; p < 4; ++p) {
    float r2[2];
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const float x = e ? bf16hi_f32(ow[p]) : bf16lo_f32(ow[p]);
      const float zz = e ? bf16hi_f32(zw[p]) : bf16lo_f32(zw[p]);
      const float gg = e ? bf16hi_f32(gw[p]) : bf16lo_f32(gw[p]);
      const float nrm = round_bf16(x * rstd * gg);
      const float sl = round_bf16(__fdividef(zz, 1.0f + __expf(-zz)));
      r2[e] = nrm * sl;
    }
    res[p] = pack_bf16x2(r2[0], r2[1]);
  }
  return make_uint4(res[0], res[1], res[2], res[3]);
}

// Packed f32x2 arithmetic (one instruction for two IEEE fp32 lanes).
__device__ __forceinline__ unsigned long long f2_pack(float2 v) {
  unsigned long long r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(v.x), "f"(v.y));
  return r;
}
__device__ __forceinline__ float2 f2_unpack(unsigned long long r) {
  float2 v;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(v.x), "=f"(v.y) : "l"(r));
  return v;
}
// a * b + c per lane, rounded once (fma.rn).
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
  unsigned long long d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(f2_pack(a)), "l"(f2_pack(b)), "l"(f2_pack(c)));
  return f2_unpack(d);
}

// a * b per lane, rounded (mul.rn).
__device__ __forceinline__ float2 fmul2(float2 a, float2 b) {
  unsigned long long d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(f2_pack(a)), "l"(f2_pack(b)));
  return f2_unpack(d);
}
// The two bf16 halves of a packed word as an f32 pair (low element first).
__device__ __forceinline__ float2 bf16x2_f32x2(uint32_t w) {
  return make_float2(bf16lo_f32(w), bf16hi_f32(w));
}

// ---------------------------------------------------------- mbarrier -----

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait on a phase parity.  Returns false (and records the error) when
// the limit runs out or another thread of the launch already failed.
// The clock and the launch's error word (a global load of several hundred
// cycles) are read once every 64 polls only, so a phase that completes is
// seen within one poll instead of behind that load.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint32_t* err) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long start = global_ns();
  for (uint32_t poll = 1;; ++poll) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((poll & 63u) == 0u) {
      if (global_ns() - start > kWaitLimitNs) {
        record_error(err, kErrWaitTimeout);
        return false;
      }
      if (err != nullptr && *reinterpret_cast<volatile uint32_t*>(err) != 0) return false;
    }
  }
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
// Orders generic-proxy shared-memory writes before async-proxy reads
// (tcgen05.mma operands, TMA stores).
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// -------------------------------------------------------------- TMA ------

__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// 2-D tiled bulk tensor load into this CTA's own shared memory.
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* map,
                                            uint64_t* bar, int32_t c0, int32_t c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}

// 3-D tiled bulk tensor load into this CTA's own shared memory.
__device__ __forceinline__ void tma_load_3d(void* smem_dst, const CUtensorMap* map,
                                            uint64_t* bar, int32_t c0, int32_t c1, int32_t c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

// Prefetch into L2 (no shared memory involved): a byte range, or a tensor
// box.  Sizes are multiples of 16 bytes.
__device__ __forceinline__ void prefetch_l2(const void* gmem, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(reinterpret_cast<uint64_t>(gmem)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void prefetch_l2_3d(const CUtensorMap* map, int32_t c0, int32_t c1,
                                               int32_t c2) {
  asm volatile("cp.async.bulk.prefetch.tensor.3d.L2.global [%0, {%1, %2, %3}];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(c0), "r"(c1), "r"(c2)
               : "memory");
}

// 1-D bulk copy shared -> global, tracked by the issuing thread's bulk
// groups.  Both addresses 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_store(void* gmem_dst, const void* smem_src, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(
                   reinterpret_cast<uint64_t>(gmem_dst)),
               "r"(smem_u32(smem_src)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
// Waits until at most N of this thread's committed bulk groups still read
// their shared-memory source.
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
// Waits until at most N of this thread's committed bulk groups are still
// incomplete (their writes not yet performed).
template <int N>
__device__ __forceinline__ void bulk_wait() {
  asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}
// Waits until every committed bulk group of this thread has completed.
__device__ __forceinline__ void bulk_wait_all() {
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

// 1-D bulk copy global -> this CTA's own shared memory.  Both
// addresses 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_load(void* smem_dst, const void* gmem_src, uint32_t bytes,
                                          uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(gmem_src)), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Address of the same shared-memory location in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t cluster_map(uint32_t local_addr, uint32_t rank) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(local_addr), "r"(rank));
  return remote;
}

// 1-D bulk copy from this CTA's shared memory into another CTA's shared
// memory in the cluster; completion is counted as transaction bytes on the
// destination's mbarrier (remote_bar, a cluster address).  Addresses
// 16-byte aligned, bytes a multiple of 16.  The source must stay unchanged
// until the destination has seen the bytes arrive.
__device__ __forceinline__ void bulk_push_cluster(uint32_t remote_dst, const void* smem_src,
                                                  uint32_t bytes, uint32_t remote_bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, "
      "[%3];" ::"r"(remote_dst),
      "r"(smem_u32(smem_src)), "r"(bytes), "r"(remote_bar)
      : "memory");
}

// ------------------------------------------------------------ tcgen05 ----

// UMMA shared-memory matrix descriptor (sm_100 layout: start >> 4 in [0,14),
// LBO >> 4 in [16,30), SBO >> 4 in [32,46), version 1 in [46,48),
// layout type in [61,64); 2 = 128-byte swizzle).
__device__ __forceinline__ uint64_t umma_sdesc_layout(uint32_t smem_addr, uint32_t lbo_bytes,
                                                      uint32_t sbo_bytes, uint32_t layout) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr & 0x3FFFFu) >> 4);
  d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(layout & 7u) << 61;
  return d;
}
__device__ __forceinline__ uint64_t umma_sdesc(uint32_t smem_addr, uint32_t lbo_bytes,
                                               uint32_t sbo_bytes) {
  return umma_sdesc_layout(smem_addr, lbo_bytes, sbo_bytes, 2u);
}
// 64-byte-swizzled operand (layout type 4), see sw64_chunk.
__device__ __forceinline__ uint64_t umma_sdesc_sw64(uint32_t smem_addr, uint32_t lbo_bytes,
                                                    uint32_t sbo_bytes) {
  return umma_sdesc_layout(smem_addr, lbo_bytes, sbo_bytes, 4u);
}

// Instruction descriptor, kind::f16 with bf16 A/B and f32 accumulator.
// a_mn / b_mn select MN-major operands (bit 15 / 16).
__host__ __device__ constexpr uint32_t umma_idesc_bf16(int m, int n, bool a_mn, bool b_mn) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((a_mn ? 1u : 0u) << 15) |
         ((b_mn ? 1u : 0u) << 16) | ((static_cast<uint32_t>(n) >> 3) << 17) |
         ((static_cast<uint32_t>(m) >> 4) << 24);
}

__device__ __forceinline__ void umma_bf16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                          uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrives on `bar` once every tcgen05 operation issued so far by this
// thread has completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tmem_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tmem_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Whole-warp TMEM allocation; the column base is written to *dst_smem.
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

// Warp-wide TMEM load: lane i of the warp reads TMEM lane (taddr.lane + i),
// 16 consecutive 32-bit columns starting at taddr.column.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// TMEM address of (lane, column) relative to a column base.
__device__ __forceinline__ uint32_t tmem_addr(uint32_t base, uint32_t lane, uint32_t col) {
  return base + (lane << 16) + col;
}

// ------------------------------------------------- operand smem layouts --
// 128-byte-swizzled canonical layouts used for every UMMA operand here.
// A 1024-byte atom holds 8 rows of 128 bytes (64 bf16); within the atom the
// 16-byte chunk c of row r sits at chunk position c ^ r.  Atoms must start on
// a 1024-byte boundary.
//
// K-major operand of R rows (M or N) and K columns: 64-column slabs of
// R * 128 bytes, slab s at s * R * 128; descriptor LBO = 16, SBO = 1024; the
// K step of 16 elements adds 32 bytes inside a slab.
__device__ __forceinline__ uint32_t kmajor_offset(uint32_t row, uint32_t col, uint32_t rows) {
  const uint32_t slab = col >> 6;
  const uint32_t c = col & 63u;
  return slab * rows * 128u + (row >> 3) * 1024u + (row & 7u) * 128u +
         ((((c >> 3) ^ (row & 7u)) & 7u) << 4) + (c & 7u) * 2u;
}
// MN-major operand: K rows of 64-element MN slabs.  Element (k, mn) of an
// operand with K extent kext: slab (mn / 64) at slab * kext * 128, row k at
// (k / 8) * 1024 + (k % 8) * 128; descriptor LBO = kext * 128 (slab stride),
// SBO = 1024; the K step of 16 rows adds 2048 bytes.
__device__ __forceinline__ uint32_t mnmajor_offset(uint32_t k, uint32_t mn, uint32_t kext) {
  const uint32_t slab = mn >> 6;
  const uint32_t c = mn & 63u;
  return slab * kext * 128u + (k >> 3) * 1024u + (k & 7u) * 128u +
         ((((c >> 3) ^ (k & 7u)) & 7u) << 4) + (c & 7u) * 2u;
}
// Byte offset of the 16-byte chunk holding elements [8j, 8j+8) of row `row`
// in one 128-byte-swizzled slab (same formula for both majors).
__device__ __forceinline__ uint32_t sw128_chunk(uint32_t row, uint32_t j) {
  return (row >> 3) * 1024u + (row & 7u) * 128u + (((j ^ row) & 7u) << 4);
}
// 64-byte-swizzled MN-major operand of 32-element (64-byte) K rows: a
// 512-byte atom holds 8 rows and the 16-byte chunk j (0..3) of row r sits at
// chunk position j ^ ((r / 2) % 4), i.e. address bits [4,6) XOR bits [7,9).
// Atoms start on a 512-byte boundary; descriptor SBO = 512 (8 K rows), the
// K step of 16 rows adds 1024 bytes.
__device__ __forceinline__ uint32_t sw64_chunk(uint32_t row, uint32_t j) {
  return row * 64u + (((j ^ (row >> 1)) & 3u) << 4);
}

}  // namespace gdn
