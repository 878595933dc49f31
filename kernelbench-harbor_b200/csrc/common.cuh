// Shared device/host plumbing for the b200q kernels (sm_100a only).
//
//  * mbarrier / TMA (cp.async.bulk.tensor) wrappers written as inline PTX;
//  * bounded waits: every spin on an mbarrier gives up after B200Q_WAIT_NS
//    nanoseconds of %globaltimer, records B200Q_DEV_ERR_TIMEOUT in the
//    caller-visible status word and returns false -- no trap, no endless loop;
//  * tensor-map encoding through the driver entry point (no libcuda link);
//  * the thread-local last-error string behind b200q_last_error().
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <cudaTypedefs.h>
#include <stdint.h>
#include <string>

#include "b200q.h"

#ifndef B200Q_WAIT_SLEEP_NS
#define B200Q_WAIT_SLEEP_NS 100000  // suspend-time hint of mbarrier waits in ns (0: plain polling)
#endif
#ifndef B200Q_WAIT_BACKOFF_NS
#define B200Q_WAIT_BACKOFF_NS 0  // sleep between unsuccessful polls in ns (0: none)
#endif
#ifndef B200Q_WAIT_NS
#define B200Q_WAIT_NS 2000000000ull  // 2 s: far above any legitimate wait in these kernels
#endif

// device status bits (or-ed into the workspace status word)
#define B200Q_DEV_ERR_TIMEOUT 1
#define B200Q_DEV_ERR_BOUNDS 2

namespace b200q {

// Output destinations of a GEMM: the same [M, N] tile is stored into every
// y[i] at row stride ldy, column offset col0 (elements).  One destination with
// ldy = N, col0 = 0 is a plain GEMM; the column-sharded multi-GPU GEMM passes
// every rank's full [M, ldy] output (peer pointers over NVLink), so its
// epilogue is also the all-gather.
constexpr int MAX_PEERS = 8;

// Rows from which the W4A16 tensor-core (tcgen05) path is used; fewer rows
// take the mma.sync decode kernel.
constexpr int64_t W4A16_TC_MIN_M = 17;
//
// With world > 1 the kernel also orders itself against the other ranks
// through their signal pads (64 uint32 words per rank, zero-initialised,
// every rank's mapped into each process), so that no separate barrier kernel
// is needed:
//   pad words [0, 8)   arrival epoch of call c from rank p (word p)
//   pad words [8, 16)  completion epoch of call c from rank p (word 8 + p)
//   pad word  62       ticket: CTAs of this rank's current call that finished
//   pad word  63       calls this rank completed (its epoch counter)
// At start one thread tells every peer "I am at call c+1" (this rank is done
// reading its previous output); before its first peer store each CTA waits
// until every peer is at call c+1; the last CTA to finish bumps the counter,
// tells every peer "call c+1 complete" and waits for theirs.  All waits are
// bounded.
struct OutSet {
  void* y[MAX_PEERS];
  uint32_t* pad[MAX_PEERS];
  int n;
  int ldy;
  int col0;
  int world;  // 0 or 1: no cross-rank ordering
  int rank;
};

constexpr int PAD_ARRIVE = 0, PAD_DONE = 8, PAD_BARRIER = 16, PAD_BARRIER_COUNT = 61, PAD_TICKET = 62,
              PAD_COUNT = 63, PAD_WORDS = 64;

inline OutSet single_out(void* y, int64_t N) {
  OutSet o = {};
  o.y[0] = y;
  o.n = 1;
  o.ldy = (int)N;
  o.col0 = 0;
  return o;
}

// ------------------------------------------------------------------ host side errors
void set_error(const std::string& msg);
int fail(int code, const std::string& msg);
int check_cuda(cudaError_t e, const char* what);
int num_sms(int device);
// b200q_set_weight_prefetch: whether small-M kernels may stream their weights
// before the programmatic-dependent-launch wait
bool weight_prefetch_enabled();
int current_device();

// encodes a 2D tiled tensor map; returns 0 or a negative b200q status
int encode_2d(CUtensorMap* map, CUtensorMapDataType dt, const void* base, uint64_t inner,
              uint64_t outer, uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer,
              CUtensorMapSwizzle swz);
// 3D variant (inner, mid, outer) used for batched / expert-indexed operands
int encode_3d(CUtensorMap* map, CUtensorMapDataType dt, const void* base, uint64_t d0,
              uint64_t d1, uint64_t d2, uint64_t stride1_bytes, uint64_t stride2_bytes,
              uint32_t b0, uint32_t b1, uint32_t b2, CUtensorMapSwizzle swz);

// ------------------------------------------------------------------ device helpers
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// The dynamic shared-memory base rounded up to 1024 bytes by pointer
// arithmetic on the __shared__ array itself (not through an integer), so the
// compiler still knows the result points into shared memory and emits
// shared-memory loads and stores for accesses through it, not generic ones.
__device__ __forceinline__ uint8_t* align_smem_1024(uint8_t* raw) {
  return raw + ((1024u - (smem_u32(raw) & 1023u)) & 1023u);
}

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

#ifndef B200Q_PEER_WAIT_NS
#define B200Q_PEER_WAIT_NS 10000000000ull  // 10 s: ranks may legitimately arrive seconds apart
#endif

__device__ __forceinline__ void st_release_sys(uint32_t* a, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(a), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* a) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(a) : "memory");
  return v;
}

__device__ __forceinline__ uint32_t ld_volatile(const uint32_t* a) {
  uint32_t v;
  asm volatile("ld.volatile.global.u32 %0, [%1];" : "=r"(v) : "l"(a) : "memory");
  return v;
}

// Waits until (int)(*a - target) >= 0 (wrap-safe epochs); false after
// B200Q_PEER_WAIT_NS.
__device__ __forceinline__ bool wait_epoch(const uint32_t* a, uint32_t target,
                                           uint64_t limit_ns = B200Q_PEER_WAIT_NS) {
  const uint64_t t0 = globaltimer();
  for (uint32_t it = 0;; ++it) {
    if ((int)(ld_acquire_sys(a) - target) >= 0) return true;
    if ((it & 63) == 63 && globaltimer() - t0 > limit_ns) return false;
    __nanosleep(32);
  }
}

__device__ __forceinline__ void st_relaxed_sys(uint32_t* a, uint32_t v) {
  asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(a), "r"(v) : "memory");
}

// One thread: announce "at call c+1" to every peer.  Nothing this kernel
// wrote needs ordering before it (the previous calls' reads of the output
// ended with their kernels), so plain relaxed stores do: no fence.
__device__ __forceinline__ void peer_arrive(const OutSet& o) {
  if (o.world <= 1) return;
  const uint32_t e = ld_volatile(o.pad[o.rank] + PAD_COUNT) + 1;
  for (int p = 0; p < o.world; ++p)
    if (p != o.rank) st_relaxed_sys(o.pad[p] + PAD_ARRIVE + o.rank, e);
}

// One thread, before the CTA's first store into a peer's output: every peer
// is at call c+1.  Sets the timeout bit in *status and returns false on timeout.
__device__ __forceinline__ bool peer_wait_arrivals(const OutSet& o, int* status) {
  if (o.world <= 1) return true;
  const uint32_t e = ld_volatile(o.pad[o.rank] + PAD_COUNT) + 1;
  for (int p = 0; p < o.world; ++p)
    if (p != o.rank && !wait_epoch(o.pad[o.rank] + PAD_ARRIVE + p, e)) {
      atomicOr(status, B200Q_DEV_ERR_TIMEOUT);
      return false;
    }
  return true;
}

// Warp 0 of every CTA, after all of the CTA's stores (behind a CTA barrier).
// Each CTA releases its stores at GPU scope into the ticket; the last CTA of
// the grid (whose acquire of the ticket makes every CTA's stores precede it)
// publishes "call c+1 complete" to every peer with a system-scope release,
// one lane per peer, and waits for the peers' completions.
__device__ __forceinline__ void peer_finish(const OutSet& o, int* status) {
  if (o.world <= 1) return;
  const int lane = threadIdx.x & 31;
  uint32_t last = 0, e = 0;
  if (lane == 0) {
    const uint32_t total = gridDim.x * gridDim.y * gridDim.z;
    uint32_t t;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(t) : "l"(o.pad[o.rank] + PAD_TICKET) : "memory");
    if (t == total - 1) {
      last = 1;
      o.pad[o.rank][PAD_TICKET] = 0;
      e = ld_volatile(o.pad[o.rank] + PAD_COUNT) + 1;
      o.pad[o.rank][PAD_COUNT] = e;
    }
  }
  last = __shfl_sync(0xffffffffu, last, 0);
  if (!last) return;
  e = __shfl_sync(0xffffffffu, e, 0);
  if (lane < o.world && lane != o.rank) {
    st_release_sys(o.pad[lane] + PAD_DONE + o.rank, e);
    if (!wait_epoch(o.pad[o.rank] + PAD_DONE + lane, e)) atomicOr(status, B200Q_DEV_ERR_TIMEOUT);
  }
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
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

// try_wait with a suspend-time hint: the thread sleeps in hardware until the
// phase completes or about `ns` nanoseconds pass (it does not spin).
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity, uint32_t ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(ns)
      : "memory");
  return ok != 0;
}

// Waits for phase `parity` of `bar` to complete.  Gives up after B200Q_WAIT_NS,
// or-ing B200Q_DEV_ERR_TIMEOUT into *status (when non-null); returns false then.
// The wall clock (%globaltimer, a slow special-register read) is consulted only
// once per 64 unsuccessful polls, so waiting warps do not load the pipes that
// working warps need.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* status) {
  if (mbar_try_wait(bar, parity)) return true;
  uint64_t t0 = 0;
  for (uint32_t i = 0;; ++i) {
#if B200Q_WAIT_SLEEP_NS > 0
    if (mbar_try_wait_sleep(bar, parity, B200Q_WAIT_SLEEP_NS)) return true;
#else
    if (mbar_try_wait(bar, parity)) return true;
#endif
#if B200Q_WAIT_BACKOFF_NS > 0
    __nanosleep(B200Q_WAIT_BACKOFF_NS);
#endif
    if ((i & 63) == 0) {
      const uint64_t t = globaltimer();
      if (i == 0) {
        t0 = t;
      } else if (t - t0 > B200Q_WAIT_NS) {
        if (status) atomicOr(status, B200Q_DEV_ERR_TIMEOUT);
        return false;
      }
    }
  }
}

__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* m) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(m)) : "memory");
}

// 2D tiled TMA load into shared memory, completion counted on `bar` (bytes).
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* m, int c0, int c1,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(c0), "r"(c1), "r"(smem_u32(bar))
      : "memory");
}

// Contiguous global -> shared copy of `bytes` (a multiple of 16, both
// addresses 16-byte aligned) by the bulk-copy engine, completion counted on
// `bar`.  No multicast.
__device__ __forceinline__ void bulk_load(void* smem_dst, const void* gsrc, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(gsrc)), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Orders this thread's earlier generic-proxy view of global memory (data
// another CTA published) before its later async-proxy (bulk copy) reads.
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

// Same with an L2 eviction-priority hint (createpolicy result).
__device__ __forceinline__ void tma_load_2d_hint(void* smem_dst, const CUtensorMap* m, int c0, int c1,
                                                 uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(c0), "r"(c1), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

__device__ __forceinline__ void tma_load_3d(void* smem_dst, const CUtensorMap* m, int c0, int c1, int c2,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

__device__ __forceinline__ uint64_t policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
  return r;
}

// (a & mask) | bits in one LOP3
__device__ __forceinline__ uint32_t and_or(uint32_t a, uint32_t mask, uint32_t bits) {
  uint32_t r;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r) : "r"(a), "r"(mask), "r"(bits));
  return r;
}

// Hardware named barrier `id` (1..15) over `threads` threads (a multiple of 32).
__device__ __forceinline__ void named_barrier_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

__device__ __forceinline__ uint32_t elect_one_sync() {
  uint32_t pred = 0;
  asm volatile(
      "{\n\t.reg .b32 %%rx;\n\t.reg .pred %%px;\n\t"
      "elect.sync %%rx|%%px, %1;\n\t"
      "@%%px mov.s32 %0, 1;\n\t}"
      : "+r"(pred)
      : "r"(0xffffffffu));
  return pred;
}

}  // namespace b200q

// ------------------------------------------------------------------ tcgen05 (5th-gen tensor core) helpers
namespace b200q {

// Shared-memory matrix descriptor (sm_100 format): start address, leading /
// stride byte offsets (16-byte units), version 1, swizzle mode in bits 61..63
// (2 = 128-byte swizzle).  Buffers are 1024-byte aligned, so base offset 0.
__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes,
                                              uint32_t swizzle_mode) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFF) << 32;
  d |= (uint64_t)1 << 46;  // descriptor version for sm_100
  d |= (uint64_t)(swizzle_mode & 7) << 61;
  return d;
}

// Instruction descriptor for kind::f16 with fp32 accumulation.
// ab_fmt: 0 = fp16, 1 = bf16.  a_mn / b_mn: operand is MN-major (1) or K-major (0).
__host__ __device__ constexpr uint32_t idesc_f16(int M, int N, int ab_fmt, int a_mn, int b_mn) {
  return (1u << 4) | ((uint32_t)ab_fmt << 7) | ((uint32_t)ab_fmt << 10) | ((uint32_t)a_mn << 15) |
         ((uint32_t)b_mn << 16) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void tc_mma_f16_ss(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                              uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrives once on `bar` when every tcgen05.mma issued so far by this thread has completed.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Whole-warp TMEM allocation; the base address is written to *dst (shared).
__device__ __forceinline__ void tmem_alloc(uint32_t* dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns (one register per column).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
        "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),
        "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]),
        "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
// 32 lanes x 16 consecutive columns
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, "
      "[%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
        "=r"(r[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

}  // namespace b200q

namespace b200q {
// Instruction descriptor for kind::i8 (signed int8 x signed int8 -> int32).
__host__ __device__ constexpr uint32_t idesc_i8(int M, int N, int a_mn, int b_mn) {
  return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)a_mn << 15) | ((uint32_t)b_mn << 16) |
         ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void tc_mma_i8_ss(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                             uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
}  // namespace b200q

namespace b200q {
// Instruction descriptor for kind::mxf8f6f4.block_scale, e4m3 x e4m3, E8M0
// scales (one per 32 K), K = 32 per instruction; a_sf / b_sf select the byte of
// the 32-bit scale-factor TMEM column this instruction reads.
__host__ __device__ constexpr uint32_t idesc_mxf8(int M, int N, int a_sf, int b_sf) {
  return ((uint32_t)b_sf << 4) | (0u << 7) | (0u << 10) | ((uint32_t)(N >> 3) << 17) | (1u << 23) |
         ((uint32_t)(M >> 4) << 24) | ((uint32_t)a_sf << 29);
}

__device__ __forceinline__ void tc_mma_mxf8_ss(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                               uint32_t sfa_tmem, uint32_t sfb_tmem, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(sfa_tmem), "r"(sfb_tmem)
      : "memory");
}

// 32 lanes x 4 / 8 consecutive 32-bit columns from registers
__device__ __forceinline__ void tmem_st4(uint32_t taddr, const uint32_t* r) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1,%2,%3,%4};" ::"r"(taddr), "r"(r[0]), "r"(r[1]),
               "r"(r[2]), "r"(r[3])
               : "memory");
}
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t* r) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr), "r"(r[0]),
               "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
               : "memory");
}
// 32 lanes x 32 consecutive columns
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]),
      "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]),
      "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
}  // namespace b200q

namespace b200q {
// ------------------------------------------------------------------ thread-block clusters (DSMEM)
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// All threads of all CTAs of the cluster (release / acquire of shared memory).
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Address of the same shared-memory location in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t map_shared_rank(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}
__device__ __forceinline__ void st_cluster_v4(uint32_t addr, float a, float b, float c, float d) {
  asm volatile("st.shared::cluster.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "f"(a), "f"(b), "f"(c), "f"(d)
               : "memory");
}
}  // namespace b200q
