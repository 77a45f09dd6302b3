// Thin inline-PTX wrappers for the sm_100a features the kernels use:
// mbarriers, TMA tile loads (no multicast, ever), tcgen05 MMA / TMEM
// alloc / load / store / commit, and the UMMA shared-memory and instruction
// descriptors.  Every wait in this file is bounded: a wait that runs past its
// time limit records an error code in a device-global flag and returns false,
// so a protocol bug ends the kernel with an error status instead of a hang.
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

namespace fab {

// ---------------------------------------------------------------- errors ---
// Error codes written to the device error word (first error wins).
enum DeviceError : int {
  kDevOk = 0,
  kDevTimeoutQ = 1,
  kDevTimeoutKV = 2,
  kDevTimeoutS = 3,
  kDevTimeoutP = 4,
  kDevTimeoutO = 5,
  kDevTimeoutEmpty = 6,
  kDevTimeoutAcc = 7,
  kDevTimeoutTeardown = 8,
  kDevTimeoutPeerTile = 9,   // a tile's partial sums from every rank never all arrived
  kDevTimeoutPeerDone = 10,  // the reduced tiles from every owner never all arrived
  kDevTimeoutPartial = 11,   // a stream-K partial tile from another CTA pair never arrived
  kDevTimeoutSched = 12,     // the next tile from the cluster scheduler, or its slot's release, never came
  kDevTimeoutMerge = 13,     // the split-KV merge's copies of the partial rows never landed
};

// Device-global status word of the kernels of one translation unit (internal
// linkage: capi.cu and gemm.cu each have one; fab_get_device_error reads
// both).  A kernel that starts after a failed wait of its unit skips its work.
static __device__ int g_fab_device_error = 0;

// A single wait may take at most this long before the kernel gives up.
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s

// The limit the waits of this unit apply: kWaitLimitNs unless a test has set
// a shorter one through fab_debug_set_wait_limit_ns (attention unit only).
static __device__ uint64_t g_fab_wait_limit_ns = kWaitLimitNs;

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void record_device_error(int code) {
  atomicCAS(&g_fab_device_error, 0, code);
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// -------------------------------------------------------------- mbarrier ---
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
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

// Bounded wait for the phase with the given parity to complete.  `abort` is a
// CTA-shared flag: once any thread of the CTA has given up, the others stop
// waiting at their next poll.  Returns false on timeout or abort.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort, int code) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  uint32_t spins = 0;
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((++spins & 63u) == 0u) {
      if (*abort) return false;
      if (globaltimer_ns() - t0 > g_fab_wait_limit_ns) {
        record_device_error(code);
        *abort = 1;
        return false;
      }
    }
  }
}

// Warp-collective bounded wait: every lane polls, and the warp continues only
// if all lanes saw the phase complete, so a timeout can never leave a warp
// divergent in front of a .sync.aligned tcgen05 instruction.
__device__ __forceinline__ bool mbar_wait_warp(uint64_t* bar, uint32_t parity, volatile int* abort, int code) {
  const bool ok = mbar_wait(bar, parity, abort, code);
  return __all_sync(0xffffffffu, ok) != 0;
}

// Named barrier over `count` threads (a multiple of 32); id 0 is __syncthreads.
// It has no time limit: every thread that can reach one must reach it.
__device__ __forceinline__ void named_barrier_sync(uint32_t id, uint32_t count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// ----------------------------------------------------- TMA tensor stores ---
// Store one box of shared memory (laid out as the map's box, swizzle
// included) to global memory at the given coordinates; the box is clipped at
// the tensor's bounds.  Generic-proxy writes to `src` must be fenced with
// fence_proxy_async_smem() first; the store is complete for shared memory
// (may be overwritten / the CTA may exit) after bulk_wait_read_all().
__device__ __forceinline__ void tma_store_4d(const CUtensorMap* map, const void* src, int c0, int c1, int c2,
                                             int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.global.shared::cta.bulk_group [%0, {%2, %3, %4, %5}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(smem_u32(src)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}
__device__ __forceinline__ void bulk_commit_group() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read_all() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
// Orders this thread's view of global memory (generic proxy: e.g. data other
// CTAs published before an atomic this thread observed) before its later
// bulk copies (async proxy) read it.
__device__ __forceinline__ void fence_proxy_async_global() { asm volatile("fence.proxy.async.global;" ::: "memory"); }

// Contiguous bulk copy global -> this CTA's shared memory (no tensor map):
// both addresses 16-byte aligned, bytes a multiple of 16; completes `bytes`
// transaction bytes on `bar`.
__device__ __forceinline__ void bulk_load_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// ------------------------------------------------- cross-GPU signalling ---
// Counters in (possibly peer) global memory, ordered at system scope so that
// NVLink peer stores issued before a release are visible after the matching
// acquire on the other GPU.
__device__ __forceinline__ void fence_acq_rel_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }

__device__ __forceinline__ void red_release_sys_add(unsigned long long* addr, unsigned long long v) {
  asm volatile("red.release.sys.global.add.u64 [%0], %1;" ::"l"(addr), "l"(v) : "memory");
}

__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long* addr) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(addr) : "memory");
  return v;
}

// Bounded spin until *counter >= target.  Returns false (after recording
// `code`) when the limit passes or another thread of the CTA gave up.
__device__ __forceinline__ bool wait_counter_at_least(const unsigned long long* counter, unsigned long long target,
                                                      volatile int* abort, int code) {
  if (ld_acquire_sys(counter) >= target) return true;
  const uint64_t t0 = globaltimer_ns();
  uint32_t spins = 0;
  while (true) {
    __nanosleep(64);
    if (ld_acquire_sys(counter) >= target) return true;
    if ((++spins & 63u) == 0u) {
      if (*abort) return false;
      if (globaltimer_ns() - t0 > kWaitLimitNs) {
        record_device_error(code);
        *abort = 1;
        return false;
      }
    }
  }
}

// ------------------------------------------------- flags within one GPU ---
// A word in global memory that one warp sets after writing data and another
// waits for before reading it (GPU scope: both on this device).
__device__ __forceinline__ void st_release_gpu(int* addr, int v) {
  asm volatile("st.release.gpu.global.b32 [%0], %1;" ::"l"(addr), "r"(v) : "memory");
}

__device__ __forceinline__ int ld_acquire_gpu(const int* addr) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(addr) : "memory");
  return v;
}

// Bounded spin until *flag != 0.  Returns false (after recording `code`) when
// the limit passes or another thread of the CTA gave up.
__device__ __forceinline__ bool wait_flag_set(const int* flag, volatile int* abort, int code) {
  if (ld_acquire_gpu(flag) != 0) return true;
  const uint64_t t0 = globaltimer_ns();
  uint32_t spins = 0;
  while (true) {
    __nanosleep(32);
    if (ld_acquire_gpu(flag) != 0) return true;
    if ((++spins & 63u) == 0u) {
      if (*abort) return false;
      if (globaltimer_ns() - t0 > g_fab_wait_limit_ns) {
        record_device_error(code);
        *abort = 1;
        return false;
      }
    }
  }
}

// ------------------------------------------------------------------- TMA ---
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// Tiled 2-D / 4-D bulk tensor loads into this CTA's shared memory, completing
// on `bar` by transaction bytes.  The innermost coordinate must be a multiple
// of 16 bytes; all callers pass multiples of the 128-byte swizzle atom.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1, int c2,
                                            int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_u32(bar))
      : "memory");
}

// Warpgroup register re-split.  Every warp of a warpgroup executes these
// together; the register pool they draw on is the block's launch allocation
// (threads x registers per thread at launch), so callers must keep the sum of
// the new per-warpgroup budgets within it.
template <uint32_t kRegs>
__device__ __forceinline__ void setmaxnreg_dec() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kRegs));
}
template <uint32_t kRegs>
__device__ __forceinline__ void setmaxnreg_inc() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kRegs));
}

// --------------------------------------------------------------- tcgen05 ---
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem] * B[smem]
// One elected lane of a converged warp: the lane that issues a warp's
// tcgen05.mma and tcgen05.commit instructions.
__device__ __forceinline__ bool elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "elect.sync _|p, 0xffffffff;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(pred));
  return pred != 0;
}

__device__ __forceinline__ void mma_ss_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                           uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void mma_ss_tf32(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem]
__device__ __forceinline__ void mma_ts_f16(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                           uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void mma_ts_tf32(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// ------------------------------------------------ CTA pairs (cta_group::2) ---
// A kernel that issues one tcgen05 instruction with cta_group::2 issues all of
// them (alloc, relinquish, mma, commit, dealloc) with it.  The pair is a
// cluster of two CTAs; rank 0 issues the MMAs for both.
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// Every thread of every CTA of the cluster: barrier over the cluster (no time
// limit, so only at points every thread of the cluster always reaches, with
// its warp converged).
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// The shared::cluster address of `addr` (a shared::cta address of this CTA's
// layout) in the CTA of the given cluster rank.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}

// 16-byte store into the shared memory of any CTA of the cluster
// (shared::cluster address); ordered for the owner by the next cluster barrier.
__device__ __forceinline__ void st_cluster_v4(uint32_t cluster_addr, float a, float b, float c, float d) {
  asm volatile("st.shared::cluster.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(cluster_addr), "f"(a), "f"(b), "f"(c),
               "f"(d)
               : "memory");
}

// Arrive on an mbarrier of any CTA of the cluster (shared::cluster address).
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

// 4-byte store into the shared memory of any CTA of the cluster; published to
// that CTA by a later mbar_arrive_cluster (release at cluster scope) on a
// barrier it waits on with mbar_wait_cluster.
__device__ __forceinline__ void st_cluster_u32(uint32_t cluster_addr, uint32_t v) {
  asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(cluster_addr), "r"(v) : "memory");
}

// mbar_wait with acquire at cluster scope: for phases completed by arrivals
// (and stores before them) from the other CTA of the cluster.
__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity, volatile int* abort, int code) {
  if (mbar_try_wait_cluster(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  uint32_t spins = 0;
  while (true) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    if ((++spins & 63u) == 0u) {
      if (*abort) return false;
      if (globaltimer_ns() - t0 > g_fab_wait_limit_ns) {
        record_device_error(code);
        *abort = 1;
        return false;
      }
    }
  }
}

// ------------------------------------------------ cluster launch control ---
// Ask the hardware scheduler to cancel one cluster of this grid that has not
// started yet and hand its work to the caller.  The 16-byte response lands in
// `resp` (shared::cta, 16-byte aligned) and completes 16 transaction bytes on
// `bar`, whose phase the caller armed with mbar_arrive_expect_tx(bar, 16).
// One thread per cluster issues it; the response must land before the CTA
// exits.
__device__ __forceinline__ void clc_try_cancel(uint32_t resp, uint64_t* bar) {
  asm volatile(
      "clusterlaunchcontrol.try_cancel.async.shared::cta.mbarrier::complete_tx::bytes.b128 [%0], [%1];" ::"r"(resp),
      "r"(smem_u32(bar))
      : "memory");
}

// The x index of the first CTA of the cancelled cluster, or -1 when the
// request failed (no cluster was left to cancel).
__device__ __forceinline__ int clc_first_cta_x(uint32_t resp) {
  uint32_t ok, x;
  asm volatile(
      "{\n\t.reg .pred p;\n\t.reg .b128 h;\n\t"
      "ld.shared.b128 h, [%2];\n\t"
      "clusterlaunchcontrol.query_cancel.is_canceled.pred.b128 p, h;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t"
      "mov.u32 %1, 0;\n\t"
      "@p clusterlaunchcontrol.query_cancel.get_first_ctaid::x.b32.b128 %1, h;\n\t}"
      : "=r"(ok), "=r"(x)
      : "r"(resp)
      : "memory");
  return ok ? static_cast<int>(x) : -1;
}

__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// D[tmem of both CTAs] (+)= A[smem of both] * B[smem of both]: M = 256 rows,
// 128 from each CTA's A; N columns, N/2 from each CTA's B; each CTA's TMEM
// receives its 128 rows x N.  Descriptors hold this CTA's shared::cta
// offsets; the peer's operands sit at the same offsets.
__device__ __forceinline__ void mma_ss_f16_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                                uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive once on the mbarrier at `bar`'s offset in every CTA of `cta_mask`
// when the pair's tcgen05 ops issued so far by this thread have completed.
__device__ __forceinline__ void mma_commit_pair(uint64_t* bar, uint16_t cta_mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"(cta_mask)
      : "memory");
}

// Tiled 2-D load into this CTA's shared memory whose transaction bytes
// complete on an mbarrier of either CTA of the pair (shared::cluster address:
// the pair's rank-0 CTA counts both CTAs' bytes).  No multicast.
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* map, uint32_t bar_cluster, int c0,
                                                 int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(bar_cluster)
      : "memory");
}

// Arrive once on `bar` when every tcgen05 async op issued so far by this
// thread has completed.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// 32 lanes x 32 bits, 32 consecutive columns: thread t receives lane
// (addr.lane + t), registers r[i] = column (addr.col + i).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]),
      "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]),
      "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31]), "r"(r[32])
      : "memory");
}

// ----------------------------------------------------------- descriptors ---
// UMMA shared-memory matrix descriptor for a 128-byte-swizzled operand.
//   bits [0,14)  start address >> 4
//   bits [16,30) leading-dimension byte offset >> 4
//   bits [32,46) stride-dimension byte offset >> 4
//   bits [46,48) descriptor version (1 on sm_100)
//   bits [61,64) layout: 2 = SWIZZLE_128B
// K-major operands: 8-row groups are `sbo` bytes apart, LBO is unused.
// MN-major operands: 64-element (128 B) column atoms are `lbo` bytes apart,
// 8-row groups along K are `sbo` bytes apart.
// Layout codes (bits [61,64)): 2 = SWIZZLE_128B (16-byte chunks XOR row%8),
// 1 = SWIZZLE_128B_BASE32B (32-byte chunks XOR row%4; the only layout an
// MN-major tf32 operand may use, with 4-row K groups).
enum UmmaLayout : uint32_t { kLayoutSw128Base32B = 1, kLayoutSw128 = 2 };

__host__ __device__ constexpr uint64_t umma_desc(uint32_t smem_addr, uint32_t lbo, uint32_t sbo, uint32_t layout) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32;
  d |= 1ull << 46;
  d |= static_cast<uint64_t>(layout) << 61;
  return d;
}

__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t smem_addr, uint32_t lbo, uint32_t sbo) {
  return umma_desc(smem_addr, lbo, sbo, kLayoutSw128);
}

// The same descriptor as two 32-bit words, for issue loops that step through
// a buffer: the low word holds (address >> 4) and LBO, the high word SBO,
// version and layout.  Shared-memory addresses stay below 2^18, so a byte
// offset added to the low word as (offset >> 4) never carries out of the
// 14-bit address field.
__host__ __device__ constexpr uint32_t umma_desc_lo(uint32_t smem_addr, uint32_t lbo) {
  return ((smem_addr >> 4) & 0x3FFFu) | (((lbo >> 4) & 0x3FFFu) << 16);
}
__host__ __device__ constexpr uint32_t umma_desc_hi(uint32_t sbo, uint32_t layout) {
  return ((sbo >> 4) & 0x3FFFu) | (1u << 14) | (layout << 29);
}
__host__ __device__ constexpr uint64_t umma_desc_join(uint32_t lo, uint32_t hi) {
  return (static_cast<uint64_t>(hi) << 32) | lo;
}
static_assert(umma_desc_join(umma_desc_lo(0x2F3A0u, 16384), umma_desc_hi(512, kLayoutSw128Base32B)) ==
                  umma_desc(0x2F3A0u, 16384, 512, kLayoutSw128Base32B),
              "split descriptor words");
static_assert(umma_desc_join(umma_desc_lo(0x1230u, 16) + (0x400u >> 4), umma_desc_hi(1024, kLayoutSw128)) ==
                  umma_desc(0x1630u, 16, 1024, kLayoutSw128),
              "offset added to the low word");

// MN-major operand descriptor: 128-byte column atoms `lbo` bytes apart.  For
// 16-bit types 8-row K groups (1024 B) with the 16-byte-chunk swizzle; for
// tf32 4-row K groups (512 B) with the 32-byte-chunk swizzle.
template <int kElt>
__device__ __forceinline__ uint64_t umma_desc_mn(uint32_t smem_addr, uint32_t lbo) {
  if constexpr (kElt == 4)
    return umma_desc(smem_addr, lbo, 512, kLayoutSw128Base32B);
  else
    return umma_desc(smem_addr, lbo, 1024, kLayoutSw128);
}

// Operand formats for the instruction descriptor.
enum UmmaFormat : uint32_t { kFmtF16 = 0, kFmtBF16 = 1, kFmtTF32 = 2 };

// UMMA instruction descriptor (kind::f16 / kind::tf32, fp32 accumulator).
//   bits [4,6)   D format (1 = f32)
//   bits [7,10)  A format, [10,13) B format
//   bit 15 / 16  A / B major (0 = K-major, 1 = MN-major)
//   bits [17,23) N >> 3,  bits [24,29) M >> 4
__host__ __device__ constexpr uint32_t umma_idesc(uint32_t fmt, uint32_t m, uint32_t n, uint32_t a_mn_major,
                                                  uint32_t b_mn_major) {
  return (1u << 4) | (fmt << 7) | (fmt << 10) | (a_mn_major << 15) | (b_mn_major << 16) | ((n >> 3) << 17) |
         ((m >> 4) << 24);
}

// ------------------------------------------------------------- numerics ---
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// max(a, b, c) in one instruction (three-input max.f32, sm_100).
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// 2^x for two values on the FMA pipe, leaving the MUFU unit to other work.
// Method: Cody & Waite range reduction, x = n + f with n = round(x) taken from
// the low mantissa bits of x + 1.5*2^23 and f in [-1/2, 1/2]; 2^f from a
// degree-3 polynomial whose coefficients are a relative-error minimax (Remez)
// fit made for this library (max relative error 7.5e-5, below the rounding of
// P to bf16/fp16/tf32); 2^n applied by adding n to the exponent field.
// Inputs below -126 are clamped there (the result is then < 1e-37).
constexpr float kExp2C0 = 0.9999280571937561f;
constexpr float kExp2C1 = 0.6932609677314758f;
constexpr float kExp2C2 = 0.2426111251115799f;
constexpr float kExp2C3 = 0.0551716685295105f;
constexpr float kRoundMagic = 12582912.0f;  // 1.5 * 2^23

__device__ __forceinline__ float2 exp2_poly2(float2 x) {
  x.x = fmaxf(x.x, -126.0f);
  x.y = fmaxf(x.y, -126.0f);
  const float2 j = __fadd2_rn(x, make_float2(kRoundMagic, kRoundMagic));
  const float2 n = __fadd2_rn(j, make_float2(-kRoundMagic, -kRoundMagic));
  const float2 f = __ffma2_rn(n, make_float2(-1.0f, -1.0f), x);
  float2 p = __ffma2_rn(f, make_float2(kExp2C3, kExp2C3), make_float2(kExp2C2, kExp2C2));
  p = __ffma2_rn(p, f, make_float2(kExp2C1, kExp2C1));
  p = __ffma2_rn(p, f, make_float2(kExp2C0, kExp2C0));
  const uint32_t rx = __float_as_uint(p.x) + (__float_as_uint(j.x) << 23);
  const uint32_t ry = __float_as_uint(p.y) + (__float_as_uint(j.y) << 23);
  return make_float2(__uint_as_float(rx), __uint_as_float(ry));
}

}  // namespace fab
