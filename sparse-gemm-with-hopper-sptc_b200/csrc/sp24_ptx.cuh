// sp24_ptx.cuh — thin inline-PTX wrappers for the sm_100a features the 2:4
// sparse GEMM uses: mbarriers, TMA bulk-tensor loads, and the tcgen05 family
// (TMEM allocation, tcgen05.cp, tcgen05.mma.sp, tcgen05.commit, tcgen05.ld).
//
// Everything here is written from the PTX ISA description of the instructions.
// Every spin-wait is bounded: a wait gives up after the caller's timeout of
// %globaltimer (or 2^26 polls), raises a CTA-wide abort flag and returns
// false, so a broken pipeline turns into an error status instead of a hung
// GPU.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace sp24 {

#define SP24_DEV __device__ __forceinline__

SP24_DEV uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

SP24_DEV uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------- mbarrier
SP24_DEV void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}

// Makes initialised barriers visible to the async proxy (TMA, tcgen05).
SP24_DEV void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// Orders this thread's ordinary shared-memory stores before later reads of
// the same bytes by the async proxy (tcgen05.mma operands, TMA).
SP24_DEV void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

SP24_DEV void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(
                   smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

SP24_DEV void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// kCluster: acquire at cluster scope (the phase was completed by arrivals
// from another CTA of the cluster that released at cluster scope).
template <bool kCluster = false>
SP24_DEV bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  if constexpr (kCluster) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
  } else {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
  }
  return ok != 0;
}

// Slow path of mbar_wait, kept out of line so the issue loops stay short.
template <bool kCluster>
__device__ __noinline__ bool mbar_wait_slow(uint64_t* bar, uint32_t parity, volatile int* abort,
                                            uint64_t timeout_ns) {
  const uint64_t t0 = globaltimer_ns();
  uint32_t it = 0;
  while (true) {
    if (mbar_try_wait<kCluster>(bar, parity)) return true;
    if ((++it & 63u) == 0) {
      if (*abort) return false;
      if (globaltimer_ns() - t0 > timeout_ns || it > (1u << 26)) {
        *abort = 1;
        return false;
      }
    }
  }
}

// Bounded wait for the phase of parity `parity` to complete: one inline
// try_wait (itself a bounded hardware wait), then the out-of-line loop.
// Returns false (and raises *abort) when the wait times out, or when another
// role of the CTA already raised *abort.
template <bool kCluster = false>
SP24_DEV bool mbar_wait_fast(uint64_t* bar, uint32_t parity, volatile int* abort,
                             uint64_t timeout_ns) {
  if (__builtin_expect(mbar_try_wait<kCluster>(bar, parity), 1)) return true;
  return mbar_wait_slow<kCluster>(bar, parity, abort, timeout_ns);
}

// Bounded wait for long waits on a busy SM (e.g. epilogue warps waiting for
// a whole tile): after a few polls it sleeps between polls, so idle waiters
// do not compete with the producers and the MMA issuer for issue slots and
// shared-memory bandwidth.
SP24_DEV bool mbar_wait_sleepy(uint64_t* bar, uint32_t parity, volatile int* abort,
                               uint64_t timeout_ns) {
  if (mbar_try_wait<false>(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  uint32_t it = 0;
  while (true) {
    if (mbar_try_wait<false>(bar, parity)) return true;
    ++it;
    if (it > 8) __nanosleep(256);
    if ((it & 15u) == 0) {
      if (*abort) return false;
      if (globaltimer_ns() - t0 > timeout_ns || it > (1u << 26)) {
        *abort = 1;
        return false;
      }
    }
  }
}

template <bool kCluster = false>
SP24_DEV bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort, uint64_t timeout_ns) {
  if (mbar_try_wait<kCluster>(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  uint32_t it = 0;
  while (true) {
    if (mbar_try_wait<kCluster>(bar, parity)) return true;
    if ((++it & 63u) == 0) {
      if (*abort) return false;
      if (globaltimer_ns() - t0 > timeout_ns || it > (1u << 26)) {
        *abort = 1;
        return false;
      }
    }
  }
}

// ---------------------------------------------------------------- programmatic dependent launch
// A GEMM launched with programmatic stream serialization may start while the
// previous kernel of the stream is still finishing.  It triggers its own
// dependents once its prologue is done, and every thread that reads global
// memory written by earlier work (the TMA producers) first waits for the
// previous grid's completion and memory flush.  Everything else (epilogue
// loads and stores) is ordered after that wait through the mbarrier chain.
// Without the launch attribute both instructions are no-ops.
SP24_DEV void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
SP24_DEV void griddep_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---------------------------------------------------------------- TMA
SP24_DEV void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// 2-D tiled load of one box into shared memory; completes `bytes` on `bar`.
SP24_DEV void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// Untiled bulk copy global -> shared (16-byte aligned, size multiple of 16).
SP24_DEV void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// ---------------------------------------------------------------- tcgen05
SP24_DEV void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
SP24_DEV void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
SP24_DEV void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
SP24_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
SP24_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Arrive once on `bar` when every tcgen05 async op issued so far by this
// thread (mma, cp) has completed.
SP24_DEV void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

// Shared memory -> TMEM copy of 128 lanes x 128 bits (4 columns).
SP24_DEV void tc_cp_128x128b(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::1.128x128b [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
}

// Sparse MMA, both operands from shared memory, D and metadata in TMEM.
//   kind 0: kind::f16 (fp16 / bf16 inputs), kind 1: kind::f8f6f4 (e4m3).
template <int KIND>
SP24_DEV void tc_mma_sp(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t e_tmem,
                        uint32_t idesc, uint32_t accumulate) {
  if constexpr (KIND == 0) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %5, 0;\n\t"
        "tcgen05.mma.sp.cta_group::1.kind::f16 [%0], %1, %2, [%3], %4, p;\n\t}\n" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(e_tmem), "r"(idesc), "r"(accumulate)
        : "memory");
  } else {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %5, 0;\n\t"
        "tcgen05.mma.sp.cta_group::1.kind::f8f6f4 [%0], %1, %2, [%3], %4, p;\n\t}\n" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(e_tmem), "r"(idesc), "r"(accumulate)
        : "memory");
  }
}

// TMEM -> registers: warp reads its 32 lanes x N consecutive 32-bit columns.
SP24_DEV void tmem_ld_x16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
SP24_DEV void tmem_ld_x32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
// Completes outstanding tcgen05.ld; the "+r" pins make every loaded register
// depend on the wait so no use is scheduled before it.
template <int N>
SP24_DEV void tmem_ld_wait(uint32_t (&r)[N]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < N; ++i) asm volatile("" : "+r"(r[i]));
}

// ---------------------------------------------------------------- clusters / CTA pairs
SP24_DEV uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// Address of the same shared variable in CTA `rank` of the cluster.
SP24_DEV uint32_t mapa_shared(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}
SP24_DEV void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr)
               : "memory");
}
// 16-byte load from a cluster shared-memory address (any CTA of the cluster).
SP24_DEV float4 ld_dsmem_f4(uint32_t cluster_addr) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0,%1,%2,%3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(cluster_addr)
               : "memory");
  return v;
}
SP24_DEV void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::
                   : "memory");
}
// TMA load issued by either CTA of a pair; completion bytes go to the
// mbarrier at `bar_cluster` (may live in the peer CTA).
SP24_DEV void tma_load_2d_pair(void* dst, const CUtensorMap* map, uint32_t bar_cluster, int x,
                               int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar_cluster)
      : "memory");
}
// The same load under an L2 cache policy (createpolicy).
SP24_DEV void tma_load_2d_pair_hint(void* dst, const CUtensorMap* map, uint32_t bar_cluster, int x,
                                    int y, uint64_t pol) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      ".L2::cache_hint [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar_cluster), "l"(pol)
      : "memory");
}
SP24_DEV void tmem_alloc_pair(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
SP24_DEV void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
SP24_DEV void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
// Arrive on the barrier at the same offset in every CTA of `mask` once the
// pair's outstanding tcgen05 ops complete.
SP24_DEV void tc_commit_pair(uint64_t* bar, uint16_t mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64"
      " [%0], %1;" ::"r"(smem_u32(bar)),
      "h"(mask)
      : "memory");
}
SP24_DEV void tc_cp_128x128b_pair(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::2.128x128b [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
}
template <int KIND>
SP24_DEV void tc_mma_sp_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t e_tmem,
                             uint32_t idesc, uint32_t accumulate) {
  if constexpr (KIND == 0) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %5, 0;\n\t"
        "tcgen05.mma.sp.cta_group::2.kind::f16 [%0], %1, %2, [%3], %4, p;\n\t}\n" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(e_tmem), "r"(idesc), "r"(accumulate)
        : "memory");
  } else {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %5, 0;\n\t"
        "tcgen05.mma.sp.cta_group::2.kind::f8f6f4 [%0], %1, %2, [%3], %4, p;\n\t}\n" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(e_tmem), "r"(idesc), "r"(accumulate)
        : "memory");
  }
}

// ---------------------------------------------------------------- stage issue
// The MMA-issuing warp runs its loop converged (every operand warp-uniform)
// and elects ONE lane per stage, which then issues the stage's tcgen05.cp,
// MMAs and commit as plain instructions:
//
//   if (elect_one()) { tc_cp<CG>(...); tc_mma<CG, KIND>(...); ...; tc_commit<CG>(...); }
//   __syncwarp();
//
// Measured on B200 in the narrow-N kernel (%globaltimer stamps): a separate
// elect.sync around every instruction costs ~56 ns per MMA, four MMAs per
// elected asm block ~24 ns each, one election per stage ~20 ns each.  With
// skinny tiles (8 MMAs per 44 KB stage) the per-instruction form made the
// issuing warp, not HBM, the limit.  The same lane is elected every time
// (the lowest active lane), so its commits track all the MMAs it issued.

// True in exactly one lane of the converged warp.
SP24_DEV bool elect_one() {
  uint32_t p;
  asm volatile(
      "{\n\t.reg .pred e;\n\telect.sync _|e, 0xffffffff;\n\tselp.u32 %0, 1, 0, e;\n\t}\n"
      : "=r"(p));
  return p != 0;
}

template <int CG>
SP24_DEV void tc_cp(uint32_t taddr, uint64_t sdesc) {
  if constexpr (CG == 1) tc_cp_128x128b(taddr, sdesc);
  else tc_cp_128x128b_pair(taddr, sdesc);
}

template <int CG, int KIND>
SP24_DEV void tc_mma(uint32_t d, uint64_t a, uint64_t b, uint32_t e, uint32_t idesc, uint32_t acc) {
  if constexpr (CG == 1) tc_mma_sp<KIND>(d, a, b, e, idesc, acc);
  else tc_mma_sp_pair<KIND>(d, a, b, e, idesc, acc);
}

// CG 1: arrive on this CTA's barrier; CG 2: on the barrier at the same offset
// in every CTA of `mask`.
template <int CG>
SP24_DEV void tc_commit_to(uint64_t* bar, uint16_t mask) {
  if constexpr (CG == 1) {
    tc_commit(bar);
    (void)mask;
  } else {
    tc_commit_pair(bar, mask);
  }
}

// Lane 0 runs the bounded wait; the verdict is broadcast so the warp stays
// converged.
template <bool kCluster = false>
SP24_DEV bool mbar_wait_warp(uint64_t* bar, uint32_t parity, volatile int* abort,
                             uint64_t timeout_ns) {
  int ok = 1;
  if ((threadIdx.x & 31) == 0) ok = mbar_wait_fast<kCluster>(bar, parity, abort, timeout_ns) ? 1 : 0;
  ok = __shfl_sync(0xffffffffu, ok, 0);
  return ok != 0;
}

// 32-byte global store (one full sector per thread).
SP24_DEV void st_global_v8(float* p, const float* v) {
  asm volatile("st.global.v8.f32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"l"(p), "f"(v[0]), "f"(v[1]),
               "f"(v[2]), "f"(v[3]), "f"(v[4]), "f"(v[5]), "f"(v[6]), "f"(v[7])
               : "memory");
}

// L2 cache policy that marks the lines it touches first for eviction: for
// output that nothing in the kernel reads again, so it does not push the
// reused operand tiles out of L2.
SP24_DEV uint64_t l2_evict_first_policy() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

// L2 cache policy that keeps the lines it touches over others: for operand
// tiles that other CTAs read again much later.
SP24_DEV uint64_t l2_evict_last_policy() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

// 32-byte global stores under an L2 cache policy.
SP24_DEV void st_global_v8_hint(float* p, const float* v, uint64_t pol) {
  asm volatile("st.global.L2::cache_hint.v8.f32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8}, %9;" ::"l"(p),
               "f"(v[0]), "f"(v[1]), "f"(v[2]), "f"(v[3]), "f"(v[4]), "f"(v[5]), "f"(v[6]),
               "f"(v[7]), "l"(pol)
               : "memory");
}

SP24_DEV void st_global_v8_u32_hint(void* p, const uint32_t* v, uint64_t pol) {
  asm volatile("st.global.L2::cache_hint.v8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8}, %9;" ::"l"(p),
               "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]),
               "r"(v[7]), "l"(pol)
               : "memory");
}

// 16-byte global store under an L2 cache policy.
SP24_DEV void st_global_v4_u32_hint(void* p, const uint32_t* v, uint64_t pol) {
  asm volatile("st.global.L2::cache_hint.v4.b32 [%0], {%1,%2,%3,%4}, %5;" ::"l"(p), "r"(v[0]),
               "r"(v[1]), "r"(v[2]), "r"(v[3]), "l"(pol)
               : "memory");
}

// ---------------------------------------------------------------- descriptors
// Shared-memory matrix descriptor (tcgen05 format):
//   [0,14) start address >> 4, [16,30) leading byte offset >> 4,
//   [32,46) stride byte offset >> 4, [46,48) version = 1,
//   [49,52) base offset = 0, [61,64) layout (0 none, 2 SW128, 4 SW64, 6 SW32).
enum : uint32_t { kLayoutNone = 0, kLayoutSW128 = 2, kLayoutSW64 = 4, kLayoutSW32 = 6 };

SP24_DEV uint64_t make_sdesc(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes,
                             uint32_t layout) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1u) << 46;
  d |= static_cast<uint64_t>(layout & 7u) << 61;
  return d;
}

// Instruction descriptor for kind::f16 / kind::f8f6f4 with fp32 accumulate:
//   [0,2) sparsity selector, [2] sparse, [4,6) D format (1 = f32),
//   [7,10) A format, [10,13) B format, [15] A major (0 = K), [16] B major
//   (1 = MN), [17,23) N >> 3, [24,29) M >> 4.
__host__ __device__ constexpr uint32_t make_idesc_sparse(uint32_t fmt, uint32_t n, uint32_t m,
                                                         bool b_mn_major) {
  return (1u << 2) | (1u << 4) | (fmt << 7) | (fmt << 10) | (0u << 15) |
         ((b_mn_major ? 1u : 0u) << 16) | ((n >> 3) << 17) | ((m >> 4) << 24);
}

}  // namespace sp24
