// Device-side building blocks for the sm_100a kernels of this package: mbarriers, bulk async copies, tcgen05
// (TMEM allocation, UMMA issue/commit, TMEM loads), shared-memory / instruction descriptors, FP4/FP8 conversions
// and bounded waits.  Written against the PTX ISA; descriptor bit positions cross-checked with CUTLASS's
// cute/arch/mma_sm100_desc.hpp (SmemDescriptor / InstrDescriptor).  No multicast variants exist here on purpose:
// nothing in this package issues a cluster-multicast load.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <stdint.h>

namespace iob {

// ----------------------------------------------------------------------------------------------- status words
// Kernels that wait on anything (mbarrier, peer flag) take an `int* status` in global memory.  A wait that runs
// past its limit records one of these codes (first writer wins) and the kernel unwinds instead of hanging.
enum StatusCode : int {
  kOk = 0,
  kTimeoutProducer = 1,
  kTimeoutMma = 2,
  kTimeoutConsumer = 3,
  kTimeoutPeer = 4,
  kBadIndex = 5,
};

constexpr unsigned long long kWaitLimitNs = 2000000000ull;  // 2 s: far above any legitimate wait

// Programmatic dependent launch.  A kernel launched with the programmatic-serialization attribute may start while
// the previous kernel of its stream is still running; before reading anything that kernel wrote it calls
// griddep_wait() (returns once the previous grid has completed and its writes are visible; a no-op for a kernel
// launched normally).  griddep_launch() lets the NEXT kernel's CTAs be scheduled once every CTA of this grid has
// issued it (no effect when the next kernel was launched normally).
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void record_status(int* status, int code) {
  if (status) atomicCAS(status, 0, code);
}

// ----------------------------------------------------------------------------------------------- small helpers
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ int lane_id() { return threadIdx.x & 31; }
__device__ __forceinline__ int warp_id() { return threadIdx.x >> 5; }

__device__ __forceinline__ bool elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n\t.reg .pred P;\n\t"
      "elect.sync _|P, 0xffffffff;\n\t"
      "selp.u32 %0, 1, 0, P;\n\t}\n"
      : "=r"(pred));
  return pred != 0;
}

template <typename T>
__device__ __forceinline__ T warp_max(T v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = max(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
template <typename T>
__device__ __forceinline__ T warp_sum(T v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// ----------------------------------------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// try_wait with a suspend-time hint: the thread sleeps (up to hint_ns) instead of re-issuing, so waiting warps do
// not steal issue slots from the warps doing the work.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity, uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}
// Bounded wait.  `abort` is a shared-memory flag: once any role of the CTA gave up, every later wait returns false
// at once so the whole CTA unwinds within one limit.  The clock is read once per 64 polls.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort, int* status,
                                          int code) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = global_ns();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait_sleep(bar, parity, 20000)) return true;
    if ((it & 63) == 0) {
      if (abort && *abort) return false;
      if (global_ns() - t0 > kWaitLimitNs) {
        if (abort) *abort = 1;
        record_status(status, code);
        return false;
      }
    }
  }
}

// ----------------------------------------------------------------------------------------------- clusters
// Distributed shared memory between the CTAs of a thread-block cluster: plain stores and mbarrier arrivals into a
// peer CTA's shared memory (no multicast anywhere).
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_nctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(r));
  return r;
}
// Address of this CTA's shared-memory location `addr` in the shared window of cluster CTA `rank`.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
__device__ __forceinline__ void st_cluster_v4(uint32_t addr, uint4 v) {
  asm volatile("st.shared::cluster.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}
__device__ __forceinline__ uint32_t ld_cluster_u32(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.shared::cluster.u32 %0, [%1];" : "=r"(v) : "r"(addr) : "memory");
  return v;
}
__device__ __forceinline__ void st_cluster_f32(uint32_t addr, float v) {
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}
// Arrive (release, cluster scope) on an mbarrier in a peer CTA (address from mapa_shared).
__device__ __forceinline__ void mbar_arrive_remote(uint32_t bar_cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar_cluster_addr) : "memory");
}
// Bulk copy of `bytes` (multiple of 16, both addresses 16-byte aligned) from this CTA's shared memory into a peer
// CTA's shared memory (dst and the peer's mbarrier as mapa_shared addresses), completing as tx bytes on that mbarrier.
__device__ __forceinline__ void bulk_s2peer(uint32_t dst_cluster, const void* src, uint32_t bytes,
                                            uint32_t bar_cluster) {
  asm volatile(
      "cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst_cluster),
      "r"(smem_u32(src)), "r"(bytes), "r"(bar_cluster)
      : "memory");
}
__device__ __forceinline__ void bulk_commit_group() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Wait until at most N of this thread's committed bulk-copy groups still have source reads pending.
template <int N>
__device__ __forceinline__ void bulk_wait_group_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void fence_proxy_async_cluster() {
  asm volatile("fence.proxy.async.shared::cluster;" ::: "memory");
}
// Whole-cluster barrier (every thread of every CTA of the cluster).
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Wait on a local mbarrier whose arrivals may come from peer CTAs (acquire at cluster scope); bounded like mbar_wait.
__device__ __forceinline__ bool mbar_try_wait_cl(uint64_t* bar, uint32_t parity, uint32_t hint_ns = 20000) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}
// Non-blocking test (acquire at cluster scope): for issue loops that poll several barriers.
__device__ __forceinline__ bool mbar_test_cl(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Non-blocking test of a CTA-local phase.
__device__ __forceinline__ bool mbar_test(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ bool mbar_wait_cl(uint64_t* bar, uint32_t parity, volatile int* abort, int* status,
                                             int code) {
  const unsigned long long t0 = global_ns();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait_cl(bar, parity)) return true;
    if ((it & 63) == 0) {
      if (abort && *abort) return false;
      if (global_ns() - t0 > kWaitLimitNs) {
        if (abort) *abort = 1;
        record_status(status, code);
        return false;
      }
    }
  }
}

// ----------------------------------------------------------------------------------------------- async copies
// Plain (non-tensor, non-multicast) bulk copy global -> this CTA's shared memory, completing on an mbarrier.
// Both addresses 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* smem_dst, const void* gsrc, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(smem_dst)),
      "l"(gsrc), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
// Warm L2 with a global range (no shared memory involved); 16-byte aligned, size a multiple of 16.
__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ----------------------------------------------------------------------------------------------- tcgen05 / TMEM
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {  // whole warp
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {  // whole warp
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D(tmem) (+)= A(smem desc) * B(smem desc)^T, kind::f16 (f16 or bf16 inputs, fp32 accumulate); one thread issues.
__device__ __forceinline__ void umma_f16_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// D(tmem) (+)= A(smem desc) * B(smem desc)^T, kind::f8f6f4 (E4M3/E5M2/... inputs, fp32 accumulate).
__device__ __forceinline__ void umma_f8_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                           uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// D(tmem) (+)= A(tmem) * B(smem desc)^T, kind::f16.  A occupies 128 lanes (row m = lane m), K packed two 16-bit
// values per 32-bit column: one K=16 step spans 8 columns.
__device__ __forceinline__ void umma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive on `bar` once every previously issued tcgen05.mma of this thread has completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Warp w (w = warp index % 4) reads TMEM lanes 32w..32w+31; thread t gets lane 32w+t, columns [col, col+16).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
// Warp w (w = warp index % 4) reads TMEM lanes 32w..32w+31; thread t gets lane 32w+t, columns [col, col+32).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,"
      "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
// Warp w writes TMEM lanes 32(w%4)..+31; thread t writes lane 32(w%4)+t, columns [col, col+32).
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]),
      "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]),
      "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tmem_ld2(uint32_t taddr, uint32_t* r) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x2.b32 {%0,%1}, [%2];" : "=r"(r[0]), "=r"(r[1]) : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld4(uint32_t taddr, uint32_t* r) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t* r) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
}

// Shared-memory matrix descriptor, K-major operand in the 128-byte-swizzle canonical layout: rows of 128 bytes,
// the 16-byte chunk c of row r stored at chunk c ^ (r & 7), 8-row groups 1024 bytes apart (SBO).  Tiles whose K
// extent exceeds one 128-byte row are stored as separate [rows x 128 B] slabs; a K step inside a slab advances the
// start address by its byte offset.  Bits: [0,14) addr>>4, [16,30) LBO>>4, [32,46) SBO>>4, [46,48) version = 1,
// [49,52) base offset, [61,64) layout (2 = SWIZZLE_128B).  Slab bases must be 1024-byte aligned.
__device__ __forceinline__ uint64_t desc_sw128(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr & 0x3FFFFu) >> 4);
  d |= static_cast<uint64_t>(1) << 16;
  d |= static_cast<uint64_t>(1024 >> 4) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(2) << 61;
  return d;
}

// K-major operand in the 64-byte-swizzle layout: rows of 64 bytes, 16-byte chunk c of row r at c ^ ((r >> 1) & 3),
// 8-row groups 512 bytes apart; layout code 4 (SWIZZLE_64B).  Base 512-byte aligned.
__device__ __forceinline__ uint64_t desc_sw64(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr & 0x3FFFFu) >> 4);
  d |= static_cast<uint64_t>(1) << 16;
  d |= static_cast<uint64_t>(512 >> 4) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(4) << 61;
  return d;
}
__device__ __forceinline__ uint32_t sw64_chunk(uint32_t row, uint32_t c) {
  return row * 64u + ((c ^ ((row >> 1) & 3)) * 16u);
}
// MN-major operand, 128-byte swizzle: 8 K-rows x 128 B atoms; `lbo_bytes` = stride between atoms along M/N,
// 1024 B between 8-row groups along K.
__device__ __forceinline__ uint64_t desc_mn128(uint32_t addr, uint32_t lbo_bytes) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((addr & 0x3FFFFu) >> 4);
  d |= static_cast<uint64_t>(lbo_bytes >> 4) << 16;
  d |= static_cast<uint64_t>(1024 >> 4) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(2) << 61;
  return d;
}

// Instruction descriptor for kind::f16 / kind::f8f6f4 dense MMA, both operands K-major, fp32 accumulator.
// fmt: kind::f16 -> 0 = f16, 1 = bf16;  kind::f8f6f4 -> 0 = E4M3, 1 = E5M2.
__host__ __device__ constexpr uint32_t idesc_dense(uint32_t a_fmt, uint32_t b_fmt, uint32_t m, uint32_t n) {
  return (1u << 4) | (a_fmt << 7) | (b_fmt << 10) | ((n >> 3) << 17) | ((m >> 4) << 24);
}

// Byte offset of element (row, k) of 2-byte elements inside a [rows x 64] SW128 K-major slab.
__device__ __forceinline__ uint32_t sw128_off16(uint32_t row, uint32_t k) {
  const uint32_t chunk = (k >> 3) ^ (row & 7);
  return row * 128u + chunk * 16u + (k & 7) * 2u;
}
// Byte offset of the 16-byte chunk `c` (0..7) of row `row` inside a SW128 slab.
__device__ __forceinline__ uint32_t sw128_chunk(uint32_t row, uint32_t c) {
  return row * 128u + ((c ^ (row & 7)) * 16u);
}

// Register re-partition between warpgroups (all four warps of a warpgroup execute the same instruction).  The
// sum over warpgroups must stay within the registers the block was launched with.
template <uint32_t R>
__device__ __forceinline__ void regs_inc() { asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;\n" ::"n"(R)); }
template <uint32_t R>
__device__ __forceinline__ void regs_dec() { asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;\n" ::"n"(R)); }

// ----------------------------------------------------------------------------------------------- FP4 / FP8
// Two E2M1 codes (one byte, element 2i in the low nibble) -> f16x2, exact.
__device__ __forceinline__ uint32_t e2m1x2_to_f16x2(uint8_t b) {
  uint32_t out;
  asm volatile(
      "{\n\t.reg .b8 t;\n\t"
      "mov.b16 {t, _}, %1;\n\t"
      "cvt.rn.f16x2.e2m1x2 %0, t;\n\t}\n"
      : "=r"(out)
      : "h"(static_cast<uint16_t>(b)));
  return out;
}
// Four bytes of E2M1 pairs (one 32-bit word) -> four f16x2, exact: one register unpack, four conversions.
__device__ __forceinline__ void e2m1x8_to_f16x2x4(uint32_t w, uint32_t (&o)[4]) {
  asm volatile(
      "{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
      "mov.b32 {b0, b1, b2, b3}, %4;\n\t"
      "cvt.rn.f16x2.e2m1x2 %0, b0;\n\t"
      "cvt.rn.f16x2.e2m1x2 %1, b1;\n\t"
      "cvt.rn.f16x2.e2m1x2 %2, b2;\n\t"
      "cvt.rn.f16x2.e2m1x2 %3, b3;\n\t}\n"
      : "=r"(o[0]), "=r"(o[1]), "=r"(o[2]), "=r"(o[3])
      : "r"(w));
}
// Two E4M3 bytes (low byte = first element) -> f16x2, exact.
__device__ __forceinline__ uint32_t e4m3x2_to_f16x2(uint16_t v) {
  uint32_t out;
  asm volatile("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(out) : "h"(v));
  return out;
}
// f16x2 -> two E4M3 bytes (round to nearest even, saturating), low half -> low byte.
__device__ __forceinline__ uint16_t f16x2_to_e4m3x2(uint32_t h2) {
  uint16_t out;
  asm volatile("cvt.rn.satfinite.e4m3x2.f16x2 %0, %1;" : "=h"(out) : "r"(h2));
  return out;
}
// two fp32 -> two E4M3 bytes (a -> low byte), round to nearest even, saturating.
__device__ __forceinline__ uint16_t f32x2_to_e4m3x2(float lo, float hi) {
  uint16_t out;
  asm volatile("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(out) : "f"(hi), "f"(lo));
  return out;
}
// D(tmem) (+)= A(tmem) * B(smem desc)^T, kind::f8f6f4 (four 8-bit K values per 32-bit TMEM column, K = 32 / MMA).
__device__ __forceinline__ void umma_f8_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                           uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Batched issue: four kind::f8f6f4 MMAs in one asm statement.  Issued one per statement, consecutive tcgen05.mma
// instructions measured ~150 cycles apart (~250 with a memory clobber) whatever the MMA shape; four per statement
// issue at the tensor pipe's rate (a 128 x 256 x 32 E4M3 MMA every 128 cycles, 128 x 128 x 32 every 64).  MMA i
// writes d[i]; MMA 0 accumulates iff acc0 != 0, MMAs 1-3 iff the matching bit of acc_mask (bit i) is set.
__device__ __forceinline__ void umma_f8_ss_x4(const uint32_t (&d)[4], const uint64_t (&a)[4], const uint64_t (&b)[4],
                                              uint32_t idesc, uint32_t acc_mask) {
  asm volatile(
      "{\n\t.reg .pred p0, p1, p2, p3;\n\t"
      "setp.ne.b32 p0, %13, 0;\n\t"
      "setp.ne.b32 p1, %14, 0;\n\t"
      "setp.ne.b32 p2, %15, 0;\n\t"
      "setp.ne.b32 p3, %16, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %4, %8, %12, p0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%1], %5, %9, %12, p1;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%2], %6, %10, %12, p2;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%3], %7, %11, %12, p3;\n\t}\n" ::"r"(d[0]),
      "r"(d[1]), "r"(d[2]), "r"(d[3]), "l"(a[0]), "l"(a[1]), "l"(a[2]), "l"(a[3]), "l"(b[0]), "l"(b[1]), "l"(b[2]),
      "l"(b[3]), "r"(idesc), "r"(acc_mask & 1u), "r"(acc_mask & 2u), "r"(acc_mask & 4u), "r"(acc_mask & 8u));
}
// The same with A in TMEM (a[i] = TMEM address of MMA i's A columns).
__device__ __forceinline__ void umma_f8_ts_x4(const uint32_t (&d)[4], const uint32_t (&a)[4], const uint64_t (&b)[4],
                                              uint32_t idesc, uint32_t acc_mask) {
  asm volatile(
      "{\n\t.reg .pred p0, p1, p2, p3;\n\t"
      "setp.ne.b32 p0, %13, 0;\n\t"
      "setp.ne.b32 p1, %14, 0;\n\t"
      "setp.ne.b32 p2, %15, 0;\n\t"
      "setp.ne.b32 p3, %16, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], [%4], %8, %12, p0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%1], [%5], %9, %12, p1;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%2], [%6], %10, %12, p2;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%3], [%7], %11, %12, p3;\n\t}\n" ::"r"(d[0]),
      "r"(d[1]), "r"(d[2]), "r"(d[3]), "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "l"(b[0]), "l"(b[1]), "l"(b[2]),
      "l"(b[3]), "r"(idesc), "r"(acc_mask & 1u), "r"(acc_mask & 2u), "r"(acc_mask & 4u), "r"(acc_mask & 8u));
}
// Four K steps of one accumulation into d, one asm statement: MMA k reads A at a0 + k SA and B at b0 + k SB (the
// descriptors' address fields, 16-byte units, advanced inside the statement so only two descriptors cross into
// it).  MMA 0 accumulates iff acc0 != 0; MMAs 1-3 accumulate.
template <int SA, int SB>
__device__ __forceinline__ void umma_f8_ss_k4(uint32_t d, uint64_t a0, uint64_t b0, uint32_t idesc, uint32_t acc0) {
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t.reg .b64 a1, a2, a3, b1, b2, b3;\n\t"
      "setp.ne.b32 p, %4, 0;\n\tsetp.eq.u32 q, 0, 0;\n\t"
      "add.s64 a1, %1, %5;\n\tadd.s64 a2, %1, %6;\n\tadd.s64 a3, %1, %7;\n\t"
      "add.s64 b1, %2, %8;\n\tadd.s64 b2, %2, %9;\n\tadd.s64 b3, %2, %10;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], a1, b1, %3, q;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], a2, b2, %3, q;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], a3, b3, %3, q;\n\t}\n" ::"r"(d),
      "l"(a0), "l"(b0), "r"(idesc), "r"(acc0), "n"(SA), "n"(2 * SA), "n"(3 * SA), "n"(SB), "n"(2 * SB), "n"(3 * SB));
}
// The same with A in TMEM: MMA k reads A columns a0 + k SA.
template <int SA, int SB>
__device__ __forceinline__ void umma_f8_ts_k4(uint32_t d, uint32_t a0, uint64_t b0, uint32_t idesc, uint32_t acc0) {
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t.reg .b32 a1, a2, a3;\n\t.reg .b64 b1, b2, b3;\n\t"
      "setp.ne.b32 p, %4, 0;\n\tsetp.eq.u32 q, 0, 0;\n\t"
      "add.s32 a1, %1, %5;\n\tadd.s32 a2, %1, %6;\n\tadd.s32 a3, %1, %7;\n\t"
      "add.s64 b1, %2, %8;\n\tadd.s64 b2, %2, %9;\n\tadd.s64 b3, %2, %10;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], [%1], %2, %3, p;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], [a1], b1, %3, q;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], [a2], b2, %3, q;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], [a3], b3, %3, q;\n\t}\n" ::"r"(d),
      "r"(a0), "l"(b0), "r"(idesc), "r"(acc0), "n"(SA), "n"(2 * SA), "n"(3 * SA), "n"(SB), "n"(2 * SB), "n"(3 * SB));
}
// Warp w writes TMEM lanes 32(w%4)..+31; thread t writes lane 32(w%4)+t, columns [col, col+16).
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}
__device__ __forceinline__ float e4m3_to_float(uint8_t v) {
  __half_raw h = __nv_cvt_fp8_to_halfraw(static_cast<__nv_fp8_storage_t>(v), __NV_E4M3);
  return __half2float(__half(h));
}
__device__ __forceinline__ uint8_t float_to_e4m3(float x) {
  return static_cast<uint8_t>(__nv_cvt_float_to_fp8(x, __NV_SATFINITE, __NV_E4M3));
}
__device__ __forceinline__ uint32_t hmul2_u32(uint32_t a, uint32_t b) {
  __half2 r = __hmul2(*reinterpret_cast<__half2*>(&a), *reinterpret_cast<__half2*>(&b));
  return *reinterpret_cast<uint32_t*>(&r);
}
__device__ __forceinline__ uint32_t half2_bcast(__half h) {
  __half2 r = __halves2half2(h, h);
  return *reinterpret_cast<uint32_t*>(&r);
}

// E2M1 x E4M3 -> f16 (exact) -> E4M3 (round to nearest even): 8 values of one code word, one scale.
__device__ __forceinline__ uint2 f4_word_to_e4m3(uint32_t w, uint32_t scale_h2) {
  uint32_t h[4];
  e2m1x8_to_f16x2x4(w, h);
  const uint32_t e0 = f16x2_to_e4m3x2(hmul2_u32(h[0], scale_h2));
  const uint32_t e1 = f16x2_to_e4m3x2(hmul2_u32(h[1], scale_h2));
  const uint32_t e2 = f16x2_to_e4m3x2(hmul2_u32(h[2], scale_h2));
  const uint32_t e3 = f16x2_to_e4m3x2(hmul2_u32(h[3], scale_h2));
  return make_uint2(e0 | (e1 << 16), e2 | (e3 << 16));
}

// NVFP4 -> E4M3 without per-value conversions (conversions share the 16/clk/SM XU pipe with the softmax's exp).
// For each 16-value block the eight possible products {0, .5, 1, 1.5, 2, 3, 4, 6} x scale are formed once in f16
// (exact) and rounded to E4M3 (round to nearest even): an 8-byte table in two registers, byte k = code k.  A byte
// permute with the codes' magnitude nibbles as selector then decodes four values at a time; the sign bits are
// moved to bit 7 of each byte with a second permute.  Bit-identical to converting each value separately for every
// non-negative scale (block scales are amax / 6 >= 0 by construction).
__device__ __forceinline__ uint2 f4_scale_table(uint32_t sb) {
  const uint32_t s2 = e4m3x2_to_f16x2(static_cast<uint16_t>(sb | (sb << 8)));
  const uint32_t e01 = f16x2_to_e4m3x2(hmul2_u32(s2, 0x38000000u));   // (0, 0.5)
  const uint32_t e23 = f16x2_to_e4m3x2(hmul2_u32(s2, 0x3E003C00u));   // (1, 1.5)
  const uint32_t e45 = f16x2_to_e4m3x2(hmul2_u32(s2, 0x42004000u));   // (2, 3)
  const uint32_t e67 = f16x2_to_e4m3x2(hmul2_u32(s2, 0x46004400u));   // (4, 6)
  return make_uint2(e01 | (e23 << 16), e45 | (e67 << 16));
}
// Eight E2M1 codes (nibble i = value i) -> eight E4M3 bytes through the block's table.  The sign masks come from a
// byte permute in sign-replicate mode (selector nibble bit 3): value 2k + 1's sign is the msb of code byte k, value
// 2k's sign is the msb of byte k of (codes << 4).
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}
__device__ __forceinline__ uint2 f4_decode8(uint32_t w, uint2 tab) {
  const uint32_t mag = w & 0x77777777u;
  const uint32_t lo = prmt(tab.x, tab.y, mag);
  const uint32_t hi = prmt(tab.x, tab.y, mag >> 16);
  const uint32_t y = w << 4;
  const uint32_t slo = prmt(y, w, 0xD9C8u);
  const uint32_t shi = prmt(y, w, 0xFBEAu);
  return make_uint2(lo | (slo & 0x80808080u), hi | (shi & 0x80808080u));
}
// Shared-memory table of f4_scale_table for every scale byte (256 x 8 B), filled cooperatively by the CTA; a 16-value
// block then costs one 8-byte shared load instead of building its table.
__device__ __forceinline__ void f4_table_fill(uint2* tab) {
  for (int i = threadIdx.x; i < 256; i += blockDim.x) tab[i] = f4_scale_table(static_cast<uint32_t>(i));
}

// E2M1 magnitude code of y >= 0: number of midpoints strictly below y (ties round down), saturating at 7 (= 6.0).
__device__ __forceinline__ uint32_t e2m1_code_mag(float y) {
  return (y > 0.25f) + (y > 0.75f) + (y > 1.25f) + (y > 1.75f) + (y > 2.5f) + (y > 3.5f) + (y > 5.0f);
}
// GELU, tanh approximation: 0.5 g (1 + tanh(sqrt(2 / pi) (g + 0.044715 g^3))).
__device__ __forceinline__ float gelu_tanh_f(float g) {
  const float k0 = 0.7978845608028654f;  // sqrt(2 / pi)
  return 0.5f * g * (1.f + tanhf(k0 * (g + 0.044715f * g * g * g)));
}
__device__ __forceinline__ uint32_t e2m1_code(float y) {  // signed, no negative zero
  const uint32_t m = e2m1_code_mag(fabsf(y));
  return m | ((y < 0.f && m > 0) ? 8u : 0u);
}
// UE8M0 exponent byte of the smallest power of two s with amax / s <= 448 (clamped to [1, 253]): the activation
// scale rule of the FP8 block-scaled GEMMs (one scale per 128 values), shared by every kernel that quantizes for them.
__device__ __forceinline__ uint32_t ue8m0_for(float amax) {
  const float x = amax * (1.0f / 448.0f);
  const uint32_t b = __float_as_uint(x);
  int e = static_cast<int>((b >> 23) & 0xFF) - 127 + ((b & 0x7FFFFF) ? 1 : 0);
  if (x == 0.f) e = -126;
  e = max(-126, min(126, e));
  return static_cast<uint32_t>(e + 127);
}
// Block scale rule shared by every NVFP4 writer: e4m3(clamp(amax / 6, 2^-9, 448)).
__device__ __forceinline__ uint8_t nvfp4_block_scale(float amax) {
  const float s = fminf(fmaxf(amax / 6.0f, 0.001953125f), 448.0f);
  return float_to_e4m3(s);
}

}  // namespace iob

#define IOB_CUDA_CHECK(expr)                                                                   \
  do {                                                                                         \
    cudaError_t _e = (expr);                                                                   \
    if (_e != cudaSuccess) return _e;                                                          \
  } while (0)
