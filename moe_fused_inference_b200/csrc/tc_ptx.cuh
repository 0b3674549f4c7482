// tc_ptx.cuh — sm_100a primitives for the tcgen05 block-scaled MXFP4 GEMMs:
// mbarriers with bounded waits, TMA tile loads, bulk copies, TMEM
// allocation, tcgen05.mma (kind::mxf4, E8M0 scale per 32 K), tcgen05.cp of
// scale factors into TMEM, tcgen05.ld of the fp32 accumulator.
//
// Descriptor encodings follow the public PTX ISA (tcgen05 matrix / instruction
// descriptors) as restated by CUTLASS's cute/arch/mma_sm100_desc.hpp
// (SmemDescriptor, InstrDescriptorBlockScaled).  No multicast anywhere: every
// load is issued by the CTA that consumes it.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace mfi {
namespace tc {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
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
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Abort word of the calling CTA (shared memory, one per CTA of every kernel
// that uses it).  A role of the CTA that gives up a wait raises it, and the
// CTA's other roles stop at their next wait instead of waiting out the limit
// as well.  It belongs to this launch only: the device-wide error flag (`err`
// below) reports to the host and never stops a later call.  Every kernel that
// waits with mbar_wait clears the word from thread 0 (cta_abort_init) before
// its first __syncthreads.
__device__ __forceinline__ volatile int* cta_abort_word() {
  __shared__ int word;
  return &word;
}
__device__ __forceinline__ void cta_abort_init() { *cta_abort_word() = 0; }
__device__ __forceinline__ bool cta_aborted() { return *cta_abort_word() != 0; }
// Record `code` in the device error flag (first error wins) and stop this CTA.
__device__ __forceinline__ void cta_fail(int* err, int code) {
  if (err) atomicCAS(err, 0, code);
  *cta_abort_word() = 1;
}

// Bounded wait: gives up after kWaitLimitNs, records `code` (cta_fail) and
// returns false; it also returns false once another role of the CTA has
// failed.  The caller then skips its remaining work.  With err == nullptr it
// is a drain wait (for the CTA's own copies or MMAs still in flight after a
// failure): it ignores the abort word and only gives up at the limit.
// try_wait suspends in hardware between polls; the clock and the abort word
// are only consulted every 1024 polls, so a wait that is satisfied within a
// few microseconds costs nothing extra.
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err, int code) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 1023u) == 0) {
      if (err && cta_aborted()) return false;  // another role of this CTA failed
      if (globaltimer_ns() - t0 > kWaitLimitNs) {
        if (err) cta_fail(err, code);
        return false;
      }
    }
  }
}

// ---------------------------------------------------------------- TMA / bulk
__device__ __forceinline__ void tma_load_2d(void* dst, const void* tmap, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
      "l"(tmap), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
// A bulk copy whose lines L2 should drop first: for data streamed exactly
// once per call (the decode weight stream), so that what is reused across
// calls (the routers, the activations) stays resident.
__device__ __forceinline__ void bulk_load_stream(void* dst, const void* src, uint32_t bytes,
                                                 uint64_t* bar) {
  asm volatile(
      "{\n .reg .b64 pol;\n createpolicy.fractional.L2::evict_first.b64 pol, 1.0;\n"
      " cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1], %2, [%3], pol;\n}\n" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
// Bring [src, src + bytes) into L2 without waiting (bytes a multiple of 16).
__device__ __forceinline__ void prefetch_l2(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}
__device__ __forceinline__ void prefetch_tmap(const void* tmap) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(tmap) : "memory");
}

// ---------------------------------------------------------------- TMEM
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
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// ---------------------------------------------------------------- descriptors
// Shared-memory matrix descriptor (Blackwell version 1).
//   [0,14) start>>4  [16,30) LBO>>4  [32,46) SBO>>4  [46,48) version=1
//   [49,52) base offset=0  [52] LBO mode=0  [61,64) layout type
constexpr uint32_t kLayoutNone = 0;
constexpr uint32_t kLayoutSW128 = 2;
__device__ __forceinline__ uint64_t make_sdesc(uint32_t saddr, uint32_t lbo, uint32_t sbo,
                                               uint32_t layout) {
  uint64_t d = 0;
  d |= uint64_t((saddr >> 4) & 0x3FFFu);
  d |= uint64_t((lbo >> 4) & 0x3FFFu) << 16;
  d |= uint64_t((sbo >> 4) & 0x3FFFu) << 32;
  d |= 1ull << 46;
  d |= uint64_t(layout & 7u) << 61;
  return d;
}

// Instruction descriptor for kind::mxf4 (E2M1 x E2M1, UE8M0 scales, K = 64,
// both operands K-major, fp32 accumulate).
//   [4,6) B scale id  [7,10) A fmt=E2M1(1)  [10,13) B fmt=E2M1(1)
//   [17,23) N>>3  [23] scale fmt UE8M0(1)  [24,29) M>>4  [29,31) A scale id
__host__ __device__ constexpr uint32_t make_idesc_mxf4(int M, int N, int a_sf_id, int b_sf_id) {
  return (uint32_t(b_sf_id & 3) << 4) | (1u << 7) | (1u << 10) | (uint32_t(N >> 3) << 17) |
         (1u << 23) | (uint32_t(M >> 4) << 24) | (uint32_t(a_sf_id & 3) << 29);
}

// Instruction descriptor for kind::i8 (signed 8-bit A and B, K = 32, both
// operands K-major, s32 accumulate).
//   [4,6) D fmt=S32(2)  [7,10) A fmt=S8(1)  [10,13) B fmt=S8(1)  [17,23) N>>3
//   [24,29) M>>4
__host__ __device__ constexpr uint32_t make_idesc_i8(int M, int N) {
  return (2u << 4) | (1u << 7) | (1u << 10) | (uint32_t(N >> 3) << 17) | (uint32_t(M >> 4) << 24);
}

// ---------------------------------------------------------------- tcgen05 ops
// D(tmem) (+)= A(smem) . B(smem)^T, signed 8-bit operands, s32 accumulators.
__device__ __forceinline__ void mma_i8(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                       uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n}\n"
      ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Order this thread's generic-proxy shared-memory writes before later
// async-proxy accesses (tensor-core operand reads, TMA writes) of the CTA.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// D(tmem) (+)= A(smem) . B(smem)^T with block scales from TMEM.  The scale
// addresses carry the byte-in-word selector in bits 31:30, matching the
// sf_id fields of the instruction descriptor.
__device__ __forceinline__ void mma_mxf4(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                         uint32_t idesc, uint32_t accumulate, uint32_t tsfa,
                                         uint32_t tsfb) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::mxf4.block_scale.block32 [%0], %1, %2, %3, [%5], [%6], p;\n}\n"
      ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(tsfa), "r"(tsfb)
      : "memory");
}

// Copy one 512-byte scale-factor atom (32 rows x 16 bytes) from shared memory
// to 4 TMEM columns of lanes 0-31, replicated to lanes 32-127.
__device__ __forceinline__ void tmem_cp_sf(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc)
               : "memory");
}

// Arrive on an mbarrier once all prior tcgen05 operations of this thread finish.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

// Error-path drains, so that no copy or MMA of a CTA is still landing in its
// shared memory or TMEM when the CTA frees them and exits.
// Producer: the ring stages it filled, [issued - stages, issued), each
// complete on full[j % stages] in phase j / stages (later stages were never
// issued, earlier ones completed before their slots were refilled).
__device__ __forceinline__ void drain_ring(uint64_t* full, uint32_t stages, uint32_t issued) {
  for (uint32_t j = issued > stages ? issued - stages : 0u; j < issued; ++j)
    mbar_wait(&full[j % stages], (j / stages) & 1u, nullptr, 0);
}
// MMA issuer: commit whatever tcgen05 work it has issued to `bar` (an
// mbarrier of count 1 used for nothing else) and wait for it.
__device__ __forceinline__ void drain_mma(uint64_t* bar) {
  tc_commit(bar);
  mbar_wait(bar, 0, nullptr, 0);
}

// 32 lanes x 32 consecutive fp32 columns: thread i of the warp gets row
// (lane base + i), columns [col, col+32).
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,"
      "%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]),
        "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]),
        "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
// 32 lanes x 16 consecutive fp32 columns.
__device__ __forceinline__ void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,"
      "%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
// 32 lanes x 4 consecutive fp32 columns.
__device__ __forceinline__ void tmem_ld_32x32b_x4(uint32_t taddr, uint32_t (&r)[4]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(taddr));
}
// 32 lanes x 8 consecutive fp32 columns.
__device__ __forceinline__ void tmem_ld_32x32b_x8(uint32_t taddr, uint32_t (&r)[8]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// ---------------------------------------------------------------- peer flags
// System-scope flag traffic between GPUs.  A fence at system scope is costly
// (microseconds), so each CTA issues it once, from one thread, around relaxed
// flag accesses: a writer stores its data (all threads), bar.sync, then one
// thread fences and stores the flag (release pattern); a reader polls the
// flag with relaxed loads, fences once, then bar.sync before the data reads
// (acquire pattern).
__device__ __forceinline__ unsigned ld_relaxed_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_relaxed_sys(unsigned* p, unsigned v) {
  asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void fence_acq_rel_sys() {
  asm volatile("fence.acq_rel.sys;" ::: "memory");
}

// Programmatic dependent launch.  grid_dep_wait() returns once every grid
// this one depends on has completed and its memory is visible (immediately
// for a launch without the programmatic-serialisation attribute), so a kernel
// may run its prologue before it and must read upstream outputs only after
// it.  grid_dep_launch() lets the next launch in the stream start its
// prologue early; it carries no memory ordering.
__device__ __forceinline__ void grid_dep_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void grid_dep_launch() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ bool elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n .reg .b32 rx;\n .reg .pred px;\n elect.sync rx|px, 0xffffffff;\n"
      " selp.b32 %0, 1, 0, px;\n}\n"
      : "=r"(pred));
  return pred != 0;
}

}  // namespace tc
}  // namespace mfi
