// Thin inline-PTX wrappers for the sm_100a features the MoE kernels use:
// mbarriers with bounded waits, TMA tile loads, cp.async row gathers,
// tcgen05 (TMEM allocation, UMMA issue/commit, TMEM loads) and cluster DSMEM.
//
// Every spin-wait in this library goes through wait_bounded(): after
// kWaitLimitNs of globaltimer time it ORs an error code into the status word
// and returns false, so a kernel that lost a producer ends instead of hanging.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#define B200_DEVI __device__ __forceinline__

namespace b200 {

// Status bits ORed into the device status word (see status.cu).
enum StatusBits : int {
  kStatusWaitTimeout = 1 << 0,   // an mbarrier wait ran past its limit
  kStatusBadTile = 1 << 1,       // tile bookkeeping found an impossible value
  kStatusBadIndex = 1 << 2,      // an expert index outside [0, E)
  kStatusPeerTimeout = 1 << 3,   // a wait for another rank's signal ran past its limit
};

constexpr unsigned long long kWaitLimitNs = 2000000000ull;  // 2 s

B200_DEVI uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

B200_DEVI uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

B200_DEVI uint32_t lane_id() {
  uint32_t l;
  asm volatile("mov.u32 %0, %%laneid;" : "=r"(l));
  return l;
}

// ---------------------------------------------------------------- mbarrier
B200_DEVI void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}

B200_DEVI void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

B200_DEVI void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

B200_DEVI void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(
                   smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

B200_DEVI bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Wait for the phase with the given parity to complete. Returns false (and
// records kStatusWaitTimeout) if it does not within kWaitLimitNs. Waiters off
// the critical path pass sleep_ns > 0 to back off between polls and leave
// issue slots to the warps doing the work.
B200_DEVI bool wait_bounded(uint64_t* bar, uint32_t parity, int* status, unsigned sleep_ns = 0) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 32; ++i) {
      if (sleep_ns) __nanosleep(sleep_ns);
      if (mbar_try_wait(bar, parity)) return true;
    }
    if (globaltimer_ns() - t0 > kWaitLimitNs) {
      if (status) atomicOr(status, kStatusWaitTimeout);
      return false;
    }
  }
}

B200_DEVI bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// wait_bounded for waiters on the critical path: polls with the non-blocking
// test_wait, so the thread sees the phase complete within one short sleep
// instead of after a suspended try_wait resumes; the sleep between polls
// leaves the scheduler's issue slots to the warps being waited for. Same
// limit and status on timeout.
B200_DEVI bool wait_spin(uint64_t* bar, uint32_t parity, int* status, unsigned sleep_ns = 20) {
  if (mbar_test_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 64; ++i) {
      __nanosleep(sleep_ns);
      if (mbar_test_wait(bar, parity)) return true;
    }
    if (globaltimer_ns() - t0 > kWaitLimitNs) {
      if (status) atomicOr(status, kStatusWaitTimeout);
      return false;
    }
  }
}

// Make this thread's generic-proxy shared-memory writes visible to the async
// proxy (TMA, tcgen05.mma) before signalling a barrier.
B200_DEVI void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------- TMA
// 2D tiled load of a box into shared memory; completion is reported as
// transaction bytes on `bar`. c0 is the innermost (contiguous) coordinate.
B200_DEVI void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}

// Contiguous global -> shared copy by the TMA engine (both addresses 16-byte
// aligned, bytes a multiple of 16), completing on `bar`'s transaction count.
B200_DEVI void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Four rows (arbitrary row coordinates r0..r3, box one row high) of a 2D
// tensor into four consecutive box rows of shared memory.
B200_DEVI void tma_gather4(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int r0, int r1,
                           int r2, int r3) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile::gather4.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6, %7}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(r0), "r"(r1), "r"(r2),
      "r"(r3)
      : "memory");
}

// Barrier among `count` threads (a multiple of 32) on hardware barrier `id`.
B200_DEVI void named_bar_sync(int id, int count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// Barrier among `count` threads that also ANDs `v` over them (all threads
// get the same result, so they agree on a decision before more barriers).
B200_DEVI bool named_bar_and(int id, int count, bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %3, 0;\n\t"
      "bar.red.and.pred q, %1, %2, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}\n"
      : "=r"(r)
      : "r"(id), "r"(count), "r"(static_cast<uint32_t>(v))
      : "memory");
  return r != 0;
}

// (a, b) *= s with one packed fp32 multiply (round to nearest, like two fmul).
B200_DEVI void mul2_f32(float& a, float& b, float s) {
  uint64_t x, y, r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(x) : "f"(a), "f"(b));
  asm("mov.b64 %0, {%1, %1};" : "=l"(y) : "f"(s));
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(x), "l"(y));
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(r));
}

B200_DEVI void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ---------------------------------------------------------------- cp.async
// 16-byte async copy global->shared; src_bytes == 0 zero-fills the chunk.
B200_DEVI void cp_async_16(uint32_t dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src),
               "r"(src_bytes)
               : "memory");
}
// 4- and 8-byte async copies global->shared (through L1); src_bytes == 0
// zero-fills the destination.
B200_DEVI void cp_async_4(uint32_t dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(dst), "l"(src), "r"(src_bytes)
               : "memory");
}
B200_DEVI void cp_async_8(uint32_t dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;" ::"r"(dst), "l"(src), "r"(src_bytes)
               : "memory");
}
B200_DEVI void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
B200_DEVI void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// ---------------------------------------------------------------- tcgen05
B200_DEVI void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
B200_DEVI void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
B200_DEVI void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
B200_DEVI void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
B200_DEVI void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Shared-memory matrix descriptor for a K-major operand stored in the
// 128-byte-swizzled canonical layout: rows of 128 bytes, 8-row (1024-byte)
// swizzle atoms stacked along M/N. The tile base must be 1024-byte aligned.
B200_DEVI uint64_t sdesc_k_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4);  // start address  [0,14)
  d |= static_cast<uint64_t>(1) << 16;                   // LBO (unused here) [16,30)
  d |= static_cast<uint64_t>(1024 >> 4) << 32;           // SBO = 1024 B  [32,46)
  d |= static_cast<uint64_t>(1) << 46;                   // descriptor version (sm_100)
  d |= static_cast<uint64_t>(2) << 61;                   // layout: 128-byte swizzle
  return d;
}

// As sdesc_k_sw128 for rows of 64 bytes in the 64-byte-swizzled canonical
// layout (16-byte chunk c of row r at c ^ ((r >> 1) & 3); 8-row atoms of 512
// bytes). The tile base must be 512-byte aligned.
B200_DEVI uint64_t sdesc_k_sw64(uint32_t saddr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4);  // start address  [0,14)
  d |= static_cast<uint64_t>(1) << 16;                   // LBO (unused here) [16,30)
  d |= static_cast<uint64_t>(512 >> 4) << 32;            // SBO = 512 B  [32,46)
  d |= static_cast<uint64_t>(1) << 46;                   // descriptor version (sm_100)
  d |= static_cast<uint64_t>(4) << 61;                   // layout: 64-byte swizzle
  return d;
}

// Instruction descriptor: kind::f8f6f4, A = B = E4M3, D = F32, both K-major.
__host__ __device__ constexpr uint32_t idesc_e4m3_f32(int M, int N) {
  return (1u << 4)                                  // D format F32 (A, B format 0 = E4M3)
         | (static_cast<uint32_t>(N >> 3) << 17)    // N / 8
         | (static_cast<uint32_t>(M >> 4) << 24);   // M / 16
}

// D (+)= A * B for one 32-byte (32 x e4m3) slice of K.
B200_DEVI void umma_e4m3(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Instruction descriptor: kind::f16, A = B = BF16, D = F32, both K-major.
__host__ __device__ constexpr uint32_t idesc_bf16_f32(int M, int N) {
  return (1u << 4)                                  // D format F32
         | (1u << 7)                                // A format BF16
         | (1u << 10)                               // B format BF16
         | (static_cast<uint32_t>(N >> 3) << 17)    // N / 8
         | (static_cast<uint32_t>(M >> 4) << 24);   // M / 16
}

B200_DEVI void umma_bf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// As umma_bf16 with the A operand (128 rows x 16 k, row r in TMEM lane r,
// two bf16 per 32-bit column) read from tensor memory at tmem_a.
B200_DEVI void umma_bf16_tmem_a(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc,
                                uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(tmem_d),
      "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// The four K = 16 MMAs of one 64-column k-block, in one asm block: A from
// tensor memory (columns a, a + 8, a + 16, a + 24) and B by its shared-memory
// descriptor (advanced 32 bytes per MMA); the first accumulates iff acc != 0.
B200_DEVI void umma_kblock_tmem_a(uint32_t d, uint32_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred q0, qt;\n\t.reg .b64 bd;\n\t.reg .b32 ta;\n\t"
      "setp.ne.b32 q0, %4, 0;\n\t"
      "setp.eq.b32 qt, %3, %3;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, q0;\n\t"
      "add.s64 bd, %2, 2;\n\tadd.u32 ta, %1, 8;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [ta], bd, %3, qt;\n\t"
      "add.s64 bd, bd, 2;\n\tadd.u32 ta, ta, 8;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [ta], bd, %3, qt;\n\t"
      "add.s64 bd, bd, 2;\n\tadd.u32 ta, ta, 8;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [ta], bd, %3, qt;\n\t}\n" ::"r"(d),
      "r"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}

// As umma_kblock_tmem_a with A by its shared-memory descriptor (advanced 32
// bytes per MMA, like B).
B200_DEVI void umma_kblock_smem_a(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred q0, qt;\n\t.reg .b64 ad, bd;\n\t"
      "setp.ne.b32 q0, %4, 0;\n\t"
      "setp.eq.b32 qt, %3, %3;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, q0;\n\t"
      "add.s64 ad, %1, 2;\n\tadd.s64 bd, %2, 2;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], ad, bd, %3, qt;\n\t"
      "add.s64 ad, ad, 2;\n\tadd.s64 bd, bd, 2;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], ad, bd, %3, qt;\n\t"
      "add.s64 ad, ad, 2;\n\tadd.s64 bd, bd, 2;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], ad, bd, %3, qt;\n\t}\n" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}

// Arrive once on `bar` when every tcgen05.mma issued so far by this thread
// has completed.
B200_DEVI void umma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

// 32 lanes x 16 consecutive 32-bit columns; thread i of the warp receives
// lane (base_lane + i). Must be followed by tmem_ld_wait() before use.
B200_DEVI void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}
// 32 lanes x 8 consecutive 32-bit columns (as tmem_ld16).
B200_DEVI void tmem_ld8(uint32_t taddr, uint32_t (&r)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
                 "=r"(r[7])
               : "r"(taddr)
               : "memory");
}
B200_DEVI void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }


// 32 consecutive 32-bit columns of this thread's TMEM lane (32x32b shape:
// warp w writes lanes 32 * (w % 4) .. + 31, thread i lane 32 * (w % 4) + i).
B200_DEVI void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, "
      "%28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),
      "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),
      "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
// 16 consecutive 32-bit columns of this thread's TMEM lane (32x32b shape).
B200_DEVI void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15, %16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}
B200_DEVI void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// ---------------------------------------------------------------- cluster
B200_DEVI uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
B200_DEVI void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\t"
               "barrier.cluster.wait.acquire.aligned;" ::
                   : "memory");
}
// Address of the same shared variable in CTA `rank` of this cluster.
B200_DEVI uint32_t mapa_shared(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}
B200_DEVI void st_cluster_f32x4(uint32_t addr, float a, float b, float c, float d) {
  asm volatile("st.shared::cluster.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "f"(a), "f"(b),
               "f"(c), "f"(d)
               : "memory");
}

// ---------------------------------------------------------------- register-operand MMA
// D += A (16 x 16 bf16, row-major fragments) x B (16 x 8 bf16, column-major
// fragments), fp32 accumulators. Lane l holds group g = l / 4, t = l % 4:
// a0 = A[g][2t..2t+1], a1 = A[g+8][2t..2t+1], a2 = A[g][2t+8..+9],
// a3 = A[g+8][2t+8..+9]; b0 = B[2t..2t+1][g], b1 = B[2t+8..+9][g];
// d0, d1 = D[g][2t..2t+1], d2, d3 = D[g+8][2t..2t+1].
B200_DEVI void mma_16816_bf16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                              uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
      "{%8, %9}, {%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// 16-byte global -> shared copy through L2 (cp.async.cg); the bytes past
// src_bytes (0..16) are zero-filled.
B200_DEVI void cp_async16(void* dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(src_bytes)
               : "memory");
}

// One arrival on `bar` once every cp.async this thread issued so far has
// landed (counts toward the barrier's expected arrivals).
B200_DEVI void cp_async_mbar_arrive(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}

B200_DEVI void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// ---------------------------------------------------------------- numerics
// Round-to-nearest-even float -> bf16, returned as a float holding the bf16
// value (exactly the value torch produces for `x.to(torch.bfloat16)`).
B200_DEVI float bf16r(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// Round-to-nearest-even float -> bf16 bits with integer ops (keeps the
// conversion pipe free; identical to cvt.rn for finite values and infinities).
B200_DEVI uint32_t bf16_rn_bits(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u + 0x7fffu + ((u >> 16) & 1u)) >> 16;
}
B200_DEVI float bf16_rn(float f) { return __uint_as_float(bf16_rn_bits(f) << 16); }

B200_DEVI uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

}  // namespace b200
