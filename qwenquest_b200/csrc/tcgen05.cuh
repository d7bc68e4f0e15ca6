// tcgen05 (fifth-generation tensor core) and mbarrier helpers shared by the
// kernels that run on the tensor cores (sm_100a): shared-memory matrix and
// instruction descriptors, MMA issue and commit, tensor-memory loads and
// stores, bounded mbarrier waits.
#pragma once

#include "common.cuh"

namespace qq {
namespace tc {

// Byte offset of 16-byte chunk `chunk` (0..15) of row `row` of a tile of
// 256-byte rows in the 128-byte swizzled layout: two 64-column blocks of
// 128-byte rows (`half` bytes apart), chunk c of row r at position
// c ^ (r mod 8) within its row.
__device__ __forceinline__ uint32_t sw128(int row, int chunk, int half) {
  return (uint32_t)((chunk >> 3) * half + row * 128 + (((chunk & 7) ^ (row & 7)) << 4));
}

// Shared-memory matrix descriptor (tcgen05): start address >> 4 in bits 0-13,
// leading byte offset >> 4 in 16-29, stride byte offset >> 4 in 32-45,
// version 1 in 46-47, swizzle mode in 61-63 (2 = 128-byte swizzle).
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
  return (uint64_t)((addr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46) | (2ull << 61);
}
// K-major operand in the 128-byte swizzled layout: 8-row groups of 128-byte
// rows 1024 bytes apart (a k-step of 16 bf16 adds 32 bytes to the start).
__device__ __forceinline__ uint64_t desc_k(uint32_t addr) { return smem_desc(addr, 16, 1024); }
// MN-major operand in the 128-byte swizzled layout: 64-element blocks of the
// MN dimension `block_bytes` apart, 8-row (K) groups 1024 bytes apart.
__device__ __forceinline__ uint64_t desc_mn(uint32_t addr, uint32_t block_bytes) {
  return smem_desc(addr, block_bytes, 1024);
}

// Instruction descriptor, kind::f16: fp32 accumulator (bits 4-5 = 1), A and B
// bf16 (bits 7-9, 10-12 = 1), A K-major (bit 15 = 0), B major in bit 16,
// N >> 3 in bits 17-22, M >> 4 in bits 24-28.
__host__ __device__ constexpr uint32_t instr_desc(uint32_t b_mn_major, uint32_t m, uint32_t n) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (b_mn_major << 16) | ((n >> 3) << 17) | ((m >> 4) << 24);
}

__device__ __forceinline__ void umma_bf16(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}
// The same with A (K-major, bf16 pairs) read from tensor memory at a_tmem.
__device__ __forceinline__ void umma_bf16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b, uint32_t idesc,
                                             uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}
// Four MMAs into one accumulator, issued back to back from one asm block: A
// and B descriptors advance by a_step / b_step (in 16-byte units) per MMA;
// the first MMA accumulates when acc != 0, the others always.
__device__ __forceinline__ void umma_bf16_x4(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t a_step,
                                             uint32_t b_step, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p, t;\n\t.reg .b64 a1, a2, a3, b1, b2, b3;\n\t"
      "setp.ne.b32 p, %5, 0;\n\tsetp.eq.b32 t, %5, %5;\n\t"
      "add.s64 a1, %1, %6;\n\tadd.s64 a2, a1, %6;\n\tadd.s64 a3, a2, %6;\n\t"
      "add.s64 b1, %2, %7;\n\tadd.s64 b2, b1, %7;\n\tadd.s64 b3, b2, %7;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], a1, b1, %3, t;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], a2, b2, %3, t;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], a3, b3, %3, t;\n\t}\n" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(idesc), "n"(0), "r"(acc), "l"((uint64_t)a_step), "l"((uint64_t)b_step)
      : "memory");
}
// The same with A read from tensor memory: its column advances by a_step per MMA.
__device__ __forceinline__ void umma_bf16_ts_x4(uint32_t d_tmem, uint32_t a_tmem, uint64_t b, uint32_t a_step,
                                                uint32_t b_step, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p, t;\n\t.reg .b32 a1, a2, a3;\n\t.reg .b64 b1, b2, b3;\n\t"
      "setp.ne.b32 p, %5, 0;\n\tsetp.eq.b32 t, %5, %5;\n\t"
      "add.u32 a1, %1, %6;\n\tadd.u32 a2, a1, %6;\n\tadd.u32 a3, a2, %6;\n\t"
      "add.s64 b1, %2, %7;\n\tadd.s64 b2, b1, %7;\n\tadd.s64 b3, b2, %7;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [a1], b1, %3, t;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [a2], b2, %3, t;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [a3], b3, %3, t;\n\t}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b), "r"(idesc), "n"(0), "r"(acc), "r"(a_step), "l"((uint64_t)b_step)
      : "memory");
}
// The mbarrier gets one arrival once every tcgen05 operation this thread issued before has completed.
__device__ __forceinline__ void umma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_async_shared() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}\n" ::"r"(bar) : "memory");
}
// One arrival on the mbarrier, made by the hardware once every cp.async this
// thread issued before has completed (counts against the barrier's expected
// arrivals).  The tensor core may read the copied data once the phase completes.
__device__ __forceinline__ void cp_async_arrive(uint32_t bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait for the phase of `bar` with parity `parity`.  False once the
// CTA has given up (this wait ran out, or another thread's did).
// With `drain` the wait ignores an earlier give-up (the last wait for the
// CTA's own MMAs before its tensor memory is freed).
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag, uint32_t* err,
                                          bool drain = false) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (;;) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort_flag && !drain) return false;
    if (globaltimer_ns() - t0 > kWaitLimitNs) {
      *abort_flag = 1;
      raise_error(err, QQ_DEV_ERR_TIMEOUT);
      return false;
    }
  }
}

#define QQ_R32(r) \
  "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), \
  "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),     \
  "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),    \
  "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
#define QQ_W32(r) \
  "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]), \
  "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),  \
  "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),  \
  "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])

// 32 consecutive fp32 columns of this thread's TMEM lane (the warp's 32 lanes).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,"
      "%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : QQ_R32(r)
      : "r"(taddr)
      : "memory");
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,"
      "%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      QQ_W32(r)
      : "memory");
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
// bf16 pair: lo in bits 0-15 (the lower address), hi in 16-31.
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem), "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void mbar_init_fence() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }

}  // namespace tc
}  // namespace qq
