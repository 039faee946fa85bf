// Inline-PTX wrappers for the sm_100a features the tensor-core SSD uses:
// mbarriers with bounded waits, TMA tile loads, tcgen05 (UMMA) issue,
// commit and TMEM allocation / load / store, and the UMMA descriptors.
#pragma once

#include <cuda.h>
#include <stdint.h>

namespace alloy {
namespace tc {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}
// Tests the phase; if it is not complete the thread may sleep until it
// completes or `hint_ns` nanoseconds pass (so waiting warps do not take issue
// slots from working ones).  Callers bound the number of retries.
__device__ __forceinline__ uint32_t mbar_try_wait(uint32_t bar, uint32_t parity,
                                                  uint32_t hint_ns = 1000000u) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok;
}

// ---------------------------------------------------------------- TMA
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, uint32_t bar,
                                            int c0, int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1)
      : "memory");
}
// shared -> global tile store (writes outside the tensor's bounds are dropped),
// tracked by this thread's bulk async-groups
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, uint32_t src, int c0, int c1) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.tile.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(src), "r"(c0), "r"(c1)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// waits until at most N of this thread's bulk groups still read their shared memory
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
// waits until all of this thread's bulk groups have completed
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
// contiguous global -> shared copy (addresses 16-byte aligned, size a multiple of 16)
__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(bar)
      : "memory");
}
// contiguous range into L2 only
__device__ __forceinline__ void bulk_prefetch_l2(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(reinterpret_cast<uint64_t>(src)), "r"(bytes)
               : "memory");
}
// one cache line into L2
__device__ __forceinline__ void prefetch_l2(const void* p) {
  asm volatile("prefetch.global.L2 [%0];" ::"l"(reinterpret_cast<uint64_t>(p)));
}
// the same box into L2 only (no shared memory, no barrier)
__device__ __forceinline__ void tma_prefetch_3d(const CUtensorMap* map, int c0, int c1, int c2) {
  asm volatile("cp.async.bulk.prefetch.tensor.3d.L2.global.tile [%0, {%1, %2, %3}];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(c0), "r"(c1), "r"(c2)
               : "memory");
}
__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ---------------------------------------------------------------- programmatic dependent launch
// The kernel launched after this one with programmatic stream serialization
// may start once every CTA of this grid has executed pdl_trigger (or exited).
__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
// Blocks until the grid this one depends on (the previous kernel on the
// stream, when this one was launched with programmatic stream serialization)
// has completed and its memory operations are visible; returns at once for
// an ordinary launch.
__device__ __forceinline__ void pdl_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}

// ---------------------------------------------------------------- register split
// Executed by all four warps of a warpgroup at one program point.  The block
// is launched with R registers a thread; the decreases of some warpgroups must
// free at least what the increases of the others take.
template <int N>
__device__ __forceinline__ void reg_alloc() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}
template <int N>
__device__ __forceinline__ void reg_dealloc() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}

// ---------------------------------------------------------------- fences
__device__ __forceinline__ void fence_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// ---------------------------------------------------------------- TMEM
__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns; lane i of the warp gets row
// (warp quadrant * 32 + i) of the addressed columns.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
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
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),
      "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),
      "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
// 32 lanes x 16 columns
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
// 32 lanes x 8 columns
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&r)[8]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
      : "memory");
}
// 32 lanes x 8 columns
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t (&r)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
                 "=r"(r[7])
               : "r"(taddr));
}
// 32 lanes x 16 columns
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}
// wait for this thread's tensor-memory loads, with the registers of the
// load being waited on tied to the wait, so no use of them is scheduled
// before it (used when another load is issued ahead of the wait)
__device__ __forceinline__ void tmem_ld_wait_regs(uint32_t (&r)[16]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]),
                 "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]),
                 "+r"(r[13]), "+r"(r[14]), "+r"(r[15])
               :
               : "memory");
}
__device__ __forceinline__ void tmem_ld_wait_regs(uint32_t (&r)[8], uint32_t (&u)[8]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]),
                 "+r"(r[7]), "+r"(u[0]), "+r"(u[1]), "+r"(u[2]), "+r"(u[3]), "+r"(u[4]), "+r"(u[5]),
                 "+r"(u[6]), "+r"(u[7])
               :
               : "memory");
}
__device__ __forceinline__ void tmem_ld_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_st_wait() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// ---------------------------------------------------------------- UMMA
// D[tmem] (+)= A[smem] * B[smem], bf16 inputs, fp32 accumulation.
__device__ __forceinline__ void umma_bf16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                          uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Same with A read from tensor memory: `a_tmem` addresses the first of the
// K/2 columns holding A's rows as packed bf16 pairs (lane = row, low half =
// even k).
__device__ __forceinline__ void umma_bf16_ta(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc,
                                             uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Low and high 32-bit words of sw128_desc (below): the high word holds only
// the stride byte offset and the constant version / layout fields.
__device__ __forceinline__ uint32_t sw128_lo(uint32_t saddr, uint32_t lbo) {
  return ((saddr >> 4) & 0x3FFFu) | (((lbo >> 4) & 0x3FFFu) << 16);
}
__host__ __device__ constexpr uint32_t sw128_hi(uint32_t sbo) {
  return ((sbo >> 4) & 0x3FFFu) | (1u << 14) | (2u << 29);
}

// A chain of 4 or 8 MMAs D (+)= A_i B_i in one asm block (one issue sequence
// for the issuing thread, no per-MMA descriptor arithmetic in C++).  The
// operands are SW128 descriptors given by their low words (sw128_lo) and
// constant high words (sw128_hi); operand i's start addresses are the first
// ones advanced by i * A_STEP / i * B_STEP (units of 16 bytes; the 14-bit
// start-address field cannot overflow for shared-memory addresses).  The
// first MMA accumulates when `acc0` is nonzero, every later one always.
template <int A_STEP, int B_STEP, uint32_t A_HI, uint32_t B_HI>
__device__ __forceinline__ void umma_bf16_chain4(uint32_t d_tmem, uint32_t alo, uint32_t blo, uint32_t idesc,
                                                 uint32_t acc0) {
  asm volatile(
      "{\n\t.reg .pred p, t;\n\t.reg .b32 al, bl;\n\t.reg .b64 a, b;\n\t"
      "setp.ne.b32 p, %4, 0;\n\tsetp.eq.u32 t, 0, 0;\n\t"
      "mov.b64 a, {%1, %7};\n\tmov.b64 b, {%2, %8};\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], a, b, %3, p;\n\t"
      "add.u32 al, %1, %5;\n\tadd.u32 bl, %2, %6;\n\t"
      "mov.b64 a, {al, %7};\n\tmov.b64 b, {bl, %8};\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], a, b, %3, t;\n\t"
      "add.u32 al, al, %5;\n\tadd.u32 bl, bl, %6;\n\t"
      "mov.b64 a, {al, %7};\n\tmov.b64 b, {bl, %8};\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], a, b, %3, t;\n\t"
      "add.u32 al, al, %5;\n\tadd.u32 bl, bl, %6;\n\t"
      "mov.b64 a, {al, %7};\n\tmov.b64 b, {bl, %8};\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], a, b, %3, t;\n\t}" ::"r"(d_tmem),
      "r"(alo), "r"(blo), "r"(idesc), "r"(acc0), "n"(A_STEP), "n"(B_STEP), "r"(A_HI), "r"(B_HI)
      : "memory");
}
template <int A_STEP, int B_STEP, uint32_t A_HI, uint32_t B_HI>
__device__ __forceinline__ void umma_bf16_chain8(uint32_t d_tmem, uint32_t alo, uint32_t blo, uint32_t idesc,
                                                 uint32_t acc0) {
  umma_bf16_chain4<A_STEP, B_STEP, A_HI, B_HI>(d_tmem, alo, blo, idesc, acc0);
  umma_bf16_chain4<A_STEP, B_STEP, A_HI, B_HI>(d_tmem, alo + 4 * A_STEP, blo + 4 * B_STEP, idesc, 1);
}
// 8 MMAs with A read from tensor memory: A_i at a_tmem + i * A_COLS columns,
// B_i's start address advanced by i * B_STEP; the first accumulates when acc0 != 0.
template <int A_COLS, int B_STEP, uint32_t B_HI>
__device__ __forceinline__ void umma_bf16_ta_chain8(uint32_t d_tmem, uint32_t a_tmem, uint32_t blo, uint32_t idesc,
                                                    uint32_t acc0) {
  asm volatile(
      "{\n\t.reg .pred p, t;\n\t.reg .b32 a, bl;\n\t.reg .b64 b;\n\t"
      "setp.ne.b32 p, %4, 0;\n\tsetp.eq.u32 t, 0, 0;\n\t"
      "mov.b64 b, {%2, %7};\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], b, %3, p;\n\t"
      "mov.b32 a, %1;\n\tmov.b32 bl, %2;\n\t"
      "add.u32 a, a, %5;\n\tadd.u32 bl, bl, %6;\n\tmov.b64 b, {bl, %7};\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [a], b, %3, t;\n\t"
      "add.u32 a, a, %5;\n\tadd.u32 bl, bl, %6;\n\tmov.b64 b, {bl, %7};\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [a], b, %3, t;\n\t"
      "add.u32 a, a, %5;\n\tadd.u32 bl, bl, %6;\n\tmov.b64 b, {bl, %7};\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [a], b, %3, t;\n\t"
      "add.u32 a, a, %5;\n\tadd.u32 bl, bl, %6;\n\tmov.b64 b, {bl, %7};\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [a], b, %3, t;\n\t"
      "add.u32 a, a, %5;\n\tadd.u32 bl, bl, %6;\n\tmov.b64 b, {bl, %7};\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [a], b, %3, t;\n\t"
      "add.u32 a, a, %5;\n\tadd.u32 bl, bl, %6;\n\tmov.b64 b, {bl, %7};\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [a], b, %3, t;\n\t"
      "add.u32 a, a, %5;\n\tadd.u32 bl, bl, %6;\n\tmov.b64 b, {bl, %7};\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [a], b, %3, t;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "r"(blo), "r"(idesc), "r"(acc0), "n"(A_COLS), "n"(B_STEP), "r"(B_HI)
      : "memory");
}
// The same with 4 MMAs.
template <int A_COLS, int B_STEP, uint32_t B_HI>
__device__ __forceinline__ void umma_bf16_ta_chain4(uint32_t d_tmem, uint32_t a_tmem, uint32_t blo, uint32_t idesc,
                                                    uint32_t acc0) {
  asm volatile(
      "{\n\t.reg .pred p, t;\n\t.reg .b32 a, bl;\n\t.reg .b64 b;\n\t"
      "setp.ne.b32 p, %4, 0;\n\tsetp.eq.u32 t, 0, 0;\n\t"
      "mov.b64 b, {%2, %7};\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], b, %3, p;\n\t"
      "mov.b32 a, %1;\n\tmov.b32 bl, %2;\n\t"
      "add.u32 a, a, %5;\n\tadd.u32 bl, bl, %6;\n\tmov.b64 b, {bl, %7};\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [a], b, %3, t;\n\t"
      "add.u32 a, a, %5;\n\tadd.u32 bl, bl, %6;\n\tmov.b64 b, {bl, %7};\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [a], b, %3, t;\n\t"
      "add.u32 a, a, %5;\n\tadd.u32 bl, bl, %6;\n\tmov.b64 b, {bl, %7};\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [a], b, %3, t;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "r"(blo), "r"(idesc), "r"(acc0), "n"(A_COLS), "n"(B_STEP), "r"(B_HI)
      : "memory");
}

// Arrive once on an mbarrier when all previously issued tcgen05.mma of this
// thread have completed.
__device__ __forceinline__ void umma_commit(uint32_t bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
      : "memory");
}

// Shared-memory matrix descriptor for a 128-byte-swizzled operand tile
// (sm_100 format: start, leading and stride byte offsets in 16-byte units,
// version 1 at bit 46, layout SWIZZLE_128B = 2 at bits 61-63).  The tile's
// 1024-byte swizzle atoms must be 1024-byte aligned.
//  K-major  (K contiguous): rows of 128 bytes, 8-row atoms every `sbo` bytes.
//  MN-major (M/N contiguous): 64-element rows along M/N, 8 K-rows per atom,
//           K-atoms every `sbo` bytes, M/N atoms every `lbo` bytes.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(2) << 61;
  return d;
}

// Instruction descriptor of tcgen05.mma.kind::f16 with bf16 A/B and fp32 D.
// a_mn / b_mn select MN-major (transposed) operands.
__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N, int a_mn, int b_mn) {
  return (1u << 4)                                    // D format f32
         | (1u << 7)                                  // A format bf16
         | (1u << 10)                                 // B format bf16
         | (static_cast<uint32_t>(a_mn) << 15)        // A major
         | (static_cast<uint32_t>(b_mn) << 16)        // B major
         | (static_cast<uint32_t>(N >> 3) << 17)      // N / 8
         | (static_cast<uint32_t>(M >> 4) << 24);     // M / 16
}

// ---------------------------------------------------------------- math
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float tanh_approx(float x) {
  float y;
  asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
// silu(x) = x * sigmoid(x), sigmoid(x) = 0.5 + 0.5 tanh(x / 2)
__device__ __forceinline__ float silu_fast(float x) {
  return x * fmaf(0.5f, tanh_approx(0.5f * x), 0.5f);
}
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}
__device__ __forceinline__ float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

// ---------------------------------------------------------------- f32 pairs
// Two fp32 values in one 64-bit register pair, for the sm_100 packed
// fma/mul.f32x2 instructions (two IEEE fp32 operations per instruction).
__device__ __forceinline__ uint64_t f2_pack(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1,%2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void f2_unpack(uint64_t v, float& lo, float& hi) {
  asm("mov.b64 {%0,%1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
__device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t f2_splat(float x) { return f2_pack(x, x); }
// a bf16 pair (low half = first element) as an f32 pair
__device__ __forceinline__ uint64_t f2_from_bf2(uint32_t w) {
  return f2_pack(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
}
__device__ __forceinline__ uint32_t f2_to_bf2(uint64_t v) {
  float lo, hi;
  f2_unpack(v, lo, hi);
  return pack_bf16x2(lo, hi);
}
// silu of both halves: x * (0.5 + 0.5 tanh(x / 2))
__device__ __forceinline__ uint64_t f2_silu(uint64_t x) {
  const uint64_t half = f2_splat(0.5f);
  float a, b;
  f2_unpack(f2_mul(x, half), a, b);
  const uint64_t th = f2_pack(tanh_approx(a), tanh_approx(b));
  return f2_mul(x, f2_fma(th, half, half));
}

}  // namespace tc
}  // namespace alloy
