// 5th-generation tensor-core building blocks (tcgen05, sm_100a): shared-memory operand
// layouts and descriptors, instruction descriptors, TMEM allocation / loads, mbarriers with
// bounded waits, and bulk (TMA) global -> shared copies.
//
// Operand layouts (bf16, no swizzle, canonical 8 x 16-byte core matrices).  An operand tile has
// R rows (the M or N index r) and Kd reduction columns (k), Kd a multiple of 16:
//   K-major  (k contiguous in a core-matrix row): byte (r/8)*16*Kd + (k/8)*128 + (r%8)*16 + (k%8)*2
//   MN-major (r contiguous in a core-matrix row): byte (r/8)*16*Kd + (k/8)*128 + (k%8)*16 + (r%8)*2
// i.e. the leading-dimension byte offset (between core matrices along k) is 128 and the stride
// byte offset (between core matrices along r) is 16*Kd in both; a 16-wide k step of one MMA
// starts 256 bytes further.  Accumulators are fp32 in TMEM: for M = 128, row m of D is TMEM
// lane m and column n is column (base + n); warp w of a CTA reads lanes 32*(w%4) .. +31.
#pragma once
#include <cstdint>

#include "common.cuh"

namespace gpa {
namespace tc5 {

// a bounded mbarrier wait gives up after this long (ns of %globaltimer): far above any
// legitimate wait of these kernels (microseconds), far below a hang
constexpr uint64_t kWaitNs = 1000000000ull;

GPA_DEV uint64_t gtime_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

GPA_DEV uint32_t saddr(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

__host__ __device__ inline uint32_t kmajor_off(int r, int k, int Kd) {
  return (uint32_t)((r >> 3) * (Kd * 16) + (k >> 3) * 128 + (r & 7) * 16 + (k & 7) * 2);
}
__host__ __device__ inline uint32_t mnmajor_off(int r, int k, int Kd) {
  return (uint32_t)((r >> 3) * (Kd * 16) + (k >> 3) * 128 + (k & 7) * 16 + (r & 7) * 2);
}

// Shared-memory matrix descriptor of the tile at shared address `a` (16-byte aligned) whose
// operand has Kd reduction columns, advanced to the 16-wide reduction step `ks`.
GPA_DEV uint64_t sdesc(uint32_t a, int Kd, int ks) {
  const uint32_t start = a + (uint32_t)ks * 256u;
  uint64_t d = (uint64_t)((start & 0x3FFFFu) >> 4);
  d |= (uint64_t)(128u >> 4) << 16;                 // leading byte offset (along k)
  d |= (uint64_t)(((uint32_t)Kd * 16u) >> 4) << 32;  // stride byte offset (along r)
  d |= (uint64_t)1 << 46;                           // descriptor version of sm_100
  return d;                                         // base offset 0, no swizzle
}

// Descriptor of a K-major tile X [rows r][cols c] (bytes kmajor_off(r, c, cols)) read as an
// MN-major operand whose reduction index is r and whose M / N index is c: core matrices of 8 r
// x 8 c, 128 bytes apart along c (stride byte offset) and 16 * cols bytes apart along r
// (leading byte offset); the 16-wide reduction step `ks` starts 32 * cols bytes further.
GPA_DEV uint64_t sdesc_mn_view(uint32_t a, int cols, int ks) {
  const uint32_t start = a + (uint32_t)ks * 32u * (uint32_t)cols;
  uint64_t d = (uint64_t)((start & 0x3FFFFu) >> 4);
  d |= (uint64_t)((16u * (uint32_t)cols) >> 4) << 16;  // leading byte offset (along r)
  d |= (uint64_t)(128u >> 4) << 32;                    // stride byte offset (along c)
  d |= (uint64_t)1 << 46;
  return d;
}

// Instruction descriptor of kind::f16 with bf16 A and B, fp32 D; a_mn / b_mn select MN-major.
__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N, bool a_mn, bool b_mn) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)a_mn << 15) | ((uint32_t)b_mn << 16) |
         ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// D[tmem] (+)= A * B for one 16-wide reduction step (issued by one thread).
GPA_DEV void mma(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, bool accumulate) {
  asm volatile(
      "{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(idesc), "r"((uint32_t)accumulate));
}

// Arrive on `bar` once every MMA this thread issued so far has completed.
GPA_DEV void commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   saddr(bar))
               : "memory");
}

GPA_DEV void fence_before_sync() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
GPA_DEV void fence_after_sync() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
// make this thread's generic-proxy shared-memory writes visible to the tensor core / TMA
GPA_DEV void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// ------------------------------------------------------------------ mbarriers
GPA_DEV void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(saddr(bar)), "r"(count) : "memory");
}
GPA_DEV void mbar_fence_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }

GPA_DEV bool mbar_try(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n.reg .pred p;\nmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      "selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(saddr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Wait for the phase with `parity` to complete; false when the wait gave up (kWaitNs).
GPA_DEV bool mbar_wait(uint64_t* bar, uint32_t parity) {
  if (mbar_try(bar, parity)) return true;
  const uint64_t t0 = gtime_ns();
  for (;;) {
    if (mbar_try(bar, parity)) return true;
    if (gtime_ns() - t0 > kWaitNs) return false;
  }
}

// expect `bytes` of bulk copies on `bar` (and arrive once)
GPA_DEV void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(saddr(bar)), "r"(bytes)
               : "memory");
}

// Bulk copy (TMA engine, no tensor map) of `bytes` from global to shared memory, completing
// on `bar`.  Both addresses 16-byte aligned, bytes a multiple of 16.  No multicast.
GPA_DEV void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          saddr(dst)),
      "l"(src), "r"(bytes), "r"(saddr(bar))
      : "memory");
}

// Bulk prefetch of `bytes` (a multiple of 16, address 16-byte aligned) from global memory into
// L2; nothing waits on it.
GPA_DEV void prefetch_l2(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// ------------------------------------------------------------------ TMEM
// Allocate `ncols` (a power of two >= 32) columns; one whole warp executes it; the address is
// written to shared memory at `slot`.
GPA_DEV void tmem_alloc(uint32_t* slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(saddr(slot)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
GPA_DEV void tmem_free(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

// 16 consecutive fp32 columns of this thread's TMEM lane (warp-collective, 32x32b shape);
// taddr carries the warp's lane quarter in its upper half.  Follow with tmem_wait_ld().
GPA_DEV void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}
// 16 lanes x 16 columns (16x256b shape, two repetitions along the columns), every thread of
// the warp holding data: thread t gets lane t/4, columns 2 (t%4) + {0, 1} in v[0..1] and lane
// 8 + t/4, the same columns, in v[2..3]; v[4..7] repeat that for columns 8 .. 15.  This is the
// layout of an M = 64 accumulator's rows 16 q .. 16 q + 15 (lanes 32 q .. 32 q + 15).
GPA_DEV void tmem_ld16x16(uint32_t taddr, float (&v)[8]) {
  uint32_t r[8];
  asm volatile(
      "tcgen05.ld.sync.aligned.16x256b.x2.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}

GPA_DEV void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// TMEM address of lane quarter (warp % 4), column `col`, from the allocation base.
GPA_DEV uint32_t tmem_at(uint32_t base, int col) {
  const uint32_t quarter = (threadIdx.x >> 5) & 3;
  return base + ((quarter * 32u) << 16) + (uint32_t)col;
}

}  // namespace tc5
}  // namespace gpa
