// Thin wrappers over the sm_100a instructions used by the tensor-core kernels:
// mbarriers (with bounded waits), TMA tensor / bulk copies, and tcgen05 (TMEM
// allocation, UMMA issue/commit, TMEM loads/stores, fences), plus the UMMA
// shared-memory and instruction descriptors.
//
// Descriptor formats (PTX ISA "tcgen05 matrix descriptors"; the same bit layout
// CUTLASS's UMMA::SmemDescriptor / InstrDescriptor encode):
//   smem descriptor: [0,14) start address >> 4, [16,30) leading byte offset >> 4,
//                    [32,46) stride byte offset >> 4, [46,48) version = 1,
//                    [49,52) base offset, [61,64) layout (2 = 128-byte swizzle)
//   instr descriptor (kind::f16): [4,6) D format (1 = f32), [7,10) A format,
//                    [10,13) B format (1 = bf16), [15] A major, [16] B major
//                    (0 = K-major, 1 = MN-major), [17,23) N >> 3, [24,29) M >> 4
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace kvs {
namespace sm100 {

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ------------------------------------------------------------------ mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(smem_addr(bar)), "r"(count));
}
__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;\n" ::);
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(smem_addr(bar)) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(smem_addr(bar)), "r"(bytes)
               : "memory");
}
// try_wait with a suspend-time hint: a waiting thread sleeps until the phase
// completes or about `hint_ns` nanoseconds pass, instead of spinning on issue slots.
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity, uint32_t hint_ns = 100000) {
  uint32_t ok;
  asm volatile(
      "{\n.reg .pred p;\n"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n"
      "selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}
// Wait for phase `parity` of `bar` to complete, giving up after `limit` suspended polls.
// Returns false on timeout; the caller records an error and winds down instead of hanging.
// An unanswered poll lasts ~4 us on B200 (the 100 us hint is an upper bound the hardware does
// not reach), so the default bound is ~1.6 s.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, const volatile int* abort_flag,
                                          uint32_t limit = 400000) {
  for (uint32_t i = 0; i < limit; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if (abort_flag && *abort_flag) return false;
  }
  return false;
}

// try_wait without a suspend hint (the hardware's default time slice)
__device__ __forceinline__ bool mbar_try_wait_default(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n.reg .pred p;\n"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      "selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Latency-critical wait: default time slices, bounded by `limit` polls.  An unanswered poll
// lasts ~4 us on B200, so the default bound is ~2 s.
__device__ __forceinline__ bool mbar_wait_fast(uint64_t* bar, uint32_t parity, const volatile int* abort_flag,
                                               uint32_t limit = 1u << 19) {
  for (uint32_t i = 0; i < limit; ++i) {
    if (mbar_try_wait_default(bar, parity)) return true;
    if (abort_flag && *abort_flag) return false;
  }
  return false;
}

// 2^x on the MUFU unit (hardware approximation, flush-to-zero; 2^-inf = +0)
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;\n" : "=f"(y) : "f"(x));
  return y;
}

// Packed fp32 pairs (sm_100 .f32x2 forms): one instruction for two lanes of work.
// (d0, d1) = (a0, a1) * b + c
__device__ __forceinline__ void ffma2(float& d0, float& d1, float a0, float a1, float b, float c) {
  asm("{\n.reg .b64 a, b, c, d;\n"
      "mov.b64 a, {%2, %3};\n"
      "mov.b64 b, {%4, %4};\n"
      "mov.b64 c, {%5, %5};\n"
      "fma.rn.f32x2 d, a, b, c;\n"
      "mov.b64 {%0, %1}, d;\n}\n"
      : "=f"(d0), "=f"(d1)
      : "f"(a0), "f"(a1), "f"(b), "f"(c));
}
// (s0, s1) += (a0, a1)
__device__ __forceinline__ void fadd2(float& s0, float& s1, float a0, float a1) {
  asm("{\n.reg .b64 a, s;\n"
      "mov.b64 a, {%2, %3};\n"
      "mov.b64 s, {%0, %1};\n"
      "add.rn.f32x2 s, s, a;\n"
      "mov.b64 {%0, %1}, s;\n}\n"
      : "+f"(s0), "+f"(s1)
      : "f"(a0), "f"(a1));
}

// (d0, d1) = (a0, a1) * b + (c0, c1)
__device__ __forceinline__ void ffma2v(float& d0, float& d1, float a0, float a1, float b, float c0, float c1) {
  asm("{\n.reg .b64 a, b, c, d;\n"
      "mov.b64 a, {%2, %3};\n"
      "mov.b64 b, {%4, %4};\n"
      "mov.b64 c, {%5, %6};\n"
      "fma.rn.f32x2 d, a, b, c;\n"
      "mov.b64 {%0, %1}, d;\n}\n"
      : "=f"(d0), "=f"(d1)
      : "f"(a0), "f"(a1), "f"(b), "f"(c0), "f"(c1));
}
// (d0, d1) = ((a0, a1) + (b0, b1)) * (c0, c1), each step rounded as in scalar code
__device__ __forceinline__ void addmul2(float& d0, float& d1, float a0, float a1, float b0, float b1, float c0,
                                        float c1) {
  asm("{\n.reg .b64 a, b, c, d;\n"
      "mov.b64 a, {%2, %3};\n"
      "mov.b64 b, {%4, %5};\n"
      "mov.b64 c, {%6, %7};\n"
      "add.rn.f32x2 d, a, b;\n"
      "mul.rn.f32x2 d, d, c;\n"
      "mov.b64 {%0, %1}, d;\n}\n"
      : "=f"(d0), "=f"(d1)
      : "f"(a0), "f"(a1), "f"(b0), "f"(b1), "f"(c0), "f"(c1));
}

// max of three (sm_100 three-input form)
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;\n" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// Per-warpgroup register budgets (all four warps of a warpgroup execute the same one).
// The sum over warpgroups must stay within the registers the block was launched with.
template <uint32_t R> __device__ __forceinline__ void regs_dealloc() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;\n" ::"n"(R));
}
template <uint32_t R> __device__ __forceinline__ void regs_alloc() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;\n" ::"n"(R));
}

// ------------------------------------------------------------------ TMA
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int x, int y, int z, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];\n" ::
          "r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_addr(bar))
      : "memory");
}
// Pull a box of a tiled tensor into L2 ahead of its load (no shared memory, no barrier)
__device__ __forceinline__ void tma_prefetch_3d(const CUtensorMap* map, int x, int y, int z) {
  asm volatile("cp.async.bulk.prefetch.tensor.3d.L2.global [%0, {%1, %2, %3}];\n" ::"l"(reinterpret_cast<uint64_t>(map)),
               "r"(x), "r"(y), "r"(z)
               : "memory");
}
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(
                   smem_addr(dst)),
               "l"(src), "r"(bytes), "r"(smem_addr(bar))
               : "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
}

// ------------------------------------------------------------------ tcgen05
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(smem_addr(dst_smem)),
               "r"(ncols));
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::);
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(taddr), "r"(ncols));
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory"); }

// D[tmem] (+)= A[smem] * B[smem]^T, one UMMA (M x N x 16 for bf16)
__device__ __forceinline__ void umma_bf16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n.reg .pred p;\n"
      "setp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate));
}
// D[tmem] (+)= A[tmem] * B[smem]^T: A (M x 16, bf16) from TMEM, lane = row, two consecutive
// K elements per 32-bit column (the lower half holds the even one)
__device__ __forceinline__ void umma_bf16_tmem_a(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                                 uint32_t accumulate) {
  asm volatile(
      "{\n.reg .pred p;\n"
      "setp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate));
}
// arrive on `bar` when every tcgen05 op issued so far by this thread has completed
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(smem_addr(bar))
               : "memory");
}

// Warp-collective forms: the whole (converged) warp executes them with warp-uniform
// operands and one elected lane issues the instruction.  Keeping the issuing code
// warp-uniform lets the compiler hold descriptors in uniform registers, so an UMMA
// costs a few issue cycles instead of a register-to-uniform transfer each.
// The K-step offsets are added inside the instruction block: A_OFF / B_OFF (compile-time)
// go to the descriptors' start-address fields (byte offset >> 4; a TMEM column for an A
// operand in TMEM), so the compiler cannot hoist one 64-bit descriptor per step out of the
// tile loop and run short of registers.
template <uint32_t A_OFF, uint32_t B_OFF>
__device__ __forceinline__ void umma_bf16_warp_at(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                                  uint32_t accumulate) {
  asm volatile(
      "{\n.reg .pred p, e;\n.reg .b64 a, b;\n"
      "add.s64 a, %1, %5;\n"
      "add.s64 b, %2, %6;\n"
      "elect.sync _|e, 0xffffffff;\n"
      "setp.ne.b32 p, %4, 0;\n"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], a, b, %3, p;\n}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "n"(A_OFF), "n"(B_OFF));
}
template <uint32_t A_COL, uint32_t B_OFF>
__device__ __forceinline__ void umma_bf16_tmem_a_warp_at(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                                         uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n.reg .pred p, e;\n.reg .b32 a;\n.reg .b64 b;\n"
      "add.u32 a, %1, %5;\n"
      "add.s64 b, %2, %6;\n"
      "elect.sync _|e, 0xffffffff;\n"
      "setp.ne.b32 p, %4, 0;\n"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [a], b, %3, p;\n}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate), "n"(A_COL), "n"(B_OFF));
}
__device__ __forceinline__ void umma_commit_warp(uint64_t* bar) {
  asm volatile(
      "{\n.reg .pred e;\n"
      "elect.sync _|e, 0xffffffff;\n"
      "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n}\n" ::"r"(smem_addr(bar))
      : "memory");
}

#define KVS_R32(r)                                                                                              \
  "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),   \
      "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),    \
      "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),   \
      "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
#define KVS_W32(r)                                                                                           \
  "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]), \
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]),          \
      "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]),         \
      "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])

// 32 consecutive 32-bit TMEM columns of this thread's lane (warp-collective)
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,"
      "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n"
      : KVS_R32(r)
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,"
      "%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};\n" ::"r"(taddr),
      KVS_W32(r)
      : "memory");
}
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};\n" ::"r"(
          taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;\n" ::: "memory"); }

// ------------------------------------------------------------------ CTA pairs (cta_group::2)
// Two CTAs of a 2-CTA cluster work as one MMA unit: the even CTA issues M = 256 UMMAs whose
// A rows and B columns come half from each CTA's shared memory (same offsets), and whose
// accumulator rows 0..127 / 128..255 land in the even / odd CTA's TMEM.
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;\n" : "=r"(r));
  return r;
}
// every thread of both CTAs; orders shared-memory writes (barrier inits) across the cluster
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;\n" ::: "memory");
}
// the shared::cluster address of the same shared-memory offset in CTA `rank` of the cluster
__device__ __forceinline__ uint32_t mapa_shared(const void* p, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;\n" : "=r"(r) : "r"(smem_addr(p)), "r"(rank));
  return r;
}
// arrive on a barrier given by its shared::cluster address (possibly the peer CTA's).  The
// arrivals order tcgen05 work (after tcgen05.fence::before_thread_sync), not memory writes, so
// the default release scope is used: a cluster-scope release costs about a thousand cycles.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t bar_cluster_addr) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];\n" ::"r"(bar_cluster_addr) : "memory");
}
// 2-D tiled TMA load into this CTA's shared memory whose completion is counted on a barrier
// of either CTA of the pair (shared::cluster address); each CTA loads only its own tile.
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* map, int x, int y,
                                                 uint32_t bar_cluster_addr) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
      "[%4];\n" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar_cluster_addr)
      : "memory");
}
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(smem_addr(dst_smem)),
               "r"(ncols));
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;\n" ::);
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;\n" ::"r"(taddr), "r"(ncols));
}
// D (+)= A * B^T over the pair, both operands from shared memory (warp-collective, one lane
// issues); A_OFF / B_OFF are added to the descriptors' start-address fields
template <uint32_t A_OFF, uint32_t B_OFF>
__device__ __forceinline__ void umma_pair_warp_at(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                                  uint32_t accumulate) {
  asm volatile(
      "{\n.reg .pred p, e;\n.reg .b64 a, b;\n"
      "add.s64 a, %1, %5;\n"
      "add.s64 b, %2, %6;\n"
      "elect.sync _|e, 0xffffffff;\n"
      "setp.ne.b32 p, %4, 0;\n"
      "@e tcgen05.mma.cta_group::2.kind::f16 [%0], a, b, %3, p;\n}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "n"(A_OFF), "n"(B_OFF));
}
// arrive once on the barrier at shared::cluster address `bar` (this CTA's or the peer's) when
// this thread's pair UMMAs so far have completed (warp-collective, one lane issues)
__device__ __forceinline__ void umma_commit_pair_warp(uint32_t bar_cluster_addr) {
  asm volatile(
      "{\n.reg .pred e;\n"
      "elect.sync _|e, 0xffffffff;\n"
      "@e tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];\n}\n" ::"r"(bar_cluster_addr)
      : "memory");
}

// ------------------------------------------------------------------ descriptors
// K-major operand, 128-byte swizzle: rows of 128 B (64 bf16 of K), 8-row atoms
// 1024 B apart (SBO); tiles of 64 K-columns are separate regions (the caller
// offsets the start address).  Start address must sit in a 1024-byte aligned atom.
__device__ __forceinline__ uint64_t desc_kmajor_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)1 << 16;               // LBO (unused for swizzled K-major)
  d |= (uint64_t)(1024 >> 4) << 32;     // SBO: next 8-row atom
  d |= (uint64_t)1 << 46;               // version
  d |= (uint64_t)2 << 61;               // SWIZZLE_128B
  return d;
}
// MN-major operand, 128-byte swizzle: rows of 128 B hold 64 consecutive MN elements
// of one K index; 8 K-rows form a 1024-byte atom; SBO = next 8 K-rows,
// LBO = next 64 MN elements.
__device__ __forceinline__ uint64_t desc_mnmajor_sw128(uint32_t saddr, uint32_t lbo_bytes) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)(1024 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}
// bf16 x bf16 -> f32, M x N, A K-major, B K-major (b_mn = 0) or MN-major (b_mn = 1)
__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N, int b_mn) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)b_mn << 16) | ((uint32_t)(N >> 3) << 17) |
         ((uint32_t)(M >> 4) << 24);
}
// f16 x f16 -> f32 (A and B format fields 0), otherwise as idesc_bf16
__host__ __device__ constexpr uint32_t idesc_f16(int M, int N, int b_mn) {
  return (1u << 4) | ((uint32_t)b_mn << 16) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

}  // namespace sm100
}  // namespace kvs
