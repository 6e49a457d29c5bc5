// Thin inline-PTX wrappers for the sm_100a features the fast kernels use:
// mbarriers (with bounded waits), TMA tile loads, tcgen05 MMA / TMEM
// load-store / alloc, and UMMA shared-memory + instruction descriptors.
#pragma once

#include <cuda.h>
#include <stdint.h>

namespace pnft {
namespace sm100 {

// A pipeline wait that has not completed after this long reports
// PNFT_DEV_WAIT_TIMEOUT and the kernel unwinds instead of hanging.
constexpr uint64_t kWaitTimeoutNs = 1000000000ull;  // 1 s

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Records a device-side failure in the caller's status word: a system-scope
// store, so the word may live in device memory or in pinned host memory mapped
// into the device's address space (the host then sees it without a copy).
__device__ __forceinline__ void report_status(int32_t* status, int32_t code) {
  if (status) asm volatile("st.relaxed.sys.global.s32 [%0], %1;" ::"l"(status), "r"(code) : "memory");
}

// Shared abort word of a CTA: the first role whose wait times out sets it, so
// every other role stops waiting on work that will never arrive.
struct Abort {
  volatile int* flag;   // shared memory
  int32_t* status;      // status word (device or mapped host memory; may be null)
};

// Bounded wait on the phase with the given parity; false if the CTA aborted.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, const Abort& ab) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 32; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (*ab.flag) return false;
    if (globaltimer() - t0 > kWaitTimeoutNs) {
      *ab.flag = 1;
      report_status(ab.status, PNFT_DEV_WAIT_TIMEOUT);
      return false;
    }
  }
}

// Warp-uniform bounded wait: every lane polls and each decision is a warp vote,
// so the warp never diverges (a lane-0 poll with the other lanes parked at a
// shuffle costs hundreds of cycles of reconvergence after the phase lands).
__device__ __forceinline__ bool warp_wait(uint32_t bar, uint32_t parity, const Abort& ab) {
  constexpr uint32_t kAll = 0xffffffffu;
  if (__any_sync(kAll, mbar_try_wait(bar, parity))) return true;
  const uint64_t t0 = globaltimer();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 8; ++i)
      if (__any_sync(kAll, mbar_try_wait(bar, parity))) return true;
    if (__any_sync(kAll, *ab.flag != 0)) return false;
    if (__any_sync(kAll, globaltimer() - t0 > kWaitTimeoutNs)) {
      if ((threadIdx.x & 31) == 0) {
        *ab.flag = 1;
        report_status(ab.status, PNFT_DEV_WAIT_TIMEOUT);
      }
      __syncwarp();
      return false;
    }
  }
}

// warp_wait on three phases at once (one poll and one vote per round).
__device__ __forceinline__ bool warp_wait3(uint32_t b0, uint32_t p0, uint32_t b1, uint32_t p1, uint32_t b2,
                                           uint32_t p2, const Abort& ab) {
  constexpr uint32_t kAll = 0xffffffffu;
  auto all3 = [&]() { return mbar_try_wait(b0, p0) && mbar_try_wait(b1, p1) && mbar_try_wait(b2, p2); };
  if (__any_sync(kAll, all3())) return true;
  const uint64_t t0 = globaltimer();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 8; ++i)
      if (__any_sync(kAll, all3())) return true;
    if (__any_sync(kAll, *ab.flag != 0)) return false;
    if (__any_sync(kAll, globaltimer() - t0 > kWaitTimeoutNs)) {
      if ((threadIdx.x & 31) == 0) {
        *ab.flag = 1;
        report_status(ab.status, PNFT_DEV_WAIT_TIMEOUT);
      }
      __syncwarp();
      return false;
    }
  }
}

// Wait that ignores the abort flag: used at teardown to let this CTA's own
// copies / MMAs land before its shared memory and TMEM are released.
__device__ __forceinline__ void drain_wait(uint32_t bar, uint32_t parity) {
  const uint64_t t0 = globaltimer();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer() - t0 > 50000000ull) return;  // 50 ms: far beyond any copy latency
  }
}

// ---------------------------------------------------------------- bulk (non-tensor) copies
// 1-D global -> shared copy completing on an mbarrier (16-byte aligned, size % 16 == 0).
__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "l"(src), "r"(bytes), "r"(bar)
               : "memory");
}
// 1-D shared -> global fp32 add-reduction, tracked by the bulk async-group of this thread.
__device__ __forceinline__ void bulk_reduce_add_f32(void* dst, uint32_t src, uint32_t bytes) {
  asm volatile("cp.reduce.async.bulk.global.shared::cta.bulk_group.add.f32 [%0], [%1], %2;" ::"l"(dst), "r"(src),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
// Order this thread's generic shared-memory writes before later async-proxy reads.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// One lane of a converged warp (the lowest active lane, so the same lane on
// every call with all 32 active): the issuer of tcgen05 MMAs and their commits.
__device__ __forceinline__ bool elect_one() {
  uint32_t pred;
  asm volatile(
      "{\n\t.reg .pred p;\n\t.reg .b32 r;\n\t"
      "elect.sync r|p, 0xffffffff;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(pred));
  return pred != 0;
}

// ---------------------------------------------------------------- named barriers
__device__ __forceinline__ void named_bar_sync(uint32_t id, uint32_t nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// ---------------------------------------------------------------- TMA
__device__ __forceinline__ void tma_load_4d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int c0, int c1,
                                            int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1)
      : "memory");
}
__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ---------------------------------------------------------------- tcgen05
__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Shared-memory matrix descriptors are passed as their low 32 bits (start
// address >> 4, leading-byte offset >> 4) and assembled with the constant high
// word inside the asm: every tile here is 128-byte swizzled with 1024-byte
// 8-row groups, and a 64-bit descriptor operand was seen to reach the tensor
// core without its high word in a register-tight build (MN-major B operands then
// read as unswizzled, repeating every 8 columns).
constexpr uint32_t kSw128DescHi = (1024u >> 4) | (1u << 14) | (2u << 29);  // SBO 1024, version 1, SWIZZLE_128B

// D[tmem] (+)= A[smem desc] * B[smem desc]
__device__ __forceinline__ void mma_ss(uint32_t d_tmem, uint32_t a_lo, uint32_t b_lo, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t.reg .b64 da, db;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "mov.b64 da, {%1, %5};\n\t"
      "mov.b64 db, {%2, %5};\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], da, db, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_lo), "r"(b_lo), "r"(idesc), "r"(accumulate), "r"(kSw128DescHi)
      : "memory");
}
// D[tmem] (+)= A[tmem] * B[smem desc]
__device__ __forceinline__ void mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint32_t b_lo, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t.reg .b64 db;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "mov.b64 db, {%2, %5};\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], db, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "r"(b_lo), "r"(idesc), "r"(accumulate), "r"(kSw128DescHi)
      : "memory");
}
// Arrive on `bar` once every tcgen05 op issued so far by this thread completes.
__device__ __forceinline__ void mma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

#define PNFT_R8(i) "=r"(r[i + 0]), "=r"(r[i + 1]), "=r"(r[i + 2]), "=r"(r[i + 3]), "=r"(r[i + 4]), "=r"(r[i + 5]), "=r"(r[i + 6]), "=r"(r[i + 7])
#define PNFT_W8(i) "r"(r[i + 0]), "r"(r[i + 1]), "r"(r[i + 2]), "r"(r[i + 3]), "r"(r[i + 4]), "r"(r[i + 5]), "r"(r[i + 6]), "r"(r[i + 7])

// TMEM loads. Each helper issues its tcgen05.ld and the tcgen05.wait::ld in ONE
// asm statement: the loaded registers are undefined until the wait, and with two
// statements the compiler may schedule their consumers in between.
#define PNFT_LD32 "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
#define PNFT_LD16 "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
#define PNFT_WAIT_LD "tcgen05.wait::ld.sync.aligned;"

// 32 lanes x 32 consecutive 32-bit columns -> r[0..31] of each thread (lane = row)
__device__ __forceinline__ void tmem_load32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(PNFT_LD32
               "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
               "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n\t" PNFT_WAIT_LD
               : PNFT_R8(0), PNFT_R8(8), PNFT_R8(16), PNFT_R8(24)
               : "r"(taddr)
               : "memory");
}
// 32 lanes x 16 consecutive 32-bit columns -> r[0..15]
__device__ __forceinline__ void tmem_load16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(PNFT_LD16 "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n\t" PNFT_WAIT_LD
               : PNFT_R8(0), PNFT_R8(8)
               : "r"(taddr)
               : "memory");
}
// two 16-column loads, one wait
__device__ __forceinline__ void tmem_load16x2(uint32_t ta, uint32_t (&r)[16], uint32_t tb, uint32_t (&q)[16]) {
  asm volatile(PNFT_LD16 "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%32];\n\t" PNFT_LD16
                         "{%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%33];\n\t" PNFT_WAIT_LD
               : PNFT_R8(0), PNFT_R8(8), "=r"(q[0]), "=r"(q[1]), "=r"(q[2]), "=r"(q[3]), "=r"(q[4]), "=r"(q[5]),
                 "=r"(q[6]), "=r"(q[7]), "=r"(q[8]), "=r"(q[9]), "=r"(q[10]), "=r"(q[11]), "=r"(q[12]), "=r"(q[13]),
                 "=r"(q[14]), "=r"(q[15])
               : "r"(ta), "r"(tb)
               : "memory");
}
// two 32-column loads, one wait
__device__ __forceinline__ void tmem_load32x2(uint32_t ta, uint32_t (&r)[32], uint32_t tb, uint32_t (&q)[32]) {
#define PNFT_Q8(i) "=r"(q[i + 0]), "=r"(q[i + 1]), "=r"(q[i + 2]), "=r"(q[i + 3]), "=r"(q[i + 4]), "=r"(q[i + 5]), "=r"(q[i + 6]), "=r"(q[i + 7])
  asm volatile(PNFT_LD32
               "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
               "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%64];\n\t" PNFT_LD32
               "{%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47,"
               "%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63}, [%65];\n\t" PNFT_WAIT_LD
               : PNFT_R8(0), PNFT_R8(8), PNFT_R8(16), PNFT_R8(24), PNFT_Q8(0), PNFT_Q8(8), PNFT_Q8(16), PNFT_Q8(24)
               : "r"(ta), "r"(tb)
               : "memory");
#undef PNFT_Q8
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      PNFT_W8(0), PNFT_W8(8), PNFT_W8(16), PNFT_W8(24)
      : "memory");
}
// 32 lanes x 16 consecutive columns <- r[0..15]
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      PNFT_W8(0), PNFT_W8(8)
      : "memory");
}
// 32 lanes x 8 consecutive columns <- r[0..7]
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&r)[8]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr), "r"(r[0]),
               "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
               : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

#undef PNFT_R8
#undef PNFT_W8
#undef PNFT_LD32
#undef PNFT_LD16
#undef PNFT_WAIT_LD

// ---------------------------------------------------------------- descriptors
// Low word of the UMMA shared-memory descriptor of a 128-byte-swizzled tile
// (tile base 1024-aligned): start>>4 in [0,14), LBO>>4 in [16,30); the high word
// (SBO>>4 = 64 in [32,46), version 1 at 46, layout SWIZZLE_128B = 2 in [61,64))
// is kSw128DescHi. A k-step adds (bytes >> 4) to the low word: shared addresses
// stay below 256 KB, so the start field never carries into LBO.
__device__ __forceinline__ uint32_t sw128_desc(uint32_t saddr, uint32_t lbo_bytes) {
  return ((saddr & 0x3FFFFu) >> 4) | (((lbo_bytes >> 4) & 0x3FFFu) << 16);
}

// kind::f16 instruction descriptor: f32 accumulate, A/B bf16 (fmt 1) or f16 (fmt 0),
// a_mn/b_mn = 1 for MN-major operands, N>>3 at bit 17, M>>4 at bit 24.
__host__ __device__ constexpr uint32_t idesc_f16(int M, int N, uint32_t ab_fmt, uint32_t a_mn, uint32_t b_mn) {
  return (1u << 4) | (ab_fmt << 7) | (ab_fmt << 10) | (a_mn << 15) | (b_mn << 16) | ((uint32_t)(N >> 3) << 17) |
         ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

__device__ __forceinline__ float max3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

}  // namespace sm100
}  // namespace pnft
