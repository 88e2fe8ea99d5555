// Thin inline-PTX layer for sm_100a: mbarriers, TMA tensor loads, tcgen05
// (TMEM allocation, UMMA issue/commit, TMEM loads/stores) and the bounded-wait
// watchdog every pipelined kernel in this library uses.
//
// Nothing here issues a multicast load: every TMA copy reads this GPU's own
// memory into this CTA's shared memory.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <stdint.h>

namespace tt {

// ---------------------------------------------------------------------------
// Device error word layout (written by kernels, read back by the host).
// ---------------------------------------------------------------------------
constexpr unsigned kDevErrTimeout = 0x10000u;  // | site id in the low 16 bits

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// Programmatic dependent launch.  A kernel launched with programmatic stream
// serialization may start while the previous kernel of the stream is still
// running; pdl_wait() blocks until that kernel has completed and its memory
// is visible (a no-op for an ordinary launch), so everything before it may
// only touch shared memory, TMEM and data that was final before the previous
// kernel started (weights).  pdl_trigger() lets the next kernel's CTAs start
// their own set-up; it is issued after pdl_wait(), so a kernel's successor
// can only start once the kernel's own predecessor is done.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

__device__ __forceinline__ unsigned long long globaltimer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

// Potentially blocking probe: the thread may be suspended (up to the hint,
// 1 ms) until the phase completes, so a waiting warp does not spin and take
// issue slots from the warps that do the work.
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(1000000u)
      : "memory");
  return ok != 0;
}

// Non-blocking probe of a phase (no suspend hint): used by roles that poll
// several pipelines and must never block on one while another could proceed.
__device__ __forceinline__ bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Every wait in this library is bounded.  A CTA-wide abort flag in shared
// memory lets the other roles of the same CTA stop promptly, and the global
// error word lets every later CTA of the grid (and of later launches, until the
// host clears it) skip its work instead of waiting out its own limit.
struct Watchdog {
  unsigned int* err;              // global error word (device memory)
  volatile int* abort;            // CTA-wide abort flag (shared memory)
  unsigned long long timeout_ns;  // per-wait limit
};

__device__ __forceinline__ bool grid_failed(const Watchdog& wd) {
  return *reinterpret_cast<volatile unsigned int*>(wd.err) != 0u;
}

__device__ __forceinline__ bool wait_slow(uint64_t* bar, uint32_t parity, const Watchdog& wd,
                                       uint32_t site) {
  const unsigned long long t0 = globaltimer_ns();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 4; ++i) {
      if (mbar_try_wait(bar, parity)) return true;
    }
    if (*wd.abort) return false;
    if (grid_failed(wd)) {
      *wd.abort = 1;
      return false;
    }
    if (globaltimer_ns() - t0 > wd.timeout_ns) {
      atomicCAS(wd.err, 0u, kDevErrTimeout | (site & 0xffffu));
      *wd.abort = 1;
      return false;
    }
  }
}

// Single-thread wait (producer and MMA warps): straight to try_wait.
__device__ __forceinline__ bool wait_phase(uint64_t* bar, uint32_t parity, const Watchdog& wd,
                                           uint32_t site) {
  if (mbar_try_wait(bar, parity)) return true;
  return wait_slow(bar, parity, wd, site);
}

// Whole-warp wait: every lane observes the phase, then the warp reconverges
// and agrees on the outcome, so the warp-collective tcgen05.ld/st that follow
// always run converged.  It probes with the non-blocking test first: a
// try_wait that may suspend costs a couple of hundred cycles even when the
// phase completed long ago.
__device__ __forceinline__ bool warp_wait_phase(uint64_t* bar, uint32_t parity,
                                                const Watchdog& wd, uint32_t site) {
  const bool ok = mbar_test_wait(bar, parity) || wait_phase(bar, parity, wd, site);
  return __all_sync(0xffffffffu, ok);
}

// Bounded wait used only while tearing a CTA down after an abort: it ignores
// the abort flag and gives up after `limit_ns`.
__device__ __forceinline__ bool wait_drain(uint64_t* bar, uint32_t parity,
                                           unsigned long long limit_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = globaltimer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer_ns() - t0 > limit_ns) return false;
  }
  return true;
}

constexpr unsigned long long kDrainLimitNs = 100000000ull;  // 100 ms

// ---------------------------------------------------------------------------
// Proxy / TMEM fences
// ---------------------------------------------------------------------------
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// ---------------------------------------------------------------------------
// TMA (no multicast)
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* tm) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(tm)) : "memory");
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* tm, uint64_t* bar,
                                            int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(tm)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}

__device__ __forceinline__ void tma_load_2d_u32(uint32_t dst, const CUtensorMap* tm, uint64_t* bar,
                                                int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(tm)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* tm, uint64_t* bar,
                                            int c0, int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(tm)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

// TMA stores (shared -> global), tracked per issuing thread in bulk groups.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* tm, uint32_t src, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(tm)),
      "r"(src), "r"(c0), "r"(c1)
      : "memory");
}

__device__ __forceinline__ void tma_store_3d(const CUtensorMap* tm, uint32_t src, int c0, int c1,
                                             int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(tm)),
      "r"(src), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

__device__ __forceinline__ void bulk_commit_group() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

// Wait until at most N committed bulk groups of this thread still read shared memory.
template <int N>
__device__ __forceinline__ void bulk_wait_group_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

// Wait until every bulk group of this thread has fully completed.
__device__ __forceinline__ void bulk_wait_group_all() {
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

// ---------------------------------------------------------------------------
// tcgen05: TMEM allocation
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  __syncwarp();  // warp-collective: every lane must arrive converged
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

// ---------------------------------------------------------------------------
// tcgen05: UMMA descriptors
//
// Shared-memory matrix descriptor for a K-major operand tile written by TMA
// with a 32/64/128-byte swizzle (the swizzle width equals the tile's K extent
// in bytes per swizzle block).  Fields: start address >> 4 (bits 0-13),
// leading byte offset >> 4 (16-29; unused for swizzled K-major, set to 1),
// stride byte offset >> 4 (32-45; the distance between 8-row groups),
// descriptor version 1 (bits 46-47), layout/swizzle type (bits 61-63).
// ---------------------------------------------------------------------------
enum SwizzleKind : uint32_t { kSw32 = 6u, kSw64 = 4u, kSw128 = 2u };

__host__ __device__ constexpr uint32_t swizzle_kind_for_bytes(int row_bytes) {
  return row_bytes == 128 ? kSw128 : (row_bytes == 64 ? kSw64 : kSw32);
}

__device__ __forceinline__ uint64_t umma_sdesc(uint32_t saddr, uint32_t sbo_bytes,
                                               uint32_t swz) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>(1u) << 16;
  d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1u) << 46;
  d |= static_cast<uint64_t>(swz & 0x7u) << 61;
  return d;
}

// Instruction descriptor for kind::f16 with FP16 A/B, FP32 accumulator, both
// operands K-major: D format (bits 4-5) = F32, A/B format (7-9, 10-12) = F16,
// N >> 3 (bits 17-22), M >> 4 (bits 24-28).
__host__ __device__ constexpr uint32_t umma_idesc_f16_f32(int M, int N) {
  return (1u << 4) | (static_cast<uint32_t>(N >> 3) << 17) |
         (static_cast<uint32_t>(M >> 4) << 24);
}

__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                         uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Same MMA with the A operand in TMEM (lane = row; each 32-bit column holds two
// consecutive FP16 K elements, the lower k in the low half): one K = 16 step
// reads 8 columns starting at a_tmem.
__device__ __forceinline__ void umma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc,
                                            uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrives on `bar` once every tcgen05.mma issued so far by this thread is done.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

// ---------------------------------------------------------------------------
// tcgen05: TMEM <-> registers.  Shape 32x32b: warp w (w % 4 = q) reaches TMEM
// lanes 32q..32q+31; thread t gets lane 32q+t, register i = column base + i.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tmem_ld_x32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, "
      "[%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
        "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
        "=r"(r[31])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld_x16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_st_x32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
      "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(
          taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),
      "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),
      "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

__device__ __forceinline__ void tmem_ld_x8(uint32_t taddr, uint32_t (&r)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
                 "=r"(r[7])
               : "r"(taddr));
}
__device__ __forceinline__ void tmem_st_x8(uint32_t taddr, const uint32_t (&r)[8]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"r"(taddr),
               "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
               : "memory");
}

__device__ __forceinline__ void tmem_st_x16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15])
      : "memory");
}

__device__ __forceinline__ void tmem_ld_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// tcgen05.ld fills its destination registers asynchronously, until
// tcgen05.wait::ld.  These waits name the destination registers as in/out
// operands, so the compiler can neither read nor reuse them before the wait.
__device__ __forceinline__ void tmem_ld_wait_tied(uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.wait::ld.sync.aligned;"
      : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]),
        "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]),
        "+r"(r[14]), "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]),
        "+r"(r[21]), "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]),
        "+r"(r[28]), "+r"(r[29]), "+r"(r[30]), "+r"(r[31])
      :
      : "memory");
}

__device__ __forceinline__ void tmem_ld_wait_tied(uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.wait::ld.sync.aligned;"
      : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]),
        "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]),
        "+r"(r[14]), "+r"(r[15])
      :
      : "memory");
}

__device__ __forceinline__ void tmem_ld_wait_tied(uint32_t (&r)[8]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]),
                 "+r"(r[7])
               :
               : "memory");
}

// Load 32 / 16 columns and wait for them (registers tied to the wait).
__device__ __forceinline__ void tmem_ld_x32_sync(uint32_t taddr, uint32_t (&r)[32]) {
  tmem_ld_x32(taddr, r);
  tmem_ld_wait_tied(r);
}
__device__ __forceinline__ void tmem_ld_x16_sync(uint32_t taddr, uint32_t (&r)[16]) {
  tmem_ld_x16(taddr, r);
  tmem_ld_wait_tied(r);
}
__device__ __forceinline__ void tmem_st_wait() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// ---------------------------------------------------------------------------
// Small math helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Packed FP32 pair arithmetic (sm_100): one instruction for two lanes of work.
__device__ __forceinline__ uint64_t f2_pack(float lo, float hi) {
  return (static_cast<uint64_t>(__float_as_uint(hi)) << 32) | __float_as_uint(lo);
}
__device__ __forceinline__ float f2_lo(uint64_t v) { return __uint_as_float(static_cast<uint32_t>(v)); }
__device__ __forceinline__ float f2_hi(uint64_t v) { return __uint_as_float(static_cast<uint32_t>(v >> 32)); }
__device__ __forceinline__ uint64_t ffma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t fmul2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t fadd2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

// fma with the result clamped to [0, 1] (NaN -> 0).
__device__ __forceinline__ float fma_sat(float a, float b, float c) {
  float d;
  asm("fma.rn.sat.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// Inputs of the FMA-pipe exponential: y = saturate((x + 26) / 128), which
// clamps x to [-26, 102] in the same instruction that produces it (2^-26
// and smaller all round to FP16 zero; -inf gives y = 0).  The attention
// softmax folds its scale and row maximum into the same fma.
constexpr float kExp2YScale = 1.0f / 128.0f;
constexpr float kExp2YBias = 26.0f / 128.0f;

// 2^x for a pair of inputs on the FP32 pipe (no MUFU), x given as
// y = saturate((x + 26) / 128) (x = 128 y - 26; the rounding of y costs at
// most 2^-19 in x for x <= 8, 2^-18 below 64).  x = j + f with j = rint(x)
// (the 1.5*2^23 shifter, here with the -26 folded in) and |f| <= 1/2; 2^f
// comes from a degree-3 polynomial fitted for relative error on [-1/2, 1/2]
// by iteratively reweighted least squares (max 7.5e-5, a sixth of FP16's
// half-unit rounding error, which the probabilities receive next); 2^j is
// added into the exponent field.  The result is 2^max(x, -26); x must stay
// below 64.
__device__ __forceinline__ uint64_t exp2_pair_fma_y(uint64_t yy) {
  constexpr float kShift = 12582912.f - 26.f;  // 1.5*2^23 - 26, exact in FP32
  const uint64_t s128 = f2_pack(128.f, 128.f);
  const uint64_t t = ffma2(yy, s128, f2_pack(kShift, kShift));               // 1.5*2^23 + j
  const uint64_t u = ffma2(t, f2_pack(-1.f, -1.f), f2_pack(kShift, kShift));  // -26 - j, exact
  const uint64_t f = ffma2(yy, s128, u);                                     // x - j
  uint64_t q = ffma2(f2_pack(5.517162383e-02f, 5.517162383e-02f), f, f2_pack(2.426111251e-01f, 2.426111251e-01f));
  q = ffma2(q, f, f2_pack(6.932609677e-01f, 6.932609677e-01f));
  q = ffma2(q, f, f2_pack(9.999280572e-01f, 9.999280572e-01f));
  const uint32_t r0 = static_cast<uint32_t>(q) + (static_cast<uint32_t>(t) << 23);
  const uint32_t r1 = static_cast<uint32_t>(q >> 32) + (static_cast<uint32_t>(t >> 32) << 23);
  return (static_cast<uint64_t>(r1) << 32) | r0;
}
// The same from x directly.
__device__ __forceinline__ uint64_t exp2_pair_fma(uint64_t xx) {
  return exp2_pair_fma_y(f2_pack(fma_sat(f2_lo(xx), kExp2YScale, kExp2YBias),
                                 fma_sat(f2_hi(xx), kExp2YScale, kExp2YBias)));
}
// The same rounded to an FP16 pair.
__device__ __forceinline__ uint32_t exp2_pair_fma_f16(uint64_t xx) {
  const uint64_t y = exp2_pair_fma(xx);
  return pack_half2(f2_lo(y), f2_hi(y));
}

// 16-byte asynchronous global -> shared copy (LDGSTS); src_bytes = 0 fills zeros
// without reading global memory.
__device__ __forceinline__ void cp_async_16(uint32_t dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
// Bulk prefetch of [p, p + bytes) into L2 (bytes a multiple of 16).
__device__ __forceinline__ void prefetch_l2_bulk(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}
__device__ __forceinline__ uint4 ld_shared_v4(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr));
  return v;
}

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c,
                                             uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c),
               "r"(d)
               : "memory");
}

// Exact-erf GELU, x * Phi(x) with Phi the standard normal CDF (the form the
// reference evaluates: 0.5 * x * (1 + erf(x / sqrt(2)))), in FP32 as
//   GELU(x) = max(x, 0) - g,   g = z * Phi(-z) = z * exp(-z^2 / 2) * q(z),
//   z = |x|,  q(z) = Phi(-z) * exp(z^2 / 2) = erfcx(z / sqrt(2)) / 2,
// with exp through the MUFU exp2 and q a degree-8 polynomial in z, stored
// negated so that the last step is one FMA: GELU = fma(z * e, -q, max(x, 0)).
// The coefficients are an iteratively reweighted least-squares fit of q on
// Chebyshev nodes of [0, 7], weighted by z * exp(-z^2 / 2) (the factor that
// scales an error in q into g) over the error allowed at that point
// (1e-7 + 1e-4 |GELU|); evaluated in FP32 the GELU error is below 6.7e-6
// absolute and 6.5e-5 relative (near zero too), under a seventh of the FP16
// rounding the hidden activation receives next.  z is clamped to 12, past
// which exp(-z^2 / 2) is zero in FP32.
#define TT_GELU_Q8 -1.09531793e-05f
#define TT_GELU_Q7 2.38329638e-04f
#define TT_GELU_Q6 -2.26454716e-03f
#define TT_GELU_Q5 1.25273047e-02f
#define TT_GELU_Q4 -4.58019190e-02f
#define TT_GELU_Q3 1.20613545e-01f
#define TT_GELU_Q2 -2.45005265e-01f
#define TT_GELU_Q1 3.98084313e-01f
#define TT_GELU_Q0 -4.99967933e-01f
__device__ __forceinline__ float gelu_erf(float x) {
  const float z = fminf(fabsf(x), 12.0f);
  const float e = ex2_approx(z * z * -0.72134752044448170f);  // exp(-z^2/2)
  float q = fmaf(TT_GELU_Q8, z, TT_GELU_Q7);
  q = fmaf(q, z, TT_GELU_Q6);
  q = fmaf(q, z, TT_GELU_Q5);
  q = fmaf(q, z, TT_GELU_Q4);
  q = fmaf(q, z, TT_GELU_Q3);
  q = fmaf(q, z, TT_GELU_Q2);
  q = fmaf(q, z, TT_GELU_Q1);
  q = fmaf(q, z, TT_GELU_Q0);
  return fmaf(z * e, q, fmaxf(x, 0.0f));
}

// gelu_erf on a pair of inputs, on packed FP32 pairs (same coefficients and
// rounding steps, half the instructions).
__device__ __forceinline__ uint64_t gelu_erf_pair(uint64_t xx) {
  const float x0 = f2_lo(xx), x1 = f2_hi(xx);
  const uint64_t z = f2_pack(fminf(fabsf(x0), 12.0f), fminf(fabsf(x1), 12.0f));
  const uint64_t a = fmul2(fmul2(z, z), f2_pack(-0.72134752044448170f, -0.72134752044448170f));
  const uint64_t e = f2_pack(ex2_approx(f2_lo(a)), ex2_approx(f2_hi(a)));
#define TT_C2(c) f2_pack(c, c)
  uint64_t q = ffma2(TT_C2(TT_GELU_Q8), z, TT_C2(TT_GELU_Q7));
  q = ffma2(q, z, TT_C2(TT_GELU_Q6));
  q = ffma2(q, z, TT_C2(TT_GELU_Q5));
  q = ffma2(q, z, TT_C2(TT_GELU_Q4));
  q = ffma2(q, z, TT_C2(TT_GELU_Q3));
  q = ffma2(q, z, TT_C2(TT_GELU_Q2));
  q = ffma2(q, z, TT_C2(TT_GELU_Q1));
  q = ffma2(q, z, TT_C2(TT_GELU_Q0));
  return ffma2(fmul2(z, e), q, f2_pack(fmaxf(x0, 0.0f), fmaxf(x1, 0.0f)));
#undef TT_C2
}

}  // namespace tt
