// Shared device helpers for the Enilnets B200 attention kernels (sm_100a only).
//
// Everything here is a thin inline-PTX wrapper around one Blackwell feature:
// mbarriers, TMA tensor/bulk copies (each CTA loads its own tiles), tcgen05
// tensor-memory allocation / MMA / loads / stores, plus the device error word
// that every bounded wait reports into instead of trapping.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda.h>

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "enilnets_b200 kernels are written for sm_100a only"
#endif

namespace enl {

// ---------------------------------------------------------------------------
// Device error word. Kernels never trap: a failed bound check or a wait that
// ran out of time records a code here (first writer wins) and the kernel
// returns. The host reads and clears it through enl_device_error().
// ---------------------------------------------------------------------------
enum DeviceError : int {
  kDevOk = 0,
  kDevWaitTimeout = 1,     // an mbarrier wait exceeded its time budget
  kDevBadIndex = 2,        // an index (slot, gather row) was out of range
  kDevBadShape = 3,        // launch-time shape invariants violated
};

// Defined here: the library is built as a single translation unit (enl_lib.cu).
__device__ int g_device_error = 0;
__device__ int g_device_error_info = 0;

__device__ __forceinline__ void report_error(int code, int info) {
  if (atomicCAS(&g_device_error, 0, code) == 0) {
    g_device_error_info = info;
  }
}

// Wait budget for every spin on an mbarrier: about one second of wall time.
constexpr uint64_t kWaitBudgetNs = 1000ull * 1000ull * 1000ull;

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(
                   smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// try_wait with a suspend-time hint: a thread whose phase is not complete
// sleeps until it completes or `hint_ns` passes instead of polling, so
// waiting warps leave the issue slots to the warps that have work.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity,
                                                    uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}

// Bounded wait on `parity`. Returns false (after recording kDevWaitTimeout and
// raising *abort) when the budget runs out or when another role already
// aborted; the caller then stops issuing work and drains.
__device__ __forceinline__ bool mbar_wait_budget(uint64_t* bar, uint32_t parity,
                                                 volatile int* abort_flag, int site,
                                                 uint64_t budget_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
    if (mbar_try_wait_sleep(bar, parity, 20000)) return true;
    if (*abort_flag) return false;
    if (globaltimer_ns() - t0 > budget_ns) {
      report_error(kDevWaitTimeout, site);
      *abort_flag = 1;
      return false;
    }
  }
}

__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity,
                                          volatile int* abort_flag, int site) {
  return mbar_wait_budget(bar, parity, abort_flag, site, kWaitBudgetNs);
}

// Barrier over the first `threads` threads' warps that name barrier `id` (0 is
// __syncthreads).
__device__ __forceinline__ void named_bar_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// ---------------------------------------------------------------------------
// TMA tensor copies (global <-> shared, one CTA each) and bulk groups.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

__device__ __forceinline__ void tma_load_4d(void* smem_dst, const CUtensorMap* map, uint64_t* bar,
                                            int c0, int c1, int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2),
      "r"(c3)
      : "memory");
}

// shared -> global tensor store of one box (bulk-group completion). Its
// coordinates start inside the tensor (TMA drops the parts of the box past
// the tensor's extents).
__device__ __forceinline__ void tma_store_4d(const CUtensorMap* map, const void* smem_src, int c0,
                                             int c1, int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.global.shared::cta.tile.bulk_group [%0, {%2, %3, %4, %5}], [%1];"
      ::"l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(smem_src)), "r"(c0), "r"(c1), "r"(c2),
      "r"(c3)
      : "memory");
}
__device__ __forceinline__ void bulk_commit_group() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
// Wait until every committed bulk store has finished reading shared memory.
__device__ __forceinline__ void bulk_wait_read_all() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
// Wait until every committed bulk store has completed (writes visible).
__device__ __forceinline__ void bulk_wait_all() {
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}
// Order this thread's generic-proxy shared-memory writes before later
// async-proxy (TMA) reads of them.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------------------
// tcgen05: tensor memory, MMA, loads and stores.
// ---------------------------------------------------------------------------
template <uint32_t kCols>
__device__ __forceinline__ void tmem_alloc(uint32_t* smem_result) {
  static_assert(kCols >= 32 && (kCols & (kCols - 1)) == 0 && kCols <= 512, "TMEM columns");
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(smem_result)),
               "n"(kCols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

template <uint32_t kCols>
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "n"(kCols)
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, kind::f16 (bf16 in, fp32 acc).
__device__ __forceinline__ void umma_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                        uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem desc], kind::f16. A lives in tensor memory.
__device__ __forceinline__ void umma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                        uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// MMAs issued from a warp-uniform loop: every lane of the MMA warp computes
// the same descriptor words (so they stay in uniform registers) and
// elect.sync picks the one lane that issues. The descriptor high word
// (stride offset, version, swizzle) is loop-invariant and the low word
// (start address, leading offset) advances by immediates.
template <bool kAccumulate>
__device__ __forceinline__ void umma_ss_elect(uint32_t d_tmem, uint32_t a_lo, uint32_t b_lo,
                                              uint32_t desc_hi, uint32_t idesc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t.reg .b64 da, db;\n\t"
      "elect.sync _|p, 0xffffffff;\n\t"
      "mov.b64 da, {%1, %3};\n\t"
      "mov.b64 db, {%2, %3};\n\t"
      "@p tcgen05.mma.cta_group::1.kind::f16 [%0], da, db, %4, %5;\n\t}" ::"r"(d_tmem),
      "r"(a_lo), "r"(b_lo), "r"(desc_hi), "r"(idesc), "n"(kAccumulate ? 1 : 0)
      : "memory");
}

__device__ __forceinline__ void umma_ts_elect(uint32_t d_tmem, uint32_t a_tmem, uint32_t b_lo,
                                              uint32_t desc_hi, uint32_t idesc,
                                              uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, acc;\n\t.reg .b64 db;\n\t"
      "elect.sync _|p, 0xffffffff;\n\t"
      "mov.b64 db, {%2, %3};\n\t"
      "setp.ne.b32 acc, %5, 0;\n\t"
      "@p tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], db, %4, acc;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "r"(b_lo), "r"(desc_hi), "r"(idesc), "r"(accumulate)
      : "memory");
}

// tcgen05.commit by one elected lane of a converged warp.
__device__ __forceinline__ void umma_commit_elect(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .pred p;\n\telect.sync _|p, 0xffffffff;\n\t"
      "@p tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}" ::"r"(
          smem_u32(bar))
      : "memory");
}

// High word of a SW128 descriptor with a 1024-byte stride offset.
constexpr uint32_t kDescHiSw128 = (1024u >> 4) | (1u << 14) | (2u << 29);
// Low word: start address and leading byte offset.
__device__ __forceinline__ uint32_t desc_lo(uint32_t saddr, uint32_t lbo_bytes) {
  return ((saddr >> 4) & 0x3FFFu) | ((lbo_bytes >> 4) << 16);
}

// Arrive on `bar` once every tcgen05.mma issued so far by this thread is done.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

// 32 lanes x 32 bit, 32 consecutive columns: thread i of the warp receives
// lane (base_lane + i), columns [col, col + 32). The array is indexed with a
// compile-time offset so it stays in registers.
#define ENL_R32(a, o)                                                                        \
  "=r"(a[(o) + 0]), "=r"(a[(o) + 1]), "=r"(a[(o) + 2]), "=r"(a[(o) + 3]), "=r"(a[(o) + 4]),  \
      "=r"(a[(o) + 5]), "=r"(a[(o) + 6]), "=r"(a[(o) + 7]), "=r"(a[(o) + 8]),                \
      "=r"(a[(o) + 9]), "=r"(a[(o) + 10]), "=r"(a[(o) + 11]), "=r"(a[(o) + 12]),             \
      "=r"(a[(o) + 13]), "=r"(a[(o) + 14]), "=r"(a[(o) + 15]), "=r"(a[(o) + 16]),            \
      "=r"(a[(o) + 17]), "=r"(a[(o) + 18]), "=r"(a[(o) + 19]), "=r"(a[(o) + 20]),            \
      "=r"(a[(o) + 21]), "=r"(a[(o) + 22]), "=r"(a[(o) + 23]), "=r"(a[(o) + 24]),            \
      "=r"(a[(o) + 25]), "=r"(a[(o) + 26]), "=r"(a[(o) + 27]), "=r"(a[(o) + 28]),            \
      "=r"(a[(o) + 29]), "=r"(a[(o) + 30]), "=r"(a[(o) + 31])
#define ENL_W32(a, o)                                                                        \
  "r"(a[(o) + 0]), "r"(a[(o) + 1]), "r"(a[(o) + 2]), "r"(a[(o) + 3]), "r"(a[(o) + 4]),       \
      "r"(a[(o) + 5]), "r"(a[(o) + 6]), "r"(a[(o) + 7]), "r"(a[(o) + 8]), "r"(a[(o) + 9]),   \
      "r"(a[(o) + 10]), "r"(a[(o) + 11]), "r"(a[(o) + 12]), "r"(a[(o) + 13]),                \
      "r"(a[(o) + 14]), "r"(a[(o) + 15]), "r"(a[(o) + 16]), "r"(a[(o) + 17]),                \
      "r"(a[(o) + 18]), "r"(a[(o) + 19]), "r"(a[(o) + 20]), "r"(a[(o) + 21]),                \
      "r"(a[(o) + 22]), "r"(a[(o) + 23]), "r"(a[(o) + 24]), "r"(a[(o) + 25]),                \
      "r"(a[(o) + 26]), "r"(a[(o) + 27]), "r"(a[(o) + 28]), "r"(a[(o) + 29]),                \
      "r"(a[(o) + 30]), "r"(a[(o) + 31])

// Loads carry their own tcgen05.wait::ld inside the same asm statement: the
// compiler treats asm outputs as ready when the statement ends, so a separate
// wait could let it schedule uses of the registers before the data lands.
#define ENL_TMEM_LD32(taddr, a, o)                                                           \
  asm volatile(                                                                              \
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];\n\t"                       \
      "tcgen05.wait::ld.sync.aligned;"                                                       \
      : ENL_R32(a, o)                                                                        \
      : "r"(taddr)                                                                           \
      : "memory")

// Two 32-column loads (from two addresses) under one wait.
#define ENL_TMEM_LD32X2(ta, a, tb, b)                                                        \
  asm volatile(                                                                              \
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%64];\n\t" \
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%32, %33, %34, %35, %36, %37, %38, %39, %40, %41, %42, %43, %44, %45, %46, %47, %48, %49, %50, %51, %52, %53, %54, %55, %56, %57, %58, %59, %60, %61, %62, %63}, [%65];\n\t" \
      "tcgen05.wait::ld.sync.aligned;"                                                       \
      : ENL_R32(a, 0), ENL_R32(b, 0)                                                         \
      : "r"(ta), "r"(tb)                                                                     \
      : "memory")

// 128 consecutive columns in one instruction (a full 128-key score row).
#define ENL_TMEM_LD128(taddr, a)                                                             \
  asm volatile(                                                                              \
      "tcgen05.ld.sync.aligned.32x32b.x128.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32, %33, %34, %35, %36, %37, %38, %39, %40, %41, %42, %43, %44, %45, %46, %47, %48, %49, %50, %51, %52, %53, %54, %55, %56, %57, %58, %59, %60, %61, %62, %63, %64, %65, %66, %67, %68, %69, %70, %71, %72, %73, %74, %75, %76, %77, %78, %79, %80, %81, %82, %83, %84, %85, %86, %87, %88, %89, %90, %91, %92, %93, %94, %95, %96, %97, %98, %99, %100, %101, %102, %103, %104, %105, %106, %107, %108, %109, %110, %111, %112, %113, %114, %115, %116, %117, %118, %119, %120, %121, %122, %123, %124, %125, %126, %127}, [%128];\n\t"                     \
      "tcgen05.wait::ld.sync.aligned;"                                                       \
      : ENL_R32(a, 0), ENL_R32(a, 32), ENL_R32(a, 64), ENL_R32(a, 96)                        \
      : "r"(taddr)                                                                           \
      : "memory")

#define ENL_TMEM_ST64(taddr, a)                                                              \
  asm volatile(                                                                              \
      "tcgen05.st.sync.aligned.32x32b.x64.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32, %33, %34, %35, %36, %37, %38, %39, %40, %41, %42, %43, %44, %45, %46, %47, %48, %49, %50, %51, %52, %53, %54, %55, %56, %57, %58, %59, %60, %61, %62, %63, %64};"                              \
      ::"r"(taddr), ENL_W32(a, 0), ENL_W32(a, 32)                                           \
      : "memory")

#define ENL_TMEM_ST32(taddr, a, o)                                                           \
  asm volatile(                                                                              \
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "                                        \
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "            \
      "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};"   \
      ::"r"(taddr),                                                                          \
      ENL_W32(a, o)                                                                          \
      : "memory")

// 16 consecutive columns (load includes the wait), for low-register paths.
#define ENL_TMEM_LD16(taddr, a)                                                              \
  asm volatile(                                                                              \
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "  \
      "%11, %12, %13, %14, %15}, [%16];\n\t"                                                  \
      "tcgen05.wait::ld.sync.aligned;"                                                       \
      : "=r"(a[0]), "=r"(a[1]), "=r"(a[2]), "=r"(a[3]), "=r"(a[4]), "=r"(a[5]), "=r"(a[6]),   \
        "=r"(a[7]), "=r"(a[8]), "=r"(a[9]), "=r"(a[10]), "=r"(a[11]), "=r"(a[12]),           \
        "=r"(a[13]), "=r"(a[14]), "=r"(a[15])                                                \
      : "r"(taddr)                                                                           \
      : "memory")

#define ENL_TMEM_ST16(taddr, a)                                                              \
  asm volatile(                                                                              \
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "                                        \
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};"             \
      ::"r"(taddr), "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(a[4]), "r"(a[5]),        \
      "r"(a[6]), "r"(a[7]), "r"(a[8]), "r"(a[9]), "r"(a[10]), "r"(a[11]), "r"(a[12]),        \
      "r"(a[13]), "r"(a[14]), "r"(a[15])                                                     \
      : "memory")

// Two 16-column loads (from two addresses) under one wait.
#define ENL_TMEM_LD16X2(ta, a, tb, b)                                                        \
  asm volatile(                                                                              \
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "  \
      "%11, %12, %13, %14, %15}, [%32];\n\t"                                                  \
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%16, %17, %18, %19, %20, %21, %22, %23, %24, "  \
      "%25, %26, %27, %28, %29, %30, %31}, [%33];\n\t"                                        \
      "tcgen05.wait::ld.sync.aligned;"                                                       \
      : "=r"(a[0]), "=r"(a[1]), "=r"(a[2]), "=r"(a[3]), "=r"(a[4]), "=r"(a[5]), "=r"(a[6]),   \
        "=r"(a[7]), "=r"(a[8]), "=r"(a[9]), "=r"(a[10]), "=r"(a[11]), "=r"(a[12]),           \
        "=r"(a[13]), "=r"(a[14]), "=r"(a[15]), "=r"(b[0]), "=r"(b[1]), "=r"(b[2]),           \
        "=r"(b[3]), "=r"(b[4]), "=r"(b[5]), "=r"(b[6]), "=r"(b[7]), "=r"(b[8]), "=r"(b[9]),   \
        "=r"(b[10]), "=r"(b[11]), "=r"(b[12]), "=r"(b[13]), "=r"(b[14]), "=r"(b[15])         \
      : "r"(ta), "r"(tb)                                                                     \
      : "memory")

__device__ __forceinline__ void tmem_ld_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_st_wait() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// ---------------------------------------------------------------------------
// UMMA descriptors (tcgen05 shared-memory matrix descriptor, version 1).
//   bits  0-13 start address >> 4     bits 16-29 leading byte offset >> 4
//   bits 32-45 stride byte offset >> 4 bits 46-47 version (1 on sm_100)
//   bits 49-51 base offset (0: tiles are 1024-byte aligned)
//   bits 61-63 layout (2 = 128-byte swizzle)
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t saddr, uint32_t lbo_bytes,
                                                    uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(2) << 61;
  return d;
}

// Instruction descriptor, kind::f16 with bf16 A/B and fp32 accumulation.
//   bits 4-5 D format (1 = f32); 7-9 A format (1 = bf16); 10-12 B format;
//   bit 15 A major (0 = K); bit 16 B major (1 = MN); 17-22 N >> 3; 24-28 M >> 4.
__host__ __device__ constexpr uint32_t idesc_bf16_f32(uint32_t M, uint32_t N, bool b_mn_major) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((b_mn_major ? 1u : 0u) << 16) |
         ((N >> 3) << 17) | ((M >> 4) << 24);
}

// ---------------------------------------------------------------------------
// Small numeric helpers.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Three-input maximum (sm_100 PTX).
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// Packed fp32 pairs on the FMA pipe (sm_100 f32x2 instructions).
__device__ __forceinline__ uint64_t f2_pack(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void f2_unpack(uint64_t v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

// 2^x on the FMA/ALU pipes, for x in (-inf, 8]: round-to-nearest range
// reduction x = n + f, f in [-0.5, 0.5], via the 1.5 * 2^23 magic constant,
// then a cubic for 2^f whose coefficients minimise the relative error on that
// interval (Lawson-weighted least squares), then n is added to the exponent.
// Max relative error, fp32 rounding included: 7.64e-5 (measured over
// [-125, 8] against exact 2^x), well under the 2^-9 of the bf16 P it feeds.
// Inputs below -125 are clamped (results ~1e-38 instead of 0); only used on
// tiles with no masked scores.
__device__ __forceinline__ float exp2_poly(float x) {
  x = fmaxf(x, -125.0f);
  const float t = x + 12582912.0f;
  const float f = x - (t - 12582912.0f);
  float p = fmaf(0.05522262f, f, 0.24261537f);
  p = fmaf(p, f, 0.6932516f);
  p = fmaf(p, f, 0.9999276f);
  return __int_as_float(__float_as_int(p) + (__float_as_int(t) << 23));
}

// exp2_poly on a packed pair: the range reduction and the cubic run as f32x2
// instructions (half the issue slots of the scalar form).
__device__ __forceinline__ void exp2_poly2(float x0, float x1, float& y0, float& y1) {
  const uint64_t magic = f2_pack(12582912.0f, 12582912.0f);
  const uint64_t neg_magic = f2_pack(-12582912.0f, -12582912.0f);
  const uint64_t x = f2_pack(fmaxf(x0, -125.0f), fmaxf(x1, -125.0f));
  const uint64_t t = f2_add(x, magic);
  const uint64_t f = f2_fma(f2_add(t, neg_magic), f2_pack(-1.0f, -1.0f), x);  // x - round(x)
  uint64_t p = f2_fma(f2_pack(0.05522262f, 0.05522262f), f, f2_pack(0.24261537f, 0.24261537f));
  p = f2_fma(p, f, f2_pack(0.6932516f, 0.6932516f));
  p = f2_fma(p, f, f2_pack(0.9999276f, 0.9999276f));
  float p0, p1, t0, t1;
  f2_unpack(p, p0, p1);
  f2_unpack(t, t0, t1);
  y0 = __int_as_float(__float_as_int(p0) + (__float_as_int(t0) << 23));
  y1 = __int_as_float(__float_as_int(p1) + (__float_as_int(t1) << 23));
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

__device__ __forceinline__ float bf16lo_to_f32(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16hi_to_f32(uint32_t w) {
  return __uint_as_float(w & 0xFFFF0000u);
}

// Unsigned 32-bit division by a run-time invariant divisor d >= 1 as a
// multiply-high, an add and a shift (Granlund and Montgomery, "Division by
// invariant integers using multiplication", PLDI 1994, the N+1-bit multiplier
// form): l = ceil(log2 d), m = floor(2^32 (2^l - d) / d) + 1, and
// n / d = (mulhi(m, n) + n) >> l for every 0 <= n < 2^32 (the add is done in
// 64 bits). Elementwise kernels use it for their index decomposition, where a
// 64-bit division costs more than the element's own work.
struct DivU32 {
  uint32_t d, m, l;
  static DivU32 make(uint32_t d) {
    uint32_t l = 0;
    while (l < 32 && (1ull << l) < d) ++l;
    const uint64_t m = (((1ull << l) - d) << 32) / d + 1;
    return DivU32{d, (uint32_t)m, l};
  }
  __device__ __forceinline__ uint32_t div(uint32_t n) const {
    return (uint32_t)(((uint64_t)__umulhi(n, m) + n) >> l);
  }
};

}  // namespace enl
