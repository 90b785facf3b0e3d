// PTX wrappers shared by the sm_100a tensor-core kernels (GEMM, attention):
// mbarriers with bounded waits, 2-D TMA loads, tcgen05 MMA / commit / TMEM
// loads and stores, and the shared-memory matrix descriptors for tiles that
// TMA writes with the 128-byte swizzle.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cudaTypedefs.h>
#include <stdint.h>

#include "common.cuh"

namespace fcu {
namespace tc {

constexpr long long kWaitCycles = 4000000000ll;  // ~2 s at 2 GHz

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
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

// Bounded wait: false if the phase did not complete within kWaitCycles or
// another role of this CTA has already aborted.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, volatile int *abort_flag) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort_flag) return false;
    if (clock64() - t0 > kWaitCycles) return false;
  }
}

// mbar_wait by all 32 lanes of a warp with one warp-uniform result, so a warp
// that goes on to warp-collective tcgen05.ld / tcgen05.st never diverges
// (those .sync.aligned instructions need every lane).
__device__ __forceinline__ bool warp_wait(uint64_t *bar, uint32_t parity, volatile int *abort_flag) {
  const bool ok = mbar_wait(bar, parity, abort_flag);
  return __all_sync(0xffffffffu, ok);
}

// Bounded wait that ignores the abort flag: for draining copies and MMAs this
// CTA issued before it exits (they always complete; the bound is a backstop).
__device__ __forceinline__ bool mbar_wait_drain(uint64_t *bar, uint32_t parity) {
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity))
    if (clock64() - t0 > kWaitCycles) return false;
  return true;
}

__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int c0, int c1,
                                            uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
      "l"((uint64_t)map), "r"(c0), "r"(c1), "r"(smem_u32(bar))
      : "memory");
}

// Untiled bulk copy of `bytes` contiguous bytes global -> shared memory,
// completing on an mbarrier.  Both addresses 16-byte aligned, bytes a
// multiple of 16.
__device__ __forceinline__ void bulk_load_1d(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"((uint64_t)src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// 2-D TMA store / reduce-add of a shared-memory box to global memory, as a
// bulk async-group (commit with bulk_commit, reuse the source after
// bulk_wait_read).  The start coordinates must not be negative.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap *map, const void *src, int c0, int c1) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
                   (uint64_t)map),
               "r"(c0), "r"(c1), "r"(smem_u32(src))
               : "memory");
}

__device__ __forceinline__ void tma_reduce_add_2d(const CUtensorMap *map, const void *src, int c0, int c1) {
  asm volatile(
      "cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
          (uint64_t)map),
      "r"(c0), "r"(c1), "r"(smem_u32(src))
      : "memory");
}

__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }

// Waits until at most N committed bulk groups still read their shared-memory source.
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

// Waits until every committed bulk group has completed.
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Generic-proxy shared-memory writes (st.shared) made visible to the async
// proxy (tcgen05.mma operand reads, TMA).
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void umma_bf16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                          uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

// The same with A read from TMEM (M rows on lanes, K packed two bf16 per
// 32-bit column, lower k in the low half): a_tmem is the column of k = 0.
__device__ __forceinline__ void umma_bf16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc,
                                             uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

// The same three, executed by every lane of a converged warp with warp-uniform
// operands: elect.sync picks one lane (the lowest, so MMAs and their commit
// come from the same thread) to issue.  Keeping the whole warp on the issue
// path lets the operands stay in uniform registers; a single-lane branch
// pays a per-instruction conversion that makes small (N = 64) MMAs
// issue-bound.
__device__ __forceinline__ void umma_bf16_w(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                            uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred e, p;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

__device__ __forceinline__ void umma_bf16_ts_w(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc,
                                               uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred e, p;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

__device__ __forceinline__ void umma_commit_w(uint64_t *bar) {
  asm volatile(
      "{\n\t.reg .pred e;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}\n" ::"r"(
          smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t *bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

// ---- CTA pairs (cluster of 2, tcgen05 .cta_group::2).  Every tcgen05
// instruction of a pair kernel uses .cta_group::2: the even CTA of the
// cluster issues the MMAs, which read A rows 0..127 and B rows 0..N/2-1 from
// its own shared memory and the rest from its peer's at the same offsets, and
// write each CTA's 128 accumulator rows into that CTA's TMEM.
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// Every thread of every CTA of the cluster (converged warps).
__device__ __forceinline__ void cluster_sync() {
  __syncwarp();
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// The shared::cluster address of `addr` (a shared::cta address) in CTA `rank`.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}

__device__ __forceinline__ void mbar_arrive_remote(uint32_t cl_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cl_addr) : "memory");
}

// try_wait with cluster-scope acquire: for a barrier that threads of the
// peer CTA arrive on.
__device__ __forceinline__ bool mbar_try_wait_cl(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ bool warp_wait_cl(uint64_t *bar, uint32_t parity, volatile int *abort_flag) {
  bool ok = true;
  if (!mbar_try_wait_cl(bar, parity)) {
    const long long t0 = clock64();
    while (true) {
      if (mbar_try_wait_cl(bar, parity)) break;
      if (*abort_flag || clock64() - t0 > kWaitCycles) {
        ok = false;
        break;
      }
    }
  }
  return __all_sync(0xffffffffu, ok);
}

// 2-D TMA load into this CTA's shared memory that completes on an mbarrier
// of either CTA of the pair (bar_cl: a shared::cluster address).  Each CTA
// loads only its own half of the operands, into its own shared memory.
__device__ __forceinline__ void tma_load_2d_pair(void *dst, const CUtensorMap *map, int c0, int c1,
                                                 uint32_t bar_cl) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
      "l"((uint64_t)map), "r"(c0), "r"(c1), "r"(bar_cl)
      : "memory");
}

__device__ __forceinline__ void umma2_bf16_w(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                             uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred e, p;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "@e tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

// Arrives on the mbarrier at shared::cluster address bar_cl (this CTA's or
// the peer's) once every pair MMA this thread issued has completed.
__device__ __forceinline__ void umma2_commit_w(uint32_t bar_cl) {
  asm volatile(
      "{\n\t.reg .pred e;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "@e tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}\n" ::"r"(bar_cl)
      : "memory");
}

// Pair allocation: one warp of each CTA of the pair executes it.
__device__ __forceinline__ void tmem_alloc2(uint32_t *slot, uint32_t cols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)),
               "r"(cols));
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
}

__device__ __forceinline__ void tmem_dealloc2(uint32_t base, uint32_t cols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(base), "r"(cols));
}

__device__ __forceinline__ void tmem_alloc(uint32_t *slot, uint32_t cols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(slot)),
               "r"(cols));
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t base, uint32_t cols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(base), "r"(cols));
}

// 32 consecutive fp32 columns of this thread's TMEM lane (32x32b shape: warp
// q of a warpgroup reads lanes 32q..32q+31).  The _nw form issues the load
// only; tmem_wait_ld() completes every load issued before it.
__device__ __forceinline__ void tmem_ld32_nw(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32"
      " {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15,"
      " %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31},"
      " [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// tcgen05.wait::ld that also names the registers of the loads it completes
// ("+r"), so the compiler keeps every use of them after the wait.
__device__ __forceinline__ void tmem_wait_ld_r(uint32_t (&r)[32]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]),
                 "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]),
                 "+r"(r[14]), "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]),
                 "+r"(r[20]), "+r"(r[21]), "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]),
                 "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]), "+r"(r[30]), "+r"(r[31])
               :
               : "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  tmem_ld32_nw(taddr, r);
  tmem_wait_ld();
}

// 64 consecutive fp32 columns of this thread's TMEM lane, waited for.
__device__ __forceinline__ void tmem_ld64(uint32_t taddr, float *f) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x64.b32"
      " {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15,"
      " %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31,"
      " %32, %33, %34, %35, %36, %37, %38, %39, %40, %41, %42, %43, %44, %45, %46, %47,"
      " %48, %49, %50, %51, %52, %53, %54, %55, %56, %57, %58, %59, %60, %61, %62, %63},"
      " [%64];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=f"(f[0]), "=f"(f[1]), "=f"(f[2]), "=f"(f[3]), "=f"(f[4]), "=f"(f[5]), "=f"(f[6]),
        "=f"(f[7]), "=f"(f[8]), "=f"(f[9]), "=f"(f[10]), "=f"(f[11]), "=f"(f[12]), "=f"(f[13]),
        "=f"(f[14]), "=f"(f[15]), "=f"(f[16]), "=f"(f[17]), "=f"(f[18]), "=f"(f[19]),
        "=f"(f[20]), "=f"(f[21]), "=f"(f[22]), "=f"(f[23]), "=f"(f[24]), "=f"(f[25]),
        "=f"(f[26]), "=f"(f[27]), "=f"(f[28]), "=f"(f[29]), "=f"(f[30]), "=f"(f[31]),
        "=f"(f[32]), "=f"(f[33]), "=f"(f[34]), "=f"(f[35]), "=f"(f[36]), "=f"(f[37]),
        "=f"(f[38]), "=f"(f[39]), "=f"(f[40]), "=f"(f[41]), "=f"(f[42]), "=f"(f[43]),
        "=f"(f[44]), "=f"(f[45]), "=f"(f[46]), "=f"(f[47]), "=f"(f[48]), "=f"(f[49]),
        "=f"(f[50]), "=f"(f[51]), "=f"(f[52]), "=f"(f[53]), "=f"(f[54]), "=f"(f[55]),
        "=f"(f[56]), "=f"(f[57]), "=f"(f[58]), "=f"(f[59]), "=f"(f[60]), "=f"(f[61]),
        "=f"(f[62]), "=f"(f[63])
      : "r"(taddr)
      : "memory");
}

// 128 consecutive fp32 columns of this thread's TMEM lane, waited for.
__device__ __forceinline__ void tmem_ld128(uint32_t taddr, float *f) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x128.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32, %33, %34, %35, %36, %37, %38, %39, %40, %41, %42, %43, %44, %45, %46, %47, %48, %49, %50, %51, %52, %53, %54, %55, %56, %57, %58, %59, %60, %61, %62, %63, %64, %65, %66, %67, %68, %69, %70, %71, %72, %73, %74, %75, %76, %77, %78, %79, %80, %81, %82, %83, %84, %85, %86, %87, %88, %89, %90, %91, %92, %93, %94, %95, %96, %97, %98, %99, %100, %101, %102, %103, %104, %105, %106, %107, %108, %109, %110, %111, %112, %113, %114, %115, %116, %117, %118, %119, %120, %121, %122, %123, %124, %125, %126, %127}, [%128];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=f"(f[0]), "=f"(f[1]), "=f"(f[2]), "=f"(f[3]), "=f"(f[4]), "=f"(f[5]), "=f"(f[6]), "=f"(f[7]), "=f"(f[8]), "=f"(f[9]), "=f"(f[10]), "=f"(f[11]), "=f"(f[12]), "=f"(f[13]), "=f"(f[14]), "=f"(f[15]), "=f"(f[16]), "=f"(f[17]), "=f"(f[18]), "=f"(f[19]), "=f"(f[20]), "=f"(f[21]), "=f"(f[22]), "=f"(f[23]), "=f"(f[24]), "=f"(f[25]), "=f"(f[26]), "=f"(f[27]), "=f"(f[28]), "=f"(f[29]), "=f"(f[30]), "=f"(f[31]), "=f"(f[32]), "=f"(f[33]), "=f"(f[34]), "=f"(f[35]), "=f"(f[36]), "=f"(f[37]), "=f"(f[38]), "=f"(f[39]), "=f"(f[40]), "=f"(f[41]), "=f"(f[42]), "=f"(f[43]), "=f"(f[44]), "=f"(f[45]), "=f"(f[46]), "=f"(f[47]), "=f"(f[48]), "=f"(f[49]), "=f"(f[50]), "=f"(f[51]), "=f"(f[52]), "=f"(f[53]), "=f"(f[54]), "=f"(f[55]), "=f"(f[56]), "=f"(f[57]), "=f"(f[58]), "=f"(f[59]), "=f"(f[60]), "=f"(f[61]), "=f"(f[62]), "=f"(f[63]), "=f"(f[64]), "=f"(f[65]), "=f"(f[66]), "=f"(f[67]), "=f"(f[68]), "=f"(f[69]), "=f"(f[70]), "=f"(f[71]), "=f"(f[72]), "=f"(f[73]), "=f"(f[74]), "=f"(f[75]), "=f"(f[76]), "=f"(f[77]), "=f"(f[78]), "=f"(f[79]), "=f"(f[80]), "=f"(f[81]), "=f"(f[82]), "=f"(f[83]), "=f"(f[84]), "=f"(f[85]), "=f"(f[86]), "=f"(f[87]), "=f"(f[88]), "=f"(f[89]), "=f"(f[90]), "=f"(f[91]), "=f"(f[92]), "=f"(f[93]), "=f"(f[94]), "=f"(f[95]), "=f"(f[96]), "=f"(f[97]), "=f"(f[98]), "=f"(f[99]), "=f"(f[100]), "=f"(f[101]), "=f"(f[102]), "=f"(f[103]), "=f"(f[104]), "=f"(f[105]), "=f"(f[106]), "=f"(f[107]), "=f"(f[108]), "=f"(f[109]), "=f"(f[110]), "=f"(f[111]), "=f"(f[112]), "=f"(f[113]), "=f"(f[114]), "=f"(f[115]), "=f"(f[116]), "=f"(f[117]), "=f"(f[118]), "=f"(f[119]), "=f"(f[120]), "=f"(f[121]), "=f"(f[122]), "=f"(f[123]), "=f"(f[124]), "=f"(f[125]), "=f"(f[126]), "=f"(f[127])
      : "r"(taddr)
      : "memory");
}

// Two 64-column TMEM loads (this thread's lane) completed by one wait.
__device__ __forceinline__ void tmem_ld64x2(uint32_t ta, uint32_t tb, float *a, float *b) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x64.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32, %33, %34, %35, %36, %37, %38, %39, %40, %41, %42, %43, %44, %45, %46, %47, %48, %49, %50, %51, %52, %53, %54, %55, %56, %57, %58, %59, %60, %61, %62, %63}, [%128];\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x64.b32 {%64, %65, %66, %67, %68, %69, %70, %71, %72, %73, %74, %75, %76, %77, %78, %79, %80, %81, %82, %83, %84, %85, %86, %87, %88, %89, %90, %91, %92, %93, %94, %95, %96, %97, %98, %99, %100, %101, %102, %103, %104, %105, %106, %107, %108, %109, %110, %111, %112, %113, %114, %115, %116, %117, %118, %119, %120, %121, %122, %123, %124, %125, %126, %127}, [%129];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=f"(a[0]), "=f"(a[1]), "=f"(a[2]), "=f"(a[3]), "=f"(a[4]), "=f"(a[5]), "=f"(a[6]), "=f"(a[7]), "=f"(a[8]), "=f"(a[9]), "=f"(a[10]), "=f"(a[11]), "=f"(a[12]), "=f"(a[13]), "=f"(a[14]), "=f"(a[15]), "=f"(a[16]), "=f"(a[17]), "=f"(a[18]), "=f"(a[19]), "=f"(a[20]), "=f"(a[21]), "=f"(a[22]), "=f"(a[23]), "=f"(a[24]), "=f"(a[25]), "=f"(a[26]), "=f"(a[27]), "=f"(a[28]), "=f"(a[29]), "=f"(a[30]), "=f"(a[31]), "=f"(a[32]), "=f"(a[33]), "=f"(a[34]), "=f"(a[35]), "=f"(a[36]), "=f"(a[37]), "=f"(a[38]), "=f"(a[39]), "=f"(a[40]), "=f"(a[41]), "=f"(a[42]), "=f"(a[43]), "=f"(a[44]), "=f"(a[45]), "=f"(a[46]), "=f"(a[47]), "=f"(a[48]), "=f"(a[49]), "=f"(a[50]), "=f"(a[51]), "=f"(a[52]), "=f"(a[53]), "=f"(a[54]), "=f"(a[55]), "=f"(a[56]), "=f"(a[57]), "=f"(a[58]), "=f"(a[59]), "=f"(a[60]), "=f"(a[61]), "=f"(a[62]), "=f"(a[63]), "=f"(b[0]), "=f"(b[1]), "=f"(b[2]), "=f"(b[3]), "=f"(b[4]), "=f"(b[5]), "=f"(b[6]), "=f"(b[7]), "=f"(b[8]), "=f"(b[9]), "=f"(b[10]), "=f"(b[11]), "=f"(b[12]), "=f"(b[13]), "=f"(b[14]), "=f"(b[15]), "=f"(b[16]), "=f"(b[17]), "=f"(b[18]), "=f"(b[19]), "=f"(b[20]), "=f"(b[21]), "=f"(b[22]), "=f"(b[23]), "=f"(b[24]), "=f"(b[25]), "=f"(b[26]), "=f"(b[27]), "=f"(b[28]), "=f"(b[29]), "=f"(b[30]), "=f"(b[31]), "=f"(b[32]), "=f"(b[33]), "=f"(b[34]), "=f"(b[35]), "=f"(b[36]), "=f"(b[37]), "=f"(b[38]), "=f"(b[39]), "=f"(b[40]), "=f"(b[41]), "=f"(b[42]), "=f"(b[43]), "=f"(b[44]), "=f"(b[45]), "=f"(b[46]), "=f"(b[47]), "=f"(b[48]), "=f"(b[49]), "=f"(b[50]), "=f"(b[51]), "=f"(b[52]), "=f"(b[53]), "=f"(b[54]), "=f"(b[55]), "=f"(b[56]), "=f"(b[57]), "=f"(b[58]), "=f"(b[59]), "=f"(b[60]), "=f"(b[61]), "=f"(b[62]), "=f"(b[63])
      : "r"(ta), "r"(tb)
      : "memory");
}

// 2^x on the MUFU unit; subnormal results flush to zero.
__device__ __forceinline__ float ex2_ftz(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Packed fp32 pairs (sm_100 f32x2 arithmetic, round-to-nearest, no flush):
// the same results as two scalar fmaf / + / * in half the instructions.
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\tmov.b64 rc, {%6, %7};\n\t"
      "fma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return d;
}
__device__ __forceinline__ float2 add2(float2 a, float2 b) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "add.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}
__device__ __forceinline__ float2 mul2(float2 a, float2 b) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "mul.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}

// 2^x for a pair on the FMA pipe instead of the MUFU unit (the softmax loops
// are bound by MUFU throughput, 16 ex2 per clock per SM, so a share of their
// exponentials is computed here).  Cody-Waite range reduction x = j + f with
// j = rint(x) (adding 1.5 * 2^23 rounds to an integer in the low mantissa
// bits) and |f| <= 1/2, then a degree-3 polynomial for 2^f whose coefficients
// were fitted for minimal maximum relative error on [-1/2, 1/2] (7.5e-5, far
// below the bf16 rounding of P), and j added to the exponent field.  x is
// clamped below at -126, so scores that should vanish give 2^-126 rather than
// 0; inputs are at most a few units above 0 here.
__device__ __forceinline__ float2 exp2_poly2(float2 x) {
  constexpr float kRound = 12582912.f;         // 1.5 * 2^23
  x.x = fmaxf(x.x, -126.f);
  x.y = fmaxf(x.y, -126.f);
  const float2 t = add2(x, make_float2(kRound, kRound));
  const float2 j = add2(t, make_float2(-kRound, -kRound));
  const float2 f = fma2(j, make_float2(-1.f, -1.f), x);
  float2 q = fma2(f, make_float2(0.05517232418060303f, 0.05517232418060303f),
                  make_float2(0.24261125922203064f, 0.24261125922203064f));
  q = fma2(q, f, make_float2(0.6932607293128967f, 0.6932607293128967f));
  q = fma2(q, f, make_float2(0.9999279975891113f, 0.9999279975891113f));
  // t's bits are 0x4B400000 + j; shifted left by 23 only j << 23 remains
  return make_float2(__int_as_float(__float_as_int(q.x) + (__float_as_int(t.x) << 23)),
                     __int_as_float(__float_as_int(q.y) + (__float_as_int(t.y) << 23)));
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t *r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0],"
      " {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16,"
      " %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(
          taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),
      "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),
      "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// Shared-memory matrix descriptor (sm_100 "version 1" format), 128B swizzle:
// bits 0-13 start>>4, 16-29 LBO>>4, 32-45 SBO>>4, 46-47 version=1,
// 61-63 layout (2 = SWIZZLE_128B).
__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)((lbo >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFF) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

// Descriptor of the k-th 16-deep slice of a staged operand tile whose K depth
// is `kdepth` elements.
//   K-major : rows of 64 elements (128 B), 8-row swizzle atoms 1024 B apart;
//             the slice starts k*32 B into each row (k < 4: one 64-deep block).
//   MN-major: boxes of 64 (MN) x kdepth (K) elements, one 128-B row per k,
//             box j at j*kdepth*128 B (LBO), 8-row K groups 1024 B apart
//             (SBO); the slice starts 16 rows = 2048 B further.
__device__ __forceinline__ uint64_t operand_desc(uint32_t tile, int k, int mn_major, int kdepth) {
  if (!mn_major) return smem_desc(tile + (uint32_t)k * 32u, 16u, 1024u);
  return smem_desc(tile + (uint32_t)k * 2048u, (uint32_t)kdepth * 128u, 1024u);
}

// Descriptor arithmetic without rebuilding: the start-address field counts
// 16-byte units in the low bits, so a k-slice or a later tile of the same
// layout is the base descriptor plus a constant.
constexpr uint64_t kDescKStep = 32 >> 4;       // K-major: next 16-deep slice
constexpr uint64_t kDescMNStep = 2048 >> 4;    // MN-major: next 16-deep slice
__device__ __forceinline__ uint64_t desc_k(uint32_t tile) { return smem_desc(tile, 16u, 1024u); }
__device__ __forceinline__ uint64_t desc_mn(uint32_t tile, int kdepth) {
  return smem_desc(tile, (uint32_t)kdepth * 128u, 1024u);
}

// Instruction descriptor, kind::f16: D f32 (bits 4-5 = 1), A/B bf16 (bits
// 7-9 / 10-12 = 1), majors (bits 15/16), N>>3 (bits 17-22), M>>4 (bits 24-28).
__device__ __forceinline__ uint32_t instr_desc_bf16(int a_mn, int b_mn, int m, int n) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)a_mn << 15) | ((uint32_t)b_mn << 16) |
         ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

__device__ __forceinline__ uint32_t pack2_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t *>(&v);
}

// Byte offset of the 16-byte chunk `c` (elements 8c..8c+7) of row `r` in a
// K-major tile of 64-element rows written with the 128-byte swizzle (the
// layout TMA produces and operand_desc describes).  The tile base must be
// 1024-byte aligned.
__device__ __forceinline__ uint32_t sw128_offset(int r, int c) {
  return (uint32_t)((r >> 3) * 1024 + (r & 7) * 128 + ((c ^ (r & 7)) << 4));
}

}  // namespace tc

// Host side (defined in gemm_tc.cu): the driver's tensor-map encoder and a
// 2-D bf16 map over a row-major [rows, cols] matrix with row stride
// `row_stride` elements, a {box_cols, box_rows} box and 128-byte swizzle.
int tc_get_encode();
// Device word the tensor-core kernels set when a bounded wait runs out
// (read and reported by fcu_check_device_error).
int tc_error_word(fcu_ctx *ctx, int **err);
int tc_make_map(CUtensorMap *map, const void *base, uint64_t rows, uint64_t cols,
                uint64_t row_stride, uint32_t box_cols, uint32_t box_rows);
// The same for fp32 (box_cols * 4 == 128).
int tc_make_map_f32(CUtensorMap *map, const void *base, uint64_t rows, uint64_t cols,
                    uint64_t row_stride, uint32_t box_cols, uint32_t box_rows);

}  // namespace fcu
