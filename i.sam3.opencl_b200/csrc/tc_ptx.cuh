// SPDX-License-Identifier: Unlicense
// Blackwell (sm_100a) building blocks written as inline PTX: mbarriers with
// bounded waits, TMA tile loads, tcgen05 tensor-memory allocation, MMA,
// commit and loads, and the shared-memory / instruction descriptors of
// tcgen05.mma (PTX ISA "Matrix Descriptors" and "Instruction descriptor").
#pragma once

#include "pdl.cuh"

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace sam3 {

// Error codes a kernel writes to the device error word (first one wins).
enum : int {
    kErrNone = 0,
    kErrWaitTimeout = 1,   // an mbarrier wait exceeded its time limit
};

// Time limit of every spin-wait, in nanoseconds of %globaltimer.
constexpr uint64_t kWaitLimitNs = 4000000000ull;

__device__ __forceinline__ uint32_t smem_addr(const void *p)
{
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer()
{
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ uint32_t lane_id()
{
    uint32_t l;
    asm volatile("mov.u32 %0, %%laneid;" : "=r"(l));
    return l;
}

__device__ __forceinline__ bool elect_one()
{
    uint32_t pred = 0;
    asm volatile(
        "{\n\t.reg .pred P;\n\t"
        "elect.sync _|P, %1;\n\t"
        "selp.b32 %0, 1, 0, P;\n\t}"
        : "=r"(pred)
        : "r"(0xffffffffu));
    return pred != 0;
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count)
                 : "memory");
}

__device__ __forceinline__ void fence_mbar_init()
{
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar)
{
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes)
{
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity)
{
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred P;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 P, [%1], %2;\n\t"
        "selp.b32 %0, 1, 0, P;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}

// Waits for the phase with the given parity to complete. Bounded: after
// limit_ns (default kWaitLimitNs) it records kErrWaitTimeout in *err,
// raises the CTA's abort flag and returns false. Also returns false at
// once when another thread of the CTA has raised the abort flag, so every
// role unwinds.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, int *err,
                                          volatile int *abort_flag,
                                          uint64_t limit_ns = kWaitLimitNs)
{
    const uint32_t a = smem_addr(bar);
    if (mbar_try_wait(a, parity))
        return true;
    const uint64_t t0 = globaltimer();
    for (uint32_t it = 1;; it++) {
        if (mbar_try_wait(a, parity))
            return true;
        if ((it & 63) == 0) {
            if (*abort_flag)
                return false;
            if (globaltimer() - t0 > limit_ns) {
                atomicCAS(err, kErrNone, kErrWaitTimeout);
                *abort_flag = 1;
                return false;
            }
        }
    }
}

// ---------------------------------------------------------------- CTA pairs
// A cluster of two CTAs on the two SMs of one TPC: rank 0 issues the
// pair's tcgen05.mma (cta_group::2) over both CTAs' shared memory and
// tensor memory.
__device__ __forceinline__ uint32_t cluster_ctarank()
{
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

// The shared::cluster address of the variable at shared::cta address
// `addr` in the CTA of the cluster with rank `rank`.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank)
{
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
    return r;
}

// All threads of both CTAs: every shared-memory write before it (barrier
// initialisation included) is visible to the cluster after it.
__device__ __forceinline__ void cluster_sync_all()
{
    asm volatile("barrier.cluster.arrive.release.aligned;\n\t"
                 "barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Arrival on an mbarrier of any CTA of the cluster (shared::cluster
// address), releasing this thread's prior writes at cluster scope.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr)
{
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait_cluster(uint32_t bar, uint32_t parity)
{
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred P;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 P, [%1], %2;\n\t"
        "selp.b32 %0, 1, 0, P;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}

// mbar_wait for a barrier that CTAs of the cluster other than this one
// also signal (acquire at cluster scope); bounded in the same way.
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t *bar, uint32_t parity, int *err,
                                                  volatile int *abort_flag)
{
    const uint32_t a = smem_addr(bar);
    if (mbar_try_wait_cluster(a, parity))
        return true;
    const uint64_t t0 = globaltimer();
    for (uint32_t it = 1;; it++) {
        if (mbar_try_wait_cluster(a, parity))
            return true;
        if ((it & 63) == 0) {
            if (*abort_flag)
                return false;
            if (globaltimer() - t0 > kWaitLimitNs) {
                atomicCAS(err, kErrNone, kErrWaitTimeout);
                *abort_flag = 1;
                return false;
            }
        }
    }
}

// ---------------------------------------------------------------- TMA
__device__ __forceinline__ void tma_load_2d(void *smem_dst, const CUtensorMap *map, uint64_t *bar,
                                            int32_t x, int32_t y)
{
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_addr(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_addr(bar))
        : "memory");
}

// 3-D tile load (innermost coordinate first); coordinates outside the
// tensor read as zero.
__device__ __forceinline__ void tma_load_3d(void *smem_dst, const CUtensorMap *map, uint64_t *bar,
                                            int32_t c0, int32_t c1, int32_t c2)
{
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_addr(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(smem_addr(bar))
        : "memory");
}

// 4-D tile load (innermost coordinate first); coordinates outside the
// tensor read as zero.
__device__ __forceinline__ void tma_load_4d(void *smem_dst, const CUtensorMap *map, uint64_t *bar,
                                            int32_t c0, int32_t c1, int32_t c2, int32_t c3)
{
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(smem_addr(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3),
        "r"(smem_addr(bar))
        : "memory");
}

// 4-D tile store (elements outside the tensor are not written).
__device__ __forceinline__ void tma_store_4d(const CUtensorMap *map, const void *smem_src,
                                             int32_t c0, int32_t c1, int32_t c2, int32_t c3)
{
    asm volatile(
        "cp.async.bulk.tensor.4d.global.shared::cta.bulk_group [%0, {%1, %2, %3, %4}], [%5];" ::"l"(
            reinterpret_cast<uint64_t>(map)),
        "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_addr(smem_src))
        : "memory");
}

// Tile store shared -> global through a tensor map (out-of-range rows and
// columns of the box are not written), tracked by the bulk-group mechanism.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap *map, const void *smem_src,
                                             int32_t x, int32_t y)
{
    asm volatile(
        "cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
            reinterpret_cast<uint64_t>(map)),
        "r"(x), "r"(y), "r"(smem_addr(smem_src))
        : "memory");
}

// 2-D tile load by either CTA of a pair, completing on the mbarrier at
// shared::cluster address `bar` (rank 0's, which counts both CTAs' bytes).
__device__ __forceinline__ void tma_load_2d_pair(void *smem_dst, const CUtensorMap *map,
                                                 uint32_t bar, int32_t x, int32_t y)
{
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_addr(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
        : "memory");
}

// Tile reduce-add shared -> global through a tensor map: every element of
// the box is added (fp32, one rounding) to the global element in L2;
// out-of-range rows and columns are skipped. Tracked like tma_store_2d.
__device__ __forceinline__ void tma_reduce_add_2d(const CUtensorMap *map, const void *smem_src,
                                                  int32_t x, int32_t y)
{
    asm volatile(
        "cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.bulk_group [%0, {%1, %2}], [%3];" ::
            "l"(reinterpret_cast<uint64_t>(map)),
        "r"(x), "r"(y), "r"(smem_addr(smem_src))
        : "memory");
}

// 4-D tile load by either CTA of a pair (see tma_load_2d_pair).
__device__ __forceinline__ void tma_load_4d_pair(void *smem_dst, const CUtensorMap *map,
                                                 uint32_t bar, int32_t c0, int32_t c1, int32_t c2,
                                                 int32_t c3)
{
    asm volatile(
        "cp.async.bulk.tensor.4d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(smem_addr(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(bar)
        : "memory");
}

__device__ __forceinline__ void bulk_commit()
{
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

// Wait until at most N committed bulk groups of this thread still read
// shared memory (their source may then be overwritten).
template <int N>
__device__ __forceinline__ void bulk_wait_read()
{
    asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

// Wait until all committed bulk groups of this thread have completed.
__device__ __forceinline__ void bulk_wait_all()
{
    asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

__device__ __forceinline__ void prefetch_tmap(const CUtensorMap *map)
{
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// Orders this thread's generic-proxy shared-memory writes before later
// async-proxy reads (tcgen05.mma operands, TMA stores).
__device__ __forceinline__ void fence_proxy_async_smem()
{
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------- tcgen05
__device__ __forceinline__ void tmem_alloc(uint32_t *dst_smem, uint32_t ncols)
{
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_addr(dst_smem)),
                 "r"(ncols)
                 : "memory");
}

__device__ __forceinline__ void tmem_relinquish()
{
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols)
{
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
}

// Pair forms, issued by the same warp in both CTAs: the allocation is
// made at the same address in both CTAs' tensor memory.
__device__ __forceinline__ void tmem_alloc_pair(uint32_t *dst_smem, uint32_t ncols)
{
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_addr(dst_smem)),
                 "r"(ncols)
                 : "memory");
}

__device__ __forceinline__ void tmem_relinquish_pair()
{
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols)
{
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before()
{
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after()
{
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T-or-not, per the instruction descriptor.
__device__ __forceinline__ void tc_mma(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                       uint32_t idesc, uint32_t accumulate)
{
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// D (+)= A * B with A read from tensor memory (M rows in TMEM lanes, each
// 32-bit column holding two consecutive K elements, K = 16 per instruction
// in 8 columns from a_tmem) and B from a shared-memory descriptor.
__device__ __forceinline__ void tc_mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc,
                                          uint32_t idesc, uint32_t accumulate)
{
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Pair MMA (issued by rank 0 only): D rows 0..M/2-1 in rank 0's tensor
// memory, M/2..M-1 in rank 1's; A rows split the same way between the two
// CTAs' shared memory, B rows (the N dimension) half in each; the
// descriptors name the same shared-memory offsets in both CTAs.
__device__ __forceinline__ void tc_mma_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                            uint32_t idesc, uint32_t accumulate)
{
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// One arrival on the mbarrier at the same shared-memory offset in each CTA
// of `cta_mask` once the pair MMAs issued so far by this thread complete.
__device__ __forceinline__ void tc_commit_pair(uint64_t *bar, uint16_t cta_mask)
{
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64"
        " [%0], %1;" ::"r"(smem_addr(bar)),
        "h"(cta_mask)
        : "memory");
}

// The mbarrier receives one arrival when all tcgen05 operations issued so
// far by this thread have completed.
__device__ __forceinline__ void tc_commit(uint64_t *bar)
{
    asm volatile(
        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
            smem_addr(bar))
        : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns: thread t of the warp receives
// lane (base lane + t), columns col .. col + 31.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32])
{
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
          "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
          "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
          "=r"(r[31])
        : "r"(taddr));
}

// 32 lanes x 16 consecutive 32-bit columns.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16])
{
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
          "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}

__device__ __forceinline__ void tmem_wait_ld()
{
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// 32 lanes x 32 consecutive 32-bit columns from registers into TMEM (the
// inverse of tmem_ld32).
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32])
{
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

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16])
{
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
        "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
        "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
        "r"(r[15])
        : "memory");
}

__device__ __forceinline__ void tmem_wait_st()
{
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// Shared-memory matrix descriptor for a 128-byte-swizzled operand tile
// whose rows are 128 bytes (64 bf16): start address, leading byte offset,
// stride byte offset (between 8-row groups), version 1, SWIZZLE_128B.
// K-major tiles: SBO = 1024 (8 rows x 128 B), LBO unused (16 B).
// MN-major tiles (K rows of 64 N-values): SBO = 1024 between 8-row groups
// along K, LBO = byte distance between 64-wide N groups.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr, uint32_t lbo_bytes,
                                               uint32_t sbo_bytes)
{
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFF);
    d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFF) << 16;
    d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFF) << 32;
    d |= (uint64_t)1 << 46;  // descriptor version (Blackwell)
    d |= (uint64_t)2 << 61;  // SWIZZLE_128B
    return d;
}

// Instruction descriptor of tcgen05.mma kind::f16: bf16 A and B, fp32 D,
// M x N tile, A/B K-major (0) or MN-major (1).
__host__ __device__ constexpr uint32_t idesc_bf16_f32(int M, int N, int a_mn_major,
                                                      int b_mn_major)
{
    return (1u << 4)                          // D format: F32
           | (1u << 7)                        // A format: BF16
           | (1u << 10)                       // B format: BF16
           | ((uint32_t)a_mn_major << 15)     // A major
           | ((uint32_t)b_mn_major << 16)     // B major
           | ((uint32_t)(N >> 3) << 17)       // N / 8
           | ((uint32_t)(M >> 4) << 24);      // M / 16
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi)
{
    uint32_t r;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
}

__device__ __forceinline__ float rcp_approx(float x)
{
    float y;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}


__device__ __forceinline__ float ex2_approx(float x)
{
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// ---------------------------------------------------------------- packed fp32
// Pairs of fp32 in one 64-bit register for the sm_100 .f32x2 arithmetic
// (one instruction for two lanes of add / mul / fma).
__device__ __forceinline__ uint64_t f2_make(float lo, float hi)
{
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}

__device__ __forceinline__ void f2_split(uint64_t v, float &lo, float &hi)
{
    asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}

__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c)
{
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}

__device__ __forceinline__ uint64_t add2(uint64_t a, uint64_t b)
{
    uint64_t d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}

__device__ __forceinline__ uint64_t mul2(uint64_t a, uint64_t b)
{
    uint64_t d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}

__device__ __forceinline__ float max3f(float a, float b, float c)
{
    float d;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}

// 2^x for two values x <= 0 on the FMA pipe, leaving the MUFU unit to the
// other exponentials of the softmax. Method: Cody-Waite style range
// reduction x = n + f with n = round(x) (add and subtract 1.5 * 2^23, exact
// for |x| < 2^22) and f in [-0.5, 0.5]; 2^f from a degree-3 polynomial whose
// coefficients minimise the maximum relative error on [-0.5, 0.5] (fitted
// for this kernel by linear programming: 7.5e-5 max relative error in fp32
// Horner form); 2^n applied by adding n to the exponent field. x is clamped
// to -125 so the result stays a normal number (2^-125 ~ 2.4e-38, i.e. 0 for
// a softmax weight). Accuracy is far below the bf16 rounding of P (2^-9).
__device__ __forceinline__ void exp2_poly2(float x0, float x1, float &y0, float &y1)
{
    const float kMagic = 12582912.0f;  // 1.5 * 2^23
    const uint64_t x = f2_make(fmaxf(x0, -125.0f), fmaxf(x1, -125.0f));
    const uint64_t j = add2(x, f2_make(kMagic, kMagic));
    const uint64_t n = add2(j, f2_make(-kMagic, -kMagic));
    const uint64_t f = fma2(n, f2_make(-1.0f, -1.0f), x);
    uint64_t p = fma2(f2_make(0.05517221987247467f, 0.05517221987247467f), f,
                      f2_make(0.24261115491390228f, 0.24261115491390228f));
    p = fma2(p, f, f2_make(0.6932608485221863f, 0.6932608485221863f));
    p = fma2(p, f, f2_make(0.9999280571937561f, 0.9999280571937561f));
    float p0, p1, j0, j1;
    f2_split(p, p0, p1);
    f2_split(j, j0, j1);
    // bits(j) = bits(1.5 * 2^23) + n; shifted left by 23 the constant part
    // leaves 32 bits and n lands in the exponent field.
    y0 = __uint_as_float(__float_as_uint(j0) * 8388608u + __float_as_uint(p0));
    y1 = __uint_as_float(__float_as_uint(j1) * 8388608u + __float_as_uint(p1));
}

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c,
                                             uint32_t d)
{
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c),
                 "r"(d)
                 : "memory");
}

}  // namespace sam3
