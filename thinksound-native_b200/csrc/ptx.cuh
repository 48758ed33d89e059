// ptx.cuh — sm_100a building blocks: mbarriers, TMA tensor loads, tcgen05 (UMMA + TMEM).
//
// Every wait on an mbarrier is bounded: after TSN_WAIT_NS of wall time (globaltimer) it records
// an error code in a device-global word, raises the CTA's abort flag and returns false, so a
// broken pipeline ends the kernel with a status the host reads instead of hanging the GPU.
// No TMA load here uses .multicast::cluster.
#pragma once
#include <cstdint>
#include <cuda.h>

namespace tsn {

#ifndef TSN_WAIT_NS
#define TSN_WAIT_NS 2000000000ull   // 2 s: every legitimate wait in these kernels is microseconds
#endif

// error codes written to the device error word
enum : int { DEV_OK = 0, DEV_TIMEOUT_FULL = 1, DEV_TIMEOUT_EMPTY = 2, DEV_TIMEOUT_TMEM = 3, DEV_BAD_ARGS = 4 };

__device__ __forceinline__ uint32_t smem_u32(const void * p) {
    return (uint32_t) __cvta_generic_to_shared(p);
}

__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t * bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t * bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t * bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Bounded wait. abort_flag is a CTA-shared word: once any role gives up, the others stop too.
__device__ __forceinline__ bool mbar_wait(uint64_t * bar, uint32_t parity, volatile int * abort_flag,
                                          int * err, int code) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_ns();
    for (uint32_t i = 1;; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 255u) == 0) {
            if (*abort_flag) return false;
            if (global_ns() - t0 > TSN_WAIT_NS) {
                *abort_flag = 1;
                if (err) atomicCAS(err, 0, code);
                return false;
            }
        }
    }
}

// ---------------------------------------------------------------- TMA (no multicast)
__device__ __forceinline__ void tma_prefetch(const CUtensorMap * m) {
    asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t) m) : "memory");
}
__device__ __forceinline__ void tma_load_2d(void * dst, const CUtensorMap * m, uint64_t * bar, int c0, int c1) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];"
        ::"r"(smem_u32(dst)), "l"((uint64_t) m), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
        : "memory");
}
__device__ __forceinline__ void tma_load_3d(void * dst, const CUtensorMap * m, uint64_t * bar, int c0, int c1, int c2) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];"
        ::"r"(smem_u32(dst)), "l"((uint64_t) m), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
        : "memory");
}

// TMA tensor store of a shared-memory box into a 4-D view, as one bulk async-group of this thread.
// The box must have been written and made visible to the async proxy (fence_proxy_async_smem)
// first; bulk_wait_read0() returns once every committed store has finished reading shared memory
// (the writes reach global memory by the grid's completion).
__device__ __forceinline__ void tma_store_4d(const CUtensorMap * m, const void * src, int c0, int c1, int c2, int c3) {
    asm volatile("cp.async.bulk.tensor.4d.global.shared::cta.bulk_group [%0, {%2, %3, %4, %5}], [%1];"
                 ::"l"((uint64_t) m), "r"(smem_u32(src)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
                 : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read0() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }

// Untiled bulk copy global -> this CTA's shared memory (16-byte aligned addresses, size a multiple
// of 16), completing `bytes` transactions on `bar`.
__device__ __forceinline__ void bulk_load(void * dst, const void * src, uint32_t bytes, uint64_t * bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 ::"r"(smem_u32(dst)), "l"((uint64_t) src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}

// 2-SM (cta_group::2) loads: the data lands in this CTA's shared memory, the transaction bytes are
// counted on `bar_cluster` (a shared::cluster address: the pair leader's barrier). No multicast.
__device__ __forceinline__ void tma_load_2d_cg2(void * dst, const CUtensorMap * m, uint32_t bar_cluster, int c0, int c1) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];"
        ::"r"(smem_u32(dst)), "l"((uint64_t) m), "r"(bar_cluster), "r"(c0), "r"(c1)
        : "memory");
}
__device__ __forceinline__ void tma_load_3d_cg2(void * dst, const CUtensorMap * m, uint32_t bar_cluster, int c0, int c1, int c2) {
    asm volatile(
        "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];"
        ::"r"(smem_u32(dst)), "l"((uint64_t) m), "r"(bar_cluster), "r"(c0), "r"(c1), "r"(c2)
        : "memory");
}

// ---------------------------------------------------------------- tcgen05
__device__ __forceinline__ void tmem_alloc(uint32_t * slot, uint32_t ncols) {      // whole warp
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)), "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {     // whole warp
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[smem] · B[smem]^T, M=128, one elected thread issues.
__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n"
        ::"r"(d_tmem), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc)
        : "memory");
}
// D[tmem] (+)= A[tmem] · B[smem]^T: the A operand (M=128 rows on the TMEM lanes, two 16-bit
// elements per 32-bit column, K=16 per instruction = 8 columns) read from tensor memory.
__device__ __forceinline__ void umma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n"
        ::"r"(d_tmem), "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(acc)
        : "memory");
}
// CTA-pair versions: TMEM allocation by the same warp of both CTAs; the MMA issued by the pair
// leader with M = 256 (each CTA holds 128 rows of A and half of B's N); commits arrive on the
// barrier at the same offset in both CTAs.
__device__ __forceinline__ void tmem_alloc2(uint32_t * slot, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)), "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc2(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void umma2_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n}\n"
        ::"r"(d_tmem), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc)
        : "memory");
}
__device__ __forceinline__ void umma2_commit_pair(uint64_t * bar) {
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;"
        ::"r"(smem_u32(bar)), "h"((uint16_t) 3)
        : "memory");
}

// Arrive once on bar when every tcgen05 op issued so far by this thread has completed.
__device__ __forceinline__ void umma_commit(uint64_t * bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

// Shared-memory matrix descriptor, K-major, 128-byte swizzle, 8-row core groups 1024 B apart.
__device__ __forceinline__ uint64_t umma_desc_sw128(const void * smem_tile) {
    const uint32_t a = smem_u32(smem_tile);
    uint64_t d = 0;
    d |= (uint64_t) ((a & 0x3FFFFu) >> 4);          // start address   [0,14)
    d |= (uint64_t) 1u << 16;                        // LBO (unused for swizzled K-major) [16,30)
    d |= (uint64_t) (1024u >> 4) << 32;              // SBO = 1024 B    [32,46)
    d |= (uint64_t) 1u << 46;                        // descriptor version (sm100) [46,48)
    d |= (uint64_t) 2u << 61;                        // layout: SWIZZLE_128B [61,64)
    return d;
}

// Same, MN-major (the N index contiguous in 128-byte rows, one row per K index), for an operand whose
// N extent is one 64-element swizzle atom: 8-row groups along K are 1024 B apart (SBO); a K step of
// 16 advances the start address by 2048 B.
__device__ __forceinline__ uint64_t umma_desc_sw128_mn(const void * smem_tile) {
    const uint32_t a = smem_u32(smem_tile);
    uint64_t d = 0;
    d |= (uint64_t) ((a & 0x3FFFFu) >> 4);          // start address
    d |= (uint64_t) 1u << 16;                        // LBO (one atom along N: unused)
    d |= (uint64_t) (1024u >> 4) << 32;              // SBO = 1024 B between 8-row groups along K
    d |= (uint64_t) 1u << 46;                        // descriptor version (sm100)
    d |= (uint64_t) 2u << 61;                        // SWIZZLE_128B
    return d;
}

// Instruction descriptor, kind::f16: f32 accumulate, A/B both f16 (ab_bf16=0) or both bf16 (1),
// A K-major, B K-major (b_mn = 0) or MN-major (1), M=128, N=n.
__host__ __device__ constexpr uint32_t umma_idesc_f16(int n, int ab_bf16, int b_mn = 0, int m = 128) {
    return (1u << 4)                                   // D format f32
         | ((uint32_t) ab_bf16 << 7) | ((uint32_t) ab_bf16 << 10)
         | ((uint32_t) b_mn << 16)                     // B major-ness
         | ((uint32_t) (n >> 3) << 17)
         | ((uint32_t) (m >> 4) << 24);
}

// make this thread's generic-proxy shared-memory writes visible to the async proxy (tcgen05.mma)
__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// plain arrive on a CTA-local mbarrier
__device__ __forceinline__ void mbar_arrive(uint64_t * bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// 32 consecutive 32-bit columns of this thread's TMEM lane from registers (warp-collective), and
// the wait for this thread's TMEM stores to complete.
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t * r) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};"
        ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
          "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]),
          "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]),
          "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// 32 lanes x 32 consecutive f32 columns from TMEM into registers (one row per thread).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float * v) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// 32 lanes x 16 consecutive f32 columns (one row per thread); the load and its wait in one statement.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float * v) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n"
        "tcgen05.wait::ld.sync.aligned;"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr)
        : "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// ---------------------------------------------------------------- programmatic dependent launch
// Kernels are launched with programmatic stream serialisation: the next kernel may start while
// this one runs. pdl_wait() blocks until every upstream grid has completed and its writes are
// visible; every thread calls it before its first read of upstream outputs or its first global
// write. pdl_trigger() lets the downstream grid begin launching (it still waits in pdl_wait).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ---------------------------------------------------------------- thread-block clusters
__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
// Every thread of every CTA in the cluster must execute this (it is a hardware barrier, so the
// kernels place it on paths that all threads take, abort paths included).
__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Address of the same shared-memory location in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t dsmem_map(uint32_t saddr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
    return r;
}
__device__ __forceinline__ float4 dsmem_ld4(uint32_t addr) {
    float4 v;
    asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(addr)
                 : "memory");
    return v;
}

// named barrier over the 128 epilogue threads (warps 0-3)
__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, 128;" ::: "memory"); }
// named barrier 1 over the first n threads of the block (n a multiple of 32)
__device__ __forceinline__ void epi_bar_n(int n) { asm volatile("bar.sync 1, %0;" ::"r"(n) : "memory"); }

} // namespace tsn
