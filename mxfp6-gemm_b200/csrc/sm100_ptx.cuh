#pragma once
// Thin inline-PTX wrappers for the sm_100a features the MXFP6 kernels use: mbarriers, TMA
// (cp.async.bulk[.tensor]), tensor memory (tcgen05.alloc / cp / mma / commit / ld) and the
// shared-memory matrix descriptors tcgen05.mma and tcgen05.cp read. Field layouts follow the
// PTX ISA (tcgen05 "shared memory descriptor" and "instruction descriptor" tables).
//
// Every wait in this library is bounded: wait_parity_bounded() gives up after a cycle budget
// and returns false, and the callers turn that into a status bit instead of spinning forever.
#include <cstdint>

namespace mxfp6 {
namespace sm100 {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---- mbarrier --------------------------------------------------------------------------------

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_async_shared() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(bar),
                 "r"(bytes)
                 : "memory");
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

// Non-blocking probe: has the phase with the given parity completed?
__device__ __forceinline__ bool mbar_test_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}

// try_wait with a suspend-time hint: the thread may be suspended in hardware until the phase
// completes (which wakes it at once) or about `ns` nanoseconds have passed.
__device__ __forceinline__ bool mbar_try_wait_suspend(uint32_t bar, uint32_t parity, uint32_t ns) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity), "r"(ns)
        : "memory");
    return ok != 0;
}

// Longest suspension per poll of a bounded wait. It only delays noticing *abort or the end of
// the budget; a completed phase ends the suspension at once.
constexpr uint32_t WAIT_SUSPEND_NS = 100000;

// Wait until the phase with the given parity has completed. Returns false when `budget` clock
// cycles pass first, or once *abort has become non-zero (another role already gave up). Polls
// after the first one suspend the thread instead of re-issuing at once: the waiting producer,
// MMA and epilogue threads then take no issue slots and little power while the tensor cores run,
// which on B200 measures 1-3.5% faster on power-capped shapes, with no cost on small ones.
__device__ __forceinline__ bool wait_parity_bounded(uint32_t bar, uint32_t parity,
                                                    const volatile int* abort, long long budget) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    while (true) {
        if (mbar_try_wait_suspend(bar, parity, WAIT_SUSPEND_NS)) return true;
        if (*abort) return false;
        if (clock64() - t0 > budget) return false;
    }
}

// Spin for about `ns` nanoseconds (bounded settle time on abort paths).
__device__ __forceinline__ void settle_ns(unsigned long long ns) {
    unsigned long long t0, t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
    do {
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    } while (t - t0 < ns);
}

// ---- cp.async (non-bulk) ------------------------------------------------------------------------
// 4-byte asynchronous global -> shared copies for operands the tensor-memory accelerator cannot
// address. src_bytes < 4 zero-fills the rest of the word (0 reads nothing). Completion is
// signalled to an mbarrier with cp_async_mbar_arrive_noinc; the consumer waits on that barrier
// before tcgen05.mma reads the data.
__device__ __forceinline__ void cp_async_4(uint32_t dst, const void* src, uint32_t src_bytes) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}

__device__ __forceinline__ void cp_async_wait_all() {
    asm volatile("cp.async.wait_all;" ::: "memory");
}

// Arrive on a local mbarrier once every cp.async this thread issued so far has landed; counts as
// one of the barrier's expected arrivals (.noinc). The thread does not wait.
__device__ __forceinline__ void cp_async_mbar_arrive_noinc(uint32_t bar) {
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(bar) : "memory");
}

// ---- programmatic dependent launch --------------------------------------------------------------
// The GEMM, split-K reduce and A re-pad kernels are launched with programmatic stream
// serialization: such a kernel may begin while the previous kernel in its stream is still
// running, and touches global memory only after griddep_wait(), which returns once that kernel has
// completed and its memory is visible (a no-op for a kernel launched without the attribute). Each
// of them waits before its first global access, so stream order holds for whatever kernels precede
// or follow it. The library's other kernels (quantiser, layout import) launch without the
// attribute and keep plain stream order.

// Let the next kernel in the stream begin its set-up once every CTA of this grid has issued this
// (or exited).
__device__ __forceinline__ void griddep_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void griddep_wait() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
}

// ---- TMA ---------------------------------------------------------------------------------------

__device__ __forceinline__ void prefetch_tmap(const void* tmap) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(tmap) : "memory");
}

// 2-D tiled tensor load into this CTA's shared memory, completion on `bar` (bytes counted).
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const void* tmap, uint32_t bar, int c0,
                                            int c1) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
        "l"(tmap), "r"(bar), "r"(c0), "r"(c1)
        : "memory");
}

// Untiled bulk copy global -> shared (16-byte aligned addresses, size a multiple of 16).
__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes,
                                          uint32_t bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
            "r"(dst),
        "l"(src), "r"(bytes), "r"(bar)
        : "memory");
}

// ---- tensor memory -------------------------------------------------------------------------------

// Warp-wide: allocate `ncols` columns (power of two >= 32); the address lands in shared memory.
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

__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Shared-memory matrix descriptor (tcgen05 "matrix descriptor"):
//   [0,14) start address >> 4 | [16,30) leading byte offset >> 4 | [32,46) stride byte offset >> 4
//   [46,48) fixed 0b01 | [49,52) base offset | [52] LBO mode | [61,64) swizzle mode
//   (0 none, 2 = 128-byte swizzle).
__device__ __forceinline__ uint64_t make_smem_desc(uint32_t saddr, uint32_t lbo_bytes,
                                                   uint32_t sbo_bytes, uint32_t swizzle) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr & 0x3FFFF) >> 4);
    d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFF) << 16;
    d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFF) << 32;
    d |= (uint64_t)1 << 46;
    d |= (uint64_t)(swizzle & 7) << 61;
    return d;
}

// K-major operand staged by TMA with 128-byte swizzle: rows of 128 bytes, 8-row groups
// 1024 bytes apart. Stepping K by 32 elements (32 bytes in the padded FP6 layout) adds 2 to
// the start-address field.
__device__ __forceinline__ uint64_t make_kmajor_sw128_desc(uint32_t saddr) {
    return make_smem_desc(saddr, 16, 1024, 2);
}

// Scale-factor source for tcgen05.cp.32x128b: 32 rows of 16 bytes, contiguous, no swizzle.
__device__ __forceinline__ uint64_t make_sf_desc(uint32_t saddr) {
    return make_smem_desc(saddr, 0, 128, 0);
}

// Source for tcgen05.cp.128x256b: 128 rows of 32 bytes as two 16-byte columns, no swizzle. Column
// h (2048 bytes apart) holds rows 0..127 of 16 bytes each, 8-row groups 128 bytes apart; with
// scale atom h staged four times over, row i reads that atom's row i % 32.
__device__ __forceinline__ uint64_t make_sf_wide_desc(uint32_t saddr) {
    return make_smem_desc(saddr, 2048, 128, 0);
}

// Copy one 32-row x 128-bit scale chunk from shared memory into tensor memory columns
// [taddr, taddr+4), replicated into all four 32-lane quarters.
__device__ __forceinline__ void tc_cp_32x128b_warpx4(uint32_t taddr, uint64_t sdesc) {
    asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc)
                 : "memory");
}

// Block-scaled MXF8F6F4 MMA, A and B from shared memory, D (FP32) in tensor memory:
//   D = (accumulate ? D : 0) + (A * sfA) x (B * sfB)^T
__device__ __forceinline__ void tc_mma_mxf8f6f4(uint32_t d_taddr, uint64_t adesc, uint64_t bdesc,
                                                uint32_t idesc, uint32_t sfa_taddr,
                                                uint32_t sfb_taddr, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], p;\n\t}" ::
            "r"(d_taddr),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(sfa_taddr), "r"(sfb_taddr)
        : "memory");
}

// Arrive once on `bar` when every tcgen05 operation this thread issued so far has completed.
__device__ __forceinline__ void tc_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                 : "memory");
}

// Instruction descriptor for kind::mxf8f6f4 with E2M3 x E2M3, E8M0 scales, K-major A and B.
//   [4,6) B scale id | [7,10) A format (3 = E2M3) | [10,13) B format | [15] A major | [16] B major
//   [17,23) N >> 3 | [23] scale format (1 = E8M0) | [24,29) M >> 4 | [29,31) A scale id
__host__ __device__ constexpr uint32_t make_idesc_e2m3(int M, int N) {
    return (3u << 7) | (3u << 10) | ((uint32_t)(N >> 3) << 17) | (1u << 23) |
           ((uint32_t)(M >> 4) << 24);
}
__device__ __forceinline__ uint32_t idesc_with_sf_ids(uint32_t idesc, uint32_t a_id, uint32_t b_id) {
    return idesc | (b_id << 4) | (a_id << 29);
}

// 32 lanes x 32 consecutive 32-bit columns per warp (one row per thread).
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
          "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
          "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
          "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr)
        : "memory");
}
__device__ __forceinline__ void tmem_ld_wait() {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// tcgen05.wait::ld naming the registers a tcgen05.ld wrote: their values are valid only after
// the wait, and the in-out operands keep every use of them after it (a plain wait carries no
// dependency on them, so the compiler could move a use above it). No instruction is added.
__device__ __forceinline__ void tmem_ld_wait(uint32_t (&r)[32]) {
    asm volatile("tcgen05.wait::ld.sync.aligned;"
        : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
          "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15]),
          "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]), "+r"(r[22]), "+r"(r[23]),
          "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]), "+r"(r[30]), "+r"(r[31])
        :
        : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns per warp from registers (one row per thread).
__device__ __forceinline__ void tmem_st_32x32b_x32(uint32_t taddr, const uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
        "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]),
        "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]),
        "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}
__device__ __forceinline__ void tmem_st_wait() {
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// ---- global flags between CTAs of one grid ----------------------------------------------------

__device__ __forceinline__ unsigned long long ld_acquire_gpu_u64(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_gpu_u64(unsigned long long* p, unsigned long long v) {
    asm volatile("st.release.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
// 16 bytes from global memory, cached in L2 only (data another CTA wrote during this grid).
__device__ __forceinline__ uint4 ld_cg_v4(const void* p) {
    uint4 v;
    asm volatile("ld.global.cg.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p)
                 : "memory");
    return v;
}


// ---- clusters and CTA pairs (cta_group::2) ------------------------------------------------------
//
// Two CTAs of a (2,1,1) cluster share one tcgen05.mma: rank 0 (the leader) issues it, reading
// A rows [0,128) and B rows [0,128) from its own shared memory and rows [128,256) from the same
// offsets in rank 1's. Loads of either CTA report to the leader's mbarriers.

__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

// Address of the same shared-memory offset in CTA `rank` of this cluster.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
    return r;
}

__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Arrive on an mbarrier of any CTA in the cluster (shared::cluster address), releasing this
// thread's prior memory operations at cluster scope: for a barrier that hands over shared-memory
// data this thread's CTA wrote and another CTA's tensor core reads.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_bar) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_bar) : "memory");
}

// The same arrive with the release at CTA scope, for barriers that only order tensor-memory
// accesses: the epilogue has finished its tcgen05.ld / tcgen05.st (tcgen05.wait::ld / ::st, then
// tcgen05.fence::before_thread_sync), and the MMA thread that waits on the barrier issues
// tcgen05.fence::after_thread_sync before touching those columns. The cluster-scope release costs
// about 1000 cycles per arrive on B200 and sits on the path between two tiles' MMAs; on the pair
// kernel this form measured 1-4.6% faster (cfg2 +2.4%), with identical results.
__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_bar) {
    asm volatile("mbarrier.arrive.release.cta.shared::cluster.b64 _, [%0];" ::"r"(cluster_bar) : "memory");
}

// Tensor loads into this CTA's shared memory that complete on an mbarrier of either CTA of the
// pair (`bar` is a shared::cluster address, normally the leader's).
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const void* tmap, uint32_t bar, int c0, int c1) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
        "l"(tmap), "r"(bar), "r"(c0), "r"(c1)
        : "memory");
}
__device__ __forceinline__ void tma_load_3d_pair(uint32_t dst, const void* tmap, uint32_t bar, int c0, int c1,
                                                 int c2) {
    asm volatile(
        "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(dst),
        "l"(tmap), "r"(bar), "r"(c0), "r"(c1), "r"(c2)
        : "memory");
}

__device__ __forceinline__ void tma_load_4d_pair(uint32_t dst, const void* tmap, uint32_t bar, int c0, int c1,
                                                 int c2, int c3) {
    asm volatile(
        "cp.async.bulk.tensor.4d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(dst),
        "l"(tmap), "r"(bar), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
        : "memory");
}

__device__ __forceinline__ void tmem_alloc_pair(uint32_t dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem), "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// Each CTA of the pair copies its own shared-memory scale chunk into its own tensor memory.
__device__ __forceinline__ void tc_cp_32x128b_warpx4_pair(uint32_t taddr, uint64_t sdesc) {
    asm volatile("tcgen05.cp.cta_group::2.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
}

// 128 rows x 256 bits from shared memory into tensor memory columns [taddr, taddr+8): row i lands in
// lane i, no broadcast. taddr's column is a multiple of 8.
__device__ __forceinline__ void tc_cp_128x256b_pair(uint32_t taddr, uint64_t sdesc) {
    asm volatile("tcgen05.cp.cta_group::2.128x256b [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
}

__device__ __forceinline__ void tc_mma_mxf8f6f4_pair(uint32_t d_taddr, uint64_t adesc, uint64_t bdesc,
                                                     uint32_t idesc, uint32_t sfa_taddr, uint32_t sfb_taddr,
                                                     uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], p;\n\t}" ::"r"(d_taddr),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(sfa_taddr), "r"(sfb_taddr)
        : "memory");
}

// Arrive once on the mbarrier at this offset in every CTA of `cta_mask` when all tcgen05
// operations issued so far by this thread have completed.
__device__ __forceinline__ void tc_commit_pair(uint32_t bar, uint16_t cta_mask) {
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(bar),
        "h"(cta_mask)
        : "memory");
}

}  // namespace sm100
}  // namespace mxfp6
