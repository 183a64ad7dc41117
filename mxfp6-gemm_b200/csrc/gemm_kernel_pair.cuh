#pragma once
// The B200 MXFP6 GEMM kernel for large shapes: a CTA pair (cluster of 2, tcgen05 cta_group::2)
// computes a 256 x 256 output tile with one MMA stream.
//
// Same math as gemm_mxfp6_sm100 (gemm_kernel.cuh); the pair layout halves what each SM stages:
//   * CTA r of the pair loads A rows [m0 + 128r, +128) and B^T rows [n0 + 128r, +128) of every
//     128-deep K slab (16U6 unpack, 128-byte swizzle), its own A scale atom, and both B scale
//     atoms four times over (one tensor load through a zero-stride repeat dimension), with zero
//     fill past the edges, into a 5-stage ring; all loads of both CTAs report to the leader's
//     (rank 0) full barrier.
//   * The leader's MMA thread copies the scales into each CTA's tensor memory, two copies per
//     slab: A's atom with the broadcasting 32x128b.warpx4 copy, and B's 256 rows with one
//     128x256b copy from the fourfold-staged atoms. B's scales are needed in all four lane
//     quarters. One wide copy instead of two broadcast copies made the kernel 4-5% faster.
//     It then issues tcgen05.mma.cta_group::2 (M = 256, N = 256, K = 32) four times per slab;
//     each CTA's tensor memory receives its 128 rows x 256 FP32 columns. tcgen05.commit
//     multicasts slot releases and "accumulator ready" to both CTAs.
//   * Two accumulators share tensor memory with a 32-column overlap: buffer 0 = columns [0,256),
//     buffer 1 = [224,480); B scales at [480,488), A scales at [488,492). The epilogue reads buffer 0 from its top chunk
//     down and buffer 1 from its bottom chunk up, so the overlap chunk is read first and the
//     next tile's MMAs may start as soon as that one chunk has left tensor memory; the rest of
//     the epilogue runs under the next tile's main loop.
//   * The persistent pairs take 256 x 256 tiles round-robin. When the tiles do not fill whole
//     waves (and the router finds the idle part of the last wave deep enough to repay it, see
//     route.hpp), the last wave and one before it run stream-K: their tiles' K slabs, in tile order,
//     are cut into one contiguous range per pair, so every pair does the same number of slabs.
//     A tile that straddles two ranges is summed by one accumulator chain: the first pair's
//     epilogue hands its FP32 accumulator to the second through the workspace (a flag released
//     at GPU scope), and the second loads it into tensor memory (tcgen05.st) and continues the
//     same MMA sequence. Each output element sums its K slabs in order exactly as in the
//     whole-tile schedule, so results are bit-identical. A pair computes its hand-off first and the
//     tile it takes over last, so the handing pair finished long before (the wait is bounded).
//   * No TMA multicast anywhere: each CTA fetches its own operands.
//   * A compact A (a row stride the 16U6 load cannot address) is copied into the A stages by
//     four extra loader warps per CTA instead (AMODE = A_CPASYNC, compact_a.cuh).
//   * The epilogue writes D to every destination of p.dst (one for a plain GEMM; this rank's and
//     its peers' gathered outputs for mxfp6_gemm_gather). With several destinations each warp
//     regroups its rows through a small shared-memory area so that every destination receives
//     128-byte runs of a row (store_rows_regrouped).
// Every wait is bounded (see gemm_kernel.cuh); a timeout also raises the peer's abort flag.
#include "gemm_kernel.cuh"

namespace mxfp6 {
namespace kern {

template <int AMODE = A_TMA>
struct PairConfig {
    static constexpr int BM = 256;  // rows per pair tile (128 per CTA)
    static constexpr int BN = 256;  // columns per pair tile (B rows 128 per CTA)
    static constexpr int SUB = 1;                        // 128-deep slabs per stage
    static constexpr int STAGES = 5;
    static constexpr int SLAB_BYTES = 128 * BK;          // one 128-row x 128-K box in shared memory
    static constexpr int A_BYTES = SUB * SLAB_BYTES;
    static constexpr int B_BYTES = SUB * SLAB_BYTES;
    static constexpr int AB_STAGE = A_BYTES + B_BYTES;
    static constexpr int SFA_BYTES = 512;                // own A atom
    // B's two atoms, each four times over (atom 0 x4, then atom 1 x4): the source of one
    // 128x256b tensor-memory copy, which fills all four lane quarters without broadcasting.
    static constexpr int SFB_BYTES = 4 * 1024;
    static constexpr int SF_STAGE = SFA_BYTES + SFB_BYTES;
    static constexpr int TMEM_COLS = 512;
    static constexpr int BUF1_COL = 224;  // buffer 1 starts 32 columns below buffer 0's end
    static constexpr int TMEM_SFB = 480;  // B scales: 8 columns (8-column aligned for the wide copy)
    static constexpr int TMEM_SFA = 488;  // A scales: 4 columns
    static_assert(TMEM_SFA + 4 <= 512, "tensor memory budget");
    static constexpr int EPI_WARPS = 4;
    static constexpr int BAR_BYTES = 256;
    static constexpr int SK_TILE_FLOATS = BM * BN;  // one hand-off slot: a 256 x 256 FP32 accumulator
    static constexpr int SMEM_BYTES = 1024 + STAGES * (AB_STAGE + SF_STAGE) + BAR_BYTES + EPI_STG_BYTES;
    static_assert(SMEM_BYTES <= 227 * 1024, "shared memory budget");
};

__device__ __forceinline__ void store_cluster_u32(uint32_t cluster_addr, uint32_t v) {
    asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(cluster_addr), "r"(v) : "memory");
}

// Work of one CTA pair, in the order the pair processes it. The pair owns its whole tiles
// (round-robin over tiles [0, sk_first)) and its stream-K range [lo, hi) of the remaining tiles'
// K slabs (flattened in tile order, k_slabs per tile). It first computes the start segment of the
// tile its range ends inside and hands that accumulator off, so the next pair finds it ready long
// before it needs it; then its round-robin tiles; then the whole tiles inside its range; last the
// end segment of the tile its range begins inside, taken over from the previous pair. A range is
// at least one tile long, so no tile has a middle segment.
constexpr int UNIT_WHOLE = 0;      // all K slabs of a tile (or one split-K segment)
constexpr int UNIT_HAND_OFF = 1;   // a tile's first slabs: the accumulator goes to the next pair
constexpr int UNIT_TAKE_OVER = 2;  // a tile's last slabs, continuing the previous pair's accumulator

struct PairUnit {
    TileCoord tc;  // tile coordinates; kb_begin / kb_count are this unit's K slabs
    int mode;
    int slot;      // hand-off slot (the handing pair's index)
};

struct PairWork {
    int n_whole;        // round-robin whole tiles
    int n;              // units in all
    long long lo, hi;   // stream-K slab range
    bool hand_off, take_over;
    int f0, f1;         // whole tiles inside the range, as indices from sk_first
};

// Banded split: first slab of short band j of band_n over [band_L * band_a, k_slabs).
__device__ __forceinline__ int band_short_begin(const Params& p, int j) {
    const int ks = p.k_slabs - p.band_L * p.band_a;
    return p.band_L * p.band_a + (int)((long long)ks * j / p.band_n);
}

// SK: the launch may run a stream-K tail (hand-offs between pairs). A launch without one is
// instantiated without that code (SK = false).
template <bool SK>
__device__ __forceinline__ PairWork pair_work(const Params& p, int pair, int npairs) {
    PairWork w;
    if (p.band_L > 0) {
        // banded split: one long band per pair on the first band_L * T pairs, short bands
        // round-robin on the rest (pair_unit)
        const int T = p.m_blocks * p.n_blocks, longp = p.band_L * T;
        const int R = npairs - longp, units = p.band_n * T, r = pair - longp;
        w.n_whole = 0;
        w.n = pair < longp ? 1 : (R > 0 && r < units ? (units - r + R - 1) / R : 0);
        w.lo = w.hi = 0;
        w.hand_off = w.take_over = false;
        w.f0 = w.f1 = 0;
        return w;
    }
    const int tiles = p.m_blocks * p.n_blocks * p.splits;
    const int rr = SK && p.sk_total > 0 ? p.sk_first : tiles;
    w.n_whole = pair < rr ? (rr - pair + npairs - 1) / npairs : 0;
    w.n = w.n_whole;
    w.lo = w.hi = 0;
    w.hand_off = w.take_over = false;
    w.f0 = w.f1 = 0;
    if (SK && p.sk_total > 0) {
        const long long ks = p.k_slabs;
        w.lo = p.sk_total * pair / npairs;
        w.hi = p.sk_total * (pair + 1) / npairs;
        w.hand_off = (w.hi % ks) != 0;
        w.take_over = (w.lo % ks) != 0;
        w.f0 = (int)((w.lo + ks - 1) / ks);
        w.f1 = (int)(w.hi / ks);
        w.n += (w.hand_off ? 1 : 0) + (w.f1 - w.f0) + (w.take_over ? 1 : 0);
    }
    return w;
}

template <bool SK>
__device__ __forceinline__ PairUnit pair_unit(const Params& p, const PairWork& w, int pair, int npairs, int i) {
    PairUnit u;
    u.mode = UNIT_WHOLE;
    u.slot = 0;
    const int ks = p.k_slabs;
    if (p.band_L > 0) {
        const int T = p.m_blocks * p.n_blocks, longp = p.band_L * T;
        if (pair < longp) {
            u.tc = decode_tile(pair % T, p);
            u.tc.split = pair / T;
            u.tc.kb_begin = u.tc.split * p.band_a;
            u.tc.kb_count = p.band_a;
        } else {
            const int v = (pair - longp) + i * (npairs - longp), j = v / T;
            u.tc = decode_tile(v % T, p);
            u.tc.split = p.band_L + j;
            u.tc.kb_begin = band_short_begin(p, j);
            u.tc.kb_count = band_short_begin(p, j + 1) - u.tc.kb_begin;
        }
        return u;
    }
    if (SK && w.hand_off) {
        if (i == 0) {
            u.tc = decode_tile(p.sk_first + (int)(w.hi / ks), p);
            u.tc.kb_begin = 0;
            u.tc.kb_count = (int)(w.hi % ks);
            u.mode = UNIT_HAND_OFF;
            u.slot = pair;
            return u;
        }
        i--;
    }
    if (i < w.n_whole) {
        u.tc = decode_tile(pair + i * npairs, p);
        return u;
    }
    const int j = i - w.n_whole;
    if (j < w.f1 - w.f0) {
        u.tc = decode_tile(p.sk_first + w.f0 + j, p);
        return u;
    }
    u.tc = decode_tile(p.sk_first + (int)(w.lo / ks), p);
    u.tc.kb_begin = (int)(w.lo % ks);
    u.tc.kb_count = ks - u.tc.kb_begin;
    u.mode = UNIT_TAKE_OVER;
    u.slot = pair - 1;
    return u;
}

// AMODE (compact_a.cuh): A_TMA loads A with the 16U6 tensor load; A_CPASYNC adds four
// loader warps per CTA that build the A image from p.a_ptr, and whose arrivals join the leader's
// full barrier.
// EPI (non-partial launches): which optional epilogue paths the instantiation carries. EPI_LEAN
// has neither; EPI_STREAM_K adds the stream-K tail's hand-offs; EPI_ALL also writes several
// destinations (gather). A launch uses the smallest that covers it: the unused code measured
// 2-11% slower on shapes that never ran it.
constexpr int EPI_LEAN = 0, EPI_STREAM_K = 1, EPI_ALL = 2;
template <typename OutT, bool PARTIAL, int AMODE = A_TMA, int EPI = EPI_ALL>
__global__ void __launch_bounds__(threads_for(AMODE), 1)
    gemm_mxfp6_sm100_pair(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                          const __grid_constant__ CUtensorMap tmSA, const __grid_constant__ CUtensorMap tmSB,
                          const Params p) {
    using C = PairConfig<AMODE>;
    constexpr bool COMPACT = AMODE != A_TMA;
    static_assert(C::SUB == 1, "one 128-deep slab per stage");
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    const uint32_t raw_u32 = sm100::smem_u32(smem_raw);
    const uint32_t base = (raw_u32 + 1023u) & ~1023u;
    uint8_t* base_ptr = smem_raw + (base - raw_u32);

    const uint32_t ab_base = base;
    const uint32_t sf_base = base + C::STAGES * C::AB_STAGE;
    const uint32_t bar_base = sf_base + C::STAGES * C::SF_STAGE;
    uint8_t* bar_ptr = base_ptr + (bar_base - base);
    // barriers: full[S], empty[S], acc_full[2], acc_empty[2], ovl_free, drain, fill, handed
    auto full_bar = [&](int s) { return bar_base + 8u * s; };
    auto empty_bar = [&](int s) { return bar_base + 8u * (C::STAGES + s); };
    const uint32_t acc_full0 = bar_base + 8u * (2 * C::STAGES);
    const uint32_t acc_empty0 = acc_full0 + 16u;
    const uint32_t ovl_free = acc_full0 + 32u;
    const uint32_t drain_bar = acc_full0 + 40u;
    const uint32_t fill_bar = acc_full0 + 48u;    // leader: both CTAs loaded a taken-over accumulator
    const uint32_t handed_bar = acc_full0 + 56u;  // this CTA's epilogue warps stored a hand-off
    const int slot_off = 8 * (2 * C::STAGES + 8);
    static_assert(8 * (2 * C::STAGES + 8) + 16 <= C::BAR_BYTES, "barrier area");
    uint8_t* epi_stg = bar_ptr + C::BAR_BYTES;  // EPI_STG_BYTES: output regrouping (several destinations)
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar_ptr + slot_off);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(bar_ptr + slot_off + 8);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t rank = sm100::cluster_ctarank();
    const uint32_t peer = rank ^ 1u;
    const uint32_t peer_abort = sm100::mapa_shared(sm100::smem_u32((const void*)abort_flag), peer);
    auto raise = [&](unsigned int bit) {
        atomicOr(&g_device_status, bit);
        *abort_flag = 1;
        store_cluster_u32(peer_abort, 1);
    };

    if (threadIdx.x == 0) {
        for (int s = 0; s < C::STAGES; s++) {
            // A_CPASYNC: leader = producer + own loader threads + the peer's relay; the peer's
            // barrier counts its own loader threads.
            uint32_t n = 1;
            if (AMODE == A_CPASYNC) n = rank == 0 ? 2 + LOADER_THREADS : LOADER_THREADS;
            sm100::mbar_init(full_bar(s), n);
            sm100::mbar_init(empty_bar(s), 1);
        }
        for (int b = 0; b < 2; b++) {
            sm100::mbar_init(acc_full0 + 8u * b, 1);
            sm100::mbar_init(acc_empty0 + 8u * b, 2 * C::EPI_WARPS);
        }
        sm100::mbar_init(ovl_free, 2 * C::EPI_WARPS);
        sm100::mbar_init(drain_bar, 1);
        sm100::mbar_init(fill_bar, 2 * C::EPI_WARPS);
        sm100::mbar_init(handed_bar, C::EPI_WARPS);
        *abort_flag = 0;
        sm100::fence_mbar_init();
        sm100::fence_async_shared();
        if (AMODE == A_TMA) sm100::prefetch_tmap(&tmA);
        sm100::prefetch_tmap(&tmB);
        sm100::prefetch_tmap(&tmSA);
        sm100::prefetch_tmap(&tmSB);
    }

    if (warp == 1) {
        sm100::tmem_alloc_pair(sm100::smem_u32(tmem_slot), C::TMEM_COLS);
        sm100::tmem_relinquish_pair();
    }
    sm100::tc_fence_before();
    __syncthreads();
    sm100::cluster_sync();  // the peer's loads and arrivals target barriers initialised above
    sm100::tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    // Set-up done (it reads only kernel parameters): the next kernel may start its own, and this
    // one waits for the previous kernel's memory before its first global access.
    sm100::griddep_launch_dependents();
    sm100::griddep_wait();

    const int cluster_id = blockIdx.x >> 1;
    const int num_clusters = gridDim.x >> 1;
    constexpr bool XF = EPI >= EPI_STREAM_K && !PARTIAL;  // stream-K hand-offs possible
    constexpr bool XG = EPI == EPI_ALL && !PARTIAL;        // several destinations possible
    const PairWork work = pair_work<XF>(p, cluster_id, num_clusters);
    // Abort bookkeeping, read after the roles have finished (see the end of the kernel): the
    // producer's last load per stage and its phase parity, and whether any MMA was issued.
    uint32_t issued_mask = 0, issued_phase = 0;
    bool mma_issued = false;

    if (warp == 0) {
        if (lane == 0) {
            // ---------------- TMA producer (both CTAs) ----------------
            int stage = 0;
            uint32_t phase = 0;
            bool ok = true;
            // the leader's barrier counts both CTAs' bytes: A (unless compact), B, scales
            constexpr uint32_t tx = 2u * ((COMPACT ? 0u : (uint32_t)A_TMA_BYTES) + 128u * (BK * 3 / 4) +
                                          (uint32_t)C::SF_STAGE);
            for (int ui = 0; ui < work.n && ok; ui++) {
                const PairUnit u = pair_unit<XF>(p, work, cluster_id, num_clusters, ui);
                const TileCoord& tc = u.tc;
                const int a_row = tc.mb * C::BM + 128 * (int)rank;
                const int b_row = tc.nb * C::BN + 128 * (int)rank;
                for (int i = 0; i < tc.kb_count; i++) {
                    if (!sm100::wait_parity_bounded(empty_bar(stage), phase ^ 1u, abort_flag, p.wait_budget)) {
                        if (!*abort_flag) raise(0x1u);
                        *abort_flag = 1;
                        ok = false;
                        break;
                    }
                    const int kb = tc.kb_begin + i;
                    const uint32_t fb = sm100::mapa_shared(full_bar(stage), 0);
                    if (rank == 0) sm100::mbar_arrive_expect_tx(full_bar(stage), tx);
                    const uint32_t a_dst = ab_base + stage * C::AB_STAGE;
                    if (!COMPACT) sm100::tma_load_2d_pair(a_dst, &tmA, fb, kb * BK, a_row);
                    sm100::tma_load_2d_pair(a_dst + C::A_BYTES, &tmB, fb, kb * BK, b_row);
                    // scale atoms past the last row block read as zero
                    const uint32_t sf_dst = sf_base + stage * C::SF_STAGE;
                    sm100::tma_load_3d_pair(sf_dst, &tmSA, fb, 0, kb, tc.mb * 2 + (int)rank);
                    sm100::tma_load_4d_pair(sf_dst + C::SFA_BYTES, &tmSB, fb, 0, 0, kb, tc.nb * 2);
                    issued_mask |= 1u << stage;
                    issued_phase = (issued_phase & ~(1u << stage)) | (phase << stage);
                    if (++stage == C::STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0 && rank == 0) {
            // ---------------- MMA issuer (leader only) ----------------
            const uint64_t a_desc0 = sm100::make_kmajor_sw128_desc(ab_base);
            const uint64_t b_desc0 = sm100::make_kmajor_sw128_desc(ab_base + C::A_BYTES);
            int stage = 0;
            uint32_t phase = 0;
            bool ok = true;
            constexpr uint32_t idesc = sm100::make_idesc_e2m3(C::BM, C::BN);
            uint32_t idesc_k[BK / 32];  // scale id k selects byte k of each scale word
#pragma unroll
            for (int k = 0; k < BK / 32; k++) idesc_k[k] = sm100::idesc_with_sf_ids(idesc, k, k);
            const uint32_t sfa_t = tmem_base + C::TMEM_SFA;
            const uint32_t sfb_t = tmem_base + C::TMEM_SFB;
            int local = 0;  // units this pair has computed: selects the accumulator buffer
            for (int ui = 0; ui < work.n && ok; ui++) {
                const PairUnit u = pair_unit<XF>(p, work, cluster_id, num_clusters, ui);
                const TileCoord& tc = u.tc;
                const int b = local & 1;
                const uint32_t d_taddr = tmem_base + (b ? C::BUF1_COL : 0);
                if (!sm100::wait_parity_bounded(acc_empty0 + 8u * b, ((local >> 1) & 1) ^ 1u, abort_flag,
                                                        p.wait_budget) ||
                    (local >= 1 && !sm100::wait_parity_bounded(ovl_free, (local - 1) & 1, abort_flag,
                                                                       p.wait_budget))) {
                    if (!*abort_flag) raise(0x2u);
                    *abort_flag = 1;
                    ok = false;
                    break;
                }
                // A taken-over tile continues the accumulator the epilogue loaded (one per launch)
                if (XF && u.mode == UNIT_TAKE_OVER && !sm100::wait_parity_bounded(fill_bar, 0, abort_flag, p.wait_budget)) {
                    if (!*abort_flag) raise(0x2u);
                    *abort_flag = 1;
                    ok = false;
                    break;
                }
                const uint32_t acc0 = XF && u.mode == UNIT_TAKE_OVER ? 1u : 0u;
                sm100::tc_fence_after();
                // The issuing thread keeps the tensor pipe's short queue fed: it polls the next
                // slab's barrier without blocking right after issuing the current one, and
                // blocks only when that slab's data has not landed yet.
                bool ready = sm100::mbar_test_wait(full_bar(stage), phase);
                for (int i = 0; i < tc.kb_count; i++) {
                    if (!ready && !sm100::wait_parity_bounded(full_bar(stage), phase, abort_flag, p.wait_budget)) {
                        if (!*abort_flag) raise(0x2u);
                        *abort_flag = 1;
                        ok = false;
                        break;
                    }
                    const uint32_t sf_src = sf_base + stage * C::SF_STAGE;
                    // A's atom: one broadcast copy; B's two atoms, staged four times over: one wide copy
                    sm100::tc_cp_32x128b_warpx4_pair(tmem_base + C::TMEM_SFA, sm100::make_sf_desc(sf_src));
                    sm100::tc_cp_128x256b_pair(tmem_base + C::TMEM_SFB, sm100::make_sf_wide_desc(sf_src + C::SFA_BYTES));
                    const uint32_t off16 = (uint32_t)(stage * C::AB_STAGE) >> 4;
#pragma unroll
                    for (int k = 0; k < BK / 32; k++) {
                        const uint32_t sel = (uint32_t)k << 30;
                        sm100::tc_mma_mxf8f6f4_pair(d_taddr, a_desc0 + off16 + 2 * k, b_desc0 + off16 + 2 * k,
                                                    idesc_k[k], sfa_t | sel, sfb_t | sel,
                                                    (acc0 || i > 0 || k > 0) ? 1u : 0u);
                    }
                    mma_issued = true;
                    sm100::tc_commit_pair(empty_bar(stage), 0x3);
                    if (++stage == C::STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                    ready = sm100::mbar_test_wait(full_bar(stage), phase);
                }
                if (!ok) break;
                sm100::tc_commit_pair(acc_full0 + 8u * b, 0x3);
                local++;
            }
        } else if (AMODE == A_CPASYNC && lane == 0) {
            // ---------------- relay (peer only, A_CPASYNC) ----------------
            // The peer's full barrier completes when its loaders' copies have landed; pass each
            // completed phase on to the leader's full barrier of the same stage.
            int stage = 0;
            uint32_t phase = 0;
            bool ok = true;
            for (int ui = 0; ui < work.n && ok; ui++) {
                const TileCoord tc = pair_unit<XF>(p, work, cluster_id, num_clusters, ui).tc;
                for (int i = 0; i < tc.kb_count; i++) {
                    if (!sm100::wait_parity_bounded(full_bar(stage), phase, abort_flag, p.wait_budget)) {
                        if (!*abort_flag) raise(0x1u);
                        *abort_flag = 1;
                        ok = false;
                        break;
                    }
                    sm100::mbar_arrive_cluster(sm100::mapa_shared(full_bar(stage), 0));
                    if (++stage == C::STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            }
        }
    } else if (AMODE == A_CPASYNC && warp >= LOADER_WARP0) {
        // ---------------- A loader (A_CPASYNC, warps 6..9 of both CTAs) ----------------
        // Copies signal this CTA's own full barrier (a cp.async completion can only arrive on a
        // barrier of its own CTA); the peer's relay forwards its barrier to the leader's.
        const int lt = threadIdx.x - 32 * LOADER_WARP0;
        const CompactA a{p.a_ptr, p.a_stride, p.a_valid};
        int stage = 0;
        uint32_t phase = 0;
        bool ok = true;
        for (int ui = 0; ui < work.n && ok; ui++) {
            const TileCoord tc = pair_unit<XF>(p, work, cluster_id, num_clusters, ui).tc;
            const int a_row = tc.mb * C::BM + 128 * (int)rank;
            for (int i = 0; i < tc.kb_count; i++) {
                int got = 1;
                if (lane == 0)
                    got = sm100::wait_parity_bounded(empty_bar(stage), phase ^ 1u, abort_flag, p.wait_budget) ? 1 : 0;
                got = __shfl_sync(0xffffffffu, got, 0);
                if (!got) {
                    if (lane == 0 && !*abort_flag) raise(0x1u);
                    *abort_flag = 1;
                    ok = false;
                    break;
                }
                sm100::mbar_try_wait(empty_bar(stage), phase ^ 1u);
                compact_issue_slab(ab_base + stage * C::AB_STAGE, a, p.M, a_row, tc.kb_begin + i, lt);
                sm100::cp_async_mbar_arrive_noinc(full_bar(stage));
                if (++stage == C::STAGES) {
                    stage = 0;
                    phase ^= 1u;
                }
            }
        }
        sm100::cp_async_wait_all();
    } else {
        // ---------------- epilogue (warps 2..5 of both CTAs) ----------------
        const int quarter = warp & 3;
        const uint32_t t_lane = tmem_base + ((uint32_t)(32 * quarter) << 16);
        const uint32_t leader_acc_empty = sm100::mapa_shared(acc_empty0, 0);
        const uint32_t leader_ovl_free = sm100::mapa_shared(ovl_free, 0);
        const uint32_t leader_fill = sm100::mapa_shared(fill_bar, 0);
        // This thread's row within a 256 x 256 tile (hand-off slots are whole tiles, row-major).
        const int tile_row = 128 * (int)rank + 32 * quarter + lane;
        // Load the previous pair's accumulator for a taken-over tile into buffer `bb` (this CTA's
        // 128 rows), once that pair has released it. The chunk buffer `bb` shares with the other
        // buffer ([224, 256): chunk 7 of buffer 0, chunk 0 of buffer 1) can only be written once
        // the running unit's epilogue has read it, so the load comes in two parts: FILL_REST (every
        // other chunk; waits for the flag), then FILL_SHARED, which also reports to the leader's
        // fill barrier; FILL_ALL does both. Returns false on a timeout (the flag never came).
        constexpr int FILL_REST = 1, FILL_SHARED = 2, FILL_ALL = 3;
        auto take_over = [&](const PairUnit& nu, int bb, int part) -> bool {
            if (part & FILL_REST) {
                int got = 1;
                if (lane == 0) {
                    const unsigned long long* flag = p.sk_flags + 2 * nu.slot + rank;
                    got = sm100::ld_acquire_gpu_u64(flag) == p.sk_epoch ? 1 : 0;
                    const long long t0 = clock64();
                    while (!got && !*abort_flag && clock64() - t0 <= p.wait_budget)
                        got = sm100::ld_acquire_gpu_u64(flag) == p.sk_epoch ? 1 : 0;
                }
                got = __shfl_sync(0xffffffffu, got, 0);
                if (!got) return false;
            }
            const int shared_chunk = bb ? 0 : C::BN / 32 - 1;
            const float* src = p.sk_ws + (size_t)nu.slot * C::SK_TILE_FLOATS + (size_t)tile_row * C::BN;
#pragma unroll 1
            for (int c = 0; c < C::BN / 32; c++) {
                if (!((c == shared_chunk ? FILL_SHARED : FILL_REST) & part)) continue;
                uint32_t r[32];
#pragma unroll
                for (int q = 0; q < 8; q++) {
                    const uint4 v = sm100::ld_cg_v4(src + 32 * c + 4 * q);
                    r[4 * q] = v.x;
                    r[4 * q + 1] = v.y;
                    r[4 * q + 2] = v.z;
                    r[4 * q + 3] = v.w;
                }
                sm100::tmem_st_32x32b_x32(t_lane + (bb ? C::BUF1_COL : 0) + 32 * c, r);
            }
            sm100::tmem_st_wait();
            if (part & FILL_SHARED) {
                sm100::tc_fence_before();
                __syncwarp();
                if (lane == 0) sm100::mbar_arrive_remote(leader_fill);
            }
            return true;
        };
        int local = 0;  // units this pair has computed: selects the accumulator buffer
        for (int ui = 0; ui < work.n; ui++) {
            const PairUnit u = pair_unit<XF>(p, work, cluster_id, num_clusters, ui);
            const TileCoord& tc = u.tc;
            const int b = local & 1;
            // The unit after this one, when it takes over a tile, gets its accumulator loaded into
            // the other buffer: all but the shared chunk now, while this unit's MMAs still run (the
            // other buffer's previous unit is drained), the shared chunk once this unit's epilogue
            // has read it. After a hand-off, the whole load waits until this pair's own flag is out
            // (the next pair may be waiting for it).
            const bool next_takes_over = XF && ui + 1 < work.n &&
                                         pair_unit<XF>(p, work, cluster_id, num_clusters, ui + 1).mode == UNIT_TAKE_OVER;
            const bool hand_off = XF && u.mode == UNIT_HAND_OFF;
            const bool early = next_takes_over && !hand_off;
            if (early && !take_over(pair_unit<XF>(p, work, cluster_id, num_clusters, ui + 1), b ^ 1, FILL_REST)) {
                if (lane == 0 && !*abort_flag) raise(0x4u);
                *abort_flag = 1;
                break;
            }
            if (XF && u.mode == UNIT_TAKE_OVER && local == 0 && !take_over(u, b, FILL_ALL)) {
                if (lane == 0 && !*abort_flag) raise(0x4u);
                *abort_flag = 1;
                break;
            }
            // The tile's set-up comes before the wait: from the accumulator's completion to the
            // release of the shared chunk, the MMA thread waits and the tensor pipe idles.
            const int row = tc.mb * C::BM + tile_row;
            const int col0 = tc.nb * C::BN;
            const bool regroup = XG && !hand_off && p.dst.n > 1;
            // The whole warp waits (a suspended wait takes no issue slots), so it is still converged
            // when the accumulator completes. Measured on B200: 1.7% on cfg2 against one polling
            // lane and a shuffle.
            const int got = __all_sync(0xffffffffu, sm100::wait_parity_bounded(acc_full0 + 8u * b, (local >> 1) & 1,
                                                                               abort_flag, p.wait_budget));
            if (!got) {
                if (lane == 0 && !*abort_flag) raise(0x4u);
                *abort_flag = 1;
                break;
            }
            sm100::tc_fence_after();
            uint32_t pend[16];  // FP16/BF16 with several destinations: first chunk of a 64-column pair
#pragma unroll 1
            for (int j = 0; j < C::BN / 32; j++) {
                // buffer 0 top-down, buffer 1 bottom-up: the shared chunk [224, 256) goes first
                const int c = b ? j : (C::BN / 32 - 1 - j);
                const uint32_t tcol = (b ? C::BUF1_COL : 0) + 32 * c;
                uint32_t r[32];
                sm100::tmem_ld_32x32b_x32(t_lane + tcol, r);
                sm100::tmem_ld_wait(r);
                if (j == 0) {
                    sm100::tc_fence_before();
                    __syncwarp();
                    if (lane == 0) sm100::mbar_arrive_remote(leader_ovl_free);
                    if (early) take_over(pair_unit<XF>(p, work, cluster_id, num_clusters, ui + 1), b ^ 1, FILL_SHARED);
                }
                const int col = col0 + 32 * c;
                if (hand_off) {
                    // the raw FP32 accumulator, whole tile, for the next pair to continue
                    store_words<32>(p.sk_ws + (size_t)u.slot * C::SK_TILE_FLOATS + (size_t)tile_row * C::BN + 32 * c, r,
                                    true);
                } else if (regroup) {
                    // chunks are processed in pairs (c, c ^ 1) in both orders; col < N is uniform
                    if (col < p.N) {
                        uint8_t* stg = epi_stg + quarter * EPI_STG_WARP;
                        const int row0 = row - lane;
                        if constexpr (std::is_same<OutT, float>::value) {
                            store_rows_regrouped<float>(p.dst, stg, row0, p.M, col, r, p.out_align32 != 0);
                        } else {
                            uint32_t w[16];
                            convert_chunk<OutT>(r, w);
                            if ((j & 1) == 0) {
#pragma unroll
                                for (int i = 0; i < 16; i++) pend[i] = w[i];
                            } else {
                                const bool lower_first = (c ^ 1) < c;  // the pending chunk holds the lower columns
                                uint32_t w32[32];
#pragma unroll
                                for (int i = 0; i < 16; i++) {
                                    w32[i] = lower_first ? pend[i] : w[i];
                                    w32[16 + i] = lower_first ? w[i] : pend[i];
                                }
                                store_rows_regrouped<OutT>(p.dst, stg, row0, p.M, col0 + 32 * (c & ~1), w32,
                                                           p.out_align32 != 0);
                            }
                        }
                    }
                } else if (row < p.M && col < p.N) {
                    if constexpr (PARTIAL) {
                        store_words<32>(p.ws + ((size_t)tc.split * p.M + row) * p.N + col, r, p.out_align32 != 0);
                    } else {
                        uint32_t w[ChunkWords<OutT>::N];
                        convert_chunk<OutT>(r, w);
                        store_chunk_all<OutT>(p.dst, row, col, w, p.out_align32 != 0);
                    }
                }
            }
            if (hand_off) {
                // Release the hand-off: every warp's stores, then one flag per CTA (128 rows) at
                // GPU scope for the next pair to acquire.
                __threadfence();
                __syncwarp();
                if (lane == 0) sm100::mbar_arrive(handed_bar);
                if (warp == 2 && lane == 0) {
                    if (sm100::wait_parity_bounded(handed_bar, 0, abort_flag, p.wait_budget)) {
                        __threadfence();
                        sm100::st_release_gpu_u64(p.sk_flags + 2 * u.slot + rank, p.sk_epoch);
                    } else if (!*abort_flag) {
                        raise(0x4u);
                    }
                }
                __syncwarp();
                if (next_takes_over && !take_over(pair_unit<XF>(p, work, cluster_id, num_clusters, ui + 1), b ^ 1, FILL_ALL)) {
                    if (lane == 0 && !*abort_flag) raise(0x4u);
                    *abort_flag = 1;
                    break;
                }
            }
            sm100::tc_fence_before();
            __syncwarp();
            if (lane == 0) sm100::mbar_arrive_remote(leader_acc_empty + 8u * b);
            local++;
        }
    }

    sm100::tc_fence_before();
    // After a timeout anywhere in the pair, wait out everything still in flight before shared and
    // tensor memory are released (any role may have given up while another finished normally):
    // the leader's MMAs and scale copies, and the loads no MMA consumed. The leader's full
    // barriers count both CTAs' bytes; the peer, whose loads report there, gives its own loads
    // a bounded settle time. A role that leaves its loop on a timeout, its own or one it saw in
    // the flag, sets this CTA's flag before the barrier above; without a timeout the epilogue has
    // waited for every tile, so nothing is in flight. The peer may still set this CTA's flag
    // remotely: the barrier ORs every thread's view of it, so the whole CTA takes the same branch.
    const int aborted = __syncthreads_or(*abort_flag != 0);
    if (aborted) {
        const int zero = 0;
        if (warp == 0 && lane == 0) {
            if (rank == 0 && !COMPACT) {
                for (int s = 0; s < C::STAGES; s++)
                    if ((issued_mask >> s) & 1u)
                        if (!sm100::wait_parity_bounded(full_bar(s), (issued_phase >> s) & 1u, &zero,
                                                        WAIT_BUDGET / 4))
                            atomicOr(&g_device_status, 0x8u);
            } else {
                sm100::settle_ns(200000);
            }
        }
        if (warp == 1 && lane == 0 && rank == 0 && mma_issued) {
            sm100::tc_commit_pair(drain_bar, 0x1);
            if (!sm100::wait_parity_bounded(drain_bar, 0, &zero, WAIT_BUDGET / 4)) atomicOr(&g_device_status, 0x8u);
        }
        sm100::tc_fence_before();
        __syncthreads();
    }
    sm100::cluster_sync();  // no CTA leaves while its peer may still touch its shared memory
    if (warp == 1) {
        __syncwarp();
        sm100::tc_fence_after();
        sm100::tmem_dealloc_pair(tmem_base, C::TMEM_COLS);
    }
}

}  // namespace kern
}  // namespace mxfp6
