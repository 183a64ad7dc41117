#pragma once
// The B200 MXFP6 GEMM kernel: persistent, warp-specialised, block-scaled tcgen05 MMA.
//
// Replaces the reference's lds_gemm_hybrid_dripA (reference: src/kernel.hpp:73-300) and, in
// partial mode, its split-K first stage; reduce_splitk (reference: src/kernel.hpp:305-313) is
// reduce_partials() below. The math is the same: for every output element
//   D[m][n] = sum over K-blocks b of 2^(sa[m][b]-127) * 2^(sb[n][b]-127) * sum_k a[m][k] * b[n][k]
// accumulated in FP32 and converted once to the output type; the schedule is B200's:
//
//   warp 0 (one lane)  TMA producer: per 128-wide K slab, one 2-D tensor load of A (128 rows)
//                      and of B^T (BN rows) in the 16U6 unpack mode (packed FP6 in HBM -> one
//                      byte per code in shared memory, 128-byte swizzle), plus untiled bulk
//                      loads of the 512-byte scale atoms, into a STAGES-deep mbarrier ring.
//   warp 1 (one lane)  MMA issuer: tcgen05.cp of the scale atoms into tensor memory, then four
//                      tcgen05.mma.kind::mxf8f6f4.block_scale (K = 32 each) per slab into an
//                      FP32 accumulator of 128 lanes x BN columns in tensor memory; tcgen05.commit
//                      returns the ring slot and, after the last slab, hands the tile to:
//   warps 2..5         epilogue: tcgen05.ld 32 columns at a time (warp w owns lanes 32*(w%4)..),
//                      convert to FP32 / FP16 / BF16 (round to nearest even) and store; in
//                      partial mode store FP32 partial sums into the split-K workspace.
//
// Tiles (128 x BN output blocks, times the split-K factor) are handed out round-robin over a
// persistent grid of at most one CTA per SM, in groups of GROUP_M row-blocks for L2 reuse.
// Every wait is bounded; a timeout sets a bit in the device status word, makes the other roles
// leave their loops, lets in-flight copies and MMAs settle (again bounded) and frees tensor
// memory before the CTA exits.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <type_traits>

#include "compact_a.cuh"
#include "sm100_ptx.cuh"

namespace mxfp6 {

// Sticky status bits written by kernels (MXFP6_DEV_* in mxfp6_gemm.h). This header is compiled
// into exactly one translation unit (gemm.cu), which owns the definition.
__device__ unsigned int g_device_status = 0;

namespace kern {

constexpr int BM = 128;             // output rows per tile (tensor-memory lanes)
constexpr int BK = 128;             // K elements per pipeline slab
// Row-blocks per rasterisation group. At 8192^3 with 256-row tiles, 16 means two groups, so B^T
// streams from DRAM twice per launch: 164 MB read against 258 MB with 8. The speed is the same.
constexpr int GROUP_M = 16;
constexpr int NUM_THREADS = 192;    // 6 warps
constexpr int EPI_WARP0 = 2;        // first epilogue warp
constexpr int A_TMA_BYTES = BM * BK * 3 / 4;  // packed bytes one A slab moves
// Default cycle budget of a bounded wait (about 2 s at 1.9 GHz); Params::wait_budget carries
// the one a launch uses. Drains after a timeout always use WAIT_BUDGET / 4.
constexpr long long WAIT_BUDGET = 4000000000LL;

template <int BN, int AMODE = A_TMA>
struct Config {
    static_assert(BN == 128 || BN == 256, "tile width");
    static constexpr int STAGES = BN == 256 ? 4 : 6;
    static constexpr int A_BYTES = BM * BK;  // one byte per code in shared memory
    static constexpr int B_BYTES = BN * BK;
    static constexpr int AB_STAGE = A_BYTES + B_BYTES;
    static constexpr int SFA_BYTES = 512;
    static constexpr int SFB_ATOMS = BN / 128;
    static constexpr int SF_STAGE = SFA_BYTES + SFB_ATOMS * 512;
    static constexpr int B_TMA_BYTES = BN * BK * 3 / 4;
    // tensor-memory columns: accumulator [0,BN), A scales [BN, BN+4), B scales after them
    static constexpr int TMEM_SFA = BN;
    static constexpr int TMEM_SFB = BN + 4;
    static constexpr int TMEM_COLS = BN == 256 ? 512 : 256;
    static constexpr int BAR_BYTES = 256;
    static constexpr int SMEM_BYTES = 1024 + STAGES * (AB_STAGE + SF_STAGE) + BAR_BYTES;
    static_assert(SMEM_BYTES <= 227 * 1024, "shared memory budget");
};

// Output destinations: D is written into each of n row-major [M][ldd] matrices at column col0
// (one destination, ldd = N, col0 = 0 for a plain GEMM; several for a GEMM whose epilogue also
// delivers its column shard into peers' gathered outputs).
constexpr int MAX_DST = 8;
struct DstList {
    void* p[MAX_DST];
    int n;
    int col0;
    long long ldd;
};

struct Params {
    const uint8_t* sfA;  // A scales, atom layout
    const uint8_t* sfB;  // B scales, atom layout
    DstList dst;         // outputs (OutT); unused in partial mode
    float* ws;           // FP32 partials [splits][M][N] in partial mode
    int M, N, Kp;
    int m_blocks, n_blocks, k_slabs, splits;
    int out_align32;  // every output row chunk (or ws in partial mode) is 32-byte aligned: 256-bit stores
    // compact A (software producer, compact_a.cuh): packed rows, stride and valid bytes per row
    const uint8_t* a_ptr;
    int a_stride, a_valid;
    long long wait_budget;  // cycles a role waits on a barrier before it gives up (WAIT_BUDGET by default)
    // Pair kernel only, stream-K tail (gemm_kernel_pair.cuh): tiles [0, sk_first) go to the pairs
    // round-robin as whole tiles; the K slabs of tiles [sk_first, tiles), sk_total in all, are cut
    // into one contiguous range per pair. sk_total == 0: no stream-K. A pair that ends inside a
    // tile hands its FP32 accumulator to the next pair through sk_ws ([pairs][256][256]) and
    // sk_flags ([pairs][2]: set to sk_epoch when a CTA's 128 rows are written).
    int sk_first;
    long long sk_total;
    float* sk_ws;
    unsigned long long* sk_flags;
    unsigned long long sk_epoch;
    // Pair kernel, partial mode, banded split (band_L > 0): the first band_L * tiles pairs each
    // take one long band [l * band_a, (l + 1) * band_a) of one tile (partial l); the other pairs
    // take the band_n short bands that cut [band_L * band_a, k_slabs) evenly, round-robin, band
    // by band (partial band_L + j).
    int band_L, band_a, band_n;
};

struct TileCoord {
    int mb, nb, split, kb_begin, kb_count;
};

__device__ __forceinline__ TileCoord decode_tile(int t, const Params& p) {
    const int tiles_mn = p.m_blocks * p.n_blocks;
    TileCoord c;
    c.split = t / tiles_mn;
    const int mn = t - c.split * tiles_mn;
    const int group_tiles = GROUP_M * p.n_blocks;
    const int g = mn / group_tiles;
    const int first_m = g * GROUP_M;
    const int gm = min(p.m_blocks - first_m, GROUP_M);
    const int within = mn - g * group_tiles;
    c.mb = first_m + within % gm;
    c.nb = within / gm;
    const int per = p.k_slabs / p.splits, rem = p.k_slabs % p.splits;
    c.kb_begin = c.split * per + min(c.split, rem);
    c.kb_count = per + (c.split < rem ? 1 : 0);
    return c;
}

__device__ __forceinline__ void raise_status(unsigned int bit, volatile int* abort_flag) {
    atomicOr(&g_device_status, bit);
    *abort_flag = 1;
}

// 32 consecutive outputs of one row from 32 FP32 accumulator words. With a 32-byte aligned
// destination the stores are 256-bit (full L2 sectors), otherwise 128-bit.
__device__ __forceinline__ void st_v8(void* dst, const uint32_t* w) {
    asm volatile("st.global.v8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"l"(dst), "r"(w[0]), "r"(w[1]), "r"(w[2]),
                 "r"(w[3]), "r"(w[4]), "r"(w[5]), "r"(w[6]), "r"(w[7])
                 : "memory");
}

template <int NWORDS>
__device__ __forceinline__ void store_words(void* dst, const uint32_t* w, bool align32) {
    if (align32) {
#pragma unroll
        for (int i = 0; i < NWORDS / 8; i++) st_v8(static_cast<uint8_t*>(dst) + 32 * i, w + 8 * i);
    } else {
        uint4* d = reinterpret_cast<uint4*>(dst);
#pragma unroll
        for (int i = 0; i < NWORDS / 4; i++) d[i] = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
    }
}

// 32 FP32 accumulator words of one row -> OutT words (RNE): 32 words for float, 16 for half
// and bfloat16 (two values per word).
template <typename OutT>
struct ChunkWords {
    static constexpr int N = std::is_same<OutT, float>::value ? 32 : 16;
};

template <typename OutT>
__device__ __forceinline__ void convert_chunk(const uint32_t (&r)[32], uint32_t (&w)[ChunkWords<OutT>::N]) {
    if constexpr (std::is_same<OutT, float>::value) {
#pragma unroll
        for (int i = 0; i < 32; i++) w[i] = r[i];
    } else if constexpr (std::is_same<OutT, __half>::value) {
#pragma unroll
        for (int i = 0; i < 16; i++) {
            __half2 v = __floats2half2_rn(__uint_as_float(r[2 * i]), __uint_as_float(r[2 * i + 1]));
            w[i] = *reinterpret_cast<uint32_t*>(&v);
        }
    } else {
#pragma unroll
        for (int i = 0; i < 16; i++) {
            __nv_bfloat162 v = __floats2bfloat162_rn(__uint_as_float(r[2 * i]), __uint_as_float(r[2 * i + 1]));
            w[i] = *reinterpret_cast<uint32_t*>(&v);
        }
    }
}

// Store one converted row chunk (32 columns starting at `col` of output row `row`) into every
// destination of the list.
template <typename OutT>
__device__ __forceinline__ void store_chunk_all(const DstList& dl, int row, int col,
                                                const uint32_t (&w)[ChunkWords<OutT>::N], bool align32) {
    for (int d = 0; d < dl.n; d++)
        store_words<ChunkWords<OutT>::N>(static_cast<OutT*>(dl.p[d]) + (size_t)row * dl.ldd + dl.col0 + col, w,
                                        align32);
}

// Output staging for several destinations (the fused gather): per epilogue warp a [32 rows] x
// [128 + 16 bytes] shared-memory area, the 16 padding bytes spreading a warp's row writes over
// all banks.
constexpr int EPI_STG_PITCH = 144;
constexpr int EPI_STG_WARP = 32 * EPI_STG_PITCH;
constexpr int EPI_STG_BYTES = 4 * EPI_STG_WARP;

// Multi-destination store of 128 bytes per row: lane l holds 32 words of row row0 + l starting
// at column `col` (32 FP32 or 64 FP16/BF16 columns). The warp regroups them through its staging
// area so that in each store instruction four lanes write one row's 128 bytes as consecutive
// 32-byte pieces: every destination, local or a peer's over NVLink, receives 128-byte runs
// instead of one 32-byte piece per row and instruction. Rows at or past M are skipped.
template <typename OutT>
__device__ __forceinline__ void store_rows_regrouped(const DstList& dl, uint8_t* stg, int row0, int M, int col,
                                                     const uint32_t (&w)[32], bool align32) {
    const int lane = threadIdx.x & 31;
    uint4* mine = reinterpret_cast<uint4*>(stg + lane * EPI_STG_PITCH);
#pragma unroll
    for (int i = 0; i < 8; i++) mine[i] = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
    __syncwarp();
    const int k = lane >> 2, j = lane & 3;
    constexpr int COLS_PER_32B = 32 / (int)sizeof(OutT);
#pragma unroll
    for (int q = 0; q < 4; q++) {
        const int r = 8 * q + k;
        const uint4* src = reinterpret_cast<const uint4*>(stg + r * EPI_STG_PITCH + 32 * j);
        const uint4 a = src[0], b = src[1];
        const uint32_t v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
        const int row = row0 + r;
        if (row < M)
            for (int d = 0; d < dl.n; d++)
                store_words<8>(static_cast<OutT*>(dl.p[d]) + (size_t)row * dl.ldd + dl.col0 + col + COLS_PER_32B * j,
                               v, align32);
    }
    __syncwarp();  // the staging area is rewritten by the next group
}

// OutT: float / __half / __nv_bfloat16. PARTIAL: write FP32 partial sums to p.ws instead of D.
// AMODE (compact_a.cuh): A_TMA loads A with the 16U6 tensor load; A_CPASYNC adds four
// loader warps that copy the A image from p.a_ptr (tmA unused).
template <int BN, typename OutT, bool PARTIAL, int AMODE = A_TMA>
__global__ void __launch_bounds__(threads_for(AMODE), 1)
    gemm_mxfp6_sm100(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const Params p) {
    using C = Config<BN, AMODE>;
    constexpr bool COMPACT = AMODE != A_TMA;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    // 1024-byte alignment for the 128-byte-swizzled operand tiles.
    const uint32_t raw_u32 = sm100::smem_u32(smem_raw);
    const uint32_t base = (raw_u32 + 1023u) & ~1023u;
    uint8_t* base_ptr = smem_raw + (base - raw_u32);

    const uint32_t ab_base = base;                                   // STAGES x (A | B)
    const uint32_t sf_base = base + C::STAGES * C::AB_STAGE;         // STAGES x (sfA | sfB)
    const uint32_t bar_base = sf_base + C::STAGES * C::SF_STAGE;     // barriers
    uint8_t* bar_ptr = base_ptr + (bar_base - base);
    // barrier map (8 bytes each): full[S], empty[S], acc_full, acc_empty, drain
    auto full_bar = [&](int s) { return bar_base + 8u * s; };
    auto empty_bar = [&](int s) { return bar_base + 8u * (C::STAGES + s); };
    const uint32_t acc_full = bar_base + 8u * (2 * C::STAGES);
    const uint32_t acc_empty = acc_full + 8u;
    const uint32_t drain_bar = acc_full + 16u;
    const int slot_off = 8 * (2 * C::STAGES + 3);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar_ptr + slot_off);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(bar_ptr + slot_off + 8);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < C::STAGES; s++) {
            // producer, plus one arrival per loader thread (A_CPASYNC)
            sm100::mbar_init(full_bar(s), AMODE == A_CPASYNC ? 1 + LOADER_THREADS : 1);
            sm100::mbar_init(empty_bar(s), 1);
        }
        sm100::mbar_init(acc_full, 1);
        sm100::mbar_init(acc_empty, 4 * 32);
        sm100::mbar_init(drain_bar, 1);
        *abort_flag = 0;
        sm100::fence_mbar_init();
        sm100::fence_async_shared();
        if (AMODE == A_TMA) sm100::prefetch_tmap(&tmA);
        sm100::prefetch_tmap(&tmB);
    }

    if (warp == 1) {
        sm100::tmem_alloc(sm100::smem_u32(tmem_slot), C::TMEM_COLS);
        sm100::tmem_relinquish();
    }
    sm100::tc_fence_before();
    __syncthreads();
    sm100::tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    // Set-up done (it reads only kernel parameters): the next kernel may start its own, and this
    // one waits for the previous kernel's memory before its first global access.
    sm100::griddep_launch_dependents();
    sm100::griddep_wait();

    const int total_tiles = p.m_blocks * p.n_blocks * p.splits;
    // Abort bookkeeping, read after the roles have finished (see the end of the kernel): the
    // producer's last load per stage and its phase parity, and whether any MMA was issued.
    uint32_t issued_mask = 0, issued_phase = 0;
    bool mma_issued = false;

    if (warp == 0) {
        if (lane == 0) {
            // ---------------- TMA producer ----------------
            int stage = 0;
            uint32_t phase = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < total_tiles && ok; t += gridDim.x) {
                const TileCoord tc = decode_tile(t, p);
                int sfb_atoms = 0;
#pragma unroll
                for (int j = 0; j < C::SFB_ATOMS; j++)
                    if (tc.nb * BN + j * 128 < p.N) sfb_atoms++;
                const uint32_t tx = (COMPACT ? 0u : (uint32_t)A_TMA_BYTES) + C::B_TMA_BYTES + 512u * (1 + sfb_atoms);
                for (int i = 0; i < tc.kb_count; i++) {
                    if (!sm100::wait_parity_bounded(empty_bar(stage), phase ^ 1u, abort_flag, p.wait_budget)) {
                        if (!*abort_flag) raise_status(0x1u, abort_flag);
                        ok = false;
                        break;
                    }
                    const int kb = tc.kb_begin + i;
                    const uint32_t fb = full_bar(stage);
                    sm100::mbar_arrive_expect_tx(fb, tx);
                    const uint32_t a_dst = ab_base + stage * C::AB_STAGE;
                    if (!COMPACT) sm100::tma_load_2d(a_dst, &tmA, fb, kb * BK, tc.mb * BM);
                    sm100::tma_load_2d(a_dst + C::A_BYTES, &tmB, fb, kb * BK, tc.nb * BN);
                    const uint32_t sf_dst = sf_base + stage * C::SF_STAGE;
                    sm100::bulk_load(sf_dst, p.sfA + ((size_t)tc.mb * p.k_slabs + kb) * 512, 512, fb);
                    for (int j = 0; j < sfb_atoms; j++)
                        sm100::bulk_load(
                            sf_dst + 512 + 512 * j,
                            p.sfB + ((size_t)(tc.nb * C::SFB_ATOMS + j) * p.k_slabs + kb) * 512, 512, fb);
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
        if (lane == 0) {
            // ---------------- MMA issuer ----------------
            constexpr uint32_t idesc = sm100::make_idesc_e2m3(BM, BN);
            int stage = 0;
            uint32_t phase = 0, acc_phase = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < total_tiles && ok; t += gridDim.x) {
                const TileCoord tc = decode_tile(t, p);
                if (!sm100::wait_parity_bounded(acc_empty, acc_phase ^ 1u, abort_flag, p.wait_budget)) {
                    if (!*abort_flag) raise_status(0x2u, abort_flag);
                    ok = false;
                    break;
                }
                sm100::tc_fence_after();
                for (int i = 0; i < tc.kb_count; i++) {
                    if (!sm100::wait_parity_bounded(full_bar(stage), phase, abort_flag, p.wait_budget)) {
                        if (!*abort_flag) raise_status(0x2u, abort_flag);
                        ok = false;
                        break;
                    }
                    sm100::tc_fence_after();
                    const uint32_t sf_src = sf_base + stage * C::SF_STAGE;
                    sm100::tc_cp_32x128b_warpx4(tmem_base + C::TMEM_SFA, sm100::make_sf_desc(sf_src));
#pragma unroll
                    for (int j = 0; j < C::SFB_ATOMS; j++)
                        sm100::tc_cp_32x128b_warpx4(tmem_base + C::TMEM_SFB + 4 * j,
                                                    sm100::make_sf_desc(sf_src + 512 + 512 * j));
                    const uint32_t a_src = ab_base + stage * C::AB_STAGE;
                    const uint32_t b_src = a_src + C::A_BYTES;
#pragma unroll
                    for (int k = 0; k < BK / 32; k++) {
                        const uint64_t adesc = sm100::make_kmajor_sw128_desc(a_src + 32 * k);
                        const uint64_t bdesc = sm100::make_kmajor_sw128_desc(b_src + 32 * k);
                        const uint32_t sel = (uint32_t)k << 30;
                        sm100::tc_mma_mxf8f6f4(tmem_base, adesc, bdesc,
                                               sm100::idesc_with_sf_ids(idesc, k, k),
                                               (tmem_base + C::TMEM_SFA) | sel,
                                               (tmem_base + C::TMEM_SFB) | sel, (i > 0 || k > 0) ? 1u : 0u);
                    }
                    mma_issued = true;
                    sm100::tc_commit(empty_bar(stage));
                    if (++stage == C::STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
                if (!ok) break;
                sm100::tc_commit(acc_full);
                acc_phase ^= 1u;
            }
        }
    } else if (AMODE == A_CPASYNC && warp >= LOADER_WARP0) {
        // ---------------- A loader (A_CPASYNC, warps 6..9) ----------------
        const int lt = threadIdx.x - 32 * LOADER_WARP0;
        const CompactA a{p.a_ptr, p.a_stride, p.a_valid};
        int stage = 0;
        uint32_t phase = 0;
        bool ok = true;
        for (int t = blockIdx.x; t < total_tiles && ok; t += gridDim.x) {
            const TileCoord tc = decode_tile(t, p);
            for (int i = 0; i < tc.kb_count; i++) {
                int got = 1;
                if (lane == 0)
                    got = sm100::wait_parity_bounded(empty_bar(stage), phase ^ 1u, abort_flag, p.wait_budget) ? 1 : 0;
                got = __shfl_sync(0xffffffffu, got, 0);
                if (!got) {
                    if (lane == 0 && !*abort_flag) raise_status(0x1u, abort_flag);
                    ok = false;
                    break;
                }
                sm100::mbar_try_wait(empty_bar(stage), phase ^ 1u);
                compact_issue_slab(ab_base + stage * C::AB_STAGE, a, p.M, tc.mb * BM, tc.kb_begin + i, lt);
                sm100::cp_async_mbar_arrive_noinc(full_bar(stage));
                if (++stage == C::STAGES) {
                    stage = 0;
                    phase ^= 1u;
                }
            }
        }
        sm100::cp_async_wait_all();
    } else {
        // ---------------- epilogue (warps 2..5) ----------------
        const int quarter = warp & 3;  // tensor-memory lanes 32*quarter .. 32*quarter+31
        const uint32_t t_row = tmem_base + ((uint32_t)(32 * quarter) << 16);
        uint32_t acc_phase = 0;
        for (int t = blockIdx.x; t < total_tiles; t += gridDim.x) {
            const TileCoord tc = decode_tile(t, p);
            if (!sm100::wait_parity_bounded(acc_full, acc_phase, abort_flag, p.wait_budget)) {
                if (!*abort_flag) raise_status(0x4u, abort_flag);
                break;
            }
            sm100::tc_fence_after();
            const int row = tc.mb * BM + 32 * quarter + lane;
            const int col0 = tc.nb * BN;
#pragma unroll 1
            for (int c = 0; c < BN; c += 32) {
                if (col0 + c >= p.N) break;  // masked half tile (uniform across the warp)
                uint32_t r[32];
                sm100::tmem_ld_32x32b_x32(t_row + (uint32_t)c, r);
                sm100::tmem_ld_wait(r);
                if (row < p.M) {
                    if constexpr (PARTIAL) {
                        float* dst = p.ws + ((size_t)tc.split * p.M + row) * p.N + col0 + c;
                        store_words<32>(dst, r, p.out_align32 != 0);
                    } else {
                        uint32_t w[ChunkWords<OutT>::N];
                        convert_chunk<OutT>(r, w);
                        store_chunk_all<OutT>(p.dst, row, col0 + c, w, p.out_align32 != 0);
                    }
                }
            }
            sm100::tc_fence_before();
            sm100::mbar_arrive(acc_empty);
            acc_phase ^= 1u;
        }
    }

    sm100::tc_fence_before();
    // After a timeout anywhere in the CTA (any role may have given up while another finished
    // normally), wait out everything still in flight before shared and tensor memory are
    // released: the producer's loads that no MMA consumed, and every MMA and scale copy issued.
    // Without an abort the epilogue has waited for every tile, so nothing is in flight. The barrier
    // ORs every thread's view of the flag, so the whole CTA takes the same branch.
    const int aborted = __syncthreads_or(*abort_flag != 0);
    if (aborted) {
        const int zero = 0;
        if (warp == 0 && lane == 0) {
            if (COMPACT) {
                // The full barriers also count loader arrivals that may never come: give the
                // tensor loads in flight time to land instead.
                sm100::settle_ns(200000);
            } else {
                for (int s = 0; s < C::STAGES; s++)
                    if ((issued_mask >> s) & 1u)
                        if (!sm100::wait_parity_bounded(full_bar(s), (issued_phase >> s) & 1u, &zero,
                                                        WAIT_BUDGET / 4))
                            atomicOr(&g_device_status, 0x8u);
            }
        }
        if (warp == 1 && lane == 0 && mma_issued) {
            sm100::tc_commit(drain_bar);
            if (!sm100::wait_parity_bounded(drain_bar, 0, &zero, WAIT_BUDGET / 4)) atomicOr(&g_device_status, 0x8u);
        }
        sm100::tc_fence_before();
        __syncthreads();
    }
    if (warp == 1) {
        __syncwarp();
        sm100::tc_fence_after();
        sm100::tmem_dealloc(tmem_base, C::TMEM_COLS);
    }
}

// Split-K second stage (reference: src/kernel.hpp:305-313): D = sum_{s=0..S-1} ws[s], in that
// fixed order, converted once and written to every destination of the list. Four elements per
// thread per step (N % 4 == 0, so the four stay in one row).
template <typename OutT>
__global__ void __launch_bounds__(256) reduce_partials(const float* __restrict__ ws, const DstList dl, int N,
                                                       long long total, int S) {
    sm100::griddep_launch_dependents();
    sm100::griddep_wait();  // the partials of the GEMM before it
    const long long n4 = total / 4;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n4;
         i += (long long)gridDim.x * blockDim.x) {
        float4 acc = reinterpret_cast<const float4*>(ws)[i];
        for (int s = 1; s < S; s++) {
            const float4 v = reinterpret_cast<const float4*>(ws + (size_t)s * total)[i];
            acc.x += v.x;
            acc.y += v.y;
            acc.z += v.z;
            acc.w += v.w;
        }
        const long long e = 4 * i;
        const long long row = e / N;
        const int col = (int)(e - row * N);
        const size_t off = (size_t)row * dl.ldd + dl.col0 + col;
        if constexpr (std::is_same<OutT, float>::value) {
            for (int d = 0; d < dl.n; d++) *reinterpret_cast<float4*>(static_cast<float*>(dl.p[d]) + off) = acc;
        } else if constexpr (std::is_same<OutT, __half>::value) {
            __half2 lo = __floats2half2_rn(acc.x, acc.y), hi = __floats2half2_rn(acc.z, acc.w);
            const uint2 o = make_uint2(*reinterpret_cast<uint32_t*>(&lo), *reinterpret_cast<uint32_t*>(&hi));
            for (int d = 0; d < dl.n; d++) *reinterpret_cast<uint2*>(static_cast<__half*>(dl.p[d]) + off) = o;
        } else {
            __nv_bfloat162 lo = __floats2bfloat162_rn(acc.x, acc.y), hi = __floats2bfloat162_rn(acc.z, acc.w);
            const uint2 o = make_uint2(*reinterpret_cast<uint32_t*>(&lo), *reinterpret_cast<uint32_t*>(&hi));
            for (int d = 0; d < dl.n; d++)
                *reinterpret_cast<uint2*>(static_cast<__nv_bfloat16*>(dl.p[d]) + off) = o;
        }
    }
}

}  // namespace kern
}  // namespace mxfp6
