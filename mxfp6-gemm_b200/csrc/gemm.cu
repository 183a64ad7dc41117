// libmxfp6gemm host side: validation, routing, tensor-map construction and launches.
//
// Counterparts in the reference (paths within eeezio/mxfp6-gemm):
//   mxfp6::gemm / gemm_workspace_size / choose_tile   src/gemm.cpp:12-83
//   detail::splitk_S / dispatch_gemm                  src/dispatch.hpp:30-187
//   gemm_force_tile (test hook)                       src/gemm.cpp:89-107
// The reference routes over four gfx950 tiles with a 256-CU wave table; this file routes over
// the B200 kernel's two tile widths with a wave-count cost model on the device's SM count.
#include <cuda.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <random>

#include "gemm_kernel.cuh"
#include "gemm_kernel_pair.cuh"
#include "mxfp6/gemm.hpp"
#include "mxfp6_gemm.h"
#include "route.hpp"

namespace mxfp6 {

cudaError_t launch_repad(const uint8_t* src, int rows, int src_row_bytes, int bytes_used, uint8_t* dst,
                         int dst_row_bytes, cudaStream_t stream);  // quantize.cu
void note_launch();

namespace {

thread_local int t_last_error = MXFP6_OK;
thread_local long long t_wait_budget = 0;  // 0: the kernels' default (kern::WAIT_BUDGET)
std::atomic<uint64_t> g_launches{0};

// Tag of one stream-K launch, written into the workspace's hand-off flags: the flags are never
// cleared, so a flag counts only when it holds this launch's tag. The high half is drawn once per
// process, so stale flags from another process's use of the same memory do not match either.
uint64_t next_sk_epoch() {
    static std::atomic<uint64_t> counter{((uint64_t)std::random_device{}() << 32) | 1u};
    return counter.fetch_add(1, std::memory_order_relaxed);
}

long long wait_budget() {
    return t_wait_budget > 0 ? t_wait_budget : kern::WAIT_BUDGET;
}

void set_error(int code, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
void set_error(int code, const char* fmt, ...) {
    t_last_error = code;
    va_list ap;
    va_start(ap, fmt);
    std::fprintf(stderr, "[mxfp6] ");
    std::vfprintf(stderr, fmt, ap);
    std::fprintf(stderr, "\n");
    va_end(ap);
}

// ---- device properties ------------------------------------------------------------------------

constexpr int kMaxDevices = 64;
int g_sm_count[kMaxDevices];
std::once_flag g_sm_once[kMaxDevices];

int current_device() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return -1;
    return dev;
}

// SM count of the current device; 148 (B200) when no device is visible, so host-only queries
// (choose_tile, gemm_workspace_size) stay answerable on a machine without a GPU.
int sm_count() {
    int dev = current_device();
    if (dev < 0 || dev >= kMaxDevices) {
        cudaGetLastError();
        return 148;
    }
    std::call_once(g_sm_once[dev], [dev] {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
            n = 148;
        g_sm_count[dev] = n;
    });
    return g_sm_count[dev];
}

// ---- tensor maps ---------------------------------------------------------------------------------

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            p = nullptr;
        return reinterpret_cast<EncodeTiledFn>(p);
    }();
    return fn;
}

// Tensor maps depend only on their encode arguments, so each host thread keeps its last few:
// a caller that repeats a call (same buffers, same shape) skips the driver's encode. The key holds
// every argument that varies; the rest of each encode is fixed per map kind.
struct TmapKey {
    int kind;  // 0: FP6 operand, 1: scale atoms, 2: scale atoms read four times (pair B)
    int v[4];
    const void* ptr;
    bool operator==(const TmapKey& o) const {
        return kind == o.kind && ptr == o.ptr && v[0] == o.v[0] && v[1] == o.v[1] && v[2] == o.v[2] &&
               v[3] == o.v[3];
    }
};
struct TmapCache {
    static constexpr int kEntries = 16;
    TmapKey key[kEntries];
    CUtensorMap map[kEntries];
    int used = 0, next = 0;
    const CUtensorMap* find(const TmapKey& k) const {
        for (int i = 0; i < used; i++)
            if (key[i] == k) return &map[i];
        return nullptr;
    }
    void put(const TmapKey& k, const CUtensorMap& m) {
        key[next] = k;
        map[next] = m;
        next = (next + 1) % kEntries;
        if (used < kEntries) used++;
    }
};
thread_local TmapCache t_tmaps;
thread_local int t_encode_status;  // CUresult of this thread's last failed encode (-1: no driver entry)

// Driver calls (tensor-map encodes, address-range queries) need a current context. The runtime
// binds its primary context to a host thread lazily, so a thread whose first CUDA work is such a
// call (its streams and buffers made elsewhere) has none yet: bind the current device's primary
// context and retry once.
template <typename F>
CUresult driver_call_in_context(F&& call) {
    CUresult r = call();
    if (r == CUDA_ERROR_INVALID_CONTEXT) {
        int dev = 0;
        if (cudaGetDevice(&dev) == cudaSuccess && cudaSetDevice(dev) == cudaSuccess) r = call();
    }
    return r;
}

// Packed FP6 matrix [rows][Kp] with row_bytes stride, read in 128 (K) x box_rows boxes through
// the 16U6 unpack mode with 128-byte swizzle.
bool make_fp6_tmap(CUtensorMap* map, const void* ptr, int rows, int Kp, int row_bytes, int box_rows) {
    const TmapKey k{0, {rows, Kp, row_bytes, box_rows}, ptr};
    if (const CUtensorMap* hit = t_tmaps.find(k)) {
        *map = *hit;
        return true;
    }
    EncodeTiledFn fn = encode_fn();
    if (!fn) {
        t_encode_status = -1;
        return false;
    }
    cuuint64_t dims[2] = {(cuuint64_t)Kp, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)row_bytes};
    cuuint32_t box[2] = {128u, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1u, 1u};
    const CUresult r = driver_call_in_context([&] {
        return fn(map, CU_TENSOR_MAP_DATA_TYPE_16U6_ALIGN16B, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    });
    if (r != CUDA_SUCCESS) {
        t_encode_status = (int)r;
        return false;
    }
    t_tmaps.put(k, *map);
    return true;
}

// Tiled scales viewed as [row_atoms][k_slabs][128 x u32] (512-byte atoms), read one or two
// atoms at a time; atoms past the last row block read as zero.
bool make_sf_tmap(CUtensorMap* map, const void* ptr, int rows, int Kp, int box_atoms, int box_slabs = 1) {
    const TmapKey k{1, {rows, Kp, box_atoms, box_slabs}, ptr};
    if (const CUtensorMap* hit = t_tmaps.find(k)) {
        *map = *hit;
        return true;
    }
    EncodeTiledFn fn = encode_fn();
    if (!fn) {
        t_encode_status = -1;
        return false;
    }
    const int k_slabs = Kp / 128, atoms = (rows + 127) / 128;
    cuuint64_t dims[3] = {128u, (cuuint64_t)k_slabs, (cuuint64_t)atoms};
    cuuint64_t strides[2] = {512u, (cuuint64_t)k_slabs * 512u};
    cuuint32_t box[3] = {128u, (cuuint32_t)box_slabs, (cuuint32_t)box_atoms};
    cuuint32_t estr[3] = {1u, 1u, 1u};
    const CUresult r = driver_call_in_context([&] {
        return fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT32, 3, const_cast<void*>(ptr), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    });
    if (r != CUDA_SUCCESS) {
        t_encode_status = (int)r;
        return false;
    }
    t_tmaps.put(k, *map);
    return true;
}

// B's scale atoms for the pair kernel, each read four times: a repeat dimension of stride 0 after
// the atom's 128 words, so one box lands as atom 0 four times then atom 1 four times. That is
// the source layout of one tcgen05.cp.128x256b, which fills all four lane quarters of the
// accumulator's tensor memory with the same 256 columns' scales.
bool make_sf_tmap_x4(CUtensorMap* map, const void* ptr, int rows, int Kp) {
    const TmapKey k{2, {rows, Kp, 0, 0}, ptr};
    if (const CUtensorMap* hit = t_tmaps.find(k)) {
        *map = *hit;
        return true;
    }
    EncodeTiledFn fn = encode_fn();
    if (!fn) {
        t_encode_status = -1;
        return false;
    }
    const int k_slabs = Kp / 128, atoms = (rows + 127) / 128;
    cuuint64_t dims[4] = {128u, 4u, (cuuint64_t)k_slabs, (cuuint64_t)atoms};
    cuuint64_t strides[3] = {0u, 512u, (cuuint64_t)k_slabs * 512u};
    cuuint32_t box[4] = {128u, 4u, 1u, 2u};
    cuuint32_t estr[4] = {1u, 1u, 1u, 1u};
    const CUresult r = driver_call_in_context([&] {
        return fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, const_cast<void*>(ptr), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    });
    if (r != CUDA_SUCCESS) {
        t_encode_status = (int)r;
        return false;
    }
    t_tmaps.put(k, *map);
    return true;
}

// ---- validation -----------------------------------------------------------------------------------

bool aligned(const void* p, uintptr_t a) {
    return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0;
}

// A operands the tensor-memory accelerator can read: stride a multiple of 32 bytes, at least the
// packed Kp codes, 32-byte aligned base. Other A operands go through the software producer
// (compact_a.cuh) when their stride is a multiple of 4 bytes and holds the row's real K codes:
// 0.75*Kp - 96 < A_row_bytes, i.e. kpad(4*A_row_bytes/3) == Kp — the reference's compact-A
// recipe (row stride 3K/4) is exactly this case.
bool a_uses_tma(int Kp, const void* dA, int A_row_bytes) {
    return A_row_bytes % 32 == 0 && (long long)A_row_bytes >= (long long)Kp * 3 / 4 && aligned(dA, 32);
}

// One destination: the plain GEMM's row-major [M][N] D.
kern::DstList single_dst(void* dD, int N) {
    kern::DstList dl{};
    dl.p[0] = dD;
    dl.n = 1;
    dl.col0 = 0;
    dl.ldd = N;
    return dl;
}

// 256-bit stores need every destination row chunk 32-byte aligned.
bool dst_align32(const kern::DstList& dl, size_t esize) {
    if ((dl.ldd * (long long)esize) % 32 || ((long long)dl.col0 * (long long)esize) % 32) return false;
    for (int d = 0; d < dl.n; d++)
        if (!aligned(dl.p[d], 32)) return false;
    return true;
}

// Producer for A: the 16U6 tensor load, or the loader warps' 4-byte cp.async copies.
int a_mode(int Kp, const void* dA, int A_row_bytes) {
    return a_uses_tma(Kp, dA, A_row_bytes) ? kern::A_TMA : kern::A_CPASYNC;
}

bool validate(int ot, int M, int N, int Kp, const void* dA, const void* dB, const void* sA,
              const void* sB, const void* dD, int A_row_bytes, int B_row_bytes) {
    if (ot < MXFP6_OUT_F32 || ot > MXFP6_OUT_BF16) {
        set_error(MXFP6_ERR_INVALID_OUT_TYPE, "invalid output type %d", ot);
        return false;
    }
    if (M <= 0 || N <= 0 || Kp <= 0 || M % 128 || N % 128 || Kp % K_TILE) {
        set_error(MXFP6_ERR_INVALID_SHAPE,
                  "unsupported shape %dx%dx%d: M and N must be positive multiples of 128 and Kp a "
                  "positive multiple of %d (pad with kpad())",
                  M, N, Kp, K_TILE);
        return false;
    }
    const long long need = (long long)Kp * 3 / 4;
    if (B_row_bytes < need || B_row_bytes % 32) {
        set_error(MXFP6_ERR_INVALID_STRIDE,
                  "B row stride %d bytes: must be >= %lld (= 0.75*Kp) and a multiple of 32 for the "
                  "tensor-memory accelerator's FP6 unpack mode (pad B to Kp)",
                  B_row_bytes, need);
        return false;
    }
    if (A_row_bytes % 4 || A_row_bytes <= need - 96) {
        set_error(MXFP6_ERR_INVALID_STRIDE,
                  "A row stride %d bytes: must be a multiple of 4 and hold the row's K codes "
                  "(> %lld = 0.75*Kp - 96; the compact stride 3K/4 of any K with kpad(K) == Kp)",
                  A_row_bytes, need - 96);
        return false;
    }
    if (!dA || !dB || !sA || !sB || !dD) {
        set_error(MXFP6_ERR_NULL_POINTER, "null device pointer (A=%p B=%p sA=%p sB=%p D=%p)", dA, dB,
                  sA, sB, dD);
        return false;
    }
    if (!aligned(dA, 4) || !aligned(dB, 32) || !aligned(sA, 16) || !aligned(sB, 16) || !aligned(dD, 16)) {
        set_error(MXFP6_ERR_MISALIGNED,
                  "misaligned pointer: A needs 4-byte (32-byte for the tensor-load path), B 32-byte, "
                  "scales and D 16-byte alignment");
        return false;
    }
    return true;
}

// ---- launch ----------------------------------------------------------------------------------------

// Compact-A fields of the kernel parameters (unused on the tensor-load path).
void set_compact(kern::Params& p, int Kp, const void* dA, int A_row_bytes) {
    p.a_ptr = static_cast<const uint8_t*>(dA);
    p.a_stride = A_row_bytes;
    const int need = Kp / 4 * 3;
    p.a_valid = A_row_bytes < need ? A_row_bytes : need;
}

// A tensor map for the 16U6 tensor load (unused, zeroed, by the loader-warp producers).
bool make_a_tmap(int amode, CUtensorMap* map, const void* dA, int M, int Kp, int A_row_bytes, int box_rows) {
    std::memset(map, 0, sizeof(*map));
    if (amode == kern::A_TMA) return make_fp6_tmap(map, dA, M, Kp, A_row_bytes, box_rows);
    return true;
}

// Programmatic stream serialization: the kernel may start its set-up while the previous kernel in
// the stream finishes; it waits (griddepcontrol.wait) before touching global memory, so stream
// order is kept for its inputs and outputs.
void set_pdl(cudaLaunchAttribute& a) {
    a.id = cudaLaunchAttributeProgrammaticStreamSerialization;
    a.val.programmaticStreamSerializationAllowed = 1;
}

template <int BN, typename OutT, bool PARTIAL, int AMODE>
bool launch_gemm(int M, int N, int Kp, const void* dA, const void* dB, const uint8_t* sA,
                 const uint8_t* sB, const kern::DstList& dl, float* ws, int A_row_bytes, int B_row_bytes,
                 int splits, cudaStream_t stream) {
    using C = kern::Config<BN, AMODE>;
    auto kernel = kern::gemm_mxfp6_sm100<BN, OutT, PARTIAL, AMODE>;
    static std::once_flag attr_once[kMaxDevices];
    const int dev = current_device();
    if (dev < 0 || dev >= kMaxDevices) {
        set_error(MXFP6_ERR_CUDA, "no CUDA device");
        return false;
    }
    cudaError_t attr_err = cudaSuccess;
    std::call_once(attr_once[dev], [&] {
        attr_err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES);
    });
    if (attr_err != cudaSuccess) {
        set_error(MXFP6_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(attr_err));
        return false;
    }
    CUtensorMap tmA, tmB;
    if (!make_a_tmap(AMODE, &tmA, dA, M, Kp, A_row_bytes, kern::BM) ||
        !make_fp6_tmap(&tmB, dB, N, Kp, B_row_bytes, BN)) {
        set_error(MXFP6_ERR_CUDA, "cuTensorMapEncodeTiled failed for %dx%dx%d (status %d)", M, N, Kp,
                  t_encode_status);
        return false;
    }
    kern::Params p;
    p.sfA = sA;
    p.sfB = sB;
    p.dst = dl;
    p.ws = ws;
    p.M = M;
    p.N = N;
    p.Kp = Kp;
    p.m_blocks = M / kern::BM;
    p.n_blocks = (N + BN - 1) / BN;
    p.k_slabs = Kp / kern::BK;
    p.splits = splits;
    p.out_align32 = (PARTIAL ? aligned(ws, 32) : dst_align32(dl, sizeof(OutT))) ? 1 : 0;
    set_compact(p, Kp, dA, A_row_bytes);
    p.wait_budget = wait_budget();
    const long long tiles = (long long)p.m_blocks * p.n_blocks * splits;
    p.sk_first = (int)tiles;
    p.sk_total = 0;
    p.sk_ws = nullptr;
    p.sk_flags = nullptr;
    p.sk_epoch = 0;
    p.band_L = p.band_a = p.band_n = 0;
    const int grid = (int)(tiles < sm_count() ? tiles : sm_count());
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid, 1, 1);
    cfg.blockDim = dim3(kern::threads_for(AMODE), 1, 1);
    cfg.dynamicSmemBytes = C::SMEM_BYTES;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    set_pdl(attr[0]);
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, tmA, tmB, p);
    if (e == cudaSuccess) e = cudaGetLastError();
    if (e != cudaSuccess) {
        set_error(MXFP6_ERR_CUDA, "GEMM launch failed: %s", cudaGetErrorString(e));
        return false;
    }
    g_launches.fetch_add(1, std::memory_order_relaxed);
    return true;
}

template <typename OutT, bool PARTIAL, int AMODE>
bool launch_pair(int M, int N, int Kp, const void* dA, const void* dB, const uint8_t* sA, const uint8_t* sB,
                 const kern::DstList& dl, float* ws, int A_row_bytes, int B_row_bytes, int splits, void* sk_area,
                 cudaStream_t stream, const BandedSplit* band = nullptr) {
    using C = kern::PairConfig<AMODE>;
    // the kernel without stream-K hand-offs and multi-destination stores, with hand-offs, and with
    // both (one instantiation in partial mode, which has neither)
    auto kernel_lean = kern::gemm_mxfp6_sm100_pair<OutT, PARTIAL, AMODE, kern::EPI_LEAN>;
    auto kernel_sk = kern::gemm_mxfp6_sm100_pair<OutT, PARTIAL, AMODE, PARTIAL ? kern::EPI_LEAN : kern::EPI_STREAM_K>;
    auto kernel_all = kern::gemm_mxfp6_sm100_pair<OutT, PARTIAL, AMODE, PARTIAL ? kern::EPI_LEAN : kern::EPI_ALL>;
    static std::once_flag attr_once[kMaxDevices];
    const int dev = current_device();
    if (dev < 0 || dev >= kMaxDevices) {
        set_error(MXFP6_ERR_CUDA, "no CUDA device");
        return false;
    }
    cudaError_t attr_err = cudaSuccess;
    std::call_once(attr_once[dev], [&] {
        for (auto k : {kernel_lean, kernel_sk, kernel_all})
            if (attr_err == cudaSuccess)
                attr_err = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES);
    });
    if (attr_err != cudaSuccess) {
        set_error(MXFP6_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(attr_err));
        return false;
    }
    const int m_blocks = (M + C::BM - 1) / C::BM, n_blocks = (N + C::BN - 1) / C::BN;
    const long long tiles = (long long)m_blocks * n_blocks * splits;
    const int pairs = sm_count() / 2;
    // a banded split (partial mode) keeps every pair busy
    const bool banded = PARTIAL && band && band->L > 0;
    const int clusters = banded ? pairs : (int)(tiles < pairs ? tiles : pairs);
    CUtensorMap tmA, tmB, tmSA, tmSB;
    if (!make_a_tmap(AMODE, &tmA, dA, M, Kp, A_row_bytes, 128) || !make_fp6_tmap(&tmB, dB, N, Kp, B_row_bytes, 128) ||
        !make_sf_tmap(&tmSA, sA, M, Kp, 1, C::SUB) || !make_sf_tmap_x4(&tmSB, sB, N, Kp)) {
        set_error(MXFP6_ERR_CUDA, "cuTensorMapEncodeTiled failed for %dx%dx%d (status %d)", M, N, Kp,
                  t_encode_status);
        return false;
    }
    kern::Params p;
    p.sfA = sA;
    p.sfB = sB;
    p.dst = dl;
    p.ws = ws;
    p.M = M;
    p.N = N;
    p.Kp = Kp;
    p.m_blocks = m_blocks;
    p.n_blocks = n_blocks;
    p.k_slabs = Kp / kern::BK;
    p.splits = splits;
    p.out_align32 = (PARTIAL ? aligned(ws, 32) : dst_align32(dl, sizeof(OutT))) ? 1 : 0;
    set_compact(p, Kp, dA, A_row_bytes);
    p.wait_budget = wait_budget();
    // Stream-K tail (sk_area non-null, laid out as stream_k_bytes(clusters)): the last waves'
    // tiles, one whole wave plus the partial one, are shared out by K slabs.
    p.sk_first = (int)tiles;
    p.sk_total = 0;
    p.sk_ws = nullptr;
    p.sk_flags = nullptr;
    p.sk_epoch = 0;
    if (sk_area && !PARTIAL && pair_stream_k(tiles, splits, clusters)) {
        p.sk_first = (int)((tiles / clusters - 1) * clusters);
        p.sk_total = (tiles - p.sk_first) * (long long)p.k_slabs;
        p.sk_ws = static_cast<float*>(sk_area);
        p.sk_flags = reinterpret_cast<unsigned long long*>(static_cast<uint8_t*>(sk_area) +
                                                           (size_t)clusters * C::SK_TILE_FLOATS * sizeof(float));
        p.sk_epoch = next_sk_epoch();
    }
    p.band_L = banded ? band->L : 0;
    p.band_a = banded ? band->a : 0;
    p.band_n = banded ? band->n : 0;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * clusters, 1, 1);
    cfg.blockDim = dim3(kern::threads_for(AMODE), 1, 1);
    cfg.dynamicSmemBytes = C::SMEM_BYTES;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    set_pdl(attr[1]);
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    const auto kernel = PARTIAL ? kernel_lean : dl.n > 1 ? kernel_all : p.sk_total > 0 ? kernel_sk : kernel_lean;
    cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, tmA, tmB, tmSA, tmSB, p);
    if (e == cudaSuccess) e = cudaGetLastError();
    if (e != cudaSuccess) {
        set_error(MXFP6_ERR_CUDA, "pair GEMM launch failed: %s", cudaGetErrorString(e));
        return false;
    }
    g_launches.fetch_add(1, std::memory_order_relaxed);
    return true;
}

template <typename OutT>
bool launch_reduce(const float* ws, const kern::DstList& dl, int M, int N, int splits, cudaStream_t stream) {
    const long long total = (long long)M * N;
    const long long n4 = total / 4;
    long long blocks = (n4 + 255) / 256;
    const long long cap = (long long)sm_count() * 8;
    if (blocks > cap) blocks = cap;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)blocks, 1, 1);
    cfg.blockDim = dim3(256, 1, 1);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    set_pdl(attr[0]);
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, kern::reduce_partials<OutT>, ws, dl, N, total, splits);
    if (e == cudaSuccess) e = cudaGetLastError();
    if (e != cudaSuccess) {
        set_error(MXFP6_ERR_CUDA, "split-K reduce launch failed: %s", cudaGetErrorString(e));
        return false;
    }
    g_launches.fetch_add(1, std::memory_order_relaxed);
    return true;
}

// Partial (split-K) launches write FP32 whatever the output type, so they share the float
// instantiation; the reduce pass converts.
template <typename OutT, int AMODE>
bool run_route(const Route& r, int M, int N, int Kp, const void* dA, const void* dB, const uint8_t* sA,
               const uint8_t* sB, const kern::DstList& dl, int Ar, int Br, void* ws, cudaStream_t stream) {
    float* wsf = static_cast<float*>(ws);
    const bool part = r.splits > 1;
    bool ok;
    if (r.MT == 256) {
        // the stream-K hand-off area follows the split-K partials in the workspace
        void* sk = r.stream_k ? static_cast<uint8_t*>(ws) + (part ? splitk_bytes(M, N, r.splits) : 0) : nullptr;
        BandedSplit band;
        if (r.banded) {
            const long long tiles = (long long)((M + 255) / 256) * ((N + 255) / 256);
            const int L = (int)((sm_count() / 2) / tiles);
            band = banded_split(tiles, sm_count() / 2, Kp / K_TILE, r.splits - L);
        }
        ok = part ? launch_pair<float, true, AMODE>(M, N, Kp, dA, dB, sA, sB, dl, wsf, Ar, Br, r.splits, nullptr,
                                                    stream, r.banded ? &band : nullptr)
                  : launch_pair<OutT, false, AMODE>(M, N, Kp, dA, dB, sA, sB, dl, wsf, Ar, Br, 1, sk, stream);
    } else if (r.NT == 256) {
        ok = part ? launch_gemm<256, float, true, AMODE>(M, N, Kp, dA, dB, sA, sB, dl, wsf, Ar, Br, r.splits,
                                                           stream)
                  : launch_gemm<256, OutT, false, AMODE>(M, N, Kp, dA, dB, sA, sB, dl, wsf, Ar, Br, 1, stream);
    } else {
        ok = part ? launch_gemm<128, float, true, AMODE>(M, N, Kp, dA, dB, sA, sB, dl, wsf, Ar, Br, r.splits,
                                                           stream)
                  : launch_gemm<128, OutT, false, AMODE>(M, N, Kp, dA, dB, sA, sB, dl, wsf, Ar, Br, 1, stream);
    }
    return ok && (!part || launch_reduce<OutT>(wsf, dl, M, N, r.splits, stream));
}

template <typename OutT>
bool run_typed(const Route& r, int M, int N, int Kp, const void* dA, const void* dB, const uint8_t* sA,
               const uint8_t* sB, const kern::DstList& dl, int Ar, int Br, void* ws, cudaStream_t stream) {
    return a_mode(Kp, dA, Ar) == kern::A_TMA
               ? run_route<OutT, kern::A_TMA>(r, M, N, Kp, dA, dB, sA, sB, dl, Ar, Br, ws, stream)
               : run_route<OutT, kern::A_CPASYNC>(r, M, N, Kp, dA, dB, sA, sB, dl, Ar, Br, ws, stream);
}

bool run(int ot, const Route& r, int M, int N, int Kp, const void* dA, const void* dB, const uint8_t* sA,
         const uint8_t* sB, const kern::DstList& dl, int Ar, int Br, void* ws, cudaStream_t stream) {
    switch (ot) {
        case MXFP6_OUT_F32:
            return run_typed<float>(r, M, N, Kp, dA, dB, sA, sB, dl, Ar, Br, ws, stream);
        case MXFP6_OUT_F16:
            return run_typed<__half>(r, M, N, Kp, dA, dB, sA, sB, dl, Ar, Br, ws, stream);
        default:
            return run_typed<__nv_bfloat16>(r, M, N, Kp, dA, dB, sA, sB, dl, Ar, Br, ws, stream);
    }
}

// Route for an output type: FP32 output keeps split segments short enough for its tolerance.
Route route_for_out(int ot, int M, int N, int Kp) {
    return route_for(M, N, Kp, sm_count(), ot == MXFP6_OUT_F32 ? fp32_min_splits(Kp) : 1);
}

// Bytes of a padded copy of A (rows of 0.75*Kp) placed after the split-K partials in the
// workspace; the offset keeps the copy 256-byte aligned for the tensor load.
size_t padded_a_bytes(int M, int Kp) {
    return (size_t)M * (size_t)(Kp / 4 * 3);
}
size_t padded_a_offset(size_t split_bytes) {
    return (split_bytes + 255) / 256 * 256;
}

// ---- re-pad scratch for compact A (library-owned, stream-ordered) -------------------------------
//
// gemm() re-pads an A whose row stride the tensor load cannot address (the compact stride 3K/4
// with K % 128 != 0) before the tensor-load kernel runs. The padded copy goes into the caller's
// workspace when that was sized for it (gemm_workspace_size with A_row_bytes). Otherwise it goes
// to scratch from a memory pool this library creates per device, taken and given back in stream
// order around the two launches (cudaMallocFromPoolAsync before, cudaFreeAsync after), so a caller
// that sized its workspace with the reference's three-argument query runs at the same speed. The
// pool keeps the memory it has mapped for later calls (release threshold unlimited) until
// mxfp6_release_repad_scratch() trims it. The scratch is not used while the stream captures a
// graph (the call then allocates nothing), when it is switched off (mxfp6_set_repad_scratch(0),
// or MXFP6_REPAD_SCRATCH=0 in the environment at load time), or when the allocation fails: the
// kernels' loader warps then read A in place, with identical results.
std::atomic<int> g_repad_scratch{[] {
    const char* e = std::getenv("MXFP6_REPAD_SCRATCH");
    return e && std::strcmp(e, "0") == 0 ? 0 : 1;
}()};
cudaMemPool_t g_repad_pool[kMaxDevices];
std::mutex g_repad_pool_mutex[kMaxDevices];

cudaMemPool_t repad_pool(int dev, bool create) {
    std::lock_guard<std::mutex> lock(g_repad_pool_mutex[dev]);
    if (!g_repad_pool[dev] && create) {
        cudaMemPoolProps props{};
        props.allocType = cudaMemAllocationTypePinned;
        props.handleTypes = cudaMemHandleTypeNone;
        props.location.type = cudaMemLocationTypeDevice;
        props.location.id = dev;
        cudaMemPool_t pool = nullptr;
        if (cudaMemPoolCreate(&pool, &props) == cudaSuccess) {
            uint64_t keep = UINT64_MAX;
            if (cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &keep) != cudaSuccess)
                cudaGetLastError();
            g_repad_pool[dev] = pool;
        } else {
            cudaGetLastError();
        }
    }
    return g_repad_pool[dev];
}

// Smallest M*N*Kp for which the scratch is taken. Taking and giving back the scratch plus the
// extra launch cost about 5 us of host and launch time per call. Measured on B200 (FP16, compact A,
// per call in place -> with scratch): 256x256x480 8.0 -> 13.3 us back to back; 1024x1024x2016
// 18.4 -> 18.7 us L2-flushed (even); 2048x2048x4064 30.7 -> 28.9 us; 4096x4096x4064 125 -> 74 us;
// 8192x8192x8160 825 -> 468 us.
constexpr double kRepadScratchMinWork = 2147483648.0;

// `bytes` of 256-byte aligned scratch ordered on `stream`, or nullptr (switched off, capturing,
// no pool, out of memory). A failed attempt leaves no sticky runtime error behind.
void* repad_scratch_alloc(size_t bytes, cudaStream_t stream) {
    if (g_repad_scratch.load(std::memory_order_relaxed) == 0) return nullptr;
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(stream, &cs) != cudaSuccess) {
        cudaGetLastError();
        return nullptr;
    }
    if (cs != cudaStreamCaptureStatusNone) return nullptr;
    const int dev = current_device();
    if (dev < 0 || dev >= kMaxDevices) {
        cudaGetLastError();
        return nullptr;
    }
    cudaMemPool_t pool = repad_pool(dev, true);
    if (!pool) return nullptr;
    void* p = nullptr;
    if (cudaMallocFromPoolAsync(&p, bytes, pool, stream) != cudaSuccess || !p) {
        cudaGetLastError();
        return nullptr;
    }
    if (!aligned(p, 256)) {
        cudaFreeAsync(p, stream);
        return nullptr;
    }
    return p;
}

void gemm_entry(int ot, int M, int N, int Kp, const void* dA, const void* dB, const uint8_t* sA,
                const uint8_t* sB, const kern::DstList& dl, int Ar, int Br, void* ws, size_t ws_bytes,
                cudaStream_t stream) {
    t_last_error = MXFP6_OK;
    if (!validate(ot, M, N, Kp, dA, dB, sA, sB, dl.p[0], Ar, Br)) return;
    Route r = route_for_out(ot, M, N, Kp);
    const int sms = sm_count();
    if (r.splits > 1 || r.stream_k) {
        const size_t need = route_ws_bytes(r, M, N, sms);
        // the stream-K hand-off area takes 256-bit stores: a 256-byte aligned workspace
        if (!ws || ws_bytes < need || !aligned(ws, r.stream_k ? 256 : 16)) {
            // Same contract as the reference (src/dispatch.hpp:76-87): correct, only slower.
            if (r.splits > 1)
                std::fprintf(stderr,
                             "[mxfp6] split-K skipped for %dx%dx%d: workspace %zu bytes, need %zu — "
                             "running unsplit (slower). Size it with gemm_workspace_size().\n",
                             M, N, Kp, ws_bytes, need);
            else
                std::fprintf(stderr,
                             "[mxfp6] stream-K tail skipped for %dx%dx%d: workspace %zu bytes (256-byte aligned), "
                             "need %zu — running whole tiles (slower). Size it with gemm_workspace_size().\n",
                             M, N, Kp, ws_bytes, need);
            r.splits = 1;
            r.stream_k = false;
            r.banded = false;
        }
    }
    // An A the tensor load cannot address (the compact stride 3K/4 with K % 128 != 0) is re-padded
    // first: one HBM pass, then the tensor-load kernel. The copy goes into the workspace, after
    // the split-K partials, when the caller sized the workspace for it (gemm_workspace_size with
    // A_row_bytes), else, for a GEMM of at least kRepadScratchMinWork, into the library's re-pad
    // scratch. Otherwise the kernels' loader warps read A in place (same results, slower on
    // large shapes).
    void* scratch = nullptr;
    if (a_mode(Kp, dA, Ar) == kern::A_CPASYNC) {
        const size_t off = padded_a_offset(route_ws_bytes(r, M, N, sms));
        const int prb = Kp / 4 * 3;
        uint8_t* pa = nullptr;
        if (ws && aligned(ws, 256) && ws_bytes >= off + padded_a_bytes(M, Kp))
            pa = static_cast<uint8_t*>(ws) + off;
        else if ((double)M * N * Kp >= kRepadScratchMinWork)
            pa = static_cast<uint8_t*>(scratch = repad_scratch_alloc(padded_a_bytes(M, Kp), stream));
        if (pa) {
            const cudaError_t e = launch_repad(static_cast<const uint8_t*>(dA), M, Ar, Ar < prb ? Ar : prb, pa, prb,
                                               stream);
            if (e != cudaSuccess) {
                if (scratch) cudaFreeAsync(scratch, stream);
                set_error(MXFP6_ERR_CUDA, "A re-pad launch failed: %s", cudaGetErrorString(e));
                return;
            }
            note_launch();
            dA = pa;
            Ar = prb;
        }
    }
    run(ot, r, M, N, Kp, dA, dB, sA, sB, dl, Ar, Br, ws, stream);
    if (scratch && cudaFreeAsync(scratch, stream) != cudaSuccess && t_last_error == MXFP6_OK)
        set_error(MXFP6_ERR_CUDA, "returning the A re-pad scratch failed: %s", cudaGetErrorString(cudaGetLastError()));
}

// ---- split-K scratch owned by the library (mxfp6_gemm_static_workspace) --------------------------------
//
// For callers that cannot allocate device memory themselves. The FP32 split-K partials go to
// this fixed-size array instead of a caller workspace. It is an ordinary module global: every
// device that loads this library reserves kStaticWorkspaceBytes for it until the process exits.
// Host code must not hand `g_static_split_ws` to a kernel directly (on the host the name is a
// stand-in, not a device address); its device address is looked up once per device with
// cudaGetSymbolAddress, with that device current, on the first call made there.
constexpr size_t kStaticWorkspaceBytes = size_t(32) << 20;
static __device__ __align__(256) unsigned char g_static_split_ws[kStaticWorkspaceBytes];
void* g_static_ws_addr[kMaxDevices];
std::mutex g_static_ws_mutex[kMaxDevices];

// Only a successful lookup is cached: a lookup that failed (inside a stream capture, say) is
// retried by the next call on that device. The runtime's sticky error from a failed lookup is
// cleared so that it does not surface in the caller's next error check; the failure itself is
// reported through *err.
void* static_workspace_address(int dev, cudaError_t* err) {
    std::lock_guard<std::mutex> lock(g_static_ws_mutex[dev]);
    *err = cudaSuccess;
    if (!g_static_ws_addr[dev]) {
        void* addr = nullptr;
        *err = cudaGetSymbolAddress(&addr, g_static_split_ws);
        if (*err == cudaSuccess && addr)
            g_static_ws_addr[dev] = addr;
        else
            cudaGetLastError();
    }
    return g_static_ws_addr[dev];
}

}  // namespace

void note_launch() {
    g_launches.fetch_add(1, std::memory_order_relaxed);
}

// ---- C++ API ------------------------------------------------------------------------------------------

TileChoice choose_tile(int M, int N, int Kp) {
    Route r = route_for(M, N, Kp, sm_count());
    return TileChoice{r.MT, r.NT, r.MT / 32, r.NT / 32};
}

// The query has no output type (same signature as the reference), so it returns the larger of
// the FP16/BF16 and FP32 needs: a workspace sized here fits every call on this shape.
size_t gemm_workspace_size(int M, int N, int Kp) {
    size_t need = 0;
    for (int ot : {MXFP6_OUT_F16, MXFP6_OUT_F32}) {
        const size_t b = route_ws_bytes(route_for_out(ot, M, N, Kp), M, N, sm_count());
        if (b > need) need = b;
    }
    return need;
}

size_t gemm_workspace_size(int M, int N, int Kp, int A_row_bytes) {
    const size_t split = gemm_workspace_size(M, N, Kp);
    const bool tma_stride = A_row_bytes % 32 == 0 && (long long)A_row_bytes >= (long long)Kp * 3 / 4;
    return tma_stride ? split : padded_a_offset(split) + padded_a_bytes(M, Kp);
}

void gemm(OutType ot, int M, int N, int Kp, const void* dA, const void* dBsh, const uint8_t* dsA,
          const uint8_t* dsB, void* dD, int A_row_bytes, int B_row_bytes, void* ws, size_t ws_bytes) {
    gemm_entry((int)ot, M, N, Kp, dA, dBsh, dsA, dsB, single_dst(dD, N), A_row_bytes, B_row_bytes, ws, ws_bytes,
               0);
}

}  // namespace mxfp6

// ---- C ABI --------------------------------------------------------------------------------------------

using namespace mxfp6;

extern "C" {

void mxfp6_gemm(int ot, int M, int N, int Kp, const void* dA, const void* dBsh, const uint8_t* dsA,
                const uint8_t* dsB, void* dD, int A_row_bytes, int B_row_bytes, void* ws,
                size_t ws_bytes) {
    gemm_entry(ot, M, N, Kp, dA, dBsh, dsA, dsB, single_dst(dD, N), A_row_bytes, B_row_bytes, ws, ws_bytes, 0);
}

void mxfp6_gemm_stream(int ot, int M, int N, int Kp, const void* dA, const void* dBsh,
                       const uint8_t* dsA, const uint8_t* dsB, void* dD, int A_row_bytes,
                       int B_row_bytes, void* ws, size_t ws_bytes, void* stream) {
    gemm_entry(ot, M, N, Kp, dA, dBsh, dsA, dsB, single_dst(dD, N), A_row_bytes, B_row_bytes, ws, ws_bytes,
               static_cast<cudaStream_t>(stream));
}

size_t mxfp6_gemm_workspace_size(int M, int N, int Kp) {
    return gemm_workspace_size(M, N, Kp);
}

size_t mxfp6_gemm_workspace_size_a(int M, int N, int Kp, int A_row_bytes) {
    return gemm_workspace_size(M, N, Kp, A_row_bytes);
}

size_t mxfp6_gemm_workspace_size_out(int ot, int M, int N, int Kp) {
    if (ot < MXFP6_OUT_F32 || ot > MXFP6_OUT_BF16) return 0;
    return route_ws_bytes(route_for_out(ot, M, N, Kp), M, N, sm_count());
}

void mxfp6_choose_tile(int M, int N, int Kp, int* out4) {
    TileChoice t = choose_tile(M, N, Kp);
    if (out4) {
        out4[0] = t.MT;
        out4[1] = t.NT;
        out4[2] = t.MPW;
        out4[3] = t.NPW;
    }
}

void mxfp6_route(int ot, int M, int N, int Kp, int* out3) {
    if (!out3) return;
    const Route r = route_for_out(ot, M, N, Kp);
    out3[0] = r.MT;
    out3[1] = r.NT;
    out3[2] = r.splits;
}

int mxfp6_route_stream_k(int ot, int M, int N, int Kp) {
    return route_for_out(ot, M, N, Kp).stream_k ? 1 : 0;
}

int mxfp6_route_banded(int ot, int M, int N, int Kp) {
    return route_for_out(ot, M, N, Kp).banded ? 1 : 0;
}

int mxfp6_set_repad_scratch(int enable) {
    return g_repad_scratch.exchange(enable ? 1 : 0);
}

size_t mxfp6_repad_scratch_bytes(void) {
    const int dev = current_device();
    if (dev < 0 || dev >= kMaxDevices) {
        cudaGetLastError();
        return 0;
    }
    cudaMemPool_t pool = repad_pool(dev, false);
    uint64_t held = 0;
    if (pool && cudaMemPoolGetAttribute(pool, cudaMemPoolAttrReservedMemCurrent, &held) != cudaSuccess) {
        cudaGetLastError();
        held = 0;
    }
    return (size_t)held;
}

int mxfp6_release_repad_scratch(void) {
    t_last_error = MXFP6_OK;
    const int dev = current_device();
    if (dev < 0 || dev >= kMaxDevices) {
        cudaGetLastError();
        return MXFP6_OK;
    }
    cudaMemPool_t pool = repad_pool(dev, false);
    if (!pool) return MXFP6_OK;
    const cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess || cudaMemPoolTrimTo(pool, 0) != cudaSuccess) {
        set_error(MXFP6_ERR_CUDA, "releasing the A re-pad scratch failed: %s",
                  cudaGetErrorString(e != cudaSuccess ? e : cudaGetLastError()));
        return t_last_error;
    }
    return MXFP6_OK;
}

size_t mxfp6_stream_k_workspace_bytes(void) {
    return stream_k_bytes(sm_count() / 2);
}

int mxfp6_k_tile(void) {
    return K_TILE;
}

int mxfp6_kpad(int K) {
    return kpad(K);
}

void mxfp6_gemm_force_route(int ot, int M, int N, int Kp, int MT, int NT, int splits, int stream_k, const void* dA,
                            const void* dBsh, const uint8_t* dsA, const uint8_t* dsB, void* dD, int A_row_bytes,
                            int B_row_bytes, void* ws, size_t ws_bytes, void* stream) {
    t_last_error = MXFP6_OK;
    if (stream_k == 1 && (MT != 256 || splits != 1)) {
        set_error(MXFP6_ERR_UNSUPPORTED, "stream-K tail: the 256x256 pair tile without a K split only");
        return;
    }
    if (stream_k < 0 || stream_k > 2) {
        set_error(MXFP6_ERR_UNSUPPORTED, "forced route mode %d (0 plain, 1 stream-K tail, 2 banded split)", stream_k);
        return;
    }
    BandedSplit band;
    if (stream_k == 2) {
        // banded split with `splits` short bands
        const long long tiles = (long long)((M + 255) / 256) * ((N + 255) / 256);
        band = banded_split(tiles, sm_count() / 2, Kp / K_TILE, splits);
        if (MT != 256 || NT != 256 || band.L == 0) {
            set_error(MXFP6_ERR_UNSUPPORTED, "banded split of %dx%dx%d with %d short bands: not available", M, N, Kp,
                      splits);
            return;
        }
        splits = band.splits();
    }
    if (!validate(ot, M, N, Kp, dA, dBsh, dsA, dsB, dD, A_row_bytes, B_row_bytes)) return;
    const bool tile_ok = (MT == 256 && NT == 256) || (MT == 128 && (NT == 128 || NT == 256));
    if (!tile_ok || splits < 1 || splits > Kp / K_TILE) {
        set_error(MXFP6_ERR_UNSUPPORTED, "forced route %dx%d splits=%d not available for Kp=%d", MT, NT,
                  splits, Kp);
        return;
    }
    if (splits > 1 && (!ws || ws_bytes < splitk_bytes(M, N, splits) || !aligned(ws, 16))) {
        set_error(MXFP6_ERR_WORKSPACE, "forced split %d needs %zu workspace bytes, got %zu", splits,
                  splitk_bytes(M, N, splits), ws_bytes);
        return;
    }
    const size_t sk_need = stream_k_bytes(sm_count() / 2);
    if (stream_k == 1 && (!ws || ws_bytes < sk_need || !aligned(ws, 256))) {
        set_error(MXFP6_ERR_WORKSPACE, "forced stream-K tail needs %zu workspace bytes (256-byte aligned), got %zu",
                  sk_need, ws_bytes);
        return;
    }
    Route r{MT, NT, splits};
    r.stream_k = stream_k == 1;
    r.banded = stream_k == 2;
    run(ot, r, M, N, Kp, dA, dBsh, dsA, dsB, single_dst(dD, N), A_row_bytes, B_row_bytes, ws,
        static_cast<cudaStream_t>(stream));
}

void mxfp6_gemm_force_tile(int ot, int M, int N, int Kp, int MT, int NT, int splits, const void* dA,
                           const void* dBsh, const uint8_t* dsA, const uint8_t* dsB, void* dD,
                           int A_row_bytes, int B_row_bytes, void* ws, size_t ws_bytes,
                           void* stream) {
    mxfp6_gemm_force_route(ot, M, N, Kp, MT, NT, splits, 0, dA, dBsh, dsA, dsB, dD, A_row_bytes, B_row_bytes, ws,
                           ws_bytes, stream);
}

void mxfp6_gemm_static_workspace(int ot, int M, int N, int Kp, const void* dA, const void* dBsh,
                                 const uint8_t* dsA, const uint8_t* dsB, void* dD, int A_row_bytes,
                                 int B_row_bytes, void* stream) {
    t_last_error = MXFP6_OK;
    if (!validate(ot, M, N, Kp, dA, dBsh, dsA, dsB, dD, A_row_bytes, B_row_bytes)) return;
    const Route r = route_for_out(ot, M, N, Kp);
    void* ws = nullptr;
    if (r.splits > 1 || r.stream_k) {
        const size_t need = route_ws_bytes(r, M, N, sm_count());
        if (need > kStaticWorkspaceBytes) {
            set_error(MXFP6_ERR_WORKSPACE,
                      "%dx%dx%d splits K %d ways and needs %zu bytes of split-K scratch; the library's "
                      "static workspace holds %zu bytes. Use mxfp6_gemm with a caller workspace.",
                      M, N, Kp, r.splits, need, kStaticWorkspaceBytes);
            return;
        }
        const int dev = current_device();
        if (dev < 0 || dev >= kMaxDevices) {
            set_error(MXFP6_ERR_CUDA, "no CUDA device");
            return;
        }
        cudaError_t lookup_err = cudaSuccess;
        ws = static_workspace_address(dev, &lookup_err);
        if (!ws) {
            set_error(MXFP6_ERR_CUDA, "cudaGetSymbolAddress for the static split-K workspace failed: %s",
                      cudaGetErrorString(lookup_err));
            return;
        }
    }
    run(ot, r, M, N, Kp, dA, dBsh, dsA, dsB, single_dst(dD, N), A_row_bytes, B_row_bytes, ws,
        static_cast<cudaStream_t>(stream));
}

void mxfp6_gemm_gather(int ot, int M, int N, int Kp, const void* dA, const void* dBsh, const uint8_t* dsA,
                       const uint8_t* dsB, void* const* dDs, int n_dst, long long ldd, int col0, int A_row_bytes,
                       int B_row_bytes, void* ws, size_t ws_bytes, void* stream) {
    t_last_error = MXFP6_OK;
    if (!dDs || n_dst < 1 || n_dst > kern::MAX_DST) {
        set_error(MXFP6_ERR_NULL_POINTER, "gather: %d destinations (1..%d, non-null list)", n_dst, kern::MAX_DST);
        return;
    }
    const long long esize = ot == MXFP6_OUT_F32 ? 4 : 2;
    if (col0 < 0 || ldd < (long long)col0 + N || (ldd * esize) % 16 || ((long long)col0 * esize) % 16) {
        set_error(MXFP6_ERR_INVALID_STRIDE,
                  "gather: destination pitch %lld and column offset %d must hold N=%d columns and keep "
                  "16-byte aligned rows",
                  ldd, col0, N);
        return;
    }
    kern::DstList dl{};
    for (int d = 0; d < n_dst; d++) {
        if (!dDs[d] || !aligned(dDs[d], 16)) {
            set_error(dDs[d] ? MXFP6_ERR_MISALIGNED : MXFP6_ERR_NULL_POINTER,
                      "gather: destination %d is null or not 16-byte aligned", d);
            return;
        }
        dl.p[d] = dDs[d];
    }
    dl.n = n_dst;
    dl.col0 = col0;
    dl.ldd = ldd;
    gemm_entry(ot, M, N, Kp, dA, dBsh, dsA, dsB, dl, A_row_bytes, B_row_bytes, ws, ws_bytes,
               static_cast<cudaStream_t>(stream));
}

int mxfp6_ipc_export(const void* dptr, void* handle_out, size_t* offset_out) {
    using GetRangeFn = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);
    static GetRangeFn range = [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &f, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            f = nullptr;
        return reinterpret_cast<GetRangeFn>(f);
    }();
    if (!dptr || !handle_out || !offset_out || !range) return MXFP6_ERR_NULL_POINTER;
    CUdeviceptr base = 0;
    size_t size = 0;
    if (driver_call_in_context([&] { return range(&base, &size, reinterpret_cast<CUdeviceptr>(dptr)); }) !=
        CUDA_SUCCESS)
        return MXFP6_ERR_CUDA;
    cudaIpcMemHandle_t h;
    if (cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base)) != cudaSuccess) return MXFP6_ERR_CUDA;
    std::memcpy(handle_out, &h, sizeof(h));
    *offset_out = (size_t)(reinterpret_cast<CUdeviceptr>(dptr) - base);
    return MXFP6_OK;
}

int mxfp6_ipc_import(const void* handle, size_t offset, void** base_out, void** dptr_out) {
    if (!handle || !base_out || !dptr_out) return MXFP6_ERR_NULL_POINTER;
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle, sizeof(h));
    void* base = nullptr;
    if (cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) return MXFP6_ERR_CUDA;
    *base_out = base;
    *dptr_out = static_cast<uint8_t*>(base) + offset;
    return MXFP6_OK;
}

int mxfp6_ipc_close(void* base) {
    return cudaIpcCloseMemHandle(base) == cudaSuccess ? MXFP6_OK : MXFP6_ERR_CUDA;
}

long long mxfp6_set_wait_budget(long long cycles) {
    const long long prev = t_wait_budget;
    t_wait_budget = cycles > 0 ? cycles : 0;
    return prev;
}

size_t mxfp6_static_workspace_bytes(void) {
    return kStaticWorkspaceBytes;
}

int mxfp6_last_error(void) {
    return t_last_error;
}

const char* mxfp6_last_error_string(void) {
    switch (t_last_error) {
        case MXFP6_OK: return "ok";
        case MXFP6_ERR_INVALID_SHAPE: return "invalid shape";
        case MXFP6_ERR_INVALID_STRIDE: return "invalid row stride";
        case MXFP6_ERR_MISALIGNED: return "misaligned pointer";
        case MXFP6_ERR_NULL_POINTER: return "null pointer";
        case MXFP6_ERR_INVALID_OUT_TYPE: return "invalid output type";
        case MXFP6_ERR_CUDA: return "CUDA error";
        case MXFP6_ERR_DEVICE_TIMEOUT: return "device wait timed out";
        case MXFP6_ERR_WORKSPACE: return "workspace too small";
        case MXFP6_ERR_UNSUPPORTED: return "unsupported route";
        default: return "unknown error";
    }
}

int mxfp6_device_status(void) {
    if (cudaDeviceSynchronize() != cudaSuccess) return -1;
    unsigned int v = 0, zero = 0;
    if (cudaMemcpyFromSymbol(&v, g_device_status, sizeof(v)) != cudaSuccess) return -1;
    if (cudaMemcpyToSymbol(g_device_status, &zero, sizeof(zero)) != cudaSuccess) return -1;
    if (v) t_last_error = MXFP6_ERR_DEVICE_TIMEOUT;
    return (int)v;
}

uint64_t mxfp6_launch_count(void) {
    return g_launches.load(std::memory_order_relaxed);
}

}  // extern "C"
